// Rotary position embedding (RoPE) forward/backward for sm_100a.
//
// Math follows src/picotron/nn/rope.py:35-51 (interleaved pairs) of the reference:
//   out[2i]   = x[2i] * cos[s, i] - x[2i+1] * sin[s, i]
//   out[2i+1] = x[2i] * sin[s, i] + x[2i+1] * cos[s, i]
// The backward is the rotation by -angle (sin -> -sin), which is what autograd computes
// for that forward. ROTATE_HALF pairs x[i] with x[i + D/2] instead.
//
// Layout: a logical [B, H, S, D] tensor with arbitrary strides in elements (stride of D
// = 1), e.g. the reference's transposed view of [B, S, H, D] projections
// (src/picotron/nn/attention.py:196-203), read in place with no .contiguous() copy.
// Three paths, chosen per call on the host:
//  * rows (rope_rows, interleaved pairs): every (b, s) row of heads x head_dim is
//    contiguous, as in that view; q and k rows of one position are rotated together with
//    one load of the table entries per thread and row;
//  * vector (rope_vec): any strides with 16-byte aligned rows; the host orders the outer
//    dimensions by decreasing input stride so consecutive threads walk memory in address
//    order, and each thread rotates U 16-byte vectors per iteration (loads first);
//  * scalar (rope_scalar): any even head_dim, any alignment.
// All three use the same explicitly rounded fp32 rotation, so they agree bit for bit.
#include <algorithm>

#include "common.cuh"

namespace pt {
namespace {

constexpr int kThreads = 256;  // scalar path
constexpr int kUnroll = 4;     // 16-byte vectors in flight per thread (vector path)
// Vector-path block size (measured back to back on B200 at config 4: interleaved 0.88 of
// the HBM peak with 64-thread CTAs against 0.85 with 256; rotate-half 0.92 with 128 against
// 0.89 with 256): many small CTAs keep more of each SM's 2048 threads busy to the end.
template <bool kRotateHalf> constexpr int vec_threads() { return kRotateHalf ? 128 : 64; }

struct RopeGeom {
  uint32_t n0, n1, n2;          // outer sizes, outermost first (memory order of x)
  FastDiv div_vpr, div_n2, div_n1;  // divisions of the flat vector index
  int64_t xs0, xs1, xs2;         // x strides of those dims (elements)
  int64_t os0, os1, os2;         // out strides
  int s_axis;                    // which of the three is the sequence axis
  bool same;                     // out strides == x strides
  bool small;                    // every element offset of x and out is below 2^31
  uint32_t vpr;                  // vectors handled per row (per (b, h, s))
  int64_t table_stride;          // elements between table rows
  float sign;                    // +1 forward, -1 backward
};

// One rotation in fp32 with explicit roundings (no contraction into fused multiply-adds), so
// that the rows, vector and scalar paths give bit-identical results:
//   r1 = e * c - o * s,  r2 = e * s + o * c.
__device__ __forceinline__ void rotate(float e, float o, float c, float s, float& r1, float& r2) {
  r1 = __fsub_rn(__fmul_rn(e, c), __fmul_rn(o, s));
  r2 = __fadd_rn(__fmul_rn(e, s), __fmul_rn(o, c));
}

// Loads N consecutive table entries of TT starting at p as fp32. The host guarantees
// that p is aligned to min(16, N * sizeof(TT)) bytes on the vector path.
template <typename TT, int N>
__device__ __forceinline__ void load_table(const TT* p, float* f) {
  constexpr int kBytes = N * (int)sizeof(TT);
  if constexpr (kBytes >= 16) {
    constexpr int V = Vec16<TT>::N;
#pragma unroll
    for (int i = 0; i < N / V; ++i) unpack<TT>(ld_cached(p + i * V), f + i * V);
  } else if constexpr (kBytes == 8) {
    uint2 r = ld_cached8(p);
    if constexpr (sizeof(TT) == 4) {
      f[0] = __uint_as_float(r.x);
      f[1] = __uint_as_float(r.y);
    } else {
      uint4 q = make_uint4(r.x, r.y, 0, 0);
      float t[8];
      unpack<TT>(q, t);
#pragma unroll
      for (int i = 0; i < 4; ++i) f[i] = t[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) f[i] = to_float(p[i]);
  }
}

// Up to two tensors rotated by one launch (query and key share positions and tables): CTAs
// [0, blocks0) walk tensor 0, the rest tensor 1, each in proportion to its size.
template <typename T> struct RopeJobs {
  RopeGeom g[2];
  const T* x[2];
  T* out[2];
  uint32_t total[2];  // vectors
  uint32_t blocks0;
};

template <typename T, typename TT, bool kRotateHalf>
__device__ __forceinline__ void rope_vec_body(const T* __restrict__ x, T* __restrict__ out,
                                              const TT* __restrict__ cosine,
                                              const TT* __restrict__ sine, const RopeGeom& g,
                                              int half_dim, uint32_t total, uint32_t block,
                                              uint32_t nblocks) {
  constexpr int V = Vec16<T>::N;
  const uint32_t step = nblocks * blockDim.x * kUnroll;
  for (uint32_t i0 = block * blockDim.x * kUnroll + threadIdx.x; i0 < total; i0 += step) {
    uint4 a[kUnroll], b[kUnroll];
    int64_t xo[kUnroll], oo[kUnroll];
    uint32_t srow[kUnroll], vj[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const uint32_t idx = i0 + k * blockDim.x;
      if (idx >= total) continue;
      const uint32_t row = g.div_vpr.div(idx);
      vj[k] = idx - row * g.vpr;
      const uint32_t r2 = g.div_n2.div(row);
      const uint32_t i2 = row - r2 * g.n2;
      const uint32_t i0_ = g.div_n1.div(r2);
      const uint32_t i1 = r2 - i0_ * g.n1;
      srow[k] = g.s_axis == 0 ? i0_ : (g.s_axis == 1 ? i1 : i2);
      if (g.small) {  // every offset fits in 32 bits: cheaper index arithmetic
        xo[k] = (int64_t)(i0_ * (uint32_t)g.xs0 + i1 * (uint32_t)g.xs1 + i2 * (uint32_t)g.xs2);
        oo[k] = g.same ? xo[k]
                       : (int64_t)(i0_ * (uint32_t)g.os0 + i1 * (uint32_t)g.os1 +
                                   i2 * (uint32_t)g.os2);
      } else {
        xo[k] = (int64_t)i0_ * g.xs0 + (int64_t)i1 * g.xs1 + (int64_t)i2 * g.xs2;
        oo[k] = g.same ? xo[k] : (int64_t)i0_ * g.os0 + (int64_t)i1 * g.os1 + (int64_t)i2 * g.os2;
      }
      const int64_t d0 = (int64_t)vj[k] * V;
      a[k] = ld_stream(x + xo[k] + d0);
      if (kRotateHalf) b[k] = ld_stream(x + xo[k] + d0 + half_dim);
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const uint32_t idx = i0 + k * blockDim.x;
      if (idx >= total) continue;
      const int64_t d0 = (int64_t)vj[k] * V;
      if (!kRotateHalf) {
        // V elements = V/2 interleaved pairs starting at pair index d0/2.
        float c[V / 2], s[V / 2], f[V];
        const int64_t t = (int64_t)srow[k] * g.table_stride + d0 / 2;
        load_table<TT, V / 2>(cosine + t, c);
        load_table<TT, V / 2>(sine + t, s);
        unpack<T>(a[k], f);
#pragma unroll
        for (int p = 0; p < V / 2; ++p)
          rotate(f[2 * p], f[2 * p + 1], c[p], g.sign * s[p], f[2 * p], f[2 * p + 1]);
        st_stream(out + oo[k] + d0, pack<T>(f));
      } else {
        // First-half vector at d0 pairs with the second-half vector at d0 + D/2.
        float c[V], s[V], f1[V], f2[V];
        const int64_t t = (int64_t)srow[k] * g.table_stride + d0;
        load_table<TT, V>(cosine + t, c);
        load_table<TT, V>(sine + t, s);
        unpack<T>(a[k], f1);
        unpack<T>(b[k], f2);
#pragma unroll
        for (int p = 0; p < V; ++p) rotate(f1[p], f2[p], c[p], g.sign * s[p], f1[p], f2[p]);
        st_stream(out + oo[k] + d0, pack<T>(f1));
        st_stream(out + oo[k] + d0 + half_dim, pack<T>(f2));
      }
    }
  }
}

template <typename T, typename TT, bool kRotateHalf>
__global__ void __launch_bounds__(vec_threads<kRotateHalf>())
rope_vec(const __grid_constant__ RopeJobs<T> jobs, const TT* __restrict__ cosine,
         const TT* __restrict__ sine, int half_dim) {
  // Two copies of the loop, each reading its tensor's geometry at fixed parameter offsets.
  if (blockIdx.x < jobs.blocks0)
    rope_vec_body<T, TT, kRotateHalf>(jobs.x[0], jobs.out[0], cosine, sine, jobs.g[0],
                                      half_dim, jobs.total[0], blockIdx.x, jobs.blocks0);
  else
    rope_vec_body<T, TT, kRotateHalf>(jobs.x[1], jobs.out[1], cosine, sine, jobs.g[1],
                                      half_dim, jobs.total[1], blockIdx.x - jobs.blocks0,
                                      gridDim.x - jobs.blocks0);
}

// Rows path (interleaved pairs), for the layout the attention projections produce: each
// (b, s) row of a tensor is contiguous (head stride = head_dim, head_dim stride 1), as in the
// [B,H,S,D] view of [B,S,H,D] memory. A CTA takes whole rows of q and k together (the same
// position, so one row of the angle tables); a unit is one 16-byte vector. Units per head
// divide the block size, so every unit a thread touches sits at the same place in its head
// and needs the same table entries: the thread loads them once per row, and no index
// division is left but b = r / S. (For rotate-half pairs this layout ran slower than the
// vector path in A/B runs, so those keep it.)
// 4 units per thread in flight: A/B on B200 at config 4 (q + k, bf16) gave 0.917 of the HBM
// peak, against 0.851 / 0.895 / 0.913 with 2 / 5 / 8 and 0.879 on the vector path.
#ifndef PT_ROPE_ROW_UNITS
#define PT_ROPE_ROW_UNITS 4
#endif
constexpr int kRowThreads = 128;
constexpr int kRowUnits = PT_ROPE_ROW_UNITS;  // units of a row per thread in flight

template <typename T> struct RopeRows {
  const T* x[2];
  T* out[2];
  int64_t xb[2], xs[2], ob[2], os[2];  // batch and sequence strides (elements)
  uint32_t units0, units;              // units per row: of tensor 0, of both tensors
  uint32_t rows, S;                    // rows = B * S
  FastDiv div_s;
  int64_t table_stride;
  int uh_log2;  // log2 of the units per head
  float sign;   // +1 forward, -1 backward
};

template <typename T, typename TT>
__global__ void __launch_bounds__(kRowThreads)
rope_rows(const __grid_constant__ RopeRows<T> p, const TT* __restrict__ cosine,
          const TT* __restrict__ sine) {
  constexpr int V = Vec16<T>::N;
  constexpr int NT = V / 2;  // table entries (pairs) per unit
  const uint32_t t = threadIdx.x;
  const int dj = (int)(t & ((1u << p.uh_log2) - 1)) * V;  // the unit's offset in its head
  for (uint32_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
    const uint32_t b = p.div_s.div(r);
    const uint32_t s = r - b * p.S;
    float c[NT], sn[NT];
    const int64_t tb = (int64_t)s * p.table_stride + dj / 2;
    load_table<TT, NT>(cosine + tb, c);
    load_table<TT, NT>(sine + tb, sn);
#pragma unroll
    for (int e = 0; e < NT; ++e) sn[e] = p.sign * sn[e];
    const T* xr0 = p.x[0] + (int64_t)b * p.xb[0] + (int64_t)s * p.xs[0];
    const T* xr1 = p.x[1] + (int64_t)b * p.xb[1] + (int64_t)s * p.xs[1];
    T* or0 = p.out[0] + (int64_t)b * p.ob[0] + (int64_t)s * p.os[0];
    T* or1 = p.out[1] + (int64_t)b * p.ob[1] + (int64_t)s * p.os[1];
    for (uint32_t u0 = t; u0 < p.units; u0 += kRowThreads * kRowUnits) {
      uint4 a[kRowUnits];
      int64_t off[kRowUnits];
#pragma unroll
      for (int k = 0; k < kRowUnits; ++k) {
        const uint32_t u = u0 + k * kRowThreads;
        if (u >= p.units) continue;
        const bool second = u >= p.units0;
        off[k] = (int64_t)(second ? u - p.units0 : u) * V;
        a[k] = ld_stream((second ? xr1 : xr0) + off[k]);
      }
#pragma unroll
      for (int k = 0; k < kRowUnits; ++k) {
        const uint32_t u = u0 + k * kRowThreads;
        if (u >= p.units) continue;
        float f[V];
        unpack<T>(a[k], f);
#pragma unroll
        for (int q = 0; q < V / 2; ++q)
          rotate(f[2 * q], f[2 * q + 1], c[q], sn[q], f[2 * q], f[2 * q + 1]);
        st_stream((u >= p.units0 ? or1 : or0) + off[k], pack<T>(f));
      }
    }
  }
}

// Scalar path: one pair per thread iteration, any even D, any strides and alignment.
template <typename T, typename TT, bool kRotateHalf>
__global__ void __launch_bounds__(kThreads)
rope_scalar(const T* __restrict__ x, T* __restrict__ out, const TT* __restrict__ cosine,
            const TT* __restrict__ sine, RopeGeom g, int half_dim, int64_t total) {
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t pi = idx % half_dim;  // pair index within the head
    int64_t row = idx / half_dim;
    const int64_t i2 = row % g.n2;
    row /= g.n2;
    const int64_t i1 = row % g.n1;
    const int64_t i0 = row / g.n1;
    const int64_t s_idx = g.s_axis == 0 ? i0 : (g.s_axis == 1 ? i1 : i2);
    const int64_t xo = i0 * g.xs0 + i1 * g.xs1 + i2 * g.xs2;
    const int64_t oo = i0 * g.os0 + i1 * g.os1 + i2 * g.os2;
    const int64_t de = kRotateHalf ? pi : 2 * pi;
    const int64_t dod = kRotateHalf ? pi + half_dim : 2 * pi + 1;
    const float c = to_float(cosine[s_idx * g.table_stride + pi]);
    const float sn = g.sign * to_float(sine[s_idx * g.table_stride + pi]);
    float r1, r2;
    rotate(to_float(x[xo + de]), to_float(x[xo + dod]), c, sn, r1, r2);
    out[oo + de] = from_float<T>(r1);
    out[oo + dod] = from_float<T>(r2);
  }
}

// Geometry of one tensor: outer dims (B, H, S) ordered by decreasing x stride, and whether
// the 16-byte vector path can take it.
template <typename T, typename TT>
bool make_geom(RopeGeom& g, const void* x, const int64_t* xst, const void* out,
               const int64_t* ost, const int64_t* sizes, const void* cosine, const void* sine,
               int64_t tstride, bool rh, float sign, int64_t* total_vec) {
  int order[3] = {0, 1, 2};
  std::stable_sort(order, order + 3, [&](int a, int b) { return xst[a] > xst[b]; });
  g.n0 = (uint32_t)sizes[order[0]];
  g.n1 = (uint32_t)sizes[order[1]];
  g.n2 = (uint32_t)sizes[order[2]];
  g.xs0 = xst[order[0]]; g.xs1 = xst[order[1]]; g.xs2 = xst[order[2]];
  g.os0 = ost[order[0]]; g.os1 = ost[order[1]]; g.os2 = ost[order[2]];
  g.s_axis = order[0] == 2 ? 0 : (order[1] == 2 ? 1 : 2);
  g.table_stride = tstride;
  g.sign = sign;
  const int64_t D = sizes[3];
  const int64_t rows = sizes[0] * sizes[1] * sizes[2];
  g.same = xst[0] == ost[0] && xst[1] == ost[1] && xst[2] == ost[2];
  int64_t xmax = D, omax = D;
  for (int i = 0; i < 3; ++i) {
    xmax += (sizes[i] > 0 ? sizes[i] - 1 : 0) * xst[i];
    omax += (sizes[i] > 0 ? sizes[i] - 1 : 0) * ost[i];
  }
  g.small = xmax < ((int64_t)1 << 31) && omax < ((int64_t)1 << 31);
  constexpr int V = Vec16<T>::N;
  // Vector path: whole vectors per row, 16-byte aligned rows, table runs aligned to
  // their own size.
  const int64_t span = rh ? D / 2 : D;  // elements covered by the vectors of one row
  const int tbytes = (rh ? V : V / 2) * (int)sizeof(TT);
  const int talign = tbytes >= 16 ? 16 : tbytes;
  bool vec = span % V == 0 && aligned16(x) && aligned16(out);
  for (int i = 0; i < 3 && vec; ++i)
    vec = (xst[i] * (int64_t)sizeof(T)) % 16 == 0 && (ost[i] * (int64_t)sizeof(T)) % 16 == 0;
  vec = vec && (reinterpret_cast<uintptr_t>(cosine) % talign == 0) &&
        (reinterpret_cast<uintptr_t>(sine) % talign == 0) &&
        ((tstride * (int64_t)sizeof(TT)) % talign == 0);
  *total_vec = rows * (span / V);
  vec = vec && *total_vec < (int64_t)UINT32_MAX / 2;
  g.vpr = (uint32_t)(span / V);
  g.div_vpr = FastDiv(g.vpr > 0 ? g.vpr : 1);
  g.div_n2 = FastDiv(g.n2 > 0 ? g.n2 : 1);
  g.div_n1 = FastDiv(g.n1 > 0 ? g.n1 : 1);
  return vec;
}

// Whether the rows path can take these tensors (see rope_rows), and its parameters.
template <typename T, typename TT>
bool make_rows(RopeRows<T>& p, int n, const void* const* xs, const int64_t* const* xsts,
               void* const* outs, const int64_t* const* osts, const int64_t* const* sizes,
               const void* cosine, const void* sine, int64_t tstride, bool rh, float sign) {
  constexpr int V = Vec16<T>::N;
  if (rh) return false;
  const int64_t B = sizes[0][0], S = sizes[0][2], D = sizes[0][3];
  const int64_t uh = D / V;  // units per head
  if (D % V != 0 || uh < 1 || uh > kRowThreads || (uh & (uh - 1)) != 0) return false;
  const int tbytes = (V / 2) * (int)sizeof(TT);
  const int talign = tbytes >= 16 ? 16 : tbytes;
  if (reinterpret_cast<uintptr_t>(cosine) % talign || reinterpret_cast<uintptr_t>(sine) % talign ||
      (tstride * (int64_t)sizeof(TT)) % talign)
    return false;
  if (B * S >= (int64_t)UINT32_MAX) return false;
  int64_t units[2] = {0, 0};
  for (int i = 0; i < n; ++i) {
    const int64_t* sz = sizes[i];
    const int64_t* xst = xsts[i];
    const int64_t* ost = osts[i];
    if (sz[0] != B || sz[2] != S || sz[3] != D) return false;
    if (xst[1] != D || ost[1] != D) return false;  // contiguous (b, s) rows of heads
    if (!aligned16(xs[i]) || !aligned16(outs[i])) return false;
    for (int a : {0, 2})
      if ((xst[a] * (int64_t)sizeof(T)) % 16 || (ost[a] * (int64_t)sizeof(T)) % 16) return false;
    units[i] = sz[1] * uh;
  }
  if (units[0] + units[1] >= (int64_t)UINT32_MAX / 2) return false;
  for (int i = 0; i < 2; ++i) {
    const int k = i < n ? i : 0;
    p.x[i] = static_cast<const T*>(xs[k]);
    p.out[i] = static_cast<T*>(outs[k]);
    p.xb[i] = xsts[k][0];
    p.xs[i] = xsts[k][2];
    p.ob[i] = osts[k][0];
    p.os[i] = osts[k][2];
  }
  p.units0 = (uint32_t)units[0];
  p.units = (uint32_t)(units[0] + units[1]);
  p.rows = (uint32_t)(B * S);
  p.S = (uint32_t)S;
  p.div_s = FastDiv((uint32_t)(S > 0 ? S : 1));
  p.table_stride = tstride;
  int lg = 0;
  while ((int64_t(1) << lg) < uh) ++lg;
  p.uh_log2 = lg;
  p.sign = sign;
  return p.units > 0;
}

template <typename T, typename TT>
void launch_scalar(const T* x, T* out, const TT* cosine, const TT* sine, const RopeGeom& g,
                   int half, int64_t rows, bool rh, int sms, cudaStream_t stream) {
  const int64_t total = rows * half;
  const int64_t blocks = (total + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)sms * (2048 / kThreads);
  const int grid = (int)std::max<int64_t>(1, std::min(blocks, cap));
  if (rh)
    rope_scalar<T, TT, true><<<grid, kThreads, 0, stream>>>(x, out, cosine, sine, g, half, total);
  else
    rope_scalar<T, TT, false><<<grid, kThreads, 0, stream>>>(x, out, cosine, sine, g, half,
                                                             total);
}

// Rotates one or two tensors (n = 1 or 2) that share head_dim, the sequence length and the
// tables; two vector-path tensors go in one launch.
template <typename T, typename TT>
int rope_impl(int n, const void* const* xs, const int64_t* const* xsts, void* const* outs,
              const int64_t* const* osts, const int64_t* const* sizes, const void* cos_,
              const void* sin_, int64_t tstride, int layout, float sign, cudaStream_t stream,
              const char* what) {
  const TT* cosine = static_cast<const TT*>(cos_);
  const TT* sine = static_cast<const TT*>(sin_);
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  const bool rh = layout == PT_ROPE_ROTATE_HALF;
  const int half = (int)(sizes[0][3] / 2);
  RopeRows<T> rp;
  if (make_rows<T, TT>(rp, n, xs, xsts, outs, osts, sizes, cos_, sin_, tstride, rh, sign)) {
    const int grid = (int)std::max<int64_t>(
        1, std::min<int64_t>(rp.rows, (int64_t)sms * (2048 / kRowThreads)));
    rope_rows<T, TT><<<grid, kRowThreads, 0, stream>>>(rp, cosine, sine);
    return check_launch(what);
  }
  RopeJobs<T> jobs;
  int nvec = 0;
  for (int i = 0; i < n; ++i) {
    const int64_t rows = sizes[i][0] * sizes[i][1] * sizes[i][2];
    if (rows == 0) continue;
    RopeGeom g;
    int64_t total = 0;
    const bool vec = make_geom<T, TT>(g, xs[i], xsts[i], outs[i], osts[i], sizes[i], cos_, sin_,
                                      tstride, rh, sign, &total);
    if (!vec) {
      launch_scalar<T, TT>(static_cast<const T*>(xs[i]), static_cast<T*>(outs[i]), cosine,
                           sine, g, half, rows, rh, sms, stream);
      continue;
    }
    jobs.g[nvec] = g;
    jobs.x[nvec] = static_cast<const T*>(xs[i]);
    jobs.out[nvec] = static_cast<T*>(outs[i]);
    jobs.total[nvec] = (uint32_t)total;
    ++nvec;
  }
  if (nvec > 0) {
    if (nvec == 1) {
      jobs.g[1] = jobs.g[0];
      jobs.x[1] = jobs.x[0];
      jobs.out[1] = jobs.out[0];
      jobs.total[1] = 0;
    }
    const int threads = rh ? vec_threads<true>() : vec_threads<false>();
    const int64_t cap = (int64_t)sms * (2048 / threads);
    const int64_t per_block = (int64_t)threads * kUnroll;
    const int64_t need0 = (jobs.total[0] + per_block - 1) / per_block;
    const int64_t need1 = (jobs.total[1] + per_block - 1) / per_block;
    int64_t b0, b1;
    if (need0 + need1 <= cap) {
      b0 = need0;
      b1 = need1;
    } else {
      // Split the resident CTAs in proportion to the work, at least one each.
      b0 = std::max<int64_t>(1, (int64_t)((double)cap * jobs.total[0] /
                                         ((double)jobs.total[0] + (double)jobs.total[1])));
      b1 = jobs.total[1] > 0 ? std::max<int64_t>(1, cap - b0) : 0;
    }
    jobs.blocks0 = (uint32_t)b0;
    const int grid = (int)std::max<int64_t>(1, b0 + b1);
    if (rh)
      rope_vec<T, TT, true><<<grid, threads, 0, stream>>>(jobs, cosine, sine, half);
    else
      rope_vec<T, TT, false><<<grid, threads, 0, stream>>>(jobs, cosine, sine, half);
  }
  return check_launch(what);
}

int check_tensor(const void* x, const int64_t* xst, const void* out, const int64_t* ost,
                 const int64_t* sizes, int64_t tstride, const char* what) {
  if (xst == nullptr || ost == nullptr || sizes == nullptr)
    return set_error(PT_ERR_INVALID_ARGUMENT, "%s: strides/sizes must not be NULL", what);
  for (int i = 0; i < 4; ++i)
    if (sizes[i] < 0)
      return set_error(PT_ERR_SHAPE, "%s: sizes[%d] = %lld < 0", what, i, (long long)sizes[i]);
  const int64_t D = sizes[3];
  if (D <= 0 || D % 2 != 0)
    return set_error(PT_ERR_SHAPE, "%s: head_dim must be even and positive (got %lld)", what,
                     (long long)D);
  if (xst[3] != 1 || ost[3] != 1)
    return set_error(PT_ERR_SHAPE, "%s: the head_dim stride must be 1", what);
  for (int i = 0; i < 3; ++i)
    if (xst[i] < 0 || ost[i] < 0 || sizes[i] > (int64_t)UINT32_MAX)
      return set_error(PT_ERR_SHAPE, "%s: negative stride or outer size too large", what);
  if (tstride < D / 2)
    return set_error(PT_ERR_SHAPE, "%s: table_row_stride (%lld) < head_dim/2 (%lld)", what,
                     (long long)tstride, (long long)(D / 2));
  if (sizes[0] * sizes[1] * sizes[2] == 0) return PT_OK;
  if (int st = check_device_ptr(x, "x")) return st;
  if (int st = check_device_ptr(out, "out")) return st;
  return PT_OK;
}

// n = 1 or 2 tensors sharing head_dim, sequence length and the cosine/sine tables.
int rope_entry(int n, const void* const* xs, const int64_t* const* xsts, void* const* outs,
               const int64_t* const* osts, const int64_t* const* sizes, const void* cosine,
               const void* sine, int64_t tstride, int layout, int dtype, int table_dtype,
               float sign, void* stream, const char* what) {
  if (layout != PT_ROPE_INTERLEAVED && layout != PT_ROPE_ROTATE_HALF)
    return set_error(PT_ERR_INVALID_ARGUMENT, "%s: unknown layout %d", what, layout);
  int64_t rows = 0;
  for (int i = 0; i < n; ++i) {
    if (int st = check_tensor(xs[i], xsts[i], outs[i], osts[i], sizes[i], tstride, what))
      return st;
    rows += sizes[i][0] * sizes[i][1] * sizes[i][2];
  }
  if (n == 2 && (sizes[0][3] != sizes[1][3] || sizes[0][2] != sizes[1][2]))
    return set_error(PT_ERR_SHAPE, "%s: query and key must share head_dim and sequence length",
                     what);
  if (dtype_size(dtype) == 0 || dtype_size(table_dtype) == 0)
    return set_error(PT_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype (%d, table %d)", what, dtype,
                     table_dtype);
  if (rows == 0) return ok();
  if (int st = check_device_ptr(cosine, "cosine")) return st;
  if (int st = check_device_ptr(sine, "sine")) return st;
  cudaStream_t s = as_stream(stream);
#define PT_ROPE_CASE(DT, T, TDT, TT)                                                        \
  if (dtype == DT && table_dtype == TDT)                                                    \
    return rope_impl<T, TT>(n, xs, xsts, outs, osts, sizes, cosine, sine, tstride, layout,   \
                            sign, s, what);
  PT_ROPE_CASE(PT_BFLOAT16, __nv_bfloat16, PT_BFLOAT16, __nv_bfloat16)
  PT_ROPE_CASE(PT_BFLOAT16, __nv_bfloat16, PT_FLOAT32, float)
  PT_ROPE_CASE(PT_FLOAT16, __half, PT_FLOAT16, __half)
  PT_ROPE_CASE(PT_FLOAT16, __half, PT_FLOAT32, float)
  PT_ROPE_CASE(PT_FLOAT32, float, PT_FLOAT32, float)
#undef PT_ROPE_CASE
  return set_error(PT_ERR_UNSUPPORTED_DTYPE,
                   "%s: unsupported (dtype, table_dtype) = (%d, %d); the table must have the "
                   "states dtype or float32",
                   what, dtype, table_dtype);
}

}  // namespace
}  // namespace pt

extern "C" {

int pt_rope_fwd(const void* x, const int64_t x_strides[4], void* out, const int64_t out_strides[4],
                const int64_t sizes[4], const void* cosine, const void* sine,
                int64_t table_row_stride, int layout, int dtype, int table_dtype, void* stream) {
  const void* xs[1] = {x};
  const int64_t* xst[1] = {x_strides};
  void* outs[1] = {out};
  const int64_t* ost[1] = {out_strides};
  const int64_t* sz[1] = {sizes};
  return pt::rope_entry(1, xs, xst, outs, ost, sz, cosine, sine, table_row_stride, layout, dtype,
                        table_dtype, 1.0f, stream, "pt_rope_fwd");
}

int pt_rope_bwd(const void* dy, const int64_t dy_strides[4], void* dx, const int64_t dx_strides[4],
                const int64_t sizes[4], const void* cosine, const void* sine,
                int64_t table_row_stride, int layout, int dtype, int table_dtype, void* stream) {
  const void* xs[1] = {dy};
  const int64_t* xst[1] = {dy_strides};
  void* outs[1] = {dx};
  const int64_t* ost[1] = {dx_strides};
  const int64_t* sz[1] = {sizes};
  return pt::rope_entry(1, xs, xst, outs, ost, sz, cosine, sine, table_row_stride, layout, dtype,
                        table_dtype, -1.0f, stream, "pt_rope_bwd");
}

static int rope_qk(const void* q, const int64_t q_strides[4], void* q_out,
                   const int64_t q_out_strides[4], const int64_t q_sizes[4], const void* k,
                   const int64_t k_strides[4], void* k_out, const int64_t k_out_strides[4],
                   const int64_t k_sizes[4], const void* cosine, const void* sine,
                   int64_t table_row_stride, int layout, int dtype, int table_dtype, float sign,
                   void* stream, const char* what) {
  const void* xs[2] = {q, k};
  const int64_t* xst[2] = {q_strides, k_strides};
  void* outs[2] = {q_out, k_out};
  const int64_t* ost[2] = {q_out_strides, k_out_strides};
  const int64_t* sz[2] = {q_sizes, k_sizes};
  return pt::rope_entry(2, xs, xst, outs, ost, sz, cosine, sine, table_row_stride, layout, dtype,
                        table_dtype, sign, stream, what);
}

int pt_rope_qk_fwd(const void* q, const int64_t q_strides[4], void* q_out,
                   const int64_t q_out_strides[4], const int64_t q_sizes[4], const void* k,
                   const int64_t k_strides[4], void* k_out, const int64_t k_out_strides[4],
                   const int64_t k_sizes[4], const void* cosine, const void* sine,
                   int64_t table_row_stride, int layout, int dtype, int table_dtype,
                   void* stream) {
  return rope_qk(q, q_strides, q_out, q_out_strides, q_sizes, k, k_strides, k_out, k_out_strides,
                 k_sizes, cosine, sine, table_row_stride, layout, dtype, table_dtype, 1.0f,
                 stream, "pt_rope_qk_fwd");
}

int pt_rope_qk_bwd(const void* dq, const int64_t dq_strides[4], void* dq_out,
                   const int64_t dq_out_strides[4], const int64_t q_sizes[4], const void* dk,
                   const int64_t dk_strides[4], void* dk_out, const int64_t dk_out_strides[4],
                   const int64_t k_sizes[4], const void* cosine, const void* sine,
                   int64_t table_row_stride, int layout, int dtype, int table_dtype,
                   void* stream) {
  return rope_qk(dq, dq_strides, dq_out, dq_out_strides, q_sizes, dk, dk_strides, dk_out,
                 dk_out_strides, k_sizes, cosine, sine, table_row_stride, layout, dtype,
                 table_dtype, -1.0f, stream, "pt_rope_qk_bwd");
}

}  // extern "C"
