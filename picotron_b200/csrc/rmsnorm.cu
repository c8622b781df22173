// RMSNorm forward/backward and the deterministic dweight reduction for sm_100a.
//
// Math follows src/picotron/nn/triton_kernels/rmsnorm.py of the reference:
//   forward  (:25-46, :49-60)   r = rsqrt(mean(x^2) + eps), y = (x * r) * w, fp32 math
//   backward (:109-134)          g = dy * w, dx = r * (g - (x * r^2) * mean(g * x)),
//                                dw = sum_rows (dy * x) * r, fp32 math
//
// Layout: x, y, dy, dx are [rows, hidden] with a row stride and contiguous columns.
//
// Fast path ("column-owner" kernels): each CTA owns a fixed set of 16-byte column
// vectors (thread t owns vectors t, t + blockDim, ...; a warp therefore touches
// contiguous 512-byte runs). The weight of those columns lives in registers for the
// whole kernel, and so does the backward's dweight accumulator, so weight is read once
// per CTA and dweight leaves the kernel as one fp32 partial row per CTA. A CTA
// processes R rows per iteration (R rows' loads in flight before the first reduction),
// one __syncthreads per iteration (the reduction buffer is double-buffered).
//
// Generic path: any hidden size, stride or alignment; one row per CTA iteration with
// scalar accesses and two passes over the row (the second one hits L2).
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"

namespace pt {
namespace {

// Tuning table. A fast-path CTA has at most kMaxThreads threads; each thread owns VPT
// 16-byte column vectors and keeps R rows in flight. Forward holds one input row per
// row in flight, backward two (x and dy) plus the dweight accumulator, so backward
// keeps fewer rows in flight to stay clear of register spills.
#ifndef PT_RMS_MAX_THREADS
#define PT_RMS_MAX_THREADS 512
#endif
constexpr int kMaxThreads = PT_RMS_MAX_THREADS;
constexpr int kGenericThreads = 256;

constexpr int fwd_rows_in_flight(int vpt) { return vpt == 1 ? 4 : (vpt == 2 ? 2 : 1); }
constexpr int bwd_rows_in_flight(int vpt) { return vpt == 1 ? 2 : 1; }

// Sum of `v` over the CTA; `red` is a 32-float shared buffer owned by the caller.
// Leaves the result in every thread. No trailing barrier: callers alternate buffers.
__device__ __forceinline__ float block_sum_nosync(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nwarps ? red[lane] : 0.0f;
  return warp_sum(t);
}

// ---------------------------------------------------------------- fast forward -----
template <typename T, typename TW, int VPT, int R>
__global__ void __launch_bounds__(kMaxThreads)
rmsnorm_fwd_vec(const T* __restrict__ x, int64_t xs, const TW* __restrict__ w,
                T* __restrict__ y, int64_t ys, float* __restrict__ rstd, int64_t rows,
                int nvec, float hidden_f, float eps) {
  constexpr int V = Vec16<T>::N;
  __shared__ float red[2][R][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;

  float wf[VPT][V];
  bool valid[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = tid + k * blockDim.x;
    valid[k] = v < nvec;
    if (valid[k]) {
      load_row_f32<TW, V>(w + (int64_t)v * V, wf[k]);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) wf[k][j] = 0.0f;
    }
  }

  int p = 0;
  for (int64_t base = (int64_t)blockIdx.x * R; base < rows; base += (int64_t)gridDim.x * R) {
    uint4 xv[R][VPT];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = base + r;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (row < rows && valid[k])
          xv[r][k] = ld_stream(x + row * xs + (int64_t)(tid + k * blockDim.x) * V);
        else
          xv[r][k] = make_uint4(0, 0, 0, 0);
      }
    }
    float ss[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      ss[r] = 0.0f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        float f[V];
        unpack<T>(xv[r][k], f);
#pragma unroll
        for (int j = 0; j < V; ++j) ss[r] = fmaf(f[j], f[j], ss[r]);
      }
      ss[r] = warp_sum(ss[r]);
      if (lane == 0) red[p][r][warp] = ss[r];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float t = lane < nwarps ? red[p][r][lane] : 0.0f;
      t = warp_sum(t);
      const float inv = rsqrtf(t / hidden_f + eps);
      const int64_t row = base + r;
      if (row < rows) {
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          if (!valid[k]) continue;
          float f[V];
          unpack<T>(xv[r][k], f);
#pragma unroll
          for (int j = 0; j < V; ++j) f[j] = (f[j] * inv) * wf[k][j];
          st_stream(y + row * ys + (int64_t)(tid + k * blockDim.x) * V, pack<T>(f));
        }
        if (rstd != nullptr && tid == 0) rstd[row] = inv;
      }
    }
    p ^= 1;
  }
}

// --------------------------------------------------------------- fast backward -----
template <typename T, typename TW, int VPT, int R, bool kHasRstd>
__global__ void __launch_bounds__(kMaxThreads)
rmsnorm_bwd_vec(const T* __restrict__ dy, int64_t dys, const T* __restrict__ x, int64_t xs,
                const TW* __restrict__ w, const float* __restrict__ rstd, T* __restrict__ dx,
                int64_t dxs, float* __restrict__ partials, int64_t rows, int nvec, int hidden,
                float hidden_f, float eps) {
  constexpr int V = Vec16<T>::N;
  __shared__ float red[2][2 * R][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;

  float wf[VPT][V];
  float acc[VPT][V];
  bool valid[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = tid + k * blockDim.x;
    valid[k] = v < nvec;
#pragma unroll
    for (int j = 0; j < V; ++j) acc[k][j] = 0.0f;
    if (valid[k]) {
      load_row_f32<TW, V>(w + (int64_t)v * V, wf[k]);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) wf[k][j] = 0.0f;
    }
  }

  int p = 0;
  for (int64_t base = (int64_t)blockIdx.x * R; base < rows; base += (int64_t)gridDim.x * R) {
    uint4 xv[R][VPT], gv[R][VPT];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = base + r;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int64_t col = (int64_t)(tid + k * blockDim.x) * V;
        if (row < rows && valid[k]) {
          xv[r][k] = ld_stream(x + row * xs + col);
          gv[r][k] = ld_stream(dy + row * dys + col);
        } else {
          xv[r][k] = make_uint4(0, 0, 0, 0);
          gv[r][k] = make_uint4(0, 0, 0, 0);
        }
      }
    }
    // Per-row partial sums: sum(x^2) (unless rstd is given) and sum(g * x), g = dy * w.
    float ss[R], dot[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      ss[r] = 0.0f;
      dot[r] = 0.0f;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        float fx[V], fg[V];
        unpack<T>(xv[r][k], fx);
        unpack<T>(gv[r][k], fg);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          if (!kHasRstd) ss[r] = fmaf(fx[j], fx[j], ss[r]);
          dot[r] = fmaf(fg[j] * wf[k][j], fx[j], dot[r]);
        }
      }
      if (!kHasRstd) ss[r] = warp_sum(ss[r]);
      dot[r] = warp_sum(dot[r]);
      if (lane == 0) {
        red[p][2 * r][warp] = ss[r];
        red[p][2 * r + 1][warp] = dot[r];
      }
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int64_t row = base + r;
      float tdot = lane < nwarps ? red[p][2 * r + 1][lane] : 0.0f;
      tdot = warp_sum(tdot);
      float inv;
      if (kHasRstd) {
        inv = row < rows ? __ldg(rstd + row) : 0.0f;
      } else {
        float tss = lane < nwarps ? red[p][2 * r][lane] : 0.0f;
        tss = warp_sum(tss);
        inv = rsqrtf(tss / hidden_f + eps);
      }
      if (row < rows) {
        const float dot_mean = tdot / hidden_f;
        const float c = (inv * inv) * dot_mean;
#pragma unroll
        for (int k = 0; k < VPT; ++k) {
          if (!valid[k]) continue;
          float fx[V], fg[V], fo[V];
          unpack<T>(xv[r][k], fx);
          unpack<T>(gv[r][k], fg);
#pragma unroll
          for (int j = 0; j < V; ++j) {
            const float g = fg[j] * wf[k][j];
            fo[j] = inv * (g - fx[j] * c);
            acc[k][j] = fmaf(fg[j] * fx[j], inv, acc[k][j]);
          }
          st_stream(dx + row * dxs + (int64_t)(tid + k * blockDim.x) * V, pack<T>(fo));
        }
      }
    }
    p ^= 1;
  }

  // This CTA's dweight partial row (zeros when it owned no rows).
  float* prow = partials + (int64_t)blockIdx.x * hidden;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    if (!valid[k]) continue;
    float4* dst = reinterpret_cast<float4*>(prow + (int64_t)(tid + k * blockDim.x) * V);
#pragma unroll
    for (int j = 0; j < V / 4; ++j)
      dst[j] = make_float4(acc[k][4 * j], acc[k][4 * j + 1], acc[k][4 * j + 2], acc[k][4 * j + 3]);
  }
}

// --------------------------------------------------------------- generic paths -----
template <typename T, typename TW>
__global__ void __launch_bounds__(kGenericThreads)
rmsnorm_fwd_generic(const T* __restrict__ x, int64_t xs, const TW* __restrict__ w,
                    T* __restrict__ y, int64_t ys, float* __restrict__ rstd, int64_t rows,
                    int hidden, float eps) {
  __shared__ float red[2][32];
  int p = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * xs;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float f = to_float(xr[c]);
      ss = fmaf(f, f, ss);
    }
    const float inv = rsqrtf(block_sum_nosync(ss, red[p]) / (float)hidden + eps);
    T* yr = y + row * ys;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x)
      yr[c] = from_float<T>((to_float(xr[c]) * inv) * to_float(w[c]));
    if (rstd != nullptr && threadIdx.x == 0) rstd[row] = inv;
    p ^= 1;
  }
}

template <typename T, typename TW>
__global__ void __launch_bounds__(kGenericThreads)
rmsnorm_bwd_generic(const T* __restrict__ dy, int64_t dys, const T* __restrict__ x, int64_t xs,
                    const TW* __restrict__ w, const float* __restrict__ rstd,
                    T* __restrict__ dx, int64_t dxs, float* __restrict__ partials,
                    int64_t rows, int hidden, float eps) {
  __shared__ float red[4][32];
  // Each thread only ever touches the partial columns c = threadIdx.x + k * blockDim.x of
  // this CTA's partial row, so no barrier is needed around the accumulation.
  float* prow = partials + (int64_t)blockIdx.x * hidden;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) prow[c] = 0.0f;
  int p = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * xs;
    const T* gr = dy + row * dys;
    float ss = 0.0f, dot = 0.0f;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float fx = to_float(xr[c]);
      ss = fmaf(fx, fx, ss);
      dot = fmaf(to_float(gr[c]) * to_float(w[c]), fx, dot);
    }
    float inv;
    if (rstd != nullptr) {
      inv = rstd[row];
    } else {
      inv = rsqrtf(block_sum_nosync(ss, red[2 * p]) / (float)hidden + eps);
    }
    const float dot_mean = block_sum_nosync(dot, red[2 * p + 1]) / (float)hidden;
    const float cc = (inv * inv) * dot_mean;
    T* dr = dx + row * dxs;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float fx = to_float(xr[c]);
      const float fg = to_float(gr[c]);
      dr[c] = from_float<T>(inv * (fg * to_float(w[c]) - fx * cc));
      prow[c] = fmaf(fg * fx, inv, prow[c]);
    }
    p ^= 1;
  }
}

template <typename TW>
__global__ void __launch_bounds__(256)
rmsnorm_dw_reduce_kernel(const float* __restrict__ partials, int num_partials, int64_t hidden,
                         TW* __restrict__ dw) {
  // 32 columns per CTA (one per lane), 8 warps split the partial rows; warp w sums rows
  // w, w + 8, ... in increasing order, then warp sums are added in warp order. The order
  // depends only on num_partials, so the result is deterministic.
  __shared__ float s[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t c = (int64_t)blockIdx.x * 32 + lane;
  float acc = 0.0f;
  if (c < hidden)
    for (int p = warp; p < num_partials; p += 8) acc += partials[(int64_t)p * hidden + c];
  s[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && c < hidden) {
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += s[i][lane];
    dw[c] = from_float<TW>(t);
  }
}

// ------------------------------------------------------------------ host helpers ---

// Resident CTAs per SM for a kernel at a block size; cached, the value never changes.
int blocks_per_sm(const void* func, int threads) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t key = (reinterpret_cast<uint64_t>(func) * 1315423911ull) ^
                       ((uint64_t)threads << 8) ^ (uint64_t)dev;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, 0) != cudaSuccess) {
    cudaGetLastError();
    n = 1;
  }
  if (n < 1) n = 1;
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

struct FastPlan {
  bool ok = false;
  int vpt = 0;
  int threads = 0;
  int nvec = 0;
};

// Chooses the column-owner layout: the fewest vectors per thread that keep the CTA
// within kMaxThreads. Returns ok=false when the row shape needs the generic path.
template <typename T>
FastPlan plan_fast(int64_t hidden) {
  FastPlan plan;
  constexpr int V = Vec16<T>::N;
  if (hidden <= 0 || hidden % V != 0) return plan;
  const int64_t nvec = hidden / V;
  for (int vpt : {1, 2, 4}) {
    const int64_t need = (nvec + vpt - 1) / vpt;
    if (need <= kMaxThreads) {
      plan.ok = true;
      plan.vpt = vpt;
      plan.nvec = (int)nvec;
      plan.threads = (int)((need + 31) / 32 * 32);
      return plan;
    }
  }
  return plan;
}

template <typename T>
bool rows_aligned(const void* p, int64_t stride) {
  return aligned16(p) && ((stride * (int64_t)sizeof(T)) % 16 == 0);
}

template <typename T, typename TW>
int fwd_impl(const void* x_, int64_t xs, const void* w_, void* y_, int64_t ys, float* rstd,
             int64_t rows, int64_t hidden, float eps, cudaStream_t stream) {
  const T* x = static_cast<const T*>(x_);
  const TW* w = static_cast<const TW*>(w_);
  T* y = static_cast<T*>(y_);
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  FastPlan plan = plan_fast<T>(hidden);
  const bool fast = plan.ok && rows_aligned<T>(x, xs) && rows_aligned<T>(y, ys) && aligned16(w);
  if (fast) {
#define PT_FWD_KERNEL(VPT) rmsnorm_fwd_vec<T, TW, VPT, fwd_rows_in_flight(VPT)>
    const void* fn = plan.vpt == 1   ? (const void*)PT_FWD_KERNEL(1)
                     : plan.vpt == 2 ? (const void*)PT_FWD_KERNEL(2)
                                     : (const void*)PT_FWD_KERNEL(4);
    const int R = fwd_rows_in_flight(plan.vpt);
    const int64_t groups = (rows + R - 1) / R;
    const int64_t resident = (int64_t)sms * blocks_per_sm(fn, plan.threads);
    const int grid = (int)(groups < resident ? groups : resident);
    const float hf = (float)hidden;
    switch (plan.vpt) {
      case 1:
        PT_FWD_KERNEL(1)<<<grid, plan.threads, 0, stream>>>(x, xs, w, y, ys, rstd, rows,
                                                            plan.nvec, hf, eps);
        break;
      case 2:
        PT_FWD_KERNEL(2)<<<grid, plan.threads, 0, stream>>>(x, xs, w, y, ys, rstd, rows,
                                                            plan.nvec, hf, eps);
        break;
      default:
        PT_FWD_KERNEL(4)<<<grid, plan.threads, 0, stream>>>(x, xs, w, y, ys, rstd, rows,
                                                            plan.nvec, hf, eps);
        break;
    }
#undef PT_FWD_KERNEL
  } else {
    const void* fn = (const void*)rmsnorm_fwd_generic<T, TW>;
    const int64_t resident = (int64_t)sms * blocks_per_sm(fn, kGenericThreads);
    const int grid = (int)(rows < resident ? rows : resident);
    rmsnorm_fwd_generic<T, TW><<<grid, kGenericThreads, 0, stream>>>(x, xs, w, y, ys, rstd, rows,
                                                                     (int)hidden, eps);
  }
  return check_launch("pt_rmsnorm_fwd");
}

#define PT_BWD_KERNEL(VPT, HR) rmsnorm_bwd_vec<T, TW, VPT, bwd_rows_in_flight(VPT), HR>

template <typename T, typename TW>
const void* bwd_kernel_for(const FastPlan& plan, bool has_rstd) {
  switch (plan.vpt) {
    case 1: return has_rstd ? (const void*)PT_BWD_KERNEL(1, true) : (const void*)PT_BWD_KERNEL(1, false);
    case 2: return has_rstd ? (const void*)PT_BWD_KERNEL(2, true) : (const void*)PT_BWD_KERNEL(2, false);
    default: return has_rstd ? (const void*)PT_BWD_KERNEL(4, true) : (const void*)PT_BWD_KERNEL(4, false);
  }
}

template <typename T, typename TW>
int num_partials_impl(int64_t rows, int64_t hidden, int* out) {
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  FastPlan plan = plan_fast<T>(hidden);
  int64_t n;
  if (plan.ok) {
    const int R = bwd_rows_in_flight(plan.vpt);
    const int64_t groups = (rows + R - 1) / R;
    n = (int64_t)sms * blocks_per_sm(bwd_kernel_for<T, TW>(plan, false), plan.threads);
    if (groups < n) n = groups;
  } else {
    n = (int64_t)sms * blocks_per_sm((const void*)rmsnorm_bwd_generic<T, TW>, kGenericThreads);
    if (rows < n) n = rows;
  }
  if (n < 1) n = 1;
  *out = (int)n;
  return ok();
}

template <typename T, typename TW>
int bwd_impl(const void* dy_, int64_t dys, const void* x_, int64_t xs, const void* w_,
             const float* rstd, void* dx_, int64_t dxs, float* partials, int num_partials,
             int64_t rows, int64_t hidden, float eps, cudaStream_t stream) {
  const T* dy = static_cast<const T*>(dy_);
  const T* x = static_cast<const T*>(x_);
  const TW* w = static_cast<const TW*>(w_);
  T* dx = static_cast<T*>(dx_);
  FastPlan plan = plan_fast<T>(hidden);
  const bool fast = plan.ok && rows_aligned<T>(x, xs) && rows_aligned<T>(dy, dys) &&
                    rows_aligned<T>(dx, dxs) && aligned16(w) && aligned16(partials);
  const float hf = (float)hidden;
  if (fast) {
    const bool hr = rstd != nullptr;
#define PT_BWD_LAUNCH(VPT, HR)                                                              \
  PT_BWD_KERNEL(VPT, HR)<<<num_partials, plan.threads, 0, stream>>>(                        \
      dy, dys, x, xs, w, rstd, dx, dxs, partials, rows, plan.nvec, (int)hidden, hf, eps)
    switch (plan.vpt) {
      case 1: if (hr) PT_BWD_LAUNCH(1, true); else PT_BWD_LAUNCH(1, false); break;
      case 2: if (hr) PT_BWD_LAUNCH(2, true); else PT_BWD_LAUNCH(2, false); break;
      default: if (hr) PT_BWD_LAUNCH(4, true); else PT_BWD_LAUNCH(4, false); break;
    }
#undef PT_BWD_LAUNCH
  } else {
    rmsnorm_bwd_generic<T, TW><<<num_partials, kGenericThreads, 0, stream>>>(
        dy, dys, x, xs, w, rstd, dx, dxs, partials, rows, (int)hidden, eps);
  }
  return check_launch("pt_rmsnorm_bwd");
}

// Dispatch on the (x, w) dtype pair. Returns PT_ERR_UNSUPPORTED_DTYPE for pairs that
// are not built.
template <typename F>
int dispatch_xw(int x_dtype, int w_dtype, F&& f) {
  if (x_dtype == PT_FLOAT32 && w_dtype == PT_FLOAT32) return f((float*)0, (float*)0);
  if (x_dtype == PT_BFLOAT16 && w_dtype == PT_BFLOAT16)
    return f((__nv_bfloat16*)0, (__nv_bfloat16*)0);
  if (x_dtype == PT_BFLOAT16 && w_dtype == PT_FLOAT32) return f((__nv_bfloat16*)0, (float*)0);
  if (x_dtype == PT_FLOAT16 && w_dtype == PT_FLOAT16) return f((__half*)0, (__half*)0);
  if (x_dtype == PT_FLOAT16 && w_dtype == PT_FLOAT32) return f((__half*)0, (float*)0);
  return set_error(PT_ERR_UNSUPPORTED_DTYPE,
                   "unsupported (x_dtype, w_dtype) = (%d, %d); supported: (f32,f32) "
                   "(f16,f16) (f16,f32) (bf16,bf16) (bf16,f32)",
                   x_dtype, w_dtype);
}

int check_shape(int64_t rows, int64_t hidden) {
  if (rows < 0) return set_error(PT_ERR_SHAPE, "rows must be >= 0 (got %lld)", (long long)rows);
  if (hidden <= 0 || hidden > (int64_t)(1 << 30))
    return set_error(PT_ERR_SHAPE, "hidden must be in [1, 2^30] (got %lld)", (long long)hidden);
  return PT_OK;
}

int check_row_stride(int64_t stride, int64_t hidden, const char* name) {
  if (stride < hidden)
    return set_error(PT_ERR_SHAPE, "%s (%lld) must be >= hidden (%lld)", name, (long long)stride,
                     (long long)hidden);
  return PT_OK;
}

}  // namespace
}  // namespace pt

using namespace pt;

extern "C" {

int pt_rmsnorm_fwd(const void* x, int64_t x_row_stride, const void* weight, void* y,
                   int64_t y_row_stride, float* rstd, int64_t rows, int64_t hidden, int x_dtype,
                   int w_dtype, float eps, void* stream) {
  if (int st = check_shape(rows, hidden)) return st;
  if (!(eps >= 0.0f)) return set_error(PT_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (rows == 0) return ok();
  if (int st = check_row_stride(x_row_stride, hidden, "x_row_stride")) return st;
  if (int st = check_row_stride(y_row_stride, hidden, "y_row_stride")) return st;
  if (int st = check_device_ptr(x, "x")) return st;
  if (int st = check_device_ptr(weight, "weight")) return st;
  if (int st = check_device_ptr(y, "y")) return st;
  if (rstd)
    if (int st = check_device_ptr(rstd, "rstd")) return st;
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return fwd_impl<T, TW>(x, x_row_stride, weight, y, y_row_stride, rstd, rows, hidden, eps,
                           as_stream(stream));
  });
}

int pt_rmsnorm_bwd_num_partials(int64_t rows, int64_t hidden, int x_dtype, int w_dtype,
                                int* num_partials) {
  if (num_partials == nullptr)
    return set_error(PT_ERR_INVALID_ARGUMENT, "num_partials is NULL");
  if (int st = check_shape(rows, hidden)) return st;
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return num_partials_impl<T, TW>(rows, hidden, num_partials);
  });
}

int pt_rmsnorm_bwd(const void* dy, int64_t dy_row_stride, const void* x, int64_t x_row_stride,
                   const void* weight, const float* rstd, void* dx, int64_t dx_row_stride,
                   float* dw_partials, int num_partials, int64_t rows, int64_t hidden,
                   int x_dtype, int w_dtype, float eps, void* stream) {
  if (int st = check_shape(rows, hidden)) return st;
  if (!(eps >= 0.0f)) return set_error(PT_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (num_partials < 1)
    return set_error(PT_ERR_INVALID_ARGUMENT, "num_partials must be >= 1 (got %d)", num_partials);
  if (int st = check_device_ptr(dw_partials, "dw_partials")) return st;
  if (int st = check_device_ptr(weight, "weight")) return st;
  if (rows > 0) {
    if (int st = check_row_stride(dy_row_stride, hidden, "dy_row_stride")) return st;
    if (int st = check_row_stride(x_row_stride, hidden, "x_row_stride")) return st;
    if (int st = check_row_stride(dx_row_stride, hidden, "dx_row_stride")) return st;
    if (int st = check_device_ptr(dy, "dy")) return st;
    if (int st = check_device_ptr(x, "x")) return st;
    if (int st = check_device_ptr(dx, "dx")) return st;
    if (rstd)
      if (int st = check_device_ptr(rstd, "rstd")) return st;
  }
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return bwd_impl<T, TW>(dy, dy_row_stride, x, x_row_stride, weight, rstd, dx, dx_row_stride,
                           dw_partials, num_partials, rows, hidden, eps, as_stream(stream));
  });
}

int pt_rmsnorm_dw_reduce(const float* dw_partials, int num_partials, int64_t hidden, void* dw,
                         int dw_dtype, void* stream) {
  if (num_partials < 1)
    return set_error(PT_ERR_INVALID_ARGUMENT, "num_partials must be >= 1 (got %d)", num_partials);
  if (hidden <= 0 || hidden > (int64_t)(1 << 30))
    return set_error(PT_ERR_SHAPE, "hidden must be in [1, 2^30] (got %lld)", (long long)hidden);
  if (int st = check_device_ptr(dw_partials, "dw_partials")) return st;
  if (int st = check_device_ptr(dw, "dw")) return st;
  const int grid = (int)((hidden + 31) / 32);
  cudaStream_t s = as_stream(stream);
  switch (dw_dtype) {
    case PT_FLOAT32:
      rmsnorm_dw_reduce_kernel<float><<<grid, 256, 0, s>>>(dw_partials, num_partials, hidden,
                                                           static_cast<float*>(dw));
      break;
    case PT_FLOAT16:
      rmsnorm_dw_reduce_kernel<__half><<<grid, 256, 0, s>>>(dw_partials, num_partials, hidden,
                                                            static_cast<__half*>(dw));
      break;
    case PT_BFLOAT16:
      rmsnorm_dw_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          dw_partials, num_partials, hidden, static_cast<__nv_bfloat16*>(dw));
      break;
    default:
      return set_error(PT_ERR_UNSUPPORTED_DTYPE, "unsupported dw_dtype %d", dw_dtype);
  }
  return check_launch("pt_rmsnorm_dw_reduce");
}

}  // extern "C"
