// Cross-entropy over vocabulary rows on sm_100a: per-row loss and log-sum-exp (forward), the
// deterministic mean over the non-ignored rows, and the logits gradient (backward).
//
// Replaces picotron's loss: F.cross_entropy(logits[:, :-1, :].transpose(1, 2), input_ids[:, 1:])
// (src/picotron/training/train_loop.py:95-97, 141-145; mean reduction, ignore_index -100) and
// its forward-only Triton kernel (src/picotron/nn/triton_kernels/cross_entropy.py:28-87). The
// rows are addressed as [outer, inner] with two strides, so the training call's strided view
// of [B, S, V] logits (positions 0..S-2 of every sequence) is read in place, with no copy.
//
// One CTA per row (grid-stride): 16-byte loads of the row, an online max / sum-of-exponentials
// per thread (the running sum is rescaled when the maximum grows), then a CTA reduction of the
// (max, sum) pairs. The backward recomputes exp(x - lse) from the saved per-row lse and writes
// (softmax - onehot) * grad / count with streaming stores.

#include <cmath>

#include "common.cuh"

namespace pt {

__device__ int g_ce_error = 0;

namespace {

// One row per 128-thread CTA (A/B on B200 at 16384 x 128256 bf16: forward 0.92 and backward
// 0.92 of the HBM peak, against 0.85 / 0.87 with 256 threads): more rows in flight per SM.
constexpr int kCeThreads = 128;
// 16-byte vectors in flight per thread: 8 in the forward (A/B: 0.95 against 0.93 with 4),
// 4 in the backward, which also writes (0.92 against 0.90 with 8).
constexpr int kCeUnrollFwd = 8;
constexpr int kCeUnrollBwd = 4;
constexpr int kMeanThreads = 1024;
constexpr float kLog2e = 1.4426950408889634f;  // log2(e): exp(a) = 2^(a * log2(e))
constexpr int kCeErrBadTarget = 2;

// Row r of the [outer, inner] row grid sits at outer index r / inner, inner index r % inner.
struct RowGrid {
  int64_t inner;
  int64_t outer_stride, inner_stride;  // elements
  __device__ __forceinline__ int64_t offset(int64_t r) const {
    const int64_t o = r / inner;
    return o * outer_stride + (r - o * inner) * inner_stride;
  }
};

// Running (max, sum of exp(x - max)) of a set of values, merged without overflow.
struct MaxSum {
  float m, s;
};

// 2^x on the special-function unit (PTX ex2.approx.ftz: relative error below 2^-22; results
// under 2^-126 flush to zero, which is negligible next to a row's largest term, 1).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float scale_to(float a, float M) {
  return a == -INFINITY ? 0.0f : fast_exp2((a - M) * kLog2e);
}

__device__ __forceinline__ MaxSum merge(MaxSum a, MaxSum b) {
  const float M = fmaxf(a.m, b.m);
  return {M, a.s * scale_to(a.m, M) + b.s * scale_to(b.m, M)};
}

// Per-thread running state: the max and two partial sums (paired FP32 lanes).
struct Running {
  float m = -INFINITY;
  float2 s = make_float2(0.0f, 0.0f);
};

// Adds N values (N even, fp32) to the running state.
template <int N>
__device__ __forceinline__ void absorb(Running& acc, const float* x) {
  float vmax = x[0];
#pragma unroll
  for (int e = 1; e < N; ++e) vmax = fmaxf(vmax, x[e]);
  if (vmax > acc.m) {
    const float f = scale_to(acc.m, vmax);
    acc.s = __fmul2_rn(acc.s, splat2(f));
    acc.m = vmax;
  }
  if (acc.m == -INFINITY) return;  // every value so far is -inf: nothing to add
  const float2 L2 = splat2(kLog2e), nmL2 = splat2(-acc.m * kLog2e);
#pragma unroll
  for (int e = 0; e < N; e += 2) {
    const float2 t = __ffma2_rn(make_float2(x[e], x[e + 1]), L2, nmL2);
    acc.s = __fadd2_rn(acc.s, make_float2(fast_exp2(t.x), fast_exp2(t.y)));
  }
}

__device__ __forceinline__ void absorb1(Running& acc, float x) {
  if (x > acc.m) {
    const float f = scale_to(acc.m, x);
    acc.s = __fmul2_rn(acc.s, splat2(f));
    acc.m = x;
  }
  if (acc.m == -INFINITY) return;
  acc.s.x += fast_exp2(fmaf(x, kLog2e, -acc.m * kLog2e));
}

__device__ __forceinline__ MaxSum block_merge(MaxSum v, MaxSum* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    MaxSum o{__shfl_xor_sync(0xffffffffu, v.m, off), __shfl_xor_sync(0xffffffffu, v.s, off)};
    v = merge(v, o);
  }
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < nw ? red[lane] : MaxSum{-INFINITY, 0.0f};
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      MaxSum o{__shfl_xor_sync(0xffffffffu, v.m, off), __shfl_xor_sync(0xffffffffu, v.s, off)};
      v = merge(v, o);
    }
  }
  return v;  // valid in warp 0
}

// Elements before the first 16-byte boundary of a row (0 when it is aligned).
template <typename T> __device__ __forceinline__ int64_t head_elems(const T* p, int64_t vocab) {
  const int64_t mis = (int64_t)(reinterpret_cast<uintptr_t>(p) & 15u);
  const int64_t h = mis ? (16 - mis) / (int64_t)sizeof(T) : 0;
  return h < vocab ? h : vocab;
}

template <typename T>
__global__ void __launch_bounds__(kCeThreads)
ce_fwd_kernel(const T* __restrict__ logits, RowGrid lg, const int64_t* __restrict__ targets,
              RowGrid tg, int64_t rows, int64_t vocab, int64_t ignore_index,
              float* __restrict__ row_loss, float* __restrict__ row_lse) {
  constexpr int V = Vec16<T>::N;
  __shared__ MaxSum red[kCeThreads / 32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = logits + lg.offset(r);
    Running acc;
    const int64_t head = head_elems(row, vocab);
    if (threadIdx.x < head) absorb1(acc, to_float(row[threadIdx.x]));
    const T* body = row + head;
    const int64_t nvec = (vocab - head) / V;
    int64_t v = threadIdx.x;
    for (; v + (kCeUnrollFwd - 1) * kCeThreads < nvec; v += kCeUnrollFwd * kCeThreads) {
      uint4 raw[kCeUnrollFwd];
#pragma unroll
      for (int u = 0; u < kCeUnrollFwd; ++u) raw[u] = ld_stream(body + (v + u * kCeThreads) * V);
#pragma unroll
      for (int u = 0; u < kCeUnrollFwd; ++u) {
        float x[V];
        unpack<T>(raw[u], x);
        absorb<V>(acc, x);
      }
    }
    for (; v < nvec; v += kCeThreads) {
      float x[V];
      unpack<T>(ld_stream(body + v * V), x);
      absorb<V>(acc, x);
    }
    for (int64_t c = head + nvec * V + threadIdx.x; c < vocab; c += kCeThreads)
      absorb1(acc, to_float(row[c]));
    const MaxSum tot = block_merge(MaxSum{acc.m, acc.s.x + acc.s.y}, red);
    if (threadIdx.x == 0) {
      const float lse = tot.m + logf(tot.s);
      const int64_t t = targets[tg.offset(r)];
      float loss;
      if (t == ignore_index) {
        loss = 0.0f;
      } else if (t < 0 || t >= vocab) {
        loss = NAN;  // the reference raises; a kernel cannot: poison the row and flag it
        atomicExch(&g_ce_error, kCeErrBadTarget);
      } else {
        loss = lse - to_float(row[t]);
      }
      row_loss[r] = loss;
      row_lse[r] = lse;
    }
    __syncthreads();  // `red` is reused by the next row
  }
}

// out[0] = mean of row_loss over rows whose target is not ignore_index, out[1] = 1 / count.
// One CTA; thread j sums rows j, j + 1024, ... in fp64, then a fixed-order tree: the result
// depends only on the inputs. count == 0 gives NaN in both (a mean over nothing).
__global__ void __launch_bounds__(kMeanThreads)
ce_mean_kernel(const float* __restrict__ row_loss, const int64_t* __restrict__ targets,
               RowGrid tg, int64_t rows, int64_t ignore_index, float* __restrict__ out) {
  __shared__ double sum[kMeanThreads];
  __shared__ long long cnt[kMeanThreads];
  double s = 0.0;
  long long c = 0;
  for (int64_t r = threadIdx.x; r < rows; r += kMeanThreads) {
    if (targets[tg.offset(r)] != ignore_index) {
      s += (double)row_loss[r];
      ++c;
    }
  }
  sum[threadIdx.x] = s;
  cnt[threadIdx.x] = c;
  __syncthreads();
  for (int w = kMeanThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      sum[threadIdx.x] += sum[threadIdx.x + w];
      cnt[threadIdx.x] += cnt[threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const long long n = cnt[0];
    out[0] = n > 0 ? (float)(sum[0] / (double)n) : NAN;
    out[1] = n > 0 ? (float)(1.0 / (double)n) : NAN;
  }
}

// dlogits = (exp(x - lse) - onehot(target)) * grad_loss * inv_count; zeros for ignored rows.
template <typename T>
__global__ void __launch_bounds__(kCeThreads)
ce_bwd_kernel(const T* __restrict__ logits, RowGrid lg, const int64_t* __restrict__ targets,
              RowGrid tg, int64_t rows, int64_t vocab, int64_t ignore_index,
              const float* __restrict__ row_lse, const float* __restrict__ mean_out,
              const float* __restrict__ grad_loss, T* __restrict__ dlogits, RowGrid dg) {
  constexpr int V = Vec16<T>::N;
  const float scale = mean_out[1] * (grad_loss != nullptr ? *grad_loss : 1.0f);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* row = logits + lg.offset(r);
    T* drow = dlogits + dg.offset(r);
    const int64_t t = targets[tg.offset(r)];
    const bool skip = t == ignore_index || t < 0 || t >= vocab;
    const float nlL = -row_lse[r] * kLog2e;
    auto grad = [&](float x, int64_t c) {
      if (skip) return 0.0f;
      float p = fast_exp2(fmaf(x, kLog2e, nlL));
      if (c == t) p -= 1.0f;
      return p * scale;
    };
    // V consecutive values from column c0: softmax pairs, the target's 1 subtracted before
    // scaling (so a near-certain target keeps its precision), scaled by grad / count.
    const float2 L2 = splat2(kLog2e), nlL2 = splat2(nlL), sc2 = splat2(skip ? 0.0f : scale);
    auto grad_vec = [&](float* x, int64_t c0) {
#pragma unroll
      for (int e = 0; e < V; e += 2) {
        const float2 tt = __ffma2_rn(make_float2(x[e], x[e + 1]), L2, nlL2);
        x[e] = fast_exp2(tt.x);
        x[e + 1] = fast_exp2(tt.y);
      }
      if ((uint64_t)(t - c0) < (uint64_t)V) {
#pragma unroll
        for (int e = 0; e < V; ++e)
          if (c0 + e == t) x[e] -= 1.0f;
      }
#pragma unroll
      for (int e = 0; e < V; e += 2) {
        const float2 d = __fmul2_rn(make_float2(x[e], x[e + 1]), sc2);
        x[e] = d.x;
        x[e + 1] = d.y;
      }
    };
    const int64_t head = head_elems(row, vocab);
    const bool vec_ok = head == head_elems(drow, vocab);
    if (!vec_ok) {
      for (int64_t c = threadIdx.x; c < vocab; c += kCeThreads)
        drow[c] = from_float<T>(grad(to_float(row[c]), c));
      continue;
    }
    if (threadIdx.x < head) drow[threadIdx.x] = from_float<T>(grad(to_float(row[threadIdx.x]),
                                                                   threadIdx.x));
    const T* body = row + head;
    T* dbody = drow + head;
    const int64_t nvec = (vocab - head) / V;
    int64_t v = threadIdx.x;
    for (; v + (kCeUnrollBwd - 1) * kCeThreads < nvec; v += kCeUnrollBwd * kCeThreads) {
      uint4 raw[kCeUnrollBwd];
#pragma unroll
      for (int u = 0; u < kCeUnrollBwd; ++u) raw[u] = ld_stream(body + (v + u * kCeThreads) * V);
#pragma unroll
      for (int u = 0; u < kCeUnrollBwd; ++u) {
        float x[V];
        unpack<T>(raw[u], x);
        grad_vec(x, head + (v + u * kCeThreads) * V);
        st_stream(dbody + (v + u * kCeThreads) * V, pack<T>(x));
      }
    }
    for (; v < nvec; v += kCeThreads) {
      float x[V];
      unpack<T>(ld_stream(body + v * V), x);
      grad_vec(x, head + v * V);
      st_stream(dbody + v * V, pack<T>(x));
    }
    for (int64_t c = head + nvec * V + threadIdx.x; c < vocab; c += kCeThreads)
      drow[c] = from_float<T>(grad(to_float(row[c]), c));
  }
}

int ce_grid(int64_t rows) {
  int dev = 0, sms = 0;
  if (current_device_info(&dev, &sms)) return 0;
  const int64_t resident = (int64_t)sms * (2048 / kCeThreads);
  return (int)std::max<int64_t>(1, std::min<int64_t>(rows, resident));
}

int check_geometry(int64_t outer, int64_t inner, int64_t vocab) {
  if (outer < 0 || inner < 0)
    return set_error(PT_ERR_SHAPE, "outer and inner must be >= 0");
  if (vocab < 1 || vocab > (int64_t(1) << 31))
    return set_error(PT_ERR_SHAPE, "vocab must be in [1, 2^31] (got %lld)", (long long)vocab);
  return PT_OK;
}

}  // namespace

// Reads and clears this file's device error word (called by pt_take_device_error).
int take_ce_device_error(int* code);
int take_ce_device_error(int* code) {
  int v = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_ce_error, sizeof(int)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_ce_error, &zero, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_CUDA, "cannot read the device error word");
  }
  *code = v;
  return PT_OK;
}

}  // namespace pt

using namespace pt;

extern "C" {

int pt_cross_entropy_fwd(const void* logits, int64_t vocab, int64_t outer, int64_t inner,
                         int64_t logits_outer_stride, int64_t logits_inner_stride,
                         const int64_t* targets, int64_t targets_outer_stride,
                         int64_t targets_inner_stride, int64_t ignore_index, float* row_loss,
                         float* row_lse, float* mean_out, int dtype, void* stream) {
  if (int st = check_geometry(outer, inner, vocab)) return st;
  if (int st = check_device_ptr(mean_out, "mean_out")) return st;
  const int64_t rows = outer * inner;
  cudaStream_t s = as_stream(stream);
  const RowGrid tg{inner > 0 ? inner : 1, targets_outer_stride, targets_inner_stride};
  if (rows > 0) {
    if (int st = check_device_ptr(logits, "logits")) return st;
    if (int st = check_device_ptr(targets, "targets")) return st;
    if (int st = check_device_ptr(row_loss, "row_loss")) return st;
    if (int st = check_device_ptr(row_lse, "row_lse")) return st;
    const RowGrid lg{inner, logits_outer_stride, logits_inner_stride};
    const int grid = ce_grid(rows);
    switch (dtype) {
      case PT_FLOAT32:
        ce_fwd_kernel<float><<<grid, kCeThreads, 0, s>>>(static_cast<const float*>(logits), lg,
                                                         targets, tg, rows, vocab, ignore_index,
                                                         row_loss, row_lse);
        break;
      case PT_FLOAT16:
        ce_fwd_kernel<__half><<<grid, kCeThreads, 0, s>>>(static_cast<const __half*>(logits), lg,
                                                          targets, tg, rows, vocab,
                                                          ignore_index, row_loss, row_lse);
        break;
      case PT_BFLOAT16:
        ce_fwd_kernel<__nv_bfloat16><<<grid, kCeThreads, 0, s>>>(
            static_cast<const __nv_bfloat16*>(logits), lg, targets, tg, rows, vocab,
            ignore_index, row_loss, row_lse);
        break;
      default:
        return set_error(PT_ERR_UNSUPPORTED_DTYPE, "unsupported dtype %d", dtype);
    }
  }
  ce_mean_kernel<<<1, kMeanThreads, 0, s>>>(row_loss, targets, tg, rows, ignore_index, mean_out);
  return check_launch("pt_cross_entropy_fwd");
}

int pt_cross_entropy_bwd(const void* logits, int64_t vocab, int64_t outer, int64_t inner,
                         int64_t logits_outer_stride, int64_t logits_inner_stride,
                         const int64_t* targets, int64_t targets_outer_stride,
                         int64_t targets_inner_stride, int64_t ignore_index,
                         const float* row_lse, const float* mean_out, const float* grad_loss,
                         void* dlogits, int64_t dlogits_outer_stride,
                         int64_t dlogits_inner_stride, int dtype, void* stream) {
  if (int st = check_geometry(outer, inner, vocab)) return st;
  const int64_t rows = outer * inner;
  if (rows == 0) return ok();
  const void* ptrs[5] = {logits, targets, row_lse, mean_out, dlogits};
  const char* names[5] = {"logits", "targets", "row_lse", "mean_out", "dlogits"};
  for (int i = 0; i < 5; ++i)
    if (int st = check_device_ptr(ptrs[i], names[i])) return st;
  if (grad_loss)
    if (int st = check_device_ptr(grad_loss, "grad_loss")) return st;
  const RowGrid lg{inner, logits_outer_stride, logits_inner_stride};
  const RowGrid tg{inner, targets_outer_stride, targets_inner_stride};
  const RowGrid dg{inner, dlogits_outer_stride, dlogits_inner_stride};
  const int grid = ce_grid(rows);
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case PT_FLOAT32:
      ce_bwd_kernel<float><<<grid, kCeThreads, 0, s>>>(
          static_cast<const float*>(logits), lg, targets, tg, rows, vocab, ignore_index, row_lse,
          mean_out, grad_loss, static_cast<float*>(dlogits), dg);
      break;
    case PT_FLOAT16:
      ce_bwd_kernel<__half><<<grid, kCeThreads, 0, s>>>(
          static_cast<const __half*>(logits), lg, targets, tg, rows, vocab, ignore_index,
          row_lse, mean_out, grad_loss, static_cast<__half*>(dlogits), dg);
      break;
    case PT_BFLOAT16:
      ce_bwd_kernel<__nv_bfloat16><<<grid, kCeThreads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(logits), lg, targets, tg, rows, vocab, ignore_index,
          row_lse, mean_out, grad_loss, static_cast<__nv_bfloat16*>(dlogits), dg);
      break;
    default:
      return set_error(PT_ERR_UNSUPPORTED_DTYPE, "unsupported dtype %d", dtype);
  }
  return check_launch("pt_cross_entropy_bwd");
}

}  // extern "C"
