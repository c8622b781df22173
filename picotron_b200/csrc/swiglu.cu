// SwiGLU activation forward/backward for sm_100a.
//
// Math follows src/picotron/nn/triton_kernels/swiglu.py of the reference:
//   forward  (:26-41)  out = (g * sigmoid(g)) * u, fp32 math, one rounding
//   backward (:71-81)  s = sigmoid(g); dg = dout * u * (s * (1 + g * (1 - s)));
//                      du = dout * (g * s)
// The reference backward runs in the input dtype op by op; here it runs in fp32 with
// sigmoid recomputed from g and one rounding per output.
//
// Layout: flat contiguous arrays of n elements. Each thread owns U 32-byte vectors (arrays
// that are 32-byte aligned) or U 16-byte vectors (16-byte aligned) per grid-stride iteration
// (the U vectors of a thread are blockDim apart so a warp's accesses stay contiguous); all
// loads of an iteration are issued before any math. Elements past the last whole vector and
// misaligned arrays take a scalar path.
#include "common.cuh"

namespace pt {
namespace {

// Launch shapes of the vector paths, from A/B runs on B200 at 16384 x 14336 bf16 over the
// other shapes of 256-1024 threads and 1-8 vectors per thread: forward 512 threads x 2
// vectors (0.97-1.00 of the measured copy bandwidth, against 0.90-0.95 for 256 x 4),
// backward 512 threads x 4 vectors per array (1.00, against 0.90-0.95 for 512 x 2).
constexpr int kThreads = 256;     // scalar paths
constexpr int kThreadsFwd = 512;
constexpr int kThreadsBwd = 512;
constexpr int kUnrollFwd = 2;
constexpr int kUnrollBwd = 4;
constexpr int kUnrollFwd32 = 2;  // 32-byte vectors per thread and array
constexpr int kUnrollBwd32 = 2;

template <typename T, int U>
__global__ void __launch_bounds__(kThreadsFwd)
swiglu_fwd_vec(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out,
               int64_t nvec) {
  constexpr int V = Vec16<T>::N;
  const int64_t step = (int64_t)gridDim.x * blockDim.x * U;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x * U + threadIdx.x; i0 < nvec; i0 += step) {
    uint4 gv[U], uv[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec) {
        gv[k] = ld_stream(g + i * V);
        uv[k] = ld_stream(u + i * V);
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec) {
        float fg[V], fu[V];
        unpack<T>(gv[k], fg);
        unpack<T>(uv[k], fu);
#pragma unroll
        for (int j = 0; j < V; ++j) fg[j] = (fg[j] * sigmoid_f32(fg[j])) * fu[j];
        st_stream(out + i * V, pack<T>(fg));
      }
    }
  }
}

template <typename T, int U>
__global__ void __launch_bounds__(kThreadsBwd)
swiglu_bwd_vec(const T* __restrict__ dout, const T* __restrict__ g, const T* __restrict__ u,
               T* __restrict__ dg, T* __restrict__ du, int64_t nvec) {
  constexpr int V = Vec16<T>::N;
  const int64_t step = (int64_t)gridDim.x * blockDim.x * U;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x * U + threadIdx.x; i0 < nvec; i0 += step) {
    uint4 ov[U], gv[U], uv[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec) {
        ov[k] = ld_stream(dout + i * V);
        gv[k] = ld_stream(g + i * V);
        uv[k] = ld_stream(u + i * V);
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec) {
        float fo[V], fg[V], fu[V];
        unpack<T>(ov[k], fo);
        unpack<T>(gv[k], fg);
        unpack<T>(uv[k], fu);
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const float s = sigmoid_f32(fg[j]);
          const float dsilu = s * (1.0f + fg[j] * (1.0f - s));
          const float d_up = fo[j] * (fg[j] * s);
          fg[j] = (fo[j] * fu[j]) * dsilu;
          fu[j] = d_up;
        }
        st_stream(dg + i * V, pack<T>(fg));
        st_stream(du + i * V, pack<T>(fu));
      }
    }
  }
}

// The forward and backward on 32-byte vectors (two 16-byte vectors per load and store
// instruction): the paths for 32-byte aligned arrays. A/B of builds on B200 at config 3 inside
// the config-5 step, where each SwiGLU kernel follows RMSNorm kernels: the 32-byte loads make
// the backward 5 % faster there (361 against 379 us per launch; 32-byte stores alone changed
// nothing) and the step 2 % shorter (27.01 against 27.64 ms, same box), while back to back on
// their own both kernels are within 1-3 % of the 16-byte ones (slower, in that setting).
template <typename T, int U>
__global__ void __launch_bounds__(kThreadsFwd)
swiglu_fwd_vec32(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out,
                 int64_t nvec32) {
  constexpr int V = Vec16<T>::N;  // elements per 16-byte half
  const int64_t step = (int64_t)gridDim.x * blockDim.x * U;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x * U + threadIdx.x; i0 < nvec32;
       i0 += step) {
    Vec32B gv[U], uv[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec32) {
        gv[k] = ld_stream32(g + i * 2 * V);
        uv[k] = ld_stream32(u + i * 2 * V);
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec32) {
        uint4 r[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float fg[V], fu[V];
          unpack<T>(h ? gv[k].hi : gv[k].lo, fg);
          unpack<T>(h ? uv[k].hi : uv[k].lo, fu);
#pragma unroll
          for (int j = 0; j < V; ++j) fg[j] = (fg[j] * sigmoid_f32(fg[j])) * fu[j];
          r[h] = pack<T>(fg);
        }
        st_stream32(out + i * 2 * V, r[0], r[1]);
      }
    }
  }
}

template <typename T, int U>
__global__ void __launch_bounds__(kThreadsBwd)
swiglu_bwd_vec32(const T* __restrict__ dout, const T* __restrict__ g, const T* __restrict__ u,
                 T* __restrict__ dg, T* __restrict__ du, int64_t nvec32) {
  constexpr int V = Vec16<T>::N;  // elements per 16-byte half
  const int64_t step = (int64_t)gridDim.x * blockDim.x * U;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x * U + threadIdx.x; i0 < nvec32;
       i0 += step) {
    Vec32B ov[U], gv[U], uv[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec32) {
        ov[k] = ld_stream32(dout + i * 2 * V);
        gv[k] = ld_stream32(g + i * 2 * V);
        uv[k] = ld_stream32(u + i * 2 * V);
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int64_t i = i0 + (int64_t)k * blockDim.x;
      if (i < nvec32) {
        uint4 rg[2], ru[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float fo[V], fg[V], fu[V];
          unpack<T>(h ? ov[k].hi : ov[k].lo, fo);
          unpack<T>(h ? gv[k].hi : gv[k].lo, fg);
          unpack<T>(h ? uv[k].hi : uv[k].lo, fu);
#pragma unroll
          for (int j = 0; j < V; ++j) {
            const float s = sigmoid_f32(fg[j]);
            const float dsilu = s * (1.0f + fg[j] * (1.0f - s));
            const float d_up = fo[j] * (fg[j] * s);
            fg[j] = (fo[j] * fu[j]) * dsilu;
            fu[j] = d_up;
          }
          rg[h] = pack<T>(fg);
          ru[h] = pack<T>(fu);
        }
        st_stream32(dg + i * 2 * V, rg[0], rg[1]);
        st_stream32(du + i * 2 * V, ru[0], ru[1]);
      }
    }
  }
}

// Scalar path for [begin, n): the tail after the last whole vector, or whole arrays
// whose pointers are not 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(kThreads)
swiglu_fwd_scalar(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out,
                  int64_t begin, int64_t n) {
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float fg = to_float(g[i]);
    out[i] = from_float<T>((fg * sigmoid_f32(fg)) * to_float(u[i]));
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
swiglu_bwd_scalar(const T* __restrict__ dout, const T* __restrict__ g, const T* __restrict__ u,
                  T* __restrict__ dg, T* __restrict__ du, int64_t begin, int64_t n) {
  for (int64_t i = begin + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float fo = to_float(dout[i]), fg = to_float(g[i]), fu = to_float(u[i]);
    const float s = sigmoid_f32(fg);
    dg[i] = from_float<T>((fo * fu) * (s * (1.0f + fg * (1.0f - s))));
    du[i] = from_float<T>(fo * (fg * s));
  }
}

bool aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31) == 0; }

int grid_for(int64_t work_items, int sms, int per_sm, int threads = kThreads) {
  const int64_t blocks = (work_items + threads - 1) / threads;
  const int64_t cap = (int64_t)sms * per_sm;
  int64_t gsz = blocks < cap ? blocks : cap;
  return (int)(gsz < 1 ? 1 : gsz);
}

template <typename T>
int fwd_impl(const void* g_, const void* u_, void* out_, int64_t n, cudaStream_t s) {
  const T* g = static_cast<const T*>(g_);
  const T* u = static_cast<const T*>(u_);
  T* out = static_cast<T*>(out_);
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  constexpr int V = Vec16<T>::N;
  const bool vec = aligned16(g) && aligned16(u) && aligned16(out);
  const bool vec32 = aligned32(g) && aligned32(u) && aligned32(out);
  int64_t done = 0;
  if (vec32) {
    const int64_t nvec32 = n / (2 * V);
    if (nvec32 > 0) {
      const int grid = grid_for((nvec32 + kUnrollFwd32 - 1) / kUnrollFwd32, sms,
                                2048 / kThreadsFwd, kThreadsFwd);
      swiglu_fwd_vec32<T, kUnrollFwd32><<<grid, kThreadsFwd, 0, s>>>(g, u, out, nvec32);
    }
    done = nvec32 * 2 * V;
  } else if (vec) {
    const int64_t nvec = n / V;
    if (nvec > 0) {
      const int grid = grid_for((nvec + kUnrollFwd - 1) / kUnrollFwd, sms, 2048 / kThreadsFwd,
                                kThreadsFwd);
      swiglu_fwd_vec<T, kUnrollFwd><<<grid, kThreadsFwd, 0, s>>>(g, u, out, nvec);
    }
    done = nvec * V;
  }
  if (done < n)
    swiglu_fwd_scalar<T><<<grid_for(n - done, sms, 8), kThreads, 0, s>>>(g, u, out, done, n);
  return check_launch("pt_swiglu_fwd");
}

template <typename T>
int bwd_impl(const void* o_, const void* g_, const void* u_, void* dg_, void* du_, int64_t n,
             cudaStream_t s) {
  const T* o = static_cast<const T*>(o_);
  const T* g = static_cast<const T*>(g_);
  const T* u = static_cast<const T*>(u_);
  T* dg = static_cast<T*>(dg_);
  T* du = static_cast<T*>(du_);
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  constexpr int V = Vec16<T>::N;
  const bool vec = aligned16(o) && aligned16(g) && aligned16(u) && aligned16(dg) && aligned16(du);
  const bool vec32 = aligned32(o) && aligned32(g) && aligned32(u) && aligned32(dg) &&
                     aligned32(du);
  int64_t done = 0;
  if (vec32) {
    const int64_t nvec32 = n / (2 * V);
    if (nvec32 > 0) {
      const int grid = grid_for((nvec32 + kUnrollBwd32 - 1) / kUnrollBwd32, sms,
                                2048 / kThreadsBwd, kThreadsBwd);
      swiglu_bwd_vec32<T, kUnrollBwd32><<<grid, kThreadsBwd, 0, s>>>(o, g, u, dg, du, nvec32);
    }
    done = nvec32 * 2 * V;
  } else if (vec) {
    const int64_t nvec = n / V;
    if (nvec > 0) {
      const int grid = grid_for((nvec + kUnrollBwd - 1) / kUnrollBwd, sms, 2048 / kThreadsBwd,
                                kThreadsBwd);
      swiglu_bwd_vec<T, kUnrollBwd><<<grid, kThreadsBwd, 0, s>>>(o, g, u, dg, du, nvec);
    }
    done = nvec * V;
  }
  if (done < n)
    swiglu_bwd_scalar<T><<<grid_for(n - done, sms, 8), kThreads, 0, s>>>(o, g, u, dg, du, done, n);
  return check_launch("pt_swiglu_bwd");
}

}  // namespace
}  // namespace pt

using namespace pt;

extern "C" {

int pt_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, int dtype,
                  void* stream) {
  if (n < 0) return set_error(PT_ERR_SHAPE, "n must be >= 0 (got %lld)", (long long)n);
  if (dtype_size(dtype) == 0) return set_error(PT_ERR_UNSUPPORTED_DTYPE, "unsupported dtype %d", dtype);
  if (n == 0) return ok();
  if (int st = check_device_ptr(gate, "gate")) return st;
  if (int st = check_device_ptr(up, "up")) return st;
  if (int st = check_device_ptr(out, "out")) return st;
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case PT_FLOAT32: return fwd_impl<float>(gate, up, out, n, s);
    case PT_FLOAT16: return fwd_impl<__half>(gate, up, out, n, s);
    default: return fwd_impl<__nv_bfloat16>(gate, up, out, n, s);
  }
}

int pt_swiglu_bwd(const void* dout, const void* gate, const void* up, void* dgate, void* dup,
                  int64_t n, int dtype, void* stream) {
  if (n < 0) return set_error(PT_ERR_SHAPE, "n must be >= 0 (got %lld)", (long long)n);
  if (dtype_size(dtype) == 0) return set_error(PT_ERR_UNSUPPORTED_DTYPE, "unsupported dtype %d", dtype);
  if (n == 0) return ok();
  if (int st = check_device_ptr(dout, "dout")) return st;
  if (int st = check_device_ptr(gate, "gate")) return st;
  if (int st = check_device_ptr(up, "up")) return st;
  if (int st = check_device_ptr(dgate, "dgate")) return st;
  if (int st = check_device_ptr(dup, "dup")) return st;
  cudaStream_t s = as_stream(stream);
  switch (dtype) {
    case PT_FLOAT32: return bwd_impl<float>(dout, gate, up, dgate, dup, n, s);
    case PT_FLOAT16: return bwd_impl<__half>(dout, gate, up, dgate, dup, n, s);
    default: return bwd_impl<__nv_bfloat16>(dout, gate, up, dgate, dup, n, s);
  }
}

}  // extern "C"
