// Shared device and host helpers for the picotron B200 kernels (sm_100a only).
//
// Device side: element-type traits, 16-byte vector loads/stores with explicit cache
// hints, bf16/fp16 <-> fp32 conversion of packed vectors, warp reductions.
// Host side: status/error plumbing for the C ABI (pt_last_error is thread-local),
// pointer validation, and a write-once per-device cache of the SM count.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/picotron_b200.h"

namespace pt {

// ------------------------------------------------------------------ element types --

template <typename T> struct ElemTraits;
template <> struct ElemTraits<float> {
  static constexpr int kDtype = PT_FLOAT32;
};
template <> struct ElemTraits<__half> {
  static constexpr int kDtype = PT_FLOAT16;
};
template <> struct ElemTraits<__nv_bfloat16> {
  static constexpr int kDtype = PT_BFLOAT16;
};

__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) {
  return __float2half_rn(v);
}
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// Number of T elements in one 16-byte vector.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
};

// ------------------------------------------------------------- 16-byte memory ops --
// Loads of inputs that are never written by the same kernel use the non-coherent path
// without L1 allocation: every byte is used once per kernel, so L1 residency only
// evicts the rows that are still being reduced.

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

// Plain cached 16-byte load (weights, tables: reused by every row).
__device__ __forceinline__ uint4 ld_cached(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// 8-byte cached load (half of a 16-byte vector of a 16-bit table).
__device__ __forceinline__ uint2 ld_cached8(const void* p) {
  return __ldg(reinterpret_cast<const uint2*>(p));
}

// Streaming store (evict-first): outputs are consumed by a later kernel, not this one.
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};"
               :
               : "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// 32-byte streaming load / store (two 16-byte vectors in one instruction, sm_100); p must be
// 32-byte aligned.
struct Vec32B {
  uint4 lo, hi;
};
__device__ __forceinline__ Vec32B ld_stream32(const void* p) {
  Vec32B r;
  asm("ld.global.nc.L1::no_allocate.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r.lo.x), "=r"(r.lo.y), "=r"(r.lo.z), "=r"(r.lo.w), "=r"(r.hi.x), "=r"(r.hi.y),
        "=r"(r.hi.z), "=r"(r.hi.w)
      : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream32(void* p, const uint4& lo, const uint4& hi) {
  asm volatile("st.global.cs.v8.u32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
               :
               : "l"(p), "r"(lo.x), "r"(lo.y), "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y),
                 "r"(hi.z), "r"(hi.w)
               : "memory");
}

// 32-byte loads of eight floats (sm_100); p must be 32-byte aligned. The _cs form streams
// (evict-first) data read once.
__device__ __forceinline__ void ld_global_v8(const float* p, float (&v)[8]) {
  asm volatile("ld.global.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]),
                 "=f"(v[6]), "=f"(v[7])
               : "l"(p)
               : "memory");
}
__device__ __forceinline__ void ld_global_cs_v8(const float* p, float (&v)[8]) {
  asm volatile("ld.global.cs.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]),
                 "=f"(v[6]), "=f"(v[7])
               : "l"(p)
               : "memory");
}

// One 32-byte store of eight floats (sm_100: a whole L2 sector per thread); p must be 32-byte
// aligned.
__device__ __forceinline__ void st_global_v8(float* p, const float (&v)[8]) {
  asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
               :
               : "l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]),
                 "f"(v[6]), "f"(v[7])
               : "memory");
}

// Unpack a 16-byte vector of T into fp32 values.
template <typename T> __device__ __forceinline__ void unpack(const uint4& v, float* f);

template <> __device__ __forceinline__ void unpack<float>(const uint4& v, float* f) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}

template <> __device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bf16 -> fp32 is exact: the bf16 bits are the high half of the fp32 bits.
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

template <> __device__ __forceinline__ void unpack<__half>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Unpack a 16-byte vector of T into V/2 fp32 pairs (element 2i in .x, 2i+1 in .y).
template <typename T> __device__ __forceinline__ void unpack2(const uint4& v, float2* f) {
  float t[Vec16<T>::N];
  unpack<T>(v, t);
#pragma unroll
  for (int i = 0; i < Vec16<T>::N / 2; ++i) f[i] = make_float2(t[2 * i], t[2 * i + 1]);
}

__device__ __forceinline__ float2 splat2(float a) { return make_float2(a, a); }

// Division of 32-bit unsigned values by a runtime divisor d >= 1 with a multiply-high and
// shifts (Granlund and Montgomery, "Division by invariant integers using multiplication",
// 1994, the round-up method): with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1,
// n / d = (t + ((n - t) >> 1)) >> (l - 1) where t = mulhi(n, m), exact for every 32-bit n.
struct FastDiv {
  uint32_t d = 1, m = 0, l = 0;
  FastDiv() = default;
  __host__ explicit FastDiv(uint32_t divisor) : d(divisor) {
    if (d > 1) {
      l = 32u - (uint32_t)__builtin_clz(d - 1);
      m = (uint32_t)((((uint64_t)1 << 32) * (((uint64_t)1 << l) - d)) / d + 1);
    }
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    if (d == 1) return n;
    const uint32_t t = __umulhi(n, m);
    return (t + ((n - t) >> 1)) >> (l - 1);
  }
};

// Round both lanes to T (nearest even) and widen back: the value a T store would keep.
template <typename T> __device__ __forceinline__ float2 round2(float2 v);
template <> __device__ __forceinline__ float2 round2<float>(float2 v) { return v; }
template <> __device__ __forceinline__ float2 round2<__nv_bfloat16>(float2 v) {
  return __bfloat1622float2(__float22bfloat162_rn(v));
}
template <> __device__ __forceinline__ float2 round2<__half>(float2 v) {
  return __half22float2(__float22half2_rn(v));
}

// Pack fp32 values into a 16-byte vector of T with round-to-nearest-even.
template <typename T> __device__ __forceinline__ uint4 pack(const float* f);

template <> __device__ __forceinline__ uint4 pack<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}

template <> __device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <> __device__ __forceinline__ uint4 pack<__half>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Load `n` consecutive elements of TW starting at p as fp32 (n is a compile-time
// multiple of the TW vector width; p is 16-byte aligned).
template <typename TW, int N>
__device__ __forceinline__ void load_row_f32(const TW* p, float* f) {
  constexpr int V = Vec16<TW>::N;
  static_assert(N % V == 0, "N must be a multiple of the vector width");
#pragma unroll
  for (int i = 0; i < N / V; ++i) unpack<TW>(ld_cached(p + i * V), f + i * V);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// r = 1 / sqrt(m) to about 1e-14 relative: fp32 hardware estimate refined by one
// Newton step in fp64 (r1 = r0 * (1.5 - 0.5 * m * r0^2); the error squares).
__device__ __forceinline__ double rsqrt_refined(double m) {
  const double r0 = (double)rsqrtf((float)m);
  return r0 * (1.5 - 0.5 * m * r0 * r0);
}

// Ring position of a row in a `stages`-slot pipeline, advanced without division.
struct RingPos {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void advance(int n, int stages) {
    slot += n;
    while (slot >= stages) {
      slot -= stages;
      phase ^= 1u;
    }
  }
};

// Doubly compensated summation ("Sum2": Knuth's TwoSum error-free transformation with the
// errors gathered in a second accumulator). Each addition sum + t is split exactly into its
// rounded value s and its rounding error e, whatever the magnitudes of sum and t; the errors
// are summed in err, whose own rounding is second order. sum + err therefore carries the
// exact sum to about twice fp32 precision however many terms are added and however much they
// cancel (plain Kahan summation, by contrast, still loses up to one ulp of every term). The
// _rn intrinsics keep the compiler from reassociating or contracting the error terms.
__device__ __forceinline__ void sum2_add(float& sum, float& err, float t) {
  const float s = __fadd_rn(sum, t);
  const float z = __fsub_rn(s, sum);
  const float e = __fadd_rn(__fsub_rn(sum, __fsub_rn(s, z)), __fsub_rn(t, z));
  err = __fadd_rn(err, e);
  sum = s;
}

// ----------------------------------------------------- TMA bulk copies + mbarriers --
// 1-D bulk copies (cp.async.bulk, no tensor map, no multicast) from global memory into
// this CTA's shared memory, completing on an mbarrier with a transaction count.

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Plain arrival (release semantics at CTA scope: prior writes of this thread are
// visible to threads that observe the phase completion).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// dst (shared) and src (global) 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 1-D bulk copy of `bytes` from this CTA's shared memory to global memory (both addresses
// 16-byte aligned, bytes a multiple of 16), tracked by this thread's bulk-group counter.
__device__ __forceinline__ void bulk_store_row(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until this thread's committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_all_read() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Waits until this thread's committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait_all_done() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Orders this thread's earlier generic-proxy shared-memory writes before later async-proxy
// (bulk copy) accesses to them.
__device__ __forceinline__ void fence_async_proxy_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Potentially blocking test of phase `parity`: the thread may sleep until the phase
// completes or about kSuspendHintNs nanoseconds pass (0: the hardware's default limit).
#ifndef PT_SUSPEND_NS
#define PT_SUSPEND_NS 0
#endif
constexpr uint32_t kSuspendHintNs = PT_SUSPEND_NS;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  if constexpr (kSuspendHintNs > 0) {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
  } else {
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
  }
  return done != 0;
}

// Waits for phase `parity` of `bar` to complete, giving up after about one second of SM
// clock (kWaitLimitCycles); returns false on timeout. Every wait in this library is
// bounded so that a lost copy can never hang the GPU.
constexpr long long kWaitLimitCycles = 2000000000LL;
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit = kWaitLimitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}

// 16-byte shared-memory load.
__device__ __forceinline__ uint4 lds128(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// Device-side error codes reported through pt_take_device_error().
constexpr int kDeviceErrWaitTimeout = 1;

// fp32 logistic function, sigma(g) = 1 / (1 + e^-g), with the CUDA fast exponential and the
// fast division intrinsic (a reciprocal on the special-function unit and a multiply instead
// of the IEEE division sequence); both relative errors are a few fp32 ulp, far below the
// tolerances of this library. For g << 0 the exponential overflows to +inf and the quotient
// is 0 (also for 1 + e^-g above 2^126, where the true value is below 1e-38).
__device__ __forceinline__ float sigmoid_f32(float g) {
  return __fdividef(1.0f, 1.0f + __expf(-g));
}

// ----------------------------------------------------------------------- host side --

// Records `msg` as this thread's last error and returns `status`.
int set_error(int status, const char* fmt, ...);
// Clears this thread's last error and returns PT_OK.
int ok();

// Checks that `p` is device or managed memory of the current device.
int check_device_ptr(const void* p, const char* name);

// Current device and its SM count (cached per device, written once).
int current_device_info(int* device, int* sm_count);

// Maps the result of a kernel launch to a status.
int check_launch(const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int dtype_size(int dtype) {
  switch (dtype) {
    case PT_FLOAT32: return 4;
    case PT_FLOAT16: return 2;
    case PT_BFLOAT16: return 2;
    default: return 0;
  }
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace pt
