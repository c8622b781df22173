// 2-D transpose, dst[c, r] = src[r, c], for the weight operand of pt_swiglu_gemm_bwd (w_down
// as [k, n] becomes the [n, k] matrix whose rows both GEMM operands read along k).
//
// HBM-bound: each element read and written once. A CTA moves one 64 x 64 tile through
// shared memory: 16-byte global loads along the source rows, 16-byte global stores along the
// destination rows, the transposition itself in shared memory (rows padded by one 32-bit
// word). Tiles that cross the matrix edge, or rows that are not 16-byte aligned, take
// element-wise bounds-checked accesses.
#include "common.cuh"

namespace pt {
namespace {

constexpr int kTile = 64;
constexpr int kThreads = 256;
constexpr int kPitch = kTile + 2;  // 16-bit elements per shared row (one extra 32-bit word)

template <typename T>
__global__ void __launch_bounds__(kThreads)
transpose16_kernel(const T* __restrict__ src, int64_t sld, T* __restrict__ dst, int64_t dld,
                   int64_t rows, int64_t cols, int vec_ok) {
  static_assert(sizeof(T) == 2, "16-bit elements");
  __shared__ __align__(16) uint16_t tile[kTile * kPitch];
  const int64_t r0 = (int64_t)blockIdx.y * kTile, c0 = (int64_t)blockIdx.x * kTile;
  const bool full = vec_ok && r0 + kTile <= rows && c0 + kTile <= cols;
  const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
  uint16_t* d = reinterpret_cast<uint16_t*>(dst);
  if (full) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      const int r = idx >> 3, c8 = (idx & 7) * 8;
      const uint4 v = ld_stream(s + (r0 + r) * sld + c0 + c8);
      uint32_t* row = reinterpret_cast<uint32_t*>(tile + r * kPitch + c8);
      row[0] = v.x;
      row[1] = v.y;
      row[2] = v.z;
      row[3] = v.w;
    }
  } else {
    for (int idx = threadIdx.x; idx < kTile * kTile; idx += kThreads) {
      const int r = idx / kTile, c = idx % kTile;
      if (r0 + r < rows && c0 + c < cols) tile[r * kPitch + c] = s[(r0 + r) * sld + c0 + c];
    }
  }
  __syncthreads();
  if (full) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      const int c = idx >> 3, r8 = (idx & 7) * 8;
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        w[e] = (uint32_t)tile[(r8 + 2 * e) * kPitch + c] |
               ((uint32_t)tile[(r8 + 2 * e + 1) * kPitch + c] << 16);
      st_stream(d + (c0 + c) * dld + r0 + r8, make_uint4(w[0], w[1], w[2], w[3]));
    }
  } else {
    for (int idx = threadIdx.x; idx < kTile * kTile; idx += kThreads) {
      const int c = idx / kTile, r = idx % kTile;
      if (r0 + r < rows && c0 + c < cols) d[(c0 + c) * dld + r0 + r] = tile[r * kPitch + c];
    }
  }
}

__global__ void __launch_bounds__(kThreads)
transpose32_kernel(const float* __restrict__ src, int64_t sld, float* __restrict__ dst,
                   int64_t dld, int64_t rows, int64_t cols) {
  __shared__ float tile[kTile][kTile + 1];
  const int64_t r0 = (int64_t)blockIdx.y * kTile, c0 = (int64_t)blockIdx.x * kTile;
  for (int idx = threadIdx.x; idx < kTile * kTile; idx += kThreads) {
    const int r = idx / kTile, c = idx % kTile;
    if (r0 + r < rows && c0 + c < cols) tile[r][c] = src[(r0 + r) * sld + c0 + c];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kTile * kTile; idx += kThreads) {
    const int c = idx / kTile, r = idx % kTile;
    if (r0 + r < rows && c0 + c < cols) dst[(c0 + c) * dld + r0 + r] = tile[r][c];
  }
}

}  // namespace
}  // namespace pt

using namespace pt;

extern "C" {

int pt_transpose_2d(const void* src, int64_t src_row_stride, void* dst, int64_t dst_row_stride,
                    int64_t rows, int64_t cols, int dtype, void* stream) {
  if (rows < 0 || cols < 0)
    return set_error(PT_ERR_SHAPE, "rows and cols must be >= 0 (got %lld, %lld)",
                     (long long)rows, (long long)cols);
  if (rows == 0 || cols == 0) return ok();
  if (src_row_stride < cols || dst_row_stride < rows)
    return set_error(PT_ERR_SHAPE, "a row stride is smaller than its row");
  if ((rows + kTile - 1) / kTile > 65535)
    return set_error(PT_ERR_SHAPE, "rows must be below %d", 65535 * kTile);
  if (int st = check_device_ptr(src, "src")) return st;
  if (int st = check_device_ptr(dst, "dst")) return st;
  if (src == dst) return set_error(PT_ERR_INVALID_ARGUMENT, "dst must not alias src");
  const dim3 grid((unsigned)((cols + kTile - 1) / kTile), (unsigned)((rows + kTile - 1) / kTile));
  cudaStream_t s = as_stream(stream);
  const int vec_ok = aligned16(src) && aligned16(dst) && src_row_stride % 8 == 0 &&
                     dst_row_stride % 8 == 0;
  switch (dtype) {
    case PT_BFLOAT16:
      transpose16_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(src), src_row_stride,
          static_cast<__nv_bfloat16*>(dst), dst_row_stride, rows, cols, vec_ok);
      break;
    case PT_FLOAT16:
      transpose16_kernel<__half><<<grid, kThreads, 0, s>>>(
          static_cast<const __half*>(src), src_row_stride, static_cast<__half*>(dst),
          dst_row_stride, rows, cols, vec_ok);
      break;
    case PT_FLOAT32:
      transpose32_kernel<<<grid, kThreads, 0, s>>>(static_cast<const float*>(src),
                                                   src_row_stride, static_cast<float*>(dst),
                                                   dst_row_stride, rows, cols);
      break;
    default:
      return set_error(PT_ERR_UNSUPPORTED_DTYPE, "unsupported dtype %d", dtype);
  }
  return check_launch("pt_transpose_2d");
}

}  // extern "C"
