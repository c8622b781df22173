// Fused SwiGLU MLP up-projection on the 5th-generation tensor cores (sm_100a):
//
//   gate = x @ w_gate^T,  up = x @ w_up^T   (fp32 accumulation in tensor memory)
//   act  = silu(gate) * up                   (epilogue, fp32 math on the bf16-rounded gate/up)
//
// x [m, k], w_gate / w_up [n, k] (nn.Linear layout), all row-major with unit column stride;
// act [m, n] and, optionally, gate and up [m, n] (what the backward needs) in the same dtype.
// Replaces the three steps of picotron's SwiGLU.forward (src/picotron/nn/feedforward.py:
// 27-43: gate_projection, up_projection, then the activation at :29-42) up to the
// down_projection: the activation reads the accumulators straight from tensor memory, so the
// gate/up tensors are never re-read from HBM.
//
// One persistent CTA per SM walks 128 x 128 output tiles. Per tile and per 64-wide K block,
// one TMA producer thread loads the x tile [128 x 64] and the gate and up weight tiles
// [128 x 64] each (128-byte swizzle) into a 4-stage shared-memory ring; one MMA thread issues
// tcgen05.mma (kind::f16, M = 128, N = 256: the gate rows and the up rows of the B tile side
// by side, so one instruction produces both accumulators) into one of two 256-column tensor
// memory buffers; four epilogue warps read the finished buffer with tcgen05.ld while the next
// tile accumulates into the other. Barriers are mbarriers with bounded waits: a wait that
// runs out records an error word (pt_take_device_error) and the kernel drains its copies and
// MMAs, frees its tensor memory and returns. No cluster launch and no multicast of any kind.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"

namespace pt {

__device__ int g_gemm_error = 0;

namespace {

constexpr int kBM = 128;             // tile rows = tensor-memory lanes
constexpr int kBN = 128;             // output columns per tile (gate and up each)
constexpr int kBK = 64;              // K per stage: one 128-byte swizzle row of 16-bit values
constexpr int kUmmaK = 16;           // K of one tcgen05.mma for 16-bit inputs
constexpr int kStages = 4;
constexpr int kATileBytes = kBM * kBK * 2;          // 16 KB
constexpr int kBTileBytes = 2 * kBN * kBK * 2;      // 32 KB: gate rows, then up rows
constexpr int kStageBytes = kATileBytes + kBTileBytes;
constexpr int kAccCols = 2 * kBN;    // fp32 columns of one accumulator buffer (gate | up)
constexpr int kTmemCols = 2 * kAccCols;  // double-buffered: 512 columns (all of them)
constexpr int kThreads = 256;        // warp 0 TMA, 1 MMA, 2 TMEM owner, 3 idle, 4-7 epilogue
constexpr int kEpiWarp0 = 4;
constexpr int kGroupM = 16;          // m-tiles per raster group (L2 reuse of the weights)
constexpr long long kWaitCycles = 2000000000LL;  // about one second of SM clock

struct GemmBarriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
};

constexpr int kSmemBytes = 1024 /* alignment slack */ + kStages * kStageBytes +
                           (int)((sizeof(GemmBarriers) + 15) / 16 * 16);

__device__ __forceinline__ void record_gemm_error() {
  atomicExch(&g_gemm_error, kDeviceErrWaitTimeout);
}

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

// 2-D tiled TMA load (no multicast) of box {kBK, rows} at (x = column, y = row) into smem,
// completing on `bar` with the box's byte count.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      :
      : "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored as TMA wrote it with
// 128-byte swizzle: rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked densely.
// Fields (sm_100 layout): start address >> 4 in [0,14), leading byte offset >> 4 in [16,30)
// (1: unused for swizzled K-major), stride byte offset >> 4 in [32,46) (1024 bytes between
// 8-row groups), descriptor version 1 in [46,48), layout type in [61,64) (2 = 128B swizzle).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr & 0x3FFFFu) >> 4) | (uint64_t)1 << 16 | (uint64_t)(1024 >> 4) << 32 |
         (uint64_t)1 << 46 | (uint64_t)2 << 61;
}

// Instruction descriptor for kind::f16: fp32 accumulator (bits [4,6) = 1), A and B format
// (bits [7,10) and [10,13): 0 = f16, 1 = bf16), both K-major (bits 15, 16 = 0),
// N >> 3 in [17,23), M >> 4 in [24,29).
template <typename T> constexpr uint32_t instr_desc(int m, int n) {
  constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      :
      : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :
               : "r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive fp32 columns of this warp's 32 tensor-memory lanes (one lane per thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
      " [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// Ties 32 registers written by tmem_ld32 to a point after tmem_wait_ld, so the compiler
// cannot move their first use above the wait (the asm statements stay in order).
__device__ __forceinline__ void reg_fence32(uint32_t* r) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
                 "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]),
                 "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

struct TileGrid {
  int tiles_m, tiles_n;
  __device__ __forceinline__ int count() const { return tiles_m * tiles_n; }
  // Grouped raster: kGroupM m-tiles walk all n-tiles together, so a wave of CTAs shares a
  // few weight tiles and a few x tiles through L2.
  __device__ __forceinline__ void coords(int t, int& mb, int& nb) const {
    const int per_group = kGroupM * tiles_n;
    const int group = t / per_group;
    const int first = group * kGroupM;
    const int gsz = min(tiles_m - first, kGroupM);
    const int local = t - group * per_group;
    mb = first + local % gsz;
    nb = local / gsz;
  }
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
swiglu_gemm_kernel(const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ CUtensorMap map_wg,
                   const __grid_constant__ CUtensorMap map_wu, T* __restrict__ act,
                   int64_t act_stride, T* __restrict__ gate_out, T* __restrict__ up_out,
                   int64_t pre_stride, int m, int n, int k) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
  unsigned char* tiles = smem_raw + pad;
  GemmBarriers* bars = reinterpret_cast<GemmBarriers*>(tiles + kStages * kStageBytes);
  const uint32_t tiles_addr = raw + pad;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const TileGrid grid{(m + kBM - 1) / kBM, (n + kBN - 1) / kBN};
  const int kblocks = (k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], kThreads / 32 - kEpiWarp0);
    }
    mbar_init(&bars->drain, 1);
    fence_mbar_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :
                 : "r"(smem_addr(&bars->tmem_base)), "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer --
    if (lane == 0) {
      RingPos pos;
      uint32_t issued_mask = 0, issued_phase = 0;  // per slot: ever issued, parity of last
      bool ok = true;
      for (int t = blockIdx.x; ok && t < grid.count(); t += gridDim.x) {
        int mb, nb;
        grid.coords(t, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(&bars->empty[pos.slot], pos.phase ^ 1u)) {
            ok = false;
            break;
          }
          uint64_t* full = &bars->full[pos.slot];
          mbar_arrive_expect_tx(full, kStageBytes);
          const uint32_t sa = tiles_addr + pos.slot * kStageBytes;
          tma_load_2d(sa, &map_x, kb * kBK, mb * kBM, full);
          tma_load_2d(sa + kATileBytes, &map_wg, kb * kBK, nb * kBN, full);
          tma_load_2d(sa + kATileBytes + kBTileBytes / 2, &map_wu, kb * kBK, nb * kBN, full);
          issued_mask |= 1u << pos.slot;
          issued_phase = (issued_phase & ~(1u << pos.slot)) | (pos.phase << pos.slot);
          pos.advance(1, kStages);
        }
      }
      if (!ok) record_gemm_error();
      // Every copy this CTA issued must have landed before it may exit.
      for (int s = 0; s < kStages; ++s)
        if (issued_mask >> s & 1u) wait_bounded(&bars->full[s], issued_phase >> s & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc<T>(kBM, 2 * kBN);
      RingPos pos;
      bool ok = true;
      int i = 0;
      for (int t = blockIdx.x; ok && t < grid.count(); t += gridDim.x, ++i) {
        const int b = i & 1;
        if (!wait_bounded(&bars->tmem_empty[b], ((i >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(b * kAccCols);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(&bars->full[pos.slot], pos.phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = tiles_addr + pos.slot * kStageBytes;
          const uint64_t adesc = smem_desc_sw128(sa);
          const uint64_t bdesc = smem_desc_sw128(sa + kATileBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            // Advancing the start address by 32 bytes selects the next 16 K-elements inside
            // the swizzled 128-byte rows (the swizzle is a function of the address bits).
            const uint64_t step = (uint64_t)((kk * kUmmaK * 2) >> 4);
            umma_f16(d, adesc + step, bdesc + step, idesc, (kb | kk) != 0);
          }
          umma_commit(&bars->empty[pos.slot]);  // frees the stage once these MMAs finish
          pos.advance(1, kStages);
        }
        if (!ok) break;
        umma_commit(&bars->tmem_full[b]);
      }
      if (!ok) record_gemm_error();
      // All MMAs this thread issued must be complete before the tensor memory is freed.
      umma_commit(&bars->drain);
      wait_bounded(&bars->drain, 0);
    }
    __syncwarp();
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- epilogue --
    const int q = warp & 3;  // this warp may read tensor-memory lanes [32q, 32q + 32)
    int i = 0;
    for (int t = blockIdx.x; t < grid.count(); t += gridDim.x, ++i) {
      const int b = i & 1;
      if (!wait_bounded(&bars->tmem_full[b], (i >> 1) & 1)) {
        record_gemm_error();
        break;
      }
      tc_fence_after();
      int mb, nb;
      grid.coords(t, mb, nb);
      const int row = mb * kBM + q * 32 + lane;
      const uint32_t tg = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kAccCols);
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t gr[32], ur[32];
        tmem_ld32(tg + c * 32, gr);
        tmem_ld32(tg + kBN + c * 32, ur);
        tmem_wait_ld();
        reg_fence32(gr);
        reg_fence32(ur);
        const int col0 = nb * kBN + c * 32;
        if (row < m) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            const int col = col0 + v * 8;
            if (col >= n) break;  // n is a multiple of 8: vectors are all in or all out
            float g8[8], u8[8], a8[8];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              // gate and up as stored (rounded to T); the activation uses those values.
              const float2 g2 = round2<T>(make_float2(__uint_as_float(gr[v * 8 + e]),
                                                      __uint_as_float(gr[v * 8 + e + 1])));
              const float2 u2 = round2<T>(make_float2(__uint_as_float(ur[v * 8 + e]),
                                                      __uint_as_float(ur[v * 8 + e + 1])));
              g8[e] = g2.x;
              g8[e + 1] = g2.y;
              u8[e] = u2.x;
              u8[e + 1] = u2.y;
              a8[e] = (g2.x * sigmoid_f32(g2.x)) * u2.x;
              a8[e + 1] = (g2.y * sigmoid_f32(g2.y)) * u2.y;
            }
            *reinterpret_cast<uint4*>(act + (int64_t)row * act_stride + col) = pack<T>(a8);
            if (gate_out != nullptr) {
              *reinterpret_cast<uint4*>(gate_out + (int64_t)row * pre_stride + col) =
                  pack<T>(g8);
              *reinterpret_cast<uint4*>(up_out + (int64_t)row * pre_stride + col) = pack<T>(u8);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tmem_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :
                 : "r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------------ host ------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    cudaGetLastError();
  });
  return fn;
}

// Tensor map of a row-major [rows, cols] matrix (unit column stride, row stride `ld`
// elements) read in boxes of kBK columns x box_rows rows with 128-byte swizzle.
int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
             int box_rows, CUtensorMapDataType type, const char* name) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(PT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(map, type, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(PT_ERR_INVALID_ARGUMENT, "cannot describe %s for TMA (CUresult %d)", name,
                     (int)r);
  return PT_OK;
}

template <typename T>
int gemm_impl(const void* x, int64_t xs, const void* wg, const void* wu, int64_t ws, void* act,
              int64_t as, void* gate_out, void* up_out, int64_t ps, int64_t m, int64_t n,
              int64_t k, cudaStream_t stream) {
  const CUtensorMapDataType type = std::is_same<T, __nv_bfloat16>::value
                                       ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap mx, mg, mu;
  if (int st = make_map(&mx, x, m, k, xs, kBM, type, "x")) return st;
  if (int st = make_map(&mg, wg, n, k, ws, kBN, type, "w_gate")) return st;
  if (int st = make_map(&mu, wu, n, k, ws, kBN, type, "w_up")) return st;
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  static std::once_flag attr_once[2];
  std::call_once(attr_once[std::is_same<T, __nv_bfloat16>::value ? 1 : 0], [] {
    cudaFuncSetAttribute(swiglu_gemm_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSmemBytes);
  });
  const int64_t tiles = ((m + kBM - 1) / kBM) * ((n + kBN - 1) / kBN);
  const int grid = (int)std::min<int64_t>(tiles, sms);
  swiglu_gemm_kernel<T><<<grid, kThreads, kSmemBytes, stream>>>(
      mx, mg, mu, static_cast<T*>(act), as, static_cast<T*>(gate_out), static_cast<T*>(up_out),
      ps, (int)m, (int)n, (int)k);
  return check_launch("pt_swiglu_gemm_fwd");
}

}  // namespace

// Reads and clears this file's device error word (called by pt_take_device_error).
int take_gemm_device_error(int* code);
int take_gemm_device_error(int* code) {
  int v = 0;
  const int zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)) != cudaSuccess ||
      cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_CUDA, "cannot read the device error word");
  }
  *code = v;
  return PT_OK;
}

}  // namespace pt

using namespace pt;

extern "C" {

int pt_swiglu_gemm_fwd(const void* x, int64_t x_row_stride, const void* w_gate,
                       const void* w_up, int64_t w_row_stride, void* act,
                       int64_t act_row_stride, void* gate_out, void* up_out,
                       int64_t pre_row_stride, int64_t m, int64_t n, int64_t k, int dtype,
                       void* stream) {
  if (m < 0 || n < 0 || k < 0)
    return set_error(PT_ERR_SHAPE, "m, n, k must be >= 0 (got %lld, %lld, %lld)", (long long)m,
                     (long long)n, (long long)k);
  if (m == 0 || n == 0) return ok();
  if (k == 0) return set_error(PT_ERR_SHAPE, "k must be >= 1");
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2)
    return set_error(PT_ERR_SHAPE, "m, n and k must each be below 2^30");
  if (n % 8 != 0 || k % 8 != 0)
    return set_error(PT_ERR_SHAPE, "n and k must be multiples of 8 (got n=%lld, k=%lld)",
                     (long long)n, (long long)k);
  if (x_row_stride < k || w_row_stride < k || act_row_stride < n ||
      (gate_out != nullptr && pre_row_stride < n))
    return set_error(PT_ERR_SHAPE, "a row stride is smaller than its row");
  if (x_row_stride % 8 || w_row_stride % 8 || act_row_stride % 8 ||
      (gate_out != nullptr && pre_row_stride % 8))
    return set_error(PT_ERR_SHAPE, "row strides must be multiples of 8 elements");
  if ((gate_out == nullptr) != (up_out == nullptr))
    return set_error(PT_ERR_INVALID_ARGUMENT, "gate_out and up_out are given together or not");
  const void* ptrs[6] = {x, w_gate, w_up, act, gate_out, up_out};
  const char* names[6] = {"x", "w_gate", "w_up", "act", "gate_out", "up_out"};
  for (int i = 0; i < 6; ++i) {
    if (ptrs[i] == nullptr && i >= 4) continue;
    if (int st = check_device_ptr(ptrs[i], names[i])) return st;
    if (!aligned16(ptrs[i]))
      return set_error(PT_ERR_INVALID_ARGUMENT, "%s must be 16-byte aligned", names[i]);
  }
  switch (dtype) {
    case PT_BFLOAT16:
      return gemm_impl<__nv_bfloat16>(x, x_row_stride, w_gate, w_up, w_row_stride, act,
                                      act_row_stride, gate_out, up_out, pre_row_stride, m, n,
                                      k, as_stream(stream));
    case PT_FLOAT16:
      return gemm_impl<__half>(x, x_row_stride, w_gate, w_up, w_row_stride, act,
                               act_row_stride, gate_out, up_out, pre_row_stride, m, n, k,
                               as_stream(stream));
    default:
      return set_error(PT_ERR_UNSUPPORTED_DTYPE,
                       "pt_swiglu_gemm_fwd supports bfloat16 and float16 (got dtype %d)", dtype);
  }
}

}  // extern "C"
