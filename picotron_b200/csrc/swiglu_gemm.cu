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
// [128 x 64] each (128-byte swizzle) into a 3-stage shared-memory ring; one MMA thread issues
// tcgen05.mma (kind::f16, M = 128, N = 256: the gate rows and the up rows of the B tile side
// by side, so one instruction produces both accumulators) into one of two 256-column tensor
// memory buffers; four epilogue warps read the finished buffer with tcgen05.ld while the next
// tile accumulates into the other, stage each 32 x 32 output block in shared memory and write
// it with a TMA store. Barriers are mbarriers with bounded waits: a wait that
// runs out records an error word (pt_take_device_error) and the kernel drains its copies and
// MMAs, frees its tensor memory and returns. Large m runs the CTA-pair shape described below;
// no TMA load uses cluster multicast (each CTA loads its own tiles).

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace pt {

__device__ int g_gemm_error = 0;

namespace {

constexpr int kBM = 128;             // rows per CTA = tensor-memory lanes
constexpr int kBN = 128;             // output columns per tile (gate and up each)
constexpr int kBK = 64;              // K per stage: one 128-byte swizzle row of 16-bit values
constexpr int kUmmaK = 16;           // K of one tcgen05.mma for 16-bit inputs
constexpr int kATileBytes = kBM * kBK * 2;          // 16 KB: this CTA's rows of x
constexpr int kWTileBytes = kBN * kBK * 2;          // 16 KB: one weight tile (gate or up)
constexpr int kAccCols = 2 * kBN;    // fp32 columns of one accumulator buffer (gate | up)
constexpr int kTmemCols = 2 * kAccCols;  // double-buffered: 512 columns (all of them)
constexpr int kThreads = 256;        // warp 0 TMA, 1 MMA, 2 TMEM owner, 3 idle, 4-7 epilogue
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = kThreads / 32 - kEpiWarp0;
#ifndef PT_GEMM_GROUP_M
#define PT_GEMM_GROUP_M 16
#endif
constexpr int kGroupM = PT_GEMM_GROUP_M;  // m-tiles per raster group (L2 reuse of the weights)
constexpr int kMaxStages = 7;
constexpr long long kWaitCycles = 2000000000LL;  // about one second of SM clock
// Epilogue staging: each epilogue warp writes its 32 rows x 32 columns of act, gate and up
// (bf16/fp16: 64 bytes a row) into shared memory in the 64-byte swizzle pattern and hands
// them to TMA stores, instead of scattered 16-byte global stores from every thread.
constexpr int kEpiCols = 32;
constexpr int kStageOut = 32 * kEpiCols * 2;               // one 32 x 32 16-bit tile: 2 KB
constexpr int kEpiBufs = 2;  // double-buffered: a chunk is staged while the last one is stored
// Epilogue staging per warp: forward, kEpiBufs buffers of (act, gate, up); backward, a ring of
// kEpiInBufs buffers of (gate, up) loaded ahead and kEpiBufs of (dgate, dup) to store (the
// optional d_act is staged in the consumed gate tile). Two input buffers are enough (A/B on
// B200: a 4-deep ring ran no faster) and leave room for a fifth pipeline stage.
constexpr int kEpiInBufs = 2;
constexpr int kBarrierBytes = 512;  // shared memory reserved for GemmBarriers
constexpr int kBwdWarpStaging = (kEpiInBufs * 2 + kEpiBufs * 2) * kStageOut;
template <bool kBwd> constexpr int staging_bytes() {
  return kBwd ? kEpiWarps * kBwdWarpStaging : kEpiWarps * kEpiBufs * 3 * kStageOut;
}

// Two shapes of the same pipeline:
//  * single CTA (kPair = false): a 128 x 128 tile per CTA; each stage holds the x tile and
//    both weight tiles (48 KB), 3 stages; tcgen05.mma cta_group::1 with M = 128, N = 256.
//  * CTA pair (kPair = true, a cluster of two CTAs on two SMs): a 256 x 128 tile per pair;
//    each CTA stages its own 128 rows of x and one weight tile (the even CTA the gate rows,
//    the odd CTA the up rows: 32 KB), 5 stages; the even CTA issues tcgen05.mma cta_group::2
//    with M = 256, N = 256, which reads both CTAs' shared memory and leaves each CTA's 128
//    rows of both accumulators in its own tensor memory. Per SM this halves the weight bytes
//    moved per FLOP, so twice the bytes per SM can be in flight.
#ifndef PT_GEMM_PAIR_STAGES
#define PT_GEMM_PAIR_STAGES 5
#endif
// kBwd (the down projection's data gradient with the SwiGLU backward in the epilogue) keeps
// the same stage counts beside its load ring (for the pair 1.1 % faster than 4 stages with a
// 4-deep ring).
template <bool kPair, bool kBwd = false> struct Shape {
  static constexpr int kStages = kPair ? PT_GEMM_PAIR_STAGES : 3;
  static constexpr int kStageBytes = kATileBytes + (kPair ? 1 : 2) * kWTileBytes;
  static constexpr int kTileM = kPair ? 2 * kBM : kBM;
  static constexpr int kCtas = kPair ? 2 : 1;
  static constexpr int kStagingBytes = staging_bytes<kBwd>();
  static constexpr int kSmemBytes =
      1024 /* alignment slack */ + kStages * kStageBytes + kStagingBytes + kBarrierBytes;
};
static_assert(Shape<false>::kStages <= kMaxStages && Shape<true>::kStages <= kMaxStages &&
                  Shape<true, true>::kStages <= kMaxStages, "");
static_assert(Shape<false>::kSmemBytes <= 227 * 1024 && Shape<true>::kSmemBytes <= 227 * 1024 &&
                  Shape<false, true>::kSmemBytes <= 227 * 1024 &&
                  Shape<true, true>::kSmemBytes <= 227 * 1024,
              "stage ring + epilogue staging must fit the 227 KB of shared memory per CTA");

struct GemmBarriers {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t drain;
  uint64_t epi_full[kEpiWarps][kEpiInBufs];  // backward: the epilogue's gate/up tiles landed
  uint32_t tmem_base;
};
static_assert(sizeof(GemmBarriers) <= kBarrierBytes, "barrier block must fit its space");

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

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(p)), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// Arrive (release, cluster scope) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
               :
               : "r"(cluster_addr)
               : "memory");
}

// 2-D tiled TMA load of box {kBK, rows} at (x = column, y = row) into this CTA's shared
// memory, completing on the mbarrier at shared::cluster address `bar`. kPair: the
// cta_group::2 form, whose completion may be signalled on the pair's even CTA. No multicast.
template <bool kPair>
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar) {
  if constexpr (kPair) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        :
        : "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        :
        : "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
  }
}

// 2-D tiled TMA load of a box into this CTA's shared memory with an L2 cache policy (the
// backward epilogue's gate/up tiles, read once: evict-first keeps the GEMM operand tiles that
// later tiles re-read in L2; A/B on B200: 1.2 % faster). No multicast.
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int x,
                                                 int y, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;"
      :
      : "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
      : "memory");
}

// 2-D tiled TMA store of a {kEpiCols, 32} box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y,
                                             uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], "
      "[%1], %4;"
      :
      : "l"(reinterpret_cast<uint64_t>(map)), "r"(src), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// L2 policy that marks written lines first to be evicted: the outputs are not re-read by
// this kernel, the x and weight tiles are (A/B on B200: about 1 % faster than no hint).
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most kPending committed bulk-store groups of this thread still read shared
// memory.
template <int kPending>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kPending) : "memory");
}
// Wait until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Orders this thread's generic-proxy shared-memory writes before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Byte offset of 16-byte chunk `chunk` of row `row` in a tile of 64-byte rows laid out as TMA
// reads it with 64-byte swizzle: the chunk index is XORed with bits 1-2 of the row.
__device__ __forceinline__ uint32_t swz64(int row, int chunk) {
  return (uint32_t)(row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4));
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

template <bool kPair>
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  if constexpr (kPair) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        :
        : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        :
        : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Arrive once on `bar` (in this CTA, and for kPair also at the same offset in the peer CTA)
// when every tcgen05.mma this thread issued before has completed.
template <bool kPair>
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  if constexpr (kPair) {
    const uint16_t both = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;"
        :
        : "r"(smem_addr(bar)), "h"(both)
        : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :
                 : "r"(smem_addr(bar))
                 : "memory");
  }
}

// Commit to this CTA's barrier only (the drain before tensor memory is freed).
template <bool kPair>
__device__ __forceinline__ void umma_commit_local(uint64_t* bar) {
  if constexpr (kPair) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :
                 : "r"(smem_addr(bar))
                 : "memory");
  } else {
    umma_commit<false>(bar);
  }
}

template <bool kPair> __device__ __forceinline__ void tmem_alloc(uint32_t* dst) {
  if constexpr (kPair) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :
                 : "r"(smem_addr(dst)), "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  } else {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :
                 : "r"(smem_addr(dst)), "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
}

template <bool kPair> __device__ __forceinline__ void tmem_dealloc(uint32_t base) {
  if constexpr (kPair) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
                 :
                 : "r"(base), "r"(kTmemCols)
                 : "memory");
  } else {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :
                 : "r"(base), "r"(kTmemCols)
                 : "memory");
  }
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

// Epilogue of the backward GEMM (kBwd): per tile, each epilogue warp owns 32 rows (tensor
// memory lanes [32q, 32q + 32)) and walks 8 chunks of 32 columns, 4 in each accumulator half
// (columns c of d_act, then n_half + c); chunks past n_half (a last tile column narrower than
// 128) are skipped. Lane 0 loads the gate and up 32 x 32 tiles of the chunks with TMA (64-byte
// swizzle) into a ring of kEpiInBufs buffers, up to kEpiInBufs - 1 chunks ahead of the one
// being computed and across tile boundaries, so the loads' latency hides behind the work of
// the chunks before them. Per chunk the warp reads its 32 d_act values from tensor memory,
// rounds them to T (the d_act a separate GEMM would store), forms
// dgate = (d_act * up) * (s * (1 + gate * (1 - s))) and dup = d_act * (gate * s) with
// s = sigmoid(gate) in fp32 (the operation order of swiglu_bwd_vec), stages them and stores
// them with TMA. Every wait is bounded; after a timeout the warp stops, records the error
// word and waits (bounded) for its own loads in flight.
template <typename T, bool kPair>
__device__ __forceinline__ void bwd_epilogue(GemmBarriers* bars, unsigned char* staging,
                                             uint32_t tmem_base, const TileGrid& grid, int unit,
                                             int units, uint32_t rank,
                                             const CUtensorMap* map_da, const CUtensorMap* map_dg,
                                             const CUtensorMap* map_du,
                                             const CUtensorMap* map_gin,
                                             const CUtensorMap* map_uin, int save_da,
                                             int n_half) {
  using S = Shape<kPair, true>;
  constexpr int kChunks = 2 * kBN / kEpiCols;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = warp & 3, wi = warp - kEpiWarp0;
  const uint32_t empty_addr0 = kPair ? peer_addr(&bars->tmem_empty[0], 0)
                                     : smem_addr(&bars->tmem_empty[0]);
  const uint64_t policy = evict_first_policy();
  unsigned char* in0 = staging + (size_t)wi * kBwdWarpStaging;  // kEpiInBufs x (gate, up)
  unsigned char* out0 = in0 + kEpiInBufs * 2 * kStageOut;        // kEpiBufs x (dgate, dup)
  // Live chunks of a tile: the first per_half of each half; live chunk li is chunk j = li of
  // the first half or kChunks / 2 + (li - per_half) of the second.
  auto per_half_of = [&](int nb) { return min(kChunks / 2, (n_half - nb * kBN) / kEpiCols); };
  auto col_of = [&](int nb, int j) { return (j >> 2) * n_half + nb * kBN + (j & 3) * kEpiCols; };
  // Load cursor: this CTA's tile lt and its live chunk lli; L loads issued, C chunks consumed.
  int lt = unit, lli = 0;
  uint32_t L = 0, C = 0;
  auto issue_next = [&]() -> bool {
    if (lt >= grid.count()) return false;
    int mb, nb;
    grid.coords(lt, mb, nb);
    const int ph = per_half_of(nb);
    const int j = lli < ph ? lli : kChunks / 2 + (lli - ph);
    const int row = mb * S::kTileM + (int)rank * kBM + q * 32;
    const int bb = (int)(L % kEpiInBufs);
    unsigned char* st = in0 + bb * 2 * kStageOut;
    uint64_t* bar = &bars->epi_full[wi][bb];
    if (lane == 0) {
      // With d_act staged in a gate tile, its TMA store must have read it first.
      if (save_da) bulk_wait_read<0>();
      mbar_arrive_expect_tx(bar, 2 * kStageOut);
      tma_load_2d_hint(smem_addr(st), map_gin, col_of(nb, j), row, smem_addr(bar), policy);
      tma_load_2d_hint(smem_addr(st + kStageOut), map_uin, col_of(nb, j), row, smem_addr(bar),
                       policy);
    }
    ++L;
    if (++lli == 2 * ph) {
      lli = 0;
      lt += units;
    }
    return true;
  };
  // Up to kEpiInBufs loads in flight, counting the chunk being computed; the buffer a new load
  // fills was last read by chunk L - kEpiInBufs < C, already consumed and fenced.
  auto prefetch = [&]() {
    while (L < C + kEpiInBufs && issue_next()) {
    }
  };
  bool ok = true;
  int i = 0;
  for (int t = unit; ok && t < grid.count(); t += units, ++i) {
    const int b = i & 1;
    int mb, nb;
    grid.coords(t, mb, nb);
    const int row0 = mb * S::kTileM + (int)rank * kBM + q * 32;  // this warp's rows
    const int ph = per_half_of(nb);
    prefetch();
    if (!wait_bounded(&bars->tmem_full[b], (i >> 1) & 1)) {
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t tg = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kAccCols);
#pragma unroll 1
    for (int li = 0; li < 2 * ph; ++li) {
      prefetch();
      const int j = li < ph ? li : kChunks / 2 + (li - ph);
      const int bb = (int)(C % kEpiInBufs);
      if (!wait_bounded(&bars->epi_full[wi][bb], (C / kEpiInBufs) & 1)) {
        ok = false;
        break;
      }
      unsigned char* st = in0 + bb * 2 * kStageOut;
      unsigned char* so = out0 + (C & 1) * 2 * kStageOut;
      uint32_t ar[32];
      tmem_ld32(tg + (j >> 2) * kBN + (j & 3) * kEpiCols, ar);
      tmem_wait_ld();
      reg_fence32(ar);
      // The TMA stores that last used this output buffer must have read it.
      if (lane == 0) bulk_wait_read<kEpiBufs - 1>();
      __syncwarp();
#pragma unroll
      for (int v = 0; v < 4; ++v) {  // 16-byte chunk v of this thread's row
        const uint32_t off = swz64(lane, v);
        float g8[8], u8[8], dg8[8], du8[8], da8[8];
        unpack<T>(lds128(st + off), g8);
        unpack<T>(lds128(st + kStageOut + off), u8);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float2 a2 = round2<T>(make_float2(__uint_as_float(ar[v * 8 + e]),
                                                  __uint_as_float(ar[v * 8 + e + 1])));
          da8[e] = a2.x;
          da8[e + 1] = a2.y;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float sg = sigmoid_f32(g8[e]);
          dg8[e] = (da8[e] * u8[e]) * (sg * (1.0f + g8[e] * (1.0f - sg)));
          du8[e] = da8[e] * (g8[e] * sg);
        }
        *reinterpret_cast<uint4*>(so + off) = pack<T>(dg8);
        *reinterpret_cast<uint4*>(so + kStageOut + off) = pack<T>(du8);
        // The gate values at `off` were read above by this thread alone: reuse the slot.
        if (save_da) *reinterpret_cast<uint4*>(st + off) = pack<T>(da8);
      }
      // Orders this chunk's shared-memory reads (before TMA refills the buffer) and writes
      // (before the TMA stores read them) with the async proxy.
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int col = col_of(nb, j);
        tma_store_2d(map_dg, smem_addr(so), col, row0, policy);
        tma_store_2d(map_du, smem_addr(so + kStageOut), col, row0, policy);
        if (save_da) tma_store_2d(map_da, smem_addr(st), col, row0, policy);
        bulk_commit();
      }
      ++C;
    }
    if (!ok) break;
    tc_fence_before();
    __syncwarp();
    // Release this accumulator buffer to the MMA issuer (on the even CTA of a pair).
    if (lane == 0) mbar_arrive_cluster(empty_addr0 + (uint32_t)(b * sizeof(uint64_t)));
  }
  if (!ok) {
    record_gemm_error();
    // Loads still in flight must land before this CTA's shared memory is released.
    for (uint32_t c = C; c < L; ++c)
      wait_bounded(&bars->epi_full[wi][c % kEpiInBufs], (c / kEpiInBufs) & 1);
  }
  // The staging tiles must stay valid until this warp's last TMA stores have completed.
  if (lane == 0) bulk_wait_all();
  __syncwarp();
}

// Forward: A = x, B = (w_gate | w_up), epilogue act = silu(gate) * up (+ gate, up stored).
// kBwd: A = dy (the down projection's output gradient), B = the two halves of w_down^T
// (rows [0, n) and [n, 2n) of the [2n, k] transposed down weight), so the accumulator holds
// d_act for columns c and n + c of a tile; the epilogue (bwd_epilogue) reads gate and up at
// those columns and stores dgate and dup (+ d_act when save_pre). map_act/map_gate/map_up
// are then the d_act, dgate and dup outputs and map_gin/map_uin the gate and up inputs.
template <typename T, bool kPair, bool kBwd>
__device__ __forceinline__ void swiglu_gemm_body(const CUtensorMap* map_x,
                                                 const CUtensorMap* map_wg,
                                                 const CUtensorMap* map_wu,
                                                 const CUtensorMap* map_act,
                                                 const CUtensorMap* map_gate,
                                                 const CUtensorMap* map_up,
                                                 const CUtensorMap* map_gin,
                                                 const CUtensorMap* map_uin, int save_pre, int m,
                                                 int n, int k) {
  using S = Shape<kPair, kBwd>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_addr(smem_raw);
  const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;
  unsigned char* tiles = smem_raw + pad;
  unsigned char* staging = tiles + S::kStages * S::kStageBytes;  // 1024-byte aligned
  GemmBarriers* bars = reinterpret_cast<GemmBarriers*>(staging + S::kStagingBytes);
  const uint32_t tiles_addr = raw + pad;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = kPair ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const int unit = blockIdx.x / S::kCtas, units = gridDim.x / S::kCtas;
  const TileGrid grid{(m + S::kTileM - 1) / S::kTileM, (n + kBN - 1) / kBN};
  const int kblocks = (k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->tmem_full[b], 1);
      mbar_init(&bars->tmem_empty[b], kEpiWarps * S::kCtas);
    }
    mbar_init(&bars->drain, 1);
    for (int w = 0; w < kEpiWarps; ++w)
      for (int b = 0; b < kEpiInBufs; ++b) mbar_init(&bars->epi_full[w][b], 1);
    fence_mbar_init();
  }
  if (warp == 2) tmem_alloc<kPair>(&bars->tmem_base);
  tc_fence_before();
  if constexpr (kPair) cluster_sync(); else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer --
    // Both CTAs of a pair load their own halves; the copies complete on the even CTA's
    // `full` barrier, whose expected byte count covers both halves.
    if (lane == 0) {
      RingPos pos;
      uint32_t issued_mask = 0, issued_phase = 0;  // per slot: ever issued, parity of last
      bool ok = true;
      for (int t = unit; ok && t < grid.count(); t += units) {
        int mb, nb;
        grid.coords(t, mb, nb);
        const int row0 = mb * S::kTileM + (int)rank * kBM;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(&bars->empty[pos.slot], pos.phase ^ 1u)) {
            ok = false;
            break;
          }
          uint64_t* full = &bars->full[pos.slot];
          if (leader) mbar_arrive_expect_tx(full, S::kCtas * S::kStageBytes);
          const uint32_t full_addr = kPair ? peer_addr(full, 0) : smem_addr(full);
          const uint32_t sa = tiles_addr + pos.slot * S::kStageBytes;
          tma_load_2d<kPair>(sa, map_x, kb * kBK, row0, full_addr);
          if constexpr (kPair) {
            tma_load_2d<true>(sa + kATileBytes, leader ? map_wg : map_wu, kb * kBK, nb * kBN,
                              full_addr);
          } else {
            tma_load_2d<false>(sa + kATileBytes, map_wg, kb * kBK, nb * kBN, full_addr);
            tma_load_2d<false>(sa + kATileBytes + kWTileBytes, map_wu, kb * kBK, nb * kBN,
                               full_addr);
          }
          issued_mask |= 1u << pos.slot;
          issued_phase = (issued_phase & ~(1u << pos.slot)) | (pos.phase << pos.slot);
          pos.advance(1, S::kStages);
        }
      }
      if (!ok) record_gemm_error();
      // Every copy this CTA issued must have landed before it may exit (the even CTA's
      // barriers also count the odd CTA's bytes).
      if (leader)
        for (int s = 0; s < S::kStages; ++s)
          if (issued_mask >> s & 1u) wait_bounded(&bars->full[s], issued_phase >> s & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer --
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = instr_desc<T>(S::kTileM, 2 * kBN);
      RingPos pos;
      bool ok = true;
      int i = 0;
      for (int t = unit; ok && t < grid.count(); t += units, ++i) {
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
          const uint32_t sa = tiles_addr + pos.slot * S::kStageBytes;
          const uint64_t adesc = smem_desc_sw128(sa);
          const uint64_t bdesc = smem_desc_sw128(sa + kATileBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            // Advancing the start address by 32 bytes selects the next 16 K-elements inside
            // the swizzled 128-byte rows (the swizzle is a function of the address bits).
            const uint64_t step = (uint64_t)((kk * kUmmaK * 2) >> 4);
            umma_f16<kPair>(d, adesc + step, bdesc + step, idesc, (kb | kk) != 0);
          }
          umma_commit<kPair>(&bars->empty[pos.slot]);  // frees the stage in both CTAs
          pos.advance(1, S::kStages);
        }
        if (!ok) break;
        umma_commit<kPair>(&bars->tmem_full[b]);
      }
      if (!ok) record_gemm_error();
      // All MMAs this thread issued must be complete before the tensor memory is freed.
      umma_commit_local<kPair>(&bars->drain);
      wait_bounded(&bars->drain, 0);
    }
    __syncwarp();
  } else if (warp >= kEpiWarp0 && kBwd) {
    bwd_epilogue<T, kPair>(bars, staging, tmem_base, grid, unit, units, rank, map_act, map_gate,
                           map_up, map_gin, map_uin, save_pre, n);
  } else if (warp >= kEpiWarp0) {
    // ---------------------------------------------------------------- epilogue --
    const int q = warp & 3;  // this warp may read tensor-memory lanes [32q, 32q + 32)
    const uint32_t empty_addr0 = kPair ? peer_addr(&bars->tmem_empty[0], 0)
                                       : smem_addr(&bars->tmem_empty[0]);
    const uint64_t policy = evict_first_policy();
    int i = 0;
    for (int t = unit; t < grid.count(); t += units, ++i) {
      const int b = i & 1;
      if (!wait_bounded(&bars->tmem_full[b], (i >> 1) & 1)) {
        record_gemm_error();
        break;
      }
      tc_fence_after();
      int mb, nb;
      grid.coords(t, mb, nb);
      const int row0 = mb * S::kTileM + (int)rank * kBM + q * 32;  // this warp's rows
      const uint32_t tg = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kAccCols);
      unsigned char* st0 = staging + (size_t)(warp - kEpiWarp0) * kEpiBufs * 3 * kStageOut;
#pragma unroll 1
      for (int c = 0; c < kBN / kEpiCols; ++c) {
        unsigned char* st = st0 + (c % kEpiBufs) * 3 * kStageOut;
        const uint32_t st_addr = smem_addr(st);
        uint32_t gr[32], ur[32];
        tmem_ld32(tg + c * kEpiCols, gr);
        tmem_ld32(tg + kBN + c * kEpiCols, ur);
        tmem_wait_ld();
        reg_fence32(gr);
        reg_fence32(ur);
        // The TMA stores that last used this staging buffer must have read it.
        if (lane == 0) bulk_wait_read<kEpiBufs - 1>();
        __syncwarp();
#pragma unroll
        for (int v = 0; v < 4; ++v) {  // 16-byte chunk v of this thread's row
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
          const uint32_t off = swz64(lane, v);
          *reinterpret_cast<uint4*>(st + off) = pack<T>(a8);
          if (save_pre) {
            *reinterpret_cast<uint4*>(st + kStageOut + off) = pack<T>(g8);
            *reinterpret_cast<uint4*>(st + 2 * kStageOut + off) = pack<T>(u8);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // Rows past m and columns past n are clipped by the tensor maps.
          const int col0 = nb * kBN + c * kEpiCols;
          tma_store_2d(map_act, st_addr, col0, row0, policy);
          if (save_pre) {
            tma_store_2d(map_gate, st_addr + kStageOut, col0, row0, policy);
            tma_store_2d(map_up, st_addr + 2 * kStageOut, col0, row0, policy);
          }
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      // Release this buffer to the MMA issuer (on the even CTA of a pair).
      if (lane == 0) mbar_arrive_cluster(empty_addr0 + (uint32_t)(b * sizeof(uint64_t)));
    }
    // The staging tiles must stay valid until this warp's last TMA stores have completed.
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  if constexpr (kPair) cluster_sync(); else __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc<kPair>(tmem_base);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
swiglu_gemm_kernel(const __grid_constant__ CUtensorMap map_x,
                   const __grid_constant__ CUtensorMap map_wg,
                   const __grid_constant__ CUtensorMap map_wu,
                   const __grid_constant__ CUtensorMap map_act,
                   const __grid_constant__ CUtensorMap map_gate,
                   const __grid_constant__ CUtensorMap map_up, int save_pre, int m, int n, int k) {
  swiglu_gemm_body<T, false, false>(&map_x, &map_wg, &map_wu, &map_act, &map_gate, &map_up,
                                    &map_gate, &map_up, save_pre, m, n, k);
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
swiglu_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_x,
                        const __grid_constant__ CUtensorMap map_wg,
                        const __grid_constant__ CUtensorMap map_wu,
                        const __grid_constant__ CUtensorMap map_act,
                        const __grid_constant__ CUtensorMap map_gate,
                        const __grid_constant__ CUtensorMap map_up, int save_pre, int m, int n,
                        int k) {
  swiglu_gemm_body<T, true, false>(&map_x, &map_wg, &map_wu, &map_act, &map_gate, &map_up,
                                   &map_gate, &map_up, save_pre, m, n, k);
}

// The down projection's data gradient with the SwiGLU backward in the epilogue (see
// swiglu_gemm_body, kBwd): map_dy [m, k], map_w0 / map_w1 the two [n, k] halves of w_down^T,
// outputs map_da (optional d_act), map_dg, map_du [m, 2n], inputs map_gin, map_uin [m, 2n].
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
swiglu_gemm_bwd_kernel(const __grid_constant__ CUtensorMap map_dy,
                       const __grid_constant__ CUtensorMap map_w0,
                       const __grid_constant__ CUtensorMap map_w1,
                       const __grid_constant__ CUtensorMap map_da,
                       const __grid_constant__ CUtensorMap map_dg,
                       const __grid_constant__ CUtensorMap map_du,
                       const __grid_constant__ CUtensorMap map_gin,
                       const __grid_constant__ CUtensorMap map_uin, int save_da, int m, int n,
                       int k) {
  swiglu_gemm_body<T, false, true>(&map_dy, &map_w0, &map_w1, &map_da, &map_dg, &map_du,
                                   &map_gin, &map_uin, save_da, m, n, k);
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
swiglu_gemm_bwd_pair_kernel(const __grid_constant__ CUtensorMap map_dy,
                            const __grid_constant__ CUtensorMap map_w0,
                            const __grid_constant__ CUtensorMap map_w1,
                            const __grid_constant__ CUtensorMap map_da,
                            const __grid_constant__ CUtensorMap map_dg,
                            const __grid_constant__ CUtensorMap map_du,
                            const __grid_constant__ CUtensorMap map_gin,
                            const __grid_constant__ CUtensorMap map_uin, int save_da, int m,
                            int n, int k) {
  swiglu_gemm_body<T, true, true>(&map_dy, &map_w0, &map_w1, &map_da, &map_dg, &map_du,
                                  &map_gin, &map_uin, save_da, m, n, k);
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
// elements) moved in boxes of box_cols x box_rows: operands are read as kBK columns with
// 128-byte swizzle, outputs written as kEpiCols columns with 64-byte swizzle.
int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
             int box_rows, CUtensorMapDataType type, const char* name, int box_cols = kBK,
             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (fn == nullptr) return set_error(PT_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = fn(map, type, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(PT_ERR_INVALID_ARGUMENT, "cannot describe %s for TMA (CUresult %d)", name,
                     (int)r);
  return PT_OK;
}

// Raises a kernel's dynamic shared memory limit once per device.
bool allow_smem(const void* fn, int bytes, int dev) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({fn, dev})) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  done.insert({fn, dev});
  return true;
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
  // Outputs: one 32-row x kEpiCols box per TMA store. Without gate/up outputs their maps
  // repeat the activation's and are never used.
  const int save_pre = gate_out != nullptr;
  CUtensorMap ma, mgo, muo;
  if (int st = make_map(&ma, act, m, n, as, 32, type, "act", kEpiCols, CU_TENSOR_MAP_SWIZZLE_64B))
    return st;
  if (save_pre) {
    if (int st = make_map(&mgo, gate_out, m, n, ps, 32, type, "gate_out", kEpiCols,
                          CU_TENSOR_MAP_SWIZZLE_64B))
      return st;
    if (int st = make_map(&muo, up_out, m, n, ps, 32, type, "up_out", kEpiCols,
                          CU_TENSOR_MAP_SWIZZLE_64B))
      return st;
  } else {
    mgo = ma;
    muo = ma;
  }
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  const int64_t tiles_n = (n + kBN - 1) / kBN;
  // CTA pairs whenever there are at least two row blocks to pair up.
  if (m > kBM && sms >= 2) {
    using S = Shape<true>;
    const void* fn = (const void*)swiglu_gemm_pair_kernel<T>;
    if (!allow_smem(fn, S::kSmemBytes, dev))
      return set_error(PT_ERR_CUDA, "cannot raise the shared memory limit of the GEMM kernel");
    const int64_t tiles = ((m + S::kTileM - 1) / S::kTileM) * tiles_n;
    const int pairs = (int)std::min<int64_t>(tiles, sms / 2);
    swiglu_gemm_pair_kernel<T><<<2 * pairs, kThreads, S::kSmemBytes, stream>>>(
        mx, mg, mu, ma, mgo, muo, save_pre, (int)m, (int)n, (int)k);
  } else {
    using S = Shape<false>;
    const void* fn = (const void*)swiglu_gemm_kernel<T>;
    if (!allow_smem(fn, S::kSmemBytes, dev))
      return set_error(PT_ERR_CUDA, "cannot raise the shared memory limit of the GEMM kernel");
    const int64_t tiles = ((m + S::kTileM - 1) / S::kTileM) * tiles_n;
    const int grid = (int)std::min<int64_t>(tiles, sms);
    swiglu_gemm_kernel<T><<<grid, kThreads, S::kSmemBytes, stream>>>(
        mx, mg, mu, ma, mgo, muo, save_pre, (int)m, (int)n, (int)k);
  }
  return check_launch("pt_swiglu_gemm_fwd");
}

// d_act = dy @ w_down (computed as dy against w_down_t = w_down^T, [n, k] row-major, split
// into its two n/2-row halves) with dgate / dup from gate and up in the epilogue; d_act is
// stored only when dact_out is given.
template <typename T>
int gemm_bwd_impl(const void* dy, int64_t dys, const void* wdt, int64_t wds, const void* gate,
                  const void* up, int64_t ps, void* dgate, void* dup, int64_t gs, void* dact,
                  int64_t das, int64_t m, int64_t n, int64_t k, cudaStream_t stream) {
  const CUtensorMapDataType type = std::is_same<T, __nv_bfloat16>::value
                                       ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const int64_t nh = n / 2;
  const void* wdt1 = static_cast<const unsigned char*>(wdt) + nh * wds * (int64_t)sizeof(T);
  constexpr auto sw64 = CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap mdy, mw0, mw1, mgi, mui, mdg, mdu, mda;
  if (int st = make_map(&mdy, dy, m, k, dys, kBM, type, "dy")) return st;
  if (int st = make_map(&mw0, wdt, nh, k, wds, kBN, type, "w_down_t")) return st;
  if (int st = make_map(&mw1, wdt1, nh, k, wds, kBN, type, "w_down_t (second half)")) return st;
  if (int st = make_map(&mgi, gate, m, n, ps, 32, type, "gate", kEpiCols, sw64)) return st;
  if (int st = make_map(&mui, up, m, n, ps, 32, type, "up", kEpiCols, sw64)) return st;
  if (int st = make_map(&mdg, dgate, m, n, gs, 32, type, "dgate", kEpiCols, sw64)) return st;
  if (int st = make_map(&mdu, dup, m, n, gs, 32, type, "dup", kEpiCols, sw64)) return st;
  const int save_da = dact != nullptr;
  if (save_da) {
    if (int st = make_map(&mda, dact, m, n, das, 32, type, "dact_out", kEpiCols, sw64)) return st;
  } else {
    mda = mdg;  // never used
  }
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  const int64_t tiles_n = (nh + kBN - 1) / kBN;
  if (m > kBM && sms >= 2) {
    using S = Shape<true, true>;
    const void* fn = (const void*)swiglu_gemm_bwd_pair_kernel<T>;
    if (!allow_smem(fn, S::kSmemBytes, dev))
      return set_error(PT_ERR_CUDA, "cannot raise the shared memory limit of the GEMM kernel");
    const int64_t tiles = ((m + S::kTileM - 1) / S::kTileM) * tiles_n;
    const int pairs = (int)std::min<int64_t>(tiles, sms / 2);
    swiglu_gemm_bwd_pair_kernel<T><<<2 * pairs, kThreads, S::kSmemBytes, stream>>>(
        mdy, mw0, mw1, mda, mdg, mdu, mgi, mui, save_da, (int)m, (int)nh, (int)k);
  } else {
    using S = Shape<false, true>;
    const void* fn = (const void*)swiglu_gemm_bwd_kernel<T>;
    if (!allow_smem(fn, S::kSmemBytes, dev))
      return set_error(PT_ERR_CUDA, "cannot raise the shared memory limit of the GEMM kernel");
    const int64_t tiles = ((m + S::kTileM - 1) / S::kTileM) * tiles_n;
    const int grid = (int)std::min<int64_t>(tiles, sms);
    swiglu_gemm_bwd_kernel<T><<<grid, kThreads, S::kSmemBytes, stream>>>(
        mdy, mw0, mw1, mda, mdg, mdu, mgi, mui, save_da, (int)m, (int)nh, (int)k);
  }
  return check_launch("pt_swiglu_gemm_bwd");
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

int pt_swiglu_gemm_bwd(const void* dy, int64_t dy_row_stride, const void* w_down_t,
                       int64_t w_row_stride, const void* gate, const void* up,
                       int64_t pre_row_stride, void* dgate, void* dup, int64_t grad_row_stride,
                       void* dact_out, int64_t dact_row_stride, int64_t m, int64_t n, int64_t k,
                       int dtype, void* stream) {
  if (m < 0 || n < 0 || k < 0)
    return set_error(PT_ERR_SHAPE, "m, n, k must be >= 0 (got %lld, %lld, %lld)", (long long)m,
                     (long long)n, (long long)k);
  if (m == 0 || n == 0) return ok();
  if (k == 0) return set_error(PT_ERR_SHAPE, "k must be >= 1");
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2)
    return set_error(PT_ERR_SHAPE, "m, n and k must each be below 2^30");
  if (n % 64 != 0 || k % 8 != 0)
    return set_error(PT_ERR_SHAPE, "n must be a multiple of 64 and k of 8 (got n=%lld, k=%lld)",
                     (long long)n, (long long)k);
  if (dy_row_stride < k || w_row_stride < k || pre_row_stride < n || grad_row_stride < n ||
      (dact_out != nullptr && dact_row_stride < n))
    return set_error(PT_ERR_SHAPE, "a row stride is smaller than its row");
  if (dy_row_stride % 8 || w_row_stride % 8 || pre_row_stride % 8 || grad_row_stride % 8 ||
      (dact_out != nullptr && dact_row_stride % 8))
    return set_error(PT_ERR_SHAPE, "row strides must be multiples of 8 elements");
  const void* ptrs[7] = {dy, w_down_t, gate, up, dgate, dup, dact_out};
  const char* names[7] = {"dy", "w_down_t", "gate", "up", "dgate", "dup", "dact_out"};
  for (int i = 0; i < 7; ++i) {
    if (ptrs[i] == nullptr && i == 6) continue;
    if (int st = check_device_ptr(ptrs[i], names[i])) return st;
    if (!aligned16(ptrs[i]))
      return set_error(PT_ERR_INVALID_ARGUMENT, "%s must be 16-byte aligned", names[i]);
  }
  for (int o = 4; o < 7; ++o)
    for (int i = 0; i < 4; ++i)
      if (ptrs[o] != nullptr && ptrs[o] == ptrs[i])
        return set_error(PT_ERR_INVALID_ARGUMENT, "%s must not alias %s", names[o], names[i]);
  switch (dtype) {
    case PT_BFLOAT16:
      return gemm_bwd_impl<__nv_bfloat16>(dy, dy_row_stride, w_down_t, w_row_stride, gate, up,
                                          pre_row_stride, dgate, dup, grad_row_stride, dact_out,
                                          dact_row_stride, m, n, k, as_stream(stream));
    case PT_FLOAT16:
      return gemm_bwd_impl<__half>(dy, dy_row_stride, w_down_t, w_row_stride, gate, up,
                                   pre_row_stride, dgate, dup, grad_row_stride, dact_out,
                                   dact_row_stride, m, n, k, as_stream(stream));
    default:
      return set_error(PT_ERR_UNSUPPORTED_DTYPE,
                       "pt_swiglu_gemm_bwd supports bfloat16 and float16 (got dtype %d)", dtype);
  }
}

}  // extern "C"
