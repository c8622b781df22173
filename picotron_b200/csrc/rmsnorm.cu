// RMSNorm forward/backward and the deterministic dweight reduction for sm_100a.
//
// Math follows src/picotron/nn/triton_kernels/rmsnorm.py of the reference:
//   forward  (:25-46, :49-60)   r = rsqrt(mean(x^2) + eps), y = (x * r) * w, fp32 math
//   backward (:109-134)          g = dy * w, dx = r * (g - (x * r^2) * mean(g * x)),
//                                dw = sum_rows (dy * x) * r
//
// Layout: x, y, dy, dx are [rows, hidden] with a row stride and contiguous columns.
//
// Fast path: a warp-specialised, persistent pipeline per CTA.
//  * A producer warp streams the CTA's rows (b, b + G, b + 2G, ...) into a ring of
//    `stages` shared-memory slots with 1-D TMA bulk copies (cp.async.bulk; one x row, or
//    an x row and a dy row, per slot), completing on the slot's `full` mbarrier.
//  * RW reducer warps each own whole rows (warp-per-row, no cross-warp dependency): a
//    reducer reads its row from the slot, forms the row statistics (r, and in the
//    backward c = r^2 mean(dy w x)) and publishes them on the slot's `stats` mbarrier.
//  * C owner warps own fixed 16-byte column vectors of every row (lane l of warp w owns
//    vectors l + 32 (w + C k)) and keep their columns' weight, and in the backward an
//    fp64 dweight accumulator, in registers for the whole kernel. Once a row's statistics
//    are published they do only elementwise work (y, or dx and dweight), then arrive on
//    the slot's `empty` mbarrier, which hands the slot back to the producer. The forward
//    streams y out with 16-byte stores; the backward writes dx over its own x elements in
//    the slot and the producer stores the whole row with one bulk copy (cp.async.bulk)
//    before it refills the slot.
//  No CTA-wide barrier and no cross-warp reduction run in the loop: the reductions of
//  later rows proceed while owners stream out earlier rows.
// Every mbarrier wait is bounded (about 1 s); a timeout records kDeviceErrWaitTimeout in
// the device error word and the CTA stops after a bounded drain of its copies.
//
// dweight precision: r is refined to fp64 precision from an fp64 row sum; each term
// (dy * x) * r is accumulated in fp64 with one fma (dy * x of two 16-bit floats is exact
// in fp32, of two fp32 values exact in fp64). Each CTA's partial is therefore the exact
// sum to about 2^-50 relative, however many rows it reduces; it is stored as an fp32 pair
// (rounded sum, rounded remainder) and pt_rmsnorm_dw_reduce adds the partials in fp64 in a
// fixed order. One fp64 fma and one conversion per element
// leave the fp64 pipe far from saturated at HBM speed.
//
// Generic path: any hidden size, stride or alignment; one row per CTA iteration with
// scalar accesses and two passes over the row (the second one hits L2).
#include <algorithm>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"

namespace pt {

// Read and clear the device error words of the fused SwiGLU GEMM (swiglu_gemm.cu) and of
// the cross-entropy kernels (cross_entropy.cu).
int take_gemm_device_error(int* code);
int take_ce_device_error(int* code);

// Device-side error word of this library on each device (0 = none). Kernels that give up
// on a bounded wait record kDeviceErrWaitTimeout here; pt_take_device_error reads it.
__device__ int g_device_error = 0;

namespace {

// Tuning knobs (compile-time overridable for sweeps).
#ifndef PT_RMS_ELEMS_FWD
#define PT_RMS_ELEMS_FWD 32  // elements of a row owned by each forward owner thread
#endif
#ifndef PT_RMS_ELEMS_BWD
#define PT_RMS_ELEMS_BWD 16  // backward owners also hold an fp64 dweight sum each
#endif
#ifndef PT_RMS_SMEM_FWD
#define PT_RMS_SMEM_FWD (48 * 1024)  // forward ring budget per CTA (fp32 rows)
#endif
#ifndef PT_RMS_SMEM_FWD16
#define PT_RMS_SMEM_FWD16 (24 * 1024)  // forward ring budget per CTA (16-bit rows)
#endif
#ifndef PT_RMS_SMEM_BWD
#define PT_RMS_SMEM_BWD (64 * 1024)  // backward ring budget per CTA (plus the staged weight)
#endif
#ifndef PT_RMS_MIN_BLOCKS_FWD
#define PT_RMS_MIN_BLOCKS_FWD 2
#endif
#ifndef PT_RMS_MIN_BLOCKS_BWD
#define PT_RMS_MIN_BLOCKS_BWD 2
#endif
#ifndef PT_RMS_MIN_STAGES
#define PT_RMS_MIN_STAGES 3
#endif
#ifndef PT_RMS_REDUCERS
#define PT_RMS_REDUCERS 4  // reducer warps per CTA
#endif
// 16-bit backward without the fused add: 3 reducer warps and a 96 KB ring (6 slots of x and
// dy rows at hidden 4096). A/B on B200 at 16384 x 4096 bf16: 0.81 -> 0.85 of the HBM peak
// against 4 reducers and 4 slots; the same change made the fp32 backward and the forward
// slower, so they keep the defaults.
#ifndef PT_RMS_REDUCERS_BWD16
#define PT_RMS_REDUCERS_BWD16 3
#endif
#ifndef PT_RMS_SMEM_BWD16
#define PT_RMS_SMEM_BWD16 (96 * 1024)
#endif
// 16-bit forward: 3 reducer warps and 3 ring slots (24 KB at hidden 4096 bf16). A/B on B200
// at 16384 x 4096 bf16: 0.90 of the HBM peak against 0.88 with 4 reducers and 4 slots, and
// the fused add forward 0.94 against 0.85; deeper rings (6-12 slots), 2 reducers, or one CTA
// per SM were slower: the forward runs best with few rows in flight per SM. fp32 rows keep
// 4 reducers and the 48 KB budget (0.90 against 0.89).
#ifndef PT_RMS_REDUCERS_FWD
#define PT_RMS_REDUCERS_FWD 3
#endif
// Output rows written back with bulk copies of whole rows from the slot they were computed
// in (1), or with 16-byte streaming stores from every owner thread (0). A/B on B200 at
// 16384 x 4096 bf16: the backward 72.6 -> 71.7 us (with the dweight reduce after it 79.0 ->
// 76.7 us) with bulk copies; the forward 45.4 -> 46.7 us, so it keeps streaming stores.
#ifndef PT_RMS_BULK_OUT_FWD
#define PT_RMS_BULK_OUT_FWD 0
#endif
#ifndef PT_RMS_BULK_OUT_BWD
#define PT_RMS_BULK_OUT_BWD 1
#endif
#ifndef PT_RMS_REDUCERS_ADDBWD16
#define PT_RMS_REDUCERS_ADDBWD16 PT_RMS_REDUCERS
#endif
#ifndef PT_RMS_SMEM_ADDBWD16
#define PT_RMS_SMEM_ADDBWD16 (PT_RMS_SMEM_BWD * 3 / 2)
#endif
constexpr int kElemsFwd = PT_RMS_ELEMS_FWD;
constexpr int kElemsBwd = PT_RMS_ELEMS_BWD;
constexpr int kSmemFwd = PT_RMS_SMEM_FWD;
constexpr int kSmemBwd = PT_RMS_SMEM_BWD;
constexpr int kMinStages = PT_RMS_MIN_STAGES;
constexpr int kReducers = PT_RMS_REDUCERS;
constexpr int kReducersBwd16 = PT_RMS_REDUCERS_BWD16;
constexpr int kReducersFwd = PT_RMS_REDUCERS_FWD;
constexpr int kReducersAddBwd16 = PT_RMS_REDUCERS_ADDBWD16;
constexpr int kSmemBwd16 = PT_RMS_SMEM_BWD16;
constexpr int kMaxStages = 16;
static_assert(kReducers >= 1 && kReducers <= kMaxStages, "reducer count must fit the ring");
static_assert(kReducersBwd16 >= 1 && kReducersBwd16 <= kReducers && kReducersFwd >= 1 &&
                  kReducersFwd <= kReducers && kReducersAddBwd16 >= 1 &&
                  kReducersAddBwd16 <= kReducers,
              "the kernels' warp bound assumes at most kReducers reducers");
constexpr int kMaxConsumers = 16;  // owner warps per CTA
// CTAs of up to this many owner warps (rows of up to 4096 elements) get a tighter
// launch bound (two CTAs per SM); the backward owners hold half as many elements.
constexpr int kSmallConsumers(bool bwd) { return bwd ? 8 : 4; }
constexpr int kMaxSlotBytes = 64 * 1024;
constexpr int kGenericThreads = 256;

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

// Rows of this CTA in the strided assignment row(j) = blockIdx.x + j * gridDim.x.
__device__ __forceinline__ int64_t local_rows(int64_t rows) {
  const int64_t b = blockIdx.x;
  return rows > b ? (rows - 1 - b) / gridDim.x + 1 : 0;
}

__device__ __forceinline__ void record_timeout() {
  atomicExch(&g_device_error, kDeviceErrWaitTimeout);
}

// ------------------------------------------------------ deterministic dweight sums --
// The second stage of the dweight reduction, shared by the standalone reduce kernel and
// the tail of the fused backward so that both give the same bits: column c of dw is the
// sum of partial rows p = 0 .. P-1, formed as 64 group sums (group g adds rows g, g + 64,
// g + 128, ... in that order, in fp64), which a fixed shuffle tree then adds; one rounding
// at the end. The order depends only on P.
constexpr int kReduceCols = 16;   // columns per chunk (a half-warp of 64-byte loads)
constexpr int kReduceGroups = 64; // row groups per column
constexpr int kReduceBatch = 10;  // partial rows loaded per group at once (640 rows in one batch)
constexpr int kReduceItems = kReduceCols * kReduceGroups;

// Group sums of one 16-column chunk of a [P, hidden] fp32 partial buffer: this thread's
// items (column, group) = item & 15, item >> 4 for item = first + threadIdx.x + k *
// blockDim.x, k < kItems, each the fp64 sum of rows group, group + 64, ... in that order,
// written to s[column][group]. The loads of all of a thread's items are issued together,
// kReduceBatch rows per item at a time, so a thread waits for L2 once per batch, not once
// per item and batch. Partial rows written by other CTAs of the same grid are read
// through L2 (ld.global.cg), so a grid barrier before the call is enough to see them.
template <int kItems>
__device__ __forceinline__ void dw_group_sums(const float* partials, int P, int64_t hidden,
                                              int64_t chunk, int first,
                                              double (*s)[kReduceGroups + 1]) {
  double t[kItems];
  const float* base[kItems];
  int group[kItems];
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int item = first + threadIdx.x + k * blockDim.x;
    const int64_t c = chunk * kReduceCols + (item & (kReduceCols - 1));
    t[k] = 0.0;
    // Items past the chunk or past the last column read nothing (group = P).
    group[k] = (item < kReduceItems && c < hidden) ? (item >> 4) : P;
    base[k] = partials + c;
  }
  for (int p0 = 0; p0 < P; p0 += kReduceGroups * kReduceBatch) {
    float v[kItems][kReduceBatch];
#pragma unroll
    for (int k = 0; k < kItems; ++k)
#pragma unroll
      for (int u = 0; u < kReduceBatch; ++u) {
        const int p = p0 + group[k] + u * kReduceGroups;
        v[k][u] = p < P ? __ldcg(base[k] + (int64_t)p * hidden) : 0.0f;
      }
#pragma unroll
    for (int k = 0; k < kItems; ++k)
#pragma unroll
      for (int u = 0; u < kReduceBatch; ++u) t[k] += (double)v[k][u];
  }
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int item = first + threadIdx.x + k * blockDim.x;
    if (item < kReduceItems) s[item & (kReduceCols - 1)][item >> 4] = t[k];
  }
}

// Reduces the 16-column chunk `chunk` into dw with all threads of the CTA, kItems items
// per thread per pass (as many passes as the CTA's size needs): the group sums, then a
// fixed shuffle tree per column. `s` is a CTA-shared [kReduceCols][kReduceGroups + 1]
// scratch. Ends with a CTA barrier.
template <typename TW, int kItems>
__device__ __forceinline__ void dw_reduce_chunk(const float* partials, int P, int64_t hidden,
                                                int64_t chunk, TW* dw,
                                                double (*s)[kReduceGroups + 1]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int first = 0; first < kReduceItems; first += kItems * blockDim.x)
    dw_group_sums<kItems>(partials, P, hidden, chunk, first, s);
  __syncthreads();
  for (int col = warp; col < kReduceCols; col += nwarps) {
    const int64_t c = chunk * kReduceCols + col;
    double v = s[col][lane] + s[col][lane + 32];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
    if (lane == 0 && c < hidden) dw[c] = from_float<TW>((float)v);
  }
  __syncthreads();
}

// Grid-wide barrier of a cooperative launch (all CTAs resident), taken by one thread per
// CTA after a CTA barrier. `bar` is a word whose low 31 bits are zero between barriers:
// CTA 0 adds 2^31 - (G - 1) and every other CTA adds 1, so the last arrival flips bit 31
// and leaves the low bits at zero again; each CTA waits for the flip of the bit it saw.
// Works for any G and any value of bit 31, so the word never needs resetting. The
// fences make every CTA's earlier global writes visible to every CTA after the barrier.
// Bounded like every wait here: false after `limit` SM cycles.
__device__ __forceinline__ bool grid_barrier(unsigned int* bar, unsigned int nblocks,
                                             long long limit = kWaitLimitCycles) {
  __threadfence();
  const unsigned int add = blockIdx.x == 0 ? 0x80000000u - (nblocks - 1u) : 1u;
  const unsigned int old = atomicAdd(bar, add);
  const long long t0 = clock64();
  for (;;) {
    unsigned int cur;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(cur) : "l"(bar) : "memory");
    if ((cur ^ old) & 0x80000000u) break;
    if (clock64() - t0 > limit) return false;
  }
  __threadfence();
  return true;
}

// ------------------------------------------------------------ fast fwd / bwd -------
// Warp roles: warps [0, C) own columns, warps [C, C + RW) reduce rows, warp C + RW is the
// TMA producer.
// kAdd (fused residual add): the forward normalizes h = x + aux (aux = the branch output,
// h rounded to T and written to h_out); the backward adds aux (the gradient that reaches h
// from its other uses) to dx.
// kFused (backward only, cooperative launch): after writing its partial rows every CTA
// meets the others at a grid barrier on `grid_bar`, then reduces 16-column chunks of the
// partials into dw_out (chunk b, b + G, ...) with dw_reduce_chunk: dx and dw in one launch.
template <typename T, typename TW, int VPT, bool kBwd, bool kHasRstd, bool kAdd, int kMaxWarps,
          bool kFused>
__global__ void __launch_bounds__(kMaxWarps * 32,
                                  kMaxWarps <= 16 ? (kBwd ? PT_RMS_MIN_BLOCKS_BWD
                                                          : PT_RMS_MIN_BLOCKS_FWD)
                                                  : 1)
rmsnorm_ws(const T* __restrict__ x, int64_t xs, const T* __restrict__ dy, int64_t dys,
           const TW* __restrict__ w, const float* __restrict__ rstd_in, T* __restrict__ out,
           int64_t os, float* __restrict__ rstd_out, float* __restrict__ partials,
           float* __restrict__ partials_lo, float* __restrict__ zero_row,
           const T* __restrict__ aux, int64_t as, T* __restrict__ h_out, int64_t hs,
           int64_t rows, int nvec, int hidden, int stages, int C, int RW, float hidden_f,
           float eps, unsigned int* __restrict__ grid_bar, TW* __restrict__ dw_out,
           int num_partials) {
  static_assert(kBwd || !kFused, "only the backward reduces its dweight in the kernel");
  constexpr bool kBulkOut = kBwd ? PT_RMS_BULK_OUT_BWD : PT_RMS_BULK_OUT_FWD;
  constexpr int V = Vec16<T>::N;
  // Slot layout: x | dy (backward) | aux (kAdd).
  constexpr int kRowsPerSlot = (kBwd ? 2 : 1) + (kAdd ? 1 : 0);
  constexpr int kAuxRow = kRowsPerSlot - 1;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[kMaxStages];
  __shared__ __align__(8) uint64_t stats[kMaxStages];
  __shared__ __align__(8) uint64_t empty[kMaxStages];
  __shared__ double stat_inv[kMaxStages];
  __shared__ float stat_c[kMaxStages];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_elems = nvec * V;
  const uint32_t row_bytes = (uint32_t)nvec * 16u;
  T* slots = reinterpret_cast<T*>(smem);
  // Backward: the reducers need the weight of every column; it is staged once, in fp32,
  // after the ring, in planes of four floats: float4 number v of plane q holds the weights
  // of elements 4q .. 4q+3 of column vector v. A warp reading plane q of 32 consecutive
  // vectors then touches 512 contiguous bytes (no bank conflicts).
  float4* wsm = reinterpret_cast<float4*>(smem + (size_t)stages * kRowsPerSlot * row_bytes);
  constexpr int kPlanes = V / 4;
  const int64_t G = gridDim.x;
  const int64_t n_local = local_rows(rows);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&stats[s], 1);
      mbar_init(&empty[s], C);
    }
    fence_mbar_init();
  }
  // Launched as a programmatic dependent of the stream's previous kernel (ws_launch; not the
  // cooperative fused backward): the CTAs may take their SMs while that kernel finishes, and
  // wait here, before their first global memory access, until it has completed. The forward
  // lets the next kernel be scheduled from here on (the backward does so below).
  if constexpr (!kFused) asm volatile("griddepcontrol.wait;" ::: "memory");
  if constexpr (!kBwd) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __syncthreads();
  // The producer starts filling the ring at once; the reducer and owner warps stage the
  // backward's weight meanwhile and meet at named barrier 1 (A/B on B200: 1 us less per
  // launch at 16384 x 4096 bf16 than staging it before the first copy).
  if constexpr (kBwd) {
    // The dependent launch (the dweight reduce, launched with programmatic stream
    // serialization) may be scheduled from now on; it waits for this grid's completion.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (warp < C + RW) {
      const int nthr = (C + RW) * 32;
      float* wf32 = reinterpret_cast<float*>(wsm);
      for (int i = threadIdx.x; i < nvec * V; i += nthr) {
        const int v = i / V, e = i - v * V;
        wf32[((e >> 2) * nvec + v) * 4 + (e & 3)] = to_float(w[i]);
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    }
  }

  // ---------------------------------------------------------------- producer warp --
  if (warp == C + RW) {
    if (lane == 0) {
      RingPos pos;
      const T* xr = x + (int64_t)blockIdx.x * xs;
      const T* gr = kBwd ? dy + (int64_t)blockIdx.x * dys : nullptr;
      const T* ar = kAdd ? aux + (int64_t)blockIdx.x * as : nullptr;
      // Output rows leave the slot they were computed in as bulk copies: y or dx from the
      // x row's place, and the forward's h from the aux row's place.
      auto store_rows = [&](int slot, int64_t jrow) {
        const T* base = slots + (int64_t)(kRowsPerSlot * slot) * row_elems;
        const int64_t r = blockIdx.x + jrow * G;
        bulk_store_row(out + r * os, base, row_bytes);
        if constexpr (kAdd && !kBwd) bulk_store_row(h_out + r * hs, base + kAuxRow * row_elems,
                                                    row_bytes);
        bulk_commit_group();
      };
      bool ok = true;
      for (int64_t j = 0; j < n_local; ++j) {
        // The k-th refill of a slot waits for the owners to release use k-1, whose outputs
        // are then stored and read out of the slot before new rows land in it.
        if (j >= stages) {
          if (!mbar_wait_bounded(&empty[pos.slot], pos.phase ^ 1u)) {
            record_timeout();
            ok = false;
            break;
          }
          if (kBulkOut) {
            store_rows(pos.slot, j - stages);
            bulk_wait_all_read();
          }
        }
        mbar_arrive_expect_tx(&full[pos.slot], kRowsPerSlot * row_bytes);
        T* dst = slots + (int64_t)(kRowsPerSlot * pos.slot) * row_elems;
        bulk_load(dst, xr, row_bytes, &full[pos.slot]);
        xr += G * xs;
        if constexpr (kBwd) {
          bulk_load(dst + row_elems, gr, row_bytes, &full[pos.slot]);
          gr += G * dys;
        }
        if constexpr (kAdd) {
          bulk_load(dst + kAuxRow * row_elems, ar, row_bytes, &full[pos.slot]);
          ar += G * as;
        }
        pos.advance(1, stages);
      }
      if (kBulkOut && ok) {
        // The last min(stages, n_local) rows: store each once its owners release it.
        const int64_t first = n_local > stages ? n_local - stages : 0;
        for (int64_t jj = first; jj < n_local; ++jj) {
          const int slot = (int)(jj % stages);
          if (!mbar_wait_bounded(&empty[slot], (uint32_t)((jj / stages) & 1))) {
            record_timeout();
            break;
          }
          store_rows(slot, jj);
        }
      }
      // Shared memory must stay valid until every bulk store has read it.
      if (kBulkOut) bulk_wait_all_done();
    }
  } else if (warp >= C) {
  // ----------------------------------------------------------------- reducer warps --
  // Reducer r owns local rows r, r + RW, ...: it reads the whole row from its slot
  // (lane l takes vectors l, l + 32, ...), forms sum(x^2) (and sum(dy * w * x)), and
  // publishes r = rsqrt(mean(x^2) + eps) (and c = r^2 * mean(dy * w * x)) for the slot.
    const int rid = warp - C;
    RingPos pos;
    pos.advance(rid, stages);
    for (int64_t j = rid; j < n_local; j += RW) {
      if (!mbar_wait_bounded(&full[pos.slot], pos.phase)) {
        record_timeout();
        break;
      }
      const T* sx = slots + (int64_t)(kRowsPerSlot * pos.slot) * row_elems;
      // Four independent paired accumulators (one per vector of an unrolled group of four).
      float2 ss[4], dot[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) ss[q] = dot[q] = make_float2(0.0f, 0.0f);
      auto accumulate = [&](int v, int q) {
        float2 fx[V / 2];
        unpack2<T>(lds128(sx + v * V), fx);
        if constexpr (kAdd && !kBwd) {
          // h = x + aux, rounded to T as stored in h_out.
          float2 fa[V / 2];
          unpack2<T>(lds128(sx + kAuxRow * row_elems + v * V), fa);
#pragma unroll
          for (int e = 0; e < V / 2; ++e) fx[e] = round2<T>(__fadd2_rn(fx[e], fa[e]));
        }
        if constexpr (kBwd) {
          float2 fg[V / 2];
          unpack2<T>(lds128(sx + row_elems + v * V), fg);
          float2 wv[V / 2];
#pragma unroll
          for (int pl = 0; pl < kPlanes; ++pl) {
            const float4 t = wsm[pl * nvec + v];
            wv[2 * pl] = make_float2(t.x, t.y);
            wv[2 * pl + 1] = make_float2(t.z, t.w);
          }
#pragma unroll
          for (int e = 0; e < V / 2; ++e) {
            if (!kHasRstd) ss[q] = __ffma2_rn(fx[e], fx[e], ss[q]);
            dot[q] = __ffma2_rn(__fmul2_rn(fg[e], wv[e]), fx[e], dot[q]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < V / 2; ++e) ss[q] = __ffma2_rn(fx[e], fx[e], ss[q]);
        }
      };
      int v = lane;
      for (; v + 96 < nvec; v += 128) {
#pragma unroll
        for (int q = 0; q < 4; ++q) accumulate(v + 32 * q, q);
      }
      for (int q = 0; v < nvec; v += 32, ++q) {
        if (q == 0) accumulate(v, 0);
        else if (q == 1) accumulate(v, 1);
        else accumulate(v, 2);
      }
      const int64_t row = blockIdx.x + j * G;
      if constexpr (kBwd) {
        double invd;
        if constexpr (kHasRstd) {
          invd = (double)__ldg(rstd_in + row);
        } else {
          double ssd = ((double)ss[0].x + (double)ss[0].y) + ((double)ss[1].x + (double)ss[1].y) +
                       ((double)ss[2].x + (double)ss[2].y) + ((double)ss[3].x + (double)ss[3].y);
          ssd = warp_sum(ssd);
          invd = rsqrt_refined(ssd / (double)hidden + (double)eps);
        }
        float d = ((dot[0].x + dot[0].y) + (dot[1].x + dot[1].y)) +
                  ((dot[2].x + dot[2].y) + (dot[3].x + dot[3].y));
        d = warp_sum(d);
        if (lane == 0) {
          const float inv = (float)invd;
          stat_inv[pos.slot] = invd;
          stat_c[pos.slot] = (inv * inv) * (d / hidden_f);
        }
      } else {
        float t = ((ss[0].x + ss[0].y) + (ss[1].x + ss[1].y)) +
                  ((ss[2].x + ss[2].y) + (ss[3].x + ss[3].y));
        t = warp_sum(t);
        if (lane == 0) {
          const float inv = rsqrtf(t / hidden_f + eps);
          stat_inv[pos.slot] = (double)inv;
          if (rstd_out != nullptr) rstd_out[row] = inv;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&stats[pos.slot]);
      pos.advance(RW, stages);
    }
  } else {
  // ------------------------------------------------------------------ owner warps --
  // Forward: the owners' weights live in registers. Backward: they are read from the
  // staged fp32 copy, leaving the registers to the fp64 dweight accumulators (two CTAs per
  // SM fit only that way).
  float wf[kBwd ? 1 : VPT][V];
  // Backward: one fp64 dweight accumulator per element. dy * x is exact (in fp32 for 16-bit
  // inputs, in fp64 for fp32 inputs) and is multiplied by the fp64 r with one rounding per
  // row at 2^-53: the partial sums are exact to far below the fp32 result's precision, and
  // the fp64 fma pipe has throughput to spare at HBM speed (A/B on B200: 11 % faster than
  // doubly compensated fp32 pairs, which needed ten fp32 operations per element and row).
  constexpr int V2 = V / 2;
  double acc[kBwd ? VPT : 1][kBwd ? V : 1];
  bool valid[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = lane + 32 * (warp + C * k);
    valid[k] = v < nvec;
    if constexpr (!kBwd) {
      if (valid[k]) {
        load_row_f32<TW, V>(w + (int64_t)v * V, wf[k]);
      } else {
#pragma unroll
        for (int e = 0; e < V; ++e) wf[k][e] = 0.0f;
      }
    }
  }
  if constexpr (kBwd) {
#pragma unroll
    for (int k = 0; k < VPT; ++k)
#pragma unroll
      for (int e = 0; e < V; ++e) acc[k][e] = 0.0;
  }

  RingPos pos;
  int64_t j = 0;
  bool ok = true;
  for (; j < n_local; ++j) {
    // The slot's data (full) and its statistics (stats) must both have landed.
    ok = mbar_wait_bounded(&full[pos.slot], pos.phase) &&
         mbar_wait_bounded(&stats[pos.slot], pos.phase);
    if (!ok) break;
    const int64_t row = blockIdx.x + j * G;
    const T* sx = slots + (int64_t)(kRowsPerSlot * pos.slot) * row_elems;
    if constexpr (!kBwd) {
      const float inv = (float)stat_inv[pos.slot];
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (!valid[k]) continue;
        const int off = (lane + 32 * (warp + C * k)) * V;
        float2 f2[V / 2];
        unpack2<T>(lds128(sx + off), f2);
        if constexpr (kAdd) {
          float2 fa[V / 2];
          unpack2<T>(lds128(sx + kAuxRow * row_elems + off), fa);
          float hf[V];
#pragma unroll
          for (int e = 0; e < V / 2; ++e) {
            f2[e] = round2<T>(__fadd2_rn(f2[e], fa[e]));
            hf[2 * e] = f2[e].x;
            hf[2 * e + 1] = f2[e].y;
          }
          if constexpr (kBulkOut)  // over this thread's own aux elements, already read
            *reinterpret_cast<uint4*>(slots + (sx - slots) + kAuxRow * row_elems + off) =
                pack<T>(hf);
          else
            st_stream(h_out + row * hs + off, pack<T>(hf));
        }
        float f[V];
        const float2 inv2 = splat2(inv);
#pragma unroll
        for (int e = 0; e < V / 2; ++e) {
          const float2 o = __fmul2_rn(__fmul2_rn(f2[e], inv2),
                                      make_float2(wf[k][2 * e], wf[k][2 * e + 1]));
          f[2 * e] = o.x;
          f[2 * e + 1] = o.y;
        }
        if constexpr (kBulkOut)  // over this thread's own x elements, already read
          *reinterpret_cast<uint4*>(slots + (sx - slots) + off) = pack<T>(f);
        else
          st_stream(out + row * os + off, pack<T>(f));
      }
    } else {
      const double invd = stat_inv[pos.slot];
      const float inv = (float)invd;
      const float nc = -stat_c[pos.slot];
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        if (!valid[k]) continue;
        const int off = (lane + 32 * (warp + C * k)) * V;
        float2 fx[V2], fg[V2], wv[V2], fa[kAdd ? V2 : 1];
        float fo[V];
        unpack2<T>(lds128(sx + off), fx);
        unpack2<T>(lds128(sx + row_elems + off), fg);
        if constexpr (kAdd) unpack2<T>(lds128(sx + kAuxRow * row_elems + off), fa);
        const int vec = lane + 32 * (warp + C * k);
#pragma unroll
        for (int q = 0; q < kPlanes; ++q) {
          const float4 t = wsm[q * nvec + vec];
          wv[2 * q] = make_float2(t.x, t.y);
          wv[2 * q + 1] = make_float2(t.z, t.w);
        }
        const float2 inv2 = splat2(inv), nc2 = splat2(nc);
#pragma unroll
        for (int e = 0; e < V2; ++e) {
          // dx = r * (dy * w - x * c)
          float2 o = __fmul2_rn(inv2, __ffma2_rn(fx[e], nc2, __fmul2_rn(fg[e], wv[e])));
          if constexpr (kAdd) o = __fadd2_rn(o, fa[e]);
          fo[2 * e] = o.x;
          fo[2 * e + 1] = o.y;
          if constexpr (sizeof(T) == 4) {
            // fp32 inputs: the product of two fp32 values is exact in fp64.
            acc[k][2 * e] = fma((double)fg[e].x * (double)fx[e].x, invd, acc[k][2 * e]);
            acc[k][2 * e + 1] = fma((double)fg[e].y * (double)fx[e].y, invd, acc[k][2 * e + 1]);
          } else {
            const float2 pxy = __fmul2_rn(fg[e], fx[e]);  // exact for 16-bit inputs
            acc[k][2 * e] = fma((double)pxy.x, invd, acc[k][2 * e]);
            acc[k][2 * e + 1] = fma((double)pxy.y, invd, acc[k][2 * e + 1]);
          }
        }
        if constexpr (kBulkOut)  // over this thread's own x elements, already read
          *reinterpret_cast<uint4*>(slots + (sx - slots) + off) = pack<T>(fo);
        else
          st_stream(out + row * os + off, pack<T>(fo));
      }
    }
    // The producer's bulk copies read this thread's output elements after the release.
    if constexpr (kBulkOut) fence_async_proxy_shared();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[pos.slot]);
    pos.advance(1, stages);
  }

  if (!ok) {
    // Give copies that may still land in this CTA's slots a bounded chance to finish.
    record_timeout();
    for (int64_t i = j; i < n_local && i < j + stages; ++i) {
      mbar_wait_bounded(&full[pos.slot], pos.phase);
      pos.advance(1, stages);
    }
  } else if constexpr (kBwd) {
    // This CTA's dweight partial rows (zeros when it owned no rows): the running sums in
    // row blockIdx.x of `partials` and their accumulated errors in row blockIdx.x of
    // `partials_lo`, or, without a lo row, their fp32-rounded total.
    float* prow = partials + (int64_t)blockIdx.x * hidden;
    float* lrow = partials_lo != nullptr ? partials_lo + (int64_t)blockIdx.x * hidden : nullptr;
    // 16-bit rows give each thread eight consecutive columns per vector: with 32-byte aligned
    // partial rows each thread stores them as whole 32-byte sectors (the float4 pairs below
    // leave every sector half-written by each of two store instructions).
    const bool whole_sectors =
        V == 8 && (reinterpret_cast<uintptr_t>(prow) & 31) == 0 &&
        (lrow == nullptr || (reinterpret_cast<uintptr_t>(lrow) & 31) == 0) &&
        (zero_row == nullptr || (reinterpret_cast<uintptr_t>(zero_row) & 31) == 0);
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      if (!valid[k]) continue;
      const int64_t col = (int64_t)(lane + 32 * (warp + C * k)) * V;
      if constexpr (V == 8) {
        if (whole_sectors) {
          float hi[8], lo[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const double a = acc[k][e];
            hi[e] = (float)a;
            lo[e] = (float)(a - (double)hi[e]);
          }
          if (lrow != nullptr) {
            st_global_v8(prow + col, hi);
            st_global_v8(lrow + col, lo);
          } else {
            float t[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) t[e] = __fadd_rn(hi[e], lo[e]);
            st_global_v8(prow + col, t);
          }
          if (zero_row != nullptr && blockIdx.x == 0) {
            const float z[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            st_global_v8(zero_row + col, z);
          }
          continue;
        }
      }
      float4* dst = reinterpret_cast<float4*>(prow + col);
      float4* dlo = lrow != nullptr ? reinterpret_cast<float4*>(lrow + col) : nullptr;
      float4* dz = zero_row != nullptr && blockIdx.x == 0
                       ? reinterpret_cast<float4*>(zero_row + col) : nullptr;
#pragma unroll
      for (int q = 0; q < V / 4; ++q) {
        // Each fp64 sum as an fp32 pair hi + lo (hi the rounded sum, lo the rest rounded).
        float hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const double a = acc[k][4 * q + e];
          hi[e] = (float)a;
          lo[e] = (float)(a - (double)hi[e]);
        }
        const float2 a = make_float2(hi[0], hi[1]), b = make_float2(hi[2], hi[3]);
        const float2 ea = make_float2(lo[0], lo[1]), eb = make_float2(lo[2], lo[3]);
        if (dlo != nullptr) {
          dst[q] = make_float4(a.x, a.y, b.x, b.y);
          dlo[q] = make_float4(ea.x, ea.y, eb.x, eb.y);
        } else {
          const float2 ta = __fadd2_rn(a, ea), tb = __fadd2_rn(b, eb);
          dst[q] = make_float4(ta.x, ta.y, tb.x, tb.y);
        }
        if (dz != nullptr) dz[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
  }
  }  // owner warps

  if constexpr (kFused) {
    // Every CTA's partial rows are written: meet at the grid barrier (a cooperative launch
    // keeps all CTAs resident), then reduce this CTA's chunks of columns in the ring's
    // shared memory, which no copy uses any more.
    __syncwarp();
    __syncthreads();
    if (threadIdx.x == 0 && !grid_barrier(grid_bar, gridDim.x)) record_timeout();
    __syncthreads();
    auto* s = reinterpret_cast<double (*)[kReduceGroups + 1]>(smem);
    const int64_t chunks = (hidden + kReduceCols - 1) / kReduceCols;
    for (int64_t chunk = blockIdx.x; chunk < chunks; chunk += gridDim.x)
      dw_reduce_chunk<TW, 3>(partials, num_partials, hidden, chunk, dw_out, s);
  }
}

// Self-test of the bounded-wait failure path, with no GPU fault: thread 0 waits on an
// mbarrier that nothing arrives at, gives up after `limit` SM cycles, records the timeout
// in the device error word as the pipelines do, and the kernel returns normally.
__global__ void wait_timeout_selftest_kernel(long long limit) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
    if (!mbar_wait_bounded(&bar, 0, limit)) record_timeout();
  }
}

// --------------------------------------------------------------- generic paths -----
template <typename T, typename TW>
__global__ void __launch_bounds__(kGenericThreads)
rmsnorm_fwd_generic(const T* x, int64_t xs, const TW* __restrict__ w, T* __restrict__ y,
                    int64_t ys, float* __restrict__ rstd, int64_t rows, int hidden, float eps,
                    const T* aux, int64_t as, T* h_out, int64_t hs) {
  // With aux (fused residual add) the normalized row is h = x + aux, rounded to T and
  // written to h_out (which may be x itself: every element is read, then written, by the
  // same thread) and read back from there.
  __shared__ float red[2][32];
  int p = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * xs;
    T* hr = aux != nullptr ? h_out + row * hs : nullptr;
    float ss = 0.0f;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
      float f = to_float(xr[c]);
      if (aux != nullptr) {
        const T h = from_float<T>(f + to_float(aux[row * as + c]));
        hr[c] = h;
        f = to_float(h);
      }
      ss = fmaf(f, f, ss);
    }
    const float inv = rsqrtf(block_sum_nosync(ss, red[p]) / (float)hidden + eps);
    T* yr = y + row * ys;
    const T* src = aux != nullptr ? hr : xr;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x)
      yr[c] = from_float<T>((to_float(src[c]) * inv) * to_float(w[c]));
    if (rstd != nullptr && threadIdx.x == 0) rstd[row] = inv;
    p ^= 1;
  }
}

template <typename T, typename TW>
__global__ void __launch_bounds__(kGenericThreads)
rmsnorm_bwd_generic(const T* __restrict__ dy, int64_t dys, const T* __restrict__ x, int64_t xs,
                    const TW* __restrict__ w, const float* __restrict__ rstd,
                    T* dx, int64_t dxs, float* __restrict__ partials,
                    float* __restrict__ partials_lo, float* __restrict__ zero_row, int64_t rows,
                    int hidden, float eps, const T* aux, int64_t as) {
  __shared__ float red[4][32];
  // Each thread only ever touches the partial columns c = threadIdx.x + k * blockDim.x of
  // this CTA's partial rows, so no barrier is needed around the accumulation. The sums
  // (prow) and their Sum2 errors (lrow) accumulate in place; without an error row they are
  // folded together at the end.
  float* prow = partials + (int64_t)blockIdx.x * hidden;
  float* lrow = partials_lo != nullptr ? partials_lo + (int64_t)blockIdx.x * hidden : nullptr;
  for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
    prow[c] = 0.0f;
    if (lrow != nullptr) lrow[c] = 0.0f;
  }
  if (zero_row != nullptr && blockIdx.x == 0)
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) zero_row[c] = 0.0f;
  float* erow = lrow;
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
    double invd;
    if (rstd != nullptr) {
      invd = (double)rstd[row];
    } else {
      invd = rsqrt_refined((double)block_sum_nosync(ss, red[2 * p]) / (double)hidden +
                           (double)eps);
    }
    const float inv = (float)invd;
    const float inv_lo = (float)(invd - (double)inv);
    const float dot_mean = block_sum_nosync(dot, red[2 * p + 1]) / (float)hidden;
    const float cc = (inv * inv) * dot_mean;
    T* dr = dx + row * dxs;
    for (int c = threadIdx.x; c < hidden; c += blockDim.x) {
      const float fx = to_float(xr[c]);
      const float fg = to_float(gr[c]);
      float d = inv * (fg * to_float(w[c]) - fx * cc);
      if (aux != nullptr) d += to_float(aux[row * as + c]);  // may alias dr[c]: read first
      dr[c] = from_float<T>(d);
      const float pxy = __fmul_rn(fg, fx);
      const float t = __fmul_rn(pxy, inv);
      // Low-order parts: the rounding of p * inv, p * inv_lo and (fp32 inputs) of dy * x.
      float lo = fmaf(pxy, inv_lo, fmaf(pxy, inv, -t));
      if (sizeof(T) == 4) lo = fmaf(fmaf(fg, fx, -pxy), inv, lo);
      float sum = prow[c], err = erow != nullptr ? erow[c] : 0.0f;
      sum2_add(sum, err, t);
      err = __fadd_rn(err, lo);
      prow[c] = sum;
      if (erow != nullptr) erow[c] = err;
      else prow[c] = __fadd_rn(sum, err);
    }
    p ^= 1;
  }
}

constexpr int kReduceThreads = kReduceItems;  // one (column, group) item per thread

template <typename TW>
__global__ void __launch_bounds__(kReduceThreads)
rmsnorm_dw_reduce_kernel(const float* __restrict__ partials, int num_partials, int64_t hidden,
                         TW* __restrict__ dw) {
  // One 16-column chunk per CTA (64-byte half-warp loads); dw_reduce_chunk fixes the order.
  __shared__ double s[kReduceCols][kReduceGroups + 1];
  // Launched with programmatic stream serialization: the CTAs may become resident while
  // the previous kernel of the stream (normally the backward that wrote the partials) still
  // runs, and wait here until it has completed and its writes are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The next kernel, when it is a programmatic dependent (the next norm's backward), may be
  // scheduled from now on.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  dw_reduce_chunk<TW, 1>(partials, num_partials, hidden, blockIdx.x, dw, s);
}

// Launches rmsnorm_dw_reduce_kernel as a programmatic dependent of the stream's previous
// kernel (A/B on B200: the backward + reduce pair 1.1 us faster at 16384 x 4096 bf16).
template <typename TW>
cudaError_t launch_dw_reduce(const float* partials, int num_partials, int64_t hidden, TW* dw,
                             cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((hidden + kReduceCols - 1) / kReduceCols));
  cfg.blockDim = dim3((unsigned)kReduceThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rmsnorm_dw_reduce_kernel<TW>, partials, num_partials, hidden,
                            dw);
}

// ------------------------------------------------------------------ host helpers ---

// Resident CTAs per SM for a kernel at a block size and dynamic shared memory; cached.
// On first use of a kernel, raises its dynamic shared memory limit to everything the
// device allows beside the kernel's static shared memory (one fixed value per kernel, so
// launches of any smaller size stay valid). Returns 0 when the kernel cannot run with
// `smem` bytes.
int blocks_per_sm(const void* func, int threads, int smem) {
  static std::mutex mu;
  static std::unordered_map<uint64_t, int> cache;
  static std::unordered_map<uint64_t, int> limit;  // (func, device) -> max dynamic smem
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t fkey = (reinterpret_cast<uint64_t>(func) * 1315423911ull) ^ (uint64_t)dev;
  const uint64_t key = fkey ^ ((uint64_t)threads << 40) ^ ((uint64_t)smem << 8);
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  auto lt = limit.find(fkey);
  if (lt == limit.end()) {
    int optin = 0;
    cudaFuncAttributes attr;
    int max_dyn = 48 * 1024;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) ==
            cudaSuccess &&
        cudaFuncGetAttributes(&attr, func) == cudaSuccess) {
      const int want = optin - (int)attr.sharedSizeBytes;
      if (want > max_dyn &&
          cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, want) ==
              cudaSuccess)
        max_dyn = want;
    }
    cudaGetLastError();
    lt = limit.emplace(fkey, max_dyn).first;
  }
  int n = 0;
  if (smem <= lt->second &&
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, threads, smem) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

struct FastPlan {
  bool ok = false;
  int vpt = 0;        // vectors per owner thread (template parameter)
  int consumers = 0;  // owner warps
  int reducers = 0;   // reducer warps
  int nvec = 0;
  int stages = 0;
  int smem = 0;
};

// Largest vectors-per-thread built for a direction: kElemsFwd / kElemsBwd elements per
// owner thread. Smaller rows use half or a quarter of it (at least 1 vector).
template <typename T, bool kBwd> constexpr int vpt_max() {
  return (kBwd ? kElemsBwd : kElemsFwd) / Vec16<T>::N > 0
             ? (kBwd ? kElemsBwd : kElemsFwd) / Vec16<T>::N
             : 1;
}
template <typename T, bool kBwd> constexpr int vpt_half() {
  return vpt_max<T, kBwd>() / 2 > 0 ? vpt_max<T, kBwd>() / 2 : 1;
}
template <typename T, bool kBwd> constexpr int vpt_quarter() {
  return vpt_max<T, kBwd>() / 4 > 0 ? vpt_max<T, kBwd>() / 4 : 1;
}

// Owner layout and ring depth: the fewest owner warps that give each thread at most
// kElemsPerThread elements, the smallest built vectors-per-thread that covers the row
// with them, and a ring of as many slots as fit in the forward or backward budget (at
// least kMinStages, a multiple of the reducer count). ok=false when the row needs the
// generic path.
template <typename T, bool kBwd, bool kAdd = false>
FastPlan plan_fast(int64_t hidden) {
  FastPlan plan;
  constexpr int V = Vec16<T>::N;
  if (hidden <= 0 || hidden % V != 0) return plan;
  const int64_t nvec = hidden / V;
  const int64_t slot_bytes = nvec * 16 * ((kBwd ? 2 : 1) + (kAdd ? 1 : 0));
  if (slot_bytes > kMaxSlotBytes) return plan;
  const int vmax = vpt_max<T, kBwd>();
  const int64_t consumers = (nvec + 32 * vmax - 1) / (32 * vmax);
  if (consumers > kMaxConsumers) return plan;
  const int64_t need = (nvec + 32 * consumers - 1) / (32 * consumers);
  int vpt = vmax;
  if (consumers <= kSmallConsumers(kBwd)) {
    if (need <= vpt_quarter<T, kBwd>()) {
      vpt = vpt_quarter<T, kBwd>();
    } else if (need <= vpt_half<T, kBwd>()) {
      vpt = vpt_half<T, kBwd>();
    }
  }
  plan.vpt = vpt;
  plan.consumers = (int)consumers;
  plan.nvec = (int)nvec;
  // stages must be a multiple of the reducer count: then each slot is served by exactly
  // one reducer, which visits it in row order, so no waiter can reach a slot's barrier two
  // phases early (try_wait.parity cannot tell use k from use k - 2).
  constexpr bool k16 = sizeof(T) == 2;
  int reducers = kReducers;
  int64_t budget = (int64_t)(kBwd ? kSmemBwd : kSmemFwd) * (kAdd ? 3 : 2) / 2;
  if (kBwd && k16 && !kAdd) {
    reducers = kReducersBwd16;
    budget = kSmemBwd16;
  } else if (kBwd && k16 && kAdd) {
    reducers = kReducersAddBwd16;
    budget = PT_RMS_SMEM_ADDBWD16;
  } else if (!kBwd && k16) {
    reducers = kReducersFwd;
    budget = (int64_t)PT_RMS_SMEM_FWD16 * (kAdd ? 3 : 2) / 2;
  }
  int stages = (int)std::min<int64_t>(kMaxStages, budget / slot_bytes);
  stages = std::max(stages, kMinStages);
  stages = std::max(reducers, stages / reducers * reducers);
  plan.stages = stages;
  plan.reducers = reducers;
  plan.smem = (int)(stages * slot_bytes + (kBwd ? nvec * V * 4 : 0));
  plan.ok = true;
  return plan;
}

template <typename T>
bool rows_aligned(const void* p, int64_t stride) {
  return aligned16(p) && ((stride * (int64_t)sizeof(T)) % 16 == 0);
}

// Kernel instance for a plan: CTAs of up to kSmallConsumers consumer warps (rows of up to
// 4 * 32 * kElemsPerThread elements) use any of the three vectors-per-thread shapes under
// a 5-warp launch bound; bigger CTAs use the full shape under a 17-warp bound.
#define PT_WS(VPT_, MAXW_) rmsnorm_ws<T, TW, VPT_, kBwd, kHasRstd, kAdd, MAXW_, kFused>
template <bool kBwd> constexpr int small_warps() { return kSmallConsumers(kBwd) + kReducers + 1; }
constexpr int kBigWarps = kMaxConsumers + kReducers + 1;
inline int ws_threads(const FastPlan& plan) {
  return (plan.consumers + plan.reducers + 1) * 32;
}
// Dynamic shared memory of a launch: the ring and staged weight, and for the fused
// backward at least the dweight reduction's scratch, which reuses the ring.
constexpr int kReduceSmem = (int)sizeof(double) * kReduceCols * (kReduceGroups + 1);
inline int ws_smem(const FastPlan& plan, bool fused) {
  return fused ? std::max(plan.smem, kReduceSmem) : plan.smem;
}
template <typename T, typename TW, bool kBwd, bool kHasRstd, bool kAdd = false,
          bool kFused = false>
const void* ws_kernel(const FastPlan& plan) {
  constexpr int SW = small_warps<kBwd>();
  if (plan.consumers > kSmallConsumers(kBwd))
    return (const void*)PT_WS((vpt_max<T, kBwd>()), kBigWarps);
  if (plan.vpt == vpt_max<T, kBwd>()) return (const void*)PT_WS((vpt_max<T, kBwd>()), SW);
  if (plan.vpt == vpt_half<T, kBwd>()) return (const void*)PT_WS((vpt_half<T, kBwd>()), SW);
  return (const void*)PT_WS((vpt_quarter<T, kBwd>()), SW);
}

// Launches the plan's instance on `stream`; kFused launches are cooperative (all CTAs
// resident at once, which the grid barrier of the fused dweight needs: `grid` must not
// exceed the resident CTAs of the kernel).
template <typename T, typename TW, bool kBwd, bool kHasRstd, bool kAdd = false,
          bool kFused = false>
cudaError_t ws_launch(const FastPlan& plan, int grid, cudaStream_t stream, const T* x, int64_t xs,
                      const T* dy, int64_t dys, const TW* w, const float* rstd_in, T* out,
                      int64_t os, float* rstd_out, float* partials, float* partials_lo,
                      float* zero_row, int64_t rows, int hidden, float eps,
                      const T* aux = nullptr, int64_t as = 0, T* h_out = nullptr, int64_t hs = 0,
                      unsigned int* grid_bar = nullptr, TW* dw_out = nullptr,
                      int num_partials = 0) {
  constexpr int SW = small_warps<kBwd>();
  const float hf = (float)hidden;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3((unsigned)ws_threads(plan));
  cfg.dynamicSmemBytes = (size_t)ws_smem(plan, kFused);
  cfg.stream = stream;
  // The fused backward needs all CTAs resident (cooperative); the forward and the two-launch
  // backward are programmatic dependents of the previous kernel (A/B on B200 at 16384 x 4096
  // bf16, back to back: backward 68.4 against 70.8 us, forward 44.1 against 46.0 us; the
  // config-5 step 0.5 % shorter; same bits).
  cudaLaunchAttribute attr[1];
  if (kFused) {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  } else {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
#define PT_WS_ARGS                                                                         \
  x, xs, dy, dys, w, rstd_in, out, os, rstd_out, partials, partials_lo, zero_row, aux, as,  \
      h_out, hs, rows, plan.nvec, hidden, plan.stages, plan.consumers, plan.reducers, hf, eps, \
      grid_bar, dw_out, num_partials
  if (plan.consumers > kSmallConsumers(kBwd))
    return cudaLaunchKernelEx(&cfg, PT_WS((vpt_max<T, kBwd>()), kBigWarps), PT_WS_ARGS);
  if (plan.vpt == vpt_max<T, kBwd>())
    return cudaLaunchKernelEx(&cfg, PT_WS((vpt_max<T, kBwd>()), SW), PT_WS_ARGS);
  if (plan.vpt == vpt_half<T, kBwd>())
    return cudaLaunchKernelEx(&cfg, PT_WS((vpt_half<T, kBwd>()), SW), PT_WS_ARGS);
  return cudaLaunchKernelEx(&cfg, PT_WS((vpt_quarter<T, kBwd>()), SW), PT_WS_ARGS);
#undef PT_WS_ARGS
}
#undef PT_WS

// kAdd: fused residual add (aux = the branch output, h_out = x + aux); see rmsnorm_ws.
template <typename T, typename TW, bool kAdd = false>
int fwd_impl(const void* x_, int64_t xs, const void* w_, void* y_, int64_t ys, float* rstd,
             int64_t rows, int64_t hidden, float eps, cudaStream_t stream,
             const void* aux_ = nullptr, int64_t as = 0, void* h_out_ = nullptr, int64_t hs = 0) {
  const T* x = static_cast<const T*>(x_);
  const TW* w = static_cast<const TW*>(w_);
  T* y = static_cast<T*>(y_);
  const T* aux = static_cast<const T*>(aux_);
  T* h_out = static_cast<T*>(h_out_);
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  FastPlan plan = plan_fast<T, false, kAdd>(hidden);
  bool fast = plan.ok && rows_aligned<T>(x, xs) && rows_aligned<T>(y, ys) && aligned16(w);
  if (kAdd) fast = fast && rows_aligned<T>(aux, as) && rows_aligned<T>(h_out, hs);
  int occ = 0;
  if (fast) {
    occ = blocks_per_sm(ws_kernel<T, TW, false, false, kAdd>(plan), ws_threads(plan),
                        plan.smem);
    fast = occ > 0;
  }
  const char* what = kAdd ? "pt_add_rmsnorm_fwd" : "pt_rmsnorm_fwd";
  if (fast) {
    const int64_t resident = (int64_t)sms * occ;
    const int grid = (int)(rows < resident ? rows : resident);
    ws_launch<T, TW, false, false, kAdd>(plan, grid, stream, x, xs, nullptr, 0, w, nullptr, y,
                                         ys, rstd, nullptr, nullptr, nullptr, rows, (int)hidden,
                                         eps, aux, as, h_out, hs);
  } else {
    const void* fn = (const void*)rmsnorm_fwd_generic<T, TW>;
    const int64_t resident = (int64_t)sms * std::max(1, blocks_per_sm(fn, kGenericThreads, 0));
    const int grid = (int)(rows < resident ? rows : resident);
    rmsnorm_fwd_generic<T, TW><<<grid, kGenericThreads, 0, stream>>>(
        x, xs, w, y, ys, rstd, rows, (int)hidden, eps, aux, as, h_out, hs);
  }
  return check_launch(what);
}

template <typename T, typename TW, bool kAdd = false>
int num_partials_impl(int64_t rows, int64_t hidden, int* out) {
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  FastPlan plan = plan_fast<T, true, kAdd>(hidden);
  int occ = 0;
  if (plan.ok) {
    // The fused backward launches one CTA per pair of partial rows, all resident at once:
    // take the smaller occupancy of the two instances so that both can use this count.
    occ = std::min(blocks_per_sm(ws_kernel<T, TW, true, false, kAdd>(plan), ws_threads(plan),
                                 plan.smem),
                   blocks_per_sm(ws_kernel<T, TW, true, false, kAdd, true>(plan),
                                 ws_threads(plan), ws_smem(plan, true)));
  }
  int64_t n;
  if (occ > 0) {
    n = (int64_t)sms * occ;
  } else {
    n = (int64_t)sms *
        std::max(1, blocks_per_sm((const void*)rmsnorm_bwd_generic<T, TW>, kGenericThreads, 0));
  }
  if (rows < n) n = rows;
  if (n < 1) n = 1;
  *out = (int)(2 * n);  // a sum row and an error row per CTA
  return ok();
}

// How the backward lays its CTAs over a caller's [num_partials, hidden] partial buffer:
// CTA b writes its running sums to row b and their accumulated errors to row G + b
// (G = num_partials / 2 CTAs); an odd last row is zeroed. A single row holds one CTA's
// rounded total.
struct PartialLayout {
  int grid;
  float* lo;
  float* zero_row;
};
PartialLayout partial_layout(float* partials, int num_partials, int64_t hidden) {
  if (num_partials < 2) return {1, nullptr, nullptr};
  const int g = num_partials / 2;
  return {g, partials + (int64_t)g * hidden,
          (num_partials & 1) ? partials + (int64_t)2 * g * hidden : nullptr};
}

// kAdd: dx also receives aux (the gradient reaching h through the residual stream).
template <typename T, typename TW, bool kAdd = false>
int bwd_impl(const void* dy_, int64_t dys, const void* x_, int64_t xs, const void* w_,
             const float* rstd, void* dx_, int64_t dxs, float* partials, int num_partials,
             int64_t rows, int64_t hidden, float eps, cudaStream_t stream,
             const void* aux_ = nullptr, int64_t as = 0) {
  const T* dy = static_cast<const T*>(dy_);
  const T* x = static_cast<const T*>(x_);
  const TW* w = static_cast<const TW*>(w_);
  T* dx = static_cast<T*>(dx_);
  const T* aux = static_cast<const T*>(aux_);
  FastPlan plan = plan_fast<T, true, kAdd>(hidden);
  bool fast = plan.ok && rows_aligned<T>(x, xs) && rows_aligned<T>(dy, dys) &&
              rows_aligned<T>(dx, dxs) && aligned16(w) && aligned16(partials);
  if (kAdd) fast = fast && rows_aligned<T>(aux, as);
  const bool hr = rstd != nullptr;
  if (fast) {
    const void* fn = hr ? ws_kernel<T, TW, true, true, kAdd>(plan)
                        : ws_kernel<T, TW, true, false, kAdd>(plan);
    fast = blocks_per_sm(fn, ws_threads(plan), plan.smem) > 0;
  }
  const PartialLayout lay = partial_layout(partials, num_partials, hidden);
  if (fast) {
    if (hr)
      ws_launch<T, TW, true, true, kAdd>(plan, lay.grid, stream, x, xs, dy, dys, w, rstd, dx,
                                         dxs, nullptr, partials, lay.lo, lay.zero_row, rows,
                                         (int)hidden, eps, aux, as);
    else
      ws_launch<T, TW, true, false, kAdd>(plan, lay.grid, stream, x, xs, dy, dys, w, nullptr, dx,
                                          dxs, nullptr, partials, lay.lo, lay.zero_row, rows,
                                          (int)hidden, eps, aux, as);
  } else {
    rmsnorm_bwd_generic<T, TW><<<lay.grid, kGenericThreads, 0, stream>>>(
        dy, dys, x, xs, w, rstd, dx, dxs, partials, lay.lo, lay.zero_row, rows, (int)hidden,
        eps, aux, as);
  }
  return check_launch(kAdd ? "pt_add_rmsnorm_bwd" : "pt_rmsnorm_bwd");
}

// Workspace of the fused backward (pt_rmsnorm_bwd_fused): a 256-byte header whose first
// word is the grid barrier, then num_partials rows of hidden floats.
constexpr int64_t kWsHeaderFloats = 64;

template <typename T, typename TW, bool kAdd = false>
int fused_workspace_impl(int64_t rows, int64_t hidden, int64_t* floats) {
  int P = 0;
  if (int st = num_partials_impl<T, TW, kAdd>(rows, hidden, &P)) return st;
  *floats = kWsHeaderFloats + (int64_t)P * hidden;
  return ok();
}

// dx and dw in one cooperative launch of the pipeline (its CTAs reduce the dweight
// partials among themselves after a grid barrier), for the same partial count
// (num_partials_impl) and the same summation order as bwd_impl + pt_rmsnorm_dw_reduce, so
// the results are bit-identical to that pair. Rows the pipeline cannot take (misaligned,
// hidden not a multiple of 16 bytes) run the generic kernel and the reduce kernel instead.
template <typename T, typename TW, bool kAdd = false>
int fused_bwd_impl(const void* dy_, int64_t dys, const void* x_, int64_t xs, const void* w_,
                   const float* rstd, void* dx_, int64_t dxs, void* dw_, float* ws,
                   int64_t ws_floats, int64_t rows, int64_t hidden, float eps,
                   cudaStream_t stream, const void* aux_ = nullptr, int64_t as = 0) {
  const char* what = kAdd ? "pt_add_rmsnorm_bwd_fused" : "pt_rmsnorm_bwd_fused";
  const T* dy = static_cast<const T*>(dy_);
  const T* x = static_cast<const T*>(x_);
  const TW* w = static_cast<const TW*>(w_);
  T* dx = static_cast<T*>(dx_);
  TW* dw = static_cast<TW*>(dw_);
  const T* aux = static_cast<const T*>(aux_);
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  int P = 0;
  if (int st = num_partials_impl<T, TW, kAdd>(rows, hidden, &P)) return st;
  const int64_t need = kWsHeaderFloats + (int64_t)P * hidden;
  if (ws_floats < need)
    return set_error(PT_ERR_SHAPE, "%s: workspace of %lld floats is smaller than the %lld this "
                     "call needs", what, (long long)ws_floats, (long long)need);
  unsigned int* bar = reinterpret_cast<unsigned int*>(ws);
  float* partials = ws + kWsHeaderFloats;
  FastPlan plan = plan_fast<T, true, kAdd>(hidden);
  bool fast = plan.ok && rows_aligned<T>(x, xs) && rows_aligned<T>(dy, dys) &&
              rows_aligned<T>(dx, dxs) && aligned16(w) && aligned16(partials);
  if (kAdd) fast = fast && rows_aligned<T>(aux, as);
  const bool hr = rstd != nullptr;
  const PartialLayout lay = partial_layout(partials, P, hidden);
  if (fast) {
    const void* fn = hr ? ws_kernel<T, TW, true, true, kAdd, true>(plan)
                        : ws_kernel<T, TW, true, false, kAdd, true>(plan);
    fast = (int64_t)sms * blocks_per_sm(fn, ws_threads(plan), ws_smem(plan, true)) >= lay.grid;
  }
  if (fast) {
    const cudaError_t e =
        hr ? ws_launch<T, TW, true, true, kAdd, true>(
                 plan, lay.grid, stream, x, xs, dy, dys, w, rstd, dx, dxs, nullptr, partials,
                 lay.lo, lay.zero_row, rows, (int)hidden, eps, aux, as, nullptr, 0, bar, dw, P)
           : ws_launch<T, TW, true, false, kAdd, true>(
                 plan, lay.grid, stream, x, xs, dy, dys, w, nullptr, dx, dxs, nullptr, partials,
                 lay.lo, lay.zero_row, rows, (int)hidden, eps, aux, as, nullptr, 0, bar, dw, P);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(PT_ERR_CUDA, "%s: cooperative launch failed: %s", what,
                       cudaGetErrorString(e));
    }
    return check_launch(what);
  }
  rmsnorm_bwd_generic<T, TW><<<lay.grid, kGenericThreads, 0, stream>>>(
      dy, dys, x, xs, w, rstd, dx, dxs, partials, lay.lo, lay.zero_row, rows, (int)hidden, eps,
      aux, as);
  if (int st = check_launch(what)) return st;
  if (cudaError_t e = launch_dw_reduce<TW>(partials, P, hidden, dw, stream)) {
    cudaGetLastError();
    return set_error(PT_ERR_CUDA, "%s: dweight reduce launch failed: %s", what,
                     cudaGetErrorString(e));
  }
  return check_launch(what);
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

int pt_rmsnorm_bwd_fused_workspace(int64_t rows, int64_t hidden, int x_dtype, int w_dtype,
                                   int64_t* floats) {
  if (floats == nullptr) return set_error(PT_ERR_INVALID_ARGUMENT, "floats is NULL");
  if (int st = check_shape(rows, hidden)) return st;
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return fused_workspace_impl<T, TW>(rows, hidden, floats);
  });
}

int pt_rmsnorm_bwd_fused(const void* dy, int64_t dy_row_stride, const void* x,
                         int64_t x_row_stride, const void* weight, const float* rstd, void* dx,
                         int64_t dx_row_stride, void* dw, float* workspace,
                         int64_t workspace_floats, int64_t rows, int64_t hidden, int x_dtype,
                         int w_dtype, float eps, void* stream) {
  if (int st = check_shape(rows, hidden)) return st;
  if (!(eps >= 0.0f)) return set_error(PT_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (int st = check_device_ptr(weight, "weight")) return st;
  if (int st = check_device_ptr(dw, "dw")) return st;
  if (int st = check_device_ptr(workspace, "workspace")) return st;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error(PT_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
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
    return fused_bwd_impl<T, TW>(dy, dy_row_stride, x, x_row_stride, weight, rstd, dx,
                                 dx_row_stride, dw, workspace, workspace_floats, rows, hidden,
                                 eps, as_stream(stream));
  });
}

int pt_add_rmsnorm_fwd(const void* residual, int64_t residual_row_stride, const void* branch,
                       int64_t branch_row_stride, const void* weight, void* h_out,
                       int64_t h_row_stride, void* y, int64_t y_row_stride, float* rstd,
                       int64_t rows, int64_t hidden, int x_dtype, int w_dtype, float eps,
                       void* stream) {
  if (int st = check_shape(rows, hidden)) return st;
  if (!(eps >= 0.0f)) return set_error(PT_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (rows == 0) return ok();
  if (int st = check_row_stride(residual_row_stride, hidden, "residual_row_stride")) return st;
  if (int st = check_row_stride(branch_row_stride, hidden, "branch_row_stride")) return st;
  if (int st = check_row_stride(h_row_stride, hidden, "h_row_stride")) return st;
  if (int st = check_row_stride(y_row_stride, hidden, "y_row_stride")) return st;
  if (int st = check_device_ptr(residual, "residual")) return st;
  if (int st = check_device_ptr(branch, "branch")) return st;
  if (int st = check_device_ptr(weight, "weight")) return st;
  if (int st = check_device_ptr(h_out, "h_out")) return st;
  if (int st = check_device_ptr(y, "y")) return st;
  if (rstd)
    if (int st = check_device_ptr(rstd, "rstd")) return st;
  if (h_out == branch || y == residual || y == branch || y == h_out)
    return set_error(PT_ERR_INVALID_ARGUMENT,
                     "h_out may alias residual only; y must not alias any other buffer");
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return fwd_impl<T, TW, true>(residual, residual_row_stride, weight, y, y_row_stride, rstd,
                                 rows, hidden, eps, as_stream(stream), branch, branch_row_stride,
                                 h_out, h_row_stride);
  });
}

int pt_add_rmsnorm_bwd_num_partials(int64_t rows, int64_t hidden, int x_dtype, int w_dtype,
                                    int* num_partials) {
  if (num_partials == nullptr)
    return set_error(PT_ERR_INVALID_ARGUMENT, "num_partials is NULL");
  if (int st = check_shape(rows, hidden)) return st;
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return num_partials_impl<T, TW, true>(rows, hidden, num_partials);
  });
}

int pt_add_rmsnorm_bwd(const void* dy, int64_t dy_row_stride, const void* dh,
                       int64_t dh_row_stride, const void* h, int64_t h_row_stride,
                       const void* weight, const float* rstd, void* dx, int64_t dx_row_stride,
                       float* dw_partials, int num_partials, int64_t rows, int64_t hidden,
                       int x_dtype, int w_dtype, float eps, void* stream) {
  if (dh == nullptr)
    return pt_rmsnorm_bwd(dy, dy_row_stride, h, h_row_stride, weight, rstd, dx, dx_row_stride,
                          dw_partials, num_partials, rows, hidden, x_dtype, w_dtype, eps,
                          stream);
  if (int st = check_shape(rows, hidden)) return st;
  if (!(eps >= 0.0f)) return set_error(PT_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (num_partials < 1)
    return set_error(PT_ERR_INVALID_ARGUMENT, "num_partials must be >= 1 (got %d)", num_partials);
  if (int st = check_device_ptr(dw_partials, "dw_partials")) return st;
  if (int st = check_device_ptr(weight, "weight")) return st;
  if (rows > 0) {
    if (int st = check_row_stride(dy_row_stride, hidden, "dy_row_stride")) return st;
    if (int st = check_row_stride(dh_row_stride, hidden, "dh_row_stride")) return st;
    if (int st = check_row_stride(h_row_stride, hidden, "h_row_stride")) return st;
    if (int st = check_row_stride(dx_row_stride, hidden, "dx_row_stride")) return st;
    if (int st = check_device_ptr(dy, "dy")) return st;
    if (int st = check_device_ptr(dh, "dh")) return st;
    if (int st = check_device_ptr(h, "h")) return st;
    if (int st = check_device_ptr(dx, "dx")) return st;
    if (rstd)
      if (int st = check_device_ptr(rstd, "rstd")) return st;
    if (dx == dy || dx == h)
      return set_error(PT_ERR_INVALID_ARGUMENT, "dx may alias dh only");
  }
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return bwd_impl<T, TW, true>(dy, dy_row_stride, h, h_row_stride, weight, rstd, dx,
                                 dx_row_stride, dw_partials, num_partials, rows, hidden, eps,
                                 as_stream(stream), dh, dh_row_stride);
  });
}

int pt_add_rmsnorm_bwd_fused_workspace(int64_t rows, int64_t hidden, int x_dtype, int w_dtype,
                                       int64_t* floats) {
  if (floats == nullptr) return set_error(PT_ERR_INVALID_ARGUMENT, "floats is NULL");
  if (int st = check_shape(rows, hidden)) return st;
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return fused_workspace_impl<T, TW, true>(rows, hidden, floats);
  });
}

int pt_add_rmsnorm_bwd_fused(const void* dy, int64_t dy_row_stride, const void* dh,
                             int64_t dh_row_stride, const void* h, int64_t h_row_stride,
                             const void* weight, const float* rstd, void* dx,
                             int64_t dx_row_stride, void* dw, float* workspace,
                             int64_t workspace_floats, int64_t rows, int64_t hidden,
                             int x_dtype, int w_dtype, float eps, void* stream) {
  if (dh == nullptr)
    return pt_rmsnorm_bwd_fused(dy, dy_row_stride, h, h_row_stride, weight, rstd, dx,
                                dx_row_stride, dw, workspace, workspace_floats, rows, hidden,
                                x_dtype, w_dtype, eps, stream);
  if (int st = check_shape(rows, hidden)) return st;
  if (!(eps >= 0.0f)) return set_error(PT_ERR_INVALID_ARGUMENT, "eps must be >= 0");
  if (int st = check_device_ptr(weight, "weight")) return st;
  if (int st = check_device_ptr(dw, "dw")) return st;
  if (int st = check_device_ptr(workspace, "workspace")) return st;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return set_error(PT_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  if (rows > 0) {
    if (int st = check_row_stride(dy_row_stride, hidden, "dy_row_stride")) return st;
    if (int st = check_row_stride(dh_row_stride, hidden, "dh_row_stride")) return st;
    if (int st = check_row_stride(h_row_stride, hidden, "h_row_stride")) return st;
    if (int st = check_row_stride(dx_row_stride, hidden, "dx_row_stride")) return st;
    if (int st = check_device_ptr(dy, "dy")) return st;
    if (int st = check_device_ptr(dh, "dh")) return st;
    if (int st = check_device_ptr(h, "h")) return st;
    if (int st = check_device_ptr(dx, "dx")) return st;
    if (rstd)
      if (int st = check_device_ptr(rstd, "rstd")) return st;
    if (dx == dy || dx == h)
      return set_error(PT_ERR_INVALID_ARGUMENT, "dx may alias dh only");
  }
  return dispatch_xw(x_dtype, w_dtype, [&](auto* tx, auto* tw) {
    using T = std::remove_pointer_t<decltype(tx)>;
    using TW = std::remove_pointer_t<decltype(tw)>;
    return fused_bwd_impl<T, TW, true>(dy, dy_row_stride, h, h_row_stride, weight, rstd, dx,
                                       dx_row_stride, dw, workspace, workspace_floats, rows,
                                       hidden, eps, as_stream(stream), dh, dh_row_stride);
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
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaSuccess;
  switch (dw_dtype) {
    case PT_FLOAT32:
      e = launch_dw_reduce(dw_partials, num_partials, hidden, static_cast<float*>(dw), s);
      break;
    case PT_FLOAT16:
      e = launch_dw_reduce(dw_partials, num_partials, hidden, static_cast<__half*>(dw), s);
      break;
    case PT_BFLOAT16:
      e = launch_dw_reduce(dw_partials, num_partials, hidden, static_cast<__nv_bfloat16*>(dw), s);
      break;
    default:
      return set_error(PT_ERR_UNSUPPORTED_DTYPE, "unsupported dw_dtype %d", dw_dtype);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_CUDA, "pt_rmsnorm_dw_reduce: launch failed: %s",
                     cudaGetErrorString(e));
  }
  return check_launch("pt_rmsnorm_dw_reduce");
}

// ------------------------------------------------------- allocation-free backward --
// Scratch for pt_rmsnorm_bwd_noalloc: the dweight partials live in this file-scope device
// array (kNoAllocFloats floats = 16 MiB, held by every device that loads the library until
// the process exits): room for the full partial count of a B200 (two rows for each of 296
// CTAs) up to hidden 7085; wider rows run the backward with fewer CTAs. Host code must not
// use the symbol itself as a device address: its address on a device comes from
// cudaGetSymbolAddress, taken once per device and kept for the life of the process (it is
// not looked up again after cudaDeviceReset).
namespace pt {
namespace {
constexpr int64_t kNoAllocFloats = int64_t(1) << 22;
constexpr int kNoAllocMaxDevices = 64;
__device__ __align__(256) float g_noalloc_partials[kNoAllocFloats];
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};

int noalloc_scratch(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_DEVICE, "no current CUDA device");
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(PT_ERR_DEVICE, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return set_error(PT_ERR_CUDA, "cannot get the scratch address on device %d: %s", dev,
                       cudaGetErrorString(e));
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return PT_OK;
}
}  // namespace
}  // namespace pt

int pt_rmsnorm_bwd_noalloc(const void* dy, int64_t dy_row_stride, const void* x,
                           int64_t x_row_stride, const void* weight, const float* rstd, void* dx,
                           int64_t dx_row_stride, void* dw, int64_t rows, int64_t hidden,
                           int x_dtype, int w_dtype, float eps, void* stream) {
  if (int st = check_shape(rows, hidden)) return st;
  if (hidden > kNoAllocFloats)
    return set_error(PT_ERR_SHAPE,
                     "pt_rmsnorm_bwd_noalloc: hidden (%lld) exceeds its scratch of %lld floats; "
                     "use pt_rmsnorm_bwd with a caller-provided dw_partials buffer",
                     (long long)hidden, (long long)kNoAllocFloats);
  if (int st = check_device_ptr(dw, "dw")) return st;
  int num_partials = 0;
  if (int st = pt_rmsnorm_bwd_num_partials(rows, hidden, x_dtype, w_dtype, &num_partials))
    return st;
  const int64_t fit = kNoAllocFloats / hidden;
  if (num_partials > fit) num_partials = (int)fit;
  float* scratch = nullptr;
  if (int st = noalloc_scratch(&scratch)) return st;
  // Every partial row [0, num_partials) is written by the backward before the reduce
  // reads it, so the scratch needs no clearing between calls.
  if (int st = pt_rmsnorm_bwd(dy, dy_row_stride, x, x_row_stride, weight, rstd, dx,
                              dx_row_stride, scratch, num_partials, rows, hidden, x_dtype,
                              w_dtype, eps, stream))
    return st;
  return pt_rmsnorm_dw_reduce(scratch, num_partials, hidden, dw, w_dtype, stream);
}

int pt_selftest_wait_timeout(int64_t limit_cycles, void* stream) {
  if (limit_cycles < 1 || limit_cycles > kWaitLimitCycles)
    return set_error(PT_ERR_INVALID_ARGUMENT, "limit_cycles must be in [1, %lld] (got %lld)",
                     kWaitLimitCycles, (long long)limit_cycles);
  int dev = 0, sms = 0;
  if (int st = current_device_info(&dev, &sms)) return st;
  wait_timeout_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>((long long)limit_cycles);
  return check_launch("pt_selftest_wait_timeout");
}

int pt_take_device_error(int* code) {
  if (code == nullptr) return set_error(PT_ERR_INVALID_ARGUMENT, "code is NULL");
  int value = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&value, g_device_error, sizeof(int));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(PT_ERR_CUDA, "cannot read the device error word: %s", cudaGetErrorString(e));
  }
  if (value != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (e != cudaSuccess) {
      cudaGetLastError();
      return set_error(PT_ERR_CUDA, "cannot clear the device error word: %s",
                       cudaGetErrorString(e));
    }
  }
  int gemm_value = 0, ce_value = 0;
  if (int st = take_gemm_device_error(&gemm_value)) return st;
  if (int st = take_ce_device_error(&ce_value)) return st;
  *code = value != 0 ? value : gemm_value != 0 ? gemm_value : ce_value;
  return ok();
}

}  // extern "C"
