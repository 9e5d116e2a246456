// The decoder step's linear layers with their LayerNorm, bias, GELU and residual fused around them -- the reference's
// decoder_kernels.py (ln_linear :138-146 / kernel :42-75, linear_residual :149-157 / kernel :77-97, layer_norm_bias
// :127-135 / kernel :100-115), as the step calls them (runtime.py:134-151):
//   layer_norm_bias: y = LN(x) (fp32 statistics: mean, then the mean square of x - mean; rounded to the input type)
//                    and, in place, x = x + bias;
//   ln_linear:       y = LN(x) . w^T + b (fp32 accumulation), rounded; with GELU, gelu(rounded) in fp32, rounded;
//   linear_residual: y = round(round(x . w^T + b) + res), res and y may be the same tensor.
//
// B200 design. At a decode step the rows (1-320) are few and every GEMM streams its weights once: HBM-bound,
// short, and with too few 128-feature output tiles (10-40) to occupy 148 SMs. So:
//   * one tcgen05 kernel, one unit per CTA: a unit is (row chunk of <= 256, 128-feature tile, k split); the weights
//     are the MMA's A (M = 128 features), the rows its B (N = rows, padded to 16), 64-element k blocks staged by
//     TMA (128-byte swizzle) through a ring; warp 0 issues the loads, warp 1 the MMAs into a tensor-memory
//     accumulator, warps 2-5 the epilogue;
//   * the k range of a tile is split over the CTAs of a thread-block cluster (up to 8, enough to occupy the SMs):
//     each CTA parks its fp32 partial in its own shared memory (the ring, idle once its MMAs are done), and after
//     a cluster barrier each CTA sums its share of the tile's rows over all the cluster's partials through
//     distributed shared memory, in split order (the same sums whichever CTA finishes first), and applies the
//     fused epilogue -- no partial leaves the chip;
//   * the plan: the most splits whose clusters are all resident at once (cudaOccupancyMaxActiveClusters: a cluster
//     of 7 needs 7 SMs of one GPC, so 20 such clusters would run in two waves), and the rows cut into chunks of
//     >= 64 when a cost model fitted to this kernel's measured rates on B200 (a CTA streams its stages at ~75 GB/s;
//     parking and reducing its partial moves ~38 GB/s) says that smaller partials pay for re-reading the weights;
//   * while the MMAs run, the epilogue threads fetch the bias and (residual mode) their CTA's share of the residual
//     rows into shared memory; the accumulator leaves tensor memory 64 columns per wait; the reduction keeps ~32
//     partial loads in flight per thread whatever the split count;
//   * ln_linear first normalizes the rows into the workspace with a row kernel; the GEMM is launched after it with
//     programmatic dependent launch and issues its first stages' weight loads before waiting for it (the weights
//     are not its output), so the weight stream overlaps the LayerNorm;
//   * every mbarrier wait is bounded: a wait that runs out records an error in the workspace's device word and
//     raises a stop flag that every role checks, so no role issues more; every CTA still meets its cluster's
//     barriers, and before it frees its tensor memory the producer waits (bounded) for each copy it issued and the
//     MMA issuer for its MMAs (a final commit).
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

namespace wt {
namespace {

constexpr int kDlEpiWarps = 4;
constexpr int kDlThreads = 32 * (2 + kDlEpiWarps);  // producer, MMA issuer, 4 epilogue warps
constexpr int kDlTileV = 128;    // output features per unit (the MMA's M)
constexpr int kDlKBlock = 64;    // reduction elements per stage (one 128-byte swizzled row)
constexpr int kDlMaxRows = 256;  // rows per unit (the MMA's N, at most 256)
constexpr int kDlMaxSplits = 8;  // CTAs of a cluster (the portable maximum)
constexpr int kDlErrTimeout = 1;

enum DlMode { kDlBias = 0, kDlGelu = 1, kDlResidual = 2 };

struct DlArgs {
  int *err;
  const void *bias;  // [V]
  const void *res;   // [N, V] (residual mode)
  void *y;           // [N, V]
  int N, V, kblocks, splits, kb_per, vtiles, nmma, tcols, stages, ring_bytes, res_bytes;
  uint32_t polls;  // bound of every wait (wt_set_wait_limit)
  int withhold;    // test hook: CTA 0 leaves out the row block of its first stage (wt_set_test_withhold_stage)
};

// nmma: the rows of a unit (a row chunk; the MMA's N, a multiple of 16). res_bytes: a region after the ring that
// receives this CTA's share of the residual rows while the MMAs run (residual mode with k splits).
struct DlPlan {
  int chunks, vtiles, kblocks, splits, kb_per, nmma, tcols, stages, stage_bytes, ring_bytes, res_bytes, smem, grid;
  size_t xn_off, bytes;
};

// The most k splits a GEMM may take: WT_DL_MAX_SPLITS (a tuning knob), else kDlMaxSplits.
int max_splits() {
  static const int v = [] {  // (read once; a function-local static initialises thread-safely)
    const char *e = getenv("WT_DL_MAX_SPLITS");
    const int x = e ? atoi(e) : kDlMaxSplits;
    return (x >= 1 && x <= kDlMaxSplits) ? x : kDlMaxSplits;
  }();
  return v;
}

// Row chunks per 256 rows forced by WT_DL_CHUNKS (a tuning knob, 1-4), else 0 (chosen by the cost model).
int row_chunks() {
  static const int v = [] {
    const char *e = getenv("WT_DL_CHUNKS");
    const int x = e ? atoi(e) : 0;
    return (x >= 1 && x <= 4) ? x : 0;
  }();
  return v;
}

// WT_DL_TRACE=1: print every plan the chooser weighs to stderr (a tuning aid; off by default).
bool trace_plans() {
  static const bool v = [] {
    const char *e = getenv("WT_DL_TRACE");
    return e != nullptr && e[0] == '1';
  }();
  return v;
}

int min_chunks(int N) { return (N + kDlMaxRows - 1) / kDlMaxRows; }
int chunk_rows(int N, int c) { return ((N + c - 1) / c + 15) / 16 * 16; }  // rows per chunk (<= 256)

// `ln`: the plan of ln_linear (a workspace for the normalized rows), else of linear_residual. `c`: row chunks (0:
// the fewest, ceil(N / 256)); at most `smax` k splits.
DlPlan dl_plan(int N, int V, int K, bool ln, int sms, int c = 0, int smax = kDlMaxSplits) {
  DlPlan p{};
  if (c < min_chunks(N)) c = min_chunks(N);
  const int rc = chunk_rows(N, c);
  p.chunks = (N + rc - 1) / rc;
  p.vtiles = (V + kDlTileV - 1) / kDlTileV;
  p.kblocks = (K + kDlKBlock - 1) / kDlKBlock;
  const int tiles = p.chunks * p.vtiles;
  int s = sms / tiles;  // splits: enough CTAs for the SMs, at most a cluster, at least 2 k blocks each
  if (s > kDlMaxSplits) s = kDlMaxSplits;
  if (s > max_splits()) s = max_splits();
  if (s > smax) s = smax;
  if (s > p.kblocks / 2) s = p.kblocks / 2;
  if (s < 1) s = 1;
  p.kb_per = (p.kblocks + s - 1) / s;
  p.splits = (p.kblocks + p.kb_per - 1) / p.kb_per;  // (no empty split)
  p.nmma = rc;
  p.tcols = 32;
  while (p.tcols < p.nmma) p.tcols <<= 1;
  p.stage_bytes = kDlTileV * 128 + (p.nmma * 128 + 1023) / 1024 * 1024;
  // residual mode with k splits: this CTA's share of the rows (at most ceil(nmma / splits)) x 128 features
  p.res_bytes = (!ln && p.splits > 1) ? ((p.nmma + p.splits - 1) / p.splits) * kDlTileV * 2 : 0;
  const int budget = 200 * 1024 - p.res_bytes;
  const int cap = budget / p.stage_bytes < 8 ? budget / p.stage_bytes : 8;
  p.stages = p.kb_per < cap ? p.kb_per : cap;
  p.ring_bytes = p.stages * p.stage_bytes;
  const int part_bytes = p.splits > 1 ? p.nmma * kDlTileV * 4 : 0;  // the partial, parked over the idle ring
  if (p.ring_bytes < part_bytes) p.ring_bytes = part_bytes;
  p.smem = 1024 + p.ring_bytes + p.res_bytes + (2 * p.stages + 2) * 8 + 16;
  p.grid = tiles * p.splits;
  p.xn_off = 256;  // [0, 256): the device error word
  p.bytes = p.xn_off + (ln ? (static_cast<size_t>(N) * K * 2 + 255) / 256 * 256 : 0);
  return p;
}

template <typename T>
__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.f + erff(x * 0.7071067811865476f));
}

// The fused epilogue of one output element from its fp32 sum, its bias b and (residual mode) its residual r.
template <typename T, int MODE>
__device__ __forceinline__ T dl_out(float acc, float b, float r) {
  const T h = Elem<T>::from_float(acc + b);
  if (MODE == kDlBias) return h;
  if (MODE == kDlGelu) return Elem<T>::from_float(gelu_erf<T>(Elem<T>::to_float(h)));
  return Elem<T>::from_float(Elem<T>::to_float(h) + r);
}

template <typename T>
__device__ __forceinline__ float ld_f(const void *p, size_t i) {
  return Elem<T>::to_float(static_cast<const T *>(p)[i]);
}

__device__ __forceinline__ void dl_cp16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void dl_cp_commit_wait() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Four consecutive 16-bit values <-> floats (8 bytes, 8-byte aligned).
template <typename T>
__device__ __forceinline__ void unpack4(uint2 u, float (&f)[4]) {
  const T *h = reinterpret_cast<const T *>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) f[e] = Elem<T>::to_float(h[e]);
}
template <typename T>
__device__ __forceinline__ uint2 pack4(const T (&h)[4]) {
  uint2 u;
  T *o = reinterpret_cast<T *>(&u);
#pragma unroll
  for (int e = 0; e < 4; ++e) o[e] = h[e];
  return u;
}

// One CTA's share of a tile's rows, rows [r0, r1) of the unit: the sum of the cluster's S partials (read from the
// CTAs' shared memory, 16 bytes at a time, in split order: the same sums whichever CTA finished first), then the
// fused epilogue. Thread et (0-127) takes features 4 (et % 32) .. + 3 of rows r0 + et / 32 + 4 i; kR rows per batch
// keep ~32 partial loads in flight. The residual share is already in shared memory (`rsm`, [row - r0][128]).
template <typename T, int MODE, int S>
__device__ __forceinline__ void reduce_share(const DlArgs &a, const float4 *const (&peer)[kDlMaxSplits],
                                             const T *rsm, const float (&bv4)[4], int et, int n0, int r0, int r1,
                                             int v0) {
  constexpr int kR = 32 / S;
  const int f4 = et & 31, rsub = et >> 5;
  const int vv = v0 + 4 * f4;
  T *y = static_cast<T *>(a.y);
  for (int n = r0 + rsub; n < r1; n += 4 * kR) {
    float4 val[kR][S];
#pragma unroll
    for (int q = 0; q < kR; ++q) {
      const int row = n + 4 * q;
#pragma unroll
      for (int s2 = 0; s2 < S; ++s2)
        val[q][s2] = row < r1 ? peer[s2][row * (kDlTileV / 4) + f4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int q = 0; q < kR; ++q) {
      const int row = n + 4 * q;
      if (row >= r1 || vv >= a.V) continue;  // (V % 8 == 0: the 4 features are all in or all out)
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s2 = 0; s2 < S; ++s2) {
        acc[0] += val[q][s2].x;
        acc[1] += val[q][s2].y;
        acc[2] += val[q][s2].z;
        acc[3] += val[q][s2].w;
      }
      float rr[4] = {0.f, 0.f, 0.f, 0.f};
      if (MODE == kDlResidual)
        unpack4<T>(*reinterpret_cast<const uint2 *>(rsm + (row - r0) * kDlTileV + 4 * f4), rr);
      T o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = dl_out<T, MODE>(acc[e], bv4[e], rr[e]);
      *reinterpret_cast<uint2 *>(y + static_cast<size_t>(n0 + row) * a.V + vv) = pack4<T>(o);
    }
  }
}

// One unit per CTA: blockIdx.x = tile * splits + split; the splits of a tile are one cluster (rank = split).
template <typename T, int MODE>
__global__ void __launch_bounds__(kDlThreads)
    dec_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                    const DlArgs a) {
  namespace cg = cooperative_groups;
  constexpr bool kBF16 = Elem<T>::code == WT_BF16;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_bytes = kDlTileV * 128, b_bytes = a.nmma * 128;
  const int stage_bytes = a_bytes + ((b_bytes + 1023) & ~1023);
  const int stages = a.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.ring_bytes + a.res_bytes);
  uint64_t *empty = full + stages;
  uint64_t *acc_full = empty + stages;
  uint64_t *drained = acc_full + 1;  // the MMA issuer's last commit: every MMA it issued has completed
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drained + 1);
  volatile int *stop = reinterpret_cast<volatile int *>(tmem_holder + 1);  // a role's wait ran out
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = a.splits, sp = static_cast<int>(blockIdx.x) % S, t = static_cast<int>(blockIdx.x) / S;
  const int v0 = (t % a.vtiles) * kDlTileV, n0 = (t / a.vtiles) * a.nmma;
  const int nn = min(a.nmma, a.N - n0);
  const int rpc = (nn + S - 1) / S, r0 = sp * rpc, r1 = min(nn, r0 + rpc);  // this CTA's rows of the reduction
  float bv4[4] = {0.f, 0.f, 0.f, 0.f};  // (k splits: the bias of the features an epilogue thread reduces)
  const int kb0 = sp * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per), nkb = kb1 - kb0;

  if (warp == 0) {
    tmem_alloc(tmem_holder, static_cast<uint32_t>(a.tcols));
    tmem_relinquish();
  }
  if (tid == 32) {
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(drained, 1);
    *stop = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {  // producer: this unit's k blocks through the ring
      // the first stages' weight halves go out before the wait for the preceding kernel (it does not write the
      // weights); their row halves (possibly its output) after it
      // (the bounded-wait test hook: CTA 0 leaves out the row block of its first stage, whose barrier then never
      // completes)
      const bool hold = a.withhold && blockIdx.x == 0;
      bool waited = false;
      int i = 0;
      for (; i < nkb; ++i) {
        const int s = i % stages;
        if (i >= stages) {
          if (!waited) {
            pdl_wait();
            pdl_launch_dependents();
            for (int j = 0; j < stages; ++j)
              if (!(hold && j == 0))
                tma_load_2d(smem + j * stage_bytes + a_bytes, &xmap, (kb0 + j) * kDlKBlock, n0, &full[j]);
            waited = true;
          }
          if (!mbar_wait_role(&empty[s], ((i / stages) - 1) & 1, a.err, kDlErrTimeout, a.polls, stop))
            break;  // (nothing more is issued)
        }
        unsigned char *st = smem + s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(a_bytes + b_bytes));
        tma_load_2d(st, &wmap, (kb0 + i) * kDlKBlock, v0, &full[s]);
        if (waited) tma_load_2d(st + a_bytes, &xmap, (kb0 + i) * kDlKBlock, n0, &full[s]);
      }
      if (!waited) {
        pdl_wait();
        pdl_launch_dependents();
        for (int j = 0; j < min(stages, nkb); ++j)
          if (!(hold && j == 0))
            tma_load_2d(smem + j * stage_bytes + a_bytes, &xmap, (kb0 + j) * kDlKBlock, n0, &full[j]);
      }
      // every copy issued has landed before the shared memory is reused or goes away: the last fill of each stage
      // (bounded; at most one outstanding per stage, since a stage is refilled only after its MMAs released it)
      for (int j = i > stages ? i - stages : 0; j < i; ++j)
        mbar_wait_bounded(&full[j % stages], (j / stages) & 1, nullptr, 0, a.polls);
    } else {
      pdl_wait();
      pdl_launch_dependents();
    }
  } else if (warp == 1) {
    pdl_wait();
    pdl_launch_dependents();
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc = idesc_f16(kDlTileV, a.nmma, kBF16);
      bool halt = false;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        if (!mbar_wait_role(&full[s], (i / stages) & 1, a.err, kDlErrTimeout, a.polls, stop)) {
          halt = true;  // (no MMA reads a stage that has not landed)
          break;
        }
        tc_fence_after();
        const uint32_t a_addr = smem_addr(smem + s * stage_bytes), b_addr = a_addr + a_bytes;
        const uint64_t adesc = sw128_desc(a_addr), bdesc = sw128_desc(b_addr);
#pragma unroll
        for (int kk = 0; kk < kDlKBlock / 16; ++kk)  // K = 16 per instruction: +32 bytes along the swizzled row
          umma_f16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i != 0 || kk != 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      if (!halt) umma_commit(&acc_full[0]);
      // every MMA issued has completed before the tensor memory is freed (bounded)
      umma_commit(drained);
      mbar_wait_bounded(drained, 0, nullptr, 0, a.polls);
    }
  } else {  // epilogue warps: lane quarter warp % 4 = features v0 + 32 (warp % 4) + lane
    pdl_wait();
    pdl_launch_dependents();
    const int quarter = warp & 3, et = tid - 64;
    const int v = v0 + quarter * 32 + lane;
    const float bv = (S == 1 && v < a.V) ? ld_f<T>(a.bias, v) : 0.f;
    if (S > 1) {
      // while the MMAs run: the bias of this thread's reduction features and, in residual mode, this CTA's share of
      // the residual rows into shared memory (16-byte copies; out-of-range features are not needed)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int vv = v0 + 4 * (et & 31) + e;
        bv4[e] = vv < a.V ? ld_f<T>(a.bias, vv) : 0.f;
      }
      if (MODE == kDlResidual) {
        unsigned char *rsm = smem + a.ring_bytes;
        for (int c = et; c < (r1 - r0) * (kDlTileV / 8); c += 32 * kDlEpiWarps) {
          const int row = r0 + c / (kDlTileV / 8), col = v0 + (c % (kDlTileV / 8)) * 8;
          if (col < a.V) dl_cp16(rsm + c * 16, static_cast<const T *>(a.res) + static_cast<size_t>(n0 + row) * a.V + col);
        }
      }
    }
    // (the warp decides together: its tensor-memory loads are warp-wide; after a timeout it skips them and still
    // meets the cluster's barriers below)
    const bool have =
        __all_sync(0xffffffffu, mbar_wait_role(&acc_full[0], 0, a.err, kDlErrTimeout, a.polls, stop));
    tc_fence_after();
    const uint32_t base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    T *y = static_cast<T *>(a.y);
    float *part = reinterpret_cast<float *>(smem);  // [row][128 features], over the idle ring
    for (int c0 = 0; have && c0 < a.nmma; c0 += 64) {  // 64 accumulator columns (rows) per tensor-memory wait
      uint32_t r[4][16];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (c0 + 16 * j < a.nmma) tmem_ld16(base + static_cast<uint32_t>(c0 + 16 * j), r[j]);
      tmem_wait_ld();
      if (S == 1) {
        float rs[4][16];  // (every residual of the batch loaded before its stores: y may be the residual itself)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int n = c0 + 16 * j + q;
            rs[j][q] = (MODE == kDlResidual && n < nn && v < a.V) ? ld_f<T>(a.res, static_cast<size_t>(n0 + n) * a.V + v)
                                                                  : 0.f;
          }
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int n = c0 + 16 * j + q;
            if (n < nn && v < a.V)
              y[static_cast<size_t>(n0 + n) * a.V + v] = dl_out<T, MODE>(__uint_as_float(r[j][q]), bv, rs[j][q]);
          }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int n = c0 + 16 * j + q;
            if (n < nn) part[n * kDlTileV + quarter * 32 + lane] = __uint_as_float(r[j][q]);
          }
      }
    }
    if (S > 1 && MODE == kDlResidual) dl_cp_commit_wait();
    tc_fence_before();
  }
  if (S > 1) {
    // This CTA's share of the tile's rows: the sum of the splits' partials through distributed shared memory, then
    // the epilogue (reduce_share).
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every split's partial is in its CTA's shared memory (and the residual share in this one's)
    if (warp >= 2) {
      const float *part = reinterpret_cast<const float *>(smem);
      const float4 *peer[kDlMaxSplits];
#pragma unroll
      for (int s2 = 0; s2 < kDlMaxSplits; ++s2)
        peer[s2] = reinterpret_cast<const float4 *>(cluster.map_shared_rank(part, s2 < S ? s2 : 0));
      const T *rsm = reinterpret_cast<const T *>(smem + a.ring_bytes);
      const int et = tid - 64;
      switch (S) {
        case 2: reduce_share<T, MODE, 2>(a, peer, rsm, bv4, et, n0, r0, r1, v0); break;
        case 3: reduce_share<T, MODE, 3>(a, peer, rsm, bv4, et, n0, r0, r1, v0); break;
        case 4: reduce_share<T, MODE, 4>(a, peer, rsm, bv4, et, n0, r0, r1, v0); break;
        case 5: reduce_share<T, MODE, 5>(a, peer, rsm, bv4, et, n0, r0, r1, v0); break;
        case 6: reduce_share<T, MODE, 6>(a, peer, rsm, bv4, et, n0, r0, r1, v0); break;
        case 7: reduce_share<T, MODE, 7>(a, peer, rsm, bv4, et, n0, r0, r1, v0); break;
        default: reduce_share<T, MODE, 8>(a, peer, rsm, bv4, et, n0, r0, r1, v0); break;
      }
    }
    cluster.sync();  // (no CTA leaves while another may still read its shared memory)
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, static_cast<uint32_t>(a.tcols));
}

// LayerNorm of rows of K (a multiple of 8) elements, one warp per row: fp32 statistics (mean, then the mean square of
// x - mean), y = round((x - mean) * rstd * gamma + beta); with `bias`, x = round(x + bias) in place afterwards.
// Rows of up to 32 x 8 x kLnRegs elements are read once into registers, gamma / beta / bias loaded alongside
// (one round trip per row); longer rows take three passes over memory.
constexpr int kLnRegs = 8;  // 16-byte pieces per lane held in registers: K <= 2048
template <typename T>
__global__ void __launch_bounds__(128)
    ln_rows_kernel(T *x, const T *__restrict__ gamma, const T *__restrict__ beta, const T *__restrict__ bias,
                   T *__restrict__ y, int N, int K, float eps) {
  pdl_wait();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (r >= N) return;
  T *xr = x + static_cast<size_t>(r) * K;
  T *yr = y + static_cast<size_t>(r) * K;
  if (K <= 32 * 8 * kLnRegs) {
    uint4 xv[kLnRegs], gv[kLnRegs], bv[kLnRegs], cv[kLnRegs];
#pragma unroll
    for (int j = 0; j < kLnRegs; ++j) {
      const int k = (lane + 32 * j) * 8;
      if (k < K) {
        xv[j] = *reinterpret_cast<const uint4 *>(xr + k);
        gv[j] = *reinterpret_cast<const uint4 *>(gamma + k);
        bv[j] = *reinterpret_cast<const uint4 *>(beta + k);
        if (bias != nullptr) cv[j] = *reinterpret_cast<const uint4 *>(bias + k);
      }
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kLnRegs; ++j)
      if ((lane + 32 * j) * 8 < K) {
        float f[8];
        unpack8<T>(xv[j], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) s += f[i];
      }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / K;
    float v = 0.f;
#pragma unroll
    for (int j = 0; j < kLnRegs; ++j)
      if ((lane + 32 * j) * 8 < K) {
        float f[8];
        unpack8<T>(xv[j], f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float d = f[i] - mean;
          v += d * d;
        }
      }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float rstd = 1.f / sqrtf(v / K + eps);
#pragma unroll
    for (int j = 0; j < kLnRegs; ++j) {
      const int k = (lane + 32 * j) * 8;
      if (k < K) {
        float f[8], g[8], b[8], o[8];
        unpack8<T>(xv[j], f);
        unpack8<T>(gv[j], g);
        unpack8<T>(bv[j], b);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = (f[i] - mean) * rstd * g[i] + b[i];
        *reinterpret_cast<uint4 *>(yr + k) = pack8<T>(o);
        if (bias != nullptr) {
          float c[8];
          unpack8<T>(cv[j], c);
#pragma unroll
          for (int i = 0; i < 8; ++i) f[i] += c[i];
          *reinterpret_cast<uint4 *>(xr + k) = pack8<T>(f);
        }
      }
    }
    return;
  }
  float s = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    float f[8];
    unpack8<T>(*reinterpret_cast<const uint4 *>(xr + k), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += f[i];
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / K;
  float v = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    float f[8];
    unpack8<T>(*reinterpret_cast<const uint4 *>(xr + k), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float d = f[i] - mean;
      v += d * d;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const float rstd = 1.f / sqrtf(v / K + eps);
  for (int k = lane * 8; k < K; k += 256) {
    float f[8], g[8], b[8];
    unpack8<T>(*reinterpret_cast<const uint4 *>(xr + k), f);
    unpack8<T>(*reinterpret_cast<const uint4 *>(gamma + k), g);
    unpack8<T>(*reinterpret_cast<const uint4 *>(beta + k), b);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (f[i] - mean) * rstd * g[i] + b[i];
    *reinterpret_cast<uint4 *>(yr + k) = pack8<T>(o);
    if (bias != nullptr) {
      float c[8];
      unpack8<T>(*reinterpret_cast<const uint4 *>(bias + k), c);
#pragma unroll
      for (int i = 0; i < 8; ++i) f[i] += c[i];
      *reinterpret_cast<uint4 *>(xr + k) = pack8<T>(f);
    }
  }
}

// The SM count the plan is sized for (148 on a B200 if the device cannot be queried: the launch then reports the
// device's own error).
int dl_sm_count() {
  const int n = device_sm_count();
  return n > 0 ? n : 148;
}

// Thread-block clusters of `splits` CTAs of `kernel` (with `smem` bytes each) resident at once on this device --
// the clusters of one launch must fit in one wave. Cached per (kernel, device, splits, smem).
template <typename Kern>
int max_clusters(Kern kernel, int splits, int smem) {
  struct Entry {
    const void *k;
    int dev, splits, smem, n;
  };
  static Entry cache[128];
  static int used = 0;
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {  // (no device to key the cache by: assume every SM holds one CTA)
    cudaGetLastError();
    return dl_sm_count() / splits;
  }
  const void *kp = reinterpret_cast<const void *>(kernel);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (cache[i].k == kp && cache[i].dev == dev && cache[i].splits == splits && cache[i].smem == smem)
        return cache[i].n;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(splits));
  cfg.blockDim = dim3(kDlThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = static_cast<unsigned>(splits);
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = dl_sm_count() / splits;  // (the query failed: assume every SM holds one CTA)
  }
  std::lock_guard<std::mutex> lock(mu);
  if (used < 128) cache[used++] = Entry{kp, dev, splits, smem, n};
  return n;
}

// Estimated duration (us) of a plan, from measurements of this kernel on B200 at decode sizes: a CTA streams its
// stages at ~75 GB/s, and parking plus reducing its fp32 partial moves ~38 GB/s; launches of more CTAs than fit run
// in waves.
double plan_cost(const DlPlan &p, int sms) {
  const double stream = static_cast<double>(p.kb_per) * (kDlTileV * 128.0 + p.nmma * 128.0) / 75e3;
  const double reduce = p.splits > 1 ? p.nmma * 512.0 / 38e3 : 0.0;
  const int waves = p.splits > 1 ? 1 : (p.grid + sms - 1) / sms;
  return waves * (stream + reduce);
}

// The plan to launch: for each candidate row chunking (the fewest chunks, and more while a chunk keeps >= 64
// rows), the most k splits whose clusters all fit in one wave, costed by plan_cost; the cheapest wins (ties: fewer
// chunks).
template <typename Kern>
DlPlan tuned_plan(Kern kernel, int N, int V, int K, bool ln) {
  const int sms = dl_sm_count(), c0 = min_chunks(N);
  DlPlan best{};
  double best_t = 0.0;
  bool have = false;
  for (int c = c0; c <= 4 * c0; ++c) {
    if (row_chunks() != 0 && c != c0 * row_chunks()) continue;
    if (row_chunks() == 0 && c > c0 && chunk_rows(N, c) < 64) break;
    if (row_chunks() == 0 && c > c0 && chunk_rows(N, c) == chunk_rows(N, c - 1)) continue;
    int smax = kDlMaxSplits;
    DlPlan p = dl_plan(N, V, K, ln, sms, c, smax);
    while (p.splits > 1 && p.chunks * p.vtiles > max_clusters(kernel, p.splits, p.smem)) {
      if (trace_plans())
        fprintf(stderr, "[dec_linear] rows %d out %d in %d, %d chunks of %d: %d clusters of %d do not fit (%d resident)\n",
                N, V, K, p.chunks, p.nmma, p.chunks * p.vtiles, p.splits, max_clusters(kernel, p.splits, p.smem));
      smax = p.splits - 1;
      p = dl_plan(N, V, K, ln, sms, c, smax);
    }
    const double t = plan_cost(p, sms);
    if (trace_plans())
      fprintf(stderr, "[dec_linear] rows %d out %d in %d: %d chunks of %d rows, %d splits of %d k blocks, grid %d, "
              "cost %.2f us\n", N, V, K, p.chunks, p.nmma, p.splits, p.kb_per, p.grid, t);
    if (!have || t < best_t - 1e-9) {
      best = p;
      best_t = t;
      have = true;
    }
  }
  return have ? best : dl_plan(N, V, K, ln, sms, c0);
}

// The GEMM with its fused epilogue; `x` its rows (for ln_linear the normalized rows in the workspace).
template <typename T, int MODE>
int launch_gemm(int dtype, const void *x, const void *w, const void *b, const void *res, void *y, int N, int V, int K,
                bool ln, void *workspace, void *stream) {
  auto kernel = dec_gemm_kernel<T, MODE>;
  // (per instantiation, once per device: the largest dynamic shared memory the device lets a block opt into, less
  // the kernel's static shared memory; every plan stays below it, and the cluster-occupancy query needs it set)
  int dev = 0;
  int st = current_device(&dev, "dec_linear");
  if (st != WT_OK) return st;
  int optin = 0;
  cudaFuncAttributes fa{};
  if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, kernel) != cudaSuccess)
    return fail(WT_ERR_CUDA, "dec_linear: cannot read the shared-memory limits: %s",
                cudaGetErrorString(cudaGetLastError()));
  st = opt_in_smem<dec_gemm_kernel<T, MODE>>(optin - static_cast<int>(fa.sharedSizeBytes), "dec_linear");
  if (st != WT_OK) return st;
  const DlPlan p = tuned_plan(kernel, N, V, K, ln);
  CUtensorMap wm, xm;
  st = encode_tile_map(&wm, w, static_cast<unsigned long long>(V), static_cast<unsigned long long>(K), kDlTileV,
                       dtype);
  if (st != WT_OK) return st;
  st = encode_tile_map(&xm, x, static_cast<unsigned long long>(N), static_cast<unsigned long long>(K), p.nmma, dtype);
  if (st != WT_OK) return st;
  DlArgs a{reinterpret_cast<int *>(workspace), b, res, y, N, V, p.kblocks, p.splits, p.kb_per, p.vtiles, p.nmma,
           p.tcols, p.stages, p.ring_bytes, p.res_bytes, wait_limit(), test_withhold_stage()};
  return launch_clustered("dec_linear", kernel, dim3(p.grid), dim3(kDlThreads), p.smem, stream, p.splits, wm, xm, a);
}

template <typename T>
int launch_ln(T *x, const T *gamma, const T *beta, const T *bias, T *y, int N, int K, float eps, void *stream) {
  return launch("layer_norm", ln_rows_kernel<T>, dim3((N + 3) / 4), dim3(128), 0, stream, x, gamma, beta, bias, y, N,
                K, eps);
}

int check_common(const char *what, int dtype, int N, int V, int K) {
  WT_REQUIRE(N > 0 && V > 0 && K > 0, WT_ERR_ARG, "%s: sizes must be positive (rows %d, out %d, in %d)", what, N, V,
             K);
  WT_REQUIRE(K % 8 == 0, WT_ERR_UNSUPPORTED, "%s: in_features %d is not a multiple of 8", what, K);
  WT_REQUIRE(V % 8 == 0, WT_ERR_UNSUPPORTED, "%s: out_features %d is not a multiple of 8", what, V);
  WT_REQUIRE(dtype == WT_F16 || dtype == WT_BF16, WT_ERR_DTYPE, "%s: unknown dtype %d", what, dtype);
  return WT_OK;
}

int run_gemm(int dtype, int mode, const void *x, const void *w, const void *b, const void *res, void *y, int N,
             int V, int K, bool ln, void *workspace, void *stream) {
  const bool bf = dtype == WT_BF16;
  switch (mode) {
    case kDlGelu:
      return bf ? launch_gemm<__nv_bfloat16, kDlGelu>(dtype, x, w, b, res, y, N, V, K, ln, workspace, stream)
                : launch_gemm<__half, kDlGelu>(dtype, x, w, b, res, y, N, V, K, ln, workspace, stream);
    case kDlResidual:
      return bf ? launch_gemm<__nv_bfloat16, kDlResidual>(dtype, x, w, b, res, y, N, V, K, ln, workspace, stream)
                : launch_gemm<__half, kDlResidual>(dtype, x, w, b, res, y, N, V, K, ln, workspace, stream);
    default:
      return bf ? launch_gemm<__nv_bfloat16, kDlBias>(dtype, x, w, b, res, y, N, V, K, ln, workspace, stream)
                : launch_gemm<__half, kDlBias>(dtype, x, w, b, res, y, N, V, K, ln, workspace, stream);
  }
}

}  // namespace
}  // namespace wt

extern "C" {

size_t wt_dec_linear_workspace(int rows, int out_features, int in_features, int layer_norm) {
  if (rows <= 0 || out_features <= 0 || in_features <= 0) return 0;
  return wt::dl_plan(rows, out_features, in_features, layer_norm != 0, wt::dl_sm_count()).bytes;
}

int wt_layer_norm_bias(int dtype, void *x, const void *gamma, const void *beta, const void *bias, void *y, int rows,
                       int d, float eps, void *stream) {
  using namespace wt;
  WT_REQUIRE(rows > 0 && d > 0, WT_ERR_ARG, "layer_norm_bias: sizes must be positive (rows %d, d %d)", rows, d);
  WT_REQUIRE(d % 8 == 0, WT_ERR_UNSUPPORTED, "layer_norm_bias: d %d is not a multiple of 8", d);
  WT_REQUIRE(x && gamma && beta && bias && y, WT_ERR_ARG, "layer_norm_bias: null pointer");
  WT_ALIGNED(x);
  WT_ALIGNED(gamma);
  WT_ALIGNED(beta);
  WT_ALIGNED(bias);
  WT_ALIGNED(y);
  if (dtype == WT_F16)
    return launch_ln<__half>(static_cast<__half *>(x), static_cast<const __half *>(gamma),
                             static_cast<const __half *>(beta), static_cast<const __half *>(bias),
                             static_cast<__half *>(y), rows, d, eps, stream);
  if (dtype == WT_BF16)
    return launch_ln<__nv_bfloat16>(static_cast<__nv_bfloat16 *>(x), static_cast<const __nv_bfloat16 *>(gamma),
                                    static_cast<const __nv_bfloat16 *>(beta), static_cast<const __nv_bfloat16 *>(bias),
                                    static_cast<__nv_bfloat16 *>(y), rows, d, eps, stream);
  return fail(WT_ERR_DTYPE, "layer_norm_bias: unknown dtype %d", dtype);
}

int wt_ln_linear(int dtype, const void *x, const void *gamma, const void *beta, const void *w, const void *b, void *y,
                 int rows, int out_features, int in_features, int gelu, float eps, void *workspace,
                 size_t workspace_bytes, void *stream) {
  using namespace wt;
  int st = check_common("ln_linear", dtype, rows, out_features, in_features);
  if (st != WT_OK) return st;
  WT_REQUIRE(x && gamma && beta && w && b && y, WT_ERR_ARG, "ln_linear: null pointer");
  WT_ALIGNED(x);
  WT_ALIGNED(gamma);
  WT_ALIGNED(beta);
  WT_ALIGNED(w);
  WT_ALIGNED(b);
  WT_ALIGNED(y);
  const DlPlan p = dl_plan(rows, out_features, in_features, true, dl_sm_count());
  WT_REQUIRE(workspace && workspace_bytes >= p.bytes, WT_ERR_WORKSPACE,
             "ln_linear: needs a workspace of %zu bytes (given %zu)", p.bytes, workspace ? workspace_bytes : 0);
  WT_ALIGNED(workspace);
  void *xn = static_cast<char *>(workspace) + p.xn_off;
  if (dtype == WT_F16)
    st = launch_ln<__half>(const_cast<__half *>(static_cast<const __half *>(x)), static_cast<const __half *>(gamma),
                           static_cast<const __half *>(beta), nullptr, static_cast<__half *>(xn), rows, in_features,
                           eps, stream);
  else
    st = launch_ln<__nv_bfloat16>(const_cast<__nv_bfloat16 *>(static_cast<const __nv_bfloat16 *>(x)),
                                  static_cast<const __nv_bfloat16 *>(gamma), static_cast<const __nv_bfloat16 *>(beta),
                                  nullptr, static_cast<__nv_bfloat16 *>(xn), rows, in_features, eps, stream);
  if (st != WT_OK) return st;
  return run_gemm(dtype, gelu ? kDlGelu : kDlBias, xn, w, b, nullptr, y, rows, out_features, in_features, true,
                  workspace, stream);
}

int wt_linear_residual(int dtype, const void *x, const void *w, const void *b, const void *res, void *y, int rows,
                       int out_features, int in_features, void *workspace, size_t workspace_bytes, void *stream) {
  using namespace wt;
  int st = check_common("linear_residual", dtype, rows, out_features, in_features);
  if (st != WT_OK) return st;
  WT_REQUIRE(x && w && b && res && y, WT_ERR_ARG, "linear_residual: null pointer");
  WT_ALIGNED(x);
  WT_ALIGNED(w);
  WT_ALIGNED(b);
  WT_ALIGNED(res);
  WT_ALIGNED(y);
  const DlPlan p = dl_plan(rows, out_features, in_features, false, dl_sm_count());
  WT_REQUIRE(workspace && workspace_bytes >= p.bytes, WT_ERR_WORKSPACE,
             "linear_residual: needs a workspace of %zu bytes (given %zu)", p.bytes,
             workspace ? workspace_bytes : 0);
  WT_ALIGNED(workspace);
  return run_gemm(dtype, kDlResidual, x, w, b, res, y, rows, out_features, in_features, false, workspace, stream);
}

}  // extern "C"
