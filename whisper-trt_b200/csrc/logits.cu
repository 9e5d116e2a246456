// The vocabulary projection with fp32 accumulation and output: logits [N, V] = x [N, d] . w [V, d]^T, x and w fp16
// or bf16 -- the reference's logits32 (attn_plugin.py:202-212 op, :438-455 kernel, :549-560 launcher), the one
// tensor-core-bound piece next to the attention path.
//
// B200 design: 5th-generation tensor cores. The work is cut into items of G 128-entry vocabulary tiles x one chunk of
// up to 256 rows of x; a tile's rows of w are the MMA's A (M = 128), the chunk's rows of x its B (N = the rows, padded
// to 16), the reduction d in 64-element blocks staged by TMA (128-byte swizzle) through a ring. One stage holds the
// item's G w blocks and ONE x block: the G tiles share each x block (x is read from L2 once per item, not once per
// tile), and G is the smallest group that fits every item in one wave over the SMs (160 rows x 51866 entries: 406
// tiles in 136 items of 3 on 148 SMs), so no SM idles through a last partial wave. G accumulators of N fp32 columns
// sit side by side in tensor memory (two sets in turn when they fit twice in its 512 columns).
//   * warp 0's lane 0 issues the TMA loads -- the first stages' w blocks before the wait for the preceding kernel
//     (w is not its output), their x blocks after it; warp 1's lane 0 issues the tcgen05.mma instructions (kind::f16,
//     fp32 accumulators in tensor memory) and releases a stage with a tcgen05.commit on its "empty" barrier;
//   * warps 2-9 drain the accumulators (each warp its lane quarter, warp % 4, and every other 16-column slice), store
//     them as consecutive floats of each output row and hand the set back;
//   * every barrier wait is bounded: a wait that runs out records an error in the device word and raises a stop flag
//     that every role checks, so no role issues more; before the CTA frees its tensor memory and exits, the
//     producer waits (bounded) for each copy it issued and the MMA issuer for its MMAs (a final commit).
#include <cstdlib>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

namespace wt {
namespace {

constexpr int kLgEpiWarps = 8;
constexpr int kLgThreads = 32 * (2 + kLgEpiWarps);  // producer, MMA issuer, 8 epilogue warps
constexpr int kLgTileV = 128;    // vocabulary entries per tile (the MMA's M)
constexpr int kLgKBlock = 64;    // reduction elements per stage (one 128-byte swizzled row)
constexpr int kLgMaxRows = 256;  // rows of x per chunk (the MMA's N, at most 256)
constexpr int kLgMaxGroup = 4;   // vocabulary tiles per item
constexpr int kLgTmemCols = 512;
constexpr int kLgSmemBudget = 216 * 1024;  // the ring (one CTA per SM)
constexpr int kLgErrTimeout = 1;

struct LgPlan {
  int chunks, nmma, stride, vtiles, group, items, nbuf, tcols, kblocks, stage_bytes, stages, smem, grid;
};

// Vocabulary tiles per item forced by WT_LG_GROUP (a tuning knob, 1-4), else 0 (chosen by the plan).
int lg_group() {
  static const int v = [] {  // (read once; a function-local static initialises thread-safely)
    const char *e = getenv("WT_LG_GROUP");
    const int x = e ? atoi(e) : 0;
    return (x >= 1 && x <= kLgMaxGroup) ? x : 0;
  }();
  return v;
}

int lg_stage_bytes(int group, int nmma) { return group * kLgTileV * 128 + (nmma * 128 + 1023) / 1024 * 1024; }

LgPlan lg_plan(int rows, int vocab, int d_model, int sms) {
  LgPlan p{};
  p.chunks = (rows + kLgMaxRows - 1) / kLgMaxRows;
  p.nmma = ((rows + p.chunks - 1) / p.chunks + 15) / 16 * 16;  // balanced chunks
  p.stride = (p.nmma + 31) / 32 * 32;                           // tensor-memory columns per accumulator
  p.vtiles = (vocab + kLgTileV - 1) / kLgTileV;
  p.kblocks = (d_model + kLgKBlock - 1) / kLgKBlock;
  int gmax = kLgTmemCols / p.stride;
  if (gmax > kLgMaxGroup) gmax = kLgMaxGroup;
  while (gmax > 1 && 2 * lg_stage_bytes(gmax, p.nmma) > kLgSmemBudget) --gmax;  // at least two stages
  p.group = gmax;
  for (int g = 1; g <= gmax; ++g)  // the smallest group whose items all fit one wave
    if (static_cast<long long>(p.chunks) * ((p.vtiles + g - 1) / g) <= sms) {
      p.group = g;
      break;
    }
  if (lg_group() > 0 && lg_group() <= gmax) p.group = lg_group();
  p.items = p.chunks * ((p.vtiles + p.group - 1) / p.group);
  p.nbuf = 2 * p.group * p.stride <= kLgTmemCols ? 2 : 1;
  p.tcols = 32;
  while (p.tcols < p.nbuf * p.group * p.stride) p.tcols <<= 1;
  p.stage_bytes = lg_stage_bytes(p.group, p.nmma);
  p.stages = kLgSmemBudget / p.stage_bytes;
  if (p.stages > 8) p.stages = 8;
  p.smem = 1024 + p.stages * p.stage_bytes + (2 * p.stages + 5) * 8 + 16;
  p.grid = p.items < sms ? p.items : sms;
  return p;
}

// Persistent: CTA c takes items c, c + grid, ...; item i is (vocabulary group i / chunks, row chunk i % chunks), so
// the CTAs that share a group's w run side by side and the later chunks find it in L2.
template <bool BF16>
__global__ void __launch_bounds__(kLgThreads)
    logits_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                  float *__restrict__ y, int N, int V, const LgPlan p, int *err, uint32_t polls, int withhold) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int a_bytes = kLgTileV * 128;
  const int G = p.group, stages = p.stages, stage_bytes = p.stage_bytes, kblocks = p.kblocks, nmma = p.nmma;
  const int b_bytes = nmma * 128;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + stages * stage_bytes);
  uint64_t *empty = full + stages;
  uint64_t *acc_full = empty + stages;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drained = acc_empty + 2;  // the MMA issuer's last commit: every MMA it issued has completed
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(drained + 1);
  volatile int *stop = reinterpret_cast<volatile int *>(tmem_holder + 1);  // a role's wait ran out
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  if (warp == 0) {
    tmem_alloc(tmem_holder, static_cast<uint32_t>(p.tcols));
    tmem_relinquish();
  }
  if (tid == 32) {
    prefetch_tensormap(&wmap);
    prefetch_tensormap(&xmap);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kLgEpiWarps);
    }
    mbar_init(drained, 1);
    *stop = 0;
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {  // producer: every k block of every item of this CTA, through the ring
      // the first item's first stage: its w blocks before the wait for the preceding kernel, its x block after it
      // (one stage: the x block the first MMAs need then waits behind no more w than that; measured faster alone)
      const int pre = static_cast<int>(blockIdx.x) < p.items ? 1 : 0;
      // (the bounded-wait test hook: CTA 0 leaves out the x block of its first stage, whose barrier then never
      // completes)
      const bool hold = withhold && blockIdx.x == 0;
      int it = 0;
      bool halt = false;
      for (int item = blockIdx.x; item < p.items && !halt; item += gridDim.x) {
        const int t0 = (item / p.chunks) * G, n0 = (item % p.chunks) * nmma;
        const int ng = min(G, p.vtiles - t0);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % stages;
          unsigned char *st = smem + s * stage_bytes;
          if (it < pre) {
            mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(ng * a_bytes + b_bytes));
            for (int g = 0; g < ng; ++g) tma_load_2d(st + g * a_bytes, &wmap, kb * kLgKBlock, (t0 + g) * kLgTileV, &full[s]);
            if (it == pre - 1) {
              pdl_wait();
              pdl_launch_dependents();
              for (int j = 0; j < pre; ++j)
                if (!(hold && j == 0))
                  tma_load_2d(smem + j * stage_bytes + G * a_bytes, &xmap, j * kLgKBlock, n0, &full[j]);
            }
            continue;
          }
          if (it >= stages && !mbar_wait_role(&empty[s], ((it / stages) - 1) & 1, err, kLgErrTimeout, polls, stop)) {
            halt = true;  // (nothing more is issued)
            break;
          }
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(ng * a_bytes + b_bytes));
          tma_load_2d(st + G * a_bytes, &xmap, kb * kLgKBlock, n0, &full[s]);  // (x first: it is in L2)
          for (int g = 0; g < ng; ++g) tma_load_2d(st + g * a_bytes, &wmap, kb * kLgKBlock, (t0 + g) * kLgTileV, &full[s]);
        }
      }
      if (pre == 0) {
        pdl_wait();
        pdl_launch_dependents();
      }
      // every copy issued has landed before the shared memory goes away: the last fill of each stage (bounded;
      // at most one outstanding per stage, since a stage is refilled only after its MMAs released it)
      for (int i = it > stages ? it - stages : 0; i < it; ++i)
        mbar_wait_bounded(&full[i % stages], (i / stages) & 1, nullptr, 0, polls);
    } else {
      pdl_wait();
      pdl_launch_dependents();
    }
  } else if (warp == 1) {
    pdl_wait();
    pdl_launch_dependents();
    if (lane == 0) {  // MMA issuer: item j into accumulator set j % nbuf once the epilogue has drained it
      const uint32_t idesc = idesc_f16(kLgTileV, nmma, BF16);
      int it = 0, j = 0;
      bool halt = false;
      for (int item = blockIdx.x; item < p.items && !halt; item += gridDim.x, ++j) {
        const int ng = min(G, p.vtiles - (item / p.chunks) * G);
        const int b = j % p.nbuf, use = j / p.nbuf;
        if (use >= 1 && !mbar_wait_role(&acc_empty[b], (use - 1) & 1, err, kLgErrTimeout, polls, stop)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * G * p.stride);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % stages;
          if (!mbar_wait_role(&full[s], (it / stages) & 1, err, kLgErrTimeout, polls, stop)) {
            halt = true;  // (no MMA reads a stage that has not landed)
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + s * stage_bytes);
          const uint64_t bdesc = sw128_desc(a_addr + static_cast<uint32_t>(G * a_bytes));
          for (int g = 0; g < ng; ++g) {
            const uint64_t adesc = sw128_desc(a_addr + static_cast<uint32_t>(g * a_bytes));
            const uint32_t dg = d + static_cast<uint32_t>(g * p.stride);
#pragma unroll
            for (int kk = 0; kk < kLgKBlock / 16; ++kk)  // K = 16 per instruction: +32 bytes along the swizzled row
              umma_f16(dg, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          }
          umma_commit(&empty[s]);
        }
        if (!halt) umma_commit(&acc_full[b]);
      }
      // every MMA issued has completed before the tensor memory is freed (bounded)
      umma_commit(drained);
      mbar_wait_bounded(drained, 0, nullptr, 0, polls);
    }
  } else {  // epilogue warps: lane quarter warp % 4 (vocabulary entries 32 (warp % 4) + lane of each tile), and
            // the 16-column slices c0 = 16 half, 16 half + 32, ... of the rows
    pdl_wait();
    pdl_launch_dependents();
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    int j = 0;
    for (int item = blockIdx.x; item < p.items; item += gridDim.x, ++j) {
      const int t0 = (item / p.chunks) * G, n0 = (item % p.chunks) * nmma;
      const int ng = min(G, p.vtiles - t0);
      const int b = j % p.nbuf, use = j / p.nbuf;
      // (the warp decides together: its tensor-memory loads are warp-wide)
      if (!__all_sync(0xffffffffu, mbar_wait_role(&acc_full[b], use & 1, err, kLgErrTimeout, polls, stop))) break;
      tc_fence_after();
      for (int g = 0; g < ng; ++g) {
        const int v = (t0 + g) * kLgTileV + quarter * 32 + lane;
        const uint32_t base = tmem + static_cast<uint32_t>((b * G + g) * p.stride) +
                              (static_cast<uint32_t>(quarter * 32) << 16);
        // four 16-column slices per wait. With V even, lanes 2j and 2j + 1 (entries v, v + 1) swap half their rows
        // so that each stores 8-byte pairs (every row of y then starts 8-byte aligned): the even lane rows i, the odd
        // lane rows 8 + i of each slice -- one store instruction covers two rows; with V odd, one float per store
        const int vp = v & ~1;
        const bool odd = (lane & 1) != 0;
        for (int cb = 16 * half; cb < nmma; cb += 128) {
          uint32_t r[4][16];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (cb + 32 * q < nmma) tmem_ld16(base + static_cast<uint32_t>(cb + 32 * q), r[q]);
          tmem_wait_ld();
          if (V & 1) {
            if (v < V) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                if (cb + 32 * q >= nmma) break;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  const int n = n0 + cb + 32 * q + i;
                  if (n < N) y[static_cast<size_t>(n) * V + v] = __uint_as_float(r[q][i]);
                }
              }
            }
            continue;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (cb + 32 * q >= nmma) break;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint32_t mine = odd ? r[q][8 + i] : r[q][i];
              const uint32_t other = __shfl_xor_sync(0xffffffffu, odd ? r[q][i] : r[q][8 + i], 1);
              const int n = n0 + cb + 32 * q + (odd ? 8 + i : i);
              if (n < N && vp < V)  // (V even: v + 1 < V too)
                *reinterpret_cast<float2 *>(y + static_cast<size_t>(n) * V + vp) =
                    odd ? make_float2(__uint_as_float(other), __uint_as_float(mine))
                        : make_float2(__uint_as_float(mine), __uint_as_float(other));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, static_cast<uint32_t>(p.tcols));
}

}  // namespace
}  // namespace wt

extern "C" int wt_logits32(int dtype, const void *x, const void *w, float *y, int rows, int vocab, int d_model,
                           int *err, void *stream) {
  using namespace wt;
  WT_REQUIRE(rows > 0 && vocab > 0 && d_model > 0, WT_ERR_ARG,
             "logits32: sizes must be positive (rows %d, vocab %d, d_model %d)", rows, vocab, d_model);
  WT_REQUIRE(x && w && y && err, WT_ERR_ARG, "logits32: null pointer");
  WT_ALIGNED(x);
  WT_ALIGNED(w);
  WT_ALIGNED(y);
  WT_REQUIRE(d_model % 8 == 0, WT_ERR_UNSUPPORTED, "logits32: d_model %d is not a multiple of 8", d_model);
  WT_REQUIRE(dtype == WT_F16 || dtype == WT_BF16, WT_ERR_DTYPE, "logits32: unknown dtype %d", dtype);
  const int sms = device_sm_count();
  if (sms <= 0) return WT_ERR_CUDA;
  const LgPlan p = lg_plan(rows, vocab, d_model, sms);
  CUtensorMap wm, xm;
  int st = encode_tile_map(&wm, w, static_cast<unsigned long long>(vocab), static_cast<unsigned long long>(d_model),
                           kLgTileV, dtype);
  if (st != WT_OK) return st;
  st = encode_tile_map(&xm, x, static_cast<unsigned long long>(rows), static_cast<unsigned long long>(d_model),
                       p.nmma, dtype);
  if (st != WT_OK) return st;
  auto kernel = dtype == WT_BF16 ? logits_kernel<true> : logits_kernel<false>;
  st = dtype == WT_BF16 ? opt_in_smem<logits_kernel<true>>(p.smem, "logits32")
                        : opt_in_smem<logits_kernel<false>>(p.smem, "logits32");
  if (st != WT_OK) return st;
  return launch("logits32", kernel, dim3(p.grid), dim3(kLgThreads), p.smem, stream, wm, xm, y, rows, vocab, p, err,
                wait_limit(), test_withhold_stage());
}
