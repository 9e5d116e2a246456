// The vocabulary projection with fp32 accumulation and output: logits [N, V] = x [N, d] . w [V, d]^T, x and w fp16
// or bf16 -- the reference's logits32 (attn_plugin.py:202-212 op, :438-455 kernel, :549-560 launcher), the one
// tensor-core-bound piece next to the attention path.
//
// B200 design: 5th-generation tensor cores, one persistent CTA per SM over 128-entry vocabulary tiles (x 256-row
// chunks of x): a tile's rows of w are the MMA's A (M = 128), the rows of x its B (N = the rows, padded to 16), the
// reduction d in 64-element blocks staged by TMA (128-byte swizzle) through a ring of up to 8 stages. Warp 0's lane
// 0 issues the TMA loads, warp 1's lane 0 the tcgen05.mma instructions (kind::f16, fp32 accumulator in tensor
// memory, two accumulators in turn); a stage is released by a tcgen05.commit on its "empty" barrier when its MMAs
// complete, an accumulator by a commit on its "full" barrier. Warps 2-5 read the accumulator's 128 lanes
// (vocabulary entries) with tcgen05.ld, 16 rows at a time, store them as consecutive floats of each output row and
// hand the accumulator back -- under the next tile's loads and MMAs. Every barrier wait is bounded (a timeout
// records an error in the device word and the kernel goes on, then frees its tensor memory).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "tc05.cuh"
#include "tma.cuh"

namespace wt {
namespace {

constexpr int kLgEpiWarps = 4;
constexpr int kLgThreads = 32 * (2 + kLgEpiWarps);  // producer, MMA issuer, 4 epilogue warps
constexpr int kLgTileV = 128;   // vocabulary entries per CTA (the MMA's M)
constexpr int kLgKBlock = 64;   // reduction elements per stage (one 128-byte swizzled row)
constexpr int kLgMaxRows = 256; // rows of x per CTA (the MMA's N, at most 256)
constexpr int kLgErrTimeout = 1;

// Persistent: CTA c takes tiles c, c + grid, ... (tile = vocabulary tile x row chunk). Warp 0 (lane 0) streams
// the tiles' k-blocks through the ring, warp 1 (lane 0) issues their MMAs into one of two tensor-memory
// accumulators, warps 2-5 drain the other one (each warp its lane quarter, warp % 4), so a tile's epilogue runs
// under the next tile's loads and MMAs.
template <bool BF16>
__global__ void __launch_bounds__(kLgThreads)
    logits_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                  float *__restrict__ y, int N, int V, int kblocks, int nmma, int tcols, int stages, int *err,
                  uint32_t polls) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_bytes = kLgTileV * 128, b_bytes = nmma * 128;
  const int stage_bytes = a_bytes + ((b_bytes + 1023) & ~1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + stages * stage_bytes);
  uint64_t *empty = full + stages;
  uint64_t *acc_full = empty + stages;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_empty + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int vtiles = (V + kLgTileV - 1) / kLgTileV;
  const int tiles = vtiles * ((N + kLgMaxRows - 1) / kLgMaxRows);

  if (warp == 0) {
    tmem_alloc(tmem_holder, static_cast<uint32_t>(2 * tcols));
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
    fence_mbar_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  pdl_wait();
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {  // producer: every k-block of every tile of this CTA, through the ring
      int it = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int v0 = (t % vtiles) * kLgTileV, n0 = (t / vtiles) * kLgMaxRows;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % stages;
          if (it >= stages) mbar_wait_bounded(&empty[s], ((it / stages) - 1) & 1, err, kLgErrTimeout, polls);
          unsigned char *st = smem + s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(a_bytes + b_bytes));
          tma_load_2d(st, &wmap, kb * kLgKBlock, v0, &full[s]);
          tma_load_2d(st + a_bytes, &xmap, kb * kLgKBlock, n0, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer: tile j into accumulator j % 2 once the epilogue has drained it
      const uint32_t idesc = idesc_f16(kLgTileV, nmma, BF16);
      int it = 0, j = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2) mbar_wait_bounded(&acc_empty[b], ((j >> 1) - 1) & 1, err, kLgErrTimeout, polls);
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * tcols);
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % stages;
          mbar_wait_bounded(&full[s], (it / stages) & 1, err, kLgErrTimeout, polls);
          tc_fence_after();
          const uint32_t a_addr = smem_addr(smem + s * stage_bytes), b_addr = a_addr + a_bytes;
          const uint64_t adesc = sw128_desc(a_addr), bdesc = sw128_desc(b_addr);
#pragma unroll
          for (int kk = 0; kk < kLgKBlock / 16; ++kk)  // K = 16 per instruction: +32 bytes along the swizzled row
            umma_f16(d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb | kk) != 0);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
      }
    }
  } else {  // epilogue warps: lane quarter warp % 4 = vocabulary entries v0 + 32 (warp % 4) + lane
    const int quarter = warp & 3;
    int j = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int b = j & 1;
      const int v = (t % vtiles) * kLgTileV + quarter * 32 + lane, n0 = (t / vtiles) * kLgMaxRows;
      mbar_wait_bounded(&acc_full[b], (j >> 1) & 1, err, kLgErrTimeout, polls);
      tc_fence_after();
      const uint32_t base = tmem + static_cast<uint32_t>(b * tcols) + (static_cast<uint32_t>(quarter * 32) << 16);
      for (int c0 = 0; c0 < nmma; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(base + static_cast<uint32_t>(c0), r);
        tmem_wait_ld();
        if (v < V) {
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int n = n0 + c0 + q;
            if (n < N) y[static_cast<size_t>(n) * V + v] = __uint_as_float(r[q]);
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
  if (warp == 0) tmem_dealloc(tmem, static_cast<uint32_t>(2 * tcols));
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
  const int chunks = (rows + kLgMaxRows - 1) / kLgMaxRows;
  const int nrows = rows < kLgMaxRows ? rows : kLgMaxRows;
  const int nmma = (nrows + 15) / 16 * 16;
  int tcols = 32;
  while (tcols < nmma) tcols <<= 1;
  CUtensorMap wm, xm;
  int st = encode_tile_map(&wm, w, static_cast<unsigned long long>(vocab), static_cast<unsigned long long>(d_model),
                           kLgTileV, dtype);
  if (st != WT_OK) return st;
  st = encode_tile_map(&xm, x, static_cast<unsigned long long>(rows), static_cast<unsigned long long>(d_model), nmma,
                       dtype);
  if (st != WT_OK) return st;
  const int stage_bytes = kLgTileV * 128 + (nmma * 128 + 1023) / 1024 * 1024;
  const int stages = (200 * 1024) / stage_bytes < 8 ? (200 * 1024) / stage_bytes : 8;  // one CTA per SM
  const int smem = 1024 + stages * stage_bytes + (2 * stages + 4) * 8 + 16;
  const int kblocks = (d_model + kLgKBlock - 1) / kLgKBlock;
  auto kernel = dtype == WT_BF16 ? logits_kernel<true> : logits_kernel<false>;
  st = dtype == WT_BF16 ? opt_in_smem<logits_kernel<true>>(smem, "logits32")
                        : opt_in_smem<logits_kernel<false>>(smem, "logits32");
  if (st != WT_OK) return st;
  const int sms = device_sm_count();
  if (sms <= 0) return WT_ERR_CUDA;
  const int tiles = ((vocab + kLgTileV - 1) / kLgTileV) * chunks;
  const int grid = tiles < sms ? tiles : sms;
  return launch("logits32", kernel, dim3(grid), dim3(kLgThreads), smem, stream, wm, xm, y, rows, vocab, kblocks,
                nmma, tcols, stages, err, wait_limit());
}
