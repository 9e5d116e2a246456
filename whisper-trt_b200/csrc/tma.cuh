// Tensor Memory Accelerator (TMA) and mbarrier helpers for sm_100a: tensor maps encoded on the host through the
// driver entry point, 2D tiled bulk loads into shared memory completing on an mbarrier, and
// bounded mbarrier waits that record a timeout instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace wt {

// Encode a 2D tiled tensor map over a row-major [rows, 64] tensor of 16-bit elements (128-byte rows) with boxes of
// `box_rows` rows, 128-byte swizzle (16-byte chunk c of row r lands at chunk c ^ (r % 8)), zero fill out of bounds.
int encode_rows128_map(CUtensorMap *map, const void *base, unsigned long long rows, int box_rows, int dtype);
// The same for a row-major [rows, cols] tensor of 16-bit elements (cols a multiple of 8: 16-byte row stride), boxes of
// 64 columns x `box_rows` rows; elements outside the tensor read as zero.
int encode_tile_map(CUtensorMap *map, const void *base, unsigned long long rows, unsigned long long cols,
                    int box_rows, int dtype);

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`, giving up after `limit` polls (each try_wait itself suspends for a while; the
// host's wt_set_wait_limit, 2^22 by default): on a timeout the kernel records `code` in *err (if given) and returns
// false -- it never hangs the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, int *err, int code,
                                                  uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(64);
  }
  if (err != nullptr) atomicExch(err, code);
  return false;
}

// The same for the roles of a warp-specialised CTA (a producer, an MMA issuer, epilogue warps) that share a stop flag
// in shared memory: a wait that runs out records `code` in *err and raises *stop; a wait that sees *stop raised by
// another role gives up at once, without recording. A role whose wait fails issues nothing more, so the others'
// waits on it end early instead of each running out its own limit.
__device__ __forceinline__ bool mbar_wait_role(uint64_t *bar, uint32_t parity, int *err, int code, uint32_t limit,
                                               volatile int *stop) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) {  // (the flag is read only once the wait is long: the first polls stay as short as a plain wait's)
      if (*stop) return false;
      __nanosleep(64);
    }
  }
  if (err != nullptr) atomicExch(err, code);
  *stop = 1;
  return false;
}

// 2D tiled TMA load of the box at (x, y) of `map` into shared memory, completing on `bar` (complete_tx::bytes).
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// Prefetch the box at (x, y) of `map` into L2 (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// Prefetch `bytes` (a multiple of 16) at a 16-byte aligned global address into L2.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ uint4 lds16(const void *p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(smem_addr(p)));
  return r;
}

// Byte offset of 16-byte chunk `chunk` of row `row` inside a 128-byte-swizzled tile of 128-byte rows.
__device__ __forceinline__ int swz128(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

}  // namespace wt
