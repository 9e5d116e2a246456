// Shared helpers of the whisper_attn_b200 kernels: element types, vector loads, status reporting, launches.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <mutex>

#include "whisper_attn_b200.h"

namespace wt {

// ---- host-side status ------------------------------------------------------------------------------------
int fail(int status, const char *fmt, ...);  // records the calling thread's message, returns status
int launch_flags();
bool aligned16(const void *p);
unsigned wait_limit();     // polls of every bounded device wait (wt_set_wait_limit)
int test_withhold_stage();  // the bounded-wait test hook (wt_set_test_withhold_stage)

// ---- per-device queries and settings (thread safe) -------------------------------------------------------
constexpr int kMaxDevices = 64;
// The calling thread's current device into *dev; WT_ERR_CUDA (message recorded) if it cannot be read or is beyond
// kMaxDevices.
int current_device(int *dev, const char *what);
// The current device's SM count, queried once per device; 0 (message recorded) if the query fails.
int device_sm_count();

// Let `Kernel` launch with `bytes` of dynamic shared memory on the current device. The attribute is per device, so
// it is set once per (kernel, device) and again only for a larger size; the recorded size only grows, under a lock,
// so concurrent first calls from several host threads (or several devices driven by one process) stay correct.
// WT_ERR_CUDA with the runtime's message when the device refuses the size.
template <auto Kernel>
int opt_in_smem(int bytes, const char *what) {
  static std::atomic<int> granted[kMaxDevices];
  static std::mutex mu;
  int dev = 0;
  const int st = current_device(&dev, what);
  if (st != WT_OK) return st;
  if (granted[dev].load(std::memory_order_acquire) >= bytes) return WT_OK;
  std::lock_guard<std::mutex> lock(mu);
  if (granted[dev].load(std::memory_order_relaxed) >= bytes) return WT_OK;
  const cudaError_t e = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();  // (clear it: the next launch must not report this error as its own)
    return fail(WT_ERR_CUDA, "%s: cannot opt into %d bytes of dynamic shared memory on device %d: %s", what, bytes,
                dev, cudaGetErrorString(e));
  }
  granted[dev].store(bytes, std::memory_order_release);
  return WT_OK;
}

#define WT_REQUIRE(cond, status, ...)            \
  do {                                           \
    if (!(cond)) return ::wt::fail(status, __VA_ARGS__); \
  } while (0)

#define WT_ALIGNED(p) WT_REQUIRE(::wt::aligned16(p), WT_ERR_ALIGN, "%s is not 16-byte aligned", #p)

inline int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(WT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return WT_OK;
}

// Launch `kernel` with grid/block/smem on `stream`, as a programmatic dependent launch when the process-wide
// WT_LAUNCH_PDL flag is set (the kernel then starts while its predecessor drains and waits for it with
// griddepcontrol.wait before touching anything the predecessor may write).
template <typename... KArgs, typename... Args>
int launch(const char *what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void *stream,
           Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  int n = 0;
  if (launch_flags() & WT_LAUNCH_PDL) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return fail(WT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return WT_OK;
}

// A launch without the programmatic-dependent-launch attribute whatever the process-wide flag: the kernel starts
// once its predecessor has completed (its own griddepcontrol.wait is then a no-op), and may still let its successor
// start early.
template <typename... KArgs, typename... Args>
int launch_after(const char *what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void *stream,
                 Args... args) {
  kernel<<<grid, block, smem, static_cast<cudaStream_t>(stream)>>>(static_cast<KArgs>(args)...);
  return check_launch(what);
}

// The same with thread-block clusters of `cluster_x` CTAs along x (gridDim.x a multiple of it).
template <typename... KArgs, typename... Args>
int launch_clustered(const char *what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void *stream,
                     int cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (launch_flags() & WT_LAUNCH_PDL) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return fail(WT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return WT_OK;
}

// ---- device side -----------------------------------------------------------------------------------------
// Programmatic dependent launch controls (no-ops when the kernel was launched without the attribute). The kernels
// trigger their dependents right after their own wait: a dependent then starts while this kernel works, but no
// earlier than this kernel's predecessor has completed, so "not written by the kernel launched just before" is all
// a kernel's pre-wait reads need.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 16-byte streaming load through the non-coherent path (data read once per launch; not allocated in L1).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg16(const void *p) {
  return *reinterpret_cast<const uint4 *>(p);
}

// Element-type traits: conversion of packed pairs.
template <typename T> struct Elem;
template <> struct Elem<__half> {
  using pair = __half2;
  static constexpr int code = WT_F16;
  static __device__ __forceinline__ float2 to_float2(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&u));
  }
  static __device__ __forceinline__ uint32_t from_float2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  static __device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  using pair = __nv_bfloat162;
  static constexpr int code = WT_BF16;
  static __device__ __forceinline__ float2 to_float2(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&u));
  }
  static __device__ __forceinline__ uint32_t from_float2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
  }
  static __device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

// Unpack 8 packed 16-bit elements into floats.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &u, float (&f)[8]) {
  float2 a = Elem<T>::to_float2(u.x), b = Elem<T>::to_float2(u.y), c = Elem<T>::to_float2(u.z),
         d = Elem<T>::to_float2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = Elem<T>::from_float2(f[0], f[1]);
  u.y = Elem<T>::from_float2(f[2], f[3]);
  u.z = Elem<T>::from_float2(f[4], f[5]);
  u.w = Elem<T>::from_float2(f[6], f[7]);
  return u;
}

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

constexpr float kNegInf = -__builtin_huge_valf();

}  // namespace wt
