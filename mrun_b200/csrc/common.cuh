// Shared helpers for the mrun-b200 sm_100a kernels and their C-ABI wrappers.
//
// Every exported entry point returns an int status (MRB_OK on success) and records a
// human-readable message for the calling host thread, read back with mrb_last_error().
// Kernels never trap: bad arguments are rejected on the host before launch.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>
#include <stdlib.h>

#include <utility>

#include "../../include/mrun_b200.h"

namespace mrb {

// Thread-local last-error text (host side).
void set_error(const char* fmt, ...);
void clear_error();

inline int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  set_error("%s", buf);
  return status;
}

// Check the launch that was just enqueued.
inline int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(MRB_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  }
  clear_error();
  return MRB_OK;
}

// Raise `kernel`'s dynamic shared-memory limit to at least `bytes` on the CURRENT device
// (cudaFuncSetAttribute applies per device). Remembers what each (kernel, device) pair was
// given, so repeated launches pay one locked map lookup; safe from several host threads and
// for a process that drives several GPUs. Returns MRB_OK or an MRB_ERR_CUDA status.
int ensure_dynamic_smem(const void* kernel, size_t bytes, const char* what);

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

inline int num_sms() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

// Launch with programmatic dependent launch allowed (the kernel may start while the previous
// kernel on the stream finishes; it must call griddepcontrol.wait before reading that
// kernel's results). Disabled by setting MRB_PDL=0 in the environment.
inline bool pdl_enabled() {
  static int enabled = -1;
  if (enabled < 0) {
    const char* v = getenv("MRB_PDL");
    enabled = (v && v[0] == '0') ? 0 : 1;
  }
  return enabled == 1;
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                 bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const bool use = pdl && pdl_enabled();
  cfg.attrs = use ? attr : nullptr;
  cfg.numAttrs = use ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ---------------------------------------------------------------- device helpers

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Round-to-nearest-even fp32 -> bf16 -> fp32 (the value a bf16 tensor would hold).
__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

template <typename T> struct io;
template <> struct io<float> {
  static __device__ __forceinline__ float load(const float* p) { return *p; }
  static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};
template <> struct io<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};
template <> struct io<__half> {
  static __device__ __forceinline__ float load(const __half* p) { return __half2float(*p); }
  static __device__ __forceinline__ void store(__half* p, float v) { *p = __float2half_rn(v); }
};

// Bring the 128-byte line holding p into L2 (no register result, no wait).
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// Streaming 128-bit read-only load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

}  // namespace mrb
