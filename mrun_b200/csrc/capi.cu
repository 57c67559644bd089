// Library-level C ABI: version and per-thread error text.
#include "common.cuh"

#include <string.h>

#include <map>
#include <mutex>

namespace mrb {

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

int ensure_dynamic_smem(const void* kernel, size_t bytes, const char* what) {
  if (bytes <= 48 * 1024) return MRB_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  static std::mutex lock;
  static std::map<std::pair<const void*, int>, size_t> granted;  // (kernel, device) -> bytes
  std::lock_guard<std::mutex> hold(lock);
  size_t& have = granted[{kernel, dev}];
  if (bytes <= have) return MRB_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "%s: shared memory attribute: %s", what, cudaGetErrorString(e));
  have = bytes;
  return MRB_OK;
}

}  // namespace mrb

extern "C" int mrb_abi_version(void) { return 16; }

extern "C" const char* mrb_last_error(void) { return mrb::g_last_error; }

// ------------------------------------------------------------------ page streaming

// Host->device page copies for weight streaming: one cudaMemcpyAsync per page (pinned host
// source for true asynchrony) on the given copy stream, then `done` (a cudaEvent_t, may be
// NULL) is recorded so consumers can order their kernels after the copies. Replaces the
// side-stream staging of `_RingPrefetch` / the expert page cache (engine/kernels/qstore.py:
// 622-660, engine/qwen3_moe_cuda.py:1533-1546).
extern "C" int mrb_copy_pages(void* dst_base, int64_t dst_stride, const void* src_base, int64_t src_stride,
                              const int32_t* dst_slots, const int32_t* src_pages, int64_t count, int64_t page_bytes,
                              void* stream, void* done) {
  using namespace mrb;
  if (count < 0 || page_bytes <= 0 || dst_stride < page_bytes || src_stride < page_bytes)
    return fail(MRB_ERR_ARG, "copy_pages: bad sizes");
  if (count > 0 && (!dst_base || !src_base || !dst_slots || !src_pages))
    return fail(MRB_ERR_ARG, "copy_pages: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  for (int64_t i = 0; i < count; ++i) {
    if (dst_slots[i] < 0 || src_pages[i] < 0) return fail(MRB_ERR_ARG, "copy_pages: negative slot or page");
    char* dst = (char*)dst_base + (int64_t)dst_slots[i] * dst_stride;
    const char* src = (const char*)src_base + (int64_t)src_pages[i] * src_stride;
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)page_bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "copy_pages: cudaMemcpyAsync: %s", cudaGetErrorString(e));
  }
  if (done) {
    cudaError_t e = cudaEventRecord((cudaEvent_t)done, s);
    if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "copy_pages: cudaEventRecord: %s", cudaGetErrorString(e));
  }
  clear_error();
  return MRB_OK;
}
