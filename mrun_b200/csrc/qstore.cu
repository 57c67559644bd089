// QStore store-build and gather kernels: per-row int8 quantisation and dequantised row
// gathers (embedding lookup).
#include "qrow_common.cuh"

namespace mrb {

// One CTA per row: max|w| reduction, then round-half-even quantisation.
// Matches `_quant_row_int8` (engine/kernels/qstore_build.py:496-501): the scale is the
// IEEE fp32 quotient max/127, an all-zero row gets scale 1, codes are rint(w / scale)
// (true division, not a reciprocal multiply) clipped to [-127, 127].
__global__ void __launch_bounds__(256) quant_row_int8_kernel(const float* __restrict__ w,
                                                             int64_t cols, int8_t* __restrict__ codes,
                                                             float* __restrict__ scales) {
  const int64_t row = blockIdx.x;
  const float* src = w + row * cols;
  float m = 0.f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) m = fmaxf(m, fabsf(src[c]));
  __shared__ float red[8];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float scale = __fdiv_rn(red[0], 127.0f);
  if (scale == 0.0f) scale = 1.0f;
  if (threadIdx.x == 0) scales[row] = scale;
  int8_t* dst = codes + row * cols;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    float q = rintf(__fdiv_rn(src[c], scale));
    q = fminf(fmaxf(q, -127.f), 127.f);
    dst[c] = static_cast<int8_t>(q);
  }
}

template <typename OT>
__global__ void __launch_bounds__(256) embed_rows_kernel(const int8_t* __restrict__ codes,
                                                         const float* __restrict__ scales, int64_t rows,
                                                         int64_t cols, const int64_t* __restrict__ ids,
                                                         OT* __restrict__ out, int32_t* bad_ids) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t i = blockIdx.x;
  const int64_t id = ids[i];
  OT* dst = out + i * cols;
  if (id < 0 || id >= rows) {
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) io<OT>::store(dst + c, 0.f);
    if (threadIdx.x == 0 && bad_ids) *bad_ids = 1;
    return;
  }
  const int8_t* src = codes + id * cols;
  const float s = scales[id];
  // fp32 product first (the reference's `q.float() * s`), then narrow to the output type.
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    io<OT>::store(dst + c, __fmul_rn(static_cast<float>(src[c]), s));
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_quant_row_int8(const float* weight, int64_t rows, int64_t cols, int8_t* codes,
                                  float* scales, void* stream) {
  if (rows < 0 || cols <= 0) return fail(MRB_ERR_ARG, "quant_row_int8: bad shape [%lld, %lld]",
                                         (long long)rows, (long long)cols);
  if (!weight || !codes || !scales) return fail(MRB_ERR_ARG, "quant_row_int8: null pointer");
  if (rows == 0) return MRB_OK;
  if (rows > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "quant_row_int8: too many rows");
  quant_row_int8_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(weight, cols, codes, scales);
  return launch_status("quant_row_int8");
}

extern "C" int mrb_qrow_embed_rows(const int8_t* codes, const float* scales, int64_t rows, int64_t cols,
                                   const int64_t* ids, int64_t n_ids, void* out, int out_dtype,
                                   int32_t* bad_ids, void* stream) {
  if (rows <= 0 || cols <= 0 || n_ids < 0) return fail(MRB_ERR_ARG, "embed_rows: bad shape");
  if (!codes || !scales || !ids || !out) return fail(MRB_ERR_ARG, "embed_rows: null pointer");
  if (n_ids == 0) return MRB_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (out_dtype) {
    case MRB_F32:
      embed_rows_kernel<float><<<(unsigned)n_ids, 256, 0, s>>>(codes, scales, rows, cols, ids,
                                                               (float*)out, bad_ids);
      break;
    case MRB_BF16:
      launch_kernel(embed_rows_kernel<__nv_bfloat16>, dim3((unsigned)n_ids), dim3(256), 0, s, true, codes, scales, rows,
                    cols, ids, (__nv_bfloat16*)out, bad_ids);
      break;
    case MRB_F16:
      embed_rows_kernel<__half><<<(unsigned)n_ids, 256, 0, s>>>(codes, scales, rows, cols, ids,
                                                                (__half*)out, bad_ids);
      break;
    default:
      return fail(MRB_ERR_ARG, "embed_rows: bad out_dtype %d", out_dtype);
  }
  return launch_status("embed_rows");
}
