// Row RMSNorm and fused residual + RMSNorm with the reference's bf16 boundaries.
#include "qrow_common.cuh"

namespace mrb {

constexpr int NORM_THREADS = 512;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  const float r = red[32];
  __syncthreads();
  return r;
}

// y = (x * rsqrt(mean(x^2) + eps)) * w, fp32 math, stored in x's type.
// Follows `stable_rms_norm_reference` (engine/kernels/dense_qstore_cuda.py:1462-1470).
template <typename T>
__global__ void __launch_bounds__(NORM_THREADS) rms_norm_kernel(const T* __restrict__ x, int64_t width,
                                                                const float* __restrict__ w, float eps,
                                                                T* __restrict__ y) {
  __shared__ float red[33];
  pdl_launch_dependents();
  pdl_wait();
  const T* src = x + blockIdx.x * width;
  T* dst = y + blockIdx.x * width;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
    const float v = io<T>::load(src + i);
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(tot / (float)width + eps);
  for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
    const float v = io<T>::load(src + i);
    io<T>::store(dst + i, __fmul_rn(__fmul_rn(v, inv), w[i]));
  }
}

// r = bf16(residual + update) (fp32 add), normed = bf16(RMSNorm(r) * w).
// Follows `fused_residual_rms_norm_reference` (engine/kernels/dense_qstore_cuda.py:1390-1408).
// One pass: each thread keeps its (up to NORM_VPT) 8-element vectors in registers.
constexpr int NORM_VPT = 4;

__global__ void __launch_bounds__(NORM_THREADS) residual_rms_norm_vec_kernel(
    const __nv_bfloat16* res, const __nv_bfloat16* __restrict__ upd, int64_t width,
    const float* __restrict__ w, float eps, __nv_bfloat16* res_out,  // res_out may alias res
    __nv_bfloat16* __restrict__ normed) {
  __shared__ float red[33];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t base = blockIdx.x * width;
  const int nvec = (int)(width / 8);
  float r[NORM_VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NORM_VPT; ++j) {
    const int v = threadIdx.x + j * NORM_THREADS;
    if (v < nvec) {
      const uint4 a = *reinterpret_cast<const uint4*>(res + base + v * 8);
      const uint4 b = *reinterpret_cast<const uint4*>(upd + base + v * 8);
      const __nv_bfloat16* ae = reinterpret_cast<const __nv_bfloat16*>(&a);
      const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        r[j][i] = round_bf16(__fadd_rn(__bfloat162float(ae[i]), __bfloat162float(be[i])));
        ss = fmaf(r[j][i], r[j][i], ss);
      }
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(tot / (float)width + eps);
#pragma unroll
  for (int j = 0; j < NORM_VPT; ++j) {
    const int v = threadIdx.x + j * NORM_THREADS;
    if (v < nvec) {
      __align__(16) __nv_bfloat16 ro[8], no[8];
      const float4 w0 = *reinterpret_cast<const float4*>(w + v * 8);
      const float4 w1 = *reinterpret_cast<const float4*>(w + v * 8 + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ro[i] = __float2bfloat16_rn(r[j][i]);
        no[i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(r[j][i], inv), wv[i]));
      }
      *reinterpret_cast<uint4*>(res_out + base + v * 8) = *reinterpret_cast<const uint4*>(ro);
      *reinterpret_cast<uint4*>(normed + base + v * 8) = *reinterpret_cast<const uint4*>(no);
    }
  }
}

// Scalar fallback for widths that are not a multiple of 8 or exceed the register plan.
__global__ void __launch_bounds__(NORM_THREADS) residual_rms_norm_kernel(
    const __nv_bfloat16* res, const __nv_bfloat16* __restrict__ upd, int64_t width,
    const float* __restrict__ w, float eps, __nv_bfloat16* res_out,  // res_out may alias res
    __nv_bfloat16* __restrict__ normed) {
  __shared__ float red[33];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t base = blockIdx.x * width;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
    const float r = round_bf16(__fadd_rn(__bfloat162float(res[base + i]), __bfloat162float(upd[base + i])));
    ss = fmaf(r, r, ss);
  }
  const float tot = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(tot / (float)width + eps);
  for (int64_t i = threadIdx.x; i < width; i += blockDim.x) {
    const __nv_bfloat16 rb = __float2bfloat16_rn(__fadd_rn(__bfloat162float(res[base + i]), __bfloat162float(upd[base + i])));
    const float r = __bfloat162float(rb);
    res_out[base + i] = rb;
    normed[base + i] = __float2bfloat16_rn(__fmul_rn(__fmul_rn(r, inv), w[i]));
  }
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_rms_norm(const void* x, int dtype, int64_t rows, int64_t width, const float* weight,
                            float eps, void* y, void* stream) {
  if (!x || !weight || !y) return fail(MRB_ERR_ARG, "rms_norm: null pointer");
  if (rows < 0 || width <= 0) return fail(MRB_ERR_ARG, "rms_norm: bad shape");
  if (rows == 0) return MRB_OK;
  cudaStream_t s = (cudaStream_t)stream;
  switch (dtype) {
    case MRB_F32:
      launch_kernel(rms_norm_kernel<float>, dim3((unsigned)rows), dim3(NORM_THREADS), 0, s, true, (const float*)x, width,
                    weight, eps, (float*)y);
      break;
    case MRB_BF16:
      launch_kernel(rms_norm_kernel<__nv_bfloat16>, dim3((unsigned)rows), dim3(NORM_THREADS), 0, s, true,
                    (const __nv_bfloat16*)x, width, weight, eps, (__nv_bfloat16*)y);
      break;
    case MRB_F16:
      launch_kernel(rms_norm_kernel<__half>, dim3((unsigned)rows), dim3(NORM_THREADS), 0, s, true, (const __half*)x,
                    width, weight, eps, (__half*)y);
      break;
    default:
      return fail(MRB_ERR_ARG, "rms_norm: bad dtype %d", dtype);
  }
  return launch_status("rms_norm");
}

extern "C" int mrb_residual_rms_norm(const void* residual, const void* update, int64_t rows, int64_t width,
                                     const float* weight, float eps, void* residual_out, void* normed_out,
                                     void* stream) {
  if (!residual || !update || !weight || !residual_out || !normed_out)
    return fail(MRB_ERR_ARG, "residual_rms_norm: null pointer");
  if (rows < 0 || width <= 0) return fail(MRB_ERR_ARG, "residual_rms_norm: bad shape");
  if (rows == 0) return MRB_OK;
  const bool vec = width % 8 == 0 && width / 8 <= (int64_t)NORM_THREADS * NORM_VPT && aligned(residual, 16) &&
                   aligned(update, 16) && aligned(weight, 16) && aligned(residual_out, 16) && aligned(normed_out, 16);
  launch_kernel(vec ? residual_rms_norm_vec_kernel : residual_rms_norm_kernel, dim3((unsigned)rows),
                dim3(NORM_THREADS), 0, (cudaStream_t)stream, true, (const __nv_bfloat16*)residual,
                (const __nv_bfloat16*)update, width, weight, eps, (__nv_bfloat16*)residual_out,
                (__nv_bfloat16*)normed_out);
  return launch_status("residual_rms_norm");
}

