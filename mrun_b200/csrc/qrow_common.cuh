// Shared device helpers of the int8 qrow projection kernels.
#pragma once

#include "common.cuh"

namespace mrb {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Four signed int8 codes -> f16x2 of bytes (0,1) and f16x2 of bytes (2,3), exactly:
// the biased byte q + 128 placed under the f16 exponent of 1024 reads 1024 + q + 128.
__device__ __forceinline__ void i8x4_to_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  lo = hsub2(prmt(u, 0x64646464u, 0x4140u), 0x64806480u);  // (1024 + q + 128) - 1152
  hi = hsub2(prmt(u, 0x64646464u, 0x4342u), 0x64806480u);
}

// Four signed int8 codes -> bf16x2 of bytes (0,1) and bf16x2 of bytes (2,3), exactly: the
// biased byte under the fp32 exponent of 2^23 minus (2^23 + 128) is the code as an fp32
// integer, whose high half is its exact bf16.
__device__ __forceinline__ void i8x4_to_bf16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float f0 = __uint_as_float(prmt(u, 0x4B000000u, 0x7540u)) - 8388736.0f;
  const float f1 = __uint_as_float(prmt(u, 0x4B000000u, 0x7541u)) - 8388736.0f;
  const float f2 = __uint_as_float(prmt(u, 0x4B000000u, 0x7542u)) - 8388736.0f;
  const float f3 = __uint_as_float(prmt(u, 0x4B000000u, 0x7543u)) - 8388736.0f;
  lo = prmt(__float_as_uint(f0), __float_as_uint(f1), 0x7632u);
  hi = prmt(__float_as_uint(f2), __float_as_uint(f3), 0x7632u);
}

// Four signed int8 codes -> bf16x2 of bytes (0,1) and bf16x2 of bytes (2,3), exactly, in
// integer ops: the low seven bits m of each byte go under the bf16 exponent of 128 (128 + m,
// exact with 7 mantissa bits), and 128 (q >= 0) or 256 (q < 0, where m = q + 128) is
// subtracted in one bf16x2 sub, whose result q is exact.
__device__ __forceinline__ void i8x4_to_bf16x2_exact(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t mag = w & 0x7F7F7F7Fu;
  const uint32_t sgn = w & 0x80808080u;
  const uint32_t v01 = prmt(mag, 0x43434343u, 0x5140u), v23 = prmt(mag, 0x43434343u, 0x5342u);
  const uint32_t s01 = prmt(sgn, 0x43434343u, 0x5140u), s23 = prmt(sgn, 0x43434343u, 0x5342u);
  const __nv_bfloat162 d01 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v01),
                                     *reinterpret_cast<const __nv_bfloat162*>(&s01));
  const __nv_bfloat162 d23 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v23),
                                     *reinterpret_cast<const __nv_bfloat162*>(&s23));
  lo = *reinterpret_cast<const uint32_t*>(&d01);
  hi = *reinterpret_cast<const uint32_t*>(&d23);
}

// Four signed int8 codes -> f16x2 holding (q + 1152) for bytes (0,1) and (2,3), exactly:
// one xor and two byte permutes; the constant 1152 is removed after the dot product as
// 1152 * sum(x) (see the biased-code GEMV path).
__device__ __forceinline__ void i8x4_to_biased_f16x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  lo = prmt(u, 0x64646464u, 0x4140u);
  hi = prmt(u, 0x64646464u, 0x4342u);
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// SiLU as the reference writes it: g * sigmoid(g), sigmoid = 1 / (1 + exp(-g)).
__device__ __forceinline__ float silu_f32(float g) { return g * (1.0f / (1.0f + expf(-g))); }

// Order-preserving key: larger logit -> larger key; equal logits -> the lower row wins.
__device__ __forceinline__ unsigned long long pack_argmax(float v, int64_t row) {
  const unsigned u = __float_as_uint(v);
  const unsigned hi = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)hi << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)row);
}

__device__ __forceinline__ void cp_async16_zfill(void* smem, const void* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// Programmatic dependent launch: let the next kernel in the stream start its prologue, and
// wait for the previous kernel's results before reading them. Both are no-ops when the
// launch carried no programmatic dependency.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

}  // namespace mrb
