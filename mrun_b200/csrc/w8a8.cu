// W8A8 QStore linear: per-token dynamic int8 activations, exact int32 accumulation on the
// integer tensor pipe, fp32 rescale.
//
// Follows `w8a8_matmul` / `_int8_gemm` (engine/kernels/w8a8.py:33-125):
//   act_scale = max|x_row| / 127 (IEEE fp32 division; 0 -> 1)
//   q_x       = clamp(round_half_even(x / act_scale), -127, 127)   (true division)
//   acc       = q_x . q_w^T in int32 (exact: |acc| <= 127 * 127 * K < 2^31 for K < 133k)
//   y         = side + (float(acc) * act_scale) * w_scale          (left to right)
// where `side` is the exact fp32 path of protected (outlier) columns, zero when none.
// Because the int32 sum is exact and every later step is one IEEE operation in the same
// order, y is bit-identical to the reference whenever side is zero.
//
// Decode sizes (M <= 16): a weight-streaming GEMV (per-thread cp.async ring, PDL prologue
// overlap) that quantises the activations in each CTA and feeds int8 codes straight to
// mma.sync m16n8k32 s8 -- no per-element weight conversion at all.
// Larger M: a tiled int8 GEMM over activations quantised once by mrb_w8a8_quantize.
#include "qrow_common.cuh"

#include <algorithm>
#include <type_traits>

namespace mrb {

__device__ __forceinline__ void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// reference activation quantiser for one value
__device__ __forceinline__ int8_t quant_act(float x, float scale) {
  float q = rintf(__fdiv_rn(x, scale));
  q = fminf(fmaxf(q, -127.f), 127.f);
  return static_cast<int8_t>(q);
}

__device__ __forceinline__ float act_scale_of(float amax) {
  const float s = __fdiv_rn(amax, 127.0f);
  return s == 0.0f ? 1.0f : s;
}

template <typename XT>
__device__ __forceinline__ float load_x(const XT* p) {
  return io<XT>::load(p);
}

// ------------------------------------------------------------------ activation quantiser

// One CTA per activation row. keep (fp32 [k], may be null) multiplies x first: protected
// columns carry 0 there, as the reference zeroes them before taking the scale.
template <typename XT>
__global__ void __launch_bounds__(256) w8a8_quantize_kernel(const XT* __restrict__ x, int64_t k,
                                                            const float* __restrict__ keep, int8_t* __restrict__ qx,
                                                            float* __restrict__ act_scale) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const XT* src = x + row * k;
  float m = 0.f;
  for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
    float v = load_x(src + c);
    if (keep) v = __fmul_rn(v, keep[c]);
    m = fmaxf(m, fabsf(v));
  }
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
  const float scale = act_scale_of(red[0]);
  if (threadIdx.x == 0) act_scale[row] = scale;
  int8_t* dst = qx + row * k;
  for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
    float v = load_x(src + c);
    if (keep) v = __fmul_rn(v, keep[c]);
    dst[c] = quant_act(v, scale);
  }
}

// bf16 rows without a keep mask, k % 8 == 0, k <= 256 * 8 * MAXV: the row is read once with
// 16-byte loads and held in registers between the max and the quantise pass; 8-byte stores.
// Same arithmetic as w8a8_quantize_kernel, element for element.
template <int MAXV>
__global__ void __launch_bounds__(256) w8a8_quantize_bf16_vec_kernel(const __nv_bfloat16* __restrict__ x, int64_t k,
                                                                     int8_t* __restrict__ qx,
                                                                     float* __restrict__ act_scale) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int nv = (int)(k / 8);
  const uint4* src = reinterpret_cast<const uint4*>(x + row * k);
  uint4 v[MAXV];
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int idx = threadIdx.x + i * 256;
    if (idx < nv) {
      v[i] = __ldg(src + idx);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(__bfloat162float(h[j])));
    }
  }
  __shared__ float red[8];
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float scale = act_scale_of(red[0]);
  if (threadIdx.x == 0) act_scale[row] = scale;
  uint2* dst = reinterpret_cast<uint2*>(qx + row * k);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int idx = threadIdx.x + i * 256;
    if (idx < nv) {
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&v[i]);
      __align__(8) int8_t q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) q[j] = quant_act(__bfloat162float(h[j]), scale);
      dst[idx] = *reinterpret_cast<const uint2*>(q);
    }
  }
}
constexpr int QV_MAXV = 10;  // k <= 20480 on the vector path

// ------------------------------------------------------------------ protected side path

// side[m, n] = sum_{p in idx, in list order} x[m, p] * (q_w[n, p] * w_scale[n]) in fp32:
// the exact fp32 path of the protected (outlier) columns (engine/kernels/w8a8.py:107-116).
template <typename XT>
__global__ void w8a8_side_kernel(const XT* __restrict__ x, int64_t m, int64_t k, const int8_t* __restrict__ qw,
                                 const float* __restrict__ sw, int64_t n, const int64_t* __restrict__ idx, int nidx,
                                 float* __restrict__ side) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= m * n) return;
  const int64_t mi = e / n, ni = e - mi * n;
  float acc = 0.f;
  for (int j = 0; j < nidx; ++j) {
    const int64_t p = idx[j];
    const float w = __fmul_rn(static_cast<float>(qw[ni * k + p]), sw[ni]);
    acc = fmaf(load_x(x + mi * k + p), w, acc);
  }
  side[e] = acc;
}

// ------------------------------------------------------------------ decode GEMV

constexpr int A8_WARPS = 8;
constexpr int A8_THREADS = A8_WARPS * 32;
constexpr int A8_ROWS = 16;
constexpr int A8_KB = 64;
constexpr int A8_STAGES = 8;
constexpr int A8_STAGE_BYTES = 2 * A8_THREADS * 16;

struct A8Args {
  const void* x;
  int64_t m, k;
  const int8_t* qw;
  const float* sw;
  int64_t n;
  const float* keep;  // [k] or null
  const float* side;  // [m, n] fp32 or null
  float* y;           // [m, n] fp32
  int32_t* acc_out;   // [m, n] int32 or null
  float* scale_out;   // [m] or null
};

__host__ __device__ inline int a8_kpad(int64_t k) { return (int)(((k + A8_KB - 1) / A8_KB) * A8_KB); }
__host__ __device__ inline int a8_xstride(int64_t k) { return a8_kpad(k) + 16; }  // bytes per column, +16

__host__ inline size_t a8_smem_bytes(int m, int64_t k, int nt) {
  size_t xs = (size_t)m * a8_xstride(k);
  xs = (xs + 15) & ~size_t(15);
  return (size_t)A8_STAGES * A8_STAGE_BYTES + xs + (size_t)A8_WARPS * A8_ROWS * 8 * nt * 4 + 64 * 4;
}

template <typename XT, int NT>
__global__ void __launch_bounds__(A8_THREADS, 2) w8a8_gemv_kernel(A8Args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int M = (int)a.m;
  const int64_t K = a.k, n = a.n;
  const int kpad = a8_kpad(K), xstride = a8_xstride(K);
  const int nkb = kpad / A8_KB;
  unsigned char* ring = smem;
  int8_t* xs = reinterpret_cast<int8_t*>(smem + A8_STAGES * A8_STAGE_BYTES);
  const size_t xs_bytes = ((size_t)M * xstride + 15) & ~size_t(15);
  int* red = reinterpret_cast<int*>(smem + A8_STAGES * A8_STAGE_BYTES + xs_bytes);
  float* rowscale = reinterpret_cast<float*>(red + A8_WARPS * A8_ROWS * 8 * NT);
  unsigned* rowmax = reinterpret_cast<unsigned*>(rowscale + 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int ntiles = (int)((n + A8_ROWS - 1) / A8_ROWS);
  const int kpw = warp < nkb ? (nkb - warp + A8_WARPS - 1) / A8_WARPS : 0;

  pdl_launch_dependents();
  int pf_T = kpw > 0 ? (int)blockIdx.x : ntiles, pf_i = 0, slot_w = 0;
  auto issue = [&]() {
    if (pf_T < ntiles) {
      const int kb = warp + A8_WARPS * pf_i;
      const int koff = kb * A8_KB + 16 * c;
      const bool ok = koff < K;
      const int64_t r0 = min((int64_t)pf_T * A8_ROWS + g, n - 1);
      const int64_t r1 = min((int64_t)pf_T * A8_ROWS + g + 8, n - 1);
      unsigned char* st = ring + slot_w * A8_STAGE_BYTES;
      cp_async16_zfill(st + tid * 16, a.qw + (ok ? r0 * K + koff : 0), ok);
      cp_async16_zfill(st + (A8_THREADS + tid) * 16, a.qw + (ok ? r1 * K + koff : 0), ok);
      if (++pf_i == kpw) {
        pf_i = 0;
        pf_T += gridDim.x;
      }
    }
    cp_async_commit_group();
    slot_w = slot_w + 1 == A8_STAGES ? 0 : slot_w + 1;
  };
#pragma unroll
  for (int p = 0; p < A8_STAGES - 1; ++p) issue();

  // ---- activations: per-row amax, the reference scale, int8 codes (identical in every CTA)
  pdl_wait();
  const XT* x = reinterpret_cast<const XT*>(a.x);
  if (tid < 16) rowmax[tid] = 0u;
  __syncthreads();
  for (int mi = 0; mi < M; ++mi) {
    float mx = 0.f;
    for (int64_t kk = tid; kk < K; kk += A8_THREADS) {
      float v = load_x(x + mi * K + kk);
      if (a.keep) v = __fmul_rn(v, a.keep[kk]);
      mx = fmaxf(mx, fabsf(v));
    }
    mx = warp_max(mx);
    if (lane == 0) atomicMax(&rowmax[mi], __float_as_uint(mx));
  }
  __syncthreads();
  if (tid < M) {
    rowscale[tid] = act_scale_of(__uint_as_float(rowmax[tid]));
    if (a.scale_out && blockIdx.x == 0) a.scale_out[tid] = rowscale[tid];
  }
  __syncthreads();
  for (int64_t e = tid; e < (int64_t)M * kpad; e += A8_THREADS) {
    const int mi = (int)(e / kpad);
    const int kk = (int)(e - (int64_t)mi * kpad);
    int8_t q = 0;
    if (kk < K) {
      float v = load_x(x + mi * K + kk);
      if (a.keep) v = __fmul_rn(v, a.keep[kk]);
      q = quant_act(v, rowscale[mi]);
    }
    xs[mi * xstride + kk] = q;
  }
  __syncthreads();

  int acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0;

  int slot_r = 0;
  for (int T = blockIdx.x; T < ntiles; T += gridDim.x) {
    for (int i = 0; i < kpw; ++i) {
      cp_async_wait_group<A8_STAGES - 2>();
      const unsigned char* st = ring + slot_r * A8_STAGE_BYTES;
      slot_r = slot_r + 1 == A8_STAGES ? 0 : slot_r + 1;
      const uint4 wa = *reinterpret_cast<const uint4*>(st + tid * 16);
      const uint4 wb = *reinterpret_cast<const uint4*>(st + (A8_THREADS + tid) * 16);
      issue();
      const int kb = warp + A8_WARPS * i;
      uint32_t xb[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int col = t * 8 + g;
        if (col < M) {
          const uint4 v = *reinterpret_cast<const uint4*>(xs + col * xstride + kb * A8_KB + 16 * c);
          xb[t][0] = v.x; xb[t][1] = v.y; xb[t][2] = v.z; xb[t][3] = v.w;
        } else {
          xb[t][0] = xb[t][1] = xb[t][2] = xb[t][3] = 0u;
        }
      }
      const uint32_t ra[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t rb[4] = {wb.x, wb.y, wb.z, wb.w};
      // two k32 steps per 64-byte block; each lane feeds its own 4-byte words (same k order
      // for weights and activations, so the permutation cancels in the dot product)
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int t = 0; t < NT; ++t)
          mma_s8(acc[t], ra[2 * j], rb[2 * j], ra[2 * j + 1], rb[2 * j + 1], xb[t][2 * j], xb[t][2 * j + 1]);
    }
    // ---- tile end: exact int32 reduction, then the reference rescale
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      int* base = red + (warp * A8_ROWS) * (8 * NT);
      const int col = t * 8 + 2 * c;
      base[g * (8 * NT) + col] = acc[t][0];
      base[g * (8 * NT) + col + 1] = acc[t][1];
      base[(g + 8) * (8 * NT) + col] = acc[t][2];
      base[(g + 8) * (8 * NT) + col + 1] = acc[t][3];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[t][i] = 0;
    }
    __syncthreads();
    for (int idx = tid; idx < A8_ROWS * M; idx += A8_THREADS) {
      const int row = idx % A8_ROWS, mi = idx / A8_ROWS;
      const int64_t nrow = (int64_t)T * A8_ROWS + row;
      if (nrow >= n) continue;
      int tot = 0;
#pragma unroll
      for (int w = 0; w < A8_WARPS; ++w) tot += red[(w * A8_ROWS + row) * (8 * NT) + mi];
      const int64_t o = (int64_t)mi * n + nrow;
      if (a.acc_out) a.acc_out[o] = tot;
      const float v = __fmul_rn(__fmul_rn(__int2float_rn(tot), rowscale[mi]), a.sw[nrow]);
      a.y[o] = a.side ? __fadd_rn(a.side[o], v) : v;
    }
    __syncthreads();
  }
  cp_async_wait_group<0>();
}

// ------------------------------------------------------------------ prefill int8 GEMM

constexpr int I8_BN = 128, I8_BM = 128, I8_BK = 64, I8_STAGES = 4, I8_THREADS = 256;
constexpr int I8_W_STAGE = I8_BN * I8_BK;
constexpr int I8_X_STAGE = I8_BM * I8_BK;
constexpr int I8_SMEM = I8_STAGES * (I8_W_STAGE + I8_X_STAGE);

struct I8GemmArgs {
  const int8_t* qx;  // [m, k]
  const int8_t* qw;  // [n, k]
  int64_t m, n, k;
  const float* act_scale;  // [m] or null (then y is not written)
  const float* sw;         // [n]
  const float* side;       // [m, n] or null
  float* y;                // [m, n] or null
  int32_t* acc_out;        // [m, n] or null
};

// 128x128 tiles, 8 warps (4 over weight rows x 2 over tokens), 4-stage cp.async ring;
// exact int32 accumulation with mma.sync m16n8k32 s8. Shared rows: weights 64 bytes
// (conflict-free 16-byte lane reads), activations 64 bytes with an XOR swizzle.
__global__ void __launch_bounds__(I8_THREADS, 1) int8_gemm_kernel(I8GemmArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* ws = smem;
  unsigned char* xsb = smem + I8_STAGES * I8_W_STAGE;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int wn = warp & 3, wm = warp >> 2;
  const int64_t n0 = (int64_t)blockIdx.x * I8_BN, m0 = (int64_t)blockIdx.y * I8_BM;
  const int64_t K = a.k;
  const int nkb = (int)((K + I8_BK - 1) / I8_BK);
  pdl_launch_dependents();
  pdl_wait();

  auto load_stage = [&](int stage, int kb) {
    const int64_t kbase = (int64_t)kb * I8_BK;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * I8_THREADS;
      const int r = idx >> 2, ch = idx & 3;
      const int64_t row = min(n0 + r, a.n - 1);
      const int64_t kk = kbase + ch * 16;
      const bool ok = kk < K;
      cp_async16_zfill(ws + stage * I8_W_STAGE + r * I8_BK + ch * 16, a.qw + (ok ? row * K + kk : 0), ok);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * I8_THREADS;
      const int r = idx >> 2, ch = idx & 3;
      const int64_t tok = m0 + r;
      const int64_t kk = kbase + ch * 16;
      const bool ok = tok < a.m && kk < K;
      cp_async16_zfill(xsb + stage * I8_X_STAGE + r * I8_BK + ((ch ^ ((r >> 1) & 3)) * 16),
                       a.qx + (ok ? tok * K + kk : 0), ok);
    }
  };

  int acc[2][8][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int t = 0; t < 4; ++t) acc[i][j][t] = 0;

#pragma unroll
  for (int s = 0; s < I8_STAGES - 1; ++s) {
    if (s < nkb) load_stage(s, s);
    cp_async_commit_group();
  }
  for (int kb = 0; kb < nkb; ++kb) {
    cp_async_wait_group<I8_STAGES - 2>();
    __syncthreads();
    {
      const int nk = kb + I8_STAGES - 1;
      if (nk < nkb) load_stage(nk % I8_STAGES, nk);
      cp_async_commit_group();
    }
    const int stage = kb % I8_STAGES;
    const unsigned char* wst = ws + stage * I8_W_STAGE;
    const unsigned char* xst = xsb + stage * I8_X_STAGE;
    uint32_t af[2][2][4];  // [mt][row half][4 words]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int r = wn * 32 + mt * 16 + g;
      const uint4 lo = *reinterpret_cast<const uint4*>(wst + r * I8_BK + 16 * c);
      const uint4 hi = *reinterpret_cast<const uint4*>(wst + (r + 8) * I8_BK + 16 * c);
      af[mt][0][0] = lo.x; af[mt][0][1] = lo.y; af[mt][0][2] = lo.z; af[mt][0][3] = lo.w;
      af[mt][1][0] = hi.x; af[mt][1][1] = hi.y; af[mt][1][2] = hi.z; af[mt][1][3] = hi.w;
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int r = wm * 64 + nt * 8 + g;
      const uint4 b = *reinterpret_cast<const uint4*>(xst + r * I8_BK + ((c ^ ((r >> 1) & 3)) * 16));
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
          mma_s8(acc[mt][nt], af[mt][0][2 * j], af[mt][1][2 * j], af[mt][0][2 * j + 1], af[mt][1][2 * j + 1],
                 bw[2 * j], bw[2 * j + 1]);
    }
  }
  cp_async_wait_group<0>();
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int64_t row = n0 + wn * 32 + mt * 16 + g + half * 8;
      if (row >= a.n) continue;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int64_t tok = m0 + wm * 64 + nt * 8 + 2 * c + e;
          if (tok >= a.m) continue;
          const int tot = acc[mt][nt][half * 2 + e];
          const int64_t o = tok * a.n + row;
          if (a.acc_out) a.acc_out[o] = tot;
          if (a.y) {
            const float v = __fmul_rn(__fmul_rn(__int2float_rn(tot), a.act_scale[tok]), a.sw[row]);
            a.y[o] = a.side ? __fadd_rn(a.side[o], v) : v;
          }
        }
    }
}

int tc_int8_gemm(const int8_t* qx, const int8_t* qw, int64_t m, int64_t n, int64_t k, const float* act_scale,
                 const float* sw, const float* side, float* y, int32_t* acc_out, cudaStream_t s);
int tc_int8_gemm_ex(const int8_t* qx, const int8_t* qw, const int8_t* qw_up, int64_t m, int64_t n, int64_t k,
                    const float* act_scale, const float* sw, const float* sw_up, const float* side,
                    const float* bias, float* y, __nv_bfloat16* y_bf16, int32_t* acc_out, cudaStream_t s);

static int launch_int8_gemm(const I8GemmArgs& a, cudaStream_t s) {
  return tc_int8_gemm(a.qx, a.qw, a.m, a.n, a.k, a.act_scale, a.sw, a.side, a.y, a.acc_out, s);
}

[[maybe_unused]] static int launch_int8_gemm_mma_sync(const I8GemmArgs& a, cudaStream_t s) {
  const int smem_st = ensure_dynamic_smem((const void*)int8_gemm_kernel, I8_SMEM, "int8 gemm");
  if (smem_st) return smem_st;
  const int64_t gx = (a.n + I8_BN - 1) / I8_BN, gy = (a.m + I8_BM - 1) / I8_BM;
  if (gy > 65535) return fail(MRB_ERR_UNSUPPORTED, "int8 gemm: too many activation rows");
  cudaError_t e = launch_kernel(int8_gemm_kernel, dim3((unsigned)gx, (unsigned)gy), dim3(I8_THREADS), I8_SMEM, s,
                                true, a);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "int8 gemm: launch: %s", cudaGetErrorString(e));
  return launch_status("int8 gemm");
}

template <typename XT, int NT>
static int launch_a8_gemv(const A8Args& a, cudaStream_t s) {
  const size_t smem = a8_smem_bytes((int)a.m, a.k, NT);
  if (smem > 227 * 1024)
    return fail(MRB_ERR_UNSUPPORTED, "w8a8 gemv: activation block %lld x %lld too large", (long long)a.m,
                (long long)a.k);
  auto kern = w8a8_gemv_kernel<XT, NT>;
  const int smem_st = ensure_dynamic_smem((const void*)kern, smem, "w8a8 gemv");
  if (smem_st) return smem_st;
  const int per_sm = 2 * (smem + 1024) <= 227 * 1024 ? 2 : 1;
  const int64_t ntiles = (a.n + A8_ROWS - 1) / A8_ROWS;
  const int64_t grid = std::min<int64_t>(ntiles, (int64_t)num_sms() * per_sm);
  cudaError_t e = launch_kernel(kern, dim3((unsigned)grid), dim3(A8_THREADS), smem, s, true, a);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "w8a8 gemv: launch: %s", cudaGetErrorString(e));
  return launch_status("w8a8 gemv");
}

template <typename XT>
static int launch_quantize(const void* x, int64_t m, int64_t k, const float* keep, int8_t* qx, float* scale,
                           cudaStream_t s) {
  if (std::is_same<XT, __nv_bfloat16>::value && !keep && k % 8 == 0 && k <= 256 * 8 * QV_MAXV &&
      aligned(x, 16) && aligned(qx, 8)) {
    launch_kernel(w8a8_quantize_bf16_vec_kernel<QV_MAXV>, dim3((unsigned)m), dim3(256), 0, s, true,
                  (const __nv_bfloat16*)x, k, qx, scale);
    return launch_status("w8a8 quantize");
  }
  launch_kernel(w8a8_quantize_kernel<XT>, dim3((unsigned)m), dim3(256), 0, s, true, (const XT*)x, k, keep, qx, scale);
  return launch_status("w8a8 quantize");
}

static int quantize_dispatch(const void* x, int x_dtype, int64_t m, int64_t k, const float* keep, int8_t* qx,
                             float* scale, cudaStream_t s) {
  switch (x_dtype) {
    case MRB_F32: return launch_quantize<float>(x, m, k, keep, qx, scale, s);
    case MRB_BF16: return launch_quantize<__nv_bfloat16>(x, m, k, keep, qx, scale, s);
    case MRB_F16: return launch_quantize<__half>(x, m, k, keep, qx, scale, s);
    default: return fail(MRB_ERR_ARG, "w8a8: bad x_dtype %d", x_dtype);
  }
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_w8a8_quantize(const void* x, int x_dtype, int64_t m, int64_t k, const float* keep, int8_t* qx,
                                 float* act_scale, void* stream) {
  if (m < 0 || k <= 0) return fail(MRB_ERR_ARG, "w8a8_quantize: bad shape");
  if (m == 0) return MRB_OK;
  if (!x || !qx || !act_scale) return fail(MRB_ERR_ARG, "w8a8_quantize: null pointer");
  if (m > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "w8a8_quantize: too many rows");
  return quantize_dispatch(x, x_dtype, m, k, keep, qx, act_scale, (cudaStream_t)stream);
}

extern "C" int mrb_int8_gemm(const int8_t* qx, const int8_t* qw, int64_t m, int64_t n, int64_t k, int32_t* acc,
                             void* stream) {
  if (m < 0 || n <= 0 || k <= 0) return fail(MRB_ERR_ARG, "int8_gemm: bad shape");
  if (m == 0) return MRB_OK;
  if (!qx || !qw || !acc) return fail(MRB_ERR_ARG, "int8_gemm: null pointer");
  if (k % 16) return fail(MRB_ERR_UNSUPPORTED, "int8_gemm: k %lld is not a multiple of 16", (long long)k);
  if (!aligned(qx, 16) || !aligned(qw, 16)) return fail(MRB_ERR_ARG, "int8_gemm: operands must be 16-byte aligned");
  if (k > 133000) return fail(MRB_ERR_UNSUPPORTED, "int8_gemm: k %lld could overflow int32", (long long)k);
  I8GemmArgs a{qx, qw, m, n, k, nullptr, nullptr, nullptr, nullptr, acc};
  return launch_int8_gemm(a, (cudaStream_t)stream);
}

extern "C" int mrb_w8a8_matmul(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* qw, const float* sw,
                               int64_t n, const int64_t* protect_idx, int nprotect, const float* keep, float* y,
                               int32_t* acc_out, int8_t* qx_ws, float* scale_ws, float* side_ws, void* stream) {
  if (m < 0 || k <= 0 || n <= 0 || nprotect < 0) return fail(MRB_ERR_ARG, "w8a8_matmul: bad shape");
  if (m == 0) return MRB_OK;
  if (!x || !qw || !sw || !y) return fail(MRB_ERR_ARG, "w8a8_matmul: null pointer");
  if (k % 16) return fail(MRB_ERR_UNSUPPORTED, "w8a8_matmul: k %lld is not a multiple of 16", (long long)k);
  if (!aligned(qw, 16)) return fail(MRB_ERR_ARG, "w8a8_matmul: weights must be 16-byte aligned");
  if (k > 133000) return fail(MRB_ERR_UNSUPPORTED, "w8a8_matmul: k %lld could overflow int32", (long long)k);
  if (nprotect > 0 && (!protect_idx || !keep || !side_ws))
    return fail(MRB_ERR_ARG, "w8a8_matmul: protected columns need idx, keep mask and side workspace");
  cudaStream_t s = (cudaStream_t)stream;
  if (nprotect > 0) {
    const int64_t total = m * n;
    const int64_t blocks = (total + 255) / 256;
    switch (x_dtype) {
      case MRB_F32:
        launch_kernel(w8a8_side_kernel<float>, dim3((unsigned)blocks), dim3(256), 0, s, true, (const float*)x, m, k, qw, sw,
                      n, protect_idx, nprotect, side_ws);
        break;
      case MRB_BF16:
        launch_kernel(w8a8_side_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, s, true,
                      (const __nv_bfloat16*)x, m, k, qw, sw, n, protect_idx, nprotect, side_ws);
        break;
      case MRB_F16:
        launch_kernel(w8a8_side_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, s, true, (const __half*)x, m, k,
                      qw, sw, n, protect_idx, nprotect, side_ws);
        break;
      default:
        return fail(MRB_ERR_ARG, "w8a8_matmul: bad x_dtype %d", x_dtype);
    }
    const int st = launch_status("w8a8 side path");
    if (st) return st;
  }
  const float* side = nprotect > 0 ? side_ws : nullptr;
  if (m <= 16 && a8_smem_bytes((int)m, k, m <= 8 ? 1 : 2) <= 227 * 1024) {
    A8Args a{x, m, k, qw, sw, n, nprotect > 0 ? keep : nullptr, side, y, acc_out, scale_ws};
    const bool small_nt = m <= 8;
    switch (x_dtype) {
      case MRB_F32: return small_nt ? launch_a8_gemv<float, 1>(a, s) : launch_a8_gemv<float, 2>(a, s);
      case MRB_BF16: return small_nt ? launch_a8_gemv<__nv_bfloat16, 1>(a, s) : launch_a8_gemv<__nv_bfloat16, 2>(a, s);
      case MRB_F16: return small_nt ? launch_a8_gemv<__half, 1>(a, s) : launch_a8_gemv<__half, 2>(a, s);
      default: return fail(MRB_ERR_ARG, "w8a8_matmul: bad x_dtype %d", x_dtype);
    }
  }
  if (!qx_ws || !scale_ws) return fail(MRB_ERR_ARG, "w8a8_matmul: this size needs qx/scale workspaces");
  if (!aligned(qx_ws, 16)) return fail(MRB_ERR_ARG, "w8a8_matmul: qx workspace must be 16-byte aligned");
  int st = quantize_dispatch(x, x_dtype, m, k, nprotect > 0 ? keep : nullptr, qx_ws, scale_ws, s);
  if (st) return st;
  I8GemmArgs a{qx_ws, qw, m, n, k, scale_ws, sw, side, y, acc_out};
  return launch_int8_gemm(a, s);
}

extern "C" int mrb_w8a8_linear_bf16(const void* x_bf16, int64_t m, int64_t k, const int8_t* codes,
                                    const float* scales, const int8_t* up_codes, const float* up_scales,
                                    const float* bias, int64_t n, void* y_bf16, int8_t* qx_ws, float* scale_ws,
                                    void* stream) {
  if (m < 0 || k <= 0 || n <= 0) return fail(MRB_ERR_ARG, "w8a8_linear: bad shape");
  if (m == 0) return MRB_OK;
  if (!x_bf16 || !codes || !scales || !y_bf16 || !qx_ws || !scale_ws)
    return fail(MRB_ERR_ARG, "w8a8_linear: null pointer");
  if ((up_codes == nullptr) != (up_scales == nullptr))
    return fail(MRB_ERR_ARG, "w8a8_linear: up codes and up scales go together");
  if (up_codes && bias) return fail(MRB_ERR_ARG, "w8a8_linear: the paired SwiGLU takes no bias");
  if (k % 16) return fail(MRB_ERR_UNSUPPORTED, "w8a8_linear: k %lld is not a multiple of 16", (long long)k);
  if (k > 133000) return fail(MRB_ERR_UNSUPPORTED, "w8a8_linear: k %lld could overflow int32", (long long)k);
  if (!aligned(codes, 16) || !aligned(qx_ws, 16) || (up_codes && !aligned(up_codes, 16)))
    return fail(MRB_ERR_ARG, "w8a8_linear: codes and the qx workspace must be 16-byte aligned");
  cudaStream_t s = (cudaStream_t)stream;
  int st = quantize_dispatch(x_bf16, MRB_BF16, m, k, nullptr, qx_ws, scale_ws, s);
  if (st) return st;
  return tc_int8_gemm_ex(qx_ws, codes, up_codes, m, n, k, scale_ws, scales, up_scales, nullptr, bias, nullptr,
                         (__nv_bfloat16*)y_bf16, nullptr, s);
}

// ------------------------------------------------------------------ outlier column selection

namespace mrb {
// Column max |x| over all rows, then the top `topk` columns (largest first, lower column on
// ties) by repeated block arg-max; keep[col] = 0 for the chosen columns, 1 elsewhere.
// Follows the protect_k branch of `w8a8_matmul` (engine/kernels/w8a8.py:98-105).
template <typename XT>
__global__ void __launch_bounds__(1024) w8a8_topk_kernel(const XT* __restrict__ x, int64_t m, int64_t k, int topk,
                                                         int64_t* __restrict__ idx_out, float* __restrict__ keep) {
  extern __shared__ float colmax[];
  __shared__ float bv[32];
  __shared__ int bi[32];
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
    float mx = 0.f;
    for (int64_t r = 0; r < m; ++r) mx = fmaxf(mx, fabsf(io<XT>::load(x + r * k + c)));
    colmax[c] = mx;
    keep[c] = 1.0f;
  }
  __syncthreads();
  for (int t = 0; t < topk; ++t) {
    float best = -1.f;
    int besti = 0x7fffffff;
    for (int64_t c = threadIdx.x; c < k; c += blockDim.x) {
      const float v = colmax[c];
      if (v > best || (v == best && (int)c < besti)) {
        best = v;
        besti = (int)c;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (ov > best || (ov == best && oi < besti)) {
        best = ov;
        besti = oi;
      }
    }
    if ((threadIdx.x & 31) == 0) {
      bv[threadIdx.x >> 5] = best;
      bi[threadIdx.x >> 5] = besti;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int nw = blockDim.x >> 5;
      best = threadIdx.x < nw ? bv[threadIdx.x] : -1.f;
      besti = threadIdx.x < nw ? bi[threadIdx.x] : 0x7fffffff;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
        if (ov > best || (ov == best && oi < besti)) {
          best = ov;
          besti = oi;
        }
      }
      if (threadIdx.x == 0) {
        idx_out[t] = besti;
        keep[besti] = 0.0f;
        colmax[besti] = -2.0f;  // never chosen again
      }
    }
    __syncthreads();
  }
}
}  // namespace mrb

extern "C" int mrb_w8a8_protect_topk(const void* x, int x_dtype, int64_t m, int64_t k, int topk, int64_t* idx_out,
                                     float* keep, void* stream) {
  if (m <= 0 || k <= 0 || topk < 0 || topk > k) return fail(MRB_ERR_ARG, "w8a8_protect_topk: bad shape");
  if (!x || !keep || (topk > 0 && !idx_out)) return fail(MRB_ERR_ARG, "w8a8_protect_topk: null pointer");
  const size_t smem = (size_t)k * sizeof(float);
  if (smem > 200 * 1024) return fail(MRB_ERR_UNSUPPORTED, "w8a8_protect_topk: k %lld too large", (long long)k);
  cudaStream_t s = (cudaStream_t)stream;
  auto run = [&](auto kern) -> int {
    return ensure_dynamic_smem((const void*)kern, smem, "w8a8_protect_topk");
  };
  int st = MRB_OK;
  switch (x_dtype) {
    case MRB_F32:
      st = run(w8a8_topk_kernel<float>);
      if (!st) launch_kernel(w8a8_topk_kernel<float>, dim3(1), dim3(1024), smem, s, true, (const float*)x, m, k, topk,
                             idx_out, keep);
      break;
    case MRB_BF16:
      st = run(w8a8_topk_kernel<__nv_bfloat16>);
      if (!st) launch_kernel(w8a8_topk_kernel<__nv_bfloat16>, dim3(1), dim3(1024), smem, s, true,
                             (const __nv_bfloat16*)x, m, k, topk, idx_out, keep);
      break;
    case MRB_F16:
      st = run(w8a8_topk_kernel<__half>);
      if (!st) launch_kernel(w8a8_topk_kernel<__half>, dim3(1), dim3(1024), smem, s, true, (const __half*)x, m, k, topk,
                             idx_out, keep);
      break;
    default:
      return fail(MRB_ERR_ARG, "w8a8_protect_topk: bad x_dtype %d", x_dtype);
  }
  if (st) return st;
  return launch_status("w8a8_protect_topk");
}
