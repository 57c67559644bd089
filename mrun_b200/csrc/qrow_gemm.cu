// Prefill-size W8A16 projection: Y[m, n] = X[m, :] . (codes[n, :] * scale[n]) for m > 16.
//
// Tiled tensor-core GEMM (mma.sync m16n8k16, bf16 x bf16 -> fp32): a CTA computes a
// 128 (weight rows) x 128 (tokens) tile with 8 warps (4 x 2), streaming 64-wide k blocks of
// int8 weights and bf16 activations through a 4-stage cp.async ring. Weights are converted
// int8 -> bf16 exactly in registers (magic-number float, then the bf16 half of it); the
// activation tile is XOR-swizzled in shared memory so fragment loads are conflict-free.
// Within each 64-element k block the k order is permuted identically for both operands so
// every lane reads 16 contiguous bytes per row. The fp32 accumulator is scaled once per row.
#include "qrow_common.cuh"

#include <algorithm>

namespace mrb {

constexpr int GM_BN = 128;  // weight rows per CTA
constexpr int GM_BM = 128;  // tokens per CTA
constexpr int GM_BK = 64;
constexpr int GM_STAGES = 4;
constexpr int GM_THREADS = 256;
constexpr int GM_W_STAGE = GM_BN * GM_BK;      // int8 bytes
constexpr int GM_X_STAGE = GM_BM * GM_BK * 2;  // bf16 bytes
constexpr int GM_SMEM = GM_STAGES * (GM_W_STAGE + GM_X_STAGE);

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int bytes = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

struct GemmArgs {
  const __nv_bfloat16* x;  // [m, k]
  const int8_t* codes;     // [n, k] (gate codes when paired)
  const float* scales;     // [n]
  const int8_t* codes_up;  // paired SwiGLU: up codes [n, k]
  const float* scales_up;
  const float* bias;       // [n] or null
  __nv_bfloat16* y;        // [m, n]
  int64_t m, n, k;
};

// PAIRED: the CTA's 128 weight rows are 64 gate rows followed by the same 64 up rows, and the
// epilogue forms bf16(bf16(silu(bf16 g)) * bf16 u) for 64 output columns.
template <bool PAIRED>
__global__ void __launch_bounds__(GM_THREADS, 1) qrow_gemm_bf16_kernel(GemmArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  int8_t* ws = reinterpret_cast<int8_t*>(smem);
  unsigned char* xsb = smem + GM_STAGES * GM_W_STAGE;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int wn = warp & 3;   // 32-row slice of the weight tile
  const int wm = warp >> 2;  // 64-token slice of the activation tile
  const int64_t n0 = (int64_t)blockIdx.x * (PAIRED ? GM_BN / 2 : GM_BN);
  const int64_t m0 = (int64_t)blockIdx.y * GM_BM;
  const int64_t K = a.k;
  const int nkb = (int)((K + GM_BK - 1) / GM_BK);

  auto load_stage = [&](int stage, int kb) {
    const int64_t kbase = (int64_t)kb * GM_BK;
    // weights: 128 rows x 4 chunks of 16 B
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int idx = tid + i * GM_THREADS;
      const int r = idx >> 2, ch = idx & 3;
      const int rr = PAIRED ? (r & (GM_BN / 2 - 1)) : r;
      const int8_t* base = (PAIRED && r >= GM_BN / 2) ? a.codes_up : a.codes;
      const int64_t row = min(n0 + rr, a.n - 1);
      const int64_t kk = kbase + ch * 16;
      const bool ok = kk < K;
      cp_async16(ws + stage * GM_W_STAGE + r * GM_BK + ch * 16, base + row * K + (ok ? kk : 0), ok);
    }
    // activations: 128 tokens x 8 chunks of 16 B (8 bf16), swizzled
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = tid + i * GM_THREADS;
      const int r = idx >> 3, ch = idx & 7;
      const int64_t tok = m0 + r;
      const int64_t kk = kbase + ch * 8;
      const bool ok = tok < a.m && kk < K;
      const __nv_bfloat16* src = a.x + (ok ? tok * K + kk : 0);
      cp_async16(xsb + stage * GM_X_STAGE + r * (GM_BK * 2) + ((ch ^ (r & 7)) * 16), src, ok);
    }
  };

  float acc[2][8][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int t = 0; t < 4; ++t) acc[i][j][t] = 0.f;

#pragma unroll
  for (int s = 0; s < GM_STAGES - 1; ++s) {
    if (s < nkb) load_stage(s, s);
    cp_async_commit();
  }

  for (int kb = 0; kb < nkb; ++kb) {
    cp_async_wait<GM_STAGES - 2>();
    __syncthreads();
    {
      const int nk = kb + GM_STAGES - 1;
      if (nk < nkb) load_stage(nk % GM_STAGES, nk);
      cp_async_commit();
    }
    const int stage = kb % GM_STAGES;
    const int8_t* wst = ws + stage * GM_W_STAGE;
    const unsigned char* xst = xsb + stage * GM_X_STAGE;

    // A fragments for both 16-row tiles, all 4 k16 steps: [mt][j][4 regs]
    uint32_t af[2][4][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
      const int r = wn * 32 + mt * 16 + g;
      const uint4 lo = *reinterpret_cast<const uint4*>(wst + r * GM_BK + 16 * c);
      const uint4 hi = *reinterpret_cast<const uint4*>(wst + (r + 8) * GM_BK + 16 * c);
      const uint32_t wl[4] = {lo.x, lo.y, lo.z, lo.w};
      const uint32_t wh[4] = {hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        i8x4_to_bf16x2(wl[j], af[mt][j][0], af[mt][j][2]);
        i8x4_to_bf16x2(wh[j], af[mt][j][1], af[mt][j][3]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int r = wm * 64 + nt * 8 + g;
      const unsigned char* row = xst + r * (GM_BK * 2);
      const uint4 b0 = *reinterpret_cast<const uint4*>(row + (((2 * c) ^ (r & 7)) * 16));
      const uint4 b1 = *reinterpret_cast<const uint4*>(row + (((2 * c + 1) ^ (r & 7)) * 16));
      const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
          mma_bf16(acc[mt][nt], af[mt][j][0], af[mt][j][1], af[mt][j][2], af[mt][j][3], bw[2 * j], bw[2 * j + 1]);
    }
  }
  cp_async_wait<0>();

  if (!PAIRED) {
    // y[token, row] = bf16(acc * scale) (+ bf16 bias, rounded again)
#pragma unroll
    for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int64_t row = n0 + wn * 32 + mt * 16 + g + half * 8;
        if (row >= a.n) continue;
        const float sc = a.scales[row];
        const float bv = a.bias ? round_bf16(a.bias[row]) : 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int64_t tok = m0 + wm * 64 + nt * 8 + 2 * c + e;
            if (tok < a.m) {
              float v = acc[mt][nt][half * 2 + e] * sc;
              if (a.bias) v = round_bf16(v) + bv;
              a.y[tok * a.n + row] = __float2bfloat16_rn(v);
            }
          }
        }
      }
    }
    return;
  }
  // paired SwiGLU: gate warps (wn < 2) publish bf16 g through shared memory
  __syncthreads();
  float* gbuf = reinterpret_cast<float*>(smem);  // [64 rows][128 tokens]
  if (wn < 2) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int rl = wn * 32 + mt * 16 + g + half * 8;
        const int64_t row = min(n0 + rl, a.n - 1);
        const float sc = a.scales[row];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e)
            gbuf[rl * GM_BM + wm * 64 + nt * 8 + 2 * c + e] = round_bf16(acc[mt][nt][half * 2 + e] * sc);
      }
  }
  __syncthreads();
  if (wn >= 2) {
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int rl = (wn - 2) * 32 + mt * 16 + g + half * 8;
        const int64_t row = n0 + rl;
        if (row >= a.n) continue;
        const float sc = a.scales_up[row];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int tl = wm * 64 + nt * 8 + 2 * c + e;
            const int64_t tok = m0 + tl;
            if (tok < a.m) {
              const float gv = gbuf[rl * GM_BM + tl];
              const float uv = round_bf16(acc[mt][nt][half * 2 + e] * sc);
              const float sl = round_bf16(gv * (1.0f / (1.0f + expf(-gv))));
              a.y[tok * a.n + row] = __float2bfloat16_rn(sl * uv);
            }
          }
      }
  }
}

template <bool PAIRED>
static int launch_gemm(const GemmArgs& a, cudaStream_t s) {
  const int smem_st = ensure_dynamic_smem((const void*)qrow_gemm_bf16_kernel<PAIRED>, GM_SMEM, "qrow gemm");
  if (smem_st) return smem_st;
  const int64_t rows_per_cta = PAIRED ? GM_BN / 2 : GM_BN;
  const int64_t gx = (a.n + rows_per_cta - 1) / rows_per_cta;
  const int64_t gy = (a.m + GM_BM - 1) / GM_BM;
  if (gy > 65535) return fail(MRB_ERR_UNSUPPORTED, "qrow gemm: too many activation rows");
  qrow_gemm_bf16_kernel<PAIRED><<<dim3((unsigned)gx, (unsigned)gy), GM_THREADS, GM_SMEM, s>>>(a);
  return launch_status("qrow gemm");
}

int qrow_gemm_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                   int64_t n, const float* bias, __nv_bfloat16* y, cudaStream_t s) {
  GemmArgs a{x, codes, scales, nullptr, nullptr, bias, y, m, n, k};
  return launch_gemm<false>(a, s);
}

int qrow_gemm_swiglu_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* gate_codes,
                          const float* gate_scales, const int8_t* up_codes, const float* up_scales, int64_t n,
                          __nv_bfloat16* y, cudaStream_t s) {
  GemmArgs a{x, gate_codes, gate_scales, up_codes, up_scales, nullptr, y, m, n, k};
  return launch_gemm<true>(a, s);
}

}  // namespace mrb
