// Routed-MoE kernel chain: router softmax/top-k, deterministic route compilation
// (histogram -> exclusive scan -> stable expert-major permutation + inverse), grouped int8
// expert projections over ragged per-expert row counts (SwiGLU-fused gate/up, then down),
// and the fixed-rank weighted combine.
//
// References (mrun project paths):
//   router            engine/qwen3_moe_cuda.py:3700-3707 (softmax fp32 -> topk -> renorm -> bf16)
//   route compiler    engine/olmoe_cuda.py:989-1135 (CPU branch: stable argsort by expert)
//   expert pages      engine/qwen3_moe_cuda.py:187-231 (gate_up codes | scales | down codes | scales)
//   grouped GEMMs     engine/qwen3_moe_cuda.py:2740-2761 (rows[start:start+count] @ W_e.T, silu(g)*u)
//   stable reduce     engine/qwen3_moe_cuda.py:2561-2664 (fp32 products summed in route-rank order)
#include "qrow_common.cuh"

#include <algorithm>

namespace mrb {

// ------------------------------------------------------------------ router

// One warp per token: softmax over E logits in fp32 (max-subtracted exp, divided by the
// sum), then k rounds of arg-max (ties -> lower expert), optional renormalisation by the
// fp32 sum of the chosen probabilities, and the bf16 weights the reference hands on.
template <typename LT>
__global__ void router_topk_kernel(const LT* __restrict__ logits, int64_t tokens, int E, int k, int renorm,
                                   int64_t* __restrict__ top_idx, float* __restrict__ top_w_f32,
                                   __nv_bfloat16* __restrict__ top_w_bf16) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  constexpr int MAXE = 256;
  float p[MAXE / 32];
  const LT* row = logits + t * E;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < MAXE / 32; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? io<LT>::load(row + e) : -INFINITY;
    mx = fmaxf(mx, p[i]);
  }
  mx = warp_max(mx);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < MAXE / 32; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? expf(p[i] - mx) : 0.f;
    sum += p[i];
  }
  sum = warp_sum(sum);
#pragma unroll
  for (int i = 0; i < MAXE / 32; ++i) p[i] = (lane + 32 * i) < E ? p[i] / sum : -1.f;
  float chosen_sum = 0.f;
  float wsel[16];
  int isel[16];
  for (int j = 0; j < k; ++j) {
    float best = -2.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < MAXE / 32; ++i) {
      const int e = lane + 32 * i;
      if (p[i] > best || (p[i] == best && e < bi)) {
        best = p[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < MAXE / 32; ++i)
      if (lane + 32 * i == bi) p[i] = -2.f;  // taken
    if (j < 16) {
      wsel[j] = best;
      isel[j] = bi;
    }
    chosen_sum += best;
  }
  if (lane == 0) {
    for (int j = 0; j < k && j < 16; ++j) {
      const float w = renorm ? wsel[j] / chosen_sum : wsel[j];
      top_idx[t * k + j] = isel[j];
      if (top_w_f32) top_w_f32[t * k + j] = w;
      if (top_w_bf16) top_w_bf16[t * k + j] = __float2bfloat16_rn(w);
    }
  }
}

// ------------------------------------------------------------------ route compiler

// Single CTA of 1024 threads. Assignments are ranked in chunks of 1024 in flat (token,
// rank) order: inside a warp, peers with the same expert are found with match_any, warps
// are ordered through a per-warp histogram, and a running per-expert cursor carries the
// order across chunks -- exactly the stable expert-major order of the reference's CPU
// branch (argsort(experts, stable=True)), with no atomics deciding positions.
constexpr int RC_THREADS = 1024;
constexpr int RC_WARPS = RC_THREADS / 32;
constexpr int RC_MAXE = 512;

__global__ void __launch_bounds__(RC_THREADS) route_compile_kernel(
    const int64_t* __restrict__ top_idx, const float* __restrict__ top_w, int64_t assignments, int k, int E,
    int32_t* __restrict__ counts, int32_t* __restrict__ starts, int64_t* __restrict__ token_ids,
    float* __restrict__ coef, int64_t* __restrict__ inverse, int32_t* __restrict__ error_flag) {
  __shared__ int hist[RC_MAXE];
  __shared__ int cursor[RC_MAXE];
  __shared__ int whist[RC_WARPS][RC_MAXE / 4];  // reused per expert quarter
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E; e += RC_THREADS) hist[e] = 0;
  __syncthreads();
  for (int64_t a = tid; a < assignments; a += RC_THREADS) {
    const int64_t e = top_idx[a];
    if (e >= 0 && e < E) {
      atomicAdd(&hist[e], 1);
    } else if (error_flag) {
      atomicExch(error_flag, 1);
    }
  }
  __syncthreads();
  if (tid == 0) {  // exclusive scan (E <= 512, serial is cheap and exact)
    int run = 0;
    for (int e = 0; e < E; ++e) {
      starts[e] = run;
      counts[e] = hist[e];
      cursor[e] = run;
      run += hist[e];
    }
  }
  __syncthreads();
  for (int64_t base = 0; base < assignments; base += RC_THREADS) {
    const int64_t a = base + tid;
    const bool valid = a < assignments;
    int e = valid ? (int)top_idx[a] : -1;
    if (e < 0 || e >= E) e = -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    const int warp_count = __popc(peers);
    // per-warp counts for this chunk, processed in quarters of the expert range
    int offset = 0;
    for (int q0 = 0; q0 < E; q0 += RC_MAXE / 4) {
      for (int i = lane; i < RC_MAXE / 4; i += 32) whist[warp][i] = 0;
      __syncthreads();
      const bool mine = e >= q0 && e < q0 + RC_MAXE / 4;
      if (mine && rank_in_warp == 0) whist[warp][e - q0] = warp_count;
      __syncthreads();
      if (mine) {
        int before = 0;
        for (int w = 0; w < warp; ++w) before += whist[w][e - q0];
        offset = before;
      }
      __syncthreads();
      // advance cursors by this chunk's totals (thread per expert of the quarter)
      if (tid < RC_MAXE / 4 && q0 + tid < E) {
        int tot = 0;
        for (int w = 0; w < RC_WARPS; ++w) tot += whist[w][tid];
        hist[q0 + tid] = tot;  // chunk total, applied below
      }
      __syncthreads();
    }
    if (e >= 0) {
      const int pos = cursor[e] + offset + rank_in_warp;
      token_ids[pos] = a / k;
      coef[pos] = top_w[a];
      inverse[a] = pos;
    }
    __syncthreads();
    for (int i = tid; i < E; i += RC_THREADS) cursor[i] += hist[i];
    __syncthreads();
  }
}

// ------------------------------------------------------------------ grouped expert GEMV

constexpr int GX_WARPS = 8;
constexpr int GX_THREADS = GX_WARPS * 32;
constexpr int GX_ROWS = 16;
constexpr int GX_KB = 64;
constexpr int GX_UNROLL = 4;
constexpr int GX_MAXR = 8;  // activation rows per pass (one n8 mma tile)

struct GroupedArgs {
  const __nv_bfloat16* x;    // activation rows
  const int64_t* row_ids;    // [A]: row of x for assignment a (null: a itself)
  const int32_t* starts;     // [E]
  const int32_t* counts;     // [E]
  int E;
  const int8_t* codes;       // expert slot 0 codes
  int64_t codes_stride;      // bytes between expert slots
  const float* scales;       // expert slot 0 scales
  int64_t scales_stride;     // floats between expert slots
  const int32_t* slot_of;    // [E] expert -> slot (null: identity)
  int64_t n, k;              // per-expert output rows (gate rows for SwiGLU) and in_features
  int64_t up_rows;           // SwiGLU: up rows start at this row offset inside the page
  __nv_bfloat16* y;          // [A, n]
};

// Work item = (expert, 16-row tile). A CTA streams the tile's weights with 8 warps
// splitting k (L1-bypassing 16-byte loads, 4 blocks in flight per warp) and applies them to
// the expert's rows in passes of 8 (activations staged as exact power-of-two-scaled f16).
// Each output row depends only on its own activation row, so results do not depend on how
// many rows an expert received (bit-identical across expert-parallel world sizes).
template <bool SWIGLU>
__global__ void __launch_bounds__(GX_THREADS, 2) grouped_qrow_kernel(GroupedArgs a) {
  constexpr int NSTREAM = SWIGLU ? 2 : 1;
  extern __shared__ __align__(16) unsigned char smem[];
  const int64_t K = a.k;
  const int kpad = (int)((K + GX_KB - 1) / GX_KB) * GX_KB;
  const int xstride = kpad + 8;
  const int nkb = kpad / GX_KB;
  __half* xs = reinterpret_cast<__half*>(smem);
  float* red = reinterpret_cast<float*>(smem + (((size_t)GX_MAXR * xstride * 2 + 15) & ~size_t(15)));
  float* rscale = red + GX_WARPS * NSTREAM * GX_ROWS * 8;  // [8] 2^-e, [8..16) 2^e
  unsigned* rmax = reinterpret_cast<unsigned*>(rscale + 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int64_t rtiles = (a.n + GX_ROWS - 1) / GX_ROWS;
  const int64_t items = (int64_t)a.E * rtiles;
  pdl_launch_dependents();
  pdl_wait();
  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const int e = (int)(item / rtiles);
    const int64_t tile = item - (int64_t)e * rtiles;
    const int cnt = a.counts[e];
    if (cnt == 0) continue;  // uniform across the CTA
    const int st = a.starts[e];
    const int slot = a.slot_of ? a.slot_of[e] : e;
    const int8_t* codes = a.codes + (int64_t)slot * a.codes_stride;
    const float* scales = a.scales + (int64_t)slot * a.scales_stride;
    const int64_t r0 = min(tile * GX_ROWS + g, a.n - 1), r1 = min(tile * GX_ROWS + g + 8, a.n - 1);
    for (int p0 = 0; p0 < cnt; p0 += GX_MAXR) {
      const int rows = min(GX_MAXR, cnt - p0);
      // ---- stage this pass's activation rows
      if (tid < GX_MAXR) rmax[tid] = 0u;
      __syncthreads();
      for (int idx = tid; idx < rows * (int)(K / 8); idx += GX_THREADS) {
        const int r = idx / (int)(K / 8), v = idx - r * (int)(K / 8);
        const int64_t arow = st + p0 + r;
        const int64_t src = a.row_ids ? a.row_ids[arow] : arow;
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(a.x + src * K) + v);
        *reinterpret_cast<uint4*>(xs + r * xstride + v * 8) = raw;
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
        float mx = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(__bfloat162float(h[i])));
        atomicMax(&rmax[r], __float_as_uint(mx));
      }
      __syncthreads();
      if (tid < rows) {
        const float mx = __uint_as_float(rmax[tid]);
        int ex = 0, e2 = 0;
        if (mx > 0.f && isfinite(mx)) {
          frexpf(mx, &ex);
          e2 = max(-100, min(100, 15 - ex));
        }
        rscale[tid] = ldexpf(1.0f, -e2);
        rscale[8 + tid] = ldexpf(1.0f, e2);
      }
      __syncthreads();
      for (int idx = tid; idx < GX_MAXR * (kpad / 8); idx += GX_THREADS) {
        const int r = idx / (kpad / 8), v = idx - r * (kpad / 8);
        uint4* slotp = reinterpret_cast<uint4*>(xs + r * xstride + v * 8);
        __align__(16) __half hv[8];
        if (r < rows && v * 8 < K) {
          const uint4 raw = *slotp;
          const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
          for (int i = 0; i < 8; ++i) hv[i] = __float2half_rn(__bfloat162float(h[i]) * rscale[8 + r]);
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) hv[i] = __float2half_rn(0.f);
        }
        *slotp = *reinterpret_cast<const uint4*>(hv);
      }
      __syncthreads();
      // ---- stream the tile's weights
      float acc[NSTREAM][4];
#pragma unroll
      for (int s = 0; s < NSTREAM; ++s)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[s][i] = 0.f;
      for (int kb0 = warp; kb0 < nkb; kb0 += GX_WARPS * GX_UNROLL) {
        uint4 wa[GX_UNROLL][NSTREAM], wb[GX_UNROLL][NSTREAM];
#pragma unroll
        for (int u = 0; u < GX_UNROLL; ++u) {
          const int kb = kb0 + u * GX_WARPS;
          const int64_t koff = (int64_t)kb * GX_KB + 16 * c;
          const bool ok = kb < nkb && koff < K;
#pragma unroll
          for (int s = 0; s < NSTREAM; ++s) {
            const int64_t roff = s == 0 ? 0 : a.up_rows;
            wa[u][s] = ok ? ld_stream_u4(codes + (roff + r0) * K + koff) : make_uint4(0, 0, 0, 0);
            wb[u][s] = ok ? ld_stream_u4(codes + (roff + r1) * K + koff) : make_uint4(0, 0, 0, 0);
          }
        }
#pragma unroll
        for (int u = 0; u < GX_UNROLL; ++u) {
          const int kb = kb0 + u * GX_WARPS;
          if (kb >= nkb) break;
          uint32_t xb[8];
          if (g < GX_MAXR) {
            const uint4* p = reinterpret_cast<const uint4*>(xs + g * xstride + kb * GX_KB + 16 * c);
            const uint4 v0 = p[0], v1 = p[1];
            xb[0] = v0.x; xb[1] = v0.y; xb[2] = v0.z; xb[3] = v0.w;
            xb[4] = v1.x; xb[5] = v1.y; xb[6] = v1.z; xb[7] = v1.w;
          }
#pragma unroll
          for (int s = 0; s < NSTREAM; ++s) {
            const uint32_t ra[4] = {wa[u][s].x, wa[u][s].y, wa[u][s].z, wa[u][s].w};
            const uint32_t rb[4] = {wb[u][s].x, wb[u][s].y, wb[u][s].z, wb[u][s].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t a_lo, a_hi, b_lo, b_hi;
              i8x4_to_f16x2(ra[j], a_lo, a_hi);
              i8x4_to_f16x2(rb[j], b_lo, b_hi);
              mma_f16(acc[s], a_lo, b_lo, a_hi, b_hi, xb[2 * j], xb[2 * j + 1]);
            }
          }
        }
      }
      // ---- reduce over warps and write this pass's rows
#pragma unroll
      for (int s = 0; s < NSTREAM; ++s) {
        float* base = red + ((warp * NSTREAM + s) * GX_ROWS) * 8;
        base[g * 8 + 2 * c] = acc[s][0];
        base[g * 8 + 2 * c + 1] = acc[s][1];
        base[(g + 8) * 8 + 2 * c] = acc[s][2];
        base[(g + 8) * 8 + 2 * c + 1] = acc[s][3];
      }
      __syncthreads();
      for (int idx = tid; idx < GX_ROWS * rows; idx += GX_THREADS) {
        const int row = idx % GX_ROWS, r = idx / GX_ROWS;
        const int64_t nrow = tile * GX_ROWS + row;
        if (nrow >= a.n) continue;
        float v[NSTREAM];
#pragma unroll
        for (int s = 0; s < NSTREAM; ++s) {
          float tot = 0.f;
#pragma unroll
          for (int w = 0; w < GX_WARPS; ++w) tot += red[((w * NSTREAM + s) * GX_ROWS + row) * 8 + r];
          v[s] = tot * rscale[r] * scales[(s == 0 ? 0 : a.up_rows) + nrow];
        }
        __nv_bfloat16* out = a.y + (int64_t)(st + p0 + r) * a.n + nrow;
        if (SWIGLU) {
          const float gt = round_bf16(v[0]);
          const float up = round_bf16(v[NSTREAM - 1]);
          *out = __float2bfloat16_rn(round_bf16(silu_f32(gt)) * up);
        } else {
          *out = __float2bfloat16_rn(v[0]);
        }
      }
      __syncthreads();
    }
  }
}

// ------------------------------------------------------------------ fixed-rank combine

// out[t, h] = sum over r < k, in rank order, of coef[p] * float(eo[p, h]) with p = inverse[t*k + r];
// each product rounded to fp32, then added left to right (the reference's CPU branch).
__global__ void stable_route_reduce_kernel(const __nv_bfloat16* __restrict__ eo, const float* __restrict__ coef,
                                           const int64_t* __restrict__ inverse, int64_t tokens, int k, int64_t H,
                                           float* __restrict__ out_f32, __nv_bfloat16* __restrict__ out_bf16) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t t = blockIdx.y;
  for (int64_t h = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; h < H; h += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < k; ++r) {
      const int64_t p = inverse[t * k + r];
      const float prod = __fmul_rn(__bfloat162float(eo[p * H + h]), coef[p]);
      acc = r == 0 ? prod : __fadd_rn(acc, prod);
    }
    if (out_f32) out_f32[t * H + h] = acc;
    if (out_bf16) out_bf16[t * H + h] = __float2bfloat16_rn(acc);
  }
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_router_topk(const void* logits, int logits_dtype, int64_t tokens, int64_t experts, int64_t k,
                               int renorm, int64_t* top_idx, float* top_w_f32, void* top_w_bf16, void* stream) {
  if (tokens < 0 || experts <= 0 || k <= 0 || k > experts) return fail(MRB_ERR_ARG, "router_topk: bad shape");
  if (tokens == 0) return MRB_OK;
  if (experts > 256 || k > 16) return fail(MRB_ERR_UNSUPPORTED, "router_topk: experts <= 256 and k <= 16");
  if (!logits || !top_idx) return fail(MRB_ERR_ARG, "router_topk: null pointer");
  const unsigned warps = 8;
  const dim3 grid((unsigned)((tokens + warps - 1) / warps));
  cudaStream_t s = (cudaStream_t)stream;
  switch (logits_dtype) {
    case MRB_F32:
      launch_kernel(router_topk_kernel<float>, grid, dim3(32 * warps), 0, s, true, (const float*)logits, tokens,
                    (int)experts, (int)k, renorm, top_idx, top_w_f32, (__nv_bfloat16*)top_w_bf16);
      break;
    case MRB_BF16:
      launch_kernel(router_topk_kernel<__nv_bfloat16>, grid, dim3(32 * warps), 0, s, true,
                    (const __nv_bfloat16*)logits, tokens, (int)experts, (int)k, renorm, top_idx, top_w_f32,
                    (__nv_bfloat16*)top_w_bf16);
      break;
    default:
      return fail(MRB_ERR_ARG, "router_topk: bad logits dtype %d", logits_dtype);
  }
  return launch_status("router_topk");
}

extern "C" int mrb_route_compile(const int64_t* top_idx, const float* top_w, int64_t tokens, int64_t k,
                                 int64_t experts, int32_t* counts, int32_t* starts, int64_t* token_ids, float* coef,
                                 int64_t* inverse, int32_t* error_flag, void* stream) {
  if (tokens < 0 || k <= 0 || experts <= 0) return fail(MRB_ERR_ARG, "route_compile: bad shape");
  if (experts > RC_MAXE) return fail(MRB_ERR_UNSUPPORTED, "route_compile: at most %d experts", RC_MAXE);
  if (!counts || !starts) return fail(MRB_ERR_ARG, "route_compile: null pointer");
  if (tokens > 0 && (!top_idx || !top_w || !token_ids || !coef || !inverse))
    return fail(MRB_ERR_ARG, "route_compile: null pointer");
  if (tokens * k > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "route_compile: too many assignments");
  launch_kernel(route_compile_kernel, dim3(1), dim3(RC_THREADS), 0, (cudaStream_t)stream, true, top_idx, top_w,
                tokens * k, (int)k, (int)experts, counts, starts, token_ids, coef, inverse, error_flag);
  return launch_status("route_compile");
}

extern "C" int mrb_grouped_qrow(const void* x_bf16, const int64_t* row_ids, const int32_t* starts,
                                const int32_t* counts, int64_t experts, const int8_t* codes, int64_t codes_stride,
                                const float* scales, int64_t scales_stride, const int32_t* slot_of, int64_t n,
                                int64_t k, int64_t up_rows, int swiglu, void* y_bf16, void* stream) {
  if (experts <= 0 || n <= 0 || k <= 0) return fail(MRB_ERR_ARG, "grouped_qrow: bad shape");
  if (!x_bf16 || !starts || !counts || !codes || !scales || !y_bf16) return fail(MRB_ERR_ARG, "grouped_qrow: null pointer");
  if (k % 16) return fail(MRB_ERR_UNSUPPORTED, "grouped_qrow: in_features %lld is not a multiple of 16", (long long)k);
  if (!aligned(codes, 16) || (codes_stride % 16) || !aligned(x_bf16, 16))
    return fail(MRB_ERR_ARG, "grouped_qrow: codes and activation rows must be 16-byte aligned");
  if (swiglu && up_rows < n) return fail(MRB_ERR_ARG, "grouped_qrow: up rows overlap the gate rows");
  const int kpad = (int)((k + GX_KB - 1) / GX_KB) * GX_KB;
  const size_t xs = (((size_t)GX_MAXR * (kpad + 8) * 2) + 15) & ~size_t(15);
  const size_t smem = xs + (size_t)GX_WARPS * (swiglu ? 2 : 1) * GX_ROWS * 8 * 4 + 32 * 4;
  if (smem > 200 * 1024) return fail(MRB_ERR_UNSUPPORTED, "grouped_qrow: in_features %lld too large", (long long)k);
  GroupedArgs a{(const __nv_bfloat16*)x_bf16, row_ids, starts, counts, (int)experts, codes, codes_stride, scales,
                scales_stride, slot_of, n, k, up_rows, (__nv_bfloat16*)y_bf16};
  const int64_t items = experts * ((n + GX_ROWS - 1) / GX_ROWS);
  const int64_t grid = std::min<int64_t>(items, (int64_t)num_sms() * 2);
  cudaStream_t s = (cudaStream_t)stream;
  auto run = [&](auto kern) -> int {
    static size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "grouped_qrow: smem attribute: %s", cudaGetErrorString(e));
      configured = smem;
    }
    launch_kernel(kern, dim3((unsigned)grid), dim3(GX_THREADS), smem, s, true, a);
    return launch_status("grouped_qrow");
  };
  return swiglu ? run(grouped_qrow_kernel<true>) : run(grouped_qrow_kernel<false>);
}

extern "C" int mrb_stable_route_reduce(const void* expert_out_bf16, const float* coef, const int64_t* inverse,
                                       int64_t tokens, int64_t k, int64_t hidden, float* out_f32, void* out_bf16,
                                       void* stream) {
  if (tokens < 0 || k <= 0 || hidden <= 0) return fail(MRB_ERR_ARG, "stable_route_reduce: bad shape");
  if (tokens == 0) return MRB_OK;
  if (!expert_out_bf16 || !coef || !inverse || (!out_f32 && !out_bf16))
    return fail(MRB_ERR_ARG, "stable_route_reduce: null pointer");
  if (tokens > 65535) return fail(MRB_ERR_UNSUPPORTED, "stable_route_reduce: at most 65535 tokens per call");
  const unsigned bx = (unsigned)std::min<int64_t>((hidden + 255) / 256, 64);
  launch_kernel(stable_route_reduce_kernel, dim3(bx, (unsigned)tokens), dim3(256), 0, (cudaStream_t)stream, true,
                (const __nv_bfloat16*)expert_out_bf16, coef, inverse, tokens, (int)k, hidden, out_f32,
                (__nv_bfloat16*)out_bf16);
  return launch_status("stable_route_reduce");
}
