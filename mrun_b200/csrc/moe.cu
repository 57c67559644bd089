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
#include "moe_route.cuh"

#include <algorithm>

namespace mrb {

// ------------------------------------------------------------------ router

constexpr int ROUTER_MAXE = 256;

// The selection shared by the router kernels, for one token held by one warp: lane l holds
// the logits of experts l, l + 32, ... in p[]. Softmax in fp32 (max-subtracted exp, divided by
// the sum), then k rounds of arg-max (ties -> lower expert), optional renormalisation by the
// fp32 sum of the chosen probabilities, and the bf16 weights the reference hands on.
// Outputs (each optional but top_idx): fp32 weights before the bf16 rounding, the bf16
// weights, and the bf16 weights as fp32 (the coefficients the route compiler takes).
//
// Latency is the cost here (one warp, a few thousand cycles), so: slots past the last expert
// are skipped by uniform branches; each lane sorts its own probabilities once (by key, then
// expert), so its best is always at the head; and each arg-max round is two warp reductions
// (redux.sync) over an order-preserving key -- the probability's bits + 1 (probabilities are
// >= 0, so their bits order like the values; 0 marks an absent or taken expert) -- and then
// the lowest expert among the lanes holding that key. The winning lane shifts its list.
__device__ __forceinline__ uint32_t router_key(float prob) { return __float_as_uint(prob) + 1u; }

// (key, expert) ordering: larger key first, then the lower expert
__device__ __forceinline__ void router_cx(uint32_t& ka, uint32_t& ia, uint32_t& kb, uint32_t& ib) {
  const bool swap = kb > ka || (kb == ka && ib < ia);
  const uint32_t k0 = swap ? kb : ka, i0 = swap ? ib : ia;
  kb = swap ? ka : kb;
  ib = swap ? ia : ib;
  ka = k0;
  ia = i0;
}

template <int NS>
__device__ __forceinline__ void router_pick(const float (&p)[ROUTER_MAXE / 32], int E, int k, int renorm, int64_t t,
                                            int64_t* __restrict__ top_idx, float* __restrict__ top_w_f32,
                                            __nv_bfloat16* __restrict__ top_w_bf16, float* __restrict__ top_w_coef) {
  const int lane = threadIdx.x & 31;
  uint32_t key[NS], idx[NS];
#pragma unroll
  for (int i = 0; i < NS; ++i) {
    const int e = lane + 32 * i;
    key[i] = e < E ? router_key(p[i]) : 0u;
    idx[i] = e < E ? (uint32_t)e : 0xffffffffu;
  }
  // odd-even transposition sort of the lane's NS slots
#pragma unroll
  for (int r = 0; r < NS; ++r)
#pragma unroll
    for (int i = r & 1; i + 1 < NS; i += 2) router_cx(key[i], idx[i], key[i + 1], idx[i + 1]);
  float chosen_sum = 0.f, my_w = 0.f;
  uint32_t my_i = 0;
  for (int j = 0; j < k; ++j) {
    const uint32_t m = __reduce_max_sync(0xffffffffu, key[0]);
    const uint32_t bi = __reduce_min_sync(0xffffffffu, key[0] == m ? idx[0] : 0xffffffffu);
    const float best = __uint_as_float(m - 1u);
    if (lane == j) {
      my_w = best;
      my_i = bi;
    }
    chosen_sum += best;
    if (idx[0] == bi) {
#pragma unroll
      for (int i = 0; i + 1 < NS; ++i) {
        key[i] = key[i + 1];
        idx[i] = idx[i + 1];
      }
      key[NS - 1] = 0u;
      idx[NS - 1] = 0xffffffffu;
    }
  }
  if (lane < k) {
    const float w = renorm ? my_w / chosen_sum : my_w;
    top_idx[t * k + lane] = (int64_t)my_i;
    if (top_w_f32) top_w_f32[t * k + lane] = w;
    const __nv_bfloat16 wb = __float2bfloat16_rn(w);
    if (top_w_bf16) top_w_bf16[t * k + lane] = wb;
    if (top_w_coef) top_w_coef[t * k + lane] = __bfloat162float(wb);
  }
}

__device__ __forceinline__ void router_select(float (&p)[ROUTER_MAXE / 32], int E, int k, int renorm, int64_t t,
                                              int64_t* __restrict__ top_idx, float* __restrict__ top_w_f32,
                                              __nv_bfloat16* __restrict__ top_w_bf16, float* __restrict__ top_w_coef) {
  const int lane = threadIdx.x & 31;
  const int slots = (E + 31) >> 5;  // slots that hold an expert in some lane (uniform)
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < ROUTER_MAXE / 32; ++i)
    if (i < slots) mx = fmaxf(mx, p[i]);
  // order-preserving u32 image of a float: flip all bits of negatives, the sign bit of the rest
  const uint32_t mb = __float_as_uint(mx);
  const uint32_t mflip = __reduce_max_sync(0xffffffffu, (mb & 0x80000000u) ? ~mb : (mb | 0x80000000u));
  mx = __uint_as_float((mflip & 0x80000000u) ? (mflip & 0x7fffffffu) : ~mflip);
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < ROUTER_MAXE / 32; ++i)
    if (i < slots) {
      p[i] = (lane + 32 * i) < E ? expf(p[i] - mx) : 0.f;
      sum += p[i];
    }
  sum = warp_sum(sum);
#pragma unroll
  for (int i = 0; i < ROUTER_MAXE / 32; ++i)
    if (i < slots) p[i] = (lane + 32 * i) < E ? p[i] / sum : 0.f;
  if (slots <= 1)
    router_pick<1>(p, E, k, renorm, t, top_idx, top_w_f32, top_w_bf16, top_w_coef);
  else if (slots <= 2)
    router_pick<2>(p, E, k, renorm, t, top_idx, top_w_f32, top_w_bf16, top_w_coef);
  else if (slots <= 4)
    router_pick<4>(p, E, k, renorm, t, top_idx, top_w_f32, top_w_bf16, top_w_coef);
  else
    router_pick<8>(p, E, k, renorm, t, top_idx, top_w_f32, top_w_bf16, top_w_coef);
}

// One warp per token over logits already computed.
template <typename LT>
__global__ void router_topk_kernel(const LT* __restrict__ logits, int64_t tokens, int E, int k, int renorm,
                                   int64_t* __restrict__ top_idx, float* __restrict__ top_w_f32,
                                   __nv_bfloat16* __restrict__ top_w_bf16, float* __restrict__ top_w_coef) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= tokens) return;
  float p[ROUTER_MAXE / 32];
  const LT* row = logits + t * E;
#pragma unroll
  for (int i = 0; i < ROUTER_MAXE / 32; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < E ? io<LT>::load(row + e) : -INFINITY;
  }
  router_select(p, E, k, renorm, t, top_idx, top_w_f32, top_w_bf16, top_w_coef);
}

// The router's logits, expert-major: CTA b computes the logits of experts b, b + grid, ...
// for every token (exact int8 x bf16 products, fp32 sums in a fixed order, times the row
// scale, rounded to bf16 -- the W8A16 projection's boundary). Each warp converts the expert's
// codes to fp32 once and reuses them for its tokens, so the conversions do not scale with the
// token count and the E x K router matrix is read from memory about once. The selection runs
// next as router_topk_kernel (one warp per token), launched to wait on this grid.
//
// Conversion: 2^23 + u for the biased byte u = q + 128 is a float whose low mantissa byte is
// u (built with one byte permute), and subtracting 2^23 + 128 gives q exactly.
constexpr int RQ_WARPS = 16;
constexpr int RQ_CHUNK = 8;  // 8-element vectors per lane and pass over k
constexpr int RQ_TPW = 2;    // tokens per warp and token group (RQ_WARPS * RQ_TPW per group)

__device__ __forceinline__ void rq_codes_to_f32(uint2 w, float (&f)[8]) {
  const uint32_t lo = w.x ^ 0x80808080u, hi = w.y ^ 0x80808080u;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    f[u] = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440u + u)) - 8388736.0f;
    f[4 + u] = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440u + u)) - 8388736.0f;
  }
}

__global__ void __launch_bounds__(RQ_WARPS * 32) router_qrow_logits_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t T, int64_t K, const int8_t* __restrict__ codes,
    const float* __restrict__ scales, int E, __nv_bfloat16* __restrict__ logits) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = (int)(K / 8);
  for (int e = blockIdx.x; e < E; e += gridDim.x) {
    const uint2* wr = reinterpret_cast<const uint2*>(codes + (int64_t)e * K);
    const float sc = scales[e];
    for (int64_t t0 = 0; t0 < T; t0 += RQ_WARPS * RQ_TPW) {
      float acc[RQ_TPW] = {};
      for (int v0 = 0; v0 < nv; v0 += 32 * RQ_CHUNK) {
        float cf[RQ_CHUNK][8];
#pragma unroll
        for (int i = 0; i < RQ_CHUNK; ++i) {
          const int v = v0 + lane + 32 * i;
          rq_codes_to_f32(v < nv ? __ldg(wr + v) : make_uint2(0x80808080u, 0x80808080u) /* zeros */, cf[i]);
        }
#pragma unroll
        for (int j = 0; j < RQ_TPW; ++j) {
          const int64_t t = t0 + warp + RQ_WARPS * j;
          if (t >= T) break;
          const uint4* xr = reinterpret_cast<const uint4*>(x + t * K);
          uint4 xv[RQ_CHUNK];
#pragma unroll
          for (int i = 0; i < RQ_CHUNK; ++i) {
            const int v = v0 + lane + 32 * i;
            xv[i] = v < nv ? __ldg(xr + v) : make_uint4(0u, 0u, 0u, 0u);
          }
          float a = acc[j];
#pragma unroll
          for (int i = 0; i < RQ_CHUNK; ++i) {
            const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&xv[i]);
#pragma unroll
            for (int u = 0; u < 8; ++u) a = fmaf(cf[i][u], __bfloat162float(h[u]), a);  // exact product
          }
          acc[j] = a;
        }
      }
#pragma unroll
      for (int j = 0; j < RQ_TPW; ++j) {
        const int64_t t = t0 + warp + RQ_WARPS * j;
        const float sum = warp_sum(acc[j]);
        if (lane == 0 && t < T) logits[t * E + e] = __float2bfloat16_rn(round_bf16(sum * sc));
      }
    }
  }
}

// ------------------------------------------------------------------ route compiler

// Single CTA of 1024 threads. Assignments are ranked in chunks of 1024 in flat (token,
// rank) order: inside a warp, peers with the same expert are found with match_any, warps
// are ordered through a per-warp histogram, and a running per-expert cursor carries the
// order across chunks -- exactly the stable expert-major order of the reference's CPU
// branch (argsort(experts, stable=True)), with no atomics deciding positions.
__global__ void __launch_bounds__(RC_THREADS) route_compile_kernel(
    const int64_t* __restrict__ top_idx, const float* __restrict__ top_w, int64_t assignments, int k, int E,
    int32_t* __restrict__ counts, int32_t* __restrict__ starts, int64_t* __restrict__ token_ids,
    float* __restrict__ coef, int64_t* __restrict__ inverse, int32_t* __restrict__ error_flag) {
  pdl_launch_dependents();
  pdl_wait();
  route_compile_block(top_idx, top_w, assignments, k, E, counts, starts, token_ids, coef, inverse, error_flag);
}

// ------------------------------------------------------------------ grouped expert GEMV

// acquire load of a counter another CTA publishes (GPU scope)
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

constexpr int GX_WARPS = 8;
constexpr int GX_THREADS = GX_WARPS * 32;
constexpr int GX_ROWS = 16;       // weight rows per warp tile (mma M)
constexpr int GX_KB = 64;         // k elements per step and stream
constexpr int GX_MAXR = 16;       // activation rows per pass (up to two n8 mma tiles)
constexpr int GX_STAGES = 4;      // cp.async ring depth per thread
constexpr int GX_STAGE_BYTES = 2 * 2 * GX_THREADS * 16;  // 2 streams x rows (g, g+8) x 16 B per thread

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
  int chunks;                // tile chunks per expert (work items per expert)
  int chunk_tiles;           // 16-row tiles per chunk
  int maxr;                  // activation rows per pass (<= GX_MAXR; fewer when k is large)
  // Gate/up -> down overlap (mrb_grouped_expert_mlp): 0 = a lone launch; 1 = the gate/up
  // launch, which counts finished items per expert in ready[]; 2 = the down launch, which
  // starts on an expert once ready[e] == ready_target, counts its own items in done[] and,
  // on an expert's last item, leaves both counters at zero.
  int overlap;
  int ready_target;
  unsigned* ready;
  unsigned* done;
  int32_t* error_flag;       // overlap 2: set when a wait gave up
  int64_t wait_polls;        // overlap 2: bound of one expert's wait
};

__host__ __device__ inline int gx_steps(int64_t k, bool halves) {
  const int nkb = (int)((k + GX_KB - 1) / GX_KB);
  return halves ? (nkb + 1) / 2 : nkb;
}
__host__ __device__ inline int gx_xlen(int64_t k, bool halves) { return gx_steps(k, halves) * GX_KB * (halves ? 2 : 1); }
__host__ __device__ inline size_t gx_xs_bytes(int64_t k, bool halves, int maxr) {
  return ((size_t)maxr * (gx_xlen(k, halves) + 8) * 2 + 15) & ~size_t(15);
}
__host__ inline size_t gx_smem_bytes(int64_t k, bool halves, int maxr) {
  return (size_t)GX_STAGES * GX_STAGE_BYTES + gx_xs_bytes(k, halves, maxr) + 64 * 4;  // + rscale[32] (and spare)
}

// Grouped int8 expert projection over ragged per-expert row counts.
//
// Work item = (expert, chunk of 16-row tiles); a CTA walks items blockIdx.x, +gridDim.x, ...
// (experts without rows are skipped). Per item and pass of up to maxr rows (16 -- two n8 mma
// tiles sharing every weight fragment, one tile when the pass has 8 rows or fewer -- or fewer
// rows when they do not fit in shared memory) it stages the
// expert's activation rows once (gathered through row_ids, exact power-of-two-scaled f16),
// then each warp owns whole tiles of the chunk: it streams the tile's weights over the full
// k through a per-thread cp.async ring (rows g and g+8, two streams per step: the gate and
// up rows for SwiGLU, the two k halves otherwise), accumulates on mma.sync in fp32 and
// writes its outputs directly -- no cross-warp reduction, no barrier inside an item. The
// ring prefetches across tiles, passes and items. Codes convert to exact f16, so each output
// row depends only on its own activation row (bit-identical for any row grouping, hence
// across expert-parallel world sizes).
template <bool SWIGLU, int NT>  // NT: n8 mma tiles per pass (16-row passes when 2)
__global__ void __launch_bounds__(GX_THREADS, 2) grouped_qrow_kernel(GroupedArgs a) {
  constexpr bool HALVES = !SWIGLU;
  extern __shared__ __align__(16) unsigned char smem[];
  const int64_t K = a.k;
  const int nks = gx_steps(K, HALVES);    // k steps per tile
  const int xlen = gx_xlen(K, HALVES);
  const int xstride = xlen + 8;
  const int kspan = HALVES ? nks * GX_KB : 0;
  unsigned char* ring = smem;
  __half* xs = reinterpret_cast<__half*>(smem + (size_t)GX_STAGES * GX_STAGE_BYTES);
  float* rscale = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(xs) + gx_xs_bytes(K, HALVES, a.maxr));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int rtiles = (int)((a.n + GX_ROWS - 1) / GX_ROWS);
  const int items = a.E * a.chunks;
  const bool k_check = (int64_t)xlen != K;

  if (a.overlap == 1) {
    // the down launch may start once every CTA here has passed the wait: by then the routes
    // exist, and it reads gate/up outputs only behind ready[]
    pdl_wait();
    pdl_launch_dependents();
  } else if (a.overlap == 2) {
    pdl_launch_dependents();  // no grid-wide wait: experts start as their gate/up items finish
  } else {
    pdl_launch_dependents();
    pdl_wait();  // routes and activations come from the previous kernels
  }

  auto item_expert = [&](int item) { return item / a.chunks; };
  auto item_t0 = [&](int item) { return (item - item_expert(item) * a.chunks) * a.chunk_tiles; };
  auto item_t1 = [&](int item) { return min(rtiles, item_t0(item) + a.chunk_tiles); };
  const int maxr = a.maxr;
  auto item_passes = [&](int item) { return (a.counts[item_expert(item)] + maxr - 1) / maxr; };

  // ---- per-thread prefetch cursor over (item, pass, this warp's tile, k step)
  int pf_item = blockIdx.x, pf_pass = 0, pf_tile = 0, pf_step = 0, pf_koff = 0, slot_w = 0;
  const int8_t* pf_row0 = nullptr;
  const int8_t* pf_row1 = nullptr;
  int64_t pf_delta = 0;
  auto pf_load_tile = [&]() {  // pointers of (pf_item, pf_tile) at step 0
    const int e = item_expert(pf_item);
    const int slot = a.slot_of ? a.slot_of[e] : e;
    const int8_t* codes = a.codes + (int64_t)slot * a.codes_stride;
    const int64_t r0 = min((int64_t)pf_tile * GX_ROWS + g, a.n - 1);
    const int64_t r1 = min((int64_t)pf_tile * GX_ROWS + g + 8, a.n - 1);
    pf_koff = 16 * c;
    pf_row0 = codes + r0 * K + pf_koff;
    pf_row1 = codes + r1 * K + pf_koff;
    pf_delta = SWIGLU ? a.up_rows * K : (int64_t)kspan;
    pf_step = 0;
  };
  // settle on the next (item, pass, tile) that holds work for this warp, from pf_item/pf_pass/pf_tile
  auto pf_settle = [&](bool fresh_item) {
    for (; pf_item < items; pf_item += gridDim.x, fresh_item = true) {
      if (fresh_item) {
        if (a.counts[item_expert(pf_item)] == 0) continue;
        pf_pass = 0;
        pf_tile = item_t0(pf_item) + warp;
      }
      const int t1 = item_t1(pf_item), passes = item_passes(pf_item);
      while (pf_pass < passes) {
        if (pf_tile < t1 && nks > 0) {
          pf_load_tile();
          return;
        }
        ++pf_pass;
        pf_tile = item_t0(pf_item) + warp;
      }
    }
  };
  pf_settle(true);
  auto issue = [&]() {
    if (pf_item < items) {
      unsigned char* st = ring + slot_w * GX_STAGE_BYTES + tid * 16;
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int64_t d = s == 0 ? 0 : pf_delta;
        const bool ok = !k_check || pf_koff + (HALVES ? s * kspan : 0) < K;
        cp_async16_zfill(st + (s * 2 + 0) * GX_THREADS * 16, ok ? pf_row0 + d : a.codes, ok);
        cp_async16_zfill(st + (s * 2 + 1) * GX_THREADS * 16, ok ? pf_row1 + d : a.codes, ok);
      }
      pf_row0 += GX_KB;
      pf_row1 += GX_KB;
      pf_koff += GX_KB;
      if (++pf_step == nks) {
        pf_tile += GX_WARPS;
        pf_settle(false);
      }
    }
    cp_async_commit_group();
    slot_w = slot_w + 1 == GX_STAGES ? 0 : slot_w + 1;
  };
#pragma unroll
  for (int p = 0; p < GX_STAGES - 1; ++p) issue();

  int slot_r = 0;
  for (int item = blockIdx.x; item < items; item += gridDim.x) {
    const int e = item_expert(item);
    const int cnt = a.counts[e];
    if (cnt == 0) continue;  // uniform across the CTA
    const int st0 = a.starts[e];
    const int slot = a.slot_of ? a.slot_of[e] : e;
    const float* scales = a.scales + (int64_t)slot * a.scales_stride;
    const int t0 = item_t0(item), t1 = item_t1(item);
    if (a.overlap == 2 && tid == 0) {  // the expert's activation rows are complete
      int64_t polls = 0;
      while (ld_acquire_u32(a.ready + e) < (unsigned)a.ready_target) {
        if (++polls > a.wait_polls) {
          if (a.error_flag) atomicExch(a.error_flag, 1);
          break;
        }
        __nanosleep(64);
      }
    }
    for (int p0 = 0; p0 < cnt; p0 += maxr) {
      const int rows = min(maxr, cnt - p0);
      // ---- stage this pass's activation rows as exact power-of-two-scaled f16: one warp per
      // row -- raw copy into shared memory and the row max by warp shuffles, the scale, then
      // the conversion in place (each lane converts the vectors it copied); rows past `rows`
      // and k past K are zero
      const bool two = NT == 2 && rows > 8;
      const int prow = two ? maxr : min(8, maxr);
      __syncthreads();  // every warp is done with the previous pass's rows
      {
        const int vpr = (int)(K / 8), vlen = xlen / 8;
        for (int r = warp; r < prow; r += GX_WARPS) {
          uint4* row = reinterpret_cast<uint4*>(xs + r * xstride);
          if (r >= rows) {
            for (int v = lane; v < vlen; v += 32) row[v] = make_uint4(0u, 0u, 0u, 0u);
            continue;
          }
          const int64_t arow = st0 + p0 + r;
          const int64_t src = a.row_ids ? a.row_ids[arow] : arow;
          const uint4* xrow = reinterpret_cast<const uint4*>(a.x + src * K);
          float mx = 0.f;
          for (int v = lane; v < vpr; v += 32) {
            // rows written by the overlapping gate/up launch are read through L2 only
            const uint4 raw = a.overlap == 2 ? __ldcg(xrow + v) : __ldg(xrow + v);
            row[v] = raw;
            const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
            for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(__bfloat162float(h[i])));
          }
          mx = warp_max(mx);
          int ex = 0, e2 = 0;
          if (mx > 0.f && isfinite(mx)) {
            frexpf(mx, &ex);
            e2 = max(-100, min(100, 15 - ex));  // max * 2^e2 in [2^14, 2^15): exact in f16
          }
          const float up = ldexpf(1.0f, e2);
          if (lane == 0) {
            rscale[r] = ldexpf(1.0f, -e2);
            rscale[16 + r] = up;
          }
          for (int v = lane; v < vlen; v += 32) {
            __align__(16) __half hv[8];
            if (v < vpr) {
              const uint4 raw = row[v];
              const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
              for (int i = 0; i < 8; ++i) hv[i] = __float2half_rn(__bfloat162float(h[i]) * up);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) hv[i] = __float2half_rn(0.f);
            }
            row[v] = *reinterpret_cast<const uint4*>(hv);
          }
        }
      }
      __syncthreads();
      // ---- this warp's tiles of the chunk
      for (int tile = t0 + warp; tile < t1; tile += GX_WARPS) {
        float acc[2][NT][4];  // [stream][n8 tile][fragment]
#pragma unroll
        for (int s = 0; s < 2; ++s)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[s][nt][i] = 0.f;
        // activation rows g and g + 8 of the pass (mma column g of tiles 0 and 1); columns at
        // or past the staged width read the last staged row and are dropped in the epilogue
        const __half* xp = xs + min(g, prow - 1) * xstride + 16 * c;
        const int64_t x1off = (int64_t)(min(g + 8, prow - 1) - min(g, prow - 1)) * xstride;
        for (int ks = 0; ks < nks; ++ks, xp += GX_KB) {
          cp_async_wait_group<GX_STAGES - 2>();
          const unsigned char* st = ring + slot_r * GX_STAGE_BYTES + tid * 16;
          slot_r = slot_r + 1 == GX_STAGES ? 0 : slot_r + 1;
          uint4 wa[2], wb[2];
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            wa[s] = *reinterpret_cast<const uint4*>(st + (s * 2 + 0) * GX_THREADS * 16);
            wb[s] = *reinterpret_cast<const uint4*>(st + (s * 2 + 1) * GX_THREADS * 16);
          }
          issue();
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const uint4* p = reinterpret_cast<const uint4*>(xp + (HALVES ? s * kspan : 0));
            const uint4 v0 = p[0], v1 = p[1];
            const uint32_t xb[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
            uint32_t xc[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
            if (NT == 2 && two) {
              const uint4* p1 = reinterpret_cast<const uint4*>(xp + x1off + (HALVES ? s * kspan : 0));
              const uint4 u0 = p1[0], u1 = p1[1];
              xc[0] = u0.x; xc[1] = u0.y; xc[2] = u0.z; xc[3] = u0.w;
              xc[4] = u1.x; xc[5] = u1.y; xc[6] = u1.z; xc[7] = u1.w;
            }
            const uint32_t ra[4] = {wa[s].x, wa[s].y, wa[s].z, wa[s].w};
            const uint32_t rb[4] = {wb[s].x, wb[s].y, wb[s].z, wb[s].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t a_lo, a_hi, b_lo, b_hi;
              i8x4_to_f16x2(ra[j], a_lo, a_hi);
              i8x4_to_f16x2(rb[j], b_lo, b_hi);
              mma_f16(acc[s][0], a_lo, b_lo, a_hi, b_hi, xb[2 * j], xb[2 * j + 1]);
              if (NT == 2 && two) mma_f16(acc[s][NT - 1], a_lo, b_lo, a_hi, b_hi, xc[2 * j], xc[2 * j + 1]);
            }
          }
        }
        // ---- epilogue: lane holds weight rows (g, g+8) x activation rows (nt*8 + 2c, +1)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if (nt == 1 && !two) break;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = nt * 8 + 2 * c + (i & 1);
            const int64_t nrow = (int64_t)tile * GX_ROWS + g + (i >> 1) * 8;
            if (r >= rows || nrow >= a.n) continue;
            __nv_bfloat16* out = a.y + (int64_t)(st0 + p0 + r) * a.n + nrow;
            if (SWIGLU) {
              const float gt = round_bf16(acc[0][nt][i] * rscale[r] * scales[nrow]);
              const float up = round_bf16(acc[1][nt][i] * rscale[r] * scales[a.up_rows + nrow]);
              *out = __float2bfloat16_rn(round_bf16(silu_f32(gt)) * up);
            } else {
              *out = __float2bfloat16_rn((acc[0][nt][i] + acc[1][nt][i]) * rscale[r] * scales[nrow]);
            }
          }
        }
      }
    }
    if (a.overlap) {  // the item's outputs are stored: publish (gate/up) or retire (down) it
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        if (a.overlap == 1) {
          atomicAdd(a.ready + e, 1u);
        } else if (atomicAdd(a.done + e, 1u) + 1u == (unsigned)a.chunks) {
          a.ready[e] = 0u;  // every down item of this expert has finished: reset for the next call
          a.done[e] = 0u;
        }
      }
    }
  }
  cp_async_wait_group<0>();
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


// ------------------------------------------------------------------ expert-parallel dispatch

// Fixed-capacity dispatch plan for expert parallelism (expert e on rank e / experts_per_rank).
// Every (source, destination) block has `capacity` slots (>= tokens * k, so nothing can
// overflow); assignment a goes to slot dst * capacity + pos, pos = its rank among the
// assignments to dst in route order (stable). Unused slots carry the dummy local expert id
// experts_per_rank, coefficient 0 and source -1. One CTA: the plan is tiny.
__global__ void __launch_bounds__(1024) ep_pack_kernel(const int64_t* __restrict__ top_idx,
                                                       const float* __restrict__ top_w, int assignments,
                                                       int experts_per_rank, int world, int capacity, int k,
                                                       int32_t* __restrict__ send_expert, float* __restrict__ coef_slot,
                                                       int64_t* __restrict__ slot_of_assign,
                                                       int32_t* __restrict__ slot_src, int32_t* __restrict__ error_flag) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ int32_t ep_dst[];
  const int slots = world * capacity;
  for (int i = threadIdx.x; i < slots; i += blockDim.x) {
    send_expert[i] = experts_per_rank;
    coef_slot[i] = 0.f;
    slot_src[i] = -1;
  }
  for (int a = threadIdx.x; a < assignments; a += blockDim.x) {
    const int64_t e = top_idx[a];
    int d = (int)(e / experts_per_rank);
    if (e < 0 || d >= world) {
      if (error_flag) atomicExch(error_flag, 1);
      d = -1;
    }
    ep_dst[a] = d;
  }
  __syncthreads();
  for (int a = threadIdx.x; a < assignments; a += blockDim.x) {
    const int d = ep_dst[a];
    if (d < 0) {
      slot_of_assign[a] = 0;
      continue;
    }
    int pos = 0;
    for (int b = 0; b < a; ++b) pos += ep_dst[b] == d;
    const int slot = d * capacity + pos;
    slot_of_assign[a] = slot;
    send_expert[slot] = (int)(top_idx[a] - (int64_t)d * experts_per_rank);
    coef_slot[slot] = top_w[a];
    slot_src[slot] = a / k;
  }
}

// send_rows[s, :] = source[slot_src[s], :] for used slots (one CTA per slot).
__global__ void ep_gather_rows_kernel(const __nv_bfloat16* __restrict__ source, int64_t hidden,
                                      const int32_t* __restrict__ slot_src, __nv_bfloat16* __restrict__ send_rows) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t s = blockIdx.x;
  const int src = slot_src[s];
  if (src < 0) return;
  const uint4* in = reinterpret_cast<const uint4*>(source + (int64_t)src * hidden);
  uint4* out = reinterpret_cast<uint4*>(send_rows + s * hidden);
  for (int64_t i = threadIdx.x; i < hidden / 8; i += blockDim.x) out[i] = __ldg(in + i);
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_router_topk(const void* logits, int logits_dtype, int64_t tokens, int64_t experts, int64_t k,
                               int renorm, int64_t* top_idx, float* top_w_f32, void* top_w_bf16, void* stream) {
  if (tokens < 0 || experts <= 0 || k <= 0 || k > experts) return fail(MRB_ERR_ARG, "router_topk: bad shape");
  if (tokens == 0) return MRB_OK;
  if (experts > ROUTER_MAXE || k > 16) return fail(MRB_ERR_UNSUPPORTED, "router_topk: experts <= 256 and k <= 16");
  if (!logits || !top_idx) return fail(MRB_ERR_ARG, "router_topk: null pointer");
  const unsigned warps = 8;
  const dim3 grid((unsigned)((tokens + warps - 1) / warps));
  cudaStream_t s = (cudaStream_t)stream;
  switch (logits_dtype) {
    case MRB_F32:
      launch_kernel(router_topk_kernel<float>, grid, dim3(32 * warps), 0, s, true, (const float*)logits, tokens,
                    (int)experts, (int)k, renorm, top_idx, top_w_f32, (__nv_bfloat16*)top_w_bf16, nullptr);
      break;
    case MRB_BF16:
      launch_kernel(router_topk_kernel<__nv_bfloat16>, grid, dim3(32 * warps), 0, s, true,
                    (const __nv_bfloat16*)logits, tokens, (int)experts, (int)k, renorm, top_idx, top_w_f32,
                    (__nv_bfloat16*)top_w_bf16, nullptr);
      break;
    default:
      return fail(MRB_ERR_ARG, "router_topk: bad logits dtype %d", logits_dtype);
  }
  return launch_status("router_topk");
}

extern "C" int mrb_router_qrow_topk(const void* x_bf16, int64_t tokens, int64_t hidden, const int8_t* codes,
                                    const float* scales, int64_t experts, int64_t k, int renorm, void* logits_bf16,
                                    int64_t* top_idx, float* top_w_f32, void* top_w_bf16, float* top_w_coef,
                                    void* stream) {
  if (tokens < 0 || hidden <= 0 || experts <= 0 || k <= 0 || k > experts)
    return fail(MRB_ERR_ARG, "router_qrow_topk: bad shape");
  if (tokens == 0) return MRB_OK;
  if (experts > ROUTER_MAXE || k > 16) return fail(MRB_ERR_UNSUPPORTED, "router_qrow_topk: experts <= 256 and k <= 16");
  if (hidden % 8) return fail(MRB_ERR_UNSUPPORTED, "router_qrow_topk: hidden %lld is not a multiple of 8",
                              (long long)hidden);
  if (!x_bf16 || !codes || !scales || !logits_bf16 || !top_idx) return fail(MRB_ERR_ARG, "router_qrow_topk: null pointer");
  if (!aligned(x_bf16, 16) || !aligned(codes, 8))
    return fail(MRB_ERR_ARG, "router_qrow_topk: activation rows 16-byte and codes 8-byte aligned");
  if (tokens * experts > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "router_qrow_topk: too many tokens");
  const cudaStream_t s = (cudaStream_t)stream;
  // one CTA per expert up to one wave, else two experts per CTA; the selection's CTAs
  // (8 tokens each) wait for the logits on the SMs left over
  const int grid = experts <= num_sms() ? (int)experts : (int)((experts + 1) / 2);
  launch_kernel(router_qrow_logits_kernel, dim3((unsigned)grid), dim3(RQ_WARPS * 32), 0, s, true,
                (const __nv_bfloat16*)x_bf16, tokens, hidden, codes, scales, (int)experts,
                (__nv_bfloat16*)logits_bf16);
  int rc = launch_status("router_qrow_topk");
  if (rc) return rc;
  const int warps = 8;
  launch_kernel(router_topk_kernel<__nv_bfloat16>, dim3((unsigned)((tokens + warps - 1) / warps)), dim3(32 * warps), 0,
                s, true, (const __nv_bfloat16*)logits_bf16, tokens, (int)experts, (int)k, renorm, top_idx, top_w_f32,
                (__nv_bfloat16*)top_w_bf16, top_w_coef);
  return launch_status("router_qrow_topk");
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

namespace mrb {
// Checks, plans and launches one grouped projection (see mrb_grouped_qrow); `ov` carries the
// overlap fields of GroupedArgs (all zero for a lone launch).
static int grouped_launch(const void* x_bf16, const int64_t* row_ids, const int32_t* starts, const int32_t* counts,
                          int64_t experts, const int8_t* codes, int64_t codes_stride, const float* scales,
                          int64_t scales_stride, const int32_t* slot_of, int64_t n, int64_t k, int64_t up_rows,
                          int swiglu, int64_t rows_hint, void* y_bf16, const GroupedArgs& ov, int* chunks_out,
                          cudaStream_t s) {
  if (experts <= 0 || n <= 0 || k <= 0) return fail(MRB_ERR_ARG, "grouped_qrow: bad shape");
  if (!x_bf16 || !starts || !counts || !codes || !scales || !y_bf16) return fail(MRB_ERR_ARG, "grouped_qrow: null pointer");
  if (k % 16) return fail(MRB_ERR_UNSUPPORTED, "grouped_qrow: in_features %lld is not a multiple of 16", (long long)k);
  if (!aligned(codes, 16) || (codes_stride % 16) || !aligned(x_bf16, 16))
    return fail(MRB_ERR_ARG, "grouped_qrow: codes and activation rows must be 16-byte aligned");
  if (swiglu && up_rows < n) return fail(MRB_ERR_ARG, "grouped_qrow: up rows overlap the gate rows");
  // rows per pass: 16 (two n8 tiles) when experts average 8 rows or more, else 8, then the
  // most whose staged activations fit next to the ring
  int maxr = (rows_hint >= 8 * experts) ? GX_MAXR : GX_MAXR / 2;
  while (maxr > 1 && gx_smem_bytes(k, !swiglu, maxr) > 227 * 1024) maxr /= 2;
  const size_t smem = gx_smem_bytes(k, !swiglu, maxr);
  if (smem > 227 * 1024) return fail(MRB_ERR_UNSUPPORTED, "grouped_qrow: in_features %lld too large", (long long)k);
  if (experts * ((n + GX_ROWS - 1) / GX_ROWS) > 0x7fffffffLL)
    return fail(MRB_ERR_UNSUPPORTED, "grouped_qrow: too many expert tiles");
  GroupedArgs a = ov;
  a.x = (const __nv_bfloat16*)x_bf16;
  a.row_ids = row_ids;
  a.starts = starts;
  a.counts = counts;
  a.E = (int)experts;
  a.codes = codes;
  a.codes_stride = codes_stride;
  a.scales = scales;
  a.scales_stride = scales_stride;
  a.slot_of = slot_of;
  a.n = n;
  a.k = k;
  a.up_rows = up_rows;
  a.y = (__nv_bfloat16*)y_bf16;
  a.maxr = maxr;
  // two CTAs per SM when two fit; chunks of whole tiles per warp sized for about two work
  // items per CTA. The grid never exceeds one resident wave (the overlapped down launch
  // relies on every gate/up CTA running).
  const int64_t slots = (int64_t)num_sms() * (2 * (smem + 1024) <= 228 * 1024 ? 2 : 1);
  const int64_t rtiles = (n + GX_ROWS - 1) / GX_ROWS;
  const int64_t per_warp = std::max<int64_t>(1, experts * rtiles / (GX_WARPS * 2 * slots));
  // few experts (an expert-parallel shard): smaller chunks so the items still cover every
  // CTA slot -- some warps of a CTA idle, but every SM streams weights
  const int64_t fill = std::max<int64_t>(1, (experts * rtiles + slots - 1) / slots);
  a.chunk_tiles = (int)std::min<int64_t>(rtiles, std::min<int64_t>(per_warp * GX_WARPS, fill));
  a.chunks = (int)((rtiles + a.chunk_tiles - 1) / a.chunk_tiles);
  if (chunks_out) *chunks_out = a.chunks;
  const int64_t grid = std::min<int64_t>(experts * a.chunks, slots);
  auto run = [&](auto kern) -> int {
    const int smem_st = ensure_dynamic_smem((const void*)kern, smem, "grouped_qrow");
    if (smem_st) return smem_st;
    launch_kernel(kern, dim3((unsigned)grid), dim3(GX_THREADS), smem, s, true, a);
    return launch_status("grouped_qrow");
  };
  if (maxr > 8) return swiglu ? run(grouped_qrow_kernel<true, 2>) : run(grouped_qrow_kernel<false, 2>);
  return swiglu ? run(grouped_qrow_kernel<true, 1>) : run(grouped_qrow_kernel<false, 1>);
}

}  // namespace mrb

extern "C" int mrb_grouped_qrow(const void* x_bf16, const int64_t* row_ids, const int32_t* starts,
                                const int32_t* counts, int64_t experts, const int8_t* codes, int64_t codes_stride,
                                const float* scales, int64_t scales_stride, const int32_t* slot_of, int64_t n,
                                int64_t k, int64_t up_rows, int swiglu, int64_t rows_hint, void* y_bf16,
                                void* stream) {
  const GroupedArgs lone{};
  return grouped_launch(x_bf16, row_ids, starts, counts, experts, codes, codes_stride, scales, scales_stride, slot_of,
                        n, k, up_rows, swiglu, rows_hint, y_bf16, lone, nullptr, (cudaStream_t)stream);
}

extern "C" int mrb_grouped_expert_mlp(const void* x_bf16, const int64_t* row_ids, const int32_t* starts,
                                      const int32_t* counts, int64_t experts, const void* pages, int64_t page_stride,
                                      int64_t gate_up_codes_offset, int64_t gate_up_scales_offset,
                                      int64_t down_codes_offset, int64_t down_scales_offset, const int32_t* slot_of,
                                      int64_t hidden, int64_t ffn, int64_t rows_hint, void* act_bf16, void* y_bf16,
                                      uint32_t* sync, void* stream) {
  if (experts <= 0 || hidden <= 0 || ffn <= 0 || page_stride <= 0) return fail(MRB_ERR_ARG, "grouped_expert_mlp: bad shape");
  if (!pages || !act_bf16 || !sync) return fail(MRB_ERR_ARG, "grouped_expert_mlp: null pointer");
  if ((page_stride % 16) || (gate_up_codes_offset % 16) || (down_codes_offset % 16) || (gate_up_scales_offset % 4) ||
      (down_scales_offset % 4) || !aligned(sync, 4))
    return fail(MRB_ERR_ARG, "grouped_expert_mlp: page parts must be aligned (codes 16 B, scales and sync 4 B)");
  const char* base = (const char*)pages;
  const cudaStream_t s = (cudaStream_t)stream;
  GroupedArgs ov{};
  ov.overlap = 1;
  ov.ready = sync;
  ov.done = sync + experts;
  ov.error_flag = (int32_t*)(sync + 2 * experts);
  int gu_chunks = 0;
  int st = grouped_launch(x_bf16, row_ids, starts, counts, experts, (const int8_t*)(base + gate_up_codes_offset),
                          page_stride, (const float*)(base + gate_up_scales_offset), page_stride / 4, slot_of, ffn,
                          hidden, ffn, 1, rows_hint, act_bf16, ov, &gu_chunks, s);
  if (st) return st;
  ov.overlap = 2;
  ov.ready_target = gu_chunks;
  ov.wait_polls = 1LL << 22;  // x ~64 ns: ~0.3 s, far beyond any gate/up launch
  return grouped_launch(act_bf16, nullptr, starts, counts, experts, (const int8_t*)(base + down_codes_offset),
                        page_stride, (const float*)(base + down_scales_offset), page_stride / 4, slot_of, hidden, ffn,
                        0, 0, rows_hint, y_bf16, ov, nullptr, s);
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

extern "C" int mrb_ep_pack(const int64_t* top_idx, const float* top_w, int64_t tokens, int64_t k,
                           int64_t experts_per_rank, int64_t world, int64_t capacity, int32_t* send_expert,
                           float* coef_slot, int64_t* slot_of_assign, int32_t* slot_src, int32_t* error_flag,
                           void* stream) {
  const int64_t a = tokens * k;
  if (tokens < 0 || k <= 0 || experts_per_rank <= 0 || world <= 0 || capacity < a)
    return fail(MRB_ERR_ARG, "ep_pack: bad shape (capacity must hold tokens * k)");
  if (a > 8192 || world * capacity > (1LL << 24)) return fail(MRB_ERR_UNSUPPORTED, "ep_pack: too many assignments");
  if (!top_idx || !top_w || !send_expert || !coef_slot || !slot_of_assign || !slot_src)
    return fail(MRB_ERR_ARG, "ep_pack: null pointer");
  launch_kernel(ep_pack_kernel, dim3(1), dim3(1024), (size_t)std::max<int64_t>(a, 1) * sizeof(int32_t),
                (cudaStream_t)stream, true, top_idx, top_w, (int)a, (int)experts_per_rank, (int)world, (int)capacity,
                (int)k, send_expert, coef_slot, slot_of_assign, slot_src, error_flag);
  return launch_status("ep_pack");
}

extern "C" int mrb_ep_gather_rows(const void* source_bf16, int64_t hidden, const int32_t* slot_src, int64_t slots,
                                  void* send_rows_bf16, void* stream) {
  if (hidden <= 0 || hidden % 8 || slots < 0) return fail(MRB_ERR_ARG, "ep_gather_rows: bad shape");
  if (slots == 0) return MRB_OK;
  if (!source_bf16 || !slot_src || !send_rows_bf16) return fail(MRB_ERR_ARG, "ep_gather_rows: null pointer");
  if (!aligned(source_bf16, 16) || !aligned(send_rows_bf16, 16))
    return fail(MRB_ERR_ARG, "ep_gather_rows: rows must be 16-byte aligned");
  if (slots > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "ep_gather_rows: too many slots");
  launch_kernel(ep_gather_rows_kernel, dim3((unsigned)slots), dim3(128), 0, (cudaStream_t)stream, true,
                (const __nv_bfloat16*)source_bf16, hidden, slot_src, (__nv_bfloat16*)send_rows_bf16);
  return launch_status("ep_gather_rows");
}
