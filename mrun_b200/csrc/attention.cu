// Decode attention over a block-paged KV cache, plus the RoPE + KV-append step before it.
//
// KV layout: element (page, kv_head, slot, d) at page*stride_page + kv_head*stride_head +
// slot*stride_tok + d. The 16-token paged pool uses [pages, Hkv, 16, D] (the block-paged
// layout of mrun's paged attention, runtime/mlx_paged_attention.py:56-67); the same kernel
// reads mrun's contiguous caches by viewing each slot as one page: [slots, Hkv, cap, D]
// (engine/kernels/segmented_gqa_decode.py) or [B, S, Hkv, D] (engine/kernels/
// dense_qstore_cuda.py:1690-1760, with the provisional new K/V as an extra token).
//
// Split-K: each CTA owns (query row, KV head, split) and walks a contiguous range of
// 16-token tiles with an fp32 online softmax for all query heads of the group (GQA: K/V are
// read once per group). Splits publish (max, sum, acc) partials; the last CTA of a
// (row, head) group to finish merges them in split order, so results are deterministic.
#include "common.cuh"

#include <algorithm>

namespace mrb {

constexpr int AT_THREADS = 128;
constexpr int AT_TILE = 16;
constexpr int AT_MAX_GROUP = 16;

// ------------------------------------------------------------------ RoPE + KV append

struct RopeArgs {
  const __nv_bfloat16* q_in;
  const __nv_bfloat16* k_in;
  const __nv_bfloat16* v_in;
  int64_t in_stride;  // elements between consecutive tokens of q_in/k_in/v_in
  int64_t tokens, hq, hkv, d;
  const int32_t* positions;
  const int32_t* token_rows;
  const float* cos_tab;  // [rope_len, d/2] or null (no rotation)
  const float* sin_tab;
  int64_t rope_len;
  __nv_bfloat16* q_out;  // [tokens, hq, d] or null
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t stride_page, stride_head, stride_tok, page_size;
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t num_pages;
  int32_t* error_flag;
};

// Rotate-half RoPE exactly as the reference evaluates it in fp32
// (engine/dense_qstore_cuda.py:689-704): out = bf16(v*cos + rot(v)*sin), with separately
// rounded products (no fused multiply-add) and rot(v) = cat(-v[h:], v[:h]).
__device__ __forceinline__ float rope_elem(const __nv_bfloat16* v, int i, int half, const float* c, const float* s) {
  const int j = i < half ? i : i - half;
  const float x = __bfloat162float(v[i]);
  const float r = i < half ? -__bfloat162float(v[i + half]) : __bfloat162float(v[i - half]);
  return __fadd_rn(__fmul_rn(x, c[j]), __fmul_rn(r, s[j]));
}

__global__ void __launch_bounds__(256) rope_kv_append_kernel(RopeArgs a) {
  const int64_t t = blockIdx.x;
  const int half = (int)(a.d / 2);
  const int64_t pos = a.positions[t];
  const int64_t row = a.token_rows ? a.token_rows[t] : 0;
  const float* c = nullptr;
  const float* s = nullptr;
  bool ok = pos >= 0;
  if (a.cos_tab) {
    ok = ok && pos < a.rope_len;
    c = a.cos_tab + pos * half;
    s = a.sin_tab + pos * half;
  }
  int64_t page = -1;
  if (ok) {
    const int64_t lp = pos / a.page_size;
    page = a.block_table[row * a.bt_stride + lp];
    ok = page >= 0 && page < a.num_pages;
  }
  if (!ok) {
    if (threadIdx.x == 0 && a.error_flag) atomicExch(a.error_flag, 1);
    return;
  }
  const int64_t slot = pos % a.page_size;
  // queries
  if (a.q_out) {
    const __nv_bfloat16* qi = a.q_in + t * a.in_stride;
    for (int64_t e = threadIdx.x; e < a.hq * a.d; e += blockDim.x) {
      const int64_t h = e / a.d;
      const int i = (int)(e - h * a.d);
      const float v = c ? rope_elem(qi + h * a.d, i, half, c, s) : __bfloat162float(qi[e]);
      a.q_out[t * a.hq * a.d + e] = __float2bfloat16_rn(v);
    }
  }
  const __nv_bfloat16* ki = a.k_in + t * a.in_stride;
  const __nv_bfloat16* vi = a.v_in + t * a.in_stride;
  for (int64_t e = threadIdx.x; e < a.hkv * a.d; e += blockDim.x) {
    const int64_t h = e / a.d;
    const int i = (int)(e - h * a.d);
    const int64_t dst = page * a.stride_page + h * a.stride_head + slot * a.stride_tok + i;
    const float kv = c ? rope_elem(ki + h * a.d, i, half, c, s) : __bfloat162float(ki[e]);
    a.k_cache[dst] = __float2bfloat16_rn(kv);
    a.v_cache[dst] = vi[e];
  }
}

// ------------------------------------------------------------------ paged attention

struct AttnArgs {
  const __nv_bfloat16* q;  // [rows, hq, d]
  int64_t rows, hq, hkv;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  int64_t stride_page, stride_head, stride_tok, page_size;
  const int32_t* block_table;
  int64_t bt_stride;
  const int32_t* row_seq;  // block-table row per query row (null: identity)
  const int32_t* row_len;  // committed tokens per query row
  const __nv_bfloat16* k_new;  // [rows, hkv, d] provisional token at position row_len (or null)
  const __nv_bfloat16* v_new;
  float scale;
  int nsplit;
  int tiles_per_split;
  __nv_bfloat16* out;  // [rows, hq, d]
  float* part;         // [rows*hkv][nsplit][group][2 + d]
  unsigned* counters;  // [rows*hkv]
};

template <int D>
__global__ void __launch_bounds__(AT_THREADS) paged_attention_kernel(AttnArgs a) {
  static_assert(D <= AT_THREADS && D % 64 == 0, "one thread per head dimension");
  constexpr int PARTS = 8;          // threads cooperating on one (token, head) dot product
  constexpr int DPP = D / PARTS;    // dims per part
  const int group = (int)(a.hq / a.hkv);
  const int64_t rh = blockIdx.x;  // row * hkv + kv head
  const int split = blockIdx.y;
  const int64_t r = rh / a.hkv;
  const int kvh = (int)(rh - r * a.hkv);
  const int tid = threadIdx.x;

  __shared__ float qs[AT_MAX_GROUP][D];
  __shared__ float ps[AT_MAX_GROUP][AT_TILE];
  __shared__ float m_s[AT_MAX_GROUP], l_s[AT_MAX_GROUP], alpha_s[AT_MAX_GROUP];
  __shared__ bool is_last;

  for (int e = tid; e < group * D; e += AT_THREADS) {
    const int g = e / D, dd = e - g * D;
    qs[g][dd] = __bfloat162float(a.q[(r * a.hq + (int64_t)kvh * group + g) * D + dd]);
  }
  if (tid < group) {
    m_s[tid] = -INFINITY;
    l_s[tid] = 0.f;
  }
  float acc[AT_MAX_GROUP];
#pragma unroll
  for (int g = 0; g < AT_MAX_GROUP; ++g) acc[g] = 0.f;
  __syncthreads();

  const int64_t seq = a.row_seq ? a.row_seq[r] : r;
  const int64_t len = a.row_len[r];
  const bool has_new = a.k_new != nullptr;
  const int64_t total = len + (has_new ? 1 : 0);
  const int64_t t_begin = (int64_t)split * a.tiles_per_split * AT_TILE;
  const int64_t t_end = min(total, t_begin + (int64_t)a.tiles_per_split * AT_TILE);
  const int64_t khead = (int64_t)kvh * a.stride_head;

  const int my_tok = tid / PARTS;  // token within the tile for the score phase
  const int part = tid % PARTS;
  for (int64_t t0 = t_begin; t0 < t_end; t0 += AT_TILE) {
    // ---- scores: 16 tokens x group heads, 8 threads per (token) dot product
    const int64_t tok = t0 + my_tok;
    float kreg[DPP];
    const bool valid = tok < t_end;
    if (valid) {
      const __nv_bfloat16* kp;
      if (has_new && tok == len) {
        kp = a.k_new + (r * a.hkv + kvh) * D;
      } else {
        const int64_t page = a.block_table[seq * a.bt_stride + tok / a.page_size];
        kp = a.k_cache + page * a.stride_page + khead + (tok % a.page_size) * a.stride_tok;
      }
      const uint4* kv = reinterpret_cast<const uint4*>(kp + part * DPP);
#pragma unroll
      for (int v = 0; v < DPP / 8; ++v) {
        const uint4 raw = __ldg(kv + v);
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) kreg[v * 8 + i] = __bfloat162float(e[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < DPP; ++i) kreg[i] = 0.f;
    }
    for (int g = 0; g < group; ++g) {
      float sdot = 0.f;
#pragma unroll
      for (int i = 0; i < DPP; ++i) sdot = fmaf(qs[g][part * DPP + i], kreg[i], sdot);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 4);
      if (part == 0) ps[g][my_tok] = valid ? sdot * a.scale : -INFINITY;
    }
    __syncthreads();
    // ---- online softmax update, 16 lanes per head (all lanes take part in the shuffles)
    {
      const bool active = tid < group * AT_TILE;
      const int g = active ? tid / AT_TILE : 0;
      const int j = tid % AT_TILE;
      const float sc = active ? ps[g][j] : -INFINITY;
      float mx = sc;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_old = active ? m_s[g] : -INFINITY;
      const float m_new = fmaxf(m_old, mx);
      const float p = (m_new == -INFINITY) ? 0.f : expf(sc - m_new);
      float sum = p;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (active) {
        ps[g][j] = p;
        if (j == 0) {
          const float alpha = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
          alpha_s[g] = alpha;
          l_s[g] = l_s[g] * alpha + sum;
          m_s[g] = m_new;
        }
      }
    }
    __syncthreads();
    // ---- acc[g][d] = acc * alpha + sum_j p[g][j] * V[j][d]
    if (tid < D) {
      const int dd = tid;
      float vv[AT_TILE];
#pragma unroll
      for (int j = 0; j < AT_TILE; ++j) {
        const int64_t tj = t0 + j;
        if (tj < t_end) {
          const __nv_bfloat16* vp;
          if (has_new && tj == len) {
            vp = a.v_new + (r * a.hkv + kvh) * D;
          } else {
            const int64_t page = a.block_table[seq * a.bt_stride + tj / a.page_size];
            vp = a.v_cache + page * a.stride_page + khead + (tj % a.page_size) * a.stride_tok;
          }
          vv[j] = __bfloat162float(vp[dd]);
        } else {
          vv[j] = 0.f;
        }
      }
#pragma unroll
      for (int g = 0; g < AT_MAX_GROUP; ++g) {
        if (g < group) {
          float s = acc[g] * alpha_s[g];
#pragma unroll
          for (int j = 0; j < AT_TILE; ++j) s = fmaf(ps[g][j], vv[j], s);
          acc[g] = s;
        }
      }
    }
    __syncthreads();
  }

  // ---- finish: direct store, or publish a partial and let the last split merge
  if (a.nsplit == 1) {
    if (tid < D) {
#pragma unroll
      for (int g = 0; g < AT_MAX_GROUP; ++g) {
        if (g < group) {
          const float l = l_s[g];
          const float v = l > 0.f ? acc[g] / l : 0.f;
          a.out[(r * a.hq + (int64_t)kvh * group + g) * D + tid] = __float2bfloat16_rn(v);
        }
      }
    }
    return;
  }
  float* my = a.part + ((rh * a.nsplit + split) * group) * (2 + D);
  if (tid < D) {
#pragma unroll
    for (int g = 0; g < AT_MAX_GROUP; ++g)
      if (g < group) my[g * (2 + D) + 2 + tid] = acc[g];
  }
  if (tid < group) {
    my[tid * (2 + D)] = m_s[tid];
    my[tid * (2 + D) + 1] = l_s[tid];
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&a.counters[rh], 1u);
    is_last = prev == (unsigned)(a.nsplit - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* base = a.part + (rh * a.nsplit) * group * (2 + D);
  for (int dd = tid; dd < D; dd += AT_THREADS) {
    for (int g = 0; g < group; ++g) {
      float mx = -INFINITY;
      for (int s = 0; s < a.nsplit; ++s) mx = fmaxf(mx, __ldcg(base + (s * group + g) * (2 + D)));
      float l = 0.f, o = 0.f;
      for (int s = 0; s < a.nsplit; ++s) {
        const float* p = base + (s * group + g) * (2 + D);
        const float ms = __ldcg(p);
        const float w = (ms == -INFINITY) ? 0.f : expf(ms - mx);
        l = fmaf(__ldcg(p + 1), w, l);
        o = fmaf(__ldcg(p + 2 + dd), w, o);
      }
      a.out[(r * a.hq + (int64_t)kvh * group + g) * D + dd] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
    }
  }
  if (tid == 0) a.counters[rh] = 0u;  // ready for the next launch (graph replays)
}

struct SplitPlan {
  int nsplit;
  int tiles_per_split;
};

static SplitPlan plan_splits(int64_t rows, int64_t hkv, int64_t max_total) {
  const int64_t tiles = std::max<int64_t>(1, (max_total + AT_TILE - 1) / AT_TILE);
  const int64_t groups = std::max<int64_t>(1, rows * hkv);
  const int64_t target = (2LL * num_sms() + groups - 1) / groups;  // splits wanted per group
  int64_t tps = std::max<int64_t>(2, (tiles + target - 1) / target);
  tps = std::min<int64_t>(tps, tiles);
  const int64_t ns = (tiles + tps - 1) / tps;
  return SplitPlan{(int)ns, (int)tps};
}

// Workspace layout: AT_MAX_COUNTERS merge counters at offset 0 (fixed, so that a buffer
// reused across different shapes never finds stale partials where counters live), then the
// fp32 partials. Splitting only happens for fewer than 2 * SMs (row, head) groups.
constexpr int64_t AT_MAX_COUNTERS = 4096;
constexpr size_t AT_COUNTER_BYTES = AT_MAX_COUNTERS * sizeof(unsigned);

static size_t workspace_bytes(int64_t rows, int64_t hq, int64_t hkv, int64_t d, const SplitPlan& p) {
  if (p.nsplit <= 1) return 0;
  const int64_t group = hq / hkv;
  return AT_COUNTER_BYTES + (size_t)rows * hkv * p.nsplit * group * (2 + d) * sizeof(float);
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_rope_kv_append(const void* q_in, const void* k_in, const void* v_in, int64_t in_row_stride,
                                  int64_t tokens, int64_t hq, int64_t hkv, int64_t head_dim,
                                  const int32_t* positions, const int32_t* token_rows, const float* rope_cos,
                                  const float* rope_sin, int64_t rope_len, void* q_out, void* k_cache,
                                  void* v_cache, int64_t stride_page, int64_t stride_head, int64_t stride_tok,
                                  int64_t page_size, const int32_t* block_table, int64_t block_table_stride,
                                  int64_t num_pages, int32_t* error_flag, void* stream) {
  if (tokens < 0 || hkv <= 0 || head_dim <= 0 || head_dim % 2 || page_size <= 0 || num_pages <= 0)
    return fail(MRB_ERR_ARG, "rope_kv_append: bad shape");
  if (tokens == 0) return MRB_OK;
  if (!k_in || !v_in || !positions || !k_cache || !v_cache || !block_table)
    return fail(MRB_ERR_ARG, "rope_kv_append: null pointer");
  if (q_out && (!q_in || hq <= 0)) return fail(MRB_ERR_ARG, "rope_kv_append: q_out needs q_in and hq");
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return fail(MRB_ERR_ARG, "rope_kv_append: cos/sin mismatch");
  if (tokens > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "rope_kv_append: too many tokens");
  RopeArgs a{(const __nv_bfloat16*)q_in, (const __nv_bfloat16*)k_in, (const __nv_bfloat16*)v_in, in_row_stride,
             tokens, hq, hkv, head_dim, positions, token_rows, rope_cos, rope_sin, rope_len,
             (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, stride_page, stride_head,
             stride_tok, page_size, block_table, block_table_stride, num_pages, error_flag};
  rope_kv_append_kernel<<<(unsigned)tokens, 256, 0, (cudaStream_t)stream>>>(a);
  return launch_status("rope_kv_append");
}

extern "C" size_t mrb_paged_attention_workspace(int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                                int64_t max_total_tokens) {
  if (rows <= 0 || hkv <= 0 || hq % hkv) return 0;
  return workspace_bytes(rows, hq, hkv, head_dim, plan_splits(rows, hkv, max_total_tokens));
}

extern "C" int mrb_paged_attention(const void* q, int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                   const void* k_cache, const void* v_cache, int64_t stride_page,
                                   int64_t stride_head, int64_t stride_tok, int64_t page_size,
                                   const int32_t* block_table, int64_t block_table_stride, const int32_t* row_seq,
                                   const int32_t* row_len, const void* k_new, const void* v_new, float scale,
                                   int64_t max_total_tokens, void* out, void* workspace, size_t workspace_size,
                                   void* stream) {
  if (rows < 0 || hq <= 0 || hkv <= 0 || hq % hkv || page_size <= 0 || max_total_tokens < 0)
    return fail(MRB_ERR_ARG, "paged_attention: bad shape");
  if (rows == 0) return MRB_OK;
  if (hq / hkv > AT_MAX_GROUP)
    return fail(MRB_ERR_UNSUPPORTED, "paged_attention: query group %lld exceeds %d", (long long)(hq / hkv),
                AT_MAX_GROUP);
  if (head_dim != 64 && head_dim != 128)
    return fail(MRB_ERR_UNSUPPORTED, "paged_attention: head_dim %lld (supported: 64, 128)", (long long)head_dim);
  if (!q || !k_cache || !v_cache || !block_table || !row_len || !out)
    return fail(MRB_ERR_ARG, "paged_attention: null pointer");
  if ((k_new == nullptr) != (v_new == nullptr)) return fail(MRB_ERR_ARG, "paged_attention: k_new/v_new mismatch");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || (stride_page % 8) || (stride_head % 8) || (stride_tok % 8) ||
      (k_new && !aligned(k_new, 16)))
    return fail(MRB_ERR_ARG, "paged_attention: K/V rows must be 16-byte aligned");
  const SplitPlan plan = plan_splits(rows, hkv, max_total_tokens);
  const size_t need = workspace_bytes(rows, hq, hkv, head_dim, plan);
  if (need > 0 && (workspace == nullptr || workspace_size < need))
    return fail(MRB_ERR_ARG, "paged_attention: workspace of %zu bytes required (got %zu)", need, workspace_size);
  if (rows * hkv > 0x7fffffffLL || plan.nsplit > 65535)
    return fail(MRB_ERR_UNSUPPORTED, "paged_attention: grid too large");
  AttnArgs a{(const __nv_bfloat16*)q, rows, hq, hkv, (const __nv_bfloat16*)k_cache, (const __nv_bfloat16*)v_cache,
             stride_page, stride_head, stride_tok, page_size, block_table, block_table_stride, row_seq, row_len,
             (const __nv_bfloat16*)k_new, (const __nv_bfloat16*)v_new, scale, plan.nsplit, plan.tiles_per_split,
             (__nv_bfloat16*)out, nullptr, nullptr};
  if (need > 0) {
    if (rows * hkv > AT_MAX_COUNTERS) return fail(MRB_ERR_UNSUPPORTED, "paged_attention: too many split groups");
    a.counters = (unsigned*)workspace;
    a.part = (float*)((char*)workspace + AT_COUNTER_BYTES);
  }
  dim3 grid((unsigned)(rows * hkv), (unsigned)plan.nsplit);
  if (head_dim == 128)
    paged_attention_kernel<128><<<grid, AT_THREADS, 0, (cudaStream_t)stream>>>(a);
  else
    paged_attention_kernel<64><<<grid, AT_THREADS, 0, (cudaStream_t)stream>>>(a);
  return launch_status("paged_attention");
}

// ------------------------------------------------------------------ decode-step bookkeeping

// After a greedy decode step: the chosen token becomes the next input, every row advances
// one position. Runs inside the captured decode graph so replays need no host writes.
__global__ void decode_advance_kernel(const int64_t* __restrict__ next_ids, int64_t* __restrict__ input_ids,
                                      int32_t* __restrict__ positions, int32_t* __restrict__ row_len,
                                      int64_t rows) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < rows) {
    input_ids[i] = next_ids[i];
    positions[i] += 1;
    row_len[i] += 1;
  }
}

extern "C" int mrb_decode_advance(const int64_t* next_ids, int64_t* input_ids, int32_t* positions,
                                  int32_t* row_len, int64_t rows, void* stream) {
  if (rows < 0) return fail(MRB_ERR_ARG, "decode_advance: bad rows");
  if (rows == 0) return MRB_OK;
  if (!next_ids || !input_ids || !positions || !row_len) return fail(MRB_ERR_ARG, "decode_advance: null pointer");
  decode_advance_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, (cudaStream_t)stream>>>(next_ids, input_ids,
                                                                                           positions, row_len, rows);
  return launch_status("decode_advance");
}
