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
#include "qrow_common.cuh"
#include "tc_common.cuh"

#include <algorithm>
#include <mutex>

namespace mrb {

constexpr int AT_TILE = 16;
constexpr int AT_MAX_GROUP = 16;
constexpr int AT_MAX_SPLIT = 128;  // splits per (row, head); merge stats live in wacc
constexpr int AT_STAGES = 4;       // K/V tiles per CTA in shared memory (cp.async ring)
#ifndef AT_CTAS_PER_SM
#define AT_CTAS_PER_SM 8  // split-K target: CTAs per SM
#endif
#ifndef AT_MIN_TILES
#define AT_MIN_TILES 4  // split-K: fewest 16-token tiles per split
#endif
#ifndef AT_MMA_CTAS_PER_SM
#define AT_MMA_CTAS_PER_SM 3  // split-K target of the tensor-core kernel (its resident CTAs per SM)
#endif

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
  const __nv_bfloat16* q_norm;  // [d] per-head RMSNorm weight for queries, or null
  const __nv_bfloat16* k_norm;  // [d] for keys, or null
  float norm_eps;
};

// Rotate-half RoPE exactly as the reference evaluates it in fp32
// (engine/dense_qstore_cuda.py:689-704): out = bf16(v*cos + rot(v)*sin), with separately
// rounded products (no fused multiply-add) and rot(v) = cat(-v[h:], v[:h]).
// With a norm weight the head is first RMS-normalised as the reference's per-head q/k norm
// (engine/qwen3_moe_cuda.py:3282-3285, 3903-3904): fp32 mean of squares, normalised value
// rounded to bf16, times the bf16 weight rounded to bf16.
// CTAs (token, group of 8 heads), one warp per head (queries, then keys, then values). Lane j handles
// the rotation pairs (2j, 2j+1) of the first half and their partners in the second half.
__device__ __forceinline__ void rope_head(const __nv_bfloat16* src, __nv_bfloat16* dst, int half, const float* c,
                                          const float* s, int lane, const __nv_bfloat16* nw = nullptr,
                                          float eps = 0.f) {
  float rs = 1.f;
  if (nw) {
    float ss = 0.f;
    for (int j = 2 * lane; j < half; j += 64) {
      const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + j));
      const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + half + j));
      ss += lo.x * lo.x + lo.y * lo.y + hi.x * hi.x + hi.y * hi.y;
    }
    ss = warp_sum(ss);
    rs = rsqrtf(ss / (float)(2 * half) + eps);
  }
  for (int j = 2 * lane; j < half; j += 64) {
    float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + j));
    float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(src + half + j));
    if (nw) {
      const float2 wl = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(nw + j));
      const float2 wh = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(nw + half + j));
      lo.x = round_bf16(round_bf16(lo.x * rs) * wl.x);
      lo.y = round_bf16(round_bf16(lo.y * rs) * wl.y);
      hi.x = round_bf16(round_bf16(hi.x * rs) * wh.x);
      hi.y = round_bf16(round_bf16(hi.y * rs) * wh.y);
    }
    float2 o_lo, o_hi;
    if (c) {
      const float2 cc = *reinterpret_cast<const float2*>(c + j);
      const float2 ss = *reinterpret_cast<const float2*>(s + j);
      o_lo.x = __fadd_rn(__fmul_rn(lo.x, cc.x), __fmul_rn(-hi.x, ss.x));
      o_lo.y = __fadd_rn(__fmul_rn(lo.y, cc.y), __fmul_rn(-hi.y, ss.y));
      o_hi.x = __fadd_rn(__fmul_rn(hi.x, cc.x), __fmul_rn(lo.x, ss.x));
      o_hi.y = __fadd_rn(__fmul_rn(hi.y, cc.y), __fmul_rn(lo.y, ss.y));
    } else {
      o_lo = lo;
      o_hi = hi;
    }
    *reinterpret_cast<__nv_bfloat162*>(dst + j) = __floats2bfloat162_rn(o_lo.x, o_lo.y);
    *reinterpret_cast<__nv_bfloat162*>(dst + half + j) = __floats2bfloat162_rn(o_hi.x, o_hi.y);
  }
}

__global__ void __launch_bounds__(256) rope_kv_append_kernel(RopeArgs a) {
  pdl_launch_dependents();
  pdl_wait();
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const int64_t nq = a.q_out ? a.hq : 0;
  // heads spread over the CTAs of grid y, one warp per head: each head is a short chain of
  // dependent loads, so they run side by side instead of one after another
  for (int64_t h = (int64_t)blockIdx.y * nwarps + warp; h < nq + 2 * a.hkv; h += (int64_t)nwarps * gridDim.y) {
    if (h < nq) {
      rope_head(a.q_in + t * a.in_stride + h * a.d, a.q_out + (t * a.hq + h) * a.d, half, c, s, lane, a.q_norm,
                a.norm_eps);
    } else if (h < nq + a.hkv) {
      const int64_t kh = h - nq;
      rope_head(a.k_in + t * a.in_stride + kh * a.d,
                a.k_cache + page * a.stride_page + kh * a.stride_head + slot * a.stride_tok, half, c, s, lane,
                a.k_norm, a.norm_eps);
    } else {
      const int64_t vh = h - nq - a.hkv;
      rope_head(a.v_in + t * a.in_stride + vh * a.d,
                a.v_cache + page * a.stride_page + vh * a.stride_head + slot * a.stride_tok, half, nullptr, nullptr,
                lane);
    }
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
  float* part;         // fixed splits: [rows*hkv][nsplit][group][2 + d]; balanced: [bal_ctas + rows*hkv][group][2 + d]
  unsigned* counters;  // [rows*hkv], zero between launches
  unsigned* meta;      // [rows*hkv]: per group (first partial slot << 16) | partials (warp schedule)
  int bal_ctas;        // > 0: balanced schedule over this many CTAs (tensor-core kernel)
  int max_tiles;       // balanced: tiles per group at most (the host's context bound)
  int tma;             // 1: the TMA kernel (canonical paged pool); kmap/vmap are set
  int warp_sched;      // with tma and bal_ctas: one tile range per warp, then the merge kernel
  CUtensorMap kmap;    // K pool as [rows, 128] bf16, box [16, 64], 128-byte swizzle
  CUtensorMap vmap;
};

__device__ __forceinline__ int64_t kv_offset(const AttnArgs& a, int64_t seq, int64_t tok, int64_t khead) {
  const unsigned t = (unsigned)tok, ps = (unsigned)a.page_size;  // positions < 2^31
  const unsigned lp = t / ps;
  const int64_t page = a.block_table[seq * a.bt_stride + lp];
  return page * a.stride_page + khead + (int64_t)(t - lp * ps) * a.stride_tok;
}

// One 16-token tile of the scalar decode attention for one warp (= one query head): the
// lane's token score (lane = token + 16 * half of the head dim, K rows XOR-swizzled by 16-byte
// chunk), the fp32 online-softmax update of (m, l) and acc += p_t * V[t][lane's D/32 dims].
// `valid`: this lane's token lies inside the range being attended.
template <int D>
__device__ __forceinline__ void attend_tile(const __nv_bfloat16 (*ks)[D], const __nv_bfloat16 (*vs)[D],
                                            const float (&qreg)[D / 2], bool valid, int lane, float& m, float& l,
                                            float (&acc)[D / 32]) {
  constexpr int HALF = D / 2, VD = D / 32;
  const int my_tok = lane & 15, half = lane >> 4;
  float sc = 0.f;
#pragma unroll
  for (int c8 = 0; c8 < HALF / 8; ++c8) {
    const int c = half * (HALF / 8) + c8;
    const uint4 raw = reinterpret_cast<const uint4*>(&ks[my_tok][0])[c ^ (my_tok & 7)];
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h2[j]);
      sc = fmaf(qreg[c8 * 8 + 2 * j], f.x, sc);
      sc = fmaf(qreg[c8 * 8 + 2 * j + 1], f.y, sc);
    }
  }
  sc += __shfl_xor_sync(0xffffffffu, sc, 16);
  if (!valid) sc = -INFINITY;
  float mx = sc;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float m_new = fmaxf(m, mx);
  const float p = (m_new == -INFINITY) ? 0.f : expf(sc - m_new);
  float sum = p;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float alpha = (m == -INFINITY) ? 0.f : expf(m - m_new);
  l = l * alpha + sum;
  m = m_new;
#pragma unroll
  for (int k = 0; k < VD; ++k) acc[k] *= alpha;
#pragma unroll
  for (int t = 0; t < AT_TILE; ++t) {
    const float pt = __shfl_sync(0xffffffffu, p, t);
    if (VD == 4) {
      const uint2 raw = *reinterpret_cast<const uint2*>(&vs[t][lane * 4]);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 f0 = __bfloat1622float2(h2[0]), f1 = __bfloat1622float2(h2[1]);
      acc[0] = fmaf(pt, f0.x, acc[0]);
      acc[1 % VD] = fmaf(pt, f0.y, acc[1 % VD]);
      acc[2 % VD] = fmaf(pt, f1.x, acc[2 % VD]);
      acc[3 % VD] = fmaf(pt, f1.y, acc[3 % VD]);
    } else {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vs[t][lane * 2]));
      acc[0] = fmaf(pt, f.x, acc[0]);
      acc[1 % VD] = fmaf(pt, f.y, acc[1 % VD]);
    }
  }
}

// Decode attention, one warp per query head of the GQA group (blockDim = 32 * group).
// The CTA owns (query row, KV head, split) and walks the split's 16-token tiles through a
// 4-stage cp.async ring in shared memory (K XOR-swizzled so the score reads are
// conflict-free; three tiles in flight while one is scored, one barrier per tile), and every
// warp runs an fp32 online softmax for its head. Score phase:
// lane = (token, half of the head dim); value phase: lane owns D/32 consecutive dims.
// Splits publish (max, sum, acc) partials; the last CTA of the (row, head) group merges them
// in split order (deterministic), each warp merging its own head.
template <int D>
__global__ void __launch_bounds__(AT_MAX_GROUP * 32) paged_attention_kernel(const __grid_constant__ AttnArgs a) {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  constexpr int HALF = D / 2;     // dims per lane in the score phase
  constexpr int VD = D / 32;      // dims per lane in the value phase
  constexpr int CH = D / 8;       // 16-byte chunks per K/V row
  const int group = blockDim.x >> 5;
  const int64_t rh = blockIdx.x;  // row * hkv + kv head
  const int split = blockIdx.y;
  const int64_t r = rh / a.hkv;
  const int kvh = (int)(rh - r * a.hkv);
  const int tid = threadIdx.x, g = tid >> 5, lane = tid & 31;
  pdl_launch_dependents();
  pdl_wait();

  __shared__ __align__(16) __nv_bfloat16 ks[AT_STAGES][AT_TILE][D];
  __shared__ __align__(16) __nv_bfloat16 vs[AT_STAGES][AT_TILE][D];
  __shared__ bool is_last;

  const int64_t seq = a.row_seq ? a.row_seq[r] : r;
  const int64_t len = a.row_len[r];
  const bool has_new = a.k_new != nullptr;
  const int64_t total = len + (has_new ? 1 : 0);
  const int64_t t_begin = (int64_t)split * a.tiles_per_split * AT_TILE;
  const int64_t t_end = min(total, t_begin + (int64_t)a.tiles_per_split * AT_TILE);
  const int ntile = t_end > t_begin ? (int)((t_end - t_begin + AT_TILE - 1) / AT_TILE) : 0;
  const int64_t khead = (int64_t)kvh * a.stride_head;
  const int my_tok = lane & 15, half = lane >> 4;

  // ---- K/V tile ring: tile i of this split lands in stage i % AT_STAGES (cp.async, zero fill
  // past the split's end); AT_STAGES - 1 tiles are in flight while one is scored
  auto issue = [&](int i) {
    if (i < ntile) {
      const int st = i % AT_STAGES;
      const int64_t t0 = t_begin + (int64_t)i * AT_TILE;
      for (int e = tid; e < AT_TILE * CH; e += blockDim.x) {
        const int t = e / CH, c = e - t * CH;
        const int64_t tok = t0 + t;
        const bool ok = tok < t_end;
        const __nv_bfloat16 *kp = a.k_cache, *vp = a.v_cache;
        if (ok) {
          if (has_new && tok == len) {
            kp = a.k_new + (r * a.hkv + kvh) * D;
            vp = a.v_new + (r * a.hkv + kvh) * D;
          } else {
            const int64_t off = kv_offset(a, seq, tok, khead);
            kp = a.k_cache + off;
            vp = a.v_cache + off;
          }
        }
        cp_async16_zfill(reinterpret_cast<uint4*>(&ks[st][t][0]) + (c ^ (t & 7)),
                         reinterpret_cast<const uint4*>(kp) + (ok ? c : 0), ok);
        cp_async16_zfill(reinterpret_cast<uint4*>(&vs[st][t][0]) + c, reinterpret_cast<const uint4*>(vp) + (ok ? c : 0),
                         ok);
      }
    }
    cp_async_commit_group();
  };
#pragma unroll
  for (int i = 0; i < AT_STAGES - 1; ++i) issue(i);

  // this warp's query head, pre-scaled, for this lane's half of the dims
  float qreg[HALF];
  {
    const __nv_bfloat16* qp = a.q + (r * a.hq + (int64_t)kvh * group + g) * D + half * HALF;
#pragma unroll
    for (int i = 0; i < HALF; i += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(qp + i);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h2[j]);
        qreg[i + 2 * j] = f.x * a.scale;
        qreg[i + 2 * j + 1] = f.y * a.scale;
      }
    }
  }
  float m = -INFINITY, l = 0.f, acc[VD];
#pragma unroll
  for (int i = 0; i < VD; ++i) acc[i] = 0.f;

  for (int i = 0; i < ntile; ++i) {
    cp_async_wait_group<AT_STAGES - 2>();
    __syncthreads();  // tile i is in shared memory; every warp is done with tile i - 1
    issue(i + AT_STAGES - 1);  // refills the stage tile i - 1 used
    const int st = i % AT_STAGES;
    const int64_t t0 = t_begin + (int64_t)i * AT_TILE;
    attend_tile<D>(ks[st], vs[st], qreg, t0 + my_tok < t_end, lane, m, l, acc);
  }
  cp_async_wait_group<0>();

  __nv_bfloat16* out = a.out + (r * a.hq + (int64_t)kvh * group + g) * D + lane * VD;
  if (a.nsplit == 1) {
#pragma unroll
    for (int i = 0; i < VD; ++i) out[i] = __float2bfloat16_rn(l > 0.f ? acc[i] / l : 0.f);
    return;
  }
  // ---- publish this split's partial for the warp's head
  float* mine = a.part + ((rh * a.nsplit + split) * group + g) * (2 + D);
#pragma unroll
  for (int i = 0; i < VD; ++i) mine[2 + lane * VD + i] = acc[i];
  if (lane == 0) {
    mine[0] = m;
    mine[1] = l;
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
  // ---- last split: each warp merges its head over all splits, in split order
  const float* base = a.part + (rh * a.nsplit * group + g) * (2 + D);
  const int64_t sstride = (int64_t)group * (2 + D);
  float mx_all = -INFINITY;
  for (int s0 = lane; s0 < a.nsplit; s0 += 32) mx_all = fmaxf(mx_all, __ldcg(base + s0 * sstride));
  mx_all = warp_max(mx_all);
  float lsum = 0.f, o[VD];
#pragma unroll
  for (int i = 0; i < VD; ++i) o[i] = 0.f;
  for (int s0 = 0; s0 < a.nsplit; s0 += 8) {
    float ms[8], ls[8], av[8][VD];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool ok = s0 + j < a.nsplit;
      const float* p = base + (s0 + j) * sstride;
      ms[j] = ok ? __ldcg(p) : -INFINITY;
      ls[j] = ok ? __ldcg(p + 1) : 0.f;
#pragma unroll
      for (int i = 0; i < VD; ++i) av[j][i] = ok ? __ldcg(p + 2 + lane * VD + i) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float wt = (ms[j] == -INFINITY) ? 0.f : expf(ms[j] - mx_all);
      lsum = fmaf(ls[j], wt, lsum);
#pragma unroll
      for (int i = 0; i < VD; ++i) o[i] = fmaf(av[j][i], wt, o[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < VD; ++i) out[i] = __float2bfloat16_rn(lsum > 0.f ? o[i] / lsum : 0.f);
  __syncthreads();
  if (tid == 0) a.counters[rh] = 0u;  // ready for the next launch (graph replays)
}

// ------------------------------------------------------------------ fused decode step

// One new token per query row in one launch: the RoPE (and optional per-head q/k norm) of the
// row's query heads and key, the K/V append into the paged cache, and the grouped-query
// attention over tokens [0, pos] (the cached ones plus the new one). A cluster of S CTAs owns
// one (row, KV head); CTA c takes an even share of the row's tiles, computed on the device
// from the row's position, so a captured graph stays balanced as the context grows. The S
// partials (max, sum, acc) of every query head are merged in rank order through distributed
// shared memory -- no global scratch, no atomics.
constexpr int FD_MAX_CLUSTER = 16;
constexpr int FD_MIN_TILES = 2;  // fewest 16-token tiles per CTA when sizing the cluster

struct FusedArgs {
  const __nv_bfloat16* q_in;  // row r's query heads at q_in + r * in_stride, [hq, d]
  const __nv_bfloat16* k_in;  // [hkv, d] at k_in + r * in_stride
  const __nv_bfloat16* v_in;
  int64_t in_stride;
  int64_t rows, hq, hkv;
  const int32_t* positions;  // position of row r's new token (= its committed length)
  const int32_t* row_seq;    // block-table row per query row (null: identity)
  const float* cos_tab;      // [rope_len, d/2] or null (no rotation)
  const float* sin_tab;
  int64_t rope_len;
  const __nv_bfloat16* q_norm;  // [d] or null
  const __nv_bfloat16* k_norm;
  float norm_eps;
  __nv_bfloat16* k_cache;
  __nv_bfloat16* v_cache;
  int64_t stride_page, stride_head, stride_tok, page_size;
  const int32_t* block_table;
  int64_t bt_stride;
  int64_t num_pages;
  int32_t* error_flag;
  float scale;
  __nv_bfloat16* out;  // [rows, hq, d]
  int state_ready;     // positions, row_seq, block table and cached K/V may be read before the wait
};

template <int D>
__global__ void __launch_bounds__(AT_MAX_GROUP * 32) rope_append_attention_kernel(FusedArgs a) {
  constexpr int HALF = D / 2, VD = D / 32, CH = D / 8;
  const int group = blockDim.x >> 5;
  const int S = (int)gridDim.x;      // the cluster spans grid x
  const int rank = (int)blockIdx.x;  // = %cluster_ctarank
  const int64_t rh = blockIdx.y;     // row * hkv + kv head
  const int64_t r = rh / a.hkv;
  const int kvh = (int)(rh - r * a.hkv);
  const int tid = threadIdx.x, g = tid >> 5, lane = tid & 31;

  __shared__ __align__(16) __nv_bfloat16 ks[AT_STAGES][AT_TILE][D];
  __shared__ __align__(16) __nv_bfloat16 vs[AT_STAGES][AT_TILE][D];
  __shared__ __align__(16) __nv_bfloat16 qs[AT_MAX_GROUP][D];
  __shared__ __align__(16) __nv_bfloat16 knew[D];
  __shared__ __align__(16) __nv_bfloat16 vnew[D];
  __shared__ __align__(16) float pacc[AT_MAX_GROUP][D];
  __shared__ __align__(8) float pstat[AT_MAX_GROUP][2];

  pdl_launch_dependents();
  pdl_wait();

  // ---- the row's new position and its cache slot (every CTA of the cluster agrees)
  const int64_t seq = a.row_seq ? a.row_seq[r] : r;
  const int64_t pos = a.positions[r];
  bool ok = pos >= 0 && (a.cos_tab == nullptr || pos < a.rope_len);
  int64_t new_off = 0;
  if (ok) {
    const int64_t lp = pos / a.page_size;
    const int64_t page = a.block_table[seq * a.bt_stride + lp];
    ok = page >= 0 && page < a.num_pages;
    new_off = page * a.stride_page + (int64_t)kvh * a.stride_head + (pos - lp * a.page_size) * a.stride_tok;
  }
  __nv_bfloat16* out_base = a.out + (r * a.hq + (int64_t)kvh * group) * D;
  if (!ok) {  // cluster-uniform: no CTA reaches a cluster barrier
    if (rank == 0) {
      if (tid == 0 && a.error_flag) atomicExch(a.error_flag, 1);
      for (int e = tid; e < group * D; e += blockDim.x) out_base[e] = __float2bfloat16_rn(0.f);
    }
    return;
  }

  // ---- this CTA's share of the row's 16-token tiles
  const int64_t total = pos + 1;
  const int64_t tiles = (total + AT_TILE - 1) / AT_TILE;
  const int64_t per = (tiles + S - 1) / S;
  const int64_t tb = min(tiles, (int64_t)rank * per), te = min(tiles, tb + per);
  const int ntile = (int)(te - tb);
  const int64_t t_begin = tb * AT_TILE, t_end = min(total, te * AT_TILE);
  const bool owns_new = pos >= t_begin && pos < t_end;
  const int64_t khead = (int64_t)kvh * a.stride_head;
  bool bad_page = false;

  // K/V ring as in the split kernel; the new token's slot is zero-filled here and written
  // from shared memory once its tile has landed
  auto issue = [&](int i) {
    if (i < ntile) {
      const int st = i % AT_STAGES;
      const int64_t t0 = t_begin + (int64_t)i * AT_TILE;
      for (int e = tid; e < AT_TILE * CH; e += blockDim.x) {
        const int t = e / CH, c = e - t * CH;
        const int64_t tok = t0 + t;
        bool ld = tok < pos;
        int64_t off = 0;
        if (ld) {
          const unsigned lp = (unsigned)tok / (unsigned)a.page_size;
          const int64_t page = a.block_table[seq * a.bt_stride + lp];
          if (page < 0 || page >= a.num_pages) {
            ld = false;
            bad_page = true;
          } else {
            off = page * a.stride_page + khead + (int64_t)((unsigned)tok - lp * (unsigned)a.page_size) * a.stride_tok;
          }
        }
        cp_async16_zfill(reinterpret_cast<uint4*>(&ks[st][t][0]) + (c ^ (t & 7)),
                         reinterpret_cast<const uint4*>(a.k_cache + off) + (ld ? c : 0), ld);
        cp_async16_zfill(reinterpret_cast<uint4*>(&vs[st][t][0]) + c,
                         reinterpret_cast<const uint4*>(a.v_cache + off) + (ld ? c : 0), ld);
      }
    }
    cp_async_commit_group();
  };
#pragma unroll
  for (int i = 0; i < AT_STAGES - 1; ++i) issue(i);

  // ---- RoPE of this warp's query head (and of the new key in the CTA that owns it)
  const float* cr = a.cos_tab ? a.cos_tab + pos * HALF : nullptr;
  const float* sr = a.sin_tab ? a.sin_tab + pos * HALF : nullptr;
  const __nv_bfloat16* qrow = a.q_in + r * a.in_stride;
  rope_head(qrow + ((int64_t)kvh * group + g) * D, &qs[g][0], HALF, cr, sr, lane, a.q_norm, a.norm_eps);
  if (owns_new) {
    if (g == 0)
      rope_head(a.k_in + r * a.in_stride + (int64_t)kvh * D, knew, HALF, cr, sr, lane, a.k_norm, a.norm_eps);
    if (g == (group > 1 ? 1 : 0))
      rope_head(a.v_in + r * a.in_stride + (int64_t)kvh * D, vnew, HALF, nullptr, nullptr, lane);
  }
  __syncthreads();
  if (owns_new) {  // commit the new row to the cache (this CTA alone touches slot pos)
    for (int e = tid; e < 2 * CH; e += blockDim.x) {
      if (e < CH)
        reinterpret_cast<uint4*>(a.k_cache + new_off)[e] = reinterpret_cast<const uint4*>(knew)[e];
      else
        reinterpret_cast<uint4*>(a.v_cache + new_off)[e - CH] = reinterpret_cast<const uint4*>(vnew)[e - CH];
    }
  }
  const int half = lane >> 4, my_tok = lane & 15;
  float qreg[HALF];
#pragma unroll
  for (int i = 0; i < HALF; i += 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(&qs[g][half * HALF + i]);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h2[j]);
      qreg[i + 2 * j] = f.x * a.scale;
      qreg[i + 2 * j + 1] = f.y * a.scale;
    }
  }
  float m = -INFINITY, l = 0.f, acc[VD];
#pragma unroll
  for (int i = 0; i < VD; ++i) acc[i] = 0.f;

  for (int i = 0; i < ntile; ++i) {
    cp_async_wait_group<AT_STAGES - 2>();
    __syncthreads();  // tile i is in shared memory; every warp is done with tile i - 1
    issue(i + AT_STAGES - 1);
    const int st = i % AT_STAGES;
    const int64_t t0 = t_begin + (int64_t)i * AT_TILE;
    if (owns_new && pos < t0 + AT_TILE && pos >= t0) {  // CTA-uniform
      const int t = (int)(pos - t0);
      for (int c = tid; c < 2 * CH; c += blockDim.x) {
        if (c < CH)
          reinterpret_cast<uint4*>(&ks[st][t][0])[c ^ (t & 7)] = reinterpret_cast<const uint4*>(knew)[c];
        else
          reinterpret_cast<uint4*>(&vs[st][t][0])[c - CH] = reinterpret_cast<const uint4*>(vnew)[c - CH];
      }
      __syncthreads();
    }
    attend_tile<D>(ks[st], vs[st], qreg, t0 + my_tok < t_end, lane, m, l, acc);
  }
  cp_async_wait_group<0>();
  if (bad_page && a.error_flag) atomicExch(a.error_flag, 1);

  if (S == 1) {
#pragma unroll
    for (int i = 0; i < VD; ++i) out_base[g * D + lane * VD + i] = __float2bfloat16_rn(l > 0.f ? acc[i] / l : 0.f);
    return;
  }
  // ---- publish this CTA's partial of every head, then merge across the cluster
#pragma unroll
  for (int i = 0; i < VD; ++i) pacc[g][lane * VD + i] = acc[i];
  if (lane == 0) {
    pstat[g][0] = m;
    pstat[g][1] = l;
  }
  cluster_sync_all();
  const int h = rank + S * g;  // heads rank, rank + S, ... are merged by this CTA's warps 0, 1, ...
  if (h < group) {
    float ms = -INFINITY, ls = 0.f;
    if (lane < S) {
      const uint32_t ra = mapa_shared(smem_u32(&pstat[h][0]), (unsigned)lane);
      ms = ld_shared_cluster_f32(ra);
      ls = ld_shared_cluster_f32(ra + 4);
    }
    const float mx = warp_max(ms);
    const float wt = (ms == -INFINITY) ? 0.f : expf(ms - mx);
    const float lsum = warp_sum(ls * wt);
    const uint32_t acc_addr = smem_u32(&pacc[h][lane * VD]);
    float o[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) o[i] = 0.f;
    for (int s0 = 0; s0 < S; s0 += 8) {
      float av[8][VD];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool in = s0 + j < S;
        const uint32_t ra = mapa_shared(acc_addr, (unsigned)(in ? s0 + j : 0));
        if (VD == 4) {
          const float4 v = in ? ld_shared_cluster_v4f32(ra) : make_float4(0.f, 0.f, 0.f, 0.f);
          av[j][0] = v.x;
          av[j][1 % VD] = v.y;
          av[j][2 % VD] = v.z;
          av[j][3 % VD] = v.w;
        } else {
          const float2 v = in ? ld_shared_cluster_v2f32(ra) : make_float2(0.f, 0.f);
          av[j][0] = v.x;
          av[j][1 % VD] = v.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float w = __shfl_sync(0xffffffffu, wt, (s0 + j) & 31);
#pragma unroll
        for (int i = 0; i < VD; ++i) o[i] = fmaf(av[j][i], w, o[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < VD; ++i) out_base[h * D + lane * VD + i] = __float2bfloat16_rn(lsum > 0.f ? o[i] / lsum : 0.f);
  }
  cluster_sync_all();  // peers' shared memory stays alive until every merge has read it
}

// ------------------------------------------------------------------ tensor-core decode attention

// Two stages per warp keep a CTA at 70 KB of shared memory, so 3 CTAs (12 warps) share an
// SM: 64 rows x 28/4 heads, ctx U[128,2048] went 63.5 -> 48.2 us against 3 stages at 2 CTAs
// per SM (32 rows x 32/4 heads, ctx U[256,4096]: 50.4 -> 48.3 us).
#ifndef AM_RING_STAGES
#define AM_RING_STAGES 2
#endif
constexpr int AM_STAGES = AM_RING_STAGES;             // K/V tiles in flight per warp
constexpr int AM_ROW = 128 + 8;                       // padded smem row (bf16): conflict-free fragments
constexpr int AM_TILE_ELEMS = AT_TILE * AM_ROW;       // one K or V tile
constexpr int AM_STAGE_ELEMS = 2 * AM_TILE_ELEMS;     // K and V
constexpr int AM_MAX_WARPS = 4;

__host__ __device__ inline size_t am_smem_bytes(int warps) {
  const size_t ring = (size_t)warps * AM_STAGES * AM_STAGE_ELEMS * sizeof(__nv_bfloat16);
  // merge area: per-warp states [W][16][2 + D], then weights [W][16] and per-head (max, sum)
  const size_t merge = ((size_t)warps * 16 * (2 + 128) + (size_t)warps * 16 + 2 * 16) * sizeof(float);
  return ring > merge ? ring : merge;
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Decode attention on the tensor pipe (head_dim 128, GQA group <= 16).
//
// One work item: tiles [tile_lo, tile_hi) of (query row, KV head) group rh, attended by the
// CTA's W <= 4 warps, which take the item's 16-token tiles in turn (warp w: tiles w, w + W,
// ...), each through its own AM_STAGES-deep cp.async ring of K and V tiles (rows padded to
// 272 B so fragment reads are conflict-free). Per tile a warp computes S = Q K^T for all query heads of the group at
// once -- heads are the 16 rows of mma.sync m16n8k16 (bf16 inputs, fp32 accumulation), two
// 8-token column blocks, eight 16-dim k steps -- scales it in fp32, runs the online softmax
// per head row in fp32, and accumulates O += P V on the tensor pipe with P (rounded to
// bf16) reused straight from the score fragments and V fragments from ldmatrix.trans. The
// W partial states are merged through shared memory in warp order. With nparts == 1 the item
// is the whole group and writes the output; otherwise it publishes its state in slot `slot`
// of a.part, and the last of the group's nparts items to arrive merges slots [slot0, slot0 +
// nparts) in slot order (deterministic). Every thread of the CTA calls it with the same
// arguments, and the shared memory is free again when it returns.
__device__ __forceinline__ void am_item(const AttnArgs& a, int64_t rh, int64_t tile_lo, int64_t tile_hi, int64_t slot,
                                        int64_t slot0, int nparts) {
  constexpr int D = 128;
  const int W = blockDim.x >> 5;
  const int group = (int)(a.hq / a.hkv);
  const int64_t r = rh / a.hkv;
  const int kvh = (int)(rh - r * a.hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;

  extern __shared__ __align__(16) unsigned char am_smem[];
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(am_smem) + (size_t)warp * AM_STAGES * AM_STAGE_ELEMS;
  __shared__ bool is_last;

  const int64_t seq = a.row_seq ? a.row_seq[r] : r;
  const int64_t len = a.row_len[r];
  const bool has_new = a.k_new != nullptr;
  const int64_t total = len + (has_new ? 1 : 0);
  const int64_t t_begin = tile_lo * AT_TILE;
  const int64_t t_end = min(total, tile_hi * AT_TILE);
  // scores in base-2 units: exp(x * scale) = exp2(x * scale * log2(e)); running maxima and
  // the published partial maxima are in the same units
  const float scale2 = a.scale * 1.4426950408889634f;
  const int ntile = t_end > t_begin ? (int)((t_end - t_begin + AT_TILE - 1) / AT_TILE) : 0;
  const int nmine = warp < ntile ? (ntile - warp + W - 1) / W : 0;
  const int64_t khead = (int64_t)kvh * a.stride_head;

  // a 16-token tile (tiles start at multiples of 16) lies inside one page when the page size
  // is a multiple of 16: one block-table lookup per tile, then affine addresses
  const bool tile_in_page = (a.page_size % AT_TILE) == 0;
  // ---- this warp's K/V ring: its j-th tile (split tile warp + j*W) in stage j % AM_STAGES
  auto issue = [&](int j) {
    if (j < nmine && tile_in_page) {
      __nv_bfloat16* kst = ring + (j % AM_STAGES) * AM_STAGE_ELEMS;
      __nv_bfloat16* vst = kst + AM_TILE_ELEMS;
      const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
      const int64_t base = t0 < len ? kv_offset(a, seq, t0, khead) : 0;  // committed tokens only
      const int lim = (int)(t_end - t0), newt = has_new ? (int)(len - t0) : -1;
#pragma unroll
      for (int i = 0; i < AT_TILE * (D / 8) / 32; ++i) {
        const int e = lane + 32 * i;
        const int t = e >> 4, ch = e & 15;
        const bool ok = t < lim;
        const __nv_bfloat16 *kp = a.k_cache, *vp = a.v_cache;
        if (ok) {
          if (t == newt) {
            kp = a.k_new + (r * a.hkv + kvh) * D;
            vp = a.v_new + (r * a.hkv + kvh) * D;
          } else {
            const int64_t off = base + (int64_t)t * a.stride_tok;
            kp = a.k_cache + off;
            vp = a.v_cache + off;
          }
        }
        cp_async16_zfill(kst + t * AM_ROW + ch * 8, kp + (ok ? ch * 8 : 0), ok);
        cp_async16_zfill(vst + t * AM_ROW + ch * 8, vp + (ok ? ch * 8 : 0), ok);
      }
    } else if (j < nmine) {
      __nv_bfloat16* kst = ring + (j % AM_STAGES) * AM_STAGE_ELEMS;
      __nv_bfloat16* vst = kst + AM_TILE_ELEMS;
      const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
#pragma unroll 4
      for (int e = lane; e < AT_TILE * (D / 8); e += 32) {
        const int t = e >> 4, ch = e & 15;
        const int64_t tok = t0 + t;
        const bool ok = tok < t_end;
        const __nv_bfloat16 *kp = a.k_cache, *vp = a.v_cache;
        if (ok) {
          if (has_new && tok == len) {
            kp = a.k_new + (r * a.hkv + kvh) * D;
            vp = a.v_new + (r * a.hkv + kvh) * D;
          } else {
            const int64_t off = kv_offset(a, seq, tok, khead);
            kp = a.k_cache + off;
            vp = a.v_cache + off;
          }
        }
        cp_async16_zfill(kst + t * AM_ROW + ch * 8, kp + (ok ? ch * 8 : 0), ok);
        cp_async16_zfill(vst + t * AM_ROW + ch * 8, vp + (ok ? ch * 8 : 0), ok);
      }
    }
    cp_async_commit_group();
  };
#pragma unroll
  for (int j = 0; j < AM_STAGES - 1; ++j) issue(j);

  // ---- Q of the group as the mma A operand: rows g and g + 8 are query heads (zero beyond
  // the group), eight 16-dim k steps
  const bool two_halves = group > 8;
  uint32_t qa[D / 16][4];
  {
    const __nv_bfloat16* q0 = a.q + (r * a.hq + (int64_t)kvh * group) * D;
    const bool v0 = g < group, v1 = g + 8 < group;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d0 = ks * 16 + 2 * c;
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + g * D + d0) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(q0 + (g + 8) * D + d0) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + g * D + d0 + 8) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(q0 + (g + 8) * D + d0 + 8) : 0u;
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  for (int j = 0; j < nmine; ++j) {
    cp_async_wait_group<AM_STAGES - 2>();
    __syncwarp();  // the whole tile is in shared memory; the stage of tile j - 1 is free
    issue(j + AM_STAGES - 1);
    const __nv_bfloat16* kst = ring + (j % AM_STAGES) * AM_STAGE_ELEMS;
    const __nv_bfloat16* vst = kst + AM_TILE_ELEMS;
    const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
    // ---- scores: s[nt] = (head g | g+8) x (tokens nt*8 + 2c, +1)
    // K fragments by ldmatrix.x4: lane l addresses token nt*8 + (l & 7), dims
    // ks*16 + (l >> 3)*8, so the four matrices are (b0, b1) of k steps ks and ks + 1
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      const __nv_bfloat16* kr = kst + (nt * 8 + (lane & 7)) * AM_ROW + (lane >> 3) * 8;
#pragma unroll
      for (int ks = 0; ks < D / 16; ks += 2) {
        uint32_t kb[4];
        ldmatrix_x4(kb, kr + ks * 16);
        mma_bf16_16816(s[nt], qa[ks], kb[0], kb[1]);
        mma_bf16_16816(s[nt], qa[ks + 1], kb[2], kb[3]);
      }
    }
    // ---- online softmax per head row (rows g and g + 8), fp32
    const int lim = (int)(t_end - t0);  // tokens of this tile inside the split
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[nt][i] = nt * 8 + 2 * c + (i & 1) < lim ? s[nt][i] * scale2 : -INFINITY;
    // rows g + 8 hold query heads only for groups above 8; otherwise they stay empty
    float alpha[2] = {1.f, 1.f};
    if (!two_halves) s[0][2] = s[0][3] = s[1][2] = s[1][3] = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h == 1 && !two_halves) break;
      float mx = fmaxf(fmaxf(s[0][2 * h], s[0][2 * h + 1]), fmaxf(s[1][2 * h], s[1][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(mrow[h], mx);
      alpha[h] = (mrow[h] == -INFINITY) ? 0.f : exp2f(mrow[h] - m_new);
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float p = (m_new == -INFINITY) ? 0.f : exp2f(s[nt][2 * h + i] - m_new);
          s[nt][2 * h + i] = p;
          sum += p;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow[h] = lrow[h] * alpha[h] + sum;
      mrow[h] = m_new;
    }
    // ---- O = O * alpha + P V (P in bf16 as the A operand, V via ldmatrix.trans)
    const uint32_t pa[4] = {pack_bf16x2(s[0][0], s[0][1]), pack_bf16x2(s[0][2], s[0][3]),
                            pack_bf16x2(s[1][0], s[1][1]), pack_bf16x2(s[1][2], s[1][3])};
    // V fragments by ldmatrix.x4.trans: lanes 0-15 address tokens 0-15 at dims dt*8, lanes
    // 16-31 the same tokens at dims (dt+1)*8
    const __nv_bfloat16* vrow = vst + (lane & 15) * AM_ROW + (lane >> 4) * 8;
    // rescale only when some row's running max moved (alpha is exactly 1 otherwise)
    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][0] *= alpha[0];
        o[dt][1] *= alpha[0];
        o[dt][2] *= alpha[1];
        o[dt][3] *= alpha[1];
      }
    }
#pragma unroll
    for (int dt = 0; dt < D / 8; dt += 2) {
      uint32_t vb[4];
      ldmatrix_x4_trans(vb, vrow + dt * 8);
      mma_bf16_16816(o[dt], pa, vb[0], vb[1]);
      mma_bf16_16816(o[dt + 1], pa, vb[2], vb[3]);
    }
  }
  cp_async_wait_group<0>();
  __syncthreads();  // every warp is done with its ring: the space becomes the merge area

  // ---- merge the W warp states per head row in warp order
  float* mb = reinterpret_cast<float*>(am_smem);  // [W][16 rows][2 + D]
  {
    float* mine = mb + (size_t)warp * 16 * (2 + D);
    if (c == 0) {
      mine[g * (2 + D)] = mrow[0];
      mine[g * (2 + D) + 1] = lrow[0];
      mine[(g + 8) * (2 + D)] = mrow[1];
      mine[(g + 8) * (2 + D) + 1] = lrow[1];
    }
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      mine[g * (2 + D) + 2 + dt * 8 + 2 * c] = o[dt][0];
      mine[g * (2 + D) + 2 + dt * 8 + 2 * c + 1] = o[dt][1];
      mine[(g + 8) * (2 + D) + 2 + dt * 8 + 2 * c] = o[dt][2];
      mine[(g + 8) * (2 + D) + 2 + dt * 8 + 2 * c + 1] = o[dt][3];
    }
  }
  __syncthreads();
  // per head: the combined max and sum, and one weight per warp state (exp2f once per (warp,
  // head) instead of once per element)
  float* wts = mb + (size_t)W * 16 * (2 + D);  // [W][16]
  float* hstat = wts + (size_t)W * 16;         // [16] max, [16] sum
  if (tid < group) {
    const int h = tid;
    float mx = -INFINITY;
    for (int w = 0; w < W; ++w) mx = fmaxf(mx, mb[((size_t)w * 16 + h) * (2 + D)]);
    float l = 0.f;
    for (int w = 0; w < W; ++w) {
      const float* st = mb + ((size_t)w * 16 + h) * (2 + D);
      const float wt = (st[0] == -INFINITY) ? 0.f : exp2f(st[0] - mx);
      wts[w * 16 + h] = wt;
      l = fmaf(st[1], wt, l);
    }
    hstat[h] = mx;
    hstat[16 + h] = l;
  }
  __syncthreads();
  float* part_base = nparts > 1 ? a.part + slot * (int64_t)group * (2 + D) : nullptr;
  for (int idx = tid; idx < group * D; idx += blockDim.x) {
    const int h = idx / D, d = idx - h * D;
    const float mx = hstat[h], l = hstat[16 + h];
    float acc = 0.f;
    for (int w = 0; w < W; ++w) acc = fmaf(mb[((size_t)w * 16 + h) * (2 + D) + 2 + d], wts[w * 16 + h], acc);
    if (nparts == 1) {
      a.out[(r * a.hq + (int64_t)kvh * group + h) * D + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
    } else {
      float* p = part_base + (int64_t)h * (2 + D);
      p[2 + d] = acc;
      if (d == 0) {
        p[0] = mx;
        p[1] = l;
      }
    }
  }
  __syncthreads();  // the merge area is read; the next item may reuse the shared memory
  if (nparts == 1) return;
  __threadfence();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&a.counters[rh], 1u);
    is_last = prev == (unsigned)(nparts - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // ---- last split: warps merge the heads over all splits, in split order
  constexpr int VD = D / 32;
  const int64_t sstride = (int64_t)group * (2 + D);
  for (int h = warp; h < group; h += W) {
    const float* base = a.part + (slot0 * group + h) * (2 + D);
    float mx_all = -INFINITY;
    for (int s0 = lane; s0 < nparts; s0 += 32) mx_all = fmaxf(mx_all, __ldcg(base + s0 * sstride));
    mx_all = warp_max(mx_all);
    float lsum = 0.f, ov[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) ov[i] = 0.f;
    for (int s0 = 0; s0 < nparts; s0 += 8) {  // 8 partials' loads in flight at a time
      float ms[8], ls[8], av[8][VD];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const bool ok = s0 + jj < nparts;
        const float* p = base + (s0 + jj) * sstride;
        ms[jj] = ok ? __ldcg(p) : -INFINITY;
        ls[jj] = ok ? __ldcg(p + 1) : 0.f;
#pragma unroll
        for (int i = 0; i < VD; ++i) av[jj][i] = ok ? __ldcg(p + 2 + lane * VD + i) : 0.f;
      }
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const float wt = (ms[jj] == -INFINITY) ? 0.f : exp2f(ms[jj] - mx_all);
        lsum = fmaf(ls[jj], wt, lsum);
#pragma unroll
        for (int i = 0; i < VD; ++i) ov[i] = fmaf(av[jj][i], wt, ov[i]);
      }
    }
    __nv_bfloat16* out = a.out + (r * a.hq + (int64_t)kvh * group + h) * D + lane * VD;
#pragma unroll
    for (int i = 0; i < VD; ++i) out[i] = __float2bfloat16_rn(lsum > 0.f ? ov[i] / lsum : 0.f);
  }
  __syncthreads();
  if (tid == 0) a.counters[rh] = 0u;  // ready for the next launch (graph replays)
}


// Tiles of one (query row, KV head) group for the balanced schedule: the row's committed
// tokens plus the provisional one, at least one tile (an empty row still writes zeros), at
// most the host's bound.
__device__ __forceinline__ int am_row_tiles(const AttnArgs& a, int64_t r) {
  const int64_t total = (int64_t)a.row_len[r] + (a.k_new != nullptr ? 1 : 0);
  return (int)max((int64_t)1, min((int64_t)a.max_tiles, (total + AT_TILE - 1) / AT_TILE));
}

// Two schedules, one instantiation each (one copy of the item body per kernel keeps the code
// inside the instruction cache). Fixed splits: the CTA is (group blockIdx.x, split
// blockIdx.y) of tiles_per_split tiles. Balanced (a.bal_ctas > 0): the groups' tiles, as the
// rows' lengths give them, are laid end to end (group-major) and CTA c of P = min(bal_ctas,
// T) takes tiles [c*T/P, (c+1)*T/P) of the T in all, walking the groups its range touches;
// a group cut by a range boundary is finished by the last of its CTAs, which merges their
// partials in CTA order. Partial slot of (CTA c, group rh) = c + rh: along the tile order c
// and rh never both decrease, so no two (c, rh) pairs of one launch share a slot, and a
// group's slots are consecutive. The plan is recomputed from row_len by every CTA, so it
// follows the lengths of each launch (a captured graph needs no host update).
template <bool BALANCED, typename Item>
__device__ __forceinline__ void attn_schedule(const AttnArgs& a, Item&& item) {
  if constexpr (!BALANCED) {
    const int64_t rh = blockIdx.x;
    const int64_t split = blockIdx.y;
    item(rh, split * a.tiles_per_split, (split + 1) * a.tiles_per_split, rh * a.nsplit + split, rh * a.nsplit,
         a.nsplit);
    return;
  }
  extern __shared__ __align__(16) unsigned char am_smem[];
  int* pre = reinterpret_cast<int*>(am_smem);  // [rows + 1]: tiles of all groups of the rows before r
  const int R = (int)a.rows, hkv = (int)a.hkv;
  const int tid = threadIdx.x, lane = tid & 31;
  for (int r = tid; r < R; r += blockDim.x) pre[r + 1] = am_row_tiles(a, r) * hkv;
  if (tid == 0) pre[0] = 0;
  __syncthreads();
  if (tid < 32) {  // inclusive scan of pre[1..R], 32 rows at a time
    int carry = 0;
    for (int b = 1; b <= R; b += 32) {
      int v = b + lane <= R ? pre[b + lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (b + lane <= R) pre[b + lane] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  const int64_t T = pre[R];
  const int64_t P = min((int64_t)a.bal_ctas, T);
  const int64_t cta = blockIdx.x;
  const int64_t lo = cta * T / P, hi = (cta + 1) * T / P;
  int r = 0;  // the row holding tile lo: the largest r with pre[r] <= lo
  for (int L = 0, H = R; H - L > 1;) {
    const int M = (L + H) >> 1;
    if (pre[M] <= lo) L = M; else H = M;
    r = L;
  }
  int64_t rowstart = pre[r];
  int tr = (pre[r + 1] - pre[r]) / hkv;
  __syncthreads();  // the plan is read; the shared memory becomes the K/V rings
  if (cta >= P) return;
  int kvh = (int)((lo - rowstart) / tr);
  int64_t toff = lo - rowstart - (int64_t)kvh * tr;
  for (int64_t cur = lo; cur < hi;) {
    const int64_t gstart = rowstart + (int64_t)kvh * tr;  // the group's first tile
    const int64_t seg = min(hi - cur, (int64_t)tr - toff);
    const int64_t cf = ((gstart + 1) * P - 1) / T;      // the CTA holding the group's first tile
    const int64_t cl = ((gstart + tr) * P - 1) / T;     // ... and its last
    const int64_t rh = (int64_t)r * hkv + kvh;
    item(rh, toff, toff + seg, cta + rh, cf + rh, (int)(cl - cf + 1));
    cur += seg;
    toff = 0;
    if (++kvh == hkv && cur < hi) {
      kvh = 0;
      rowstart += (int64_t)hkv * tr;
      tr = am_row_tiles(a, ++r);
    }
  }
}

template <bool BALANCED>
__global__ void __launch_bounds__(AM_MAX_WARPS * 32, AT_MMA_CTAS_PER_SM) paged_attention_mma_kernel(const __grid_constant__ AttnArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  attn_schedule<BALANCED>(a, [&](int64_t rh, int64_t lo, int64_t hi, int64_t slot, int64_t slot0, int nparts) {
    am_item(a, rh, lo, hi, slot, slot0, nparts);
  });
}

// ------------------------------------------------------------------ TMA decode attention

// Decode attention for the canonical paged pool ([pages, Hkv, page_size, 128] bf16, page
// size a multiple of 16), head_dim 128, GQA group <= 8 * NT.
//
// Loads: each warp keeps an A2_STAGES-deep ring of 16-token tiles; one lane fetches a tile
// as four TMA boxes ([16 tokens x 64 dims] of K and of V, 128-byte swizzle) completing on
// the stage's mbarrier, so a tile costs a handful of instructions to request, and the page
// numbers of the warp's next 32 tiles are read in one go ahead of time (no block-table load
// on the path from one tile's request to the next).
// Math, transposed so that tokens (not the 8 heads of a group) fill the 16 rows of
// mma.sync m16n8k16 (bf16 inputs, fp32 accumulation): S^T = K Q^T (A = K tile by ldmatrix,
// B = the group's queries held in registers), online softmax per head column in base 2,
// then O^T += V^T P^T (A = V tile by ldmatrix.trans, B = P^T moved out of the score
// fragments with movmatrix.trans). Per tile 8 + 8 MMAs per 8 heads. Row sums stay per lane
// until the item ends. Partial states merge exactly as in am_item (same layouts, base-2
// maxima), so the schedules and the cross-CTA merge are shared.
#ifndef A2_RING_STAGES
#define A2_RING_STAGES 2
#endif
constexpr int A2_STAGES = A2_RING_STAGES;
constexpr int A2_BOX = AT_TILE * 64 * 2;        // [16 tokens x 64 dims] bf16: 2 KB
constexpr int A2_STAGE_BYTES = 4 * A2_BOX;      // K dims 0-63, K 64-127, V 0-63, V 64-127
constexpr int A2_TBL = 32;                      // page numbers fetched per batch, one per lane
constexpr int AT_BAL_MAX_ROWS_DEV = 1024;       // rows the balanced schedules take (prefix in shared memory)

__host__ __device__ inline size_t a2_smem_bytes(int warps) {
  const size_t ring = (size_t)warps * A2_STAGES * A2_STAGE_BYTES;
  const size_t merge = ((size_t)warps * 16 * (2 + 128) + (size_t)warps * 16 + 2 * 16) * sizeof(float);
  return (ring > merge ? ring : merge) + 1024;  // + alignment of the rings to the 1024-byte swizzle atom
}

__device__ unsigned g_attn_timeouts = 0;

__device__ __forceinline__ void movmatrix_trans(uint32_t& d, uint32_t s) {
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(s));
}

// byte offset of 16-byte chunk c (0-7) of row r inside a 128-byte-swizzled box
__device__ __forceinline__ uint32_t a2_swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// One work item (same contract as am_item). `ring` is this warp's ring, `bars` its stage
// barriers, `seq` the number of tiles the warp has taken through the ring so far (stage
// and phase of its next tile), carried from item to item.
template <int NT>
__device__ __forceinline__ void a2_item(const AttnArgs& a, unsigned char* ring, uint64_t* bars, uint32_t& seq,
                                        float* mb, int64_t rh, int64_t tile_lo, int64_t tile_hi, int64_t slot,
                                        int64_t slot0, int nparts) {
  constexpr int D = 128;
  const int W = blockDim.x >> 5;
  const int group = (int)(a.hq / a.hkv);
  const int64_t r = rh / a.hkv;
  const int kvh = (int)(rh - r * a.hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3;
  __shared__ bool is_last;

  const int64_t seq_row = a.row_seq ? a.row_seq[r] : r;
  const int64_t len = a.row_len[r];
  const bool has_new = a.k_new != nullptr;
  const int64_t total = len + (has_new ? 1 : 0);
  const int64_t t_begin = tile_lo * AT_TILE;
  const int64_t t_end = min(total, tile_hi * AT_TILE);
  const int ntile = t_end > t_begin ? (int)((t_end - t_begin + AT_TILE - 1) / AT_TILE) : 0;
  const int nmine = warp < ntile ? (ntile - warp + W - 1) / W : 0;
  const float scale2 = a.scale * 1.4426950408889634f;  // exp(x s) = exp2(x s log2(e))
  const uint32_t seq0 = seq;

  // page numbers of this warp's tiles [base, base + 32): lane i holds tile base + i's
  int tbl = 0;
  auto load_tbl = [&](int base) {
    const int j = base + lane;
    tbl = 0;
    if (j < nmine) {
      const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
      if (t0 < len) tbl = a.block_table[seq_row * a.bt_stride + t0 / a.page_size];
    }
  };
  load_tbl(0);
  // request tile j of this item (whole warp; lane 0 issues)
  auto issue = [&](int j) {
    if (j >= nmine) return;
    if ((j & (A2_TBL - 1)) == 0 && j) load_tbl(j);
    const int page = __shfl_sync(0xffffffffu, tbl, j & (A2_TBL - 1));
    if (lane == 0) {
      const uint32_t u = seq0 + (uint32_t)j;
      unsigned char* st = ring + (u % A2_STAGES) * A2_STAGE_BYTES;
      uint64_t* bar = bars + (u % A2_STAGES);
      const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
      if (t0 < len) {
        const int y = (int)(((int64_t)page * a.hkv + kvh) * a.page_size + (t0 % a.page_size));
        fence_proxy_async_smem();  // this lane's earlier generic writes to the stage come first
        mbar_arrive_expect_tx(bar, A2_STAGE_BYTES);
        tma_load_2d(st, &a.kmap, 0, y, bar);
        tma_load_2d(st + A2_BOX, &a.kmap, 64, y, bar);
        tma_load_2d(st + 2 * A2_BOX, &a.vmap, 0, y, bar);
        tma_load_2d(st + 3 * A2_BOX, &a.vmap, 64, y, bar);
      } else {
        mbar_arrive(bar);  // the tile holds only the provisional token: nothing to fetch
      }
    }
  };
#pragma unroll
  for (int j = 0; j < A2_STAGES - 1; ++j) issue(j);

  // the group's queries as the B operand: head nt*8 + gq, dims ks*16 + 2cq (+1) and + 8
  uint32_t qb[NT][D / 16][2];
  {
    const __nv_bfloat16* q0 = a.q + (r * a.hq + (int64_t)kvh * group) * D;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int h = nt * 8 + gq;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int d0 = ks * 16 + 2 * cq;
        qb[nt][ks][0] = h < group ? *reinterpret_cast<const uint32_t*>(q0 + h * D + d0) : 0u;
        qb[nt][ks][1] = h < group ? *reinterpret_cast<const uint32_t*>(q0 + h * D + d0 + 8) : 0u;
      }
    }
  }
  // O^T accumulators: dims mt*16 + gq (+8) x heads nt*8 + 2cq (+1)
  float o[D / 16][NT][4];
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
  float mrow[NT][2], lrow[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) mrow[nt][0] = mrow[nt][1] = -INFINITY, lrow[nt][0] = lrow[nt][1] = 0.f;

  const int mi = lane >> 3, rr = lane & 7;
  for (int j = 0; j < nmine; ++j) {
    const uint32_t u = seq0 + (uint32_t)j;
    unsigned char* st = ring + (u % A2_STAGES) * A2_STAGE_BYTES;
    if (!mbar_wait_bounded(bars + (u % A2_STAGES), (u / A2_STAGES) & 1u) && lane == 0) atomicAdd(&g_attn_timeouts, 1u);
    __syncwarp();
    issue(j + A2_STAGES - 1);  // into the stage the previous tile used
    const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
    const int lim = (int)min((int64_t)AT_TILE, t_end - t0);  // tokens of this tile inside the item
    // the provisional token (not in the pool) and zeroed V rows past the item's end, so that
    // stale rows never meet a zero probability as 0 * inf
    bool patched = false;
    if (has_new && len >= t0 && len < t0 + AT_TILE) {
      const int row = (int)(len - t0), ch = lane & 15;
      const __nv_bfloat16* src = (lane < 16 ? a.k_new : a.v_new) + (r * a.hkv + kvh) * D + ch * 8;
      unsigned char* box = st + (lane < 16 ? 0 : 2 * A2_BOX) + (ch >> 3) * A2_BOX;
      *reinterpret_cast<uint4*>(box + a2_swz(row, ch & 7)) = *reinterpret_cast<const uint4*>(src);
      patched = true;
    }
    if (lim < AT_TILE) {
      for (int e = lane; e < (AT_TILE - lim) * 16; e += 32) {
        const int row = lim + (e >> 4), ch = e & 15;
        *reinterpret_cast<uint4*>(st + 2 * A2_BOX + (ch >> 3) * A2_BOX + a2_swz(row, ch & 7)) = make_uint4(0, 0, 0, 0);
      }
      patched = true;
    }
    if (patched) fence_proxy_async_smem();  // before a later TMA overwrites the stage
    __syncwarp();

    // ---- S^T = K Q^T: two accumulator chains (even and odd 16-dim steps)
    float sa[NT][4], sb[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
    {
      const int tok = (mi & 1) * 8 + rr;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t ka[4];
        ldmatrix_x4(ka, st + (ks >> 2) * A2_BOX + a2_swz(tok, ((ks & 3) * 2 + (mi >> 1))));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16_16816((ks & 1) ? sb[nt] : sa[nt], ka, qb[nt][ks][0], qb[nt][ks][1]);
      }
    }
    // ---- online softmax per head column (base 2); tokens gq and gq + 8 of heads 2cq, 2cq + 1
    float alpha[NT][2];
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float s[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) s[e] = (gq + (e >> 1) * 8) < lim ? (sa[nt][e] + sb[nt][e]) * scale2 : -INFINITY;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float mx = fmaxf(s[i], s[2 + i]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(mrow[nt][i], mx);
        alpha[nt][i] = (mrow[nt][i] == -INFINITY) ? 0.f : exp2f(mrow[nt][i] - m_new);
        const float p0 = (m_new == -INFINITY) ? 0.f : exp2f(s[i] - m_new);
        const float p1 = (m_new == -INFINITY) ? 0.f : exp2f(s[2 + i] - m_new);
        s[i] = p0;
        s[2 + i] = p1;
        lrow[nt][i] = lrow[nt][i] * alpha[nt][i] + (p0 + p1);  // this lane's tokens only
        mrow[nt][i] = m_new;
      }
      // P^T as the B operand: transpose the two 8x8 (tokens x heads) blocks
      movmatrix_trans(pb[nt][0], pack_bf16x2(s[0], s[1]));
      movmatrix_trans(pb[nt][1], pack_bf16x2(s[2], s[3]));
    }
    bool moved = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) moved |= alpha[nt][0] != 1.f || alpha[nt][1] != 1.f;
    if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          o[mt][nt][0] *= alpha[nt][0];
          o[mt][nt][1] *= alpha[nt][1];
          o[mt][nt][2] *= alpha[nt][0];
          o[mt][nt][3] *= alpha[nt][1];
        }
    }
    // ---- O^T += V^T P^T
    {
      const int tok = (mi >> 1) * 8 + rr;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        uint32_t va[4];
        ldmatrix_x4_trans(va, st + 2 * A2_BOX + (mt >> 2) * A2_BOX + a2_swz(tok, ((mt & 3) * 2 + (mi & 1))));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(o[mt][nt], va, pb[nt][0], pb[nt][1]);
      }
    }
    __syncwarp();  // every lane is done with the stage before it is requested again
  }
  seq = seq0 + (uint32_t)nmine;
  // row sums over the 8 token lanes of each head
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      lrow[nt][i] += __shfl_xor_sync(0xffffffffu, lrow[nt][i], 4);
      lrow[nt][i] += __shfl_xor_sync(0xffffffffu, lrow[nt][i], 8);
      lrow[nt][i] += __shfl_xor_sync(0xffffffffu, lrow[nt][i], 16);
    }
  __syncthreads();  // every warp is done with its ring: the space becomes the merge area

  // ---- merge the W warp states per head in warp order (layout of am_item)
  {
    float* mine = mb + (size_t)warp * 16 * (2 + D);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int h = nt * 8 + 2 * cq + i;
        if (gq == 0) {
          mine[h * (2 + D)] = mrow[nt][i];
          mine[h * (2 + D) + 1] = lrow[nt][i];
        }
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          mine[h * (2 + D) + 2 + mt * 16 + gq] = o[mt][nt][i];
          mine[h * (2 + D) + 2 + mt * 16 + gq + 8] = o[mt][nt][2 + i];
        }
      }
  }
  __syncthreads();
  float* wts = mb + (size_t)W * 16 * (2 + D);  // [W][16]
  float* hstat = wts + (size_t)W * 16;         // [16] max, [16] sum
  if (tid < group) {
    const int h = tid;
    float mx = -INFINITY;
    for (int w = 0; w < W; ++w) mx = fmaxf(mx, mb[((size_t)w * 16 + h) * (2 + D)]);
    float l = 0.f;
    for (int w = 0; w < W; ++w) {
      const float* sw = mb + ((size_t)w * 16 + h) * (2 + D);
      const float wt = (sw[0] == -INFINITY) ? 0.f : exp2f(sw[0] - mx);
      wts[w * 16 + h] = wt;
      l = fmaf(sw[1], wt, l);
    }
    hstat[h] = mx;
    hstat[16 + h] = l;
  }
  __syncthreads();
  float* part_base = nparts > 1 ? a.part + slot * (int64_t)group * (2 + D) : nullptr;
  for (int idx = tid; idx < group * D; idx += blockDim.x) {
    const int h = idx / D, d = idx - h * D;
    const float mx = hstat[h], l = hstat[16 + h];
    float acc = 0.f;
    for (int w = 0; w < W; ++w) acc = fmaf(mb[((size_t)w * 16 + h) * (2 + D) + 2 + d], wts[w * 16 + h], acc);
    if (nparts == 1) {
      a.out[(r * a.hq + (int64_t)kvh * group + h) * D + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
    } else {
      float* pp = part_base + (int64_t)h * (2 + D);
      pp[2 + d] = acc;
      if (d == 0) {
        pp[0] = mx;
        pp[1] = l;
      }
    }
  }
  fence_proxy_async_smem();  // the merge area is written generically; TMA refills it next
  __syncthreads();
  if (nparts == 1) return;
  __threadfence();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&a.counters[rh], 1u);
    is_last = prev == (unsigned)(nparts - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // ---- last of the group's items: warps merge the heads over the partials in slot order
  constexpr int VD = D / 32;
  const int64_t sstride = (int64_t)group * (2 + D);
  for (int h = warp; h < group; h += W) {
    const float* base = a.part + (slot0 * group + h) * (2 + D);
    float mx_all = -INFINITY;
    for (int s0 = lane; s0 < nparts; s0 += 32) mx_all = fmaxf(mx_all, __ldcg(base + s0 * sstride));
    mx_all = warp_max(mx_all);
    float lsum = 0.f, ov[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) ov[i] = 0.f;
    for (int s0 = 0; s0 < nparts; s0 += 8) {
      float ms[8], ls[8], av[8][VD];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const bool ok = s0 + jj < nparts;
        const float* pp = base + (s0 + jj) * sstride;
        ms[jj] = ok ? __ldcg(pp) : -INFINITY;
        ls[jj] = ok ? __ldcg(pp + 1) : 0.f;
#pragma unroll
        for (int i = 0; i < VD; ++i) av[jj][i] = ok ? __ldcg(pp + 2 + lane * VD + i) : 0.f;
      }
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const float wt = (ms[jj] == -INFINITY) ? 0.f : exp2f(ms[jj] - mx_all);
        lsum = fmaf(ls[jj], wt, lsum);
#pragma unroll
        for (int i = 0; i < VD; ++i) ov[i] = fmaf(av[jj][i], wt, ov[i]);
      }
    }
    __nv_bfloat16* out = a.out + (r * a.hq + (int64_t)kvh * group + h) * D + lane * VD;
#pragma unroll
    for (int i = 0; i < VD; ++i) out[i] = __float2bfloat16_rn(lsum > 0.f ? ov[i] / lsum : 0.f);
  }
  __syncthreads();
  if (tid == 0) a.counters[rh] = 0u;  // ready for the next launch (graph replays)
}

template <bool BALANCED, int NT>
__global__ void __launch_bounds__(AM_MAX_WARPS * 32, AT_MMA_CTAS_PER_SM)
    paged_attention_tma_kernel(const __grid_constant__ AttnArgs a) {
  __shared__ __align__(8) uint64_t bars[AM_MAX_WARPS * A2_STAGES];
  extern __shared__ __align__(16) unsigned char am_smem[];
  const int warp = threadIdx.x >> 5;
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(am_smem) + 1023) & ~uintptr_t(1023));
  if (threadIdx.x == 0)
    for (int i = 0; i < AM_MAX_WARPS * A2_STAGES; ++i) mbar_init(&bars[i], 1);
  fence_proxy_async_smem();
  pdl_launch_dependents();
  pdl_wait();
  __syncthreads();
  unsigned char* ring = base + (size_t)warp * A2_STAGES * A2_STAGE_BYTES;
  uint32_t seq = 0;
  attn_schedule<BALANCED>(a, [&](int64_t rh, int64_t lo, int64_t hi, int64_t slot, int64_t slot0, int nparts) {
    a2_item<NT>(a, ring, bars + warp * A2_STAGES, seq, reinterpret_cast<float*>(base), rh, lo, hi, slot, slot0,
                nparts);
  });
  // every requested tile was waited for; after a timed-out wait, wait (bounded) once more for
  // the last tile of each stage so that no copy is still landing when the CTA exits
  for (uint32_t u = seq >= A2_STAGES ? seq - A2_STAGES : 0; u < seq; ++u)
    mbar_wait_bounded(bars + warp * A2_STAGES + (u % A2_STAGES), (u / A2_STAGES) & 1u);
}

// ---- warp-granular schedule of the TMA kernel
//
// The groups' tiles, laid end to end (group-major, as attn_schedule lays them), are cut into
// one contiguous range per warp: warp w of NW = min(warps launched, T) takes tiles
// [w*T/NW, (w+1)*T/NW). A warp walks its range with one ring that runs on across group
// boundaries (no block barrier, no pipeline restart), keeps one online-softmax state per
// group segment, and at a segment's end either writes the output (the group lies inside its
// range) or publishes the partial in slot w + rh (the staircase argument of attn_schedule,
// per warp). paged_attention_merge_kernel then merges each cut group's partials in warp
// order (deterministic). Measured reason: per-CTA items paid a block-wide merge, a fence and
// an atomic per item and restarted the ring at every item; their slowest CTAs set the time.

// Tiles before each row (all kv heads) in pre[0..rows]; returns T. Whole CTA; ends synced.
__device__ __forceinline__ int64_t attn_row_prefix(const AttnArgs& a, int* pre) {
  const int R = (int)a.rows, hkv = (int)a.hkv;
  const int tid = threadIdx.x, lane = tid & 31;
  for (int r = tid; r < R; r += blockDim.x) pre[r + 1] = am_row_tiles(a, r) * hkv;
  if (tid == 0) pre[0] = 0;
  __syncthreads();
  if (tid < 32) {
    int carry = 0;
    for (int b = 1; b <= R; b += 32) {
      int v = b + lane <= R ? pre[b + lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      if (b + lane <= R) pre[b + lane] = v + carry;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
  __syncthreads();
  return pre[R];
}

// the largest r with pre[r] <= x (pre[0] = 0 <= x < pre[R])
__device__ __forceinline__ int attn_row_of(const int* pre, int R, int64_t x) {
  int lo = 0, hi = R;
  while (hi - lo > 1) {
    const int m = (lo + hi) >> 1;
    if (pre[m] <= x) lo = m; else hi = m;
  }
  return lo;
}

// Position in the flattened tile order: row r, kv head kvh, tile toff of the group; tr =
// tiles per group of row r; rowstart = tiles before row r. Advancing moves to the next tile.
struct AttnCursor {
  int r, kvh, toff, tr;
  int64_t rowstart;
  __device__ __forceinline__ void seek(const AttnArgs& a, const int* pre, int64_t x) {
    r = attn_row_of(pre, (int)a.rows, x);
    rowstart = pre[r];
    tr = (pre[r + 1] - pre[r]) / (int)a.hkv;
    kvh = (int)((x - rowstart) / tr);
    toff = (int)(x - rowstart - (int64_t)kvh * tr);
  }
  __device__ __forceinline__ void next(const AttnArgs& a, bool more) {
    if (++toff < tr) return;
    toff = 0;
    if (++kvh < (int)a.hkv) return;
    kvh = 0;
    rowstart += (int64_t)a.hkv * tr;
    ++r;
    if (more) tr = am_row_tiles(a, r);
  }
};

template <int NT>
__global__ void __launch_bounds__(AM_MAX_WARPS * 32, AT_MMA_CTAS_PER_SM)
    paged_attention_tma_warp_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int D = 128;
  __shared__ __align__(8) uint64_t bars[AM_MAX_WARPS * A2_STAGES];
  extern __shared__ __align__(16) unsigned char am_smem[];
  const int W = blockDim.x >> 5;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, cq = lane & 3, mi = lane >> 3, rr = lane & 7;
  const int group = (int)(a.hq / a.hkv);
  unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(am_smem) + 1023) & ~uintptr_t(1023));
  if (tid == 0)
    for (int i = 0; i < AM_MAX_WARPS * A2_STAGES; ++i) mbar_init(&bars[i], 1);
  fence_proxy_async_smem();
  pdl_launch_dependents();
  pdl_wait();
  int* pre = reinterpret_cast<int*>(am_smem);  // the rows' tile prefix, until the rings start
  const int64_t T = attn_row_prefix(a, pre);
  const int64_t NW = min((int64_t)gridDim.x * W, T);
  const int64_t gw = (int64_t)blockIdx.x * W + warp;
  const int64_t lo = gw < NW ? gw * T / NW : 0, hi = gw < NW ? (gw + 1) * T / NW : 0;
  AttnCursor ci, cc;  // issue and consume positions
  if (gw < NW) {
    ci.seek(a, pre, lo);
    cc = ci;
  }
  __syncthreads();  // the prefix is read: the space becomes the rings
  if (gw >= NW) return;
  const int n = (int)(hi - lo);
  unsigned char* ring = base + (size_t)warp * A2_STAGES * A2_STAGE_BYTES;
  uint64_t* wbars = bars + warp * A2_STAGES;
  const bool has_new = a.k_new != nullptr;
  const float scale2 = a.scale * 1.4426950408889634f;  // exp(x s) = exp2(x s log2(e))

  // ---- issue side: page numbers of 32 consecutive tiles of one row, one per lane
  int tbl = 0, tbl_row = -1, tbl_base = 0;
  int64_t len_i = 0, seq_i = 0;
  int len_row = -1;
  auto issue = [&](int k) {  // the k-th tile of the range (whole warp; lane 0 requests)
    if (k >= n) return;
    if (len_row != ci.r) {
      len_row = ci.r;
      len_i = a.row_len[ci.r];
      seq_i = a.row_seq ? a.row_seq[ci.r] : ci.r;
    }
    if (tbl_row != ci.r || ci.toff < tbl_base || ci.toff >= tbl_base + A2_TBL) {
      tbl_row = ci.r;
      tbl_base = ci.toff;
      const int64_t t0 = (int64_t)(tbl_base + lane) * AT_TILE;
      tbl = t0 < len_i ? a.block_table[seq_i * a.bt_stride + t0 / a.page_size] : 0;
    }
    const int page = __shfl_sync(0xffffffffu, tbl, ci.toff - tbl_base);
    if (lane == 0) {
      unsigned char* st = ring + (k % A2_STAGES) * A2_STAGE_BYTES;
      uint64_t* bar = wbars + (k % A2_STAGES);
      const int64_t t0 = (int64_t)ci.toff * AT_TILE;
      if (t0 < len_i) {
        const int y = (int)(((int64_t)page * a.hkv + ci.kvh) * a.page_size + (t0 % a.page_size));
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, A2_STAGE_BYTES);
        tma_load_2d(st, &a.kmap, 0, y, bar);
        tma_load_2d(st + A2_BOX, &a.kmap, 64, y, bar);
        tma_load_2d(st + 2 * A2_BOX, &a.vmap, 0, y, bar);
        tma_load_2d(st + 3 * A2_BOX, &a.vmap, 64, y, bar);
      } else {
        mbar_arrive(bar);
      }
    }
    ci.next(a, k + 1 < n);
  };
#pragma unroll
  for (int k = 0; k < A2_STAGES - 1; ++k) issue(k);

  // ---- consume side: one online-softmax state per group segment
  uint32_t qb[NT][D / 16][2];
  float o[D / 16][NT][4];
  float mrow[NT][2], lrow[NT][2];
  int64_t len_c = 0;
  int seg_toff0 = 0;
  unsigned* meta = a.meta;  // per group: (first partial slot << 16) | partials, for the merge
  for (int k = 0; k < n; ++k) {
    const bool seg_start = k == 0 || cc.toff == 0;
    if (seg_start) {  // a new group: its queries and row length, state reset
      seg_toff0 = cc.toff;
      len_c = a.row_len[cc.r];
      const __nv_bfloat16* q0 = a.q + ((int64_t)cc.r * a.hq + (int64_t)cc.kvh * group) * D;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int h = nt * 8 + gq;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int d0 = ks * 16 + 2 * cq;
          qb[nt][ks][0] = h < group ? *reinterpret_cast<const uint32_t*>(q0 + h * D + d0) : 0u;
          qb[nt][ks][1] = h < group ? *reinterpret_cast<const uint32_t*>(q0 + h * D + d0 + 8) : 0u;
        }
        mrow[nt][0] = mrow[nt][1] = -INFINITY;
        lrow[nt][0] = lrow[nt][1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.f;
      }
    }
    unsigned char* st = ring + (k % A2_STAGES) * A2_STAGE_BYTES;
    if (!mbar_wait_bounded(wbars + (k % A2_STAGES), ((uint32_t)k / A2_STAGES) & 1u) && lane == 0)
      atomicAdd(&g_attn_timeouts, 1u);
    __syncwarp();
    issue(k + A2_STAGES - 1);
    const int64_t total = len_c + (has_new ? 1 : 0);
    const int64_t t0 = (int64_t)cc.toff * AT_TILE;
    const int lim = (int)min((int64_t)AT_TILE, total - t0);
    bool patched = false;
    if (has_new && len_c >= t0 && len_c < t0 + AT_TILE) {
      const int row = (int)(len_c - t0), ch = lane & 15;
      const __nv_bfloat16* src = (lane < 16 ? a.k_new : a.v_new) + ((int64_t)cc.r * a.hkv + cc.kvh) * D + ch * 8;
      unsigned char* box = st + (lane < 16 ? 0 : 2 * A2_BOX) + (ch >> 3) * A2_BOX;
      *reinterpret_cast<uint4*>(box + a2_swz(row, ch & 7)) = *reinterpret_cast<const uint4*>(src);
      patched = true;
    }
    if (lim < AT_TILE) {
      for (int e = lane; e < (AT_TILE - lim) * 16; e += 32) {
        const int row = lim + (e >> 4), ch = e & 15;
        *reinterpret_cast<uint4*>(st + 2 * A2_BOX + (ch >> 3) * A2_BOX + a2_swz(row, ch & 7)) = make_uint4(0, 0, 0, 0);
      }
      patched = true;
    }
    if (patched) fence_proxy_async_smem();
    __syncwarp();
    // ---- S^T = K Q^T
    float sa[NT][4], sb[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
    {
      const int tok = (mi & 1) * 8 + rr;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t ka[4];
        ldmatrix_x4(ka, st + (ks >> 2) * A2_BOX + a2_swz(tok, ((ks & 3) * 2 + (mi >> 1))));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16_16816((ks & 1) ? sb[nt] : sa[nt], ka, qb[nt][ks][0], qb[nt][ks][1]);
      }
    }
    // ---- online softmax per head column (base 2)
    float alpha[NT][2];
    uint32_t pb[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float sv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) sv[e] = (gq + (e >> 1) * 8) < lim ? (sa[nt][e] + sb[nt][e]) * scale2 : -INFINITY;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float mx = fmaxf(sv[i], sv[2 + i]);
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(mrow[nt][i], mx);
        alpha[nt][i] = (mrow[nt][i] == -INFINITY) ? 0.f : exp2f(mrow[nt][i] - m_new);
        const float p0 = (m_new == -INFINITY) ? 0.f : exp2f(sv[i] - m_new);
        const float p1 = (m_new == -INFINITY) ? 0.f : exp2f(sv[2 + i] - m_new);
        sv[i] = p0;
        sv[2 + i] = p1;
        lrow[nt][i] = lrow[nt][i] * alpha[nt][i] + (p0 + p1);
        mrow[nt][i] = m_new;
      }
      movmatrix_trans(pb[nt][0], pack_bf16x2(sv[0], sv[1]));
      movmatrix_trans(pb[nt][1], pack_bf16x2(sv[2], sv[3]));
    }
    bool moved = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) moved |= alpha[nt][0] != 1.f || alpha[nt][1] != 1.f;
    if (__any_sync(0xffffffffu, moved)) {
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          o[mt][nt][0] *= alpha[nt][0];
          o[mt][nt][1] *= alpha[nt][1];
          o[mt][nt][2] *= alpha[nt][0];
          o[mt][nt][3] *= alpha[nt][1];
        }
    }
    // ---- O^T += V^T P^T
    {
      const int tok = (mi >> 1) * 8 + rr;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        uint32_t va[4];
        ldmatrix_x4_trans(va, st + 2 * A2_BOX + (mt >> 2) * A2_BOX + a2_swz(tok, ((mt & 3) * 2 + (mi & 1))));
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_bf16_16816(o[mt][nt], va, pb[nt][0], pb[nt][1]);
      }
    }
    __syncwarp();
    // ---- segment end: the output, or this warp's partial of the group
    if (cc.toff + 1 == cc.tr || k + 1 == n) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          lrow[nt][i] += __shfl_xor_sync(0xffffffffu, lrow[nt][i], 4);
          lrow[nt][i] += __shfl_xor_sync(0xffffffffu, lrow[nt][i], 8);
          lrow[nt][i] += __shfl_xor_sync(0xffffffffu, lrow[nt][i], 16);
        }
      const int64_t rh = (int64_t)cc.r * a.hkv + cc.kvh;
      const int64_t gstart = cc.rowstart + (int64_t)cc.kvh * cc.tr;
      const int64_t wf = ((gstart + 1) * NW - 1) / T, wl = ((gstart + cc.tr) * NW - 1) / T;
      if (seg_toff0 == 0 && lane == 0) meta[rh] = (unsigned)((wf + rh) << 16) | (unsigned)(wl - wf + 1);
      if (wf == wl) {
        __nv_bfloat16* out = a.out + ((int64_t)cc.r * a.hq + (int64_t)cc.kvh * group) * D;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int h = nt * 8 + 2 * cq + i;
            if (h >= group) continue;
            const float inv = lrow[nt][i] > 0.f ? 1.f / lrow[nt][i] : 0.f;
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
              out[h * D + mt * 16 + gq] = __float2bfloat16_rn(o[mt][nt][i] * inv);
              out[h * D + mt * 16 + gq + 8] = __float2bfloat16_rn(o[mt][nt][2 + i] * inv);
            }
          }
      } else {
        float* part = a.part + (gw + rh) * (int64_t)group * (2 + D);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int h = nt * 8 + 2 * cq + i;
            if (h >= group) continue;
            float* ph = part + (int64_t)h * (2 + D);
            if (gq == 0) {
              ph[0] = mrow[nt][i];
              ph[1] = lrow[nt][i];
            }
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
              ph[2 + mt * 16 + gq] = o[mt][nt][i];
              ph[2 + mt * 16 + gq + 8] = o[mt][nt][2 + i];
            }
          }
      }
    }
    cc.next(a, k + 1 < n);
  }
  // every requested tile was waited for; after a timed-out wait, wait (bounded) once more for
  // the last tile of each stage so that no copy is still landing when the warp exits
  for (int k = n > A2_STAGES ? n - A2_STAGES : 0; k < n; ++k)
    mbar_wait_bounded(wbars + (k % A2_STAGES), ((uint32_t)k / A2_STAGES) & 1u);
}

// The merge after paged_attention_tma_warp_kernel: CTA rh (one warp per query head) merges
// the partials of group rh in slot order when the attention kernel cut the group (its
// per-group record says where they are); whole groups were written by their warp. Up to 16
// partials' loads are in flight at once, folded into a running maximum and sum.
__global__ void __launch_bounds__(AT_MAX_GROUP * 32) paged_attention_merge_kernel(const __grid_constant__ AttnArgs a) {
  constexpr int D = 128, VD = D / 32, CH = 16;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t rh = blockIdx.x;
  const unsigned meta = a.meta[rh];
  const int nparts = (int)(meta & 0xffffu);
  if (nparts <= 1) return;
  const int64_t slot0 = meta >> 16;
  const int group = (int)(a.hq / a.hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = rh / a.hkv, kvh = rh - r * a.hkv;
  const int64_t sstride = (int64_t)group * (2 + D);
  for (int h = warp; h < group; h += blockDim.x >> 5) {
    const float* base = a.part + (slot0 * group + h) * (2 + D);
    float M = -INFINITY, L = 0.f, acc[VD];
#pragma unroll
    for (int i = 0; i < VD; ++i) acc[i] = 0.f;
    for (int s0 = 0; s0 < nparts; s0 += CH) {
      float ms[CH], ls[CH];
      float2 av[CH][VD / 2];
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const bool ok = s0 + j < nparts;
        const float* pp = base + (int64_t)(s0 + j) * sstride;
        const float2 st = ok ? *reinterpret_cast<const float2*>(pp) : make_float2(-INFINITY, 0.f);
        ms[j] = st.x;
        ls[j] = st.y;
#pragma unroll
        for (int i = 0; i < VD / 2; ++i)
          av[j][i] = ok ? *reinterpret_cast<const float2*>(pp + 2 + lane * VD + 2 * i) : make_float2(0.f, 0.f);
      }
      float cm = M;
#pragma unroll
      for (int j = 0; j < CH; ++j) cm = fmaxf(cm, ms[j]);
      if (cm != M && M != -INFINITY) {  // rescale what was folded under the old maximum
        const float f = exp2f(M - cm);
        L *= f;
#pragma unroll
        for (int i = 0; i < VD; ++i) acc[i] *= f;
      }
      M = cm;
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const float wt = (ms[j] == -INFINITY) ? 0.f : exp2f(ms[j] - M);
        L = fmaf(ls[j], wt, L);
#pragma unroll
        for (int i = 0; i < VD / 2; ++i) {
          acc[2 * i] = fmaf(av[j][i].x, wt, acc[2 * i]);
          acc[2 * i + 1] = fmaf(av[j][i].y, wt, acc[2 * i + 1]);
        }
      }
    }
    __nv_bfloat16* out = a.out + (r * a.hq + kvh * group + h) * D + lane * VD;
#pragma unroll
    for (int i = 0; i < VD; ++i) out[i] = __float2bfloat16_rn(L > 0.f ? acc[i] / L : 0.f);
  }
}

// The fused decode step (rope_append_attention_kernel's prologue and cluster merge) around
// the tensor-core tile loop of paged_attention_mma_kernel, for head_dim 128: W warps per CTA
// take the CTA's 16-token tiles in turn (one block-table lookup per tile -- the page size is
// a multiple of 16), compute S = Q K^T for all query heads of the group with heads as the mma
// rows, and accumulate O += P V; the warp owning the new token's tile writes its rotated K
// and V into the staged tile. The W warp states merge in shared memory in warp order, then
// the cluster's CTA states through distributed shared memory in rank order (deterministic).
__global__ void __launch_bounds__(AM_MAX_WARPS * 32) rope_append_attention_mma_kernel(FusedArgs a) {
  constexpr int D = 128, HALF = D / 2, CH = D / 8;
  const int W = blockDim.x >> 5;
  const int group = (int)(a.hq / a.hkv);
  const int S = (int)gridDim.x;      // the cluster spans grid x
  const int rank = (int)blockIdx.x;  // = %cluster_ctarank
  const int64_t rh = blockIdx.y;     // row * hkv + kv head
  const int64_t r = rh / a.hkv;
  const int kvh = (int)(rh - r * a.hkv);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;

  extern __shared__ __align__(16) unsigned char am_smem[];
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(am_smem) + (size_t)warp * AM_STAGES * AM_STAGE_ELEMS;
  __shared__ __align__(16) __nv_bfloat16 qs[AT_MAX_GROUP][D];
  __shared__ __align__(16) __nv_bfloat16 knew[D];
  __shared__ __align__(16) __nv_bfloat16 vnew[D];
  __shared__ __align__(16) float pacc[AT_MAX_GROUP][D];
  __shared__ __align__(8) float pstat[AT_MAX_GROUP][2];

  pdl_launch_dependents();
  // With state_ready the step state and the cached K/V are not written by any kernel that may
  // still run, so their reads (and the K/V tile loads) overlap the previous kernel; only the
  // new token's q/k/v rows wait for it.
  if (!a.state_ready) pdl_wait();

  // ---- the row's new position and its cache slot (every CTA of the cluster agrees)
  const int64_t seq = a.row_seq ? a.row_seq[r] : r;
  const int64_t pos = a.positions[r];
  bool ok = pos >= 0 && (a.cos_tab == nullptr || pos < a.rope_len);
  int64_t new_off = 0;
  if (ok) {
    const int64_t lp = pos / a.page_size;
    const int64_t page = a.block_table[seq * a.bt_stride + lp];
    ok = page >= 0 && page < a.num_pages;
    new_off = page * a.stride_page + (int64_t)kvh * a.stride_head + (pos - lp * a.page_size) * a.stride_tok;
  }
  __nv_bfloat16* out_base = a.out + (r * a.hq + (int64_t)kvh * group) * D;
  if (!ok) {  // cluster-uniform: no CTA reaches a cluster barrier
    if (a.state_ready) pdl_wait();  // the output may still be read by an earlier kernel
    if (rank == 0) {
      if (tid == 0 && a.error_flag) atomicExch(a.error_flag, 1);
      for (int e = tid; e < group * D; e += blockDim.x) out_base[e] = __float2bfloat16_rn(0.f);
    }
    return;
  }

  // ---- this CTA's share of the row's tiles; warp w takes tiles w, w + W, ...
  const int64_t total = pos + 1;
  const int64_t tiles = (total + AT_TILE - 1) / AT_TILE;
  const int64_t per = (tiles + S - 1) / S;
  const int64_t tb = min(tiles, (int64_t)rank * per), te = min(tiles, tb + per);
  const int ntile = (int)(te - tb);
  const int64_t t_begin = tb * AT_TILE, t_end = min(total, te * AT_TILE);
  const bool owns_new = pos >= t_begin && pos < t_end;
  const int nmine = warp < ntile ? (ntile - warp + W - 1) / W : 0;
  const int64_t khead = (int64_t)kvh * a.stride_head;
  bool bad_page = false;

  auto issue = [&](int j) {
    if (j < nmine) {
      __nv_bfloat16* kst = ring + (j % AM_STAGES) * AM_STAGE_ELEMS;
      __nv_bfloat16* vst = kst + AM_TILE_ELEMS;
      const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
      const int64_t lp = t0 / a.page_size;
      const int64_t page = a.block_table[seq * a.bt_stride + lp];
      const bool page_ok = page >= 0 && page < a.num_pages;
      bad_page |= !page_ok;
      const int64_t base = page_ok ? page * a.stride_page + khead + (t0 - lp * a.page_size) * a.stride_tok : 0;
      const int lim = (int)(t_end - t0), newt = (int)(pos - t0);  // the new token is staged below
#pragma unroll
      for (int i = 0; i < AT_TILE * CH / 32; ++i) {
        const int e = lane + 32 * i;
        const int t = e >> 4, ch = e & 15;
        const bool ld = page_ok && t < lim && t != newt;
        const int64_t off = ld ? base + (int64_t)t * a.stride_tok + ch * 8 : 0;
        cp_async16_zfill(kst + t * AM_ROW + ch * 8, a.k_cache + off, ld);
        cp_async16_zfill(vst + t * AM_ROW + ch * 8, a.v_cache + off, ld);
      }
    }
    cp_async_commit_group();
  };
#pragma unroll
  for (int j = 0; j < AM_STAGES - 1; ++j) issue(j);
  if (a.state_ready) pdl_wait();

  // ---- RoPE of the group's query heads into shared memory (and of the new key / value in
  // the CTA whose range holds the new position)
  const float* cr = a.cos_tab ? a.cos_tab + pos * HALF : nullptr;
  const float* sr = a.sin_tab ? a.sin_tab + pos * HALF : nullptr;
  const __nv_bfloat16* qrow = a.q_in + r * a.in_stride + (int64_t)kvh * group * D;
  for (int h = warp; h < group; h += W) rope_head(qrow + (int64_t)h * D, &qs[h][0], HALF, cr, sr, lane, a.q_norm, a.norm_eps);
  if (owns_new) {
    if (warp == 0)
      rope_head(a.k_in + r * a.in_stride + (int64_t)kvh * D, knew, HALF, cr, sr, lane, a.k_norm, a.norm_eps);
    if (warp == (W > 1 ? 1 : 0))
      rope_head(a.v_in + r * a.in_stride + (int64_t)kvh * D, vnew, HALF, nullptr, nullptr, lane);
  }
  __syncthreads();
  if (owns_new && tid < 2 * CH) {  // commit the new row to the cache (this CTA alone touches slot pos)
    if (tid < CH)
      reinterpret_cast<uint4*>(a.k_cache + new_off)[tid] = reinterpret_cast<const uint4*>(knew)[tid];
    else
      reinterpret_cast<uint4*>(a.v_cache + new_off)[tid - CH] = reinterpret_cast<const uint4*>(vnew)[tid - CH];
  }

  // ---- Q of the group as the mma A operand (rows g and g + 8 are query heads, zero beyond)
  const bool two_halves = group > 8;
  uint32_t qa[D / 16][4];
  {
    const bool v0 = g < group, v1 = g + 8 < group;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d0 = ks * 16 + 2 * c;
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(&qs[g][d0]) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(&qs[g + 8][d0]) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(&qs[g][d0 + 8]) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(&qs[g + 8][d0 + 8]) : 0u;
    }
  }
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  for (int j = 0; j < nmine; ++j) {
    cp_async_wait_group<AM_STAGES - 2>();
    __syncwarp();  // the whole tile is in shared memory; the stage of tile j - 1 is free
    issue(j + AM_STAGES - 1);
    __nv_bfloat16* kst = ring + (j % AM_STAGES) * AM_STAGE_ELEMS;
    __nv_bfloat16* vst = kst + AM_TILE_ELEMS;
    const int64_t t0 = t_begin + (int64_t)(warp + j * W) * AT_TILE;
    const int64_t newt = pos - t0;
    if (newt >= 0 && newt < AT_TILE) {  // warp-uniform: stage the new token's K and V row
      if (lane < CH)
        reinterpret_cast<uint4*>(kst + newt * AM_ROW)[lane] = reinterpret_cast<const uint4*>(knew)[lane];
      else
        reinterpret_cast<uint4*>(vst + newt * AM_ROW)[lane - CH] = reinterpret_cast<const uint4*>(vnew)[lane - CH];
      __syncwarp();
    }
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      const __nv_bfloat16* kr = kst + (nt * 8 + (lane & 7)) * AM_ROW + (lane >> 3) * 8;
#pragma unroll
      for (int ks = 0; ks < D / 16; ks += 2) {
        uint32_t kb[4];
        ldmatrix_x4(kb, kr + ks * 16);
        mma_bf16_16816(s[nt], qa[ks], kb[0], kb[1]);
        mma_bf16_16816(s[nt], qa[ks + 1], kb[2], kb[3]);
      }
    }
    const int lim = (int)(t_end - t0);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) s[nt][i] = nt * 8 + 2 * c + (i & 1) < lim ? s[nt][i] * a.scale : -INFINITY;
    float alpha[2] = {1.f, 1.f};
    if (!two_halves) s[0][2] = s[0][3] = s[1][2] = s[1][3] = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h == 1 && !two_halves) break;
      float mx = fmaxf(fmaxf(s[0][2 * h], s[0][2 * h + 1]), fmaxf(s[1][2 * h], s[1][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(mrow[h], mx);
      alpha[h] = (mrow[h] == -INFINITY) ? 0.f : expf(mrow[h] - m_new);
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float p = (m_new == -INFINITY) ? 0.f : expf(s[nt][2 * h + i] - m_new);
          s[nt][2 * h + i] = p;
          sum += p;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow[h] = lrow[h] * alpha[h] + sum;
      mrow[h] = m_new;
    }
    const uint32_t pa[4] = {pack_bf16x2(s[0][0], s[0][1]), pack_bf16x2(s[0][2], s[0][3]),
                            pack_bf16x2(s[1][0], s[1][1]), pack_bf16x2(s[1][2], s[1][3])};
    const __nv_bfloat16* vrow = vst + (lane & 15) * AM_ROW + (lane >> 4) * 8;
    if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) {
        o[dt][0] *= alpha[0];
        o[dt][1] *= alpha[0];
        o[dt][2] *= alpha[1];
        o[dt][3] *= alpha[1];
      }
    }
#pragma unroll
    for (int dt = 0; dt < D / 8; dt += 2) {
      uint32_t vb[4];
      ldmatrix_x4_trans(vb, vrow + dt * 8);
      mma_bf16_16816(o[dt], pa, vb[0], vb[1]);
      mma_bf16_16816(o[dt + 1], pa, vb[2], vb[3]);
    }
  }
  cp_async_wait_group<0>();
  if (bad_page && a.error_flag) atomicExch(a.error_flag, 1);
  __syncthreads();  // every warp is done with its ring: the space becomes the merge area

  // ---- merge the W warp states per head in warp order
  float* mb = reinterpret_cast<float*>(am_smem);  // [W][16 rows][2 + D]
  {
    float* mine = mb + (size_t)warp * 16 * (2 + D);
    if (c == 0) {
      mine[g * (2 + D)] = mrow[0];
      mine[g * (2 + D) + 1] = lrow[0];
      mine[(g + 8) * (2 + D)] = mrow[1];
      mine[(g + 8) * (2 + D) + 1] = lrow[1];
    }
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      mine[g * (2 + D) + 2 + dt * 8 + 2 * c] = o[dt][0];
      mine[g * (2 + D) + 2 + dt * 8 + 2 * c + 1] = o[dt][1];
      mine[(g + 8) * (2 + D) + 2 + dt * 8 + 2 * c] = o[dt][2];
      mine[(g + 8) * (2 + D) + 2 + dt * 8 + 2 * c + 1] = o[dt][3];
    }
  }
  __syncthreads();
  float* wts = mb + (size_t)W * 16 * (2 + D);  // [W][16]
  if (tid < group) {
    const int h = tid;
    float mx = -INFINITY;
    for (int w = 0; w < W; ++w) mx = fmaxf(mx, mb[((size_t)w * 16 + h) * (2 + D)]);
    float l = 0.f;
    for (int w = 0; w < W; ++w) {
      const float* st = mb + ((size_t)w * 16 + h) * (2 + D);
      const float wt = (st[0] == -INFINITY) ? 0.f : expf(st[0] - mx);
      wts[w * 16 + h] = wt;
      l = fmaf(st[1], wt, l);
    }
    pstat[h][0] = mx;
    pstat[h][1] = l;
  }
  __syncthreads();
  for (int idx = tid; idx < group * D; idx += blockDim.x) {
    const int h = idx / D, d = idx - h * D;
    float acc = 0.f;
    for (int w = 0; w < W; ++w) acc = fmaf(mb[((size_t)w * 16 + h) * (2 + D) + 2 + d], wts[w * 16 + h], acc);
    if (S == 1) {
      const float l = pstat[h][1];
      out_base[idx] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
    } else {
      pacc[h][d] = acc;
    }
  }
  if (S == 1) return;

  // ---- merge the cluster's CTA states per head in rank order
  constexpr int VD = D / 32;
  cluster_sync_all();
  for (int h = rank + S * warp; h < group; h += S * W) {
    float ms = -INFINITY, ls = 0.f;
    if (lane < S) {
      const uint32_t ra = mapa_shared(smem_u32(&pstat[h][0]), (unsigned)lane);
      ms = ld_shared_cluster_f32(ra);
      ls = ld_shared_cluster_f32(ra + 4);
    }
    const float mx = warp_max(ms);
    const float wt = (ms == -INFINITY) ? 0.f : expf(ms - mx);
    const float lsum = warp_sum(ls * wt);
    const uint32_t acc_addr = smem_u32(&pacc[h][lane * VD]);
    float ov[VD] = {0.f, 0.f, 0.f, 0.f};
    for (int s0 = 0; s0 < S; s0 += 8) {
      float4 av[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        av[jj] = s0 + jj < S ? ld_shared_cluster_v4f32(mapa_shared(acc_addr, (unsigned)(s0 + jj)))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const float w = __shfl_sync(0xffffffffu, wt, (s0 + jj) & 31);
        ov[0] = fmaf(av[jj].x, w, ov[0]);
        ov[1] = fmaf(av[jj].y, w, ov[1]);
        ov[2] = fmaf(av[jj].z, w, ov[2]);
        ov[3] = fmaf(av[jj].w, w, ov[3]);
      }
    }
#pragma unroll
    for (int i = 0; i < VD; ++i)
      out_base[h * D + lane * VD + i] = __float2bfloat16_rn(lsum > 0.f ? ov[i] / lsum : 0.f);
  }
  cluster_sync_all();  // peers' shared memory stays alive until every merge has read it
}

// ------------------------------------------------------------------ prefill attention

// Causal attention of a prefill block: n tokens of one sequence at positions start ..
// start + n - 1, already appended to the paged cache, each attending to positions [0, its own].
// Flash-attention on the tensor pipe for head_dim 128: a CTA owns (16-token query block, KV
// head) with one warp per query head of the GQA group; all warps share each 16-token K/V tile,
// staged through a cp.async ring in shared memory (rows padded to 272 B for conflict-free
// fragments), and every warp computes S = Q K^T for its head with the block's 16 tokens as
// the rows of mma.sync m16n8k16 (bf16 in, fp32 out), masks keys past each token's position,
// runs the fp32 online softmax per token row and accumulates O += P V (P rounded to bf16 as
// the A operand, V through ldmatrix.trans). The K/V prefix is read once per (query block,
// KV head) instead of once per token. Deterministic (no atomics, fixed order).
//
// The (query block, KV head) pair is a thread-block cluster of a.cluster CTAs (up to
// PF_MAX_CLUSTER, and only while the pairs still fit one resident wave): rank r takes a
// contiguous share of the block's causal key tiles, so the longest serial walk is
// ceil(tiles / cluster) tiles instead of all of them. Query blocks are laid out last block
// first, so the longest walks start first when the grid takes several waves. Each warp then
// leaves its online-softmax state (running max and sum per token row, the unnormalised O
// fragments) in its CTA's shared memory, and rank 0 merges the ranks' states in rank order
// through distributed shared memory and writes the output.
constexpr int PF_MAX_CLUSTER = 2;
constexpr int PF_MERGE_WORDS = 64 + 4;  // per lane: 16 x 4 O fragments, max and sum of rows g, g + 8
constexpr int PF_STAGES = 3;
constexpr int PF_ROW = 128 + 8;                    // padded smem row (bf16)
constexpr int PF_TILE_ELEMS = AT_TILE * PF_ROW;    // one K or V tile
constexpr int PF_STAGE_ELEMS = 2 * PF_TILE_ELEMS;  // K and V
constexpr size_t PF_SMEM = (size_t)PF_STAGES * PF_STAGE_ELEMS * sizeof(__nv_bfloat16);

struct PrefillArgs {
  const __nv_bfloat16* q;  // [n, hq, 128]
  int64_t n, hq, hkv, start;
  const __nv_bfloat16* k_cache;
  const __nv_bfloat16* v_cache;
  int64_t stride_page, stride_head, stride_tok, page_size;
  const int32_t* block_table;  // the sequence's row
  int64_t num_pages;
  int32_t* error_flag;
  float scale;
  __nv_bfloat16* out;  // [n, hq, 128]
  int cluster;         // CTAs per (query block, KV head); gridDim.x = query blocks x cluster
};

__host__ __device__ inline size_t pf_smem_bytes(int group) {
  return PF_SMEM + (size_t)group * 32 * PF_MERGE_WORDS * sizeof(float);
}

__global__ void __launch_bounds__(AT_MAX_GROUP * 32) paged_prefill_attention_kernel(PrefillArgs a) {
  constexpr int D = 128, CH = D / 8;
  const int group = blockDim.x >> 5;
  const int rank = (int)(blockIdx.x % (unsigned)a.cluster);  // = %cluster_ctarank
  const int64_t nblk = (a.n + AT_TILE - 1) / AT_TILE;
  const int64_t q0 = (nblk - 1 - (int64_t)(blockIdx.x / (unsigned)a.cluster)) * AT_TILE;  // first token of the block
  const int kvh = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int head = kvh * group + warp;
  extern __shared__ __align__(16) unsigned char pf_smem[];
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(pf_smem);
  pdl_launch_dependents();
  pdl_wait();

  const int64_t ntok = min((int64_t)AT_TILE, a.n - q0);         // tokens of this block
  const int64_t last_pos = a.start + q0 + ntok - 1;              // the block's highest position
  const int ntile = (int)(last_pos / AT_TILE) + 1;               // key tiles [0, last_pos]
  const int share = (ntile + a.cluster - 1) / a.cluster;         // this rank: tiles [tb, te)
  const int tb = min(ntile, rank * share), te = min(ntile, tb + share);
  const int64_t khead = (int64_t)kvh * a.stride_head;
  bool bad_page = false;

  auto issue = [&](int i) {
    if (i < te) {
      __nv_bfloat16* kst = ring + (i % PF_STAGES) * PF_STAGE_ELEMS;
      __nv_bfloat16* vst = kst + PF_TILE_ELEMS;
      const int64_t t0 = (int64_t)i * AT_TILE;
      const int64_t lp = t0 / a.page_size;
      const int64_t page = a.block_table[lp];
      const bool page_ok = page >= 0 && page < a.num_pages;
      bad_page |= !page_ok;
      const int64_t base = page_ok ? page * a.stride_page + khead + (t0 - lp * a.page_size) * a.stride_tok : 0;
      const int lim = (int)min((int64_t)AT_TILE, last_pos + 1 - t0);
      for (int e = tid; e < AT_TILE * CH; e += blockDim.x) {
        const int t = e / CH, ch = e - t * CH;
        const bool ld = page_ok && t < lim;
        const int64_t off = ld ? base + (int64_t)t * a.stride_tok + ch * 8 : 0;
        cp_async16_zfill(kst + t * PF_ROW + ch * 8, a.k_cache + off, ld);
        cp_async16_zfill(vst + t * PF_ROW + ch * 8, a.v_cache + off, ld);
      }
    }
    cp_async_commit_group();
  };
#pragma unroll
  for (int i = 0; i < PF_STAGES - 1; ++i) issue(tb + i);

  // Q of this warp's head for the block's tokens (rows g and g + 8; zero past the block)
  uint32_t qa[D / 16][4];
  {
    const bool v0 = g < ntok, v1 = g + 8 < ntok;
    const __nv_bfloat16* r0 = a.q + ((q0 + g) * a.hq + head) * D;
    const __nv_bfloat16* r1 = a.q + ((q0 + g + 8) * a.hq + head) * D;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int d0 = ks * 16 + 2 * c;
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(r0 + d0) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(r1 + d0) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(r0 + d0 + 8) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(r1 + d0 + 8) : 0u;
    }
  }
  const int64_t pos_row[2] = {a.start + q0 + g, a.start + q0 + g + 8};  // key limit per row
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};

  for (int i = tb; i < te; ++i) {
    cp_async_wait_group<PF_STAGES - 2>();
    __syncthreads();  // tile i is staged; every warp is done with tile i - 1
    issue(i + PF_STAGES - 1);
    const __nv_bfloat16* kst = ring + (i % PF_STAGES) * PF_STAGE_ELEMS;
    const __nv_bfloat16* vst = kst + PF_TILE_ELEMS;
    const int64_t t0 = (int64_t)i * AT_TILE;
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      const __nv_bfloat16* kr = kst + (nt * 8 + (lane & 7)) * PF_ROW + (lane >> 3) * 8;
#pragma unroll
      for (int ks = 0; ks < D / 16; ks += 2) {
        uint32_t kb[4];
        ldmatrix_x4(kb, kr + ks * 16);
        mma_bf16_16816(s[nt], qa[ks], kb[0], kb[1]);
        mma_bf16_16816(s[nt], qa[ks + 1], kb[2], kb[3]);
      }
    }
    // causal mask: key position <= the row's token position
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int64_t key = t0 + nt * 8 + 2 * c + (e & 1);
        s[nt][e] = key <= pos_row[e >> 1] ? s[nt][e] * a.scale : -INFINITY;
      }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = fmaxf(fmaxf(s[0][2 * h], s[0][2 * h + 1]), fmaxf(s[1][2 * h], s[1][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(mrow[h], mx);
      alpha[h] = (mrow[h] == -INFINITY) ? 0.f : expf(mrow[h] - m_new);
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p = (m_new == -INFINITY) ? 0.f : expf(s[nt][2 * h + e] - m_new);
          s[nt][2 * h + e] = p;
          sum += p;
        }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow[h] = lrow[h] * alpha[h] + sum;
      mrow[h] = m_new;
    }
    const uint32_t pa[4] = {pack_bf16x2(s[0][0], s[0][1]), pack_bf16x2(s[0][2], s[0][3]),
                            pack_bf16x2(s[1][0], s[1][1]), pack_bf16x2(s[1][2], s[1][3])};
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      o[dt][0] *= alpha[0];
      o[dt][1] *= alpha[0];
      o[dt][2] *= alpha[1];
      o[dt][3] *= alpha[1];
    }
    const __nv_bfloat16* vrow = vst + (lane & 15) * PF_ROW + (lane >> 4) * 8;
#pragma unroll
    for (int dt = 0; dt < D / 8; dt += 2) {
      uint32_t vb[4];
      ldmatrix_x4_trans(vb, vrow + dt * 8);
      mma_bf16_16816(o[dt], pa, vb[0], vb[1]);
      mma_bf16_16816(o[dt + 1], pa, vb[2], vb[3]);
    }
  }
  cp_async_wait_group<0>();
  if (bad_page && a.error_flag) atomicExch(a.error_flag, 1);
  if (a.cluster > 1) {
    // this rank's state, lane-major (conflict-free), then rank 0 folds the ranks in order
    float* mine = reinterpret_cast<float*>(pf_smem + PF_SMEM) + (size_t)warp * 32 * PF_MERGE_WORDS;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) mine[(dt * 4 + e) * 32 + lane] = o[dt][e];
    mine[64 * 32 + lane] = mrow[0];
    mine[65 * 32 + lane] = mrow[1];
    mine[66 * 32 + lane] = lrow[0];
    mine[67 * 32 + lane] = lrow[1];
    cluster_sync_all();
    if (rank == 0) {
      const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(mine));
      float M[2] = {-INFINITY, -INFINITY};
      for (int r = 0; r < a.cluster; ++r) {
        const uint32_t ra = mapa_shared(base, (unsigned)r);
        M[0] = fmaxf(M[0], ld_shared_cluster_f32(ra + (64 * 32 + lane) * 4));
        M[1] = fmaxf(M[1], ld_shared_cluster_f32(ra + (65 * 32 + lane) * 4));
      }
      float L[2] = {0.f, 0.f};
#pragma unroll
      for (int dt = 0; dt < D / 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
      for (int r = 0; r < a.cluster; ++r) {
        const uint32_t ra = mapa_shared(base, (unsigned)r);
        float w[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float m_r = ld_shared_cluster_f32(ra + ((64 + h) * 32 + lane) * 4);
          w[h] = m_r == -INFINITY ? 0.f : expf(m_r - M[h]);
          L[h] = fmaf(ld_shared_cluster_f32(ra + ((66 + h) * 32 + lane) * 4), w[h], L[h]);
        }
#pragma unroll
        for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            o[dt][e] = fmaf(ld_shared_cluster_f32(ra + ((dt * 4 + e) * 32 + lane) * 4), w[e >> 1], o[dt][e]);
      }
      lrow[0] = L[0];
      lrow[1] = L[1];
    }
    cluster_sync_all();  // the peers' shared memory stays alive until rank 0 has read it
    if (rank != 0) return;
  }
  // O / l for rows g and g + 8 of the block
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int64_t tok = q0 + g + 8 * h;
    if (tok >= a.n) continue;
    const float inv = lrow[h] > 0.f ? 1.f / lrow[h] : 0.f;
    __nv_bfloat16* dst = a.out + (tok * a.hq + head) * D + 2 * c;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt)
      *reinterpret_cast<__nv_bfloat162*>(dst + dt * 8) =
          __floats2bfloat162_rn(o[dt][2 * h] * inv, o[dt][2 * h + 1] * inv);
  }
}

static bool use_mma(int64_t rows, int64_t hkv, int64_t max_total, int64_t head_dim);

// Launch the decode attention for a checked AttnArgs planned with plan_splits: the TMA
// kernel for the canonical paged pool ([pages, Hkv, page_size, 128], page size a multiple of
// 16) where use_mma selects the tensor pipe, the ldmatrix/cp.async tensor-core kernel for
// other layouts there, else the scalar kernel.
static int launch_attention(AttnArgs a, int64_t head_dim, int64_t max_total, cudaStream_t s) {
  const bool canonical = head_dim == 128 && a.hq / a.hkv <= 16 && a.page_size % AT_TILE == 0 &&
                         a.stride_tok == 128 && a.stride_head == a.page_size * 128 &&
                         a.stride_page == a.hkv * a.page_size * 128;
  if (canonical && use_mma(a.rows, a.hkv, max_total, head_dim)) {
    // the pool as rows of 128 dims; its page count is not passed, so the map spans the
    // largest row index a TMA coordinate can name and the block table bounds the reads (as it
    // does for the copy-based kernels)
    const int64_t rows = 0x7fffffffLL;
    int st = encode_map_2d(&a.kmap, a.k_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, 128, AT_TILE, 64,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (!st)
      st = encode_map_2d(&a.vmap, a.v_cache, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, 128, AT_TILE, 64,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    a.tma = 1;
  }
  dim3 grid((unsigned)(a.rows * a.hkv), (unsigned)a.nsplit);
  if (a.bal_ctas > 0) grid = dim3((unsigned)a.bal_ctas);
  if (a.tma && a.warp_sched && a.bal_ctas > 0) {
    const bool two = a.hq / a.hkv > 8;
    auto kern = two ? paged_attention_tma_warp_kernel<2> : paged_attention_tma_warp_kernel<1>;
    const size_t smem = a2_smem_bytes(AM_MAX_WARPS);
    const int st = ensure_dynamic_smem((const void*)kern, smem, "paged_attention");
    if (st) return st;
    launch_kernel(kern, dim3((unsigned)a.bal_ctas), dim3(32 * AM_MAX_WARPS), smem, s, true, a);
    const int rc = launch_status("paged_attention");
    if (rc) return rc;
    launch_kernel(paged_attention_merge_kernel, dim3((unsigned)(a.rows * a.hkv)), dim3((unsigned)(32 * (a.hq / a.hkv))), 0,
                  s, true, a);
  } else if (a.tma) {
    const bool two = a.hq / a.hkv > 8;
    auto kern = a.bal_ctas > 0 ? (two ? paged_attention_tma_kernel<true, 2> : paged_attention_tma_kernel<true, 1>)
                               : (two ? paged_attention_tma_kernel<false, 2> : paged_attention_tma_kernel<false, 1>);
    const size_t smem = a2_smem_bytes(AM_MAX_WARPS);
    const int st = ensure_dynamic_smem((const void*)kern, smem, "paged_attention");
    if (st) return st;
    launch_kernel(kern, grid, dim3(32 * AM_MAX_WARPS), smem, s, true, a);
  } else if (a.bal_ctas > 0 || use_mma(a.rows, a.hkv, max_total, head_dim)) {
    const int warps = a.bal_ctas > 0 ? AM_MAX_WARPS : std::min(AM_MAX_WARPS, std::max(1, a.tiles_per_split));
    const size_t smem = am_smem_bytes(warps);
    auto kern = a.bal_ctas > 0 ? paged_attention_mma_kernel<true> : paged_attention_mma_kernel<false>;
    const int st = ensure_dynamic_smem((const void*)kern, am_smem_bytes(AM_MAX_WARPS), "paged_attention");
    if (st) return st;
    launch_kernel(kern, grid, dim3(32 * warps), smem, s, true, a);
  } else {
    launch_kernel(head_dim == 128 ? paged_attention_kernel<128> : paged_attention_kernel<64>, grid,
                  dim3((unsigned)(32 * (a.hq / a.hkv))), 0, s, true, a);
  }
  return launch_status("paged_attention");
}

struct SplitPlan {
  int nsplit;
  int tiles_per_split;
  int bal_ctas;   // > 0: the balanced schedule over this many CTAs (nsplit, tiles_per_split unused)
  int max_tiles;  // balanced: tiles per group at most
  int warp;       // balanced: scratch for one partial slot per warp (the TMA kernel's warp schedule)
};

// Splits per (row, head): enough CTAs for about 8 per SM (the kernel is latency-bound per
// CTA; its 32 KB tile ring and 32-512 threads let several share an SM), each split at least
// 4 tiles (2 for contexts up to 64 tiles) so the ring has tiles to overlap, at most
// AT_MAX_SPLIT splits.
// Kernel choice: the tensor-core kernel (head_dim 128) once the (row, head) groups times
// the context tiles reach 4096 -- long contexts or many rows, where the scalar kernel is
// instruction-bound; short decode batches keep the scalar kernel, whose fixed latency is
// lower.
static bool use_mma(int64_t rows, int64_t hkv, int64_t max_total, int64_t head_dim) {
  const int64_t tiles = std::max<int64_t>(1, (max_total + AT_TILE - 1) / AT_TILE);
  return head_dim == 128 && rows * hkv * tiles >= 4096;
}

// The balanced schedule (tensor-core kernel): rows up to this many (each CTA scans their
// lengths into shared memory once).
constexpr int64_t AT_BAL_MAX_ROWS = AT_BAL_MAX_ROWS_DEV;
constexpr int64_t AT_MAX_COUNTERS = 4096;
// scratch head: merge counters (kept at zero between launches), then the warp schedule's
// per-group records, each region fixed in size so that a buffer reused across shapes and
// schedules never finds one where the other lives; the fp32 partials follow
constexpr size_t AT_COUNTER_BYTES = 2 * AT_MAX_COUNTERS * sizeof(unsigned);

static size_t balanced_bytes(int64_t rows, int64_t hq, int64_t hkv, int64_t d, int64_t units) {
  return AT_COUNTER_BYTES + (size_t)(units + rows * hkv) * (hq / hkv) * (2 + d) * sizeof(float);
}

// The tensor-core kernel takes the balanced schedule whenever it can: one resident wave of
// CTAs (3 per SM) sharing the tiles the rows actually hold, so ragged contexts neither
// leave splits empty nor add a partial second wave (32 rows x 32/4 heads, contexts
// U[256,4096]: the fixed splits ran 512 CTAs, the longest row's splits deciding the time).
// Scratch: counters plus (CTAs + groups) partial slots; under a scratch cap the CTA count
// shrinks to fit, down to one per SM, else the fixed splits stay.
// Fixed splits otherwise: the tensor-core kernel wants at least 8 tiles per split (its 4
// warps take 2 each; fewer, longer splits keep the final merge -- dependent L2 round trips
// -- short).
static SplitPlan plan_splits(int64_t rows, int64_t hq, int64_t hkv, int64_t max_total, int64_t head_dim,
                             size_t scratch_cap = SIZE_MAX) {
  const int64_t tiles = std::max<int64_t>(1, (max_total + AT_TILE - 1) / AT_TILE);
  const int64_t groups = std::max<int64_t>(1, rows * hkv);
  const bool mma = use_mma(rows, hkv, max_total, head_dim);
  if (mma && rows <= AT_BAL_MAX_ROWS && groups <= AT_MAX_COUNTERS && groups * tiles < (1LL << 31)) {
    const int64_t ctas = std::min<int64_t>((int64_t)AT_MMA_CTAS_PER_SM * num_sms(), groups * tiles);
    // one partial slot per warp when the scratch allows (the warp schedule), else per CTA
    if (balanced_bytes(rows, hq, hkv, head_dim, ctas * AM_MAX_WARPS) <= scratch_cap)
      return SplitPlan{1, 0, (int)ctas, (int)tiles, 1};
    const size_t slot = (size_t)(hq / hkv) * (2 + head_dim) * sizeof(float);
    int64_t fit = ctas;
    if (balanced_bytes(rows, hq, hkv, head_dim, ctas) > scratch_cap)
      fit = scratch_cap > AT_COUNTER_BYTES ? (int64_t)((scratch_cap - AT_COUNTER_BYTES) / slot) - groups : 0;
    if (fit >= std::min<int64_t>(num_sms(), groups * tiles))
      return SplitPlan{1, 0, (int)std::min(fit, ctas), (int)tiles, 0};
  }
  // the tensor-core kernel holds 3 CTAs per SM (2-stage rings): aim at one resident wave, so
  // each warp has enough tiles to amortise its prologue and merge (3 measured best of 2-4 at
  // the config-3 and config-4 shapes together)
  const int64_t per_sm = mma ? AT_MMA_CTAS_PER_SM : AT_CTAS_PER_SM;
  const int64_t target = (per_sm * num_sms() + groups - 1) / groups;  // splits per group
  const int64_t min_tiles = mma ? 2 * AM_MAX_WARPS : (tiles <= 64 ? 2 : AT_MIN_TILES);
  int64_t tps = std::max<int64_t>(min_tiles, (tiles + target - 1) / target);
  tps = std::min<int64_t>(tps, tiles);
  tps = std::max<int64_t>(tps, (tiles + AT_MAX_SPLIT - 1) / AT_MAX_SPLIT);
  const int64_t ns = (tiles + tps - 1) / tps;
  return SplitPlan{(int)ns, (int)tps, 0, 0, 0};
}

// Workspace layout: AT_MAX_COUNTERS merge counters at offset 0, AT_MAX_COUNTERS per-group
// records after them (both fixed, so that a buffer reused across different shapes never
// finds stale partials where counters live), then the fp32 partials. Fixed splits only split
// for fewer than 8 * SMs (row, head) groups.
static size_t workspace_bytes(int64_t rows, int64_t hq, int64_t hkv, int64_t d, const SplitPlan& p) {
  if (p.bal_ctas > 0) return balanced_bytes(rows, hq, hkv, d, (int64_t)p.bal_ctas * (p.warp ? AM_MAX_WARPS : 1));
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
                                  int64_t num_pages, int32_t* error_flag, const void* q_norm, const void* k_norm,
                                  float norm_eps, void* stream) {
  if (tokens < 0 || hkv <= 0 || head_dim <= 0 || head_dim % 4 || page_size <= 0 || num_pages <= 0)
    return fail(MRB_ERR_ARG, "rope_kv_append: bad shape");
  if ((q_norm && !aligned(q_norm, 4)) || (k_norm && !aligned(k_norm, 4)))
    return fail(MRB_ERR_ARG, "rope_kv_append: norm weights must be 4-byte aligned");
  if (tokens == 0) return MRB_OK;
  if (!k_in || !v_in || !positions || !k_cache || !v_cache || !block_table)
    return fail(MRB_ERR_ARG, "rope_kv_append: null pointer");
  if (q_out && (!q_in || hq <= 0)) return fail(MRB_ERR_ARG, "rope_kv_append: q_out needs q_in and hq");
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return fail(MRB_ERR_ARG, "rope_kv_append: cos/sin mismatch");
  if ((in_row_stride % 2) || (stride_page % 2) || (stride_head % 2) || (stride_tok % 2) || !aligned(k_in, 4) ||
      !aligned(v_in, 4) || (q_in && !aligned(q_in, 4)) || !aligned(k_cache, 4) || !aligned(v_cache, 4) ||
      (q_out && !aligned(q_out, 4)) || (rope_cos && (!aligned(rope_cos, 8) || !aligned(rope_sin, 8) || (head_dim % 4))))
    return fail(MRB_ERR_ARG, "rope_kv_append: rows must be 4-byte aligned (8-byte tables, head_dim % 4 == 0)");
  if (tokens > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "rope_kv_append: too many tokens");
  RopeArgs a{(const __nv_bfloat16*)q_in, (const __nv_bfloat16*)k_in, (const __nv_bfloat16*)v_in, in_row_stride,
             tokens, hq, hkv, head_dim, positions, token_rows, rope_cos, rope_sin, rope_len,
             (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, stride_page, stride_head,
             stride_tok, page_size, block_table, block_table_stride, num_pages, error_flag,
             (const __nv_bfloat16*)q_norm, (const __nv_bfloat16*)k_norm, norm_eps};
  const int64_t heads = (q_out ? hq : 0) + 2 * hkv;
  const unsigned hgroups = (unsigned)std::min<int64_t>(65535, (heads + 7) / 8);
  launch_kernel(rope_kv_append_kernel, dim3((unsigned)tokens, hgroups), dim3(256), 0, (cudaStream_t)stream, true, a);
  return launch_status("rope_kv_append");
}

extern "C" int64_t mrb_paged_attention_timeouts(void) {
  unsigned v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, g_attn_timeouts, sizeof(v));
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "paged_attention_timeouts: %s", cudaGetErrorString(e));
  return (int64_t)v;
}

extern "C" size_t mrb_paged_attention_workspace(int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                                int64_t max_total_tokens) {
  if (rows <= 0 || hkv <= 0 || hq % hkv) return 0;
  return workspace_bytes(rows, hq, hkv, head_dim, plan_splits(rows, hq, hkv, max_total_tokens, head_dim));
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
  const SplitPlan plan = plan_splits(rows, hq, hkv, max_total_tokens, head_dim);
  const size_t need = workspace_bytes(rows, hq, hkv, head_dim, plan);
  if (need > 0 && (workspace == nullptr || workspace_size < need))
    return fail(MRB_ERR_ARG, "paged_attention: workspace of %zu bytes required (got %zu)", need, workspace_size);
  if (rows * hkv > 0x7fffffffLL || plan.nsplit > 65535)
    return fail(MRB_ERR_UNSUPPORTED, "paged_attention: grid too large");
  AttnArgs a{(const __nv_bfloat16*)q, rows, hq, hkv, (const __nv_bfloat16*)k_cache, (const __nv_bfloat16*)v_cache,
             stride_page, stride_head, stride_tok, page_size, block_table, block_table_stride, row_seq, row_len,
             (const __nv_bfloat16*)k_new, (const __nv_bfloat16*)v_new, scale, plan.nsplit, plan.tiles_per_split,
             (__nv_bfloat16*)out, nullptr, nullptr, nullptr, plan.bal_ctas, plan.max_tiles};
  a.warp_sched = plan.warp;
  if (need > 0) {
    if (rows * hkv > AT_MAX_COUNTERS) return fail(MRB_ERR_UNSUPPORTED, "paged_attention: too many split groups");
    a.counters = (unsigned*)workspace;
    a.meta = (unsigned*)workspace + AT_MAX_COUNTERS;
    a.part = (float*)((char*)workspace + AT_COUNTER_BYTES);
  }
  return launch_attention(a, head_dim, max_total_tokens, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ prefill attention (host)

extern "C" int mrb_paged_prefill_attention(const void* q, int64_t n, int64_t hq, int64_t hkv, int64_t head_dim,
                                           int64_t start, const void* k_cache, const void* v_cache,
                                           int64_t stride_page, int64_t stride_head, int64_t stride_tok,
                                           int64_t page_size, const int32_t* block_table, int64_t num_pages,
                                           int32_t* error_flag, float scale, void* out, void* stream) {
  if (n < 0 || hq <= 0 || hkv <= 0 || hq % hkv || start < 0 || page_size <= 0 || num_pages <= 0)
    return fail(MRB_ERR_ARG, "paged_prefill_attention: bad shape");
  if (hq / hkv > AT_MAX_GROUP)
    return fail(MRB_ERR_UNSUPPORTED, "paged_prefill_attention: query group %lld exceeds %d",
                (long long)(hq / hkv), AT_MAX_GROUP);
  if (head_dim != 128 || page_size % AT_TILE)
    return fail(MRB_ERR_UNSUPPORTED, "paged_prefill_attention: head_dim 128 and pages of a multiple of 16 tokens "
                "(got %lld, %lld)", (long long)head_dim, (long long)page_size);
  if (n == 0) return MRB_OK;
  if (!q || !k_cache || !v_cache || !block_table || !out)
    return fail(MRB_ERR_ARG, "paged_prefill_attention: null pointer");
  if (!aligned(q, 16) || !aligned(out, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || (stride_page % 8) ||
      (stride_head % 8) || (stride_tok % 8))
    return fail(MRB_ERR_ARG, "paged_prefill_attention: q/out and K/V rows must be 16-byte aligned");
  if ((n + AT_TILE - 1) / AT_TILE * PF_MAX_CLUSTER > 0x7fffffffLL || hkv > 65535)
    return fail(MRB_ERR_UNSUPPORTED, "paged_prefill_attention: grid too large");
  // CTAs per (query block, KV head): PF_MAX_CLUSTER when the longest causal walk has 8 key
  // tiles or more and the clusters fit one resident wave (two CTAs per SM), else 1 -- a
  // second wave costs more than the shorter walk saves (measured at a 512-token prompt:
  // 2 CTAs 40 us, 4 CTAs 49 us, 8 CTAs 93 us, 1 CTA 59 us)
  const int group = (int)(hq / hkv);
  const int64_t tiles = (start + n + AT_TILE - 1) / AT_TILE;
  const int64_t pairs = ((n + AT_TILE - 1) / AT_TILE) * hkv;
  const int cluster = tiles >= 8 && pairs * PF_MAX_CLUSTER <= 2 * (int64_t)num_sms() ? PF_MAX_CLUSTER : 1;
  const size_t smem = pf_smem_bytes(group);
  const int smem_st = ensure_dynamic_smem((const void*)paged_prefill_attention_kernel, smem, "paged_prefill_attention");
  if (smem_st) return smem_st;
  PrefillArgs a{(const __nv_bfloat16*)q, n, hq, hkv, start, (const __nv_bfloat16*)k_cache,
                (const __nv_bfloat16*)v_cache, stride_page, stride_head, stride_tok, page_size, block_table,
                num_pages, error_flag, scale, (__nv_bfloat16*)out, cluster};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(((n + AT_TILE - 1) / AT_TILE) * cluster), (unsigned)hkv);
  cfg.blockDim = dim3((unsigned)(32 * group));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = (unsigned)cluster;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, paged_prefill_attention_kernel, a);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "paged_prefill_attention: launch: %s", cudaGetErrorString(e));
  return launch_status("paged_prefill_attention");
}

// ------------------------------------------------------------------ fused decode step (host)

// Whether the 16-CTA cluster fits for this kernel and block (non-portable size; 8 otherwise).
template <typename Kern>
static bool fused_cluster16_fits(Kern kern, int threads, size_t smem) {
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
      (smem > 48 * 1024 &&
       cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)) {
    cudaGetLastError();
    return false;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(FD_MAX_CLUSTER, 1);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = FD_MAX_CLUSTER;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  const bool ok = cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0;
  cudaGetLastError();
  return ok;
}

// Launch plan of the fused step: CTAs per (row, KV head) cluster and warps per CTA.
//  * tensor-core kernel (head_dim 128, pages of a multiple of 16 tokens): a power of two of
//    CTAs with about FD_MMA_MIN_TILES tiles each at max_total_tokens, up to 4 warps;
//  * scalar kernel: about FD_MIN_TILES tiles per CTA, one warp per query head.
// At most 16 CTAs (8 where the device cannot co-schedule 16 of them) and two per SM over
// all (row, KV head) clusters.
#ifndef FD_MMA_MIN_TILES
#define FD_MMA_MIN_TILES 4
#endif
struct FusedPlan {
  bool mma;
  int cluster;
  int warps;
};

static FusedPlan fused_plan(int64_t rows, int64_t hkv, int64_t head_dim, int64_t page_size, int64_t max_total,
                            int group) {
  FusedPlan p{head_dim == 128 && page_size % AT_TILE == 0, 1, group};
  const int64_t tiles = std::max<int64_t>(1, (max_total + AT_TILE - 1) / AT_TILE);
  const int64_t groups = std::max<int64_t>(1, rows * hkv);
  int64_t s = (tiles + (p.mma ? FD_MMA_MIN_TILES : FD_MIN_TILES) - 1) / (p.mma ? FD_MMA_MIN_TILES : FD_MIN_TILES);
  s = std::min<int64_t>(s, FD_MAX_CLUSTER);
  s = std::min<int64_t>(s, std::max<int64_t>(1, 2 * num_sms() / groups));
  if (p.mma) {
    int64_t pw = 1;
    while (pw * 2 <= s) pw *= 2;
    s = pw;
    p.warps = (int)std::min<int64_t>(AM_MAX_WARPS, (tiles + s - 1) / s);
  }
  if (s > 8) {
    static int fits[2][AT_MAX_GROUP + 1] = {};  // 0 unknown, 1 yes, -1 no
    int& f = fits[p.mma ? 1 : 0][p.mma ? p.warps : group];
    if (f == 0) {
      const bool ok = p.mma ? fused_cluster16_fits(rope_append_attention_mma_kernel, 32 * p.warps,
                                                   am_smem_bytes(AM_MAX_WARPS))
                            : (head_dim == 128 ? fused_cluster16_fits(rope_append_attention_kernel<128>, 32 * group, 0)
                                               : fused_cluster16_fits(rope_append_attention_kernel<64>, 32 * group, 0));
      f = ok ? 1 : -1;
    }
    if (f < 0) s = 8;
  }
  p.cluster = (int)s;
  return p;
}

static int launch_fused(const FusedArgs& a, int64_t head_dim, int64_t max_total, cudaStream_t st) {
  const int group = (int)(a.hq / a.hkv);
  const FusedPlan p = fused_plan(a.rows, a.hkv, head_dim, a.page_size, max_total, group);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.cluster, (unsigned)(a.rows * a.hkv));
  cfg.blockDim = dim3((unsigned)(32 * (p.mma ? p.warps : group)));
  cfg.dynamicSmemBytes = p.mma ? am_smem_bytes(p.warps) : 0;
  cfg.stream = st;
  if (p.mma) {
    const int smem_st = ensure_dynamic_smem((const void*)rope_append_attention_mma_kernel,
                                            am_smem_bytes(AM_MAX_WARPS), "rope_append_attention");
    if (smem_st) return smem_st;
  }
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (p.cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)p.cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = n ? attr : nullptr;
  cfg.numAttrs = n;
  const cudaError_t e =
      p.mma ? cudaLaunchKernelEx(&cfg, rope_append_attention_mma_kernel, a)
            : (head_dim == 128 ? cudaLaunchKernelEx(&cfg, rope_append_attention_kernel<128>, a)
                               : cudaLaunchKernelEx(&cfg, rope_append_attention_kernel<64>, a));
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "rope_append_attention: launch: %s", cudaGetErrorString(e));
  return launch_status("rope_append_attention");
}

extern "C" int mrb_rope_append_attention_cluster(int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                                 int64_t max_total_tokens) {
  if (rows <= 0 || hq <= 0 || hkv <= 0 || hq % hkv || hq / hkv > AT_MAX_GROUP) return 0;
  if (head_dim != 128 && head_dim != 64) return 0;
  return fused_plan(rows, hkv, head_dim, AT_TILE, max_total_tokens, (int)(hq / hkv)).cluster;
}

extern "C" int mrb_rope_append_attention(const void* q_in, const void* k_in, const void* v_in, int64_t in_row_stride,
                                         int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                         const int32_t* positions, const int32_t* row_seq, const float* rope_cos,
                                         const float* rope_sin, int64_t rope_len, const void* q_norm,
                                         const void* k_norm, float norm_eps, void* k_cache, void* v_cache,
                                         int64_t stride_page, int64_t stride_head, int64_t stride_tok,
                                         int64_t page_size, const int32_t* block_table, int64_t block_table_stride,
                                         int64_t num_pages, int32_t* error_flag, float scale,
                                         int64_t max_total_tokens, int state_ready, void* out, void* stream) {
  if (rows < 0 || hq <= 0 || hkv <= 0 || hq % hkv || page_size <= 0 || num_pages <= 0 || max_total_tokens < 0)
    return fail(MRB_ERR_ARG, "rope_append_attention: bad shape");
  if (hq / hkv > AT_MAX_GROUP)
    return fail(MRB_ERR_UNSUPPORTED, "rope_append_attention: query group %lld exceeds %d", (long long)(hq / hkv),
                AT_MAX_GROUP);
  if (head_dim != 64 && head_dim != 128)
    return fail(MRB_ERR_UNSUPPORTED, "rope_append_attention: head_dim %lld (supported: 64, 128)",
                (long long)head_dim);
  if (rows == 0) return MRB_OK;
  if (!q_in || !k_in || !v_in || !positions || !k_cache || !v_cache || !block_table || !out)
    return fail(MRB_ERR_ARG, "rope_append_attention: null pointer");
  if ((rope_cos == nullptr) != (rope_sin == nullptr))
    return fail(MRB_ERR_ARG, "rope_append_attention: cos/sin mismatch");
  if ((in_row_stride % 2) || !aligned(q_in, 4) || !aligned(k_in, 4) || !aligned(v_in, 4) ||
      (rope_cos && (!aligned(rope_cos, 8) || !aligned(rope_sin, 8))) || (q_norm && !aligned(q_norm, 4)) ||
      (k_norm && !aligned(k_norm, 4)))
    return fail(MRB_ERR_ARG, "rope_append_attention: q/k/v rows and norms must be 4-byte aligned (8-byte tables)");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || (stride_page % 8) || (stride_head % 8) || (stride_tok % 8))
    return fail(MRB_ERR_ARG, "rope_append_attention: K/V rows must be 16-byte aligned");
  if (rows * hkv > 65535) return fail(MRB_ERR_UNSUPPORTED, "rope_append_attention: grid too large");
  FusedArgs a{(const __nv_bfloat16*)q_in, (const __nv_bfloat16*)k_in, (const __nv_bfloat16*)v_in, in_row_stride,
              rows, hq, hkv, positions, row_seq, rope_cos, rope_sin, rope_len, (const __nv_bfloat16*)q_norm,
              (const __nv_bfloat16*)k_norm, norm_eps, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, stride_page,
              stride_head, stride_tok, page_size, block_table, block_table_stride, num_pages, error_flag, scale,
              (__nv_bfloat16*)out, state_ready ? 1 : 0};
  return launch_fused(a, head_dim, max_total_tokens, (cudaStream_t)stream);
}

// ------------------------------------------------------------------ decode-step bookkeeping

// After a greedy decode step: the chosen token becomes the next input, every row advances
// one position. Runs inside the captured decode graph so replays need no host writes.
__global__ void decode_advance_kernel(const int64_t* __restrict__ next_ids, int64_t* __restrict__ input_ids,
                                      int32_t* __restrict__ positions, int32_t* __restrict__ row_len,
                                      int64_t rows) {
  pdl_launch_dependents();
  pdl_wait();
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
  launch_kernel(decode_advance_kernel, dim3((unsigned)((rows + 255) / 256)), dim3(256), 0, (cudaStream_t)stream, true,
                next_ids, input_ids, positions, row_len, rows);
  return launch_status("decode_advance");
}

// ------------------------------------------------------------------ allocation-free variant
//
// Some callers cannot allocate device memory at all: a host process that reserves all GPU
// memory for its own pool up front (so a plugin's cudaMalloc would fail or fragment it),
// code on a latency-critical path where cudaMalloc/cudaFree may synchronise the device, and
// thin bindings that only ever receive raw pointers from their host. For them,
// mrb_paged_attention_static runs the same split-K kernel with its scratch in a fixed
// static device array instead of a caller workspace.

// Scratch of mrb_paged_attention_static: merge counters, then split partials. Zero at load
// (static storage); the kernel returns every counter to zero, so each call starts clean.
static __device__ __align__(256) unsigned char g_attn_static_scratch[MRB_ATTN_STATIC_SCRATCH_BYTES];

namespace mrb {
namespace {
constexpr int kMaxDevices = 64;
// Per device: the context the address was resolved in and the array's device address there.
// A device reset (cudaDeviceReset) makes a new primary context in which the module, and so
// the array, is loaded again at a possibly different address; a changed context handle sends
// the next call back through cudaGetSymbolAddress.
std::mutex g_static_lock;
void* g_static_ctx[kMaxDevices] = {nullptr};
void* g_static_ptr[kMaxDevices] = {nullptr};

using CtxGetCurrentFn = int (*)(void**);  // the driver's cuCtxGetCurrent(CUcontext*)

CtxGetCurrentFn ctx_get_current() {
  static const CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (CtxGetCurrentFn) nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

// The device address of g_attn_static_scratch on the current device (nullptr on error, with
// the message set). Looked up once per device and context, with that device current.
void* static_scratch_address(int dev) {
  const CtxGetCurrentFn get_ctx = ctx_get_current();
  void* ctx = nullptr;
  if (!get_ctx || get_ctx(&ctx) != 0 || ctx == nullptr) {
    fail(MRB_ERR_CUDA, "paged_attention_static: no current CUDA context");
    return nullptr;
  }
  std::lock_guard<std::mutex> hold(g_static_lock);
  if (g_static_ctx[dev] != ctx || g_static_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_attn_static_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      fail(MRB_ERR_CUDA, "paged_attention_static: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    g_static_ctx[dev] = ctx;
    g_static_ptr[dev] = ptr;
  }
  return g_static_ptr[dev];
}
}  // namespace
}  // namespace mrb

extern "C" size_t mrb_paged_attention_static_capacity(void) { return MRB_ATTN_STATIC_SCRATCH_BYTES; }

extern "C" int mrb_paged_attention_static(const void* q, int64_t rows, int64_t hq, int64_t hkv, int64_t head_dim,
                                          const void* k_cache, const void* v_cache, int64_t stride_page,
                                          int64_t stride_head, int64_t stride_tok, int64_t page_size,
                                          const int32_t* block_table, int64_t block_table_stride,
                                          const int32_t* row_seq, const int32_t* row_len, const void* k_new,
                                          const void* v_new, float scale, int64_t max_total_tokens, void* out,
                                          void* stream) {
  if (rows < 0 || hq <= 0 || hkv <= 0 || hq % hkv || page_size <= 0 || max_total_tokens < 0)
    return fail(MRB_ERR_ARG, "paged_attention_static: bad shape");
  if (rows == 0) return MRB_OK;
  if (hq / hkv > AT_MAX_GROUP)
    return fail(MRB_ERR_UNSUPPORTED, "paged_attention_static: query group %lld exceeds %d", (long long)(hq / hkv),
                AT_MAX_GROUP);
  if (head_dim != 64 && head_dim != 128)
    return fail(MRB_ERR_UNSUPPORTED, "paged_attention_static: head_dim %lld (supported: 64, 128)",
                (long long)head_dim);
  if (!q || !k_cache || !v_cache || !block_table || !row_len || !out)
    return fail(MRB_ERR_ARG, "paged_attention_static: null pointer");
  if ((k_new == nullptr) != (v_new == nullptr))
    return fail(MRB_ERR_ARG, "paged_attention_static: k_new/v_new mismatch");
  if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || (stride_page % 8) || (stride_head % 8) || (stride_tok % 8) ||
      (k_new && !aligned(k_new, 16)))
    return fail(MRB_ERR_ARG, "paged_attention_static: K/V rows must be 16-byte aligned");
  const SplitPlan plan = plan_splits(rows, hq, hkv, max_total_tokens, head_dim, MRB_ATTN_STATIC_SCRATCH_BYTES);
  const size_t need = workspace_bytes(rows, hq, hkv, head_dim, plan);
  if (need > MRB_ATTN_STATIC_SCRATCH_BYTES)
    return fail(MRB_ERR_UNSUPPORTED,
                "paged_attention_static: these sizes need %zu bytes of scratch, above the static %d; "
                "use mrb_paged_attention with a workspace",
                need, MRB_ATTN_STATIC_SCRATCH_BYTES);
  if (rows * hkv > 0x7fffffffLL || plan.nsplit > 65535)
    return fail(MRB_ERR_UNSUPPORTED, "paged_attention_static: grid too large");
  void* scratch = nullptr;
  if (need > 0) {
    if (rows * hkv > AT_MAX_COUNTERS)
      return fail(MRB_ERR_UNSUPPORTED, "paged_attention_static: too many split groups");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "paged_attention_static: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(MRB_ERR_UNSUPPORTED, "paged_attention_static: device %d", dev);
    // the device address of the static array (host code only has a host-side stand-in for
    // it), resolved once per device and context with that device current
    scratch = static_scratch_address(dev);
    if (!scratch) return MRB_ERR_CUDA;
  }
  AttnArgs a{(const __nv_bfloat16*)q, rows, hq, hkv, (const __nv_bfloat16*)k_cache, (const __nv_bfloat16*)v_cache,
             stride_page, stride_head, stride_tok, page_size, block_table, block_table_stride, row_seq, row_len,
             (const __nv_bfloat16*)k_new, (const __nv_bfloat16*)v_new, scale, plan.nsplit, plan.tiles_per_split,
             (__nv_bfloat16*)out, nullptr, nullptr, nullptr, plan.bal_ctas, plan.max_tiles};
  a.warp_sched = plan.warp;
  if (scratch) {
    a.counters = (unsigned*)scratch;
    a.meta = (unsigned*)scratch + AT_MAX_COUNTERS;
    a.part = (float*)((char*)scratch + AT_COUNTER_BYTES);
  }
  return launch_attention(a, head_dim, max_total_tokens, (cudaStream_t)stream);
}
