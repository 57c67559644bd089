// Prefill / large-batch W8A16 projection on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   y[m, j] = bf16(acc[m, j] * scale[j])                      (plain; + bf16 bias, rounded again)
//   y[m, j] = bf16(bf16(silu(bf16(g * sg[j]))) * bf16(u * su[j]))   (paired gate/up, SwiGLU)
// with acc[m, j] = sum_k x[m, k] * codes[j, k], bf16 x bf16 products accumulated in fp32
// (kind::f16). int8 codes convert to bf16 exactly, so this is the W8A16 contract of the
// reference's QStore linear (engine/kernels/qstore.py:95-128) with the per-row scale applied
// once to the accumulator.
//
// The tensor core reads both operands from shared memory, but the weights arrive as int8:
//  * warp 0, one thread: TMA producer of the raw int8 weight boxes ([BN x 64 B], no swizzle;
//    the gate and up halves as two boxes when paired) into a ring of its own, running ahead
//    of the conversion;
//  * warp 6, one thread: TMA producer of the activation boxes ([BM x 64 bf16], 128-byte
//    swizzle) into the activation ring;
//  * warps 7-14 (256 threads): converters. Per stage they wait for a raw box and a free
//    converted-weight stage, turn the raw int8 box into bf16 rows in the 128-byte-swizzled
//    K-major layout the MMA descriptor reads (chunk c of row r at c ^ (r & 7)), fence the
//    writes to the async proxy and arrive on the stage barrier (one arrival per warp);
//    the three rings (activations, raw weights, converted weights) run ahead independently;
//  * warp 1: TMEM owner; one thread issues tcgen05.mma (M=128 per accumulator half, N=BN,
//    K=16) and commits stages and finished tiles;
//  * warps 2-5: epilogue, TMEM -> registers -> bf16 rows.
// Tiles are HALVES 128-row activation accumulators x BN weight rows, chosen by SM fill like
// the int8 GEMM; persistent CTAs walk tiles with the M tiles of one weight tile adjacent.
// Skinny activation blocks (17-128 rows) whose tiles fill few SMs split k over the CTAs of a
// thread-block cluster: each parks its fp32 partial tile in its own shared memory, and after
// a cluster barrier every CTA sums one column slice over the cluster's partials in rank order
// through distributed shared memory (deterministic for a given shape) and writes it.
// Every wait is bounded; on a timeout the CTA records it, stops, and still frees its TMEM.
// No load uses cluster multicast.
#include "qrow_common.cuh"
#include "tc_common.cuh"

#include <algorithm>

namespace mrb {

constexpr int TW_HM = 128;            // MMA M (activation rows of one accumulator)
constexpr int TW_BKE = 64;            // k elements per stage: one 128-byte bf16 swizzle row
constexpr int TW_UK_BYTES = 32;       // k bytes per MMA (16 bf16)
constexpr int TW_A_WARP = 6;          // activation TMA producer warp
constexpr int TW_CVT_WARP0 = 7;       // first converter warp
constexpr int TW_CVT_THREADS = 256;   // 8 converter warps
constexpr int TW_CVT_WARPS = TW_CVT_THREADS / 32;
constexpr int TW_EPI_THREADS = 128;
constexpr int TW_THREADS = TW_CVT_WARP0 * 32 + TW_CVT_THREADS;
constexpr size_t TW_SMEM_LIMIT = 227 * 1024;

template <int HALVES, int BN>
struct TwTile {
  static constexpr int BM = TW_HM * HALVES;
  static constexpr int A_BYTES = BM * 128;   // bf16 activations [BM x 64]
  static constexpr int B_BYTES = BN * 128;   // converted bf16 weights [BN x 64]
  static constexpr int RAW_BYTES = BN * 64;  // int8 weights [BN x 64]
  // ring depths: activations, converted weights, raw weights (about 224 KB in all)
  static constexpr int A_STAGES = HALVES == 2 ? 3 : (BN == 256 ? 4 : 6);
  static constexpr int B_STAGES = HALVES == 2 ? 2 : (BN == 256 ? 2 : 3);
  static constexpr int RAW_STAGES = HALVES == 2 ? 4 : (BN == 256 ? 6 : 8);
  static constexpr size_t RING_AB = (size_t)A_STAGES * A_BYTES + (size_t)B_STAGES * B_BYTES;
  static constexpr int NBUF = HALVES == 1 ? 2 : 1;
  static constexpr unsigned TMEM_COLS = HALVES * BN * NBUF <= 256 ? 256u : 512u;
  static constexpr size_t SMEM = 1024 + RING_AB + (size_t)RAW_STAGES * RAW_BYTES + 512;
  static_assert(SMEM <= TW_SMEM_LIMIT, "tile does not fit in shared memory");
  static_assert(HALVES * BN * NBUF <= 512, "accumulators exceed TMEM");
  static constexpr int PSTRIDE = BN + 4;  // fp32 row stride of a parked partial (bank spread)
  // a split-K partial is parked over the rings (all three are idle by then)
  static_assert((size_t)TW_HM * PSTRIDE * 4 <= RING_AB + (size_t)RAW_STAGES * RAW_BYTES, "partial exceeds the rings");
};
constexpr int TW_MAX_CLUSTER = 8;

struct TwGemmArgs {
  CUtensorMap map_x;   // x [m, k] bf16, box [BM rows, 64], 128-byte swizzle
  CUtensorMap map_w;   // codes [n, k] int8, box [BN (paired: BN/2) rows, 64 B]
  CUtensorMap map_u;   // paired: up codes [n, k] int8, box [BN/2 rows, 64 B]
  int64_t m, n, k;     // n: output columns
  int tiles_m, tiles_n, kblocks;
  bool paired;
  const float* scales;     // [n]
  const float* scales_up;  // [n] (paired)
  const float* bias;       // [n] or null (plain only)
  __nv_bfloat16* y;        // [m, n] (null in argmax mode)
  bool vec_store;          // n % 8 == 0 and y 16-byte aligned
  // greedy-head mode (packed non-null): per activation row, atomicMax of pack(logit, col)
  // over columns < semantic; logits (fp32 [m, n]) optionally written
  unsigned long long* packed;
  float* logits;
  int64_t semantic;
  int splits, kb_per;  // split-K: k blocks [split * kb_per, +kb_per); splits > 1 = cluster of splits CTAs
};

__device__ unsigned g_tw_timeouts = 0;

template <int HALVES, int BN>
__global__ void __launch_bounds__(TW_THREADS, 1) tc_w8a16_gemm_kernel(const __grid_constant__ TwGemmArgs a) {
  using Tile = TwTile<HALVES, BN>;
  constexpr int A_STAGES = Tile::A_STAGES, B_STAGES = Tile::B_STAGES, RAW_STAGES = Tile::RAW_STAGES;
  constexpr int NBUF = Tile::NBUF, BM = Tile::BM;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* a_base = smem;                                         // activation ring
  unsigned char* b_base = smem + (size_t)A_STAGES * Tile::A_BYTES;      // converted-weight ring
  unsigned char* raw_base = smem + Tile::RING_AB;                       // raw int8 ring
  uint64_t* a_full = reinterpret_cast<uint64_t*>(raw_base + RAW_STAGES * Tile::RAW_BYTES);
  uint64_t* a_empty = a_full + A_STAGES;
  uint64_t* b_full = a_empty + A_STAGES;
  uint64_t* b_empty = b_full + B_STAGES;
  uint64_t* raw_full = b_empty + B_STAGES;
  uint64_t* raw_empty = raw_full + RAW_STAGES;
  uint64_t* acc_full = raw_empty + RAW_STAGES;
  uint64_t* acc_empty = acc_full + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < A_STAGES; ++s) {
      mbar_init(a_full + s, 1);  // the activation TMA (expect_tx)
      mbar_init(a_empty + s, 1);
    }
    for (int s = 0; s < B_STAGES; ++s) {
      mbar_init(b_full + s, TW_CVT_WARPS);  // one arrival per converter warp
      mbar_init(b_empty + s, 1);
    }
    for (int s = 0; s < RAW_STAGES; ++s) {
      mbar_init(raw_full + s, 1);
      mbar_init(raw_empty + s, TW_CVT_WARPS);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, TW_EPI_THREADS);
    }
    *abort_flag = 0;
    fence_proxy_async_smem();
  }
  if (warp == 1) tmem_alloc(tmem_slot, Tile::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  const int ntiles = a.tiles_m * a.tiles_n;
  const int items = ntiles * a.splits;
  auto fail_wait = [&]() {
    *abort_flag = 1;
    atomicAdd(&g_tw_timeouts, 1u);
  };
  auto acc_col = [&](int b, int h) { return (uint32_t)((b * HALVES + h) * BN); };
  const int out_cols = a.paired ? BN / 2 : BN;

  if (warp == 0) {
    // ---------------- raw int8 weight producer
    if (lane == 0) {
      pdl_wait();
      int rs = 0;
      unsigned rphase = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int tn = (it / a.splits) / a.tiles_m;
        const int kb0 = (it % a.splits) * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(raw_empty + rs, rphase ^ 1u)) {
            fail_wait();
            break;
          }
          unsigned char* dst = raw_base + rs * Tile::RAW_BYTES;
          mbar_arrive_expect_tx(raw_full + rs, Tile::RAW_BYTES);
          if (a.paired) {
            tma_load_2d(dst, &a.map_w, kb * TW_BKE, tn * (BN / 2), raw_full + rs);
            tma_load_2d(dst + Tile::RAW_BYTES / 2, &a.map_u, kb * TW_BKE, tn * (BN / 2), raw_full + rs);
          } else {
            tma_load_2d(dst, &a.map_w, kb * TW_BKE, tn * BN, raw_full + rs);
          }
          if (++rs == RAW_STAGES) {
            rs = 0;
            rphase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(UMMA_D_F32, UMMA_BF16, UMMA_BF16, TW_HM, BN);
      int as = 0, bs = 0, buf = 0;
      unsigned aphase = 0, bphase = 0, acc_phase = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int t = it / a.splits;
        const int kb0 = (it % a.splits) * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
        if (!mbar_wait_bounded(acc_empty + buf, acc_phase ^ 1u)) {
          fail_wait();
          break;
        }
        tc_fence_after();
        int halves = HALVES;
        while (halves > 1 && (int64_t)(t % a.tiles_m) * BM + (halves - 1) * TW_HM >= a.m) --halves;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(a_full + as, aphase) || !mbar_wait_bounded(b_full + bs, bphase)) {
            fail_wait();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(a_base + as * Tile::A_BYTES);
          const uint32_t sb = smem_u32(b_base + bs * Tile::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < 128 / TW_UK_BYTES; ++kk) {
            const uint64_t db = umma_desc_k_sw128(sb + kk * TW_UK_BYTES);
#pragma unroll
            for (int h = 0; h < HALVES; ++h)
              if (h < halves)
                umma_f16(tmem + acc_col(buf, h), umma_desc_k_sw128(sa + h * TW_HM * 128 + kk * TW_UK_BYTES), db,
                         idesc, kb > kb0 || kk > 0);
          }
          umma_commit(a_empty + as);  // both stages are free once these MMAs have read them
          umma_commit(b_empty + bs);
          if (++as == A_STAGES) {
            as = 0;
            aphase ^= 1u;
          }
          if (++bs == B_STAGES) {
            bs = 0;
            bphase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(acc_full + buf);
        if (++buf == NBUF) {
          buf = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else if (warp < TW_A_WARP) {
    // ---------------- epilogue
    pdl_wait();
    const int q = warp & 3;
    int buf = 0;
    unsigned acc_phase = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
      const int t = it / a.splits;
      bool ok = !*abort_flag && mbar_wait_bounded(acc_full + buf, acc_phase);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !*abort_flag) fail_wait();
        break;
      }
      tc_fence_after();
      const int tm = t % a.tiles_m, tn = t / a.tiles_m;
      if (a.splits > 1) {
        // cluster split-K (one work item per CTA, single-half tiles): park this k range's
        // fp32 partial in shared memory for the reduction after the role loops
        float* part = reinterpret_cast<float*>(smem) + (q * 32 + lane) * Tile::PSTRIDE;
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + acc_col(buf, 0);
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32cols(tbase + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<uint4*>(part + c0 + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
      }
      for (int h = 0; h < HALVES && a.splits == 1; ++h) {
        if ((int64_t)tm * BM + h * TW_HM >= a.m) break;
        const int64_t row = (int64_t)tm * BM + h * TW_HM + q * 32 + lane;
        const bool row_ok = row < a.m;
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + acc_col(buf, h);
        unsigned long long best = 0ull;  // argmax mode: this row's best key over the tile
        for (int c0 = 0; c0 < out_cols; c0 += 32) {
          uint32_t v[32], u[32];
          __syncwarp();
          tmem_ld_32cols(tbase + (uint32_t)c0, v);
          if (a.paired) tmem_ld_32cols(tbase + (uint32_t)(BN / 2 + c0), u);
          const int64_t col0 = (int64_t)tn * out_cols + c0;
          if (!row_ok || col0 >= a.n) continue;
          if (a.packed) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int64_t col = col0 + j;
              const float val = __uint_as_float(v[j]) * __ldg(a.scales + (col < a.n ? col : a.n - 1));
              if (col < a.n && a.logits) a.logits[row * a.n + col] = val;
              if (col < a.semantic) {
                const unsigned long long key = pack_argmax(val, col);
                best = key > best ? key : best;
              }
            }
            continue;
          }
          __align__(16) __nv_bfloat16 out[32];
          if (a.paired) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int64_t col = col0 + j < a.n ? col0 + j : a.n - 1;
              const float gv = round_bf16(__uint_as_float(v[j]) * __ldg(a.scales + col));
              const float uv = round_bf16(__uint_as_float(u[j]) * __ldg(a.scales_up + col));
              out[j] = __float2bfloat16_rn(round_bf16(silu_f32(gv)) * uv);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int64_t col = col0 + j < a.n ? col0 + j : a.n - 1;
              float r = __uint_as_float(v[j]) * __ldg(a.scales + col);
              if (a.bias) r = round_bf16(r) + round_bf16(__ldg(a.bias + col));
              out[j] = __float2bfloat16_rn(r);
            }
          }
          __nv_bfloat16* dst = a.y + row * a.n + col0;
          if (a.vec_store && col0 + 32 <= a.n) {
#pragma unroll
            for (int j = 0; j < 32; j += 8)
              *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(out + j);
          } else {
            for (int j = 0; j < 32 && col0 + j < a.n; ++j) dst[j] = out[j];
          }
        }
        if (a.packed && row_ok && best != 0ull) atomicMax(a.packed + row, best);
      }
      tc_fence_before();
      mbar_arrive(acc_empty + buf);
      if (++buf == NBUF) {
        buf = 0;
        acc_phase ^= 1u;
      }
    }
  } else if (warp == TW_A_WARP) {
    // ---------------- activation TMA producer
    if (lane == 0) {
      pdl_wait();  // the activations come from the previous kernel
      int as = 0;
      unsigned aphase = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int tm = (it / a.splits) % a.tiles_m;
        const int kb0 = (it % a.splits) * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(a_empty + as, aphase ^ 1u)) {
            fail_wait();
            break;
          }
          mbar_arrive_expect_tx(a_full + as, Tile::A_BYTES);
          tma_load_2d(a_base + as * Tile::A_BYTES, &a.map_x, kb * TW_BKE, tm * BM, a_full + as);
          if (++as == A_STAGES) {
            as = 0;
            aphase ^= 1u;
          }
        }
      }
    }
  } else {
    // ---------------- converters: int8 raw box -> swizzled bf16 B operand
    const int ct = tid - TW_CVT_WARP0 * 32;
    int bs = 0, rs = 0;
    unsigned bphase = 0, rphase = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const int kb0 = (it % a.splits) * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
      for (int kb = kb0; kb < kb1; ++kb) {
        // waits are made warp-uniform: the warp signals with one lane after __syncwarp
        ok = __all_sync(0xffffffffu, !*abort_flag && mbar_wait_bounded(b_empty + bs, bphase ^ 1u));
        ok = __all_sync(0xffffffffu, ok && mbar_wait_bounded(raw_full + rs, rphase));
        if (!ok) {
          if (lane == 0 && !*abort_flag) fail_wait();
          break;
        }
        const unsigned char* raw = raw_base + rs * Tile::RAW_BYTES;
        unsigned char* dst = b_base + bs * Tile::B_BYTES;
#pragma unroll
        for (int j = 0; j < BN * 4 / TW_CVT_THREADS; ++j) {
          const int i = ct + j * TW_CVT_THREADS;  // 16-byte chunk of the raw box
          const int r = i >> 2, qk = i & 3;       // weight row, k quarter (16 codes)
          const uint4 w = *reinterpret_cast<const uint4*>(raw + r * 64 + qk * 16);
          uint4 lo, hi;
          i8x4_to_bf16x2(w.x, lo.x, lo.y);
          i8x4_to_bf16x2(w.y, lo.z, lo.w);
          i8x4_to_bf16x2(w.z, hi.x, hi.y);
          i8x4_to_bf16x2(w.w, hi.z, hi.w);
          unsigned char* row = dst + r * 128;
          *reinterpret_cast<uint4*>(row + (((2 * qk) ^ (r & 7)) << 4)) = lo;
          *reinterpret_cast<uint4*>(row + (((2 * qk + 1) ^ (r & 7)) << 4)) = hi;
        }
        // every writer fences its rows to the async proxy; one lane per warp then signals
        // (one arrival per warp keeps the barrier traffic off the shared-memory atomics)
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(raw_empty + rs);
          mbar_arrive(b_full + bs);
        }
        if (++rs == RAW_STAGES) {
          rs = 0;
          rphase ^= 1u;
        }
        if (++bs == B_STAGES) {
          bs = 0;
          bphase ^= 1u;
        }
      }
    }
  }

  if (a.splits > 1) {
    // ---------------- cluster split-K reduction (every thread takes part in both barriers)
    __syncwarp();
    cluster_sync_all();  // every CTA of the cluster has parked its partial tile
    if (warp >= 2 && warp < TW_A_WARP) {
      const unsigned nsplit = (unsigned)a.splits, rank = cluster_ctarank();
      const int t = blockIdx.x / a.splits;
      const int tm = t % a.tiles_m, tn = t / a.tiles_m;
      const int groups = out_cols / 4;  // 4-column output groups; this CTA reduces [g0, g1)
      const int g0 = (int)(rank * groups / nsplit), g1 = (int)((rank + 1) * groups / nsplit), ng = g1 - g0;
      const int64_t rows_left = a.m - (int64_t)tm * BM;
      const int rows = rows_left < BM ? (int)rows_left : BM;
      const uint32_t base = smem_u32(smem);
      for (int unit = tid - 64; unit < rows * ng; unit += TW_EPI_THREADS) {
        const int r = unit / ng, c = (g0 + unit % ng) * 4;  // tile row, tile-local output column
        float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (unsigned p = 0; p < (unsigned)TW_MAX_CLUSTER; ++p) {
          if (p < nsplit) {  // rank order: the same sum on every run
            const int4 g = ld_shared_cluster_v4(mapa_shared(base + (uint32_t)(r * Tile::PSTRIDE + c) * 4u, p));
            sg[0] += __int_as_float(g.x); sg[1] += __int_as_float(g.y);
            sg[2] += __int_as_float(g.z); sg[3] += __int_as_float(g.w);
            if (a.paired) {
              const int4 w =
                  ld_shared_cluster_v4(mapa_shared(base + (uint32_t)(r * Tile::PSTRIDE + BN / 2 + c) * 4u, p));
              su[0] += __int_as_float(w.x); su[1] += __int_as_float(w.y);
              su[2] += __int_as_float(w.z); su[3] += __int_as_float(w.w);
            }
          }
        }
        const int64_t row = (int64_t)tm * BM + r, col0 = (int64_t)tn * out_cols + c;
        if (col0 >= a.n) continue;
        __align__(8) __nv_bfloat16 out[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t col = col0 + j < a.n ? col0 + j : a.n - 1;
          if (a.paired) {
            const float gv = round_bf16(sg[j] * __ldg(a.scales + col));
            const float uv = round_bf16(su[j] * __ldg(a.scales_up + col));
            out[j] = __float2bfloat16_rn(round_bf16(silu_f32(gv)) * uv);
          } else {
            float v = sg[j] * __ldg(a.scales + col);
            if (a.bias) v = round_bf16(v) + round_bf16(__ldg(a.bias + col));
            out[j] = __float2bfloat16_rn(v);
          }
        }
        __nv_bfloat16* dst = a.y + row * a.n + col0;
        if (a.vec_store && col0 + 4 <= a.n) {
          *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(out);
        } else {
          for (int j = 0; j < 4 && col0 + j < a.n; ++j) dst[j] = out[j];
        }
      }
    }
    __syncwarp();
    cluster_sync_all();  // every peer has read this CTA's partial
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Tile::TMEM_COLS);
}

template <int HALVES, int BN>
static int tw_launch(TwGemmArgs& a, const __nv_bfloat16* x, const int8_t* codes, const int8_t* up_codes,
                     cudaStream_t s) {
  using Tile = TwTile<HALVES, BN>;
  auto kern = tc_w8a16_gemm_kernel<HALVES, BN>;
  const int smem_st = ensure_dynamic_smem((const void*)kern, Tile::SMEM, "tc w8a16 gemm");
  if (smem_st) return smem_st;
  const int wrows = a.paired ? BN / 2 : BN;
  int st = encode_map_2d(&a.map_x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.m, a.k, Tile::BM, TW_BKE,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (!st)
    st = encode_map_2d(&a.map_w, codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.n, a.k, wrows, TW_BKE,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  if (!st && a.paired)
    st = encode_map_2d(&a.map_u, up_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.n, a.k, wrows, TW_BKE,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  if (st) return st;
  a.tiles_m = (int)((a.m + Tile::BM - 1) / Tile::BM);
  a.tiles_n = (int)((a.n + wrows - 1) / wrows);
  const int64_t items = (int64_t)a.tiles_m * a.tiles_n * a.splits;
  if (items > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "tc w8a16 gemm: too many tiles");
  cudaError_t e;
  if (a.splits > 1) {
    // one work item per CTA, the splits of a tile as one cluster
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)items);
    cfg.blockDim = dim3(TW_THREADS);
    cfg.dynamicSmemBytes = Tile::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)a.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
  } else {
    const int grid = (int)std::min<int64_t>(items, num_sms());
    e = launch_kernel(kern, dim3(grid), dim3(TW_THREADS), Tile::SMEM, s, true, a);
  }
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "tc w8a16 gemm: launch: %s", cudaGetErrorString(e));
  return launch_status("tc w8a16 gemm");
}

// Clusters of `size` 128 x 128-tile CTAs that can be resident at once (0 if none).
static int tw_cluster_capacity(int size) {
  static int cached[TW_MAX_CLUSTER + 1] = {};
  static bool done[TW_MAX_CLUSTER + 1] = {};
  if (size < 2 || size > TW_MAX_CLUSTER) return 0;
  if (!done[size]) {
    using Tile = TwTile<1, 128>;
    auto kern = tc_w8a16_gemm_kernel<1, 128>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Tile::SMEM);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(size * 64));
    cfg.blockDim = dim3(TW_THREADS);
    cfg.dynamicSmemBytes = Tile::SMEM;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    cached[size] = n;
    done[size] = true;
  }
  return cached[size];
}

// Split-K plan for 128 x 128 tiles that leave most SMs idle: the largest cluster size (k
// ranges of at least 4 k blocks) whose clusters all fit on the GPU at once. 1 = no split.
static int tw_split_plan(int64_t m, int64_t n, int64_t k, bool paired) {
  const int64_t out_cols = paired ? 64 : 128;
  const int64_t tiles = ((m + 127) / 128) * ((n + out_cols - 1) / out_cols);
  const int64_t kblocks = (k + TW_BKE - 1) / TW_BKE;
  if (2 * tiles > num_sms() || kblocks < 8) return 1;
  int best = 1;
  for (int size = 2; size <= TW_MAX_CLUSTER && 4 * size <= kblocks; ++size)
    if (tiles <= tw_cluster_capacity(size)) best = size;
  return best;
}

// Whether the tensor-core path takes this problem: TMA needs 16-byte aligned bases and row
// strides (k % 16 for the int8 codes, which also covers the bf16 activations).
bool tc_w8a16_supported(const void* x, int64_t k, const int8_t* codes, const int8_t* up_codes) {
  return k % 16 == 0 && aligned(x, 16) && aligned(codes, 16) && (!up_codes || aligned(up_codes, 16));
}

// Launch the tensor-core W8A16 GEMM (see the file comment); the caller checked the shapes and
// tc_w8a16_supported(). up_codes non-null selects the paired SwiGLU epilogue (n outputs from
// n gate rows and n up rows).
int tc_w8a16_gemm(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                  const int8_t* up_codes, const float* up_scales, int64_t n, const float* bias, __nv_bfloat16* y,
                  cudaStream_t s) {
  TwGemmArgs a{};
  a.m = m;
  a.n = n;
  a.k = k;
  a.kblocks = (int)((k + TW_BKE - 1) / TW_BKE);
  a.paired = up_codes != nullptr;
  a.scales = scales;
  a.scales_up = up_scales;
  a.bias = a.paired ? nullptr : bias;
  a.y = y;
  a.vec_store = (n % 8) == 0 && aligned(y, 16);
  a.splits = 1;
  a.kb_per = a.kblocks;
  const int splits = tw_split_plan(m, n, k, a.paired);
  if (splits > 1) {
    a.kb_per = (a.kblocks + splits - 1) / splits;
    a.splits = (a.kblocks + a.kb_per - 1) / a.kb_per;  // no empty k range
    if (a.splits > 1) return tw_launch<1, 128>(a, x, codes, up_codes, s);
    a.kb_per = a.kblocks;
  }
  const int64_t sms = num_sms();
  const int64_t per_tile = a.paired ? 2 : 1;  // weight rows per output column
  auto tiles = [&](int bm, int bn) { return ((m + bm - 1) / bm) * ((n * per_tile + bn - 1) / bn); };
  if (m > 128 && tiles(256, 256) >= 2 * sms) return tw_launch<2, 256>(a, x, codes, up_codes, s);
  if (tiles(128, 256) >= sms) return tw_launch<1, 256>(a, x, codes, up_codes, s);
  return tw_launch<1, 128>(a, x, codes, up_codes, s);
}

// Greedy head on the tensor cores: packed[r] = max over columns < semantic of
// pack_argmax(x[r] . codes[col] * scales[col], col) (packed must start at 0; atomicMax), fp32
// logits optionally written. Same requirements as tc_w8a16_gemm.
int tc_w8a16_argmax(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                    int64_t n, int64_t semantic, float* logits, unsigned long long* packed, cudaStream_t s) {
  TwGemmArgs a{};
  a.m = m;
  a.n = n;
  a.k = k;
  a.kblocks = (int)((k + TW_BKE - 1) / TW_BKE);
  a.paired = false;
  a.scales = scales;
  a.packed = packed;
  a.logits = logits;
  a.semantic = semantic;
  a.splits = 1;
  a.kb_per = a.kblocks;
  const int64_t sms = num_sms();
  auto tiles = [&](int bm, int bn) { return ((m + bm - 1) / bm) * ((n + bn - 1) / bn); };
  if (m > 128 && tiles(256, 256) >= 2 * sms) return tw_launch<2, 256>(a, x, codes, nullptr, s);
  if (tiles(128, 256) >= sms) return tw_launch<1, 256>(a, x, codes, nullptr, s);
  return tw_launch<1, 128>(a, x, codes, nullptr, s);
}

int tc_w8a16_timeouts(unsigned* out) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tw_timeouts, sizeof(v));
  if (e == cudaSuccess && v) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_tw_timeouts, &zero, sizeof(zero));
  }
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "tensor-core status: %s", cudaGetErrorString(e));
  *out = v;
  return MRB_OK;
}

}  // namespace mrb
