// Prefill / large-batch W8A8 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// acc[m, n] = sum_k qx[m, k] * qw[n, k] exactly in int32 (kind::i8), then optionally
//   y[m, n] = side[m, n] + (float(acc) * act_scale[m]) * w_scale[n]   (left to right, fp32)
// which is the reference's W8A8 rescale (engine/kernels/w8a8.py:67-125), bit-identical for
// every accumulator because the accumulation is exact.
//
// Design: one persistent CTA per SM walks output tiles with the M tiles of one N tile
// adjacent in the walk, so CTAs running together share the weight tile in L2. A tile is
// HALVES 128-row accumulators x BN weight rows (256x256, 128x256 or 128x128, chosen by how
// well the tiles fill the SMs): two halves share every weight stage, which halves the weight
// bytes each CTA pulls from L2 per multiply-add (large problems are L2-bandwidth-bound with
// 128-row tiles); smaller tiles keep more SMs busy on small problems.
//  * warp 0, one thread: TMA producer. Each stage is a [BM x 128 B] activation box and a
//    [BN x 128 B] weight box with the 128-byte swizzle; 3 to 6 stages (192 KB) in flight.
//  * warp 1: allocates the TMEM accumulators (double-buffered for single-half tiles); one
//    thread issues tcgen05.mma (M=128, N=BN, K=32) and commits each stage back to the
//    producer and each finished tile to the epilogue.
//  * warps 2-5: epilogue. Each warp owns the 32 TMEM lanes (tile rows) its index selects,
//    loads 32 columns at a time with tcgen05.ld, rescales and stores, then releases the
//    accumulators to the MMA thread.
// Engine outputs: y_bf16 = bf16((float(acc)·s_x)·s_w + bias), or, with paired gate/up weight
// pages (a B tile of BN/2 gate rows then the same BN/2 up rows), the SwiGLU
// bf16(bf16(silu(bf16 g))·bf16 u) of the two rescaled accumulators.
// Split-K (skinny activation blocks, e.g. 64-row W8A8 decode, whose output tiles fill few
// SMs; bf16 outputs): the k ranges of one output tile run as the CTAs of one thread-block
// cluster. Each parks its int32 partial tile in its own shared memory (the stage ring is idle
// by then); after a cluster barrier every CTA sums one column slice of the tile over all the
// cluster's partials through distributed shared memory and writes those outputs; a second
// barrier keeps the partials alive until every peer has read them. int32 addition is exact,
// so the result does not depend on the split.
// Every wait is bounded: on a timeout the CTA records the failure, stops, and still frees
// its TMEM. No load uses cluster multicast.
#include "qrow_common.cuh"
#include "tc_common.cuh"

#include <algorithm>

namespace mrb {

constexpr int TC_HM = 128;             // MMA M (rows of one accumulator)
constexpr int TC_BK = 128;             // bytes of k per stage: one 128-byte swizzle row
constexpr int TC_UK = 32;              // k per MMA (kind::i8)
constexpr int TC_THREADS = 192;        // warp 0 TMA, warp 1 MMA + TMEM owner, warps 2-5 epilogue
constexpr int TC_EPI_THREADS = 128;
constexpr size_t TC_RING_BUDGET = 192 * 1024;

// Tile shape: HALVES 128-row accumulators (sharing each weight stage) x BN weight rows.
template <int HALVES, int BN>
struct TcTile {
  static constexpr int BM = TC_HM * HALVES;
  static constexpr int A_BYTES = BM * TC_BK;
  static constexpr int B_BYTES = BN * TC_BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (int)(TC_RING_BUDGET / STAGE_BYTES) < 6 ? (int)(TC_RING_BUDGET / STAGE_BYTES) : 6;
  static constexpr int NBUF = HALVES == 1 ? 2 : 1;  // accumulator sets (double-buffered when they fit)
  static constexpr unsigned TMEM_COLS = HALVES * BN * NBUF <= 256 ? 256u : 512u;
  static constexpr size_t SCALE_BYTES = 4 * 2 * BN * sizeof(float);  // per epilogue warp: [BN] + [BN]
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256 + SCALE_BYTES;
  static constexpr int PSTRIDE = BN + 4;  // int32 row stride of a parked partial (bank spread)
  static_assert((size_t)TC_HM * PSTRIDE * 4 <= (size_t)STAGES * STAGE_BYTES, "partial tile exceeds the ring");
};
constexpr int TC_MAX_CLUSTER = 8;

struct TcGemmArgs {
  CUtensorMap map_x;  // qx [m, k] int8, box [BM rows, 128 B], 128-byte swizzle
  CUtensorMap map_w;  // qw [n, k] int8, box [BN (paired: BN/2) rows, 128 B], 128-byte swizzle
  CUtensorMap map_u;  // paired: up codes [n, k] int8, box [BN/2 rows, 128 B]
  int64_t m, n, k;    // n: output columns
  int tiles_m, tiles_n, kblocks;
  bool paired;
  const float* act_scale;  // [m] or null (then y / y_bf16 are not written)
  const float* sw;         // [n]
  const float* sw_up;      // [n] (paired)
  const float* side;       // [m, n] or null (fp32 output only)
  const float* bias;       // [n] or null (bf16 output only), added in fp32
  float* y;                // [m, n] or null
  __nv_bfloat16* y_bf16;   // [m, n] or null
  int32_t* acc_out;        // [m, n] or null (not paired)
  bool vec_store;          // 16-byte aligned outputs with n % 4 == 0 (n % 8 for bf16)
  int splits, kb_per;      // split-K: k blocks [split * kb_per, +kb_per); splits > 1 = cluster of splits CTAs
};

// Timed-out waits of the tensor-core GEMM since the last status read (0 in normal operation).
__device__ unsigned g_tc_timeouts = 0;

template <int HALVES, int BN>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_int8_gemm_kernel(const __grid_constant__ TcGemmArgs a) {
  using Tile = TcTile<HALVES, BN>;
  constexpr int STAGES = Tile::STAGES, NBUF = Tile::NBUF, BM = Tile::BM;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Tile::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + NBUF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* scale_smem = reinterpret_cast<float*>(smem + STAGES * Tile::STAGE_BYTES + 256);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, TC_EPI_THREADS);
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
    atomicAdd(&g_tc_timeouts, 1u);
  };
  // accumulator of half h in buffer b
  auto acc_col = [&](int b, int h) { return (uint32_t)((b * HALVES + h) * BN); };

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      pdl_wait();  // the quantised activations come from the previous kernel
      int stage = 0;
      unsigned phase = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int t = it / a.splits;
        const int tm = t % a.tiles_m, tn = t / a.tiles_m;
        const int kb0 = (it % a.splits) * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(empty + stage, phase ^ 1u)) {
            fail_wait();
            break;
          }
          unsigned char* st = smem + stage * Tile::STAGE_BYTES;
          mbar_arrive_expect_tx(full + stage, Tile::STAGE_BYTES);
          tma_load_2d(st, &a.map_x, kb * TC_BK, tm * BM, full + stage);
          if (a.paired) {
            tma_load_2d(st + Tile::A_BYTES, &a.map_w, kb * TC_BK, tn * (BN / 2), full + stage);
            tma_load_2d(st + Tile::A_BYTES + (BN / 2) * TC_BK, &a.map_u, kb * TC_BK, tn * (BN / 2), full + stage);
          } else {
            tma_load_2d(st + Tile::A_BYTES, &a.map_w, kb * TC_BK, tn * BN, full + stage);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(UMMA_D_S32, UMMA_S8, UMMA_S8, TC_HM, BN);
      int stage = 0, buf = 0;
      unsigned phase = 0, acc_phase = 0;
      for (int it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
        const int t = it / a.splits;
        const int kb0 = (it % a.splits) * a.kb_per, kb1 = min(a.kblocks, kb0 + a.kb_per);
        if (!mbar_wait_bounded(acc_empty + buf, acc_phase ^ 1u)) {
          fail_wait();
          break;
        }
        tc_fence_after();
        // halves beyond the last activation row are skipped (their rows are all zero)
        int halves = HALVES;
        while (halves > 1 && (int64_t)(t % a.tiles_m) * BM + (halves - 1) * TC_HM >= a.m) --halves;
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(full + stage, phase)) {
            fail_wait();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Tile::STAGE_BYTES);
          const uint32_t sb = sa + Tile::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < TC_BK / TC_UK; ++kk) {
            const uint64_t db = umma_desc_k_sw128(sb + kk * TC_UK);
#pragma unroll
            for (int h = 0; h < HALVES; ++h)
              if (h < halves)
                umma_i8(tmem + acc_col(buf, h), umma_desc_k_sw128(sa + h * TC_HM * TC_BK + kk * TC_UK), db, idesc,
                        kb > kb0 || kk > 0);
          }
          umma_commit(empty + stage);  // the stage is free once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(acc_full + buf);  // accumulators complete
        if (++buf == NBUF) {
          buf = 0;
          acc_phase ^= 1u;
        }
      }
    }
  } else {
    // ---------------- epilogue: TMEM -> registers -> global
    pdl_wait();  // act_scale and side come from earlier kernels
    const int q = warp & 3;  // TMEM lane quarter of this warp
    int buf = 0;
    unsigned acc_phase = 0;
    const bool vec = a.vec_store;
    const int out_cols = a.paired ? BN / 2 : BN;
    // this warp's copy of the tile's column scales: [BN] weight scales, [BN] up scales (paired)
    // or bias; loaded in one batch per tile so the epilogue never waits on them one by one
    float* sc = scale_smem + q * 2 * BN;
    auto stage_scales = [&](int tn) {
      float g[BN / 32], u[BN / 32];
#pragma unroll
      for (int i = 0; i < BN / 32; ++i) {
        const int c = lane + 32 * i;
        const int64_t col = (int64_t)tn * out_cols + c;
        const bool ok = c < out_cols && col < a.n;
        g[i] = (ok && a.sw) ? __ldg(a.sw + col) : 0.f;
        u[i] = !ok ? 0.f : a.paired ? __ldg(a.sw_up + col) : (a.bias ? __ldg(a.bias + col) : 0.f);
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < BN / 32; ++i) {
        sc[lane + 32 * i] = g[i];
        sc[BN + lane + 32 * i] = u[i];
      }
      __syncwarp();
    };
    // 32 output columns from int32 accumulators v (gate or plain) and u (up, paired); c0 is
    // the tile-local output column, col0 the global one
    auto emit = [&](int64_t row, float as, int c0, int64_t col0, const uint32_t (&v)[32], const uint32_t (&u)[32]) {
      const int64_t o0 = row * a.n + col0;
      const bool full_run = vec && col0 + 32 <= a.n;
      if (a.acc_out) {
        if (full_run) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<int4*>(a.acc_out + o0 + j) =
                make_int4((int)v[j], (int)v[j + 1], (int)v[j + 2], (int)v[j + 3]);
        } else {
          for (int j = 0; j < 32 && col0 + j < a.n; ++j) a.acc_out[o0 + j] = (int)v[j];
        }
      }
      if (!a.act_scale) return;
      if (a.y) {
        float out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float r = __fmul_rn(__fmul_rn(__int2float_rn((int)v[j]), as), sc[c0 + j]);
          if (a.side && col0 + j < a.n) r = __fadd_rn(a.side[o0 + j], r);
          out[j] = r;
        }
        if (full_run) {
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(a.y + o0 + j) = make_float4(out[j], out[j + 1], out[j + 2], out[j + 3]);
        } else {
          for (int j = 0; j < 32 && col0 + j < a.n; ++j) a.y[o0 + j] = out[j];
        }
      }
      if (a.y_bf16) {
        __align__(16) __nv_bfloat16 out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float g = __fmul_rn(__fmul_rn(__int2float_rn((int)v[j]), as), sc[c0 + j]);
          if (a.paired) {
            const float up = __fmul_rn(__fmul_rn(__int2float_rn((int)u[j]), as), sc[BN + c0 + j]);
            const float gv = round_bf16(g), uv = round_bf16(up);
            out[j] = __float2bfloat16_rn(round_bf16(silu_f32(gv)) * uv);
          } else {
            out[j] = __float2bfloat16_rn(a.bias ? __fadd_rn(g, sc[BN + c0 + j]) : g);
          }
        }
        __nv_bfloat16* dst = a.y_bf16 + o0;
        if (full_run) {
#pragma unroll
          for (int j = 0; j < 32; j += 8)
            *reinterpret_cast<uint4*>(dst + j) = *reinterpret_cast<const uint4*>(out + j);
        } else {
          for (int j = 0; j < 32 && col0 + j < a.n; ++j) dst[j] = out[j];
        }
      }
    };
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
      const int t = it / a.splits;
      // warp-uniform: tcgen05.ld below is a whole-warp instruction
      bool ok = !*abort_flag && mbar_wait_bounded(acc_full + buf, acc_phase);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !*abort_flag) fail_wait();
        break;
      }
      tc_fence_after();
      const int tm = t % a.tiles_m, tn = t / a.tiles_m;
      if (a.splits == 1) {
        stage_scales(tn);
        for (int h = 0; h < HALVES; ++h) {
          if ((int64_t)tm * BM + h * TC_HM >= a.m) break;  // uniform: an empty half
          const int64_t row = (int64_t)tm * BM + h * TC_HM + q * 32 + lane;
          const bool row_ok = row < a.m;
          const float as = (row_ok && a.act_scale) ? a.act_scale[row] : 0.f;
          const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + acc_col(buf, h);
          for (int c0 = 0; c0 < out_cols; c0 += 32) {
            uint32_t v[32], u[32];
            __syncwarp();
            tmem_ld_32cols(tbase + (uint32_t)c0, v);
            if (a.paired) tmem_ld_32cols(tbase + (uint32_t)(BN / 2 + c0), u);
            const int64_t col0 = (int64_t)tn * out_cols + c0;
            if (!row_ok || col0 >= a.n) continue;
            emit(row, as, c0, col0, v, u);
          }
        }
      } else {
        // cluster split-K (one work item per CTA, single-half tiles): park this k range's
        // int32 partial in shared memory for the reduction after the role loops
        int32_t* part = reinterpret_cast<int32_t*>(smem) + (q * 32 + lane) * Tile::PSTRIDE;
        const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + acc_col(buf, 0);
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32cols(tbase + (uint32_t)c0, v);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<int4*>(part + c0 + j) = make_int4((int)v[j], (int)v[j + 1], (int)v[j + 2], (int)v[j + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty + buf);  // accumulators drained
      if (++buf == NBUF) {
        buf = 0;
        acc_phase ^= 1u;
      }
    }
  }

  if (a.splits > 1) {
    // ---------------- cluster split-K reduction (every thread takes part in both barriers)
    __syncwarp();
    cluster_sync_all();  // every CTA of the cluster has parked its partial tile
    if (warp >= 2 && a.act_scale && a.y_bf16) {
      const unsigned nsplit = (unsigned)a.splits, rank = cluster_ctarank();
      const int t = blockIdx.x / a.splits;
      const int tm = t % a.tiles_m, tn = t / a.tiles_m;
      const int out_cols = a.paired ? BN / 2 : BN;
      const int groups = out_cols / 4;  // 4-column output groups; this CTA reduces [g0, g1)
      const int g0 = (int)(rank * groups / nsplit), g1 = (int)((rank + 1) * groups / nsplit), ng = g1 - g0;
      const int64_t rows_left = a.m - (int64_t)tm * BM;
      const int rows = rows_left < BM ? (int)rows_left : BM;
      const uint32_t base = smem_u32(smem);
      for (int unit = tid - 64; unit < rows * ng; unit += TC_EPI_THREADS) {
        const int r = unit / ng, c = (g0 + unit % ng) * 4;  // tile row, tile-local output column
        int4 sg = make_int4(0, 0, 0, 0), su = make_int4(0, 0, 0, 0);
#pragma unroll
        for (unsigned p = 0; p < (unsigned)TC_MAX_CLUSTER; ++p) {
          if (p < nsplit) {
            const int4 g = ld_shared_cluster_v4(mapa_shared(base + (uint32_t)(r * Tile::PSTRIDE + c) * 4u, p));
            sg.x += g.x; sg.y += g.y; sg.z += g.z; sg.w += g.w;
            if (a.paired) {
              const int4 w =
                  ld_shared_cluster_v4(mapa_shared(base + (uint32_t)(r * Tile::PSTRIDE + BN / 2 + c) * 4u, p));
              su.x += w.x; su.y += w.y; su.z += w.z; su.w += w.w;
            }
          }
        }
        const int64_t row = (int64_t)tm * BM + r, col0 = (int64_t)tn * out_cols + c;
        if (col0 >= a.n) continue;
        const float as = a.act_scale[row];
        const int gv4[4] = {sg.x, sg.y, sg.z, sg.w}, uv4[4] = {su.x, su.y, su.z, su.w};
        __align__(8) __nv_bfloat16 out[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int64_t col = col0 + j < a.n ? col0 + j : a.n - 1;
          const float g = __fmul_rn(__fmul_rn(__int2float_rn(gv4[j]), as), __ldg(a.sw + col));
          if (a.paired) {
            const float up = __fmul_rn(__fmul_rn(__int2float_rn(uv4[j]), as), __ldg(a.sw_up + col));
            const float gr = round_bf16(g), ur = round_bf16(up);
            out[j] = __float2bfloat16_rn(round_bf16(silu_f32(gr)) * ur);
          } else {
            out[j] = __float2bfloat16_rn(a.bias ? __fadd_rn(g, __ldg(a.bias + col)) : g);
          }
        }
        __nv_bfloat16* dst = a.y_bf16 + row * a.n + col0;
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
static int tc_launch(TcGemmArgs& a, const int8_t* qx, const int8_t* qw, const int8_t* qw_up, cudaStream_t s) {
  using Tile = TcTile<HALVES, BN>;
  auto kern = tc_int8_gemm_kernel<HALVES, BN>;
  const int smem_st = ensure_dynamic_smem((const void*)kern, Tile::SMEM, "tc int8 gemm");
  if (smem_st) return smem_st;
  int st = encode_map_2d(&a.map_x, qx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.m, a.k, Tile::BM, TC_BK,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  const int wrows = a.paired ? BN / 2 : BN;
  if (!st)
    st = encode_map_2d(&a.map_w, qw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.n, a.k, wrows, TC_BK,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (!st && a.paired)
    st = encode_map_2d(&a.map_u, qw_up, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.n, a.k, wrows, TC_BK,
                       CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  a.tiles_m = (int)((a.m + Tile::BM - 1) / Tile::BM);
  a.tiles_n = (int)((a.n + wrows - 1) / wrows);
  const int64_t items = (int64_t)a.tiles_m * a.tiles_n * a.splits;
  if (items > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "tc int8 gemm: too many tiles");
  cudaError_t e;
  if (a.splits > 1) {
    // one work item per CTA, the splits of a tile as one cluster
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)items);
    cfg.blockDim = dim3(TC_THREADS);
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
    e = launch_kernel(kern, dim3(grid), dim3(TC_THREADS), Tile::SMEM, s, true, a);
  }
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "tc int8 gemm: launch: %s", cudaGetErrorString(e));
  return launch_status("tc int8 gemm");
}

// Clusters of `size` 128 x 128-tile CTAs that can be resident at once (0 if none).
static int tc_cluster_capacity(int size) {
  static int cached[TC_MAX_CLUSTER + 1] = {};
  static bool done[TC_MAX_CLUSTER + 1] = {};
  if (size < 2 || size > TC_MAX_CLUSTER) return 0;
  if (!done[size]) {
    using Tile = TcTile<1, 128>;
    auto kern = tc_int8_gemm_kernel<1, 128>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Tile::SMEM);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(size * 64));
    cfg.blockDim = dim3(TC_THREADS);
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

// Split-K plan for a problem whose 128 x 128 output tiles leave most SMs idle: the largest
// cluster size (k ranges per tile, at least 4 k blocks each) whose clusters all fit on the
// GPU at once. 1 = no split.
static int tc_split_plan(int64_t m, int64_t n, int64_t k, bool paired) {
  const int64_t out_cols = paired ? 64 : 128;
  const int64_t tiles = ((m + 127) / 128) * ((n + out_cols - 1) / out_cols);
  const int64_t kblocks = (k + TC_BK - 1) / TC_BK;
  if (2 * tiles > num_sms() || kblocks < 8) return 1;
  int best = 1;
  for (int size = 2; size <= TC_MAX_CLUSTER && 4 * size <= kblocks; ++size)
    if (tiles <= tc_cluster_capacity(size)) best = size;
  return best;
}

// Launch the tensor-core W8A8 GEMM (see the file comment); arguments are checked by callers.
// Tile shape by SM fill: 256-row tiles when they give every SM at least two, else 128 x 256
// double-buffered tiles when those fill the SMs, else 128 x 128 — split over k in clusters
// when those leave most SMs idle and the only output is y_bf16.
// qw_up non-null: paired gate/up pages (n outputs, SwiGLU epilogue, y_bf16 only).
int tc_int8_gemm_ex(const int8_t* qx, const int8_t* qw, const int8_t* qw_up, int64_t m, int64_t n, int64_t k,
                    const float* act_scale, const float* sw, const float* sw_up, const float* side,
                    const float* bias, float* y, __nv_bfloat16* y_bf16, int32_t* acc_out, cudaStream_t s) {
  TcGemmArgs a{};
  a.m = m;
  a.n = n;
  a.k = k;
  a.kblocks = (int)((k + TC_BK - 1) / TC_BK);
  a.paired = qw_up != nullptr;
  a.act_scale = act_scale;
  a.sw = sw;
  a.sw_up = sw_up;
  a.side = side;
  a.bias = bias;
  a.y = y;
  a.y_bf16 = y_bf16;
  a.acc_out = acc_out;
  a.vec_store = (n % 8) == 0 && (!y || aligned(y, 16)) && (!acc_out || aligned(acc_out, 16)) &&
                (!y_bf16 || aligned(y_bf16, 16));
  a.splits = 1;
  a.kb_per = a.kblocks;
  const int splits = (y_bf16 && act_scale && !y && !acc_out) ? tc_split_plan(m, n, k, a.paired) : 1;
  if (splits > 1) {
    a.kb_per = (a.kblocks + splits - 1) / splits;
    a.splits = (a.kblocks + a.kb_per - 1) / a.kb_per;  // no empty k range
    if (a.splits > 1) return tc_launch<1, 128>(a, qx, qw, qw_up, s);
    a.kb_per = a.kblocks;
  }
  const int64_t sms = num_sms();
  const int64_t wr = a.paired ? 2 : 1;  // weight rows per output column
  auto ntiles = [&](int bm, int bn) { return ((m + bm - 1) / bm) * ((n * wr + bn - 1) / bn); };
  if (m > 128 && ntiles(256, 256) >= 2 * sms) return tc_launch<2, 256>(a, qx, qw, qw_up, s);
  if (ntiles(128, 256) >= sms) return tc_launch<1, 256>(a, qx, qw, qw_up, s);
  return tc_launch<1, 128>(a, qx, qw, qw_up, s);
}

int tc_int8_gemm(const int8_t* qx, const int8_t* qw, int64_t m, int64_t n, int64_t k, const float* act_scale,
                 const float* sw, const float* side, float* y, int32_t* acc_out, cudaStream_t s) {
  return tc_int8_gemm_ex(qx, qw, nullptr, m, n, k, act_scale, sw, nullptr, side, nullptr, y, nullptr, acc_out, s);
}

// Read and reset the count of timed-out waits (synchronises the device).
int tc_gemm_timeouts(unsigned* out) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_timeouts, sizeof(v));
  if (e == cudaSuccess && v) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_tc_timeouts, &zero, sizeof(zero));
  }
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "tensor-core status: %s", cudaGetErrorString(e));
  *out = v;
  return MRB_OK;
}

}  // namespace mrb

namespace mrb {
int tc_w8a16_timeouts(unsigned* out);
}

extern "C" int mrb_tc_status(unsigned* timeouts) {
  if (!timeouts) return mrb::fail(MRB_ERR_ARG, "tc_status: null pointer");
  unsigned a = 0, b = 0;
  int st = mrb::tc_gemm_timeouts(&a);
  if (!st) st = mrb::tc_w8a16_timeouts(&b);
  if (st) return st;
  *timeouts = a + b;
  return MRB_OK;
}
