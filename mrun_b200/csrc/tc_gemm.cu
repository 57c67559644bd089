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
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 256;
};

struct TcGemmArgs {
  CUtensorMap map_x;  // qx [m, k] int8, box [BM rows, 128 B], 128-byte swizzle
  CUtensorMap map_w;  // qw [n, k] int8, box [BN rows, 128 B], 128-byte swizzle
  int64_t m, n, k;
  int tiles_m, tiles_n, kblocks;
  const float* act_scale;  // [m] or null (then y is not written)
  const float* sw;         // [n]
  const float* side;       // [m, n] or null
  float* y;                // [m, n] or null
  int32_t* acc_out;        // [m, n] or null
  bool vec_store;          // n % 4 == 0 and 16-byte aligned outputs: 16-byte stores
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
      for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x) {
        const int tm = t % a.tiles_m, tn = t / a.tiles_m;
        for (int kb = 0; kb < a.kblocks; ++kb) {
          if (!mbar_wait_bounded(empty + stage, phase ^ 1u)) {
            fail_wait();
            break;
          }
          unsigned char* st = smem + stage * Tile::STAGE_BYTES;
          mbar_arrive_expect_tx(full + stage, Tile::STAGE_BYTES);
          tma_load_2d(st, &a.map_x, kb * TC_BK, tm * BM, full + stage);
          tma_load_2d(st + Tile::A_BYTES, &a.map_w, kb * TC_BK, tn * BN, full + stage);
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
      for (int t = blockIdx.x; t < ntiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait_bounded(acc_empty + buf, acc_phase ^ 1u)) {
          fail_wait();
          break;
        }
        tc_fence_after();
        // halves beyond the last activation row are skipped (their rows are all zero)
        int halves = HALVES;
        while (halves > 1 && (int64_t)(t % a.tiles_m) * BM + (halves - 1) * TC_HM >= a.m) --halves;
        bool ok = true;
        for (int kb = 0; kb < a.kblocks; ++kb) {
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
                        kb > 0 || kk > 0);
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
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      // warp-uniform: tcgen05.ld below is a whole-warp instruction
      bool ok = !*abort_flag && mbar_wait_bounded(acc_full + buf, acc_phase);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !*abort_flag) fail_wait();
        break;
      }
      tc_fence_after();
      const int tm = t % a.tiles_m, tn = t / a.tiles_m;
      for (int h = 0; h < HALVES; ++h) {
        if ((int64_t)tm * BM + h * TC_HM >= a.m) break;  // uniform: an empty half
        const int64_t row = (int64_t)tm * BM + h * TC_HM + q * 32 + lane;
        const bool row_ok = row < a.m;
        const float as = (row_ok && a.act_scale) ? a.act_scale[row] : 0.f;
        for (int c0 = 0; c0 < BN; c0 += 32) {
          uint32_t v[32];
          __syncwarp();
          tmem_ld_32cols(tmem + ((uint32_t)(q * 32) << 16) + acc_col(buf, h) + (uint32_t)c0, v);
          const int64_t col0 = (int64_t)tn * BN + c0;
          if (!row_ok || col0 >= a.n) continue;
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
          if (a.y && a.act_scale) {
            float out[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int64_t col = col0 + j;
              const float wsc = col < a.n ? a.sw[col] : 0.f;
              float r = __fmul_rn(__fmul_rn(__int2float_rn((int)v[j]), as), wsc);
              if (a.side && col < a.n) r = __fadd_rn(a.side[o0 + j], r);
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

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Tile::TMEM_COLS);
}

template <int HALVES, int BN>
static int tc_launch(TcGemmArgs& a, const int8_t* qx, const int8_t* qw, cudaStream_t s) {
  using Tile = TcTile<HALVES, BN>;
  auto kern = tc_int8_gemm_kernel<HALVES, BN>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Tile::SMEM);
    if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "tc int8 gemm: smem attribute: %s", cudaGetErrorString(e));
    configured = true;
  }
  int st = encode_map_2d(&a.map_x, qx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.m, a.k, Tile::BM, TC_BK,
                         CU_TENSOR_MAP_SWIZZLE_128B);
  if (!st)
    st = encode_map_2d(&a.map_w, qw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.n, a.k, BN, TC_BK, CU_TENSOR_MAP_SWIZZLE_128B);
  if (st) return st;
  a.tiles_m = (int)((a.m + Tile::BM - 1) / Tile::BM);
  a.tiles_n = (int)((a.n + BN - 1) / BN);
  const int64_t ntiles = (int64_t)a.tiles_m * a.tiles_n;
  if (ntiles > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "tc int8 gemm: too many tiles");
  const int grid = (int)std::min<int64_t>(ntiles, num_sms());
  cudaError_t e = launch_kernel(kern, dim3(grid), dim3(TC_THREADS), Tile::SMEM, s, true, a);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "tc int8 gemm: launch: %s", cudaGetErrorString(e));
  return launch_status("tc int8 gemm");
}

// Launch the tensor-core W8A8 GEMM (see the file comment); arguments are checked by callers.
// Tile shape by SM fill: 256-row tiles when they give every SM at least two, else 128 x 256
// double-buffered tiles when those fill the SMs, else 128 x 128.
int tc_int8_gemm(const int8_t* qx, const int8_t* qw, int64_t m, int64_t n, int64_t k, const float* act_scale,
                 const float* sw, const float* side, float* y, int32_t* acc_out, cudaStream_t s) {
  TcGemmArgs a{};
  a.m = m;
  a.n = n;
  a.k = k;
  a.kblocks = (int)((k + TC_BK - 1) / TC_BK);
  a.act_scale = act_scale;
  a.sw = sw;
  a.side = side;
  a.y = y;
  a.acc_out = acc_out;
  a.vec_store = (n % 4) == 0 && (!y || aligned(y, 16)) && (!acc_out || aligned(acc_out, 16));
  const int64_t sms = num_sms();
  auto tiles = [&](int bm, int bn) { return ((m + bm - 1) / bm) * ((n + bn - 1) / bn); };
  if (tiles(256, 256) >= 2 * sms) return tc_launch<2, 256>(a, qx, qw, s);
  if (tiles(128, 256) >= sms) return tc_launch<1, 256>(a, qx, qw, s);
  return tc_launch<1, 128>(a, qx, qw, s);
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

extern "C" int mrb_tc_status(unsigned* timeouts) {
  if (!timeouts) return mrb::fail(MRB_ERR_ARG, "tc_status: null pointer");
  return mrb::tc_gemm_timeouts(timeouts);
}
