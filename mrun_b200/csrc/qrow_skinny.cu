// Skinny W8A16 projection for decode batches of 17-32 activation rows.
//
// y[m, n] = bf16(scale[n] * sum_k x[m, k] * code[n, k]) (+ bf16 bias, rounded again), bf16
// activations, int8 codes, fp32 accumulation -- the contract of mrb_qrow_matmul.
//
// At these row counts the weight stream is the whole cost (qkv of the config-4 decoder:
// 10.5 MB for 32 x 5120 x 2048), but neither the 16-row GEMV (it stages every activation row
// per CTA as scaled f16) nor the tcgen05 GEMM (128-row activation tiles, three quarters
// padding) reaches it. Here:
//  * a CTA owns 128 weight rows (8 warps x 16) and one K range; the K ranges of a row group
//    form a thread-block cluster and their fp32 partials are summed in rank order through
//    distributed shared memory (deterministic for a given shape);
//  * each warp streams its 16 rows straight into registers with 16-byte loads, the first
//    blocks requested before the programmatic-dependent-launch wait (weights do not depend
//    on the previous kernel), so a CTA has its whole K range of weights in flight early;
//  * codes become bf16 exactly with integer ops (the low 7 bits into the mantissa of 128.0,
//    then 128 or 256 subtracted according to the sign bit), so the activations are used as
//    they are: the CTA's 32 rows of its K range are staged once in shared memory (rows
//    padded for conflict-free 16-byte reads) and feed mma.sync m16n8k16 bf16 as four 8-row
//    B tiles;
//  * inside each 64-wide k block the k order is permuted identically for weights and
//    activations (lane c of a quad takes bytes [16c, 16c + 16) of its rows; k step ks uses
//    bytes 16c + 4ks .. + 3), so every load is 16 bytes wide and no shuffles are needed.
#include "qrow_common.cuh"
#include "tc_common.cuh"

#include <algorithm>

namespace mrb {

constexpr int SK_WARPS = 8;
constexpr int SK_THREADS = SK_WARPS * 32;
constexpr int SK_ROWS = SK_WARPS * 16;  // weight rows per CTA
constexpr int SK_M = 32;                // activation rows (four n8 tiles)
constexpr int SK_KB = 64;               // k per block
constexpr int SK_MAXB = 16;             // k blocks per CTA at most (staged activations <= 64 KB)
constexpr int SK_PF = 4;                // k blocks of weights in flight per warp
constexpr int SK_PSTRIDE = SK_M + 1;    // fp32 row stride of a parked partial (bank spread)
constexpr int SK_MAX_CLUSTER = 8;

struct SkinnyArgs {
  const __nv_bfloat16* x;  // [m, k]
  int64_t m, n, k;
  const int8_t* codes;     // [n, k]
  const float* scales;     // [n]
  const float* bias;       // [n] or null
  __nv_bfloat16* y;        // [m, n]
  int splits;              // cluster size: K ranges per row group
  int nbk;                 // k blocks in all
  int xstride;             // staged activation row stride, bf16 elements
};

__host__ __device__ inline int sk_xstride(int blocks) { return blocks * SK_KB + 8; }  // + 16 bytes
__host__ inline size_t sk_smem_bytes(int blocks) {
  const size_t xs = (size_t)SK_M * sk_xstride(blocks) * 2;
  const size_t part = (size_t)SK_ROWS * SK_PSTRIDE * 4;
  return xs > part ? xs : part;
}

__global__ void __launch_bounds__(SK_THREADS, 2) qrow_skinny_kernel(const __grid_constant__ SkinnyArgs a) {
  extern __shared__ __align__(16) unsigned char sk_smem[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(sk_smem);
  float* part = reinterpret_cast<float*>(sk_smem);
  const int S = a.splits;
  const int rank = (int)(blockIdx.x % (unsigned)S);
  const int64_t group = blockIdx.x / S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int b_lo = (int)((int64_t)rank * a.nbk / S), b_hi = (int)((int64_t)(rank + 1) * a.nbk / S);
  const int nb = b_hi - b_lo;
  const int64_t K = a.k;

  // ---- this warp's weight rows (rows past n read row n - 1 and are dropped at the end)
  const int64_t r0 = min(group * SK_ROWS + warp * 16 + g, a.n - 1);
  const int64_t r1 = min(group * SK_ROWS + warp * 16 + g + 8, a.n - 1);
  const int8_t* w0 = a.codes + r0 * K + (int64_t)b_lo * SK_KB + 16 * c;
  const int8_t* w1 = a.codes + r1 * K + (int64_t)b_lo * SK_KB + 16 * c;
  auto load_w = [&](int b, uint4& u0, uint4& u1) {
    const int64_t koff = (int64_t)b * SK_KB;
    const bool ok = b < nb && (int64_t)(b_lo + b) * SK_KB + 16 * c + 16 <= K;  // whole 16-byte chunks
    u0 = ok ? __ldcs(reinterpret_cast<const uint4*>(w0 + koff)) : make_uint4(0u, 0u, 0u, 0u);
    u1 = ok ? __ldcs(reinterpret_cast<const uint4*>(w1 + koff)) : make_uint4(0u, 0u, 0u, 0u);
  };
  uint4 wb[SK_PF][2];
#pragma unroll
  for (int p = 0; p < SK_PF; ++p) load_w(p, wb[p][0], wb[p][1]);

  pdl_launch_dependents();
  pdl_wait();  // the activations come from the previous kernel

  // ---- stage the CTA's activation rows for its K range (rows past m and k past K are zero)
  const int xst = a.xstride;
  const int vpr = nb * (SK_KB / 8);  // 16-byte vectors per staged row
  for (int idx = tid; idx < SK_M * vpr; idx += SK_THREADS) {
    const int r = idx / vpr, v = idx - r * vpr;
    const int64_t kk = (int64_t)b_lo * SK_KB + (int64_t)v * 8;
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (r < a.m && kk + 8 <= K) val = __ldg(reinterpret_cast<const uint4*>(a.x + (int64_t)r * K + kk));
    *reinterpret_cast<uint4*>(xs + r * xst + v * 8) = val;
  }
  __syncthreads();

  // ---- k blocks: weights from registers, activations from shared memory
  float acc[4][4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  for (int b0 = 0; b0 < nb; b0 += SK_PF) {
#pragma unroll
    for (int p = 0; p < SK_PF; ++p) {
      const int b = b0 + p;
      if (b < nb) {
        const uint32_t wr0[4] = {wb[p][0].x, wb[p][0].y, wb[p][0].z, wb[p][0].w};
        const uint32_t wr1[4] = {wb[p][1].x, wb[p][1].y, wb[p][1].z, wb[p][1].w};
        load_w(b + SK_PF, wb[p][0], wb[p][1]);  // this register slot's next block
        // activations of rows nt*8 + g: k = 16c .. 16c + 15 of block b (32 bytes)
        uint4 xv[4][2];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const uint4* xp = reinterpret_cast<const uint4*>(xs + (nt * 8 + g) * xst + b * SK_KB + 16 * c);
          xv[nt][0] = xp[0];
          xv[nt][1] = xp[1];
        }
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          uint32_t a0, a2, a1, a3;
          i8x4_to_bf16x2_exact(wr0[ks], a0, a2);
          i8x4_to_bf16x2_exact(wr1[ks], a1, a3);
#pragma unroll
          for (int nt = 0; nt < 4; ++nt) {
            const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv[nt][ks >> 1]);
            mma_bf16(acc[nt], a0, a1, a2, a3, xw[(ks & 1) * 2], xw[(ks & 1) * 2 + 1]);
          }
        }
      }
    }
  }

  // ---- park the partial [128 rows x 32 activation rows], then sum the cluster's in rank order
  __syncthreads();  // every warp is done with the staged activations
  {
    const int row = warp * 16 + g;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      part[row * SK_PSTRIDE + nt * 8 + 2 * c] = acc[nt][0];
      part[row * SK_PSTRIDE + nt * 8 + 2 * c + 1] = acc[nt][1];
      part[(row + 8) * SK_PSTRIDE + nt * 8 + 2 * c] = acc[nt][2];
      part[(row + 8) * SK_PSTRIDE + nt * 8 + 2 * c + 1] = acc[nt][3];
    }
  }
  cluster_sync_all();
  const int rows_per = (SK_ROWS + S - 1) / S;
  const int row_lo = rank * rows_per, row_hi = min(SK_ROWS, row_lo + rows_per);
  const uint32_t base = smem_u32(part);
  // neighbouring threads read neighbouring floats of the peers' partials (one output row of
  // 32 activation rows per warp): the remote reads, S per output, are what this phase costs --
  // walking the output columns instead (coalesced stores, strided remote reads) measured
  // 15.6 us against 11.3 at the config-4 o projection
  for (int idx = tid; idx < (row_hi - row_lo) * SK_M; idx += SK_THREADS) {
    const int row = row_lo + idx / SK_M, m = idx % SK_M;
    const int64_t col = group * SK_ROWS + row;
    const uint32_t off = base + (uint32_t)((row * SK_PSTRIDE + m) * 4);
    float sum = 0.f;
    for (int r = 0; r < S; ++r) sum += ld_shared_cluster_f32(mapa_shared(off, (unsigned)r));
    if (m < a.m && col < a.n) {
      float v = sum * __ldg(a.scales + col);
      if (a.bias) v = round_bf16(v) + round_bf16(__ldg(a.bias + col));
      a.y[(int64_t)m * a.n + col] = __float2bfloat16_rn(v);
    }
  }
  cluster_sync_all();  // every peer has read this CTA's partial
}

// Plan: clusters of 8 K ranges per 128-row group, else 4, taken only when every group's
// cluster fits at two CTAs per SM and a CTA holds at most SK_MAXB k blocks; other shapes stay
// on the tensor-core GEMM. Measured at the config-4 decode shapes, 32 rows, same box:
// o (2048 x 4096, 16 groups x 8 = 128 CTAs) 11.3 us alone against 13.8 on tcgen05, decode
// step 9.59 -> 9.37 ms; qkv (5120 x 2048, 40 groups x 4 = 160 CTAs) 14.0 us alone against
// 13.8, but step 9.34 -> 9.07 ms -- in the step its weight requests, issued before the
// dependency wait, overlap the previous kernel. 0: not taken.
static int sk_splits(int64_t n, int64_t k) {
  const int64_t nbk = (k + SK_KB - 1) / SK_KB;
  const int64_t groups = (n + SK_ROWS - 1) / SK_ROWS;
  int64_t s = SK_MAX_CLUSTER;
  if (groups * s > 2 * num_sms()) s = SK_MAX_CLUSTER / 2;
  if (groups * s > 2 * num_sms() || nbk < s || (nbk + s - 1) / s > SK_MAXB) return 0;
  return (int)s;
}

bool qrow_skinny_supported(int64_t m, int64_t n, int64_t k) {
  return m > 16 && m <= SK_M && k % 16 == 0 && n > 0 && sk_splits(n, k) > 0 && (n + SK_ROWS - 1) / SK_ROWS <= (1 << 24);
}

int qrow_skinny_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                     int64_t n, const float* bias, __nv_bfloat16* y, cudaStream_t s) {
  const int S = sk_splits(n, k);
  if (!S) return fail(MRB_ERR_UNSUPPORTED, "qrow skinny: in_features %lld too large", (long long)k);
  SkinnyArgs a{x, m, n, k, codes, scales, bias, y, S, (int)((k + SK_KB - 1) / SK_KB), 0};
  const int blocks = (a.nbk + S - 1) / S;
  a.xstride = sk_xstride(blocks);
  const size_t smem = sk_smem_bytes(blocks);
  const int st = ensure_dynamic_smem((const void*)qrow_skinny_kernel, smem, "qrow skinny");
  if (st) return st;
  const int64_t groups = (n + SK_ROWS - 1) / SK_ROWS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(groups * S));
  cfg.blockDim = dim3(SK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, qrow_skinny_kernel, a);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "qrow skinny: launch: %s", cudaGetErrorString(e));
  return launch_status("qrow skinny");
}

}  // namespace mrb
