// Decode-size W8A16 projection: an HBM-bound int8 GEMV on the tensor pipe.
//
// y[m, n] = scale[n] * sum_k x[m, k] * code[n, k] for m <= 16 rows of activations.
//
// Design (B200, sm_100a):
//  * Weights stream once from HBM with 128-bit L1-bypassing loads. A CTA (8 warps) owns a
//    16-row weight tile; its warps split K in 64-byte blocks, interleaved so the CTA reads
//    each row as one contiguous stream, and reduce the partial sums through shared memory
//    in a fixed order (deterministic).
//  * Dequantisation is exact and costs ~1.25 integer/half instructions per weight byte:
//    int8 -> biased byte -> f16 (0x6400 | byte) - 1152 gives the code as an exact f16.
//  * The dot product runs on mma.sync m16n8k16 (f16 x f16 -> f32). Activations are staged
//    once per CTA in shared memory as f16 scaled by a per-row power of two so every bf16
//    value is represented exactly (8 significant bits fit f16's 11); fp32 activations are
//    split into hi + lo f16 halves (22 significant bits) occupying two mma columns.
//    Products are therefore exact and accumulate in fp32, the contract of the reference's
//    `tl.dot(..., fp32 acc)`; the row scale is applied once in fp32 after the reduction.
//  * The k order inside each 64-element block is permuted identically for weights and
//    activations (each lane consumes 4 consecutive bytes per mma), so every lane issues one
//    16-byte load per weight row per block and no shuffles are needed.
#include "qrow_common.cuh"

#include <algorithm>
#include <cmath>

namespace mrb {

constexpr int GV_WARPS = 8;
constexpr int GV_THREADS = GV_WARPS * 32;
constexpr int GV_ROWS = 16;  // weight rows per tile (mma M)
constexpr int GV_KB = 64;    // k elements per lane-group block

enum { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_ARGMAX = 2 };

struct GemvArgs {
  const void* x;
  int64_t m;
  int64_t k;
  const int8_t* codes0;
  const float* scales0;
  const int8_t* codes1;  // up projection for EPI_SWIGLU
  const float* scales1;
  const float* bias;
  int64_t n;
  void* y;                     // EPI_ARGMAX: fp32 logits or null
  int64_t semantic;            // EPI_ARGMAX: rows eligible for the argmax
  unsigned long long* packed;  // EPI_ARGMAX: per activation row, max of pack(logit, row)
};

// Prefetch ring depth (k blocks in flight per thread) by number of weight streams.
template <int NSTREAM>
struct GvRing {
  static constexpr int STAGES = NSTREAM == 2 ? 5 : 8;
  // one stage: NSTREAM streams x 2 rows (g, g+8) x 16 bytes per thread
  static constexpr int STAGE_BYTES = NSTREAM * 2 * GV_THREADS * 16;
  static constexpr int BYTES = STAGES * STAGE_BYTES;
};

__host__ __device__ inline int gv_kpad(int64_t k) { return (int)(((k + GV_KB - 1) / GV_KB) * GV_KB); }
__host__ __device__ inline int gv_xstride(int64_t k) { return gv_kpad(k) + 8; }  // f16 elems, +16 B

template <int NSTREAM>
__host__ inline size_t gv_smem_bytes(int ncols, int64_t k, int nt) {
  size_t xs = (size_t)ncols * gv_xstride(k) * 2;
  xs = (xs + 15) & ~size_t(15);
  const size_t red = (size_t)GV_WARPS * NSTREAM * GV_ROWS * 8 * nt * 4;
  return GvRing<NSTREAM>::BYTES + xs + red + 64 * 4;  // + per-column factors, maxima and sums
}

// Weight-streaming W8A16 GEMV (M <= 16 activation rows).
//
// A CTA (8 warps, two per SM) owns every gridDim-th 16-row weight tile. Within a
// tile the warps split the 64-element k blocks; every thread streams its two 16-byte
// slices per block (rows g and g+8) through a private cp.async ring in shared memory, so
// 7 (one stream) or 4 (two streams) blocks per thread -- over 100 KB per SM -- are in flight
// without holding registers and with no barrier between blocks (each thread reads back only
// the bytes it requested). The first blocks are requested before the programmatic-
// dependent-launch wait, so weight streaming overlaps the previous kernel's tail; only the
// activation staging waits for it. Codes become exact f16 with integer/half ops,
// activations are staged once per CTA as exact power-of-two-scaled f16, mma.sync
// accumulates in fp32, and a tile's warps reduce through shared memory in a fixed order.
template <typename XT, typename YT, bool SPLIT, int NT, int EPI>
__global__ void __launch_bounds__(GV_THREADS, 2) qrow_gemv_kernel(GemvArgs a) {
  constexpr int NSTREAM = (EPI == EPI_SWIGLU) ? 2 : 1;
  constexpr int STAGES = GvRing<NSTREAM>::STAGES;
  constexpr int STAGE_BYTES = GvRing<NSTREAM>::STAGE_BYTES;
  extern __shared__ __align__(128) unsigned char smem[];
  const int M = (int)a.m;
  const int64_t K = a.k;
  const int64_t n = a.n;
  const int ncols = SPLIT ? 2 * M : M;
  const int kpad = gv_kpad(K);
  const int xstride = gv_xstride(K);
  const int nkb_tile = kpad / GV_KB;
  unsigned char* ring = smem;
  __half* xs = reinterpret_cast<__half*>(smem + GvRing<NSTREAM>::BYTES);
  const size_t xs_bytes = ((size_t)ncols * xstride * 2 + 15) & ~size_t(15);
  float* red = reinterpret_cast<float*>(smem + GvRing<NSTREAM>::BYTES + xs_bytes);
  float* colscale = red + GV_WARPS * NSTREAM * GV_ROWS * 8 * NT;  // [0,16): 2^-e, [16,32): 2^e
  unsigned* colmax = reinterpret_cast<unsigned*>(colscale + 32);
  float* colsum = colscale + 48;  // sum of the staged f16 activations per column (biased codes)

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  // tiles blockIdx.x, +gridDim.x, ...: the CTAs sweep the matrix together (one window of
  // adjacent tiles at a time), which keeps DRAM pages and TLB entries shared between SMs
  const int ntiles = (int)((n + GV_ROWS - 1) / GV_ROWS);  // 16-row tiles (< 2^27 by the host check)
  // this warp's k blocks per tile: warp, warp + 8, ...
  const int kpw = warp < nkb_tile ? (nkb_tile - warp + GV_WARPS - 1) / GV_WARPS : 0;

  pdl_launch_dependents();

  // ---- per-thread prefetch stream: (tile pf_T, this warp's pf_i-th k block of it)
  int pf_T = kpw > 0 ? (int)blockIdx.x : ntiles, pf_i = 0, slot_w = 0;
  auto issue = [&]() {
    if (pf_T < ntiles) {
      const int kb = warp + GV_WARPS * pf_i;
      const int koff = kb * GV_KB + 16 * c;
      const bool ok = koff < K;
      const int64_t r0 = min((int64_t)pf_T * GV_ROWS + g, n - 1);
      const int64_t r1 = min((int64_t)pf_T * GV_ROWS + g + 8, n - 1);
      unsigned char* st = ring + slot_w * STAGE_BYTES;
#pragma unroll
      for (int s = 0; s < NSTREAM; ++s) {
        const int8_t* codes = s == 0 ? a.codes0 : a.codes1;
        cp_async16_zfill(st + ((s * 2 + 0) * GV_THREADS + tid) * 16, codes + (ok ? r0 * K + koff : 0), ok);
        cp_async16_zfill(st + ((s * 2 + 1) * GV_THREADS + tid) * 16, codes + (ok ? r1 * K + koff : 0), ok);
      }
      if (++pf_i == kpw) {
        pf_i = 0;
        pf_T += gridDim.x;
      }
    }
    cp_async_commit_group();
    slot_w = slot_w + 1 == STAGES ? 0 : slot_w + 1;
  };
#pragma unroll
  for (int p = 0; p < STAGES - 1; ++p) issue();  // before the dependency wait

  // ---- activations: wait for the producer kernel, then stage exact scaled f16 copies
  pdl_wait();
  constexpr int VEC = 16 / sizeof(XT);
  if (tid < 16) colmax[tid] = 0u;
  __syncthreads();
  const int vpr = (int)(K / VEC);
  const int nvec = M * vpr;
  const uint4* xv = reinterpret_cast<const uint4*>(a.x);
  if (!SPLIT) {
    // one global round trip: copy the raw 16-bit rows into their staging slots while
    // tracking each row's max |x|, then convert in place with the power-of-two factor
    int cur = -1;
    float mx = 0.f;
#pragma unroll 4
    for (int v = tid; v < nvec; v += GV_THREADS) {
      const int mi = v / vpr;
      const uint4 raw = __ldg(xv + v);
      *reinterpret_cast<uint4*>(xs + mi * xstride + (v - mi * vpr) * VEC) = raw;
      if (mi != cur) {
        if (cur >= 0) atomicMax(&colmax[cur], __float_as_uint(mx));
        cur = mi;
        mx = 0.f;
      }
      const XT* e = reinterpret_cast<const XT*>(&raw);
#pragma unroll
      for (int i = 0; i < VEC; ++i) mx = fmaxf(mx, fabsf(io<XT>::load(e + i)));
    }
    if (cur >= 0) atomicMax(&colmax[cur], __float_as_uint(mx));
  } else {
    int cur = -1;
    float mx = 0.f;
#pragma unroll 4
    for (int v = tid; v < nvec; v += GV_THREADS) {
      const int mi = v / vpr;
      if (mi != cur) {
        if (cur >= 0) atomicMax(&colmax[cur], __float_as_uint(mx));
        cur = mi;
        mx = 0.f;
      }
      const uint4 raw = __ldg(xv + v);
      const XT* e = reinterpret_cast<const XT*>(&raw);
#pragma unroll
      for (int i = 0; i < VEC; ++i) mx = fmaxf(mx, fabsf(io<XT>::load(e + i)));
    }
    if (cur >= 0) atomicMax(&colmax[cur], __float_as_uint(mx));
  }
  __syncthreads();
  if (tid < M) {
    const float mx = __uint_as_float(colmax[tid]);
    int e = 0;
    if (mx > 0.f && isfinite(mx)) {
      int ex;
      frexpf(mx, &ex);                   // mx in [2^(ex-1), 2^ex)
      e = max(-100, min(100, 15 - ex));  // mx * 2^e in [2^14, 2^15)
    }
    colscale[tid] = ldexpf(1.0f, -e);
    colscale[16 + tid] = ldexpf(1.0f, e);
  }
  __syncthreads();
#pragma unroll 4
  for (int v = tid; v < nvec; v += GV_THREADS) {
    const int mi = v / vpr;
    const int kk = (v - mi * vpr) * VEC;
    const float f = colscale[16 + mi];
    if (SPLIT) {
      const uint4 raw = __ldg(xv + v);
      const XT* e = reinterpret_cast<const XT*>(&raw);
      __half hi[VEC], lo[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        const float val = io<XT>::load(e + i) * f;  // exact power-of-two scaling
        hi[i] = __float2half_rn(val);
        lo[i] = __float2half_rn((val - __half2float(hi[i])) * 2048.0f);
      }
      *reinterpret_cast<uint2*>(xs + (2 * mi) * xstride + kk) = *reinterpret_cast<const uint2*>(hi);
      *reinterpret_cast<uint2*>(xs + (2 * mi + 1) * xstride + kk) = *reinterpret_cast<const uint2*>(lo);
    } else {
      uint4* slot = reinterpret_cast<uint4*>(xs + mi * xstride + kk);
      const uint4 raw = *slot;
      const XT* e = reinterpret_cast<const XT*>(&raw);
      __align__(16) __half h[VEC];
#pragma unroll
      for (int i = 0; i < VEC; ++i) h[i] = __float2half_rn(io<XT>::load(e + i) * f);
      *slot = *reinterpret_cast<const uint4*>(h);
    }
  }
  const int padw = kpad - (int)K;
  for (int idx = tid; idx < ncols * padw; idx += GV_THREADS) {
    const int col = idx / padw;
    xs[col * xstride + (int)K + (idx - col * padw)] = __float2half_rn(0.f);
  }
  __syncthreads();
  if (!SPLIT) {
    // fixed-order column sums of exactly the f16 values the mma consumes: warp w sums
    // columns w, w + 8 with lanes striding k, then a fixed shuffle tree
    for (int col = warp; col < ncols; col += GV_WARPS) {
      float sum = 0.f;
      for (int kk = lane * 8; kk < kpad; kk += 32 * 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(xs + col * xstride + kk);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h2[j]);
          sum += f.x + f.y;
        }
      }
      sum = warp_sum(sum);
      if (lane == 0) colsum[col] = sum;
    }
    __syncthreads();
  }

  float acc[NSTREAM][NT][4];
#pragma unroll
  for (int s = 0; s < NSTREAM; ++s)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s][t][i] = 0.f;
  unsigned long long best_key = 0ull;  // EPI_ARGMAX: running max over this CTA's tiles

  int slot_r = 0;  // ring slot this thread reads next
  for (int T = blockIdx.x; T < ntiles; T += gridDim.x) {
    const int64_t tile = T;
    for (int i = 0; i < kpw; ++i) {
      cp_async_wait_group<STAGES - 2>();
      const unsigned char* st = ring + slot_r * STAGE_BYTES;
      slot_r = slot_r + 1 == STAGES ? 0 : slot_r + 1;
      uint4 wa[NSTREAM], wb[NSTREAM];
#pragma unroll
      for (int s = 0; s < NSTREAM; ++s) {
        wa[s] = *reinterpret_cast<const uint4*>(st + ((s * 2 + 0) * GV_THREADS + tid) * 16);
        wb[s] = *reinterpret_cast<const uint4*>(st + ((s * 2 + 1) * GV_THREADS + tid) * 16);
      }
      issue();
      const int kb = warp + GV_WARPS * i;
      uint32_t xb[NT][8];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int col = t * 8 + g;
        if (col < ncols) {
          const uint4* p = reinterpret_cast<const uint4*>(xs + col * xstride + kb * GV_KB + 16 * c);
          const uint4 v0 = p[0], v1 = p[1];
          xb[t][0] = v0.x; xb[t][1] = v0.y; xb[t][2] = v0.z; xb[t][3] = v0.w;
          xb[t][4] = v1.x; xb[t][5] = v1.y; xb[t][6] = v1.z; xb[t][7] = v1.w;
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) xb[t][j] = 0u;
        }
      }
#pragma unroll
      for (int s = 0; s < NSTREAM; ++s) {
        const uint32_t ra[4] = {wa[s].x, wa[s].y, wa[s].z, wa[s].w};
        const uint32_t rb[4] = {wb[s].x, wb[s].y, wb[s].z, wb[s].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a_lo, a_hi, b_lo, b_hi;
          if (SPLIT) {  // fp32 activations keep the exact code (no bias term in the sum)
            i8x4_to_f16x2(ra[j], a_lo, a_hi);
            i8x4_to_f16x2(rb[j], b_lo, b_hi);
          } else {
            i8x4_to_biased_f16x2(ra[j], a_lo, a_hi);
            i8x4_to_biased_f16x2(rb[j], b_lo, b_hi);
          }
#pragma unroll
          for (int t = 0; t < NT; ++t) mma_f16(acc[s][t], a_lo, b_lo, a_hi, b_hi, xb[t][2 * j], xb[t][2 * j + 1]);
        }
      }
    }

    // ---- tile end: cross-warp reduction in a fixed order, then the epilogue
#pragma unroll
    for (int s = 0; s < NSTREAM; ++s)
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float* base = red + ((warp * NSTREAM + s) * GV_ROWS) * (8 * NT);
        const int col = t * 8 + 2 * c;
        base[g * (8 * NT) + col] = acc[s][t][0];
        base[g * (8 * NT) + col + 1] = acc[s][t][1];
        base[(g + 8) * (8 * NT) + col] = acc[s][t][2];
        base[(g + 8) * (8 * NT) + col + 1] = acc[s][t][3];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[s][t][j] = 0.f;
      }
    __syncthreads();
    auto total = [&](int s, int row, int col) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < GV_WARPS; ++w) tot += red[((w * NSTREAM + s) * GV_ROWS + row) * (8 * NT) + col];
      // remove the code bias: sum (q+1152) x - 1152 sum x over this tile's k range
      return SPLIT ? tot : tot - 1152.0f * colsum[col];
    };
    if (EPI == EPI_ARGMAX) {
      const int row = tid % GV_ROWS, mi = tid / GV_ROWS;  // all threads: converged shuffles
      const int64_t nrow = tile * GV_ROWS + row;
      unsigned long long key = 0ull;
      if (mi < M && nrow < n) {
        const float t = SPLIT ? total(0, row, 2 * mi) + total(0, row, 2 * mi + 1) * (1.0f / 2048.0f)
                              : total(0, row, mi);
        const float v = t * colscale[mi] * a.scales0[nrow];
        if (a.y) reinterpret_cast<float*>(a.y)[(int64_t)mi * n + nrow] = v;
        if (nrow < a.semantic) key = pack_argmax(v, nrow);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if (key > best_key) best_key = key;
    } else {
      for (int idx = tid; idx < GV_ROWS * M; idx += GV_THREADS) {
        const int row = idx % GV_ROWS, mi = idx / GV_ROWS;
        const int64_t nrow = tile * GV_ROWS + row;
        if (nrow >= n) continue;
        float v[NSTREAM];
#pragma unroll
        for (int s = 0; s < NSTREAM; ++s) {
          const float t = SPLIT ? total(s, row, 2 * mi) + total(s, row, 2 * mi + 1) * (1.0f / 2048.0f)
                                : total(s, row, mi);
          v[s] = t * colscale[mi] * (s == 0 ? a.scales0 : a.scales1)[nrow];
        }
        YT* y = reinterpret_cast<YT*>(a.y) + (int64_t)mi * n + nrow;
        if (EPI == EPI_SWIGLU) {
          const float gt = round_bf16(v[0]);
          const float up = round_bf16(v[NSTREAM - 1]);
          io<YT>::store(y, round_bf16(silu_f32(gt)) * up);
        } else {
          float out = v[0];
          if (a.bias) {  // the reference adds a compute-dtype bias to the compute-dtype projection
            YT tmp, b;
            io<YT>::store(&tmp, out);
            io<YT>::store(&b, a.bias[nrow]);
            out = io<YT>::load(&tmp) + io<YT>::load(&b);
          }
          io<YT>::store(y, out);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait_group<0>();
  if (EPI == EPI_ARGMAX && (tid % GV_ROWS) == 0 && tid / GV_ROWS < M && best_key != 0ull)
    atomicMax(a.packed + tid / GV_ROWS, best_key);
}

// Unpack the argmax keys into indices (int64) and logit values, in place.
__global__ void argmax_unpack_kernel(unsigned long long* packed, float* out_value, int64_t m) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= m) return;
  const unsigned long long key = packed[i];
  const unsigned hi = (unsigned)(key >> 32);
  const unsigned u = (hi & 0x80000000u) ? (hi & 0x7FFFFFFFu) : ~hi;
  const int64_t row = (int64_t)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFull));
  reinterpret_cast<int64_t*>(packed)[i] = row;
  if (out_value) out_value[i] = __uint_as_float(u);
}

// ------------------------------------------------------------------ argmax over logits

// First maximal index per row over the first `semantic` columns (lowest index on ties).
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* __restrict__ logits, int64_t n,
                                                           int64_t semantic, int64_t* __restrict__ out_index,
                                                           float* __restrict__ out_value) {
  const int64_t row = blockIdx.x;
  const float* p = logits + row * n;
  float best = -INFINITY;
  int64_t bi = 0x7fffffffffffffffLL;
  for (int64_t i = threadIdx.x; i < semantic; i += blockDim.x) {
    const float v = p[i];
    if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    sv[w] = best;
    si[w] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    const int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffffffffffffLL;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) {
      out_index[row] = bi == 0x7fffffffffffffffLL ? 0 : bi;
      if (out_value) out_value[row] = best;
    }
  }
}

// ------------------------------------------------------------------ host dispatch

template <typename XT, typename YT, bool SPLIT, int NT, int EPI>
static int launch_gemv(const GemvArgs& a, cudaStream_t s) {
  constexpr int NSTREAM = EPI == EPI_SWIGLU ? 2 : 1;
  const int ncols = SPLIT ? 2 * (int)a.m : (int)a.m;
  const size_t smem = gv_smem_bytes<NSTREAM>(ncols, a.k, NT);
  if (smem > 227 * 1024)
    return fail(MRB_ERR_UNSUPPORTED, "qrow gemv: activation block %lld x %lld too large for one CTA",
                (long long)a.m, (long long)a.k);
  if (a.n > (1LL << 27)) return fail(MRB_ERR_UNSUPPORTED, "qrow gemv: %lld output rows", (long long)a.n);
  auto kern = qrow_gemv_kernel<XT, YT, SPLIT, NT, EPI>;
  static size_t configured = 0;  // per instantiation
  if (smem > configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "qrow gemv: smem attribute: %s", cudaGetErrorString(e));
    configured = smem;
  }
  // two CTAs per SM when shared memory allows (the register bound allows two)
  const int per_sm = 2 * (smem + 1024) <= 227 * 1024 ? 2 : 1;
  const int64_t ntiles = (a.n + GV_ROWS - 1) / GV_ROWS;
  const int64_t grid = std::min<int64_t>(ntiles, (int64_t)num_sms() * per_sm);
  // the argmax head is preceded by a memset node, which takes no programmatic edge
  cudaError_t e = launch_kernel(kern, dim3((unsigned)grid), dim3(GV_THREADS), smem, s, EPI != EPI_ARGMAX, a);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "qrow gemv: launch: %s", cudaGetErrorString(e));
  return launch_status("qrow gemv");
}

template <typename XT, typename YT, bool SPLIT, int EPI>
static int dispatch_nt(const GemvArgs& a, cudaStream_t s) {
  // Activation rows per launch: at most 16 mma columns, and a staged f16 copy that fits
  // one CTA's shared memory; wider requests re-stream the weights once per chunk.
  constexpr int NSTREAM = EPI == EPI_SWIGLU ? 2 : 1;
  const size_t fixed = gv_smem_bytes<NSTREAM>(0, a.k, 2);
  const size_t per_col = (size_t)gv_xstride(a.k) * 2;
  if (fixed + per_col > 227 * 1024)
    return fail(MRB_ERR_UNSUPPORTED, "qrow gemv: in_features %lld too large", (long long)a.k);
  const int max_rows = (int)std::min<size_t>((227 * 1024 - fixed) / per_col, 16) / (SPLIT ? 2 : 1);
  if (max_rows < 1) return fail(MRB_ERR_UNSUPPORTED, "qrow gemv: in_features %lld too large", (long long)a.k);
  for (int64_t r0 = 0; r0 < a.m; r0 += max_rows) {
    GemvArgs part = a;
    part.m = std::min<int64_t>(max_rows, a.m - r0);
    part.x = reinterpret_cast<const XT*>(a.x) + r0 * a.k;
    part.y = a.y ? reinterpret_cast<YT*>(a.y) + r0 * a.n : nullptr;
    if (a.packed) part.packed = a.packed + r0;
    const int pcols = SPLIT ? 2 * (int)part.m : (int)part.m;
    const int st = pcols <= 8 ? launch_gemv<XT, YT, SPLIT, 1, EPI>(part, s) : launch_gemv<XT, YT, SPLIT, 2, EPI>(part, s);
    if (st) return st;
  }
  return MRB_OK;
}

static int check_common(const void* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                        int64_t n, const void* y, const char* what) {
  if (m < 0 || k <= 0 || n <= 0) return fail(MRB_ERR_ARG, "%s: bad shape m=%lld k=%lld n=%lld", what,
                                             (long long)m, (long long)k, (long long)n);
  if (!codes || !scales) return fail(MRB_ERR_ARG, "%s: null pointer", what);
  if (m > 0 && (!x || !y)) return fail(MRB_ERR_ARG, "%s: null pointer", what);
  if (k % 16 != 0) return fail(MRB_ERR_UNSUPPORTED, "%s: in_features %lld is not a multiple of 16", what,
                               (long long)k);
  if (!aligned(codes, 16)) return fail(MRB_ERR_ARG, "%s: codes must be 16-byte aligned", what);
  if (m > 0 && !aligned(x, 16)) return fail(MRB_ERR_ARG, "%s: activations must be 16-byte aligned", what);
  return MRB_OK;
}

int qrow_gemm_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                   int64_t n, const float* bias, __nv_bfloat16* y, cudaStream_t s);
int qrow_gemm_swiglu_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* gate_codes,
                          const float* gate_scales, const int8_t* up_codes, const float* up_scales, int64_t n,
                          __nv_bfloat16* y, cudaStream_t s);

// Activation rows above which bf16 projections use the tensor-core GEMM.
constexpr int64_t GEMV_MAX_ROWS = 16;

static GemvArgs make_args(const void* x, int64_t m, int64_t k, const int8_t* c0, const float* s0, const int8_t* c1,
                          const float* s1, const float* bias, int64_t n, void* y) {
  GemvArgs a{};
  a.x = x; a.m = m; a.k = k; a.codes0 = c0; a.scales0 = s0; a.codes1 = c1; a.scales1 = s1;
  a.bias = bias; a.n = n; a.y = y;
  return a;
}

int qrow_gemv_dispatch(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* codes,
                       const float* scales, int64_t n, const float* bias, void* y, cudaStream_t s) {
  const GemvArgs a = make_args(x, m, k, codes, scales, nullptr, nullptr, bias, n, y);
  switch (x_dtype) {
    case MRB_BF16:
      if (m > GEMV_MAX_ROWS)
        return qrow_gemm_bf16((const __nv_bfloat16*)x, m, k, codes, scales, n, bias, (__nv_bfloat16*)y, s);
      return dispatch_nt<__nv_bfloat16, __nv_bfloat16, false, EPI_STORE>(a, s);
    case MRB_F16: return dispatch_nt<__half, __half, false, EPI_STORE>(a, s);
    case MRB_F32: return dispatch_nt<float, float, true, EPI_STORE>(a, s);
    default: return fail(MRB_ERR_ARG, "qrow_matmul: bad x_dtype %d", x_dtype);
  }
}

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_qrow_matmul(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* codes,
                               const float* scales, int64_t n, const float* bias, void* y, int y_dtype,
                               void* stream) {
  int st = check_common(x, m, k, codes, scales, n, y, "qrow_matmul");
  if (st) return st;
  if (y_dtype != x_dtype) return fail(MRB_ERR_ARG, "qrow_matmul: output dtype must equal activation dtype");
  if (m == 0) return MRB_OK;
  return qrow_gemv_dispatch(x, x_dtype, m, k, codes, scales, n, bias, y, (cudaStream_t)stream);
}

extern "C" int mrb_qrow_swiglu(const void* x_bf16, int64_t m, int64_t k, const int8_t* gate_codes,
                               const float* gate_scales, const int8_t* up_codes, const float* up_scales,
                               int64_t n, void* y_bf16, void* stream) {
  int st = check_common(x_bf16, m, k, gate_codes, gate_scales, n, y_bf16, "qrow_swiglu");
  if (st) return st;
  if (!up_codes || !up_scales) return fail(MRB_ERR_ARG, "qrow_swiglu: null up page");
  if (!aligned(up_codes, 16)) return fail(MRB_ERR_ARG, "qrow_swiglu: codes must be 16-byte aligned");
  if (m == 0) return MRB_OK;
  if (m > GEMV_MAX_ROWS)
    return qrow_gemm_swiglu_bf16((const __nv_bfloat16*)x_bf16, m, k, gate_codes, gate_scales, up_codes, up_scales,
                                 n, (__nv_bfloat16*)y_bf16, (cudaStream_t)stream);
  const GemvArgs a = make_args(x_bf16, m, k, gate_codes, gate_scales, up_codes, up_scales, nullptr, n, y_bf16);
  return dispatch_nt<__nv_bfloat16, __nv_bfloat16, false, EPI_SWIGLU>(a, (cudaStream_t)stream);
}

extern "C" int mrb_qrow_argmax(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* codes,
                               const float* scales, int64_t n, int64_t semantic_rows, float* logits,
                               int64_t* out_index, float* out_value, void* stream) {
  int st = check_common(x, m, k, codes, scales, n, out_index, "qrow_argmax");
  if (st) return st;
  if (semantic_rows < 1 || semantic_rows > n)
    return fail(MRB_ERR_ARG, "qrow_argmax: semantic_rows %lld outside [1, %lld]", (long long)semantic_rows,
                (long long)n);
  if (n > 0xFFFFFFFFLL) return fail(MRB_ERR_UNSUPPORTED, "qrow_argmax: more than 2^32 rows");
  if (m == 0) return MRB_OK;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(out_index, 0, (size_t)m * sizeof(int64_t), s);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "qrow_argmax: memset: %s", cudaGetErrorString(e));
  GemvArgs a = make_args(x, m, k, codes, scales, nullptr, nullptr, nullptr, n, logits);
  a.semantic = semantic_rows;
  a.packed = reinterpret_cast<unsigned long long*>(out_index);
  switch (x_dtype) {
    case MRB_BF16: st = dispatch_nt<__nv_bfloat16, float, false, EPI_ARGMAX>(a, s); break;
    case MRB_F16: st = dispatch_nt<__half, float, false, EPI_ARGMAX>(a, s); break;
    case MRB_F32: st = dispatch_nt<float, float, true, EPI_ARGMAX>(a, s); break;
    default: return fail(MRB_ERR_ARG, "qrow_argmax: bad x_dtype %d", x_dtype);
  }
  if (st) return st;
  argmax_unpack_kernel<<<(unsigned)((m + 127) / 128), 128, 0, s>>>(reinterpret_cast<unsigned long long*>(out_index),
                                                                    out_value, m);
  return launch_status("qrow_argmax");
}
