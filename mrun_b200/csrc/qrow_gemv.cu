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
  int64_t units;               // stream-K: tiles x k blocks (0: round-robin whole tiles)
  unsigned* ws_counters;       // stream-K: per-tile arrival counters (zero between launches)
  float* ws_parts;             // stream-K: per-CTA partial tiles
  int stages;                  // cp.async ring depth per thread (3..6)
};

// Per-thread ring stage: 2 weight streams x 2 rows (g, g+8) x 16 bytes.
constexpr int GV_STREAMS = 2;
constexpr int GV_STAGE_BYTES = GV_STREAMS * 2 * GV_THREADS * 16;
#ifndef MRB_GEMV_MAX_STAGES
#define MRB_GEMV_MAX_STAGES 4
#endif
constexpr int GV_MAX_STAGES = MRB_GEMV_MAX_STAGES;

// K blocks the schedule walks: a single matrix is streamed as its two K halves (block kb of
// each half per step, two independent mma chains per warp); the paired SwiGLU streams the
// gate and up matrices over the same k.
__host__ __device__ inline int gv_nkb(int64_t k) { return (int)((k + GV_KB - 1) / GV_KB); }
__host__ __device__ inline int gv_sched_blocks(int64_t k, bool halves) {
  return halves ? (gv_nkb(k) + 1) / 2 : gv_nkb(k);
}
// staged activation length (f16 elements, zero beyond k) and row stride (+16 B)
__host__ __device__ inline int gv_xlen(int64_t k, bool halves) {
  return gv_sched_blocks(k, halves) * GV_KB * (halves ? 2 : 1);
}
__host__ __device__ inline int gv_xstride(int64_t k, bool halves) { return gv_xlen(k, halves) + 8; }

// Shared-memory misc area (floats): [0,16) 2^-e and [16,32) 2^e per column, [32,48) column
// max |x| bits, [48,64) column sums, [64,192) per-warp column-sum parts, [192] merge flag.
constexpr int GV_MISC = 256;

__host__ __device__ inline size_t gv_xs_bytes(int ncols, int64_t k, bool halves) {
  return ((size_t)ncols * gv_xstride(k, halves) * 2 + 15) & ~size_t(15);
}
// double-buffered cross-warp reduction: [2][warp][stream][16 rows][ncols] fp32
__host__ __device__ inline size_t gv_red_bytes(int ncols) {
  return (size_t)2 * GV_WARPS * GV_STREAMS * GV_ROWS * ncols * 4;
}
__host__ inline size_t gv_smem_bytes(int stages, int ncols, int64_t k, bool halves) {
  return (size_t)stages * GV_STAGE_BYTES + gv_xs_bytes(ncols, k, halves) + gv_red_bytes(ncols) + GV_MISC * 4;
}

// Stream-K partial slot: 2 streams x 16 rows x 16 columns fp32. A CTA has two (its first
// and last tile segment).
constexpr int GV_SLOT_FLOATS = GV_STREAMS * GV_ROWS * 16;

template <int N>
__device__ __forceinline__ void gv_wait_ring(int stages) {
  // groups still allowed in flight = stages - 2 (the ring keeps stages - 1 requested)
  switch (stages) {
    case 6: cp_async_wait_group<4>(); break;
    case 5: cp_async_wait_group<3>(); break;
    case 4: cp_async_wait_group<2>(); break;
    default: cp_async_wait_group<1>(); break;
  }
}

// Weight-streaming W8A16 GEMV (M <= 16 activation rows).
//
// Work is a sequence of tile segments: (16-row tile T, k steps [lo, hi)). With the
// round-robin schedule a CTA owns every gridDim-th tile whole. With the stream-K schedule
// (a.units = tiles x k steps) CTA c owns units [c*U/G, (c+1)*U/G) of the tile-major order,
// so every CTA streams the same number of weight bytes; a tile split over several CTAs is
// finished by the last of them to arrive, which adds the partial sums in CTA order
// (deterministic).
//
// Every k step carries two weight streams: for a single matrix, block kb of its first and
// of its second K half; for the paired SwiGLU, block kb of the gate and of the up matrix.
// The two streams feed independent mma accumulators, which doubles the work in flight per
// warp (the kernel is latency-bound per warp at two CTAs per SM). Within a segment the
// warps split the k steps; every thread streams its 16-byte slices of rows g and g+8 per
// stream through a private cp.async ring in shared memory, so 3 to 5 steps per thread are in
// flight without holding registers and with no barrier between steps (each thread reads
// back only the bytes it requested). The first steps are requested before the
// programmatic-dependent-launch wait, so weight streaming overlaps the previous kernel's
// tail; only the activation staging waits for it. Codes become exact f16 with integer/half
// ops, activations are staged once per CTA as exact power-of-two-scaled f16, mma.sync
// accumulates in fp32, and a segment's warps reduce through a double-buffered
// shared-memory area in a fixed order (one barrier per segment).
template <typename XT, typename YT, bool SPLIT, int NT, int EPI>
__global__ void __launch_bounds__(GV_THREADS, 2) qrow_gemv_kernel(GemvArgs a) {
  constexpr bool HALVES = EPI != EPI_SWIGLU;
  extern __shared__ __align__(128) unsigned char smem[];
  const int stages = a.stages;
  const int M = (int)a.m;
  const int64_t K = a.k;
  const int64_t n = a.n;
  const int ncols = SPLIT ? 2 * M : M;
  const int nkb = gv_sched_blocks(K, HALVES);  // k steps per tile
  const int xlen = gv_xlen(K, HALVES);
  const int xstride = xlen + 8;
  const int kspan = HALVES ? nkb * GV_KB : 0;  // k offset of the second stream
  unsigned char* ring = smem;
  __half* xs = reinterpret_cast<__half*>(smem + (size_t)stages * GV_STAGE_BYTES);
  float* red = reinterpret_cast<float*>(smem + (size_t)stages * GV_STAGE_BYTES + gv_xs_bytes(ncols, K, HALVES));
  const int red_elems = GV_WARPS * GV_STREAMS * GV_ROWS * ncols;
  float* colscale = red + 2 * red_elems;
  unsigned* colmax = reinterpret_cast<unsigned*>(colscale + 32);
  float* colsum = colscale + 48;   // sum of the staged f16 activations per column (biased codes)
  float* colpart = colscale + 64;  // [column][warp] parts of colsum
  int* merge_flag = reinterpret_cast<int*>(colscale + 192);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c = lane & 3;
  const int ntiles = (int)((n + GV_ROWS - 1) / GV_ROWS);  // < 2^27 by the host check

  // ---- schedule
  const bool streamk = a.units > 0;
  const int64_t U = a.units;
  const int G = (int)gridDim.x;
  int64_t u0 = 0, u1 = 0;
  if (streamk) {
    u0 = (int64_t)blockIdx.x * U / G;
    u1 = ((int64_t)blockIdx.x + 1) * U / G;
  }
  const int t_first = streamk ? (int)(u0 / nkb) : (int)blockIdx.x;
  auto seg_valid = [&](int T) { return streamk ? (int64_t)T * nkb < u1 : T < ntiles; };
  auto seg_next = [&](int T) { return streamk ? T + 1 : T + G; };
  auto seg_lo = [&](int T) { return streamk ? (int)max((int64_t)0, u0 - (int64_t)T * nkb) : 0; };
  auto seg_hi = [&](int T) { return streamk ? (int)min((int64_t)nkb, u1 - (int64_t)T * nkb) : nkb; };
  auto warp_blocks = [&](int lo, int hi) {
    const int nb = hi - lo;
    return warp < nb ? (nb - warp + GV_WARPS - 1) / GV_WARPS : 0;
  };

  pdl_launch_dependents();

  // ---- per-thread prefetch cursor: the rows (g, g+8) of this warp's next k step, the steps
  // left in its segment, and the lane's k offset (checked only when the k steps overhang K)
  const bool k_check = (int64_t)xlen != K;
  const int64_t delta1 = HALVES ? (int64_t)kspan : (int64_t)((uintptr_t)a.codes1 - (uintptr_t)a.codes0);
  int pf_T = t_first, pf_left = 0, pf_koff = 0, slot_w = 0;
  const int8_t* pf_row0 = a.codes0;
  const int8_t* pf_row1 = a.codes0;
  auto pf_enter = [&]() {  // enter segment pf_T, or the next one holding a step for this warp
    for (; seg_valid(pf_T); pf_T = seg_next(pf_T)) {
      const int lo = seg_lo(pf_T);
      pf_left = warp_blocks(lo, seg_hi(pf_T));
      if (pf_left > 0) {
        pf_koff = (lo + warp) * GV_KB + 16 * c;
        const int64_t r0 = min((int64_t)pf_T * GV_ROWS + g, n - 1);
        const int64_t r1 = min((int64_t)pf_T * GV_ROWS + g + 8, n - 1);
        pf_row0 = a.codes0 + r0 * K + pf_koff;
        pf_row1 = a.codes0 + r1 * K + pf_koff;
        return;
      }
    }
    pf_left = 0;
  };
  if (streamk || warp < nkb) pf_enter();  // round-robin warps beyond the k steps never load
  auto issue = [&]() {
    if (pf_left > 0) {
      unsigned char* st = ring + slot_w * GV_STAGE_BYTES + tid * 16;
#pragma unroll
      for (int s = 0; s < GV_STREAMS; ++s) {
        const int64_t d = s == 0 ? 0 : delta1;
        const bool ok = !k_check || pf_koff + (HALVES ? s * kspan : 0) < K;
        cp_async16_zfill(st + (s * 2 + 0) * GV_THREADS * 16, ok ? pf_row0 + d : a.codes0, ok);
        cp_async16_zfill(st + (s * 2 + 1) * GV_THREADS * 16, ok ? pf_row1 + d : a.codes0, ok);
      }
      pf_row0 += GV_WARPS * GV_KB;
      pf_row1 += GV_WARPS * GV_KB;
      pf_koff += GV_WARPS * GV_KB;
      if (--pf_left == 0) {
        pf_T = seg_next(pf_T);
        pf_enter();
      }
    }
    cp_async_commit_group();
    slot_w = slot_w + 1 == stages ? 0 : slot_w + 1;
  };
  for (int p = 0; p < stages - 1; ++p) issue();  // before the dependency wait
  // the epilogue's per-row scales (and bias) of every tile this CTA finishes: pull them into
  // L2 now, so the last tile's epilogue does not wait on HBM
  for (int idx = tid;; idx += GV_THREADS) {
    const int j = idx / 3, which = idx - 3 * (idx / 3);
    const int T = streamk ? t_first + j : t_first + j * G;  // round-robin tiles are G apart
    if (!seg_valid(T)) break;
    const float* p = which == 0 ? a.scales0 : which == 1 ? a.scales1 : a.bias;
    if (p) prefetch_l2(p + (int64_t)T * GV_ROWS);
  }

  // ---- activations: wait for the producer kernel, then stage exact scaled f16 copies
  pdl_wait();
  constexpr int VEC = 16 / sizeof(XT);
  if (tid < 16) colmax[tid] = 0u;
  __syncthreads();
  const int vpr = (int)(K / VEC);
  const int nvec = M * vpr;
  const uint4* xv = reinterpret_cast<const uint4*>(a.x);
  {
    // one global round trip for 16-bit rows: copy the raw rows into their staging slots
    // while tracking each row's max |x|, then convert in place with the power-of-two factor
    int cur = -1;
    float mx = 0.f;
#pragma unroll 4
    for (int v = tid; v < nvec; v += GV_THREADS) {
      const int mi = v / vpr;
      const uint4 raw = __ldg(xv + v);
      if (!SPLIT) *reinterpret_cast<uint4*>(xs + mi * xstride + (v - mi * vpr) * VEC) = raw;
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
  const int padw = xlen - (int)K;
  for (int idx = tid; idx < ncols * padw; idx += GV_THREADS) {
    const int col = idx / padw;
    xs[col * xstride + (int)K + (idx - col * padw)] = __float2half_rn(0.f);
  }
  __syncthreads();
  if (!SPLIT) {
    // fixed-order column sums of exactly the f16 values the mma consumes: warp w sums the
    // w-th eighth of every column (lanes striding k, then a fixed shuffle tree); the eight
    // parts are added in warp order before the first segment's epilogue reads them
    const int chunk = xlen / GV_WARPS;  // a multiple of 8 elements
    for (int col = 0; col < ncols; ++col) {
      const __half* base = xs + col * xstride + warp * chunk;
      float sum = 0.f;
      for (int kk = lane * 8; kk < chunk; kk += 32 * 8) {
        const uint4 raw = *reinterpret_cast<const uint4*>(base + kk);
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(h2[j]);
          sum += f.x + f.y;
        }
      }
      sum = warp_sum(sum);
      if (lane == 0) colpart[col * GV_WARPS + warp] = sum;
    }
    __syncthreads();
    if (tid < ncols) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < GV_WARPS; ++w) s += colpart[tid * GV_WARPS + w];
      colsum[tid] = s;  // read after the first segment's barrier
    }
  }

  float acc[GV_STREAMS][NT][4];
#pragma unroll
  for (int s = 0; s < GV_STREAMS; ++s)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[s][t][i] = 0.f;
  unsigned long long best_key = 0ull;  // EPI_ARGMAX: running max over this CTA's tiles

  // bias-corrected, scaled outputs of one finished tile from its raw per-stream column totals
  auto finish = [&](int64_t tile, auto&& total) {
    auto raw = [&](int s, int row, int col) {
      return HALVES ? total(0, row, col) + total(1, row, col) : total(s, row, col);
    };
    auto value = [&](int s, int row, int mi) {
      float t;
      if (SPLIT) {
        t = raw(s, row, 2 * mi) + raw(s, row, 2 * mi + 1) * (1.0f / 2048.0f);
      } else {
        // remove the code bias: sum (q+1152) x - 1152 sum x over the whole k range
        t = raw(s, row, mi) - 1152.0f * colsum[mi];
      }
      return t * colscale[mi] * (s == 0 ? a.scales0 : a.scales1)[tile * GV_ROWS + row];
    };
    if (EPI == EPI_ARGMAX) {
      const int row = tid % GV_ROWS, mi = tid / GV_ROWS;  // all threads: converged shuffles
      const int64_t nrow = tile * GV_ROWS + row;
      unsigned long long key = 0ull;
      if (mi < M && nrow < n) {
        const float v = value(0, row, mi);
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
        YT* y = reinterpret_cast<YT*>(a.y) + (int64_t)mi * n + nrow;
        if (EPI == EPI_SWIGLU) {
          const float gt = round_bf16(value(0, row, mi));
          const float up = round_bf16(value(1, row, mi));
          io<YT>::store(y, round_bf16(silu_f32(gt)) * up);
        } else {
          float out = value(0, row, mi);
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
  };

  int slot_r = 0;  // ring slot this thread reads next
  int parity = 0;  // reduction buffer of this segment
  for (int T = t_first; seg_valid(T); T = seg_next(T), parity ^= 1) {
    const int lo = seg_lo(T), hi = seg_hi(T);
    const int nb = warp_blocks(lo, hi);
    const __half* xp = xs + (lo + warp) * GV_KB + 16 * c;  // this lane's activations of the step
    for (int i = 0; i < nb; ++i, xp += GV_WARPS * GV_KB) {
      gv_wait_ring<0>(stages);
      const unsigned char* st = ring + slot_r * GV_STAGE_BYTES + tid * 16;
      slot_r = slot_r + 1 == stages ? 0 : slot_r + 1;
      uint4 wa[GV_STREAMS], wb[GV_STREAMS];
#pragma unroll
      for (int s = 0; s < GV_STREAMS; ++s) {
        wa[s] = *reinterpret_cast<const uint4*>(st + (s * 2 + 0) * GV_THREADS * 16);
        wb[s] = *reinterpret_cast<const uint4*>(st + (s * 2 + 1) * GV_THREADS * 16);
      }
      issue();
#pragma unroll
      for (int s = 0; s < GV_STREAMS; ++s) {
        uint32_t xb[NT][8];
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const int col = t * 8 + g;
          if (col < ncols) {
            const uint4* p = reinterpret_cast<const uint4*>(xp + col * xstride + (HALVES ? s * kspan : 0));
            const uint4 v0 = p[0], v1 = p[1];
            xb[t][0] = v0.x; xb[t][1] = v0.y; xb[t][2] = v0.z; xb[t][3] = v0.w;
            xb[t][4] = v1.x; xb[t][5] = v1.y; xb[t][6] = v1.z; xb[t][7] = v1.w;
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) xb[t][j] = 0u;
          }
        }
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

    // ---- segment end: cross-warp reduction in a fixed order, then the epilogue. The
    // buffer alternates, so the next segment's writes cannot race this one's reads.
    float* rbuf = red + parity * red_elems;
#pragma unroll
    for (int s = 0; s < GV_STREAMS; ++s)
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        float* base = rbuf + ((warp * GV_STREAMS + s) * GV_ROWS) * ncols;
        const int col = t * 8 + 2 * c;
        if (col < ncols) {
          base[g * ncols + col] = acc[s][t][0];
          base[(g + 8) * ncols + col] = acc[s][t][2];
        }
        if (col + 1 < ncols) {
          base[g * ncols + col + 1] = acc[s][t][1];
          base[(g + 8) * ncols + col + 1] = acc[s][t][3];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[s][t][j] = 0.f;
      }
    __syncthreads();
    auto warp_total = [&](int s, int row, int col) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < GV_WARPS; ++w) tot += rbuf[((w * GV_STREAMS + s) * GV_ROWS + row) * ncols + col];
      return tot;
    };
    if (lo == 0 && hi == nkb) {
      finish(T, warp_total);
      continue;
    }
    if constexpr (EPI != EPI_ARGMAX) {
      // ---- stream-K: publish this CTA's partial tile, the last arrival finishes it
      const int64_t ub = (int64_t)T * nkb;
      auto owner = [&](int64_t u) { return (int)(((u + 1) * G + U - 1) / U) - 1; };
      auto slot_of = [&](int cta) {
        const int64_t cu0 = (int64_t)cta * U / G;
        return 2 * cta + ((int)(cu0 / nkb) == T ? 0 : 1);
      };
      float* mine = a.ws_parts + (size_t)slot_of((int)blockIdx.x) * GV_SLOT_FLOATS;
      for (int idx = tid; idx < GV_STREAMS * GV_ROWS * ncols; idx += GV_THREADS) {
        const int col = idx % ncols, row = (idx / ncols) % GV_ROWS, s = idx / (ncols * GV_ROWS);
        mine[(s * GV_ROWS + row) * 16 + col] = warp_total(s, row, col);
      }
      __threadfence();
      __syncthreads();
      const int c_first = owner(ub), c_last = owner(ub + nkb - 1);
      if (tid == 0) {
        const unsigned prev = atomicAdd(a.ws_counters + T, 1u);
        const int last = prev == (unsigned)(c_last - c_first);
        if (last) a.ws_counters[T] = 0u;  // ready for the next launch
        *merge_flag = last;
      }
      __syncthreads();
      if (*merge_flag) {
        __threadfence();
        auto merged = [&](int s, int row, int col) {
          float tot = 0.f;
          for (int cta = c_first; cta <= c_last; ++cta)
            tot += __ldcg(a.ws_parts + (size_t)slot_of(cta) * GV_SLOT_FLOATS + (s * GV_ROWS + row) * 16 + col);
          return tot;
        };
        finish(T, merged);
      }
    }
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

// Shared memory the GEMV may use per SM (B200: 228 KB; 1 KB of it is reserved per CTA).
constexpr size_t GV_SM_SMEM = 228 * 1024;

struct GvPlan {
  int stages;
  size_t smem;
  int per_sm;
};

// Deepest ring (3..6 steps) that keeps two CTAs per SM; one CTA per SM when even three do not.
static GvPlan gv_plan(int ncols, int64_t k, bool halves) {
  for (int st = GV_MAX_STAGES; st >= 3; --st) {
    const size_t smem = gv_smem_bytes(st, ncols, k, halves);
    if (2 * (smem + 1024) <= GV_SM_SMEM) return {st, smem, 2};
  }
  for (int st = GV_MAX_STAGES; st >= 3; --st) {
    const size_t smem = gv_smem_bytes(st, ncols, k, halves);
    if (smem <= 227 * 1024) return {st, smem, 1};
  }
  return {0, 0, 0};
}

// Stream-K workspace: two partial slots per CTA slot first (a size that does not depend on
// the call), then one arrival counter per 16-row tile. Calls of different widths can share
// one workspace: partial writes never reach the counters, which are zero between launches.
static size_t gv_parts_bytes() { return (size_t)2 * num_sms() * 2 * GV_SLOT_FLOATS * sizeof(float); }

static size_t gv_workspace_bytes(int64_t n) {
  const int64_t ntiles = (n + GV_ROWS - 1) / GV_ROWS;
  return gv_parts_bytes() + (((size_t)ntiles * 4 + 255) & ~size_t(255));
}

struct GvWorkspace {
  void* ptr;
  size_t bytes;
};

template <typename XT, typename YT, bool SPLIT, int NT, int EPI>
static int launch_gemv(const GemvArgs& a0, GvWorkspace ws, cudaStream_t s) {
  constexpr bool HALVES = EPI != EPI_SWIGLU;
  const int ncols = SPLIT ? 2 * (int)a0.m : (int)a0.m;
  const GvPlan plan = gv_plan(ncols, a0.k, HALVES);
  if (!plan.stages)
    return fail(MRB_ERR_UNSUPPORTED, "qrow gemv: activation block %lld x %lld too large for one CTA",
                (long long)a0.m, (long long)a0.k);
  if (a0.n > (1LL << 27)) return fail(MRB_ERR_UNSUPPORTED, "qrow gemv: %lld output rows", (long long)a0.n);
  auto kern = qrow_gemv_kernel<XT, YT, SPLIT, NT, EPI>;
  const int smem_st = ensure_dynamic_smem((const void*)kern, plan.smem, "qrow gemv");
  if (smem_st) return smem_st;
  GemvArgs a = a0;
  a.units = 0;
  a.stages = plan.stages;
  const int64_t ntiles = (a.n + GV_ROWS - 1) / GV_ROWS;
  const int64_t slots = (int64_t)num_sms() * plan.per_sm;
  int64_t grid = std::min<int64_t>(ntiles, slots);
  // Stream-K when whole tiles fill under half of the CTA slots in their last wave and the
  // caller lent a workspace: split tiles add segment boundaries and a partial-tile merge
  // (measured: 224 tiles of 3584 x 18944 take 24.5 us split over 296 CTAs against 17.5 us as
  // whole tiles), which only pays when the imbalance is large.
  const int64_t waves = (ntiles + slots - 1) / slots;
  if (EPI != EPI_ARGMAX && ws.ptr && 2 * ntiles < waves * slots) {
    const size_t need = gv_workspace_bytes(a.n);
    if (ws.bytes < need)
      return fail(MRB_ERR_ARG, "qrow gemv: workspace of %zu bytes, %zu needed", ws.bytes, need);
    a.units = ntiles * gv_sched_blocks(a.k, HALVES);
    a.ws_parts = reinterpret_cast<float*>(ws.ptr);
    a.ws_counters = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(ws.ptr) + gv_parts_bytes());
    grid = std::min<int64_t>(slots, a.units);
  }
  // the argmax head is preceded by a memset node, which takes no programmatic edge
  cudaError_t e =
      launch_kernel(kern, dim3((unsigned)grid), dim3(GV_THREADS), plan.smem, s, EPI != EPI_ARGMAX, a);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "qrow gemv: launch: %s", cudaGetErrorString(e));
  return launch_status("qrow gemv");
}

template <typename XT, typename YT, bool SPLIT, int EPI>
static int dispatch_nt(const GemvArgs& a, GvWorkspace ws, cudaStream_t s) {
  // Activation rows per launch: at most 16 mma columns, and a staged f16 copy that fits
  // one CTA's shared memory next to a 3-step ring; wider requests re-stream the weights
  // once per chunk.
  constexpr bool HALVES = EPI != EPI_SWIGLU;
  int max_cols = 16;
  while (max_cols > 0 && !gv_plan(max_cols, a.k, HALVES).stages) --max_cols;
  const int max_rows = (SPLIT ? max_cols / 2 : max_cols);
  if (max_rows < 1) return fail(MRB_ERR_UNSUPPORTED, "qrow gemv: in_features %lld too large", (long long)a.k);
  for (int64_t r0 = 0; r0 < a.m; r0 += max_rows) {
    GemvArgs part = a;
    part.m = std::min<int64_t>(max_rows, a.m - r0);
    part.x = reinterpret_cast<const XT*>(a.x) + r0 * a.k;
    part.y = a.y ? reinterpret_cast<YT*>(a.y) + r0 * a.n : nullptr;
    if (a.packed) part.packed = a.packed + r0;
    const int pcols = SPLIT ? 2 * (int)part.m : (int)part.m;
    const int st = pcols <= 8 ? launch_gemv<XT, YT, SPLIT, 1, EPI>(part, ws, s)
                              : launch_gemv<XT, YT, SPLIT, 2, EPI>(part, ws, s);
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

bool tc_w8a16_supported(const void* x, int64_t k, const int8_t* codes, const int8_t* up_codes);
int tc_w8a16_argmax(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                    int64_t n, int64_t semantic, float* logits, unsigned long long* packed, cudaStream_t s);
int tc_w8a16_gemm(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                  const int8_t* up_codes, const float* up_scales, int64_t n, const float* bias, __nv_bfloat16* y,
                  cudaStream_t s);
int qrow_gemm_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                   int64_t n, const float* bias, __nv_bfloat16* y, cudaStream_t s);
bool qrow_skinny_supported(int64_t m, int64_t n, int64_t k);
int qrow_skinny_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* codes, const float* scales,
                     int64_t n, const float* bias, __nv_bfloat16* y, cudaStream_t s);
int qrow_gemm_swiglu_bf16(const __nv_bfloat16* x, int64_t m, int64_t k, const int8_t* gate_codes,
                          const float* gate_scales, const int8_t* up_codes, const float* up_scales, int64_t n,
                          __nv_bfloat16* y, cudaStream_t s);

// Activation rows above which bf16 projections (and the greedy head) use the tensor-core
// GEMM: one GEMV launch stages at most 16 activation rows per CTA, and a wider block makes
// that staging cost more than the weight stream it serves.
#ifndef MRB_GEMV_MAX_ROWS
#define MRB_GEMV_MAX_ROWS 16
#endif
constexpr int64_t GEMV_MAX_ROWS = MRB_GEMV_MAX_ROWS;

static GemvArgs make_args(const void* x, int64_t m, int64_t k, const int8_t* c0, const float* s0, const int8_t* c1,
                          const float* s1, const float* bias, int64_t n, void* y) {
  GemvArgs a{};
  a.x = x; a.m = m; a.k = k; a.codes0 = c0; a.scales0 = s0; a.codes1 = c1; a.scales1 = s1;
  a.bias = bias; a.n = n; a.y = y;
  return a;
}

static int qrow_gemv_dispatch(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* codes,
                              const float* scales, int64_t n, const float* bias, void* y, GvWorkspace ws,
                              cudaStream_t s) {
  const GemvArgs a = make_args(x, m, k, codes, scales, nullptr, nullptr, bias, n, y);
  switch (x_dtype) {
    case MRB_BF16:
      if (m > GEMV_MAX_ROWS) {
        // 17-32 rows: the skinny kernel (weights in registers, cluster split-K)
        if (qrow_skinny_supported(m, n, k))
          return qrow_skinny_bf16((const __nv_bfloat16*)x, m, k, codes, scales, n, bias, (__nv_bfloat16*)y, s);
        if (tc_w8a16_supported(x, k, codes, nullptr))
          return tc_w8a16_gemm((const __nv_bfloat16*)x, m, k, codes, scales, nullptr, nullptr, n, bias,
                               (__nv_bfloat16*)y, s);
        return qrow_gemm_bf16((const __nv_bfloat16*)x, m, k, codes, scales, n, bias, (__nv_bfloat16*)y, s);
      }
      return dispatch_nt<__nv_bfloat16, __nv_bfloat16, false, EPI_STORE>(a, ws, s);
    case MRB_F16: return dispatch_nt<__half, __half, false, EPI_STORE>(a, ws, s);
    case MRB_F32: return dispatch_nt<float, float, true, EPI_STORE>(a, ws, s);
    default: return fail(MRB_ERR_ARG, "qrow_matmul: bad x_dtype %d", x_dtype);
  }
}

static int check_workspace(const void* workspace, size_t workspace_bytes, const char* what) {
  if (workspace && !aligned(workspace, 256)) return fail(MRB_ERR_ARG, "%s: workspace must be 256-byte aligned", what);
  if (!workspace && workspace_bytes) return fail(MRB_ERR_ARG, "%s: workspace size without a workspace", what);
  return MRB_OK;
}

}  // namespace mrb

using namespace mrb;

extern "C" size_t mrb_qrow_workspace(int64_t n) {
  if (n <= 0) return 0;
  return gv_workspace_bytes(n);
}

extern "C" int mrb_qrow_matmul(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* codes,
                               const float* scales, int64_t n, const float* bias, void* y, int y_dtype,
                               void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_common(x, m, k, codes, scales, n, y, "qrow_matmul");
  if (st) return st;
  if ((st = check_workspace(workspace, workspace_bytes, "qrow_matmul"))) return st;
  if (y_dtype != x_dtype) return fail(MRB_ERR_ARG, "qrow_matmul: output dtype must equal activation dtype");
  if (m == 0) return MRB_OK;
  return qrow_gemv_dispatch(x, x_dtype, m, k, codes, scales, n, bias, y, GvWorkspace{workspace, workspace_bytes},
                            (cudaStream_t)stream);
}

extern "C" int mrb_qrow_swiglu(const void* x_bf16, int64_t m, int64_t k, const int8_t* gate_codes,
                               const float* gate_scales, const int8_t* up_codes, const float* up_scales,
                               int64_t n, void* y_bf16, void* workspace, size_t workspace_bytes, void* stream) {
  int st = check_common(x_bf16, m, k, gate_codes, gate_scales, n, y_bf16, "qrow_swiglu");
  if (st) return st;
  if ((st = check_workspace(workspace, workspace_bytes, "qrow_swiglu"))) return st;
  if (!up_codes || !up_scales) return fail(MRB_ERR_ARG, "qrow_swiglu: null up page");
  if (!aligned(up_codes, 16)) return fail(MRB_ERR_ARG, "qrow_swiglu: codes must be 16-byte aligned");
  if (m == 0) return MRB_OK;
  if (m > GEMV_MAX_ROWS) {
    if (tc_w8a16_supported(x_bf16, k, gate_codes, up_codes))
      return tc_w8a16_gemm((const __nv_bfloat16*)x_bf16, m, k, gate_codes, gate_scales, up_codes, up_scales, n,
                           nullptr, (__nv_bfloat16*)y_bf16, (cudaStream_t)stream);
    return qrow_gemm_swiglu_bf16((const __nv_bfloat16*)x_bf16, m, k, gate_codes, gate_scales, up_codes, up_scales,
                                 n, (__nv_bfloat16*)y_bf16, (cudaStream_t)stream);
  }
  const GemvArgs a = make_args(x_bf16, m, k, gate_codes, gate_scales, up_codes, up_scales, nullptr, n, y_bf16);
  return dispatch_nt<__nv_bfloat16, __nv_bfloat16, false, EPI_SWIGLU>(a, GvWorkspace{workspace, workspace_bytes},
                                                                      (cudaStream_t)stream);
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
    case MRB_BF16:
      // many rows: one tensor-core pass over the head instead of one GEMV pass per 16 rows
      if (m > GEMV_MAX_ROWS && tc_w8a16_supported(x, k, codes, nullptr))
        st = tc_w8a16_argmax((const __nv_bfloat16*)x, m, k, codes, scales, n, semantic_rows, logits, a.packed, s);
      else
        st = dispatch_nt<__nv_bfloat16, float, false, EPI_ARGMAX>(a, GvWorkspace{}, s);
      break;
    case MRB_F16: st = dispatch_nt<__half, float, false, EPI_ARGMAX>(a, GvWorkspace{}, s); break;
    case MRB_F32: st = dispatch_nt<float, float, true, EPI_ARGMAX>(a, GvWorkspace{}, s); break;
    default: return fail(MRB_ERR_ARG, "qrow_argmax: bad x_dtype %d", x_dtype);
  }
  if (st) return st;
  argmax_unpack_kernel<<<(unsigned)((m + 127) / 128), 128, 0, s>>>(reinterpret_cast<unsigned long long*>(out_index),
                                                                    out_value, m);
  return launch_status("qrow_argmax");
}
