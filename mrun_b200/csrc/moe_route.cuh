// The route compiler (stable expert-major order of the reference's CPU branch,
// engine/olmoe_cuda.py:989-1135) as a block-level routine: one block of RC_THREADS threads
// ranks `assignments` (token, slot) choices by expert with __match_any_sync, producing
// counts, starts, token ids, coefficients and the inverse permutation. Ids outside [0, E)
// are left out (and flagged in *error_flag when one is given). Shared by the route-compile
// kernel and the expert-parallel receive kernel.
#pragma once

#include "qrow_common.cuh"

namespace mrb {

constexpr int RC_THREADS = 1024;
constexpr int RC_WARPS = RC_THREADS / 32;
constexpr int RC_MAXE = 512;

__device__ __forceinline__ void route_compile_block(const int64_t* __restrict__ top_idx, const float* __restrict__ top_w,
                                                    int64_t assignments, int k, int E, int32_t* __restrict__ counts,
                                                    int32_t* __restrict__ starts, int64_t* __restrict__ token_ids,
                                                    float* __restrict__ coef, int64_t* __restrict__ inverse,
                                                    int32_t* __restrict__ error_flag) {
  __shared__ int hist[RC_MAXE];
  __shared__ int cursor[RC_MAXE];
  __shared__ int whist[RC_WARPS][RC_MAXE / 4];  // reused per expert quarter
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

}  // namespace mrb
