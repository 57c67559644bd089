// Expert-parallel dispatch and return over NVLink peer memory (one process per GPU).
//
// Every rank owns one "mailbox" in its HBM, mapped into every peer through CUDA IPC:
//   [dispatch flags: world u32 | return flags: world u32 | counts: world i32 |
//    ids: world x capacity i32 | rows: world x capacity x hidden bf16 |
//    back: world x capacity x hidden bf16]
// Dispatch (source rank r): the rows of the fixed-capacity plan (mrb_ep_pack) are stored
// straight into destination d's mailbox, rows[r][pos] and ids[r][pos], with plain stores over
// NVLink -- only the real rows, no padding crosses the link. The last CTA to finish (a local
// arrival counter) writes counts[r] = rows sent to each destination, fences at system scope
// and release-stores dispatch_flag[r] = epoch in every destination's mailbox.
// Receive: one thread per source acquire-loads its flag until it equals the epoch (bounded
// spin), then the ids of unused slots are set to the dummy local expert and all ids are
// widened to int64 for the route compiler; the grouped expert MLP reads rows in place.
// Return (destination d): expert outputs go straight back into the source's mailbox,
// back[d * capacity + j], then flags as above; the source waits for every destination's
// return flag and the fixed-rank combine reads its back rows.
// The epoch is a per-exchange device counter, advanced by the dispatch's last CTA, so a
// CUDA graph replays the exchange with fresh flag values. Buffer reuse is safe without extra
// barriers: a rank dispatches into layer L's mailboxes again only after its own combine of
// layer L, which waited for every owner's return, which each owner issued after reading the
// rows. Every wait is bounded (mrb_ep_set_wait_limit polls, 2^22 by default): on a timeout
// the kernel sets state[3] (error) and proceeds, so the step completes and the host can
// read the error.
// No TMA and no cluster multicast is involved; peers are reached by ordinary loads/stores.
#include "qrow_common.cuh"
#include "moe_route.cuh"

#include <algorithm>
#include <cstring>

namespace mrb {

constexpr size_t EPM_ALIGN = 256;
constexpr int EPM_MAX_WORLD = 64;
constexpr int EPM_SPIN = 1 << 22;  // default bound of a wait: polls with a short sleep between them
// Poll bound given to the wait kernels launched from now on (a captured graph keeps the value
// it was captured with). mrb_ep_set_wait_limit changes it; tests shorten it to make a wait run
// out quickly.
static int g_epm_spin_limit = EPM_SPIN;

struct MailboxLayout {
  size_t flags_dispatch, flags_return, counts, ids, rows, back, total;
};

__host__ __device__ inline size_t epm_up(size_t v) { return (v + EPM_ALIGN - 1) & ~(EPM_ALIGN - 1); }

__host__ __device__ inline MailboxLayout epm_layout(int64_t world, int64_t cap, int64_t hidden) {
  MailboxLayout m{};
  m.flags_dispatch = 0;
  m.flags_return = EPM_ALIGN;
  m.counts = 2 * EPM_ALIGN;
  m.ids = 3 * EPM_ALIGN;
  m.rows = m.ids + epm_up((size_t)(world * cap) * 4);
  m.back = m.rows + epm_up((size_t)(world * cap * hidden) * 2);
  m.total = m.back + epm_up((size_t)(world * cap * hidden) * 2);
  return m;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// state: [0] epoch of the last dispatch, [1] dispatch arrivals, [2] return arrivals, [3] error

__global__ void ep_p2p_dispatch_kernel(const __nv_bfloat16* __restrict__ x, int64_t hidden,
                                       const int32_t* __restrict__ slot_src, const int32_t* __restrict__ send_expert,
                                       int world, int rank, int cap, unsigned char* const* __restrict__ mailboxes,
                                       MailboxLayout lay, int32_t* __restrict__ state) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned epoch = (unsigned)state[0] + 1u;  // advanced by the last CTA below
  const int slots = world * cap;
  const int vecs = (int)(hidden / 8);
  for (int s = blockIdx.x; s < slots; s += gridDim.x) {
    const int src = slot_src[s];
    if (src < 0) continue;
    const int d = s / cap, j = s - d * cap;
    unsigned char* mb = mailboxes[d];
    uint4* out = reinterpret_cast<uint4*>(mb + lay.rows) + ((int64_t)rank * cap + j) * vecs;
    const uint4* in = reinterpret_cast<const uint4*>(x + (int64_t)src * hidden);
    for (int i = threadIdx.x; i < vecs; i += blockDim.x) out[i] = __ldg(in + i);
    if (threadIdx.x == 0) reinterpret_cast<int32_t*>(mb + lay.ids)[rank * cap + j] = send_expert[s];
  }
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(state + 1, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  // rows to each destination: the plan fills every block from position 0
  for (int d = threadIdx.x; d < world; d += blockDim.x) {
    int count = 0;
    while (count < cap && slot_src[d * cap + count] >= 0) ++count;
    reinterpret_cast<int32_t*>(mailboxes[d] + lay.counts)[rank] = count;
  }
  __threadfence_system();
  __syncthreads();
  for (int d = threadIdx.x; d < world; d += blockDim.x)
    st_release_sys(reinterpret_cast<unsigned*>(mailboxes[d] + lay.flags_dispatch) + rank, epoch);
  if (threadIdx.x == 0) {
    state[1] = 0;
    state[0] = (int32_t)epoch;
  }
}

__device__ bool epm_wait_flags(const unsigned* flags, int world, unsigned epoch, int spin_limit) {
  bool ok = true;
  for (int s = threadIdx.x; s < world; s += blockDim.x) {
    int i = 0;
    while (ld_acquire_sys(flags + s) != epoch) {
      if (++i >= spin_limit) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  return __syncthreads_and(ok);
}

__global__ void ep_p2p_wait_dispatch_kernel(unsigned char* __restrict__ mailbox, MailboxLayout lay, int world, int cap,
                                            int dummy, int64_t* __restrict__ ids64, int32_t* __restrict__ state,
                                            int spin_limit) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned epoch = (unsigned)state[0];
  const bool ok =
      epm_wait_flags(reinterpret_cast<const unsigned*>(mailbox + lay.flags_dispatch), world, epoch, spin_limit);
  if (!ok && threadIdx.x == 0) state[3] = 1;
  const int32_t* counts = reinterpret_cast<const int32_t*>(mailbox + lay.counts);
  const int32_t* ids = reinterpret_cast<const int32_t*>(mailbox + lay.ids);
  for (int s = threadIdx.x; s < world * cap; s += blockDim.x) {
    const int src = s / cap, j = s - src * cap;
    const int id = ids[s];
    const bool real = ok && j < counts[src] && id >= 0 && id < dummy;
    ids64[s] = real ? id : dummy;
  }
}

__global__ void ep_p2p_return_kernel(const __nv_bfloat16* __restrict__ eo, const int64_t* __restrict__ inverse,
                                     int64_t hidden, int world, int rank, int cap,
                                     unsigned char* const* __restrict__ mailboxes, MailboxLayout lay,
                                     int32_t* __restrict__ state) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned epoch = (unsigned)state[0];
  const int32_t* counts = reinterpret_cast<const int32_t*>(mailboxes[rank] + lay.counts);
  const int vecs = (int)(hidden / 8);
  for (int s = blockIdx.x; s < world * cap; s += gridDim.x) {
    const int src = s / cap, j = s - src * cap;
    if (j >= counts[src]) continue;
    const uint4* in = reinterpret_cast<const uint4*>(eo + inverse[s] * hidden);
    uint4* out = reinterpret_cast<uint4*>(mailboxes[src] + lay.back) + ((int64_t)rank * cap + j) * vecs;
    for (int i = threadIdx.x; i < vecs; i += blockDim.x) out[i] = in[i];
  }
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(state + 2, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence_system();
  for (int d = threadIdx.x; d < world; d += blockDim.x)
    st_release_sys(reinterpret_cast<unsigned*>(mailboxes[d] + lay.flags_return) + rank, epoch);
  if (threadIdx.x == 0) state[2] = 0;
}

__global__ void ep_p2p_wait_return_kernel(unsigned char* __restrict__ mailbox, MailboxLayout lay, int world,
                                          int32_t* __restrict__ state, int spin_limit) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned epoch = (unsigned)state[0];
  const bool ok =
      epm_wait_flags(reinterpret_cast<const unsigned*>(mailbox + lay.flags_return), world, epoch, spin_limit);
  if (!ok && threadIdx.x == 0) state[3] = 1;
}

// The receive side of a dispatch and the route compile in one CTA of RC_THREADS threads (one
// launch instead of two on every layer's critical path): wait for every source's flag, keep
// the local expert id of each real row (padding slots get -1, so the route compiler leaves
// them out and ranks only the rows that arrived), then compile the routes over those ids.
__global__ void __launch_bounds__(RC_THREADS) ep_p2p_wait_route_kernel(
    unsigned char* __restrict__ mailbox, MailboxLayout lay, int world, int cap, int experts_local,
    int64_t* __restrict__ ids64, const float* __restrict__ coef_in, int32_t* __restrict__ counts_out,
    int32_t* __restrict__ starts, int64_t* __restrict__ token_ids, float* __restrict__ coef,
    int64_t* __restrict__ inverse, int32_t* __restrict__ state, int spin_limit) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned epoch = (unsigned)state[0];
  const bool ok =
      epm_wait_flags(reinterpret_cast<const unsigned*>(mailbox + lay.flags_dispatch), world, epoch, spin_limit);
  if (!ok && threadIdx.x == 0) state[3] = 1;
  const int32_t* counts = reinterpret_cast<const int32_t*>(mailbox + lay.counts);
  const int32_t* ids = reinterpret_cast<const int32_t*>(mailbox + lay.ids);
  for (int s = threadIdx.x; s < world * cap; s += blockDim.x) {
    const int src = s / cap, j = s - src * cap;
    const int id = ids[s];
    const bool real = ok && j < counts[src] && id >= 0 && id < experts_local;
    ids64[s] = real ? id : -1;
  }
  __syncthreads();  // the ids are stored (block scope) before the block ranks them
  route_compile_block(ids64, coef_in, (int64_t)world * cap, 1, experts_local, counts_out, starts, token_ids, coef,
                      inverse, nullptr);
}

// The source side of a return and the fixed-rank combine in one launch: every CTA waits for
// every owner's return flag (bounded), then combines as stable_route_reduce_kernel does --
// out[t, h] = sum over r < k, in rank order, of coef[p] * float(back[p, h]), p =
// slot_of_assign[t*k + r], each product rounded to fp32 and added left to right.
__global__ void ep_p2p_combine_kernel(unsigned char* __restrict__ mailbox, MailboxLayout lay, int world,
                                      const float* __restrict__ coef, const int64_t* __restrict__ slot_of_assign,
                                      int64_t tokens, int k, int64_t H, __nv_bfloat16* __restrict__ out,
                                      int32_t* __restrict__ state, int spin_limit) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned epoch = (unsigned)state[0];
  const bool ok =
      epm_wait_flags(reinterpret_cast<const unsigned*>(mailbox + lay.flags_return), world, epoch, spin_limit);
  if (!ok && threadIdx.x == 0) state[3] = 1;
  const __nv_bfloat16* eo = reinterpret_cast<const __nv_bfloat16*>(mailbox + lay.back);
  const int64_t t = blockIdx.y;
  for (int64_t h = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; h < H; h += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < k; ++r) {
      const int64_t p = slot_of_assign[t * k + r];
      const float prod = __fmul_rn(__bfloat162float(__ldcg(eo + p * H + h)), coef[p]);
      acc = r == 0 ? prod : __fadd_rn(acc, prod);
    }
    out[t * H + h] = __float2bfloat16_rn(acc);
  }
}

static int ep_check(int64_t world, int64_t rank, int64_t cap, int64_t hidden, const char* what) {
  if (world < 1 || world > EPM_MAX_WORLD || rank < 0 || rank >= world || cap < 1 || hidden <= 0 || hidden % 8)
    return fail(MRB_ERR_ARG, "%s: bad shape", what);
  if (world * cap > 0x7fffffffLL) return fail(MRB_ERR_UNSUPPORTED, "%s: too many slots", what);
  return MRB_OK;
}

static int ep_grid(int64_t slots) { return (int)std::max<int64_t>(1, std::min<int64_t>(slots, 2 * num_sms())); }

}  // namespace mrb

using namespace mrb;

extern "C" int mrb_ep_set_wait_limit(int64_t polls) {
  if (polls < 1 || polls > (1LL << 30)) return fail(MRB_ERR_ARG, "ep_set_wait_limit: polls must be in [1, 2^30]");
  g_epm_spin_limit = (int)polls;
  clear_error();
  return MRB_OK;
}

extern "C" int64_t mrb_ep_wait_limit(void) { return g_epm_spin_limit; }

extern "C" size_t mrb_ep_mailbox_bytes(int64_t world, int64_t capacity, int64_t hidden) {
  if (world < 1 || world > EPM_MAX_WORLD || capacity < 1 || hidden <= 0) return 0;
  return epm_layout(world, capacity, hidden).total;
}

extern "C" int mrb_ep_mailbox_offsets(int64_t world, int64_t capacity, int64_t hidden, int64_t* out6) {
  if (!out6) return fail(MRB_ERR_ARG, "ep_mailbox_offsets: null pointer");
  if (world < 1 || world > EPM_MAX_WORLD || capacity < 1 || hidden <= 0)
    return fail(MRB_ERR_ARG, "ep_mailbox_offsets: bad shape");
  const MailboxLayout m = epm_layout(world, capacity, hidden);
  out6[0] = (int64_t)m.flags_dispatch;
  out6[1] = (int64_t)m.flags_return;
  out6[2] = (int64_t)m.counts;
  out6[3] = (int64_t)m.ids;
  out6[4] = (int64_t)m.rows;
  out6[5] = (int64_t)m.back;
  return MRB_OK;
}

extern "C" int mrb_ep_mailbox_create(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return fail(MRB_ERR_ARG, "ep_mailbox_create: bad argument");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "ep_mailbox_create: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(MRB_ERR_CUDA, "ep_mailbox_create: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return MRB_OK;
}

extern "C" int mrb_ep_mailbox_open(const void* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return fail(MRB_ERR_ARG, "ep_mailbox_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "ep_mailbox_open: %s", cudaGetErrorString(e));
  return MRB_OK;
}

extern "C" int mrb_ep_mailbox_close(void* ptr, int owned) {
  if (!ptr) return MRB_OK;
  cudaError_t e = owned ? cudaFree(ptr) : cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return fail(MRB_ERR_CUDA, "ep_mailbox_close: %s", cudaGetErrorString(e));
  return MRB_OK;
}

extern "C" int mrb_ep_p2p_dispatch(const void* x_bf16, int64_t hidden, const int32_t* slot_src,
                                   const int32_t* send_expert, int64_t world, int64_t rank, int64_t capacity,
                                   void* const* mailboxes, int32_t* state, void* stream) {
  int st = ep_check(world, rank, capacity, hidden, "ep_p2p_dispatch");
  if (st) return st;
  if (!x_bf16 || !slot_src || !send_expert || !mailboxes || !state)
    return fail(MRB_ERR_ARG, "ep_p2p_dispatch: null pointer");
  if (!aligned(x_bf16, 16)) return fail(MRB_ERR_ARG, "ep_p2p_dispatch: rows must be 16-byte aligned");
  const MailboxLayout lay = epm_layout(world, capacity, hidden);
  launch_kernel(ep_p2p_dispatch_kernel, dim3(ep_grid(world * capacity)), dim3(128), 0, (cudaStream_t)stream, true,
                (const __nv_bfloat16*)x_bf16, hidden, slot_src, send_expert, (int)world, (int)rank, (int)capacity,
                (unsigned char* const*)mailboxes, lay, state);
  return launch_status("ep_p2p_dispatch");
}

extern "C" int mrb_ep_p2p_wait_dispatch(void* mailbox, int64_t world, int64_t capacity, int64_t hidden,
                                        int32_t dummy_expert, int64_t* ids64, int32_t* state, void* stream) {
  int st = ep_check(world, 0, capacity, hidden, "ep_p2p_wait_dispatch");
  if (st) return st;
  if (!mailbox || !ids64 || !state) return fail(MRB_ERR_ARG, "ep_p2p_wait_dispatch: null pointer");
  const MailboxLayout lay = epm_layout(world, capacity, hidden);
  launch_kernel(ep_p2p_wait_dispatch_kernel, dim3(1), dim3(256), 0, (cudaStream_t)stream, true,
                (unsigned char*)mailbox, lay, (int)world, (int)capacity, (int)dummy_expert, ids64, state,
                g_epm_spin_limit);
  return launch_status("ep_p2p_wait_dispatch");
}

extern "C" int mrb_ep_p2p_return(const void* eo_bf16, const int64_t* inverse, int64_t hidden, int64_t world,
                                 int64_t rank, int64_t capacity, void* const* mailboxes, int32_t* state,
                                 void* stream) {
  int st = ep_check(world, rank, capacity, hidden, "ep_p2p_return");
  if (st) return st;
  if (!eo_bf16 || !inverse || !mailboxes || !state) return fail(MRB_ERR_ARG, "ep_p2p_return: null pointer");
  if (!aligned(eo_bf16, 16)) return fail(MRB_ERR_ARG, "ep_p2p_return: rows must be 16-byte aligned");
  const MailboxLayout lay = epm_layout(world, capacity, hidden);
  launch_kernel(ep_p2p_return_kernel, dim3(ep_grid(world * capacity)), dim3(128), 0, (cudaStream_t)stream, true,
                (const __nv_bfloat16*)eo_bf16, inverse, hidden, (int)world, (int)rank, (int)capacity,
                (unsigned char* const*)mailboxes, lay, state);
  return launch_status("ep_p2p_return");
}

extern "C" int mrb_ep_p2p_wait_return(void* mailbox, int64_t world, int64_t capacity, int64_t hidden, int32_t* state,
                                      void* stream) {
  int st = ep_check(world, 0, capacity, hidden, "ep_p2p_wait_return");
  if (st) return st;
  if (!mailbox || !state) return fail(MRB_ERR_ARG, "ep_p2p_wait_return: null pointer");
  const MailboxLayout lay = epm_layout(world, capacity, hidden);
  launch_kernel(ep_p2p_wait_return_kernel, dim3(1), dim3(64), 0, (cudaStream_t)stream, true, (unsigned char*)mailbox,
                lay, (int)world, state, g_epm_spin_limit);
  return launch_status("ep_p2p_wait_return");
}

extern "C" int mrb_ep_p2p_wait_route(void* mailbox, int64_t world, int64_t capacity, int64_t hidden,
                                     int64_t experts_local, int64_t* ids64, const float* coef_in, int32_t* counts,
                                     int32_t* starts, int64_t* token_ids, float* coef, int64_t* inverse, int32_t* state,
                                     void* stream) {
  int st = ep_check(world, 0, capacity, hidden, "ep_p2p_wait_route");
  if (st) return st;
  if (experts_local < 1 || experts_local > RC_MAXE)
    return fail(MRB_ERR_UNSUPPORTED, "ep_p2p_wait_route: 1 to %d local experts", RC_MAXE);
  if (!mailbox || !ids64 || !coef_in || !counts || !starts || !token_ids || !coef || !inverse || !state)
    return fail(MRB_ERR_ARG, "ep_p2p_wait_route: null pointer");
  launch_kernel(ep_p2p_wait_route_kernel, dim3(1), dim3(RC_THREADS), 0, (cudaStream_t)stream, true,
                (unsigned char*)mailbox, epm_layout(world, capacity, hidden), (int)world, (int)capacity,
                (int)experts_local, ids64, coef_in, counts, starts, token_ids, coef, inverse, state, g_epm_spin_limit);
  return launch_status("ep_p2p_wait_route");
}

extern "C" int mrb_ep_p2p_combine(void* mailbox, int64_t world, int64_t capacity, int64_t hidden, const float* coef,
                                  const int64_t* slot_of_assign, int64_t tokens, int64_t k, void* out_bf16,
                                  int32_t* state, void* stream) {
  int st = ep_check(world, 0, capacity, hidden, "ep_p2p_combine");
  if (st) return st;
  if (tokens < 0 || k <= 0 || tokens * k > capacity) return fail(MRB_ERR_ARG, "ep_p2p_combine: bad shape");
  if (tokens == 0) return MRB_OK;
  if (tokens > 65535) return fail(MRB_ERR_UNSUPPORTED, "ep_p2p_combine: at most 65535 tokens per call");
  if (!mailbox || !coef || !slot_of_assign || !out_bf16 || !state) return fail(MRB_ERR_ARG, "ep_p2p_combine: null pointer");
  const unsigned bx = (unsigned)std::min<int64_t>((hidden + 255) / 256, 64);
  launch_kernel(ep_p2p_combine_kernel, dim3(bx, (unsigned)tokens), dim3(256), 0, (cudaStream_t)stream, true,
                (unsigned char*)mailbox, epm_layout(world, capacity, hidden), (int)world, coef, slot_of_assign, tokens,
                (int)k, hidden, (__nv_bfloat16*)out_bf16, state, g_epm_spin_limit);
  return launch_status("ep_p2p_combine");
}
