// Expert-parallel token exchange over peer memory: one process per GPU, every
// rank owning a contiguous range of each layer's experts.
//
// The reference's only expert-parallel code (the DeepSeek remote code,
// models/deepseek/modeling_deepseek.py:604-660) counts the tokens per rank,
// exchanges the counts, sends every token row only to the ranks that own one
// of its experts (all_to_all with those splits), runs the local experts, and
// sends the outputs back the same way.  Here the same exchange is two kernels
// that write and read the other GPUs' memory directly over NVLink, so that a
// layer needs no host synchronisation and can be captured in a CUDA graph:
//
//   blut_ep_dispatch  stores each token row (with its local expert ids and
//                     weights) into the window of every rank that owns one of
//                     its experts, at the next free row of this rank's region
//                     there; then publishes the row count and a flag to every
//                     rank, and waits for every rank's flag to reach this
//                     exchange's epoch.
//   (the caller runs blut_moe_forward on its own window's received rows and
//    writes the fp32 results into the window's output region)
//   blut_ep_combine   flags every rank that this rank's output rows are in
//                     place, waits for every rank's flag, then sums for each of
//                     its own tokens the output rows the owners hold for it
//                     (peer loads, in rank order) plus the shared expert's
//                     output, and rounds once.
//
// Every rank runs both kernels once per layer, with or without rows for a
// peer, so the epochs (a per-window counter the dispatch advances) stay
// equal across ranks.  A rank writes a peer's input region for exchange e+1
// only after its own combine of exchange e saw that peer's flag, which the
// peer raises after its experts finished reading the region; the same
// handshake protects the output regions, so one window serves every layer.
// Every wait is bounded (the library's wait limit): on timeout the kernel
// records a status bit, marks the rows it could not trust empty and returns.
// No load or store uses cluster multicast.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "blut_common.cuh"
#include "blut_internal.h"

namespace blut {
namespace {

constexpr int kEpRanks = BLUT_EP_MAX_RANKS;
constexpr int kEpThreads = 256;

// First 256 bytes of a window.  flags_in / count_in / flags_ret are written
// by peers; the rest only by this rank.
struct EpCtl {
  int flags_in[kEpRanks];   // [s] epoch of source s's last dispatch into this window
  int count_in[kEpRanks];   // [s] rows source s placed in its region
  int flags_ret[kEpRanks];  // [d] epoch whose output rows owner d holds for this rank
  int epoch;                // exchanges this rank has dispatched
  int done;                 // CTAs of the running dispatch that have finished
  int status;               // kDevTimeout when a wait gave up
};
static_assert(sizeof(EpCtl) <= 256, "window header");

// Byte offsets of a window's regions (each 256-byte aligned).
struct EpLayout {
  int64_t slot;  // [cap][kEpRanks] int32: row of own token t in rank d's region (-1: not sent)
  int64_t x;     // [world][cap][hidden] f16/bf16: rows received from each source
  int64_t ids;   // [world][cap][top_k] int32: their local expert ids (-1: not owned here)
  int64_t w;     // [world][cap][top_k] f32: their routing weights
  int64_t ret;   // [world][cap][hidden] f32: this rank's expert outputs for each source's rows
  int64_t total;
};

__host__ __device__ inline EpLayout ep_layout(int world, int cap, int hidden, int top_k) {
  auto al = [](int64_t v) { return (v + 255) & ~(int64_t)255; };
  EpLayout L;
  int64_t o = 256;
  L.slot = o;
  o = al(o + (int64_t)cap * kEpRanks * 4);
  L.x = o;
  o = al(o + (int64_t)world * cap * hidden * 2);
  L.ids = o;
  o = al(o + (int64_t)world * cap * top_k * 4);
  L.w = o;
  o = al(o + (int64_t)world * cap * top_k * 4);
  L.ret = o;
  o = al(o + (int64_t)world * cap * hidden * 4);
  L.total = o;
  return L;
}

struct EpArgs {
  uint8_t* win[kEpRanks];  // window of every rank as mapped in this process
  int world, rank, cap, hidden, top_k;
  EpLayout L;
  uint64_t wait_ns;
};

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag has reached epoch e (flags only grow; a peer is never
// more than one exchange ahead of the rank that waits for it).  Once a wait
// of this rank has given up (status set, until blut_ep_check_status clears
// it), later waits give up at once, so a rank whose peer is gone drains its
// queued exchanges quickly instead of waiting out every one.
__device__ bool ep_wait_flag(const int* flag, int e, const int* status, uint64_t limit_ns) {
  if (ld_acquire_sys(flag) - e >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0; i < (1u << 31); ++i) {
    if (*reinterpret_cast<const volatile int*>(status) & kDevTimeout) return false;
    __nanosleep(256);
    if (ld_acquire_sys(flag) - e >= 0) return true;
    if ((i & 15) == 15 && globaltimer_ns() - t0 > limit_ns) return false;
  }
  return false;
}

// Ranks owning at least one valid expert of token i (bit d set for rank d).
__device__ __forceinline__ uint32_t ep_dest_mask(const int* __restrict__ ids, int i, int top_k,
                                                 const int* __restrict__ owner, int num_experts, int world) {
  uint32_t m = 0;
  for (int j = 0; j < top_k; ++j) {
    const int id = ids[(int64_t)i * top_k + j];
    if (id >= 0 && id < num_experts) {
      const int d = owner[id];
      if (d >= 0 && d < world) m |= 1u << d;
    }
  }
  return m;
}

// Per-rank counts of tokens [0, n) with a row for that rank, into cnt[] (shared).
__device__ void ep_count_rows(const int* __restrict__ ids, int n, int top_k, const int* __restrict__ owner,
                              int num_experts, int world, int* cnt) {
  int c[kEpRanks];
#pragma unroll
  for (int d = 0; d < kEpRanks; ++d) c[d] = 0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t m = ep_dest_mask(ids, i, top_k, owner, num_experts, world);
#pragma unroll
    for (int d = 0; d < kEpRanks; ++d) c[d] += (m >> d) & 1u;
  }
#pragma unroll
  for (int d = 0; d < kEpRanks; ++d)
    if (c[d]) atomicAdd(cnt + d, c[d]);
}

// One CTA per own token (one CTA when T == 0, carrying only the flags).
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(const EpArgs a, const uint16_t* __restrict__ x,
                                                                 const int* __restrict__ ids,
                                                                 const float* __restrict__ tw, int T,
                                                                 const int* __restrict__ owner,
                                                                 const int* __restrict__ local, int num_experts) {
  uint8_t* mine = a.win[a.rank];
  EpCtl* ctl = reinterpret_cast<EpCtl*>(mine);
  const int e = ctl->epoch + 1;  // only the last CTA of this launch advances it, after every CTA read it
  const int K = a.top_k, H = a.hidden, W = a.world;
  __shared__ int cnt[kEpRanks];
  __shared__ uint32_t tmask;
  __shared__ int last, all_ok;
  if (threadIdx.x < kEpRanks) cnt[threadIdx.x] = 0;
  __syncthreads();
  const int t = blockIdx.x;
  // the row of token t at rank d is the number of earlier tokens with a row there
  ep_count_rows(ids, min(t, T), K, owner, num_experts, W, cnt);
  if (threadIdx.x == 0) tmask = t < T ? ep_dest_mask(ids, t, K, owner, num_experts, W) : 0u;
  __syncthreads();
  int* send_slot = reinterpret_cast<int*>(mine + a.L.slot);
  if (t < T) {
    const uint32_t m = tmask;
    for (int d = 0; d < W; ++d) {
      const bool to_d = (m >> d) & 1u;
      const int slot = cnt[d];
      if (threadIdx.x == 0) send_slot[(int64_t)t * kEpRanks + d] = to_d ? slot : -1;
      if (!to_d) continue;
      uint8_t* peer = a.win[d];
      const int64_t row = (int64_t)a.rank * a.cap + slot;
      const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)t * H);
      uint4* dst = reinterpret_cast<uint4*>(peer + a.L.x + row * H * 2);
      for (int v = threadIdx.x; v < H / 8; v += blockDim.x) dst[v] = src[v];
      for (int j = threadIdx.x; j < K; j += blockDim.x) {
        const int id = ids[(int64_t)t * K + j];
        const bool own = id >= 0 && id < num_experts && owner[id] == d;
        reinterpret_cast<int*>(peer + a.L.ids)[row * K + j] = own ? local[id] : -1;
        reinterpret_cast<float*>(peer + a.L.w)[row * K + j] = tw[(int64_t)t * K + j];
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&ctl->done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  // -- the launch's last CTA: every row of this rank is stored --
  __threadfence_system();
  if (threadIdx.x < kEpRanks) cnt[threadIdx.x] = 0;
  if (threadIdx.x == 0) {
    ctl->done = 0;
    all_ok = 1;
  }
  __syncthreads();
  ep_count_rows(ids, T, K, owner, num_experts, W, cnt);
  __syncthreads();
  if (threadIdx.x < W) {
    EpCtl* pc = reinterpret_cast<EpCtl*>(a.win[threadIdx.x]);
    pc->count_in[a.rank] = cnt[threadIdx.x];
    __threadfence_system();
    st_release_sys(&pc->flags_in[a.rank], e);
  }
  // wait for every source's rows (this rank's own included)
  if (threadIdx.x < W && !ep_wait_flag(&ctl->flags_in[threadIdx.x], e, &ctl->status, a.wait_ns)) {
    atomicOr(&ctl->status, kDevTimeout);
    all_ok = 0;
  }
  __syncthreads();
  // rows past a source's count still hold an earlier exchange's ids (or the
  // window's zeros): mark them empty; after a timeout, every row
  int* rids = reinterpret_cast<int*>(mine + a.L.ids);
  const int ok = all_ok;
  for (int64_t idx = threadIdx.x; idx < (int64_t)W * a.cap; idx += blockDim.x) {
    const int s = (int)(idx / a.cap), r = (int)(idx - (int64_t)s * a.cap);
    const int n = ok ? ld_acquire_sys(&ctl->count_in[s]) : 0;
    if (r >= n)
      for (int j = 0; j < K; ++j) rids[idx * K + j] = -1;
  }
  if (threadIdx.x == 0) ctl->epoch = e;
}

// One CTA per (own token, 1024 columns); (1, 1) when T == 0.
template <bool BF16>
__global__ void __launch_bounds__(kEpThreads) ep_combine_kernel(const EpArgs a, int T,
                                                                const float* __restrict__ shared,
                                                                void* __restrict__ out, int out_f32) {
  uint8_t* mine = a.win[a.rank];
  EpCtl* ctl = reinterpret_cast<EpCtl*>(mine);
  const int e = ctl->epoch;
  const int W = a.world, H = a.hidden;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  // this rank's output rows for every source were written by the launches
  // before this one: tell every rank (any CTA may be first, so every CTA does)
  if (threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(&reinterpret_cast<EpCtl*>(a.win[threadIdx.x])->flags_ret[a.rank], e);
  }
  __syncthreads();
  if (threadIdx.x < W && !ep_wait_flag(&ctl->flags_ret[threadIdx.x], e, &ctl->status, a.wait_ns)) {
    atomicOr(&ctl->status, kDevTimeout);
    ok = 0;
  }
  __syncthreads();
  const int t = blockIdx.x;
  const int h = (blockIdx.y * blockDim.x + threadIdx.x) * 4;
  if (t >= T || h >= H) return;
  const int* send_slot = reinterpret_cast<const int*>(mine + a.L.slot) + (int64_t)t * kEpRanks;
  float4 v[kEpRanks];
#pragma unroll
  for (int d = 0; d < kEpRanks; ++d) {
    v[d] = make_float4(0.f, 0.f, 0.f, 0.f);
    const int slot = d < W && ok ? send_slot[d] : -1;
    if (slot >= 0 && slot < a.cap)
      v[d] = __ldcv(reinterpret_cast<const float4*>(a.win[d] + a.L.ret) +
                    (((int64_t)a.rank * a.cap + slot) * H + h) / 4);
  }
  float4 acc = v[0];
#pragma unroll
  for (int d = 1; d < kEpRanks; ++d) {
    acc.x += v[d].x; acc.y += v[d].y; acc.z += v[d].z; acc.w += v[d].w;
  }
  if (shared) {
    const float4 s = *reinterpret_cast<const float4*>(shared + (int64_t)t * H + h);
    acc.x += s.x; acc.y += s.y; acc.z += s.z; acc.w += s.w;
  }
  if (out_f32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + (int64_t)t * H + h) = acc;
  } else {
    uint2 o;
    o.x = uint32_t(f32_to_act<BF16>(acc.x)) | (uint32_t(f32_to_act<BF16>(acc.y)) << 16);
    o.y = uint32_t(f32_to_act<BF16>(acc.z)) | (uint32_t(f32_to_act<BF16>(acc.w)) << 16);
    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + (int64_t)t * H + h) = o;
  }
}

bool ep_valid(const blut_ep_desc* d) {
  if (!d || d->world < 1 || d->world > kEpRanks || d->rank < 0 || d->rank >= d->world || d->capacity < 1 ||
      d->hidden < 8 || d->hidden % 8 != 0 || d->top_k < 1 || d->top_k > 64 ||
      (d->dtype != BLUT_F16 && d->dtype != BLUT_BF16))
    return false;
  for (int r = 0; r < d->world; ++r)
    if (!d->windows[r] || reinterpret_cast<uintptr_t>(d->windows[r]) % 256 != 0) return false;
  return true;
}

EpArgs ep_args(const blut_ep_desc* d) {
  EpArgs a{};
  for (int r = 0; r < kEpRanks; ++r) a.win[r] = r < d->world ? static_cast<uint8_t*>(d->windows[r]) : nullptr;
  a.world = d->world;
  a.rank = d->rank;
  a.cap = d->capacity;
  a.hidden = d->hidden;
  a.top_k = d->top_k;
  a.L = ep_layout(d->world, d->capacity, d->hidden, d->top_k);
  a.wait_ns = wait_limit_ns();
  return a;
}

}  // namespace
}  // namespace blut

using namespace blut;

extern "C" {

BLUT_API size_t blut_ep_window_bytes(int world, int capacity, int hidden, int top_k) {
  if (world < 1 || world > kEpRanks || capacity < 1 || hidden < 8 || hidden % 8 || top_k < 1 || top_k > 64) return 0;
  return (size_t)ep_layout(world, capacity, hidden, top_k).total;
}

BLUT_API int blut_ep_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return BLUT_ERR_INVALID;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return BLUT_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return BLUT_ERR_CUDA;
  }
  *ptr = p;
  return BLUT_OK;
}

BLUT_API int blut_ep_free(void* ptr) {
  if (!ptr) return BLUT_OK;
  return cudaFree(ptr) == cudaSuccess ? BLUT_OK : BLUT_ERR_CUDA;
}

BLUT_API int blut_ep_ipc_handle(const void* ptr, void* handle) {
  if (!ptr || !handle) return BLUT_ERR_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == BLUT_EP_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return BLUT_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return BLUT_OK;
}

BLUT_API int blut_ep_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return BLUT_ERR_INVALID;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return BLUT_ERR_CUDA;
  *ptr = p;
  return BLUT_OK;
}

BLUT_API int blut_ep_ipc_close(void* ptr) {
  if (!ptr) return BLUT_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? BLUT_OK : BLUT_ERR_CUDA;
}

BLUT_API int blut_ep_views(const blut_ep_desc* d, void** x, int32_t** ids, float** w, float** ret) {
  if (!ep_valid(d)) return BLUT_ERR_INVALID;
  const EpLayout L = ep_layout(d->world, d->capacity, d->hidden, d->top_k);
  uint8_t* mine = static_cast<uint8_t*>(d->windows[d->rank]);
  if (x) *x = mine + L.x;
  if (ids) *ids = reinterpret_cast<int32_t*>(mine + L.ids);
  if (w) *w = reinterpret_cast<float*>(mine + L.w);
  if (ret) *ret = reinterpret_cast<float*>(mine + L.ret);
  return BLUT_OK;
}

BLUT_API int blut_ep_dispatch(const blut_ep_desc* d, const void* x, const int32_t* topk_ids,
                              const float* topk_weights, int num_tokens, const int32_t* owner,
                              const int32_t* local, int num_experts, void* stream) {
  if (!ep_valid(d) || num_tokens < 0 || num_tokens > d->capacity || num_experts < 1 || !owner || !local ||
      (num_tokens > 0 && (!x || !topk_ids || !topk_weights)) || reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return BLUT_ERR_INVALID;
  const EpArgs a = ep_args(d);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  ep_dispatch_kernel<<<num_tokens > 0 ? num_tokens : 1, kEpThreads, 0, s>>>(
      a, static_cast<const uint16_t*>(x), topk_ids, topk_weights, num_tokens, owner, local, num_experts);
  return stage_done("ep dispatch", s);
}

BLUT_API int blut_ep_combine(const blut_ep_desc* d, int num_tokens, const float* shared_out, void* out,
                             int out_f32, void* stream) {
  if (!ep_valid(d) || num_tokens < 0 || num_tokens > d->capacity || (num_tokens > 0 && !out) ||
      reinterpret_cast<uintptr_t>(out) % 16 != 0 || reinterpret_cast<uintptr_t>(shared_out) % 16 != 0)
    return BLUT_ERR_INVALID;
  const EpArgs a = ep_args(d);
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(num_tokens > 0 ? num_tokens : 1, (d->hidden + 4 * kEpThreads - 1) / (4 * kEpThreads));
  if (d->dtype == BLUT_BF16)
    ep_combine_kernel<true><<<grid, kEpThreads, 0, s>>>(a, num_tokens, shared_out, out, out_f32);
  else
    ep_combine_kernel<false><<<grid, kEpThreads, 0, s>>>(a, num_tokens, shared_out, out, out_f32);
  return stage_done("ep combine", s);
}

BLUT_API int blut_ep_check_status(const blut_ep_desc* d, void* stream) {
  if (!ep_valid(d)) return BLUT_ERR_INVALID;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return BLUT_ERR_CUDA;
  int* st = &reinterpret_cast<EpCtl*>(d->windows[d->rank])->status;
  int v = 0;
  if (cudaMemcpy(&v, st, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return BLUT_ERR_CUDA;
  if (v == 0) return BLUT_OK;
  const int zero = 0;
  if (cudaMemcpy(st, &zero, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) return BLUT_ERR_CUDA;
  return BLUT_ERR_TIMEOUT;
}

}  // extern "C"
