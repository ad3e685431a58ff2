// Head-sharded forward: exchange buffers, their route table, and the device
// signal / wait between ranks.
//
// Each rank's exchange buffer holds what other ranks store into it during a
// block: the q|k planes and transposed v planes of this rank's heads (written
// by every rank's Q|K|V projection epilogue) and the context planes of this
// rank's positions (written by every rank's attention epilogue).  A rank
// signals after its stores by writing an epoch count into every rank's
// signal words with a system-scope release; a reader waits until all ranks'
// words reach the epoch with system-scope acquire loads.  The epoch counter
// lives in device memory, so a captured CUDA graph replays correctly.
//
// Every wait is bounded by the group's timeout; when it runs out the waiter
// sets NSRL_FLAG_WAIT_TIMEOUT and returns, so a rank that never signals
// ends the call with an error instead of a hung GPU.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "internal.h"

namespace nsrl {

namespace {

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

struct PostArgs {
  const ShardTable* tab;
  unsigned long long* epoch;  // this rank's counter
  int nranks, rank;
  const nsrl_device_status* post;  // optional: status words to post
};

struct WaitArgs {
  const ShardTable* tab;
  const unsigned long long* epoch;
  int nranks, rank, combine;
  unsigned long long limit_ns;
  nsrl_device_status* st;
};

// Thread t < n of one warp: post (optionally) the status words into this
// rank's slot of rank t, then signal rank t with epoch e.  The kernel boundary
// orders the stores of the kernels before it; the system-scope fence makes
// them visible to the other GPUs before the release store of the signal.
__device__ __forceinline__ void post_one(const PostArgs& a, int t, unsigned long long e) {
  if (a.post) {
    unsigned long long* slot = a.tab->slots[t] + 4 * a.rank;
    slot[0] = a.post->flags;
    slot[1] = a.post->attention_saturations;
    slot[2] = a.post->mlp_saturations;
  }
  __threadfence_system();
  st_release_sys(a.tab->signal[t] + a.rank, e);
}

// Thread t < n: wait (bounded) for rank t's signal of epoch e; with combine,
// fetch the status words rank t posted.  Returns whether the signal came.
__device__ __forceinline__ bool wait_one(const WaitArgs& a, int t, unsigned long long e,
                                         unsigned long long (&got)[kMaxShardRanks][3]) {
  const unsigned long long* sig = a.tab->signal[a.rank] + t;
  bool done = ld_acquire_sys(sig) >= e;
  if (!done) {
    const unsigned long long t0 = global_ns();
    while (!done) {
      __nanosleep(100);
      done = ld_acquire_sys(sig) >= e;
      if (!done && global_ns() - t0 > a.limit_ns) break;
    }
  }
  if (!done) nsrl_flag(a.st, NSRL_FLAG_WAIT_TIMEOUT);
  if (done && a.combine && t != a.rank) {
    const unsigned long long* slot = a.tab->slots[a.rank] + 4 * t;
    got[t][0] = slot[0];
    got[t][1] = slot[1];
    got[t][2] = slot[2];
  }
  return done;
}

// Adds the other ranks' posted status words into this rank's status (thread 0).
__device__ __forceinline__ void combine(const WaitArgs& a, const int (&ok)[kMaxShardRanks],
                                        const unsigned long long (&got)[kMaxShardRanks][3]) {
  unsigned long long f = 0, as = 0, ms = 0;
  for (int p = 0; p < a.nranks; ++p) {
    if (p == a.rank || !ok[p]) continue;
    f |= got[p][0];
    as += got[p][1];
    ms += got[p][2];
  }
  if (f) nsrl_flag(a.st, f);
  if (as) atomicAdd(&a.st->attention_saturations, as);
  if (ms) atomicAdd(&a.st->mlp_saturations, ms);
}

// mode 1: post; mode 2: wait (the epoch of this rank's last post); mode 3:
// post, then wait -- the form for ranks in separate processes.
__global__ void shard_sync_kernel(const PostArgs pa, const WaitArgs wa, int mode) {
  __shared__ unsigned long long e;
  __shared__ unsigned long long got[kMaxShardRanks][3];
  __shared__ int ok[kMaxShardRanks];
  if (threadIdx.x == 0) {
    e = *pa.epoch + ((mode & 1) ? 1 : 0);
    if (mode & 1) *pa.epoch = e;
  }
  __syncwarp();
  const int t = threadIdx.x;
  if (t < pa.nranks) {
    if (mode & 1) post_one(pa, t, e);
    if (mode & 2) ok[t] = wait_one(wa, t, e, got) ? 1 : 0;
  }
  __syncwarp();
  if (t == 0 && (mode & 2) && wa.combine) combine(wa, ok, got);
}

struct PushArgs {
  const ShardTable* tab;   // destinations: every rank's exchange regions
  const uint8_t* own;      // this rank's exchange buffer (its staging slots)
  size_t stage, stride;    // slot p at own + stage + p * stride
  size_t slot_qk_lo, slot_vt_hi, slot_vt_lo;  // regions within a slot (q|k hi at 0)
  long long S, s_loc, d_loc, B;
  int nranks, rank;
  long long qk_chunks, vt_chunks, per_peer;  // 16-byte chunks of one plane of q|k and of v, and per peer
};

// Grid-stride copy in 16-byte chunks: for each other rank p, its q|k rows of
// this rank's positions (one run of s_loc * 2 d_loc bytes per sequence) and
// its v rows (one run of s_loc bytes per (sequence, column)), hi and lo
// planes, from the staging slot to the same offsets of p's regions.
__global__ void shard_push_kernel(const PushArgs a) {
  const long long total = (long long)(a.nranks - 1) * a.per_peer;
  const long long qk_run = a.s_loc * 2 * a.d_loc / 16;
  const long long vt_run = a.s_loc / 16;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int q = (int)(i / a.per_peer);
    const int p = q < a.rank ? q : q + 1;
    long long j = i - (long long)q * a.per_peer;
    const uint8_t* slot = a.own + a.stage + (size_t)p * a.stride;
    const uint8_t* src;
    uint8_t* dst;
    if (j < 2 * a.qk_chunks) {
      const int plane = (int)(j / a.qk_chunks);
      const long long k = j - plane * a.qk_chunks;
      const long long b = k / qk_run, c = k - b * qk_run;
      const long long off = (b * a.S + a.rank * a.s_loc) * 2 * a.d_loc + c * 16;
      src = slot + (plane ? a.slot_qk_lo : 0) + off;
      dst = (plane ? a.tab->qk_lo[p] : reinterpret_cast<uint8_t*>(a.tab->qk_hi[p])) + off;
    } else {
      j -= 2 * a.qk_chunks;
      const int plane = (int)(j / a.vt_chunks);
      const long long k = j - plane * a.vt_chunks;
      const long long row = k / vt_run, c = k - row * vt_run;
      const long long off = row * a.S + a.rank * a.s_loc + c * 16;
      src = slot + (plane ? a.slot_vt_lo : a.slot_vt_hi) + off;
      dst = (plane ? a.tab->vt_lo[p] : reinterpret_cast<uint8_t*>(a.tab->vt_hi[p])) + off;
    }
    *reinterpret_cast<uint4*>(dst) = __ldg(reinterpret_cast<const uint4*>(src));
  }
}

}  // namespace

bool shard_layout(size_t B, size_t S, size_t d, size_t H, size_t n, ShardLayout* L) {
  if (n == 0 || n > (size_t)kMaxShardRanks || B == 0 || S == 0 || d == 0 || H == 0) return false;
  if (S % n != 0 || H % n != 0 || d % H != 0) return false;
  ShardLayout l;
  l.B = B;
  l.S = S;
  l.d = d;
  l.H = H;
  l.n = n;
  l.s_loc = S / n;
  l.h_loc = H / n;
  l.d_loc = d / n;
  size_t off = kShardHeaderBytes;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = al256(off + bytes);
    return o;
  };
  l.qk_hi = take(B * S * 2 * l.d_loc);
  l.qk_lo = take(B * S * 2 * l.d_loc);
  l.vt_hi = take(B * l.d_loc * S);
  l.vt_lo = take(B * l.d_loc * S);
  l.ctx_hi = take(B * l.s_loc * d);
  l.ctx_lo = take(B * l.s_loc * d);
  l.ctx_l1 = take(B * l.s_loc * sizeof(unsigned long long));
  if (n > 1 && l.s_loc % 16 == 0) {  // staging slots: q|k hi, lo, v hi, lo of one destination each
    l.stage = off;
    const size_t slot = al256(B * S * 2 * l.d_loc) * 2 + al256(B * l.d_loc * S) * 2;
    l.stage_stride = slot;
    off += n * slot;
  }
  l.total = off;
  *L = l;
  return true;
}

namespace {
cudaError_t launch_sync(const nsrl_shard_group* g, int mode, const nsrl_device_status* post, bool combine,
                        nsrl_device_status* st, cudaStream_t s, const char* name) {
  PostArgs pa;
  pa.tab = g->tab;
  pa.epoch = reinterpret_cast<unsigned long long*>(g->base[g->rank] + kShardEpochOff);
  pa.nranks = g->nranks;
  pa.rank = g->rank;
  pa.post = post;
  WaitArgs wa;
  wa.tab = g->tab;
  wa.epoch = pa.epoch;
  wa.nranks = g->nranks;
  wa.rank = g->rank;
  wa.combine = combine ? 1 : 0;
  wa.limit_ns = g->timeout_ns;
  wa.st = st;
  ProfScope prof(name, s, 0.0, 0.0);
  shard_sync_kernel<<<1, 32, 0, s>>>(pa, wa, mode);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_shard_post(const nsrl_shard_group* g, const nsrl_device_status* post_status, cudaStream_t s) {
  return launch_sync(g, 1, post_status, false, nullptr, s, "shard_post");
}

cudaError_t launch_shard_wait(const nsrl_shard_group* g, bool combine, nsrl_device_status* st, cudaStream_t s) {
  return launch_sync(g, 2, nullptr, combine, st, s, "shard_wait");
}

cudaError_t launch_shard_barrier(const nsrl_shard_group* g, const nsrl_device_status* post, bool combine,
                                 nsrl_device_status* st, cudaStream_t s) {
  return launch_sync(g, 3, post, combine, st, s, "shard_barrier");
}

cudaError_t launch_shard_push(const nsrl_shard_group* g, cudaStream_t s) {
  const ShardLayout& L = g->L;
  if (!g->stab || g->nranks < 2) return cudaSuccess;
  PushArgs a;
  a.tab = g->tab;
  a.own = g->base[g->rank];
  a.stage = L.stage;
  a.stride = L.stage_stride;
  a.slot_qk_lo = al256(L.B * L.S * 2 * L.d_loc);
  a.slot_vt_hi = 2 * a.slot_qk_lo;
  a.slot_vt_lo = a.slot_vt_hi + al256(L.B * L.d_loc * L.S);
  a.S = (long long)L.S;
  a.s_loc = (long long)L.s_loc;
  a.d_loc = (long long)L.d_loc;
  a.B = (long long)L.B;
  a.nranks = g->nranks;
  a.rank = g->rank;
  a.qk_chunks = a.B * a.s_loc * 2 * a.d_loc / 16;
  a.vt_chunks = a.B * a.d_loc * a.s_loc / 16;
  a.per_peer = 2 * a.qk_chunks + 2 * a.vt_chunks;
  const long long total = (long long)(g->nranks - 1) * a.per_peer;
  const unsigned blocks = (unsigned)std::min<long long>((total + 255) / 256, 148 * 8);
  ProfScope prof("shard_push", s, 0.0, 2.0 * 16.0 * (double)total);
  shard_push_kernel<<<blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace nsrl

using namespace nsrl;

namespace {
nsrl_status shard_cuda_fail(cudaError_t e, const char* what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return NSRL_CUDA_ERROR;
}
}  // namespace

extern "C" {

size_t nsrl_shard_exchange_bytes(size_t batch, size_t seq_len, size_t d_model, size_t heads, size_t nranks) {
  ShardLayout L;
  return shard_layout(batch, seq_len, d_model, heads, nranks, &L) ? L.total : 0;
}

nsrl_status nsrl_shard_alloc(size_t bytes, void** buffer) {
  if (!buffer || bytes == 0) {
    set_error("nsrl_shard_alloc: NULL buffer or zero bytes");
    return NSRL_INVALID_SHAPE;
  }
  *buffer = nullptr;
  cudaError_t e = cudaMalloc(buffer, bytes);
  if (e != cudaSuccess) return shard_cuda_fail(e, "exchange buffer");
  e = cudaMemset(*buffer, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(*buffer);
    *buffer = nullptr;
    return shard_cuda_fail(e, "exchange buffer");
  }
  return NSRL_OK;
}

nsrl_status nsrl_shard_free(void* buffer) {
  if (!buffer) return NSRL_OK;
  const cudaError_t e = cudaFree(buffer);
  return e == cudaSuccess ? NSRL_OK : shard_cuda_fail(e, "exchange buffer free");
}

nsrl_status nsrl_ipc_get_handle(const void* buffer, uint8_t handle[NSRL_IPC_HANDLE_BYTES]) {
  static_assert(sizeof(cudaIpcMemHandle_t) == NSRL_IPC_HANDLE_BYTES, "IPC handle size");
  if (!buffer || !handle) {
    set_error("nsrl_ipc_get_handle: NULL argument");
    return NSRL_INVALID_SHAPE;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(buffer));
  if (e != cudaSuccess) return shard_cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle, &h, sizeof(h));
  return NSRL_OK;
}

nsrl_status nsrl_ipc_open(const uint8_t handle[NSRL_IPC_HANDLE_BYTES], void** buffer) {
  if (!buffer || !handle) {
    set_error("nsrl_ipc_open: NULL argument");
    return NSRL_INVALID_SHAPE;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *buffer = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(buffer, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? NSRL_OK : shard_cuda_fail(e, "cudaIpcOpenMemHandle");
}

nsrl_status nsrl_ipc_close(void* buffer) {
  if (!buffer) return NSRL_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(buffer);
  return e == cudaSuccess ? NSRL_OK : shard_cuda_fail(e, "cudaIpcCloseMemHandle");
}

nsrl_status nsrl_shard_group_create(nsrl_shard_group** group, int nranks, int rank, void* const* exchange,
                                    size_t exchange_bytes, size_t batch, size_t seq_len, size_t d_model,
                                    size_t heads, uint64_t timeout_ms) {
  if (!group || !exchange) {
    set_error("nsrl_shard_group_create: NULL argument");
    return NSRL_INVALID_SHAPE;
  }
  *group = nullptr;
  if (nranks < 1 || nranks > kMaxShardRanks || rank < 0 || rank >= nranks) {
    set_error("nsrl_shard_group_create: need 1 <= nranks <= %d and 0 <= rank < nranks", kMaxShardRanks);
    return NSRL_INVALID_SHAPE;
  }
  ShardLayout L;
  if (!shard_layout(batch, seq_len, d_model, heads, (size_t)nranks, &L)) {
    set_error("nsrl_shard_group_create: seq_len and heads must be multiples of nranks (d_model of heads)");
    return NSRL_INVALID_SHAPE;
  }
  if (!attention_tc_supported(seq_len, L.d_loc, L.h_loc)) {
    set_error("nsrl_shard_group_create: head_dim 64, seq_len a multiple of 16 and at most 16384 required");
    return NSRL_INVALID_SHAPE;
  }
  if (exchange_bytes < L.total) {
    set_error("nsrl_shard_group_create: exchange buffers of %zu bytes, %zu needed", exchange_bytes, L.total);
    return NSRL_INVALID_SHAPE;
  }
  for (int r = 0; r < nranks; ++r)
    if (!exchange[r] || (reinterpret_cast<uintptr_t>(exchange[r]) & 255) != 0) {
      set_error("nsrl_shard_group_create: exchange buffer %d is NULL or not 256-byte aligned", r);
      return NSRL_INVALID_SHAPE;
    }
  nsrl_shard_group* g = new nsrl_shard_group();
  g->nranks = nranks;
  g->rank = rank;
  g->L = L;
  g->timeout_ns = (timeout_ms ? timeout_ms : 10000ull) * 1000000ull;
  cudaGetDevice(&g->device);
  ShardTable t;
  memset(&t, 0, sizeof(t));
  for (int r = 0; r < nranks; ++r) {
    uint8_t* b = static_cast<uint8_t*>(exchange[r]);
    g->base[r] = b;
    t.qk_hi[r] = reinterpret_cast<int8_t*>(b + L.qk_hi);
    t.qk_lo[r] = b + L.qk_lo;
    t.vt_hi[r] = reinterpret_cast<int8_t*>(b + L.vt_hi);
    t.vt_lo[r] = b + L.vt_lo;
    t.ctx_hi[r] = reinterpret_cast<int8_t*>(b + L.ctx_hi);
    t.ctx_lo[r] = b + L.ctx_lo;
    t.ctx_l1[r] = reinterpret_cast<unsigned long long*>(b + L.ctx_l1);
    t.signal[r] = reinterpret_cast<unsigned long long*>(b + kShardSignalOff);
    t.slots[r] = reinterpret_cast<unsigned long long*>(b + kShardSlotsOff);
  }
  cudaError_t e = cudaMalloc(&g->tab, sizeof(ShardTable));
  if (e == cudaSuccess) e = cudaMemcpy(g->tab, &t, sizeof(t), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && L.stage) {
    // the projection's view: other ranks' q|k and v in this rank's staging slots
    ShardTable st = t;
    uint8_t* own = g->base[rank];
    const size_t qk = al256(L.B * L.S * 2 * L.d_loc), vt = al256(L.B * L.d_loc * L.S);
    for (int r = 0; r < nranks; ++r) {
      if (r == rank) continue;
      uint8_t* slot = own + L.stage + (size_t)r * L.stage_stride;
      st.qk_hi[r] = reinterpret_cast<int8_t*>(slot);
      st.qk_lo[r] = slot + qk;
      st.vt_hi[r] = reinterpret_cast<int8_t*>(slot + 2 * qk);
      st.vt_lo[r] = slot + 2 * qk + vt;
    }
    e = cudaMalloc(&g->stab, sizeof(ShardTable));
    if (e == cudaSuccess) e = cudaMemcpy(g->stab, &st, sizeof(st), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaMemset(g->base[rank], 0, kShardHeaderBytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (g->tab) cudaFree(g->tab);
    if (g->stab) cudaFree(g->stab);
    delete g;
    return shard_cuda_fail(e, "shard group");
  }
  *group = g;
  return NSRL_OK;
}

nsrl_status nsrl_shard_group_destroy(nsrl_shard_group* group) {
  if (!group) return NSRL_OK;
  cudaError_t e = cudaSuccess;
  if (group->tab) e = cudaFree(group->tab);
  if (group->stab && e == cudaSuccess) e = cudaFree(group->stab);
  delete group;
  return e == cudaSuccess ? NSRL_OK : shard_cuda_fail(e, "shard group free");
}

nsrl_status nsrl_shard_status_post(const nsrl_shard_group* group, const nsrl_device_status* status, void* stream) {
  if (!group || !status) {
    set_error("nsrl_shard_status_post: NULL argument");
    return NSRL_INVALID_SHAPE;
  }
  const cudaError_t e = launch_shard_post(group, status, (cudaStream_t)stream);
  return e == cudaSuccess ? NSRL_OK : shard_cuda_fail(e, "status post");
}

nsrl_status nsrl_shard_status_allreduce(const nsrl_shard_group* group, nsrl_device_status* status, void* stream) {
  if (!group || !status) {
    set_error("nsrl_shard_status_allreduce: NULL argument");
    return NSRL_INVALID_SHAPE;
  }
  const cudaError_t e = launch_shard_barrier(group, status, true, status, (cudaStream_t)stream);
  return e == cudaSuccess ? NSRL_OK : shard_cuda_fail(e, "status all-reduce");
}

nsrl_status nsrl_shard_status_combine(const nsrl_shard_group* group, nsrl_device_status* status, void* stream) {
  if (!group || !status) {
    set_error("nsrl_shard_status_combine: NULL argument");
    return NSRL_INVALID_SHAPE;
  }
  const cudaError_t e = launch_shard_wait(group, true, status, (cudaStream_t)stream);
  return e == cudaSuccess ? NSRL_OK : shard_cuda_fail(e, "status combine");
}

}  // extern "C"
