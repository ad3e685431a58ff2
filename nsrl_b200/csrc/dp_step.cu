// The data-parallel training step behind the C ABI: windows -> exchange ->
// apply, with no host round trip between them.
//
// Reference: crates/nsrl-train/src/lib.rs:6970-7399 (map-reduce batch),
// :7401-7471 (ordered, checked merge of the workers' accumulators),
// :6249-6400 (the shift optimizer's apply), :4270-4465 (the integer-Adam
// batch apply), crates/nsrl-train-core/src/lib.rs:386-465 and :469-661 (the
// per-element rules), :1732-1775 (rounding helpers).
//
// Per step, on the caller's stream:
//   1. nsrl_train_windows runs this rank's windows into a private gradient
//      arena [arena | counts | batch stats] (one int64 vector).
//   2. bound_kernel: max |x| over the vector and this rank's rejection flag.
//   3. One NCCL group: all-reduce MAX of {max |x|, rejected} and all-reduce
//      SUM of the vector (out of place: the local vector is kept).
//   4. decide_kernel: a rejection anywhere rejects the batch on every rank
//      (lib.rs:5371-5375); else nranks * max|x| <= i64::MAX proves that no
//      prefix of any merge order leaves i64, so the sum is the reference's
//      ordered merge; else the step falls back to an all-gather and the
//      ordered merge with overflow detection (merge_kernel), as the
//      reference's checked adds in worker order.  decide_kernel also turns
//      the accepted-window count into every apply shift on the device.
//   5. apply_kernel: ONE launch over the whole arena, driven by a segment
//      table (offset, length, weights, kind, count index, shift class, Adam
//      state offset), skipped unless the decision is "apply".
// The host waits once, at the end, polling the event and the communicator
// against its deadline.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <climits>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "internal.h"

#define NSRL_FLAG_BATCH_REJECTED 0x200ull   // another rank (or the merge) rejected the batch
#define NSRL_FLAG_INVALID_CONFIG 0x400ull   // a shift went below the batch shift (InvalidConfig)

// --------------------------------------------------------------- NCCL ------
namespace nsrl {
namespace {

struct NcclApi {
  bool ok = false;
  std::string err;
  decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&ncclCommInitRankConfig) CommInitRankConfig = nullptr;
  decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&ncclCommAbort) CommAbort = nullptr;
  decltype(&ncclCommFinalize) CommFinalize = nullptr;
  decltype(&ncclCommDestroy) CommDestroy = nullptr;
  decltype(&ncclAllReduce) AllReduce = nullptr;
  decltype(&ncclAllGather) AllGather = nullptr;
  decltype(&ncclGroupStart) GroupStart = nullptr;
  decltype(&ncclGroupEnd) GroupEnd = nullptr;
  decltype(&ncclGetErrorString) GetErrorString = nullptr;
};

// NCCL is loaded on first use, so that the library loads (and its
// single-GPU entry points run) where no NCCL is installed.  A process that
// already holds libnccl.so.2 (PyTorch's copy) gets that one.
NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      api.err = std::string("cannot load libnccl.so.2: ") + dlerror();
      return;
    }
    bool ok = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      ok = ok && fn != nullptr;
    };
    get(api.GetUniqueId, "ncclGetUniqueId");
    get(api.CommInitRankConfig, "ncclCommInitRankConfig");
    get(api.CommGetAsyncError, "ncclCommGetAsyncError");
    get(api.CommAbort, "ncclCommAbort");
    get(api.CommFinalize, "ncclCommFinalize");
    get(api.CommDestroy, "ncclCommDestroy");
    get(api.AllReduce, "ncclAllReduce");
    get(api.AllGather, "ncclAllGather");
    get(api.GroupStart, "ncclGroupStart");
    get(api.GroupEnd, "ncclGroupEnd");
    get(api.GetErrorString, "ncclGetErrorString");
    if (!ok) {
      api.err = "libnccl.so.2 lacks a non-blocking communicator entry point (NCCL >= 2.14 needed)";
      return;
    }
    api.ok = true;
  });
  return api;
}

// ------------------------------------------------------- bounded waits -----
// One wait of the host on the device or the communicator, with a deadline.
// The step uses it with real CUDA / NCCL queries; nsrl_comm_selftest_wait
// runs the same loop on fakes.
struct WaitOps {
  void* ctx;
  int (*done)(void* ctx);        // 1 finished, 0 pending, -1 a CUDA error
  int (*comm_error)(void* ctx);  // 0 none, else the error code
  void (*abort)(void* ctx);
  uint64_t (*now_ns)(void* ctx);
  void (*pause)(void* ctx);
};

nsrl_status wait_bounded(const WaitOps& o, uint64_t timeout_ns, const char* what, uint64_t* polls = nullptr) {
  const uint64_t t0 = o.now_ns(o.ctx);
  for (uint64_t n = 1;; ++n) {
    if (polls) *polls = n;
    const int d = o.done(o.ctx);
    if (d > 0) return NSRL_OK;
    if (d < 0) {
      if (o.abort) o.abort(o.ctx);  // the peers then fail instead of waiting for this rank
      set_error("%s: a CUDA error on this rank", what);
      return NSRL_CUDA_ERROR;
    }
    const int ce = o.comm_error ? o.comm_error(o.ctx) : 0;
    if (ce != 0) {
      if (o.abort) o.abort(o.ctx);
      set_error("%s: the communicator reported error %d (a peer failed or left); it is aborted", what, ce);
      return NSRL_COMM_ERROR;
    }
    if (o.now_ns(o.ctx) - t0 > timeout_ns) {
      if (o.abort) o.abort(o.ctx);
      set_error("%s: not finished after %llu ms; the communicator is aborted", what,
                (unsigned long long)(timeout_ns / 1000000ull));
      return NSRL_COMM_TIMEOUT;
    }
    o.pause(o.ctx);
  }
}

uint64_t steady_ns(void*) {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}
void short_pause(void*) { std::this_thread::sleep_for(std::chrono::microseconds(20)); }

}  // namespace
}  // namespace nsrl

struct nsrl_comm {
  ncclComm_t comm = nullptr;
  int nranks = 1, rank = 0, device = 0;
  uint64_t timeout_ns = 0;
  bool dead = false;
  cudaEvent_t ev = nullptr;
};

namespace nsrl {
namespace {

struct CommWait {
  nsrl_comm* c;
  cudaEvent_t ev;  // null: wait for the communicator's own pending work
};

int comm_async(nsrl_comm* c) {
  ncclResult_t r = ncclSuccess;
  if (nccl().CommGetAsyncError(c->comm, &r) != ncclSuccess) return (int)ncclInternalError;
  return (int)r;
}

WaitOps comm_ops(CommWait* w) {
  WaitOps o{};
  o.ctx = w;
  o.done = [](void* p) -> int {
    CommWait* w = static_cast<CommWait*>(p);
    if (!w->ev) {
      const int r = comm_async(w->c);
      return r == (int)ncclSuccess ? 1 : 0;  // in progress: pending; errors go to comm_error
    }
    const cudaError_t e = cudaEventQuery(w->ev);
    if (e == cudaSuccess) return 1;
    if (e == cudaErrorNotReady) return 0;
    return -1;
  };
  o.comm_error = [](void* p) -> int {
    CommWait* w = static_cast<CommWait*>(p);
    if (!w->c) return 0;
    const int r = comm_async(w->c);
    return (r == (int)ncclSuccess || r == (int)ncclInProgress) ? 0 : r;
  };
  o.abort = [](void* p) {
    CommWait* w = static_cast<CommWait*>(p);
    if (w->c && !w->c->dead) {
      w->c->dead = true;
      nccl().CommAbort(w->c->comm);
    }
  };
  o.now_ns = steady_ns;
  o.pause = short_pause;
  return o;
}

// After a non-blocking NCCL call returned ncclInProgress, its operations are
// enqueued on the stream only once the communicator's state leaves
// in-progress: wait for that (bounded) before the next launch.
nsrl_status comm_settle(nsrl_comm* c, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return NSRL_OK;
  if (r != ncclInProgress) {
    c->dead = true;
    nccl().CommAbort(c->comm);
    set_error("%s: %s; the communicator is aborted", what, nccl().GetErrorString(r));
    return NSRL_COMM_ERROR;
  }
  CommWait w{c, nullptr};
  return wait_bounded(comm_ops(&w), c->timeout_ns, what);
}

// ----------------------------------------------------------- kernels -------
enum Decision : int { DEC_APPLY = 0, DEC_REJECT = 1, DEC_MERGE = 2, DEC_INVALID = 3 };
enum SegKind : int { SEG_SGD_I8 = 0, SEG_SGD_EMB_I16 = 1, SEG_ADAM_I8 = 2, SEG_ADAM_I16 = 3 };

constexpr int MAX_SEGS = 128;
constexpr int APPLY_THREADS = 256;
constexpr int APPLY_PER = 16;
constexpr int APPLY_BATCH = 8;  // loads a thread issues before their arithmetic
constexpr int APPLY_TILE = APPLY_THREADS * APPLY_PER;  // elements of one apply tile

struct ApplySeg {
  long long off;        // first element in the arena
  long long len;
  void* w;              // int8_t* (SGD_I8, ADAM_I8) or int16_t*
  long long state_off;  // Adam state index of the first element
  int kind;
  int count_idx;
  int shift_class;      // SGD: index into the shift table
  int tile0;            // first apply tile of the segment
};

struct ApplyTable {
  int nseg, ntiles;
  ApplySeg seg[MAX_SEGS];
};

// Shift table layout: [0] output head, [1] embeddings, then per layer l:
// [2 + 4l] MLP, [3 + 4l] attention (v, o), [4 + 4l] q, [5 + 4l] k.
struct ShiftCfg {
  int lr;
  int output, mlp, embedding, attention, attention_q, attention_qk;
  int layers;
};

__device__ __forceinline__ bool add_ovf(long long a, long long b, long long& out) {
  const long long s = (long long)((unsigned long long)a + (unsigned long long)b);
  out = s;
  return ((a ^ s) & (b ^ s)) < 0;
}
__device__ __forceinline__ bool mul_ovf(long long a, long long b, long long& out) {
  const long long lo = (long long)((unsigned long long)a * (unsigned long long)b);
  const long long hi = __mul64hi(a, b);
  out = lo;
  return hi != (lo >> 63);
}
// train-core lib.rs:1732-1757 for den > 0 (half away from zero); false on overflow.
__device__ __forceinline__ bool round_div(long long num, long long den, long long& out) {
  const long long half = den / 2;
  if (num >= 0) {
    if (num > LLONG_MAX - half) return false;
    out = (num + half) / den;
  } else {
    if (num == LLONG_MIN) return false;
    const long long m = -num;
    if (m > LLONG_MAX - half) return false;
    out = -((m + half) / den);
  }
  return true;
}

// round_div by one divisor over many numerators, with the divisor's
// constants computed once.  Three quotient paths, all exact:
//  - u < 2^32 and den < 2^32: Granlund and Montgomery's division by an
//    invariant integer ("Division by Invariant Integers using Multiplication",
//    PLDI 1994, figure 4.1): with l = ceil(log2 den) and
//    m = floor(2^32 (2^l - den) / den) + 1 (< 2^32), t = hi32(m u) and
//    floor(u / den) = (t + ((u - t) >> min(l, 1))) >> max(l - 1, 0);
//  - u < 2^52 and den < 2^52: the double product u * (1 / den), within one of
//    the quotient (u is exact as a double and the correctly rounded 1 / den
//    is within a relative 2^-53), then one exact integer step (r = u - q den,
//    then q - 1 for r < 0 or q + 1 for r >= den);
//  - otherwise 64-bit integer division.
// Same results as round_div.
struct RoundDiv {
  long long den, half;
  double rd;
  uint32_t m32;  // the 32-bit path's multiplier and shifts (den < 2^32)
  int sh1, sh2;
  bool d32;
};
__device__ __forceinline__ RoundDiv round_div_by(long long den) {
  RoundDiv d;
  d.den = den;
  d.half = den / 2;
  d.rd = 1.0 / (double)den;
  d.d32 = den <= 0xFFFFFFFFll;
  d.m32 = 0;
  d.sh1 = d.sh2 = 0;
  if (d.d32) {
    const unsigned long long ud = (unsigned long long)den;
    const int l = ud <= 1 ? 0 : 64 - __clzll((long long)(ud - 1));  // ceil(log2 den), 0..32
    d.m32 = (uint32_t)((((1ull << l) - ud) << 32) / ud + 1);        // (2^l - den) < den <= 2^32
    d.sh1 = l < 1 ? l : 1;
    d.sh2 = l > 1 ? l - 1 : 0;
  }
  return d;
}
// floor(u / den) for den < 2^32 (the first path of udiv).
__device__ __forceinline__ uint32_t div32(uint32_t u, const RoundDiv& d) {
  const uint32_t t = __umulhi(d.m32, u);
  return (t + ((u - t) >> d.sh1)) >> d.sh2;
}
__device__ __forceinline__ long long udiv(unsigned long long u, const RoundDiv& d) {
  if (d.d32 && (u >> 32) == 0) return (long long)div32((uint32_t)u, d);
  if (u < (1ull << 52) && d.den < (1ll << 52)) {
    long long q = (long long)((double)u * d.rd);
    const long long r = (long long)u - q * d.den;
    if (r < 0)
      --q;
    else if (r >= d.den)
      ++q;
    return q;
  }
  return (long long)(u / (unsigned long long)d.den);
}
__device__ __forceinline__ bool round_div(long long num, const RoundDiv& d, long long& out) {
  // one quotient for either sign: rounding half away from zero is the
  // magnitude's rounding with the sign put back
  if (num == LLONG_MIN) return false;
  const long long m = num < 0 ? -num : num;
  if (m > LLONG_MAX - d.half) return false;
  const long long q = udiv((unsigned long long)(m + d.half), d);
  out = num < 0 ? -q : q;
  return true;
}

// The apply's divider over an array (nsrl_selftest_round_div).
__global__ void round_div_selftest_kernel(const long long* num, long long n, long long den, long long* out,
                                          unsigned char* ok) {
  const RoundDiv d = round_div_by(den);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long q = 0;
    ok[i] = round_div(num[i], d, q) ? 1 : 0;
    out[i] = q;
  }
}

__device__ __forceinline__ unsigned long long mag(long long v) {
  return v == LLONG_MIN ? (unsigned long long)LLONG_MAX + 1ull : (unsigned long long)(v < 0 ? -v : v);
}

// vec[0] = max |x| over the exchange vector, vec[1] = this rank rejected (zeroed before).
__global__ void bound_kernel(const long long* __restrict__ x, long long n, const nsrl_device_status* st,
                             unsigned long long* vec) {
  unsigned long long m = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    m = max(m, mag(x[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m) atomicMax(&vec[0], m);
  if (blockIdx.x == 0 && threadIdx.x == 0) vec[1] = st->flags != 0 ? 1ull : 0ull;
}

// ceil(log2(n)) for n >= 1 (lib.rs:13591-13605).
__device__ __forceinline__ int batch_shift(unsigned long long n) {
  int s = 0;
  unsigned long long c = 1;
  while (c < n) {
    c <<= 1;
    ++s;
  }
  return s;
}

// The decision and, for "apply", the shift table.  merged: the sum came from
// merge_kernel (whose overflow flag then rejects).
__global__ void decide_kernel(const unsigned long long* vec_red, int nranks, const unsigned long long* batch_stats,
                              ShiftCfg c, int merged, const int* merge_overflow, int* decision, int* shifts,
                              nsrl_device_status* st) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (vec_red[1] != 0 || (merged && *merge_overflow)) {
    *decision = DEC_REJECT;
    nsrl_flag(st, NSRL_FLAG_BATCH_REJECTED);
    return;
  }
  if (!merged && vec_red[0] > (unsigned long long)(LLONG_MAX / nranks)) {
    *decision = DEC_MERGE;
    return;
  }
  const unsigned long long accepted = batch_stats[0];
  if (accepted == 0) {
    *decision = DEC_INVALID;
    nsrl_flag(st, NSRL_FLAG_INVALID_CONFIG);
    return;
  }
  // mini_transformer_batch_component_shift_config (lib.rs:13607-13650)
  const int b = batch_shift(accepted);
  const int base[6] = {c.output - b, c.embedding - b, c.mlp - b, c.attention - b, c.attention_q - b,
                       c.attention_qk - b};
  for (int i = 0; i < 6; ++i)
    if (base[i] < 0) {
      *decision = DEC_INVALID;
      nsrl_flag(st, NSRL_FLAG_INVALID_CONFIG);
      return;
    }
  shifts[0] = base[0];
  // embeddings: + MINI_TRANSFORMER_STACKED_EMBEDDING_LEARNING_RATE_EXTRA_SHIFT (0) when stacked (lib.rs:6372-6380)
  shifts[1] = base[1] > 62 ? 62 : base[1];
  for (int l = 0; l < c.layers; ++l) {
    // mini_transformer_stacked_layer_runtime_config (lib.rs:15454-15495): +2 when
    // stacked, +14 more below the top layer, each capped at MAX_RIGHT_SHIFT 62
    for (int j = 0; j < 4; ++j) {
      int v = base[2 + j];
      if (c.layers > 1) {
        v = min(v + 2, 62);
        if (l + 1 < c.layers) v = min(v + 14, 62);
      }
      shifts[2 + 4 * l + j] = v;
    }
  }
  *decision = DEC_APPLY;
}

// Ordered merge of the ranks' vectors (lib.rs:7443-7471): the arena part with
// checked i64 adds in rank order, counts and stats with plain adds.
__global__ void merge_kernel(const long long* __restrict__ parts, int nranks, long long n_arena, long long n_ext,
                             long long* __restrict__ out, int* overflow) {
  bool ovf = false;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n_ext;
       i += (long long)gridDim.x * blockDim.x) {
    long long s = parts[i];
    for (int r = 1; r < nranks; ++r) {
      const long long v = parts[(long long)r * n_ext + i];
      if (i < n_arena) {
        ovf |= add_ovf(s, v, s);
      } else {
        s = (long long)((unsigned long long)s + (unsigned long long)v);
      }
    }
    out[i] = s;
  }
  if (ovf) atomicOr(overflow, 1);
}

__global__ void merge_flag_kernel(int* overflow, nsrl_device_status* st) {
  if (*overflow) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
  *overflow = 0;
}

struct AdamRule {
  int lr, step_shift, b1, b2;
  unsigned long long eps;
};

__device__ __forceinline__ bool rhu128_i64(__int128 v, int s, long long& out) {
  if (s) v += (__int128)1 << (s - 1);
  v >>= s;
  if (v < (__int128)LLONG_MIN || v > (__int128)LLONG_MAX) return false;
  out = (long long)v;
  return true;
}

// integer_adam_delta (nsrl-train-core/src/lib.rs:602-661) with its i128
// intermediates as __int128; false on a rejection.
__device__ __forceinline__ bool adam_delta(long long g, const AdamRule& c, long long& m1, unsigned long long& m2,
                                           long long& res, long long& delta, bool& sat) {
  const long long lim = 2147483647ll;
  const long long bg = g < -lim ? -lim : (g > lim ? lim : g);
  sat = bg != g;
  if (!rhu128_i64((__int128)m1 * (((__int128)1 << c.b1) - 1) + bg, c.b1, m1)) return false;
  __int128 n2 = (__int128)m2 * (((__int128)1 << c.b2) - 1) + (__int128)bg * bg;
  if (c.b2) n2 += (__int128)1 << (c.b2 - 1);
  n2 >>= c.b2;
  if (n2 < 0 || n2 > (__int128)0xFFFFFFFFFFFFFFFFull) return false;
  m2 = (unsigned long long)n2;
  const unsigned long long var = m2 + c.eps;
  if (var < m2) return false;
  const long long inv = rsqrt_q30(var);
  long long n15;
  if (!rhu128_i64((__int128)m1 * inv, 15, n15)) return false;
  n15 = n15 < -32767 ? -32767 : (n15 > 32767 ? 32767 : n15);
  long long num;
  if (mul_ovf(n15, (long long)c.lr, num) || add_ovf(num, res, num)) return false;
  const int eff = 15 + c.step_shift;
  const long long scaled = rhu64(num, (uint32_t)eff);
  const __int128 r = (__int128)num - ((__int128)scaled << eff);
  if (r < (__int128)LLONG_MIN || r > (__int128)LLONG_MAX) return false;
  res = (long long)r;
  delta = -scaled;
  return true;
}

// Constants of the SGD rules for one segment: the divider, the learning
// rate, the shift and the uniform conditions of the 32-bit fast path (a
// 32-bit divisor and a shift in [0, 30]; bias = 2^(shift-1), or 0).
struct SgdRule {
  RoundDiv den;
  int lr, shift, sh;
  long long bias;
  uint32_t half32;
  bool fast;
};
__device__ __forceinline__ SgdRule sgd_rule(const RoundDiv& den, int lr, int shift) {
  SgdRule c;
  c.den = den;
  c.lr = lr;
  c.shift = shift;
  c.fast = den.d32 && shift >= 0 && shift <= 30;
  c.sh = shift & 31;
  c.bias = c.sh ? (1ll << (c.sh - 1)) : 0;
  c.half32 = (uint32_t)den.half;
  return c;
}

// What sgd_element asks its caller to store, and whether the reference's
// checked arithmetic failed.
enum : int { SGD_RES = 1, SGD_W = 2, SGD_BAD = 4 };

// One element of apply_linear_weight_gradient_i64_to_i8 (train-core
// lib.rs:386-465) with the residual carried (i8), or of
// apply_embedding_accumulators_i64_to_i16 (nsrl-train/src/lib.rs:14457-14510):
// the new residual and weight and which of them to store.
__device__ __forceinline__ int sgd_element(bool i8, long long raw, long long r0, int prev, const SgdRule& c,
                                           long long& res_out, int& w_out, unsigned& sat, unsigned& zero,
                                           unsigned long long& l1) {
  // the i8 rule skips a zero gradient, the embedding rule only with a zero residual
  if (raw == 0 && (i8 || r0 == 0)) return 0;
  const long long lo = i8 ? -128 : -32768, hi = i8 ? 127 : 32767;
  if (c.fast && (unsigned long long)(raw + (1ll << 30)) < (1ull << 31) &&
      (unsigned long long)(r0 + (1ll << 31)) < (1ull << 32)) {
    // |raw| <= 2^30 and r0 an i32: |avg| <= 2^30, |product| < 2^62, so no
    // step can overflow, the rounding shift needs no saturation and the new
    // residual (|.| <= 2^(shift-1)) is exact in 32 bits
    const int rr = (int)raw;
    const uint32_t m = rr < 0 ? 0u - (uint32_t)rr : (uint32_t)rr;
    const int q = (int)div32(m + c.half32, c.den);
    const long long product = (long long)(rr < 0 ? -q : q) * c.lr + r0;
    const long long scaled = (product + c.bias) >> c.sh;
    const int next_res = (int)((uint32_t)product - ((uint32_t)scaled << c.sh));
    zero += scaled == 0;
    const long long un = (long long)prev - scaled;
    const int cl = (int)(un < lo ? lo : (un > hi ? hi : un));
    const bool clipped = (long long)cl != un;
    sat += clipped;
    res_out = (i8 && clipped) ? 0 : (long long)next_res;  // the i8 rule drops a saturated weight's residual
    l1 += (unsigned long long)abs(cl - prev);
    w_out = cl;
    return SGD_RES | SGD_W;
  }
  long long avg, product;
  if (!round_div(raw, c.den, avg)) return SGD_BAD;
  if (avg == (long long)(int)avg) {
    product = (long long)(int)avg * (long long)c.lr;  // |.| < 2^62: no overflow
  } else if (mul_ovf(avg, (long long)c.lr, product)) {
    return SGD_BAD;
  }
  if (add_ovf(product, r0, product)) return SGD_BAD;
  const long long scaled = rhu64(product, (uint32_t)c.shift);
  // product - (scaled << shift) is exact: |.| <= 2^(shift-1)
  const long long next_res =
      c.shift ? (long long)((unsigned long long)product - ((unsigned long long)scaled << c.shift)) : 0;
  if (scaled == 0) ++zero;
  int out = 0;
  if (!i8) {  // the embedding rule stores its residual before the weight's check
    res_out = next_res;
    out = SGD_RES;
  }
  long long un;
  if (add_ovf((long long)prev, -scaled, un)) return out | SGD_BAD;
  const int cl = (int)(un < lo ? lo : (un > hi ? hi : un));
  const bool clipped = (long long)cl != un;
  if (clipped) ++sat;
  if (i8) res_out = clipped ? 0 : next_res;
  l1 += (unsigned long long)abs(cl - prev);
  w_out = cl;
  return SGD_RES | SGD_W;
}

// One thread's elements of an SGD tile: entries k * APPLY_THREADS (k <
// APPLY_PER, k * APPLY_THREADS < rem) of the arrays from the given pointers.
// The loads of APPLY_BATCH elements are issued before any of their
// arithmetic, so each thread has that many independent loads in flight, and
// every access is at a constant offset from pointers bumped once per batch.
template <bool I8>
__device__ __forceinline__ void sgd_tile(const long long* __restrict__ psum, long long* __restrict__ pres,
                                         typename std::conditional<I8, int8_t, int16_t>::type* __restrict__ pw,
                                         int rem, const SgdRule& rule, unsigned& sat, unsigned& zero,
                                         unsigned long long& l1, bool& bad) {
#pragma unroll 1
  for (int j0 = 0; j0 < APPLY_PER; j0 += APPLY_BATCH) {
    long long rv[APPLY_BATCH], qv[APPLY_BATCH];
    int pv[APPLY_BATCH];
#pragma unroll
    for (int j = 0; j < APPLY_BATCH; ++j) {
      rv[j] = 0;
      qv[j] = 0;
      pv[j] = 0;
      if (j * APPLY_THREADS < rem) {
        rv[j] = __ldcs(psum + j * APPLY_THREADS);
        qv[j] = pres[j * APPLY_THREADS];
        pv[j] = (int)pw[j * APPLY_THREADS];
      }
    }
#pragma unroll
    for (int j = 0; j < APPLY_BATCH; ++j) {
      if (j * APPLY_THREADS >= rem) continue;
      long long nres;
      int nw;
      const int r = sgd_element(I8, rv[j], qv[j], pv[j], rule, nres, nw, sat, zero, l1);
      bad |= (r & SGD_BAD) != 0;
      if (r & SGD_RES) pres[j * APPLY_THREADS] = nres;
      if (r & SGD_W) pw[j * APPLY_THREADS] = (typename std::conditional<I8, int8_t, int16_t>::type)nw;
    }
    psum += APPLY_BATCH * APPLY_THREADS;
    pres += APPLY_BATCH * APPLY_THREADS;
    pw += APPLY_BATCH * APPLY_THREADS;
    rem -= APPLY_BATCH * APPLY_THREADS;
  }
}

// The SGD rules over arrays, one element per thread (nsrl_selftest_sgd_apply).
__global__ void sgd_apply_selftest_kernel(const long long* __restrict__ raw, long long* __restrict__ res, void* w,
                                          int i8, long long n, long long count, int lr, int shift,
                                          unsigned long long* stats, unsigned char* bad) {
  const SgdRule rule = sgd_rule(round_div_by(count), lr, shift);
  unsigned sat = 0, zero = 0;
  unsigned long long l1 = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int prev = i8 ? (int)static_cast<int8_t*>(w)[i] : (int)static_cast<int16_t*>(w)[i];
    long long nres;
    int nw;
    const int r = sgd_element(i8 != 0, raw[i], res[i], prev, rule, nres, nw, sat, zero, l1);
    if (r & SGD_BAD) *bad = 1;
    if (r & SGD_RES) res[i] = nres;
    if (r & SGD_W) {
      if (i8)
        static_cast<int8_t*>(w)[i] = (int8_t)nw;
      else
        static_cast<int16_t*>(w)[i] = (int16_t)nw;
    }
  }
  if (sat) atomicAdd(&stats[0], (unsigned long long)sat);
  if (zero) atomicAdd(&stats[1], (unsigned long long)zero);
  if (l1) atomicAdd(&stats[2], l1);
}

// One launch applies every parameter: each block takes apply tiles, finds the
// tile's segment and runs that segment's rule on up to APPLY_TILE elements.
__global__ void __launch_bounds__(APPLY_THREADS, 3)
    apply_kernel(const ApplyTable* __restrict__ tab, const long long* __restrict__ sum,
                 const unsigned long long* __restrict__ counts, const int* decision, const int* shifts, int lr,
                 AdamRule ac, long long* __restrict__ res, long long* __restrict__ m1,
                 unsigned long long* __restrict__ m2, long long* __restrict__ ares, unsigned long long* adam_step,
                 unsigned long long* stats, nsrl_device_status* st) {
  if (*decision != DEC_APPLY) return;
  if (adam_step && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(adam_step, 1ull);  // once per batch
  // The segment table, each segment's divider constants and shift are set
  // up once per block in shared memory, so a tile's set-up reads no global
  // memory and the block streams its tiles back to back.
  __shared__ ApplySeg s_seg[MAX_SEGS];
  __shared__ RoundDiv s_div[MAX_SEGS];
  __shared__ int s_shift[MAX_SEGS];
  __shared__ unsigned char s_state[MAX_SEGS];  // 0 apply, 1 nothing accumulated, 2 count out of range
  const int nseg = tab->nseg, ntiles = tab->ntiles;
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) {
    const ApplySeg g = tab->seg[i];
    s_seg[i] = g;
    const unsigned long long count = counts[g.count_idx];
    s_state[i] = count == 0 ? 1 : (count > (unsigned long long)LLONG_MAX ? 2 : 0);
    s_div[i] = round_div_by(s_state[i] ? 1 : (long long)count);
    s_shift[i] = g.shift_class >= 0 ? shifts[g.shift_class] : 0;
  }
  __syncthreads();
  unsigned sat = 0, zero = 0;  // per thread at most 16 per tile it takes
  unsigned long long l1 = 0;
  bool bad = false;
  for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
    int si = 0, hi = nseg - 1;  // last segment with tile0 <= t
    while (si < hi) {
      const int mid = (si + hi + 1) >> 1;
      if (s_seg[mid].tile0 <= t)
        si = mid;
      else
        hi = mid - 1;
    }
    const ApplySeg& sg = s_seg[si];
    if (s_state[si] == 1) continue;  // nothing accumulated: weights and state untouched
    if (s_state[si] == 2) {
      bad = true;
      continue;
    }
    const RoundDiv den = s_div[si];
    const long long e0 = (long long)(t - sg.tile0) * APPLY_TILE;
    const long long e1 = min(sg.len, e0 + APPLY_TILE);
    const int shift = s_shift[si];
    if (sg.kind == SEG_SGD_I8 || sg.kind == SEG_SGD_EMB_I16) {
      const SgdRule rule = sgd_rule(den, lr, shift);
      const long long first = e0 + threadIdx.x;  // this thread's elements: first + k * APPLY_THREADS
      const int rem = (int)(e1 - first);          // <= APPLY_TILE
      if (sg.kind == SEG_SGD_I8)
        sgd_tile<true>(sum + sg.off + first, res + sg.off + first, static_cast<int8_t*>(sg.w) + first, rem, rule,
                       sat, zero, l1, bad);
      else
        sgd_tile<false>(sum + sg.off + first, res + sg.off + first, static_cast<int16_t*>(sg.w) + first, rem, rule,
                        sat, zero, l1, bad);
    } else {
      for (long long e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
        const long long a = sg.off + e;
        const long long raw = sum[a];
        // apply_integer_adam_accumulators_i64_to_i8 / _i16 (train-core lib.rs:469-593)
        const long long k = sg.state_off + e;
        long long g, f = m1[k], r = ares[k], delta;
        unsigned long long s2 = m2[k];
        bool gs;
        if (!round_div(raw, den, g) || !adam_delta(g, ac, f, s2, r, delta, gs)) {
          bad = true;
          continue;
        }
        sat += gs;
        zero += delta == 0;
        const bool i8 = sg.kind == SEG_ADAM_I8;
        const long long prev =
            i8 ? (long long)static_cast<int8_t*>(sg.w)[e] : (long long)static_cast<int16_t*>(sg.w)[e];
        long long un;
        if (add_ovf(prev, delta, un)) {
          bad = true;
          continue;
        }
        const long long lo = i8 ? -128 : -32768, hi = i8 ? 127 : 32767;
        const long long cl = un < lo ? lo : (un > hi ? hi : un);
        if (cl != un) {
          ++sat;
          r = 0;
        }
        l1 += (unsigned long long)(cl > prev ? cl - prev : prev - cl);
        if (i8) static_cast<int8_t*>(sg.w)[e] = (int8_t)cl;
        else static_cast<int16_t*>(sg.w)[e] = (int16_t)cl;
        m1[k] = f;
        m2[k] = s2;
        ares[k] = r;
      }
    }
  }
  if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sat += __shfl_xor_sync(0xffffffffu, sat, o);
    zero += __shfl_xor_sync(0xffffffffu, zero, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if ((threadIdx.x & 31) == 0) {
    if (sat) atomicAdd(&stats[0], (unsigned long long)sat);
    if (zero) atomicAdd(&stats[1], (unsigned long long)zero);
    if (l1) atomicAdd(&stats[2], l1);
  }
}

// ------------------------------------------------------------ layout -------
size_t up256(size_t b) { return (b + 255) & ~size_t(255); }

// Small device block: vec[2], vec_red[2], stats3[3], decision, merge overflow, shifts.
constexpr size_t SMALL_BYTES = 1024;

struct DpLayout {
  size_t n_arena, nc, n_ext;  // arena, counts, exchange vector (arena | counts | 4 stats)
  size_t ext, sum, gather, small, table, wws;  // byte offsets in the workspace
  size_t wws_bytes, bytes;
};

DpLayout dp_layout(const nsrl_train_model* m, size_t windows, int nranks) {
  DpLayout o{};
  o.n_arena = nsrl_train_arena_len(m);
  o.nc = 2 + 9 * m->layers;
  o.n_ext = o.n_arena + o.nc + 4;
  size_t off = 0;
  o.ext = off;
  off += up256(o.n_ext * 8);
  o.sum = off;
  if (nranks > 1) off += up256(o.n_ext * 8);
  o.gather = off;
  if (nranks > 1) off += up256((size_t)nranks * o.n_ext * 8);
  o.small = off;
  off += SMALL_BYTES;
  o.table = off;
  off += up256(sizeof(ApplyTable));
  o.wws = off;
  o.wws_bytes = nsrl_train_workspace_size(m, windows);
  off += up256(o.wws_bytes);
  o.bytes = off;
  return o;
}

size_t adam_len(const nsrl_train_model* m) {
  const size_t d = m->d_model, F = m->hidden_dim, L = m->layers;
  const bool rms = m->layer[0].attn_gamma != nullptr;
  return 256 * d + (m->positions ? m->seq_len * d : 0) + (rms ? 2 * L * d : 0) + L * (4 * d * d + 3 * F * d) +
         256 * d;
}

// The segment table of one step.  Arena order: head [256][d]; per layer q k
// v o [d][d], up gate [F][d], down [d][F], rms attention [d], rms mlp [d];
// token embeddings [256][d]; positions [S][d].  Counts: head, 9 per layer,
// embeddings.
// Algorithmic bytes of one apply over the table: the i64 gradient sum read
// once, then per kind the residual (SGD) or the three Adam state words read
// and written, and the weight read and written.
double apply_bytes(const ApplyTable& tab) {
  double b = 0;
  for (int i = 0; i < tab.nseg; ++i) {
    const ApplySeg& g = tab.seg[i];
    const int per = g.kind == SEG_SGD_I8 ? 8 + 16 + 2
                    : g.kind == SEG_SGD_EMB_I16 ? 8 + 16 + 4
                    : g.kind == SEG_ADAM_I8 ? 8 + 48 + 2
                                            : 8 + 48 + 4;
    b += (double)per * (double)g.len;
  }
  return b;
}

bool build_table(const nsrl_train_model* m, const nsrl_train_config* cfg, ApplyTable& tab) {
  const size_t d = m->d_model, F = m->hidden_dim, L = m->layers, S = m->seq_len;
  const size_t per_layer = 4 * d * d + 3 * F * d + 2 * d;
  const size_t layer0 = 256 * d, emb = layer0 + L * per_layer, pos = emb + 256 * d;
  const size_t lin_off[7] = {0, d * d, 2 * d * d, 3 * d * d, 4 * d * d, 4 * d * d + F * d, 4 * d * d + 2 * F * d};
  const size_t lin_len[7] = {d * d, d * d, d * d, d * d, F * d, F * d, d * F};
  const size_t ce = 1 + 9 * L;
  const bool rms = m->layer[0].attn_gamma != nullptr;
  tab.nseg = 0;
  auto add = [&](size_t off, size_t len, const void* w, int kind, size_t count_idx, int shift_class,
                 long long state_off) {
    if (tab.nseg >= MAX_SEGS) return false;
    ApplySeg& s = tab.seg[tab.nseg++];
    s.off = (long long)off;
    s.len = (long long)len;
    s.w = const_cast<void*>(w);
    s.kind = kind;
    s.count_idx = (int)count_idx;
    s.shift_class = shift_class;
    s.state_off = state_off;
    return true;
  };
  bool ok = true;
  if (cfg->optimizer == NSRL_OPTIMIZER_SHIFT) {
    // lib.rs:6249-6400: head, then per layer the MLP and q/k/v/o, then embeddings
    ok = ok && add(0, 256 * d, m->head.weights, SEG_SGD_I8, 0, 0, -1);
    for (size_t l = 0; l < L; ++l) {
      const int cls[7] = {4, 5, 3, 3, 2, 2, 2};  // q, k, v, o, up, gate, down
      for (int j = 0; j < 7; ++j)
        ok = ok && add(layer0 + l * per_layer + lin_off[j], lin_len[j], m->layer[l].lin[j].weights, SEG_SGD_I8,
                       1 + 9 * l + j, cls[j] + 4 * (int)l, -1);
    }
    ok = ok && add(emb, 256 * d, m->embeddings, SEG_SGD_EMB_I16, ce, 1, -1);
    if (m->positions) ok = ok && add(pos, S * d, m->positions, SEG_SGD_EMB_I16, ce, 1, -1);
  } else {
    // Adam state ranges (lib.rs:4165-4196): embeddings, positions, attention rms,
    // mlp rms, q, k, v, o, up, gate, down (all layers each), output
    const size_t st_emb = 0, st_pos = st_emb + 256 * d, st_rms_a = st_pos + (m->positions ? S * d : 0);
    const size_t st_rms_m = st_rms_a + (rms ? L * d : 0), st_q = st_rms_m + (rms ? L * d : 0);
    size_t st_lin[7];
    st_lin[0] = st_q;
    for (int j = 1; j < 7; ++j) st_lin[j] = st_lin[j - 1] + L * lin_len[j - 1];
    const size_t st_out = st_lin[6] + L * lin_len[6];
    const int sc = cfg->adam_scope;
    const bool all = sc == NSRL_ADAM_SCOPE_ALL;
    if (all || sc == NSRL_ADAM_SCOPE_OUTPUT || sc == NSRL_ADAM_SCOPE_FINAL_MLP_AND_OUTPUT)
      ok = ok && add(0, 256 * d, m->head.weights, SEG_ADAM_I8, 0, -1, (long long)st_out);
    for (size_t l = 0; l < L; ++l) {
      const size_t base = layer0 + l * per_layer;
      if (all)
        for (int j = 0; j < 4; ++j)
          ok = ok && add(base + lin_off[j], lin_len[j], m->layer[l].lin[j].weights, SEG_ADAM_I8, 1 + 9 * l + j, -1,
                         (long long)(st_lin[j] + l * lin_len[j]));
      const bool last = l + 1 == L;
      if (all || ((sc == NSRL_ADAM_SCOPE_FINAL_MLP || sc == NSRL_ADAM_SCOPE_FINAL_MLP_AND_OUTPUT) && last))
        for (int j = 4; j < 7; ++j)
          ok = ok && add(base + lin_off[j], lin_len[j], m->layer[l].lin[j].weights, SEG_ADAM_I8, 1 + 9 * l + j, -1,
                         (long long)(st_lin[j] + l * lin_len[j]));
      if ((all || sc == NSRL_ADAM_SCOPE_RMS_NORM) && rms) {
        ok = ok && add(base + 4 * d * d + 3 * F * d, d, m->layer[l].attn_gamma, SEG_ADAM_I16, 1 + 9 * l + 7, -1,
                       (long long)(st_rms_a + l * d));
        ok = ok && add(base + 4 * d * d + 3 * F * d + d, d, m->layer[l].mlp_gamma, SEG_ADAM_I16, 1 + 9 * l + 8, -1,
                       (long long)(st_rms_m + l * d));
      }
    }
    if (all) {
      ok = ok && add(emb, 256 * d, m->embeddings, SEG_ADAM_I16, ce, -1, (long long)st_emb);
      if (m->positions) ok = ok && add(pos, S * d, m->positions, SEG_ADAM_I16, ce, -1, (long long)st_pos);
    }
  }
  if (!ok) return false;
  int t = 0;
  for (int i = 0; i < tab.nseg; ++i) {
    tab.seg[i].tile0 = t;
    t += (int)((tab.seg[i].len + APPLY_TILE - 1) / APPLY_TILE);
  }
  tab.ntiles = t;
  return true;
}

nsrl_status fail(const char* what) {
  set_error("invalid shape: %s", what);
  return NSRL_INVALID_SHAPE;
}

bool adam_cfg_ok(const nsrl_integer_adam_config& c) {
  // IntegerAdamConfig::is_valid (train-core lib.rs:299-309)
  return c.learning_rate > 0 && c.beta1_decay_shift > 0 && c.beta2_decay_shift > 0 && c.beta1_decay_shift <= 62 &&
         c.beta2_decay_shift <= 62 && c.step_shift <= 62 - 15 && c.epsilon > 0;
}

}  // namespace
}  // namespace nsrl

using namespace nsrl;

#define DP_TRY(call, what)                               \
  do {                                                   \
    cudaError_t _e = (call);                             \
    if (_e != cudaSuccess) {                             \
      set_error("%s: %s", what, cudaGetErrorString(_e)); \
      return NSRL_CUDA_ERROR;                            \
    }                                                    \
  } while (0)

extern "C" {

nsrl_status nsrl_comm_unique_id(uint8_t id[NSRL_COMM_ID_BYTES]) {
  static_assert(sizeof(ncclUniqueId) == NSRL_COMM_ID_BYTES, "ncclUniqueId is 128 bytes");
  if (!id) return fail("null id");
  NcclApi& api = nccl();
  if (!api.ok) {
    set_error("%s", api.err.c_str());
    return NSRL_COMM_ERROR;
  }
  ncclUniqueId u;
  const ncclResult_t r = api.GetUniqueId(&u);
  if (r != ncclSuccess) {
    set_error("ncclGetUniqueId: %s", api.GetErrorString(r));
    return NSRL_COMM_ERROR;
  }
  memcpy(id, &u, NSRL_COMM_ID_BYTES);
  return NSRL_OK;
}

nsrl_status nsrl_comm_init(nsrl_comm** out, int nranks, int rank, const uint8_t id[NSRL_COMM_ID_BYTES],
                           uint64_t timeout_ms) {
  if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks) return fail("communicator rank / size");
  *out = nullptr;
  NcclApi& api = nccl();
  if (!api.ok) {
    set_error("%s", api.err.c_str());
    return NSRL_COMM_ERROR;
  }
  nsrl_comm* c = new nsrl_comm();
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_ns = (timeout_ms ? timeout_ms : 120000ull) * 1000000ull;
  if (cudaGetDevice(&c->device) != cudaSuccess ||
      cudaEventCreateWithFlags(&c->ev, cudaEventDisableTiming) != cudaSuccess) {
    delete c;
    set_error("communicator: no CUDA device");
    return NSRL_CUDA_ERROR;
  }
  ncclUniqueId u;
  memcpy(&u, id, NSRL_COMM_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // every wait on it is ours, and bounded
  ncclResult_t r = api.CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
  nsrl_status s = NSRL_OK;
  if (r == ncclInProgress || r == ncclSuccess) {
    CommWait w{c, nullptr};
    s = wait_bounded(comm_ops(&w), c->timeout_ns, "communicator init");
  } else {
    set_error("ncclCommInitRankConfig: %s", api.GetErrorString(r));
    s = NSRL_COMM_ERROR;
    if (c->comm) api.CommAbort(c->comm);
    c->dead = true;
  }
  if (s != NSRL_OK) {
    cudaEventDestroy(c->ev);
    delete c;
    return s;
  }
  *out = c;
  return NSRL_OK;
}

nsrl_status nsrl_comm_destroy(nsrl_comm* c) {
  if (!c) return NSRL_OK;
  NcclApi& api = nccl();
  nsrl_status s = NSRL_OK;
  if (!c->dead) {
    const ncclResult_t r = api.CommFinalize(c->comm);
    s = comm_settle(c, r, "communicator finalize");
    if (s == NSRL_OK) api.CommDestroy(c->comm);  // else the wait aborted (and freed) it
  }
  if (c->ev) cudaEventDestroy(c->ev);
  delete c;
  return s;
}

nsrl_status nsrl_comm_abort(nsrl_comm* c) {
  if (!c) return fail("null communicator");
  if (!c->dead) {
    c->dead = true;
    nccl().CommAbort(c->comm);
  }
  return NSRL_OK;
}

int nsrl_comm_nranks(const nsrl_comm* c) { return c ? c->nranks : 0; }
int nsrl_comm_rank(const nsrl_comm* c) { return c ? c->rank : -1; }

nsrl_status nsrl_comm_selftest_wait(int scenario, uint64_t timeout_ms, uint64_t* polls, int* aborted) {
  if (!polls || !aborted || scenario < 0 || scenario > 2) return fail("self-test scenario 0..2");
  struct Fake {
    int scenario;
    uint64_t clock, polls;
    int aborted;
  } f{scenario, 0, 0, 0};
  WaitOps o{};
  o.ctx = &f;
  o.done = [](void* p) -> int {
    Fake* f = static_cast<Fake*>(p);
    ++f->polls;
    return (f->scenario == 0 && f->polls >= 3) ? 1 : 0;
  };
  o.comm_error = [](void* p) -> int {
    Fake* f = static_cast<Fake*>(p);
    return (f->scenario == 2 && f->polls >= 3) ? (int)ncclRemoteError : 0;
  };
  o.abort = [](void* p) { static_cast<Fake*>(p)->aborted = 1; };
  o.now_ns = [](void* p) -> uint64_t { return static_cast<Fake*>(p)->clock; };
  o.pause = [](void* p) { static_cast<Fake*>(p)->clock += 1000000ull; };  // 1 ms per poll
  const nsrl_status s = wait_bounded(o, timeout_ms * 1000000ull, "self-test", polls);
  *aborted = f.aborted;
  return s;
}

nsrl_status nsrl_selftest_round_div(const long long* num, size_t n, long long den, long long* out,
                                    unsigned char* ok, void* stream) {
  if (!num || !out || !ok || den <= 0) {
    set_error("nsrl_selftest_round_div: NULL argument or den <= 0");
    return NSRL_INVALID_SHAPE;
  }
  if (n == 0) return NSRL_OK;
  const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
  round_div_selftest_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(num, (long long)n, den, out, ok);
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return NSRL_OK;
  set_error("round_div selftest: %s", cudaGetErrorString(e));
  return NSRL_CUDA_ERROR;
}

nsrl_status nsrl_selftest_sgd_apply(const long long* sums, long long* residuals, void* weights, int weights_i8,
                                    size_t n, unsigned long long count, int learning_rate, int shift,
                                    unsigned long long* stats, unsigned char* bad, void* stream) {
  if (!sums || !residuals || !weights || !stats || !bad || count == 0 || count > (unsigned long long)LLONG_MAX) {
    set_error("nsrl_selftest_sgd_apply: NULL argument or count outside [1, 2^63)");
    return NSRL_INVALID_SHAPE;
  }
  if (n == 0) return NSRL_OK;
  const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
  sgd_apply_selftest_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
      sums, residuals, weights, weights_i8, (long long)n, (long long)count, learning_rate, shift, stats, bad);
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return NSRL_OK;
  set_error("sgd apply selftest: %s", cudaGetErrorString(e));
  return NSRL_CUDA_ERROR;
}

nsrl_status nsrl_merge_worker_parts_i64(const long long* parts, size_t workers, size_t checked_len, size_t len,
                                        long long* out, nsrl_device_status* status, void* stream) {
  if (!parts || !out || !status || workers == 0 || checked_len > len || workers > (size_t)INT32_MAX)
    return fail("merge: null buffer, zero workers or checked_len > len");
  if (len == 0) return NSRL_OK;
  cudaStream_t s = (cudaStream_t)stream;
  // the overflow word is the status's first reserved slot, cleared here and after
  int* ovf = reinterpret_cast<int*>(&status->reserved[0]);
  DP_TRY(cudaMemsetAsync(ovf, 0, sizeof(int), s), "merge");
  merge_kernel<<<148 * 4, 256, 0, s>>>(parts, (int)workers, (long long)checked_len, (long long)len, out, ovf);
  DP_TRY(cudaGetLastError(), "merge");
  merge_flag_kernel<<<1, 1, 0, s>>>(ovf, status);
  DP_TRY(cudaGetLastError(), "merge");
  return NSRL_OK;
}

size_t nsrl_train_adam_state_len(const nsrl_train_model* m) {
  if (!m || !m->layer || m->layers == 0) return 0;
  return adam_len(m);
}

size_t nsrl_train_dp_workspace_size(const nsrl_train_model* m, size_t windows, int nranks) {
  if (!m || !m->layer || m->layers == 0 || windows == 0 || nranks < 1) return 0;
  if (nsrl_train_workspace_size(m, windows) == 0) return 0;
  return dp_layout(m, windows, nranks).bytes;
}

nsrl_status nsrl_train_dp_step(const nsrl_train_model* m, const uint8_t* contexts, const uint8_t* targets,
                               const int16_t* freq_weights, size_t windows, const nsrl_train_config* cfg,
                               const nsrl_train_state* state, nsrl_comm* comm, nsrl_train_step_stats* out,
                               void* workspace, size_t workspace_bytes, nsrl_device_status* status, void* stream) {
  if (!m || !m->layer || m->layers == 0) return fail("model");
  if (!cfg || !state || !state->residuals || !out || !status || !contexts || !targets || windows == 0)
    return fail("null argument or zero windows");
  if (cfg->learning_rate <= 0) return fail("learning_rate must be positive (InvalidConfig)");
  const uint8_t sh[6] = {cfg->output_learning_rate_shift, cfg->mlp_learning_rate_shift,
                         cfg->embedding_learning_rate_shift, cfg->attention_learning_rate_shift,
                         cfg->attention_q_learning_rate_shift, cfg->attention_qk_learning_rate_shift};
  for (uint8_t v : sh)
    if (v > 62) return fail("learning-rate shifts must be <= 62");
  const bool adam = cfg->optimizer == NSRL_OPTIMIZER_INTEGER_ADAM;
  if (!adam && cfg->optimizer != NSRL_OPTIMIZER_SHIFT) return fail("optimizer");
  if (adam) {
    if (!adam_cfg_ok(cfg->adam)) return fail("integer Adam config (IntegerAdamConfig::is_valid)");
    if (cfg->adam_scope > NSRL_ADAM_SCOPE_FINAL_MLP_AND_OUTPUT) return fail("Adam scope");
    if (!state->adam_first_moments || !state->adam_second_moments || !state->adam_update_residuals ||
        !state->adam_step)
      return fail("integer Adam state");
  }
  const int nranks = comm ? comm->nranks : 1;
  if (comm) {
    if (comm->dead) {
      set_error("the communicator was aborted by an earlier failure; destroy it and make a new one");
      return NSRL_COMM_ERROR;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != comm->device)
      return fail("the communicator's device is not current");
  }
  if (nsrl_train_workspace_size(m, windows) == 0) return NSRL_INVALID_SHAPE;  // its own message
  const DpLayout lay = dp_layout(m, windows, nranks);
  if (!workspace || workspace_bytes < lay.bytes) return fail("workspace too small");
  if ((size_t)(2 + 4 * m->layers) * sizeof(int) + 8 * 8 + 8 > SMALL_BYTES) return fail("too many layers");
  ApplyTable tab;
  if (!build_table(m, cfg, tab)) return fail("too many parameter tensors for one apply launch");
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  long long* ext = reinterpret_cast<long long*>(ws + lay.ext);
  long long* sum = nranks > 1 ? reinterpret_cast<long long*>(ws + lay.sum) : ext;
  long long* gather = reinterpret_cast<long long*>(ws + lay.gather);
  unsigned long long* small = reinterpret_cast<unsigned long long*>(ws + lay.small);
  unsigned long long* vec = small;                             // [0..1]
  unsigned long long* vec_red = nranks > 1 ? small + 2 : vec;  // [2..3]
  unsigned long long* stats3 = small + 4;                      // [4..6]
  int* decision = reinterpret_cast<int*>(small + 8);
  int* merge_ovf = decision + 1;
  int* shifts = decision + 2;  // 2 + 4 * layers ints
  ApplyTable* dtab = reinterpret_cast<ApplyTable*>(ws + lay.table);
  const size_t n_arena = lay.n_arena, nc = lay.nc, n_ext = lay.n_ext;
  unsigned long long* counts = reinterpret_cast<unsigned long long*>(ext + n_arena);
  unsigned long long* bstats = counts + nc;
  unsigned long long* sum_counts = reinterpret_cast<unsigned long long*>(sum + n_arena);
  unsigned long long* sum_bstats = sum_counts + nc;

  DP_TRY(cudaMemsetAsync(status, 0, sizeof(nsrl_device_status), s), "status");
  DP_TRY(cudaMemsetAsync(ext, 0, n_ext * 8, s), "arena");
  DP_TRY(cudaMemsetAsync(small, 0, SMALL_BYTES, s), "step scratch");
  // from pageable memory: staged before the call returns, so `tab` may go
  DP_TRY(cudaMemcpyAsync(dtab, &tab, sizeof(ApplyTable), cudaMemcpyHostToDevice, s), "apply table");
  nsrl_status r = nsrl_train_windows(m, contexts, targets, freq_weights, windows, ext, counts, bstats, ws + lay.wws,
                                     lay.wws_bytes, status, stream);
  if (r != NSRL_OK) return r;
  {
    ProfScope prof("dp_bound", s, 0.0, 8.0 * (double)n_ext);
    bound_kernel<<<148 * 2, 256, 0, s>>>(ext, (long long)n_ext, status, vec);
  }
  DP_TRY(cudaGetLastError(), "bound");
  NcclApi& api = nccl();
  if (nranks > 1) {
    ProfScope prof("dp_allreduce", s, 0.0, 8.0 * (double)n_ext);
    api.GroupStart();
    const ncclResult_t e1 = api.AllReduce(vec, vec_red, 2, ncclUint64, ncclMax, comm->comm, s);
    const ncclResult_t e2 = api.AllReduce(ext, sum, n_ext, ncclInt64, ncclSum, comm->comm, s);
    const ncclResult_t e3 = api.GroupEnd();
    auto bad = [](ncclResult_t e) { return e != ncclSuccess && e != ncclInProgress; };
    const ncclResult_t e = bad(e1) ? e1 : (bad(e2) ? e2 : e3);
    if ((r = comm_settle(comm, e, "exchange all-reduce")) != NSRL_OK) return r;
  }
  const ShiftCfg scfg{cfg->learning_rate,
                      cfg->output_learning_rate_shift,
                      cfg->mlp_learning_rate_shift,
                      cfg->embedding_learning_rate_shift,
                      cfg->attention_learning_rate_shift,
                      cfg->attention_q_learning_rate_shift,
                      cfg->attention_qk_learning_rate_shift,
                      (int)m->layers};
  const AdamRule arule{cfg->adam.learning_rate, cfg->adam.step_shift, cfg->adam.beta1_decay_shift,
                       cfg->adam.beta2_decay_shift, cfg->adam.epsilon};
  const unsigned apply_blocks = (unsigned)std::max(1, std::min(tab.ntiles, 148 * 3));  // 3 resident per SM
  auto launch_apply = [&]() -> nsrl_status {
    ProfScope prof("dp_apply", s, 0.0, apply_bytes(tab));
    apply_kernel<<<apply_blocks, APPLY_THREADS, 0, s>>>(dtab, sum, sum_counts, decision, shifts, cfg->learning_rate, arule,
                                              state->residuals, state->adam_first_moments,
                                              state->adam_second_moments, state->adam_update_residuals,
                                              adam ? state->adam_step : nullptr, stats3, status);
    DP_TRY(cudaGetLastError(), "apply");
    return NSRL_OK;
  };
  auto wait_stream = [&](const char* what) -> nsrl_status {
    if (nranks > 1) {
      DP_TRY(cudaEventRecord(comm->ev, s), "event");
      CommWait w{comm, comm->ev};
      return wait_bounded(comm_ops(&w), comm->timeout_ns, what);
    }
    DP_TRY(cudaStreamSynchronize(s), what);
    return NSRL_OK;
  };
  decide_kernel<<<1, 32, 0, s>>>(vec_red, nranks, sum_bstats, scfg, 0, merge_ovf, decision, shifts, status);
  DP_TRY(cudaGetLastError(), "decide");
  if ((r = launch_apply()) != NSRL_OK) return r;
  if ((r = wait_stream("training step")) != NSRL_OK) return r;
  int dec = 0;
  DP_TRY(cudaMemcpy(&dec, decision, sizeof(int), cudaMemcpyDeviceToHost), "decision");
  if (dec == DEC_MERGE) {
    // the bound could not rule out an overflow: the reference's ordered, checked merge
    const long long* parts = ext;
    if (nranks > 1) {
      const ncclResult_t e = api.AllGather(ext, gather, n_ext, ncclInt64, comm->comm, s);
      if ((r = comm_settle(comm, e, "exchange all-gather")) != NSRL_OK) return r;
      parts = gather;
    }
    merge_kernel<<<148 * 4, 256, 0, s>>>(parts, nranks, (long long)n_arena, (long long)n_ext, sum, merge_ovf);
    DP_TRY(cudaGetLastError(), "merge");
    decide_kernel<<<1, 32, 0, s>>>(vec_red, nranks, sum_bstats, scfg, 1, merge_ovf, decision, shifts, status);
    DP_TRY(cudaGetLastError(), "decide");
    if ((r = launch_apply()) != NSRL_OK) return r;
    if ((r = wait_stream("training step (ordered merge)")) != NSRL_OK) return r;
  }
  unsigned long long b4[4], a3[3];
  nsrl_device_status h;
  DP_TRY(cudaMemcpy(b4, sum_bstats, sizeof(b4), cudaMemcpyDeviceToHost), "stats");
  DP_TRY(cudaMemcpy(a3, stats3, sizeof(a3), cudaMemcpyDeviceToHost), "stats");
  DP_TRY(cudaMemcpy(&h, status, sizeof(h), cudaMemcpyDeviceToHost), "status");
  out->accepted_windows = b4[0];
  out->mlp_saturations = b4[1];
  out->attention_saturations = b4[2];
  out->residual_saturations = b4[3];
  out->gradient_saturations = a3[0];
  out->zero_deltas = a3[1];
  out->weight_delta_l1 = a3[2];
  if (h.flags & NSRL_FLAG_INVALID_CONFIG) {
    set_error("invalid config: a learning-rate shift is below the batch shift ceil(log2(accepted windows))");
    return NSRL_INVALID_SHAPE;
  }
  return h.flags ? NSRL_CORE_REJECTED : NSRL_OK;
}

}  // extern "C"
