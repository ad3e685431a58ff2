// Shared device code for the NSRL integer hot path on B200 (sm_100a):
// the integer numeric rules of the reference's nsrl-core, the device status
// word, and thin inline-PTX wrappers for mbarrier, TMA and tcgen05.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/nsrl_b200.h"
#include "nsrl_luts.h"

// Device copies of the three integer tables (one per translation unit).
static __device__ const int16_t d_rsqrt_lut[128] = {NSRL_RSQRT_LUT_VALUES};
static __device__ const int16_t d_exp2_lut[256] = {NSRL_EXP2_LUT_VALUES};
static __device__ const uint32_t d_recip_lut[128] = {NSRL_RECIP_LUT_VALUES};
#define NSRL_RECIP_LUT_DEV(i) d_recip_lut[(i)]

// ----------------------------------------------------------------------------
// Status word.  Kernels never trap: a condition under which the reference
// returns `None` sets a bit in nsrl_device_status.flags (atomicOr) and the
// host reports NSRL_CORE_REJECTED for the whole call.
// ----------------------------------------------------------------------------
#define NSRL_FLAG_LINEAR_OVERFLOW 0x1ull   // an i32 prefix of a linear dot overflowed
#define NSRL_FLAG_LOGIT_RANGE 0x2ull       // (q.k) >> shift left the i32 range
#define NSRL_FLAG_ALL_MASKED 0x4ull        // a softmax row had no unmasked logit
#define NSRL_FLAG_RMS_ZERO 0x8ull          // mean square + eps == 0 (integer rsqrt of 0)
#define NSRL_FLAG_BAD_LENGTH 0x10ull       // a KV-cache length outside (0, Lmax]
#define NSRL_FLAG_WAIT_TIMEOUT 0x100ull    // a bounded device wait gave up (internal error)

__device__ __forceinline__ void nsrl_flag(nsrl_device_status* st, unsigned long long bits) {
  atomicOr(reinterpret_cast<unsigned long long*>(&st->flags), bits);
}

// ----------------------------------------------------------------------------
// Integer numerics (crates/nsrl-core/src/numeric.rs).
// ----------------------------------------------------------------------------
__device__ __forceinline__ int16_t sat_i16(long long v) {
  return (int16_t)(v < -32768 ? -32768 : (v > 32767 ? 32767 : v));
}
__device__ __forceinline__ int8_t sat_i8(long long v) {
  return (int8_t)(v < -128 ? -128 : (v > 127 ? 127 : v));
}
__device__ __forceinline__ int16_t sat_i16_i32(int v) { return (int16_t)max(-32768, min(32767, v)); }

// numeric.rs:47-57: (v saturating+ 2^(s-1)) >> s, s clamped to 62, s = 0 is identity.
__device__ __forceinline__ long long rhu64(long long v, uint32_t s) {
  if (s == 0) return v;
  s = s > 62 ? 62 : s;
  long long bias = 1ll << (s - 1);
  long long r = (v > LLONG_MAX - bias) ? LLONG_MAX : v + bias;
  return r >> s;
}

// rhu64(v, s) for |v| <= 2^15 in 32-bit arithmetic: for s >= 16 the rounded
// shift of such a v is 0 (v + 2^(s-1) lies in [0, 2^s)).
__device__ __forceinline__ int rhu_i16(int v, int s) {
  if (s == 0) return v;
  if (s >= 16) return 0;
  return (v + (1 << (s - 1))) >> s;
}

// numeric.rs:59-70: identity scale saturates; otherwise i64 multiply, rhu, saturate.
__device__ __forceinline__ int16_t requant_i32(int acc, int mult, uint32_t shift) {
  if (mult == 1 && shift == 0) return sat_i16_i32(acc);
  return sat_i16(rhu64((long long)acc * (long long)mult, shift));
}

// rms_norm.rs:47-66 for value > 0.  The normalised exponent + 7 equals the
// index of the most significant bit, so the shift is always to the right.
__device__ __forceinline__ long long rsqrt_q30(unsigned long long v) {
  const int msb = 63 - __clzll((long long)v);
  const uint32_t mant = msb >= 7 ? (uint32_t)(v >> (msb - 7)) : (uint32_t)(v << (7 - msb));
  long long inv = (long long)d_rsqrt_lut[(mant & 255u) - 128] << 15;
  if (msb & 1) inv = rhu64(inv * 23170ll, 15);
  const int half = msb / 2;
  return half >= 63 ? 0 : (inv >> half);
}

// floor(ss / d) from a double reciprocal, corrected to the exact quotient
// (ss < 2^53, so the double product is within one of it).
__device__ __forceinline__ unsigned long long div_exact(unsigned long long ss, unsigned d, double rd) {
  unsigned long long q = (unsigned long long)((double)ss * rd);
  if (q * d > ss) --q;
  if ((q + 1) * d <= ss) ++q;
  return q;
}

// Exact warp sums through the 32-bit reduction unit: an unsigned partial
// below 2^37 as two 16-bit-split halves, a signed one below 2^52 in magnitude
// as three pieces (each piece sums below 2^27 over 32 lanes).
__device__ __forceinline__ unsigned long long warp_sum_u37(unsigned long long p) {
  const unsigned a = __reduce_add_sync(0xffffffffu, (unsigned)(p >> 16));
  const unsigned b = __reduce_add_sync(0xffffffffu, (unsigned)(p & 0xFFFF));
  return ((unsigned long long)a << 16) + b;
}
__device__ __forceinline__ long long warp_sum_s52(long long q) {
  const int h = __reduce_add_sync(0xffffffffu, (int)(q >> 32));
  const unsigned m = __reduce_add_sync(0xffffffffu, (unsigned)((q >> 16) & 0xFFFF));
  const unsigned l = __reduce_add_sync(0xffffffffu, (unsigned)(q & 0xFFFF));
  return (long long)h * 4294967296ll + (long long)m * 65536ll + (long long)l;
}

// Eight int16 values of a 16-byte load.
__device__ __forceinline__ void unpack8(const uint4& u, int (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = (int)(int16_t)(w[i] & 0xFFFF);
    v[2 * i + 1] = (int)(int16_t)(w[i] >> 16);
  }
}
__device__ __forceinline__ uint4 pack8(const int (&v)[8]) {
  return make_uint4((uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16), (uint32_t)(v[2] & 0xFFFF) | ((uint32_t)v[3] << 16),
                    (uint32_t)(v[4] & 0xFFFF) | ((uint32_t)v[5] << 16), (uint32_t)(v[6] & 0xFFFF) | ((uint32_t)v[7] << 16));
}
// hi bytes (s8) and lo bytes (u8) of eight values, as two 8-byte words.
__device__ __forceinline__ void planes8(const int (&v)[8], uint2& hi, uint2& lo) {
  uint32_t h[2] = {0, 0}, l[2] = {0, 0};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h[i >> 2] |= (uint32_t)((v[i] >> 8) & 255) << (8 * (i & 3));
    l[i >> 2] |= (uint32_t)(v[i] & 255) << (8 * (i & 3));
  }
  hi = make_uint2(h[0], h[1]);
  lo = make_uint2(l[0], l[1]);
}

// 16-byte global -> shared copies that complete asynchronously (cp.async,
// L2 only); a thread sees its own copies after cp_async_wait.
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Saturating i32 -> i16 (one cvt.sat), returned sign-extended.
__device__ __forceinline__ int sat16(int v) {
  short r;
  asm("cvt.sat.s16.s32 %0, %1;" : "=h"(r) : "r"(v));
  return (int)r;
}

// sat_i16(hi) in the upper 16 bits and sat_i16(lo) in the lower, one instruction.
__device__ __forceinline__ uint32_t pack_sat16(int hi, int lo) {
  uint32_t d;
  asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(d) : "r"(hi), "r"(lo));
  return d;
}

// rhu(p * m, 30) = (p * m + 2^29) >> 30 for a result inside i32 (|p * m| <
// 2^61): one widening multiply-add and a funnel shift of its two words.
__device__ __forceinline__ int rhu30_mul(int p, int m) {
  long long t;
  asm("mad.wide.s32 %0, %1, %2, %3;" : "=l"(t) : "r"(p), "r"(m), "l"(1ll << 29));
  uint32_t r;
  asm("shf.r.wrap.b32 %0, %1, %2, 30;" : "=r"(r) : "r"((uint32_t)t), "r"((uint32_t)(t >> 32)));
  return (int)r;
}

// mlp.rs:150-170: hard-SiLU gate and the gated activation.  For an i16 gate
// g, (g >> 2) + 16384 lies in [8192, 24575], so the clamp to [0, 32767] never
// acts; |g * gate| and |up * silu| stay below 32768 * 24575 < 2^30, so
// rhu(v, 15) = (v + 2^14) >> 15 in i32 is exact and both results lie within
// +-24575: neither saturation acts either.
__device__ __forceinline__ int16_t gated_act(int16_t up, int16_t gate) {
  const int gv = ((int)gate >> 2) + 16384;
  const int silu = ((int)gate * gv + 16384) >> 15;
  return (int16_t)(((int)up * silu + 16384) >> 15);
}

// attention.rs:142-158 with the table in shared memory.
__device__ __forceinline__ int exp2_neg_q15(const int16_t* lut, long long delta) {
  if (delta >= 0) return 32767;
  long long mag = -delta;
  long long ish = mag >> 8;
  if (ish >= 15) return 0;
  return (int)lut[mag & 255] >> (int)ish;
}

// lut.rs:16-40 + attention.rs:181-193: Q31 reciprocal of a positive sum.
__device__ __forceinline__ uint32_t recip_sum_q31(unsigned long long sum) {
  int msb = 63 - __clzll((long long)sum);
  unsigned long long base;
  if (msb >= 7) {
    int sh = msb - 7;
    uint32_t mant = (uint32_t)(sum >> sh) & 255u;
    base = NSRL_RECIP_LUT_DEV(mant - 128);
    base = sh >= 63 ? 0ull : (base >> sh);
  } else {
    int sh = 7 - msb;
    uint32_t mant = (uint32_t)(sum << sh) & 255u;
    base = NSRL_RECIP_LUT_DEV(mant - 128);
    base = base << sh;
  }
  return (uint32_t)(base > 0xFFFFFFFFull ? 0xFFFFFFFFull : base);
}

// ----------------------------------------------------------------------------
// Small PTX helpers.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete may
// sleep for up to `hint_ns` nanoseconds instead of returning at once, so a
// waiting warp does not spin through issue slots that others could use.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Every wait is bounded in time: after limit_ns nanoseconds the waiter
// records NSRL_FLAG_WAIT_TIMEOUT and returns false so that the kernel can
// unwind (the host then reports the call as failed).  The kernels use
// NSRL_WAIT_NS; nsrl_selftest_bounded_wait runs the same loop with a short
// limit on a barrier that never completes.
#define NSRL_WAIT_NS 2000000000ull
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, nsrl_device_status* st,
                                              unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;  // the common case reads no timer
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait_hint(bar, parity, 20000u)) return true;
    if ((i & 15u) == 15u && global_ns() - t0 > limit_ns) {
      nsrl_flag(st, NSRL_FLAG_WAIT_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, nsrl_device_status* st) {
  return mbar_wait_for(bar, parity, st, NSRL_WAIT_NS);
}

// True once any bounded wait of the call has timed out (read by one thread,
// broadcast by the caller); later CTAs then skip their work.
__device__ __forceinline__ bool timed_out(const nsrl_device_status* st) {
  return (*reinterpret_cast<const volatile unsigned long long*>(&st->flags) & NSRL_FLAG_WAIT_TIMEOUT) != 0;
}

// 2-D tiled TMA load (no multicast) into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// 3-D tiled TMA load (no multicast); coordinates beyond the tensor read zeros.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// TMA tile store shared -> global (bulk-group completion): the tile is read
// from shared memory in the tensor map's swizzled layout; coordinates outside
// the tensor are not written.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1)
               : "memory");
}
// Orders this thread's completed async-proxy (TMA) global writes before its later generic accesses.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// All but the newest N bulk groups of this thread have finished reading their shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// All bulk groups of this thread have completed (their global writes are done).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Stores 32 bytes (o: 8 words) of this lane's row r at base + r * ld as lane
// pairs: partners 2i and 2i+1 swap halves, so each of the two store
// instructions writes whole 32-byte runs (rows 2i, then rows 2i+1) instead of
// one 16-byte half of 32 rows.  Every lane of the warp calls it (the swap is a
// shuffle); r has the parity of the lane, rows at or past M are not written,
// and base and ld (bytes) are 16-byte multiples.
__device__ __forceinline__ void store32b_pairs(uint8_t* base, long long ld, int r, int M, const uint32_t (&o)[8],
                                               int lane) {
  const bool odd = lane & 1;
  uint32_t x[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) x[k] = __shfl_xor_sync(0xffffffffu, odd ? o[k] : o[4 + k], 1);
  const int re = r & ~1;  // the pair's even row
  uint8_t* d = base + (long long)re * ld + (odd ? 16 : 0);
  if (re < M)
    *reinterpret_cast<uint4*>(d) = odd ? make_uint4(x[0], x[1], x[2], x[3]) : make_uint4(o[0], o[1], o[2], o[3]);
  if (re + 1 < M)
    *reinterpret_cast<uint4*>(d + ld) = odd ? make_uint4(o[4], o[5], o[6], o[7]) : make_uint4(x[0], x[1], x[2], x[3]);
}
// ---- programmatic dependent launch -------------------------------------------
// A kernel started by launch_pdl() may begin while the previous kernel of its
// stream still runs.  griddep_wait() returns once that kernel has completed and
// its writes are visible (at once for a launch without that dependency), so
// such a kernel touches no global memory before it: only shared memory, its
// barriers, TMEM and its tensor maps.  griddep_launch() lets the next such
// kernel start its own prologue on the SMs this grid leaves free; a CTA issues
// it only after its TMEM allocation, so an early CTA of the next kernel never
// holds TMEM that a CTA of this one still waits for.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... P, typename... A>
inline cudaError_t launch_pdl(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              const A&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---- tcgen05 ----------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8, s32 accumulate.
__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when all previously issued tcgen05.mma of this thread complete.
// The same two from a whole warp: every lane runs the issuing loop, so that
// descriptors, TMEM addresses and loop counters are warp-uniform values kept
// in uniform registers (the operands tcgen05.mma reads), and one elected lane
// issues.  The elected lane is the same on every call of a full warp, so the
// commit tracks the MMAs it issued.
__device__ __forceinline__ void umma_i8_warp(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane
// (base lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row atoms of 1024 bytes, tile base
// 1024-byte aligned).  SBO = 1024 B between 8-row groups; LBO is unused for
// swizzled K-major layouts; version field = 1 (sm_100).
__device__ __forceinline__ uint64_t sdesc_k128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// The same layout with the 8-row atoms `sbo` bytes apart (e.g. two planes
// interleaved atom by atom).
__device__ __forceinline__ uint64_t sdesc_k128_sbo(uint32_t saddr, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: kind::i8, D = s32, K-major A and B, shape M x N.
// a_signed / b_signed select s8 (1) or u8 (0) per operand.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t M, uint32_t N, uint32_t a_signed, uint32_t b_signed) {
  return (2u << 4) | (a_signed << 7) | (b_signed << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// Byte offset of element (row r, byte c) in a 128-byte-swizzled tile whose
// base is 1024-byte aligned (the layout TMA writes with SWIZZLE_128B).
__device__ __forceinline__ uint32_t swz128(uint32_t r, uint32_t c) {
  return r * 128u + ((((c >> 4) ^ (r & 7u)) << 4) | (c & 15u));
}
