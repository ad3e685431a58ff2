// Integer linear (recurrent) attention on the GPU: the full causal or
// non-causal forward over a sequence, and the streaming step (plain or
// test-time-training) of independent streams with a carried state.
//
// Reference: crates/nsrl-core/src/attention.rs:879-1041 (forward), :1045-1158
// (step), :1160-1344 (TTT step and delta), :1391-1477 (phi, state update,
// projection, round_div).
//
// phi(x) = x + 32769 in [1, 65536].  Per head the state is S[i][j] =
// sum_t phi(k_t[i]) v_t[j] and key_sums[i] = sum_t phi(k_t[i]) (checked i64);
// a query projects to round_div(sum_i phi(q[i]) S[i][j], sum_i phi(q[i])
// key_sums[i]).  One CTA per (sequence, head); thread j owns value column j
// of S, so every sum runs in the reference's order (tokens, then key index)
// and an i64 overflow rejects exactly where the reference's checked
// arithmetic does.  q, k, v come as the byte planes of the q|k|v projection
// ([rows][3d], q at column 0, k at d, v at 2d); the context leaves as byte
// planes (+ row L1) for the output projection.
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

__device__ __forceinline__ long long phi(int v) { return (long long)v + 32769; }

__device__ __forceinline__ bool add_ovf(long long a, long long b, long long& out) {
  const long long s = (long long)((unsigned long long)a + (unsigned long long)b);
  out = s;
  return ((a ^ s) & (b ^ s)) < 0;
}
__device__ __forceinline__ bool mul_ovf(long long a, long long b, long long& out) {
  const long long lo = (long long)((unsigned long long)a * (unsigned long long)b);
  out = lo;
  return __mul64hi(a, b) != (lo >> 63);
}

// attention.rs:1468-1477: saturating +- den/2, truncating division (den > 0).
__device__ __forceinline__ long long la_round_div(long long num, long long den) {
  const long long half = den >> 1;
  long long t;
  if (num >= 0) {
    t = num > LLONG_MAX - half ? LLONG_MAX : num + half;
  } else {
    t = num < LLONG_MIN + half ? LLONG_MIN : num - half;
  }
  return t / den;
}

__device__ __forceinline__ int plane_val(const int8_t* hi, const uint8_t* lo, long long idx) {
  return (int)hi[idx] * 256 + (int)lo[idx];
}

// Projection of thread j's column: returns false on an overflow or a
// non-positive denominator (attention.rs:1432-1466).
__device__ __forceinline__ bool project_col(const int16_t* sq, const long long* S, int hd, int j,
                                            const long long* ks, int& out) {
  long long den = 0;
  for (int i = 0; i < hd; ++i) {
    long long p;
    if (mul_ovf(phi(sq[i]), ks[i], p) || add_ovf(den, p, den)) return false;
  }
  if (den <= 0) return false;
  long long num = 0;
  for (int i = 0; i < hd; ++i) {
    long long p;
    if (mul_ovf(phi(sq[i]), S[(long long)i * hd + j], p) || add_ovf(num, p, num)) return false;
  }
  const long long r = la_round_div(num, den);
  out = (int)(r < -32768 ? -32768 : (r > 32767 ? 32767 : r));
  return true;
}

// Writes thread j's context value as byte planes and adds the head's |ctx|
// to the row L1 (one atomic per warp).
__device__ __forceinline__ void store_ctx(int8_t* ch, uint8_t* cl, unsigned long long* l1, long long idx, long long row,
                                          int val, bool active) {
  if (active) {
    ch[idx] = (int8_t)(val >> 8);
    cl[idx] = (uint8_t)(val & 255);
  }
  unsigned a = active ? (unsigned)abs(val) : 0u;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  if (l1 && (threadIdx.x & 31) == 0 && a) atomicAdd(&l1[row], (unsigned long long)a);
}

struct LaArgs {
  const int8_t* qh;
  const uint8_t* ql;
  long long ld;  // row stride of the q|k|v planes
  int B, S, d, H, hd, causal;
  int8_t* ch;
  uint8_t* cl;
  unsigned long long* cl1;  // may be null
  long long ldc;
  // streaming step: per stream b the state [H][hd][hd] and key sums [H][hd]
  long long* state;
  long long* key_sums;
  int ttt;           // apply the TTT delta (attention.rs:1290-1344) after the update
  int lr_shift;
  unsigned long long* delta_l1;  // [B], added to (TTT)
  nsrl_device_status* st;
};

// Full forward: one CTA per (sequence, head), the state in shared memory.
__global__ void linear_attention_kernel(LaArgs a) {
  extern __shared__ long long smem[];
  const int hd = a.hd, j = threadIdx.x;
  const bool act = j < hd;
  long long* S = smem;            // [hd][hd]
  long long* ks = S + hd * hd;    // [hd]
  int16_t* sk = reinterpret_cast<int16_t*>(ks + hd);
  int16_t* sv = sk + hd;
  int16_t* sq = sv + hd;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  for (int i = j; i < hd * hd; i += blockDim.x) S[i] = 0;
  if (act) ks[j] = 0;
  bool bad = false;
  const long long c0 = (long long)h * hd + j;
  for (int t = 0; t < a.S; ++t) {
    const long long row = (long long)b * a.S + t;
    __syncthreads();  // the previous token's reads of sk / sv / sq are done
    if (act) {
      const long long base = row * a.ld + c0;
      sq[j] = (int16_t)plane_val(a.qh, a.ql, base);
      sk[j] = (int16_t)plane_val(a.qh, a.ql, base + a.d);
      sv[j] = (int16_t)plane_val(a.qh, a.ql, base + 2 * a.d);
    }
    __syncthreads();
    if (act) {
      // attention.rs:1398-1430 (identity decay): key sums, then the state rows in key order
      bad |= add_ovf(ks[j], phi(sk[j]), ks[j]);
      const long long vj = sv[j];
      for (int i = 0; i < hd; ++i) bad |= add_ovf(S[(long long)i * hd + j], phi(sk[i]) * vj, S[(long long)i * hd + j]);
    }
    __syncthreads();  // every key sum of this token is in place
    if (a.causal) {
      int out = 0;
      if (act && !project_col(sq, S, hd, j, ks, out)) bad = true;
      store_ctx(a.ch, a.cl, a.cl1, row * a.ldc + c0, row, out, act);
    }
  }
  if (!a.causal) {
    for (int t = 0; t < a.S; ++t) {
      const long long row = (long long)b * a.S + t;
      __syncthreads();
      if (act) sq[j] = (int16_t)plane_val(a.qh, a.ql, row * a.ld + c0);
      __syncthreads();
      int out = 0;
      if (act && !project_col(sq, S, hd, j, ks, out)) bad = true;
      store_ctx(a.ch, a.cl, a.cl1, row * a.ldc + c0, row, out, act);
    }
  }
  if (bad) nsrl_flag(a.st, NSRL_FLAG_LINEAR_OVERFLOW);
}

// Streaming step of B independent streams (one row each): one CTA per
// (stream, head), thread j updates column j of the carried state in global
// memory (attention.rs:1085-1158), then (TTT) predicts v from the updated
// state, corrects its column by rhu(phi(k[i]) (v[j] - pred[j]), shift)
// (:1290-1344), then projects q.
__global__ void linear_attention_step_kernel(LaArgs a) {
  extern __shared__ long long smem[];
  const int hd = a.hd, j = threadIdx.x;
  const bool act = j < hd;
  long long* ks = smem;  // [hd]: this head's key sums after the update
  int16_t* sk = reinterpret_cast<int16_t*>(ks + hd);
  int16_t* sv = sk + hd;
  int16_t* sq = sv + hd;
  const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
  const long long c0 = (long long)h * hd + j;
  long long* S = a.state + ((long long)b * a.H + h) * hd * hd;
  long long* gks = a.key_sums + ((long long)b * a.H + h) * hd;
  bool bad = false;
  if (act) {
    const long long base = (long long)b * a.ld + c0;
    sq[j] = (int16_t)plane_val(a.qh, a.ql, base);
    sk[j] = (int16_t)plane_val(a.qh, a.ql, base + a.d);
    sv[j] = (int16_t)plane_val(a.qh, a.ql, base + 2 * a.d);
  }
  __syncthreads();
  if (act) {
    long long kj;
    bad |= add_ovf(gks[j], phi(sk[j]), kj);
    gks[j] = kj;
    ks[j] = kj;
    const long long vj = sv[j];
    for (int i = 0; i < hd; ++i) bad |= add_ovf(S[(long long)i * hd + j], phi(sk[i]) * vj, S[(long long)i * hd + j]);
  }
  __syncthreads();
  if (a.ttt && act) {
    long long den = 0;
    bool dbad = false;
    for (int i = 0; i < hd; ++i) {
      long long p;
      dbad |= mul_ovf(phi(sk[i]), ks[i], p) || add_ovf(den, p, den);
    }
    int pred = 0;
    if (den > 0) {
      long long num = 0;
      for (int i = 0; i < hd; ++i) {
        long long p;
        dbad |= mul_ovf(phi(sk[i]), S[(long long)i * hd + j], p) || add_ovf(num, p, num);
      }
      const long long r = la_round_div(num, den);
      pred = (int)(r < -32768 ? -32768 : (r > 32767 ? 32767 : r));
    }
    const long long err = (long long)sv[j] - pred;
    unsigned long long l1 = 0;
    for (int i = 0; i < hd; ++i) {
      const long long upd = rhu64(phi(sk[i]) * err, (uint32_t)a.lr_shift);
      dbad |= add_ovf(S[(long long)i * hd + j], upd, S[(long long)i * hd + j]);
      l1 += upd < 0 ? (unsigned long long)(-(upd + 1)) + 1ull : (unsigned long long)upd;
    }
    bad |= dbad;
    if (l1) atomicAdd(&a.delta_l1[b], l1);
  }
  int out = 0;
  if (act && !project_col(sq, S, hd, j, ks, out)) bad = true;
  store_ctx(a.ch, a.cl, a.cl1, (long long)b * a.ldc + c0, b, out, act);
  if (bad) nsrl_flag(a.st, NSRL_FLAG_LINEAR_OVERFLOW);
}

LaArgs la_args(const Planes& qkv, size_t B, size_t S, size_t d, size_t H, const Planes& ctx,
               nsrl_device_status* st) {
  LaArgs a{};
  a.qh = qkv.hi;
  a.ql = qkv.lo;
  a.ld = (long long)qkv.ld;
  a.B = (int)B;
  a.S = (int)S;
  a.d = (int)d;
  a.H = (int)H;
  a.hd = (int)(d / H);
  a.ch = ctx.hi;
  a.cl = ctx.lo;
  a.cl1 = ctx.l1;
  a.ldc = (long long)ctx.ld;
  a.st = st;
  return a;
}

unsigned la_threads(int hd) { return (unsigned)((hd + 31) / 32 * 32); }

}  // namespace

bool linear_attention_supported(size_t d, size_t H) { return H != 0 && d % H == 0 && d / H <= 64; }

cudaError_t launch_linear_attention(const Planes& qkv, size_t B, size_t S, size_t d, size_t H, bool causal,
                                    Planes ctx, nsrl_device_status* st, cudaStream_t stream) {
  LaArgs a = la_args(qkv, B, S, d, H, ctx, st);
  a.causal = causal ? 1 : 0;
  const size_t hd = d / H;
  const size_t smem = (hd * hd + hd) * sizeof(long long) + 3 * hd * sizeof(int16_t) + 16;
  if (smem > 48 * 1024)
    if (cudaFuncSetAttribute(linear_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return cudaGetLastError();
  ProfScope prof("linear_attention", stream, 4.0 * (double)B * S * d * hd, 6.0 * (double)B * S * d);
  linear_attention_kernel<<<(unsigned)(B * H), la_threads((int)hd), smem, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_linear_attention_step(const Planes& qkv, size_t B, size_t d, size_t H, long long* state,
                                         long long* key_sums, int ttt_shift, unsigned long long* delta_l1,
                                         Planes ctx, nsrl_device_status* st, cudaStream_t stream) {
  LaArgs a = la_args(qkv, B, 1, d, H, ctx, st);
  a.state = state;
  a.key_sums = key_sums;
  a.ttt = ttt_shift >= 0 ? 1 : 0;
  a.lr_shift = ttt_shift >= 0 ? ttt_shift : 0;
  a.delta_l1 = delta_l1;
  const size_t hd = d / H;
  const size_t smem = hd * sizeof(long long) + 3 * hd * sizeof(int16_t) + 16;
  ProfScope prof("linear_attention_step", stream, (a.ttt ? 8.0 : 4.0) * (double)B * d * hd,
                 (a.ttt ? 32.0 : 16.0) * (double)B * d * hd);
  linear_attention_step_kernel<<<(unsigned)(B * H), la_threads((int)hd), smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace nsrl
