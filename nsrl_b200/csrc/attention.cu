// Integer causal self-attention core and KV-cache decode attention.
//
// Reference: crates/nsrl-core/src/attention.rs:742-877 (full attention),
// :671-725 (one query row), :261-293 (base-2 softmax), :117-140 (QK dot).
// Per query t and head h: logit_j = i32((sum_d q[t][d] k[j][d]) >> log4(hd))
// (None if outside i32) for j <= t; max over unmasked logits; w_j =
// LUT(logit_j - max) in Q15; sum in u64; inv = Q31 LUT reciprocal of the sum;
// p_j = sat_i16(rhu(w_j * inv, 16)); ctx = sat_i16(rhu(sum_j p_j v[j], 15)).
//
// The probability is rounded to Q15 with the reciprocal of the *complete*
// row sum before the AV product, so an online (rescaling) softmax would
// round differently.  The prefill kernel therefore makes three exact passes
// over the keys of a query tile: row max, row sum, then probabilities and AV.
//
// prefill_attention_kernel: int8 tensor-core MMAs (m16n8k32) on byte planes.
//   q.k = 65536*(qh.kh) + 256*(qh.kl + ql.kh) + ql.kl and p.v likewise, every
//   partial an exact s32; recombined in i64.
// attention_rows_kernel: one CTA per (query row, head), logits in shared
//   memory, 16-byte vector loads; the HBM-bound decode kernel and the
//   fallback for head dims / lengths the prefill kernel does not take.
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

// --------------------------------------------------------------- MMA ------
#define NSRL_MMA_I8(NAME, TA, TB)                                                                            \
  __device__ __forceinline__ void NAME(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {      \
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." TA "." TB                                         \
                 ".s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"                                \
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])                                            \
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));                            \
  }
NSRL_MMA_I8(mma_ss, "s8", "s8")
NSRL_MMA_I8(mma_su, "s8", "u8")
NSRL_MMA_I8(mma_us, "u8", "s8")
NSRL_MMA_I8(mma_uu, "u8", "u8")

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t ldg32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

constexpr int QT = 64;  // queries per CTA (4 warps x 16 rows)
constexpr int KT = 32;  // keys per tile

template <int HD>
struct PrefillSmem {
  static constexpr int KSTR = HD == 16 ? 48 : HD + 16;  // bank-conflict-free B-fragment loads
  static constexpr int VSTR = 48;
  uint8_t k_hi[KT * KSTR];
  uint8_t k_lo[KT * KSTR];
  uint8_t vt_hi[HD * VSTR];
  uint8_t vt_lo[HD * VSTR];
  int16_t lut[256];
};

// Position, inside a 32-key MMA k-block, of key j: the P fragment is built
// straight from the S accumulator layout, so V is stored in that key order.
__device__ __forceinline__ int key_slot(int j) {
  return 16 * (j >> 4) + 4 * ((j & 7) >> 1) + 2 * ((j & 15) >> 3) + (j & 1);
}

struct PrefillArgs {
  const int8_t* qkv_hi;
  const uint8_t* qkv_lo;
  long long ld;  // row stride of the q|k|v planes (3 * d)
  int S, d, H, causal, shift;
  int8_t* ctx_hi;
  uint8_t* ctx_lo;
  unsigned long long* ctx_l1;
  long long ldc;
  nsrl_device_status* st;
};

template <int HD>
__global__ void __launch_bounds__(128) prefill_attention_kernel(const PrefillArgs a) {
  constexpr int KC = HD >= 32 ? HD / 32 : 1;  // 32-wide k chunks of the QK product
  constexpr int NT = HD / 8;                  // 8-wide n tiles of the AV product
  __shared__ __align__(16) PrefillSmem<HD> sm;
  constexpr int KSTR = PrefillSmem<HD>::KSTR, VSTR = PrefillSmem<HD>::VSTR;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = blockIdx.x * QT, h = blockIdx.y, b = blockIdx.z;
  const long long seq_row0 = (long long)b * a.S;
  for (int i = tid; i < 256; i += 128) sm.lut[i] = d_exp2_lut[i];

  // Query rows of this thread: r0 = qw + g and r1 = r0 + 8.
  const int qw = q0 + warp * 16;
  const int r0 = qw + g, r1 = r0 + 8;
  uint32_t qa_hi[KC][4], qa_lo[KC][4];
  {
    const long long col = (long long)h * HD;
#pragma unroll
    for (int c = 0; c < KC; ++c) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = (i & 1) ? r1 : r0;
        const int k = 32 * c + 4 * t + ((i & 2) ? 16 : 0);
        const bool ok = r < a.S && k < HD;
        const long long off = (seq_row0 + r) * a.ld + col + k;
        qa_hi[c][i] = ok ? ldg32(a.qkv_hi + off) : 0u;
        qa_lo[c][i] = ok ? ldg32(a.qkv_lo + off) : 0u;
      }
    }
  }

  const int kend = a.causal ? min(a.S, q0 + QT) : a.S;
  const int ntiles = (kend + KT - 1) / KT;
  const int wlast = min(qw + 15, a.S - 1);  // last live query of this warp

  long long rmax[2] = {0, 0};
  bool rany[2] = {false, false};
  unsigned long long rsum[2] = {0, 0};
  uint32_t rinv[2] = {0, 0};
  int pv_hh[NT][4], pv_mid[NT][4], pv_ll[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) pv_hh[n][i] = pv_mid[n][i] = pv_ll[n][i] = 0;
  bool range_bad = false;

#pragma unroll 1
  for (int pass = 0; pass < 3; ++pass) {
#pragma unroll 1
    for (int kt = 0; kt < ntiles; ++kt) {
      const int kb = kt * KT;
      __syncthreads();
      // ---- stage the K tile (and in the last pass the V tile, transposed) ----
      {
        constexpr int CH = HD / 16 > 0 ? HD / 16 : 1;  // 16-byte chunks per row (HD >= 16)
        for (int i = tid; i < KT * CH; i += 128) {
          const int j = i / CH, c = i % CH;
          const int key = kb + j;
          uint4 vh = make_uint4(0, 0, 0, 0), vl = vh;
          if (key < kend) {
            const long long off = (seq_row0 + key) * a.ld + a.d + (long long)h * HD + 16 * c;
            vh = *reinterpret_cast<const uint4*>(a.qkv_hi + off);
            vl = *reinterpret_cast<const uint4*>(a.qkv_lo + off);
          }
          *reinterpret_cast<uint4*>(&sm.k_hi[j * KSTR + 16 * c]) = vh;
          *reinterpret_cast<uint4*>(&sm.k_lo[j * KSTR + 16 * c]) = vl;
        }
        if (pass == 2) {
          for (int i = tid; i < KT * CH; i += 128) {
            const int j = i / CH, c = i % CH;
            const int key = kb + j;
            uint4 vh = make_uint4(0, 0, 0, 0), vl = vh;
            if (key < kend) {
              const long long off = (seq_row0 + key) * a.ld + 2 * a.d + (long long)h * HD + 16 * c;
              vh = *reinterpret_cast<const uint4*>(a.qkv_hi + off);
              vl = *reinterpret_cast<const uint4*>(a.qkv_lo + off);
            }
            const uint8_t* bh = reinterpret_cast<const uint8_t*>(&vh);
            const uint8_t* bl = reinterpret_cast<const uint8_t*>(&vl);
            const int slot = key_slot(j);
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              sm.vt_hi[(16 * c + e) * VSTR + slot] = bh[e];
              sm.vt_lo[(16 * c + e) * VSTR + slot] = bl[e];
            }
          }
        }
      }
      __syncthreads();
      if ((a.causal && kb > wlast) || qw >= a.S) continue;  // tile fully masked for this warp

      // ---- S = Q K^T for 16 rows x 32 keys ----
      int s_hh[4][4], s_mid[4][4], s_ll[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) s_hh[j][i] = s_mid[j][i] = s_ll[j][i] = 0;
        const uint8_t* kh = &sm.k_hi[(8 * j + g) * KSTR + 4 * t];
        const uint8_t* kl = &sm.k_lo[(8 * j + g) * KSTR + 4 * t];
#pragma unroll
        for (int c = 0; c < KC; ++c) {
          const uint32_t bh0 = lds32(kh + 32 * c), bl0 = lds32(kl + 32 * c);
          const uint32_t bh1 = HD >= 32 ? lds32(kh + 32 * c + 16) : 0u;
          const uint32_t bl1 = HD >= 32 ? lds32(kl + 32 * c + 16) : 0u;
          mma_ss(s_hh[j], qa_hi[c], bh0, bh1);
          mma_su(s_mid[j], qa_hi[c], bl0, bl1);
          mma_us(s_mid[j], qa_lo[c], bh0, bh1);
          mma_uu(s_ll[j], qa_lo[c], bl0, bl1);
        }
      }
      // ---- logits, masks, and the pass-specific row work ----
      int pr[2][8];  // probabilities of rows r0 / r1 at this thread's 8 keys
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = (i & 2) ? 1 : 0;
          const int r = row ? r1 : r0;
          const int key = kb + 8 * j + 2 * t + (i & 1);
          const long long raw =
              (long long)s_hh[j][i] * 65536 + (long long)s_mid[j][i] * 256 + (long long)s_ll[j][i];
          const long long lg = raw >> a.shift;
          const bool live = r < a.S && key < kend && (!a.causal || key <= r);
          bool masked = !live;
          if (live) {
            if (lg < INT_MIN || lg > INT_MAX) range_bad = true;
            if (lg == (long long)INT_MIN) masked = true;  // equals MASKED_LOGIT: excluded like a mask
          }
          int p = 0;
          if (pass == 0) {
            if (!masked) {
              if (!rany[row] || lg > rmax[row]) rmax[row] = lg;
              rany[row] = true;
            }
          } else if (!masked) {
            const int w = exp2_neg_q15(sm.lut, lg - rmax[row]);
            if (pass == 1)
              rsum[row] += (unsigned long long)w;
            else
              p = (int)sat_i16(rhu64((long long)w * (long long)rinv[row], 16));
          }
          pr[row][2 * j + (i & 1)] = p;
        }
      }
      if (pass == 2) {
        // A fragments of P (rows x 32 keys) in the key order of key_slot().
        uint32_t ph[4], pl[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = i & 1;             // a0, a2: row r0; a1, a3: row r1
          const int base = (i & 2) ? 4 : 0;  // a0/a1: n tiles 0,1; a2/a3: n tiles 2,3
          uint32_t hv = 0, lv = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int pv = pr[row][base + e];
            hv |= (uint32_t)(pv >> 8) << (8 * e);
            lv |= (uint32_t)(pv & 255) << (8 * e);
          }
          ph[i] = hv;
          pl[i] = lv;
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const uint8_t* vh = &sm.vt_hi[(8 * n + g) * VSTR + 4 * t];
          const uint8_t* vl = &sm.vt_lo[(8 * n + g) * VSTR + 4 * t];
          const uint32_t bh0 = lds32(vh), bh1 = lds32(vh + 16), bl0 = lds32(vl), bl1 = lds32(vl + 16);
          mma_us(pv_hh[n], ph, bh0, bh1);
          mma_uu(pv_mid[n], ph, bl0, bl1);
          mma_us(pv_mid[n], pl, bh0, bh1);
          mma_uu(pv_ll[n], pl, bl0, bl1);
        }
      }
    }
    // ---- reduce the row statistics over the 4 threads of each quad ----
    if (pass == 0) {
#pragma unroll
      for (int row = 0; row < 2; ++row) {
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          const long long om = __shfl_xor_sync(0xffffffffu, rmax[row], o);
          const int oa = __shfl_xor_sync(0xffffffffu, (int)rany[row], o);
          if (oa && (!rany[row] || om > rmax[row])) rmax[row] = om;
          rany[row] = rany[row] || oa;
        }
      }
    } else if (pass == 1) {
#pragma unroll
      for (int row = 0; row < 2; ++row) {
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) rsum[row] += __shfl_xor_sync(0xffffffffu, rsum[row], o);
        rinv[row] = rany[row] ? recip_sum_q31(rsum[row]) : 0u;
      }
    }
  }

  if (range_bad) nsrl_flag(a.st, NSRL_FLAG_LOGIT_RANGE);
  if (t == 0) {
    if (r0 < a.S && !rany[0]) nsrl_flag(a.st, NSRL_FLAG_ALL_MASKED);
    if (r1 < a.S && !rany[1]) nsrl_flag(a.st, NSRL_FLAG_ALL_MASKED);
  }
  // ---- context: sat(rhu(sum p.v, 15)) written as byte planes (+ row L1) ----
  unsigned long long l1[2] = {0, 0};
#pragma unroll
  for (int n = 0; n < NT; ++n) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? r1 : r0;
      uint32_t hv = 0, lv = 0;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * half + e;
        const long long tot =
            (long long)pv_hh[n][i] * 65536 + (long long)pv_mid[n][i] * 256 + (long long)pv_ll[n][i];
        const int v = (int)sat_i16(rhu64(tot, 15));
        l1[half] += (unsigned long long)abs(v);
        hv |= (uint32_t)((v >> 8) & 255) << (8 * e);
        lv |= (uint32_t)(v & 255) << (8 * e);
      }
      if (r < a.S) {
        const long long off = (seq_row0 + r) * a.ldc + (long long)h * HD + 8 * n + 2 * t;
        *reinterpret_cast<uint16_t*>(a.ctx_hi + off) = (uint16_t)hv;
        *reinterpret_cast<uint16_t*>(a.ctx_lo + off) = (uint16_t)lv;
      }
    }
  }
  if (a.ctx_l1) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
#pragma unroll
      for (int o = 1; o <= 2; o <<= 1) l1[half] += __shfl_xor_sync(0xffffffffu, l1[half], o);
      const int r = half ? r1 : r0;
      if (t == 0 && r < a.S) atomicAdd(&a.ctx_l1[seq_row0 + r], l1[half]);
    }
  }
}

// ------------------------------------------------------ row attention -----
// One CTA of 256 threads per (query row, head).  LPK lanes cooperate on one
// key / value row with 16-byte loads (8 int16 each); HD = 8 * LPK.  HD < 8
// uses the scalar variant (LPK = 0).
struct RowArgs {
  const int16_t* q;
  long long ldq;
  const int16_t* k;
  const int16_t* v;
  long long ldkv;        // row stride of k and v (elements)
  long long kv_seq;      // stride between sequences of k/v (elements)
  int rows_per_seq;      // query rows per sequence (1 for decode)
  int mode;              // 0: decode (lens), 1: causal prefill, 2: full prefill
  int len_offset;        // decode: keys attended = lens[b] + len_offset
  const int32_t* lens;
  int Lmax;
  int hd, shift;
  int16_t* out;
  long long ldo;
  int16_t* probs;  // optional: causal prefill rows of P [B][H][S][S] (zero above the diagonal)
  nsrl_device_status* st;
};

template <int LPK>
__global__ void __launch_bounds__(256) attention_rows_kernel(const RowArgs a) {
  extern __shared__ __align__(16) uint8_t dsm[];
  int32_t* logits = reinterpret_cast<int32_t*>(dsm);
  __shared__ int16_t lut[256];
  __shared__ long long red_ll[8];
  __shared__ unsigned long long red_u[8];
  __shared__ int red_i[8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < 256; i += 256) lut[i] = d_exp2_lut[i];

  const long long row = blockIdx.x;
  const int h = blockIdx.y;
  const long long b = row / a.rows_per_seq;
  const int tq = (int)(row % a.rows_per_seq);
  int L;
  if (a.mode == 0)
    L = a.lens[b] + a.len_offset;
  else if (a.mode == 1)
    L = tq + 1;
  else
    L = a.rows_per_seq;
  if (L <= 0 || L > a.Lmax) {
    if (tid == 0) nsrl_flag(a.st, NSRL_FLAG_BAD_LENGTH);
    return;
  }
  const int16_t* qp = a.q + row * a.ldq + (long long)h * a.hd;
  const int16_t* kp = a.k + b * a.kv_seq + (long long)h * a.hd;
  const int16_t* vp = a.v + b * a.kv_seq + (long long)h * a.hd;
  __syncthreads();

  // ---- phase 1: logits ----
  bool bad = false;
  if (LPK > 0) {
    constexpr int GROUPS = 256 / (LPK > 0 ? LPK : 1);
    const int sub = tid % LPK, grp = tid / LPK;
    int qv[8];
    {
      uint4 u = *reinterpret_cast<const uint4*>(qp + 8 * sub);
      const int16_t* e = reinterpret_cast<const int16_t*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) qv[i] = e[i];
    }
    // The trip count is uniform over the CTA so that every lane of a warp
    // takes part in the shuffles.
    const int rounds = (L + GROUPS - 1) / GROUPS;
#pragma unroll 4
    for (int it = 0; it < rounds; ++it) {
      const int j = grp + it * GROUPS;
      long long s = 0;
      if (j < L) {
        uint4 u = *reinterpret_cast<const uint4*>(kp + (long long)j * a.ldkv + 8 * sub);
        const int16_t* e = reinterpret_cast<const int16_t*>(&u);
#pragma unroll
        for (int i = 0; i < 8; ++i) s += (long long)(qv[i] * (int)e[i]);
      }
#pragma unroll
      for (int o = 1; o < LPK; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (sub == 0 && j < L) {
        const long long lg = s >> a.shift;
        if (lg < INT_MIN || lg > INT_MAX) bad = true;
        logits[j] = (int32_t)lg;
      }
    }
  } else {
    for (int j = tid; j < L; j += 256) {
      long long s = 0;
      for (int i = 0; i < a.hd; ++i) s += (long long)((int)qp[i] * (int)kp[(long long)j * a.ldkv + i]);
      const long long lg = s >> a.shift;
      if (lg < INT_MIN || lg > INT_MAX) bad = true;
      logits[j] = (int32_t)lg;
    }
  }
  if (bad) nsrl_flag(a.st, NSRL_FLAG_LOGIT_RANGE);
  __syncthreads();

  // ---- phase 2: max, weights, sum, probabilities ----
  long long mx = LLONG_MIN;
  int any = 0;
  for (int j = tid; j < L; j += 256) {
    const int32_t lg = logits[j];
    if (lg != INT_MIN) {
      any = 1;
      mx = max(mx, (long long)lg);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    any |= __shfl_xor_sync(0xffffffffu, any, o);
  }
  if (lane == 0) {
    red_ll[warp] = mx;
    red_i[warp] = any;
  }
  __syncthreads();
  mx = LLONG_MIN;
  any = 0;
  for (int w = 0; w < 8; ++w) {
    mx = max(mx, red_ll[w]);
    any |= red_i[w];
  }
  if (!any) {
    if (tid == 0) nsrl_flag(a.st, NSRL_FLAG_ALL_MASKED);
    return;
  }
  unsigned long long sum = 0;
  for (int j = tid; j < L; j += 256) {
    const int32_t lg = logits[j];
    const int w = lg == INT_MIN ? 0 : exp2_neg_q15(lut, (long long)lg - mx);
    logits[j] = w;  // weight replaces the logit in place
    sum += (unsigned long long)w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red_u[warp] = sum;
  __syncthreads();
  sum = 0;
  for (int w = 0; w < 8; ++w) sum += red_u[w];
  const long long inv = (long long)recip_sum_q31(sum);
  for (int j = tid; j < L; j += 256) logits[j] = (int32_t)sat_i16(rhu64((long long)logits[j] * inv, 16));
  __syncthreads();
  if (a.probs) {  // nsrl-train/src/lib.rs:15353-15418: the row of P, zeros past the causal limit
    int16_t* pr = a.probs + ((b * gridDim.y + h) * (long long)a.rows_per_seq + tq) * a.rows_per_seq;
    for (int j = tid; j < a.rows_per_seq; j += 256) pr[j] = j < L ? (int16_t)logits[j] : (int16_t)0;
  }

  // ---- phase 3: context = sat(rhu(sum_j p_j v[j], 15)) ----
  if (LPK > 0) {
    constexpr int GROUPS = 256 / (LPK > 0 ? LPK : 1);
    const int sub = tid % LPK, grp = tid / LPK;
    long long acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0;
#pragma unroll 4
    for (int j = grp; j < L; j += GROUPS) {
      const int p = logits[j];
      uint4 u = *reinterpret_cast<const uint4*>(vp + (long long)j * a.ldkv + 8 * sub);
      const int16_t* e = reinterpret_cast<const int16_t*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += (long long)(p * (int)e[i]);
    }
    // reduce over groups: warp-level first (groups within a warp), then smem
    long long* part = reinterpret_cast<long long*>(dsm + 4 * (size_t)a.Lmax + 16 - ((4 * (size_t)a.Lmax) & 15));
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
    __syncthreads();
    if (lane < LPK)
#pragma unroll
      for (int i = 0; i < 8; ++i) part[warp * (8 * LPK) + 8 * sub + i] = acc[i];
    __syncthreads();
    for (int c = tid; c < 8 * LPK; c += 256) {
      long long s = 0;
      for (int w = 0; w < 8; ++w) s += part[w * (8 * LPK) + c];
      a.out[row * a.ldo + (long long)h * a.hd + c] = sat_i16(rhu64(s, 15));
    }
  } else {
    for (int c = tid; c < a.hd; c += 256) {
      long long s = 0;
      for (int j = 0; j < L; ++j) s += (long long)(logits[j] * (int)vp[(long long)j * a.ldkv + c]);
      a.out[row * a.ldo + (long long)h * a.hd + c] = sat_i16(rhu64(s, 15));
    }
  }
}

size_t rows_smem(int Lmax, int lpk) {
  size_t s = 4 * (size_t)Lmax;
  s = (s + 15) & ~size_t(15);
  return s + 16 + (lpk > 0 ? (size_t)8 * 8 * lpk * 8 : 0);
}

cudaError_t launch_rows(const RowArgs& a, long long rows, int H, cudaStream_t stream) {
  const int lpk = (a.hd >= 8 && a.hd <= 256 && a.hd % 8 == 0) ? a.hd / 8 : 0;
  const size_t smem = rows_smem(a.Lmax, lpk);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  dim3 grid((unsigned)rows, (unsigned)H);
  // Work at the longest key range (decode lengths live on the device).
  const double keys = (double)rows * (double)a.Lmax;
  ProfScope prof(a.mode == 0 ? "attention_decode" : "attention_rows", stream, 4.0 * a.hd * (double)H * keys,
                 2.0 * (2.0 * keys + 2.0 * (double)rows) * (double)a.hd * (double)H);
  cudaError_t e = cudaSuccess;
#define NSRL_ROWS_CASE(L)                                                                                  \
  case L:                                                                                                  \
    e = cudaFuncSetAttribute(attention_rows_kernel<L>, cudaFuncAttributeMaxDynamicSharedMemorySize,        \
                             (int)smem);                                                                   \
    if (e == cudaSuccess) attention_rows_kernel<L><<<grid, 256, smem, stream>>>(a);                       \
    break;
  switch (lpk) {
    NSRL_ROWS_CASE(0)
    NSRL_ROWS_CASE(2)
    NSRL_ROWS_CASE(8)
    NSRL_ROWS_CASE(32)
    default:
      return cudaErrorInvalidValue;
  }
#undef NSRL_ROWS_CASE
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention(const Planes& qkv, size_t B, size_t S, size_t d, size_t H, bool causal, Planes ctx,
                             nsrl_device_status* st, cudaStream_t stream) {
  const int hd = (int)(d / H);
  const int shift = __builtin_ctz((unsigned)hd) / 2;
  if ((hd == 64 || hd == 16) && S <= 32768) {
    PrefillArgs a{};
    a.qkv_hi = qkv.hi;
    a.qkv_lo = qkv.lo;
    a.ld = (long long)qkv.ld;
    a.S = (int)S;
    a.d = (int)d;
    a.H = (int)H;
    a.causal = causal ? 1 : 0;
    a.shift = shift;
    a.ctx_hi = ctx.hi;
    a.ctx_lo = ctx.lo;
    a.ctx_l1 = ctx.l1;
    a.ldc = (long long)ctx.ld;
    a.st = st;
    dim3 grid((unsigned)((S + QT - 1) / QT), (unsigned)H, (unsigned)B);
    const double pairs = causal ? (double)S * (S + 1) / 2.0 : (double)S * S;
    ProfScope prof(hd == 64 ? "attention_prefill_hd64" : "attention_prefill_hd16", stream,
                   4.0 * hd * (double)H * (double)B * pairs, 8.0 * (double)(B * S) * (double)d);
    if (hd == 64)
      prefill_attention_kernel<64><<<grid, 128, 0, stream>>>(a);
    else
      prefill_attention_kernel<16><<<grid, 128, 0, stream>>>(a);
    return cudaGetLastError();
  }
  return cudaErrorNotSupported;  // caller falls back to the row kernel on int16 operands
}

// Causal attention over int16 q, k, v rows of stride ld (sequence b at row
// b * S) -> ctx int16 [B*S][d] and the probabilities P [B][H][S][S].
cudaError_t launch_attention_rows_probs(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld, size_t B,
                                        size_t S, size_t d, size_t H, int16_t* ctx, int16_t* probs,
                                        nsrl_device_status* st, cudaStream_t stream) {
  RowArgs a{};
  a.q = q;
  a.ldq = (long long)ld;
  a.k = k;
  a.v = v;
  a.ldkv = (long long)ld;
  a.kv_seq = (long long)(S * ld);
  a.rows_per_seq = (int)S;
  a.mode = 1;
  a.lens = nullptr;
  a.Lmax = (int)S;
  a.hd = (int)(d / H);
  a.shift = __builtin_ctz((unsigned)a.hd) / 2;
  a.out = ctx;
  a.ldo = (long long)d;
  a.probs = probs;
  a.st = st;
  return launch_rows(a, (long long)(B * S), (int)H, stream);
}

// Fallback core over int16 q|k|v [B*S][3d] -> ctx int16 [B*S][d].
cudaError_t launch_attention_rows_i16(const int16_t* qkv, size_t B, size_t S, size_t d, size_t H, bool causal,
                                      int16_t* ctx, nsrl_device_status* st, cudaStream_t stream) {
  RowArgs a{};
  a.q = qkv;
  a.ldq = (long long)(3 * d);
  a.k = qkv + d;
  a.v = qkv + 2 * d;
  a.ldkv = (long long)(3 * d);
  a.kv_seq = (long long)(S * 3 * d);
  a.rows_per_seq = (int)S;
  a.mode = causal ? 1 : 2;
  a.lens = nullptr;
  a.Lmax = (int)S;
  a.hd = (int)(d / H);
  a.shift = __builtin_ctz((unsigned)a.hd) / 2;
  a.out = ctx;
  a.ldo = (long long)d;
  a.st = st;
  return launch_rows(a, (long long)(B * S), (int)H, stream);
}

__global__ void kv_append_kernel(const int8_t* __restrict__ hi, const uint8_t* __restrict__ lo, long long ld, int d,
                                 int hd, const int32_t* __restrict__ pos, int Lmax, int16_t* __restrict__ q16,
                                 int16_t* __restrict__ kc, int16_t* __restrict__ vc, nsrl_device_status* st) {
  const int b = blockIdx.x;
  const int p = pos[b];
  const bool ok = p >= 0 && p < Lmax;
  if (!ok) {
    if (threadIdx.x == 0) nsrl_flag(st, NSRL_FLAG_BAD_LENGTH);
    return;
  }
  const long long row = (long long)b * ld;
  const int H = d / hd;
  for (int c = threadIdx.x; c < d; c += blockDim.x) {
    // cache [B][H][Lmax][hd]: head c / hd, dim c % hd
    const long long off = (((long long)b * H + c / hd) * Lmax + p) * hd + c % hd;
    q16[(long long)b * d + c] = (int16_t)((int)hi[row + c] * 256 + (int)lo[row + c]);
    kc[off] = (int16_t)((int)hi[row + d + c] * 256 + (int)lo[row + d + c]);
    vc[off] = (int16_t)((int)hi[row + 2 * d + c] * 256 + (int)lo[row + 2 * d + c]);
  }
}

cudaError_t launch_kv_append(const Planes& qkv, size_t B, size_t d, size_t hd, const int32_t* pos, size_t Lmax,
                             int16_t* q16, int16_t* k_cache, int16_t* v_cache, nsrl_device_status* st,
                             cudaStream_t stream) {
  if (B == 0) return cudaSuccess;
  ProfScope prof("kv_append", stream, 0.0, 6.0 * (double)(B * d) + 6.0 * (double)(B * d));
  kv_append_kernel<<<(unsigned)B, 256, 0, stream>>>(qkv.hi, qkv.lo, (long long)qkv.ld, (int)d, (int)hd, pos, (int)Lmax,
                                                     q16, k_cache, v_cache, st);
  return cudaGetLastError();
}

cudaError_t launch_decode_tma(const int16_t* q, const int16_t* kc, const int16_t* vc, const int32_t* lens,
                              size_t B, size_t H, size_t hd, size_t Lmax, int16_t* ctx, nsrl_device_status* st,
                              cudaStream_t stream, int len_offset, bool head_major);

cudaError_t launch_decode_attention(const int16_t* q, const int16_t* kc, const int16_t* vc, const int32_t* lens,
                                    size_t B, size_t H, size_t hd, size_t Lmax, int16_t* ctx,
                                    nsrl_device_status* st, cudaStream_t stream, int len_offset, bool head_major) {
  if (B == 0) return cudaSuccess;
  const cudaError_t e = launch_decode_tma(q, kc, vc, lens, B, H, hd, Lmax, ctx, st, stream, len_offset, head_major);
  if (e != cudaErrorNotSupported || head_major) return e;
  const size_t d = H * hd;
  RowArgs a{};
  a.q = q;
  a.ldq = (long long)d;
  a.k = kc;
  a.v = vc;
  a.ldkv = (long long)d;
  a.kv_seq = (long long)(Lmax * d);
  a.rows_per_seq = 1;
  a.mode = 0;
  a.len_offset = len_offset;
  a.lens = lens;
  a.Lmax = (int)Lmax;
  a.hd = (int)hd;
  a.shift = __builtin_ctz((unsigned)hd) / 2;
  a.out = ctx;
  a.ldo = (long long)d;
  a.st = st;
  return launch_rows(a, (long long)B, (int)H, stream);
}

}  // namespace nsrl
