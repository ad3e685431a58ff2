// Softmax-attention backward on the int8 tensor cores (mma.sync m16n8k32),
// crates/nsrl-train/src/lib.rs:16623-16900, per (sequence, head):
//   dP[t][j] = sat(rhu(dC[t] . V[j], 15))                          j <= t
//   dL[t][j] = sat(rhu(P[t][j] (dP[t][j] - rhu(sum_j dP P, 15)) 22713, 30))
//   dQ[t]    = sat(rhu(sum_{j<=t} dL[t][j] K[j], log4 hd))
//   dK[j]    = sat(rhu(sum_{t>=j} dL[t][j] Q[t], log4 hd))
//   dV[j]    = sat(rhu(sum_t P[t][j] dC[t], 15))
// Every product is i16 x i16 = (256 ah + al)(256 bh + bl): four int8 MMAs
// into three s32 sums (hh, mid = ah bl + al bh, ll), recombined in i64.  Per
// product |mid| <= 65280 and ll <= 65025, so the sums are exact for up to
// 32768 terms (seq_len <= 16384, head_dim <= 64).
//
// attn_bwd_q_kernel: one CTA of 4 warps per 64 query rows.  Pass 1 forms dP
//   tile by tile and the row sums sum_j dP P; pass 2 forms dP again, then dL
//   (written to global for the key side) and dQ += dL K, dL entering the MMA
//   as A fragments straight from the dP accumulator layout (K^T is staged in
//   the matching key order).
// attn_bwd_kv_kernel: one CTA per 64 keys; dK (A = dL^T) or dV (A = P^T)
//   over the query tiles at or after the keys, operands staged transposed as
//   byte planes in shared memory.
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

#define NSRL_BWD_MMA(NAME, TA, TB)                                                                          \
  __device__ __forceinline__ void NAME(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {     \
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." TA "." TB                                        \
                 ".s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"                               \
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])                                           \
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));                           \
  }
NSRL_BWD_MMA(bmma_ss, "s8", "s8")
NSRL_BWD_MMA(bmma_su, "s8", "u8")
NSRL_BWD_MMA(bmma_us, "u8", "s8")
NSRL_BWD_MMA(bmma_uu, "u8", "u8")

__device__ __forceinline__ uint32_t lds32b(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Position of key j (0..31) in the MMA k order that matches the C-fragment
// layout of an S tile (see the forward prefill kernel).
__device__ __forceinline__ int bkey_slot(int j) {
  return 16 * (j >> 4) + 4 * ((j & 7) >> 1) + 2 * ((j & 15) >> 3) + (j & 1);
}

// Four int16 values -> their hi bytes and lo bytes, packed.
__device__ __forceinline__ void split4(const int16_t* v, uint32_t& hi, uint32_t& lo) {
  uint32_t h = 0, l = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    h |= (uint32_t)(((int)v[e] >> 8) & 255) << (8 * e);
    l |= (uint32_t)((int)v[e] & 255) << (8 * e);
  }
  hi = h;
  lo = l;
}

constexpr int BQ = 64;  // query rows per CTA (4 warps x 16)
constexpr int BK = 32;  // keys per tile

// ---------------------------------------------------------------- planes --
// Row p of a 32-key block holds key bkey_inv(p): the inverse of bkey_slot.
__device__ __forceinline__ int bkey_inv(int p) { return 16 * (p >> 4) + 8 * ((p >> 1) & 1) + 2 * ((p >> 2) & 3) + (p & 1); }

// X rows (row b*S + s, columns h*HD .. +HD, stride ld) -> per-head transposed
// byte planes XT[((b*H + h)*HD + dim)*Sp + p]: p = s, or with perm the
// MMA key order inside each 32-key block (zeros past S up to Sp).
template <int HD>
__global__ void __launch_bounds__(256) head_transpose_kernel(const int16_t* __restrict__ x, long long ld, int S, int Sp,
                                                             int H, bool perm, int8_t* __restrict__ th,
                                                             uint8_t* __restrict__ tl) {
  __shared__ int16_t tile[64][HD + 2];
  const int s0 = blockIdx.x * 64, h = blockIdx.y, b = blockIdx.z;
  for (int i = threadIdx.x; i < 64 * (HD / 4); i += 256) {
    const int r = i / (HD / 4), c4 = 4 * (i % (HD / 4));
    int16_t v[4] = {0, 0, 0, 0};
    if (s0 + r < S) {
      const uint2 u = *reinterpret_cast<const uint2*>(x + ((long long)b * S + s0 + r) * ld + (long long)h * HD + c4);
      v[0] = (int16_t)(u.x & 0xFFFF);
      v[1] = (int16_t)(u.x >> 16);
      v[2] = (int16_t)(u.y & 0xFFFF);
      v[3] = (int16_t)(u.y >> 16);
    }
#pragma unroll
    for (int z = 0; z < 4; ++z) tile[r][c4 + z] = v[z];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < HD * 16; i += 256) {
    const int dim = i / 16, w = i % 16;  // word w: positions s0 + 4w .. +3
    const int p0 = s0 + 4 * w;
    if (p0 >= Sp) continue;
    uint32_t hv = 0, lv = 0;
#pragma unroll
    for (int z = 0; z < 4; ++z) {
      const int pl = 4 * w + z;  // position inside this 64-wide tile
      const int src = perm ? (pl & ~31) + bkey_inv(pl & 31) : pl;
      const int v = (s0 + src < S) ? tile[src][dim] : 0;
      hv |= (uint32_t)((v >> 8) & 255) << (8 * z);
      lv |= (uint32_t)(v & 255) << (8 * z);
    }
    const long long off = (((long long)b * H + h) * HD + dim) * Sp + p0;
    *reinterpret_cast<uint32_t*>(th + off) = hv;
    *reinterpret_cast<uint32_t*>(tl + off) = lv;
  }
}

// M [BH][S][S] int16 -> MT byte planes, MT[bh][j][i] = M[bh][i][j], for the
// tiles with i-tile >= j-tile (the causal part the key side reads).
__global__ void __launch_bounds__(256) sq_transpose_kernel(const int16_t* __restrict__ M, int S,
                                                           int8_t* __restrict__ th, uint8_t* __restrict__ tl) {
  const int j0 = blockIdx.x * 64, i0 = blockIdx.y * 64;
  if (i0 + 63 < j0) return;
  __shared__ int16_t tile[64][66];  // [i][j]
  const long long base = (long long)blockIdx.z * S * S;
  for (int e = threadIdx.x; e < 64 * 16; e += 256) {
    const int r = e >> 4, c4 = 4 * (e & 15);
    int16_t v[4] = {0, 0, 0, 0};
    if (i0 + r < S && j0 + c4 < S) {  // S % 4 == 0: the four columns are all inside
      const uint2 u = *reinterpret_cast<const uint2*>(M + base + (long long)(i0 + r) * S + j0 + c4);
      v[0] = (int16_t)(u.x & 0xFFFF);
      v[1] = (int16_t)(u.x >> 16);
      v[2] = (int16_t)(u.y & 0xFFFF);
      v[3] = (int16_t)(u.y >> 16);
    }
#pragma unroll
    for (int z = 0; z < 4; ++z) tile[r][c4 + z] = v[z];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 64 * 16; e += 256) {
    const int jr = e >> 4, i4 = 4 * (e & 15);
    if (j0 + jr >= S || i0 + i4 >= S) continue;
    uint32_t hv = 0, lv = 0;
#pragma unroll
    for (int z = 0; z < 4; ++z) {
      const int v = tile[i4 + z][jr];
      hv |= (uint32_t)((v >> 8) & 255) << (8 * z);
      lv |= (uint32_t)(v & 255) << (8 * z);
    }
    const long long off = base + (long long)(j0 + jr) * S + i0 + i4;
    *reinterpret_cast<uint32_t*>(th + off) = hv;
    *reinterpret_cast<uint32_t*>(tl + off) = lv;
  }
}

// ---------------------------------------------------------------- query side --
struct QArgs {
  const int16_t* dC;
  long long ldc;
  const int8_t* v_hi;   // V planes [T][d]
  const uint8_t* v_lo;
  int d;
  const int8_t* kt_hi;  // K^T planes [B][H][HD][Sp], MMA key order per 32-key block
  const uint8_t* kt_lo;
  int Sp;
  const int16_t* P;
  int S, H, shift;
  int16_t* dL;
  int16_t* dQ;
  long long ldo;
  nsrl_device_status* st;
};

template <int HD>
struct QSmem {
  static constexpr int KSTR = HD == 16 ? 48 : HD + 16;
  static constexpr int VSTR = 48;
  uint8_t v_hi[BK * KSTR];
  uint8_t v_lo[BK * KSTR];
  uint8_t kt_hi[HD * VSTR];
  uint8_t kt_lo[HD * VSTR];
};

template <int HD>
__global__ void __launch_bounds__(128) attn_bwd_q_kernel(const QArgs a) {
  constexpr int KC = HD >= 32 ? HD / 32 : 1;
  constexpr int NT = HD / 8;
  __shared__ __align__(16) QSmem<HD> sm;
  constexpr int KSTR = QSmem<HD>::KSTR, VSTR = QSmem<HD>::VSTR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S;
  const long long row0 = (long long)b * S;
  const int qw = q0 + warp * 16;
  const int r0 = qw + g, r1 = r0 + 8;
  const int16_t* Pbh = a.P + ((long long)b * a.H + h) * S * (long long)S;
  int16_t* dLbh = a.dL + ((long long)b * a.H + h) * S * (long long)S;
  const long long ktb = ((long long)b * a.H + h) * HD * (long long)a.Sp;

  // A fragments of dC rows r0 / r1 (k = dims)
  uint32_t ca_hi[KC][4], ca_lo[KC][4];
#pragma unroll
  for (int c = 0; c < KC; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (i & 1) ? r1 : r0;
      const int k = 32 * c + 4 * t + ((i & 2) ? 16 : 0);
      uint32_t hv = 0, lv = 0;
      if (r < S && k < HD) {
        const uint2 u = *reinterpret_cast<const uint2*>(a.dC + (row0 + r) * a.ldc + (long long)h * HD + k);
        split4(reinterpret_cast<const int16_t*>(&u), hv, lv);
      }
      ca_hi[c][i] = hv;
      ca_lo[c][i] = lv;
    }
  if (HD == 16) {  // the k half past the head's 16 dims is zero in every V row
    for (int i = tid; i < BK; i += 128) {
      *reinterpret_cast<uint4*>(&sm.v_hi[i * KSTR + 16]) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(&sm.v_lo[i * KSTR + 16]) = make_uint4(0, 0, 0, 0);
    }
  }

  const int kend = min(S, q0 + BQ);  // keys visited by this CTA (causal)
  const int ntiles = (kend + BK - 1) / BK;
  const int wlast = min(qw + 15, S - 1);
  long long wsum[2] = {0, 0}, wq[2] = {0, 0};
  int dq_hh[NT][4], dq_mid[NT][4], dq_ll[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) dq_hh[n][i] = dq_mid[n][i] = dq_ll[n][i] = 0;
  bool neg = false;

  for (int pass = 0; pass < 2; ++pass) {
    for (int kt = 0; kt < ntiles; ++kt) {
      const int kb = kt * BK;
      __syncthreads();
      // V rows [key][dim]: 16-byte copies of the planes
      for (int i = tid; i < BK * (HD / 16); i += 128) {
        const int j = i / (HD / 16), c16 = 16 * (i % (HD / 16));
        const int key = kb + j;
        uint4 vh = make_uint4(0, 0, 0, 0), vl = vh;
        if (key < kend) {
          const long long off = (row0 + key) * a.d + (long long)h * HD + c16;
          vh = *reinterpret_cast<const uint4*>(a.v_hi + off);
          vl = *reinterpret_cast<const uint4*>(a.v_lo + off);
        }
        *reinterpret_cast<uint4*>(&sm.v_hi[j * KSTR + c16]) = vh;
        *reinterpret_cast<uint4*>(&sm.v_lo[j * KSTR + c16]) = vl;
      }
      if (pass == 1) {  // K^T [dim][32 key slots]: two 16-byte copies per dim and plane
        for (int i = tid; i < HD * 2; i += 128) {
          const int dim = i >> 1, half = 16 * (i & 1);
          const long long off = ktb + (long long)dim * a.Sp + kb + half;
          *reinterpret_cast<uint4*>(&sm.kt_hi[dim * VSTR + half]) = *reinterpret_cast<const uint4*>(a.kt_hi + off);
          *reinterpret_cast<uint4*>(&sm.kt_lo[dim * VSTR + half]) = *reinterpret_cast<const uint4*>(a.kt_lo + off);
        }
      }
      __syncthreads();
      if (kb > wlast || qw >= S) continue;  // fully masked for this warp

      // dP raw sums for 16 rows x 32 keys
      int s_hh[4][4], s_mid[4][4], s_ll[4][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) s_hh[j][i] = s_mid[j][i] = s_ll[j][i] = 0;
        const uint8_t* vh = &sm.v_hi[(8 * j + g) * KSTR + 4 * t];
        const uint8_t* vl = &sm.v_lo[(8 * j + g) * KSTR + 4 * t];
#pragma unroll
        for (int c = 0; c < KC; ++c) {
          const uint32_t bh0 = lds32b(vh + 32 * c), bl0 = lds32b(vl + 32 * c);
          const uint32_t bh1 = lds32b(vh + 32 * c + 16), bl1 = lds32b(vl + 32 * c + 16);
          bmma_ss(s_hh[j], ca_hi[c], bh0, bh1);
          bmma_su(s_mid[j], ca_hi[c], bl0, bl1);
          bmma_us(s_mid[j], ca_lo[c], bh0, bh1);
          bmma_uu(s_ll[j], ca_lo[c], bl0, bl1);
        }
      }
      int dl[2][8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {  // row r0 (hf 0) or r1 (hf 1): C elements 2 hf, 2 hf + 1
          const int r = hf ? r1 : r0;
          const int key = kb + 8 * j + 2 * t;
          int pv[2] = {0, 0};
          const bool rl = r < S;
          if (rl && key < S) {  // the two probabilities of this pair of keys
            const uint32_t u = *reinterpret_cast<const uint32_t*>(Pbh + (long long)r * S + key);
            pv[0] = (int)(int16_t)(u & 0xFFFF);
            pv[1] = (int)(int16_t)(u >> 16);
          }
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int i = 2 * hf + e;
            const int kk = key + e;
            const bool live = rl && kk <= r && kk < S;
            int out = 0;
            if (live) {
              // dP = sat(rhu(65536 hh + rm, 15)) with rm = 256 mid + ll (|rm| < 2^31 for
              // head_dim <= 64): 65536 hh is a multiple of 2^15, so the rounded shift is
              // 2 hh + ((rm + 2^14) >> 15), all in i32 (|hh| <= 2^20).
              const int rm = s_mid[j][i] * 256 + s_ll[j][i];
              const int dp = sat16(2 * s_hh[j][i] + ((rm + 16384) >> 15));
              neg |= pv[e] < 0;
              if (pass == 0) {
                wsum[hf] += (long long)(dp * pv[e]);  // |dp * p| <= 2^30
              } else {
                // P (dP - wq) 22713 = (22713 P) (dP - wq): 22713 P < 2^30, |dP - wq| < 2^18
                const long long prod = (long long)(pv[e] * 22713) * (long long)(dp - (int)wq[hf]);
                out = sat16((int)((prod + (1ll << 29)) >> 30));
              }
            }
            dl[hf][2 * j + e] = out;
          }
        }
      }
      if (pass == 0) continue;
      // dL to global (the key side reads it), then the dQ product
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = hf ? r1 : r0;
          const int key = kb + 8 * j + 2 * t;
          if (r < S && key < S)
            *reinterpret_cast<uint32_t*>(dLbh + (long long)r * S + key) =
                (uint32_t)(dl[hf][2 * j] & 0xFFFF) | ((uint32_t)dl[hf][2 * j + 1] << 16);
        }
      uint32_t ah[4], al[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int hf = i & 1;
        const int base = (i & 2) ? 4 : 0;
        uint32_t hv = 0, lv = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int v = dl[hf][base + e];
          hv |= (uint32_t)((v >> 8) & 255) << (8 * e);
          lv |= (uint32_t)(v & 255) << (8 * e);
        }
        ah[i] = hv;
        al[i] = lv;
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint8_t* kh = &sm.kt_hi[(8 * n + g) * VSTR + 4 * t];
        const uint8_t* kl = &sm.kt_lo[(8 * n + g) * VSTR + 4 * t];
        const uint32_t bh0 = lds32b(kh), bh1 = lds32b(kh + 16), bl0 = lds32b(kl), bl1 = lds32b(kl + 16);
        bmma_ss(dq_hh[n], ah, bh0, bh1);
        bmma_su(dq_mid[n], ah, bl0, bl1);
        bmma_us(dq_mid[n], al, bh0, bh1);
        bmma_uu(dq_ll[n], al, bl0, bl1);
      }
    }
    if (pass == 0) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) wsum[hf] += __shfl_xor_sync(0xffffffffu, wsum[hf], o);
        wq[hf] = rhu64(wsum[hf], 15);
      }
    }
  }
  if (neg) nsrl_flag(a.st, NSRL_FLAG_LINEAR_OVERFLOW);  // a negative probability: the reference rejects
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = hf ? r1 : r0;
      if (r >= S) continue;
      int v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * hf + e;
        const long long tot = (long long)dq_hh[n][i] * 65536 + (long long)dq_mid[n][i] * 256 + (long long)dq_ll[n][i];
        v[e] = sat_i16(rhu64(tot, (uint32_t)a.shift));
      }
      *reinterpret_cast<uint32_t*>(a.dQ + (row0 + r) * a.ldo + (long long)h * HD + 8 * n + 2 * t) =
          (uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16);
    }
}

// ------------------------------------------------------------------ key side --
struct KVArgs {
  const int8_t* mt_hi;  // M^T planes [BH][S][S]: row = key, column = query
  const uint8_t* mt_lo;
  const int8_t* xt_hi;  // X^T planes [BH][HD][S]
  const uint8_t* xt_lo;
  int S, H, shift;
  int16_t* out;
  long long ldo;
};

template <int HD>
struct KVSmem {
  static constexpr int ASTR = 48;  // 32 queries + padding, bytes
  uint8_t at_hi[BQ * ASTR];        // [key][query]
  uint8_t at_lo[BQ * ASTR];
  uint8_t xt_hi[HD * ASTR];        // [dim][query]
  uint8_t xt_lo[HD * ASTR];
};

// out[j] = sat(rhu(sum_{t >= j} M[t][j] X[t], shift)) for the 64 keys j of this CTA.
template <int HD>
__global__ void __launch_bounds__(128) attn_bwd_kv_kernel(const KVArgs a) {
  constexpr int NT = HD / 8;
  __shared__ __align__(16) KVSmem<HD> sm;
  constexpr int ASTR = KVSmem<HD>::ASTR;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int k0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S;
  const long long row0 = (long long)b * S;
  const long long bh = (long long)b * a.H + h;
  const int kw = k0 + warp * 16;  // this warp's keys kw + g, kw + g + 8
  int acc_hh[NT][4], acc_mid[NT][4], acc_ll[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc_hh[n][i] = acc_mid[n][i] = acc_ll[n][i] = 0;

  for (int tq = k0; tq < S; tq += BK) {
    __syncthreads();
    // M^T rows (keys) x 32 queries, 4-byte copies (S % 4 == 0)
    for (int i = tid; i < BQ * 8; i += 128) {
      const int kr = i >> 3, w4 = 4 * (i & 7);
      uint32_t vh = 0, vl = 0;
      if (k0 + kr < S && tq + w4 < S) {
        const long long off = (bh * S + k0 + kr) * (long long)S + tq + w4;
        vh = *reinterpret_cast<const uint32_t*>(a.mt_hi + off);
        vl = *reinterpret_cast<const uint32_t*>(a.mt_lo + off);
      }
      *reinterpret_cast<uint32_t*>(&sm.at_hi[kr * ASTR + w4]) = vh;
      *reinterpret_cast<uint32_t*>(&sm.at_lo[kr * ASTR + w4]) = vl;
    }
    // X^T dims x 32 queries
    for (int i = tid; i < HD * 8; i += 128) {
      const int dim = i >> 3, w4 = 4 * (i & 7);
      uint32_t vh = 0, vl = 0;
      if (tq + w4 < S) {
        const long long off = (bh * HD + dim) * (long long)S + tq + w4;
        vh = *reinterpret_cast<const uint32_t*>(a.xt_hi + off);
        vl = *reinterpret_cast<const uint32_t*>(a.xt_lo + off);
      }
      *reinterpret_cast<uint32_t*>(&sm.xt_hi[dim * ASTR + w4]) = vh;
      *reinterpret_cast<uint32_t*>(&sm.xt_lo[dim * ASTR + w4]) = vl;
    }
    __syncthreads();
    if (kw >= S || tq + BK - 1 < kw) continue;  // keys past the sequence, or queries all before them
    uint32_t ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int kr = warp * 16 + g + ((i & 1) ? 8 : 0);
      const int qc = 4 * t + ((i & 2) ? 16 : 0);
      ah[i] = lds32b(&sm.at_hi[kr * ASTR + qc]);
      al[i] = lds32b(&sm.at_lo[kr * ASTR + qc]);
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const uint8_t* xh = &sm.xt_hi[(8 * n + g) * ASTR + 4 * t];
      const uint8_t* xl = &sm.xt_lo[(8 * n + g) * ASTR + 4 * t];
      const uint32_t bh0 = lds32b(xh), bh1 = lds32b(xh + 16), bl0 = lds32b(xl), bl1 = lds32b(xl + 16);
      bmma_ss(acc_hh[n], ah, bh0, bh1);
      bmma_su(acc_mid[n], ah, bl0, bl1);
      bmma_us(acc_mid[n], al, bh0, bh1);
      bmma_uu(acc_ll[n], al, bl0, bl1);
    }
  }
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int kr = kw + g + (hf ? 8 : 0);
      if (kr >= S) continue;
      int v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * hf + e;
        const long long tot =
            (long long)acc_hh[n][i] * 65536 + (long long)acc_mid[n][i] * 256 + (long long)acc_ll[n][i];
        v[e] = sat_i16(rhu64(tot, (uint32_t)a.shift));
      }
      *reinterpret_cast<uint32_t*>(a.out + (row0 + kr) * a.ldo + (long long)h * HD + 8 * n + 2 * t) =
          (uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16);
    }
}

// attn_bwd_kv_kernel for S % 16 == 0 with 16-byte staging prefetched one
// tile ahead into registers (double-buffered shared memory), and 8 warps for
// head_dim 64: warp w owns keys 16 (w & 3) .. +15 and dims 32 (w >> 2) .. +31,
// so each warp keeps 48 accumulator registers instead of 96.
template <int HD>
__global__ void __launch_bounds__(HD == 64 ? 256 : 128) attn_bwd_kv2_kernel(const KVArgs a) {
  constexpr int WN = HD < 32 ? HD : 32;  // dims per warp
  constexpr int NT = WN / 8;
  constexpr int NTHREADS = 128 * (HD / WN);
  constexpr int ASTR = 48;
  constexpr int MWORDS = BQ * 2;        // 16-byte words of one M^T tile plane (64 keys x 32 q)
  constexpr int XWORDS = HD * 2;        // of one X^T tile plane
  constexpr int WORDS = 2 * (MWORDS + XWORDS);
  constexpr int PER = (WORDS + NTHREADS - 1) / NTHREADS;
  __shared__ __align__(16) uint8_t buf[2][2 * (BQ + HD) * ASTR];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int k0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S;
  const long long row0 = (long long)b * S;
  const long long bh = (long long)b * a.H + h;
  const int kw = k0 + (warp & 3) * 16;
  const int d0 = (warp >> 2) * WN;
  int acc_hh[NT][4], acc_mid[NT][4], acc_ll[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc_hh[n][i] = acc_mid[n][i] = acc_ll[n][i] = 0;

  // word e of a tile: [M^T hi | M^T lo | X^T hi | X^T lo], two 16-byte words per row
  auto load_tile = [&](int tq, uint4 (&r)[PER]) {
#pragma unroll
    for (int z = 0; z < PER; ++z) {
      const int e = tid + z * NTHREADS;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (e < WORDS) {
        const int part = e < 2 * MWORDS ? 0 : 1;
        const int ee = part == 0 ? e : e - 2 * MWORDS;
        const int pw = part == 0 ? MWORDS : XWORDS;
        const int plane = ee / pw, w = ee % pw;
        const int row = w >> 1, half = 16 * (w & 1);
        const int q = tq + half;
        if (q < S) {
          if (part == 0) {
            if (k0 + row < S) {
              const long long off = (bh * S + k0 + row) * (long long)S + q;
              v = plane ? *reinterpret_cast<const uint4*>(a.mt_lo + off) : *reinterpret_cast<const uint4*>(a.mt_hi + off);
            }
          } else {
            const long long off = (bh * HD + row) * (long long)S + q;
            v = plane ? *reinterpret_cast<const uint4*>(a.xt_lo + off) : *reinterpret_cast<const uint4*>(a.xt_hi + off);
          }
        }
      }
      r[z] = v;
    }
  };
  auto store_tile = [&](int sb, const uint4 (&r)[PER]) {
#pragma unroll
    for (int z = 0; z < PER; ++z) {
      const int e = tid + z * NTHREADS;
      if (e >= WORDS) continue;
      const int part = e < 2 * MWORDS ? 0 : 1;
      const int ee = part == 0 ? e : e - 2 * MWORDS;
      const int pw = part == 0 ? MWORDS : XWORDS;
      const int plane = ee / pw, w = ee % pw;
      const int row = w >> 1, half = 16 * (w & 1);
      // layout: at_hi [BQ][ASTR], at_lo, xt_hi [HD][ASTR], xt_lo
      const int base = part == 0 ? plane * BQ * ASTR : 2 * BQ * ASTR + plane * HD * ASTR;
      *reinterpret_cast<uint4*>(&buf[sb][base + row * ASTR + half]) = r[z];
    }
  };

  uint4 pre[PER];
  load_tile(k0, pre);
  store_tile(0, pre);
  __syncthreads();
  int sb = 0;
  for (int tq = k0; tq < S; tq += BK, sb ^= 1) {
    const bool more = tq + BK < S;
    if (more) load_tile(tq + BK, pre);  // in flight during the MMAs below
    if (kw < S && tq + BK - 1 >= kw) {
      const uint8_t* at_hi = &buf[sb][0];
      const uint8_t* at_lo = &buf[sb][BQ * ASTR];
      const uint8_t* xt_hi = &buf[sb][2 * BQ * ASTR];
      const uint8_t* xt_lo = &buf[sb][2 * BQ * ASTR + HD * ASTR];
      uint32_t ah[4], al[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int kr = (warp & 3) * 16 + g + ((i & 1) ? 8 : 0);
        const int qc = 4 * t + ((i & 2) ? 16 : 0);
        ah[i] = lds32b(at_hi + kr * ASTR + qc);
        al[i] = lds32b(at_lo + kr * ASTR + qc);
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint8_t* xh = xt_hi + (d0 + 8 * n + g) * ASTR + 4 * t;
        const uint8_t* xl = xt_lo + (d0 + 8 * n + g) * ASTR + 4 * t;
        const uint32_t bh0 = lds32b(xh), bh1 = lds32b(xh + 16), bl0 = lds32b(xl), bl1 = lds32b(xl + 16);
        bmma_ss(acc_hh[n], ah, bh0, bh1);
        bmma_su(acc_mid[n], ah, bl0, bl1);
        bmma_us(acc_mid[n], al, bh0, bh1);
        bmma_uu(acc_ll[n], al, bl0, bl1);
      }
    }
    if (more) store_tile(sb ^ 1, pre);
    __syncthreads();
  }
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int kr = kw + g + (hf ? 8 : 0);
      if (kr >= S) continue;
      int v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * hf + e;
        const long long tot =
            (long long)acc_hh[n][i] * 65536 + (long long)acc_mid[n][i] * 256 + (long long)acc_ll[n][i];
        v[e] = sat_i16(rhu64(tot, (uint32_t)a.shift));
      }
      *reinterpret_cast<uint32_t*>(a.out + (row0 + kr) * a.ldo + (long long)h * HD + d0 + 8 * n + 2 * t) =
          (uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16);
    }
}

}  // namespace

size_t attention_backward_tc_scratch_bytes(size_t B, size_t S, size_t d, size_t H) {
  const size_t Sp = (S + 31) & ~size_t(31);
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  // V planes [T][d], K^T (padded rows), Q^T, dC^T, P^T, dL^T: two planes each
  return 2 * (up(B * S * d) + up(B * d * Sp) + 2 * up(B * d * S) + 2 * up(B * H * S * S));
}

// dQ, dK, dV (and dL into `dl`, zeroed here) of causal attention on int16
// operands: q, k, v rows of stride ld, P [B][H][S][S], dC rows of stride ldc;
// outputs [B*S][d].  head_dim 16 or 64, S a multiple of 4, d a multiple of 16
// (else cudaErrorNotSupported).  scratch: attention_backward_tc_scratch_bytes.
cudaError_t launch_attention_backward_tc(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld,
                                         const int16_t* P, const int16_t* dC, size_t ldc, size_t B, size_t S, size_t d,
                                         size_t H, int16_t* dl, int16_t* dq, int16_t* dk, int16_t* dv,
                                         void* scratch, size_t scratch_bytes, nsrl_device_status* st,
                                         cudaStream_t s) {
  const size_t hd = d / H;
  // 8-byte loads of P / dL rows, dC, q, k, v need S, ld, ldc multiples of 4
  if ((hd != 16 && hd != 64) || S % 4 != 0 || ld % 4 != 0 || ldc % 4 != 0 || d % 16 != 0 || S > 16384 ||
      !scratch || scratch_bytes < attention_backward_tc_scratch_bytes(B, S, d, H))
    return cudaErrorNotSupported;
  const int shift = __builtin_ctzll(hd) / 2;
  const size_t Sp = (S + 31) & ~size_t(31);
  uint8_t* w = static_cast<uint8_t*>(scratch);
  size_t off = 0;
  auto take = [&](size_t n) {
    uint8_t* p = w + off;
    off += (n + 255) & ~size_t(255);
    return p;
  };
  int8_t* vph = reinterpret_cast<int8_t*>(take(B * S * d));
  uint8_t* vpl = take(B * S * d);
  int8_t* kth = reinterpret_cast<int8_t*>(take(B * d * Sp));
  uint8_t* ktl = take(B * d * Sp);
  int8_t* qth = reinterpret_cast<int8_t*>(take(B * d * S));
  uint8_t* qtl = take(B * d * S);
  int8_t* cth = reinterpret_cast<int8_t*>(take(B * d * S));
  uint8_t* ctl = take(B * d * S);
  int8_t* pth = reinterpret_cast<int8_t*>(take(B * H * S * S));
  uint8_t* ptl = take(B * H * S * S);
  int8_t* lth = reinterpret_cast<int8_t*>(take(B * H * S * S));
  uint8_t* ltl = take(B * H * S * S);
  cudaError_t e = cudaMemsetAsync(dl, 0, B * H * S * S * sizeof(int16_t), s);
  if (e != cudaSuccess) return e;
  const double pairs = (double)B * (double)H * (double)S * (double)(S + 1) / 2.0;
  {
    ProfScope prof("attention_bwd_planes", s, 0.0, 8.0 * (double)B * S * d + 2.0 * 2.0 * (double)B * H * S * S);
    e = launch_split_planes(v, B * S, d, ld, Planes{vph, vpl, nullptr, d}, s);
    if (e != cudaSuccess) return e;
    dim3 tg((unsigned)((S + 63) / 64), (unsigned)H, (unsigned)B);
    if (hd == 64) {
      head_transpose_kernel<64><<<tg, 256, 0, s>>>(k, (long long)ld, (int)S, (int)Sp, (int)H, true, kth, ktl);
      head_transpose_kernel<64><<<tg, 256, 0, s>>>(q, (long long)ld, (int)S, (int)S, (int)H, false, qth, qtl);
      head_transpose_kernel<64><<<tg, 256, 0, s>>>(dC, (long long)ldc, (int)S, (int)S, (int)H, false, cth, ctl);
    } else {
      head_transpose_kernel<16><<<tg, 256, 0, s>>>(k, (long long)ld, (int)S, (int)Sp, (int)H, true, kth, ktl);
      head_transpose_kernel<16><<<tg, 256, 0, s>>>(q, (long long)ld, (int)S, (int)S, (int)H, false, qth, qtl);
      head_transpose_kernel<16><<<tg, 256, 0, s>>>(dC, (long long)ldc, (int)S, (int)S, (int)H, false, cth, ctl);
    }
    dim3 sg((unsigned)((S + 63) / 64), (unsigned)((S + 63) / 64), (unsigned)(B * H));
    sq_transpose_kernel<<<sg, 256, 0, s>>>(P, (int)S, pth, ptl);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  dim3 grid((unsigned)((S + BQ - 1) / BQ), (unsigned)H, (unsigned)B);
  QArgs qa{dC, (long long)ldc, vph, vpl, (int)d, kth, ktl, (int)Sp, P, (int)S, (int)H, shift, dl, dq, (long long)d, st};
  {
    ProfScope prof("attention_bwd_q", s, 3.0 * 2.0 * (double)hd * pairs,
                   2.0 * 2.0 * (double)B * H * S * S + 8.0 * (double)B * S * d);
    if (hd == 64)
      attn_bwd_q_kernel<64><<<grid, 128, 0, s>>>(qa);
    else
      attn_bwd_q_kernel<16><<<grid, 128, 0, s>>>(qa);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  {
    dim3 sg((unsigned)((S + 63) / 64), (unsigned)((S + 63) / 64), (unsigned)(B * H));
    ProfScope prof("attention_bwd_planes", s, 0.0, 4.0 * (double)B * H * S * S);
    sq_transpose_kernel<<<sg, 256, 0, s>>>(dl, (int)S, lth, ltl);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  KVArgs ka{lth, ltl, qth, qtl, (int)S, (int)H, shift, dk, (long long)d};
  KVArgs va{pth, ptl, cth, ctl, (int)S, (int)H, 15, dv, (long long)d};
  ProfScope prof("attention_bwd_kv", s, 2.0 * 2.0 * (double)hd * pairs,
                 2.0 * 2.0 * (double)B * H * S * S + 8.0 * (double)B * S * d);
  if (S % 16 == 0) {  // 16-byte staging of the M^T and X^T rows
    if (hd == 64) {
      attn_bwd_kv2_kernel<64><<<grid, 256, 0, s>>>(ka);
      attn_bwd_kv2_kernel<64><<<grid, 256, 0, s>>>(va);
    } else {
      attn_bwd_kv2_kernel<16><<<grid, 128, 0, s>>>(ka);
      attn_bwd_kv2_kernel<16><<<grid, 128, 0, s>>>(va);
    }
  } else if (hd == 64) {
    attn_bwd_kv_kernel<64><<<grid, 128, 0, s>>>(ka);
    attn_bwd_kv_kernel<64><<<grid, 128, 0, s>>>(va);
  } else {
    attn_bwd_kv_kernel<16><<<grid, 128, 0, s>>>(ka);
    attn_bwd_kv_kernel<16><<<grid, 128, 0, s>>>(va);
  }
  return cudaGetLastError();
}

}  // namespace nsrl
