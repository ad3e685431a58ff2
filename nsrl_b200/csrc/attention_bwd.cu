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
// attn_bwd_dl_kernel: one CTA of 4 warps per 64 query rows.  Pass 1 forms
//   dP tile by tile and the row sums sum_j dP P; pass 2 turns the stored dP
//   into dL in place (written to global for the dQ and key-side products).
// attn_bwd_dq_kernel: dQ += dL K with the A fragments taken straight from the
//   dL rows (K^T is staged in the matching key order).
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

// The prescaled planes of two adjacent columns col, col + 1 of one row.
__device__ __forceinline__ void store_grad_planes2(const GradPlanes& gp, long long off, int col, const int (&v)[2]) {
  int p[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) p[e] = rhu_i16(v[e], gp.sc[col + e].right_shift);
  *reinterpret_cast<uint16_t*>(gp.hi + off) = (uint16_t)(((p[0] >> 8) & 255) | (((p[1] >> 8) & 255) << 8));
  *reinterpret_cast<uint16_t*>(gp.lo + off) = (uint16_t)((p[0] & 255) | ((p[1] & 255) << 8));
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

// head_transpose_kernel<64> with 16-byte loads and stores (ld % 8 == 0,
// Sp % 16 == 0): the 64 x 64 tile is kept as 32-bit words (two dims) with the
// word index XORed by 8 ((s / 16) mod 4); each thread gathers 16 positions of
// one dim pair.  With perm, position p of a 32-key block reads key
// bkey_inv(p), which stays inside the same 16-row group.
__global__ void __launch_bounds__(128) head_transpose16_kernel(const int16_t* __restrict__ x, long long ld, int S,
                                                               int Sp, int H, bool perm, int8_t* __restrict__ th,
                                                               uint8_t* __restrict__ tl) {
  constexpr int HD = 64;
  __shared__ __align__(16) uint32_t tile[64 * 32];  // [s][dim pair ^ swizzle]
  const int s0 = blockIdx.x * 64, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
#pragma unroll
  for (int z = 0; z < 4; ++z) {
    const int e = tid + 128 * z;
    const int r = e >> 3, c8 = (e & 7) * 8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (s0 + r < S) u = *reinterpret_cast<const uint4*>(x + ((long long)b * S + s0 + r) * ld + (long long)h * HD + c8);
    *reinterpret_cast<uint4*>(&tile[r * 32 + ((c8 >> 1) ^ (((r >> 4) & 3) << 3))]) = u;
  }
  __syncthreads();
  const int dw = tid >> 2;        // dim pair 0..31
  const int pb = (tid & 3) * 16;  // positions s0 + pb .. +15
  const int wc = dw ^ (((pb >> 4) & 3) << 3);
  if (s0 + pb >= Sp) return;
  uint32_t hi[2][4], lo[2][4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int z = 0; z < 4; ++z) {
      const int pl = pb + 4 * q + z;
      const int src = perm ? (pl & ~31) + bkey_inv(pl & 31) : pl;
      w[z] = tile[src * 32 + wc];
    }
    const uint32_t ah = __byte_perm(w[0], w[1], 0x7531), bh = __byte_perm(w[2], w[3], 0x7531);
    const uint32_t al = __byte_perm(w[0], w[1], 0x6420), bl = __byte_perm(w[2], w[3], 0x6420);
    hi[0][q] = __byte_perm(ah, bh, 0x6420);
    hi[1][q] = __byte_perm(ah, bh, 0x7531);
    lo[0][q] = __byte_perm(al, bl, 0x6420);
    lo[1][q] = __byte_perm(al, bl, 0x7531);
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const long long off = (((long long)b * H + h) * HD + 2 * dw + e) * Sp + s0 + pb;
    *reinterpret_cast<uint4*>(th + off) = make_uint4(hi[e][0], hi[e][1], hi[e][2], hi[e][3]);
    *reinterpret_cast<uint4*>(tl + off) = make_uint4(lo[e][0], lo[e][1], lo[e][2], lo[e][3]);
  }
}

// M [BH][S][S] int16 -> MT byte planes, MT[bh][j][i] = M[bh][i][j], for the
// 64 x 64 tiles with i-tile >= j-tile (the causal part the key side reads),
// S % 16 == 0.  16-byte loads of eight j into shared memory, kept as 32-bit
// words (two j) with the word index XORed by 8 ((i / 16) mod 4) so that the
// column reads are conflict-free; each thread then gathers 16 i of one j pair
// and writes 16-byte words of both planes for both j.
__global__ void __launch_bounds__(128) sq_transpose16_kernel(const int16_t* __restrict__ M, int S,
                                                             int8_t* __restrict__ th, uint8_t* __restrict__ tl) {
  const int j0 = blockIdx.x * 64, i0 = blockIdx.y * 64;
  if (i0 + 63 < j0) return;
  __shared__ __align__(16) uint32_t tile[64 * 32];  // [i][j pair ^ swizzle]
  const long long base = (long long)blockIdx.z * S * S;
  const int tid = threadIdx.x;
#pragma unroll
  for (int z = 0; z < 4; ++z) {
    const int e = tid + 128 * z;
    const int r = e >> 3, j8 = (e & 7) * 8;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (i0 + r < S && j0 + j8 < S)  // S % 16 == 0: all eight j are inside
      u = *reinterpret_cast<const uint4*>(M + base + (long long)(i0 + r) * S + j0 + j8);
    *reinterpret_cast<uint4*>(&tile[r * 32 + ((j8 >> 1) ^ (((r >> 4) & 3) << 3))]) = u;
  }
  __syncthreads();
  const int jw = tid >> 2;        // j pair 0..31
  const int ib = (tid & 3) * 16;  // i rows ib .. ib + 15
  const int wc = jw ^ (((ib >> 4) & 3) << 3);
  uint32_t hi[2][4], lo[2][4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t w0 = tile[(ib + 4 * q) * 32 + wc], w1 = tile[(ib + 4 * q + 1) * 32 + wc];
    const uint32_t w2 = tile[(ib + 4 * q + 2) * 32 + wc], w3 = tile[(ib + 4 * q + 3) * 32 + wc];
    const uint32_t ah = __byte_perm(w0, w1, 0x7531), bh = __byte_perm(w2, w3, 0x7531);
    const uint32_t al = __byte_perm(w0, w1, 0x6420), bl = __byte_perm(w2, w3, 0x6420);
    hi[0][q] = __byte_perm(ah, bh, 0x6420);
    hi[1][q] = __byte_perm(ah, bh, 0x7531);
    lo[0][q] = __byte_perm(al, bl, 0x6420);
    lo[1][q] = __byte_perm(al, bl, 0x7531);
  }
  if (i0 + ib >= S) return;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int j = j0 + 2 * jw + e;
    if (j >= S) continue;
    const long long off = base + (long long)j * S + i0 + ib;
    *reinterpret_cast<uint4*>(th + off) = make_uint4(hi[e][0], hi[e][1], hi[e][2], hi[e][3]);
    *reinterpret_cast<uint4*>(tl + off) = make_uint4(lo[e][0], lo[e][1], lo[e][2], lo[e][3]);
  }
}

// The same for S % 4 == 0: 64 x 64 tiles, 8-byte loads, 4-byte stores.
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
struct DlArgs {
  const int16_t* dC;
  long long ldc;
  const int8_t* v_hi;  // V planes [T][d] (row stride d)
  const uint8_t* v_lo;
  int d;
  const int16_t* P;
  int S, H;
  int16_t* dL;  // [BH][S][S]: dP after the first pass, dL after the second
  nsrl_device_status* st;
  // planes form (PL): P read from, and dP / dL written to, [BH][S][S] byte planes
  const int8_t* p_hi;
  const uint8_t* p_lo;
  int8_t* l_hi;
  uint8_t* l_lo;
};

// attn_bwd_dl_kernel: one CTA of 4 warps per 64 query rows.  Pass 1 forms dP
// tile by tile on the tensor cores (V staged 16 bytes at a time, prefetched a
// tile ahead into double-buffered shared memory), stores it into the dL
// buffer and sums dP P per row; pass 2 reads back the values each lane stored
// (its own writes, so no barrier) and turns them into dL in place.  Every key
// below min(S, end of the block) is written, zeros above the diagonal, so the
// causal 64 x 64 tiles the key side reads need no clearing.
//
// PL (S % 16 == 0): P comes from byte planes and dP / dL go to byte planes.
// Lane l of a warp owns the 16-key piece (row qw + l / 2, keys 16 (l % 2) ..
// +15) of each 32-key tile: pass 1 moves P in and dP out as 16-byte plane
// pieces through a per-warp shared tile (the MMA fragments hold 2-key pairs),
// pass 2 works on its own pieces.  The first 64-row block of each 128-row
// block also writes zero planes for keys [q0 + 64, q0 + 128), so every
// 128 x 128 causal tile the tensor-core kernels read is written.
constexpr int PSTR = 20;  // words per row of a warp's staged 16 x 32 pair tile (conflict-free fragment access)

template <int HD, bool PL>
__global__ void __launch_bounds__(128, 5) attn_bwd_dl_kernel(const DlArgs a) {
  constexpr int KC = HD >= 32 ? HD / 32 : 1;
  constexpr int KSTR = HD == 16 ? 48 : HD + 16;  // bytes per staged V row
  constexpr int VW = BK * (HD / 16);            // 16-byte words of one V plane tile
  constexpr int PER = (2 * VW + 127) / 128;
  __shared__ __align__(16) uint8_t vbuf[2][2][BK * KSTR];  // [stage][plane]
  __shared__ __align__(16) uint32_t pstage[PL ? 4 : 1][PL ? 16 * PSTR : 4];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S;
  const long long row0 = (long long)b * S;
  const int qw = q0 + warp * 16;
  const int r0 = qw + g, r1 = r0 + 8;
  const long long mat = ((long long)b * a.H + h) * S * (long long)S;
  const int16_t* Pbh = PL ? nullptr : a.P + mat;
  int16_t* dLbh = PL ? nullptr : a.dL + mat;
  // PL: this lane's piece and the warp's staged tile of key pairs
  const int pr = qw + (lane >> 1), ph = 16 * (lane & 1);
  uint32_t* ps = pstage[PL ? warp : 0];
  uint32_t* pmine = ps + (lane >> 1) * PSTR + 8 * (lane & 1);
  // the piece of tile kb of a plane pair as 8 packed pairs (zeros outside the matrix)
  auto piece_ld = [&](const int8_t* hi, const uint8_t* lo, int kb, uint32_t(&wv)[8]) {
    uint4 H = make_uint4(0, 0, 0, 0), L = H;
    if (pr < S && kb + ph < S) {
      const long long o = mat + (long long)pr * S + kb + ph;
      H = *reinterpret_cast<const uint4*>(hi + o);
      L = *reinterpret_cast<const uint4*>(lo + o);
    }
    const uint32_t hw[4] = {H.x, H.y, H.z, H.w}, lw[4] = {L.x, L.y, L.z, L.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      wv[2 * k] = __byte_perm(lw[k], hw[k], 0x5140);
      wv[2 * k + 1] = __byte_perm(lw[k], hw[k], 0x7362);
    }
  };
  auto piece_st = [&](int kb, const uint32_t(&wv)[8]) {
    if (pr >= S || kb + ph >= S) return;
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      hw[k] = __byte_perm(wv[2 * k], wv[2 * k + 1], 0x7531);
      lw[k] = __byte_perm(wv[2 * k], wv[2 * k + 1], 0x6420);
    }
    const long long o = mat + (long long)pr * S + kb + ph;
    *reinterpret_cast<uint4*>(a.l_hi + o) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(a.l_lo + o) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  };
  if (PL && q0 % 128 == 0 && q0 + BQ < S) {
    // zero planes of rows [q0, q0 + 64) x keys [q0 + 64, min(S, q0 + 128))
    const int kz = q0 + BQ, nz = (min(S, q0 + 128) - kz) / 16;
    for (int i = tid; i < 2 * BQ * nz; i += 128) {
      const int pl = i / (BQ * nz), w = i % (BQ * nz);
      const int r = q0 + w / nz, key = kz + 16 * (w % nz);
      if (r >= S) continue;
      const long long o = mat + (long long)r * S + key;
      uint4* dst = pl ? reinterpret_cast<uint4*>(a.l_lo + o) : reinterpret_cast<uint4*>(a.l_hi + o);
      *dst = make_uint4(0, 0, 0, 0);
    }
  }

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
  if (HD == 16) {  // the k half past the head's 16 dims (A is zero there too)
    for (int i = tid; i < 2 * 2 * BK; i += 128) {
      const int st = i / (2 * BK), pl = (i / BK) & 1, j = i % BK;
      *reinterpret_cast<uint4*>(&vbuf[st][pl][j * KSTR + 16]) = make_uint4(0, 0, 0, 0);
    }
  }

  const int kend = min(S, q0 + BQ);  // keys visited by this CTA (causal)
  const int ntiles = (kend + BK - 1) / BK;
  const int wlast = min(qw + 15, S - 1);

  // word e: plane e / VW, key row (e % VW) / (HD / 16), 16-byte column
  auto load_tile = [&](int kb, uint4(&r)[PER]) {
#pragma unroll
    for (int z = 0; z < PER; ++z) {
      const int e = tid + z * 128;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (e < 2 * VW) {
        const int pl = e / VW, w = e % VW;
        const int key = kb + w / (HD / 16), c16 = 16 * (w % (HD / 16));
        if (key < kend) {
          const long long off = (row0 + key) * a.d + (long long)h * HD + c16;
          v = pl ? *reinterpret_cast<const uint4*>(a.v_lo + off) : *reinterpret_cast<const uint4*>(a.v_hi + off);
        }
      }
      r[z] = v;
    }
  };
  auto store_tile = [&](int sb, const uint4(&r)[PER]) {
#pragma unroll
    for (int z = 0; z < PER; ++z) {
      const int e = tid + z * 128;
      if (e >= 2 * VW) continue;
      const int pl = e / VW, w = e % VW;
      *reinterpret_cast<uint4*>(&vbuf[sb][pl][(w / (HD / 16)) * KSTR + 16 * (w % (HD / 16))]) = r[z];
    }
  };

  long long wsum[2] = {0, 0};
  bool neg = false;
  {
    uint4 pre[PER];
    load_tile(0, pre);
    store_tile(0, pre);
    __syncthreads();
  }
  for (int kt = 0; kt < ntiles; ++kt) {
    const int kb = kt * BK, sb = kt & 1;
    const bool more = kt + 1 < ntiles;
    uint4 pre[PER];
    if (more) load_tile(kb + BK, pre);  // in flight during the MMAs below
    // the probabilities of this tile: rows r0 / r1, key pairs kb + 8 j + 2 t
    uint32_t pw[2][4];
    if constexpr (PL) {
      uint32_t wv[8];
      piece_ld(a.p_hi, a.p_lo, kb, wv);
      reinterpret_cast<uint4*>(pmine)[0] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      reinterpret_cast<uint4*>(pmine)[1] = make_uint4(wv[4], wv[5], wv[6], wv[7]);
      __syncwarp();
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int j = 0; j < 4; ++j) pw[hf][j] = ps[(g + 8 * hf) * PSTR + 4 * j + t];
      __syncwarp();  // read before the dP pairs overwrite the tile
    } else {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = hf ? r1 : r0, key = kb + 8 * j + 2 * t;
          pw[hf][j] = (r < S && key < S) ? *reinterpret_cast<const uint32_t*>(Pbh + (long long)r * S + key) : 0u;
        }
    }
    const bool active = qw < S && kb <= wlast;
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // 8 keys at a time: dP raw sums for 16 rows x 8 keys, then their values
      int s_hh[4] = {0, 0, 0, 0}, s_mid[4] = {0, 0, 0, 0}, s_ll[4] = {0, 0, 0, 0};
      if (active) {
        const uint8_t* vh = &vbuf[sb][0][(8 * j + g) * KSTR + 4 * t];
        const uint8_t* vl = &vbuf[sb][1][(8 * j + g) * KSTR + 4 * t];
#pragma unroll
        for (int c = 0; c < KC; ++c) {
          const uint32_t bh0 = lds32b(vh + 32 * c), bl0 = lds32b(vl + 32 * c);
          const uint32_t bh1 = lds32b(vh + 32 * c + 16), bl1 = lds32b(vl + 32 * c + 16);
          bmma_ss(s_hh, ca_hi[c], bh0, bh1);
          bmma_su(s_mid, ca_hi[c], bl0, bl1);
          bmma_us(s_mid, ca_lo[c], bh0, bh1);
          bmma_uu(s_ll, ca_lo[c], bl0, bl1);
        }
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {  // row r0 (hf 0) or r1 (hf 1): C elements 2 hf, 2 hf + 1
        const int r = hf ? r1 : r0;
        const int key = kb + 8 * j + 2 * t;
        if (r >= S || key >= S) continue;  // S % 4 == 0: key + 1 < S as well
        int dp[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int i = 2 * hf + e;
          const int p = (int)(int16_t)(pw[hf][j] >> (16 * e));
          dp[e] = 0;
          if (key + e <= r) {
            // dP = sat(rhu(65536 hh + rm, 15)) with rm = 256 mid + ll (|rm| < 2^31 for
            // head_dim <= 64): 65536 hh is a multiple of 2^15, so the rounded shift is
            // 2 hh + ((rm + 2^14) >> 15), all in i32 (|hh| <= 2^20).
            const int rm = s_mid[i] * 256 + s_ll[i];
            dp[e] = sat16(2 * s_hh[i] + ((rm + 16384) >> 15));
            neg |= p < 0;
            wsum[hf] += (long long)(dp[e] * p);  // |dP P| <= 2^30
          }
        }
        const uint32_t pk = (uint32_t)(dp[0] & 0xFFFF) | ((uint32_t)dp[1] << 16);
        if constexpr (PL)
          ps[(g + 8 * hf) * PSTR + 4 * j + t] = pk;
        else
          *reinterpret_cast<uint32_t*>(dLbh + (long long)r * S + key) = pk;
      }
    }
    if constexpr (PL) {  // the dP pieces out as planes (pieces outside the matrix are skipped)
      __syncwarp();
      const uint4 u0 = reinterpret_cast<const uint4*>(pmine)[0], u1 = reinterpret_cast<const uint4*>(pmine)[1];
      const uint32_t wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      piece_st(kb, wv);
      __syncwarp();  // the next tile's P overwrites the staged tile
    }
    if (more) store_tile(sb ^ 1, pre);
    __syncthreads();
  }
  int wq[2];
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) wsum[hf] += __shfl_xor_sync(0xffffffffu, wsum[hf], o);
    wq[hf] = (int)rhu64(wsum[hf], 15);
  }
  if (neg) nsrl_flag(a.st, NSRL_FLAG_LINEAR_OVERFLOW);  // a negative probability: the reference rejects
  // pass 2: dL = sat(rhu(P (dP - wq) 22713, 30)) over the values this lane stored
  if (qw >= S) return;
  if constexpr (PL) {
    // wq of this lane's piece row (qw + l / 2) from the quad that reduced it
    const int rr = lane >> 1;
    const int w0 = __shfl_sync(0xffffffffu, wq[0], 4 * (rr & 7)), w1 = __shfl_sync(0xffffffffu, wq[1], 4 * (rr & 7));
    const int myw = rr >= 8 ? w1 : w0;
    for (int kt = 0; kt < ntiles; ++kt) {
      const int kb = kt * BK;
      if (pr >= S || kb + ph >= S || kb + ph > pr) continue;  // outside, or above the diagonal (zeros already)
      uint32_t pv[8], dv[8], ov[8];
      piece_ld(a.p_hi, a.p_lo, kb, pv);
      piece_ld(a.l_hi, a.l_lo, kb, dv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int dl[2];
#pragma unroll
        for (int z = 0; z < 2; ++z) {
          const int p = (int)(int16_t)(pv[e] >> (16 * z));
          const int dp = (int)(int16_t)(dv[e] >> (16 * z));
          const long long prod = (long long)(p * 22713) * (long long)(dp - myw);
          dl[z] = kb + ph + 2 * e + z <= pr ? sat16((int)((prod + (1ll << 29)) >> 30)) : 0;
        }
        ov[e] = (uint32_t)(dl[0] & 0xFFFF) | ((uint32_t)dl[1] << 16);
      }
      piece_st(kb, ov);
    }
    return;
  }
  for (int kt = 0; kt < ntiles; ++kt) {
    const int kb = kt * BK;
    uint32_t pw[2][4], dw[2][4];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = hf ? r1 : r0, key = kb + 8 * j + 2 * t;
        const bool in = r < S && key < S && key <= r;
        pw[hf][j] = in ? *reinterpret_cast<const uint32_t*>(Pbh + (long long)r * S + key) : 0u;
        dw[hf][j] = in ? *reinterpret_cast<const uint32_t*>(dLbh + (long long)r * S + key) : 0u;
      }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = hf ? r1 : r0, key = kb + 8 * j + 2 * t;
        if (r >= S || key >= S || key > r) continue;  // zeros already there
        int dl[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int p = (int)(int16_t)(pw[hf][j] >> (16 * e));
          const int dp = (int)(int16_t)(dw[hf][j] >> (16 * e));
          // P (dP - wq) 22713 = (22713 P) (dP - wq): |22713 P| < 2^30, |dP - wq| < 2^30
          const long long prod = (long long)(p * 22713) * (long long)(dp - wq[hf]);
          dl[e] = key + e <= r ? sat16((int)((prod + (1ll << 29)) >> 30)) : 0;
        }
        *reinterpret_cast<uint32_t*>(dLbh + (long long)r * S + key) = (uint32_t)(dl[0] & 0xFFFF) | ((uint32_t)dl[1] << 16);
      }
  }
}

struct DqArgs {
  const int8_t* kt_hi;  // K^T planes [B][H][HD][Sp], MMA key order per 32-key block
  const uint8_t* kt_lo;
  int Sp;
  const int16_t* dL;  // [BH][S][S]
  int S, H, shift;
  int16_t* dQ;
  long long ldo;
  GradPlanes gp;  // optional prescaled planes of dQ
};

// dQ[t] = sat(rhu(sum_{j <= t} dL[t][j] K[j], shift)): one CTA per 64 query
// rows; for head_dim 64, 8 warps, warp w owning rows 16 (w & 3) .. +15 and
// dims 32 (w >> 2) .. +31.  The A fragments come straight from the dL rows
// (two 4-byte key pairs per fragment register, matching the key order of the
// K^T planes), prefetched a tile ahead; K^T is staged 16 bytes at a time into
// double-buffered shared memory.
template <int HD>
__global__ void __launch_bounds__(HD == 64 ? 256 : 128, 2) attn_bwd_dq_kernel(const DqArgs a) {
  constexpr int WN = HD < 32 ? HD : 32;  // dims per warp
  constexpr int NT = WN / 8;
  constexpr int NTHREADS = 128 * (HD / WN);
  constexpr int VSTR = 48;
  constexpr int KW = HD * 2;  // 16-byte words of one K^T plane tile (HD dims x 32 slots)
  constexpr int PER = (2 * KW + NTHREADS - 1) / NTHREADS;
  __shared__ __align__(16) uint8_t kbuf[2][2][HD * VSTR];  // [stage][plane]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int q0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int S = a.S;
  const long long row0 = (long long)b * S;
  const int qw = q0 + (warp & 3) * 16;
  const int d0 = (warp >> 2) * WN;
  const int r0 = qw + g, r1 = r0 + 8;
  const long long ktb = ((long long)b * a.H + h) * HD * (long long)a.Sp;
  const int16_t* dLbh = a.dL + ((long long)b * a.H + h) * S * (long long)S;
  const int kend = min(S, q0 + BQ);
  const int ntiles = (kend + BK - 1) / BK;
  const int wlast = min(qw + 15, S - 1);

  // K^T tile kb -> stage sb with cp.async (no registers held across the MMAs)
  auto issue_tile = [&](int kb, int sb) {
#pragma unroll
    for (int z = 0; z < PER; ++z) {
      const int e = tid + z * NTHREADS;
      if (e < 2 * KW) {
        const int pl = e / KW, w = e % KW;
        const long long off = ktb + (long long)(w >> 1) * a.Sp + kb + 16 * (w & 1);
        cp_async16(smem_u32(&kbuf[sb][pl][(w >> 1) * VSTR + 16 * (w & 1)]), pl ? (const void*)(a.kt_lo + off)
                                                                               : (const void*)(a.kt_hi + off));
      }
    }
    cp_async_commit();
  };
  // fragment register i: row (i & 1 ? r1 : r0), key pairs kb + 2t + (i & 2 ? 16 : 0) and + 8
  auto load_dl = [&](int kb, uint32_t (&u)[4][2]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (i & 1) ? r1 : r0;
      const int key = kb + 2 * t + ((i & 2) ? 16 : 0);
#pragma unroll
      for (int z = 0; z < 2; ++z) {
        const int kk = key + 8 * z;
        u[i][z] = (r < S && kk < S) ? *reinterpret_cast<const uint32_t*>(dLbh + (long long)r * S + kk) : 0u;
      }
    }
  };

  int acc_hh[NT][4], acc_mid[NT][4], acc_ll[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc_hh[n][i] = acc_mid[n][i] = acc_ll[n][i] = 0;
  uint32_t du[4][2];
  issue_tile(0, 0);
  load_dl(0, du);
  for (int kt = 0; kt < ntiles; ++kt) {
    const int kb = kt * BK, sb = kt & 1;
    const bool more = kt + 1 < ntiles;
    uint32_t dn[4][2];
    if (more) {
      issue_tile(kb + BK, sb ^ 1);  // stage sb ^ 1 was last read before the previous barrier
      load_dl(kb + BK, dn);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // every thread's copies of stage sb have landed
    if (qw < S && kb <= wlast) {
      uint32_t ah[4], al[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {  // the hi / lo bytes of the four int16 values
        ah[i] = __byte_perm(du[i][0], du[i][1], 0x7531);
        al[i] = __byte_perm(du[i][0], du[i][1], 0x6420);
      }
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint8_t* kh = &kbuf[sb][0][(d0 + 8 * n + g) * VSTR + 4 * t];
        const uint8_t* kl = &kbuf[sb][1][(d0 + 8 * n + g) * VSTR + 4 * t];
        const uint32_t bh0 = lds32b(kh), bh1 = lds32b(kh + 16), bl0 = lds32b(kl), bl1 = lds32b(kl + 16);
        bmma_ss(acc_hh[n], ah, bh0, bh1);
        bmma_su(acc_mid[n], ah, bl0, bl1);
        bmma_us(acc_mid[n], al, bh0, bh1);
        bmma_uu(acc_ll[n], al, bl0, bl1);
      }
    }
    if (more) {
#pragma unroll
      for (int i = 0; i < 4; ++i) du[i][0] = dn[i][0], du[i][1] = dn[i][1];
    }
    __syncthreads();  // stage sb is read before the next iteration's copies reuse it
  }
  // the 64 x HD block goes through shared memory (the K^T buffers are free
  // after the last barrier), then out as 16-byte rows of dQ and 8-byte rows
  // of its prescaled planes
  constexpr int OSTR = HD + 8;
  static_assert(64 * OSTR * 2 <= (int)sizeof(kbuf), "dQ staging fits the K^T buffers");
  int16_t* so = reinterpret_cast<int16_t*>(&kbuf[0][0][0]);
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      int v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int i = 2 * hf + e;
        const long long tot = (long long)acc_hh[n][i] * 65536 + (long long)acc_mid[n][i] * 256 + (long long)acc_ll[n][i];
        v[e] = sat_i16(rhu64(tot, (uint32_t)a.shift));
      }
      const int lr = (warp & 3) * 16 + g + 8 * hf;
      *reinterpret_cast<uint32_t*>(&so[lr * OSTR + d0 + 8 * n + 2 * t]) = (uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16);
    }
  __syncthreads();
  for (int e = tid; e < 64 * (HD / 8); e += NTHREADS) {
    const int lr = e / (HD / 8), c8 = 8 * (e % (HD / 8));
    if (q0 + lr >= S) continue;
    const uint4 u = *reinterpret_cast<const uint4*>(&so[lr * OSTR + c8]);
    const long long off = (row0 + q0 + lr) * a.ldo + (long long)h * HD + c8;
    if (a.dQ) *reinterpret_cast<uint4*>(a.dQ + off) = u;
    if (a.gp.hi) {
      int v[8];
      unpack8(u, v);
#pragma unroll
      for (int z = 0; z < 8; ++z) v[z] = rhu_i16(v[z], a.gp.sc[h * HD + c8 + z].right_shift);
      uint2 ph, pl;
      planes8(v, ph, pl);
      *reinterpret_cast<uint2*>(a.gp.hi + off) = ph;
      *reinterpret_cast<uint2*>(a.gp.lo + off) = pl;
    }
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
  GradPlanes gp;  // optional prescaled planes of the output
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
      const int col = h * HD + 8 * n + 2 * t;
      if (a.out)
        *reinterpret_cast<uint32_t*>(a.out + (row0 + kr) * a.ldo + col) = (uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16);
      if (a.gp.hi) store_grad_planes2(a.gp, (row0 + kr) * a.ldo + col, col, v);
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
      const int col = h * HD + d0 + 8 * n + 2 * t;
      if (a.out)
        *reinterpret_cast<uint32_t*>(a.out + (row0 + kr) * a.ldo + col) = (uint32_t)(v[0] & 0xFFFF) | ((uint32_t)v[1] << 16);
      if (a.gp.hi) store_grad_planes2(a.gp, (row0 + kr) * a.ldo + col, col, v);
    }
}

cudaError_t launch_sq_transpose(const int16_t* M, size_t BH, size_t S, int8_t* th, uint8_t* tl, cudaStream_t s) {
  dim3 sg((unsigned)((S + 63) / 64), (unsigned)((S + 63) / 64), (unsigned)BH);
  if (S % 16 == 0)
    sq_transpose16_kernel<<<sg, 128, 0, s>>>(M, (int)S, th, tl);
  else
    sq_transpose_kernel<<<sg, 256, 0, s>>>(M, (int)S, th, tl);
  return cudaGetLastError();
}

}  // namespace

size_t attention_backward_tc_scratch_bytes(size_t B, size_t S, size_t d, size_t H) {
  const size_t Sp = (S + 31) & ~size_t(31);
  auto up = [](size_t b) { return (b + 255) & ~size_t(255); };
  // V planes [T][d], K^T (padded rows), Q^T, dC^T, P^T, dL^T: two planes each
  return 2 * (up(B * S * d) + up(B * d * Sp) + 2 * up(B * d * S) + 2 * up(B * H * S * S));
}

// dQ, dK, dV of causal attention on int16 operands (and dL into `dl`: every
// causal 64 x 64 tile written, the rest untouched; with `planes`, also the
// prescaled byte planes of dQ, dK, dV): q, k, v rows of stride ld,
// P [B][H][S][S], dC rows of stride ldc; outputs [B*S][d].  head_dim 16 or 64, S a multiple of 4, d a multiple of 16
// (else cudaErrorNotSupported).  scratch: attention_backward_tc_scratch_bytes.
cudaError_t launch_attention_backward_tc(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld,
                                         const int16_t* P, const int16_t* dC, size_t ldc, size_t B, size_t S, size_t d,
                                         size_t H, int16_t* dl, int16_t* dq, int16_t* dk, int16_t* dv,
                                         void* scratch, size_t scratch_bytes, nsrl_device_status* st,
                                         cudaStream_t s, const GradPlanes* planes, const Planes* p_planes,
                                         const Planes* qkv_planes) {
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
  cudaError_t e = cudaSuccess;
  const double pairs = (double)B * (double)H * (double)S * (double)(S + 1) / 2.0;
  if ((p_planes || qkv_planes) && !attention_kv_tc_supported(S, d, H)) return cudaErrorInvalidValue;
  if (attention_kv_tc_supported(S, d, H)) {
    // Tensor-core path (head_dim 64, S % 16 == 0): V, K, Q, dC as row-major
    // planes [B*S][d] (q|k|v as given, or split here), P (unless given as
    // planes) and dL as causal planes [B*H][S][S]; the dL kernel reads and
    // writes planes, one persistent tcgen05 kernel forms dK, dV and dQ.  The
    // K^T / Q^T / dC^T / P^T / dL^T scratch buffers hold these instead; the
    // int16 dl is not written.
    Planes qp{qth, qtl, nullptr, d}, kp{kth, ktl, nullptr, d}, vp{vph, vpl, nullptr, d};
    if (qkv_planes) {
      const Planes& a = *qkv_planes;
      qp = Planes{a.hi, a.lo, nullptr, a.ld};
      kp = Planes{a.hi + d, a.lo + d, nullptr, a.ld};
      vp = Planes{a.hi + 2 * d, a.lo + 2 * d, nullptr, a.ld};
    } else {
      e = launch_split_planes(v, B * S, d, ld, vp, s);
      if (e == cudaSuccess) e = launch_split_planes(k, B * S, d, ld, kp, s);
      if (e == cudaSuccess) e = launch_split_planes(q, B * S, d, ld, qp, s);
      if (e != cudaSuccess) return e;
    }
    e = launch_split_planes(dC, B * S, d, ldc, Planes{cth, ctl, nullptr, d}, s);
    if (e != cudaSuccess) return e;
    const Planes pp = p_planes ? *p_planes : Planes{pth, ptl, nullptr, S};
    if (!p_planes) {
      e = launch_split_causal(P, B * H, S, pth, ptl, s);
      if (e != cudaSuccess) return e;
    }
    e = launch_attention_bwd_dl_tc(Planes{cth, ctl, nullptr, d}, vp, pp, lth, ltl, B, S, d, H, st, s);
    if (e == cudaErrorNotSupported) {  // plane buffers the tensor maps cannot describe: the mma.sync kernel
      (void)cudaGetLastError();
      DlArgs la{dC, (long long)ldc, vp.hi, vp.lo, (int)vp.ld, nullptr, (int)S, (int)H, nullptr, st, pp.hi, pp.lo, lth, ltl};
      ProfScope prof("attention_bwd_dl", s, 2.0 * (double)hd * pairs,
                     2.0 * 2.0 * (double)B * H * S * S + 4.0 * (double)B * S * d);
      attn_bwd_dl_kernel<64, true><<<dim3((unsigned)((S + BQ - 1) / BQ), (unsigned)H, (unsigned)B), 128, 0, s>>>(la);
      e = cudaGetLastError();
    }
    if (e != cudaSuccess) return e;
    return launch_attention_kv_tc(Planes{lth, ltl, nullptr, S}, pp, qp, Planes{cth, ctl, nullptr, d}, B, S, d, H,
                                  planes ? nullptr : dk,
                                  planes ? nullptr : dv, planes ? planes[1] : GradPlanes{},
                                  planes ? planes[2] : GradPlanes{}, st, s, &kp, planes ? nullptr : dq,
                                  planes ? planes[0] : GradPlanes{});
  }
  {
    ProfScope prof("attention_bwd_planes", s, 0.0, 8.0 * (double)B * S * d + 2.0 * 2.0 * (double)B * H * S * S);
    e = launch_split_planes(v, B * S, d, ld, Planes{vph, vpl, nullptr, d}, s);
    if (e != cudaSuccess) return e;
    dim3 tg((unsigned)((S + 63) / 64), (unsigned)H, (unsigned)B);
    if (hd == 64 && S % 16 == 0 && ld % 8 == 0 && ldc % 8 == 0) {
      head_transpose16_kernel<<<tg, 128, 0, s>>>(k, (long long)ld, (int)S, (int)Sp, (int)H, true, kth, ktl);
      head_transpose16_kernel<<<tg, 128, 0, s>>>(q, (long long)ld, (int)S, (int)S, (int)H, false, qth, qtl);
      head_transpose16_kernel<<<tg, 128, 0, s>>>(dC, (long long)ldc, (int)S, (int)S, (int)H, false, cth, ctl);
    } else if (hd == 64) {
      head_transpose_kernel<64><<<tg, 256, 0, s>>>(k, (long long)ld, (int)S, (int)Sp, (int)H, true, kth, ktl);
      head_transpose_kernel<64><<<tg, 256, 0, s>>>(q, (long long)ld, (int)S, (int)S, (int)H, false, qth, qtl);
      head_transpose_kernel<64><<<tg, 256, 0, s>>>(dC, (long long)ldc, (int)S, (int)S, (int)H, false, cth, ctl);
    } else {
      head_transpose_kernel<16><<<tg, 256, 0, s>>>(k, (long long)ld, (int)S, (int)Sp, (int)H, true, kth, ktl);
      head_transpose_kernel<16><<<tg, 256, 0, s>>>(q, (long long)ld, (int)S, (int)S, (int)H, false, qth, qtl);
      head_transpose_kernel<16><<<tg, 256, 0, s>>>(dC, (long long)ldc, (int)S, (int)S, (int)H, false, cth, ctl);
    }
    e = launch_sq_transpose(P, B * H, S, pth, ptl, s);
    if (e != cudaSuccess) return e;
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  dim3 grid((unsigned)((S + BQ - 1) / BQ), (unsigned)H, (unsigned)B);
  {
    DlArgs la{dC, (long long)ldc, vph, vpl, (int)d, P, (int)S, (int)H, dl, st, nullptr, nullptr, nullptr, nullptr};
    ProfScope prof("attention_bwd_dl", s, 2.0 * (double)hd * pairs,
                   2.0 * 2.0 * (double)B * H * S * S + 4.0 * (double)B * S * d);
    if (hd == 64)
      attn_bwd_dl_kernel<64, false><<<grid, 128, 0, s>>>(la);
    else
      attn_bwd_dl_kernel<16, false><<<grid, 128, 0, s>>>(la);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  {
    // with plane outputs the int16 gradients are not written (nothing reads them)
    DqArgs qa{kth, ktl, (int)Sp, dl, (int)S, (int)H, shift, planes ? nullptr : dq, (long long)d,
              planes ? planes[0] : GradPlanes{}};
    ProfScope prof("attention_bwd_dq", s, 2.0 * (double)hd * pairs,
                   2.0 * (double)B * H * S * S + 4.0 * (double)B * S * d);
    if (hd == 64)
      attn_bwd_dq_kernel<64><<<grid, 256, 0, s>>>(qa);
    else
      attn_bwd_dq_kernel<16><<<grid, 128, 0, s>>>(qa);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  {
    ProfScope prof("attention_bwd_planes", s, 0.0, 4.0 * (double)B * H * S * S);
    e = launch_sq_transpose(dl, B * H, S, lth, ltl, s);
    if (e != cudaSuccess) return e;
  }
  KVArgs ka{lth, ltl, qth, qtl, (int)S, (int)H, shift, planes ? nullptr : dk, (long long)d,
            planes ? planes[1] : GradPlanes{}};
  KVArgs va{pth, ptl, cth, ctl, (int)S, (int)H, 15, planes ? nullptr : dv, (long long)d,
            planes ? planes[2] : GradPlanes{}};
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
