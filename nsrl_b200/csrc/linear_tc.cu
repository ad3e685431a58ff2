// i16 x i8 -> i16 per-channel linear on the B200 tensor cores (tcgen05, kind::i8).
//
// Reference: crates/nsrl-core/src/linear.rs:228-324.  y[m][n] =
// requantize_i32_to_i16(bias[n] + sum_k x[m][k] * W[n][k], scale[n]) with an
// i32 accumulator whose every prefix must fit (else the call is `None`).
//
// Exactness on int8 tensor cores: x is held as byte planes x = 256*hi + lo
// (hi signed, lo unsigned).  Two MMAs share the weight tile: hi x W (s8.s8)
// and lo x W (u8.s8), each into its own s32 TMEM accumulator; both partial
// sums are exact (|hi*w| <= 16256, |lo*w| <= 32385 per product).  The true
// sum 256*acc_hi + acc_lo + bias fits i32 whenever no i32 prefix of the
// reference's accumulation overflows, so the epilogue recombines it with
// wrapping i32 arithmetic (exact in that case).  A prefix can only overflow
// when |bias| + 127 * sum_k |x[m][k]| > i32::MAX; only then does
// prefix_check_kernel rescan those rows in reference order and reject the
// call (linear.rs:144-173, :282-296).
//
// Persistent kernel, one CTA per SM, 18 warps:
//   warp 0      TMA producer: A hi/lo planes + W tile per 128-wide K block,
//               through a 4-stage shared-memory ring
//   warp 1      TMEM allocator + MMA issuer (whole warp, one elected lane issues)
//   warps 2..17 epilogue: TMEM -> registers -> requant -> global; four
//               warps per TMEM lane quarter, 32 columns each (or, for the
//               gated form without caches, two sets of eight taking
//               alternate tiles, 64 columns each)
// The two accumulator pairs (hi, lo) of a 128 x 128 tile take 256 TMEM
// columns; two tiles are in flight (512 columns) so that the epilogue of
// tile i overlaps the MMAs of tile i+1.  Operand tiles are K-major with the
// 128-byte swizzle, one 128-byte row per tile row, as written by TMA.
#include <algorithm>
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int TILE_A = BM * BK;                   // one plane, 16 KB
constexpr int TILE_B = BN * BK;                   // 16 KB
constexpr int STAGE_BYTES = 2 * TILE_A + TILE_B;  // 48 KB
constexpr int STAGES = 4;
constexpr int ACC_COLS = 2 * BN;                  // acc_hi: [0,128), acc_lo: [128,256)
constexpr uint32_t TMEM_COLS = 2 * ACC_COLS;      // two tiles in flight
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 64 + 32 * EPI_WARPS;      // 576
// The int16-input form: four more warps turn each stage's int16 A tile into the
// two byte planes in place (see the converter below).
constexpr int CONV_WARPS = 4;
constexpr int threads_for(bool a16) { return THREADS + (a16 ? 32 * CONV_WARPS : 0); }
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + 1024 + 256;

struct TcMaps {
  CUtensorMap a_hi, a_lo, b[3];
};

// ---------------------------------------------------------------------------
// Exact i32 prefix check (linear.rs:282-296): for rows where
// |bias| + 127 * L1(x_row) can exceed i32::MAX, rescan every output in the
// reference's order (bias first, then k = 0, 1, ...) with checked adds.
// One warp per row; rows within the bound exit after one comparison.
// ---------------------------------------------------------------------------
struct CheckParams {
  const int8_t* a_hi;
  const uint8_t* a_lo;
  const int16_t* a16;  // int16 A instead of the planes (row stride lda elements)
  long long lda;
  const unsigned long long* l1;
  int M, K;
  int nseg;
  const int8_t* w[3];
  const int32_t* bias[3];
  int rows[3];
  nsrl_device_status* st;
};

constexpr int PREFIX_CHECK_THREADS = 256;

// Rescans row m of the linear in the reference's order (bias, then k = 0, 1,
// ...): any i32 prefix outside the range flags the call (linear.rs:282-296).
__device__ void prefix_rescan_row(const CheckParams& c, int m, int lane) {
  const int8_t* ah = c.a16 ? nullptr : c.a_hi + (long long)m * c.lda;
  const uint8_t* al = c.a16 ? nullptr : c.a_lo + (long long)m * c.lda;
  const int16_t* a16 = c.a16 ? c.a16 + (long long)m * c.lda : nullptr;
  for (int sg = 0; sg < c.nseg; ++sg) {
    for (int n = lane; n < c.rows[sg]; n += 32) {
      const int8_t* w = c.w[sg] + (long long)n * c.K;
      int acc = c.bias[sg] ? c.bias[sg][n] : 0;
      bool bad = false;
      for (int k = 0; k < c.K && !bad; ++k) {
        const int x = a16 ? (int)a16[k] : (int)ah[k] * 256 + (int)al[k];
        long long t = (long long)acc + (long long)(x * (int)w[k]);
        if (t < INT_MIN || t > INT_MAX) bad = true;
        acc = (int)t;
      }
      if (bad) nsrl_flag(c.st, NSRL_FLAG_LINEAR_OVERFLOW);
    }
  }
}

struct TcParams {
  int M, K, N;  // N = output columns (GATED: hidden channels)
  int nseg, seg_rows;
  int tiles_n, tiles;
  const int32_t* bias[3];
  const nsrl_fixed_scale* scales[3];
  int16_t* y;
  long long ldy;
  int16_t* y2;  // GATED: with y, the up (y) and gate (y2) values as int16
  int8_t* yh;
  uint8_t* yl;
  unsigned long long* yl1;
  long long ldp;
  const int16_t* skip;
  long long ldskip;
  unsigned long long* sat;
  int8_t* vth;
  uint8_t* vtl;
  int vt_S, vt_H, vt_hd, vt_col0;  // QKV_VT: output columns >= vt_col0 go to the transposed planes
  bool v_rows;                      // QKV_VT: and to the row-major planes as well
  QkvRoute route;                   // QKV_VT: head-sharded destinations (route.nranks > 0)
  bool small_acc;                   // K * 127 * 32767 < 2^30: every accumulator is below 2^30
  bool wide;                        // i64 accumulator, requantize_i64_to_i16 (backward-input linears)
  // The i32 prefix check, in the epilogue of each row block's first column
  // tile (planes input with the rows' L1 given): rows past the L1 bound are
  // rescanned there, one warp per row.
  bool fuse_check;
  CheckParams chk;
  nsrl_device_status* st;
};

// requantize_i32_to_i16 (numeric.rs:59-70) with the i32 fast paths of a
// multiplier of 1: rhu(acc, s) = (acc >> s) + bit (s - 1) of acc, s in 1..31.
__device__ __forceinline__ int requant_fast(int acc, int mult, uint32_t shift) {
  if (mult == 1) {
    if (shift == 0) return max(-32768, min(32767, acc));
    if (shift < 32) {
      const int r = (acc >> shift) + ((acc >> (shift - 1)) & 1);
      return max(-32768, min(32767, r));
    }
  }
  return (int)sat_i16(rhu64((long long)acc * (long long)mult, shift));
}

__device__ __forceinline__ int clamp16(int v) { return max(-32768, min(32767, v)); }

__device__ __forceinline__ uint32_t pack2(int a, int b) { return (uint32_t)(a & 0xFFFF) | ((uint32_t)b << 16); }

// Per-lane copy of the scale (and bias) of column `lane` of a chunk, plus a
// warp-uniform flag for the common case: every valid column has multiplier 1,
// one shared right shift and no bias.  Lanes past the valid columns hold an
// identity scale.
struct ColScale {
  int mult, shift, bias;
  int ushift;
  bool uniform;
};

__device__ __forceinline__ ColScale load_scales(const nsrl_fixed_scale* sc, const int32_t* bias, int n, bool valid) {
  ColScale c;
  c.mult = 1;
  c.shift = 0;
  c.bias = 0;
  if (valid) {
    const nsrl_fixed_scale s = sc[n];
    c.mult = s.multiplier;
    c.shift = s.right_shift;
    c.bias = bias ? bias[n] : 0;
  }
  c.ushift = __shfl_sync(0xffffffffu, c.shift, 0);
  c.uniform = __all_sync(0xffffffffu, !valid || (c.mult == 1 && c.shift == c.ushift && c.bias == 0)) != 0;
  return c;
}

// The scale of a segment whose every column has multiplier 1, one right
// shift and no bias (the reference's per-layer tables): no table reads.
__device__ __forceinline__ ColScale uniform_scale(int shift) {
  ColScale c;
  c.mult = 1;
  c.shift = shift;
  c.bias = 0;
  c.ushift = shift;
  c.uniform = true;
  return c;
}

// AND of v over the epilogue warps (named barrier 1, their threads only).
__device__ __forceinline__ bool epilogue_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(32 * EPI_WARPS)
      : "memory");
  return r != 0;
}

// requantize_i32_to_i16 of W columns: acc = 256*hi + lo (+ bias), wrapping
// u32 arithmetic (exact whenever the true i32 sum fits).
// `small`: |acc| < 2^30 (K * 127 * 32767 < 2^30, no bias), so acc + 2^(s-1)
// cannot overflow and rhu is one add and one shift.  Column i of the chunk
// takes the scale held by lane base + i.
template <int W>
__device__ __forceinline__ void requant_cols(const uint32_t (&h)[W], const uint32_t (&l)[W], const ColScale& c,
                                             int (&v)[W], bool small, int base = 0) {
  if (c.uniform) {
    const uint32_t s = (uint32_t)c.ushift;
    if (s == 0) {
#pragma unroll
      for (int i = 0; i < W; ++i) v[i] = clamp16((int)(h[i] * 256u + l[i]));
    } else if (s < 32 && small) {
      const int half = 1 << (s - 1);
#pragma unroll
      for (int i = 0; i < W; ++i) v[i] = clamp16(((int)(h[i] * 256u + l[i]) + half) >> s);
    } else if (s < 32) {
#pragma unroll
      for (int i = 0; i < W; ++i) {
        const int acc = (int)(h[i] * 256u + l[i]);
        v[i] = clamp16((acc >> s) + ((acc >> (s - 1)) & 1));
      }
    } else {
#pragma unroll
      for (int i = 0; i < W; ++i) v[i] = (int)sat_i16(rhu64((long long)(int)(h[i] * 256u + l[i]), s));
    }
  } else {
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const int mult = __shfl_sync(0xffffffffu, c.mult, base + i);
      const int shift = __shfl_sync(0xffffffffu, c.shift, base + i);
      const int b = __shfl_sync(0xffffffffu, c.bias, base + i);
      v[i] = requant_fast((int)(h[i] * 256u + l[i] + (uint32_t)b), mult, (uint32_t)shift);
    }
  }
}
// linear.rs:744-751 (requantize_i64_to_i16) of an i64 accumulator held as
// two exact s32 plane sums: acc = 256 * hi + lo.  A multiplier that takes the
// product out of i64 is the reference's `None` (flagged).
__device__ __forceinline__ int requant_wide1(uint32_t h, uint32_t l, int mult, int shift, bool& bad) {
  const long long acc = (long long)(int)h * 256ll + (long long)(int)l;
  long long wide = acc;
  if (mult != 1) {
    const long long lo = (long long)((unsigned long long)acc * (unsigned long long)(long long)mult);
    if (__mul64hi(acc, (long long)mult) != (lo >> 63)) bad = true;
    wide = lo;
  }
  return (int)sat_i16(rhu64(wide, (uint32_t)shift));
}
__device__ __forceinline__ void requant_wide16(const uint32_t (&h)[16], const uint32_t (&l)[16], const ColScale& c,
                                               int (&v)[16], bool& bad, int base) {
  if (c.uniform) {
    // multiplier 1 and one shift s for every column: |256 hi + lo| < 2^40, so
    // rhu64's saturating add cannot saturate; the sum is one wide
    // multiply-add and the rounded shift one 64-bit shift
    const uint32_t sh = min((uint32_t)c.ushift, 62u);
    const long long bias = sh ? (1ll << (sh - 1)) : 0ll;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const long long a = ((long long)(int)h[i] * 256ll + ((long long)(int)l[i] + bias)) >> sh;
      const int lo = (int)a, hi = (int)(a >> 32);
      v[i] = hi == (lo >> 31) ? max(-32768, min(32767, lo)) : (hi < 0 ? -32768 : 32767);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int mult = c.uniform ? 1 : __shfl_sync(0xffffffffu, c.mult, base + i);
    const int shift = c.uniform ? c.ushift : __shfl_sync(0xffffffffu, c.shift, base + i);
    v[i] = requant_wide1(h[i], l[i], mult, shift, bad);
  }
}
__device__ __forceinline__ void requant16(const uint32_t (&h)[16], const uint32_t (&l)[16], const ColScale& c,
                                          int (&v)[16], bool small) {
  requant_cols<16>(h, l, c, v, small);
}

// Splits 16 packed int16 values into hi / lo byte planes.
__device__ __forceinline__ void store16_planes_nol1(int8_t* dh, uint8_t* dl, const uint32_t (&o)[8], int nvalid,
                                                    bool vec_ok) {
  if (vec_ok && nvalid == 16) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      hw[i] = __byte_perm(o[2 * i], o[2 * i + 1], 0x7531);
      lw[i] = __byte_perm(o[2 * i], o[2 * i + 1], 0x6420);
    }
    *reinterpret_cast<uint4*>(dh) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(dl) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < nvalid) {
        const int v = (int16_t)(o[i / 2] >> (16 * (i & 1)));
        dh[i] = (int8_t)(v >> 8);
        dl[i] = (uint8_t)(v & 255);
      }
    }
  }
}

// Head-sharded Q|K|V stores.  Row m of this rank's projection is position
// rank * s_loc + (m % s_loc) of sequence m / s_loc; column c of segment seg
// (q, k, v) belongs to rank c / d_loc.  q and k go to that rank's planes
// [B*S][2 d_loc] (q at column 0, k at d_loc), v to its transposed planes
// [B][d_loc][S].  Sixteen columns starting at a multiple of 16 never cross
// a rank (d_loc is a multiple of the head dim, itself a multiple of 16).
__device__ __forceinline__ void qkv_route_store16(const TcParams& p, int m, int n, const int (&v)[16],
                                                  const uint32_t (&o)[8], int nv) {
  const QkvRoute& R = p.route;
  const int d = p.seg_rows;
  const int b = m / R.s_loc;
  const int pos = R.rank * R.s_loc + (m - b * R.s_loc);
  const int seg = n / d, c = n - seg * d;
  const int own = c / R.d_loc, cl = c - own * R.d_loc;
  if (seg < 2) {
    const long long ld = 2LL * R.d_loc;
    const long long col = (long long)seg * R.d_loc + cl;
    const long long off = ((long long)b * R.S + pos) * ld + col;
    store16_planes_nol1(R.tab->qk_hi[own] + off, R.tab->qk_lo[own] + off, o, nv, ((ld | col) & 15) == 0);
  } else {
    int8_t* vh = R.tab->vt_hi[own];
    uint8_t* vl = R.tab->vt_lo[own];
    const long long off0 = ((long long)b * R.d_loc + cl) * R.S + pos;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      if (i < nv) {
        const long long off = off0 + (long long)i * R.S;
        vh[off] = (int8_t)(v[i] >> 8);
        vl[off] = (uint8_t)(v[i] & 255);
      }
    }
  }
}

__device__ __forceinline__ void qkv_route_store1(const TcParams& p, int m, int n, int v) {
  const QkvRoute& R = p.route;
  const int d = p.seg_rows;
  const int b = m / R.s_loc;
  const int pos = R.rank * R.s_loc + (m - b * R.s_loc);
  const int seg = n / d, c = n - seg * d;
  const int own = c / R.d_loc, cl = c - own * R.d_loc;
  long long off;
  int8_t* h;
  uint8_t* l;
  if (seg < 2) {
    off = ((long long)b * R.S + pos) * (2LL * R.d_loc) + (long long)seg * R.d_loc + cl;
    h = R.tab->qk_hi[own];
    l = R.tab->qk_lo[own];
  } else {
    off = ((long long)b * R.d_loc + cl) * R.S + pos;
    h = R.tab->vt_hi[own];
    l = R.tab->vt_lo[own];
  }
  h[off] = (int8_t)(v >> 8);
  l[off] = (uint8_t)(v & 255);
}

// mlp.rs:150-170 on values already in [-32768, 32767] (int arguments, no
// conversions); the result lies within +-24575 (see gated_act).
__device__ __forceinline__ int gated_act_i32(int up, int gate) {
  const int gv = (gate >> 2) + 16384;
  const int silu = (gate * gv + 16384) >> 15;
  return (up * silu + 16384) >> 15;
}

__device__ __forceinline__ void store16_i16(int16_t* dst, const uint32_t (&o)[8], int nvalid, bool vec_ok) {
  if (vec_ok && nvalid == 16) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    d[0] = make_uint4(o[0], o[1], o[2], o[3]);
    d[1] = make_uint4(o[4], o[5], o[6], o[7]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (i < nvalid) dst[i] = (int16_t)(o[i / 2] >> (16 * (i & 1)));
  }
}

// 16 int16 columns (o: 8 packed words) at base + r * ld + col, as above.
__device__ __forceinline__ void store16_i16_pairs(int16_t* base, long long ld, int r, int M, int col,
                                                  const uint32_t (&o)[8], int lane) {
  store32b_pairs(reinterpret_cast<uint8_t*>(base + col), 2 * ld, r, M, o, lane);
}

// WIDE (= p.wide) is a template parameter so that each kernel holds only one
// requantisation form: a smaller epilogue for the instruction cache.
// A16: A is int16 [M][K] in global memory.  TMA loads each 128 x 128 int16
// tile into the stage (the 32 KB the two planes take); warps 2 + EPI_WARPS ..
// turn it in place into the hi and lo planes in the MMA's K-major
// 128-byte-swizzled layout, and only then hand the stage to the MMA.  The
// separate split pass over A disappears; the i32 prefix check, where K or a
// bias needs it, takes the rows' L1 from the int16 rows itself.
template <int EPI, bool WIDE, bool A16, int SETS>
__global__ void __launch_bounds__(threads_for(A16), 1)
    gemm_tc_kernel(const __grid_constant__ TcMaps maps, const TcParams p) {
  static_assert(SETS == 1 || SETS == 2, "one or two epilogue sets");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]: MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;   // [2]: epilogue -> MMA
  uint64_t* ready = acc_empty + 2;      // [STAGES]: converter -> MMA (A16)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(ready + STAGES);
  uint32_t* skip_flag = tslot + 1;

  __shared__ unsigned long long s_maxb;  // max |bias| of the fused prefix check
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) s_maxb = 0ull;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], EPI_WARPS / SETS);  // the epilogue warps that take buffer b's tiles
    }
    if (A16)
      for (int s = 0; s < STAGES; ++s) mbar_init(&ready[s], CONV_WARPS);
    fence_barrier_init();
    prefetch_tmap(&maps.a_hi);
    prefetch_tmap(&maps.a_lo);
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  // The prologue above touches no global memory: from here on the previous
  // kernel's outputs (and the status it may have flagged) are visible.
  griddep_wait();
  if (threadIdx.x == 0) *skip_flag = timed_out(p.st) ? 1u : 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  const uint32_t tmem = *tslot;
  if (*skip_flag) {  // a wait of this call already timed out: do nothing
    if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
    return;
  }
  const int nkb = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;  // global k-block counter over all tiles of this CTA
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.tiles_n) * BM, nt = t % p.tiles_n;
        int seg = 0, brow = nt * BN;
        if (EPI == (int)Epi::GATED) {
          brow = nt * (BN / 2);
        } else if (p.nseg == 3) {
          seg = (nt * BN) / p.seg_rows;
          brow = (nt * BN) % p.seg_rows;
        }
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (it >= STAGES && !mbar_wait(&empty[s], ph ^ 1, p.st)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          uint8_t* sa = smem + s * STAGE_BYTES;
          if (A16) {  // the int16 tile [128 rows][128 k] (32 KB) where the planes will be
            tma_load_2d(sa, &maps.a_hi, &full[s], kb * BK, m0);
          } else {
            tma_load_2d(sa, &maps.a_hi, &full[s], kb * BK, m0);
            tma_load_2d(sa + TILE_A, &maps.a_lo, &full[s], kb * BK, m0);
          }
          if (EPI == (int)Epi::GATED) {
            tma_load_2d(sa + 2 * TILE_A, &maps.b[0], &full[s], kb * BK, brow);
            tma_load_2d(sa + 2 * TILE_A + TILE_B / 2, &maps.b[1], &full[s], kb * BK, brow);
          } else {
            tma_load_2d(sa + 2 * TILE_A, &maps.b[seg], &full[s], kb * BK, brow);
          }
        }
      }
      // Drain: the last loads in flight must land before the CTA exits.
      for (uint32_t j = (it > STAGES ? it - STAGES : 0); j < it; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, p.st);
    }
  } else if (warp == 1) {
    {  // the whole warp runs the loop (warp-uniform operands), one elected lane issues
      const uint32_t id_hi = idesc_i8(BM, BN, 1, 1);  // s8 x s8
      const uint32_t id_lo = idesc_i8(BM, BN, 0, 1);  // u8 x s8
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++local) {
        const uint32_t buf = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait(&acc_empty[buf], (use - 1) & 1, p.st)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * ACC_COLS;
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(A16 ? &ready[s] : &full[s], ph, p.st)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
          for (int j = 0; j < BK / 32; ++j) {
            // int16 input: the converter interleaves the planes atom by atom
            const uint64_t ah = A16 ? sdesc_k128_sbo(base + 32 * j, 2048) : sdesc_k128(base + 32 * j);
            const uint64_t al = A16 ? sdesc_k128_sbo(base + 1024 + 32 * j, 2048) : sdesc_k128(base + TILE_A + 32 * j);
            const uint64_t bd = sdesc_k128(base + 2 * TILE_A + 32 * j);
            const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
            umma_i8_warp(d, ah, bd, id_hi, acc);
            umma_i8_warp(d + BN, al, bd, id_lo, acc);
          }
          umma_commit_warp(&empty[s]);
        }
        umma_commit_warp(&acc_full[buf]);
      }
    }
  } else if (A16 && warp >= 2 + EPI_WARPS) {
    // --------------------------------------------------------- converter
    // The int16 tile is [128 rows][256 bytes]; its 8-row group g (2 KB at
    // 2048 g) becomes, in place, the hi plane's 8-row swizzle atom g (the
    // first 1 KB) and the lo plane's (the second): the MMA reads both planes
    // with 2048-byte atom strides.  A group's bytes hold only that group's
    // rows before and after, so each warp converts its own four groups (rows
    // 32 cw .. +31) with no barrier but its own: all eight rows are read
    // before any is written.  Each lane reads 16 bytes (8 int16) of a
    // row pair (a warp reads 512 bytes at once) and writes its 8 bytes of
    // each plane row at the chunk's swizzled place (chunk ^ (row & 7)).
    const int cw = warp - (2 + EPI_WARPS);
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        if (!mbar_wait(&full[s], (it / STAGES) & 1, p.st)) {
          ok = false;
          break;
        }
        uint8_t* sa = smem + s * STAGE_BYTES;
        // lane l: row (l >> 4) of each row pair, int16 elements 8 (l & 15) ..
        // +7, i.e. plane bytes 8 (l & 15) .. +7 = half (l & 1) of 16-byte
        // chunk (l & 15) >> 1
        const uint32_t hr = (uint32_t)lane >> 4, ch = ((uint32_t)lane & 15u) >> 1, hb = ((uint32_t)lane & 1u) * 8u;
#pragma unroll
        for (int grp = 0; grp < 4; ++grp) {
          uint8_t* gb = sa + 2048 * (4 * cw + grp);
          uint4 raw[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) raw[q] = *reinterpret_cast<const uint4*>(gb + 512 * q + lane * 16);
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t r = 2u * (uint32_t)q + hr;  // row within the 8-row group
            const uint32_t off = r * 128u + ((ch ^ r) << 4) + hb;
            *reinterpret_cast<uint2*>(gb + off) =
                make_uint2(__byte_perm(raw[q].x, raw[q].y, 0x7531), __byte_perm(raw[q].z, raw[q].w, 0x7531));
            *reinterpret_cast<uint2*>(gb + 1024 + off) =
                make_uint2(__byte_perm(raw[q].x, raw[q].y, 0x6420), __byte_perm(raw[q].z, raw[q].w, 0x6420));
          }
        }
        fence_proxy_async_smem();  // the planes, written by the threads, are read by the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(&ready[s]);
      }
    }
  } else {
    // Epilogue: warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32).  With one
    // set (SETS = 1) all sixteen warps take every tile, warp w column group
    // cg = (w-2)/4: columns [32*cg, 32*cg+32), or for the gated form up
    // channels [16*cg, +16) with their gate channels.  With two sets, eight
    // warps each take alternate tiles (set s the tiles of accumulator buffer
    // s), so that one set's accumulator loads and their latency overlap the
    // other set's arithmetic; warp w then owns column groups 2 cgs and
    // 2 cgs + 1, cgs = ((w-2)/4) % 2.  Two sets hold more registers live and
    // pay off where the epilogue has the fewest stores (the gated form
    // without its int16 caches).
    const int q = warp & 3;
    const int set = SETS == 2 ? (warp - 2) >> 3 : 0;
    const int cg0 = SETS == 2 ? 2 * (((warp - 2) >> 2) & 1) : (warp - 2) >> 2;
    uint32_t local = (uint32_t)set;
    unsigned long long sat = 0;
    // Every segment's scales uniform (multiplier 1, one shift, no bias)?  Then
    // the tiles take that shift and read no table: checked once per CTA by the
    // epilogue warps, each column by one thread.
    int ush0 = 0, ush1 = 0, ush2 = 0;
    bool uni = true;
    for (int sg = 0; sg < p.nseg; ++sg) {
      const nsrl_fixed_scale s0 = p.scales[sg][0];
      bool ok = p.bias[sg] == nullptr && s0.multiplier == 1;
      for (int i = (int)threadIdx.x - 64; i < p.seg_rows && ok; i += 32 * EPI_WARPS) {
        const nsrl_fixed_scale si = p.scales[sg][i];
        ok = si.multiplier == 1 && si.right_shift == s0.right_shift;
      }
      uni = uni && ok;
      if (sg == 0) ush0 = s0.right_shift;
      if (sg == 1) ush1 = s0.right_shift;
      if (sg == 2) ush2 = s0.right_shift;
    }
    if (p.fuse_check) {  // max |bias| over every segment, for the rows' prefix bound
      long long mb = 0;
      for (int sg = 0; sg < p.chk.nseg; ++sg)
        if (p.chk.bias[sg])
          for (int i = (int)threadIdx.x - 64; i < p.chk.rows[sg]; i += 32 * EPI_WARPS)
            mb = max(mb, llabs((long long)p.chk.bias[sg][i]));
      if (mb) atomicMax(&s_maxb, (unsigned long long)mb);
    }
    uni = epilogue_all(uni);  // a barrier of the epilogue warps: the maximum above is complete
    const long long maxb = (long long)s_maxb;
    for (int t = blockIdx.x + set * (int)gridDim.x; t < p.tiles; t += SETS * (int)gridDim.x, local += SETS) {
      const uint32_t buf = local & 1, use = local >> 1;
      const int m0 = (t / p.tiles_n) * BM, nt = t % p.tiles_n;
      const int r = m0 + q * 32 + lane;
      const bool row_ok = r < p.M;
      const uint32_t lrow = tmem + buf * ACC_COLS + ((uint32_t)(q * 32) << 16);
      unsigned long long l1 = 0;
      bool stop = false;  // a wait of this call timed out
#pragma unroll 1
      for (int sub = 0; sub < SETS; ++sub) {  // the warp's column groups of the tile
        const int cg = cg0 + sub;
        if (EPI == (int)Epi::GATED) {
          const int fb = nt * (BN / 2) + 16 * cg;
          const int nvalid = max(0, min(16, p.N - fb));
          const ColScale su =
              uni ? uniform_scale(ush0) : load_scales(p.scales[0], p.bias[0], fb + (lane & 15), (lane & 15) < nvalid);
          const ColScale sg =
              uni ? uniform_scale(ush1) : load_scales(p.scales[1], p.bias[1], fb + (lane & 15), (lane & 15) < nvalid);
          uint32_t hu[16], lu[16], hg[16], lg[16];
          if (sub == 0 && !mbar_wait(&acc_full[buf], use & 1, p.st)) {
            stop = true;
            break;
          }
          tc_fence_after();
          tmem_ld16(lrow + 16 * cg, hu);
          tmem_ld16(lrow + BN + 16 * cg, lu);
          tmem_ld16(lrow + 64 + 16 * cg, hg);
          tmem_ld16(lrow + BN + 64 + 16 * cg, lg);
          tmem_wait_ld();
          tc_fence_before();
          if (sub == SETS - 1 && lane == 0) mbar_arrive(&acc_empty[buf]);  // every group loaded
          int up[16], gt[16];
          requant16(hu, lu, su, up, p.small_acc);
          requant16(hg, lg, sg, gt, p.small_acc);
          // the up and gate values themselves (the training step's caches)
          const bool vok = ((p.ldy | fb) & 7) == 0;
          if (p.y && nvalid == 16 && vok) {  // whole 32-byte runs per store (lane pairs)
            uint32_t ou[8], og[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              ou[i] = __byte_perm((uint32_t)up[2 * i], (uint32_t)up[2 * i + 1], 0x5410);
              og[i] = __byte_perm((uint32_t)gt[2 * i], (uint32_t)gt[2 * i + 1], 0x5410);
            }
            store16_i16_pairs(p.y, p.ldy, r, p.M, fb, ou, lane);
            store16_i16_pairs(p.y2, p.ldy, r, p.M, fb, og, lane);
          } else if (p.y && row_ok && nvalid > 0) {
            uint32_t ou[8], og[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              ou[i] = __byte_perm((uint32_t)up[2 * i], (uint32_t)up[2 * i + 1], 0x5410);
              og[i] = __byte_perm((uint32_t)gt[2 * i], (uint32_t)gt[2 * i + 1], 0x5410);
            }
            store16_i16(p.y + (long long)r * p.ldy + fb, ou, nvalid, vok);
            store16_i16(p.y2 + (long long)r * p.ldy + fb, og, nvalid, vok);
          }
          int act[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) act[i] = gated_act_i32(up[i], gt[i]);
          unsigned a1 = 0;
          if (nvalid == 16) {
#pragma unroll
            for (int i = 0; i < 16; ++i) a1 += (unsigned)abs(act[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) a1 += (i < nvalid) ? (unsigned)abs(act[i]) : 0u;
          }
          uint32_t o[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = __byte_perm((uint32_t)act[2 * i], (uint32_t)act[2 * i + 1], 0x5410);
          if (row_ok && nvalid > 0) {
            const long long off = (long long)r * p.ldp + fb;
            l1 += a1;
            store16_planes_nol1(p.yh + off, p.yl + off, o, nvalid, ((p.ldp | fb) & 15) == 0);
          }
        } else {
          const int nb = nt * BN;
          const int sseg = (p.nseg == 3) ? nb / p.seg_rows : 0;
          const int nloc = ((p.nseg == 3) ? nb % p.seg_rows : nb) + 32 * cg;
          const int n = nb + 32 * cg;
          const int nvalid = max(0, min(32, p.N - n));
          const ColScale sc = uni ? uniform_scale(sseg == 0 ? ush0 : sseg == 1 ? ush1 : ush2)
                                  : load_scales(p.scales[sseg], p.bias[sseg], nloc + lane, lane < nvalid);
          // The residual rows do not depend on the accumulator: fetch them first.
          uint32_t s16[16];
          const bool vec_skip = EPI == (int)Epi::RESID && ((p.ldskip | p.ldy | n) & 7) == 0 && nvalid == 32;  // both halves full
          if (EPI == (int)Epi::RESID && row_ok && nvalid > 0) {
            const int16_t* sk = p.skip + (long long)r * p.ldskip + n;
            if (vec_skip) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint4 v = reinterpret_cast<const uint4*>(sk)[i];
                s16[4 * i] = v.x;
                s16[4 * i + 1] = v.y;
                s16[4 * i + 2] = v.z;
                s16[4 * i + 3] = v.w;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int a = (2 * i < nvalid) ? (int)sk[2 * i] : 0;
                const int b = (2 * i + 1 < nvalid) ? (int)sk[2 * i + 1] : 0;
                s16[i] = pack2(a, b);
              }
            }
          }
          if (sub == 0 && !mbar_wait(&acc_full[buf], use & 1, p.st)) {
            stop = true;
            break;
          }
          tc_fence_after();
          // All 32 columns come out of TMEM at once and the buffer is released
          // before any arithmetic, so the next tile's MMAs overlap this
          // epilogue; the columns are then finished in two halves of 16.  The
          // residual form, which also holds the skip rows, and the int16-input
          // form, which has fewer registers per thread, load and release half
          // by half.
          constexpr bool kOnce = EPI != (int)Epi::RESID && !A16;
          uint32_t hq[2][16], lq[2][16];
          if (kOnce) {
            tmem_ld16(lrow + 32 * cg, hq[0]);
            tmem_ld16(lrow + BN + 32 * cg, lq[0]);
            tmem_ld16(lrow + 32 * cg + 16, hq[1]);
            tmem_ld16(lrow + BN + 32 * cg + 16, lq[1]);
            tmem_wait_ld();
            tc_fence_before();
            if (sub == SETS - 1 && lane == 0) mbar_arrive(&acc_empty[buf]);  // every group loaded
          }
          uint32_t ph0[4], pl0[4];  // planes: the first half's bytes, held for the paired stores
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            if (!kOnce) {
              tmem_ld16(lrow + 32 * cg + 16 * hf, hq[hf]);
              tmem_ld16(lrow + BN + 32 * cg + 16 * hf, lq[hf]);
              tmem_wait_ld();
              if (hf == 1 && sub == SETS - 1) {  // every group loaded
                tc_fence_before();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
              }
            }
            const uint32_t(&h)[16] = hq[hf];
            const uint32_t(&l)[16] = lq[hf];
            const int nv = max(0, min(16, nvalid - 16 * hf));
            const int nh = n + 16 * hf;
            int v[16];
            if (WIDE) {
              bool bad = false;
              requant_wide16(h, l, sc, v, bad, 16 * hf);
              if (bad && row_ok && nv > 0) nsrl_flag(p.st, NSRL_FLAG_LINEAR_OVERFLOW);
            } else {
              requant_cols<16>(h, l, sc, v, p.small_acc, 16 * hf);
            }
            // int16 outputs of whole 16-column runs go out as lane pairs
            // (every lane takes part, valid row or not).  Not in the wide
            // form (it spills with the swap and measured slower) nor the
            // residual one (bound by its skip-row loads; no gain).
            const bool pairs = !WIDE && (EPI == (int)Epi::I16 || (EPI == (int)Epi::QKV_VT && p.y && !p.route.nranks)) &&
                               nv == 16 && ((p.ldy | nh) & 7) == 0;
            // planes: a lane's 32 columns are one 32-byte run per plane; the
            // first half waits in registers for the second, then both go out
            // as lane pairs
            const bool ppairs = !WIDE && EPI == (int)Epi::PLANES && nvalid == 32 && ((p.ldp | n) & 15) == 0;
            if (ppairs) {
              uint32_t hw[4], lw[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const uint32_t a = __byte_perm((uint32_t)v[4 * i], (uint32_t)v[4 * i + 1], 0x5410);
                const uint32_t b = __byte_perm((uint32_t)v[4 * i + 2], (uint32_t)v[4 * i + 3], 0x5410);
                hw[i] = __byte_perm(a, b, 0x7531);
                lw[i] = __byte_perm(a, b, 0x6420);
              }
              if (p.yl1 && row_ok) {
#pragma unroll
                for (int i = 0; i < 16; ++i) l1 += (unsigned)abs(v[i]);
              }
              if (hf == 0) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  ph0[i] = hw[i];
                  pl0[i] = lw[i];
                }
                continue;
              }
              const uint32_t hi8[8] = {ph0[0], ph0[1], ph0[2], ph0[3], hw[0], hw[1], hw[2], hw[3]};
              const uint32_t lo8[8] = {pl0[0], pl0[1], pl0[2], pl0[3], lw[0], lw[1], lw[2], lw[3]};
              store32b_pairs(reinterpret_cast<uint8_t*>(p.yh + n), p.ldp, r, p.M, hi8, lane);
              store32b_pairs(p.yl + n, p.ldp, r, p.M, lo8, lane);
              continue;
            }
            if (!pairs && (!row_ok || nv == 0)) continue;
            uint32_t o[8];
            if (EPI == (int)Epi::RESID) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const uint32_t sk = s16[8 * hf + i];
                const int a = (int)(int16_t)(sk & 0xFFFF) + v[2 * i];
                const int b = (int)(int16_t)(sk >> 16) + v[2 * i + 1];
                const int sa = clamp16(a), sb = clamp16(b);
                if (2 * i < nv && sa != a) ++sat;
                if (2 * i + 1 < nv && sb != b) ++sat;
                o[i] = __byte_perm((uint32_t)sa, (uint32_t)sb, 0x5410);
              }
              store16_i16(p.y + (long long)r * p.ldy + nh, o, nv, vec_skip);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] = __byte_perm((uint32_t)v[2 * i], (uint32_t)v[2 * i + 1], 0x5410);
              if (EPI == (int)Epi::QKV_VT && p.route.nranks) {
                qkv_route_store16(p, r, nh, v, o, nv);
                continue;
              }
              if (EPI == (int)Epi::I16 || (EPI == (int)Epi::QKV_VT && p.y)) {  // QKV_VT: the training step's int16 cache
                if (pairs)
                  store16_i16_pairs(p.y, p.ldy, r, p.M, nh, o, lane);
                else
                  store16_i16(p.y + (long long)r * p.ldy + nh, o, nv, ((p.ldy | nh) & 7) == 0);
              }
              if (EPI == (int)Epi::I16 || !row_ok) continue;
              if (EPI == (int)Epi::QKV_VT && nh >= p.vt_col0) {
                // v columns: byte stores into [b][h][dim][s]; the 32 lanes of the
                // warp hold 32 consecutive positions, so each store instruction
                // writes one contiguous 32-byte run per plane.  [b][h][dim][s] is
                // contiguous over (h, dim): row (b, c) of the planes is
                // b * H * hd + c for value column c.
                const int b = r / p.vt_S, spos = r % p.vt_S;
                const long long off0 = ((long long)b * (p.vt_H * p.vt_hd) + (nh - p.vt_col0)) * p.vt_S + spos;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  if (i < nv) {
                    const long long off = off0 + (long long)i * p.vt_S;
                    p.vth[off] = (int8_t)(v[i] >> 8);
                    p.vtl[off] = (uint8_t)(v[i] & 255);
                  }
                }
              }
              if (EPI != (int)Epi::QKV_VT || nh < p.vt_col0 || p.v_rows) {
                if (p.yl1) {
#pragma unroll
                  for (int i = 0; i < 16; ++i) l1 += (i < nv) ? (unsigned)abs(v[i]) : 0u;
                }
                const long long off = (long long)r * p.ldp + nh;
                store16_planes_nol1(p.yh + off, p.yl + off, o, nv, ((p.ldp | nh) & 15) == 0);
              }
            }
          }
        }
      }
      if (stop) break;
      if ((EPI == (int)Epi::PLANES || EPI == (int)Epi::GATED) && p.yl1 && row_ok && l1) atomicAdd(&p.yl1[r], l1);
      if (p.fuse_check && nt == 0 && cg0 == 0) {
        // The row block's prefix check, once (its first column tile): rows
        // whose |bias| + 127 L1 bound passes i32::MAX are rescanned in the
        // reference's order by the whole warp (rare).
        const bool bad = row_ok && 127ll * (long long)p.chk.l1[r] + maxb > (long long)INT_MAX;
        for (unsigned m = __ballot_sync(0xffffffffu, bad); m; m &= m - 1)
          prefix_rescan_row(p.chk, m0 + q * 32 + (__ffs(m) - 1), lane);
      }
    }
    if (EPI == (int)Epi::RESID) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sat += __shfl_xor_sync(0xffffffffu, sat, o);
      if (lane == 0 && sat) atomicAdd(p.sat, sat);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// SIMT fallback for shapes the TMA path cannot take (K or strides not a
// multiple of 16 bytes, tiny problems).  One thread per output element.
// ---------------------------------------------------------------------------
struct SimtParams {
  const int8_t* a_hi;
  const uint8_t* a_lo;
  long long lda;
  int M, K, N, nseg, seg_rows, epi;
  const int8_t* w[3];
  TcParams tp;
};

__device__ __forceinline__ int16_t finish1(int hi, int lo, const int32_t* bias, const nsrl_fixed_scale* sc, int n) {
  const int acc = (int)((uint32_t)hi * 256u + (uint32_t)lo + (bias ? (uint32_t)bias[n] : 0u));
  const nsrl_fixed_scale s = sc[n];
  return (int16_t)requant_fast(acc, s.multiplier, s.right_shift);
}

__device__ __forceinline__ void simt_dot(const SimtParams& s, int m, int sg, int nl, int& hi, int& lo) {
  const int8_t* ah = s.a_hi + (long long)m * s.lda;
  const uint8_t* al = s.a_lo + (long long)m * s.lda;
  const int8_t* w = s.w[sg] + (long long)nl * s.K;
  int h = 0, l = 0;
  for (int k = 0; k < s.K; ++k) {
    h += (int)ah[k] * (int)w[k];
    l += (int)al[k] * (int)w[k];
  }
  hi = h;
  lo = l;
}

__global__ void gemm_simt_kernel(const SimtParams s) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)s.M * s.N) return;
  const int m = (int)(idx / s.N), n = (int)(idx % s.N);
  const TcParams& p = s.tp;
  int16_t v;
  if (s.epi == (int)Epi::GATED) {
    int h, l;
    simt_dot(s, m, 0, n, h, l);
    int16_t up = finish1(h, l, p.bias[0], p.scales[0], n);
    simt_dot(s, m, 1, n, h, l);
    int16_t g = finish1(h, l, p.bias[1], p.scales[1], n);
    if (p.y) {
      p.y[(long long)m * p.ldy + n] = up;
      p.y2[(long long)m * p.ldy + n] = g;
    }
    v = gated_act(up, g);
  } else {
    const int sg = s.nseg == 3 ? n / s.seg_rows : 0;
    const int nl = s.nseg == 3 ? n % s.seg_rows : n;
    int h, l;
    simt_dot(s, m, sg, nl, h, l);
    if (p.wide) {
      bool bad = false;
      const nsrl_fixed_scale sc = p.scales[sg][nl];
      v = (int16_t)requant_wide1((uint32_t)h, (uint32_t)l, sc.multiplier, sc.right_shift, bad);
      if (bad) nsrl_flag(p.st, NSRL_FLAG_LINEAR_OVERFLOW);
    } else {
      v = finish1(h, l, p.bias[sg], p.scales[sg], nl);
    }
  }
  if (s.epi == (int)Epi::QKV_VT && p.route.nranks) {
    qkv_route_store1(p, m, n, v);
    return;
  }
  if (s.epi == (int)Epi::I16) {
    p.y[(long long)m * p.ldy + n] = v;
  } else if (s.epi == (int)Epi::RESID) {
    int w = (int)p.skip[(long long)m * p.ldskip + n] + (int)v;
    if (w < -32768 || w > 32767) atomicAdd(p.sat, 1ull);
    p.y[(long long)m * p.ldy + n] = sat_i16_i32(w);
  } else if (s.epi == (int)Epi::QKV_VT && n >= p.vt_col0) {
    if (p.y) p.y[(long long)m * p.ldy + n] = v;
    const int b = m / p.vt_S, spos = m % p.vt_S, c = n - p.vt_col0;
    const long long off = ((long long)(b * p.vt_H + c / p.vt_hd) * p.vt_hd + c % p.vt_hd) * p.vt_S + spos;
    p.vth[off] = (int8_t)(v >> 8);
    p.vtl[off] = (uint8_t)(v & 255);
    if (p.v_rows) {
      p.yh[(long long)m * p.ldp + n] = (int8_t)(v >> 8);
      p.yl[(long long)m * p.ldp + n] = (uint8_t)(v & 255);
    }
  } else {
    if (s.epi == (int)Epi::QKV_VT && p.y) p.y[(long long)m * p.ldy + n] = v;
    p.yh[(long long)m * p.ldp + n] = (int8_t)(v >> 8);
    p.yl[(long long)m * p.ldp + n] = (uint8_t)(v & 255);
    if (p.yl1) atomicAdd(&p.yl1[m], (unsigned long long)abs((int)v));
  }
}

// A row can overflow an i32 prefix only if |bias| + 127 * sum |x| > i32::MAX.
// One thread per row tests that bound; the rows outside it (rare) are queued
// in shared memory and rescanned exactly, one warp per row.
__global__ void __launch_bounds__(PREFIX_CHECK_THREADS) prefix_check_kernel(const CheckParams c) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  __shared__ long long s_maxb;
  __shared__ int s_rows[PREFIX_CHECK_THREADS];
  __shared__ unsigned long long s_l1[PREFIX_CHECK_THREADS];  // int16 rows: their L1, computed here
  __shared__ int s_n;
  if (threadIdx.x == 0) s_maxb = 0;
  __syncthreads();
  long long mb = 0;
  for (int sg = 0; sg < c.nseg; ++sg)
    if (c.bias[sg])
      for (int i = threadIdx.x; i < c.rows[sg]; i += blockDim.x) mb = max(mb, llabs((long long)c.bias[sg][i]));
  atomicMax(reinterpret_cast<unsigned long long*>(&s_maxb), (unsigned long long)mb);
  __syncthreads();
  const long long maxb = s_maxb;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int base = blockIdx.x * PREFIX_CHECK_THREADS; base < c.M; base += gridDim.x * PREFIX_CHECK_THREADS) {
    if (threadIdx.x == 0) s_n = 0;
    __syncthreads();
    const int m = base + (int)threadIdx.x;
    if (c.a16) {
      // int16 rows: each warp sums |x| of 32 rows, one 512-byte stretch of a row per step
      for (int j = 0; j < 32; ++j) {
        const int mr = base + (threadIdx.x >> 5) * 32 + j;
        unsigned long long sum = 0;
        if (mr < c.M) {
          const int16_t* xr = c.a16 + (long long)mr * c.lda;
          for (int k = lane * 8; k < c.K; k += 256) {
            const uint4 v = *reinterpret_cast<const uint4*>(xr + k);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) sum += (unsigned)(abs((int)(int16_t)(w[q] & 0xFFFFu)) + abs((int)w[q] >> 16));
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == j) s_l1[threadIdx.x] = sum;
      }
      __syncwarp();
    }
    const unsigned long long l1m = c.a16 ? s_l1[threadIdx.x] : (m < c.M ? c.l1[m] : 0ull);
    if (m < c.M && 127ll * (long long)l1m + maxb > (long long)INT_MAX) s_rows[atomicAdd(&s_n, 1)] = m;
    __syncthreads();
    const int nq = s_n;
    for (int qi = threadIdx.x >> 5; qi < nq; qi += warps) prefix_rescan_row(c, s_rows[qi], lane);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Split / join between int16 rows and byte planes.
// ---------------------------------------------------------------------------
__global__ void split_planes_kernel(const int16_t* x, long long rows, int K, long long ldx, int8_t* hi, uint8_t* lo,
                                    unsigned long long* l1, long long ldp) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long long r = (long long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long long)gridDim.x * warps) {
    const int16_t* xr = x + r * ldx;
    unsigned long long s = 0;
    for (int k = lane; k < K; k += 32) {
      int v = xr[k];
      hi[r * ldp + k] = (int8_t)(v >> 8);
      lo[r * ldp + k] = (uint8_t)(v & 255);
      s += (unsigned long long)abs(v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0 && l1) l1[r] = s;
  }
}

// Vectorised split for K % 8 == 0 and 16-byte aligned rows: 8 elements per thread-step.
__global__ void split_planes_vec_kernel(const int16_t* x, long long rows, int K, long long ldx, int8_t* hi,
                                        uint8_t* lo, unsigned long long* l1, long long ldp) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long long r = (long long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long long)gridDim.x * warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + r * ldx);
    unsigned long long s = 0;
    for (int k8 = lane; k8 < K / 8; k8 += 32) {
      uint4 v = xr[k8];
      const int16_t* e = reinterpret_cast<const int16_t*>(&v);
      uint32_t h0 = 0, h1 = 0, l0 = 0, l1w = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        h0 |= (uint32_t)((e[j] >> 8) & 255) << (8 * j);
        l0 |= (uint32_t)(e[j] & 255) << (8 * j);
        h1 |= (uint32_t)((e[4 + j] >> 8) & 255) << (8 * j);
        l1w |= (uint32_t)(e[4 + j] & 255) << (8 * j);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s += (unsigned long long)abs((int)e[j]);
      reinterpret_cast<uint2*>(hi + r * ldp)[k8] = make_uint2(h0, h1);
      reinterpret_cast<uint2*>(lo + r * ldp)[k8] = make_uint2(l0, l1w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0 && l1) l1[r] = s;
  }
}

__global__ void join_planes_kernel(const int8_t* hi, const uint8_t* lo, long long ldp, long long rows, int cols,
                                   int16_t* y, long long ldy) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  const long long n = rows * cols;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    long long r = i / cols;
    int c = (int)(i % cols);
    y[r * ldy + c] = (int16_t)((int)hi[r * ldp + c] * 256 + (int)lo[r * ldp + c]);
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D uint8 tensor map [rows][inner] with row stride `ld` bytes, box
// [box_rows][128 bytes], 128-byte swizzle, zero fill out of bounds.
// int16 [rows][inner] (row stride ld bytes), box [box_rows][BK elements], no
// swizzle: the int16-input form's A tiles, rows of 256 bytes in shared memory.
bool make_map16(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {(cuuint32_t)BK, box_rows};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int EPI, bool WIDE, bool A16 = false, int SETS = 1>
cudaError_t launch_tc(const TcMaps& maps, const TcParams& p, int grid, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<EPI, WIDE, A16, SETS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const cudaError_t e =
      launch_pdl(gemm_tc_kernel<EPI, WIDE, A16, SETS>, dim3(grid), dim3(threads_for(A16)), SMEM_BYTES, stream, maps, p);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_tc_epi(Epi epi, const TcMaps& maps, const TcParams& p, int grid, cudaStream_t stream) {
  switch (epi) {
    case Epi::I16:
      return p.wide ? launch_tc<(int)Epi::I16, true>(maps, p, grid, stream)
                    : launch_tc<(int)Epi::I16, false, false, 2>(maps, p, grid, stream);
    case Epi::PLANES:
      return p.wide ? launch_tc<(int)Epi::PLANES, true>(maps, p, grid, stream)
                    : launch_tc<(int)Epi::PLANES, false>(maps, p, grid, stream);
    case Epi::RESID:
      return p.wide ? launch_tc<(int)Epi::RESID, true>(maps, p, grid, stream)
                    : launch_tc<(int)Epi::RESID, false, false, 2>(maps, p, grid, stream);
    case Epi::GATED:  // the wide form takes neither of these (launch_gemm rejects it)
      // without the int16 caches (inference) the gated epilogue takes two sets
      return p.y ? launch_tc<(int)Epi::GATED, false>(maps, p, grid, stream)
                 : launch_tc<(int)Epi::GATED, false, false, 2>(maps, p, grid, stream);
    case Epi::QKV_VT:
      return launch_tc<(int)Epi::QKV_VT, false>(maps, p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool tma_supported() { return encode_fn() != nullptr; }

// The prefix check's view of a linear (its A, weights, biases and rows' L1).
static CheckParams check_params(const GemmArgs& a) {
  CheckParams c{};
  c.a_hi = a.a_hi;
  c.a_lo = a.a_lo;
  c.a16 = a.a16;
  c.lda = (long long)a.lda;
  c.l1 = a.a_l1;
  c.M = (int)a.M;
  c.K = (int)a.K;
  c.nseg = a.nseg;
  for (int i = 0; i < a.nseg; ++i) {
    c.w[i] = a.seg[i].w;
    c.bias[i] = a.seg[i].bias;
    c.rows[i] = (int)a.seg[i].rows;
  }
  c.st = a.st;
  return c;
}

cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  const bool gated = a.epi == Epi::GATED;
  int N = 0;
  if (gated)
    N = (int)a.seg[0].rows;
  else
    for (int i = 0; i < a.nseg; ++i) N += (int)a.seg[i].rows;
  if (a.M == 0 || N == 0) return cudaSuccess;

  TcParams p{};
  p.M = (int)a.M;
  p.K = (int)a.K;
  p.N = N;
  p.nseg = a.nseg;
  p.seg_rows = (int)a.seg[0].rows;
  for (int i = 0; i < a.nseg; ++i) {
    p.bias[i] = a.seg[i].bias;
    p.scales[i] = a.seg[i].scales;
  }
  p.y = a.y;
  p.ldy = (long long)a.ldy;
  p.y2 = a.y2;
  p.yh = a.yp.hi;
  p.yl = a.yp.lo;
  p.yl1 = a.yp.l1;
  p.ldp = (long long)a.yp.ld;
  p.skip = a.skip;
  p.ldskip = (long long)a.ldskip;
  p.sat = a.sat_counter;
  p.vth = a.vt.hi;
  p.vtl = a.vt.lo;
  p.vt_S = a.vt.S;
  p.vt_H = a.vt.H;
  p.vt_hd = a.vt.hd;
  p.vt_col0 = a.epi == Epi::QKV_VT ? 2 * (int)a.seg[0].rows : INT_MAX;
  p.v_rows = a.v_rows;
  p.route = a.route;
  if (a.route.nranks && (a.epi != Epi::QKV_VT || a.nseg != 3 || a.route.tab == nullptr || a.route.s_loc <= 0 ||
                         a.route.d_loc <= 0 || a.route.d_loc % 16 != 0 || a.M % (size_t)a.route.s_loc != 0))
    return cudaErrorInvalidValue;
  p.small_acc = (unsigned long long)a.K * 127ull * 32767ull < (1ull << 30);
  p.wide = a.wide;
  p.st = a.st;
  const bool a16 = a.a16 != nullptr;
  const bool need_check = [&] {
    bool b = false;
    for (int i = 0; i < a.nseg; ++i) b = b || a.seg[i].bias != nullptr;
    return !a.wide && (b || (unsigned long long)a.K * 127ull * 32767ull > 2147483647ull);
  }();
  // int16 A: only the plain int16 epilogue, on the tensor-core path (the
  // caller splits A into planes itself otherwise)
  if (a16 && (a.epi != Epi::I16 || a.wide || a.nseg != 1 || !tma_supported() || (a.K % 8) != 0 ||
              ((a.lda * 2) % 16) != 0 || !aligned16(a.a16)))
    return cudaErrorInvalidValue;

  // The wide form keeps each plane's s32 sum exact: K * 255 * 127 < 2^31.
  if (a.wide && (a.K > 66000 || gated || a.epi == Epi::QKV_VT || a.nseg != 1)) return cudaErrorInvalidValue;

  bool tc = a16 || (tma_supported() && (a.K % 16) == 0 && (a.lda % 16) == 0 && aligned16(a.a_hi) && aligned16(a.a_lo));
  for (int i = 0; i < a.nseg; ++i) tc = tc && aligned16(a.seg[i].w);
  if (a.nseg == 3 && (a.seg[0].rows % BN) != 0) tc = false;
  if (a.nseg == 3 && (a.seg[1].rows != a.seg[0].rows || a.seg[2].rows != a.seg[0].rows)) tc = false;

  const double Mx = (double)a.M, Kx = (double)a.K, Nx = (double)N;
  const double nw = gated ? 2.0 * Nx : Nx;  // weight rows read
  double out_bytes = 2.0 * Mx * Nx;
  if (a.epi == Epi::RESID) out_bytes *= 2.0;  // skip read + output write
  if (a.epi == Epi::PLANES || a.epi == Epi::GATED) out_bytes += a.yp.l1 ? 8.0 * Mx : 0.0;
  static const char* names[2][5] = {
      {"linear_simt_i16", "linear_simt_planes", "linear_simt_resid", "linear_simt_gated", "linear_simt_qkv"},
      {"linear_tc_i16", "linear_tc_planes", "linear_tc_resid", "linear_tc_gated", "linear_tc_qkv"}};
  cudaError_t err = cudaSuccess;
  if (tc) {
    TcMaps maps;
    bool ok = a16 ? make_map16(&maps.a_hi, a.a16, a.K, a.M, a.lda * 2, BM)
                  : make_map(&maps.a_hi, a.a_hi, a.K, a.M, a.lda, BM) && make_map(&maps.a_lo, a.a_lo, a.K, a.M, a.lda, BM);
    if (a16) maps.a_lo = maps.a_hi;  // unused
    const uint32_t brows = gated ? BN / 2 : BN;
    for (int i = 0; i < a.nseg && ok; ++i) ok = make_map(&maps.b[i], a.seg[i].w, a.K, a.seg[i].rows, a.K, brows);
    for (int i = a.nseg; i < 3; ++i) maps.b[i] = maps.b[0];
    if (!ok) {
      if (a16) return cudaErrorInvalidValue;
      tc = false;
    } else {
      // planes input with the rows' L1: the prefix check runs in the GEMM's epilogue
      p.fuse_check = need_check && !a16 && a.a_l1 != nullptr;
      if (p.fuse_check) p.chk = check_params(a);
      p.tiles_n = gated ? (N + BN / 2 - 1) / (BN / 2) : (N + BN - 1) / BN;
      p.tiles = p.tiles_n * (int)((a.M + BM - 1) / BM);
      const int grid = std::min(p.tiles, sm_count());
      ProfScope prof(names[1][(int)a.epi], stream, 2.0 * Mx * nw * Kx, 2.0 * Mx * Kx + nw * Kx + out_bytes);
      err = a16 ? launch_tc<(int)Epi::I16, false, true>(maps, p, grid, stream)
                : launch_tc_epi(a.epi, maps, p, grid, stream);
    }
  }
  if (!tc) {
    SimtParams s{};
    s.a_hi = a.a_hi;
    s.a_lo = a.a_lo;
    s.lda = (long long)a.lda;
    s.M = (int)a.M;
    s.K = (int)a.K;
    s.N = N;
    s.nseg = a.nseg;
    s.seg_rows = (int)a.seg[0].rows;
    s.epi = (int)a.epi;
    for (int i = 0; i < a.nseg; ++i) s.w[i] = a.seg[i].w;
    s.tp = p;
    const long long total = (long long)a.M * N;
    ProfScope prof(names[0][(int)a.epi], stream, 2.0 * Mx * nw * Kx, 2.0 * Mx * Kx + nw * Kx + out_bytes);
    gemm_simt_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(s);
    err = cudaGetLastError();
  }
  if (err != cudaSuccess) return err;

  // The i32 prefix can only overflow when |bias| + K * 127 * 32767 > i32::MAX
  // (linear.rs:144-173); then rows outside the L1 bound are rescanned.
  if (need_check && !(tc && p.fuse_check)) {
    if (!a.a_l1) return cudaErrorInvalidValue;
    const CheckParams c = check_params(a);
    const unsigned blocks =
        (unsigned)std::min<size_t>((a.M + PREFIX_CHECK_THREADS - 1) / PREFIX_CHECK_THREADS, 148 * 8);
    ProfScope prof("linear_prefix_check", stream, 0.0, 8.0 * Mx);
    err = launch_pdl(prefix_check_kernel, dim3(blocks), dim3(PREFIX_CHECK_THREADS), 0, stream, c);
    if (err == cudaSuccess) err = cudaGetLastError();
  }
  return err;
}

cudaError_t launch_split_planes(const int16_t* x, size_t rows, size_t K, size_t ldx, Planes out, cudaStream_t stream) {
  if (rows == 0 || K == 0) return cudaSuccess;
  unsigned blocks = (unsigned)std::min<size_t>((rows + 7) / 8, 148 * 16);
  ProfScope prof("split_planes", stream, 0.0, 4.0 * rows * K + 8.0 * rows);
  const bool vec = K % 8 == 0 && ldx % 8 == 0 && out.ld % 8 == 0 && aligned16(x) &&
                   (reinterpret_cast<uintptr_t>(out.hi) & 7) == 0 && (reinterpret_cast<uintptr_t>(out.lo) & 7) == 0;
  const cudaError_t e = launch_pdl(vec ? split_planes_vec_kernel : split_planes_kernel, dim3(blocks), dim3(256), 0,
                                   stream, x, (long long)rows, (int)K, (long long)ldx, out.hi, out.lo, out.l1,
                                   (long long)out.ld);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_join_planes(Planes in, size_t rows, size_t cols, int16_t* y, size_t ldy, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  long long n = (long long)rows * cols;
  unsigned blocks = (unsigned)std::min<long long>((n + 255) / 256, 148 * 32);
  ProfScope prof("join_planes", stream, 0.0, 4.0 * (double)n);
  const cudaError_t e = launch_pdl(join_planes_kernel, dim3(blocks), dim3(256), 0, stream, (const int8_t*)in.hi,
                                   (const uint8_t*)in.lo, (long long)in.ld, (long long)rows, (int)cols, y, (long long)ldy);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace nsrl
