// Integer causal self-attention on the B200 tensor cores (tcgen05, kind::i8),
// head_dim 64, or 16 for the forward alone (Q and K rows padded to the MMA's
// 32-byte K step, logit shift 2).
//
// Reference: crates/nsrl-core/src/attention.rs:742-877 (full attention),
// :261-293 (base-2 softmax), :117-140 (QK dot), :596-668 (AV).
//
// One CTA per (128-query tile, head, pair of sequences): two independent
// groups of 10 warps, one per sequence, so that the row exchanges, the
// first-tile latency and the tail of one group overlap the steady state of the
// other.  The warps of a group:
//   warp 0     TMA producer: Q planes once, then per 32-key tile the K planes
//              (max and sum passes) or the transposed V planes (last pass)
//   warp 1     TMEM allocator + MMA issuer (the whole warp runs the loop, one elected lane issues)
//   warps 2..9 softmax: warp w owns query rows 32*(w%4) .. +31 (its TMEM lane
//              quarter) and keys [16*g, 16*g+16) of each 32-key tile,
//              g = (w-2)/4
// q.k = 65536*(qh.kh) + 256*(qh.kl + ql.kh) + ql.kl: each S tile (128 x 32)
// is three s32 TMEM accumulators (hh, mid, ll) that the softmax warps
// recombine, in exact 32-bit arithmetic where a guard proves it exact and in
// i64 otherwise.  The probabilities are rounded to Q15 with the reciprocal of
// the complete row sum before the AV product (attention.rs:285-290), so the
// keys are swept three times: row max, row sum (whose weights go to a global
// scratch), then P = sat(rhu(w * inv, 16)) and O = P V.  P is written to
// shared memory as byte planes (ph <= 127, pl) in the MMA's K-major layout;
// O = P V uses three more s32 accumulators (65536*hh + 256*mid + ll), exact
// for up to 16384 keys.
//
// TMEM (256 columns per group): two S buffers of 3 x 32 columns at [0, 96) and
// [96, 192) in the max and sum passes; O hh/mid/ll (3 x 64 columns) at
// [0, 192) in the last pass, which reads no S.
// Q and K tiles use the 64-byte swizzle (rows of 64 bytes), P and V^T tiles
// the 32-byte swizzle (rows of 32 bytes), as TMA writes them.
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int QT = 128, KT = 32, HD = 64;  // HD: the largest head dim (it sizes the shared-memory layout)
constexpr int ST = 4;                 // K / V^T stage ring
constexpr int PLANE_Q = QT * HD;      // 8 KB per plane
constexpr int PLANE_K = KT * HD;      // 2 KB: 32 keys x 64 dims
constexpr int PLANE_V = HD * KT;      // 2 KB: 64 dims x 32 keys
static_assert(PLANE_K == PLANE_V, "a stage holds either K or V^T planes");
constexpr int STAGE_BYTES = 2 * PLANE_K;
constexpr int PLANE_P = QT * KT;      // 4 KB
constexpr int SOFTMAX_WARPS = 8;
constexpr int GROUP_WARPS = 2 + SOFTMAX_WARPS;          // producer, MMA issuer, softmax warps
constexpr int GROUPS = 2;
constexpr int GROUP_THREADS = 32 * GROUP_WARPS;
constexpr int THREADS = GROUPS * GROUP_THREADS;
constexpr uint32_t TMEM_COLS = 512;                     // 256 per group
constexpr uint32_t S_HH = 0, S_MID = 32, S_LL = 64, S_BUF1 = 96;
constexpr uint32_t O_HH = 0, O_MID = 64, O_LL = 128;
// Bound on |256 * mid + ll| of one 64-dim dot product: |mid| <= 64 * 2 * 128 * 255,
// 0 <= ll <= 64 * 255 * 255 (a 16-dim product stays below it too).
constexpr long long B_MID = 64LL * 2 * 128 * 255 * 256 + 64LL * 255 * 255;

// Per head dim (64 or 16): Q and K rows in shared memory are ROW bytes (16
// dims are padded to the MMA's 32-byte K step: Q's upper 16 bytes are zeroed,
// so whatever K holds there adds nothing), the logit shift is
// log2(sqrt(head_dim)) (attention.rs:77-87), and the transfer sizes.
template <int HDIM>
struct HeadDim {
  static constexpr int ROW = HDIM < 32 ? 32 : HDIM;
  static constexpr int SH = HDIM == 64 ? 3 : 2;
  static constexpr int PQ = QT * ROW, PK = KT * ROW, PV = HDIM * KT;
  static_assert(HDIM == 64 || HDIM == 16, "head dims 64 and 16");
};

constexpr int OFF_Q = 0;
constexpr int OFF_STAGE = OFF_Q + 2 * PLANE_Q;
constexpr int OFF_P = OFF_STAGE + ST * STAGE_BYTES;
constexpr int OFF_X = OFF_P + 2 * 2 * PLANE_P;  // row-statistics exchange: max, min, sum of [2][QT]
constexpr int X_BYTES = 2 * QT * 8 * 3;
constexpr int OFF_LUT = OFF_X + X_BYTES;
constexpr int WPF_BUF = QT * KT * 2;  // weights of one tile: [128 rows][32 keys] int16, 64-byte swizzle
constexpr int WPF_N = 4;              // last-pass weight ring slots (the sum pass stages its stores in 3 of them)
constexpr int OFF_WPF = OFF_LUT + 512;
constexpr int OFF_BAR = OFF_WPF + WPF_N * WPF_BUF;
constexpr int GROUP_BYTES = (OFF_BAR + 256 + 1023) / 1024 * 1024;  // one group's region (offsets above are within it)
constexpr size_t SMEM_BYTES = (size_t)GROUPS * GROUP_BYTES + 1024;

struct Maps {
  CUtensorMap q_hi, q_lo, k_hi, k_lo, vt_hi, vt_lo;  // q: 128-row boxes, k: 32-row boxes, vt: 64 x 32-byte boxes
  CUtensorMap p_hi, p_lo;  // P planes [B*H][S][S], 128 x 32-byte boxes (stores of the cached P)
  CUtensorMap w;           // weight scratch as bytes [rows][2 wstride], 128 x 64-byte boxes (last-pass loads)
  CUtensorMap ws;          // the same, 32 x 32-byte boxes: one softmax warp's weights of a tile (sum-pass stores)
  CUtensorMap v_hi, v_lo;  // V rows [T][d] (the q|k|v planes' V columns), 32 keys x 64-byte boxes (vrow)
};

struct Args {
  int S, d, H, causal, b0, nb;  // sequences [b0, b0 + nb) in this launch (batch chunks)
  int16_t* wscr;     // per-CTA scratch of the sum pass's weights w, [128 rows][wstride]
  long long wstride; // S rounded up to a multiple of 64
  int8_t* ctx_hi;
  uint8_t* ctx_lo;
  unsigned long long* ctx_l1;
  long long ldc;
  int16_t* probs;    // optional P [B][H][S][S]: the visited key tiles only, zeros above the diagonal
  int pstore;        // write P as byte planes [B][H][S][S] (the same entries) through maps.p_hi / p_lo
  CtxRoute rt;       // head-sharded context destinations (rt.nranks > 0)
  int vrow;          // head dim 64: the last pass reads V as row-major planes (an MN-major B operand)
  nsrl_device_status* st;
};

// Shared-memory descriptor, K-major, 64-byte swizzle: 8-row atoms of 512 B.
__device__ __forceinline__ uint64_t sdesc_k64(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}
// Shared-memory descriptor of an MN-major tile of 64-byte rows (64 dims of
// one key per row), 64-byte swizzle, 8-row groups 512 bytes apart: V rows as
// the B operand of P V without a transposed copy.
__device__ __forceinline__ uint64_t sdesc_mn64(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}
// Shared-memory descriptor, K-major, 32-byte swizzle: 8-row atoms of 256 B.
__device__ __forceinline__ uint64_t sdesc_k32(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(256 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)6 << 61);
}

// Byte offset of 16-byte chunk c (0..1) of row r in a 32-byte-swizzled tile
// (address bit 4 ^= bit 7).
__device__ __forceinline__ uint32_t swz32_chunk(uint32_t r, uint32_t c) { return r * 32u + ((c ^ ((r >> 2) & 1u)) << 4); }

struct Ctl {
  uint64_t q_full, full[ST], empty[ST], s_full[2], s_empty[2], p_full[2], p_empty[2], o_full;
  uint64_t w_ready, w_full[WPF_N], w_empty[WPF_N];  // the weight scratch written / its last-pass tile ring
  uint64_t q_ready;  // head dim 16: Q's padding zeroed by the softmax warps
  uint32_t tslot, abort;
};
static_assert(sizeof(Ctl) <= 256, "barrier area");

__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, Ctl* c, nsrl_device_status* st) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*reinterpret_cast<volatile uint32_t*>(&c->abort)) return false;
  if (mbar_wait(bar, parity, st)) return true;
  *reinterpret_cast<volatile uint32_t*>(&c->abort) = 1u;
  return false;
}

// Barrier of one group's softmax warps (ids 1 and 2; 0 is __syncthreads).
__device__ __forceinline__ void named_sync_softmax(int grp) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + grp), "n"(32 * SOFTMAX_WARPS));
}

// Pass-0 update of one warp's 16 scores.  raw = 65536*hh + 256*mid + ll is an
// exact i32 when |hh| <= 16384 (|256*mid + ll| <= B_MID < 2^30); then the
// logit raw >> 3 is inside i32 too and only the max matters.  Larger |hh|
// take the i64 path, which also keeps the min for the i32 range check.
template <bool FULL>
__device__ __forceinline__ void scores_max(const uint32_t (&hh)[16], const uint32_t (&mid)[16],
                                           const uint32_t (&ll)[16], int nlive, int& mx32, long long& mx64,
                                           long long& mn64) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if (FULL || i < nlive) {
      const int h = (int)hh[i];
      if ((unsigned)(h + 16384) <= 32768u) {
        mx32 = max(mx32, (int)((uint32_t)h * 65536u + mid[i] * 256u + ll[i]));
      } else {
        const long long raw = (long long)h * 65536 + (long long)(int)mid[i] * 256 + (long long)(int)ll[i];
        mx64 = max(mx64, raw);
        mn64 = min(mn64, raw);
      }
    }
  }
}

// Base-2 weights w = LUT(lg - lgmax) (attention.rs:142-158) of 16 scores.  w
// != 0 needs mag = lgmax - lg < 3840, i.e. raw > rawmax - (3840 << SH); that
// needs hh > hh_floor, and then rawmax - raw < 2^32 is exact in u32, with
// mag = (diff + cround) >> SH (SH = 3 for head dim 64: the logit is raw >> 3).
template <bool FULL, int SH>
__device__ __forceinline__ void scores_weight(const uint32_t (&hh)[16], const uint32_t (&mid)[16],
                                              const uint32_t (&ll)[16], int nlive, int hh_floor, uint32_t rawmax_lo,
                                              uint32_t cround, const int16_t* lut, int (&w)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    int wi = 0;
    if ((FULL || i < nlive) && (int)hh[i] > hh_floor) {
      const uint32_t diff = rawmax_lo - (hh[i] * 65536u + mid[i] * 256u + ll[i]);
      if (diff < (3840u << SH) - cround) {
        const uint32_t mag = (diff + cround) >> SH;
        wi = (int)lut[mag & 255u] >> (mag >> 8);
      }
    }
    w[i] = wi;
  }
}

constexpr uint32_t FULLMASK = 0xffffffffu;

// The exp2 table replicated once per lane, s_lutr[32 * f + lane] =
// EXP2_NEG_FRAC_LUT_8BIT[f] (attention.rs:142-158): lane i reads bank i only,
// so the random table lookups of a warp never conflict.  A static shared
// array, so its address is a constant of the load instruction; 16-byte
// aligned for the vector stores that fill it.
__shared__ __align__(16) uint32_t s_lutr[256 * 32];

// x >> s for every s; amounts of 32 or more give 0 (PTX shr clamps them).
__device__ __forceinline__ uint32_t shr_clamp(uint32_t x, uint32_t s) {
  uint32_t r;
  asm("shr.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(s));
  return r;
}

__device__ __forceinline__ int max3i(int a, int b, int c) { return __vimax3_s32(a, b, c); }
__device__ __forceinline__ int min3i(int a, int b, int c) { return __vimin3_s32(a, b, c); }
__device__ __forceinline__ int max16(const int (&v)[16]) {
  const int a = max3i(v[0], v[1], v[2]), b = max3i(v[3], v[4], v[5]), c = max3i(v[6], v[7], v[8]);
  const int d = max3i(v[9], v[10], v[11]), e = max3i(v[12], v[13], v[14]);
  return max(max3i(a, b, c), max3i(d, e, v[15]));
}
__device__ __forceinline__ int min16(const int (&v)[16]) {
  const int a = min3i(v[0], v[1], v[2]), b = min3i(v[3], v[4], v[5]), c = min3i(v[6], v[7], v[8]);
  const int d = min3i(v[9], v[10], v[11]), e = min3i(v[12], v[13], v[14]);
  return min(min3i(a, b, c), min3i(d, e, v[15]));
}

// Pass 0 on one S tile of a warp (32 rows x 16 keys).  When every hh of the
// warp's tile lies in [-16384, 16384], raw = 65536*hh + 256*mid + ll is an
// exact i32 (|raw| <= 2^30 + B_MID < 2^31) and wrapping 32-bit arithmetic
// gives it; the guard looks at all 16 elements, live or not, so a masked
// element can only send the tile to the per-element path, never change a
// result.
template <bool FULL>
__device__ __forceinline__ void tile_max(const uint32_t (&hh)[16], const uint32_t (&mid)[16],
                                         const uint32_t (&ll)[16], int nlive, int& mx32, long long& mx64,
                                         long long& mn64) {
  int hv[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) hv[i] = (int)hh[i];
  const int hmax = max16(hv), hmin = min16(hv);
  if (__all_sync(FULLMASK, hmax <= 16384 && hmin >= -16384)) {
    int r[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int raw = (int)(hh[i] * 65536u + mid[i] * 256u + ll[i]);
      r[i] = (FULL || i < nlive) ? raw : INT_MIN;
    }
    mx32 = max(mx32, max16(r));
  } else {
    scores_max<FULL>(hh, mid, ll, nlive, mx32, mx64, mn64);
  }
}

// Pass 0 on one S tile of a warp whose rows all have L1(q_hi) <= 128, so
// |hh| <= 128 * 128 and every raw value is an exact i32 without a range check.
template <bool FULL>
__device__ __forceinline__ void tile_max_bounded(const uint32_t (&hh)[16], const uint32_t (&mid)[16],
                                                 const uint32_t (&ll)[16], int nlive, int& mx32) {
  int r[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int raw = (int)(hh[i] * 65536u + mid[i] * 256u + ll[i]);
    r[i] = (FULL || i < nlive) ? raw : INT_MIN;
  }
  mx32 = max(mx32, max16(r));
}

// Per 16-bit half min of two packed unsigned pairs.
__device__ __forceinline__ uint32_t min_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// Sum of the absolute values of the 16 signed bytes of v.
__device__ __forceinline__ uint32_t abs_sum16(const uint4 v) {
  uint32_t s = __dp4a(__vabs4(v.x), 0x01010101u, 0u);  // __vabs4(-128) = 0x80: 128 as a byte sum term
  s = __dp4a(__vabs4(v.y), 0x01010101u, s);
  s = __dp4a(__vabs4(v.z), 0x01010101u, s);
  return __dp4a(__vabs4(v.w), 0x01010101u, s);
}

// Pass-1 weights of a warp whose 32 rows all have exact i32 raw values
// (|raw| <= 2^30 + B_MID).  With C = rawmax + cround (mod 2^32),
// t = C - raw = (rawmax - raw) + cround < 2^32 exactly, mag = lgmax - lg =
// t >> SH, and w = LUT[mag & 255] >> (mag >> 8) = lutr[(t >> SH) & 255] >> (t >> (SH + 8)):
// t >= 3840 << SH (mag >= 3840) shifts by 15 or more and gives 0 as the
// reference's `shift >= 15` test does, since every table value is below 2^15.
// Masked keys get t = 2^32 - 1, hence w = 0.
template <bool FULL, int SH>
__device__ __forceinline__ void weights_fast(const uint32_t (&hh)[16], const uint32_t (&mid)[16],
                                             const uint32_t (&ll)[16], int nlive, uint32_t C, uint32_t lane4,
                                             uint32_t (&w)[16]) {
  const uint8_t* tab = reinterpret_cast<const uint8_t*>(s_lutr);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    uint32_t t = C - (hh[i] * 65536u + mid[i] * 256u + ll[i]);
    if (!FULL && i >= nlive) t = 0xFFFFFFFFu;
    const uint32_t v = *reinterpret_cast<const uint32_t*>(tab + (((t << (7 - SH)) & 0x7F80u) | lane4));
    w[i] = shr_clamp(v, t >> (SH + 8));
  }
}

// A kernel that allocates TMEM runs one CTA per SM, so the CTA holds two
// independent groups of 10 warps (producer, MMA issuer, 8 softmax warps), each
// on its own sequence with its own shared-memory region, barriers and 256 TMEM
// columns: the row exchanges, first-tile latency and tail of one group overlap
// the steady state of the other.
template <int HDIM>
__global__ void __launch_bounds__(THREADS, 1) attention_tc_kernel(const __grid_constant__ Maps maps, const Args a) {
  using Hd = HeadDim<HDIM>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t s_abort, s_tslot;
  const int gw = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = gw / GROUP_WARPS, warp = gw % GROUP_WARPS;  // group, warp within the group
  const int gtid = (int)threadIdx.x - grp * GROUP_THREADS;    // thread within the group
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023)) +
                grp * GROUP_BYTES;
  Ctl* ctl = reinterpret_cast<Ctl*>(sm + OFF_BAR);
  int16_t* lut = reinterpret_cast<int16_t*>(sm + OFF_LUT);
  long long* xmax = reinterpret_cast<long long*>(sm + OFF_X);  // [2][QT]
  long long* xmin = xmax + 2 * QT;                             // [2][QT]
  unsigned long long* xsum = reinterpret_cast<unsigned long long*>(xmin + 2 * QT);

  // The query tile is the slowest grid dimension and runs in reverse: every
  // causal CTA with the most key tiles starts before any with fewer, and the
  // shortest fill the tail of the grid.
  const int nq = (int)gridDim.z, qt = nq - 1 - (int)blockIdx.z;
  const int q0 = qt * QT, h = blockIdx.x, bl = GROUPS * blockIdx.y + grp, b = a.b0 + bl;
  const bool active = bl < a.nb;  // an odd batch leaves the last CTA's second group idle
  const int S = a.S;
  const int kend = a.causal ? min(S, q0 + QT) : S;
  const int ntiles = (kend + KT - 1) / KT;
  const int wy = ((bl * a.H + h) * nq + qt) * QT;  // first row of this group's block of the weight scratch

  if (gtid == 0) ctl->abort = 0u;
  if (warp == 0 && lane == 0) {
    mbar_init(&ctl->q_full, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->s_empty[i], SOFTMAX_WARPS);
      mbar_init(&ctl->p_full[i], SOFTMAX_WARPS);
      // the MMAs that read the P buffer, and (storing P) the TMA store that reads it
      mbar_init(&ctl->p_empty[i], a.pstore ? 2 : 1);
    }
    mbar_init(&ctl->o_full, 1);
    mbar_init(&ctl->w_ready, SOFTMAX_WARPS);
    mbar_init(&ctl->q_ready, SOFTMAX_WARPS);
    for (int i = 0; i < WPF_N; ++i) {
      mbar_init(&ctl->w_full[i], 1);
      mbar_init(&ctl->w_empty[i], SOFTMAX_WARPS);
    }
    fence_barrier_init();
  }
  if (gw == 1) {
    tmem_alloc(&s_tslot, TMEM_COLS);
    tmem_relinquish();
  }
  // The prologue above touches no global memory: from here on the previous
  // kernel's outputs (and the status it may have flagged) are visible.
  griddep_wait();
  if (threadIdx.x == 0) s_abort = timed_out(a.st) ? 1u : 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  if (s_abort) {  // a wait of this call already timed out: the whole CTA skips its work
    if (gw == 1) tmem_dealloc(s_tslot, TMEM_COLS);
    return;
  }
  const uint32_t tmem = s_tslot + 256u * (uint32_t)grp;  // this group's 256 columns
  const int row0 = b * S;  // first token row of this sequence

  if (!active) {
    // idle group: nothing to do before the final barrier
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&ctl->q_full, 2 * Hd::PQ);
      tma_load_2d(sm + OFF_Q, &maps.q_hi, &ctl->q_full, h * HDIM, row0 + q0);
      tma_load_2d(sm + OFF_Q + PLANE_Q, &maps.q_lo, &ctl->q_full, h * HDIM, row0 + q0);
      uint32_t it = 0;
      bool ok = true;
      for (int pass = 0; pass < 3 && ok; ++pass) {
        for (int j = 0; j < ntiles; ++j, ++it) {
          const int s = it % ST;
          if (it >= ST && !wait_bar(&ctl->empty[s], ((it / ST) - 1) & 1, ctl, a.st)) {
            ok = false;
            break;
          }
          uint8_t* stg = sm + OFF_STAGE + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&ctl->full[s], pass < 2 ? 2 * Hd::PK : 2 * Hd::PV);
          if (pass < 2) {  // K rows j*32 .. +31 of this head
            tma_load_2d(stg, &maps.k_hi, &ctl->full[s], a.d + h * HDIM, row0 + j * KT);
            tma_load_2d(stg + PLANE_K, &maps.k_lo, &ctl->full[s], a.d + h * HDIM, row0 + j * KT);
          } else {
            if (HDIM == 64 && a.vrow) {  // V rows: keys j*32 .. +31 x the head's 64 dims
              // (keys past the sequence are the next one's rows: their P is 0)
              tma_load_2d(stg, &maps.v_hi, &ctl->full[s], h * HDIM, row0 + j * KT);
              tma_load_2d(stg + PLANE_V, &maps.v_lo, &ctl->full[s], h * HDIM, row0 + j * KT);
            } else {  // V^T: the head's dims x keys j*32 .. +31
              const int vrow = (b * a.H + h) * HDIM;
              tma_load_2d(stg, &maps.vt_hi, &ctl->full[s], j * KT, vrow);
              tma_load_2d(stg + PLANE_V, &maps.vt_lo, &ctl->full[s], j * KT, vrow);
            }
            // the sum pass's weights of tile j, into ring slot j % WPF_N, once
            // the whole scratch block is written
            const int wb = j % WPF_N;
            if ((j == 0 && !wait_bar(&ctl->w_ready, 0, ctl, a.st)) ||
                (j >= WPF_N && !wait_bar(&ctl->w_empty[wb], ((j / WPF_N) - 1) & 1, ctl, a.st))) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&ctl->w_full[wb], WPF_BUF);
            tma_load_2d(sm + OFF_WPF + wb * WPF_BUF, &maps.w, &ctl->w_full[wb], j * KT * 2, wy);
          }
        }
      }
      mbar_wait(&ctl->q_full, 0, a.st);
      for (uint32_t k = (it > ST ? it - ST : 0); k < it; ++k) mbar_wait(&ctl->full[k % ST], (k / ST) & 1, a.st);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    // The whole warp runs the loop (warp-uniform operands); one elected lane
    // issues each MMA and commit, lane 0 the P stores.
    {
      const uint32_t id_ss = idesc_i8(QT, KT, 1, 1), id_su = idesc_i8(QT, KT, 1, 0);
      const uint32_t id_us = idesc_i8(QT, KT, 0, 1), id_uu = idesc_i8(QT, KT, 0, 0);
      const uint32_t pv_us = idesc_i8(QT, HDIM, 0, 1), pv_uu = idesc_i8(QT, HDIM, 0, 0);
      const uint32_t qh = smem_u32(sm + OFF_Q), ql = qh + PLANE_Q;
      uint32_t use0 = 0, use1 = 0;  // uses of each S buffer
      wait_bar(HDIM < 32 ? &ctl->q_ready : &ctl->q_full, 0, ctl, a.st);
      uint32_t it = 0;
      for (int pass = 0; pass < 2; ++pass) {
        for (int j = 0; j < ntiles; ++j, ++it) {
          const int s = it % ST;
          const int sb = (int)(it & 1);
          wait_bar(&ctl->full[s], (it / ST) & 1, ctl, a.st);
          const uint32_t n = sb ? use1 : use0;
          if (n > 0) wait_bar(&ctl->s_empty[sb], (n - 1) & 1, ctl, a.st);
          tc_fence_after();
          const uint32_t kh = smem_u32(sm + OFF_STAGE + s * STAGE_BYTES), kl = kh + PLANE_K;
          const uint32_t d = tmem + (uint32_t)sb * S_BUF1;
#pragma unroll
          for (int ks = 0; ks < Hd::ROW / 32; ++ks) {
            // 64-byte rows (64-byte swizzle) for head dim 64, 32-byte rows for 16
            const uint64_t aqh = Hd::ROW == 64 ? sdesc_k64(qh + 32 * ks) : sdesc_k32(qh);
            const uint64_t aql = Hd::ROW == 64 ? sdesc_k64(ql + 32 * ks) : sdesc_k32(ql);
            const uint64_t bkh = Hd::ROW == 64 ? sdesc_k64(kh + 32 * ks) : sdesc_k32(kh);
            const uint64_t bkl = Hd::ROW == 64 ? sdesc_k64(kl + 32 * ks) : sdesc_k32(kl);
            const uint32_t acc = ks > 0 ? 1u : 0u;
            umma_i8_warp(d + S_HH, aqh, bkh, id_ss, acc);
            umma_i8_warp(d + S_MID, aqh, bkl, id_su, acc);
            umma_i8_warp(d + S_MID, aql, bkh, id_us, 1u);
            umma_i8_warp(d + S_LL, aql, bkl, id_uu, acc);
          }
          umma_commit_warp(&ctl->s_full[sb]);
          umma_commit_warp(&ctl->empty[s]);
          if (sb)
            ++use1;
          else
            ++use0;
        }
      }
      // last pass: O += P(j) V(j), one 32-key K step per tile
      const int pz = b * a.H + h;  // this (sequence, head)'s P matrix
      for (int j = 0; j < ntiles; ++j, ++it) {
        const int s = it % ST;
        wait_bar(&ctl->full[s], (it / ST) & 1, ctl, a.st);
        const int pb = j & 1;
        wait_bar(&ctl->p_full[pb], (j >> 1) & 1, ctl, a.st);
        tc_fence_after();
        if (a.pstore && lane == 0) {  // the cached P of rows q0.. (keys j*32 ..): straight from the MMA's P tile
          const uint8_t* pt = sm + OFF_P + pb * 2 * PLANE_P;
          tma_store_3d(&maps.p_hi, pt, j * KT, q0, pz);
          tma_store_3d(&maps.p_lo, pt + PLANE_P, j * KT, q0, pz);
          bulk_commit();
        }
        const uint32_t vh = smem_u32(sm + OFF_STAGE + s * STAGE_BYTES), vl = vh + PLANE_V;
        const uint32_t ph = smem_u32(sm + OFF_P + pb * 2 * PLANE_P), pl = ph + PLANE_P;
        const uint64_t aph = sdesc_k32(ph), apl = sdesc_k32(pl);
        // V^T tiles are K-major (32-byte rows of keys); V rows are an MN-major
        // B operand (64-byte rows of dims), bit 16 of the instruction descriptor
        const bool mn = HDIM == 64 && a.vrow;
        const uint64_t bvh = mn ? sdesc_mn64(vh) : sdesc_k32(vh), bvl = mn ? sdesc_mn64(vl) : sdesc_k32(vl);
        const uint32_t i_us = mn ? (pv_us | (1u << 16)) : pv_us, i_uu = mn ? (pv_uu | (1u << 16)) : pv_uu;
        const uint32_t acc = j > 0 ? 1u : 0u;
        umma_i8_warp(tmem + O_HH, aph, bvh, i_us, acc);
        umma_i8_warp(tmem + O_MID, aph, bvl, i_uu, acc);
        umma_i8_warp(tmem + O_MID, apl, bvh, i_us, 1u);
        umma_i8_warp(tmem + O_LL, apl, bvl, i_uu, acc);
        umma_commit_warp(&ctl->p_empty[pb]);
        umma_commit_warp(&ctl->empty[s]);
        if (a.pstore && j > 0 && lane == 0) {  // the previous tile's store has read its P buffer
          bulk_wait_read<1>();
          mbar_arrive(&ctl->p_empty[pb ^ 1]);
        }
      }
      umma_commit_warp(&ctl->o_full);
      if (a.pstore && lane == 0) bulk_wait_all();  // the P stores are complete before the CTA (and its shared memory) ends
      // every MMA of this CTA completes before TMEM is released
      mbar_wait(&ctl->o_full, 0, a.st);
    }
  } else {
    // -------------------------------------------------------------- softmax
    // Warp w owns query rows 32*(w%4)..+31 and keys [16*g, 16*g+16) of each
    // 32-key tile, g = (w-2)/4.
    // The exp2 tables are first read in the sum pass, after the max pass's
    // exchange barrier: each group's softmax warps fill them while the first
    // S tiles load (both groups write the same values into the shared
    // lane-replicated copy, and each reads it only after its own fill).
    for (int i = gtid - 64; i < 256; i += 32 * SOFTMAX_WARPS) lut[i] = d_exp2_lut[i];
    for (int i = gtid - 64; i < 256 * 8; i += 32 * SOFTMAX_WARPS) {
      const uint32_t v = (uint32_t)(uint16_t)d_exp2_lut[i >> 3];
      reinterpret_cast<uint4*>(s_lutr)[i] = make_uint4(v, v, v, v);
    }
    if (HDIM < 32) {
      // Head dim 16: each Q row was loaded as 32 bytes (this head's 16, then
      // the next 16 of the row); the upper 16 become zeros, so the 32-byte MMA
      // K step adds nothing for them.  Thread t zeroes row t & 127 of plane
      // t >> 7: logical chunk 1 of the 32-byte-swizzled row.
      wait_bar(&ctl->q_full, 0, ctl, a.st);
      const uint32_t t = (uint32_t)(gtid - 64), r = t & 127u;
      *reinterpret_cast<uint4*>(sm + OFF_Q + (t >> 7) * PLANE_Q + swz32_chunk(r, 1u)) = make_uint4(0u, 0u, 0u, 0u);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->q_ready);
    }
    const int q = gw & 3, g = (warp - 2) >> 2;  // TMEM lane quarter follows the warp's index in the CTA
    const int row = q * 32 + lane;
    const int qi = q0 + row;
    const bool row_live = qi < S;
    const int last_key = row_live ? (a.causal ? min(qi, S - 1) : S - 1) : -1;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t lane4 = (uint32_t)lane * 4u;
    uint32_t use0 = 0, use1 = 0;  // uses of each S buffer, in the MMA issuer's order
    // This warp's 32 rows x 16 keys of an S tile, from TMEM into registers;
    // the buffer is released as soon as the values are loaded.
    auto fetch_s = [&](int sb, uint32_t(&hh)[16], uint32_t(&mid)[16], uint32_t(&ll)[16]) {
      wait_bar(&ctl->s_full[sb], (sb ? use1 : use0) & 1, ctl, a.st);
      if (sb)
        ++use1;
      else
        ++use0;
      tc_fence_after();
      const uint32_t tb = trow + (uint32_t)sb * S_BUF1 + 16 * g;
      tmem_ld16(tb + S_HH, hh);
      tmem_ld16(tb + S_MID, mid);
      tmem_ld16(tb + S_LL, ll);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->s_empty[sb]);
    };
    auto live_keys = [&](int j) { return max(0, min(16, last_key - (j * KT + 16 * g) + 1)); };

    // |hh| = |sum q_hi k_hi| <= L1(q_hi) * 128 for any key, so a warp whose
    // rows all have L1(q_hi) <= 128 skips the per-tile range check of hh.
    // (Head dim 16: the head's 16 bytes are the row's logical chunk 0.)
    bool qbounded;
    {
      wait_bar(&ctl->q_full, 0, ctl, a.st);
      uint32_t l1 = 0;
      if (HDIM < 32) {
        l1 = abs_sum16(*reinterpret_cast<const uint4*>(sm + OFF_Q + swz32_chunk((uint32_t)row, 0u)));
      } else {
#pragma unroll
        for (int c = 0; c < Hd::ROW / 16; ++c)  // the swizzle permutes chunks within the row
          l1 += abs_sum16(*reinterpret_cast<const uint4*>(sm + OFF_Q + row * Hd::ROW + 16 * c));
      }
      qbounded = __all_sync(FULLMASK, l1 <= 128u);
    }

    // ---- pass 0: row max of raw = q.k ----
    // With head_dim 64 |256*mid + ll| <= B_MID (< 2^30), so raw is an exact
    // i32 whenever |hh| <= 16384 (mx32); other elements take an i64 path that
    // also keeps the row min for the i32 range check of the logits.
    int mx32 = INT_MIN;
    long long mx64 = LLONG_MIN, mn64 = LLONG_MAX;
    uint32_t it = 0;  // S tiles of passes 0 and 1, which alternate the two S buffers
    for (int j = 0; j < ntiles; ++j, ++it) {
      uint32_t hh[16], mid[16], ll[16];
      fetch_s((int)(it & 1), hh, mid, ll);
      const int nlive = live_keys(j);
      const bool full = __all_sync(FULLMASK, nlive == 16);
      if (qbounded) {
        if (full)
          tile_max_bounded<true>(hh, mid, ll, nlive, mx32);
        else
          tile_max_bounded<false>(hh, mid, ll, nlive, mx32);
      } else if (full) {
        tile_max<true>(hh, mid, ll, nlive, mx32, mx64, mn64);
      } else {
        tile_max<false>(hh, mid, ll, nlive, mx32, mx64, mn64);
      }
    }
    // Per-row constants of passes 1 and 2.
    uint32_t rawmax_lo = 0, cround = 0;
    int hh_floor = INT_MAX;
    bool slow_row = false, row_fast = false, range_bad = false, masked_bad = false;
    long long rawmax = 0, lgmax = 0;
    {
      // INT_MIN is never an exact-i32 raw value (> -2^30 - B_MID), so it marks "none".
      long long rmx = max(mx32 == INT_MIN ? LLONG_MIN : (long long)mx32, mx64);
      long long rmn = mn64;
      xmax[g * QT + row] = rmx;
      xmin[g * QT + row] = rmn;
      named_sync_softmax(grp);
      rmx = max(rmx, xmax[(g ^ 1) * QT + row]);
      rmn = min(rmn, xmin[(g ^ 1) * QT + row]);
      if (row_live) {
        rawmax = rmx;
        lgmax = rawmax >> Hd::SH;
        if (lgmax > INT_MAX || (rmn != LLONG_MAX && (rmn >> Hd::SH) < INT_MIN)) range_bad = true;
        if (lgmax <= (long long)INT_MIN) masked_bad = true;  // every live logit masked or out of range
        slow_row = lgmax < (long long)INT_MIN + 15 * 256;
        rawmax_lo = (uint32_t)rawmax;
        cround = ((1u << Hd::SH) - 1u) - (uint32_t)(rawmax & ((1 << Hd::SH) - 1));
        // candidates for w != 0: 65536*hh + B_MID > rawmax - (3840 << SH)
        const long long fl = (rawmax - (3840LL << Hd::SH) - B_MID) >> 16;
        hh_floor = (int)max((long long)INT_MIN, min((long long)INT_MAX, fl));
        // no element of the row took the i64 path: every raw value of the
        // row, rawmax included, is an exact i32 of magnitude <= 2^30 + B_MID
        row_fast = rmn == LLONG_MAX;
      }
    }
    const uint32_t cfast = rawmax_lo + cround;
    const bool warp_fast = __all_sync(FULLMASK, row_fast || !row_live);
    // Weights w of one S tile of this warp (0 for masked keys).
    auto weights = [&](const uint32_t(&hh)[16], const uint32_t(&mid)[16], const uint32_t(&ll)[16], int nlive,
                       uint32_t(&w)[16]) {
      const bool full = __all_sync(FULLMASK, nlive == 16);
      if (warp_fast) {
        if (full)
          weights_fast<true, Hd::SH>(hh, mid, ll, nlive, cfast, lane4, w);
        else
          weights_fast<false, Hd::SH>(hh, mid, ll, nlive, cfast, lane4, w);
        return;
      }
      int wi[16];
      if (!slow_row) {
        if (full)
          scores_weight<true, Hd::SH>(hh, mid, ll, nlive, hh_floor, rawmax_lo, cround, lut, wi);
        else
          scores_weight<false, Hd::SH>(hh, mid, ll, nlive, hh_floor, rawmax_lo, cround, lut, wi);
      } else {
        // Rows whose max logit lies within 15 * 256 of i32::MIN: exact i64
        // path, with logits equal to MASKED_LOGIT excluded (attention.rs:266-276).
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          int v = 0;
          if (i < nlive) {
            const long long raw = (long long)(int)hh[i] * 65536 + (long long)(int)mid[i] * 256 + (long long)(int)ll[i];
            const long long lg = raw >> Hd::SH;
            const long long delta = lg - lgmax;
            if (delta > -15 * 256 && lg != (long long)INT_MIN) {
              const int mag = (int)(-delta);
              v = (int)lut[mag & 255] >> (mag >> 8);
            }
          }
          wi[i] = v;
        }
      }
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = (uint32_t)wi[i];
    };

    // ---- pass 1: weights and the row sum ----
    // Each warp's 32 rows x 16 weights of a tile go through its own 1 KB of
    // shared memory (32-byte rows, 32-byte swizzle: conflict-free 16-byte
    // stores) and out with one TMA store of that box, so the warps never wait
    // on one another.  Three slots per warp, in the last pass's prefetch
    // region: before slot j % 3 is rewritten, lane 0 waits until all but its
    // two newest stores have read shared memory.
    uint8_t* wst = sm + OFF_WPF + (q * 2 + g) * 1024;
    uint32_t rsum = 0;  // this thread's keys: at most 16384 / 2 weights below 2^15
    const uint32_t c0 = swz32_chunk((uint32_t)lane, 0u), c1 = swz32_chunk((uint32_t)lane, 1u);
    for (int j = 0; j < ntiles; ++j, ++it) {
      uint32_t hh[16], mid[16], ll[16], w[16];
      fetch_s((int)(it & 1), hh, mid, ll);
      weights(hh, mid, ll, live_keys(j), w);
      // weights are below 2^15: pairs packed as 16-bit halves for the store,
      // and each pair added to the row sum by one dp2a (lo * 1 + hi * 1)
      uint32_t wp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        wp[i] = __byte_perm(w[2 * i], w[2 * i + 1], 0x5410);
        rsum = __dp2a_lo(wp[i], 0x0101u, rsum);
      }
      uint8_t* tb = wst + (j % 3) * (QT * 64);
      if (j >= 3) {
        if (lane == 0) bulk_wait_read<2>();
        __syncwarp();
      }
      *reinterpret_cast<uint4*>(tb + c0) = make_uint4(wp[0], wp[1], wp[2], wp[3]);
      *reinterpret_cast<uint4*>(tb + c1) = make_uint4(wp[4], wp[5], wp[6], wp[7]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&maps.ws, tb, j * KT * 2 + 32 * g, wy + 32 * q);
        bulk_commit();
      }
    }
    if (lane == 0) {  // this warp's stores are complete before the producer loads the tiles back
      bulk_wait_all();
      fence_proxy_async_global();
      mbar_arrive(&ctl->w_ready);
    }
    uint32_t inv = 0;
    {
      unsigned long long tot = rsum;
      xsum[g * QT + row] = tot;
      named_sync_softmax(grp);
      tot += xsum[(g ^ 1) * QT + row];
      inv = (row_live && tot) ? recip_sum_q31(tot) : 0u;
    }

    // ---- pass 2: P = sat_i16(rhu(w * inv, 16)) as byte planes, O += P V ----
    // The weights come back as 128 x 32 tiles that the producer loads by TMA
    // into a WPF_N-slot ring ([row][64 bytes], 64-byte swizzle).
    const uint32_t wsw = ((uint32_t)row >> 1) & 3u;
    for (int j = 0; j < ntiles; ++j) {
      const int key0 = j * KT + 16 * g;
      uint32_t w[16];
      const int wb = j % WPF_N;
      wait_bar(&ctl->w_full[wb], (j / WPF_N) & 1, ctl, a.st);
      const uint8_t* wt = sm + OFF_WPF + wb * WPF_BUF + row * 64;
      const uint4 u0 = *reinterpret_cast<const uint4*>(wt + (((2u * g) ^ wsw) << 4));
      const uint4 u1 = *reinterpret_cast<const uint4*>(wt + (((2u * g + 1u) ^ wsw) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->w_empty[wb]);
      const uint32_t wv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        w[2 * i] = wv[i] & 0xFFFFu;
        w[2 * i + 1] = wv[i] >> 16;
      }
      // w <= sum(w) and inv <= 2^31 * (129/128) / sum(w), so rhu(w * inv, 16)
      // <= 33025 < 2^16: two of them pack into 16-bit halves before the
      // saturation to 32767, which is one packed min per pair
      uint32_t pw[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t p0 = (uint32_t)(((unsigned long long)w[2 * i] * inv + 32768ull) >> 16);
        const uint32_t p1 = (uint32_t)(((unsigned long long)w[2 * i + 1] * inv + 32768ull) >> 16);
        pw[i] = min_u16x2(__byte_perm(p0, p1, 0x5410), 0x7FFF7FFFu);
      }
      if (a.probs && row_live && key0 < S) {  // nsrl-train/src/lib.rs:15353-15418: the cached P
        uint4* dst = reinterpret_cast<uint4*>(a.probs + (((long long)b * a.H + h) * S + qi) * (long long)S + key0);
        dst[0] = make_uint4(pw[0], pw[1], pw[2], pw[3]);
        dst[1] = make_uint4(pw[4], pw[5], pw[6], pw[7]);
      }
      const int pb = j & 1;
      if (j >= 2) wait_bar(&ctl->p_empty[pb], ((j >> 1) - 1) & 1, ctl, a.st);
      uint8_t* ph = sm + OFF_P + pb * 2 * PLANE_P;
      uint8_t* pl = ph + PLANE_P;
      uint32_t hw[4], lw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        hw[k] = __byte_perm(pw[2 * k], pw[2 * k + 1], 0x7531);
        lw[k] = __byte_perm(pw[2 * k], pw[2 * k + 1], 0x6420);
      }
      const uint32_t off = swz32_chunk((uint32_t)row, (uint32_t)g);
      *reinterpret_cast<uint4*>(ph + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
      *reinterpret_cast<uint4*>(pl + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->p_full[pb]);
    }
    if (range_bad) nsrl_flag(a.st, NSRL_FLAG_LOGIT_RANGE);
    if (masked_bad) nsrl_flag(a.st, NSRL_FLAG_ALL_MASKED);
    // ---- context: sat(rhu(65536*hh + 256*mid + ll, 15)) as byte planes ----
    // The exact sum fits i32: p <= w * inv / 2^16 + 1/2 with inv <= 2^31 *
    // (129/128) / sum(w) (8-bit reciprocal mantissa), so sum(p) <= 33024 +
    // keys / 2 <= 41216 for at most 16384 keys, and |sum(p * v)| <=
    // 41216 * 32768 < 2^31 - 2^14.  Wrapping 32-bit recombination is exact
    // and rhu(tot, 15) = (tot + 2^14) >> 15 cannot overflow.
    wait_bar(&ctl->o_full, 0, ctl, a.st);
    tc_fence_after();
    // Destination row: this rank's context rows, or (head-sharded) the rows
    // of the rank that owns position qi.
    int8_t* chi = a.ctx_hi;
    uint8_t* clo = a.ctx_lo;
    unsigned long long* cl1 = a.ctx_l1;
    long long crow = (long long)row0 + qi;
    if (a.rt.nranks && row_live) {  // rows past the sequence store nothing
      const int own = qi / a.rt.s_loc;
      chi = a.rt.tab->ctx_hi[own];
      clo = a.rt.tab->ctx_lo[own];
      cl1 = a.ctx_l1 ? a.rt.tab->ctx_l1[own] : nullptr;
      crow = (long long)b * a.rt.s_loc + (qi - own * a.rt.s_loc);
    }
    unsigned l1 = 0;
    // Head dim 64, unrouted: a lane's 32 dims are one 32-byte run per plane;
    // the first 16 wait in registers for the second, then both go out as
    // lane pairs (every lane takes part, live row or not; qi has the lane's
    // parity).
    const bool pairs = HDIM == 64 && !a.rt.nranks && (a.ldc & 15) == 0;
    uint32_t h0[4], l0[4];
#pragma unroll
    for (int c = 0; c < 2; ++c) {  // dims [32g + 16c, +16) of the head's HDIM
      uint32_t oh[16], om[16], ol[16];
      const uint32_t col = (uint32_t)(32 * g + 16 * c);
      if (col >= (uint32_t)HDIM) continue;
      tmem_ld16(trow + O_HH + col, oh);
      tmem_ld16(trow + O_MID + col, om);
      tmem_ld16(trow + O_LL + col, ol);
      tmem_wait_ld();
      if (row_live || pairs) {
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int t0 = (int)(oh[2 * i] * 65536u + om[2 * i] * 256u + ol[2 * i]);
          const int t1 = (int)(oh[2 * i + 1] * 65536u + om[2 * i + 1] * 256u + ol[2 * i + 1]);
          const int v0 = max(-32768, min(32767, (t0 + 16384) >> 15));
          const int v1 = max(-32768, min(32767, (t1 + 16384) >> 15));
          if (row_live) l1 += (unsigned)(abs(v0) + abs(v1));
          pk[i] = __byte_perm((uint32_t)v0, (uint32_t)v1, 0x5410);
        }
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          hw[k] = __byte_perm(pk[2 * k], pk[2 * k + 1], 0x7531);
          lw[k] = __byte_perm(pk[2 * k], pk[2 * k + 1], 0x6420);
        }
        if (pairs) {
          if (c == 0) {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              h0[k] = hw[k];
              l0[k] = lw[k];
            }
            continue;
          }
          const uint32_t hi8[8] = {h0[0], h0[1], h0[2], h0[3], hw[0], hw[1], hw[2], hw[3]};
          const uint32_t lo8[8] = {l0[0], l0[1], l0[2], l0[3], lw[0], lw[1], lw[2], lw[3]};
          const long long base = (long long)row0 * a.ldc + h * HDIM + 32 * g;
          store32b_pairs(reinterpret_cast<uint8_t*>(chi + base), a.ldc, qi, S, hi8, lane);
          store32b_pairs(clo + base, a.ldc, qi, S, lo8, lane);
          continue;
        }
        const long long off = crow * a.ldc + a.rt.col0 + h * HDIM + col;
        *reinterpret_cast<uint4*>(chi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        *reinterpret_cast<uint4*>(clo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
      }
    }
    if (row_live && cl1 && 32 * g < HDIM) atomicAdd(&cl1[crow], (unsigned long long)l1);
  }
  tc_fence_before();
  __syncthreads();
  if (gw == 1) {
    tc_fence_after();
    tmem_dealloc(s_tslot, TMEM_COLS);
  }
}

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

// 2-D uint8 map [rows][inner] (row stride ld bytes), box [box_rows][box_inner
// bytes] with the swizzle of that row width (64 or 32 bytes).
bool make_map(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_inner,
              uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t es[2] = {1, 1};
  const CUtensorMapSwizzle sw = box_inner == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B;
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Bytes of weight scratch per sequence, and the sequences one launch covers:
// at most 4 GiB of scratch (at least one sequence), reused by the launches of
// a larger batch in stream order.
size_t scratch_per_seq(size_t S, size_t H) {
  const size_t nq = (S + QT - 1) / QT;
  return H * nq * QT * attention_tc_wstride(S) * sizeof(int16_t);
}
size_t chunk_seqs(size_t B, size_t S, size_t H) {
  const size_t per = scratch_per_seq(S, H);
  return std::max<size_t>(1, std::min<size_t>(B, ((size_t)4 << 30) / per));
}

// 3-D uint8 map of the P planes [BH][S][S] (keys contiguous), box [1][QT
// rows][KT bytes], 32-byte swizzle (the layout of the MMA's P tile); rows and
// keys past S lie outside the tensor, so a store of the last query tile stops
// at the sequence's end.
bool make_p_map(CUtensorMap* m, const void* ptr, uint64_t S, uint64_t BH) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {S, S, BH};
  cuuint64_t strides[2] = {S, S * S};
  cuuint32_t box[3] = {(cuuint32_t)KT, (cuuint32_t)QT, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attention_tc_supported(size_t S, size_t d, size_t H) {
  return H != 0 && d / H == (size_t)HD && d % H == 0 && S % 16 == 0 && S <= 16384 && (3 * d) % 16 == 0;
}

bool attention_tc_forward_supported(size_t S, size_t d, size_t H) {
  return H != 0 && d % H == 0 && (d / H == 64 || d / H == 16) && S % 16 == 0 && S <= 16384 && (3 * d) % 16 == 0;
}

size_t attention_tc_wstride(size_t S) { return (S + 63) / 64 * 64; }

size_t attention_tc_scratch_bytes(size_t B, size_t S, size_t d, size_t H) {
  if (!attention_tc_forward_supported(S, d, H) || B == 0) return 0;
  return chunk_seqs(B, S, H) * scratch_per_seq(S, H);
}

cudaError_t launch_attention_tc(const Planes& qkv, const VtPlanes& vt, size_t B, size_t S, size_t d, size_t H,
                                bool causal, Planes ctx, int16_t* wscr, nsrl_device_status* st,
                                cudaStream_t stream, int16_t* probs, const Planes* probs_planes,
                                const CtxRoute* route, bool v_rows) {
  if (!attention_tc_forward_supported(S, d, H) || encode_fn() == nullptr || wscr == nullptr)
    return cudaErrorNotSupported;
  const size_t hd = d / H;
  // head dim 16: the forward only (no P for a backward, no head-sharded routing)
  if (hd == 16 && (probs || probs_planes || (route && route->nranks))) return cudaErrorNotSupported;
  if (probs_planes && (!causal || probs_planes->ld != S)) return cudaErrorInvalidValue;
  // V as row-major planes (the q|k|v planes' V columns): head dim 64, not routed
  if (v_rows && (hd != 64 || (route && route->nranks))) return cudaErrorInvalidValue;
  if (route && route->nranks &&
      (route->tab == nullptr || route->s_loc <= 0 || S % (size_t)route->s_loc != 0 || probs || probs_planes))
    return cudaErrorInvalidValue;
  if (B == 0) return cudaSuccess;
  const size_t T = B * S;
  Maps m;
  const bool ok =
      // q and k rows of a head: 64 bytes (64-byte swizzle), or for head dim 16
      // 32 bytes from the head's first (32-byte swizzle; Q's extra 16 zeroed
      // in the kernel)
      make_map(&m.q_hi, qkv.hi, 2 * d, T, qkv.ld, hd == 64 ? 64 : 32, QT) &&
      make_map(&m.q_lo, qkv.lo, 2 * d, T, qkv.ld, hd == 64 ? 64 : 32, QT) &&
      make_map(&m.k_hi, qkv.hi, 2 * d, T, qkv.ld, hd == 64 ? 64 : 32, KT) &&
      make_map(&m.k_lo, qkv.lo, 2 * d, T, qkv.ld, hd == 64 ? 64 : 32, KT) &&
      (v_rows || (make_map(&m.vt_hi, vt.hi, S, B * H * hd, S, KT, (uint32_t)hd) &&
                  make_map(&m.vt_lo, vt.lo, S, B * H * hd, S, KT, (uint32_t)hd))) &&
      // V rows of a head: 32 keys x 64 bytes (64-byte swizzle) from the V columns
      (!v_rows || (make_map(&m.v_hi, qkv.hi + 2 * d, d, T, qkv.ld, 64, KT) &&
                   make_map(&m.v_lo, qkv.lo + 2 * d, d, T, qkv.ld, 64, KT))) &&
      (!probs_planes || (make_p_map(&m.p_hi, probs_planes->hi, S, B * H) && make_p_map(&m.p_lo, probs_planes->lo, S, B * H))) &&
      make_map(&m.w, wscr, 2 * attention_tc_wstride(S), chunk_seqs(B, S, H) * H * ((S + QT - 1) / QT) * QT,
               2 * attention_tc_wstride(S), 64, QT) &&
      make_map(&m.ws, wscr, 2 * attention_tc_wstride(S), chunk_seqs(B, S, H) * H * ((S + QT - 1) / QT) * QT,
               2 * attention_tc_wstride(S), 32, 32);
  if (!ok) return cudaErrorNotSupported;
  if (!probs_planes) {
    m.p_hi = m.q_hi;  // unused
    m.p_lo = m.q_lo;
  }
  if (v_rows) {
    m.vt_hi = m.q_hi;  // unused
    m.vt_lo = m.q_lo;
  } else {
    m.v_hi = m.q_hi;  // unused
    m.v_lo = m.q_lo;
  }
  Args a{};
  a.S = (int)S;
  a.d = (int)d;
  a.H = (int)H;
  a.causal = causal ? 1 : 0;
  a.ctx_hi = ctx.hi;
  a.ctx_lo = ctx.lo;
  a.ctx_l1 = ctx.l1;
  a.ldc = (long long)ctx.ld;
  a.vrow = v_rows ? 1 : 0;
  a.probs = probs;
  a.pstore = probs_planes ? 1 : 0;
  if (route) a.rt = *route;
  a.st = st;
  a.wscr = wscr;
  a.wstride = (long long)attention_tc_wstride(S);
  static bool configured[2] = {false, false};
  if (!configured[hd == 16]) {
    const cudaError_t e = cudaFuncSetAttribute(hd == 16 ? attention_tc_kernel<16> : attention_tc_kernel<64>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[hd == 16] = true;
  }
  const double pairs = causal ? (double)S * (S + 1) / 2.0 : (double)S * S;
  ProfScope prof(hd == 16 ? "attention_tc_hd16" : "attention_tc_hd64", stream,
                 4.0 * (double)hd * (double)H * (double)B * pairs, 8.0 * (double)T * (double)d);
  const size_t chunk = chunk_seqs(B, S, H);
  for (size_t b0 = 0; b0 < B; b0 += chunk) {
    a.b0 = (int)b0;
    a.nb = (int)std::min(chunk, B - b0);
    const dim3 grid((unsigned)H, (unsigned)((a.nb + GROUPS - 1) / GROUPS), (unsigned)((S + QT - 1) / QT));
    cudaError_t e = hd == 16 ? launch_pdl(attention_tc_kernel<16>, grid, dim3(THREADS), SMEM_BYTES, stream, m, a)
                             : launch_pdl(attention_tc_kernel<64>, grid, dim3(THREADS), SMEM_BYTES, stream, m, a);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace nsrl
