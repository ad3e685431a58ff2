// i16 x i8 -> i16 per-channel linear on the B200 tensor cores (tcgen05, kind::i8).
//
// Reference: crates/nsrl-core/src/linear.rs:228-324.  y[m][n] =
// requantize_i32_to_i16(bias[n] + sum_k x[m][k] * W[n][k], scale[n]) with an
// i32 accumulator whose every prefix must fit (else the call is `None`).
//
// Exactness on int8 tensor cores: x is held as byte planes x = 256*hi + lo
// (hi signed, lo unsigned).  Two MMAs share the weight tile: hi x W (s8.s8)
// and lo x W (u8.s8), each into its own s32 TMEM accumulator; both partial
// sums are exact (|hi*w| <= 16256, |lo*w| <= 32385 per product), and the
// epilogue recombines 256*acc_hi + acc_lo + bias in i64.  A final sum outside
// i32 is flagged here; an overflow of an intermediate prefix can only happen
// when |bias| + 127 * sum_k |x[m][k]| > i32::MAX, and those rows (if any) are
// re-scanned in reference order by prefix_check_kernel.
//
// Kernel shape: one 128 x 128 output tile per CTA, 6 warps:
//   warp 0      TMA producer (A hi/lo planes + W tile per 128-wide K block)
//   warp 1      TMEM allocator + single-thread MMA issuer
//   warps 2..5  epilogue (TMEM -> registers -> requant -> global)
// Operand tiles use the 128-byte swizzle, K-major, one 128-byte row per
// tile row, as written by TMA.
#include <cstdio>

#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;
constexpr int TILE_A = BM * BK;                   // one plane, 16 KB
constexpr int TILE_B = BN * BK;                   // 16 KB
constexpr int STAGE_BYTES = 2 * TILE_A + TILE_B;  // 48 KB
constexpr uint32_t TMEM_COLS = 256;               // acc_hi: cols [0,128), acc_lo: [128,256)

struct TcMaps {
  CUtensorMap a_hi, a_lo, b[3];
};

struct TcParams {
  int M, K, N;  // N = output columns (GATED: hidden channels)
  int nseg, seg_rows;
  const int32_t* bias[3];
  const nsrl_fixed_scale* scales[3];
  int16_t* y;
  long long ldy;
  int8_t* yh;
  uint8_t* yl;
  unsigned long long* yl1;
  long long ldp;
  const int16_t* skip;
  long long ldskip;
  unsigned long long* sat;
  nsrl_device_status* st;
};

// Combine the two partial sums of one output, apply bias and the scale.
__device__ __forceinline__ int16_t finish(int hi, int lo, const int32_t* bias, const nsrl_fixed_scale* sc, int n,
                                          bool& overflow) {
  long long acc = (long long)hi * 256 + (long long)lo + (bias ? (long long)bias[n] : 0ll);
  if (acc < INT_MIN || acc > INT_MAX) overflow = true;
  nsrl_fixed_scale s = sc[n];
  return requant_i32((int)acc, s.multiplier, s.right_shift);
}

__device__ __forceinline__ void store_i16x32(int16_t* dst, const int16_t (&v)[32], int nvalid, bool vec_ok) {
  if (vec_ok && nvalid == 32) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    const uint4* s = reinterpret_cast<const uint4*>(v);
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = s[i];
  } else {
    for (int i = 0; i < nvalid; ++i) dst[i] = v[i];
  }
}

__device__ __forceinline__ void store_planes32(int8_t* dh, uint8_t* dl, const int16_t* v, int nvalid, bool vec_ok,
                                               unsigned long long& l1) {
  uint32_t hw[8], lw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t h = 0, l = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int x = v[4 * i + j];
      h |= (uint32_t)((x >> 8) & 255) << (8 * j);
      l |= (uint32_t)(x & 255) << (8 * j);
    }
    hw[i] = h;
    lw[i] = l;
  }
  for (int i = 0; i < nvalid; ++i) l1 += (unsigned long long)abs((int)v[i]);
  if (vec_ok && nvalid == 32) {
    uint4* a = reinterpret_cast<uint4*>(dh);
    uint4* b = reinterpret_cast<uint4*>(dl);
    a[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    a[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    b[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    b[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
  } else {
    for (int i = 0; i < nvalid; ++i) {
      dh[i] = (int8_t)(v[i] >> 8);
      dl[i] = (uint8_t)(v[i] & 255);
    }
  }
}

template <int EPI, int STAGES>
__global__ void __launch_bounds__(192, 1) gemm_tc_kernel(const __grid_constant__ TcMaps maps, const TcParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);
  uint32_t* skip_flag = tslot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) *skip_flag = timed_out(p.st) ? 1u : 0u;
  __syncthreads();
  if (*skip_flag) return;  // a wait of this call already timed out: do nothing
  const int m0 = blockIdx.y * BM;
  const int nt = blockIdx.x;
  const int nkb = (p.K + BK - 1) / BK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    fence_barrier_init();
    prefetch_tmap(&maps.a_hi);
    prefetch_tmap(&maps.a_lo);
  }
  if (warp == 1) {
    tmem_alloc(tslot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  // Which weight rows feed this N tile.
  int seg = 0, brow = nt * BN;
  if (EPI == (int)Epi::GATED) {
    brow = nt * (BN / 2);
  } else if (p.nseg == 3) {
    seg = (nt * BN) / p.seg_rows;
    brow = (nt * BN) % p.seg_rows;
  }

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (kb >= STAGES && !mbar_wait(&empty[s], ph ^ 1, p.st)) break;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        uint8_t* sa = smem + s * STAGE_BYTES;
        tma_load_2d(sa, &maps.a_hi, &full[s], kb * BK, m0);
        tma_load_2d(sa + TILE_A, &maps.a_lo, &full[s], kb * BK, m0);
        if (EPI == (int)Epi::GATED) {
          tma_load_2d(sa + 2 * TILE_A, &maps.b[0], &full[s], kb * BK, brow);
          tma_load_2d(sa + 2 * TILE_A + TILE_B / 2, &maps.b[1], &full[s], kb * BK, brow);
        } else {
          tma_load_2d(sa + 2 * TILE_A, &maps.b[seg], &full[s], kb * BK, brow);
        }
        issued = kb + 1;
      }
      // Drain: the loads still in flight must land before the CTA can exit.
      for (int kb = (issued > STAGES ? issued - STAGES : 0); kb < issued; ++kb)
        mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1, p.st);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_hi = idesc_i8(BM, BN, 1, 1);  // s8 x s8
      const uint32_t id_lo = idesc_i8(BM, BN, 0, 1);  // u8 x s8
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, p.st)) break;
        tc_fence_after();
        const uint32_t base = smem_u32(smem + s * STAGE_BYTES);
#pragma unroll
        for (int j = 0; j < BK / 32; ++j) {
          const uint64_t ah = sdesc_k128(base + 32 * j);
          const uint64_t al = sdesc_k128(base + TILE_A + 32 * j);
          const uint64_t bd = sdesc_k128(base + 2 * TILE_A + 32 * j);
          const uint32_t acc = (kb > 0 || j > 0) ? 1u : 0u;
          umma_i8(tmem, ah, bd, id_hi, acc);
          umma_i8(tmem + BN, al, bd, id_lo, acc);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accf);
    }
  } else {
    // Epilogue: warp w reads TMEM lanes [32*(w%4), 32*(w%4)+32).
    const bool ok = mbar_wait(accf, 0, p.st);
    tc_fence_after();
    const int q = warp & 3;
    const int r = m0 + q * 32 + lane;
    const bool row_ok = ok && r < p.M;
    const uint32_t lrow = tmem + ((uint32_t)(q * 32) << 16);
    bool overflow = false;
    unsigned long long l1 = 0, sat = 0;
    if (EPI == (int)Epi::GATED) {
      const int f0 = nt * (BN / 2);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t h[32], l[32];
        int16_t up[32], out[32];
        tmem_ld32(lrow + 32 * c, h);
        tmem_ld32(lrow + BN + 32 * c, l);
        tmem_wait_ld();
        const int fb = f0 + 32 * c;
        const int nvalid = max(0, min(32, p.N - fb));
#pragma unroll
        for (int i = 0; i < 32; ++i)
          up[i] = i < nvalid ? finish((int)h[i], (int)l[i], p.bias[0], p.scales[0], fb + i, overflow) : 0;
        tmem_ld32(lrow + 64 + 32 * c, h);
        tmem_ld32(lrow + BN + 64 + 32 * c, l);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          int16_t g = i < nvalid ? finish((int)h[i], (int)l[i], p.bias[1], p.scales[1], fb + i, overflow) : 0;
          out[i] = gated_act(up[i], g);
        }
        if (row_ok && nvalid > 0) {
          const long long o = (long long)r * p.ldp + fb;
          store_planes32(p.yh + o, p.yl + o, out, nvalid, ((p.ldp | fb) & 15) == 0, l1);
        }
      }
    } else {
      const int nb = nt * BN;
      const int sseg = (p.nseg == 3) ? nb / p.seg_rows : 0;
      const int nloc0 = (p.nseg == 3) ? nb % p.seg_rows : nb;
      const int32_t* bias = p.bias[sseg];
      const nsrl_fixed_scale* sc = p.scales[sseg];
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t h[32], l[32];
        int16_t out[32];
        tmem_ld32(lrow + 32 * c, h);
        tmem_ld32(lrow + BN + 32 * c, l);
        tmem_wait_ld();
        const int n = nb + 32 * c;
        const int nvalid = max(0, min(32, p.N - n));
#pragma unroll
        for (int i = 0; i < 32; ++i)
          out[i] = i < nvalid ? finish((int)h[i], (int)l[i], bias, sc, nloc0 + 32 * c + i, overflow) : 0;
        if (!row_ok || nvalid == 0) continue;
        if (EPI == (int)Epi::I16) {
          store_i16x32(p.y + (long long)r * p.ldy + n, out, nvalid, ((p.ldy | n) & 7) == 0);
        } else if (EPI == (int)Epi::RESID) {
          const int16_t* sk = p.skip + (long long)r * p.ldskip + n;
          int16_t res[32];
          const bool vec = ((p.ldskip | p.ldy | n) & 7) == 0 && nvalid == 32;
          if (vec) {
#pragma unroll
            for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(res)[i] = reinterpret_cast<const uint4*>(sk)[i];
          } else {
            for (int i = 0; i < nvalid; ++i) res[i] = sk[i];
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            int w = (int)res[i] + (int)out[i];
            if (i < nvalid && (w < -32768 || w > 32767)) ++sat;
            res[i] = sat_i16_i32(w);
          }
          store_i16x32(p.y + (long long)r * p.ldy + n, res, nvalid, vec);
        } else {
          const long long o = (long long)r * p.ldp + n;
          store_planes32(p.yh + o, p.yl + o, out, nvalid, ((p.ldp | n) & 15) == 0, l1);
        }
      }
    }
    if (overflow && row_ok) nsrl_flag(p.st, NSRL_FLAG_LINEAR_OVERFLOW);
    if ((EPI == (int)Epi::PLANES || EPI == (int)Epi::GATED) && p.yl1 && row_ok) atomicAdd(&p.yl1[r], l1);
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
  bool overflow = false;
  int16_t v;
  if (s.epi == (int)Epi::GATED) {
    int h, l;
    simt_dot(s, m, 0, n, h, l);
    int16_t up = finish(h, l, p.bias[0], p.scales[0], n, overflow);
    simt_dot(s, m, 1, n, h, l);
    int16_t g = finish(h, l, p.bias[1], p.scales[1], n, overflow);
    v = gated_act(up, g);
  } else {
    const int sg = s.nseg == 3 ? n / s.seg_rows : 0;
    const int nl = s.nseg == 3 ? n % s.seg_rows : n;
    int h, l;
    simt_dot(s, m, sg, nl, h, l);
    v = finish(h, l, p.bias[sg], p.scales[sg], nl, overflow);
  }
  if (overflow) nsrl_flag(p.st, NSRL_FLAG_LINEAR_OVERFLOW);
  if (s.epi == (int)Epi::I16) {
    p.y[(long long)m * p.ldy + n] = v;
  } else if (s.epi == (int)Epi::RESID) {
    int w = (int)p.skip[(long long)m * p.ldskip + n] + (int)v;
    if (w < -32768 || w > 32767) atomicAdd(p.sat, 1ull);
    p.y[(long long)m * p.ldy + n] = sat_i16_i32(w);
  } else {
    p.yh[(long long)m * p.ldp + n] = (int8_t)(v >> 8);
    p.yl[(long long)m * p.ldp + n] = (uint8_t)(v & 255);
    if (p.yl1) atomicAdd(&p.yl1[m], (unsigned long long)abs((int)v));
  }
}

// ---------------------------------------------------------------------------
// Exact i32 prefix check (linear.rs:282-296): for rows where
// |bias| + 127 * L1(x_row) can exceed i32::MAX, rescan every output in the
// reference's order (bias first, then k = 0, 1, ...) with checked adds.
// One warp per row; rows within the bound exit after one comparison.
// ---------------------------------------------------------------------------
struct CheckParams {
  const int8_t* a_hi;
  const uint8_t* a_lo;
  long long lda;
  const unsigned long long* l1;
  int M, K;
  int nseg;
  const int8_t* w[3];
  const int32_t* bias[3];
  int rows[3];
  nsrl_device_status* st;
};

__global__ void prefix_check_kernel(const CheckParams c) {
  __shared__ long long s_maxb;
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
  for (int m = blockIdx.x * warps + (threadIdx.x >> 5); m < c.M; m += gridDim.x * warps) {
    const long long bound = 127ll * (long long)c.l1[m] + maxb;
    if (bound <= (long long)INT_MAX) continue;
    const int8_t* ah = c.a_hi + (long long)m * c.lda;
    const uint8_t* al = c.a_lo + (long long)m * c.lda;
    for (int sg = 0; sg < c.nseg; ++sg) {
      for (int n = lane; n < c.rows[sg]; n += 32) {
        const int8_t* w = c.w[sg] + (long long)n * c.K;
        int acc = c.bias[sg] ? c.bias[sg][n] : 0;
        bool bad = false;
        for (int k = 0; k < c.K && !bad; ++k) {
          int x = (int)ah[k] * 256 + (int)al[k];
          long long t = (long long)acc + (long long)(x * (int)w[k]);
          if (t < INT_MIN || t > INT_MAX) bad = true;
          acc = (int)t;
        }
        if (bad) nsrl_flag(c.st, NSRL_FLAG_LINEAR_OVERFLOW);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Split / join between int16 rows and byte planes.
// ---------------------------------------------------------------------------
__global__ void split_planes_kernel(const int16_t* x, long long rows, int K, long long ldx, int8_t* hi, uint8_t* lo,
                                    unsigned long long* l1, long long ldp) {
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

template <int EPI, int STAGES>
cudaError_t launch_tc(const TcMaps& maps, const TcParams& p, dim3 grid, cudaStream_t stream) {
  const size_t smem = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<EPI, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  gemm_tc_kernel<EPI, STAGES><<<grid, 192, smem, stream>>>(maps, p);
  return cudaGetLastError();
}

template <int STAGES>
cudaError_t launch_tc_epi(Epi epi, const TcMaps& maps, const TcParams& p, dim3 grid, cudaStream_t stream) {
  switch (epi) {
    case Epi::I16:
      return launch_tc<(int)Epi::I16, STAGES>(maps, p, grid, stream);
    case Epi::PLANES:
      return launch_tc<(int)Epi::PLANES, STAGES>(maps, p, grid, stream);
    case Epi::RESID:
      return launch_tc<(int)Epi::RESID, STAGES>(maps, p, grid, stream);
    case Epi::GATED:
      return launch_tc<(int)Epi::GATED, STAGES>(maps, p, grid, stream);
  }
  return cudaErrorInvalidValue;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

bool tma_supported() { return encode_fn() != nullptr; }

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
  p.yh = a.yp.hi;
  p.yl = a.yp.lo;
  p.yl1 = a.yp.l1;
  p.ldp = (long long)a.yp.ld;
  p.skip = a.skip;
  p.ldskip = (long long)a.ldskip;
  p.sat = a.sat_counter;
  p.st = a.st;

  bool tc = tma_supported() && (a.K % 16) == 0 && (a.lda % 16) == 0 && aligned16(a.a_hi) && aligned16(a.a_lo);
  for (int i = 0; i < a.nseg; ++i) tc = tc && aligned16(a.seg[i].w);
  if (a.nseg == 3 && (a.seg[0].rows % BN) != 0) tc = false;
  if (a.nseg == 3 && (a.seg[1].rows != a.seg[0].rows || a.seg[2].rows != a.seg[0].rows)) tc = false;

  const double Mx = (double)a.M, Kx = (double)a.K, Nx = (double)N;
  const double nw = gated ? 2.0 * Nx : Nx;  // weight rows read
  double out_bytes = 2.0 * Mx * Nx;
  if (a.epi == Epi::RESID) out_bytes *= 2.0;  // skip read + output write
  if (a.epi == Epi::PLANES || a.epi == Epi::GATED) out_bytes += a.yp.l1 ? 8.0 * Mx : 0.0;
  static const char* names[2][4] = {{"linear_simt_i16", "linear_simt_planes", "linear_simt_resid", "linear_simt_gated"},
                                    {"linear_tc_i16", "linear_tc_planes", "linear_tc_resid", "linear_tc_gated"}};
  cudaError_t err = cudaSuccess;
  if (tc) {
    TcMaps maps;
    bool ok = make_map(&maps.a_hi, a.a_hi, a.K, a.M, a.lda, BM) && make_map(&maps.a_lo, a.a_lo, a.K, a.M, a.lda, BM);
    const uint32_t brows = gated ? BN / 2 : BN;
    for (int i = 0; i < a.nseg && ok; ++i) ok = make_map(&maps.b[i], a.seg[i].w, a.K, a.seg[i].rows, a.K, brows);
    for (int i = a.nseg; i < 3; ++i) maps.b[i] = maps.b[0];
    if (!ok) {
      tc = false;
    } else {
      const int ntn = gated ? (N + BN / 2 - 1) / (BN / 2) : (N + BN - 1) / BN;
      dim3 grid(ntn, (unsigned)((a.M + BM - 1) / BM));
      ProfScope prof(names[1][(int)a.epi], stream, 2.0 * Mx * nw * Kx, 2.0 * Mx * Kx + nw * Kx + out_bytes);
      err = (a.K <= 2 * BK) ? launch_tc_epi<2>(a.epi, maps, p, grid, stream)
                            : launch_tc_epi<4>(a.epi, maps, p, grid, stream);
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
  bool any_bias = false;
  for (int i = 0; i < a.nseg; ++i) any_bias = any_bias || a.seg[i].bias != nullptr;
  if (any_bias || (unsigned long long)a.K * 127ull * 32767ull > 2147483647ull) {
    if (!a.a_l1) return cudaErrorInvalidValue;
    CheckParams c{};
    c.a_hi = a.a_hi;
    c.a_lo = a.a_lo;
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
    unsigned blocks = (unsigned)std::min<size_t>((a.M + 7) / 8, 4096);
    ProfScope prof("linear_prefix_check", stream, 0.0, 8.0 * Mx);
    prefix_check_kernel<<<blocks, 256, 0, stream>>>(c);
    err = cudaGetLastError();
  }
  return err;
}

cudaError_t launch_split_planes(const int16_t* x, size_t rows, size_t K, size_t ldx, Planes out, cudaStream_t stream) {
  if (rows == 0 || K == 0) return cudaSuccess;
  unsigned blocks = (unsigned)std::min<size_t>((rows + 7) / 8, 148 * 16);
  ProfScope prof("split_planes", stream, 0.0, 4.0 * rows * K + 8.0 * rows);
  if (K % 8 == 0 && ldx % 8 == 0 && out.ld % 8 == 0 && aligned16(x) && (reinterpret_cast<uintptr_t>(out.hi) & 7) == 0 &&
      (reinterpret_cast<uintptr_t>(out.lo) & 7) == 0)
    split_planes_vec_kernel<<<blocks, 256, 0, stream>>>(x, (long long)rows, (int)K, (long long)ldx, out.hi, out.lo,
                                                        out.l1, (long long)out.ld);
  else
    split_planes_kernel<<<blocks, 256, 0, stream>>>(x, (long long)rows, (int)K, (long long)ldx, out.hi, out.lo, out.l1,
                                                    (long long)out.ld);
  return cudaGetLastError();
}

cudaError_t launch_join_planes(Planes in, size_t rows, size_t cols, int16_t* y, size_t ldy, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return cudaSuccess;
  long long n = (long long)rows * cols;
  unsigned blocks = (unsigned)std::min<long long>((n + 255) / 256, 148 * 32);
  ProfScope prof("join_planes", stream, 0.0, 4.0 * (double)n);
  join_planes_kernel<<<blocks, 256, 0, stream>>>(in.hi, in.lo, (long long)in.ld, (long long)rows, (int)cols, y,
                                                 (long long)ldy);
  return cudaGetLastError();
}

}  // namespace nsrl
