// Key and query sides of the softmax-attention backward on the B200 tensor
// cores (tcgen05, kind::i8), head_dim 64, crates/nsrl-train/src/lib.rs:16623-16900:
//   dK[j] = sat(rhu(sum_{t >= j} dL[t][j] Q[t], log4 hd))
//   dV[j] = sat(rhu(sum_{t >= j} P[t][j] dC[t], 15))
//   dQ[t] = sat(rhu(sum_{j <= t} dL[t][j] K[j], log4 hd))
// per (sequence, head).  dK and dV are (S x S)^T (S x 64) products, dQ an
// (S x S) (S x 64) product; every operand is read in place from row-major
// byte planes: dL and P as [B*H][S][S] (keys contiguous; entries above the
// diagonal zero up to the end of each row's 128-key block), Q, K and dC as
// [B][S][d] (dims contiguous).  dL^T and P^T are MN-major A operands, dL a
// K-major one; Q, K and dC are MN-major B operands.  Nothing is transposed.
//
// Every product is i16 x i16 = (256 ah + al)(256 bh + bl): four int8 MMAs into
// three s32 TMEM accumulators (hh, mid = ah bl + al bh, ll); per term
// |mid| <= 65280 and ll <= 65025, so the sums are exact for up to 32768 terms
// (seq_len <= 16384).  The epilogue recombines them in i64 and applies the
// reference's rounded shift and saturation.
//
// Persistent kernel, one CTA per SM; a work item is dK or dV of one 128-key
// tile, or dQ of one 128-query tile, of one (sequence, head); items with the
// most steps first.  10 warps: warp 0 issues TMA (a 6-stage ring of 64-wide
// steps: a dL or P tile of 64 x 128 or 128 x 64 bytes per plane and a Q, K or
// dC tile of 64 x 64 bytes per plane; larger boxes, half the TMA issues of
// 32-wide steps), warp 1 owns TMEM (two accumulator sets of 3 x 64 columns)
// and issues two K = 32 sub-steps of MMAs per stage, warps 2..9 run the
// epilogue of one item while the next accumulates.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int KQ = 64;    // queries (dK, dV) or keys (dQ) per stage: two K = 32 MMA sub-steps
constexpr int KK = 128;   // keys per work item (MMA M)
constexpr int KD = 64;    // head dim (MMA N)
constexpr int KST = 6;    // stages
constexpr int TM = KQ * KK;  // 8 KB: one plane of a dL or P stage, [64 queries][128 keys] or [128 queries][64 keys]
constexpr int TX = KQ * KD;  // 4 KB: one plane of a Q, K or dC stage, [64 rows][64 dims]
constexpr int OFF_AH = 0, OFF_AL = TM, OFF_BH = 2 * TM, OFF_BL = 2 * TM + TX;
constexpr int KSTAGE = 2 * TM + 2 * TX;  // 24 KB
constexpr int KEPI = 8;                  // epilogue warps: two per TMEM lane quarter
constexpr int KTHREADS = 64 + 32 * KEPI;
constexpr uint32_t KTMEM = 512;
constexpr uint32_t ACC_COLS = 256;       // one item's hh, mid, ll (3 x 64) per buffer, two buffers
// ring + 1024-byte alignment slack + barriers (full/empty per stage, two acc
// pairs) and the TMEM slot / skip words
constexpr size_t KBAR_BYTES = (2 * KST + 4) * 8 + 8;
static_assert(KBAR_BYTES <= 512, "barrier area");
constexpr size_t KSMEM = (size_t)KST * KSTAGE + 1024 + 512;

struct KvMaps {
  CUtensorMap l_hi, l_lo, p_hi, p_lo, q_hi, q_lo, c_hi, c_lo;
  CUtensorMap lr_hi, lr_lo, k_hi, k_lo;  // dL row tiles (K-major, 128 x 64) and K, for dQ
};

struct KvArgs {
  int S, H, d, k_shift;
  int B, nk, kinds, items;
  int16_t* dk;  // int16 outputs [B*S][d] (row stride d), or NULL
  int16_t* dv;
  int16_t* dq;
  GradPlanes gk, gv, gq;  // optional prescaled planes of dK, dV, dQ ([B*S][d])
  nsrl_device_status* st;
};

// A work item is dK (kind 0) or dV (kind 1) of the 128-key tile at k0, or dQ
// (kind 2) of the 128-query tile at k0, of one (sequence, head).  Level L
// holds the key tile 128 L and the query tile 128 (nk - 1 - L): both take
// about (S - 128 L) / 64 steps, and the levels run longest first.
struct KvItem {
  int kind, h, b, k0;
  int x0, x1;  // the steps' queries (dK, dV) or keys (dQ): [x0, x1) by KQ
};
__device__ __forceinline__ KvItem kv_item(const KvArgs& a, int i) {
  const int per = a.kinds * a.B * a.H;
  const int level = i / per, r = i % per;
  KvItem it;
  it.kind = r % a.kinds;
  it.h = (r / a.kinds) % a.H;
  it.b = (r / a.kinds) / a.H;
  if (it.kind < 2) {
    it.k0 = level * KK;
    it.x0 = it.k0;  // queries t >= k0 (entries with t < j are zero)
    it.x1 = a.S;
  } else {
    it.k0 = (a.nk - 1 - level) * KK;
    it.x0 = 0;  // keys j < the end of the query tile (entries with j > t are zero)
    it.x1 = min(a.S, it.k0 + KK);
  }
  return it;
}

// K-major tile of 64-byte rows (64 keys of one query), 64-byte swizzle:
// 8-row groups 512 bytes apart; a K = 32 sub-step starts 32 bytes into the row.
__device__ __forceinline__ uint64_t sdesc_k64(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

// MN-major operand tiles: rows of 128 (keys) or 64 (dims) bytes, one per
// query; 8-row groups 1024 or 512 bytes apart (the stride byte offset).
__device__ __forceinline__ uint64_t sdesc_mn(uint32_t saddr, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(sbo >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}
constexpr uint32_t LAYOUT_SW128 = 2, LAYOUT_SW64 = 4;
constexpr uint32_t idesc_mn(uint32_t a_signed, uint32_t b_signed) {
  return idesc_i8(KK, KD, a_signed, b_signed) | (1u << 15) | (1u << 16);
}
constexpr uint32_t idesc_kmn(uint32_t a_signed, uint32_t b_signed) {  // K-major A, MN-major B
  return idesc_i8(KK, KD, a_signed, b_signed) | (1u << 16);
}

// Byte planes of 16 values of one output row, prescaled by rhu(v, shift_col).
__device__ __forceinline__ void store_planes16(const GradPlanes& gp, long long off, int col0, const int (&v)[16]) {
  int p[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) p[i] = rhu_i16(v[i], gp.sc[col0 + i].right_shift);
  uint32_t hw[4], lw[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    hw[k] = 0;
    lw[k] = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      hw[k] |= (uint32_t)((p[4 * k + e] >> 8) & 255) << (8 * e);
      lw[k] |= (uint32_t)(p[4 * k + e] & 255) << (8 * e);
    }
  }
  *reinterpret_cast<uint4*>(gp.hi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
  *reinterpret_cast<uint4*>(gp.lo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
}

// Persistent: CTA c takes items c, c + gridDim.x, ...; two TMEM accumulator
// sets, so the epilogue of one item overlaps the MMAs of the next.
__global__ void __launch_bounds__(KTHREADS, 1) attn_kv_tc_kernel(const __grid_constant__ KvMaps maps, const KvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + KST * KSTAGE);
  uint64_t* empty = full + KST;
  uint64_t* acc_full = empty + KST;    // [2]: MMA -> epilogue
  uint64_t* acc_empty = acc_full + 2;  // [2]: epilogue -> MMA
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint32_t* skip = tslot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.S;
  if (threadIdx.x == 0) *skip = timed_out(a.st) ? 1u : 0u;
  __syncthreads();
  if (*skip) return;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < KST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], KEPI);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tslot, KTMEM);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;  // steps over all items of this CTA
      bool ok = true;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x) {
        const KvItem w = kv_item(a, item);
        const int bh = w.b * a.H + w.h;
        const CUtensorMap* ma_hi = w.kind == 2 ? &maps.lr_hi : w.kind ? &maps.p_hi : &maps.l_hi;
        const CUtensorMap* ma_lo = w.kind == 2 ? &maps.lr_lo : w.kind ? &maps.p_lo : &maps.l_lo;
        const CUtensorMap* mb_hi = w.kind == 2 ? &maps.k_hi : w.kind ? &maps.c_hi : &maps.q_hi;
        const CUtensorMap* mb_lo = w.kind == 2 ? &maps.k_lo : w.kind ? &maps.c_lo : &maps.q_lo;
        for (int x = w.x0; x < w.x1; x += KQ, ++it) {
          const int s = it % KST;
          if (it >= KST && !mbar_wait(&empty[s], ((it / KST) - 1) & 1, a.st)) {
            ok = false;
            break;
          }
          uint8_t* stg = sm + s * KSTAGE;
          // A: dL / P rows x..x+31, keys k0..k0+127 (dK, dV) or rows k0..k0+127, keys x..x+31 (dQ)
          const int ac0 = w.kind == 2 ? x : w.k0, ac1 = w.kind == 2 ? w.k0 : x;
          mbar_arrive_expect_tx(&full[s], KSTAGE);
          tma_load_3d(stg + OFF_AH, ma_hi, &full[s], ac0, ac1, bh);
          tma_load_3d(stg + OFF_AL, ma_lo, &full[s], ac0, ac1, bh);
          tma_load_3d(stg + OFF_BH, mb_hi, &full[s], w.h * KD, x, w.b);
          tma_load_3d(stg + OFF_BL, mb_lo, &full[s], w.h * KD, x, w.b);
        }
      }
      // the last loads in flight land before the CTA exits
      for (uint32_t j = (it > KST ? it - KST : 0); j < it; ++j) mbar_wait(&full[j % KST], (j / KST) & 1, a.st);
    }
  } else if (warp == 1) {
    {  // the whole warp runs the loop (warp-uniform operands), one elected lane issues
      // dK: dL (s8 hi / u8 lo) x Q (s8 / u8); dV: P (hi <= 127, as u8) x dC (s8 / u8);
      // dQ: dL x K (s8 / u8), A K-major
      const uint32_t id_ss = idesc_mn(1, 1), id_su = idesc_mn(1, 0), id_us = idesc_mn(0, 1), id_uu = idesc_mn(0, 0);
      const uint32_t iq_ss = idesc_kmn(1, 1), iq_su = idesc_kmn(1, 0), iq_us = idesc_kmn(0, 1), iq_uu = idesc_kmn(0, 0);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < a.items && ok; item += gridDim.x, ++local) {
        const KvItem w = kv_item(a, item);
        const uint32_t buf = local & 1, use = local >> 1;
        if (use > 0 && !mbar_wait(&acc_empty[buf], (use - 1) & 1, a.st)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * ACC_COLS;
        const bool kq = w.kind == 2;
        const uint32_t i_hh = kq ? iq_ss : w.kind ? id_us : id_ss, i_hl = kq ? iq_su : w.kind ? id_uu : id_su;
        const uint32_t i_lh = kq ? iq_us : id_us, i_ll = kq ? iq_uu : id_uu;
        for (int x = w.x0; x < w.x1; x += KQ, ++it) {
          const int s = it % KST;
          if (!mbar_wait(&full[s], (it / KST) & 1, a.st)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(sm + s * KSTAGE);
#pragma unroll
          for (int j = 0; j < KQ / 32; ++j) {
            // sub-step j: rows 32 j .. of the MN-major tiles (4096 / 2048 bytes
            // per 32 rows), or bytes 32 j .. of the K-major dL rows
            const uint64_t ah = kq ? sdesc_k64(base + OFF_AH + 32 * j)
                                   : sdesc_mn(base + OFF_AH + 4096 * j, 1024, LAYOUT_SW128);
            const uint64_t al = kq ? sdesc_k64(base + OFF_AL + 32 * j)
                                   : sdesc_mn(base + OFF_AL + 4096 * j, 1024, LAYOUT_SW128);
            const uint64_t bhd = sdesc_mn(base + OFF_BH + 2048 * j, 512, LAYOUT_SW64);
            const uint64_t bld = sdesc_mn(base + OFF_BL + 2048 * j, 512, LAYOUT_SW64);
            const uint32_t acc = (x > w.x0 || j > 0) ? 1u : 0u;
            umma_i8_warp(d, ah, bhd, i_hh, acc);            // hh
            umma_i8_warp(d + 64, ah, bld, i_hl, acc);       // mid: hi x lo
            umma_i8_warp(d + 64, al, bhd, i_lh, 1u);        //      lo x hi
            umma_i8_warp(d + 128, al, bld, i_ll, acc);      // ll
          }
          umma_commit_warp(&empty[s]);
        }
        umma_commit_warp(&acc_full[buf]);
      }
    }
  } else {
    // Epilogue: warp w reads TMEM lanes [32 (w % 4), +32) (key j, or query t
    // for dQ, of the item) and dims [32 g, 32 g + 32), g = (w - 2) / 4.
    const int q = warp & 3, g = (warp - 2) >> 2;
    uint32_t local = 0;
    for (int item = blockIdx.x; item < a.items; item += gridDim.x, ++local) {
      const KvItem w = kv_item(a, item);
      const uint32_t buf = local & 1, use = local >> 1;
      if (!mbar_wait(&acc_full[buf], use & 1, a.st)) break;
      tc_fence_after();
      const int j = w.k0 + q * 32 + lane;
      const uint32_t row = tmem + buf * ACC_COLS + ((uint32_t)(q * 32) << 16);
      const uint32_t shift = w.kind == 1 ? 15u : (uint32_t)a.k_shift;
      int16_t* out = w.kind == 2 ? a.dq : w.kind ? a.dv : a.dk;
      const GradPlanes& gp = w.kind == 2 ? a.gq : w.kind ? a.gv : a.gk;
      const long long orow = ((long long)w.b * S + j) * a.d + (long long)w.h * KD;
#pragma unroll
      for (int c = 32 * g; c < 32 * g + 32; c += 16) {
        uint32_t hh[16], md[16], lw[16];
        tmem_ld16(row + c, hh);
        tmem_ld16(row + 64 + c, md);
        tmem_ld16(row + 128 + c, lw);
        tmem_wait_ld();
        if (c == 32 * g + 16) {  // both chunks loaded: the buffer may take the next item
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        if (j >= S) continue;
        int v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const long long tot = (long long)(int)hh[i] * 65536 + (long long)(int)md[i] * 256 + (long long)(int)lw[i];
          v[i] = (int)sat_i16(rhu64(tot, shift));
        }
        const long long off = orow + c;
        if (out) {
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) pk[i] = __byte_perm((uint32_t)v[2 * i], (uint32_t)v[2 * i + 1], 0x5410);
          uint4* dst = reinterpret_cast<uint4*>(out + off);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
        if (gp.hi) store_planes16(gp, off, w.h * KD + c, v);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, KTMEM);
  }
}

// Row t of an S x S matrix (int16, [BH][S][S]) -> byte planes of columns
// j < the end of t's 128-column block, entries above the diagonal (j > t)
// written as zeros: the region the key-side kernel reads, causal-masked.
// A CTA of 64 x 4 threads covers 4 rows (threadIdx.y) of the B*H*S rows,
// eight columns per thread and step; S % 8 == 0.
__global__ void __launch_bounds__(256) split_causal_kernel(const int16_t* __restrict__ M, long long rows, int S,
                                                           int8_t* __restrict__ hi, uint8_t* __restrict__ lo) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  const long long rid = (long long)blockIdx.x * 4 + threadIdx.y;  // bh * S + t
  if (rid >= rows) return;
  const int c8 = S / 8;
  {
    const int t = (int)(rid % S);
    const int jend = min(S, (t / KK + 1) * KK);  // past it the kernel reads nothing
    const long long rowoff = rid * (long long)S;
    for (int c = threadIdx.x; c < c8 && 8 * c < jend; c += 64) {
      const int j0 = 8 * c;
      int v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (j0 <= t) {
        unpack8(*reinterpret_cast<const uint4*>(M + rowoff + j0), v);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (j0 + e > t) v[e] = 0;
      }
      uint2 h, l;
      planes8(v, h, l);
      *reinterpret_cast<uint2*>(hi + rowoff + j0) = h;
      *reinterpret_cast<uint2*>(lo + rowoff + j0) = l;
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn kv_encode_fn() {
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

// uint8 [n2][n1][n0] (strides s1, s2 bytes), box [1][box1 rows][box0 bytes]
// (box0 = 128, 64 or 32) with the swizzle of the row width; rows past n1 and
// columns past n0 (the sequence) read zeros.
bool kv_map(CUtensorMap* m, const void* ptr, uint64_t n0, uint64_t n1, uint64_t n2, uint64_t s1, uint64_t s2,
            uint32_t box0, uint32_t box1 = KQ) {
  EncodeTiledFn fn = kv_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {n0, n1, n2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = box0 == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : box0 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                             : CU_TENSOR_MAP_SWIZZLE_32B;
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool attention_kv_tc_supported(size_t S, size_t d, size_t H) {
  return H != 0 && d == 64 * H && S % 16 == 0 && S <= 16384 && kv_encode_fn() != nullptr;
}

cudaError_t launch_split_causal(const int16_t* M, size_t BH, size_t S, int8_t* hi, uint8_t* lo, cudaStream_t s) {
  if (BH == 0 || S == 0) return cudaSuccess;
  const size_t rows = BH * S;
  if (S % 8 != 0 || (rows + 3) / 4 > 0x7fffffffull) return cudaErrorInvalidValue;
  ProfScope prof("attention_bwd_split", s, 0.0, 2.0 * (double)BH * S * S);
  const cudaError_t le =
      launch_pdl(split_causal_kernel, dim3((unsigned)((rows + 3) / 4)), dim3(64, 4), 0, s, M, (long long)rows, (int)S, hi, lo);
  if (le != cudaSuccess) return le;
  return cudaGetLastError();
}

cudaError_t launch_attention_kv_tc(const Planes& l, const Planes& p, const Planes& qp, const Planes& cp, size_t B,
                                   size_t S, size_t d, size_t H, int16_t* dk, int16_t* dv, const GradPlanes& gk,
                                   const GradPlanes& gv, nsrl_device_status* st, cudaStream_t s, const Planes* kp,
                                   int16_t* dq, const GradPlanes& gq) {
  if (!attention_kv_tc_supported(S, d, H)) return cudaErrorNotSupported;
  if (B == 0) return cudaSuccess;
  KvMaps m{};
  const uint64_t BH = (uint64_t)B * H;
  const bool ok = kv_map(&m.l_hi, l.hi, S, S, BH, S, (uint64_t)S * S, KK) &&
                  kv_map(&m.l_lo, l.lo, S, S, BH, S, (uint64_t)S * S, KK) &&
                  kv_map(&m.p_hi, p.hi, S, S, BH, S, (uint64_t)S * S, KK) &&
                  kv_map(&m.p_lo, p.lo, S, S, BH, S, (uint64_t)S * S, KK) &&
                  kv_map(&m.q_hi, qp.hi, d, S, B, qp.ld, (uint64_t)S * qp.ld, KD) &&
                  kv_map(&m.q_lo, qp.lo, d, S, B, qp.ld, (uint64_t)S * qp.ld, KD) &&
                  kv_map(&m.c_hi, cp.hi, d, S, B, cp.ld, (uint64_t)S * cp.ld, KD) &&
                  kv_map(&m.c_lo, cp.lo, d, S, B, cp.ld, (uint64_t)S * cp.ld, KD) &&
                  (!kp || (kv_map(&m.lr_hi, l.hi, S, S, BH, S, (uint64_t)S * S, KQ, KK) &&
                           kv_map(&m.lr_lo, l.lo, S, S, BH, S, (uint64_t)S * S, KQ, KK) &&
                           kv_map(&m.k_hi, kp->hi, d, S, B, kp->ld, (uint64_t)S * kp->ld, KD) &&
                           kv_map(&m.k_lo, kp->lo, d, S, B, kp->ld, (uint64_t)S * kp->ld, KD)));
  if (!ok) return cudaErrorNotSupported;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_kv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)KSMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  KvArgs a{};
  a.S = (int)S;
  a.H = (int)H;
  a.d = (int)d;
  a.k_shift = 3;  // log4(64)
  a.B = (int)B;
  a.nk = (int)((S + KK - 1) / KK);
  a.kinds = kp ? 3 : 2;
  if ((size_t)a.kinds * B * H * a.nk > 0x7fffffffull) return cudaErrorNotSupported;
  a.items = a.kinds * a.B * a.H * a.nk;
  a.dk = dk;
  a.dv = dv;
  a.dq = dq;
  a.gk = gk;
  a.gv = gv;
  a.gq = gq;
  a.st = st;
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)std::min(a.items, sms > 0 ? sms : 148);
  const double pairs = (double)B * (double)H * (double)S * (double)(S + 1) / 2.0;
  ProfScope prof(kp ? "attention_bwd_qkv" : "attention_bwd_kv", s, a.kinds * 2.0 * 64.0 * pairs,
                 a.kinds * 2.0 * pairs + 4.0 * a.kinds * (double)B * S * d);
  attn_kv_tc_kernel<<<grid, KTHREADS, KSMEM, s>>>(m, a);
  return cudaGetLastError();
}

}  // namespace nsrl
