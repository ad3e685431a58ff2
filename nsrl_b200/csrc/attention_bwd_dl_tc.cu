// Query side of the softmax-attention backward on the B200 tensor cores
// (tcgen05, kind::i8), head_dim 64, crates/nsrl-train/src/lib.rs:16623-16900,
// per (sequence, head) and query row t:
//   dP[t][j] = sat(rhu(dC[t] . V[j], 15))                                j <= t
//   w[t]     = rhu(sum_j dP[t][j] P[t][j], 15)
//   dL[t][j] = sat(rhu(P[t][j] (dP[t][j] - w[t]) 22713, 30))            j <= t
// with dL written as the causal byte planes [B*H][S][S] that the key and query
// side kernel reads (entries above the diagonal zero up to the end of each
// row's 128-key block).
//
// dC . V is i16 x i16 = (256 ch + cl)(256 vh + vl): four int8 MMAs into three
// s32 TMEM accumulators (hh, mid = ch vl + cl vh, ll), exact for a 64-dim
// dot product; dP = sat(2 hh + ((256 mid + ll + 2^14) >> 15)) in i32
// (65536 hh is a multiple of 2^15 and |256 mid + ll| < 2^31).  dP is formed
// twice, once per pass over the keys (the row sum w needs every key first),
// rather than stored to memory and read back.
//
// Persistent kernel, one CTA per SM; a work item is one 128-query tile of one
// (sequence, head), the tiles with the most keys first.  18 warps:
//   warp 0     TMA producer: the dC planes of an item (double-buffered), then
//              per 64-key tile and pass the V planes (4-stage ring) and the P
//              planes (5-stage ring)
//   warp 1     TMEM allocator + MMA issuer: per tile eight K = 32 MMAs into
//              one of two dP buffers of 3 x 64 columns
//   warps 2-17 warp w owns query rows 32 (w % 4) .. +31 (its TMEM lane
//              quarter) and keys 16 ((w - 2) / 4) .. +15 of each tile; in the
//              second pass it stages its 32 x 16 dL bytes per plane in shared
//              memory and writes them with its own TMA store
// dC, V and P tiles use the 64-byte swizzle (rows of 64 bytes), as TMA
// writes them.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int DQT = 128;  // query rows per item (MMA M)
constexpr int DKT = 64;   // keys per tile (MMA N)
constexpr int DHD = 64;   // head dim (MMA K, two K = 32 steps)
constexpr int DL_WARPS = 16;
constexpr int DTHREADS = 64 + 32 * DL_WARPS;  // 576
constexpr int VST = 4, PST = 5;                // V and P rings
constexpr int PLANE_C = DQT * DHD;             // 8 KB: [128 rows][64 dims]
constexpr int PLANE_V = DKT * DHD;             // 4 KB: [64 keys][64 dims]
constexpr int PLANE_P = DQT * DKT;             // 8 KB: [128 rows][64 keys]
constexpr int SLOT_O = 2 * 32 * 16;            // one warp's dL bytes of a tile: [plane][32 rows][16 keys]
constexpr int OFF_C = 0;                                // [2 buffers][2 planes]
constexpr int OFF_V = OFF_C + 2 * 2 * PLANE_C;          // [VST][2 planes]
constexpr int OFF_P = OFF_V + VST * 2 * PLANE_V;        // [PST][2 planes]
constexpr int OFF_O = OFF_P + PST * 2 * PLANE_P;        // [16 warps][2 slots]
constexpr int OFF_X = OFF_O + DL_WARPS * 2 * SLOT_O;    // row sums [2 items][4 key quarters][128 rows] i64
constexpr int OFF_BAR = OFF_X + 2 * 4 * DQT * 8;
constexpr size_t DSMEM = (size_t)OFF_BAR + 256 + 1024;  // + barriers, 1024-byte alignment slack
constexpr uint32_t DTMEM = 512;
constexpr uint32_t S_HH = 0, S_MID = 64, S_LL = 128, S_BUF1 = 192;

struct DlMaps {
  CUtensorMap c_hi, c_lo;  // dC planes [B][S][d], box [128 rows][64 bytes]
  CUtensorMap v_hi, v_lo;  // V planes [B][S][d], box [64 keys][64 bytes]
  CUtensorMap p_hi, p_lo;  // P planes [B*H][S][S], box [128 rows][64 keys]
  CUtensorMap l_hi, l_lo;  // dL planes [B*H][S][S], box [32 rows][16 keys] (one warp's store)
};

struct DlTcArgs {
  int S, H, B, nq, items;
  nsrl_device_status* st;
};

struct DlCtl {
  uint64_t c_full[2], c_empty[2];
  uint64_t v_full[VST], v_empty[VST];
  uint64_t p_full[PST], p_empty[PST];
  uint64_t s_full[2], s_empty[2];
  uint32_t tslot, abort;
};
static_assert(sizeof(DlCtl) <= 256, "barrier area");

// Item i: the query tile nq - 1 - i / (B H) (most keys first) of (sequence,
// head) i % (B H).
struct DlItem {
  int b, h, bh, q0, ntiles;
};
__device__ __forceinline__ DlItem dl_item(const DlTcArgs& a, int i) {
  const int per = a.B * a.H;
  DlItem it;
  it.bh = i % per;
  it.b = it.bh / a.H;
  it.h = it.bh % a.H;
  it.q0 = (a.nq - 1 - i / per) * DQT;
  const int kend = min(a.S, it.q0 + DQT);  // causal: keys below the end of the tile
  it.ntiles = (kend + DKT - 1) / DKT;
  return it;
}

// K-major tile of 64-byte rows, 64-byte swizzle: 8-row atoms 512 bytes apart.
__device__ __forceinline__ uint64_t dl_sdesc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

// A bounded wait that also ends, without waiting, once another role of the
// CTA has given up (its wait timed out), so that every role unwinds.
__device__ __forceinline__ bool dl_wait(uint64_t* bar, uint32_t parity, DlCtl* c, nsrl_device_status* st) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*reinterpret_cast<volatile uint32_t*>(&c->abort)) return false;
  if (mbar_wait(bar, parity, st)) return true;
  *reinterpret_cast<volatile uint32_t*>(&c->abort) = 1u;
  return false;
}

// Barrier of the four warps that share a TMEM lane quarter (ids 1..4).
__device__ __forceinline__ void quarter_sync(int q) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + q), "n"(128));
}

// 3-D TMA store (no multicast) of a shared-memory box to the tensor; parts
// of the box outside the tensor are not written.
__device__ __forceinline__ void dl_store_3d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// dP of 16 keys of one row from the three accumulators, before saturation:
// 2 hh + ((256 mid + ll + 2^14) >> 15), saturated to i16 in pairs later.
__device__ __forceinline__ void dp16_raw(const uint32_t (&hh)[16], const uint32_t (&mid)[16],
                                         const uint32_t (&ll)[16], int (&dp)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) dp[i] = 2 * (int)hh[i] + (((int)(mid[i] * 256u + ll[i]) + 16384) >> 15);
}

// Two-way dot products of the two i16 halves of a with two bytes of b plus c:
// bytes 0, 1 of b (lo) or 2, 3 (hi); b's bytes signed (ss) or unsigned (su).
__device__ __forceinline__ int dp2_ss_lo(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2_ss_hi(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2_su_lo(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2_su_hi(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__global__ void __launch_bounds__(DTHREADS, 1) attn_bwd_dl_tc_kernel(const __grid_constant__ DlMaps maps,
                                                                   const DlTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint32_t s_skip;
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DlCtl* ctl = reinterpret_cast<DlCtl*>(sm + OFF_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->c_full[i], 1);
      mbar_init(&ctl->c_empty[i], 1);
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->s_empty[i], DL_WARPS);
    }
    for (int i = 0; i < VST; ++i) {
      mbar_init(&ctl->v_full[i], 1);
      mbar_init(&ctl->v_empty[i], 1);
    }
    for (int i = 0; i < PST; ++i) {
      mbar_init(&ctl->p_full[i], 1);
      mbar_init(&ctl->p_empty[i], DL_WARPS);
    }
    ctl->abort = 0u;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&ctl->tslot, DTMEM);
    tmem_relinquish();
  }
  // The prologue above touches no global memory: from here on the previous
  // kernel's outputs (and the status it may have flagged) are visible.
  griddep_wait();
  if (threadIdx.x == 0) s_skip = timed_out(a.st) ? 1u : 0u;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  const uint32_t tmem = ctl->tslot;
  if (s_skip) {  // a wait of this call already timed out: do nothing
    if (warp == 1) tmem_dealloc(tmem, DTMEM);
    return;
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&maps.c_hi);
      prefetch_tmap(&maps.v_hi);
      prefetch_tmap(&maps.p_hi);
      uint32_t vi = 0, pi = 0;  // V and P loads issued
      int n = 0;                // items of this CTA
      bool ok = true;
      for (int i = blockIdx.x; i < a.items && ok; i += gridDim.x, ++n) {
        const DlItem it = dl_item(a, i);
        const int cb = n & 1;
        if (n >= 2 && !dl_wait(&ctl->c_empty[cb], ((n >> 1) - 1) & 1, ctl, a.st)) {
          ok = false;
          break;
        }
        uint8_t* cdst = sm + OFF_C + cb * 2 * PLANE_C;
        mbar_arrive_expect_tx(&ctl->c_full[cb], 2 * PLANE_C);
        tma_load_3d(cdst, &maps.c_hi, &ctl->c_full[cb], it.h * DHD, it.q0, it.b);
        tma_load_3d(cdst + PLANE_C, &maps.c_lo, &ctl->c_full[cb], it.h * DHD, it.q0, it.b);
        for (int pass = 0; pass < 2 && ok; ++pass) {
          for (int j = 0; j < it.ntiles; ++j) {
            const uint32_t vs = vi % VST;
            if (vi >= VST && !dl_wait(&ctl->v_empty[vs], ((vi / VST) - 1) & 1, ctl, a.st)) {
              ok = false;
              break;
            }
            uint8_t* vdst = sm + OFF_V + vs * 2 * PLANE_V;
            mbar_arrive_expect_tx(&ctl->v_full[vs], 2 * PLANE_V);
            tma_load_3d(vdst, &maps.v_hi, &ctl->v_full[vs], it.h * DHD, j * DKT, it.b);
            tma_load_3d(vdst + PLANE_V, &maps.v_lo, &ctl->v_full[vs], it.h * DHD, j * DKT, it.b);
            ++vi;
            const uint32_t ps = pi % PST;
            if (pi >= PST && !dl_wait(&ctl->p_empty[ps], ((pi / PST) - 1) & 1, ctl, a.st)) {
              ok = false;
              break;
            }
            uint8_t* pdst = sm + OFF_P + ps * 2 * PLANE_P;
            mbar_arrive_expect_tx(&ctl->p_full[ps], 2 * PLANE_P);
            tma_load_3d(pdst, &maps.p_hi, &ctl->p_full[ps], j * DKT, it.q0, it.bh);
            tma_load_3d(pdst + PLANE_P, &maps.p_lo, &ctl->p_full[ps], j * DKT, it.q0, it.bh);
            ++pi;
          }
        }
      }
      // Drain: every load issued lands before the CTA exits.
      for (int k = (n > 2 ? n - 2 : 0); k < n; ++k) mbar_wait(&ctl->c_full[k & 1], (k >> 1) & 1, a.st);
      for (uint32_t k = (vi > VST ? vi - VST : 0); k < vi; ++k) mbar_wait(&ctl->v_full[k % VST], (k / VST) & 1, a.st);
      for (uint32_t k = (pi > PST ? pi - PST : 0); k < pi; ++k) mbar_wait(&ctl->p_full[k % PST], (k / PST) & 1, a.st);
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    // The whole warp runs the loop (warp-uniform operands); one elected lane
    // issues each MMA and commit.
    const uint32_t id_ss = idesc_i8(DQT, DKT, 1, 1), id_su = idesc_i8(DQT, DKT, 1, 0);
    const uint32_t id_us = idesc_i8(DQT, DKT, 0, 1), id_uu = idesc_i8(DQT, DKT, 0, 0);
    uint32_t vi = 0, t = 0;  // V stages consumed, dP tiles formed (alternating buffers)
    int n = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < a.items && ok; i += gridDim.x, ++n) {
      const DlItem it = dl_item(a, i);
      const int cb = n & 1;
      if (!dl_wait(&ctl->c_full[cb], (n >> 1) & 1, ctl, a.st)) break;
      const uint32_t ch = smem_u32(sm + OFF_C + cb * 2 * PLANE_C), cl = ch + PLANE_C;
      for (int pass = 0; pass < 2 && ok; ++pass) {
        for (int j = 0; j < it.ntiles; ++j, ++vi, ++t) {
          const uint32_t vs = vi % VST, sb = t & 1, use = t >> 1;
          if (!dl_wait(&ctl->v_full[vs], (vi / VST) & 1, ctl, a.st) ||
              (use > 0 && !dl_wait(&ctl->s_empty[sb], (use - 1) & 1, ctl, a.st))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t vh = smem_u32(sm + OFF_V + vs * 2 * PLANE_V), vl = vh + PLANE_V;
          const uint32_t d = tmem + sb * S_BUF1;
#pragma unroll
          for (int ks = 0; ks < DHD / 32; ++ks) {
            const uint64_t ach = dl_sdesc(ch + 32 * ks), acl = dl_sdesc(cl + 32 * ks);
            const uint64_t bvh = dl_sdesc(vh + 32 * ks), bvl = dl_sdesc(vl + 32 * ks);
            const uint32_t acc = ks > 0 ? 1u : 0u;
            umma_i8_warp(d + S_HH, ach, bvh, id_ss, acc);
            umma_i8_warp(d + S_MID, ach, bvl, id_su, acc);
            umma_i8_warp(d + S_MID, acl, bvh, id_us, 1u);
            umma_i8_warp(d + S_LL, acl, bvl, id_uu, acc);
          }
          umma_commit_warp(&ctl->s_full[sb]);
          umma_commit_warp(&ctl->v_empty[vs]);
        }
      }
      if (ok) umma_commit_warp(&ctl->c_empty[cb]);  // the item's dC planes are free once its MMAs complete
    }
  } else {
    // --------------------------------------------------------------- dL warps
    // Every warp runs every tile of every item (a failed wait only skips the
    // arithmetic), so the four warps of a lane quarter always meet at their
    // row-sum barrier.
    const int q = warp & 3, kq = (warp - 2) >> 2;  // TMEM lane quarter, key quarter of a tile
    const int rloc = q * 32 + lane;                // row within the item
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + 16u * (uint32_t)kq;
    long long* xsum = reinterpret_cast<long long*>(sm + OFF_X);  // [item parity][key quarter][row]
    uint8_t* oslot = sm + OFF_O + (warp - 2) * 2 * SLOT_O;
    // this thread's 16-byte chunk of a P tile row (64-byte swizzle: chunk ^ ((row >> 1) & 3))
    const uint32_t pchunk = (uint32_t)rloc * 64u + ((((uint32_t)kq) ^ (((uint32_t)rloc >> 1) & 3u)) << 4);
    uint32_t t = 0, pi = 0, stores = 0, negw = 0;
    int n = 0;
    for (int i = blockIdx.x; i < a.items; i += gridDim.x, ++n) {
      const DlItem it = dl_item(a, i);
      long long wsum = 0;
      int wq = 0;
      for (int pass = 0; pass < 2; ++pass) {
        for (int j = 0; j < it.ntiles; ++j, ++t, ++pi) {
          const uint32_t sb = t & 1, ps = pi % PST;
          uint32_t hh[16], mid[16], ll[16];
          bool good = dl_wait(&ctl->s_full[sb], (t >> 1) & 1, ctl, a.st);
          tc_fence_after();
          tmem_ld16(trow + sb * S_BUF1 + S_HH, hh);
          tmem_ld16(trow + sb * S_BUF1 + S_MID, mid);
          tmem_ld16(trow + sb * S_BUF1 + S_LL, ll);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->s_empty[sb]);
          good = dl_wait(&ctl->p_full[ps], (pi / PST) & 1, ctl, a.st) && good;
          const uint8_t* pt = sm + OFF_P + ps * 2 * PLANE_P + pchunk;
          const uint4 ph = *reinterpret_cast<const uint4*>(pt), pl = *reinterpret_cast<const uint4*>(pt + PLANE_P);
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->p_empty[ps]);
          if (!good) continue;
          const int key0 = j * DKT + 16 * kq;
          // The cached P is zero above the diagonal and past the sequence: those
          // entries add nothing to the row sum and give dL = rhu(0, 30) = 0,
          // so no key needs a mask.
          int dr[16];
          dp16_raw(hh, mid, ll, dr);
          uint32_t dpk[8];  // sat(dP) of keys 2k, 2k + 1 as i16 halves
#pragma unroll
          for (int k = 0; k < 8; ++k) dpk[k] = pack_sat16(dr[2 * k + 1], dr[2 * k]);
          const uint32_t hw[4] = {ph.x, ph.y, ph.z, ph.w}, lw[4] = {pl.x, pl.y, pl.z, pl.w};
          if (pass == 0) {
            // sum dP P = 256 sum dP P_hi + sum dP P_lo over the byte planes as
            // they are (P_hi signed, P_lo unsigned): per tile |.| < 2^27
            negw |= hw[0] | hw[1] | hw[2] | hw[3];  // any negative P (the reference rejects it)
            int hs = 0, ls = 0;
#pragma unroll
            for (int k = 0; k < 8; k += 2) {
              hs = dp2_ss_lo(dpk[k], hw[k >> 1], hs);
              hs = dp2_ss_hi(dpk[k + 1], hw[k >> 1], hs);
              ls = dp2_su_lo(dpk[k], lw[k >> 1], ls);
              ls = dp2_su_hi(dpk[k + 1], lw[k >> 1], ls);
            }
            wsum += (long long)hs * 256 + ls;
            continue;
          }
          // dL = sat(rhu((22713 P) (dP - w), 30)): |22713 P| < 2^30 and |dP - w|
          // < 2^30, so the product is below 2^60 and the rounded result an i32
          uint32_t dlk[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            // P of keys 2k, 2k + 1 as i16 halves: their lo and hi bytes interleaved
            const uint32_t pp = __byte_perm(lw[k >> 1], hw[k >> 1], (k & 1) ? 0x7362 : 0x5140);
            const int p0 = (int)(int16_t)(pp & 0xFFFFu), p1 = (int)pp >> 16;
            const int d0 = (int)(int16_t)(dpk[k] & 0xFFFFu), d1 = (int)dpk[k] >> 16;
            dlk[k] = pack_sat16(rhu30_mul(p1 * 22713, d1 - wq), rhu30_mul(p0 * 22713, d0 - wq));
          }
          uint32_t ow_h[4], ow_l[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            ow_h[k] = __byte_perm(dlk[2 * k], dlk[2 * k + 1], 0x7531);  // the four hi bytes (signed)
            ow_l[k] = __byte_perm(dlk[2 * k], dlk[2 * k + 1], 0x6420);  // the four lo bytes
          }
          uint8_t* slot = oslot + (stores & 1) * SLOT_O;
          if (stores >= 2) {  // the store issued from this slot two tiles ago has read it
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
          }
          *reinterpret_cast<uint4*>(slot + lane * 16) = make_uint4(ow_h[0], ow_h[1], ow_h[2], ow_h[3]);
          *reinterpret_cast<uint4*>(slot + 512 + lane * 16) = make_uint4(ow_l[0], ow_l[1], ow_l[2], ow_l[3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            dl_store_3d(&maps.l_hi, slot, key0, it.q0 + q * 32, it.bh);
            dl_store_3d(&maps.l_lo, slot + 512, key0, it.q0 + q * 32, it.bh);
            bulk_commit();
          }
          ++stores;
        }
        if (pass == 0) {  // the row's sum over the four key quarters
          long long* xs = xsum + (n & 1) * 4 * DQT;
          xs[kq * DQT + rloc] = wsum;
          quarter_sync(q);
          const long long tot = (xs[rloc] + xs[DQT + rloc]) + (xs[2 * DQT + rloc] + xs[3 * DQT + rloc]);
          wq = (int)rhu64(tot, 15);
        }
      }
    }
    if (lane == 0) bulk_wait_all();  // this warp's stores are complete before the CTA exits
    if (negw & 0x80808080u) nsrl_flag(a.st, NSRL_FLAG_LINEAR_OVERFLOW);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, DTMEM);
}

typedef CUresult (*DlEncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                               const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

DlEncodeFn dl_encode_fn() {
  static DlEncodeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<DlEncodeFn>(p);
  }
  return fn;
}

// uint8 [n2][n1][n0] (strides s1, s2 bytes), box [1][box1][box0 bytes]: the
// 64-byte swizzle for 64-byte boxes, none for the 16-byte store boxes.  Loads
// outside the tensor read zeros; stores outside it are dropped.
bool dl_map(CUtensorMap* m, const void* ptr, uint64_t n0, uint64_t n1, uint64_t n2, uint64_t s1, uint64_t s2,
            uint32_t box0, uint32_t box1) {
  DlEncodeFn fn = dl_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {n0, n1, n2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = box0 == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_attention_bwd_dl_tc(const Planes& cp, const Planes& vp, const Planes& pp, int8_t* l_hi,
                                       uint8_t* l_lo, size_t B, size_t S, size_t d, size_t H,
                                       nsrl_device_status* st, cudaStream_t s) {
  if (H == 0 || d != (size_t)DHD * H || S % 16 != 0 || S > 16384 || !dl_encode_fn()) return cudaErrorNotSupported;
  if (B == 0 || S == 0) return cudaSuccess;
  const uint64_t BH = (uint64_t)B * H;
  DlMaps m{};
  const bool ok = dl_map(&m.c_hi, cp.hi, d, S, B, cp.ld, (uint64_t)S * cp.ld, DHD, DQT) &&
                  dl_map(&m.c_lo, cp.lo, d, S, B, cp.ld, (uint64_t)S * cp.ld, DHD, DQT) &&
                  dl_map(&m.v_hi, vp.hi, d, S, B, vp.ld, (uint64_t)S * vp.ld, DHD, DKT) &&
                  dl_map(&m.v_lo, vp.lo, d, S, B, vp.ld, (uint64_t)S * vp.ld, DHD, DKT) &&
                  dl_map(&m.p_hi, pp.hi, S, S, BH, S, (uint64_t)S * S, DKT, DQT) &&
                  dl_map(&m.p_lo, pp.lo, S, S, BH, S, (uint64_t)S * S, DKT, DQT) &&
                  dl_map(&m.l_hi, l_hi, S, S, BH, S, (uint64_t)S * S, 16, 32) &&
                  dl_map(&m.l_lo, l_lo, S, S, BH, S, (uint64_t)S * S, 16, 32);
  if (!ok) return cudaErrorNotSupported;
  static bool configured = false;
  if (!configured) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_bwd_dl_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)DSMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  DlTcArgs a{};
  a.S = (int)S;
  a.H = (int)H;
  a.B = (int)B;
  a.nq = (int)((S + DQT - 1) / DQT);
  if ((size_t)a.nq * BH > 0x7fffffffull) return cudaErrorNotSupported;
  a.items = a.nq * (int)BH;
  a.st = st;
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)std::min(a.items, sms > 0 ? sms : 148);
  const double pairs = (double)B * (double)H * (double)S * (double)(S + 1) / 2.0;
  // algorithmic: dC . V twice (2 ops per MAC); P read twice and dL written (2 bytes each per entry)
  ProfScope prof("attention_bwd_dl", s, 2.0 * 2.0 * DHD * pairs, 3.0 * 2.0 * pairs + 4.0 * (double)B * S * d);
  const cudaError_t le = launch_pdl(attn_bwd_dl_tc_kernel, dim3(grid), dim3(DTHREADS), DSMEM, s, m, a);
  if (le != cudaSuccess) return le;
  return cudaGetLastError();
}

}  // namespace nsrl
