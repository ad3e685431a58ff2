// i64 weight-gradient accumulation on the tensor cores (tcgen05, kind::i8):
//   acc[n][k] += sum_t g'[t][n] * x[t][k]
// for the rows t of a batch: crates/nsrl-train-core/src/lib.rs:344-384 summed
// over rows (integer addition is exact in any order; i64 overflow is ruled
// out by the caller's bound).
//
// Operands are the byte planes of the row-major tensors, G [T][N] and X [T][K]
// (hi = v >> 8, s8; lo = v & 255, u8), as their producers write them; the MMAs
// read them MN-major (n and k contiguous, the reduction index t across rows),
// so nothing is transposed.
// With g = 256 gh + gl and x = 256 xh + xl,
//   g x = 65536 gh xh + 256 (gh xl + gl xh) + gl xl,
// so per 128-row block four MMAs fill three s32 TMEM accumulators:
//   hh  += xh . gh        (s8 x s8, |term| <= 16384)
//   mid += xh . gl + xl . gh  (s8 x u8 and u8 x s8, |two terms| <= 65280)
//   ll  += xl . gl        (u8 x u8, term <= 65025)
// X is the A operand (TMEM lane = k) and G the B operand (column = n), so a
// warp's 32 lanes add into 32 consecutive k of one accumulator row.
// A work item covers at most 32768 rows, so every accumulator stays below
// 2^31 and is exact.  The epilogue forms 65536 hh + 256 mid + ll in i64 and
// adds it to acc with red.global.add.u64 (two's-complement, exact).
//
// Persistent kernel, 18 warps: warp 0 issues TMA (a 3-stage ring of four
// 16 KB plane tiles of 128 rows x 128 columns), warp 1 owns TMEM and issues
// the MMAs, warps 2..17 run the epilogue (one TMEM lane quarter and 32 columns
// each).  Work items are (n tile, k tile, row chunk) triples; several CTAs add
// into one tile.
#include <algorithm>

#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int WB = 128;                  // n tile = k tile = row block
constexpr int WTILE = WB * WB;           // one plane tile, 16 KB
constexpr int WSTAGE = 4 * WTILE;        // gh, gl, xh, xl
constexpr int WSTAGES = 3;
constexpr int WEPI = 16;
constexpr int WTHREADS = 64 + 32 * WEPI;
constexpr uint32_t WTMEM = 512;          // hh [0,128), mid [128,256), ll [256,384)
constexpr size_t WSMEM = (size_t)WSTAGES * WSTAGE + 1024 + 256;

struct WgMaps {
  CUtensorMap gh, gl, xh, xl;
};

struct WgParams {
  int N, K;            // acc is [N][K]
  int tiles_k;         // K tiles
  int chunks;          // row chunks per tile
  int chunk_blocks;    // 128-row blocks per chunk
  int nblocks;         // 128-row blocks of T
  int items;
  long long* acc;
  nsrl_device_status* st;
};

// Shared-memory descriptor of an MN-major operand tile in the 128-byte
// swizzle: each 128-byte row holds 128 consecutive n (or k) of one t, 8-row
// groups 1024 B apart (stride byte offset); the tile is one 128-byte MN chunk.
__device__ __forceinline__ uint64_t sdesc_mn128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::i8 instruction descriptor with both operands MN-major.
constexpr uint32_t idesc_i8_mn(uint32_t M, uint32_t N, uint32_t a_signed, uint32_t b_signed) {
  return idesc_i8(M, N, a_signed, b_signed) | (1u << 15) | (1u << 16);
}

__device__ __forceinline__ void red_add_u64(long long* p, long long v) {
  asm volatile("red.global.add.u64 [%0], %1;" ::"l"(p), "l"((unsigned long long)v) : "memory");
}

__global__ void __launch_bounds__(WTHREADS, 1) wgrad_tc_kernel(const __grid_constant__ WgMaps maps,
                                                                const WgParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + WSTAGES * WSTAGE);
  uint64_t* empty = full + WSTAGES;
  uint64_t* acc_full = empty + WSTAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  uint32_t* skip_flag = tslot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, WEPI);
    fence_barrier_init();
    prefetch_tmap(&maps.gh);
    prefetch_tmap(&maps.gl);
    prefetch_tmap(&maps.xh);
    prefetch_tmap(&maps.xl);
  }
  if (warp == 1) {
    tmem_alloc(tslot, WTMEM);
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
    if (warp == 1) tmem_dealloc(tmem, WTMEM);
    return;
  }

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
        const int c = item % p.chunks, tile = item / p.chunks;
        const int n0 = (tile / p.tiles_k) * WB, k0 = (tile % p.tiles_k) * WB;
        const int b0 = c * p.chunk_blocks, b1 = min(p.nblocks, b0 + p.chunk_blocks);
        for (int b = b0; b < b1; ++b, ++it) {
          const int s = it % WSTAGES;
          const uint32_t ph = (it / WSTAGES) & 1;
          if (it >= WSTAGES && !mbar_wait(&empty[s], ph ^ 1, p.st)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], WSTAGE);
          uint8_t* sa = smem + s * WSTAGE;
          tma_load_2d(sa, &maps.gh, &full[s], n0, b * WB);
          tma_load_2d(sa + WTILE, &maps.gl, &full[s], n0, b * WB);
          tma_load_2d(sa + 2 * WTILE, &maps.xh, &full[s], k0, b * WB);
          tma_load_2d(sa + 3 * WTILE, &maps.xl, &full[s], k0, b * WB);
        }
      }
      // the last loads in flight land before the CTA exits
      for (uint32_t j = (it > WSTAGES ? it - WSTAGES : 0); j < it; ++j)
        mbar_wait(&full[j % WSTAGES], (j / WSTAGES) & 1, p.st);
    }
  } else if (warp == 1) {
    {  // the whole warp runs the loop (warp-uniform operands), one elected lane issues
      const uint32_t id_ss = idesc_i8_mn(WB, WB, 1, 1);
      const uint32_t id_su = idesc_i8_mn(WB, WB, 1, 0);
      const uint32_t id_us = idesc_i8_mn(WB, WB, 0, 1);
      const uint32_t id_uu = idesc_i8_mn(WB, WB, 0, 0);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < p.items && ok; item += gridDim.x, ++local) {
        const int c = item % p.chunks;
        const int b0 = c * p.chunk_blocks, b1 = min(p.nblocks, b0 + p.chunk_blocks);
        if (local > 0 && !mbar_wait(acc_empty, (local - 1) & 1, p.st)) break;
        tc_fence_after();
        for (int b = b0; b < b1; ++b, ++it) {
          const int s = it % WSTAGES;
          const uint32_t ph = (it / WSTAGES) & 1;
          if (!mbar_wait(&full[s], ph, p.st)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * WSTAGE);
#pragma unroll
          for (int j = 0; j < WB / 32; ++j) {  // 32 rows t (4 KB of each tile) per MMA
            const uint64_t gh = sdesc_mn128(base + 4096 * j);
            const uint64_t gl = sdesc_mn128(base + WTILE + 4096 * j);
            const uint64_t xh = sdesc_mn128(base + 2 * WTILE + 4096 * j);
            const uint64_t xl = sdesc_mn128(base + 3 * WTILE + 4096 * j);
            const uint32_t acc = (b > b0 || j > 0) ? 1u : 0u;
            umma_i8_warp(tmem, xh, gh, id_ss, acc);
            umma_i8_warp(tmem + WB, xh, gl, id_su, acc);
            umma_i8_warp(tmem + WB, xl, gh, id_us, 1u);
            umma_i8_warp(tmem + 2 * WB, xl, gl, id_uu, acc);
          }
          umma_commit_warp(&empty[s]);
        }
        umma_commit_warp(acc_full);
      }
    }
  } else {
    // Epilogue: warp w reads TMEM lanes [32*(w%4), +32) (k) and columns
    // [32*cg, +32) (n) of the three accumulators.
    const int q = warp & 3;
    const int cg = (warp - 2) >> 2;
    uint32_t local = 0;
    for (int item = blockIdx.x; item < p.items; item += gridDim.x, ++local) {
      const int tile = item / p.chunks;
      const int n0 = (tile / p.tiles_k) * WB, k0 = (tile % p.tiles_k) * WB;
      const int k = k0 + q * 32 + lane;
      const int nb = n0 + 32 * cg;
      if (!mbar_wait(acc_full, local & 1, p.st)) break;
      tc_fence_after();
      const uint32_t row = tmem + ((uint32_t)(q * 32) << 16) + 32 * cg;
      // two halves of 16 columns keep the three accumulators in 48 registers
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t hh[16], md[16], ll[16];
        tmem_ld16(row + 16 * half, hh);
        tmem_ld16(row + WB + 16 * half, md);
        tmem_ld16(row + 2 * WB + 16 * half, ll);
        tmem_wait_ld();
        if (half == 1) {
          tc_fence_before();
          if (lane == 0) mbar_arrive(acc_empty);
        }
        if (k < p.K) {
          long long* dst = p.acc + (long long)(nb + 16 * half) * p.K + k;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const long long v = (long long)(int)hh[i] * 65536ll + (long long)(int)md[i] * 256ll + (long long)ll[i];
            if (nb + 16 * half + i < p.N && v != 0) red_add_u64(dst + (long long)i * p.K, v);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, WTMEM);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn wg_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// uint8 [rows][inner] (row stride ld bytes), box 128 rows x 128 bytes, 128-byte swizzle.
bool wg_map(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t rows, uint64_t ld) {
  EncodeTiledFn fn = wg_encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld};
  cuuint32_t box[2] = {(cuuint32_t)WB, (cuuint32_t)WB};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// acc [N][K] += G^T X from the row-major planes G [T][N] (row stride ldg
// bytes) and X [T][K] (ldx).  Returns cudaErrorNotSupported when TMA cannot
// take them (no TMA, or a stride / base not 16-byte aligned).
cudaError_t launch_wgrad_tc(const int8_t* gh, const uint8_t* gl, size_t ldg, const int8_t* xh, const uint8_t* xl,
                            size_t ldx, size_t T, size_t N, size_t K, long long* acc, nsrl_device_status* st,
                            cudaStream_t s) {
  if (T == 0 || N == 0 || K == 0) return cudaSuccess;
  if (T > (size_t)INT32_MAX || N > (size_t)INT32_MAX || K > (size_t)INT32_MAX) return cudaErrorInvalidValue;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (ldg % 16 != 0 || ldx % 16 != 0 || !al16(gh) || !al16(gl) || !al16(xh) || !al16(xl))
    return cudaErrorNotSupported;
  WgMaps maps;
  if (!wg_map(&maps.gh, gh, N, T, ldg) || !wg_map(&maps.gl, gl, N, T, ldg) || !wg_map(&maps.xh, xh, K, T, ldx) ||
      !wg_map(&maps.xl, xl, K, T, ldx))
    return cudaErrorNotSupported;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(wgrad_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)WSMEM);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  WgParams p{};
  p.N = (int)N;
  p.K = (int)K;
  p.tiles_k = (int)((K + WB - 1) / WB);
  const int tiles = (int)((N + WB - 1) / WB) * p.tiles_k;
  p.nblocks = (int)((T + WB - 1) / WB);
  int sms = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (sms <= 0) sms = 148;
  // Rows per item: at most 32768 (exact s32 accumulators).  Items are equal,
  // so the time is about rounds x (blocks per item + one block's worth of
  // epilogue), rounds = ceil(items / SMs): take the chunking that minimises it
  // (fewer items on a tie: fewer atomic adds).
  const int max_blocks = 32768 / WB;
  int best_cb = 0;
  long long best_cost = 0;
  for (int chunks = (p.nblocks + max_blocks - 1) / max_blocks; chunks <= std::min(p.nblocks, 8 * sms); ++chunks) {
    const int cb = (p.nblocks + chunks - 1) / chunks;
    const long long items = (long long)tiles * ((p.nblocks + cb - 1) / cb);
    const long long cost = (items + sms - 1) / sms * (cb + 1);
    if (best_cb == 0 || cost < best_cost) {
      best_cb = cb;
      best_cost = cost;
    }
  }
  p.chunk_blocks = best_cb;
  p.chunks = (p.nblocks + p.chunk_blocks - 1) / p.chunk_blocks;
  p.items = tiles * p.chunks;
  p.acc = acc;
  p.st = st;
  const int grid = std::min(p.items, sms);
  ProfScope prof("accumulate_weight_grad_tc", s, 2.0 * (double)T * (double)N * (double)K,
                 2.0 * (double)T * (double)(N + K) + 16.0 * (double)N * (double)K * p.chunks);
  const cudaError_t le = launch_pdl(wgrad_tc_kernel, dim3(grid), dim3(WTHREADS), WSMEM, s, maps, p);
  if (le != cudaSuccess) return le;
  return cudaGetLastError();
}

}  // namespace nsrl
