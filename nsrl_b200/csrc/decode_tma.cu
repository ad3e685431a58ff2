// KV-cache decode attention, head_dim 64, with TMA-streamed K and V tiles.
//
// Reference: crates/nsrl-core/src/attention.rs:671-725 (one query row:
// logits, base-2 softmax :261-293, AV :596-668).
//
// One CTA per (sequence, head): warp 8 streams the head's cached K rows, then
// its V rows, as [128 keys x 64 dims] int16 tiles (16 KB) through a 4-stage
// shared-memory ring with TMA; warps 0..7 consume them.  Logits stay in
// shared memory (4 bytes per key), so K and V are each read from HBM once.
//   keys:   8 lanes per key (16 bytes = 8 dims each), dot in i64, >> 3
//   softmax: row max, LUT weights, u64 sum, Q31 reciprocal, Q15 probabilities
//   values: 32 groups of 8 lanes, each group a quarter of the tile's keys,
//           i64 accumulators, reduced across groups in shared memory
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int HD = 64, TKEYS = 128, ST = 4;
constexpr int TILE_BYTES = TKEYS * HD * 2;  // 16 KB
constexpr int CONSUMERS = 8;
constexpr int THREADS = 32 * (CONSUMERS + 1);

struct DecArgs {
  const int16_t* q;
  const int32_t* lens;
  int len_offset, Lmax, H, d;
  int head_major;  // cache [B][H][Lmax][64] instead of [B][Lmax][H*64]
  int16_t* ctx;
  nsrl_device_status* st;
};

struct DecMaps {
  CUtensorMap k, v;
};

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * CONSUMERS)); }

__global__ void __launch_bounds__(THREADS, 2) decode_tma_kernel(const __grid_constant__ DecMaps maps, const DecArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* ring = sm;                                               // ST x 16 KB
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + ST * TILE_BYTES);
  uint64_t* empty = full + ST;
  int16_t* lut = reinterpret_cast<int16_t*>(empty + ST);            // 256
  long long* red = reinterpret_cast<long long*>(lut + 256);         // [8 warps][64 dims] partial contexts
  long long* scal = red + CONSUMERS * HD;                           // [8] per-warp max / sum
  int32_t* logits = reinterpret_cast<int32_t*>(scal + 2 * CONSUMERS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x, h = blockIdx.y;
  const int L = a.lens[b] + a.len_offset;
  if (L <= 0 || L > a.Lmax) {
    if (threadIdx.x == 0) nsrl_flag(a.st, NSRL_FLAG_BAD_LENGTH);
    return;
  }
  const int ntiles = (L + TKEYS - 1) / TKEYS;
  for (int i = threadIdx.x; i < 256; i += THREADS) lut[i] = d_exp2_lut[i];
  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], CONSUMERS);
    }
    fence_barrier_init();
  }
  __syncthreads();

  // first cache row of this (sequence, head) and the head's column offset
  const int row0 = a.head_major ? (b * a.H + h) * a.Lmax : b * a.Lmax;
  const int col0 = a.head_major ? 0 : h * HD;
  if (warp == CONSUMERS) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&maps.k);
      prefetch_tmap(&maps.v);
      const int items = 2 * ntiles;
      int issued = 0;
      for (int it = 0; it < items; ++it) {
        const int s = it % ST;
        if (it >= ST && !mbar_wait(&empty[s], ((it / ST) - 1) & 1, a.st)) break;
        mbar_arrive_expect_tx(&full[s], TILE_BYTES);
        const int tile = it < ntiles ? it : it - ntiles;
        tma_load_2d(ring + s * TILE_BYTES, it < ntiles ? &maps.k : &maps.v, &full[s], col0, row0 + tile * TKEYS);
        issued = it + 1;
      }
      for (int it = (issued > ST ? issued - ST : 0); it < issued; ++it) mbar_wait(&full[it % ST], (it / ST) & 1, a.st);
    }
    return;
  }

  // ------------------------------------------------------------------ keys
  const int sub = lane & 7;  // 8 lanes per key, 8 dims each
  int qv[8];
  {
    const uint4 u = *reinterpret_cast<const uint4*>(a.q + (long long)b * a.d + h * HD + 8 * sub);
    const int16_t* e = reinterpret_cast<const int16_t*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[i] = e[i];
  }
  bool bad = false;
  long long mx = LLONG_MIN;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % ST;
    mbar_wait(&full[s], (t / ST) & 1, a.st);
    const int16_t* tile = reinterpret_cast<const int16_t*>(ring + s * TILE_BYTES);
    // warp w: keys 16w .. 16w+15 of the tile, 4 keys per pass
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int kk = 16 * warp + 4 * p + (lane >> 3);
      const uint4 u = *reinterpret_cast<const uint4*>(tile + kk * HD + 8 * sub);
      const int16_t* e = reinterpret_cast<const int16_t*>(&u);
      long long dot = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) dot += (long long)(qv[i] * (int)e[i]);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 4);
      const int key = t * TKEYS + kk;
      if (sub == 0 && key < L) {
        const long long lg = dot >> 3;
        if (lg < INT_MIN || lg > INT_MAX) bad = true;
        logits[key] = (int32_t)lg;
        if ((int32_t)lg != INT_MIN) mx = max(mx, lg);  // MASKED_LOGIT is excluded from the max
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (bad) nsrl_flag(a.st, NSRL_FLAG_LOGIT_RANGE);
  // ---------------------------------------------------------------- softmax
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) scal[warp] = mx;
  consumers_sync();
  mx = LLONG_MIN;
#pragma unroll
  for (int w = 0; w < CONSUMERS; ++w) mx = max(mx, scal[w]);
  const bool any = mx != LLONG_MIN;
  unsigned long long sum = 0;
  for (int j = threadIdx.x; j < L; j += 32 * CONSUMERS) {
    const int32_t lg = logits[j];
    const int w = (!any || lg == INT_MIN) ? 0 : exp2_neg_q15(lut, (long long)lg - mx);
    logits[j] = w;
    sum += (unsigned long long)w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  consumers_sync();  // every warp has read scal[] as the max
  if (lane == 0) scal[CONSUMERS + warp] = (long long)sum;
  consumers_sync();
  sum = 0;
#pragma unroll
  for (int w = 0; w < CONSUMERS; ++w) sum += (unsigned long long)scal[CONSUMERS + w];
  if (!any && threadIdx.x == 0) nsrl_flag(a.st, NSRL_FLAG_ALL_MASKED);
  const long long inv = any ? (long long)recip_sum_q31(sum) : 0;
  for (int j = threadIdx.x; j < L; j += 32 * CONSUMERS)
    logits[j] = (int32_t)sat_i16(rhu64((long long)logits[j] * inv, 16));
  consumers_sync();
  // ----------------------------------------------------------------- values
  // group g (32 groups of 8 lanes) takes keys g, g+32, g+64, g+96 of each tile
  // i32 accumulators are exact here: the Q15 probabilities of a row sum to
  // at most 32768 * (1 + 2^-7) + L / 2 < 2^16 for L <= 24576, so every partial
  // sum of p * v is below 2^31 in magnitude.
  const int grp = threadIdx.x >> 3;
  int acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0;
  for (int t = 0; t < ntiles; ++t) {
    const int it = ntiles + t;
    const int s = it % ST;
    mbar_wait(&full[s], (it / ST) & 1, a.st);
    const int16_t* tile = reinterpret_cast<const int16_t*>(ring + s * TILE_BYTES);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int kk = grp + 32 * p;
      const int key = t * TKEYS + kk;
      const int pr = key < L ? logits[key] : 0;
      const uint4 u = *reinterpret_cast<const uint4*>(tile + kk * HD + 8 * sub);
      const int16_t* e = reinterpret_cast<const int16_t*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] += pr * (int)e[i];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // reduce the 4 groups of a warp, then the 8 warps
#pragma unroll
  for (int o = 8; o < 32; o <<= 1)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  if (lane < 8)
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * HD + 8 * sub + i] = (long long)acc[i];
  consumers_sync();
  if (threadIdx.x < HD) {
    long long tot = 0;
#pragma unroll
    for (int w = 0; w < CONSUMERS; ++w) tot += red[w * HD + threadIdx.x];
    a.ctx[(long long)b * a.d + h * HD + threadIdx.x] = sat_i16(rhu64(tot, 15));
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

// int16 cache [rows][d], box [128 rows][64 elements], no swizzle.
bool make_cache_map(CUtensorMap* m, const int16_t* ptr, uint64_t d, uint64_t rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {d, rows};
  cuuint64_t strides[1] = {d * 2};
  cuuint32_t box[2] = {(cuuint32_t)HD, (cuuint32_t)TKEYS};
  cuuint32_t es[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<int16_t*>(ptr), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// Returns cudaErrorNotSupported when the shape is outside this kernel
// (head_dim != 64, unaligned, or too long for the shared-memory logits).
cudaError_t launch_decode_tma(const int16_t* q, const int16_t* kc, const int16_t* vc, const int32_t* lens,
                              size_t B, size_t H, size_t hd, size_t Lmax, int16_t* ctx, nsrl_device_status* st,
                              cudaStream_t stream, int len_offset, bool head_major) {
  const size_t d = H * hd;
  if (hd != (size_t)HD || (d * 2) % 16 != 0 || Lmax > 24576 || ((reinterpret_cast<uintptr_t>(kc) |
                                                                reinterpret_cast<uintptr_t>(vc)) & 15) != 0)
    return cudaErrorNotSupported;
  DecMaps m;
  const uint64_t width = head_major ? HD : d, rows = head_major ? B * H * Lmax : B * Lmax;
  if (!make_cache_map(&m.k, kc, width, rows) || !make_cache_map(&m.v, vc, width, rows)) return cudaErrorNotSupported;
  DecArgs a{q, lens, len_offset, (int)Lmax, (int)H, (int)d, head_major ? 1 : 0, ctx, st};
  const size_t smem = 128 + ST * TILE_BYTES + 2 * ST * 8 + 512 + CONSUMERS * HD * 8 + 2 * CONSUMERS * 8 +
                      4 * (((Lmax + TKEYS - 1) / TKEYS) * TKEYS);
  cudaError_t e = cudaFuncSetAttribute(decode_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const double keys = (double)B * (double)Lmax;
  ProfScope prof("attention_decode", stream, 4.0 * HD * (double)H * keys, 2.0 * 2.0 * keys * (double)d);
  decode_tma_kernel<<<dim3((unsigned)B, (unsigned)H), THREADS, smem, stream>>>(m, a);
  return cudaGetLastError();
}

}  // namespace nsrl
