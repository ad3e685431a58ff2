// Data-parallel training exchange: i64 weight-gradient accumulation and the
// requantising apply into i8 weights.
//
// Reference: crates/nsrl-train-core/src/lib.rs:344-384
// (accumulate_linear_weight_gradient_i64_prescaled), :386-465
// (apply_linear_weight_gradient_i64_to_i8), :1732-1775 (rounding helpers).
//
// accumulate: acc[n][k] += g[r][n] * x[r][k] over rows r, with checked i64
//   adds in row order (zero terms skipped), sample_count += 1 per row.  The
//   sums are order-independent; overflow is not.  A bound kernel first checks
//   max|acc| + sum_r max_n|g[r][n]| * max_k|x[r][k]| <= i64::MAX, which
//   rules out every prefix overflow; only if it fails does a sequential
//   kernel replay each element's additions in reference order.
// apply: per weight, avg = round_div(acc, count) (half away from zero),
//   product = avg * lr (+ residual), u = rhu(product, shift), residual' =
//   product - (u << shift), w = sat_i8(w - u) (residual := 0 on saturation);
//   zero sums are skipped; stats = {saturations, zero deltas, sum |dw|}; then
//   the accumulators and the count are cleared.
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

// a + b with a signed-overflow flag (two's complement wrap, then sign test).
__device__ __forceinline__ bool add_ovf(long long a, long long b, long long& out) {
  const long long s = (long long)((unsigned long long)a + (unsigned long long)b);
  out = s;
  return ((a ^ s) & (b ^ s)) < 0;
}

// a * b with a signed-overflow flag: the high 64 bits of the 128-bit product
// must be the sign extension of the low 64 bits.
__device__ __forceinline__ bool mul_ovf(long long a, long long b, long long& out) {
  const long long lo = (long long)((unsigned long long)a * (unsigned long long)b);
  const long long hi = __mul64hi(a, b);
  out = lo;
  return hi != (lo >> 63);
}

constexpr int TN = 64, TK = 64, TR = 32;  // output tile and row chunk of the accumulation

// acc[n][k] += sum_r g[r][n] * x[r][k]: 256 threads, 4 x 4 outputs each.
__global__ void __launch_bounds__(256) accumulate_kernel(const int16_t* __restrict__ x, const int32_t* __restrict__ g,
                                                         int rows, int K, int N, long long* __restrict__ acc) {
  __shared__ int32_t sg[TR][TN];
  __shared__ int32_t sx[TR][TK + 1];
  const int n0 = blockIdx.y * TN, k0 = blockIdx.x * TK;
  const int tn = threadIdx.x / 16, tk = threadIdx.x % 16;
  long long c[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0;
  for (int r0 = 0; r0 < rows; r0 += TR) {
    for (int i = threadIdx.x; i < TR * TN; i += 256) {
      const int rr = i / TN, nn = i % TN;
      sg[rr][nn] = (r0 + rr < rows && n0 + nn < N) ? g[(long long)(r0 + rr) * N + n0 + nn] : 0;
    }
    for (int i = threadIdx.x; i < TR * TK; i += 256) {
      const int rr = i / TK, kk = i % TK;
      sx[rr][kk] = (r0 + rr < rows && k0 + kk < K) ? (int)x[(long long)(r0 + rr) * K + k0 + kk] : 0;
    }
    __syncthreads();
#pragma unroll 4
    for (int rr = 0; rr < TR; ++rr) {
      long long gv[4];
      int xv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) gv[i] = sg[rr][tn + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) xv[j] = sx[rr][tk + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) c[i][j] += gv[i] * xv[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = n0 + tn + 16 * i;
    if (n >= N) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + tk + 16 * j;
      if (k < K) acc[(long long)n * K + k] += c[i][j];
    }
  }
}

// Overflow bound of an accumulation call (see the file comment), reduced
// over the grid into bound[0] (sum, double) and bound[1] (max |acc|, u64).
__global__ void accumulate_bound_kernel(const int16_t* x, const int32_t* g, int rows, int K, int N,
                                        const long long* acc, long long len, double* sum_out,
                                        unsigned long long* max_out) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  double sum = 0.0;
  // one warp per row: max_n |g[r][n]| * max_k |x[r][k]|
  for (int r = blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += gridDim.x * warps) {
    long long gm = 0;
    int xm = 0;
    for (int n = lane; n < N; n += 32) gm = max(gm, llabs((long long)g[(long long)r * N + n]));
    for (int k = lane; k < K; k += 32) xm = max(xm, abs((int)x[(long long)r * K + k]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      gm = max(gm, __shfl_xor_sync(0xffffffffu, gm, o));
      xm = max(xm, __shfl_xor_sync(0xffffffffu, xm, o));
    }
    if (lane == 0) sum += (double)gm * (double)xm;
  }
  unsigned long long am = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (long long)gridDim.x * blockDim.x) {
    const long long v = acc[i];
    am = max(am, v == LLONG_MIN ? (unsigned long long)LLONG_MAX + 1ull : (unsigned long long)llabs(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) am = max(am, __shfl_xor_sync(0xffffffffu, am, o));
  if (lane == 0) {
    if (sum != 0.0) atomicAdd(sum_out, sum);
    if (am) atomicMax(max_out, am);
  }
}

// Decides whether the exact replay is needed and adds `rows` to the count.
__global__ void accumulate_bound_finish_kernel(const double* sum, const unsigned long long* mx, int rows,
                                               unsigned long long* count, int* needs_exact) {
  // 2^62 leaves margin for the rounding of the double sum.
  *needs_exact = (*sum + (double)*mx >= 4611686018427387904.0) ? 1 : 0;
  *count += (unsigned long long)rows;
}

// Reference-order replay of every element's additions (only when the bound
// failed): rows in order, checked i64 adds; the sum itself is left to
// accumulate_kernel.
__global__ void accumulate_exact_check_kernel(const int16_t* x, const int32_t* g, int rows, int K, int N,
                                              const long long* acc_before, const int* needs_exact,
                                              nsrl_device_status* st) {
  if (!*needs_exact) return;
  const long long total = (long long)N * K;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i / K), k = (int)(i % K);
    long long a = acc_before[i];
    for (int r = 0; r < rows; ++r) {
      const long long p = (long long)g[(long long)r * N + n] * (long long)x[(long long)r * K + k];
      long long s;
      if (add_ovf(a, p, s)) {
        nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
        break;
      }
      a = s;
    }
  }
}

// train-core lib.rs:1732-1757 for den > 0; false on i64 overflow.
__device__ __forceinline__ bool round_div(long long num, long long den, long long& out) {
  const long long half = den / 2;
  if (num >= 0) {
    if (num > LLONG_MAX - half) return false;
    out = (num + half) / den;
  } else {
    if (num == LLONG_MIN) return false;
    const long long m = -num;
    if (m > LLONG_MAX - half) return false;
    out = -((m + half) / den);
  }
  return true;
}

__global__ void apply_kernel(long long* __restrict__ acc, long long* __restrict__ res, int8_t* __restrict__ w,
                             long long len, const unsigned long long* count_p, int lr, int shift, int carry,
                             unsigned long long* stats, nsrl_device_status* st) {
  const unsigned long long count = *count_p;
  if (count == 0) return;  // nothing accumulated: weights, residuals and accumulators untouched
  if (count > (unsigned long long)LLONG_MAX) {
    if (blockIdx.x == 0 && threadIdx.x == 0) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
    return;
  }
  const long long den = (long long)count;
  unsigned long long sat = 0, zero = 0, l1 = 0;
  bool bad = false;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (long long)gridDim.x * blockDim.x) {
    const long long raw = acc[i];
    acc[i] = 0;
    if (raw == 0) continue;
    long long avg;
    if (!round_div(raw, den, avg)) {
      bad = true;
      continue;
    }
    long long product;
    if (mul_ovf(avg, (long long)lr, product)) {
      bad = true;
      continue;
    }
    if (carry && add_ovf(product, res[i], product)) {
      bad = true;
      continue;
    }
    const long long scaled = rhu64(product, (uint32_t)shift);
    long long next_res = 0;
    if (carry && shift != 0) {
      // product - (scaled << shift): scaled = rhu(product, shift) (saturating
      // add), so scaled << shift stays in i64 and the difference is at most
      // 2^(shift-1) in magnitude; the reference's i128 check never fails.
      next_res = (long long)((unsigned long long)product - ((unsigned long long)scaled << shift));
    }
    const long long delta = -scaled;
    if (delta == 0) ++zero;
    const int prev = w[i];
    long long unclamped;
    if (add_ovf((long long)prev, delta, unclamped)) {
      bad = true;
      continue;
    }
    const int clamped = (int)sat_i8(unclamped);
    if ((long long)clamped != unclamped) {
      ++sat;
      res[i] = 0;
    } else {
      res[i] = next_res;
    }
    l1 += (unsigned long long)abs(clamped - prev);
    w[i] = (int8_t)clamped;
  }
  if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sat += __shfl_xor_sync(0xffffffffu, sat, o);
    zero += __shfl_xor_sync(0xffffffffu, zero, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if ((threadIdx.x & 31) == 0) {
    if (sat) atomicAdd(&stats[0], sat);
    if (zero) atomicAdd(&stats[1], zero);
    if (l1) atomicAdd(&stats[2], l1);
  }
}

// nsrl-train/src/lib.rs:14457-14510 (apply_embedding_accumulators_i64_to_i16):
// unlike the i8 apply, an entry is skipped only when both its sum and its
// residual are zero, the residual is always carried (also on saturation),
// and the accumulators are left for the caller to clear.
__global__ void apply_embedding_kernel(const long long* __restrict__ acc, long long* __restrict__ res,
                                       int16_t* __restrict__ w, long long len, const unsigned long long* count_p,
                                       int lr, int shift, unsigned long long* stats, nsrl_device_status* st) {
  const unsigned long long count = *count_p;
  if (count == 0) return;
  if (count > (unsigned long long)LLONG_MAX) {
    if (blockIdx.x == 0 && threadIdx.x == 0) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
    return;
  }
  const long long den = (long long)count;
  unsigned long long sat = 0, zero = 0, l1 = 0;
  bool bad = false;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (long long)gridDim.x * blockDim.x) {
    const long long raw = acc[i], r0 = res[i];
    if (raw == 0 && r0 == 0) continue;
    long long avg, product;
    if (!round_div(raw, den, avg) || mul_ovf(avg, (long long)lr, product) || add_ovf(product, r0, product)) {
      bad = true;
      continue;
    }
    const long long scaled = rhu64(product, (uint32_t)shift);
    // product - (scaled << shift), exact as in the i8 apply
    res[i] = shift ? (long long)((unsigned long long)product - ((unsigned long long)scaled << shift)) : 0;
    const long long delta = -scaled;
    if (delta == 0) ++zero;
    const int prev = w[i];
    long long unclamped;
    if (add_ovf((long long)prev, delta, unclamped)) {
      bad = true;
      continue;
    }
    const int clamped = (int)sat_i16(unclamped);
    if ((long long)clamped != unclamped) ++sat;
    l1 += (unsigned long long)abs(clamped - prev);
    w[i] = (int16_t)clamped;
  }
  if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sat += __shfl_xor_sync(0xffffffffu, sat, o);
    zero += __shfl_xor_sync(0xffffffffu, zero, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if ((threadIdx.x & 31) == 0) {
    if (sat) atomicAdd(&stats[0], sat);
    if (zero) atomicAdd(&stats[1], zero);
    if (l1) atomicAdd(&stats[2], l1);
  }
}

// average_i8_movement / average_i16_movement (nsrl-train/src/lib.rs:14552-14583):
// w = sat(base + round_div(w - base, divisor)), half away from zero.
template <class W>
__global__ void average_movement_kernel(const W* __restrict__ base, W* __restrict__ w, long long len, long long div,
                                        int lo, int hi) {
  const long long half = div / 2;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (long long)gridDim.x * blockDim.x) {
    const long long b = base[i], m = (long long)w[i] - b;  // |m| < 2^17: no overflow anywhere
    const long long avg = m >= 0 ? (m + half) / div : -((-m + half) / div);
    const long long v = b + avg;
    w[i] = (W)(v < lo ? lo : (v > hi ? hi : v));
  }
}

// ---------------------------------------------------------- integer Adam --
// crates/nsrl-train-core/src/lib.rs:602-661 (integer_adam_delta) with the
// reference's i128 intermediates as __int128.  Returns false on a rejection.
struct AdamCfg {
  int lr;
  int step_shift, b1, b2;
  unsigned long long eps;
};

__device__ __forceinline__ bool rhu128_i64(__int128 v, int s, long long& out) {
  if (s) v += (__int128)1 << (s - 1);  // |v| < 2^127 - 2^61 here: no overflow
  v >>= s;
  if (v < (__int128)LLONG_MIN || v > (__int128)LLONG_MAX) return false;
  out = (long long)v;
  return true;
}

__device__ __forceinline__ bool adam_delta(long long g, const AdamCfg& c, long long& m1, unsigned long long& m2,
                                           long long& res, long long& delta, bool& sat) {
  const long long lim = 2147483647ll;
  const long long bg = g < -lim ? -lim : (g > lim ? lim : g);
  sat = bg != g;
  // |m1| < 2^63 and 2^b1 - 1 < 2^62: the product stays below 2^125
  if (!rhu128_i64((__int128)m1 * (((__int128)1 << c.b1) - 1) + bg, c.b1, m1)) return false;
  __int128 n2 = (__int128)m2 * (((__int128)1 << c.b2) - 1) + (__int128)bg * bg;  // < 2^126 + 2^62
  if (c.b2) n2 += (__int128)1 << (c.b2 - 1);
  n2 >>= c.b2;
  if (n2 < 0 || n2 > (__int128)0xFFFFFFFFFFFFFFFFull) return false;
  m2 = (unsigned long long)n2;
  const unsigned long long var = m2 + c.eps;
  if (var < m2) return false;  // u64 overflow: the reference's checked_add
  const long long inv = rsqrt_q30(var);
  long long n15;
  if (!rhu128_i64((__int128)m1 * inv, 15, n15)) return false;
  n15 = n15 < -32767 ? -32767 : (n15 > 32767 ? 32767 : n15);
  long long num;
  if (mul_ovf(n15, (long long)c.lr, num) || add_ovf(num, res, num)) return false;
  const int eff = 15 + c.step_shift;
  const long long scaled = rhu64(num, (uint32_t)eff);
  const __int128 r = (__int128)num - ((__int128)scaled << eff);
  if (r < (__int128)LLONG_MIN || r > (__int128)LLONG_MAX) return false;
  res = (long long)r;
  delta = -scaled;
  return true;
}

// apply_integer_adam_accumulators_i64_to_i8 / _to_i16 (lib.rs:469-593):
// weights W (int8 or int16) clamped to [lo, hi]; stats added to; the step
// advances once per call with a nonzero sample count.
template <class W>
__global__ void adam_kernel(const long long* __restrict__ acc, const unsigned long long* count_p, W* __restrict__ w,
                            long long len, AdamCfg c, long long* __restrict__ m1, unsigned long long* __restrict__ m2,
                            long long* __restrict__ res, unsigned long long* step, unsigned long long* stats, int lo,
                            int hi, nsrl_device_status* st) {
  const unsigned long long count = *count_p;
  if (count == 0) return;
  if (count > (unsigned long long)LLONG_MAX) {
    if (blockIdx.x == 0 && threadIdx.x == 0) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
    return;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(step, 1ull);
  const long long den = (long long)count;
  unsigned long long sat = 0, zero = 0, l1 = 0;
  bool bad = false;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += (long long)gridDim.x * blockDim.x) {
    long long g, a = m1[i], r = res[i], delta;
    unsigned long long b = m2[i];
    bool gs;
    if (!round_div(acc[i], den, g) || !adam_delta(g, c, a, b, r, delta, gs)) {
      bad = true;
      continue;
    }
    sat += gs;
    zero += delta == 0;
    const long long prev = w[i];
    long long un;
    if (add_ovf(prev, delta, un)) {
      bad = true;
      continue;
    }
    const long long cl = un < lo ? lo : (un > hi ? hi : un);
    if (cl != un) {
      ++sat;
      r = 0;
    }
    l1 += (unsigned long long)(cl > prev ? cl - prev : prev - cl);
    w[i] = (W)cl;
    m1[i] = a;
    m2[i] = b;
    res[i] = r;
  }
  if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sat += __shfl_xor_sync(0xffffffffu, sat, o);
    zero += __shfl_xor_sync(0xffffffffu, zero, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  if ((threadIdx.x & 31) == 0) {
    if (sat) atomicAdd(&stats[0], sat);
    if (zero) atomicAdd(&stats[1], zero);
    if (l1) atomicAdd(&stats[2], l1);
  }
}

template <class W>
nsrl_status launch_adam(const long long* acc, const unsigned long long* count, W* w, size_t len,
                        const nsrl_integer_adam_config* cfg, long long* m1, unsigned long long* m2, long long* res,
                        unsigned long long* step, unsigned long long* stats, int lo, int hi, nsrl_device_status* st,
                        void* stream, const char* name) {
  // lib.rs:299-309 (is_valid) and the shape rule of :476-478
  if (!cfg || cfg->learning_rate <= 0 || cfg->beta1_decay_shift == 0 || cfg->beta2_decay_shift == 0 ||
      cfg->beta1_decay_shift > 62 || cfg->beta2_decay_shift > 62 || cfg->step_shift > 62 - 15 || cfg->epsilon == 0 ||
      len == 0 || !acc || !count || !w || !m1 || !m2 || !res || !step || !stats || !st) {
    set_error("invalid config or shape: integer Adam");
    return NSRL_INVALID_SHAPE;
  }
  AdamCfg c{cfg->learning_rate, cfg->step_shift, cfg->beta1_decay_shift, cfg->beta2_decay_shift, cfg->epsilon};
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned blocks = (unsigned)std::min<size_t>((len + 255) / 256, 148 * 8);
  ProfScope prof(name, s, 0.0, (8.0 + 8.0 + 8.0 + 8.0 + 8.0 + 8.0 + 2.0 * sizeof(W)) * (double)len);
  adam_kernel<W><<<blocks, 256, 0, s>>>(acc, count, w, (long long)len, c, m1, m2, res, step, stats, lo, hi, st);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("integer Adam: %s", cudaGetErrorString(e));
    return NSRL_CUDA_ERROR;
  }
  return NSRL_OK;
}

}  // namespace
}  // namespace nsrl

using namespace nsrl;

extern "C" {

size_t nsrl_accumulate_workspace_size(size_t input_dim, size_t output_dim) {
  return 256 + ((input_dim * output_dim * sizeof(long long) + 255) & ~size_t(255));
}

nsrl_status nsrl_accumulate_linear_weight_gradient_i64(const int16_t* x, const int32_t* scaled_grad, size_t rows,
                                                       size_t input_dim, size_t output_dim, long long* accumulators,
                                                       unsigned long long* sample_count, void* workspace,
                                                       size_t workspace_bytes, nsrl_device_status* status,
                                                       void* stream) {
  if (input_dim == 0 || output_dim == 0 || !accumulators || !sample_count || !status) {
    set_error("invalid shape: accumulate");
    return NSRL_INVALID_SHAPE;
  }
  if (rows > (size_t)INT32_MAX || input_dim > (size_t)INT32_MAX || output_dim > (size_t)INT32_MAX) {
    set_error("invalid shape: dimension too large");
    return NSRL_INVALID_SHAPE;
  }
  if (rows == 0) return NSRL_OK;
  if (!workspace || workspace_bytes < nsrl_accumulate_workspace_size(input_dim, output_dim)) {
    set_error("invalid shape: workspace too small");
    return NSRL_INVALID_SHAPE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* needs_exact = reinterpret_cast<int*>(ws);
  double* bsum = reinterpret_cast<double*>(ws + 8);
  unsigned long long* bmax = reinterpret_cast<unsigned long long*>(ws + 16);
  long long* before = reinterpret_cast<long long*>(ws + 256);
  const long long len = (long long)input_dim * (long long)output_dim;
  cudaError_t e = cudaMemsetAsync(ws, 0, 32, s);
  if (e != cudaSuccess) goto fail;
  {
    ProfScope prof("accumulate_bound", s, 0.0, 2.0 * rows * input_dim + 4.0 * rows * output_dim + 8.0 * len);
    accumulate_bound_kernel<<<148 * 4, 256, 0, s>>>(x, scaled_grad, (int)rows, (int)input_dim, (int)output_dim,
                                                    accumulators, len, bsum, bmax);
    accumulate_bound_finish_kernel<<<1, 1, 0, s>>>(bsum, bmax, (int)rows, sample_count, needs_exact);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) goto fail;
  e = cudaMemcpyAsync(before, accumulators, len * sizeof(long long), cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) goto fail;
  {
    dim3 grid((unsigned)((input_dim + TK - 1) / TK), (unsigned)((output_dim + TN - 1) / TN));
    ProfScope prof("accumulate_i64", s, 2.0 * rows * input_dim * output_dim,
                   2.0 * rows * input_dim + 4.0 * rows * output_dim + 16.0 * len);
    accumulate_kernel<<<grid, 256, 0, s>>>(x, scaled_grad, (int)rows, (int)input_dim, (int)output_dim, accumulators);
  }
  if ((e = cudaGetLastError()) != cudaSuccess) goto fail;
  accumulate_exact_check_kernel<<<148 * 4, 256, 0, s>>>(x, scaled_grad, (int)rows, (int)input_dim,
                                                        (int)output_dim, before, needs_exact, status);
  if ((e = cudaGetLastError()) != cudaSuccess) goto fail;
  return NSRL_OK;
fail:
  set_error("accumulate: %s", cudaGetErrorString(e));
  return NSRL_CUDA_ERROR;
}

nsrl_status nsrl_apply_linear_weight_gradient_i64_to_i8(long long* accumulators, long long* residuals, int8_t* weights,
                                                        size_t len, unsigned long long* sample_count,
                                                        int32_t learning_rate, uint8_t learning_rate_shift,
                                                        int carry_residual, unsigned long long* stats,
                                                        nsrl_device_status* status, void* stream) {
  // train-core lib.rs:393-399: InvalidConfig
  if (len == 0 || learning_rate <= 0 || learning_rate_shift > 62 || !accumulators || !residuals || !weights ||
      !sample_count || !stats || !status) {
    set_error("invalid shape: apply");
    return NSRL_INVALID_SHAPE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(stats, 0, 3 * sizeof(unsigned long long), s);
  if (e == cudaSuccess) {
    const unsigned blocks = (unsigned)std::min<size_t>((len + 255) / 256, 148 * 8);
    ProfScope prof("apply_i64_to_i8", s, 0.0, 34.0 * (double)len);
    apply_kernel<<<blocks, 256, 0, s>>>(accumulators, residuals, weights, (long long)len, sample_count, learning_rate,
                                        learning_rate_shift, carry_residual, stats, status);
    e = cudaGetLastError();
  }
  // the count is cleared after every thread of apply_kernel has read it
  if (e == cudaSuccess) e = cudaMemsetAsync(sample_count, 0, sizeof(unsigned long long), s);
  if (e != cudaSuccess) {
    set_error("apply: %s", cudaGetErrorString(e));
    return NSRL_CUDA_ERROR;
  }
  return NSRL_OK;
}

nsrl_status nsrl_average_movement_i8(const int8_t* base, int8_t* values, size_t len, uint64_t divisor, void* stream) {
  if (!base || !values || divisor == 0 || divisor > (uint64_t)LLONG_MAX) {
    set_error("invalid config: movement average (divisor must be nonzero)");
    return NSRL_INVALID_SHAPE;
  }
  if (len == 0) return NSRL_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned blocks = (unsigned)std::min<size_t>((len + 255) / 256, 148 * 8);
  ProfScope prof("average_movement_i8", s, 0.0, 3.0 * (double)len);
  average_movement_kernel<int8_t><<<blocks, 256, 0, s>>>(base, values, (long long)len, (long long)divisor, -128, 127);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("movement average: %s", cudaGetErrorString(e));
    return NSRL_CUDA_ERROR;
  }
  return NSRL_OK;
}

nsrl_status nsrl_average_movement_i16(const int16_t* base, int16_t* values, size_t len, uint64_t divisor,
                                      void* stream) {
  if (!base || !values || divisor == 0 || divisor > (uint64_t)LLONG_MAX) {
    set_error("invalid config: movement average (divisor must be nonzero)");
    return NSRL_INVALID_SHAPE;
  }
  if (len == 0) return NSRL_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned blocks = (unsigned)std::min<size_t>((len + 255) / 256, 148 * 8);
  ProfScope prof("average_movement_i16", s, 0.0, 6.0 * (double)len);
  average_movement_kernel<int16_t><<<blocks, 256, 0, s>>>(base, values, (long long)len, (long long)divisor, -32768,
                                                          32767);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("movement average: %s", cudaGetErrorString(e));
    return NSRL_CUDA_ERROR;
  }
  return NSRL_OK;
}

nsrl_status nsrl_apply_integer_adam_i64_to_i8(const long long* accumulators, const unsigned long long* sample_count,
                                              int8_t* weights, size_t len, const nsrl_integer_adam_config* config,
                                              long long* first_moments, unsigned long long* second_moments,
                                              long long* update_residuals, unsigned long long* step,
                                              unsigned long long* stats, nsrl_device_status* status, void* stream) {
  return launch_adam(accumulators, sample_count, weights, len, config, first_moments, second_moments,
                     update_residuals, step, stats, -128, 127, status, stream, "integer_adam_i8");
}

nsrl_status nsrl_apply_integer_adam_i64_to_i16(const long long* accumulators, const unsigned long long* sample_count,
                                               int16_t* weights, size_t len, const nsrl_integer_adam_config* config,
                                               long long* first_moments, unsigned long long* second_moments,
                                               long long* update_residuals, unsigned long long* step,
                                               unsigned long long* stats, nsrl_device_status* status, void* stream) {
  return launch_adam(accumulators, sample_count, weights, len, config, first_moments, second_moments,
                     update_residuals, step, stats, -32768, 32767, status, stream, "integer_adam_i16");
}

nsrl_status nsrl_apply_embedding_gradient_i64_to_i16(const long long* accumulators, long long* residuals,
                                                     int16_t* embeddings, size_t len,
                                                     const unsigned long long* sample_count, int32_t learning_rate,
                                                     uint8_t learning_rate_shift, unsigned long long* stats,
                                                     nsrl_device_status* status, void* stream) {
  // nsrl-train/src/lib.rs:14416-14421: InvalidConfig
  if (len == 0 || learning_rate <= 0 || learning_rate_shift > 62 || !accumulators || !residuals || !embeddings ||
      !sample_count || !stats || !status) {
    set_error("invalid shape: embedding apply");
    return NSRL_INVALID_SHAPE;
  }
  cudaStream_t s = (cudaStream_t)stream;
  const unsigned blocks = (unsigned)std::min<size_t>((len + 255) / 256, 148 * 8);
  ProfScope prof("apply_i64_to_i16", s, 0.0, 26.0 * (double)len);
  apply_embedding_kernel<<<blocks, 256, 0, s>>>(accumulators, residuals, embeddings, (long long)len, sample_count,
                                                learning_rate, learning_rate_shift, stats, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("embedding apply: %s", cudaGetErrorString(e));
    return NSRL_CUDA_ERROR;
  }
  return NSRL_OK;
}

}  // extern "C"
