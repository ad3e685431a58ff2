// Kernels of the integer training step (backward pass and gradient
// accumulation).  Included by train_step.cu only.
//
// Every kernel restates one reference function; the file:line is given per
// kernel.  Range notes explain why a `checked_*` of the reference can never
// fail for int16 operands, where a check is left out.
#pragma once
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace ts {

// Column of flat element e in rows of N: a mask when N is a power of two
// (every width of the training step), a 64-bit remainder otherwise.
__device__ __forceinline__ int col_of(long long e, int N) {
  return (N & (N - 1)) == 0 ? (int)(e & (long long)(N - 1)) : (int)(e % N);
}

// W [R][C] int8 -> WT [C][R] (the B operand of a backward-input linear).
__global__ void transpose_i8_kernel(const int8_t* __restrict__ w, int R, int C, int8_t* __restrict__ wt) {
  __shared__ int8_t tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = w[(long long)r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) wt[(long long)c * R + r] = tile[threadIdx.x][i];
  }
}

// linear.rs:573-592 with multiplier 1 (the only form the tensor-core
// backward path takes): g' = rhu(g, s), which stays in [-32768, 32767], split
// into byte planes.
__global__ void prescale_split_kernel(const int16_t* __restrict__ g, long long M, int N, long long ldg,
                                      const nsrl_fixed_scale* __restrict__ sc, int8_t* __restrict__ hi,
                                      uint8_t* __restrict__ lo, long long ldp) {
  const long long total = M * N;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / N;
    const int n = col_of(i, N);
    int v = g[r * ldg + n];
    const int s = sc[n].right_shift;
    if (s) v = (int)rhu64(v, (uint32_t)s);
    hi[r * ldp + n] = (int8_t)(v >> 8);
    lo[r * ldp + n] = (uint8_t)(v & 255);
  }
}

// linear.rs:548-640 for any scales: one thread per dx[m][k], the prescaled
// grads and the i64 sum in reference order.  Used where a forward multiplier
// is not 1 (the tensor-core path needs g' to fit int16).
__global__ void bwd_input_simt_kernel(const int16_t* __restrict__ g, long long M, int N, const int8_t* __restrict__ w,
                                      int K, const nsrl_fixed_scale* __restrict__ fsc,
                                      const nsrl_fixed_scale* __restrict__ gsc, int16_t* __restrict__ dx,
                                      nsrl_device_status* st) {
  const long long total = M * K;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / K;
    const int k = (int)(i % K);
    long long acc = 0;
    bool bad = false;
    for (int n = 0; n < N; ++n) {
      const nsrl_fixed_scale f = fsc[n];
      const long long gs = rhu64((long long)g[m * N + n] * (long long)f.multiplier, f.right_shift);
      if (gs < INT_MIN || gs > INT_MAX) bad = true;
      acc += gs * (long long)w[(long long)n * K + k];  // |acc| < N * 2^38: no i64 overflow
    }
    const nsrl_fixed_scale s = gsc ? gsc[k] : nsrl_fixed_scale{1, 0, {0, 0, 0}};
    const long long lo = (long long)((unsigned long long)acc * (unsigned long long)(long long)s.multiplier);
    if (__mul64hi(acc, (long long)s.multiplier) != (lo >> 63)) bad = true;
    dx[m * K + k] = sat_i16(rhu64(lo, s.right_shift));
    if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
  }
}

// mlp.rs:172-194 for every hidden unit, plus the prescaled byte planes of
// both results for the up^T / gate^T linears.  Ranges: the hard-SiLU gate
// (g >> 2) + 16384 lies in [8192, 24575], so |silu| <= 24575 and every
// saturation of the reference is a no-op except the final two; all
// products are below 2^31 in magnitude.
__global__ void gated_backward_kernel(const int16_t* __restrict__ gg, const int16_t* __restrict__ up,
                                      const int16_t* __restrict__ gate, long long n, int F,
                                      const nsrl_fixed_scale* __restrict__ su, const nsrl_fixed_scale* __restrict__ sg,
                                      int16_t* __restrict__ gup, int16_t* __restrict__ ggate, int8_t* __restrict__ uh,
                                      uint8_t* __restrict__ ul, int8_t* __restrict__ gh, uint8_t* __restrict__ gl) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int g = gg[i], u = up[i], ga = gate[i];
    const int silu = (ga * ((ga >> 2) + 16384) + 16384) >> 15;
    const int grad_up = (g * silu + 16384) >> 15;
    const int grad_silu = (g * u + 16384) >> 15;  // in [-32768, 32768]
    const int deriv = (ga >> 1) + 16384;
    const int grad_gate = sat16((grad_silu * deriv + 16384) >> 15);
    gup[i] = (int16_t)grad_up;
    ggate[i] = (int16_t)grad_gate;
    const int f = col_of(i, F);
    const int pu = su[f].right_shift ? (int)rhu64(grad_up, su[f].right_shift) : grad_up;
    const int pg = sg[f].right_shift ? (int)rhu64(grad_gate, sg[f].right_shift) : grad_gate;
    uh[i] = (int8_t)(pu >> 8);
    ul[i] = (uint8_t)(pu & 255);
    gh[i] = (int8_t)(pg >> 8);
    gl[i] = (uint8_t)(pg & 255);
  }
}

// gated_backward_kernel on eight consecutive hidden units per thread
// (F % 8 == 0, 16-byte aligned rows).
__global__ void gated_backward_vec_kernel(const int16_t* __restrict__ gg, const int16_t* __restrict__ up,
                                          const int16_t* __restrict__ gate, long long n8, int F,
                                          const nsrl_fixed_scale* __restrict__ su,
                                          const nsrl_fixed_scale* __restrict__ sg, int16_t* __restrict__ gup,
                                          int16_t* __restrict__ ggate, int8_t* __restrict__ uh,
                                          uint8_t* __restrict__ ul, int8_t* __restrict__ gh,
                                          uint8_t* __restrict__ gl) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  int fcur = -1, s1[8], s2[8];  // the shifts of columns fcur .. +7
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    int g[8], u[8], ga[8], ou[8], og[8], pu[8], pg[8];
    unpack8(reinterpret_cast<const uint4*>(gg)[i], g);
    unpack8(reinterpret_cast<const uint4*>(up)[i], u);
    unpack8(reinterpret_cast<const uint4*>(gate)[i], ga);
    const int f0 = col_of(i * 8, F);
    if (f0 != fcur) {
      fcur = f0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        s1[e] = su[f0 + e].right_shift;
        s2[e] = sg[f0 + e].right_shift;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int silu = (ga[e] * ((ga[e] >> 2) + 16384) + 16384) >> 15;
      ou[e] = (g[e] * silu + 16384) >> 15;
      const int grad_silu = (g[e] * u[e] + 16384) >> 15;
      og[e] = sat16((grad_silu * ((ga[e] >> 1) + 16384) + 16384) >> 15);
      pu[e] = rhu_i16(ou[e], s1[e]);  // |ou|, |og| <= 2^15
      pg[e] = rhu_i16(og[e], s2[e]);
    }
    if (gup) reinterpret_cast<uint4*>(gup)[i] = pack8(ou);
    if (ggate) reinterpret_cast<uint4*>(ggate)[i] = pack8(og);
    uint2 h, l;
    planes8(pu, h, l);
    reinterpret_cast<uint2*>(uh)[i] = h;
    reinterpret_cast<uint2*>(ul)[i] = l;
    planes8(pg, h, l);
    reinterpret_cast<uint2*>(gh)[i] = h;
    reinterpret_cast<uint2*>(gl)[i] = l;
  }
}

// prescale_split_kernel on eight consecutive columns (N % 8 == 0, ldg == ldp == N).
__global__ void prescale_split_vec_kernel(const int16_t* __restrict__ g, long long n8, int N,
                                          const nsrl_fixed_scale* __restrict__ sc, int8_t* __restrict__ hi,
                                          uint8_t* __restrict__ lo) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  // two words in flight per thread; each slot keeps the shifts of its
  // columns cur[k] .. +7 (the same every pass when the stride is a multiple of N)
  const long long stride = (long long)gridDim.x * blockDim.x;
  int cur[2] = {-1, -1}, sh[2][8];
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += 2 * stride) {
    const uint4 u[2] = {reinterpret_cast<const uint4*>(g)[i],
                        i + stride < n8 ? reinterpret_cast<const uint4*>(g)[i + stride] : make_uint4(0, 0, 0, 0)};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const long long ik = i + k * stride;
      if (ik >= n8) break;
      int v[8];
      unpack8(u[k], v);
      const int c0 = col_of(ik * 8, N);
      if (c0 != cur[k]) {
        cur[k] = c0;
#pragma unroll
        for (int e = 0; e < 8; ++e) sh[k][e] = sc[c0 + e].right_shift;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = rhu_i16(v[e], sh[k][e]);
      uint2 h, l;
      planes8(v, h, l);
      reinterpret_cast<uint2*>(hi)[ik] = h;
      reinterpret_cast<uint2*>(lo)[ik] = l;
    }
  }
}

// add_sat_kernel / fanin3_kernel on eight elements per thread (n % 8 == 0).
__global__ void add_sat_vec_kernel(const int16_t* __restrict__ a, const int16_t* __restrict__ b, long long n8,
                                   int16_t* __restrict__ out, unsigned long long* sat) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  unsigned long long c = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    int x[8], y[8], o[8];
    unpack8(reinterpret_cast<const uint4*>(a)[i], x);
    unpack8(reinterpret_cast<const uint4*>(b)[i], y);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int w = x[e] + y[e];
      o[e] = sat16(w);
      c += o[e] != w;
    }
    reinterpret_cast<uint4*>(out)[i] = pack8(o);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(sat, c);
}
__global__ void fanin3_vec_kernel(const int16_t* __restrict__ a, const int16_t* __restrict__ b,
                                  const int16_t* __restrict__ c3, long long n8, int16_t* __restrict__ out,
                                  unsigned long long* sat) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  unsigned long long cnt = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    int x[8], y[8], z[8], o[8];
    unpack8(reinterpret_cast<const uint4*>(a)[i], x);
    unpack8(reinterpret_cast<const uint4*>(b)[i], y);
    unpack8(reinterpret_cast<const uint4*>(c3)[i], z);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int w = (x[e] + y[e] + z[e] + 1) >> 1;
      o[e] = sat16(w);
      cnt += o[e] != w;
    }
    reinterpret_cast<uint4*>(out)[i] = pack8(o);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(sat, cnt);
}

// out = sat(a + b) with the saturation count (numeric.rs:25-45,
// nsrl-train/src/lib.rs:17490-17506).
__global__ void add_sat_kernel(const int16_t* __restrict__ a, const int16_t* __restrict__ b, long long n,
                               int16_t* __restrict__ out, unsigned long long* sat) {
  unsigned long long c = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int w = (int)a[i] + (int)b[i];
    const int v = sat16(w);
    c += v != w;
    out[i] = (int16_t)v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0 && c) atomicAdd(sat, c);
}

// nsrl-train/src/lib.rs:15940-15956: sat(rhu(gq + gk + gv, 1)) with the count.
__global__ void fanin3_kernel(const int16_t* __restrict__ a, const int16_t* __restrict__ b,
                              const int16_t* __restrict__ c, long long n, int16_t* __restrict__ out,
                              unsigned long long* sat) {
  unsigned long long cnt = 0;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int w = ((int)a[i] + (int)b[i] + (int)c[i] + 1) >> 1;
    const int v = sat16(w);
    cnt += v != w;
    out[i] = (int16_t)v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if ((threadIdx.x & 31) == 0 && cnt) atomicAdd(sat, cnt);
}

// Rows of x [rows][d] that hold a nonzero value, added to counts[0..2]
// (nsrl-train/src/lib.rs:13828-13831 skips all-zero gradient rows before
// counting the gated-MLP samples).  One warp per row.
__global__ void nonzero_rows_kernel(const int16_t* __restrict__ x, long long rows, int d, unsigned long long* c0,
                                    unsigned long long* c1, unsigned long long* c2) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  unsigned long long cnt = 0;
  for (long long r = (long long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long long)gridDim.x * warps) {
    bool any = false;
    for (int k = lane; k < d; k += 32) any |= x[r * d + k] != 0;
    if (__any_sync(0xffffffffu, any) && lane == 0) ++cnt;
  }
  if (lane == 0 && cnt) {
    atomicAdd(c0, cnt);
    atomicAdd(c1, cnt);
    atomicAdd(c2, cnt);
  }
}

// nsrl-train/src/lib.rs:14862-14897: x[t] = sat(embedding[token] + position[t]).
__global__ void embed_forward_kernel(const uint8_t* __restrict__ ctx, long long T, int S, int d,
                                     const int16_t* __restrict__ emb, const int16_t* __restrict__ pos,
                                     int16_t* __restrict__ x) {
  const long long n = T * d;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / d;
    const int k = (int)(i % d);
    int v = emb[(long long)ctx[t] * d + k];
    if (pos) v += pos[(long long)(t % S) * d + k];
    x[i] = (int16_t)sat16(v);
  }
}

// nsrl-train/src/lib.rs:14336-14405: token and position gradient sums (i64;
// |sum| <= T * 32768, far from overflow; two's-complement adds are exact).
__global__ void embed_grad_kernel(const uint8_t* __restrict__ ctx, long long T, int S, int d,
                                  const int16_t* __restrict__ g, long long* __restrict__ emb_acc,
                                  long long* __restrict__ pos_acc) {
  const long long n = T * d;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int v = g[i];
    if (v == 0) continue;
    const long long t = i / d;
    const int k = (int)(i % d);
    atomicAdd(reinterpret_cast<unsigned long long*>(&emb_acc[(long long)ctx[t] * d + k]), (unsigned long long)(long long)v);
    if (pos_acc)
      atomicAdd(reinterpret_cast<unsigned long long*>(&pos_acc[(long long)(t % S) * d + k]),
                (unsigned long long)(long long)v);
  }
}

// nsrl-train/src/lib.rs:17455-17488 (softmax of the byte head) and
// :18845-18949 (p - 32767 at the target, the frequency weight, int16):
// one 256-thread CTA per window.
__global__ void __launch_bounds__(256) head_grad_kernel(const int16_t* __restrict__ logits,
                                                        const uint8_t* __restrict__ targets,
                                                        const int16_t* __restrict__ freq_w, int16_t* __restrict__ grad,
                                                        nsrl_device_status* st) {
  __shared__ int16_t lut[256];
  __shared__ int red_i[8];
  __shared__ unsigned long long red_u[8];
  const int w = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  lut[tid] = d_exp2_lut[tid];
  const int lg = logits[(long long)w * 256 + tid];
  int mx = lg;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red_i[warp] = mx;
  __syncthreads();
  mx = red_i[0];
  for (int i = 1; i < 8; ++i) mx = max(mx, red_i[i]);
  const int wv = exp2_neg_q15(lut, (long long)lg - mx);
  unsigned long long s = (unsigned long long)wv;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) red_u[warp] = s;
  __syncthreads();
  s = 0;
  for (int i = 0; i < 8; ++i) s += red_u[i];
  const long long inv = (long long)recip_sum_q31(s);  // s >= 32767: the max logit has weight 32767
  const int p = sat_i16(rhu64((long long)wv * inv, 16));
  const int target = targets[w];
  long long gv = (long long)p - (tid == target ? 32767 : 0);
  const int fw = freq_w ? freq_w[target] : 32767;
  if (fw != 32767) gv = rhu64(gv * (long long)fw, 15);
  grad[(long long)w * 256 + tid] = sat_i16(gv);
  (void)st;
}

// acc[n][k] += sum_r g'[r][n] * x[r][k], g' = rhu(g * mult, shift) per
// output channel n (nsrl-train-core/src/lib.rs:344-384 after the prescale of
// linear.rs:573-592).  256 threads, a 64 x 64 tile of acc, 4 x 4 each.
// With multiplier 1, |g'| <= 32768 and |acc| grows by at most 2^30 per row:
// no i64 overflow below 2^32 rows in one batch.
constexpr int ATN = 64, ATK = 64, ATR = 32;
__global__ void __launch_bounds__(256) accumulate_pre_kernel(const int16_t* __restrict__ x, long long ldx,
                                                             const int16_t* __restrict__ g, long long ldg,
                                                             const nsrl_fixed_scale* __restrict__ sc, int rows, int K,
                                                             int N, long long* __restrict__ acc,
                                                             nsrl_device_status* st) {
  __shared__ int32_t sg[ATR][ATN];
  __shared__ int32_t sx[ATR][ATK + 1];
  const int n0 = blockIdx.y * ATN, k0 = blockIdx.x * ATK;
  const int tn = threadIdx.x / 16, tk = threadIdx.x % 16;
  long long c[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0;
  bool bad = false;
  for (int r0 = 0; r0 < rows; r0 += ATR) {
    for (int i = threadIdx.x; i < ATR * ATN; i += 256) {
      const int rr = i / ATN, nn = i % ATN;
      int v = 0;
      if (r0 + rr < rows && n0 + nn < N) {
        const nsrl_fixed_scale s = sc[n0 + nn];
        const long long w = rhu64((long long)g[(long long)(r0 + rr) * ldg + n0 + nn] * (long long)s.multiplier,
                                  s.right_shift);
        if (w < INT_MIN || w > INT_MAX) bad = true;
        v = (int)w;
      }
      sg[rr][nn] = v;
    }
    for (int i = threadIdx.x; i < ATR * ATK; i += 256) {
      const int rr = i / ATK, kk = i % ATK;
      sx[rr][kk] = (r0 + rr < rows && k0 + kk < K) ? (int)x[(long long)(r0 + rr) * ldx + k0 + kk] : 0;
    }
    __syncthreads();
#pragma unroll 4
    for (int rr = 0; rr < ATR; ++rr) {
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
  if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
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

// acc[n][k] += sum_r g'[r][n] * x[r][k] from byte planes (g' already
// prescaled: 256 * gh + gl; x = 256 * xh + xl), the SIMT form of the
// tensor-core weight gradient for operands TMA cannot take.
__global__ void __launch_bounds__(256) accumulate_planes_kernel(const int8_t* __restrict__ gh,
                                                                const uint8_t* __restrict__ gl, long long ldg,
                                                                const int8_t* __restrict__ xh,
                                                                const uint8_t* __restrict__ xl, long long ldx,
                                                                int rows, int K, int N, long long* __restrict__ acc) {
  __shared__ int32_t sg[ATR][ATN];
  __shared__ int32_t sx[ATR][ATK + 1];
  const int n0 = blockIdx.y * ATN, k0 = blockIdx.x * ATK;
  const int tn = threadIdx.x / 16, tk = threadIdx.x % 16;
  long long c[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0;
  for (int r0 = 0; r0 < rows; r0 += ATR) {
    for (int i = threadIdx.x; i < ATR * ATN; i += 256) {
      const int rr = i / ATN, nn = i % ATN;
      const long long o = (long long)(r0 + rr) * ldg + n0 + nn;
      sg[rr][nn] = (r0 + rr < rows && n0 + nn < N) ? (int)gh[o] * 256 + (int)gl[o] : 0;
    }
    for (int i = threadIdx.x; i < ATR * ATK; i += 256) {
      const int rr = i / ATK, kk = i % ATK;
      const long long o = (long long)(r0 + rr) * ldx + k0 + kk;
      sx[rr][kk] = (r0 + rr < rows && k0 + kk < K) ? (int)xh[o] * 256 + (int)xl[o] : 0;
    }
    __syncthreads();
#pragma unroll 4
    for (int rr = 0; rr < ATR; ++rr) {
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

// rms_norm.rs:96-170 per row; gamma gradients summed per CTA in shared
// memory, then added to gw.  One warp per row.  Ranges (int16 x, w, go):
// inv <= 2^30, so x * inv < 2^45, x * w * inv <= 2^60, |normalized| <= 2^30,
// |scaled * normalized| < 2^46 (dot < d * 2^46), |mean_dot| < 2^31,
// |normalized * mean_dot| < 2^61 and |correction * inv| < 2^62: none of the
// reference's checked operations can fail, so none is repeated here.
__global__ void __launch_bounds__(256) rms_backward_kernel(const int16_t* __restrict__ x, long long rows, int d,
                                                           double rd, const int16_t* __restrict__ w,
                                                           const int16_t* __restrict__ go, unsigned long long eps,
                                                           int16_t* __restrict__ gi, long long* __restrict__ gw,
                                                           unsigned long long* sat, nsrl_device_status* st) {
  extern __shared__ long long sgw[];
  for (int i = threadIdx.x; i < d; i += blockDim.x) sgw[i] = 0;
  __syncthreads();
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  unsigned long long nsat = 0;
  for (long long r = (long long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long long)gridDim.x * warps) {
    const int16_t* xr = x + r * d;
    const int16_t* gr = go + r * d;
    unsigned long long ss = 0;
    for (int k = lane; k < d; k += 32) ss += (unsigned long long)((int)xr[k] * (int)xr[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const unsigned long long mean = div_exact(ss, (unsigned)d, rd);
    const unsigned long long v = mean + eps;
    if (v < mean || v == 0) {
      if (lane == 0) nsrl_flag(st, NSRL_FLAG_RMS_ZERO);
      continue;
    }
    const long long inv = rsqrt_q30(v);
    long long dot = 0;
    for (int k = lane; k < d; k += 32) {
      const long long nm = rhu64((long long)xr[k] * inv, 15);
      const long long proj = rhu64((long long)(xr[k] * (int)w[k]) * inv, 30);
      const bool active = proj >= -32768 && proj <= 32767;
      if (active) {
        const long long sg = rhu64((long long)(gr[k] * (int)w[k]), 15);
        dot += sg * nm;
        const long long gg = rhu64((long long)gr[k] * nm, 15);
        if (gg) atomicAdd(reinterpret_cast<unsigned long long*>(&sgw[k]), (unsigned long long)gg);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    // rms_norm.rs:172-179: floor((dot + den / 2) / den), den = d << 15
    const long long den = (long long)d << 15;
    const long long t = dot + den / 2;
    long long mdot = t / den;
    if ((t % den) != 0 && t < 0) --mdot;
    for (int k = lane; k < d; k += 32) {
      const long long nm = rhu64((long long)xr[k] * inv, 15);
      const long long proj = rhu64((long long)(xr[k] * (int)w[k]) * inv, 30);
      const bool active = proj >= -32768 && proj <= 32767;
      const long long sg = active ? rhu64((long long)(gr[k] * (int)w[k]), 15) : 0;
      const long long cross = rhu64(nm * mdot, 15);
      const long long g = rhu64((sg - cross) * inv, 30);
      const int16_t cl = sat_i16(g);
      nsat += (long long)cl != g;
      gi[r * d + k] = cl;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    if (sgw[i]) atomicAdd(reinterpret_cast<unsigned long long*>(&gw[i]), (unsigned long long)sgw[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) nsat += __shfl_xor_sync(0xffffffffu, nsat, o);
  if (lane == 0 && nsat) atomicAdd(sat, nsat);
}

// rms_backward_kernel with the row held in registers: D32 = d / 32 columns per
// lane (lane + 32 i), gamma gradients summed per lane over the warp's rows and
// added once per warp.  Same arithmetic; the rounding adds cannot saturate
// here (see the range note above), so rhu is (v + 2^(s-1)) >> s.
template <int D32>
__global__ void __launch_bounds__(256) rms_backward_reg_kernel(const int16_t* __restrict__ x, long long rows,
                                                               const int16_t* __restrict__ w,
                                                               const int16_t* __restrict__ go, unsigned long long eps,
                                                               int16_t* __restrict__ gi, long long* __restrict__ gw,
                                                               unsigned long long* sat, nsrl_device_status* st) {
  constexpr int d = 32 * D32;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  int wv[D32];
  long long gacc[D32];
#pragma unroll
  for (int i = 0; i < D32; ++i) {
    wv[i] = w[lane + 32 * i];
    gacc[i] = 0;
  }
  unsigned long long nsat = 0;
  for (long long r = (long long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long long)gridDim.x * warps) {
    int xv[D32], gv[D32];
#pragma unroll
    for (int i = 0; i < D32; ++i) {
      xv[i] = x[r * d + lane + 32 * i];
      gv[i] = go[r * d + lane + 32 * i];
    }
    unsigned long long ss = 0;
#pragma unroll
    for (int i = 0; i < D32; ++i) ss += (unsigned long long)(unsigned)(xv[i] * xv[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const unsigned long long mean = ss / (unsigned long long)d;
    const unsigned long long v = mean + eps;
    if (v < mean || v == 0) {
      if (lane == 0) nsrl_flag(st, NSRL_FLAG_RMS_ZERO);
      continue;
    }
    const long long inv = rsqrt_q30(v);
    int nm[D32], sg[D32];
    long long dot = 0;
#pragma unroll
    for (int i = 0; i < D32; ++i) {
      nm[i] = (int)(((long long)xv[i] * inv + (1ll << 14)) >> 15);
      const long long proj = ((long long)(xv[i] * wv[i]) * inv + (1ll << 29)) >> 30;
      const bool active = proj >= -32768 && proj <= 32767;
      sg[i] = active ? ((gv[i] * wv[i] + (1 << 14)) >> 15) : 0;
      dot += (long long)sg[i] * (long long)nm[i];
      if (active) gacc[i] += ((long long)gv[i] * (long long)nm[i] + (1ll << 14)) >> 15;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const long long den = (long long)d << 15;
    const long long tq = dot + den / 2;
    long long mdot = tq / den;
    if ((tq % den) != 0 && tq < 0) --mdot;
#pragma unroll
    for (int i = 0; i < D32; ++i) {
      const long long cross = ((long long)nm[i] * mdot + (1ll << 14)) >> 15;
      const long long gg = (((long long)sg[i] - cross) * inv + (1ll << 29)) >> 30;
      const int16_t cl = sat_i16(gg);
      nsat += (long long)cl != gg;
      gi[r * d + lane + 32 * i] = cl;
    }
  }
  // gamma gradients: the block's warps add into shared memory, then one
  // global add per column and block
  __shared__ unsigned long long gsum[d];
  for (int i = threadIdx.x; i < d; i += blockDim.x) gsum[i] = 0;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < D32; ++i)
    if (gacc[i]) atomicAdd(&gsum[lane + 32 * i], (unsigned long long)gacc[i]);
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    if (gsum[i]) atomicAdd(reinterpret_cast<unsigned long long*>(&gw[i]), gsum[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) nsat += __shfl_xor_sync(0xffffffffu, nsat, o);
  if (lane == 0 && nsat) atomicAdd(sat, nsat);
}

// rms_backward_reg_kernel for d = 256 with 16-byte rows: lane l owns columns
// 8 l .. 8 l + 7, each warp works on RPW rows at once (independent chains for
// the scheduler), the row sums go through the reduction unit, and the
// products run on 32-bit operands (inv <= 2^30, |nm| <= 2^30, |x w|, |g w| <=
// 2^30) into 64-bit results.  Per lane |sum x^2| <= 2^33 and |sum sg nm| <=
// 2^48, inside the exact ranges of the warp sums.  With `res`, the residual
// add that follows the norm in the block backward is fused: out = sat(res +
// gi), its saturations counted in res_sat (gi is not written); otherwise gi is
// written as in rms_backward_reg_kernel.
template <int RPW>
__global__ void __launch_bounds__(256) rms_backward_vec_kernel(
    const int16_t* __restrict__ x, long long rows, const int16_t* __restrict__ w, const int16_t* __restrict__ go,
    unsigned long long eps, int16_t* __restrict__ gi, long long* __restrict__ gw, unsigned long long* sat,
    nsrl_device_status* st, const int16_t* __restrict__ res, int16_t* __restrict__ out, unsigned long long* res_sat) {
  griddep_wait();  // launched as a dependent: the previous kernel's outputs are visible from here
  griddep_launch();
  constexpr int d = 256;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  int wv[8];
  long long gacc[8];
  unpack8(*reinterpret_cast<const uint4*>(w + 8 * lane), wv);
#pragma unroll
  for (int i = 0; i < 8; ++i) gacc[i] = 0;
  unsigned long long nsat = 0, rsat = 0;
  const long long step = (long long)gridDim.x * warps * RPW;
  for (long long r0 = ((long long)blockIdx.x * warps + (threadIdx.x >> 5)) * RPW; r0 < rows; r0 += step) {
    int xv[RPW][8], gv[RPW][8];
    bool live[RPW];
#pragma unroll
    for (int k = 0; k < RPW; ++k) {
      live[k] = r0 + k < rows;
      const long long o = (r0 + k) * d + 8 * lane;
      unpack8(live[k] ? *reinterpret_cast<const uint4*>(x + o) : make_uint4(0, 0, 0, 0), xv[k]);
      unpack8(live[k] ? *reinterpret_cast<const uint4*>(go + o) : make_uint4(0, 0, 0, 0), gv[k]);
    }
    int inv[RPW];
    bool ok[RPW];
#pragma unroll
    for (int k = 0; k < RPW; ++k) {
      unsigned long long ss = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += (unsigned long long)(unsigned)(xv[k][i] * xv[k][i]);
      ss = warp_sum_u37(ss);
      const unsigned long long mean = ss / (unsigned long long)d;
      const unsigned long long v = mean + eps;
      ok[k] = live[k] && !(v < mean || v == 0);
      if (live[k] && !ok[k] && lane == 0) nsrl_flag(st, NSRL_FLAG_RMS_ZERO);
      inv[k] = ok[k] ? (int)rsqrt_q30(v) : 0;  // <= 2^30
    }
    int nm[RPW][8], sg[RPW][8];
    long long mdot[RPW];
    bool fast[RPW];
#pragma unroll
    for (int k = 0; k < RPW; ++k) {
      long long dot = 0;
      unsigned nmax = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        nm[k][i] = (int)(((long long)xv[k][i] * inv[k] + (1ll << 14)) >> 15);
        nmax = max(nmax, (unsigned)abs(nm[k][i]));
        // proj = t >> 30 lies in [-2^15, 2^15) iff t in [-2^45, 2^45), i.e. iff
        // the high word of t lies in [-2^13, 2^13)
        const long long t = (long long)(xv[k][i] * wv[i]) * inv[k] + (1ll << 29);
        const bool active = ok[k] && (unsigned)((int)(t >> 32) + 8192) < 16384u;
        sg[k][i] = active ? ((gv[k][i] * wv[i] + (1 << 14)) >> 15) : 0;
        dot += (long long)sg[k][i] * nm[k][i];
        if (active) gacc[i] += ((long long)gv[k][i] * nm[k][i] + (1ll << 14)) >> 15;
      }
      dot = warp_sum_s52(dot);
      constexpr long long den = (long long)d << 15;
      const long long tq = dot + den / 2;
      mdot[k] = tq / den;
      if ((tq % den) != 0 && tq < 0) --mdot[k];
      // 32-bit cross terms when every |nm * mdot| + 2^14 of the row fits an int
      nmax = __reduce_max_sync(0xffffffffu, nmax);
      const unsigned long long amd = (unsigned long long)(mdot[k] < 0 ? -mdot[k] : mdot[k]);
      fast[k] = amd < (1ull << 31) && (unsigned long long)nmax * amd < (1ull << 31) - (1ull << 14);
    }
#pragma unroll
    for (int k = 0; k < RPW; ++k) {
      if (!ok[k]) continue;
      const long long o = (r0 + k) * d + 8 * lane;
      uint4 rn = make_uint4(0, 0, 0, 0);
      if (res) rn = *reinterpret_cast<const uint4*>(res + o);
      int o16[8];
      if (fast[k]) {
        // |cross| < 2^16 and |sg| <= 2^15, so |(sg - cross) inv| < 2^47 and
        // the rounded shift fits an int
        const int md = (int)mdot[k];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int cross = (nm[k][i] * md + (1 << 14)) >> 15;
          const int gg = (int)(((long long)(sg[k][i] - cross) * inv[k] + (1ll << 29)) >> 30);
          const int cl = max(-32768, min(32767, gg));
          nsat += cl != gg;
          o16[i] = cl;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const long long cross = ((long long)nm[k][i] * mdot[k] + (1ll << 14)) >> 15;
          const long long gg = (((long long)sg[k][i] - cross) * inv[k] + (1ll << 29)) >> 30;
          const int cl = sat_i16(gg);
          nsat += (long long)cl != gg;
          o16[i] = cl;
        }
      }
      if (res) {
        int rv[8];
        unpack8(rn, rv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int sum = rv[i] + o16[i];
          o16[i] = sat16(sum);
          rsat += o16[i] != sum;
        }
        *reinterpret_cast<uint4*>(out + o) = pack8(o16);
      } else {
        *reinterpret_cast<uint4*>(gi + o) = pack8(o16);
      }
    }
  }
  __shared__ unsigned long long gsum[d];
  for (int i = threadIdx.x; i < d; i += blockDim.x) gsum[i] = 0;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (gacc[i]) atomicAdd(&gsum[8 * lane + i], (unsigned long long)gacc[i]);
  __syncthreads();
  for (int i = threadIdx.x; i < d; i += blockDim.x)
    if (gsum[i]) atomicAdd(reinterpret_cast<unsigned long long*>(&gw[i]), gsum[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    nsat += __shfl_xor_sync(0xffffffffu, nsat, o);
    rsat += __shfl_xor_sync(0xffffffffu, rsat, o);
  }
  if (lane == 0 && nsat) atomicAdd(sat, nsat);
  if (lane == 0 && rsat) atomicAdd(res_sat, rsat);
}

// nsrl-train/src/lib.rs:16623-16747 for one (query row, head, sequence):
// dP[j] = sat(rhu(dC[t] . V[j], 15)) for j <= t, then
// dL[j] = sat(rhu(P[j] * (dP[j] - rhu(sum_j dP[j] P[j], 15)) * 22713, 30)),
// written as the full row of dL [B][H][S][S] (zeros past the diagonal).
// LPK lanes share one value row (8 int16 each); hd = 8 * LPK.
template <int LPK>
__global__ void __launch_bounds__(256) attn_dlogit_kernel(const int16_t* __restrict__ dC, long long ldc,
                                                          const int16_t* __restrict__ V, long long ldv,
                                                          const int16_t* __restrict__ P, int S, int H,
                                                          int16_t* __restrict__ dL, nsrl_device_status* st) {
  extern __shared__ int32_t sdp[];  // [S]
  __shared__ long long red[8];
  constexpr int HD = 8 * LPK, GROUPS = 256 / LPK;
  const int t = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sub = tid % LPK, grp = tid / LPK;
  const long long row0 = (long long)b * S;
  int dv[8];
  {
    const uint4 u = *reinterpret_cast<const uint4*>(dC + (row0 + t) * ldc + (long long)h * HD + 8 * sub);
    const int16_t* e = reinterpret_cast<const int16_t*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) dv[i] = e[i];
  }
  const int L = t + 1;
  const int rounds = (L + GROUPS - 1) / GROUPS;
  for (int it = 0; it < rounds; ++it) {
    const int j = grp + it * GROUPS;
    long long s = 0;
    if (j < L) {
      const uint4 u = *reinterpret_cast<const uint4*>(V + (row0 + j) * ldv + (long long)h * HD + 8 * sub);
      const int16_t* e = reinterpret_cast<const int16_t*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) s += (long long)(dv[i] * (int)e[i]);
    }
#pragma unroll
    for (int o = 1; o < LPK; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (sub == 0 && j < L) sdp[j] = sat_i16(rhu64(s, 15));
  }
  __syncthreads();
  const int16_t* pr = P + (((long long)b * H + h) * S + t) * S;
  long long ws = 0;
  bool neg = false;
  for (int j = tid; j < L; j += 256) {
    const int p = pr[j];
    neg |= p < 0;
    ws += (long long)sdp[j] * (long long)p;
  }
  if (neg) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o);
  if (lane == 0) red[warp] = ws;
  __syncthreads();
  ws = 0;
  for (int i = 0; i < 8; ++i) ws += red[i];
  const long long wq = rhu64(ws, 15);
  int16_t* out = dL + (((long long)b * H + h) * S + t) * S;
  for (int j = tid; j < S; j += 256) {
    int16_t v = 0;
    if (j < L) v = sat_i16(rhu64((long long)pr[j] * ((long long)sdp[j] - wq) * 22713ll, 30));
    out[j] = v;
  }
}

// nsrl-train/src/lib.rs:16749-16900: per (64-row tile, head, sequence)
//   MODE 0 (dQ):  out[i] = sat(rhu(sum_{j<=i} dL[i][j] K[j], shift))
//   MODE 1 (dK):  out[i] = sat(rhu(sum_{j>=i} dL[j][i] Q[j], shift))
//   MODE 2 (dV):  out[i] = sat(rhu(sum_{j>=i} P[j][i] dC[j], 15))
// M is the [S][S] matrix of the head (dL or P, zero above the diagonal),
// B the int16 operand rows (stride ldb).  256 threads, HD / 16 outputs of
// four rows each per thread, i64 sums.
template <int MODE, int HD>
__global__ void __launch_bounds__(256) attn_grad_gemm_kernel(const int16_t* __restrict__ Mx,
                                                             const int16_t* __restrict__ Bm, long long ldb, int S,
                                                             int H, int shift, int16_t* __restrict__ out,
                                                             long long ldo) {
  constexpr int RT = 64, JT = 32, CPT = HD / 16;  // rows per tile, j chunk, columns per thread
  __shared__ int32_t sa[JT][RT + 1];
  __shared__ int32_t sb[JT][HD];
  const int i0 = blockIdx.x * RT, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, tr = tid / 16, tc = tid % 16;
  const int16_t* M = Mx + ((long long)b * H + h) * S * (long long)S;
  const long long brow0 = (long long)b * S;
  long long c[4][CPT];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < CPT; ++j) c[i][j] = 0;
  const int iend = min(S, i0 + RT);
  const int jbeg = MODE == 0 ? 0 : i0;
  const int jend = MODE == 0 ? iend : S;
  for (int j0 = jbeg; j0 < jend; j0 += JT) {
    for (int e = tid; e < JT * RT; e += 256) {
      int jj, ii;
      if (MODE == 0) {  // M[i][j]: j fastest
        ii = e / JT;
        jj = e % JT;
      } else {  // M[j][i]: i fastest
        jj = e / RT;
        ii = e % RT;
      }
      const int i = i0 + ii, j = j0 + jj;
      int v = 0;
      if (i < S && j < S) v = MODE == 0 ? M[(long long)i * S + j] : M[(long long)j * S + i];
      sa[jj][ii] = v;
    }
    for (int e = tid; e < JT * HD; e += 256) {
      const int jj = e / HD, cc = e % HD;
      const int j = j0 + jj;
      sb[jj][cc] = j < S ? (int)Bm[(brow0 + j) * ldb + (long long)h * HD + cc] : 0;
    }
    __syncthreads();
#pragma unroll 4
    for (int jj = 0; jj < JT; ++jj) {
      int av[4], bv[CPT];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = sa[jj][tr + 16 * i];
#pragma unroll
      for (int j = 0; j < CPT; ++j) bv[j] = sb[jj][tc + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < CPT; ++j) c[i][j] += (long long)av[i] * (long long)bv[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i0 + tr + 16 * i;
    if (r >= S) continue;
#pragma unroll
    for (int j = 0; j < CPT; ++j)
      out[(brow0 + r) * ldo + (long long)h * HD + tc + 16 * j] = sat_i16(rhu64(c[i][j], (uint32_t)shift));
  }
}

// Adds per-slot increments to the sample counts.
struct CountInc {
  int n;
  int idx[64];
  unsigned long long v[64];
};
__global__ void count_add_kernel(unsigned long long* counts, const CountInc inc) {
  for (int i = threadIdx.x; i < inc.n; i += blockDim.x) atomicAdd(&counts[inc.idx[i]], inc.v[i]);
}

// stats[3] += 2 * forward residual saturations (nsrl-train/src/lib.rs:7333-7338
// adds the window's forward count twice); stats[0] += accepted windows.
__global__ void stats_finish_kernel(unsigned long long* stats, const unsigned long long* fwd_res,
                                    unsigned long long windows) {
  stats[0] += windows;
  stats[3] += 2ull * *fwd_res;
}

}  // namespace ts
}  // namespace nsrl
