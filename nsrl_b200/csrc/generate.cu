// Device kernels of byte generation with the mini transformer: the context
// windows, the embedding, the byte-head row of the last position and the
// selection of the next byte, so that a whole generation runs on the stream
// without a host round trip per token.
//
// Reference: crates/nsrl-train/src/lib.rs:12702-12800 (the generation loop:
// the last seq_len bytes of the context, left-padded with b' ', run the full
// forward), :14862-14897 (embeddings + learned positions), :17455-17490 (the
// byte head on the last position and its base-2 softmax), :18951-19100 (the
// selection: greedy argmax, or seeded top-k sampling), :19334-19347
// (decode_sample_u64), :19468-19519 (StableHasher).
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {

constexpr int VOCAB = 256;

// win[b][t]: the last min(S, len[b]) context bytes of sequence b, right
// aligned, after S - min(S, len[b]) spaces.
__global__ void window_kernel(const uint8_t* __restrict__ ctx, long long cap, const int32_t* __restrict__ lens, int S,
                              int B, uint8_t* __restrict__ win) {
  const long long n = (long long)B * S;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / S), t = (int)(i % S);
    const int len = lens[b];
    const int L = min(S, len);
    const int pad = S - L;
    win[i] = t < pad ? (uint8_t)' ' : ctx[(long long)b * cap + (len - L) + (t - pad)];
  }
}

// x[b*S + t][i] = sat_i16(emb[win[b][t]][i] + pos[t][i]) (lib.rs:14862-14897).
__global__ void embed_kernel(const uint8_t* __restrict__ win, int S, int d, const int16_t* __restrict__ emb,
                             const int16_t* __restrict__ pos, long long rows, int16_t* __restrict__ x) {
  const long long n = rows * d;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / d;
    const int c = (int)(i % d);
    int v = emb[(int)win[r] * d + c];
    if (pos) v += pos[(int)(r % S) * d + c];
    x[i] = (int16_t)max(-32768, min(32767, v));
  }
}

// The byte head on row `rows[b]` of x (one CTA of 256 threads per sequence,
// thread c = class c): the linear's i32 accumulation with the reference's
// prefix rule (linear.rs:144-173, :282-296), requantised, then the base-2
// softmax of the 256 logits (attention.rs:261-293).
__global__ void __launch_bounds__(VOCAB) head_row_kernel(const int16_t* __restrict__ x, long long row_stride,
                                                         long long row0, int d, const int8_t* __restrict__ w,
                                                         const int32_t* __restrict__ bias,
                                                         const nsrl_fixed_scale* __restrict__ scales,
                                                         int32_t* __restrict__ logits_out,
                                                         int16_t* __restrict__ probs_out, nsrl_device_status* st) {
  __shared__ int16_t s_x[4096];
  __shared__ int16_t lut[256];
  __shared__ int s_max[VOCAB / 32];
  __shared__ unsigned long long s_sum[VOCAB / 32];
  const int b = blockIdx.x, c = threadIdx.x, lane = c & 31, wp = c >> 5;
  const int16_t* xr = x + (long long)b * row_stride + row0;
  for (int k = c; k < d; k += VOCAB) s_x[k] = xr[k];
  lut[c] = d_exp2_lut[c];
  __syncthreads();
  const int8_t* wr = w + (long long)c * d;
  const int bv = bias ? bias[c] : 0;
  const long long babs = bv < 0 ? -(long long)bv : bv;
  const bool fits = babs + (long long)d * 127 * 32767 <= 2147483647ll;
  long long acc = bv;
  bool bad = false;
  for (int k = 0; k < d; ++k) {
    acc += (long long)s_x[k] * wr[k];
    if (!fits && (acc > 2147483647ll || acc < -2147483648ll)) bad = true;  // a prefix left i32: checked_add fails
  }
  if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
  const int logit = (int)requant_i32((int)acc, scales[c].multiplier, scales[c].right_shift);
  // row max (no logit of an i16 head is masked)
  int m = logit;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) s_max[wp] = m;
  __syncthreads();
  m = s_max[0];
  for (int i = 1; i < VOCAB / 32; ++i) m = max(m, s_max[i]);
  const int wgt = exp2_neg_q15(lut, (long long)logit - m);
  unsigned long long s = (unsigned long long)wgt;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) s_sum[wp] = s;
  __syncthreads();
  unsigned long long tot = 0;
  for (int i = 0; i < VOCAB / 32; ++i) tot += s_sum[i];
  const uint32_t inv = recip_sum_q31(tot);
  const int p = (int)sat_i16(rhu64((long long)wgt * (long long)inv, 16));
  logits_out[b * VOCAB + c] = logit;
  probs_out[b * VOCAB + c] = (int16_t)p;
}

// x[b] = emb[ctx[b][pos]] with pos = fixed_pos >= 0 ? fixed_pos : lens[b] - 1
// (the token embedding without positions, lib.rs:13275-13289).
__global__ void embed_token_kernel(const uint8_t* __restrict__ ctx, long long cap, const int32_t* __restrict__ lens,
                                   int fixed_pos, const int16_t* __restrict__ emb, int d, int B, int16_t* __restrict__ x) {
  const long long n = (long long)B * d;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int b = (int)(i / d), c = (int)(i % d);
    const int pos = fixed_pos >= 0 ? fixed_pos : lens[b] - 1;
    x[i] = emb[(int)ctx[(long long)b * cap + pos] * d + c];
  }
}

__device__ __forceinline__ uint64_t fnv_byte(uint64_t h, uint8_t v) { return (h ^ v) * 0x100000001b3ull; }
__device__ __forceinline__ uint64_t fnv_u64(uint64_t h, uint64_t v) {
#pragma unroll
  for (int i = 0; i < 8; ++i) h = fnv_byte(h, (uint8_t)(v >> (8 * i)));
  return h;
}

// One CTA of 256 threads per sequence: pick the next byte from the row,
// append it to the context and record it (select_byte_from_row_with_priors
// with no priors and no constraints, lib.rs:18979-19100).
__global__ void __launch_bounds__(VOCAB) select_kernel(const int32_t* __restrict__ logits,
                                                       const int16_t* __restrict__ probs, int strategy, int top_k,
                                                       unsigned long long seed, int step, uint8_t* __restrict__ ctx,
                                                       long long cap, int32_t* __restrict__ lens, int steps,
                                                       uint8_t* __restrict__ tokens, int32_t* __restrict__ pick_logit,
                                                       int16_t* __restrict__ pick_prob) {
  __shared__ int s_logit[VOCAB];
  __shared__ unsigned long long s_w[VOCAB];  // weight of the candidate of each rank
  __shared__ int s_cand[VOCAB];              // class of each rank
  __shared__ unsigned long long s_hash;
  __shared__ int s_pick;
  const int b = blockIdx.x, c = threadIdx.x;
  const int lg = logits[b * VOCAB + c];
  const int pr = probs[b * VOCAB + c];
  s_logit[c] = lg;
  __syncthreads();
  // rank of class c in the order (logit descending, index ascending)
  int rank = 0;
  for (int j = 0; j < VOCAB; ++j) {
    const int l = s_logit[j];
    rank += (l > lg) || (l == lg && j < c);
  }
  const int k = (top_k <= 0 || top_k > VOCAB) ? VOCAB : top_k;
  s_cand[rank] = c;
  s_w[rank] = rank < k ? (unsigned long long)max(pr, 0) : 0ull;
  const int len = lens[b];
  if (c == 0 && strategy == 1) {
    // decode_sample_u64: StableHasher over the seed, the step and the whole context
    uint64_t h = 0xcbf29ce484222325ull;
    h = fnv_u64(h, seed);
    h = fnv_u64(h, (uint64_t)step);
    h = fnv_u64(h, (uint64_t)len);
    const uint8_t* cb = ctx + (long long)b * cap;
    for (int i = 0; i < len; ++i) h = fnv_byte(h, cb[i]);
    h += 0x9e3779b97f4a7c15ull;  // splitmix64
    h = (h ^ (h >> 30)) * 0xbf58476d1ce4e5b9ull;
    h = (h ^ (h >> 27)) * 0x94d049bb133111ebull;
    s_hash = h ^ (h >> 31);
  }
  __syncthreads();
  if (c == 0) {
    int pick = s_cand[0];  // greedy: the argmax (lowest index among equal logits)
    if (strategy == 1) {
      unsigned long long mass = 0;
      for (int r = 0; r < k; ++r) mass += s_w[r];
      if (mass != 0) {
        unsigned long long th = s_hash % mass;
        for (int r = 0; r < k; ++r) {
          if (th < s_w[r]) {
            pick = s_cand[r];
            break;
          }
          th -= s_w[r];
        }
      }
    }
    s_pick = pick;
    ctx[(long long)b * cap + len] = (uint8_t)pick;
    lens[b] = len + 1;
    tokens[(long long)b * steps + step] = (uint8_t)pick;
  }
  __syncthreads();
  if (c == s_pick) {
    if (pick_logit) pick_logit[(long long)b * steps + step] = lg;
    if (pick_prob) pick_prob[(long long)b * steps + step] = (int16_t)pr;
  }
}

}  // namespace

cudaError_t launch_gen_windows(const uint8_t* ctx, size_t cap, const int32_t* lens, size_t S, size_t B, uint8_t* win,
                               cudaStream_t s) {
  const size_t n = B * S;
  const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
  ProfScope prof("gen_windows", s, 0.0, 2.0 * (double)n);
  window_kernel<<<blocks, 256, 0, s>>>(ctx, (long long)cap, lens, (int)S, (int)B, win);
  return cudaGetLastError();
}

cudaError_t launch_embed(const uint8_t* win, size_t rows, size_t S, size_t d, const int16_t* emb,
                         const int16_t* pos, int16_t* x, cudaStream_t s) {
  const size_t n = rows * d;
  const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 16);
  ProfScope prof("embed", s, 0.0, 6.0 * (double)n);
  embed_kernel<<<blocks, 256, 0, s>>>(win, (int)S, (int)d, emb, pos, (long long)rows, x);
  return cudaGetLastError();
}

cudaError_t launch_embed_token(const uint8_t* ctx, size_t cap, const int32_t* lens, int fixed_pos,
                               const int16_t* emb, size_t d, size_t B, int16_t* x, cudaStream_t s) {
  const size_t n = B * d;
  const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
  ProfScope prof("embed_token", s, 0.0, 4.0 * (double)n);
  embed_token_kernel<<<blocks, 256, 0, s>>>(ctx, (long long)cap, lens, fixed_pos, emb, (int)d, (int)B, x);
  return cudaGetLastError();
}

cudaError_t launch_head_rows(const int16_t* x, size_t row_stride, size_t row0, size_t B, size_t d,
                             const nsrl_linear_params* head, int32_t* logits, int16_t* probs, nsrl_device_status* st,
                             cudaStream_t s) {
  if (d > 4096) return cudaErrorInvalidValue;
  ProfScope prof("head_rows", s, 2.0 * (double)B * VOCAB * d, 2.0 * B * d + (double)VOCAB * d + 6.0 * B * VOCAB);
  head_row_kernel<<<(unsigned)B, VOCAB, 0, s>>>(x, (long long)row_stride, (long long)row0, (int)d, head->weights,
                                               head->bias, head->scales, logits, probs, st);
  return cudaGetLastError();
}

cudaError_t launch_select(const int32_t* logits, const int16_t* probs, size_t B, int strategy, int top_k,
                          uint64_t seed, int step, uint8_t* ctx, size_t cap, int32_t* lens, int steps,
                          uint8_t* tokens, int32_t* pick_logit, int16_t* pick_prob, cudaStream_t s) {
  ProfScope prof("select_byte", s, 0.0, 6.0 * B * VOCAB);
  select_kernel<<<(unsigned)B, VOCAB, 0, s>>>(logits, probs, strategy, top_k, (unsigned long long)seed, step, ctx,
                                             (long long)cap, lens, steps, tokens, pick_logit, pick_prob);
  return cudaGetLastError();
}

}  // namespace nsrl
