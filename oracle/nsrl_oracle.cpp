// CPU oracle for the NSRL integer transformer hot path -- TEST INFRASTRUCTURE.
//
// A scalar restatement of the reference's Rust CPU kernels, used only by the
// parity tests, the smoke check and the CPU-baseline leg of the benchmark.
// The product (nsrl_b200/) never links or calls it.  Each function cites the
// reference file:line whose behaviour it restates; paths are relative to the
// reference project root.
#include "nsrl_oracle.hpp"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace orc {

int16_t RSQRT_LUT[128];
int16_t EXP2_LUT[256];
uint32_t RECIP_LUT[128];

// crates/nsrl-core/src/rsqrt_lut_8bit.rs:1-56 (tables), re-derived from their
// definitions with exact integer arithmetic where that is cheap.
void init_luts() {
  for (int m = 128; m < 256; ++m) {
    // largest r with m * (2r - 1)^2 <= 2^39  <=>  r = round(32768 / sqrt(m / 128))
    uint64_t r = (uint64_t)std::sqrt((long double)(1ULL << 39) / m) / 2 + 3;
    while ((uint64_t)m * (2 * r - 1) * (2 * r - 1) > (1ULL << 39)) --r;
    RSQRT_LUT[m - 128] = (int16_t)std::min<uint64_t>(r, 32767);
    RECIP_LUT[m - 128] = (uint32_t)(((1ULL << 31) + (uint64_t)(m / 2)) / (uint64_t)m);
  }
  for (int f = 0; f < 256; ++f) {
    long double v = 32768.0L * std::exp2l(-(long double)f / 256.0L);
    long long r = std::llroundl(v);
    EXP2_LUT[f] = (int16_t)std::min<long long>(r, 32767);
  }
}

// numeric.rs:13-19
int8_t saturate_i8(int64_t v) { return (int8_t)std::clamp<int64_t>(v, -128, 127); }
int16_t saturate_i16(int64_t v) { return (int16_t)std::clamp<int64_t>(v, -32768, 32767); }

static int64_t sat_add_i64(int64_t a, int64_t b) {
  int64_t r;
  if (__builtin_add_overflow(a, b, &r)) return b > 0 ? INT64_MAX : INT64_MIN;
  return r;
}

// numeric.rs:47-57 (release build: the shift is clamped to MAX_RIGHT_SHIFT)
int64_t rhu(int64_t v, uint8_t shift) {
  if (shift == 0) return v;
  int s = std::min<int>(shift, MAX_RIGHT_SHIFT);
  int64_t bias = (int64_t)1 << (s - 1);
  return sat_add_i64(v, bias) >> s;
}

// numeric.rs:59-70
int16_t requantize_i32_to_i16(int32_t acc, FixedScale s) {
  if (s.multiplier == 1 && s.right_shift == 0) return saturate_i16(acc);
  int64_t wide = (int64_t)acc * (int64_t)s.multiplier;
  return saturate_i16(rhu(wide, s.right_shift));
}

// numeric.rs:25-45
static bool residual_add(const int16_t* skip, const int16_t* block, int16_t* out, size_t n,
                         uint64_t* sat_count) {
  uint64_t c = 0;
  for (size_t i = 0; i < n; ++i) {
    int32_t wide = (int32_t)skip[i] + (int32_t)block[i];
    if (wide < -32768 || wide > 32767) ++c;
    out[i] = saturate_i16(wide);
  }
  if (sat_count) *sat_count += c;
  return true;
}

// lut.rs:16-40
struct Norm {
  uint8_t mantissa;
  int16_t exponent;
};
static bool normalize_u64(uint64_t v, Norm* out) {
  if (v == 0) return false;
  int msb = 63 - __builtin_clzll(v);
  if (msb >= 7) {
    int sh = msb - 7;
    out->mantissa = (uint8_t)(v >> sh);
    out->exponent = (int16_t)sh;
  } else {
    int sh = 7 - msb;
    out->mantissa = (uint8_t)(v << sh);
    out->exponent = (int16_t)(-sh);
  }
  return true;
}

// ---------------------------------------------------------------- linear ---
// linear.rs:144-173 -- the i32 wrapping fast path is exact when
// |bias| + K * 127 * 32767 <= i32::MAX; otherwise every prefix is checked.
static const int64_t MAX_I8_I16_PRODUCT = 127LL * 32767LL;

static bool linear_params_valid(const LinearParams& p) {  // linear.rs:56-78
  return p.input_dim != 0 && p.output_dim != 0 && p.weights != nullptr && p.scales != nullptr;
}

// linear.rs:228-324 (generic i8 kernel; the tile-4 grouping only changes the
// order in which rows are visited, not any row's result)
static bool linear_row(const int16_t* x, const LinearParams& p, int16_t* y) {
  const size_t K = p.input_dim, N = p.output_dim;
  __int128 mps128 = (__int128)K * MAX_I8_I16_PRODUCT;
  int64_t mps = mps128 > INT64_MAX ? INT64_MAX : (int64_t)mps128;
  for (size_t n = 0; n < N; ++n) {
    const int8_t* w = p.weights + n * K;
    int32_t b = p.bias ? p.bias[n] : 0;
    int64_t babs = b < 0 ? -(int64_t)b : (int64_t)b;
    bool fits = sat_add_i64(babs, mps) <= (int64_t)INT32_MAX;
    int32_t acc;
    if (fits) {
      int64_t a = b;
      for (size_t k = 0; k < K; ++k) a += (int64_t)x[k] * (int64_t)w[k];
      acc = (int32_t)a;
    } else {
      acc = b;
      for (size_t k = 0; k < K; ++k) {
        int32_t prod = (int32_t)x[k] * (int32_t)w[k];
        if (__builtin_add_overflow(acc, prod, &acc)) return false;
      }
    }
    y[n] = requantize_i32_to_i16(acc, p.scales[n]);
  }
  return true;
}

// ------------------------------------------------------------- attention ---
// attention.rs:77-87
static bool is_power_of_four(size_t v) {
  return v != 0 && (v & (v - 1)) == 0 && (__builtin_ctzll(v) % 2 == 0);
}
static int sqrt_power_of_four_shift(size_t v) { return is_power_of_four(v) ? __builtin_ctzll(v) / 2 : -1; }

// attention.rs:117-140 (head dims stay far below the i64 bound of
// 8,589,934,591 products, so the wrapping branch is the exact one)
static bool qk_dot(const int16_t* q, const int16_t* k, size_t h, int shift, int32_t* out) {
  int64_t acc = 0;
  for (size_t i = 0; i < h; ++i) acc += (int64_t)q[i] * (int64_t)k[i];
  int64_t s = acc >> shift;
  if (s < INT32_MIN || s > INT32_MAX) return false;
  *out = (int32_t)s;
  return true;
}

// attention.rs:142-158
int16_t base2_exp_neg_q15(int32_t delta) {
  if (delta >= 0) return 32767;
  int64_t mag = -(int64_t)delta;
  int64_t ish = mag >> LOGIT_FRAC_BITS;
  if (ish >= 15) return 0;
  int frac = (int)(mag & 255);
  return (int16_t)(EXP2_LUT[frac] >> ish);
}

// attention.rs:181-193
static bool reciprocal_sum_q31(uint64_t sum, uint32_t* out) {
  Norm n;
  if (!normalize_u64(sum, &n)) return false;
  uint64_t base = RECIP_LUT[n.mantissa - 128];
  uint64_t r;
  if (n.exponent >= 0) {
    unsigned sh = (unsigned)n.exponent;
    r = sh >= 63 ? 0 : base >> sh;
  } else {
    unsigned sh = (unsigned)(-n.exponent);  // at most 7: Rust's checked_shl only rejects sh >= 64
    r = base << sh;
  }
  *out = (uint32_t)std::min<uint64_t>(r, 0xFFFFFFFFULL);
  return true;
}

static int32_t sat_sub_i32(int32_t a, int32_t b) {
  int64_t r = (int64_t)a - (int64_t)b;
  return (int32_t)std::clamp<int64_t>(r, INT32_MIN, INT32_MAX);
}

// attention.rs:261-293
static bool base2_softmax(const int32_t* logits, size_t n, int16_t* out, uint64_t* sum_out) {
  if (n == 0) return false;
  bool any = false;
  int32_t mx = INT32_MIN;
  for (size_t i = 0; i < n; ++i)
    if (logits[i] != MASKED_LOGIT) {
      if (!any || logits[i] > mx) mx = logits[i];
      any = true;
    }
  if (!any) return false;
  uint64_t sum = 0;
  for (size_t i = 0; i < n; ++i) {
    if (logits[i] == MASKED_LOGIT) {
      out[i] = 0;
      continue;
    }
    int16_t w = base2_exp_neg_q15(sat_sub_i32(logits[i], mx));
    out[i] = w;
    sum += (uint64_t)w;  // never overflows: n * 32767 < 2^64
  }
  uint32_t inv;
  if (!reciprocal_sum_q31(sum, &inv)) return false;
  for (size_t i = 0; i < n; ++i) out[i] = saturate_i16(rhu((int64_t)out[i] * (int64_t)inv, 16));
  if (sum_out) *sum_out = sum;
  return true;
}

// attention.rs:596-668
static bool weight_v(const int16_t* p, size_t L, const int16_t* values, size_t vstride, size_t vd,
                     int16_t* out) {
  for (size_t i = 0; i < L; ++i)
    if (p[i] < 0) return false;
  for (size_t c = 0; c < vd; ++c) {
    int64_t acc = 0;
    for (size_t i = 0; i < L; ++i) acc += (int64_t)p[i] * (int64_t)values[i * vstride + c];
    out[c] = saturate_i16(rhu(acc, Q15_SHIFT));
  }
  return true;
}

// attention.rs:671-725
static bool attention_row(const int16_t* q, const int16_t* keys, const int16_t* values, size_t kd,
                          size_t vd, size_t L, const uint8_t* mask, int32_t* logits, int16_t* probs,
                          int16_t* out, uint64_t* sum) {
  if (kd == 0 || vd == 0 || L == 0) return false;
  int shift = sqrt_power_of_four_shift(kd);
  if (shift < 0) return false;
  for (size_t i = 0; i < L; ++i) {
    if (mask && mask[i]) {
      logits[i] = MASKED_LOGIT;
      continue;
    }
    if (!qk_dot(q, keys + i * kd, kd, shift, &logits[i])) return false;
  }
  if (!base2_softmax(logits, L, probs, sum)) return false;
  return weight_v(probs, L, values, vd, vd, out);
}

// attention.rs:1585-1634 (shape rules of validate_self_attention_shapes)
static bool attention_shapes_valid(size_t S, size_t d, size_t H, const LinearParams* lp) {
  if (S == 0 || d == 0 || H == 0 || d % H != 0) return false;
  if (!is_power_of_four(d / H)) return false;
  for (int i = 0; i < 4; ++i)
    if (lp[i].input_dim != d || lp[i].output_dim != d || !linear_params_valid(lp[i])) return false;
  return true;
}

// attention.rs:742-877 -- one sequence of S tokens.
static bool self_attention_seq(const int16_t* x, size_t S, size_t d, size_t H, bool causal,
                               const LinearParams* lp, int16_t* out) {
  if (!attention_shapes_valid(S, d, H, lp)) return false;
  const size_t hd = d / H;
  const int shift = sqrt_power_of_four_shift(hd);
  std::vector<int16_t> q(S * d), k(S * d), v(S * d), ctx(S * d), probs(S);
  std::vector<int32_t> logits(S);
  for (size_t t = 0; t < S; ++t) {
    if (!linear_row(x + t * d, lp[0], &q[t * d])) return false;
    if (!linear_row(x + t * d, lp[1], &k[t * d])) return false;
    if (!linear_row(x + t * d, lp[2], &v[t * d])) return false;
  }
  for (size_t t = 0; t < S; ++t) {
    for (size_t h = 0; h < H; ++h) {
      const size_t off = h * hd;
      const size_t L = causal ? t + 1 : S;
      for (size_t j = 0; j < L; ++j)
        if (!qk_dot(&q[t * d + off], &k[j * d + off], hd, shift, &logits[j])) return false;
      if (!base2_softmax(logits.data(), L, probs.data(), nullptr)) return false;
      // the context product reads values with a stride of d_model
      for (size_t c = 0; c < hd; ++c) {
        int64_t acc = 0;
        for (size_t j = 0; j < L; ++j) acc += (int64_t)probs[j] * (int64_t)v[j * d + off + c];
        ctx[t * d + off + c] = saturate_i16(rhu(acc, Q15_SHIFT));
      }
    }
  }
  for (size_t t = 0; t < S; ++t)
    if (!linear_row(&ctx[t * d], lp[3], out + t * d)) return false;
  return true;
}

// -------------------------------------------------------------- rms norm ---
// rms_norm.rs:48-66
static bool integer_rsqrt_q30(uint64_t value, int64_t* out) {
  Norm n;
  if (!normalize_u64(value, &n)) return false;
  int64_t inv = (int64_t)RSQRT_LUT[n.mantissa - 128] << 15;
  int32_t exponent = (int32_t)n.exponent + 7;
  if (exponent & 1) {
    int64_t m;
    if (__builtin_mul_overflow(inv, INV_SQRT_2_Q15, &m)) return false;
    inv = rhu(m, 15);
  }
  int32_t half = exponent >= 0 ? exponent / 2 : -((-exponent + 1) / 2);  // div_euclid by 2
  if (half >= 0) {
    inv = half >= 63 ? 0 : inv >> half;
  } else {
    int sh = -half;
    if (sh >= 64) return false;
    inv = (int64_t)((uint64_t)inv << sh);
  }
  *out = inv;
  return true;
}

// rms_norm.rs:68-89
static bool rms_norm_row(const int16_t* x, const int16_t* g, size_t d, uint64_t eps, int16_t* y) {
  if (d == 0) return false;
  uint64_t sum = 0;
  for (size_t i = 0; i < d; ++i) sum += (uint64_t)((int64_t)x[i] * (int64_t)x[i]);
  uint64_t mean = sum / d;
  uint64_t v;
  if (__builtin_add_overflow(mean, eps, &v)) return false;
  int64_t inv;
  if (!integer_rsqrt_q30(v, &inv)) return false;
  for (size_t i = 0; i < d; ++i) {
    int64_t vw = (int64_t)x[i] * (int64_t)g[i];
    int64_t sc;
    if (__builtin_mul_overflow(vw, inv, &sc)) return false;
    y[i] = saturate_i16(rhu(sc, RMSNORM_INV_RMS_SHIFT));
  }
  return true;
}

// ------------------------------------------------------------------- mlp ---
// mlp.rs:150-170
static int16_t hard_silu_gate_q15(int16_t v) {
  int32_t b = ((int32_t)v >> HARD_SILU_GATE_SHIFT) + HARD_SILU_GATE_BIAS_Q15;
  return (int16_t)std::clamp<int32_t>(b, 0, 32767);
}
static int16_t hard_silu_q15(int16_t v) {
  return saturate_i16(rhu((int64_t)v * (int64_t)hard_silu_gate_q15(v), 15));
}
int16_t gated_activation(int16_t up, int16_t gate) {
  return saturate_i16(rhu((int64_t)up * (int64_t)hard_silu_q15(gate), 15));
}

// mlp.rs:211-254 -- per token: up, gate, gated activation, down.
static bool gated_mlp_rows(const int16_t* x, size_t T, size_t d, size_t F, const LinearParams* lp,
                           int16_t* out) {
  if (T == 0 || d == 0 || F == 0) return false;
  if (lp[0].input_dim != d || lp[0].output_dim != F || lp[1].input_dim != d || lp[1].output_dim != F ||
      lp[2].input_dim != F || lp[2].output_dim != d)
    return false;
  for (int i = 0; i < 3; ++i)
    if (!linear_params_valid(lp[i])) return false;
  std::vector<int16_t> up(F), gate(F), gated(F);
  for (size_t t = 0; t < T; ++t) {
    if (!linear_row(x + t * d, lp[0], up.data())) return false;
    if (!linear_row(x + t * d, lp[1], gate.data())) return false;
    for (size_t f = 0; f < F; ++f) gated[f] = gated_activation(up[f], gate[f]);
    if (!linear_row(gated.data(), lp[2], out + t * d)) return false;
  }
  return true;
}

// ------------------------------------------------------------ threading ---
// Runs fn(i) for i in [0, n) over `threads` workers; returns false if any
// call returned false (the reference rejects the whole batch then).
template <class Fn>
static bool parallel_for(size_t n, int threads, Fn fn) {
  if (threads <= 1 || n <= 1) {
    for (size_t i = 0; i < n; ++i)
      if (!fn(i)) return false;
    return true;
  }
  std::atomic<size_t> next{0};
  std::atomic<bool> ok{true};
  std::vector<std::thread> pool;
  int nt = (int)std::min<size_t>((size_t)threads, n);
  for (int t = 0; t < nt; ++t)
    pool.emplace_back([&]() {
      for (;;) {
        size_t i = next.fetch_add(1);
        if (i >= n || !ok.load()) break;
        if (!fn(i)) ok.store(false);
      }
    });
  for (auto& th : pool) th.join();
  return ok.load();
}

// ------------------------------------------------------- bench-1m preset ---
// crates/nsrl-demo/src/bench.rs:912-925
struct SplitMix64 {
  uint64_t s;
  uint64_t next() {
    s += 0x9e3779b97f4a7c15ULL;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
  }
};

// bench.rs:928-975 (FNV-1a over little-endian bytes)
struct Fnv {
  uint64_t h = 0xcbf29ce484222325ULL;
  void u8(uint8_t v) { h = (h ^ v) * 0x100000001b3ULL; }
  void bytes(const void* p, size_t n) {
    const uint8_t* b = (const uint8_t*)p;
    for (size_t i = 0; i < n; ++i) u8(b[i]);
  }
  void str(const char* s) {
    bytes(s, strlen(s));
    u8(0xff);
  }
  void usize(uint64_t v) { bytes(&v, 8); }
  void i32(int32_t v) { bytes(&v, 4); }
  void i16s(const int16_t* v, size_t n) {
    usize(n);
    bytes(v, n * 2);
  }
  void i8s(const int8_t* v, size_t n) {
    usize(n);
    bytes(v, n);
  }
};

}  // namespace orc

using namespace orc;

extern "C" {

int orc_init() {
  init_luts();
  return 0;
}

void orc_luts(int16_t* rsqrt, int16_t* exp2, uint32_t* recip) {
  memcpy(rsqrt, RSQRT_LUT, sizeof(RSQRT_LUT));
  memcpy(exp2, EXP2_LUT, sizeof(EXP2_LUT));
  memcpy(recip, RECIP_LUT, sizeof(RECIP_LUT));
}

int64_t orc_rhu(int64_t v, uint8_t s) { return rhu(v, s); }
int16_t orc_requantize_i32_to_i16(int32_t acc, int32_t mult, uint8_t shift) {
  FixedScale s{mult, shift, {0, 0, 0}};
  return requantize_i32_to_i16(acc, s);
}
int orc_normalize_u64(uint64_t v, uint8_t* mant, int16_t* expo) {
  Norm n;
  if (!normalize_u64(v, &n)) return 1;
  *mant = n.mantissa;
  *expo = n.exponent;
  return 0;
}
int16_t orc_base2_exp_neg_q15(int32_t d) { return base2_exp_neg_q15(d); }
int orc_reciprocal_sum_q31(uint64_t s, uint32_t* out) { return reciprocal_sum_q31(s, out) ? 0 : 1; }
int orc_base2_softmax_i32_q15(const int32_t* l, size_t n, int16_t* out, uint64_t* sum) {
  return base2_softmax(l, n, out, sum) ? 0 : 1;
}
int orc_integer_rsqrt_q30(uint64_t v, int64_t* out) { return integer_rsqrt_q30(v, out) ? 0 : 1; }
int16_t orc_gated_activation(int16_t up, int16_t gate) { return gated_activation(up, gate); }
int orc_residual_add(const int16_t* skip, const int16_t* block, int16_t* out, size_t n, uint64_t* sat) {
  if (sat) *sat = 0;
  return residual_add(skip, block, out, n, sat) ? 0 : 1;
}

// linear.rs:228-324 over M independent rows.
int orc_linear(const int16_t* x, size_t M, const LinearParams* p, int16_t* y, int threads) {
  if (!linear_params_valid(*p)) return 1;
  const size_t K = p->input_dim, N = p->output_dim;
  const size_t chunk = 256;
  size_t nchunks = (M + chunk - 1) / chunk;
  bool ok = parallel_for(nchunks, threads, [&](size_t c) {
    for (size_t m = c * chunk; m < std::min(M, (c + 1) * chunk); ++m)
      if (!linear_row(x + m * K, *p, y + m * N)) return false;
    return true;
  });
  return ok ? 0 : 1;
}

int orc_rms_norm_rows(const int16_t* x, size_t T, size_t d, const int16_t* g, uint64_t eps, int16_t* y) {
  for (size_t t = 0; t < T; ++t)
    if (!rms_norm_row(x + t * d, g, d, eps, y + t * d)) return 1;
  return 0;
}

int orc_attention_row(const int16_t* q, const int16_t* keys, const int16_t* values, size_t kd, size_t vd,
                      size_t L, const uint8_t* mask, int32_t* logits, int16_t* probs, int16_t* out,
                      uint64_t* sum) {
  return attention_row(q, keys, values, kd, vd, L, mask, logits, probs, out, sum) ? 0 : 1;
}

// attention.rs:742-877 over B independent sequences of S tokens.
// lp = {q, k, v, o}.
int orc_self_attention(const int16_t* x, size_t B, size_t S, size_t d, size_t H, int causal,
                       const LinearParams* lp, int16_t* out, int threads) {
  bool ok = parallel_for(B, threads, [&](size_t b) {
    return self_attention_seq(x + b * S * d, S, d, H, causal != 0, lp, out + b * S * d);
  });
  return ok ? 0 : 1;
}

// attention.rs:1541-1583 over B sequences: RMS rows, attention, residual.
int orc_prenorm_attention_block(const int16_t* x, size_t B, size_t S, size_t d, size_t H, int causal,
                                const int16_t* gamma, uint64_t eps, const LinearParams* lp, int16_t* y,
                                uint64_t* sat_count, int threads) {
  std::vector<uint64_t> sats(B, 0);
  bool ok = parallel_for(B, threads, [&](size_t b) {
    const int16_t* xb = x + b * S * d;
    std::vector<int16_t> norm(S * d), att(S * d);
    for (size_t t = 0; t < S; ++t)
      if (!rms_norm_row(xb + t * d, gamma, d, eps, &norm[t * d])) return false;
    if (!self_attention_seq(norm.data(), S, d, H, causal != 0, lp, att.data())) return false;
    return residual_add(xb, att.data(), y + b * S * d, S * d, &sats[b]);
  });
  if (sat_count) {
    *sat_count = 0;
    for (auto s : sats) *sat_count += s;
  }
  return ok ? 0 : 1;
}

// mlp.rs:555-594 over T tokens: RMS rows, gated MLP, residual.  lp = {up, gate, down}.
int orc_prenorm_mlp_block(const int16_t* x, size_t T, size_t d, size_t F, const int16_t* gamma,
                          uint64_t eps, const LinearParams* lp, int16_t* y, uint64_t* sat_count,
                          int threads) {
  const size_t chunk = 128;
  size_t nchunks = (T + chunk - 1) / chunk;
  std::vector<uint64_t> sats(nchunks, 0);
  bool ok = parallel_for(nchunks, threads, [&](size_t c) {
    size_t t0 = c * chunk, t1 = std::min(T, t0 + chunk), n = t1 - t0;
    std::vector<int16_t> norm(n * d), mo(n * d);
    for (size_t t = 0; t < n; ++t)
      if (!rms_norm_row(x + (t0 + t) * d, gamma, d, eps, &norm[t * d])) return false;
    if (!gated_mlp_rows(norm.data(), n, d, F, lp, mo.data())) return false;
    return residual_add(x + t0 * d, mo.data(), y + t0 * d, n * d, &sats[c]);
  });
  if (sat_count) {
    *sat_count = 0;
    for (auto s : sats) *sat_count += s;
  }
  return ok ? 0 : 1;
}

// KV-cache decode attention: for each (sequence b, head h) the single query
// q[b][h] attends over the first lens[b] cached keys/values of that head,
// which is attention.rs:671-725 with no mask.  Cache layout [B][Lmax][d].
int orc_decode_attention(const int16_t* q, const int16_t* kc, const int16_t* vc, const int32_t* lens,
                         size_t B, size_t H, size_t hd, size_t Lmax, int16_t* ctx, int threads) {
  const size_t d = H * hd;
  bool ok = parallel_for(B * H, threads, [&](size_t i) {
    size_t b = i / H, h = i % H;
    size_t L = (size_t)lens[b];
    if (L == 0 || L > Lmax) return false;
    std::vector<int16_t> kk(L * hd), vv(L * hd), probs(L);
    std::vector<int32_t> logits(L);
    for (size_t j = 0; j < L; ++j) {
      memcpy(&kk[j * hd], kc + (b * Lmax + j) * d + h * hd, hd * 2);
      memcpy(&vv[j * hd], vc + (b * Lmax + j) * d + h * hd, hd * 2);
    }
    return attention_row(q + b * d + h * hd, kk.data(), vv.data(), hd, hd, L, nullptr, logits.data(),
                         probs.data(), ctx + b * d + h * hd, nullptr);
  });
  return ok ? 0 : 1;
}

// crates/nsrl-demo/src/bench.rs:230-380 and :707-843 -- the bench-1m preset
// (4 blocks, seq 128, d_model 128, 2 heads, hidden 512, ternary weights,
// shifts qk 10 / v 7 / o 5 / up 9 / gate 8 / down 5, RMS gamma 8192, eps 1).
// Writes the model, input and output FNV-1a hashes and the residual
// saturation total.
int orc_bench1m(uint64_t* model_hash, uint64_t* input_hash, uint64_t* output_hash, uint64_t* sat_total) {
  const size_t S = 128, d = 128, H = 2, F = 512, blocks = 4;
  const uint64_t seed = 0x4e53524c5f314d21ULL;
  SplitMix64 rng{seed};
  Fnv mh;
  mh.str("nsrl.benchmark_trace.v1");
  mh.str("bench-1m");
  mh.usize(S);
  mh.usize(d);
  mh.usize(H);
  mh.usize(F);
  mh.usize(blocks);
  auto ternary = [&](size_t n) {
    std::vector<int8_t> w(n);
    for (size_t i = 0; i < n; ++i) {
      uint64_t r = rng.next() & 7;
      w[i] = r == 0 ? -1 : (r == 1 ? 1 : 0);
    }
    return w;
  };
  auto scales = [](size_t n, uint8_t sh) { return std::vector<FixedScale>(n, FixedScale{1, sh, {0, 0, 0}}); };
  auto hash_scales = [&](const std::vector<FixedScale>& s) {
    mh.usize(s.size());
    for (auto& x : s) {
      mh.i32(x.multiplier);
      mh.u8(x.right_shift);
    }
  };
  struct Blk {
    std::vector<int8_t> q, k, v, o, up, gate, down;
  };
  std::vector<Blk> bl(blocks);
  auto qk_s = scales(d, 10), v_s = scales(d, 7), o_s = scales(d, 5), up_s = scales(F, 9),
       gate_s = scales(F, 8), down_s = scales(d, 5);
  for (auto& b : bl) {
    b.q = ternary(d * d);
    b.k = ternary(d * d);
    b.v = ternary(d * d);
    b.o = ternary(d * d);
    b.up = ternary(F * d);
    b.gate = ternary(F * d);
    b.down = ternary(d * F);
    for (auto* w : {&b.q, &b.k, &b.v, &b.o, &b.up, &b.gate, &b.down}) mh.i8s(w->data(), w->size());
    for (auto* s : {&qk_s, &v_s, &o_s, &up_s, &gate_s, &down_s}) hash_scales(*s);
  }
  // bench.rs:822-832
  SplitMix64 irng{seed ^ 0xa17e57116d5a1234ULL};
  std::vector<int16_t> cur(S * d), next(S * d), mid(S * d);
  for (size_t i = 0; i < S * d; ++i) {
    int16_t token = (int16_t)(i / d), channel = (int16_t)(i % d);
    int16_t noise = (int16_t)((int16_t)(irng.next() >> 53) - 512);
    cur[i] = (int16_t)(((token & 31) - 16) * 16 + ((channel & 15) - 8) * 8 + noise);
  }
  Fnv ih;
  ih.i16s(cur.data(), cur.size());
  std::vector<int16_t> gamma(d, 8192);
  uint64_t sat = 0;
  for (auto& b : bl) {
    LinearParams ap[4] = {{b.q.data(), nullptr, qk_s.data(), d, d},
                          {b.k.data(), nullptr, qk_s.data(), d, d},
                          {b.v.data(), nullptr, v_s.data(), d, d},
                          {b.o.data(), nullptr, o_s.data(), d, d}};
    LinearParams mp[3] = {{b.up.data(), nullptr, up_s.data(), d, F},
                          {b.gate.data(), nullptr, gate_s.data(), d, F},
                          {b.down.data(), nullptr, down_s.data(), F, d}};
    uint64_t s1 = 0, s2 = 0;
    if (orc_prenorm_attention_block(cur.data(), 1, S, d, H, 1, gamma.data(), 1, ap, mid.data(), &s1, 1))
      return 1;
    if (orc_prenorm_mlp_block(mid.data(), S, d, F, gamma.data(), 1, mp, next.data(), &s2, 1)) return 1;
    sat += s1 + s2;
    std::swap(cur, next);
  }
  Fnv oh;
  oh.i16s(cur.data(), cur.size());
  *model_hash = mh.h;
  *input_hash = ih.h;
  *output_hash = oh.h;
  *sat_total = sat;
  return 0;
}

}  // extern "C"

// ------------------------------------------------------ training exchange ---
// crates/nsrl-train-core/src/lib.rs:1732-1757 (round half away from zero)
static bool round_ratio_i64(int64_t num, int64_t den, int64_t* out) {
  if (den <= 0) return false;
  int64_t half = den / 2;
  if (num >= 0) {
    int64_t t;
    if (__builtin_add_overflow(num, half, &t)) return false;
    *out = t / den;
  } else {
    if (num == INT64_MIN) return false;
    int64_t t;
    if (__builtin_add_overflow(-num, half, &t)) return false;
    *out = -(t / den);
  }
  return true;
}

extern "C" {

// crates/nsrl-train-core/src/lib.rs:344-384, one call per row r:
// acc[n][k] += g[r][n] * x[r][k] (checked i64, zeros skipped), count += 1.
int orc_accumulate_linear_gradient_i64(const int16_t* x, const int32_t* g, size_t rows, size_t K, size_t N,
                                       int64_t* acc, uint64_t* count) {
  if (K == 0 || N == 0) return 1;
  for (size_t r = 0; r < rows; ++r) {
    const int16_t* xr = x + r * K;
    const int32_t* gr = g + r * N;
    for (size_t n = 0; n < N; ++n) {
      if (gr[n] == 0) continue;
      for (size_t k = 0; k < K; ++k) {
        if (xr[k] == 0) continue;
        int64_t prod = (int64_t)gr[n] * (int64_t)xr[k];
        if (__builtin_add_overflow(acc[n * K + k], prod, &acc[n * K + k])) return 2;
      }
    }
    *count += 1;
  }
  return 0;
}

// crates/nsrl-train-core/src/lib.rs:386-465.  stats = {saturations, zero deltas, |delta| sum}.
int orc_apply_linear_gradient_i64_to_i8(int64_t* acc, int64_t* residuals, int8_t* weights, size_t len,
                                        uint64_t* count, int32_t lr, uint8_t shift, int carry, uint64_t* stats) {
  stats[0] = stats[1] = stats[2] = 0;
  if (lr <= 0 || shift > MAX_RIGHT_SHIFT) return 1;
  if (*count == 0) return 0;
  if (*count > (uint64_t)INT64_MAX) return 1;
  const int64_t den = (int64_t)*count;
  for (size_t i = 0; i < len; ++i) {
    if (acc[i] == 0) continue;
    int64_t avg;
    if (!round_ratio_i64(acc[i], den, &avg)) return 2;
    int64_t product;
    if (__builtin_mul_overflow(avg, (int64_t)lr, &product)) return 2;
    if (carry && __builtin_add_overflow(product, residuals[i], &product)) return 2;
    int64_t scaled = rhu(product, shift);
    int64_t next_res = 0;
    if (carry && shift != 0) {
      __int128 applied = (__int128)scaled << shift;
      __int128 res = (__int128)product - applied;
      if (res < INT64_MIN || res > INT64_MAX) return 2;
      next_res = (int64_t)res;
    }
    int64_t delta = -scaled;
    if (delta == 0) stats[1] += 1;
    int8_t prev = weights[i];
    int64_t unclamped;
    if (__builtin_add_overflow((int64_t)prev, delta, &unclamped)) return 2;
    int8_t clamped = saturate_i8(unclamped);
    if ((int64_t)clamped != unclamped) {
      stats[0] += 1;
      residuals[i] = 0;
    } else {
      residuals[i] = next_res;
    }
    int64_t applied_delta = (int64_t)clamped - (int64_t)prev;
    stats[2] += (uint64_t)(applied_delta < 0 ? -applied_delta : applied_delta);
    weights[i] = clamped;
  }
  for (size_t i = 0; i < len; ++i) acc[i] = 0;
  *count = 0;
  return 0;
}

// crates/nsrl-train/src/lib.rs:7443-7471: merge worker results in worker
// order with checked adds.  parts: [workers][len].
int orc_merge_i64(const int64_t* parts, size_t workers, size_t len, const uint64_t* counts, int64_t* out,
                  uint64_t* count_out) {
  uint64_t c = 0;
  for (size_t i = 0; i < len; ++i) out[i] = 0;
  for (size_t w = 0; w < workers; ++w) {
    if (__builtin_add_overflow(c, counts[w], &c)) return 2;
    for (size_t i = 0; i < len; ++i)
      if (__builtin_add_overflow(out[i], parts[w * len + i], &out[i])) return 2;
  }
  *count_out = c;
  return 0;
}

}  // extern "C"

// ============================================================ training step ==
// Rows of the integer training step: backward-input linears, gated-MLP and
// RMS-norm backward, softmax-attention backward, i64 weight-gradient
// accumulation, the byte-vocabulary output head and the map-reduce worker
// loop of the reference's mini transformer.
namespace orc {

static const FixedScale IDENTITY_SCALE = {1, 0, {0, 0, 0}};
static const FixedScale OUTPUT_SCALE = {1, 8, {0, 0, 0}};  // nsrl-train-core/src/lib.rs:84-87
constexpr uint8_t FANIN_SHIFT = 1;                            // nsrl-train-core/src/lib.rs:48
constexpr int64_t LN2_Q15 = 22713;                            // nsrl-train/src/lib.rs:117
constexpr uint64_t TRAIN_RMS_EPS = 1;                         // nsrl-train/src/lib.rs:104
constexpr size_t VOCAB = 256;

static bool scale_ok(FixedScale s) { return s.multiplier >= 0 && s.right_shift <= MAX_RIGHT_SHIFT; }

// linear.rs:735-742 then the i32 conversion of :573-592
static bool prescale_grad(int16_t g, FixedScale s, int32_t* out) {
  if (!scale_ok(s)) return false;
  int64_t wide = rhu((int64_t)g * (int64_t)s.multiplier, s.right_shift);
  if (wide < INT32_MIN || wide > INT32_MAX) return false;
  *out = (int32_t)wide;
  return true;
}

// linear.rs:744-751
static bool requantize_i64_to_i16(int64_t acc, FixedScale s, int16_t* out) {
  if (!scale_ok(s)) return false;
  int64_t wide;
  if (__builtin_mul_overflow(acc, (int64_t)s.multiplier, &wide)) return false;
  *out = saturate_i16(rhu(wide, s.right_shift));
  return true;
}

// linear.rs:548-640: dx[k] = requant_i64(sum_n g'[n] * W[n][k]) for one row,
// g' the grad prescaled by the forward scales.  gin = null: identity scales.
static bool linear_backward_input_row(const int16_t* g, const LinearParams& p, const FixedScale* gin,
                                      int16_t* dx) {
  const size_t K = p.input_dim, N = p.output_dim;
  if (K == 0 || N == 0) return false;
  std::vector<int32_t> gs(N);
  for (size_t n = 0; n < N; ++n)
    if (!prescale_grad(g[n], p.scales[n], &gs[n])) return false;
  for (size_t k = 0; k < K; ++k) {
    int64_t acc = 0;
    for (size_t n = 0; n < N; ++n) {
      int64_t prod = (int64_t)gs[n] * (int64_t)p.weights[n * K + k];
      if (__builtin_add_overflow(acc, prod, &acc)) return false;
    }
    if (!requantize_i64_to_i16(acc, gin ? gin[k] : IDENTITY_SCALE, &dx[k])) return false;
  }
  return true;
}

// mlp.rs:162-164
static int16_t hard_silu_derivative_q15(int16_t v) { return (int16_t)(((int32_t)v >> 1) + HARD_SILU_GATE_BIAS_Q15); }

// mlp.rs:172-194
static void gated_activation_backward(int16_t up, int16_t gate, int16_t g, int16_t* gu, int16_t* gg) {
  const int64_t silu = hard_silu_q15(gate);
  const int64_t grad_up = rhu((int64_t)g * silu, 15);
  const int64_t grad_silu = rhu((int64_t)g * (int64_t)up, 15);
  const int64_t grad_gate = rhu(grad_silu * (int64_t)hard_silu_derivative_q15(gate), 15);
  *gu = saturate_i16(grad_up);
  *gg = saturate_i16(grad_gate);
}

// mlp.rs:256-357 (with identity grad-input scales, as the mini transformer
// passes them): per token down^T, the product rule, up^T and gate^T, and the
// saturating sum of the two input gradients (mlp.rs:712-727).
static bool gated_mlp_backward_input_rows(const int16_t* grad_out, size_t T, size_t d, size_t F,
                                          const LinearParams* lp, const int16_t* up, const int16_t* gate,
                                          int16_t* grad_up, int16_t* grad_gate, int16_t* grad_in, uint64_t* sat) {
  std::vector<int16_t> gg(F), gui(d), ggi(d);
  for (size_t t = 0; t < T; ++t) {
    if (!linear_backward_input_row(grad_out + t * d, lp[2], nullptr, gg.data())) return false;
    for (size_t f = 0; f < F; ++f)
      gated_activation_backward(up[t * F + f], gate[t * F + f], gg[f], &grad_up[t * F + f], &grad_gate[t * F + f]);
    if (!linear_backward_input_row(grad_up + t * F, lp[0], nullptr, gui.data())) return false;
    if (!linear_backward_input_row(grad_gate + t * F, lp[1], nullptr, ggi.data())) return false;
    for (size_t i = 0; i < d; ++i) {
      int32_t w = (int32_t)gui[i] + (int32_t)ggi[i];
      if (w < -32768 || w > 32767) ++*sat;
      grad_in[t * d + i] = saturate_i16(w);
    }
  }
  return true;
}

// rms_norm.rs:172-179: (num + den / 2).div_euclid(den)
static int64_t round_ratio_rhu(int64_t num, int64_t den) {
  __int128 t = (__int128)num + den / 2;
  __int128 q = t / den;
  if (t % den < 0) q -= 1;
  return (int64_t)q;
}

// rms_norm.rs:96-170 for one row; gamma gradients added into gw (i64).
static bool rms_norm_backward_row(const int16_t* x, const int16_t* w, const int16_t* go, size_t d, uint64_t eps,
                                  int16_t* gi, int64_t* gw, uint64_t* sat) {
  if (d == 0) return false;
  uint64_t sum = 0;
  for (size_t i = 0; i < d; ++i) sum += (uint64_t)((int64_t)x[i] * (int64_t)x[i]);
  uint64_t mean = sum / d, v;
  if (__builtin_add_overflow(mean, eps, &v)) return false;
  int64_t inv;
  if (!integer_rsqrt_q30(v, &inv)) return false;
  std::vector<int32_t> normalized(d), scaled(d);
  int64_t dot = 0;
  for (size_t i = 0; i < d; ++i) {
    int64_t t;
    if (__builtin_mul_overflow((int64_t)x[i], inv, &t)) return false;
    int64_t nm = rhu(t, 15);
    if (nm < INT32_MIN || nm > INT32_MAX) return false;
    normalized[i] = (int32_t)nm;
    int64_t xw = (int64_t)x[i] * (int64_t)w[i], pr;
    if (__builtin_mul_overflow(xw, inv, &pr)) return false;
    const int64_t projected = rhu(pr, RMSNORM_INV_RMS_SHIFT);
    const bool active = projected >= -32768 && projected <= 32767;
    int32_t sg = 0;
    if (active) {
      int64_t s = rhu((int64_t)go[i] * (int64_t)w[i], 15);
      if (s < INT32_MIN || s > INT32_MAX) return false;
      sg = (int32_t)s;
    }
    scaled[i] = sg;
    int64_t prod;
    if (__builtin_mul_overflow((int64_t)sg, (int64_t)nm, &prod)) return false;
    if (__builtin_add_overflow(dot, prod, &dot)) return false;
    int64_t gg = 0;
    if (active) {
      int64_t q;
      if (__builtin_mul_overflow((int64_t)go[i], nm, &q)) return false;
      gg = rhu(q, 15);
    }
    if (__builtin_add_overflow(gw[i], gg, &gw[i])) return false;
  }
  const int64_t mean_dot = round_ratio_rhu(dot, (int64_t)d << 15);
  for (size_t i = 0; i < d; ++i) {
    int64_t c;
    if (__builtin_mul_overflow((int64_t)normalized[i], mean_dot, &c)) return false;
    const int64_t cross = rhu(c, 15);
    int64_t corr;
    if (__builtin_sub_overflow((int64_t)scaled[i], cross, &corr)) return false;
    int64_t wide;
    if (__builtin_mul_overflow(corr, inv, &wide)) return false;
    const int64_t g = rhu(wide, RMSNORM_INV_RMS_SHIFT);
    const int16_t cl = saturate_i16(g);
    if ((int64_t)cl != g) ++*sat;
    gi[i] = cl;
  }
  return true;
}

// nsrl-train/src/lib.rs:15353-15418: P[h][q][k] of a causal sequence, 0 above the diagonal.
static bool attention_probabilities(const int16_t* q, const int16_t* k, size_t S, size_t d, size_t H, int16_t* P) {
  const size_t hd = d / H;
  const int shift = sqrt_power_of_four_shift(hd);
  if (shift < 0) return false;
  std::vector<int32_t> logits(S);
  for (size_t h = 0; h < H; ++h)
    for (size_t t = 0; t < S; ++t) {
      int16_t* row = P + (h * S + t) * S;
      for (size_t j = 0; j <= t; ++j)
        if (!qk_dot(q + t * d + h * hd, k + j * d + h * hd, hd, shift, &logits[j])) return false;
      if (!base2_softmax(logits.data(), t + 1, row, nullptr)) return false;
      for (size_t j = t + 1; j < S; ++j) row[j] = 0;
    }
  return true;
}

// nsrl-train/src/lib.rs:16623-16900: gradients of the causal base-2 softmax
// attention of one sequence.  dC = grad of the context [S][d].
static bool attention_backward(const int16_t* q, const int16_t* k, const int16_t* v, const int16_t* P,
                               const int16_t* dC, size_t S, size_t d, size_t H, int16_t* dq, int16_t* dk,
                               int16_t* dv) {
  const size_t hd = d / H;
  const int shift = sqrt_power_of_four_shift(hd);
  if (shift < 0) return false;
  std::vector<int16_t> dP(H * S * S, 0), dL(H * S * S, 0);
  for (size_t h = 0; h < H; ++h) {
    const size_t o = h * hd;
    // probability gradient (:16623-16677)
    for (size_t t = 0; t < S; ++t)
      for (size_t j = 0; j <= t; ++j) {
        int64_t acc = 0;
        for (size_t c = 0; c < hd; ++c) acc += (int64_t)dC[t * d + o + c] * (int64_t)v[j * d + o + c];
        dP[(h * S + t) * S + j] = saturate_i16(rhu(acc, Q15_SHIFT));
      }
    // logit gradient (:16679-16747)
    for (size_t t = 0; t < S; ++t) {
      const int16_t* pr = P + (h * S + t) * S;
      const int16_t* gp = &dP[(h * S + t) * S];
      int64_t wsum = 0;
      for (size_t j = 0; j <= t; ++j) {
        if (pr[j] < 0) return false;
        wsum += (int64_t)gp[j] * (int64_t)pr[j];
      }
      const int64_t wq = rhu(wsum, Q15_SHIFT);
      for (size_t j = 0; j <= t; ++j) {
        const int64_t centered = (int64_t)gp[j] - wq;
        int64_t prod;
        if (__builtin_mul_overflow((int64_t)pr[j] * centered, LN2_Q15, &prod)) return false;
        dL[(h * S + t) * S + j] = saturate_i16(rhu(prod, 2 * Q15_SHIFT));
      }
    }
    // q / k gradients (:16749-16839)
    for (size_t t = 0; t < S; ++t)
      for (size_t c = 0; c < hd; ++c) {
        int64_t acc = 0;
        for (size_t j = 0; j <= t; ++j) acc += (int64_t)dL[(h * S + t) * S + j] * (int64_t)k[j * d + o + c];
        dq[t * d + o + c] = saturate_i16(rhu(acc, (uint8_t)shift));
      }
    for (size_t j = 0; j < S; ++j)
      for (size_t c = 0; c < hd; ++c) {
        int64_t acc = 0;
        for (size_t t = j; t < S; ++t) acc += (int64_t)dL[(h * S + t) * S + j] * (int64_t)q[t * d + o + c];
        dk[j * d + o + c] = saturate_i16(rhu(acc, (uint8_t)shift));
      }
    // value gradient (:16841-16900)
    for (size_t j = 0; j < S; ++j)
      for (size_t c = 0; c < hd; ++c) {
        int64_t acc = 0;
        for (size_t t = 0; t < S; ++t) {
          const int16_t p = P[(h * S + t) * S + j];
          if (p < 0) return false;
          acc += (int64_t)p * (int64_t)dC[t * d + o + c];
        }
        dv[j * d + o + c] = saturate_i16(rhu(acc, Q15_SHIFT));
      }
  }
  return true;
}

// nsrl-train-core/src/lib.rs:344-384 for one row, with the prescale of
// linear.rs:573-592 in front (the wrappers at nsrl-train/src/lib.rs:13783-14055).
static bool accumulate_row(const int16_t* x, const int16_t* g, const LinearParams& p, int64_t* acc,
                           uint64_t* count) {
  const size_t K = p.input_dim, N = p.output_dim;
  for (size_t n = 0; n < N; ++n) {
    int32_t gs;
    if (!prescale_grad(g[n], p.scales[n], &gs)) return false;
    if (gs == 0) continue;
    for (size_t kk = 0; kk < K; ++kk) {
      if (x[kk] == 0) continue;
      if (__builtin_add_overflow(acc[n * K + kk], (int64_t)gs * (int64_t)x[kk], &acc[n * K + kk])) return false;
    }
  }
  *count += 1;
  return true;
}

}  // namespace orc

// ---------------------------------------------------------------------------
// C ABI of the training restatement.
// ---------------------------------------------------------------------------
extern "C" {

// linear.rs:548-640 over rows.  gin: grad-input scales [K] or null (identity).
int orc_linear_backward_input(const int16_t* g, size_t M, const LinearParams* p, const FixedScale* gin,
                              int16_t* dx) {
  for (size_t m = 0; m < M; ++m)
    if (!linear_backward_input_row(g + m * p->output_dim, *p, gin, dx + m * p->input_dim)) return 1;
  return 0;
}

void orc_gated_activation_backward(int16_t up, int16_t gate, int16_t g, int16_t* gu, int16_t* gg) {
  gated_activation_backward(up, gate, g, gu, gg);
}

// mlp.rs:256-357; lp = {up, gate, down}.
int orc_gated_mlp_backward_input(const int16_t* grad_out, size_t T, size_t d, size_t F, const LinearParams* lp,
                                 const int16_t* up, const int16_t* gate, int16_t* grad_up, int16_t* grad_gate,
                                 int16_t* grad_in, uint64_t* sat) {
  *sat = 0;
  return gated_mlp_backward_input_rows(grad_out, T, d, F, lp, up, gate, grad_up, grad_gate, grad_in, sat) ? 0 : 1;
}

// rms_norm.rs:96-170 over rows (nsrl-train/src/lib.rs:15030-15077).
int orc_rms_norm_backward_rows(const int16_t* x, size_t T, size_t d, const int16_t* w, const int16_t* go,
                               uint64_t eps, int16_t* gi, int64_t* gw, uint64_t* sat) {
  *sat = 0;
  for (size_t t = 0; t < T; ++t)
    if (!rms_norm_backward_row(x + t * d, w, go + t * d, d, eps, gi + t * d, gw, sat)) return 1;
  return 0;
}

int orc_attention_probabilities(const int16_t* q, const int16_t* k, size_t B, size_t S, size_t d, size_t H,
                                int16_t* P) {
  for (size_t b = 0; b < B; ++b)
    if (!attention_probabilities(q + b * S * d, k + b * S * d, S, d, H, P + b * H * S * S)) return 1;
  return 0;
}

int orc_attention_backward(const int16_t* q, const int16_t* k, const int16_t* v, const int16_t* P,
                           const int16_t* dC, size_t B, size_t S, size_t d, size_t H, int16_t* dq, int16_t* dk,
                           int16_t* dv) {
  for (size_t b = 0; b < B; ++b) {
    const size_t o = b * S * d;
    if (!attention_backward(q + o, k + o, v + o, P + b * H * S * S, dC + o, S, d, H, dq + o, dk + o, dv + o))
      return 1;
  }
  return 0;
}

}  // extern "C"

// ------------------------------------------------- mini-transformer step ---
namespace orc {

struct TrainLayer {  // one block: RMS gammas (both null: RMS disabled) and q, k, v, o, up, gate, down
  const int16_t* attn_gamma;
  const int16_t* mlp_gamma;
  LinearParams lin[7];
};

struct TrainModel {
  size_t d, H, F, layers, S;
  const int16_t* embeddings;  // [256][d]
  const int16_t* positions;   // [S][d], or null for the position-free policy
  const TrainLayer* layer;
  LinearParams head;          // [256][d]
  int32_t attention_kind;     // 0: base-2 softmax, 1: linear (MiniTransformerAttentionKind, lib.rs:1017-1023)
};

// Offsets of the i64 gradient arena: head, per layer (q k v o up gate down
// rms_attention rms_mlp), token embeddings, position embeddings.
struct Arena {
  size_t head, layer0, per_layer, emb, pos, total;
  size_t lin[7], rms_a, rms_m;  // offsets inside a layer
  Arena(const TrainModel& m) {
    const size_t d = m.d, F = m.F;
    head = 0;
    layer0 = VOCAB * d;
    size_t o = 0;
    for (int i = 0; i < 4; ++i) lin[i] = o, o += d * d;
    for (int i = 4; i < 7; ++i) lin[i] = o, o += F * d;
    rms_a = o, o += d;
    rms_m = o, o += d;
    per_layer = o;
    emb = layer0 + m.layers * per_layer;
    pos = emb + VOCAB * d;
    total = pos + m.S * d;
  }
  // counts: [0] head, [1 + 9 l + i] layer l item i, [1 + 9 L] embeddings
};

// ------------------------------------------------------ linear attention --
// crates/nsrl-core/src/attention.rs:1391-1466: phi(x) = x + 32769, the
// per-head state S[key][value] = sum phi(k) v and key sums sum phi(k) in
// checked i64, the projection round_div(sum phi(q) S, sum phi(q) K_s).
static inline int64_t la_phi(int16_t v) { return (int64_t)v + 32769; }

// attention.rs:1468-1477 (denominator > 0; saturating +- half, truncating division)
static int64_t la_round_div(int64_t num, int64_t den) {
  const int64_t half = den >> 1;
  int64_t t;
  if (num >= 0) {
    if (__builtin_add_overflow(num, half, &t)) t = INT64_MAX;
  } else {
    if (__builtin_sub_overflow(num, half, &t)) t = INT64_MIN;
  }
  return t / den;
}

// attention.rs:1346-1396 (decay of the state; identity is a no-op)
static bool la_decay(int64_t* S, int64_t* ks, size_t hd, FixedScale decay) {
  if (decay.multiplier == 1 && decay.right_shift == 0) return true;
  for (size_t i = 0; i < hd; ++i) {
    int64_t w;
    if (__builtin_mul_overflow(ks[i], (int64_t)decay.multiplier, &w)) return false;
    ks[i] = rhu(w, decay.right_shift);
  }
  for (size_t i = 0; i < hd * hd; ++i) {
    int64_t w;
    if (__builtin_mul_overflow(S[i], (int64_t)decay.multiplier, &w)) return false;
    S[i] = rhu(w, decay.right_shift);
  }
  return true;
}

// attention.rs:1398-1430
static bool la_accumulate(const int16_t* k, const int16_t* v, int64_t* S, int64_t* ks, size_t hd, FixedScale decay) {
  if (!la_decay(S, ks, hd, decay)) return false;
  for (size_t i = 0; i < hd; ++i) {
    const int64_t pk = la_phi(k[i]);
    if (__builtin_add_overflow(ks[i], pk, &ks[i])) return false;
    for (size_t j = 0; j < hd; ++j) {
      const int64_t p = pk * (int64_t)v[j];  // |p| <= 2^31
      if (__builtin_add_overflow(S[i * hd + j], p, &S[i * hd + j])) return false;
    }
  }
  return true;
}

// attention.rs:1432-1466
static bool la_project(const int16_t* q, const int64_t* S, const int64_t* ks, size_t hd, int16_t* out) {
  int64_t den = 0;
  for (size_t i = 0; i < hd; ++i) {
    int64_t p;
    if (__builtin_mul_overflow(la_phi(q[i]), ks[i], &p) || __builtin_add_overflow(den, p, &den)) return false;
  }
  if (den <= 0) return false;
  for (size_t j = 0; j < hd; ++j) {
    int64_t num = 0;
    for (size_t i = 0; i < hd; ++i) {
      int64_t p;
      if (__builtin_mul_overflow(la_phi(q[i]), S[i * hd + j], &p) || __builtin_add_overflow(num, p, &num))
        return false;
    }
    out[j] = saturate_i16(la_round_div(num, den));
  }
  return true;
}

// attention.rs:1290-1344 (linear_attention_ttt_delta_state_i16_q15_checked)
static bool la_ttt_delta(const int16_t* k, const int16_t* v, int64_t* S, const int64_t* ks, size_t hd,
                         uint8_t lr_shift, int16_t* pred, uint64_t* delta_l1) {
  int64_t den = 0;
  for (size_t i = 0; i < hd; ++i) {
    int64_t p;
    if (__builtin_mul_overflow(la_phi(k[i]), ks[i], &p) || __builtin_add_overflow(den, p, &den)) return false;
  }
  for (size_t j = 0; j < hd; ++j) {
    if (den > 0) {
      int64_t num = 0;
      for (size_t i = 0; i < hd; ++i) {
        int64_t p;
        if (__builtin_mul_overflow(la_phi(k[i]), S[i * hd + j], &p) || __builtin_add_overflow(num, p, &num))
          return false;
      }
      pred[j] = saturate_i16(la_round_div(num, den));
    } else {
      pred[j] = 0;
    }
  }
  uint64_t l1 = 0;
  for (size_t i = 0; i < hd; ++i) {
    const int64_t pk = la_phi(k[i]);
    for (size_t j = 0; j < hd; ++j) {
      const int64_t err = (int64_t)v[j] - (int64_t)pred[j];
      const int64_t upd = rhu(pk * err, lr_shift);
      if (__builtin_add_overflow(S[i * hd + j], upd, &S[i * hd + j])) return false;
      const uint64_t a = upd < 0 ? (uint64_t)(-(upd + 1)) + 1 : (uint64_t)upd;
      if (__builtin_add_overflow(l1, a, &l1)) return false;
    }
  }
  *delta_l1 += l1;
  return true;
}

// attention.rs:911-1041: q, k, v of every token, then per token and head the
// state update and (causal) the projection; non-causal accumulates every
// token first.  x, out [S][d]; q, k, v, ctx scratch [S][d].
static bool linear_attention_seq(const int16_t* x, size_t S, size_t d, size_t H, bool causal, const LinearParams* lp,
                                 FixedScale decay, int16_t* out) {
  if (S == 0 || d == 0 || H == 0 || d % H) return false;
  const size_t hd = d / H, T = S * d;
  std::vector<int16_t> q(T), k(T), v(T), ctx(T);
  std::vector<int64_t> st(H * hd * hd, 0), ks(H * hd, 0);
  for (size_t t = 0; t < S; ++t)
    if (!linear_row(x + t * d, lp[0], &q[t * d]) || !linear_row(x + t * d, lp[1], &k[t * d]) ||
        !linear_row(x + t * d, lp[2], &v[t * d]))
      return false;
  for (size_t t = 0; t < S; ++t)
    for (size_t h = 0; h < H; ++h) {
      const size_t rb = t * d + h * hd;
      if (!la_accumulate(&k[rb], &v[rb], &st[h * hd * hd], &ks[h * hd], hd, decay)) return false;
      if (causal && !la_project(&q[rb], &st[h * hd * hd], &ks[h * hd], hd, &ctx[rb])) return false;
    }
  if (!causal)
    for (size_t t = 0; t < S; ++t)
      for (size_t h = 0; h < H; ++h) {
        const size_t rb = t * d + h * hd;
        if (!la_project(&q[rb], &st[h * hd * hd], &ks[h * hd], hd, &ctx[rb])) return false;
      }
  for (size_t t = 0; t < S; ++t)
    if (!linear_row(&ctx[t * d], lp[3], out + t * d)) return false;
  return true;
}

// attention.rs:1085-1158 / :1186-1283: one row through q, k, v, the state
// update (+ the TTT delta when ttt) and the projection, then o.
static bool linear_attention_row_step(const int16_t* x, size_t d, size_t H, const LinearParams* lp, int64_t* st,
                                      int64_t* ks, bool ttt, uint8_t lr_shift, int16_t* out, uint64_t* delta_l1) {
  if (d == 0 || H == 0 || d % H) return false;
  const size_t hd = d / H;
  std::vector<int16_t> q(d), k(d), v(d), ctx(d), pred(d);
  if (!linear_row(x, lp[0], q.data()) || !linear_row(x, lp[1], k.data()) || !linear_row(x, lp[2], v.data()))
    return false;
  const FixedScale id{1, 0, {0, 0, 0}};
  for (size_t h = 0; h < H; ++h) {
    const size_t o = h * hd;
    if (!la_accumulate(&k[o], &v[o], &st[h * hd * hd], &ks[h * hd], hd, id)) return false;
    if (ttt && !la_ttt_delta(&k[o], &v[o], &st[h * hd * hd], &ks[h * hd], hd, lr_shift, &pred[o], delta_l1))
      return false;
    if (!la_project(&q[o], &st[h * hd * hd], &ks[h * hd], hd, &ctx[o])) return false;
  }
  return linear_row(ctx.data(), lp[3], out);
}

struct BlockCache {
  std::vector<int16_t> in, an, q, k, v, ctx, P, ares, mn, up, gate, gated, out;
};

static bool sat_add_rows(const int16_t* a, const int16_t* b, int16_t* out, size_t n, uint64_t* sat) {
  return residual_add(a, b, out, n, sat);
}

// The base-2 softmax attention of a block with its caches (q, k, v, context, P).
static bool softmax_attention_part(const TrainModel& m, const TrainLayer& L, const int16_t* x, BlockCache& c,
                                   std::vector<int16_t>& aout, std::vector<int16_t>& probs, uint64_t* res_sat) {
  const size_t S = m.S, d = m.d, H = m.H, T = S * d;
  std::vector<int32_t> logits(S);
  if (!attention_shapes_valid(S, d, H, L.lin)) return false;
  c.q.resize(T), c.k.resize(T), c.v.resize(T), c.ctx.resize(T);
  for (size_t t = 0; t < S; ++t) {
    if (!linear_row(&c.an[t * d], L.lin[0], &c.q[t * d])) return false;
    if (!linear_row(&c.an[t * d], L.lin[1], &c.k[t * d])) return false;
    if (!linear_row(&c.an[t * d], L.lin[2], &c.v[t * d])) return false;
  }
  const size_t hd = d / H;
  const int shift = sqrt_power_of_four_shift(hd);
  for (size_t t = 0; t < S; ++t)
    for (size_t h = 0; h < H; ++h) {
      const size_t off = h * hd;
      for (size_t j = 0; j <= t; ++j)
        if (!qk_dot(&c.q[t * d + off], &c.k[j * d + off], hd, shift, &logits[j])) return false;
      if (!base2_softmax(logits.data(), t + 1, probs.data(), nullptr)) return false;
      for (size_t cc = 0; cc < hd; ++cc) {
        int64_t acc = 0;
        for (size_t j = 0; j <= t; ++j) acc += (int64_t)probs[j] * (int64_t)c.v[j * d + off + cc];
        c.ctx[t * d + off + cc] = saturate_i16(rhu(acc, Q15_SHIFT));
      }
    }
  for (size_t t = 0; t < S; ++t)
    if (!linear_row(&c.ctx[t * d], L.lin[3], &aout[t * d])) return false;
  c.P.resize(H * S * S);
  if (!attention_probabilities(c.q.data(), c.k.data(), S, d, H, c.P.data())) return false;
  c.ares.resize(T);
  sat_add_rows(x, aout.data(), c.ares.data(), T, res_sat);
  return true;
}

// nsrl-train/src/lib.rs:15079-15300 (base-2 softmax attention kind)
static bool block_forward_cache(const TrainModel& m, const TrainLayer& L, const int16_t* x, BlockCache& c,
                                uint64_t* res_sat) {
  const size_t S = m.S, d = m.d, F = m.F, H = m.H, T = S * d;
  c.in.assign(x, x + T);
  c.an.resize(T);
  if (L.attn_gamma) {
    for (size_t t = 0; t < S; ++t)
      if (!rms_norm_row(x + t * d, L.attn_gamma, d, TRAIN_RMS_EPS, &c.an[t * d])) return false;
  } else {
    c.an = c.in;
  }
  std::vector<int16_t> aout(T), probs(S);
  if (m.attention_kind == 1) {
    // the Linear kind of mini_transformer_forward_block_for_attention_kind (lib.rs:15079-15294)
    const FixedScale id{1, 0, {0, 0, 0}};
    if (!linear_attention_seq(c.an.data(), S, d, H, true, L.lin, id, aout.data())) return false;
    c.ares.resize(T);
    sat_add_rows(x, aout.data(), c.ares.data(), T, res_sat);
  } else if (!softmax_attention_part(m, L, x, c, aout, probs, res_sat)) {
    return false;
  }
  c.mn.resize(T);
  if (L.mlp_gamma) {
    for (size_t t = 0; t < S; ++t)
      if (!rms_norm_row(&c.ares[t * d], L.mlp_gamma, d, TRAIN_RMS_EPS, &c.mn[t * d])) return false;
  } else {
    c.mn = c.ares;
  }
  c.up.resize(S * F), c.gate.resize(S * F), c.gated.resize(S * F);
  std::vector<int16_t> mout(T);
  for (size_t t = 0; t < S; ++t) {
    if (!linear_row(&c.mn[t * d], L.lin[4], &c.up[t * F])) return false;
    if (!linear_row(&c.mn[t * d], L.lin[5], &c.gate[t * F])) return false;
    for (size_t f = 0; f < F; ++f) c.gated[t * F + f] = gated_activation(c.up[t * F + f], c.gate[t * F + f]);
    if (!linear_row(&c.gated[t * F], L.lin[6], &mout[t * d])) return false;
  }
  c.out.resize(T);
  sat_add_rows(c.ares.data(), mout.data(), c.out.data(), T, res_sat);
  return true;
}

struct WindowStats {
  uint64_t accepted, mlp_sat, attn_sat, res_sat;
};

// nsrl-train/src/lib.rs:15623-15775 with the attention update of
// :15777-16075 in its accumulate form and the accumulations of :13783-14055.
static bool block_backward_accumulate(const TrainModel& m, const TrainLayer& L, const BlockCache& c,
                                      const int16_t* G, int64_t* acc, uint64_t* cnt, const Arena& ar,
                                      std::vector<int16_t>& grad_in, WindowStats& ws) {
  const size_t S = m.S, d = m.d, F = m.F, H = m.H, T = S * d;
  const LinearParams mlp_lp[3] = {L.lin[4], L.lin[5], L.lin[6]};
  std::vector<int16_t> gup(S * F), ggate(S * F), gmi(T), gmr(T), gao(T);
  uint64_t sat_m = 0, sat_mr = 0, sat_res = 0, sat_a = 0, sat_ar = 0, sat_in = 0;
  if (!gated_mlp_backward_input_rows(G, S, d, F, mlp_lp, c.up.data(), c.gate.data(), gup.data(), ggate.data(),
                                     gmi.data(), &sat_m))
    return false;
  if (L.mlp_gamma) {
    for (size_t t = 0; t < S; ++t)
      if (!rms_norm_backward_row(&c.ares[t * d], L.mlp_gamma, &gmi[t * d], d, TRAIN_RMS_EPS, &gmr[t * d],
                                 acc + ar.rms_m, &sat_mr))
        return false;
    cnt[8] += S;
  } else {
    gmr = gmi;
  }
  sat_add_rows(G, gmr.data(), gao.data(), T, &sat_res);
  // gated-MLP weight gradients: rows whose output gradient is all zero are skipped (:13828-13831)
  for (size_t t = 0; t < S; ++t) {
    bool any = false;
    for (size_t i = 0; i < d; ++i) any |= G[t * d + i] != 0;
    if (!any) continue;
    if (!accumulate_row(&c.gated[t * F], &G[t * d], L.lin[6], acc + ar.lin[6], &cnt[6])) return false;
    if (!accumulate_row(&c.mn[t * d], &gup[t * F], L.lin[4], acc + ar.lin[4], &cnt[4])) return false;
    if (!accumulate_row(&c.mn[t * d], &ggate[t * F], L.lin[5], acc + ar.lin[5], &cnt[5])) return false;
  }
  // attention update (accumulate form)
  std::vector<int16_t> gctx(T), dq(T), dk(T), dv(T), gni(T), gq(d), gk(d), gv(d);
  for (size_t t = 0; t < S; ++t)
    if (!linear_backward_input_row(&gao[t * d], L.lin[3], nullptr, &gctx[t * d])) return false;
  if (!attention_backward(c.q.data(), c.k.data(), c.v.data(), c.P.data(), gctx.data(), S, d, H, dq.data(),
                          dk.data(), dv.data()))
    return false;
  for (size_t t = 0; t < S; ++t) {
    if (!linear_backward_input_row(&dq[t * d], L.lin[0], nullptr, gq.data())) return false;
    if (!linear_backward_input_row(&dk[t * d], L.lin[1], nullptr, gk.data())) return false;
    if (!linear_backward_input_row(&dv[t * d], L.lin[2], nullptr, gv.data())) return false;
    for (size_t i = 0; i < d; ++i) {
      const int64_t s = rhu((int64_t)gq[i] + (int64_t)gk[i] + (int64_t)gv[i], FANIN_SHIFT);
      if (s < -32768 || s > 32767) ++sat_a;
      gni[t * d + i] = saturate_i16(s);
    }
  }
  for (size_t t = 0; t < S; ++t) {
    if (!accumulate_row(&c.an[t * d], &dq[t * d], L.lin[0], acc + ar.lin[0], &cnt[0])) return false;
    if (!accumulate_row(&c.an[t * d], &dk[t * d], L.lin[1], acc + ar.lin[1], &cnt[1])) return false;
    if (!accumulate_row(&c.an[t * d], &dv[t * d], L.lin[2], acc + ar.lin[2], &cnt[2])) return false;
    if (!accumulate_row(&c.ctx[t * d], &gao[t * d], L.lin[3], acc + ar.lin[3], &cnt[3])) return false;
  }
  std::vector<int16_t> gai(T);
  if (L.attn_gamma) {
    for (size_t t = 0; t < S; ++t)
      if (!rms_norm_backward_row(&c.in[t * d], L.attn_gamma, &gni[t * d], d, TRAIN_RMS_EPS, &gai[t * d],
                                 acc + ar.rms_a, &sat_ar))
        return false;
    cnt[7] += S;
  } else {
    gai = gni;
  }
  grad_in.resize(T);
  sat_add_rows(gao.data(), gai.data(), grad_in.data(), T, &sat_in);
  ws.mlp_sat += sat_m + sat_mr;
  ws.attn_sat += sat_a;
  ws.res_sat += sat_res + sat_in + sat_ar;
  return true;
}

// nsrl-train/src/lib.rs:7051-7399: forward, output head, softmax gradient and
// the backward of every layer for one window, accumulated into `acc`/`cnt`.
static bool train_window(const TrainModel& m, const uint8_t* ctx, uint8_t target, const int16_t* freq_w,
                         int64_t* acc, uint64_t* cnt, WindowStats& ws) {
  const Arena ar(m);
  const size_t S = m.S, d = m.d, T = S * d;
  // embeddings (:14862-14897)
  std::vector<int16_t> x(T);
  for (size_t t = 0; t < S; ++t)
    for (size_t i = 0; i < d; ++i) {
      int64_t v = m.embeddings[(size_t)ctx[t] * d + i];
      if (m.positions) v += m.positions[t * d + i];
      x[t * d + i] = saturate_i16(v);
    }
  std::vector<BlockCache> caches(m.layers);
  uint64_t fwd_res = 0;
  const int16_t* cur = x.data();
  for (size_t l = 0; l < m.layers; ++l) {
    if (!block_forward_cache(m, m.layer[l], cur, caches[l], &fwd_res)) return false;
    cur = caches[l].out.data();
  }
  // output head on the last position (:17455-17488)
  const int16_t* feat = cur + (S - 1) * d;
  int16_t logits16[VOCAB], probs[VOCAB];
  int32_t logits[VOCAB];
  if (!linear_row(feat, m.head, logits16)) return false;
  for (size_t i = 0; i < VOCAB; ++i) logits[i] = logits16[i];
  if (!base2_softmax(logits, VOCAB, probs, nullptr)) return false;
  // softmax gradient, frequency weight, i16 conversion (:18845-18949)
  int16_t grad[VOCAB];
  const int16_t fw = freq_w ? freq_w[target] : 32767;
  for (size_t i = 0; i < VOCAB; ++i) {
    int64_t g = (int64_t)probs[i] - (i == target ? 32767 : 0);
    if (fw != 32767) g = (int32_t)rhu(g * (int64_t)fw, Q15_SHIFT);
    grad[i] = saturate_i16(g);
  }
  std::vector<int16_t> G(T, 0);
  if (!linear_backward_input_row(grad, m.head, nullptr, &G[(S - 1) * d])) return false;
  if (!accumulate_row(feat, grad, m.head, acc + ar.head, &cnt[0])) return false;
  std::vector<int16_t> gin;
  for (size_t l = m.layers; l-- > 0;) {
    if (!block_backward_accumulate(m, m.layer[l], caches[l], G.data(), acc + ar.layer0 + l * ar.per_layer,
                                   cnt + 1 + 9 * l, ar, gin, ws))
      return false;
    G.swap(gin);
  }
  // embedding gradients (:14336-14405)
  const size_t ce = 1 + 9 * m.layers;
  for (size_t t = 0; t < S; ++t)
    for (size_t i = 0; i < d; ++i) {
      const int64_t g = G[t * d + i];
      if (g == 0) continue;
      if (__builtin_add_overflow(acc[ar.emb + (size_t)ctx[t] * d + i], g, &acc[ar.emb + (size_t)ctx[t] * d + i]))
        return false;
      if (m.positions && __builtin_add_overflow(acc[ar.pos + t * d + i], g, &acc[ar.pos + t * d + i])) return false;
    }
  cnt[ce] += 1;
  ws.accepted += 1;
  ws.res_sat += 2 * fwd_res;
  return true;
}

// nsrl-train/src/lib.rs:14911-15008 (softmax attention, learned or no
// positions) and :17455-17490: the forward of one window and the byte-head
// row of its last position.  false = CoreRejected.
static bool output_row(const TrainModel& m, const uint8_t* window, int32_t* logits_q8, int16_t* probs_q15) {
  const size_t S = m.S, d = m.d, T = S * d;
  std::vector<int16_t> x(T);
  for (size_t t = 0; t < S; ++t)
    for (size_t i = 0; i < d; ++i) {
      int64_t v = m.embeddings[(size_t)window[t] * d + i];
      if (m.positions) v += m.positions[t * d + i];
      x[t * d + i] = saturate_i16(v);
    }
  BlockCache c;
  uint64_t sat = 0;
  std::vector<int16_t> cur = x;
  for (size_t l = 0; l < m.layers; ++l) {
    if (!block_forward_cache(m, m.layer[l], cur.data(), c, &sat)) return false;
    cur = c.out;
  }
  int16_t logits16[VOCAB];
  if (!linear_row(cur.data() + (S - 1) * d, m.head, logits16)) return false;
  for (size_t i = 0; i < VOCAB; ++i) logits_q8[i] = logits16[i];
  return base2_softmax(logits_q8, VOCAB, probs_q15, nullptr);
}

static uint64_t splitmix64(uint64_t v) {  // lib.rs:19342-19347
  v += 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

// decode_sample_u64 (lib.rs:19334-19340) over the StableHasher (FNV-1a,
// :19468-19519; usize values as 8 little-endian bytes, slices length-prefixed).
static uint64_t decode_sample_u64(uint64_t seed, size_t step, const uint8_t* ctx, size_t n) {
  Fnv f;
  f.usize(seed);
  f.usize((uint64_t)step);
  f.usize((uint64_t)n);
  f.bytes(ctx, n);
  return splitmix64(f.h);
}

// select_byte_from_row_with_priors (lib.rs:18979-19083) with no priors and no
// constraints: greedy = byte_argmax_i32 (lowest index among equal logits,
// :18951-18958); sample = the top_k candidates by (logit desc, index asc),
// weights max(p, 0), threshold = decode_sample_u64 % mass, walked in that
// order; a zero mass falls back to the first candidate (:19085-19100).
static uint8_t select_byte(const int32_t* logits, const int16_t* probs, int strategy, size_t top_k, uint64_t seed,
                           size_t step, const uint8_t* ctx, size_t n) {
  int best = 0;
  for (int i = 1; i < (int)VOCAB; ++i)
    if (logits[i] > logits[best]) best = i;
  if (strategy == 0) return (uint8_t)best;
  const size_t k = (top_k == 0 || top_k > VOCAB) ? VOCAB : top_k;
  std::vector<int> cand(VOCAB);
  for (int i = 0; i < (int)VOCAB; ++i) cand[i] = i;
  std::stable_sort(cand.begin(), cand.end(), [&](int a, int b) { return logits[a] > logits[b]; });
  cand.resize(k);
  uint64_t mass = 0;
  for (int c : cand) mass += (uint64_t)std::max<int>(probs[c], 0);
  if (mass == 0) return (uint8_t)cand[0];
  uint64_t th = decode_sample_u64(seed, step, ctx, n) % mass;
  for (int c : cand) {
    const uint64_t w = (uint64_t)std::max<int>(probs[c], 0);
    if (th < w) return (uint8_t)c;
    th -= w;
  }
  return (uint8_t)cand[0];
}

}  // namespace orc

extern "C" {

// linear_attention_i16_q15_checked (attention.rs:879-1041) over `batch`
// sequences [batch][S][d]; 0 = ok, 2 = rejected.
int orc_linear_attention(const int16_t* x, size_t batch, size_t S, size_t d, size_t H, int causal,
                         const LinearParams* lp, int16_t* out) {
  const FixedScale id{1, 0, {0, 0, 0}};
  for (size_t b = 0; b < batch; ++b)
    if (!linear_attention_seq(x + b * S * d, S, d, H, causal != 0, lp, id, out + b * S * d)) return 2;
  return 0;
}

// linear_attention_step_i16_q15_checked / linear_attention_ttt_step_i16_q15_checked
// (attention.rs:1045-1283) for `batch` independent streams: rows x [batch][d],
// states [batch][H][hd][hd] and key sums [batch][H][hd] updated in place,
// delta_l1 [batch] (TTT only, added to).
int orc_linear_attention_step(const int16_t* x, size_t batch, size_t d, size_t H, const LinearParams* lp,
                              int64_t* state, int64_t* key_sums, int ttt, uint8_t lr_shift, int16_t* out,
                              uint64_t* delta_l1) {
  if (H == 0 || d % H) return 1;
  const size_t hd = d / H;
  for (size_t b = 0; b < batch; ++b) {
    uint64_t dl = 0;
    if (!linear_attention_row_step(x + b * d, d, H, lp, state + b * H * hd * hd, key_sums + b * H * hd, ttt != 0,
                                   lr_shift, out + b * d, &dl))
      return 2;
    if (delta_l1) delta_l1[b] += dl;
  }
  return 0;
}

// mini_transformer_streaming_linear_nope_step / _ttt_nope_step (nsrl-train/src/
// lib.rs:13035-13150): the token's embedding, the linear-attention step of
// layer 0 with its state, the residual, the gated MLP (no RMS norm: the
// streaming step applies none), the residual and the byte-head row.
static bool streaming_step(const TrainModel& m, uint8_t token, int64_t* st, int64_t* ks, bool ttt, uint8_t lr_shift,
                           int32_t* logits, int16_t* probs) {
  const size_t d = m.d, F = m.F;
  const TrainLayer& L = m.layer[0];
  std::vector<int16_t> e(m.embeddings + (size_t)token * d, m.embeddings + (size_t)token * d + d);
  std::vector<int16_t> a(d), r(d), up(F), gate(F), gated(F), mo(d), out(d);
  uint64_t dl = 0, sat = 0;
  if (!linear_attention_row_step(e.data(), d, m.H, L.lin, st, ks, ttt, lr_shift, a.data(), &dl)) return false;
  sat_add_rows(e.data(), a.data(), r.data(), d, &sat);
  if (!linear_row(r.data(), L.lin[4], up.data()) || !linear_row(r.data(), L.lin[5], gate.data())) return false;
  for (size_t f = 0; f < F; ++f) gated[f] = gated_activation(up[f], gate[f]);
  if (!linear_row(gated.data(), L.lin[6], mo.data())) return false;
  sat_add_rows(r.data(), mo.data(), out.data(), d, &sat);
  int16_t l16[VOCAB];
  if (!linear_row(out.data(), m.head, l16)) return false;
  for (size_t i = 0; i < VOCAB; ++i) logits[i] = l16[i];
  return base2_softmax(logits, VOCAB, probs, nullptr);
}

// generate_mini_transformer_streaming_linear_nope_with_priors (lib.rs:12802-12878)
// and its TTT variant (:12880-12980), no priors: the prompt runs through the
// step token by token, then each chosen byte.
int orc_generate_streaming(const TrainModel* m, uint8_t* ctx, size_t n, size_t steps, int strategy, size_t top_k,
                           uint64_t seed, int ttt, uint8_t lr_shift, uint8_t* tokens, int32_t* logit_out,
                           int16_t* prob_out) {
  if (n == 0 || m->H == 0 || m->d % m->H) return 1;
  const size_t hd = m->d / m->H;
  std::vector<int64_t> st(m->H * hd * hd, 0), ks(m->H * hd, 0);
  int32_t logits[VOCAB];
  int16_t probs[VOCAB];
  for (size_t i = 0; i < n; ++i)
    if (!streaming_step(*m, ctx[i], st.data(), ks.data(), ttt != 0, lr_shift, logits, probs)) return 2;
  for (size_t step = 0; step < steps; ++step) {
    const uint8_t tok = select_byte(logits, probs, strategy, top_k, seed, step, ctx, n);
    tokens[step] = tok;
    if (logit_out) logit_out[step] = logits[tok];
    if (prob_out) prob_out[step] = probs[tok];
    ctx[n++] = tok;
    if ((step + 1 < steps || ttt) && !streaming_step(*m, tok, st.data(), ks.data(), ttt != 0, lr_shift, logits, probs))
      return 2;
  }
  return 0;
}

// linear_attention_ttt_delta_state_i16_q15_checked and the state projection
// (attention.rs:1290-1344, :1432-1466) on one head, for known-answer tests.
int orc_linear_attention_ttt_delta(const int16_t* k, const int16_t* v, int64_t* S, int64_t* ks, size_t hd,
                                   uint8_t lr_shift, int16_t* pred, uint64_t* delta_l1) {
  if (hd == 0 || lr_shift > MAX_RIGHT_SHIFT) return 1;
  *delta_l1 = 0;
  return la_ttt_delta(k, v, S, ks, hd, lr_shift, pred, delta_l1) ? 0 : 2;
}
int orc_linear_attention_project(const int16_t* q, const int64_t* S, const int64_t* ks, size_t hd, int16_t* out) {
  return la_project(q, S, ks, hd, out) ? 0 : 2;
}

// The byte-head rows of B windows [B][S] (one per thread of `threads`).
int orc_output_rows(const TrainModel* m, const uint8_t* windows, size_t B, int32_t* logits_q8, int16_t* probs_q15,
                    int threads) {
  std::atomic<int> bad{0};
  std::atomic<size_t> next{0};
  auto run = [&]() {
    for (size_t b; (b = next++) < B;)
      if (!output_row(*m, windows + b * m->S, logits_q8 + b * VOCAB, probs_q15 + b * VOCAB)) bad = 1;
  };
  std::vector<std::thread> pool;
  for (int t = 1; t < std::max(1, threads); ++t) pool.emplace_back(run);
  run();
  for (auto& t : pool) t.join();
  return bad ? 2 : 0;
}

// generate_mini_transformer_with_attention_kind_position_policy_priors_and_ttt_shift
// (nsrl-train/src/lib.rs:12702-12800), base-2 softmax attention, no priors:
// per step the last S bytes of the context, left-padded with ' ', run the
// full forward; the selected byte is appended.  ctx holds the prompt (n
// bytes) and has room for `steps` more; tokens, logit, prob: [steps].
int orc_generate(const TrainModel* m, uint8_t* ctx, size_t n, size_t steps, int strategy, size_t top_k,
                 uint64_t seed, uint8_t* tokens, int32_t* logit_out, int16_t* prob_out) {
  if (n == 0 || m->S == 0) return 1;
  std::vector<uint8_t> win(m->S);
  int32_t logits[VOCAB];
  int16_t probs[VOCAB];
  for (size_t step = 0; step < steps; ++step) {
    const size_t len = std::min(m->S, n);
    std::fill(win.begin(), win.end(), (uint8_t)' ');
    memcpy(win.data() + (m->S - len), ctx + (n - len), len);
    if (!output_row(*m, win.data(), logits, probs)) return 2;
    const uint8_t tok = select_byte(logits, probs, strategy, top_k, seed, step, ctx, n);
    tokens[step] = tok;
    if (logit_out) logit_out[step] = logits[tok];
    if (prob_out) prob_out[step] = probs[tok];
    ctx[n++] = tok;
  }
  return 0;
}

size_t orc_train_arena_len(const TrainModel* m) { return Arena(*m).total; }

// nsrl-train/src/lib.rs:6970-7050 + 7401-7471: windows split into `workers`
// contiguous chunks, each run into private accumulators, merged in worker
// order with checked adds.  stats = {accepted, mlp_sat, attention_sat, residual_sat}.
// Returns 0, or 2 when any window (or the merge) is rejected: the whole batch is.
int orc_train_windows(const TrainModel* m, const uint8_t* contexts, const uint8_t* targets, const int16_t* freq_w,
                      size_t W, int64_t* acc, uint64_t* counts, uint64_t* stats, int workers) {
  const Arena ar(*m);
  const size_t nc = 2 + 9 * m->layers;
  if (W == 0) return 1;
  const size_t nw = (size_t)std::max(1, std::min<int>(workers, (int)W));
  const size_t chunk = (W + nw - 1) / nw;
  std::vector<std::vector<int64_t>> pacc(nw, std::vector<int64_t>(ar.total, 0));
  std::vector<std::vector<uint64_t>> pcnt(nw, std::vector<uint64_t>(nc, 0));
  std::vector<WindowStats> pst(nw, WindowStats{0, 0, 0, 0});
  std::vector<int> pok(nw, 1);
  auto run = [&](size_t w) {
    for (size_t i = w * chunk; i < std::min(W, (w + 1) * chunk); ++i)
      if (!train_window(*m, contexts + i * m->S, targets[i], freq_w, pacc[w].data(), pcnt[w].data(), pst[w])) {
        pok[w] = 0;
        return;
      }
  };
  if (nw == 1) {
    run(0);
  } else {
    std::vector<std::thread> pool;
    for (size_t w = 0; w < nw; ++w) pool.emplace_back(run, w);
    for (auto& t : pool) t.join();
  }
  for (size_t w = 0; w < nw; ++w)
    if (!pok[w]) return 2;
  for (size_t i = 0; i < ar.total; ++i) acc[i] = 0;
  for (size_t c = 0; c < nc; ++c) counts[c] = 0;
  for (int s = 0; s < 4; ++s) stats[s] = 0;
  for (size_t w = 0; w < nw; ++w) {
    for (size_t i = 0; i < ar.total; ++i)
      if (__builtin_add_overflow(acc[i], pacc[w][i], &acc[i])) return 2;
    for (size_t c = 0; c < nc; ++c) counts[c] += pcnt[w][c];
    stats[0] += pst[w].accepted;
    stats[1] += pst[w].mlp_sat;
    stats[2] += pst[w].attn_sat;
    stats[3] += pst[w].res_sat;
  }
  return 0;
}

// One block forward with its caches, for tests of the forward half:
// out = block output, P = probabilities [H][S][S].
int orc_train_block_forward(const TrainModel* m, size_t layer, const int16_t* x, int16_t* out, int16_t* P,
                            uint64_t* res_sat) {
  BlockCache c;
  *res_sat = 0;
  if (!block_forward_cache(*m, m->layer[layer], x, c, res_sat)) return 1;
  memcpy(out, c.out.data(), c.out.size() * 2);
  memcpy(P, c.P.data(), c.P.size() * 2);
  return 0;
}

}  // extern "C"

extern "C" {

// nsrl-train/src/lib.rs:14457-14510: i16 embedding apply (see the CUDA entry
// point of the same name for the rules); stats added to, accumulators kept.
int orc_apply_embedding_gradient_i64_to_i16(const int64_t* acc, int64_t* residuals, int16_t* emb, size_t len,
                                            uint64_t count, int32_t lr, uint8_t shift, uint64_t* stats) {
  if (lr <= 0 || shift > MAX_RIGHT_SHIFT) return 1;
  if (count == 0) return 0;
  if (count > (uint64_t)INT64_MAX) return 1;
  for (size_t i = 0; i < len; ++i) {
    if (acc[i] == 0 && residuals[i] == 0) continue;
    int64_t avg, product;
    if (!round_ratio_i64(acc[i], (int64_t)count, &avg)) return 2;
    if (__builtin_mul_overflow(avg, (int64_t)lr, &product)) return 2;
    if (__builtin_add_overflow(product, residuals[i], &product)) return 2;
    const int64_t scaled = rhu(product, shift);
    if (shift == 0) {
      residuals[i] = 0;
    } else {
      __int128 r = (__int128)product - ((__int128)scaled << shift);
      if (r < INT64_MIN || r > INT64_MAX) return 2;
      residuals[i] = (int64_t)r;
    }
    const int64_t delta = -scaled;
    if (delta == 0) stats[1] += 1;
    const int16_t prev = emb[i];
    int64_t unclamped;
    if (__builtin_add_overflow((int64_t)prev, delta, &unclamped)) return 2;
    const int16_t cl = saturate_i16(unclamped);
    if ((int64_t)cl != unclamped) stats[0] += 1;
    const int64_t ad = (int64_t)cl - (int64_t)prev;
    stats[2] += (uint64_t)(ad < 0 ? -ad : ad);
    emb[i] = cl;
  }
  return 0;
}

}  // extern "C"

// ------------------------------------------------------------ integer Adam --
// crates/nsrl-train-core/src/lib.rs:276-310 (config), :469-661 (apply and delta).
namespace orc {

struct AdamConfig {
  int32_t learning_rate;
  uint8_t step_shift, beta1_decay_shift, beta2_decay_shift, pad;
  uint64_t epsilon;
};

static bool adam_valid(const AdamConfig& c) {  // lib.rs:299-309
  return c.learning_rate > 0 && c.beta1_decay_shift > 0 && c.beta2_decay_shift > 0 &&
         c.beta1_decay_shift <= MAX_RIGHT_SHIFT && c.beta2_decay_shift <= MAX_RIGHT_SHIFT &&
         c.step_shift <= MAX_RIGHT_SHIFT - Q15_SHIFT && c.epsilon > 0;
}

// lib.rs:663-679
static bool rhu128(__int128 v, uint8_t s, __int128* out) {
  if (s == 0) {
    *out = v;
    return true;
  }
  const __int128 off = (__int128)1 << (s - 1);
  const __int128 lim = ~((__int128)1 << 127);
  if (v > lim - off) return false;
  *out = (v + off) >> s;
  return true;
}
static bool rhu128_i64(__int128 v, uint8_t s, int64_t* out) {
  __int128 r;
  if (!rhu128(v, s, &r) || r < INT64_MIN || r > INT64_MAX) return false;
  *out = (int64_t)r;
  return true;
}

// lib.rs:602-661
static bool adam_delta(int64_t g, const AdamConfig& c, int64_t* m1, uint64_t* m2, int64_t* res, int64_t* delta,
                       bool* sat) {
  const int64_t lim = INT32_MAX;
  const int64_t bg = std::clamp<int64_t>(g, -lim, lim);
  *sat = bg != g;
  const __int128 b1 = (__int128)1 << c.beta1_decay_shift;
  if (!rhu128_i64((__int128)*m1 * (b1 - 1) + bg, c.beta1_decay_shift, m1)) return false;
  const __int128 sq = (__int128)bg * bg;
  const __int128 b2 = (__int128)1 << c.beta2_decay_shift;
  __int128 n2;
  if (!rhu128((__int128)*m2 * (b2 - 1) + sq, c.beta2_decay_shift, &n2)) return false;
  if (n2 < 0 || n2 > (__int128)UINT64_MAX) return false;
  *m2 = (uint64_t)n2;
  uint64_t var;
  if (__builtin_add_overflow(*m2, c.epsilon, &var)) return false;
  int64_t inv;
  if (!integer_rsqrt_q30(var, &inv)) return false;
  int64_t n15;
  if (!rhu128_i64((__int128)*m1 * inv, Q15_SHIFT, &n15)) return false;
  n15 = std::clamp<int64_t>(n15, -32767, 32767);
  int64_t num;
  if (__builtin_mul_overflow(n15, (int64_t)c.learning_rate, &num)) return false;
  if (__builtin_add_overflow(num, *res, &num)) return false;
  const uint8_t eff = Q15_SHIFT + c.step_shift;
  const int64_t scaled = rhu(num, eff);
  const __int128 r = (__int128)num - ((__int128)scaled << eff);
  if (r < INT64_MIN || r > INT64_MAX) return false;
  *res = (int64_t)r;
  *delta = -scaled;
  return true;
}

template <class W>
static int adam_apply(const int64_t* acc, uint64_t count, W* w, size_t len, const AdamConfig& c, int64_t* m1,
                      uint64_t* m2, int64_t* res, uint64_t* step, uint64_t* stats, int64_t lo, int64_t hi) {
  stats[0] = stats[1] = stats[2] = 0;
  if (!adam_valid(c)) return 1;
  if (count == 0) return 0;
  if (count > (uint64_t)INT64_MAX) return 1;
  for (size_t i = 0; i < len; ++i) {
    int64_t g;
    if (!round_ratio_i64(acc[i], (int64_t)count, &g)) return 2;
    int64_t delta;
    bool sat;
    if (!adam_delta(g, c, &m1[i], &m2[i], &res[i], &delta, &sat)) return 2;
    if (sat) stats[0] += 1;
    if (delta == 0) stats[1] += 1;
    int64_t un;
    if (__builtin_add_overflow((int64_t)w[i], delta, &un)) return 2;
    const int64_t cl = std::clamp<int64_t>(un, lo, hi);
    if (cl != un) {
      stats[0] += 1;
      res[i] = 0;
    }
    const int64_t ad = cl - (int64_t)w[i];
    stats[2] += (uint64_t)(ad < 0 ? -ad : ad);
    w[i] = (W)cl;
  }
  *step += 1;
  return 0;
}

}  // namespace orc

extern "C" {

// apply_integer_adam_accumulators_i64_to_i8 / _to_i16 (lib.rs:469-593):
// 0 = ok, 1 = invalid config, 2 = rejected.  stats = {saturations, zero deltas, sum |delta|}.
int orc_integer_adam_i8(const int64_t* acc, uint64_t count, int8_t* w, size_t len, const AdamConfig* c, int64_t* m1,
                        uint64_t* m2, int64_t* res, uint64_t* step, uint64_t* stats) {
  return adam_apply(acc, count, w, len, *c, m1, m2, res, step, stats, -128, 127);
}
int orc_integer_adam_i16(const int64_t* acc, uint64_t count, int16_t* w, size_t len, const AdamConfig* c, int64_t* m1,
                         uint64_t* m2, int64_t* res, uint64_t* step, uint64_t* stats) {
  return adam_apply(acc, count, w, len, *c, m1, m2, res, step, stats, -32768, 32767);
}

}  // extern "C"
