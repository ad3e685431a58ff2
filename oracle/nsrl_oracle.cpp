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
