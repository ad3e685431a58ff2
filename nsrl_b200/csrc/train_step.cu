// The integer training step of the reference's mini transformer on one GPU:
// backward-input linears, gated-MLP / RMS-norm / softmax-attention backward,
// i64 weight-gradient accumulation and the map-reduce window loop
// (crates/nsrl-train/src/lib.rs:7051-7399 and the functions it calls).
//
// Layout: every activation is token-major int16 [windows * seq_len][dim]; a
// batch of W windows is one T = W * seq_len row problem, so each linear of
// the reference's per-token loops is one GEMM over T rows.
//   * Forward linears: the tcgen05 GEMM of linear_tc.cu (byte planes).
//   * Backward-input linears (dx = g' W): the same GEMM in its wide form, A =
//     byte planes of the prescaled gradient, B = W transposed once per call,
//     i64 recombination and requantize_i64_to_i16 in the epilogue.
//   * Weight gradients acc += g'^T x: tiled SIMT in i64.
//   * Attention backward: a row kernel for dP / dL and three tiled SIMT
//     products for dQ, dK, dV.
// Caches of every layer (the reference's MiniTransformerBlockForwardCache,
// lib.rs:15282-15299) stay in the workspace between the forward and the
// backward.
#include <algorithm>
#include <vector>

#include "train_step_kernels.cuh"

namespace nsrl {
namespace {

using namespace ts;

constexpr size_t ALIGN = 256;
size_t up256(size_t b) { return (b + ALIGN - 1) & ~(ALIGN - 1); }

struct Carve {
  uint8_t* base;
  size_t off = 0;
  explicit Carve(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t count) {
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += up256(count * sizeof(T));
    return p;
  }
  Planes planes(size_t rows, size_t ld, bool l1) {
    Planes p;
    p.hi = take<int8_t>(rows * ld);
    p.lo = take<uint8_t>(rows * ld);
    p.l1 = l1 ? take<unsigned long long>(rows) : nullptr;
    p.ld = ld;
    return p;
  }
};

unsigned blocks_for(long long n, long long cap = 148 * 16) {
  return (unsigned)std::max<long long>(1, std::min<long long>((n + 255) / 256, cap));
}

nsrl_status fail_cuda(cudaError_t e, const char* what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return NSRL_CUDA_ERROR;
}
nsrl_status fail_shape(const char* what) {
  set_error("invalid shape: %s", what);
  return NSRL_INVALID_SHAPE;
}

#define TS_TRY(call, what)                           \
  do {                                               \
    cudaError_t _e = (call);                         \
    if (_e != cudaSuccess) return fail_cuda(_e, what); \
  } while (0)

#define TS_TRY_RET(call)                 \
  do {                                   \
    cudaError_t _e = (call);             \
    if (_e != cudaSuccess) return _e;    \
  } while (0)

bool aligned_to(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

bool is_pow4(size_t v) { return v != 0 && (v & (v - 1)) == 0 && (__builtin_ctzll(v) % 2) == 0; }

__global__ void fill_identity_kernel(nsrl_fixed_scale* s, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    s[i] = nsrl_fixed_scale{1, 0, {0, 0, 0}};
}

// Flags a forward multiplier other than 1: the tensor-core backward path
// needs the prescaled gradient to fit int16.
#define NSRL_FLAG_SCALE_UNSUPPORTED 0x20ull
__global__ void check_mult_one_kernel(const nsrl_fixed_scale* s, int n, int* out_flag, nsrl_device_status* st) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    if (s[i].multiplier != 1) {
      if (out_flag) atomicOr(out_flag, 1);
      if (st) nsrl_flag(st, NSRL_FLAG_SCALE_UNSUPPORTED);
    }
}

// SIMT backward-input, run only when the device flag says a multiplier is not 1.
__global__ void bwd_input_simt_if_kernel(const int* flag, const int16_t* g, long long M, int N, const int8_t* w, int K,
                                         const nsrl_fixed_scale* fsc, const nsrl_fixed_scale* gsc, int16_t* dx,
                                         nsrl_device_status* st) {
  if (!*flag) return;
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
      acc += gs * (long long)w[(long long)n * K + k];
    }
    const nsrl_fixed_scale s = gsc[k];
    const long long lo = (long long)((unsigned long long)acc * (unsigned long long)(long long)s.multiplier);
    if (__mul64hi(acc, (long long)s.multiplier) != (lo >> 63)) bad = true;
    dx[m * K + k] = sat_i16(rhu64(lo, s.right_shift));
    if (bad) nsrl_flag(st, NSRL_FLAG_LINEAR_OVERFLOW);
  }
}

cudaError_t transpose(const int8_t* w, size_t R, size_t C, int8_t* wt, cudaStream_t s) {
  dim3 grid((unsigned)((C + 31) / 32), (unsigned)((R + 31) / 32));
  ProfScope prof("transpose_weights", s, 0.0, 2.0 * (double)R * (double)C);
  transpose_i8_kernel<<<grid, dim3(32, 8), 0, s>>>(w, (int)R, (int)C, wt);
  return cudaGetLastError();
}

cudaError_t prescale_split(const int16_t* g, size_t M, size_t N, size_t ldg, const nsrl_fixed_scale* sc, Planes out,
                           cudaStream_t s) {
  const long long n = (long long)M * (long long)N;
  ProfScope prof("prescale_split", s, 0.0, 4.0 * (double)n);
  if (N % 8 == 0 && ldg == N && out.ld == N && aligned_to(g, 16) && aligned_to(out.hi, 8) && aligned_to(out.lo, 8))
    return launch_pdl(prescale_split_vec_kernel, dim3(blocks_for(n / 8, 148 * 32)), dim3(256), 0, s, g, n / 8, (int)N,
                      sc, out.hi, out.lo);
  else
    prescale_split_kernel<<<blocks_for(n, 148 * 32), 256, 0, s>>>(g, (long long)M, (int)N, (long long)ldg, sc,
                                                                   out.hi, out.lo, (long long)out.ld);
  return cudaGetLastError();
}

// dx [M][K_out] (+ skip, saturating, counted) from planes of g' [M][N_red] and W^T [K_out][N_red].
cudaError_t bwd_gemm(const Planes& a, size_t M, size_t N_red, const int8_t* wt, size_t K_out,
                     const nsrl_fixed_scale* gin, int16_t* y, size_t ldy, const int16_t* skip,
                     unsigned long long* sat, nsrl_device_status* st, cudaStream_t s) {
  GemmArgs g{};
  g.a_hi = a.hi;
  g.a_lo = a.lo;
  g.a_l1 = nullptr;
  g.lda = a.ld;
  g.M = M;
  g.K = N_red;
  g.nseg = 1;
  g.seg[0] = WeightSeg{wt, nullptr, gin, K_out};
  g.epi = skip ? Epi::RESID : Epi::I16;
  g.y = y;
  g.ldy = ldy;
  g.skip = skip;
  g.ldskip = ldy;
  g.sat_counter = sat;
  g.st = st;
  g.wide = true;
  return launch_gemm(g, s);
}

cudaError_t fwd_gemm(const Planes& a, size_t M, size_t K, const nsrl_linear_params* p, Epi epi, int16_t* y, size_t ldy,
                     const int16_t* skip, unsigned long long* sat, nsrl_device_status* st, cudaStream_t s) {
  GemmArgs g{};
  g.a_hi = a.hi;
  g.a_lo = a.lo;
  g.a_l1 = a.l1;
  g.lda = a.ld;
  g.M = M;
  g.K = K;
  g.nseg = 1;
  g.seg[0] = WeightSeg{p->weights, p->bias, p->scales, p->output_dim};
  g.epi = epi;
  g.y = y;
  g.ldy = ldy;
  g.skip = skip;
  g.ldskip = ldy;
  g.sat_counter = sat;
  g.st = st;
  return launch_gemm(g, s);
}

cudaError_t accumulate(const int16_t* x, size_t ldx, const int16_t* g, size_t ldg, const nsrl_fixed_scale* sc,
                       size_t rows, size_t K, size_t N, long long* acc, nsrl_device_status* st, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  dim3 grid((unsigned)((K + ATK - 1) / ATK), (unsigned)((N + ATN - 1) / ATN));
  ProfScope prof("accumulate_weight_grad", s, 2.0 * (double)rows * (double)K * (double)N,
                 2.0 * (double)rows * (double)(K + N) + 16.0 * (double)K * (double)N);
  accumulate_pre_kernel<<<grid, 256, 0, s>>>(x, (long long)ldx, g, (long long)ldg, sc, (int)rows, (int)K, (int)N, acc,
                                             st);
  return cudaGetLastError();
}

// acc [N][K] += sum over rows of g'[r][n] x[r][k] from byte planes: g' [rows][N]
// already prescaled by rhu(g, shift_n) (multipliers are 1 here) and x
// [rows][K], as their producers write them.  The tensor-core kernel reads them
// in place; the SIMT kernel takes operands TMA cannot.
cudaError_t accumulate_planes(const Planes& g, const Planes& x, size_t rows, size_t K, size_t N, long long* acc,
                              nsrl_device_status* st, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const cudaError_t e = launch_wgrad_tc(g.hi, g.lo, g.ld, x.hi, x.lo, x.ld, rows, N, K, acc, st, s);
  if (e != cudaErrorNotSupported) return e;
  dim3 grid((unsigned)((K + ATK - 1) / ATK), (unsigned)((N + ATN - 1) / ATN));
  ProfScope prof("accumulate_weight_grad", s, 2.0 * (double)rows * (double)K * (double)N,
                 2.0 * (double)rows * (double)(K + N) + 16.0 * (double)K * (double)N);
  accumulate_planes_kernel<<<grid, 256, 0, s>>>(g.hi, g.lo, (long long)g.ld, x.hi, x.lo, (long long)x.ld, (int)rows,
                                                (int)K, (int)N, acc);
  return cudaGetLastError();
}

cudaError_t add_sat(const int16_t* a, const int16_t* b, size_t n, int16_t* out, unsigned long long* sat,
                    cudaStream_t s);

// RMS-norm backward of the rows of x (rms_norm.rs:140-190).  With res, out =
// sat(res + gi) (the residual add of the block backward, saturations into
// res_sat); gi is then scratch that only the fallback path writes.
cudaError_t rms_backward(const int16_t* x, size_t rows, size_t d, const int16_t* w, const int16_t* go, uint64_t eps,
                         int16_t* gi, long long* gw, unsigned long long* sat, nsrl_device_status* st, cudaStream_t s,
                         const int16_t* res = nullptr, int16_t* out = nullptr,
                         unsigned long long* res_sat = nullptr) {
  if (rows == 0) return cudaSuccess;
  const size_t smem = d * sizeof(long long);
  // d = 256: the 16-byte row kernel, two rows per warp (wider rows stay on
  // the kernels below, which hold fewer values per lane)
  if (d == 256 && aligned_to(x, 16) && aligned_to(w, 16) && aligned_to(go, 16) &&
      aligned_to(res ? (const void*)res : (const void*)gi, 16) && aligned_to(res ? (void*)out : (void*)gi, 16)) {
    ProfScope prof("rms_backward", s, 0.0, (res ? 8.0 : 6.0) * (double)rows * (double)d);
    return launch_pdl(rms_backward_vec_kernel<2>, dim3(blocks_for((long long)(rows + 1) / 2 * 32, 148 * 8)), dim3(256),
                      0, s, x, (long long)rows, w, go, (unsigned long long)eps, gi, gw, sat, st, res, out, res_sat);
  }
  if (res) {
    const cudaError_t e = rms_backward(x, rows, d, w, go, eps, gi, gw, sat, st, s);
    if (e != cudaSuccess) return e;
    return add_sat(res, gi, rows * d, out, res_sat, s);
  }
  ProfScope prof("rms_backward", s, 0.0, 6.0 * (double)rows * (double)d);
  if (d % 32 == 0 && d <= 512) {
    const unsigned blocks = blocks_for((long long)rows * 32, 148 * 8);
#define TS_RMS_CASE(N)                                                                                   \
  case N:                                                                                                \
    rms_backward_reg_kernel<N><<<blocks, 256, 0, s>>>(x, (long long)rows, w, go, eps, gi, gw, sat, st); \
    return cudaGetLastError();
    switch (d / 32) {
      TS_RMS_CASE(1)
      TS_RMS_CASE(2)
      TS_RMS_CASE(4)
      TS_RMS_CASE(8)
      TS_RMS_CASE(16)
      default:
        break;
    }
#undef TS_RMS_CASE
  }
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(rms_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  rms_backward_kernel<<<blocks_for((long long)rows * 32, 148 * 8), 256, smem, s>>>(
      x, (long long)rows, (int)d, 1.0 / (double)d, w, go, eps, gi, gw, sat, st);
  return cudaGetLastError();
}

cudaError_t add_sat(const int16_t* a, const int16_t* b, size_t n, int16_t* out, unsigned long long* sat,
                    cudaStream_t s) {
  ProfScope prof("add_saturating", s, 0.0, 6.0 * (double)n);
  if (n % 8 == 0 && aligned_to(a, 16) && aligned_to(b, 16) && aligned_to(out, 16))
    return launch_pdl(add_sat_vec_kernel, dim3(blocks_for((long long)n / 8, 148 * 32)), dim3(256), 0, s, a, b,
                      (long long)n / 8, out, sat);
  else
    add_sat_kernel<<<blocks_for((long long)n), 256, 0, s>>>(a, b, (long long)n, out, sat);
  return cudaGetLastError();
}

// dL, then dQ, dK, dV of one attention layer (nsrl-train/src/lib.rs:16623-16900);
// with `planes`, the prescaled planes of dQ, dK, dV (ld d) for their
// backward-input linears and weight gradients (the tensor-core kernels then
// leave the int16 dq, dk, dv unwritten).
cudaError_t attn_backward(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld, const int16_t* P,
                          const int16_t* dC, size_t ldc, size_t B, size_t S, size_t d, size_t H, int16_t* dL,
                          int16_t* dq, int16_t* dk, int16_t* dv, void* scratch, size_t scratch_bytes,
                          nsrl_device_status* st, cudaStream_t s, const GradPlanes* planes = nullptr,
                          const Planes* p_planes = nullptr, const Planes* qkv_planes = nullptr) {
  const cudaError_t tce = launch_attention_backward_tc(q, k, v, ld, P, dC, ldc, B, S, d, H, dL, dq, dk, dv, scratch,
                                                       scratch_bytes, st, s, planes, p_planes, qkv_planes);
  if (tce != cudaErrorNotSupported) return tce;
  if (p_planes || qkv_planes) return cudaErrorInvalidValue;  // only the tensor-core path reads planes
  if (planes) {
    const cudaError_t e = attn_backward(q, k, v, ld, P, dC, ldc, B, S, d, H, dL, dq, dk, dv, scratch, scratch_bytes,
                                        st, s, nullptr);
    if (e != cudaSuccess) return e;
    const int16_t* g[3] = {dq, dk, dv};
    for (int i = 0; i < 3; ++i)
      TS_TRY_RET(prescale_split(g[i], B * S, d, d, planes[i].sc, Planes{planes[i].hi, planes[i].lo, nullptr, d}, s));
    return cudaSuccess;
  }
  const size_t hd = d / H;
  const int shift = __builtin_ctzll(hd) / 2;
  const size_t smem = S * sizeof(int32_t);
  const double pairs = (double)B * (double)H * (double)S * (double)(S + 1) / 2.0;
  {
    dim3 grid((unsigned)S, (unsigned)H, (unsigned)B);
    ProfScope prof("attention_dlogit", s, 2.0 * (double)hd * pairs, 4.0 * (double)B * (double)H * (double)S * S);
    if (hd == 64) {
      if (smem > 48 * 1024)
        TS_TRY_RET(cudaFuncSetAttribute(attn_dlogit_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attn_dlogit_kernel<8><<<grid, 256, smem, s>>>(dC, (long long)ldc, v, (long long)ld, P, (int)S, (int)H, dL, st);
    } else {
      if (smem > 48 * 1024)
        TS_TRY_RET(cudaFuncSetAttribute(attn_dlogit_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      attn_dlogit_kernel<2><<<grid, 256, smem, s>>>(dC, (long long)ldc, v, (long long)ld, P, (int)S, (int)H, dL, st);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  dim3 grid((unsigned)((S + 63) / 64), (unsigned)H, (unsigned)B);
  ProfScope prof("attention_grad_products", s, 3.0 * 2.0 * (double)hd * pairs,
                 3.0 * 2.0 * (double)B * (double)H * (double)S * S + 12.0 * (double)B * S * d);
  if (hd == 64) {
    attn_grad_gemm_kernel<0, 64><<<grid, 256, 0, s>>>(dL, k, (long long)ld, (int)S, (int)H, shift, dq, (long long)d);
    attn_grad_gemm_kernel<1, 64><<<grid, 256, 0, s>>>(dL, q, (long long)ld, (int)S, (int)H, shift, dk, (long long)d);
    attn_grad_gemm_kernel<2, 64><<<grid, 256, 0, s>>>(P, dC, (long long)ldc, (int)S, (int)H, 15, dv, (long long)d);
  } else {
    attn_grad_gemm_kernel<0, 16><<<grid, 256, 0, s>>>(dL, k, (long long)ld, (int)S, (int)H, shift, dq, (long long)d);
    attn_grad_gemm_kernel<1, 16><<<grid, 256, 0, s>>>(dL, q, (long long)ld, (int)S, (int)H, shift, dk, (long long)d);
    attn_grad_gemm_kernel<2, 16><<<grid, 256, 0, s>>>(P, dC, (long long)ldc, (int)S, (int)H, 15, dv, (long long)d);
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------------ layout --
struct LayerCache {
  // P: [W][H][S][S] int16, or (p_planes) the same bytes as its two byte planes,
  // hi then lo, in the causal form the tensor-core forward writes
  int16_t *in, *qkv, *P, *ares, *up, *gate, *out;
  bool p_planes;
  // q|k|v as row-major byte planes [T][3d] (the tensor-core attention's input;
  // with p_planes the backward reads them too and qkv is not written)
  Planes pqkv;
  // inputs of the linears as byte planes (+ row L1): the forward GEMMs read
  // them and the weight gradients read them again in the backward
  Planes an, ctx, mn, gated;  // q|k|v input, o input, up|gate input, down input
  int8_t *wt[7];  // transposed q k v o (d x d), up, gate ([d][F]), down ([F][d])
};

// The cached P buffer (n int16 entries) viewed as two byte planes of row length ld.
Planes p_cache_planes(const LayerCache& c, size_t n, size_t ld) {
  int8_t* hi = reinterpret_cast<int8_t*>(c.P);
  return Planes{hi, reinterpret_cast<uint8_t*>(hi + n), nullptr, ld};
}

struct StepLayout {
  size_t W, S, T, d, F, H, L;
  bool rms;
  std::vector<LayerCache> lc;
  int16_t* xemb;
  Planes pa, pb;
  int16_t *G, *Gn, *gg, *gui, *gmi, *gmr, *gao, *gctx, *dq, *dk, *dv, *gq, *gk, *gv, *gni, *gai, *dL;
  int16_t *feat, *logits, *hgrad, *glast;
  Planes fp, hp;
  int8_t* headT;
  nsrl_fixed_scale* ident;
  unsigned long long* fwd_res;
  Planes pg[3];  // prescaled planes of dQ, dK, dV
  VtPlanes vt;
  void* abw;    // scratch of the tensor-core attention backward
  size_t abw_bytes;
  size_t bytes;
};

void carve_step(const nsrl_train_model* m, size_t W, bool rms, void* base, StepLayout& o) {
  Carve c(base);
  o.W = W;
  o.S = m->seq_len;
  o.T = W * o.S;
  o.d = m->d_model;
  o.F = m->hidden_dim;
  o.H = m->heads;
  o.L = m->layers;
  o.rms = rms;
  const size_t T = o.T, d = o.d, F = o.F, S = o.S, H = o.H;
  const size_t wide = std::max(d, F);
  o.xemb = c.take<int16_t>(T * d);
  o.lc.resize(o.L);
  for (size_t l = 0; l < o.L; ++l) {
    LayerCache& lc = o.lc[l];
    lc.in = l == 0 ? o.xemb : o.lc[l - 1].out;
    lc.an = c.planes(T, d, true);
    lc.qkv = c.take<int16_t>(T * 3 * d);
    lc.ctx = c.planes(T, d, true);
    lc.P = c.take<int16_t>(W * H * S * S);
    lc.p_planes = false;
    lc.pqkv = attention_tc_supported(S, d, H) ? c.planes(T, 3 * d, false) : Planes{nullptr, nullptr, nullptr, 3 * d};
    lc.ares = c.take<int16_t>(T * d);
    lc.mn = c.planes(T, d, true);
    lc.up = c.take<int16_t>(T * F);
    lc.gate = c.take<int16_t>(T * F);
    lc.gated = c.planes(T, F, true);
    lc.out = c.take<int16_t>(T * d);
    for (int i = 0; i < 4; ++i) lc.wt[i] = c.take<int8_t>(d * d);
    for (int i = 4; i < 7; ++i) lc.wt[i] = c.take<int8_t>(d * F);
  }
  o.pa = c.planes(T, wide, true);
  o.pb = c.planes(T, wide, false);
  int16_t** td[] = {&o.G, &o.Gn, &o.gui, &o.gmi, &o.gmr, &o.gao, &o.gctx, &o.dq, &o.dk, &o.dv,
                    &o.gq, &o.gk, &o.gv, &o.gni, &o.gai};
  for (int16_t** p : td) *p = c.take<int16_t>(T * d);
  o.gg = c.take<int16_t>(T * F);
  o.dL = c.take<int16_t>(W * H * S * S);
  for (int i = 0; i < 3; ++i) o.pg[i] = c.planes(T, d, false);
  o.feat = c.take<int16_t>(W * d);
  o.logits = c.take<int16_t>(W * 256);
  o.hgrad = c.take<int16_t>(W * 256);
  o.glast = c.take<int16_t>(W * d);
  o.fp = c.planes(W, d, true);
  o.hp = c.planes(W, 256, false);
  o.headT = c.take<int8_t>(d * 256);
  o.ident = c.take<nsrl_fixed_scale>(std::max<size_t>(wide, 256));
  o.fwd_res = c.take<unsigned long long>(4);
  o.vt = VtPlanes{nullptr, nullptr, (int)S, (int)H, (int)(d / H), nullptr};
  if (attention_tc_supported(S, d, H)) {
    o.vt.hi = c.take<int8_t>(T * d);
    o.vt.lo = c.take<uint8_t>(T * d);
    const size_t ws = attention_tc_scratch_bytes(W, S, d, H);
    if (ws) o.vt.wscr = c.take<int16_t>(ws / sizeof(int16_t));
  }
  o.abw_bytes = attention_backward_tc_scratch_bytes(W, S, d, H);
  o.abw = c.take<uint8_t>(o.abw_bytes);
  o.bytes = c.off;
}

size_t arena_len(const nsrl_train_model* m) {
  const size_t d = m->d_model, F = m->hidden_dim;
  return 256 * d + m->layers * (4 * d * d + 3 * F * d + 2 * d) + 256 * d + m->seq_len * d;
}

nsrl_status validate_model(const nsrl_train_model* m, bool* rms) {
  if (!m || !m->layer || m->layers == 0) return fail_shape("model with at least one layer");
  if (m->attention_kind != 0) return fail_shape("the training step takes base-2 softmax attention (attention_kind 0)");
  const size_t d = m->d_model, H = m->heads, F = m->hidden_dim, S = m->seq_len;
  if (d == 0 || H == 0 || F == 0 || S == 0 || d % H != 0) return fail_shape("d_model, heads, hidden_dim, seq_len");
  const size_t hd = d / H;
  if (!is_pow4(hd)) return fail_shape("head_dim must be a power of four (attention.rs:1599-1602)");
  if (hd != 16 && hd != 64) return fail_shape("training step: head_dim 16 or 64");
  if (d % 16 != 0 || F % 16 != 0) return fail_shape("training step: d_model and hidden_dim multiples of 16");
  if (!m->embeddings) return fail_shape("embeddings");
  auto lin_ok = [](const nsrl_linear_params& p, size_t in, size_t out) {
    return p.weights && p.scales && p.input_dim == in && p.output_dim == out;
  };
  if (!lin_ok(m->head, d, 256)) return fail_shape("head must be [256][d_model]");
  *rms = m->layer[0].attn_gamma != nullptr;
  for (size_t l = 0; l < m->layers; ++l) {
    const nsrl_train_layer& L = m->layer[l];
    if ((L.attn_gamma != nullptr) != *rms || (L.mlp_gamma != nullptr) != *rms)
      return fail_shape("RMS gammas: both or neither, the same in every layer");
    for (int i = 0; i < 4; ++i)
      if (!lin_ok(L.lin[i], d, d)) return fail_shape("q, k, v, o must be [d][d]");
    if (!lin_ok(L.lin[4], d, F) || !lin_ok(L.lin[5], d, F)) return fail_shape("up, gate must be [hidden][d]");
    if (!lin_ok(L.lin[6], F, d)) return fail_shape("down must be [d][hidden]");
  }
  return NSRL_OK;
}

}  // namespace
}  // namespace nsrl

using namespace nsrl;

extern "C" {

// ---------------------------------------------------- backward primitives --
size_t nsrl_linear_backward_input_workspace_size(size_t rows, size_t input_dim, size_t output_dim) {
  return up256(rows * output_dim) * 2 + up256(input_dim * output_dim) + up256(input_dim * sizeof(nsrl_fixed_scale)) +
         ALIGN;
}

nsrl_status nsrl_linear_backward_input(const int16_t* grad_output, size_t rows, const nsrl_linear_params* p,
                                       const nsrl_fixed_scale* gin, int16_t* dx, void* workspace,
                                       size_t workspace_bytes, nsrl_device_status* st, void* stream) {
  if (!p || !p->weights || !p->scales || p->input_dim == 0 || p->output_dim == 0 || !st)
    return fail_shape("linear backward input params");
  if (rows == 0) return NSRL_OK;
  if (p->output_dim > 66000 || rows > (size_t)INT32_MAX) return fail_shape("output_dim <= 66000");
  const size_t K = p->input_dim, N = p->output_dim;
  if (!workspace || workspace_bytes < nsrl_linear_backward_input_workspace_size(rows, K, N))
    return fail_shape("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  Carve c(workspace);
  Planes a;
  a.hi = c.take<int8_t>(rows * N);
  a.lo = c.take<uint8_t>(rows * N);
  a.l1 = nullptr;
  a.ld = N;
  int8_t* wt = c.take<int8_t>(K * N);
  nsrl_fixed_scale* ident = c.take<nsrl_fixed_scale>(K);
  int* flag = c.take<int>(1);
  if (!gin) {
    fill_identity_kernel<<<blocks_for((long long)K), 256, 0, s>>>(ident, (int)K);
    gin = ident;
  }
  TS_TRY(cudaMemsetAsync(flag, 0, sizeof(int), s), "backward input");
  check_mult_one_kernel<<<blocks_for((long long)N), 256, 0, s>>>(p->scales, (int)N, flag, nullptr);
  TS_TRY(transpose(p->weights, N, K, wt, s), "transpose");
  TS_TRY(prescale_split(grad_output, rows, N, N, p->scales, a, s), "prescale");
  TS_TRY(bwd_gemm(a, rows, N, wt, K, gin, dx, K, nullptr, nullptr, st, s), "backward-input linear");
  // a multiplier other than 1: the tensor-core result is replaced by the exact SIMT one
  bwd_input_simt_if_kernel<<<blocks_for((long long)rows * K, 148 * 32), 256, 0, s>>>(
      flag, grad_output, (long long)rows, (int)N, p->weights, (int)K, p->scales, gin, dx, st);
  TS_TRY(cudaGetLastError(), "backward input");
  return NSRL_OK;
}

size_t nsrl_gated_mlp_backward_input_workspace_size(size_t rows, size_t d, size_t F) {
  return 4 * up256(rows * F) + up256(rows * F * 2) + up256(rows * d * 2) + 3 * up256(d * F) +
         up256(std::max(d, F) * sizeof(nsrl_fixed_scale)) + ALIGN;
}

nsrl_status nsrl_gated_mlp_backward_input(const int16_t* grad_output, size_t rows, size_t d, size_t F,
                                          const nsrl_linear_params* up, const nsrl_linear_params* gate,
                                          const nsrl_linear_params* down, const int16_t* fwd_up,
                                          const int16_t* fwd_gate, int16_t* grad_up, int16_t* grad_gate,
                                          int16_t* grad_input, unsigned long long* sat, void* workspace,
                                          size_t workspace_bytes, nsrl_device_status* st, void* stream) {
  auto ok = [](const nsrl_linear_params* p, size_t in, size_t out) {
    return p && p->weights && p->scales && p->input_dim == in && p->output_dim == out;
  };
  if (!ok(up, d, F) || !ok(gate, d, F) || !ok(down, F, d) || !st || !sat) return fail_shape("gated MLP params");
  if (rows == 0) return NSRL_OK;
  if (d % 16 != 0 || F % 16 != 0) return fail_shape("d_model and hidden_dim multiples of 16");
  if (d > F) return fail_shape("gated MLP backward: d_model <= hidden_dim");
  if (!workspace || workspace_bytes < nsrl_gated_mlp_backward_input_workspace_size(rows, d, F))
    return fail_shape("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  Carve c(workspace);
  Planes pu{c.take<int8_t>(rows * F), c.take<uint8_t>(rows * F), nullptr, F};
  Planes pg{c.take<int8_t>(rows * F), c.take<uint8_t>(rows * F), nullptr, F};
  int16_t* gg = c.take<int16_t>(rows * F);
  int16_t* gui = c.take<int16_t>(rows * d);
  int8_t* downT = c.take<int8_t>(d * F);
  int8_t* upT = c.take<int8_t>(d * F);
  int8_t* gateT = c.take<int8_t>(d * F);
  nsrl_fixed_scale* ident = c.take<nsrl_fixed_scale>(std::max(d, F));
  fill_identity_kernel<<<blocks_for((long long)std::max(d, F)), 256, 0, s>>>(ident, (int)std::max(d, F));
  for (const nsrl_linear_params* p : {up, gate})
    check_mult_one_kernel<<<blocks_for((long long)F), 256, 0, s>>>(p->scales, (int)F, nullptr, st);
  check_mult_one_kernel<<<blocks_for((long long)d), 256, 0, s>>>(down->scales, (int)d, nullptr, st);
  TS_TRY(transpose(down->weights, d, F, downT, s), "transpose");
  TS_TRY(transpose(up->weights, F, d, upT, s), "transpose");
  TS_TRY(transpose(gate->weights, F, d, gateT, s), "transpose");
  // down^T: the grad planes reuse pu (rows * d <= rows * F)
  Planes pd{pu.hi, pu.lo, nullptr, d};
  TS_TRY(prescale_split(grad_output, rows, d, d, down->scales, pd, s), "prescale");
  TS_TRY(bwd_gemm(pd, rows, d, downT, F, ident, gg, F, nullptr, nullptr, st, s), "down^T");
  {
    const long long n = (long long)rows * F;
    ProfScope prof("gated_backward", s, 0.0, 14.0 * (double)n);
    gated_backward_kernel<<<blocks_for(n, 148 * 32), 256, 0, s>>>(gg, fwd_up, fwd_gate, n, (int)F, up->scales,
                                                                  gate->scales, grad_up, grad_gate, pu.hi, pu.lo,
                                                                  pg.hi, pg.lo);
    TS_TRY(cudaGetLastError(), "gated backward");
  }
  TS_TRY(bwd_gemm(pu, rows, F, upT, d, ident, gui, d, nullptr, nullptr, st, s), "up^T");
  TS_TRY(bwd_gemm(pg, rows, F, gateT, d, ident, grad_input, d, gui, sat, st, s), "gate^T");
  return NSRL_OK;
}

nsrl_status nsrl_rms_norm_backward_rows(const int16_t* x, size_t rows, size_t d, const int16_t* gamma,
                                        const int16_t* go, uint64_t eps, int16_t* gi, long long* gw,
                                        unsigned long long* sat, nsrl_device_status* st, void* stream) {
  if (d == 0 || d > 16384 || !x || !gamma || !go || !gi || !gw || !sat || !st) return fail_shape("rms backward");
  TS_TRY(rms_backward(x, rows, d, gamma, go, eps, gi, gw, sat, st, (cudaStream_t)stream), "rms backward");
  return NSRL_OK;
}

nsrl_status nsrl_attention_with_probabilities(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld,
                                              size_t B, size_t S, size_t d, size_t H, int16_t* ctx, int16_t* P,
                                              nsrl_device_status* st, void* stream) {
  if (B == 0 || S == 0 || d == 0 || H == 0 || d % H != 0 || !is_pow4(d / H)) return fail_shape("attention shape");
  if (S > 16384) return fail_shape("seq_len <= 16384");
  TS_TRY(launch_attention_rows_probs(q, k, v, ld, B, S, d, H, ctx, P, st, (cudaStream_t)stream), "attention");
  return NSRL_OK;
}

size_t nsrl_attention_backward_workspace_size(size_t B, size_t S, size_t d, size_t H) {
  return up256(B * H * S * S * 2) + attention_backward_tc_scratch_bytes(B, S, d, H);
}

nsrl_status nsrl_attention_backward(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld, const int16_t* P,
                                    const int16_t* dC, size_t B, size_t S, size_t d, size_t H, int16_t* dq,
                                    int16_t* dk, int16_t* dv, void* workspace, size_t workspace_bytes,
                                    nsrl_device_status* st, void* stream) {
  if (B == 0 || S == 0 || d == 0 || H == 0 || d % H != 0) return fail_shape("attention backward shape");
  const size_t hd = d / H;
  if (!is_pow4(hd)) return fail_shape("head_dim must be a power of four");
  if (hd != 16 && hd != 64) return fail_shape("attention backward: head_dim 16 or 64");
  if (ld % 8 != 0 || d % 8 != 0 || S > 16384) return fail_shape("row strides multiples of 8, seq_len <= 16384");
  if (!workspace || workspace_bytes < nsrl_attention_backward_workspace_size(B, S, d, H))
    return fail_shape("workspace too small");
  const size_t dl_bytes = up256(B * H * S * S * 2);
  TS_TRY(attn_backward(q, k, v, ld, P, dC, d, B, S, d, H, static_cast<int16_t*>(workspace), dq, dk, dv,
                       static_cast<uint8_t*>(workspace) + dl_bytes, workspace_bytes - dl_bytes, st,
                       (cudaStream_t)stream),
         "attention backward");
  return NSRL_OK;
}

// Rows of the byte planes of the standalone weight gradient: 16-byte multiples (TMA strides).
size_t plane_ld(size_t dim) { return (dim + 15) & ~size_t(15); }

size_t nsrl_accumulate_weight_gradient_i16_workspace_size(size_t rows, size_t input_dim, size_t output_dim) {
  return 2 * up256(rows * plane_ld(output_dim)) + 2 * up256(rows * plane_ld(input_dim));
}

nsrl_status nsrl_accumulate_weight_gradient_i16(const int16_t* x, const int16_t* grad_output, size_t rows,
                                                size_t input_dim, size_t output_dim, const nsrl_fixed_scale* scales,
                                                long long* accumulators, unsigned long long* sample_count,
                                                void* workspace, size_t workspace_bytes, nsrl_device_status* st,
                                                void* stream) {
  if (input_dim == 0 || output_dim == 0 || !x || !grad_output || !scales || !accumulators || !sample_count || !st)
    return fail_shape("weight-gradient accumulation");
  if (rows > (size_t)INT32_MAX || input_dim > (size_t)INT32_MAX || output_dim > (size_t)INT32_MAX)
    return fail_shape("dimension too large");
  if (rows == 0) return NSRL_OK;
  if (!workspace || workspace_bytes < nsrl_accumulate_weight_gradient_i16_workspace_size(rows, input_dim, output_dim))
    return fail_shape("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  Carve c(workspace);
  // byte planes of g' = rhu(g, shift_n) and of x, row-major as the kernel reads them
  const Planes gp = c.planes(rows, plane_ld(output_dim), false);
  const Planes xp = c.planes(rows, plane_ld(input_dim), false);
  check_mult_one_kernel<<<blocks_for((long long)output_dim), 256, 0, s>>>(scales, (int)output_dim, nullptr, st);
  TS_TRY(prescale_split(grad_output, rows, output_dim, output_dim, scales, gp, s), "prescale");
  TS_TRY(launch_split_planes(x, rows, input_dim, input_dim, xp, s), "split");
  TS_TRY(accumulate_planes(gp, xp, rows, input_dim, output_dim, accumulators, st, s), "weight-gradient accumulation");
  CountInc inc{};
  inc.n = 1;
  inc.idx[0] = 0;
  inc.v[0] = rows;
  count_add_kernel<<<1, 32, 0, s>>>(sample_count, inc);
  TS_TRY(cudaGetLastError(), "count");
  return NSRL_OK;
}

// ------------------------------------------------------------ window step --
size_t nsrl_train_arena_len(const nsrl_train_model* m) { return m ? arena_len(m) : 0; }

size_t nsrl_train_workspace_size(const nsrl_train_model* m, size_t windows) {
  bool rms = false;
  if (validate_model(m, &rms) != NSRL_OK || windows == 0) return 0;
  StepLayout o;
  carve_step(m, windows, rms, nullptr, o);
  return o.bytes;
}

nsrl_status nsrl_train_windows(const nsrl_train_model* m, const uint8_t* contexts, const uint8_t* targets,
                               const int16_t* freq_w, size_t W, long long* arena, unsigned long long* counts,
                               unsigned long long* stats, void* workspace, size_t workspace_bytes,
                               nsrl_device_status* st, void* stream) {
  bool rms = false;
  nsrl_status vs = validate_model(m, &rms);
  if (vs != NSRL_OK) return vs;
  if (!contexts || !targets || !arena || !counts || !stats || !st) return fail_shape("null buffer");
  if (W == 0) return NSRL_OK;
  if (m->seq_len > 16384 || W * m->seq_len > (size_t)INT32_MAX) return fail_shape("seq_len <= 16384");
  StepLayout o;
  carve_step(m, W, rms, nullptr, o);
  if (!workspace || workspace_bytes < o.bytes) return fail_shape("workspace too small");
  carve_step(m, W, rms, workspace, o);
  cudaStream_t s = (cudaStream_t)stream;
  const size_t T = o.T, d = o.d, F = o.F, S = o.S, H = o.H, L = o.L;
  const size_t per_layer = 4 * d * d + 3 * F * d + 2 * d;
  long long* acc_head = arena;
  long long* acc_layer0 = arena + 256 * d;
  long long* acc_emb = acc_layer0 + L * per_layer;
  long long* acc_pos = acc_emb + 256 * d;
  const size_t lin_off[7] = {0, d * d, 2 * d * d, 3 * d * d, 4 * d * d, 4 * d * d + F * d, 4 * d * d + 2 * F * d};
  const size_t rms_a_off = 4 * d * d + 3 * F * d, rms_m_off = rms_a_off + d;
  unsigned long long* mlp_sat = stats + 1;
  unsigned long long* attn_sat = stats + 2;
  unsigned long long* res_sat = stats + 3;

  // ---- setup: identity grad-input scales, multiplier check, transposed weights
  const size_t nident = std::max<size_t>(std::max(d, F), 256);
  fill_identity_kernel<<<blocks_for((long long)nident), 256, 0, s>>>(o.ident, (int)nident);
  TS_TRY(cudaMemsetAsync(o.fwd_res, 0, 4 * sizeof(unsigned long long), s), "memset");
  check_mult_one_kernel<<<1, 256, 0, s>>>(m->head.scales, 256, nullptr, st);
  TS_TRY(transpose(m->head.weights, 256, d, o.headT, s), "transpose");
  for (size_t l = 0; l < L; ++l) {
    const nsrl_train_layer& ly = m->layer[l];
    for (int i = 0; i < 7; ++i) {
      const nsrl_linear_params& p = ly.lin[i];
      check_mult_one_kernel<<<blocks_for((long long)p.output_dim), 256, 0, s>>>(p.scales, (int)p.output_dim, nullptr,
                                                                                  st);
      TS_TRY(transpose(p.weights, p.output_dim, p.input_dim, o.lc[l].wt[i], s), "transpose");
    }
  }

  // ---- forward with caches (nsrl-train/src/lib.rs:14911-15026, :15079-15300)
  {
    const long long n = (long long)T * d;
    ProfScope prof("embed_forward", s, 0.0, 4.0 * (double)n);
    embed_forward_kernel<<<blocks_for(n, 148 * 32), 256, 0, s>>>(contexts, (long long)T, (int)S, (int)d,
                                                                  m->embeddings, m->positions, o.xemb);
    TS_TRY(cudaGetLastError(), "embed");
  }
  for (size_t l = 0; l < L; ++l) {
    const nsrl_train_layer& ly = m->layer[l];
    LayerCache& c = o.lc[l];
    if (rms)
      TS_TRY(launch_rms_norm(c.in, T, d, ly.attn_gamma, 1, nullptr, c.an, st, s), "rms");
    else
      TS_TRY(launch_split_planes(c.in, T, d, d, c.an, s), "split");
    // Q|K|V: with the tcgen05 attention, one GEMM writes the row-major q|k|v
    // planes (cached for the backward); at head dim 64 the attention reads V's
    // rows from them, otherwise the GEMM also writes the transposed V planes.
    // The int16 rows only when the backward cannot take the planes.
    const bool tc_attn = o.vt.hi && tma_supported() && attention_tc_supported(S, d, H);
    const bool planes_bwd = tc_attn && attention_kv_tc_supported(S, d, H);
    const bool v_rows = planes_bwd && d / H == 64;
    {
      GemmArgs g{};
      g.a_hi = c.an.hi;
      g.a_lo = c.an.lo;
      g.a_l1 = c.an.l1;
      g.lda = d;
      g.M = T;
      g.K = d;
      g.nseg = 3;
      for (int i = 0; i < 3; ++i)
        g.seg[i] = WeightSeg{ly.lin[i].weights, ly.lin[i].bias, ly.lin[i].scales, d};
      g.epi = !tc_attn ? Epi::I16 : v_rows ? Epi::PLANES : Epi::QKV_VT;
      g.y = planes_bwd ? nullptr : c.qkv;
      g.ldy = 3 * d;
      if (tc_attn) {
        g.yp = c.pqkv;
        if (!v_rows) {
          g.vt = o.vt;
          g.v_rows = planes_bwd;
        }
      }
      g.st = st;
      TS_TRY(launch_gemm(g, s), "qkv");
    }
    bool done = false;
    c.p_planes = false;
    if (tc_attn) {
      // every P entry the backward reads is written: the visited key tiles of
      // each 128-query tile, zeros above the diagonal; as byte planes when the
      // tensor-core backward takes the shape (it reads them in place)
      TS_TRY(cudaMemsetAsync(c.ctx.l1, 0, T * sizeof(unsigned long long), s), "memset");
      const Planes pv = p_cache_planes(c, W * H * S * S, S);
      const cudaError_t e = launch_attention_tc(c.pqkv, o.vt, W, S, d, H, true, c.ctx, o.vt.wscr, st, s,
                                                planes_bwd ? nullptr : c.P, planes_bwd ? &pv : nullptr, nullptr,
                                                v_rows);
      // without the int16 q|k|v rows there is no other path
      if (e != cudaErrorNotSupported || planes_bwd) {
        TS_TRY(e, "attention");
        done = true;
        c.p_planes = planes_bwd;
      }
    }
    if (!done) {  // int16 context in a backward buffer that is free during the forward
      TS_TRY(launch_attention_rows_probs(c.qkv, c.qkv + d, c.qkv + 2 * d, 3 * d, W, S, d, H, o.gctx, c.P, st, s),
             "attention");
      TS_TRY(launch_split_planes(o.gctx, T, d, d, c.ctx, s), "split");
    }
    TS_TRY(fwd_gemm(c.ctx, T, d, &ly.lin[3], Epi::RESID, c.ares, d, c.in, o.fwd_res, st, s), "o");
    if (rms)
      TS_TRY(launch_rms_norm(c.ares, T, d, ly.mlp_gamma, 1, nullptr, c.mn, st, s), "rms");
    else
      TS_TRY(launch_split_planes(c.ares, T, d, d, c.mn, s), "split");
    {
      // up and gate in one GEMM: the cached up and gate values, the gated
      // product as planes with its row L1 (mlp.rs:211-254)
      TS_TRY(cudaMemsetAsync(c.gated.l1, 0, T * sizeof(unsigned long long), s), "memset");
      GemmArgs g{};
      g.a_hi = c.mn.hi;
      g.a_lo = c.mn.lo;
      g.a_l1 = c.mn.l1;
      g.lda = d;
      g.M = T;
      g.K = d;
      g.nseg = 2;
      g.seg[0] = WeightSeg{ly.lin[4].weights, ly.lin[4].bias, ly.lin[4].scales, F};
      g.seg[1] = WeightSeg{ly.lin[5].weights, ly.lin[5].bias, ly.lin[5].scales, F};
      g.epi = Epi::GATED;
      g.y = c.up;
      g.y2 = c.gate;
      g.ldy = F;
      g.yp = c.gated;
      g.st = st;
      TS_TRY(launch_gemm(g, s), "up/gate");
    }
    TS_TRY(fwd_gemm(c.gated, T, F, &ly.lin[6], Epi::RESID, c.out, d, c.ares, o.fwd_res, st, s), "down");
  }

  // ---- byte head on the last position, softmax gradient (lib.rs:17455-17488, :18845-18949)
  const int16_t* last = o.lc[L - 1].out;
  TS_TRY(cudaMemcpy2DAsync(o.feat, d * 2, last + (S - 1) * d, S * d * 2, d * 2, W, cudaMemcpyDeviceToDevice, s),
         "gather");
  TS_TRY(launch_split_planes(o.feat, W, d, d, o.fp, s), "split");
  TS_TRY(fwd_gemm(o.fp, W, d, &m->head, Epi::I16, o.logits, 256, nullptr, nullptr, st, s), "head");
  {
    ProfScope prof("head_softmax_grad", s, 0.0, 4.0 * 256.0 * (double)W);
    head_grad_kernel<<<(unsigned)W, 256, 0, s>>>(o.logits, targets, freq_w, o.hgrad, st);
    TS_TRY(cudaGetLastError(), "head grad");
  }
  TS_TRY(prescale_split(o.hgrad, W, 256, 256, m->head.scales, o.hp, s), "prescale");
  TS_TRY(bwd_gemm(o.hp, W, 256, o.headT, d, o.ident, o.glast, d, nullptr, nullptr, st, s), "head^T");
  TS_TRY(cudaMemsetAsync(o.G, 0, T * d * 2, s), "memset");
  TS_TRY(cudaMemcpy2DAsync(o.G + (S - 1) * d, S * d * 2, o.glast, d * 2, d * 2, W, cudaMemcpyDeviceToDevice, s),
         "scatter");
  TS_TRY(accumulate(o.feat, d, o.hgrad, 256, m->head.scales, W, d, 256, acc_head, st, s), "head grad");

  // ---- backward of every block (lib.rs:15623-16075)
  Planes pbF{o.pb.hi, o.pb.lo, nullptr, F};
  Planes paFn{o.pa.hi, o.pa.lo, nullptr, F};
  Planes padn{o.pa.hi, o.pa.lo, nullptr, d};
  CountInc inc{};
  auto add_count = [&](size_t idx, unsigned long long v) {
    if (inc.n == 64) {  // flush a full batch of increments
      count_add_kernel<<<1, 64, 0, s>>>(counts, inc);
      inc.n = 0;
    }
    inc.idx[inc.n] = (int)idx;
    inc.v[inc.n] = v;
    ++inc.n;
  };
  add_count(0, W);
  for (size_t l = L; l-- > 0;) {
    const nsrl_train_layer& ly = m->layer[l];
    LayerCache& c = o.lc[l];
    long long* acc = acc_layer0 + l * per_layer;
    unsigned long long* cnt = counts + 1 + 9 * l;
    // gated MLP backward input (mlp.rs:256-357)
    TS_TRY(prescale_split(o.G, T, d, d, ly.lin[6].scales, padn, s), "prescale");
    TS_TRY(bwd_gemm(padn, T, d, c.wt[6], F, o.ident, o.gg, F, nullptr, nullptr, st, s), "down^T");
    // down weight gradient (lib.rs:13783-13871) from the prescaled G planes,
    // before the gated backward reuses their buffer
    TS_TRY(accumulate_planes(padn, c.gated, T, F, d, acc + lin_off[6], st, s), "down grad");
    {
      const long long n = (long long)T * F;
      ProfScope prof("gated_backward", s, 0.0, 14.0 * (double)n);
      TS_TRY(launch_pdl(gated_backward_vec_kernel, dim3(blocks_for(n / 8, 148 * 32)), dim3(256), 0, s, o.gg, c.up,
                        c.gate, n / 8, (int)F, ly.lin[4].scales, ly.lin[5].scales, (int16_t*)nullptr,
                        (int16_t*)nullptr, paFn.hi, paFn.lo, pbF.hi, pbF.lo),
             "gated backward");
    }
    TS_TRY(bwd_gemm(paFn, T, F, c.wt[4], d, o.ident, o.gui, d, nullptr, nullptr, st, s), "up^T");
    TS_TRY(bwd_gemm(pbF, T, F, c.wt[5], d, o.ident, o.gmi, d, o.gui, mlp_sat, st, s), "gate^T");
    if (rms) {  // the norm's backward with the residual add fused: gao = sat(G + rms'(gmi))
      TS_TRY(rms_backward(c.ares, T, d, ly.mlp_gamma, o.gmi, 1, o.gmr, acc + rms_m_off, mlp_sat, st, s, o.G, o.gao,
                          res_sat),
             "rms bwd");
      add_count(1 + 9 * l + 8, T);
    } else {
      TS_TRY(add_sat(o.G, o.gmi, T * d, o.gao, res_sat, s), "residual");
    }
    // gated-MLP weight gradients (lib.rs:13783-13871)
    {
      ProfScope prof("nonzero_rows", s, 0.0, 2.0 * (double)T * (double)d);
      nonzero_rows_kernel<<<blocks_for((long long)T * 32, 148 * 8), 256, 0, s>>>(o.G, (long long)T, (int)d, &cnt[4],
                                                                                 &cnt[5], &cnt[6]);
      TS_TRY(cudaGetLastError(), "nonzero rows");
    }
    // up and gate weight gradients from the gated backward's prescaled planes
    TS_TRY(accumulate_planes(paFn, c.mn, T, d, F, acc + lin_off[4], st, s), "up grad");
    TS_TRY(accumulate_planes(pbF, c.mn, T, d, F, acc + lin_off[5], st, s), "gate grad");
    // attention update, accumulate form (lib.rs:15777-16075)
    TS_TRY(prescale_split(o.gao, T, d, d, ly.lin[3].scales, padn, s), "prescale");
    TS_TRY(bwd_gemm(padn, T, d, c.wt[3], d, o.ident, o.gctx, d, nullptr, nullptr, st, s), "o^T");
    TS_TRY(accumulate_planes(padn, c.ctx, T, d, d, acc + lin_off[3], st, s), "o grad");
    GradPlanes gp[3];
    for (int i = 0; i < 3; ++i) gp[i] = GradPlanes{ly.lin[i].scales, o.pg[i].hi, o.pg[i].lo};
    const Planes pv = p_cache_planes(c, W * H * S * S, S);
    TS_TRY(attn_backward(c.p_planes ? nullptr : c.qkv, c.p_planes ? nullptr : c.qkv + d,
                         c.p_planes ? nullptr : c.qkv + 2 * d, 3 * d, c.p_planes ? nullptr : c.P, o.gctx, d, W, S, d,
                         H, o.dL, o.dq, o.dk, o.dv, o.abw, o.abw_bytes, st, s, gp, c.p_planes ? &pv : nullptr,
                         c.p_planes ? &c.pqkv : nullptr),
           "attention backward");
    int16_t* gin[3] = {o.gq, o.gk, o.gv};
    for (int i = 0; i < 3; ++i)
      TS_TRY(bwd_gemm(Planes{o.pg[i].hi, o.pg[i].lo, nullptr, d}, T, d, c.wt[i], d, o.ident, gin[i], d, nullptr,
                      nullptr, st, s),
             "qkv^T");
    {
      const long long n = (long long)T * d;
      ProfScope prof("fanin", s, 0.0, 8.0 * (double)n);
      if (n % 8 == 0)  // carved buffers are 256-byte aligned
        TS_TRY(launch_pdl(fanin3_vec_kernel, dim3(blocks_for(n / 8, 148 * 32)), dim3(256), 0, s, o.gq, o.gk, o.gv,
                          n / 8, o.gni, attn_sat),
               "fanin");
      else
        fanin3_kernel<<<blocks_for(n), 256, 0, s>>>(o.gq, o.gk, o.gv, n, o.gni, attn_sat);
      TS_TRY(cudaGetLastError(), "fanin");
    }
    for (int i = 0; i < 3; ++i)  // from the prescaled dQ, dK, dV planes of the attention backward
      TS_TRY(accumulate_planes(Planes{o.pg[i].hi, o.pg[i].lo, nullptr, d}, c.an, T, d, d, acc + lin_off[i], st, s),
             "qkv grad");
    for (int i = 0; i < 4; ++i) add_count(1 + 9 * l + i, T);
    if (rms) {  // Gn = sat(gao + rms'(gni))
      TS_TRY(rms_backward(c.in, T, d, ly.attn_gamma, o.gni, 1, o.gai, acc + rms_a_off, res_sat, st, s, o.gao, o.Gn,
                          res_sat),
             "rms bwd");
      add_count(1 + 9 * l + 7, T);
    } else {
      TS_TRY(add_sat(o.gao, o.gni, T * d, o.Gn, res_sat, s), "residual");
    }
    std::swap(o.G, o.Gn);
  }
  // embedding gradients (lib.rs:14336-14405)
  {
    const long long n = (long long)T * d;
    ProfScope prof("embed_grad", s, 0.0, 2.0 * (double)n);
    embed_grad_kernel<<<blocks_for(n, 148 * 32), 256, 0, s>>>(contexts, (long long)T, (int)S, (int)d, o.G, acc_emb,
                                                              m->positions ? acc_pos : nullptr);
    TS_TRY(cudaGetLastError(), "embed grad");
  }
  add_count(1 + 9 * L, W);
  count_add_kernel<<<1, 64, 0, s>>>(counts, inc);
  stats_finish_kernel<<<1, 1, 0, s>>>(stats, o.fwd_res, (unsigned long long)W);
  TS_TRY(cudaGetLastError(), "counts");
  return NSRL_OK;
}

}  // extern "C"
