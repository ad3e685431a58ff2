// C ABI of libnsrl_b200 (include/nsrl_b200.h): host-side validation with the
// reference's shape rules, workspace carving, and the kernel sequence of each
// operation.  No entry point allocates device memory.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include <algorithm>

#include <vector>

#include "common.cuh"
#include "internal.h"

namespace nsrl {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

// Attention core over int16 operands (used when the tensor-core prefill
// kernel does not take the head dim); defined in attention.cu.
cudaError_t launch_attention_rows_i16(const int16_t* qkv, size_t B, size_t S, size_t d, size_t H, bool causal,
                                      int16_t* ctx, nsrl_device_status* st, cudaStream_t stream);

namespace {

constexpr size_t ALIGN = 256;
size_t up(size_t v) { return (v + ALIGN - 1) & ~(ALIGN - 1); }

// Bump allocator over the caller's workspace.
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t count) {
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += up(count * sizeof(T));
    return p;
  }
  Planes planes(size_t rows, size_t ld, bool with_l1) {
    Planes p;
    p.hi = take<int8_t>(rows * ld);
    p.lo = take<uint8_t>(rows * ld);
    p.l1 = with_l1 ? take<unsigned long long>(rows) : nullptr;
    p.ld = ld;
    return p;
  }
};

bool is_power_of_four(size_t v) { return v != 0 && (v & (v - 1)) == 0 && (__builtin_ctzll(v) % 2) == 0; }

// linear.rs:56-78 (LinearI16I8Params::is_valid) with the expected dims.
bool linear_ok(const nsrl_linear_params* p, size_t in, size_t out) {
  return p && p->input_dim == in && p->output_dim == out && in != 0 && out != 0 && p->weights && p->scales;
}

// True when a linear with these inputs may need the exact i32 prefix check
// (linear.rs:144-173), which reads the row L1 norms of its input.
bool needs_l1(size_t K, const nsrl_linear_params* a, const nsrl_linear_params* b = nullptr,
              const nsrl_linear_params* c = nullptr) {
  const bool bias = (a && a->bias) || (b && b->bias) || (c && c->bias);
  return bias || (unsigned long long)K * 127ull * 32767ull > 2147483647ull;
}

WeightSeg seg_of(const nsrl_linear_params* p) { return WeightSeg{p->weights, p->bias, p->scales, p->output_dim}; }

nsrl_status cuda_fail(cudaError_t e, const char* what) {
  set_error("%s: %s", what, cudaGetErrorString(e));
  return NSRL_CUDA_ERROR;
}

nsrl_status shape_fail(const char* what) {
  set_error("invalid shape: %s", what);
  return NSRL_INVALID_SHAPE;
}

#define NSRL_TRY(call, what)                  \
  do {                                        \
    cudaError_t _e = (call);                  \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

bool attention_prefill_native(size_t d, size_t H, size_t S) {
  const size_t hd = d / H;
  return (hd == 64 || hd == 16) && S <= 32768;
}

// Transposed V planes for the tensor-core attention (empty when it does not apply).
VtPlanes carve_vt(Carver& c, size_t B, size_t S, size_t d, size_t H) {
  VtPlanes vt{nullptr, nullptr, (int)S, (int)H, (int)(d / H), nullptr};
  if (attention_tc_forward_supported(S, d, H)) {
    vt.hi = c.take<int8_t>(B * S * d);
    vt.lo = c.take<uint8_t>(B * S * d);
    const size_t ws = attention_tc_scratch_bytes(B, S, d, H);
    if (ws) vt.wscr = c.take<int16_t>(ws / sizeof(int16_t));
  }
  return vt;
}

// ---- attention workspace: xn planes + l1, qkv planes, ctx planes + l1 [, int16 fallback buffers]
size_t attention_ws(size_t B, size_t S, size_t d, size_t H, Carver* c = nullptr) {
  Carver local(nullptr);
  Carver& k = c ? *c : local;
  const size_t T = B * S;
  const size_t start = k.off;
  k.planes(T, d, true);
  k.planes(T, 3 * d, false);
  k.planes(T, d, true);
  if (attention_tc_forward_supported(S, d, H)) {
    k.take<int8_t>(T * d);
    k.take<uint8_t>(T * d);
    const size_t ws = attention_tc_scratch_bytes(B, S, d, H);
    if (ws) k.take<int16_t>(ws / sizeof(int16_t));
  }
  if (!attention_prefill_native(d, H, S)) {
    k.take<int16_t>(T * 3 * d);
    k.take<int16_t>(T * d);
  }
  return k.off - start;
}

size_t mlp_ws(size_t T, size_t d, size_t F, Carver* c = nullptr) {
  Carver local(nullptr);
  Carver& k = c ? *c : local;
  const size_t start = k.off;
  k.planes(T, d, true);
  k.planes(T, F, true);
  return k.off - start;
}

// Attention core: (normalised or raw) input planes -> q|k|v -> ctx -> O linear.
nsrl_status attention_core(const Planes& xin, size_t B, size_t S, size_t d, size_t H, bool causal,
                           const nsrl_linear_params* q, const nsrl_linear_params* k, const nsrl_linear_params* v,
                           const nsrl_linear_params* o, Planes qkv, Planes ctx, VtPlanes vt, int16_t* qkv16,
                           int16_t* ctx16, Epi out_epi, const int16_t* skip, int16_t* out, unsigned long long* sat,
                           nsrl_device_status* st, cudaStream_t stream) {
  const size_t T = B * S;
  const bool tc = vt.hi != nullptr && tma_supported();
  // head dim 64: V stays in the q|k|v planes and the attention reads its rows
  // (an MN-major operand); head dim 16 takes the transposed V planes
  const bool v_rows = tc && d / H == 64;
  GemmArgs g{};
  g.a_hi = xin.hi;
  g.a_lo = xin.lo;
  g.a_l1 = xin.l1;
  g.lda = xin.ld;
  g.M = T;
  g.K = d;
  g.nseg = 3;
  g.seg[0] = seg_of(q);
  g.seg[1] = seg_of(k);
  g.seg[2] = seg_of(v);
  g.epi = tc && !v_rows ? Epi::QKV_VT : Epi::PLANES;
  g.yp = qkv;
  g.vt = vt;
  g.st = st;
  NSRL_TRY(launch_gemm(g, stream), "qkv projection");

  if (!needs_l1(d, o)) ctx.l1 = nullptr;
  if (ctx.l1) NSRL_TRY(cudaMemsetAsync(ctx.l1, 0, T * sizeof(unsigned long long), stream), "memset");
  if (tc) {
    NSRL_TRY(launch_attention_tc(qkv, vt, B, S, d, H, causal, ctx, vt.wscr, st, stream, nullptr, nullptr, nullptr,
                                 v_rows),
             "attention");
  } else if (attention_prefill_native(d, H, S)) {
    NSRL_TRY(launch_attention(qkv, B, S, d, H, causal, ctx, st, stream), "attention");
  } else {
    NSRL_TRY(launch_join_planes(qkv, T, 3 * d, qkv16, 3 * d, stream), "join planes");
    NSRL_TRY(launch_attention_rows_i16(qkv16, B, S, d, H, causal, ctx16, st, stream), "attention rows");
    NSRL_TRY(launch_split_planes(ctx16, T, d, d, ctx, stream), "split planes");
  }

  GemmArgs og{};
  og.a_hi = ctx.hi;
  og.a_lo = ctx.lo;
  og.a_l1 = ctx.l1;
  og.lda = ctx.ld;
  og.M = T;
  og.K = d;
  og.nseg = 1;
  og.seg[0] = seg_of(o);
  og.epi = out_epi;
  og.y = out;
  og.ldy = d;
  og.skip = skip;
  og.ldskip = d;
  og.sat_counter = sat;
  og.st = st;
  NSRL_TRY(launch_gemm(og, stream), "output projection");
  return NSRL_OK;
}

nsrl_status validate_attention(size_t S, size_t d, size_t H, const nsrl_linear_params* q,
                               const nsrl_linear_params* k, const nsrl_linear_params* v,
                               const nsrl_linear_params* o) {
  // attention.rs:1585-1634
  if (S == 0 || d == 0 || H == 0) return shape_fail("seq_len, d_model and heads must be nonzero");
  if (d % H != 0) return shape_fail("d_model must be a multiple of heads");
  if (!is_power_of_four(d / H)) return shape_fail("head_dim must be a power of four");
  if (!linear_ok(q, d, d) || !linear_ok(k, d, d) || !linear_ok(v, d, d) || !linear_ok(o, d, d))
    return shape_fail("q/k/v/o must be d_model x d_model linears");
  if (d > (size_t)INT32_MAX / 3 || S > (size_t)INT32_MAX) return shape_fail("dimension too large");
  return NSRL_OK;
}

nsrl_status validate_mlp(size_t T, size_t d, size_t F, const nsrl_linear_params* upp,
                         const nsrl_linear_params* gatep, const nsrl_linear_params* downp) {
  // mlp.rs:108-122 (GatedMlpI16Params::is_valid)
  if (T == 0 || d == 0 || F == 0) return shape_fail("seq_len, d_model and hidden_dim must be nonzero");
  if (!linear_ok(upp, d, F) || !linear_ok(gatep, d, F) || !linear_ok(downp, F, d))
    return shape_fail("up/gate must be d_model -> hidden, down hidden -> d_model");
  return NSRL_OK;
}

nsrl_status mlp_block(const int16_t* x, size_t T, size_t d, size_t F, const int16_t* gamma, uint64_t eps,
                      const nsrl_linear_params* upp, const nsrl_linear_params* gatep,
                      const nsrl_linear_params* downp, int16_t* y, Carver& c, nsrl_device_status* st,
                      cudaStream_t stream) {
  Planes xn = c.planes(T, d, true);
  Planes gated = c.planes(T, F, true);
  if (!needs_l1(d, upp, gatep)) xn.l1 = nullptr;
  if (!needs_l1(F, downp)) gated.l1 = nullptr;
  // cleared first, so that the norm, up/gate and down kernels follow one
  // another directly (each may start its prologue while the previous drains)
  if (gated.l1) NSRL_TRY(cudaMemsetAsync(gated.l1, 0, T * sizeof(unsigned long long), stream), "memset");
  if (gamma)
    NSRL_TRY(launch_rms_norm(x, T, d, gamma, eps, nullptr, xn, st, stream), "rms norm");
  else  // the mini transformer without RMS norm: the block reads x itself
    NSRL_TRY(launch_split_planes(x, T, d, d, xn, stream), "split");
  GemmArgs g{};
  g.a_hi = xn.hi;
  g.a_lo = xn.lo;
  g.a_l1 = xn.l1;
  g.lda = d;
  g.M = T;
  g.K = d;
  g.nseg = 2;
  g.seg[0] = seg_of(upp);
  g.seg[1] = seg_of(gatep);
  g.epi = Epi::GATED;
  g.yp = gated;
  g.st = st;
  NSRL_TRY(launch_gemm(g, stream), "up/gate projection");
  GemmArgs dg{};
  dg.a_hi = gated.hi;
  dg.a_lo = gated.lo;
  dg.a_l1 = gated.l1;
  dg.lda = F;
  dg.M = T;
  dg.K = F;
  dg.nseg = 1;
  dg.seg[0] = seg_of(downp);
  dg.epi = Epi::RESID;
  dg.y = y;
  dg.ldy = d;
  dg.skip = x;
  dg.ldskip = d;
  dg.sat_counter = &st->mlp_saturations;
  dg.st = st;
  NSRL_TRY(launch_gemm(dg, stream), "down projection");
  return NSRL_OK;
}

nsrl_status attention_block(const int16_t* x, size_t B, size_t S, size_t d, size_t H, bool causal,
                            const int16_t* gamma, uint64_t eps, const nsrl_linear_params* q,
                            const nsrl_linear_params* k, const nsrl_linear_params* v, const nsrl_linear_params* o,
                            int16_t* y, Carver& c, nsrl_device_status* st, cudaStream_t stream) {
  const size_t T = B * S;
  Planes xn = c.planes(T, d, true);
  Planes qkv = c.planes(T, 3 * d, false);
  Planes ctx = c.planes(T, d, true);
  VtPlanes vt = carve_vt(c, B, S, d, H);
  int16_t *qkv16 = nullptr, *ctx16 = nullptr;
  if (!attention_prefill_native(d, H, S)) {
    qkv16 = c.take<int16_t>(T * 3 * d);
    ctx16 = c.take<int16_t>(T * d);
  }
  if (!needs_l1(d, q, k, v)) xn.l1 = nullptr;
  if (gamma)
    NSRL_TRY(launch_rms_norm(x, T, d, gamma, eps, nullptr, xn, st, stream), "rms norm");
  else  // the mini transformer without RMS norm: the block reads x itself
    NSRL_TRY(launch_split_planes(x, T, d, d, xn, stream), "split");
  return attention_core(xn, B, S, d, H, causal, q, k, v, o, qkv, ctx, vt, qkv16, ctx16, Epi::RESID, x, y,
                        &st->attention_saturations, st, stream);
}

// Linear attention core: input planes -> q|k|v planes -> linear attention ->
// context planes -> O linear (epilogue out_epi).
size_t linear_attention_ws(size_t T, size_t d, Carver* c = nullptr) {
  Carver local(nullptr);
  Carver& k = c ? *c : local;
  const size_t start = k.off;
  k.planes(T, d, true);
  k.planes(T, 3 * d, false);
  k.planes(T, d, true);
  return k.off - start;
}

nsrl_status linear_attention_core(const Planes& xin, size_t B, size_t S, size_t d, size_t H, bool causal,
                                  const nsrl_linear_params* q, const nsrl_linear_params* k,
                                  const nsrl_linear_params* v, const nsrl_linear_params* o, Planes qkv, Planes ctx,
                                  Epi out_epi, const int16_t* skip, int16_t* out, unsigned long long* sat,
                                  nsrl_device_status* st, cudaStream_t stream, long long* state = nullptr,
                                  long long* key_sums = nullptr, int ttt_shift = -1,
                                  unsigned long long* delta_l1 = nullptr) {
  const size_t T = B * S;
  GemmArgs g{};
  g.a_hi = xin.hi;
  g.a_lo = xin.lo;
  g.a_l1 = xin.l1;
  g.lda = xin.ld;
  g.M = T;
  g.K = d;
  g.nseg = 3;
  g.seg[0] = seg_of(q);
  g.seg[1] = seg_of(k);
  g.seg[2] = seg_of(v);
  g.epi = Epi::PLANES;
  g.yp = qkv;
  g.st = st;
  NSRL_TRY(launch_gemm(g, stream), "qkv projection");
  if (!needs_l1(d, o)) ctx.l1 = nullptr;
  if (ctx.l1) NSRL_TRY(cudaMemsetAsync(ctx.l1, 0, T * sizeof(unsigned long long), stream), "memset");
  if (state)
    NSRL_TRY(launch_linear_attention_step(qkv, B, d, H, state, key_sums, ttt_shift, delta_l1, ctx, st, stream),
             "linear attention step");
  else
    NSRL_TRY(launch_linear_attention(qkv, B, S, d, H, causal, ctx, st, stream), "linear attention");
  GemmArgs og{};
  og.a_hi = ctx.hi;
  og.a_lo = ctx.lo;
  og.a_l1 = ctx.l1;
  og.lda = ctx.ld;
  og.M = T;
  og.K = d;
  og.nseg = 1;
  og.seg[0] = seg_of(o);
  og.epi = out_epi;
  og.y = out;
  og.ldy = d;
  og.skip = skip;
  og.ldskip = d;
  og.sat_counter = sat;
  og.st = st;
  NSRL_TRY(launch_gemm(og, stream), "output projection");
  return NSRL_OK;
}

// y = x + linear_attention(rms(x) or x): the Linear kind of the mini
// transformer's block (nsrl-train/src/lib.rs:15079-15294).
nsrl_status linear_attention_block(const int16_t* x, size_t B, size_t S, size_t d, size_t H, const int16_t* gamma,
                                   uint64_t eps, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                   const nsrl_linear_params* v, const nsrl_linear_params* o, int16_t* y, Carver& c,
                                   nsrl_device_status* st, cudaStream_t stream) {
  const size_t T = B * S;
  Planes xn = c.planes(T, d, true);
  Planes qkv = c.planes(T, 3 * d, false);
  Planes ctx = c.planes(T, d, true);
  if (!needs_l1(d, q, k, v)) xn.l1 = nullptr;
  if (gamma)
    NSRL_TRY(launch_rms_norm(x, T, d, gamma, eps, nullptr, xn, st, stream), "rms norm");
  else
    NSRL_TRY(launch_split_planes(x, T, d, d, xn, stream), "split");
  return linear_attention_core(xn, B, S, d, H, true, q, k, v, o, qkv, ctx, Epi::RESID, x, y,
                               &st->attention_saturations, st, stream);
}

nsrl_status validate_linear_attention(size_t d, size_t H, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                      const nsrl_linear_params* v, const nsrl_linear_params* o) {
  // attention.rs:1636-1684 (any head_dim; this path takes head_dim <= 64)
  if (d == 0 || H == 0 || d % H != 0) return shape_fail("d_model must be a nonzero multiple of heads");
  if (!linear_attention_supported(d, H)) return shape_fail("linear attention: head_dim <= 64");
  if (!linear_ok(q, d, d) || !linear_ok(k, d, d) || !linear_ok(v, d, d) || !linear_ok(o, d, d))
    return shape_fail("q/k/v/o must be d_model x d_model linears");
  if (d > (size_t)INT32_MAX / 3) return shape_fail("dimension too large");
  return NSRL_OK;
}

}  // namespace
}  // namespace nsrl

using namespace nsrl;

extern "C" {

const char* nsrl_last_error(void) { return g_err; }

nsrl_status nsrl_status_reset(nsrl_device_status* status, void* stream) {
  if (!status) return shape_fail("status is NULL");
  NSRL_TRY(cudaMemsetAsync(status, 0, sizeof(nsrl_device_status), (cudaStream_t)stream), "status reset");
  return NSRL_OK;
}

nsrl_status nsrl_status_fetch(const nsrl_device_status* status, nsrl_device_status* host_out, void* stream) {
  if (!status) return shape_fail("status is NULL");
  nsrl_device_status h;
  NSRL_TRY(cudaMemcpyAsync(&h, status, sizeof(h), cudaMemcpyDeviceToHost, (cudaStream_t)stream), "status fetch");
  NSRL_TRY(cudaStreamSynchronize((cudaStream_t)stream), "status fetch");
  if (host_out) *host_out = h;
  if (h.flags) {
    set_error("core rejected (flags 0x%llx)", h.flags);
    return NSRL_CORE_REJECTED;
  }
  return NSRL_OK;
}

size_t nsrl_linear_workspace_size(size_t rows, size_t input_dim, size_t output_dim) {
  (void)output_dim;
  Carver c(nullptr);
  c.planes(rows, input_dim, true);
  return c.off;
}

nsrl_status nsrl_linear_i16_i8_i16(const int16_t* x, size_t rows, const nsrl_linear_params* params, int16_t* y,
                                   void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                   void* stream) {
  if (!params || params->input_dim == 0 || params->output_dim == 0 || !params->weights || !params->scales)
    return shape_fail("linear params");
  if (!status) return shape_fail("status is NULL");
  if (rows == 0) return NSRL_OK;
  if (!x || !y) return shape_fail("x / y is NULL");
  const size_t K = params->input_dim, N = params->output_dim;
  if (K > (size_t)INT32_MAX || N > (size_t)INT32_MAX || rows > (size_t)INT32_MAX)
    return shape_fail("dimension too large");
  if (workspace_bytes < nsrl_linear_workspace_size(rows, K, N) || !workspace) return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  Carver c(workspace);
  Planes xp = c.planes(rows, K, true);
  GemmArgs g{};
  g.a_l1 = xp.l1;
  g.lda = K;
  g.M = rows;
  g.K = K;
  g.nseg = 1;
  g.seg[0] = seg_of(params);
  g.epi = Epi::I16;
  g.y = y;
  g.ldy = N;
  g.st = status;
  // With at most two 128-column output tiles the tensor-core kernel splits
  // the int16 rows into planes itself (K % 8 == 0, 16-byte aligned rows): it
  // converts each A tile once per output tile, which costs less than a split
  // pass over A only while there are few of them.  Otherwise a split pass first.
  g.a16 = N <= 256 ? x : nullptr;
  cudaError_t e = g.a16 ? launch_gemm(g, s) : cudaErrorInvalidValue;
  if (e == cudaErrorInvalidValue) {
    cudaGetLastError();  // nothing was launched
    g.a16 = nullptr;
    NSRL_TRY(launch_split_planes(x, rows, K, K, xp, s), "split planes");
    g.a_hi = xp.hi;
    g.a_lo = xp.lo;
    e = launch_gemm(g, s);
  }
  NSRL_TRY(e, "linear");
  return NSRL_OK;
}

nsrl_status nsrl_rms_norm_rows(const int16_t* x, size_t rows, size_t dim, const int16_t* gamma, uint64_t eps,
                               int16_t* y, nsrl_device_status* status, void* stream) {
  if (dim == 0) return shape_fail("rms norm dim is zero");  // rms_norm.rs:74-76
  if (!status || !gamma) return shape_fail("status / gamma is NULL");
  if (rows == 0) return NSRL_OK;
  Planes none{nullptr, nullptr, nullptr, 0};
  NSRL_TRY(launch_rms_norm(x, rows, dim, gamma, eps, y, none, status, (cudaStream_t)stream), "rms norm");
  return NSRL_OK;
}

size_t nsrl_attention_workspace_size(size_t batch, size_t seq_len, size_t d_model, size_t heads) {
  if (heads == 0) return 0;
  return attention_ws(batch, seq_len, d_model, heads);
}

nsrl_status nsrl_self_attention(const int16_t* x, size_t batch, size_t seq_len, size_t d_model, size_t heads,
                                int causal, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                const nsrl_linear_params* v, const nsrl_linear_params* o, int16_t* out,
                                void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                void* stream) {
  nsrl_status r = validate_attention(seq_len, d_model, heads, q, k, v, o);
  if (r != NSRL_OK) return r;
  if (!status) return shape_fail("status is NULL");
  if (batch == 0) return NSRL_OK;
  if (!workspace || workspace_bytes < attention_ws(batch, seq_len, d_model, heads))
    return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t T = batch * seq_len;
  Carver c(workspace);
  Planes xp = c.planes(T, d_model, true);
  Planes qkv = c.planes(T, 3 * d_model, false);
  Planes ctx = c.planes(T, d_model, true);
  VtPlanes vt = carve_vt(c, batch, seq_len, d_model, heads);
  int16_t *qkv16 = nullptr, *ctx16 = nullptr;
  if (!attention_prefill_native(d_model, heads, seq_len)) {
    qkv16 = c.take<int16_t>(T * 3 * d_model);
    ctx16 = c.take<int16_t>(T * d_model);
  }
  NSRL_TRY(launch_split_planes(x, T, d_model, d_model, xp, s), "split planes");
  return attention_core(xp, batch, seq_len, d_model, heads, causal != 0, q, k, v, o, qkv, ctx, vt, qkv16, ctx16,
                        Epi::I16, nullptr, out, nullptr, status, s);
}

nsrl_status nsrl_prenorm_attention_residual_block(const int16_t* x, size_t batch, size_t seq_len, size_t d_model,
                                                  size_t heads, int causal, const int16_t* rms_gamma,
                                                  uint64_t rms_eps, const nsrl_linear_params* q,
                                                  const nsrl_linear_params* k, const nsrl_linear_params* v,
                                                  const nsrl_linear_params* o, int16_t* y, void* workspace,
                                                  size_t workspace_bytes, nsrl_device_status* status,
                                                  void* stream) {
  nsrl_status r = validate_attention(seq_len, d_model, heads, q, k, v, o);
  if (r != NSRL_OK) return r;
  if (!status || !rms_gamma) return shape_fail("status / gamma is NULL");
  if (batch == 0) return NSRL_OK;
  if (!workspace || workspace_bytes < attention_ws(batch, seq_len, d_model, heads))
    return shape_fail("workspace too small");
  Carver c(workspace);
  return attention_block(x, batch, seq_len, d_model, heads, causal != 0, rms_gamma, rms_eps, q, k, v, o, y, c,
                         status, (cudaStream_t)stream);
}

size_t nsrl_mlp_workspace_size(size_t rows, size_t d_model, size_t hidden_dim) {
  return mlp_ws(rows, d_model, hidden_dim);
}

nsrl_status nsrl_prenorm_gated_mlp_residual_block(const int16_t* x, size_t rows, size_t d_model,
                                                  size_t hidden_dim, const int16_t* rms_gamma, uint64_t rms_eps,
                                                  const nsrl_linear_params* up, const nsrl_linear_params* gate,
                                                  const nsrl_linear_params* down, int16_t* y, void* workspace,
                                                  size_t workspace_bytes, nsrl_device_status* status,
                                                  void* stream) {
  nsrl_status r = validate_mlp(rows, d_model, hidden_dim, up, gate, down);
  if (r != NSRL_OK) return r;
  if (!status || !rms_gamma) return shape_fail("status / gamma is NULL");
  if (!workspace || workspace_bytes < mlp_ws(rows, d_model, hidden_dim)) return shape_fail("workspace too small");
  Carver c(workspace);
  return mlp_block(x, rows, d_model, hidden_dim, rms_gamma, rms_eps, up, gate, down, y, c, status,
                   (cudaStream_t)stream);
}

size_t nsrl_transformer_block_workspace_size(size_t batch, size_t seq_len, size_t d_model, size_t heads,
                                             size_t hidden_dim) {
  if (heads == 0) return 0;
  const size_t T = batch * seq_len;
  size_t a = attention_ws(batch, seq_len, d_model, heads);
  size_t m = mlp_ws(T, d_model, hidden_dim);
  return up(T * d_model * sizeof(int16_t)) + (a > m ? a : m);
}

nsrl_status nsrl_prenorm_transformer_block(const int16_t* x, size_t batch, size_t seq_len, size_t d_model,
                                           size_t heads, size_t hidden_dim, const int16_t* attn_gamma,
                                           const int16_t* mlp_gamma, uint64_t rms_eps,
                                           const nsrl_linear_params* q, const nsrl_linear_params* k,
                                           const nsrl_linear_params* v, const nsrl_linear_params* o,
                                           const nsrl_linear_params* up_p, const nsrl_linear_params* gate,
                                           const nsrl_linear_params* down, int16_t* y, void* workspace,
                                           size_t workspace_bytes, nsrl_device_status* status, void* stream) {
  nsrl_status r = validate_attention(seq_len, d_model, heads, q, k, v, o);
  if (r != NSRL_OK) return r;
  r = validate_mlp(seq_len, d_model, hidden_dim, up_p, gate, down);
  if (r != NSRL_OK) return r;
  if (!status || !attn_gamma || !mlp_gamma) return shape_fail("status / gamma is NULL");
  if (batch == 0) return NSRL_OK;
  if (x == y) return shape_fail("x and y may not alias");
  if (!workspace ||
      workspace_bytes < nsrl_transformer_block_workspace_size(batch, seq_len, d_model, heads, hidden_dim))
    return shape_fail("workspace too small");
  const size_t T = batch * seq_len;
  cudaStream_t s = (cudaStream_t)stream;
  Carver c(workspace);
  int16_t* h = c.take<int16_t>(T * d_model);
  const size_t mark = c.off;
  r = attention_block(x, batch, seq_len, d_model, heads, true, attn_gamma, rms_eps, q, k, v, o, h, c, status, s);
  if (r != NSRL_OK) return r;
  c.off = mark;  // the MLP block reuses the attention scratch
  return mlp_block(h, T, d_model, hidden_dim, mlp_gamma, rms_eps, up_p, gate, down, y, c, status, s);
}

// ---- transformer block over host buffers: chunked copy / compute overlap ----
namespace {
constexpr int HOST_BUFS = 2;  // device buffers per direction of the host-buffer pipeline

// Step i of the pipeline uses device buffers i % HOST_BUFS and compute
// stream i % HOST_BUFS (with its own block workspace), so that the block of
// one step can overlap the tail of the previous one: a block on a few
// sequences leaves much of the GPU idle at its end (its longest attention
// tiles run alone).
struct HostPipe {
  cudaStream_t h2d = nullptr, d2h = nullptr, comp_s[HOST_BUFS] = {nullptr, nullptr};
  cudaEvent_t in[HOST_BUFS], comp[HOST_BUFS], out[HOST_BUFS], done, fin[HOST_BUFS], h2d_fin;
  bool ok = false;
};

constexpr int kPipeDevices = 64;

// One pipeline (streams and events) per device and host thread, created on
// the first call on that device and kept for the life of the thread, so a
// thread that alternates between GPUs reuses each device's own.
HostPipe* host_pipe() {
  static thread_local HostPipe pipes[kPipeDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kPipeDevices) return nullptr;
  HostPipe& p = pipes[dev];
  if (p.ok) return &p;
  if (cudaStreamCreateWithFlags(&p.h2d, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
  if (cudaStreamCreateWithFlags(&p.d2h, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
  for (int b = 0; b < HOST_BUFS; ++b)
    if (cudaStreamCreateWithFlags(&p.comp_s[b], cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&p.in[b], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&p.comp[b], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&p.out[b], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&p.fin[b], cudaEventDisableTiming) != cudaSuccess)
      return nullptr;
  if (cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&p.h2d_fin, cudaEventDisableTiming) != cudaSuccess)
    return nullptr;
  p.ok = true;
  return &p;
}
}  // namespace

size_t nsrl_transformer_block_host_workspace_size(size_t chunk, size_t seq_len, size_t d_model, size_t heads,
                                                  size_t hidden_dim) {
  if (heads == 0 || chunk == 0) return 0;
  return 2 * HOST_BUFS * up(chunk * seq_len * d_model * sizeof(int16_t)) +
         HOST_BUFS * up(nsrl_transformer_block_workspace_size(chunk, seq_len, d_model, heads, hidden_dim));
}

namespace {
// Sequences per step of the host-buffer pipeline: chunk / 4, chunk / 2, then
// full chunks, and the same ramp backwards at the end.  Only the first step's
// copy in and the last step's copy out are not hidden behind a block, so they
// are made small; the steps in between keep the block's grid full.
std::vector<size_t> host_steps(size_t batch, size_t chunk) {
  std::vector<size_t> ramp, out;
  size_t rest = batch;
  for (size_t c = std::max<size_t>(1, chunk / 4); c < chunk && rest > 2 * c; c *= 2) {
    ramp.push_back(c);
    rest -= 2 * c;
  }
  out = ramp;
  while (rest > 0) {
    const size_t c = std::min(chunk, rest);
    out.push_back(c);
    rest -= c;
  }
  out.insert(out.end(), ramp.rbegin(), ramp.rend());
  return out;
}
}  // namespace

namespace {
// The steps of nsrl_prenorm_transformer_block_host after validation: copies
// in on P.h2d, blocks on the two compute streams, copies out on P.d2h.
nsrl_status host_pipeline(HostPipe& P, cudaStream_t s, const int16_t* x_host, int16_t* y_host, int16_t* const* xd,
                          int16_t* const* yd, void* const* bws, size_t bws_bytes, const std::vector<size_t>& steps,
                          const std::vector<size_t>& first, size_t row, size_t seq_len, size_t d_model, size_t heads,
                          size_t hidden_dim, const int16_t* attn_gamma, const int16_t* mlp_gamma, uint64_t rms_eps,
                          const nsrl_linear_params* q, const nsrl_linear_params* k, const nsrl_linear_params* v,
                          const nsrl_linear_params* o, const nsrl_linear_params* up_p,
                          const nsrl_linear_params* gate, const nsrl_linear_params* down,
                          nsrl_device_status* status) {
  const size_t n = steps.size();
  // the copies may start once the caller's earlier work on `stream` is done
  NSRL_TRY(cudaEventRecord(P.done, s), "event");

  NSRL_TRY(cudaStreamWaitEvent(P.h2d, P.done, 0), "event");
  NSRL_TRY(cudaStreamWaitEvent(P.d2h, P.done, 0), "event");
  for (int b = 0; b < HOST_BUFS; ++b) NSRL_TRY(cudaStreamWaitEvent(P.comp_s[b], P.done, 0), "event");
  auto h2d = [&](size_t i) -> nsrl_status {
    const int b = (int)(i % HOST_BUFS);
    const size_t nb = steps[i];
    if (i >= HOST_BUFS) NSRL_TRY(cudaStreamWaitEvent(P.h2d, P.comp[b], 0), "event");  // x[b] free
    NSRL_TRY(cudaMemcpyAsync(xd[b], x_host + first[i] * row, nb * row * sizeof(int16_t), cudaMemcpyHostToDevice,
                             P.h2d),
             "copy in");
    NSRL_TRY(cudaEventRecord(P.in[b], P.h2d), "event");
    return NSRL_OK;
  };
  // The copies in run up to HOST_BUFS - 1 steps ahead of the blocks.
  nsrl_status r = NSRL_OK;
  for (size_t i = 0; i + 1 < (size_t)HOST_BUFS && i < n; ++i)
    if ((r = h2d(i)) != NSRL_OK) return r;
  for (size_t i = 0; i < n; ++i) {
    const int b = (int)(i % HOST_BUFS);
    const size_t nb = steps[i];
    if (i + HOST_BUFS - 1 < n && (r = h2d(i + HOST_BUFS - 1)) != NSRL_OK) return r;
    cudaStream_t cs = P.comp_s[b];
    NSRL_TRY(cudaStreamWaitEvent(cs, P.in[b], 0), "event");
    if (i >= (size_t)HOST_BUFS) NSRL_TRY(cudaStreamWaitEvent(cs, P.out[b], 0), "event");  // y[b] copied out
    r = nsrl_prenorm_transformer_block(xd[b], nb, seq_len, d_model, heads, hidden_dim, attn_gamma, mlp_gamma, rms_eps,
                                       q, k, v, o, up_p, gate, down, yd[b], bws[b], bws_bytes, status, cs);
    if (r != NSRL_OK) return r;
    NSRL_TRY(cudaEventRecord(P.comp[b], cs), "event");
    NSRL_TRY(cudaStreamWaitEvent(P.d2h, P.comp[b], 0), "event");
    NSRL_TRY(cudaMemcpyAsync(y_host + first[i] * row, yd[b], nb * row * sizeof(int16_t), cudaMemcpyDeviceToHost,
                             P.d2h),
             "copy out");
    NSRL_TRY(cudaEventRecord(P.out[b], P.d2h), "event");
  }
  // the caller joins the copy and compute streams into `stream`: the call is
  // complete there once the last copy out has landed and both compute streams
  // are idle (the next call reuses their workspaces)
  return NSRL_OK;
}
}  // namespace

nsrl_status nsrl_prenorm_transformer_block_host(const int16_t* x_host, size_t batch, size_t chunk, size_t seq_len,
                                                size_t d_model, size_t heads, size_t hidden_dim,
                                                const int16_t* attn_gamma, const int16_t* mlp_gamma, uint64_t rms_eps,
                                                const nsrl_linear_params* q, const nsrl_linear_params* k,
                                                const nsrl_linear_params* v, const nsrl_linear_params* o,
                                                const nsrl_linear_params* up_p, const nsrl_linear_params* gate,
                                                const nsrl_linear_params* down, int16_t* y_host, void* workspace,
                                                size_t workspace_bytes, nsrl_device_status* status, void* stream) {
  if (chunk == 0 || !x_host || !y_host) return shape_fail("chunk must be nonzero, host buffers non-NULL");
  if (batch == 0) return NSRL_OK;
  if (chunk > batch) chunk = batch;
  if (!workspace ||
      workspace_bytes < nsrl_transformer_block_host_workspace_size(chunk, seq_len, d_model, heads, hidden_dim))
    return shape_fail("workspace too small");
  HostPipe* pp = host_pipe();
  if (!pp) return cuda_fail(cudaGetLastError(), "copy streams");
  HostPipe& P = *pp;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t elems = chunk * seq_len * d_model;
  Carver c(workspace);
  int16_t* xd[HOST_BUFS];
  int16_t* yd[HOST_BUFS];
  for (int b = 0; b < HOST_BUFS; ++b) xd[b] = c.take<int16_t>(elems);
  for (int b = 0; b < HOST_BUFS; ++b) yd[b] = c.take<int16_t>(elems);
  const size_t bws_bytes = up(nsrl_transformer_block_workspace_size(chunk, seq_len, d_model, heads, hidden_dim));
  void* bws[HOST_BUFS];
  for (int b = 0; b < HOST_BUFS; ++b) bws[b] = c.take<uint8_t>(bws_bytes);
  const std::vector<size_t> steps = host_steps(batch, chunk);
  const size_t n = steps.size();
  std::vector<size_t> first(n + 1, 0);  // first sequence of each step
  for (size_t i = 0; i < n; ++i) first[i + 1] = first[i] + steps[i];
  const size_t row = seq_len * d_model;
  // Joins every pipeline stream into the caller's stream.  It runs on every
  // exit once work may have been enqueued, failures included, so that the
  // caller never frees the workspace or the host buffers under a copy or a
  // block still in flight (best effort: its own errors are not reported).
  auto join = [&]() {
    if (cudaEventRecord(P.h2d_fin, P.h2d) == cudaSuccess) cudaStreamWaitEvent(s, P.h2d_fin, 0);
    if (cudaEventRecord(P.done, P.d2h) == cudaSuccess) cudaStreamWaitEvent(s, P.done, 0);
    for (int b = 0; b < HOST_BUFS; ++b)
      if (cudaEventRecord(P.fin[b], P.comp_s[b]) == cudaSuccess) cudaStreamWaitEvent(s, P.fin[b], 0);
  };
  const nsrl_status res = host_pipeline(P, s, x_host, y_host, xd, yd, bws, bws_bytes, steps, first, row, seq_len,
                                        d_model, heads, hidden_dim, attn_gamma, mlp_gamma, rms_eps, q, k, v, o, up_p,
                                        gate, down, status);
  join();
  return res;
}

size_t nsrl_decode_block_workspace_size(size_t batch, size_t d_model, size_t heads) {
  (void)heads;
  Carver c(nullptr);
  c.planes(batch, d_model, true);
  c.planes(batch, 3 * d_model, false);
  c.take<int16_t>(batch * d_model);
  c.take<int16_t>(batch * d_model);
  c.planes(batch, d_model, true);
  return c.off;
}

nsrl_status nsrl_prenorm_attention_decode_block(const int16_t* x, size_t batch, size_t d_model, size_t heads,
                                                const int16_t* rms_gamma, uint64_t rms_eps,
                                                const nsrl_linear_params* q, const nsrl_linear_params* k,
                                                const nsrl_linear_params* v, const nsrl_linear_params* o,
                                                int16_t* k_cache, int16_t* v_cache, const int32_t* positions,
                                                size_t max_len, int16_t* y, void* workspace, size_t workspace_bytes,
                                                nsrl_device_status* status, void* stream) {
  nsrl_status r = validate_attention(1, d_model, heads, q, k, v, o);
  if (r != NSRL_OK) return r;
  if (d_model / heads != 64) return shape_fail("the decode block takes head_dim 64");
  if (!status || !rms_gamma || !positions || !k_cache || !v_cache) return shape_fail("NULL argument");
  if (max_len == 0 || max_len > 24576) return shape_fail("max_len must be in 1..24576");
  if (batch == 0) return NSRL_OK;
  if (((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) != 0 || d_model % 8 != 0)
    return shape_fail("caches must be 16-byte aligned and d_model a multiple of 8");
  if (!workspace || workspace_bytes < nsrl_decode_block_workspace_size(batch, d_model, heads))
    return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t d = d_model, hd = d / heads;
  Carver c(workspace);
  Planes xn = c.planes(batch, d, true);
  Planes qkv = c.planes(batch, 3 * d, false);
  int16_t* q16 = c.take<int16_t>(batch * d);
  int16_t* ctx16 = c.take<int16_t>(batch * d);
  Planes ctx = c.planes(batch, d, true);
  if (!needs_l1(d, q, k, v)) xn.l1 = nullptr;
  if (!needs_l1(d, o)) ctx.l1 = nullptr;
  NSRL_TRY(launch_rms_norm(x, batch, d, rms_gamma, rms_eps, nullptr, xn, status, s), "rms norm");
  GemmArgs g{};
  g.a_hi = xn.hi;
  g.a_lo = xn.lo;
  g.a_l1 = xn.l1;
  g.lda = d;
  g.M = batch;
  g.K = d;
  g.nseg = 3;
  g.seg[0] = seg_of(q);
  g.seg[1] = seg_of(k);
  g.seg[2] = seg_of(v);
  g.epi = Epi::PLANES;
  g.yp = qkv;
  g.st = status;
  NSRL_TRY(launch_gemm(g, s), "qkv projection");
  NSRL_TRY(launch_kv_append(qkv, batch, d, hd, positions, max_len, q16, k_cache, v_cache, status, s), "kv append");
  NSRL_TRY(launch_decode_attention(q16, k_cache, v_cache, positions, batch, heads, hd, max_len, ctx16, status, s, 1,
                                   true),
           "decode attention");
  NSRL_TRY(launch_split_planes(ctx16, batch, d, d, ctx, s), "split planes");
  GemmArgs og{};
  og.a_hi = ctx.hi;
  og.a_lo = ctx.lo;
  og.a_l1 = ctx.l1;
  og.lda = d;
  og.M = batch;
  og.K = d;
  og.nseg = 1;
  og.seg[0] = seg_of(o);
  og.epi = Epi::RESID;
  og.y = y;
  og.ldy = d;
  og.skip = x;
  og.ldskip = d;
  og.sat_counter = &status->attention_saturations;
  og.st = status;
  NSRL_TRY(launch_gemm(og, s), "output projection");
  return NSRL_OK;
}

nsrl_status nsrl_attention_decode(const int16_t* q, const int16_t* k_cache, const int16_t* v_cache,
                                  const int32_t* lens, size_t batch, size_t heads, size_t head_dim, size_t max_len,
                                  int16_t* ctx, nsrl_device_status* status, void* stream) {
  // attention.rs:682-708
  if (heads == 0 || head_dim == 0 || max_len == 0) return shape_fail("heads, head_dim and max_len must be nonzero");
  if (!is_power_of_four(head_dim)) return shape_fail("head_dim must be a power of four");
  if (!status || !lens) return shape_fail("status / lens is NULL");
  if (max_len > 50000) return shape_fail("max_len above the shared-memory logit buffer (50000)");
  if (batch == 0) return NSRL_OK;
  const size_t d = heads * head_dim;
  const bool vec = head_dim >= 8 && (reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) |
                                     reinterpret_cast<uintptr_t>(v_cache)) % 16 == 0 && d % 8 == 0;
  if (!vec && head_dim >= 8) return shape_fail("q / cache pointers must be 16-byte aligned");
  NSRL_TRY(launch_decode_attention(q, k_cache, v_cache, lens, batch, heads, head_dim, max_len, ctx, status,
                                   (cudaStream_t)stream),
           "decode attention");
  return NSRL_OK;
}

// ------------------------------------------------------------- generation --
namespace {
// The forward of B windows of the mini transformer (softmax attention): the
// embedding, then per layer the prenorm attention block and the prenorm
// gated-MLP block (the training model's block, nsrl-train/src/lib.rs:
// 15079-15294; RMS norm off when the layer has no gammas), then the byte
// head and its softmax on the last position of every window.
size_t gen_ws(const nsrl_train_model* m, size_t B, Carver* c) {
  Carver local(nullptr);
  Carver& k = c ? *c : local;
  const size_t start = k.off;
  const size_t T = B * m->seq_len;
  k.take<uint8_t>(T);                 // windows
  k.take<int16_t>(T * m->d_model);    // x
  k.take<int16_t>(T * m->d_model);    // h
  k.take<int32_t>(B * 256);           // logits
  k.take<int16_t>(B * 256);           // probabilities
  k.take<int32_t>(B);                 // context lengths
  const size_t aws = m->attention_kind == 1 ? linear_attention_ws(T, m->d_model)
                                             : attention_ws(B, m->seq_len, m->d_model, m->heads);
  k.off += std::max(aws, mlp_ws(T, m->d_model, m->hidden_dim));
  return k.off - start;
}

nsrl_status validate_gen_model(const nsrl_train_model* m) {
  if (!m || !m->layer || m->layers == 0 || !m->embeddings) return shape_fail("model with embeddings and layers");
  const size_t d = m->d_model, S = m->seq_len;
  if (m->attention_kind != 0 && m->attention_kind != 1) return shape_fail("attention_kind: 0 softmax, 1 linear");
  const bool lin = m->attention_kind == 1;
  auto vattn = [&](const nsrl_train_layer& L) {
    return lin ? validate_linear_attention(d, m->heads, &L.lin[0], &L.lin[1], &L.lin[2], &L.lin[3])
               : validate_attention(S, d, m->heads, &L.lin[0], &L.lin[1], &L.lin[2], &L.lin[3]);
  };
  nsrl_status r = vattn(m->layer[0]);
  if (r != NSRL_OK) return r;
  if (d > 4096) return shape_fail("d_model <= 4096 for the byte head");
  if (!linear_ok(&m->head, d, 256)) return shape_fail("head must be [256][d_model]");
  const bool rms = m->layer[0].attn_gamma != nullptr;
  for (size_t l = 0; l < m->layers; ++l) {
    const nsrl_train_layer& L = m->layer[l];
    if ((L.attn_gamma != nullptr) != rms || (L.mlp_gamma != nullptr) != rms)
      return shape_fail("RMS gammas: both or neither, the same in every layer");
    if ((r = vattn(L)) != NSRL_OK) return r;
    if ((r = validate_mlp(S, d, m->hidden_dim, &L.lin[4], &L.lin[5], &L.lin[6])) != NSRL_OK) return r;
  }
  return NSRL_OK;
}

// windows (device [B][S]) -> logits / probabilities [B][256] through the workspace carver.
nsrl_status gen_forward(const nsrl_train_model* m, const uint8_t* win, size_t B, int32_t* logits, int16_t* probs,
                        Carver& c, int16_t* x, int16_t* h, nsrl_device_status* st, cudaStream_t s) {
  const size_t S = m->seq_len, d = m->d_model, T = B * S;
  NSRL_TRY(launch_embed(win, T, S, d, m->embeddings, m->positions, x, s), "embedding");
  const size_t mark = c.off;
  for (size_t l = 0; l < m->layers; ++l) {
    const nsrl_train_layer& L = m->layer[l];
    c.off = mark;
    nsrl_status r = m->attention_kind == 1
                        ? linear_attention_block(x, B, S, d, m->heads, L.attn_gamma, 1, &L.lin[0], &L.lin[1],
                                                 &L.lin[2], &L.lin[3], h, c, st, s)
                        : attention_block(x, B, S, d, m->heads, true, L.attn_gamma, 1, &L.lin[0], &L.lin[1],
                                          &L.lin[2], &L.lin[3], h, c, st, s);
    if (r != NSRL_OK) return r;
    c.off = mark;
    r = mlp_block(h, T, d, m->hidden_dim, L.mlp_gamma, 1, &L.lin[4], &L.lin[5], &L.lin[6], x, c, st, s);
    if (r != NSRL_OK) return r;
  }
  NSRL_TRY(launch_head_rows(x, S * d, (S - 1) * d, B, d, &m->head, logits, probs, st, s), "byte head");
  return NSRL_OK;
}
}  // namespace

size_t nsrl_generate_workspace_size(const nsrl_train_model* model, size_t batch) {
  if (validate_gen_model(model) != NSRL_OK || batch == 0) return 0;
  return gen_ws(model, batch, nullptr);
}

nsrl_status nsrl_mini_transformer_output_rows(const nsrl_train_model* m, const uint8_t* windows, size_t batch,
                                              int32_t* logits_q8, int16_t* probs_q15, void* workspace,
                                              size_t workspace_bytes, nsrl_device_status* status, void* stream) {
  nsrl_status r = validate_gen_model(m);
  if (r != NSRL_OK) return r;
  if (!windows || !logits_q8 || !probs_q15 || !status) return shape_fail("NULL argument");
  if (batch == 0) return NSRL_OK;
  if (!workspace || workspace_bytes < gen_ws(m, batch, nullptr)) return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t T = batch * m->seq_len;
  Carver c(workspace);
  c.take<uint8_t>(T);
  int16_t* x = c.take<int16_t>(T * m->d_model);
  int16_t* h = c.take<int16_t>(T * m->d_model);
  c.take<int32_t>(batch * 256);
  c.take<int16_t>(batch * 256);
  c.take<int32_t>(batch);
  return gen_forward(m, windows, batch, logits_q8, probs_q15, c, x, h, status, s);
}

nsrl_status nsrl_mini_transformer_generate(const nsrl_train_model* m, uint8_t* contexts, size_t capacity,
                                           const int32_t* prompt_lens, size_t batch, size_t steps,
                                           const nsrl_decode_config* decode, uint8_t* tokens, int32_t* pick_logits,
                                           int16_t* pick_probs, void* workspace, size_t workspace_bytes,
                                           nsrl_device_status* status, void* stream) {
  nsrl_status r = validate_gen_model(m);
  if (r != NSRL_OK) return r;
  if (!contexts || !prompt_lens || !decode || !tokens || !status) return shape_fail("NULL argument");
  if (decode->strategy != 0 && decode->strategy != 1) return shape_fail("decode strategy: 0 greedy, 1 sample");
  if (batch == 0 || steps == 0) return NSRL_OK;
  if (steps > (size_t)INT32_MAX || capacity > (size_t)INT32_MAX) return shape_fail("steps / capacity too large");
  for (size_t b = 0; b < batch; ++b)  // lib.rs:12735: an empty prompt is InvalidConfig
    if (prompt_lens[b] <= 0 || (size_t)prompt_lens[b] + steps > capacity)
      return shape_fail("every prompt needs 1..capacity-steps bytes");
  if (!workspace || workspace_bytes < gen_ws(m, batch, nullptr)) return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t T = batch * m->seq_len;
  Carver c(workspace);
  uint8_t* win = c.take<uint8_t>(T);
  int16_t* x = c.take<int16_t>(T * m->d_model);
  int16_t* h = c.take<int16_t>(T * m->d_model);
  int32_t* logits = c.take<int32_t>(batch * 256);
  int16_t* probs = c.take<int16_t>(batch * 256);
  int32_t* lens = c.take<int32_t>(batch);
  // from pageable memory: staged before the call returns
  NSRL_TRY(cudaMemcpyAsync(lens, prompt_lens, batch * sizeof(int32_t), cudaMemcpyHostToDevice, s), "lengths");
  const size_t mark = c.off;
  for (size_t step = 0; step < steps; ++step) {
    c.off = mark;
    NSRL_TRY(launch_gen_windows(contexts, capacity, lens, m->seq_len, batch, win, s), "windows");
    r = gen_forward(m, win, batch, logits, probs, c, x, h, status, s);
    if (r != NSRL_OK) return r;
    NSRL_TRY(launch_select(logits, probs, batch, decode->strategy, (int)decode->top_k, decode->sample_seed, (int)step,
                           contexts, capacity, lens, (int)steps, tokens, pick_logits, pick_probs, s),
             "select");
  }
  return NSRL_OK;
}

// ------------------------------------------------------- linear attention --
size_t nsrl_linear_attention_workspace_size(size_t batch, size_t seq_len, size_t d_model) {
  return linear_attention_ws(batch * seq_len, d_model);
}

nsrl_status nsrl_linear_attention(const int16_t* x, size_t batch, size_t seq_len, size_t d_model, size_t heads,
                                  int causal, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                  const nsrl_linear_params* v, const nsrl_linear_params* o, int16_t* out,
                                  void* workspace, size_t workspace_bytes, nsrl_device_status* status,
                                  void* stream) {
  nsrl_status r = validate_linear_attention(d_model, heads, q, k, v, o);
  if (r != NSRL_OK) return r;
  if (seq_len == 0) return shape_fail("seq_len must be nonzero");
  if (!x || !out || !status) return shape_fail("NULL argument");
  if (batch == 0) return NSRL_OK;
  if (!workspace || workspace_bytes < linear_attention_ws(batch * seq_len, d_model))
    return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t T = batch * seq_len;
  Carver c(workspace);
  Planes xp = c.planes(T, d_model, true);
  Planes qkv = c.planes(T, 3 * d_model, false);
  Planes ctx = c.planes(T, d_model, true);
  if (!needs_l1(d_model, q, k, v)) xp.l1 = nullptr;
  NSRL_TRY(launch_split_planes(x, T, d_model, d_model, xp, s), "split");
  return linear_attention_core(xp, batch, seq_len, d_model, heads, causal != 0, q, k, v, o, qkv, ctx, Epi::I16,
                               nullptr, out, nullptr, status, s);
}

size_t nsrl_linear_attention_step_workspace_size(size_t batch, size_t d_model) {
  return linear_attention_ws(batch, d_model);
}

nsrl_status nsrl_linear_attention_step(const int16_t* x, size_t batch, size_t d_model, size_t heads,
                                       const nsrl_linear_params* q, const nsrl_linear_params* k,
                                       const nsrl_linear_params* v, const nsrl_linear_params* o, long long* state,
                                       long long* key_sums, int ttt_shift, unsigned long long* delta_l1,
                                       int16_t* out, void* workspace, size_t workspace_bytes,
                                       nsrl_device_status* status, void* stream) {
  nsrl_status r = validate_linear_attention(d_model, heads, q, k, v, o);
  if (r != NSRL_OK) return r;
  if (!x || !out || !status || !state || !key_sums) return shape_fail("NULL argument");
  if (ttt_shift > 62) return shape_fail("TTT learning-rate shift <= 62");
  if (ttt_shift >= 0 && !delta_l1) return shape_fail("the TTT step needs delta_l1");
  if (batch == 0) return NSRL_OK;
  if (!workspace || workspace_bytes < linear_attention_ws(batch, d_model)) return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  Carver c(workspace);
  Planes xp = c.planes(batch, d_model, true);
  Planes qkv = c.planes(batch, 3 * d_model, false);
  Planes ctx = c.planes(batch, d_model, true);
  if (!needs_l1(d_model, q, k, v)) xp.l1 = nullptr;
  NSRL_TRY(launch_split_planes(x, batch, d_model, d_model, xp, s), "split");
  return linear_attention_core(xp, batch, 1, d_model, heads, true, q, k, v, o, qkv, ctx, Epi::I16, nullptr, out,
                               nullptr, status, s, state, key_sums, ttt_shift < 0 ? -1 : ttt_shift, delta_l1);
}

// ------------------------------------------------- streaming generation --
namespace {
size_t stream_gen_ws(const nsrl_train_model* m, size_t B, Carver* c) {
  Carver local(nullptr);
  Carver& k = c ? *c : local;
  const size_t start = k.off;
  const size_t d = m->d_model, H = m->heads, hd = d / H;
  k.take<int16_t>(B * d);              // x
  k.take<int16_t>(B * d);              // h
  k.take<int16_t>(B * d);              // y
  k.take<int32_t>(B * 256);            // logits
  k.take<int16_t>(B * 256);            // probabilities
  k.take<int32_t>(B);                  // context lengths
  k.take<long long>(B * H * hd * hd);  // states
  k.take<long long>(B * H * hd);       // key sums
  k.take<unsigned long long>(B);       // TTT delta L1
  k.off += std::max(linear_attention_ws(B, d), mlp_ws(B, d, m->hidden_dim));
  return k.off - start;
}

nsrl_status validate_stream_model(const nsrl_train_model* m) {
  if (!m || !m->layer || m->layers != 1 || !m->embeddings || m->attention_kind != 1)
    return shape_fail("streaming generation: a one-layer linear-attention model");
  const nsrl_train_layer& L = m->layer[0];
  nsrl_status r = validate_linear_attention(m->d_model, m->heads, &L.lin[0], &L.lin[1], &L.lin[2], &L.lin[3]);
  if (r != NSRL_OK) return r;
  if ((r = validate_mlp(1, m->d_model, m->hidden_dim, &L.lin[4], &L.lin[5], &L.lin[6])) != NSRL_OK) return r;
  if (m->d_model > 4096 || !linear_ok(&m->head, m->d_model, 256)) return shape_fail("head must be [256][d_model]");
  return NSRL_OK;
}
}  // namespace

size_t nsrl_generate_streaming_workspace_size(const nsrl_train_model* model, size_t batch) {
  if (validate_stream_model(model) != NSRL_OK || batch == 0) return 0;
  return stream_gen_ws(model, batch, nullptr);
}

nsrl_status nsrl_mini_transformer_generate_streaming(const nsrl_train_model* m, uint8_t* contexts, size_t capacity,
                                                     size_t prompt_len, size_t batch, size_t steps,
                                                     const nsrl_decode_config* decode, int ttt_shift,
                                                     uint8_t* tokens, int32_t* pick_logits, int16_t* pick_probs,
                                                     void* workspace, size_t workspace_bytes,
                                                     nsrl_device_status* status, void* stream) {
  nsrl_status r = validate_stream_model(m);
  if (r != NSRL_OK) return r;
  if (!contexts || !decode || !tokens || !status) return shape_fail("NULL argument");
  if (decode->strategy != 0 && decode->strategy != 1) return shape_fail("decode strategy: 0 greedy, 1 sample");
  if (ttt_shift > 62) return shape_fail("TTT learning-rate shift <= 62");
  if (batch == 0 || steps == 0) return NSRL_OK;
  if (prompt_len == 0 || prompt_len + steps > capacity || capacity > (size_t)INT32_MAX)
    return shape_fail("prompts need 1..capacity-steps bytes");
  if (!workspace || workspace_bytes < stream_gen_ws(m, batch, nullptr)) return shape_fail("workspace too small");
  cudaStream_t s = (cudaStream_t)stream;
  const size_t d = m->d_model, H = m->heads, hd = d / H, F = m->hidden_dim;
  const nsrl_train_layer& L = m->layer[0];
  Carver c(workspace);
  int16_t* x = c.take<int16_t>(batch * d);
  int16_t* h = c.take<int16_t>(batch * d);
  int16_t* y = c.take<int16_t>(batch * d);
  int32_t* logits = c.take<int32_t>(batch * 256);
  int16_t* probs = c.take<int16_t>(batch * 256);
  int32_t* lens = c.take<int32_t>(batch);
  long long* state = c.take<long long>(batch * H * hd * hd);
  long long* ks = c.take<long long>(batch * H * hd);
  unsigned long long* dl1 = c.take<unsigned long long>(batch);
  const size_t mark = c.off;
  NSRL_TRY(cudaMemsetAsync(state, 0, batch * H * hd * hd * sizeof(long long), s), "state");
  NSRL_TRY(cudaMemsetAsync(ks, 0, batch * H * hd * sizeof(long long), s), "state");
  NSRL_TRY(cudaMemsetAsync(dl1, 0, batch * sizeof(unsigned long long), s), "state");
  std::vector<int32_t> hl(batch, (int32_t)prompt_len);
  NSRL_TRY(cudaMemcpyAsync(lens, hl.data(), batch * sizeof(int32_t), cudaMemcpyHostToDevice, s), "lengths");
  // mini_transformer_streaming_linear_nope_step (lib.rs:13035-13150): one token of every stream
  auto step = [&](int fixed_pos) -> nsrl_status {
    c.off = mark;
    NSRL_TRY(launch_embed_token(contexts, capacity, lens, fixed_pos, m->embeddings, d, batch, x, s), "embedding");
    Planes xp = c.planes(batch, d, true);
    Planes qkv = c.planes(batch, 3 * d, false);
    Planes ctx = c.planes(batch, d, true);
    if (!needs_l1(d, &L.lin[0], &L.lin[1], &L.lin[2])) xp.l1 = nullptr;
    NSRL_TRY(launch_split_planes(x, batch, d, d, xp, s), "split");
    nsrl_status rr = linear_attention_core(xp, batch, 1, d, H, true, &L.lin[0], &L.lin[1], &L.lin[2], &L.lin[3], qkv,
                                           ctx, Epi::RESID, x, h, &status->attention_saturations, status, s, state,
                                           ks, ttt_shift < 0 ? -1 : ttt_shift, dl1);
    if (rr != NSRL_OK) return rr;
    c.off = mark;
    rr = mlp_block(h, batch, d, F, nullptr, 1, &L.lin[4], &L.lin[5], &L.lin[6], y, c, status, s);
    if (rr != NSRL_OK) return rr;
    NSRL_TRY(launch_head_rows(y, d, 0, batch, d, &m->head, logits, probs, status, s), "byte head");
    return NSRL_OK;
  };
  for (size_t i = 0; i < prompt_len; ++i)
    if ((r = step((int)i)) != NSRL_OK) return r;
  for (size_t t = 0; t < steps; ++t) {
    NSRL_TRY(launch_select(logits, probs, batch, decode->strategy, (int)decode->top_k, decode->sample_seed, (int)t,
                           contexts, capacity, lens, (int)steps, tokens, pick_logits, pick_probs, s),
             "select");
    if (t + 1 < steps && (r = step(-1)) != NSRL_OK) return r;
  }
  return NSRL_OK;
}

// ---- head-sharded forward: the three phases of one block on one rank ----
namespace {
// Workspace: input planes of the Q|K|V projection, the attention's weight
// scratch, then the attention block's output h and the MLP scratch.
struct ShardWs {
  Planes xn;
  int16_t* wscr;
  int16_t* h;
  size_t mlp_off;
};

ShardWs shard_ws(Carver& c, const ShardLayout& L) {
  ShardWs w;
  const size_t T = L.B * L.s_loc;
  w.xn = c.planes(T, L.d, true);
  const size_t ws = attention_tc_scratch_bytes(L.B, L.S, L.d_loc, L.h_loc);
  w.wscr = c.take<int16_t>(ws / sizeof(int16_t));
  w.h = c.take<int16_t>(T * L.d);
  w.mlp_off = c.off;
  return w;
}

size_t shard_ws_bytes(const ShardLayout& L, size_t F) {
  Carver c(nullptr);
  shard_ws(c, L);
  if (F) mlp_ws(L.B * L.s_loc, L.d, F, &c);
  return c.off;
}

nsrl_status shard_check(const nsrl_shard_group* g, void* ws, size_t bytes, size_t F, nsrl_device_status* st,
                        const char* what) {
  if (!g || !st) return shape_fail("sharded block: NULL group or status");
  if (!ws || bytes < shard_ws_bytes(g->L, F)) {
    set_error("%s: workspace too small", what);
    return NSRL_INVALID_SHAPE;
  }
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != g->device) return shape_fail("sharded block: wrong device");
  return NSRL_OK;
}

Planes own_ctx(const nsrl_shard_group* g, bool l1) {
  uint8_t* b = g->base[g->rank];
  Planes p;
  p.hi = reinterpret_cast<int8_t*>(b + g->L.ctx_hi);
  p.lo = b + g->L.ctx_lo;
  p.l1 = l1 ? reinterpret_cast<unsigned long long*>(b + g->L.ctx_l1) : nullptr;
  p.ld = g->L.d;
  return p;
}
}  // namespace

size_t nsrl_sharded_block_workspace_size(const nsrl_shard_group* group, size_t hidden_dim) {
  return group ? shard_ws_bytes(group->L, hidden_dim) : 0;
}

namespace {
// The phases' work without their signal and wait.
nsrl_status qkv_body(const nsrl_shard_group* g, const int16_t* x, const int16_t* rms_gamma, uint64_t rms_eps,
                     const nsrl_linear_params* q, const nsrl_linear_params* k, const nsrl_linear_params* v,
                     const nsrl_linear_params* o, void* workspace, nsrl_device_status* status, cudaStream_t s) {
  const ShardLayout& L = g->L;
  const size_t T = L.B * L.s_loc;
  Carver c(workspace);
  ShardWs w = shard_ws(c, L);
  if (!needs_l1(L.d, q, k, v)) w.xn.l1 = nullptr;
  if (rms_gamma)
    NSRL_TRY(launch_rms_norm(x, T, L.d, rms_gamma, rms_eps, nullptr, w.xn, status, s), "rms norm");
  else
    NSRL_TRY(launch_split_planes(x, T, L.d, L.d, w.xn, s), "split");
  // The context's row L1 is summed by every rank's attention: zero it before the signal.
  if (needs_l1(L.d, o))
    NSRL_TRY(cudaMemsetAsync(own_ctx(g, true).l1, 0, T * sizeof(unsigned long long), s), "memset");
  GemmArgs ga{};
  ga.a_hi = w.xn.hi;
  ga.a_lo = w.xn.lo;
  ga.a_l1 = w.xn.l1;
  ga.lda = L.d;
  ga.M = T;
  ga.K = L.d;
  ga.nseg = 3;
  ga.seg[0] = seg_of(q);
  ga.seg[1] = seg_of(k);
  ga.seg[2] = seg_of(v);
  ga.epi = Epi::QKV_VT;
  ga.vt = VtPlanes{nullptr, nullptr, (int)L.S, (int)L.h_loc, (int)(L.d / L.H), nullptr};
  ga.route.nranks = g->nranks;
  ga.route.rank = g->rank;
  ga.route.S = (int)L.S;
  ga.route.s_loc = (int)L.s_loc;
  ga.route.d_loc = (int)L.d_loc;
  // other ranks' rows: into this rank's staging slots, then one coalesced push
  // over NVLink (or, without staging, peer stores from the epilogue)
  ga.route.tab = g->stab ? g->stab : g->tab;
  ga.st = status;
  NSRL_TRY(launch_gemm(ga, s), "qkv projection");
  NSRL_TRY(launch_shard_push(g, s), "qkv push");
  return NSRL_OK;
}

nsrl_status attention_body(const nsrl_shard_group* g, const nsrl_linear_params* o, void* workspace,
                           nsrl_device_status* status, cudaStream_t s) {
  const ShardLayout& L = g->L;
  Carver c(workspace);
  ShardWs w = shard_ws(c, L);
  uint8_t* b = g->base[g->rank];
  Planes qk{reinterpret_cast<int8_t*>(b + L.qk_hi), b + L.qk_lo, nullptr, 2 * L.d_loc};
  VtPlanes vt{reinterpret_cast<int8_t*>(b + L.vt_hi), b + L.vt_lo, (int)L.S, (int)L.h_loc, (int)(L.d / L.H), w.wscr};
  Planes ctx{nullptr, nullptr, needs_l1(L.d, o) ? own_ctx(g, true).l1 : nullptr, L.d};
  CtxRoute rt;
  rt.nranks = g->nranks;
  rt.s_loc = (int)L.s_loc;
  rt.col0 = (int)(g->rank * L.d_loc);
  rt.tab = g->tab;
  NSRL_TRY(launch_attention_tc(qk, vt, L.B, L.S, L.d_loc, L.h_loc, true, ctx, w.wscr, status, s, nullptr, nullptr,
                               &rt),
           "attention");
  return NSRL_OK;
}

nsrl_status output_body(const nsrl_shard_group* g, const int16_t* x, const nsrl_linear_params* o,
                        const int16_t* mlp_gamma, uint64_t rms_eps, const nsrl_linear_params* up_p,
                        const nsrl_linear_params* gate, const nsrl_linear_params* down, size_t hidden_dim,
                        int16_t* y, void* workspace, nsrl_device_status* status, cudaStream_t s) {
  const ShardLayout& L = g->L;
  const size_t T = L.B * L.s_loc;
  Carver c(workspace);
  ShardWs w = shard_ws(c, L);
  const Planes ctx = own_ctx(g, needs_l1(L.d, o));
  int16_t* h = up_p ? w.h : y;
  GemmArgs og{};
  og.a_hi = ctx.hi;
  og.a_lo = ctx.lo;
  og.a_l1 = ctx.l1;
  og.lda = L.d;
  og.M = T;
  og.K = L.d;
  og.nseg = 1;
  og.seg[0] = seg_of(o);
  og.epi = Epi::RESID;
  og.y = h;
  og.ldy = L.d;
  og.skip = x;
  og.ldskip = L.d;
  og.sat_counter = &status->attention_saturations;
  og.st = status;
  NSRL_TRY(launch_gemm(og, s), "output projection");
  if (!up_p) return NSRL_OK;
  c.off = w.mlp_off;
  return mlp_block(h, T, L.d, hidden_dim, mlp_gamma, rms_eps, up_p, gate, down, y, c, status, s);
}

nsrl_status check_qkv(const nsrl_shard_group* g, const int16_t* x, const nsrl_linear_params* q,
                      const nsrl_linear_params* k, const nsrl_linear_params* v, const nsrl_linear_params* o) {
  const ShardLayout& L = g->L;
  nsrl_status r = validate_attention(L.S, L.d, L.H, q, k, v, o);
  if (r != NSRL_OK) return r;
  return x ? NSRL_OK : shape_fail("x is NULL");
}

nsrl_status check_output(const nsrl_shard_group* g, const int16_t* x, const nsrl_linear_params* o,
                         const nsrl_linear_params* up_p, const nsrl_linear_params* gate,
                         const nsrl_linear_params* down, size_t hidden_dim, const int16_t* y) {
  const ShardLayout& L = g->L;
  if (!linear_ok(o, L.d, L.d)) return shape_fail("o must be a d_model x d_model linear");
  if (up_p) {
    nsrl_status r = validate_mlp(L.S, L.d, hidden_dim, up_p, gate, down);
    if (r != NSRL_OK) return r;
  }
  if (!x || !y) return shape_fail("x / y is NULL");
  if (x == y) return shape_fail("x and y may not alias");
  return NSRL_OK;
}
}  // namespace

nsrl_status nsrl_sharded_block_qkv(const nsrl_shard_group* g, const int16_t* x, const int16_t* rms_gamma,
                                   uint64_t rms_eps, const nsrl_linear_params* q, const nsrl_linear_params* k,
                                   const nsrl_linear_params* v, const nsrl_linear_params* o, void* workspace,
                                   size_t workspace_bytes, nsrl_device_status* status, void* stream) {
  nsrl_status r = shard_check(g, workspace, workspace_bytes, 0, status, "nsrl_sharded_block_qkv");
  if (r == NSRL_OK) r = check_qkv(g, x, q, k, v, o);
  if (r != NSRL_OK) return r;
  cudaStream_t s = (cudaStream_t)stream;
  if ((r = qkv_body(g, x, rms_gamma, rms_eps, q, k, v, o, workspace, status, s)) != NSRL_OK) return r;
  NSRL_TRY(launch_shard_post(g, nullptr, s), "signal");
  return NSRL_OK;
}

nsrl_status nsrl_sharded_block_attention(const nsrl_shard_group* g, const nsrl_linear_params* o, void* workspace,
                                         size_t workspace_bytes, nsrl_device_status* status, void* stream) {
  nsrl_status r = shard_check(g, workspace, workspace_bytes, 0, status, "nsrl_sharded_block_attention");
  if (r != NSRL_OK) return r;
  if (!linear_ok(o, g->L.d, g->L.d)) return shape_fail("o must be a d_model x d_model linear");
  cudaStream_t s = (cudaStream_t)stream;
  NSRL_TRY(launch_shard_wait(g, false, status, s), "wait");
  if ((r = attention_body(g, o, workspace, status, s)) != NSRL_OK) return r;
  NSRL_TRY(launch_shard_post(g, nullptr, s), "signal");
  return NSRL_OK;
}

nsrl_status nsrl_sharded_block_output(const nsrl_shard_group* g, const int16_t* x, const nsrl_linear_params* o,
                                      const int16_t* mlp_gamma, uint64_t rms_eps, const nsrl_linear_params* up_p,
                                      const nsrl_linear_params* gate, const nsrl_linear_params* down,
                                      size_t hidden_dim, int16_t* y, void* workspace, size_t workspace_bytes,
                                      nsrl_device_status* status, void* stream) {
  nsrl_status r = shard_check(g, workspace, workspace_bytes, up_p ? hidden_dim : 0, status,
                              "nsrl_sharded_block_output");
  if (r == NSRL_OK) r = check_output(g, x, o, up_p, gate, down, hidden_dim, y);
  if (r != NSRL_OK) return r;
  cudaStream_t s = (cudaStream_t)stream;
  NSRL_TRY(launch_shard_wait(g, false, status, s), "wait");
  return output_body(g, x, o, mlp_gamma, rms_eps, up_p, gate, down, hidden_dim, y, workspace, status, s);
}

nsrl_status nsrl_sharded_transformer_block(const nsrl_shard_group* g, const int16_t* x, const int16_t* attn_gamma,
                                           const int16_t* mlp_gamma, uint64_t rms_eps, const nsrl_linear_params* q,
                                           const nsrl_linear_params* k, const nsrl_linear_params* v,
                                           const nsrl_linear_params* o, const nsrl_linear_params* up_p,
                                           const nsrl_linear_params* gate, const nsrl_linear_params* down,
                                           size_t hidden_dim, int16_t* y, void* workspace, size_t workspace_bytes,
                                           nsrl_device_status* status, void* stream) {
  nsrl_status r = shard_check(g, workspace, workspace_bytes, up_p ? hidden_dim : 0, status,
                              "nsrl_sharded_transformer_block");
  if (r == NSRL_OK) r = check_qkv(g, x, q, k, v, o);
  if (r == NSRL_OK) r = check_output(g, x, o, up_p, gate, down, hidden_dim, y);
  if (r != NSRL_OK) return r;
  cudaStream_t s = (cudaStream_t)stream;
  if ((r = qkv_body(g, x, attn_gamma, rms_eps, q, k, v, o, workspace, status, s)) != NSRL_OK) return r;
  NSRL_TRY(launch_shard_barrier(g, nullptr, false, status, s), "barrier");
  if ((r = attention_body(g, o, workspace, status, s)) != NSRL_OK) return r;
  NSRL_TRY(launch_shard_barrier(g, nullptr, false, status, s), "barrier");
  return output_body(g, x, o, mlp_gamma, rms_eps, up_p, gate, down, hidden_dim, y, workspace, status, s);
}

}  // extern "C"
