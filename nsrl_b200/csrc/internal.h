// Host-side declarations shared by the translation units of libnsrl_b200.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/nsrl_b200.h"

namespace nsrl {

// An activation tensor [rows][ld] stored as two byte planes: hi = x >> 8
// (int8) and lo = x & 255 (uint8), so that x = 256 * hi + lo.  Tensor-core
// kernels consume and produce activations in this form; `l1` (optional,
// [rows] uint64) receives sum_k |x[row][k]| for the i32 prefix bound.
struct Planes {
  int8_t* hi;
  uint8_t* lo;
  unsigned long long* l1;
  size_t ld;
};

// One weight matrix [rows][K] with its bias / scales (device pointers).
struct WeightSeg {
  const int8_t* w;
  const int32_t* bias;
  const nsrl_fixed_scale* scales;
  size_t rows;
};

enum class Epi : int {
  I16 = 0,     // y = requant(acc) as int16
  PLANES = 1,  // y = requant(acc) as byte planes (+ row L1)
  RESID = 2,   // y = skip (+sat) requant(acc) as int16, saturations counted
  GATED = 3,   // y = gated_act(requant(up), requant(gate)) as byte planes (+ row L1)
  QKV_VT = 4,  // Q|K|V projection: q, k as byte planes [T][3d]; v transposed per head
               // into byte planes [B][H][hd][S] (the AV operand of the attention)
};

// Per-head transposed V planes: row (b * H + h) * hd + dim, column = position.
struct VtPlanes {
  int8_t* hi;
  uint8_t* lo;
  int S, H, hd;
  int16_t* wscr;  // weight scratch of the tensor-core attention (may be null)
};

// ---- head-sharded forward (shard.cu) ----
// Ranks r = 0..n-1 own the positions [r s_loc, (r+1) s_loc) of every sequence
// for the token-wise work (norms, linears, MLP) and the heads [r Hr, (r+1) Hr)
// for attention.  Every rank's exchange buffer has the same layout; the
// table holds each rank's regions as mapped in this process (device memory).
constexpr int kMaxShardRanks = 8;
struct ShardTable {
  int8_t* qk_hi[kMaxShardRanks];  // [B*S][2 d_loc]: q | k of the rank's heads, all positions
  uint8_t* qk_lo[kMaxShardRanks];
  int8_t* vt_hi[kMaxShardRanks];  // [B][d_loc][S]: v of the rank's heads, transposed per head
  uint8_t* vt_lo[kMaxShardRanks];
  int8_t* ctx_hi[kMaxShardRanks];  // [B*s_loc][d]: the context of the rank's positions, all heads
  uint8_t* ctx_lo[kMaxShardRanks];
  unsigned long long* ctx_l1[kMaxShardRanks];  // [B*s_loc]
  unsigned long long* signal[kMaxShardRanks];  // [kMaxShardRanks]: epoch last signalled by each rank
  unsigned long long* slots[kMaxShardRanks];   // [kMaxShardRanks][4]: status words posted by each rank
};
// Q|K|V projection of the rank's positions: columns go to the head owner's
// q|k planes and transposed v planes instead of local planes.
struct QkvRoute {
  int nranks = 0;  // 0: local stores
  int rank = 0, S = 0, s_loc = 0, d_loc = 0;
  const ShardTable* tab = nullptr;
};
// Context of the rank's heads: rows go to the position owner's context planes
// at column col0 + h * hd (and its row L1).
struct CtxRoute {
  int nranks = 0;  // 0: local stores
  int s_loc = 0, col0 = 0;
  const ShardTable* tab = nullptr;
};

struct GemmArgs {
  const int8_t* a_hi;
  const uint8_t* a_lo;
  const unsigned long long* a_l1;  // row L1 of A (needed when the i32 prefix bound can fail)
  size_t lda;
  size_t M, K;
  int nseg;  // 1 = plain, 3 = concatenated along N (Q|K|V), 2 = gated (up, gate)
  WeightSeg seg[3];
  Epi epi;
  int16_t* y;
  size_t ldy;
  int16_t* y2 = nullptr;  // GATED with y set: y takes the up values and y2 the gate values (int16, ldy)
  Planes yp;
  const int16_t* skip;
  size_t ldskip;
  unsigned long long* sat_counter;
  VtPlanes vt;
  bool v_rows = false;  // QKV_VT: the v columns also go to yp (row-major q|k|v planes)
  QkvRoute route;       // QKV_VT: the head-sharded destinations (route.nranks > 0)
  // int16 A [M][lda] instead of the planes (Epi::I16 only): the kernel splits
  // it into planes in shared memory, and the i32 prefix check, where needed,
  // takes row L1 from the int16 rows.  cudaErrorInvalidValue when the shape or
  // alignment does not allow it (the caller then splits A itself).
  const int16_t* a16 = nullptr;
  nsrl_device_status* st;
  // Backward-input form (linear.rs:594-640): the sum is an i64 (no prefix
  // rule) requantised by requantize_i64_to_i16; A holds the prescaled grads.
  bool wide = false;
};

// Launches the linear on `stream` (tcgen05 path when the shape allows TMA,
// SIMT otherwise), then the exact i32-prefix check where the bound requires it.
cudaError_t launch_gemm(const GemmArgs& a, cudaStream_t stream);

// x [rows][K] int16 -> planes (+ row L1).
cudaError_t launch_split_planes(const int16_t* x, size_t rows, size_t K, size_t ldx, Planes out,
                                cudaStream_t stream);

// RMS norm rows; writes int16 output and/or planes (+ row L1).
cudaError_t launch_rms_norm(const int16_t* x, size_t rows, size_t d, const int16_t* gamma, uint64_t eps,
                            int16_t* y_i16, Planes y_planes, nsrl_device_status* st, cudaStream_t stream);

// Causal / full self-attention core on projected q|k|v planes [B*S][3d]
// (q at column 0, k at d, v at 2d); writes ctx planes [B*S][d] (+ row L1,
// which must be zeroed by the caller).
cudaError_t launch_attention(const Planes& qkv, size_t B, size_t S, size_t d, size_t H, bool causal, Planes ctx,
                             nsrl_device_status* st, cudaStream_t stream);

// Tensor-core (tcgen05) attention core for head_dim 64 (or 16: the forward
// only): q, k from the q|k|v planes, v from the transposed planes of
// Epi::QKV_VT.  Returns
// cudaErrorNotSupported when the shape is outside what it takes.
// wscr (optional, attention_tc_scratch_bytes): weights of the sum pass, so
// that the last pass does not recompute Q K^T.
// probs (optional): P [B][H][S][S] int16 of every visited key tile; the
// causal tiles past a query tile's last row are not visited (zero them first).
// probs_planes (optional, causal only, ld S): the same entries as byte planes;
// row t is written for keys below the end of its 128-key block, zeros above
// the diagonal, which is the causal plane form the backward reads.
// route (optional): the head-sharded context destinations; d and H are then
// the rank's columns and heads, and qkv holds q | k only (ld >= 2 d).
cudaError_t launch_attention_tc(const Planes& qkv, const VtPlanes& vt, size_t B, size_t S, size_t d, size_t H,
                                bool causal, Planes ctx, int16_t* wscr, nsrl_device_status* st,
                                cudaStream_t stream, int16_t* probs = nullptr,
                                const Planes* probs_planes = nullptr, const CtxRoute* route = nullptr,
                                bool v_rows = false);
size_t attention_tc_wstride(size_t S);
size_t attention_tc_scratch_bytes(size_t B, size_t S, size_t d, size_t H);
// Shape rule of the tensor-core attention (head_dim 64, seq_len % 16 == 0,
// seq_len <= 16384); the workspace reserves the transposed V planes for it.
bool attention_tc_supported(size_t S, size_t d, size_t H);
// The forward alone (no cached P, no head-sharded routing) also takes head_dim 16.
bool attention_tc_forward_supported(size_t S, size_t d, size_t H);

// KV-cache decode attention (int16 operands).
// Caches are [B][Lmax][H*hd] (the reference's row layout) or, head_major,
// [B][H][Lmax][hd] (each head's keys contiguous; head_dim 64 only).
cudaError_t launch_decode_attention(const int16_t* q, const int16_t* kc, const int16_t* vc, const int32_t* lens,
                                    size_t B, size_t H, size_t hd, size_t Lmax, int16_t* ctx,
                                    nsrl_device_status* st, cudaStream_t stream, int len_offset = 0,
                                    bool head_major = false);

// Decode step support: q planes -> int16 q, k/v planes -> row pos[b] of the
// head-major KV caches of sequence b (pos[b] < Lmax, else NSRL_FLAG_BAD_LENGTH).
cudaError_t launch_kv_append(const Planes& qkv, size_t B, size_t d, size_t hd, const int32_t* pos, size_t Lmax,
                             int16_t* q16, int16_t* k_cache, int16_t* v_cache, nsrl_device_status* st,
                             cudaStream_t stream);

// Causal attention on int16 q, k, v rows (row stride ld; sequence b starts at
// row b * S) -> ctx int16 [B*S][d] and probabilities P [B][H][S][S] int16.
cudaError_t launch_attention_rows_probs(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld, size_t B,
                                        size_t S, size_t d, size_t H, int16_t* ctx, int16_t* probs,
                                        nsrl_device_status* st, cudaStream_t stream);

// Weight-gradient accumulation on the tensor cores: acc [N][K] (int64) +=
// G^T X over T rows, from the byte planes of G [T][N] and X [T][K] as their
// producers write them (row strides ldg, ldx bytes, multiples of 16; 16-byte
// aligned bases).  cudaErrorNotSupported when TMA cannot take them.
cudaError_t launch_wgrad_tc(const int8_t* gh, const uint8_t* gl, size_t ldg, const int8_t* xh, const uint8_t* xl,
                            size_t ldx, size_t T, size_t N, size_t K, long long* acc, nsrl_device_status* st,
                            cudaStream_t s);

// Softmax-attention backward on the int8 tensor cores (mma.sync): dQ, dK, dV
// and dL (zeroed, then written) from int16 q, k, v (row stride ld), P and dC.
// cudaErrorNotSupported outside head_dim 16/64, S % 4 == 0, d % 16 == 0,
// S <= 16384, or with a scratch below attention_backward_tc_scratch_bytes.
// Optional second form of an attention gradient: byte planes [B*S][d] of
// rhu(g, sc[col].right_shift) (the backward-input prescale with multiplier 1);
// with them, dq, dk and dv themselves are not written.
struct GradPlanes {
  const nsrl_fixed_scale* sc = nullptr;
  int8_t* hi = nullptr;
  uint8_t* lo = nullptr;
};
size_t attention_backward_tc_scratch_bytes(size_t B, size_t S, size_t d, size_t H);
cudaError_t launch_attention_backward_tc(const int16_t* q, const int16_t* k, const int16_t* v, size_t ld,
                                         const int16_t* P, const int16_t* dC, size_t ldc, size_t B, size_t S, size_t d,
                                         size_t H, int16_t* dl, int16_t* dq, int16_t* dk, int16_t* dv,
                                         void* scratch, size_t scratch_bytes, nsrl_device_status* st,
                                         cudaStream_t s, const GradPlanes* planes = nullptr,
                                         const Planes* p_planes = nullptr, const Planes* qkv_planes = nullptr);

// Key and query sides of the attention backward on the tensor cores
// (head_dim 64): dK = dL^T Q, dV = P^T dC and, with kp, dQ = dL K per
// (sequence, head) from row-major byte planes read in place: l, p =
// [B*H][S][S] with entries above the diagonal zero up to the end of each
// row's 128-column block (as launch_split_causal writes them), qp, cp, kp =
// [B][S][d] (row stride ld).  Outputs int16 [B*S][d] (NULL to skip) and/or
// prescaled planes.
bool attention_kv_tc_supported(size_t S, size_t d, size_t H);
cudaError_t launch_split_causal(const int16_t* M, size_t BH, size_t S, int8_t* hi, uint8_t* lo, cudaStream_t s);
// dL of the softmax-attention backward on the tensor cores (head_dim 64,
// S % 16 == 0): dC and V as row-major planes [B*S][d], P as causal planes
// [B*H][S][S]; dL written as causal planes [B*H][S][S] (zeros above the
// diagonal up to the end of each row's 128-key block).  cudaErrorNotSupported
// for other shapes.
cudaError_t launch_attention_bwd_dl_tc(const Planes& cp, const Planes& vp, const Planes& pp, int8_t* l_hi,
                                       uint8_t* l_lo, size_t B, size_t S, size_t d, size_t H,
                                       nsrl_device_status* st, cudaStream_t s);
cudaError_t launch_attention_kv_tc(const Planes& l, const Planes& p, const Planes& qp, const Planes& cp, size_t B,
                                   size_t S, size_t d, size_t H, int16_t* dk, int16_t* dv, const GradPlanes& gk,
                                   const GradPlanes& gv, nsrl_device_status* st, cudaStream_t s,
                                   const Planes* kp = nullptr, int16_t* dq = nullptr,
                                   const GradPlanes& gq = GradPlanes{});

// Planes -> int16.
cudaError_t launch_join_planes(Planes in, size_t rows, size_t cols, int16_t* y, size_t ldy, cudaStream_t stream);

// While nsrl_profile_enable(1) is in force, brackets the kernel launched in
// its scope with CUDA events on `s` and records the launch with its
// algorithmic integer ops and HBM bytes.
class ProfScope {
 public:
  ProfScope(const char* name, cudaStream_t s, double ops, double bytes);
  ~ProfScope();
  ProfScope(const ProfScope&) = delete;
  ProfScope& operator=(const ProfScope&) = delete;

 private:
  const char* name_;
  cudaStream_t stream_;
  double ops_, bytes_;
  cudaEvent_t ev_;
};

// Generation (generate.cu): context windows [B][S] (last bytes, left-padded
// with ' '), embeddings + positions, the byte head with its softmax on one row
// per sequence, and the device-side choice of the next byte.
cudaError_t launch_gen_windows(const uint8_t* ctx, size_t cap, const int32_t* lens, size_t S, size_t B, uint8_t* win,
                               cudaStream_t s);
cudaError_t launch_embed(const uint8_t* win, size_t rows, size_t S, size_t d, const int16_t* emb,
                         const int16_t* pos, int16_t* x, cudaStream_t s);
cudaError_t launch_embed_token(const uint8_t* ctx, size_t cap, const int32_t* lens, int fixed_pos,
                               const int16_t* emb, size_t d, size_t B, int16_t* x, cudaStream_t s);
cudaError_t launch_head_rows(const int16_t* x, size_t row_stride, size_t row0, size_t B, size_t d,
                             const nsrl_linear_params* head, int32_t* logits, int16_t* probs, nsrl_device_status* st,
                             cudaStream_t s);
cudaError_t launch_select(const int32_t* logits, const int16_t* probs, size_t B, int strategy, int top_k,
                          uint64_t seed, int step, uint8_t* ctx, size_t cap, int32_t* lens, int steps,
                          uint8_t* tokens, int32_t* pick_logit, int16_t* pick_prob, cudaStream_t s);

// Linear attention (linear_attention.cu) on the byte planes of the q|k|v
// projection [rows][3d] -> context planes [rows][d] (+ row L1, zeroed by the
// caller).  Head dims up to 64.
bool linear_attention_supported(size_t d, size_t H);
cudaError_t launch_linear_attention(const Planes& qkv, size_t B, size_t S, size_t d, size_t H, bool causal,
                                    Planes ctx, nsrl_device_status* st, cudaStream_t stream);
// One step of B streams (one q|k|v row each) with carried states [B][H][hd][hd]
// and key sums [B][H][hd] (int64); ttt_shift >= 0 applies the TTT delta with
// that shift and adds each stream's |update| to delta_l1[b].
cudaError_t launch_linear_attention_step(const Planes& qkv, size_t B, size_t d, size_t H, long long* state,
                                         long long* key_sums, int ttt_shift, unsigned long long* delta_l1,
                                         Planes ctx, nsrl_device_status* st, cudaStream_t stream);

void set_error(const char* fmt, ...);
bool tma_supported();

// Byte offsets of one exchange buffer of a head-sharded forward (the same on
// every rank): a 4 KiB header (signal words, the epoch counter, posted status
// slots), then the q|k planes, the transposed v planes, and the context planes
// with their row L1, each 256-byte aligned.  When every rank's positions make
// 16-byte runs (S / n a multiple of 16), n staging slots follow, each with the
// q|k and v regions of one destination rank at the same relative offsets: the
// Q|K|V projection writes the parts of other ranks there, and one copy kernel
// pushes them over NVLink in long contiguous runs.
struct ShardLayout {
  size_t B = 0, S = 0, d = 0, H = 0, n = 0, s_loc = 0, d_loc = 0, h_loc = 0;
  size_t qk_hi = 0, qk_lo = 0, vt_hi = 0, vt_lo = 0, ctx_hi = 0, ctx_lo = 0, ctx_l1 = 0;
  size_t stage = 0, stage_stride = 0;  // slot p's q|k hi plane at stage + p * stage_stride (0: no staging)
  size_t total = 0;
};
constexpr size_t kShardSignalOff = 0;    // u64 [kMaxShardRanks]
constexpr size_t kShardEpochOff = 64;    // u64: this rank's signals so far
constexpr size_t kShardSlotsOff = 256;   // u64 [kMaxShardRanks][4]
constexpr size_t kShardHeaderBytes = 4096;
// false when the shape does not split over n ranks.
bool shard_layout(size_t B, size_t S, size_t d, size_t H, size_t n, ShardLayout* L);

// Signal every rank that this rank's stores so far are complete (epoch + 1).
cudaError_t launch_shard_post(const nsrl_shard_group* g, const nsrl_device_status* post_status, cudaStream_t s);
// Wait (bounded) until every rank has signalled this rank's current epoch;
// with combine, add the status words the ranks posted into *st.
cudaError_t launch_shard_wait(const nsrl_shard_group* g, bool combine, nsrl_device_status* st, cudaStream_t s);
// Signal and wait in one launch (ranks in separate processes only); with post,
// the status words go out with the signal, and with combine the other ranks'
// posted words are added into *st.
cudaError_t launch_shard_barrier(const nsrl_shard_group* g, const nsrl_device_status* post, bool combine,
                                 nsrl_device_status* st, cudaStream_t s);
// Copies this rank's staged q|k and v rows of every other rank into that
// rank's exchange buffer (no-op without staging).
cudaError_t launch_shard_push(const nsrl_shard_group* g, cudaStream_t s);

}  // namespace nsrl

// One rank's view of a head-sharded forward: the shape it is bound to, the
// exchange buffers of all ranks as mapped in this process, and the device
// copy of their route table.
struct nsrl_shard_group {
  int nranks = 0, rank = 0, device = 0;
  nsrl::ShardLayout L;
  unsigned long long timeout_ns = 0;
  uint8_t* base[nsrl::kMaxShardRanks] = {};
  nsrl::ShardTable* tab = nullptr;    // device memory: every rank's regions
  nsrl::ShardTable* stab = nullptr;   // device memory: the same, other ranks' q|k, v in the staging slots (or null)
};
