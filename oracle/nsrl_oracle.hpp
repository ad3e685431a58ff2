// CPU oracle for the NSRL integer transformer hot path.
//
// TEST INFRASTRUCTURE ONLY.  This is a scalar C++ restatement of the
// reference's Rust CPU kernels (crates/nsrl-core, crates/nsrl-train-core,
// crates/nsrl-demo bench preset).  It exists so that the parity tests, the
// smoke check and the CPU-baseline leg of the benchmark have something to
// compare the CUDA path against.  Nothing in the product (nsrl_b200/) links,
// loads or calls it.
//
// Every function names the reference file:line it restates.  Semantics are
// the reference's *release* semantics: `debug_assert!`s are not checks, and
// every `Option::None` / `checked_*` failure becomes `false` / a rejected
// return code here.
#pragma once
#include <cstddef>
#include <cstdint>

namespace orc {

struct FixedScale {  // crates/nsrl-core/src/numeric.rs:1-5
  int32_t multiplier;
  uint8_t right_shift;
  uint8_t pad[3];
};

// linear.rs:6-13 (LinearI16I8Params): weights [output_dim][input_dim] i8,
// optional i32 bias and one FixedScale per output channel.
struct LinearParams {
  const int8_t* weights;
  const int32_t* bias;
  const FixedScale* scales;
  size_t input_dim;
  size_t output_dim;
};

constexpr uint8_t MAX_RIGHT_SHIFT = 62;      // numeric.rs:7
constexpr int LOGIT_FRAC_BITS = 8;           // attention.rs:11
constexpr int32_t MASKED_LOGIT = INT32_MIN;  // attention.rs:12
constexpr int Q15_SHIFT = 15;                // attention.rs:13
constexpr int64_t INV_SQRT_2_Q15 = 23170;    // rms_norm.rs:4
constexpr int RMSNORM_INV_RMS_SHIFT = 30;    // rms_norm.rs:5
constexpr int HARD_SILU_GATE_SHIFT = 2;      // mlp.rs:14
constexpr int32_t HARD_SILU_GATE_BIAS_Q15 = 16384;  // mlp.rs:15

// The three 8-bit tables of crates/nsrl-core/src/rsqrt_lut_8bit.rs, derived
// here from their definitions (round-to-nearest of 32768/sqrt(m/128),
// 32768*2^(-f/256) and 2^31/m, the first two clamped to 32767).
extern int16_t RSQRT_LUT[128];
extern int16_t EXP2_LUT[256];
extern uint32_t RECIP_LUT[128];
void init_luts();

int8_t saturate_i8(int64_t v);
int16_t saturate_i16(int64_t v);
int64_t rhu(int64_t v, uint8_t shift);
int16_t requantize_i32_to_i16(int32_t acc, FixedScale s);

}  // namespace orc
