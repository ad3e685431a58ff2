// Integer RMS norm rows (crates/nsrl-core/src/rms_norm.rs:12-89).
//
// One warp per row: sum of squares in u64, mean = floor(sum / d) + eps,
// inverse RMS in Q30 from the 8-bit rsqrt table with the odd-exponent
// 1/sqrt(2) correction (rms_norm.rs:47-66), then y = sat(rhu(x * g * inv, 30)).
// |x * g| <= 2^30 and inv < 2^30, so the i64 product of rms_norm.rs:84 never
// overflows and needs no check.  The output is written as int16 and/or as
// byte planes with the row's L1 norm (the operand format of the tensor-core
// linears).
#include "common.cuh"
#include "internal.h"

namespace nsrl {
namespace {


// sat_i16(rhu(x * g * inv, 30)): |x * g| <= 2^30 and 0 <= inv < 2^30, so the
// product fits i64 with no saturation and rhu is (v + 2^29) >> 30.
__device__ __forceinline__ int16_t rms_scale(int x, int g, long long inv) {
  const long long v = (long long)(x * g) * inv + (1ll << 29);
  return (int16_t)max(-32768ll, min(32767ll, v >> 30));
}

template <bool VEC>
__global__ void rms_norm_kernel(const int16_t* __restrict__ x, long long rows, int d, double rd,
                                const int16_t* __restrict__ g, unsigned long long eps, int16_t* __restrict__ y,
                                int8_t* __restrict__ yh, uint8_t* __restrict__ yl, unsigned long long* __restrict__ yl1,
                                long long ldp, nsrl_device_status* st) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (long long r = (long long)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (long long)gridDim.x * warps) {
    const int16_t* xr = x + r * d;
    unsigned long long ss = 0;
    if (VEC) {
      for (int k8 = lane; k8 < d / 8; k8 += 32) {
        const uint4 v = reinterpret_cast<const uint4*>(xr)[k8];
        const int16_t* e = reinterpret_cast<const int16_t*>(&v);
#pragma unroll
        for (int j = 0; j < 8; j += 2)  // a pair of squares is at most 2^31
          ss += (unsigned long long)((unsigned)((int)e[j] * (int)e[j]) + (unsigned)((int)e[j + 1] * (int)e[j + 1]));
      }
    } else {
      for (int k = lane; k < d; k += 32) ss += (unsigned long long)((int)xr[k] * (int)xr[k]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const unsigned long long mean = div_exact(ss, (unsigned)d, rd);
    const unsigned long long v = mean + eps;
    long long inv = 0;
    if (v < mean || v == 0) {  // u64 overflow of mean + eps, or rsqrt(0): the reference returns None
      if (lane == 0) nsrl_flag(st, NSRL_FLAG_RMS_ZERO);
    } else {
      inv = rsqrt_q30(v);
    }
    unsigned l1 = 0;  // per lane: at most d / 32 * 32768
    if (VEC) {
      for (int k8 = lane; k8 < d / 8; k8 += 32) {
        const uint4 xv = reinterpret_cast<const uint4*>(xr)[k8];
        const uint4 gv = reinterpret_cast<const uint4*>(g)[k8];
        const int16_t* xe = reinterpret_cast<const int16_t*>(&xv);
        const int16_t* ge = reinterpret_cast<const int16_t*>(&gv);
        uint32_t pk[4];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          const int o0 = rms_scale(xe[j], ge[j], inv), o1 = rms_scale(xe[j + 1], ge[j + 1], inv);
          if (yl1) l1 += (unsigned)(abs(o0) + abs(o1));
          pk[j / 2] = (uint32_t)(o0 & 0xFFFF) | ((uint32_t)o1 << 16);
        }
        if (y) reinterpret_cast<uint4*>(y + r * d)[k8] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        if (yh) {
          reinterpret_cast<uint2*>(yh + r * ldp)[k8] =
              make_uint2(__byte_perm(pk[0], pk[1], 0x7531), __byte_perm(pk[2], pk[3], 0x7531));
          reinterpret_cast<uint2*>(yl + r * ldp)[k8] =
              make_uint2(__byte_perm(pk[0], pk[1], 0x6420), __byte_perm(pk[2], pk[3], 0x6420));
        }
      }
    } else {
      for (int k = lane; k < d; k += 32) {
        const int o = rms_scale(xr[k], g[k], inv);
        l1 += (unsigned)abs(o);
        if (y) y[r * d + k] = (int16_t)o;
        if (yh) {
          yh[r * ldp + k] = (int8_t)(o >> 8);
          yl[r * ldp + k] = (uint8_t)(o & 255);
        }
      }
    }
    if (yl1) {
      unsigned long long l1w = l1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) l1w += __shfl_xor_sync(0xffffffffu, l1w, o);
      if (lane == 0) yl1[r] = l1w;
    }
  }
}

// Rows of d = 256 * VPL (VPL a power of two, so floor(ss / d) is a shift):
// each warp normalises RPW rows at once with every row held in registers
// (lane l owns 16-byte vectors l, l + 32, ...), so the loads of RPW rows are in
// flight together and each row is read from memory once.
template <int VPL, int RPW>
__global__ void __launch_bounds__(256, VPL >= 4 ? 2 : 3) rms_norm_reg_kernel(
    const int16_t* __restrict__ x, long long rows, const int16_t* __restrict__ g, unsigned long long eps,
    int16_t* __restrict__ y, int8_t* __restrict__ yh, uint8_t* __restrict__ yl, unsigned long long* __restrict__ yl1,
    long long ldp, nsrl_device_status* st) {
  constexpr int D = 256 * VPL;
  constexpr int LOG2D = VPL == 1 ? 8 : (VPL == 2 ? 9 : 10);
  griddep_wait();  // launched as a dependent: the previous kernel's rows (and gamma) are visible from here
  griddep_launch();
  const int lane = threadIdx.x & 31;
  const long long warp0 = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  int gs[VPL][8];  // this lane's gamma values, sign-extended once
#pragma unroll
  for (int v = 0; v < VPL; ++v) {
    const uint4 g4 = reinterpret_cast<const uint4*>(g)[v * 32 + lane];
    const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      gs[v][2 * k] = (int)(int16_t)(gw[k] & 0xFFFFu);
      gs[v][2 * k + 1] = (int)gw[k] >> 16;
    }
  }
  // rows of the group starting at r0 (a ragged last group re-reads the last row)
  auto load_group = [&](long long r0, uint4(&xv)[RPW][VPL]) {
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
      const long long r = min(r0 + rr, rows - 1);
#pragma unroll
      for (int v = 0; v < VPL; ++v) xv[rr][v] = __ldcs(reinterpret_cast<const uint4*>(x + r * D) + v * 32 + lane);
    }
  };
  uint4 nxt[RPW][VPL];
  if (warp0 * RPW < rows) load_group(warp0 * RPW, nxt);
  for (long long r0 = warp0 * RPW; r0 < rows; r0 += nwarps * RPW) {
    uint4 xv[RPW][VPL];
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr)
#pragma unroll
      for (int v = 0; v < VPL; ++v) xv[rr][v] = nxt[rr][v];
    // the next group's loads are in flight while this group is normalised
    if (r0 + nwarps * RPW < rows) load_group(r0 + nwarps * RPW, nxt);
    unsigned long long ss[RPW];
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
      unsigned long long s = 0;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        const uint32_t w[4] = {xv[rr][v].x, xv[rr][v].y, xv[rr][v].z, xv[rr][v].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // a pair of squares is at most 2^31
          const int lo = (int)(int16_t)(w[k] & 0xFFFFu), hi = (int)w[k] >> 16;
          s += (unsigned long long)((unsigned)(lo * lo) + (unsigned)(hi * hi));
        }
      }
      ss[rr] = s;
    }
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {  // per lane at most 8 VPL squares of at most 2^30
      static_assert(8 * VPL <= 128, "warp_sum_u37 takes partials below 2^37");
      ss[rr] = warp_sum_u37(ss[rr]);
    }
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr) {
      const long long r = r0 + rr;
      const unsigned long long mean = ss[rr] >> LOG2D;
      const unsigned long long vsum = mean + eps;
      int inv = 0;  // < 2^30
      if (vsum < mean || vsum == 0) {  // u64 overflow of mean + eps, or rsqrt(0): the reference returns None
        if (lane == 0 && r < rows) nsrl_flag(st, NSRL_FLAG_RMS_ZERO);
      } else {
        inv = (int)rsqrt_q30(vsum);
      }
      unsigned l1 = 0;
#pragma unroll
      for (int v = 0; v < VPL; ++v) {
        const uint32_t xw[4] = {xv[rr][v].x, xv[rr][v].y, xv[rr][v].z, xv[rr][v].w};
        uint32_t pk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          // sat_i16(rhu(x * g * inv, 30)) with |x * g| <= 2^30, 0 <= inv < 2^30,
          // two values saturated and packed by one instruction; the row L1
          // adds the packed pair's absolute values (|-32768| = 0x8000)
          const int p0 = (int)(int16_t)(xw[k] & 0xFFFFu) * gs[v][2 * k];
          const int p1 = ((int)xw[k] >> 16) * gs[v][2 * k + 1];
          pk[k] = pack_sat16(rhu30_mul(p1, inv), rhu30_mul(p0, inv));
          l1 = __dp2a_lo(__vabs2(pk[k]), 0x0101u, l1);
        }
        if (r < rows) {
          if (y) __stcs(reinterpret_cast<uint4*>(y + r * D) + v * 32 + lane, make_uint4(pk[0], pk[1], pk[2], pk[3]));
          if (yh) {
            reinterpret_cast<uint2*>(yh + r * ldp)[v * 32 + lane] =
                make_uint2(__byte_perm(pk[0], pk[1], 0x7531), __byte_perm(pk[2], pk[3], 0x7531));
            reinterpret_cast<uint2*>(yl + r * ldp)[v * 32 + lane] =
                make_uint2(__byte_perm(pk[0], pk[1], 0x6420), __byte_perm(pk[2], pk[3], 0x6420));
          }
        }
      }
      if (yl1) {  // per row at most D * 32768 < 2^26
        l1 = __reduce_add_sync(0xffffffffu, l1);
        if (lane == 0 && r < rows) yl1[r] = l1;
      }
    }
  }
}

}  // namespace

cudaError_t launch_rms_norm(const int16_t* x, size_t rows, size_t d, const int16_t* gamma, uint64_t eps,
                            int16_t* y_i16, Planes yp, nsrl_device_status* st, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)std::min<size_t>((rows + 7) / 8, 148 * 16);
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = d % 8 == 0 && al16(x) && al16(gamma) && (!y_i16 || al16(y_i16)) &&
                   (!yp.hi || ((reinterpret_cast<uintptr_t>(yp.hi) | reinterpret_cast<uintptr_t>(yp.lo)) % 8 == 0 &&
                               yp.ld % 8 == 0));
  ProfScope prof("rms_norm", stream, 0.0, 4.0 * rows * d + (yp.l1 ? 8.0 * rows : 0.0));
  if (vec && (d == 256 || d == 512 || d == 1024)) {
    const size_t rpw = d == 256 ? 2 : 1;
    const size_t groups = (rows + rpw - 1) / rpw;
    const unsigned nb = (unsigned)std::min<size_t>((groups + 7) / 8, d == 1024 ? 148 * 2 : 148 * 3);
#define NSRL_RMS_REG(VPL)                                                                                    \
  launch_pdl(rms_norm_reg_kernel<VPL, (VPL == 1 ? 2 : 1)>, dim3(nb), dim3(256), 0, stream, x, (long long)rows, gamma, \
             (unsigned long long)eps, y_i16, yp.hi, yp.lo, yp.l1, (long long)yp.ld, st)
    const cudaError_t e = d == 256 ? NSRL_RMS_REG(1) : d == 512 ? NSRL_RMS_REG(2) : NSRL_RMS_REG(4);
#undef NSRL_RMS_REG
    if (e != cudaSuccess) return e;
  } else if (vec)
    rms_norm_kernel<true><<<blocks, 256, 0, stream>>>(x, (long long)rows, (int)d, 1.0 / (double)d, gamma, eps, y_i16,
                                                      yp.hi, yp.lo, yp.l1, (long long)yp.ld, st);
  else
    rms_norm_kernel<false><<<blocks, 256, 0, stream>>>(x, (long long)rows, (int)d, 1.0 / (double)d, gamma, eps,
                                                       y_i16, yp.hi, yp.lo, yp.l1, (long long)yp.ld, st);
  return cudaGetLastError();
}

}  // namespace nsrl
