// Shared device-side numerics for the PTQ hot path (sm_100a).
//
// Every routine here reproduces, bit for bit, a torch/compressed-tensors
// operation the reference runs on its tensors:
//   * bf16 arithmetic = float32 op then round-to-nearest-even to bf16;
//   * x / s as torch computes it (IEEE float32 quotient, then the tensor's
//     dtype rounding), with a cheap multiply-by-reciprocal path that is exact
//     whenever the result cannot differ (see bf16_quotient / f32_quotient);
//   * float8_e4m3fn RNE casts, the E2M1 thresholds of compressed-tensors'
//     cast_to_fp4, and the E8M0 (MX) scale derivation on bf16 bit patterns.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/llmc_b200.h"

namespace llmc {

// Host-side count of kernel launches issued by this library (llmc_kernel_launches).
void note_launch();

// Records which CUDA runtime/driver call failed, and why, for
// llmc_last_cuda_error (per host thread); returns LLMC_ECUDA.
int cuda_fail(const char* where, int cuda_error);

// ----------------------------------------------------------------- bf16
__device__ __forceinline__ float bf16_to_f(uint16_t b) { return __uint_as_float(((uint32_t)b) << 16); }
__device__ __forceinline__ uint16_t f_to_bf16(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float rbf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// ----------------------------------------------------------------- division
// Quotient of a bf16 tensor by a bf16 (or float32-valued) scale, rounded to bf16
// exactly as torch does it: q = RN_f32(x / s), result RN_bf16(q).
//
// Fast path: t = x * r with r = RN(1/s).  |t - RN(x/s)| < 4 float32 ulps, so
// RN_bf16(t) == RN_bf16(RN(x/s)) unless t's low 16 bits lie within 16 units
// of the bf16 rounding midpoint 0x8000 (the only place a few-ulp error can
// change a bf16 rounding).  Those rare cases, and every case where the fast
// path's error bound does not apply (non-finite t, reciprocal outside the
// normal range), recompute with the IEEE division __fdiv_rn.
__device__ __forceinline__ float bf16_quotient(float x, float s, float r, bool fast) {
  if (fast) {
    float t = x * r;
    uint32_t b = __float_as_uint(t);
    uint32_t near_mid = (b - 0x7FF0u) & 0xFFFFu;  // in [0, 32] <=> low16 in [0x7FF0, 0x8010]
    if (near_mid > 32u && fabsf(t) < 3.0e38f) return rbf(t);
  }
  return rbf(__fdiv_rn(x, s));
}

// x / y correctly rounded from r = RN(1/y) (Markstein's correction: one fma
// residual, one fma step) while the quotient stays in the normal range;
// IEEE division otherwise (zeros, subnormals, huge values).
__device__ __forceinline__ float div_by_recip(float x, float y, float r) {
  const float q0 = __fmul_rn(x, r);
  const float aq = fabsf(q0);
  if (aq > 1.0e-30f && aq < 1.0e30f && fabsf(r) > 1.0e-30f && fabsf(r) < 1.0e30f) {
    const float e = __fmaf_rn(-q0, y, x);
    return __fmaf_rn(e, r, q0);
  }
  return __fdiv_rn(x, y);
}

// Reciprocal and fast-path flag for a scale; the error bound above needs a
// normal, finite reciprocal.
__device__ __forceinline__ float scale_recip(float s, bool* fast) {
  float r = __frcp_rn(s);
  float ar = fabsf(r);
  *fast = (ar > 1.0e-36f) && (ar < 1.0e36f);
  return r;
}

// float32 quotient RN(x / s) for the E2M1 decision (NVFP4 keeps the quotient
// in float32).  The E2M1 thresholds 0.25 .. 5.0 (and 6.0) have zeros in the
// low 21 mantissa bits, so a t more than 16 ulps away from any float with
// that property decides exactly like RN(x/s); otherwise divide exactly.
__device__ __forceinline__ float f32_quotient_for_fp4(float x, float s, float r, bool fast) {
  if (fast) {
    float t = x * r;
    uint32_t m = (__float_as_uint(t) + 16u) & 0x1FFFFFu;  // in [0, 32] <=> within 16 ulps of ...000
    if (m > 32u && fabsf(t) < 3.0e38f) return t;
  }
  return __fdiv_rn(x, s);
}

// ----------------------------------------------------------------- fp8 e4m3
// Inputs are clamped to +-448 first (as compressed-tensors does), so the
// saturating RNE hardware conversion equals torch's float -> e4m3fn cast.
__device__ __forceinline__ uint8_t f_to_e4m3(float x) {
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float e4m3_to_f(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}
__device__ __forceinline__ float round_e4m3(float x) { return e4m3_to_f(f_to_e4m3(x)); }

// ----------------------------------------------------------------- fp4 e2m1
// compressed-tensors cast_to_fp4 thresholds (closed/open ends as the
// reference writes them) returning the E2M1 code: magnitude index 0..7,
// sign bit 8.  sign follows torch.sign(x)*|v|: a negative x that rounds to
// zero gives -0.0 (code 8); x == +-0.0 gives +0.0 (code 0).
__device__ __forceinline__ uint32_t e2m1_code(float x) {
  float a = fabsf(x);
  uint32_t idx = (a <= 0.25f) ? 0u : (a < 0.75f) ? 1u : (a <= 1.25f) ? 2u : (a < 1.75f) ? 3u
               : (a <= 2.5f) ? 4u : (a < 3.5f) ? 5u : (a <= 5.0f) ? 6u : 7u;
  uint32_t neg = (x < 0.0f) ? 8u : 0u;
  return idx | neg;
}

// ----------------------------------------------------------------- quant args
struct QArgs {
  int bits, is_float, symmetric, strategy, scale_dtype, zp_dtype;
  int64_t group, bh, bw;
  __host__ __device__ bool is_mx() const {
    return (bits == 4 || bits == 8) && is_float && group == 32 && scale_dtype == LLMC_SCALE_U8;
  }
  __host__ __device__ float qmin() const {
    if (!is_float) return -(float)(1 << (bits - 1));
    return bits == 8 ? -448.0f : -6.0f;
  }
  __host__ __device__ float qmax() const {
    if (!is_float) return (float)((1 << (bits - 1)) - 1);
    return bits == 8 ? 448.0f : 6.0f;
  }
};

__host__ __device__ inline QArgs to_qargs(const LlmcQuantArgs& a) {
  QArgs q;
  q.bits = a.num_bits; q.is_float = a.type; q.symmetric = a.symmetric; q.strategy = a.strategy;
  q.scale_dtype = a.scale_dtype; q.zp_dtype = a.zp_dtype;
  q.group = a.group_size; q.bh = a.block_rows; q.bw = a.block_cols;
  return q;
}

// Power-of-two exponent scale of the MX formats (compressed-tensors
// generate_mx_scales + round_to_power_2 on the bf16 bit pattern, then the
// uint8 scale-dtype rounding): returns the E8M0 byte.
__device__ __forceinline__ uint32_t mx_e8m0_from_absmax(float mvp_bf16, int bits) {
  uint32_t b16 = (uint32_t)f_to_bf16(mvp_bf16);
  uint32_t p = (b16 + 32u) & 0xFF80u;        // sign+exponent after rounding up half an fp4 ulp
  uint32_t expf = (p >> 7) & 0xFFu;
  int offset = (bits == 4) ? 2 : 8;
  float v;
  if ((p & 0x7FFFu) == 0) v = -INFINITY;     // log2(0)
  else if (expf == 0xFFu) v = INFINITY;      // log2(inf)
  else v = (float)(127 + ((int)expf - 127) - offset);
  v = fminf(fmaxf(v, 0.0f), 255.0f);
  return (uint32_t)v;
}
// 2^(e - 127) as torch computes it, rounded to bf16 (exact for these values).
__device__ __forceinline__ float e8m0_to_f(uint32_t e) {
  int k = (int)e - 127;
  if (k >= 128) return INFINITY;
  if (k >= -126) return __uint_as_float((uint32_t)(k + 127) << 23);
  return __uint_as_float(1u << (k + 149));    // subnormal (k = -127)
}

// Scale/zero-point of one group from its min/max: compressed-tensors
// calculate_qparams with the reference's dtype semantics.  The statistics
// are bf16 (the observed weight's dtype; every step rounds to bf16) unless
// f32stats (a float32 observed tensor: every step stays float32).  has_gs: a
// float32 global scale multiplies the scale (the product is float32).
// Returns the scale as a float value on the grid of the stored scale dtype;
// *zp_out gets the zero point (already rounded to its integer dtype).
__device__ __forceinline__ float group_qparams(float mn, float mx, const QArgs& a, bool has_gs, float gs,
                                               float* zp_out, bool f32stats = false) {
  mn = fminf(mn, 0.0f);
  mx = fmaxf(mx, 0.0f);
  float qmin = a.qmin(), qmax = a.qmax();
  float br = qmax - qmin;
  float scale, zp = 0.0f;
  bool f32dtype = f32stats;
  auto R = [f32stats](float v) { return f32stats ? v : rbf(v); };
  if (a.symmetric) {
    float mvp = fmaxf(fabsf(mn), fabsf(mx));
    if (a.is_mx()) {
      uint32_t e = mx_e8m0_from_absmax(mvp, a.bits);
      scale = (float)e;  // the bf16 exponent value, converted below
    } else {
      const float half = br * 0.5f;  // the reciprocal depends on the args only: computed once per kernel
      scale = R(div_by_recip(mvp, half, __frcp_rn(half)));
    }
  } else {
    scale = R(div_by_recip(R(mx - mn), br, __frcp_rn(br)));
    zp = R(qmin - R(__fdiv_rn(mn, scale)));
    if (!isnan(zp)) zp = fminf(fmaxf(zp, qmin), qmax);
  }
  if (has_gs) { scale = gs * scale; f32dtype = true; }
  if (a.is_mx()) {
    scale = e8m0_to_f((uint32_t)scale);
  } else if (a.scale_dtype == LLMC_SCALE_FP8) {
    scale = round_e4m3(fminf(fmaxf(scale, -448.0f), 448.0f));
  } else if (a.scale_dtype == LLMC_SCALE_U8) {
    scale = isnan(scale) ? 0.0f : rintf(fminf(fmaxf(scale, 0.0f), 255.0f));
  } else if (a.scale_dtype == LLMC_SCALE_F32) {
    f32dtype = true;
  }
  float eps = (a.scale_dtype == LLMC_SCALE_FP8) ? 0.125f
            : (a.scale_dtype == LLMC_SCALE_U8) ? 1.0f
            : f32dtype ? 1.1920928955078125e-07f : 0.0078125f;
  if (scale == 0.0f) scale = eps;
  if (a.zp_dtype == LLMC_ZP_INT8) zp = isnan(zp) ? 0.0f : rintf(fminf(fmaxf(zp, -128.0f), 127.0f));
  else if (a.zp_dtype == LLMC_ZP_UINT8) zp = isnan(zp) ? 0.0f : rintf(fminf(fmaxf(zp, 0.0f), 255.0f));
  *zp_out = zp;
  return scale;
}

// NVFP4 global scale from a fused set's absmax (generate_gparam as the
// reference evaluates it: 2688 / a == a.reciprocal() * 2688 in bf16, two
// roundings; NaN/Inf -> 1).
__device__ __forceinline__ float global_scale_from_absmax(float a) {
  a = fmaxf(a, 1.1754943508222875e-38f);  // torch.finfo(bf16).tiny
  float r = rbf(__fdiv_rn(1.0f, a));
  float g = rbf(r * 2688.0f);
  if (!isfinite(g)) g = 1.0f;
  return g;
}

}  // namespace llmc
