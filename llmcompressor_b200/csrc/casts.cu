// Observers, qparams, casts and packers of the PTQ hot path (sm_100a).
//
// Two kernel shapes cover every strategy:
//  * k_group_vec   -- GROUP / TENSOR_GROUP with a power-of-two group of 8..256
//                     columns: one thread per 16-byte chunk (8 bf16), a group
//                     is 1..32 adjacent lanes reduced with shuffles; single
//                     pass over HBM (W4A16 g128, NVFP4 g16, MXFP4 g32).
//  * k_paramgroup  -- one CTA per quantization-parameter group (a row for
//                     CHANNEL, a 128x128 tile for BLOCK, the whole tensor for
//                     TENSOR, any odd group): pass 1 reduces min/max, pass 2
//                     re-reads the group (an L2 hit for rows and tiles) and
//                     quantizes.
// Both run in three modes: FUSED (observe + qparams + quantize + pack),
// STATS (min/max only) and GIVEN (quantize + pack with stored qparams).
#include "llmc_common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <cstdio>

#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>

namespace llmc {

static std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

enum Mode { MODE_FUSED = 0, MODE_STATS = 1, MODE_GIVEN = 2 };

struct CastParams {
  const uint16_t* w;
  int64_t rows, cols;
  QArgs a;
  int mode;
  int fmt;
  // GIVEN inputs
  const void* scale_in;
  int scale_in_f32;
  const int8_t* zp_in;
  const float* gs;  // global scale (device scalar) or null
  // outputs
  void* out;          // packed codes
  void* scale_out;    // FUSED: bf16 / fp8 byte / e8m0 byte
  int8_t* zp_out;     // FUSED asymmetric int
  uint16_t* min_out;  // STATS
  uint16_t* max_out;
};

// Per-group quantization state shared by the element routine.
struct ElemQ {
  float s;     // scale the element divides by (effective scale for NVFP4)
  float r;     // RN(1/s)
  bool fast;   // reciprocal path valid
  float zp;    // zero point (float) -- only used when has_zp
  bool has_zp;
  bool f32q;   // quotient stays float32 (float32 scale) instead of bf16
  float qmin, qmax;
};

// Quantized code of one bf16 value as compressed-tensors' quantize() does it.
//   INT formats: signed integer code; FP8: e4m3 byte; FP4: E2M1 nibble code.
template <int FMT>
__device__ __forceinline__ uint32_t quant_code(float x, const ElemQ& e) {
  if (FMT == LLMC_FMT_NVFP4) {
    float q = f32_quotient_for_fp4(x, e.s, e.r, e.fast);
    q = fminf(fmaxf(q, -6.0f), 6.0f);
    return e2m1_code(q);
  }
  float q;
  if (e.f32q) {
    q = __fdiv_rn(x, e.s);
    if (e.has_zp) q = q + e.zp;
  } else {
    q = bf16_quotient(x, e.s, e.r, e.fast);
    if (e.has_zp) q = rbf(q + e.zp);
  }
  q = fminf(fmaxf(q, e.qmin), e.qmax);
  if (FMT == LLMC_FMT_MXFP4) return e2m1_code(q);
  if (FMT == LLMC_FMT_FP8) return (uint32_t)f_to_e4m3(q);
  return (uint32_t)(int32_t)rintf(q);  // INT8 / PACK_INT32: signed code
}

// NVFP4 group scale (group_qparams for symmetric E2M1 with a float32 global
// scale and FP8 scales): rbf(amax / 6) * gs rounded to E4M3 (0 -> 0.125),
// with the division by 6 as a multiplication by RN(1/6) plus correction.
__device__ __forceinline__ float nvfp4_group_scale(float mn, float mx, float gs) {
  const float mvp = fmaxf(fabsf(fminf(mn, 0.0f)), fabsf(fmaxf(mx, 0.0f)));
  float scale = rbf(div_by_recip(mvp, 6.0f, __uint_as_float(0x3E2AAAABu)));  // RN(1/6)
  scale = round_e4m3(fminf(fmaxf(gs * scale, -448.0f), 448.0f));
  return scale == 0.0f ? 0.125f : scale;
}

// Per-group qparams -> ElemQ (+ the stored scale bits) in FUSED mode.
template <int FMT>
__device__ __forceinline__ ElemQ make_elemq_fused(const CastParams& p, float mn, float mx, float* s_store,
                                                   float* zp_store) {
  ElemQ e;
  bool has_gs = (FMT == LLMC_FMT_NVFP4);
  float gs = has_gs ? *p.gs : 0.0f;
  float zp = 0.0f;
  if constexpr (FMT == LLMC_FMT_NVFP4) {
    if (p.a.symmetric && p.a.is_float && p.a.bits == 4 && p.a.scale_dtype == LLMC_SCALE_FP8) {
      const float s = nvfp4_group_scale(mn, mx, gs);
      *s_store = s;
      *zp_store = 0.0f;
      e.s = div_by_recip(s, gs, __frcp_rn(gs));  // the effective scale s / gs
      e.r = scale_recip(e.s, &e.fast);
      e.zp = 0.0f;
      e.has_zp = false;
      e.f32q = false;
      e.qmin = p.a.qmin();
      e.qmax = p.a.qmax();
      return e;
    }
  }
  float s = group_qparams(mn, mx, p.a, has_gs, gs, &zp);
  *s_store = s;
  *zp_store = zp;
  e.s = (FMT == LLMC_FMT_NVFP4) ? __fdiv_rn(s, gs) : s;
  e.r = scale_recip(e.s, &e.fast);
  e.zp = zp;
  e.has_zp = !p.a.symmetric;
  e.f32q = false;
  e.qmin = p.a.qmin();
  e.qmax = p.a.qmax();
  return e;
}

template <int FMT>
__device__ __forceinline__ ElemQ make_elemq_given(const CastParams& p, int64_t gi) {
  ElemQ e;
  float s = p.scale_in_f32 ? ((const float*)p.scale_in)[gi] : bf16_to_f(((const uint16_t*)p.scale_in)[gi]);
  if (FMT == LLMC_FMT_NVFP4) {
    e.s = __fdiv_rn(s, *p.gs);  // scale / global_scale in float32
    e.f32q = true;
  } else {
    e.s = s;
    e.f32q = p.scale_in_f32 != 0;  // bf16 / float32 -> float32 quotient
  }
  e.r = scale_recip(e.s, &e.fast);
  e.has_zp = p.zp_in != nullptr;
  e.zp = e.has_zp ? (float)p.zp_in[gi] : 0.0f;
  e.qmin = p.a.qmin();
  e.qmax = p.a.qmax();
  return e;
}

template <int FMT>
__device__ __forceinline__ void store_scale(const CastParams& p, int64_t gi, float s, float zp) {
  if (FMT == LLMC_FMT_NVFP4) ((uint8_t*)p.scale_out)[gi] = f_to_e4m3(s);
  else if (FMT == LLMC_FMT_MXFP4) {
    // compress_mx_scale: 127 + floor(log2(scale)); scale is 2^(e-127)
    uint32_t b = __float_as_uint(s);
    uint32_t ex = (b >> 23) & 0xFF;
    // normal: floor(log2) = ex - 127; subnormal: the top mantissa bit's weight
    uint32_t e8 = ex ? ex : (uint32_t)((31 - __clz(b & 0x7FFFFF)) - 149 + 127);
    ((uint8_t*)p.scale_out)[gi] = (uint8_t)e8;
  } else {
    ((uint16_t*)p.scale_out)[gi] = f_to_bf16(s);
  }
  if (p.zp_out) p.zp_out[gi] = (int8_t)(int32_t)zp;
}

__device__ __forceinline__ void unpack8(const uint4& v, float* x) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// Store 8 codes starting at element index `elem` (a multiple of 8).
template <int FMT>
__device__ __forceinline__ void store8(const CastParams& p, int64_t elem, const uint32_t* c) {
  if (FMT == LLMC_FMT_PACK_INT32) {
    if (p.a.bits == 4) {
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) word |= ((c[j] + 8u) & 0xFu) << (4 * j);
      __stcs((uint32_t*)p.out + elem / 8, word);
    } else {
      uint2 w2;
      w2.x = ((c[0] + 128u) & 0xFFu) | (((c[1] + 128u) & 0xFFu) << 8) | (((c[2] + 128u) & 0xFFu) << 16) |
             (((c[3] + 128u) & 0xFFu) << 24);
      w2.y = ((c[4] + 128u) & 0xFFu) | (((c[5] + 128u) & 0xFFu) << 8) | (((c[6] + 128u) & 0xFFu) << 16) |
             (((c[7] + 128u) & 0xFFu) << 24);
      __stcs((uint2*)p.out + elem / 8, w2);
    }
  } else if (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) word |= (c[j] & 0xFu) << (4 * j);
    __stcs((uint32_t*)((uint8_t*)p.out + elem / 2), word);
  } else {  // FP8 / INT8 bytes
    uint2 w2;
    w2.x = (c[0] & 0xFFu) | ((c[1] & 0xFFu) << 8) | ((c[2] & 0xFFu) << 16) | ((c[3] & 0xFFu) << 24);
    w2.y = (c[4] & 0xFFu) | ((c[5] & 0xFFu) << 8) | ((c[6] & 0xFFu) << 16) | ((c[7] & 0xFFu) << 24);
    __stcs((uint2*)((uint8_t*)p.out + elem), w2);
  }
}

// ------------------------------------------------------------------------
// k_group_vec: power-of-two groups of 8..256 columns, cols % group == 0.
// ------------------------------------------------------------------------
constexpr int VEC_UNROLL = 4;

template <int FMT, int TPG>
__global__ void __launch_bounds__(256) k_group_vec(CastParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t total = p.rows * p.cols / 8;  // chunks
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t base = warp * 32 * VEC_UNROLL; base < total; base += nwarps * 32 * VEC_UNROLL) {
    uint4 v[VEC_UNROLL];
#pragma unroll
    for (int u = 0; u < VEC_UNROLL; ++u) {
      int64_t ch = base + u * 32 + lane;
      if (ch < total) v[u] = __ldcs((const uint4*)p.w + ch);
      else v[u] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < VEC_UNROLL; ++u) {
      int64_t ch = base + u * 32 + lane;
      bool valid = ch < total;  // a whole group is valid or not (total % TPG == 0)
      float x[8];
      unpack8(v[u], x);
      int64_t gi = ch / TPG;
      ElemQ e;
      float s_store = 0.f, zp_store = 0.f;
      if (p.mode != MODE_GIVEN) {
        float mn = x[0], mx = x[0];
#pragma unroll
        for (int j = 1; j < 8; ++j) { mn = fminf(mn, x[j]); mx = fmaxf(mx, x[j]); }
#pragma unroll
        for (int o = 1; o < TPG; o <<= 1) {
          mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        if (p.mode == MODE_STATS) {
          if (valid && (lane % TPG) == 0) { p.min_out[gi] = f_to_bf16(mn); p.max_out[gi] = f_to_bf16(mx); }
          continue;
        }
        e = make_elemq_fused<FMT>(p, mn, mx, &s_store, &zp_store);
      } else {
        if (!valid) continue;
        e = make_elemq_given<FMT>(p, gi);
      }
      if (!valid) continue;
      uint32_t c[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) c[j] = quant_code<FMT>(x[j], e);
      store8<FMT>(p, ch * 8, c);
      if (p.mode == MODE_FUSED && (lane % TPG) == 0) store_scale<FMT>(p, gi, s_store, zp_store);
    }
  }
}

// ------------------------------------------------------------------------
// k_paramgroup: one CTA per parameter group.
// ------------------------------------------------------------------------
struct Rect { int64_t r0, r1, c0, c1; };

__device__ __forceinline__ Rect group_rect(const CastParams& p, int64_t gi) {
  Rect R;
  const QArgs& a = p.a;
  if (a.strategy == LLMC_STRAT_TENSOR) { R.r0 = 0; R.r1 = p.rows; R.c0 = 0; R.c1 = p.cols; }
  else if (a.strategy == LLMC_STRAT_CHANNEL) { R.r0 = gi; R.r1 = gi + 1; R.c0 = 0; R.c1 = p.cols; }
  else if (a.strategy == LLMC_STRAT_BLOCK) {
    int64_t br, bc;
    if (gi < (1ll << 31) && p.cols < (1ll << 30) && a.bw < (1ll << 30)) {  // 32-bit divisions are far cheaper
      const uint32_t bc_n = ((uint32_t)p.cols + (uint32_t)a.bw - 1u) / (uint32_t)a.bw;
      const uint32_t q = (uint32_t)gi / bc_n;
      br = q;
      bc = (uint32_t)gi - q * bc_n;
    } else {
      const int64_t bc_n = (p.cols + a.bw - 1) / a.bw;
      br = gi / bc_n;
      bc = gi % bc_n;
    }
    R.r0 = br * a.bh; R.r1 = min(p.rows, R.r0 + a.bh);
    R.c0 = bc * a.bw; R.c1 = min(p.cols, R.c0 + a.bw);
  } else {
    int64_t G = p.cols / a.group;
    R.r0 = gi / G; R.r1 = R.r0 + 1;
    R.c0 = (gi % G) * a.group; R.c1 = R.c0 + a.group;
  }
  return R;
}

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* sh) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float t = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, t) : fminf(v, t);
  }
  __syncthreads();
  if (lane == 0) sh[wid] = v;
  __syncthreads();
  int nw = blockDim.x >> 5;
  v = sh[0];
  for (int i = 1; i < nw; ++i) v = is_max ? fmaxf(v, sh[i]) : fminf(v, sh[i]);
  return v;
}

template <int FMT>
__global__ void __launch_bounds__(256) k_paramgroup(CastParams p) {
  __shared__ float sh[32];
  const int64_t gi = blockIdx.x;
  const Rect R = group_rect(p, gi);
  const int64_t w = R.c1 - R.c0, h = R.r1 - R.r0;
  const bool vec = ((w & 7) == 0) && ((R.c0 & 7) == 0) && ((p.cols & 7) == 0);
  ElemQ e;
  float s_store = 0.f, zp_store = 0.f;
  if (p.mode != MODE_GIVEN) {
    float mn = INFINITY, mx = -INFINITY;
    if (vec) {
      const int64_t wc = w / 8, n = h * wc;
      for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        int64_t r = R.r0 + i / wc, c = R.c0 + (i % wc) * 8;
        uint4 v = __ldg((const uint4*)(p.w + r * p.cols + c));
        float x[8];
        unpack8(v, x);
#pragma unroll
        for (int j = 0; j < 8; ++j) { mn = fminf(mn, x[j]); mx = fmaxf(mx, x[j]); }
      }
    } else {
      const int64_t n = h * w;
      for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        int64_t r = R.r0 + i / w, c = R.c0 + i % w;
        float x = bf16_to_f(p.w[r * p.cols + c]);
        mn = fminf(mn, x); mx = fmaxf(mx, x);
      }
    }
    // zero padding of partial blocks joins the statistics (maybe_pad_tensor_for_block_quant)
    if (p.a.strategy == LLMC_STRAT_BLOCK && (h < p.a.bh || w < p.a.bw)) { mn = fminf(mn, 0.f); mx = fmaxf(mx, 0.f); }
    mn = block_reduce(mn, false, sh);
    mx = block_reduce(mx, true, sh);
    if (p.mode == MODE_STATS) {
      if (threadIdx.x == 0) { p.min_out[gi] = f_to_bf16(mn); p.max_out[gi] = f_to_bf16(mx); }
      return;
    }
    e = make_elemq_fused<FMT>(p, mn, mx, &s_store, &zp_store);
    if (threadIdx.x == 0) store_scale<FMT>(p, gi, s_store, zp_store);
  } else {
    e = make_elemq_given<FMT>(p, gi);
  }
  // pass 2: quantize + pack
  if (vec && !(FMT == LLMC_FMT_PACK_INT32 && p.a.bits == 4 && (p.cols & 7))) {
    const int64_t wc = w / 8, n = h * wc;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      int64_t r = R.r0 + i / wc, c = R.c0 + (i % wc) * 8;
      uint4 v = __ldg((const uint4*)(p.w + r * p.cols + c));
      float x[8];
      unpack8(v, x);
      uint32_t cd[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) cd[j] = quant_code<FMT>(x[j], e);
      if (FMT == LLMC_FMT_PACK_INT32) {
        // row-wise packing: element (r, c) -> word r * ceil(cols/pf) + c/pf
        const int pf = 32 / p.a.bits;
        const int64_t wpr = (p.cols + pf - 1) / pf;
        if (p.a.bits == 4) {
          uint32_t word = 0;
          for (int j = 0; j < 8; ++j) word |= ((cd[j] + 8u) & 0xFu) << (4 * j);
          ((uint32_t*)p.out)[r * wpr + c / 8] = word;
        } else {
          for (int k = 0; k < 2; ++k) {
            uint32_t word = 0;
            for (int j = 0; j < 4; ++j) word |= ((cd[4 * k + j] + 128u) & 0xFFu) << (8 * j);
            ((uint32_t*)p.out)[r * wpr + c / 4 + k] = word;
          }
        }
      } else if (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) {
        uint32_t word = 0;
        for (int j = 0; j < 8; ++j) word |= (cd[j] & 0xFu) << (4 * j);
        *(uint32_t*)((uint8_t*)p.out + (r * p.cols + c) / 2) = word;
      } else {
        uint2 w2;
        w2.x = (cd[0] & 0xFFu) | ((cd[1] & 0xFFu) << 8) | ((cd[2] & 0xFFu) << 16) | ((cd[3] & 0xFFu) << 24);
        w2.y = (cd[4] & 0xFFu) | ((cd[5] & 0xFFu) << 8) | ((cd[6] & 0xFFu) << 16) | ((cd[7] & 0xFFu) << 24);
        *(uint2*)((uint8_t*)p.out + r * p.cols + c) = w2;
      }
    }
  } else {
    // scalar path: one output word per iteration
    int pf = 1;
    if (FMT == LLMC_FMT_PACK_INT32) pf = 32 / p.a.bits;
    else if (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) pf = 2;
    const int64_t c0w = R.c0 / pf;
    const int64_t c1w = (R.c1 + pf - 1) / pf;
    const int64_t ww = c1w - c0w, n = h * ww;
    const int64_t wpr = (p.cols + pf - 1) / pf;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
      int64_t r = R.r0 + i / ww, wc = c0w + i % ww;
      uint32_t word = 0;
      for (int j = 0; j < pf; ++j) {
        int64_t c = wc * pf + j;
        if (c >= p.cols) break;  // padding of the last int32 word stays 0
        uint32_t cd = quant_code<FMT>(bf16_to_f(p.w[r * p.cols + c]), e);
        if (FMT == LLMC_FMT_PACK_INT32) word |= ((cd + (1u << (p.a.bits - 1))) & ((1u << p.a.bits) - 1)) << (p.a.bits * j);
        else if (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) word |= (cd & 0xFu) << (4 * j);
        else word = cd & 0xFFu;
      }
      if (FMT == LLMC_FMT_PACK_INT32) ((uint32_t*)p.out)[r * wpr + wc] = word;
      else ((uint8_t*)p.out)[r * wpr + wc] = (uint8_t)word;
    }
  }
}

// ------------------------------------------------------------------------
// Streaming kernels on packed pairs (sm_100a f32x2 / bf16x2 / e4m3x2 /
// e2m1x2 instructions).  Same results as quant_code, fewer instructions:
//
//  * quotient of two bf16 values at once by Markstein's correction:
//    q0 = x * r (r = RN(1/s)), e = x - q0 * s (exact by fma), q = q0 + e * r
//    (evaluated on -x so that zeros keep their sign, see quot2).
//    With r the correctly rounded reciprocal and q0 within an ulp of x / s,
//    q is the correctly rounded float32 quotient (Markstein 1990; Muller et
//    al., Handbook of Floating-Point Arithmetic, division with fma) when
//    nothing overflows or underflows.  For a bf16 x and a scale with at most
//    8 significant bits, x / s is either exactly a bf16 rounding midpoint or
//    at least 2^-17 (relative) away from one, so RN_bf16(q) equals torch's
//    RN_bf16(RN_f32(x / s)) in both cases.  Groups whose reciprocal is not a
//    normal float divide exactly; with stored (caller-given) scales a pair
//    whose quotient is not finite is recomputed by exact division.
//  * int4: RN_bf16(q + 136) of a clamped code c in [-8, 7] is the bf16
//    number 128 + (c + 8), whose low byte is c + 8: byte permutes pack it.
//  * E2M1: the hardware RNE conversion of a value in [-6, 6] picks the same
//    code as compressed-tensors' thresholds (ties 0.25, 1.25, 2.5, 5 go to
//    the even code below, 0.75, 1.75, 3.5 to the even code above); the
//    reference's "+ zero_point" turns -0.0 into +0.0 first.
// ------------------------------------------------------------------------
__device__ __forceinline__ void pair_f2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_pair(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
// float32 quotients of the two bf16 values of w (low half = first element).
// Written on nx = -x: q0 = nx * (-r), e = q0 * s + nx (= q0 s - x, exact),
// q = q0 + e * (-r).  For x = +-0 every step keeps the zero's sign (the
// form x - q0 s would turn -0 into +0); needs s > 0.
__device__ __forceinline__ uint64_t quot2(uint32_t w, uint64_t nr2, uint64_t s2) {
  uint64_t q;
  asm("{\n\t.reg .b32 lo, hi, t;\n\t.reg .b64 nx, q0, e;\n\t"
      "xor.b32 t, %1, 0x8000;\n\tshl.b32 lo, t, 16;\n\tlop3.b32 hi, %1, 0xFFFF0000, 0x80000000, 0x6A;\n\t"
      "mov.b64 nx, {lo, hi};\n\t"
      "mul.rn.f32x2 q0, nx, %2;\n\tfma.rn.f32x2 e, q0, %3, nx;\n\tfma.rn.f32x2 %0, e, %2, q0;\n\t}"
      : "=l"(q) : "r"(w), "l"(nr2), "l"(s2));
  return q;
}
// The same quotients for outputs where the sign of a zero code does not
// matter (integer codes): q0 = x * r, e = q0 * (-s) + x, q = q0 + e * r
// (the same correctly rounded quotient; x = -0 gives +0).  ns2 = (-s, -s).
__device__ __forceinline__ uint64_t quot2_int(uint32_t w, uint64_t r2, uint64_t ns2) {
  uint64_t q;
  asm("{\n\t.reg .b32 lo, hi;\n\t.reg .b64 x, q0, e;\n\t"
      "shl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xFFFF0000;\n\tmov.b64 x, {lo, hi};\n\t"
      "mul.rn.f32x2 q0, x, %2;\n\tfma.rn.f32x2 e, q0, %3, x;\n\tfma.rn.f32x2 %0, e, %2, q0;\n\t}"
      : "=l"(q) : "r"(w), "l"(r2), "l"(ns2));
  return q;
}
// (lo + 0, hi + 0) rounded to nearest: -0 -> +0, everything else unchanged
__device__ __forceinline__ uint64_t add2_zero(uint64_t v) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(v), "l"(0ull));
  return d;
}
__device__ __forceinline__ uint32_t bf2_of(uint64_t q) {
  uint32_t d;
  asm("{\n\t.reg .b32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.bf16x2.f32 %0, hi, lo;\n\t}" : "=r"(d) : "l"(q));
  return d;
}
__device__ __forceinline__ uint32_t hmax2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmin2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t bf2_dup(float v) { uint32_t b = f_to_bf16(v); return b | (b << 16); }
__device__ __forceinline__ bool finite_bf2(uint32_t q) {
  return ((q & 0x7F80u) != 0x7F80u) && ((q & 0x7F800000u) != 0x7F800000u);
}
// e4m3 bytes of (lo, hi), lo in the low byte; saturating RNE
__device__ __forceinline__ uint32_t e4m3x2(float lo, float hi) {
  uint16_t h;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(h) : "f"(hi), "f"(lo));
  return h;
}
// E2M1 codes of v[0..7], element 2k in the low nibble of byte k
__device__ __forceinline__ uint32_t e2m1x8(const float* v) {
  uint32_t d;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\tcvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\tcvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(d)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return d;
}
__device__ __forceinline__ void ld_v8(const void* p, uint32_t* w) {
  asm volatile("ld.global.cs.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}
__device__ __forceinline__ void st_v8(void* p, const uint32_t* w) {
  asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]),
               "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}
__device__ __forceinline__ void st_v4(void* p, const uint32_t* w) {
  asm volatile("st.global.cs.v4.b32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
               : "memory");
}

// Per-group divisor in the forms the pair routines take.
struct GQ {
  uint64_t nr2, s2;  // (-r, -r), (s, s)
  uint64_t r2, ns2;  // (r, r), (-s, -s)
  float s, zp;
  uint32_t zp2;      // zero point as bf16x2
  bool fast, has_zp, f32q;
};
__device__ __forceinline__ GQ to_gq(const ElemQ& e) {
  GQ g;
  g.s = e.s; g.zp = e.zp; g.has_zp = e.has_zp; g.f32q = e.f32q;
  g.fast = e.fast && e.s > 0.0f;  // the pair form keeps zero signs for positive scales only
  g.nr2 = f2_pair(-e.r, -e.r);
  g.s2 = f2_pair(e.s, e.s);
  g.r2 = f2_pair(e.r, e.r);
  g.ns2 = f2_pair(-e.s, -e.s);
  g.zp2 = e.has_zp ? bf2_dup(e.zp) : 0u;
  return g;
}

template <int FMT, int BITS>
struct OutOf {
  static constexpr bool OUT4 = (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4 || (FMT == LLMC_FMT_PACK_INT32 && BITS == 4));
  static constexpr int WORDS_PER_8 = OUT4 ? 1 : 2;  // output words per 8 elements
};

// Codes of the 2*NW bf16 values in w (one parameter group) -> output words o
// (NW/4 words for 4-bit outputs, NW/2 for 8-bit).  CHECK: scales come from
// the caller, so a quotient may overflow.
// sat (NVFP4): every value of the group is finite, so the saturating E2M1
// conversion does the clamp to [-6, 6] by itself (it differs from fmin/fmax
// only for NaN).  (For MXFP4 the finiteness test cost more than the clamp it
// saves: measured 11% slower.)
template <int FMT, int BITS, bool F32Q, bool CHECK, int NW>
__device__ __forceinline__ void quant_group(const uint32_t* w, const GQ& g, float qmin, float qmax, uint32_t* o,
                                            bool sat = false) {
  constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
  if (!F32Q) {
    uint32_t Q[NW];
    constexpr bool INT_CODES = (FMT == LLMC_FMT_PACK_INT32 || FMT == LLMC_FMT_INT8);
    if (g.fast) {
#pragma unroll
      for (int k = 0; k < NW; ++k)
        Q[k] = bf2_of(INT_CODES ? quot2_int(w[k], g.r2, g.ns2) : quot2(w[k], g.nr2, g.s2));
      if (CHECK) {
#pragma unroll
        for (int k = 0; k < NW; ++k)
          if (!finite_bf2(Q[k]))
            Q[k] = (uint32_t)f_to_bf16(__fdiv_rn(bf_lo(w[k]), g.s)) |
                   ((uint32_t)f_to_bf16(__fdiv_rn(bf_hi(w[k]), g.s)) << 16);
      }
    } else {
#pragma unroll
      for (int k = 0; k < NW; ++k)
        Q[k] = (uint32_t)f_to_bf16(__fdiv_rn(bf_lo(w[k]), g.s)) |
               ((uint32_t)f_to_bf16(__fdiv_rn(bf_hi(w[k]), g.s)) << 16);
    }
    const uint32_t QMIN2 = bf2_dup(qmin), QMAX2 = bf2_dup(qmax);
    if (g.has_zp) {
#pragma unroll
      for (int k = 0; k < NW; ++k) Q[k] = hadd2(Q[k], g.zp2);  // rbf(q + zp)
    }
    if (FMT == LLMC_FMT_PACK_INT32 || FMT == LLMC_FMT_INT8) {
#pragma unroll
      for (int k = 0; k < NW; ++k) Q[k] = hmin2(hmax2(Q[k], QMIN2), QMAX2);
      if (OUT4) {
#pragma unroll
        for (int j = 0; j < NW / 4; ++j) {
          uint32_t v0 = hadd2(Q[4 * j], 0x43084308u), v1 = hadd2(Q[4 * j + 1], 0x43084308u);
          uint32_t v2 = hadd2(Q[4 * j + 2], 0x43084308u), v3 = hadd2(Q[4 * j + 3], 0x43084308u);
          uint32_t p0 = __byte_perm(v0, v1, 0x6420), p1 = __byte_perm(v2, v3, 0x6420);
          o[j] = __byte_perm(p0 | (p0 >> 4), p1 | (p1 >> 4), 0x6420);
        }
      } else {
        const int bias = (FMT == LLMC_FMT_PACK_INT32) ? 128 : 0;
#pragma unroll
        for (int j = 0; j < NW / 2; ++j) {
          uint32_t b0 = (uint32_t)(__float2int_rn(bf_lo(Q[2 * j])) + bias) & 0xFFu;
          uint32_t b1 = (uint32_t)(__float2int_rn(bf_hi(Q[2 * j])) + bias) & 0xFFu;
          uint32_t b2 = (uint32_t)(__float2int_rn(bf_lo(Q[2 * j + 1])) + bias) & 0xFFu;
          uint32_t b3 = (uint32_t)(__float2int_rn(bf_hi(Q[2 * j + 1])) + bias) & 0xFFu;
          o[j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
      }
    } else if (FMT == LLMC_FMT_FP8) {
      // no clamp to [-448, 448]: the saturating E4M3 conversion does it (and,
      // like torch.clamp, keeps NaN a NaN, where a bf16x2 min/max would not)
#pragma unroll
      for (int j = 0; j < NW / 2; ++j)
        o[j] = e4m3x2(bf_lo(Q[2 * j]), bf_hi(Q[2 * j])) | (e4m3x2(bf_lo(Q[2 * j + 1]), bf_hi(Q[2 * j + 1])) << 16);
    } else {  // FP4 from a bf16 quotient (MXFP4)
#pragma unroll
      for (int j = 0; j < NW / 4; ++j) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t a = hadd2(hmin2(hmax2(Q[4 * j + k], QMIN2), QMAX2), 0u);  // -0 -> +0
          v[2 * k] = bf_lo(a);
          v[2 * k + 1] = bf_hi(a);
        }
        o[j] = e2m1x8(v);
      }
    }
  } else {
    float f[2 * NW];
    if (g.fast) {
#pragma unroll
      for (int k = 0; k < NW; ++k) pair_f2(quot2(w[k], g.nr2, g.s2), f[2 * k], f[2 * k + 1]);
      // an infinite value makes the correction step NaN: NVFP4 groups that are
      // not all finite take the IEEE quotient there (as the general kernels do)
      if (CHECK || (FMT == LLMC_FMT_NVFP4 && !sat)) {
#pragma unroll
        for (int k = 0; k < NW; ++k)
          if (!(fabsf(f[2 * k]) <= 3.4028234663852886e38f && fabsf(f[2 * k + 1]) <= 3.4028234663852886e38f)) {
            f[2 * k] = __fdiv_rn(bf_lo(w[k]), g.s);
            f[2 * k + 1] = __fdiv_rn(bf_hi(w[k]), g.s);
          }
      }
    } else {
#pragma unroll
      for (int k = 0; k < NW; ++k) {
        f[2 * k] = __fdiv_rn(bf_lo(w[k]), g.s);
        f[2 * k + 1] = __fdiv_rn(bf_hi(w[k]), g.s);
      }
    }
    if (FMT != LLMC_FMT_NVFP4 && g.has_zp) {
#pragma unroll
      for (int k = 0; k < 2 * NW; ++k) f[k] = f[k] + g.zp;
    }
    if (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) {
      if (sat) {
#pragma unroll
        for (int j = 0; j < NW / 4; ++j) {
          float v[8];
#pragma unroll
          for (int k = 0; k < 4; ++k) pair_f2(add2_zero(f2_pair(f[8 * j + 2 * k], f[8 * j + 2 * k + 1])), v[2 * k], v[2 * k + 1]);
          o[j] = e2m1x8(v);
        }
      } else {
#pragma unroll
        for (int j = 0; j < NW / 4; ++j) {
          float v[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) v[k] = fminf(fmaxf(__fadd_rn(f[8 * j + k], 0.0f), qmin), qmax);
          o[j] = e2m1x8(v);
        }
      }
    } else if (FMT == LLMC_FMT_FP8) {
#pragma unroll
      for (int j = 0; j < NW / 2; ++j) {
        float a0 = fminf(fmaxf(f[4 * j], qmin), qmax), a1 = fminf(fmaxf(f[4 * j + 1], qmin), qmax);
        float a2 = fminf(fmaxf(f[4 * j + 2], qmin), qmax), a3 = fminf(fmaxf(f[4 * j + 3], qmin), qmax);
        o[j] = e4m3x2(a0, a1) | (e4m3x2(a2, a3) << 16);
      }
    } else {
      int c[2 * NW];
#pragma unroll
      for (int k = 0; k < 2 * NW; ++k) c[k] = __float2int_rn(fminf(fmaxf(f[k], qmin), qmax));
      if (OUT4) {
#pragma unroll
        for (int j = 0; j < NW / 4; ++j) {
          uint32_t word = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) word |= ((uint32_t)(c[8 * j + k] + 8) & 0xFu) << (4 * k);
          o[j] = word;
        }
      } else {
        const int bias = (FMT == LLMC_FMT_PACK_INT32) ? 128 : 0;
#pragma unroll
        for (int j = 0; j < NW / 2; ++j) {
          uint32_t word = 0;
#pragma unroll
          for (int k = 0; k < 4; ++k) word |= ((uint32_t)(c[4 * j + k] + bias) & 0xFFu) << (8 * k);
          o[j] = word;
        }
      }
    }
  }
}

// max |x| over the bf16 values in w[0..NW) (NaNs skipped; 0 for none): what
// a symmetric scheme's scale needs of min(min, 0) and max(max, 0).
template <int NW>
__device__ __forceinline__ float absmax_words(const uint32_t* w) {
  uint32_t M = 0u;
#pragma unroll
  for (int k = 0; k < NW; ++k) asm("max.xorsign.abs.bf16x2 %0, %0, %1;" : "+r"(M) : "r"(w[k]));
  return fmaxf(fabsf(bf_lo(M)), fabsf(bf_hi(M)));
}

// Largest magnitude bit pattern (bits & 0x7FFF) over the bf16 values in
// w[0..NW): below 0x7F80 when every value is finite, and then the bf16 bits
// of max |x| (magnitudes order like their bit patterns).
template <int NW>
__device__ __forceinline__ uint32_t absmax_bits(const uint32_t* w) {
  uint32_t M = 0u;
#pragma unroll
  for (int k = 0; k < NW; ++k) asm("max.u16x2 %0, %0, %1;" : "+r"(M) : "r"(w[k] & 0x7FFF7FFFu));
  return max(M & 0xFFFFu, M >> 16);
}

// min / max of the bf16 values in w[0..NW)
template <int NW>
__device__ __forceinline__ void minmax_words(const uint32_t* w, float& mn, float& mx) {
  uint32_t M = w[0], m = w[0];
#pragma unroll
  for (int k = 1; k < NW; ++k) { M = hmax2(M, w[k]); m = hmin2(m, w[k]); }
  mx = fmaxf(bf_lo(M), bf_hi(M));
  mn = fminf(bf_lo(m), bf_hi(m));
}

// ------------------------------------------------------------------------
// k_stream: power-of-two groups of 8..256 columns over the flat tensor.
// A warp step covers 1024 elements; each lane owns a contiguous span of 32
// (two 32-byte loads), so a group is LPG = GROUP/32 adjacent lanes (reduced
// with shuffles) or a lane holds GPL = 32/GROUP whole groups.  Persistent
// grid; each warp loads its next span before quantizing the current one.
// Needs numel % 32 == 0 and 32-byte aligned input (16 / 32 for the output).
// ------------------------------------------------------------------------
// GROUP == 0: one group for the whole tensor (TENSOR strategy, GIVEN mode).
template <int FMT, int BITS, int GROUP, int MODE>
__device__ __forceinline__ void stream_span(const CastParams& p, int64_t e0, bool valid, const uint32_t* w) {
  constexpr int LPG = GROUP >= 32 ? GROUP / 32 : 1;
  constexpr int GPL = (GROUP >= 32 || GROUP == 0) ? 1 : 32 / GROUP;
  constexpr int NW = 16 / GPL;
  constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
  static_assert(GROUP != 0 || MODE == MODE_GIVEN, "whole-tensor spans take stored qparams");
  const int lane = threadIdx.x & 31;
  const int64_t g0 = GROUP ? e0 / (GROUP ? GROUP : 1) : 0;
  constexpr bool FP4 = (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4);
  constexpr bool NV = (FMT == LLMC_FMT_NVFP4);
  float mns[GPL], mxs[GPL];
  bool sat[GPL];
#pragma unroll
  for (int j = 0; j < GPL; ++j) sat[j] = false;
  static_assert(!FP4 || LPG == 1, "FP4 groups (16 / 32 values) lie within one lane");
  if (MODE == MODE_FUSED && p.a.symmetric && NV) {
    // a symmetric scale reads max(|min(mn, 0)|, |max(mx, 0)|) = max |x| only;
    // the magnitude bit patterns give it and tell whether the group is finite
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
      const uint32_t mb = absmax_bits<NW>(w + j * NW);
      sat[j] = mb < 0x7F80u;
      if (sat[j]) mxs[j] = bf16_to_f((uint16_t)mb);
      else mxs[j] = absmax_words<NW>(w + j * NW);
      mns[j] = 0.0f;
    }
  } else if (MODE == MODE_FUSED && p.a.symmetric) {
    // a symmetric scale reads max(|min(mn, 0)|, |max(mx, 0)|) = max |x| only
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
      mxs[j] = absmax_words<NW>(w + j * NW);
#pragma unroll
      for (int o = 1; o < LPG; o <<= 1) mxs[j] = fmaxf(mxs[j], __shfl_xor_sync(0xffffffffu, mxs[j], o));
      mns[j] = 0.0f;
    }
  } else if (MODE != MODE_GIVEN) {
#pragma unroll
    for (int j = 0; j < GPL; ++j) {
      minmax_words<NW>(w + j * NW, mns[j], mxs[j]);
#pragma unroll
      for (int o = 1; o < LPG; o <<= 1) {
        mns[j] = fminf(mns[j], __shfl_xor_sync(0xffffffffu, mns[j], o));
        mxs[j] = fmaxf(mxs[j], __shfl_xor_sync(0xffffffffu, mxs[j], o));
      }
    }
    if (MODE == MODE_STATS) {
      if (valid && (lane % LPG) == 0) {
#pragma unroll
        for (int j = 0; j < GPL; ++j) { p.min_out[g0 + j] = f_to_bf16(mns[j]); p.max_out[g0 + j] = f_to_bf16(mxs[j]); }
      }
      return;
    }
  }
  if (!valid) return;
  const float qmin = p.a.qmin(), qmax = p.a.qmax();
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < GPL; ++j) {
    ElemQ e;
    float s_store = 0.f, zp_store = 0.f;
    if (MODE == MODE_FUSED) e = make_elemq_fused<FMT>(p, mns[j], mxs[j], &s_store, &zp_store);
    else e = make_elemq_given<FMT>(p, g0 + j);
    GQ g = to_gq(e);
    uint32_t* oj = o + j * (OUT4 ? NW / 4 : NW / 2);
    if (FMT == LLMC_FMT_NVFP4) quant_group<FMT, BITS, true, MODE == MODE_GIVEN, NW>(w + j * NW, g, qmin, qmax, oj, sat[j]);
    else if (MODE == MODE_GIVEN && g.f32q) quant_group<FMT, BITS, true, true, NW>(w + j * NW, g, qmin, qmax, oj);
    else quant_group<FMT, BITS, false, MODE == MODE_GIVEN, NW>(w + j * NW, g, qmin, qmax, oj, sat[j]);
    if (MODE == MODE_FUSED && (lane % LPG) == 0) store_scale<FMT>(p, g0 + j, s_store, zp_store);
  }
  if (OUT4) st_v4((uint8_t*)p.out + e0 / 2, o);
  else st_v8((uint8_t*)p.out + e0, o);
}

// Two ways to keep a warp's next spans in flight while it quantizes one.
//
// span_regs: the next span is loaded into registers (double buffer); one span
// in flight per warp.  Used for the whole-tensor (TENSOR strategy) pass.
//
// span_ring: asynchronous copies into a per-warp ring of NBUF spans in shared
// memory (2 KB each), NBUF - 1 spans in flight per warp without holding them
// in registers, and four CTAs per SM instead of three (measured faster for
// every group size: W4A16 4.52 -> 4.67 TB/s batched).  A lane copies and later reads back only
// its own 64 bytes (so no warp barrier is needed); its four 16-byte chunks
// are stored in an order rotated by lane so that the reads are free of bank
// conflicts.
//
// Both walk work units u = it, it + nwarps, ...; src(u, ptr) gives the
// lane's 32 values of unit u (false past the end of its tensor: nothing is
// read) and proc(u, w) quantizes them (it knows itself which lanes lie past
// the end; their words are not used).  Each is called once per unit, in
// increasing u, so either may keep a cursor.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

constexpr int SPAN_WORDS = 512;  // 1024 bf16 values
constexpr int NBUF = 3;
template <int GROUP>
constexpr bool use_ring() { return GROUP == 16 || GROUP == 32 || GROUP == 64 || GROUP == 128; }
// resident CTAs per SM (the ring takes 48 KB of shared memory per CTA;
// quantizing with stored qparams needs more than 64 registers a thread)
template <int GROUP, int MODE>
constexpr int stream_ctas() { return use_ring<GROUP>() && MODE != MODE_GIVEN ? 4 : 3; }

template <class Src, class Proc>
__device__ __forceinline__ void span_regs(int64_t it, int64_t units, int64_t nwarps, Src src, Proc proc) {
  uint32_t a[16], b[16];
  auto load = [&](int64_t u, uint32_t* buf) {
    const uint16_t* ptr = nullptr;
    if (src(u, ptr)) {
      ld_v8(ptr, buf);
      ld_v8(ptr + 16, buf + 8);
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) buf[k] = 0u;
    }
  };
  if (it < units) load(it, a);
  while (it < units) {
    int64_t nx = it + nwarps;
    if (nx < units) load(nx, b);
    proc(it, a);
    it = nx;
    if (it >= units) break;
    nx = it + nwarps;
    if (nx < units) load(nx, a);
    proc(it, b);
    it = nx;
  }
}

template <class Src, class Proc>
__device__ __forceinline__ void span_ring(int64_t it, int64_t units, int64_t nwarps, Src src, Proc proc) {
  __shared__ __align__(16) uint32_t ring[8][NBUF][SPAN_WORDS];  // 48 KB for 8 warps
  const int lane = threadIdx.x & 31;
  const int rot = (lane >> 1) & 3;
  uint32_t* mine = &ring[threadIdx.x >> 5][0][0] + lane * 16;
  auto issue = [&](int64_t u, int slot) {
    const uint16_t* ptr = nullptr;
    if (u < units && src(u, ptr)) {
      uint32_t* dst = mine + slot * SPAN_WORDS;
#pragma unroll
      for (int k = 0; k < 4; ++k) cp_async16(dst + ((k ^ rot) << 2), ptr + 8 * k);
    }
    cp_async_commit();  // one group per span, empty or not, so the counts stay aligned
  };
#pragma unroll
  for (int s = 0; s < NBUF; ++s) issue(it + s * nwarps, s);
  int slot = 0;
  for (; it < units; it += nwarps) {
    cp_async_wait_group<NBUF - 1>();  // this span's copies have landed
    const uint32_t* from = mine + slot * SPAN_WORDS;
    uint32_t w[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 v = *(const uint4*)(from + ((k ^ rot) << 2));
      w[4 * k] = v.x; w[4 * k + 1] = v.y; w[4 * k + 2] = v.z; w[4 * k + 3] = v.w;
    }
    proc(it, w);
    issue(it + NBUF * nwarps, slot);  // the slot is free again: its values are consumed
    slot = (slot + 1 == NBUF) ? 0 : slot + 1;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

template <int GROUP, class Src, class Proc>
__device__ __forceinline__ void span_loop(int64_t units, Src src, Proc proc) {
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t it = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if constexpr (use_ring<GROUP>()) span_ring(it, units, nwarps, src, proc);
  else span_regs(it, units, nwarps, src, proc);
}

template <int FMT, int BITS, int GROUP, int MODE>
__global__ void __launch_bounds__(256, stream_ctas<GROUP, MODE>()) k_stream(CastParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t n = p.rows * p.cols;
  auto src = [&](int64_t u, const uint16_t*& ptr) {
    const int64_t e0 = (u << 10) + lane * 32;
    ptr = p.w + e0;
    return e0 < n;
  };
  auto proc = [&](int64_t u, const uint32_t* w) {
    const int64_t e0 = (u << 10) + lane * 32;
    stream_span<FMT, BITS, GROUP, MODE>(p, e0, e0 < n, w);
  };
  span_loop<GROUP>((n + 1023) >> 10, src, proc);
}

// ------------------------------------------------------------------------
// TENSOR strategy: a grid-wide min/max (16-bit compare-and-swap on an
// order-preserving encoding of the bf16 bits) into two 16-bit slots, one
// thread turning them into the qparams, then k_stream<GROUP = 0>.
// ------------------------------------------------------------------------
__device__ __forceinline__ uint16_t enc_bf16(uint16_t b) { return (b & 0x8000u) ? (uint16_t)~b : (uint16_t)(b | 0x8000u); }
__device__ __forceinline__ uint16_t dec_bf16(uint16_t e) { return (e & 0x8000u) ? (uint16_t)(e & 0x7FFFu) : (uint16_t)~e; }

__device__ __forceinline__ void cas_extreme(uint16_t* slot, uint16_t v, bool is_max) {
  unsigned short* a = (unsigned short*)slot;
  unsigned short cur = *(volatile unsigned short*)a;
  for (int t = 0; t < (1 << 16); ++t) {  // lock-free: each failed swap means another thread's succeeded
    if (is_max ? (v <= cur) : (v >= cur)) return;
    unsigned short seen = atomicCAS(a, cur, (unsigned short)v);
    if (seen == cur) return;
    cur = seen;
  }
}

__global__ void __launch_bounds__(256) k_tensor_minmax(const uint16_t* w, int64_t n, uint16_t* slot_min,
                                                       uint16_t* slot_max) {
  uint32_t M = 0xFF80FF80u, m = 0x7F807F80u;
  const int64_t pieces = n / 16;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, st = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < pieces; i += st) {
    uint32_t v[8];
    ld_v8(w + i * 16, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) { M = hmax2(M, v[k]); m = hmin2(m, v[k]); }
  }
  float mx = fmaxf(bf_lo(M), bf_hi(M)), mn = fminf(bf_lo(m), bf_hi(m));
  for (int64_t i = pieces * 16 + tid; i < n; i += st) {
    float x = bf16_to_f(w[i]);
    mn = fminf(mn, x); mx = fmaxf(mx, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if ((threadIdx.x & 31) == 0) {
    if (mn <= INFINITY) cas_extreme(slot_min, enc_bf16(f_to_bf16(mn)), false);  // skips NaN
    if (mx >= -INFINITY) cas_extreme(slot_max, enc_bf16(f_to_bf16(mx)), true);
  }
}

template <int FMT>
__global__ void k_tensor_finish(CastParams p, uint16_t* slot_min, uint16_t* slot_max) {
  float mn = bf16_to_f(dec_bf16(*slot_min)), mx = bf16_to_f(dec_bf16(*slot_max));
  if (p.mode == MODE_STATS) {
    p.min_out[0] = f_to_bf16(mn);
    p.max_out[0] = f_to_bf16(mx);
    return;
  }
  float s_store, zp_store;
  make_elemq_fused<FMT>(p, mn, mx, &s_store, &zp_store);
  store_scale<FMT>(p, 0, s_store, zp_store);
}

// ------------------------------------------------------------------------
// k_tile: CHANNEL rows and BLOCK tiles, one CTA per group at a time, the
// whole group held in registers (NP 16-value pieces per thread): one HBM
// read.  Persistent over groups; with PF the CTA loads its next group while
// it quantizes the current one.  Needs cols % 16 == 0, block width % 16 == 0,
// 32-byte aligned input.
// ------------------------------------------------------------------------
template <int NP>
__device__ __forceinline__ void tile_load(const CastParams& p, int64_t gi, uint32_t (&w)[NP][8]) {
  const Rect R = group_rect(p, gi);
  const int64_t ppr = (R.c1 - R.c0) / 16, npc = (R.r1 - R.r0) * ppr;
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int64_t pc = threadIdx.x + (int64_t)blockDim.x * j;
    if (pc < npc) ld_v8(p.w + (R.r0 + pc / ppr) * p.cols + R.c0 + (pc % ppr) * 16, w[j]);
  }
}

template <int FMT, int BITS, int MODE, int NP>
__device__ __forceinline__ void tile_process(const CastParams& p, int64_t gi, const uint32_t (&w)[NP][8], float* sh) {
  constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
  const Rect R = group_rect(p, gi);
  const int64_t ppr = (R.c1 - R.c0) / 16, npc = (R.r1 - R.r0) * ppr;
  ElemQ e;
  float s_store = 0.f, zp_store = 0.f;
  if (MODE != MODE_GIVEN) {
    uint32_t M = 0xFF80FF80u, m = 0x7F807F80u;  // (-inf, -inf), (+inf, +inf)
#pragma unroll
    for (int j = 0; j < NP; ++j)
      if (threadIdx.x + (int64_t)blockDim.x * j < npc) {
#pragma unroll
        for (int k = 0; k < 8; ++k) { M = hmax2(M, w[j][k]); m = hmin2(m, w[j][k]); }
      }
    float mx = fmaxf(bf_lo(M), bf_hi(M)), mn = fminf(bf_lo(m), bf_hi(m));
    const int64_t h = R.r1 - R.r0, wd = R.c1 - R.c0;
    if (p.a.strategy == LLMC_STRAT_BLOCK && (h < p.a.bh || wd < p.a.bw)) { mn = fminf(mn, 0.f); mx = fmaxf(mx, 0.f); }
    mn = block_reduce(mn, false, sh);
    mx = block_reduce(mx, true, sh);
    if (MODE == MODE_STATS) {
      if (threadIdx.x == 0) { p.min_out[gi] = f_to_bf16(mn); p.max_out[gi] = f_to_bf16(mx); }
      return;
    }
    e = make_elemq_fused<FMT>(p, mn, mx, &s_store, &zp_store);
    if (threadIdx.x == 0) store_scale<FMT>(p, gi, s_store, zp_store);
  } else {
    e = make_elemq_given<FMT>(p, gi);
  }
  const GQ g = to_gq(e);
  const float qmin = p.a.qmin(), qmax = p.a.qmax();
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int64_t pc = threadIdx.x + (int64_t)blockDim.x * j;
    if (pc >= npc) break;
    const int64_t el = (R.r0 + pc / ppr) * p.cols + R.c0 + (pc % ppr) * 16;
    uint32_t o[4];
    if (FMT == LLMC_FMT_NVFP4 || (MODE == MODE_GIVEN && g.f32q))
      quant_group<FMT, BITS, true, MODE == MODE_GIVEN, 8>(w[j], g, qmin, qmax, o);
    else quant_group<FMT, BITS, false, MODE == MODE_GIVEN, 8>(w[j], g, qmin, qmax, o);
    if (OUT4) *(uint2*)((uint8_t*)p.out + el / 2) = make_uint2(o[0], o[1]);
    else st_v4((uint8_t*)p.out + el, o);
  }
}

// THR threads per CTA; 128-thread CTAs holding a whole 128x128 block (NP = 8)
// put four blocks in flight per SM without prefetch registers.
template <int FMT, int BITS, int MODE, int NP, bool PF, int THR = 256>
__global__ void __launch_bounds__(THR, PF ? 2 : (THR == 128 ? (NP <= 4 ? 6 : 4) : 2)) k_tile(CastParams p, int64_t ng) {
  __shared__ float sh[32];
  int64_t gi = blockIdx.x;
  if (!PF) {
    for (; gi < ng; gi += gridDim.x) {
      uint32_t w[NP][8];
      tile_load<NP>(p, gi, w);
      tile_process<FMT, BITS, MODE, NP>(p, gi, w, sh);
    }
    return;
  }
  uint32_t a[NP][8], b[NP][8];
  if (gi < ng) tile_load<NP>(p, gi, a);
  while (gi < ng) {
    int64_t nx = gi + gridDim.x;
    if (nx < ng) tile_load<NP>(p, nx, b);
    tile_process<FMT, BITS, MODE, NP>(p, gi, a, sh);
    gi = nx;
    if (gi >= ng) break;
    nx = gi + gridDim.x;
    if (nx < ng) tile_load<NP>(p, nx, a);
    tile_process<FMT, BITS, MODE, NP>(p, gi, b, sh);
    gi = nx;
  }
}

// ------------------------------------------------------------------------
// k_rowwarp: CHANNEL rows of up to 4096 columns, one warp per row, NPL
// 16-value pieces per lane (32-byte loads, consecutive across the warp);
// shuffles only, no CTA barrier, so many rows are in flight per SM.
// ------------------------------------------------------------------------
template <int FMT, int BITS, int MODE, int NPL>
__device__ __forceinline__ void rowwarp_row(const CastParams& p, int64_t row) {
  constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
  const int lane = threadIdx.x & 31;
  const int64_t pieces = p.cols / 16;
  const uint16_t* src = p.w + row * p.cols;
  uint32_t w[NPL][8];
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int64_t pc = lane + 32 * j;
    if (pc < pieces) ld_v8(src + pc * 16, w[j]);
  }
  ElemQ e;
  float s_store = 0.f, zp_store = 0.f;
  if (MODE != MODE_GIVEN) {
    uint32_t M = 0xFF80FF80u, m = 0x7F807F80u;
#pragma unroll
    for (int j = 0; j < NPL; ++j)
      if (lane + 32 * j < pieces) {
#pragma unroll
        for (int k = 0; k < 8; ++k) { M = hmax2(M, w[j][k]); m = hmin2(m, w[j][k]); }
      }
    float mx = fmaxf(bf_lo(M), bf_hi(M)), mn = fminf(bf_lo(m), bf_hi(m));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (MODE == MODE_STATS) {
      if (lane == 0) { p.min_out[row] = f_to_bf16(mn); p.max_out[row] = f_to_bf16(mx); }
      return;
    }
    e = make_elemq_fused<FMT>(p, mn, mx, &s_store, &zp_store);
    if (lane == 0) store_scale<FMT>(p, row, s_store, zp_store);
  } else {
    e = make_elemq_given<FMT>(p, row);
  }
  const GQ g = to_gq(e);
  const float qmin = p.a.qmin(), qmax = p.a.qmax();
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int64_t pc = lane + 32 * j;
    if (pc >= pieces) break;
    const int64_t el = row * p.cols + pc * 16;
    uint32_t o[4];
    if (FMT == LLMC_FMT_NVFP4 || (MODE == MODE_GIVEN && g.f32q))
      quant_group<FMT, BITS, true, MODE == MODE_GIVEN, 8>(w[j], g, qmin, qmax, o);
    else quant_group<FMT, BITS, false, MODE == MODE_GIVEN, 8>(w[j], g, qmin, qmax, o);
    if (OUT4) *(uint2*)((uint8_t*)p.out + el / 2) = make_uint2(o[0], o[1]);
    else st_v4((uint8_t*)p.out + el, o);
  }
}

template <int FMT, int BITS, int MODE, int NPL>
__global__ void __launch_bounds__(256) k_rowwarp(CastParams p) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= p.rows) return;  // whole warp
  rowwarp_row<FMT, BITS, MODE, NPL>(p, row);
}

// ------------------------------------------------------------------------
// Batched launches: many tensors (model-free shards, MoE experts) in one
// persistent launch.  The job table travels in the kernel parameters; a work
// unit is a 1024-value span (group strategies) or a parameter group (CHANNEL
// rows, BLOCK tiles), numbered across the jobs.
// ------------------------------------------------------------------------
constexpr int kBatchMax = 48;
struct CastJob {
  const uint16_t* w;
  int64_t rows, cols;
  int64_t first;  // first work unit of this job
  const float* gs;
  void* out;
  void* scale_out;
  int8_t* zp_out;
  // k_stream_batch: the pointers rebased to the batch's global element
  // numbering (moved back by the elements before the job, first * 1024), so
  // global element e addresses the job's data directly; the job's elements
  // end at lim.  Set on the host (launch_batch_fmt).
  const uint16_t* w_rb;
  void* out_rb;
  void* scale_rb;
  int8_t* zp_rb;
  int64_t lim;
};
struct CastBatch {
  CastParams base;  // arguments, format and mode shared by the jobs
  int njobs;
  int64_t units;
  CastJob job[kBatchMax];
};

__device__ __forceinline__ int find_job(const CastBatch& b, int64_t u) {
  int lo = 0, hi = b.njobs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (b.job[mid].first <= u) lo = mid; else hi = mid - 1;
  }
  return lo;
}
__device__ __forceinline__ CastParams job_params(const CastBatch& b, int j) {
  CastParams p = b.base;
  const CastJob& jb = b.job[j];
  p.w = jb.w; p.rows = jb.rows; p.cols = jb.cols; p.gs = jb.gs;
  p.out = jb.out; p.scale_out = jb.scale_out; p.zp_out = jb.zp_out;
  return p;
}

template <int FMT, int BITS, int GROUP>
__global__ void __launch_bounds__(256, stream_ctas<GROUP, MODE_FUSED>()) k_stream_batch(const __grid_constant__ CastBatch b) {
  const int lane = threadIdx.x & 31;
  // job cursors: units arrive in increasing order, so the job index only
  // moves forward; a warp compares each unit with the next job's first unit
  // and otherwise reads the job's rebased pointers (no per-unit arithmetic)
  const int64_t u0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int js = u0 < b.units ? find_job(b, u0) : 0, jp = js;
  auto next_first = [&](int j) { return j + 1 < b.njobs ? b.job[j + 1].first : INT64_MAX; };
  int64_t snext = next_first(js), pnext = snext;
  auto src = [&](int64_t u, const uint16_t*& ptr) {
    if (u >= snext) {
      while (js + 1 < b.njobs && b.job[js + 1].first <= u) ++js;
      snext = next_first(js);
    }
    const int64_t e0 = (u << 10) + lane * 32;
    ptr = b.job[js].w_rb + e0;
    return e0 < b.job[js].lim;
  };
  auto proc = [&](int64_t u, const uint32_t* w) {
    if (u >= pnext) {
      while (jp + 1 < b.njobs && b.job[jp + 1].first <= u) ++jp;
      pnext = next_first(jp);
    }
    const CastJob& jb = b.job[jp];
    CastParams p = b.base;
    p.gs = jb.gs; p.out = jb.out_rb; p.scale_out = jb.scale_rb; p.zp_out = jb.zp_rb;
    const int64_t e0 = (u << 10) + lane * 32;
    stream_span<FMT, BITS, GROUP, MODE_FUSED>(p, e0, e0 < jb.lim, w);
  };
  span_loop<GROUP>(b.units, src, proc);
}

// CHANNEL rows of up to 4096 columns across the jobs of a batch: one warp
// per row as in k_rowwarp (the whole row's loads issued at once, a
// non-persistent grid); the warp finds its row's job by a search of the job
// table.
template <int FMT, int BITS, int NPL>
__global__ void __launch_bounds__(256) k_rowwarp_batch(const __grid_constant__ CastBatch b) {
  const int64_t u = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (u >= b.units) return;  // whole warp
  const int j = find_job(b, u);
  rowwarp_row<FMT, BITS, MODE_FUSED, NPL>(job_params(b, j), u - b.job[j].first);
}

// Group strategies over the flat tensor, NS consecutive 1024-value spans per
// warp: every load of the warp's spans is issued before the first is
// quantized, and the grid is not persistent (a warp's 2 KB x NS stay in
// flight while the SM's other warps compute), the structure of k_rowwarp.
// Used for single FP4 tensors (groups of 16 / 32), where two spans per warp
// measured faster than k_stream's ring (NVFP4 4.20 -> 4.57 TB/s on a
// 28672 x 8192 weight); batches and the other groups measured faster with
// k_stream / k_stream_batch.
template <int FMT, int BITS, int GROUP, int MODE, int NS>
__global__ void __launch_bounds__(256) k_spans(CastParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t n = p.rows * p.cols;
  const int64_t u0 = (((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5) * NS;
  uint32_t w[NS][16];
#pragma unroll
  for (int k = 0; k < NS; ++k) {
    const int64_t e0 = ((u0 + k) << 10) + lane * 32;
    if (e0 < n) {
      ld_v8(p.w + e0, w[k]);
      ld_v8(p.w + e0 + 16, w[k] + 8);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[k][i] = 0u;
    }
  }
#pragma unroll
  for (int k = 0; k < NS; ++k) {
    const int64_t e0 = ((u0 + k) << 10) + lane * 32;
    if ((u0 + k) << 10 >= n) break;  // whole warp
    stream_span<FMT, BITS, GROUP, MODE>(p, e0, e0 < n, w[k]);
  }
}

// Groups of 64 / 128 values with one lane per group: a warp covers 32
// consecutive groups (2048 / 4096 values), each lane loads its own group
// (whole 32-byte sectors, so no DRAM bytes are wasted although a load
// instruction spans 32 sectors) and computes its own group's scale, where the
// span kernels compute every scale once per lane of the group (2 / 4 times)
// and combine the statistics by shuffles.  All loads of a warp are issued
// before the first value is quantized; the grid is not persistent (the
// structure of k_rowwarp).  src_of(gi, ptr, p) gives group gi's values and
// parameters (false past the end).
template <int FMT, int BITS, int GROUP, class Src>
__device__ __forceinline__ void lane_group(int64_t gi, Src src_of) {
  constexpr int NW = GROUP / 2;  // bf16x2 words per group
  constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
  static_assert(GROUP == 64 || GROUP == 128, "lane groups of 64 or 128 values");
  const uint16_t* ptr = nullptr;
  CastParams p;
  if (!src_of(gi, ptr, p)) return;
  uint32_t w[NW];
#pragma unroll
  for (int k = 0; k < NW / 8; ++k) ld_v8(ptr + 16 * k, w + 8 * k);
  float mn, mx;
  if (p.a.symmetric) {
    mx = absmax_words<NW>(w);
    mn = 0.0f;
  } else {
    minmax_words<NW>(w, mn, mx);
  }
  float s_store = 0.f, zp_store = 0.f;
  const ElemQ e = make_elemq_fused<FMT>(p, mn, mx, &s_store, &zp_store);
  const GQ g = to_gq(e);
  const float qmin = p.a.qmin(), qmax = p.a.qmax();
  uint32_t o[OUT4 ? NW / 4 : NW / 2];
  quant_group<FMT, BITS, false, false, NW>(w, g, qmin, qmax, o);
  uint8_t* out = (uint8_t*)p.out + (OUT4 ? gi * (GROUP / 2) : gi * GROUP);
#pragma unroll
  for (int k = 0; k < (OUT4 ? NW / 4 : NW / 2) / 4; ++k) st_v4(out + 16 * k, o + 4 * k);
  store_scale<FMT>(p, gi, s_store, zp_store);
}

// Batches of groups of 64 / 128 values (W4A16 and other integer group
// schemes), one lane per group; a unit is a group, numbered across the jobs
// (CastJob::first counts groups here).  Measured against k_stream_batch on
// 32 weights of 4096 x 4096: W4A16 4.67 -> 4.80 TB/s, 5.75 in two-warp CTAs
// (single tensors stay on k_stream, which measured the same as this layout).
template <int FMT, int BITS, int GROUP>
__global__ void __launch_bounds__(256) k_lanegroup_batch(const __grid_constant__ CastBatch b) {
  const int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  lane_group<FMT, BITS, GROUP>(gi, [&](int64_t u, const uint16_t*& ptr, CastParams& q) {
    if (u >= b.units) return false;
    const int j = find_job(b, u);
    q = job_params(b, j);
    const int64_t lg = u - b.job[j].first;  // the group within its job
    ptr = q.w + lg * GROUP;
    // rebase the outputs so that lane_group's global group index addresses them
    q.out = (uint8_t*)q.out - (OutOf<FMT, BITS>::OUT4 ? b.job[j].first * (GROUP / 2) : b.job[j].first * GROUP);
    q.scale_out = (uint8_t*)q.scale_out - b.job[j].first * ((FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) ? 1 : 2);
    if (q.zp_out) q.zp_out -= b.job[j].first;
    return true;
  });
}

// 128-thread CTAs, one group at a time without prefetch: several CTAs per SM
// keep their loads in flight (the batched form of k_tile<..., THR = 128>).
template <int FMT, int BITS, int NP>
__global__ void __launch_bounds__(128, 4) k_tile_batch128(const __grid_constant__ CastBatch b) {
  __shared__ float sh[32];
  for (int64_t gi = blockIdx.x; gi < b.units; gi += gridDim.x) {
    const int j = find_job(b, gi);
    const CastParams p = job_params(b, j);
    uint32_t w[NP][8];
    tile_load<NP>(p, gi - b.job[j].first, w);
    tile_process<FMT, BITS, MODE_FUSED, NP>(p, gi - b.job[j].first, w, sh);
  }
}

template <int FMT, int BITS, int NP>
__global__ void __launch_bounds__(256, 2) k_tile_batch(const __grid_constant__ CastBatch b) {
  __shared__ float sh[32];
  int64_t gi = blockIdx.x;
  uint32_t a[NP][8], c[NP][8];
  int ja = 0, jc = 0;
  if (gi < b.units) { ja = find_job(b, gi); const CastParams p = job_params(b, ja); tile_load<NP>(p, gi - b.job[ja].first, a); }
  while (gi < b.units) {
    int64_t nx = gi + gridDim.x;
    if (nx < b.units) { jc = find_job(b, nx); const CastParams p = job_params(b, jc); tile_load<NP>(p, nx - b.job[jc].first, c); }
    { const CastParams p = job_params(b, ja); tile_process<FMT, BITS, MODE_FUSED, NP>(p, gi - b.job[ja].first, a, sh); }
    gi = nx;
    if (gi >= b.units) break;
    nx = gi + gridDim.x;
    if (nx < b.units) { ja = find_job(b, nx); const CastParams p = job_params(b, ja); tile_load<NP>(p, nx - b.job[ja].first, a); }
    { const CastParams p = job_params(b, jc); tile_process<FMT, BITS, MODE_FUSED, NP>(p, gi - b.job[jc].first, c, sh); }
    gi = nx;
  }
}

// ------------------------------------------------------------------------
// k_block_tma: 128 x 128 BLOCK groups (FP8_BLOCK and other block schemes of
// that size) streamed through shared memory by the tensor-memory accelerator.
// Persistent CTAs, three per SM; each keeps a ring of two 32 KB stages, one
// whole block per stage, filled by one 2-D bulk tensor copy (out-of-range
// rows and columns arrive as zeros, which is the reference's zero padding of
// partial blocks).  The 256 threads read the block from shared memory twice
// (consecutive 16-byte chunks across a warp: conflict-free): once for the
// block's min/max, once to quantize and write the codes straight to global
// memory.  Nothing of a block is held in registers, so three CTAs (24 warps)
// fit an SM with six blocks in flight.  Jobs
// (tensors) of a batch each have their own tensor map.  Every wait is
// bounded; a timeout raises the library's device status word and the CTA
// stops (llmc_device_status reads it).
// ------------------------------------------------------------------------
constexpr int TB_STAGES = 2;
constexpr int TB_BYTES = 128 * 128 * 2;
constexpr int TB_SMEM = TB_STAGES * TB_BYTES + 1024 + 64;
constexpr int kTmaJobsMax = kBatchMax;  // maps in the kernel parameters: 6 KB (parameter space up to 32 KB)
__device__ int g_async_status;  // LLMC_ETIMEOUT after a bounded wait ran out (llmc_device_status)

struct TmaMaps {
  CUtensorMap map[kTmaJobsMax];
};

template <int FMT, int BITS, int MODE>
__global__ void __launch_bounds__(256, 3) k_block_tma(const __grid_constant__ CastBatch b,
                                                      const __grid_constant__ TmaMaps m) {
  using namespace sm100;
  constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
  extern __shared__ uint8_t tb_raw[];
  uint8_t* ring = (uint8_t*)(((uintptr_t)tb_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(ring + TB_STAGES * TB_BYTES);
  __shared__ float sh[32];
  __shared__ int abort_flag;
  const int t = threadIdx.x;
  if (t == 0) {
    for (int s = 0; s < TB_STAGES; ++s) mbar_init(smem_u32(&full[s]), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  int jl = 0;  // job cursor of the loads (units only increase)
  auto issue = [&](int64_t u, int s) {
    while (jl + 1 < b.njobs && b.job[jl + 1].first <= u) ++jl;
    const CastParams p = job_params(b, jl);
    const Rect R = group_rect(p, u - b.job[jl].first);
    const uint32_t bar = smem_u32(&full[s]);
    mbar_arrive_expect_tx(bar, TB_BYTES);
    tma_load_2d(smem_u32(ring + s * TB_BYTES), &m.map[jl], (int32_t)R.c0, (int32_t)R.r0, bar);
  };
  const int64_t stride = gridDim.x;
  if (t == 0) {
    for (int s = 0; s < TB_STAGES; ++s) {
      const int64_t u = blockIdx.x + s * stride;
      if (u < b.units) issue(u, s);
    }
  }
  int jp = 0;
  int s = 0;
  uint32_t phase = 0;
  const float qmin = b.base.a.qmin(), qmax = b.base.a.qmax();
  // this thread's chunks: c = j * 256 + t -> row j * 16 + t / 16, columns (t % 16) * 8 .. + 7
  const int crow = t >> 4, ccol = (t & 15) * 8;
  for (int64_t u = blockIdx.x; u < b.units; u += stride) {
    if (t == 0 && !mbar_wait(smem_u32(&full[s]), phase, (volatile int*)&abort_flag)) {
      atomicMax(&g_async_status, (int)LLMC_ETIMEOUT);
    }
    __syncthreads();  // the block has landed (or the wait gave up)
    if (abort_flag) break;
    const uint4* stage = (const uint4*)(ring + s * TB_BYTES) + t;
    while (jp + 1 < b.njobs && b.job[jp + 1].first <= u) ++jp;
    const CastParams p = job_params(b, jp);
    const int64_t gi = u - b.job[jp].first;
    const Rect R = group_rect(p, gi);
    ElemQ e;
    float s_store = 0.f, zp_store = 0.f;
    if (MODE != MODE_GIVEN) {
      float mx, mn;
      if (MODE == MODE_FUSED && b.base.a.symmetric) {
        // a symmetric scale reads max |x| only
        uint32_t v8[8 * 4];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 v = stage[j * 256];
          v8[4 * j] = v.x; v8[4 * j + 1] = v.y; v8[4 * j + 2] = v.z; v8[4 * j + 3] = v.w;
        }
        mx = block_reduce(absmax_words<32>(v8), true, sh);
        mn = 0.0f;
      } else {
        uint32_t M = 0xFF80FF80u, mn2 = 0x7F807F80u;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 v = stage[j * 256];
          M = hmax2(hmax2(M, v.x), hmax2(v.y, hmax2(v.z, v.w)));
          mn2 = hmin2(hmin2(mn2, v.x), hmin2(v.y, hmin2(v.z, v.w)));
        }
        mx = fmaxf(bf_lo(M), bf_hi(M));
        mn = fminf(bf_lo(mn2), bf_hi(mn2));
        mn = block_reduce(mn, false, sh);
        mx = block_reduce(mx, true, sh);
      }
      if (MODE == MODE_STATS) {
        if (t == 0) { p.min_out[gi] = f_to_bf16(mn); p.max_out[gi] = f_to_bf16(mx); }
      } else {
        e = make_elemq_fused<FMT>(p, mn, mx, &s_store, &zp_store);
        if (t == 0) store_scale<FMT>(p, gi, s_store, zp_store);
      }
    } else {
      e = make_elemq_given<FMT>(p, gi);
    }
    if (MODE != MODE_STATS) {
      const GQ g = to_gq(e);
      const int64_t h = R.r1 - R.r0, wd = R.c1 - R.c0;
      const bool full_block = h == 128 && wd == 128;
      uint8_t* out0 = (uint8_t*)p.out;
      const int64_t el0 = (R.r0 + crow) * p.cols + R.c0 + ccol;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (!full_block && (j * 16 + crow >= h || ccol >= wd)) continue;
        const uint4 v = stage[j * 256];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[2];
        if (MODE == MODE_GIVEN && g.f32q) quant_group<FMT, BITS, true, true, 4>(w, g, qmin, qmax, o);
        else quant_group<FMT, BITS, false, MODE == MODE_GIVEN, 4>(w, g, qmin, qmax, o);
        const int64_t el = el0 + (int64_t)j * 16 * p.cols;
        if (OUT4) *(uint32_t*)(out0 + el / 2) = o[0];
        else *(uint2*)(out0 + el) = make_uint2(o[0], o[1]);
      }
    }
    __syncthreads();  // every thread is done with the stage: refill it
    if (t == 0) {
      fence_proxy_async_smem();
      const int64_t nu = u + TB_STAGES * stride;
      if (nu < b.units) issue(nu, s);
    }
    if (++s == TB_STAGES) { s = 0; phase ^= 1; }
  }
  if (abort_flag && t == 0) {
    // let the copies issued before the stop land before the CTA exits
    volatile int dummy = 0;
    for (int k = 0; k < TB_STAGES; ++k) {
      mbar_wait(smem_u32(&full[s]), phase, &dummy, 100000000ull);
      if (++s == TB_STAGES) { s = 0; phase ^= 1; }
    }
  }
}

static int n_groups(const CastParams& p);

static PFN_cuTensorMapEncodeTiled_v12000 tb_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)ptr;
  });
  return fn;
}

// Whether the TMA block kernel takes these jobs: 128 x 128 blocks, 16-byte
// aligned rows and bases, outputs aligned for their vector stores.
static bool tma_block_ok(const CastParams& p) {
  const QArgs& a = p.a;
  const bool out4 = p.fmt == LLMC_FMT_NVFP4 || p.fmt == LLMC_FMT_MXFP4 || (p.fmt == LLMC_FMT_PACK_INT32 && a.bits == 4);
  return a.strategy == LLMC_STRAT_BLOCK && a.bh == 128 && a.bw == 128 && p.cols % 16 == 0 &&
         (uintptr_t)p.w % 16 == 0 && (p.mode == MODE_STATS || (uintptr_t)p.out % (out4 ? 4 : 8) == 0) &&
         p.rows < (1ll << 31) && p.cols < (1ll << 31) && tb_encoder() != nullptr;
}

template <int FMT, int BITS, int MODE>
static bool launch_block_tma(CastBatch& b, cudaStream_t st) {
  if (b.njobs > kTmaJobsMax) return false;
  TmaMaps m;
  memset(&m, 0, sizeof(m));
  int64_t units = 0;
  for (int i = 0; i < b.njobs; ++i) {
    CastJob& j = b.job[i];
    j.first = units;
    CastParams p = b.base;
    p.rows = j.rows; p.cols = j.cols;
    units += n_groups(p);
    cuuint64_t dims[2] = {(cuuint64_t)j.cols, (cuuint64_t)j.rows};
    cuuint64_t strides[1] = {(cuuint64_t)j.cols * 2};
    cuuint32_t box[2] = {128, 128};
    cuuint32_t estr[2] = {1, 1};
    if (tb_encoder()(&m.map[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(j.w), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return false;
  }
  b.units = units;
  if (units == 0) return true;
  static std::mutex mu;
  static uint64_t done = 0;
  {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (dev < 64 && !((done >> dev) & 1ull)) {
      if (cudaFuncSetAttribute(k_block_tma<FMT, BITS, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, TB_SMEM) !=
          cudaSuccess)
        return false;
      done |= 1ull << dev;
    }
  }
  const unsigned grid = (unsigned)std::min<int64_t>(units, 148 * 3);
  k_block_tma<FMT, BITS, MODE><<<grid, 256, TB_SMEM, st>>>(b, m);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess;
}

template <int FMT, int BITS, int MODE>
static bool launch_block_tma_one(const CastParams& p, cudaStream_t st) {
  CastBatch b;
  memset(&b, 0, sizeof(b));
  b.base = p;
  b.njobs = 1;
  CastJob& j = b.job[0];
  j.w = p.w; j.rows = p.rows; j.cols = p.cols; j.gs = p.gs;
  j.out = p.out; j.scale_out = p.scale_out; j.zp_out = p.zp_out;
  return launch_block_tma<FMT, BITS, MODE>(b, st);
}

// ------------------------------------------------------------------------
// small kernels
// ------------------------------------------------------------------------
__global__ void k_absmax(const uint16_t* w, int64_t n, float* out) {
  float m = 0.0f;
  const int64_t n8 = n / 8;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, st = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < n8; i += st) {
    uint4 v = __ldcs((const uint4*)w + i);
    float x[8];
    unpack8(v, x);
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(x[j]));
  }
  for (int64_t i = n8 * 8 + tid; i < n; i += st) m = fmaxf(m, fabsf(bf16_to_f(w[i])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax((unsigned int*)out, __float_as_uint(m));  // m >= 0: uint order == float order
}

__global__ void k_global_scale(const float* absmax, float* gs) { *gs = global_scale_from_absmax(*absmax); }

__global__ void k_qparams(const uint16_t* mn, const uint16_t* mx, int64_t n, QArgs a, const float* gs,
                          void* scale_out, void* zp_out, int f32stats) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float zp;
  bool has_gs = gs != nullptr;
  float s = group_qparams(bf16_to_f(mn[i]), bf16_to_f(mx[i]), a, has_gs, has_gs ? *gs : 0.f, &zp, f32stats != 0);
  // otherwise the statistics' dtype (bf16), as round_to_quantized_type_dtype casts back
  bool f32out = has_gs || f32stats;
  if (f32out) ((float*)scale_out)[i] = s;
  else ((uint16_t*)scale_out)[i] = f_to_bf16(s);
  if (zp_out) {
    if (a.zp_dtype == LLMC_ZP_INT8) ((int8_t*)zp_out)[i] = (int8_t)(int32_t)zp;
    else if (a.zp_dtype == LLMC_ZP_UINT8) ((uint8_t*)zp_out)[i] = (uint8_t)(int32_t)zp;
    else ((float*)zp_out)[i] = 0.0f;
  }
}

// int8 tensors holding int4 codes -> two codes per byte, even column in the
// low nibble (S/utils/pack_int4_to_int8.py:13-28 `_pack_int4_to_int8`).  A
// thread packs 32 values (two 16-byte loads, one 16-byte store) when the
// row length and pointers allow, else one output byte.
__global__ void k_pack_int4_int8(const int8_t* __restrict__ in, int64_t rows, int64_t cols, int8_t* __restrict__ out,
                                 int vec) {
  const int64_t half = cols / 2, n = rows * half;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x, st = (int64_t)gridDim.x * blockDim.x;
  if (vec) {  // cols % 32 == 0, 16-byte aligned: 16 output bytes per step
    const int64_t n16 = n / 16;
    for (int64_t i = tid; i < n16; i += st) {
      const uint4 a = __ldcs((const uint4*)in + 2 * i), b = __ldcs((const uint4*)in + 2 * i + 1);
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t lo = w[2 * k] & 0x0F0F0F0Fu, hi = w[2 * k + 1] & 0x0F0F0F0Fu;
        // bytes b0..b3 of lo (cols 0..3 of 8) and hi (cols 4..7): pair (0,1) (2,3) of each
        const uint32_t plo = (lo & 0x000F000Fu) | ((lo >> 4) & 0x00F000F0u);  // [c0|c1<<4, -, c2|c3<<4, -]
        const uint32_t phi = (hi & 0x000F000Fu) | ((hi >> 4) & 0x00F000F0u);
        o[k] = __byte_perm(plo, phi, 0x6420);
      }
      __stcs((uint4*)out + i, make_uint4(o[0], o[1], o[2], o[3]));
    }
    return;
  }
  for (int64_t i = tid; i < n; i += st) {
    const int64_t r = i / half, c = i % half;
    const uint8_t lo = (uint8_t)in[r * cols + 2 * c] & 0x0F, hi = (uint8_t)in[r * cols + 2 * c + 1] & 0x0F;
    out[i] = (int8_t)(uint8_t)((hi << 4) | lo);
  }
}

__global__ void k_pack_zp(const int8_t* zp, int64_t rows, int64_t groups, int bits, int32_t* out) {
  // packed along dim 0: out[(r/pf), g] holds rows r..r+pf-1 of column g
  const int pf = 32 / bits;
  const int64_t prow = (rows + pf - 1) / pf;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= prow * groups) return;
  int64_t pr = i / groups, g = i % groups;
  uint32_t word = 0;
  for (int j = 0; j < pf; ++j) {
    int64_t r = pr * pf + j;
    if (r >= rows) break;
    uint32_t v = ((uint32_t)((int32_t)zp[r * groups + g] + (1 << (bits - 1)))) & ((1u << bits) - 1);
    word |= v << (bits * j);
  }
  out[i] = (int32_t)word;
}

// ------------------------------------------------------------------------
// host-side dispatch
// ------------------------------------------------------------------------
static int n_groups(const CastParams& p) {
  const QArgs& a = p.a;
  switch (a.strategy) {
    case LLMC_STRAT_TENSOR: return 1;
    case LLMC_STRAT_CHANNEL: return (int)p.rows;
    case LLMC_STRAT_BLOCK: return (int)(((p.rows + a.bh - 1) / a.bh) * ((p.cols + a.bw - 1) / a.bw));
    default: return (int)(p.rows * (p.cols / a.group));
  }
}

static int validate(const CastParams& p) {
  const QArgs& a = p.a;
  if ((!p.w && p.rows * p.cols > 0) || p.rows < 0 || p.cols < 0) return LLMC_EINVAL_ARG;
  if (a.bits != 4 && a.bits != 8) return LLMC_ENOSUPPORT;
  if (a.strategy < 0 || a.strategy > LLMC_STRAT_BLOCK) return LLMC_EINVAL_ARG;
  if (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) {
    if (a.group <= 0) return LLMC_EINVAL_ARG;
    if (p.cols % a.group) return LLMC_EINVAL_SHAPE;  // strategy_cdiv(strict=True)
  }
  if (a.strategy == LLMC_STRAT_BLOCK && (a.bh <= 0 || a.bw <= 0)) return LLMC_EINVAL_ARG;
  if (a.is_float && !a.symmetric && a.bits == 4) return LLMC_ENOSUPPORT;  // asymmetric FP4
  if (p.mode != MODE_STATS) {
    // a packed word must not straddle two parameter groups
    int pf = (p.fmt == LLMC_FMT_PACK_INT32) ? 32 / a.bits : (p.fmt == LLMC_FMT_NVFP4 || p.fmt == LLMC_FMT_MXFP4) ? 2 : 1;
    if ((a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) && (a.group % pf)) return LLMC_ENOSUPPORT;
    if (a.strategy == LLMC_STRAT_BLOCK && (a.bw % pf) && a.bw < p.cols) return LLMC_ENOSUPPORT;
  }
  return LLMC_OK;
}

template <int FMT, int BITS, int MODE>
static bool launch_stream(const CastParams& p, int64_t group, cudaStream_t st) {
  const int64_t steps = (p.rows * p.cols + 1023) / 1024;
  const auto grid = [&](int ctas) { return dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>((steps + 7) / 8, 148 * ctas))); };
  const dim3 b(256);
  constexpr bool fp4 = (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4);
  constexpr int NS = 2;
  // two-warp CTAs: more warps per SM than 256-thread CTAs at the register
  // counts of these kernels (single NVFP4 4.54 -> 4.72 TB/s, FP8 channel rows 6.23 -> 6.75)
  const dim3 sg((unsigned)std::max<int64_t>(1, (steps + 2 * NS - 1) / (2 * NS)));
  if (fp4 && group == 16) k_spans<FMT, BITS, 16, MODE, NS><<<sg, 64, 0, st>>>(p);
  else if (fp4 && group == 32) k_spans<FMT, BITS, 32, MODE, NS><<<sg, 64, 0, st>>>(p);
  else if (group == 16) k_stream<FMT, BITS, 16, MODE><<<grid(stream_ctas<16, MODE>()), b, 0, st>>>(p);
  else if (group == 32) k_stream<FMT, BITS, 32, MODE><<<grid(stream_ctas<32, MODE>()), b, 0, st>>>(p);
  else if constexpr (fp4) return false;
  else if (group == 64) k_stream<FMT, BITS, 64, MODE><<<grid(stream_ctas<64, MODE>()), b, 0, st>>>(p);
  else if (group == 128) k_stream<FMT, BITS, 128, MODE><<<grid(stream_ctas<128, MODE>()), b, 0, st>>>(p);
  else return false;
  llmc::note_launch();
  return true;
}

template <int FMT, int BITS, int MODE>
static bool launch_tile(const CastParams& p, int64_t pieces, cudaStream_t st) {
  if constexpr (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) {
    return false;  // FP4 formats only come with group strategies
  } else {
    const int64_t ng = n_groups(p);
    if (ng <= 0) return true;
    if (p.a.strategy == LLMC_STRAT_CHANNEL && pieces <= 256) {
      const unsigned blocks = (unsigned)((p.rows * 32 + 63) / 64);  // two-warp CTAs
      if (pieces <= 32) k_rowwarp<FMT, BITS, MODE, 1><<<blocks, 64, 0, st>>>(p);
      else if (pieces <= 64) k_rowwarp<FMT, BITS, MODE, 2><<<blocks, 64, 0, st>>>(p);
      else if (pieces <= 128) k_rowwarp<FMT, BITS, MODE, 4><<<blocks, 64, 0, st>>>(p);
      else k_rowwarp<FMT, BITS, MODE, 8><<<blocks, 64, 0, st>>>(p);
      llmc::note_launch();
      return true;
    }
    const unsigned pg = (unsigned)std::min<int64_t>(ng, 148 * 2);
    if (p.a.strategy == LLMC_STRAT_BLOCK && pieces > 512 && pieces <= 1024)
      k_tile<FMT, BITS, MODE, 8, false, 128><<<(unsigned)std::min<int64_t>(ng, 148 * 16), 128, 0, st>>>(p, ng);
    else if (pieces <= 256) k_tile<FMT, BITS, MODE, 1, true><<<pg, 256, 0, st>>>(p, ng);
    // groups of 257..1024 pieces (rows of 4097..16384 values): 128-thread CTAs
    // holding the group in registers, several CTAs (groups in flight) per SM
    else if (pieces <= 512)
      k_tile<FMT, BITS, MODE, 4, false, 128><<<(unsigned)std::min<int64_t>(ng, 148 * 16), 128, 0, st>>>(p, ng);
    else if (pieces <= 1024)
      k_tile<FMT, BITS, MODE, 8, false, 128><<<(unsigned)std::min<int64_t>(ng, 148 * 16), 128, 0, st>>>(p, ng);
    else if (pieces <= 2048) k_tile<FMT, BITS, MODE, 8, false><<<(unsigned)std::min<int64_t>(ng, 148 * 16), 256, 0, st>>>(p, ng);
    else return false;
  }
  llmc::note_launch();
  return true;
}

// The register-resident kernels (k_stream, k_tile) when the shape and the
// pointers allow them; false leaves the launch to the general kernels.
template <int FMT, int BITS>
static bool launch_fast(const CastParams& p, cudaStream_t st) {
  const QArgs& a = p.a;
  const int64_t n = p.rows * p.cols;
  constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
  if ((uintptr_t)p.w % 32) return false;
  if (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) {
    if (n % 32) return false;
    if (p.mode == MODE_STATS) return launch_stream<LLMC_FMT_INT8, 8, MODE_STATS>(p, a.group, st);
    if ((uintptr_t)p.out % (OUT4 ? 16 : 32)) return false;
    if (p.mode == MODE_FUSED) return launch_stream<FMT, BITS, MODE_FUSED>(p, a.group, st);
    return launch_stream<FMT, BITS, MODE_GIVEN>(p, a.group, st);
  }
  if (a.strategy == LLMC_STRAT_TENSOR) {
    if constexpr (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) {
      return false;
    } else {
      const int64_t steps = (n + 1023) / 1024;
      dim3 g((unsigned)std::max<int64_t>(1, std::min<int64_t>((steps + 7) / 8, 148 * 3))), b(256);
      if (p.mode == MODE_GIVEN) {  // stored scale: quantize only
        if (n % 32 || (uintptr_t)p.out % (OUT4 ? 16 : 32)) return false;
        k_stream<FMT, BITS, 0, MODE_GIVEN><<<g, b, 0, st>>>(p); llmc::note_launch();
        return true;
      }
      // FUSED / STATS: grid-wide statistics first
      const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((n / 16 + 255) / 256, 148 * 4));
      uint16_t *smin, *smax;
      if (p.mode == MODE_STATS) {
        smin = p.min_out; smax = p.max_out;
      } else {
        // the first 4 bytes of the packed output hold the two slots until
        // the quantize pass overwrites them
        if (n % 32 || (uintptr_t)p.out % (OUT4 ? 16 : 32) || n * (OUT4 ? 4 : 8) < 32) return false;
        smin = (uint16_t*)p.out; smax = smin + 1;
      }
      if (cudaMemsetAsync(smin, 0xFF, 2, st) != cudaSuccess || cudaMemsetAsync(smax, 0x00, 2, st) != cudaSuccess)
        return false;
      k_tensor_minmax<<<(unsigned)blocks, 256, 0, st>>>(p.w, n, smin, smax); llmc::note_launch();
      k_tensor_finish<FMT><<<1, 1, 0, st>>>(p, smin, smax); llmc::note_launch();
      if (p.mode == MODE_STATS) return true;
      CastParams q = p;  // FUSED: quantize with the qparams just stored
      q.mode = MODE_GIVEN;
      q.scale_in = p.scale_out;
      q.scale_in_f32 = 0;
      q.zp_in = p.zp_out;
      k_stream<FMT, BITS, 0, MODE_GIVEN><<<g, b, 0, st>>>(q); llmc::note_launch();
      return true;
    }
  }
  if (a.strategy == LLMC_STRAT_CHANNEL || a.strategy == LLMC_STRAT_BLOCK) {
    if (p.cols % 16) return false;
    int64_t pieces = p.cols / 16;
    if (a.strategy == LLMC_STRAT_BLOCK) {
      if (a.bw % 16) return false;
      pieces = std::min<int64_t>(a.bh, p.rows) * (std::min<int64_t>(a.bw, p.cols) / 16);
    }
    if constexpr (FMT != LLMC_FMT_NVFP4 && FMT != LLMC_FMT_MXFP4) {
      if (tma_block_ok(p)) {
        if (p.mode == MODE_STATS) return launch_block_tma_one<LLMC_FMT_INT8, 8, MODE_STATS>(p, st);
        if (p.mode == MODE_FUSED) return launch_block_tma_one<FMT, BITS, MODE_FUSED>(p, st);
        return launch_block_tma_one<FMT, BITS, MODE_GIVEN>(p, st);
      }
    }
    if (p.mode == MODE_STATS) return launch_tile<LLMC_FMT_INT8, 8, MODE_STATS>(p, pieces, st);
    if ((uintptr_t)p.out % 16) return false;
    if (p.mode == MODE_FUSED) return launch_tile<FMT, BITS, MODE_FUSED>(p, pieces, st);
    return launch_tile<FMT, BITS, MODE_GIVEN>(p, pieces, st);
  }
  return false;
}

template <int FMT>
static int launch_fmt(const CastParams& p, cudaStream_t st) {
  const QArgs& a = p.a;
  if (p.rows * p.cols == 0) return LLMC_OK;
  bool fast = (FMT == LLMC_FMT_PACK_INT32 && a.bits == 4) ? launch_fast<FMT, 4>(p, st) : launch_fast<FMT, 8>(p, st);
  if (fast) return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  bool grp = (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP);
  int64_t tpg = grp ? a.group / 8 : 0;
  bool pow2 = grp && (a.group % 8 == 0) && tpg >= 1 && tpg <= 32 && ((tpg & (tpg - 1)) == 0);
  if (FMT == LLMC_FMT_PACK_INT32 && grp && (a.group * a.bits) % 32) pow2 = false;
  if (p.rows * p.cols == 0) return LLMC_OK;
  if (pow2) {
    int64_t chunks = p.rows * p.cols / 8;
    int64_t blocks = std::min<int64_t>((chunks + 256 * VEC_UNROLL - 1) / (256 * VEC_UNROLL), 148 * 16);
    dim3 g((unsigned)std::max<int64_t>(blocks, 1)), b(256);
    switch (tpg) {
      case 1: k_group_vec<FMT, 1><<<g, b, 0, st>>>(p); llmc::note_launch(); break;
      case 2: k_group_vec<FMT, 2><<<g, b, 0, st>>>(p); llmc::note_launch(); break;
      case 4: k_group_vec<FMT, 4><<<g, b, 0, st>>>(p); llmc::note_launch(); break;
      case 8: k_group_vec<FMT, 8><<<g, b, 0, st>>>(p); llmc::note_launch(); break;
      case 16: k_group_vec<FMT, 16><<<g, b, 0, st>>>(p); llmc::note_launch(); break;
      default: k_group_vec<FMT, 32><<<g, b, 0, st>>>(p); llmc::note_launch(); break;
    }
  } else {
    int ng = n_groups(p);
    if (ng > 0) { k_paramgroup<FMT><<<ng, 256, 0, st>>>(p); llmc::note_launch(); }
  }
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

static int launch(const CastParams& p, cudaStream_t st) {
  switch (p.fmt) {
    case LLMC_FMT_PACK_INT32: return launch_fmt<LLMC_FMT_PACK_INT32>(p, st);
    case LLMC_FMT_FP8: return launch_fmt<LLMC_FMT_FP8>(p, st);
    case LLMC_FMT_NVFP4: return launch_fmt<LLMC_FMT_NVFP4>(p, st);
    case LLMC_FMT_MXFP4: return launch_fmt<LLMC_FMT_MXFP4>(p, st);
    case LLMC_FMT_INT8: return launch_fmt<LLMC_FMT_INT8>(p, st);
    default: return LLMC_EINVAL_ARG;
  }
}

// One batched launch for jobs[0..n) that all meet the fast kernels' shape
// and alignment rules (the caller checked); false if the strategy has no
// batched kernel.
template <int FMT, int BITS>
static bool launch_batch_fmt(CastBatch& b, cudaStream_t st) {
  const QArgs& a = b.base.a;
  int64_t units = 0;
  int64_t pieces = 0;
  for (int i = 0; i < b.njobs; ++i) {
    CastJob& j = b.job[i];
    j.first = units;
    if (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) {
      // rebased pointers for k_stream_batch (integer arithmetic on the
      // addresses; a rebased pointer is only dereferenced at or past the
      // job's own start)
      constexpr bool OUT4 = OutOf<FMT, BITS>::OUT4;
      constexpr int64_t SCALE_BYTES = (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) ? 1 : 2;
      const int64_t off = units * 1024, goff = a.group > 0 ? off / a.group : 0;
      j.w_rb = (const uint16_t*)((uintptr_t)j.w - (uintptr_t)(off * 2));
      j.out_rb = (void*)((uintptr_t)j.out - (uintptr_t)(OUT4 ? off / 2 : off));
      j.scale_rb = (void*)((uintptr_t)j.scale_out - (uintptr_t)(goff * SCALE_BYTES));
      j.zp_rb = j.zp_out ? (int8_t*)((uintptr_t)j.zp_out - (uintptr_t)goff) : nullptr;
      j.lim = off + j.rows * j.cols;
      units += (j.rows * j.cols + 1023) / 1024;
    } else {
      CastParams p = b.base;
      p.rows = j.rows; p.cols = j.cols;
      units += n_groups(p);
      const int64_t pc = a.strategy == LLMC_STRAT_CHANNEL ? j.cols / 16
                                                           : std::min<int64_t>(a.bh, j.rows) * (std::min<int64_t>(a.bw, j.cols) / 16);
      pieces = std::max(pieces, pc);
    }
  }
  b.units = units;
  if (units == 0) return true;
  if constexpr (!(FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4)) {
    if ((a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) && (a.group == 64 || a.group == 128)) {
      int64_t groups = 0;  // units are groups, one lane each (k_lanegroup_batch)
      for (int i = 0; i < b.njobs; ++i) { b.job[i].first = groups; groups += b.job[i].rows * b.job[i].cols / a.group; }
      b.units = groups;
      // two-warp CTAs: at 104 registers a thread, 256-thread CTAs leave the
      // SM at 16 warps (two CTAs), 64-thread CTAs fit 18 (4.80 -> 5.75 TB/s)
      const dim3 lg((unsigned)std::max<int64_t>(1, (groups + 63) / 64));
      if (a.group == 64) k_lanegroup_batch<FMT, BITS, 64><<<lg, 64, 0, st>>>(b);
      else k_lanegroup_batch<FMT, BITS, 128><<<lg, 64, 0, st>>>(b);
      llmc::note_launch();
      return true;
    }
  }
  if (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) {
    const auto grid = [&](int ctas) { return dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>((units + 7) / 8, 148 * ctas))); };
    const dim3 bl(256);
    const int64_t group = a.group;
    if (group == 16) k_stream_batch<FMT, BITS, 16><<<grid(stream_ctas<16, MODE_FUSED>()), bl, 0, st>>>(b);
    else if (group == 32) k_stream_batch<FMT, BITS, 32><<<grid(stream_ctas<32, MODE_FUSED>()), bl, 0, st>>>(b);
    else return false;  // 64 / 128: k_lanegroup_batch above
    llmc::note_launch();
    return true;
  }
  if constexpr (FMT == LLMC_FMT_NVFP4 || FMT == LLMC_FMT_MXFP4) {
    return false;
  } else {
    if (a.strategy != LLMC_STRAT_CHANNEL && a.strategy != LLMC_STRAT_BLOCK) return false;
    if (a.strategy == LLMC_STRAT_BLOCK && b.njobs <= kTmaJobsMax) {
      bool all = true;
      for (int i = 0; i < b.njobs && all; ++i) {
        CastParams p = b.base;  // the job's parameters, built on the host
        const CastJob& jb = b.job[i];
        p.w = jb.w; p.rows = jb.rows; p.cols = jb.cols; p.gs = jb.gs;
        p.out = jb.out; p.scale_out = jb.scale_out; p.zp_out = jb.zp_out;
        all = tma_block_ok(p);
      }
      if (all) return launch_block_tma<FMT, BITS, MODE_FUSED>(b, st);
    }
    if (a.strategy == LLMC_STRAT_CHANNEL && pieces <= 256) {
      // two-warp CTAs (as k_lanegroup_batch: more warps per SM at ~96
      // registers a thread; FP8 channel 5.80 -> 6.80 TB/s)
      const unsigned blocks = (unsigned)((units * 32 + 63) / 64);
      if (pieces <= 32) k_rowwarp_batch<FMT, BITS, 1><<<blocks, 64, 0, st>>>(b);
      else if (pieces <= 64) k_rowwarp_batch<FMT, BITS, 2><<<blocks, 64, 0, st>>>(b);
      else if (pieces <= 128) k_rowwarp_batch<FMT, BITS, 4><<<blocks, 64, 0, st>>>(b);
      else k_rowwarp_batch<FMT, BITS, 8><<<blocks, 64, 0, st>>>(b);
      llmc::note_launch();
      return true;
    }
    const unsigned g = (unsigned)std::min<int64_t>(units, 148 * 2);
    const unsigned g128 = (unsigned)std::min<int64_t>(units, 148 * 16);
    if (pieces <= 256) k_tile_batch<FMT, BITS, 1><<<g, 256, 0, st>>>(b);
    else if (pieces <= 512) k_tile_batch128<FMT, BITS, 4><<<g128, 128, 0, st>>>(b);
    else if (pieces <= 1024) k_tile_batch128<FMT, BITS, 8><<<g128, 128, 0, st>>>(b);
    else return false;
    llmc::note_launch();
    return true;
  }
}

static bool launch_batch(CastBatch& b, cudaStream_t st) {
  const bool b4 = b.base.a.bits == 4;
  switch (b.base.fmt) {
    case LLMC_FMT_PACK_INT32: return b4 ? launch_batch_fmt<LLMC_FMT_PACK_INT32, 4>(b, st) : launch_batch_fmt<LLMC_FMT_PACK_INT32, 8>(b, st);
    case LLMC_FMT_FP8: return launch_batch_fmt<LLMC_FMT_FP8, 8>(b, st);
    case LLMC_FMT_NVFP4: return launch_batch_fmt<LLMC_FMT_NVFP4, 8>(b, st);
    case LLMC_FMT_MXFP4: return launch_batch_fmt<LLMC_FMT_MXFP4, 8>(b, st);
    case LLMC_FMT_INT8: return launch_batch_fmt<LLMC_FMT_INT8, 8>(b, st);
    default: return false;
  }
}

// Whether one model-free job can ride in a batched launch.
static bool batchable(const CastParams& p) {
  const QArgs& a = p.a;
  const bool out4 = (p.fmt == LLMC_FMT_NVFP4 || p.fmt == LLMC_FMT_MXFP4 || (p.fmt == LLMC_FMT_PACK_INT32 && a.bits == 4));
  if ((uintptr_t)p.w % 32 || p.rows * p.cols == 0) return false;
  if (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) {
    if ((p.rows * p.cols) % 32) return false;
    if (a.group != 16 && a.group != 32 && a.group != 64 && a.group != 128) return false;
    return (uintptr_t)p.out % (out4 ? 16 : 32) == 0;
  }
  if (a.strategy == LLMC_STRAT_CHANNEL || a.strategy == LLMC_STRAT_BLOCK) {
    if (p.cols % 16 || (uintptr_t)p.out % 16) return false;
    if (a.strategy == LLMC_STRAT_BLOCK && a.bw % 16) return false;
    const int64_t pc = a.strategy == LLMC_STRAT_CHANNEL ? p.cols / 16
                                                         : std::min<int64_t>(a.bh, p.rows) * (std::min<int64_t>(a.bw, p.cols) / 16);
    return pc <= 1024;
  }
  return false;
}

static int check_fmt(const QArgs& a, int fmt) {
  switch (fmt) {
    case LLMC_FMT_PACK_INT32:
    case LLMC_FMT_INT8: return a.is_float ? LLMC_EINVAL_DTYPE : LLMC_OK;
    case LLMC_FMT_FP8: return (a.is_float && a.bits == 8) ? LLMC_OK : LLMC_EINVAL_DTYPE;
    case LLMC_FMT_NVFP4: return (a.is_float && a.bits == 4 && a.strategy == LLMC_STRAT_TENSOR_GROUP) ? LLMC_OK : LLMC_EINVAL_DTYPE;
    case LLMC_FMT_MXFP4: return (a.is_float && a.bits == 4 && a.is_mx()) ? LLMC_OK : LLMC_EINVAL_DTYPE;
    default: return LLMC_EINVAL_ARG;
  }
}

}  // namespace llmc

using namespace llmc;

namespace llmc {
static thread_local char g_last_error[256] = "";
int cuda_fail(const char* where, int e) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%d)", where, cudaGetErrorString((cudaError_t)e), e);
  return LLMC_ECUDA;
}
}  // namespace llmc

extern "C" {

int llmc_version(void) { return 100; }

const char* llmc_last_cuda_error(void) { return llmc::g_last_error; }

int llmc_device_status(int clear, int* status) {
  if (!status) return LLMC_EINVAL_ARG;
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, llmc::g_async_status, sizeof(int));
  if (e != cudaSuccess) return llmc::cuda_fail("llmc_device_status: cudaMemcpyFromSymbol", e);
  if (clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(llmc::g_async_status, &zero, sizeof(int));
    if (e != cudaSuccess) return llmc::cuda_fail("llmc_device_status: cudaMemcpyToSymbol", e);
  }
  *status = v;
  return LLMC_OK;
}

int64_t llmc_kernel_launches(void) { return (int64_t)g_launches.load(std::memory_order_relaxed); }

const char* llmc_status_string(int s) {
  switch (s) {
    case LLMC_OK: return "ok";
    case LLMC_EINVAL_SHAPE: return "invalid shape";
    case LLMC_EINVAL_DTYPE: return "invalid dtype";
    case LLMC_ENOT_PD: return "matrix not positive definite";
    case LLMC_ETIMEOUT: return "device wait timed out";
    case LLMC_ECUDA: return "CUDA error";
    case LLMC_EINVAL_ARG: return "invalid argument";
    case LLMC_ENOSUPPORT: return "not supported";
    default: return "unknown status";
  }
}

int llmc_observe_minmax(const void* w, int64_t rows, int64_t cols, const LlmcQuantArgs* args, void* mn, void* mx,
                        void* stream) {
  if (!args || !mn || !mx) return LLMC_EINVAL_ARG;
  CastParams p = {};
  p.w = (const uint16_t*)w; p.rows = rows; p.cols = cols; p.a = to_qargs(*args);
  p.mode = MODE_STATS; p.fmt = LLMC_FMT_INT8;
  p.min_out = (uint16_t*)mn; p.max_out = (uint16_t*)mx;
  int v = validate(p);
  if (v) return v;
  return launch_fmt<LLMC_FMT_INT8>(p, (cudaStream_t)stream);
}

int llmc_absmax_accumulate(const void* w, int64_t n, float* absmax, void* stream) {
  if (!w || !absmax || n < 0) return LLMC_EINVAL_ARG;
  if (n == 0) return LLMC_OK;
  int64_t blocks = std::min<int64_t>((n / 8 + 255) / 256 + 1, 148 * 8);
  k_absmax<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>((const uint16_t*)w, n, absmax); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_global_scale(const float* absmax, float* gs, void* stream) {
  if (!absmax || !gs) return LLMC_EINVAL_ARG;
  k_global_scale<<<1, 1, 0, (cudaStream_t)stream>>>(absmax, gs); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_calculate_qparams_ex(const void* mn, const void* mx, int64_t n, const LlmcQuantArgs* args, const float* gs,
                              int f32stats, void* scale_out, void* zp_out, void* stream) {
  if (!mn || !mx || !args || !scale_out || n < 0) return LLMC_EINVAL_ARG;
  QArgs a = to_qargs(*args);
  if (a.is_float && !a.symmetric && a.bits == 4) return LLMC_ENOSUPPORT;
  if (f32stats && a.is_mx()) return LLMC_ENOSUPPORT;  // MX exponents are taken from bf16 bit patterns
  if (n == 0) return LLMC_OK;
  k_qparams<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const uint16_t*)mn, (const uint16_t*)mx,
                                                                            n, a, gs, scale_out, zp_out, f32stats);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_calculate_qparams(const void* mn, const void* mx, int64_t n, const LlmcQuantArgs* args, const float* gs,
                           void* scale_out, void* zp_out, void* stream) {
  return llmc_calculate_qparams_ex(mn, mx, n, args, gs, 0, scale_out, zp_out, stream);
}

int llmc_quantize_pack(const void* w, int64_t rows, int64_t cols, const LlmcQuantArgs* args, const void* scale,
                       int scale_is_f32, const void* zp, const float* gs, int fmt, void* out, void* stream) {
  if (!args || ((!scale || !out) && rows * cols > 0)) return LLMC_EINVAL_ARG;
  CastParams p = {};
  p.w = (const uint16_t*)w; p.rows = rows; p.cols = cols; p.a = to_qargs(*args);
  p.mode = MODE_GIVEN; p.fmt = fmt; p.scale_in = scale; p.scale_in_f32 = scale_is_f32;
  p.zp_in = (const int8_t*)zp; p.gs = gs; p.out = out;
  int v = validate(p);
  if (v) return v;
  if ((v = check_fmt(p.a, fmt))) return v;
  if (fmt == LLMC_FMT_NVFP4 && !gs) return LLMC_EINVAL_ARG;
  if ((fmt == LLMC_FMT_NVFP4 || fmt == LLMC_FMT_MXFP4) && (cols & 1)) return LLMC_EINVAL_SHAPE;
  return launch(p, (cudaStream_t)stream);
}

int llmc_modelfree_quantize(const void* w, int64_t rows, int64_t cols, const LlmcQuantArgs* args, const float* gs,
                            int fmt, void* out, void* scale_out, void* zp_out, void* stream) {
  if (!args || ((!out || !scale_out) && rows * cols > 0)) return LLMC_EINVAL_ARG;
  CastParams p = {};
  p.w = (const uint16_t*)w; p.rows = rows; p.cols = cols; p.a = to_qargs(*args);
  p.mode = MODE_FUSED; p.fmt = fmt; p.gs = gs; p.out = out; p.scale_out = scale_out;
  p.zp_out = p.a.symmetric ? nullptr : (int8_t*)zp_out;
  int v = validate(p);
  if (v) return v;
  if ((v = check_fmt(p.a, fmt))) return v;
  if (fmt == LLMC_FMT_NVFP4 && !gs) return LLMC_EINVAL_ARG;
  if (!p.a.symmetric && !zp_out && rows * cols > 0) return LLMC_EINVAL_ARG;
  if ((fmt == LLMC_FMT_NVFP4 || fmt == LLMC_FMT_MXFP4) && (cols & 1)) return LLMC_EINVAL_SHAPE;
  return launch(p, (cudaStream_t)stream);
}

int llmc_modelfree_quantize_batch(const LlmcCastJob* jobs, int njobs, const LlmcQuantArgs* args, int fmt,
                                  void* stream) {
  if (!args || njobs < 0 || (njobs > 0 && !jobs)) return LLMC_EINVAL_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  CastBatch b;
  memset(&b, 0, sizeof(b));
  b.base.a = to_qargs(*args);
  b.base.mode = MODE_FUSED;
  b.base.fmt = fmt;
  if (int v = check_fmt(b.base.a, fmt)) return v;
  CastBatch br;
  memcpy(&br, &b, sizeof(b));
  for (int i = 0; i < njobs; ++i) {
    const LlmcCastJob& j = jobs[i];
    CastParams p = b.base;
    p.w = (const uint16_t*)j.w; p.rows = j.rows; p.cols = j.cols; p.gs = j.global_scale;
    p.out = j.out; p.scale_out = j.scale_out; p.zp_out = p.a.symmetric ? nullptr : (int8_t*)j.zp_out;
    if (int v = validate(p)) return v;
    if ((!p.out || !p.scale_out) && p.rows * p.cols > 0) return LLMC_EINVAL_ARG;
    if (fmt == LLMC_FMT_NVFP4 && !p.gs) return LLMC_EINVAL_ARG;
    if (!p.a.symmetric && !j.zp_out && p.rows * p.cols > 0) return LLMC_EINVAL_ARG;
    if ((fmt == LLMC_FMT_NVFP4 || fmt == LLMC_FMT_MXFP4) && (p.cols & 1)) return LLMC_EINVAL_SHAPE;
    if (!batchable(p)) {  // odd shape or alignment: its own launch
      if (int v = launch(p, st)) return v;
      continue;
    }
    // CHANNEL rows of up to 4096 values go to their own batch (one warp per row)
    CastBatch& t = (p.a.strategy == LLMC_STRAT_CHANNEL && p.cols <= 4096) ? br : b;
    CastJob& q = t.job[t.njobs++];
    q.w = p.w; q.rows = p.rows; q.cols = p.cols; q.gs = p.gs;
    q.out = p.out; q.scale_out = p.scale_out; q.zp_out = p.zp_out;
    if (t.njobs == kBatchMax) {
      if (!launch_batch(t, st)) return LLMC_ENOSUPPORT;
      t.njobs = 0;
    }
  }
  if (b.njobs > 0 && !launch_batch(b, st)) return LLMC_ENOSUPPORT;
  if (br.njobs > 0 && !launch_batch(br, st)) return LLMC_ENOSUPPORT;
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_pack_int4_to_int8(const int8_t* in, int64_t rows, int64_t cols, int8_t* out, void* stream) {
  if (rows < 0 || cols < 0 || ((!in || !out) && rows * cols > 0)) return LLMC_EINVAL_ARG;
  if (cols % 2) return LLMC_EINVAL_SHAPE;
  if (rows * cols == 0) return LLMC_OK;
  const int vec = (cols % 32 == 0) && ((uintptr_t)in % 16 == 0) && ((uintptr_t)out % 16 == 0);
  const int64_t work = vec ? rows * cols / 32 : rows * cols / 2;
  const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 148 * 8));
  k_pack_int4_int8<<<blocks, 256, 0, (cudaStream_t)stream>>>(in, rows, cols, out, vec); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_pack_zero_point(const int8_t* zp, int64_t rows, int64_t groups, int bits, int32_t* out, void* stream) {
  if (!zp || !out || (bits != 4 && bits != 8)) return LLMC_EINVAL_ARG;
  int64_t n = ((rows + 32 / bits - 1) / (32 / bits)) * groups;
  if (n == 0) return LLMC_OK;
  k_pack_zp<<<(unsigned)((n + 255) / 256), 256, 0, (cudaStream_t)stream>>>(zp, rows, groups, bits, out); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

}  // extern "C"
