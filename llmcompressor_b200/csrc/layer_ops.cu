// Fused elementwise parts of a Llama-family decoder layer for the calibration
// pipeline's forward passes (the GEMMs stay cuBLAS, attention stays cuDNN).
// In the reference's pipeline these run as HF eager torch ops -- about a
// third of a layer step's kernel time on the Llama-3-8B shape, each op a
// full pass over the activations.  Same roundings as those ops:
//
//  * RMSNorm (LlamaRMSNorm.forward): h = x (or bf16(residual + x)), float32
//    mean of h^2 (sum times 1/cols), r = rsqrt(mean + eps), y = bf16(h * r),
//    out = bf16(w * y).
//    The mean's summation order differs from torch's reduction (float32, so
//    y can differ by one bf16 unit in rare rows); everything else is the
//    same sequence of roundings.
//  * rotary (apply_rotary_pos_emb): out = bf16(bf16(x * cos) +
//    bf16(rotate_half(x) * sin)), rotate_half(x) = cat(-x[D/2:], x[:D/2]):
//    every product and the sum round once, as in torch -- bit-identical.
//  * SiLU * up (LlamaMLP): bf16(bf16(g / (1 + expf(-g))) * up).
//
// All are memory-bound: one read of each input and one write per output,
// 16-byte vector accesses.
#include "llmc_common.cuh"

#include <algorithm>

namespace llmc {
namespace layer {

__device__ __forceinline__ float lo_f(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  return (uint32_t)f_to_bf16(lo) | ((uint32_t)f_to_bf16(hi) << 16);
}

// bf16(silu(x)) = bf16(x / (1 + expf(-x))) for a bf16 value x, as the eager
// op rounds it (float32 quotient, then bf16).  The quotient comes from the
// approximate reciprocal (rcp.approx.f32, within one unit in the last place)
// times x, within a few float32 units of the correctly rounded quotient; its bf16 rounding can differ from that of the correctly
// rounded quotient only where the quotient lies within those few units of a
// bf16 rounding midpoint (low 16 bits near 0x8000) -- there the IEEE
// division decides.  Zeros, infinities and NaNs come out as the division's.
__device__ __forceinline__ float silu_bf16(float x) {
  const float d = 1.0f + expf(-x);
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(d));
  const float q = x * r;
  if ((__float_as_uint(q) & 0xFFFFu) - 0x7FF8u < 16u) return rbf(__fdiv_rn(x, d));
  return rbf(q);
}

// RMSNorm over rows of `cols` values (cols % 8 == 0); TPR threads per row
// (a power of two <= 32; several rows per warp when TPR < 32).  With a
// residual: h = bf16(residual + x) is written to res_out and normalised.
template <int TPR>
__global__ void __launch_bounds__(256) k_rmsnorm(const uint4* __restrict__ x, const uint4* __restrict__ res,
                                                 int64_t rows, int64_t cols, const uint4* __restrict__ w, float eps,
                                                 uint4* __restrict__ out, uint4* __restrict__ res_out) {
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = gt / TPR;
  const int sub = (int)(gt % TPR);
  const bool valid = row < rows;
  const int64_t cw = cols / 8;  // 16-byte chunks per row
  const int64_t base = valid ? row * cw : 0;
  float ss = 0.f;
  if (valid) {
    for (int64_t c = sub; c < cw; c += TPR) {
      uint4 v = x[base + c];
      if (res) {
        const uint4 r = res[base + c];
        v.x = pack_bf2(lo_f(r.x) + lo_f(v.x), hi_f(r.x) + hi_f(v.x));
        v.y = pack_bf2(lo_f(r.y) + lo_f(v.y), hi_f(r.y) + hi_f(v.y));
        v.z = pack_bf2(lo_f(r.z) + lo_f(v.z), hi_f(r.z) + hi_f(v.z));
        v.w = pack_bf2(lo_f(r.w) + lo_f(v.w), hi_f(r.w) + hi_f(v.w));
        res_out[base + c] = v;
      }
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float a = lo_f(u[k]), b = hi_f(u[k]);
        ss += __fmul_rn(a, a);
        ss += __fmul_rn(b, b);
      }
    }
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o, TPR);
  if (!valid) return;
  const float r = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / (float)cols), eps));
  const uint4* src = res ? res_out : x;
  for (int64_t c = sub; c < cw; c += TPR) {
    const uint4 v = src[base + c];
    const uint4 wv = w[c];
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float ylo = bf16_to_f(f_to_bf16(lo_f(u[k]) * r)), yhi = bf16_to_f(f_to_bf16(hi_f(u[k]) * r));
      o[k] = pack_bf2(lo_f(ww[k]) * ylo, hi_f(ww[k]) * yhi);
    }
    out[base + c] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Rotary embedding of x (batch, heads, seq, D) given by element strides
// (sb, sh, ss; unit stride inside a head) into out, laid out (batch, seq,
// heads, D) contiguous -- the memory order torch gives the eager result for
// the transposed projection views.  cos / sin rows: (batch or 1, seq, D)
// with batch stride cb (0 when shared) and seq stride D.  One thread per 8
// values of the first half of a head (it also produces the matching 8 of the
// second half).
__global__ void __launch_bounds__(256) k_rotary(const uint16_t* __restrict__ x, int64_t S, int64_t heads, int64_t D,
                                                int64_t sb, int64_t sh, int64_t ss, const uint16_t* __restrict__ cs,
                                                const uint16_t* __restrict__ sn, int64_t cb, int64_t total,
                                                uint16_t* __restrict__ out) {
  const int64_t half = D / 2, per_head = half / 8;
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gt >= total) return;
  const int64_t j = (gt % per_head) * 8;
  int64_t r = gt / per_head;
  const int64_t h = r % heads;
  r /= heads;
  const int64_t s = r % S, b = r / S;
  const uint16_t* xr = x + b * sb + s * ss + h * sh;
  const int64_t crow = b * cb + s * D;
  const uint4 a = *(const uint4*)(xr + j);          // x[j .. j+8)
  const uint4 bb = *(const uint4*)(xr + half + j);  // x[D/2 + j .. )
  const uint4 c0 = *(const uint4*)(cs + crow + j), c1 = *(const uint4*)(cs + crow + half + j);
  const uint4 s0 = *(const uint4*)(sn + crow + j), s1 = *(const uint4*)(sn + crow + half + j);
  const uint32_t A[4] = {a.x, a.y, a.z, a.w}, B[4] = {bb.x, bb.y, bb.z, bb.w};
  const uint32_t C0[4] = {c0.x, c0.y, c0.z, c0.w}, C1[4] = {c1.x, c1.y, c1.z, c1.w};
  const uint32_t S0[4] = {s0.x, s0.y, s0.z, s0.w}, S1[4] = {s1.x, s1.y, s1.z, s1.w};
  uint32_t O0[4], O1[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    // first half: x * cos + (-x[D/2 + i]) * sin
    const float l0 = rbf(lo_f(A[k]) * lo_f(C0[k])) + rbf(-lo_f(B[k]) * lo_f(S0[k]));
    const float h0 = rbf(hi_f(A[k]) * hi_f(C0[k])) + rbf(-hi_f(B[k]) * hi_f(S0[k]));
    O0[k] = pack_bf2(l0, h0);
    // second half: x * cos + x[i] * sin
    const float l1 = rbf(lo_f(B[k]) * lo_f(C1[k])) + rbf(lo_f(A[k]) * lo_f(S1[k]));
    const float h1 = rbf(hi_f(B[k]) * hi_f(C1[k])) + rbf(hi_f(A[k]) * hi_f(S1[k]));
    O1[k] = pack_bf2(l1, h1);
  }
  uint16_t* orow = out + ((b * S + s) * heads + h) * D;
  *(uint4*)(orow + j) = make_uint4(O0[0], O0[1], O0[2], O0[3]);
  *(uint4*)(orow + half + j) = make_uint4(O1[0], O1[1], O1[2], O1[3]);
}

__global__ void __launch_bounds__(256) k_silu_mul(const uint4* __restrict__ g, const uint4* __restrict__ u,
                                                  int64_t n8, uint4* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint4 a = g[i], b = u[i];
  const uint32_t A[4] = {a.x, a.y, a.z, a.w}, B[4] = {b.x, b.y, b.z, b.w};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float s0 = silu_bf16(lo_f(A[k])), s1 = silu_bf16(hi_f(A[k]));
    o[k] = pack_bf2(s0 * lo_f(B[k]), s1 * hi_f(B[k]));
  }
  out[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

// MoE all-expert combine input: gate / up (rows, E*I) from the stacked
// expert projections; act = bf16(bf16(silu(g)) * u) and / or
// scaled = bf16(act * w[row, e]) with e = column / I and w the float32 dense
// routing weights (rows, E); a zero weight (token not routed to expert e)
// gives an exact zero, as the routed combine leaves that token out.
// Grid: x over a row's 16-byte chunks, y (strided) over rows -- no 64-bit
// divisions per thread.
__global__ void __launch_bounds__(256) k_silu_mul_scaled(const uint4* __restrict__ g, const uint4* __restrict__ u,
                                                         int64_t rows, int cols8, int group8,
                                                         const float* __restrict__ w, int64_t w_ld,
                                                         uint4* __restrict__ out, uint4* __restrict__ outs) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 >= cols8) return;
  const int e = c8 / group8;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const int64_t i = row * cols8 + c8;
    const float s = w ? w[row * w_ld + e] : 1.0f;
    const uint4 a = g[i], b = u[i];
    const uint32_t A[4] = {a.x, a.y, a.z, a.w}, B[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4], os[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float s0 = silu_bf16(lo_f(A[k])), s1 = silu_bf16(hi_f(A[k]));
      const float y0 = rbf(s0 * lo_f(B[k])), y1 = rbf(s1 * hi_f(B[k]));
      o[k] = pack_bf2(y0, y1);
      os[k] = s == 0.0f ? 0u : pack_bf2(y0 * s, y1 * s);
    }
    if (out) out[i] = make_uint4(o[0], o[1], o[2], o[3]);
    if (outs) outs[i] = make_uint4(os[0], os[1], os[2], os[3]);
  }
}

// scaled = bf16(x * w[row, column / group]) (zero weight: exact zero).
__global__ void __launch_bounds__(256) k_scale_groups(const uint4* __restrict__ x, int64_t rows, int cols8,
                                                      int group8, const float* __restrict__ w, int64_t w_ld,
                                                      uint4* __restrict__ out) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 >= cols8) return;
  const int e = c8 / group8;
  for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
    const int64_t i = row * cols8 + c8;
    const float s = w[row * w_ld + e];
    if (s == 0.0f) {
      out[i] = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    const uint4 a = x[i];
    const uint32_t A[4] = {a.x, a.y, a.z, a.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) o[k] = pack_bf2(lo_f(A[k]) * s, hi_f(A[k]) * s);
    out[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Routed MoE combine: out[t] = sum over k of bf16(y[pos[t, k]] * w[t, k]),
// added in k order (the token's experts in increasing index) with a bf16
// rounding after every add, starting from zero -- the per-expert
// ``index_add_`` of weighted bf16 expert outputs into a zero tensor.
// One thread per 8 hidden values of a token.
__global__ void __launch_bounds__(256) k_moe_combine(const uint4* __restrict__ y, int64_t y_rows,
                                                     const int* __restrict__ pos, const float* __restrict__ w,
                                                     int64_t tokens, int K, int h8, uint4* __restrict__ out) {
  const int c8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (c8 >= h8) return;
  for (int64_t t = blockIdx.y; t < tokens; t += gridDim.y) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float s = w[t * K + k];
      const int64_t r = pos[t * K + k];
      if (r < 0 || r >= y_rows) continue;  // not a row of y: contributes nothing
      const uint4 v = y[r * h8 + c8];
      const uint32_t V[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = rbf(acc[2 * j] + rbf(lo_f(V[j]) * s));
        acc[2 * j + 1] = rbf(acc[2 * j + 1] + rbf(hi_f(V[j]) * s));
      }
    }
    out[t * h8 + c8] = make_uint4(pack_bf2(acc[0], acc[1]), pack_bf2(acc[2], acc[3]), pack_bf2(acc[4], acc[5]),
                                  pack_bf2(acc[6], acc[7]));
  }
}

}  // namespace layer
}  // namespace llmc

using namespace llmc;
using namespace llmc::layer;

namespace {
bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }
}  // namespace

extern "C" {

int llmc_rmsnorm_bf16(const void* x, const void* residual, int64_t rows, int64_t cols, const void* weight, float eps,
                      void* out, void* residual_out, void* stream) {
  if (rows < 0 || cols <= 0) return LLMC_EINVAL_ARG;
  if (rows == 0) return LLMC_OK;
  if (!x || !weight || !out || (residual && !residual_out)) return LLMC_EINVAL_ARG;
  if (cols % 8 || !al16(x) || !al16(weight) || !al16(out) || (residual && (!al16(residual) || !al16(residual_out))))
    return LLMC_EINVAL_SHAPE;
  const int64_t cw = cols / 8;
  int tpr = 32;
  while (tpr > 1 && tpr / 2 >= cw) tpr /= 2;  // threads per row: no more than the row's 16-byte chunks
  const int64_t threads = rows * tpr;
  const unsigned grid = (unsigned)((threads + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
  const uint4 *X = (const uint4*)x, *R = (const uint4*)residual, *W = (const uint4*)weight;
  uint4 *O = (uint4*)out, *RO = (uint4*)residual_out;
  switch (tpr) {
    case 32: k_rmsnorm<32><<<grid, 256, 0, st>>>(X, R, rows, cols, W, eps, O, RO); break;
    case 16: k_rmsnorm<16><<<grid, 256, 0, st>>>(X, R, rows, cols, W, eps, O, RO); break;
    case 8: k_rmsnorm<8><<<grid, 256, 0, st>>>(X, R, rows, cols, W, eps, O, RO); break;
    case 4: k_rmsnorm<4><<<grid, 256, 0, st>>>(X, R, rows, cols, W, eps, O, RO); break;
    case 2: k_rmsnorm<2><<<grid, 256, 0, st>>>(X, R, rows, cols, W, eps, O, RO); break;
    default: k_rmsnorm<1><<<grid, 256, 0, st>>>(X, R, rows, cols, W, eps, O, RO); break;
  }
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_rotary_bf16(const void* x, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t sb,
                     int64_t sh, int64_t ss, const void* cos, const void* sin, int64_t cos_batch_stride, void* out,
                     void* stream) {
  if (batch < 0 || seq < 0 || heads <= 0 || head_dim <= 0 || sb < 0 || sh < 0 || ss < 0 || cos_batch_stride < 0)
    return LLMC_EINVAL_ARG;
  if (batch == 0 || seq == 0) return LLMC_OK;
  if (!x || !cos || !sin || !out) return LLMC_EINVAL_ARG;
  if (head_dim % 16 || sb % 8 || sh % 8 || ss % 8 || cos_batch_stride % 8 || !al16(x) || !al16(cos) || !al16(sin) ||
      !al16(out))
    return LLMC_EINVAL_SHAPE;
  const int64_t total = batch * seq * heads * (head_dim / 16);
  k_rotary<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint16_t*)x, seq, heads, head_dim, sb, sh, ss, (const uint16_t*)cos, (const uint16_t*)sin,
      cos_batch_stride, total, (uint16_t*)out);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_silu_mul_bf16(const void* gate, const void* up, int64_t n, void* out, void* stream) {
  if (n < 0) return LLMC_EINVAL_ARG;
  if (n == 0) return LLMC_OK;
  if (!gate || !up || !out) return LLMC_EINVAL_ARG;
  if (n % 8 || !al16(gate) || !al16(up) || !al16(out)) return LLMC_EINVAL_SHAPE;
  const int64_t n8 = n / 8;
  k_silu_mul<<<(unsigned)((n8 + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const uint4*)gate, (const uint4*)up,
                                                                            n8, (uint4*)out);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_silu_mul_scaled_bf16(const void* gate, const void* up, int64_t rows, int64_t cols, int64_t group,
                              const float* weights, int64_t weights_ld, void* out, void* out_scaled, void* stream) {
  if (rows < 0 || cols < 0 || group <= 0 || weights_ld < 0) return LLMC_EINVAL_ARG;
  if (rows == 0 || cols == 0) return LLMC_OK;
  if (!gate || !up || (!out && !out_scaled) || (out_scaled && !weights)) return LLMC_EINVAL_ARG;
  if (cols % 8 || group % 8 || cols % group || !al16(gate) || !al16(up) || (out && !al16(out)) ||
      (out_scaled && !al16(out_scaled)) || (weights && weights_ld < cols / group))
    return LLMC_EINVAL_SHAPE;
  if (!out_scaled) {  // the plain product over the flat tensor
    const int64_t n8 = rows * cols / 8;
    k_silu_mul<<<(unsigned)((n8 + 255) / 256), 256, 0, (cudaStream_t)stream>>>((const uint4*)gate, (const uint4*)up,
                                                                              n8, (uint4*)out);
    llmc::note_launch();
    return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  if (cols / 8 >= (1ll << 31)) return LLMC_EINVAL_SHAPE;
  const int cols8 = (int)(cols / 8);
  const dim3 grid((unsigned)((cols8 + 255) / 256), (unsigned)std::min<int64_t>(rows, 65535));
  k_silu_mul_scaled<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint4*)gate, (const uint4*)up, rows, cols8,
                                                            (int)(group / 8), out_scaled ? weights : nullptr,
                                                            weights_ld, (uint4*)out, (uint4*)out_scaled);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_scale_groups_bf16(const void* x, int64_t rows, int64_t cols, int64_t group, const float* weights,
                           int64_t weights_ld, void* out, void* stream) {
  if (rows < 0 || cols < 0 || group <= 0 || weights_ld < 0) return LLMC_EINVAL_ARG;
  if (rows == 0 || cols == 0) return LLMC_OK;
  if (!x || !weights || !out) return LLMC_EINVAL_ARG;
  if (cols % 8 || group % 8 || cols % group || !al16(x) || !al16(out) || weights_ld < cols / group)
    return LLMC_EINVAL_SHAPE;
  if (cols / 8 >= (1ll << 31)) return LLMC_EINVAL_SHAPE;
  const int cols8 = (int)(cols / 8);
  const dim3 grid((unsigned)((cols8 + 255) / 256), (unsigned)std::min<int64_t>(rows, 65535));
  k_scale_groups<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint4*)x, rows, cols8, (int)(group / 8), weights,
                                                         weights_ld, (uint4*)out);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_moe_combine_bf16(const void* y, int64_t y_rows, const int* pos, const float* weights, int64_t tokens,
                          int64_t top_k, int64_t hidden, void* out, void* stream) {
  if (tokens < 0 || top_k <= 0 || hidden <= 0 || y_rows < 0) return LLMC_EINVAL_ARG;
  if (tokens == 0) return LLMC_OK;
  if (!y || !pos || !weights || !out) return LLMC_EINVAL_ARG;
  if (hidden % 8 || !al16(y) || !al16(out) || top_k > 64 || hidden / 8 >= (1ll << 31)) return LLMC_EINVAL_SHAPE;
  const int h8 = (int)(hidden / 8);
  const dim3 grid((unsigned)((h8 + 255) / 256), (unsigned)std::min<int64_t>(tokens, 65535));
  k_moe_combine<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint4*)y, y_rows, pos, weights, tokens, (int)top_k,
                                                        h8, (uint4*)out);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

}  // extern "C"
