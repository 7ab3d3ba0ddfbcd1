// Activation min/max observers: the statistics that static activation
// schemes (input / output activations, KV-cache q/k/v states) accumulate
// over the calibration batches.
//
// Reference: S/observers/min_max.py:16-110 (MemorylessMinMaxObserver,
// StaticMinMaxObserver, MinMaxObserver with its moving average
// S/observers/helpers.py:219-221 `lerp`) over the activation layouts of
// `flatten_for_calibration` (S/observers/helpers.py:104-130,133-153):
//   TENSOR                 one statistic over the whole tensor;
//   GROUP / TENSOR_GROUP   one statistic per group of `group` consecutive
//                          features, over all tokens.
//
// The reduction is HBM-bound: a thread streams 8 consecutive features of a
// slab of tokens with 16-byte loads, keeps one running min/max (its 8
// features share a group), the threads of a group combine by shuffles and
// one lane per group folds the result into an order-preserving integer key
// with atomicMin / atomicMax.  A one-thread-per-group pass then applies the
// observer's update rule in the statistics' dtype.
#include "llmc_b200.h"
#include "llmc_common.cuh"

#include <algorithm>

namespace llmc {
namespace actobs {

// float <-> uint32 key with the order of the floats (-0 < +0)
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float kfloat(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__global__ void k_act_init(uint32_t* kmin, uint32_t* kmax, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    kmin[i] = 0xFFFFFFFFu;
    kmax[i] = 0u;
  }
}

template <int DT>  // 0: bf16, 1: float32
__device__ __forceinline__ void load8(const void* x, int64_t e, float (&v)[8]) {
  if (DT == 0) {
    const uint4 a = __ldcs((const uint4*)((const uint16_t*)x + e));
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[2 * k] = __uint_as_float(w[k] << 16);
      v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    }
  } else {
    const float4 a = __ldcs((const float4*)((const float*)x + e));
    const float4 b = __ldcs((const float4*)((const float*)x + e) + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// grid: x over 8-feature columns (blockDim.x threads each), y over token slabs.
// gv = features per group / 8 (a power of two up to 32, or 0: the whole tensor)
template <int DT>
__global__ void __launch_bounds__(256) k_act_reduce(const void* __restrict__ x, int64_t n_tok, int64_t hidden,
                                                    int64_t slab, int gv, int64_t group, uint32_t* kmin,
                                                    uint32_t* kmax) {
  const int64_t nv = hidden / 8;
  const int64_t vc = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t0 = (int64_t)blockIdx.y * slab, t1 = min(n_tok, t0 + slab);
  float mn = INFINITY, mx = -INFINITY;
  if (vc < nv) {
    int64_t t = t0;
    for (; t + 4 <= t1; t += 4) {  // four rows in flight
      float v[4][8];
#pragma unroll
      for (int u = 0; u < 4; ++u) load8<DT>(x, (t + u) * hidden + vc * 8, v[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int k = 0; k < 8; ++k) { mn = fminf(mn, v[u][k]); mx = fmaxf(mx, v[u][k]); }
    }
    for (; t < t1; ++t) {
      float v[8];
      load8<DT>(x, t * hidden + vc * 8, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) { mn = fminf(mn, v[k]); mx = fmaxf(mx, v[k]); }
    }
  }
  const int lane = threadIdx.x & 31;
  const int width = (gv == 0 || gv > 32) ? 32 : gv;  // threads combined by shuffles
  for (int o = 1; o < width; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if ((lane & (width - 1)) == 0 && vc < nv && t0 < t1) {
    const int64_t g = (gv == 0) ? 0 : (vc * 8) / group;
    atomicMin(kmin + g, fkey(mn));
    atomicMax(kmax + g, fkey(mx));
  }
}

// the observer's update rule, in the statistics' dtype
//   mode 0 (memoryless) or no previous statistics: the new min / max;
//   mode 1 (static): elementwise min / max with the previous ones;
//   mode 2 (moving average): prev * w0 + new * w1, each product and the sum
//          rounded to the dtype (torch evaluates `start * (1 - c) + end * c`
//          on bf16 tensors with float32 arithmetic, one rounding per op).
template <int DT>
__global__ void k_act_finish(const uint32_t* kmin, const uint32_t* kmax, int64_t n, int mode, int has_prev, float w0,
                             float w1, void* min_io, void* max_io) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float nmn = kfloat(kmin[i]), nmx = kfloat(kmax[i]);
  auto rd = [](const void* p, int64_t j) {
    return DT == 0 ? bf16_to_f(((const uint16_t*)p)[j]) : ((const float*)p)[j];
  };
  auto R = [](float v) { return DT == 0 ? rbf(v) : v; };
  if (has_prev && mode == 1) {
    nmn = fminf(rd(min_io, i), nmn);
    nmx = fmaxf(rd(max_io, i), nmx);
  } else if (has_prev && mode == 2) {
    nmn = R(__fadd_rn(R(__fmul_rn(rd(min_io, i), w0)), R(__fmul_rn(nmn, w1))));
    nmx = R(__fadd_rn(R(__fmul_rn(rd(max_io, i), w0)), R(__fmul_rn(nmx, w1))));
  }
  if (DT == 0) {
    ((uint16_t*)min_io)[i] = f_to_bf16(nmn);
    ((uint16_t*)max_io)[i] = f_to_bf16(nmx);
  } else {
    ((float*)min_io)[i] = nmn;
    ((float*)max_io)[i] = nmx;
  }
}

}  // namespace actobs
}  // namespace llmc

using namespace llmc;
using namespace llmc::actobs;

extern "C" {

int llmc_observe_activation_workspace_size(int64_t hidden, int64_t group, int64_t* bytes) {
  if (!bytes || hidden <= 0 || group < 0) return LLMC_EINVAL_ARG;
  const int64_t ng = group > 0 ? hidden / group : 1;
  *bytes = 2 * ng * (int64_t)sizeof(uint32_t);
  return LLMC_OK;
}

int llmc_observe_activation(const void* x, int64_t n_tok, int64_t hidden, int dtype, int64_t group, int mode,
                            float avg_w0, float avg_w1, int has_prev, void* min_io, void* max_io, void* workspace,
                            void* stream) {
  if (hidden <= 0 || n_tok < 0 || group < 0 || dtype < 0 || dtype > 1 || mode < 0 || mode > 2) return LLMC_EINVAL_ARG;
  if (!min_io || !max_io || !workspace || (!x && n_tok > 0)) return LLMC_EINVAL_ARG;
  if (group > 0 && hidden % group) return LLMC_EINVAL_SHAPE;
  if (n_tok == 0) return LLMC_OK;  // an empty observation changes nothing
  // 8-feature vectors: rows of whole vectors, 16-byte aligned, groups of 8 .. 256 features
  if (hidden % 8 || ((uintptr_t)x % 16)) return LLMC_ENOSUPPORT;
  int gv = 0;
  if (group > 0) {
    if (group % 8) return LLMC_ENOSUPPORT;
    gv = (int)(group / 8);
    if (gv > 32 || (gv & (gv - 1))) return LLMC_ENOSUPPORT;  // a power of two up to 256 features
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t ng = group > 0 ? hidden / group : 1;
  uint32_t* kmin = (uint32_t*)workspace;
  uint32_t* kmax = kmin + ng;
  k_act_init<<<(unsigned)std::min<int64_t>((ng + 255) / 256, 1024), 256, 0, st>>>(kmin, kmax, ng);
  llmc::note_launch();
  const int64_t nv = hidden / 8;
  const unsigned gx = (unsigned)((nv + 255) / 256);
  const int64_t want = std::max<int64_t>(1, (148 * 8) / (int64_t)gx);  // about 8 CTAs per SM in all
  const int64_t slabs = std::min<int64_t>(std::min<int64_t>(n_tok, want), 65535);
  const int64_t slab = (n_tok + slabs - 1) / slabs;
  const dim3 grid(gx, (unsigned)((n_tok + slab - 1) / slab));
  if (dtype == 0) k_act_reduce<0><<<grid, 256, 0, st>>>(x, n_tok, hidden, slab, gv, group, kmin, kmax);
  else k_act_reduce<1><<<grid, 256, 0, st>>>(x, n_tok, hidden, slab, gv, group, kmin, kmax);
  llmc::note_launch();
  const unsigned fb = (unsigned)((ng + 255) / 256);
  if (dtype == 0) k_act_finish<0><<<fb, 256, 0, st>>>(kmin, kmax, ng, mode, has_prev, avg_w0, avg_w1, min_io, max_io);
  else k_act_finish<1><<<fb, 256, 0, st>>>(kmin, kmax, ng, mode, has_prev, avg_w0, avg_w1, min_io, max_io);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

}  // extern "C"
