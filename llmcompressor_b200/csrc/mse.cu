// MSE grid-search weight observer (memoryless_mse) on sm_100a.
//
// Reference: S/observers/mse_quant.py:19-141 (_grid_search_mse, eager
// search) and :235-273 (_calculate_error).  Per parameter group, candidate
// ranges (min, max) * p with p = 1 - i/grid for i < int(maxshrink * grid);
// error = sum over the group of |fake_quant(x) - x| ** norm, every op in
// bf16 as torch evaluates it on a bf16 weight (the exponent itself is a
// bf16 scalar, 2.4 -> 2.40625); a candidate wins when its error is strictly
// lower than the best so far.  The search stops for the whole tensor once
// `patience` consecutive steps improved no group.
//
// GPU shape: one pass over the weight.  Each group is held in registers by a
// team of lanes (groups of <= 1024 columns) or a CTA (channel rows, blocks,
// small tensors) and every candidate is evaluated from registers; the group
// records which steps improved it (a bit mask).  The tensor-wide early stop
// is resolved afterwards: the masks are OR-ed into one word, the stop step
// follows from it, and each group keeps its last improvement before it.
//
// |d| ** norm for the bf16 differences d is a 32768-entry table of bf16
// results, computed on the host with the C library's powf (the function
// torch's CPU path and numpy call) and kept on every device in a
// __device__ array, so the kernel's powers equal the reference's bit for bit.
#include "llmc_common.cuh"

#include <math.h>
#include <string.h>

#include <algorithm>
#include <mutex>

namespace llmc {
namespace mse {

constexpr int kMaxSteps = 64;  // improvement masks are 64-bit

__device__ uint16_t g_pow_tbl[32768];

struct MseArgs {
  const uint16_t* w;
  int64_t rows, cols;
  QArgs a;
  int steps, patience;
  float grid;
  uint16_t* mn_out;  // bf16 per group: raw min, then the chosen min
  uint16_t* mx_out;
  unsigned long long* masks;  // per group, then one tensor-wide word
  int64_t ngroups;
};

// bf16 candidate bound: RN_bf16(v * float(p)), p = 1 - i/grid in double
__device__ __forceinline__ float shrink(float v, int i, float grid) {
  const float p = (float)(1.0 - (double)i / (double)grid);
  return rbf(v * p);
}

__device__ __forceinline__ float e2m1_value(uint32_t code) {
  const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const float v = mag[code & 7u];
  return (code & 8u) ? -v : v;
}

// bf16 fake-quant error term of one value: RN_bf16(|fq(x) - x| ** norm)
// (CT forward_helpers.py _quantize_dequantize: x / s, + zp, clamp, round,
// - zp, * s, all in bf16).
__device__ __forceinline__ float err_term(float x, float s, float r, bool fast, float zp, bool has_zp, const QArgs& a,
                                          float qmin, float qmax) {
  float q;
  if (fast) {  // Markstein-corrected quotient, exact for bf16 operands (see casts.cu)
    const float q0 = __fmul_rn(-x, -r);
    const float e = __fmaf_rn(q0, s, -x);
    q = rbf(__fmaf_rn(e, -r, q0));
  } else {
    q = rbf(__fdiv_rn(x, s));
  }
  if (has_zp) q = rbf(q + zp);
  q = fminf(fmaxf(q, qmin), qmax);
  if (!a.is_float) q = rintf(q);
  else if (a.bits == 8) q = round_e4m3(q);
  else q = e2m1_value(e2m1_code(__fadd_rn(q, 0.0f)));
  if (has_zp) q = rbf(q - zp);
  const float dq = rbf(q * s);
  const uint32_t db = (uint32_t)f_to_bf16(dq - x) & 0x7FFFu;
  return bf16_to_f(g_pow_tbl[db]);
}

struct StepQ {
  float s, r, zp, qmin, qmax;
  bool fast, has_zp;
};
__device__ __forceinline__ StepQ step_qparams(float mn0, float mx0, int i, const MseArgs& m, float* smn, float* smx) {
  StepQ q;
  *smn = shrink(mn0, i, m.grid);
  *smx = shrink(mx0, i, m.grid);
  float zp = 0.f;
  q.s = group_qparams(*smn, *smx, m.a, false, 0.f, &zp);
  q.zp = zp;
  q.has_zp = !m.a.symmetric;
  const float r = __frcp_rn(q.s);
  q.r = r;
  q.fast = r > 1.0e-36f && r < 1.0e36f;
  q.qmin = m.a.qmin();
  q.qmax = m.a.qmax();
  return q;
}

// Bit i set: candidate i lowered the group's best error (strictly), the
// best being updated at every step before i.
__device__ __forceinline__ bool improves(float err, float& best) {
  const float e = rbf(err);  // torch.sum of a bf16 tensor returns bf16
  if (e < best) { best = e; return true; }
  return false;
}

// ------------------------------------------------------------------ teams
// GROUP / TENSOR_GROUP: a team of T = min(32, gs) lanes per group, E = gs/T
// consecutive values per lane (E <= 32).
template <int E>
__global__ void __launch_bounds__(256) k_mse_team(MseArgs m, int T) {
  const int lane = threadIdx.x & 31;
  const int gs = (int)m.a.group;
  const int teams_per_warp = 32 / T;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t g = warp * teams_per_warp + lane / T;
  const int tl = lane % T;
  const bool valid = g < m.ngroups;
  float x[E];
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < E; ++k) {
    x[k] = valid ? bf16_to_f(m.w[g * gs + tl * E + k]) : 0.f;
    mn = fminf(mn, x[k]);
    mx = fmaxf(mx, x[k]);
  }
  for (int o = 1; o < T; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  float best = 3.3895313892515355e38f;  // torch.finfo(bf16).max
  unsigned long long mask = 0ull;
  for (int i = 0; i < m.steps; ++i) {
    float smn, smx;
    const StepQ q = step_qparams(mn, mx, i, m, &smn, &smx);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < E; ++k) acc += err_term(x[k], q.s, q.r, q.fast, q.zp, q.has_zp, m.a, q.qmin, q.qmax);
    for (int o = 1; o < T; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (improves(acc, best)) mask |= 1ull << i;
  }
  if (valid && tl == 0) {
    m.mn_out[g] = f_to_bf16(mn);
    m.mx_out[g] = f_to_bf16(mx);
    m.masks[g] = mask;
    if (mask) atomicOr(m.masks + m.ngroups, mask);
  }
}

// ------------------------------------------------------------------ CTAs
// CHANNEL rows, BLOCK tiles (zero padding joins the group, as
// maybe_pad_tensor_for_block_quant does) and small TENSOR groups: one CTA,
// NP 16-value pieces per thread.
__device__ __forceinline__ float cta_sum(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += sh[i];
  return s;
}
__device__ __forceinline__ float cta_ext(float v, bool is_max, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, t) : fminf(v, t);
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = sh[0];
  for (int i = 1; i < (int)(blockDim.x >> 5); ++i) s = is_max ? fmaxf(s, sh[i]) : fminf(s, sh[i]);
  return s;
}

template <int NP>
__global__ void __launch_bounds__(256) k_mse_cta(MseArgs m) {
  __shared__ float sh[32];
  const int64_t gi = blockIdx.x;
  int64_t r0, r1, c0, c1;
  const QArgs& a = m.a;
  if (a.strategy == LLMC_STRAT_TENSOR) { r0 = 0; r1 = m.rows; c0 = 0; c1 = m.cols; }
  else if (a.strategy == LLMC_STRAT_CHANNEL) { r0 = gi; r1 = gi + 1; c0 = 0; c1 = m.cols; }
  else {
    const int64_t bcn = (m.cols + a.bw - 1) / a.bw;
    r0 = (gi / bcn) * a.bh; r1 = min(m.rows, r0 + a.bh);
    c0 = (gi % bcn) * a.bw; c1 = min(m.cols, c0 + a.bw);
  }
  const int64_t w = c1 - c0, n = (r1 - r0) * w;
  uint32_t xp[NP * 8];  // bf16 pairs: value k in half (k & 1) of word k / 2
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < NP * 16; ++k) {
    const int64_t e = (int64_t)threadIdx.x + (int64_t)k * blockDim.x;
    uint32_t b = 0u;
    if (e < n) {
      b = m.w[(r0 + e / w) * m.cols + c0 + e % w];
      const float v = bf16_to_f((uint16_t)b);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    if (k & 1) xp[k >> 1] |= b << 16;
    else xp[k >> 1] = b;
  }
  const bool padded = a.strategy == LLMC_STRAT_BLOCK && ((r1 - r0) < a.bh || w < a.bw);
  if (padded) { mn = fminf(mn, 0.f); mx = fmaxf(mx, 0.f); }
  mn = cta_ext(mn, false, sh);
  mx = cta_ext(mx, true, sh);
  float best = 3.3895313892515355e38f;
  unsigned long long mask = 0ull;
  for (int i = 0; i < m.steps; ++i) {
    float smn, smx;
    const StepQ q = step_qparams(mn, mx, i, m, &smn, &smx);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < NP * 16; ++k) {
      const int64_t e = (int64_t)threadIdx.x + (int64_t)k * blockDim.x;
      const float v = (k & 1) ? __uint_as_float(xp[k >> 1] & 0xFFFF0000u) : __uint_as_float(xp[k >> 1] << 16);
      if (e < n) acc += err_term(v, q.s, q.r, q.fast, q.zp, q.has_zp, a, q.qmin, q.qmax);
    }
    // padding zeros: fake_quant(0) == 0 for every format, so they add nothing
    acc = cta_sum(acc, sh);
    if (improves(acc, best)) mask |= 1ull << i;
  }
  if (threadIdx.x == 0) {
    m.mn_out[gi] = f_to_bf16(mn);
    m.mx_out[gi] = f_to_bf16(mx);
    m.masks[gi] = mask;
    if (mask) atomicOr(m.masks + m.ngroups, mask);
  }
}

// The tensor-wide stop and each group's last improvement before it.
__global__ void k_mse_finish(MseArgs m) {
  const unsigned long long any = m.masks[m.ngroups];
  int stop = m.steps, quiet = 0;
  for (int i = 0; i < m.steps; ++i) {
    if ((any >> i) & 1ull) quiet = 0;
    else if (++quiet >= m.patience) { stop = i + 1; break; }
  }
  const unsigned long long keep = stop >= 64 ? ~0ull : ((1ull << stop) - 1ull);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < m.ngroups;
       g += (int64_t)gridDim.x * blockDim.x) {
    const unsigned long long mk = m.masks[g] & keep;
    if (!mk) continue;  // never improved: the unshrunk range stays
    const int i = 63 - __clzll((long long)mk);
    m.mn_out[g] = f_to_bf16(shrink(bf16_to_f(m.mn_out[g]), i, m.grid));
    m.mx_out[g] = f_to_bf16(shrink(bf16_to_f(m.mx_out[g]), i, m.grid));
  }
}

// ------------------------------------------------------------------ host
std::mutex g_tbl_mu;
float g_tbl_norm[64];
bool g_tbl_ready[64];

uint16_t host_f_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);  // NaN stays NaN
  const uint32_t lsb = (u >> 16) & 1u;
  return (uint16_t)((u + 0x7FFFu + lsb) >> 16);
}

// Fills the power table of the current device for this exponent (the
// caller's stream is synchronised only when the table changes).
int ensure_pow_table(float norm, cudaStream_t st) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return LLMC_ECUDA;
  if (dev < 0 || dev >= 64) return LLMC_ENOSUPPORT;
  std::lock_guard<std::mutex> lock(g_tbl_mu);
  if (g_tbl_ready[dev] && g_tbl_norm[dev] == norm) return LLMC_OK;
  // the exponent as torch holds it for a bf16 tensor: rounded to bf16
  uint16_t nb = host_f_to_bf16(norm);
  uint32_t nu = (uint32_t)nb << 16;
  float ne;
  memcpy(&ne, &nu, 4);
  static uint16_t tbl[32768];
  for (uint32_t b = 0; b < 32768u; ++b) {
    uint32_t u = b << 16;
    float v;
    memcpy(&v, &u, 4);
    tbl[b] = host_f_to_bf16(powf(v, ne));
  }
  if (cudaStreamSynchronize(st) != cudaSuccess) return LLMC_ECUDA;
  if (cudaMemcpyToSymbol(g_pow_tbl, tbl, sizeof(tbl)) != cudaSuccess) return LLMC_ECUDA;
  g_tbl_norm[dev] = norm;
  g_tbl_ready[dev] = true;
  return LLMC_OK;
}

int64_t n_groups(const QArgs& a, int64_t rows, int64_t cols) {
  switch (a.strategy) {
    case LLMC_STRAT_TENSOR: return 1;
    case LLMC_STRAT_CHANNEL: return rows;
    case LLMC_STRAT_BLOCK: return ((rows + a.bh - 1) / a.bh) * ((cols + a.bw - 1) / a.bw);
    default: return a.group > 0 ? rows * (cols / a.group) : 0;
  }
}

}  // namespace mse
}  // namespace llmc

using namespace llmc;
using namespace llmc::mse;

extern "C" {

int llmc_observe_mse_workspace_size(int64_t rows, int64_t cols, const LlmcQuantArgs* args, int64_t* bytes) {
  if (!args || !bytes || rows < 0 || cols < 0) return LLMC_EINVAL_ARG;
  const QArgs a = to_qargs(*args);
  *bytes = (int64_t)sizeof(unsigned long long) * (n_groups(a, rows, cols) + 1);
  return LLMC_OK;
}

int llmc_observe_mse(const void* w, int64_t rows, int64_t cols, const LlmcQuantArgs* args, float maxshrink,
                     int patience, float grid, float norm, void* mn, void* mx, void* workspace, void* stream) {
  if (!args || rows < 0 || cols < 0 || !(grid > 0.f) || patience < 0) return LLMC_EINVAL_ARG;
  if ((rows * cols > 0) && (!w || !mn || !mx || !workspace)) return LLMC_EINVAL_ARG;
  const QArgs a = to_qargs(*args);
  if (a.bits != 4 && a.bits != 8) return LLMC_ENOSUPPORT;
  if (a.is_float && !a.symmetric && a.bits == 4) return LLMC_ENOSUPPORT;
  const double st_d = (double)maxshrink * (double)grid;
  const int steps = st_d > 0 ? (int)st_d : 0;  // int(maxshrink * grid)
  if (steps > kMaxSteps) return LLMC_ENOSUPPORT;
  if (rows * cols == 0) return LLMC_OK;
  cudaStream_t st = (cudaStream_t)stream;
  MseArgs m;
  m.w = (const uint16_t*)w; m.rows = rows; m.cols = cols; m.a = a;
  m.steps = steps; m.patience = patience; m.grid = grid;
  m.mn_out = (uint16_t*)mn; m.mx_out = (uint16_t*)mx;
  m.masks = (unsigned long long*)workspace;
  m.ngroups = n_groups(a, rows, cols);
  if (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) {
    if (a.group <= 0) return LLMC_EINVAL_ARG;
    if (cols % a.group) return LLMC_EINVAL_SHAPE;
  }
  if (a.strategy == LLMC_STRAT_BLOCK && (a.bh <= 0 || a.bw <= 0)) return LLMC_EINVAL_ARG;
  int s = ensure_pow_table(norm, st);
  if (s != LLMC_OK) return s;
  if (cudaMemsetAsync(m.masks + m.ngroups, 0, sizeof(unsigned long long), st) != cudaSuccess) return LLMC_ECUDA;
  if (a.strategy == LLMC_STRAT_GROUP || a.strategy == LLMC_STRAT_TENSOR_GROUP) {
    const int64_t gs = a.group;
    int T, E;
    if (gs >= 32) {
      if (gs % 32 || gs / 32 > 32) return LLMC_ENOSUPPORT;
      T = 32; E = (int)(gs / 32);
    } else {
      if (gs & (gs - 1)) return LLMC_ENOSUPPORT;
      T = (int)gs; E = 1;
    }
    const int64_t warps = (m.ngroups + (32 / T) - 1) / (32 / T);
    const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
    switch (E) {
      case 1: mse::k_mse_team<1><<<blocks, 256, 0, st>>>(m, T); break;
      case 2: mse::k_mse_team<2><<<blocks, 256, 0, st>>>(m, T); break;
      case 4: mse::k_mse_team<4><<<blocks, 256, 0, st>>>(m, T); break;
      case 8: mse::k_mse_team<8><<<blocks, 256, 0, st>>>(m, T); break;
      case 16: mse::k_mse_team<16><<<blocks, 256, 0, st>>>(m, T); break;
      case 32: mse::k_mse_team<32><<<blocks, 256, 0, st>>>(m, T); break;
      default: return LLMC_ENOSUPPORT;  // group sizes 32 * {1,2,4,8,16,32} and powers of two below 32
    }
  } else {
    int64_t n;
    if (a.strategy == LLMC_STRAT_TENSOR) n = rows * cols;
    else if (a.strategy == LLMC_STRAT_CHANNEL) n = cols;
    else n = a.bh * a.bw;
    if (n <= 256 * 16) mse::k_mse_cta<1><<<(unsigned)m.ngroups, 256, 0, st>>>(m);
    else if (n <= 256 * 32) mse::k_mse_cta<2><<<(unsigned)m.ngroups, 256, 0, st>>>(m);
    else if (n <= 256 * 64) mse::k_mse_cta<4><<<(unsigned)m.ngroups, 256, 0, st>>>(m);
    else if (n <= 256 * 128) mse::k_mse_cta<8><<<(unsigned)m.ngroups, 256, 0, st>>>(m);
    else return LLMC_ENOSUPPORT;  // a parameter group above 32768 values
  }
  llmc::note_launch();
  const unsigned fb = (unsigned)std::min<int64_t>((m.ngroups + 255) / 256, 148 * 8);
  mse::k_mse_finish<<<fb, 256, 0, st>>>(m);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

}  // extern "C"
