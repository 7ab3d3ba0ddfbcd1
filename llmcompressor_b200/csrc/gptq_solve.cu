// GPTQ solve on sm_100a: damping + dead-column mask, the upper Cholesky
// factor of the inverse Hessian, and the blockwise quantize / error-propagate
// loop.  Reference: quantize_weight, S/modifiers/gptq/gptq_quantize.py:100-296.
//
// Inverse factor.  The reference computes U = chol(chol_inverse(chol(A)), upper)
// with A = H + damp*I.  Here A is factored from the bottom-right corner
// instead: with J the reversal permutation, JAJ = L L^T (lower Cholesky), so
// A = R R^T with R = J L J upper, and A^-1 = (R^-1)^T R^-1.  R^-1 is upper
// with a positive diagonal, hence it *is* U.  So U = J L^-1 J: one Cholesky
// (d^3/3) plus one triangular inverse (d^3/3) instead of the reference's
// Cholesky + cholesky_inverse + Cholesky.  Same matrix, float32 throughout.
//
// Both factorisations are blocked (128): a one-CTA kernel factors and inverts
// each diagonal block in shared memory; panels and trailing updates are
// float32 GEMMs (k_sgemm).  A non-positive pivot sets LLMC_ENOT_PD in the
// caller's status word; the quantize kernels then use the identity (the
// reference's round-to-nearest fallback) without a host round trip.
//
// Block loop.  Rows of W are independent, so one thread owns one row; a CTA
// stages its rows' 128-column block and the 128x128 block of U in shared
// memory.  Within a 32-column sub-block the per-column update follows the
// reference exactly (float32 product, then subtraction, column by column);
// across sub-blocks and across 128-column blocks the update is the lazy
// batched form W -= Err * U (the reference's `Err1.matmul(Hinv[i1:i2, i2:])`).
#include "llmc_common.cuh"
#include "tc32.cuh"

#include <algorithm>
#include <mutex>

namespace llmc {
namespace gq {

// ---------------------------------------------------------------------------
// float32 GEMM: C (m x n, ldc) {=, -=, = -} A * op(B)
//   A: !TA row-major (m x k, lda);  TA: stored k-major (k x m, lda)
//   B: !TB row-major (k x n, ldb);  TB: stored n-major (n x k, ldb)
//   tri:     only output tiles that touch the lower triangle (row >= col)
//   b_lower: B is lower triangular -> for an output column tile starting at
//            n0 only k >= n0 contributes
//   skip:    optional device flag; the kernel does nothing when it is set
// ---------------------------------------------------------------------------
struct GemmArgs {
  int m, n, k;
  const float* A;
  int64_t lda;
  const float* B;
  int64_t ldb;
  float* C;
  int64_t ldc;
  int mode;  // 0: C = AB, 1: C = C - AB, 2: C = -AB
  int tri, b_lower;
  const int* skip;
  int max_ctas;  // tensor-core path: at most this many CTAs (0: one per SM)
  int* status;   // tensor-core path: raised to LLMC_ETIMEOUT if a bounded wait runs out
};

constexpr int GBM = 128, GBN = 128, GBK = 8;

template <bool TA, bool TB>
__global__ void __launch_bounds__(256) k_sgemm(GemmArgs g) {
  if (g.skip && *g.skip) return;
  const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
  if (g.tri && n0 > m0 + GBM - 1) return;
  __shared__ __align__(16) float As[2][GBK][GBM + 4];
  __shared__ __align__(16) float Bs[2][GBK][GBN + 4];
  const int t = threadIdx.x;
  const int tx = t & 15, ty = t >> 4;
  int kbeg = 0;
  if (g.b_lower) kbeg = (n0 / GBK) * GBK;
  const int kend = g.k;

  float a_ld[4], b_ld[4];
  auto load_tiles = [&](int k0) {
    // A
    if (!TA) {
      const int mm = t >> 1, kq = (t & 1) * 4;
      const int gm = m0 + mm;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int gk = k0 + kq + i;
        a_ld[i] = (gm < g.m && gk < kend) ? g.A[(int64_t)gm * g.lda + gk] : 0.f;
      }
    } else {
      const int kk = t >> 5, mq = (t & 31) * 4;
      const int gk = k0 + kk;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int gm = m0 + mq + i;
        a_ld[i] = (gm < g.m && gk < kend) ? g.A[(int64_t)gk * g.lda + gm] : 0.f;
      }
    }
    // B
    if (TB) {
      const int nn = t >> 1, kq = (t & 1) * 4;
      const int gn = n0 + nn;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int gk = k0 + kq + i;
        b_ld[i] = (gn < g.n && gk < kend) ? g.B[(int64_t)gn * g.ldb + gk] : 0.f;
      }
    } else {
      const int kk = t >> 5, nq = (t & 31) * 4;
      const int gk = k0 + kk;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int gn = n0 + nq + i;
        b_ld[i] = (gn < g.n && gk < kend) ? g.B[(int64_t)gk * g.ldb + gn] : 0.f;
      }
    }
  };
  auto store_tiles = [&](int buf) {
    if (!TA) {
      const int mm = t >> 1, kq = (t & 1) * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) As[buf][kq + i][mm] = a_ld[i];
    } else {
      const int kk = t >> 5, mq = (t & 31) * 4;
      *(float4*)&As[buf][kk][mq] = make_float4(a_ld[0], a_ld[1], a_ld[2], a_ld[3]);
    }
    if (TB) {
      const int nn = t >> 1, kq = (t & 1) * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) Bs[buf][kq + i][nn] = b_ld[i];
    } else {
      const int kk = t >> 5, nq = (t & 31) * 4;
      *(float4*)&Bs[buf][kk][nq] = make_float4(b_ld[0], b_ld[1], b_ld[2], b_ld[3]);
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  int buf = 0;
  if (kbeg < kend) {
    load_tiles(kbeg);
    store_tiles(0);
    __syncthreads();
    for (int k0 = kbeg; k0 < kend; k0 += GBK) {
      const bool more = k0 + GBK < kend;
      if (more) load_tiles(k0 + GBK);
#pragma unroll
      for (int kk = 0; kk < GBK; ++kk) {
        float4 a0 = *(const float4*)&As[buf][kk][ty * 4];
        float4 a1 = *(const float4*)&As[buf][kk][64 + ty * 4];
        float4 b0 = *(const float4*)&Bs[buf][kk][tx * 4];
        float4 b1 = *(const float4*)&Bs[buf][kk][64 + tx * 4];
        const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
      }
      if (more) {
        store_tiles(buf ^ 1);
        __syncthreads();
        buf ^= 1;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
    if (gm >= g.m) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
      if (gn >= g.n) continue;
      float* c = g.C + (int64_t)gm * g.ldc + gn;
      if (g.mode == 0) *c = acc[i][j];
      else if (g.mode == 1) *c = *c - acc[i][j];
      else *c = -acc[i][j];
    }
  }
}

// The tensor-core GEMM is used by the solve once it has passed its own parity
// test against float64 for every operand layout.
static bool g_use_tc32 = true;

static int launch_gemm(bool ta, bool tb, const GemmArgs& g, cudaStream_t st) {
  if (g.m <= 0 || g.n <= 0) return LLMC_OK;
  // Wide updates go to the tensor cores (3xTF32, float32 accuracy); small or
  // TMA-unaligned ones stay on the CUDA cores.
  if (g_use_tc32 && !g.b_lower && (int64_t)g.m * g.n * g.k >= (int64_t)128 * 128 * 128) {
    tc32::Gemm t = {};
    t.m = g.m; t.n = g.n; t.k = g.k;
    t.A = g.A; t.lda = g.lda; t.a_mn = ta;
    t.B = g.B; t.ldb = g.ldb; t.b_mn = !tb;
    t.C = g.C; t.ldc = g.ldc; t.mode = g.mode; t.tri = g.tri; t.skip = g.skip; t.max_ctas = g.max_ctas;
    t.status = g.status;
    const int s = tc32::gemm(t, st);
    if (s != LLMC_ENOSUPPORT) return s;
  }
  dim3 grid((g.n + GBN - 1) / GBN, (g.m + GBM - 1) / GBM);
  if (!ta && !tb) k_sgemm<false, false><<<grid, 256, 0, st>>>(g);
  else if (!ta && tb) k_sgemm<false, true><<<grid, 256, 0, st>>>(g);
  else if (ta && !tb) k_sgemm<true, false><<<grid, 256, 0, st>>>(g);
  else k_sgemm<true, true><<<grid, 256, 0, st>>>(g);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

// ---------------------------------------------------------------------------
// Hessian preparation: dead columns (diag == 0 -> 1, flagged), then
// damp = percdamp * mean(diag), diag += damp  (gptq_quantize.py:35-38,178-185)
// ---------------------------------------------------------------------------
__global__ void k_prep_hessian(float* H, int64_t d, float percdamp, uint8_t* dead) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
    float v = H[i * d + i];
    const bool dd = (v == 0.0f);
    if (dd) { v = 1.0f; H[i * d + i] = 1.0f; }
    dead[i] = dd ? 1 : 0;
    s += v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean = __fdiv_rn(red[0], (float)d);
  const float damp = percdamp * mean;
  for (int64_t i = threadIdx.x; i < d; i += blockDim.x) H[i * d + i] += damp;
}

// reversed copy: B[i][j] = A[d-1-i][d-1-j]  (only the lower triangle of B is used)
__global__ void k_reverse(const float* __restrict__ A, float* __restrict__ B, int64_t d) {
  const int64_t i = blockIdx.y, j0 = (int64_t)blockIdx.x * blockDim.x;
  const int64_t j = j0 + threadIdx.x;
  if (i < d && j < d && j <= i) B[i * d + j] = A[(d - 1 - i) * d + (d - 1 - j)];
}

// From Xt = L^-T (upper):  U = J L^-1 J = (J Xt J)^T, i.e. U[i][j] = Xt[d-1-j][d-1-i]
// for j >= i and 0 below the diagonal.  32x32 tiles through shared memory so
// that both the read and the write are coalesced.
__global__ void k_xt_to_u(const float* __restrict__ Xt, float* __restrict__ U, int64_t d) {
  __shared__ float tile[32][33];
  const int64_t I0 = (int64_t)blockIdx.y * 32, J0 = (int64_t)blockIdx.x * 32;
  for (int jj = threadIdx.y; jj < 32; jj += 8) {
    const int ii = threadIdx.x;
    const int64_t a = d - 1 - J0 - jj, b = d - 1 - I0 - ii;
    tile[jj][ii] = (a >= 0 && b >= 0) ? Xt[a * d + b] : 0.0f;
  }
  __syncthreads();
  for (int ii = threadIdx.y; ii < 32; ii += 8) {
    const int jj = threadIdx.x;
    const int64_t i = I0 + ii, j = J0 + jj;
    if (i < d && j < d) U[i * d + j] = (j >= i) ? tile[jj][ii] : 0.0f;
  }
}

// U^T (lower): Ut[i][j] = U[j][i] = Xt[d-1-i][d-1-j] for j <= i, 0 above.
__global__ void k_xt_to_ut(const float* __restrict__ Xt, float* __restrict__ Ut, int64_t d) {
  const int64_t i = blockIdx.y;
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < d && j < d) Ut[i * d + j] = (j <= i) ? Xt[(d - 1 - i) * d + (d - 1 - j)] : 0.0f;
}

// Factor one diagonal block (kb <= 128) of B in place (lower Cholesky) and
// write its lower-triangular inverse to Linv (row stride 128).
constexpr int PB = 128;
constexpr int PLD = PB + 1;  // padded row stride of the shared-memory blocks
// 16 warps: warp w walks rows (w, w+16, ...), its lanes walk the columns of a row.
// Step J of the warp's 32x32 Cholesky (lane = row): pivot, column J solved,
// rank-1 update of the columns after J.  A template chain, so that every
// register index is a compile-time constant.
template <int J>
__device__ __forceinline__ void chol_col(float (&a)[32], int lane, bool& failed) {
  if constexpr (J < 32) {
    float p = __shfl_sync(0xffffffffu, a[J], J);
    if (!(p > 0.0f)) { failed = true; p = 1.0f; }
    const float piv = sqrtf(p);
    const float l = lane > J ? __fdiv_rn(a[J], piv) : (lane == J ? piv : a[J]);
    a[J] = l;
#pragma unroll
    for (int c = J + 1; c < 32; ++c) {
      const float lcj = __shfl_sync(0xffffffffu, l, c);
      if (lane >= c) a[c] -= l * lcj;
    }
    chol_col<J + 1>(a, lane, failed);
  }
}

// Cholesky factor and inverse of the 32x32 diagonal sub-block at (o, o) of S
// (row stride PLD) by one warp, written back as L into S and as L^-1 into X.
//   factor:  lane i holds row i in registers (every index known at compile
//            time); right-looking, one column per step, the pivot and the
//            solved column broadcast by shuffles -- no barriers;
//   inverse: lane c solves column c of L^-1 by forward substitution, reading
//            the rows of L from shared memory (every lane the same address).
// Both follow the element-wise order of the textbook loops (each element's
// updates in increasing column order), and rows / columns >= sz are padded
// with the identity.
__device__ __forceinline__ void warp_chol_inv32(float* S, float* X, int o, int sz, int* bad) {
  const int lane = threadIdx.x & 31;
  float a[32];
#pragma unroll
  for (int c = 0; c < 32; ++c)
    a[c] = (lane < sz && c < sz) ? (c <= lane ? S[(o + lane) * PLD + o + c] : 0.0f) : (lane == c ? 1.0f : 0.0f);
  bool failed = false;
  chol_col<0>(a, lane, failed);
  if (failed && lane == 0) *bad = 1;
  if (lane < sz) {
#pragma unroll
    for (int c = 0; c < 32; ++c)
      if (c <= lane) S[(o + lane) * PLD + o + c] = a[c];
  }
  __syncwarp();
  // padded rows of L are the identity: read them as such
  float x[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    float acc = (i == lane) ? 1.0f : 0.0f;
    const float* Li = S + (o + i) * PLD + o;
#pragma unroll
    for (int k = 0; k < i; ++k) acc -= (i < sz ? Li[k] : 0.0f) * x[k];
    x[i] = __fdiv_rn(acc, i < sz ? Li[i] : 1.0f);
  }
  if (lane < sz) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      if (i >= lane && i < sz) X[(o + i) * PLD + o + lane] = x[i];
  }
}

__global__ void __launch_bounds__(512) k_potrf_diag(float* B, int64_t ld, int64_t k0, int n, float* Linv,
                                                    int* status) {
  // Blocked in 32-column sub-steps: one warp factors and inverts each 32x32
  // diagonal sub-block (warp_chol_inv32), then all 16 warps apply the panel
  // solve and the trailing update; the off-diagonal blocks of the inverse
  // follow block-row by block-row.
  extern __shared__ float sm[];
  float* S = sm;             // [PB][PLD]  L of this block (lower)
  float* X = sm + PB * PLD;  // [PB][PLD]  its inverse (lower)
  __shared__ int bad;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  constexpr int NW = 16, SB = 32;
  if (t == 0) bad = 0;
  // stage the lower triangle: all of a thread's loads are issued before its stores
  {
    float v[PB / NW][PB / 32];
#pragma unroll
    for (int a = 0; a < PB / NW; ++a)
#pragma unroll
      for (int b = 0; b < PB / 32; ++b) {
        const int i = warp + a * NW, j = lane + b * 32;
        v[a][b] = (i < n && j <= i) ? B[(k0 + i) * ld + k0 + j] : 0.f;
      }
#pragma unroll
    for (int a = 0; a < PB / NW; ++a)
#pragma unroll
      for (int b = 0; b < PB / 32; ++b) {
        const int i = warp + a * NW, j = lane + b * 32;
        S[i * PLD + j] = v[a][b];
        X[i * PLD + j] = 0.f;
      }
  }
  __syncthreads();
  const int nsub = (n + SB - 1) / SB;
  for (int kb = 0; kb < nsub; ++kb) {
    const int o = kb * SB, sz = min(SB, n - o);
    if (warp == 0) warp_chol_inv32(S, X, o, sz, &bad);
    __syncthreads();
    const int r0 = o + sz, rem = n - r0;
    if (rem <= 0) break;
    // (3) panel: L21 = A21 * X11^T.  Lane c keeps row c of X11 in registers;
    // warps take the rows (at most 96 = 16 warps x 6).
    {
      float xr[32];
#pragma unroll
      for (int l = 0; l < 32; ++l) xr[l] = (l <= lane && lane < sz) ? X[(o + lane) * PLD + o + l] : 0.f;
      float v[6];
#pragma unroll
      for (int k = 0; k < 6; ++k) {
        const int r = r0 + warp + NW * k;
        float acc = 0.f;
        if (r < n) {
#pragma unroll
          for (int l = 0; l < 32; ++l) acc = fmaf(S[r * PLD + o + l], xr[l], acc);
        }
        v[k] = acc;
      }
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 6; ++k) {
        const int r = r0 + warp + NW * k;
        if (r < n && lane < sz) S[r * PLD + o + lane] = v[k];
      }
      __syncthreads();
    }
    // (4) trailing update of the lower triangle: A22 -= L21 L21^T.  Lane
    // keeps row l of L21 in registers; warps take the rows r >= l.
#pragma unroll
    for (int m = 0; m < 3; ++m) {
      const int l = r0 + lane + 32 * m;
      float lr[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) lr[c] = (l < n && c < sz) ? S[l * PLD + o + c] : 0.f;
#pragma unroll
      for (int k = 0; k < 6; ++k) {
        const int r = r0 + warp + NW * k;
        if (r < n && l <= r) {
          float acc = 0.f;
#pragma unroll
          for (int c = 0; c < 32; ++c) acc = fmaf(S[r * PLD + o + c], lr[c], acc);
          S[r * PLD + l] -= acc;
        }
      }
    }
    __syncthreads();
  }
  if (t == 0 && bad && status) atomicMax(status, (int)LLMC_ENOT_PD);
  // off-diagonal blocks of the inverse, by block row bi:
  //   T = L[rows of bi, :oi] * X[:oi, :oi],  X[rows of bi, :oi] = -X_ii * T.
  // A thread holds 2 rows x 3 columns of the block row (16 warps x 32 lanes);
  // X is zero above its diagonal, so every sum runs over the full range.
  for (int bi = 1; bi < nsub; ++bi) {
    const int oi = bi * SB, szi = min(SB, n - oi);
    const int r0 = warp, r1 = warp + NW;
    float acc[2][3];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int v = 0; v < 3; ++v) acc[u][v] = 0.f;
    for (int k = 0; k < oi; ++k) {
      const float l0 = S[(oi + r0) * PLD + k], l1 = S[(oi + r1) * PLD + k];
#pragma unroll
      for (int v = 0; v < 3; ++v) {
        const int c = lane + 32 * v;
        const float xk = (c < oi) ? X[k * PLD + c] : 0.f;
        acc[0][v] = fmaf(l0, xk, acc[0][v]);
        acc[1][v] = fmaf(l1, xk, acc[1][v]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int v = 0; v < 3; ++v) {
      const int c = lane + 32 * v;
      if (c < oi) {
        if (r0 < szi) X[(oi + r0) * PLD + c] = acc[0][v];
        if (r1 < szi) X[(oi + r1) * PLD + c] = acc[1][v];
      }
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int v = 0; v < 3; ++v) acc[u][v] = 0.f;
    for (int m = 0; m < szi; ++m) {
      const float x0 = X[(oi + r0) * PLD + oi + m], x1 = X[(oi + r1) * PLD + oi + m];
#pragma unroll
      for (int v = 0; v < 3; ++v) {
        const int c = lane + 32 * v;
        const float tm = (c < oi) ? X[(oi + m) * PLD + c] : 0.f;
        acc[0][v] = fmaf(x0, tm, acc[0][v]);
        acc[1][v] = fmaf(x1, tm, acc[1][v]);
      }
    }
    __syncthreads();
#pragma unroll
    for (int v = 0; v < 3; ++v) {
      const int c = lane + 32 * v;
      if (c < oi) {
        if (r0 < szi) X[(oi + r0) * PLD + c] = -acc[0][v];
        if (r1 < szi) X[(oi + r1) * PLD + c] = -acc[1][v];
      }
    }
    __syncthreads();
  }
  for (int i = warp; i < PB; i += NW)
    for (int j = lane; j < PB; j += 32) {
      const bool in = i < n && j < n && j <= i;
      Linv[i * PB + j] = in ? X[i * PLD + j] : 0.f;
      if (in) B[(k0 + i) * ld + k0 + j] = S[i * PLD + j];
    }
}

__global__ void k_eye(float* X, int64_t d) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < d) X[i * d + i] = 1.0f;
}

__global__ void k_copy2d(const float* __restrict__ src, int64_t lds, float* __restrict__ dst, int64_t ldd, int rows,
                         int cols) {
  const int r = blockIdx.y;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x)
    if (r < rows) dst[(int64_t)r * ldd + c] = src[(int64_t)r * lds + c];
}

// ---------------------------------------------------------------------------
// GPTQ column loop over one 128-column block
// ---------------------------------------------------------------------------
constexpr int QB = 128;     // GPTQ block size handled by the kernel
// Columns whose errors are applied together beyond them: after each QB-column
// block only the rest of its QOB-column outer block is updated; the columns
// after the outer block get one update with K = QOB (the same lazy-batch
// argument that lets GPTQ defer updates across blocks: exact in exact terms),
// which reads and writes the rest of W a quarter as often.
constexpr int QOB = 4 * QB;
constexpr int SUB = 32;     // sub-block held in registers
constexpr int CH = 8;       // columns per unrolled chunk of the sub-block
constexpr int ROWS = 64;    // rows (threads) per CTA
constexpr int QS_LD = QB + 1;

// quantized value types of the fake-quantization step
enum { QF_INT = 0, QF_FP8 = 1, QF_FP4 = 2 };

struct BlockArgs {
  float* W;            // r x c float32 working weight
  int64_t r, c;
  int i1, count;
  const float* U;      // c x c upper factor
  const uint16_t* scale;  // bf16 scales: tensor (1), channel (r,1), group (r, c/gs)
  const int8_t* zp;       // optional
  int strategy;
  int64_t gs;
  float qmin, qmax;
  float* err;          // row-major errors (row stride eld); this block's start at column ecol
  int64_t eld, ecol;
  float* loss;         // r per-row losses
  const int* status;   // ENOT_PD -> identity
  // per-column variant (k_gptq_block<true>) only:
  const float* scale_f;   // float32 scales instead of `scale`
  const float* gsc;       // global scale (device scalar): effective scale = scale / gsc
  int qf;                 // QF_*
  int f32deq;             // dequantize in float32 (float32 scales) instead of bf16
  const int32_t* perm;    // activation ordering WEIGHT: the group of solve column j is that of perm[j]
  int64_t gdiv;           // columns per scale column (group size, block width; 0: one scale column)
  int64_t rdiv;           // rows per scale row (1, block height; 0: one scale row)
  int64_t sld;            // scale columns per scale row
};

__device__ __forceinline__ void scale_of(const BlockArgs& a, int64_t row, int col, float& s, float& z) {
  int64_t idx;
  if (a.strategy == LLMC_STRAT_TENSOR) idx = 0;
  else if (a.strategy == LLMC_STRAT_CHANNEL) idx = row;
  else idx = row * (a.c / a.gs) + col / a.gs;
  s = bf16_to_f(a.scale[idx]);
  z = a.zp ? (float)a.zp[idx] : 0.0f;
}

// Correctly rounded x / y from r = RN(1/y) (Markstein's correction: with r
// the correctly rounded reciprocal and x*r within an ulp of x/y, one fma
// residual and one fma step give RN(x/y) when nothing overflows or
// underflows).  Callers use it only where 1/y is a normal float.
__device__ __forceinline__ float div_mk(float x, float y, float r) {
  // on -x, so that x = +-0 keeps its sign through the correction (y > 0)
  const float q0 = __fmul_rn(-x, -r);
  const float e = __fmaf_rn(q0, y, -x);
  return __fmaf_rn(e, -r, q0);
}
__device__ __forceinline__ bool recip_ok(float r) { return r > 1.0e-30f && r < 1.0e30f; }

// fake_quantize of one float32 value with a bf16 scale (CT forward_helpers.py:175-210):
// float32 quotient, + zp, clamp, round half-even, -> bf16, - zp, * scale rounded to bf16.
__device__ __forceinline__ float fake_quant(float w, float s, float rs, bool fast, float z, float qmin, float qmax) {
  float q = (fast ? div_mk(w, s, rs) : __fdiv_rn(w, s)) + z;
  q = rintf(fminf(fmaxf(q, qmin), qmax));
  float deq = rbf(q - z);
  return rbf(deq * s);
}

// perm[j], kept inside [0, c) so that a caller's malformed permutation
// cannot send a load or store out of bounds (it gives wrong results instead)
__device__ __forceinline__ int64_t perm_at(const int32_t* perm, int64_t j, int64_t c) {
  const int64_t p = perm[j];
  return p < 0 ? 0 : (p >= c ? c - 1 : p);
}

// E2M1 grid value of a code from e2m1_code (magnitude index, sign bit 8)
__device__ __forceinline__ float fp4_grid(uint32_t code) {
  const uint32_t m = code & 7u;
  const float v = (m < 4u) ? 0.5f * (float)m : (m == 4u) ? 2.0f : (m == 5u) ? 3.0f : (m == 6u) ? 4.0f : 6.0f;
  return (code & 8u) ? -v : v;
}

// fake_quantize of one float32 value for every quantized type
// (CT forward_helpers.py _quantize_dequantize): float32 quotient, + zp,
// clamp, round (half-even integer, RNE E4M3 cast, cast_to_fp4 thresholds),
// back to the scale's dtype, - zp, times the scale: bf16 products for bf16
// scales, float32 for float32 scales (NVFP4's effective scale
// scale / global_scale, or statistics observed in float32).
__device__ __forceinline__ float fake_quant_any(float w, float s, float rs, bool fast, float z, float qmin, float qmax,
                                               int qf, bool f32deq) {
  float q = (fast ? div_mk(w, s, rs) : __fdiv_rn(w, s)) + z;
  q = fminf(fmaxf(q, qmin), qmax);
  if (qf == QF_INT) q = rintf(q);
  else if (qf == QF_FP8) q = round_e4m3(q);
  else q = fp4_grid(e2m1_code(q));
  if (f32deq) return __fmul_rn(q - z, s);
  return rbf(rbf(q - z) * s);
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// One 128-column GPTQ block for ROWS rows per CTA, one row per thread.  The
// block's factor rows (64 KB) are staged with asynchronous 16-byte copies and
// the rows of W with batched vector loads, so staging costs a few memory
// round trips; the 32 columns of a sub-block live in registers with every
// index known at compile time; divisions use per-column reciprocals.
//
// PERCOL = true: every column looks up its own scale and zero point (loaded
// eight columns ahead), for activation ordering, block scales, float32
// scales and the FP8 / FP4 types; PERCOL = false: integer types with bf16
// scales in column order, the scale reloaded only where a group starts.
template <bool PERCOL>
__global__ void __launch_bounds__(ROWS, 2) k_gptq_block(BlockArgs a) {
  extern __shared__ float sm[];
  float* U1 = sm;                  // [QB][QB]
  float* QS = U1 + QB * QB;        // [ROWS][QS_LD]
  float* RD = QS + ROWS * QS_LD;   // [QB]  RN(1/d)
  float* D2 = RD + QB;             // [QB]  RN(d*d)
  float* RD2 = D2 + QB;            // [QB]  RN(1/(d*d))
  int* G = (int*)(RD2 + QB);       // [QB]  scale column of each column (PERCOL)
  const int t = threadIdx.x;
  const int64_t row0 = (int64_t)blockIdx.x * ROWS;
  const int64_t row = row0 + t;
  const bool identity = a.status && *a.status == LLMC_ENOT_PD;
  const int cnt = a.count;
  // rows of U and W start on 16-byte boundaries
  const bool vec = (a.c % 4) == 0 && ((uintptr_t)a.U % 16) == 0 && ((uintptr_t)a.W % 16) == 0;

  if (identity || !vec || cnt < QB) {
    for (int e = t; e < QB * QB; e += ROWS) {
      const int i = e / QB, j = e % QB;
      float v = 0.f;
      if (i < cnt && j < cnt) v = identity ? (i == j ? 1.f : 0.f) : a.U[(int64_t)(a.i1 + i) * a.c + a.i1 + j];
      U1[e] = v;
    }
  } else {
    for (int e = t; e < QB * QB / 4; e += ROWS) {
      const int i = e >> 5, j4 = (e & 31) * 4;
      cp_async16(U1 + i * QB + j4, a.U + (int64_t)(a.i1 + i) * a.c + a.i1 + j4);
    }
  }
  // rows of W: 8 independent 16-byte loads in flight per thread
  constexpr int PER = ROWS * QB / 4 / ROWS;  // float4 per thread (32)
#pragma unroll
  for (int b0 = 0; b0 < PER; b0 += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = (b0 + u) * ROWS + t;
      const int rr = e >> 5, j4 = (e & 31) * 4;
      const int64_t gr = row0 + rr;
      v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gr < a.r) {
        const float* src = a.W + gr * a.c + a.i1 + j4;
        if (vec && j4 + 4 <= cnt) v[u] = *(const float4*)src;
        else {
          if (j4 + 0 < cnt) v[u].x = src[0];
          if (j4 + 1 < cnt) v[u].y = src[1];
          if (j4 + 2 < cnt) v[u].z = src[2];
          if (j4 + 3 < cnt) v[u].w = src[3];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = (b0 + u) * ROWS + t;
      float* d = QS + (e >> 5) * QS_LD + (e & 31) * 4;
      d[0] = v[u].x; d[1] = v[u].y; d[2] = v[u].z; d[3] = v[u].w;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  for (int i = t; i < QB; i += ROWS) {
    const float d = U1[i * QB + i];
    const float d2 = __fmul_rn(d, d);
    RD[i] = __frcp_rn(d);
    D2[i] = d2;
    RD2[i] = __frcp_rn(d2);
    if (PERCOL) {
      const int64_t col = a.i1 + i;
      const int64_t src = (a.perm && col < a.c) ? perm_at(a.perm, col, a.c) : col;
      G[i] = a.gdiv > 0 ? (int)(src / a.gdiv) : 0;
    }
  }
  __syncthreads();

  float loss = 0.f;
  if (row < a.r) {
    float s = 0.f, z = 0.f, rs = 0.f;
    bool sfast = false;
    int64_t next_g = -1;  // first column of the next scale group
    const int64_t rowpart = PERCOL ? (a.rdiv > 0 ? row / a.rdiv : 0) * a.sld : 0;
    const float gsv = (PERCOL && a.gsc) ? *a.gsc : 1.0f;
    for (int s0 = 0; s0 < cnt; s0 += SUB) {
      // w[j]: column s0 + c8 + j of this row (a window that shifts left by CH
      // columns per chunk), e: the sub-block's errors in column order.  The
      // chunk body is the same for every c8, which keeps the code small
      // enough for the instruction cache.
      float w[SUB], e[SUB];
#pragma unroll
      for (int j = 0; j < SUB; ++j) { w[j] = QS[t * QS_LD + s0 + j]; e[j] = 0.f; }
      const int n = min(SUB, cnt - s0);
      for (int c8 = 0; c8 < SUB; c8 += CH) {
        float ebuf[CH];
        float sk[CH], zk[CH];
        if (PERCOL) {  // this chunk's scales, all loads in flight together
#pragma unroll
          for (int k = 0; k < CH; ++k) {
            sk[k] = 1.0f; zk[k] = 0.0f;
            if (c8 + k < n) {
              const int64_t idx = rowpart + G[s0 + c8 + k];
              sk[k] = a.scale_f ? a.scale_f[idx] : bf16_to_f(a.scale[idx]);
              zk[k] = a.zp ? (float)a.zp[idx] : 0.0f;
            }
          }
          if (a.gsc) {
#pragma unroll
            for (int k = 0; k < CH; ++k) sk[k] = __fdiv_rn(sk[k], gsv);
          }
        }
#pragma unroll
        for (int k = 0; k < CH; ++k) {
          const int ii = c8 + k;
          float err = 0.f;
          if (ii < n) {
            const int i = s0 + ii;
            const int col = a.i1 + i;
            const float d = U1[i * QB + i];
            const float wi = w[k];
            float q;
            if (PERCOL) {
              s = sk[k]; z = zk[k];
              rs = __frcp_rn(s);
              sfast = s > 0.0f && recip_ok(rs);
              q = fake_quant_any(wi, s, rs, sfast, z, a.qmin, a.qmax, a.qf, a.f32deq != 0);
            } else {
              if (col >= next_g) {
                scale_of(a, row, col, s, z);
                rs = __frcp_rn(s);
                sfast = recip_ok(rs);
                next_g = (a.strategy == LLMC_STRAT_GROUP) ? (col / a.gs + 1) * a.gs : (int64_t)1 << 62;
              }
              q = fake_quant(wi, s, rs, sfast, z, a.qmin, a.qmax);
            }
            QS[t * QS_LD + i] = q;
            const float diff = wi - q;
            const bool dfast = recip_ok(RD[i]) && recip_ok(RD2[i]);
            const float dd = __fmul_rn(diff, diff);
            loss += dfast ? div_mk(dd, D2[i], RD2[i]) : __fdiv_rn(dd, D2[i]);
            err = dfast ? div_mk(diff, d, RD[i]) : __fdiv_rn(diff, d);
            const float* urow = U1 + i * QB + s0 + c8;
#pragma unroll
            for (int j = k + 1; j < SUB; ++j)
              if (c8 + j < SUB) w[j] -= err * urow[j];
          }
          ebuf[k] = err;
        }
#pragma unroll
        for (int j = 0; j < SUB - CH; ++j) { w[j] = w[j + CH]; e[j] = e[j + CH]; }
#pragma unroll
        for (int k = 0; k < CH; ++k) { w[SUB - CH + k] = 0.f; e[SUB - CH + k] = ebuf[k]; }
      }
      // this sub-block's errors, row-major (rows x 128), as the K-major operand of the trailing update
      float4* erow = (float4*)(a.err + row * a.eld + a.ecol + s0);
#pragma unroll
      for (int j = 0; j < SUB / 4; ++j) erow[j] = make_float4(e[4 * j], e[4 * j + 1], e[4 * j + 2], e[4 * j + 3]);
      // lazy update of the later columns of this block, four columns at a time
      for (int j = s0 + SUB; j < cnt; j += 4) {
        float acc0 = 0.f, acc1 = 0.f, acc2 = 0.f, acc3 = 0.f;
#pragma unroll
        for (int ii = 0; ii < SUB; ++ii) {
          const float4 u = *(const float4*)(U1 + (s0 + ii) * QB + j);  // one broadcast 16-byte read
          acc0 = fmaf(e[ii], u.x, acc0);
          acc1 = fmaf(e[ii], u.y, acc1);
          acc2 = fmaf(e[ii], u.z, acc2);
          acc3 = fmaf(e[ii], u.w, acc3);
        }
        QS[t * QS_LD + j] -= acc0;
        QS[t * QS_LD + j + 1] -= acc1;
        QS[t * QS_LD + j + 2] -= acc2;
        QS[t * QS_LD + j + 3] -= acc3;
      }
    }
    a.loss[row] += loss / 2.0f;
  }
  __syncthreads();
  // write the quantized block back (coalesced)
  for (int e = t; e < ROWS * QB; e += ROWS) {
    const int rr = e / QB, j = e % QB;
    const int64_t gr = row0 + rr;
    if (gr < a.r && j < cnt) a.W[gr * a.c + a.i1 + j] = QS[rr * QS_LD + j];
  }
}

// W (float32, solve column order) from the bf16 weight; solve column j is
// weight column perm[j] (activation ordering) and dead columns are zero.
__global__ void k_init_w(const uint16_t* __restrict__ w, float* __restrict__ W, int64_t r, int64_t c,
                         const uint8_t* dead, const int32_t* perm) {
  const int64_t n = r * c;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t col = i % c;
    const int64_t src = perm ? (i - col) + perm_at(perm, col, c) : i;
    W[i] = (dead && dead[col]) ? 0.0f : bf16_to_f(w[src]);
  }
}

__global__ void k_finish(const float* __restrict__ W, uint16_t* __restrict__ out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = f_to_bf16(W[i]);
}

// back to the weight's column order: out[:, perm[j]] = W[:, j]
__global__ void k_finish_perm(const float* __restrict__ W, uint16_t* __restrict__ out, int64_t r, int64_t c,
                              const int32_t* __restrict__ perm) {
  const int64_t n = r * c;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t col = i % c;
    out[(i - col) + perm_at(perm, col, c)] = f_to_bf16(W[i]);
  }
}

// g_idx of activation ordering GROUP (S/modifiers/gptq/gptq_quantize.py:166,292-293):
// weight column perm[j] belongs to group j / gs
__global__ void k_gidx_group(const int32_t* __restrict__ perm, int64_t c, int64_t gs, int32_t* __restrict__ g_idx) {
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < c; j += (int64_t)gridDim.x * blockDim.x)
    g_idx[perm_at(perm, j, c)] = (int32_t)(j / gs);
}

// Activation order (S/modifiers/gptq/gptq_quantize.py:299-310,
// torch.argsort(diag(H), descending=True)): perm[rank] = i with rank = the
// number of diagonal entries that sort before entry i -- larger values
// first, equal values in index order.  Keys are the float bits made
// monotonic (every value, NaN included, gets a distinct total order), so
// the ranks are a permutation of 0..d-1.
__device__ __forceinline__ uint32_t desc_key(float f) {
  if (f == 0.0f) f = 0.0f;  // -0 ties with +0
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__global__ void __launch_bounds__(256) k_actorder_perm(const float* __restrict__ H, int64_t d, int32_t* __restrict__ perm) {
  __shared__ uint32_t keys[256];
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t ki = i < d ? desc_key(H[i * d + i]) : 0u;
  int64_t rank = 0;
  for (int64_t t0 = 0; t0 < d; t0 += 256) {
    __syncthreads();
    const int64_t j = t0 + threadIdx.x;
    keys[threadIdx.x] = j < d ? desc_key(H[j * d + j]) : 0u;
    __syncthreads();
    const int m = (d - t0) < 256 ? (int)(d - t0) : 256;
    for (int jj = 0; jj < m; ++jj) {
      const uint32_t kj = keys[jj];
      rank += (kj > ki) || (kj == ki && t0 + jj < i);
    }
  }
  if (i < d) perm[rank] = (int32_t)i;
}

// Hp = H[perm][:, perm]
__global__ void k_permute_sym(const float* __restrict__ H, int64_t d, const int32_t* __restrict__ perm,
                              float* __restrict__ Hp) {
  const int64_t i = blockIdx.y;
  const float* src = H + perm_at(perm, i, d) * d;
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < d; j += (int64_t)gridDim.x * blockDim.x)
    Hp[i * d + j] = src[perm_at(perm, j, d)];
}

// dst[:, j] = src[:, perm[j]] for 2-byte elements
__global__ void k_permute_cols16(const uint16_t* __restrict__ src, int64_t r, int64_t c, const int32_t* __restrict__ perm,
                                 uint16_t* __restrict__ dst) {
  const int64_t n = r * c;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t col = i % c;
    dst[i] = src[(i - col) + perm_at(perm, col, c)];
  }
}

__global__ void k_sum(const float* __restrict__ x, int64_t n, float* out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) v += red[i];
    *out = v;
  }
}

// cudaFuncSetAttribute is per device: remember which devices have it.
template <typename F>
static bool set_smem_attr(F* fn, int bytes, uint64_t* done_mask) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && (*done_mask >> dev) & 1ull) return true;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  if (dev < 64) *done_mask |= (1ull << dev);
  return true;
}

static unsigned grid_for(int64_t n) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16)); }

}  // namespace gq
}  // namespace llmc

using namespace llmc;
using namespace llmc::gq;

extern "C" {

// workspace: Cholesky working copy B (d*d) + inverse X (d*d) + diag inverses (d*128) + two panels (2 * d*128)
int llmc_gptq_hinv_workspace_size(int64_t d, int64_t* bytes) {
  if (!bytes || d <= 0) return LLMC_EINVAL_ARG;
  const int64_t nbp = ((d + PB - 1) / PB) * PB;
  *bytes = (int64_t)sizeof(float) * (2 * d * d + 3 * nbp * PB) + 256;
  return LLMC_OK;
}

int llmc_gptq_prepare_hessian(float* H, int64_t d, float percdamp, uint8_t* dead, void* stream) {
  if (!H || !dead || d <= 0) return LLMC_EINVAL_ARG;
  k_prep_hessian<<<1, 1024, 0, (cudaStream_t)stream>>>(H, d, percdamp, dead); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

}  // extern "C"

namespace llmc {
namespace gq {

// A side stream of the current device for the lookahead of the
// factorisation (a few per device, handed out in turn so that concurrent
// factorisations on different streams rarely share one).  NULL if none can
// be made: the caller then runs everything on its own stream.
static cudaStream_t side_stream() {
  static std::mutex mu;
  static cudaStream_t pool[64][4] = {};
  static unsigned next[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!pool[dev][0]) {  // all at once: creating a stream inside a timed region would cost there
    for (int k = 0; k < 4; ++k)
      if (cudaStreamCreateWithFlags(&pool[dev][k], cudaStreamNonBlocking) != cudaSuccess) {
        for (int m = 0; m < k; ++m) cudaStreamDestroy(pool[dev][m]);
        for (int m = 0; m < 4; ++m) pool[dev][m] = nullptr;
        return nullptr;
      }
  }
  return pool[dev][next[dev]++ & 3u];
}

// CTAs of a side-stream GEMM: the persistent GEMM keeps one CTA per SM, so
// a full grid would leave no SM for the diagonal kernel and the skinny
// panel GEMMs of the caller's stream until it ends.
constexpr int kSideCtas = 148 - 12;

// Fork/join helper: work put on `side` is ordered after everything already
// on `main`; `join` makes `main` wait for all of it.
struct Lookahead {
  cudaStream_t main = nullptr, side = nullptr;
  cudaEvent_t ev_main = nullptr, ev_side = nullptr;
  bool ok() const { return side != nullptr; }
  int open(cudaStream_t st) {
    main = st;
    side = side_stream();
    if (!side) return LLMC_OK;
    if (cudaEventCreateWithFlags(&ev_main, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ev_side, cudaEventDisableTiming) != cudaSuccess)
      return LLMC_ECUDA;
    if (cudaEventRecord(ev_main, main) != cudaSuccess || cudaStreamWaitEvent(side, ev_main, 0) != cudaSuccess)
      return LLMC_ECUDA;
    return LLMC_OK;
  }
  // main waits for the side work enqueued so far
  int main_waits_side() {
    if (!side) return LLMC_OK;
    return cudaStreamWaitEvent(main, ev_side, 0) == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  // side waits for the main work enqueued so far
  int side_waits_main() {
    if (!side) return LLMC_OK;
    if (cudaEventRecord(ev_main, main) != cudaSuccess) return LLMC_ECUDA;
    return cudaStreamWaitEvent(side, ev_main, 0) == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  int side_done() {
    if (!side) return LLMC_OK;
    return cudaEventRecord(ev_side, side) == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  cudaStream_t side_or_main() const { return side ? side : main; }
  int close() {
    int r = LLMC_OK;
    if (side) {
      if (side_done() || main_waits_side()) r = LLMC_ECUDA;
    }
    if (ev_main) cudaEventDestroy(ev_main);
    if (ev_side) cudaEventDestroy(ev_side);
    ev_main = ev_side = nullptr;
    return r;
  }
};

}  // namespace gq
}  // namespace llmc

extern "C" {

namespace llmc {
namespace gq {
// The factorisation; `lookahead` puts the wide trailing updates on a side
// stream (worth it for large d; the batched solve of many small Hessians
// runs without it, on its own streams).
static int hinv_impl(const float* A, int64_t d, float* Hinv, float* HinvT, void* workspace, int* status,
                     cudaStream_t st, bool lookahead);
}  // namespace gq
}  // namespace llmc

int llmc_gptq_hinv(const float* A, int64_t d, float* Hinv, float* HinvT, void* workspace, int* status,
                   void* stream) {
  if (!A || !Hinv || !workspace || !status || d <= 0) return LLMC_EINVAL_ARG;
  return llmc::gq::hinv_impl(A, d, Hinv, HinvT, workspace, status, (cudaStream_t)stream, true);
}

}  // extern "C"

namespace llmc {
namespace gq {
static int hinv_impl(const float* A, int64_t d, float* Hinv, float* HinvT, void* workspace, int* status,
                     cudaStream_t st, bool lookahead) {
  const int64_t nb = (d + PB - 1) / PB;
  float* B = (float*)workspace;
  float* X = B + d * d;
  float* LinvD = X + d * d;             // nb blocks of PB x PB
  float* T0 = LinvD + nb * PB * PB;     // panel scratch, up to d x PB, double-buffered
  float* T1 = T0 + nb * PB * PB;
  static uint64_t attr_mask = 0;
  if (!set_smem_attr(k_potrf_diag, 2 * PB * (PB + 1) * (int)sizeof(float), &attr_mask)) return LLMC_ECUDA;
  dim3 rg((unsigned)((d + 255) / 256), (unsigned)d);
  k_reverse<<<rg, 256, 0, st>>>(A, B, d); llmc::note_launch();
  // Blocked lower Cholesky of B = J A J with a lookahead of one panel: after
  // panel k is solved, the caller's stream updates only the next block
  // column (a) and goes on to factor it, while the rest of the trailing
  // update (b) runs on a side stream.  (a) of panel k + 1 waits for (b) of
  // panel k (both write the block column after it); the panel buffers
  // alternate so that (b) still reads its own panel.
  Lookahead la;
  la.main = st;
  if (lookahead && la.open(st)) return LLMC_ECUDA;
  int k = 0;
  for (int64_t kb0 = 0; kb0 < d; kb0 += PB, ++k) {
    const int kb = (int)std::min<int64_t>(PB, d - kb0);
    float* Ld = LinvD + (kb0 / PB) * PB * PB;
    float* T = (k & 1) ? T1 : T0;
    k_potrf_diag<<<1, 512, 2 * PB * (PB + 1) * sizeof(float), st>>>(B, d, kb0, kb, Ld, status); llmc::note_launch();
    const int rem = (int)(d - kb0 - kb);
    if (rem > 0) {
      // T = B[kb0+kb:, kb0:kb0+kb] * Linv_kk^T, then the panel back into B
      GemmArgs g1 = {rem, kb, kb, B + (kb0 + kb) * d + kb0, d, Ld, PB, T, PB, 0, 0, 0, nullptr, 0, status};
      if (launch_gemm(false, true, g1, st)) return LLMC_ECUDA;
      k_copy2d<<<dim3(1, rem), 128, 0, st>>>(T, PB, B + (kb0 + kb) * d + kb0, d, rem, kb); llmc::note_launch();
      // (a) the next block column: B[kb0+kb:, kb0+kb : +kn] -= T T[:kn]^T
      const int kn = std::min(PB, rem);
      if (la.main_waits_side()) return LLMC_ECUDA;
      GemmArgs ga = {rem, kn, kb, T, PB, T, PB, B + (kb0 + kb) * d + kb0 + kb, d, 1, 0, 0, nullptr, 0, status};
      if (launch_gemm(false, true, ga, st)) return LLMC_ECUDA;
      // (b) the rest of the lower trailing block, on the side stream
      if (rem > kn) {
        if (la.side_waits_main()) return LLMC_ECUDA;
        const int64_t o = kb0 + kb + kn;
        GemmArgs gb = {rem - kn, rem - kn, kb, T + (int64_t)kn * PB, PB, T + (int64_t)kn * PB, PB, B + o * d + o, d,
                       1, 1, 0, nullptr, kSideCtas, status};
        if (launch_gemm(false, true, gb, la.side_or_main())) return LLMC_ECUDA;
        if (la.side_done()) return LLMC_ECUDA;
      }
    }
  }
  // Xt = L^-T (upper), by right-looking blocked substitution on column blocks of Xt = I:
  //   Xt[:, i] = Xt[:, i] * Linv_ii^T,   Xt[:, >i] -= Xt[:, i] * L[>i, i]^T
  // -- every update is an A * B^T product with K = 128 (both operands K-major).
  // The same lookahead: the next column block is updated on the caller's
  // stream, the remaining columns on the side stream.
  float* Xt = X;
  if (la.main_waits_side()) return LLMC_ECUDA;
  if (cudaMemsetAsync(Xt, 0, sizeof(float) * d * d, st) != cudaSuccess) return LLMC_ECUDA;
  k_eye<<<(unsigned)((d + 255) / 256), 256, 0, st>>>(Xt, d); llmc::note_launch();
  for (int64_t i0 = 0; i0 < d; i0 += PB) {
    const int ib = (int)std::min<int64_t>(PB, d - i0);
    const int nc = (int)(i0 + ib);  // rows of Xt that can be non-zero in these columns
    const float* Ld = LinvD + (i0 / PB) * PB * PB;
    k_copy2d<<<dim3(1, nc), 128, 0, st>>>(Xt + i0, d, T0, PB, nc, ib); llmc::note_launch();
    GemmArgs g1 = {nc, ib, ib, T0, PB, Ld, PB, Xt + i0, d, 0, 0, 0, nullptr, 0, status};
    if (launch_gemm(false, true, g1, st)) return LLMC_ECUDA;
    const int rem = (int)(d - i0 - ib);
    if (rem > 0) {
      const int kn = std::min(PB, rem);
      if (la.main_waits_side()) return LLMC_ECUDA;
      GemmArgs ga = {nc, kn, ib, Xt + i0, d, B + (i0 + ib) * d + i0, d, Xt + i0 + ib, d, 1, 0, 0, nullptr, 0, status};
      if (launch_gemm(false, true, ga, st)) return LLMC_ECUDA;
      if (rem > kn) {
        if (la.side_waits_main()) return LLMC_ECUDA;
        const int64_t o = i0 + ib + kn;
        GemmArgs gb = {nc, rem - kn, ib, Xt + i0, d, B + o * d + i0, d, Xt + o, d, 1, 0, 0, nullptr, kSideCtas, status};
        if (launch_gemm(false, true, gb, la.side_or_main())) return LLMC_ECUDA;
        if (la.side_done()) return LLMC_ECUDA;
      }
    }
  }
  if (la.close()) return LLMC_ECUDA;
  k_xt_to_u<<<dim3((unsigned)((d + 31) / 32), (unsigned)((d + 31) / 32)), dim3(32, 8), 0, st>>>(Xt, Hinv, d);
  llmc::note_launch();
  if (HinvT) { k_xt_to_ut<<<rg, 256, 0, st>>>(Xt, HinvT, d); llmc::note_launch(); }
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}
}  // namespace gq
}  // namespace llmc

extern "C" {

int llmc_gptq_quantize_workspace_size(int64_t rows, int64_t cols, int64_t* bytes) {
  if (!bytes || rows < 0 || cols < 0) return LLMC_EINVAL_ARG;
  *bytes = (int64_t)sizeof(float) * (rows * cols + (int64_t)QOB * rows + rows + 4) + 256;
  return LLMC_OK;
}

int llmc_gptq_quantize_ex(const void* w_bf16, int64_t rows, int64_t cols, const float* Hinv, const float* HinvT,
                          const uint8_t* dead, const LlmcQuantArgs* args, const void* scale, const int8_t* zp,
                          const LlmcGptqColumns* cx, int64_t blocksize, void* wq_bf16, float* loss_out,
                          void* workspace, int* status, void* stream) {
  if (!args || !Hinv || !loss_out || !workspace || rows < 0 || cols <= 0 || blocksize < 1) return LLMC_EINVAL_ARG;
  const LlmcGptqColumns none = {};
  const LlmcGptqColumns& x = cx ? *cx : none;
  QArgs q = to_qargs(*args);
  if (q.strategy != LLMC_STRAT_TENSOR && q.strategy != LLMC_STRAT_CHANNEL && q.strategy != LLMC_STRAT_GROUP &&
      q.strategy != LLMC_STRAT_TENSOR_GROUP && q.strategy != LLMC_STRAT_BLOCK)
    return LLMC_ENOSUPPORT;
  if (q.is_float && (q.bits != 8 && q.bits != 4)) return LLMC_ENOSUPPORT;
  if (!q.is_float && (q.bits < 2 || q.bits > 8)) return LLMC_ENOSUPPORT;
  if (q.is_float && !q.symmetric && q.bits == 4) return LLMC_ENOSUPPORT;  // asymmetric FP4
  const bool grouped = q.strategy == LLMC_STRAT_GROUP || q.strategy == LLMC_STRAT_TENSOR_GROUP;
  if (grouped && (q.group <= 0 || cols % q.group)) return LLMC_EINVAL_SHAPE;
  if (q.strategy == LLMC_STRAT_BLOCK && (q.bh <= 0 || q.bw <= 0)) return LLMC_EINVAL_ARG;
  if (q.strategy == LLMC_STRAT_TENSOR_GROUP && !x.global_scale) return LLMC_EINVAL_ARG;
  if (x.order < 0 || x.order > 2 || (x.order != 0 && !x.perm)) return LLMC_EINVAL_ARG;
  if (x.order == 2 && (!grouped || !x.g_idx_out)) return LLMC_EINVAL_ARG;
  if (!scale && rows > 0) return LLMC_EINVAL_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (x.order == 2) {
    k_gidx_group<<<grid_for(cols), 256, 0, st>>>(x.perm, cols, q.group, x.g_idx_out); llmc::note_launch();
  }
  if (rows == 0) {
    return cudaMemsetAsync(loss_out, 0, sizeof(float), st) == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  if ((uintptr_t)workspace % 16) return LLMC_EINVAL_ARG;
  // the per-column kernel for everything but integer types with bf16 scales in column order
  const bool percol = q.is_float || x.order != 0 || x.scale_is_f32 || x.global_scale ||
                      q.strategy == LLMC_STRAT_TENSOR_GROUP || q.strategy == LLMC_STRAT_BLOCK;
  float* W = (float*)workspace;
  float* E = W + ((rows * cols + 3) & ~(int64_t)3);  // 16-byte aligned rows for the vector stores
  float* L = E + (int64_t)QOB * rows;
  k_init_w<<<grid_for(rows * cols), 256, 0, st>>>((const uint16_t*)w_bf16, W, rows, cols, dead, x.perm);
  llmc::note_launch();
  if (cudaMemsetAsync(L, 0, sizeof(float) * rows, st) != cudaSuccess) return LLMC_ECUDA;
  static uint64_t attr_mask[2] = {0, 0};
  const int smem = (QB * QB + ROWS * QS_LD + 4 * QB) * (int)sizeof(float);
  if (!set_smem_attr(k_gptq_block<false>, smem, &attr_mask[0])) return LLMC_ECUDA;
  if (!set_smem_attr(k_gptq_block<true>, smem, &attr_mask[1])) return LLMC_ECUDA;
  BlockArgs ba = {};
  ba.W = W; ba.r = rows; ba.c = cols; ba.U = Hinv;
  ba.zp = q.symmetric ? nullptr : zp;
  ba.strategy = q.strategy; ba.gs = q.group > 0 ? q.group : 1;
  ba.qmin = q.qmin(); ba.qmax = q.qmax();
  ba.err = E; ba.loss = L; ba.status = status;
  const bool f32s = x.scale_is_f32 || x.global_scale;
  ba.scale = f32s ? nullptr : (const uint16_t*)scale;
  ba.scale_f = f32s ? (const float*)scale : nullptr;
  ba.gsc = x.global_scale;
  ba.qf = !q.is_float ? QF_INT : (q.bits == 8 ? QF_FP8 : QF_FP4);
  ba.f32deq = f32s ? 1 : 0;
  ba.perm = x.order == 1 ? x.perm : nullptr;  // GROUP ordering: scale groups follow the solve order
  switch (q.strategy) {
    case LLMC_STRAT_TENSOR: ba.gdiv = 0; ba.rdiv = 0; ba.sld = 0; break;
    case LLMC_STRAT_CHANNEL: ba.gdiv = 0; ba.rdiv = 1; ba.sld = 1; break;
    case LLMC_STRAT_BLOCK: ba.gdiv = q.bw; ba.rdiv = q.bh; ba.sld = (cols + q.bw - 1) / q.bw; break;
    default: ba.gdiv = q.group; ba.rdiv = 1; ba.sld = cols / q.group; break;
  }
  // blocks of min(blocksize, 128) columns: for blocksize > 128 the lazy
  // updates are applied in more steps, which is the same arithmetic in
  // exact terms (GPTQ's result does not depend on the block size)
  const int64_t step = std::min<int64_t>(blocksize, QB);
  // outer blocks of QOB columns for 128-column blocks; other block sizes
  // update everything after each block, as the reference does
  const int64_t ostep = step == QB ? QOB : step;
  const unsigned nblk = (unsigned)((rows + ROWS - 1) / ROWS);
  ba.eld = QOB;
  // W[:, n0:n1] -= E[:, e0:e0+k] * Hinv[h0:h0+k, n0:n1].  With the transposed
  // factor the product is A * B^T on the tensor cores.  The identity fallback
  // has no off-diagonal Hinv (`status` makes the GEMM a no-op), so the
  // reference's update is a no-op there.
  auto update = [&](int64_t n0, int64_t n1, int64_t e0, int64_t h0, int k) -> bool {
    if (HinvT) {
      GemmArgs g = {(int)rows, (int)(n1 - n0), k, E + e0, QOB, HinvT + n0 * cols + h0, cols, W + n0, cols, 1, 0, 0,
                    status, 0, status};
      return launch_gemm(false, true, g, st) == LLMC_OK;
    }
    GemmArgs g = {(int)rows, (int)(n1 - n0), k, E + e0, QOB, Hinv + h0 * cols + n0, cols, W + n0, cols, 1, 0, 0,
                  status, 0, status};
    return launch_gemm(false, false, g, st) == LLMC_OK;
  };
  for (int64_t o1 = 0; o1 < cols; o1 += ostep) {
    const int64_t o2 = std::min<int64_t>(o1 + ostep, cols);
    for (int64_t i1 = o1; i1 < o2; i1 += step) {
      const int cnt = (int)std::min<int64_t>(step, o2 - i1);
      ba.i1 = (int)i1; ba.count = cnt; ba.ecol = i1 - o1;
      if (percol) k_gptq_block<true><<<nblk, ROWS, smem, st>>>(ba);
      else k_gptq_block<false><<<nblk, ROWS, smem, st>>>(ba);
      llmc::note_launch();
      const int64_t i2 = i1 + cnt;
      // the rest of this outer block, from this block's errors
      if (i2 < o2 && !update(i2, o2, i1 - o1, i1, cnt)) return LLMC_ECUDA;
    }
    // everything after the outer block, from all of its errors at once
    if (o2 < cols && !update(o2, cols, 0, o1, (int)(o2 - o1))) return LLMC_ECUDA;
  }
  if (x.perm) k_finish_perm<<<grid_for(rows * cols), 256, 0, st>>>(W, (uint16_t*)wq_bf16, rows, cols, x.perm);
  else k_finish<<<grid_for(rows * cols), 256, 0, st>>>(W, (uint16_t*)wq_bf16, rows * cols);
  llmc::note_launch();
  k_sum<<<1, 1024, 0, st>>>(L, rows, loss_out); llmc::note_launch();
  if (x.row_loss_out &&
      cudaMemcpyAsync(x.row_loss_out, L, sizeof(float) * rows, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return LLMC_ECUDA;
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_gptq_quantize(const void* w_bf16, int64_t rows, int64_t cols, const float* Hinv, const float* HinvT,
                       const uint8_t* dead, const LlmcQuantArgs* args, const void* scale_bf16, const int8_t* zp,
                       int64_t blocksize, void* wq_bf16, float* loss_out, void* workspace, int* status,
                       void* stream) {
  return llmc_gptq_quantize_ex(w_bf16, rows, cols, Hinv, HinvT, dead, args, scale_bf16, zp, nullptr, blocksize,
                               wq_bf16, loss_out, workspace, status, stream);
}

int llmc_gptq_actorder_perm(const float* H, int64_t d, int32_t* perm, void* stream) {
  if (!H || !perm || d <= 0) return LLMC_EINVAL_ARG;
  k_actorder_perm<<<(unsigned)((d + 255) / 256), 256, 0, (cudaStream_t)stream>>>(H, d, perm); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_gptq_permute_hessian(const float* H, int64_t d, const int32_t* perm, float* Hp, void* stream) {
  if (!H || !perm || !Hp || d <= 0 || d > 0x7FFFFFFF || H == Hp) return LLMC_EINVAL_ARG;
  dim3 g((unsigned)std::min<int64_t>((d + 255) / 256, 8), (unsigned)d);
  k_permute_sym<<<g, 256, 0, (cudaStream_t)stream>>>(H, d, perm, Hp); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_permute_columns_bf16(const void* src, int64_t rows, int64_t cols, const int32_t* perm, void* dst,
                              void* stream) {
  if (!perm || rows < 0 || cols <= 0 || ((!src || !dst) && rows > 0) || (src == dst && rows > 0))
    return LLMC_EINVAL_ARG;
  if (rows == 0) return LLMC_OK;
  k_permute_cols16<<<grid_for(rows * cols), 256, 0, (cudaStream_t)stream>>>((const uint16_t*)src, rows, cols, perm,
                                                                            (uint16_t*)dst);
  llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

// ---------------------------------------------------------------- batched solve
// Many Hessians of one size with one weight each (the down projections of an
// MoE layer's experts): every expert's prepare / factor / block loop is the
// single-Hessian sequence, issued from C across a pool of streams so that
// the small, latency-bound kernels of different experts overlap and the
// host pays one call instead of one per expert.

namespace {
constexpr int kBatchStreamsMax = 16;

int64_t align256(int64_t b) { return (b + 255) & ~(int64_t)255; }

// Streams of the current device for the batched solve, made once.
int batch_streams(cudaStream_t* out, int n) {
  static std::mutex mu;
  static cudaStream_t pool[64][kBatchStreamsMax] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LLMC_ECUDA;
  std::lock_guard<std::mutex> lock(mu);
  if (!pool[dev][0]) {
    for (int k = 0; k < kBatchStreamsMax; ++k)
      if (cudaStreamCreateWithFlags(&pool[dev][k], cudaStreamNonBlocking) != cudaSuccess) {
        for (int m = 0; m < k; ++m) cudaStreamDestroy(pool[dev][m]);
        for (int m = 0; m < kBatchStreamsMax; ++m) pool[dev][m] = nullptr;
        return LLMC_ECUDA;
      }
  }
  for (int k = 0; k < n; ++k) out[k] = pool[dev][k];
  return LLMC_OK;
}

struct BatchLayout {
  int64_t hinv_ws, hinv, quant_ws, slot, dead;
};

int batch_layout(int64_t E, int64_t rows, int64_t d, int nstreams, BatchLayout* L, int64_t* total) {
  int64_t hws = 0, qws = 0;
  if (llmc_gptq_hinv_workspace_size(d, &hws) || llmc_gptq_quantize_workspace_size(rows, d, &qws))
    return LLMC_EINVAL_ARG;
  L->hinv_ws = align256(hws);
  L->hinv = align256(d * d * (int64_t)sizeof(float));
  L->quant_ws = align256(qws);
  L->slot = L->hinv_ws + 2 * L->hinv + L->quant_ws;
  L->dead = align256(E * d);
  *total = L->dead + (int64_t)std::min<int64_t>(nstreams, E) * L->slot;
  return LLMC_OK;
}

int clamp_streams(int n) { return std::max(1, std::min(n, kBatchStreamsMax)); }
}  // namespace

int llmc_gptq_solve_batch_workspace_size(int64_t E, int64_t rows, int64_t d, int nstreams, int64_t* bytes) {
  if (!bytes || E <= 0 || rows < 0 || d <= 0) return LLMC_EINVAL_ARG;
  BatchLayout L;
  return batch_layout(E, rows, d, clamp_streams(nstreams), &L, bytes);
}

int llmc_gptq_solve_batch(float* H, int64_t E, int64_t d, float percdamp, const void* w_bf16, int64_t rows,
                          const LlmcQuantArgs* args, const void* scale_bf16, const int8_t* zp, int64_t blocksize,
                          void* wq_bf16, float* loss, int* status, void* workspace, int nstreams, void* stream) {
  if (!H || !args || !w_bf16 || !scale_bf16 || !wq_bf16 || !loss || !status || !workspace || E <= 0 || d <= 0 ||
      rows <= 0 || blocksize < 1)
    return LLMC_EINVAL_ARG;
  if ((uintptr_t)workspace % 256) return LLMC_EINVAL_ARG;
  const QArgs q = to_qargs(*args);
  int64_t per_scale = 0;  // scale (and zero-point) values of one expert
  switch (q.strategy) {
    case LLMC_STRAT_TENSOR: per_scale = 1; break;
    case LLMC_STRAT_CHANNEL: per_scale = rows; break;
    case LLMC_STRAT_GROUP:
      if (q.group <= 0 || d % q.group) return LLMC_EINVAL_SHAPE;
      per_scale = rows * (d / q.group);
      break;
    case LLMC_STRAT_BLOCK:
      if (q.bh <= 0 || q.bw <= 0) return LLMC_EINVAL_ARG;
      per_scale = ((rows + q.bh - 1) / q.bh) * ((d + q.bw - 1) / q.bw);
      break;
    default: return LLMC_ENOSUPPORT;  // TENSOR_GROUP needs a global scale per expert
  }
  const int ns = (int)std::min<int64_t>(clamp_streams(nstreams), E);
  BatchLayout L;
  int64_t total = 0;
  if (batch_layout(E, rows, d, ns, &L, &total)) return LLMC_EINVAL_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  cudaStream_t sts[kBatchStreamsMax];
  if (batch_streams(sts, ns)) return cuda_fail("gptq_solve_batch: streams", cudaErrorUnknown);
  if (cudaMemsetAsync(status, 0, sizeof(int) * E, st) != cudaSuccess) return LLMC_ECUDA;
  cudaEvent_t ev_start = nullptr, ev_done[kBatchStreamsMax] = {};
  auto cleanup = [&]() {
    if (ev_start) cudaEventDestroy(ev_start);
    for (int k = 0; k < ns; ++k)
      if (ev_done[k]) cudaEventDestroy(ev_done[k]);
  };
  if (cudaEventCreateWithFlags(&ev_start, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventRecord(ev_start, st) != cudaSuccess) {
    cleanup();
    return LLMC_ECUDA;
  }
  for (int k = 0; k < ns; ++k)
    if (cudaStreamWaitEvent(sts[k], ev_start, 0) != cudaSuccess) {
      cleanup();
      return LLMC_ECUDA;
    }
  char* ws = (char*)workspace;
  uint8_t* dead = (uint8_t*)ws;
  int rc = LLMC_OK;
  for (int64_t e = 0; e < E && rc == LLMC_OK; ++e) {
    const int k = (int)(e % ns);
    char* slot = ws + L.dead + (int64_t)k * L.slot;
    void* hws = slot;
    float* hinv = (float*)(slot + L.hinv_ws);
    float* hinv_t = (float*)(slot + L.hinv_ws + L.hinv);
    void* qws = slot + L.hinv_ws + 2 * L.hinv;
    float* He = H + e * d * d;
    uint8_t* de = dead + e * d;
    rc = llmc_gptq_prepare_hessian(He, d, percdamp, de, sts[k]);
    if (rc == LLMC_OK) rc = hinv_impl(He, d, hinv, hinv_t, hws, status + e, sts[k], false);
    if (rc == LLMC_OK)
      rc = llmc_gptq_quantize_ex((const uint16_t*)w_bf16 + e * rows * d, rows, d, hinv, hinv_t, de, args,
                                 (const uint16_t*)scale_bf16 + e * per_scale, zp ? zp + e * per_scale : nullptr,
                                 nullptr, blocksize, (uint16_t*)wq_bf16 + e * rows * d, loss + e, qws, status + e,
                                 sts[k]);
  }
  // join every stream back to the caller's, also after an error (what was
  // enqueued stays ordered before the caller's later work)
  for (int k = 0; k < ns; ++k) {
    if (cudaEventCreateWithFlags(&ev_done[k], cudaEventDisableTiming) != cudaSuccess ||
        cudaEventRecord(ev_done[k], sts[k]) != cudaSuccess || cudaStreamWaitEvent(st, ev_done[k], 0) != cudaSuccess)
      rc = rc == LLMC_OK ? LLMC_ECUDA : rc;
  }
  cleanup();
  return rc;
}

}  // extern "C"
