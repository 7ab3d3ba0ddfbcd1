// Float32-accurate GEMM on the tcgen05 tensor cores (3xTF32 split), used by
// the GPTQ solve for its wide rank-K updates:  C (m x n) {=, -=, = -} A * B.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace llmc {
namespace tc32 {

struct Gemm {
  int m, n, k;
  const float* A;
  int64_t lda;
  bool a_mn;  // A stored k-major, A[m][k] at A[k*lda + m] (MN-major operand); else row-major m x k
  const float* B;
  int64_t ldb;
  bool b_mn;  // B stored row-major k x n, B[k][n] at B[k*ldb + n] (MN-major operand); else stored n x k
  float* C;
  int64_t ldc;
  int mode;  // 0: C = AB, 1: C = C - AB, 2: C = -AB
  int tri;   // only output tiles touching the lower triangle (row >= col)
  const int* skip;  // optional device flag: do nothing when set
  int max_ctas;     // > 0: at most this many CTAs (leaves SMs to concurrent work); else one per SM
  int* status;      // optional device word: raised to LLMC_ETIMEOUT if a bounded wait runs out
};

// Launches the tensor-core GEMM; returns LLMC_ENOSUPPORT (launching nothing)
// when the operands do not meet the TMA constraints, so the caller can use
// the CUDA-core GEMM instead.
int gemm(const Gemm& g, cudaStream_t st);

}  // namespace tc32
}  // namespace llmc
