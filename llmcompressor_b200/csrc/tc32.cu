// Float32-accurate GEMM on tcgen05 tensor cores: 3xTF32.
//
//   C (m x n) {=, -=, = -} A (m x k) * B (k x n), float32 in and out.
//
// Each float32 operand is split into hi = a with its low 13 mantissa bits
// cleared (exactly a TF32 value) and lo = a - hi (exact in float32); the
// product is accumulated in TMEM as hi*hi + lo*hi + hi*lo (the lo*lo term,
// ~2^-22 relative, is dropped).  Because hi is written back as an exact TF32
// value, the result does not depend on whether the tensor core truncates or
// rounds its float32 inputs.
//
// Persistent kernel, one CTA per SM, 320 threads:
//   warp 0      TMA producer: A and B tiles (128 x 32 float32, 128B swizzle),
//               K-major or MN-major as the operands are stored, 3 stages
//   warp 1      TMEM owner and single-thread tcgen05.mma issuer (kind::tf32,
//               M=128 N=128 K=8), two 128-column accumulators
//   warps 2..5  epilogue: tcgen05.ld, then C read-modify-write in place
//   warps 6..9  split: hi/lo of each stage in shared memory
// Every wait is bounded (sm100.cuh); a timeout sets *status = LLMC_ETIMEOUT.
#include "llmc_common.cuh"
#include "sm100.cuh"
#include "tc32.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace llmc {
namespace tc32 {

using namespace sm100;

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int TILE_BYTES = 128 * BK * 4;          // 16 KB per operand tile
constexpr int BOX_MN_BYTES = 32 * BK * 4;         // 4 KB: one 32-element MN chunk x 32 K rows
constexpr int STAGE_BYTES = 4 * TILE_BYTES;       // A_hi, B_hi, A_lo, B_lo
constexpr int SMEM_STAGES = STAGES * STAGE_BYTES;  // 192 KB
constexpr int EPI_BOX_BYTES = 32 * 32 * 4;           // 4 KB float32 box
constexpr int EPI_WARP_BYTES = 2 * EPI_BOX_BYTES;     // double-buffered per epilogue warp
constexpr int SMEM_EPI = 4 * EPI_WARP_BYTES;          // 32 KB
constexpr int SMEM_TOTAL = SMEM_STAGES + SMEM_EPI + 256 + 1024;
constexpr int THREADS = 320;
constexpr int XF_WARP0 = 6, NXF = 4;  // split warps 6..9 (epilogue warps are 2..5)
constexpr uint32_t TMEM_COLS = 256;

struct Params {
  int m, n, k;
  int tiles_m, tiles_n, num_tiles;
  int mode, tri;
  bool a_mn, b_mn;
  float* C;
  int64_t ldc;
  int* status;
};

__device__ __forceinline__ void tile_of(const Params& p, int t, int& bm, int& bn) {
  if (p.tri) {  // lower-triangle tiles of a square tiling: t -> (bm, bn <= bm)
    int r = (int)((sqrtf(8.0f * (float)t + 1.0f) - 1.0f) * 0.5f);
    while ((r + 1) * (r + 2) / 2 <= t) ++r;
    while (r * (r + 1) / 2 > t) --r;
    bm = r;
    bn = t - r * (r + 1) / 2;
  } else {
    bm = t / p.tiles_n;
    bn = t % p.tiles_n;
  }
}

__global__ void __launch_bounds__(THREADS, 1)
k_gemm_tc32(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
            const __grid_constant__ CUtensorMap cmap, Params p, const int* skip) {
  if (skip && *skip) return;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = (uint64_t*)(smem + SMEM_STAGES + SMEM_EPI);
  uint64_t* full = bars;                // TMA landed            [STAGES]
  uint64_t* split = bars + STAGES;      // hi/lo written         [STAGES]
  uint64_t* empty = bars + 2 * STAGES;  // MMAs done reading     [STAGES]
  uint64_t* tfull = bars + 3 * STAGES;  // accumulator ready     [2]
  uint64_t* tempty = bars + 3 * STAGES + 2;  // accumulator drained [2]
  uint64_t* drain = bars + 3 * STAGES + 4;
  uint32_t* tmem_slot = (uint32_t*)(bars + 3 * STAGES + 5);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.k + BK - 1) / BK;
  constexpr uint32_t IDESC_KK = instr_desc(2, false, false, BM, BN);
  const uint32_t idesc = IDESC_KK | ((p.a_mn ? 1u : 0u) << 15) | ((p.b_mn ? 1u : 0u) << 16);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&split[s]), NXF);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) { mbar_init(smem_u32(&tfull[b]), 1); mbar_init(smem_u32(&tempty[b]), 4); }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&amap);
    prefetch_tmap(&bmap);
    prefetch_tmap(&cmap);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        int bm, bn;
        tile_of(p, t, bm, bn);
        const int m0 = bm * BM, n0 = bn * BN;
        for (int ks = 0; ks < nk; ++ks) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) break;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, 2 * TILE_BYTES);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + TILE_BYTES;
          const int k0 = ks * BK;
          if (p.a_mn) {
#pragma unroll
            for (int j = 0; j < 4; ++j) tma_load_2d(sa + j * BOX_MN_BYTES, &amap, m0 + 32 * j, k0, fb);
          } else {
            tma_load_2d(sa, &amap, k0, m0, fb);
          }
          if (p.b_mn) {
#pragma unroll
            for (int j = 0; j < 4; ++j) tma_load_2d(sb + j * BOX_MN_BYTES, &bmap, n0 + 32 * j, k0, fb);
          } else {
            tma_load_2d(sb, &bmap, k0, n0, fb);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag) {
        volatile int dummy = 0;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
          mbar_wait(smem_u32(&full[stage]), phase, &dummy);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      const uint32_t a_step = p.a_mn ? 1024u : 32u, b_step = p.b_mn ? 1024u : 32u;
      const uint32_t a_lbo = p.a_mn ? (uint32_t)BOX_MN_BYTES : 16u, b_lbo = p.b_mn ? (uint32_t)BOX_MN_BYTES : 16u;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t dt = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int ks = 0; ks < nk; ++ks) {
          if (!mbar_wait(smem_u32(&split[stage]), phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES), sb = sa + TILE_BYTES;
          const uint32_t sal = sa + 2 * TILE_BYTES, sbl = sa + 3 * TILE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint64_t ah = smem_desc(sa + kk * a_step, a_lbo, 1024, SWZ_128B);
            const uint64_t bh = smem_desc(sb + kk * b_step, b_lbo, 1024, SWZ_128B);
            const uint64_t al = smem_desc(sal + kk * a_step, a_lbo, 1024, SWZ_128B);
            const uint64_t bl = smem_desc(sbl + kk * b_step, b_lbo, 1024, SWZ_128B);
            mma_tf32_ss(dt, al, bh, idesc, (ks | kk) != 0);
            mma_tf32_ss(dt, ah, bl, idesc, 1);
            mma_tf32_ss(dt, ah, bh, idesc, 1);
          }
          mma_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(smem_u32(&tfull[acc]));
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      mma_commit(smem_u32(drain));
      volatile int dummy = 0;
      mbar_wait(smem_u32(drain), 0, &dummy);
    }
  } else if (warp >= XF_WARP0) {
    // ------------------------------------------------------------ hi / lo split
    const int xt = threadIdx.x - XF_WARP0 * 32;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    bool run = true;
    for (int t = blockIdx.x; t < p.num_tiles && run && !*abort_flag; t += gridDim.x) {
      for (int ks = 0; ks < nk; ++ks) {
        if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag)) { run = false; break; }
        uint8_t* base = smem + stage * STAGE_BYTES;
        // A and B hi tiles are the first 32 KB of the stage, their lo tiles the next 32 KB
#pragma unroll 4
        for (int i = xt; i < 2 * TILE_BYTES / 16; i += NXF * 32) {
          float4 v = ((float4*)base)[i];
          float4 h, l;
          h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u); l.x = v.x - h.x;
          h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u); l.y = v.y - h.y;
          h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u); l.z = v.z - h.z;
          h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u); l.w = v.w - h.w;
          ((float4*)base)[i] = h;
          ((float4*)(base + 2 * TILE_BYTES))[i] = l;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&split[stage]));
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    int acc = 0, ebuf = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
      int bm, bn;
      tile_of(p, t, bm, bn);
      const int m0 = bm * BM, n0 = bn * BN;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag)) break;
      tc_fence_after();
      // 32x32 boxes of the tile go through swizzled shared memory to a TMA
      // store (C = +-AB) or a TMA reduce-add of -AB (C -= AB, the read-modify-
      // write happens in L2).  Out-of-range rows/columns are clipped by TMA.
      const int gr = m0 + 32 * q;
      const float sgn = (p.mode == 0) ? 1.0f : -1.0f;
      uint8_t* wbuf = smem + SMEM_STAGES + (warp - 2) * EPI_WARP_BYTES;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * BN + 32 * c), r);
        tmem_ld_wait();
        const int gc = n0 + 32 * c;
        if (gr >= p.m || gc >= p.n) continue;
        uint8_t* box = wbuf + ebuf * EPI_BOX_BYTES;
        if (lane == 0) bulk_wait_read<1>();  // the copy that last read this buffer is done with it
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 v = make_float4(sgn * __uint_as_float(r[4 * j]), sgn * __uint_as_float(r[4 * j + 1]),
                                 sgn * __uint_as_float(r[4 * j + 2]), sgn * __uint_as_float(r[4 * j + 3]));
          *(float4*)(box + lane * 128 + ((j ^ (lane & 7)) << 4)) = v;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (p.mode == 1) tma_reduce_add_2d(&cmap, smem_u32(box), gc, gr);
          else tma_store_2d(&cmap, smem_u32(box), gc, gr);
          bulk_commit();
        }
        ebuf ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicMax(p.status, (int)LLMC_ETIMEOUT);
}

// ------------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

static bool map2d(CUtensorMap* m, const float* base, uint64_t inner, uint64_t outer, int64_t ld, uint32_t box_inner,
                  uint32_t box_outer) {
  auto enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int gemm(const Gemm& g, cudaStream_t st) {
  if (g.m <= 0 || g.n <= 0) return LLMC_OK;
  if (g.k <= 0) return LLMC_ENOSUPPORT;
  if (g.tri && g.m != g.n) return LLMC_ENOSUPPORT;
  // MN-major 32-bit operands need a different shared-memory swizzle; only the
  // K-major x K-major form (C = A * B^T with both stored row-major) is used.
  if (g.a_mn || g.b_mn) return LLMC_ENOSUPPORT;
  auto al = [](const void* p) { return (((uintptr_t)p) & 15) == 0; };
  if (!al(g.A) || !al(g.B) || (g.lda & 3) || (g.ldb & 3) || !encoder()) return LLMC_ENOSUPPORT;
  CUtensorMap am, bm;
  const bool ok_a = g.a_mn ? map2d(&am, g.A, (uint64_t)g.m, (uint64_t)g.k, g.lda, 32, 32)
                           : map2d(&am, g.A, (uint64_t)g.k, (uint64_t)g.m, g.lda, 32, 128);
  const bool ok_b = g.b_mn ? map2d(&bm, g.B, (uint64_t)g.n, (uint64_t)g.k, g.ldb, 32, 32)
                           : map2d(&bm, g.B, (uint64_t)g.k, (uint64_t)g.n, g.ldb, 32, 128);
  CUtensorMap cm;
  if ((((uintptr_t)g.C) & 15) || (g.ldc & 3)) return LLMC_ENOSUPPORT;
  const bool ok_c = map2d(&cm, g.C, (uint64_t)g.n, (uint64_t)g.m, g.ldc, 32, 32);
  if (!ok_a || !ok_b || !ok_c) return LLMC_ENOSUPPORT;
  Params p;
  p.m = g.m; p.n = g.n; p.k = g.k;
  p.tiles_m = (g.m + BM - 1) / BM;
  p.tiles_n = (g.n + BN - 1) / BN;
  p.num_tiles = g.tri ? p.tiles_m * (p.tiles_m + 1) / 2 : p.tiles_m * p.tiles_n;
  p.mode = g.mode; p.tri = g.tri; p.a_mn = g.a_mn; p.b_mn = g.b_mn;
  p.C = g.C; p.ldc = g.ldc; p.status = g.status;
  {
    static std::mutex mu;
    static uint64_t done = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 64 && !((done >> dev) & 1ull)) {
      if (cudaFuncSetAttribute(k_gemm_tc32, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL) != cudaSuccess)
        return LLMC_ECUDA;
      done |= 1ull << dev;
    }
  }
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  const int grid = std::min(p.num_tiles, g.max_ctas > 0 ? std::min(g.max_ctas, sms) : sms);
  k_gemm_tc32<<<grid, THREADS, SMEM_TOTAL, st>>>(am, bm, cm, p, g.skip); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

}  // namespace tc32
}  // namespace llmc

extern "C" int llmc_gemm_f32_nt(int64_t m, int64_t n, int64_t k, const float* A, int64_t lda, const float* B,
                                int64_t ldb, float* C, int64_t ldc, int mode, void* stream) {
  if (m < 0 || n < 0 || k < 0 || m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return LLMC_EINVAL_ARG;
  if (mode < 0 || mode > 2) return LLMC_EINVAL_ARG;
  if (m == 0 || n == 0) return LLMC_OK;
  if (!A || !B || !C) return LLMC_EINVAL_ARG;
  llmc::tc32::Gemm g = {};
  g.m = (int)m; g.n = (int)n; g.k = (int)k;
  g.A = A; g.lda = lda; g.a_mn = false;
  g.B = B; g.ldb = ldb; g.b_mn = false;
  g.C = C; g.ldc = ldc; g.mode = mode; g.tri = 0; g.skip = nullptr;
  return llmc::tc32::gemm(g, (cudaStream_t)stream);
}
