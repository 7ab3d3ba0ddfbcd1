// GPTQ Hessian accumulation H += alpha * X^T X on sm_100a tensor cores.
//
// X: (n_tokens, d) bf16, row stride ld; H: (d, d) float32 row-major, kept
// fully symmetric.  Reference: accumulate_hessian / _hessian_update,
// S/modifiers/gptq/gptq_quantize.py:22-32,63-97 (alpha = 2 there: the input
// is scaled by sqrt(2) before the product; bf16*bf16 products are exact in
// float32, so scaling the float32 sum by 2 is the same arithmetic up to
// summation order).
//
// Design (one persistent CTA per SM, 192 threads, warp-specialised), output
// tiles of 256 x 256:
//   warp 0      TMA producer: X tiles (64 tokens x 64 features, 128B swizzle)
//               into a 3-stage ring of 64 KB (A: 256 features, B: 256
//               features); both operands are MN-major views of X.
//   warp 1      allocates all 512 TMEM columns and issues tcgen05.mma
//               (M=128, N=256, K=16, bf16 -> f32): two MMAs per K step, the
//               two 128-row halves of A against the same B, into two 256-column
//               accumulators.  A 256 x 256 tile per SM reads a third fewer
//               operand bytes per flop than 128 x 256 tiles, which outweighs
//               the accumulators no longer being double-buffered (the MMAs of
//               the next tile wait for this tile's epilogue).
//   warps 2..5  epilogue: tcgen05.ld 32x32 boxes, x alpha, stage in swizzled
//               smem (one buffer per warp), TMA reduce-add into H -- the box
//               itself and, for boxes strictly below the diagonal, its
//               transpose (the mirror).
// Only tiles that touch the lower triangle are computed; boxes entirely
// above the diagonal inside those tiles are skipped (their values arrive as
// mirrors), so every element of H receives exactly one reduce-add per call.
#include "llmc_common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace llmc {
namespace hess {

using namespace sm100;

constexpr int BM = 256, BN = 256, BK = 64, STAGES = 3;
constexpr int A_BYTES = BM * BK * 2;   // 32 KB: four 64-feature chunks
constexpr int B_BYTES = BN * BK * 2;   // 32 KB: four 64-feature chunks
constexpr int CHUNK_BYTES = 64 * BK * 2;  // 8 KB: one TMA box (64 features x 64 tokens)
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int EPI_WARPS = 4;
constexpr int EPI_BOX_BYTES = 32 * 32 * 4;                 // 4 KB fp32 32x32 box
constexpr int EPI_WARP_BYTES = 2 * EPI_BOX_BYTES;          // one buffer: direct + mirror box
constexpr int SMEM_STAGES = STAGES * STAGE_BYTES;          // 192 KB (3 x 64 KB)
constexpr int SMEM_EPI = EPI_WARPS * EPI_WARP_BYTES;       // 32 KB
constexpr int SMEM_BAR = 256;
constexpr int SMEM_TOTAL = SMEM_STAGES + SMEM_EPI + SMEM_BAR + 1024;  // + alignment slack
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t IDESC = instr_desc(1, true, true, 128, BN);  // two M=128 MMAs per K step

struct Params {
  int64_t d, n_tokens;
  int num_tiles;
  int mb;  // row tiles
  float alpha;
  int* status;
  float* num_samples;
  float num_add;
};

// Tiles touching the lower triangle: row tile bi (256 rows) pairs with column
// tiles bj = 0 .. bi.  tiles_before(bi) = sum_{r<bi} (r + 1).
__device__ __forceinline__ int tiles_before(int bi) { return bi * (bi + 1) / 2; }
// Tile order.  The persistent CTAs walk the tile list in waves of one tile
// per CTA and move through the token dimension in step, so each wave reads
// every X column its tiles touch once from DRAM and serves the rest from L2.
// Enumerating the lower triangle row by row makes every wave touch nearly all
// column panels; here row tiles are grouped in bands of RB and, inside a
// band, column tiles in chunks of CB, so consecutive tiles form compact
// RB x CB blocks (d = 14336: X read ~6 times per launch instead of ~11).
constexpr int RB = 16, CB = 8;
__device__ __forceinline__ int chunk_tiles(int r0, int r1, int c) {
  int n = 0;
  for (int bi = r0; bi < r1; ++bi) n += max(0, min(CB, bi + 1 - c * CB));
  return n;
}
__device__ __forceinline__ void tile_coords(int t, int mb, int& bi, int& bj) {
  int lo = 0, hi = (mb + RB - 1) / RB - 1;
  while (lo < hi) {  // last band whose first tile is <= t
    const int mid = (lo + hi + 1) >> 1;
    if (tiles_before(mid * RB) <= t) lo = mid; else hi = mid - 1;
  }
  const int r0 = lo * RB, r1 = min(mb, r0 + RB);
  int u = t - tiles_before(r0);
  int c = 0;
  const int cmax = (mb + CB) / CB;  // chunks of the widest row: the walk ends by then
  for (int cnt = chunk_tiles(r0, r1, c); u >= cnt && c < cmax; cnt = chunk_tiles(r0, r1, ++c)) u -= cnt;
  for (bi = r0; bi < r1; ++bi) {
    const int k = max(0, min(CB, bi + 1 - c * CB));
    if (u < k) { bj = c * CB + u; return; }
    u -= k;
  }
  bi = mb - 1;  // not reached for t < num_tiles
  bj = 0;
}

__global__ void __launch_bounds__(THREADS, 1)
k_hessian_tc(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap hmap, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = smem;
  uint8_t* epi = smem + SMEM_STAGES;
  uint64_t* bars = (uint64_t*)(smem + SMEM_STAGES + SMEM_EPI);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;   // [1] (slot 2 unused)
  uint64_t* tempty = bars + 2 * STAGES + 2;  // [1] (slot 2 unused)
  uint64_t* drain = bars + 2 * STAGES + 4;  // MMA completion before TMEM is freed
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * STAGES + 5);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (int)((p.n_tokens + BK - 1) / BK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(smem_u32(&full[s]), 1); mbar_init(smem_u32(&empty[s]), 1); }
    mbar_init(smem_u32(&tfull[0]), 1);           // the tile's MMAs are done
    mbar_init(smem_u32(&tempty[0]), EPI_WARPS);  // the epilogue has read the accumulators
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&xmap);
    prefetch_tmap(&hmap);
    if (blockIdx.x == 0 && p.num_samples) *p.num_samples += p.num_add;
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
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        int bi, bj;
        tile_coords(t, p.mb, bi, bj);
        const int row0 = bi * BM, col0 = bj * BN;
        for (int ks = 0; ks < nk; ++ks) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag)) break;
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          const uint32_t sa = smem_u32(stages + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          const int k0 = ks * BK;
#pragma unroll
          for (int m = 0; m < BM / 64; ++m) tma_load_2d(sa + m * CHUNK_BYTES, &xmap, row0 + 64 * m, k0, fb);
#pragma unroll
          for (int n = 0; n < BN / 64; ++n) tma_load_2d(sb + n * CHUNK_BYTES, &xmap, col0 + 64 * n, k0, fb);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (*abort_flag) {
        // let the loads already in flight land before the CTA's smem goes away
        volatile int dummy = 0;
        for (int i = 0; i < STAGES && i < issued; ++i) {
          if (--stage < 0) { stage = STAGES - 1; phase ^= 1; }
          mbar_wait(smem_u32(&full[stage]), phase, &dummy);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
        if (!mbar_wait(smem_u32(&tempty[0]), acc_phase ^ 1, abort_flag)) break;
        tc_fence_after();
        const uint32_t dt = tmem_base;
        bool ok = true;
        for (int ks = 0; ks < nk; ++ks) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(stages + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t bd = smem_desc(sb + kk * 2048, CHUNK_BYTES, 1024, SWZ_128B);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint64_t ad = smem_desc(sa + h * 2 * CHUNK_BYTES + kk * 2048, CHUNK_BYTES, 1024, SWZ_128B);
              mma_f16_ss(dt + (uint32_t)(h * BN), ad, bd, IDESC, (ks | kk) != 0);
            }
          }
          mma_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(smem_u32(&tfull[0]));
        acc_phase ^= 1;
      }
      // every MMA this thread issued has finished before TMEM can be freed
      mma_commit(smem_u32(drain));
      volatile int dummy = 0;
      mbar_wait(smem_u32(drain), 0, &dummy);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t* wbuf = epi + (warp - 2) * EPI_WARP_BYTES;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.num_tiles && !*abort_flag; t += gridDim.x) {
      int bi, bj;
      tile_coords(t, p.mb, bi, bj);
      const int row0 = bi * BM, col0 = bj * BN;
      if (!mbar_wait(smem_u32(&tfull[0]), acc_phase, abort_flag)) break;
      tc_fence_after();
      for (int hc = 0; hc < 2 * (BN / 32); ++hc) {
        const int h = hc / (BN / 32), c = hc % (BN / 32);
        const int gr = row0 + 128 * h + 32 * q;
        const int gc = col0 + 32 * c;
        if (gr >= p.d || gc >= p.d || gr < gc) continue;  // out of range, or strictly above the diagonal
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(32 * q) << 16) + (uint32_t)(h * BN + 32 * c), r);
        tmem_ld_wait();
        uint8_t* dbox = wbuf;
        uint8_t* mbox = dbox + EPI_BOX_BYTES;
        if (lane == 0) bulk_wait_read<0>();  // the previous box's reduce has read the buffer
        __syncwarp();
        // direct box: row `lane`, 32 columns, 128B-swizzled rows
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 v;
          v.x = __uint_as_float(r[4 * j + 0]) * p.alpha;
          v.y = __uint_as_float(r[4 * j + 1]) * p.alpha;
          v.z = __uint_as_float(r[4 * j + 2]) * p.alpha;
          v.w = __uint_as_float(r[4 * j + 3]) * p.alpha;
          *(float4*)(dbox + lane * 128 + ((j ^ (lane & 7)) << 4)) = v;
        }
        const bool mirror = gr > gc;
        if (mirror) {
          // transposed box: row = column index jj, column = lane
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            *(float*)(mbox + jj * 128 + ((((lane >> 2) ^ (jj & 7))) << 4) + (lane & 3) * 4) =
                __uint_as_float(r[jj]) * p.alpha;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&hmap, smem_u32(dbox), gc, gr);
          if (mirror) tma_reduce_add_2d(&hmap, smem_u32(mbox), gr, gc);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[0]));
      acc_phase ^= 1;
    }
    if (lane == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicExch(p.status, LLMC_ETIMEOUT);
}

// ---------------------------------------------------------------------------
// CUDA-core fallback for shapes TMA cannot describe (d % 8 != 0, unaligned
// rows): 64x64 output tiles of the lower triangle, mirrored on write.
// ---------------------------------------------------------------------------
__global__ void k_hessian_simt(const uint16_t* __restrict__ x, int64_t n, int64_t d, int64_t ld, float* H,
                               float alpha, float* num_samples, float num_add) {
  const int bi = blockIdx.y, bj = blockIdx.x;
  if (bj > bi) return;
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0 && threadIdx.y == 0 && num_samples)
    *num_samples += num_add;
  __shared__ float sa[16][65], sb[16][65];
  const int tx = threadIdx.x, ty = threadIdx.y;  // 16 x 16, each computes 4x4
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < n; k0 += 16) {
    for (int i = ty * 16 + tx; i < 16 * 64; i += 256) {
      int kk = i / 64, cc = i % 64;
      int64_t k = k0 + kk;
      int64_t ra = (int64_t)bi * 64 + cc, rb = (int64_t)bj * 64 + cc;
      sa[kk][cc] = (k < n && ra < d) ? bf16_to_f(x[k * ld + ra]) : 0.f;
      sb[kk][cc] = (k < n && rb < d) ? bf16_to_f(x[k * ld + rb]) : 0.f;
    }
    __syncthreads();
    for (int kk = 0; kk < 16; ++kk)
      for (int a = 0; a < 4; ++a)
        for (int b = 0; b < 4; ++b) acc[a][b] = fmaf(sa[kk][ty * 4 + a], sb[kk][tx * 4 + b], acc[a][b]);
    __syncthreads();
  }
  for (int a = 0; a < 4; ++a)
    for (int b = 0; b < 4; ++b) {
      int64_t i = (int64_t)bi * 64 + ty * 4 + a, j = (int64_t)bj * 64 + tx * 4 + b;
      if (i >= d || j >= d || j > i) continue;
      float v = acc[a][b] * alpha;
      H[i * d + j] += v;
      if (i != j) H[j * d + i] += v;
    }
}

__global__ void k_add_scalar(float* p, float v) { *p += v; }

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                     uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  (void)esize;
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

}  // namespace hess
}  // namespace llmc

using namespace llmc;
using namespace llmc::hess;

extern "C" {

int llmc_hessian_accumulate(const void* x, int64_t n_tokens, int64_t d, int64_t ld, float* H, float alpha,
                            float* num_samples, float num_add, int* status, void* stream) {
  if ((!x && n_tokens > 0) || !H || d <= 0 || n_tokens < 0 || ld < d) return LLMC_EINVAL_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (n_tokens == 0) {
    if (num_samples && num_add != 0.f) { k_add_scalar<<<1, 1, 0, st>>>(num_samples, num_add); llmc::note_launch(); }
    return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  const bool tma_ok = (d % 8 == 0) && (ld % 8 == 0) && (((uintptr_t)x & 15) == 0) && (((uintptr_t)H & 15) == 0) &&
                      d < (1 << 24) && n_tokens < (1ll << 31) && get_encode() != nullptr;
  if (!tma_ok) {
    int64_t nt = (d + 63) / 64;
    k_hessian_simt<<<dim3((unsigned)nt, (unsigned)nt), dim3(16, 16), 0, st>>>((const uint16_t*)x, n_tokens, d, ld, H,
                                                                             alpha, num_samples, num_add); llmc::note_launch();
    return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  CUtensorMap xmap, hmap;
  if (!make_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)d, (uint64_t)n_tokens, (uint64_t)ld * 2, 64,
                BK))
    return LLMC_ECUDA;
  if (!make_map(&hmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, H, (uint64_t)d, (uint64_t)d, (uint64_t)d * 4, 32, 32))
    return LLMC_ECUDA;
  Params p;
  p.d = d;
  p.n_tokens = n_tokens;
  p.mb = (int)((d + BM - 1) / BM);
  p.num_tiles = p.mb * (p.mb + 1) / 2;
  p.alpha = alpha;
  p.status = status;
  p.num_samples = num_samples;
  p.num_add = num_add;
  {
    static std::mutex mu;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (dev < 64 && !attr_set[dev]) {
      if (cudaFuncSetAttribute(k_hessian_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL) != cudaSuccess)
        return LLMC_ECUDA;
      attr_set[dev] = true;
    }
  }
  int grid = std::min(p.num_tiles, num_sms());
  k_hessian_tc<<<grid, THREADS, SMEM_TOTAL, st>>>(xmap, hmap, p); llmc::note_launch();
  return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
}

int llmc_hessian_tiles(int64_t d) {
  int64_t mb = (d + BM - 1) / BM;
  return (int)(mb * (mb + 1) / 2);
}

}  // extern "C"
