// GPTQ Hessian accumulation H += alpha * X^T X on sm_100a tensor cores.
//
// X: (n_tokens, d) bf16, row stride ld; H: (d, d) float32 row-major, kept
// fully symmetric.  Reference: accumulate_hessian / _hessian_update,
// S/modifiers/gptq/gptq_quantize.py:22-32,63-97 (alpha = 2 there: the input
// is scaled by sqrt(2) before the product; bf16*bf16 products are exact in
// float32, so scaling the float32 sum by 2 is the same arithmetic up to
// summation order).
//
// Design: persistent CTA pairs (clusters of two CTAs on two SMs), one
// 256 x 256 output tile per pair at a time, 320 threads per CTA:
//   warp 0      TMA producer (both CTAs): this CTA's 128 features of the A
//               panel and 128 features of the B panel (64 tokens x 64
//               features per box, 128B swizzle) into a ring of six 32 KB stages;
//               both CTAs' loads complete on the even CTA's barrier.
//   warp 1      TMEM (both CTAs: two 256-column accumulators, allocated for
//               the pair); in the even CTA one thread issues tcgen05.mma
//               (cta_group::2, M=256, N=256, K=16, bf16 -> f32), which reads
//               A and B from both CTAs' shared memory and leaves 128 rows of
//               the tile in each CTA's TMEM.
//   warps 2..9  epilogue: every `fold` K steps (64 tokens each) the MMAs
//               start a fresh accumulator in the other TMEM buffer; the
//               epilogue loads the finished partial (tcgen05.ld) and adds it
//               into float32 running sums held in registers (a warp owns 32
//               rows x 128 columns).  After the tile's last partial it scales
//               the sums by alpha and TMA reduce-adds them into H: the box
//               and, for boxes strictly below the diagonal, its transpose.
// Folding bounds the tokens one tensor-core accumulator absorbs: the
// accumulation inside tcgen05 loses a little precision on every step, with a
// bias that grows with the magnitude the accumulator has reached, so a
// 16384-token launch keeps the accuracy of a `fold`-token one.
//
// Work units: (group, tile, token split).  Groups give block-diagonal
// Hessians over consecutive column blocks of X (one Hessian per MoE expert
// from the experts' concatenated inputs); a token split lets small Hessians
// use every SM pair (each split reduce-adds its part into H).  Only tiles
// that touch the lower triangle are computed; boxes strictly above the
// diagonal are skipped (their values arrive as mirrors), so every element of
// H receives one reduce-add per unit.
#include "llmc_common.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

namespace llmc {
namespace hess {

using namespace sm100;

constexpr int BM = 256, BN = 256, BK = 64;    // pair tile; a CTA holds 128 rows of A and 128 columns of B
constexpr int STAGES = 6;
constexpr int CHUNK_BYTES = 64 * BK * 2;      // one TMA box: 64 features x 64 tokens, 8 KB
constexpr int A_BYTES = 2 * CHUNK_BYTES;      // 128 features
constexpr int B_BYTES = 2 * CHUNK_BYTES;      // 128 features
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 32 KB per CTA
constexpr int EPI_WARPS = 8;
constexpr int EPI_BOX_BYTES = 32 * 32 * 4;      // 4 KB fp32 32x32 box
constexpr int EPI_WARP_BYTES = EPI_BOX_BYTES;      // one staging box per warp (direct, then mirror)
constexpr int SMEM_STAGES = STAGES * STAGE_BYTES;
constexpr int SMEM_EPI = EPI_WARPS * EPI_WARP_BYTES;
constexpr int SMEM_BAR = 256;
constexpr int SMEM_TOTAL = SMEM_STAGES + SMEM_EPI + SMEM_BAR + 1024;  // + alignment slack
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t TMEM_COLS = 512;             // two 256-column accumulators
constexpr uint32_t IDESC = instr_desc(1, true, true, BM, BN);

struct Params {
  int64_t n_tokens;
  int dg;        // Hessian size (of each group)
  int ngroups;   // block-diagonal groups (1: one Hessian)
  int mb;        // 256-row tiles per group
  int tiles;     // lower-triangle tiles per group
  int kunit;     // K steps per token split
  int nk;        // K steps in total
  int fold;      // K steps per TMEM partial
  int units;     // ngroups * tiles * splits
  float alpha;
  int* status;
  float* num_samples;
  float num_add;
  unsigned long long wait_ns;
  int stall;     // test hook: the MMA issuer waits on a barrier nothing arrives on
};

// Tiles touching the lower triangle: row tile bi (256 rows) pairs with column
// tiles bj = 0 .. bi.  tiles_before(bi) = sum_{r<bi} (r + 1).
__device__ __forceinline__ int tiles_before(int bi) { return bi * (bi + 1) / 2; }
// Tile order.  The persistent pairs walk the tile list in waves of one tile
// per pair and move through the token dimension in step, so each wave reads
// every X column its tiles touch once from DRAM and serves the rest from L2.
// Enumerating the lower triangle row by row makes every wave touch nearly all
// column panels; here row tiles are grouped in bands of RB and, inside a
// band, column tiles in chunks of CB, so consecutive tiles form compact
// RB x CB blocks.  Every other wave walks its tokens backwards (part_begin),
// so it starts on the tokens the previous wave read last, still in L2 for
// the panels the two waves share.  RB = 12, CB = 4 measured best at
// d = 14336 (X re-reads down by a sixth against 16 x 8 in one direction).
constexpr int RB = 12, CB = 4;
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
  bi = mb - 1;  // not reached for t < tiles
  bj = 0;
}

struct Unit {
  int g, bi, bj, ks0, ks1;
};
// A unit's K steps go in partials of `fold` steps; the j-th partial walked is
// partial j, or partial np-1-j when the unit runs in reverse (odd waves).
__device__ __forceinline__ int part_begin(const Unit& w, int j, int np, bool rev, int fold) {
  return w.ks0 + (rev ? np - 1 - j : j) * fold;
}
__device__ __forceinline__ int part_end(const Unit& w, int j, int np, bool rev, int fold) {
  return min(w.ks1, part_begin(w, j, np, rev, fold) + fold);
}
// Unit u: split-major, so consecutive units share a token range and their
// X panels in L2.
__device__ __forceinline__ Unit unit_of(const Params& p, int u) {
  const int per_split = p.ngroups * p.tiles;
  const int s = u / per_split, r = u - s * per_split;
  Unit w;
  w.g = r / p.tiles;
  tile_coords(r - w.g * p.tiles, p.mb, w.bi, w.bj);
  w.ks0 = s * p.kunit;
  w.ks1 = min(p.nk, w.ks0 + p.kunit);
  return w;
}

__global__ void __launch_bounds__(THREADS, 1)
k_hessian_pair(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap hmap, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = smem;
  uint8_t* epi = smem + SMEM_STAGES;
  uint64_t* bars = (uint64_t*)(smem + SMEM_STAGES + SMEM_EPI);
  uint64_t* full = bars;                    // [STAGES] (the even CTA's are used)
  uint64_t* empty = bars + STAGES;          // [STAGES]
  uint64_t* tfull = bars + 2 * STAGES;      // [2] a partial is complete in TMEM buffer b
  uint64_t* tempty = bars + 2 * STAGES + 2; // [2] both CTAs' epilogues have read buffer b (even CTA's)
  uint64_t* drain = bars + 2 * STAGES + 4;  // MMA completion before TMEM is freed
  uint64_t* stallbar = bars + 2 * STAGES + 5;
  uint32_t* tmem_slot = (uint32_t*)(bars + 2 * STAGES + 6);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const uint64_t wait_ns = p.wait_ns;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(smem_u32(&full[s]), 1); mbar_init(smem_u32(&empty[s]), 1); }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), 2 * EPI_WARPS);  // every epilogue warp of both CTAs
    }
    mbar_init(smem_u32(drain), 1);
    mbar_init(smem_u32(stallbar), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&xmap);
    prefetch_tmap(&hmap);
    if (blockIdx.x == 0 && p.num_samples) *p.num_samples += p.num_add;
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // raise the abort flag in both CTAs of the pair
  auto abort_pair = [&]() {
    *abort_flag = 1;
    st_cluster_u32(mapa_shared(smem_u32((const void*)abort_flag), rank ^ 1u), 1u);
  };

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int u = pair; u < p.units && !*abort_flag; u += npairs) {
        const Unit w = unit_of(p, u);
        const int xa = w.g * p.dg + w.bi * BM + (int)rank * 128;
        const int xb = w.g * p.dg + w.bj * BN + (int)rank * 128;
        const int np = (w.ks1 - w.ks0 + p.fold - 1) / p.fold;
        const bool rev = ((u / npairs) & 1) != 0;
        bool ok = true;
        for (int j = 0; ok && j < np; ++j) {
          const int kb = part_begin(w, j, np, rev, p.fold), ke = part_end(w, j, np, rev, p.fold);
          for (int ks = kb; ks < ke; ++ks) {
            if (!mbar_wait_cluster(smem_u32(&empty[stage]), phase ^ 1, abort_flag, wait_ns)) { ok = false; break; }
            const uint32_t fb_local = smem_u32(&full[stage]);
            if (rank == 0) mbar_arrive_expect_tx(fb_local, 2 * STAGE_BYTES);
            const uint32_t fb = mapa_shared(fb_local, 0);
            const uint32_t sa = smem_u32(stages + stage * STAGE_BYTES);
            const uint32_t sb = sa + A_BYTES;
            const int k0 = ks * BK;
            tma_load_2d_pair(sa, &xmap, xa, k0, fb);
            tma_load_2d_pair(sa + CHUNK_BYTES, &xmap, xa + 64, k0, fb);
            tma_load_2d_pair(sb, &xmap, xb, k0, fb);
            tma_load_2d_pair(sb + CHUNK_BYTES, &xmap, xb + 64, k0, fb);
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
        }
        if (!ok) break;
      }
      if (*abort_flag) abort_pair();
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (even CTA)
    if (rank == 0 && lane == 0) {
      bool ok = true;
      if (p.stall) ok = mbar_wait(smem_u32(stallbar), 0, abort_flag, wait_ns);  // nothing arrives: times out
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ctr = 0;  // partials issued: buffer ctr & 1, use (ctr >> 1)
      for (int u = pair; ok && u < p.units && !*abort_flag; u += npairs) {
        const Unit w = unit_of(p, u);
        const int np = (w.ks1 - w.ks0 + p.fold - 1) / p.fold;
        const bool rev = ((u / npairs) & 1) != 0;
        for (int j = 0; ok && j < np; ++j, ++ctr) {
          const uint32_t buf = ctr & 1;
          if (!mbar_wait_cluster(smem_u32(&tempty[buf]), ((ctr >> 1) & 1) ^ 1, abort_flag, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dt = tmem_base + buf * 256;
          const int ks0 = part_begin(w, j, np, rev, p.fold);
          const int ks1 = part_end(w, j, np, rev, p.fold);
          for (int ks = ks0; ks < ks1; ++ks) {
            if (!mbar_wait_cluster(smem_u32(&full[stage]), phase, abort_flag, wait_ns)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = smem_u32(stages + stage * STAGE_BYTES);
            const uint32_t sb = sa + A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t ad = smem_desc(sa + kk * 2048, CHUNK_BYTES, 1024, SWZ_128B);
              const uint64_t bd = smem_desc(sb + kk * 2048, CHUNK_BYTES, 1024, SWZ_128B);
              mma_f16_ss_pair(dt, ad, bd, IDESC, (ks != ks0 || kk != 0) ? 1u : 0u);
            }
            const uint32_t eb = smem_u32(&empty[stage]);
            mma_commit_pair(mapa_shared(eb, 0));
            mma_commit_pair(mapa_shared(eb, 1));
            if (++stage == STAGES) { stage = 0; phase ^= 1; }
          }
          if (!ok) break;
          const uint32_t fb = smem_u32(&tfull[buf]);
          mma_commit_pair(mapa_shared(fb, 0));
          mma_commit_pair(mapa_shared(fb, 1));
        }
      }
      if (!ok || *abort_flag) abort_pair();
      // every MMA this thread issued has finished before TMEM can be freed
      mma_commit_pair(mapa_shared(smem_u32(drain), 0));
      volatile int dummy = 0;
      mbar_wait(smem_u32(drain), 0, &dummy, wait_ns);
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int hh = (warp - 2) >> 2;    // column half of the 256-column tile
    const uint32_t wbuf_s = smem_u32(epi + (warp - 2) * EPI_WARP_BYTES);
    uint32_t ctr = 0;
    float acc[128];
    bool ok = true;
    for (int u = pair; ok && u < p.units && !*abort_flag; u += npairs) {
      const Unit w = unit_of(p, u);
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      for (int ks0 = w.ks0; ks0 < w.ks1; ks0 += p.fold, ++ctr) {
        const uint32_t buf = ctr & 1;
        if (!mbar_wait_cluster(smem_u32(&tfull[buf]), (ctr >> 1) & 1, abort_flag, wait_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(32 * q) << 16) + buf * 256 + (uint32_t)(hh * 128);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(taddr + 16 * c, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) acc[16 * c + j] += __uint_as_float(r[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[buf]), 0));
      }
      if (!ok) break;
      // the tile's sums: reduce-add into H (the box and its mirror)
      const int grl = w.bi * BM + (int)rank * 128 + 32 * q;  // row of this warp's strip within the group
      const int hrow = w.g * p.dg;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int gcl = w.bj * BN + hh * 128 + 32 * c;
        if (grl >= p.dg || gcl >= p.dg || grl < gcl) continue;  // out of range, or strictly above the diagonal
        const uint32_t box = wbuf_s;
        if (lane == 0) bulk_wait_read<0>();  // the previous reduce has read the buffer
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          st_shared_v4(box + lane * 128 + ((j ^ (lane & 7)) << 4), acc[32 * c + 4 * j + 0] * p.alpha,
                       acc[32 * c + 4 * j + 1] * p.alpha, acc[32 * c + 4 * j + 2] * p.alpha,
                       acc[32 * c + 4 * j + 3] * p.alpha);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&hmap, box, gcl, hrow + grl);
          bulk_commit();
        }
        if (grl > gcl) {
          // the mirror: the transposed box (row jj, column lane) reduce-added at (grl, gcl)
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
          const uint32_t mb = box + (lane & 3) * 4;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            st_shared_f32(mb + jj * 128 + ((((uint32_t)lane >> 2) ^ (jj & 7)) << 4), acc[32 * c + jj] * p.alpha);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_reduce_add_2d(&hmap, box, grl, hrow + gcl);
            bulk_commit();
          }
        }
      }
    }
    if (!ok || *abort_flag) {
      if (lane == 0) abort_pair();
    }
    if (lane == 0) bulk_wait<0>();
  }

  if (*abort_flag) spin_ns(200000);  // let copies issued before the abort land (they take microseconds)
  tc_fence_before();
  cluster_sync();  // the pair's MMAs are done and no CTA touches the other's shared memory any more
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if (threadIdx.x == 0 && *abort_flag && p.status) atomicMax(p.status, (int)LLMC_ETIMEOUT);
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

// Concurrent CTA pairs on this device (clusters of two that fit at once with
// the kernel's shared memory); cached per device.
static int max_pairs(int dev) {
  static std::mutex mu;
  static int cached[64] = {};
  std::lock_guard<std::mutex> g(mu);
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  cudaError_t e = cudaFuncSetAttribute(k_hessian_pair, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_TOTAL);
  if (e != cudaSuccess) return -(int)e;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)(sms & ~1));
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_TOTAL;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, (const void*)k_hessian_pair, &cfg);
  if (e != cudaSuccess || n <= 0) {
    cudaGetLastError();
    return e != cudaSuccess ? -(int)e : -(int)cudaErrorUnknown;
  }
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

// Token splits for a launch: the count that minimises the estimated time
// (waves of units x partials per unit, plus one partial's worth per unit for
// its write-out), fewer splits on a tie.
static int choose_splits(int64_t units_per_split, int64_t partials, int pairs) {
  int best = 1;
  double best_cost = 1e300;
  for (int64_t s = 1; s <= partials && s <= 64; ++s) {
    const int64_t per = (partials + s - 1) / s;
    if ((s - 1) * per >= partials) continue;  // an empty split
    const int64_t waves = (units_per_split * s + pairs - 1) / pairs;
    const double cost = (double)waves * (double)(per + 1);
    if (cost < best_cost - 1e-9) { best_cost = cost; best = (int)s; }
  }
  return best;
}

// Launch over `ngroups` block-diagonal Hessians of size dg each: group g reads
// columns [g*dg, (g+1)*dg) of X and accumulates into rows [g*dg, (g+1)*dg) of
// H (ngroups*dg x dg).
static int launch_pair(const void* x, int64_t n_tokens, int64_t ngroups, int64_t dg, int64_t ld, float* H,
                       float alpha, float* num_samples, float num_add, int* status, int64_t fold_tokens,
                       uint64_t wait_ns, int stall, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
  const int pairs = max_pairs(dev);
  if (pairs <= 0) return cuda_fail("hessian: cluster occupancy", -pairs);
  CUtensorMap xmap, hmap;
  if (!make_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, (uint64_t)(ngroups * dg), (uint64_t)n_tokens,
                (uint64_t)ld * 2, 64, BK))
    return cuda_fail("hessian: cuTensorMapEncodeTiled (X)", cudaErrorInvalidValue);
  if (!make_map(&hmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, H, (uint64_t)dg, (uint64_t)(ngroups * dg),
                (uint64_t)dg * 4, 32, 32))
    return cuda_fail("hessian: cuTensorMapEncodeTiled (H)", cudaErrorInvalidValue);
  Params p;
  p.n_tokens = n_tokens;
  p.dg = (int)dg;
  p.ngroups = (int)ngroups;
  p.mb = (int)((dg + BM - 1) / BM);
  p.tiles = p.mb * (p.mb + 1) / 2;
  p.nk = (int)((n_tokens + BK - 1) / BK);
  p.fold = (int)std::max<int64_t>(1, fold_tokens / BK);
  const int64_t partials = (p.nk + p.fold - 1) / p.fold;
  const int64_t per_split = (int64_t)p.tiles * ngroups;
  const int splits = choose_splits(per_split, partials, pairs);
  p.kunit = (int)(((partials + splits - 1) / splits) * p.fold);
  const int64_t used_splits = (p.nk + p.kunit - 1) / p.kunit;
  const int64_t units = per_split * used_splits;
  if (units >= (1ll << 31)) return LLMC_EINVAL_SHAPE;
  p.units = (int)units;
  p.alpha = alpha;
  p.status = status;
  p.num_samples = num_samples;
  p.num_add = num_add;
  p.wait_ns = wait_ns;
  p.stall = stall;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(units, pairs)));
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = SMEM_TOTAL;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, k_hessian_pair, xmap, hmap, p);
  if (e != cudaSuccess) return cuda_fail("hessian: cudaLaunchKernelEx", e);
  llmc::note_launch();
  return LLMC_OK;
}

}  // namespace hess
}  // namespace llmc

using namespace llmc;
using namespace llmc::hess;

namespace {
int hessian_common(const void* x, int64_t n_tokens, int64_t ngroups, int64_t d, int64_t ld, float* H, float alpha,
                   float* num_samples, float num_add, int* status, const LlmcHessianOpts* opts, void* stream) {
  if ((!x && n_tokens > 0) || !H || d <= 0 || ngroups <= 0 || n_tokens < 0 || ld < ngroups * d)
    return LLMC_EINVAL_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (n_tokens == 0) {
    if (num_samples && num_add != 0.f) { k_add_scalar<<<1, 1, 0, st>>>(num_samples, num_add); llmc::note_launch(); }
    return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  int64_t fold = LLMC_HESSIAN_FOLD_TOKENS;
  uint64_t wait_ns = LLMC_WAIT_NS;
  int stall = 0;
  if (opts) {
    if (opts->fold_tokens < 0 || (opts->fold_tokens > 0 && opts->fold_tokens % BK != 0)) return LLMC_EINVAL_ARG;
    if (opts->fold_tokens > 0) fold = opts->fold_tokens;
    if (opts->wait_ns > 0) wait_ns = (uint64_t)opts->wait_ns;
    stall = opts->test_stall ? 1 : 0;
  }
  const bool tma_ok = (d % 8 == 0) && (ld % 8 == 0) && (ngroups == 1 || d % 32 == 0) &&
                      (((uintptr_t)x & 15) == 0) && (((uintptr_t)H & 15) == 0) && ngroups * d < (1 << 24) &&
                      n_tokens < (1ll << 31) && get_encode() != nullptr;
  if (!tma_ok) {
    if (stall) return LLMC_EINVAL_ARG;  // the test hook belongs to the tensor-core path
    const int64_t nt = (d + 63) / 64;
    for (int64_t g = 0; g < ngroups; ++g) {
      k_hessian_simt<<<dim3((unsigned)nt, (unsigned)nt), dim3(16, 16), 0, st>>>(
          (const uint16_t*)x + g * d, n_tokens, d, ld, H + g * d * d, alpha, g == 0 ? num_samples : nullptr,
          num_add);
      llmc::note_launch();
    }
    return cudaGetLastError() == cudaSuccess ? LLMC_OK : LLMC_ECUDA;
  }
  return launch_pair(x, n_tokens, ngroups, d, ld, H, alpha, num_samples, num_add, status, fold, wait_ns, stall, st);
}
}  // namespace

extern "C" {

int llmc_hessian_accumulate(const void* x, int64_t n_tokens, int64_t d, int64_t ld, float* H, float alpha,
                            float* num_samples, float num_add, int* status, void* stream) {
  return hessian_common(x, n_tokens, 1, d, ld, H, alpha, num_samples, num_add, status, nullptr, stream);
}

int llmc_hessian_accumulate_grouped(const void* x, int64_t n_tokens, int64_t ngroups, int64_t d, int64_t ld,
                                    float* H, float alpha, float* num_samples, float num_add, int* status,
                                    const LlmcHessianOpts* opts, void* stream) {
  return hessian_common(x, n_tokens, ngroups, d, ld, H, alpha, num_samples, num_add, status, opts, stream);
}

int llmc_hessian_tiles(int64_t d) {
  int64_t mb = (d + BM - 1) / BM;
  return (int)(mb * (mb + 1) / 2);
}

}  // extern "C"
