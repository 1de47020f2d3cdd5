// FP16 / BF16 GEMM with f32 accumulation on tcgen05 tensor cores.
//
// Replaces the reference's tensor-core lowering (ptx_tensor.py:160-473): per
// warp a 128x32 C tile of m16n8k16 mma.sync fragments fed by per-element
// global loads or ldmatrix, stored per element with a fused scalar epilogue.
//
// Here a persistent, warp-specialised kernel per SM:
//   warp 0      one thread issues TMA loads (128-byte swizzle, no multicast)
//               of A[128 x 64] and B[64 x 256] per k-block into a 4-stage
//               shared-memory ring guarded by full/empty mbarriers;
//   warp 1      allocates 512 TMEM columns (two 128 x 256 f32 accumulators)
//               and one thread issues tcgen05.mma (M=128, N=256, K=16, four
//               per k-block), committing each stage back to the producer and
//               each finished tile to the epilogue;
//   warps 2-5   epilogue: tcgen05.ld the accumulator (each warp its 32-lane
//               quarter), apply the fused erf/tanh GELU, convert to the output
//               type and store, then release the accumulator buffer so the
//               MMA of the next tile overlaps this tile's epilogue.
// Tiles are visited in groups of 8 M-blocks so concurrently running CTAs
// share A and B k-slices in L2.  The 2-SM kernel loads A with an evict-last
// L2 policy and, for plain 16-bit products, walks K backwards on every other
// tile of a CTA, so a wave of tiles starts on the A slices the previous wave
// (same A rows) left in L2 (DRAM reads at 8192^3: 1.12 -> 0.91 GB).  The f32
// split keeps the forward order: its K order is its rounding order.  Every mbarrier wait is bounded (1 s); a wait
// that gives up writes the device error word, stops the other roles and lets
// in-flight copies land before the CTA frees TMEM.
//
// A is [M, K] row-major (K-major operand).  B is [K, N] row-major ("kn",
// an MN-major operand, descriptor bit 16) or [N, K] row-major ("nk", K-major).
// Shapes TMA cannot describe (K or N not a multiple of 8, unaligned bases)
// and tiny problems take a SIMT kernel with the same arithmetic contract.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "epilogue.cuh"
#include "sm100.cuh"

namespace lc {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BK * BN * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 512;
constexpr int GROUP_M = 8;  // M-blocks per raster group

struct GemmParams {
  int m, n, k;
  void *c;
  const float *bias;  // f32 [N] added before the activation, or null
  int64_t ldc;
  int tiles_m, tiles_n;
  int vec_store;
  int serpentine;     // the 2-SM kernel may walk K backwards on every other tile
  int c_vec8;        // f32 C rows may be stored as 32-byte vectors (32-byte aligned)
  int *err;
};

__device__ __forceinline__ void tile_coords(int tile, const GemmParams &p, int &tm, int &tn) {
  const int group_size = GROUP_M * p.tiles_n;
  const int group = tile / group_size;
  const int first_m = group * GROUP_M;
  const int rem = p.tiles_m - first_m;
  const int gm = rem < GROUP_M ? rem : GROUP_M;
  const int in_group = tile - group * group_size;
  tm = first_m + in_group % gm;
  tn = in_group / gm;
}

__device__ __forceinline__ void raise_error(const GemmParams &p, volatile int *abort, int code) {
  *abort = 1;
  atomicCAS(p.err, 0, code);
}

// One 32-byte store of eight f32 values (the address is 32-byte aligned).
__device__ __forceinline__ void st_global_v8(float *dst, const float *v) {
  asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "f"(v[0]), "f"(v[1]),
               "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

template <int OUT, int EPI>
__device__ __forceinline__ void store_chunk(const GemmParams &p, int gm, int gn0,
                                            const uint32_t (&r)[32]) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (gn0 + j < p.n) v[j] = __fadd_rn(v[j], p.bias[gn0 + j]);
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = apply_epilogue<EPI>(v[j]);
  if (gm >= p.m) return;
  const bool full = p.vec_store && gn0 + 32 <= p.n;
  if constexpr (OUT == LC_F32) {
    float *row = static_cast<float *>(p.c) + (int64_t)gm * p.ldc + gn0;
    if (full && p.c_vec8) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) st_global_v8(row + j, v + j);
    } else if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4 *>(row + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gn0 + j < p.n) row[j] = v[j];
    }
  } else {
    using T = typename OutType<OUT>::type;
    T *row = static_cast<T *>(p.c) + (int64_t)gm * p.ldc + gn0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 pack;
        T *e = reinterpret_cast<T *>(&pack);
#pragma unroll
        for (int i = 0; i < 8; ++i) e[i] = to_out<T>(v[j + i]);
        *reinterpret_cast<uint4 *>(row + j) = pack;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gn0 + j < p.n) row[j] = to_out<T>(v[j]);
    }
  }
}

// The 32 f32 results of one accumulator chunk with bias and activation applied
// (the arithmetic of store_chunk, without the store).
template <int EPI>
__device__ __forceinline__ void chunk_values(const GemmParams &p, int gn0, const uint32_t (&r)[32],
                                             float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (p.bias) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (gn0 + j < p.n) v[j] = __fadd_rn(v[j], p.bias[gn0 + j]);
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = apply_epilogue<EPI>(v[j]);
}

template <bool BF16, bool B_MN, int OUT, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_b, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int *abort = &abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int num_kb = (p.k + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, p, tm, tn);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort)) {
            raise_error(p, abort, kErrTimeoutProducer);
            ok = false;
            break;
          }
          uint8_t *a_s = smem + stage * STAGE_BYTES;
          uint8_t *b_s = a_s + A_BYTES;
          mbar_expect_tx(&full_bar[stage], STAGE_BYTES);
          tma_load_2d(a_s, &tma_a, &full_bar[stage], kb * BK, tm * BM);
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(b_s + c * (BK * 128), &tma_b, &full_bar[stage], tn * BN + c * 64, kb * BK);
          } else {
            tma_load_2d(b_s, &tma_b, &full_bar[stage], kb * BK, tn * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BF16, false, B_MN, BM, BN);
      const uint64_t a_desc0 = smem_desc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = B_MN ? smem_desc_sw128(smem_u32(smem) + A_BYTES, BK * 128, 1024)
                                    : smem_desc_sw128(smem_u32(smem) + A_BYTES, 16, 1024);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort)) {
          raise_error(p, abort, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort)) {
            raise_error(p, abort, kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors of stage 0 plus the stage's offset / 16 (start-address field)
          const uint64_t ad = a_desc0 + (uint64_t)(stage * (STAGE_BYTES / 16));
          const uint64_t bd = b_desc0 + (uint64_t)(stage * (STAGE_BYTES / 16));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16(d_tmem, ad + (uint64_t)(k * 2), bd + (uint64_t)(B_MN ? k * 128 : k * 2), idesc,
                    (kb | k) != 0);
          mma_commit(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (ok) mma_commit(&tfull_bar[acc]);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int ok = 0;
      if (lane == 0) {
        ok = mbar_wait(&tfull_bar[acc], acc_phase, abort);
        if (!ok) raise_error(p, abort, kErrTimeoutEpilogue);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(tile, p, tm, tn);
      const int gm = tm * BM + row;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + acc * BN + c * 32, r);
        tmem_wait_ld();
        store_chunk<OUT, EPI>(p, gm, tn * BN + c * 32, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }

  __syncthreads();
  if (abort_flag) drain_delay();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- 2-SM path
//
// A cluster of two CTAs (one per SM of a pair) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M=256, N=256, K=16): each CTA stages its 128 rows
// of A and its 128 columns of B per k-block (32 KB per stage, 6 stages), so
// each SM's shared memory carries half the B traffic of the 1-SM kernel.
// The even CTA issues the MMAs; both CTAs' TMA loads complete on the even
// CTA's `full` barrier; the MMA commits arrive on the `empty` and
// `tmem_full` barriers of both CTAs (the commit's CTA-mask form), and the odd
// CTA's epilogue arrives remotely on the even CTA's `tmem_empty`.  No TMA
// load multicasts.
constexpr int PBM = 128;   // rows of A per CTA (256 per pair)
constexpr int PBN = 128;   // columns of B per CTA (256 per pair, all 256 accumulated per CTA)
constexpr int PSTAGES = 6;
constexpr int PA_BYTES = PBM * BK * 2;
constexpr int PB_BYTES = BK * PBN * 2;
constexpr int PSTAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr int PSMEM_BYTES = PSTAGES * PSTAGE_BYTES + 1024;
constexpr int PTILE = 256;

template <bool BF16, bool B_MN, int OUT, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tma_a,
                    const __grid_constant__ CUtensorMap tma_b, GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ __align__(8) uint64_t full_bar[PSTAGES];
  __shared__ __align__(8) uint64_t empty_bar[PSTAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int *abort = &abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 8);  // 4 epilogue warps in each CTA of the pair
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  cluster_sync();  // every barrier of the pair is initialised before any remote use
  if (warp == 1) {
    tmem_alloc_pair(&tmem_base, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int tiles_m = (p.m + PTILE - 1) / PTILE;
  const int tiles_n = (p.n + PTILE - 1) / PTILE;
  const int num_tiles = tiles_m * tiles_n;
  const int num_kb = (p.k + BK - 1) / BK;
  const int cluster = blockIdx.x >> 1;
  const int clusters = gridDim.x >> 1;
  GemmParams tp = p;
  tp.tiles_m = tiles_m;
  tp.tiles_n = tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // A's rows are shared by the consecutive tiles of a raster group, B's
      // columns are not: A's lines are kept in L2 ahead of B's.
      const uint64_t pol_a = l2_policy_evict_last(), pol_b = l2_policy_evict_normal();
      int it = 0;
      bool ok = true;
      int local = 0;
      for (int tile = cluster; ok && tile < num_tiles; tile += clusters, ++local) {
        int tm, tn;
        tile_coords(tile, tp, tm, tn);
        // every other tile of a CTA walks K backwards, starting on the k-slices
        // that the previous wave of tiles (same A rows) left in L2
        const bool back = p.serpentine && (local & 1);
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int kk = back ? num_kb - 1 - kb : kb;
          const int stage = it % PSTAGES;
          const uint32_t phase = (it / PSTAGES) & 1;
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort)) {
            raise_error(p, abort, kErrTimeoutProducer);
            ok = false;
            break;
          }
          uint8_t *a_s = smem + stage * PSTAGE_BYTES;
          uint8_t *b_s = a_s + PA_BYTES;
          const uint32_t full = mapa(smem_u32(&full_bar[stage]), 0);
          if (leader) mbar_expect_tx(&full_bar[stage], 2 * PSTAGE_BYTES);
          tma_load_2d_pair_hint(a_s, &tma_a, full, kk * BK, tm * PTILE + rank * PBM, pol_a);
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < PBN / 64; ++c)
              tma_load_2d_pair_hint(b_s + c * (BK * 128), &tma_b, full, tn * PTILE + rank * PBN + c * 64,
                                    kk * BK, pol_b);
          } else {
            tma_load_2d_pair_hint(b_s, &tma_b, full, kk * BK, tn * PTILE + rank * PBN, pol_b);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BF16, false, B_MN, 2 * PBM, PTILE);
      const uint64_t a_desc0 = smem_desc_sw128(smem_u32(smem), 16, 1024);
      const uint64_t b_desc0 = B_MN ? smem_desc_sw128(smem_u32(smem) + PA_BYTES, BK * 128, 1024)
                                    : smem_desc_sw128(smem_u32(smem) + PA_BYTES, 16, 1024);
      int it = 0;
      int local = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < num_tiles; tile += clusters, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, abort)) {
          raise_error(p, abort, kErrTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * PTILE;
        for (int kb = 0; kb < num_kb; ++kb, ++it) {
          const int stage = it % PSTAGES;
          const uint32_t phase = (it / PSTAGES) & 1;
          if (!mbar_wait(&full_bar[stage], phase, abort)) {
            raise_error(p, abort, kErrTimeoutMma);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + (uint64_t)(stage * (PSTAGE_BYTES / 16));
          const uint64_t bd = b_desc0 + (uint64_t)(stage * (PSTAGE_BYTES / 16));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_f16_pair(d_tmem, ad + (uint64_t)(k * 2), bd + (uint64_t)(B_MN ? k * 128 : k * 2), idesc,
                         (kb | k) != 0);
          mma_commit_pair_both(&empty_bar[stage]);
        }
        if (ok) mma_commit_pair_both(&tfull_bar[acc]);
      }
    }
  } else {
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int tile = cluster; tile < num_tiles; tile += clusters, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      int ok = 0;
      if (lane == 0) {
        ok = mbar_wait(&tfull_bar[acc], acc_phase, abort);
        if (!ok) raise_error(p, abort, kErrTimeoutEpilogue);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(tile, tp, tm, tn);
      const int gm = tm * PTILE + rank * PBM + row;
      if (OUT == LC_F32 && p.c_vec8) {
        // f32 C: each thread writes its row's 32 columns of a chunk as four
        // 32-byte vectors (full sectors).  The epilogue's stores run while the
        // next tile's MMAs do, and stores of 16 bytes to 32 rows per warp
        // instruction (256 partial-sector requests per chunk) had kept the
        // load/store unit, which also serves the MMA thread's barrier polls,
        // saturated for most of a 2048-deep tile; these take half the requests.
        float *crow = static_cast<float *>(p.c) + (int64_t)gm * p.ldc;
#pragma unroll 1
        for (int c = 0; c < PTILE / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + acc * PTILE + c * 32, r);
          tmem_wait_ld();
          if (c == PTILE / 32 - 1) {  // the accumulator is in registers: release it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa(smem_u32(&tempty_bar[acc]), 0));
          }
          const int gn0 = tn * PTILE + c * 32;
          if (gm < p.m && gn0 + 32 <= p.n) {
            float v[32];
            chunk_values<EPI>(p, gn0, r, v);
#pragma unroll
            for (int q = 0; q < 4; ++q) st_global_v8(crow + gn0 + 8 * q, v + 8 * q);
          } else {
            store_chunk<OUT, EPI>(p, gm, gn0, r);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < PTILE / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + acc * PTILE + c * 32, r);
          tmem_wait_ld();
          store_chunk<OUT, EPI>(p, gm, tn * PTILE + c * 32, r);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa(smem_u32(&tempty_bar[acc]), 0));
      }
    }
  }

  __syncthreads();
  cluster_sync();  // neither CTA leaves while the pair's MMAs may touch its memory
  if (abort_flag) drain_delay();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- SIMT path

template <typename TI, int OUT, int EPI>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const TI *__restrict__ a,
                                                        const TI *__restrict__ b,
                                                        const float *__restrict__ bias, void *c,
                                                        int m, int n, int k, int b_nk) {
  __shared__ float as[16][17];
  __shared__ float bs[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  float acc = 0.f;
  for (int k0 = 0; k0 < k; k0 += 16) {
    const int ka = k0 + tx, kb = k0 + ty;
    as[ty][tx] = (row < m && ka < k) ? in_to_float(a[(int64_t)row * k + ka]) : 0.f;
    float bv = 0.f;
    if (col < n && kb < k) bv = in_to_float(b_nk ? b[(int64_t)col * k + kb] : b[(int64_t)kb * n + col]);
    bs[ty][tx] = bv;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) acc = fmaf(as[ty][i], bs[i][tx], acc);
    __syncthreads();
  }
  if (row < m && col < n) {
    if (bias) acc = __fadd_rn(acc, bias[col]);
    const float v = apply_epilogue<EPI>(acc);
    if constexpr (OUT == LC_F32) static_cast<float *>(c)[(int64_t)row * n + col] = v;
    else {
      using T = typename OutType<OUT>::type;
      static_cast<T *>(c)[(int64_t)row * n + col] = to_out<T>(v);
    }
  }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

int make_map_2d(CUtensorMap *map, bool bf16, const void *base, uint64_t inner, uint64_t outer,
                uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer) {
  auto fn = encode_fn();
  if (!fn) return fail(LC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LC_OK;
}

template <bool BF16, bool B_MN, int OUT, int EPI>
int launch_tc(const void *a, const void *b, const float *bias, void *c, int m, int n, int k,
              cudaStream_t s) {
  CUtensorMap ta, tb;
  if (int rc = make_map_2d(&ta, BF16, a, k, m, (uint64_t)k * 2, BK, BM)) return rc;
  if (B_MN) {
    if (int rc = make_map_2d(&tb, BF16, b, n, k, (uint64_t)n * 2, 64, BK)) return rc;
  } else {
    if (int rc = make_map_2d(&tb, BF16, b, k, n, (uint64_t)k * 2, BK, BN)) return rc;
  }
  GemmParams p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.c = c;
  p.bias = bias;
  p.ldc = n;
  p.tiles_m = (m + BM - 1) / BM;
  p.tiles_n = (n + BN - 1) / BN;
  const int elem = OUT == LC_F32 ? 4 : 2;
  p.vec_store = aligned(c, 16) && ((int64_t)n * elem) % 16 == 0;
  p.serpentine = 0;
  p.c_vec8 = OUT == LC_F32 && aligned(c, 32) && n % 8 == 0;
  if (int rc = device_error_word(&p.err)) return rc;
  auto kernel = gemm_tc_kernel<BF16, B_MN, OUT, EPI>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 SMEM_BYTES),
                            "gemm smem attribute"))
      return rc;
    configured[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  kernel<<<grid, THREADS, SMEM_BYTES, s>>>(ta, tb, p);
  return check_launch("lc_gemm");
}

template <bool BF16, bool B_MN, int OUT, int EPI>
int launch_tc2(const void *a, const void *b, const float *bias, void *c, int m, int n, int k,
               cudaStream_t s, bool any_k_order) {
  CUtensorMap ta, tb;
  if (int rc = make_map_2d(&ta, BF16, a, k, m, (uint64_t)k * 2, BK, PBM)) return rc;
  if (B_MN) {
    if (int rc = make_map_2d(&tb, BF16, b, n, k, (uint64_t)n * 2, 64, BK)) return rc;
  } else {
    if (int rc = make_map_2d(&tb, BF16, b, k, n, (uint64_t)k * 2, BK, PBN)) return rc;
  }
  GemmParams p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.c = c;
  p.bias = bias;
  p.ldc = n;
  p.tiles_m = (m + PTILE - 1) / PTILE;
  p.tiles_n = (n + PTILE - 1) / PTILE;
  const int elem = OUT == LC_F32 ? 4 : 2;
  p.vec_store = aligned(c, 16) && ((int64_t)n * elem) % 16 == 0;
  p.serpentine = any_k_order ? 1 : 0;
  // f32 C rows as 32-byte vectors when its base and rows are 32-byte aligned
  p.c_vec8 = OUT == LC_F32 && aligned(c, 32) && n % 8 == 0;
  if (int rc = device_error_word(&p.err)) return rc;
  auto kernel = gemm_tc2_kernel<BF16, B_MN, OUT, EPI>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 PSMEM_BYTES),
                            "gemm (2-SM) smem attribute"))
      return rc;
    configured[dev] = true;
  }
  const int tiles = p.tiles_m * p.tiles_n;
  // persistent: as many pairs as can be resident at once (GPC boundaries may
  // leave fewer than SMs / 2)
  static int resident[64] = {0};
  if (dev >= 0 && dev < 64 && resident[dev] == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count(), 1, 1);
    cfg.blockDim = dim3(THREADS, 1, 1);
    cfg.dynamicSmemBytes = PSMEM_BYTES;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters < 1) {
      cudaGetLastError();
      clusters = sm_count() / 2;
    }
    resident[dev] = clusters;
  }
  int clusters = (dev >= 0 && dev < 64) ? resident[dev] : sm_count() / 2;
  if (clusters > tiles) clusters = tiles;
  if (clusters < 1) clusters = 1;
  kernel<<<2 * clusters, THREADS, PSMEM_BYTES, s>>>(ta, tb, p);
  return check_launch("lc_gemm (2-SM)");
}

template <bool BF16, bool B_MN>
int dispatch_tc(int out, int epi, const void *a, const void *b, const float *bias, void *c, int m,
                int n, int k, cudaStream_t s, bool pair, bool any_k_order) {
#define LC_TC(O, E)                                                                    \
  if (out == O && epi == E)                                                            \
    return pair ? launch_tc2<BF16, B_MN, O, E>(a, b, bias, c, m, n, k, s, any_k_order) \
                : launch_tc<BF16, B_MN, O, E>(a, b, bias, c, m, n, k, s);
  LC_TC(LC_F32, LC_EPI_NONE) LC_TC(LC_F32, LC_EPI_GELU_ERF) LC_TC(LC_F32, LC_EPI_GELU_TANH)
  LC_TC(LC_F16, LC_EPI_NONE) LC_TC(LC_F16, LC_EPI_GELU_ERF) LC_TC(LC_F16, LC_EPI_GELU_TANH)
  LC_TC(LC_BF16, LC_EPI_NONE) LC_TC(LC_BF16, LC_EPI_GELU_ERF) LC_TC(LC_BF16, LC_EPI_GELU_TANH)
#undef LC_TC
  return fail(LC_ERR_INVALID, "lc_gemm: bad output type or epilogue");
}

template <typename TI>
int dispatch_simt(int out, int epi, const void *a, const void *b, const float *bias, void *c, int m,
                  int n, int k, int b_nk, cudaStream_t s) {
  dim3 grid((n + 15) / 16, (m + 15) / 16);
  const TI *ai = static_cast<const TI *>(a);
  const TI *bi = static_cast<const TI *>(b);
#define LC_SIMT(O, E)                                                       \
  if (out == O && epi == E) {                                               \
    gemm_simt_kernel<TI, O, E><<<grid, 256, 0, s>>>(ai, bi, bias, c, m, n, k, b_nk); \
    return check_launch("lc_gemm (simt)");                                  \
  }
  LC_SIMT(LC_F32, LC_EPI_NONE) LC_SIMT(LC_F32, LC_EPI_GELU_ERF) LC_SIMT(LC_F32, LC_EPI_GELU_TANH)
  LC_SIMT(LC_F16, LC_EPI_NONE) LC_SIMT(LC_F16, LC_EPI_GELU_ERF) LC_SIMT(LC_F16, LC_EPI_GELU_TANH)
  LC_SIMT(LC_BF16, LC_EPI_NONE) LC_SIMT(LC_BF16, LC_EPI_GELU_ERF) LC_SIMT(LC_BF16, LC_EPI_GELU_TANH)
#undef LC_SIMT
  return fail(LC_ERR_INVALID, "lc_gemm: bad output type or epilogue");
}

}  // namespace

// Chooses the path of one 16-bit GEMM: 2 = tcgen05 on SM pairs, 1 = tcgen05 on
// one SM, 0 = SIMT.
int gemm_path16(int b_layout, const void *a, const void *b, int64_t m, int64_t n, int64_t k) {
  return gemm_path16_shape(b_layout, aligned(a, 16), aligned(b, 16), m, n, k);
}

int gemm_path16_shape(int b_layout, bool a_aligned, bool b_aligned, int64_t m, int64_t n, int64_t k) {
  const bool tma_ok = k % 8 == 0 && a_aligned && b_aligned && (b_layout == LC_B_NK || n % 8 == 0) &&
                      k >= 16;
  const bool big = m * n * k >= ((int64_t)1 << 24);
  if (!(tma_ok && big)) return 0;
  const int64_t pair_tiles = ((m + PTILE - 1) / PTILE) * ((n + PTILE - 1) / PTILE);
  return m >= PTILE && n >= PTILE && pair_tiles >= 16 ? 2 : 1;
}

int gemm_tc_launch(bool bf16, bool b_mn, int out, int epi, const void *a, const void *b,
                   const float *bias, void *c, int m, int n, int k, cudaStream_t s, bool pair,
                   bool any_k_order) {
  const bool o = any_k_order;
  if (bf16) return b_mn ? dispatch_tc<true, true>(out, epi, a, b, bias, c, m, n, k, s, pair, o)
                        : dispatch_tc<true, false>(out, epi, a, b, bias, c, m, n, k, s, pair, o);
  return b_mn ? dispatch_tc<false, true>(out, epi, a, b, bias, c, m, n, k, s, pair, o)
              : dispatch_tc<false, false>(out, epi, a, b, bias, c, m, n, k, s, pair, o);
}

}  // namespace lc

extern "C" int lc_gemm_ex(int ab_dtype, int c_dtype, int b_layout, int epilogue, const void *a,
                          const void *b, const void *bias, void *c, int64_t m, int64_t n,
                          int64_t k, void *stream) {
  using namespace lc;
  if (ab_dtype != LC_F32 && ab_dtype != LC_F16 && ab_dtype != LC_BF16)
    return fail(LC_ERR_INVALID, "lc_gemm: unknown operand type %d", ab_dtype);
  if (c_dtype != LC_F32 && c_dtype != LC_F16 && c_dtype != LC_BF16)
    return fail(LC_ERR_INVALID, "lc_gemm: unknown output type %d", c_dtype);
  if (b_layout != LC_B_KN && b_layout != LC_B_NK)
    return fail(LC_ERR_INVALID, "lc_gemm: unknown B layout %d", b_layout);
  if (epilogue < LC_EPI_NONE || epilogue > LC_EPI_GELU_TANH)
    return fail(LC_ERR_INVALID, "lc_gemm: unknown epilogue %d", epilogue);
  if (m < 0 || n < 0 || k < 0) return fail(LC_ERR_INVALID, "lc_gemm: negative shape");
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return fail(LC_ERR_UNSUPPORTED, "lc_gemm: dimensions above 2^31-1");
  if (m == 0 || n == 0) return LC_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(LC_ERR_INVALID, "lc_gemm: null buffer");
  const float *bias_f = static_cast<const float *>(bias);
  cudaStream_t s = as_stream(stream);
  if (ab_dtype == LC_F32)
    return gemm_f32(c_dtype, b_layout, epilogue, a, b, bias_f, c, (int)m, (int)n, (int)k, s);
  const bool bf16 = ab_dtype == LC_BF16;
  const bool b_mn = b_layout == LC_B_KN;
  if (const int path = gemm_path16(b_layout, a, b, m, n, k))
    return gemm_tc_launch(bf16, b_mn, c_dtype, epilogue, a, b, bias_f, c, (int)m, (int)n, (int)k,
                          s, path == 2, true);
  if (bf16)
    return dispatch_simt<__nv_bfloat16>(c_dtype, epilogue, a, b, bias_f, c, m, n, k, !b_mn, s);
  return dispatch_simt<__half>(c_dtype, epilogue, a, b, bias_f, c, m, n, k, !b_mn, s);
}

extern "C" int lc_gemm(int ab_dtype, int c_dtype, int b_layout, int epilogue, const void *a,
                       const void *b, void *c, int64_t m, int64_t n, int64_t k, void *stream) {
  return lc_gemm_ex(ab_dtype, c_dtype, b_layout, epilogue, a, b, nullptr, c, m, n, k, stream);
}

extern "C" int lc_gemm_f32_dot2(int b_layout, int epilogue, const float *a, const float *b,
                                const float *bias, float *c, int64_t m, int64_t n, int64_t k,
                                void *stream) {
  using namespace lc;
  if (b_layout != LC_B_KN && b_layout != LC_B_NK)
    return fail(LC_ERR_INVALID, "lc_gemm_f32_dot2: unknown B layout %d", b_layout);
  if (epilogue < LC_EPI_NONE || epilogue > LC_EPI_GELU_TANH)
    return fail(LC_ERR_INVALID, "lc_gemm_f32_dot2: unknown epilogue %d", epilogue);
  if (m < 0 || n < 0 || k < 0) return fail(LC_ERR_INVALID, "lc_gemm_f32_dot2: negative shape");
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff)
    return fail(LC_ERR_UNSUPPORTED, "lc_gemm_f32_dot2: dimensions above 2^31-1");
  if (m == 0 || n == 0) return LC_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(LC_ERR_INVALID, "lc_gemm_f32_dot2: null buffer");
  return gemm_f32_dot2(b_layout, epilogue, a, b, bias, c, (int)m, (int)n, (int)k, as_stream(stream));
}

extern "C" int lc_gemm_path(int ab_dtype, int b_layout, const void *a, const void *b, int64_t m,
                            int64_t n, int64_t k) {
  if (ab_dtype == LC_F32) return lc::gemm_path32(b_layout, a, b, m, n, k);
  return lc::gemm_path16(b_layout, a, b, m, n, k);
}
