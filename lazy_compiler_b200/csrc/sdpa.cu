// Fused scaled-dot-product attention, f16 in/out, f32 softmax statistics.
//
// Replaces the reference's attention lowerings: the scalar per-output-element
// online softmax of a01/a02 (every thread recomputes a full QK dot per key),
// and the single 16x16 fragment tile of ptx_tensor.py:459-618 (QK mma.sync,
// FragmentRowReduce, FragmentApply exp/div, FragmentRepack to f16, PV mma.sync).
//
// Here, per CTA, two 128-row query tiles of one (batch, head), FlashAttention
// style on tcgen05 (the Blackwell "ping-pong" schedule):
//   warp 0     TMA: both Q tiles once, then K and V tiles of 128 keys through
//              a 2-stage ring (3-D tensor maps [bh, s, d] so a ragged tail
//              zero-fills inside its own head; 128-byte swizzle; no multicast);
//   warp 1     allocates all 512 TMEM columns (S0, S1, O0, O1: 128 columns of
//              f32 each) and one thread issues the MMAs in the order
//              PV0(j), S0(j+1), PV1(j), S1(j+1), so the tensor core computes one
//              tile's products while the other tile's softmax runs;
//   warps 2-9  two softmax warpgroups, one per query tile: each thread owns one
//              query row (its TMEM lane), loads the 128 scores, keeps the
//              running max m and sum l in f32, writes P = 2^(s*scale*log2e - m)
//              as f16 back into TMEM over the scores (the A operand of the PV
//              MMA is read from TMEM), and rescales O only when a row max grows
//              by more than 2^8 (the stale max is exact math: it cancels in
//              O / l); finally O / l is stored as f16.
// P is rounded to f16 before the PV product, as the reference's f16 attention
// tile rounds its normalised weights (FragmentRepack).  Every mbarrier wait is
// bounded; a wait that gives up writes the device error word.
// Other head sizes, unaligned bases or tiny problems use a SIMT kernel.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "sm100.cuh"

namespace lc {
namespace {

using namespace sm100;

constexpr int BQ = 128;       // rows of one query tile
constexpr int QT = 2;         // query tiles per CTA (one softmax warpgroup each)
constexpr int BKV = 128;
constexpr int HEAD = 128;
constexpr int CHUNK_BYTES = 128 * 64 * 2;     // 128 rows x 64 columns of f16 (one swizzle span)
constexpr int TILE_BYTES = 2 * CHUNK_BYTES;   // 128 rows x 128 columns
constexpr int KV_STAGES = 2;
constexpr int Q_BYTES = QT * TILE_BYTES;
constexpr int SMEM_BYTES = Q_BYTES + KV_STAGES * 2 * TILE_BYTES + 1024;
constexpr int THREADS = 64 + QT * 128;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 256;               // O tile t at O_COL + t * 128; S tile t at t * 128
constexpr float kRescaleThreshold = 8.0f;     // log2 units

struct SdpaParams {
  int s_q, s_kv, n_kv;
  int q_blocks, items;  // QT-tile query blocks per head; work items = heads x q_blocks
  float scale_log2;
  __half *o;
  int o_vec8;  // O is 32-byte aligned: rows are written with 32-byte stores
  int *err;
};

// One 32-byte store of eight 32-bit words (the address is 32-byte aligned).
__device__ __forceinline__ void st_global_v8_b32(void *dst, const uint32_t *v) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed pairs of f32 (Blackwell's f32x2 ALU forms: one instruction for two
// lanes of FMA, ADD or SUB).
__device__ __forceinline__ uint64_t pack2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair on the FMA pipe, for a share of the exponentials so the MUFU
// unit is not the limiter.  Range reduction: x = n + f with n = round(x) taken
// from the low mantissa bits of x + 1.5*2^23 and f in [-0.5, 0.5]; 2^f from a
// degree-3 polynomial fitted here by the Remez exchange algorithm for minimax
// relative error on [-0.5, 0.5] (max relative error 7.5e-5, below half an f16
// ulp); 2^n is added to the exponent field.  x is clamped at -125 so the
// exponent stays normal; the caller's x never exceeds 8.
__device__ __forceinline__ uint64_t ex2_poly2(uint64_t x2) {
  const float2 x = unpack2(x2);
  const uint64_t xc = pack2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
  const uint64_t magic = pack2(12582912.0f, 12582912.0f);
  const uint64_t t = fadd2(xc, magic);
  const uint64_t f = fsub2(xc, fsub2(t, magic));
  uint64_t q = ffma2(pack2(0.0551716685f, 0.0551716685f), f, pack2(0.242611125f, 0.242611125f));
  q = ffma2(q, f, pack2(0.693260968f, 0.693260968f));
  q = ffma2(q, f, pack2(0.999928057f, 0.999928057f));
  const float2 qq = unpack2(q), tt = unpack2(t);
  return pack2(__int_as_float(__float_as_int(qq.x) + (__float_as_int(tt.x) << 23)),
               __int_as_float(__float_as_int(qq.y) + (__float_as_int(tt.y) << 23)));
}

__device__ __forceinline__ void raise_error(const SdpaParams &p, volatile int *abort, int code) {
  *abort = 1;
  atomicCAS(p.err, 0, code);
}

// Every lane waits (one lane waiting and broadcasting costs a divergent
// branch and a shuffle on the softmax's critical path); the warp agrees on
// the outcome, so a wait that gave up in any lane fails for all.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          const SdpaParams &p, int code) {
  const int ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, abort) ? 1 : 0);
  if (!ok && (threadIdx.x & 31) == 0) raise_error(p, abort, code);
  return ok != 0;
}

__global__ void __launch_bounds__(THREADS, 1)
    sdpa_tc_kernel(const __grid_constant__ CUtensorMap tma_q, const __grid_constant__ CUtensorMap tma_k,
                   const __grid_constant__ CUtensorMap tma_v, SdpaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t *q_s = smem;
  uint8_t *kv_s = smem + Q_BYTES;
  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t q_empty;
  __shared__ __align__(8) uint64_t k_full[KV_STAGES];
  __shared__ __align__(8) uint64_t v_full[KV_STAGES];
  __shared__ __align__(8) uint64_t k_empty[KV_STAGES];
  __shared__ __align__(8) uint64_t v_empty[KV_STAGES];
  __shared__ __align__(8) uint64_t s_full[QT];
  __shared__ __align__(8) uint64_t p_full[QT];
  __shared__ __align__(8) uint64_t o_done[QT];
  __shared__ __align__(8) uint64_t o_empty[QT];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int *abort = &abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int t = 0; t < QT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&o_done[t], 1);
      mbar_init(&o_empty[t], 4);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_q);
    prefetch_tmap(&tma_k);
    prefetch_tmap(&tma_v);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int n = p.n_kv;
  // Persistent: work item w is query block w % q_blocks of head w / q_blocks;
  // CTA c takes items c, c + gridDim.x, ...  Every barrier phase counts over
  // all items of the CTA: KV block g (g = local item * n + j) uses K/V stage
  // g & 1, and s_full / p_full / o_done complete once per block.

  if (warp == 0) {
    if (lane == 0) {
      int g = 0, local = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.items; item += gridDim.x, ++local) {
        const int bh = item / p.q_blocks, qb = item - bh * p.q_blocks;
        // Q of the previous item is free once its last S products completed
        if (local > 0 && !mbar_wait(&q_empty, (local - 1) & 1, abort)) {
          raise_error(p, abort, kErrTimeoutProducer);
          break;
        }
        mbar_expect_tx(&q_full, Q_BYTES);
        for (int t = 0; t < QT; ++t) {
          const int row0 = (qb * QT + t) * BQ;
          tma_load_3d(q_s + t * TILE_BYTES, &tma_q, &q_full, 0, row0, bh);
          tma_load_3d(q_s + t * TILE_BYTES + CHUNK_BYTES, &tma_q, &q_full, 64, row0, bh);
        }
        // K(j) is released once both S(j) products completed, V(j) once both PV(j)
        // products completed, so K(j+2) loads while V(j) is still in use.
        for (int j = 0; j < n; ++j, ++g) {
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          uint8_t *k_s = kv_s + st * 2 * TILE_BYTES;
          uint8_t *v_s = k_s + TILE_BYTES;
          if (!mbar_wait(&k_empty[st], ph ^ 1, abort)) {
            raise_error(p, abort, kErrTimeoutProducer);
            ok = false;
            break;
          }
          mbar_expect_tx(&k_full[st], TILE_BYTES);
          tma_load_3d(k_s, &tma_k, &k_full[st], 0, j * BKV, bh);
          tma_load_3d(k_s + CHUNK_BYTES, &tma_k, &k_full[st], 64, j * BKV, bh);
          if (!mbar_wait(&v_empty[st], ph ^ 1, abort)) {
            raise_error(p, abort, kErrTimeoutProducer);
            ok = false;
            break;
          }
          mbar_expect_tx(&v_full[st], TILE_BYTES);
          tma_load_3d(v_s, &tma_v, &v_full[st], 0, j * BKV, bh);
          tma_load_3d(v_s + CHUNK_BYTES, &tma_v, &v_full[st], 64, j * BKV, bh);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_f16(false, false, false, BQ, BKV);
      constexpr uint32_t idesc_o = idesc_f16(false, false, true, BQ, HEAD);
      // Shared-memory descriptors are built once; an MMA adds its operand's
      // byte offset / 16 to the 14-bit start-address field (no carry: every
      // address is below 256 KB), so issuing one costs a single integer add.
      const uint64_t q_desc = smem_desc_sw128(smem_u32(q_s), 16, 1024);
      const uint64_t k_desc = smem_desc_sw128(smem_u32(kv_s), 16, 1024);
      const uint64_t v_desc = smem_desc_sw128(smem_u32(kv_s) + TILE_BYTES, CHUNK_BYTES, 1024);
      constexpr uint32_t kStageStep = 2 * TILE_BYTES / 16;
      // S_t = Q_t K(block g)^T into TMEM columns [t*128, t*128+128)
      auto issue_s = [&](int t, int g) {
        const uint64_t qd = q_desc + (uint64_t)(t * TILE_BYTES / 16);
        const uint64_t kd = k_desc + (uint64_t)((g & 1) * kStageStep);
        const uint32_t d_tmem = tmem + t * BKV;
#pragma unroll
        for (int k = 0; k < HEAD / 16; ++k) {
          const uint32_t off = ((k >> 2) * CHUNK_BYTES + (k & 3) * 32) / 16;
          mma_f16(d_tmem, qd + off, kd + off, idesc_s, k > 0);
        }
        mma_commit(&s_full[t]);
      };
      // O_t (+)= P_t V(block g), P_t read from TMEM over S_t; the item's first
      // block overwrites O
      auto issue_pv = [&](int t, int g, bool first) {
        const uint64_t vd = v_desc + (uint64_t)((g & 1) * kStageStep);
        const uint32_t d_tmem = tmem + O_COL + t * HEAD;
        const uint32_t a_tmem = tmem + t * BKV;
#pragma unroll
        for (int k = 0; k < BKV / 16; ++k)
          mma_f16_tmem_a(d_tmem, a_tmem + k * 8, vd + (uint64_t)(k * 2048 / 16), idesc_o,
                         !(first && k == 0));
        mma_commit(&o_done[t]);
      };
      int g0 = 0, local = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < p.items; item += gridDim.x, ++local, g0 += n) {
        ok = mbar_wait(&q_full, local & 1, abort) && mbar_wait(&k_full[g0 & 1], (g0 >> 1) & 1, abort);
        if (!ok) break;
        tc_fence_after();
        for (int t = 0; t < QT; ++t) issue_s(t, g0);
        mma_commit(&k_empty[g0 & 1]);
        if (n == 1) mma_commit(&q_empty);
        for (int j = 0; ok && j < n; ++j) {
          const int g = g0 + j;
          const int st = g & 1;
          const uint32_t ph = (g >> 1) & 1;
          const bool next = j + 1 < n;
          for (int t = 0; t < QT; ++t) {
            // The operands (V(j), K(j+1), a free O) are ready long before the
            // softmax's P, so they are waited for first: a wait costs a
            // shared-memory round trip even when its phase has completed, and
            // only the P wait should sit between the softmax and the MMAs.
            if ((t == 0 && !mbar_wait(&v_full[st], ph, abort)) ||
                (t == 0 && next && !mbar_wait(&k_full[(g + 1) & 1], ((g + 1) >> 1) & 1, abort)) ||
                (j == 0 && local > 0 && !mbar_wait(&o_empty[t], (local - 1) & 1, abort)) ||
                !mbar_wait(&p_full[t], g & 1, abort)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, g, j == 0);
            if (t == QT - 1) mma_commit(&v_empty[st]);
            if (next) {
              issue_s(t, g + 1);
              if (t == QT - 1) {
                mma_commit(&k_empty[(g + 1) & 1]);
                if (j + 2 == n) mma_commit(&q_empty);  // the item's last S products
              }
            }
          }
        }
      }
      if (!ok) raise_error(p, abort, kErrTimeoutMma);
    }
  } else {
    const int t = (warp - 2) >> 2;  // query tile of this softmax warpgroup
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = t * BKV;
    const uint32_t o_col = O_COL + t * HEAD;
    int g0 = 0;
    bool ok = true;
    for (int item = blockIdx.x; ok && item < p.items; item += gridDim.x, g0 += n) {
      const int bh = item / p.q_blocks, qb = item - bh * p.q_blocks;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        const int g = g0 + j;
        if (!warp_wait(&s_full[t], g & 1, abort, p, kErrTimeoutSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sr[4][32];
  #pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(tmem + lane_base + s_col + c * 32, sr[c]);
        tmem_wait_ld();
        const int valid = p.s_kv - j * BKV;
        if (valid < BKV) {  // ragged last KV tile (uniform across the CTA): mask absent keys
  #pragma unroll
          for (int c = 0; c < 4; ++c)
  #pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c * 32 + i >= valid) sr[c][i] = __float_as_uint(-INFINITY);
        }
        // max of the raw scores (the positive scale commutes with max), as 8
        // independent chains so the reduction is not one 128-deep dependency
        float mx8[8];
  #pragma unroll
        for (int k = 0; k < 8; ++k) mx8[k] = -INFINITY;
  #pragma unroll
        for (int c = 0; c < 4; ++c)
  #pragma unroll
          for (int i = 0; i < 32; i += 2)
            mx8[(i >> 1) & 7] = max3(mx8[(i >> 1) & 7], __uint_as_float(sr[c][i]),
                                     __uint_as_float(sr[c][i + 1]));
        float mx = max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]),
                        fmaxf(mx8[6], mx8[7]));
        mx *= p.scale_log2;
        const float m_new = fmaxf(m, mx);
        const bool need = m_new > m + kRescaleThreshold;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2(m - m_new) : 1.0f;
          if (need) {
            l *= alpha;
            m = m_new;
          }
          if (j > 0) {
            if (!warp_wait(&o_done[t], (g - 1) & 1, abort, p, kErrTimeoutCorrection)) {
              ok = false;
              break;
            }
            tc_fence_after();
  #pragma unroll 1
            for (int c = 0; c < HEAD / 16; ++c) {
              uint32_t o[16];
              tmem_ld16(tmem + lane_base + o_col + c * 16, o);
              tmem_wait_ld();
  #pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16(tmem + lane_base + o_col + c * 16, o);
            }
            tmem_wait_st();
          }
        }
        // independent row-sum chains, each a pair of f32 lanes
        uint64_t part2[4] = {0ull, 0ull, 0ull, 0ull};
        const uint64_t scale2 = pack2(p.scale_log2, p.scale_log2);
        const uint64_t neg_m2 = pack2(-m, -m);
  #pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t packed[16];
  #pragma unroll
          for (int i = 0; i < 16; ++i) {
            // p = 2^(s * scale * log2 e - m): one paired FMA, then MUFU ex2 or
            // (one pair in sixteen) the paired polynomial
            const uint64_t x2 = ffma2(pack2(__uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1])),
                                      scale2, neg_m2);
            uint64_t p2;
            if (i == 15) {
              p2 = ex2_poly2(x2);
            } else {
              const float2 x = unpack2(x2);
              p2 = pack2(ex2(x.x), ex2(x.y));
            }
            part2[i & 3] = fadd2(part2[i & 3], p2);
            const float2 pp = unpack2(p2);
            __half2 h = __floats2half2_rn(pp.x, pp.y);
            packed[i] = *reinterpret_cast<uint32_t *>(&h);
          }
          tmem_st16(tmem + lane_base + s_col + c * 16, packed);
        }
        tmem_wait_st();
        const float2 s01 = unpack2(fadd2(fadd2(part2[0], part2[1]), fadd2(part2[2], part2[3])));
        l += s01.x + s01.y;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      if (!ok || n == 0) break;
      if (!warp_wait(&o_done[t], (g0 + n - 1) & 1, abort, p, kErrTimeoutSoftmax)) break;
      tc_fence_after();
      const float inv = 1.0f / l;
      const int q = (qb * QT + t) * BQ + row;
      __half *out = p.o + ((int64_t)bh * p.s_q + q) * HEAD;
      // Each thread writes its row; 32-byte vector stores (full sectors) where
      // O is 32-byte aligned keep the load/store unit's request count, which
      // the other tile's barrier polls share, at half that of 16-byte stores.
#pragma unroll 1
      for (int c = 0; c < HEAD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_base + o_col + c * 32, o);
        tmem_wait_ld();
        if (c == HEAD / 32 - 1) {
          // O of this tile may now be overwritten by the next item's first PV
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_empty[t]);
        }
        if (q < p.s_q) {
          uint32_t h[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            __half2 hh = __floats2half2_rn(__uint_as_float(o[2 * i]) * inv, __uint_as_float(o[2 * i + 1]) * inv);
            h[i] = *reinterpret_cast<uint32_t *>(&hh);
          }
          if (p.o_vec8) {
            st_global_v8_b32(out + c * 32, h);
            st_global_v8_b32(out + c * 32 + 16, h + 8);
          } else {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<uint4 *>(out + c * 32)[i] = make_uint4(h[4 * i], h[4 * i + 1], h[4 * i + 2], h[4 * i + 3]);
          }
        }
      }
    }
  }

  __syncthreads();
  if (abort_flag) drain_delay();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- SIMT path
// One warp per query row, online softmax in f32, any head size up to 256.
__global__ void __launch_bounds__(256) sdpa_simt_kernel(const __half *__restrict__ q,
                                                        const __half *__restrict__ k,
                                                        const __half *__restrict__ v,
                                                        __half *__restrict__ o, int s_q, int s_kv,
                                                        int d, float scale) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  const int64_t bh = blockIdx.y;
  if (row >= s_q) return;
  constexpr int kMaxPerLane = 8;
  float qv[kMaxPerLane], acc[kMaxPerLane];
  const __half *qr = q + (bh * s_q + row) * d;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    qv[i] = c < d ? __half2float(qr[c]) : 0.f;
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int key = 0; key < s_kv; ++key) {
    const __half *kr = k + (bh * s_kv + key) * d;
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int c = lane + 32 * i;
      if (c < d) dot = fmaf(qv[i], __half2float(kr[c]), dot);
    }
    dot = warp_sum(dot) * scale;
    const float m_new = fmaxf(m, dot);
    const float alpha = expf(m - m_new);
    const float pw = expf(dot - m_new);
    l = l * alpha + pw;
    const float ph = __half2float(__float2half_rn(pw));
    const __half *vr = v + (bh * s_kv + key) * d;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int c = lane + 32 * i;
      acc[i] = acc[i] * alpha + (c < d ? ph * __half2float(vr[c]) : 0.f);
    }
    m = m_new;
  }
  __half *orow = o + (bh * s_q + row) * d;
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int c = lane + 32 * i;
    if (c < d) orow[c] = __float2half_rn(acc[i] / l);
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

// [bh, s, 128] f16 viewed as a 3-D tensor, box 64 x 128 x 1, 128-byte swizzle.
int make_map_3d(CUtensorMap *map, const void *base, int64_t bh, int64_t s) {
  auto fn = encode_fn();
  if (!fn) return fail(LC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)HEAD, (cuuint64_t)s, (cuuint64_t)bh};
  cuuint64_t strides[2] = {(cuuint64_t)HEAD * 2, (cuuint64_t)s * HEAD * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LC_OK;
}

}  // namespace

int sdpa_path(const void *q, const void *k, const void *v, const void *o, int64_t s_q,
              int64_t s_kv, int64_t d) {
  const bool tc = d == HEAD && aligned(q, 16) && aligned(k, 16) && aligned(v, 16) &&
                  aligned(o, 16) && s_q >= 1 && s_kv >= 1 && s_q * s_kv >= 128 * 128;
  return tc ? 1 : 0;
}

}  // namespace lc

extern "C" int lc_sdpa_f16(const void *q, const void *k, const void *v, void *o, int64_t bh,
                           int64_t s_q, int64_t s_kv, int64_t d, float scale, void *stream) {
  using namespace lc;
  if (bh < 0 || s_q < 0 || s_kv < 0 || d < 0) return fail(LC_ERR_INVALID, "lc_sdpa_f16: negative shape");
  if (bh == 0 || s_q == 0) return LC_OK;
  if (s_kv == 0) return fail(LC_ERR_INVALID, "lc_sdpa_f16: softmax over zero keys is undefined");
  if (d == 0 || d > 256) return fail(LC_ERR_UNSUPPORTED, "lc_sdpa_f16: head size %lld", (long long)d);
  if (!q || !k || !v || !o) return fail(LC_ERR_INVALID, "lc_sdpa_f16: null buffer");
  if (bh > 65535 || s_q > 0x7fffffff / 2 || s_kv > 0x7fffffff / 2)
    return fail(LC_ERR_UNSUPPORTED, "lc_sdpa_f16: shape too large");
  if (!(scale > 0.f)) return fail(LC_ERR_INVALID, "lc_sdpa_f16: scale must be positive");
  cudaStream_t s = as_stream(stream);
  if (!sdpa_path(q, k, v, o, s_q, s_kv, d)) {
    dim3 grid((unsigned)((s_q + 7) / 8), (unsigned)bh);
    sdpa_simt_kernel<<<grid, 256, 0, s>>>(static_cast<const __half *>(q), static_cast<const __half *>(k),
                                          static_cast<const __half *>(v), static_cast<__half *>(o),
                                          (int)s_q, (int)s_kv, (int)d, scale);
    return check_launch("lc_sdpa_f16 (simt)");
  }
  CUtensorMap tq, tk, tv;
  if (int rc = make_map_3d(&tq, q, bh, s_q)) return rc;
  if (int rc = make_map_3d(&tk, k, bh, s_kv)) return rc;
  if (int rc = make_map_3d(&tv, v, bh, s_kv)) return rc;
  SdpaParams p;
  p.s_q = (int)s_q;
  p.s_kv = (int)s_kv;
  p.n_kv = (int)((s_kv + BKV - 1) / BKV);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = static_cast<__half *>(o);
  p.o_vec8 = aligned(o, 32) ? 1 : 0;
  if (int rc = device_error_word(&p.err)) return rc;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(sdpa_tc_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 SMEM_BYTES),
                            "sdpa smem attribute"))
      return rc;
    configured[dev] = true;
  }
  // persistent: one CTA per SM (shared memory and TMEM admit one)
  p.q_blocks = (int)((s_q + QT * BQ - 1) / (QT * BQ));
  p.items = (int)(bh * p.q_blocks);
  const int grid = p.items < sm_count() ? p.items : sm_count();
  sdpa_tc_kernel<<<grid, THREADS, SMEM_BYTES, s>>>(tq, tk, tv, p);
  return check_launch("lc_sdpa_f16");
}

extern "C" int lc_sdpa_path(const void *q, const void *k, const void *v, const void *o,
                            int64_t s_q, int64_t s_kv, int64_t d) {
  return lc::sdpa_path(q, k, v, o, s_q, s_kv, d);
}
