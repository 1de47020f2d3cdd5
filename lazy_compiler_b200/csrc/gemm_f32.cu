// FP32 GEMM, C = epilogue(A B + bias), at FP32 accuracy and without TF32.
//
// Replaces the reference's scalar FP32 matmul lowering: Emmy-scheduled tiles
// whose operands are staged by cp.async (ptx_backend.py:1457-1492), summed per
// element with FMA or the Dot2 compensated dot product (ptx_backend.py:337-374,
// 571-593) and, for split-K schedules, combined with red.global.add into
// launcher-zeroed outputs (ptx_backend.py:1307-1318).  Packages of this class:
// problems/m01_matmul_512, problems/m02_matmul_rect and
// examples/phase9/generated/phase9_bias_gelu_gemm.
//
// Two paths (lc_gemm_path reports which one runs):
//  * lc_gemm_f32_dot2 (packages that state a tolerance, where the reference
//    compensates each output's dot product): the SIMT kernel below with every
//    output a Dot2 pair (dot2_step / dot2_value, common.cuh), 64x64 tiles.
//  * SIMT (path 0): a persistent FFMA kernel over 128x128 (or, when there are
//    fewer such tiles than SMs, 64x64) output tiles, 8x8 (4x4) outputs per
//    thread, k-slices of 8 double-buffered in shared memory.  Small problems and
//    shapes TMA cannot describe take it.  When even 64x64 tiles leave SMs idle,
//    the contraction is split into up to 16 chunks whose partial products a
//    second kernel adds in a fixed order (deterministic), with the bias and
//    activation.
//  * Tensor cores (paths 1, 2): every f32 value x is split exactly into three
//    bf16 pieces, hi = bf16(x), mid = bf16(x - hi), lo = bf16(x - hi - mid)
//    (both subtractions are exact; |x - hi - mid - lo| <= 2^-24 |x|).  The six
//    piece products down to 2^-16 of the leading one are summed by the bf16
//    tcgen05 GEMM as one product of K-concatenated operands,
//        A' = [A_mid A_lo A_hi A_mid A_hi A_hi]      (M x 6K)
//        B' = [B_mid;B_hi;B_lo;B_hi;B_mid;B_hi]      (6K x N, or N x 6K for [N,K] B)
//    so the small products enter the f32 accumulator first.  The three dropped
//    products are below 2^-23 of |a b|, the size of one f32 rounding.  A value
//    whose hi piece is not finite (inf, NaN, or above the bf16 range) sets a
//    device flag; a SIMT kernel launched behind the GEMM returns at once when
//    the flag is clear and otherwise recomputes C in plain f32, so IEEE
//    special values propagate as they do in the reference.
// The split operands live in a library-owned scratch buffer (12 (M + N) K
// bytes) per device and stream.
#include "common.cuh"
#include "epilogue.cuh"

namespace lc {
namespace {

constexpr int SK = 8;                   // k-slice of the SIMT kernel
constexpr int kThreads = 256;
constexpr int64_t kSplitMacs = (int64_t)1 << 30;  // tensor-core path from here up
constexpr int kScratchSlot = 0;      // bf16 split operands of the tensor-core path
constexpr int kSplitSlot = 1;        // split-K partial products of the SIMT path
constexpr int kMinChunk = 64;        // smallest contraction chunk of a split
constexpr int kMaxSplits = 16;

// Piece orders of A' and B' slots: 0 = hi, 1 = mid, 2 = lo (two bits a slot).
constexpr int pack_order(int s0, int s1, int s2, int s3, int s4, int s5) {
  return s0 | s1 << 2 | s2 << 4 | s3 << 6 | s4 << 8 | s5 << 10;
}
constexpr int kOrderA = pack_order(1, 2, 0, 1, 0, 0);
constexpr int kOrderB = pack_order(1, 0, 2, 0, 1, 0);

__device__ __forceinline__ void split3(float x, __nv_bfloat16 (&p)[3], bool &bad) {
  p[0] = __float2bfloat16_rn(x);
  const float hi = __bfloat162float(p[0]);
  const float r1 = __fsub_rn(x, hi);
  p[1] = __float2bfloat16_rn(r1);
  const float r2 = __fsub_rn(r1, __bfloat162float(p[1]));
  p[2] = __float2bfloat16_rn(r2);
  if (!isfinite(hi)) {
    bad = true;
    p[1] = p[2] = __float2bfloat16_rn(0.f);
  }
}

// Splits a row-major [rows, cols] f32 matrix (cols % 4 == 0, 16-byte aligned)
// into six bf16 slots: element (r, c) of slot s goes to
// out[r * row_stride + s * slot_stride + c].
template <int ORDER>
__global__ void __launch_bounds__(kThreads) split3_kernel(const float *__restrict__ x,
                                                          __nv_bfloat16 *__restrict__ out,
                                                          int64_t rows, int64_t cols,
                                                          int64_t row_stride, int64_t slot_stride,
                                                          int *nonfinite) {
  const int64_t c4 = cols >> 2;
  const int64_t total = rows * c4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / c4;
    const int64_t c = (i - r * c4) << 2;
    const float4 v = ld_stream(reinterpret_cast<const float4 *>(x + r * cols + c));
    __nv_bfloat16 p0[3], p1[3], p2[3], p3[3];
    bool bad = false;
    split3(v.x, p0, bad);
    split3(v.y, p1, bad);
    split3(v.z, p2, bad);
    split3(v.w, p3, bad);
    if (bad) atomicOr(nonfinite, 1);
    __nv_bfloat16 *dst = out + r * row_stride + c;
#pragma unroll
    for (int s = 0; s < 6; ++s) {
      const int piece = (ORDER >> (2 * s)) & 3;
      __nv_bfloat16 q[4] = {p0[piece], p1[piece], p2[piece], p3[piece]};
      *reinterpret_cast<uint2 *>(dst + s * slot_stride) = *reinterpret_cast<const uint2 *>(q);
    }
  }
}

// SIMT FP32 GEMM.  TM = 8: 128x128 tiles, rows ty*4+{0..3} and 64+ty*4+{0..3}
// of a thread (likewise columns); TM = 4: 64x64 tiles.  `flag`, when given,
// makes the kernel a guard: it returns unless *flag is non-zero.  With
// `partial`, blockIdx.y picks the k range [y * k_chunk, (y + 1) * k_chunk) and
// the raw sums go to partial[y][M][N] (no bias, no activation) for
// split_k_reduce_kernel.  COMP: every output accumulates as a Dot2 pair
// (dot2_step in k order), read as dot2_value.
template <int TM, int EPI, bool B_NK, bool COMP = false>
__global__ void __launch_bounds__(kThreads, 2) gemm_f32_simt_kernel(
    const float *__restrict__ a, const float *__restrict__ b, const float *__restrict__ bias,
    float *__restrict__ c, int m, int n, int k, const int *flag, int k_chunk,
    float *__restrict__ partial) {
  if (flag && *reinterpret_cast<const volatile int *>(flag) == 0) return;
  constexpr int ST = 16 * TM;         // tile edge
  constexpr int LPT = TM / 2;         // elements of each operand a thread loads per slice
  constexpr int KT = SK / LPT;        // threads along k for A and [N,K] B
  __shared__ __align__(16) float As[2][SK][ST];
  __shared__ __align__(16) float Bs[2][SK][ST];
  const int t = threadIdx.x, tx = t & 15, ty = t >> 4;
  const int tiles_n = (n + ST - 1) / ST;
  const int tiles = ((m + ST - 1) / ST) * tiles_n;
  const int a_row = t / KT, a_k = (t % KT) * LPT;     // A and [N,K] B
  const int b_k = t / (ST / LPT), b_col = (t % (ST / LPT)) * LPT;  // [K,N] B
  const int k_lo = partial ? blockIdx.y * k_chunk : 0;
  const int k_hi = partial ? min(k, k_lo + k_chunk) : k;
  float *out = partial ? partial + (int64_t)blockIdx.y * m * n : c;
  const bool vec_out = (n & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;

  for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int m0 = (tile / tiles_n) * ST, n0 = (tile % tiles_n) * ST;
    float ra[LPT], rb[LPT];
    auto load = [&](int k0) {
      const int gr = m0 + a_row;
#pragma unroll
      for (int q = 0; q < LPT; ++q) {
        const int kk = k0 + a_k + q;
        ra[q] = (gr < m && kk < k_hi) ? a[(int64_t)gr * k + kk] : 0.f;
      }
      if constexpr (B_NK) {
        const int gc = n0 + a_row;
#pragma unroll
        for (int q = 0; q < LPT; ++q) {
          const int kk = k0 + a_k + q;
          rb[q] = (gc < n && kk < k_hi) ? b[(int64_t)gc * k + kk] : 0.f;
        }
      } else {
        const int kk = k0 + b_k;
#pragma unroll
        for (int q = 0; q < LPT; ++q) {
          const int gc = n0 + b_col + q;
          rb[q] = (kk < k_hi && gc < n) ? b[(int64_t)kk * n + gc] : 0.f;
        }
      }
    };
    auto store = [&](int buf) {
#pragma unroll
      for (int q = 0; q < LPT; ++q) As[buf][a_k + q][a_row] = ra[q];
      if constexpr (B_NK) {
#pragma unroll
        for (int q = 0; q < LPT; ++q) Bs[buf][a_k + q][a_row] = rb[q];
      } else {
#pragma unroll
        for (int q = 0; q < LPT; ++q) Bs[buf][b_k][b_col + q] = rb[q];
      }
    };

    float acc[TM][TM];
    float low[COMP ? TM : 1][COMP ? TM : 1];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TM; ++j) acc[i][j] = 0.f;
    if constexpr (COMP) {
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TM; ++j) low[i][j] = 0.f;
    }

    load(k_lo);
    store(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = k_lo; k0 < k_hi; k0 += SK) {
      const bool more = k0 + SK < k_hi;
      if (more) load(k0 + SK);
#pragma unroll
      for (int kk = 0; kk < SK; ++kk) {
        float av[TM], bv[TM];
#pragma unroll
        for (int h = 0; h < TM / 4; ++h) {
          const float4 x = *reinterpret_cast<const float4 *>(&As[buf][kk][h * 64 + ty * 4]);
          const float4 y = *reinterpret_cast<const float4 *>(&Bs[buf][kk][h * 64 + tx * 4]);
          av[h * 4 + 0] = x.x, av[h * 4 + 1] = x.y, av[h * 4 + 2] = x.z, av[h * 4 + 3] = x.w;
          bv[h * 4 + 0] = y.x, bv[h * 4 + 1] = y.y, bv[h * 4 + 2] = y.z, bv[h * 4 + 3] = y.w;
        }
        if constexpr (COMP) {
#pragma unroll
          for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TM; ++j) dot2_step(acc[i][j], low[i][j], av[i], bv[j]);
        } else {
#pragma unroll
          for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TM; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
      }
      if (more) store(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }

#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int row = m0 + (i >> 2) * 64 + ty * 4 + (i & 3);
      if (row >= m) continue;
#pragma unroll
      for (int h = 0; h < TM / 4; ++h) {
        const int col = n0 + h * 64 + tx * 4;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float x;
          if constexpr (COMP) x = dot2_value(acc[i][h * 4 + j], low[i][h * 4 + j]);
          else x = acc[i][h * 4 + j];
          if (!partial) {
            if (bias && col + j < n) x = __fadd_rn(x, bias[col + j]);
            x = apply_epilogue<EPI>(x);
          }
          v[j] = x;
        }
        float *dst = out + (int64_t)row * n + col;
        if (vec_out && col + 3 < n) {
          *reinterpret_cast<float4 *>(dst) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (col + j < n) dst[j] = v[j];
        }
      }
    }
    __syncthreads();  // the next tile's first slice overwrites shared memory
  }
}

// Sums the split-K partial products in a fixed order, adds the bias and
// applies the activation: deterministic for a given shape.
template <int EPI>
__global__ void __launch_bounds__(kThreads) split_k_reduce_kernel(const float *__restrict__ partial,
                                                                  const float *__restrict__ bias,
                                                                  float *__restrict__ c, int m, int n,
                                                                  int splits) {
  const int64_t total = (int64_t)m * n;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    float x = partial[i];
    for (int sp = 1; sp < splits; ++sp) x = __fadd_rn(x, partial[sp * total + i]);
    if (bias) x = __fadd_rn(x, bias[i % n]);
    c[i] = apply_epilogue<EPI>(x);
  }
}

template <int TM, int EPI, bool COMP = false>
int launch_simt_tm(bool b_nk, const float *a, const float *b, const float *bias, float *c, int m,
                   int n, int k, const int *flag, cudaStream_t s) {
  constexpr int ST = 16 * TM;
  const int64_t tiles = (int64_t)((m + ST - 1) / ST) * ((n + ST - 1) / ST);
  const int64_t cap = 2LL * sm_count();
  const int grid = (int)(tiles < cap ? tiles : cap);
  // Too few output tiles to fill the GPU: split the contraction into chunks
  // of at least kMinChunk and reduce the partial products in a second pass.
  int splits = 1;
  if (!flag && tiles < sm_count() && k >= 2 * kMinChunk) {
    const int64_t want = (2LL * sm_count() + tiles - 1) / tiles;
    const int64_t most = k / kMinChunk;
    splits = (int)(want < most ? want : most);
    if (splits > kMaxSplits) splits = kMaxSplits;
  }
  if (splits > 1) {
    const int k_chunk = ((k + splits - 1) / splits + SK - 1) / SK * SK;
    splits = (k + k_chunk - 1) / k_chunk;
    void *ws = nullptr;
    if (int rc = scratch_buffer(s, kSplitSlot, (size_t)splits * m * n * sizeof(float), &ws)) return rc;
    float *part = static_cast<float *>(ws);
    dim3 g2((unsigned)grid, (unsigned)splits);
    if (b_nk)
      gemm_f32_simt_kernel<TM, EPI, true, COMP><<<g2, kThreads, 0, s>>>(a, b, bias, c, m, n, k, flag, k_chunk,
                                                                        part);
    else
      gemm_f32_simt_kernel<TM, EPI, false, COMP><<<g2, kThreads, 0, s>>>(a, b, bias, c, m, n, k, flag,
                                                                         k_chunk, part);
    if (int rc = check_launch("lc_gemm (f32 simt, split k)")) return rc;
    const int64_t total = (int64_t)m * n;
    const int64_t blocks = (total + kThreads - 1) / kThreads;
    const int rgrid = (int)(blocks < 4LL * sm_count() ? blocks : 4LL * sm_count());
    split_k_reduce_kernel<EPI><<<rgrid, kThreads, 0, s>>>(part, bias, c, m, n, splits);
    return check_launch("lc_gemm (f32 split-k reduce)");
  }
  if (b_nk)
    gemm_f32_simt_kernel<TM, EPI, true, COMP><<<grid, kThreads, 0, s>>>(a, b, bias, c, m, n, k, flag, 0, nullptr);
  else
    gemm_f32_simt_kernel<TM, EPI, false, COMP><<<grid, kThreads, 0, s>>>(a, b, bias, c, m, n, k, flag, 0,
                                                                         nullptr);
  return check_launch("lc_gemm (f32 simt)");
}

// Dot2-compensated SIMT GEMM (64x64 tiles: two registers per output).
int launch_simt_dot2(int epi, bool b_nk, const float *a, const float *b, const float *bias, float *c, int m,
                     int n, int k, cudaStream_t s) {
#define LC_F32_DOT2(E) \
  if (epi == E) return launch_simt_tm<4, E, true>(b_nk, a, b, bias, c, m, n, k, nullptr, s);
  LC_F32_DOT2(LC_EPI_NONE) LC_F32_DOT2(LC_EPI_GELU_ERF) LC_F32_DOT2(LC_EPI_GELU_TANH)
#undef LC_F32_DOT2
  return fail(LC_ERR_INVALID, "lc_gemm_f32_dot2: bad epilogue");
}

int launch_simt(int epi, bool b_nk, const float *a, const float *b, const float *bias, float *c,
                int m, int n, int k, const int *flag, cudaStream_t s) {
  const int64_t big_tiles = (int64_t)((m + 127) / 128) * ((n + 127) / 128);
  const bool small = big_tiles < sm_count();
#define LC_F32_SIMT(E)                                                              \
  if (epi == E)                                                                     \
    return small ? launch_simt_tm<4, E>(b_nk, a, b, bias, c, m, n, k, flag, s)      \
                 : launch_simt_tm<8, E>(b_nk, a, b, bias, c, m, n, k, flag, s);
  LC_F32_SIMT(LC_EPI_NONE) LC_F32_SIMT(LC_EPI_GELU_ERF) LC_F32_SIMT(LC_EPI_GELU_TANH)
#undef LC_F32_SIMT
  return fail(LC_ERR_INVALID, "lc_gemm: bad epilogue");
}

template <int ORDER>
int launch_split(const float *x, __nv_bfloat16 *out, int64_t rows, int64_t cols,
                 int64_t row_stride, int64_t slot_stride, int *flag, cudaStream_t s) {
  const int64_t work = rows * (cols / 4);
  const int64_t blocks = (work + kThreads - 1) / kThreads;
  const int64_t cap = 8LL * sm_count();
  const int grid = (int)(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
  split3_kernel<ORDER><<<grid, kThreads, 0, s>>>(x, out, rows, cols, row_stride, slot_stride, flag);
  return check_launch("lc_gemm (f32 split)");
}

size_t round_up(size_t v, size_t to) { return (v + to - 1) / to * to; }

}  // namespace

int gemm_path32(int b_layout, const void *a, const void *b, int64_t m, int64_t n, int64_t k) {
  const bool shape_ok = k % 4 == 0 && k >= 16 && 6 * k <= 0x7fffffff && aligned(a, 16) &&
                        aligned(b, 16) && (b_layout == LC_B_NK || n % 8 == 0);
  if (!shape_ok || m * n * k < kSplitMacs) return 0;
  return gemm_path16(b_layout, a, b, m, n, 6 * k);
}

int gemm_f32_dot2(int b_layout, int epi, const float *a, const float *b, const float *bias, float *c,
                  int m, int n, int k, cudaStream_t s) {
  return launch_simt_dot2(epi, b_layout == LC_B_NK, a, b, bias, c, m, n, k, s);
}

int gemm_f32(int out, int b_layout, int epi, const void *a_, const void *b_, const float *bias,
             void *c_, int m, int n, int k, cudaStream_t s) {
  if (out != LC_F32) return fail(LC_ERR_UNSUPPORTED, "lc_gemm: f32 operands need an f32 output");
  const float *a = static_cast<const float *>(a_);
  const float *b = static_cast<const float *>(b_);
  float *c = static_cast<float *>(c_);
  const bool b_nk = b_layout == LC_B_NK;
  const int path = gemm_path32(b_layout, a, b, m, n, k);
  if (path == 0) return launch_simt(epi, b_nk, a, b, bias, c, m, n, k, nullptr, s);

  const int64_t k6 = 6LL * k;
  const size_t a_bytes = round_up((size_t)m * k6 * 2, 256);
  const size_t b_bytes = round_up((size_t)k6 * n * 2, 256);
  void *ws = nullptr;
  if (int rc = scratch_buffer(s, kScratchSlot, a_bytes + b_bytes + 256, &ws)) return rc;
  auto *a2 = static_cast<__nv_bfloat16 *>(ws);
  auto *b2 = reinterpret_cast<__nv_bfloat16 *>(static_cast<char *>(ws) + a_bytes);
  int *flag = reinterpret_cast<int *>(static_cast<char *>(ws) + a_bytes + b_bytes);
  if (int rc = check_cuda(cudaMemsetAsync(flag, 0, sizeof(int), s), "lc_gemm: flag reset"))
    return rc;
  if (int rc = launch_split<kOrderA>(a, a2, m, k, k6, k, flag, s)) return rc;
  if (b_nk) {
    if (int rc = launch_split<kOrderB>(b, b2, n, k, k6, k, flag, s)) return rc;
  } else {
    if (int rc = launch_split<kOrderB>(b, b2, k, n, n, (int64_t)k * n, flag, s)) return rc;
  }
  if (int rc = gemm_tc_launch(true, !b_nk, LC_F32, epi, a2, b2, bias, c, m, n, (int)k6, s,
                              path == 2))
    return rc;
  // plain f32 recomputation, which returns at once unless a non-finite value was split
  return launch_simt(epi, b_nk, a, b, bias, c, m, n, k, flag, s);
}

}  // namespace lc
