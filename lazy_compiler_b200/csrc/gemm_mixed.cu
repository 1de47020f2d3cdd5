// GEMM whose operands are stored at another precision than the tensor-core
// MMA reads them at, with the fragment-store variants of the reference's
// tensor lowering:
//
//   * operand gathers round every element to the MMA type (f16 or bf16) on
//     the way into a fragment (ptx_tensor.py:315-357, `c.convert(value,
//     fragment.dtype)`, round-to-nearest-even), the product accumulates in f32;
//   * RegStore epilogues: bias[col] added in f32, then identity, erf-GELU,
//     tanh-GELU or ReLU = max(x, 0) (ptx_tensor.py:431-457; ptx_backend.py:1058);
//   * transposed stores (row_dim = 1, col_dim = 0: C[i, j] lands at c[j * M + i],
//     ptx_tensor.py:398-426) and accumulating stores (`atomic`: red.global.add
//     into an output the launcher zeroed first);
//   * the C -> A fragment repack chain Q(Q(X) Q(Y)) Q(Z) (ptx_tensor.py:459-477),
//     whose intermediate is rounded to the MMA type exactly like the repack's
//     cvt.rn.
//
// Paths: a problem of at least 2^24 multiply-adds whose shape the TMA GEMM
// takes rounds its operands once into 16-bit scratch (an HBM-bound pass of
// 6 bytes per f32 element) and runs the tcgen05 GEMM of gemm.cu on them; the
// store variants the tcgen05 epilogue does not have (ReLU, transposed,
// accumulating) then run as one f32 pass over C.  Smaller problems run one
// fused SIMT kernel that rounds, multiplies, applies the epilogue and stores.
#include <type_traits>

#include "common.cuh"
#include "epilogue.cuh"

namespace lc {
namespace {

// scratch slots of this file (gemm_f32.cu uses 0 and 1)
constexpr int kSlotA = 2, kSlotB = 3, kSlotAcc = 4, kSlotChain = 5;

__device__ __forceinline__ float load_any(const void *p, int type, int64_t i) {
  if (type == LC_F32) return static_cast<const float *>(p)[i];
  if (type == LC_F16) return __half2float(static_cast<const __half *>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
}

__device__ __forceinline__ float round_to(float v, bool bf16) {
  return bf16 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}

__device__ __forceinline__ float epilogue_rt(int epi, float v) {
  if (epi == LC_EPI_GELU_ERF) return gelu_erf(v);
  if (epi == LC_EPI_GELU_TANH) return gelu_tanh(v);
  if (epi == LC_EPI_RELU) return fmaxf(v, 0.0f);  // max.f32: max(NaN, 0) = 0, as the reference's relu
  return v;
}

__device__ __forceinline__ void store_any(void *c, int type, int64_t i, float v, bool accumulate) {
  if (type == LC_F32) {
    float *p = static_cast<float *>(c) + i;
    if (accumulate) atomicAdd(p, v);
    else *p = v;
  } else if (type == LC_F16) {
    static_cast<__half *>(c)[i] = __float2half_rn(v);
  } else {
    static_cast<__nv_bfloat16 *>(c)[i] = __float2bfloat16_rn(v);
  }
}

struct MixedArgs {
  const void *a, *b;
  const float *bias;
  void *c;
  int m, n, k;
  int a_type, b_type, c_type;
  int b_nk, bf16, epi, transpose, accumulate;
};

// One 16 x 16 output tile per 256-thread block: both operand tiles are
// rounded to the MMA type as they are staged, the f32 FMA chain runs in K
// order (the products of two 16-bit values are exact in f32).
__global__ void __launch_bounds__(256) gemm_mixed_simt_kernel(MixedArgs p) {
  __shared__ float as[16][17];
  __shared__ float bs[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int row = blockIdx.y * 16 + ty, col = blockIdx.x * 16 + tx;
  const bool bf16 = p.bf16;
  float acc = 0.f;
  for (int k0 = 0; k0 < p.k; k0 += 16) {
    const int ka = k0 + tx, kb = k0 + ty;
    as[ty][tx] = (row < p.m && ka < p.k) ? round_to(load_any(p.a, p.a_type, (int64_t)row * p.k + ka), bf16)
                                         : 0.f;
    float bv = 0.f;
    if (col < p.n && kb < p.k)
      bv = round_to(load_any(p.b, p.b_type, p.b_nk ? (int64_t)col * p.k + kb : (int64_t)kb * p.n + col),
                    bf16);
    bs[ty][tx] = bv;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) acc = fmaf(as[ty][i], bs[i][tx], acc);
    __syncthreads();
  }
  if (row < p.m && col < p.n) {
    if (p.bias) acc = __fadd_rn(acc, p.bias[col]);
    const float v = epilogue_rt(p.epi, acc);
    const int64_t at = p.transpose ? (int64_t)col * p.m + row : (int64_t)row * p.n + col;
    store_any(p.c, p.c_type, at, v, p.accumulate);
  }
}

// Rounds `count` elements of `src` (f32, f16 or bf16) to f16/bf16; eight per
// thread with 16-byte stores (count is a multiple of 8 on this path); `vec`:
// an f32 source is 16-byte aligned and read with 16-byte loads.
template <bool BF16>
__global__ void __launch_bounds__(256) quantise_kernel(const void *__restrict__ src, int src_type,
                                                       int vec, void *__restrict__ dst, int64_t count) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * 8;
  for (int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; i < count; i += stride) {
    float v[8];
    if (vec) {
      const float4 lo = ld_stream(reinterpret_cast<const float4 *>(static_cast<const float *>(src) + i));
      const float4 hi = ld_stream(reinterpret_cast<const float4 *>(static_cast<const float *>(src) + i + 4));
      v[0] = lo.x; v[1] = lo.y; v[2] = lo.z; v[3] = lo.w;
      v[4] = hi.x; v[5] = hi.y; v[6] = hi.z; v[7] = hi.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = load_any(src, src_type, i + j);
    }
    uint4 pack;
    T *e = reinterpret_cast<T *>(&pack);
#pragma unroll
    for (int j = 0; j < 8; ++j) e[j] = to_out<T>(v[j]);
    *reinterpret_cast<uint4 *>(static_cast<T *>(dst) + i) = pack;
  }
}

// c (op)= epilogue(acc + bias[col]) over an f32 m x n accumulator, stored
// row-major or transposed; 32 x 32 tiles through shared memory so that both
// the accumulator reads and the transposed writes are coalesced.
__global__ void __launch_bounds__(256) finish_kernel(const float *__restrict__ acc,
                                                     const float *__restrict__ bias, void *c,
                                                     int c_type, int m, int n, int epi,
                                                     int transpose, int accumulate) {
  __shared__ float t[32][33];
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, col = c0 + tx;
    float v = 0.f;
    if (r < m && col < n) {
      v = acc[(int64_t)r * n + col];
      if (bias) v = __fadd_rn(v, bias[col]);
      v = epilogue_rt(epi, v);
      if (!transpose) store_any(c, c_type, (int64_t)r * n + col, v, accumulate);
    }
    t[i][tx] = v;
  }
  if (!transpose) return;
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int col = c0 + i, r = r0 + tx;
    if (r < m && col < n) store_any(c, c_type, (int64_t)col * m + r, t[tx][i], accumulate);
  }
}

int quantise(const void *src, int src_type, bool bf16, int64_t count, int slot, cudaStream_t s,
             const void **out) {
  void *dst = nullptr;
  if (int rc = scratch_buffer(s, slot, (size_t)count * 2, &dst)) return rc;
  const int64_t threads = (count + 7) / 8;
  int64_t blocks = (threads + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const int vec = src_type == LC_F32 && aligned(src, 16);
  if (bf16) quantise_kernel<true><<<(unsigned)blocks, 256, 0, s>>>(src, src_type, vec, dst, count);
  else quantise_kernel<false><<<(unsigned)blocks, 256, 0, s>>>(src, src_type, vec, dst, count);
  *out = dst;
  return check_launch("lc_gemm_mixed (operand rounding)");
}

bool known_type(int t) { return t == LC_F32 || t == LC_F16 || t == LC_BF16; }

}  // namespace

int gemm_mixed(int mma_type, int a_type, int b_type, int c_type, int b_layout, int epilogue,
               int flags, const void *a, const void *b, const float *bias, void *c, int m, int n,
               int k, cudaStream_t s) {
  const bool bf16 = mma_type == LC_BF16;
  const bool transpose = flags & LC_GEMM_TRANSPOSE_C, accumulate = flags & LC_GEMM_ACCUMULATE;
  const bool round_a = a_type != mma_type, round_b = b_type != mma_type;
  // the shape test of the TMA GEMM; rounded operands live in 256-byte aligned scratch
  const int path = gemm_path16_shape(b_layout, round_a || aligned(a, 16), round_b || aligned(b, 16),
                                     m, n, k);
  if (path) {
    const void *qa = a, *qb = b;
    if (round_a)
      if (int rc = quantise(a, a_type, bf16, (int64_t)m * k, kSlotA, s, &qa)) return rc;
    if (round_b)
      if (int rc = quantise(b, b_type, bf16, (int64_t)k * n, kSlotB, s, &qb)) return rc;
    const bool b_mn = b_layout == LC_B_KN;
    if (!transpose && !accumulate && epilogue != LC_EPI_RELU)
      return gemm_tc_launch(bf16, b_mn, c_type, epilogue, qa, qb, bias, c, m, n, k, s, path == 2);
    void *accbuf = nullptr;
    if (int rc = scratch_buffer(s, kSlotAcc, (size_t)m * n * 4, &accbuf)) return rc;
    if (int rc = gemm_tc_launch(bf16, b_mn, LC_F32, LC_EPI_NONE, qa, qb, nullptr, accbuf, m, n, k, s,
                                path == 2))
      return rc;
    dim3 grid((n + 31) / 32, (m + 31) / 32);
    finish_kernel<<<grid, 256, 0, s>>>(static_cast<const float *>(accbuf), bias, c, c_type, m, n,
                                       epilogue, transpose, accumulate);
    return check_launch("lc_gemm_mixed (store)");
  }
  MixedArgs p;
  p.a = a;
  p.b = b;
  p.bias = bias;
  p.c = c;
  p.m = m;
  p.n = n;
  p.k = k;
  p.a_type = a_type;
  p.b_type = b_type;
  p.c_type = c_type;
  p.b_nk = b_layout == LC_B_NK;
  p.bf16 = bf16;
  p.epi = epilogue;
  p.transpose = transpose;
  p.accumulate = accumulate;
  dim3 grid((n + 15) / 16, (m + 15) / 16);
  gemm_mixed_simt_kernel<<<grid, 256, 0, s>>>(p);
  return check_launch("lc_gemm_mixed (simt)");
}

}  // namespace lc

extern "C" int lc_gemm_mixed(int mma_type, int a_type, int b_type, int c_type, int b_layout,
                             int epilogue, int flags, const void *a, const void *b,
                             const void *bias, void *c, int64_t m, int64_t n, int64_t k,
                             void *stream) {
  using namespace lc;
  if (mma_type != LC_F16 && mma_type != LC_BF16)
    return fail(LC_ERR_INVALID, "lc_gemm_mixed: the MMA type must be f16 or bf16, not %d", mma_type);
  if (!known_type(a_type) || !known_type(b_type) || !known_type(c_type))
    return fail(LC_ERR_INVALID, "lc_gemm_mixed: unknown storage type");
  if (b_layout != LC_B_KN && b_layout != LC_B_NK)
    return fail(LC_ERR_INVALID, "lc_gemm_mixed: unknown B layout %d", b_layout);
  if (epilogue < LC_EPI_NONE || epilogue > LC_EPI_RELU)
    return fail(LC_ERR_INVALID, "lc_gemm_mixed: unknown epilogue %d", epilogue);
  if (flags & ~(LC_GEMM_TRANSPOSE_C | LC_GEMM_ACCUMULATE))
    return fail(LC_ERR_INVALID, "lc_gemm_mixed: unknown flags 0x%x", flags);
  if ((flags & LC_GEMM_ACCUMULATE) && c_type != LC_F32)
    return fail(LC_ERR_INVALID, "lc_gemm_mixed: accumulating stores need an f32 output");
  if (m < 0 || n < 0 || k < 0) return fail(LC_ERR_INVALID, "lc_gemm_mixed: negative shape");
  if (m > 0x7fffffff || n > 0x7fffffff || k > 0x7fffffff || m * n > ((int64_t)1 << 40))
    return fail(LC_ERR_UNSUPPORTED, "lc_gemm_mixed: dimensions too large");
  if (m == 0 || n == 0) return LC_OK;
  if (!c || (k > 0 && (!a || !b))) return fail(LC_ERR_INVALID, "lc_gemm_mixed: null buffer");
  return gemm_mixed(mma_type, a_type, b_type, c_type, b_layout, epilogue, flags, a, b,
                    static_cast<const float *>(bias), c, (int)m, (int)n, (int)k, as_stream(stream));
}

extern "C" int lc_gemm_chain(int mma_type, int x_type, int y_type, int z_type, int c_type,
                             int y_layout, int z_layout, const void *x, const void *y,
                             const void *z, void *c, int64_t m, int64_t k, int64_t n1, int64_t n2,
                             void *stream) {
  using namespace lc;
  if (mma_type != LC_F16 && mma_type != LC_BF16)
    return fail(LC_ERR_INVALID, "lc_gemm_chain: the MMA type must be f16 or bf16, not %d", mma_type);
  if (!known_type(x_type) || !known_type(y_type) || !known_type(z_type) || !known_type(c_type))
    return fail(LC_ERR_INVALID, "lc_gemm_chain: unknown storage type");
  if ((y_layout != LC_B_KN && y_layout != LC_B_NK) || (z_layout != LC_B_KN && z_layout != LC_B_NK))
    return fail(LC_ERR_INVALID, "lc_gemm_chain: unknown B layout");
  if (m < 0 || k < 0 || n1 < 0 || n2 < 0) return fail(LC_ERR_INVALID, "lc_gemm_chain: negative shape");
  if (m > 0x7fffffff || k > 0x7fffffff || n1 > 0x7fffffff || n2 > 0x7fffffff ||
      m * n1 > ((int64_t)1 << 40))
    return fail(LC_ERR_UNSUPPORTED, "lc_gemm_chain: dimensions too large");
  if (m == 0 || n2 == 0) return LC_OK;
  if (!c || (n1 > 0 && !z) || (n1 > 0 && k > 0 && (!x || !y)))
    return fail(LC_ERR_INVALID, "lc_gemm_chain: null buffer");
  cudaStream_t s = as_stream(stream);
  // T = Q(X) Q(Y) in f32; the second product rounds T to the MMA type as it
  // gathers it, which is the repack's f32 -> 16-bit conversion
  void *t = nullptr;
  if (int rc = scratch_buffer(s, kSlotChain, (size_t)(m * (n1 > 0 ? n1 : 1)) * 4, &t)) return rc;
  if (n1 > 0)
    if (int rc = gemm_mixed(mma_type, x_type, y_type, LC_F32, y_layout, LC_EPI_NONE, 0, x, y, nullptr,
                            t, (int)m, (int)n1, (int)k, s))
      return rc;
  return gemm_mixed(mma_type, LC_F32, z_type, c_type, z_layout, LC_EPI_NONE, 0, t, z, nullptr, c,
                    (int)m, (int)n2, (int)n1, s);
}
