// Pointwise programs: one register program (lc_pw_program, built by the
// plan compiler from a straight-line Tile body) run per tile point.
//
// Each thread walks tile points in a grid-stride loop, decodes the point's
// coordinates and runs the program; every operation is one PTX instruction
// of the reference's scalar lowering (ptx_backend.py:406-1177), so the
// program computes what the reference's kernel computes, step for step.
// The program itself lives in the kernel's parameter space (a
// __grid_constant__ struct): every lane of a warp reads the same operation
// at the same time, a broadcast from the constant bank.
#include <cuda.h>

#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace lc {
namespace {

struct PointwiseArgs {
  lc_pw_program prog;
  void *buffers[LC_PW_MAX_BUFFERS];
  int64_t points;
};

__device__ __forceinline__ float f(uint32_t w) { return __uint_as_float(w); }
// Mask of the lanes of the calling thread's warp that exist in its CTA (all 32
// unless the CTA's thread count leaves this warp partial).
__device__ __forceinline__ unsigned int warp_lanes() {
  const unsigned int first = threadIdx.x & ~31u;
  const unsigned int n = blockDim.x - first;
  return n >= 32u ? 0xffffffffu : ((1u << n) - 1u);
}
__device__ __forceinline__ uint32_t w(float x) { return __float_as_uint(x); }

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float sin_approx(float x) {
  float y;
  asm("sin.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float cos_approx(float x) {
  float y;
  asm("cos.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float round_half(float x) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Runs operations [begin, end) of a program for one point with coordinates
// x.  `states` (STATE), `partials` (PARTIAL, SETP) and `partners` (PARTNER)
// belong to row programs; `smem` and `bl` (LDS, STS) to block programs.
__device__ __forceinline__ void exec_range(const lc_pw_program &g, void *const *buffers, int64_t *x,
                                           uint32_t *r, int begin, int end, const float *states,
                                           float *partials, const float *partners,
                                           uint32_t *smem = nullptr, const lc_bp_layout *bl = nullptr) {
  for (int pc = begin; pc < end; ++pc) {
    const uint32_t w0 = g.code[pc][0], w1 = g.code[pc][1];
    const int op = w0 & 255, dst = (w0 >> 8) & 255;
    const uint32_t A = r[(w0 >> 16) & 255], B = r[w0 >> 24], C = r[w1 & 255];
    const int aux = (int)(w1 >> 8);
    const int32_t ia = (int32_t)A, ib = (int32_t)B;
    uint32_t out = 0;
    if (op >= LC_PW_LD_F32 && op <= LC_PW_ST_S32) {
      const lc_pw_form &fm = g.forms[aux];
      int64_t at = fm.base;
      for (int d = 0; d < g.n_axes + g.n_loops; ++d) at += fm.coef[d] * x[d];
      void *base = buffers[fm.buffer];
      switch (op) {
        case LC_PW_LD_F32: out = static_cast<const uint32_t *>(base)[at]; break;
        case LC_PW_LD_F16: out = w(__half2float(static_cast<const __half *>(base)[at])); break;
        case LC_PW_LD_BF16: out = w(__bfloat162float(static_cast<const __nv_bfloat16 *>(base)[at])); break;
        case LC_PW_LD_S32: out = static_cast<const uint32_t *>(base)[at]; break;
        case LC_PW_ST_F32: static_cast<uint32_t *>(base)[at] = A; continue;
        case LC_PW_ST_F16: static_cast<__half *>(base)[at] = __float2half_rn(f(A)); continue;
        case LC_PW_ST_BF16: static_cast<__nv_bfloat16 *>(base)[at] = __float2bfloat16_rn(f(A)); continue;
        default: static_cast<uint32_t *>(base)[at] = A; continue;  // LC_PW_ST_S32
      }
      r[dst] = out;
      continue;
    }
    switch (op) {
      case LC_PW_MOV: out = A; break;
      case LC_PW_CONST: out = g.consts[aux]; break;
      case LC_PW_FADD: out = w(__fadd_rn(f(A), f(B))); break;
      case LC_PW_FSUB: out = w(__fsub_rn(f(A), f(B))); break;
      case LC_PW_FMUL: out = w(__fmul_rn(f(A), f(B))); break;
      case LC_PW_FDIV: out = w(__fdiv_rn(f(A), f(B))); break;
      case LC_PW_FFMA: out = w(__fmaf_rn(f(A), f(B), f(C))); break;
      case LC_PW_FNEG: out = A ^ 0x80000000u; break;
      case LC_PW_FABS: out = A & 0x7fffffffu; break;
      case LC_PW_FMAX: out = w(fmaxf(f(A), f(B))); break;
      case LC_PW_FMIN: out = w(fminf(f(A), f(B))); break;
      case LC_PW_FSQRT: out = w(__fsqrt_rn(f(A))); break;
      case LC_PW_FFLOOR: out = w(floorf(f(A))); break;
      case LC_PW_FCEIL: out = w(ceilf(f(A))); break;
      case LC_PW_FTRUNC: out = w(truncf(f(A))); break;
      case LC_PW_FRINT: out = w(rintf(f(A))); break;
      case LC_PW_FEX2: out = w(ex2_approx(f(A))); break;
      case LC_PW_FLG2: out = w(lg2_approx(f(A))); break;
      case LC_PW_FSIN: out = w(sin_approx(f(A))); break;
      case LC_PW_FCOS: out = w(cos_approx(f(A))); break;
      case LC_PW_FCOPYSIGN: out = (B & 0x7fffffffu) | (A & 0x80000000u); break;  // |b| with a's sign
      case LC_PW_RND_F16: out = w(round_half(f(A))); break;
      case LC_PW_RND_BF16: out = w(round_bf16(f(A))); break;
      case LC_PW_F2I: out = (uint32_t)__float2int_rz(f(A)); break;
      case LC_PW_I2F: out = w(__int2float_rn(ia)); break;
      case LC_PW_I2H: out = w(__half2float(__int2half_rn(ia))); break;
      case LC_PW_I2BF: out = w(__bfloat162float(__int2bfloat16_rn(ia))); break;
      case LC_PW_IADD: out = A + B; break;
      case LC_PW_ISUB: out = A - B; break;
      case LC_PW_IMUL: out = A * B; break;
      case LC_PW_IDIV:  // integer division by zero has no defined result; it yields 0 here
        out = ib == 0 ? 0u : (ib == -1 ? 0u - A : (uint32_t)(ia / ib));
        break;
      case LC_PW_IREM: out = (ib == 0 || ib == -1) ? (ib == 0 ? A : 0u) : (uint32_t)(ia % ib); break;
      case LC_PW_ISHL: out = B >= 32u ? 0u : A << B; break;  // shl.b32 clamps the count
      case LC_PW_ISHR: out = (uint32_t)(ia >> (B >= 32u ? 31u : B)); break;
      case LC_PW_IAND: out = A & B; break;
      case LC_PW_IOR: out = A | B; break;
      case LC_PW_IXOR: out = A ^ B; break;
      case LC_PW_INOT: out = ~A; break;
      case LC_PW_INEG: out = 0u - A; break;
      case LC_PW_IABS: out = ia < 0 ? 0u - A : A; break;
      case LC_PW_IMAX: out = (uint32_t)max(ia, ib); break;
      case LC_PW_IMIN: out = (uint32_t)min(ia, ib); break;
      case LC_PW_IPOPC: out = (uint32_t)__popc(A); break;
      case LC_PW_FEQ: out = f(A) == f(B); break;
      case LC_PW_FNE: out = !(f(A) == f(B)); break;  // unordered: true when either is NaN
      case LC_PW_FLT: out = f(A) < f(B); break;
      case LC_PW_FLE: out = f(A) <= f(B); break;
      case LC_PW_FGT: out = f(A) > f(B); break;
      case LC_PW_FGE: out = f(A) >= f(B); break;
      case LC_PW_IEQ: out = ia == ib; break;
      case LC_PW_INE: out = ia != ib; break;
      case LC_PW_ILT: out = ia < ib; break;
      case LC_PW_ILE: out = ia <= ib; break;
      case LC_PW_IGT: out = ia > ib; break;
      case LC_PW_IGE: out = ia >= ib; break;
      case LC_PW_PAND: out = (A != 0u) & (B != 0u); break;
      case LC_PW_POR: out = (A != 0u) | (B != 0u); break;
      case LC_PW_SEL: out = A != 0u ? B : C; break;
      case LC_PW_COORD: out = (uint32_t)x[aux]; break;
      case LC_PW_LDX_F32: case LC_PW_LDX_F16: case LC_PW_LDX_BF16: case LC_PW_LDX_S32: {
        const int64_t size = g.sizes[aux];
        int64_t at = (int64_t)ia;
        at = at < 0 ? 0 : (at >= size ? size - 1 : at);  // clamped: a load never leaves its buffer
        const void *base = buffers[aux];
        if (op == LC_PW_LDX_F16) out = w(__half2float(static_cast<const __half *>(base)[at]));
        else if (op == LC_PW_LDX_BF16) out = w(__bfloat162float(static_cast<const __nv_bfloat16 *>(base)[at]));
        else out = static_cast<const uint32_t *>(base)[at];
        break;
      }
      case LC_PW_STX_F32: case LC_PW_STX_F16: case LC_PW_STX_BF16: case LC_PW_STX_S32:
      case LC_PW_STX_ADD_F32: {
        const int64_t at = (int64_t)ia;
        if (C != 0u && at >= 0 && at < g.sizes[aux]) {
          void *base = buffers[aux];
          if (op == LC_PW_STX_F16) static_cast<__half *>(base)[at] = __float2half_rn(f(B));
          else if (op == LC_PW_STX_BF16) static_cast<__nv_bfloat16 *>(base)[at] = __float2bfloat16_rn(f(B));
          else if (op == LC_PW_STX_ADD_F32) atomicAdd(static_cast<float *>(base) + at, f(B));
          else static_cast<uint32_t *>(base)[at] = B;
        }
        continue;
      }
      case LC_PW_SHFL_XOR: {
        // the lanes of this warp that exist: a block program's CTA may be one
        // partial warp (its butterfly is then confined to that power-of-two group)
        const unsigned int mask = warp_lanes();
        __syncwarp(mask);
        out = __shfl_xor_sync(mask, A, aux);
        break;
      }
      case LC_PW_PACK_F16X2: {
        __half2 h = __floats2half2_rn(f(A), f(B));
        out = *reinterpret_cast<uint32_t *>(&h);
        break;
      }
      case LC_PW_PACK_BF16X2: {
        __nv_bfloat162 h = __floats2bfloat162_rn(f(A), f(B));
        out = *reinterpret_cast<uint32_t *>(&h);
        break;
      }
      case LC_PW_MMA_F16: case LC_PW_MMA_BF16: {
        const int ra = (w0 >> 16) & 255, rb = w0 >> 24, rc = w1 & 255;
        uint32_t d0, d1, d2, d3;
        __syncwarp();
        if (op == LC_PW_MMA_F16)
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
              " {%8, %9}, {%10, %11, %12, %13};"
              : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
              : "r"(r[ra]), "r"(r[ra + 1]), "r"(r[ra + 2]), "r"(r[ra + 3]), "r"(r[rb]), "r"(r[rb + 1]),
                "r"(r[rc]), "r"(r[rc + 1]), "r"(r[rc + 2]), "r"(r[rc + 3]));
        else
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
              " {%8, %9}, {%10, %11, %12, %13};"
              : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3)
              : "r"(r[ra]), "r"(r[ra + 1]), "r"(r[ra + 2]), "r"(r[ra + 3]), "r"(r[rb]), "r"(r[rb + 1]),
                "r"(r[rc]), "r"(r[rc + 1]), "r"(r[rc + 2]), "r"(r[rc + 3]));
        r[dst] = d0;
        r[dst + 1] = d1;
        r[dst + 2] = d2;
        r[dst + 3] = d3;
        continue;
      }
      case LC_PW_FREM: {  // floor remainder (fmodf is exact; one rounded add adjusts the sign)
        const float xv = f(A), yv = f(B);
        float rv = __int_as_float(0x7fc00000);
        if (isfinite(xv) && !isnan(yv) && yv != 0.0f) {
          rv = fmodf(xv, yv);
          if (rv != 0.0f && ((xv < 0.0f) != (yv < 0.0f))) rv = __fadd_rn(rv, yv);
          if (rv == 0.0f) rv = copysignf(0.0f, yv);
        }
        out = w(rv);
        break;
      }
      case LC_PW_LOOPB: {  // enter a loop at depth aux & 15: count from 0, skip an empty body
        const int d = g.n_axes + (aux & 15);
        const int64_t limit = min((int64_t)ia, g.extents[d]);  // never past the validated extent
        x[d] = 0;
        if (limit <= 0) pc = aux >> 4;
        continue;
      }
      case LC_PW_LOOPE: {  // next iteration, back to the matching LOOPB
        const int d = g.n_axes + (aux & 15);
        const int64_t limit = min((int64_t)ia, g.extents[d]);
        if (++x[d] < limit) pc = aux >> 4;
        continue;
      }
      case LC_PW_BRA: pc = aux - 1; continue;  // forward only (checked on the host)
      case LC_PW_BRZ:
        if (A == 0u) pc = aux - 1;
        continue;
      case LC_PW_SLB: {  // strided loop: counter = start (a), run while below the limit (b)
        const int d = g.n_axes + (aux & 15);
        const int64_t limit = min((int64_t)ib, g.extents[d]);  // never past the validated extent
        x[d] = (int64_t)ia;
        if (x[d] < 0 || x[d] >= limit) pc = aux >> 4;
        continue;
      }
      case LC_PW_SLE: {  // counter += step (a, at least 1); repeat while below the limit (b)
        const int d = g.n_axes + (aux & 15);
        const int64_t limit = min((int64_t)ib, g.extents[d]);
        x[d] += ia < 1 ? 1 : ia;
        if (x[d] < limit) pc = aux >> 4;
        continue;
      }
      case LC_PW_LDS: {
        const int64_t size = bl->smem_size[aux];
        int64_t at = (int64_t)ia;
        at = at < 0 ? 0 : (at >= size ? size - 1 : at);
        out = smem[bl->smem_offset[aux] + at];
        break;
      }
      case LC_PW_STS: {
        const int64_t at = (int64_t)ia;
        if (at >= 0 && at < bl->smem_size[aux]) smem[bl->smem_offset[aux] + at] = B;
        continue;
      }
      case LC_PW_BAR: __syncthreads(); continue;
      case LC_PW_WSYNC: __syncwarp(warp_lanes()); continue;
      case LC_PW_TID: out = threadIdx.x; break;
      case LC_PW_STATE: out = w(states[aux]); break;
      case LC_PW_PARTIAL: out = w(partials[aux]); break;
      case LC_PW_PARTNER: out = w(partners[aux]); break;
      case LC_PW_SETP: partials[aux] = f(A); continue;
      default: out = 0u; break;  // the host admits no other opcode
    }
    r[dst] = out;
  }
}

__global__ void __launch_bounds__(256) pointwise_kernel(const __grid_constant__ PointwiseArgs p) {
  uint32_t r[LC_PW_MAX_REGS];
  for (int i = 0; i < LC_PW_MAX_REGS; ++i) r[i] = 0u;
  const lc_pw_program &g = p.prog;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gid < p.points; gid += stride) {
    int64_t x[LC_PW_MAX_AXES] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t rest = gid;
    for (int d = g.n_axes - 1; d >= 0; --d) {
      x[d] = rest % g.extents[d];
      rest /= g.extents[d];
    }
    exec_range(g, p.buffers, x, r, 0, g.n_code, nullptr, nullptr, nullptr);
  }
}

struct RowProgArgs {
  lc_pw_program prog;
  lc_rp_layout lay;
  void *buffers[LC_PW_MAX_BUFFERS];
};

// One CTA per row (grid-stride over rows).  Each pass: seed the partials,
// stride the threads over the row's columns, combine the partials with the
// program's own combine steps — a lane butterfly in each warp, then the
// warps' results folded in warp order by one thread — and broadcast the
// states.  Every barrier is reached by every thread of the CTA.
__global__ void __launch_bounds__(1024) rowprog_kernel(const __grid_constant__ RowProgArgs p) {
  __shared__ float warp_part[32][LC_RP_MAX_STATES];
  __shared__ float combined[LC_RP_MAX_STATES];
  uint32_t r[LC_PW_MAX_REGS];
  for (int i = 0; i < LC_PW_MAX_REGS; ++i) r[i] = 0u;
  float states[LC_RP_MAX_STATES], partials[LC_RP_MAX_STATES], partners[LC_RP_MAX_STATES];
  for (int k = 0; k < LC_RP_MAX_STATES; ++k) states[k] = partials[k] = partners[k] = 0.0f;
  const lc_pw_program &g = p.prog;
  const lc_rp_layout &lay = p.lay;
  const int R = g.n_axes - 1;   // row coordinates, then the column
  int64_t rows = 1;
  for (int d = 0; d < R; ++d) rows *= g.extents[d];
  const int64_t cols = g.extents[R];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    int64_t xr[LC_PW_MAX_AXES] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int64_t rest = row, d = R - 1; d >= 0; --d) {
      xr[d] = rest % g.extents[d];
      rest /= g.extents[d];
    }
    for (int pass = 0; pass < lay.n_passes; ++pass) {
      bool has_states = false;
      for (int k = 0; k < lay.n_states; ++k)
        if (lay.state_pass[k] == pass) {
          partials[k] = __uint_as_float(lay.state_init[k]);
          has_states = true;
        }
      for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        int64_t x[LC_PW_MAX_AXES];
        for (int d = 0; d < LC_PW_MAX_AXES; ++d) x[d] = xr[d];
        x[R] = c;
        exec_range(g, p.buffers, x, r, lay.begin[pass], lay.end[pass], states, partials, partners);
      }
      if (!has_states) continue;  // uniform: the layout is the same for every thread
      for (int o = 16; o > 0; o >>= 1) {
        for (int k = 0; k < lay.n_states; ++k)
          if (lay.state_pass[k] == pass) partners[k] = __shfl_xor_sync(0xffffffffu, partials[k], o);
        exec_range(g, p.buffers, xr, r, lay.warp_begin[pass], lay.warp_end[pass], states, partials, partners);
      }
      if (lane == 0)
        for (int k = 0; k < lay.n_states; ++k)
          if (lay.state_pass[k] == pass) warp_part[warp][k] = partials[k];
      __syncthreads();
      if (threadIdx.x == 0) {
        // the reference's tree: at each level warp i takes warp i + d, d halving
        for (int d = nwarps >> 1; d > 0; d >>= 1)
          for (int i = 0; i < d; ++i) {
            for (int k = 0; k < lay.n_states; ++k)
              if (lay.state_pass[k] == pass) {
                partials[k] = warp_part[i][k];
                partners[k] = warp_part[i + d][k];
              }
            exec_range(g, p.buffers, xr, r, lay.tree_begin[pass], lay.tree_end[pass], states, partials, partners);
            for (int k = 0; k < lay.n_states; ++k)
              if (lay.state_pass[k] == pass) warp_part[i][k] = partials[k];
          }
        for (int k = 0; k < lay.n_states; ++k)
          if (lay.state_pass[k] == pass) combined[k] = warp_part[0][k];
      }
      __syncthreads();
      for (int k = 0; k < lay.n_states; ++k)
        if (lay.state_pass[k] == pass) states[k] = combined[k];
      __syncthreads();
    }
    if (threadIdx.x == 0)
      exec_range(g, p.buffers, xr, r, lay.final_begin, lay.final_end, states, partials, partners);
  }
}

struct BlockProgArgs {
  lc_pw_program prog;
  lc_bp_layout lay;
  void *buffers[LC_PW_MAX_BUFFERS];
  int64_t blocks;
};

// One CTA per block of the Tile (grid-stride over blocks): every thread
// decodes its block and thread coordinates and runs the whole program;
// the program's own barriers order its shared memory.
__global__ void __launch_bounds__(1024) blockprog_kernel(const __grid_constant__ BlockProgArgs p) {
  extern __shared__ uint32_t bp_smem[];
  uint32_t r[LC_PW_MAX_REGS];
  for (int i = 0; i < LC_PW_MAX_REGS; ++i) r[i] = 0u;
  const lc_pw_program &g = p.prog;
  const int nb = p.lay.n_block_axes;
  for (int64_t blk = blockIdx.x; blk < p.blocks; blk += gridDim.x) {
    int64_t x[LC_PW_MAX_AXES] = {0, 0, 0, 0, 0, 0, 0, 0};
    int64_t rest = threadIdx.x;
    for (int d = g.n_axes - 1; d >= nb; --d) {
      x[d] = rest % g.extents[d];
      rest /= g.extents[d];
    }
    rest = blk;
    for (int d = nb - 1; d >= 0; --d) {
      x[d] = rest % g.extents[d];
      rest /= g.extents[d];
    }
    exec_range(g, p.buffers, x, r, 0, g.n_code, nullptr, nullptr, nullptr, bp_smem, &p.lay);
    __syncthreads();  // the next block reuses the shared arrays
  }
}

bool form_in_range(const lc_pw_program &g, const lc_pw_form &fm) {
  int64_t lo = fm.base, hi = fm.base;
  for (int d = 0; d < g.n_axes + g.n_loops; ++d) {
    const int64_t span = fm.coef[d] * (g.extents[d] - 1);
    if (span < 0) lo += span;
    else hi += span;
  }
  return lo >= 0 && hi < g.sizes[fm.buffer];
}

int storage_of(int op) {
  switch (op) {
    case LC_PW_LD_F32: case LC_PW_ST_F32: return LC_F32;
    case LC_PW_LD_F16: case LC_PW_ST_F16: return LC_F16;
    case LC_PW_LD_BF16: case LC_PW_ST_BF16: return LC_BF16;
    default: return LC_S32;
  }
}

}  // namespace
}  // namespace lc

namespace lc {
namespace {
// Checks a program before any launch; returns LC_OK or the failure, and the point count.
constexpr int kPointwise = 0, kRowProgram = 1, kBlockProgram = 2;

bool block_only(int op) { return op >= LC_PW_BRA && op <= LC_PW_TID; }

// A block program's barriers, warp syncs and shuffles must be reached by
// every thread: none may sit inside a branch region, and every loop around
// one must start and step by registers written exactly once, by CONST.
int check_uniform_sync(const char *name, const lc_pw_program &g) {
  int writes[LC_PW_MAX_REGS] = {0};
  bool by_const[LC_PW_MAX_REGS] = {false};
  for (int pc = 0; pc < g.n_code; ++pc) {
    const int op = g.code[pc][0] & 255, dst = (g.code[pc][0] >> 8) & 255;
    const bool writes_dst = !(op == LC_PW_BRA || op == LC_PW_BRZ || op == LC_PW_SLB || op == LC_PW_SLE ||
                              op == LC_PW_STS || op == LC_PW_BAR || op == LC_PW_WSYNC || op == LC_PW_LOOPB ||
                              op == LC_PW_LOOPE || op == LC_PW_SETP || (op >= LC_PW_ST_F32 && op <= LC_PW_ST_S32) ||
                              (op >= LC_PW_STX_F32 && op <= LC_PW_STX_ADD_F32));
    if (!writes_dst) continue;
    const int n = (op == LC_PW_MMA_F16 || op == LC_PW_MMA_BF16) ? 4 : 1;
    for (int k = 0; k < n; ++k) {
      ++writes[dst + k];
      by_const[dst + k] = op == LC_PW_CONST;
    }
  }
  for (int pc = 0; pc < g.n_code; ++pc) {
    const int op = g.code[pc][0] & 255;
    if (!(op == LC_PW_BAR || op == LC_PW_WSYNC || op == LC_PW_SHFL_XOR)) continue;
    for (int q = 0; q < pc; ++q) {
      const int oq = g.code[q][0] & 255, aq = (int)(g.code[q][1] >> 8);
      if ((oq == LC_PW_BRA || oq == LC_PW_BRZ) && aq > pc)
        return fail(LC_ERR_INVALID, "%s: barrier or shuffle at %d inside the branch at %d", name, pc, q);
      if (oq == LC_PW_SLB && (aq >> 4) > pc) {  // a loop around pc
        const int start = (g.code[q][0] >> 16) & 255, limit = g.code[q][0] >> 24;
        const int end = aq >> 4, step = (g.code[end][0] >> 16) & 255, limit2 = g.code[end][0] >> 24;
        const auto once = [&](int reg) { return writes[reg] == 1 && by_const[reg]; };
        if (!once(start) || !once(step) || !once(limit) || !once(limit2))
          return fail(LC_ERR_INVALID, "%s: barrier or shuffle at %d inside a loop with a per-thread range", name,
                      pc);
      }
      if (oq == LC_PW_LOOPB && (aq >> 4) > pc)
        return fail(LC_ERR_INVALID, "%s: barrier or shuffle at %d inside a counted loop", name, pc);
    }
  }
  return LC_OK;
}

int validate_program(const char *name, const lc_pw_program *program, void *const *buffers, int mode,
                     int64_t *points_out, const lc_bp_layout *bl = nullptr) {
  const bool row_program = mode == kRowProgram;
  if (!program || !buffers) return fail(LC_ERR_INVALID, "%s: null program or buffers", name);
  const lc_pw_program &g = *program;
  if (g.n_code < 0 || g.n_code > LC_PW_MAX_CODE || g.n_consts < 0 || g.n_consts > LC_PW_MAX_CONST ||
      g.n_forms < 0 || g.n_forms > LC_PW_MAX_FORMS || g.n_buffers < 1 || g.n_buffers > LC_PW_MAX_BUFFERS ||
      g.n_axes < 1 || g.n_axes > LC_PW_MAX_AXES || g.n_regs < 1 || g.n_regs > LC_PW_MAX_REGS ||
      g.n_loops < 0 || g.n_axes + g.n_loops > LC_PW_MAX_AXES || (row_program && g.n_loops != 0))
    return fail(LC_ERR_INVALID, "%s: program counts out of range", name);
  int64_t points = 1;
  for (int d = 0; d < g.n_axes; ++d) {
    if (g.extents[d] < 1 || g.extents[d] > ((int64_t)1 << 40))
      return fail(LC_ERR_INVALID, "%s: bad extent", name);
    points *= g.extents[d];
    if (points > ((int64_t)1 << 40)) return fail(LC_ERR_INVALID, "%s: tile too large", name);
  }
  for (int d = g.n_axes; d < g.n_axes + g.n_loops; ++d)
    if (g.extents[d] < 0 || g.extents[d] > 0x7fffffff) return fail(LC_ERR_INVALID, "%s: bad loop extent", name);
  for (int i = 0; i < g.n_buffers; ++i)
    if (!buffers[i] || g.sizes[i] < 1) return fail(LC_ERR_INVALID, "%s: buffer slot %d", name, i);
  for (int i = 0; i < g.n_forms; ++i) {
    const lc_pw_form &fm = g.forms[i];
    bool sane = fm.base >= -((int64_t)1 << 50) && fm.base <= ((int64_t)1 << 50);
    for (int d = 0; d < g.n_axes + g.n_loops; ++d)
      sane = sane && fm.coef[d] >= -((int64_t)1 << 40) && fm.coef[d] <= ((int64_t)1 << 40);
    if (!sane || fm.buffer < 0 || fm.buffer >= g.n_buffers || !form_in_range(g, fm))
      return fail(LC_ERR_INVALID, "%s: form %d leaves its buffer", name, i);
  }
  bool lockstep = false;
  for (int pc = 0; pc < g.n_code; ++pc) {
    const uint32_t w0 = g.code[pc][0], w1 = g.code[pc][1];
    const int op = w0 & 255;
    const uint32_t dst = (w0 >> 8) & 255, a = (w0 >> 16) & 255, b = w0 >> 24, c = w1 & 255;
    const int aux = (int)(w1 >> 8);
    if (op >= LC_PW_NUM_OPS) return fail(LC_ERR_INVALID, "%s: bad opcode at %d", name, pc);
    if ((int)dst >= g.n_regs || (int)a >= g.n_regs || (int)b >= g.n_regs || (int)c >= g.n_regs)
      return fail(LC_ERR_INVALID, "%s: register out of range at %d", name, pc);
    if (op == LC_PW_CONST && aux >= g.n_consts)
      return fail(LC_ERR_INVALID, "%s: constant out of range at %d", name, pc);
    if (op == LC_PW_COORD && aux >= g.n_axes + g.n_loops)
      return fail(LC_ERR_INVALID, "%s: coordinate out of range at %d", name, pc);
    if (op >= LC_PW_LDX_F32 && op <= LC_PW_STX_ADD_F32 && aux >= g.n_buffers)
      return fail(LC_ERR_INVALID, "%s: buffer slot out of range at %d", name, pc);
    if (op == LC_PW_SHFL_XOR && (aux < 1 || aux > 31))
      return fail(LC_ERR_INVALID, "%s: shuffle distance out of range at %d", name, pc);
    if ((op == LC_PW_MMA_F16 || op == LC_PW_MMA_BF16) &&
        ((int)dst + 3 >= g.n_regs || (int)a + 3 >= g.n_regs || (int)b + 1 >= g.n_regs || (int)c + 3 >= g.n_regs))
      return fail(LC_ERR_INVALID, "%s: MMA register tuple out of range at %d", name, pc);
    if (op == LC_PW_SHFL_XOR || op == LC_PW_MMA_F16 || op == LC_PW_MMA_BF16) lockstep = true;
    if (block_only(op) && mode != kBlockProgram)
      return fail(LC_ERR_INVALID, "%s: block-program operation outside a block program at %d", name, pc);
    if ((op == LC_PW_BRA || op == LC_PW_BRZ) && (aux <= pc || aux > g.n_code))
      return fail(LC_ERR_INVALID, "%s: branch at %d is not forward", name, pc);
    if ((op == LC_PW_LDS || op == LC_PW_STS) && (!bl || aux >= bl->n_smem))
      return fail(LC_ERR_INVALID, "%s: shared array out of range at %d", name, pc);
    if (op == LC_PW_SLB || op == LC_PW_SLE) {
      const int slot = aux & 15, other = aux >> 4;
      const bool begin = op == LC_PW_SLB;
      if (slot >= g.n_loops || other < 0 || other >= g.n_code || (begin ? other <= pc : other >= pc))
        return fail(LC_ERR_INVALID, "%s: malformed loop at %d", name, pc);
      const uint32_t m0 = g.code[other][0], m1 = g.code[other][1];
      if ((int)(m0 & 255) != (begin ? LC_PW_SLE : LC_PW_SLB) || (int)((m1 >> 8) & 15) != slot ||
          (int)(m1 >> 12) != pc)
        return fail(LC_ERR_INVALID, "%s: unmatched loop at %d", name, pc);
    }
    if (op == LC_PW_LOOPB || op == LC_PW_LOOPE) {
      // a well-formed pair: LOOPB at pc names its LOOPE, which names it back, on the same loop
      const int slot = aux & 15, other = aux >> 4;
      const bool begin = op == LC_PW_LOOPB;
      if (slot >= g.n_loops || other < 0 || other >= g.n_code || (begin ? other <= pc : other >= pc))
        return fail(LC_ERR_INVALID, "%s: malformed loop at %d", name, pc);
      const uint32_t m0 = g.code[other][0], m1 = g.code[other][1];
      if ((int)(m0 & 255) != (begin ? LC_PW_LOOPE : LC_PW_LOOPB) || (int)((m1 >> 8) & 15) != slot ||
          (int)(m1 >> 12) != pc)
        return fail(LC_ERR_INVALID, "%s: unmatched loop at %d", name, pc);
    }
    if ((op == LC_PW_STATE || op == LC_PW_PARTIAL || op == LC_PW_PARTNER || op == LC_PW_SETP) &&
        (!row_program || aux >= LC_RP_MAX_STATES))
      return fail(LC_ERR_INVALID, "%s: state operation outside a row program at %d", name, pc);
    if (op >= LC_PW_LD_F32 && op <= LC_PW_ST_S32 &&
        (aux >= g.n_forms || g.forms[aux].dtype != storage_of(op)))
      return fail(LC_ERR_INVALID, "%s: form or storage type mismatch at %d", name, pc);
  }
  if (row_program && (lockstep || g.n_axes < 2))
    return fail(LC_ERR_INVALID, "%s: a row program runs over (row, column) without warp operations", name);
  if (mode == kBlockProgram) {
    if (int rc = check_uniform_sync(name, g)) return rc;
    *points_out = points;
    return LC_OK;
  }
  if (lockstep && points % 32 != 0)
    return fail(LC_ERR_INVALID, "%s: a program that shuffles or multiplies needs whole warps of points", name);
  *points_out = points;
  return LC_OK;
}
}  // namespace
}  // namespace lc

extern "C" int lc_pointwise(const lc_pw_program *program, void *const *buffers, void *stream) {
  using namespace lc;
  int64_t points = 0;
  if (int rc = validate_program("lc_pointwise", program, buffers, kPointwise, &points)) return rc;
  const lc_pw_program &g = *program;
  PointwiseArgs args;
  args.prog = g;
  for (int i = 0; i < LC_PW_MAX_BUFFERS; ++i) args.buffers[i] = i < g.n_buffers ? buffers[i] : nullptr;
  args.points = points;
  int64_t blocks = (points + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  pointwise_kernel<<<(unsigned)blocks, 256, 0, as_stream(stream)>>>(args);
  return check_launch("lc_pointwise");
}

namespace lc {
namespace {
// Validates a row program and its layout; returns the row count.
int prepare_rowprog(const char *name, const lc_pw_program *program, const lc_rp_layout *layout,
                    void *const *buffers, int64_t *rows_out) {
  int64_t points = 0;
  if (int rc = validate_program(name, program, buffers, kRowProgram, &points)) return rc;
  if (!layout) return fail(LC_ERR_INVALID, "%s: null layout", name);
  const lc_rp_layout &lay = *layout;
  const int n_code = program->n_code;
  if (lay.n_passes < 0 || lay.n_passes > LC_RP_MAX_PASSES || lay.n_states < 0 || lay.n_states > LC_RP_MAX_STATES)
    return fail(LC_ERR_INVALID, "%s: layout counts out of range", name);
  auto range_ok = [&](int b, int e) { return 0 <= b && b <= e && e <= n_code; };
  for (int i = 0; i < lay.n_passes; ++i)
    if (!range_ok(lay.begin[i], lay.end[i]) || !range_ok(lay.warp_begin[i], lay.warp_end[i]) ||
        !range_ok(lay.tree_begin[i], lay.tree_end[i]))
      return fail(LC_ERR_INVALID, "%s: pass %d range", name, i);
  if (!range_ok(lay.final_begin, lay.final_end)) return fail(LC_ERR_INVALID, "%s: final range", name);
  for (int k = 0; k < lay.n_states; ++k)
    if (lay.state_pass[k] < 0 || lay.state_pass[k] >= lay.n_passes)
      return fail(LC_ERR_INVALID, "%s: state %d", name, k);
  if (lay.threads < 32 || lay.threads > 1024 || lay.threads % 32 || ((lay.threads / 32) & (lay.threads / 32 - 1)))
    return fail(LC_ERR_INVALID, "%s: %d threads is not 32 times a power of two up to 1024", name, lay.threads);
  for (int pc = 0; pc < n_code; ++pc) {
    const int op = program->code[pc][0] & 255, aux = (int)(program->code[pc][1] >> 8);
    if ((op == LC_PW_STATE || op == LC_PW_PARTIAL || op == LC_PW_PARTNER || op == LC_PW_SETP) && aux >= lay.n_states)
      return fail(LC_ERR_INVALID, "%s: state index out of range at %d", name, pc);
  }
  int64_t rows = 1;
  for (int d = 0; d + 1 < program->n_axes; ++d) rows *= program->extents[d];
  *rows_out = rows;
  return LC_OK;
}
}  // namespace
}  // namespace lc

extern "C" int lc_rowprog(const lc_pw_program *program, const lc_rp_layout *layout, void *const *buffers,
                          void *stream) {
  using namespace lc;
  int64_t rows = 0;
  if (int rc = prepare_rowprog("lc_rowprog", program, layout, buffers, &rows)) return rc;
  RowProgArgs args;
  args.prog = *program;
  args.lay = *layout;
  for (int i = 0; i < LC_PW_MAX_BUFFERS; ++i) args.buffers[i] = i < program->n_buffers ? buffers[i] : nullptr;
  int64_t blocks = rows;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  rowprog_kernel<<<(unsigned)blocks, (unsigned)layout->threads, 0, as_stream(stream)>>>(args);
  return check_launch("lc_rowprog");
}

namespace lc {
namespace {
// Validates a block program and fills the launch: the kernel arguments, the
// dynamic shared memory and the grid.
int prepare_blockprog(const char *name, const lc_pw_program *program, const lc_bp_layout *layout,
                      void *const *buffers, BlockProgArgs *args, size_t *smem_bytes, int64_t *grid) {
  if (!layout) return fail(LC_ERR_INVALID, "%s: null layout", name);
  const lc_bp_layout &lay = *layout;
  if (lay.n_smem < 0 || lay.n_smem > LC_BP_MAX_SMEM) return fail(LC_ERR_INVALID, "%s: shared arrays", name);
  int64_t words = 0;
  for (int i = 0; i < lay.n_smem; ++i) {
    if (lay.smem_size[i] < 1 || lay.smem_offset[i] < 0 ||
        (int64_t)lay.smem_offset[i] + lay.smem_size[i] > (int64_t)(200 * 1024 / 4))
      return fail(LC_ERR_INVALID, "%s: shared array %d", name, i);
    const int64_t top = (int64_t)lay.smem_offset[i] + lay.smem_size[i];
    if (top > words) words = top;
  }
  int64_t points = 0;
  if (int rc = validate_program(name, program, buffers, kBlockProgram, &points, &lay)) return rc;
  const lc_pw_program &g = *program;
  if (lay.threads < 1 || lay.threads > 1024 || lay.n_block_axes < 0 || lay.n_block_axes >= g.n_axes)
    return fail(LC_ERR_INVALID, "%s: thread block", name);
  int64_t threads = 1, blocks = 1;
  for (int d = 0; d < g.n_axes; ++d) (d < lay.n_block_axes ? blocks : threads) *= g.extents[d];
  if (threads != lay.threads)
    return fail(LC_ERR_INVALID, "%s: thread axes do not make %d threads", name, lay.threads);
  args->prog = g;
  args->lay = lay;
  for (int i = 0; i < LC_PW_MAX_BUFFERS; ++i) args->buffers[i] = i < g.n_buffers ? buffers[i] : nullptr;
  args->blocks = blocks;
  *smem_bytes = (size_t)words * 4;
  const int64_t cap = (int64_t)sm_count() * 8;
  *grid = blocks > cap ? cap : blocks;
  return LC_OK;
}

// Modules of natively compiled block programs, loaded once per device and image.
// A loaded native program: the lookup compares the whole image and kernel
// name, the hash only narrows the search.
struct JitModule {
  uint64_t key;
  int device;
  std::vector<uint8_t> image;
  std::string kernel;
  CUfunction function;
};
std::mutex jit_mutex;
std::vector<JitModule> jit_modules;

template <typename T>
T driver_entry(const char *symbol) {
  void *ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(symbol, &ptr, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<T>(ptr);
}

int jit_function(const void *image, size_t size, const char *kernel, CUfunction *out) {
  uint64_t key = 1469598103934665603ull;  // FNV-1a over the image
  for (size_t i = 0; i < size; ++i) key = (key ^ static_cast<const uint8_t *>(image)[i]) * 1099511628211ull;
  key ^= size;
  for (const char *c = kernel; *c; ++c) key = (key ^ (uint8_t)*c) * 1099511628211ull;
  int dev = 0;
  if (int rc = check_cuda(cudaGetDevice(&dev), "native program: device")) return rc;
  std::lock_guard<std::mutex> guard(jit_mutex);
  for (const JitModule &m : jit_modules)
    if (m.key == key && m.device == dev && m.image.size() == size && m.kernel == kernel &&
        std::memcmp(m.image.data(), image, size) == 0) {
      *out = m.function;
      return LC_OK;
    }
  using LoadFn = CUresult (*)(CUmodule *, const void *);
  using GetFn = CUresult (*)(CUfunction *, CUmodule, const char *);
  using AttrFn = CUresult (*)(CUfunction, CUfunction_attribute, int);
  using UnloadFn = CUresult (*)(CUmodule);
  auto load = driver_entry<LoadFn>("cuModuleLoadData");
  auto get = driver_entry<GetFn>("cuModuleGetFunction");
  auto attr = driver_entry<AttrFn>("cuFuncSetAttribute");
  auto unload = driver_entry<UnloadFn>("cuModuleUnload");
  if (!load || !get || !attr || !unload)
    return fail(LC_ERR_CUDA, "lc_jit_blockprog: driver entry points unavailable");
  cudaFree(nullptr);  // the primary context is current for this thread
  CUmodule module = nullptr;
  CUfunction function = nullptr;
  if (load(&module, image) != CUDA_SUCCESS) return fail(LC_ERR_CUDA, "lc_jit_blockprog: module load failed");
  if (get(&function, module, kernel) != CUDA_SUCCESS) {
    unload(module);
    return fail(LC_ERR_CUDA, "native program: kernel %s not in the module", kernel);
  }
  if (attr(function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, 200 * 1024) != CUDA_SUCCESS) {
    unload(module);
    return fail(LC_ERR_CUDA, "lc_jit_blockprog: shared memory attribute");
  }
  const uint8_t *bytes = static_cast<const uint8_t *>(image);
  jit_modules.push_back({key, dev, std::vector<uint8_t>(bytes, bytes + size), std::string(kernel), function});
  *out = function;
  return LC_OK;
}
}  // namespace
}  // namespace lc

extern "C" int lc_blockprog(const lc_pw_program *program, const lc_bp_layout *layout, void *const *buffers,
                            void *stream) {
  using namespace lc;
  BlockProgArgs args;
  size_t smem_bytes = 0;
  int64_t grid = 0;
  if (int rc = prepare_blockprog("lc_blockprog", program, layout, buffers, &args, &smem_bytes, &grid)) return rc;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (int rc = check_cuda(cudaFuncSetAttribute(blockprog_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 200 * 1024),
                            "lc_blockprog smem attribute"))
      return rc;
    configured[dev] = true;
  }
  blockprog_kernel<<<(unsigned)grid, (unsigned)args.lay.threads, smem_bytes, as_stream(stream)>>>(args);
  return check_launch("lc_blockprog");
}

extern "C" int lc_jit_blockprog(const void *image, size_t image_size, const lc_pw_program *program,
                                const lc_bp_layout *layout, void *const *buffers, void *stream) {
  using namespace lc;
  if (!image || image_size < 16) return fail(LC_ERR_INVALID, "lc_jit_blockprog: no module image");
  BlockProgArgs args;
  size_t smem_bytes = 0;
  int64_t grid = 0;
  if (int rc = prepare_blockprog("lc_jit_blockprog", program, layout, buffers, &args, &smem_bytes, &grid))
    return rc;
  CUfunction function = nullptr;
  if (int rc = jit_function(image, image_size, "lc_jit_block", &function)) return rc;
  using LaunchFn = CUresult (*)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                                CUstream, void **, void **);
  static LaunchFn launch = driver_entry<LaunchFn>("cuLaunchKernel");
  if (!launch) return fail(LC_ERR_CUDA, "lc_jit_blockprog: cuLaunchKernel unavailable");
  struct {
    void *buffers[LC_PW_MAX_BUFFERS];
    long long blocks;
  } kargs;
  for (int i = 0; i < LC_PW_MAX_BUFFERS; ++i) kargs.buffers[i] = args.buffers[i];
  kargs.blocks = (long long)args.blocks;
  void *params[] = {&kargs};
  if (launch(function, (unsigned)grid, 1, 1, (unsigned)args.lay.threads, 1, 1, (unsigned)smem_bytes,
             reinterpret_cast<CUstream>(stream), params, nullptr) != CUDA_SUCCESS)
    return fail(LC_ERR_CUDA, "lc_jit_blockprog: launch failed");
  return LC_OK;
}

extern "C" int lc_jit_pointwise(const void *image, size_t image_size, const lc_pw_program *program,
                                void *const *buffers, void *stream) {
  using namespace lc;
  if (!image || image_size < 16) return fail(LC_ERR_INVALID, "lc_jit_pointwise: no module image");
  int64_t points = 0;
  if (int rc = validate_program("lc_jit_pointwise", program, buffers, kPointwise, &points)) return rc;
  CUfunction function = nullptr;
  if (int rc = jit_function(image, image_size, "lc_jit_point", &function)) return rc;
  using LaunchFn = CUresult (*)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                                CUstream, void **, void **);
  static LaunchFn launch = driver_entry<LaunchFn>("cuLaunchKernel");
  if (!launch) return fail(LC_ERR_CUDA, "lc_jit_pointwise: cuLaunchKernel unavailable");
  struct {
    void *buffers[LC_PW_MAX_BUFFERS];
    long long points;
  } kargs;
  for (int i = 0; i < LC_PW_MAX_BUFFERS; ++i) kargs.buffers[i] = i < program->n_buffers ? buffers[i] : nullptr;
  kargs.points = (long long)points;
  int64_t blocks = (points + 255) / 256;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  void *params[] = {&kargs};
  if (launch(function, (unsigned)blocks, 1, 1, 256, 1, 1, 0, reinterpret_cast<CUstream>(stream), params,
             nullptr) != CUDA_SUCCESS)
    return fail(LC_ERR_CUDA, "lc_jit_pointwise: launch failed");
  return LC_OK;
}

extern "C" int lc_jit_rowprog(const void *image, size_t image_size, const lc_pw_program *program,
                              const lc_rp_layout *layout, void *const *buffers, void *stream) {
  using namespace lc;
  if (!image || image_size < 16) return fail(LC_ERR_INVALID, "lc_jit_rowprog: no module image");
  int64_t rows = 0;
  if (int rc = prepare_rowprog("lc_jit_rowprog", program, layout, buffers, &rows)) return rc;
  CUfunction function = nullptr;
  if (int rc = jit_function(image, image_size, "lc_jit_rows", &function)) return rc;
  using LaunchFn = CUresult (*)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                                CUstream, void **, void **);
  static LaunchFn launch = driver_entry<LaunchFn>("cuLaunchKernel");
  if (!launch) return fail(LC_ERR_CUDA, "lc_jit_rowprog: cuLaunchKernel unavailable");
  struct {
    void *buffers[LC_PW_MAX_BUFFERS];
    long long rows;
  } kargs;
  for (int i = 0; i < LC_PW_MAX_BUFFERS; ++i) kargs.buffers[i] = i < program->n_buffers ? buffers[i] : nullptr;
  kargs.rows = (long long)rows;
  int64_t blocks = rows;
  const int64_t cap = (int64_t)sm_count() * 8;
  if (blocks > cap) blocks = cap;
  void *params[] = {&kargs};
  if (launch(function, (unsigned)blocks, 1, 1, (unsigned)layout->threads, 1, 1, 0,
             reinterpret_cast<CUstream>(stream), params, nullptr) != CUDA_SUCCESS)
    return fail(LC_ERR_CUDA, "lc_jit_rowprog: launch failed");
  return LC_OK;
}
