// Activation prologues of the weight-only GEMMs (qtts_w8a16_gemm_prologue) and
// of their standalone kernels (qtts_rms_norm, qtts_silu_mul). One definition
// of each element, shared by every kernel that computes it, so the fused GEMM
// and the standalone kernel followed by the plain GEMM give the same bits.
//
// RMSNorm (qtts/layers/norm.py:49-76 fused, 123-137 eager):
//   y[m, k] = cast( w[k] * (x[m, k] * inv[m]) ),
//   inv[m]  = 1 / sqrt( sum_k x[m, k]^2 / width + eps )
// in fp32, the elementwise steps in the reference's order (x * inv first, the
// weight after: norm.py:75, 134-136) and 1 / sqrt correctly rounded, as the
// reference's fused kernel has it (norm.py:67-74). The sum of squares is
// taken in one fixed order: lane l of a warp takes the 8-element chunks
// c = l, l + 32, l + 64, ... of the row in increasing c, each chunk's elements
// in order, accumulating with fp32 fma (exact products for 16-bit inputs);
// the 32 lane sums then meet in a butterfly (xor 16, 8, 4, 2, 1), which
// leaves the same value in every lane because fp32 addition is commutative.
// The reference's own two forms differ from each other in the reduction order
// and in rsqrt; its tests hold them within one bf16 step of each other.
//
// SiLU·up (qtts/layers/activation.py:147, F.silu(gate) * up):
//   s = cast( g / (1 + exp(-g)) ),  y = cast( float(s) * float(up) )
// each step rounded to the activation type, as torch's two elementwise kernels
// do (silu computed in fp32 and stored, then the product in fp32 and stored).
// The division is IEEE (the library is built without fast-math).
#pragma once

#include "common.cuh"

namespace qtts {

constexpr int kProNone = 0;     // QTTS_PROLOGUE_NONE
constexpr int kProRmsNorm = 1;  // QTTS_PROLOGUE_RMSNORM
constexpr int kProSiluMul = 2;  // QTTS_PROLOGUE_SILU_MUL

// Eight elements starting at p as fp32 (zeros past n). `vec`: p is 16-byte
// aligned (32-byte for fp32) and all eight exist.
template <typename XT>
__device__ __forceinline__ void load8(const XT* p, int n, bool vec, float (&v)[8]) {
  if (vec && n >= 8) {
    if constexpr (sizeof(XT) == 2) {
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(p));
      const XT* e = reinterpret_cast<const XT*>(&u);
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = to_float(e[q]);
    } else {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(p));
      const float4 b = __ldcg(reinterpret_cast<const float4*>(p) + 1);
      v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    }
    return;
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = q < n ? to_float(p[q]) : 0.f;
}

// Sum of squares of row[0, width) in the fixed order above; every lane of the
// calling warp returns the same value.
template <typename XT>
__device__ __forceinline__ float warp_row_sumsq(const XT* row, int width, bool vec, int lane) {
  const int chunks = (width + 7) >> 3;
  float ss = 0.f;
  int c = lane;
  // Four chunks in flight per lane; accumulated in increasing c all the same.
  for (; c + 96 < chunks; c += 128) {
    float v[4][8];
#pragma unroll
    for (int j = 0; j < 4; ++j) load8<XT>(row + 8 * (c + 32 * j), width - 8 * (c + 32 * j), vec, v[j]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int q = 0; q < 8; ++q) ss = fmaf(v[j][q], v[j][q], ss);
    }
  }
  for (; c < chunks; c += 32) {
    float v[8];
    load8<XT>(row + 8 * c, width - 8 * c, vec, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) ss = fmaf(v[q], v[q], ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  return ss;
}

__device__ __forceinline__ float rms_inv(float sumsq, int width, float eps) {
  const float var = __fdiv_rn(sumsq, static_cast<float>(width));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

__device__ __forceinline__ float rms_apply(float x, float inv, float w) { return __fmul_rn(w, __fmul_rn(x, inv)); }

template <typename XT>
__device__ __forceinline__ float silu_mul(float g, float up) {
  const float s = to_float(from_float<XT>(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g)))));
  return __fmul_rn(s, up);
}

// The 16-bit activation chunk (eight elements at column k of one row) that a
// GEMM stages, after the prologue. `xrow` is the row of the GEMM's input: the
// raw activation (RMSNorm; `wnorm` the norm weight, `inv` the row's factor)
// or the gate half of a [gate | up] row whose up half starts `width` columns
// later (SiLU·up). k is a multiple of 8 and the row 16-byte aligned.
template <typename XT, int PRO>
__device__ __forceinline__ uint4 prologue_chunk(const XT* xrow, int k, int width, const XT* wnorm, float inv) {
  const uint4 u = __ldcg(reinterpret_cast<const uint4*>(xrow + k));
  if constexpr (PRO == kProNone) {
    return u;
  } else {
    const XT* e = reinterpret_cast<const XT*>(&u);
    uint4 o;
    XT* r = reinterpret_cast<XT*>(&o);
    if constexpr (PRO == kProRmsNorm) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wnorm + k));
      const XT* we = reinterpret_cast<const XT*>(&wv);
#pragma unroll
      for (int q = 0; q < 8; ++q) r[q] = from_float<XT>(rms_apply(to_float(e[q]), inv, to_float(we[q])));
    } else {
      const uint4 uv = __ldcg(reinterpret_cast<const uint4*>(xrow + width + k));
      const XT* ue = reinterpret_cast<const XT*>(&uv);
#pragma unroll
      for (int q = 0; q < 8; ++q) r[q] = from_float<XT>(silu_mul<XT>(to_float(e[q]), to_float(ue[q])));
    }
    return o;
  }
}

}  // namespace qtts
