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
// taken in one fixed order, so that every kernel of this library that
// normalizes a row (the standalone kernel, and every CTA of a GEMM that fuses
// the norm, whatever its warp count) gets the same bits:
//   leaf c   the 8-element chunk c (zeros past the row): fp32 fma chain over
//            its elements in order (exact products for 16-bit inputs);
//   group g  leaves 32g .. 32g+31: xor butterfly, strides 16, 8, 4, 2, 1
//            (one warp's coalesced 512-byte load; fp32 addition is
//            commutative, so every lane ends with the same sum);
//   row      stride-halving tree over the group sums, padded with zeros to
//            G = the next power of two: for h = G/2 .. 1, S[j] += S[j + h].
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
// RMSNorm whose CTA loads the whole rows for the factor (the split-K kernel
// takes it when its slices are not aligned to the norm's 256-column groups).
constexpr int kProRmsNormRows = 3;

__host__ __device__ constexpr bool is_rms(int pro) { return pro == kProRmsNorm || pro == kProRmsNormRows; }

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

__device__ __forceinline__ float rms_inv(float sumsq, int width, float eps) {
  const float var = __fdiv_rn(sumsq, static_cast<float>(width));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

__device__ __forceinline__ float rms_apply(float x, float inv, float w) { return __fmul_rn(w, __fmul_rn(x, inv)); }

constexpr int kMaxNormGroups = 256;       // standalone kernel: width <= 65536
constexpr int kMaxFusedNormGroups = 32;   // fused into a GEMM: K <= 8192

__device__ __forceinline__ float leaf_sumsq(const float (&v)[8]) {
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) s = fmaf(v[q], v[q], s);
  return s;
}

__device__ __forceinline__ float group_butterfly(float s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  return s;
}

// Stride-halving tree over the values of lanes [0, n) (n <= 32, zeros past n,
// padded to the next power of two); every lane returns the total.
__device__ __forceinline__ float lanes_stride_tree(float v, int n) {
  int g = 1;
  while (g < n) g <<= 1;
  for (int h = g >> 1; h > 0; h >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, h));
  return __shfl_sync(0xffffffffu, v, 0);
}

// Sum of squares of row[0, width) (width <= 65536) by one warp, in the fixed
// order above. `wgs` is this warp's shared scratch of kMaxNormGroups floats.
// Every lane returns the same value.
template <typename XT>
__device__ __forceinline__ float warp_row_sumsq(const XT* row, int width, bool vec, int lane, float* wgs) {
  const int chunks = (width + 7) >> 3;
  const int groups = (chunks + 31) >> 5;
  for (int g0 = 0; g0 < groups; g0 += 8) {
    float v[8][8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = 32 * (g0 + u) + lane;
      if (g0 + u < groups && c < chunks) {
        load8<XT>(row + 8 * c, width - 8 * c, vec, v[u]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[u][q] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (g0 + u < groups) {
        const float s = group_butterfly(leaf_sumsq(v[u]));
        if (lane == 0) wgs[g0 + u] = s;
      }
    }
  }
  __syncwarp();
  int gp = 1;
  while (gp < groups) gp <<= 1;
  float total;
  if (gp <= 32) {
    total = lanes_stride_tree(lane < groups ? wgs[lane] : 0.f, groups);
  } else {
    // Levels h >= 32 pair values of the same lane: S[l + 32i] with S[l + 32(i + hh)].
    const int per_lane = gp >> 5;  // 2, 4 or 8
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = (i < per_lane && lane + 32 * i < groups) ? wgs[lane + 32 * i] : 0.f;
#pragma unroll
    for (int hh = 4; hh > 0; hh >>= 1) {
      if (hh < per_lane) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (i < hh) s[i] = __fadd_rn(s[i], s[i + hh]);
        }
      }
    }
    total = lanes_stride_tree(s[0], 32);
  }
  __syncwarp();  // wgs is reused by this warp's next row
  return total;
}

// Norm factors rinv[m] of rows [0, rows) of x (leading dimension ldx, width
// a multiple of 8 and at most 8192, 16-byte aligned rows) by the `nwarps`
// warps of a CTA, in the same fixed order: each (row, group) is one warp's
// task, the group sums meet in `gs` (shared, rows x groups floats) and one warp
// per row finishes the tree. Called by all nwarps*32 threads; ends with a
// barrier (named barrier `bar_id`) after which rinv is visible to all of them.
template <typename XT>
__device__ __forceinline__ void cta_norm_factors(const XT* x, int64_t ldx, int rows, int width, float eps,
                                                 float* gs, float* rinv, int warp, int lane, int nwarps,
                                                 int bar_id) {
  const int chunks = width >> 3;
  const int groups = (chunks + 31) >> 5;
  const int tasks = rows * groups;
  for (int t0 = warp; t0 < tasks; t0 += 4 * nwarps) {
    float v[4][8];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u * nwarps;
      const int m = t / groups;
      const int c = 32 * (t - m * groups) + lane;
      if (t < tasks && c < chunks) {
        load8<XT>(x + static_cast<int64_t>(m) * ldx + 8 * c, 8, true, v[u]);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[u][q] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = t0 + u * nwarps;
      if (t < tasks) {
        const float s = group_butterfly(leaf_sumsq(v[u]));
        if (lane == 0) gs[t] = s;
      }
    }
  }
  named_bar_sync(bar_id, nwarps * 32);
  for (int m = warp; m < rows; m += nwarps) {
    const float s = lanes_stride_tree(lane < groups ? gs[m * groups + lane] : 0.f, groups);
    if (lane == 0) rinv[m] = rms_inv(s, width, eps);
  }
  named_bar_sync(bar_id, nwarps * 32);
}

template <typename XT>
__device__ __forceinline__ float silu_mul(float g, float up) {
  const float s = to_float(from_float<XT>(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g)))));
  return __fmul_rn(s, up);
}

// RMSNorm of a raw 16-bit chunk `u` with its norm-weight chunk `wv`.
template <typename XT>
__device__ __forceinline__ uint4 normalize_chunk(const uint4& u, const uint4& wv, float inv) {
  const XT* e = reinterpret_cast<const XT*>(&u);
  const XT* we = reinterpret_cast<const XT*>(&wv);
  uint4 o;
  XT* r = reinterpret_cast<XT*>(&o);
#pragma unroll
  for (int q = 0; q < 8; ++q) r[q] = from_float<XT>(rms_apply(to_float(e[q]), inv, to_float(we[q])));
  return o;
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
    if constexpr (is_rms(PRO)) {
      return normalize_chunk<XT>(u, __ldg(reinterpret_cast<const uint4*>(wnorm + k)), inv);
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
