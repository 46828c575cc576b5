// Standalone activation prologues: RMSNorm (qtts_rms_norm; replaces
// _rms_norm_kernel and RMSNorm.forward, qtts/layers/norm.py:49-76, 102-137)
// and SiLU·up (qtts_silu_mul; replaces F.silu(gate) * up,
// qtts/layers/activation.py:147). They also serve as the first half of
// qtts_w8a16_gemm_prologue when the chosen GEMM kernel cannot fuse the
// prologue: they write the activation the GEMM then reads, and let it launch
// early (programmatic dependent launch) so its weights stream in meanwhile.
// The element arithmetic is csrc/prologue.cuh's, shared with the fused forms.
//
// RMSNorm: one warp per row, two passes over the row (sum of squares in the
// fixed order, then scale and store; the second pass hits L2). SiLU·up: one thread per 8-element chunk, grid-stride.
#include "kernels.h"
#include "prologue.cuh"

namespace qtts {

namespace {

constexpr int kPrThreads = 256;
constexpr int kPrRowsPerCta = kPrThreads / 32;

template <typename XT>
__device__ __forceinline__ void store8(XT* p, int n, bool vec, const float (&v)[8]) {
  if (vec && n >= 8) {
    if constexpr (sizeof(XT) == 2) {
      uint4 o;
      XT* r = reinterpret_cast<XT*>(&o);
#pragma unroll
      for (int q = 0; q < 8; ++q) r[q] = from_float<XT>(v[q]);
      *reinterpret_cast<uint4*>(p) = o;
    } else {
      reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    return;
  }
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    if (q < n) p[q] = from_float<XT>(v[q]);
  }
}

// Rows of at most kRegGroups * 256 16-bit elements: each lane keeps its chunks
// of the row and of the weight in registers, so the row is read once.
constexpr int kRegGroups = 8;

template <typename XT>
__device__ __forceinline__ void rms_norm_row_regs(const XT* xr, const XT* w, XT* orow, int width, float eps,
                                                  int lane, float* wgs) {
  const int chunks = width >> 3;
  const int groups = (chunks + 31) >> 5;
  uint4 xv[kRegGroups], wv[kRegGroups];
#pragma unroll
  for (int g = 0; g < kRegGroups; ++g) {
    const int c = 32 * g + lane;
    xv[g] = wv[g] = make_uint4(0u, 0u, 0u, 0u);
    if (c < chunks) {
      xv[g] = __ldcg(reinterpret_cast<const uint4*>(xr + 8 * c));
      wv[g] = __ldg(reinterpret_cast<const uint4*>(w + 8 * c));
    }
  }
#pragma unroll
  for (int g = 0; g < kRegGroups; ++g) {
    if (g < groups) {
      const XT* e = reinterpret_cast<const XT*>(&xv[g]);
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = to_float(e[q]);
      const float s = group_butterfly(leaf_sumsq(v));
      if (lane == 0) wgs[g] = s;
    }
  }
  __syncwarp();
  const float inv = rms_inv(lanes_stride_tree(lane < groups ? wgs[lane] : 0.f, groups), width, eps);
#pragma unroll
  for (int g = 0; g < kRegGroups; ++g) {
    const int c = 32 * g + lane;
    if (c < chunks) *reinterpret_cast<uint4*>(orow + 8 * c) = normalize_chunk<XT>(xv[g], wv[g], inv);
  }
}

template <typename XT>
__global__ void __launch_bounds__(kPrThreads) rms_norm_kernel(const XT* x, int64_t ldx, const XT* w, XT* out,
                                                              int64_t ldo, int rows, int width, float eps, bool vec) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ float wgs[kPrRowsPerCta][kMaxNormGroups];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row = blockIdx.x * kPrRowsPerCta + warp;
  if (row >= rows) return;
  const XT* xr = x + static_cast<int64_t>(row) * ldx;
  XT* orow = out + static_cast<int64_t>(row) * ldo;
  if constexpr (sizeof(XT) == 2) {
    if (vec && width <= 256 * kRegGroups) {
      rms_norm_row_regs<XT>(xr, w, orow, width, eps, lane, wgs[warp]);
      return;
    }
  }
  const float inv = rms_inv(warp_row_sumsq<XT>(xr, width, vec, lane, wgs[warp]), width, eps);
  const int chunks = (width + 7) >> 3;
  for (int c = lane; c < chunks; c += 32) {
    const int n = width - 8 * c;
    float v[8], g[8];
    load8<XT>(xr + 8 * c, n, vec, v);
    load8<XT>(w + 8 * c, n, vec, g);
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = rms_apply(v[q], inv, g[q]);
    store8<XT>(orow + 8 * c, n, vec, v);
  }
}

template <typename XT>
__global__ void __launch_bounds__(kPrThreads) silu_mul_kernel(const XT* in, int64_t ldi, XT* out, int64_t ldo,
                                                              int rows, int width, bool vec) {
  pdl_launch_dependents();
  pdl_wait();
  const int chunks = (width + 7) >> 3;
  const int64_t total = static_cast<int64_t>(rows) * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kPrThreads + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kPrThreads) {
    const int r = static_cast<int>(i / chunks);
    const int c = static_cast<int>(i - static_cast<int64_t>(r) * chunks);
    const int n = width - 8 * c;
    const XT* gate = in + static_cast<int64_t>(r) * ldi + 8 * c;
    float g[8], u[8];
    load8<XT>(gate, n, vec, g);
    load8<XT>(gate + width, n, vec, u);
#pragma unroll
    for (int q = 0; q < 8; ++q) g[q] = silu_mul<XT>(g[q], u[q]);
    store8<XT>(out + static_cast<int64_t>(r) * ldo + 8 * c, n, vec, g);
  }
}

template <typename KernT, typename... Args>
int launch_pr(KernT kern, dim3 grid, bool pdl, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kPrThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, args...) == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

template <typename XT>
int launch_prologue_t(const PrologueArgs& p, bool pdl, cudaStream_t stream) {
  const XT* x = static_cast<const XT*>(p.x);
  XT* out = static_cast<XT*>(p.out);
  if (p.kind == kProRmsNorm) {
    const dim3 grid((p.rows + kPrRowsPerCta - 1) / kPrRowsPerCta);
    return launch_pr(rms_norm_kernel<XT>, grid, pdl, stream, x, p.ldx, static_cast<const XT*>(p.weight), out, p.ldo,
                     p.rows, p.width, p.eps, p.vec);
  }
  if (p.kind == kProSiluMul) {
    const int64_t chunks = static_cast<int64_t>(p.rows) * ((p.width + 7) / 8);
    const int64_t ctas = (chunks + kPrThreads - 1) / kPrThreads;
    const dim3 grid(static_cast<unsigned>(ctas < 4 * kNumSMs ? ctas : 4 * kNumSMs));
    return launch_pr(silu_mul_kernel<XT>, grid, pdl, stream, x, p.ldx, out, p.ldo, p.rows, p.width, p.vec);
  }
  return QTTS_ERR_VARIANT;
}

}  // namespace

int launch_prologue(const PrologueArgs& p, int dtype, bool pdl, cudaStream_t stream) {
  if (p.rows == 0 || p.width == 0) return QTTS_OK;
  switch (dtype) {
    case QTTS_BF16:
      return launch_prologue_t<__nv_bfloat16>(p, pdl, stream);
    case QTTS_FP16:
      return launch_prologue_t<__half>(p, pdl, stream);
    case QTTS_FP32:
      return launch_prologue_t<float>(p, pdl, stream);
    default:
      return QTTS_ERR_DTYPE;
  }
}

}  // namespace qtts
