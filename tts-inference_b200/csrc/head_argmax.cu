// Fused codebook head of a decode step: RMSNorm -> int8 weight-only head ->
// greedy code -> the embedding row of that code, in one launch.
//
// One step of the code predictor's codebook loop (qtts/models/code_predictor.py
// :229-242) ends with
//   logits = lm_head[step](norm(hidden)[:, step])     (1024 -> 2048, bf16 out)
//   code   = logits.argmax(-1)                         (greedy)
//   next   = codec_embedding[step](code)               (the next position's input)
// and the talker's codec head the same way with logits masked to the codec
// vocabulary (qtts/models/talker.py:354-356). As separate kernels that is the
// norm, the head GEMM, a cast, the argmax, the index handling and the
// embedding gather, each a dependent launch on a few kilobytes.
//
// Here one grid does all of it:
//   * every CTA owns 16 weight rows and prefetches them into registers before
//     the programmatic-dependent-launch wait (the head weights are constant);
//   * after the wait each CTA computes the rows' RMSNorm factors in the
//     library's fixed order (csrc/prologue.cuh, equal bit for bit to the other
//     norm paths) and stages the normalized activations in shared memory;
//   * each warp takes two weight rows: lane l holds k = 4l..4l+3 of every
//     128-column block (coalesced 4-byte weight loads, conflict-free float4
//     activation loads), fp32 products, one warp reduction per batch row; the
//     per-channel scale applies after the sum, the result is rounded to the
//     activation type (the head's output dtype, which is what the argmax sees),
//     then the optional fp32 logit bias is added (0 or -inf: a mask);
//   * the greedy code is the first index of the maximum, as torch.argmax: each
//     batch row's candidates are packed as (order-preserving float bits << 32 |
//     ~index) and combined with 64-bit atomic max, first within the CTA, then
//     in a caller-provided state array;
//   * the last CTA to finish (a counter in the same state array) writes the
//     codes, copies the embedding rows of those codes and re-zeroes the state,
//     so consecutive calls and CUDA-graph replays need no reset.
// No waits: nothing here spins, so nothing can hang.
#include "common.cuh"
#include "kernels.h"
#include "prologue.cuh"

namespace qtts {
namespace {

constexpr int kHaThreads = 256;
constexpr int kHaWarps = kHaThreads / 32;
constexpr int kHaRows = 2 * kHaWarps;  // weight rows per CTA
constexpr int kHaMaxKBlocks = 16;      // K <= 2048 (128-column blocks held per row)

__device__ __forceinline__ uint32_t order_bits(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long pack_candidate(float v, int n) {
  return (static_cast<unsigned long long>(order_bits(v)) << 32) | (0xFFFFFFFFull - static_cast<uint32_t>(n));
}

template <typename XT, int MR>
__global__ void __launch_bounds__(kHaThreads) head_argmax_kernel(const HeadArgs a) {
  extern __shared__ float ha_smem[];
  const int K = a.K;
  const int groups = ((K >> 3) + 31) >> 5;
  float* xs = ha_smem;                    // [MR][K] normalized activations
  float* gs = xs + MR * K;                // [MR][groups] norm group sums
  float* rinv = gs + MR * groups;         // [MR]
  __shared__ unsigned long long best[MR];
  __shared__ int last_cta;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n0 = blockIdx.x * kHaRows + 2 * warp;
  const int kb = K >> 7;  // 128-column blocks

  // Weights first: constant, so they load while the previous kernel drains.
  uint32_t wr[2][kHaMaxKBlocks];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int n = n0 + r;
#pragma unroll
    for (int b = 0; b < kHaMaxKBlocks; ++b) {
      wr[r][b] = 0u;
      if (n < a.N && b < kb) {
        wr[r][b] = __ldg(reinterpret_cast<const uint32_t*>(a.w + static_cast<int64_t>(n) * a.ldw + 128 * b + 4 * lane));
      }
    }
  }
  if (tid < MR) best[tid] = 0ull;
  pdl_launch_dependents();
  pdl_wait();

  const XT* x = static_cast<const XT*>(a.x);
  const XT* nw = static_cast<const XT*>(a.norm_weight);
  if (nw != nullptr) {
    cta_norm_factors<XT>(x, a.ldx, a.M, K, a.eps, gs, rinv, warp, lane, kHaWarps, 1);
  }
  // Normalized activations (the library's RMSNorm element: cast(w * (x * inv)))
  // as fp32 in shared memory; rows past M are zeros.
  const int cpr = K >> 3;
  for (int i = tid; i < MR * cpr; i += kHaThreads) {
    const int m = i / cpr;
    const int c = i - m * cpr;
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (m < a.M) {
      u = __ldcg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(m) * a.ldx + 8 * c));
      if (nw != nullptr) u = normalize_chunk<XT>(u, __ldg(reinterpret_cast<const uint4*>(nw + 8 * c)), rinv[m]);
    }
    const XT* e = reinterpret_cast<const XT*>(&u);
    float4* dst = reinterpret_cast<float4*>(xs + m * K + 8 * c);
    dst[0] = make_float4(to_float(e[0]), to_float(e[1]), to_float(e[2]), to_float(e[3]));
    dst[1] = make_float4(to_float(e[4]), to_float(e[5]), to_float(e[6]), to_float(e[7]));
  }
  named_bar_sync(1, kHaThreads);

  // Two rows per warp: partial dot products over this lane's columns.
  float acc[2][MR];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[r][m] = 0.f;
  }
#pragma unroll
  for (int b = 0; b < kHaMaxKBlocks; ++b) {
    if (b < kb) {
      float wf[2][4];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int q = 0; q < 4; ++q) wf[r][q] = static_cast<float>(static_cast<int8_t>((wr[r][b] >> (8 * q)) & 0xFF));
      }
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        const float4 xv = *reinterpret_cast<const float4*>(xs + m * K + 128 * b + 4 * lane);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          acc[r][m] = fmaf(wf[r][0], xv.x, acc[r][m]);
          acc[r][m] = fmaf(wf[r][1], xv.y, acc[r][m]);
          acc[r][m] = fmaf(wf[r][2], xv.z, acc[r][m]);
          acc[r][m] = fmaf(wf[r][3], xv.w, acc[r][m]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
#pragma unroll
    for (int m = 0; m < MR; ++m) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], off);
    }
  }
  // Logits of this warp's rows, rounded to the head's output type, masked,
  // and folded into the CTA's best candidate per batch row.
  if (lane < MR && lane < a.M) {
    unsigned long long cand = 0ull;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int n = n0 + r;
      if (n < a.N) {
        float v = 0.f;
#pragma unroll
        for (int m = 0; m < MR; ++m) {
          if (m == lane) v = acc[r][m];
        }
        v = to_float(from_float<XT>(v * load_as_float(a.scale, a.scale_dtype, n)));
        if (a.logit_bias != nullptr) v = __fadd_rn(v, a.logit_bias[n]);
        const unsigned long long c = pack_candidate(v, n);
        cand = c > cand ? c : cand;
      }
    }
    if (cand != 0ull) atomicMax(&best[lane], cand);
  }
  __syncthreads();
  if (tid < a.M) {
    atomicMax(reinterpret_cast<unsigned long long*>(a.state) + tid, best[tid]);
    __threadfence();  // this CTA's candidates are in before it counts itself done
  }
  __syncthreads();
  if (tid == 0) {
    const unsigned long long done =
        atomicAdd(reinterpret_cast<unsigned long long*>(a.state) + a.M, 1ull);
    last_cta = done == static_cast<unsigned long long>(gridDim.x) - 1ull;
  }
  __syncthreads();
  if (!last_cta) return;

  // The last CTA: every candidate is in; codes out, embedding rows out, state re-zeroed.
  __threadfence();
  __shared__ int codes_s[MR];
  if (tid < a.M) {
    const unsigned long long key = atomicMax(reinterpret_cast<unsigned long long*>(a.state) + tid, 0ull);
    const int code = static_cast<int>(0xFFFFFFFFull - (key & 0xFFFFFFFFull));
    codes_s[tid] = code;
    a.codes[tid] = code;
    reinterpret_cast<unsigned long long*>(a.state)[tid] = 0ull;
  }
  if (tid == 0) reinterpret_cast<unsigned long long*>(a.state)[a.M] = 0ull;
  __syncthreads();
  if (a.embed != nullptr) {
    const XT* emb = static_cast<const XT*>(a.embed);
    XT* eo = static_cast<XT*>(a.embed_out);
    const int epr = a.E >> 3;  // 16-byte chunks per row
    for (int i = tid; i < a.M * epr; i += kHaThreads) {
      const int m = i / epr;
      const int c = i - m * epr;
      const int code = codes_s[m];
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (code >= 0 && code < a.vocab) {
        v = __ldg(reinterpret_cast<const uint4*>(emb + static_cast<int64_t>(code) * a.lde + 8 * c));
      } else if (c == 0) {
        record_status(QTTS_ERR_SHAPE);
      }
      *reinterpret_cast<uint4*>(eo + static_cast<int64_t>(m) * a.ldeo + 8 * c) = v;
    }
  }
}

template <typename XT, int MR>
int launch_ha(const HeadArgs& a, bool pdl, cudaStream_t stream) {
  const int groups = ((a.K >> 3) + 31) >> 5;
  const size_t smem = sizeof(float) * (static_cast<size_t>(MR) * a.K + MR * groups + MR);
  auto kern = head_argmax_kernel<XT, MR>;
  if (smem > 48 * 1024) {
    // Exactly what this launch needs: the kernel also has a little static shared
    // memory, and dynamic + static must stay within the per-block limit.
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess) {
      (void)cudaGetLastError();
      return QTTS_ERR_LAUNCH;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + kHaRows - 1) / kHaRows);
  cfg.blockDim = dim3(kHaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

template <typename XT>
int launch_ha_m(const HeadArgs& a, bool pdl, cudaStream_t stream) {
  if (a.M <= 8) return launch_ha<XT, 8>(a, pdl, stream);
  return launch_ha<XT, 16>(a, pdl, stream);
}

}  // namespace

size_t head_argmax_smem(int M, int K) {
  const int mr = M <= 8 ? 8 : 16;
  const int groups = ((K >> 3) + 31) >> 5;
  return sizeof(float) * (static_cast<size_t>(mr) * K + mr * groups + mr);
}

int launch_head_argmax(const HeadArgs& a, int x_dtype, bool pdl, cudaStream_t stream) {
  if (x_dtype == QTTS_BF16) return launch_ha_m<__nv_bfloat16>(a, pdl, stream);
  if (x_dtype == QTTS_FP16) return launch_ha_m<__half>(a, pdl, stream);
  return QTTS_ERR_DTYPE;
}

}  // namespace qtts
