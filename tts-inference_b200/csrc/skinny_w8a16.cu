// Skinny int8 weight-only GEMM (W8A16) for decode batch sizes.
//
// Replaces the Triton kernel _w8_gemm_kernel (qtts/quant/kernels.py:89-135):
//   out[m, n] = cast( sum_k x[m, k] * dequant(w[n, k]) * scale[n] + bias[n] )
// with the int8 -> bf16/fp16 convert done in registers, fp32 accumulation and
// the per-output-channel scale applied once after the K loop
// (kernels.py:123, 129-130).
//
// Design (B200, sm_100a):
//   * A CTA owns 64 weight rows and one K slice. A producer warp streams the
//     weight slice HBM -> shared memory with 2-D TMA boxes of 64 rows x 128
//     bytes (128-byte swizzle) through a ring of mbarrier-tracked stages.
//     Weights are constant, so the producer starts streaming before the
//     programmatic-dependent-launch wait: in a chain of linears the next
//     layer's weight stream overlaps the previous kernel's tail.
//   * 8 consumer warps wait on the dependency, stage the activation slice in
//     shared memory, then per stage each warp takes 16 rows x 64 k: one
//     128-bit shared load per row pair, dequantize in registers and issue
//     mma.sync.m16n8k16 with the weight as the M=16 operand and the
//     activations as the N=8 operand ("swap AB"), so batch rows 1..8 cost one
//     MMA per 256 weights. K is permuted inside each 64-wide chunk (thread q
//     owns k = 16q..16q+15) so that weight and activation fragments are
//     plain contiguous loads; the dot product does not depend on the order.
//   * Split-K across the CTAs of a thread-block cluster (1, 2, 4 or 8 CTAs):
//     partial sums are reduced through distributed shared memory, each CTA
//     finishing 64/split rows. No global workspace, no second kernel.
//   * Every wait is bounded (globaltimer); on expiry the kernel records
//     QTTS_ERR_TIMEOUT in the device status word and takes an error path that
//     still meets every barrier and drains its own copies in flight.
#include <cooperative_groups.h>

#include "common.cuh"
#include "kernels.h"

namespace cg = cooperative_groups;

namespace qtts {

constexpr int kSkBN = 64;                         // weight rows per CTA
constexpr int kSkBK = 128;                        // k bytes per stage (one swizzle span)
constexpr int kSkStageBytes = kSkBN * kSkBK;      // 8 KiB
constexpr int kSkConsumerWarps = 8;
constexpr int kSkThreads = (kSkConsumerWarps + 1) * 32;

template <int MT, typename XT>
__global__ void __launch_bounds__(kSkThreads, 2)
    skinny_w8a16_kernel(const __grid_constant__ CUtensorMap wmap, const SkinnyArgs a) {
  constexpr int MB = MT * 8;  // batch rows per CTA (MMA N dimension)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wbuf = smem;
  XT* xbuf = reinterpret_cast<XT*>(smem + a.stages * kSkStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(xbuf + MB * a.x_pitch) + 15) & ~uintptr_t(15));
  uint64_t* empty = full + a.stages;
  int* err_flag = reinterpret_cast<int*>(empty + a.stages);
  float* red = reinterpret_cast<float*>(wbuf);  // reused after the main loop

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int split = gridDim.y;
  const int kidx = blockIdx.y;
  const int n0 = blockIdx.x * kSkBN;
  const int mchunk = blockIdx.z % a.m_chunks;
  int group = blockIdx.z / a.m_chunks;
  const int m0 = mchunk * MB;
  const int k0 = kidx * a.k_per_cta;
  const int klen = max(0, min(a.K - k0, a.k_per_cta));
  int n_iters = (klen + kSkBK - 1) / kSkBK;

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSkConsumerWarps);
    }
    *err_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  // Device-indexed single group: the index may be produced by the preceding
  // kernel, so everything (including the weight stream) waits for it.
  bool valid = true;
  if (a.group_index != nullptr) {
    pdl_wait();
    const int64_t gi = __ldcg(a.group_index);
    if (gi < 0 || gi >= a.G) {
      valid = false;
      n_iters = 0;
      if (tid == 0) record_status(QTTS_ERR_SHAPE);
    } else {
      group = static_cast<int>(gi);
    }
  }
  const int64_t wrow0 = static_cast<int64_t>(group) * a.N + n0;
  const int64_t goff_x = a.group_index ? 0 : static_cast<int64_t>(group) * a.gsx;
  const int64_t goff_o = a.group_index ? 0 : static_cast<int64_t>(group) * a.gso;
  const XT* xg = static_cast<const XT*>(a.x) + goff_x + static_cast<int64_t>(m0) * a.ldx;
  XT* og = static_cast<XT*>(a.out) + goff_o + static_cast<int64_t>(m0) * a.ldo;
  const int mrows = min(MB, a.M - m0);

  int n_issued = 0;  // meaningful in the producer lane only
  if (warp == kSkConsumerWarps) {
    // ---------------- producer: weight stream ----------------
    if (lane == 0 && n_iters > 0) {
      tma_prefetch_desc(&wmap);
      for (int it = 0; it < n_iters; ++it) {
        const int s = it % a.stages;
        if (it >= a.stages) {
          if (!mbar_wait_bounded(&empty[s], ((it / a.stages) - 1) & 1, a.wait_ns)) {
            record_status(QTTS_ERR_TIMEOUT);
            *reinterpret_cast<volatile int*>(err_flag) = 1;
            break;
          }
        }
        mbar_arrive_expect_tx(&full[s], kSkStageBytes);
        tma_load_2d(wbuf + s * kSkStageBytes, &wmap, k0 + it * kSkBK, static_cast<int>(wrow0), &full[s]);
        n_issued = it + 1;
      }
    }
  } else {
    // ---------------- consumers ----------------
    pdl_wait();
    // Stage the activation slice [MB, n_iters*128] (zero padded) in shared memory.
    {
      constexpr int kVec = 16 / sizeof(XT);
      const int kpad = n_iters * kSkBK;
      const int per_row = kpad / kVec;
      for (int i = tid; i < MB * per_row; i += kSkConsumerWarps * 32) {
        const int m = i / per_row;
        const int kv = (i - m * per_row) * kVec;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (valid && m < mrows && kv < klen) {
          v = __ldcg(reinterpret_cast<const uint4*>(xg + static_cast<int64_t>(m) * a.ldx + k0 + kv));
        }
        *reinterpret_cast<uint4*>(xbuf + m * a.x_pitch + kv) = v;
      }
    }
    named_bar_sync(1, kSkConsumerWarps * 32);

    const int rg = warp >> 1;  // row group of 16
    const int cc = warp & 1;   // 64-wide k chunk within the 128-byte stage
    const int g = lane >> 2;
    const int q = lane & 3;
    // MMA row g <-> weight row 8*(g&1)/2 permutation: rows g and g^1 of an
    // LDS phase land in opposite 64-byte halves of the swizzled span.
    const int pr = (g >> 1) | ((g & 1) << 2);
    const int rowA = rg * 16 + pr;
    const int rowB = rowA + 8;
    const int c16 = cc * 4 + q;
    const uint32_t wbase = smem_u32(wbuf);
    const uint32_t offA = rowA * kSkBK + ((c16 ^ (rowA & 7)) << 4);
    const uint32_t offB = rowB * kSkBK + ((c16 ^ (rowB & 7)) << 4);
    const uint32_t xbase = smem_u32(xbuf) + (g * a.x_pitch + cc * 64 + q * 16) * sizeof(XT);
    const uint32_t xtile = 8 * a.x_pitch * sizeof(XT);

    float acc[MT][4];
#pragma unroll
    for (int t = 0; t < MT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

    bool ok = true;
    for (int it = 0; it < n_iters; ++it) {
      const int s = it % a.stages;
      const bool got = mbar_wait_bounded(&full[s], (it / a.stages) & 1, a.wait_ns);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      const uint32_t sb = wbase + s * kSkStageBytes;
      const uint4 wa = lds128(sb + offA);
      const uint4 wb = lds128(sb + offB);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);

      uint32_t A[4][4];
      Dequant<XT>::run(wa.x, A[0][0], A[0][2]);
      Dequant<XT>::run(wb.x, A[0][1], A[0][3]);
      Dequant<XT>::run(wa.y, A[1][0], A[1][2]);
      Dequant<XT>::run(wb.y, A[1][1], A[1][3]);
      Dequant<XT>::run(wa.z, A[2][0], A[2][2]);
      Dequant<XT>::run(wb.z, A[2][1], A[2][3]);
      Dequant<XT>::run(wa.w, A[3][0], A[3][2]);
      Dequant<XT>::run(wb.w, A[3][1], A[3][3]);

      const uint32_t xs = xbase + it * kSkBK * sizeof(XT);
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const uint4 x0 = lds128(xs + t * xtile);
        const uint4 x1 = lds128(xs + t * xtile + 16);
        Mma16816<XT>::run(acc[t], A[0], x0.x, x0.y);
        Mma16816<XT>::run(acc[t], A[1], x0.z, x0.w);
        Mma16816<XT>::run(acc[t], A[2], x1.x, x1.y);
        Mma16816<XT>::run(acc[t], A[3], x1.z, x1.w);
      }
    }
    if (!ok) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *reinterpret_cast<volatile int*>(err_flag) = 1;
    }
    // Every consumer warp is done reading the stage ring before it is reused
    // as the reduction buffer.
    named_bar_sync(1, kSkConsumerWarps * 32);
    if (*reinterpret_cast<volatile int*>(err_flag) == 0) {
      float* r = red + cc * kSkBN * MB;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int n = t * 8 + 2 * q;
        *reinterpret_cast<float2*>(&r[rowA * MB + n]) = make_float2(acc[t][0], acc[t][1]);
        *reinterpret_cast<float2*>(&r[rowB * MB + n]) = make_float2(acc[t][2], acc[t][3]);
      }
    }
  }
  __syncthreads();
  const bool cta_err = *reinterpret_cast<volatile int*>(err_flag) != 0;
  if (!cta_err) {
    for (int i = tid; i < kSkBN * MB; i += kSkThreads) red[i] += red[kSkBN * MB + i];
  }

  // ---------------- split-K reduction across the cluster + epilogue ----------------
  cg::cluster_group cluster = cg::this_cluster();
  if (split > 1) {
    cluster.sync();
  } else {
    __syncthreads();
  }
  const int rows_per = kSkBN / split;
  const int r0 = kidx * rows_per;
  if (!cta_err && valid) {
    for (int i = tid; i < rows_per * mrows; i += kSkThreads) {
      const int m = i / rows_per;
      const int row = r0 + (i - m * rows_per);
      const int n = n0 + row;
      if (n < a.N) {
        float v = 0.f;
        for (int p = 0; p < split; ++p) {
          const float* pr = split > 1 ? cluster.map_shared_rank(red, p) : red;
          v += pr[row * MB + m];
        }
        const int64_t ch = static_cast<int64_t>(group) * a.N + n;
        v *= load_as_float(a.scale, a.scale_dtype, ch);
        if (a.bias != nullptr) v += to_float(static_cast<const XT*>(a.bias)[ch]);
        og[static_cast<int64_t>(m) * a.ldo + n] = from_float<XT>(v);
      }
    }
  }
  if (split > 1) cluster.sync();

  // Error path: make sure no copy of ours is still landing in shared memory.
  if (cta_err && warp == kSkConsumerWarps && lane == 0) {
    for (int s = 0; s < a.stages && s < n_issued; ++s) {
      const int last = ((n_issued - 1 - s) / a.stages) * a.stages + s;
      mbar_wait_bounded(&full[s], (last / a.stages) & 1, a.wait_ns);
    }
  }
}

// ------------------------------------------------------------------------------------
// Host side

namespace {

template <int MT, typename XT>
int launch_skinny_t(const CUtensorMap& map, const SkinnyArgs& args, dim3 grid, int split, size_t smem,
                    bool pdl, cudaStream_t stream) {
  auto kern = skinny_w8a16_kernel<MT, XT>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem) != cudaSuccess) {
      return QTTS_ERR_CUDA;
    }
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (split > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = split;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, map, args);
  return e == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

template <typename XT>
int launch_skinny_mt(int mt, const CUtensorMap& map, const SkinnyArgs& args, dim3 grid, int split,
                     size_t smem, bool pdl, cudaStream_t stream) {
  switch (mt) {
    case 1:
      return launch_skinny_t<1, XT>(map, args, grid, split, smem, pdl, stream);
    case 2:
      return launch_skinny_t<2, XT>(map, args, grid, split, smem, pdl, stream);
    case 4:
      return launch_skinny_t<4, XT>(map, args, grid, split, smem, pdl, stream);
    default:
      return launch_skinny_t<8, XT>(map, args, grid, split, smem, pdl, stream);
  }
}

}  // namespace

SkinnyPlan plan_skinny(int M, int N, int K, int G, int split_req) {
  SkinnyPlan p{};
  p.mt = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
  const int mb = p.mt * 8;
  p.m_chunks = (M + mb - 1) / mb;
  const int n_tiles = (N + kSkBN - 1) / kSkBN;
  const int ctas_base = n_tiles * G * p.m_chunks;
  auto xbytes_for = [&](int split) {
    const int kpc = ((K + split - 1) / split + kSkBK - 1) / kSkBK * kSkBK;
    return static_cast<size_t>(mb) * (kpc + 8) * 2;
  };
  int split = split_req;
  if (split == 0) {
    // Smallest split that fills the machine once (148 SMs), keeping the
    // activation slice within 64 KiB of shared memory.
    split = 8;
    for (int s = 1; s <= 8; s *= 2) {
      if (xbytes_for(s) <= 64 * 1024 && ctas_base * s >= kNumSMs) {
        split = s;
        break;
      }
    }
  }
  p.split = split;
  p.k_per_cta = ((K + split - 1) / split + kSkBK - 1) / kSkBK * kSkBK;
  p.x_pitch = p.k_per_cta + 8;
  const size_t xbytes = static_cast<size_t>(mb) * p.x_pitch * 2;
  const int n_iters = (p.k_per_cta + kSkBK - 1) / kSkBK;
  // Stage count: fill a ~100 KiB budget so two CTAs fit per SM (the running
  // kernel and the next, PDL-launched one); at least enough stage bytes to
  // hold the 2 x 64 x MB fp32 reduction buffer.
  const size_t budget = 100 * 1024;
  int stages = xbytes + 2048 < budget ? static_cast<int>((budget - xbytes - 2048) / kSkStageBytes) : 0;
  stages = stages > 12 ? 12 : stages;
  stages = stages < n_iters ? stages : n_iters;
  const int min_stages = (2 * kSkBN * mb * 4 + kSkStageBytes - 1) / kSkStageBytes;
  stages = stages < min_stages ? min_stages : stages;
  stages = stages < 2 ? 2 : stages;
  p.stages = stages;
  p.smem = 1024 + static_cast<size_t>(stages) * kSkStageBytes + xbytes + 16 + 16 * stages + 16;
  p.grid = dim3(n_tiles, split, G * p.m_chunks);
  return p;
}

int launch_skinny_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, int x_dtype,
                        bool pdl, cudaStream_t stream) {
  if (p.smem > kMaxDynSmem) return QTTS_ERR_SHAPE;
  if (x_dtype == QTTS_BF16) return launch_skinny_mt<__nv_bfloat16>(p.mt, map, args, p.grid, p.split, p.smem, pdl, stream);
  if (x_dtype == QTTS_FP16) return launch_skinny_mt<__half>(p.mt, map, args, p.grid, p.split, p.smem, pdl, stream);
  return QTTS_ERR_DTYPE;
}

}  // namespace qtts
