// Skinny int8 weight-only GEMM (W8A16) for decode batch sizes.
//
// Replaces the Triton kernel _w8_gemm_kernel (qtts/quant/kernels.py:89-135):
//   out[m, n] = cast( sum_k x[m, k] * w[n, k] * scale[n] + bias[n] )
// with the int8 convert done in registers, fp32 accumulation and the
// per-output-channel scale applied once after the K loop (kernels.py:123,
// 129-130).
//
// Design (B200, sm_100a). A decode GEMM streams N*K weight bytes once and does
// 2*M flops per byte, so the kernel is built around the weight stream:
//   * A CTA owns 128 weight rows and one K slice. A producer warp streams the
//     slice HBM -> shared memory as 2-D TMA boxes of 128 rows x 128 bytes
//     (128-byte swizzle) through a ring of mbarrier-tracked stages. Weights
//     are constant, so streaming starts before the programmatic-dependent-
//     launch wait: in a chain of linears the next layer's weights arrive while
//     the previous kernel drains.
//   * 8 consumer warps wait on the dependency and stage the activation slice
//     in shared memory as fp16 with a per-row power-of-two scale (exact for
//     every element within 2^28 of the row's largest magnitude; smaller ones
//     round as fp16 subnormals, far below the bf16 output resolution).
//   * Dequantization is one byte-permute per two weights: 0x64 above a byte u
//     is the fp16 1024 + u, so (b ^ 0x80) placed there and 1152 subtracted
//     gives b exactly. The MMA is mma.sync m16n8k16 f16 with fp32 accumulation,
//     weights as the M=16 operand and activations as the N=8 operand ("swap
//     AB"): batch rows 1..8 cost one MMA per 256 weights.
//   * Each warp owns 16 rows over the whole 128-k stage, so no reduction is
//     needed inside the CTA. K is permuted inside each 64-wide chunk (thread q
//     owns k = 16q..16q+15) so weight and activation fragments are plain
//     128-bit shared loads; a dot product does not depend on the order.
//   * Split-K runs across the CTAs of a thread-block cluster (1, 2, 4 or 8).
//     Each CTA owns 128/split rows of the result; partial sums travel to their
//     owner with st.async into its shared memory, counted on the owner's
//     mbarrier. One split cluster barrier (arrive at start, wait before the
//     first remote store) is the only cluster-wide synchronization.
//   * Every wait is bounded (globaltimer). On expiry the kernel records
//     QTTS_ERR_TIMEOUT in the device status word, keeps the remote-store
//     protocol (so no peer waits on it), skips its global stores and drains its
//     own copies in flight before exiting.
#include "common.cuh"
#include "kernels.h"

namespace qtts {

constexpr int kSkBN = 128;                     // weight rows per CTA
constexpr int kSkBK = 128;                     // k bytes per stage (one swizzle span)
constexpr int kSkStageBytes = kSkBN * kSkBK;   // 16 KiB
constexpr int kSkConsumerWarps = 8;
constexpr int kSkThreads = (kSkConsumerWarps + 1) * 32;

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

template <int MT, typename XT>
__global__ void __launch_bounds__(kSkThreads, 2)
    skinny_w8a16_kernel(const __grid_constant__ CUtensorMap wmap, const SkinnyArgs a) {
  constexpr int MB = MT * 8;  // batch rows per CTA (MMA N dimension)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wbuf = smem;
  __half* xs = reinterpret_cast<__half*>(smem + a.stages * kSkStageBytes);  // [MB][x_pitch]
  float* xinv = reinterpret_cast<float*>(xs + MB * a.x_pitch);               // [MB] 2^-scale
  float* recv = xinv + MB;                                                   // [split][128/split][MB]
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(recv + (gridDim.y > 1 ? kSkBN * MB : 0)) + 15) & ~uintptr_t(15));
  uint64_t* empty = full + a.stages;
  uint64_t* recv_bar = empty + a.stages;
  int* err_flag = reinterpret_cast<int*>(recv_bar + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int split = gridDim.y;
  const int kidx = blockIdx.y;
  const uint32_t crank = split > 1 ? cluster_ctarank() : 0u;
  const int rows_per_owner = kSkBN / split;
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
    mbar_init(recv_bar, 1);
    if (split > 1) {
      // The single arrival happens now; the phase completes once every peer's
      // partial sums (split-1 slices) have landed.
      mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((split - 1) * rows_per_owner * MB * 4));
    }
    *err_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (split > 1) cluster_arrive_relaxed();
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
      if (tid == 0 && kidx == 0) record_status(QTTS_ERR_SHAPE);
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
    __syncwarp();
    if (split > 1) cluster_wait();
  } else {
    // ---------------- consumers ----------------
    pdl_wait();
    const int kpad = n_iters * kSkBK;
    // 1) Activation slice [MB, kpad] -> shared memory as raw 16-bit values,
    //    zero padded past K and past the last batch row.
    {
      constexpr int kVec = 8;  // 16-bit elements per 16-byte chunk
      const int per_row = kpad / kVec;
      for (int i = tid; i < MB * per_row; i += kSkConsumerWarps * 32) {
        const int m = i / per_row;
        const int kv = (i - m * per_row) * kVec;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (valid && m < mrows && kv < klen) {
          v = __ldcg(reinterpret_cast<const uint4*>(xg + static_cast<int64_t>(m) * a.ldx + k0 + kv));
        }
        *reinterpret_cast<uint4*>(xs + m * a.x_pitch + kv) = v;
      }
    }
    named_bar_sync(1, kSkConsumerWarps * 32);
    // 2) Per batch row: power-of-two scale that puts max|x| in [2^14, 2^15),
    //    then convert in place to fp16 (exact for all but tiny elements).
    for (int m = warp; m < MB; m += kSkConsumerWarps) {
      uint4* row = reinterpret_cast<uint4*>(xs + m * a.x_pitch);
      const int nvec = kpad / 8;
      float mx = 0.f;
      for (int v = lane; v < nvec; v += 32) {
        const uint4 u = row[v];
        const XT* e = reinterpret_cast<const XT*>(&u);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(to_float(e[j])));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      int sexp = 0;
      if (mx > 0.f) {
        const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFF) - 127;  // floor(log2 mx), normal mx
        sexp = min(max(14 - e, -100), 100);
      }
      const float sc = pow2f(sexp);
      for (int v = lane; v < nvec; v += 32) {
        const uint4 u = row[v];
        const XT* e = reinterpret_cast<const XT*>(&u);
        uint4 o;
        __half* h = reinterpret_cast<__half*>(&o);
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(to_float(e[j]) * sc);
        row[v] = o;
      }
      if (lane == 0) xinv[m] = pow2f(-sexp);
    }
    named_bar_sync(1, kSkConsumerWarps * 32);

    // 3) Main loop.
    const int g = lane >> 2;
    const int q = lane & 3;
    // MMA row g <-> weight row permutation: the rows of one shared-load phase
    // (g = 2p, 2p+1 -> p, p+4) land in opposite 64-byte halves of the span.
    const int pr = (g >> 1) | ((g & 1) << 2);
    const int rowA = warp * 16 + pr;
    const int rowB = rowA + 8;
    const uint32_t wbase = smem_u32(wbuf);
    const uint32_t offA0 = rowA * kSkBK + (((0 * 4 + q) ^ (rowA & 7)) << 4);
    const uint32_t offA1 = rowA * kSkBK + (((1 * 4 + q) ^ (rowA & 7)) << 4);
    const uint32_t offB0 = rowB * kSkBK + (((0 * 4 + q) ^ (rowB & 7)) << 4);
    const uint32_t offB1 = rowB * kSkBK + (((1 * 4 + q) ^ (rowB & 7)) << 4);
    const uint32_t xbase = smem_u32(xs) + (g * a.x_pitch + q * 16) * 2;
    const uint32_t xtile = 8 * a.x_pitch * 2;

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
      const uint4 wa0 = lds128(sb + offA0);
      const uint4 wb0 = lds128(sb + offB0);
      const uint4 wa1 = lds128(sb + offA1);
      const uint4 wb1 = lds128(sb + offB1);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);

      uint32_t A[2][4][4];
      i8x4_to_f16x2x2(wa0.x, A[0][0][0], A[0][0][2]);
      i8x4_to_f16x2x2(wb0.x, A[0][0][1], A[0][0][3]);
      i8x4_to_f16x2x2(wa0.y, A[0][1][0], A[0][1][2]);
      i8x4_to_f16x2x2(wb0.y, A[0][1][1], A[0][1][3]);
      i8x4_to_f16x2x2(wa0.z, A[0][2][0], A[0][2][2]);
      i8x4_to_f16x2x2(wb0.z, A[0][2][1], A[0][2][3]);
      i8x4_to_f16x2x2(wa0.w, A[0][3][0], A[0][3][2]);
      i8x4_to_f16x2x2(wb0.w, A[0][3][1], A[0][3][3]);
      i8x4_to_f16x2x2(wa1.x, A[1][0][0], A[1][0][2]);
      i8x4_to_f16x2x2(wb1.x, A[1][0][1], A[1][0][3]);
      i8x4_to_f16x2x2(wa1.y, A[1][1][0], A[1][1][2]);
      i8x4_to_f16x2x2(wb1.y, A[1][1][1], A[1][1][3]);
      i8x4_to_f16x2x2(wa1.z, A[1][2][0], A[1][2][2]);
      i8x4_to_f16x2x2(wb1.z, A[1][2][1], A[1][2][3]);
      i8x4_to_f16x2x2(wa1.w, A[1][3][0], A[1][3][2]);
      i8x4_to_f16x2x2(wb1.w, A[1][3][1], A[1][3][3]);

      const uint32_t xk = xbase + it * kSkBK * 2;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t xa = xk + t * xtile + h * 64 * 2;
          const uint4 x0 = lds128(xa);
          const uint4 x1 = lds128(xa + 16);
          Mma16816<__half>::run(acc[t], A[h][0], x0.x, x0.y);
          Mma16816<__half>::run(acc[t], A[h][1], x0.z, x0.w);
          Mma16816<__half>::run(acc[t], A[h][2], x1.x, x1.y);
          Mma16816<__half>::run(acc[t], A[h][3], x1.z, x1.w);
        }
      }
    }
    if (!ok) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *reinterpret_cast<volatile int*>(err_flag) = 1;
    }

    // 4) Undo the activation scale; hand the partial sums to their owner.
    float v[MT][4];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int c0 = t * 8 + 2 * q;
      const float i0 = xinv[c0];
      const float i1 = xinv[c0 + 1];
      v[t][0] = acc[t][0] * i0;
      v[t][1] = acc[t][1] * i1;
      v[t][2] = acc[t][2] * i0;
      v[t][3] = acc[t][3] * i1;
    }
    if (split == 1) {
      // This warp owns its 16 rows outright: finish them from registers.
      const bool store = valid && *reinterpret_cast<volatile int*>(err_flag) == 0;
      if (store) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = (e < 2) ? rowA : rowB;
            const int m = t * 8 + 2 * q + (e & 1);
            const int n = n0 + row;
            if (m < mrows && n < a.N) {
              const int64_t ch = static_cast<int64_t>(group) * a.N + n;
              float r = v[t][e] * load_as_float(a.scale, a.scale_dtype, ch);
              if (a.bias != nullptr) r += to_float(static_cast<const XT*>(a.bias)[ch]);
              og[static_cast<int64_t>(m) * a.ldo + n] = from_float<XT>(r);
            }
          }
        }
      }
    } else {
      cluster_wait();  // every peer's receive barrier is initialized
      const int owner = (warp * 16) / rows_per_owner;
      const int lrA = rowA - owner * rows_per_owner;
      const int lrB = rowB - owner * rows_per_owner;
      float* slot = recv + (crank * rows_per_owner) * MB;  // my slice in the owner's buffer
      if (owner == static_cast<int>(crank)) {
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int c0 = t * 8 + 2 * q;
          *reinterpret_cast<float2*>(&slot[lrA * MB + c0]) = make_float2(v[t][0], v[t][1]);
          *reinterpret_cast<float2*>(&slot[lrB * MB + c0]) = make_float2(v[t][2], v[t][3]);
        }
      } else {
        const uint32_t rslot = mapa_shared(smem_u32(slot), owner);
        const uint32_t rbar = mapa_shared(smem_u32(recv_bar), owner);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int c0 = t * 8 + 2 * q;
          st_async_f32x2(rslot + (lrA * MB + c0) * 4, v[t][0], v[t][1], rbar);
          st_async_f32x2(rslot + (lrB * MB + c0) * 4, v[t][2], v[t][3], rbar);
        }
      }
      // 5) Owner: reduce the split partial sums of its rows in rank order.
      named_bar_sync(1, kSkConsumerWarps * 32);
      bool have = mbar_wait_bounded(recv_bar, 0, a.wait_ns);
      if (!have) {
        if (tid == 0) record_status(QTTS_ERR_TIMEOUT);
        // Peers always send; keep this CTA alive until their stores land.
        have = mbar_wait_bounded(recv_bar, 0, 4 * a.wait_ns);
      }
      const bool store = have && valid && *reinterpret_cast<volatile int*>(err_flag) == 0;
      if (store) {
        const int rbase = static_cast<int>(crank) * rows_per_owner;
        for (int i = tid; i < rows_per_owner * mrows; i += kSkConsumerWarps * 32) {
          const int m = i / rows_per_owner;
          const int lr = i - m * rows_per_owner;
          const int n = n0 + rbase + lr;
          if (n < a.N) {
            float r = 0.f;
            for (int p = 0; p < split; ++p) r += recv[(p * rows_per_owner + lr) * MB + m];
            const int64_t ch = static_cast<int64_t>(group) * a.N + n;
            r *= load_as_float(a.scale, a.scale_dtype, ch);
            if (a.bias != nullptr) r += to_float(static_cast<const XT*>(a.bias)[ch]);
            og[static_cast<int64_t>(m) * a.ldo + n] = from_float<XT>(r);
          }
        }
      }
    }
  }

  // Error path: make sure no copy of ours is still landing in shared memory.
  if (warp == kSkConsumerWarps && lane == 0 && *reinterpret_cast<volatile int*>(err_flag) != 0) {
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

size_t skinny_smem(int mb, int x_pitch, int stages, int split) {
  const size_t xbytes = static_cast<size_t>(mb) * x_pitch * 2 + mb * 4;
  const size_t recv = split > 1 ? static_cast<size_t>(kSkBN) * mb * 4 : 0;
  return 1024 + static_cast<size_t>(stages) * kSkStageBytes + xbytes + recv + 16 + 16 * stages + 32;
}

}  // namespace

SkinnyPlan plan_skinny(int M, int N, int K, int G, int split_req) {
  SkinnyPlan p{};
  p.mt = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
  const int mb = p.mt * 8;
  p.m_chunks = (M + mb - 1) / mb;
  const int n_tiles = (N + kSkBN - 1) / kSkBN;
  const int ctas_base = n_tiles * G * p.m_chunks;
  auto kpc_for = [&](int split) { return ((K + split - 1) / split + kSkBK - 1) / kSkBK * kSkBK; };
  int split = split_req;
  if (split == 0) {
    // Smallest split that puts a CTA on (most of) the 148 SMs while the
    // activation slice stays within 48 KiB of shared memory; the largest
    // otherwise.
    split = 8;
    for (int s = 1; s <= 8; s *= 2) {
      const size_t xb = static_cast<size_t>(mb) * (kpc_for(s) + 8) * 2;
      if (xb <= 48 * 1024 && ctas_base * s >= 120) {
        split = s;
        break;
      }
    }
  }
  p.split = split;
  p.k_per_cta = kpc_for(split);
  p.x_pitch = p.k_per_cta + 8;  // +16 bytes: rows of one LDS phase hit distinct banks
  const int n_iters = p.k_per_cta / kSkBK;
  // Stage ring: fill a ~100 KiB budget (so the next kernel's CTA fits beside
  // this one under programmatic dependent launch), 2..6 stages, never more
  // than the slice needs.
  const size_t fixed = skinny_smem(mb, p.x_pitch, 0, split);
  const size_t budget = 100 * 1024;
  int stages = fixed < budget ? static_cast<int>((budget - fixed) / kSkStageBytes) : 0;
  stages = stages > 6 ? 6 : stages;
  stages = stages < n_iters ? stages : n_iters;
  stages = stages < 2 ? 2 : stages;
  p.stages = stages;
  p.smem = skinny_smem(mb, p.x_pitch, stages, split);
  p.grid = dim3(n_tiles, split, G * p.m_chunks);
  return p;
}

int launch_skinny_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, int x_dtype,
                        bool pdl, cudaStream_t stream) {
  if (p.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
  if (x_dtype == QTTS_BF16) return launch_skinny_mt<__nv_bfloat16>(p.mt, map, args, p.grid, p.split, p.smem, pdl, stream);
  if (x_dtype == QTTS_FP16) return launch_skinny_mt<__half>(p.mt, map, args, p.grid, p.split, p.smem, pdl, stream);
  return QTTS_ERR_DTYPE;
}

}  // namespace qtts
