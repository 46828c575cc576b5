// fp8-e4m3 (and int8) W8A8 GEMM on the 5th-generation tensor cores.
//
// Replaces torch._scaled_mm in Fp8Method.apply (qtts/quant/fp8.py:79-88):
//   out[m, n] = cast( (sum_k xq[m,k] * wq[n,k]) * scale_x[m] * scale_w[n] + bias[n] )
// with e4m3 operands, fp32 accumulation, and the row/column scales (and the
// bias the reference adds afterwards) applied once in the epilogue.
//
// Both operands are e4m3 in memory, so nothing is converted on the way: the
// producer warp streams 128 weight rows x 128 k (16 KiB) per stage and the
// matching activation tile [NB rows x 128 k] with 2-D TMA (128-byte swizzle)
// straight into the K-major shared-memory layout tcgen05 reads. The weight
// stream starts before the programmatic-dependent-launch wait (weights are
// constant); the activation tiles -- written by the quantization kernel that
// precedes this one -- after it. Two threads issue tcgen05.mma kind::f8f6f4
// (M = 128 weight rows, N = NB batch columns, K = 32 per instruction; 4096
// weights per instruction), each the MMAs of one 64-k half of every stage into
// its own fp32 accumulator in tensor memory, and release each stage with
// tcgen05.commit. Four epilogue warps read both accumulators with tcgen05.ld
// (one row per thread) and add them. K can be split over a cluster of up to 4
// CTAs whose partial sums reach the row owner by st.async. All waits are
// bounded; tensor memory is always freed.
//
// The same kernel with I8 = true is the int8 W8A8 GEMM of Int8Method
// (qtts/quant/int8.py:120-155, which uses torch._int_mm): tcgen05.mma kind::i8
// on signed int8 operands with an exact int32 accumulator, the split-K
// partials added as int32, and the epilogue (float(acc) * scale_x) * scale_w +
// bias in the reference's order.
#include "common.cuh"
#include "kernels.h"

namespace qtts {

constexpr int kF8StageW = 16384;  // 128 rows x 128 k e4m3
constexpr int kF8EpiWarps = 4;
constexpr int kF8ProducerWarp = 4;
constexpr int kF8MmaWarp = 5;   // issues the first 64-k half of every stage into accumulator 0
constexpr int kF8MmaWarp2 = 6;  // the second half into accumulator 1 (added in the epilogue)
constexpr int kF8Threads = 7 * 32;

template <int N>
__device__ __forceinline__ void f8_tmem_ld(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void f8_tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Epilogue value of one accumulator word, before the final cast to OT.
// e4m3 (I8 false, Fp8Method, qtts/quant/fp8.py:79-88): the fp32 sum scaled,
// rounded to the output dtype as _scaled_mm(out_dtype=x.dtype) returns it, and
// the bias then added as torch adds two tensors of that dtype (in fp32, one
// rounding by the caller's cast). int8 (I8 true, Int8Method,
// qtts/quant/int8.py:148-153): the int32 sum converted and scaled in the
// reference's order and roundings, ((float(acc) * sx) * sw) + bias in fp32, no
// fused multiply-add.
template <bool I8, typename OT>
__device__ __forceinline__ float w8a8_out(uint32_t acc_bits, float sx, float sw, float bias, bool has_bias) {
  if (I8) {
    float y = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(acc_bits)), sx), sw);
    return has_bias ? __fadd_rn(y, bias) : y;
  }
  const float y = __uint_as_float(acc_bits) * sx * sw;
  return has_bias ? __fadd_rn(to_float(from_float<OT>(y)), bias) : y;
}

template <int NB, typename OT, bool I8 = false>
__global__ void __launch_bounds__(kF8Threads, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                    const Fp8Args a) {
  constexpr int XS = NB * 128;  // activation tile bytes per 128-k stage
  // TMEM: two fp32 accumulators of NB columns, allocated as a power of two >= 32.
  constexpr uint32_t kCols = 2 * NB < 32 ? 32 : 2 * NB;
  constexpr uint32_t kIdesc = I8 ? umma_idesc_i8(128, NB) : umma_idesc(0u /*E4M3*/, 0u /*E4M3*/, 128, NB);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int split = gridDim.y;
  const int S = a.stages;
  uint8_t* wbuf = smem;
  uint8_t* xbuf = wbuf + S * kF8StageW;
  float* recv = reinterpret_cast<float*>(xbuf + S * XS);  // [split][128/split][NB] when split > 1
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(recv + (split > 1 ? 128 * NB : 0)) + 15) & ~uintptr_t(15));
  uint64_t* wfull = bars;
  uint64_t* xfull = wfull + S;
  uint64_t* sempty = xfull + S;
  uint64_t* dfull = sempty + S;
  uint64_t* recv_bar = dfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  int* err_flag = reinterpret_cast<int*>(tmem_slot + 1);
  // The tile's activation row scales, staged once by the epilogue warps and
  // read into registers a group at a time ahead of the group's output stores.
  float* sx_s = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(err_flag + 2) + 15) & ~uintptr_t(15));

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int kidx = blockIdx.y;
  const uint32_t crank = split > 1 ? cluster_ctarank() : 0u;
  const int rpo = 128 / split;
  const int n0 = blockIdx.x * 128;
  const int m0 = blockIdx.z * NB;
  const int k0 = kidx * a.k_per_cta;
  const int klen = max(0, min(a.K - k0, a.k_per_cta));
  const int n_iters = (klen + 127) / 128;
  const int mrows = min(NB, a.M - m0);

  if (tid == 0) {
    QTTS_TRACE_STAMP(0);
    for (int s = 0; s < S; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&xfull[s], 1);
      mbar_init(&sempty[s], 2);  // one commit from each MMA issuer
    }
    mbar_init(dfull, 2);
    mbar_init(recv_bar, 1);
    if (split > 1) mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((split - 1) * rpo * NB * 4));
    err_flag[0] = 0;
    fence_mbarrier_init();
  }
  if (warp == kF8MmaWarp) {
    tmem_alloc(tmem_slot, kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  if (split > 1) cluster_arrive_relaxed();
  pdl_launch_dependents();
  volatile int* verr = err_flag;

  int w_issued = 0, x_issued = 0;
  if (warp == kF8ProducerWarp) {
    if (lane == 0 && n_iters > 0) {
      tma_prefetch_desc(&wmap);
      tma_prefetch_desc(&xmap);
      const int pre = min(S, n_iters);
      for (int it = 0; it < pre; ++it) {
        mbar_arrive_expect_tx(&wfull[it], kF8StageW);
        tma_load_2d(wbuf + it * kF8StageW, &wmap, k0 + it * 128, n0, &wfull[it]);
      }
      w_issued = pre;
      pdl_wait();
      QTTS_TRACE_STAMP(1);
      for (int it = 0; it < n_iters; ++it) {
        const int s = it % S;
        if (it >= S) {
          if (!mbar_wait_bounded(&sempty[s], ((it / S) - 1) & 1, a.wait_ns)) {
            record_status(QTTS_ERR_TIMEOUT);
            *verr = 1;
            break;
          }
          QTTS_TRACE_DETAIL(2, it);
          mbar_arrive_expect_tx(&wfull[s], kF8StageW);
          tma_load_2d(wbuf + s * kF8StageW, &wmap, k0 + it * 128, n0, &wfull[s]);
          w_issued = it + 1;
        }
        mbar_arrive_expect_tx(&xfull[s], XS);
        tma_load_2d(xbuf + s * XS, &xmap, k0 + it * 128, m0, &xfull[s]);
        x_issued = it + 1;
      }
    }
    __syncwarp();
  } else if (warp == kF8MmaWarp || warp == kF8MmaWarp2) {
    // Two issuing threads, one per 64-k half of every stage, each into its own
    // accumulator: a single issuer that commits to release its stages measured
    // ~60-90 cycles per instruction, two measured ~32.
    if (lane == 0) {
      const int h = warp - kF8MmaWarp;
      const uint32_t dcol = tmem + static_cast<uint32_t>(h * NB);
      const uint32_t waddr = smem_u32(wbuf);
      const uint32_t xaddr = smem_u32(xbuf);
      bool ok = true;
      for (int it = 0; ok && it < n_iters; ++it) {
        const int s = it % S;
        const uint32_t ph = (it / S) & 1;
        if (!mbar_wait_bounded(&wfull[s], ph, a.wait_ns)) {
          ok = false;
          break;
        }
        if (h == 0) QTTS_TRACE_DETAIL(3, it);
        if (!mbar_wait_bounded(&xfull[s], ph, a.wait_ns)) {
          ok = false;
          break;
        }
        if (h == 0) QTTS_TRACE_DETAIL(0, it);
        tc_fence_after();
#pragma unroll
        for (int i = 2 * h; i < 2 * h + 2; ++i) {
          const uint64_t adesc = smem_desc_k_sw128(waddr + s * kF8StageW + i * 32);
          const uint64_t bdesc = smem_desc_k_sw128(xaddr + s * XS + i * 32);
          const uint32_t acc = (it != 0 || i != 2 * h) ? 1u : 0u;
          if (I8) {
            umma_i8_ss(dcol, adesc, bdesc, kIdesc, acc);
          } else {
            umma_f8_ss(dcol, adesc, bdesc, kIdesc, acc);
          }
        }
        tc_commit(&sempty[s]);
        if (h == 0) QTTS_TRACE_DETAIL(1, it);
      }
      if (!ok) {
        record_status(QTTS_ERR_TIMEOUT);
        *verr = 1;
      }
      if (h == 0) QTTS_TRACE_STAMP(2);
      tc_commit(dfull);  // arrives once every MMA this thread issued has completed
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps 0..3: one accumulator row per thread ----------------
    pdl_wait();
    if (tid == 0) QTTS_TRACE_STAMP(5);
    const int row = warp * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    for (int c = tid; c < NB; c += kF8EpiWarps * 32) sx_s[c] = (m0 + c < a.M) ? a.scale_x[m0 + c] : 0.f;
    named_bar_sync(1, kF8EpiWarps * 32);
    const bool dready = mbar_wait_bounded(dfull, 0, a.wait_ns);
    if (tid == 0) QTTS_TRACE_STAMP(6);
    if (!dready) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *verr = 1;
    }
    tc_fence_after();
    const bool cta_err = *verr != 0;
    const int n = n0 + row;
    float sw = 0.f, bias = 0.f;
    if (split == 1 && n < a.N) {
      sw = a.scale_w[n];
      if (a.bias != nullptr) bias = to_float(static_cast<const OT*>(a.bias)[n]);
    }
    OT* og = static_cast<OT*>(a.out) + static_cast<int64_t>(m0) * a.ldo;
    // Accumulator columns 16 at a time (one TMEM load and wait per group).
    constexpr int kGrp = 16;
#pragma unroll 1
    for (int g0 = 0; g0 < NB; g0 += kGrp) {
    uint32_t dg[kGrp], dh[kGrp];
    f8_tmem_ld<16>(tmem + lane_base + g0, dg);
    f8_tmem_ld<16>(tmem + lane_base + NB + g0, dh);
    tc_wait_ld();
    if (tid == 0) QTTS_TRACE_DETAIL(4, g0 / kGrp);
    // The loaded registers are only valid after the wait: tie them to it so no
    // use is scheduled above it.
#pragma unroll
    for (int q = 0; q < kGrp; ++q) asm volatile("" : "+r"(dg[q]), "+r"(dh[q]));
    // The two issuers' accumulators: exact int32 adds (I8) or one fp32 add.
#pragma unroll
    for (int q = 0; q < kGrp; ++q)
      dg[q] = I8 ? static_cast<uint32_t>(static_cast<int>(dg[q]) + static_cast<int>(dh[q]))
                 : __float_as_uint(__uint_as_float(dg[q]) + __uint_as_float(dh[q]));
    {
      const int c0 = g0;
      // The group's activation scales into registers before any output store:
      // read between stores, each load waited for the previous store (the
      // compiler cannot tell the output from the scales apart), a serial
      // chain of load latencies.
      float sxv[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 t = lds128(smem_u32(sx_s + c0 + 4 * q));
        sxv[4 * q] = __uint_as_float(t.x);
        sxv[4 * q + 1] = __uint_as_float(t.y);
        sxv[4 * q + 2] = __uint_as_float(t.z);
        sxv[4 * q + 3] = __uint_as_float(t.w);
      }
      // Raw accumulator words (fp32 bits, or int32 for I8; zero either way).
      uint32_t v[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) v[c] = (n_iters > 0 && !cta_err) ? dg[c0 - g0 + c] : 0u;
      if (split == 1) {
        if (!cta_err && n < a.N) {
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int col = c0 + c;
            if (col < mrows) {
              og[static_cast<int64_t>(col) * a.ldo + n] =
                  from_float<OT>(w8a8_out<I8, OT>(v[c], sxv[c], sw, bias, a.bias != nullptr));
            }
          }
        }
      } else {
        if (c0 == 0) cluster_wait();
        const int owner = row / rpo;
        const int lr = row - owner * rpo;
        const int rrow = static_cast<int>(crank) * rpo + lr;
        if (owner == static_cast<int>(crank)) {
#pragma unroll
          for (int c = 0; c < 16; c += 4)
            *reinterpret_cast<uint4*>(recv + recv_offset(rrow, (c0 + c) >> 2, NB)) =
                make_uint4(v[c], v[c + 1], v[c + 2], v[c + 3]);
        } else {
          const uint32_t rbar = mapa_shared(smem_u32(recv_bar), owner);
#pragma unroll
          for (int c = 0; c < 16; c += 4) {
            const uint32_t rdst = mapa_shared(smem_u32(recv + recv_offset(rrow, (c0 + c) >> 2, NB)), owner);
            st_async_f32x4(rdst, __uint_as_float(v[c]), __uint_as_float(v[c + 1]), __uint_as_float(v[c + 2]),
                           __uint_as_float(v[c + 3]), rbar);
          }
        }
      }
    }
    if (tid == 0) QTTS_TRACE_DETAIL(5, g0 / kGrp);
    }
    if (split > 1) {
      named_bar_sync(1, kF8EpiWarps * 32);
      bool have = mbar_wait_bounded(recv_bar, 0, a.wait_ns);
      if (!have) {
        if (tid == 0) record_status(QTTS_ERR_TIMEOUT);
        have = mbar_wait_bounded(recv_bar, 0, 4 * a.wait_ns);  // peers always send
      }
      if (have && !cta_err) {
        // Thread = (owned row, 4 batch columns): one 16-byte load per peer.
        const int rbase = static_cast<int>(crank) * rpo;
        const int quads = (mrows + 3) / 4;
        for (int i = tid; i < rpo * quads; i += kF8EpiWarps * 32) {
          const int mq = i / rpo;
          const int lr = i - mq * rpo;
          const int nn = n0 + rbase + lr;
          if (nn < a.N) {
            // Partial sums in rank order: fp32 adds, or exact int32 adds (I8).
            uint32_t rv[4] = {0u, 0u, 0u, 0u};
            for (int p = 0; p < split; ++p) {
              const uint4 t = *reinterpret_cast<const uint4*>(recv + recv_offset(p * rpo + lr, mq, NB));
              const uint32_t tv[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                rv[q] = I8 ? static_cast<uint32_t>(static_cast<int>(rv[q]) + static_cast<int>(tv[q]))
                           : __float_as_uint(__uint_as_float(rv[q]) + __uint_as_float(tv[q]));
              }
            }
            const float sw = a.scale_w[nn];
            const float bias = a.bias != nullptr ? to_float(static_cast<const OT*>(a.bias)[nn]) : 0.f;
            float sxq[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) sxq[q] = sx_s[min(4 * mq + q, NB - 1)];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int m = 4 * mq + q;
              if (m < mrows)
                og[static_cast<int64_t>(m) * a.ldo + nn] =
                    from_float<OT>(w8a8_out<I8, OT>(rv[q], sxq[q], sw, bias, a.bias != nullptr));
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (tid == 0) QTTS_TRACE_STAMP(7);
  if (warp == kF8MmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
  if (split > 1 && (warp == kF8ProducerWarp || warp == kF8MmaWarp || warp == kF8MmaWarp2)) cluster_wait();
  if (warp == kF8ProducerWarp && lane == 0 && *verr != 0) {
    for (int s = 0; s < S && s < w_issued; ++s) {
      const int last = ((w_issued - 1 - s) / S) * S + s;
      mbar_wait_bounded(&wfull[s], (last / S) & 1, a.wait_ns);
    }
    for (int s = 0; s < S && s < x_issued; ++s) {
      const int last = ((x_issued - 1 - s) / S) * S + s;
      mbar_wait_bounded(&xfull[s], (last / S) & 1, a.wait_ns);
    }
  }
}

namespace {

template <int NB, typename OT, bool I8>
int launch_fp8_t(const CUtensorMap& wmap, const CUtensorMap& xmap, const Fp8Args& args, const Fp8Plan& p,
                 bool pdl, cudaStream_t stream) {
  auto kern = fp8_gemm_kernel<NB, OT, I8>;
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
  cfg.gridDim = p.grid;
  cfg.blockDim = dim3(kF8Threads, 1, 1);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (p.split > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = p.split;
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
  return cudaLaunchKernelEx(&cfg, kern, wmap, xmap, args) == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

template <typename OT, bool I8>
int launch_fp8_nb(const CUtensorMap& wmap, const CUtensorMap& xmap, const Fp8Args& args, const Fp8Plan& p, bool pdl,
                  cudaStream_t stream) {
  switch (p.nb) {
    case 16:
      return launch_fp8_t<16, OT, I8>(wmap, xmap, args, p, pdl, stream);
    case 32:
      return launch_fp8_t<32, OT, I8>(wmap, xmap, args, p, pdl, stream);
    case 64:
      return launch_fp8_t<64, OT, I8>(wmap, xmap, args, p, pdl, stream);
    default:
      return launch_fp8_t<128, OT, I8>(wmap, xmap, args, p, pdl, stream);
  }
}

template <bool I8>
int launch_w8a8_out(const CUtensorMap& wmap, const CUtensorMap& xmap, const Fp8Args& args, const Fp8Plan& p,
                    int out_dtype, bool pdl, cudaStream_t stream) {
  switch (out_dtype) {
    case QTTS_BF16:
      return launch_fp8_nb<__nv_bfloat16, I8>(wmap, xmap, args, p, pdl, stream);
    case QTTS_FP16:
      return launch_fp8_nb<__half, I8>(wmap, xmap, args, p, pdl, stream);
    default:
      return launch_fp8_nb<float, I8>(wmap, xmap, args, p, pdl, stream);
  }
}

size_t fp8_smem(int nb, int stages, int split) {
  return 1024 + static_cast<size_t>(stages) * (kF8StageW + static_cast<size_t>(nb) * 128) +
         (split > 1 ? static_cast<size_t>(128) * nb * 4 : 0) + 16 + 24 * stages + 16 + 32 + 16 +
         static_cast<size_t>(nb) * 4;
}

}  // namespace

Fp8Plan plan_fp8(int M, int N, int K, int split_req) {
  Fp8Plan p{};
  p.nb = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
  const int m_chunks = (M + p.nb - 1) / p.nb;
  const int n_tiles = (N + 127) / 128;
  int split = split_req;
  if (split == 0) {
    // One CTA per SM at most (each MMA instruction is the unit of tensor
    // work), K split within 4 CTAs: a narrow weight (32 row tiles) otherwise
    // leaves most SMs idle, and the partial-sum exchange is cheap.
    split = 1;
    for (int s = 1; s <= 4; s *= 2) {
      if (n_tiles * m_chunks * s <= kNumSMs) split = s;
    }
  }
  p.split = split;
  p.k_per_cta = ((K + split - 1) / split + 127) / 128 * 128;
  const int n_iters = p.k_per_cta / 128;
  // Stage ring as deep as shared memory allows: after the dependency wait a
  // CTA streams at (bytes in flight) / (memory latency), and the grid is at
  // most one CTA per SM.
  const size_t fixed = fp8_smem(p.nb, 0, split);
  const size_t budget = 200 * 1024;
  int stages = fixed < budget ? static_cast<int>((budget - fixed) / (kF8StageW + p.nb * 128)) : 0;
  stages = stages > 12 ? 12 : stages;
  stages = stages < n_iters ? stages : n_iters;
  stages = stages < 2 ? 2 : stages;
  p.stages = stages;
  p.smem = fp8_smem(p.nb, stages, split);
  p.grid = dim3(n_tiles, split, m_chunks);
  return p;
}

int launch_fp8_gemm(const Fp8Plan& p, const CUtensorMap& wmap, const CUtensorMap& xmap, const Fp8Args& args,
                    int out_dtype, bool pdl, cudaStream_t stream, bool int8) {
  if (p.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
  return int8 ? launch_w8a8_out<true>(wmap, xmap, args, p, out_dtype, pdl, stream)
              : launch_w8a8_out<false>(wmap, xmap, args, p, out_dtype, pdl, stream);
}

}  // namespace qtts
