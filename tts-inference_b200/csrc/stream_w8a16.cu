// Weight-streaming int8 weight-only GEMM (W8A16) for decode batches, M <= 16.
//
// Replaces the Triton kernel _w8_gemm_kernel (qtts/quant/kernels.py:89-135):
//   out[m, n] = cast( sum_k x[m, k] * w[n, k] * scale[n] + bias[n] )
// with fp32 accumulation and the per-output-channel scale applied once after
// the K loop (kernels.py:123, 129-130).
//
// Design (B200, sm_100a). In a decode step each linear waits for the previous
// one, so a call costs (dependency gap) + (activation fetch) + (work that can
// only start once the activations are known) + (epilogue). The weights do not
// depend on the previous kernel: a producer warp streams them into shared
// memory before the programmatic-dependent-launch wait, so by the time the
// activations arrive most of a CTA's weight slice is already on chip. What is
// left is made short:
//   * One CTA owns BN = 16*R output rows over the whole of K, so partial sums
//     meet in shared memory; no split-K across CTAs, no cluster exchange. R is
//     picked so that about one CTA lands on each of the 148 SMs.
//   * 12 consumer warps = R row groups x KG k groups (R * KG = 12). A stage is
//     KG TMA boxes of [BN rows x 128 B] (128-byte swizzle), 24 KiB; warp
//     (rg, kg) owns rows rg*16..+16 of box kg. 416 threads and <= 110 KiB of
//     shared memory, so the next kernel's CTA fits beside this one.
//   * Dequantization is one byte-permute per two weights: with u = b ^ 0x80,
//     the fp16 with bit pattern 0x64uu is 1024 + u = 1152 + b, exactly. The
//     1152 is not subtracted per weight; the kernel subtracts 1152 * sum_k x[m,
//     k] once per output instead (the activation row sums are formed while
//     staging, per warp and then over warps in a fixed order). mma.sync m16n8k16 with the weights as
//     the 16-row operand and the batch as the 8-column operand; four
//     independent accumulator chains per warp hide the MMA latency.
//   * Activations: only the M real rows are staged, converted to fp16 with a
//     per-row power of two (exact for every element within 2^28 of the row's
//     largest magnitude), with warp-level reductions before the few shared
//     atomics.
//   * Optional activation prologue (template PRO, csrc/prologue.cuh): SiLU·up
//     of [gate | up] rows, applied to each chunk as it is loaded, or RMSNorm,
//     whose row factors come from the staged rows themselves (K a multiple of
//     256) or from one more load of the rows by all warps.
//   * Every wait is bounded (globaltimer); on expiry the kernel records
//     QTTS_ERR_TIMEOUT, skips its stores and drains its own copies in flight.
#include "common.cuh"
#include "kernels.h"
#include "prologue.cuh"

namespace qtts {

constexpr int kStConsumerWarps = 12;
constexpr int kStThreads = (kStConsumerWarps + 1) * 32;
constexpr int kStStageBytes = kStConsumerWarps * 16 * 128;  // 24 KiB
constexpr float kStBias = 1152.0f;

namespace {

__device__ __forceinline__ float pow2f_st(int e) { return __int_as_float((e + 127) << 23); }

// Scale exponent that puts a row maximum `mx` (> 0) just below 2^15.
__device__ __forceinline__ int row_exponent(float mx) {
  if (!(mx > 0.f)) return 0;
  const int e = static_cast<int>((__float_as_uint(mx) >> 23) & 0xFF) - 127;
  return min(max(14 - e, -100), 100);
}

// fp16 pairs (1152 + b0, 1152 + b1), (1152 + b2, 1152 + b3) of four int8 weights.
__device__ __forceinline__ void i8x4_to_f16_biased(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  lo = __byte_perm(u, 0x64646464u, 0x5140);
  hi = __byte_perm(u, 0x64646464u, 0x7362);
}

// D += A x B, m16n8k16 fp16 -> fp32; a pure register operation.
__device__ __forceinline__ void hmma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Sum over the warp in a fixed butterfly order (every lane gets the result).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename XT>
__device__ __forceinline__ uint4 load_x_chunk(const XT* xg, int64_t ldx, int m, int kv, bool load) {
  if (!load) return make_uint4(0u, 0u, 0u, 0u);
  return __ldcg(reinterpret_cast<const uint4*>(xg + static_cast<int64_t>(m) * ldx + kv));
}

template <typename XT>
__device__ __forceinline__ unsigned chunk_absmax(const uint4& u) {
  const XT* e = reinterpret_cast<const XT*>(&u);
  float mx = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) mx = fmaxf(mx, fabsf(to_float(e[q])));
  return __float_as_uint(mx);
}

// Writes the fp16 image of eight activations scaled by the row's power of two
// and returns the sum of the eight scaled values.
template <typename XT>
__device__ __forceinline__ float convert_x_chunk(const uint4& u, unsigned row_max, __half* dst) {
  const float sc = pow2f_st(row_exponent(__uint_as_float(row_max)));
  const XT* e = reinterpret_cast<const XT*>(&u);
  uint4 o;
  __half2* h = reinterpret_cast<__half2*>(&o);
  float sum = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    h[q] = __floats2half2_rn(to_float(e[2 * q]) * sc, to_float(e[2 * q + 1]) * sc);
    sum += __low2float(h[q]);
    sum += __high2float(h[q]);
  }
  *reinterpret_cast<uint4*>(dst) = o;
  return sum;
}

}  // namespace

template <int MT, int R, typename XT, int PRO = kProNone>
__global__ void __launch_bounds__(kStThreads, 2)
    stream_w8a16_kernel(const __grid_constant__ CUtensorMap wmap, const SkinnyArgs a) {
  constexpr int KG = kStConsumerWarps / R;  // k groups
  constexpr int BN = 16 * R;                // weight rows per CTA
  constexpr int SW = 128 * KG;              // k per stage
  constexpr int MB = 8 * MT;                // batch rows per CTA
  constexpr int NACC = 4;
  constexpr int NT = kStConsumerWarps * 32;
  static_assert(R * KG == kStConsumerWarps, "row groups x k groups must use every consumer warp");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wbuf = smem;
  // Staged activations: only min(M, MB) rows are ever real, so only those are allocated.
  const int xrows = min(MB, a.M);
  __half* xs = reinterpret_cast<__half*>(smem + a.stages * kStStageBytes);  // [xrows][x_pitch]
  float* xpart = reinterpret_cast<float*>(xs + xrows * a.x_pitch);  // [warp][MB] partial row sums
  unsigned* xmax = reinterpret_cast<unsigned*>(xpart + kStConsumerWarps * MB);  // [MB] float bits
  float* rinv = reinterpret_cast<float*>(xmax + MB);                             // [MB] RMSNorm factors
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(rinv + MB) + 15) & ~uintptr_t(15));
  uint64_t* empty = full + a.stages;
  int* err_flag = reinterpret_cast<int*>(empty + a.stages);
  // RMSNorm prologue: [MB][K / 256] group sums (the launch adds MB * 128 bytes).
  float* ngs = reinterpret_cast<float*>(err_flag + 4);
  float* red = reinterpret_cast<float*>(wbuf);  // [KG][BN][MB], reuses the ring after the loop

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int n0 = blockIdx.x * BN;
  const int mchunk = blockIdx.z % a.m_chunks;
  int group = blockIdx.z / a.m_chunks;
  const int m0 = mchunk * MB;
  int n_iters = (a.K + SW - 1) / SW;

  if (tid == 0) {
    QTTS_TRACE_STAMP(0);
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStConsumerWarps);
    }
    for (int i = 0; i < kStConsumerWarps * MB; ++i) xpart[i] = 0.f;
    for (int i = 0; i < MB; ++i) xmax[i] = 0u;
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
      if (tid == 0 && blockIdx.x == 0) record_status(QTTS_ERR_SHAPE);
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
  if (warp == kStConsumerWarps) {
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
        mbar_arrive_expect_tx(&full[s], kStStageBytes);
        uint8_t* dst = wbuf + s * kStStageBytes;
#pragma unroll
        for (int c = 0; c < KG; ++c) {
          tma_load_2d(dst + c * BN * 128, &wmap, it * SW + c * 128, static_cast<int>(wrow0), &full[s]);
        }
        n_issued = it + 1;
        if (it == 0) QTTS_TRACE_STAMP(1);
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    // The scale and bias of the output channel this thread finishes (the
    // epilogue gives thread t row t mod BN, and BN divides NT) are constants of
    // the layer: loaded before the dependency wait.
    float pre_sc = 0.f, pre_bias = 0.f;
    if (valid && n0 + tid % BN < a.N) {
      const int64_t ch = static_cast<int64_t>(group) * a.N + n0 + tid % BN;
      pre_sc = load_as_float(a.scale, a.scale_dtype, ch);
      if (a.bias != nullptr) pre_bias = to_float(static_cast<const XT*>(a.bias)[ch]);
    }
    pdl_wait();
    if (tid == 0) QTTS_TRACE_STAMP(2);
    // Staged activation extent: K rounded up to whole 128-wide boxes (zeros
    // past K); boxes that start at or past K are skipped by the main loop.
    const int kstage = (a.K + 127) / 128 * 128;
    const int cpr = kstage / 8;  // 16-byte chunks per staged row
    const int total = valid ? mrows * cpr : 0;
    const int nj = (total + NT - 1) / NT;
    // When a row holds a multiple of 32 chunks, the 32 chunks a warp handles
    // in one step always lie in one row: the row reductions are warp-wide.
    const bool uniform_rows = cpr % 32 == 0;
    constexpr int kBatch = 4;
    const bool in_regs = nj <= kBatch;
    uint4 held[kBatch];
    const XT* wnorm = static_cast<const XT*>(a.pro_weight);
    bool normalized = false;  // held[] already holds normalized chunks
    if constexpr (PRO == kProRmsNorm) {
      // The whole of K is staged here and, with K a multiple of 256, a warp's
      // 32 consecutive chunks are one group of the norm's fixed order: the
      // group sums come from the raw chunks as they are loaded (norm weights
      // alongside), the factors from the group sums, then the chunks held in
      // registers are normalized; past one batch the staging below reloads
      // and normalizes them.
      const int groups = a.K >> 8;
      uint4 heldw[kBatch];
      for (int j0 = 0; j0 < nj; j0 += kBatch) {
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int ci = tid + NT * (j0 + b);
          const bool act = j0 + b < nj && ci < total;
          const int m = act ? ci / cpr : 0;
          const int kv = act ? (ci - m * cpr) * 8 : 0;
          held[b] = load_x_chunk<XT>(xg, a.ldx, m, kv, act && kv < a.K);
          heldw[b] = (in_regs && act && kv < a.K) ? __ldg(reinterpret_cast<const uint4*>(wnorm + kv))
                                                  : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int ci = tid + NT * (j0 + b);
          if (j0 + b < nj && ci < total) {  // warp-uniform: total is a multiple of 32
            const int m = ci / cpr;
            const int kv = (ci - m * cpr) * 8;
            const XT* e = reinterpret_cast<const XT*>(&held[b]);
            float v[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) v[q] = to_float(e[q]);
            const float gsum = group_butterfly(leaf_sumsq(v));
            if (lane == 0) ngs[m * groups + (kv >> 8)] = gsum;
          }
        }
      }
      named_bar_sync(1, NT);
      for (int m = warp; m < mrows; m += kStConsumerWarps) {
        const float ssq = lanes_stride_tree(lane < groups ? ngs[m * groups + lane] : 0.f, groups);
        if (lane == 0) rinv[m] = rms_inv(ssq, a.K, a.pro_eps);
      }
      named_bar_sync(1, NT);
      if (in_regs) {
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int ci = tid + NT * b;
          const bool act = b < nj && ci < total;
          const int m = act ? ci / cpr : 0;
          const int kv = act ? (ci - m * cpr) * 8 : 0;
          if (act && kv < a.K) held[b] = normalize_chunk<XT>(held[b], heldw[b], rinv[m]);
        }
        normalized = true;
      }
    } else if constexpr (PRO == kProRmsNormRows) {
      // The norm's factor of each real row before any chunk is staged. When the
      // rows fit in registers their raw chunks and norm weights are loaded
      // first, so those loads overlap the norm's; the factors' scratch aliases
      // the (not yet written) staged rows.
      uint4 heldw[kBatch];
      if (in_regs) {
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int ci = tid + NT * b;
          const bool act = b < nj && ci < total;
          const int m = act ? ci / cpr : 0;
          const int kv = act ? (ci - m * cpr) * 8 : 0;
          held[b] = load_x_chunk<XT>(xg, a.ldx, m, kv, act && kv < a.K);
          heldw[b] = (act && kv < a.K) ? __ldg(reinterpret_cast<const uint4*>(wnorm + kv)) : make_uint4(0u, 0u, 0u, 0u);
        }
      }
      cta_norm_factors<XT>(xg, a.ldx, valid ? mrows : 0, a.K, a.pro_eps, reinterpret_cast<float*>(xs), rinv, warp,
                           lane, kStConsumerWarps, 1);
      if (in_regs) {
#pragma unroll
        for (int b = 0; b < kBatch; ++b) {
          const int ci = tid + NT * b;
          const bool act = b < nj && ci < total;
          const int m = act ? ci / cpr : 0;
          const int kv = act ? (ci - m * cpr) * 8 : 0;
          if (act && kv < a.K) held[b] = normalize_chunk<XT>(held[b], heldw[b], rinv[m]);
        }
        normalized = true;
      }
    }
    // 1) Load the real rows (a thread's chunks of one batch in flight at
    //    once), per-row maximum. Past one batch, raw chunks are parked in
    //    shared memory until the maximum is known.
    for (int j0 = 0; j0 < nj; j0 += kBatch) {
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int ci = tid + NT * (j0 + b);
        const bool act = j0 + b < nj && ci < total;
        const int m = act ? ci / cpr : 0;
        const int kv = act ? (ci - m * cpr) * 8 : 0;
        if (PRO == kProNone) {
          held[b] = load_x_chunk<XT>(xg, a.ldx, m, kv, act && kv < a.K);
        } else if (normalized) {
          // loaded and normalized above
        } else {
          held[b] = (act && kv < a.K) ? prologue_chunk<XT, PRO>(xg + static_cast<int64_t>(m) * a.ldx, kv, a.K, wnorm,
                                                                 is_rms(PRO) ? rinv[m] : 0.f)
                                      : make_uint4(0u, 0u, 0u, 0u);
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (j0 + b < nj) {
          const int ci = tid + NT * (j0 + b);
          const bool act = ci < total;
          const int m = act ? ci / cpr : 0;
          const unsigned mx = act ? chunk_absmax<XT>(held[b]) : 0u;
          if (uniform_rows) {
            const unsigned wmx = __reduce_max_sync(0xffffffffu, mx);
            if (lane == 0 && act && wmx != 0u) atomicMax(&xmax[m], wmx);
          } else if (act && mx != 0u) {
            atomicMax(&xmax[m], mx);
          }
          if (act && !in_regs) *reinterpret_cast<uint4*>(xs + m * a.x_pitch + (ci - m * cpr) * 8) = held[b];
        }
      }
    }
    if (tid == 0) QTTS_TRACE_DETAIL(2, 0);
    named_bar_sync(1, NT);
    if (tid == 0) QTTS_TRACE_DETAIL(2, 1);
    // 2) Scale to fp16 by the row's power of two; per-warp row sums of the
    //    scaled values in a fixed order (deterministic).
    float* mypart = xpart + warp * MB;
    for (int j0 = 0; j0 < nj; j0 += kBatch) {
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (j0 + b < nj) {
          const int ci = tid + NT * (j0 + b);
          const bool act = ci < total;
          const int m = act ? ci / cpr : 0;
          float fx = 0.f;
          if (act) {
            __half* dst = xs + m * a.x_pitch + (ci - m * cpr) * 8;
            const uint4 u = in_regs ? held[b] : *reinterpret_cast<const uint4*>(dst);
            fx = convert_x_chunk<XT>(u, xmax[m], dst);
          }
          if (uniform_rows) {
            const float wsum = warp_sum(fx);
            if (lane == 0 && act) mypart[m] += wsum;
          } else {
            // Rows change inside the warp: one warp-wide sum per row present.
            unsigned pending = __ballot_sync(0xffffffffu, act);
            while (pending != 0u) {
              const int r = __shfl_sync(0xffffffffu, m, __ffs(pending) - 1);
              const float wsum = warp_sum((act && m == r) ? fx : 0.f);
              if (lane == 0) mypart[r] += wsum;
              pending &= ~__ballot_sync(0xffffffffu, act && m == r);
            }
          }
        }
      }
    }
    if (tid == 0) QTTS_TRACE_DETAIL(2, 2);
    named_bar_sync(1, NT);
    if (tid == 0) QTTS_TRACE_STAMP(3);
    if (tid == 0) QTTS_TRACE_DETAIL(2, 3);

    // 3) Main loop: warp (rg, kg) multiplies rows rg*16..+16 of box kg.
    const int rg = warp / KG;
    const int kg = warp % KG;
    const int g = lane >> 2;
    const int q = lane & 3;
    // MMA row g <-> weight row permutation: the rows of one shared-load phase
    // (g = 2p, 2p+1 -> p, p+4) land in opposite 64-byte halves of the span.
    const int pr = (g >> 1) | ((g & 1) << 2);
    const int rowA = rg * 16 + pr;
    const int rowB = rowA + 8;
    const uint32_t box = kg * BN * 128;
    const uint32_t offA0 = box + rowA * 128 + (((0 * 4 + q) ^ (rowA & 7)) << 4);
    const uint32_t offA1 = box + rowA * 128 + (((1 * 4 + q) ^ (rowA & 7)) << 4);
    const uint32_t offB0 = box + rowB * 128 + (((0 * 4 + q) ^ (rowB & 7)) << 4);
    const uint32_t offB1 = box + rowB * 128 + (((1 * 4 + q) ^ (rowB & 7)) << 4);
    const uint32_t wbase = smem_u32(wbuf);
    // Batch row of this lane in tile t is t*8 + g; rows past M contribute zeros.
    bool xrow[MT];
    uint32_t xaddr[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      xrow[t] = t * 8 + g < mrows;
      xaddr[t] = smem_u32(xs) + ((t * 8 + g) * a.x_pitch + kg * 128 + q * 16) * 2;
    }

    float acc[NACC][MT][4];
#pragma unroll
    for (int i = 0; i < NACC; ++i)
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[i][t][0] = acc[i][t][1] = acc[i][t][2] = acc[i][t][3] = 0.f;

#ifdef QTTS_TRACE
    long long trace_c0 = clock64();
#endif
    // Stages whose box for this warp starts before K; later ones only hold zeros.
    const int n_live = a.K > kg * 128 ? (a.K - kg * 128 + SW - 1) / SW : 0;
    bool ok = *reinterpret_cast<volatile int*>(err_flag) == 0;
    int s = 0;
    uint32_t phase = 0;
    for (int it = 0; ok && it < n_iters; ++it, s = (s + 1 == a.stages) ? 0 : s + 1, phase ^= (s == 0)) {
      const bool got = mbar_wait_bounded(&full[s], phase, a.wait_ns);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      if (tid == 0) QTTS_TRACE_DETAIL(0, it);
      if (it >= n_live) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        continue;
      }
      const uint32_t sb = wbase + s * kStStageBytes;
      const uint4 wa0 = lds128(sb + offA0);
      const uint4 wb0 = lds128(sb + offB0);
      const uint4 wa1 = lds128(sb + offA1);
      const uint4 wb1 = lds128(sb + offB1);

      const uint32_t wA[2][4] = {{wa0.x, wa0.y, wa0.z, wa0.w}, {wa1.x, wa1.y, wa1.z, wa1.w}};
      const uint32_t wB[2][4] = {{wb0.x, wb0.y, wb0.z, wb0.w}, {wb1.x, wb1.y, wb1.z, wb1.w}};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint4 xv[MT][2];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          if (xrow[t]) {
            const uint32_t xa = xaddr[t] + (it * SW + h * 64) * 2;
            xv[t][0] = lds128(xa);
            xv[t][1] = lds128(xa + 16);
          } else {
            xv[t][0] = make_uint4(0u, 0u, 0u, 0u);
            xv[t][1] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a0, a1, a2, a3;
          i8x4_to_f16_biased(wA[h][j], a0, a2);
          i8x4_to_f16_biased(wB[h][j], a1, a3);
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const uint4& x0 = xv[t][j >> 1];
            const uint32_t b0 = (j & 1) ? x0.z : x0.x;
            const uint32_t b1 = (j & 1) ? x0.w : x0.y;
            hmma(acc[(h * 4 + j) % NACC][t], a0, a1, a2, a3, b0, b1);
          }
        }
      }
      // The stage goes back to the producer only after every loaded word has
      // been consumed (a TMA refill cannot overtake a read of the stage).
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (!ok) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *reinterpret_cast<volatile int*>(err_flag) = 1;
    }
    if (tid == 0) QTTS_TRACE_STAMP(5);
    if (lane == 0) QTTS_TRACE_DETAIL(4, warp);
#ifdef QTTS_TRACE
    if (tid == 0 && a.trace_slot == 5 && blockIdx.x == 0 && blockIdx.z == 0)
      g_trace_detail[5][0] = static_cast<unsigned long long>(clock64() - trace_c0);
#endif
    // Every warp is done with the stage ring before it becomes `red`.
    named_bar_sync(1, NT);
    const bool cta_err = *reinterpret_cast<volatile int*>(err_flag) != 0;
    if (!cta_err) {
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int c0 = t * 8 + 2 * q;
        float v0 = acc[0][t][0], v1 = acc[0][t][1], v2 = acc[0][t][2], v3 = acc[0][t][3];
#pragma unroll
        for (int i = 1; i < NACC; ++i) {
          v0 += acc[i][t][0];
          v1 += acc[i][t][1];
          v2 += acc[i][t][2];
          v3 += acc[i][t][3];
        }
        float* r = red + kg * BN * MB;
        *reinterpret_cast<float2*>(&r[rowA * MB + c0]) = make_float2(v0, v1);
        *reinterpret_cast<float2*>(&r[rowB * MB + c0]) = make_float2(v2, v3);
      }
    }
    named_bar_sync(1, NT);
    if (tid == 0) QTTS_TRACE_DETAIL(2, 4);
    // 4) Sum the k groups in fixed order, remove the dequantization bias, scale.
    if (valid && !cta_err) {
      for (int i = tid; i < BN * mrows; i += NT) {
        const int m = i / BN;
        const int row = i - m * BN;
        const int n = n0 + row;
        if (n < a.N) {
          float sum = red[row * MB + m];
#pragma unroll
          for (int c = 1; c < KG; ++c) sum += red[c * BN * MB + row * MB + m];
          float xsum = xpart[m];
#pragma unroll
          for (int w = 1; w < kStConsumerWarps; ++w) xsum += xpart[w * MB + m];
          const float inv = pow2f_st(-row_exponent(__uint_as_float(xmax[m])));
          const float dot = fmaf(-kStBias, xsum, sum) * inv;
          const float r = dot * pre_sc + pre_bias;
          og[static_cast<int64_t>(m) * a.ldo + n] = from_float<XT>(r);
        }
      }
    }
  }

  if (tid == 0) QTTS_TRACE_STAMP(6);
  // Error path: make sure no copy of ours is still landing in shared memory.
  if (warp == kStConsumerWarps && lane == 0 && *reinterpret_cast<volatile int*>(err_flag) != 0) {
    for (int s = 0; s < a.stages && s < n_issued; ++s) {
      const int last = ((n_issued - 1 - s) / a.stages) * a.stages + s;
      mbar_wait_bounded(&full[s], (last / a.stages) & 1, a.wait_ns);
    }
  }
}

// ------------------------------------------------------------------------------------
// Host side

namespace {

template <int MT, int R, typename XT, int PRO>
int launch_stream_t(const CUtensorMap& map, const SkinnyArgs& args, dim3 grid, size_t smem, bool pdl,
                    cudaStream_t stream) {
  auto kern = stream_w8a16_kernel<MT, R, XT, PRO>;
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
  cfg.blockDim = dim3(kStThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[1];
  int na = 0;
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

template <int MT, typename XT, int PRO>
int launch_stream_rp(int r, const CUtensorMap& map, const SkinnyArgs& args, dim3 grid, size_t smem, bool pdl,
                     cudaStream_t stream) {
  switch (r) {
    case 1:
      return launch_stream_t<MT, 1, XT, PRO>(map, args, grid, smem, pdl, stream);
    case 2:
      return launch_stream_t<MT, 2, XT, PRO>(map, args, grid, smem, pdl, stream);
    case 3:
      return launch_stream_t<MT, 3, XT, PRO>(map, args, grid, smem, pdl, stream);
    case 4:
      return launch_stream_t<MT, 4, XT, PRO>(map, args, grid, smem, pdl, stream);
    default:
      return launch_stream_t<MT, 6, XT, PRO>(map, args, grid, smem, pdl, stream);
  }
}

template <int MT, typename XT>
int launch_stream_r(int r, const CUtensorMap& map, const SkinnyArgs& args, dim3 grid, size_t smem, bool pdl,
                    cudaStream_t stream) {
  if (args.prologue == kProRmsNorm) return launch_stream_rp<MT, XT, kProRmsNorm>(r, map, args, grid, smem, pdl, stream);
  if (args.prologue == kProRmsNormRows) {
    return launch_stream_rp<MT, XT, kProRmsNormRows>(r, map, args, grid, smem, pdl, stream);
  }
  if (args.prologue == kProSiluMul) return launch_stream_rp<MT, XT, kProSiluMul>(r, map, args, grid, smem, pdl, stream);
  return launch_stream_rp<MT, XT, kProNone>(r, map, args, grid, smem, pdl, stream);
}

size_t stream_smem(int mb, int xrows, int x_pitch, int stages) {
  // xpart [warps][mb], xmax [mb], rinv [mb], then the barriers.
  return 1024 + static_cast<size_t>(stages) * kStStageBytes + static_cast<size_t>(xrows) * x_pitch * 2 +
         (kStConsumerWarps + 2) * mb * 4 + 16 + 16 * stages + 16;
}

}  // namespace

bool stream_rows_ok(int r) { return r == 1 || r == 2 || r == 3 || r == 4 || r == 6; }

SkinnyPlan plan_stream(int M, int N, int K, int G, int r_req) {
  SkinnyPlan p{};
  p.mt = M <= 8 ? 1 : 2;
  const int mb = p.mt * 8;
  p.m_chunks = (M + mb - 1) / mb;
  p.split = 1;
  int r = r_req;
  if (r == 0) {
    // Fewest rows per CTA that keeps the grid within one wave of 148 SMs.
    const int cands[5] = {1, 2, 3, 4, 6};
    r = 6;
    for (int i = 0; i < 5; ++i) {
      const long long ctas = static_cast<long long>((N + 16 * cands[i] - 1) / (16 * cands[i])) * G * p.m_chunks;
      if (ctas <= kNumSMs) {
        r = cands[i];
        break;
      }
    }
  }
  p.r = r;
  const int sw = 128 * (kStConsumerWarps / r);
  const int n_iters = (K + sw - 1) / sw;
  p.k_per_cta = n_iters * sw;
  p.x_pitch = (K + 127) / 128 * 128 + 8;  // +16 bytes: rows of one LDS phase hit distinct banks
  // Stage ring: the whole slice when it fits a ~110 KiB budget (two CTAs per
  // SM, so the next kernel's weights stream in beside this one), else as
  // many stages as fit; at least two, and enough to hold the k-group sums.
  const int xrows = M < mb ? M : mb;
  const size_t fixed = stream_smem(mb, xrows, p.x_pitch, 0);
  const size_t budget = 110 * 1024;
  int stages = fixed < budget ? static_cast<int>((budget - fixed) / kStStageBytes) : 0;
  stages = stages < n_iters ? stages : n_iters;
  const int red_bytes = kStConsumerWarps * 16 * mb * 4;
  const int min_stages = (red_bytes + kStStageBytes - 1) / kStStageBytes;
  stages = stages < min_stages ? min_stages : stages;
  stages = stages < 2 ? 2 : stages;
  p.stages = stages;
  p.smem = stream_smem(mb, xrows, p.x_pitch, stages);
  p.grid = dim3((N + 16 * r - 1) / (16 * r), 1, G * p.m_chunks);
  return p;
}

int launch_stream_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, int x_dtype, bool pdl,
                        cudaStream_t stream) {
  if (p.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
  if (x_dtype == QTTS_BF16) {
    return p.mt == 1 ? launch_stream_r<1, __nv_bfloat16>(p.r, map, args, p.grid, p.smem, pdl, stream)
                     : launch_stream_r<2, __nv_bfloat16>(p.r, map, args, p.grid, p.smem, pdl, stream);
  }
  if (x_dtype == QTTS_FP16) {
    return p.mt == 1 ? launch_stream_r<1, __half>(p.r, map, args, p.grid, p.smem, pdl, stream)
                     : launch_stream_r<2, __half>(p.r, map, args, p.grid, p.smem, pdl, stream);
  }
  return QTTS_ERR_DTYPE;
}

}  // namespace qtts
