// Skinny int8 weight-only GEMM (W8A16) for decode batch sizes.
//
// Replaces the Triton kernel _w8_gemm_kernel (qtts/quant/kernels.py:89-135):
//   out[m, n] = cast( sum_k x[m, k] * w[n, k] * scale[n] + bias[n] )
// with the int8 convert done in registers, fp32 accumulation and the
// per-output-channel scale applied once after the K loop (kernels.py:123,
// 129-130).
//
// Design (B200, sm_100a). A decode GEMM streams N*K weight bytes once and does
// 2*M flops per byte; in a decode step every linear waits on the previous one,
// so per-kernel latency matters as much as bandwidth.
//   * A CTA owns BN = 16*R weight rows (R = 1, 2, 4 or 8 row groups) and one K
//     slice. Its 8 consumer warps form R row groups x (8/R) k groups. A stage
//     is 16 KiB: 8/R TMA boxes of BN rows x 128 bytes (128-byte swizzle), one
//     per k group, so small shapes split K inside the CTA (reduced through
//     shared memory) instead of across CTAs.
//   * A producer warp streams the weight slice through a ring of
//     mbarrier-tracked stages. Weights are constant, so streaming starts before
//     the programmatic-dependent-launch wait: in a chain of linears the next
//     layer's weights arrive while the previous kernel drains.
//   * After the dependency wait every consumer thread loads 16-byte chunks of
//     the activation slice into registers, the per-row maximum is combined in
//     shared memory, and each thread stores its chunks as fp16 scaled by a
//     per-row power of two (exact for every element within 2^28 of the row's
//     largest magnitude; smaller ones round as fp16 subnormals, far below the
//     bf16 output resolution).
//   * Dequantization: 0x64 above a byte u is the fp16 1024 + u, so (b ^ 0x80)
//     placed there by one byte-permute per two weights, minus 1152, is b
//     exactly. MMA: mma.sync m16n8k16 f16 -> fp32, weights as the M=16 operand
//     and activations as the N=8 operand ("swap AB"), so batch rows 1..8 cost
//     one MMA per 256 weights. K is permuted inside each 64-wide chunk (thread
//     q owns k = 16q..16q+15) so weight and activation fragments are plain
//     128-bit shared loads; the dot product does not depend on the order.
//   * Optional split-K across a thread-block cluster (S = 2, 4, 8) for large
//     M*K: each CTA owns BN/S rows of the result and receives the other CTAs'
//     partial sums (k groups already added) by st.async from registers into
//     its shared memory, counted on its own mbarrier; a split cluster barrier
//     (arrive at start, wait before the first remote store) plus one closing
//     phase, so that a cluster's CTAs leave together, are the only
//     cluster-wide synchronization.
//   * Optional activation prologue (template PRO, csrc/prologue.cuh): SiLU·up
//     of [gate | up] rows, applied to each chunk as it is staged, or RMSNorm.
//     The norm's factor needs the whole row. When K and the slice are
//     multiples of 256, each warp's 32 staged chunks are exactly one group of
//     the norm's fixed order, so every CTA sums its own slice and sends the
//     group sums to its cluster peers (st.async on a bounded mbarrier): no
//     extra loads. Otherwise all warps load the rows once more.
//   * Every wait is bounded (globaltimer). On expiry the kernel records
//     QTTS_ERR_TIMEOUT in the device status word, keeps the remote-store
//     protocol (so no peer waits on it), skips its global stores and drains its
//     own copies in flight before exiting.
#include "allgather.cuh"
#include "common.cuh"
#include "kernels.h"
#include "prologue.cuh"

namespace qtts {

constexpr int kSkStageBytes = 16384;
constexpr int kSkConsumerWarps = 8;
constexpr int kSkThreads = (kSkConsumerWarps + 1) * 32;

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

template <int MT, int R, typename XT, bool E4M3 = false, bool AG = false, int PRO = kProNone>
__global__ void __launch_bounds__(kSkThreads, 2)
    skinny_w8a16_kernel(const __grid_constant__ CUtensorMap wmap, const SkinnyArgs a) {
  constexpr int MB = MT * 8;       // batch rows per CTA (MMA N dimension)
  constexpr int KG = 8 / R;        // k groups
  constexpr int BN = 16 * R;       // weight rows per CTA
  constexpr int SW = 128 * KG;     // k per stage
  // Independent accumulator sets (MMA latency). More sets (8 at up to 8 rows)
  // measured 4-6 % slower in chained calls: the loop is bound by the dequant
  // and MMA issue of two CTAs per SM, not by the MMA chain.
  constexpr int NACC = MT <= 2 ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wbuf = smem;
  __half* xs = reinterpret_cast<__half*>(smem + a.stages * kSkStageBytes);  // [MB][x_pitch]
  float* xinv = reinterpret_cast<float*>(xs + MB * a.x_pitch);               // [MB] 2^-scale
  float* rinv = xinv + MB;                                                   // [MB] RMSNorm factors
  float* recv = rinv + MB;                                                   // [S][BN/S][MB]
  const int split = gridDim.y;
  uint64_t* full = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(recv + (split > 1 ? BN * MB : 0)) + 15) & ~uintptr_t(15));
  uint64_t* empty = full + a.stages;
  uint64_t* recv_bar = empty + a.stages;
  uint64_t* norm_bar = recv_bar + 1;  // RMSNorm prologue: the peers' group sums have landed
  int* err_flag = reinterpret_cast<int*>(recv_bar + 2);
  int* gate_flag = err_flag + 1;  // all-gather form: every rank is ready to receive
  // RMSNorm prologue: [MB][K / 256] group sums (the launch adds MB * 128 bytes).
  float* ngs = reinterpret_cast<float*>(recv_bar + 4);
  float* red = reinterpret_cast<float*>(wbuf);  // [KG][BN][MB], reuses the ring after the loop

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int kidx = blockIdx.y;
  const uint32_t crank = split > 1 ? cluster_ctarank() : 0u;
  const int rpo = BN / split;  // result rows owned per CTA
  const int n0 = blockIdx.x * BN;
  const int mchunk = blockIdx.z % a.m_chunks;
  int group = blockIdx.z / a.m_chunks;
  const int m0 = mchunk * MB;
  const int k0 = kidx * a.k_per_cta;
  const int klen = max(0, min(a.K - k0, a.k_per_cta));
  int n_iters = (klen + SW - 1) / SW;
  // RMSNorm from the CTAs' own slices (group-aligned slices, K <= 8192).
  // (the host picks this form only when K and the slices are multiples of 256).
  constexpr bool slice_norm = PRO == kProRmsNorm;

  if (tid == 0) {
    QTTS_TRACE_STAMP(0);
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSkConsumerWarps);
    }
    mbar_init(recv_bar, 1);
    if constexpr (slice_norm) {
      // One arrival now; the phase completes when every peer's group sums
      // (its slice's groups x the real rows of this m chunk) have landed.
      mbar_init(norm_bar, 1);
      uint32_t bytes = 0;
      for (int p = 0; p < split; ++p) {
        if (p == kidx) continue;
        const int len = max(0, min(a.K - p * a.k_per_cta, a.k_per_cta));
        bytes += static_cast<uint32_t>((len >> 8) * min(MB, a.M - m0) * 4);
      }
      mbar_arrive_expect_tx(norm_bar, bytes);
    }
    for (int i = 0; i < MB; ++i) xinv[i] = 0.f;
    if (split > 1) {
      // The single arrival happens now; the phase completes once every peer's
      // partial sums for my rows have landed.
      mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((split - 1) * rpo * MB * 4));
    }
    *err_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  if (split > 1) cluster_arrive_relaxed();
  pdl_launch_dependents();
  if (AG && tid == 0) ag_prefetch_tables(a);

  // Device-indexed single group: the index may be produced by the preceding
  // kernel, so everything (including the weight stream) waits for it.
  bool valid = true;
  if (a.group_index != nullptr) {
    pdl_wait();
    const int64_t gi = __ldcg(a.group_index);
    if (gi < 0 || gi >= a.G) {
      valid = false;
      n_iters = 0;
      if (tid == 0 && kidx == 0 && blockIdx.x == 0) record_status(QTTS_ERR_SHAPE);
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
  const int64_t pbase = static_cast<int64_t>(m0) * a.ldo + a.col_offset;  // all-gather form
  uint32_t ag_ep = 0;  // all-gather form: epoch of this call (consumer threads)

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
        uint8_t* dst = wbuf + s * kSkStageBytes;
#pragma unroll
        for (int c = 0; c < KG; ++c) {
          tma_load_2d(dst + c * BN * 128, &wmap, k0 + it * SW + c * 128, static_cast<int>(wrow0), &full[s]);
        }
        n_issued = it + 1;
        if (it == 0) QTTS_TRACE_STAMP(1);
      }
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    // The scale and bias of the output channel this thread finishes (every
    // epilogue below gives thread t the owned row t mod (rows owned), which
    // divides 256) are constants of the layer: loaded before the dependency
    // wait, so the end of the chain does not wait on a cold global load.
    float pre_sc = 0.f, pre_bias = 0.f;
    {
      const int own = split > 1 ? rpo : BN;
      const int n = n0 + (split > 1 ? static_cast<int>(crank) * rpo : 0) + tid % own;
      if (valid && n < a.N) {
        const int64_t ch = static_cast<int64_t>(group) * a.N + n;
        pre_sc = load_as_float(a.scale, a.scale_dtype, ch);
        if (a.bias != nullptr) pre_bias = to_float(static_cast<const XT*>(a.bias)[ch]);
      }
    }
    pdl_wait();
    if (tid == 0) QTTS_TRACE_STAMP(2);
    if (AG) ag_ep = ag_epoch(a);  // consumed after the activation staging
#ifdef QTTS_TRACE
    if (tid == 0 && a.trace_slot == 5 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
      g_trace_detail[3][0] = globaltimer_ns();
      for (int s = 0; s < a.stages && s < n_iters && s < 63; ++s)
        g_trace_detail[1][s] = mbar_try_wait(&full[s], 0) ? 1ull : 0ull;
    }
#endif
    const int kpad = n_iters * SW;
    const XT* wnorm = static_cast<const XT*>(a.pro_weight);
    // 1) Activation slice [MB, kpad]: each thread loads 16-byte chunks into
    //    registers (zeros past K and past the last batch row), the per-row
    //    maximum is combined with shared-memory atomics, then every thread
    //    scales its own chunks to fp16 and stores them.
    {
      const int cpr = kpad / 8;  // chunks per row
      const int total = MB * cpr;
      const bool warp_rows = cpr % 32 == 0;
      constexpr int kHeld = 4;
      const bool in_regs = total <= kHeld * kSkConsumerWarps * 32;
      uint4 held[kHeld];
      const int nj = in_regs ? kHeld : (total + kSkConsumerWarps * 32 - 1) / (kSkConsumerWarps * 32);
      uint4 heldw[kHeld];  // norm weights of the chunks held in registers (slice form)
      if constexpr (slice_norm) {
        // Raw chunks (registers, or parked in the staged slice); a warp's 32
        // consecutive chunks are one row's group g = k / 256: leaf sums and
        // butterfly, then the group sum goes to this CTA's table and to every
        // peer's (the cluster wait makes sure the peers' barriers exist).
        const int groups = a.K >> 8;
        if (split > 1) cluster_wait();
#pragma unroll 4
        for (int j = 0; j < nj; ++j) {
          const int ci = tid + kSkConsumerWarps * 32 * j;
          if (ci >= total) break;  // total is a multiple of 32: warp-uniform
          const int m = ci / cpr;
          const int kv = (ci - m * cpr) * 8;
          const bool real = valid && m < mrows && kv < klen;  // warp-uniform
          uint4 u = make_uint4(0u, 0u, 0u, 0u);
          if (real) u = __ldcg(reinterpret_cast<const uint4*>(xg + static_cast<int64_t>(m) * a.ldx + k0 + kv));
          if (in_regs) {
            held[j & (kHeld - 1)] = u;
            heldw[j & (kHeld - 1)] =
                real ? __ldg(reinterpret_cast<const uint4*>(wnorm + k0 + kv)) : make_uint4(0u, 0u, 0u, 0u);
          } else {
            *reinterpret_cast<uint4*>(xs + m * a.x_pitch + kv) = u;
          }
          if (real) {
            const XT* e = reinterpret_cast<const XT*>(&u);
            float v[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) v[q] = to_float(e[q]);
            const float gsum = group_butterfly(leaf_sumsq(v));
            const int idx = m * groups + ((k0 + kv) >> 8);
            if (lane == 0) ngs[idx] = gsum;
            if (lane < split && lane != static_cast<int>(crank)) {
              st_async_f32(mapa_shared(smem_u32(ngs + idx), lane), gsum,
                           mapa_shared(smem_u32(norm_bar), lane));
            }
          }
        }
        named_bar_sync(1, kSkConsumerWarps * 32);  // own group sums written
        if (!mbar_wait_bounded(norm_bar, 0, a.wait_ns)) {
          if (tid == 0) record_status(QTTS_ERR_TIMEOUT);
          // Peers always send; keep this CTA's table alive until their stores land.
          mbar_wait_bounded(norm_bar, 0, 4 * a.wait_ns);
        }
        for (int m = warp; m < mrows; m += kSkConsumerWarps) {
          const float ssq = lanes_stride_tree(lane < groups ? ngs[m * groups + lane] : 0.f, groups);
          if (lane == 0) rinv[m] = rms_inv(ssq, a.K, a.pro_eps);
        }
        named_bar_sync(1, kSkConsumerWarps * 32);
      } else if constexpr (PRO == kProRmsNormRows) {
        // The rows are loaded once more, by all warps. When the slice fits in
        // registers its raw chunks and their norm weights are loaded first,
        // so those loads overlap the norm's; the factors' scratch aliases the
        // (not yet written) staged slice.
        if (in_regs) {
#pragma unroll
          for (int j = 0; j < kHeld; ++j) {
            const int ci = tid + kSkConsumerWarps * 32 * j;
            const int m = ci / cpr;
            const int kv = (ci - m * cpr) * 8;
            held[j] = heldw[j] = make_uint4(0u, 0u, 0u, 0u);
            if (ci < total && valid && m < mrows && kv < klen) {
              held[j] = __ldcg(reinterpret_cast<const uint4*>(xg + static_cast<int64_t>(m) * a.ldx + k0 + kv));
              heldw[j] = __ldg(reinterpret_cast<const uint4*>(wnorm + k0 + kv));
            }
          }
        }
        cta_norm_factors<XT>(xg, a.ldx, valid ? mrows : 0, a.K, a.pro_eps, reinterpret_cast<float*>(xs), rinv, warp,
                             lane, kSkConsumerWarps, 1);
        if (in_regs) {
#pragma unroll
          for (int j = 0; j < kHeld; ++j) {
            const int ci = tid + kSkConsumerWarps * 32 * j;
            const int m = ci / cpr;
            const int kv = (ci - m * cpr) * 8;
            if (ci < total && valid && m < mrows && kv < klen) held[j] = normalize_chunk<XT>(held[j], heldw[j], rinv[m]);
          }
        }
      }
#pragma unroll 4
      for (int j = 0; j < nj; ++j) {
        const int ci = tid + kSkConsumerWarps * 32 * j;
        if (ci >= total) break;
        const int m = ci / cpr;
        const int kv = (ci - m * cpr) * 8;
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (slice_norm) {
          // Raw chunk staged above; normalized now that the factors are known.
          if (valid && m < mrows && kv < klen) {
            if (in_regs) {
              u = normalize_chunk<XT>(held[j & (kHeld - 1)], heldw[j & (kHeld - 1)], rinv[m]);
            } else {
              u = normalize_chunk<XT>(*reinterpret_cast<const uint4*>(xs + m * a.x_pitch + kv),
                                      __ldg(reinterpret_cast<const uint4*>(wnorm + k0 + kv)), rinv[m]);
            }
          }
        } else {
          if (PRO == kProRmsNormRows && in_regs) {
            u = held[j & (kHeld - 1)];  // normalized above
          } else if (valid && m < mrows && kv < klen) {
            u = prologue_chunk<XT, PRO>(xg + static_cast<int64_t>(m) * a.ldx, k0 + kv, a.K, wnorm,
                                        is_rms(PRO) ? rinv[m] : 0.f);
          }
        }
        const XT* e = reinterpret_cast<const XT*>(&u);
        float mx = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) mx = fmaxf(mx, fabsf(to_float(e[q])));
        if (warp_rows) {
          // The warp's 32 chunks lie in one row (and the loop exits warp-wide):
          // one shared atomic per warp instead of one per chunk.
          const unsigned wmx = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
          if (lane == 0 && wmx != 0u) atomicMax(reinterpret_cast<unsigned int*>(&xinv[m]), wmx);
        } else if (mx > 0.f) {
          atomicMax(reinterpret_cast<unsigned int*>(&xinv[m]), __float_as_uint(mx));
        }
        if (in_regs) {
          held[j & (kHeld - 1)] = u;
        } else {
          *reinterpret_cast<uint4*>(xs + m * a.x_pitch + kv) = u;  // raw; converted below
        }
      }
      if (tid == 0) QTTS_TRACE_DETAIL(2, 0);
      named_bar_sync(1, kSkConsumerWarps * 32);
      if (tid == 0) QTTS_TRACE_DETAIL(2, 1);
#pragma unroll 4
      for (int j = 0; j < nj; ++j) {
        const int ci = tid + kSkConsumerWarps * 32 * j;
        if (ci >= total) break;
        const int m = ci / cpr;
        const int kv = (ci - m * cpr) * 8;
        uint4* dst = reinterpret_cast<uint4*>(xs + m * a.x_pitch + kv);
        const uint4 u = in_regs ? held[j & (kHeld - 1)] : *dst;
        const float mxr = xinv[m];
        int sexp = 0;
        if (mxr > 0.f) sexp = min(max(14 - (static_cast<int>((__float_as_uint(mxr) >> 23) & 0xFF) - 127), -100), 100);
        const float sc = pow2f(sexp);
        const XT* e = reinterpret_cast<const XT*>(&u);
        uint4 o;
        __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) h[q] = __floats2half2_rn(to_float(e[2 * q]) * sc, to_float(e[2 * q + 1]) * sc);
        *dst = o;
      }
      if (tid == 0) QTTS_TRACE_DETAIL(2, 2);
      named_bar_sync(1, kSkConsumerWarps * 32);
      if (tid == 0) QTTS_TRACE_DETAIL(2, 3);
      if (tid < MB) {
        // xinv held the row maximum (as bits); turn it into 2^-scale.
        const float mxr = xinv[tid];
        int sexp = 0;
        if (mxr > 0.f) sexp = min(max(14 - (static_cast<int>((__float_as_uint(mxr) >> 23) & 0xFF) - 127), -100), 100);
        xinv[tid] = pow2f(-sexp);  // next read after the loop-end barrier
      }
    }
    if (tid == 0) QTTS_TRACE_STAMP(3);
    // Every CTA announces (no wait depends on another CTA of this grid having started).
    if (AG && tid == 0) ag_announce_ready(a, ag_ep);

    // 2) Main loop.
    const int rg = warp / KG;  // row group
    const int kg = warp % KG;  // k group (which 128-byte box of the stage)
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
    const uint32_t xbase = smem_u32(xs) + (g * a.x_pitch + kg * 128 + q * 16) * 2;
    const uint32_t xtile = 8 * a.x_pitch * 2;

    float acc[NACC][MT][4];
#pragma unroll
    for (int i = 0; i < NACC; ++i)
#pragma unroll
      for (int t = 0; t < MT; ++t) acc[i][t][0] = acc[i][t][1] = acc[i][t][2] = acc[i][t][3] = 0.f;

    bool ok = *reinterpret_cast<volatile int*>(err_flag) == 0;
    for (int it = 0; ok && it < n_iters; ++it) {
      const int s = it % a.stages;
      const bool got = mbar_wait_bounded(&full[s], (it / a.stages) & 1, a.wait_ns);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      if (it == 0 && tid == 0) QTTS_TRACE_STAMP(4);
      if (tid == 0) QTTS_TRACE_DETAIL(0, it);
      const uint32_t sb = wbase + s * kSkStageBytes;
      const uint4 wa0 = lds128(sb + offA0);
      const uint4 wb0 = lds128(sb + offB0);
      const uint4 wa1 = lds128(sb + offA1);
      const uint4 wb1 = lds128(sb + offB1);

      uint32_t A[2][4][4];
      WDequant<__half, E4M3>::run(wa0.x, A[0][0][0], A[0][0][2]);
      WDequant<__half, E4M3>::run(wb0.x, A[0][0][1], A[0][0][3]);
      WDequant<__half, E4M3>::run(wa0.y, A[0][1][0], A[0][1][2]);
      WDequant<__half, E4M3>::run(wb0.y, A[0][1][1], A[0][1][3]);
      WDequant<__half, E4M3>::run(wa0.z, A[0][2][0], A[0][2][2]);
      WDequant<__half, E4M3>::run(wb0.z, A[0][2][1], A[0][2][3]);
      WDequant<__half, E4M3>::run(wa0.w, A[0][3][0], A[0][3][2]);
      WDequant<__half, E4M3>::run(wb0.w, A[0][3][1], A[0][3][3]);
      WDequant<__half, E4M3>::run(wa1.x, A[1][0][0], A[1][0][2]);
      WDequant<__half, E4M3>::run(wb1.x, A[1][0][1], A[1][0][3]);
      WDequant<__half, E4M3>::run(wa1.y, A[1][1][0], A[1][1][2]);
      WDequant<__half, E4M3>::run(wb1.y, A[1][1][1], A[1][1][3]);
      WDequant<__half, E4M3>::run(wa1.z, A[1][2][0], A[1][2][2]);
      WDequant<__half, E4M3>::run(wb1.z, A[1][2][1], A[1][2][3]);
      WDequant<__half, E4M3>::run(wa1.w, A[1][3][0], A[1][3][2]);
      WDequant<__half, E4M3>::run(wb1.w, A[1][3][1], A[1][3][3]);
      // The stage goes back to the producer only after every loaded word has
      // been consumed: the conversions above wait for the shared loads, so a
      // TMA refill cannot overtake a read of the stage.
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);

      const uint32_t xk = xbase + it * SW * 2;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t xa = xk + t * xtile + h * 64 * 2;
          const uint4 x0 = lds128(xa);
          const uint4 x1 = lds128(xa + 16);
          float(&c)[4] = acc[h % NACC][t];
          Mma16816<__half>::run(c, A[h][0], x0.x, x0.y);
          Mma16816<__half>::run(c, A[h][1], x0.z, x0.w);
          Mma16816<__half>::run(c, A[h][2], x1.x, x1.y);
          Mma16816<__half>::run(c, A[h][3], x1.z, x1.w);
        }
      }
    }
    if (!ok) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *reinterpret_cast<volatile int*>(err_flag) = 1;
    }
    if (tid == 0) QTTS_TRACE_STAMP(5);
    if (tid == 32) QTTS_TRACE_DETAIL(4, 0);
    if (tid == 224) QTTS_TRACE_DETAIL(4, 1);
    // Every warp is done with the stage ring before it becomes `red`.
    named_bar_sync(1, kSkConsumerWarps * 32);
    const bool cta_err = *reinterpret_cast<volatile int*>(err_flag) != 0;
    if (!cta_err) {
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int c0 = t * 8 + 2 * q;
        const float i0 = xinv[c0];
        const float i1 = xinv[c0 + 1];
        float v0 = acc[0][t][0], v1 = acc[0][t][1], v2 = acc[0][t][2], v3 = acc[0][t][3];
#pragma unroll
        for (int i = 1; i < NACC; ++i) {
          v0 += acc[i][t][0];
          v1 += acc[i][t][1];
          v2 += acc[i][t][2];
          v3 += acc[i][t][3];
        }
        float* r = red + kg * BN * MB;
        *reinterpret_cast<float2*>(&r[rowA * MB + c0]) = make_float2(v0 * i0, v1 * i1);
        *reinterpret_cast<float2*>(&r[rowB * MB + c0]) = make_float2(v2 * i0, v3 * i1);
      }
    }
    named_bar_sync(1, kSkConsumerWarps * 32);
    if (split == 1) {
      // 3) Sum the k groups in fixed order: red[0] = CTA partial sums [BN][MB].
      if (KG > 1 && !cta_err) {
        for (int i = tid; i < BN * MB; i += kSkConsumerWarps * 32) {
          float sum = red[i];
#pragma unroll
          for (int c = 1; c < KG; ++c) sum += red[c * BN * MB + i];
          red[i] = sum;
        }
        named_bar_sync(1, kSkConsumerWarps * 32);
      }
      bool store_ok = valid && !cta_err;
      if (AG) store_ok = ag_gate_stores(a, ag_ep, gate_flag, 1, kSkConsumerWarps * 32, tid == 0) && store_ok;
      if (store_ok) {
        for (int i = tid; i < BN * mrows; i += kSkConsumerWarps * 32) {
          const int m = i / BN;
          const int row = i - m * BN;
          const int n = n0 + row;
          if (n < a.N) {
            const float r = red[row * MB + m] * pre_sc + pre_bias;
            put_out<AG>(a, og, pbase, static_cast<int64_t>(m) * a.ldo + n, from_float<XT>(r));
          }
        }
      }
    } else {
      // 4) Each 16-byte chunk of the CTA's partial sums (k groups added in
      //    fixed order) goes straight to its row owner's receive slot for this
      //    rank: a plain store for own rows, st.async from registers for a
      //    peer's, counted on the owner's mbarrier. Peers always send, even
      //    after an error, so no owner waits in vain.
      if (!slice_norm) cluster_wait();  // every peer's receive barrier is initialized (waited already otherwise)
      constexpr int kCpr = MB / 4;  // 16-byte chunks per row
      const uint32_t own_recv = smem_u32(recv);
      for (int i = tid; i < BN * kCpr; i += kSkConsumerWarps * 32) {
        const int row = i / kCpr;
        const int c4 = (i - row * kCpr) * 4;
        float4 v = *reinterpret_cast<const float4*>(red + row * MB + c4);
#pragma unroll
        for (int c = 1; c < KG; ++c) {
          const float4 t = *reinterpret_cast<const float4*>(red + c * BN * MB + row * MB + c4);
          v.x += t.x;
          v.y += t.y;
          v.z += t.z;
          v.w += t.w;
        }
        const int owner = row / rpo;
        const int lr = row - owner * rpo;
        const int slot = (static_cast<int>(crank) * rpo + lr) * MB + c4;
        if (owner == static_cast<int>(crank)) {
          *reinterpret_cast<float4*>(recv + slot) = v;
        } else {
          st_async_f32x4(mapa_shared(own_recv + slot * 4, owner), v.x, v.y, v.z, v.w,
                         mapa_shared(smem_u32(recv_bar), owner));
        }
      }
      named_bar_sync(1, kSkConsumerWarps * 32);  // own slot written
      // 5) Owner: reduce the split partial sums of its rows in rank order.
      bool have = mbar_wait_bounded(recv_bar, 0, a.wait_ns);
      if (!have) {
        if (tid == 0) record_status(QTTS_ERR_TIMEOUT);
        // Peers always send; keep this CTA alive until their stores land.
        have = mbar_wait_bounded(recv_bar, 0, 4 * a.wait_ns);
      }
      if (tid == 0) QTTS_TRACE_STAMP(7);
      if (AG) have = ag_gate_stores(a, ag_ep, gate_flag, 1, kSkConsumerWarps * 32, tid == 0) && have;
      if (have && valid && !cta_err && mrows <= 2) {
        // One or two real batch rows: thread = (owned row, batch row).
        const int rbase = static_cast<int>(crank) * rpo;
        for (int i = tid; i < rpo * mrows; i += kSkConsumerWarps * 32) {
          const int m = i / rpo;
          const int lr = i - m * rpo;
          const int n = n0 + rbase + lr;
          if (n < a.N) {
            float r = 0.f;
            for (int p = 0; p < split; ++p) r += recv[(p * rpo + lr) * MB + m];
            r = r * pre_sc + pre_bias;
            put_out<AG>(a, og, pbase, static_cast<int64_t>(m) * a.ldo + n, from_float<XT>(r));
          }
        }
      } else if (have && valid && !cta_err) {
        // Thread = (owned row, 4 batch columns): one 16-byte load per rank.
        const int rbase = static_cast<int>(crank) * rpo;
        const int quads = (mrows + 3) / 4;
        for (int i = tid; i < rpo * quads; i += kSkConsumerWarps * 32) {
          const int mq = i / rpo;
          const int lr = i - mq * rpo;
          const int n = n0 + rbase + lr;
          if (n < a.N) {
            float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p = 0; p < split; ++p) {
              const float4 t = *reinterpret_cast<const float4*>(recv + (p * rpo + lr) * MB + 4 * mq);
              r.x += t.x;
              r.y += t.y;
              r.z += t.z;
              r.w += t.w;
            }
            const float rv[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int m = 4 * mq + q;
              if (m < mrows) put_out<AG>(a, og, pbase, static_cast<int64_t>(m) * a.ldo + n, from_float<XT>(rv[q] * pre_sc + pre_bias));
            }
          }
        }
      }
    }
  }

  if (tid == 0) QTTS_TRACE_STAMP(6);
  // The consumer warps completed phase 0 of the cluster barrier (arrived at
  // start) before their remote stores; the producer warp completes it here.
  // Remote stores come from registers and each CTA waited for everything sent
  // to it, so the closing phase is not needed for memory safety: it makes the
  // CTAs of a cluster leave together. Measured on B200 in chained calls,
  // clusters whose CTAs exit one by one leave the next kernel's clusters
  // unplaced for microseconds (every other call of qkv at M = 1 stretched
  // from 4.3 to 9.5 us); with the closing phase the chain is the fastest.
  if (split > 1) {
    if (warp == kSkConsumerWarps) cluster_wait();
    cluster_arrive_relaxed();
    cluster_wait();
  }
  if (AG) ag_finish(a, ag_ep);
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

template <int MT, int R, typename XT, bool E4M3, bool AG, int PRO>
int launch_skinny_t(const CUtensorMap& map, const SkinnyArgs& args, dim3 grid, int split, size_t smem,
                    bool pdl, cudaStream_t stream) {
  auto kern = skinny_w8a16_kernel<MT, R, XT, E4M3, AG, PRO>;
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

template <int MT, typename XT, bool E4M3, bool AG = false, int PRO = kProNone>
int launch_skinny_r(int r, const CUtensorMap& map, const SkinnyArgs& args, dim3 grid, int split, size_t smem,
                    bool pdl, cudaStream_t stream) {
  switch (r) {
    case 1:
      return launch_skinny_t<MT, 1, XT, E4M3, AG, PRO>(map, args, grid, split, smem, pdl, stream);
    case 2:
      return launch_skinny_t<MT, 2, XT, E4M3, AG, PRO>(map, args, grid, split, smem, pdl, stream);
    case 4:
      return launch_skinny_t<MT, 4, XT, E4M3, AG, PRO>(map, args, grid, split, smem, pdl, stream);
    default:
      return launch_skinny_t<MT, 8, XT, E4M3, AG, PRO>(map, args, grid, split, smem, pdl, stream);
  }
}

template <typename XT>
int launch_skinny_mt(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, bool pdl,
                     cudaStream_t stream) {
  if (args.peer_out != nullptr) {
    // The all-gather form: int8 weights, up to 16 rows (AUTO's range for it).
    if (args.w_fmt != kWInt8) return QTTS_ERR_VARIANT;
    if (p.mt == 1) return launch_skinny_r<1, XT, false, true>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
    if (p.mt == 2) return launch_skinny_r<2, XT, false, true>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
    return QTTS_ERR_VARIANT;
  }
  if (args.prologue != kProNone) {
    // Fused prologues: int8 weights, up to 16 rows (AUTO's range for this kernel).
    if (args.w_fmt != kWInt8 || p.mt > 2) return QTTS_ERR_VARIANT;
    if (args.prologue == kProRmsNorm) {
      return p.mt == 1 ? launch_skinny_r<1, XT, false, false, kProRmsNorm>(p.r, map, args, p.grid, p.split, p.smem,
                                                                           pdl, stream)
                       : launch_skinny_r<2, XT, false, false, kProRmsNorm>(p.r, map, args, p.grid, p.split, p.smem,
                                                                           pdl, stream);
    }
    if (args.prologue == kProRmsNormRows) {
      return p.mt == 1 ? launch_skinny_r<1, XT, false, false, kProRmsNormRows>(p.r, map, args, p.grid, p.split,
                                                                               p.smem, pdl, stream)
                       : launch_skinny_r<2, XT, false, false, kProRmsNormRows>(p.r, map, args, p.grid, p.split,
                                                                               p.smem, pdl, stream);
    }
    return p.mt == 1 ? launch_skinny_r<1, XT, false, false, kProSiluMul>(p.r, map, args, p.grid, p.split, p.smem, pdl,
                                                                         stream)
                     : launch_skinny_r<2, XT, false, false, kProSiluMul>(p.r, map, args, p.grid, p.split, p.smem, pdl,
                                                                         stream);
  }
  if (args.w_fmt == kWE4M3) {
    // fp8 weight-only takes this kernel up to 16 rows only.
    if (p.mt == 1) return launch_skinny_r<1, XT, true>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
    if (p.mt == 2) return launch_skinny_r<2, XT, true>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
    return QTTS_ERR_VARIANT;
  }
  switch (p.mt) {
    case 1:
      return launch_skinny_r<1, XT, false>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
    case 2:
      return launch_skinny_r<2, XT, false>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
    case 4:
      return launch_skinny_r<4, XT, false>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
    default:
      return launch_skinny_r<8, XT, false>(p.r, map, args, p.grid, p.split, p.smem, pdl, stream);
  }
}

size_t skinny_smem(int mb, int bn, int x_pitch, int stages, int split) {
  const size_t xbytes = static_cast<size_t>(mb) * x_pitch * 2 + mb * 8;  // + row scales, norm factors
  const size_t recv = split > 1 ? static_cast<size_t>(bn) * mb * 4 : 0;
  return 1024 + static_cast<size_t>(stages) * kSkStageBytes + xbytes + recv + 16 + 16 * stages + 48;
}

int kpc_for(int K, int split, int sw) { return ((K + split - 1) / split + sw - 1) / sw * sw; }

}  // namespace

SkinnyPlan plan_skinny(int M, int N, int K, int G, int split_req, int r_req) {
  SkinnyPlan p{};
  p.mt = M <= 8 ? 1 : (M <= 16 ? 2 : (M <= 32 ? 4 : 8));
  const int mb = p.mt * 8;
  p.m_chunks = (M + mb - 1) / mb;
  const size_t x_cap = 64 * 1024;
  auto xbytes = [&](int s, int r) { return static_cast<size_t>(mb) * (kpc_for(K, s, 128 * (8 / r)) + 8) * 2; };
  auto ctas = [&](int s, int r) { return ((N + 16 * r - 1) / (16 * r)) * s * G * p.m_chunks; };
  const int splits[4] = {1, 2, 4, 8};
  const int rgs[4] = {8, 4, 2, 1};
  int split = split_req, r = r_req;
  if (split == 0 || r == 0) {
    // The most CTAs with work (a slice of K) among the plans that still run
    // two to an SM (the chained decode calls are latency-bound: two CTAs per
    // SM overlap each other's activation fetch, loop and split-K exchange),
    // activation slice within 48 KiB; ties go to the larger row tile, then the
    // smaller split. Slices are whole stages, so a split may leave its last
    // CTAs without K (they add zeros to the exchange). Measured on B200 in
    // chains of talker linears: qkv and down_proj at M = 1..16 gain 10-15 %
    // over one CTA per SM; code-predictor down (1024 x 3072) at M = 1 and 8
    // runs 4.5 / 5.0 us with 8 splits of 512 k (6 with work, 192 of 256 CTAs)
    // against 7.4 / 8.8 us with 2 splits of 16 rows (128 CTAs). Up to 8 rows,
    // plans whose CTAs hold at least two stages of K go first while they keep >= 128 CTAs
    // with work (row tiles of 64 or 128: narrower tiles reduce 4-8 k groups per
    // stage in shared memory): a one-stage CTA's fixed costs (activation staging, exchange)
    // are paid for 16 KiB of weights (talker o_proj 2048 x 2048 at M = 1..8:
    // 128 CTAs of 128 rows x 2 stages 3.8-3.9 us against 256 one-stage CTAs
    // 4.0-4.2 us; code-predictor qkv 4096 x 1024 3.7-3.9 against 4.1-4.2 us).
    // When every choice exceeds two per SM: the fewest CTAs.
    int best_c = -1, best_s = 0, best_r = 0, min_c = 0, min_s = 0, min_r = 0;
    int best2_c = -1, best2_s = 0, best2_r = 0;  // the same over plans of >= 2 stages per CTA
    for (int ri = 0; ri < 4; ++ri) {
      if (r != 0 && rgs[ri] != r) continue;
      for (int si = 0; si < 4; ++si) {
        if (split != 0 && splits[si] != split) continue;
        if (xbytes(splits[si], rgs[ri]) > 48 * 1024) continue;
        const int kpc = kpc_for(K, splits[si], 128 * (8 / rgs[ri]));
        const int with_k = min(splits[si], (K + kpc - 1) / kpc);
        const int c = ctas(splits[si], rgs[ri]);
        const int working = c / splits[si] * with_k;
        if (c <= kCtaSlots && working > best_c) {
          best_c = working;
          best_s = splits[si];
          best_r = rgs[ri];
        }
        if (c <= kCtaSlots && rgs[ri] >= 4 && kpc >= 2 * 128 * (8 / rgs[ri]) && working > best2_c) {
          best2_c = working;
          best2_s = splits[si];
          best2_r = rgs[ri];
        }
        if (min_c == 0 || c < min_c) {
          min_c = c;
          min_s = splits[si];
          min_r = rgs[ri];
        }
      }
    }
    if (p.mt == 1 && best2_c >= 128) {
      split = best2_s;
      r = best2_r;
    } else if (best_c > 0) {
      split = best_s;
      r = best_r;
    } else if (min_c > 0) {
      split = min_s;
      r = min_r;
    } else {
      // No activation slice fits 48 KiB: the largest split (smallest slice).
      if (r == 0) r = 8;
      if (split == 0) split = 8;
    }
  }
  (void)x_cap;
  p.split = split;
  p.r = r;
  const int bn = 16 * r;
  const int sw = 128 * (8 / r);
  p.k_per_cta = kpc_for(K, split, sw);
  p.x_pitch = p.k_per_cta + 8;  // +16 bytes: rows of one LDS phase hit distinct banks
  const int n_iters = p.k_per_cta / sw;
  // Stage ring: fill a ~100 KiB budget (two CTAs per SM), 2..6 stages, never
  // more than the slice needs; at least enough to hold the k-group reduction.
  // (Three CTAs per SM up to 8 rows -- 64 registers, 72 KiB -- measured 10-25 %
  // slower in chained calls.)
  const size_t fixed = skinny_smem(mb, bn, p.x_pitch, 0, split);
  const size_t budget = 100 * 1024;
  int stages = fixed < budget ? static_cast<int>((budget - fixed) / kSkStageBytes) : 0;
  stages = stages > 6 ? 6 : stages;
  stages = stages < n_iters ? stages : n_iters;
  const int min_stages = (512 * mb + kSkStageBytes - 1) / kSkStageBytes;
  stages = stages < min_stages ? min_stages : stages;
  stages = stages < 2 ? 2 : stages;
  p.stages = stages;
  p.smem = skinny_smem(mb, bn, p.x_pitch, stages, split);
  p.grid = dim3((N + bn - 1) / bn, split, G * p.m_chunks);
  return p;
}

int launch_skinny_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, int x_dtype,
                        bool pdl, cudaStream_t stream) {
  if (p.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
  if (x_dtype == QTTS_BF16) return launch_skinny_mt<__nv_bfloat16>(p, map, args, pdl, stream);
  if (x_dtype == QTTS_FP16) return launch_skinny_mt<__half>(p, map, args, pdl, stream);
  return QTTS_ERR_DTYPE;
}

}  // namespace qtts

#ifdef QTTS_TRACE
#include <atomic>
namespace qtts {
__device__ unsigned long long g_trace[kTraceSlots][kTraceEvents];
__device__ unsigned long long g_trace_detail[8][64];
static std::atomic<int> g_trace_slot{0};
int qtts_trace_next_slot() { return g_trace_slot.fetch_add(1) % 16; }
}  // namespace qtts
extern "C" __attribute__((visibility("default"))) int qtts_trace_read(void* dst, size_t bytes) {
  return cudaMemcpyFromSymbol(dst, qtts::g_trace, bytes) == cudaSuccess ? 0 : 9;
}
extern "C" __attribute__((visibility("default"))) void qtts_trace_reset(void) { qtts::g_trace_slot = 0; }
extern "C" __attribute__((visibility("default"))) int qtts_trace_read_detail(void* dst, size_t bytes) {
  return cudaMemcpyFromSymbol(dst, qtts::g_trace_detail, bytes) == cudaSuccess ? 0 : 9;
}
extern "C" __attribute__((visibility("default"))) int qtts_trace_clear(void) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, qtts::g_trace) != cudaSuccess) return 9;
  return cudaMemset(p, 0, sizeof(qtts::g_trace)) == cudaSuccess ? 0 : 9;
}
#endif
