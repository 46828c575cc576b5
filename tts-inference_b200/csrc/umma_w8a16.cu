// int8 weight-only GEMM (W8A16) on the 5th-generation tensor cores.
//
// Same contract as the skinny kernel and the reference's _w8_gemm_kernel
// (qtts/quant/kernels.py:89-135): out = cast(x @ (w * scale).T + bias) with an
// fp32 accumulator and the per-channel scale applied after the K loop.
//
// tcgen05 has no int8 x 16-bit MMA, so the weights are dequantized on the way
// into tensor memory:
//   * warp 8 (producer) streams the CTA's 128 weight rows x K slice HBM ->
//     shared memory as 2-D TMA boxes of 128 rows x 128 bytes (128-byte
//     swizzle), starting before the programmatic-dependent-launch wait; after
//     the wait it also brings each stage's activation tile [NB rows x 128 k]
//     in with TMA, already in the K-major 128-byte-swizzled layout the MMA
//     reads (B operand), straight from the caller's tensor;
//   * warps 0-7 (dequant) each take one 32-lane quarter of the rows and one
//     64-byte half of a stage: four 128-bit shared loads per thread (one row
//     segment), int8 -> the activations' 16-bit type in registers, exactly
//     (every int8 value has at most 8 significant bits: fp16 through the
//     0x64uu = 1024 + u pattern and one subtract per pair, bf16 through the
//     fp32 2^23 + u pattern, one subtract per weight and a truncating repack),
//     tcgen05.st into a ring of six A-operand slots in tensor memory (128
//     lanes x 32 columns = 64 k each). They run ahead of the previous
//     kernel's completion; only the epilogue waits for it. One MMA per 16 k
//     for either type: at decode N the tensor core is bound by instruction
//     issue, not by FLOPs (a 128-row MMA takes ~45 cycles back to back for
//     N <= 64, but a single issuing thread that also waits and commits gets
//     one out every ~60-150 cycles);
//   * warps 9 and 10 (MMA) issue tcgen05.mma kind::f16, A from tensor memory,
//     B from shared memory: warp 9 the first 64-k half of every 128-k stage,
//     warp 10 the second, each into its own fp32 accumulator [128 x NB] in
//     tensor memory (two issuing threads keep the tensor core at ~32 cycles
//     per MMA, measured); tcgen05.commit releases A slots and activation tiles
//     as they are used.
// The epilogue reads both accumulators with tcgen05.ld and adds them. K can be split over a
// cluster of CTAs whose partial sums reach the row owner through st.async, as
// in the skinny kernel. All waits are bounded; tensor memory is always
// released.
#include <type_traits>

#include "allgather.cuh"
#include "common.cuh"
#include "kernels.h"

namespace qtts {

constexpr int kUmStageBytes = 16384;  // 128 rows x 128 k
constexpr int kUmDqWarps = 8;
constexpr int kUmProducerWarp = 8;
constexpr int kUmMmaWarp = 9;    // first MMA issuer (also allocates tensor memory)
constexpr int kUmMmaWarp2 = 10;  // second MMA issuer
constexpr int kUmThreads = (kUmDqWarps + 3) * 32;
// Tensor-memory columns: the A ring (192, or 128 at NB = 128) and two
// accumulators of NB columns, rounded up to a power of two.
__host__ __device__ constexpr uint32_t umma_tmem_cols(int nb) {
  return ((nb > 64 ? 128 : 192) + 2 * nb) <= 256 ? 256u : 512u;
}
// A grid that takes all 512 columns also takes more than half of an SM's
// shared memory, so that no two of its CTAs share an SM (the second would wait
// in tcgen05.alloc for the first, which may wait on a cluster peer).
constexpr size_t kUmFullTmemMinSmem = 116 * 1024;

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

template <int NB, typename XT, bool E4M3 = false, bool AG = false>
__global__ void __launch_bounds__(kUmThreads, 1)
    umma_w8a16_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const SkinnyArgs a) {
  // Weights and activations share one 16-bit type per MMA: every int8 value is
  // exact in bf16 (8 significant bits) and in fp16, so one MMA per 16 k.
  constexpr uint32_t kFmt = std::is_same<XT, __nv_bfloat16>::value ? 1u : 0u;
  constexpr int HALF = NB / 2;      // accumulator columns per dequant warpgroup
  constexpr int XS = NB * 256;      // activation tile bytes per 128-k stage
  constexpr int kSlotCols = 32;     // tensor-memory columns per 64-k A slot
  // NB = 128 (M = 65..128 in one tile) keeps four A slots so that the two
  // accumulators' 2 x 128 columns fit beside them.
  constexpr int kACols = NB > 64 ? 128 : 192;
  constexpr int kNA = kACols / kSlotCols;  // A slots
  constexpr uint32_t kDCol = kACols;
  constexpr uint32_t kIdesc = umma_idesc(kFmt, kFmt, 128, NB);
  constexpr uint32_t kTmemCols = umma_tmem_cols(NB);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int split = gridDim.y;
  const int WS = a.stages;   // weight ring depth
  const int XD = a.x_pitch;  // activation ring depth (x_pitch carries it for this kernel)
  uint8_t* wbuf = smem;
  uint8_t* xbuf = wbuf + WS * kUmStageBytes;                   // [XD][2 boxes][NB rows][128 B]
  float* recv = reinterpret_cast<float*>(xbuf + XD * XS);      // [split][128/split][NB] when split > 1
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(recv + (split > 1 ? 128 * NB : 0)) + 15) & ~uintptr_t(15));
  uint64_t* wfull = bars;
  uint64_t* wempty = wfull + WS;
  uint64_t* xfull = wempty + WS;
  uint64_t* xempty = xfull + XD;
  uint64_t* afull = xempty + XD;   // [kNA]
  uint64_t* aempty = afull + kNA;  // [kNA]
  uint64_t* dfull = aempty + kNA;
  uint64_t* recv_bar = dfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  int* err_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* gate_flag = err_flag + 1;  // all-gather form: every rank is ready to receive

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int kidx = blockIdx.y;
  const uint32_t crank = split > 1 ? cluster_ctarank() : 0u;
  const int rpo = 128 / split;
  const int n0 = blockIdx.x * 128;
  const int mchunk = blockIdx.z % a.m_chunks;
  int group = blockIdx.z / a.m_chunks;
  const int m0 = mchunk * NB;
  const int k0 = kidx * a.k_per_cta;
  const int klen = max(0, min(a.K - k0, a.k_per_cta));
  int n_iters = (klen + 127) / 128;

  if (tid == 0) {
    QTTS_TRACE_STAMP(0);
    for (int s = 0; s < WS; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kUmDqWarps);
    }
    for (int s = 0; s < XD; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 2);  // one commit from each MMA issuer
    }
    for (int b = 0; b < kNA; ++b) {
      mbar_init(&afull[b], kUmDqWarps / 2);
      mbar_init(&aempty[b], 1);
    }
    mbar_init(dfull, 2);  // one commit from each MMA issuer
    mbar_init(recv_bar, 1);
    if (split > 1) mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((split - 1) * rpo * NB * 4));
    err_flag[0] = 0;
    fence_mbarrier_init();
  }
  if (warp == kUmMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  if (split > 1) cluster_arrive_relaxed();
  pdl_launch_dependents();
  if (AG && tid == 0) ag_prefetch_tables(a);

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
  const int xrow0 = static_cast<int>((a.group_index ? 0 : static_cast<int64_t>(group) * a.gsx_rows) + m0);
  const int64_t goff_o = a.group_index ? 0 : static_cast<int64_t>(group) * a.gso;
  XT* og = static_cast<XT*>(a.out) + goff_o + static_cast<int64_t>(m0) * a.ldo;
  const int mrows = min(NB, a.M - m0);
  volatile int* verr = err_flag;
  const int64_t pbase = static_cast<int64_t>(m0) * a.ldo + a.col_offset;  // all-gather form
  uint32_t ag_ep = 0;  // all-gather form: epoch of this call (dequant threads)

  int w_issued = 0, x_issued = 0;
  if (warp == kUmProducerWarp) {
    // ---------------- producer ----------------
    // Weights of the first WS stages before the dependency; then activation
    // tile `it` and weight stage `it + WS`, in that order.
    if (lane == 0 && n_iters > 0) {
      tma_prefetch_desc(&wmap);
      tma_prefetch_desc(&xmap);
      const int pre = min(WS, n_iters);
      for (int it = 0; it < pre; ++it) {
        mbar_arrive_expect_tx(&wfull[it], kUmStageBytes);
        tma_load_2d(wbuf + it * kUmStageBytes, &wmap, k0 + it * 128, static_cast<int>(wrow0), &wfull[it]);
      }
      w_issued = pre;
      pdl_wait();
      QTTS_TRACE_STAMP(1);
      for (int it = 0; it < n_iters; ++it) {
        const int xs = it % XD;
        if (it >= XD && !mbar_wait_bounded(&xempty[xs], ((it / XD) - 1) & 1, a.wait_ns)) {
          record_status(QTTS_ERR_TIMEOUT);
          *verr = 1;
          break;
        }
        mbar_arrive_expect_tx(&xfull[xs], XS);
        uint8_t* xt = xbuf + xs * XS;
        tma_load_2d(xt, &xmap, k0 + it * 128, xrow0, &xfull[xs]);
        tma_load_2d(xt + NB * 128, &xmap, k0 + it * 128 + 64, xrow0, &xfull[xs]);
        x_issued = it + 1;
        const int wi = it + WS;
        if (wi < n_iters) {
          const int s = wi % WS;
          if (!mbar_wait_bounded(&wempty[s], ((wi / WS) - 1) & 1, a.wait_ns)) {
            record_status(QTTS_ERR_TIMEOUT);
            *verr = 1;
            break;
          }
          mbar_arrive_expect_tx(&wfull[s], kUmStageBytes);
          tma_load_2d(wbuf + s * kUmStageBytes, &wmap, k0 + wi * 128, static_cast<int>(wrow0), &wfull[s]);
          w_issued = wi + 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == kUmMmaWarp || warp == kUmMmaWarp2) {
    // ---------------- MMA issuers: half h of every stage into accumulator h ----------------
    if (lane == 0) {
      const int h = warp - kUmMmaWarp;
      const uint32_t xaddr = smem_u32(xbuf);
      const uint32_t dcol = tmem + kDCol + static_cast<uint32_t>(h * NB);
      bool ok = true;
      for (int it = 0; ok && it < n_iters; ++it) {
        const int xs = it % XD;
        if (!mbar_wait_bounded(&xfull[xs], (it / XD) & 1, a.wait_ns)) {
          ok = false;
          break;
        }
        if (it == 0 && h == 0) QTTS_TRACE_STAMP(2);
        const int hs = 2 * it + h;
        const int slot = hs % kNA;
        if (!mbar_wait_bounded(&afull[slot], (hs / kNA) & 1, a.wait_ns)) {
          ok = false;
          break;
        }
        QTTS_TRACE_DETAIL(0, hs);
        tc_fence_after();
        const uint32_t acol = tmem + kSlotCols * slot;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint64_t bdesc = smem_desc_k_sw128(xaddr + xs * XS + h * (NB * 128) + i * 32);
          umma_f16_ts(dcol, acol + 8 * i, bdesc, kIdesc, (it | i) != 0 ? 1u : 0u);
        }
        tc_commit(&aempty[slot]);
        QTTS_TRACE_DETAIL(1, hs);
        tc_commit(&xempty[xs]);
      }
      if (!ok) {
        record_status(QTTS_ERR_TIMEOUT);
        *verr = 1;
      }
      if (h == 0) QTTS_TRACE_STAMP(3);
      tc_commit(dfull);  // arrives once every MMA this thread issued has completed
    }
    __syncwarp();
  } else {
    // ---------------- dequant warps: A operand into tensor memory, epilogue ----------------
    // They never wait on the previous kernel before the epilogue: the A ring
    // alone throttles them.
    const int quarter = warp & 3;
    const int half = warp >> 2;
    const int row = quarter * 32 + lane;  // weight row within the tile == TMEM lane
    // Scale and bias of the output channel this thread finishes (split 1: its
    // TMEM lane's row; split > 1: owned row tid mod the rows owned, which
    // divides 256): constants of the layer, loaded now so the epilogue does
    // not wait on them.
    float pre_sc = 0.f, pre_bias = 0.f;
    {
      const int n = n0 + (split > 1 ? static_cast<int>(crank) * rpo + tid % rpo : row);
      if (valid && n < a.N) {
        const int64_t ch = static_cast<int64_t>(group) * a.N + n;
        pre_sc = load_as_float(a.scale, a.scale_dtype, ch);
        if (a.bias != nullptr) pre_bias = to_float(static_cast<const XT*>(a.bias)[ch]);
      }
    }
    const uint32_t wbase = smem_u32(wbuf);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    for (int it = 0; ok && it < n_iters; ++it) {
      const int s = it % WS;
      const bool got = mbar_wait_bounded(&wfull[s], (it / WS) & 1, a.wait_ns);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      const int hs = 2 * it + half;
      if (lane == 0 && quarter == 0) QTTS_TRACE_DETAIL(2, hs);
      const uint32_t rb = wbase + s * kUmStageBytes + row * 128;
      uint4 v[4];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) v[cc] = lds128(rb + (((half * 4 + cc) ^ (row & 7)) << 4));
      uint32_t r1[32];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const uint32_t wd[4] = {v[cc].x, v[cc].y, v[cc].z, v[cc].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) WDequant<XT, E4M3>::run(wd[e], r1[8 * cc + 2 * e], r1[8 * cc + 2 * e + 1]);
      }
      // The weight stage goes back to the producer only after the conversions
      // above have consumed every loaded word (a TMA refill cannot overtake a
      // read of the stage).
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[s]);
      const int slot = hs % kNA;
      if (hs >= kNA) {
        const bool freed = mbar_wait_bounded(&aempty[slot], ((hs / kNA) - 1) & 1, a.wait_ns);
        if (!__all_sync(0xffffffffu, freed)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if (lane == 0 && quarter == 0) QTTS_TRACE_DETAIL(3, hs);
      tmem_st_x32(tmem + lane_base + kSlotCols * slot, r1);
      tc_wait_st();
      if (lane == 0 && quarter == 0) QTTS_TRACE_DETAIL(4, hs);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[slot]);
    }
    if (!ok) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *verr = 1;
    }

    // Epilogue: accumulator -> registers -> output (or the row owners).
    pdl_wait();
    if (tid == 0) QTTS_TRACE_STAMP(5);
    if (AG) ag_ep = ag_epoch(a);  // the load overlaps the accumulator wait
    const bool dready = mbar_wait_bounded(dfull, 0, a.wait_ns);
    // Every CTA announces (no wait depends on another CTA of this grid having started).
    if (AG && tid == 0) ag_announce_ready(a, ag_ep);
    if (!dready) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *verr = 1;
    }
    if (tid == 0) QTTS_TRACE_STAMP(6);
    tc_fence_after();
    uint32_t d[HALF];
    if constexpr (HALF <= 32) {
      tmem_ld<HALF>(tmem + lane_base + kDCol + HALF * half, d);
    } else {
      uint32_t (&d0)[32] = *reinterpret_cast<uint32_t(*)[32]>(d);
      uint32_t (&d1)[32] = *reinterpret_cast<uint32_t(*)[32]>(d + 32);
      tmem_ld<32>(tmem + lane_base + kDCol + HALF * half, d0);
      tmem_ld<32>(tmem + lane_base + kDCol + HALF * half + 32, d1);
    }
    tc_wait_ld();
    // The loaded registers are only valid after the wait: tie them to it.
#pragma unroll
    for (int c = 0; c < HALF; ++c) asm volatile("" : "+r"(d[c]));
    // The second issuer's accumulator (the other 64-k half of every stage).
    {
      constexpr int kC = HALF < 32 ? HALF : 32;
#pragma unroll
      for (int c0 = 0; c0 < HALF; c0 += kC) {
        uint32_t e[kC];
        tmem_ld<kC>(tmem + lane_base + kDCol + NB + HALF * half + c0, e);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < kC; ++c) asm volatile("" : "+r"(e[c]));
#pragma unroll
        for (int c = 0; c < kC; ++c) d[c0 + c] = __float_as_uint(__uint_as_float(d[c0 + c]) + __uint_as_float(e[c]));
      }
    }
    const bool cta_err = *verr != 0;
    float v[HALF];
#pragma unroll
    for (int c = 0; c < HALF; ++c) v[c] = (n_iters > 0 && !cta_err) ? __uint_as_float(d[c]) : 0.f;
    if (split == 1) {
      const int n = n0 + row;
      bool store_ok = valid && !cta_err;
      if (AG) store_ok = ag_gate_stores(a, ag_ep, gate_flag, 1, kUmDqWarps * 32, tid == 0) && store_ok;
      if (store_ok && n < a.N) {
#pragma unroll
        for (int c = 0; c < HALF; ++c) {
          const int col = HALF * half + c;
          if (col < mrows) put_out<AG>(a, og, pbase, static_cast<int64_t>(col) * a.ldo + n, from_float<XT>(v[c] * pre_sc + pre_bias));
        }
      }
    } else {
      // Partial sums travel to the row owner from registers (st.async into
      // its receive slot, counted on its mbarrier); a CTA's own rows go
      // through its own slot.
      cluster_wait();  // every peer's receive barrier is initialized
      const int owner = row / rpo;
      const int lr = row - owner * rpo;
      const int rrow = static_cast<int>(crank) * rpo + lr;
      if (owner == static_cast<int>(crank)) {
#pragma unroll
        for (int c = 0; c < HALF; c += 4)
          *reinterpret_cast<float4*>(recv + recv_offset(rrow, (HALF * half + c) >> 2, NB)) =
              make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
      } else {
        const uint32_t rbar = mapa_shared(smem_u32(recv_bar), owner);
#pragma unroll
        for (int c = 0; c < HALF; c += 4) {
          const uint32_t rdst = mapa_shared(smem_u32(recv + recv_offset(rrow, (HALF * half + c) >> 2, NB)), owner);
          st_async_f32x4(rdst, v[c], v[c + 1], v[c + 2], v[c + 3], rbar);
        }
      }
      named_bar_sync(1, kUmDqWarps * 32);
      bool have = mbar_wait_bounded(recv_bar, 0, a.wait_ns);
      if (!have) {
        if (tid == 0) record_status(QTTS_ERR_TIMEOUT);
        have = mbar_wait_bounded(recv_bar, 0, 4 * a.wait_ns);  // peers always send
      }
      if (AG) have = ag_gate_stores(a, ag_ep, gate_flag, 1, kUmDqWarps * 32, tid == 0) && have;
      if (have && valid && !cta_err) {
        // Thread = (owned row, 4 batch columns): one 16-byte load per peer.
        const int rbase = static_cast<int>(crank) * rpo;
        const int quads = (mrows + 3) / 4;
        for (int i = tid; i < rpo * quads; i += kUmDqWarps * 32) {
          const int mq = i / rpo;
          const int lr = i - mq * rpo;
          const int n = n0 + rbase + lr;
          if (n < a.N) {
            float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p = 0; p < split; ++p) {
              const float4 t = *reinterpret_cast<const float4*>(recv + recv_offset(p * rpo + lr, mq, NB));
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

  // Teardown: every tensor-memory access is complete before the columns are freed.
  tc_fence_before();
  __syncthreads();
  if (tid == 0) QTTS_TRACE_STAMP(7);
  if (warp == kUmMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  // The dequant warps waited on the cluster barrier before their remote
  // stores; the producer and MMA warps complete it here. Stores that came from
  // registers need no source kept alive, and each CTA waited for everything
  // sent to it.
  if (split > 1 && (warp == kUmProducerWarp || warp == kUmMmaWarp || warp == kUmMmaWarp2)) cluster_wait();
  if (AG) ag_finish(a, ag_ep);
  if (warp == kUmProducerWarp && lane == 0 && *verr != 0) {
    // Drain our own copies in flight (weights and activations).
    for (int s = 0; s < WS && s < w_issued; ++s) {
      const int last = ((w_issued - 1 - s) / WS) * WS + s;
      mbar_wait_bounded(&wfull[s], (last / WS) & 1, a.wait_ns);
    }
    for (int s = 0; s < XD && s < x_issued; ++s) {
      const int last = ((x_issued - 1 - s) / XD) * XD + s;
      mbar_wait_bounded(&xfull[s], (last / XD) & 1, a.wait_ns);
    }
  }
}

// ------------------------------------------------------------------------------------
// Host side

namespace {

template <int NB, typename XT, bool E4M3, bool AG>
int launch_umma_t(const CUtensorMap& map, const CUtensorMap& xmap, const SkinnyArgs& args, const SkinnyPlan& p,
                  bool pdl, cudaStream_t stream) {
  auto kern = umma_w8a16_kernel<NB, XT, E4M3, AG>;
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
  cfg.blockDim = dim3(kUmThreads, 1, 1);
  cfg.dynamicSmemBytes = umma_tmem_cols(NB) > 256 && p.smem < kUmFullTmemMinSmem ? kUmFullTmemMinSmem : p.smem;
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
  return cudaLaunchKernelEx(&cfg, kern, map, xmap, args) == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

template <typename XT, bool E4M3, bool AG = false>
int launch_umma_w(const CUtensorMap& map, const CUtensorMap& xmap, const SkinnyArgs& args, const SkinnyPlan& p,
                  bool pdl, cudaStream_t stream) {
  switch (p.mt) {
    case 2:
      return launch_umma_t<16, XT, E4M3, AG>(map, xmap, args, p, pdl, stream);
    case 4:
      return launch_umma_t<32, XT, E4M3, AG>(map, xmap, args, p, pdl, stream);
    case 8:
      return launch_umma_t<64, XT, E4M3, AG>(map, xmap, args, p, pdl, stream);
    default:
      return launch_umma_t<128, XT, E4M3, AG>(map, xmap, args, p, pdl, stream);
  }
}

template <typename XT>
int launch_umma_nb(const CUtensorMap& map, const CUtensorMap& xmap, const SkinnyArgs& args, const SkinnyPlan& p,
                   bool pdl, cudaStream_t stream) {
  if (args.peer_out != nullptr) {
    // The all-gather form: int8 weights only.
    return args.w_fmt == kWInt8 ? launch_umma_w<XT, false, true>(map, xmap, args, p, pdl, stream) : QTTS_ERR_VARIANT;
  }
  return args.w_fmt == kWE4M3 ? launch_umma_w<XT, true>(map, xmap, args, p, pdl, stream)
                              : launch_umma_w<XT, false>(map, xmap, args, p, pdl, stream);
}

size_t umma_smem(int nb, int wstages, int xstages, int split) {
  return 1024 + static_cast<size_t>(wstages) * kUmStageBytes + static_cast<size_t>(xstages) * nb * 256 + nb * 8 +
         (split > 1 ? static_cast<size_t>(128) * nb * 4 : 0) + 16 + 16 * wstages + 24 * xstages + 14 * 8 + 32;
}

}  // namespace

SkinnyPlan plan_umma(int M, int N, int K, int G, int split_req) {
  SkinnyPlan p{};
  const int n_tiles = (N + 127) / 128;
  // Batch columns per tile. Past 64 rows, 64-column tiles give more CTAs (each
  // redoing the dequantization and the MMAs of its weight tile: a 128-row
  // tcgen05.mma costs the same for any N), which pays while they fit one CTA
  // per SM; beyond that two tiles share an SM's tensor core and one
  // 128-column tile is faster. Measured on B200 at M = 128: talker gate_up
  // (96 weight tiles) 34.2 us as 64-column tiles, 18.9 us as one; the code
  // predictor's 1024-wide matrices (8..48 tiles) 8.0-10.5 us as 64-column
  // tiles, 10-20 % slower as one.
  int nb = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
  if (M > 64 && static_cast<long long>(n_tiles) * G * ((M + 63) / 64) > kNumSMs) nb = 128;
  p.mt = nb / 8;
  p.r = 8;
  p.m_chunks = (M + nb - 1) / nb;
  const int ctas_base = n_tiles * G * p.m_chunks;
  auto kpc_for = [&](int s) { return ((K + s - 1) / s + 127) / 128 * 128; };
  int split = split_req;
  if (split == 0) {
    // A tcgen05.mma of 128 rows costs about the same for any N <= 256, so with
    // decode-sized N the tensor core is bound by instruction count: spread
    // the tiles over as many SMs as possible, one CTA per SM, but keep the
    // K split within 4 CTAs (the exchange of larger clusters costs more than
    // it buys) except on the smallest grids (below).
    split = 1;
    for (int s_ = 1; s_ <= 4; s_ *= 2) {
      if (ctas_base * s_ <= kNumSMs) split = s_;
    }
    // Clusters of 8 pay on the smallest grids only: measured on B200 for the
    // code predictor's o_proj and down_proj (8 weight tiles, M = 24..64) 20-25 %
    // faster than clusters of 4 at 64 CTAs, but slower at 128 CTAs (o_proj,
    // down_proj of the talker, M = 128 as two 64-column tiles).
    if (split == 4 && ctas_base * 8 <= 64) split = 8;
  }
  p.split = split;
  p.k_per_cta = kpc_for(split);
  const int n_iters = p.k_per_cta / 128;
  // Activation ring: 4 tiles (never more than the slice); weight ring: fill
  // a ~100 KiB budget (grids whose tensor memory fills the SM are raised to
  // 116 KiB at launch). On long slices a deeper ring does not help (swept 2-12
  // weight stages, 2-4 activation stages, 100-220 KiB): a 128-k stage of 128
  // rows takes ~0.65 us per CTA in the dequant warps' chain (convert, store to
  // tensor memory, wait for the store, hand the slot to the MMA).
  const int xmax = nb > 64 ? 2 : 4;  // 32 KiB activation tiles at NB = 128
  int xstages = n_iters < xmax ? n_iters : xmax;
  xstages = xstages < 1 ? 1 : xstages;
  const size_t fixed = umma_smem(nb, 0, xstages, split);
  const size_t budget = 100 * 1024;
  int stages = fixed < budget ? static_cast<int>((budget - fixed) / kUmStageBytes) : 0;
  stages = stages > 6 ? 6 : stages;
  stages = stages < n_iters ? stages : n_iters;
  stages = stages < 2 ? 2 : stages;  // the ring also holds the 128 x NB fp32 partial sums at the end
  // A slice of up to 8 stages is held whole (up to 200 KiB): all of its weights are requested
  // before the dependency wait. Measured on B200 in chains at M = 64..128: talker o_proj
  // (4 stages) 6.84 -> 6.27 us, code-predictor gate_up 7.65 -> 7.46, down 7.88 -> 7.58; a
  // deeper ring on longer slices (talker gate_up, 16 stages) was 3 % slower.
  if (n_iters <= 8 && n_iters > stages && umma_smem(nb, n_iters, xstages, split) <= 200 * 1024) stages = n_iters;
  p.stages = stages;
  p.x_pitch = xstages;  // the tcgen05 kernel carries its activation ring depth here
  p.smem = umma_smem(nb, stages, xstages, split);
  p.grid = dim3(n_tiles, split, G * p.m_chunks);
  return p;
}

int launch_umma_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const CUtensorMap& xmap, const SkinnyArgs& args,
                      int x_dtype, bool pdl, cudaStream_t stream) {
  if (p.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
  if (x_dtype == QTTS_BF16) return launch_umma_nb<__nv_bfloat16>(map, xmap, args, p, pdl, stream);
  if (x_dtype == QTTS_FP16) return launch_umma_nb<__half>(map, xmap, args, p, pdl, stream);
  return QTTS_ERR_DTYPE;
}

}  // namespace qtts
