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
//     swizzle), starting before the programmatic-dependent-launch wait;
//   * warps 0-7 (dequant) each take one 32-lane quarter of the rows and one
//     64-byte half of a stage: four 128-bit shared loads per thread (one row
//     segment), int8 -> fp16 in registers (one byte-permute per two weights
//     plus a subtract; exact), then tcgen05.st into a double-buffered A
//     operand in tensor memory (128 lanes x 64 columns per 128-k stage);
//   * warp 9 (MMA) issues tcgen05.mma kind::f16 with A from tensor memory, the
//     activations as the B operand from shared memory (K-major, 128-byte
//     swizzle, N = 16/32/64 batch columns) and the fp32 accumulator in tensor
//     memory; tcgen05.commit releases each A buffer.
// The dequant warps convert the first two stages before the dependency wait,
// then stage the activations (fp16 with a per-row power-of-two scale, exact
// within 2^28 of the row maximum), then finish the stream. The epilogue reads
// the accumulator with tcgen05.ld. K can be split over a cluster of CTAs
// whose partial sums reach the row owner through st.async, as in the skinny
// kernel. All waits are bounded; tensor memory is always released.
#include "common.cuh"
#include "kernels.h"

namespace qtts {

constexpr int kUmStageBytes = 16384;  // 128 rows x 128 k
constexpr int kUmDqWarps = 8;
constexpr int kUmProducerWarp = 8;
constexpr int kUmMmaWarp = 9;
constexpr int kUmThreads = (kUmDqWarps + 2) * 32;
constexpr uint32_t kUmTmemCols = 256;  // A: 2 x 64 columns, D: up to 128 columns
constexpr uint32_t kUmDCol = 128;

__device__ __forceinline__ float um_pow2f(int e) { return __int_as_float((e + 127) << 23); }

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

// Byte offset of activation element (row n, k) in the B operand region:
// k-blocks of 64 elements, each [NB rows x 128 bytes] in 8-row x 128-byte
// atoms with the 16-byte chunks XOR-swizzled by (row % 8).
template <int NB>
__device__ __forceinline__ uint32_t xb_offset(int n, int k) {
  const int kb = k >> 6;
  const int c16 = (k & 63) >> 3;
  return kb * (NB * 128) + (n >> 3) * 1024 + (n & 7) * 128 + ((c16 ^ (n & 7)) << 4);
}

template <int NB, typename XT>
__global__ void __launch_bounds__(kUmThreads, 1)
    umma_w8a16_kernel(const __grid_constant__ CUtensorMap wmap, const SkinnyArgs a) {
  constexpr int HALF = NB / 2;  // accumulator columns per dequant warpgroup
  constexpr uint32_t kIdesc = umma_idesc(0u /*F16*/, 0u /*F16*/, 128, NB);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int split = gridDim.y;
  const int kpad_max = a.k_per_cta;  // multiple of 128
  uint8_t* wbuf = smem;
  uint8_t* xb = wbuf + a.stages * kUmStageBytes;  // B operand, NB x kpad_max fp16
  uint32_t* rowmax = reinterpret_cast<uint32_t*>(xb + NB * kpad_max * 2);
  float* xinv = reinterpret_cast<float*>(rowmax + NB);
  float* recv = xinv + NB;  // [128][NB] when split > 1
  uint64_t* bars = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(recv + (split > 1 ? 128 * NB : 0)) + 15) & ~uintptr_t(15));
  uint64_t* wfull = bars;
  uint64_t* wempty = wfull + a.stages;
  uint64_t* afull = wempty + a.stages;  // [2]
  uint64_t* aempty = afull + 2;         // [2]
  uint64_t* xready = aempty + 2;
  uint64_t* dfull = xready + 1;
  uint64_t* recv_bar = dfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv_bar + 1);
  int* err_flag = reinterpret_cast<int*>(tmem_slot + 1);

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
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], kUmDqWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&afull[b], kUmDqWarps);
      mbar_init(&aempty[b], 1);
    }
    mbar_init(xready, 1);
    mbar_init(dfull, 1);
    mbar_init(recv_bar, 1);
    if (split > 1) mbar_arrive_expect_tx(recv_bar, static_cast<uint32_t>((split - 1) * rpo * NB * 4));
    for (int i = 0; i < NB; ++i) rowmax[i] = 0u;
    *err_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == kUmMmaWarp) {
    tmem_alloc(tmem_slot, kUmTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  if (split > 1) cluster_arrive_relaxed();
  pdl_launch_dependents();

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
  const int mrows = min(NB, a.M - m0);
  volatile int* verr = err_flag;

  int n_issued = 0;
  if (warp == kUmProducerWarp) {
    // ---------------- producer: weight stream ----------------
    if (lane == 0 && n_iters > 0) {
      tma_prefetch_desc(&wmap);
      for (int it = 0; it < n_iters; ++it) {
        const int s = it % a.stages;
        if (it >= a.stages && !mbar_wait_bounded(&wempty[s], ((it / a.stages) - 1) & 1, a.wait_ns)) {
          record_status(QTTS_ERR_TIMEOUT);
          *verr = 1;
          break;
        }
        mbar_arrive_expect_tx(&wfull[s], kUmStageBytes);
        tma_load_2d(wbuf + s * kUmStageBytes, &wmap, k0 + it * 128, static_cast<int>(wrow0), &wfull[s]);
        n_issued = it + 1;
      }
    }
    __syncwarp();
  } else if (warp == kUmMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t xaddr = smem_u32(xb);
      bool ok = true;
      if (n_iters > 0 && !mbar_wait_bounded(xready, 0, a.wait_ns)) ok = false;
      for (int it = 0; ok && it < n_iters; ++it) {
        const int b = it & 1;
        if (!mbar_wait_bounded(&afull[b], (it >> 1) & 1, a.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int kb = it * 2 + (i >> 2);
          const uint32_t baddr = xaddr + kb * (NB * 128) + (i & 3) * 32;
          umma_f16_ts(tmem + kUmDCol, tmem + 64 * b + 8 * i, smem_desc_k_sw128(baddr), kIdesc,
                      (it | i) != 0 ? 1u : 0u);
        }
        tc_commit(&aempty[b]);
      }
      if (!ok) {
        record_status(QTTS_ERR_TIMEOUT);
        *verr = 1;
      }
      tc_commit(dfull);  // arrives once every MMA issued above has completed
    }
    __syncwarp();
  } else {
    // ---------------- dequant warps: A operand, activations, epilogue ----------------
    const int quarter = warp & 3;
    const int half = warp >> 2;
    const int row = quarter * 32 + lane;  // weight row within the tile == TMEM lane
    const uint32_t wbase = smem_u32(wbuf);
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;

    auto dequant_stage = [&](int it) {
      const int s = it % a.stages;
      const bool got = mbar_wait_bounded(&wfull[s], (it / a.stages) & 1, a.wait_ns);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        return;
      }
      const uint32_t rb = wbase + s * kUmStageBytes + row * 128;
      uint4 v[4];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) v[cc] = lds128(rb + (((half * 4 + cc) ^ (row & 7)) << 4));
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[s]);
      uint32_t r[32];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        i8x4_to_f16x2x2(v[cc].x, r[8 * cc + 0], r[8 * cc + 1]);
        i8x4_to_f16x2x2(v[cc].y, r[8 * cc + 2], r[8 * cc + 3]);
        i8x4_to_f16x2x2(v[cc].z, r[8 * cc + 4], r[8 * cc + 5]);
        i8x4_to_f16x2x2(v[cc].w, r[8 * cc + 6], r[8 * cc + 7]);
      }
      const int b = it & 1;
      if (it >= 2) {
        const bool freed = mbar_wait_bounded(&aempty[b], ((it >> 1) - 1) & 1, a.wait_ns);
        if (!__all_sync(0xffffffffu, freed)) {
          ok = false;
          return;
        }
        tc_fence_after();
      }
      tmem_st_x32(tmem + lane_base + 64 * b + 32 * half, r);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[b]);
    };

    // (1) The first two stages do not depend on the previous kernel.
    int it = 0;
    for (; ok && it < min(2, n_iters); ++it) dequant_stage(it);

    // (2) Activations: wait for the producer of x, stage it as the B operand.
    pdl_wait();
    {
      const int kpad = n_iters * 128;
      const int cpr = kpad / 8;  // 16-byte chunks per row
      const int total = NB * cpr;
      const int dq = tid;  // 0..255
      constexpr int kHeld = 4;
      uint4 held[kHeld];
      const bool in_regs = total <= kHeld * 256;
      // pass 1: load (or zero), row max
      for (int j = 0; j < (in_regs ? kHeld : (total + 255) / 256); ++j) {
        const int ci = dq + 256 * j;
        if (ci >= total) break;
        const int n = ci / cpr;
        const int k = (ci - n * cpr) * 8;
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (valid && n < mrows && k < klen) {
          u = __ldcg(reinterpret_cast<const uint4*>(xg + static_cast<int64_t>(n) * a.ldx + k0 + k));
        }
        const XT* e = reinterpret_cast<const XT*>(&u);
        float mx = 0.f;
#pragma unroll
        for (int q = 0; q < 8; ++q) mx = fmaxf(mx, fabsf(to_float(e[q])));
        if (mx > 0.f) atomicMax(&rowmax[n], __float_as_uint(mx));
        if (in_regs) {
          held[j < kHeld ? j : 0] = u;
        } else {
          *reinterpret_cast<uint4*>(xb + xb_offset<NB>(n, k)) = u;  // raw, converted in pass 2
        }
      }
      named_bar_sync(1, kUmDqWarps * 32);
      // pass 2: scale to fp16 in place
      for (int j = 0; j < (in_regs ? kHeld : (total + 255) / 256); ++j) {
        const int ci = dq + 256 * j;
        if (ci >= total) break;
        const int n = ci / cpr;
        const int k = (ci - n * cpr) * 8;
        const uint32_t off = xb_offset<NB>(n, k);
        const uint4 u = in_regs ? held[j < kHeld ? j : 0] : *reinterpret_cast<const uint4*>(xb + off);
        const float mxr = __uint_as_float(rowmax[n]);
        int sexp = 0;
        if (mxr > 0.f) sexp = min(max(14 - (static_cast<int>((__float_as_uint(mxr) >> 23) & 0xFF) - 127), -100), 100);
        const float sc = um_pow2f(sexp);
        const XT* e = reinterpret_cast<const XT*>(&u);
        uint4 o;
        __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) h[q] = __floats2half2_rn(to_float(e[2 * q]) * sc, to_float(e[2 * q + 1]) * sc);
        *reinterpret_cast<uint4*>(xb + off) = o;
      }
      if (dq < NB) {
        const float mxr = __uint_as_float(rowmax[dq]);
        int sexp = 0;
        if (mxr > 0.f) sexp = min(max(14 - (static_cast<int>((__float_as_uint(mxr) >> 23) & 0xFF) - 127), -100), 100);
        xinv[dq] = um_pow2f(-sexp);
      }
      fence_proxy_async_smem();
      named_bar_sync(1, kUmDqWarps * 32);
      if (dq == 0) mbar_arrive(xready);
    }

    // (3) The rest of the weight stream.
    for (; ok && it < n_iters; ++it) dequant_stage(it);
    if (!ok) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *verr = 1;
    }

    // (4) Epilogue: accumulator -> registers.
    const bool dready = mbar_wait_bounded(dfull, 0, a.wait_ns);
    if (!dready) {
      if (lane == 0) record_status(QTTS_ERR_TIMEOUT);
      *verr = 1;
    }
    tc_fence_after();
    uint32_t d[HALF];
    tmem_ld<HALF>(tmem + lane_base + kUmDCol + HALF * half, d);
    tc_wait_ld();
    const bool cta_err = *verr != 0;
    float v[HALF];
#pragma unroll
    for (int c = 0; c < HALF; ++c) {
      const int col = HALF * half + c;
      v[c] = (n_iters > 0 && !cta_err) ? __uint_as_float(d[c]) * xinv[col] : 0.f;
    }
    if (split == 1) {
      const int n = n0 + row;
      if (valid && !cta_err && n < a.N) {
        const int64_t ch = static_cast<int64_t>(group) * a.N + n;
        const float s = load_as_float(a.scale, a.scale_dtype, ch);
        const float bias = a.bias != nullptr ? to_float(static_cast<const XT*>(a.bias)[ch]) : 0.f;
#pragma unroll
        for (int c = 0; c < HALF; ++c) {
          const int col = HALF * half + c;
          if (col < mrows) og[static_cast<int64_t>(col) * a.ldo + n] = from_float<XT>(v[c] * s + bias);
        }
      }
    } else {
      cluster_wait();
      const int owner = row / rpo;
      const int lr = row - owner * rpo;
      float* dst = recv + (crank * rpo + lr) * NB + HALF * half;
      if (owner == static_cast<int>(crank)) {
#pragma unroll
        for (int c = 0; c < HALF; c += 2) *reinterpret_cast<float2*>(dst + c) = make_float2(v[c], v[c + 1]);
      } else {
        const uint32_t rdst = mapa_shared(smem_u32(dst), owner);
        const uint32_t rbar = mapa_shared(smem_u32(recv_bar), owner);
#pragma unroll
        for (int c = 0; c < HALF; c += 2) st_async_f32x2(rdst + c * 4, v[c], v[c + 1], rbar);
      }
      named_bar_sync(1, kUmDqWarps * 32);
      bool have = mbar_wait_bounded(recv_bar, 0, a.wait_ns);
      if (!have) {
        if (tid == 0) record_status(QTTS_ERR_TIMEOUT);
        have = mbar_wait_bounded(recv_bar, 0, 4 * a.wait_ns);  // peers always send
      }
      if (have && valid && !cta_err) {
        const int rbase = static_cast<int>(crank) * rpo;
        for (int i = tid; i < rpo * mrows; i += kUmDqWarps * 32) {
          const int m = i / rpo;
          const int lr2 = i - m * rpo;
          const int n = n0 + rbase + lr2;
          if (n < a.N) {
            float r = 0.f;
            for (int p = 0; p < split; ++p) r += recv[(p * rpo + lr2) * NB + m];
            const int64_t ch = static_cast<int64_t>(group) * a.N + n;
            r *= load_as_float(a.scale, a.scale_dtype, ch);
            if (a.bias != nullptr) r += to_float(static_cast<const XT*>(a.bias)[ch]);
            og[static_cast<int64_t>(m) * a.ldo + n] = from_float<XT>(r);
          }
        }
      }
    }
  }

  // Teardown: every tensor-memory access is complete before the columns are freed.
  tc_fence_before();
  __syncthreads();
  if (warp == kUmMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kUmTmemCols);
  }
  if (split > 1 && (warp == kUmProducerWarp || warp == kUmMmaWarp)) cluster_wait();
  if (warp == kUmProducerWarp && lane == 0 && *verr != 0) {
    for (int s = 0; s < a.stages && s < n_issued; ++s) {
      const int last = ((n_issued - 1 - s) / a.stages) * a.stages + s;
      mbar_wait_bounded(&wfull[s], (last / a.stages) & 1, a.wait_ns);
    }
  }
}

// ------------------------------------------------------------------------------------
// Host side

namespace {

template <int NB, typename XT>
int launch_umma_t(const CUtensorMap& map, const SkinnyArgs& args, const SkinnyPlan& p, bool pdl,
                  cudaStream_t stream) {
  auto kern = umma_w8a16_kernel<NB, XT>;
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
  return cudaLaunchKernelEx(&cfg, kern, map, args) == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

template <typename XT>
int launch_umma_nb(const CUtensorMap& map, const SkinnyArgs& args, const SkinnyPlan& p, bool pdl,
                   cudaStream_t stream) {
  switch (p.mt) {
    case 2:
      return launch_umma_t<16, XT>(map, args, p, pdl, stream);
    case 4:
      return launch_umma_t<32, XT>(map, args, p, pdl, stream);
    default:
      return launch_umma_t<64, XT>(map, args, p, pdl, stream);
  }
}

size_t umma_smem(int nb, int kpc, int stages, int split) {
  return 1024 + static_cast<size_t>(stages) * kUmStageBytes + static_cast<size_t>(nb) * kpc * 2 + nb * 8 +
         (split > 1 ? static_cast<size_t>(128) * nb * 4 : 0) + 16 + 16 * stages + 64 + 32;
}

}  // namespace

SkinnyPlan plan_umma(int M, int N, int K, int G, int split_req) {
  SkinnyPlan p{};
  const int nb = M <= 16 ? 16 : (M <= 32 ? 32 : 64);
  p.mt = nb / 8;
  p.r = 8;
  p.m_chunks = (M + nb - 1) / nb;
  const int n_tiles = (N + 127) / 128;
  const int ctas_base = n_tiles * G * p.m_chunks;
  auto kpc_for = [&](int s) { return ((K + s - 1) / s + 127) / 128 * 128; };
  int split = split_req;
  if (split == 0) {
    split = 8;
    for (int s = 1; s <= 8; s *= 2) {
      if (static_cast<size_t>(nb) * kpc_for(s) * 2 <= 64 * 1024 && ctas_base * s >= 120) {
        split = s;
        break;
      }
    }
  }
  p.split = split;
  p.k_per_cta = kpc_for(split);
  p.x_pitch = 0;
  const int n_iters = p.k_per_cta / 128;
  const size_t fixed = umma_smem(nb, p.k_per_cta, 0, split);
  const size_t budget = 100 * 1024;
  int stages = fixed < budget ? static_cast<int>((budget - fixed) / kUmStageBytes) : 0;
  stages = stages > 6 ? 6 : stages;
  stages = stages < n_iters ? stages : n_iters;
  stages = stages < 2 ? 2 : stages;
  p.stages = stages;
  p.smem = umma_smem(nb, p.k_per_cta, stages, split);
  p.grid = dim3(n_tiles, split, G * p.m_chunks);
  return p;
}

int launch_umma_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, int x_dtype, bool pdl,
                      cudaStream_t stream) {
  if (p.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
  if (x_dtype == QTTS_BF16) return launch_umma_nb<__nv_bfloat16>(map, args, p, pdl, stream);
  if (x_dtype == QTTS_FP16) return launch_umma_nb<__half>(map, args, p, pdl, stream);
  return QTTS_ERR_DTYPE;
}

}  // namespace qtts
