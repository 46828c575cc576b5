// Device-side building blocks shared by the sm_100a kernels of this library:
// mbarrier pipeline primitives with bounded waits, TMA tile loads, programmatic
// dependent launch controls, int8/e4m3 -> bf16/fp16 register dequantization and
// the legacy mma.sync fragments used by the skinny (decode-M) kernel.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qtts_b200.h"

namespace qtts {

// Per-device status word. Kernels record the first failure here (bounded wait
// expired, device-side index out of range); the host reads it with
// qtts_device_status(). Defined in capi.cu.
extern __device__ int g_device_status;
// Bounded-wait limit in nanoseconds, set per launch from the host.
struct WaitLimit {
  uint64_t ns;
};

__device__ __forceinline__ void record_status(int code) {
  atomicCAS(&g_device_status, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete. Gives up after
// `limit_ns` of wall time and returns false; the caller records the failure
// and takes its error path (which never waits unboundedly again).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// ---- TMA ----------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load into this CTA's shared memory, completion counted
// on `bar` in bytes. c0 is the innermost (contiguous) coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// ---- thread-block clusters ------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Split cluster barrier: arrive early (after the mbarriers are initialized and
// fenced), wait just before the first access to a peer's shared memory.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Store two floats into a peer CTA's shared memory; completion is counted in
// bytes on the peer's mbarrier.
__device__ __forceinline__ void st_async_f32(uint32_t remote_addr, float a, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(remote_addr),
               "r"(__float_as_uint(a)), "r"(remote_bar)
               : "memory");
}

__device__ __forceinline__ void st_async_f32x2(uint32_t remote_addr, float a, float b, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                   remote_addr),
               "f"(a), "f"(b), "r"(remote_bar)
               : "memory");
}

// ---- tcgen05 / tensor memory ----------------------------------------------------

// Allocates `ncols` (power of two >= 32) TMEM columns; the base address is
// written to shared memory. Executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Makes generic-proxy shared-memory writes visible to the async proxy
// (tensor-core operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// The mbarrier arrives once every tcgen05 operation this thread issued so far
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem desc], kind::f16 (fp16/bf16 in, fp32 accumulate).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n"
      "}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], kind::f8f6f4 (e4m3 in, fp32 accumulate).
__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc], kind::i8 (signed int8 in, int32 accumulate).
__device__ __forceinline__ void umma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n"
      "}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand in the canonical
// 128-byte-swizzled layout: 8-row x 128-byte atoms, atoms of consecutive row
// groups 1024 bytes apart (stride byte offset), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor: fp32 accumulator, A/B formats, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc(uint32_t a_fmt, uint32_t b_fmt, int m, int n) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
// Instruction descriptor for kind::i8: int32 accumulator (format 2), signed
// 8-bit A and B (format 1), both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}


__device__ __forceinline__ void st_async_f32x4(uint32_t remote_addr, float a, float b, float c, float d,
                                               uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   remote_addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(remote_bar)
               : "memory");
}

// ---- programmatic dependent launch ------------------------------------------

// Blocks until the preceding grid of the stream has completed and its memory
// operations are visible. A no-op when the kernel was launched without the
// programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allows the next grid of the stream (if launched with PDL) to start launching.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- split-K receive rows ------------------------------------------------------
// A receive row holds NB fp32 partial sums (NB / 4 chunks of 16 bytes). Chunk c
// of row r is stored at chunk c ^ (r & mask): writers keep 16-byte st.async
// stores, and a reader taking the same chunk of consecutive rows spreads over
// the banks instead of hitting one.
__host__ __device__ constexpr int recv_chunk_mask(int nb) { return (nb / 4 > 16 ? 16 : nb / 4) - 1; }
__device__ __forceinline__ int recv_offset(int row, int chunk, int nb) {
  return row * nb + ((chunk ^ (row & recv_chunk_mask(nb))) << 2);
}

// ---- named barriers ------------------------------------------------------------

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---- shared memory vector loads ------------------------------------------------

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}


// ---- int8 -> 16-bit float dequantization in registers ----------------------------
//
// A 32-bit word holds four int8 weights b0..b3 (little endian). Each routine
// returns two packed 16-bit pairs: lo = (b0, b1), hi = (b2, b3), exactly.
//
// bf16 route: bf16 has 8 significant bits, so a signed byte cannot be placed in
// one binade of it directly. Flip the sign bit (u = b + 128, 0..255), place u in
// the low mantissa byte of the fp32 2^23 (the exponent makes the mantissa an
// integer), subtract 2^23 + 128 in fp32 (exact), and keep the top half of each
// fp32 -- truncation is exact because |b| <= 128 needs at most 8 bits.
__device__ __forceinline__ void i8x4_to_bf16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const float kBias = 8388736.0f;  // 2^23 + 128
  const float f0 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - kBias;
  const float f1 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - kBias;
  const float f2 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - kBias;
  const float f3 = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - kBias;
  lo = __byte_perm(__float_as_uint(f0), __float_as_uint(f1), 0x7632);
  hi = __byte_perm(__float_as_uint(f2), __float_as_uint(f3), 0x7632);
}

// fp16 route: fp16 has 11 significant bits, so u = b + 128 fits the mantissa of
// 1024 (0x6400 | u == 1024 + u); one half-precision subtract of 1152 gives b.
__device__ __forceinline__ void i8x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a = __byte_perm(u, 0x64646464u, 0x4140);
  uint32_t b = __byte_perm(u, 0x64646464u, 0x4342);
  const uint32_t kBias = 0x64806480u;  // (1152, 1152) in fp16
  asm("sub.f16x2 %0, %1, %2;" : "=r"(lo) : "r"(a), "r"(kBias));
  asm("sub.f16x2 %0, %1, %2;" : "=r"(hi) : "r"(b), "r"(kBias));
}

// e4m3 weights (fp8 weight-only): every e4m3 value (3 mantissa bits, 2^-9 ..
// 448) is exact in fp16 and in bf16. Two bytes -> one f16 pair in a single
// conversion; bf16 goes through fp32 (exact) and a pair repack.
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const unsigned short w01 = static_cast<unsigned short>(w & 0xFFFFu);
  const unsigned short w23 = static_cast<unsigned short>(w >> 16);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(lo) : "h"(w01));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(hi) : "h"(w23));
}
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
  uint32_t r;
  asm("{\n.reg .f32 f0, f1;\n.reg .b16 h0, h1;\nmov.b32 {h0, h1}, %1;\ncvt.f32.f16 f0, h0;\ncvt.f32.f16 f1, h1;\n"
      "cvt.rn.bf16x2.f32 %0, f1, f0;\n}"
      : "=r"(r)
      : "r"(h));
  return r;
}
__device__ __forceinline__ void e4m3x4_to_bf16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  uint32_t a, b;
  e4m3x4_to_f16x2x2(w, a, b);
  lo = f16x2_to_bf16x2(a);
  hi = f16x2_to_bf16x2(b);
}

template <typename T>
struct Dequant;
template <>
struct Dequant<__nv_bfloat16> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& lo, uint32_t& hi) {
    i8x4_to_bf16x2x2(w, lo, hi);
  }
};
template <>
struct Dequant<__half> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& lo, uint32_t& hi) {
    i8x4_to_f16x2x2(w, lo, hi);
  }
};

// Weight format dispatch: int8 (W8A16) or e4m3 (fp8 weight-only).
template <typename T, bool kE4M3>
struct WDequant {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& lo, uint32_t& hi) { Dequant<T>::run(w, lo, hi); }
};
template <>
struct WDequant<__half, true> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& lo, uint32_t& hi) { e4m3x4_to_f16x2x2(w, lo, hi); }
};
template <>
struct WDequant<__nv_bfloat16, true> {
  static __device__ __forceinline__ void run(uint32_t w, uint32_t& lo, uint32_t& hi) { e4m3x4_to_bf16x2x2(w, lo, hi); }
};

// ---- mma.sync m16n8k16, fp32 accumulate ---------------------------------------------

template <typename T>
struct Mma16816;
template <>
struct Mma16816<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <>
struct Mma16816<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// ---- scalar conversions -----------------------------------------------------------

__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case QTTS_BF16:
      return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case QTTS_FP16:
      return __half2float(static_cast<const __half*>(p)[i]);
    default:
      return static_cast<const float*>(p)[i];
  }
}

template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_float<__half>(float v) {
  return __float2half_rn(v);
}
template <>
__device__ __forceinline__ float from_float<float>(float v) {
  return v;
}

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float to_float<__half>(__half v) {
  return __half2float(v);
}
template <>
__device__ __forceinline__ float to_float<float>(float v) {
  return v;
}

// Timeline probe, compiled in only with -DQTTS_TRACE (never in the shipped
// library): globaltimer stamps per CTA at each phase of a kernel, read back by
// qtts_trace_read(). `a` must be the kernel's argument block (trace_slot).
#ifdef QTTS_TRACE
constexpr int kTraceEvents = 8;
constexpr int kTraceSlots = 4096;
extern __device__ unsigned long long g_trace[kTraceSlots][kTraceEvents];
#define QTTS_TRACE_STAMP(ev)                                                             \
  do {                                                                                   \
    if (a.trace_slot >= 0) {                                                             \
      const int _c = a.trace_slot * 256 + blockIdx.x + gridDim.x * blockIdx.y;           \
      if (_c < kTraceSlots) g_trace[_c][ev] = globaltimer_ns();                          \
    }                                                                                    \
  } while (0)
// Per-step stamps of CTA (0,0,0) of trace slot 5: g_trace_detail[kind][step].
extern __device__ unsigned long long g_trace_detail[8][64];
#define QTTS_TRACE_DETAIL(kind, step)                                                               \
  do {                                                                                              \
    if (a.trace_slot == 5 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (step) < 64) \
      g_trace_detail[kind][step] = globaltimer_ns();                                                \
  } while (0)
#else
#define QTTS_TRACE_DETAIL(kind, step) \
  do {                                \
  } while (0)
#define QTTS_TRACE_STAMP(ev) \
  do {                       \
  } while (0)
#endif

}  // namespace qtts
