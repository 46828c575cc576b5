// C ABI of the library (include/qtts_b200.h): host-side validation, variant
// dispatch and the small kernels that need no pipeline -- the SIMT fallback
// GEMMs, the load-time weight quantizers and the per-token fp8 activation
// quantizer.
#include <cuda_fp8.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "prologue.cuh"

namespace qtts {

__device__ int g_device_status = 0;

namespace {

std::atomic<uint64_t> g_wait_limit_ns{2000000000ull};

bool is_float_dtype(int d) { return d == QTTS_BF16 || d == QTTS_FP16 || d == QTTS_FP32; }
size_t dtype_size(int d) {
  switch (d) {
    case QTTS_BF16:
    case QTTS_FP16:
      return 2;
    case QTTS_FP32:
      return 4;
    default:
      return 1;
  }
}
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---- device capability ------------------------------------------------------------
int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return QTTS_ERR_ARCH;
  static int cc_major[64] = {0};
  if (dev < 0 || dev >= 64) return QTTS_ERR_ARCH;
  if (cc_major[dev] == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return QTTS_ERR_ARCH;
    cc_major[dev] = major;
  }
  return cc_major[dev] == 10 ? QTTS_OK : QTTS_ERR_ARCH;
}

// ---- driver entry point for tensor-map encoding -------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// ---- SIMT fallback: W8A16 ---------------------------------------------------------
// One warp per output channel and up to 8 activation rows; lanes stride K.
struct GenericArgs {
  const void* x;
  int64_t ldx, gsx;
  const int8_t* w;  // int8 codes, or e4m3 bytes when w_fmt == kWE4M3
  int64_t ldw;
  const void* scale;
  int scale_dtype;
  const void* bias;
  void* out;
  int64_t ldo, gso;
  int M, N, K, G;
  const int64_t* group_index;
  int w_fmt;
};

__device__ __forceinline__ float e4m3_to_float(uint8_t v) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(v), __NV_E4M3);
  return __half2float(__half(h));
}

template <typename XT>
__global__ void __launch_bounds__(256) generic_w8a16_kernel(const GenericArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const int m0 = blockIdx.y * 8;
  int group = blockIdx.z;
  if (a.group_index != nullptr) {
    const int64_t gi = __ldcg(a.group_index);
    if (gi < 0 || gi >= a.G) {
      if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) record_status(QTTS_ERR_SHAPE);
      return;
    }
    group = static_cast<int>(gi);
  }
  if (n >= a.N) return;
  const int64_t ch = static_cast<int64_t>(group) * a.N + n;
  const int64_t goff_x = a.group_index ? 0 : static_cast<int64_t>(group) * a.gsx;
  const int64_t goff_o = a.group_index ? 0 : static_cast<int64_t>(group) * a.gso;
  const XT* xg = static_cast<const XT*>(a.x) + goff_x;
  XT* og = static_cast<XT*>(a.out) + goff_o;
  const int8_t* wr = a.w + ch * a.ldw;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int k = lane; k < a.K; k += 32) {
    const float wv = a.w_fmt == kWE4M3 ? e4m3_to_float(static_cast<uint8_t>(wr[k])) : static_cast<float>(wr[k]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (m0 + i < a.M) acc[i] += to_float(xg[static_cast<int64_t>(m0 + i) * a.ldx + k]) * wv;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (lane == 0) {
    const float s = load_as_float(a.scale, a.scale_dtype, ch);
    const float b = a.bias != nullptr ? to_float(static_cast<const XT*>(a.bias)[ch]) : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (m0 + i < a.M) og[static_cast<int64_t>(m0 + i) * a.ldo + n] = from_float<XT>(acc[i] * s + b);
    }
  }
}

template <typename KernT, typename ArgT>
int launch_simple(KernT kern, dim3 grid, dim3 block, const ArgT& args, bool pdl, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, args) == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

int launch_generic_w8a16(const GenericArgs& a, int x_dtype, bool pdl, cudaStream_t stream) {
  const int zg = a.group_index != nullptr ? 1 : a.G;
  const dim3 grid((a.N + 7) / 8, (a.M + 7) / 8, zg);
  if (grid.y > 65535u) return QTTS_ERR_SHAPE;
  switch (x_dtype) {
    case QTTS_BF16:
      return launch_simple(generic_w8a16_kernel<__nv_bfloat16>, grid, dim3(256), a, pdl, stream);
    case QTTS_FP16:
      return launch_simple(generic_w8a16_kernel<__half>, grid, dim3(256), a, pdl, stream);
    case QTTS_FP32:
      return launch_simple(generic_w8a16_kernel<float>, grid, dim3(256), a, pdl, stream);
    default:
      return QTTS_ERR_DTYPE;
  }
}

// ---- SIMT fallback: fp8 scaled GEMM --------------------------------------------------
struct GenericFp8Args {
  const uint8_t* xq;
  int64_t ldxq;
  const float* scale_x;
  const uint8_t* wq;
  int64_t ldw;
  const float* scale_w;
  const void* bias;
  void* out;
  int64_t ldo;
  int M, N, K;
};

template <typename OT>
__global__ void __launch_bounds__(256) generic_fp8_kernel(const GenericFp8Args a) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const int m0 = blockIdx.y * 8;
  if (n >= a.N) return;
  const uint8_t* wr = a.wq + static_cast<int64_t>(n) * a.ldw;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int k = lane; k < a.K; k += 32) {
    const float wv = e4m3_to_float(wr[k]);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (m0 + i < a.M) acc[i] += e4m3_to_float(a.xq[static_cast<int64_t>(m0 + i) * a.ldxq + k]) * wv;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (lane == 0) {
    const float sw = a.scale_w[n];
    const float b = a.bias != nullptr ? to_float(static_cast<const OT*>(a.bias)[n]) : 0.f;
    OT* o = static_cast<OT*>(a.out);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (m0 + i < a.M) {
        // _scaled_mm's output in the output dtype, then + bias in that dtype (qtts/quant/fp8.py:79-88).
        const float y = acc[i] * a.scale_x[m0 + i] * sw;
        o[static_cast<int64_t>(m0 + i) * a.ldo + n] =
            from_float<OT>(a.bias != nullptr ? __fadd_rn(to_float(from_float<OT>(y)), b) : y);
      }
    }
  }
}

// SIMT int8 W8A8 for shapes the tensor-core kernel cannot take: exact int32
// sums, epilogue in the reference's order (qtts/quant/int8.py:148-153).
template <typename OT>
__global__ void __launch_bounds__(256) generic_i8_kernel(const GenericFp8Args a) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp;
  const int m0 = blockIdx.y * 8;
  if (n >= a.N) return;
  const int8_t* wr = reinterpret_cast<const int8_t*>(a.wq) + static_cast<int64_t>(n) * a.ldw;
  const int8_t* xq = reinterpret_cast<const int8_t*>(a.xq);
  int acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0;
  for (int k = lane; k < a.K; k += 32) {
    const int wv = wr[k];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (m0 + i < a.M) acc[i] += static_cast<int>(xq[static_cast<int64_t>(m0 + i) * a.ldxq + k]) * wv;
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  }
  if (lane == 0) {
    const float sw = a.scale_w[n];
    OT* o = static_cast<OT*>(a.out);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (m0 + i < a.M) {
        float y = __fmul_rn(__fmul_rn(__int2float_rn(acc[i]), a.scale_x[m0 + i]), sw);
        if (a.bias != nullptr) y = __fadd_rn(y, to_float(static_cast<const OT*>(a.bias)[n]));
        o[static_cast<int64_t>(m0 + i) * a.ldo + n] = from_float<OT>(y);
      }
    }
  }
}

// ---- row quantizers ---------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float ld_elem(const void* p, int64_t i) {
  return to_float(static_cast<const T*>(p)[i]);
}

__device__ __forceinline__ float block_max_256(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) sh[warp] = v;
  __syncthreads();
  float r = sh[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) r = fmaxf(r, sh[i]);
  __syncthreads();
  return r;
}

// mode 0: int8 (quant/int8.py:45-56), mode 1: e4m3 weights (quant/fp8.py:45-49).
template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const void* w, int64_t ldw, void* q, float* scale,
                                                            int N, int K, int mode) {
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const int n = blockIdx.x;
  const int64_t row = static_cast<int64_t>(n) * ldw;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += 256) amax = fmaxf(amax, fabsf(ld_elem<T>(w, row + k)));
  amax = block_max_256(amax, sh);
  // ``amax / 127`` (``/ 448``) is a tensor divided by a Python number, which
  // torch evaluates on a CUDA tensor as a product with the fp32 reciprocal.
  const float s = fmaxf(amax, 1e-12f) * (mode == 0 ? 1.0f / 127.0f : 1.0f / 448.0f);
  if (threadIdx.x == 0) scale[n] = s;
  const int64_t qrow = static_cast<int64_t>(n) * K;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float v = ld_elem<T>(w, row + k) / s;
    if (mode == 0) {
      const float r = fminf(fmaxf(rintf(v), -127.0f), 127.0f);
      static_cast<int8_t*>(q)[qrow + k] = static_cast<int8_t>(r);
    } else {
      static_cast<uint8_t*>(q)[qrow + k] =
          static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
    }
  }
}

// Per-token activation quantization (quant/fp8.py:77-78). The amax and the
// clamp happen in the activation dtype (exact for a max), the division in fp32.
template <typename T>
__global__ void __launch_bounds__(256) fp8_quant_rows_kernel(const void* x, int64_t ldx, uint8_t* q, float* scale_x,
                                                             int M, int K) {
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int64_t row = static_cast<int64_t>(m) * ldx;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += 256) amax = fmaxf(amax, fabsf(ld_elem<T>(x, row + k)));
  amax = block_max_256(amax, sh);
  // clamp_min(1e-6) in the activation dtype: the bound is 1e-6 rounded to T.
  const float floor_t = to_float(from_float<T>(1e-6f));
  // ``.float() / 448`` on a CUDA tensor: a product with the fp32 reciprocal.
  const float s = fmaxf(amax, floor_t) * (1.0f / 448.0f);
  if (threadIdx.x == 0) scale_x[m] = s;
  const int64_t qrow = static_cast<int64_t>(m) * K;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float v = ld_elem<T>(x, row + k) / s;
    q[qrow + k] = static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
  }
}

// Per-token int8 activation quantization of Int8Method (qtts/quant/int8.py:138-140),
// every step in the activation dtype T as torch evaluates it on a CUDA tensor:
//   c  = amax.clamp_min(1e-6)               (T; the bound rounds to T)
//   s  = T(float(c) * fl32(1 / 127))        (tensor / number: fp32 reciprocal product)
//   q  = int8(clamp(rne(T(float(x) / float(s))), -127, 127))
// (x / s is a tensor-tensor division: IEEE fp32, rounded to T, then rounded
// half-to-even). scale_x receives float(s).
template <typename T>
__global__ void __launch_bounds__(256) int8_quant_rows_kernel(const void* x, int64_t ldx, int8_t* q, float* scale_x,
                                                              int M, int K) {
  __shared__ float sh[8];
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int64_t row = static_cast<int64_t>(m) * ldx;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += 256) amax = fmaxf(amax, fabsf(ld_elem<T>(x, row + k)));
  amax = block_max_256(amax, sh);
  const float c = fmaxf(amax, to_float(from_float<T>(1e-6f)));
  const float s = to_float(from_float<T>(c * (1.0f / 127.0f)));
  if (threadIdx.x == 0) scale_x[m] = s;
  const int64_t qrow = static_cast<int64_t>(m) * K;
  for (int k = threadIdx.x; k < K; k += 256) {
    const float v = rintf(to_float(from_float<T>(__fdiv_rn(ld_elem<T>(x, row + k), s))));
    // A zero scale (an all-zero fp16 row: 1e-6 / 127 underflows) gives 0 / 0;
    // torch carries the NaN through round and clamp and converts it to 0.
    q[qrow + k] = isnan(v) ? static_cast<int8_t>(0) : static_cast<int8_t>(fminf(fmaxf(v, -127.0f), 127.0f));
  }
}

}  // namespace

uint64_t current_wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

int make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_bytes,
                    uint32_t box_rows, uint32_t box_cols) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return QTTS_ERR_ARCH;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QTTS_OK : QTTS_ERR_ALIGN;
}

int make_tmap_16b_2d(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                     uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return QTTS_ERR_ARCH;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType t =
      dtype == QTTS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QTTS_OK : QTTS_ERR_ALIGN;
}

}  // namespace qtts

using namespace qtts;

// ======================================================================================
// Exported C ABI
// ======================================================================================

extern "C" {

int qtts_abi_version(void) { return QTTS_ABI_VERSION; }

const char* qtts_status_str(int status) {
  switch (status) {
    case QTTS_OK:
      return "ok";
    case QTTS_ERR_NULL:
      return "a required pointer is null";
    case QTTS_ERR_SHAPE:
      return "shape or leading dimension out of range";
    case QTTS_ERR_ALIGN:
      return "pointer or stride misaligned for the requested kernel";
    case QTTS_ERR_DTYPE:
      return "unsupported dtype";
    case QTTS_ERR_ARCH:
      return "no sm_100 device or missing driver entry point";
    case QTTS_ERR_LAUNCH:
      return "kernel launch failed";
    case QTTS_ERR_VARIANT:
      return "unknown or inapplicable kernel variant";
    case QTTS_ERR_TIMEOUT:
      return "device-side bounded wait expired";
    case QTTS_ERR_CUDA:
      return "CUDA runtime error";
    default:
      return "unknown status";
  }
}

int qtts_device_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return QTTS_ERR_CUDA;
  if (reset) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)) != cudaSuccess) return QTTS_ERR_CUDA;
  }
  return v;
}

uint64_t qtts_set_wait_limit_ns(uint64_t limit_ns) {
  return g_wait_limit_ns.exchange(limit_ns == 0 ? 2000000000ull : limit_ns);
}

// All-gather form of a call (qtts_w8a16_gemm_allgather); see csrc/allgather.cuh.
struct AllGatherForm {
  void* const* peer_out;
  uint32_t* const* peer_sig;
  uint32_t* sync;
  int64_t col_offset;
  int rank, world;
};

static void set_allgather(SkinnyArgs& sa, const AllGatherForm* ag) {
  sa.peer_out = ag != nullptr ? ag->peer_out : nullptr;
  sa.peer_sig = ag != nullptr ? ag->peer_sig : nullptr;
  sa.sync = ag != nullptr ? ag->sync : nullptr;
  sa.col_offset = ag != nullptr ? ag->col_offset : 0;
  sa.rank = ag != nullptr ? ag->rank : 0;
  sa.world = ag != nullptr ? ag->world : 1;
}

// AUTO's kernel for aligned 16-bit activations: 0x100 (split-K streaming), 0x200
// (tcgen05) or 0x300 (whole-K streaming, with its row groups in *rgroups).
// Up to 16 rows: the split-K streaming kernel with its planner's tile and split
// (up to two CTAs per SM), except at 9..16 rows where its CTAs would stream
// large slices (below). Past 16: the tcgen05 kernel, whose per-instruction
// cost does not grow with M. Up to 4 rows of int8, the whole-K streaming kernel
// where the split-K plan has more CTAs than SMs and the whole-K row tiles
// (16..96 rows) reach more CTAs within two per SM than it does (gate_up 12288 x 2048 at M = 1: 256 CTAs, 7.2 us, vs 192
// CTAs, 9.3 us, measured on B200).
static int auto_family(int M, int N, int K, int zg, int w_fmt, bool allgather, int* rgroups) {
  *rgroups = 0;
  if (M > 16) return 0x200;
  if (M > 8 && zg == 1) {
    // 9..16 rows: two 8-column MMA tiles per weight fragment double the
    // split-K kernel's mma.sync work, while a tcgen05 MMA costs the same for
    // any batch width; where the split-K plan streams >= 96 KiB per CTA the
    // tcgen05 kernel is faster (talker gate_up 12288 x 2048 at M = 12 / 16:
    // 12.8 / 12.8 us against 13.6 / 14.0 us; qkv, o_proj and down_proj, at
    // 32-48 KiB per CTA, stay on the split-K kernel).
    const SkinnyPlan sk = plan_skinny(M, N, K, zg, 0, 0);
    const long long ctas = static_cast<long long>(sk.grid.x) * sk.grid.y * sk.grid.z;
    if (ctas > 0 && static_cast<long long>(N) * K / ctas >= 96 * 1024) return 0x200;
  }
  int family = 0x100;
  if (M <= 4 && w_fmt == kWInt8 && !allgather) {
    const SkinnyPlan sk = plan_skinny(M, N, K, zg, 0, 0);
    int best = static_cast<int>(sk.grid.x * sk.grid.y * sk.grid.z);
    // Only where the split-K plan leaves SMs unevenly loaded (more CTAs than
    // SMs, some SMs with two): a plan of at most one CTA per SM is balanced
    // already (code-predictor qkv 4096 x 1024 at M = 4: 128 split-K CTAs
    // 3.9 us, the whole-K kernel's 256 CTAs 4.9 us).
    if (best <= kNumSMs) best = kCtaSlots;
    const int rows[5] = {6, 4, 3, 2, 1};
    for (int i = 0; i < 5; ++i) {
      const SkinnyPlan st = plan_stream(M, N, K, zg, rows[i]);
      const int c = static_cast<int>(st.grid.x * st.grid.y * st.grid.z);
      if (c <= kCtaSlots && c > best && st.smem <= kMaxDynSmem) {
        best = c;
        family = 0x300;
        *rgroups = rows[i];
      }
    }
  }
  return family;
}

// A prologue fused into the skinny or whole-K kernel (qtts_w8a16_gemm_prologue).
struct FusedPrologue {
  int kind;
  const void* weight;
  float eps;
};

static void set_prologue(SkinnyArgs& sa, const FusedPrologue* pro) {
  sa.prologue = pro != nullptr ? pro->kind : kProNone;
  sa.pro_weight = pro != nullptr ? pro->weight : nullptr;
  sa.pro_eps = pro != nullptr ? pro->eps : 0.f;
}

static int w8a16_dispatch(const void* x, int64_t gsx, int64_t ldx, int x_dtype, const int8_t* w, int64_t ldw,
                          const void* scale, int scale_dtype, const void* bias, void* out, int64_t gso,
                          int64_t ldo, int G, int M, int N, int K, const int64_t* group_index, int variant,
                          unsigned flags, void* stream_ptr, int w_fmt = kWInt8,
                          const AllGatherForm* ag = nullptr, const FusedPrologue* pro = nullptr) {
  if (M < 0 || N < 0 || K < 0 || G < 1) return QTTS_ERR_SHAPE;
  if (ag != nullptr && N == 0) return QTTS_ERR_SHAPE;  // every rank takes part in the exchange
  if (M == 0 || N == 0) return QTTS_OK;
  if (x == nullptr || w == nullptr || scale == nullptr || (out == nullptr && ag == nullptr)) return QTTS_ERR_NULL;
  if (!is_float_dtype(x_dtype) || !is_float_dtype(scale_dtype)) return QTTS_ERR_DTYPE;
  if (ldx < K || ldw < K || ldo < N) return QTTS_ERR_SHAPE;
  if (ag != nullptr && (ldo - ag->col_offset < N || G != 1 || group_index != nullptr)) return QTTS_ERR_SHAPE;
  if (G > 1 && group_index == nullptr && (gsx < static_cast<int64_t>(M) * ldx || gso < static_cast<int64_t>(M) * ldo))
    return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const bool pdl = (flags & QTTS_FLAG_PDL) != 0;
  const size_t xs = dtype_size(x_dtype);

  const bool skinny_ok = (x_dtype == QTTS_BF16 || x_dtype == QTTS_FP16) && K % 16 == 0 && K > 0 && aligned16(x) &&
                         aligned16(w) && (ldx * xs) % 16 == 0 && (gsx * xs) % 16 == 0 && ldw % 16 == 0;
  int family = variant & 0xF00;
  int split = variant & 0xF;
  int rgroups = (variant >> 4) & 0xF;
  if (variant == QTTS_VARIANT_AUTO) {
    family = skinny_ok ? auto_family(M, N, K, group_index != nullptr ? 1 : G, w_fmt, ag != nullptr, &rgroups) : 0;
    split = 0;
  }
  if (ag != nullptr && (family == 0 || family == 0x300)) {
    // The all-gather epilogue lives in the split-K and tcgen05 kernels.
    return skinny_ok ? QTTS_ERR_VARIANT : QTTS_ERR_ALIGN;
  }
  // Fused prologues live in the skinny and whole-K kernels (int8, M <= 16);
  // the caller has checked that the call lands there.
  if (pro != nullptr && !(skinny_ok && w_fmt == kWInt8 && M <= 16 && (family == 0x100 || family == 0x300)))
    return QTTS_ERR_VARIANT;
  if (variant == QTTS_VARIANT_GENERIC || family == 0) {
    if (variant != QTTS_VARIANT_AUTO && variant != QTTS_VARIANT_GENERIC) return QTTS_ERR_VARIANT;
    GenericArgs ga{x, ldx, gsx, w, ldw, scale, scale_dtype, bias, out, ldo, gso, M, N, K, G, group_index, w_fmt};
    return launch_generic_w8a16(ga, x_dtype, pdl, stream);
  }
  if (family == 0x300) {
    if (w_fmt != kWInt8) return QTTS_ERR_VARIANT;  // the whole-K kernel folds the int8 bias
    if (!skinny_ok) return QTTS_ERR_ALIGN;
    if (M > 16) return QTTS_ERR_VARIANT;
    if (!(rgroups == 0 || stream_rows_ok(rgroups))) return QTTS_ERR_VARIANT;
    if ((variant & 0xF00F) != 0) return QTTS_ERR_VARIANT;
    const int zg = group_index != nullptr ? 1 : G;
    SkinnyPlan plan = plan_stream(M, N, K, zg, rgroups);
    FusedPrologue pro_st{};
    if (pro != nullptr) {
      pro_st = *pro;
      if (pro->kind == kProRmsNorm) {
        // K a multiple of 256: the factors come from the staged rows ([MB][K / 256]
        // group sums kept past the barriers); otherwise from one more load of the rows.
        if (K % 256 == 0) {
          plan.smem += static_cast<size_t>(plan.mt) * 8 * 32 * 4;
        } else {
          pro_st.kind = kProRmsNormRows;
        }
      }
      pro = &pro_st;
    }
    if (plan.grid.z > 65535u || plan.grid.x > 2147483647u) return QTTS_ERR_SHAPE;
    if (plan.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
    CUtensorMap map;
    const uint64_t rows = static_cast<uint64_t>(G) * N;
    const int r = make_tmap_u8_2d(&map, w, rows, static_cast<uint64_t>(K), static_cast<uint64_t>(ldw),
                                  static_cast<uint32_t>(16 * plan.r), 128);
    if (r != QTTS_OK) return r;
    SkinnyArgs sa{};
    sa.x = x;
    sa.ldx = ldx;
    sa.gsx = gsx;
    sa.scale = scale;
    sa.scale_dtype = scale_dtype;
    sa.bias = bias;
    sa.out = out;
    sa.ldo = ldo;
    sa.gso = gso;
    sa.M = M;
    sa.N = N;
    sa.K = K;
    sa.G = G;
    sa.k_per_cta = plan.k_per_cta;
    sa.stages = plan.stages;
    sa.x_pitch = plan.x_pitch;
    sa.m_chunks = plan.m_chunks;
    sa.group_index = group_index;
    sa.w_fmt = w_fmt;
    set_allgather(sa, ag);
    set_prologue(sa, pro);
    sa.wait_ns = current_wait_limit_ns();
    sa.trace_slot = -1;
#ifdef QTTS_TRACE
    sa.trace_slot = qtts_trace_next_slot();
#endif
    return launch_stream_w8a16(plan, map, sa, x_dtype, pdl, stream);
  }
  if (family == 0x100) {
    if (!skinny_ok) return QTTS_ERR_ALIGN;
    if (w_fmt == kWE4M3 && M > 16) return QTTS_ERR_VARIANT;
    if (!(split == 0 || split == 1 || split == 2 || split == 4 || split == 8)) return QTTS_ERR_VARIANT;
    if (!(rgroups == 0 || rgroups == 1 || rgroups == 2 || rgroups == 4 || rgroups == 8)) return QTTS_ERR_VARIANT;
    if ((variant & 0xF000) != 0) return QTTS_ERR_VARIANT;
    const int zg = group_index != nullptr ? 1 : G;
    SkinnyPlan plan = plan_skinny(M, N, K, zg, split, rgroups);
    FusedPrologue pro_sk{};
    if (pro != nullptr) {
      pro_sk = *pro;
      if (pro->kind == kProRmsNorm) {
        // Slices aligned to the norm's 256-column groups: each CTA sums its own
        // slice and the cluster exchanges the group sums ([MB][K / 256] floats
        // kept past the barriers); otherwise the CTAs load the rows once more.
        if (K % 256 == 0 && plan.k_per_cta % 256 == 0) {
          plan.smem += static_cast<size_t>(plan.mt) * 8 * 32 * 4;
        } else {
          pro_sk.kind = kProRmsNormRows;
        }
      }
      pro = &pro_sk;
    }
    if (plan.grid.z > 65535u) return QTTS_ERR_SHAPE;
    if (plan.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;  // activation slice does not fit this split
    CUtensorMap map;
    const uint64_t rows = static_cast<uint64_t>(G) * N;
    const int r = make_tmap_u8_2d(&map, w, rows, static_cast<uint64_t>(K), static_cast<uint64_t>(ldw),
                                  static_cast<uint32_t>(16 * plan.r), 128);
    if (r != QTTS_OK) return r;
    SkinnyArgs sa{};
    sa.x = x;
    sa.ldx = ldx;
    sa.gsx = gsx;
    sa.scale = scale;
    sa.scale_dtype = scale_dtype;
    sa.bias = bias;
    sa.out = out;
    sa.ldo = ldo;
    sa.gso = gso;
    sa.M = M;
    sa.N = N;
    sa.K = K;
    sa.G = G;
    sa.k_per_cta = plan.k_per_cta;
    sa.stages = plan.stages;
    sa.x_pitch = plan.x_pitch;
    sa.m_chunks = plan.m_chunks;
    sa.group_index = group_index;
    sa.w_fmt = w_fmt;
    set_allgather(sa, ag);
    set_prologue(sa, pro);
    sa.wait_ns = current_wait_limit_ns();
    sa.trace_slot = -1;
#ifdef QTTS_TRACE
    sa.trace_slot = qtts_trace_next_slot();
#endif
    return launch_skinny_w8a16(plan, map, sa, x_dtype, pdl, stream);
  }
  if (family == 0x200) {
    if (!skinny_ok) return QTTS_ERR_ALIGN;
    if (!(split == 0 || split == 1 || split == 2 || split == 4 || split == 8) || rgroups != 0) return QTTS_ERR_VARIANT;
    if ((variant & 0xF000) != 0) return QTTS_ERR_VARIANT;
    const int zg = group_index != nullptr ? 1 : G;
    if (group_index == nullptr && G > 1 && gsx % ldx != 0) return QTTS_ERR_ALIGN;
    const SkinnyPlan plan = plan_umma(M, N, K, zg, split);
    if (plan.grid.z > 65535u) return QTTS_ERR_SHAPE;
    if (plan.smem > kMaxDynSmem) return QTTS_ERR_VARIANT;
    CUtensorMap map, xmap;
    const uint64_t rows = static_cast<uint64_t>(G) * N;
    int r = make_tmap_u8_2d(&map, w, rows, static_cast<uint64_t>(K), static_cast<uint64_t>(ldw), 128, 128);
    if (r != QTTS_OK) return r;
    const int64_t gsx_rows = (group_index == nullptr && G > 1) ? gsx / ldx : 0;
    const uint64_t xrows = static_cast<uint64_t>(gsx_rows) * (group_index == nullptr ? G - 1 : 0) + M;
    r = make_tmap_16b_2d(&xmap, x, x_dtype, xrows, static_cast<uint64_t>(K), static_cast<uint64_t>(ldx) * 2,
                         static_cast<uint32_t>(plan.mt * 8), 64);
    if (r != QTTS_OK) return r;
    SkinnyArgs sa{};
    sa.x = x;
    sa.ldx = ldx;
    sa.gsx = gsx;
    sa.scale = scale;
    sa.scale_dtype = scale_dtype;
    sa.bias = bias;
    sa.out = out;
    sa.ldo = ldo;
    sa.gso = gso;
    sa.M = M;
    sa.N = N;
    sa.K = K;
    sa.G = G;
    sa.k_per_cta = plan.k_per_cta;
    sa.stages = plan.stages;
    sa.x_pitch = plan.x_pitch;  // activation ring depth
    sa.m_chunks = plan.m_chunks;
    sa.group_index = group_index;
    sa.w_fmt = w_fmt;
    set_allgather(sa, ag);
    set_prologue(sa, pro);
    sa.wait_ns = current_wait_limit_ns();
    sa.trace_slot = -1;
#ifdef QTTS_TRACE
    sa.trace_slot = qtts_trace_next_slot();
#endif
    sa.gsx_rows = gsx_rows;
    return launch_umma_w8a16(plan, map, xmap, sa, x_dtype, pdl, stream);
  }
  return QTTS_ERR_VARIANT;
}

int qtts_w8a16_gemm(const void* x, int64_t ldx, int x_dtype, const int8_t* w, int64_t ldw, const void* scale,
                    int scale_dtype, const void* bias, void* out, int64_t ldo, int M, int N, int K, int variant,
                    unsigned flags, void* stream) {
  return w8a16_dispatch(x, 0, ldx, x_dtype, w, ldw, scale, scale_dtype, bias, out, 0, ldo, 1, M, N, K, nullptr,
                        variant, flags, stream);
}

int qtts_fp8w_gemm(const void* x, int64_t ldx, int x_dtype, const uint8_t* w, int64_t ldw, const void* scale,
                   int scale_dtype, const void* bias, void* out, int64_t ldo, int M, int N, int K, int variant,
                   unsigned flags, void* stream) {
  return w8a16_dispatch(x, 0, ldx, x_dtype, reinterpret_cast<const int8_t*>(w), ldw, scale, scale_dtype, bias, out,
                        0, ldo, 1, M, N, K, nullptr, variant, flags, stream, kWE4M3);
}

// ---- activation prologues ------------------------------------------------------------

int qtts_rms_norm(const void* x, int64_t ldx, const void* weight, void* out, int64_t ldo, int dtype, int rows,
                  int width, float eps, unsigned flags, void* stream) {
  if (rows < 0 || width < 0 || width > 8 * 32 * kMaxNormGroups) return QTTS_ERR_SHAPE;
  if (rows == 0 || width == 0) return QTTS_OK;
  if (x == nullptr || weight == nullptr || out == nullptr) return QTTS_ERR_NULL;
  if (!is_float_dtype(dtype)) return QTTS_ERR_DTYPE;
  if (ldx < width || ldo < width) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  const size_t sz = dtype_size(dtype);
  PrologueArgs pa{};
  pa.kind = kProRmsNorm;
  pa.x = x;
  pa.ldx = ldx;
  pa.weight = weight;
  pa.eps = eps;
  pa.out = out;
  pa.ldo = ldo;
  pa.rows = rows;
  pa.width = width;
  pa.vec = width % 8 == 0 && aligned16(x) && aligned16(weight) && aligned16(out) && (ldx * sz) % 16 == 0 &&
           (ldo * sz) % 16 == 0;
  return launch_prologue(pa, dtype, (flags & QTTS_FLAG_PDL) != 0, static_cast<cudaStream_t>(stream));
}

int qtts_silu_mul(const void* gate_up, int64_t ld_in, void* out, int64_t ldo, int dtype, int rows, int width,
                  unsigned flags, void* stream) {
  if (rows < 0 || width < 0) return QTTS_ERR_SHAPE;
  if (rows == 0 || width == 0) return QTTS_OK;
  if (gate_up == nullptr || out == nullptr) return QTTS_ERR_NULL;
  if (!is_float_dtype(dtype)) return QTTS_ERR_DTYPE;
  if (ld_in < 2 * static_cast<int64_t>(width) || ldo < width) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  const size_t sz = dtype_size(dtype);
  PrologueArgs pa{};
  pa.kind = kProSiluMul;
  pa.x = gate_up;
  pa.ldx = ld_in;
  pa.out = out;
  pa.ldo = ldo;
  pa.rows = rows;
  pa.width = width;
  pa.vec = width % 8 == 0 && aligned16(gate_up) && aligned16(out) && (ld_in * sz) % 16 == 0 && (ldo * sz) % 16 == 0;
  return launch_prologue(pa, dtype, (flags & QTTS_FLAG_PDL) != 0, static_cast<cudaStream_t>(stream));
}

int qtts_w8a16_head_argmax(const void* x, int64_t ldx, int x_dtype, const void* norm_weight, float eps,
                           const int8_t* w, int64_t ldw, const void* scale, int scale_dtype, const float* logit_bias,
                           int64_t* codes, const void* embed, int64_t lde, int vocab, void* embed_out, int64_t ldeo,
                           int E, uint64_t* state, int M, int N, int K, unsigned flags, void* stream) {
  if (M < 0 || N < 0 || K < 0 || E < 0 || vocab < 0) return QTTS_ERR_SHAPE;
  if (M == 0) return QTTS_OK;
  if (x == nullptr || w == nullptr || scale == nullptr || codes == nullptr || state == nullptr) return QTTS_ERR_NULL;
  if (embed != nullptr && embed_out == nullptr) return QTTS_ERR_NULL;
  if (x_dtype != QTTS_BF16 && x_dtype != QTTS_FP16) return QTTS_ERR_DTYPE;
  if (!is_float_dtype(scale_dtype)) return QTTS_ERR_DTYPE;
  if (M > 16 || N < 1 || K < 128 || K > 2048 || K % 128 != 0) return QTTS_ERR_SHAPE;
  if (ldx < K || ldw < K) return QTTS_ERR_SHAPE;
  if (embed != nullptr && (E < 8 || E % 8 != 0 || lde < E || ldeo < E || vocab < 1)) return QTTS_ERR_SHAPE;
  if (!aligned16(x) || (ldx * 2) % 16 != 0 || (norm_weight != nullptr && !aligned16(norm_weight))) {
    return QTTS_ERR_ALIGN;
  }
  if ((reinterpret_cast<uintptr_t>(w) & 3u) != 0 || ldw % 4 != 0) return QTTS_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(state) & 7u) != 0) return QTTS_ERR_ALIGN;
  if (embed != nullptr && (!aligned16(embed) || !aligned16(embed_out) || (lde * 2) % 16 != 0 || (ldeo * 2) % 16 != 0)) {
    return QTTS_ERR_ALIGN;
  }
  if (head_argmax_smem(M, K) + 1024 > kMaxDynSmem) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  HeadArgs ha{};
  ha.x = x;
  ha.ldx = ldx;
  ha.norm_weight = norm_weight;
  ha.eps = eps;
  ha.w = w;
  ha.ldw = ldw;
  ha.scale = scale;
  ha.scale_dtype = scale_dtype;
  ha.logit_bias = logit_bias;
  ha.codes = codes;
  ha.embed = embed;
  ha.lde = lde;
  ha.embed_out = embed_out;
  ha.ldeo = ldeo;
  ha.E = E;
  ha.vocab = vocab;
  ha.state = reinterpret_cast<unsigned long long*>(state);
  ha.M = M;
  ha.N = N;
  ha.K = K;
  return launch_head_argmax(ha, x_dtype, (flags & QTTS_FLAG_PDL) != 0, static_cast<cudaStream_t>(stream));
}

// Which kernel family the call lands on (the same choice w8a16_dispatch makes).
static int chosen_family(const void* x, int64_t ldx, int x_dtype, const int8_t* w, int64_t ldw, int M, int N, int K,
                         int variant) {
  const size_t xs = dtype_size(x_dtype);
  const bool skinny_ok = (x_dtype == QTTS_BF16 || x_dtype == QTTS_FP16) && K % 16 == 0 && K > 0 && aligned16(x) &&
                         aligned16(w) && (ldx * xs) % 16 == 0 && ldw % 16 == 0;
  if (variant == QTTS_VARIANT_GENERIC) return 0;
  if (variant != QTTS_VARIANT_AUTO) return skinny_ok ? (variant & 0xF00) : -1;
  int rgroups = 0;
  return skinny_ok ? auto_family(M, N, K, 1, kWInt8, false, &rgroups) : 0;
}

int qtts_w8a16_gemm_prologue(const void* x, int64_t ldx, int x_dtype, int prologue, const void* norm_weight,
                             float eps, const int8_t* w, int64_t ldw, const void* scale, int scale_dtype,
                             const void* bias, void* out, int64_t ldo, int M, int N, int K, void* workspace,
                             int variant, unsigned flags, void* stream) {
  if (prologue == QTTS_PROLOGUE_NONE) {
    return w8a16_dispatch(x, 0, ldx, x_dtype, w, ldw, scale, scale_dtype, bias, out, 0, ldo, 1, M, N, K, nullptr,
                          variant, flags, stream);
  }
  if (prologue != QTTS_PROLOGUE_RMSNORM && prologue != QTTS_PROLOGUE_SILU_MUL) return QTTS_ERR_VARIANT;
  if (M < 0 || N < 0 || K < 0) return QTTS_ERR_SHAPE;
  if (M == 0 || N == 0) return QTTS_OK;
  if (x == nullptr || w == nullptr || scale == nullptr || out == nullptr) return QTTS_ERR_NULL;
  if (prologue == QTTS_PROLOGUE_RMSNORM && norm_weight == nullptr) return QTTS_ERR_NULL;
  if (!is_float_dtype(x_dtype) || !is_float_dtype(scale_dtype)) return QTTS_ERR_DTYPE;
  const int64_t x_width = prologue == QTTS_PROLOGUE_SILU_MUL ? 2 * static_cast<int64_t>(K) : K;
  if (ldx < x_width || ldw < K || ldo < N) return QTTS_ERR_SHAPE;
  const int family = chosen_family(x, ldx, x_dtype, w, ldw, M, N, K, variant);
  if (family < 0) return QTTS_ERR_ALIGN;
  const bool fusable = M <= 16 && (family == 0x100 || family == 0x300) &&
                       (prologue != QTTS_PROLOGUE_RMSNORM || (aligned16(norm_weight) && K <= 8 * 32 * kMaxFusedNormGroups));
  if (fusable) {
    const FusedPrologue pro{prologue == QTTS_PROLOGUE_RMSNORM ? kProRmsNorm : kProSiluMul, norm_weight, eps};
    return w8a16_dispatch(x, 0, ldx, x_dtype, w, ldw, scale, scale_dtype, bias, out, 0, ldo, 1, M, N, K, nullptr,
                          variant, flags, stream, kWInt8, nullptr, &pro);
  }
  // Two launches: the prologue writes the activation into the workspace
  // [M, K] (leading dimension K), then the GEMM reads it. The GEMM launches
  // with programmatic dependent launch behind the prologue kernel, which
  // writes no weights.
  if (workspace == nullptr) return QTTS_ERR_NULL;
  if (prologue == QTTS_PROLOGUE_RMSNORM && K > 8 * 32 * kMaxNormGroups) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  const size_t sz = dtype_size(x_dtype);
  PrologueArgs pa{};
  pa.kind = prologue == QTTS_PROLOGUE_RMSNORM ? kProRmsNorm : kProSiluMul;
  pa.x = x;
  pa.ldx = ldx;
  pa.weight = norm_weight;
  pa.eps = eps;
  pa.out = workspace;
  pa.ldo = K;
  pa.rows = M;
  pa.width = K;
  pa.vec = K % 8 == 0 && aligned16(x) && aligned16(workspace) && (ldx * sz) % 16 == 0 && (K * sz) % 16 == 0 &&
           (pa.kind != kProRmsNorm || aligned16(norm_weight));
  const int r = launch_prologue(pa, x_dtype, (flags & QTTS_FLAG_PDL) != 0, static_cast<cudaStream_t>(stream));
  if (r != QTTS_OK) return r;
  return w8a16_dispatch(workspace, 0, K, x_dtype, w, ldw, scale, scale_dtype, bias, out, 0, ldo, 1, M, N, K, nullptr,
                        variant, flags | QTTS_FLAG_PDL, stream);
}

int qtts_w8a16_gemm_prologue_fused(int M, int N, int K, int prologue, int variant) {
  if (M < 1 || N < 1 || K < 16 || K % 16 != 0) return 0;
  if (prologue != QTTS_PROLOGUE_RMSNORM && prologue != QTTS_PROLOGUE_SILU_MUL) return 0;
  int family = variant & 0xF00;
  if (variant == QTTS_VARIANT_AUTO) {
    int rgroups = 0;
    family = auto_family(M, N, K, 1, kWInt8, false, &rgroups);
  }
  // The fused norm keeps one group sum per 256 columns of a row: K <= 8192.
  if (prologue == QTTS_PROLOGUE_RMSNORM && K > 8 * 32 * kMaxFusedNormGroups) return 0;
  return (M <= 16 && (family == 0x100 || family == 0x300)) ? 1 : 0;
}

int qtts_w8a16_plan(int M, int N, int K, int G, int variant, int* kernel, int* split, int* row_tile, int* ctas) {
  if (M < 1 || N < 1 || K < 16 || K % 16 != 0 || G < 1) return QTTS_ERR_SHAPE;
  if (kernel == nullptr || split == nullptr || row_tile == nullptr || ctas == nullptr) return QTTS_ERR_NULL;
  int family = variant & 0xF00, s = variant & 0xF, r = (variant >> 4) & 0xF;
  if (variant == QTTS_VARIANT_AUTO) {
    family = auto_family(M, N, K, G, kWInt8, false, &r);
    s = 0;
  }
  SkinnyPlan p{};
  if (variant == QTTS_VARIANT_GENERIC) {
    *kernel = 0;
    *split = 1;
    *row_tile = 8;
    *ctas = ((N + 7) / 8) * ((M + 7) / 8) * G;
    return QTTS_OK;
  } else if (family == 0x100) {
    p = plan_skinny(M, N, K, G, s, r);
    *kernel = 1;
  } else if (family == 0x200) {
    p = plan_umma(M, N, K, G, s);
    *kernel = 2;
  } else if (family == 0x300) {
    if (M > 16 || !(r == 0 || stream_rows_ok(r))) return QTTS_ERR_VARIANT;
    p = plan_stream(M, N, K, G, r);
    *kernel = 3;
  } else {
    return QTTS_ERR_VARIANT;
  }
  *split = p.split;
  *row_tile = 16 * p.r;
  *ctas = static_cast<int>(p.grid.x * p.grid.y * p.grid.z);
  return QTTS_OK;
}

int qtts_w8a16_gemm_allgather(const void* x, int64_t ldx, int x_dtype, const int8_t* w, int64_t ldw,
                              const void* scale, int scale_dtype, const void* bias, void* const* peer_out,
                              int64_t ldo, int64_t col_offset, uint32_t* const* peer_signal, uint32_t* sync,
                              int rank, int world, int M, int N, int K, int variant, unsigned flags, void* stream) {
  if (peer_out == nullptr || peer_signal == nullptr || sync == nullptr) return QTTS_ERR_NULL;
  if (world < 1 || world > QTTS_ALLGATHER_MAX_WORLD || rank < 0 || rank >= world || col_offset < 0)
    return QTTS_ERR_SHAPE;
  const AllGatherForm ag{peer_out, peer_signal, sync, col_offset, rank, world};
  return w8a16_dispatch(x, 0, ldx, x_dtype, w, ldw, scale, scale_dtype, bias, nullptr, 0, ldo, 1, M, N, K, nullptr,
                        variant, flags, stream, kWInt8, &ag);
}

int qtts_w8a16_grouped_gemm(const void* x, int64_t group_stride_x, int64_t ldx, int x_dtype, const int8_t* w,
                            int64_t ldw, const void* scale, int scale_dtype, const void* bias, void* out,
                            int64_t group_stride_out, int64_t ldo, int G, int M, int N, int K,
                            const int64_t* group_index, int variant, unsigned flags, void* stream) {
  return w8a16_dispatch(x, group_stride_x, ldx, x_dtype, w, ldw, scale, scale_dtype, bias, out, group_stride_out,
                        ldo, G, M, N, K, group_index, variant, flags, stream);
}

static int quantize_rows(const void* w, int64_t ldw, int w_dtype, void* q, float* scale, int N, int K, int mode,
                         void* stream) {
  if (N < 0 || K < 0) return QTTS_ERR_SHAPE;
  if (N == 0) return QTTS_OK;
  if (w == nullptr || q == nullptr || scale == nullptr) return QTTS_ERR_NULL;
  if (ldw < K) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(N), block(256);
  switch (w_dtype) {
    case QTTS_BF16:
      quantize_rows_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(w, ldw, q, scale, N, K, mode);
      break;
    case QTTS_FP16:
      quantize_rows_kernel<__half><<<grid, block, 0, s>>>(w, ldw, q, scale, N, K, mode);
      break;
    case QTTS_FP32:
      quantize_rows_kernel<float><<<grid, block, 0, s>>>(w, ldw, q, scale, N, K, mode);
      break;
    default:
      return QTTS_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

int qtts_quantize_int8_rows(const void* w, int64_t ldw, int w_dtype, int8_t* q, float* scale, int N, int K,
                            void* stream) {
  return quantize_rows(w, ldw, w_dtype, q, scale, N, K, 0, stream);
}

int qtts_quantize_fp8_rows(const void* w, int64_t ldw, int w_dtype, uint8_t* q, float* scale, int N, int K,
                           void* stream) {
  return quantize_rows(w, ldw, w_dtype, q, scale, N, K, 1, stream);
}

int qtts_fp8_quant_rows(const void* x, int64_t ldx, int x_dtype, uint8_t* q, float* scale_x, int M, int K,
                        unsigned flags, void* stream) {
  if (M < 0 || K < 0) return QTTS_ERR_SHAPE;
  if (M == 0) return QTTS_OK;
  if (x == nullptr || q == nullptr || scale_x == nullptr) return QTTS_ERR_NULL;
  if (ldx < K) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & QTTS_FLAG_PDL) != 0;
  const dim3 grid(M), block(256);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e;
  switch (x_dtype) {
    case QTTS_BF16:
      e = cudaLaunchKernelEx(&cfg, fp8_quant_rows_kernel<__nv_bfloat16>, x, ldx, q, scale_x, M, K);
      break;
    case QTTS_FP16:
      e = cudaLaunchKernelEx(&cfg, fp8_quant_rows_kernel<__half>, x, ldx, q, scale_x, M, K);
      break;
    case QTTS_FP32:
      e = cudaLaunchKernelEx(&cfg, fp8_quant_rows_kernel<float>, x, ldx, q, scale_x, M, K);
      break;
    default:
      return QTTS_ERR_DTYPE;
  }
  return e == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

int qtts_fp8_gemm(const uint8_t* xq, int64_t ldxq, const float* scale_x, const uint8_t* wq, int64_t ldw,
                  const float* scale_w, const void* bias, void* out, int64_t ldo, int out_dtype, int M, int N, int K,
                  int variant, unsigned flags, void* stream) {
  if (M < 0 || N < 0 || K < 0) return QTTS_ERR_SHAPE;
  if (M == 0 || N == 0) return QTTS_OK;
  if (xq == nullptr || scale_x == nullptr || wq == nullptr || scale_w == nullptr || out == nullptr)
    return QTTS_ERR_NULL;
  if (!is_float_dtype(out_dtype)) return QTTS_ERR_DTYPE;
  if (ldxq < K || ldw < K || ldo < N) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & QTTS_FLAG_PDL) != 0;
  const bool tc_ok = K % 16 == 0 && aligned16(xq) && aligned16(wq) && ldxq % 16 == 0 && ldw % 16 == 0;
  const int family = variant == QTTS_VARIANT_AUTO ? (tc_ok ? 0x200 : 0) : (variant & 0xF00);
  if (family == 0x200) {
    if (!tc_ok) return QTTS_ERR_ALIGN;
    const int split = variant == QTTS_VARIANT_AUTO ? 0 : (variant & 0xF);
    if (!(split == 0 || split == 1 || split == 2 || split == 4) || (variant & 0xF0F0) != 0) return QTTS_ERR_VARIANT;
    const Fp8Plan plan = plan_fp8(M, N, K, split);
    if (plan.grid.z > 65535u) return QTTS_ERR_SHAPE;
    CUtensorMap wmap, xmap;
    int r = make_tmap_u8_2d(&wmap, wq, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(ldw),
                            128, 128);
    if (r != QTTS_OK) return r;
    r = make_tmap_u8_2d(&xmap, xq, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(ldxq),
                        static_cast<uint32_t>(plan.nb), 128);
    if (r != QTTS_OK) return r;
    Fp8Args fa{};
    fa.scale_x = scale_x;
    fa.scale_w = scale_w;
    fa.bias = bias;
    fa.out = out;
    fa.ldo = ldo;
    fa.M = M;
    fa.N = N;
    fa.K = K;
    fa.k_per_cta = plan.k_per_cta;
    fa.stages = plan.stages;
    fa.wait_ns = current_wait_limit_ns();
    fa.trace_slot = -1;
#ifdef QTTS_TRACE
    fa.trace_slot = qtts_trace_next_slot();
#endif
    return launch_fp8_gemm(plan, wmap, xmap, fa, out_dtype, pdl, s);
  }
  if (variant != QTTS_VARIANT_AUTO && variant != QTTS_VARIANT_GENERIC) return QTTS_ERR_VARIANT;
  GenericFp8Args ga{xq, ldxq, scale_x, wq, ldw, scale_w, bias, out, ldo, M, N, K};
  const dim3 grid((N + 7) / 8, (M + 7) / 8);
  if (grid.y > 65535u) return QTTS_ERR_SHAPE;
  switch (out_dtype) {
    case QTTS_BF16:
      return launch_simple(generic_fp8_kernel<__nv_bfloat16>, grid, dim3(256), ga, pdl, s);
    case QTTS_FP16:
      return launch_simple(generic_fp8_kernel<__half>, grid, dim3(256), ga, pdl, s);
    default:
      return launch_simple(generic_fp8_kernel<float>, grid, dim3(256), ga, pdl, s);
  }
}

int qtts_int8_quant_rows(const void* x, int64_t ldx, int x_dtype, int8_t* q, float* scale_x, int M, int K,
                         unsigned flags, void* stream) {
  if (M < 0 || K < 0) return QTTS_ERR_SHAPE;
  if (M == 0) return QTTS_OK;
  if (x == nullptr || q == nullptr || scale_x == nullptr) return QTTS_ERR_NULL;
  if (ldx < K) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(256);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  if ((flags & QTTS_FLAG_PDL) != 0) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t e;
  switch (x_dtype) {
    case QTTS_BF16:
      e = cudaLaunchKernelEx(&cfg, int8_quant_rows_kernel<__nv_bfloat16>, x, ldx, q, scale_x, M, K);
      break;
    case QTTS_FP16:
      e = cudaLaunchKernelEx(&cfg, int8_quant_rows_kernel<__half>, x, ldx, q, scale_x, M, K);
      break;
    case QTTS_FP32:
      e = cudaLaunchKernelEx(&cfg, int8_quant_rows_kernel<float>, x, ldx, q, scale_x, M, K);
      break;
    default:
      return QTTS_ERR_DTYPE;
  }
  return e == cudaSuccess ? QTTS_OK : QTTS_ERR_LAUNCH;
}

int qtts_i8_gemm(const int8_t* xq, int64_t ldxq, const float* scale_x, const int8_t* wq, int64_t ldw,
                 const float* scale_w, const void* bias, void* out, int64_t ldo, int out_dtype, int M, int N, int K,
                 int variant, unsigned flags, void* stream) {
  if (M < 0 || N < 0 || K < 0) return QTTS_ERR_SHAPE;
  if (M == 0 || N == 0) return QTTS_OK;
  if (xq == nullptr || scale_x == nullptr || wq == nullptr || scale_w == nullptr || out == nullptr)
    return QTTS_ERR_NULL;
  if (!is_float_dtype(out_dtype)) return QTTS_ERR_DTYPE;
  if (ldxq < K || ldw < K || ldo < N) return QTTS_ERR_SHAPE;
  const int dev_ok = check_device();
  if (dev_ok != QTTS_OK) return dev_ok;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pdl = (flags & QTTS_FLAG_PDL) != 0;
  const bool tc_ok = K % 16 == 0 && aligned16(xq) && aligned16(wq) && ldxq % 16 == 0 && ldw % 16 == 0;
  const int family = variant == QTTS_VARIANT_AUTO ? (tc_ok ? 0x200 : 0) : (variant & 0xF00);
  if (family == 0x200) {
    if (!tc_ok) return QTTS_ERR_ALIGN;
    const int split = variant == QTTS_VARIANT_AUTO ? 0 : (variant & 0xF);
    if (!(split == 0 || split == 1 || split == 2 || split == 4) || (variant & 0xF0F0) != 0) return QTTS_ERR_VARIANT;
    const Fp8Plan plan = plan_fp8(M, N, K, split);
    if (plan.grid.z > 65535u) return QTTS_ERR_SHAPE;
    CUtensorMap wmap, xmap;
    int r = make_tmap_u8_2d(&wmap, wq, static_cast<uint64_t>(N), static_cast<uint64_t>(K), static_cast<uint64_t>(ldw),
                            128, 128);
    if (r != QTTS_OK) return r;
    r = make_tmap_u8_2d(&xmap, xq, static_cast<uint64_t>(M), static_cast<uint64_t>(K), static_cast<uint64_t>(ldxq),
                        static_cast<uint32_t>(plan.nb), 128);
    if (r != QTTS_OK) return r;
    Fp8Args fa{};
    fa.scale_x = scale_x;
    fa.scale_w = scale_w;
    fa.bias = bias;
    fa.out = out;
    fa.ldo = ldo;
    fa.M = M;
    fa.N = N;
    fa.K = K;
    fa.k_per_cta = plan.k_per_cta;
    fa.stages = plan.stages;
    fa.wait_ns = current_wait_limit_ns();
    fa.trace_slot = -1;
#ifdef QTTS_TRACE
    fa.trace_slot = qtts_trace_next_slot();
#endif
    return launch_fp8_gemm(plan, wmap, xmap, fa, out_dtype, pdl, s, /*int8=*/true);
  }
  if (variant != QTTS_VARIANT_AUTO && variant != QTTS_VARIANT_GENERIC) return QTTS_ERR_VARIANT;
  GenericFp8Args ga{reinterpret_cast<const uint8_t*>(xq), ldxq, scale_x, reinterpret_cast<const uint8_t*>(wq), ldw,
                    scale_w, bias, out, ldo, M, N, K};
  const dim3 grid((N + 7) / 8, (M + 7) / 8);
  if (grid.y > 65535u) return QTTS_ERR_SHAPE;
  switch (out_dtype) {
    case QTTS_BF16:
      return launch_simple(generic_i8_kernel<__nv_bfloat16>, grid, dim3(256), ga, pdl, s);
    case QTTS_FP16:
      return launch_simple(generic_i8_kernel<__half>, grid, dim3(256), ga, pdl, s);
    default:
      return launch_simple(generic_i8_kernel<float>, grid, dim3(256), ga, pdl, s);
  }
}

}  // extern "C"
