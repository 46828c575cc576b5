// fp8 W8A8 linear whose activation codes live in a fixed device array.
//
// The fp8 linear runs in two steps: per-token quantization of the activations
// into e4m3 codes plus one fp32 scale per row, then the scaled e4m3 GEMM that
// reads them. Those codes and scales are scratch: global memory beyond the
// call's inputs and outputs. qtts_fp8_quant_rows + qtts_fp8_gemm leave the
// caller to provide it; this entry point keeps it in a file-scope device
// array instead, so one call needs no device memory from anyone.
//
// Who needs that: a caller that binds the C ABI without a device allocator
// of its own (a ctypes or cgo binding with no torch underneath). Such a
// caller would otherwise cudaMalloc and cudaFree the intermediate on every
// call -- both synchronise the whole device and cost far more than the GEMM
// at decode sizes -- or keep one buffer alive per layer and size it itself.
//
// Limits and sharing:
//   * the array holds at most kMaxCodes e4m3 codes (M * K) and kMaxRows row
//     scales; larger problems are rejected with QTTS_ERR_SHAPE before anything
//     is launched;
//   * nothing in it has to start at zero: the GEMM reads only codes and scales
//     that the quantization step of the same call has just written (the GEMM's
//     TMA copies fill rows past M with zeros instead of reading them);
//   * there is one array per device, so two calls in flight on one device at
//     the same time (different streams, or different host threads without
//     ordering between their streams) race on it. Calls ordered on one stream
//     are safe.
//   * the address is looked up with cudaGetSymbolAddress the first time the
//     entry point runs on a device, with that device current, and cached
//     together with the device's current context; a call under another context
//     (after cudaDeviceReset the primary context, and with it the module, is
//     created anew) looks it up again. A caller that records its launches into
//     a CUDA graph should make one call on each device before the capture
//     starts, so the look-up (which may load the module) happens outside it.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "qtts_b200.h"

namespace {

constexpr int64_t kMaxCodes = QTTS_NOALLOC_MAX_CODES;
constexpr int kMaxRows = QTTS_NOALLOC_MAX_ROWS;
constexpr int kMaxDevices = 64;

// [0, kMaxCodes): e4m3 codes, row m at m * K. [kMaxCodes, +4 * kMaxRows): fp32
// row scales. kMaxCodes is a multiple of 256, so both parts stay 256-aligned.
static_assert(kMaxCodes % 256 == 0, "the scale block must stay aligned");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kMaxCodes + 4 * kMaxRows];

struct ScratchEntry {
  CUcontext ctx = nullptr;
  unsigned char* addr = nullptr;
};
ScratchEntry g_scratch[kMaxDevices];
int g_cc_major[kMaxDevices] = {0};
std::mutex g_scratch_mu;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (the library links
// no driver library directly).
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return static_cast<CtxGetCurrentFn>(nullptr);
    }
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

CUcontext current_context() {
  CtxGetCurrentFn fn = ctx_get_current();
  CUcontext ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}

// The current device is an sm_100 part (QTTS_ERR_ARCH otherwise, as every
// other entry point answers), checked before anything loads the module.
int check_arch(int* dev_out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    (void)cudaGetLastError();
    return QTTS_ERR_ARCH;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_cc_major[dev] == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) {
      (void)cudaGetLastError();
      return QTTS_ERR_ARCH;
    }
    g_cc_major[dev] = major;
  }
  *dev_out = dev;
  return g_cc_major[dev] == 10 ? QTTS_OK : QTTS_ERR_ARCH;
}

// The array's device address under the current device's context, looked up
// once per device and context.
int scratch_address(int dev, unsigned char** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchEntry& e = g_scratch[dev];
  CUcontext ctx = current_context();
  if (e.addr == nullptr || ctx == nullptr || ctx != e.ctx) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || addr == nullptr) {
      (void)cudaGetLastError();
      return QTTS_ERR_CUDA;
    }
    e.addr = static_cast<unsigned char*>(addr);
    e.ctx = current_context();  // the look-up makes the primary context current
  }
  *out = e.addr;
  return QTTS_OK;
}

bool is_act_dtype(int d) { return d == QTTS_BF16 || d == QTTS_FP16 || d == QTTS_FP32; }

}  // namespace

extern "C" {

int qtts_fp8_linear_noalloc(const void* x, int64_t ldx, int x_dtype, const uint8_t* wq, int64_t ldw,
                            const float* scale_w, const void* bias, void* out, int64_t ldo, int out_dtype, int M,
                            int N, int K, unsigned flags, void* stream) {
  // Arguments either step would reject are rejected here, before the first
  // launch; a failure of the second launch itself leaves only the array written.
  if (M < 0 || N < 0 || K < 0) return QTTS_ERR_SHAPE;
  if (M == 0 || N == 0) return QTTS_OK;
  if (x == nullptr || wq == nullptr || scale_w == nullptr || out == nullptr) return QTTS_ERR_NULL;
  if (!is_act_dtype(x_dtype) || !is_act_dtype(out_dtype)) return QTTS_ERR_DTYPE;
  if (ldx < K || ldw < K || ldo < N) return QTTS_ERR_SHAPE;
  if (M > kMaxRows || static_cast<int64_t>(M) * K > kMaxCodes) return QTTS_ERR_SHAPE;
  int dev = -1;
  const int arch = check_arch(&dev);
  if (arch != QTTS_OK) return arch;
  unsigned char* scratch = nullptr;
  const int r = scratch_address(dev, &scratch);
  if (r != QTTS_OK) return r;
  uint8_t* xq = scratch;
  float* scale_x = reinterpret_cast<float*>(scratch + kMaxCodes);
  const int q = qtts_fp8_quant_rows(x, ldx, x_dtype, xq, scale_x, M, K, flags, stream);
  if (q != QTTS_OK) return q;
  return qtts_fp8_gemm(xq, K, scale_x, wq, ldw, scale_w, bias, out, ldo, out_dtype, M, N, K, QTTS_VARIANT_AUTO,
                       flags, stream);
}

}  // extern "C"
