// Internal host-side interface between the C ABI (capi.cu) and the kernel
// translation units. Not part of the public ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/qtts_b200.h"

namespace qtts {

constexpr int kNumSMs = 148;                 // B200: 2 dies x 74 SMs
constexpr int kCtaSlots = 2 * kNumSMs;        // two weight-streaming CTAs per SM
constexpr size_t kMaxDynSmem = 227 * 1024;   // opt-in dynamic shared memory per CTA

// ---- skinny W8A16 ------------------------------------------------------------
struct SkinnyArgs {
  const void* x;
  int64_t ldx;
  int64_t gsx;  // group stride of x (elements)
  const void* scale;
  int scale_dtype;
  const void* bias;
  void* out;
  int64_t ldo;
  int64_t gso;  // group stride of out (elements)
  int M, N, K;  // N is per group
  int G;
  int k_per_cta;  // multiple of 128
  int stages;
  int x_pitch;  // elements per staged activation row
  int m_chunks;
  const int64_t* group_index;  // device pointer or NULL
  uint64_t wait_ns;
  int trace_slot;  // timeline probe slot (-1: off); only read in -DQTTS_TRACE builds
  int64_t gsx_rows;  // group stride of x in rows (tcgen05 kernel: x is read through a tensor map)
  int w_fmt;         // kWInt8 or kWE4M3
  // All-gather form (qtts_w8a16_gemm_allgather, csrc/allgather.cuh); peer_out
  // is nullptr otherwise.
  void* const* peer_out;      // [world] every rank's gathered output (device pointers)
  uint32_t* const* peer_sig;  // [world] every rank's signal pad, uint32[2 * world] each
  uint32_t* sync;             // this rank's uint32[2]: CTA arrivals, epoch of the last call
  int64_t col_offset;         // gathered column of this rank's first output channel
  int rank;
  int world;
  // Fused activation prologue (qtts_w8a16_gemm_prologue, csrc/prologue.cuh):
  // kProNone, kProRmsNorm (pro_weight = the norm weight [K] of the activation
  // type, pro_eps) or kProSiluMul (x rows are [gate | up], 2*K wide).
  int prologue;
  const void* pro_weight;
  float pro_eps;
};

constexpr int kWInt8 = 0;  // int8 weights (W8A16)
constexpr int kWE4M3 = 1;  // e4m3 weights (fp8 weight-only)

struct SkinnyPlan {
  int mt;        // batch n-tiles of 8 (1, 2, 4, 8)
  int r;         // row groups of 16 per CTA (1, 2, 4, 8): BN = 16*r
  int m_chunks;  // ceil(M / (8*mt))
  int split;     // CTAs per cluster along K
  int k_per_cta;
  int x_pitch;
  int stages;
  size_t smem;
  dim3 grid;
};

// split_req / r_req: 0 = choose.
SkinnyPlan plan_skinny(int M, int N, int K, int G, int split_req, int r_req);
int launch_skinny_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, int x_dtype,
                        bool pdl, cudaStream_t stream);

// ---- weight-streaming W8A16 for M <= 16 (same argument block; plan.split = 1) ---
bool stream_rows_ok(int r);
SkinnyPlan plan_stream(int M, int N, int K, int G, int r_req);
int launch_stream_w8a16(const SkinnyPlan& p, const CUtensorMap& map, const SkinnyArgs& args, int x_dtype, bool pdl,
                        cudaStream_t stream);

// ---- tcgen05 W8A16 (same argument block; plan.mt = NB/8, plan.r = 8) ----------
SkinnyPlan plan_umma(int M, int N, int K, int G, int split_req);
int launch_umma_w8a16(const SkinnyPlan& p, const CUtensorMap& wmap, const CUtensorMap& xmap, const SkinnyArgs& args,
                      int x_dtype, bool pdl, cudaStream_t stream);

// ---- fp8 e4m3 W8A8 (tcgen05) ------------------------------------------------------
struct Fp8Args {
  const float* scale_x;
  const float* scale_w;
  const void* bias;
  void* out;
  int64_t ldo;
  int M, N, K;
  int k_per_cta;
  int stages;
  uint64_t wait_ns;
  int trace_slot;  // timeline probe slot (-1: off); only read in -DQTTS_TRACE builds
};

struct Fp8Plan {
  int nb;     // batch columns per CTA (MMA N): 16, 32, 64, 128
  int split;  // CTAs per cluster along K
  int k_per_cta;
  int stages;
  size_t smem;
  dim3 grid;
};

// ---- fused codebook head (csrc/head_argmax.cu) --------------------------------
struct HeadArgs {
  const void* x;  // [M, K] activations (pre-norm), 16-bit
  int64_t ldx;
  const void* norm_weight;  // [K] of the activation type, or nullptr (no norm)
  float eps;
  const int8_t* w;  // [N, K] int8
  int64_t ldw;
  const void* scale;  // [N]
  int scale_dtype;
  const float* logit_bias;  // [N] fp32 added to the rounded logits, or nullptr
  int64_t* codes;           // [M]
  const void* embed;        // [vocab, E] of the activation type, or nullptr
  int64_t lde;
  void* embed_out;  // [M, E]
  int64_t ldeo;
  int E;
  int vocab;
  unsigned long long* state;  // [M + 1], zero before the first call; left zero
  int M, N, K;
};
size_t head_argmax_smem(int M, int K);
int launch_head_argmax(const HeadArgs& a, int x_dtype, bool pdl, cudaStream_t stream);

Fp8Plan plan_fp8(int M, int N, int K, int split_req);
// int8 = true: the int8 W8A8 form (signed int8 operands, int32 accumulator).
int launch_fp8_gemm(const Fp8Plan& p, const CUtensorMap& wmap, const CUtensorMap& xmap, const Fp8Args& args,
                    int out_dtype, bool pdl, cudaStream_t stream, bool int8 = false);

// ---- standalone activation prologues (csrc/prologue.cu) ------------------------
struct PrologueArgs {
  int kind;  // kProRmsNorm or kProSiluMul
  const void* x;
  int64_t ldx;
  const void* weight;  // RMSNorm weight [width], of the activation type
  float eps;
  void* out;
  int64_t ldo;
  int rows, width;
  bool vec;  // 16-byte aligned rows and width % 8 == 0: vector loads and stores
};
int launch_prologue(const PrologueArgs& p, int dtype, bool pdl, cudaStream_t stream);

// ---- tensor maps ---------------------------------------------------------------
// 2-D uint8 tensor map over a row-major [rows, cols] byte matrix with row pitch
// `pitch_bytes`, box [box_rows, box_cols] and 128-byte swizzle.
int make_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_bytes,
                    uint32_t box_rows, uint32_t box_cols);
// Same for a 16-bit element matrix (dtype QTTS_BF16 or QTTS_FP16); cols and
// box_cols in elements.
int make_tmap_16b_2d(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                     uint64_t pitch_bytes, uint32_t box_rows, uint32_t box_cols);

uint64_t current_wait_limit_ns();

#ifdef QTTS_TRACE
int qtts_trace_next_slot();
#endif

}  // namespace qtts
