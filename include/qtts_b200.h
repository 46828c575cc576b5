/*
 * qtts_b200.h -- C ABI of the B200 (sm_100a) quantized-linear library.
 *
 * This library replaces the device code behind the `LinearBase.quant_method`
 * hook of qtts (danielhua23/tts-inference):
 *
 *   - int8 weight-only GEMM/GEMV (W8A16), the Triton kernel `_w8_gemm_kernel`
 *     and its launcher `w8_gemm` (qtts/quant/kernels.py:89-135, 138-177);
 *   - fp8-e4m3 W8A8: the eager per-token activation quantization plus
 *     `torch._scaled_mm` of `Fp8Method.apply` (qtts/quant/fp8.py:72-89);
 *   - the load-time quantizers `quantize_weight_per_channel`
 *     (qtts/quant/int8.py:45-56) and `quantize_weight_fp8`
 *     (qtts/quant/fp8.py:45-49);
 *   - int8 W8A8 (`Int8Method.apply`, qtts/quant/int8.py:120-155), fp8
 *     weight-only, and the RMSNorm / SiLU·up prologues of the decoder layer's
 *     linears (qtts/layers/norm.py, activation.py:147), standalone or fused.
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers owned by the caller; the library never
 *     allocates or frees device memory and never synchronizes the stream.
 *   - Matrices are row-major with an explicit leading dimension in ELEMENTS.
 *     Weights are [N, K] (output channel major, K contiguous), activations
 *     [M, K], outputs [M, N].
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Every launch
 *     goes to that stream only, so calls are CUDA-graph capturable.
 *   - Return value is a status code (QTTS_OK on success). Validation happens
 *     on the host before any launch: a non-OK status means nothing was
 *     launched. Device-side failures (an expired bounded wait) are recorded in
 *     a per-device status word readable with qtts_device_status().
 *   - No C++ exceptions cross this boundary.
 */
#ifndef QTTS_B200_H
#define QTTS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QTTS_ABI_VERSION 1

#if defined(__GNUC__)
#define QTTS_API __attribute__((visibility("default")))
#else
#define QTTS_API
#endif

/* ---- status codes ------------------------------------------------------ */
enum qtts_status {
  QTTS_OK = 0,
  QTTS_ERR_NULL = 1,    /* a required pointer is NULL                        */
  QTTS_ERR_SHAPE = 2,   /* M/N/K/G or a leading dimension is out of range    */
  QTTS_ERR_ALIGN = 3,   /* pointer or stride misaligned for the variant      */
  QTTS_ERR_DTYPE = 4,   /* unsupported dtype code or dtype combination       */
  QTTS_ERR_ARCH = 5,    /* no sm_100 device, or a driver entry point missing */
  QTTS_ERR_LAUNCH = 6,  /* the kernel launch itself failed                   */
  QTTS_ERR_VARIANT = 7, /* unknown variant, or not applicable to the shape   */
  QTTS_ERR_TIMEOUT = 8, /* a device-side bounded wait expired                */
  QTTS_ERR_CUDA = 9     /* another CUDA runtime error                        */
};

/* ---- dtype codes ------------------------------------------------------- */
enum qtts_dtype {
  QTTS_BF16 = 0,
  QTTS_FP16 = 1,
  QTTS_FP32 = 2,
  QTTS_E4M3 = 3, /* float8_e4m3fn, one byte per element */
  QTTS_INT8 = 4
};

/* ---- launch flags ------------------------------------------------------ */
/* Launch with programmatic dependent launch: the kernel starts while the
 * previous kernel of the stream drains and streams its (constant) weights in
 * before waiting on the dependency. Activations, scales, bias and outputs are
 * touched only after the wait. The weights must not be written by the
 * immediately preceding kernel of the same stream. */
#define QTTS_FLAG_PDL 0x1u

/* ---- kernel variants ---------------------------------------------------- */
/* 0 lets the library choose from (M, N, K): up to 16 rows the split-K
 * streaming kernel (up to 4 rows of int8 the whole-K streaming kernel where
 * the split-K plan loads some SMs twice and the whole-K plan reaches more
 * CTAs; at 9..16 rows the tcgen05 kernel where the split-K CTAs would each
 * stream >= 96 KiB of weights), past 16 rows the tcgen05 kernel. The others
 * force one kernel; calibration (qtts_b200.quant.calibrate) times them per
 * shape. */
#define QTTS_VARIANT_AUTO 0
#define QTTS_VARIANT_GENERIC 1 /* SIMT kernel: any shape, stride, dtype    */
/* TMA-streamed weights + mma.sync. `split`: K split over a thread-block
 * cluster of 1, 2, 4 or 8 CTAs reduced through distributed shared memory;
 * `rows`: row groups of 16 per CTA (1, 2, 4 or 8; the rest of the CTA's 8
 * warps split K inside it). 0 in either field lets the library choose. */
#define QTTS_VARIANT_SKINNY(split) (0x100 | (split))
#define QTTS_VARIANT_SKINNY_R(split, rows) (0x100 | (split) | ((rows) << 4))
/* tcgen05/TMEM tile kernel (128 weight rows per CTA converted to the
 * activations' 16-bit type straight into tensor memory, activation tiles by
 * TMA in shared memory, fp32 accumulators in tensor memory), split-K over a
 * cluster of `split` CTAs. */
#define QTTS_VARIANT_UMMA(split) (0x200 | (split))
/* Whole-K streaming kernel for M <= 16: each CTA owns 16*`rows` output rows
 * (rows = 1, 2, 3, 4 or 6; 0 lets the library choose) over the whole of K, no
 * cross-CTA reduction; weights dequantized with one byte-permute per two and
 * the bias removed once per output. Refused (QTTS_ERR_VARIANT) when the
 * activation rows do not fit in shared memory. */
#define QTTS_VARIANT_STREAM(rows) (0x300 | ((rows) << 4))

/* ---- library information ------------------------------------------------ */
QTTS_API int qtts_abi_version(void);
QTTS_API const char* qtts_status_str(int status);

/* Reads (and, when `reset` != 0, clears) the device-side status word of the
 * current device. Returns QTTS_OK when no kernel has recorded a failure.
 * This call synchronizes with the device (it copies 4 bytes). */
QTTS_API int qtts_device_status(int reset);

/* Sets the bounded-wait limit (nanoseconds) of subsequent launches on the
 * current device; 0 restores the default of 2 s. Returns the previous
 * limit. */
QTTS_API uint64_t qtts_set_wait_limit_ns(uint64_t limit_ns);

/* ---- int8 weight-only (W8A16) ---------------------------------------------
 * out[m, n] = cast_out( sum_k float(x[m, k]) * float(w[n, k]) * float(scale[n])
 *                       + float(bias[n]) )
 * accumulated in fp32, the scale applied once after the K loop.
 *
 * Replaces: w8_gemm (qtts/quant/kernels.py:138-177) and _w8_gemm_kernel
 * (qtts/quant/kernels.py:89-135).
 *   x      [M, K] of x_dtype (BF16, FP16 or FP32), leading dimension ldx
 *   w      [N, K] int8, leading dimension ldw
 *   scale  [N] of scale_dtype (BF16, FP16 or FP32)
 *   bias   [N] of x_dtype, or NULL
 *   out    [M, N] of x_dtype, leading dimension ldo
 * M == 0 is a no-op. The skinny and UMMA variants need K % 16 == 0, 16-byte
 * aligned x/w rows and a BF16 or FP16 x; AUTO falls back to the SIMT kernel
 * otherwise. */
QTTS_API int qtts_w8a16_gemm(const void* x, int64_t ldx, int x_dtype,
                    const int8_t* w, int64_t ldw,
                    const void* scale, int scale_dtype,
                    const void* bias,
                    void* out, int64_t ldo,
                    int M, int N, int K,
                    int variant, unsigned flags, void* stream);

/* Grouped W8A16 over G independent problems of one shape: the 15 codebook
 * heads of the code predictor, lm_head[i] 1024->2048
 * (qtts/models/code_predictor.py:159-161, 235), in one launch.
 *   x     group g at x + g*group_stride_x, [M, K] with leading dim ldx
 *   w     [G*N, K] int8, group g owns rows [g*N, (g+1)*N)
 *   scale [G*N];  bias [G*N] or NULL
 *   out   group g at out + g*group_stride_out, [M, N] with leading dim ldo
 * When `group_index` (device pointer to one int64) is non-NULL, exactly one
 * group is computed -- the one whose index is read on the device at run
 * time -- with x and out taken WITHOUT the group offset. That is the
 * graph-capturable "head chosen on the device" form; G then only bounds the
 * index (an index outside [0, G) records QTTS_ERR_SHAPE on the device and
 * writes nothing). */
QTTS_API int qtts_w8a16_grouped_gemm(const void* x, int64_t group_stride_x, int64_t ldx, int x_dtype,
                            const int8_t* w, int64_t ldw,
                            const void* scale, int scale_dtype,
                            const void* bias,
                            void* out, int64_t group_stride_out, int64_t ldo,
                            int G, int M, int N, int K,
                            const int64_t* group_index,
                            int variant, unsigned flags, void* stream);

/* The kernel qtts_w8a16_gemm would launch for int8 weights and aligned bf16 or
 * fp16 activations (G groups of N rows, as qtts_w8a16_grouped_gemm without a
 * device index): *kernel 0 = SIMT (QTTS_VARIANT_GENERIC), 1 = split-K
 * streaming (QTTS_VARIANT_SKINNY), 2 = tcgen05 (QTTS_VARIANT_UMMA),
 * 3 = whole-K streaming (QTTS_VARIANT_STREAM); its K split, weight rows per
 * CTA and grid size. Host-only: needs no GPU. */
QTTS_API int qtts_w8a16_plan(int M, int N, int K, int G, int variant, int* kernel, int* split, int* row_tile,
                             int* ctas);

/* ---- activation prologues -------------------------------------------------
 * RMSNorm and SiLU·up, standalone and fused into the W8A16 GEMM that consumes
 * them (the decoder layer's input / post-attention norm feeding qkv_proj /
 * gate_up_proj, qtts/models/talker.py:249, 271; SiLU·up between gate_up_proj
 * and down_proj, qtts/layers/activation.py:147). Element arithmetic:
 *   RMSNorm   y = cast( w[k] * (x[k] * inv) ),
 *             inv = 1 / sqrt( sum_k x[k]^2 / width + eps )   (fp32; the sum
 *             in the library's fixed order, identical in every form: fma
 *             over each 8-element chunk, a butterfly over each 32 consecutive
 *             chunks, a stride-halving tree over those group sums)
 *   SiLU·up   y = cast( float(cast(g / (1 + exp(-g)))) * float(up) )
 *             (each step rounded to the activation type, as torch's
 *             F.silu(gate) * up) */
#define QTTS_PROLOGUE_NONE 0
#define QTTS_PROLOGUE_RMSNORM 1
#define QTTS_PROLOGUE_SILU_MUL 2

/* RMSNorm over the last dimension of x [rows, width] (leading dimension ldx)
 * with weight [width], into out [rows, width] (ldo); dtype BF16, FP16 or
 * FP32 for x, weight and out; width <= 65536. out may be x (same ld): in
 * place.
 * Replaces: _rms_norm_kernel and RMSNorm.forward (qtts/layers/norm.py:49-76,
 * 102-121; the reduction reaches the reference's eager form,
 * norm.py:123-137, within one bf16 step, as the reference's own fused
 * kernel does). */
QTTS_API int qtts_rms_norm(const void* x, int64_t ldx, const void* weight, void* out, int64_t ldo, int dtype,
                           int rows, int width, float eps, unsigned flags, void* stream);

/* out [rows, width] = silu(gate) * up of gate_up [rows, 2*width] (leading
 * dimension ld_in >= 2*width; gate = columns [0, width), up = [width,
 * 2*width), MergedLinear.split order). out may be gate_up (ldo = ld_in).
 * Replaces: F.silu(gate) * up in GatedMLP.forward (qtts/layers/activation.py:
 * 143-147); equal bit for bit to torch's two CUDA kernels. */
QTTS_API int qtts_silu_mul(const void* gate_up, int64_t ld_in, void* out, int64_t ldo, int dtype, int rows,
                           int width, unsigned flags, void* stream);

/* out = W8A16( prologue(x) ): qtts_w8a16_gemm on the RMSNorm of x [M, K]
 * (norm_weight [K] of x_dtype, eps), or on SiLU·up of x [M, 2K] (ldx >= 2K;
 * norm_weight and eps unused). Equal bit for bit to qtts_rms_norm /
 * qtts_silu_mul followed by qtts_w8a16_gemm with the same variant. Where the
 * chosen kernel is the split-K or whole-K streaming kernel (int8 weights,
 * M <= 16, bf16/fp16 activations, 16-byte aligned rows and norm weight,
 * K <= 8192 for RMSNorm) the
 * prologue runs inside it as the activations are staged: one launch. Otherwise
 * the prologue kernel writes workspace [M, K] (x_dtype, leading dimension K,
 * 16-byte aligned for the tensor-core kernels) and the GEMM, launched with
 * programmatic dependent launch behind it, reads that; workspace may be NULL
 * only when the call fuses (QTTS_ERR_NULL otherwise;
 * qtts_w8a16_gemm_prologue_fused tells in advance). Other arguments as for
 * qtts_w8a16_gemm. */
QTTS_API int qtts_w8a16_gemm_prologue(const void* x, int64_t ldx, int x_dtype, int prologue,
                                      const void* norm_weight, float eps, const int8_t* w, int64_t ldw,
                                      const void* scale, int scale_dtype, const void* bias, void* out, int64_t ldo,
                                      int M, int N, int K, void* workspace, int variant, unsigned flags,
                                      void* stream);

/* 1 when qtts_w8a16_gemm_prologue with this shape, prologue and variant runs
 * as one fused launch (given aligned bf16/fp16 operands), else 0. Host-only. */
QTTS_API int qtts_w8a16_gemm_prologue_fused(int M, int N, int K, int prologue, int variant);

/* fp8 weight-only GEMM (no counterpart in the reference, which leaves
 * Fp8WeightOnlyMethod unimplemented, qtts/quant/fp8.py:92-122): the W8A16
 * contract with e4m3 weights,
 *   out[m,n] = cast( (sum_k x[m,k] * e4m3(w[n,k])) * scale[n] + bias[n] )
 * w: [N, K] e4m3 bytes (ld ldw), scale [N] (e.g. from qtts_quantize_fp8_rows);
 * every other argument, the variants and the status codes as for
 * qtts_w8a16_gemm. The weights are converted to 16-bit floats in registers
 * (exactly); the whole-K streaming variant (QTTS_VARIANT_STREAM) does not
 * apply, and the split-K streaming variants take M <= 16. */
QTTS_API int qtts_fp8w_gemm(const void* x, int64_t ldx, int x_dtype, const uint8_t* w, int64_t ldw,
                   const void* scale, int scale_dtype, const void* bias, void* out, int64_t ldo,
                   int M, int N, int K, int variant, unsigned flags, void* stream);

/* N-sharded W8A16 GEMM fused with the all-gather of its output. Replaces the
 * per-rank w8a16 GEMM followed by ncclAllGather of the bf16 blocks (the
 * multi-GPU form of the standalone GEMM, one exchange step): this rank
 * computes out = x @ (w * scale).T + bias for its N output channels and the
 * kernel stores every element straight into the gathered output of EVERY
 * rank, over peer memory (P2P stores through NVLink), at columns
 * [col_offset, col_offset + N) of rows [0, M) with leading dimension ldo.
 *   peer_out    device array [world] of device pointers: rank q's gathered
 *               buffer (this rank's own included, at index rank), x_dtype
 *   peer_signal device array [world] of device pointers: rank q's signal pad,
 *               uint32[2 * world], zero before the first call
 *   sync        this rank's uint32[2], zero before the first call
 * Calls are numbered on the device, so the call is CUDA-graph capturable.
 * When the kernel completes, this rank's gathered buffer holds every rank's
 * block of the same call. Every rank must make the same sequence of calls
 * (same M and ldo) with its own shard; a rank that stops calling makes the
 * others record QTTS_ERR_TIMEOUT after the wait limit instead of hanging.
 * Every rank owns at least one output channel (N >= 1; M == 0 on every rank
 * is a no-op). One signal pad / sync pair serves one stream. Other arguments as for
 * qtts_w8a16_gemm (bf16/fp16 activations, 16-byte aligned rows, K % 16 == 0;
 * AUTO or the split-K (M <= 16) and tcgen05 variants). */
#define QTTS_ALLGATHER_MAX_WORLD 64
QTTS_API int qtts_w8a16_gemm_allgather(const void* x, int64_t ldx, int x_dtype, const int8_t* w, int64_t ldw,
                              const void* scale, int scale_dtype, const void* bias,
                              void* const* peer_out, int64_t ldo, int64_t col_offset,
                              uint32_t* const* peer_signal, uint32_t* sync, int rank, int world,
                              int M, int N, int K, int variant, unsigned flags, void* stream);

/* ---- load-time weight quantizers ------------------------------------------
 * Division by a constant (`amax / 127`, `/ 448`) follows torch on a CUDA
 * tensor, where `tensor / number` is evaluated as `tensor * fl32(1 / number)`:
 * the quantizers reproduce the reference as it runs on the GPU (on the CPU,
 * torch divides, and about half of the scales differ in the last bit).
 *
 * Symmetric per-output-channel int8, bit-exact with
 * quantize_weight_per_channel (qtts/quant/int8.py:45-56) on a CUDA tensor:
 *   scale[n] = max(max_k |float(w[n,k])|, 1e-12f) * fl32(1 / 127)
 *   q[n,k]   = clamp(round_half_even(float(w[n,k]) / scale[n]), -127, 127)
 * w: [N, K] of w_dtype (BF16, FP16, FP32); q: [N, K] int8 (ld = K);
 * scale: [N] fp32. */
QTTS_API int qtts_quantize_int8_rows(const void* w, int64_t ldw, int w_dtype,
                            int8_t* q, float* scale, int N, int K, void* stream);

/* Symmetric per-output-channel e4m3, bit-exact with quantize_weight_fp8
 * (qtts/quant/fp8.py:45-49) on a CUDA tensor:
 *   scale[n] = max(max_k |float(w[n,k])|, 1e-12f) * fl32(1 / 448)
 *   q[n,k]   = e4m3_rne(float(w[n,k]) / scale[n])
 * q: [N, K] e4m3 bytes (ld = K); scale: [N] fp32. */
QTTS_API int qtts_quantize_fp8_rows(const void* w, int64_t ldw, int w_dtype,
                           uint8_t* q, float* scale, int N, int K, void* stream);

/* ---- fp8 e4m3 W8A8 ---------------------------------------------------------
 * Per-token dynamic activation quantization, bit-exact with
 * Fp8Method.apply (qtts/quant/fp8.py:77-78) on a CUDA tensor:
 *   amax_m     = max_k |x[m,k]|                (in x_dtype, exact)
 *   scale_x[m] = float(max(amax_m, x_dtype(1e-6))) * fl32(1 / 448)
 *   q[m,k]     = e4m3_rne(float(x[m,k]) / scale_x[m])
 * x: [M, K] (BF16/FP16/FP32, ld ldx); q: [M, K] e4m3 (ld = K); scale_x: [M]. */
QTTS_API int qtts_fp8_quant_rows(const void* x, int64_t ldx, int x_dtype,
                        uint8_t* q, float* scale_x, int M, int K,
                        unsigned flags, void* stream);

/* Scaled e4m3 GEMM, the torch._scaled_mm call of Fp8Method.apply
 * (qtts/quant/fp8.py:79-88):
 *   y[m,n]   = cast_out( (sum_k xq[m,k] * wq[n,k]) * scale_x[m] * scale_w[n] )
 *   out[m,n] = bias ? cast_out( float(y[m,n]) + float(bias[n]) ) : y[m,n]
 * i.e. _scaled_mm(out_dtype) rounded first and the bias added in the output
 * dtype, as the reference does. xq: [M, K] e4m3 (ld ldxq); wq: [N, K] e4m3
 * (ld ldw); out: [M, N] of out_dtype (BF16/FP16/FP32) with leading dim ldo;
 * bias [N] of out_dtype or NULL. The tcgen05 variants need K % 16 == 0 and
 * 16-byte aligned rows; AUTO takes a SIMT kernel (QTTS_VARIANT_GENERIC, any
 * K and stride) for shapes they cannot. */
QTTS_API int qtts_fp8_gemm(const uint8_t* xq, int64_t ldxq, const float* scale_x,
                  const uint8_t* wq, int64_t ldw, const float* scale_w,
                  const void* bias, void* out, int64_t ldo, int out_dtype,
                  int M, int N, int K, int variant, unsigned flags, void* stream);

/* ---- fused codebook head -------------------------------------------------------
 * The end of one greedy decode step in one launch: the code predictor's
 *   logits = lm_head[step](norm(hidden)); code = logits.argmax(-1);
 *   next = codec_embedding[step](code)
 * (qtts/models/code_predictor.py:229-242) and the talker's masked codec head
 * (qtts/models/talker.py:354-356):
 *   y[m]     = norm_weight ? RMSNorm(x[m]) (the library's element, as
 *              qtts_rms_norm) : x[m]
 *   l[m, n]  = float(cast_x( (sum_k y[m,k] * w[n,k]) * scale[n] )) + logit_bias[n]
 *   codes[m] = the first n with the largest l[m, n] (torch.argmax)
 *   embed_out[m, 0:E] = embed[codes[m], 0:E]   (when embed is not NULL)
 * x: [M, K] BF16/FP16 (ld ldx, 16-byte aligned rows); norm_weight: [K] of x's
 * dtype or NULL; w: [N, K] int8 (ld ldw, 4-byte aligned rows); scale: [N] of
 * scale_dtype; logit_bias: [N] fp32 or NULL (0 keeps a logit, -inf masks it);
 * codes: [M] int64; embed: [vocab, E] of x's dtype or NULL, embed_out [M, E].
 * state: M + 1 zeroed uint64 words of device memory the caller owns (the
 * per-row best candidates and a CTA counter); the call leaves them zero, so
 * one state array serves every call ordered on a stream (calls that may run
 * at the same time need separate arrays). M <= 16, K % 128 == 0, K <= 2048,
 * E % 8 == 0. Replaces lm_head[step] + argmax + the embedding lookup. */
QTTS_API int qtts_w8a16_head_argmax(const void* x, int64_t ldx, int x_dtype, const void* norm_weight, float eps,
                                    const int8_t* w, int64_t ldw, const void* scale, int scale_dtype,
                                    const float* logit_bias, int64_t* codes, const void* embed, int64_t lde,
                                    int vocab, void* embed_out, int64_t ldeo, int E, uint64_t* state, int M, int N,
                                    int K, unsigned flags, void* stream);

/* ---- int8 W8A8 (Int8Method) --------------------------------------------------
 * Per-token int8 quantization of the activations of Int8Method.apply
 * (qtts/quant/int8.py:138-140), each step in the activation dtype as torch
 * evaluates it on a CUDA tensor: c = max(amax_k |x[m,k]|, 1e-6 rounded to the
 * dtype); s = dtype(c * fl32(1 / 127)); q[m,k] = clamp(round_half_even(
 * dtype(x[m,k] / s)), -127, 127). q: [M, K] int8 (ld = K); scale_x: [M] fp32
 * holding s. Bit-exact with the reference's op sequence on the GPU. */
QTTS_API int qtts_int8_quant_rows(const void* x, int64_t ldx, int x_dtype, int8_t* q, float* scale_x, int M, int K,
                                  unsigned flags, void* stream);

/* int8 W8A8 GEMM: replaces torch._int_mm and the scaling of Int8Method.apply
 * (qtts/quant/int8.py:142-153, no 17-row padding):
 *   out[m,n] = cast( ((float(sum_k xq[m,k] * wq[n,k]) * scale_x[m]) * scale_w[n]) + bias[n] )
 * with an exact int32 sum (tcgen05.mma kind::i8) and the reference's fp32
 * roundings in that order. xq: [M, K] int8; wq: [N, K] int8 (K-major, i.e.
 * the reference's [K, N] int8_weight transposed); scale_w [N] fp32; bias [N]
 * of out_dtype or NULL. Variants as for qtts_fp8_gemm. */
QTTS_API int qtts_i8_gemm(const int8_t* xq, int64_t ldxq, const float* scale_x, const int8_t* wq, int64_t ldw,
                          const float* scale_w, const void* bias, void* out, int64_t ldo, int out_dtype, int M, int N,
                          int K, int variant, unsigned flags, void* stream);

/* ---- fp8 linear without caller-provided scratch ----------------------------
 * No counterpart in the reference. qtts_fp8_quant_rows followed by
 * qtts_fp8_gemm (variant AUTO) -- the whole of Fp8Method.apply -- with the
 * intermediate e4m3 codes and row scales kept in one fixed device array of the
 * library instead of memory the caller allocates, for callers with no device
 * allocator of their own. Nothing is allocated by the call.
 *   out[m,n] = same value as the two-step sequence on the same inputs.
 * x: [M, K] (BF16/FP16/FP32, ld ldx); wq: [N, K] e4m3 (ld ldw); scale_w: [N]
 * fp32; bias [N] of out_dtype or NULL; out: [M, N] of out_dtype (ld ldo).
 * Limits: M <= QTTS_NOALLOC_MAX_ROWS and M * K <= QTTS_NOALLOC_MAX_CODES, else
 * QTTS_ERR_SHAPE and nothing is launched. The array is shared by every call on
 * a device: calls that may run at the same time on one device (different
 * streams) race on it; calls ordered on one stream are safe. Nothing in it
 * needs to start at zero. The first call on each device looks its address up
 * (with that device current), so make one call before recording a graph. */
#define QTTS_NOALLOC_MAX_ROWS 1024
#define QTTS_NOALLOC_MAX_CODES (1 << 20)
QTTS_API int qtts_fp8_linear_noalloc(const void* x, int64_t ldx, int x_dtype,
                            const uint8_t* wq, int64_t ldw, const float* scale_w,
                            const void* bias, void* out, int64_t ldo, int out_dtype,
                            int M, int N, int K, unsigned flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QTTS_B200_H */
