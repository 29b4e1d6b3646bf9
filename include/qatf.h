/*
 * qatf.h -- C ABI of libqatf.so, the sm_100a (B200) kernels behind QATFactory's
 * fake-quantization path.
 *
 * Conventions shared by every entry point:
 *   - Pointers are raw CUDA device pointers owned by the caller; nothing here allocates
 *     device memory.  Tensors are row-major.  `ld` is the row stride of an input in
 *     elements (ld >= cols); outputs are dense ([rows, cols] with stride cols).
 *   - `dtype` of a floating-point tensor: QATF_F32, QATF_F16 or QATF_BF16.  Outputs that
 *     mirror an input ("y", "recon", "grad_in") have the input's dtype.
 *   - STE masks are bit masks over the flattened element index e = row * cols + col:
 *     element e is bit (e % 8) of byte (e / 8).  A mask buffer holds ceil(rows*cols/8)
 *     bytes.  Bit set = in range (gradient passes), exactly the reference's bool mask.
 *   - Every call is asynchronous on `stream` (a cudaStream_t passed as void*; NULL is
 *     the legacy default stream) and never synchronises the host.  Scalars that the
 *     reference reads from tensors (the NVFP4 tensor amax) are read from device memory.
 *   - Return value: QATF_OK (0) or a negative QATF_ERR_* code; qatf_status_string()
 *     names it.  Argument errors are detected before any launch.
 *
 * Each entry point names the reference function (file:line, relative to the
 * QATFactory checkout) whose semantics it reproduces bit for bit, and the Triton launch
 * wrapper it replaces where one exists.
 */
#ifndef QATF_H
#define QATF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QATF_F32 0
#define QATF_F16 1
#define QATF_BF16 2

#define QATF_OK 0
#define QATF_ERR_INVALID (-1)     /* null pointer, bad shape or bad argument */
#define QATF_ERR_DTYPE (-2)       /* unsupported dtype code */
#define QATF_ERR_LAUNCH (-3)      /* a CUDA launch or runtime call failed */
#define QATF_ERR_DEVICE (-4)      /* current device is not sm_100 */
#define QATF_ERR_TIMEOUT (-5)     /* a device-side bounded wait expired */
#define QATF_ERR_UNSUPPORTED (-6) /* shape outside what this entry point supports */

/* Library version (major * 10000 + minor * 100 + patch). */
int qatf_version(void);

/* Human-readable text for a status code (static storage). */
const char *qatf_status_string(int status);

/* Number of kernels this library has launched successfully in the calling process (all
 * devices and threads).  Diagnostics only; no counterpart in the reference. */
uint64_t qatf_launch_count(void);

/* ------------------------------------------------------------------------ amax */

/* amax_out[0] = max |x| over n elements of a dense tensor, as FP32; NaN propagates.
 * Replaces `weight.detach().abs().amax().float()` (qatfactory/quant/formats/nvfp4.py:531,
 * :635, :655; refresh :271). */
int qatf_tensor_amax(const void *x, int dtype, int64_t n, float *amax_out, void *stream);

/* Running maximum: amax_inout[0] = max(amax_inout[0], max |x|) in one launch; amax_inout must
 * hold an earlier maximum of absolute values (+0 or more, or NaN); NaN propagates.  The
 * training-input running maximum of NVFP4Linear.forward, `torch.maximum(self._input_amax,
 * x.abs().amax())` (qatfactory/quant/formats/nvfp4.py:654-656), without the separate
 * maximum. */
int qatf_tensor_amax_update(const void *x, int dtype, int64_t n, float *amax_inout, void *stream);

/* amax_out[b] = max |x[b * n .. b * n + n)| for b < batches (dense, one launch); NaN propagates.
 * The per-expert tensor amax of a fused MoE expert weight [experts, rows, cols]:
 * `weight.detach().abs().amax(dim=(1, 2)).float()` (qatfactory/quant/formats/nvfp4_experts.py:
 * 609-610).  batches <= 65535. */
int qatf_tensor_amax_batched(const void *x, int dtype, int64_t batches, int64_t n, float *amax_out, void *stream);

/* ----------------------------------------------------------------------- NVFP4 */

/* NVFP4 fake quantize-dequantize with E4M3 block-16 scales and the FP32 tensor scale
 * tensor_amax[0] / 2688 read from device memory; y has x's dtype; mask_bits may be NULL.
 * cols need not be a multiple of 16 (rows are zero-padded per block).
 * Semantics: _fake_quantize_nvfp4_torch (qatfactory/quant/formats/nvfp4.py:465-501) with
 * the zero-amax rule of fake_quantize_nvfp4 (:540-543).
 * Replaces triton_fake_quantize_nvfp4 (qatfactory/quant/formats/fp4_triton.py:259-272). */
int qatf_nvfp4_qdq(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float *tensor_amax,
                   void *y, uint8_t *mask_bits, void *stream);

/* NVFP4 fake quantization of the BF16 rounding of an FP32 tensor, written back in FP32:
 * out = float(qdq(bf16(latent))) and the STE mask of bf16(latent), bit-identical (finite
 * inputs) to qatf_nvfp4_qdq on latent.to(bfloat16) followed by a widening copy.  Dense
 * [rows, cols], cols % 16 == 0, latent and out 32-byte aligned, mask_bits 2-byte aligned (all
 * required).  It quantizes a rank's FP32 latent shard once per optimizer step so that FSDP2
 * gathers the quantized weight: the reference instead fake-quantizes the gathered BF16 weight
 * in every forward (NVFP4Linear.forward, qatfactory/quant/formats/nvfp4.py:657-658, after the
 * FSDP2 cast to BF16); row sharding keeps every block inside one shard.  No single reference
 * function corresponds. */
int qatf_nvfp4_qdq_shadow(const float *latent, int64_t rows, int64_t cols, const float *tensor_amax, float *out,
                          uint8_t *mask_bits, void *stream);

/* NVFP4 QDQ of a fused MoE expert weight [experts, rows, cols] (dense, cols % 16 == 0) with one
 * tensor amax per expert (tensor_amax[experts] on the device): expert e is exactly
 * qatf_nvfp4_qdq of its [rows, cols] slice with tensor_amax + e (a zero amax gives zeros and an
 * all-true mask); y and mask_bits cover the flattened [experts, rows, cols] tensor.  BF16 runs
 * as one launch over all experts.  Semantics: _fake_quantize_nvfp4_experts_values
 * (qatfactory/quant/formats/nvfp4_experts.py:438-462); the reference validates the amax vector
 * on the host first (:433-435), which the caller does. */
int qatf_nvfp4_qdq_experts(const void *x, int dtype, int64_t experts, int64_t rows, int64_t cols,
                           const float *tensor_amax, void *y, uint8_t *mask_bits, void *stream);

/* As qatf_nvfp4_qdq with the tensor amax computed on the device first (written to
 * amax_scratch[0], one caller-owned FP32 scratch word).  This is fake_quantize_nvfp4(weight)
 * without tensor_amax (qatfactory/quant/formats/nvfp4.py:531-539). */
int qatf_nvfp4_fake_quant(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, float *amax_scratch,
                          void *y, uint8_t *mask_bits, void *stream);

/* Largest tensor (rows * cols elements) qatf_nvfp4_fake_quant_noalloc accepts. */
#define QATF_NOALLOC_MAX_ELEMENTS (8192LL * 65536LL)

/* As qatf_nvfp4_fake_quant, for callers that cannot allocate device memory: the tensor
 * amax is reduced in a static device array inside the library instead of a caller-owned
 * scratch word, so only x, y and mask_bits are passed.  No counterpart in the reference
 * (the reference always has torch's allocator).  Dense tensors only (ld == cols); tensors
 * of more than QATF_NOALLOC_MAX_ELEMENTS elements return QATF_ERR_UNSUPPORTED.  Every call
 * resolves the array's address on the CURRENT device (cudaGetSymbolAddress), so call it with
 * the device that owns `stream` current; the first call on a device loads the library's
 * module there and should come before any stream capture.  The array is shared by every call
 * on a device: calls that overlap on the GPU race and must be serialised by the caller. */
int qatf_nvfp4_fake_quant_noalloc(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, void *y,
                                  uint8_t *mask_bits, void *stream);

/* NVFP4 pack for export (cols % 16 == 0): packed [rows, cols/2] nibbles (even column in
 * the low nibble), scales [rows, cols/16] E4M3 bytes, weight_scale_2[0] FP32 and an
 * optional reconstruction (recon may be NULL; x's dtype).
 * Semantics: quantize_nvfp4 (qatfactory/quant/formats/nvfp4.py:400-462). */
int qatf_nvfp4_pack(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float *tensor_amax,
                    uint8_t *packed, uint8_t *scales, float *weight_scale_2, void *recon, void *stream);

/* FP32 dequantization of packed NVFP4 (cols % 16 == 0, weight_scale_2 on device).
 * Semantics: dequantize_nvfp4 (qatfactory/quant/formats/nvfp4.py:104-121). */
int qatf_nvfp4_dequant(const uint8_t *packed, const uint8_t *scales, const float *weight_scale_2, int64_t rows,
                       int64_t cols, float *out, void *stream);

/* ----------------------------------------------------------------------- MXFP4 */

/* MXFP4 weight QDQ, EVEN-rule E8M0 block-32 scales; mask_bits may be NULL; cols need
 * not be a multiple of 32.  Semantics: _fake_quantize_mxfp4_torch
 * (qatfactory/quant/formats/mxfp4.py:154-174).  Replaces triton_fake_quantize_mxfp4
 * (qatfactory/quant/formats/fp4_triton.py:275-285). */
int qatf_mxfp4_qdq_even(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, void *y,
                        uint8_t *mask_bits, void *stream);

/* MXFP4 activation QDQ, CEIL-rule E8M0 block-32 scales (cols % 32 == 0); the STE mask is
 * all-true so none is written.  Semantics: _fake_quantize_mxfp4_activation_torch
 * (qatfactory/quant/formats/mxfp4.py:205-222).  Replaces
 * triton_fake_quantize_mxfp4_activation (qatfactory/quant/formats/fp4_triton.py:288-297). */
int qatf_mxfp4_qdq_ceil(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, void *y, void *stream);

/* MXFP4 pack (cols % 32 == 0): packed [rows, cols/2], biased E8M0 scales [rows, cols/32],
 * optional reconstruction.  Semantics: quantize_mxfp4 (qatfactory/quant/formats/mxfp4.py:126-151). */
int qatf_mxfp4_pack(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, uint8_t *packed,
                    uint8_t *scales, void *recon, void *stream);

/* FP32 dequantization of packed MXFP4.  Semantics: dequantize_mxfp4
 * (qatfactory/quant/formats/mxfp4.py:101-116). */
int qatf_mxfp4_dequant(const uint8_t *packed, const uint8_t *scales, int64_t rows, int64_t cols, float *out,
                       void *stream);

/* ------------------------------------------------------------- shared FP4 pieces */

/* grad_in = grad_out * in_range over n dense elements (mask as above).
 * Semantics: _MaskedStraightThrough.backward (qatfactory/quant/formats/nvfp4.py:39-41,
 * q4_k.py:62-65). */
int qatf_ste_backward(const void *grad_out, int dtype, int64_t n, const uint8_t *mask_bits, void *grad_in,
                      void *stream);

/* Pack canonical E2M1 nibbles [rows, cols] (cols even) into bytes [rows, cols/2], even
 * column in the low nibble.  Semantics: pack_e2m1_rows (qatfactory/quant/formats/nvfp4.py:76-85). */
int qatf_e2m1_pack_rows(const uint8_t *nibbles, int64_t rows, int64_t cols, uint8_t *packed, void *stream);

/* Inverse of qatf_e2m1_pack_rows.  Semantics: unpack_e2m1_rows (nvfp4.py:88-101). */
int qatf_e2m1_unpack_rows(const uint8_t *packed, int64_t rows, int64_t packed_cols, uint8_t *nibbles,
                          void *stream);

/* ------------------------------------------------------------------------ Q4_K */

#define QATF_Q4K_GRID_SEARCH 0
#define QATF_Q4K_MINMAX 1

/* Q4_K super-block encoder (cols % 256 == 0).  Any of recon (x's dtype), mask_bits and
 * blocks ([rows, cols/256*144] bytes of ggml block_q4_K) may be NULL.
 * Semantics: _encode_superblocks_torch + quantize_q4_k / fake_quantize_q4_k
 * (qatfactory/quant/formats/q4_k.py:139-340).  Replaces triton_encode_superblocks
 * (qatfactory/quant/formats/q4_k_triton.py:146-204), and is bit-exact where that kernel
 * agrees only on ~99.4% of weights. */
int qatf_q4k_encode(const void *x, int dtype, int64_t rows, int64_t cols, int64_t ld, int method, void *recon,
                    uint8_t *mask_bits, uint8_t *blocks, void *stream);

/* FP32 dequantization of block_q4_K bytes.  Semantics: dequantize_q4_k
 * (qatfactory/quant/formats/q4_k.py:359-385). */
int qatf_q4k_dequant(const uint8_t *blocks, int64_t rows, int64_t cols, float *out, void *stream);

/* ------------------------------------------------------------ block-FP8 frozen bases */

#define QATF_FP8_E4M3 0
#define QATF_FP8_E5M2 1

/* out[b, r, c] = float(codes[b, r, c]) * scale_inv[b, r / (rows / scale_rows), c / (cols /
 * scale_cols)], rounded to out_dtype (QATF_F32 / F16 / BF16), over `batches` dense
 * [rows, cols] FP8 code tensors (float8_e4m3fn or float8_e5m2 bytes) with dense FP32 scale
 * grids [batches, scale_rows, scale_cols]; rows % scale_rows == 0 and cols % scale_cols == 0.
 * Bit-identical to dequantize_fp8_blocks (qatfactory/quant/formats/fp8_base.py:27-52), which
 * frozen block-FP8 LoRA bases call per weight and per fused expert tensor (nvfp4.py:623-627,
 * nvfp4_experts.py:213-223). */
int qatf_fp8_block_dequant(const uint8_t *codes, int fp8_format, int64_t batches, int64_t rows, int64_t cols,
                           const float *scale_inv, int64_t scale_rows, int64_t scale_cols, void *out, int out_dtype,
                           void *stream);

/* -------------------------------------------------------------- W4A4 GEMMs (tcgen05) */

/* Operand layouts of qatf_bf16_gemm: A [M, K] (K_MAJOR) or stored transposed as [K, M]
 * (MN_MAJOR); B [N, K] (K_MAJOR) or [K, N] (MN_MAJOR); all dense row-major. */
#define QATF_K_MAJOR 0
#define QATF_MN_MAJOR 1

/* Roles of an NVFP4 GEMM operand; the role fixes the byte layout of its block scales, which
 * follows the tensor-memory layout the tcgen05 block-scaled MMA reads (scales of one 16-column
 * block are E4M3 bytes; the four blocks of a 64-column K-block kb form one 32-bit word
 * w(r, kb)).  Both layouts are made of 4096-byte blocks that one tcgen05.cp 128x256b copies:
 * lane L (0..127) of a block holds eight words, word v at (L / 8) * 256 + (L % 8) * 16 +
 * (v / 4) * 128 + (v % 4) * 4, and w(r, kb) is stored in each of the four lanes
 * L = r % 32 + 32 q (q = 0..3).
 *   QATF_OPERAND_A (rows % 128 == 0, cols % 128 == 0): block (r / 128, kb / 2) at
 *     ((r / 128) * (cols / 128) + kb / 2) * 4096, word v = 4 * (kb % 2) + (r / 32) % 4.
 *   QATF_OPERAND_B (rows % 256 == 0, cols % 64 == 0): block (r / 256, kb) at
 *     ((r / 256) * (cols / 64) + kb) * 4096, word v = (r / 32) % 8.
 * Either way 4 * rows * cols / 16 bytes. */
#define QATF_OPERAND_A 0
#define QATF_OPERAND_B 1
#define QATF_NVFP4_OPERAND_SCALE_BYTES(rows, cols) (4 * (rows) * ((cols) / 16))

/* NVFP4 quantization of a BF16 [rows, cols] tensor into the operand form of qatf_nvfp4_gemm,
 * in one pass: E2M1 codes [rows, cols/2] (even column in the low nibble), E4M3 block scales in
 * the layout of `role` (above), and optionally the dequantized tensor (deq, BF16, equal to
 * qatf_nvfp4_qdq's y) and the STE mask bits.
 * Codes and scales are those of quantize_nvfp4 (qatfactory/quant/formats/nvfp4.py:400-462);
 * deq and mask are _fake_quantize_nvfp4_torch's (nvfp4.py:465-501); a zero tensor amax gives
 * zero codes, scale bytes 0x01 (2^-9), zero deq and an all-true mask.  This is the producer
 * half of fake_quantize_nvfp4_activation + F.linear in NVFP4Linear.forward (nvfp4.py:636-658). */
int qatf_nvfp4_operand(const void *x, int dtype, int64_t rows, int64_t cols, const float *tensor_amax, int role,
                       uint8_t *codes, uint8_t *scales, void *deq, uint8_t *mask_bits, void *stream);

/* qatf_nvfp4_operand that also folds max |x| into a running maximum in the same pass:
 * running_amax[0] = max(running_amax[0], max |x|) when running_amax is not NULL (FP32 on the
 * device, 4-byte aligned, holding +0 or more, or NaN; NaN propagates).  This is the
 * training-input running maximum NVFP4Linear keeps for W4A4 (`self._input_amax =
 * torch.maximum(self._input_amax, input.detach().abs().amax().float())`,
 * qatfactory/quant/formats/nvfp4.py:634-648) without a separate pass over the activation. */
int qatf_nvfp4_operand_tracked(const void *x, int dtype, int64_t rows, int64_t cols, const float *tensor_amax,
                               int role, uint8_t *codes, uint8_t *scales, void *deq, uint8_t *mask_bits,
                               float *running_amax, void *stream);

/* Block-scaled NVFP4 GEMM on the tensor cores: out[M, N] (BF16, row-major) =
 * (a_amax/2688) * (b_amax/2688) * sum_k A[m, k] * B[n, k] with A and B from
 * qatf_nvfp4_operand in the roles QATF_OPERAND_A and QATF_OPERAND_B.  M % 128, N % 256 and K % 256 must be 0 (else
 * QATF_ERR_UNSUPPORTED).  All the GEMM entry points below also refuse M > 128 * 65535,
 * N or K > 2^30, and grids of more than 2^31 - 1 output tiles of 128 x 256 (QATF_ERR_UNSUPPORTED).
 * `err` is a caller-owned device int, zero on entry: a kernel whose
 * bounded waits expire sets it to nonzero and leaves its tile unwritten.  Replaces
 * F.linear(fq_act(x), fq(w)) of NVFP4Linear.forward for W4A4 (nvfp4.py:636-658). */
int qatf_nvfp4_gemm(const uint8_t *a_codes, const uint8_t *a_scales, const float *a_amax, const uint8_t *b_codes,
                    const uint8_t *b_scales, const float *b_amax, int64_t m, int64_t n, int64_t k, void *out,
                    int *err, void *stream);

/* E8M0 exponent rules of an MXFP4 operand: EVEN for weights (_e8m0_exponent_even,
 * qatfactory/quant/formats/mxfp4.py:48-60), CEIL for activations (_e8m0_exponent_ceil, :63-98). */
#define QATF_MXFP4_EVEN 0
#define QATF_MXFP4_CEIL 1

/* MXFP4 quantization of a BF16 [rows, cols] tensor into the operand form of qatf_mxfp4_gemm, in
 * one pass: E2M1 codes [rows, cols/2] (even column in the low nibble), E8M0 block-32 scale bytes
 * in the layout of `role`, and optionally the dequantized tensor (deq, BF16, equal to
 * qatf_mxfp4_qdq_even's / qatf_mxfp4_qdq_ceil's y) and the STE mask bits (EVEN: |x| <= 6 * 2^k;
 * all true under CEIL, whose straight-through gradient is unmasked, mxfp4.py:225-255).  The
 * scale layout is that of the NVFP4 roles above with 128-column K-blocks: the four block-32
 * scales of columns [128 kb, 128 kb + 128) of row r form the word w(r, kb);
 *   QATF_OPERAND_A (rows % 128 == 0, cols % 256 == 0): block (r / 128, kb / 2) at
 *     ((r / 128) * (cols / 256) + kb / 2) * 4096, word v = 4 * (kb % 2) + (r / 32) % 4;
 *   QATF_OPERAND_B (rows % 256 == 0, cols % 128 == 0): block (r / 256, kb) at
 *     ((r / 256) * (cols / 128) + kb) * 4096, word v = (r / 32) % 8;
 * either way 4 * rows * cols / 32 bytes.  Codes and scales are quantize_mxfp4's for EVEN
 * (mxfp4.py:126-151).  This is the producer half of MXFP4Linear.forward with W4A4
 * (F.linear(fake_quantize_mxfp4_activation(x), fake_quantize_mxfp4(w)), mxfp4.py:285-290). */
#define QATF_MXFP4_OPERAND_SCALE_BYTES(rows, cols) (4 * (rows) * ((cols) / 32))
int qatf_mxfp4_operand(const void *x, int dtype, int64_t rows, int64_t cols, int role, int rule, uint8_t *codes,
                       uint8_t *scales, void *deq, uint8_t *mask_bits, void *stream);

/* Block-scaled MXFP4 GEMM on the tensor cores (tcgen05 kind::mxf4, UE8M0 block-32 scales):
 * out[M, N] (BF16, row-major) = sum_k A[m, k] * B[n, k] with A and B from qatf_mxfp4_operand
 * in the roles QATF_OPERAND_A and QATF_OPERAND_B.  M % 128, N % 256 and K % 256 must be 0 (else
 * QATF_ERR_UNSUPPORTED); `err` as for qatf_nvfp4_gemm.  Replaces the F.linear of
 * MXFP4Linear.forward for W4A4 (mxfp4.py:290). */
int qatf_mxfp4_gemm(const uint8_t *a_codes, const uint8_t *a_scales, const uint8_t *b_codes, const uint8_t *b_scales,
                    int64_t m, int64_t n, int64_t k, void *out, int *err, void *stream);

/* Words of the caller-owned `sync` scratch of qatf_nvfp4_linear_fwd: one readiness counter per
 * (128-row tile, 256-column K stage) of X plus one work counter. */
#define QATF_NVFP4_LINEAR_SYNC_WORDS(m, k) (((m) / 128) * ((k) / 256) + 1)

/* W4A4 NVFP4 linear forward with the activation quantizer inside the GEMM kernel: out[M, N]
 * (BF16) = F.linear(fq_act(x), fq(w)) for BF16 x [M, K] with the static tensor amax x_amax[0],
 * the weight already in operand form (w_codes / w_scales from qatf_nvfp4_operand in role
 * QATF_OPERAND_B, tensor amax w_amax[0]).  One launch: beside the GEMM's producer, MMA and
 * epilogue warps, every CTA runs quantizer warps that encode X, 32 rows x 256 columns at a time
 * in the order the GEMM's tile schedule consumes them, into x_codes / x_scales (exactly
 * qatf_nvfp4_operand's codes and QATF_OPERAND_A scales, which the GEMM reads back by TMA,
 * mostly from L2) and, when not NULL, x_deq and x_mask (qatf_nvfp4_qdq's y and mask, for the
 * backward pass).  The producer loads an A stage once its four quarter panels are published
 * (one release counter per panel in `sync`, QATF_NVFP4_LINEAR_SYNC_WORDS(m, k) caller-owned
 * words, zeroed by this call on `stream`); any resident CTA's quantizer warps take the next
 * panel, so a wait always ends.  The output equals qatf_nvfp4_operand(x) followed by
 * qatf_nvfp4_gemm bit for bit.  M % 128, N % 256 and K % 256 must be 0; `err` as for
 * qatf_nvfp4_gemm (value 2: a panel wait expired).  Replaces fake_quantize_nvfp4_activation +
 * F.linear in NVFP4Linear.forward (qatfactory/quant/formats/nvfp4.py:636-658). */
int qatf_nvfp4_linear_fwd(const void *x, const float *x_amax, const uint8_t *w_codes, const uint8_t *w_scales,
                          const float *w_amax, int64_t m, int64_t n, int64_t k, uint8_t *x_codes, uint8_t *x_scales,
                          void *x_deq, uint8_t *x_mask, uint32_t *sync, void *out, int *err, void *stream);

/* BF16 GEMM on the tensor cores with FP32 accumulation: out[M, N] (BF16) = A B^T, optionally
 * multiplied by STE mask bits over out's flat index (mask_bits may be NULL).  M % 128,
 * N % 256 and K % 64 must be 0.  `err` as for qatf_nvfp4_gemm.  The backward of the W4A4
 * linear: dX = STE_x(dY @ W_q) (A = dY K-major, B = W_q MN-major) and dW = STE_w(dY^T @ X_q)
 * (A = dY MN-major, B = X_q MN-major) (nvfp4.py:32-41 applied to F.linear). */
int qatf_bf16_gemm(const void *a, int a_layout, const void *b, int b_layout, int64_t m, int64_t n, int64_t k,
                   const uint8_t *mask_bits, void *out, int *err, void *stream);

/* Bytes of caller-owned workspace with which qatf_bf16_gemm_ws splits the K dimension of a
 * last wave of 256 x 256 tiles that would otherwise leave most SM pairs idle (0 when the shape
 * does not need it or M % 256 != 0).  Depends on the current device's co-resident CTA pairs. */
int64_t qatf_bf16_gemm_workspace_size(int64_t m, int64_t n, int64_t k);

/* qatf_bf16_gemm with a workspace (32-byte aligned): given at least
 * qatf_bf16_gemm_workspace_size(m, n, k) bytes, the last wave's tiles are computed as K-slices
 * whose FP32 partial tiles are summed in slice order by a second kernel before the mask and
 * the BF16 rounding (FP32 accumulation order differs from the whole-tile path only there);
 * with a NULL or smaller workspace it is exactly qatf_bf16_gemm.  The wgrad of the W4A4
 * backward (dW = STE_w(dY^T @ X_q), nvfp4.py:32-41) is the shape this is for. */
int qatf_bf16_gemm_ws(const void *a, int a_layout, const void *b, int b_layout, int64_t m, int64_t n, int64_t k,
                      const uint8_t *mask_bits, void *out, int *err, void *workspace, int64_t workspace_bytes,
                      void *stream);

/* ------------------------------------------------------- distillation loss (config 5) */

/* Forward KL of student logits s against teacher logits t over the vocabulary, row by row:
 * row_loss[r] = T^2 * KL(softmax(t_r / T) || softmax(s_r / T)) (FP32; 0 where row_valid[r] == 0,
 * row_valid may be NULL), and, when grad is not NULL, grad[r, :] (dense, s's dtype) =
 * grad_scale * T * (softmax(s_r / T) - softmax(t_r / T)) (0 for invalid rows).  ld_s / ld_t are
 * the row strides of s and t in elements.  Semantics: distill_loss with hard_label_weight 0
 * (qatfactory/distill/kd_loss.py:147-195), which sums kl_div over FP32 chunks of log_softmax /
 * softmax; this computes the same quantities in one pass per row (online softmax), so results
 * agree to FP32 rounding, not bit for bit. */
int qatf_kd_forward_kl(const void *student, const void *teacher, int dtype, int64_t rows, int64_t vocab,
                       int64_t ld_s, int64_t ld_t, float temperature, const uint8_t *row_valid, float *row_loss,
                       void *grad, float grad_scale, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* QATF_H */
