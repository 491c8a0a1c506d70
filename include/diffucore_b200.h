/* C-ABI of diffucore_b200: the sm_100a W8A8 linear, activation quantizer and INT8 flash
 * attention that replace diffucore's quantized hot path.
 *
 * Conventions
 *  - Every function returns an int status: DC_OK (0) or a DC_ERR_* code; dc_last_error()
 *    then holds a one-line reason for the calling thread.
 *  - Pointers are device pointers unless stated. The library allocates and frees no device
 *    memory: outputs and workspaces come from the caller.
 *  - `stream` is a cudaStream_t (passed as void*); all work is enqueued on it, nothing
 *    synchronizes the host. Calls on distinct streams may run concurrently.
 *  - Shapes are int64_t; strides are in elements.
 *  - There is no CPU path: on a device other than sm_100 every compute entry point fails with
 *    DC_ERR_INVALID and says why.
 */
#ifndef DIFFUCORE_B200_H_
#define DIFFUCORE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DC_ABI_VERSION 1

#define DC_OK 0
#define DC_ERR_INVALID 1   /* bad argument, shape, stride, alignment or device */
#define DC_ERR_CUDA 2      /* a CUDA runtime call or launch failed */

#define DC_DTYPE_F32 0
#define DC_DTYPE_F16 1
#define DC_DTYPE_BF16 2
#define DC_DTYPE_I8 3
#define DC_DTYPE_I32 4

#define DC_GELU_NONE 0
#define DC_GELU_ERF 1      /* 0.5 x (1 + erf(x / sqrt 2)), rounded to the input dtype */
#define DC_GELU_TANH 2     /* 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), rounded likewise */

#define DC_ATTN_MODE_REF 0      /* Q per token, K per 64 keys after subtracting K's mean */
#define DC_ATTN_MODE_BLOCK64 1  /* Q and K per 64-token block, symmetric abs-max */

#define DC_QDIV_IEEE 0          /* correctly rounded divisions: the reference's torch-op (CPU) path */
#define DC_QDIV_FULL 1          /* div.full.f32 divisions: the reference's Triton (GPU) quantizers */

int dc_version(void);
const char* dc_last_error(void);

/* Division arithmetic of the per-row activation quantizers (dc_quant_rows, dc_quant_rows_seg,
 * dc_ln_mod_quant and the GEMM callers' codes), process-wide, taking effect for launches enqueued
 * after the call. The reference computes the two quotients of its quantizer,
 * scale = max(amax / 127, 1e-30) and code = rint(x / scale), differently depending on where it runs:
 * its torch-op path on the CPU (src/diffucore/models/_int8.py:87-97) rounds both correctly
 * (DC_QDIV_IEEE, the default: bit-exact with that path), its Triton kernels on a GPU
 * (`_store_quantized`, _int8.py:393-397, behind `quantize_activation` :299-310) divide with
 * div.full.f32 (DC_QDIV_FULL: bit-exact with those kernels). The two differ by one code step at
 * ~1.5e-4 of elements. The attention's Q/K codes follow the reference's CUDA kernels, whose
 * divisions are correctly rounded, in both modes. dc_quant_division() returns the current mode. */
int dc_set_quant_division(int mode);
int dc_quant_division(void);

/* Read (and optionally clear) the device-global error word that bounded in-kernel waits set
 * when they give up (1 = a wait timed out, 2 = the timeout self-test fired). Synchronous. */
int dc_device_error(unsigned int* code, int clear);

/* Per-row symmetric int8 quantization of x [M, K] (row stride ldx elements):
 *   (optional GELU, rounded to x's dtype) -> (optional 256-wide ConvRot rotation) ->
 *   s[m] = max(amax_m / 127, 1e-30);  q[m, k] = clamp(rint(x / s[m]), -128, 127)
 * q is [M, K] contiguous int8, s is [M] fp32. group is 0 or 256 (K % 256 == 0).
 * Replaces diffucore `quantize_activation` (src/diffucore/models/_int8.py:299-310), its
 * `_quantize_rows` / `_rotate` (:79-97) and the Triton `_rot_quant_kernel` (:399-406); with a
 * GELU mode it is `_gelu_quantize` / `_gelu_f16_rot_quant_kernel` (:348-358, :436-443). */
int dc_quant_rows(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int group, int gelu,
                  int8_t* q, float* s, void* stream);

/* out[M, N] = q[M, K] . w[N, K]^T with int32 accumulation on the tensor core, then
 *   out_dtype BF16 / F16:  y = dtype(float(acc) * (sx[m] * sw[n]));
 *                          if bias: y = dtype(float(y) + float(bias[n]))  (bias in out_dtype)
 *                          if gelu: y = GELU(y) rounded to dtype
 *   out_dtype I32:         out = acc (sx, sw, bias unused; gelu must be 0)
 * Leading dimensions ldq, ldw (bytes = elements) must be multiples of 16; K % 16 == 0.
 * Replaces `int_mm` (src/diffucore/models/_int8.py:200-207), `rescale` (:313-323),
 * `scaled_mm` (:266-276, whose sm75 kernel is src/diffucore/kernels/int8_gemm_sm75.cu:75-88)
 * and, with gelu, the first half of `int8_mlp` (:326-345). */
int dc_gemm_w8a8(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* sw,
                 const void* bias, void* out, int64_t ldo, int out_dtype, int64_t M, int64_t N, int64_t K,
                 int gelu, void* stream);

/* dc_gemm_w8a8 with the epilogue options a DiT block needs (bf16 / fp16 output):
 *  - gate [N] and residual [M, N] (row stride ldr), both or neither: after rescale and bias,
 *      out = dtype(residual + dtype(gate[n] * y))
 *    the gated residual branch `x + mod.gate * linear(h)` of FLUX blocks
 *    (src/diffucore/models/flux_dit.py:302-305, :339); residual may be out itself (in place).
 *    No GELU with a residual.
 *  - col_block > 0 (a multiple of 128; block_stride a multiple of 8): column n of row m goes to
 *      out + (n / col_block) * block_stride + m * ldo + n % col_block
 *    i.e. the output is laid out as [N / col_block, M, col_block] blocks, the send layout of an
 *    all-to-all that gives each destination its contiguous block. col_block = 0: plain [M, N]
 *    with row stride ldo (then block_stride must be 0).
 * Any out / residual alignment is accepted: stores and residual loads are 16 bytes wide where the
 * base pointer is 16-byte aligned and the row strides keep it so, element-wise otherwise. */
int dc_gemm_w8a8_ex(const int8_t* q, int64_t ldq, const int8_t* w, int64_t ldw, const float* sx, const float* sw,
                    const void* bias, int gelu, const void* gate, const void* residual, int64_t ldr, void* out,
                    int64_t ldo, int64_t col_block, int64_t block_stride, int out_dtype, int64_t M, int64_t N,
                    int64_t K, void* stream);

/* dc_quant_rows over rows gathered from segments (fp16 / bf16, no GELU): element c < k1 of row m
 * is at x + (c / seg_len) * seg_stride + m * ldx + c % seg_len, element c >= k1 at
 * x2 + m * ldx2 + (c - k1). seg_len, strides and offsets are multiples of 8 elements, seg_len
 * divides k1, k1 <= K <= 16384. With an all-to-all's receive buffer [P, M, seg_len] as x (and,
 * for a FLUX single-stream block, the MLP half as x2) this quantizes the concatenated row that
 * `linear2(cat(attn, mlp))` / `proj(attn)` consume (src/diffucore/models/flux_dit.py:335, :302)
 * without materialising it. Codes and scales equal dc_quant_rows on the gathered rows. */
int dc_quant_rows_seg(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int64_t seg_len,
                      int64_t seg_stride, int64_t k1, const void* x2, int64_t ldx2, int group, int8_t* q, float* s,
                      void* stream);

/* LayerNorm (no affine, eps 1e-6) + AdaLN modulation + int8 codes in one pass, for the
 * modulated inputs of FLUX blocks (src/diffucore/models/flux_dit.py:282, :287, :328):
 *   n = dtype(LN(x)); y = dtype(dtype(dtype(1 + scale[k]) * n) + shift[k])
 * then exactly dc_quant_rows(y, group). Rows m of batch element b = m / rows_per_mod use
 * shift/scale + b * mod_ld (fp16 / bf16 like x). K % 8 == 0, K <= 4096; x, shift, scale 16-byte
 * aligned. The modulated activation is never written. */
int dc_ln_mod_quant(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, const void* shift,
                    const void* scale, int64_t rows_per_mod, int64_t mod_ld, int group, int8_t* q, float* s,
                    void* stream);

/* In-place per-head RMSNorm + axial RoPE of q and k inside packed qkv rows (FLUX `QKNorm` and
 * `apply_rope`, src/diffucore/models/flux_dit.py:129-151, :179-184). Row r, head h (D = 128):
 * q at qkv + r * ld_row + q_off + h * D, k at + k_off + h * D.
 *   y = dtype(dtype(x * rsqrt(mean(x^2) + 1e-6)) * scale[d])
 *   (y0, y1) of rotary pair i -> dtype(f[i][0][0] y0 + f[i][0][1] y1), dtype(f[i][1][0] y0 + f[i][1][1] y1)
 * with pe fp32 [rows, D/2, 2, 2] (row r uses pe row pe_row0 + r). Rows r < split_row use
 * (q_scale0, k_scale0), the others (q_scale1, k_scale1): the text and image streams of a joint
 * double-stream attention. qkv 8-byte aligned with ld_row, q_off, k_off multiples of 4 elements;
 * scale vectors (D elements of dtype) 8-byte aligned; pe 16-byte aligned. */
int dc_qk_norm_rope(void* qkv, int dtype, int64_t L, int64_t H, int64_t D, int64_t ld_row, int64_t q_off,
                    int64_t k_off, const void* q_scale0, const void* k_scale0, const void* q_scale1,
                    const void* k_scale1, int64_t split_row, const float* pe, int64_t pe_row0, void* stream);

/* dc_qk_norm_rope that also emits the INT8 attention's Q codes and per-token scales (reference
 * quant mode) for one sequence (batch 1), straight into an attention workspace: head h of row r
 * gets codes q_codes[(h * q_lpad + r) * D ..] and scale q_rscale[h * q_lpad + r], bit for bit the
 * per-token quantization of dc_attn_int8_prep (int8_attn_sm80.cu:341-388) on the rounded q; rows
 * [L, q_lpad) get zeros. Pass the workspace's Q codes / Q scale addresses and its padded length
 * (dc_attn_workspace_layout), then run dc_attn_int8_prep_k and dc_attn_int8_main. write_q = 0
 * leaves q in qkv as it was (only the codes are produced). Fuses the reference's `QKNorm` +
 * `apply_rope` (flux_dit.py:129-151, :179-184) with the attention's Q quantization. */
int dc_qk_norm_rope_q8(void* qkv, int dtype, int64_t L, int64_t H, int64_t D, int64_t ld_row, int64_t q_off,
                       int64_t k_off, const void* q_scale0, const void* k_scale0, const void* q_scale1,
                       const void* k_scale1, int64_t split_row, const float* pe, int64_t pe_row0, int8_t* q_codes,
                       float* q_rscale, int64_t q_lpad, int write_q, void* stream);

/* out[M, N] = dtype(float(acc) * (sx[m] * sw[n])) (+ bias in dtype), acc int32 [M, N] with row
 * stride lda: the epilogue of dc_gemm_w8a8 as a separate pass, for an int32 result already in
 * hand. Replaces `rescale` (src/diffucore/models/_int8.py:313-323) and its Triton
 * `_rescale_kernel` (:408-417). */
int dc_rescale(const int32_t* acc, int64_t lda, const float* sx, const float* sw, const void* bias, void* out,
               int64_t ldo, int out_dtype, int64_t M, int64_t N, void* stream);

/* Workspace bytes (and its layout) for dc_attn_int8_fwd. layout[8] receives
 * {Lq_pad, Lk_pad, off_q_codes, off_k_codes, off_q_scale, off_k_scale, off_ksum, total}:
 * q codes int8 [B*H, Lq_pad, D], k codes int8 [B*H, Lk_pad, D], q scale fp32 [B*H, Lq_pad]
 * (per row), k scale fp32 [B*H, Lk_pad / 64], ksum fp32 [B*H, D] (mode REF only). */
int dc_attn_workspace_size(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int mode, size_t* bytes);
int dc_attn_workspace_layout(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int mode, int64_t* layout);

/* INT8 attention, non-causal: o = softmax(sm_scale * q k^T) v per (batch, head).
 * q [B, Lq, H, D], k and v [B, Lk, H, D] in fp16 or bf16 (dtype), each with its own element
 * strides {stride_b, stride_l, stride_h} (stride_d == 1), strides multiples of 8 and pointers
 * 16-byte aligned; o has the same dtype and its own strides. D is 64 or 128.
 * Q and K are quantized to int8 (mode REF: the reference's per-token Q and mean-centred
 * per-64-key K; mode BLOCK64: per-64-token blocks), S = Q.K^T is exact int32, softmax runs in
 * fp32 and P.V on the tensor core with P rounded to the input dtype and fp32 accumulation.
 * workspace: >= dc_attn_workspace_size bytes, 256-byte aligned, contents need not be zeroed.
 * The main kernel is picked by grid size (two 128-row Q tiles per CTA, or one with S double-
 * buffered when that fills the last wave better); environment DC_ATTN_KERNEL = "two_tile" or
 * "single_tile" pins one. Both give the same result within the stated tolerance.
 * Replaces the pybind `fwd(q, k, v, sm_scale)` of src/diffucore/kernels/int8_attn_sm80.cu:460-497
 * (and int8_attn_sm75.cu:477-514) called from `attention_blhd` / `attention_bhld`
 * (src/diffucore/models/_attention.py:216-217, :268-271). */
int dc_attn_int8_fwd(const void* q, const void* k, const void* v, int dtype, int64_t B, int64_t H, int64_t Lq,
                     int64_t Lk, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                     const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Only the quantization stage of dc_attn_int8_fwd: fills the workspace's Q/K codes and scales
 * (and ksum in mode REF), laid out as dc_attn_workspace_layout describes. Exposes the int8 codes
 * of the reference's prep kernels (int8_attn_sm80.cu:38-142, and the Q block of :341-388). */
int dc_attn_int8_prep(const void* q, const void* k, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk,
                      int64_t D, const int64_t* q_strides, const int64_t* k_strides, int mode, void* workspace,
                      size_t workspace_bytes, void* stream);

/* The K half of dc_attn_int8_prep (K codes, K scales and, in mode REF, ksum), for callers whose
 * Q codes are already in the workspace (dc_qk_norm_rope_q8). Replaces the reference's K prep
 * kernels (int8_attn_sm80.cu:38-142). */
int dc_attn_int8_prep_k(const void* k, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                        const int64_t* k_strides, int mode, void* workspace, size_t workspace_bytes, void* stream);

/* Only the attention stage of dc_attn_int8_fwd, over a workspace that dc_attn_int8_prep (same
 * B, H, Lq, Lk, D, mode) already filled: lets a caller quantize Q/K once (or elsewhere, e.g. before
 * a sequence-parallel exchange) and time or run the tensor-core kernel alone. */
int dc_attn_int8_main(const void* v, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                      const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                      void* workspace, size_t workspace_bytes, void* stream);

/* dc_attn_int8_main with the keys divided into ranges of ceil(n / nsplit) 128-key tiles (n = the
 * key tiles of Lk; 1 <= nsplit <= n): one CTA per (256 query rows, key range) instead of per 256
 * query rows, so a grid of few heads (a sequence-parallel rank's share) fills the GPU; each range
 * leaves its unnormalized output, running max and sum in `partials` (caller-owned, 256-byte
 * aligned, dc_attn_split_partials_size bytes) and a second kernel merges them and writes o.
 * Same inputs, workspace (from dc_attn_int8_prep) and output as dc_attn_int8_main; results agree
 * with it to rounding (the ranges are summed separately). Replaces the same reference call as
 * dc_attn_int8_fwd (pybind `fwd`, src/diffucore/kernels/int8_attn_sm80.cu:460-497), whose kernel
 * has no key split. */
int dc_attn_split_partials_size(int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D, int nsplit,
                                size_t* bytes);
int dc_attn_int8_main_split(const void* v, int dtype, int64_t B, int64_t H, int64_t Lq, int64_t Lk, int64_t D,
                            const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                            void* workspace, size_t workspace_bytes, int nsplit, void* partials,
                            size_t partial_bytes, void* stream);

/* dc_attn_int8_fwd for callers that cannot allocate device memory — an application whose GPU
 * memory is all owned by its own pool and cannot give this library a workspace, or that runs where
 * cudaMalloc's implicit synchronization is not allowed. Same arguments and results as
 * dc_attn_int8_fwd minus the workspace: the Q/K codes and scales live in one fixed device array of
 * DC_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads the library holds until
 * the process exits. Shapes whose workspace (dc_attn_workspace_size) exceeds that size are
 * rejected with DC_ERR_INVALID. Allocates nothing (no cudaMalloc / cudaFree). The first call on each
 * device looks up the array's device address (cudaGetSymbolAddress) with that device current, and
 * so does the first call after the device's context changed (cudaDeviceReset); make those calls
 * before any stream capture. All calls on a device share the one array and it
 * keeps the last call's contents (nothing in it needs to start at zero); calls that overlap on the
 * GPU (different streams) race on it, so order them on one stream or with events.
 * No counterpart in the reference (its pybind `fwd` always allocates its workspace). */
#define DC_NOALLOC_SCRATCH_BYTES (32u << 20)
int dc_attn_int8_fwd_noalloc(const void* q, const void* k, const void* v, int dtype, int64_t B, int64_t H,
                             int64_t Lq, int64_t Lk, int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, float sm_scale, int mode, void* o, const int64_t* o_strides,
                             void* stream);

/* Accuracy self-test of the attention softmax's FMA-pipe exp2 (range reduction + degree-3
 * polynomial): poly[i] = that exp2(x[i]), ref[i] = CUDA exp2f(x[i]); n even. No counterpart in the
 * reference (its kernel uses the MUFU ex2 only). */
int dc_selftest_exp2(const float* x, float* poly, float* ref, int64_t n, void* stream);

/* Failure-detection self-test: launches one CTA that waits on an mbarrier nothing arrives at,
 * bounded by limit_cycles. The wait gives up, writes 1 to *status_dev (device int) and sets the
 * device error word to 2. No counterpart in the reference (its kernels have no bounded waits). */
int dc_selftest_wait_timeout(long long limit_cycles, int* status_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DIFFUCORE_B200_H_ */
