/*
 * dollama_b200 — C ABI of the B200-native (sm_100a) dense-contraction hot path of dollama:
 * the SDXL UNet / VAE matmuls (implicit-GEMM conv2d, transformer linears, flash attention)
 * and the BitNet tag-LM ternary x int8 GEMM/GEMV.
 *
 * Conventions for every entry point:
 *   - pointers are DEVICE pointers unless the name says `host`; sizes are element counts;
 *   - work is enqueued on `stream` (0 = legacy default stream) and returns without a sync;
 *   - the return value is a dlm_status: 0 on success, negative on failure; the message of
 *     the last failure on the calling thread is available from dlm_last_error();
 *   - empty problems (any size 0) return DLM_OK without launching, as the reference's
 *     launchers silently return on empty dims (src/kernels/conv2d.cu:762-770,
 *     src/kernels/attention_fast.cu:295-298);
 *   - fp16 is IEEE binary16 passed as `void*` / `const void*` (no CUDA types in signatures);
 *     cudaStream_t is passed as `void*`.
 *
 * Activations of the UNet / VAE entry points are NHWC (token-major) inside this library;
 * the model-level entry points take and return the reference's NCHW tensors.
 */
#ifndef DOLLAMA_B200_H_
#define DOLLAMA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum dlm_status {
  DLM_OK = 0,
  DLM_ERR_INVALID = -1,      /* bad argument (null pointer, unsupported shape/alignment)     */
  DLM_ERR_CUDA = -2,         /* a CUDA runtime/driver call failed                            */
  DLM_ERR_TIMEOUT = -3,      /* a kernel gave up a bounded wait (see dlm_get_device_status)  */
  DLM_ERR_UNSUPPORTED = -4,  /* valid in the reference but not provided by this library      */
  DLM_ERR_NOMEM = -5,        /* device memory / arena exhausted                              */
  DLM_ERR_NOT_FOUND = -6     /* a named weight tensor is missing                             */
} dlm_status;

/* ------------------------------------------------------------------ library */

/* Message of the last failed call on this thread ("" if none). */
const char* dlm_last_error(void);

/* Library version string. */
const char* dlm_version(void);

/* Reads (and clears when `clear` != 0) the device status word of the current device:
 * 0 = no kernel gave up a wait; otherwise the code of the first kernel role that timed out.
 * Synchronizes `stream`. */
int dlm_get_device_status(int* out_code, int clear, void* stream);

/* Asynchronous copy between any two (device or host) buffers on `stream`. */
int dlm_memcpy(void* dst, const void* src, size_t bytes, void* stream);

/* ------------------------------------------------------------------ GEMM (tcgen05)
 *
 * Replaces launch_gemm_fp16 (reference src/kernels/gemm.cuh:44-53, gemm.cu:518):
 *   C[M,N] = alpha * op(A)[M,K] * op(B)[K,N] + beta * C, row-major fp16, fp32 accumulate.
 * transA = 0 / transB = 1 (B is [N,K], PyTorch Linear layout, the form of the reference's UNet /
 * VAE / LM paths) runs directly; the other orientations are first transposed into
 * stream-ordered scratch (cudaMallocAsync on `stream`).  M, N, K % 8 == 0 where transposed.
 */
int dlm_launch_gemm_fp16(const void* A, const void* B, void* C, int M, int N, int K, float alpha,
                         float beta, int transA, int transB, void* stream);

/* Replaces launch_gemm_fp16_batched (src/kernels/gemm.cuh:100-175): item i multiplies
 * A + i*stride_a, B + i*stride_b into C + i*stride_c (strides in elements, 0 = shared operand),
 * same alpha / beta / trans_b semantics as dlm_launch_gemm_fp16 (transA = 0). */
int dlm_gemm_fp16_batched(const void* A, const void* B, void* C, int batch, int M, int N, int K,
                          long long stride_a, long long stride_b, long long stride_c, float alpha,
                          float beta, int trans_b, void* stream);

/* Replaces launch_gemm_f32 (src/kernels/gemm.cuh:61-70): fp32 row-major
 * C = alpha * op(A) op(B) + beta * C (C not read when beta == 0), fp32 FMA accumulation on the
 * CUDA cores.  Not on any model path of this library (the VAE keeps fp32 carries through the
 * fp16 tensor-core GEMM with a scale, see dlm_vae_create). */
int dlm_gemm_f32(const float* A, const float* B, float* C, int M, int N, int K, float alpha, float beta,
                 int transA, int transB, void* stream);

/* Epilogue flags of dlm_gemm_fp16_ex. */
#define DLM_EPI_BIAS 1u     /* + bias[n]                                                */
#define DLM_EPI_RESID 2u    /* + residual[m, n] (residual may alias C, in place)        */
#define DLM_EPI_GEGLU 4u    /* columns interleaved (x1_j, x2_j): C[m, j] = x1 * gelu(x2) */
#define DLM_EPI_SILU 8u     /* SiLU after bias                                          */
#define DLM_EPI_BIAS2D 16u  /* + bias2d[m / rows_per_img, n] (per-image channel bias)   */

/* Fused linear: C[M, ldc] = epi(A[M,K] (row stride lda) * W[N,K]^T).  With DLM_EPI_GEGLU the
 * output has N/2 columns.  Fuses the reference's GEMM + launch_bias_add_rowvec +
 * launch_add + launch_geglu sequence (src/infer/unet.cu:517-526, 759-770). */
int dlm_gemm_fp16_ex(const void* A, int lda, const void* W, void* C, int ldc, int M, int N, int K,
                     unsigned flags, const void* bias, const void* bias2d, int rows_per_img,
                     const void* residual, int ldr, void* stream);

/* The same fused linear with a stream-K workspace: when the launch has fewer output tiles than
 * SMs, its k-block iterations may be split over every SM, the CTAs that hold a tile's later
 * k-blocks handing fp32 partial sums to the CTA holding its first ones through `workspace`
 * (dlm_gemm_workspace_bytes() bytes, 256-byte aligned, ZEROED once before its first use; every
 * call leaves it ready for the next).  Calls sharing a workspace must not overlap on the GPU.
 * flags: DLM_EPI_BIAS / RESID / GEGLU / SILU.  workspace == NULL behaves as dlm_gemm_fp16_ex. */
size_t dlm_gemm_workspace_bytes(void);
int dlm_gemm_fp16_ws(const void* A, int lda, const void* W, void* C, int ldc, int M, int N, int K,
                     unsigned flags, const void* bias, const void* residual, int ldr, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Tile-kernel selection for the GEMM / conv entry points planned after the call (process-wide):
 * mode & 15: 0 = automatic (cost model), 1 = single-CTA kernel only, 2 = CTA-pair
 * (cta_group::2) kernel where M > 128, 3 = stream-K over all SMs (where a workspace is given);
 * mode >> 4: forced N tile width (0 = cost model; 64, 128, 160, 192, 256).  For tests and A/B
 * measurements. */
int dlm_gemm_set_tile_mode(int mode);

/* ------------------------------------------------------------------ small reference kernels
 *
 * The reference's broadcast / activation / layout host functions with its layouts and rounding
 * (h = round to fp16, f = fp32): the model handles of this library fuse all of them into GEMM
 * epilogues; these serve other callers.  Empty sizes return DLM_OK without launching. */
/* bias_add.cuh:32   out[t, c] = h(f(in[t, c]) + f(bias[c])), [tokens, C] (in place allowed) */
int dlm_bias_add_rowvec(const void* in, const void* bias, void* out, int tokens, int C, void* stream);
/* bias_add.cuh:51   NCHW, out[n, c, h, w] = h(f(in) + f(bias[c])) */
int dlm_bias_add_channel(const void* in, const void* bias, void* out, int N, int C, int H, int W,
                         void* stream);
/* bias_add.cuh:75   NCHW, t = h(f(conv) + f(conv_bias[c])); out = h(f(t) + f(tproj[n * Cout + c])) */
int dlm_conv_bias_biasch(const void* conv, const void* conv_bias, const void* tproj, void* out, int B,
                         int Cout, int H, int W, void* stream);
/* bias_add.cuh:96   NCHW, t = h(f(conv) + f(conv_bias[c])); out = h(f(t) + f(residual)) */
int dlm_conv_bias_residual(const void* conv, const void* conv_bias, const void* residual, void* out,
                           int B, int Cout, int H, int W, void* stream);
/* activation.cuh:33-41   x * sigmoid(x); 0.5 x (1 + erf(x / sqrt 2)); tanh approximation */
int dlm_silu(const void* in, void* out, int n, void* stream);
int dlm_gelu(const void* in, void* out, int n, void* stream);
int dlm_gelu_tanh(const void* in, void* out, int n, void* stream);
/* elementwise.cuh:26   out = h(f(a) + f(b)) */
int dlm_add(const void* a, const void* b, void* out, int n, void* stream);
/* elementwise.cuh:37   NCHW [N, C, H, W] -> [N, C, 2H, 2W], nearest */
int dlm_upsample_nearest2x(const void* in, void* out, int N, int C, int H, int W, void* stream);
/* geglu.cuh:42   [tokens, 2d] -> [tokens, d], out = h(x1 * gelu_erf(x2)), x1 the first half */
int dlm_geglu(const void* in, void* out, int tokens, int d, void* stream);
/* timeembed.cuh:44   out[i] = cos(t f_i), out[dim/2 + i] = sin(t f_i),
 * f_i = exp(-ln(max_period) i / (dim/2)) (diffusers flip_sin_to_cos = True) */
int dlm_timestep_embedding(void* out, float timestep, int dim, float max_period, void* stream);

/* ------------------------------------------------------------------ conv2d (implicit GEMM)
 *
 * Replaces launch_conv2d (reference src/kernels/conv2d.cuh:38-40, conv2d.cu:757) for the
 * shapes of the UNet / VAE hot path, on NHWC activations and without an im2col buffer
 * (conv2d.cu:219 im2col + gemm.cu:425 GEMM + conv2d.cu:171 bias pass become one kernel):
 *   out[N, oH, oW, Cout] = conv(in[N, H, W, Cin], w) + bias
 * Kernels: 3x3 pad 1 stride 1, 3x3 pad 1 stride 2 (Downsample2D, unet.cu:864-868), 1x1 stride 1
 * (conv_shortcut).  Cin % 64 == 0, Cout % 32 == 0, oW divides or is a multiple of 128 pixels.
 * w_krsc is [Cout, KH, KW, Cin] (see dlm_pack_conv_weight); bias may be NULL.
 * Stride 2 needs `scratch` of dlm_conv2d_nhwc_scratch_bytes() bytes (parity planes).
 */
size_t dlm_conv2d_nhwc_scratch_bytes(int N, int H, int W, int Cin, int ksize, int stride);
int dlm_conv2d_nhwc(const void* in, int N, int H, int W, int Cin, const void* w_krsc,
                    const void* bias, void* out, int Cout, int ksize, int stride, void* scratch,
                    size_t scratch_bytes, void* stream);

/* PyTorch conv weight [Cout, Cin, KH, KW] -> [Cout, KH, KW, Cin] (the GEMM K order). */
int dlm_pack_conv_weight(const void* w_oihw, void* w_krsc, int Cout, int Cin, int KH, int KW,
                         void* stream);

/* Layout conversions between the reference's NCHW tensors and this library's NHWC. */
int dlm_nchw_to_nhwc(const void* in, void* out, int N, int C, int HW, void* stream);
int dlm_nhwc_to_nchw(const void* in, void* out, int N, int C, int HW, void* stream);

/* ------------------------------------------------------------------ attention (tcgen05 flash)
 *
 * Replaces launch_attention / launch_attention_fast (reference src/kernels/attention.cuh:53-73):
 * out = softmax(q k^T * scale) v, q/k/v/out [B, H, S, Dh] contiguous fp16, fp32 online softmax.
 * Dh = 64 (the UNet's head_dim, src/infer/unet.cu:683-684: two 128-query tiles per CTA, stream-K
 * with a workspace) or a multiple of 64 in [128, 512] (wide heads, e.g. the VAE mid-block's
 * Dh = 512 that the reference passes to launch_attention, src/kernels/vae_decode.cu:682-683:
 * one CTA per 128-query tile and 256-column output slice; the _ws workspace is not used).
 */
int dlm_launch_attention(const void* q, const void* k, const void* v, void* out, int B, int H,
                         int Sq, int Sk, int Dh, float scale, void* stream);

/* The same attention load-balanced over all SMs ("stream-K"): the KV tiles of all (batch, head,
 * 256-query block) groups are split evenly over the SMs, pieces of a group split between SMs
 * are merged by the last one to finish (fixed order).  `workspace`: at least
 * dlm_attention_workspace_bytes(B, H, Sq) bytes, 256-byte aligned, ZEROED once before first use
 * (every call leaves it ready); calls sharing a workspace must not overlap on the GPU. */
size_t dlm_attention_workspace_bytes(int B, int H, int Sq);
int dlm_launch_attention_ws(const void* q, const void* k, const void* v, void* out, int B, int H,
                            int Sq, int Sk, int Dh, float scale, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Same op on token-major projections: q is [B*Sq, ldq] with head h in columns [h*64, h*64+64),
 * k / v are [B*Sk, ldk / ldv], out is [B*Sq, ldo].  Removes the reference's split/merge-heads
 * copies (src/infer/unet.cu:198,213). */
int dlm_attention_tokens(const void* q, int ldq, const void* k, int ldk, const void* v, int ldv,
                         void* out, int ldo, int B, int H, int Sq, int Sk, int Dh, float scale,
                         void* stream);

/* ------------------------------------------------------------------ normalisation
 *
 * GroupNorm(32) over NHWC activations, optionally of the channel concatenation of two sources
 * (x2 may be NULL with C2 = 0), optionally followed by SiLU; out is [N, HW, C1 + C2].
 * Replaces launch_group_norm / launch_group_norm_mb / launch_group_norm_silu (reference
 * src/kernels/groupnorm.cuh:51-108) and the up-path concat (src/infer/unet.cu:250).
 * Deterministic (fixed-order reductions).  `scratch` holds the per-chunk partial sums, the
 * per-image statistics and arrival counters: dlm_group_norm_nhwc_scratch_bytes(N, HW) bytes of any
 * content (the call zeroes the counters on `stream` before its two kernels).
 */
size_t dlm_group_norm_nhwc_scratch_bytes(int N, int HW);
int dlm_group_norm_nhwc(const void* x1, int C1, const void* x2, int C2, int N, int HW,
                        const void* gamma, const void* beta, float eps, int groups, int silu,
                        void* out, void* scratch, size_t scratch_bytes, void* stream);

/* The same GroupNorm for callers that cannot allocate device memory (no counterpart in the
 * reference): a host whose device memory is entirely owned by its own pre-reserved arena, or a
 * loop that must not pay cudaMalloc's implicit synchronisation, cannot hand dlm_group_norm_nhwc a
 * scratch buffer.  This entry point keeps the partial sums in a static device array of the
 * library (dlm_group_norm_nhwc_noalloc_capacity() float2 entries, 256 KiB, one copy per GPU that
 * loads the library, held until exit) and allocates nothing.  Problems needing more partial sums
 * are rejected with DLM_ERR_INVALID: the count grows with the batch and the SM count, so on a
 * 148-SM B200 any image size fits for N <= 339.  Each call zeroes its own arrival counters on its
 * stream (a memset, no allocation), so calls with different N may follow one another.  All calls
 * share the array: calls that overlap on the GPU race and must be serialised.  The first call on a device looks up the array's device address
 * (with that device current) and should come before any stream capture. */
size_t dlm_group_norm_nhwc_noalloc_capacity(void);
int dlm_group_norm_nhwc_noalloc(const void* x1, int C1, const void* x2, int C2, int N, int HW,
                                const void* gamma, const void* beta, float eps, int groups,
                                int silu, void* out, void* stream);

/* GroupNorm over NCHW fp16 [N, C, H, W] (reference src/kernels/groupnorm.cuh:51-108:
 * launch_group_norm, launch_group_norm_mb and, with silu = 1, launch_group_norm_silu, whose SiLU
 * follows an fp16 rounding of the normalised value).  in == out allowed.  Scratch: any content,
 * dlm_group_norm_nchw_scratch_bytes(N, groups) bytes (the call zeroes its counters on `stream`).
 * Statistics in fp32 slices around a shift, folded in fixed order in fp64: deterministic. */
size_t dlm_group_norm_nchw_scratch_bytes(int N, int groups);
int dlm_group_norm_nchw(const void* in, const void* gamma, const void* beta, void* out, int N,
                        int C, int H, int W, int groups, float eps, int silu, void* scratch,
                        size_t scratch_bytes, void* stream);

/* Direct NCHW convolution, one thread per output value, fp32 accumulation with the bias folded in
 * and one rounding at the store (reference src/kernels/conv2d.cuh:65-69 launch_conv2d_direct;
 * with in_f32 = out_f32 = 1 it serves launch_conv2d_f32_gemm, :79-82).  Any kernel size, stride,
 * padding and dilation; weight [Cout, Cin, KH, KW] fp16; bias fp16 [Cout] or NULL; Hout / Wout
 * must match the geometry. */
int dlm_conv2d_direct_nchw(const void* in, int in_f32, const void* weight, const void* bias,
                           void* out, int out_f32, int N, int Cin, int H, int W, int Cout, int KH,
                           int KW, int Hout, int Wout, int stride_h, int stride_w, int pad_h,
                           int pad_w, int dil_h, int dil_w, void* stream);

/* 1 when a convolution of this shape runs on the implicit-GEMM tensor-core path (3x3 s1 / s2
 * pad 1 or 1x1, Cin % 64 == 0, Cout % 32 == 0, 128-pixel output tiles), 0 otherwise (reference
 * src/kernels/conv2d.cuh:54-56 conv2d_uses_gemm_bias_path: that path rounds the bias-free
 * convolution once, so the bias may be added in a later pass). */
int dlm_conv2d_uses_gemm_bias_path(int N, int Cin, int H, int W, int Cout, int KH, int KW,
                                   int stride_h, int stride_w, int pad_h, int pad_w, int dil_h,
                                   int dil_w);

/* LayerNorm over the last dim of [rows, C] (reference src/kernels/layernorm.cuh:51-57);
 * gamma / beta may be NULL.  C % 8 == 0, C <= 2048. */
int dlm_launch_layer_norm(const void* in, const void* gamma, const void* beta, void* out, int rows,
                          int C, float eps, void* stream);

/* ------------------------------------------------------------------ BitNet ternary x int8 linear
 *
 * Bit-exact with the reference's integer BitLinear (src/models/bitnet.hpp:447-471, a host loop
 * there; no GPU kernel exists in the reference, README_en.md:143):
 *   y[m, n] = float( double(sum_k wq[n,k] * xq[m,k]) * double(alpha_n) * double(scale_m) )
 * with alpha_n = mean|w[n,:]| and wq = clamp(round(w/alpha), -1, 1) per output row
 * (quantize_weight_ternary, bitnet.hpp:70-109) and scale_m = max|x[m,:]|/127,
 * xq = clamp(round(x/scale), -127, 127) per token (quantize_activation_int8, bitnet.hpp:123-165).
 * Packed weights: [N, K/16] uint32, 16 two-bit codes per word (00 = 0, 01 = +1, 11 = -1,
 * code j at bits 2j); K % 64 == 0; packed weights and activations 16-byte aligned.
 * M >= 1024 runs on the tensor cores in 128 x 128 tiles; smaller M on the tensor cores in
 * 128 x 32 (or 64) tiles when K % 128 == 0, K <= 2048 and N % 32 == 0; other shapes on dp4a.
 * Every path gives the same bits.
 */
int dlm_ternary_pack(const float* w, int N, int K, void* w_packed2b, float* row_scale, void* stream);
int dlm_quantize_act_i8(const float* x, int M, int K, int8_t* xq, float* x_scale, void* stream);
int dlm_ternary_gemm_i8(const void* w_packed2b, const float* row_scale, const int8_t* x,
                        const float* x_scale, float* y, int M, int N, int K, void* stream);
/* quantize_act_i8 + ternary_gemm_i8: BitNet::bitlinear for M tokens (scratch: M*K bytes, M floats). */
int dlm_bitlinear(const void* w_packed2b, const float* row_scale, const float* x, float* y, int M,
                  int N, int K, int8_t* xq_scratch, float* xscale_scratch, void* stream);

/* ---------------------------------------------------------------- BitNet tag LM (model level)
 *
 * The ternary LM around BitLinear: BitNet::forward (reference src/models/bitnet.hpp:376-440) with
 * the greedy decode rule of src/infer/bitnet.hpp:282-318 (argmax of the last position, ties to the
 * smallest id, stop before <eos> = 2 or at max_len tokens), batched over sequences with a K/V
 * cache.  Dimensions are parameters (the reference compiles them in, src/models/bitnet_config.hpp);
 * head_dim is 64.  The reference's double-precision context arithmetic is reproduced operation by
 * operation; BitLinear is exact. */
typedef struct dlm_bitnet_config {
  int vocab, d_model, n_layers, n_heads, ffn_dim, max_seq;
  double rope_base, rms_eps;
  int per_tensor_scale; /* 0: one ternary scale per output row (the reference); 1: per tensor */
} dlm_bitnet_config;

/* fp32 state dict (host or device pointers): "embed" [vocab, d], "final_norm" [d],
 * "layers.N.{attn_norm, wq, wk, wv, wo, ffn_norm, w_gate, w_up, w_down}" (the reference loader's
 * names, src/infer/bitnet.hpp:116-135).  BitLinear weights are quantized and 2-bit packed here. */
int dlm_bitnet_create(const dlm_bitnet_config* cfg, int n, const char* const* names,
                      const float* const* weights, const int64_t* numels, void** handle, void* stream);
int dlm_bitnet_destroy(void* handle);

/* logits [B, S, vocab] of every position of tokens [B, S] (BitNet::forward per sequence; host or
 * device pointers).  DLM_ERR_INVALID for ids outside [0, vocab) or S > max_seq. */
int dlm_bitnet_forward(void* handle, const int* tokens, int B, int S, float* logits, void* stream);

/* Greedy decode of prompts [B, P] (host or device) to at most max_len tokens per sequence
 * (max_len <= max_seq): out [B, max_len - P] the generated ids (without <eos>), out_len [B] their
 * counts.  One prefill over all prompt positions, then one decode pass per token (CUDA graph).
 * Returns when the results are in out / out_len. */
int dlm_bitnet_generate(void* handle, const int* prompts, int B, int P, int max_len, int* out,
                        int* out_len, void* stream);

/* The weight set dlm_bitnet_create expects for cfg: count, then per index its name and shape. */
int dlm_bitnet_weight_count(const dlm_bitnet_config* cfg);
int dlm_bitnet_weight_info(const dlm_bitnet_config* cfg, int index, char* name, int name_cap,
                           int64_t* shape, int* ndim);

/* ------------------------------------------------------------------ SDXL UNet (model level)
 *
 * Replaces unet_weights_create / launch_unet_batched / unet_weights_destroy (reference
 * src/infer/unet.cuh:90-146, unet.cu:1336,1475).  The handle owns a prepared copy of every
 * weight (repacked for the kernels), so the caller's tensors may be freed after create.
 *   names / dev_ptrs / numels: n fp16 device tensors keyed by the diffusers state-dict names
 *     the reference reads (unet.cu `w.get("...")`); numels may be NULL (no size check);
 *   depths: transformer layers per Transformer2D at the 1x / 1/2x / 1/4x levels ({0, 2, 10} for
 *     SDXL; NULL = SDXL) and mid_depth (10 for SDXL) — reduced depths serve tests.
 * Returns DLM_ERR_NOT_FOUND (naming the tensor in dlm_last_error) when a weight is missing.
 */
int dlm_unet_create(const int* depths, int mid_depth, int n, const char* const* names,
                    const void* const* dev_ptrs, const int64_t* numels, void** handle, void* stream);
int dlm_unet_destroy(void* handle);

/* One UNet step for a batch of B latents (CFG cond/uncond stacked as B = 2, unet.cuh:137-146):
 *   latent [B, 4, H, W], ehs [B, 77, 2048], text_embeds [B, 1280], time_ids [6] (shared),
 *   noise_out [B, 4, H, W]; all fp16 device tensors, NCHW as the reference.
 * H and W are the latent size (128 for 1024^2 images); H/4 and W/4 must tile by 128 pixels.
 * The first call for a (B, H, W) plans the step (static activation arena, all launch
 * parameters) and captures it as a CUDA graph; later calls replay it with no allocation. */
int dlm_unet_forward(void* handle, int B, int H, int W, const void* latent, float timestep,
                     const void* ehs, const void* text_embeds, const void* time_ids, void* noise_out,
                     void* stream);

/* The same step called with HOST buffers, as the reference's diffusion loop drives it
 * (src/infer/diffusion.cu:896-986: H2D of the latent before the UNet, D2H of the noise
 * prediction after): copies the inputs in, runs the step, copies noise_out back and returns
 * once it is on the host (synchronizes `stream`).  Pinned host memory gives full copy speed. */
int dlm_unet_forward_host(void* handle, int B, int H, int W, const void* latent_host, float timestep,
                          const void* ehs_host, const void* text_embeds_host,
                          const void* time_ids_host, void* noise_out_host, void* stream);

/* Measurement helper: runs the planned step once eagerly with a CUDA event between launches and
 * returns per op class (0 GEMM/conv, 1 attention, 2 GroupNorm, 3 LayerNorm, 4 other) the
 * device milliseconds, the algorithmic FLOPs and the launch count (arrays of 5).  Requires a
 * previous dlm_unet_forward for the same shape. */
int dlm_unet_time_ops(void* handle, double* ms, double* flops, int* count, void* stream);

/* The weight set dlm_unet_create expects for the given depths (NULL = SDXL): count, then per
 * index its state-dict name and shape (ndim <= 4; shape padded with 0). */
int dlm_unet_weight_count(const int* depths, int mid_depth);
int dlm_unet_weight_info(const int* depths, int mid_depth, int index, char* name, int name_cap,
                         int64_t* shape, int* ndim);

/* Enables (default) or disables CUDA-graph replay of the step. */
int dlm_unet_set_graph(void* handle, int enable);

/* Runtime LoRA (reference unet_apply_loras / unet_clear_loras, src/infer/unet.cuh:96-111,
 * unet.cu:373-458; LoraModule, src/infer/lora.hpp:136-145).  One module merges
 * W += h(scale * (B @ A)) into the resident weight named by its diffusers key (fp32
 * accumulation over the rank, one fp16 rounding of the delta, one of the sum; the handle keeps
 * its weights repacked, q|k|v-concatenated and LayerNorm-folded, and the delta is mapped into
 * that layout).  The forward path and its captured graph are unchanged: only weight bytes move.
 *   a_fp16 [rank, in_flat], b_fp16 [out_dim, rank]: HOST fp16 bits (as LoraModule holds them);
 *   in_flat = the product of the weight's dims after the first (conv: Cin * 3 * 3).
 * Keys must name a 2-D / 4-D weight of this UNet with matching [out_dim, in_flat], else
 * DLM_ERR_NOT_FOUND / DLM_ERR_INVALID (the reference throws).  Modules apply in order and
 * stack.  dlm_unet_clear_loras returns every patched weight to its bytes before the first
 * apply (bit-exact; the reference re-uploads the base bytes) and frees the saved copies.
 * dlm_unet_apply_lora is the same merge for one module whose A / B are DEVICE fp16 tensors. */
typedef struct dlm_lora_module {
  const char* base_key;
  const uint16_t* a_fp16;
  const uint16_t* b_fp16;
  int rank;
  int in_flat;
  int out_dim;
  float scale;
} dlm_lora_module;
int dlm_unet_apply_loras(void* handle, const dlm_lora_module* mods, int n, void* stream);
int dlm_unet_apply_lora(void* handle, const char* base_key, const void* A, const void* B, int rank,
                        int in_flat, int out_dim, float scale, void* stream);
int dlm_unet_clear_loras(void* handle, void* stream);

/* Test hook (the reference's unet_set_stage_hook, unet.cuh:53-54): device pointer and NHWC
 * geometry of a stage output of the last forward ("temb_final", "conv_in_out",
 * "down_block_{0,1,2}_out", "mid_block_out", "up_block_{0,1,2}_out"). */
int dlm_unet_stage(void* handle, const char* name, const void** ptr, int* C, int* H, int* W);

/* Activation arena bytes, prepared weight bytes, kernel launches per step. */
int dlm_unet_info(void* handle, int64_t* arena_bytes, int64_t* weight_bytes, int* num_launches);

/* ---------------------------------------------------------------- SDXL denoising loop
 *
 * The txt2img loop of the reference's DiffusionPipeline::generate_txt2img
 * (src/infer/diffusion.cu:896-988) on the device, without its per-step host round trip: Euler
 * (epsilon prediction) over the SDXL schedule of src/infer/scheduler.hpp (scaled_linear betas
 * 0.00085..0.012, 1000 training steps, "leading" spacing, steps_offset 1), classifier-free
 * guidance e = e_uncond + g * (e_cond - e_uncond), the UNet run at batch 2 (cond, uncond).
 * init_latent [1, 4, H, W] fp32 is the starting latent (randn * sigmas[0], as the reference
 * draws it); ehs [2, 77, 2048], text_embeds [2, 1280] (cond first), time_ids [6] fp16; device
 * pointers.  Enqueued on `stream`. */
int dlm_sdxl_schedule(int steps, float* sigmas /* [steps + 1] */, float* timesteps /* [steps] */);
int dlm_sdxl_denoise(void* unet, int H, int W, const float* init_latent, int steps, float guidance,
                     const void* ehs, const void* text_embeds, const void* time_ids,
                     float* latent_out, void* stream);
/* The same loop followed by the VAE decode of fp16(latent / vae_scaling) (diffusion.cu:979-988):
 * image [1, 3, 8H, 8W] fp16. */
int dlm_sdxl_generate(void* unet, void* vae, int H, int W, const float* init_latent, int steps,
                      float guidance, const void* ehs, const void* text_embeds, const void* time_ids,
                      float vae_scaling, void* image, void* stream);

/* ---------------------------------------------------------------- SDXL VAE decoder
 * Resident-weight handle of the AutoencoderKL decoder.  Replaces vae_weights_create /
 * vae_weights_destroy / launch_vae_decode(handle, d_latent, d_image_out)
 * (src/kernels/vae_decode.cuh:66-75): the caller passes the state dict as (name, device pointer,
 * element count) triples of fp16 tensors (decoder.* and post_quant_conv.*; the 140 names of
 * dlm_vae_weight_info); the handle copies and repacks them, so the caller's buffers may be freed
 * after create returns.  DLM_ERR_NOT_FOUND names a missing tensor in dlm_last_error. */
int dlm_vae_create(int n, const char* const* names, const void* const* dev_ptrs,
                   const int64_t* numels, void** handle, void* stream);
int dlm_vae_destroy(void* handle);

/* latent [B, 4, h, w] fp16 NCHW (already divided by the VAE scaling factor, as the reference's
 * caller does at src/infer/diffusion.cu:979-986) -> image [B, 3, 8h, 8w] fp16 NCHW, both device
 * pointers.  w must be a multiple of 128 or divide 128 (then 128 / w must divide h), and
 * h * w <= 32768.  The first call for a (B, h, w) plans the decode (static arena) and captures it
 * as a CUDA graph; later calls replay it. */
int dlm_vae_decode(void* handle, int B, int h, int w, const void* latent, void* image, void* stream);

/* Same decode with HOST latent / image: copies in, decodes, copies the image back and returns once
 * it is on the host (synchronizes `stream`). */
int dlm_vae_decode_host(void* handle, int B, int h, int w, const void* latent_host, void* image_host,
                        void* stream);

/* Enables (default) or disables CUDA-graph replay of the decode. */
int dlm_vae_set_graph(void* handle, int enable);

/* Test hook (the reference's dbg_stat points, vae_decode.cu:736-866): device pointer, dtype
 * (0 fp16, 1 fp32) and NHWC geometry of a stage output of the last decode ("mid_block_out",
 * "up_block_{0,1,2,3}_out"). */
int dlm_vae_stage(void* handle, const char* name, const void** ptr, int* dtype, int* C, int* H,
                  int* W);

/* Activation arena bytes, prepared weight bytes, kernel launches per decode. */
int dlm_vae_info(void* handle, int64_t* arena_bytes, int64_t* weight_bytes, int* num_launches);

/* Per op class device ms / algorithmic FLOPs / launches of one eager decode (as dlm_unet_time_ops). */
int dlm_vae_time_ops(void* handle, double* ms, double* flops, int* count, void* stream);

/* The weight set dlm_vae_create expects: count, then per index its name and shape (ndim <= 4). */
int dlm_vae_weight_count(void);
int dlm_vae_weight_info(int index, char* name, int name_cap, int64_t* shape, int* ndim);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* DOLLAMA_B200_H_ */
