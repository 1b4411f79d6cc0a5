/*
 * qwen_image_b200.h -- C ABI of the B200-native Qwen-Image MMDiT denoising path.
 *
 * Plain pointers and sizes only.  Every entry point returns an int status
 * (QI_OK == 0) instead of exiting; qi_status_string() names it.  Device
 * pointers are CUDA device addresses on the context's device; `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  All calls are
 * asynchronous on `stream` unless stated otherwise.
 *
 * Reference interfaces each entry replaces are cited as file:line of the
 * reference project (TheLegendOfKitty/qwen-image.cu).
 */
#ifndef QWEN_IMAGE_B200_H
#define QWEN_IMAGE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
enum {
  QI_OK = 0,
  QI_ERR_ARG = 1,         /* bad size / null pointer / unsupported shape        */
  QI_ERR_ALIGN = 2,       /* pointer or leading dimension not 16-byte aligned    */
  QI_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed                   */
  QI_ERR_OOM = 4,         /* device allocation failed                            */
  QI_ERR_UNSUPPORTED = 5, /* shape outside what the kernels implement            */
  QI_ERR_IO = 6,          /* file missing or malformed (safetensors)             */
  QI_ERR_DEVICE = 7,      /* a kernel reported a bounded-wait timeout            */
  QI_ERR_NCCL = 8         /* a collective failed or timed out                    */
};

const char* qi_status_string(int status);
int qi_version(void);

/* ------------------------------------------------------------ op level
 * Each op mirrors one reference function; the tests call these through the
 * ABI and compare with the reference's own build on the same inputs.        */

/* Load-time weight quantizer: BF16 [N,K] -> block-FWHT rows (block K & -K)
 * -> per-row INT8 codes [N,K] + FP32 scales [N].
 * Replaces quantize_weight_tensor (cuda_kernels.cuh:308, cuda_kernels.cu:2830)
 * and produces quantize.cu's "<name>" / "<name>.__scales__" pair
 * (quantize.cu:121-137).  Codes and scales are bit-exact with the reference. */
int qi_quantize_weight(const void* w_bf16, int N, int K, int8_t* codes, float* scales, void* stream);

/* Activation quantizer: FP32 [M,K] -> block-FWHT (block `had_block`) ->
 * per-token INT8 codes + FP32 scales.  had_block <= 1 skips the transform.
 * Replaces quantize_activation_int8_hadamard_fp32 (cuda_kernels.cuh:277,
 * cuda_kernels.cu:2603).  Bit-exact with the reference.                      */
int qi_fwht_quantize(const float* x, int M, int K, int had_block, int8_t* codes, float* scales, void* stream);

/* W8A8 linear on prequantized activations:
 *   out[m,n] = acc[m,n] * act_scales[m] * w_scales[n] + bias[n]   (epilogue 0)
 *   out[m,n] = gelu_tanh(...)                                     (epilogue 1)
 *   out[m,n] += gate[n] * (...)                                   (epilogue 2)
 * acc = sum_k act[m,k] * w[n,k] in INT32 (exact).  bias is BF16 [N] or NULL.
 * Requires K % 16 == 0, N % 32 == 0, ldo % 4 == 0, 16-byte aligned pointers.
 * Replaces linear_forward_int8_prequantized (cuda_kernels.cuh:297,
 * cuda_kernels.cu:2735) and, for epilogue 2, the following gate_add_fp32f
 * (cuda_kernels.cuh:567).                                                    */
int qi_linear_i8(const int8_t* act, const float* act_scales, int M, int K, const int8_t* w, const float* w_scales,
                 int N, const void* bias_bf16, int epilogue, const float* gate, float* out, int ldo, void* stream);

/* Full W8A8 linear from FP32 activations (FWHT + quantize + GEMM + dequant),
 * M == 1 included.  Replaces linear_forward_int8 (cuda_kernels.cuh:290,
 * cuda_kernels.cu:2674) / linear_forward_quantized for INT8 weights
 * (cuda_kernels.cuh:420).                                                    */
int qi_linear_i8_f32in(const float* x, int M, int K, const int8_t* w, const float* w_scales, int N,
                       const void* bias_bf16, int apply_gelu, float* out, void* stream);

/* qi_linear_i8_f32in without any device allocation: same arguments, same
 * kernels, same results.  No counterpart in the reference.
 * For callers that must not allocate device memory once running (a server
 * whose memory pool owns all of HBM, so cudaMalloc would fail; a step loop
 * that cannot take cudaMalloc's implicit device synchronisation).  The
 * quantised activations live in a fixed scratch array compiled into the
 * library (about 4 MiB per device), so:
 *   - M <= QI_NOALLOC_MAX_ROWS, M * K <= QI_NOALLOC_MAX_CODES and
 *     K <= 12288, else the call returns QI_ERR_UNSUPPORTED; K % 16 != 0, or
 *     N % 32 != 0 when M > 1 or apply_gelu, is QI_ERR_ARG; w, w_scales (and
 *     out when M > 1 or apply_gelu) not 16-byte aligned is QI_ERR_ALIGN; none
 *     of these launches anything or touches the scratch;
 *   - the first call on a device does one-time setup (looks up the scratch
 *     address with that device current): make it before any stream capture;
 *   - the scratch is shared by all calls on a device: calls that can overlap
 *     (different streams or host threads without ordering between them)
 *     race and corrupt each other's results; serialise them.
 * A GEMM whose bounded wait gives up leaves `out` undefined and records the
 * fact in the scratch's error word, which stays set until
 * qi_linear_i8_f32in_noalloc_check reads it.                                */
#define QI_NOALLOC_MAX_ROWS 4096
#define QI_NOALLOC_MAX_CODES (4 * 1024 * 1024)
int qi_linear_i8_f32in_noalloc(const float* x, int M, int K, const int8_t* w, const float* w_scales, int N,
                               const void* bias_bf16, int apply_gelu, float* out, void* stream);
/* Error report of qi_linear_i8_f32in_noalloc on the current device: waits
 * for the device, then returns QI_ERR_DEVICE (and clears the word) if any
 * call since the last check gave up a bounded wait, else QI_OK.  Allocates
 * nothing.  No counterpart in the reference.                                */
int qi_linear_i8_f32in_noalloc_check(void);
/* Failure-path self test of that report: a kernel waits on an mbarrier
 * nothing arrives on and gives up after limit_us (<= 2 s), recording the
 * timeout in the scratch's error word the way the GEMM does; the next
 * qi_linear_i8_f32in_noalloc_check returns QI_ERR_DEVICE.  No counterpart in
 * the reference.                                                            */
int qi_linear_i8_f32in_noalloc_selftest(int limit_us, void* stream);

/* Number of CUDA allocations (device memory, and pinned host memory for the
 * checkpoint upload) this library has made since it was loaded, over all
 * devices.  Lets a caller verify that a call allocated nothing.             */
long long qi_alloc_count(void);

/* SageAttention on FP16 Q, K, V laid out [BH, S, 128] (head-major):
 * K mean smoothing, per-thread INT8 Q/K quantisation, INT8 QK^T, FP16 P.V,
 * online base-2 softmax; output FP32 [BH, S, 128] (each value an FP16
 * rounding, as the reference's FP16 output converted to FP32).
 * Replaces attention_forward_sage_sm80_fp16io (cuda_kernels.cuh:560,
 * sageattention_sm80.cu:965-1027).  head_dim must be 128.                    */
int qi_sage_attention(const void* q_f16, const void* k_f16, const void* v_f16, float* out, float scale, int BH,
                      int S, int D, void* stream);

/* The FP8 P.V variant of qi_sage_attention (same arguments and output
 * layout): Q and K INT8 with one scale per 128 queries / 64 keys (after K
 * mean smoothing), V as E4M3 codes with one scale per (batch-head, dim)
 * (max |V| / 448), P as E4M3 codes of 448 P with the running max updated at
 * every increase, P.V on tcgen05.mma.kind::f8f6f4.  The reference ships the
 * FP8 building blocks of this scheme (sageattention_mma.cuh:521-680,
 * sageattention_numeric_conversion.cuh:46-140,
 * sageattention_attn_utils.cuh:141-168) but launches only the FP16 P.V
 * kernel; this variant is checked against exact attention, not against the
 * reference.  head_dim must be 128.                                          */
int qi_sage_attention_fp8pv(const void* q_f16, const void* k_f16, const void* v_f16, float* out, float scale, int BH,
                            int S, int D, void* stream);

/* The Sage quantizers alone, for bit-exact checks against the reference:
 * k_mean [BH,128]; Q codes [BH,S,128] + scales [BH, ceil(S/128)*32];
 * K codes [BH,S,128] + scales [BH, ceil(S/64)*4]
 * (sageattention_sm80.cu:759-886).                                           */
int qi_sage_quantize(const void* q_f16, const void* k_f16, int BH, int S, float* k_mean, int8_t* q_codes,
                     float* q_scales, int8_t* k_codes, float* k_scales, void* stream);

/* LayerNorm (no affine, eps) + modulate: out = norm(x) * (1 + scale) + shift.
 * Replaces layer_norm_modulate_fp32 (cuda_kernels.cuh:524).                  */
int qi_layer_norm_modulate(const float* x, const float* shift, const float* scale, float* out, int rows, int dim,
                           float eps, void* stream);

/* Per-row RMSNorm, FP32 in/out, BF16 weight.  Replaces rms_norm_fp32
 * (cuda_kernels.cuh:510).                                                    */
int qi_rms_norm(const float* x, const void* w_bf16, float* out, int rows, int dim, float eps, void* stream);

/* LayerNorm + modulate fused with the activation quantizer, the kernel the
 * forward runs before the QKV and fc1 linears: FP32 [rows, 3072] -> INT8
 * codes [rows, 3072] + FP32 scales [rows] (block-FWHT 1024).  Replaces the
 * pair layer_norm_modulate_fp32 (cuda_kernels.cuh:524) +
 * quantize_activation_int8_hadamard_fp32 (cuda_kernels.cuh:277) of
 * transformer.cu:526-563.  dim must be 3072.                                 */
int qi_layer_norm_modulate_quantize(const float* x, const float* shift, const float* scale, int rows, int dim,
                                    float eps, int8_t* codes, float* scales, void* stream);

/* q/k RMSNorm + joint [txt; img] head-major layout + RoPE -> FP16, the
 * forward's qkv_post stage on caller buffers.  qkv_img [nb*n_img, 9216] and
 * qkv_txt [nb*n_txt, 9216] FP32 rows [q | k | v]; norms_bf16 [4][128] =
 * norm_q, norm_k, norm_added_q, norm_added_k; pe as for qi_forward; output
 * FP16 [3][nb*24][n_txt + n_img][128] (q, k, v).  Replaces rms_norm_fp32 x 4
 * + concat_transpose_fused_fp32 x 3 + rope_apply_fp32_to_fp16 x 2
 * (transformer.cu:618-671; cuda_kernels.cuh:510, 536).                       */
int qi_qk_norm_rope(const float* qkv_img, const float* qkv_txt, const void* norms_bf16, const float* pe, int nb,
                    int n_img, int n_txt, void* qkv_f16, void* stream);

/* The QKV projections of both streams with qi_qk_norm_rope's arithmetic in
 * the GEMM epilogue (the forward's fused form): act_img [nb*n_img, 3072] and
 * act_txt [nb*n_txt, 3072] INT8 codes with per-row scales (as
 * qi_layer_norm_modulate_quantize gives them), w_img / w_txt [9216, 3072]
 * INT8 [q | k | v] rows with per-row scales and BF16 biases (or NULL);
 * norms_bf16, pe and the output as for qi_qk_norm_rope.  Bit-identical to
 * qi_linear_i8 (epilogue 0) of each stream followed by qi_qk_norm_rope, with
 * no FP32 projection in memory.  Needs at least 512 rows in all
 * (QI_ERR_UNSUPPORTED below).  Replaces linear_forward_int8_prequantized x 6
 * and the qkv_post chain of transformer.cu:568-671.                         */
int qi_qkv_norm_rope_i8(const int8_t* act_img, const float* act_img_scales, const int8_t* act_txt,
                        const float* act_txt_scales, const int8_t* w_img, const float* w_img_scales, const void* b_img,
                        const int8_t* w_txt, const float* w_txt_scales, const void* b_txt, const void* norms_bf16,
                        const float* pe, int nb, int n_img, int n_txt, void* qkv_f16, void* stream);

/* ------------------------------------------------------------ model level */
typedef struct qi_ctx qi_ctx;
typedef struct qi_model qi_model;

/* Device context: device ordinal, scratch workspace (grows on demand, like
 * the reference's static workspace, transformer.cu:134-215), error slot.    */
int qi_ctx_create(int device, qi_ctx** out);
int qi_ctx_destroy(qi_ctx* ctx);
/* Reads (and clears) the device error word a kernel raised; QI_ERR_DEVICE if
 * any kernel gave up a bounded wait since the last call.  Synchronous.      */
int qi_ctx_check(qi_ctx* ctx);

/* Selects the FP8 P.V variant for the attention of qi_forward /
 * qi_forward_blocks on this context (enable != 0), or the FP16 P.V kernel the
 * reference launches (0, the default).  Off the reference's numerics: its
 * outputs are checked against exact attention, not against the reference.   */
int qi_ctx_set_attention_fp8pv(qi_ctx* ctx, int enable);

/* Where qi_forward / qi_forward_blocks apply the q/k RMSNorm, RoPE and FP16
 * head-major layout of each block (transformer.cu:637-666): in the epilogue
 * of the QKV projection, so the FP32 projection never reaches HBM
 * (enable != 0, the default), or as a separate kernel after an FP32
 * projection (0).  Both give the same bits; the fused form needs the CTA-pair
 * GEMM (at least 512 rows), and shorter inputs take the separate kernel.    */
int qi_ctx_set_fused_qkv_epilogue(qi_ctx* ctx, int enable);

/* Head-parallel (Ulysses) group.  New: the reference runs on one GPU
 * (its main.cu:761-773 calls transformer_forward for cond and uncond in
 * turn).  One process (or context) per GPU; rank 0 makes the id and the
 * caller hands it to the others (any channel); every rank then calls
 * qi_ctx_set_comm with its rank (a collective: it returns when all nranks
 * have joined).  nranks divides the 24 heads and is at most 8; nranks = 1
 * leaves the context single-GPU.  With a group set, qi_forward takes the same
 * full inputs on every rank, runs each linear on 1/nranks of the tokens and
 * attention on 24/nranks heads (two all-to-all exchanges per block), and
 * returns the full output on every rank.                                     */
#define QI_COMM_ID_BYTES 128
int qi_comm_unique_id(void* id_out);
int qi_ctx_set_comm(qi_ctx* ctx, const void* id, int rank, int nranks);
/* Failure detection of the group (new: the reference has no multi-GPU path;
 * its errors print and exit, tensor.h:15-37).  The communicator is
 * non-blocking: every collective step the library takes (joining the group,
 * the exchanges of a forward, the output gather) waits at most timeout_ms
 * (default 60000) for NCCL; on an asynchronous NCCL error or a missed
 * deadline the communicator is aborted, the call returns QI_ERR_NCCL, and
 * multi-GPU calls on the context keep returning QI_ERR_NCCL until
 * qi_ctx_set_comm forms a group again (nranks = 1 returns it to one GPU).
 * A rank that never joins makes qi_ctx_set_comm return QI_ERR_NCCL after
 * the deadline instead of blocking.                                          */
int qi_ctx_set_comm_timeout(qi_ctx* ctx, int timeout_ms);
/* Waits, polling, until the work queued on `stream` has finished, at most
 * timeout_ms (<= 0: the context's collective deadline).  If the group's
 * communicator reports an error, or the deadline passes with a group set, the
 * communicator is aborted (its pending collectives end) and QI_ERR_NCCL is
 * returned; a missed deadline without a group is QI_ERR_DEVICE.  Otherwise it
 * returns what qi_ctx_check returns.                                         */
int qi_ctx_sync(qi_ctx* ctx, void* stream, int timeout_ms);
/* The per-peer byte offsets and sizes a rank uses in the two all-to-all
 * exchanges of a head-parallel block (which = 0: Q/K/V before attention,
 * which = 1: attention output after it), for a joint sequence of n_txt text
 * and n_img image tokens per batch entry.  Host only; arrays of nranks. */
int qi_exchange_plan(int which, int nb, int n_txt, int n_img, int nranks, int rank, long long* send_off,
                     long long* send_bytes, long long* recv_off, long long* recv_bytes);

/* Weight table in quantize.cu's format, one device pointer per tensor,
 * indexed by the enums below.  INT8 linears: codes I8 [N,K], scales F32 [N],
 * bias BF16 [N].  Boundary linears (img_in, txt_in, norm_out, proj_out):
 * BF16 weight [N,K] + BF16 bias (quantize.cu:467-477).  Norm weights BF16.
 * Names: transformer.h:407-563.                                              */
enum {
  QI_G_T1_W, QI_G_T1_S, QI_G_T1_B, /* time_text_embed.timestep_embedder.linear_1 [3072,256] */
  QI_G_T2_W, QI_G_T2_S, QI_G_T2_B, /* ...linear_2 [3072,3072] */
  QI_G_TXT_NORM,                   /* txt_norm.weight [3584] */
  QI_G_IMG_IN_W, QI_G_IMG_IN_B,    /* img_in [3072,64] BF16 */
  QI_G_TXT_IN_W, QI_G_TXT_IN_B,    /* txt_in [3072,3584] BF16 */
  QI_G_NORM_OUT_W, QI_G_NORM_OUT_B, /* norm_out.linear [6144,3072] BF16 */
  QI_G_PROJ_OUT_W, QI_G_PROJ_OUT_B, /* proj_out [64,3072] BF16 */
  QI_G_COUNT
};
/* Per block: 14 INT8 linears x (codes, scales, bias) then 4 norm weights. */
enum {
  QI_L_IMG_MOD, QI_L_TXT_MOD, QI_L_TO_Q, QI_L_TO_K, QI_L_TO_V, QI_L_ADD_Q, QI_L_ADD_K, QI_L_ADD_V,
  QI_L_TO_OUT, QI_L_TO_ADD_OUT, QI_L_IMG_FC1, QI_L_IMG_FC2, QI_L_TXT_FC1, QI_L_TXT_FC2, QI_L_COUNT
};
enum {
  QI_B_NORM_Q = 3 * QI_L_COUNT, QI_B_NORM_K, QI_B_NORM_ADDED_Q, QI_B_NORM_ADDED_K, QI_B_COUNT
};

/* Builds the kernels' weight layout (fused QKV, stacked modulation) from a
 * device table.  Copies; the caller may free its tensors afterwards.
 * Replaces TransformerWeights::load's INT8 path (transformer.h:144-200,
 * 515-563).  block_tables[i] points to QI_B_COUNT device pointers.           */
int qi_model_create(qi_ctx* ctx, int num_blocks, const void* const* global_table,
                    const void* const* const* block_tables, qi_model** out);
/* Reads a quantize.cu INT8 safetensors file (or a sharded index .json).
 * Replaces SafeTensorsLoader + TransformerWeights::load (safetensors.h:36-212,
 * transformer.h:144).                                                        */
int qi_model_load_safetensors(qi_ctx* ctx, const char* path, qi_model** out);
int qi_model_destroy(qi_model* model);
int qi_model_num_blocks(const qi_model* model);

/* One MMDiT forward for `nb` independent batch elements that share the
 * latent shape and timestep (nb = 2: CFG cond/uncond in one pass).
 *   x:   nb x [16, H, W] BF16 latents (contiguous)
 *   ctx: nb x [n_txt, 3584] BF16 text states (contiguous)
 *   pe:  nb x [n_txt + n_img, 64, 2, 2] FP32 RoPE tables (contiguous; the
 *        table of rope.h gen_qwen_image_pe)
 *   out: nb x [16, H, W] BF16 velocities
 * Replaces transformer_forward (transformer.h:613-621, transformer.cu:234-931)
 * with use_sage_attention = true.  H and W must be even.                     */
int qi_forward(qi_ctx* ctx, const qi_model* model, int nb, const void* x_bf16, float timestep,
               const void* ctx_bf16, int n_txt, const float* pe, int H, int W, void* out_bf16, void* stream);

/* The block loop alone (transformer.cu:497-836, with the modulation of
 * `timestep`, :506-515) on caller-held FP32 residual streams, in place:
 * img [nb*n_img, 3072] and txt [nb*n_txt, 3072] (batch-major rows), blocks
 * [block_begin, block_end).  pe as for qi_forward.  Lets a caller run the
 * forward in pieces (per-block parity checks against the reference's block
 * dumps, multi-GPU schedules that own the residual streams).              */
int qi_forward_blocks(qi_ctx* ctx, const qi_model* model, int nb, int n_img, int n_txt, float* img, float* txt,
                      float timestep, const float* pe, int block_begin, int block_end, void* stream);

/* ---- Spectrum step skipping (the reference's --spectrum: main.cu:640-748,
 * 877-885; transformer.cu:864-871, 939-1028; cuda_kernels.cu:5859-6333).
 *
 * Every qi_forward on the context copies its final image hidden state (before
 * norm_out) to hidden_out, [nb][n_img][3072] FP32, 16-byte aligned, until
 * set to NULL: the reference's transformer_forward spectrum_hidden_out.
 * Single-GPU contexts only (QI_ERR_UNSUPPORTED with a head-parallel group). */
int qi_ctx_set_hidden_capture(qi_ctx* ctx, float* hidden_out);

/* The output head on a final image hidden state [nb][n_img][3072] FP32:
 * timestep MLP, norm_out modulation, AdaLayerNormContinuous, proj_out,
 * unpatchify -> nb x [16, H, W] BF16.  Replaces transformer_spectrum_output
 * (transformer.h:627-630, transformer.cu:939-1028); runs the same kernels as
 * the end of qi_forward, so a captured state gives that forward's output.  */
int qi_spectrum_output(qi_ctx* ctx, const qi_model* model, int nb, const float* hidden, float timestep, int H, int W,
                       void* out_bf16, void* stream);

/* Feature forecaster over the states of actual forwards (SpectrumState,
 * spectrum_init / update / predict / reset, cuda_kernels.cuh:588-645):
 * feature_elems floats per state (a multiple of 4), at most max_history
 * states kept (the oldest replaced; at most 128), Chebyshev order (bases
 * T_0..T_order, at most 16) and ridge lambda.                              */
typedef struct qi_spectrum qi_spectrum;
int qi_spectrum_create(long long feature_elems, int max_history, int order, float lambda, qi_spectrum** out);
int qi_spectrum_destroy(qi_spectrum* s);
/* Stores the state of an actual forward at `step` (steps must increase);
 * the copy is enqueued on `stream`.                                        */
int qi_spectrum_update(qi_spectrum* s, const float* feature, int step, void* stream);
/* Predicts the state at target_step into out (feature_elems floats, 16-byte
 * aligned): blend x Chebyshev ridge fit + (1 - blend) x first-order Taylor
 * extrapolation from the last two states.  Needs two stored states.       */
int qi_spectrum_predict(qi_spectrum* s, int target_step, float blend, float* out, void* stream);
/* Number of stored states (SpectrumState::buffer_size).                    */
int qi_spectrum_history(const qi_spectrum* s);
int qi_spectrum_reset(qi_spectrum* s);
/* The K prediction weights of qi_spectrum_predict (host only, double):
 * out = sum_k w[k] x state_k over stored steps[0..K) (increasing).          */
int qi_spectrum_weights(const int* steps, int K, int order, float lambda, int target_step, float blend, double* w);

/* RoPE table of rope.h gen_qwen_image_pe (h, w = latent size): host memory,
 * [n_txt + n_img, 64, 2, 2] FP32.                                            */
int qi_rope_table(int h, int w, int n_txt, float* pe_host);

/* Number of kernel launches issued by the last qi_forward on this context. */
int qi_ctx_last_launch_count(const qi_ctx* ctx);

/* Failure-path self test: launches a kernel that waits on an mbarrier nothing
 * arrives on, giving up after limit_us (<= 2 s), the way every wait in the
 * tensor-core kernels gives up instead of hanging.  The next qi_ctx_check
 * returns QI_ERR_DEVICE; the context stays usable.                          */
int qi_selftest_wait_timeout(qi_ctx* ctx, int limit_us, void* stream);

/* Per-stage timing of qi_forward with CUDA events (the reference's
 * PROFILE_BLOCK hook, transformer.cu:486-495 / 838-860).  While enabled each
 * forward records an event pair around every launch; qi_ctx_profile then
 * returns, per stage (QI_PROF_*), the number of launches and the summed
 * device milliseconds since the last reset.  Synchronous.                    */
enum {
  QI_PROF_PRE = 0,       /* patchify, timestep MLP, modulation, img_in, txt_in */
  QI_PROF_QUANT_LN,      /* LayerNorm + modulate + FWHT + INT8 (2 per block)    */
  QI_PROF_GEMM_QKV,      /* fused Q/K/V INT8 GEMM                               */
  QI_PROF_QKV_POST,      /* q/k RMSNorm + RoPE + FP16 head-major                */
  QI_PROF_SAGE_QUANT,    /* K mean + Q/K per-thread INT8                         */
  QI_PROF_ATTENTION,     /* SageAttention                                       */
  QI_PROF_QUANT_O,       /* attention output FWHT + INT8                        */
  QI_PROF_GEMM_OUT,      /* out-projection INT8 GEMM + gated residual           */
  QI_PROF_GEMM_FC1,      /* fc1 INT8 GEMM + GELU                                */
  QI_PROF_QUANT_H,       /* fc2 input FWHT(4096) + INT8                         */
  QI_PROF_GEMM_FC2,      /* fc2 INT8 GEMM + gated residual                      */
  QI_PROF_POST,          /* output AdaLN, proj_out, unpatchify                  */
  QI_PROF_EXCHANGE,      /* head-parallel all-to-all exchanges + reorders       */
  QI_PROF_COUNT
};
int qi_ctx_set_profiling(qi_ctx* ctx, int enable);
int qi_ctx_profile(qi_ctx* ctx, int* launches, float* ms, int reset);

/* One flow-matching Euler step with norm-preserving CFG on the device
 * (main.cu:228-288 cfg_combine_and_norms + cfg_norm_scale, :221
 * denoiser_scaling_fp32, :210 euler_step_fp32, then fp32_to_bf16 for the next
 * forward): v = uncond + s*(cond - uncond), rescaled per 2x2 patch group so its
 * norm matches cond's; x += (x - (x - sigma*v)) / sigma * (sigma_next - sigma).
 * latent: FP32 [16,H,W] updated in place; latent_bf16 receives its BF16 copy. */
int qi_cfg_euler_step(float* latent, const void* cond_bf16, const void* uncond_bf16, float cfg_scale, float sigma,
                      float sigma_next, int H, int W, void* latent_bf16, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_IMAGE_B200_H */
