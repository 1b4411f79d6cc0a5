// qi_internal.h -- launchers shared between the kernel files and the host
// orchestration.  Not part of the public ABI (include/qwen_image_b200.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "../../include/qwen_image_b200.h"

namespace qi {

constexpr int kDim = 3072;      // inner_dim (transformer.cu:244)
constexpr int kHeads = 24;      // n_heads
constexpr int kHeadDim = 128;   // head_dim
constexpr int kMlp = 12288;     // mlp_dim
constexpr int kTxtDim = 3584;   // text-encoder hidden size
constexpr int kPatchDim = 64;   // 16 channels x 2 x 2 patch
constexpr int kOutCh = 16;

// kEpiQkv: the q/k RMSNorm + RoPE + FP16 head-major store of qkv_post_kernel,
// applied to the QKV projection's accumulators (gemm_qkv_launch)
enum Epilogue { kEpiStore = 0, kEpiGelu = 1, kEpiResidual = 2, kEpiQkv = 3 };

// Raises a kernel's dynamic shared-memory limit on the current device, once
// per device: the attribute belongs to the device, so a process that drives
// several GPUs has to set it on each.  `done` is the caller's per-kernel
// bit mask of devices already set (devices 0..63).
inline int smem_optin(const void* fn, int bytes, unsigned long long* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return QI_ERR_CUDA;
  const unsigned long long bit = 1ull << dev;
  if (__atomic_load_n(done, __ATOMIC_ACQUIRE) & bit) return QI_OK;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return QI_ERR_CUDA;
  __atomic_fetch_or(done, bit, __ATOMIC_ACQ_REL);
  return QI_OK;
}

// Sequence split of the joint [txt; img] sequence over the P ranks of a
// head-parallel (Ulysses) group: rank r owns text tokens [txt_lo[r],
// txt_lo[r+1]) and image tokens [img_lo[r], img_lo[r+1]) of every batch entry.
// Its local sequence is its text tokens followed by its image tokens.
constexpr int kMaxRanks = 8;
struct ShardMap {
  int P;
  int txt_lo[kMaxRanks + 1];
  int img_lo[kMaxRanks + 1];
  __host__ __device__ int n_txt_l(int r) const { return txt_lo[r + 1] - txt_lo[r]; }
  __host__ __device__ int n_img_l(int r) const { return img_lo[r + 1] - img_lo[r]; }
  __host__ __device__ int len(int r) const { return n_txt_l(r) + n_img_l(r); }
};

// ---------------------------------------------------------------- GEMMs
// INT8: out = acc * sa[m] * sw[n] + bias[n] (+ epilogue).  a [M,K], w [N,K].
struct GemmDesc {
  const int8_t* a;
  const float* sa;
  const int8_t* w;
  const float* sw;
  const void* bias;  // BF16 [N] or null
  float* out;
  const float* gate;  // FP32 [N] for kEpiResidual
  int M, N, K, ldo;
};
int gemm_i8_launch(const GemmDesc* descs, int n, int epi, cudaStream_t stream, int* err_dev, int num_sms);

// BF16 x BF16 -> FP32 on the tensor cores: out = a[M,K] * w[N,K]^T + bias.
struct GemmBf16Desc {
  const void* a;  // BF16 [M,K]
  const void* w;  // BF16 [N,K]
  const void* bias;
  float* out;
  int M, N, K, ldo;
};
int gemm_bf16_launch(const GemmBf16Desc& d, cudaStream_t stream, int* err_dev, int num_sms);

// ---------------------------------------------------------------- quantizers
// Row sources for the fused activation quantizer.  Rows of all segments are
// written consecutively to codes/scales.
enum RowSrc { kSrcF32 = 0, kSrcF16 = 1, kSrcLnMod = 2 };
struct RowSeg {
  const void* in;      // FP32 or FP16 rows
  long long ld;        // elements between rows
  const float* shift;  // kSrcLnMod: modulation shift [K]
  const float* scale;  // kSrcLnMod: modulation scale [K] (used as 1 + scale)
  int rows;
};
int rowquant_launch(int src, int K, int had_block, const RowSeg* segs, int nseg, int8_t* codes, float* scales,
                    float eps, cudaStream_t stream);
// Generic shared-memory FWHT + per-row INT8 for any K <= 12288 and any
// power-of-two block; BF16 or FP32 input.  Used for weights (load time) and
// for activation shapes the fused kernels do not cover.
int fwht_quant_generic(const void* in, int in_bf16, int M, int K, int had_block, int8_t* codes, float* scales,
                       cudaStream_t stream);

// LayerNorm + modulate to BF16 or FP32 (final AdaLN, transformer.cu:881-884).
int layernorm_mod_launch(const float* x, const float* shift, const float* scale, int rows, int dim, float eps,
                         float* out_f32, void* out_bf16, cudaStream_t stream);
int rmsnorm_f32_launch(const float* x, const void* w, float* out, int rows, int dim, float eps,
                       cudaStream_t stream);
int rmsnorm_bf16_launch(const void* x, const void* w, void* out, int rows, int dim, float eps, cudaStream_t stream);

// ---------------------------------------------------------------- GEMV (M = 1)
// out[j][n] = dot(act, w_j[n]) * act_scale * sw_j[n] + bias_j[n] for a batch of
// linears that share one quantized activation row.
struct GemvJob {
  const int8_t* w;
  const float* sw;
  const void* bias;
  float* out;
  int N;
};
int gemv_i8_launch(const int8_t* act, const float* act_scale, int K, const GemvJob* jobs, int njobs,
                   cudaStream_t stream);
int gemv_bf16_launch(const float* x, const void* w, const void* bias, float* out, int N, int K, cudaStream_t stream);

// ---------------------------------------------------------------- elementwise
int timestep_embedding_launch(float t, float* out256, cudaStream_t stream);
int silu_launch(const float* x, float* out, int n, cudaStream_t stream);
// Patches [p_lo, p_lo + n_loc) of every batch entry -> [nb][n_loc][64].
int patchify_launch(const void* x_bf16, void* patches_bf16, int nb, int H, int W, int p_lo, int n_loc,
                    cudaStream_t stream);
// Ranks of a head-parallel group that write into each other's buffers (CUDA
// IPC mappings): each rank's Q/K/V buffer, token-major attention output and
// flag words [2 slots][kMaxRanks].
struct PeerSet {
  int P, rank;
  void* qkvh[kMaxRanks];
  void* o[kMaxRanks];
  unsigned* flags[kMaxRanks];
};
// Raises this rank's flag `slot` = epoch on every peer, then waits (bounded)
// until every peer has raised its flag here: all earlier work on `stream`
// of every rank is then visible to the later work of every rank.
int peer_barrier_launch(const PeerSet& ps, int slot, unsigned epoch, int* err, cudaStream_t stream);
// Ulysses reorders.  gather_qkv: received [src][3][nb][Hl][len(src)][128]
// FP16 -> [3][nb*Hl][S][128] in the joint order.  gather_o: received
// [src][nb][len(r)][Hl][128] (src's heads for this rank's positions) ->
// token-major rows [nb * n_img_l image rows; nb * n_txt_l text rows][24*128].
int ulysses_gather_qkv_launch(const void* recv, void* qkvh, int nb, int Hl, int n_txt, const ShardMap& map,
                              cudaStream_t stream);
int ulysses_gather_o_launch(const void* recv, void* out, int nb, int Hl, int rank, const ShardMap& map,
                            cudaStream_t stream);
int unpatchify_launch(const float* proj, void* out_bf16, int nb, int H, int W, cudaStream_t stream);

// q/k RMSNorm + RoPE + FP16 + head-major joint layout.  qkv rows hold
// [q | k | v] (3 x 3072).  Rows [0, nb*n_img) are image tokens, rows
// [nb*n_img, nb*(n_img+n_txt)) text tokens.  Outputs [nb, 24, S, 128] FP16.
// q/k RMSNorm + RoPE + FP16 for this rank's rows.  Output layout, by
// destination rank d (heads [d*Hl, (d+1)*Hl)):
//   qkvh[d][which = q,k,v][b][head - d*Hl][local position][128]
// with local position = text rows first, then image rows.  For a single rank
// (P = 1, Hl = 24) this is [3][nb*24][S][128] in the joint order.
struct QkvPostArgs {
  const float* qkv_img;  // [nb * n_img_l, 9216]
  const float* qkv_txt;  // [nb * n_txt_l, 9216]
  const void* nq_img;  // BF16 [128] norm_q
  const void* nk_img;
  const void* nq_txt;  // norm_added_q
  const void* nk_txt;
  const float* pe;     // nb x [S, 64, 2, 2] (full sequence)
  void* qkvh;
  int nb, n_img, n_txt;        // full sizes
  int img_lo, n_img_l;         // this rank's image range
  int txt_lo, n_txt_l;         // this rank's text range
  int Hl;                      // heads per destination rank
  // direct != 0: store straight into each head owner's Q/K/V buffer (peer
  // memory over NVLink), final layout [3][nb*Hl][S][128] in joint order
  int direct;
  void* peer_qkvh[kMaxRanks];
  int norm_dim;  // set by qkv_post_launch
  float eps;
};
int qkv_post_launch(const QkvPostArgs& a, cudaStream_t stream);
// The QKV projection (descs: the image and text problems, N = 3 x 3072) with
// qkv_post's arithmetic in its epilogue: the FP32 projection never reaches
// HBM (a.qkv_img / a.qkv_txt are unused).  Outputs are bit-identical to
// gemm_i8_launch(kEpiStore) followed by qkv_post_launch.  Needs the CTA-pair
// kernel at 256-column tiles (one head per epilogue warp): gemm_qkv_fusable
// says whether the shapes get it; otherwise use the two launches.
bool gemm_qkv_fusable(const GemmDesc* descs, int n, int num_sms);
int gemm_qkv_launch(const GemmDesc* descs, int n, const QkvPostArgs& a, cudaStream_t stream, int* err_dev,
                    int num_sms);

// ---------------------------------------------------------------- attention
// Longest joint sequence the attention kernel takes (its K scales of up to
// 8192 64-key blocks fit in shared memory).
constexpr int kAttnMaxS = 131072;
// A second stream for work that may overlap the main stream's: `fork` is
// recorded on the main stream before the side work, `join` on the side stream
// after it; the main stream waits for `join` before it needs the results.
struct SideStream {
  cudaStream_t s;
  cudaEvent_t fork, join;
};
// side != nullptr: the K mean (a latency-bound chain over the tokens on a few
// CTAs) runs on the side stream beside the Q quantizer.
int sage_quantize_launch(const void* q, const void* k, int BH, int S, float* kmean, int8_t* qc, float* qs,
                         int8_t* kc, float* ks, cudaStream_t stream, const SideStream* side = nullptr);
// out_mode 0: FP32 [BH, S, 128] head-major.
// out_mode 1: FP16 token-major rows for the out-projection: joint position p
//   of batch b goes to row (p < n_txt ? nb*n_img + b*n_txt + p
//                                     : b*n_img + p - n_txt), 3072 columns.
struct AttnArgs {
  const int8_t* qc;
  const float* qs;
  const int8_t* kc;
  const float* ks;
  const void* v;  // FP16 [BH, S, 128]
  void* out;
  int BH, S, heads;  // heads per batch entry in the BH layout
  float sm_scale;
  // 0: FP32 [BH, S, 128]; 1: FP16 token-major rows (image rows of every batch
  // entry, then text rows) x [heads * 128]; 2: FP16 by destination rank of
  // the query position, [dest][nb][len(dest)][heads][128] (Ulysses return)
  int out_mode;
  int nb, n_img, n_txt;
  ShardMap map;  // out_mode 2, 3
  // out_mode 3: FP16 straight into the token owner's token-major rows (peer
  // memory), columns (head_base + head) * 128
  void* peer_o[kMaxRanks];
  int head_base;
  // FP8 P.V variant: v is then the E4M3 V^T codes [BH][128][s_pad] (token
  // stride s_pad, a multiple of 16) and vs the per (batch-head, dim) output
  // factors v_scale / 448
  int fp8;
  const float* vs;
  int s_pad;
};
int attention_launch(const AttnArgs& a, cudaStream_t stream, int* err_dev);
// Per-block Q / K INT8 (one scale per 128 queries / 64 keys, after K mean
// smoothing), written in the per-thread scale layout the attention kernel
// reads (every entry of a block the same), and V as E4M3 codes of
// V / v_scale transposed to [BH][128][s_pad] with v_scale = max |V| / 448 per
// (batch-head, dim); vs receives v_scale / 448.  vamax is [BH][128] scratch.
int sage_quantize_fp8pv_launch(const void* q, const void* k, const void* v, int BH, int S, float* kmean, int8_t* qc,
                               float* qs, int8_t* kc, float* ks, uint8_t* vt, int s_pad, float* vamax, float* vs,
                               cudaStream_t stream, const SideStream* side = nullptr);

int cfg_euler_launch(float* x, const void* cond, const void* uncond, float cfg, float sigma, float sigma_next, int H,
                     int W, void* x_bf16, cudaStream_t stream);

int selftest_wait_timeout(int* err, int limit_us, cudaStream_t stream);

// Every CUDA allocation the library makes goes through these two, which count
// it (qi_alloc_count).
cudaError_t dev_malloc(void** p, size_t bytes);
cudaError_t host_malloc_pinned(void** p, size_t bytes);

int device_num_sms();

}  // namespace qi
