// ref_harness.cu -- C entry points over the reference's OWN CUDA code.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/build_ref.sh from the reference
// sources where they lie (cuda_kernels.cu, transformer.cu and, included
// below, sageattention_sm80.cu) with the reference's own compiler flags,
// into oracle/_ref/libqiref.so.  The parity tests call it on the GPU box to
// compare the product with the reference on identical device inputs, and
// bench.py --impl reference times the reference's transformer_forward
// through it.  Nothing here is part of the product.
//
// The weight table layout is the product's public one
// (include/qwen_image_b200.h QI_G_* / QI_L_* / QI_B_*), so both sides read the
// same device tensors.
#include "transformer.h"
#include "cuda_kernels.cuh"
// Included (not linked) so the file's internal-linkage quantizer kernels are
// reachable for the bit-exact code comparisons.
#include "sageattention_sm80.cu"
#include "rope.h"

#include "../include/qwen_image_b200.h"

#include <vector>

namespace {

Tensor view_of(const void* p, std::initializer_list<int64_t> dims, DType dt) {
  Tensor t;
  t.data = const_cast<void*>(p);
  t.ndim = static_cast<int>(dims.size());
  int i = 0;
  for (auto d : dims) t.shape[i++] = d;
  t.dtype = dt;
  t.owns_data = false;
  return t;
}

QuantizedWeight qw_int8(const void* codes, const void* scales, int N, int K) {
  QuantizedWeight q;
  q.mode = QuantMode::INT8_HADAMARD;
  q.data = view_of(codes, {N, K}, DType::INT8);
  q.scales = view_of(scales, {N}, DType::FP32);
  q.had_block_size = hadamard_block_size(K);
  return q;
}

QuantizedWeight qw_bf16(const void* w, int N, int K) {
  QuantizedWeight q;
  q.mode = QuantMode::BF16;
  q.data = view_of(w, {N, K}, DType::BF16);
  return q;
}

int sync_status() { return cudaDeviceSynchronize() == cudaSuccess ? 0 : 3; }

uint64_t sm64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Same seeded generator as the product and the CPU oracle, so the reference
// arm of bench.py builds its inputs without touching the product library.
__global__ void ref_synth_kernel(uint64_t sm, long long n, float scale, float offset, void* out, int bf16) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint64_t x1 = sm + 2ull * static_cast<uint64_t>(i), x2 = x1 + 1ull;
    x1 += 0x9E3779B97F4A7C15ull;
    x1 = (x1 ^ (x1 >> 30)) * 0xBF58476D1CE4E5B9ull;
    x1 = (x1 ^ (x1 >> 27)) * 0x94D049BB133111EBull;
    x1 ^= x1 >> 31;
    x2 += 0x9E3779B97F4A7C15ull;
    x2 = (x2 ^ (x2 >> 30)) * 0xBF58476D1CE4E5B9ull;
    x2 = (x2 ^ (x2 >> 27)) * 0x94D049BB133111EBull;
    x2 ^= x2 >> 31;
    const uint64_t m24 = 0xFFFFFFull;
    const long long s = (long long)(x1 & m24) + (long long)((x1 >> 24) & m24) + (long long)(x2 & m24) +
                        (long long)((x2 >> 24) & m24);
    float v = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(s - 33554430ll)), 0x1.bb67aep-24f), scale);
    if (offset != 0.0f) v = __fadd_rn(v, offset);
    if (bf16)
      reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else
      reinterpret_cast<float*>(out)[i] = v;
  }
}

}  // namespace

extern "C" {

int ref_synth_fill(void* out, long long n, unsigned long long seed, float scale, float offset, int bf16) {
  long long blocks = (n + 255) / 256;
  if (blocks > 4736) blocks = 4736;
  if (n > 0) ref_synth_kernel<<<(unsigned)blocks, 256>>>(sm64(seed), n, scale, offset, out, bf16);
  return sync_status();
}

// quantize_weight_tensor (cuda_kernels.cu:2830).
int ref_quantize_weight(const void* w_bf16, int N, int K, int8_t* codes, float* scales) {
  Tensor w = view_of(w_bf16, {N, K}, DType::BF16);
  QuantizedWeight q = quantize_weight_tensor(w);
  cudaMemcpy(codes, q.data.data, static_cast<size_t>(N) * K, cudaMemcpyDeviceToDevice);
  cudaMemcpy(scales, q.scales.data, static_cast<size_t>(N) * 4, cudaMemcpyDeviceToDevice);
  q.free_data();
  return sync_status();
}

// quantize_activation_int8_hadamard_fp32 (cuda_kernels.cu:2603).
int ref_fwht_quantize(const float* x, int M, int K, int hbs, int8_t* codes, float* scales) {
  quantize_activation_int8_hadamard_fp32(x, codes, scales, M, K, hbs);
  return sync_status();
}

// linear_forward_int8_prequantized (cuda_kernels.cu:2735).
int ref_linear_int8_preq(const int8_t* a, const float* sa, int M, int K, const int8_t* w, const float* sw, int N,
                         const void* bias, int gelu, float* out) {
  QuantizedWeight q = qw_int8(w, sw, N, K);
  Tensor b = view_of(bias, {N}, DType::BF16);
  Tensor o = view_of(out, {M, N}, DType::FP32);
  int64_t bytes = int8_scratch_bytes(M, K, N);
  Tensor scratch = Tensor::alloc({(bytes + 3) / 4}, DType::FP32);
  linear_forward_int8_prequantized(a, sa, M, K, q, bias ? &b : nullptr, o, scratch, gelu != 0);
  int st = sync_status();
  scratch.free_data();
  return st;
}

// linear_forward_quantized on an INT8 weight (cuda_kernels.cu:4599 -> :2674).
int ref_linear_int8(const float* x, int M, int K, const int8_t* w, const float* sw, int N, const void* bias, int gelu,
                    float* out) {
  QuantizedWeight q = qw_int8(w, sw, N, K);
  Tensor xt = view_of(x, {M, K}, DType::FP32);
  Tensor b = view_of(bias, {N}, DType::BF16);
  Tensor o = view_of(out, {M, N}, DType::FP32);
  int64_t bytes = int8_scratch_bytes(M, K, N);
  Tensor scratch = Tensor::alloc({(bytes + 3) / 4}, DType::FP32);
  linear_forward_quantized(xt, q, bias ? &b : nullptr, o, scratch, gelu != 0);
  int st = sync_status();
  scratch.free_data();
  return st;
}

// The three Sage quantizers (sageattention_sm80.cu:759-886), launched as
// attention_forward_sage_sm80_fp16io launches them (:994-1007).
int ref_sage_quantize(const void* q, const void* k, int BH, int S, float* kmean, int8_t* qc, float* qs, int8_t* kc,
                      float* ks) {
  sageattention_k_mean_kernel<128><<<BH, 128>>>(reinterpret_cast<const half*>(k), kmean, BH, S);
  sageattention_query_per_thread_int8_kernel<128><<<dim3(div_ceil(S, 128) * 32, BH), 128>>>(
      reinterpret_cast<const half*>(q), qc, qs, BH, S);
  sageattention_key_per_thread_int8_kernel<128><<<dim3(div_ceil(S, 64) * 4, BH), 128>>>(
      reinterpret_cast<const half*>(k), kmean, kc, ks, BH, S);
  return sync_status();
}

// attention_forward_sage_sm80_fp16io (sageattention_sm80.cu:965).
int ref_sage_attention(const void* q, const void* k, const void* v, float* out, float scale, int BH, int S) {
  attention_forward_sage_sm80_fp16io(reinterpret_cast<const __half*>(q), reinterpret_cast<const __half*>(k),
                                     reinterpret_cast<const __half*>(v), out, scale, BH, S, 128, false, 0);
  return sync_status();
}

int ref_layer_norm_modulate(const float* x, const float* shift, const float* scale, float* out, int rows, int dim,
                            float eps) {
  layer_norm_modulate_fp32(x, shift, scale, out, rows, dim, eps);
  return sync_status();
}

int ref_rms_norm_fp32(const float* x, const void* w, float* out, int rows, int dim, float eps) {
  rms_norm_fp32(x, reinterpret_cast<const __nv_bfloat16*>(w), out, rows, dim, eps);
  return sync_status();
}

// RoPE table from the reference's own host code (rope.h:175).
int ref_rope_table(int h, int w, int n_txt, float* pe_host) {
  std::vector<float> pe = RoPE::gen_qwen_image_pe(h, w, 2, 1, n_txt, 10000, {16, 56, 56});
  memcpy(pe_host, pe.data(), pe.size() * sizeof(float));
  return 0;
}

// transformer_forward (transformer.cu:234) over a weight table.  The
// reference loops over exactly 60 blocks; block_tables must hold 60 entries
// (they may repeat).  x: [1,16,H,W] BF16, ctx: [1,n_txt,3584] BF16,
// pe: [n_txt+n_img,64,2,2] FP32, out: [1,16,H,W] BF16.
int ref_transformer_forward(const void* const* g, const void* const* const* bt, const void* x, float t,
                            const void* ctx, int n_txt, const float* pe, int H, int W, int sage, void* out) {
  TransformerWeights w;
  w.time_linear1_weight = qw_int8(g[QI_G_T1_W], g[QI_G_T1_S], 3072, 256);
  w.time_linear1_bias = view_of(g[QI_G_T1_B], {3072}, DType::BF16);
  w.time_linear2_weight = qw_int8(g[QI_G_T2_W], g[QI_G_T2_S], 3072, 3072);
  w.time_linear2_bias = view_of(g[QI_G_T2_B], {3072}, DType::BF16);
  w.txt_norm_weight = view_of(g[QI_G_TXT_NORM], {3584}, DType::BF16);
  w.img_in_weight = qw_bf16(g[QI_G_IMG_IN_W], 3072, 64);
  w.img_in_bias = view_of(g[QI_G_IMG_IN_B], {3072}, DType::BF16);
  w.txt_in_weight = qw_bf16(g[QI_G_TXT_IN_W], 3072, 3584);
  w.txt_in_bias = view_of(g[QI_G_TXT_IN_B], {3072}, DType::BF16);
  w.norm_out_linear_weight = qw_bf16(g[QI_G_NORM_OUT_W], 6144, 3072);
  w.norm_out_linear_bias = view_of(g[QI_G_NORM_OUT_B], {6144}, DType::BF16);
  w.proj_out_weight = qw_bf16(g[QI_G_PROJ_OUT_W], 64, 3072);
  w.proj_out_bias = view_of(g[QI_G_PROJ_OUT_B], {64}, DType::BF16);
  w.blocks.resize(60);
  static const int dims[QI_L_COUNT][2] = {
      {18432, 3072}, {18432, 3072}, {3072, 3072}, {3072, 3072}, {3072, 3072}, {3072, 3072}, {3072, 3072},
      {3072, 3072},  {3072, 3072},  {3072, 3072}, {12288, 3072}, {3072, 12288}, {12288, 3072}, {3072, 12288}};
  for (int i = 0; i < 60; ++i) {
    const void* const* tb = bt[i];
    auto& B = w.blocks[i];
    QuantizedWeight* lw[QI_L_COUNT] = {&B.img_mod_weight,      &B.txt_mod_weight,    &B.to_q_weight,
                                       &B.to_k_weight,         &B.to_v_weight,       &B.add_q_proj_weight,
                                       &B.add_k_proj_weight,   &B.add_v_proj_weight, &B.to_out_weight,
                                       &B.to_add_out_weight,   &B.img_mlp_fc1_weight, &B.img_mlp_fc2_weight,
                                       &B.txt_mlp_fc1_weight,  &B.txt_mlp_fc2_weight};
    Tensor* lb[QI_L_COUNT] = {&B.img_mod_bias,    &B.txt_mod_bias,    &B.to_q_bias,        &B.to_k_bias,
                              &B.to_v_bias,       &B.add_q_proj_bias, &B.add_k_proj_bias,  &B.add_v_proj_bias,
                              &B.to_out_bias,     &B.to_add_out_bias, &B.img_mlp_fc1_bias, &B.img_mlp_fc2_bias,
                              &B.txt_mlp_fc1_bias, &B.txt_mlp_fc2_bias};
    for (int l = 0; l < QI_L_COUNT; ++l) {
      *lw[l] = qw_int8(tb[3 * l], tb[3 * l + 1], dims[l][0], dims[l][1]);
      *lb[l] = view_of(tb[3 * l + 2], {dims[l][0]}, DType::BF16);
    }
    B.norm_q_weight = view_of(tb[QI_B_NORM_Q], {128}, DType::BF16);
    B.norm_k_weight = view_of(tb[QI_B_NORM_K], {128}, DType::BF16);
    B.norm_added_q_weight = view_of(tb[QI_B_NORM_ADDED_Q], {128}, DType::BF16);
    B.norm_added_k_weight = view_of(tb[QI_B_NORM_ADDED_K], {128}, DType::BF16);
  }
  const int n_img = (H / 2) * (W / 2);
  Tensor xt = view_of(x, {1, 16, H, W}, DType::BF16);
  Tensor ct = view_of(ctx, {1, n_txt, 3584}, DType::BF16);
  Tensor pt = view_of(pe, {n_txt + n_img, 64, 2, 2}, DType::FP32);
  Tensor o = transformer_forward(w, xt, t, ct, pt, H, W, nullptr, sage != 0, nullptr);
  cudaMemcpy(out, o.data, static_cast<size_t>(16) * H * W * 2, cudaMemcpyDeviceToDevice);
  o.free_data();
  return sync_status();
}

}  // extern "C"
