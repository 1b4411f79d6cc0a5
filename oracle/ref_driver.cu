// ref_driver.cu -- builds the reference's TransformerWeights from a device
// weight table and calls transformer_forward.  TEST INFRASTRUCTURE ONLY.
//
// Linked twice by oracle/build_ref.sh: with the reference's own transformer.cu
// (libqiref.so: the reference forward) and with the product's drop-in shim
// qwen-image.cu_b200/shim/transformer_b200.cpp (libshimtest.so: the same
// caller code running the product through the reference's types), which is
// how the drop-in boundary is tested.
#include "transformer.h"
#include "cuda_kernels.cuh"

#include "../include/qwen_image_b200.h"

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

// The reference's TransformerWeights over a device weight table (60 blocks;
// block_tables may repeat entries).
TransformerWeights make_weights(const void* const* g, const void* const* const* bt) {
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
  return w;
}

}  // namespace

extern "C" {

// transformer_forward (transformer.cu:234) over a weight table.  The
// reference loops over exactly 60 blocks; block_tables must hold 60 entries
// (they may repeat).  x: [1,16,H,W] BF16, ctx: [1,n_txt,3584] BF16,
// pe: [n_txt+n_img,64,2,2] FP32, out: [1,16,H,W] BF16; hidden_out (or null):
// the final image hidden state [n_img, 3072] FP32 (spectrum_hidden_out).
int ref_transformer_forward_capture(const void* const* g, const void* const* const* bt, const void* x, float t,
                                    const void* ctx, int n_txt, const float* pe, int H, int W, int sage, void* out,
                                    float* hidden_out) {
  TransformerWeights w = make_weights(g, bt);
  const int n_img = (H / 2) * (W / 2);
  Tensor xt = view_of(x, {1, 16, H, W}, DType::BF16);
  Tensor ct = view_of(ctx, {1, n_txt, 3584}, DType::BF16);
  Tensor pt = view_of(pe, {n_txt + n_img, 64, 2, 2}, DType::FP32);
  Tensor o = transformer_forward(w, xt, t, ct, pt, H, W, nullptr, sage != 0, hidden_out);
  cudaMemcpy(out, o.data, static_cast<size_t>(16) * H * W * 2, cudaMemcpyDeviceToDevice);
  o.free_data();
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : 3;
}

int ref_transformer_forward(const void* const* g, const void* const* const* bt, const void* x, float t,
                            const void* ctx, int n_txt, const float* pe, int H, int W, int sage, void* out) {
  return ref_transformer_forward_capture(g, bt, x, t, ctx, n_txt, pe, H, W, sage, out, nullptr);
}

// transformer_spectrum_output (transformer.cu:939-1028) on a final image
// hidden state [n_img, 3072] FP32; out: [1,16,H,W] BF16.
int ref_transformer_spectrum_output(const void* const* g, const void* const* const* bt, const float* hidden, float t,
                                    int H, int W, void* out) {
  TransformerWeights w = make_weights(g, bt);
  Tensor o = transformer_spectrum_output(w, hidden, t, H, W);
  cudaMemcpy(out, o.data, static_cast<size_t>(16) * H * W * 2, cudaMemcpyDeviceToDevice);
  o.free_data();
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : 3;
}

}  // extern "C"
