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

// rope_apply_fp32_to_fp16 (cuda_kernels.cu:1939-1971) on head-major [H, L, 128].
int ref_rope_fp16(const float* x, const float* pe, void* out, int H, int L) {
  rope_apply_fp32_to_fp16(x, pe, reinterpret_cast<__half*>(out), H, L, 128);
  return sync_status();
}

// gate_add_fp32f (cuda_kernels.cu:2181-2197): out = input + gate[col] * x.
int ref_gate_add(const float* input, const float* gate, const float* x, float* out, int rows, int dim) {
  gate_add_fp32f(input, gate, x, out, rows, dim);
  return sync_status();
}

// The reference's checkpoint upload path (SafeTensorsLoader::load_tensor,
// safetensors.h:174-212: per tensor fopen / fseek / fread into a host vector,
// cudaMalloc, synchronous cudaMemcpy) over every tensor of `path`, each freed
// after its upload.  Returns the bytes uploaded.  Timing baseline of the
// product's loader.
int ref_load_all(const char* path, long long* bytes) {
  SafeTensorsLoader L;
  L.load(path);
  long long total = 0;
  for (const auto& kv : L.tensors) {
    Tensor t = L.load_tensor(kv.first);
    total += static_cast<long long>(kv.second.nbytes);
    t.free_data();
  }
  *bytes = total;
  return sync_status();
}

// RoPE table from the reference's own host code (rope.h:175).
// spectrum_init / spectrum_update x K / spectrum_predict (cuda_kernels.cu:
// 6168-6333) on the states hist [K][F] stored at steps[0..K); out [F].
int ref_spectrum_predict(const float* hist, const int* steps, int K, long long F, int order, float lambda,
                         int target, float blend, float* out) {
  SpectrumState st;
  spectrum_init(st, static_cast<int>(F), 1, K, order);
  st.ridge_lambda = lambda;
  for (int k = 0; k < K; ++k) spectrum_update(st, hist + static_cast<size_t>(k) * F, steps[k]);
  spectrum_predict(st, out, target, blend);
  const int rc = sync_status();
  st.free_all();
  return rc;
}

int ref_rope_table(int h, int w, int n_txt, float* pe_host) {
  std::vector<float> pe = RoPE::gen_qwen_image_pe(h, w, 2, 1, n_txt, 10000, {16, 56, 56});
  memcpy(pe_host, pe.data(), pe.size() * sizeof(float));
  return 0;
}

}  // extern "C"
