/*
 * qi_oracle.c -- CPU restatement of qwen-image.cu's MMDiT denoising hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in qwen-image.cu_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it.  The product never links it.
 *
 * Every function restates one piece of the reference (paths are relative to
 * the reference project root) and says which.  Numerics:
 *   - The reference builds with --use_fast_math (Makefile:11), so its GPU
 *     quantizers use approximate 127/max and rsqrtf.  This oracle uses exact
 *     IEEE arithmetic; INT8 codes may therefore differ by +-1 at rounding
 *     ties and scales by an ulp.  Bit-exact code comparisons are made GPU vs
 *     GPU (product vs the reference's own CUDA build, oracle/_ref).
 *   - INT32 accumulators of the INT8 GEMM are exact, so for identical codes
 *     they must match bit for bit.
 *
 * Build: see oracle/Makefile (gcc -O3 -fopenmp -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

/* Conversions shared with qi_synth.c. */
uint16_t or_f32_to_f16(float f);
float or_f16_to_f32(uint16_t h);

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline float round_f16(float v) { return or_f16_to_f32(or_f32_to_f16(v)); }

/* ------------------------------------------------------------------------- */
/* Block Walsh-Hadamard transform, normalised by 1/sqrt(B) AFTER the
 * butterflies (cuda_kernels.cu:2209-2244 fwht_inplace_kernel and the same
 * stage order in fwht_quantize_kernel :2521-2542): stages half = 1, 2, 4, ...,
 * each (a, b) -> (a + b, a - b).  B = K & -K (cuda_kernels.cuh:253).         */

int or_hadamard_block_size(int K) { return K & (-K); }

static void fwht_row(float* row, int K, int B) {
    if (B <= 1) return;
    for (int base = 0; base < K; base += B) {
        float* v = row + base;
        for (int half = 1; half < B; half <<= 1) {
            int full = half << 1;
            for (int g = 0; g < B; g += full)
                for (int w = 0; w < half; ++w) {
                    float a = v[g + w], b = v[g + w + half];
                    v[g + w] = a + b;
                    v[g + w + half] = a - b;
                }
        }
    }
    float norm = (float)(1.0 / sqrt((double)B));
    for (int i = 0; i < K; ++i) row[i] *= norm;
}

void or_fwht_rows(float* x, int64_t M, int K, int B) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < M; ++r) fwht_row(x + r * K, K, B);
}

/* Per-row symmetric INT8: scale = max|x| / 127, code = sat(rint(x * 127/max))
 * (cuda_kernels.cu:2385-2409 quantize_per_row_fp32_kernel and the tail of
 * fwht_quantize_kernel :2544-2576).  __float2int_rn is round-half-even.     */
static void quant_row(const float* v, int K, int8_t* codes, float* scale) {
    float mx = 0.0f;
    for (int i = 0; i < K; ++i) mx = fmaxf(mx, fabsf(v[i]));
    *scale = mx / 127.0f;
    float inv = (mx > 0.0f) ? 127.0f / mx : 0.0f;
    for (int i = 0; i < K; ++i) {
        float q = nearbyintf(v[i] * inv);
        if (q > 127.0f) q = 127.0f;
        if (q < -128.0f) q = -128.0f;
        codes[i] = (int8_t)q;
    }
}

/* Activation path: fused FWHT + per-token INT8 (cuda_kernels.cu:2493-2577,
 * fwht_quantize_kernel<float>; dispatcher quantize_activation_int8_hadamard_fp32
 * :2603-2610, which skips the transform when B <= 1).                       */
void or_fwht_quant(const float* x, int64_t M, int K, int B, int8_t* codes, float* scales) {
#pragma omp parallel
    {
        float* tmp = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < M; ++r) {
            memcpy(tmp, x + r * K, sizeof(float) * (size_t)K);
            fwht_row(tmp, K, B);
            quant_row(tmp, K, codes + r * K, scales + r);
        }
        free(tmp);
    }
}

/* Weight path: BF16 -> FP32 -> FWHT rows (B = K & -K) -> per-row INT8
 * (quantize_weight_tensor, cuda_kernels.cu:2830-2862; quantize.cu:121-137
 * writes the result as "<name>" I8 [N,K] + "<name>.__scales__" F32 [N]).    */
void or_quant_weight_bf16(const uint16_t* w, int64_t N, int K, int8_t* codes, float* scales) {
    int B = or_hadamard_block_size(K);
#pragma omp parallel
    {
        float* tmp = (float*)malloc(sizeof(float) * (size_t)K);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < N; ++r) {
            for (int i = 0; i < K; ++i) tmp[i] = bf16_to_f32(w[r * K + i]);
            fwht_row(tmp, K, B);
            quant_row(tmp, K, codes + r * K, scales + r);
        }
        free(tmp);
    }
}

/* ------------------------------------------------------------------------- */
/* GEMMs.  C[M,N] = A[M,K] * B[N,K]^T, both operands K-contiguous, the layout
 * cublasGemmEx(OP_T, OP_N) consumes in cuda_kernels.cu:2711-2721.            */

void or_gemm_i8(const int8_t* A, const int8_t* B, int64_t M, int64_t N, int K, int32_t* C) {
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t i0 = 0; i0 < M; i0 += 4)
        for (int64_t j0 = 0; j0 < N; j0 += 64) {
            for (int64_t i = i0; i < i0 + 4 && i < M; ++i) {
                const int8_t* a = A + i * K;
                for (int64_t j = j0; j < j0 + 64 && j < N; ++j) {
                    const int8_t* b = B + j * K;
                    int32_t acc = 0;
#pragma omp simd reduction(+ : acc)
                    for (int k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
                    C[i * N + j] = acc;
                }
            }
        }
}

#define KB 512
void or_gemm_f32(const float* A, const float* B, int64_t M, int64_t N, int K, float* C) {
    memset(C, 0, sizeof(float) * (size_t)(M * N));
    for (int k0 = 0; k0 < K; k0 += KB) {
        int kl = (K - k0 < KB) ? (K - k0) : KB;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
        for (int64_t i0 = 0; i0 < M; i0 += 4)
            for (int64_t j0 = 0; j0 < N; j0 += 64) {
                int64_t il = (M - i0 < 4) ? (M - i0) : 4;
                int64_t jend = (N < j0 + 64) ? N : j0 + 64;
                if (il == 4) {
                    const float* a0 = A + (i0 + 0) * K + k0;
                    const float* a1 = A + (i0 + 1) * K + k0;
                    const float* a2 = A + (i0 + 2) * K + k0;
                    const float* a3 = A + (i0 + 3) * K + k0;
                    int64_t j = j0;
                    for (; j + 2 <= jend; j += 2) {
                        const float* b0 = B + j * K + k0;
                        const float* b1 = B + (j + 1) * K + k0;
                        float c00 = 0, c01 = 0, c10 = 0, c11 = 0, c20 = 0, c21 = 0, c30 = 0, c31 = 0;
#pragma omp simd reduction(+ : c00, c01, c10, c11, c20, c21, c30, c31)
                        for (int k = 0; k < kl; ++k) {
                            float x0 = b0[k], x1 = b1[k];
                            c00 += a0[k] * x0; c01 += a0[k] * x1;
                            c10 += a1[k] * x0; c11 += a1[k] * x1;
                            c20 += a2[k] * x0; c21 += a2[k] * x1;
                            c30 += a3[k] * x0; c31 += a3[k] * x1;
                        }
                        C[(i0 + 0) * N + j] += c00; C[(i0 + 0) * N + j + 1] += c01;
                        C[(i0 + 1) * N + j] += c10; C[(i0 + 1) * N + j + 1] += c11;
                        C[(i0 + 2) * N + j] += c20; C[(i0 + 2) * N + j + 1] += c21;
                        C[(i0 + 3) * N + j] += c30; C[(i0 + 3) * N + j + 1] += c31;
                    }
                    for (; j < jend; ++j) {
                        const float* b0 = B + j * K + k0;
                        for (int r = 0; r < 4; ++r) {
                            const float* a = A + (i0 + r) * K + k0;
                            float c = 0;
#pragma omp simd reduction(+ : c)
                            for (int k = 0; k < kl; ++k) c += a[k] * b0[k];
                            C[(i0 + r) * N + j] += c;
                        }
                    }
                } else {
                    for (int64_t i = i0; i < i0 + il; ++i)
                        for (int64_t j = j0; j < jend; ++j) {
                            const float* a = A + i * K + k0;
                            const float* b0 = B + j * K + k0;
                            float c = 0;
#pragma omp simd reduction(+ : c)
                            for (int k = 0; k < kl; ++k) c += a[k] * b0[k];
                            C[i * N + j] += c;
                        }
                }
            }
    }
}

/* GELU, tanh form with the reference's constants (cuda_kernels.cu:1863-1870,
 * dequantize_bias_gelu_kernel :2656-2658).                                  */
static inline float gelu_tanh(float v) {
    const float c = 0.7978845608f;
    float inner = c * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(inner));
}

/* Dequant epilogue: out = acc * sa[m] * sw[n] + bias[n] (+ GELU)
 * (cuda_kernels.cu:2623-2668).                                              */
void or_dequant(const int32_t* acc, const float* sa, const float* sw, const uint16_t* bias,
                int64_t M, int64_t N, int gelu, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j) {
            float v = (float)acc[i * N + j] * sa[i] * sw[j];
            if (bias) v += bf16_to_f32(bias[j]);
            out[i * N + j] = gelu ? gelu_tanh(v) : v;
        }
}

/* FP32 bias (+GELU) applied in place: the unquantized FP32 path of the oracle. */
void or_bias_act(float* out, const uint16_t* bias, int64_t M, int64_t N, int gelu) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j) {
            float v = out[i * N + j];
            if (bias) v += bf16_to_f32(bias[j]);
            out[i * N + j] = gelu ? gelu_tanh(v) : v;
        }
}

/* ------------------------------------------------------------------------- */
/* Norms and elementwise ops.                                                */

/* LayerNorm without affine, then modulate: (x - mu) * rsqrt(var + eps) *
 * (1 + scale) + shift (cuda_kernels.cu:1799-1853).  Accumulates in double.  */
void or_layernorm_modulate(const float* x, const float* shift, const float* scale,
                           int64_t M, int D, float eps, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < M; ++r) {
        const float* xr = x + r * D;
        double s = 0;
        for (int i = 0; i < D; ++i) s += xr[i];
        double mean = s / D;
        double v = 0;
        for (int i = 0; i < D; ++i) { double d = xr[i] - mean; v += d * d; }
        double inv = 1.0 / sqrt(v / D + eps);
        for (int i = 0; i < D; ++i)
            out[r * D + i] = (float)((xr[i] - mean) * inv * (1.0 + scale[i]) + shift[i]);
    }
}

/* RMSNorm over rows of length D with a BF16 weight (cuda_kernels.cu:1656-1693). */
void or_rmsnorm(const float* x, const uint16_t* w, int64_t rows, int D, float eps, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        double ss = 0;
        for (int i = 0; i < D; ++i) ss += (double)x[r * D + i] * x[r * D + i];
        double inv = 1.0 / sqrt(ss / D + eps);
        for (int i = 0; i < D; ++i) out[r * D + i] = (float)(x[r * D + i] * inv * bf16_to_f32(w[i]));
    }
}

/* SiLU (cuda_kernels.cu:1881-1887). */
void or_silu(const float* x, int64_t n, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] / (1.0f + expf(-x[i]));
}

/* x += gate[col] * y (cuda_kernels.cu:2181-2189). */
void or_gate_add(float* x, const float* gate, const float* y, int64_t M, int D) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < M; ++r)
        for (int i = 0; i < D; ++i) x[r * D + i] += gate[i] * y[r * D + i];
}

/* Sinusoidal timestep embedding [cos | sin], max_period 1e4
 * (cuda_kernels.cu:762-775 timestep_embedding_fp32_kernel).                 */
void or_timestep_embedding(float t, int dim, float max_period, float* out) {
    int half = dim / 2;
    for (int d = 0; d < half; ++d) {
        float freq = expf(-logf(max_period) * (float)d / (float)half);
        float a = t * freq;
        out[d] = cosf(a);
        out[half + d] = sinf(a);
    }
}

/* RoPE on interleaved pairs (2i, 2i+1) of each head row
 * (cuda_kernels.cu:1935-1963): out0 = x0*pe0 + x1*pe1, out1 = x0*pe2 + x1*pe3.
 * x: [rows, H, 128] token-major; pos[row] gives the pe row.                 */
void or_rope_apply(float* x, const float* pe, const int* pos, int64_t rows, int H) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int h = 0; h < H; ++h) {
            float* v = x + (r * H + h) * 128;
            const float* e = pe + (size_t)pos[r] * 256;
            for (int i = 0; i < 64; ++i) {
                float x0 = v[2 * i], x1 = v[2 * i + 1];
                v[2 * i] = x0 * e[4 * i] + x1 * e[4 * i + 1];
                v[2 * i + 1] = x0 * e[4 * i + 2] + x1 * e[4 * i + 3];
            }
        }
}

/* ------------------------------------------------------------------------- */
/* Attention.  q, k, v: [H, S, 128] FP32.  out: [H, S, 128].                 */

/* Exact softmax attention in double (the fp32 CPU evaluation). */
void or_attention_exact(const float* q, const float* k, const float* v, int H, int S, float scale,
                        float* out) {
#pragma omp parallel
    {
        double* p = (double*)malloc(sizeof(double) * (size_t)S);
#pragma omp for collapse(2) schedule(static)
        for (int h = 0; h < H; ++h)
            for (int i = 0; i < S; ++i) {
                const float* qi = q + ((size_t)h * S + i) * 128;
                double mx = -1e300;
                for (int j = 0; j < S; ++j) {
                    const float* kj = k + ((size_t)h * S + j) * 128;
                    double s = 0;
                    for (int d = 0; d < 128; ++d) s += (double)qi[d] * kj[d];
                    p[j] = s * scale;
                    if (p[j] > mx) mx = p[j];
                }
                double sum = 0;
                for (int j = 0; j < S; ++j) { p[j] = exp(p[j] - mx); sum += p[j]; }
                double o[128] = {0};
                for (int j = 0; j < S; ++j) {
                    const float* vj = v + ((size_t)h * S + j) * 128;
                    for (int d = 0; d < 128; ++d) o[d] += p[j] * vj[d];
                }
                for (int d = 0; d < 128; ++d) out[((size_t)h * S + i) * 128 + d] = (float)(o[d] / sum);
            }
        free(p);
    }
}

static inline int8_t cvt_rni_sat_s8(float x) {
    float r = nearbyintf(x);
    if (r > 127.0f) r = 127.0f;
    if (r < -128.0f) r = -128.0f;
    return (int8_t)r;
}

/* Per-head mean of K over all S tokens, summed serially in token order
 * (sageattention_sm80.cu:759-773).  k: FP16 values as float, [H, S, 128]. */
void or_sage_kmean(const float* k, int H, int S, float* kmean) {
    for (int h = 0; h < H; ++h)
        for (int d = 0; d < 128; ++d) {
            float s = 0.0f;
            for (int t = 0; t < S; ++t) s += k[((size_t)h * S + t) * 128 + d];
            kmean[h * 128 + d] = s / fmaxf((float)S, 1.0f);
        }
}

/* Q per-thread INT8 (sageattention_sm80.cu:775-824): 32 scales per 128-token
 * block; group g covers tokens base + {0, 8, 16, 24} with
 * base = (g/32)*128 + ((g%32)/8)*32 + g%8.  amax starts at 1e-7; scale =
 * amax/127 + 1e-7; code = cvt.rni.sat.s8(v / scale).
 * q: [H, S, 128]; codes [H, S, 128]; scales [H, ceil(S/128)*32].           */
void or_sage_quant_q(const float* q, int H, int S, int8_t* codes, float* scales) {
    int ng = ((S + 127) / 128) * 32;
    for (int h = 0; h < H; ++h)
        for (int g = 0; g < ng; ++g) {
            int base = (g / 32) * 128 + ((g % 32) / 8) * 32 + (g % 8);
            float amax = 1e-7f;
            for (int i = 0; i < 4; ++i) {
                int t = base + i * 8;
                if (t >= S) continue;
                for (int d = 0; d < 128; ++d) amax = fmaxf(amax, fabsf(q[((size_t)h * S + t) * 128 + d]));
            }
            float sc = amax / 127.0f + 1e-7f;
            scales[(size_t)h * ng + g] = sc;
            float inv = 1.0f / sc;
            for (int i = 0; i < 4; ++i) {
                int t = base + i * 8;
                if (t >= S) continue;
                for (int d = 0; d < 128; ++d)
                    codes[((size_t)h * S + t) * 128 + d] = cvt_rni_sat_s8(q[((size_t)h * S + t) * 128 + d] * inv);
            }
        }
}

/* K per-thread INT8 after mean smoothing (sageattention_sm80.cu:826-886):
 * 4 scales per 64-token block; group g covers tokens base + 8i + {0, 1},
 * i = 0..7, base = (g/4)*64 + (g%4)*2.                                      */
void or_sage_quant_k(const float* k, const float* kmean, int H, int S, int8_t* codes, float* scales) {
    int ng = ((S + 63) / 64) * 4;
    for (int h = 0; h < H; ++h)
        for (int g = 0; g < ng; ++g) {
            int base = (g / 4) * 64 + (g % 4) * 2;
            float amax = 1e-7f;
            for (int i = 0; i < 8; ++i)
                for (int e = 0; e < 2; ++e) {
                    int t = base + i * 8 + e;
                    if (t >= S) continue;
                    for (int d = 0; d < 128; ++d)
                        amax = fmaxf(amax, fabsf(k[((size_t)h * S + t) * 128 + d] - kmean[h * 128 + d]));
                }
            float sc = amax / 127.0f + 1e-7f;
            scales[(size_t)h * ng + g] = sc;
            float inv = 1.0f / sc;
            for (int i = 0; i < 8; ++i)
                for (int e = 0; e < 2; ++e) {
                    int t = base + i * 8 + e;
                    if (t >= S) continue;
                    for (int d = 0; d < 128; ++d)
                        codes[((size_t)h * S + t) * 128 + d] =
                            cvt_rni_sat_s8((k[((size_t)h * S + t) * 128 + d] - kmean[h * 128 + d]) * inv);
                }
        }
}

/* Quantized attention on the Sage codes (sageattention_sm80.cu:47-674 with
 * update_mdo / normalize_d, sageattention_attn_utils.cuh:352-456, :719-760):
 * s = int(qc . kc) * qs * ks * sm_scale * log2(e); online softmax in base 2
 * over 64-key blocks; P rounded to FP16 before both the row sum and P.V;
 * V in FP16; the result rounded to FP16.  Computed in double apart from the
 * FP16 roundings, so it differs from the GPU only by accumulation order.
 * v: FP16 values as float [H, S, 128].  out: [H, S, 128].                  */
void or_sage_attention(const int8_t* qc, const float* qs, const int8_t* kc, const float* ks,
                       const float* v, int H, int S, float sm_scale, float* out) {
    const double log2e = 1.44269504088896340736;
    int ngq = ((S + 127) / 128) * 32, ngk = ((S + 63) / 64) * 4;
#pragma omp parallel
    {
        double* p = (double*)malloc(sizeof(double) * (size_t)S);
#pragma omp for collapse(2) schedule(static)
        for (int h = 0; h < H; ++h)
            for (int i = 0; i < S; ++i) {
                int gq = (i / 128) * 32 + ((i % 128) / 32) * 8 + (i % 8);
                double qsc = qs[(size_t)h * ngq + gq];
                const int8_t* qi = qc + ((size_t)h * S + i) * 128;
                double mx = -1e300;
                for (int j = 0; j < S; ++j) {
                    const int8_t* kj = kc + ((size_t)h * S + j) * 128;
                    int32_t acc = 0;
                    for (int d = 0; d < 128; ++d) acc += (int32_t)qi[d] * (int32_t)kj[d];
                    int gk = (j / 64) * 4 + ((j % 64) % 8) / 2;
                    p[j] = (double)acc * qsc * ks[(size_t)h * ngk + gk] * sm_scale * log2e;
                    if (p[j] > mx) mx = p[j];
                }
                double sum = 0, o[128] = {0};
                for (int j = 0; j < S; ++j) {
                    double pj = round_f16((float)exp2(p[j] - mx));
                    sum += pj;
                    const float* vj = v + ((size_t)h * S + j) * 128;
                    for (int d = 0; d < 128; ++d) o[d] += pj * vj[d];
                }
                for (int d = 0; d < 128; ++d) out[((size_t)h * S + i) * 128 + d] = round_f16((float)(o[d] / sum));
            }
        free(p);
    }
}

int or_num_threads(void) { return omp_get_max_threads(); }
void or_set_num_threads(int n) { omp_set_num_threads(n); }

/* FP32 softmax attention through the blocked GEMM (for the timed CPU
 * baseline at full sequence length): per head, 256-query blocks of scores
 * S = Q K^T * scale, row softmax, O = P V.  q, k, v, out: [H, S, 128].     */
void or_attention_f32(const float* q, const float* k, const float* v, int H, int S, float scale, float* out) {
    const int QB = 256;
    float* vt = (float*)malloc(sizeof(float) * 128 * (size_t)S);
    float* sc = (float*)malloc(sizeof(float) * (size_t)QB * (size_t)S);
    for (int h = 0; h < H; ++h) {
        const float* qh = q + (size_t)h * S * 128;
        const float* kh = k + (size_t)h * S * 128;
        const float* vh = v + (size_t)h * S * 128;
#pragma omp parallel for schedule(static)
        for (int d = 0; d < 128; ++d)
            for (int s = 0; s < S; ++s) vt[(size_t)d * S + s] = vh[(size_t)s * 128 + d];
        for (int i0 = 0; i0 < S; i0 += QB) {
            int qb = (S - i0 < QB) ? (S - i0) : QB;
            or_gemm_f32(qh + (size_t)i0 * 128, kh, qb, S, 128, sc);
#pragma omp parallel for schedule(static)
            for (int r = 0; r < qb; ++r) {
                float* row = sc + (size_t)r * S;
                float mx = -INFINITY;
                for (int j = 0; j < S; ++j) { row[j] *= scale; if (row[j] > mx) mx = row[j]; }
                float sum = 0.0f;
                for (int j = 0; j < S; ++j) { row[j] = expf(row[j] - mx); sum += row[j]; }
                float inv = 1.0f / sum;
                for (int j = 0; j < S; ++j) row[j] *= inv;
            }
            or_gemm_f32(sc, vt, qb, 128, S, out + ((size_t)h * S + i0) * 128);
        }
    }
    free(vt);
    free(sc);
}
