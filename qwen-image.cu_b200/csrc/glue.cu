// glue.cu -- the memory-bound pieces of the block and the boundary layers.
//
// Expressions that feed a quantizer (timestep embedding, SiLU) are written the
// way the reference writes them so that, built with the same fast-math flags,
// they produce the same bits; the rest only has to agree within tolerance.
#include "qi_internal.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace qi {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (l < NT / 32) ? red[l] : 0.0f;
  r = warp_sum(r);
  __syncthreads();
  return r;
}

// ------------------------------------------------------------------ q/k/v
// One warp per (token, head).  Lane i holds elements 4i..4i+3 = RoPE pairs
// 2i and 2i+1.  RMSNorm (rms_norm_fp32_kernel, cuda_kernels.cu:1656-1688:
// x * rsqrt(mean(x^2) + eps) * w) then RoPE on interleaved pairs
// (rope_apply_fp32_to_fp16_kernel, cuda_kernels.cu:1935-1963) then FP16,
// written head-major in the joint [txt; img] order (transformer.cu:637-666).
__global__ void qkv_post_kernel(QkvPostArgs a) {
  const int warps = blockDim.x >> 5;
  const long long gw = static_cast<long long>(blockIdx.x) * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long rows_img = static_cast<long long>(a.nb) * a.n_img_l;
  const long long rows = rows_img + static_cast<long long>(a.nb) * a.n_txt_l;
  if (gw >= rows * kHeads) return;
  const long long r = gw / kHeads;
  const int h = static_cast<int>(gw % kHeads);
  const int S = a.n_img + a.n_txt;
  const int L = a.n_img_l + a.n_txt_l;  // local sequence length
  const float* src;
  int b, pos, lpos;                     // batch entry, joint position, local position
  const __nv_bfloat16 *wq, *wk;
  if (r < rows_img) {
    src = a.qkv_img + r * (3 * kDim);
    b = static_cast<int>(r / a.n_img_l);
    const int i = static_cast<int>(r % a.n_img_l);
    pos = a.n_txt + a.img_lo + i;
    lpos = a.n_txt_l + i;
    wq = reinterpret_cast<const __nv_bfloat16*>(a.nq_img);
    wk = reinterpret_cast<const __nv_bfloat16*>(a.nk_img);
  } else {
    const long long rt = r - rows_img;
    src = a.qkv_txt + rt * (3 * kDim);
    b = static_cast<int>(rt / a.n_txt_l);
    const int t = static_cast<int>(rt % a.n_txt_l);
    pos = a.txt_lo + t;
    lpos = t;
    wq = reinterpret_cast<const __nv_bfloat16*>(a.nq_txt);
    wk = reinterpret_cast<const __nv_bfloat16*>(a.nk_txt);
  }
  const int d0 = lane * 4;
  const float4 qv = *reinterpret_cast<const float4*>(src + h * kHeadDim + d0);
  const float4 kv = *reinterpret_cast<const float4*>(src + kDim + h * kHeadDim + d0);
  const float4 vv = *reinterpret_cast<const float4*>(src + 2 * kDim + h * kHeadDim + d0);
  const float* pe = a.pe + (static_cast<long long>(b) * S + pos) * 256 + lane * 8;
  const float4 pe0 = __ldg(reinterpret_cast<const float4*>(pe));
  const float4 pe1 = __ldg(reinterpret_cast<const float4*>(pe + 4));
  const int dest = h / a.Hl, hh = h % a.Hl;
  size_t slab, dst;
  __half* base;
  if (a.direct) {
    // the head owner's buffer, [which][b][hh][joint position][128]
    slab = static_cast<size_t>(a.nb) * a.Hl * S * kHeadDim;
    dst = ((static_cast<size_t>(b) * a.Hl + hh) * S + pos) * kHeadDim + d0;
    base = reinterpret_cast<__half*>(a.peer_qkvh[dest]);
  } else {
    // qkvh[dest][which][b][hh][lpos][128]; `which` adds one (nb * Hl * L * 128) slab
    slab = static_cast<size_t>(a.nb) * a.Hl * L * kHeadDim;
    dst = static_cast<size_t>(dest) * 3 * slab + ((static_cast<size_t>(b) * a.Hl + hh) * L + lpos) * kHeadDim + d0;
    base = reinterpret_cast<__half*>(a.qkvh);
  }

  auto norm_rope = [&](float4 x, const __nv_bfloat16* w, __half* out) {
    // sum of squares in the order of rms_norm_fp32_kernel's reduction (128
    // threads, thread t = element t, shfl_down 16..1 per warp, then warp 0
    // over the 4 warp sums): reference warp w = lane / 8 and lane bits 2..0,
    // then the float4 components (offsets 2, 1), hold its lane offsets
    // 16, 8, 4 and 2, 1; the warp sums combine as (w0 + w2) + (w1 + w3).
    float s0 = x.x * x.x, s1 = x.y * x.y, s2 = x.z * x.z, s3 = x.w * x.w;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
      s3 += __shfl_xor_sync(0xffffffffu, s3, o);
    }
    float ss = (s0 + s2) + (s1 + s3);
    ss += __shfl_xor_sync(0xffffffffu, ss, 16);
    ss += __shfl_xor_sync(0xffffffffu, ss, 8);
    const float rms = rsqrtf(ss / a.norm_dim + a.eps);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(w + d0);
    const float2 w01 = __bfloat1622float2(w2[0]);
    const float2 w23 = __bfloat1622float2(w2[1]);
    const float x0 = x.x * rms * w01.x, x1 = x.y * rms * w01.y;
    const float x2 = x.z * rms * w23.x, x3 = x.w * rms * w23.y;
    const float o0 = x0 * pe0.x + x1 * pe0.y;
    const float o1 = x0 * pe0.z + x1 * pe0.w;
    const float o2 = x2 * pe1.x + x3 * pe1.y;
    const float o3 = x2 * pe1.z + x3 * pe1.w;
    __half2 h01 = __floats2half2_rn(o0, o1), h23 = __floats2half2_rn(o2, o3);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&h01);
    pk.y = *reinterpret_cast<uint32_t*>(&h23);
    *reinterpret_cast<uint2*>(out + dst) = pk;
  };
  norm_rope(qv, wq, base);
  norm_rope(kv, wk, base + slab);
  __half2 v01 = __floats2half2_rn(vv.x, vv.y), v23 = __floats2half2_rn(vv.z, vv.w);
  uint2 pv;
  pv.x = *reinterpret_cast<uint32_t*>(&v01);
  pv.y = *reinterpret_cast<uint32_t*>(&v23);
  *reinterpret_cast<uint2*>(base + 2 * slab + dst) = pv;
}

// Received Q/K/V of this rank's heads, [src][3][nb][Hl][len(src)][128], into
// [3][nb*Hl][S][128] in the joint order: one 256-byte row per thread group of
// 16 (16 bytes each).
__global__ void ulysses_gather_qkv_kernel(const uint4* __restrict__ recv, uint4* __restrict__ out, int nb, int Hl,
                                          int n_txt, ShardMap map) {
  const int S = map.txt_lo[map.P] + map.img_lo[map.P];
  const long long total = 3LL * nb * Hl * S * 16;  // 16-byte pieces of the output
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int piece = static_cast<int>(idx & 15);
    const long long row = idx >> 4;  // [which][b][hh][pos]
    const int pos = static_cast<int>(row % S);
    const long long wbh = row / S;   // (which * nb + b) * Hl + hh
    // owner of the joint position and its local index there
    int src = 0, lpos;
    if (pos < n_txt) {
      while (src + 1 < map.P && map.txt_lo[src + 1] <= pos) ++src;
      lpos = pos - map.txt_lo[src];
    } else {
      const int gi = pos - n_txt;
      while (src + 1 < map.P && map.img_lo[src + 1] <= gi) ++src;
      lpos = map.n_txt_l(src) + gi - map.img_lo[src];
    }
    long long off = 0;  // start of src's chunk, in 128-element rows
    for (int q = 0; q < src; ++q) off += 3LL * nb * Hl * map.len(q);
    const long long in_row = off + wbh * map.len(src) + lpos;
    out[idx] = recv[in_row * 16 + piece];
  }
}

// Received attention output, [src][nb][len(r)][Hl][128] (src's heads), into
// this rank's token-major rows: image rows [nb][n_img_l] then text rows
// [nb][n_txt_l], each [24 heads][128] with head = src * Hl + hh.
__global__ void ulysses_gather_o_kernel(const uint4* __restrict__ recv, uint4* __restrict__ out, int nb, int Hl,
                                        int rank, ShardMap map) {
  const int nt = map.n_txt_l(rank), ni = map.n_img_l(rank), L = nt + ni;
  const long long rows = static_cast<long long>(nb) * L;
  const long long total = rows * kHeads * 16;
  for (long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int piece = static_cast<int>(idx & 15);
    const int h = static_cast<int>((idx >> 4) % kHeads);
    const long long orow = (idx >> 4) / kHeads;
    int b, lpos;
    if (orow < static_cast<long long>(nb) * ni) {
      b = static_cast<int>(orow / ni);
      lpos = nt + static_cast<int>(orow % ni);
    } else {
      const long long t = orow - static_cast<long long>(nb) * ni;
      b = static_cast<int>(t / nt);
      lpos = static_cast<int>(t % nt);
    }
    const int src = h / Hl, hh = h % Hl;
    const long long in_row = ((static_cast<long long>(src) * nb + b) * L + lpos) * Hl + hh;
    out[idx] = recv[in_row * 16 + piece];
  }
}

// ------------------------------------------------------------------ GEMV
// M = 1 INT8 linear over a contiguous weight matrix [N, K]:
// out[n] = dot(act, w[n]) * act_scale * sw[n] + bias[n]
// (dequantize_and_bias_kernel, cuda_kernels.cu:2623-2633).  HBM-bound on the
// weight bytes; one warp per row, 16-byte loads, dp4a.
__global__ void gemv_i8_kernel(const int8_t* __restrict__ act, const float* __restrict__ act_scale, int K,
                               const int8_t* __restrict__ w, const float* __restrict__ sw,
                               const __nv_bfloat16* __restrict__ bias, float* __restrict__ out, long long N) {
  extern __shared__ int4 sact[];
  const int nchunk = K / 16;
  for (int i = threadIdx.x; i < nchunk; i += blockDim.x) sact[i] = reinterpret_cast<const int4*>(act)[i];
  __syncthreads();
  const float sa = *act_scale;
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long n = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
    const int4* row = reinterpret_cast<const int4*>(w + n * K);
    int acc = 0;
    for (int c = lane; c < nchunk; c += 32) {
      const int4 a4 = sact[c];
      const int4 w4 = __ldg(row + c);
      acc = __dp4a(a4.x, w4.x, acc);
      acc = __dp4a(a4.y, w4.y, acc);
      acc = __dp4a(a4.z, w4.z, acc);
      acc = __dp4a(a4.w, w4.w, acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      float v = static_cast<float>(acc) * sa * sw[n];
      if (bias) v += __bfloat162float(bias[n]);
      out[n] = v;
    }
  }
}

// M = 1 BF16 linear: x (FP32) is rounded to BF16 first, as linear_forward_bf16
// does before its cuBLAS call (cuda_kernels.cu:4535-4568).
__global__ void gemv_bf16_kernel(const float* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                                 const __nv_bfloat16* __restrict__ bias, float* __restrict__ out, int N, int K) {
  extern __shared__ float sx[];
  for (int i = threadIdx.x; i < K; i += blockDim.x) sx[i] = __bfloat162float(__float2bfloat16(x[i]));
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int n = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); n < N; n += warps) {
    const __nv_bfloat162* row = reinterpret_cast<const __nv_bfloat162*>(w + static_cast<size_t>(n) * K);
    float acc = 0.0f;
    for (int c = lane; c < K / 2; c += 32) {
      const float2 wf = __bfloat1622float2(row[c]);
      acc += wf.x * sx[2 * c] + wf.y * sx[2 * c + 1];
    }
    acc = warp_sum(acc);
    if (lane == 0) out[n] = acc + (bias ? __bfloat162float(bias[n]) : 0.0f);
  }
}

// ------------------------------------------------------------------ small ops
// timestep_embedding_fp32_kernel (cuda_kernels.cu:762-775), dim 256.
__global__ void timestep_embedding_kernel(float t, float* out, float max_period) {
  const int d = threadIdx.x;
  const int half_dim = 128;
  if (d >= half_dim) return;
  float freq = expf(-logf(max_period) * static_cast<float>(d) / static_cast<float>(half_dim));
  float angle = t * freq;
  out[d] = cosf(angle);
  out[half_dim + d] = sinf(angle);
}

// silu_fp32_kernel (cuda_kernels.cu:1881-1887).
__global__ void silu_kernel(const float* x, float* out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    float v = x[i];
    out[i] = v / (1.0f + expf(-v));
  }
}

// patchify_kernel (cuda_kernels.cu:1244-1272) for N latents, 2x2 patches.
__global__ void patchify_kernel(const __nv_bfloat16* __restrict__ in, __nv_bfloat16* __restrict__ out, int nb, int H,
                                int W, int p_lo, int n_loc) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int wp_n = W / 2;
  const long long total = static_cast<long long>(nb) * n_loc * kPatchDim;
  if (idx >= total) return;
  const int d = static_cast<int>(idx % kPatchDim);
  const long long rest = idx / kPatchDim;
  const int p = p_lo + static_cast<int>(rest % n_loc);
  const int n = static_cast<int>(rest / n_loc);
  const int hp = p / wp_n, wp = p % wp_n;
  const int c = d / 4, dh = (d % 4) / 2, dw = d % 2;
  out[idx] = in[(static_cast<long long>(n) * kOutCh + c) * H * W + static_cast<long long>(hp * 2 + dh) * W + wp * 2 + dw];
}

// FP32 proj_out rows -> BF16 (fp32_to_bf16) -> unpatchify_kernel
// (cuda_kernels.cu:1286-1312).
__global__ void unpatchify_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, int nb, int H, int W) {
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(nb) * kOutCh * H * W;
  if (idx >= total) return;
  const int w = static_cast<int>(idx % W);
  long long r = idx / W;
  const int h = static_cast<int>(r % H);
  r /= H;
  const int c = static_cast<int>(r % kOutCh);
  const int n = static_cast<int>(r / kOutCh);
  const int p = (h / 2) * (W / 2) + (w / 2);
  const int d = c * 4 + (h % 2) * 2 + (w % 2);
  out[idx] = __float2bfloat16(in[(static_cast<long long>(n) * (H / 2) * (W / 2) + p) * kPatchDim + d]);
}

// LayerNorm (no affine) + modulate, one CTA per row of 3072, 8 per thread.
__global__ void __launch_bounds__(384) layernorm_mod_kernel(const float* __restrict__ x, const float* __restrict__ shift,
                                                            const float* __restrict__ scale, float eps,
                                                            float* __restrict__ out_f32,
                                                            __nv_bfloat16* __restrict__ out_bf16) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const int c0 = threadIdx.x * 8;
  const float* xr = x + row * kDim + c0;
  float v[8];
  const float4 a = *reinterpret_cast<const float4*>(xr);
  const float4 b = *reinterpret_cast<const float4*>(xr + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  float s = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) s += v[e];
  const float mean = block_sum<384>(s, red) / kDim;
  float q = 0.0f;
#pragma unroll
  for (int e = 0; e < 8; ++e) q += (v[e] - mean) * (v[e] - mean);
  const float inv_std = rsqrtf(block_sum<384>(q, red) / kDim + eps);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = (v[e] - mean) * inv_std * (1.0f + scale[c0 + e]) + shift[c0 + e];
  if (out_f32) {
    float* o = out_f32 + row * kDim + c0;
    *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(o + 4) = make_float4(v[4], v[5], v[6], v[7]);
  } else {
    __nv_bfloat162 p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    *reinterpret_cast<uint4*>(out_bf16 + row * kDim + c0) = *reinterpret_cast<const uint4*>(p);
  }
}

// Generic-dimension LayerNorm + modulate for the op-level entry point.
__global__ void layernorm_mod_generic_kernel(const float* x, const float* shift, const float* scale, float* out, int dim,
                                             float eps) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const float* xr = x + row * dim;
  float s = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) s += xr[i];
  s = warp_sum(s);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) red[w] = s;
  __syncthreads();
  float mean = 0.0f;
  for (int i = 0; i < nw; ++i) mean += red[i];
  mean /= dim;
  __syncthreads();
  float q = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) q += (xr[i] - mean) * (xr[i] - mean);
  q = warp_sum(q);
  if (l == 0) red[w] = q;
  __syncthreads();
  float var = 0.0f;
  for (int i = 0; i < nw; ++i) var += red[i];
  const float inv_std = rsqrtf(var / dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    out[row * dim + i] = (xr[i] - mean) * inv_std * (1.0f + scale[i]) + shift[i];
}

// RMSNorm rows, FP32 in/out or BF16 in/out, BF16 weight
// (rms_norm_fp32_kernel :1656-1688; rms_norm_kernel :81-121).
template <typename T>
__global__ void rmsnorm_kernel(const T* x, const __nv_bfloat16* w, T* out, int dim, float eps) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const T* xr = x + row * dim;
  auto ld = [](const T* p, int i) -> float {
    if constexpr (sizeof(T) == 2) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    else return reinterpret_cast<const float*>(p)[i];
  };
  float s = 0.0f;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = ld(xr, i);
    s += v * v;
  }
  s = warp_sum(s);
  const int wi = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) red[wi] = s;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < nw; ++i) tot += red[i];
  const float rms = rsqrtf(tot / dim + eps);
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = ld(xr, i) * rms * __bfloat162float(w[i]);
    if constexpr (sizeof(T) == 2)
      reinterpret_cast<__nv_bfloat16*>(out)[row * dim + i] = __float2bfloat16(v);
    else
      reinterpret_cast<float*>(out)[row * dim + i] = v;
  }
}

}  // namespace

static int ok_or_err() { return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA; }

int qkv_post_launch(const QkvPostArgs& a, cudaStream_t stream) {
  if (a.Hl <= 0 || kHeads % a.Hl) return QI_ERR_ARG;
  const long long items = static_cast<long long>(a.nb) * (a.n_img_l + a.n_txt_l) * kHeads;
  if (items == 0) return QI_OK;
  const int threads = 256;
  const long long blocks = (items + 7) / 8;
  QkvPostArgs b = a;
  b.norm_dim = kHeadDim;  // run-time operands, as in rms_norm_fp32 (same division and add)
  b.eps = 1e-6f;
  qkv_post_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(b);
  return ok_or_err();
}

int gemv_i8_launch(const int8_t* act, const float* act_scale, int K, const GemvJob* jobs, int njobs,
                   cudaStream_t stream) {
  if (K % 16 || K > 12288) return QI_ERR_UNSUPPORTED;
  for (int j = 0; j < njobs; ++j) {
    const GemvJob& g = jobs[j];
    const long long N = g.N;
    long long blocks = (N + 7) / 8;
    if (blocks > 148 * 16) blocks = 148 * 16;
    gemv_i8_kernel<<<static_cast<unsigned>(blocks), 256, K, stream>>>(
        act, act_scale, K, g.w, g.sw, reinterpret_cast<const __nv_bfloat16*>(g.bias), g.out, N);
  }
  return ok_or_err();
}

int gemv_bf16_launch(const float* x, const void* w, const void* bias, float* out, int N, int K, cudaStream_t stream) {
  if (K % 2) return QI_ERR_UNSUPPORTED;
  int blocks = (N + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
  gemv_bf16_kernel<<<blocks, 256, K * sizeof(float), stream>>>(x, reinterpret_cast<const __nv_bfloat16*>(w),
                                                               reinterpret_cast<const __nv_bfloat16*>(bias), out, N, K);
  return ok_or_err();
}

int timestep_embedding_launch(float t, float* out256, cudaStream_t stream) {
  timestep_embedding_kernel<<<1, 128, 0, stream>>>(t, out256, 10000.0f);
  return ok_or_err();
}

int silu_launch(const float* x, float* out, int n, cudaStream_t stream) {
  silu_kernel<<<(n + 255) / 256, 256, 0, stream>>>(x, out, n);
  return ok_or_err();
}

int patchify_launch(const void* x_bf16, void* patches_bf16, int nb, int H, int W, int p_lo, int n_loc,
                    cudaStream_t stream) {
  if (p_lo < 0 || n_loc < 0 || p_lo + n_loc > (H / 2) * (W / 2)) return QI_ERR_ARG;
  const long long total = static_cast<long long>(nb) * n_loc * kPatchDim;
  if (total == 0) return QI_OK;
  patchify_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x_bf16), reinterpret_cast<__nv_bfloat16*>(patches_bf16), nb, H, W, p_lo,
      n_loc);
  return ok_or_err();
}

static unsigned grid_for(long long total) {
  long long g = (total + 255) / 256;
  if (g > 148LL * 16) g = 148LL * 16;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

int ulysses_gather_qkv_launch(const void* recv, void* qkvh, int nb, int Hl, int n_txt, const ShardMap& map,
                              cudaStream_t stream) {
  if (map.P < 1 || map.P > kMaxRanks || Hl <= 0) return QI_ERR_ARG;
  const long long S = map.txt_lo[map.P] + map.img_lo[map.P];
  const long long total = 3LL * nb * Hl * S * 16;
  ulysses_gather_qkv_kernel<<<grid_for(total), 256, 0, stream>>>(reinterpret_cast<const uint4*>(recv),
                                                                 reinterpret_cast<uint4*>(qkvh), nb, Hl, n_txt, map);
  return ok_or_err();
}

int ulysses_gather_o_launch(const void* recv, void* out, int nb, int Hl, int rank, const ShardMap& map,
                            cudaStream_t stream) {
  if (map.P < 1 || map.P > kMaxRanks || Hl <= 0 || rank < 0 || rank >= map.P) return QI_ERR_ARG;
  const long long total = static_cast<long long>(nb) * map.len(rank) * kHeads * 16;
  if (total == 0) return QI_OK;
  ulysses_gather_o_kernel<<<grid_for(total), 256, 0, stream>>>(reinterpret_cast<const uint4*>(recv),
                                                               reinterpret_cast<uint4*>(out), nb, Hl, rank, map);
  return ok_or_err();
}

int unpatchify_launch(const float* proj, void* out_bf16, int nb, int H, int W, cudaStream_t stream) {
  const long long total = static_cast<long long>(nb) * kOutCh * H * W;
  unpatchify_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(
      proj, reinterpret_cast<__nv_bfloat16*>(out_bf16), nb, H, W);
  return ok_or_err();
}

int layernorm_mod_launch(const float* x, const float* shift, const float* scale, int rows, int dim, float eps,
                         float* out_f32, void* out_bf16, cudaStream_t stream) {
  if (rows == 0) return QI_OK;
  if (dim == kDim) {
    layernorm_mod_kernel<<<rows, 384, 0, stream>>>(x, shift, scale, eps, out_f32,
                                                  reinterpret_cast<__nv_bfloat16*>(out_bf16));
  } else {
    if (!out_f32) return QI_ERR_UNSUPPORTED;
    layernorm_mod_generic_kernel<<<rows, 256, 0, stream>>>(x, shift, scale, out_f32, dim, eps);
  }
  return ok_or_err();
}

int rmsnorm_f32_launch(const float* x, const void* w, float* out, int rows, int dim, float eps, cudaStream_t stream) {
  if (rows == 0) return QI_OK;
  const int threads = dim >= 1024 ? 1024 : ((dim + 31) / 32) * 32;
  rmsnorm_kernel<float><<<rows, threads, 0, stream>>>(x, reinterpret_cast<const __nv_bfloat16*>(w), out, dim, eps);
  return ok_or_err();
}

int rmsnorm_bf16_launch(const void* x, const void* w, void* out, int rows, int dim, float eps, cudaStream_t stream) {
  if (rows == 0) return QI_OK;
  const int threads = dim >= 1024 ? 1024 : ((dim + 31) / 32) * 32;
  rmsnorm_kernel<__nv_bfloat16><<<rows, threads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<const __nv_bfloat16*>(w),
      reinterpret_cast<__nv_bfloat16*>(out), dim, eps);
  return ok_or_err();
}

}  // namespace qi

namespace qi {
namespace {
// Norm-preserving CFG + denoiser scaling + Euler (main.cu:210-288), one warp per
// 2x2 patch group of 64 elements (16 channels x 2 x 2): the group norms are warp
// reductions instead of the reference's global atomics.
__global__ void cfg_euler_kernel(float* __restrict__ x, const __nv_bfloat16* __restrict__ cond,
                                 const __nv_bfloat16* __restrict__ uncond, float cfg, float sigma, float dt, int H,
                                 int W, __nv_bfloat16* __restrict__ x_bf16) {
  const int groups = (H / 2) * (W / 2);
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= groups) return;
  const int lane = threadIdx.x & 31;
  const int hp = gw / (W / 2), wp = gw % (W / 2);
  long long idx[2];
  float c[2], u[2], cb[2];
  float cn = 0.0f, nn = 0.0f;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int d = lane * 2 + e;  // 0..63 = channel * 4 + dh * 2 + dw
    const int ch = d >> 2, dh = (d >> 1) & 1, dw = d & 1;
    idx[e] = (static_cast<long long>(ch) * H + hp * 2 + dh) * W + wp * 2 + dw;
    c[e] = __bfloat162float(cond[idx[e]]);
    u[e] = __bfloat162float(uncond[idx[e]]);
    cb[e] = u[e] + cfg * (c[e] - u[e]);
    cn += c[e] * c[e];
    nn += cb[e] * cb[e];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    cn += __shfl_xor_sync(0xffffffffu, cn, o);
    nn += __shfl_xor_sync(0xffffffffu, nn, o);
  }
  const float r = nn > 0.0f ? sqrtf(cn) / sqrtf(nn) : 1.0f;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const float v = cb[e] * r;
    const float xv = x[idx[e]];
    const float den = xv - sigma * v;
    const float xn = xv + (xv - den) / sigma * dt;
    x[idx[e]] = xn;
    x_bf16[idx[e]] = __float2bfloat16(xn);
  }
}
}  // namespace

int cfg_euler_launch(float* x, const void* cond, const void* uncond, float cfg, float sigma, float sigma_next, int H,
                     int W, void* x_bf16, cudaStream_t stream) {
  if ((H & 1) || (W & 1) || H <= 0 || W <= 0) return QI_ERR_ARG;
  const int groups = (H / 2) * (W / 2);
  cfg_euler_kernel<<<(groups + 7) / 8, 256, 0, stream>>>(
      x, reinterpret_cast<const __nv_bfloat16*>(cond), reinterpret_cast<const __nv_bfloat16*>(uncond), cfg, sigma,
      sigma_next - sigma, H, W, reinterpret_cast<__nv_bfloat16*>(x_bf16));
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

}  // namespace qi
