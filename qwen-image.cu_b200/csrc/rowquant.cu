// rowquant.cu -- block Walsh-Hadamard transform + per-row symmetric INT8.
//
// The reference rotates every activation row with a block FWHT (block
// B = K & -K, cuda_kernels.cuh:253) and quantizes it per token
// (fwht_quantize_kernel, cuda_kernels.cu:2493-2577); weights get the same
// rotation and per-row quantization at load time (quantize_weight_tensor,
// cuda_kernels.cu:2830-2862).  Codes and scales here are bit-exact with the
// reference because every element sees the same sequence of IEEE operations:
//   * butterfly stages in the order half = 1, 2, 4, ... with (a, b) ->
//     (a + b, a - b), where a is the lower index;
//   * normalisation by rsqrtf((float)B) after the butterflies, evaluated at
//     run time (never constant-folded) with the same fast-math flags;
//   * scale = max / 127, inverse = 127 / max, code = sat(__float2int_rn(v * inv)).
// Only the placement of the butterflies differs: the fused kernel keeps EPT
// consecutive elements per thread in registers (stages < EPT), exchanges
// with warp shuffles (stages < 32 * EPT) and goes through shared memory only
// for the widest stages, instead of running every stage in shared memory.
//
// The fused kernel also takes the producing op as its prologue:
//   kSrcLnMod: LayerNorm (no affine) + modulate of the FP32 residual stream
//              (layer_norm_modulate_fp32, cuda_kernels.cu:1799-1853), so the
//              modulated FP32 activation never goes to HBM;
//   kSrcF16:   the attention output rows (FP16, as the reference's half
//              output converted to float, sageattention_sm80.cu:888-894).
#include "qi_internal.h"

#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace qi {

namespace {

struct RowSegs {
  RowSeg s[2];
  int nseg;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
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
template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = v;
  __syncthreads();
  float r = (l < NT / 32) ? red[l] : 0.0f;
  r = warp_max(r);
  __syncthreads();
  return r;
}

template <int K, int EPT, int SRC>
__global__ void __launch_bounds__(K / EPT) rowquant_fused_kernel(RowSegs segs, int had_block, int8_t* __restrict__ codes,
                                                                 float* __restrict__ scales, float eps) {
  constexpr int NT = K / EPT;
  extern __shared__ float xs[];  // K floats (wide stages) + 32 (reductions)
  float* red = xs + K;

  int row = blockIdx.x;
  const bool second = segs.nseg > 1 && row >= segs.s[0].rows;
  RowSeg sg;
  sg.in = second ? segs.s[1].in : segs.s[0].in;
  sg.ld = second ? segs.s[1].ld : segs.s[0].ld;
  sg.shift = second ? segs.s[1].shift : segs.s[0].shift;
  sg.scale = second ? segs.s[1].scale : segs.s[0].scale;
  const int local = second ? row - segs.s[0].rows : row;
  const int t = threadIdx.x;
  const int c0 = t * EPT;

  float v[EPT];
  if (SRC == kSrcF16) {
    const __half* in = reinterpret_cast<const __half*>(sg.in) + static_cast<long long>(local) * sg.ld + c0;
#pragma unroll
    for (int e = 0; e < EPT; e += 8) {
      uint4 raw = *reinterpret_cast<const uint4*>(in + e);
      const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __half22float2(h2[j]);
        v[e + 2 * j] = f.x;
        v[e + 2 * j + 1] = f.y;
      }
    }
  } else {
    const float* in = reinterpret_cast<const float*>(sg.in) + static_cast<long long>(local) * sg.ld + c0;
#pragma unroll
    for (int e = 0; e < EPT; e += 4) {
      float4 f = *reinterpret_cast<const float4*>(in + e);
      v[e] = f.x;
      v[e + 1] = f.y;
      v[e + 2] = f.z;
      v[e + 3] = f.w;
    }
  }

  if (SRC == kSrcLnMod) {
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < EPT; ++e) s += v[e];
    const float mean = block_sum<NT>(s, red) / K;
    float q = 0.0f;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      float d = v[e] - mean;
      q += d * d;
    }
    const float inv_std = rsqrtf(block_sum<NT>(q, red) / K + eps);
#pragma unroll
    for (int e = 0; e < EPT; e += 4) {
      float4 sc = __ldg(reinterpret_cast<const float4*>(sg.scale + c0 + e));
      float4 sh = __ldg(reinterpret_cast<const float4*>(sg.shift + c0 + e));
      v[e + 0] = (v[e + 0] - mean) * inv_std * (1.0f + sc.x) + sh.x;
      v[e + 1] = (v[e + 1] - mean) * inv_std * (1.0f + sc.y) + sh.y;
      v[e + 2] = (v[e + 2] - mean) * inv_std * (1.0f + sc.z) + sh.z;
      v[e + 3] = (v[e + 3] - mean) * inv_std * (1.0f + sc.w) + sh.w;
    }
  }

  // Butterfly stages, lowest first.  Register stages:
#pragma unroll
  for (int half = 1; half < EPT; half <<= 1) {
    if (half >= had_block) break;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      if ((e & half) == 0) {
        float a = v[e], b = v[e + half];
        v[e] = a + b;
        v[e + half] = a - b;
      }
    }
  }
  // Warp-shuffle stages (partner thread = t ^ (half / EPT)):
#pragma unroll
  for (int half = EPT; half < 32 * EPT; half <<= 1) {
    if (half >= had_block) break;
    const int m = half / EPT;
    const bool upper = (t & m) != 0;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      float p = __shfl_xor_sync(0xffffffffu, v[e], m);
      v[e] = upper ? (p - v[e]) : (v[e] + p);
    }
  }
  // Shared-memory stages:
  for (int half = 32 * EPT; half < had_block; half <<= 1) {
#pragma unroll
    for (int e = 0; e < EPT; e += 4)
      *reinterpret_cast<float4*>(xs + c0 + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
    __syncthreads();
    const bool upper = (c0 & half) != 0;
    const int pc = c0 ^ half;
#pragma unroll
    for (int e = 0; e < EPT; e += 4) {
      float4 p = *reinterpret_cast<const float4*>(xs + pc + e);
      v[e + 0] = upper ? (p.x - v[e + 0]) : (v[e + 0] + p.x);
      v[e + 1] = upper ? (p.y - v[e + 1]) : (v[e + 1] + p.y);
      v[e + 2] = upper ? (p.z - v[e + 2]) : (v[e + 2] + p.z);
      v[e + 3] = upper ? (p.w - v[e + 3]) : (v[e + 3] + p.w);
    }
    __syncthreads();
  }

  float mx = 0.0f;
  if (had_block > 1) {
    const float norm = rsqrtf(static_cast<float>(had_block));
#pragma unroll
    for (int e = 0; e < EPT; ++e) v[e] *= norm;
  }
#pragma unroll
  for (int e = 0; e < EPT; ++e) mx = fmaxf(mx, fabsf(v[e]));
  mx = block_max<NT>(mx, red);
  if (t == 0) scales[row] = mx / 127.0f;
  const float inv = (mx > 0.0f) ? 127.0f / mx : 0.0f;

  int8_t q[EPT];
#pragma unroll
  for (int e = 0; e < EPT; ++e) {
    int vi = __float2int_rn(v[e] * inv);
    vi = max(-128, min(127, vi));
    q[e] = static_cast<int8_t>(vi);
  }
  int8_t* dst = codes + static_cast<long long>(row) * K + c0;
  if (EPT == 8) {
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(q);
  } else {
#pragma unroll
    for (int e = 0; e < EPT; e += 16) *reinterpret_cast<uint4*>(dst + e) = *reinterpret_cast<const uint4*>(q + e);
  }
}

// Generic version: the whole row in shared memory, every stage over all
// pairs (the structure of fwht_quantize_kernel / fwht_inplace_kernel).
__global__ void fwht_quant_generic_kernel(const void* __restrict__ in, int in_bf16, int K, int had_block,
                                          int8_t* __restrict__ codes, float* __restrict__ scales) {
  extern __shared__ float sm[];
  float* red = sm + K;
  const int row = blockIdx.x;
  const long long base = static_cast<long long>(row) * K;
  for (int i = threadIdx.x; i < K; i += blockDim.x)
    sm[i] = in_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(in)[base + i])
                    : reinterpret_cast<const float*>(in)[base + i];
  __syncthreads();
  if (had_block > 1) {
    const int per_block = had_block / 2;
    const int total = (K / had_block) * per_block;
    for (int half = 1; half < had_block; half <<= 1) {
      const int full = half << 1;
      for (int p = threadIdx.x; p < total; p += blockDim.x) {
        const int blk = p / per_block;
        const int lp = p - blk * per_block;
        const int g = lp / half;
        const int w = lp - g * half;
        const int ia = blk * had_block + g * full + w;
        const int ib = ia + half;
        float a = sm[ia], b = sm[ib];
        sm[ia] = a + b;
        sm[ib] = a - b;
      }
      __syncthreads();
    }
    const float norm = rsqrtf(static_cast<float>(had_block));
    for (int i = threadIdx.x; i < K; i += blockDim.x) sm[i] *= norm;
  }
  float mx = 0.0f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(sm[i]));
  mx = warp_max(mx);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) red[w] = mx;
  __syncthreads();
  if (w == 0) {
    float r = (l < static_cast<int>((blockDim.x + 31) / 32)) ? red[l] : 0.0f;
    r = warp_max(r);
    if (l == 0) red[0] = r;
  }
  __syncthreads();
  mx = red[0];
  if (threadIdx.x == 0) scales[row] = mx / 127.0f;
  const float inv = (mx > 0.0f) ? 127.0f / mx : 0.0f;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    int vi = __float2int_rn(sm[i] * inv);
    vi = max(-128, min(127, vi));
    codes[base + i] = static_cast<int8_t>(vi);
  }
}

template <int K, int EPT, int SRC>
int launch_fused(const RowSegs& segs, int rows, int had_block, int8_t* codes, float* scales, float eps,
                 cudaStream_t stream) {
  const int smem = (K + 32) * static_cast<int>(sizeof(float));
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(rowquant_fused_kernel<K, EPT, SRC>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return QI_ERR_CUDA;
    attr = true;
  }
  rowquant_fused_kernel<K, EPT, SRC><<<rows, K / EPT, smem, stream>>>(segs, had_block, codes, scales, eps);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

}  // namespace

int rowquant_launch(int src, int K, int had_block, const RowSeg* segs, int nseg, int8_t* codes, float* scales,
                    float eps, cudaStream_t stream) {
  if (nseg < 1 || nseg > 2) return QI_ERR_ARG;
  if (had_block < 1 || (had_block & (had_block - 1)) || K % had_block) return QI_ERR_ARG;
  RowSegs s;
  memset(&s, 0, sizeof(s));
  int rows = 0;
  for (int i = 0; i < nseg; ++i) {
    s.s[i] = segs[i];
    rows += segs[i].rows;
    if (reinterpret_cast<uintptr_t>(segs[i].in) & 15) return QI_ERR_ALIGN;
    if (segs[i].ld % 8) return QI_ERR_ALIGN;
    if (src == kSrcLnMod && (!segs[i].shift || !segs[i].scale)) return QI_ERR_ARG;
  }
  s.nseg = nseg;
  if (rows == 0) return QI_OK;
  if (K == 3072 && src == kSrcF32) return launch_fused<3072, 8, kSrcF32>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 3072 && src == kSrcF16) return launch_fused<3072, 8, kSrcF16>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 3072 && src == kSrcLnMod)
    return launch_fused<3072, 8, kSrcLnMod>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 12288 && src == kSrcF32)
    return launch_fused<12288, 16, kSrcF32>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 256 && src == kSrcF32) return launch_fused<256, 8, kSrcF32>(s, rows, had_block, codes, scales, eps, stream);
  return QI_ERR_UNSUPPORTED;
}

int fwht_quant_generic(const void* in, int in_bf16, int M, int K, int had_block, int8_t* codes, float* scales,
                       cudaStream_t stream) {
  if (M < 0 || K <= 0 || K > 12288) return QI_ERR_UNSUPPORTED;
  if (had_block < 1 || (had_block & (had_block - 1)) || K % had_block) return QI_ERR_ARG;
  if (M == 0) return QI_OK;
  const int smem = (K + 32) * static_cast<int>(sizeof(float));
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(fwht_quant_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (12288 + 32) * 4) != cudaSuccess)
      return QI_ERR_CUDA;
    attr = true;
  }
  int threads = K < 1024 ? ((K + 31) / 32) * 32 : 1024;
  fwht_quant_generic_kernel<<<M, threads, smem, stream>>>(in, in_bf16, K, had_block, codes, scales);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

}  // namespace qi
