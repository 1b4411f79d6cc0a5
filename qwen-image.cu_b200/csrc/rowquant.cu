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
// Only the placement of the butterflies differs: each warp owns whole
// Hadamard blocks with a coalesced element layout and runs every stage in
// registers or warp shuffles; only the row statistics cross warps.
//
// The fused kernel also takes the producing op as its prologue:
//   kSrcLnMod: LayerNorm (no affine) + modulate of the FP32 residual stream
//              (layer_norm_modulate_fp32, cuda_kernels.cu:1799-1853), so the
//              modulated FP32 activation never goes to HBM;
//   kSrcF16:   the attention output rows (FP16, as the reference's half
//              output converted to float, sageattention_sm80.cu:888-894).
#include "qi_internal.h"
#include "sm100.cuh"

#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace qi {

namespace {

struct RowSegs {
  RowSeg s[2];
  int nseg;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// max that returns NaN if either input is NaN (fmaxf drops NaNs), flushing
// subnormal inputs like fmaxf under the build's fast-math flags.  For inputs
// without NaN it equals fmaxf, so the row maximum it gives is the reference's
// (fmaxf-based) unless the row holds a NaN, which it then reports.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.ftz.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float warp_max_nan(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// The quantizer's code for x = v * inv: the reference's
// clamp(__float2int_rn(x), -128, 127) (fwht_quantize_kernel,
// cuda_kernels.cu:2571-2575), as four bytes packed little-endian.
__device__ __forceinline__ uint32_t codes4_ref(float x0, float x1, float x2, float x3) {
  const int t0 = max(-128, min(127, __float2int_rn(x0))), t1 = max(-128, min(127, __float2int_rn(x1)));
  const int t2 = max(-128, min(127, __float2int_rn(x2))), t3 = max(-128, min(127, __float2int_rn(x3)));
  return __byte_perm(__byte_perm(t0, t1, 0x0040), __byte_perm(t2, t3, 0x0040), 0x5410);
}
// The same codes without the float-to-integer conversion unit, for rows whose
// scaled values are finite with |x| < 127.5 (no NaN in the row and a finite
// 127 / max): adding 1.5 * 2^23 rounds x to the nearest integer, ties to even
// (the rounding of __float2int_rn), and leaves it in the low mantissa bits in
// two's complement; no value reaches the clamp.  x must be the rounded
// product v * inv: the scalar __fmul_rn / __fadd_rn are never contracted into
// a fused multiply-add.  (Two-wide FP32 multiply and add were measured to
// differ here on exact ties, so this step stays scalar.)  Here for J float4s
// held as FP32 pairs, stored to dst[32 j].
template <int J>
__device__ __forceinline__ void dst_codes_fast(const uint64_t (&w)[J][2], float inv, uint32_t* dst) {
#pragma unroll
  for (int j = 0; j < J; ++j) {
    float x0, x1, x2, x3;
    f2unpack(w[j][0], x0, x1);
    f2unpack(w[j][1], x2, x3);
    const int t0 = __float_as_int(__fadd_rn(__fmul_rn(x0, inv), 12582912.0f));
    const int t1 = __float_as_int(__fadd_rn(__fmul_rn(x1, inv), 12582912.0f));
    const int t2 = __float_as_int(__fadd_rn(__fmul_rn(x2, inv), 12582912.0f));
    const int t3 = __float_as_int(__fadd_rn(__fmul_rn(x3, inv), 12582912.0f));
    dst[32 * j] = __byte_perm(__byte_perm(t0, t1, 0x0040), __byte_perm(t2, t3, 0x0040), 0x5410);
  }
}

// The reference's mean = sum / dim and inv_std = rsqrtf(var_sum / dim + eps)
// (cuda_kernels.cu:1827, 1847) under fast math: a division is a times the
// approximate reciprocal of b, and in the reference build the compiler fuses
// that product with the following + eps into one FMA.  Whether it does so
// depends on the surrounding code, so both are written out here as explicit
// instructions: measured against the reference's LayerNorm-quantizer codes,
// the fused form matches bit for bit and the separately rounded one does not
// (tens of flipped codes per million).
__device__ __forceinline__ float ln_mean(float sum, int dim) {
  float m;
  asm("div.approx.ftz.f32 %0, %1, %2;" : "=f"(m) : "f"(sum), "f"(static_cast<float>(dim)));
  return m;
}
__device__ __forceinline__ float ln_inv_std(float var_sum, int dim, float eps) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(static_cast<float>(dim)));
  return rsqrtf(__fmaf_rn(var_sum, r, eps));
}

// Sum over the 1024 threads of a reference reduction block in the order of
// its two-level shfl_down tree.  The lane stands for reference warp `lane`
// (threads 32 * lane + L, L = 0..31); part(q, p) gives the partials of threads
// L = 4q .. 4q + 3.  The warp's own tree (offsets 16, 8, 4 pair L with L + 16,
// L + 8, L + 4, i.e. q with q + 4, q + 2, q + 1 at the same L % 4; then
// offsets 2, 1 pair the components) runs in registers as
//   c[e] = ((p0 + p4) + (p2 + p6)) + ((p1 + p5) + (p3 + p7)),
//   warp sum = (c[0] + c[2]) + (c[1] + c[3]);
// the 32 warp sums then go through offsets 16 .. 1 across lanes.  The xor
// butterfly gives every lane the value the reference's lane 0 gets (each add
// is commutative).  The __syncwarp between the halves keeps the compiler from
// holding all eight float4 partials' operands in registers at once.
template <typename Part>
__device__ __forceinline__ float ref_block_tree(Part part) {
  auto quad = [&](int q0, float (&c)[4]) {  // (p[q0] + p[q0 + 4]) + (p[q0 + 2] + p[q0 + 6])
    float a[4], b[4];
    part(q0, a);
    part(q0 + 4, b);
#pragma unroll
    for (int e = 0; e < 4; ++e) a[e] = a[e] + b[e];
    float d[4];
    part(q0 + 2, d);
    part(q0 + 6, b);
#pragma unroll
    for (int e = 0; e < 4; ++e) c[e] = a[e] + (d[e] + b[e]);
  };
  float c0[4], c1[4];
  quad(0, c0);
  __syncwarp();
  quad(1, c1);
#pragma unroll
  for (int e = 0; e < 4; ++e) c0[e] = c0[e] + c1[e];
  float w = (c0[0] + c0[2]) + (c0[1] + c0[3]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
  return w;
}

// One row per CTA, NW warps per row; warp w owns the contiguous chunk
// [w*CH, (w+1)*CH) of CH = K/NW elements, which holds whole Hadamard blocks
// (had_block <= CH).  Lane l keeps float4 j at element w*CH + 128*j + 4*l, so
// every warp load and store is one contiguous 512 B (or 256/128 B) span, and
// the butterfly stages run on the element-index bits they pair:
//   half = 1, 2        -> the float4's components (registers)
//   half = 4 .. 64     -> lane bits (warp shuffles, partner lane ^ half/4)
//   half = 128 ..      -> register index bits (registers)
// in the reference's stage order.  Only the row statistics cross warps.
template <int K, int NW, int SRC>
__global__ void __launch_bounds__(NW * 32) rowquant_warp_kernel(RowSegs segs, int had_block, int8_t* __restrict__ codes,
                                                                float* __restrict__ scales, float eps, int dim) {
  constexpr int CH = K / NW;
  constexpr int J = CH / 128;
  static_assert(CH % 128 == 0, "chunk must be a multiple of 128");
  __shared__ float red[3][NW];

  const int row = blockIdx.x;
  const bool second = segs.nseg > 1 && row >= segs.s[0].rows;
  const void* in = second ? segs.s[1].in : segs.s[0].in;
  const long long ld = second ? segs.s[1].ld : segs.s[0].ld;
  const float* shift = second ? segs.s[1].shift : segs.s[0].shift;
  const float* scale = second ? segs.s[1].scale : segs.s[0].scale;
  const int local = second ? row - segs.s[0].rows : row;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int base = warp * CH + 4 * lane;

  // float4 j of this lane as two FP32 pairs: w[j][0] = (x0, x1), w[j][1] = (x2, x3)
  uint64_t w[J][2];
  if (SRC == kSrcF16) {
    const __half* src = reinterpret_cast<const __half*>(in) + static_cast<long long>(local) * ld + base;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const uint2 raw = *reinterpret_cast<const uint2*>(src + 128 * j);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      w[j][0] = f2pack(a.x, a.y);
      w[j][1] = f2pack(b.x, b.y);
    }
  } else {
    const float* src = reinterpret_cast<const float*>(in) + static_cast<long long>(local) * ld + base;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const ulonglong2 u = *reinterpret_cast<const ulonglong2*>(src + 128 * j);
      w[j][0] = u.x;
      w[j][1] = u.y;
    }
  }

  if constexpr (SRC == kSrcLnMod) {
    // Row statistics in the reference's own summation order, so that mean and
    // inv_std carry the same bits (layer_norm_modulate_fp32_kernel,
    // cuda_kernels.cu:1799-1853, launched with 1024 threads for dim 3072):
    // thread t sums x[t], x[t + 1024], x[t + 2048] in that order; each warp of
    // 32 threads reduces with shfl_down offsets 16, 8, 4, 2, 1; warp 0 reduces
    // the 32 warp sums the same way; mean = sum / dim.  The variance repeats
    // it on (x - mean)^2.  Here warp k holds chunk k (t = 128j + 4 lane + e),
    // so the three chunks go through shared memory and lane W of warp 0
    // replays reference warp W (threads 32W .. 32W + 31) in registers.
    static_assert(K == 3072 && NW == 3, "the reference-order statistics assume 3 chunks of 1024");
    __shared__ __align__(16) float xs[3][1152];  // t at t + 4 * (t / 32): conflict-free both ways
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int t = 128 * j + 4 * lane;
      *reinterpret_cast<ulonglong2*>(&xs[warp][t + 4 * (t >> 5)]) = make_ulonglong2(w[j][0], w[j][1]);
    }
    __syncthreads();
    if (warp == 0) {
      const int a0 = 36 * lane;  // padded offset of thread 32 * lane
      // thread partials of threads 32 * lane + 4q .. + 3, in the reference's
      // per-thread order: sum += x[t]; sum += x[t + 1024]; sum += x[t + 2048]
      // (components two at a time)
      auto sum_part = [&](int q, float (&o)[4]) {
        const ulonglong2 f0 = *reinterpret_cast<const ulonglong2*>(&xs[0][a0 + 4 * q]);
        const ulonglong2 f1 = *reinterpret_cast<const ulonglong2*>(&xs[1][a0 + 4 * q]);
        const ulonglong2 f2 = *reinterpret_cast<const ulonglong2*>(&xs[2][a0 + 4 * q]);
        f2unpack(f2add(f2add(f0.x, f1.x), f2.x), o[0], o[1]);
        f2unpack(f2add(f2add(f0.y, f1.y), f2.y), o[2], o[3]);
      };
      const float mean = ln_mean(ref_block_tree(sum_part), dim);
      const uint64_t mean2 = f2pack(mean, mean);
      // var_sum += v * v over the same elements, v = x - mean (the first
      // product's += onto 0 is the product itself)
      auto var_part = [&](int q, float (&o)[4]) {
        const ulonglong2 f0 = *reinterpret_cast<const ulonglong2*>(&xs[0][a0 + 4 * q]);
        const ulonglong2 f1 = *reinterpret_cast<const ulonglong2*>(&xs[1][a0 + 4 * q]);
        const ulonglong2 f2 = *reinterpret_cast<const ulonglong2*>(&xs[2][a0 + 4 * q]);
        const uint64_t x0[2] = {f0.x, f0.y}, x1[2] = {f1.x, f1.y}, x2[2] = {f2.x, f2.y};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          uint64_t d = f2sub(x0[k], mean2);
          uint64_t var_sum = f2mul(d, d);
          d = f2sub(x1[k], mean2);
          var_sum = f2fma(d, d, var_sum);
          d = f2sub(x2[k], mean2);
          var_sum = f2fma(d, d, var_sum);
          f2unpack(var_sum, o[2 * k], o[2 * k + 1]);
        }
      };
      const float inv_std = ln_inv_std(ref_block_tree(var_part), dim, eps);
      if (lane == 0) {
        red[0][0] = mean;
        red[1][0] = inv_std;
      }
    }
    __syncthreads();
    const float mean = red[0][0];
    const float inv_std = red[1][0];
    const uint64_t mean2 = f2pack(mean, mean), istd2 = f2pack(inv_std, inv_std), one2 = f2pack(1.0f, 1.0f);
    // this warp's chunk back from shared memory (not held in registers
    // across the statistics); (x - mean) * inv_std * (1 + scale) + shift with
    // the last multiply-add fused, as the reference build contracts it
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int t = 128 * j + 4 * lane;
      const ulonglong2 f = *reinterpret_cast<const ulonglong2*>(&xs[warp][t + 4 * (t >> 5)]);
      const ulonglong2 sc = __ldg(reinterpret_cast<const ulonglong2*>(scale + base + 128 * j));
      const ulonglong2 sh = __ldg(reinterpret_cast<const ulonglong2*>(shift + base + 128 * j));
      w[j][0] = f2fma(f2mul(f2sub(f.x, mean2), istd2), f2add(one2, sc.x), sh.x);
      w[j][1] = f2fma(f2mul(f2sub(f.y, mean2), istd2), f2add(one2, sc.y), sh.y);
    }
  }

  // half = 1: inside each pair; half = 2: the two pairs side by side
  if (had_block > 1) {
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float a, b;
        f2unpack(w[j][k], a, b);
        w[j][k] = f2pack(a + b, a - b);
      }
  }
  if (had_block > 2) {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const uint64_t a = w[j][0], b = w[j][1];
      w[j][0] = f2add(a, b);
      w[j][1] = f2sub(a, b);
    }
  }
  // half = 4 .. 64: across lanes
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    if (4 * m >= had_block) break;
    const float sgn = (lane & m) ? -1.0f : 1.0f;
    const uint64_t sgn2 = f2pack(sgn, sgn);
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        // lower lane: a + b = v + p; upper lane: a - b = p - v; one rounding each
        float lo, hi;
        f2unpack(w[j][k], lo, hi);
        const float plo = __shfl_xor_sync(0xffffffffu, lo, m), phi = __shfl_xor_sync(0xffffffffu, hi, m);
        w[j][k] = f2fma(w[j][k], sgn2, f2pack(plo, phi));
      }
  }
  // half = 128 ..: across registers
#pragma unroll
  for (int jm = 1; jm < J; jm <<= 1) {
    if (128 * jm >= had_block) break;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (j & jm) continue;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const uint64_t a = w[j][k], b = w[j | jm][k];
        w[j][k] = f2add(a, b);
        w[j | jm][k] = f2sub(a, b);
      }
    }
  }

  float mx = 0.0f;
  if (had_block > 1) {
    const float norm = rsqrtf(static_cast<float>(had_block));
    const uint64_t norm2 = f2pack(norm, norm);
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int k = 0; k < 2; ++k) w[j][k] = f2mul(w[j][k], norm2);
  }
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      float a, b;
      f2unpack(w[j][k], a, b);
      mx = fmax_nan(mx, fmax_nan(fabsf(a), fabsf(b)));
    }
  mx = warp_max_nan(mx);
  if (lane == 0) red[2][warp] = mx;
  __syncthreads();
  mx = red[2][0];
#pragma unroll
  for (int w2 = 1; w2 < NW; ++w2) mx = fmax_nan(mx, red[2][w2]);
  const bool nan_row = mx != mx;  // the same on every thread of the row
  if (nan_row) {  // the reference's maximum ignores NaNs
    mx = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float a, b;
        f2unpack(w[j][k], a, b);
        mx = fmaxf(mx, fmaxf(fabsf(a), fabsf(b)));
      }
    mx = warp_max(mx);
    if (lane == 0) red[0][warp] = mx;
    __syncthreads();
    mx = red[0][0];
#pragma unroll
    for (int w2 = 1; w2 < NW; ++w2) mx = fmaxf(mx, red[0][w2]);
  }
  if (threadIdx.x == 0) scales[row] = mx / 127.0f;
  const float inv = (mx > 0.0f) ? 127.0f / mx : 0.0f;
  uint32_t* dst = reinterpret_cast<uint32_t*>(codes + static_cast<long long>(row) * K + base);
  if (!nan_row && mx <= 3.40282347e38f && inv <= 3.40282347e38f) {
    dst_codes_fast(w, inv, dst);
  } else {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      float x0, x1, x2, x3;
      f2unpack(w[j][0], x0, x1);
      f2unpack(w[j][1], x2, x3);
      dst[32 * j] = codes4_ref(x0 * inv, x1 * inv, x2 * inv, x3 * inv);
    }
  }
}

// K = 12288, block 4096: one warp per 4096-block, lane l holding float4 j at
// element 128j + 4l (coalesced loads and stores).  Element-index bits 0-1 are
// the float4 components, bits 2-6 the lane, bits 7-11 the register index.
// Instead of 5 shuffle stages over 128 values per lane, the warp transposes
// its block through a private, XOR-swizzled 16 KB shared-memory tile so that
// bits 2-6 become register bits (lane L then holds elements 128L .. 128L+127),
// runs those stages in registers, and transposes back for bits 7-11; the
// stage order (half = 1, 2, 4, ..., 2048) and every butterfly's operands are
// those of the reference.
// Persistent: each CTA takes rows blockIdx.x, blockIdx.x + gridDim.x, ...; as
// soon as a warp has copied its 16 KB slice of a row from shared memory into
// registers, it issues the bulk copy of its slice of the CTA's next row, so
// the HBM latency of row r+1 overlaps the butterflies of row r.
__global__ void __launch_bounds__(96) rowquant_b4096_kernel(RowSegs segs, int had_block, int8_t* __restrict__ codes,
                                                            float* __restrict__ scales, int rows) {
  constexpr int K = 12288, NW = 3, J = 32;
  // [NW][32 rows][32 float4] transpose tiles, swizzled: (row, col) at row*32 + (col ^ row);
  // then [NW][1024 float4] prefetch slices
  extern __shared__ float4 tile4[];
  __shared__ float red[2][NW];
  __shared__ float red_nan[NW];
  __shared__ __align__(8) uint64_t pbar[NW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int base = warp * 4096 + 4 * lane;
  float4* tw = tile4 + warp * 1024;
  float4* pw = tile4 + NW * 1024 + warp * 1024;
  auto slice_of = [&](int r) {
    const bool second = segs.nseg > 1 && r >= segs.s[0].rows;
    const void* in = second ? segs.s[1].in : segs.s[0].in;
    const long long ld = second ? segs.s[1].ld : segs.s[0].ld;
    const int local = second ? r - segs.s[0].rows : r;
    return reinterpret_cast<const float*>(in) + static_cast<long long>(local) * ld + warp * 4096;
  };
  auto prefetch = [&](int r) {
    mbar_expect_tx(&pbar[warp], 16384);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(pw)),
        "l"(slice_of(r)), "r"(16384), "r"(smem_u32(&pbar[warp]))
        : "memory");
  };
  if (lane == 0) {
    mbar_init(&pbar[warp], 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (lane == 0 && static_cast<int>(blockIdx.x) < rows) prefetch(blockIdx.x);
  uint32_t phase = 0;
  int it = 0;
#pragma unroll 1
  for (int row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
  // the bulk copy needs no other work to finish; the limit only bounds the spin
  {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_test_wait(&pbar[warp], phase) && global_timer_ns() - t0 < kWaitLimitNs) {
    }
    phase ^= 1u;
  }
  // float4 j as two FP32 pairs: w[j][0] = (x0, x1), w[j][1] = (x2, x3)
  uint64_t w[J][2];
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const ulonglong2 u = reinterpret_cast<const ulonglong2*>(pw)[32 * j + lane];
    w[j][0] = u.x;
    w[j][1] = u.y;
  }
  fence_proxy_async_smem();  // every lane's reads of the slice come before the copy overwrites it
  __syncwarp();
  if (lane == 0 && row + static_cast<int>(gridDim.x) < rows) prefetch(row + gridDim.x);
  auto stage_components = [&]() {
    // half = 1: inside each pair, (x0, x1) -> (x0 + x1, x0 - x1)
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float a, b;
        f2unpack(w[j][k], a, b);
        w[j][k] = f2pack(a + b, a - b);
      }
    // half = 2: (x0, x2) and (x1, x3) side by side in the two pairs
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const uint64_t a = w[j][0], b = w[j][1];
      w[j][0] = f2add(a, b);
      w[j][1] = f2sub(a, b);
    }
  };
  auto stages_registers = [&]() {  // register-index bits, lowest first
#pragma unroll
    for (int jm = 1; jm < J; jm <<= 1)
#pragma unroll
      for (int j = 0; j < J; ++j) {
        if (j & jm) continue;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint64_t a = w[j][k], b = w[j | jm][k];
          w[j][k] = f2add(a, b);
          w[j | jm][k] = f2sub(a, b);
        }
      }
  };
  // transpose: (row j, col lane) <-> (row lane, col j) of the 32 x 32 float4 grid
  ulonglong2* tw2 = reinterpret_cast<ulonglong2*>(tw);
  auto transpose = [&]() {
#pragma unroll
    for (int j = 0; j < J; ++j) tw2[j * 32 + (lane ^ j)] = make_ulonglong2(w[j][0], w[j][1]);
    __syncwarp();
#pragma unroll
    for (int c = 0; c < J; ++c) {
      const ulonglong2 u = tw2[lane * 32 + (c ^ lane)];
      w[c][0] = u.x;
      w[c][1] = u.y;
    }
    __syncwarp();
  };
  stage_components();  // half = 1, 2
  transpose();         // lane <- bits 7-11, register <- bits 2-6
  stages_registers();  // half = 4 .. 64
  transpose();         // back: lane <- bits 2-6, register <- bits 7-11
  stages_registers();  // half = 128 .. 2048

  const float norm = rsqrtf(static_cast<float>(had_block));  // had_block == 4096, evaluated at run time
  const uint64_t norm2 = f2pack(norm, norm);
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < J; ++j)
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      w[j][k] = f2mul(w[j][k], norm2);
      float a, b;
      f2unpack(w[j][k], a, b);
      mx = fmax_nan(mx, fmax_nan(fabsf(a), fabsf(b)));
    }
  mx = warp_max_nan(mx);
  if (lane == 0) red[it & 1][warp] = mx;  // double buffered: the next row's writes go to the other slot
  __syncthreads();
  mx = fmax_nan(fmax_nan(red[it & 1][0], red[it & 1][1]), red[it & 1][2]);
  const bool nan_row = mx != mx;  // the same on every thread of the row
  if (nan_row) {  // the reference's maximum ignores NaNs
    mx = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float a, b;
        f2unpack(w[j][k], a, b);
        mx = fmaxf(mx, fmaxf(fabsf(a), fabsf(b)));
      }
    mx = warp_max(mx);
    if (lane == 0) red_nan[warp] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(red_nan[0], red_nan[1]), red_nan[2]);
  }
  if (threadIdx.x == 0) scales[row] = mx / 127.0f;
  const float inv = (mx > 0.0f) ? 127.0f / mx : 0.0f;
  uint32_t* dst = reinterpret_cast<uint32_t*>(codes + static_cast<long long>(row) * K + base);
  if (!nan_row && mx <= 3.40282347e38f && inv <= 3.40282347e38f) {
    dst_codes_fast(w, inv, dst);
  } else {
#pragma unroll
    for (int j = 0; j < J; ++j) {
      float x0, x1, x2, x3;
      f2unpack(w[j][0], x0, x1);
      f2unpack(w[j][1], x2, x3);
      dst[32 * j] = codes4_ref(x0 * inv, x1 * inv, x2 * inv, x3 * inv);
    }
  }
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

template <int K, int NW, int SRC>
int launch_warp(const RowSegs& segs, int rows, int had_block, int8_t* codes, float* scales, float eps,
                cudaStream_t stream) {
  if (had_block > K / NW) return QI_ERR_UNSUPPORTED;
  rowquant_warp_kernel<K, NW, SRC><<<rows, NW * 32, 0, stream>>>(segs, had_block, codes, scales, eps, K);
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
    if (src == kSrcLnMod && ((reinterpret_cast<uintptr_t>(segs[i].shift) & 15) || (reinterpret_cast<uintptr_t>(segs[i].scale) & 15)))
      return QI_ERR_ALIGN;
    if (src == kSrcLnMod && (!segs[i].shift || !segs[i].scale)) return QI_ERR_ARG;
  }
  s.nseg = nseg;
  if (rows == 0) return QI_OK;
  if (K == 3072 && src == kSrcF32) return launch_warp<3072, 3, kSrcF32>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 3072 && src == kSrcF16) return launch_warp<3072, 3, kSrcF16>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 3072 && src == kSrcLnMod)
    return launch_warp<3072, 3, kSrcLnMod>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 12288 && src == kSrcF32 && had_block == 4096) {
    const int smem = 2 * 3 * 1024 * 16;  // three 16 KB transpose tiles + three 16 KB prefetch slices
    static unsigned long long attr_done = 0;
    if (smem_optin(reinterpret_cast<const void*>(rowquant_b4096_kernel), smem, &attr_done) != QI_OK)
      return QI_ERR_CUDA;
    const int grid = rows < 2 * device_num_sms() ? rows : 2 * device_num_sms();
    rowquant_b4096_kernel<<<grid, 96, smem, stream>>>(s, had_block, codes, scales, rows);
    return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
  }
  if (K == 12288 && src == kSrcF32)
    return launch_warp<12288, 3, kSrcF32>(s, rows, had_block, codes, scales, eps, stream);
  if (K == 256 && src == kSrcF32) return launch_warp<256, 1, kSrcF32>(s, rows, had_block, codes, scales, eps, stream);
  return QI_ERR_UNSUPPORTED;
}

int fwht_quant_generic(const void* in, int in_bf16, int M, int K, int had_block, int8_t* codes, float* scales,
                       cudaStream_t stream) {
  if (M < 0 || K <= 0 || K > 12288) return QI_ERR_UNSUPPORTED;
  if (had_block < 1 || (had_block & (had_block - 1)) || K % had_block) return QI_ERR_ARG;
  if (M == 0) return QI_OK;
  const int smem = (K + 32) * static_cast<int>(sizeof(float));
  static unsigned long long attr_done = 0;
  if (smem_optin(reinterpret_cast<const void*>(fwht_quant_generic_kernel), (12288 + 32) * 4, &attr_done) != QI_OK)
    return QI_ERR_CUDA;
  int threads = K < 1024 ? ((K + 31) / 32) * 32 : 1024;
  fwht_quant_generic_kernel<<<M, threads, smem, stream>>>(in, in_bf16, K, had_block, codes, scales);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

}  // namespace qi
