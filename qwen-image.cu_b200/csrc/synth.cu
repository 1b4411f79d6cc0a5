// synth.cu -- seeded synthetic tensors on the device.
//
// The benchmark configurations call for seeded N(0, s^2) weights and
// activations (the reference ships no checkpoints or fixtures for this path).
// Value i of a tensor with seed s: split-mix hashes of (mix(s) + 2i) and
// (mix(s) + 2i + 1) give four 24-bit uniforms; their centred sum, converted to
// float once and multiplied by sqrt(3)/2^24, has unit variance (Irwin-Hall,
// |z| <= 3.46).  Then z * scale (+ offset) as separate IEEE roundings, so a
// host implementation of the same formula yields the same bits.
#include "qi_internal.h"

#include <cuda_bf16.h>

namespace qi {

namespace {

__host__ __device__ __forceinline__ uint64_t sm64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

__device__ __forceinline__ float unit_normal(uint64_t sm, long long i) {
  const uint64_t h1 = sm64(sm + 2ull * static_cast<uint64_t>(i));
  const uint64_t h2 = sm64(sm + 2ull * static_cast<uint64_t>(i) + 1ull);
  const uint64_t m24 = 0xFFFFFFull;
  const long long s = static_cast<long long>(h1 & m24) + static_cast<long long>((h1 >> 24) & m24) +
                      static_cast<long long>(h2 & m24) + static_cast<long long>((h2 >> 24) & m24);
  const int c = static_cast<int>(s - 33554430ll);
  return __fmul_rn(__int2float_rn(c), 0x1.bb67aep-24f);
}

__global__ void synth_kernel(uint64_t sm, long long n, float scale, float offset, void* out, int kind) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    float v = __fmul_rn(unit_normal(sm, i), scale);
    if (offset != 0.0f) v = __fadd_rn(v, offset);
    if (kind == 0)
      reinterpret_cast<float*>(out)[i] = v;
    else
      reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  }
}

}  // namespace

int synth_launch(uint64_t seed, long long n, float scale, float offset, void* out, int bf16, cudaStream_t stream) {
  if (n <= 0) return QI_OK;
  long long blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  synth_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(sm64(seed), n, scale, offset, out, bf16 ? 1 : 0);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

uint64_t synth_seed_for(uint64_t base, const char* name) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (const unsigned char* p = reinterpret_cast<const unsigned char*>(name); *p; ++p) {
    h ^= *p;
    h *= 0x100000001b3ull;
  }
  return sm64(base ^ h);
}

}  // namespace qi
