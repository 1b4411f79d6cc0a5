// noalloc.cu -- qi_linear_i8_f32in_noalloc: the FP32-input W8A8 linear
// (block FWHT + per-token INT8 quantisation, then the tcgen05 INT8 GEMM, or
// the GEMV for a single row) with its scratch in a fixed, file-scope device
// array instead of memory the library allocates.
//
// Who needs it: a caller that must not allocate device memory once it is
// running -- a server that hands all of HBM to its own pool at start-up (a
// cudaMalloc then fails), or a step loop that cannot take cudaMalloc's
// implicit device-wide synchronisation.  qi_linear_i8_f32in instead grows a
// per-device workspace with cudaMalloc on first use and whenever a call needs
// more.  This entry point has no counterpart in the reference.
#include <mutex>

#include "qi_internal.h"

namespace {

// Scratch layout (bytes): [0, 256) error word of the GEMM's bounded waits,
// [256, 256 + 4 * QI_NOALLOC_MAX_ROWS) per-token scales, then the INT8 codes.
constexpr size_t kErrBytes = 256;
constexpr size_t kScalesOff = kErrBytes;
constexpr size_t kCodesOff = kScalesOff + 4 * static_cast<size_t>(QI_NOALLOC_MAX_ROWS);
constexpr size_t kScratchBytes = kCodesOff + static_cast<size_t>(QI_NOALLOC_MAX_CODES);
static_assert(kCodesOff % 256 == 0, "codes must stay 256-byte aligned");

// Zero at module load.  The error word is sticky: a GEMM wait that gives up
// records its code there (only if the word is still zero; the kernels never
// read it back) and it stays until qi_linear_i8_f32in_noalloc_check reads and
// clears it.  Codes and scales are fully overwritten by every call.
__device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
unsigned char* g_scratch_addr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};

// One-time setup per device, with that device current: the scratch array's
// device address and the SM count.  Only the address is ever given to a
// kernel.
int setup(int dev, unsigned char** scratch, int* num_sms) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return QI_ERR_CUDA;
    const int sms = qi::device_num_sms();
    if (sms <= 0) return QI_ERR_CUDA;
    g_num_sms[dev] = sms;
    g_scratch_addr[dev] = static_cast<unsigned char*>(p);
  }
  *scratch = g_scratch_addr[dev];
  *num_sms = g_num_sms[dev];
  return QI_OK;
}

// The scratch address on the current device if a call has set it up there,
// else null.
unsigned char* scratch_if_set_up(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  *dev_out = dev;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  return g_scratch_addr[dev];
}

inline bool misaligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; }

}  // namespace

extern "C" int qi_linear_i8_f32in_noalloc_check(void) {
  int dev = 0;
  unsigned char* scratch = scratch_if_set_up(&dev);
  if (!scratch) return QI_OK;  // no call has run on this device
  if (cudaDeviceSynchronize() != cudaSuccess) return QI_ERR_CUDA;
  int h = 0;
  if (cudaMemcpy(&h, scratch, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return QI_ERR_CUDA;
  if (h && cudaMemset(scratch, 0, sizeof(int)) != cudaSuccess) return QI_ERR_CUDA;
  return h ? QI_ERR_DEVICE : QI_OK;
}

extern "C" int qi_linear_i8_f32in_noalloc_selftest(int limit_us, void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QI_ERR_CUDA;
  unsigned char* scratch = nullptr;
  int num_sms = 0;
  const int st = setup(dev, &scratch, &num_sms);
  if (st != QI_OK) return st;
  return qi::selftest_wait_timeout(reinterpret_cast<int*>(scratch), limit_us, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int qi_linear_i8_f32in_noalloc(const float* x, int M, int K, const int8_t* w, const float* w_scales, int N,
                                          const void* bias_bf16, int apply_gelu, float* out, void* stream) {
  if (!x || !w || !w_scales || !out || M < 0 || K <= 0 || N <= 0) return QI_ERR_ARG;
  if (M > QI_NOALLOC_MAX_ROWS || static_cast<long long>(M) * K > QI_NOALLOC_MAX_CODES || K > 12288)
    return QI_ERR_UNSUPPORTED;
  // everything the quantizer and the GEMM / GEMV launchers would reject, before
  // anything is enqueued or the shared scratch is touched
  const bool gemv = M == 1 && !apply_gelu;
  if (K % 16 != 0 || (!gemv && N % 32 != 0)) return QI_ERR_ARG;
  if (misaligned(w) || misaligned(w_scales) || (!gemv && misaligned(out))) return QI_ERR_ALIGN;
  if (M == 0) return QI_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return QI_ERR_CUDA;
  unsigned char* scratch = nullptr;
  int num_sms = 0;
  const int st = setup(dev, &scratch, &num_sms);
  if (st != QI_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* err = reinterpret_cast<int*>(scratch);
  float* act_scales = reinterpret_cast<float*>(scratch + kScalesOff);
  int8_t* act = reinterpret_cast<int8_t*>(scratch + kCodesOff);
  const int qst = qi_fwht_quantize(x, M, K, K & (-K), act, act_scales, stream);
  if (qst != QI_OK) return qst;
  if (gemv) {
    qi::GemvJob j{w, w_scales, bias_bf16, out, N};
    return qi::gemv_i8_launch(act, act_scales, K, &j, 1, s);
  }
  qi::GemmDesc d{act, act_scales, w, w_scales, bias_bf16, out, nullptr, M, N, K, N};
  return qi::gemm_i8_launch(&d, 1, apply_gelu ? qi::kEpiGelu : qi::kEpiStore, s, err, num_sms);
}
