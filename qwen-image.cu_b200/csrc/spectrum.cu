// spectrum.cu -- Spectrum feature forecasting for skipped denoising steps.
//
// The reference (cuda_kernels.cu:5859-6333, driven from main.cu:640-748,
// 877-885) keeps the final image hidden state of every actual forward and, on
// a skipped step, predicts it as a blend of
//   * a ridge-regularised fit of Chebyshev polynomials T_0..T_M of the step
//     index (mapped affinely onto [-1, 1] over the stored steps), evaluated at
//     the target step: C = (X^T X + lambda I)^-1 X^T H, pred = row(target) C;
//   * a first-order Taylor extrapolation from the last two states:
//     h_i + k (h_i - h_{i-1}), k = (target - t_i) / max(t_i - t_{i-1}, 1e-6);
//   out = (1 - blend) taylor + blend cheb.
// The reference's spectrum_init (cuda_kernels.cu:6168-6196) sizes its buffers
// from its max_order argument but never stores it, so its fit always uses the
// default SpectrumState::max_order = 4 (T_0..T_4), and below 4 spectrum_predict
// writes past those buffers.  Here the order given is the order used; order 4
// (the default of the reference's --spectrum-order) reproduces the reference.
// Both parts are linear in the stored states, so the prediction is
// out = sum_k w_k H_k with K scalar weights: w_cheb = X (X^T X + lambda I)^-1
// row(target) (a (M+1) x (M+1) solve), w_taylor on the last two states.  The
// weights are computed on the host in double precision and passed to one
// kernel as parameters; the kernel streams the K stored states once (HBM
// bound: 4 K bytes per output element), instead of the reference's SGEMMs,
// Cholesky factorisation and separate prediction / blend passes.
#include "qi_internal.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

namespace qi {
namespace {

constexpr int kMaxHistory = 128;  // weights passed by value to the kernel
constexpr int kMaxOrder = 16;

struct SpectrumWeights {
  float w[kMaxHistory];
  const float* src[kMaxHistory];
  int K;
};

// out[f] = sum_k w_k H_k[f], four elements per thread per iteration
__global__ void __launch_bounds__(256) spectrum_combine_kernel(const __grid_constant__ SpectrumWeights sw,
                                                               float* __restrict__ out, long long n4) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = 0; k < sw.K; ++k) {
      const float4 h = __ldcs(reinterpret_cast<const float4*>(sw.src[k]) + i);
      const float w = sw.w[k];
      acc.x = fmaf(w, h.x, acc.x);
      acc.y = fmaf(w, h.y, acc.y);
      acc.z = fmaf(w, h.z, acc.z);
      acc.w = fmaf(w, h.w, acc.w);
    }
    reinterpret_cast<float4*>(out)[i] = acc;
  }
}

}  // namespace
}  // namespace qi

using namespace qi;

struct qi_spectrum {
  float* hist = nullptr;  // [cap][F] device ring
  long long F = 0;
  int cap = 0, order = 4;
  float lambda = 0.1f;
  int head = 0, count = 0;   // next slot; stored states
  std::vector<int> step_of;  // per slot
};

// Prediction weights over the K stored states (oldest first): the reference's
// Chebyshev ridge fit (normalize_tau_kernel, chebyshev_design_kernel,
// spectrum_fit_ridge_regression, build_chebyshev_row_kernel,
// chebyshev_predict_kernel) and first-order Taylor term (taylor_predict_kernel
// with order 1), blended as blend_predictions_kernel does.
extern "C" int qi_spectrum_weights(const int* steps, int K, int order, float lambda, int target_step, float blend,
                                   double* w) {
  if (!steps || !w || K < 2 || K > kMaxHistory || order < 0 || order > kMaxOrder) return QI_ERR_ARG;
  for (int k = 1; k < K; ++k)
    if (steps[k] <= steps[k - 1]) return QI_ERR_ARG;
  const int P = order + 1;
  const double t_min = steps[0], t_max = steps[K - 1];
  const double mid = 0.5 * (t_min + t_max), range = t_max - t_min;
  auto tau_of = [&](double t) { return range < 1e-6 ? 0.0 : (t - mid) * 2.0 / range; };
  auto cheb = [&](double tau, double* row) {
    row[0] = 1.0;
    if (P > 1) row[1] = tau;
    for (int m = 2; m < P; ++m) row[m] = 2.0 * tau * row[m - 1] - row[m - 2];
  };
  std::vector<double> X(static_cast<size_t>(K) * P), A(static_cast<size_t>(P) * P, 0.0), z(P);
  for (int k = 0; k < K; ++k) cheb(tau_of(steps[k]), &X[static_cast<size_t>(k) * P]);
  for (int i = 0; i < P; ++i)
    for (int j = 0; j < P; ++j) {
      double s = 0.0;
      for (int k = 0; k < K; ++k) s += X[k * P + i] * X[k * P + j];
      A[i * P + j] = s + (i == j ? static_cast<double>(lambda) : 0.0);
    }
  // Cholesky A = L L^T (symmetric positive definite for lambda > 0)
  for (int j = 0; j < P; ++j) {
    double d = A[j * P + j];
    for (int k = 0; k < j; ++k) d -= A[j * P + k] * A[j * P + k];
    if (!(d > 0.0)) return QI_ERR_ARG;  // singular fit (lambda = 0 with too few distinct steps)
    A[j * P + j] = std::sqrt(d);
    for (int i = j + 1; i < P; ++i) {
      double s = A[i * P + j];
      for (int k = 0; k < j; ++k) s -= A[i * P + k] * A[j * P + k];
      A[i * P + j] = s / A[j * P + j];
    }
  }
  // z = A^-1 row(target): L y = row, L^T z = y
  cheb(tau_of(target_step), z.data());
  for (int i = 0; i < P; ++i) {
    double s = z[i];
    for (int k = 0; k < i; ++k) s -= A[i * P + k] * z[k];
    z[i] = s / A[i * P + i];
  }
  for (int i = P - 1; i >= 0; --i) {
    double s = z[i];
    for (int k = i + 1; k < P; ++k) s -= A[k * P + i] * z[k];
    z[i] = s / A[i * P + i];
  }
  const double b = blend;
  for (int k = 0; k < K; ++k) {
    double s = 0.0;
    for (int p = 0; p < P; ++p) s += X[k * P + p] * z[p];
    w[k] = b * s;
  }
  // Taylor: h_i + kstep (h_i - h_{i-1})
  const double dt = std::fmax(static_cast<double>(steps[K - 1]) - steps[K - 2], 1e-6);
  const double kstep = static_cast<double>(target_step - steps[K - 1]) / dt;
  w[K - 1] += (1.0 - b) * (1.0 + kstep);
  w[K - 2] += (1.0 - b) * (-kstep);
  return QI_OK;
}

extern "C" int qi_spectrum_create(long long feature_elems, int max_history, int order, float lambda,
                                  qi_spectrum** out) {
  if (!out || feature_elems <= 0 || feature_elems % 4 || max_history < 2 || max_history > kMaxHistory || order < 0 ||
      order > kMaxOrder || !(lambda >= 0.0f))
    return QI_ERR_ARG;
  qi_spectrum* s = new qi_spectrum;
  s->F = feature_elems;
  s->cap = max_history;
  s->order = order;
  s->lambda = lambda;
  s->step_of.assign(max_history, 0);
  if (dev_malloc(reinterpret_cast<void**>(&s->hist), static_cast<size_t>(max_history) * feature_elems * 4) !=
      cudaSuccess) {
    delete s;
    return QI_ERR_OOM;
  }
  *out = s;
  return QI_OK;
}

extern "C" int qi_spectrum_destroy(qi_spectrum* s) {
  if (!s) return QI_OK;
  if (s->hist) cudaFree(s->hist);
  delete s;
  return QI_OK;
}

extern "C" int qi_spectrum_reset(qi_spectrum* s) {
  if (!s) return QI_ERR_ARG;
  s->head = 0;
  s->count = 0;
  return QI_OK;
}

extern "C" int qi_spectrum_history(const qi_spectrum* s) { return s ? s->count : 0; }

// Stores the state of an actual forward at `step` (spectrum_update,
// cuda_kernels.cu:6206-6262): appended, or replacing the oldest once the
// history is full (the reference shifts its buffer; the kept states and their
// order are the same).  Steps must increase.
extern "C" int qi_spectrum_update(qi_spectrum* s, const float* feature, int step, void* stream) {
  if (!s || !feature) return QI_ERR_ARG;
  if (s->count > 0 && step <= s->step_of[(s->head + s->cap - 1) % s->cap]) return QI_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(feature) & 15) return QI_ERR_ALIGN;
  if (cudaMemcpyAsync(s->hist + static_cast<size_t>(s->head) * s->F, feature, static_cast<size_t>(s->F) * 4,
                      cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return QI_ERR_CUDA;
  s->step_of[s->head] = step;
  s->head = (s->head + 1) % s->cap;
  if (s->count < s->cap) ++s->count;
  return QI_OK;
}

// The predicted state at `target_step` into out [F] (spectrum_predict,
// cuda_kernels.cu:6268-6333).  Needs two stored states.
extern "C" int qi_spectrum_predict(qi_spectrum* s, int target_step, float blend, float* out, void* stream) {
  if (!s || !out) return QI_ERR_ARG;
  if (s->count < 2) return QI_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(out) & 15) return QI_ERR_ALIGN;
  const int K = s->count;
  const int first = (s->head + s->cap - K) % s->cap;
  std::vector<int> steps(K);
  for (int k = 0; k < K; ++k) steps[k] = s->step_of[(first + k) % s->cap];
  std::vector<double> w(K);
  const int st = qi_spectrum_weights(steps.data(), K, s->order, s->lambda, target_step, blend, w.data());
  if (st != QI_OK) return st;
  SpectrumWeights sw;
  memset(&sw, 0, sizeof(sw));
  sw.K = K;
  for (int k = 0; k < K; ++k) {
    sw.w[k] = static_cast<float>(w[k]);
    sw.src[k] = s->hist + static_cast<size_t>((first + k) % s->cap) * s->F;
  }
  const long long n4 = s->F / 4;
  const long long blocks = std::min<long long>((n4 + 255) / 256, 148LL * 8);
  spectrum_combine_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      sw, out, n4);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}
