// capi.cu -- the C ABI (include/qwen_image_b200.h) and the MMDiT forward.
//
// The forward follows transformer_forward (transformer.cu:234-931) step for
// step, with the reference's per-op launches fused:
//   reference (per block, per stream)               here (per block, both streams)
//   LN+mod; FWHT+quant                        ->    rowquant<LnMod>        (1 launch)
//   3 x (cuBLAS INT8 + dequant)               ->    fused-QKV tcgen05 GEMM  (1, img+txt grouped)
//   4 x RMSNorm; 3 x concat/transpose; 2 x RoPE ->  qkv_post               (1)
//   k_mean; Q quant; K quant; attention; h->f  ->   sage quant (3) + tcgen05 attention (1)
//   transpose/split; FWHT+quant                ->   rowquant<F16>          (1)
//   cuBLAS + dequant; gate_add                 ->   GEMM, residual epilogue (1)
//   LN+mod; FWHT+quant                         ->   rowquant<LnMod>        (1)
//   fc1 cuBLAS + dequant+GELU; FWHT+quant      ->   GEMM GELU epilogue (1) + rowquant (1)
//   fc2 cuBLAS + dequant; gate_add             ->   GEMM, residual epilogue (1)
// The 120 modulation linears of a forward depend only on the timestep
// (transformer.cu:506-515) and run as one GEMV over the stacked weights
// (split over the ranks of a head-parallel group, then all-gathered).
// `nb` batch elements (CFG cond/uncond) share every launch.
//
// Head-parallel (Ulysses) forward over the P ranks of a communicator
// (qi_ctx_set_comm): every rank runs the linears and norms of its share of
// the text and image tokens; before attention the Q/K/V rows are exchanged
// all-to-all so that each rank holds every token of 24/P heads, and the
// attention output goes back the same way.  The exchanges are NCCL
// point-to-point groups on the forward's stream.
#include "qi_internal.h"
#include "sm100.cuh"

#include <cuda_bf16.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <thread>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace qi {
int synth_launch(uint64_t seed, long long n, float scale, float offset, void* out, int bf16, cudaStream_t stream);
uint64_t synth_seed_for(uint64_t base, const char* name);
int rope_table_host(int h, int w, int n_txt, float* pe);

CUresult qi_encode_tiled(CUtensorMap* tm, CUtensorMapDataType dt, cuuint32_t rank, void* base, const cuuint64_t* dims,
                         const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* estr,
                         CUtensorMapInterleave il, CUtensorMapSwizzle sw, CUtensorMapL2promotion l2,
                         CUtensorMapFloatOOBfill oob) {
  using Fn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                          const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                          CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Fn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !p)
      return CUDA_ERROR_NOT_FOUND;
    fn = reinterpret_cast<Fn>(p);
  }
  return fn(tm, dt, rank, base, dims, strides, box, estr, il, sw, l2, oob);
}

namespace {
std::atomic<long long> g_alloc_count{0};
}

cudaError_t dev_malloc(void** p, size_t bytes) {
  g_alloc_count.fetch_add(1, std::memory_order_relaxed);
  return cudaMalloc(p, bytes);
}

cudaError_t host_malloc_pinned(void** p, size_t bytes) {
  g_alloc_count.fetch_add(1, std::memory_order_relaxed);
  return cudaMallocHost(p, bytes);
}

int device_num_sms() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}
}  // namespace qi

using namespace qi;

#define QI_TRY(expr)              \
  do {                            \
    int _st = (expr);             \
    if (_st != QI_OK) return _st; \
  } while (0)

static inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ------------------------------------------------------------------ context
enum BufId {
  B_PATCH, B_TEMB256, B_TACT, B_TACT_S, B_T1, B_TEMB, B_TSILU, B_MODS, B_ADA, B_X, B_TXTN, B_ACT, B_ACT_S, B_QKV,
  B_QKVH, B_QC, B_KC, B_QS, B_KS, B_KMEAN, B_O, B_H, B_FIN, B_PROJ, B_SEND1, B_RECV1, B_SEND2, B_RECV2,
  B_PROJF, B_V8, B_VAMAX, B_VS, B_COUNT
};

struct qi_ctx {
  int device = 0;
  int num_sms = 148;
  int* err = nullptr;  // device error word
  ncclComm_t comm = nullptr;  // head-parallel group (qi_ctx_set_comm), non-blocking
  int urank = 0, usize = 1;
  bool comm_failed = false;   // the group's communicator was aborted; multi-GPU calls fail
  bool attn_fp8 = false;      // forward attention: FP8 P.V variant (qi_ctx_set_attention_fp8pv)
  bool qkv_fused = true;      // q/k norm + RoPE in the QKV GEMM's epilogue (qi_ctx_set_fused_qkv_epilogue)
  int comm_timeout_ms = 60000;  // deadline of every collective step (qi_ctx_set_comm_timeout)
  // direct exchanges over peer memory: the group's buffers mapped here (CUDA
  // IPC), set up for one forward shape (peer_key) at a time
  PeerSet peers = {};
  bool peers_ready = false;
  long long peer_key[3] = {-1, -1, -1};
  std::vector<void*> peer_opened;
  SideStream side = {nullptr, nullptr, nullptr};  // forward work that overlaps the main stream (K mean)
  float* capture = nullptr;  // qi_ctx_set_hidden_capture: final image hidden state of every qi_forward
  unsigned* flags = nullptr;  // this rank's flag words [2][kMaxRanks]
  unsigned epoch = 0;
  void* handles = nullptr;    // device staging for the IPC handle all-gather

  void close_peers() {
    for (void* p : peer_opened) cudaIpcCloseMemHandle(p);
    peer_opened.clear();
    peers_ready = false;
    peer_key[0] = peer_key[1] = peer_key[2] = -1;
  }
  void* buf[B_COUNT] = {};
  size_t cap[B_COUNT] = {};
  int launches = 0;
  // stage profiler (qi_ctx_set_profiling): event pairs recorded around each
  // launch of a forward, resolved lazily in qi_ctx_profile
  bool profiling = false;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> pending;
  std::vector<cudaEvent_t> pool;
  int prof_launches[QI_PROF_COUNT] = {};
  double prof_ms[QI_PROF_COUNT] = {};

  cudaEvent_t ev() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e;
    cudaEventCreate(&e);
    return e;
  }

  int ensure(int id, size_t bytes) {
    bytes = (bytes + 255) & ~size_t(255);
    if (cap[id] >= bytes) return QI_OK;
    if (buf[id]) cudaFree(buf[id]);
    buf[id] = nullptr;
    cap[id] = 0;
    if (dev_malloc(&buf[id], bytes) != cudaSuccess) return QI_ERR_OOM;
    cap[id] = bytes;
    return QI_OK;
  }
  template <typename T>
  T* p(int id) const {
    return reinterpret_cast<T*>(buf[id]);
  }
};

// ------------------------------------------------------------------ model
struct Lin {  // INT8 linear in kernel layout
  int8_t* w = nullptr;
  float* s = nullptr;
  __nv_bfloat16* b = nullptr;
  int N = 0, K = 0;
};
struct BlockW {
  Lin qkv[2], out[2], fc1[2], fc2[2];  // [0] image stream, [1] text stream
  __nv_bfloat16* norms = nullptr;       // [4][128]: q, k, added_q, added_k
};
struct qi_model {
  int nblocks = 0;
  Lin t1, t2;
  Lin mod;  // stacked [nblocks][2][18432][3072]
  __nv_bfloat16 *txt_norm = nullptr, *img_in_w = nullptr, *img_in_b = nullptr, *txt_in_w = nullptr,
                *txt_in_b = nullptr, *norm_out_w = nullptr, *norm_out_b = nullptr, *proj_out_w = nullptr,
                *proj_out_b = nullptr;
  std::vector<BlockW> blocks;
  std::vector<void*> allocs;

  template <typename T>
  T* alloc(size_t n) {
    void* p = nullptr;
    if (dev_malloc(&p, n * sizeof(T)) != cudaSuccess) return nullptr;
    allocs.push_back(p);
    return reinterpret_cast<T*>(p);
  }
  ~qi_model() {
    for (void* p : allocs) cudaFree(p);
  }
};

// ------------------------------------------------------------------ collectives
// The head-parallel communicator is non-blocking (ncclConfig_t.blocking = 0):
// no NCCL call can hold the host thread.  A call that returns ncclInProgress
// is polled (ncclCommGetAsyncError) until it settles or the context's
// deadline passes; on an error or a missed deadline the communicator is
// aborted (ncclCommAbort ends its pending operations) and the call returns
// QI_ERR_NCCL.  The reference has no multi-GPU path; its CUDA errors print
// and exit (tensor.h:15-37).
namespace {

double now_ms() {
  return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void abort_comm(qi_ctx* c) {
  if (c->comm) ncclCommAbort(c->comm);
  c->comm = nullptr;
  c->comm_failed = true;
}

// Orderly teardown of a healthy communicator: finalize (non-blocking, so
// polled with the deadline), then destroy; aborted if it does not settle.
void destroy_comm(qi_ctx* c) {
  if (!c->comm) return;
  ncclResult_t r = ncclCommFinalize(c->comm);
  const double deadline = now_ms() + c->comm_timeout_ms;
  while (r == ncclInProgress && now_ms() < deadline) {
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    if (ncclCommGetAsyncError(c->comm, &r) != ncclSuccess) r = ncclSystemError;
  }
  if (r == ncclSuccess)
    ncclCommDestroy(c->comm);
  else
    ncclCommAbort(c->comm);
  c->comm = nullptr;
}

// Waits for the communicator's current call (which returned `r`) to settle.
int nccl_settle(qi_ctx* c, ncclResult_t r) {
  if (r == ncclSuccess) return QI_OK;
  if (r != ncclInProgress || !c->comm) {
    abort_comm(c);
    return QI_ERR_NCCL;
  }
  const double deadline = now_ms() + c->comm_timeout_ms;
  while (true) {
    ncclResult_t st = ncclSuccess;
    if (ncclCommGetAsyncError(c->comm, &st) != ncclSuccess) st = ncclSystemError;
    if (st == ncclSuccess) return QI_OK;
    if (st != ncclInProgress || now_ms() > deadline) {
      abort_comm(c);
      return QI_ERR_NCCL;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

}  // namespace

#define QI_NCCL(c, call) QI_TRY(nccl_settle((c), (call)))

extern "C" {

const char* qi_status_string(int st) {
  switch (st) {
    case QI_OK: return "ok";
    case QI_ERR_ARG: return "invalid argument";
    case QI_ERR_ALIGN: return "pointer or leading dimension not 16-byte aligned";
    case QI_ERR_CUDA: return "CUDA call failed";
    case QI_ERR_OOM: return "device allocation failed";
    case QI_ERR_UNSUPPORTED: return "shape not supported by the kernels";
    case QI_ERR_IO: return "file missing or malformed";
    case QI_ERR_DEVICE: return "kernel bounded wait timed out";
    case QI_ERR_NCCL: return "collective failed";
    default: return "unknown status";
  }
}

int qi_version(void) { return 1; }

long long qi_alloc_count(void) { return g_alloc_count.load(std::memory_order_relaxed); }

int qi_ctx_create(int device, qi_ctx** out) {
  if (!out) return QI_ERR_ARG;
  if (cudaSetDevice(device) != cudaSuccess) return QI_ERR_CUDA;
  qi_ctx* c = new qi_ctx();
  c->device = device;
  c->num_sms = device_num_sms();
  if (dev_malloc(reinterpret_cast<void**>(&c->err), sizeof(int)) != cudaSuccess) {
    delete c;
    return QI_ERR_OOM;
  }
  cudaMemset(c->err, 0, sizeof(int));
  *out = c;
  return QI_OK;
}

int qi_ctx_destroy(qi_ctx* c) {
  if (!c) return QI_OK;
  for (auto& p : c->pending) {
    cudaEventDestroy(p.second.first);
    cudaEventDestroy(p.second.second);
  }
  for (cudaEvent_t e : c->pool) cudaEventDestroy(e);
  if (c->side.s) cudaStreamDestroy(c->side.s);
  if (c->side.fork) cudaEventDestroy(c->side.fork);
  if (c->side.join) cudaEventDestroy(c->side.join);
  for (int i = 0; i < B_COUNT; ++i)
    if (c->buf[i]) cudaFree(c->buf[i]);
  if (c->err) cudaFree(c->err);
  c->close_peers();
  if (c->flags) cudaFree(c->flags);
  if (c->handles) cudaFree(c->handles);
  destroy_comm(c);
  delete c;
  return QI_OK;
}

int qi_ctx_set_attention_fp8pv(qi_ctx* c, int enable) {
  if (!c) return QI_ERR_ARG;
  c->attn_fp8 = enable != 0;
  return QI_OK;
}

int qi_ctx_set_fused_qkv_epilogue(qi_ctx* c, int enable) {
  if (!c) return QI_ERR_ARG;
  c->qkv_fused = enable != 0;
  return QI_OK;
}

int qi_ctx_set_comm_timeout(qi_ctx* c, int timeout_ms) {
  if (!c || timeout_ms <= 0) return QI_ERR_ARG;
  c->comm_timeout_ms = timeout_ms;
  return QI_OK;
}

int qi_ctx_sync(qi_ctx* c, void* stream, int timeout_ms) {
  if (!c) return QI_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const double deadline = now_ms() + (timeout_ms > 0 ? timeout_ms : c->comm_timeout_ms);
  while (true) {
    const cudaError_t q = cudaStreamQuery(s);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return QI_ERR_CUDA;
    if (c->comm) {
      ncclResult_t st = ncclSuccess;
      if (ncclCommGetAsyncError(c->comm, &st) != ncclSuccess) st = ncclSystemError;
      if (st != ncclSuccess && st != ncclInProgress) {
        abort_comm(c);
        return QI_ERR_NCCL;
      }
    }
    if (now_ms() > deadline) {
      // a collective that waits for a peer is the one thing on the stream that
      // cannot end by itself (the library's own waits are bounded): abort it
      if (c->comm) {
        abort_comm(c);
        return QI_ERR_NCCL;
      }
      return QI_ERR_DEVICE;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  return qi_ctx_check(c);
}

int qi_comm_unique_id(void* id_out) {
  if (!id_out) return QI_ERR_ARG;
  static_assert(sizeof(ncclUniqueId) == QI_COMM_ID_BYTES, "NCCL unique id size");
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return QI_ERR_NCCL;
  memcpy(id_out, &id, sizeof(id));
  return QI_OK;
}

int qi_ctx_set_comm(qi_ctx* c, const void* id, int rank, int nranks) {
  if (!c || nranks < 1 || nranks > kMaxRanks || kHeads % nranks || rank < 0 || rank >= nranks) return QI_ERR_ARG;
  c->close_peers();
  destroy_comm(c);
  c->comm_failed = false;
  c->urank = 0;
  c->usize = 1;
  // a new group starts its barrier epochs from zero on every rank
  if (c->flags && cudaMemset(c->flags, 0, 2 * kMaxRanks * sizeof(unsigned)) != cudaSuccess) return QI_ERR_CUDA;
  c->epoch = 0;
  if (nranks == 1) return QI_OK;
  if (!id) return QI_ERR_ARG;
  if (cudaSetDevice(c->device) != cudaSuccess) return QI_ERR_CUDA;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;  // every call returns at once; nccl_settle waits with a deadline
  const ncclResult_t r = ncclCommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  // a rank that never joins: the initialisation misses the deadline and is aborted
  QI_NCCL(c, r);
  c->urank = rank;
  c->usize = nranks;
  return QI_OK;
}

int qi_ctx_check(qi_ctx* c) {
  if (!c) return QI_ERR_ARG;
  int h = 0;
  if (cudaMemcpy(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return QI_ERR_CUDA;
  if (h) cudaMemset(c->err, 0, sizeof(int));
  return h ? QI_ERR_DEVICE : QI_OK;
}

int qi_ctx_last_launch_count(const qi_ctx* c) { return c ? c->launches : 0; }

int qi_selftest_wait_timeout(qi_ctx* c, int limit_us, void* stream) {
  if (!c) return QI_ERR_ARG;
  return selftest_wait_timeout(c->err, limit_us, reinterpret_cast<cudaStream_t>(stream));
}

int qi_ctx_set_profiling(qi_ctx* c, int enable) {
  if (!c) return QI_ERR_ARG;
  c->profiling = enable != 0;
  return QI_OK;
}

int qi_ctx_profile(qi_ctx* c, int* launches, float* ms, int reset) {
  if (!c) return QI_ERR_ARG;
  for (auto& p : c->pending) {
    if (cudaEventSynchronize(p.second.second) != cudaSuccess) return QI_ERR_CUDA;
    float t = 0.0f;
    cudaEventElapsedTime(&t, p.second.first, p.second.second);
    c->prof_ms[p.first] += t;
    c->prof_launches[p.first] += 1;
    c->pool.push_back(p.second.first);
    c->pool.push_back(p.second.second);
  }
  c->pending.clear();
  for (int i = 0; i < QI_PROF_COUNT; ++i) {
    if (launches) launches[i] = c->prof_launches[i];
    if (ms) ms[i] = static_cast<float>(c->prof_ms[i]);
    if (reset) {
      c->prof_launches[i] = 0;
      c->prof_ms[i] = 0.0;
    }
  }
  return QI_OK;
}

int qi_cfg_euler_step(float* latent, const void* cond_bf16, const void* uncond_bf16, float cfg_scale, float sigma,
                      float sigma_next, int H, int W, void* latent_bf16, void* stream) {
  if (!latent || !cond_bf16 || !uncond_bf16 || !latent_bf16 || sigma == 0.0f) return QI_ERR_ARG;
  return cfg_euler_launch(latent, cond_bf16, uncond_bf16, cfg_scale, sigma, sigma_next, H, W, latent_bf16,
                          reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// Default per-device context for the op-level entry points (they take no
// context, like the reference's functions that use static workspaces).
static qi_ctx* default_ctx() {
  static std::mutex mu;
  static std::map<int, qi_ctx*> ctxs;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  auto it = ctxs.find(dev);
  if (it != ctxs.end()) return it->second;
  qi_ctx* c = nullptr;
  if (qi_ctx_create(dev, &c) != QI_OK) return nullptr;
  ctxs[dev] = c;
  return c;
}

extern "C" {

// ------------------------------------------------------------------ op level
int qi_quantize_weight(const void* w_bf16, int N, int K, int8_t* codes, float* scales, void* stream) {
  if (!w_bf16 || !codes || !scales || N < 0 || K <= 0) return QI_ERR_ARG;
  return fwht_quant_generic(w_bf16, 1, N, K, K & (-K), codes, scales, S_(stream));
}

int qi_fwht_quantize(const float* x, int M, int K, int had_block, int8_t* codes, float* scales, void* stream) {
  if (!x || !codes || !scales || M < 0 || K <= 0) return QI_ERR_ARG;
  if (had_block < 1) had_block = 1;
  if ((K == 3072 || K == 12288 || K == 256) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0)) {
    RowSeg seg{x, K, nullptr, nullptr, M};
    int st = rowquant_launch(kSrcF32, K, had_block, &seg, 1, codes, scales, 0.0f, S_(stream));
    if (st != QI_ERR_UNSUPPORTED) return st;
  }
  return fwht_quant_generic(x, 0, M, K, had_block, codes, scales, S_(stream));
}

int qi_linear_i8(const int8_t* act, const float* act_scales, int M, int K, const int8_t* w, const float* w_scales,
                 int N, const void* bias_bf16, int epilogue, const float* gate, float* out, int ldo, void* stream) {
  if (!act || !act_scales || !w || !w_scales || !out || epilogue < 0 || epilogue > 2) return QI_ERR_ARG;
  qi_ctx* c = default_ctx();
  if (!c) return QI_ERR_CUDA;
  GemmDesc d{act, act_scales, w, w_scales, bias_bf16, out, gate, M, N, K, ldo};
  return gemm_i8_launch(&d, 1, epilogue, S_(stream), c->err, c->num_sms);
}

int qi_linear_i8_f32in(const float* x, int M, int K, const int8_t* w, const float* w_scales, int N,
                       const void* bias_bf16, int apply_gelu, float* out, void* stream) {
  qi_ctx* c = default_ctx();
  if (!c) return QI_ERR_CUDA;
  QI_TRY(c->ensure(B_ACT, static_cast<size_t>(M) * K));
  QI_TRY(c->ensure(B_ACT_S, static_cast<size_t>(M) * 4));
  QI_TRY(qi_fwht_quantize(x, M, K, K & (-K), c->p<int8_t>(B_ACT), c->p<float>(B_ACT_S), stream));
  if (M == 1 && !apply_gelu) {
    GemvJob j{w, w_scales, bias_bf16, out, N};
    return gemv_i8_launch(c->p<int8_t>(B_ACT), c->p<float>(B_ACT_S), K, &j, 1, S_(stream));
  }
  GemmDesc d{c->p<int8_t>(B_ACT), c->p<float>(B_ACT_S), w, w_scales, bias_bf16, out, nullptr, M, N, K, N};
  return gemm_i8_launch(&d, 1, apply_gelu ? kEpiGelu : kEpiStore, S_(stream), c->err, c->num_sms);
}

int qi_sage_quantize(const void* q_f16, const void* k_f16, int BH, int S, float* k_mean, int8_t* q_codes,
                     float* q_scales, int8_t* k_codes, float* k_scales, void* stream) {
  if (!q_f16 || !k_f16 || !k_mean || !q_codes || !q_scales || !k_codes || !k_scales) return QI_ERR_ARG;
  return sage_quantize_launch(q_f16, k_f16, BH, S, k_mean, q_codes, q_scales, k_codes, k_scales, S_(stream));
}

int qi_sage_attention(const void* q_f16, const void* k_f16, const void* v_f16, float* out, float scale, int BH, int S,
                      int D, void* stream) {
  if (D != 128) return QI_ERR_UNSUPPORTED;
  if (!q_f16 || !k_f16 || !v_f16 || !out || BH <= 0 || S <= 0) return QI_ERR_ARG;
  if (S > kAttnMaxS) return QI_ERR_UNSUPPORTED;  // before any workspace grows or kernel runs
  qi_ctx* c = default_ctx();
  if (!c) return QI_ERR_CUDA;
  const size_t n = static_cast<size_t>(BH) * S * 128;
  QI_TRY(c->ensure(B_QC, n));
  QI_TRY(c->ensure(B_KC, n));
  QI_TRY(c->ensure(B_QS, static_cast<size_t>(BH) * ((S + 127) / 128) * 32 * 4));
  QI_TRY(c->ensure(B_KS, static_cast<size_t>(BH) * ((S + 63) / 64) * 4 * 4));
  QI_TRY(c->ensure(B_KMEAN, static_cast<size_t>(BH) * 128 * 4));
  QI_TRY(sage_quantize_launch(q_f16, k_f16, BH, S, c->p<float>(B_KMEAN), c->p<int8_t>(B_QC), c->p<float>(B_QS),
                              c->p<int8_t>(B_KC), c->p<float>(B_KS), S_(stream)));
  AttnArgs a{c->p<int8_t>(B_QC), c->p<float>(B_QS), c->p<int8_t>(B_KC), c->p<float>(B_KS), v_f16, out, BH, S, BH,
             scale, 0, 1, 0, 0};
  return attention_launch(a, S_(stream), c->err);
}

int qi_sage_attention_fp8pv(const void* q_f16, const void* k_f16, const void* v_f16, float* out, float scale, int BH,
                            int S, int D, void* stream) {
  if (D != 128) return QI_ERR_UNSUPPORTED;
  if (!q_f16 || !k_f16 || !v_f16 || !out || BH <= 0 || S <= 0) return QI_ERR_ARG;
  if (S > kAttnMaxS) return QI_ERR_UNSUPPORTED;
  qi_ctx* c = default_ctx();
  if (!c) return QI_ERR_CUDA;
  const size_t n = static_cast<size_t>(BH) * S * 128;
  const int s_pad = (S + 15) & ~15;
  QI_TRY(c->ensure(B_QC, n));
  QI_TRY(c->ensure(B_KC, n));
  QI_TRY(c->ensure(B_QS, static_cast<size_t>(BH) * ((S + 127) / 128) * 32 * 4));
  QI_TRY(c->ensure(B_KS, static_cast<size_t>(BH) * ((S + 63) / 64) * 4 * 4));
  QI_TRY(c->ensure(B_KMEAN, static_cast<size_t>(BH) * 128 * 4));
  QI_TRY(c->ensure(B_V8, static_cast<size_t>(BH) * 128 * s_pad));
  QI_TRY(c->ensure(B_VAMAX, static_cast<size_t>(BH) * 128 * 4));
  QI_TRY(c->ensure(B_VS, static_cast<size_t>(BH) * 128 * 4));
  QI_TRY(sage_quantize_fp8pv_launch(q_f16, k_f16, v_f16, BH, S, c->p<float>(B_KMEAN), c->p<int8_t>(B_QC),
                                    c->p<float>(B_QS), c->p<int8_t>(B_KC), c->p<float>(B_KS), c->p<uint8_t>(B_V8), s_pad,
                                    c->p<float>(B_VAMAX), c->p<float>(B_VS), S_(stream)));
  AttnArgs a{c->p<int8_t>(B_QC), c->p<float>(B_QS), c->p<int8_t>(B_KC), c->p<float>(B_KS), c->buf[B_V8], out, BH, S, BH,
             scale, 0, 1, 0, 0};
  a.fp8 = 1;
  a.vs = c->p<float>(B_VS);
  a.s_pad = s_pad;
  return attention_launch(a, S_(stream), c->err);
}

int qi_layer_norm_modulate(const float* x, const float* shift, const float* scale, float* out, int rows, int dim,
                           float eps, void* stream) {
  if (!x || !shift || !scale || !out || rows < 0 || dim <= 0) return QI_ERR_ARG;
  return layernorm_mod_launch(x, shift, scale, rows, dim, eps, out, nullptr, S_(stream));
}

int qi_rms_norm(const float* x, const void* w_bf16, float* out, int rows, int dim, float eps, void* stream) {
  if (!x || !w_bf16 || !out || rows < 0 || dim <= 0) return QI_ERR_ARG;
  return rmsnorm_f32_launch(x, w_bf16, out, rows, dim, eps, S_(stream));
}

int qi_layer_norm_modulate_quantize(const float* x, const float* shift, const float* scale, int rows, int dim,
                                    float eps, int8_t* codes, float* scales, void* stream) {
  if (!x || !shift || !scale || !codes || !scales || rows < 0 || dim <= 0) return QI_ERR_ARG;
  if (dim != kDim) return QI_ERR_UNSUPPORTED;
  RowSeg seg{x, dim, shift, scale, rows};
  return rowquant_launch(kSrcLnMod, dim, dim & (-dim), &seg, 1, codes, scales, eps, S_(stream));
}

int qi_qk_norm_rope(const float* qkv_img, const float* qkv_txt, const void* norms_bf16, const float* pe, int nb,
                    int n_img, int n_txt, void* qkv_f16, void* stream) {
  if (!qkv_img || !qkv_txt || !norms_bf16 || !pe || !qkv_f16 || nb < 1 || n_img < 0 || n_txt < 0) return QI_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(qkv_img) | reinterpret_cast<uintptr_t>(qkv_txt) |
       reinterpret_cast<uintptr_t>(pe) | reinterpret_cast<uintptr_t>(qkv_f16)) & 15)
    return QI_ERR_ALIGN;
  const __nv_bfloat16* n = static_cast<const __nv_bfloat16*>(norms_bf16);
  QkvPostArgs a{qkv_img, qkv_txt, n, n + kHeadDim, n + 2 * kHeadDim, n + 3 * kHeadDim, pe, qkv_f16, nb, n_img, n_txt,
                0, n_img, 0, n_txt, kHeads, 0};
  return qkv_post_launch(a, S_(stream));
}

int qi_qkv_norm_rope_i8(const int8_t* act_img, const float* act_img_scales, const int8_t* act_txt,
                        const float* act_txt_scales, const int8_t* w_img, const float* w_img_scales, const void* b_img,
                        const int8_t* w_txt, const float* w_txt_scales, const void* b_txt, const void* norms_bf16,
                        const float* pe, int nb, int n_img, int n_txt, void* qkv_f16, void* stream) {
  if (!act_img || !act_img_scales || !act_txt || !act_txt_scales || !w_img || !w_img_scales || !w_txt ||
      !w_txt_scales || !norms_bf16 || !pe || !qkv_f16 || nb < 1 || n_img < 0 || n_txt < 0)
    return QI_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(pe) | reinterpret_cast<uintptr_t>(qkv_f16)) & 15) return QI_ERR_ALIGN;
  qi_ctx* c = default_ctx();
  if (!c) return QI_ERR_CUDA;
  const __nv_bfloat16* n = static_cast<const __nv_bfloat16*>(norms_bf16);
  QkvPostArgs a{nullptr, nullptr, n, n + kHeadDim, n + 2 * kHeadDim, n + 3 * kHeadDim, pe, qkv_f16, nb, n_img, n_txt,
                0, n_img, 0, n_txt, kHeads, 0};
  GemmDesc d[2] = {{act_img, act_img_scales, w_img, w_img_scales, b_img, nullptr, nullptr, nb * n_img, 3 * kDim, kDim,
                    3 * kDim},
                   {act_txt, act_txt_scales, w_txt, w_txt_scales, b_txt, nullptr, nullptr, nb * n_txt, 3 * kDim, kDim,
                    3 * kDim}};
  if (!gemm_qkv_fusable(d, 2, c->num_sms)) return QI_ERR_UNSUPPORTED;
  return gemm_qkv_launch(d, 2, a, S_(stream), c->err, c->num_sms);
}

int qi_rope_table(int h, int w, int n_txt, float* pe_host) {
  if (!pe_host || h <= 0 || w <= 0 || n_txt < 0) return QI_ERR_ARG;
  return rope_table_host(h, w, n_txt, pe_host);
}

// Synthetic tensors (benchmarks and tests): value i = z_i * scale + offset.
int qi_synth_fill(void* out, long long n, unsigned long long seed, float scale, float offset, int bf16, void* stream) {
  if (!out || n < 0) return QI_ERR_ARG;
  return synth_launch(seed, n, scale, offset, out, bf16, S_(stream));
}
unsigned long long qi_seed_for(unsigned long long base, const char* name) { return synth_seed_for(base, name); }

// ------------------------------------------------------------------ model
int qi_model_num_blocks(const qi_model* m) { return m ? m->nblocks : 0; }

int qi_model_destroy(qi_model* m) {
  delete m;
  return QI_OK;
}

}  // extern "C"

static int copy_lin(qi_model* m, Lin& L, const void* const* t, int base, int N, int K) {
  L.N = N;
  L.K = K;
  L.w = m->alloc<int8_t>(static_cast<size_t>(N) * K);
  L.s = m->alloc<float>(N);
  L.b = m->alloc<__nv_bfloat16>(N);
  if (!L.w || !L.s || !L.b) return QI_ERR_OOM;
  if (!t[base] || !t[base + 1]) return QI_ERR_ARG;
  cudaMemcpyAsync(L.w, t[base], static_cast<size_t>(N) * K, cudaMemcpyDeviceToDevice);
  cudaMemcpyAsync(L.s, t[base + 1], N * 4, cudaMemcpyDeviceToDevice);
  if (t[base + 2])
    cudaMemcpyAsync(L.b, t[base + 2], N * 2, cudaMemcpyDeviceToDevice);
  else
    cudaMemsetAsync(L.b, 0, N * 2);
  return QI_OK;
}

// Concatenates three [N,K] linears along N (Q, K, V share one quantized
// activation, transformer.cu:217-230 can_share_qkv_quant).
static int copy_fused3(qi_model* m, Lin& L, const void* const* t, int l0, int l1, int l2) {
  const int N = 3 * kDim, K = kDim;
  L.N = N;
  L.K = K;
  L.w = m->alloc<int8_t>(static_cast<size_t>(N) * K);
  L.s = m->alloc<float>(N);
  L.b = m->alloc<__nv_bfloat16>(N);
  if (!L.w || !L.s || !L.b) return QI_ERR_OOM;
  const int ls[3] = {l0, l1, l2};
  for (int i = 0; i < 3; ++i) {
    const void* const* e = t + 3 * ls[i];
    if (!e[0] || !e[1]) return QI_ERR_ARG;
    cudaMemcpyAsync(L.w + static_cast<size_t>(i) * kDim * K, e[0], static_cast<size_t>(kDim) * K,
                    cudaMemcpyDeviceToDevice);
    cudaMemcpyAsync(L.s + i * kDim, e[1], kDim * 4, cudaMemcpyDeviceToDevice);
    if (e[2])
      cudaMemcpyAsync(L.b + i * kDim, e[2], kDim * 2, cudaMemcpyDeviceToDevice);
    else
      cudaMemsetAsync(L.b + i * kDim, 0, kDim * 2);
  }
  return QI_OK;
}

static __nv_bfloat16* copy_bf16(qi_model* m, const void* src, size_t n) {
  __nv_bfloat16* d = m->alloc<__nv_bfloat16>(n);
  if (!d) return nullptr;
  if (src)
    cudaMemcpyAsync(d, src, n * 2, cudaMemcpyDeviceToDevice);
  else
    cudaMemsetAsync(d, 0, n * 2);
  return d;
}

extern "C" int qi_model_create(qi_ctx* ctx, int num_blocks, const void* const* g, const void* const* const* bt,
                               qi_model** out) {
  if (!ctx || !g || !bt || !out || num_blocks <= 0) return QI_ERR_ARG;
  cudaSetDevice(ctx->device);
  qi_model* m = new qi_model();
  m->nblocks = num_blocks;
  int st = QI_OK;
  auto fail = [&](int s) {
    delete m;
    return s;
  };
  if ((st = copy_lin(m, m->t1, g, QI_G_T1_W, kDim, 256)) != QI_OK) return fail(st);
  if ((st = copy_lin(m, m->t2, g, QI_G_T2_W, kDim, kDim)) != QI_OK) return fail(st);
  if (!g[QI_G_IMG_IN_W] || !g[QI_G_TXT_IN_W] || !g[QI_G_NORM_OUT_W] || !g[QI_G_PROJ_OUT_W] || !g[QI_G_TXT_NORM])
    return fail(QI_ERR_ARG);
  m->txt_norm = copy_bf16(m, g[QI_G_TXT_NORM], kTxtDim);
  m->img_in_w = copy_bf16(m, g[QI_G_IMG_IN_W], static_cast<size_t>(kDim) * kPatchDim);
  m->img_in_b = copy_bf16(m, g[QI_G_IMG_IN_B], kDim);
  m->txt_in_w = copy_bf16(m, g[QI_G_TXT_IN_W], static_cast<size_t>(kDim) * kTxtDim);
  m->txt_in_b = copy_bf16(m, g[QI_G_TXT_IN_B], kDim);
  m->norm_out_w = copy_bf16(m, g[QI_G_NORM_OUT_W], static_cast<size_t>(2 * kDim) * kDim);
  m->norm_out_b = copy_bf16(m, g[QI_G_NORM_OUT_B], 2 * kDim);
  m->proj_out_w = copy_bf16(m, g[QI_G_PROJ_OUT_W], static_cast<size_t>(kPatchDim) * kDim);
  m->proj_out_b = copy_bf16(m, g[QI_G_PROJ_OUT_B], kPatchDim);
  // stacked modulation: [block][img, txt][18432][3072]
  const size_t modN = static_cast<size_t>(num_blocks) * 2 * 6 * kDim;
  m->mod.N = static_cast<int>(modN);
  m->mod.K = kDim;
  m->mod.w = m->alloc<int8_t>(modN * kDim);
  m->mod.s = m->alloc<float>(modN);
  m->mod.b = m->alloc<__nv_bfloat16>(modN);
  if (!m->mod.w || !m->mod.s || !m->mod.b) return fail(QI_ERR_OOM);
  m->blocks.resize(num_blocks);
  for (int i = 0; i < num_blocks; ++i) {
    const void* const* t = bt[i];
    if (!t) return fail(QI_ERR_ARG);
    for (int sidx = 0; sidx < 2; ++sidx) {
      const int l = sidx == 0 ? QI_L_IMG_MOD : QI_L_TXT_MOD;
      const size_t row0 = (static_cast<size_t>(i) * 2 + sidx) * 6 * kDim;
      if (!t[3 * l] || !t[3 * l + 1]) return fail(QI_ERR_ARG);
      cudaMemcpyAsync(m->mod.w + row0 * kDim, t[3 * l], static_cast<size_t>(6) * kDim * kDim, cudaMemcpyDeviceToDevice);
      cudaMemcpyAsync(m->mod.s + row0, t[3 * l + 1], 6 * kDim * 4, cudaMemcpyDeviceToDevice);
      if (t[3 * l + 2])
        cudaMemcpyAsync(m->mod.b + row0, t[3 * l + 2], 6 * kDim * 2, cudaMemcpyDeviceToDevice);
      else
        cudaMemsetAsync(m->mod.b + row0, 0, 6 * kDim * 2);
    }
    BlockW& B = m->blocks[i];
    if ((st = copy_fused3(m, B.qkv[0], t, QI_L_TO_Q, QI_L_TO_K, QI_L_TO_V)) != QI_OK) return fail(st);
    if ((st = copy_fused3(m, B.qkv[1], t, QI_L_ADD_Q, QI_L_ADD_K, QI_L_ADD_V)) != QI_OK) return fail(st);
    if ((st = copy_lin(m, B.out[0], t, 3 * QI_L_TO_OUT, kDim, kDim)) != QI_OK) return fail(st);
    if ((st = copy_lin(m, B.out[1], t, 3 * QI_L_TO_ADD_OUT, kDim, kDim)) != QI_OK) return fail(st);
    if ((st = copy_lin(m, B.fc1[0], t, 3 * QI_L_IMG_FC1, kMlp, kDim)) != QI_OK) return fail(st);
    if ((st = copy_lin(m, B.fc2[0], t, 3 * QI_L_IMG_FC2, kDim, kMlp)) != QI_OK) return fail(st);
    if ((st = copy_lin(m, B.fc1[1], t, 3 * QI_L_TXT_FC1, kMlp, kDim)) != QI_OK) return fail(st);
    if ((st = copy_lin(m, B.fc2[1], t, 3 * QI_L_TXT_FC2, kDim, kMlp)) != QI_OK) return fail(st);
    B.norms = m->alloc<__nv_bfloat16>(4 * kHeadDim);
    if (!B.norms) return fail(QI_ERR_OOM);
    for (int k = 0; k < 4; ++k) {
      if (!t[QI_B_NORM_Q + k]) return fail(QI_ERR_ARG);
      cudaMemcpyAsync(B.norms + k * kHeadDim, t[QI_B_NORM_Q + k], kHeadDim * 2, cudaMemcpyDeviceToDevice);
    }
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(QI_ERR_CUDA);
  *out = m;
  return QI_OK;
}

// ------------------------------------------------------------------ forward
namespace {
// Even split of the text and of the image tokens over P ranks.
ShardMap make_map(int P, int n_txt, int n_img) {
  ShardMap mp;
  memset(&mp, 0, sizeof(mp));
  mp.P = P;
  for (int r = 0; r <= P; ++r) {
    mp.txt_lo[r] = static_cast<int>(static_cast<long long>(r) * n_txt / P);
    mp.img_lo[r] = static_cast<int>(static_cast<long long>(r) * n_img / P);
  }
  return mp;
}

// Byte offsets and sizes, per peer, of the two all-to-all exchanges of a
// head-parallel block (FP16 rows of 128):
//   which 0 (Q/K/V): rank r sends peer q [3][nb][Hl][len(r)][128] from offset
//     q * that size, and receives [3][nb][Hl][len(q)][128] packed by q;
//   which 1 (attention output): rank r sends peer q [nb][len(q)][Hl][128],
//     packed by q, and receives [nb][len(r)][Hl][128] at offset q * that size.
void exchange_plan(int which, int nb, const ShardMap& mp, int rank, long long* soff, long long* sbytes,
                   long long* roff, long long* rbytes) {
  const long long Hl = kHeads / mp.P, row = kHeadDim * 2;
  long long so = 0, ro = 0;
  for (int q = 0; q < mp.P; ++q) {
    if (which == 0) {
      sbytes[q] = 3LL * nb * Hl * mp.len(rank) * row;
      rbytes[q] = 3LL * nb * Hl * mp.len(q) * row;
    } else {
      sbytes[q] = static_cast<long long>(nb) * mp.len(q) * Hl * row;
      rbytes[q] = static_cast<long long>(nb) * mp.len(rank) * Hl * row;
    }
    soff[q] = so;
    roff[q] = ro;
    so += sbytes[q];
    ro += rbytes[q];
  }
}

// All-to-all with per-peer sizes on `s`: NCCL send/recv pairs in one group,
// the rank's own chunk as a device copy.
int exchange(qi_ctx* c, int which, int nb, const ShardMap& mp, const void* send, void* recv, cudaStream_t s) {
  long long so[kMaxRanks], sb[kMaxRanks], ro[kMaxRanks], rb[kMaxRanks];
  exchange_plan(which, nb, mp, c->urank, so, sb, ro, rb);
  const char* sp = static_cast<const char*>(send);
  char* rp = static_cast<char*>(recv);
  const int me = c->urank;
  if (sb[me] && cudaMemcpyAsync(rp + ro[me], sp + so[me], sb[me], cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return QI_ERR_CUDA;
  QI_NCCL(c, ncclGroupStart());
  for (int q = 0; q < mp.P; ++q) {
    if (q == me) continue;
    if (sb[q]) QI_NCCL(c, ncclSend(sp + so[q], sb[q], ncclUint8, q, c->comm, s));
    if (rb[q]) QI_NCCL(c, ncclRecv(rp + ro[q], rb[q], ncclUint8, q, c->comm, s));
  }
  QI_NCCL(c, ncclGroupEnd());
  return QI_OK;
}

// Shapes and workspace views of one forward; the stages below share it.
struct Fwd {
  qi_ctx* c;
  const qi_model* m;
  cudaStream_t s;
  int nb, n_img, n_txt, S, BH;
  int P = 1, rank = 0, Hl = kHeads;  // head-parallel group
  ShardMap map;
  int img_lo = 0, n_img_l = 0, txt_lo = 0, n_txt_l = 0;  // this rank's tokens
  long long Mi, Mt, Ma;  // this rank's image / text / all rows (nb entries)
  bool direct = false;   // exchanges by stores into peer memory (else NCCL)
  int n = 0;  // launches issued
};

// Maps the group's Q/K/V buffers, attention-output buffers and flag words
// into this process (CUDA IPC; handles all-gathered over NCCL) for the
// current forward shape.  Collective over the group: every rank runs the same
// shapes in the same order, so all of them come here together.  If any rank
// cannot map its peers, all fall back to the NCCL exchanges.
int setup_peers(Fwd& f) {
  qi_ctx* c = f.c;
  const long long key[3] = {f.nb, f.n_img, f.n_txt};
  if (c->peer_key[0] == key[0] && c->peer_key[1] == key[1] && c->peer_key[2] == key[2]) {
    f.direct = c->peers_ready;
    return QI_OK;
  }
  c->close_peers();
  const int P = f.P, me = f.rank;
  constexpr int kH = sizeof(cudaIpcMemHandle_t);
  if (!c->flags) {
    if (dev_malloc(reinterpret_cast<void**>(&c->flags), 2 * kMaxRanks * sizeof(unsigned)) != cudaSuccess) return QI_ERR_OOM;
    if (cudaMemset(c->flags, 0, 2 * kMaxRanks * sizeof(unsigned)) != cudaSuccess) return QI_ERR_CUDA;
    c->epoch = 0;
  }
  if (!c->handles && dev_malloc(&c->handles, (kMaxRanks + 1) * 3 * kH + sizeof(int) * 2) != cudaSuccess)
    return QI_ERR_OOM;
  cudaIpcMemHandle_t mine[3];
  // QI_PEER_EXCHANGE=0 selects the NCCL exchanges (the same on every rank)
  const char* env = getenv("QI_PEER_EXCHANGE");
  const bool want = !(env && env[0] == '0');
  int ok = want && cudaIpcGetMemHandle(&mine[0], c->buf[B_QKVH]) == cudaSuccess &&
           cudaIpcGetMemHandle(&mine[1], c->buf[B_O]) == cudaSuccess &&
           cudaIpcGetMemHandle(&mine[2], c->flags) == cudaSuccess;
  char* hd = static_cast<char*>(c->handles);  // [mine 3][all P x 3][ok, ok_min]
  if (cudaMemcpyAsync(hd, mine, 3 * kH, cudaMemcpyHostToDevice, f.s) != cudaSuccess) return QI_ERR_CUDA;
  QI_NCCL(c, ncclAllGather(hd, hd + 3 * kH, 3 * kH, ncclUint8, c->comm, f.s));
  std::vector<cudaIpcMemHandle_t> all(static_cast<size_t>(P) * 3);
  if (cudaMemcpyAsync(all.data(), hd + 3 * kH, static_cast<size_t>(P) * 3 * kH, cudaMemcpyDeviceToHost, f.s) !=
          cudaSuccess ||
      cudaStreamSynchronize(f.s) != cudaSuccess)
    return QI_ERR_CUDA;
  PeerSet ps = {};
  ps.P = P;
  ps.rank = me;
  for (int q = 0; q < P && ok; ++q) {
    if (q == me) {
      ps.qkvh[q] = c->buf[B_QKVH];
      ps.o[q] = c->buf[B_O];
      ps.flags[q] = c->flags;
      continue;
    }
    void* ptr[3] = {};
    for (int k = 0; k < 3 && ok; ++k) {
      if (cudaIpcOpenMemHandle(&ptr[k], all[static_cast<size_t>(q) * 3 + k], cudaIpcMemLazyEnablePeerAccess) !=
          cudaSuccess) {
        cudaGetLastError();
        ok = 0;
        break;
      }
      c->peer_opened.push_back(ptr[k]);
    }
    ps.qkvh[q] = ptr[0];
    ps.o[q] = ptr[1];
    ps.flags[q] = static_cast<unsigned*>(ptr[2]);
  }
  // every rank must take the same path
  int* okd = reinterpret_cast<int*>(hd + (kMaxRanks + 1) * 3 * kH);
  int ok_all = 0;
  if (cudaMemcpyAsync(okd, &ok, sizeof(int), cudaMemcpyHostToDevice, f.s) != cudaSuccess) return QI_ERR_CUDA;
  QI_NCCL(c, ncclAllReduce(okd, okd + 1, 1, ncclInt32, ncclMin, c->comm, f.s));
  if (cudaMemcpyAsync(&ok_all, okd + 1, sizeof(int), cudaMemcpyDeviceToHost, f.s) != cudaSuccess ||
      cudaStreamSynchronize(f.s) != cudaSuccess)
    return QI_ERR_CUDA;
  if (!ok_all) c->close_peers();
  c->peers = ps;
  c->peers_ready = ok_all != 0;
  c->peer_key[0] = key[0];
  c->peer_key[1] = key[1];
  c->peer_key[2] = key[2];
  f.direct = c->peers_ready;
  return QI_OK;
}

// One launch (or a fixed group) per QI_LAUNCH; with profiling on, an event
// pair brackets it on the stream and is resolved in qi_ctx_profile.
#define QI_LAUNCH(stage, count, expr)        \
  do {                                       \
    qi_ctx* c_ = f.c;                        \
    cudaEvent_t e0 = nullptr, e1 = nullptr;  \
    if (c_->profiling) {                     \
      e0 = c_->ev();                         \
      e1 = c_->ev();                         \
      cudaEventRecord(e0, f.s);              \
    }                                        \
    QI_TRY(expr);                            \
    if (c_->profiling) {                     \
      cudaEventRecord(e1, f.s);              \
      c_->pending.push_back({stage, {e0, e1}}); \
    }                                        \
    f.n += (count);                          \
  } while (0)

int fwd_init(Fwd& f, qi_ctx* c, const qi_model* m, int nb, int n_img, int n_txt, void* stream) {
  f.c = c;
  f.m = m;
  f.s = S_(stream);
  f.nb = nb;
  f.n_img = n_img;
  f.n_txt = n_txt;
  f.S = n_img + n_txt;
  if (c->comm_failed) return QI_ERR_NCCL;  // the group was aborted: rejoin with qi_ctx_set_comm
  if (!c->side.s) {
    if (cudaStreamCreateWithFlags(&c->side.s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->side.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&c->side.join, cudaEventDisableTiming) != cudaSuccess)
      return QI_ERR_CUDA;
  }
  f.P = c->usize;
  f.rank = c->urank;
  f.Hl = kHeads / f.P;
  f.map = make_map(f.P, n_txt, n_img);
  f.img_lo = f.map.img_lo[f.rank];
  f.n_img_l = f.map.n_img_l(f.rank);
  f.txt_lo = f.map.txt_lo[f.rank];
  f.n_txt_l = f.map.n_txt_l(f.rank);
  f.BH = nb * f.Hl;
  f.Mi = static_cast<long long>(nb) * f.n_img_l;
  f.Mt = static_cast<long long>(nb) * f.n_txt_l;
  f.Ma = f.Mi + f.Mt;
  const size_t hs = static_cast<size_t>(f.BH) * f.S * kHeadDim;
  QI_TRY(c->ensure(B_PATCH, f.Mi * kPatchDim * 2));
  QI_TRY(c->ensure(B_TEMB256, 256 * 4));
  QI_TRY(c->ensure(B_TACT, kDim));
  QI_TRY(c->ensure(B_TACT_S, 16));
  QI_TRY(c->ensure(B_T1, kDim * 4));
  QI_TRY(c->ensure(B_TEMB, kDim * 4));
  QI_TRY(c->ensure(B_TSILU, kDim * 4));
  QI_TRY(c->ensure(B_MODS, static_cast<size_t>(m->mod.N) * 4));
  QI_TRY(c->ensure(B_ADA, 2 * kDim * 4));
  QI_TRY(c->ensure(B_X, f.Ma * kDim * 4));
  QI_TRY(c->ensure(B_TXTN, f.Mt * kTxtDim * 2));
  QI_TRY(c->ensure(B_ACT, f.Ma * kMlp));
  QI_TRY(c->ensure(B_ACT_S, f.Ma * 4));
  QI_TRY(c->ensure(B_QKV, f.Ma * 3 * kDim * 4));
  QI_TRY(c->ensure(B_QKVH, 3 * hs * 2));
  QI_TRY(c->ensure(B_QC, hs));
  QI_TRY(c->ensure(B_KC, hs));
  QI_TRY(c->ensure(B_QS, static_cast<size_t>(f.BH) * ((f.S + 127) / 128) * 32 * 4));
  QI_TRY(c->ensure(B_KS, static_cast<size_t>(f.BH) * ((f.S + 63) / 64) * 4 * 4));
  QI_TRY(c->ensure(B_KMEAN, static_cast<size_t>(f.BH) * kHeadDim * 4));
  if (c->attn_fp8) {
    const int s_pad = (f.S + 15) & ~15;
    QI_TRY(c->ensure(B_V8, static_cast<size_t>(f.BH) * kHeadDim * s_pad));
    QI_TRY(c->ensure(B_VAMAX, static_cast<size_t>(f.BH) * kHeadDim * 4));
    QI_TRY(c->ensure(B_VS, static_cast<size_t>(f.BH) * kHeadDim * 4));
  }
  QI_TRY(c->ensure(B_O, f.Ma * kDim * 2));
  QI_TRY(c->ensure(B_H, f.Ma * kMlp * 4));
  QI_TRY(c->ensure(B_FIN, f.Mi * kDim * 2));
  QI_TRY(c->ensure(B_PROJ, f.Mi * kPatchDim * 4));
  if (f.P > 1) {
    QI_TRY(setup_peers(f));
    if (!f.direct) {  // NCCL exchange buffers
      QI_TRY(c->ensure(B_SEND1, f.Ma * 3 * kDim * 2));
      QI_TRY(c->ensure(B_RECV1, 3 * hs * 2));
      QI_TRY(c->ensure(B_SEND2, hs * 2));
      QI_TRY(c->ensure(B_RECV2, f.Ma * kDim * 2));
    }
    QI_TRY(c->ensure(B_PROJF, static_cast<size_t>(nb) * n_img * kPatchDim * 4));
  }
  return QI_OK;
}

// Timestep MLP (transformer.cu:330-349), all modulation vectors of the
// forward (transformer.cu:506-515: they depend only on t) and the output
// AdaLN embedding (transformer.cu:874-877).
int fwd_modulation(Fwd& f, float timestep, bool block_mods = true) {
  qi_ctx* c = f.c;
  const qi_model* m = f.m;
  cudaStream_t s = f.s;
  int8_t* tact = c->p<int8_t>(B_TACT);
  float* tact_s = c->p<float>(B_TACT_S);
  QI_LAUNCH(QI_PROF_PRE, 1, timestep_embedding_launch(timestep, c->p<float>(B_TEMB256), s));
  RowSeg seg{c->buf[B_TEMB256], 256, nullptr, nullptr, 1};
  QI_LAUNCH(QI_PROF_PRE, 1, rowquant_launch(kSrcF32, 256, 256, &seg, 1, tact, tact_s, 0.0f, s));
  GemvJob j1{m->t1.w, m->t1.s, m->t1.b, c->p<float>(B_T1), kDim};
  QI_LAUNCH(QI_PROF_PRE, 1, gemv_i8_launch(tact, tact_s, 256, &j1, 1, s));
  QI_LAUNCH(QI_PROF_PRE, 1, silu_launch(c->p<float>(B_T1), c->p<float>(B_T1), kDim, s));
  RowSeg seg2{c->buf[B_T1], kDim, nullptr, nullptr, 1};
  QI_LAUNCH(QI_PROF_PRE, 1, rowquant_launch(kSrcF32, kDim, 1024, &seg2, 1, tact, tact_s, 0.0f, s));
  GemvJob j2{m->t2.w, m->t2.s, m->t2.b, c->p<float>(B_TEMB), kDim};
  QI_LAUNCH(QI_PROF_PRE, 1, gemv_i8_launch(tact, tact_s, kDim, &j2, 1, s));
  QI_LAUNCH(QI_PROF_PRE, 1, silu_launch(c->p<float>(B_TEMB), c->p<float>(B_TSILU), kDim, s));
  RowSeg seg3{c->buf[B_TSILU], kDim, nullptr, nullptr, 1};
  QI_LAUNCH(QI_PROF_PRE, 1, rowquant_launch(kSrcF32, kDim, 1024, &seg3, 1, tact, tact_s, 0.0f, s));
  // The stacked modulation GEMV (6.8 GB of weights) is the same on every rank
  // of a head-parallel group: each rank computes 1/P of its rows and the group
  // all-gathers them.  Every row's arithmetic is unchanged, so the vectors are
  // bit-identical to one GPU's.
  float* mods = c->p<float>(B_MODS);
  if (!block_mods) {
    // output head only (qi_spectrum_output): no block modulation vectors
  } else if (f.P > 1 && m->mod.N % f.P == 0) {
    const long long cnt = m->mod.N / f.P, lo = cnt * f.rank;
    GemvJob jm{m->mod.w + lo * kDim, m->mod.s + lo, m->mod.b ? m->mod.b + lo : nullptr, mods + lo,
               static_cast<int>(cnt)};
    QI_LAUNCH(QI_PROF_PRE, 1, gemv_i8_launch(tact, tact_s, kDim, &jm, 1, s));
    QI_LAUNCH(QI_PROF_EXCHANGE, 0, nccl_settle(c, ncclAllGather(mods + lo, mods, cnt, ncclFloat32, c->comm, s)));
  } else {
    GemvJob jm{m->mod.w, m->mod.s, m->mod.b, mods, m->mod.N};
    QI_LAUNCH(QI_PROF_PRE, 1, gemv_i8_launch(tact, tact_s, kDim, &jm, 1, s));
  }
  QI_LAUNCH(QI_PROF_PRE, 1,
            gemv_bf16_launch(c->p<float>(B_TSILU), m->norm_out_w, m->norm_out_b, c->p<float>(B_ADA), 2 * kDim, kDim, s));
  return QI_OK;
}

// patchify + img_in (BF16) and txt_norm + txt_in (BF16) (transformer.cu:266-290, 396-422).
int fwd_inputs(Fwd& f, const void* x, const void* ctx_txt, int H, int W, float* x_img, float* x_txt) {
  qi_ctx* c = f.c;
  const qi_model* m = f.m;
  cudaStream_t s = f.s;
  // this rank's image patches and text rows of every batch entry
  QI_LAUNCH(QI_PROF_PRE, 1, patchify_launch(x, c->buf[B_PATCH], f.nb, H, W, f.img_lo, f.n_img_l, s));
  if (f.Mi > 0) {
    GemmBf16Desc d{c->buf[B_PATCH], m->img_in_w, m->img_in_b, x_img, static_cast<int>(f.Mi), kDim, kPatchDim, kDim};
    QI_LAUNCH(QI_PROF_PRE, 1, gemm_bf16_launch(d, s, c->err, c->num_sms));
  }
  if (f.Mt > 0) {
    const __nv_bfloat16* ctx_in = static_cast<const __nv_bfloat16*>(ctx_txt);
    __nv_bfloat16* txtn = c->p<__nv_bfloat16>(B_TXTN);
    if (f.P == 1) {
      QI_LAUNCH(QI_PROF_PRE, 1, rmsnorm_bf16_launch(ctx_in, m->txt_norm, txtn, static_cast<int>(f.Mt), kTxtDim, 1e-6f, s));
    } else {
      for (int b = 0; b < f.nb; ++b)
        QI_LAUNCH(QI_PROF_PRE, 1,
                  rmsnorm_bf16_launch(ctx_in + (static_cast<size_t>(b) * f.n_txt + f.txt_lo) * kTxtDim, m->txt_norm,
                                      txtn + static_cast<size_t>(b) * f.n_txt_l * kTxtDim, f.n_txt_l, kTxtDim, 1e-6f, s));
    }
    GemmBf16Desc e{c->buf[B_TXTN], m->txt_in_w, m->txt_in_b, x_txt, static_cast<int>(f.Mt), kDim, kTxtDim, kDim};
    QI_LAUNCH(QI_PROF_PRE, 1, gemm_bf16_launch(e, s, c->err, c->num_sms));
  }
  return QI_OK;
}

// The double-stream blocks [b0, b1) on residual streams x_img [Mi,3072] and
// x_txt [Mt,3072] (transformer.cu:497-836).
int fwd_blocks(Fwd& f, float* x_img, float* x_txt, const float* pe, int b0, int b1) {
  qi_ctx* c = f.c;
  const qi_model* m = f.m;
  cudaStream_t s = f.s;
  const long long Mi = f.Mi, Mt = f.Mt, Ma = f.Ma;
  const int nb = f.nb, n_img = f.n_img, n_txt = f.n_txt, S = f.S, BH = f.BH;
  if (Ma == 0) return QI_ERR_UNSUPPORTED;
  int8_t* act = c->p<int8_t>(B_ACT);
  float* act_s = c->p<float>(B_ACT_S);
  const float* mods = c->p<float>(B_MODS);
  float* qkv = c->p<float>(B_QKV);
  float* hbuf = c->p<float>(B_H);
  for (int bi = b0; bi < b1; ++bi) {
    const BlockW& B = m->blocks[bi];
    const float* mi = mods + (static_cast<size_t>(bi) * 2 + 0) * 6 * kDim;
    const float* mt = mods + (static_cast<size_t>(bi) * 2 + 1) * 6 * kDim;
    // chunk order [shift1, scale1, gate1, shift2, scale2, gate2] (transformer.cu:529-531, 742-764, 814-817)
    RowSeg ln1[2] = {{x_img, kDim, mi + 0 * kDim, mi + 1 * kDim, static_cast<int>(Mi)},
                     {x_txt, kDim, mt + 0 * kDim, mt + 1 * kDim, static_cast<int>(Mt)}};
    QI_LAUNCH(QI_PROF_QUANT_LN, 1, rowquant_launch(kSrcLnMod, kDim, 1024, ln1, 2, act, act_s, 1e-6f, s));
    GemmDesc gq[2] = {{act, act_s, B.qkv[0].w, B.qkv[0].s, B.qkv[0].b, qkv, nullptr, static_cast<int>(Mi), 3 * kDim,
                       kDim, 3 * kDim},
                      {act + Mi * kDim, act_s + Mi, B.qkv[1].w, B.qkv[1].s, B.qkv[1].b, qkv + Mi * 3 * kDim, nullptr,
                       static_cast<int>(Mt), 3 * kDim, kDim, 3 * kDim}};
    const bool par = f.P > 1, direct = par && f.direct;
    __half* qkvh = c->p<__half>(B_QKVH);
    const size_t hs = static_cast<size_t>(BH) * S * kHeadDim;
    QkvPostArgs qa{qkv,       qkv + Mi * 3 * kDim, B.norms, B.norms + kHeadDim, B.norms + 2 * kHeadDim,
                   B.norms + 3 * kHeadDim, pe, par ? c->buf[B_SEND1] : qkvh, nb, n_img, n_txt, f.img_lo, f.n_img_l,
                   f.txt_lo, f.n_txt_l, f.Hl, direct ? 1 : 0};
    if (direct)
      for (int q = 0; q < f.P; ++q) qa.peer_qkvh[q] = c->peers.qkvh[q];
    if (c->qkv_fused && gemm_qkv_fusable(gq, 2, c->num_sms)) {
      // q/k RMSNorm + RoPE + FP16 head-major store in the projection's epilogue
      QI_LAUNCH(QI_PROF_GEMM_QKV, 1, gemm_qkv_launch(gq, 2, qa, s, c->err, c->num_sms));
    } else {
      QI_LAUNCH(QI_PROF_GEMM_QKV, 1, gemm_i8_launch(gq, 2, kEpiStore, s, c->err, c->num_sms));
      QI_LAUNCH(QI_PROF_QKV_POST, 1, qkv_post_launch(qa, s));
    }
    if (direct) {  // every rank has stored its rows of this rank's heads
      QI_LAUNCH(QI_PROF_EXCHANGE, 1, peer_barrier_launch(c->peers, 0, ++c->epoch, c->err, s));
    } else if (par) {  // every token of this rank's heads
      QI_LAUNCH(QI_PROF_EXCHANGE, 0, exchange(c, 0, nb, f.map, c->buf[B_SEND1], c->buf[B_RECV1], s));
      QI_LAUNCH(QI_PROF_EXCHANGE, 1, ulysses_gather_qkv_launch(c->buf[B_RECV1], qkvh, nb, f.Hl, n_txt, f.map, s));
    }
    const int s_pad = (S + 15) & ~15;
    if (c->attn_fp8)
      QI_LAUNCH(QI_PROF_SAGE_QUANT, 6,
                sage_quantize_fp8pv_launch(qkvh, qkvh + hs, qkvh + 2 * hs, BH, S, c->p<float>(B_KMEAN),
                                           c->p<int8_t>(B_QC), c->p<float>(B_QS), c->p<int8_t>(B_KC),
                                           c->p<float>(B_KS), c->p<uint8_t>(B_V8), s_pad, c->p<float>(B_VAMAX),
                                           c->p<float>(B_VS), s, &c->side));
    else
      QI_LAUNCH(QI_PROF_SAGE_QUANT, 3,
                sage_quantize_launch(qkvh, qkvh + hs, BH, S, c->p<float>(B_KMEAN), c->p<int8_t>(B_QC),
                                     c->p<float>(B_QS), c->p<int8_t>(B_KC), c->p<float>(B_KS), s, &c->side));
    AttnArgs aa{c->p<int8_t>(B_QC), c->p<float>(B_QS), c->p<int8_t>(B_KC), c->p<float>(B_KS), qkvh + 2 * hs,
                par && !direct ? c->buf[B_SEND2] : c->buf[B_O], BH, S, f.Hl, 1.0f / sqrtf(128.0f),
                direct ? 3 : (par ? 2 : 1), nb, n_img, n_txt, f.map};
    if (direct) {
      for (int q = 0; q < f.P; ++q) aa.peer_o[q] = c->peers.o[q];
      aa.head_base = f.rank * f.Hl;
    }
    if (c->attn_fp8) {
      aa.v = c->buf[B_V8];
      aa.fp8 = 1;
      aa.vs = c->p<float>(B_VS);
      aa.s_pad = s_pad;
    }
    QI_LAUNCH(QI_PROF_ATTENTION, 1, attention_launch(aa, s, c->err));
    if (direct) {  // every rank has stored its heads of this rank's rows
      QI_LAUNCH(QI_PROF_EXCHANGE, 1, peer_barrier_launch(c->peers, 1, ++c->epoch, c->err, s));
    } else if (par) {  // back to the token owners, token-major
      QI_LAUNCH(QI_PROF_EXCHANGE, 0, exchange(c, 1, nb, f.map, c->buf[B_SEND2], c->buf[B_RECV2], s));
      QI_LAUNCH(QI_PROF_EXCHANGE, 1, ulysses_gather_o_launch(c->buf[B_RECV2], c->buf[B_O], nb, f.Hl, f.rank, f.map, s));
    }
    RowSeg os{c->buf[B_O], kDim, nullptr, nullptr, static_cast<int>(Ma)};
    QI_LAUNCH(QI_PROF_QUANT_O, 1, rowquant_launch(kSrcF16, kDim, 1024, &os, 1, act, act_s, 0.0f, s));
    GemmDesc go[2] = {{act, act_s, B.out[0].w, B.out[0].s, B.out[0].b, x_img, mi + 2 * kDim, static_cast<int>(Mi), kDim,
                       kDim, kDim},
                      {act + Mi * kDim, act_s + Mi, B.out[1].w, B.out[1].s, B.out[1].b, x_txt, mt + 2 * kDim,
                       static_cast<int>(Mt), kDim, kDim, kDim}};
    QI_LAUNCH(QI_PROF_GEMM_OUT, 1, gemm_i8_launch(go, 2, kEpiResidual, s, c->err, c->num_sms));
    RowSeg ln2[2] = {{x_img, kDim, mi + 3 * kDim, mi + 4 * kDim, static_cast<int>(Mi)},
                     {x_txt, kDim, mt + 3 * kDim, mt + 4 * kDim, static_cast<int>(Mt)}};
    QI_LAUNCH(QI_PROF_QUANT_LN, 1, rowquant_launch(kSrcLnMod, kDim, 1024, ln2, 2, act, act_s, 1e-6f, s));
    GemmDesc g1[2] = {{act, act_s, B.fc1[0].w, B.fc1[0].s, B.fc1[0].b, hbuf, nullptr, static_cast<int>(Mi), kMlp, kDim,
                       kMlp},
                      {act + Mi * kDim, act_s + Mi, B.fc1[1].w, B.fc1[1].s, B.fc1[1].b, hbuf + Mi * kMlp, nullptr,
                       static_cast<int>(Mt), kMlp, kDim, kMlp}};
    QI_LAUNCH(QI_PROF_GEMM_FC1, 1, gemm_i8_launch(g1, 2, kEpiGelu, s, c->err, c->num_sms));
    RowSeg hs2{hbuf, kMlp, nullptr, nullptr, static_cast<int>(Ma)};
    QI_LAUNCH(QI_PROF_QUANT_H, 1, rowquant_launch(kSrcF32, kMlp, 4096, &hs2, 1, act, act_s, 0.0f, s));
    GemmDesc g2[2] = {{act, act_s, B.fc2[0].w, B.fc2[0].s, B.fc2[0].b, x_img, mi + 5 * kDim, static_cast<int>(Mi), kDim,
                       kMlp, kDim},
                      {act + Mi * kMlp, act_s + Mi, B.fc2[1].w, B.fc2[1].s, B.fc2[1].b, x_txt, mt + 5 * kDim,
                       static_cast<int>(Mt), kDim, kMlp, kDim}};
    QI_LAUNCH(QI_PROF_GEMM_FC2, 1, gemm_i8_launch(g2, 2, kEpiResidual, s, c->err, c->num_sms));
  }
  return QI_OK;
}

// AdaLayerNormContinuous (scale = first half, shift = second half,
// transformer.cu:881-884) -> BF16 -> proj_out -> unpatchify (:889-926).
int fwd_output(Fwd& f, const float* x_img, int H, int W, void* out) {
  qi_ctx* c = f.c;
  const qi_model* m = f.m;
  cudaStream_t s = f.s;
  const float* ada = c->p<float>(B_ADA);
  QI_LAUNCH(QI_PROF_POST, 1,
            layernorm_mod_launch(x_img, ada + kDim, ada, static_cast<int>(f.Mi), kDim, 1e-6f, nullptr, c->buf[B_FIN], s));
  if (f.Mi > 0) {
    GemmBf16Desc pd{c->buf[B_FIN], m->proj_out_w, m->proj_out_b, c->p<float>(B_PROJ), static_cast<int>(f.Mi),
                    kPatchDim, kDim, kPatchDim};
    QI_LAUNCH(QI_PROF_POST, 1, gemm_bf16_launch(pd, s, c->err, c->num_sms));
  }
  const float* proj = c->p<float>(B_PROJ);
  if (f.P > 1) {  // every rank's image rows, for the full output on every rank
    float* full = c->p<float>(B_PROJF);
    const size_t rowb = kPatchDim * sizeof(float);
    for (int b = 0; b < f.nb; ++b)
      if (f.n_img_l &&
          cudaMemcpyAsync(full + (static_cast<size_t>(b) * f.n_img + f.img_lo) * kPatchDim,
                          proj + static_cast<size_t>(b) * f.n_img_l * kPatchDim, f.n_img_l * rowb,
                          cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return QI_ERR_CUDA;
    QI_NCCL(c, ncclGroupStart());
    for (int q = 0; q < f.P; ++q) {
      if (q == f.rank) continue;
      const int nq = f.map.n_img_l(q);
      for (int b = 0; b < f.nb; ++b) {
        if (f.n_img_l)
          QI_NCCL(c, ncclSend(proj + static_cast<size_t>(b) * f.n_img_l * kPatchDim,
                              static_cast<size_t>(f.n_img_l) * kPatchDim, ncclFloat32, q, c->comm, s));
        if (nq)
          QI_NCCL(c, ncclRecv(full + (static_cast<size_t>(b) * f.n_img + f.map.img_lo[q]) * kPatchDim,
                              static_cast<size_t>(nq) * kPatchDim, ncclFloat32, q, c->comm, s));
      }
    }
    QI_NCCL(c, ncclGroupEnd());
    proj = full;
  }
  QI_LAUNCH(QI_PROF_POST, 1, unpatchify_launch(proj, out, f.nb, H, W, s));
  return QI_OK;
}
#undef QI_LAUNCH
}  // namespace

extern "C" int qi_exchange_plan(int which, int nb, int n_txt, int n_img, int nranks, int rank, long long* send_off,
                                long long* send_bytes, long long* recv_off, long long* recv_bytes) {
  if ((which != 0 && which != 1) || nb < 1 || n_txt < 0 || n_img < 0 || nranks < 1 || nranks > kMaxRanks ||
      kHeads % nranks || rank < 0 || rank >= nranks || !send_off || !send_bytes || !recv_off || !recv_bytes)
    return QI_ERR_ARG;
  exchange_plan(which, nb, make_map(nranks, n_txt, n_img), rank, send_off, send_bytes, recv_off, recv_bytes);
  return QI_OK;
}

extern "C" int qi_forward(qi_ctx* c, const qi_model* m, int nb, const void* x, float timestep, const void* ctx_txt,
                          int n_txt, const float* pe, int H, int W, void* out, void* stream) {
  if (!c || !m || !x || !ctx_txt || !pe || !out) return QI_ERR_ARG;
  if (nb < 1 || nb > 8 || n_txt < 1 || H < 2 || W < 2 || (H & 1) || (W & 1)) return QI_ERR_ARG;
  if (c->capture && c->usize > 1) return QI_ERR_UNSUPPORTED;  // each rank holds only its image rows
  Fwd f;
  QI_TRY(fwd_init(f, c, m, nb, (H / 2) * (W / 2), n_txt, stream));
  float* x_img = c->p<float>(B_X);
  float* x_txt = x_img + f.Mi * kDim;
  QI_TRY(fwd_inputs(f, x, ctx_txt, H, W, x_img, x_txt));
  QI_TRY(fwd_modulation(f, timestep));
  QI_TRY(fwd_blocks(f, x_img, x_txt, pe, 0, m->nblocks));
  if (c->capture &&  // the final image hidden state, before norm_out (transformer.cu:864-871)
      cudaMemcpyAsync(c->capture, x_img, static_cast<size_t>(f.Mi) * kDim * sizeof(float), cudaMemcpyDeviceToDevice,
                      f.s) != cudaSuccess)
    return QI_ERR_CUDA;
  QI_TRY(fwd_output(f, x_img, H, W, out));
  c->launches = f.n;
  return QI_OK;
}

extern "C" int qi_ctx_set_hidden_capture(qi_ctx* c, float* hidden_out) {
  if (!c) return QI_ERR_ARG;
  if (hidden_out && (reinterpret_cast<uintptr_t>(hidden_out) & 15)) return QI_ERR_ALIGN;
  c->capture = hidden_out;
  return QI_OK;
}

// The output head on a given final image hidden state: timestep MLP,
// norm_out modulation, AdaLayerNormContinuous, proj_out, unpatchify -- the
// reference's transformer_spectrum_output (transformer.cu:939-1028), here the
// same kernels as the end of qi_forward, so a hidden state captured from a
// forward gives that forward's output bit for bit.
extern "C" int qi_spectrum_output(qi_ctx* c, const qi_model* m, int nb, const float* hidden, float timestep, int H,
                                  int W, void* out, void* stream) {
  if (!c || !m || !hidden || !out) return QI_ERR_ARG;
  if (nb < 1 || nb > 8 || H < 2 || W < 2 || (H & 1) || (W & 1)) return QI_ERR_ARG;
  if (c->usize > 1) return QI_ERR_UNSUPPORTED;
  if (reinterpret_cast<uintptr_t>(hidden) & 15) return QI_ERR_ALIGN;
  Fwd f;
  QI_TRY(fwd_init(f, c, m, nb, (H / 2) * (W / 2), 1, stream));
  QI_TRY(fwd_modulation(f, timestep, false));
  QI_TRY(fwd_output(f, hidden, H, W, out));
  c->launches = f.n;
  return QI_OK;
}

extern "C" int qi_forward_blocks(qi_ctx* c, const qi_model* m, int nb, int n_img, int n_txt, float* img, float* txt,
                                 float timestep, const float* pe, int block_begin, int block_end, void* stream) {
  if (!c || !m || !img || !txt || !pe) return QI_ERR_ARG;
  if (nb < 1 || nb > 8 || n_img < 1 || n_txt < 1 || block_begin < 0 || block_end > m->nblocks ||
      block_begin > block_end)
    return QI_ERR_ARG;
  if (c->usize > 1) return QI_ERR_UNSUPPORTED;  // the caller-owned streams are whole sequences
  if ((reinterpret_cast<uintptr_t>(img) & 15) || (reinterpret_cast<uintptr_t>(txt) & 15)) return QI_ERR_ALIGN;
  Fwd f;
  QI_TRY(fwd_init(f, c, m, nb, n_img, n_txt, stream));
  QI_TRY(fwd_modulation(f, timestep));
  QI_TRY(fwd_blocks(f, img, txt, pe, block_begin, block_end));
  c->launches = f.n;
  return QI_OK;
}
