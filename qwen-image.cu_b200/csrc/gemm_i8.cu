// gemm_i8.cu -- W8A8 (and BF16) linear layers on the 5th-generation tensor cores.
//
// Replaces the reference's three-launch INT8 linear (cuda_kernels.cu:2674-2773:
// FWHT+quant, cublasGemmEx S8xS8->S32 into HBM, dequant(+GELU) kernel) with one
// persistent tcgen05 kernel per layer group whose epilogue applies the
// reference's dequantisation  out = acc * s_act[m] * s_w[n] + bias[n]
// (cuda_kernels.cu:2623-2668) straight from TMEM, optionally GELU-tanh, or the
// gated residual update x += gate[n] * out (gate_add_fp32f, cuda_kernels.cu:
// 2181-2189), so the INT32 accumulators never touch HBM.
//
// Layout: A = activation codes [M, K] int8 row-major, B = weight codes [N, K]
// int8 row-major (quantize.cu's "<name>" I8 tensor), both K-major.  Tiles are
// 128 x 256 x 128 bytes; a 4-stage TMA ring (48 KB per stage, 128-byte
// swizzle) feeds tcgen05.mma.kind::i8 (M=128, N=256, K=32); the 128x256 S32
// accumulator lives in TMEM, double buffered (512 columns) so the epilogue of
// one tile overlaps the main loop of the next.
//
// Warp roles (192 threads): warp 0 TMA producer, warp 1 MMA issuer (and TMEM
// owner), warps 2-5 epilogue (one TMEM lane = one output row per thread); the
// epilogue writes through swizzled shared-memory sub-tiles and TMA stores, so
// global writes are full lines instead of one row per lane.
#include "qi_internal.h"
#include "sm100.cuh"

// Smallest K that runs on CTA pairs (a build-time knob for measurements).
#ifndef QI_GEMM_PAIR_MIN_K
#define QI_GEMM_PAIR_MIN_K 0
#endif

namespace qi {

namespace gemm {
constexpr int BM = 128, BN = 256, BK = 128, STAGES = 4;
constexpr int A_BYTES = BM * BK;                 // 16 KB
constexpr int B_BYTES = BN * BK;                 // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;   // 48 KB
constexpr int TMEM_COLS = 512;                   // 2 accumulators x 256 columns
constexpr int THREADS = 192;
constexpr int EPI_WARPS = 4;
constexpr int EPI_BUF = 32 * 32 * 4;                  // one warp's 32x32 FP32 sub-tile
constexpr int EPI_BYTES = EPI_WARPS * 2 * EPI_BUF;    // double buffered per warp: 32 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
}  // namespace gemm

struct alignas(64) GemmProblemDev {
  CUtensorMap tmA;
  CUtensorMap tmB;
  CUtensorMap tmO;  // FP32 output [M, N] (ldo), 32x32 boxes, 128-byte swizzle
  const float* sa;
  const float* sw;
  const __nv_bfloat16* bias;
  float* out;
  const float* gate;
  int M, N, K, ldo;
  int tiles_n, tile_begin, tile_end, pad;
};

struct alignas(64) GemmArgsDev {
  GemmProblemDev p[2];
  int nprob;
  int total_tiles;
  int epi;
  int* err;
  // L2 eviction hints on the CTA-pair kernel's copies: 0 none; 1 the output
  // (and residual) tiles and, for K >= 8192, the A panels evict_first (each is
  // used once or by the tiles running at the same time), so the weight panels
  // that every row block re-reads stay in L2; 2 also the weights evict_last
  int l2;
  QkvPostArgs qp;  // kEpiQkv: qkv_post's parameters (its qkv_img / qkv_txt unused)
  CUtensorMap tmPE;  // kEpiQkv: the RoPE table [nb * S][256] FP32, 32 x 32 boxes, 128-byte swizzle
};

__device__ __forceinline__ float gelu_tanh_dev(float v) {
  // Same expression as dequantize_bias_gelu_kernel (cuda_kernels.cu:2656-2658).
  const float c = 0.7978845608f;
  float inner = c * (v + 0.044715f * v * v * v);
  return 0.5f * v * (1.0f + tanhf(inner));
}

// Residual-load bookkeeping of one epilogue warp across tiles.
struct EpiState {
  uint32_t xphase = 0;    // parity bit per staging buffer
  uint32_t xpending = 0;  // buffers with a residual load issued and not yet waited
  // kEpiQkv's RoPE-row ring (the filling warp): parity of the next "slot
  // empty" completion per slot, and the slots filled at least once
  uint32_t ephase = 0;
  uint32_t eused = 0;
};

// One accumulator tile: this warp's 32 rows (TMEM lane quarter) of the 128
// rows starting at row0, columns n0 .. n0+255.  Per 32-column chunk: TMEM ->
// registers (thread = row) -> dequant (+GELU / gated residual) -> the warp's
// swizzled 32x32 FP32 staging buffer -> one TMA tensor store.  Two buffers
// per warp; the residual sub-tile of the next chunk is TMA-loaded into the
// free buffer while this one is computed.  False when a bounded wait gave up.
template <bool BF16>
__device__ __forceinline__ bool epilogue_tile(const GemmArgsDev& args, const GemmProblemDev& P, int row0, int n0,
                                              int buf, uint32_t acc_phase, uint32_t tmem_base, uint8_t* ebuf,
                                              uint64_t* xb, uint64_t* tfull, EpiState& es, volatile int* abort_flag,
                                              int quarter, int lane, int c_begin, int c_limit) {
  using namespace gemm;
  constexpr int NCH = BN / 32;
  const int r0 = row0 + quarter * 32;  // first output row of this warp
  const bool resid = args.epi == kEpiResidual;
  // this warp's 32-column chunks of the tile: [c_begin, nch)
  const int nch = min(min(NCH, c_limit), (P.N - n0 + 31) / 32);
  // residual: fetch the first chunk before waiting for the accumulator
  const uint64_t pol_out = args.l2 ? l2_policy_evict_first() : 0ull;  // output / residual tiles
  auto load_out = [&](void* dst, int col, uint64_t* bar) {
    if (args.l2)
      tma_load_2d_hint(dst, &P.tmO, col, r0, bar, pol_out);
    else
      tma_load_2d(dst, &P.tmO, col, r0, bar);
  };
  if (resid && r0 < P.M && c_begin < nch && lane == 0) {
    bulk_wait_read<0>();
    mbar_expect_tx(&xb[c_begin & 1], EPI_BUF);
    load_out(ebuf + (c_begin & 1) * EPI_BUF, n0 + 32 * c_begin, &xb[c_begin & 1]);
    es.xpending |= 1u << (c_begin & 1);
  }
  bool w = mbar_wait(&tfull[buf], acc_phase, abort_flag);
  if (!__all_sync(0xffffffffu, w)) return false;
  tc_fence_after();
  const int grow = r0 + lane;
  const float sa = (grow < P.M && !BF16) ? __ldg(P.sa + grow) : 0.0f;
  const uint32_t taddr_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
  if (r0 >= P.M) return true;  // the whole 32-row slab is past M (all lanes agree)
  // One chunk: dequant (+GELU / gated residual) of `acc` -> staging -> TMA store.
  auto chunk = [&](const uint32_t (&acc)[32], int c) -> bool {
    const int b = c & 1;
    uint8_t* sbuf = ebuf + b * EPI_BUF;
    bool w;
    const int gcol = n0 + c * 32;
    if (resid) {
      // prefetch the next chunk's residual into the other buffer
      if (lane == 0 && c + 1 < nch) {
        bulk_wait_read<0>();
        mbar_expect_tx(&xb[b ^ 1], EPI_BUF);
        load_out(ebuf + (b ^ 1) * EPI_BUF, gcol + 32, &xb[b ^ 1]);
        es.xpending |= 1u << (b ^ 1);
      }
      w = mbar_wait(&xb[b], (es.xphase >> b) & 1, abort_flag);
      es.xphase ^= 1u << b;
      es.xpending &= ~(1u << b);
      if (!__all_sync(0xffffffffu, w)) return false;
    } else {
      // the store issued from this buffer two chunks ago must have read it
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
    }
    float v[32];
    if (BF16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(acc[j]);
    } else {
      const float4* sw4 = reinterpret_cast<const float4*>(P.sw + gcol);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 ws = __ldg(sw4 + j / 4);
        v[j + 0] = static_cast<float>(static_cast<int32_t>(acc[j + 0])) * sa * ws.x;
        v[j + 1] = static_cast<float>(static_cast<int32_t>(acc[j + 1])) * sa * ws.y;
        v[j + 2] = static_cast<float>(static_cast<int32_t>(acc[j + 2])) * sa * ws.z;
        v[j + 3] = static_cast<float>(static_cast<int32_t>(acc[j + 3])) * sa * ws.w;
      }
    }
    if (P.bias) {
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(P.bias + gcol);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float2 bb = __bfloat1622float2(b2[j / 2]);
        v[j] += bb.x;
        v[j + 1] += bb.y;
      }
    }
    if (args.epi == kEpiGelu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh_dev(v[j]);
    }
    // row `lane` of the swizzled sub-tile: 16-byte chunk k at k ^ (lane & 7)
    float4* srow = reinterpret_cast<float4*>(sbuf + lane * 128);
    if (resid) {
      const float4* g4 = reinterpret_cast<const float4*>(P.gate + gcol);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 x = srow[k ^ (lane & 7)];
        const float4 g = __ldg(g4 + k);
        srow[k ^ (lane & 7)] = make_float4(x.x + g.x * v[4 * k + 0], x.y + g.y * v[4 * k + 1],
                                           x.z + g.z * v[4 * k + 2], x.w + g.w * v[4 * k + 3]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k)
        srow[k ^ (lane & 7)] = make_float4(v[4 * k + 0], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (args.l2)
        tma_store_2d_hint(&P.tmO, sbuf, gcol, r0, pol_out);
      else
        tma_store_2d(&P.tmO, sbuf, gcol, r0);
      bulk_commit();
    }
    return true;
  };
  // TMEM loads run one chunk ahead of the dequant: chunk c + 1 is in flight
  // while chunk c is computed (two register buffers, unrolled by two).
  if (c_begin >= nch) return true;
  uint32_t acc0[32], acc1[32];
  tmem_ld32(taddr_row + c_begin * 32, acc0);
#pragma unroll 1
  for (int c = c_begin; c < nch; c += 2) {
    tmem_ld_wait();
    tmem_reg_fence32(acc0);
    if (c + 1 < nch) tmem_ld32(taddr_row + (c + 1) * 32, acc1);
    if (!chunk(acc0, c)) {
      tmem_ld_wait();
      return false;
    }
    if (c + 1 >= nch) break;
    tmem_ld_wait();
    tmem_reg_fence32(acc1);
    if (c + 2 < nch) tmem_ld32(taddr_row + (c + 2) * 32, acc0);
    if (!chunk(acc1, c + 1)) {
      tmem_ld_wait();
      return false;
    }
  }
  return true;
}

// Stores finished and an abandoned residual load landed before the CTA exits.
__device__ __forceinline__ void epilogue_drain(const EpiState& es, uint64_t* xb, int lane, int nbars = 2) {
  if (lane == 0) {
    bulk_wait<0>();
    for (int b = 0; b < nbars; ++b) {
      if (!(es.xpending & (1u << b))) continue;
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&xb[b], (es.xphase >> b) & 1) && global_timer_ns() - t0 < kWaitLimitNs / 4) {
      }
    }
  }
}

// BF16 = false: kind::i8 with the INT8 dequant epilogue.  BF16 = true:
// kind::f16 on BF16 operands (64 elements per 128-byte K block), epilogue
// out = acc + bias (the boundary layers' cuBLAS BF16 GEMM + bias_add_fp32,
// cuda_kernels.cu:4535-4596).
template <bool BF16>
__global__ void __launch_bounds__(gemm::THREADS, 1) gemm_kernel(const __grid_constant__ GemmArgsDev args) {
  using namespace gemm;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sE = smem + STAGES * STAGE_BYTES;  // epilogue staging
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + EPI_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* xfull = tempty + 2;  // [4 warps][2 buffers] residual sub-tile loaded
  uint64_t* drain = xfull + 2 * EPI_WARPS;  // MMA completion before teardown
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    for (int b = 0; b < 2 * EPI_WARPS; ++b) mbar_init(&xfull[b], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    for (int i = 0; i < args.nprob; ++i) {
      tma_prefetch_desc(&args.p[i].tmA);
      tma_prefetch_desc(&args.p[i].tmB);
      tma_prefetch_desc(&args.p[i].tmO);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto locate = [&](int t, int& pi, int& m0, int& n0) {
    pi = (args.nprob > 1 && t >= args.p[0].tile_end) ? 1 : 0;
    const GemmProblemDev& P = args.p[pi];
    int lt = t - P.tile_begin;
    m0 = (lt / P.tiles_n) * BM;
    n0 = (lt % P.tiles_n) * BN;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;  // last phase issued per stage
      bool ok = true;
      for (int t = blockIdx.x; t < args.total_tiles && ok; t += gridDim.x) {
        int pi, m0, n0;
        locate(t, pi, m0, n0);
        const GemmProblemDev& P = args.p[pi];
        const int kblocks = (P.K * (BF16 ? 2 : 1) + BK - 1) / BK;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          const int kc = kb * (BF16 ? BK / 2 : BK);  // element coordinate
          tma_load_2d(sA + stage * A_BYTES, &P.tmA, kc, m0, &full[stage]);
          tma_load_2d(sB + stage * B_BYTES, &P.tmB, kc, n0, &full[stage]);
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kErrTimeoutProducer);
        // Let copies already in flight land before the CTA exits.
        for (int s = 0; s < STAGES; ++s) {
          if (!(issued_mask & (1u << s))) continue;
          const uint32_t par = (issued_parity >> s) & 1u;
          uint64_t t0 = global_timer_ns();
          while (!mbar_try_wait(&full[s], par) && global_timer_ns() - t0 < kWaitLimitNs / 4) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    {
      // the whole warp runs this role: every lane waits (the vote keeps the warp
      // converged) and one elected lane issues each MMA / commit
      auto wait_all = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      const uint32_t idesc = BF16 ? idesc_bf16(BM, BN) : idesc_i8(BM, BN);
      // descriptors built once; an operand at a byte offset is the base plus
      // offset / 16 in the address field (shared addresses stay below 2^18)
      const uint64_t ad0 = umma_desc_sw128(smem_u32(sA), 16, 1024), bd0 = umma_desc_sw128(smem_u32(sB), 16, 1024);
      for (int t = blockIdx.x; t < args.total_tiles && ok; t += gridDim.x, ++local) {
        int pi, m0, n0;
        locate(t, pi, m0, n0);
        const GemmProblemDev& P = args.p[pi];
        const int kblocks = (P.K * (BF16 ? 2 : 1) + BK - 1) / BK;
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_all(&tempty[buf], acc_phase ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_all(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = ad0 + static_cast<uint64_t>((stage * A_BYTES) >> 4);
          const uint64_t bd = bd0 + static_cast<uint64_t>((stage * B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            if (BF16)
              mma_f16_ss_elect(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
            else
              mma_i8_ss_elect(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          mma_commit_elect(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_elect(&tfull[buf]);
      }
      if (!ok && lane == 0) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kErrTimeoutMma);
      }
      __syncwarp();
      // every MMA issued above has completed before TMEM is released
      mma_commit_elect(drain);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(drain, 0) && global_timer_ns() - t0 < kWaitLimitNs / 4) {
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Each warp owns 32 accumulator rows (its TMEM lane quarter).  Per 32-column
    // chunk: TMEM -> registers (thread = row) -> dequant (+GELU / gated
    // residual) -> the warp's swizzled 32x32 FP32 staging buffer -> one TMA
    // tensor store.  Two buffers per warp; the residual sub-tile of the next
    // chunk is TMA-loaded into the free buffer while this one is computed.
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int ew = warp - 2;       // epilogue warp index 0..3
    uint8_t* ebuf = sE + ew * 2 * EPI_BUF;
    uint64_t* xb = xfull + ew * 2;
    EpiState es;
    int local = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < args.total_tiles && ok; t += gridDim.x, ++local) {
      int pi, m0, n0;
      locate(t, pi, m0, n0);
      const int buf = local & 1;
      ok = epilogue_tile<BF16>(args, args.p[pi], m0, n0, buf, (local >> 1) & 1, tmem_base, ebuf, xb, tfull, es,
                               abort_flag, quarter, lane, 0, BN / 32);
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    epilogue_drain(es, xb, lane);
    __syncwarp();
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicCAS(args.err, 0, kErrTimeoutEpilogue);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ fused q/k/v post
// kEpiQkv: one head of the QKV projection for this warp's 32 rows.  With
// N = 3 x 3072 and 256-column tiles, tile columns [c0, c0 + 128) are head h
// of Q, K or V.  The arithmetic is qkv_post_kernel's (glue.cu) applied to the
// values epilogue_tile would have stored:
//   * dequant + bias per 32-column chunk (epilogue_tile's expressions);
//   * Q and K: the sum of squares in the order of rms_norm_fp32_kernel's
//     reduction (cuda_kernels.cu:1656-1688: thread t = element t, each square
//     rounded, shfl_down 16..1 within each warp of 32 elements, then warp 0
//     over the 4 warp sums, i.e. (w0 + w2) + (w1 + w3)), then
//     rsqrt(ss / 128 + eps), x * rms * w and RoPE on interleaved pairs
//     (rope_apply_fp32_to_fp16_kernel, :1935-1963);
//   * V: only rounded to FP16.
// A first pass over TMEM dequantises each 32-column chunk, writes the FP32
// values back over its accumulators and sums their squares; a second pass
// reads them back chunk by chunk, so at most one chunk sits in registers.  The RoPE rows of the 32 rows (16 pairs x 16 bytes per
// row and chunk) come by TMA, as two 32-row x 128-byte boxes with 128-byte
// swizzle, into an NS-slot ring (8 KB per slot) shared by the two warps of
// this TMEM lane quarter (the same 32 rows, the tile's two heads): full[s]
// completes when a chunk has landed in slot s and empty[s] when both warps
// have read it.  The half-0 warp fills chunks 0 .. NS - 1 before it waits for
// the accumulator, and chunk c + NS once chunk c is read, so the copies run
// under the first pass and the earlier chunks.  A slab whose rows straddle
// a batch entry (its table rows are not consecutive) reads the rows per lane
// instead; the values are the same.
// Each chunk's FP16 output goes through a 2 KB per-warp staging buffer, so a
// store instruction writes eight rows' 64 contiguous bytes, to this rank's
// Q/K/V buffer or, direct, the head owner's (peer memory), addressed as in
// qkv_post_kernel.
template <int NS>
__device__ __forceinline__ bool epilogue_qkv(const GemmArgsDev& args, const GemmProblemDev& P, int pi, int row0,
                                             int c0, uint32_t tmem_col, int buf, uint32_t acc_phase,
                                             uint32_t tmem_base, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                             bool filler, uint8_t* obuf, uint64_t* tfull, EpiState& es,
                                             uint32_t tempty_addr, volatile int* abort_flag, int quarter, int lane) {
  static_assert(NS >= 2 && NS <= 4, "ring slots");
  const QkvPostArgs& q = args.qp;
  const int r0 = row0 + quarter * 32;  // first output row of this warp
  // the accumulator buffer is handed back as soon as it has been read
  auto release = [&]() {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(tempty_addr);
  };
  const int which = c0 / kDim, h = (c0 % kDim) / kHeadDim;  // which: 0 Q, 1 K, 2 V
  const int S = q.n_img + q.n_txt, L = q.n_img_l + q.n_txt_l;
  const int n_l = pi == 0 ? q.n_img_l : q.n_txt_l;              // rows per batch entry
  const int base = pi == 0 ? q.n_txt + q.img_lo : q.txt_lo;     // joint position of local row 0
  // the RoPE rows of a slab in one batch entry are consecutive table rows
  const int r_last = min(r0 + 31, P.M - 1);
  const bool tma_pe = which < 2 && r0 < P.M && r0 / n_l == r_last / n_l;
  const int pe_row0 = tma_pe ? (r0 / n_l) * S + base + r0 % n_l : 0;
  const uint64_t pol_out = l2_policy_evict_first(), pol_pe = l2_policy_evict_last();
  // chunk c's 16 pairs of the 32 rows (floats 64c .. 64c + 63) into slot c % NS,
  // once both warps have read what the slot held (filler warp only)
  auto fill = [&](int c) -> bool {
    const int sl = c % NS;
    if (es.eused & (1u << sl)) {
      const bool ok_e = mbar_wait(&empty[sl], (es.ephase >> sl) & 1u, abort_flag);
      if (!__all_sync(0xffffffffu, ok_e)) return false;
      es.ephase ^= 1u << sl;
    }
    es.eused |= 1u << sl;
    if (lane == 0) {
      uint8_t* dstb = ring + sl * 8192;
      fence_proxy_async_smem();  // the lanes' reads of the slot's previous chunk come first
      mbar_expect_tx(&full[sl], 8192);
      tma_load_2d_hint(dstb, &args.tmPE, 64 * c, pe_row0, &full[sl], pol_pe);
      tma_load_2d_hint(dstb + 4096, &args.tmPE, 64 * c + 32, pe_row0, &full[sl], pol_pe);
      es.xpending |= 1u << sl;
    }
    return true;
  };
  if (tma_pe && filler) {
    for (int c = 0; c < NS; ++c)
      if (!fill(c)) return false;
  }
  bool w = mbar_wait(&tfull[buf], acc_phase, abort_flag);
  if (!__all_sync(0xffffffffu, w)) return false;
  tc_fence_after();
  if (r0 >= P.M) {  // the whole 32-row slab is past M (all lanes agree)
    release();
    return true;
  }
  const int grow = r0 + lane;
  const bool valid = grow < P.M;
  const float sa = valid ? __ldg(P.sa + grow) : 0.0f;
  const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + tmem_col;
  auto dequant = [&](const uint32_t (&acc)[32], int gcol, float (&v)[32]) {
    const float4* sw4 = reinterpret_cast<const float4*>(P.sw + gcol);
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 ws = __ldg(sw4 + j / 4);
      v[j + 0] = static_cast<float>(static_cast<int32_t>(acc[j + 0])) * sa * ws.x;
      v[j + 1] = static_cast<float>(static_cast<int32_t>(acc[j + 1])) * sa * ws.y;
      v[j + 2] = static_cast<float>(static_cast<int32_t>(acc[j + 2])) * sa * ws.z;
      v[j + 3] = static_cast<float>(static_cast<int32_t>(acc[j + 3])) * sa * ws.w;
    }
    if (P.bias) {
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(P.bias + gcol);
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float2 bb = __bfloat1622float2(b2[j / 2]);
        v[j] += bb.x;
        v[j + 1] += bb.y;
      }
    }
  };
  auto load_chunk = [&](int c, uint32_t (&acc)[32]) {
    tmem_ld32(taddr + 32 * c, acc);
    tmem_ld_wait();
    tmem_reg_fence32(acc);
  };
  // this lane's row: batch entry, joint and local position, destination
  int b = 0, pos = 0, lpos = 0;
  if (valid) {
    b = grow / n_l;
    const int i = grow % n_l;
    pos = base + i;
    lpos = (pi == 0 ? q.n_txt_l : 0) + i;
  }
  const int dest = h / q.Hl, hh = h % q.Hl;
  __half* dst = nullptr;
  if (valid) {
    if (q.direct) {
      const size_t slab = static_cast<size_t>(q.nb) * q.Hl * S * kHeadDim;
      dst = reinterpret_cast<__half*>(q.peer_qkvh[dest]) + which * slab +
            ((static_cast<size_t>(b) * q.Hl + hh) * S + pos) * kHeadDim;
    } else {
      const size_t slab = static_cast<size_t>(q.nb) * q.Hl * L * kHeadDim;
      dst = reinterpret_cast<__half*>(q.qkvh) + (static_cast<size_t>(dest) * 3 + which) * slab +
            ((static_cast<size_t>(b) * q.Hl + hh) * L + lpos) * kHeadDim;
    }
  }
  float rms = 0.0f;
  const __nv_bfloat16* nw = nullptr;
  if (which < 2) {
    nw = reinterpret_cast<const __nv_bfloat16*>(pi == 0 ? (which == 0 ? q.nq_img : q.nk_img)
                                                        : (which == 0 ? q.nq_txt : q.nk_txt));
    float ws0 = 0.0f, ws1 = 0.0f, ws2 = 0.0f, ws3 = 0.0f;  // the 4 warp sums
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t acc[32];
      float v[32];
      load_chunk(c, acc);
      dequant(acc, c0 + 32 * c, v);
      // the dequantised values replace the chunk's accumulators, for pass 2
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = __float_as_uint(v[i]);
      tmem_st32(taddr + 32 * c, acc);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __fmul_rn(v[i], v[i]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int i = 0; i < o; ++i) v[i] = __fadd_rn(v[i], v[i + o]);
      }
      ws0 = c == 0 ? v[0] : ws0;
      ws1 = c == 1 ? v[0] : ws1;
      ws2 = c == 2 ? v[0] : ws2;
      ws3 = c == 3 ? v[0] : ws3;
    }
    const float ss = __fadd_rn(__fadd_rn(ws0, ws2), __fadd_rn(ws1, ws3));
    rms = rsqrtf(ss / q.norm_dim + q.eps);
    tmem_st_wait();  // pass 2 reads the stored values back
  }
  const float* pe_lane = q.pe + (valid ? (static_cast<long long>(b) * S + pos) * 256 : 0);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t acc[32];
    float v[32];
    load_chunk(c, acc);
    if (c == 3) release();
    if (which < 2) {  // dequantised by pass 1
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(acc[i]);
    } else {
      dequant(acc, c0 + 32 * c, v);
    }
    uint32_t pk[16];
    if (which < 2) {
      const int sl = c % NS;
      const uint8_t* slot = ring + sl * 8192;
      if (tma_pe) {
        const bool ok_pe = mbar_wait(&full[sl], (es.xphase >> sl) & 1u, abort_flag);
        if (!__all_sync(0xffffffffu, ok_pe)) return false;  // still pending: the exit drain waits for it
        es.xphase ^= 1u << sl;
        es.xpending &= ~(1u << sl);
      }
      // pairs 16c .. 16c + 15 of the head: RoPE rows [cos, -sin, sin, cos]
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(nw + 32 * c);
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        // pair p: box p / 8, 16-byte piece p % 8 of this row at (p % 8) ^ (row % 8)
        const float4 e = tma_pe ? *reinterpret_cast<const float4*>(slot + (p / 8) * 4096 + lane * 128 +
                                                                    (((p % 8) ^ (lane & 7)) * 16))
                                : __ldg(reinterpret_cast<const float4*>(pe_lane + 64 * c) + p);
        const float2 wp = __bfloat1622float2(w2[p]);
        const float x0 = v[2 * p] * rms * wp.x, x1 = v[2 * p + 1] * rms * wp.y;
        const float o0 = x0 * e.x + x1 * e.y;
        const float o1 = x0 * e.z + x1 * e.w;
        __half2 h2 = __floats2half2_rn(o0, o1);
        pk[p] = *reinterpret_cast<uint32_t*>(&h2);
      }
      if (tma_pe) {
        __syncwarp();  // every lane has read chunk c's rows
        if (lane == 0) mbar_arrive(&empty[sl]);
        if (filler && c + NS < 4 && !fill(c + NS)) return false;
      }
    } else {
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        __half2 h2 = __floats2half2_rn(v[2 * p], v[2 * p + 1]);
        pk[p] = *reinterpret_cast<uint32_t*>(&h2);
      }
    }
    // FP16 elements 32c .. 32c + 31 of the 32 rows (64 bytes each) through the
    // staging buffer: row r's 16-byte piece k at slot k ^ ((r / 2) % 4), then
    // eight rows per store instruction (in instruction i, lanes 4j .. 4j + 3
    // write the four pieces of row 8i + j)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      *reinterpret_cast<uint4*>(obuf + lane * 64 + ((k ^ ((lane >> 1) & 3)) * 16)) =
          make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 8 * i + (lane >> 2), k = lane & 3;
      const unsigned long long d = __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst), r);
      const uint4 val = *reinterpret_cast<const uint4*>(obuf + r * 64 + ((k ^ ((r >> 1) & 3)) * 16));
      if (d) {
        uint4* d4 = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(d) + 32 * c) + k;
        if (q.direct)  // peer memory: plain stores
          *d4 = val;
        else
          st_global_v4_hint(d4, val, pol_out);
      }
    }
    __syncwarp();  // the staging buffer is read before the next chunk writes it
  }
  return true;
}

// ------------------------------------------------------------------ CTA pairs
// INT8 GEMM on CTA pairs (tcgen05 cta_group::2): a cluster of two CTAs owns a
// 256 x 256 output tile; each CTA loads 128 rows of A and 128 rows (half) of
// B per 128-byte K block into its own shared memory, the even CTA issues
// M = 256, N = 256 MMAs that read both CTAs' operands and write 128
// accumulator rows into each CTA's TMEM.  Per SM that halves the B operand
// bytes the tensor core reads from shared memory (A 16 KB + B 16 KB per K
// block instead of 16 + 32).  Both CTAs run the producer and the epilogue;
// stage and accumulator hand-offs use multicast commits (to both CTAs) and
// remote arrivals on the even CTA's barriers.
// The shared memory the smaller B slice frees holds staging for eight
// epilogue warps: two per TMEM lane quarter, each owning half of the tile's
// 256 columns, so a tile's epilogue takes about half as long as with four
// and stays shorter than its main loop.
//
// Tile width BN = 256, or 192 / 128 where the 256-wide tiles would leave much
// of their last wave idle (few rows per rank): the narrower tiles use the same
// per-element arithmetic, so the outputs are identical.
namespace gemm2 {
constexpr int BM = 256, BK = 128;
constexpr int A_BYTES = 128 * BK;                // this CTA's 128 rows of A: 16 KB
template <int BN>
constexpr int b_bytes() { return (BN / 2) * BK; }  // this CTA's half of B: 16 / 8 KB
// QKV: the fused QKV projection (kEpiQkv, BN = 256) gives one stage to its
// epilogue's RoPE-row rings
template <int BN, bool QKV = false>
constexpr int stages() { return QKV ? 4 : (BN == 128 ? 6 : 5); }
template <int BN>
constexpr int stage_bytes() { return A_BYTES + b_bytes<BN>(); }
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;     // producer, MMA issuer, 8 epilogue warps
constexpr int EPI_BYTES = EPI_WARPS * 2 * gemm::EPI_BUF;  // double buffered per warp: 64 KB
constexpr int QKV_SLOTS = 2;  // RoPE-row ring slots (8 KB: one chunk) per TMEM lane quarter
constexpr int QKV_OUT = 2048;  // per-warp staging of one chunk's FP16 output (32 rows x 64 bytes)
template <bool QKV>
constexpr int epi_bytes() { return QKV ? 4 * QKV_SLOTS * 8192 + EPI_WARPS * QKV_OUT : EPI_BYTES; }
template <bool QKV>
constexpr int bar_bytes() { return QKV ? 512 : 256; }
template <int BN, bool QKV = false>
constexpr int smem_bytes() {
  return stages<BN, QKV>() * stage_bytes<BN>() + epi_bytes<QKV>() + 1024 + bar_bytes<QKV>();
}
static_assert(smem_bytes<256, true>() <= 232448, "shared memory per CTA");
static_assert(smem_bytes<256>() <= 232448 && smem_bytes<192>() <= 232448 && smem_bytes<128>() <= 232448,
              "shared memory per CTA");
constexpr int TMEM_COLS = 512;  // two accumulator buffers, 256 columns apart (narrower tiles use part of each)
}  // namespace gemm2

template <int BN, bool QKV>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm2::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ GemmArgsDev args) {
  static_assert(BN == 256 || BN == 192 || BN == 128, "pair tile width");
  static_assert(!QKV || BN == 256, "the fused QKV epilogue takes one head per epilogue warp");
  using gemm2::A_BYTES;
  using gemm2::BK;
  using gemm2::BM;
  using gemm2::TMEM_COLS;
  constexpr int B_BYTES = gemm2::b_bytes<BN>();
  constexpr int STAGE_BYTES = gemm2::stage_bytes<BN>();
  constexpr int STAGES = gemm2::stages<BN, QKV>();
  constexpr int NS = gemm2::QKV_SLOTS;
  constexpr int TMEM_BUF = 256;  // column stride of the two accumulator buffers
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sE = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sE + gemm2::epi_bytes<QKV>());  // used in the even CTA
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;  // used in the even CTA: 8 epilogue warps x 2 CTAs
  uint64_t* xfull = tempty + 2;
  uint64_t* drain = xfull + 2 * gemm2::EPI_WARPS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // QKV: per TMEM lane quarter, NS "RoPE rows landed" and NS "slot read by both warps" barriers
  uint64_t* ring_full = drain + 2;
  uint64_t* ring_empty = ring_full + 4 * NS;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cr = cluster_ctarank();
  const bool leader = cr == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * gemm2::EPI_WARPS);
    }
    for (int b = 0; b < 2 * gemm2::EPI_WARPS; ++b) mbar_init(&xfull[b], 1);
    if constexpr (QKV) {
      for (int b = 0; b < 4 * NS; ++b) {
        mbar_init(&ring_full[b], 1);
        mbar_init(&ring_empty[b], 2);
      }
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    for (int i = 0; i < args.nprob; ++i) {
      tma_prefetch_desc(&args.p[i].tmA);
      tma_prefetch_desc(&args.p[i].tmB);
      if constexpr (!QKV) tma_prefetch_desc(&args.p[i].tmO);  // no FP32 output tiles when fused
    }
    if constexpr (QKV) tma_prefetch_desc(&args.tmPE);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before either signals the other
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto locate = [&](int t, int& pi, int& m0, int& n0) {
    pi = (args.nprob > 1 && t >= args.p[0].tile_end) ? 1 : 0;
    const GemmProblemDev& P = args.p[pi];
    int lt = t - P.tile_begin;
    m0 = (lt / P.tiles_n) * BM;
    int nt = lt % P.tiles_n;
    // QKV: a row block's column tiles in the order Q, K, V, Q, K, V, ...  A
    // cluster takes every (clusters)-th tile, so its tiles then mix the q/k
    // heads' longer epilogue with the V heads' shorter one instead of running
    // a dozen q/k tiles back to back; each tile's work is unchanged.
    if constexpr (QKV) nt = (nt % 3) * (P.tiles_n / 3) + nt / 3;
    n0 = nt * BN;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(&full[0], 0);  // the even CTA's stage barriers
      const uint64_t pol_first = l2_policy_evict_first(), pol_normal = l2_policy_evict_normal(),
                     pol_last = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = cluster; t < args.total_tiles && ok; t += nclusters) {
        int pi, m0, n0;
        locate(t, pi, m0, n0);
        const GemmProblemDev& P = args.p[pi];
        const int kblocks = (P.K + BK - 1) / BK;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&full[stage], 2 * STAGE_BYTES);  // both CTAs' bytes
          const uint32_t fb = full0 + stage * 8;
          if (args.l2) {
            tma_load_2d_pair_hint(sA + stage * A_BYTES, &P.tmA, kb * BK, m0 + 128 * static_cast<int>(cr), fb,
                                  P.K >= 8192 ? pol_first : pol_normal);
            tma_load_2d_pair_hint(sB + stage * B_BYTES, &P.tmB, kb * BK, n0 + (BN / 2) * static_cast<int>(cr), fb,
                                  args.l2 >= 2 ? pol_last : pol_normal);
          } else {
            tma_load_2d_pair(sA + stage * A_BYTES, &P.tmA, kb * BK, m0 + 128 * static_cast<int>(cr), fb);
            tma_load_2d_pair(sB + stage * B_BYTES, &P.tmB, kb * BK, n0 + (BN / 2) * static_cast<int>(cr), fb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kErrTimeoutProducer);
        // copies already issued complete on the even CTA's barrier: give them
        // time to land before this CTA leaves
        const uint64_t t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 200000ull) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader) {
      // the whole warp runs this role: every lane waits (the vote keeps the warp
      // converged) and one elected lane issues each MMA / commit
      auto wait_all = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      const uint32_t idesc = idesc_i8(BM, BN);
      const uint64_t ad0 = umma_desc_sw128(smem_u32(sA), 16, 1024), bd0 = umma_desc_sw128(smem_u32(sB), 16, 1024);
      for (int t = cluster; t < args.total_tiles && ok; t += nclusters, ++local) {
        int pi, m0, n0;
        locate(t, pi, m0, n0);
        const GemmProblemDev& P = args.p[pi];
        const int kblocks = (P.K + BK - 1) / BK;
        const int buf = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!wait_all(&tempty[buf], acc_phase ^ 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * TMEM_BUF;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_all(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = ad0 + static_cast<uint64_t>((stage * A_BYTES) >> 4);
          const uint64_t bd = bd0 + static_cast<uint64_t>((stage * B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < BK / 32; ++k)
            mma_i8_ss_pair_elect(d_tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0 ? 1u : 0u);
          mma_commit_pair_elect(&empty[stage], 0x3);  // the stage is free in both CTAs
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair_elect(&tfull[buf], 0x3);  // both CTAs' accumulator rows are ready
      }
      if (!ok && lane == 0) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kErrTimeoutMma);
      }
      __syncwarp();
      // every MMA issued above (it writes both CTAs' TMEM) completes before teardown
      mma_commit_pair_elect(drain, 0x1);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(drain, 0) && global_timer_ns() - t0 < kWaitLimitNs / 4) {
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quarter = warp & 3;
    const int ew = warp - 2;
    const int half = ew >> 2;  // columns (BN / 2) * half .. of each tile
    constexpr int HCH = BN / 64;  // 32-column chunks per half
    uint8_t* ebuf = sE + ew * 2 * gemm::EPI_BUF;
    uint64_t* xb = xfull + ew * 2;
    const uint32_t tempty0 = mapa_shared(&tempty[0], 0);
    EpiState es;
    int local = 0;
    bool ok = true;
    for (int t = cluster; t < args.total_tiles && ok; t += nclusters, ++local) {
      int pi, m0, n0;
      locate(t, pi, m0, n0);
      const int buf = local & 1;
      bool released = false;  // the fused epilogue hands the accumulator back itself
      if constexpr (QKV) {
        // the ring of this TMEM lane quarter (its half-0 and half-1 warps)
        const int e0 = ew & 3;
        ok = epilogue_qkv<NS>(args, args.p[pi], pi, m0 + 128 * static_cast<int>(cr), n0 + 128 * half,
                              static_cast<uint32_t>(buf * TMEM_BUF + 128 * half), buf, (local >> 1) & 1, tmem_base,
                              sE + e0 * NS * 8192, ring_full + e0 * NS, ring_empty + e0 * NS, half == 0,
                              sE + 4 * NS * 8192 + ew * gemm2::QKV_OUT, tfull, es, tempty0 + buf * 8, abort_flag,
                              quarter, lane);
        released = true;
      } else {
        ok = epilogue_tile<false>(args, args.p[pi], m0 + 128 * static_cast<int>(cr), n0, buf, (local >> 1) & 1,
                                  tmem_base, ebuf, xb, tfull, es, abort_flag, quarter, lane, HCH * half,
                                  HCH * half + HCH);
      }
      if (!ok) break;
      if (!released) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty0 + buf * 8);
      }
    }
    if constexpr (QKV)  // RoPE-row copies this warp issued (the filling warps)
      epilogue_drain(es, ring_full + (ew & 3) * NS, lane, NS);
    else
      epilogue_drain(es, xb, lane);
    __syncwarp();
    if (!ok && lane == 0) {
      *abort_flag = 1;
      atomicCAS(args.err, 0, kErrTimeoutEpilogue);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs finished with TMEM and each other's barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host
// FP32 output (and residual) [rows, cols] with leading dimension ldo: 32x32
// boxes, 128-byte swizzle (the epilogue's staging layout).
static int encode_out(CUtensorMap* tm, const float* base, int rows, int cols, int ldo) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldo) * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = qi_encode_tiled(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QI_OK : QI_ERR_CUDA;
}

static int encode_kmajor(CUtensorMap* tm, const void* base, int rows, int K, int box_rows, bool bf16) {
  const int esize = bf16 ? 2 : 1;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * esize};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(gemm::BK / esize), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = qi_encode_tiled(tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                                      const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QI_OK : QI_ERR_CUDA;
}

template <bool BF16>
static int launch_args(GemmArgsDev& args, cudaStream_t stream, int num_sms) {
  static unsigned long long attr_done = 0;
  if (smem_optin(reinterpret_cast<const void*>(gemm_kernel<BF16>), gemm::SMEM_BYTES, &attr_done) != QI_OK)
    return QI_ERR_CUDA;
  int grid = args.total_tiles < num_sms ? args.total_tiles : num_sms;
  gemm_kernel<BF16><<<grid, gemm::THREADS, gemm::SMEM_BYTES, stream>>>(args);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

static void fill_problem(GemmProblemDev& P, int M, int N, int K, int ldo, int& tiles, int bm = gemm::BM,
                         int bn = gemm::BN) {
  P.M = M;
  P.N = N;
  P.K = K;
  P.ldo = ldo;
  P.tiles_n = (N + bn - 1) / bn;
  const int tm = (M + bm - 1) / bm;
  P.tile_begin = tiles;
  tiles += tm * P.tiles_n;
  P.tile_end = tiles;
}

template <int BN, bool QKV = false>
static int launch_pair(GemmArgsDev& args, cudaStream_t stream, int num_sms) {
  static unsigned long long attr_done = 0;
  constexpr int smem = gemm2::smem_bytes<BN, QKV>();
  if (smem_optin(reinterpret_cast<const void*>(gemm_pair_kernel<BN, QKV>), smem, &attr_done) != QI_OK)
    return QI_ERR_CUDA;
  const int clusters = args.total_tiles < num_sms / 2 ? args.total_tiles : num_sms / 2;
  gemm_pair_kernel<BN, QKV><<<2 * clusters, gemm2::THREADS, smem, stream>>>(args);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

// Pair tile width: the one whose waves of tiles over the SM pairs, times the
// tile's cost relative to a 256 x 256 tile, finish first.  Costs measured at
// the forward's shapes (per MAC a narrower tile moves more operand bytes
// through L2 and shared memory): 256 x 192 0.84-0.86, 256 x 128 0.62-0.68.
// Narrow tiles therefore win only where wide ones leave much of their last
// wave idle (few rows per rank).  QI_GEMM_PAIR_BN=256 / 192 / 128 forces a
// width (measurements).
static int pair_tile_width(const GemmDesc* descs, int n, int clusters) {
  static int forced = -1;
  if (forced < 0) {
    const char* e = getenv("QI_GEMM_PAIR_BN");
    forced = e ? atoi(e) : 0;
    if (forced != 128 && forced != 192 && forced != 256) forced = 0;
  }
  if (forced) return forced;
  constexpr int kWidths[3] = {256, 192, 128};
  constexpr double kCost[3] = {1.0, 0.85, 0.68};
  int best = 256;
  double best_t = 0.0;
  for (int c = 0; c < 3; ++c) {
    long long tiles = 0;
    for (int i = 0; i < n; ++i) {
      if (descs[i].M <= 0) continue;
      tiles += static_cast<long long>((descs[i].M + gemm2::BM - 1) / gemm2::BM) *
               ((descs[i].N + kWidths[c] - 1) / kWidths[c]);
    }
    const double t = static_cast<double>((tiles + clusters - 1) / clusters) * kCost[c];
    if (c == 0 || t < best_t * 0.97) {  // a narrower width must win clearly
      best = kWidths[c];
      best_t = t;
    }
  }
  return best;
}

// CTA pairs (256-row tiles, eight epilogue warps) whenever there are rows
// enough to fill them; the one-CTA kernel for short problems.
static bool use_pairs(const GemmDesc* descs, int n, int num_sms) {
  long long rows = 0;
  int kmin = 1 << 30;
  for (int i = 0; i < n; ++i) {
    rows += descs[i].M;
    if (descs[i].M > 0 && descs[i].K < kmin) kmin = descs[i].K;
  }
  return rows >= 512 && kmin >= QI_GEMM_PAIR_MIN_K && num_sms >= 2;
}

bool gemm_qkv_fusable(const GemmDesc* descs, int n, int num_sms) {
  if (n < 1 || n > 2) return false;
  for (int i = 0; i < n; ++i)
    if (descs[i].N != 3 * kDim) return false;
  return use_pairs(descs, n, num_sms);
}

// qp: kEpiQkv's parameters (null otherwise).
static int gemm_i8_run(const GemmDesc* descs, int n, int epi, const QkvPostArgs* qp, cudaStream_t stream,
                       int* err_dev, int num_sms) {
  if (n < 1 || n > 2) return QI_ERR_ARG;
  GemmArgsDev args;
  memset(&args, 0, sizeof(args));
  int tiles = 0;
  const bool fused = epi == kEpiQkv;
  const bool pair = use_pairs(descs, n, num_sms);
  if (fused && (!qp || !gemm_qkv_fusable(descs, n, num_sms))) return QI_ERR_UNSUPPORTED;
  const int bm = pair ? gemm2::BM : gemm::BM;
  // the fused epilogue needs whole heads per epilogue warp: 256-column tiles
  const int bn = fused ? 256 : (pair ? pair_tile_width(descs, n, num_sms / 2) : gemm::BN);
  for (int i = 0; i < n; ++i) {
    const GemmDesc& d = descs[i];
    if (d.M < 0 || d.N <= 0 || d.K <= 0) return QI_ERR_ARG;
    if (d.K % 16 != 0 || d.N % 32 != 0 || d.ldo % 4 != 0) return QI_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(d.a) & 15) || (reinterpret_cast<uintptr_t>(d.w) & 15) ||
        (!fused && (reinterpret_cast<uintptr_t>(d.out) & 15)) || (reinterpret_cast<uintptr_t>(d.sw) & 15))
      return QI_ERR_ALIGN;
    if (epi == kEpiResidual && (d.gate == nullptr || (reinterpret_cast<uintptr_t>(d.gate) & 15)))
      return QI_ERR_ARG;
    GemmProblemDev& P = args.p[i];
    if (d.M > 0) {
      if (encode_kmajor(&P.tmA, d.a, d.M, d.K, 128, false) != QI_OK) return QI_ERR_CUDA;
      if (encode_kmajor(&P.tmB, d.w, d.N, d.K, pair ? bn / 2 : gemm::BN, false) != QI_OK) return QI_ERR_CUDA;
      if (!fused && encode_out(&P.tmO, d.out, d.M, d.N, d.ldo) != QI_OK) return QI_ERR_CUDA;
    }
    P.sa = d.sa;
    P.sw = d.sw;
    P.bias = reinterpret_cast<const __nv_bfloat16*>(d.bias);
    P.out = d.out;
    P.gate = d.gate;
    fill_problem(P, d.M, d.N, d.K, d.ldo, tiles, bm, bn);
  }
  if (tiles == 0) return QI_OK;
  args.nprob = n;
  args.total_tiles = tiles;
  args.epi = epi;
  args.err = err_dev;
  static int l2_mode = -1;
  if (l2_mode < 0) {  // QI_GEMM_L2 = 0 / 1 / 2 (measurements); default 2
    const char* e = getenv("QI_GEMM_L2");
    l2_mode = e ? atoi(e) : 2;
    if (l2_mode < 0 || l2_mode > 2) l2_mode = 2;
  }
  args.l2 = pair ? l2_mode : 0;
  if (fused) {
    if (qp->Hl <= 0 || kHeads % qp->Hl || !qp->pe || (reinterpret_cast<uintptr_t>(qp->pe) & 15)) return QI_ERR_ARG;
    // the RoPE table, nb x [S][64][2][2] FP32: rows of 256 floats, boxes of
    // 32 rows x 32 floats (128 bytes) in the 128-byte swizzle
    cuuint64_t dims[2] = {256, static_cast<cuuint64_t>(qp->nb) * (qp->n_img + qp->n_txt)};
    cuuint64_t strides[1] = {1024};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    if (qi_encode_tiled(&args.tmPE, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(qp->pe), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return QI_ERR_CUDA;
    args.qp = *qp;
    args.qp.norm_dim = kHeadDim;  // run-time operands, as in qkv_post_launch
    args.qp.eps = 1e-6f;
    return launch_pair<256, true>(args, stream, num_sms);
  }
  if (!pair) return launch_args<false>(args, stream, num_sms);
  if (bn == 128) return launch_pair<128>(args, stream, num_sms);
  if (bn == 192) return launch_pair<192>(args, stream, num_sms);
  return launch_pair<256>(args, stream, num_sms);
}

int gemm_i8_launch(const GemmDesc* descs, int n, int epi, cudaStream_t stream, int* err_dev, int num_sms) {
  if (epi == kEpiQkv) return QI_ERR_ARG;  // gemm_qkv_launch
  return gemm_i8_run(descs, n, epi, nullptr, stream, err_dev, num_sms);
}

int gemm_qkv_launch(const GemmDesc* descs, int n, const QkvPostArgs& a, cudaStream_t stream, int* err_dev,
                    int num_sms) {
  return gemm_i8_run(descs, n, kEpiQkv, &a, stream, err_dev, num_sms);
}

int gemm_bf16_launch(const GemmBf16Desc& d, cudaStream_t stream, int* err_dev, int num_sms) {
  if (d.M < 0 || d.N <= 0 || d.K <= 0) return QI_ERR_ARG;
  if (d.K % 8 != 0 || d.N % 32 != 0 || d.ldo % 4 != 0) return QI_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(d.a) & 15) || (reinterpret_cast<uintptr_t>(d.w) & 15) ||
      (reinterpret_cast<uintptr_t>(d.out) & 15))
    return QI_ERR_ALIGN;
  if (d.M == 0) return QI_OK;
  GemmArgsDev args;
  memset(&args, 0, sizeof(args));
  GemmProblemDev& P = args.p[0];
  if (encode_kmajor(&P.tmA, d.a, d.M, d.K, gemm::BM, true) != QI_OK) return QI_ERR_CUDA;
  if (encode_kmajor(&P.tmB, d.w, d.N, d.K, gemm::BN, true) != QI_OK) return QI_ERR_CUDA;
  if (encode_out(&P.tmO, d.out, d.M, d.N, d.ldo) != QI_OK) return QI_ERR_CUDA;
  P.bias = reinterpret_cast<const __nv_bfloat16*>(d.bias);
  P.out = d.out;
  int tiles = 0;
  fill_problem(P, d.M, d.N, d.K, d.ldo, tiles);
  args.nprob = 1;
  args.total_tiles = tiles;
  args.epi = kEpiStore;
  args.err = err_dev;
  return launch_args<true>(args, stream, num_sms);
}

}  // namespace qi
