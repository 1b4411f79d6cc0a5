// attn.cu -- SageAttention (INT8 QK^T, FP16 P.V) on the 5th-gen tensor cores.
//
// Algorithm of the reference's launched instantiation
// qk_int_sv_f16_attn_kernel<CTA_Q=128, CTA_K=64, per-thread Q/K scales, FP32
// accumulation, tensor-core row sums> (sageattention_sm80.cu:47-674, launch
// :896-961), re-tiled for tcgen05:
//   * Q and K are INT8 codes with "per-thread" scales (32 per 128-query block,
//     4 per 64-key block, after K mean smoothing); S = Qc . Kc^T is an exact
//     INT32 tile produced by tcgen05.mma.kind::i8 into TMEM;
//   * the scales are rank-1 (row x column) so they are applied to the INT32
//     tile after the TMEM load: s = float(acc) * q_scale[row] * k_scale[col]
//     * sm_scale * log2(e);
//   * online softmax in base 2 (ex2.approx, m initialised to -5e6, the
//     reference's update_mdo, sageattention_attn_utils.cuh:352-456);
//   * P is rounded to FP16; O += P.V runs as tcgen05.mma.kind::f16 with FP32
//     accumulation in TMEM; the row sum is accumulated in FP32; the running
//     max used for P moves only when the row max grows by more than 2^8 (then
//     O is rescaled in TMEM), which leaves O / l unchanged in exact arithmetic;
//   * exponentials on MUFU (ex2.approx, 16 per clock per SM: the bound of
//     the softmax);
//   * the result is O * rcp(l) rounded to FP16 (normalize_d, :719-760).
//
// Tiling: one CTA per (256 queries, batch-head) = two 128-query tiles that
// share one K/V stream (keys in blocks of 128, two of the reference's 64-key
// scale blocks; a three-stage TMA ring).  Warp 0 issues TMA, warp 1 the MMAs
// (the whole warp, converged, with one elected lane issuing each instruction),
// warps 4-7 run the softmax of tile 0 and warps 8-11 that of tile 1 (one query
// row per thread, TMEM lane = row); the softmax warpgroups take the registers
// warpgroup 0 does not need (setmaxnreg).  TMEM holds, per tile, S (128 columns)
// and O (128 columns); the softmax writes P as packed FP16 over the first 64
// columns of its S, and P.V reads it from TMEM as the A operand.  Per tile the
// chain is QK(j) -> softmax(j) -> PV(j) -> QK(j+1); the two tiles' chains are
// interleaved so the tensor core runs one tile's MMAs while the other tile's
// softmax runs.
#include "qi_internal.h"
#include "sm100.cuh"

#include <climits>
#include <type_traits>

namespace qi {

namespace attn {
constexpr int BQ = 128, BKV = 128, D = 128;
constexpr int NT_MAX = 2;             // query tiles per CTA (the tail of a launch may use 1)
constexpr int STAGES = 3;             // K/V ring depth
constexpr int Q_BYTES = BQ * D;       // int8, one tile
constexpr int K_BYTES = BKV * D;      // int8
constexpr int V_BYTES = BKV * D * 2;  // fp16
constexpr int OFF_Q = 0;
constexpr int OFF_K = OFF_Q + NT_MAX * Q_BYTES;
constexpr int OFF_V = OFF_K + STAGES * K_BYTES;
constexpr int OFF_BAR = OFF_V + STAGES * V_BYTES;
constexpr int OFF_KS = OFF_BAR + 256;  // this batch-head's K scales (FP32), loaded once
constexpr int V8_BYTES = BKV * D;     // fp8 e4m3 V^T tile (FP8 P.V variant)
constexpr int MAX_S = kAttnMaxS;
// K scales, then the 128 per-dimension V factors of the FP8 P.V variant
constexpr int smem_bytes(int ngk) { return OFF_KS + ngk * 4 + 512 + 1024; }
constexpr int THREADS = 384;  // warpgroup 0: TMA warp, MMA warp, 2 idle; warpgroups 1, 2: softmax of tiles 0, 1
// Register split (setmaxnreg): launched at 168 per thread (384 x 168 = 64512);
// warpgroup 0 keeps 88 (the MMA warp holds its descriptors in every lane),
// the two softmax warpgroups take 208: 128 x 88 + 256 x 208 = 64512.
constexpr int LAUNCH_REGS = 168, PRODUCER_REGS = 88, SOFTMAX_REGS = 208;
static_assert(128 * PRODUCER_REGS + 256 * SOFTMAX_REGS <= THREADS * LAUNCH_REGS, "register split exceeds the launch");
constexpr int TM_S = 0;  // S / P of tile t at column 128 t; O of tile t at 128 (NT + t)
}  // namespace attn

struct alignas(64) AttnArgsDev {
  CUtensorMap tmQ, tmK, tmV;
  const float* qs;
  const float* ks;
  const float* vs;  // FP8 P.V: per (batch-head, dim) output factor v_scale / 448
  void* out;
  int BH, S, heads, out_mode, nb, n_img, n_txt, ngq, ngk;
  float qk_scale;  // sm_scale * log2(e)
  int* err;
  ShardMap map;
  void* peer_o[kMaxRanks];
  int head_base;
  int q_tile0;  // first 128-query tile of this launch (the grid's x covers the tiles from there)
};

// Not volatile: a pure function of its input, so the compiler may schedule
// the exponentials freely among the surrounding arithmetic.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for x <= 0 on the FMA and integer pipes, for the share of the softmax
// exponentials (QI_ATTN_POLY of every 16) taken off MUFU.  Cody-Waite split
// x = n + f with n = rint(x) (1.5 * 2^23 added: the sum's low mantissa bits
// hold n) and |f| <= 1/2; 2^f by the degree-QI_ATTN_POLY_DEG polynomial that
// minimises the maximum relative error on [-1/2, 1/2] (fitted here by
// Lawson's iteratively reweighted least squares; max relative error 7.5e-5
// for degree 3, 2.7e-6 for 4, 2.3e-7 for 5 in FP32 Horner evaluation); n is
// added to the exponent field.  x is clamped at -125 so the exponent cannot
// underflow (2^-125 is zero in FP16 and negligible in the row sum).
#ifndef QI_ATTN_POLY
#define QI_ATTN_POLY 0
#endif
#ifndef QI_ATTN_POLY_DEG
#define QI_ATTN_POLY_DEG 5
#endif
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float t = __fadd_rn(x, 12582912.0f);
  const float n = __fadd_rn(t, -12582912.0f);
  const float f = __fadd_rn(x, -n);
  float p;
  if (QI_ATTN_POLY_DEG == 3) {
    p = fmaf(0x1.c3f760p-5f, f, 0x1.f0de1cp-3f);
    p = fmaf(p, f, 0x1.62f31ap-1f);
    p = fmaf(p, f, 0x1.fff692p-1f);
  } else if (QI_ATTN_POLY_DEG == 4) {
    p = fmaf(0x1.3997d4p-7f, f, 0x1.ca1442p-5f);
    p = fmaf(p, f, 0x1.ec06dap-3f);
    p = fmaf(p, f, 0x1.62e0dcp-1f);
    p = fmaf(p, f, 0x1.ffffe8p-1f);
  } else {
    p = fmaf(0x1.5c08e4p-10f, f, 0x1.3d0c54p-7f);
    p = fmaf(p, f, 0x1.c6b6e4p-5f);
    p = fmaf(p, f, 0x1.ebf918p-3f);
    p = fmaf(p, f, 0x1.62e428p-1f);
    p = fmaf(p, f, 0x1.000002p+0f);
  }
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}
// Element i of a 16-key group takes the polynomial: QI_ATTN_POLY of every 16,
// spread evenly.
__host__ __device__ constexpr bool poly_slot(int i) {
  return (i % 16) * QI_ATTN_POLY / 16 != ((i % 16) + 1) * QI_ATTN_POLY / 16;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// Bounded wait that ignores the abort flag (used to drain work this thread
// itself issued before it tears down).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity) && global_timer_ns() - t0 < kWaitLimitNs / 4) {
  }
}

// E4M3 codes of four values, the first in the lowest byte (cvt.rn.satfinite
// puts its first operand in the upper byte of each pair).
__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  uint16_t lo, hi;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(lo) : "f"(b), "f"(a));
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(hi) : "f"(d), "f"(c));
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// FP8 = true: the FP8 P.V variant (SageAttention2's scheme, the FP8 e4m3
// helpers of sageattention_mma.cuh:521-680 and
// sageattention_numeric_conversion.cuh:46-140, which the reference ships but
// does not launch): V arrives as E4M3 codes of V / v_scale transposed to
// [dim][token], P is rescaled at every row-max increase (P <= 1), stored as
// E4M3 codes of 448 P, and P.V runs as tcgen05.mma.kind::f8f6f4; the output
// factor per dimension is v_scale / 448.
//
// NT = query tiles per CTA: 2 normally; 1 for the last, partial wave of a
// launch (attention_launch), where one-tile CTAs spread the remaining tiles
// over more SMs (warpgroup 2 then idles).  A query row's arithmetic is the
// same either way.
template <bool FP8, int NT>
__global__ void __launch_bounds__(attn::THREADS, 1) sage_attn_kernel(const __grid_constant__ AttnArgsDev args) {
  using namespace attn;
  static_assert(NT == 1 || NT == 2, "one or two query tiles per CTA");
  constexpr int TMEM_COLS = 256 * NT;  // S and O of NT tiles
  constexpr int TM_O = 128 * NT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + OFF_Q;
  uint8_t* sK = smem + OFF_K;
  uint8_t* sV = smem + OFF_V;
  float* sKS = reinterpret_cast<float*>(smem + OFF_KS);
  float* sVS = sKS + args.ngk;  // FP8: this batch-head's 128 V factors
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                // [STAGES]
  uint64_t* k_empty = k_full + STAGES;        // [STAGES]
  uint64_t* v_full = k_empty + STAGES;        // [STAGES]
  uint64_t* v_empty = v_full + STAGES;        // [STAGES]
  uint64_t* s_full = v_empty + STAGES;        // [NT] QK of the tile's current block complete
  uint64_t* p_half = s_full + NT;             // [NT][2] half h of the tile's P written to TMEM (4 warps)
  uint64_t* o_final = p_half + 2 * NT;        // [NT] the tile's last PV complete (single use)
  uint64_t* s_loaded = o_final + NT;          // [NT] the tile's S of the current block is in registers (4 warps)
  uint64_t* drain = s_loaded + NT;            // MMA teardown
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(drain + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = (args.q_tile0 + static_cast<int>(blockIdx.x) * NT) * BQ;
  const int bh = blockIdx.y;
  const int S = args.S;
  const int nkb = (S + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_half[2 * t], 4);
      mbar_init(&p_half[2 * t + 1], 4);
      mbar_init(&o_final[t], 1);
      mbar_init(&s_loaded[t], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&args.tmQ);
    tma_prefetch_desc(&args.tmK);
    tma_prefetch_desc(&args.tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= 4) {  // K scales of this batch-head into shared memory
    const float* ks = args.ks + static_cast<size_t>(bh) * args.ngk;
    for (int i = threadIdx.x - 128; i < args.ngk; i += THREADS - 128) sKS[i] = ks[i];
    if (FP8 && threadIdx.x - 128 < D) sVS[threadIdx.x - 128] = args.vs[static_cast<size_t>(bh) * D + threadIdx.x - 128];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PRODUCER_REGS));
    if (warp == 0) {
      if (lane == 0) {
        bool ok = true;
        uint32_t kmask = 0, kpar = 0, vmask = 0, vpar = 0;
        mbar_expect_tx(q_full, NT * Q_BYTES);
        for (int t = 0; t < NT; ++t) tma_load_3d(sQ + t * Q_BYTES, &args.tmQ, 0, q0 + t * BQ, bh, q_full);
        for (int j = 0; j < nkb && ok; ++j) {
          const int st = j % STAGES;
          const uint32_t ph = (j / STAGES) & 1;
          if (!mbar_wait(&k_empty[st], ph ^ 1u, abort_flag)) { ok = false; break; }
          mbar_expect_tx(&k_full[st], K_BYTES);
          tma_load_3d(sK + st * K_BYTES, &args.tmK, 0, j * BKV, bh, &k_full[st]);
          kmask |= 1u << st;
          kpar = (kpar & ~(1u << st)) | (ph << st);
          if (!mbar_wait(&v_empty[st], ph ^ 1u, abort_flag)) { ok = false; break; }
          if (FP8) {  // V^T codes [dim][token]: 128 dims x 128 keys, K-major
            mbar_expect_tx(&v_full[st], V8_BYTES);
            tma_load_3d(sV + st * V_BYTES, &args.tmV, j * BKV, 0, bh, &v_full[st]);
          } else {
            mbar_expect_tx(&v_full[st], V_BYTES);
            tma_load_3d(sV + st * V_BYTES, &args.tmV, 0, j * BKV, bh, &v_full[st]);
            tma_load_3d(sV + st * V_BYTES + V_BYTES / 2, &args.tmV, 64, j * BKV, bh, &v_full[st]);
          }
          vmask |= 1u << st;
          vpar = (vpar & ~(1u << st)) | (ph << st);
        }
        if (!ok) {  // let the copies already issued land before the CTA exits
          *abort_flag = 1;
          atomicCAS(args.err, 0, kErrTimeoutProducer);
          drain_wait(q_full, 0);
          for (int s = 0; s < STAGES; ++s) {
            if (kmask & (1u << s)) drain_wait(&k_full[s], (kpar >> s) & 1u);
            if (vmask & (1u << s)) drain_wait(&v_full[s], (vpar >> s) & 1u);
          }
        }
      }
    } else if (warp == 1) {
      {  // the whole warp runs this role; one elected lane issues each MMA / commit
        // every lane waits; the vote keeps the warp converged for elect.sync
        auto wait_all = [&](uint64_t* bar, uint32_t parity) {
          return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
        };
        bool ok = wait_all(q_full, 0);
        const uint32_t id_qk = idesc_i8(BQ, BKV);
        // P.V: FP16 P with MN-major FP16 V, or E4M3 P with K-major E4M3 V^T
        const uint32_t id_pv = idesc_f16(BQ, D, false, !FP8);
        const uint32_t q_addr = smem_u32(sQ);
        // Shared-memory descriptors are built once; an operand at a byte offset is
        // the base descriptor plus offset / 16 in its address field (no carry: shared
        // addresses stay below 2^18).
        const uint64_t qd0 = umma_desc_sw128(q_addr, 16, 1024);
        const uint64_t kd0 = umma_desc_sw128(smem_u32(sK), 16, 1024);
        const uint64_t vd0 = FP8 ? umma_desc_sw128(smem_u32(sV), 16, 1024) : umma_desc_sw128(smem_u32(sV), V_BYTES / 2, 1024);
        // S_t = Q_t . K^T for the block in stage st
        auto qk = [&](int t, int st) {
          const uint64_t qa = qd0 + static_cast<uint64_t>(t * (Q_BYTES >> 4));
          const uint64_t kb = kd0 + static_cast<uint64_t>((st * K_BYTES) >> 4);
          const uint32_t d = tmem + TM_S + 128 * t;
  #pragma unroll
          for (int k = 0; k < D / 32; ++k) mma_i8_ss_elect(d, qa + 2 * k, kb + 2 * k, id_qk, k > 0 ? 1u : 0u);
          mma_commit_elect(&s_full[t]);
        };
        // Keys 64 hh .. 64 hh + 63 of that product into S_t columns 64 hh ..: the
        // upper half (columns 64-127) never holds P, so it is issued as soon as the
        // softmax has read S_t of the previous block; only the lower half waits
        // for P_t . V to have read P_t.
        const uint32_t id_qk64 = idesc_i8(BQ, 64);
        auto qk_half = [&](int t, int st, int hh) {
          const uint64_t qa = qd0 + static_cast<uint64_t>(t * (Q_BYTES >> 4));
          const uint64_t kb = kd0 + static_cast<uint64_t>((st * K_BYTES + hh * (K_BYTES / 2)) >> 4);
          const uint32_t d = tmem + TM_S + 128 * t + 64 * hh;
  #pragma unroll
          for (int k = 0; k < D / 32; ++k) mma_i8_ss_elect(d, qa + 2 * k, kb + 2 * k, id_qk64, k > 0 ? 1u : 0u);
        };
        // O_t += P_t . V over keys 64h .. 64h+63 of the block in stage st; P_t is read from TMEM
        auto pv_half = [&](int t, int st, int j, int h) {
          const uint64_t vb = vd0 + static_cast<uint64_t>((st * V_BYTES) >> 4);
          const uint32_t d = tmem + TM_O + 128 * t, a = tmem + TM_S + 128 * t;
          if (FP8) {
            // 32 keys per instruction: 8 TMEM columns of P, 32 bytes along V^T's K
  #pragma unroll
            for (int k2 = 0; k2 < 2; ++k2) {
              const int kk = 2 * h + k2;
              mma_f8_ts_elect(d, a + kk * 8, vb + 2 * kk, id_pv, (j > 0 || kk > 0) ? 1u : 0u);
            }
          } else {
  #pragma unroll
            for (int k4 = 0; k4 < BKV / 32; ++k4) {
              const int kk = h * (BKV / 32) + k4;
              mma_f16_ts_elect(d, a + kk * 8, vb + 128 * kk, id_pv, (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
        };
        if (ok) ok = wait_all(&k_full[0], 0);
        if (ok) {
          tc_fence_after();
          for (int t = 0; t < NT; ++t) qk(t, 0);
          mma_commit_elect(&k_empty[0]);
        }
        for (int j = 0; j < nkb && ok; ++j) {
          const int st = j % STAGES, nst = (j + 1) % STAGES;
          const uint32_t ph = (j / STAGES) & 1, nph = ((j + 1) / STAGES) & 1;
          const bool more = j + 1 < nkb;
          for (int t = 0; t < NT && ok; ++t) {
            if (more) {  // upper half of S_t for block j + 1, once S_t of block j is read
              if (!wait_all(&s_loaded[t], j & 1)) { ok = false; break; }
              if (t == 0 && !wait_all(&k_full[nst], nph)) { ok = false; break; }
              tc_fence_after();
              qk_half(t, nst, 1);
            }
            // each half of P_t . V starts as soon as that half of P_t is in TMEM
            if (!wait_all(&p_half[2 * t], j & 1)) { ok = false; break; }
            if (t == 0 && !wait_all(&v_full[st], ph)) { ok = false; break; }
            tc_fence_after();
            pv_half(t, st, j, 0);
            if (!wait_all(&p_half[2 * t + 1], j & 1)) { ok = false; break; }
            tc_fence_after();
            pv_half(t, st, j, 1);
            if (j == nkb - 1) mma_commit_elect(&o_final[t]);
            if (t == NT - 1) mma_commit_elect(&v_empty[st]);
            if (more) {
              // the lower half of QK(j+1) overwrites the S_t / P_t columns that
              // P_t . V of block j reads; the tensor pipe runs one CTA's MMAs in
              // issue order, so it is issued right behind it.  The commit covers
              // both halves.
              qk_half(t, nst, 0);
              mma_commit_elect(&s_full[t]);
              if (t == NT - 1) mma_commit_elect(&k_empty[nst]);
            }
          }
        }
        if (!ok && lane == 0) {
          *abort_flag = 1;
          atomicCAS(args.err, 0, kErrTimeoutMma);
        }
        __syncwarp();
        // every MMA this thread issued has completed before TMEM is released
        mma_commit_elect(drain);
        drain_wait(drain, 0);
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(SOFTMAX_REGS));
    // -------------------------------------------------------------- softmax
    const int t = (warp - 4) >> 2;
    if (t < NT) {  // with one tile per CTA, warpgroup 2 has no tile
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int qrow = q0 + t * BQ + row;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_tm = tmem + lane_off + TM_S + 128 * t;
    const uint32_t o_tm = tmem + lane_off + TM_O + 128 * t;
    const int gq = (qrow / 128) * 32 + ((qrow % 128) / 32) * 8 + (qrow % 8);
    const float qsm = (qrow < S) ? args.qs[static_cast<size_t>(bh) * args.ngq + gq] * args.qk_scale : 0.0f;
    float m = -5000000.0f, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      // S_t of block j is in TMEM; P_t . V of block j-1 has completed (both
      // were issued before the commit that completes this phase), so O_t is
      // stable and the P_t columns are free
      bool w = mbar_wait(&s_full[t], j & 1, abort_flag);
      if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
      tc_fence_after();
      uint32_t r[BKV];
      tmem_ld32(s_tm + 0, *reinterpret_cast<uint32_t(*)[32]>(r + 0));
      tmem_ld32(s_tm + 32, *reinterpret_cast<uint32_t(*)[32]>(r + 32));
      tmem_ld32(s_tm + 64, *reinterpret_cast<uint32_t(*)[32]>(r + 64));
      tmem_ld32(s_tm + 96, *reinterpret_cast<uint32_t(*)[32]>(r + 96));
      // column factors kf[g] = k_scale[(2j + c/64)*4 + (c%8)/2] * q_scale * sm_scale * log2e
      // (all positive) for the 8 scale groups g of this 128-key block
      float kf[8];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int kb64 = 2 * j + h;
#pragma unroll
        for (int g = 0; g < 4; ++g) kf[h * 4 + g] = (kb64 * 64 < S) ? sKS[kb64 * 4 + g] * qsm : 1.0f;
      }
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < BKV / 32; ++q) tmem_reg_fence32(*reinterpret_cast<uint32_t(*)[32]>(r + 32 * q));
      // S_t is in registers: the MMA warp may overwrite its columns 64-127
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_loaded[t]);
      const bool tail = (j + 1) * BKV > S;  // last block reaches past the sequence end
      if (tail) {
#pragma unroll
        for (int i = 0; i < BKV; ++i)
          if (j * BKV + i >= S) r[i] = 0x80000000u;  // INT_MIN: never the max, exp -> 0 below
      }
      // Row max: the scales are positive, so max(acc * kf[g]) = kf[g] * max(acc) per
      // scale group -- integer maxima, then 8 products.
      int gmax[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) gmax[g] = INT_MIN;
#pragma unroll
      for (int i = 0; i < BKV; ++i) {
        const int g = (i >> 6) * 4 + ((i & 7) >> 1);
        gmax[g] = max(gmax[g], static_cast<int>(r[i]));
      }
      float mloc = -5000000.0f;
#pragma unroll
      for (int g = 0; g < 8; ++g)
        if (gmax[g] != INT_MIN) mloc = fmaxf(mloc, static_cast<float>(gmax[g]) * kf[g]);
      // Lazy rescale: the running max used for P only moves when the row max
      // grows by more than 8 (P stays <= 2^8, exact in FP16 range); O and l are
      // rescaled with it, so O / l is unchanged in exact arithmetic.
      const float m_new = fmaxf(m, mloc);
      // (FP8: at every increase, so that P <= 1 and 448 P fits E4M3)
      const bool grow = FP8 ? (m_new > m) : (m_new > m + 8.0f);
      const float alpha = grow ? ex2_approx(m - m_new) : 1.0f;
      const float m_use = grow ? m_new : m;
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          tmem_ld32(o_tm + c, o);
          tmem_ld_wait();
          tmem_reg_fence32(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(o_tm + c, o);
        }
      }
      // exponent argument: acc * kf - m_use = (1.5*2^23 + acc) * kf + (-1.5*2^23 * kf - m_use),
      // where the float bits of (acc + 0x4B400000) are exactly 1.5*2^23 + acc (|acc| < 2^22).
      float kb[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) kb[g] = fmaf(-12582912.0f, kf[g], -m_use);
      // P = exp2(.) -> packed FP16 pairs over columns 0-63 of S_t; the row sum
      // accumulates the FP32 values in 8 partial sums.
      float lp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      const int valid = S - j * BKV;  // keys of this block inside the sequence
      // TAIL: the last block, whose keys past the sequence end get P = 0
      auto exp_half = [&](auto tail_tag, int h) {
        const int hbase = 64 * h;
        constexpr bool TAIL = decltype(tail_tag)::value;
        if constexpr (FP8) {
          // four keys per TMEM column: E4M3 codes of 448 P
          uint32_t p8[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            float p4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int i = hbase + 4 * c + e;
              const int g = (i >> 6) * 4 + ((i & 7) >> 1);
              const float x = fmaf(__int_as_float(static_cast<int>(r[i]) + 0x4B400000), kf[g], kb[g]);
              float p = ex2_approx(x);
              if (TAIL && i >= valid) p = 0.0f;
              lp[(4 * c + e) & 7] += p;
              p4[e] = p * 448.0f;
            }
            p8[c] = pack_e4m3x4(p4[0], p4[1], p4[2], p4[3]);
          }
          tmem_st16(s_tm + hbase / 4, p8);
        } else {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int i0 = hbase + 2 * c, i1 = i0 + 1;
          const int g0 = (i0 >> 6) * 4 + ((i0 & 7) >> 1), g1 = (i1 >> 6) * 4 + ((i1 & 7) >> 1);
          const float x0 = fmaf(__int_as_float(static_cast<int>(r[i0]) + 0x4B400000), kf[g0], kb[g0]);
          const float x1 = fmaf(__int_as_float(static_cast<int>(r[i1]) + 0x4B400000), kf[g1], kb[g1]);
          float p0 = poly_slot(i0) ? exp2_poly(x0) : ex2_approx(x0);
          float p1 = poly_slot(i1) ? exp2_poly(x1) : ex2_approx(x1);
          if (TAIL) {
            if (i0 >= valid) p0 = 0.0f;
            if (i1 >= valid) p1 = 0.0f;
          }
          lp[(2 * c) & 7] += p0;
          lp[(2 * c + 1) & 7] += p1;
          __half2 h2 = __floats2half2_rn(p0, p1);
          pk[c] = *reinterpret_cast<uint32_t*>(&h2);
        }
        tmem_st32(s_tm + hbase / 2, pk);
        }
        // publish this half (and, for h = 0, the rescaled O) to the MMA warp
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_half[2 * t + h]);
      };
      if (tail) {
        exp_half(std::true_type{}, 0);
        exp_half(std::true_type{}, 1);
      } else {
        exp_half(std::false_type{}, 0);
        exp_half(std::false_type{}, 1);
      }
      l = l * alpha + (((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7])));
      m = m_use;
    }
    if (ok) {
      bool w = mbar_wait(&o_final[t], 0, abort_flag);
      ok = __all_sync(0xffffffffu, w);
    }
    if (!ok) {
      if (lane == 0) {
        *abort_flag = 1;
        atomicCAS(args.err, 0, kErrTimeoutSoftmax);
      }
    } else {
      tc_fence_after();
      const float rl = rcp_approx(l);
      const bool valid = qrow < S;
      const int b = bh / args.heads, h = bh % args.heads;
      // out_mode 2: this row's slot in the send buffer of the rank that owns it;
      // out_mode 3: its row in the owner's token-major output (peer memory)
      long long dst_off = 0;
      __half* owner_o = nullptr;
      if (args.out_mode == 3 && valid) {
        const ShardMap& mp = args.map;
        int dr = 0;
        long long orow;
        if (qrow < args.n_txt) {
          while (dr + 1 < mp.P && mp.txt_lo[dr + 1] <= qrow) ++dr;
          orow = static_cast<long long>(args.nb) * mp.n_img_l(dr) + static_cast<long long>(b) * mp.n_txt_l(dr) +
                 (qrow - mp.txt_lo[dr]);
        } else {
          const int gi = qrow - args.n_txt;
          while (dr + 1 < mp.P && mp.img_lo[dr + 1] <= gi) ++dr;
          orow = static_cast<long long>(b) * mp.n_img_l(dr) + (gi - mp.img_lo[dr]);
        }
        owner_o = reinterpret_cast<__half*>(args.peer_o[dr]) + orow * kDim + (args.head_base + h) * D;
      }
      if (args.out_mode == 2 && valid) {
        const ShardMap& mp = args.map;
        int dr = 0, lpos;
        if (qrow < args.n_txt) {
          while (dr + 1 < mp.P && mp.txt_lo[dr + 1] <= qrow) ++dr;
          lpos = qrow - mp.txt_lo[dr];
        } else {
          const int gi = qrow - args.n_txt;
          while (dr + 1 < mp.P && mp.img_lo[dr + 1] <= gi) ++dr;
          lpos = mp.n_txt_l(dr) + gi - mp.img_lo[dr];
        }
        for (int q = 0; q < dr; ++q) dst_off += static_cast<long long>(args.nb) * mp.len(q) * args.heads * D;
        dst_off += ((static_cast<long long>(b) * mp.len(dr) + lpos) * args.heads + h) * D;
      }
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        tmem_ld32(o_tm + c, r);
        tmem_ld_wait();
        tmem_reg_fence32(r);
        if (!valid) continue;
        if (FP8) {  // the per-dimension V factor folded into the accumulator
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * sVS[c + i]);
        }
        if (args.out_mode == 0) {
          float* dst = reinterpret_cast<float*>(args.out) + (static_cast<size_t>(bh) * S + qrow) * D + c;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float4 o;
            o.x = __half2float(__float2half_rn(__uint_as_float(r[i + 0]) * rl));
            o.y = __half2float(__float2half_rn(__uint_as_float(r[i + 1]) * rl));
            o.z = __half2float(__float2half_rn(__uint_as_float(r[i + 2]) * rl));
            o.w = __half2float(__float2half_rn(__uint_as_float(r[i + 3]) * rl));
            *reinterpret_cast<float4*>(dst + i) = o;
          }
        } else if (args.out_mode >= 2) {
          __half* dst = (args.out_mode == 3 ? owner_o : reinterpret_cast<__half*>(args.out) + dst_off) + c;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __half2 h2 = __floats2half2_rn(__uint_as_float(r[i + 2 * e]) * rl, __uint_as_float(r[i + 2 * e + 1]) * rl);
              pk[e] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(dst + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        } else {
          const long long orow = (qrow < args.n_txt)
                                     ? static_cast<long long>(args.nb) * args.n_img + static_cast<long long>(b) * args.n_txt + qrow
                                     : static_cast<long long>(b) * args.n_img + (qrow - args.n_txt);
          __half* dst = reinterpret_cast<__half*>(args.out) + orow * kDim + h * D + c;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint32_t pk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __half2 h2 = __floats2half2_rn(__uint_as_float(r[i + 2 * e]) * rl, __uint_as_float(r[i + 2 * e + 1]) * rl);
              pk[e] = *reinterpret_cast<uint32_t*>(&h2);
            }
            *reinterpret_cast<uint4*>(dst + i) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
        }
      }
    }
    }  // t < NT
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------- quantizers
// Restated from sageattention_sm80.cu:759-886 with the same expressions so
// that, compiled with the same fast-math flags, the codes and scales match
// the reference bit for bit.

__device__ __forceinline__ int8_t cvt_rni_sat_s8(float x) {
  uint32_t d;
  asm volatile("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(d) : "f"(x));
  return static_cast<int8_t>(d & 0xff);
}

// K mean per (batch-head, dim): the reference sums over tokens serially in
// token order (sageattention_sm80.cu:759-773); the K codes depend on it, so the
// order is kept.  One CTA per (batch-head, DPC dims): DPC/32 warps run the
// serial chains (lane = dim) over 32 KB tiles of T tokens x DPC dims in shared
// memory, which all 256 threads fill with cp.async three tiles ahead (a
// four-buffer ring, one __syncthreads per tile).  DPC is chosen so the grid is a
// single wave: the chains are the kernel's whole cost.
template <int DPC>
__global__ void __launch_bounds__(256) sage_kmean_kernel(const __half* __restrict__ k, float* __restrict__ kmean, int S) {
  constexpr int T = 16384 / DPC;  // tokens per 32 KB tile
  constexpr int NB = 4;           // ring buffers
  constexpr int PIECES = T * DPC / 8 / 256;  // 16-byte pieces per thread per tile
  extern __shared__ __align__(16) __half km_tile[];  // [NB][T][DPC]
  const int bh = blockIdx.x, d0 = blockIdx.y * DPC;
  const __half* base = k + static_cast<size_t>(bh) * S * 128 + d0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntiles = (S + T - 1) / T;
  // copies of tile c into buffer c % NB (rows past S are not copied and not read)
  auto issue = [&](int c) {
    if (c < ntiles) {
      __half* buf = km_tile + static_cast<size_t>(c % NB) * T * DPC;
#pragma unroll
      for (int r = 0; r < PIECES; ++r) {
        const int i = tid + 256 * r;
        const int t = c * T + i / (DPC / 8), piece = i % (DPC / 8);
        if (t < S) {
          const uint32_t dst = smem_u32(buf + (i / (DPC / 8)) * DPC + piece * 8);
          const __half* src = base + static_cast<size_t>(t) * 128 + piece * 8;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");  // one group per tile, empty past the end
  };
  issue(0);
  issue(1);
  issue(2);
  float sum = 0.0f;
  for (int c = 0; c < ntiles; ++c) {
    asm volatile("cp.async.wait_group 2;" ::: "memory");  // this thread's copies of tile c have landed
    __syncthreads();  // everyone's have; and every chain has left the buffer refilled next
    issue(c + 3);
    if (warp < DPC / 32) {
      const int n = min(T, S - c * T);
      const __half* col = km_tile + static_cast<size_t>(c % NB) * T * DPC + warp * 32 + lane;
      if (n == T) {
        // software-pipelined: the next 16 tokens are read from shared memory
        // while the chain adds the current 16, so only the adds' latency is
        // on the chain's path (same token order, same sum)
        float a[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) a[i] = __half2float(col[i * DPC]);
#pragma unroll 1
        for (int t = 16; t < T; t += 16) {
          float b[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) b[i] = __half2float(col[(t + i) * DPC]);
#pragma unroll
          for (int i = 0; i < 16; ++i) sum += a[i];
#pragma unroll
          for (int i = 0; i < 16; ++i) a[i] = b[i];
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) sum += a[i];
      } else {
#pragma unroll 8
        for (int t = 0; t < n; ++t) sum += __half2float(col[t * DPC]);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (warp < DPC / 32) kmean[bh * 128 + d0 + warp * 32 + lane] = sum / fmaxf(static_cast<float>(S), 1.0f);
}

template <int DPC>
static int kmean_launch(const __half* k, float* kmean, int BH, int S, cudaStream_t stream) {
  constexpr int smem = 4 * 32768;
  static unsigned long long attr_done = 0;
  if (smem_optin(reinterpret_cast<const void*>(sage_kmean_kernel<DPC>), smem, &attr_done) != QI_OK)
    return QI_ERR_CUDA;
  sage_kmean_kernel<DPC><<<dim3(BH, 128 / DPC), 256, smem, stream>>>(k, kmean, S);
  return QI_OK;
}

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Q per-thread INT8 (sageattention_sm80.cu:775-824): one CTA per (128-query
// block, batch-head), one warp per scale group at a time; group g of the
// block covers tokens (g/8)*32 + g%8 + {0, 8, 16, 24}; lane l holds dims
// 4l..4l+3.  The group max is order-free; scale and codes use the
// reference's expressions.
__global__ void __launch_bounds__(256) sage_quant_q_kernel(const __half* __restrict__ q, int8_t* __restrict__ qc,
                                                           float* __restrict__ qs, int S) {
  const int blk = blockIdx.x, bh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __half* hp = q + static_cast<size_t>(bh) * S * 128 + lane * 4;
  int8_t* out = qc + static_cast<size_t>(bh) * S * 128 + lane * 4;
  const int ngq = ((S + 127) / 128) * 32;
#pragma unroll 1
  for (int g = warp; g < 32; g += 8) {
    const int token_base = blk * 128 + (g / 8) * 32 + (g % 8);
    float vals[4][4];
    float amax = 1e-7f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = token_base + i * 8;
      uint2 raw = make_uint2(0, 0);
      if (t < S) raw = *reinterpret_cast<const uint2*>(hp + static_cast<size_t>(t) * 128);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      vals[i][0] = a.x;
      vals[i][1] = a.y;
      vals[i][2] = b.x;
      vals[i][3] = b.y;
#pragma unroll
      for (int e = 0; e < 4; ++e) amax = fmaxf(amax, fabsf(vals[i][e]));
    }
    const float block_amax = warp_max_f(amax);
    const float block_scale = block_amax / 127.0f + 1e-7f;
    if (lane == 0) qs[static_cast<size_t>(bh) * ngq + blk * 32 + g] = block_scale;
    const float inv_scale = 1.0f / block_scale;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = token_base + i * 8;
      if (t >= S) continue;
      char4 c;
      c.x = cvt_rni_sat_s8(vals[i][0] * inv_scale);
      c.y = cvt_rni_sat_s8(vals[i][1] * inv_scale);
      c.z = cvt_rni_sat_s8(vals[i][2] * inv_scale);
      c.w = cvt_rni_sat_s8(vals[i][3] * inv_scale);
      *reinterpret_cast<char4*>(out + static_cast<size_t>(t) * 128) = c;
    }
  }
}

// K per-thread INT8 after mean smoothing (sageattention_sm80.cu:826-886): one
// CTA per (128 keys, batch-head); warp w handles scale group w % 4 of 64-key
// block w / 4, tokens 2 (w % 4) + 8i + {0, 1}, i = 0..7, lane = 4 dims.  One
// pass: the group's 16 tokens are loaded at once (all loads in flight
// together), held in registers through the absolute max, then scaled and
// stored.
__global__ void __launch_bounds__(256) sage_quant_k_kernel(const __half* __restrict__ k, const float* __restrict__ kmean,
                                                           int8_t* __restrict__ kc, float* __restrict__ ks, int S) {
  const int bh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = blockIdx.x * 2 + (warp >> 2), g = warp & 3;
  if (blk * 64 >= S) return;  // the second block of the last CTA may not exist
  const __half* hp = k + static_cast<size_t>(bh) * S * 128 + lane * 4;
  int8_t* out = kc + static_cast<size_t>(bh) * S * 128 + lane * 4;
  const float4 mean = *reinterpret_cast<const float4*>(kmean + bh * 128 + lane * 4);
  const int token_base = blk * 64 + g * 2;
  uint2 raw[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int t = token_base + (i >> 1) * 8 + (i & 1);
    raw[i] = t < S ? __ldg(reinterpret_cast<const uint2*>(hp + static_cast<size_t>(t) * 128)) : make_uint2(0, 0);
  }
  float v[16][4];
  float am[4] = {1e-7f, 1e-7f, 1e-7f, 1e-7f};
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int t = token_base + (i >> 1) * 8 + (i & 1);
    const bool in = t < S;
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw[i].x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw[i].y));
    v[i][0] = in ? a.x - mean.x : 0.0f;
    v[i][1] = in ? a.y - mean.y : 0.0f;
    v[i][2] = in ? b.x - mean.z : 0.0f;
    v[i][3] = in ? b.y - mean.w : 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) am[i & 3] = fmaxf(am[i & 3], fabsf(v[i][e]));
  }
  const float block_amax = warp_max_f(fmaxf(fmaxf(am[0], am[1]), fmaxf(am[2], am[3])));
  const float block_scale = block_amax / 127.0f + 1e-7f;
  if (lane == 0) ks[static_cast<size_t>(bh) * (((S + 63) / 64) * 4) + blk * 4 + g] = block_scale;
  const float inv_scale = 1.0f / block_scale;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int t = token_base + (i >> 1) * 8 + (i & 1);
    if (t >= S) continue;
    char4 c;
    c.x = cvt_rni_sat_s8(v[i][0] * inv_scale);
    c.y = cvt_rni_sat_s8(v[i][1] * inv_scale);
    c.z = cvt_rni_sat_s8(v[i][2] * inv_scale);
    c.w = cvt_rni_sat_s8(v[i][3] * inv_scale);
    *reinterpret_cast<char4*>(out + static_cast<size_t>(t) * 128) = c;
  }
}

// ------------------------------------------------ FP8 P.V variant quantizers
// Per-block INT8 of Q (TOK = 128 queries) or of K - mean (TOK = 64 keys): one
// CTA per (block, batch-head), 8 warps, warp w on tokens w * TOK/8 .. , lane =
// 4 dims; scale = max|x| / 127 + 1e-7 (the per-thread quantizer's
// expressions over the whole block), written to the GROUPS entries of the
// block in the per-thread scale layout.
template <int TOK, int GROUPS>
__global__ void __launch_bounds__(256) sage_quant_block_kernel(const __half* __restrict__ x, const float* __restrict__ mean,
                                                               int8_t* __restrict__ codes, float* __restrict__ scales,
                                                               int S) {
  constexpr int TPW = TOK / 8;  // tokens per warp
  __shared__ float red[8];
  const int blk = blockIdx.x, bh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __half* hp = x + static_cast<size_t>(bh) * S * 128 + lane * 4;
  int8_t* out = codes + static_cast<size_t>(bh) * S * 128 + lane * 4;
  float4 mu = make_float4(0.f, 0.f, 0.f, 0.f);
  if (mean) mu = *reinterpret_cast<const float4*>(mean + bh * 128 + lane * 4);
  float v[TPW][4];
  float am = 1e-7f;
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    const int t = blk * TOK + warp * TPW + i;
    uint2 raw = make_uint2(0, 0);
    if (t < S) raw = __ldg(reinterpret_cast<const uint2*>(hp + static_cast<size_t>(t) * 128));
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    const bool in = t < S;
    v[i][0] = in ? a.x - mu.x : 0.0f;
    v[i][1] = in ? a.y - mu.y : 0.0f;
    v[i][2] = in ? b.x - mu.z : 0.0f;
    v[i][3] = in ? b.y - mu.w : 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) am = fmaxf(am, fabsf(v[i][e]));
  }
  am = warp_max_f(am);
  if (lane == 0) red[warp] = am;
  __syncthreads();
  am = red[0];
#pragma unroll
  for (int w = 1; w < 8; ++w) am = fmaxf(am, red[w]);
  const float scale = am / 127.0f + 1e-7f;
  if (threadIdx.x < GROUPS) scales[static_cast<size_t>(bh) * (((S + TOK - 1) / TOK) * GROUPS) + blk * GROUPS + threadIdx.x] = scale;
  const float inv = 1.0f / scale;
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    const int t = blk * TOK + warp * TPW + i;
    if (t >= S) continue;
    char4 c;
    c.x = cvt_rni_sat_s8(v[i][0] * inv);
    c.y = cvt_rni_sat_s8(v[i][1] * inv);
    c.z = cvt_rni_sat_s8(v[i][2] * inv);
    c.w = cvt_rni_sat_s8(v[i][3] * inv);
    *reinterpret_cast<char4*>(out + static_cast<size_t>(t) * 128) = c;
  }
}

// max |V| per (batch-head, dim) over the tokens: 256-token slices per CTA,
// combined with atomicMax on the (non-negative) float bits.
__global__ void __launch_bounds__(256) sage_v_amax_kernel(const __half* __restrict__ v, float* __restrict__ vamax, int S) {
  __shared__ float red[8][128];
  const int bh = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const __half* hp = v + static_cast<size_t>(bh) * S * 128 + lane * 4;
  float am[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int i = 0; i < 32; ++i) {
    const int t = blockIdx.x * 256 + warp + 8 * i;
    if (t >= S) break;
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(hp + static_cast<size_t>(t) * 128));
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
    am[0] = fmaxf(am[0], fabsf(a.x));
    am[1] = fmaxf(am[1], fabsf(a.y));
    am[2] = fmaxf(am[2], fabsf(b.x));
    am[3] = fmaxf(am[3], fabsf(b.y));
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) red[warp][lane * 4 + e] = am[e];
  __syncthreads();
  if (threadIdx.x < 128) {
    float m = red[0][threadIdx.x];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w][threadIdx.x]);
    atomicMax(reinterpret_cast<int*>(vamax) + bh * 128 + threadIdx.x, __float_as_int(m));
  }
}

// E4M3 codes of V / v_scale (v_scale = max|V| / 448 per dim) transposed to
// [BH][128][s_pad]: one CTA per 64 tokens of a batch-head; tokens in
// [S, s_pad) are zero.  vs = v_scale / 448, the output factor of 448 P . V.
__global__ void __launch_bounds__(256) sage_v_fp8_kernel(const __half* __restrict__ v, const float* __restrict__ vamax,
                                                         uint8_t* __restrict__ vt, float* __restrict__ vs, int S,
                                                         int s_pad) {
  __shared__ uint8_t tile[128][64 + 16];
  const int bh = blockIdx.y, t0 = blockIdx.x * 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float4 am = *reinterpret_cast<const float4*>(vamax + bh * 128 + lane * 4);
  const float inv[4] = {am.x > 0.f ? 448.0f / am.x : 0.f, am.y > 0.f ? 448.0f / am.y : 0.f,
                        am.z > 0.f ? 448.0f / am.z : 0.f, am.w > 0.f ? 448.0f / am.w : 0.f};
  if (blockIdx.x == 0 && warp == 0) {
    vs[bh * 128 + lane * 4 + 0] = am.x / (448.0f * 448.0f);
    vs[bh * 128 + lane * 4 + 1] = am.y / (448.0f * 448.0f);
    vs[bh * 128 + lane * 4 + 2] = am.z / (448.0f * 448.0f);
    vs[bh * 128 + lane * 4 + 3] = am.w / (448.0f * 448.0f);
  }
  const __half* hp = v + static_cast<size_t>(bh) * S * 128 + lane * 4;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int tl = warp * 8 + i, t = t0 + tl;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if (t < S) {
      const uint2 raw = __ldg(reinterpret_cast<const uint2*>(hp + static_cast<size_t>(t) * 128));
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      x[0] = a.x * inv[0];
      x[1] = a.y * inv[1];
      x[2] = b.x * inv[2];
      x[3] = b.y * inv[3];
    }
    const uint32_t c = pack_e4m3x4(x[0], x[1], x[2], x[3]);
#pragma unroll
    for (int e = 0; e < 4; ++e) tile[lane * 4 + e][tl] = static_cast<uint8_t>(c >> (8 * e));
  }
  __syncthreads();
  // row d of the tile: 64 bytes = four 16-byte pieces
  for (int i = threadIdx.x; i < 128 * 4; i += 256) {
    const int d = i >> 2, piece = i & 3, t = t0 + piece * 16;
    if (t >= s_pad) continue;
    const uint4 val = *reinterpret_cast<const uint4*>(&tile[d][piece * 16]);
    *reinterpret_cast<uint4*>(vt + (static_cast<size_t>(bh) * 128 + d) * s_pad + t) = val;
  }
}

// The K mean on `side` (when given) while the main stream quantizes Q; the
// main stream waits for it before the K quantizer.
static int kmean_forked(const __half* kh, float* kmean, int BH, int S, cudaStream_t stream, const SideStream* side) {
  cudaStream_t ks = stream;
  if (side) {
    if (cudaEventRecord(side->fork, stream) != cudaSuccess || cudaStreamWaitEvent(side->s, side->fork, 0) != cudaSuccess)
      return QI_ERR_CUDA;
    ks = side->s;
  }
  // one wave of CTAs: 32, 64 or 128 dims per CTA
  const int sms = device_num_sms();
  const int st = (BH * 4 <= sms) ? kmean_launch<32>(kh, kmean, BH, S, ks)
                 : (BH * 2 <= sms) ? kmean_launch<64>(kh, kmean, BH, S, ks)
                                   : kmean_launch<128>(kh, kmean, BH, S, ks);
  if (st != QI_OK) return st;
  if (side && cudaEventRecord(side->join, side->s) != cudaSuccess) return QI_ERR_CUDA;
  return QI_OK;
}
static int kmean_joined(cudaStream_t stream, const SideStream* side) {
  if (side && cudaStreamWaitEvent(stream, side->join, 0) != cudaSuccess) return QI_ERR_CUDA;
  return QI_OK;
}

int sage_quantize_fp8pv_launch(const void* q, const void* k, const void* v, int BH, int S, float* kmean, int8_t* qc,
                               float* qs, int8_t* kc, float* ks, uint8_t* vt, int s_pad, float* vamax, float* vs,
                               cudaStream_t stream, const SideStream* side) {
  if (BH <= 0 || S <= 0 || s_pad < S || s_pad % 16) return QI_ERR_ARG;
  const __half* kh = reinterpret_cast<const __half*>(k);
  const __half* vh = reinterpret_cast<const __half*>(v);
  int st = kmean_forked(kh, kmean, BH, S, stream, side);
  if (st != QI_OK) return st;
  sage_quant_block_kernel<128, 32><<<dim3((S + 127) / 128, BH), 256, 0, stream>>>(
      reinterpret_cast<const __half*>(q), nullptr, qc, qs, S);
  if ((st = kmean_joined(stream, side)) != QI_OK) return st;
  sage_quant_block_kernel<64, 4><<<dim3((S + 63) / 64, BH), 256, 0, stream>>>(kh, kmean, kc, ks, S);
  if (cudaMemsetAsync(vamax, 0, static_cast<size_t>(BH) * 128 * sizeof(float), stream) != cudaSuccess)
    return QI_ERR_CUDA;
  sage_v_amax_kernel<<<dim3((S + 255) / 256, BH), 256, 0, stream>>>(vh, vamax, S);
  sage_v_fp8_kernel<<<dim3((s_pad + 63) / 64, BH), 256, 0, stream>>>(vh, vamax, vt, vs, S, s_pad);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

int sage_quantize_launch(const void* q, const void* k, int BH, int S, float* kmean, int8_t* qc, float* qs, int8_t* kc,
                         float* ks, cudaStream_t stream, const SideStream* side) {
  if (BH <= 0 || S <= 0) return QI_ERR_ARG;
  const __half* kh = reinterpret_cast<const __half*>(k);
  int st = kmean_forked(kh, kmean, BH, S, stream, side);
  if (st != QI_OK) return st;
  sage_quant_q_kernel<<<dim3((S + 127) / 128, BH), 256, 0, stream>>>(reinterpret_cast<const __half*>(q), qc, qs, S);
  if ((st = kmean_joined(stream, side)) != QI_OK) return st;
  sage_quant_k_kernel<<<dim3((S + 127) / 128, BH), 256, 0, stream>>>(reinterpret_cast<const __half*>(k), kmean, kc, ks,
                                                                     S);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

static int encode_3d(CUtensorMap* tm, CUtensorMapDataType dt, int esize, const void* base, int S, int BH,
                     int box_d) {
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(128 * esize), static_cast<cuuint64_t>(S) * 128 * esize};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_d), 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = qi_encode_tiled(tm, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QI_OK : QI_ERR_CUDA;
}

// E4M3 V^T codes [BH][128 dims][s_pad tokens]: 128-key x 128-dim boxes
// (128 bytes along the tokens, the K dimension of P.V), 128-byte swizzle.
static int encode_vt(CUtensorMap* tm, const void* base, int s_pad, int BH) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(s_pad), 128, static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(s_pad), static_cast<cuuint64_t>(s_pad) * 128};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = qi_encode_tiled(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QI_OK : QI_ERR_CUDA;
}

int attention_launch(const AttnArgs& a, cudaStream_t stream, int* err_dev) {
  if (a.BH <= 0 || a.S <= 0) return QI_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(a.qc) & 15) || (reinterpret_cast<uintptr_t>(a.kc) & 15) ||
      (reinterpret_cast<uintptr_t>(a.v) & 15) || (reinterpret_cast<uintptr_t>(a.out) & 15))
    return QI_ERR_ALIGN;
  if (a.S > attn::MAX_S) return QI_ERR_UNSUPPORTED;
  // The setmaxnreg split assumes the kernel was built for exactly LAUNCH_REGS
  // registers per thread; with fewer, the softmax warpgroups' increase could
  // never be granted.  Refuse to launch rather than risk that.
  if (a.fp8 && (!a.vs || a.s_pad < a.S || a.s_pad % 16)) return QI_ERR_ARG;
  // the four instantiations: [fp8][tiles per CTA - 1]
  const void* kfns[2][2] = {{reinterpret_cast<const void*>(sage_attn_kernel<false, 1>),
                             reinterpret_cast<const void*>(sage_attn_kernel<false, 2>)},
                            {reinterpret_cast<const void*>(sage_attn_kernel<true, 1>),
                             reinterpret_cast<const void*>(sage_attn_kernel<true, 2>)}};
  static int regs_checked[2][2] = {{0, 0}, {0, 0}};
  static unsigned long long attr_done[2][2] = {{0, 0}, {0, 0}};
  const int f8 = a.fp8 ? 1 : 0;
  for (int nt = 0; nt < 2; ++nt) {
    if (!regs_checked[f8][nt]) {
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, kfns[f8][nt]) != cudaSuccess) return QI_ERR_CUDA;
      if (fa.numRegs != attn::LAUNCH_REGS) return QI_ERR_UNSUPPORTED;
      regs_checked[f8][nt] = 1;
    }
    if (smem_optin(kfns[f8][nt], attn::smem_bytes(((attn::MAX_S + 63) / 64) * 4), &attr_done[f8][nt]) != QI_OK)
      return QI_ERR_CUDA;
  }
  AttnArgsDev d;
  memset(&d, 0, sizeof(d));
  if (encode_3d(&d.tmQ, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.qc, a.S, a.BH, 128) != QI_OK) return QI_ERR_CUDA;
  if (encode_3d(&d.tmK, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.kc, a.S, a.BH, 128) != QI_OK) return QI_ERR_CUDA;
  if (a.fp8) {
    if (encode_vt(&d.tmV, a.v, a.s_pad, a.BH) != QI_OK) return QI_ERR_CUDA;
  } else if (encode_3d(&d.tmV, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.v, a.S, a.BH, 64) != QI_OK) {
    return QI_ERR_CUDA;
  }
  d.vs = a.vs;
  d.qs = a.qs;
  d.ks = a.ks;
  d.out = a.out;
  d.BH = a.BH;
  d.S = a.S;
  d.heads = a.heads;
  d.out_mode = a.out_mode;
  d.nb = a.nb;
  d.n_img = a.n_img;
  d.n_txt = a.n_txt;
  d.ngq = ((a.S + 127) / 128) * 32;
  d.ngk = ((a.S + 63) / 64) * 4;
  d.qk_scale = a.sm_scale * 1.44269504088896340736f;
  d.err = err_dev;
  d.map = a.map;
  for (int i = 0; i < kMaxRanks; ++i) d.peer_o[i] = a.peer_o[i];
  d.head_base = a.head_base;
  if (a.out_mode >= 2 && (a.map.P < 1 || a.map.P > kMaxRanks)) return QI_ERR_ARG;
  // Two-tile CTAs (one per SM), except that in a launch of a few waves the
  // last, partial wave is run as one-tile CTAs when that shortens it: x1
  // two-tile CTAs per batch-head cover tiles [0, 2 x1), then one-tile CTAs
  // the rest, if those fit in one wave and the estimate (a one-tile CTA takes
  // ~0.55 of a two-tile one) beats the two-tile grid alone.  Measured at the
  // C4 sequence on one B200: 6 heads (8-GPU share) 3.4 % and 12 heads 2 %
  // faster; 48 heads (ten waves, whose sparse last wave runs uncontended)
  // 3 % slower, hence the limit of four waves.  QI_ATTN_TAIL=0 turns the
  // split off (measurements).
  static int tail_split = -1;
  if (tail_split < 0) {
    const char* e = getenv("QI_ATTN_TAIL");
    tail_split = (e && atoi(e) == 0) ? 0 : 1;
  }
  const int ntiles = (a.S + attn::BQ - 1) / attn::BQ;
  const int pairs = (ntiles + 1) / 2;
  const int sms = device_num_sms();
  int x1 = pairs;
  if (tail_split) {
    const long long cover = static_cast<long long>(ntiles) * a.BH - sms;  // tiles the two-tile CTAs must take
    const int x = cover <= 0 ? 0 : static_cast<int>((cover + 2LL * a.BH - 1) / (2LL * a.BH));
    const long long waves = (static_cast<long long>(pairs) * a.BH + sms - 1) / sms;
    if (x < pairs && waves <= 4) {
      const long long waves1 = (static_cast<long long>(x) * a.BH + sms - 1) / sms;
      if (waves1 * 100 + 55 < waves * 100) x1 = x;
    }
  }
  auto launch = [&](int nt, int tile0, int nx) {
    if (nx <= 0) return;
    d.q_tile0 = tile0;
    dim3 grid(nx, a.BH);
    const size_t smem = attn::smem_bytes(d.ngk);
    if (a.fp8) {
      if (nt == 2) sage_attn_kernel<true, 2><<<grid, attn::THREADS, smem, stream>>>(d);
      else sage_attn_kernel<true, 1><<<grid, attn::THREADS, smem, stream>>>(d);
    } else {
      if (nt == 2) sage_attn_kernel<false, 2><<<grid, attn::THREADS, smem, stream>>>(d);
      else sage_attn_kernel<false, 1><<<grid, attn::THREADS, smem, stream>>>(d);
    }
  };
  launch(2, 0, x1);
  launch(1, 2 * x1, ntiles - 2 * x1);
  return cudaGetLastError() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
}

}  // namespace qi
