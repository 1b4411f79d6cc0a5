"""Benchmark: seconds per CFG denoising step of the Qwen-Image MMDiT at 1328x1328.

Workload ("C4", the headline configuration): 166x166 latent -> 6889 image
tokens + 256 text tokens, 60 double-stream blocks, W8A8 INT8 weights in
quantize.cu's format produced from seeded N(0, 0.02^2) BF16 weights, CFG
scale 4.0, flow-matching Euler with fixed shift 3.0 over 50 sigmas.  One step
= the cond and uncond forwards (batched: nb = 2 in one pass) + the
norm-preserving CFG combine and Euler update.  Synthetic inputs (no
checkpoint or dataset is available): latents and text states ~ N(0, 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun, one process per GPU), one denoising job (strong scaling):
the cond and uncond halves go to two groups of N/2 ranks; within a half the
forward is head-parallel (Ulysses) over the N/2 ranks when N/2 > 1 (two NCCL
all-to-alls per block inside the library); one NCCL all-gather of the two
halves' velocities per step, then every rank runs the same Euler step.

Prints one JSON line (rank 0).  `value` is seconds per step on the device
with inputs resident in HBM (CUDA events, max over ranks), timed with the
stage profiler off; `e2e` is the same step (forward, gather, CFG + Euler)
through the C ABI with host buffers (H2D of the step's latent, text states and
RoPE tables and D2H of the updated latent inside the timed region).  The
per-stage split and the kernel rooflines come from a separate profiled pass
over the same number of steps after the timed region (CUDA events around
every launch).  `velocity_sha256` is the SHA-256 of the first timed step's
BF16 velocities (cond, uncond) on rank 0: the forward is bit-identical on any
number of GPUs, so every N prints the same digest.  The 20.4 GB of INT8
weights streamed every step exceed the 126 MB L2, so no flush is needed
between steps.
"""
import hashlib
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen-image.cu_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

# default workload C4 (1328x1328); --workload c5 switches to the high-resolution
# scaling configuration (2048x2048: 256x256 latent, 16384 image + 512 text tokens, 20 steps)
WORKLOAD = "c4"
H_LAT = W_LAT = 166
N_TXT = 256
BLOCKS = 60
CFG_SCALE = 4.0
SHIFT = 3.0
SCHED_STEPS = 50
N_IMG = (H_LAT // 2) * (W_LAT // 2)
S_JOINT = N_IMG + N_TXT
DIM, MLP = 3072, 12288
METRIC = "MMDiT sec/denoise-step at 1328^2 @1/2/4/8 B200; % of tensor-core peak"


def sigmas_fixed_shift(n, shift):
    """FlowMatchScheduler.get_sigmas, fixed-shift branch (scheduler.h:62-101)."""
    s = [1.0 + (1.0 / n - 1.0) * i / (n - 1) for i in range(n)]
    s = [shift * t / (1.0 + (shift - 1.0) * t) for t in s]
    return s + [0.0]


def flops_per_forward(n_img, n_txt, blocks=BLOCKS):
    """Algorithmic FLOPs of one forward: INT8 linears + attention (QK + PV)."""
    toks = n_img + n_txt
    lin = 2.0 * toks * (4 * DIM * DIM + 2 * DIM * MLP) * blocks
    attn = 4.0 * toks * toks * DIM * blocks
    return lin, attn


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons of this rank's GPU, sampled
    every 50 ms through NVML on a host thread while the timed region runs
    (read-only: nothing is set).  NVML is initialised on entry, which takes a
    different time on each rank: the ranks' barrier that opens the timed
    region comes after it (with NVML started after the barrier, a 2-GPU step
    timed 0.120 s against 0.099 s for the same step untimed by it, the start-up
    skew showing up in the max over ranks).  The device is found by UUID, so
    the index under CUDA_VISIBLE_DEVICES does not matter.  Falls back to
    `nvidia-smi -lms 200` if NVML is unavailable."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index, period_s=0.05):
        self.index = index
        self.period_s = period_s
        self.rows = []  # (sm_mhz, max_mhz, set of reason names)
        self.proc = None
        self.nvml = None
        self.stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:
            uuid = str(torch.cuda.get_device_properties(self.index).uuid)
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _nvml_sample(self):
        nv, h = self.nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        masks = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                 nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        self.rows.append((float(sm), float(mx), {n for n, m in zip(self.NAMES, masks) if bits & m}))

    def _nvml_loop(self):
        while not self.stop.is_set():
            try:
                self._nvml_sample()
            except Exception:
                return
            self.stop.wait(self.period_s)

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
            self._nvml_sample()  # fails here, not silently in the thread, if NVML cannot read this GPU
            self.rows.clear()
            self.thread = threading.Thread(target=self._nvml_loop, daemon=True)
            self.thread.start()
            return self
        except Exception:
            self.nvml = None
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._smi_read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _smi_read(self):
        for line in self.proc.stdout:
            r = [v.strip() for v in line.split(",")]
            try:
                self.rows.append((float(r[1]), float(r[2]),
                                  {n for n, v in zip(self.NAMES, r[5:9]) if v.lower().startswith("active")}))
            except (ValueError, IndexError):
                continue

    def __exit__(self, *a):
        if self.nvml:
            self.stop.set()
            self.thread.join(timeout=1.0)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm = [r[0] for r in self.rows]
        reasons = set().union(*[r[2] for r in self.rows]) if self.rows else set()
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": self.rows[-1][1] if self.rows else None, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvml" if self.nvml else "nvidia-smi"}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def init_dist(world, local):
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))


def barrier(world):
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import qib200 as Q
    import topology as T

    rank, world, local = dist_env()
    init_dist(world, local)
    pair, P = T.layout(world)  # CFG split over two rank groups; head-parallel size P within a half
    role = T.roles(rank, world)
    half = role["half"]  # CFG half of this rank (None: both halves batched here)
    nb = 1 if pair else 2
    g, blocks = Q.make_weight_table(BLOCKS, base_seed=0)
    ctx = Q.Context(local)
    model = Q.Model(ctx, g, blocks)
    del g, blocks
    torch.cuda.empty_cache()
    group = None
    if pair:
        # every rank creates every group, in the same order
        ugroups = [torch.distributed.new_group([h * P + u for u in range(P)]) for h in range(2)] if P > 1 else None
        pairs = [torch.distributed.new_group([u, P + u]) for u in range(P)]
        group = pairs[role["urank"]]
        if P > 1:  # the library's NCCL communicator for this half's head-parallel group
            uid = torch.zeros(Q.COMM_ID_BYTES, dtype=torch.uint8, device="cuda")
            if role["urank"] == 0:
                uid.copy_(torch.frombuffer(bytearray(Q.comm_unique_id()), dtype=torch.uint8))
            torch.distributed.broadcast(uid, src=half * P, group=ugroups[half])
            ctx.set_comm(bytes(uid.cpu().numpy()), role["urank"], P)

    sig = sigmas_fixed_shift(SCHED_STEPS, SHIFT)
    job = 0  # one denoising job over all ranks
    latent = Q.synth((1, 16, H_LAT, W_LAT), Q.seed_for(100 + job, "noise"), sig[0])
    lat_bf = latent.to(torch.bfloat16)
    ctxs = torch.stack([Q.synth((N_TXT, 3584), Q.seed_for(100 + job, f"context_{b}"), 1.0, dtype=torch.bfloat16)
                        for b in range(2)])
    pe1 = torch.from_numpy(Q.rope_table(H_LAT, W_LAT, N_TXT)).cuda()
    pe = torch.stack([pe1, pe1]) if nb == 2 else pe1[None]
    my_ctx = ctxs if nb == 2 else ctxs[half:half + 1].contiguous()
    vel = torch.empty(nb, 16, H_LAT, W_LAT, dtype=torch.bfloat16, device="cuda")
    gathered = torch.empty(2, 16, H_LAT, W_LAT, dtype=torch.bfloat16, device="cuda")
    stream = torch.cuda.current_stream()

    snap = torch.empty(2, 16, H_LAT, W_LAT, dtype=torch.bfloat16, device="cuda")

    def step(i, lat=latent, lat16=lat_bf, text=my_ctx, rope=pe, keep=False):
        s, s_next = sig[i % SCHED_STEPS], sig[i % SCHED_STEPS + 1]
        x = lat16.expand(nb, -1, -1, -1).contiguous() if nb == 2 else lat16
        Q.forward(ctx, model, x, s * 1000.0, text, rope, out=vel)
        if pair:
            torch.distributed.all_gather_into_tensor(gathered, vel, group=group)
            v = gathered
        else:
            v = vel
        if keep:  # the first timed step's velocities, for the digest (a 1.7 MB device copy)
            snap.copy_(v)
        Q.cfg_euler_step(lat, v[0], v[1], CFG_SCALE, s, s_next, lat16)

    for i in range(args.warmup):
        step(i)
    ctx.check()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        # NVML starts up before the barrier, so the ranks enter the timed
        # region together (its start-up time differs between ranks)
        barrier(world)
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i, keep=(i == 0))
        e1.record(stream)
        barrier(world)
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world)
    launches_per_forward = ctx.launches()
    ctx.check()
    digest = hashlib.sha256(snap.view(torch.int16).cpu().numpy().tobytes()).hexdigest()

    # profiled pass (not timed): CUDA events around every launch of the same
    # number of steps give the per-stage split and the kernel durations
    Q.lib().qi_ctx_set_profiling(ctx.h, 1)
    Q.lib().qi_ctx_profile(ctx.h, None, None, 1)
    barrier(world)
    for i in range(args.steps):
        step(args.warmup + args.steps + i)
    barrier(world)
    nprof = 13
    import ctypes
    pl = (ctypes.c_int * nprof)()
    pm = (ctypes.c_float * nprof)()
    Q.check(Q.lib().qi_ctx_profile(ctx.h, pl, pm, 1))
    Q.lib().qi_ctx_set_profiling(ctx.h, 0)
    ctx.check()

    # e2e: the same step (forward, gather, CFG + Euler) through the C ABI from
    # pinned host buffers: the latent, text states and RoPE tables go up and
    # the updated latent comes back every step
    h_lat = latent.cpu().pin_memory()
    h_ctx = my_ctx.cpu().pin_memory()
    h_pe = pe.cpu().pin_memory()
    d_lat = torch.empty_like(latent)
    d_lat16 = torch.empty_like(lat_bf)
    d_ctx = torch.empty_like(my_ctx)
    d_pe = torch.empty_like(pe)
    barrier(world)
    base = args.warmup + 2 * args.steps
    e0.record(stream)
    for i in range(args.steps):
        d_lat.copy_(h_lat, non_blocking=True)
        d_ctx.copy_(h_ctx, non_blocking=True)
        d_pe.copy_(h_pe, non_blocking=True)
        d_lat16.copy_(d_lat)
        step(base + i, lat=d_lat, lat16=d_lat16, text=d_ctx, rope=d_pe)
        h_lat.copy_(d_lat, non_blocking=True)
    e1.record(stream)
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    bi = h_lat.numel() * 4 + h_ctx.numel() * 2 + h_pe.numel() * 4
    bo = h_lat.numel() * 4

    if rank != 0:
        model.close()
        ctx.close()
        if world > 1:
            torch.distributed.destroy_process_group()
        return

    peaks, psrc = measured_peaks()
    # the kernels run inside a seconds-long step: sustained (power-capped)
    # rates.  INT8 and FP16 are measured on this pool by kernel_bench.py
    # --which peaks (profiles/peaks_b200.json); without that file, INT8 is
    # taken as 2 x the driver's BF16 figure and FP16 as equal to it.
    bf16_sus = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    int8_peak, fp16_peak = 2.0 * bf16_sus, bf16_sus
    peak_note = f"INT8 = 2 x bf16_tflops_sustained, FP16 = bf16_tflops_sustained ({psrc}, MEASURED_PEAKS.json)"
    ppath = os.path.join(ROOT, "profiles", "peaks_b200.json")
    if os.path.exists(ppath):
        with open(ppath) as f:
            pk = json.load(f)
        # INT8: the larger of the library's measured sustained rate (cuBLASLt
        # through torch._int_mm, below the hardware's 2x BF16) and 2 x the
        # measured sustained BF16 rate; FP16: the measured sustained rate
        i8 = pk["peak_int8"]["sustained_tflops"]
        int8_peak = max(i8, 2.0 * bf16_sus)
        fp16_peak = pk["peak_fp16"]["sustained_tflops"]
        peak_note = (f"of measured: INT8 = max(torch._int_mm sustained {i8}, 2 x bf16_tflops_sustained "
                     f"{2.0 * bf16_sus:.1f}); FP16 = torch.matmul sustained {fp16_peak} (8192^3, 4 s; "
                     "profiles/peaks_b200.json, MEASURED_PEAKS.json)")
    # attention: the QK^T half of the FLOPs on INT8, the P.V half on FP16
    attn_peak = 2.0 / (1.0 / int8_peak + 1.0 / fp16_peak)
    lin_f, attn_f = flops_per_forward(N_IMG, N_TXT)
    gemm_stages = [2, 7, 8, 10]  # QI_PROF_GEMM_QKV, _OUT, _FC1, _FC2
    gemm_ms = sum(pm[i] for i in gemm_stages)
    gemm_n = sum(pl[i] for i in gemm_stages)
    # every INT8 linear of this rank's tokens runs in these launches (1/P of the tokens)
    gemm_flops_total = lin_f * nb * args.steps / P
    avg_launch_ms = gemm_ms / max(gemm_n, 1)
    achieved = gemm_flops_total / gemm_n / (avg_launch_ms * 1e-3) / 1e12 if gemm_n else None
    attn_ms = pm[5]
    attn_n = pl[5]
    attn_tflops = attn_f * nb * args.steps / P / (attn_ms * 1e-3) / 1e12 if attn_ms > 0 else None
    stage_names = ["pre", "quant_ln", "gemm_qkv", "qkv_post", "sage_quant", "attention", "quant_o", "gemm_out",
                   "gemm_fc1", "quant_h", "gemm_fc2", "post", "exchange"]
    stages = {n: {"launches": int(pl[i]), "ms_per_step": round(pm[i] / args.steps, 3)}
              for i, n in enumerate(stage_names)}

    cpu = cpu_baseline(args) if (world == 1 and not args.no_cpu) else None
    # DRAM bytes per launch from one ncu capture (profiles/traffic.json)
    traffic = {}
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        with open(tpath) as f:
            traffic = json.load(f)
    line = {
        "metric": METRIC,
        "value": round(ms / 1000.0, 5),
        "unit": "s/step",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded N(0,1) latents/text states; random-init N(0,0.02^2) weights quantized to INT8)",
        "config": {"workload": f"{WORKLOAD.upper()}: {H_LAT * 8}x{W_LAT * 8}, {N_IMG} img + {N_TXT} txt tokens, CFG "
                               "cond+uncond, 60 blocks, W8A8 + SageAttention (INT8 QK, FP16 PV)",
                   "latent": [16, H_LAT, W_LAT], "n_img": N_IMG, "n_txt": N_TXT, "blocks": BLOCKS,
                   "cfg": "batched (nb=2) on 1 GPU" if world == 1 else "cond/uncond on two rank groups",
                   "parallelism": "single" if world == 1 else ("cfg2" if P == 1 else f"cfg2 x ulysses{P}"),
                   "l2": "no flush: 20.4 GB of INT8 weights streamed per step >> 126 MB L2"},
        "e2e": {"value": round(e2e_ms / 1000.0, 5), "unit": "s/step", "h2d_bytes_per_step": bi,
                "d2h_bytes_per_step": bo},
        "gpu_launches": (launches_per_forward + 1) * args.steps,
        # the dominant kernel: SageAttention (INT8 QK^T + FP16 P.V)
        "roofline": {"kernel": "sage_attn_kernel (tcgen05 INT8 QK^T + FP16 P.V)", "bound": "tensor",
                     "achieved": round(attn_tflops, 1) if attn_tflops else None, "peak": round(attn_peak, 1),
                     "unit": "TFLOP/s", "frac": round(attn_tflops / attn_peak, 4) if attn_tflops else None,
                     "traffic": traffic.get("sage_attn_kernel"),
                     "peak_source": f"2 / (1 / INT8 + 1 / FP16), half the FLOPs on each; {peak_note}",
                     "flops_per_launch": attn_f * nb / P / BLOCKS,
                     "avg_launch_ms": attn_ms / max(attn_n, 1)},
        "roofline_gemm": {"kernel": "gemm_kernel / gemm_pair_kernel (tcgen05 kind::i8 W8A8 GEMM)", "bound": "tensor",
                          "achieved": round(achieved, 1) if achieved else None, "peak": round(int8_peak, 1),
                          "unit": "TFLOP/s", "frac": round(achieved / int8_peak, 4) if achieved else None,
                          "traffic": traffic.get("gemm_kernel"),
                          "peak_source": f"INT8; {peak_note}",
                          "flops_per_launch": gemm_flops_total / max(gemm_n, 1), "avg_launch_ms": avg_launch_ms},
        "attention": {"tflops": round(attn_tflops, 1) if attn_tflops else None,
                      "ms_per_step": round(attn_ms / args.steps, 3)},
        "stages": stages,
        "stages_note": "CUDA events around every launch in a profiled pass of the same steps after the timed region",
        "velocity_sha256": digest,
        "clocks": clk.summary(),
    }
    if cpu:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    model.close()
    ctx.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def cpu_baseline(args):
    """The FP32 CPU evaluation (CPU oracle, unquantized) of one double-stream
    block at the C1 size (1024 image + 64 text tokens, the reference's
    block-verify configuration), timed on the host cores and scaled by the
    algorithmic FLOP ratio to one C4 denoising step (2 x 60 blocks at 7145
    tokens)."""
    import qi_oracle as O
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    W = O.Weights(1)
    n_img, n_txt = 1024, 64
    img = O.gen_f32(1, (n_img, DIM))
    txt = O.gen_f32(2, (n_txt, DIM))
    mi = O.gen_f32(3, (6 * DIM,), 0.1)
    mt = O.gen_f32(4, (6 * DIM,), 0.1)
    pe = O.rope_table(64, 64, n_txt)
    O.block_fp32(W, img[:8], txt[:8], mi, mt, pe)  # materialise the weights
    best = None
    for _ in range(2):
        t0 = time.time()
        O.block_fp32(W, img, txt, mi, mt, pe)
        dt = time.time() - t0
        best = dt if best is None else min(best, dt)
    lin_b, attn_b = flops_per_forward(n_img, n_txt, blocks=1)
    lin_s, attn_s = flops_per_forward(N_IMG, N_TXT)
    scale = 2.0 * (lin_s + attn_s) / (lin_b + attn_b)
    return {"value": round(best * scale, 2), "unit": "s/step", "cores": threads, "kind": "port",
            "extrapolated": True,
            "sample": f"extrapolated: one FP32 block at C1 (1024+64 tokens, {best:.2f} s, best of 2) timed, x {scale:.0f} "
                      f"(FLOP ratio to one C4 CFG step)"}


# ------------------------------------------------------------------ loader
def _write_checkpoint(path, blocks):
    """A quantize.cu-format INT8 checkpoint (transformer.h:407-563 names) of
    `blocks` double-stream blocks, streamed tensor by tensor (every block
    carries the same synthetic tensors)."""
    import qib200 as Q
    g, bl = Q.make_weight_table(1, base_seed=0)
    dt = {torch.int8: "I8", torch.float32: "F32", torch.bfloat16: "BF16"}
    entries = [(name, t) for (name, kind), t in zip(Q.G_NAMES, g)]
    for i in range(blocks):
        pre = f"transformer_blocks.{i}."
        for li, (lname, N, K) in enumerate(Q.L_NAMES):
            c, sc, b = bl[0][3 * li:3 * li + 3]
            entries += [(pre + lname + ".weight", c), (pre + lname + ".weight.__scales__", sc),
                        (pre + lname + ".bias", b)]
        for k, nname in enumerate(Q.B_NORMS):
            entries.append((pre + nname, bl[0][3 * len(Q.L_NAMES) + k]))
    header, off = {}, 0
    for name, t in entries:
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": dt[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    import struct
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        host = {}
        for name, t in entries:
            key = t.data_ptr()
            if key not in host:
                host[key] = (t.view(torch.int16) if t.dtype == torch.bfloat16 else t).cpu().numpy().tobytes()
            f.write(host[key])
    return 8 + len(h) + off


def run_loader(args):
    """Checkpoint load throughput: the product's loader (qi_model_load_safetensors:
    pinned chunked upload, then the kernels' layout) against the reference's
    per-tensor path (safetensors.h:174-212) on the same file, page cache warm
    for both; GB of file per second."""
    import shutil
    import tempfile
    import qib200 as Q
    import qi_ref as R
    torch.cuda.set_device(0)
    tmp = tempfile.mkdtemp(prefix="qi_ckpt_")
    try:
        free = shutil.disk_usage(tmp).free
        blocks = max(1, min(args.loader_blocks, int(free * 0.25 // 345e6)))
        path = os.path.join(tmp, "transformer_int8.safetensors")
        size = _write_checkpoint(path, blocks)
        with open(path, "rb") as f:  # warm the page cache
            while f.read(1 << 26):
                pass
        ctx = Q.Context(0)
        res = {"metric": "INT8 safetensors checkpoint load, GB/s of file (page cache warm)", "file_gb": round(size / 1e9, 3),
               "blocks": blocks}
        best = {}
        for _ in range(2):
            for arm in ("product", "reference"):
                torch.cuda.synchronize()
                t0 = time.time()
                if arm == "product":
                    m = Q.Model.from_safetensors(ctx, path)
                    torch.cuda.synchronize()
                    dt = time.time() - t0
                    m.close()
                else:
                    if not R.available():
                        continue
                    R.load_all(path)
                    dt = time.time() - t0
                best[arm] = min(best.get(arm, 1e9), dt)
        for arm, dt in best.items():
            res[arm] = {"seconds": round(dt, 3), "gbs": round(size / dt / 1e9, 2)}
        ctx.close()
        print(json.dumps(res), flush=True)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    import qi_ref as R
    if not R.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libqiref.so (reference build) missing"}))
        return
    g, blocks = R.make_table(BLOCKS, distinct=BLOCKS)
    garr, barrs, bt = R.table_pointers(g, blocks)
    sig = sigmas_fixed_shift(SCHED_STEPS, SHIFT)
    latent = R.synth((1, 16, H_LAT, W_LAT), R.seed_for(100, "noise"), sig[0])
    ctxs = [R.synth((1, N_TXT, 3584), R.seed_for(100, f"context_{b}"), 1.0, dtype=torch.bfloat16) for b in range(2)]
    import numpy as _np  # noqa: F401
    pe = torch.from_numpy(R.rope_table(H_LAT, W_LAT, N_TXT)).cuda()
    stream = torch.cuda.current_stream()

    def step(i):
        s, s_next = sig[i % SCHED_STEPS], sig[i % SCHED_STEPS + 1]
        x = latent.to(torch.bfloat16)
        vc = R.transformer_forward(garr, bt, x, s * 1000.0, ctxs[0], pe, H_LAT, W_LAT, sage=True).float()
        vu = R.transformer_forward(garr, bt, x, s * 1000.0, ctxs[1], pe, H_LAT, W_LAT, sage=True).float()
        # the caller's norm-preserving CFG + Euler (main.cu:817-868) as plain torch ops
        comb = vu + CFG_SCALE * (vc - vu)
        grp = lambda t: t.reshape(16, H_LAT // 2, 2, W_LAT // 2, 2).permute(1, 3, 0, 2, 4).reshape(-1, 64)
        r = grp(vc).norm(dim=1) / grp(comb).norm(dim=1).clamp_min(1e-30)
        v = (grp(comb) * r[:, None]).reshape(H_LAT // 2, W_LAT // 2, 16, 2, 2).permute(2, 0, 3, 1, 4)
        v = v.reshape(1, 16, H_LAT, W_LAT)
        den = latent - s * v
        latent.copy_(latent + (latent - den) / s * (s_next - s))

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for i in range(args.steps):
            step(args.warmup + i)
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": round(ms / 1000.0, 5),
        "unit": "s/step",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 3),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (same seeds as the product arm)",
        "config": {"workload": f"{WORKLOAD.upper()}: {H_LAT * 8}x{W_LAT * 8}, {N_IMG} img + {N_TXT} txt tokens, CFG "
                               "cond+uncond, 60 blocks, W8A8 + SageAttention sm80 (reference build, transformer_forward "
                               "x2 per step)",
                   "latent": [16, H_LAT, W_LAT], "n_img": N_IMG, "n_txt": N_TXT, "blocks": BLOCKS},
        "cpu_baseline": {"value": round(ms / 1000.0, 5), "unit": "s/step", "cores": 0, "kind": "reference",
                         "sample": "the reference's own CUDA build (it has no CPU path) timed on one GPU"},
        "e2e": {"value": round(ms / 1000.0, 5), "unit": "s/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def _time_ms(fn, iters=5, warmup=2):
    for _ in range(warmup):
        fn()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def reference_kernels(args):
    """The reference's own kernels on this GPU, beside ours on the same inputs and
    shapes (`--impl reference --kernels`): its SageAttention kernel alone
    (attention_forward_sage_sm80_fp16io) at the Sage microbenchmark (C2) and the
    C4 joint sequence; its INT8 linear on pre-quantized inputs (cuBLAS INT8 +
    dequant / GELU, linear_forward_int8_prequantized) at the C4 block shapes;
    its whole forward with the default materialised-softmax attention at C4;
    and its own per-stage split of the Sage forward (the PROFILE_BLOCK hook,
    transformer.cu:486-860, read from a child process's log)."""
    rank, world, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    import qi_ref as R
    import qib200 as Q
    if not R.available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libqiref.so (reference build) missing"}))
        return
    res = {"impl": "reference", "mode": "kernels", "attention": {}, "linear_int8_preq": {}}
    for name, S in (("c2", 4352), ("c4", S_JOINT)):
        BH = 48
        q, k, v = (R.synth((BH, S, 128), R.seed_for(110, f"{n}_{S}"), 1.0).half() for n in "qkv")
        flops = 4.0 * BH * S * S * 128
        ms_ref = _time_ms(lambda: R.sage_attention(q, k, v, 1.0 / 128 ** 0.5))
        ms_our = _time_ms(lambda: Q.sage_attention(q, k, v))
        res["attention"][name] = {"BH": BH, "S": S, "reference_ms": round(ms_ref, 4), "ours_ms": round(ms_our, 4),
                                  "reference_tflops": round(flops / ms_ref / 1e9, 1),
                                  "ours_tflops": round(flops / ms_our / 1e9, 1)}
        del q, k, v
    M = 2 * N_IMG + 2 * N_TXT
    for name, N, K, gelu in (("qkv", 3 * DIM, DIM, False), ("out", DIM, DIM, False), ("fc1", MLP, DIM, True),
                             ("fc2", DIM, MLP, False)):
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
        w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
        sa = torch.rand(M, device="cuda") * 1e-3
        sw = torch.rand(N, device="cuda") * 1e-3
        b = torch.zeros(N, dtype=torch.bfloat16, device="cuda")
        out = torch.empty(M, N, device="cuda")
        ms_ref = _time_ms(lambda: R.linear_int8_preq(a, sa, w, sw, b, gelu))
        ms_our = _time_ms(lambda: Q.linear_i8(a, sa, w, sw, b, Q.EPI_GELU if gelu else Q.EPI_STORE, out=out))
        ops = 2.0 * M * N * K
        res["linear_int8_preq"][name] = {"M": M, "N": N, "K": K, "reference_ms": round(ms_ref, 4),
                                         "ours_ms": round(ms_our, 4), "reference_tops": round(ops / ms_ref / 1e9, 1),
                                         "ours_tops": round(ops / ms_our / 1e9, 1)}
        del a, w, out
    g, blocks = R.make_table(BLOCKS, distinct=BLOCKS)
    garr, _, bt = R.table_pointers(g, blocks)
    x = R.synth((1, 16, H_LAT, W_LAT), R.seed_for(100, "noise"), 1.0).to(torch.bfloat16)
    ctx0 = R.synth((1, N_TXT, 3584), R.seed_for(100, "context_0"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(R.rope_table(H_LAT, W_LAT, N_TXT)).cuda()
    for sage in (True, False):
        ms = _time_ms(lambda: R.transformer_forward(garr, bt, x, 500.0, ctx0, pe, H_LAT, W_LAT, sage=sage), 2, 1)
        res["forward_sage" if sage else "forward_default_attention"] = {"ms_per_forward": round(ms, 2)}
    del g, blocks
    torch.cuda.empty_cache()
    env = dict(os.environ, PROFILE_BLOCK="1", QWEN_VERBOSE="1")
    r = subprocess.run([sys.executable, os.path.abspath(__file__), "--impl", "reference", "--profile-block"],
                       env=env, capture_output=True, text=True, timeout=900)
    split, on = {}, False
    for line in r.stderr.splitlines():
        if "Block Loop Profile" in line:
            split, on = {}, True
        elif on and line.strip().startswith("===="):
            on = False
        elif on and ":" in line and "ms" in line:
            key, rest = line.split(":", 1)
            split[key.strip()] = float(rest.split("ms")[0])
    res["reference_stage_split_ms"] = split or {"unavailable": (r.stderr or "")[-300:]}
    print(json.dumps(res), flush=True)


def reference_profile_child():
    """One Sage forward of the reference at the bench workload, run with the
    reference's PROFILE_BLOCK hook on (per-stage events, each synchronised);
    the parent reads the printed split."""
    torch.cuda.set_device(0)
    import qi_ref as R
    g, blocks = R.make_table(BLOCKS, distinct=BLOCKS)
    garr, _, bt = R.table_pointers(g, blocks)
    x = R.synth((1, 16, H_LAT, W_LAT), R.seed_for(100, "noise"), 1.0).to(torch.bfloat16)
    ctx0 = R.synth((1, N_TXT, 3584), R.seed_for(100, "context_0"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(R.rope_table(H_LAT, W_LAT, N_TXT)).cuda()
    for _ in range(2):  # the second forward's split is the one kept
        R.transformer_forward(garr, bt, x, 500.0, ctx0, pe, H_LAT, W_LAT, sage=True)
    torch.cuda.synchronize()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--loader", action="store_true",
                    help="time the checkpoint loader against the reference's instead of the step")
    ap.add_argument("--loader-blocks", type=int, default=8, help="blocks in the --loader checkpoint")
    ap.add_argument("--kernels", action="store_true",
                    help="with --impl reference: the reference's kernels beside ours (attention, INT8 linear, "
                         "default-attention forward, the reference's per-stage split)")
    ap.add_argument("--profile-block", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--workload", default="c4", choices=["c4", "c5"],
                    help="c4: 1328x1328 (the headline metric); c5: 2048x2048, 20 steps (scaling study)")
    args = ap.parse_args()
    if args.workload == "c5":
        global WORKLOAD, H_LAT, W_LAT, N_TXT, SCHED_STEPS, N_IMG, S_JOINT, METRIC
        WORKLOAD, H_LAT, W_LAT, N_TXT, SCHED_STEPS = "c5", 256, 256, 512, 20
        N_IMG = (H_LAT // 2) * (W_LAT // 2)
        S_JOINT = N_IMG + N_TXT
        METRIC = "MMDiT sec/denoise-step at 2048^2 @1/2/4/8 B200 (scaling study)"
    if args.warmup < 3:
        print("warmup < 3 is not a valid measurement; using 3", file=sys.stderr)
        args.warmup = 3
    if args.profile_block:
        reference_profile_child()
    elif args.loader:
        run_loader(args)
    elif args.impl == "reference" and args.kernels:
        reference_kernels(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
