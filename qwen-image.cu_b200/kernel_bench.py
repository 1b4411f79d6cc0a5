"""Kernel-level timing of the hot kernels at the forward's shapes (C ABI calls,
CUDA events on the launching stream).  Also the target of the ncu captures
summarised in profiles/.

    python qwen-image.cu_b200/kernel_bench.py [--which gemm,attn,quant,spectrum,qkv,peaks] [--iters N] [--config c4|c2]
                                              [--gpus 1|2|4|8]

GEMM shapes are those of one CFG-batched C4 forward (M = 2 x 6889 image +
2 x 256 text tokens): fused QKV (N 9216), out-projection (N 3072), fc1
(N 12288), fc2 (K 12288).  Attention: the Sage microbenchmark configuration
(B 2, 24 heads, 4352 tokens) or the C4 joint sequence (7145 tokens).
`--gpus N` times one rank's share of an N-GPU job instead: the CFG halves on
separate ranks (batch 1) and 24 / (N / 2) heads, (6889 + 256) / (N / 2) rows.
Quantizers: LayerNorm-modulate + FWHT-1024 (K 3072), the attention output
(FP16, K 3072) and the MLP hidden (FWHT-4096, K 12288) at the C4 rows.
`spectrum`: a skipped Spectrum step at C4 (prediction from 28 stored states,
then the output head).
`qkv`: the fused QKV projection (q/k RMSNorm + RoPE in the GEMM epilogue)
against the FP32 projection followed by qk_norm_rope, at C4 rows.
`peaks`: the dense tensor-core rates of this GPU through the libraries
(torch._int_mm INT8 -> INT32, torch.matmul FP16 and BF16 at 8192^3), as a
burst (best of 10) and sustained (back to back for 4 s); the roofline
denominators for the INT8 and FP16 kernels.
"""
import time
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import qib200 as Q  # noqa: E402

M_IMG, M_TXT = 2 * 6889, 2 * 256
GEMMS = {"qkv": (9216, 3072), "out": (3072, 3072), "fc1": (12288, 3072), "fc2": (3072, 12288)}


def time_it(fn, iters, warmup=3):
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


def shard(n_gpus):
    """(CFG batch nb, head-parallel degree P) of one rank in an n_gpus job:
    1 GPU runs both CFG halves batched; more split CFG, then heads."""
    return (2, 1) if n_gpus == 1 else (1, n_gpus // 2)


def bench_gemm(iters, res, n_gpus=1):
    nb, P = shard(n_gpus)
    for name, (N, K) in GEMMS.items():
        M = nb * ((M_IMG // 2 + P - 1) // P + (M_TXT // 2 + P - 1) // P)
        a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
        w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda")
        sa = torch.rand(M, device="cuda") * 1e-3
        sw = torch.rand(N, device="cuda") * 1e-3
        b = torch.zeros(N, dtype=torch.bfloat16, device="cuda")
        out = torch.zeros(M, N, device="cuda")
        gate = torch.rand(N, device="cuda") * 1e-3
        # the epilogue each layer runs in the forward: QKV store, out-projection
        # and fc2 the gated residual update, fc1 GELU
        epi = {"qkv": Q.EPI_STORE, "out": Q.EPI_RESIDUAL, "fc1": Q.EPI_GELU, "fc2": Q.EPI_RESIDUAL}[name]
        g = gate if epi == Q.EPI_RESIDUAL else None
        ms = time_it(lambda: Q.linear_i8(a, sa, w, sw, b, epi, gate=g, out=out), iters)
        tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
        res[f"gemm_{name}"] = {"M": M, "N": N, "K": K, "epilogue": ["store", "gelu", "residual"][epi], "ms": round(ms, 4),
                               "tops": round(tf, 1)}
        # cuBLASLt INT8 GEMM on the same operands (INT32 output, no epilogue),
        # for reference: the library's rate on this B200 for this shape
        wt = w.t()
        ms_cb = time_it(lambda: torch._int_mm(a, wt), iters)
        res[f"cublas_int8_{name}"] = {"ms": round(ms_cb, 4), "tops": round(2.0 * M * N * K / (ms_cb * 1e-3) / 1e12, 1)}
        del a, w, out


def bench_attn(iters, res, config, n_gpus=1):
    nb, P = shard(n_gpus)
    S = 4352 if config == "c2" else 7145
    BH = nb * 24 // P
    q = Q.synth((BH, S, 128), 1, 1.0).half()
    k = Q.synth((BH, S, 128), 2, 1.0).half()
    v = Q.synth((BH, S, 128), 3, 1.0).half()
    kmean, qc, qs, kc, ks = Q.sage_quantize(q, k)
    ms_q = time_it(lambda: Q.sage_quantize(q, k), iters)
    ms = time_it(lambda: Q.sage_attention(q, k, v), iters)
    flops = 4.0 * BH * S * S * 128
    res["sage_quant"] = {"BH": BH, "S": S, "ms": round(ms_q, 4)}
    res["attention_incl_quant"] = {"BH": BH, "S": S, "ms": round(ms, 4),
                                   "tflops": round(flops / ((ms - ms_q) * 1e-3) / 1e12, 1)}
    # the FP8 P.V variant (its quantizers included; per-block Q/K, E4M3 V^T)
    ms8 = time_it(lambda: Q.sage_attention_fp8pv(q, k, v), iters)
    res["attention_fp8pv_incl_quant"] = {"BH": BH, "S": S, "ms": round(ms8, 4),
                                         "tflops_incl_quant": round(flops / (ms8 * 1e-3) / 1e12, 1)}


def bench_quant(iters, res):
    M = M_IMG + M_TXT
    for K, B in ((3072, 1024), (12288, 4096)):
        x = Q.synth((M, K), 7, 1.0)
        ms = time_it(lambda: Q.fwht_quantize(x, B), iters)
        gbs = (M * K * 4 + M * K + M * 4) / (ms * 1e-3) / 1e9
        res[f"fwht_quant_{K}"] = {"M": M, "K": K, "ms": round(ms, 4), "gbs": round(gbs, 1)}
    x = Q.synth((M, 3072), 8, 1.0)
    shift = Q.synth((3072,), 9, 0.1)
    scale = Q.synth((3072,), 10, 0.1)
    ms = time_it(lambda: Q.layer_norm_modulate_quantize(x, shift, scale), iters)
    gbs = (M * 3072 * 4 + M * 3072 + M * 4) / (ms * 1e-3) / 1e9
    res["ln_mod_quant_3072"] = {"M": M, "K": 3072, "ms": round(ms, 4), "gbs": round(gbs, 1)}


def bench_spectrum(iters, res, K=28):
    """Spectrum at C4 (one CFG half): prediction from K stored states (a 50-step
    run with 5 warm-up steps and window 2 keeps ~28) and the output head; the
    two together are a skipped step's cost, against a forward for an actual one."""
    n_img, F = 83 * 83, 83 * 83 * 3072
    hidden = Q.synth((n_img, 3072), 41, 1.0)
    sp = Q.Spectrum(F, max_history=50, order=4, lam=0.1)
    for k in range(K):
        sp.update(hidden, 5 + 2 * k)
    out = torch.empty_like(hidden)
    ms_p = time_it(lambda: sp.predict(5 + 2 * K, 1.0, out=out), iters)
    res["spectrum_predict"] = {"K": K, "F": F, "ms": round(ms_p, 4),
                               "gbs": round((K + 1) * F * 4 / (ms_p * 1e-3) / 1e9, 1)}
    ctx = Q.Context(0)
    g, blocks = Q.make_weight_table(1, base_seed=0)
    model = Q.Model(ctx, g, blocks)
    v = torch.empty(1, 16, 166, 166, dtype=torch.bfloat16, device="cuda")
    ms_h = time_it(lambda: Q.spectrum_output(ctx, model, out, 500.0, 166, 166, out=v), iters)
    res["spectrum_output_head"] = {"n_img": n_img, "ms": round(ms_h, 4)}
    sp.close()
    model.close()
    ctx.close()


def bench_qkv(iters, res, n_gpus=1):
    """The block's QKV stage at C4: the fused projection (q/k RMSNorm + RoPE
    + FP16 head-major store in the GEMM epilogue) against the two-launch form
    (FP32 projection, then qk_norm_rope), and the projection alone.  The
    fused launches come first (an ncu capture of the first CTA-pair GEMM
    launches sees them)."""
    nb, P = shard(n_gpus)
    n_img, n_txt = 6889 // P, 256 // P
    rows_i, rows_t = nb * n_img, nb * n_txt

    def stream(rows, tag):
        x = Q.synth((rows, 3072), 50 + len(tag), 1.0)
        w = Q.synth((9216, 3072), 60 + len(tag), 0.02, dtype=torch.bfloat16)
        b = Q.synth((9216,), 70 + len(tag), 0.02, dtype=torch.bfloat16)
        return Q.fwht_quantize(x), Q.quantize_weight(w) + (b,)

    act_i, w_i = stream(rows_i, "img")
    act_t, w_t = stream(rows_t, "tx")
    norms = Q.synth((4, 128), 80, 0.1, 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(Q.rope_table(166, 166, 256)).cuda()
    pe = torch.stack([pe[: n_img + n_txt]] * nb).contiguous()
    ms_f = time_it(lambda: Q.qkv_norm_rope_i8(act_i, act_t, w_i, w_t, norms, pe, nb), iters)
    qi = torch.empty(rows_i, 9216, device="cuda")
    qt = torch.empty(rows_t, 9216, device="cuda")

    def proj():
        Q.linear_i8(act_i[0], act_i[1], w_i[0], w_i[1], w_i[2], out=qi)
        Q.linear_i8(act_t[0], act_t[1], w_t[0], w_t[1], w_t[2], out=qt)

    ms_p = time_it(proj, iters)
    ms_s = time_it(lambda: (proj(), Q.qk_norm_rope(qi, qt, norms, pe, nb)), iters)
    flops = 2.0 * (rows_i + rows_t) * 9216 * 3072
    res["qkv"] = {"rows": rows_i + rows_t, "fused_ms": round(ms_f, 4), "projection_ms": round(ms_p, 4),
                  "two_launch_ms": round(ms_s, 4), "fused_tops": round(flops / (ms_f * 1e-3) / 1e12, 1)}


def bench_peaks(res, seconds=4.0):
    n = 8192
    flops = 2.0 * n ** 3
    a8 = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b8 = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
    ah = torch.randn(n, n, device="cuda").half()
    bh = torch.randn(n, n, device="cuda").half()
    ab, bb = ah.bfloat16(), bh.bfloat16()
    for name, fn in (("int8", lambda: torch._int_mm(a8, b8)), ("fp16", lambda: torch.matmul(ah, bh)),
                     ("bf16", lambda: torch.matmul(ab, bb))):
        best = min(time_it(fn, 1, warmup=3 if k == 0 else 0) for k in range(10))
        fn()
        torch.cuda.synchronize()
        count, t0 = 0, time.time()
        s = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        while time.time() - t0 < seconds:
            for _ in range(20):
                fn()
            count += 20
            torch.cuda.synchronize()
        e1.record(s)
        torch.cuda.synchronize()
        sus = e0.elapsed_time(e1) / count
        res[f"peak_{name}"] = {"n": n, "burst_tflops": round(flops / (best * 1e-3) / 1e12, 1),
                               "sustained_tflops": round(flops / (sus * 1e-3) / 1e12, 1), "iters_sustained": count}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--which", default="gemm,attn,quant")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--config", default="c2")
    ap.add_argument("--gpus", type=int, default=1, choices=(1, 2, 4, 8),
                    help="time one rank's share of an N-GPU job (CFG split, then head-parallel)")
    a = ap.parse_args()
    torch.cuda.set_device(0)
    res = {"gpus": a.gpus}
    w = a.which.split(",")
    if "gemm" in w:
        bench_gemm(a.iters, res, a.gpus)
    if "attn" in w:
        bench_attn(a.iters, res, a.config, a.gpus)
    if "quant" in w:
        bench_quant(a.iters, res)
    if "spectrum" in w:
        bench_spectrum(a.iters, res)
    if "qkv" in w:
        bench_qkv(a.iters, res, a.gpus)
    if "peaks" in w:
        bench_peaks(res)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
