"""Generates the golden fixtures in tests/golden/ from the reference itself.

Runs on a CUDA box with oracle/_ref/libqiref.so (the reference's own CUDA code
built by oracle/build_ref.sh).  Every input is produced by the seeded
generator (oracle/qi_synth.c restates it; the reference harness has its own
device copy), so fixtures only store outputs; the CPU tests regenerate the
inputs and check the CPU oracle against the reference's outputs.

    python tests/golden/make_golden.py [out_dir]

Fixtures:
  quant_act.npz     fwht_quantize_fp32 codes/scales (cuda_kernels.cu:2493)
  quant_weight.npz  quantize_weight_tensor codes/scales (cuda_kernels.cu:2830)
  sage.npz          Sage quantizers + attention output (sageattention_sm80.cu)
  rope.npz          gen_qwen_image_pe digests + one small table (rope.h:175)
  block0.npz        transformer_forward block-0 stage dumps at a tiny size
                    (the reference's DUMP_TRANSFORMER hooks, transformer.cu:352)
  spectrum.npz      spectrum_predict on seeded histories (cuda_kernels.cu:6268)

    python tests/golden/make_golden.py [out_dir] --only spectrum   (one fixture)
"""
import glob
import hashlib
import os
import sys
import tempfile

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import qi_ref as R  # noqa: E402

# Spectrum: (K, F, steps, target, order, lambda, blend); histories R.synth((K, F), seed).  Order
# 4 only: the reference's spectrum_init never stores its max_order argument
# (cuda_kernels.cu:6168-6196), so its fit always uses T_0..T_4 (SpectrumState's default), and
# below 4 its buffers are a column short of what spectrum_predict writes.
SPECTRUM_CASES = [
    (2, 4096, [5, 6], 7, 4, 0.1, 1.0),
    (6, 4096, [5, 7, 9, 11, 13, 15], 16, 4, 0.1, 1.0),
    (12, 4096, [0, 1, 2, 3, 4, 5, 7, 9, 11, 13, 15, 17], 18, 4, 0.1, 0.5),
    (20, 4096, list(range(5, 45, 2)), 46, 4, 0.01, 0.75),
    (8, 4096, [10, 12, 14, 16, 18, 20, 22, 24], 23, 4, 1.0, 0.0),
]
ACT_CASES = [(8, 3072, 1024), (4, 12288, 4096), (3, 256, 256), (5, 3584, 512)]
W_CASES = [(16, 3072), (8, 12288), (16, 256), (4, 64), (4, 3584)]
SAGE_CASES = [(2, 200), (1, 77), (2, 384)]
ROPE_CASES = [(8, 8, 8), (128, 128, 256), (166, 166, 256), (256, 256, 512), (7, 9, 5), (64, 64, 64)]
# Block-0 dumps at 64x64 latent / 64 text tokens (S = 1088).  At sequences shorter than one
# 64-key block (e.g. 8x8 latent, 8 text tokens: S = 24) the reference's sm80 Sage kernel
# returns NaN (masked keys multiply stale shared memory), so tiny sizes cannot pin anything
# past attention.  Only a fixed subsample of rows is stored.
TINY = dict(H=64, W=64, n_txt=64, t=500.0)
ROWS_IMG = [0, 1, 63, 64, 127, 200, 333, 511, 512, 700, 777, 901, 1000, 1022, 1023, 640]
ROWS_TXT = [0, 1, 7, 8, 31, 32, 62, 63]


def act_input(M, K, seed):
    x = R.synth((M, K), seed, 1.0)
    x[0] = 0.0            # an all-zero row (scale 0, codes 0)
    if M > 1:
        x[1, 7] *= 1000.0  # an outlier row
    return x


def spectrum(out):
    d = {}
    for i, (K, F, steps, target, order, lam, blend) in enumerate(SPECTRUM_CASES):
        hist = R.synth((K, F), R.seed_for(31, f"spectrum_{i}"), 1.0)
        d[f"pred_{i}"] = R.spectrum_predict(hist, steps, target, blend, order, lam).cpu().numpy()
    np.savez_compressed(os.path.join(out, "spectrum.npz"), **d)


def main(out):
    os.makedirs(out, exist_ok=True)
    torch.cuda.set_device(0)
    if "--only" in sys.argv and sys.argv[sys.argv.index("--only") + 1] == "spectrum":
        spectrum(out)
        print("wrote spectrum.npz")
        return
    # --- activation quantizer
    d = {}
    for M, K, B in ACT_CASES:
        x = act_input(M, K, R.seed_for(11, f"act_{M}_{K}"))
        c, s = R.fwht_quantize(x, B)
        d[f"codes_{M}_{K}"] = c.cpu().numpy()
        d[f"scales_{M}_{K}"] = s.cpu().numpy()
    np.savez_compressed(os.path.join(out, "quant_act.npz"), **d)
    # --- weight quantizer
    d = {}
    for N, K in W_CASES:
        w = R.synth((N, K), R.seed_for(12, f"w_{N}_{K}"), 0.02, dtype=torch.bfloat16)
        c, s = R.quantize_weight(w)
        d[f"codes_{N}_{K}"] = c.cpu().numpy()
        d[f"scales_{N}_{K}"] = s.cpu().numpy()
    np.savez_compressed(os.path.join(out, "quant_weight.npz"), **d)
    # --- Sage
    d = {}
    for BH, S in SAGE_CASES:
        q = R.synth((BH, S, 128), R.seed_for(13, f"q_{BH}_{S}"), 1.0).half()
        k = R.synth((BH, S, 128), R.seed_for(13, f"k_{BH}_{S}"), 1.0).half()
        v = R.synth((BH, S, 128), R.seed_for(13, f"v_{BH}_{S}"), 1.0).half()
        km, qc, qs, kc, ks = R.sage_quantize(q, k)
        o = R.sage_attention(q, k, v, 1.0 / np.sqrt(128.0))
        for name, t in (("kmean", km), ("qc", qc), ("qs", qs), ("kc", kc), ("ks", ks)):
            d[f"{name}_{BH}_{S}"] = t.cpu().numpy()
        d[f"out_{BH}_{S}"] = o.cpu().numpy().astype(np.float16)
    np.savez_compressed(os.path.join(out, "sage.npz"), **d)
    # --- RoPE table
    d = {}
    for h, w, n in ROPE_CASES:
        pe = R.rope_table(h, w, n)
        d[f"sha256_{h}_{w}_{n}"] = np.frombuffer(hashlib.sha256(pe.tobytes()).digest(), dtype=np.uint8)
    d["table_8_8_8"] = R.rope_table(8, 8, 8)
    np.savez_compressed(os.path.join(out, "rope.npz"), **d)
    # --- block 0 stage dumps through the reference's transformer_forward
    g, blocks = R.make_table(60, distinct=1)
    garr, barrs, bt = R.table_pointers(g, blocks)
    H, W, n_txt, t = TINY["H"], TINY["W"], TINY["n_txt"], TINY["t"]
    x = R.synth((1, 16, H, W), R.seed_for(1, "latent"), 1.0, dtype=torch.bfloat16)
    txt = R.synth((1, n_txt, 3584), R.seed_for(1, "context"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(R.rope_table(H, W, n_txt)).cuda()
    cwd = os.getcwd()
    with tempfile.TemporaryDirectory() as tmp:
        os.chdir(tmp)
        os.environ["DUMP_TRANSFORMER"] = "1"
        os.environ["DUMP_TRANSFORMER_ACTIVE"] = "1"
        y = R.transformer_forward(garr, bt, x, t, txt, pe, H, W, sage=True)
        for k in ("DUMP_TRANSFORMER", "DUMP_TRANSFORMER_ACTIVE"):
            os.environ.pop(k, None)
        d = {"out": y.float().cpu().numpy()}
        for f in sorted(glob.glob("cuda_*.bin")):
            a = np.fromfile(f, dtype=np.float32)
            key = os.path.basename(f)[5:]
            while key.endswith(".bin"):  # block stems already end in .bin (transformer.cu:503)
                key = key[:-4]
            keep32 = a.size <= 20000
            d[key] = a if keep32 else a.astype(np.float16)
        os.chdir(cwd)
    # keep only the stages the tests read (the forward dumps every 10 blocks too)
    wanted = {"out", "t_emb", "img_after_proj", "txt_after_proj", "b0_img_mods", "b0_txt_mods",
              "b0_img_modulated", "b0_img_q_normed", "b0_attn_out_img", "b0_attn_out_txt",
              "b0_img_after_attn", "b0_img_after_mlp", "b0_txt_after_mlp"}
    d = {k: v for k, v in d.items() if k in wanted}
    n_img = (H // 2) * (W // 2)
    for k in list(d):
        a = d[k]
        if k == "out":
            continue
        if a.size == n_img * 3072:
            d[k] = a.reshape(n_img, 3072)[ROWS_IMG]
        elif a.size == n_txt * 3072:
            d[k] = a.reshape(n_txt, 3072)[ROWS_TXT]
    d["rows_img"] = np.array(ROWS_IMG)
    d["rows_txt"] = np.array(ROWS_TXT)
    np.savez_compressed(os.path.join(out, "block0.npz"), **d)
    spectrum(out)
    print("wrote", sorted(os.listdir(out)))


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--") and a != "spectrum"]
    main(args[0] if args else os.path.dirname(os.path.abspath(__file__)))
