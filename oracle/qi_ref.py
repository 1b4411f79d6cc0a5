"""ctypes binding of oracle/_ref/libqiref.so -- the reference's own CUDA code.

TEST INFRASTRUCTURE ONLY (parity checker and bench.py's reference arm).  The
library is built by oracle/build_ref.sh from the reference sources; it is not
part of the product.  Inputs and outputs are torch CUDA tensors.
"""
import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_ref", "libqiref.so")

_lib = None


def available():
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError(f"{LIB_PATH} missing: run oracle/build_ref.sh where the reference sources exist")
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f, ll, ull = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_ulonglong
        sig = {
            "ref_synth_fill": [vp, ll, ull, f, f, i],
            "ref_quantize_weight": [vp, i, i, vp, vp],
            "ref_fwht_quantize": [vp, i, i, i, vp, vp],
            "ref_linear_int8_preq": [vp, vp, i, i, vp, vp, i, vp, i, vp],
            "ref_linear_int8": [vp, i, i, vp, vp, i, vp, i, vp],
            "ref_sage_quantize": [vp, vp, i, i, vp, vp, vp, vp, vp],
            "ref_sage_attention": [vp, vp, vp, vp, f, i, i],
            "ref_layer_norm_modulate": [vp, vp, vp, vp, i, i, f],
            "ref_rms_norm_fp32": [vp, vp, vp, i, i, f],
            "ref_rope_table": [i, i, i, vp],
            "ref_rope_fp16": [vp, vp, vp, i, i],
            "ref_gate_add": [vp, vp, vp, vp, i, i],
            "ref_load_all": [ctypes.c_char_p, vp],
            "ref_transformer_forward": [vp, vp, vp, f, vp, i, vp, i, i, i, vp],
            "ref_transformer_forward_capture": [vp, vp, vp, f, vp, i, vp, i, i, i, vp, vp],
            "ref_transformer_spectrum_output": [vp, vp, vp, f, i, i, vp],
            "ref_spectrum_predict": [vp, vp, i, ll, i, f, i, f, vp],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = i
        _lib = L
    return _lib


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _ok(st):
    if st != 0:
        raise RuntimeError(f"reference call failed with status {st}")


def synth(shape, seed, scale=1.0, offset=0.0, dtype=torch.float32):
    t = torch.empty(shape, dtype=dtype, device="cuda")
    _ok(lib().ref_synth_fill(_p(t), t.numel(), seed, scale, offset, int(dtype == torch.bfloat16)))
    return t


def quantize_weight(w_bf16):
    N, K = w_bf16.shape
    codes = torch.empty(N, K, dtype=torch.int8, device="cuda")
    scales = torch.empty(N, dtype=torch.float32, device="cuda")
    _ok(lib().ref_quantize_weight(_p(w_bf16), N, K, _p(codes), _p(scales)))
    return codes, scales


def fwht_quantize(x, had_block=None):
    M, K = x.shape
    if had_block is None:
        had_block = K & (-K)
    codes = torch.empty(M, K, dtype=torch.int8, device="cuda")
    scales = torch.empty(M, dtype=torch.float32, device="cuda")
    _ok(lib().ref_fwht_quantize(_p(x), M, K, had_block, _p(codes), _p(scales)))
    return codes, scales


def linear_int8_preq(a, sa, w, sw, bias=None, gelu=False):
    M, K = a.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    _ok(lib().ref_linear_int8_preq(_p(a), _p(sa), M, K, _p(w), _p(sw), N, _p(bias), int(gelu), _p(out)))
    return out


def linear_int8(x, w, sw, bias=None, gelu=False):
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    _ok(lib().ref_linear_int8(_p(x), M, K, _p(w), _p(sw), N, _p(bias), int(gelu), _p(out)))
    return out


def sage_quantize(q, k):
    BH, S, _ = q.shape
    kmean = torch.empty(BH, 128, dtype=torch.float32, device="cuda")
    qc = torch.empty(BH, S, 128, dtype=torch.int8, device="cuda")
    kc = torch.empty(BH, S, 128, dtype=torch.int8, device="cuda")
    qs = torch.empty(BH, ((S + 127) // 128) * 32, dtype=torch.float32, device="cuda")
    ks = torch.empty(BH, ((S + 63) // 64) * 4, dtype=torch.float32, device="cuda")
    _ok(lib().ref_sage_quantize(_p(q), _p(k), BH, S, _p(kmean), _p(qc), _p(qs), _p(kc), _p(ks)))
    return kmean, qc, qs, kc, ks


def sage_attention(q, k, v, scale):
    BH, S, _ = q.shape
    out = torch.empty(BH, S, 128, dtype=torch.float32, device="cuda")
    _ok(lib().ref_sage_attention(_p(q), _p(k), _p(v), _p(out), float(scale), BH, S))
    return out


def layer_norm_modulate(x, shift, scale, eps=1e-6):
    out = torch.empty_like(x)
    _ok(lib().ref_layer_norm_modulate(_p(x), _p(shift), _p(scale), _p(out), x.shape[0], x.shape[1], eps))
    return out


def rms_norm(x, w, eps=1e-6):
    out = torch.empty_like(x)
    _ok(lib().ref_rms_norm_fp32(_p(x), _p(w), _p(out), x.shape[0], x.shape[1], eps))
    return out


def rope_fp16(x, pe):
    """x: head-major [H, L, 128] FP32, pe [L, 64, 2, 2] -> FP16 [H, L, 128]."""
    H, L, _ = x.shape
    out = torch.empty(H, L, 128, dtype=torch.float16, device="cuda")
    _ok(lib().ref_rope_fp16(_p(x), _p(pe), _p(out), H, L))
    return out


def gate_add(inp, gate, x):
    out = torch.empty_like(inp)
    _ok(lib().ref_gate_add(_p(inp), _p(gate), _p(x), _p(out), inp.shape[0], inp.shape[1]))
    return out


def load_all(path):
    """The reference's per-tensor upload of every tensor in a safetensors
    checkpoint (each freed after upload); returns the bytes uploaded."""
    n = ctypes.c_longlong(0)
    _ok(lib().ref_load_all(path.encode(), ctypes.byref(n)))
    return n.value


def rope_table(h, w, n_txt):
    import numpy as np
    n = n_txt + ((h + 1) // 2) * ((w + 1) // 2)
    pe = np.empty((n, 64, 2, 2), dtype=np.float32)
    _ok(lib().ref_rope_table(h, w, n_txt, pe.ctypes.data_as(ctypes.c_void_p)))
    return pe


def transformer_forward(garr, bt, x, t, txt, pe, H, W, sage=True):
    """garr/bt: ctypes pointer arrays from qib200.table_pointers (60 blocks).
    x: [1,16,H,W] bf16, txt: [1,n_txt,3584] bf16, pe: [S,64,2,2] f32 (device)."""
    out = torch.empty_like(x)
    _ok(lib().ref_transformer_forward(garr, bt, _p(x), float(t), _p(txt), txt.shape[-2], _p(pe), H, W, int(sage),
                                      _p(out)))
    return out


def transformer_forward_capture(garr, bt, x, t, txt, pe, H, W, sage=True):
    """transformer_forward with spectrum_hidden_out: (output, final image hidden state [n_img, 3072])."""
    out = torch.empty_like(x)
    hidden = torch.empty((H // 2) * (W // 2), 3072, dtype=torch.float32, device=x.device)
    _ok(lib().ref_transformer_forward_capture(garr, bt, _p(x), float(t), _p(txt), txt.shape[-2], _p(pe), H, W,
                                              int(sage), _p(out), _p(hidden)))
    return out, hidden


def transformer_spectrum_output(garr, bt, hidden, t, H, W):
    out = torch.empty(1, 16, H, W, dtype=torch.bfloat16, device=hidden.device)
    _ok(lib().ref_transformer_spectrum_output(garr, bt, _p(hidden), float(t), H, W, _p(out)))
    return out


def spectrum_predict(hist, steps, target, blend=1.0, order=4, lam=0.1):
    """The reference's SpectrumState over hist [K, F] (device FP32) stored at `steps`."""
    K, F = hist.shape
    st = (ctypes.c_int * K)(*[int(v) for v in steps])
    out = torch.empty(F, dtype=torch.float32, device=hist.device)
    _ok(lib().ref_spectrum_predict(_p(hist), st, K, F, int(order), float(lam), int(target), float(blend), _p(out)))
    return out


# ----------------------------------------------------------------- weight table
# Tensor names and shapes of the quantize.cu INT8 format (transformer.h:407-563),
# in the table order of the product's public header.
DIM, MLP, TXT_DIM, PATCH_DIM = 3072, 12288, 3584, 64
G_NAMES = [
    ("time_text_embed.timestep_embedder.linear_1.weight", "w", (DIM, 256)),
    ("time_text_embed.timestep_embedder.linear_1.weight.__scales__", "s", None),
    ("time_text_embed.timestep_embedder.linear_1.bias", "b", (DIM,)),
    ("time_text_embed.timestep_embedder.linear_2.weight", "w", (DIM, DIM)),
    ("time_text_embed.timestep_embedder.linear_2.weight.__scales__", "s", None),
    ("time_text_embed.timestep_embedder.linear_2.bias", "b", (DIM,)),
    ("txt_norm.weight", "n", (TXT_DIM,)),
    ("img_in.weight", "bw", (DIM, PATCH_DIM)), ("img_in.bias", "b", (DIM,)),
    ("txt_in.weight", "bw", (DIM, TXT_DIM)), ("txt_in.bias", "b", (DIM,)),
    ("norm_out.linear.weight", "bw", (2 * DIM, DIM)), ("norm_out.linear.bias", "b", (2 * DIM,)),
    ("proj_out.weight", "bw", (PATCH_DIM, DIM)), ("proj_out.bias", "b", (PATCH_DIM,)),
]
L_NAMES = [
    ("img_mod.1", 6 * DIM, DIM), ("txt_mod.1", 6 * DIM, DIM),
    ("attn.to_q", DIM, DIM), ("attn.to_k", DIM, DIM), ("attn.to_v", DIM, DIM),
    ("attn.add_q_proj", DIM, DIM), ("attn.add_k_proj", DIM, DIM), ("attn.add_v_proj", DIM, DIM),
    ("attn.to_out.0", DIM, DIM), ("attn.to_add_out", DIM, DIM),
    ("img_mlp.net.0.proj", MLP, DIM), ("img_mlp.net.2", DIM, MLP),
    ("txt_mlp.net.0.proj", MLP, DIM), ("txt_mlp.net.2", DIM, MLP),
]
B_NORMS = ["attn.norm_q.weight", "attn.norm_k.weight", "attn.norm_added_q.weight", "attn.norm_added_k.weight"]


def seed_for(base, name):
    """FNV-1a of the name mixed into the base seed (same as the product's
    qi_seed_for and the CPU oracle's or_seed_for)."""
    h = 0xCBF29CE484222325
    for ch in name.encode():
        h ^= ch
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    x = (base ^ h) & 0xFFFFFFFFFFFFFFFF
    x = (x + 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & 0xFFFFFFFFFFFFFFFF
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & 0xFFFFFFFFFFFFFFFF
    return x ^ (x >> 31)


def make_table(num_blocks=60, distinct=1, base_seed=0, wscale=0.02):
    """Seeded synthetic weights built with reference code only (the harness's
    generator and quantize_weight_tensor).  Block i uses the tensors of block
    i % distinct.  Returns (global_list, block_lists) of device tensors."""
    g, scales_next = [], None
    for name, kind, shape in G_NAMES:
        if kind == "w":
            c, scales_next = quantize_weight(synth(shape, seed_for(base_seed, name), wscale, dtype=torch.bfloat16))
            g.append(c)
        elif kind == "s":
            g.append(scales_next)
        elif kind == "n":
            g.append(synth(shape, seed_for(base_seed, name), wscale, 1.0, dtype=torch.bfloat16))
        else:
            g.append(synth(shape, seed_for(base_seed, name), wscale, dtype=torch.bfloat16))
    blocks = []
    for i in range(distinct):
        pre = f"transformer_blocks.{i}."
        tl = []
        for lname, N, K in L_NAMES:
            c, s = quantize_weight(synth((N, K), seed_for(base_seed, pre + lname + ".weight"), wscale,
                                         dtype=torch.bfloat16))
            tl += [c, s, synth((N,), seed_for(base_seed, pre + lname + ".bias"), wscale, dtype=torch.bfloat16)]
        for nname in B_NORMS:
            tl.append(synth((128,), seed_for(base_seed, pre + nname), wscale, 1.0, dtype=torch.bfloat16))
        blocks.append(tl)
    return g, [blocks[i % distinct] for i in range(num_blocks)]


def table_pointers(g, block_lists):
    garr = (ctypes.c_void_p * len(g))(*[t.data_ptr() for t in g])
    barrs = [(ctypes.c_void_p * len(b))(*[t.data_ptr() for t in b]) for b in block_lists]
    bt = (ctypes.c_void_p * len(barrs))(*[ctypes.cast(a, ctypes.c_void_p) for a in barrs])
    return garr, barrs, bt
