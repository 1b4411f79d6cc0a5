"""ctypes binding of libqib200.so (include/qwen_image_b200.h) for tests and bench.

The product is the C ABI; this module only forwards torch device pointers to
it.  Every call raises QIError on a non-zero status.  There is no fallback:
if the shared library is missing, importing works but the first call raises.
"""
import ctypes
import os

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libqib200.so")
HEADER = os.path.join(os.path.dirname(_HERE), "include", "qwen_image_b200.h")

# Model constants (transformer.cu:244-250 of the reference).
DIM, HEADS, HEAD_DIM, MLP, TXT_DIM, PATCH_DIM, OUT_CH = 3072, 24, 128, 12288, 3584, 64, 16

# Weight-table indices (mirror the enums of the header).
G_NAMES = [
    ("time_text_embed.timestep_embedder.linear_1.weight", "w"),
    ("time_text_embed.timestep_embedder.linear_1.weight.__scales__", "s"),
    ("time_text_embed.timestep_embedder.linear_1.bias", "b"),
    ("time_text_embed.timestep_embedder.linear_2.weight", "w"),
    ("time_text_embed.timestep_embedder.linear_2.weight.__scales__", "s"),
    ("time_text_embed.timestep_embedder.linear_2.bias", "b"),
    ("txt_norm.weight", "n"),
    ("img_in.weight", "bw"), ("img_in.bias", "b"),
    ("txt_in.weight", "bw"), ("txt_in.bias", "b"),
    ("norm_out.linear.weight", "bw"), ("norm_out.linear.bias", "b"),
    ("proj_out.weight", "bw"), ("proj_out.bias", "b"),
]
G_SHAPES = {
    "time_text_embed.timestep_embedder.linear_1.weight": (DIM, 256),
    "time_text_embed.timestep_embedder.linear_2.weight": (DIM, DIM),
    "txt_norm.weight": (TXT_DIM,),
    "img_in.weight": (DIM, PATCH_DIM),
    "txt_in.weight": (DIM, TXT_DIM),
    "norm_out.linear.weight": (2 * DIM, DIM),
    "proj_out.weight": (PATCH_DIM, DIM),
}
# Per-block INT8 linears in table order (transformer.h:515-563 names).
L_NAMES = [
    ("img_mod.1", 6 * DIM, DIM), ("txt_mod.1", 6 * DIM, DIM),
    ("attn.to_q", DIM, DIM), ("attn.to_k", DIM, DIM), ("attn.to_v", DIM, DIM),
    ("attn.add_q_proj", DIM, DIM), ("attn.add_k_proj", DIM, DIM), ("attn.add_v_proj", DIM, DIM),
    ("attn.to_out.0", DIM, DIM), ("attn.to_add_out", DIM, DIM),
    ("img_mlp.net.0.proj", MLP, DIM), ("img_mlp.net.2", DIM, MLP),
    ("txt_mlp.net.0.proj", MLP, DIM), ("txt_mlp.net.2", DIM, MLP),
]
B_NORMS = ["attn.norm_q.weight", "attn.norm_k.weight", "attn.norm_added_q.weight", "attn.norm_added_k.weight"]
B_COUNT = 3 * len(L_NAMES) + 4

EPI_STORE, EPI_GELU, EPI_RESIDUAL = 0, 1, 2


class QIError(RuntimeError):
    pass


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise QIError(f"{LIB_PATH} is missing: build it with `make -C qwen-image.cu_b200`")
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f, ll, ull = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_ulonglong
        sig = {
            "qi_status_string": ([i], ctypes.c_char_p),
            "qi_version": ([], i),
            "qi_quantize_weight": ([vp, i, i, vp, vp, vp], i),
            "qi_fwht_quantize": ([vp, i, i, i, vp, vp, vp], i),
            "qi_linear_i8": ([vp, vp, i, i, vp, vp, i, vp, i, vp, vp, i, vp], i),
            "qi_linear_i8_f32in": ([vp, i, i, vp, vp, i, vp, i, vp, vp], i),
            "qi_linear_i8_f32in_noalloc": ([vp, i, i, vp, vp, i, vp, i, vp, vp], i),
            "qi_linear_i8_f32in_noalloc_check": ([], i),
            "qi_linear_i8_f32in_noalloc_selftest": ([i, vp], i),
            "qi_alloc_count": ([], ll),
            "qi_sage_attention": ([vp, vp, vp, vp, f, i, i, i, vp], i),
            "qi_sage_attention_fp8pv": ([vp, vp, vp, vp, f, i, i, i, vp], i),
            "qi_sage_quantize": ([vp, vp, i, i, vp, vp, vp, vp, vp, vp], i),
            "qi_layer_norm_modulate": ([vp, vp, vp, vp, i, i, f, vp], i),
            "qi_rms_norm": ([vp, vp, vp, i, i, f, vp], i),
            "qi_layer_norm_modulate_quantize": ([vp, vp, vp, i, i, f, vp, vp, vp], i),
            "qi_qk_norm_rope": ([vp, vp, vp, vp, i, i, i, vp, vp], i),
            "qi_qkv_norm_rope_i8": ([vp] * 12 + [i, i, i, vp, vp], i),
            "qi_ctx_create": ([i, ctypes.POINTER(vp)], i),
            "qi_ctx_destroy": ([vp], i),
            "qi_ctx_check": ([vp], i),
            "qi_ctx_last_launch_count": ([vp], i),
            "qi_model_create": ([vp, i, vp, vp, ctypes.POINTER(vp)], i),
            "qi_model_load_safetensors": ([vp, ctypes.c_char_p, ctypes.POINTER(vp)], i),
            "qi_model_destroy": ([vp], i),
            "qi_model_num_blocks": ([vp], i),
            "qi_forward": ([vp, vp, i, vp, f, vp, i, vp, i, i, vp, vp], i),
            "qi_forward_blocks": ([vp, vp, i, i, i, vp, vp, f, vp, i, i, vp], i),
            "qi_cfg_euler_step": ([vp, vp, vp, f, f, f, i, i, vp, vp], i),
            "qi_ctx_set_profiling": ([vp, i], i),
            "qi_selftest_wait_timeout": ([vp, i, vp], i),
            "qi_ctx_profile": ([vp, vp, vp, i], i),
            "qi_comm_unique_id": ([vp], i),
            "qi_ctx_set_comm": ([vp, vp, i, i], i),
            "qi_ctx_set_comm_timeout": ([vp, i], i),
            "qi_ctx_set_attention_fp8pv": ([vp, i], i),
            "qi_ctx_set_fused_qkv_epilogue": ([vp, i], i),
            "qi_ctx_sync": ([vp, vp, i], i),
            "qi_exchange_plan": ([i, i, i, i, i, i, vp, vp, vp, vp], i),
            "qi_rope_table": ([i, i, i, vp], i),
            "qi_synth_fill": ([vp, ll, ull, f, f, i, vp], i),
            "qi_ctx_set_hidden_capture": ([vp, vp], i),
            "qi_spectrum_output": ([vp, vp, i, vp, f, i, i, vp, vp], i),
            "qi_spectrum_create": ([ll, i, i, f, ctypes.POINTER(vp)], i),
            "qi_spectrum_destroy": ([vp], i),
            "qi_spectrum_update": ([vp, vp, i, vp], i),
            "qi_spectrum_predict": ([vp, i, f, vp, vp], i),
            "qi_spectrum_history": ([vp], i),
            "qi_spectrum_reset": ([vp], i),
            "qi_spectrum_weights": ([vp, i, i, f, i, f, vp], i),
            "qi_seed_for": ([ull, ctypes.c_char_p], ull),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(st):
    if st != 0:
        raise QIError(f"status {st}: {lib().qi_status_string(st).decode()}")


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


# ----------------------------------------------------------------- op level
def quantize_weight(w_bf16):
    N, K = w_bf16.shape
    codes = torch.empty(N, K, dtype=torch.int8, device=w_bf16.device)
    scales = torch.empty(N, dtype=torch.float32, device=w_bf16.device)
    check(lib().qi_quantize_weight(_p(w_bf16), N, K, _p(codes), _p(scales), _stream()))
    return codes, scales


def fwht_quantize(x, had_block=None):
    M, K = x.shape
    if had_block is None:
        had_block = K & (-K)
    codes = torch.empty(M, K, dtype=torch.int8, device=x.device)
    scales = torch.empty(M, dtype=torch.float32, device=x.device)
    check(lib().qi_fwht_quantize(_p(x), M, K, had_block, _p(codes), _p(scales), _stream()))
    return codes, scales


def linear_i8(act, act_scales, w, w_scales, bias=None, epilogue=EPI_STORE, gate=None, out=None):
    M, K = act.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=torch.float32, device=act.device)
    check(lib().qi_linear_i8(_p(act), _p(act_scales), M, K, _p(w), _p(w_scales), N, _p(bias), epilogue, _p(gate),
                             _p(out), out.stride(0), _stream()))
    return out


def linear_i8_f32in(x, w, w_scales, bias=None, gelu=False):
    M, K = x.shape
    N = w.shape[0]
    out = torch.empty(M, N, dtype=torch.float32, device=x.device)
    check(lib().qi_linear_i8_f32in(_p(x), M, K, _p(w), _p(w_scales), N, _p(bias), int(gelu), _p(out), _stream()))
    return out


def sage_quantize(q, k):
    BH, S, D = q.shape
    dev = q.device
    kmean = torch.empty(BH, 128, dtype=torch.float32, device=dev)
    qc = torch.empty(BH, S, 128, dtype=torch.int8, device=dev)
    kc = torch.empty(BH, S, 128, dtype=torch.int8, device=dev)
    qs = torch.empty(BH, ((S + 127) // 128) * 32, dtype=torch.float32, device=dev)
    ks = torch.empty(BH, ((S + 63) // 64) * 4, dtype=torch.float32, device=dev)
    check(lib().qi_sage_quantize(_p(q), _p(k), BH, S, _p(kmean), _p(qc), _p(qs), _p(kc), _p(ks), _stream()))
    return kmean, qc, qs, kc, ks


def sage_attention(q, k, v, scale=1.0 / np.sqrt(128.0)):
    BH, S, D = q.shape
    out = torch.empty(BH, S, D, dtype=torch.float32, device=q.device)
    check(lib().qi_sage_attention(_p(q), _p(k), _p(v), _p(out), float(scale), BH, S, D, _stream()))
    return out


def sage_attention_fp8pv(q, k, v, scale=1.0 / np.sqrt(128.0)):
    BH, S, D = q.shape
    out = torch.empty(BH, S, D, dtype=torch.float32, device=q.device)
    check(lib().qi_sage_attention_fp8pv(_p(q), _p(k), _p(v), _p(out), float(scale), BH, S, D, _stream()))
    return out


def layer_norm_modulate(x, shift, scale, eps=1e-6):
    rows, dim = x.shape
    out = torch.empty_like(x)
    check(lib().qi_layer_norm_modulate(_p(x), _p(shift), _p(scale), _p(out), rows, dim, eps, _stream()))
    return out


def rms_norm(x, w, eps=1e-6):
    rows, dim = x.shape
    out = torch.empty_like(x)
    check(lib().qi_rms_norm(_p(x), _p(w), _p(out), rows, dim, eps, _stream()))
    return out


def layer_norm_modulate_quantize(x, shift, scale, eps=1e-6):
    rows, dim = x.shape
    codes = torch.empty(rows, dim, dtype=torch.int8, device=x.device)
    scales = torch.empty(rows, dtype=torch.float32, device=x.device)
    check(lib().qi_layer_norm_modulate_quantize(_p(x), _p(shift), _p(scale), rows, dim, eps, _p(codes), _p(scales),
                                                _stream()))
    return codes, scales


def qk_norm_rope(qkv_img, qkv_txt, norms, pe, nb=1):
    """qkv_img [nb*n_img, 9216], qkv_txt [nb*n_txt, 9216] FP32; norms [4,128]
    BF16; pe nb x [S,64,2,2].  Returns FP16 [3, nb*24, S, 128] (q, k, v)."""
    n_img = qkv_img.shape[0] // nb
    n_txt = qkv_txt.shape[0] // nb
    out = torch.empty(3, nb * HEADS, n_img + n_txt, HEAD_DIM, dtype=torch.float16, device=qkv_img.device)
    check(lib().qi_qk_norm_rope(_p(qkv_img), _p(qkv_txt), _p(norms), _p(pe), nb, n_img, n_txt, _p(out), _stream()))
    return out


def qkv_norm_rope_i8(act_img, act_txt, w_img, w_txt, norms, pe, nb=1):
    """The fused QKV projection: act_* = (codes [nb*n, 3072] INT8, scales
    [nb*n]); w_* = (codes [9216, 3072], scales [9216], BF16 bias or None).
    Returns FP16 [3, nb*24, S, 128] (q, k, v), the bits of linear_i8 +
    qk_norm_rope."""
    n_img = act_img[0].shape[0] // nb
    n_txt = act_txt[0].shape[0] // nb
    out = torch.empty(3, nb * HEADS, n_img + n_txt, HEAD_DIM, dtype=torch.float16, device=act_img[0].device)
    bi = _p(w_img[2]) if w_img[2] is not None else None
    bt = _p(w_txt[2]) if w_txt[2] is not None else None
    check(lib().qi_qkv_norm_rope_i8(_p(act_img[0]), _p(act_img[1]), _p(act_txt[0]), _p(act_txt[1]), _p(w_img[0]),
                                    _p(w_img[1]), bi, _p(w_txt[0]), _p(w_txt[1]), bt, _p(norms), _p(pe), nb, n_img,
                                    n_txt, _p(out), _stream()))
    return out


def rope_table(h, w, n_txt):
    n = n_txt + ((h + 1) // 2) * ((w + 1) // 2)
    pe = np.empty((n, 64, 2, 2), dtype=np.float32)
    check(lib().qi_rope_table(h, w, n_txt, pe.ctypes.data_as(ctypes.c_void_p)))
    return pe


# ----------------------------------------------------------------- synthetic data
def seed_for(base, name):
    return lib().qi_seed_for(base, name.encode())


def synth(shape, seed, scale=1.0, offset=0.0, dtype=torch.float32, device="cuda"):
    t = torch.empty(shape, dtype=dtype, device=device)
    assert dtype in (torch.float32, torch.bfloat16)
    check(lib().qi_synth_fill(_p(t), t.numel(), seed, float(scale), float(offset), int(dtype == torch.bfloat16),
                              _stream()))
    return t


def make_weight_table(num_blocks, base_seed=0, distinct_blocks=None, device="cuda", wscale=0.02):
    """Synthetic weights in quantize.cu's format (INT8 codes + scales for the
    quantized linears, BF16 for the boundary layers), generated on the device
    from seeded N(0, wscale^2) BF16 weights and quantized with the product's
    bit-exact weight quantizer.  Returns (global_list, block_lists) of device
    tensors in header table order.  With distinct_blocks = d, block i reuses the
    tensors of block i % d (the reference loops over 60 blocks; tests repeat a
    few to keep memory small)."""
    d = num_blocks if distinct_blocks is None else distinct_blocks
    g = []
    for name, kind in G_NAMES:
        if kind == "w":
            shp = G_SHAPES[name]
            wb = synth(shp, seed_for(base_seed, name), wscale, dtype=torch.bfloat16, device=device)
            codes, scales = quantize_weight(wb)
            del wb
            g.append(codes)
        elif kind == "s":
            g.append(scales)
        elif kind == "bw":
            g.append(synth(G_SHAPES[name], seed_for(base_seed, name), wscale, dtype=torch.bfloat16, device=device))
        elif kind == "n":
            g.append(synth(G_SHAPES[name], seed_for(base_seed, name), wscale, 1.0, dtype=torch.bfloat16, device=device))
        else:  # bias: size of the preceding weight's first dim
            wname = name.rsplit(".", 1)[0] + ".weight"
            n = G_SHAPES[wname][0]
            g.append(synth((n,), seed_for(base_seed, name), wscale, dtype=torch.bfloat16, device=device))
    blocks = []
    for i in range(d):
        pre = f"transformer_blocks.{i}."
        t = []
        for lname, N, K in L_NAMES:
            wb = synth((N, K), seed_for(base_seed, pre + lname + ".weight"), wscale, dtype=torch.bfloat16,
                       device=device)
            codes, scales = quantize_weight(wb)
            del wb
            bias = synth((N,), seed_for(base_seed, pre + lname + ".bias"), wscale, dtype=torch.bfloat16,
                         device=device)
            t += [codes, scales, bias]
        for nname in B_NORMS:
            t.append(synth((HEAD_DIM,), seed_for(base_seed, pre + nname), wscale, 1.0, dtype=torch.bfloat16,
                           device=device))
        blocks.append(t)
    block_lists = [blocks[i % d] for i in range(num_blocks)]
    return g, block_lists


def _ptr_array(tensors):
    arr = (ctypes.c_void_p * len(tensors))()
    for i, t in enumerate(tensors):
        arr[i] = t.data_ptr()
    return arr


def table_pointers(g, block_lists):
    """ctypes (global, per-block) pointer arrays for a weight table; keep the
    returned objects alive while the callee runs."""
    garr = _ptr_array(g)
    barrs = [_ptr_array(b) for b in block_lists]
    bt = (ctypes.c_void_p * len(barrs))()
    for i, a in enumerate(barrs):
        bt[i] = ctypes.cast(a, ctypes.c_void_p)
    return garr, barrs, bt


COMM_ID_BYTES = 128


def comm_unique_id():
    buf = ctypes.create_string_buffer(COMM_ID_BYTES)
    check(lib().qi_comm_unique_id(buf))
    return buf.raw


def exchange_plan(which, nb, n_txt, n_img, nranks, rank):
    """Per-peer (send_off, send_bytes, recv_off, recv_bytes) of a head-parallel
    block's exchange `which` (0: Q/K/V, 1: attention output); host only."""
    arrs = [(ctypes.c_longlong * nranks)() for _ in range(4)]
    check(lib().qi_exchange_plan(which, nb, n_txt, n_img, nranks, rank, *arrs))
    return [list(a) for a in arrs]


class Context:
    def __init__(self, device=0):
        self.h = ctypes.c_void_p()
        check(lib().qi_ctx_create(device, ctypes.byref(self.h)))

    def check(self):
        check(lib().qi_ctx_check(self.h))

    def launches(self):
        return lib().qi_ctx_last_launch_count(self.h)

    def set_comm(self, uid, rank, nranks):
        """Joins the head-parallel group `uid` (bytes from comm_unique_id() on
        rank 0) as `rank` of `nranks`; collective over the group."""
        buf = ctypes.create_string_buffer(bytes(uid), COMM_ID_BYTES) if uid is not None else None
        check(lib().qi_ctx_set_comm(self.h, buf, rank, nranks))

    def set_comm_timeout(self, ms):
        check(lib().qi_ctx_set_comm_timeout(self.h, int(ms)))

    def sync(self, timeout_ms=0):
        """Bounded wait for this context's work on the current stream; raises
        QIError (QI_ERR_NCCL) if the group's collectives failed or missed the
        deadline."""
        check(lib().qi_ctx_sync(self.h, _stream(), int(timeout_ms)))

    def set_hidden_capture(self, hidden):
        """Every forward copies its final image hidden state [nb*n_img, 3072]
        FP32 into `hidden` (a device tensor; None stops)."""
        check(lib().qi_ctx_set_hidden_capture(self.h, _p(hidden) if hidden is not None else None))

    def set_fused_qkv_epilogue(self, enable):
        """q/k RMSNorm + RoPE in the QKV GEMM's epilogue (True, the default)
        or as a separate kernel after an FP32 projection; same bits."""
        check(lib().qi_ctx_set_fused_qkv_epilogue(self.h, int(bool(enable))))

    def close(self):
        if self.h:
            lib().qi_ctx_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Model:
    def __init__(self, ctx, g, block_lists):
        self.h = ctypes.c_void_p()
        garr, barrs, bt = table_pointers(g, block_lists)
        check(lib().qi_model_create(ctx.h, len(block_lists), garr, bt, ctypes.byref(self.h)))

    @classmethod
    def from_safetensors(cls, ctx, path):
        self = cls.__new__(cls)
        self.h = ctypes.c_void_p()
        check(lib().qi_model_load_safetensors(ctx.h, path.encode(), ctypes.byref(self.h)))
        return self

    def num_blocks(self):
        return lib().qi_model_num_blocks(self.h)

    def close(self):
        if self.h:
            lib().qi_model_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def forward(ctx, model, x, t, txt, pe, out=None):
    """x: [nb,16,H,W] bf16, txt: [nb,n_txt,3584] bf16, pe: [nb,S,64,2,2] f32 (device)."""
    nb, _, H, W = x.shape
    n_txt = txt.shape[1]
    if out is None:
        out = torch.empty_like(x)
    check(lib().qi_forward(ctx.h, model.h, nb, _p(x), float(t), _p(txt), n_txt, _p(pe), H, W, _p(out), _stream()))
    return out


def forward_blocks(ctx, model, img, txt, t, pe, b0, b1, nb=1):
    """Runs blocks [b0, b1) in place on FP32 residual streams img [nb*n_img,3072], txt [nb*n_txt,3072]."""
    n_img = img.shape[0] // nb
    n_txt = txt.shape[0] // nb
    check(lib().qi_forward_blocks(ctx.h, model.h, nb, n_img, n_txt, _p(img), _p(txt), float(t), _p(pe), b0, b1,
                                  _stream()))


def spectrum_output(ctx, model, hidden, t, H, W, nb=1, out=None):
    """Output head on a final image hidden state [nb*n_img, 3072] FP32 -> [nb,16,H,W] bf16."""
    if out is None:
        out = torch.empty(nb, 16, H, W, dtype=torch.bfloat16, device=hidden.device)
    check(lib().qi_spectrum_output(ctx.h, model.h, nb, _p(hidden), float(t), H, W, _p(out), _stream()))
    return out


def spectrum_weights(steps, order, lam, target, blend):
    """Prediction weights over stored steps (increasing), as qi_spectrum_predict applies them."""
    K = len(steps)
    st = (ctypes.c_int * K)(*[int(v) for v in steps])
    w = (ctypes.c_double * K)()
    check(lib().qi_spectrum_weights(st, K, int(order), float(lam), int(target), float(blend), w))
    return np.array(w[:], dtype=np.float64)


class Spectrum:
    """Feature forecaster over the states of actual forwards (SpectrumState)."""

    def __init__(self, feature_elems, max_history=50, order=4, lam=0.1):
        self.h = ctypes.c_void_p()
        check(lib().qi_spectrum_create(int(feature_elems), int(max_history), int(order), float(lam),
                                       ctypes.byref(self.h)))

    def update(self, feature, step):
        check(lib().qi_spectrum_update(self.h, _p(feature), int(step), _stream()))

    def predict(self, target_step, blend=1.0, out=None, like=None):
        if out is None:
            out = torch.empty_like(like)
        check(lib().qi_spectrum_predict(self.h, int(target_step), float(blend), _p(out), _stream()))
        return out

    def history(self):
        return lib().qi_spectrum_history(self.h)

    def reset(self):
        check(lib().qi_spectrum_reset(self.h))

    def close(self):
        if self.h:
            lib().qi_spectrum_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def cfg_euler_step(latent, cond, uncond, cfg_scale, sigma, sigma_next, latent_bf16):
    _, _, H, W = latent.shape
    check(lib().qi_cfg_euler_step(_p(latent), _p(cond), _p(uncond), float(cfg_scale), float(sigma), float(sigma_next),
                                  H, W, _p(latent_bf16), _stream()))
