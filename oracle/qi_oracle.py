"""CPU oracle for the Qwen-Image MMDiT denoising path (test infrastructure).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg may use this module; the product never does.

Heavy loops live in qi_oracle.c / qi_synth.c (liboracle.so); this module
restates transformer_forward (transformer.cu:234-931 of the reference) in
numpy on top of them, in two modes:
  mode="fp32":  unquantized evaluation -- BF16 weights used as FP32, exact
                softmax attention (the "fp32 CPU evaluation" of a block);
  mode="quant": emulates the reference's arithmetic -- block-FWHT + per-token
                INT8 activations x INT8 weights with exact INT32 accumulation
                and the reference's dequant, Sage per-thread INT8 Q/K with FP16
                V and FP16 P (sageattention_sm80.cu).
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "liboracle.so")

DIM, HEADS, HEAD_DIM, MLP, TXT_DIM, PATCH_DIM, OUT_CH = 3072, 24, 128, 12288, 3584, 64, 16

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} missing: run `make -C oracle`")
        L = ctypes.CDLL(LIB_PATH)
        vp, i, f, ll, ull = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_longlong, ctypes.c_ulonglong
        sig = {
            "or_seed_for": ([ull, ctypes.c_char_p], ull),
            "or_gen_f32": ([ull, ll, f, f, vp], None),
            "or_gen_bf16": ([ull, ll, f, f, vp], None),
            "or_bf16_to_f32": ([vp, ll, vp], None),
            "or_f32_to_bf16": ([vp, ll, vp], None),
            "or_f32_to_f16_arr": ([vp, ll, vp], None),
            "or_hadamard_block_size": ([i], i),
            "or_fwht_rows": ([vp, ll, i, i], None),
            "or_fwht_quant": ([vp, ll, i, i, vp, vp], None),
            "or_quant_weight_bf16": ([vp, ll, i, vp, vp], None),
            "or_gemm_i8": ([vp, vp, ll, ll, i, vp], None),
            "or_gemm_f32": ([vp, vp, ll, ll, i, vp], None),
            "or_dequant": ([vp, vp, vp, vp, ll, ll, i, vp], None),
            "or_bias_act": ([vp, vp, ll, ll, i], None),
            "or_layernorm_modulate": ([vp, vp, vp, ll, i, f, vp], None),
            "or_rmsnorm": ([vp, vp, ll, i, f, vp], None),
            "or_silu": ([vp, ll, vp], None),
            "or_gate_add": ([vp, vp, vp, ll, i], None),
            "or_timestep_embedding": ([f, i, f, vp], None),
            "or_rope_table": ([i, i, i, vp], None),
            "or_rope_apply": ([vp, vp, vp, ll, i], None),
            "or_attention_exact": ([vp, vp, vp, i, i, f, vp], None),
            "or_attention_f32": ([vp, vp, vp, i, i, f, vp], None),
            "or_sage_kmean": ([vp, i, i, vp], None),
            "or_sage_quant_q": ([vp, i, i, vp, vp], None),
            "or_sage_quant_k": ([vp, vp, i, i, vp, vp], None),
            "or_sage_attention": ([vp, vp, vp, vp, vp, i, i, f, vp], None),
            "or_num_threads": ([], i),
            "or_set_num_threads": ([i], None),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------- synthetic data
def seed_for(base, name):
    return lib().or_seed_for(base, name.encode())


def gen_f32(seed, shape, scale=1.0, offset=0.0):
    out = np.empty(shape, dtype=np.float32)
    lib().or_gen_f32(seed, out.size, scale, offset, _p(out))
    return out


def gen_bf16(seed, shape, scale=1.0, offset=0.0):
    """BF16 bits as uint16."""
    out = np.empty(shape, dtype=np.uint16)
    lib().or_gen_bf16(seed, out.size, scale, offset, _p(out))
    return out


def bf16_to_f32(u16):
    u16 = _c(u16, np.uint16)
    return (u16.astype(np.uint32) << 16).view(np.float32).reshape(u16.shape)


def f32_to_bf16(x):
    x = _c(x, np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().or_f32_to_bf16(_p(x), x.size, _p(out))
    return out


def round_bf16(x):
    return bf16_to_f32(f32_to_bf16(x))


def f32_to_f16(x):
    """IEEE RN-even FP16 as numpy float16."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().or_f32_to_f16_arr(_p(x), x.size, _p(out))
    return out.view(np.float16)


# ----------------------------------------------------------------- kernels
def hadamard_block_size(K):
    return K & (-K)


def fwht_rows(x, B):
    x = _c(x, np.float32).copy()
    lib().or_fwht_rows(_p(x), x.shape[0], x.shape[1], B)
    return x


def fwht_quant(x, B=None):
    x = _c(x, np.float32)
    M, K = x.shape
    if B is None:
        B = hadamard_block_size(K)
    codes = np.empty((M, K), dtype=np.int8)
    scales = np.empty(M, dtype=np.float32)
    lib().or_fwht_quant(_p(x), M, K, B, _p(codes), _p(scales))
    return codes, scales


def quant_weight(w_u16):
    w = _c(w_u16, np.uint16)
    N, K = w.shape
    codes = np.empty((N, K), dtype=np.int8)
    scales = np.empty(N, dtype=np.float32)
    lib().or_quant_weight_bf16(_p(w), N, K, _p(codes), _p(scales))
    return codes, scales


def gemm_i8(a, b):
    a, b = _c(a, np.int8), _c(b, np.int8)
    M, K = a.shape
    N = b.shape[0]
    out = np.empty((M, N), dtype=np.int32)
    lib().or_gemm_i8(_p(a), _p(b), M, N, K, _p(out))
    return out


def gemm_f32(a, b):
    a, b = _c(a, np.float32), _c(b, np.float32)
    M, K = a.shape
    N = b.shape[0]
    out = np.empty((M, N), dtype=np.float32)
    lib().or_gemm_f32(_p(a), _p(b), M, N, K, _p(out))
    return out


def dequant(acc, sa, sw, bias_u16=None, gelu=False):
    acc = _c(acc, np.int32)
    M, N = acc.shape
    out = np.empty((M, N), dtype=np.float32)
    sa, sw = _c(sa, np.float32), _c(sw, np.float32)
    b = None if bias_u16 is None else _c(bias_u16, np.uint16)
    lib().or_dequant(_p(acc), _p(sa), _p(sw), None if b is None else _p(b), M, N, int(gelu), _p(out))
    return out


def bias_act(out, bias_u16=None, gelu=False):
    out = _c(out, np.float32).copy()
    b = None if bias_u16 is None else _c(bias_u16, np.uint16)
    lib().or_bias_act(_p(out), None if b is None else _p(b), out.shape[0], out.shape[1], int(gelu))
    return out


def layernorm_modulate(x, shift, scale, eps=1e-6):
    x = _c(x, np.float32)
    out = np.empty_like(x)
    lib().or_layernorm_modulate(_p(x), _p(_c(shift, np.float32)), _p(_c(scale, np.float32)), x.shape[0], x.shape[1],
                                eps, _p(out))
    return out


def rmsnorm(x, w_u16, eps=1e-6):
    x = _c(x, np.float32)
    out = np.empty_like(x)
    lib().or_rmsnorm(_p(x), _p(_c(w_u16, np.uint16)), x.shape[0], x.shape[1], eps, _p(out))
    return out


def silu(x):
    x = _c(x, np.float32)
    out = np.empty_like(x)
    lib().or_silu(_p(x), x.size, _p(out))
    return out


def gelu_tanh(v):
    v = v.astype(np.float32)
    return (0.5 * v * (1.0 + np.tanh(0.7978845608 * (v + 0.044715 * v * v * v)))).astype(np.float32)


def timestep_embedding(t):
    out = np.empty(256, dtype=np.float32)
    lib().or_timestep_embedding(float(t), 256, 10000.0, _p(out))
    return out


def rope_table(h, w, n_txt):
    n = n_txt + ((h + 1) // 2) * ((w + 1) // 2)
    pe = np.empty((n, 64, 2, 2), dtype=np.float32)
    lib().or_rope_table(h, w, n_txt, _p(pe))
    return pe


def rope_apply(x, pe, pos):
    """x: [rows, H, 128] token-major (modified copy returned); pos: [rows] int."""
    x = _c(x, np.float32).copy()
    pos = _c(pos, np.int32)
    lib().or_rope_apply(_p(x), _p(_c(pe, np.float32)), _p(pos), x.shape[0], x.shape[1])
    return x


def attention_exact(q, k, v, scale):
    q, k, v = (_c(a, np.float32) for a in (q, k, v))
    H, S, _ = q.shape
    out = np.empty_like(q)
    lib().or_attention_exact(_p(q), _p(k), _p(v), H, S, float(scale), _p(out))
    return out


def attention_f32(q, k, v, scale):
    """FP32 softmax attention through the blocked CPU GEMM (timed baseline)."""
    q, k, v = (_c(a, np.float32) for a in (q, k, v))
    H, S, _ = q.shape
    out = np.empty_like(q)
    lib().or_attention_f32(_p(q), _p(k), _p(v), H, S, float(scale), _p(out))
    return out


def sage_quantize(q16, k16):
    """q16, k16: FP16 values (any float dtype holding FP16 values) [H, S, 128]."""
    q, k = _c(q16, np.float32), _c(k16, np.float32)
    H, S, _ = q.shape
    kmean = np.empty((H, 128), dtype=np.float32)
    lib().or_sage_kmean(_p(k), H, S, _p(kmean))
    qc = np.empty((H, S, 128), dtype=np.int8)
    kc = np.empty((H, S, 128), dtype=np.int8)
    qs = np.empty((H, ((S + 127) // 128) * 32), dtype=np.float32)
    ks = np.empty((H, ((S + 63) // 64) * 4), dtype=np.float32)
    lib().or_sage_quant_q(_p(q), H, S, _p(qc), _p(qs))
    lib().or_sage_quant_k(_p(k), _p(kmean), H, S, _p(kc), _p(ks))
    return kmean, qc, qs, kc, ks


def sage_attention(q16, k16, v16, scale):
    _, qc, qs, kc, ks = sage_quantize(q16, k16)
    v = _c(v16, np.float32)
    H, S, _ = v.shape
    out = np.empty((H, S, 128), dtype=np.float32)
    lib().or_sage_attention(_p(qc), _p(qs), _p(kc), _p(ks), _p(v), H, S, float(scale), _p(out))
    return out


# ---------------------------------------------------------------- Spectrum
def spectrum_predict(hist, steps, target, blend=1.0, order=4, lam=0.1):
    """The reference's spectrum_predict (cuda_kernels.cu:6268-6333) in float64
    on the stored states hist [K, F] (oldest first) at steps[0..K):
      tau_k = (t_k - mid) * 2 / range, mid / range over steps[0], steps[K-1]
        (normalize_tau_kernel, :5890-5904; 0 when range < 1e-6);
      X[k, m] = T_m(tau_k) by the Chebyshev recurrence (chebyshev_design_kernel,
        :5865-5886); C = (X^T X + lam I)^-1 X^T H (spectrum_fit_ridge_regression,
        :6014-6089: SGEMMs, Cholesky, two triangular solves);
      cheb = row(tau_target) C (build_chebyshev_row_kernel, chebyshev_predict_kernel);
      taylor = h_i + k (h_i - h_{i-1}), k = (target - t_i) / max(t_i - t_{i-1}, 1e-6)
        (taylor_predict_kernel with order 1, :6104-6149);
      out = (1 - blend) taylor + blend cheb (blend_predictions_kernel, :6152-6162)."""
    hist = np.asarray(hist, dtype=np.float64)
    t = np.asarray(steps, dtype=np.float64)
    P = order + 1
    mid, rng = 0.5 * (t[0] + t[-1]), t[-1] - t[0]

    def tau(v):
        return 0.0 if rng < 1e-6 else (v - mid) * 2.0 / rng

    def cheb_row(x):
        r = np.zeros(P)
        r[0] = 1.0
        if P > 1:
            r[1] = x
        for m in range(2, P):
            r[m] = 2.0 * x * r[m - 1] - r[m - 2]
        return r

    X = np.stack([cheb_row(tau(v)) for v in t])
    A = X.T @ X + lam * np.eye(P)
    C = np.linalg.solve(A, X.T @ hist)
    cheb = cheb_row(tau(float(target))) @ C
    dt = max(t[-1] - t[-2], 1e-6)
    k = (float(target) - t[-1]) / dt
    taylor = hist[-1] + k * (hist[-1] - hist[-2])
    return (1.0 - blend) * taylor + blend * cheb


def set_threads(n):
    lib().or_set_num_threads(int(n))


def num_threads():
    return lib().or_num_threads()


# ----------------------------------------------------------------- weights
G_SHAPES = {
    "time_text_embed.timestep_embedder.linear_1": (DIM, 256),
    "time_text_embed.timestep_embedder.linear_2": (DIM, DIM),
}
L_NAMES = [
    ("img_mod.1", 6 * DIM, DIM), ("txt_mod.1", 6 * DIM, DIM),
    ("attn.to_q", DIM, DIM), ("attn.to_k", DIM, DIM), ("attn.to_v", DIM, DIM),
    ("attn.add_q_proj", DIM, DIM), ("attn.add_k_proj", DIM, DIM), ("attn.add_v_proj", DIM, DIM),
    ("attn.to_out.0", DIM, DIM), ("attn.to_add_out", DIM, DIM),
    ("img_mlp.net.0.proj", MLP, DIM), ("img_mlp.net.2", DIM, MLP),
    ("txt_mlp.net.0.proj", MLP, DIM), ("txt_mlp.net.2", DIM, MLP),
]
B_NORMS = ["attn.norm_q.weight", "attn.norm_k.weight", "attn.norm_added_q.weight", "attn.norm_added_k.weight"]


class Weights:
    """Seeded synthetic weights (same seeds and generator as the product's
    make_weight_table), BF16 bits plus lazily computed INT8 codes."""

    def __init__(self, num_blocks, base_seed=0, wscale=0.02):
        self.base = base_seed
        self.wscale = wscale
        self.num_blocks = num_blocks
        self._cache = {}

    def bf16(self, name, shape, offset=0.0):
        key = ("b", name)
        if key not in self._cache:
            self._cache[key] = gen_bf16(seed_for(self.base, name), shape, self.wscale, offset)
        return self._cache[key]

    def f32(self, name, shape, offset=0.0):
        return bf16_to_f32(self.bf16(name, shape, offset))

    def int8(self, name, shape):
        key = ("q", name)
        if key not in self._cache:
            self._cache[key] = quant_weight(self.bf16(name, shape))
        return self._cache[key]

    def linear_names(self, prefix):
        return prefix + ".weight", prefix + ".bias"


def _linear(W, prefix, N, K, x, mode, gelu=False, act_q=None):
    """INT8 linear of the reference (linear_forward_int8 / _prequantized)."""
    wn, bn = prefix + ".weight", prefix + ".bias"
    bias = W.bf16(bn, (N,))
    if mode == "quant":
        codes, sw = W.int8(wn, (N, K))
        if act_q is None:
            act_q = fwht_quant(x, hadamard_block_size(K))
        acc = gemm_i8(act_q[0], codes)
        return dequant(acc, act_q[1], sw, bias, gelu)
    out = gemm_f32(x, W.f32(wn, (N, K)))
    return bias_act(out, bias, gelu)


def _linear_bf16w(W, prefix, N, K, x_bf16vals):
    """BF16 boundary linear (linear_forward_bf16*: BF16 x BF16, FP32 accumulate,
    then FP32 bias add)."""
    out = gemm_f32(x_bf16vals, W.f32(prefix + ".weight", (N, K)))
    return bias_act(out, W.bf16(prefix + ".bias", (N,)))


def patchify(x):
    """[nb,16,H,W] -> [nb*n_img, 64] (patchify_kernel, cuda_kernels.cu:1244)."""
    nb, C, H, Wd = x.shape
    t = x.reshape(nb, C, H // 2, 2, Wd // 2, 2).transpose(0, 2, 4, 1, 3, 5)
    return t.reshape(nb * (H // 2) * (Wd // 2), C * 4)


def unpatchify(p, nb, H, Wd):
    t = p.reshape(nb, H // 2, Wd // 2, OUT_CH, 2, 2).transpose(0, 3, 1, 4, 2, 5)
    return t.reshape(nb, OUT_CH, H, Wd)


def block(W, img, txt, mi, mt, pe, mode="quant", bi=0, rec=None):
    """One double-stream block (transformer.cu:497-836) on FP32 residual
    streams img [n_img,3072], txt [n_txt,3072] with modulation vectors mi, mt
    ([18432] each, chunks [shift1, scale1, gate1, shift2, scale2, gate2]).
    Returns the updated (img, txt); `rec` receives the block's stage values."""
    rec = rec if rec is not None else {}
    pre = f"transformer_blocks.{bi}."
    n_img, n_txt = img.shape[0], txt.shape[0]
    S = n_img + n_txt
    pos_img = np.arange(n_txt, S, dtype=np.int32)
    pos_txt = np.arange(0, n_txt, dtype=np.int32)
    scale = np.float32(1.0 / np.sqrt(128.0))
    ch = lambda m, k: m[k * DIM:(k + 1) * DIM]
    img_n = layernorm_modulate(img, ch(mi, 0), ch(mi, 1))
    txt_n = layernorm_modulate(txt, ch(mt, 0), ch(mt, 1))
    rec["img_modulated"] = img_n.copy()
    aq_i = fwht_quant(img_n, 1024) if mode == "quant" else None
    aq_t = fwht_quant(txt_n, 1024) if mode == "quant" else None
    qi_ = _linear(W, pre + "attn.to_q", DIM, DIM, img_n, mode, act_q=aq_i)
    ki_ = _linear(W, pre + "attn.to_k", DIM, DIM, img_n, mode, act_q=aq_i)
    vi_ = _linear(W, pre + "attn.to_v", DIM, DIM, img_n, mode, act_q=aq_i)
    qt_ = _linear(W, pre + "attn.add_q_proj", DIM, DIM, txt_n, mode, act_q=aq_t)
    kt_ = _linear(W, pre + "attn.add_k_proj", DIM, DIM, txt_n, mode, act_q=aq_t)
    vt_ = _linear(W, pre + "attn.add_v_proj", DIM, DIM, txt_n, mode, act_q=aq_t)
    nq = W.bf16(pre + "attn.norm_q.weight", (128,), 1.0)
    nk = W.bf16(pre + "attn.norm_k.weight", (128,), 1.0)
    naq = W.bf16(pre + "attn.norm_added_q.weight", (128,), 1.0)
    nak = W.bf16(pre + "attn.norm_added_k.weight", (128,), 1.0)
    qi_ = rmsnorm(qi_.reshape(-1, 128), nq).reshape(n_img, HEADS, 128)
    ki_ = rmsnorm(ki_.reshape(-1, 128), nk).reshape(n_img, HEADS, 128)
    qt_ = rmsnorm(qt_.reshape(-1, 128), naq).reshape(n_txt, HEADS, 128)
    kt_ = rmsnorm(kt_.reshape(-1, 128), nak).reshape(n_txt, HEADS, 128)
    rec["img_q_normed"] = qi_.reshape(n_img, DIM).copy()
    q = np.concatenate([rope_apply(qt_, pe, pos_txt), rope_apply(qi_, pe, pos_img)], 0)
    k = np.concatenate([rope_apply(kt_, pe, pos_txt), rope_apply(ki_, pe, pos_img)], 0)
    v = np.concatenate([vt_.reshape(n_txt, HEADS, 128), vi_.reshape(n_img, HEADS, 128)], 0)
    qh, kh, vh = (a.transpose(1, 0, 2).copy() for a in (q, k, v))  # [H, S, 128]
    if mode == "quant":
        o = sage_attention(f32_to_f16(qh).astype(np.float32), f32_to_f16(kh).astype(np.float32),
                           f32_to_f16(vh).astype(np.float32), scale)
    else:
        o = attention_exact(qh, kh, vh, scale)
    o = o.transpose(1, 0, 2).reshape(S, DIM)
    o_txt, o_img = o[:n_txt], o[n_txt:]
    rec["attn_out_img"], rec["attn_out_txt"] = o_img.copy(), o_txt.copy()
    img = img + ch(mi, 2)[None, :] * _linear(W, pre + "attn.to_out.0", DIM, DIM, o_img, mode)
    txt = txt + ch(mt, 2)[None, :] * _linear(W, pre + "attn.to_add_out", DIM, DIM, o_txt, mode)
    rec["img_after_attn"] = img.copy()
    img_n = layernorm_modulate(img, ch(mi, 3), ch(mi, 4))
    txt_n = layernorm_modulate(txt, ch(mt, 3), ch(mt, 4))
    hi = _linear(W, pre + "img_mlp.net.0.proj", MLP, DIM, img_n, mode, gelu=True)
    ht = _linear(W, pre + "txt_mlp.net.0.proj", MLP, DIM, txt_n, mode, gelu=True)
    img = img + ch(mi, 5)[None, :] * _linear(W, pre + "img_mlp.net.2", DIM, MLP, hi, mode)
    txt = txt + ch(mt, 5)[None, :] * _linear(W, pre + "txt_mlp.net.2", DIM, MLP, ht, mode)
    rec["img_after_mlp"], rec["txt_after_mlp"] = img.copy(), txt.copy()
    return img.astype(np.float32), txt.astype(np.float32)


def forward(W, x_u16, t, txt_u16, pe, mode="quant", num_blocks=None, record=None):
    """One transformer_forward for a single batch element.

    x_u16: [1,16,H,W] BF16 bits; txt_u16: [n_txt,3584] BF16 bits; pe: [S,64,2,2].
    Returns the BF16-rounded velocity [1,16,H,W] as float32.  `record`, if a
    dict, receives intermediates keyed like the reference's DUMP names."""
    L = W.num_blocks if num_blocks is None else num_blocks
    rec = record if record is not None else {}
    _, _, H, Wd = x_u16.shape
    n_txt = txt_u16.shape[0]
    n_img = (H // 2) * (Wd // 2)
    S = n_txt + n_img
    # timestep MLP (transformer.cu:330-349)
    temb = timestep_embedding(t)[None, :]
    h = _linear(W, "time_text_embed.timestep_embedder.linear_1", DIM, 256, temb, mode)
    h = silu(h)
    temb = _linear(W, "time_text_embed.timestep_embedder.linear_2", DIM, DIM, h, mode)
    rec["t_emb"] = temb[0].copy()
    tsilu = silu(temb)
    # input projections (transformer.cu:396-422)
    patches = bf16_to_f32(patchify(x_u16))
    img = _linear_bf16w(W, "img_in", DIM, PATCH_DIM, patches)
    rec["img_after_proj"] = img.copy()
    ctx = bf16_to_f32(txt_u16)
    tn = round_bf16(rmsnorm(ctx, W.bf16("txt_norm.weight", (TXT_DIM,), 1.0)))
    txt = _linear_bf16w(W, "txt_in", DIM, TXT_DIM, tn)
    rec["txt_after_proj"] = txt.copy()
    for bi in range(L):
        pre = f"transformer_blocks.{bi % W.num_blocks}."
        mi = _linear(W, pre + "img_mod.1", 6 * DIM, DIM, tsilu, mode)[0]
        mt = _linear(W, pre + "txt_mod.1", 6 * DIM, DIM, tsilu, mode)[0]
        if bi == 0:
            rec["img_mods"], rec["txt_mods"] = mi.copy(), mt.copy()
        img, txt = block(W, img, txt, mi, mt, pe, mode, bi % W.num_blocks, rec if bi == 0 else None)
    rec["img_final"] = img.copy()
    # output AdaLN (transformer.cu:873-926)
    ada = _linear_bf16w(W, "norm_out.linear", 2 * DIM, DIM, round_bf16(tsilu))[0]
    fin = layernorm_modulate(img, ada[DIM:], ada[:DIM])
    proj = _linear_bf16w(W, "proj_out", PATCH_DIM, DIM, round_bf16(fin))
    out = round_bf16(proj)
    return unpatchify(out, 1, H, Wd)


def metrics(a, b):
    """cosine similarity and normwise max relative error max|a-b| / max|b|."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
    maxrel = float(np.max(np.abs(a - b)) / (np.max(np.abs(b)) + 1e-300))
    return cos, maxrel


def block_fp32(W, img, txt, mods_img, mods_txt, pe, bi=0):
    """One double-stream block in FP32 (the unquantized CPU evaluation; the
    block body of transformer_forward, transformer.cu:497-836), using the
    GEMM-based attention.  Returns the updated (img, txt)."""
    pre = f"transformer_blocks.{bi}."
    n_img, n_txt = img.shape[0], txt.shape[0]
    S = n_img + n_txt
    ch = lambda m, k: m[k * DIM:(k + 1) * DIM]
    mi, mt = mods_img, mods_txt
    img_n = layernorm_modulate(img, ch(mi, 0), ch(mi, 1))
    txt_n = layernorm_modulate(txt, ch(mt, 0), ch(mt, 1))
    lin = lambda name, N, K, x, gelu=False: _linear(W, pre + name, N, K, x, "fp32", gelu)
    qi_, ki_, vi_ = (lin(n, DIM, DIM, img_n) for n in ("attn.to_q", "attn.to_k", "attn.to_v"))
    qt_, kt_, vt_ = (lin(n, DIM, DIM, txt_n) for n in ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"))
    nq = W.bf16(pre + "attn.norm_q.weight", (128,), 1.0)
    nk = W.bf16(pre + "attn.norm_k.weight", (128,), 1.0)
    naq = W.bf16(pre + "attn.norm_added_q.weight", (128,), 1.0)
    nak = W.bf16(pre + "attn.norm_added_k.weight", (128,), 1.0)
    qi_ = rmsnorm(qi_.reshape(-1, 128), nq).reshape(n_img, HEADS, 128)
    ki_ = rmsnorm(ki_.reshape(-1, 128), nk).reshape(n_img, HEADS, 128)
    qt_ = rmsnorm(qt_.reshape(-1, 128), naq).reshape(n_txt, HEADS, 128)
    kt_ = rmsnorm(kt_.reshape(-1, 128), nak).reshape(n_txt, HEADS, 128)
    pos_img = np.arange(n_txt, S, dtype=np.int32)
    pos_txt = np.arange(0, n_txt, dtype=np.int32)
    q = np.concatenate([rope_apply(qt_, pe, pos_txt), rope_apply(qi_, pe, pos_img)], 0)
    k = np.concatenate([rope_apply(kt_, pe, pos_txt), rope_apply(ki_, pe, pos_img)], 0)
    v = np.concatenate([vt_.reshape(n_txt, HEADS, 128), vi_.reshape(n_img, HEADS, 128)], 0)
    o = attention_f32(*(a.transpose(1, 0, 2).copy() for a in (q, k, v)), np.float32(1.0 / np.sqrt(128.0)))
    o = o.transpose(1, 0, 2).reshape(S, DIM)
    img = img + ch(mi, 2)[None, :] * lin("attn.to_out.0", DIM, DIM, np.ascontiguousarray(o[n_txt:]))
    txt = txt + ch(mt, 2)[None, :] * lin("attn.to_add_out", DIM, DIM, np.ascontiguousarray(o[:n_txt]))
    img_n = layernorm_modulate(img, ch(mi, 3), ch(mi, 4))
    txt_n = layernorm_modulate(txt, ch(mt, 3), ch(mt, 4))
    img = img + ch(mi, 5)[None, :] * lin("img_mlp.net.2", DIM, MLP, lin("img_mlp.net.0.proj", MLP, DIM, img_n, True))
    txt = txt + ch(mt, 5)[None, :] * lin("txt_mlp.net.2", DIM, MLP, lin("txt_mlp.net.0.proj", MLP, DIM, txt_n, True))
    return img.astype(np.float32), txt.astype(np.float32)
