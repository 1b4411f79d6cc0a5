"""The fused QKV projection (the q/k RMSNorm + RoPE + FP16 head-major store of
qkv_post in the CTA-pair GEMM's epilogue) against the two-launch form it
replaces: the FP32 projection (qi_linear_i8) followed by qi_qk_norm_rope,
which test_gpu_attribution.py pins bit for bit to the reference's
linear_forward_int8_prequantized + rms_norm_fp32 + rope_apply_fp32_to_fp16
(transformer.cu:568-671).  The bar is bit-identity: every FP16 element of
Q, K and V, and the whole 60-block forward with the fusion on and off."""
import pytest
import torch

import qib200 as Q

pytestmark = pytest.mark.gpu


def _stream_inputs(rows, tag, seed):
    x = Q.synth((rows, 3072), Q.seed_for(seed, f"x_{tag}"), 1.0)
    w = Q.synth((9216, 3072), Q.seed_for(seed, f"w_{tag}"), 0.02, dtype=torch.bfloat16)
    b = Q.synth((9216,), Q.seed_for(seed, f"b_{tag}"), 0.02, dtype=torch.bfloat16)
    ac, asc = Q.fwht_quantize(x)
    wc, ws = Q.quantize_weight(w)
    return (ac, asc), (wc, ws, b)


# (nb, latent H, W, text tokens): ragged image rows, a batch boundary inside
# 256-row tiles, text rows that fill less than one tile, and the C4 shape
CASES = [(1, 48, 48, 64), (2, 46, 38, 37), (2, 32, 32, 5), (2, 166, 166, 256)]


@pytest.mark.parametrize("nb,H,W,n_txt", CASES)
def test_fused_projection_equals_two_launches(nb, H, W, n_txt):
    torch.cuda.set_device(0)
    n_img = ((H + 1) // 2) * ((W + 1) // 2)
    seed = 40 + H + n_txt
    act_i, w_i = _stream_inputs(nb * n_img, "img", seed)
    act_t, w_t = _stream_inputs(nb * n_txt, "txt", seed)
    norms = Q.synth((4, 128), Q.seed_for(seed, "norms"), 0.1, 1.0, dtype=torch.bfloat16)
    pe1 = torch.from_numpy(Q.rope_table(H, W, n_txt)).cuda()
    pe = torch.stack([pe1] * nb).contiguous()
    fused = Q.qkv_norm_rope_i8(act_i, act_t, w_i, w_t, norms, pe, nb)
    qi = Q.linear_i8(act_i[0], act_i[1], w_i[0], w_i[1], w_i[2])
    qt = Q.linear_i8(act_t[0], act_t[1], w_t[0], w_t[1], w_t[2])
    sep = Q.qk_norm_rope(qi, qt, norms, pe, nb)
    torch.cuda.synchronize()
    for k, name in enumerate("qkv"):
        a, b = fused[k].view(torch.int16), sep[k].view(torch.int16)
        nd = int((a != b).sum())
        assert nd == 0, f"{name}: {nd} of {a.numel()} FP16 elements differ"


def test_fused_projection_refuses_short_inputs():
    """Fewer than 512 rows in all run on the one-CTA GEMM, which has no fused
    epilogue: the entry says so instead of falling back silently."""
    torch.cuda.set_device(0)
    act_i, w_i = _stream_inputs(100, "img", 7)
    act_t, w_t = _stream_inputs(20, "txt", 7)
    norms = Q.synth((4, 128), Q.seed_for(7, "norms"), 0.1, 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(Q.rope_table(20, 20, 20)).cuda()[None]
    with pytest.raises(Q.QIError):
        Q.qkv_norm_rope_i8(act_i, act_t, w_i, w_t, norms, pe, 1)


def test_forward_same_bits_with_and_without_fusion():
    torch.cuda.set_device(0)
    g, blocks = Q.make_weight_table(60, base_seed=0)
    ctx = Q.Context(0)
    model = Q.Model(ctx, g, blocks)
    H, W, n_txt, nb = 46, 38, 37, 2
    n_img = (H // 2) * (W // 2)
    x = Q.synth((nb, 16, H, W), Q.seed_for(41, "latent"), 1.0, dtype=torch.bfloat16)
    txt = Q.synth((nb, n_txt, 3584), Q.seed_for(41, "context"), 1.0, dtype=torch.bfloat16)
    pe1 = torch.from_numpy(Q.rope_table(H, W, n_txt)).cuda()
    pe = torch.stack([pe1] * nb).contiguous()
    outs = []
    for fused in (True, False):
        ctx.set_fused_qkv_epilogue(fused)
        hidden = torch.empty(nb * n_img, 3072, device="cuda")
        ctx.set_hidden_capture(hidden)
        y = Q.forward(ctx, model, x, 700.0, txt, pe)
        ctx.set_hidden_capture(None)
        ctx.check()
        outs.append((y, hidden))
    ctx.set_fused_qkv_epilogue(True)
    (y1, h1), (y0, h0) = outs
    assert torch.equal(h1, h0)
    assert torch.equal(y1, y0)
    model.close()
    ctx.close()
