"""Stage-by-stage attribution of block 0's differences from the reference.

The reference's block (transformer.cu:497-836) is replayed with the
reference's own kernels (oracle/_ref: layer_norm_modulate_fp32,
quantize_activation_int8_hadamard_fp32, linear_forward_int8(_prequantized),
rms_norm_fp32, rope_apply_fp32_to_fp16, the Sage kernels, gate_add_fp32f)
and checked bit for bit against the reference's own stage dumps
(DUMP_TRANSFORMER_INTERNAL_BLOCK, transformer.cu:23-29, 499-504).  Each of
the product's stages is then fed the reference's own upstream tensor, so a
difference is charged to the stage that makes it:

  LN1+quant   qi_layer_norm_modulate_quantize   codes vs the reference's
  QKV         qi_linear_i8 (store epilogue)     FP32 vs img_q/k/v_raw
  qk-norm     qi_qk_norm_rope                   FP16 vs rms_norm + RoPE
  sage quant  qi_sage_quantize                  codes/scales/k-mean
  attention   qi_sage_attention                 FP32 (FP16 values) vs ref
  quant_o     qi_fwht_quantize                  codes
  out+gate    qi_linear_i8 (residual epilogue)  FP32 vs img_after_attn
  LN2+quant   qi_layer_norm_modulate_quantize   codes
  fc1+GELU    qi_linear_i8 (GELU epilogue)      FP32 vs img_mlp_gelu
  quant_h     qi_fwht_quantize (FWHT-4096)      codes
  fc2+gate    qi_linear_i8 (residual epilogue)  FP32 vs img_after_mlp

Every stage but attention is bit-exact.  The last test closes the loop: the
reference's own post-attention stages fed the product's attention output
reproduce the product's whole block bit for bit, so every remaining code flip
of the block starts at the attention output (tcgen05 accumulation over
128-key blocks against the reference's mma.sync fragments over 64-key blocks,
with their own running-max update points: the one stage whose arithmetic
cannot be reproduced).
"""
import numpy as np
import pytest
import torch

import qib200 as Q
import qi_ref as R

from test_gpu_model import ref_dumps

pytestmark = pytest.mark.gpu

SM_SCALE = 1.0 / np.sqrt(128.0)


@pytest.fixture(scope="module")
def env():
    torch.cuda.set_device(0)
    if not R.available():
        pytest.skip("reference build oracle/_ref/libqiref.so missing")
    g, blocks = R.make_table(60, distinct=2)
    ctx = Q.Context(0)
    model = Q.Model(ctx, g, blocks)
    ptrs = R.table_pointers(g, blocks)
    yield dict(g=g, blocks=blocks, ctx=ctx, model=model, ptrs=ptrs)
    model.close()
    ctx.close()
    torch.cuda.synchronize()


def lin(blk, name):
    i = [n for n, _, _ in R.L_NAMES].index(name)
    return blk[3 * i], blk[3 * i + 1], blk[3 * i + 2]


def norms(blk):
    return torch.stack(blk[3 * len(R.L_NAMES):3 * len(R.L_NAMES) + 4])


def ndiff(a, b):
    """Elements whose bits differ."""
    a = a.contiguous().view(-1)
    b = b.contiguous().view(-1)
    if a.dtype.is_floating_point:
        a = a.view(torch.int32 if a.element_size() == 4 else torch.int16)
        b = b.view(torch.int32 if b.element_size() == 4 else torch.int16)
    return int((a != b).sum())


def maxrel(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float((a - b).abs().max() / b.abs().max())


def ref_block(blk, x_img, x_txt, mi, mt, pe, n_img, n_txt):
    """One reference block with the reference's own kernels, stage by
    stage, in transformer.cu's order.  Returns every intermediate."""
    S = n_img + n_txt
    r = {}
    for tag, x, m, names in (("img", x_img, mi, ("attn.to_q", "attn.to_k", "attn.to_v")),
                             ("txt", x_txt, mt, ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj"))):
        ln = R.layer_norm_modulate(x, m[0].contiguous(), m[1].contiguous())
        c, s = R.fwht_quantize(ln, 1024)
        r[f"{tag}_ln1"], r[f"{tag}_c1"], r[f"{tag}_s1"] = ln, c, s
        r[f"{tag}_qkv"] = [R.linear_int8_preq(c, s, *lin(blk, n)) for n in names]
    nw = norms(blk)
    qn_i = R.rms_norm(r["img_qkv"][0].view(-1, 128), nw[0]).view(n_img, 24, 128)
    kn_i = R.rms_norm(r["img_qkv"][1].view(-1, 128), nw[1]).view(n_img, 24, 128)
    qn_t = R.rms_norm(r["txt_qkv"][0].view(-1, 128), nw[2]).view(n_txt, 24, 128)
    kn_t = R.rms_norm(r["txt_qkv"][1].view(-1, 128), nw[3]).view(n_txt, 24, 128)
    joint = lambda t, i: torch.cat([t, i]).transpose(0, 1).contiguous()  # [24, S, 128], txt first
    r["q_joint"], r["k_joint"] = joint(qn_t, qn_i), joint(kn_t, kn_i)
    r["qh"] = R.rope_fp16(r["q_joint"], pe)
    r["kh"] = R.rope_fp16(r["k_joint"], pe)
    r["vh"] = joint(r["txt_qkv"][2].view(n_txt, 24, 128), r["img_qkv"][2].view(n_img, 24, 128)).half()
    r["o"] = R.sage_attention(r["qh"], r["kh"], r["vh"], SM_SCALE)
    r.update(ref_post_attention(blk, r["o"], x_img, x_txt, mi, mt, n_img, n_txt))
    assert r["o"].shape == (24, S, 128)
    return r


def split_o(o, n_img, n_txt):
    o_t = o[:, :n_txt].transpose(0, 1).reshape(n_txt, 3072).contiguous()
    o_i = o[:, n_txt:].transpose(0, 1).reshape(n_img, 3072).contiguous()
    return o_i, o_t


def ref_post_attention(blk, o, x_img, x_txt, mi, mt, n_img, n_txt):
    """transformer.cu:676-823 with the reference's kernels, from the attention
    output [24, S, 128]."""
    o_i, o_t = split_o(o, n_img, n_txt)
    r = {"o_img": o_i, "o_txt": o_t}
    for tag, x, m, oo, names in (("img", x_img, mi, o_i, ("attn.to_out.0", "img_mlp.net.0.proj", "img_mlp.net.2")),
                                 ("txt", x_txt, mt, o_t, ("attn.to_add_out", "txt_mlp.net.0.proj", "txt_mlp.net.2"))):
        r[f"{tag}_co"], r[f"{tag}_so"] = R.fwht_quantize(oo, 1024)
        proj = R.linear_int8(oo, *lin(blk, names[0]))
        x2 = R.gate_add(x, m[2].contiguous(), proj)
        ln2 = R.layer_norm_modulate(x2, m[3].contiguous(), m[4].contiguous())
        r[f"{tag}_c2"], r[f"{tag}_s2"] = R.fwht_quantize(ln2, 1024)
        h = R.linear_int8(ln2, *lin(blk, names[1]), gelu=True)
        r[f"{tag}_ch"], r[f"{tag}_sh"] = R.fwht_quantize(h, 4096)
        mlp = R.linear_int8(h, *lin(blk, names[2]))
        x3 = R.gate_add(x2, m[5].contiguous(), mlp)
        r[f"{tag}_proj"], r[f"{tag}_after_attn"], r[f"{tag}_ln2"] = proj, x2, ln2
        r[f"{tag}_h"], r[f"{tag}_mlp"], r[f"{tag}_after_mlp"] = h, mlp, x3
    return r


CASES = [(64, 64, 64, 500.0), (166, 166, 256, 980.0)]


def setup_case(env, H, W, n_txt, t, block=0):
    """The reference's input streams and modulation of `block` (from its
    dumps of that block and of the one before), on the device."""
    x = R.synth((1, 16, H, W), R.seed_for(1, "latent"), 1.0, dtype=torch.bfloat16)
    txt = R.synth((1, n_txt, 3584), R.seed_for(1, "context"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(Q.rope_table(H, W, n_txt)).cuda()
    d = ref_dumps(env, x, t, txt, pe, H, W, block)
    n_img = (H // 2) * (W // 2)
    cu = lambda dd, k, *shape: torch.from_numpy(dd[k].copy()).cuda().view(*shape)
    if block == 0:
        x_img, x_txt = cu(d, "img_after_proj", n_img, 3072), cu(d, "txt_after_proj", n_txt, 3072)
    else:
        p = ref_dumps(env, x, t, txt, pe, H, W, block - 1)
        x_img = cu(p, f"b{block - 1}_img_after_mlp", n_img, 3072)
        x_txt = cu(p, f"b{block - 1}_txt_after_mlp", n_txt, 3072)
    mi, mt = cu(d, f"b{block}_img_mods", 6, 3072), cu(d, f"b{block}_txt_mods", 6, 3072)
    return (lambda k, *shape: cu(d, k, *shape)), pe, n_img, x_img, x_txt, mi, mt


@pytest.mark.parametrize("H,W,n_txt,t", CASES)
def test_reference_replay_matches_its_dumps(env, H, W, n_txt, t):
    """The replay above is the reference's block: bit-exact with its dumps."""
    cu, pe, n_img, x_img, x_txt, mi, mt = setup_case(env, H, W, n_txt, t)
    r = ref_block(env["blocks"][0], x_img, x_txt, mi, mt, pe, n_img, n_txt)
    S = n_img + n_txt
    checks = [("img_modulated", r["img_ln1"]), ("img_q_raw", r["img_qkv"][0]), ("img_k_raw", r["img_qkv"][1]),
              ("img_v_raw", r["img_qkv"][2]), ("q_joint", r["q_joint"]), ("k_joint", r["k_joint"]),
              ("attn_out_img", r["o_img"]), ("attn_out_txt", r["o_txt"]), ("img_proj", r["img_proj"]),
              ("img_after_attn", r["img_after_attn"]), ("img_mlp_input", r["img_ln2"]),
              ("img_mlp_gelu", r["img_h"]), ("img_mlp_out", r["img_mlp"]), ("img_after_mlp", r["img_after_mlp"]),
              ("txt_after_mlp", r["txt_after_mlp"])]
    for key, ours in checks:
        ref = cu("b0_" + key, *ours.shape)
        assert ndiff(ours, ref) == 0, key
    assert r["o"].shape == (24, S, 128)


@pytest.mark.parametrize("H,W,n_txt,t", CASES)
def test_stage_attribution(env, H, W, n_txt, t):
    """Each product stage on the reference's own input of that stage."""
    cu, pe, n_img, x_img, x_txt, mi, mt = setup_case(env, H, W, n_txt, t)
    blk = env["blocks"][0]
    r = ref_block(blk, x_img, x_txt, mi, mt, pe, n_img, n_txt)
    rows = []

    def codes_row(name, mine, ref, n_elems):
        (c, s), (rc, rs) = mine, ref
        nd = ndiff(c, rc)
        rows.append((name, f"codes differ {nd}/{n_elems}", f"scales differ {ndiff(s, rs)}/{s.numel()}",
                     f"max|dcode| {int((c.int() - rc.int()).abs().max()) if nd else 0}"))
        return nd + ndiff(s, rs)

    def float_row(name, mine, ref, ulps=False):
        nd = ndiff(mine, ref)
        extra = ""
        if ulps:  # distance in FP16 ulps (values are FP16 roundings)
            a = mine.half().view(torch.int16).int()
            b = ref.half().view(torch.int16).int()
            a = torch.where(a < 0, -32768 - a, a)
            b = torch.where(b < 0, -32768 - b, b)
            extra = f"max {int((a - b).abs().max())} FP16 ulp"
        rows.append((name, f"elements differ {nd}/{mine.numel()}", f"maxrel {maxrel(mine, ref):.3g}", extra))
        return nd

    bad = {}
    for tag, x, m in (("img", x_img, mi), ("txt", x_txt, mt)):
        bad[f"ln1_{tag}"] = codes_row(f"LN1+quant {tag}", Q.layer_norm_modulate_quantize(x, m[0].contiguous(),
                                                                                          m[1].contiguous()),
                                      (r[f"{tag}_c1"], r[f"{tag}_s1"]), x.numel())
    names = {"img": ("attn.to_q", "attn.to_k", "attn.to_v"),
             "txt": ("attn.add_q_proj", "attn.add_k_proj", "attn.add_v_proj")}
    for tag in ("img", "txt"):
        for k, n in enumerate(names[tag]):
            mine = Q.linear_i8(r[f"{tag}_c1"], r[f"{tag}_s1"], *lin(blk, n))
            bad[f"qkv_{tag}{k}"] = float_row(f"{n} {tag}", mine, r[f"{tag}_qkv"][k])
    qkv_i = torch.cat(r["img_qkv"], dim=1).contiguous()
    qkv_t = torch.cat(r["txt_qkv"], dim=1).contiguous()
    qkvh = Q.qk_norm_rope(qkv_i, qkv_t, norms(blk), pe[None])
    for k, key in enumerate(("qh", "kh", "vh")):
        bad[f"post_{key}"] = float_row(f"qk-norm+RoPE {key}", qkvh[k], r[key])
    mine_sq = Q.sage_quantize(r["qh"], r["kh"])
    ref_sq = R.sage_quantize(r["qh"], r["kh"])
    bad["sage_quant"] = sum(ndiff(a, b) for a, b in zip(mine_sq, ref_sq))
    rows.append(("Sage quant", f"differ {bad['sage_quant']}", "", ""))
    o_mine = Q.sage_attention(r["qh"], r["kh"], r["vh"], SM_SCALE)
    float_row("attention", o_mine, r["o"], ulps=True)
    post = {"img": ("attn.to_out.0", "img_mlp.net.0.proj", "img_mlp.net.2"),
            "txt": ("attn.to_add_out", "txt_mlp.net.0.proj", "txt_mlp.net.2")}
    for tag, x, m in (("img", x_img, mi), ("txt", x_txt, mt)):
        oo = r[f"o_{tag}"]
        bad[f"qo_{tag}"] = codes_row(f"quant_o {tag}", Q.fwht_quantize(oo, 1024), (r[f"{tag}_co"], r[f"{tag}_so"]),
                                     oo.numel())
        x2 = x.clone()
        Q.linear_i8(r[f"{tag}_co"], r[f"{tag}_so"], *lin(blk, post[tag][0]), epilogue=Q.EPI_RESIDUAL,
                    gate=m[2].contiguous(), out=x2)
        bad[f"out_{tag}"] = float_row(f"out-proj+gate {tag}", x2, r[f"{tag}_after_attn"])
        bad[f"ln2_{tag}"] = codes_row(f"LN2+quant {tag}",
                                      Q.layer_norm_modulate_quantize(r[f"{tag}_after_attn"], m[3].contiguous(),
                                                                     m[4].contiguous()),
                                      (r[f"{tag}_c2"], r[f"{tag}_s2"]), x.numel())
        h = Q.linear_i8(r[f"{tag}_c2"], r[f"{tag}_s2"], *lin(blk, post[tag][1]), epilogue=Q.EPI_GELU)
        bad[f"fc1_{tag}"] = float_row(f"fc1+GELU {tag}", h, r[f"{tag}_h"])
        bad[f"qh_{tag}"] = codes_row(f"quant_h {tag}", Q.fwht_quantize(r[f"{tag}_h"], 4096),
                                     (r[f"{tag}_ch"], r[f"{tag}_sh"]), r[f"{tag}_h"].numel())
        x3 = r[f"{tag}_after_attn"].clone()
        Q.linear_i8(r[f"{tag}_ch"], r[f"{tag}_sh"], *lin(blk, post[tag][2]), epilogue=Q.EPI_RESIDUAL,
                    gate=m[5].contiguous(), out=x3)
        bad[f"fc2_{tag}"] = float_row(f"fc2+gate {tag}", x3, r[f"{tag}_after_mlp"])
    print(f"\nblock 0 at {H}x{W}, {n_txt} text tokens: product stage on the reference's input of that stage")
    for row in rows:
        print("  {:<26} {:<34} {:<28} {}".format(*row))
    torch.cuda.synchronize()
    nonzero = {k: v for k, v in bad.items() if v}
    print("  stages not bit-exact:", nonzero or "none")
    assert not nonzero, nonzero


@pytest.mark.parametrize("H,W,n_txt,t,block", [(64, 64, 64, 500.0, b) for b in (0, 1, 30, 59)] +
                         [(166, 166, 256, 980.0, b) for b in (0, 59)])
def test_block_deviation_starts_at_attention(env, H, W, n_txt, t, block):
    """The product's whole block (qi_forward_blocks, its own modulation from
    the timestep) on the reference's input streams, against the reference's
    block, next to the reference's own stages fed the product's attention
    output (on the reference's Q/K/V).  The product's block equals that hybrid
    bit for bit: the attention output is where every difference of the block
    starts, and the block's deviation from the reference is what the
    reference's own arithmetic makes of an attention difference of at most
    5e-4 of the largest attention output."""
    cu, pe, n_img, x_img, x_txt, mi, mt = setup_case(env, H, W, n_txt, t, block)
    blk = env["blocks"][block % 2]
    r = ref_block(blk, x_img, x_txt, mi, mt, pe, n_img, n_txt)
    for key, ours in (("img_after_mlp", r["img_after_mlp"]), ("txt_after_mlp", r["txt_after_mlp"])):
        assert ndiff(ours, cu(f"b{block}_" + key, *ours.shape)) == 0, key
    img, tx = x_img.clone(), x_txt.clone()
    Q.forward_blocks(env["ctx"], env["model"], img, tx, t, pe[None], block, block + 1)
    env["ctx"].check()
    o_mine = Q.sage_attention(r["qh"], r["kh"], r["vh"], SM_SCALE)
    hybrid = ref_post_attention(blk, o_mine, x_img, x_txt, mi, mt, n_img, n_txt)
    out = {}
    for tag, mine in (("img", img), ("txt", tx)):
        ref = r[f"{tag}_after_mlp"]
        out[tag] = (maxrel(mine, ref), maxrel(hybrid[f"{tag}_after_mlp"], ref), ndiff(mine, hybrid[f"{tag}_after_mlp"]))
        print(f"block {block} {H}x{W} {tag}: product block maxrel {out[tag][0]:.4g}; reference block on the product's "
              f"attention output maxrel {out[tag][1]:.4g}; product vs that hybrid: {out[tag][2]} elements differ")
    for tag in ("img", "txt"):
        assert out[tag][2] == 0, (tag, out[tag])
