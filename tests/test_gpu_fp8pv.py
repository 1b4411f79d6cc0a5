"""The FP8 P.V SageAttention variant (qi_sage_attention_fp8pv: per-block Q/K
INT8 scales, V and P as E4M3 codes, P.V on tcgen05 kind::f8f6f4) against exact
attention softmax(Q K^T / sqrt(128)) V evaluated in FP32 from the same FP16
Q, K, V.  The reference ships this scheme's FP8 building blocks but launches
only its FP16 P.V kernel, so the check is against exact attention, at the
Sage microbenchmark configuration (2 x 24 heads, 4096 + 256 tokens) and at
short and ragged lengths.  Bar: cosine >= 0.999 and max|a-b| / max|b| <= 6e-2.
The element-wise bound is looser than the FP16 P.V kernel's: E4M3 keeps 3
mantissa bits, so every P and V code carries up to 2^-4 relative rounding
error (measured 3.5e-2 .. 5.0e-2 here, against 0.96e-2 .. 1.4e-2 for FP16
P.V on the same inputs); the variant is off by default."""
import numpy as np
import pytest
import torch

import qib200 as Q

pytestmark = pytest.mark.gpu


def exact(q, k, v, scale):
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for h in range(q.shape[0]):
        s = (q[h].float() @ k[h].float().T) * scale
        out[h] = torch.softmax(s, dim=-1) @ v[h].float()
    return out


def metrics(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    return float(a @ b / (a.norm() * b.norm())), float((a - b).abs().max() / b.abs().max())


@pytest.mark.parametrize("BH,S", [(48, 4352), (4, 1000), (2, 77), (3, 129), (1, 7145)])
def test_fp8pv_matches_exact_attention(BH, S):
    torch.cuda.set_device(0)
    q = Q.synth((BH, S, 128), Q.seed_for(61, f"q{BH}_{S}"), 1.0).half()
    k = Q.synth((BH, S, 128), Q.seed_for(61, f"k{BH}_{S}"), 1.0).half()
    v = Q.synth((BH, S, 128), Q.seed_for(61, f"v{BH}_{S}"), 1.0).half()
    scale = 1.0 / np.sqrt(128.0)
    ref = exact(q, k, v, scale)
    o8 = Q.sage_attention_fp8pv(q, k, v, scale)
    o16 = Q.sage_attention(q, k, v, scale)
    torch.cuda.synchronize()
    c8, m8 = metrics(o8, ref)
    c16, m16 = metrics(o16, ref)
    print(f"BH={BH} S={S}: FP8 P.V cos={c8:.6f} maxrel={m8:.4g} | FP16 P.V cos={c16:.6f} maxrel={m16:.4g}")
    assert torch.isfinite(o8).all()
    assert c8 >= 0.999 and m8 <= 6e-2, (c8, m8)


def test_fp8pv_rejects_other_head_dims():
    z = torch.zeros(1, 8, 64, dtype=torch.float16, device="cuda")
    out = torch.zeros(1, 8, 64, device="cuda")
    assert Q.lib().qi_sage_attention_fp8pv(Q._p(z), Q._p(z), Q._p(z), Q._p(out), 0.1, 1, 8, 64, Q._stream()) == 5


def test_forward_with_fp8pv_attention():
    """qi_ctx_set_attention_fp8pv switches the forward's attention to the FP8
    P.V variant: a one-block model at 64x64 against the CPU oracle's FP32
    (unquantized) evaluation, next to the default FP16 P.V forward."""
    import qi_oracle as O
    torch.cuda.set_device(0)
    g, blocks = Q.make_weight_table(1, base_seed=0)
    ctx = Q.Context(0)
    model = Q.Model(ctx, g, blocks)
    H = W = 64
    n_txt = 64
    xs = O.gen_bf16(O.seed_for(1, "latent"), (1, 16, H, W), 1.0)
    ts = O.gen_bf16(O.seed_for(1, "context"), (n_txt, 3584), 1.0)
    pe = O.rope_table(H, W, n_txt)
    x = torch.from_numpy(xs.view(np.int16)).cuda().view(torch.bfloat16)
    txt = torch.from_numpy(ts.view(np.int16)).cuda().view(torch.bfloat16)[None]
    pe_d = torch.from_numpy(pe).cuda()[None]
    y16 = Q.forward(ctx, model, x, 500.0, txt, pe_d).float().cpu()
    Q.check(Q.lib().qi_ctx_set_attention_fp8pv(ctx.h, 1))
    y8 = Q.forward(ctx, model, x, 500.0, txt, pe_d).float().cpu()
    Q.check(Q.lib().qi_ctx_set_attention_fp8pv(ctx.h, 0))
    ctx.check()
    ref = torch.from_numpy(O.forward(O.Weights(1, base_seed=0), xs, 500.0, ts, pe, mode="fp32"))
    c8, m8 = metrics(y8, ref)
    c16, m16 = metrics(y16, ref)
    print(f"one-block forward vs FP32 oracle: FP8 P.V cos={c8:.6f} maxrel={m8:.4g} | FP16 P.V cos={c16:.6f} "
          f"maxrel={m16:.4g}")
    assert c8 >= 0.999, c8
    assert m8 <= 2 * m16 + 1e-2, (m8, m16)
    model.close()
    ctx.close()
