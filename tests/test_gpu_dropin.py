"""The drop-in boundary: the reference's caller-side code (TransformerWeights
built from device tensors, then transformer_forward, oracle/ref_driver.cu)
linked against the product's shim (qwen-image.cu_b200/shim/transformer_b200.cpp)
instead of the reference's transformer.cu, i.e. exactly what main.cu links
against (main.cu:761, 771).  It must reproduce qi_forward bit for bit (same
kernels, same inputs) and the reference within the north-star tolerance."""
import ctypes
import os

import pytest
import torch

import qib200 as Q
import qi_ref as R

pytestmark = pytest.mark.gpu

SHIM = os.path.join(os.path.dirname(R.LIB_PATH), "libshimtest.so")


def test_shim_forward_through_reference_types():
    if not (R.available() and os.path.exists(SHIM)):
        pytest.skip("reference / shim test build missing")
    torch.cuda.set_device(0)
    shim = ctypes.CDLL(SHIM)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    shim.ref_transformer_forward.argtypes = [vp, vp, vp, f, vp, i, vp, i, i, i, vp]
    shim.ref_transformer_forward.restype = i
    g, blocks = R.make_table(60, distinct=2)
    garr, _, bt = R.table_pointers(g, blocks)
    H, W, n_txt, t = 32, 30, 20, 700.0
    x = R.synth((1, 16, H, W), R.seed_for(4, "latent"), 1.0, dtype=torch.bfloat16)
    txt = R.synth((1, n_txt, 3584), R.seed_for(4, "context"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(R.rope_table(H, W, n_txt)).cuda()
    out = torch.empty_like(x)
    p = lambda t_: ctypes.c_void_p(t_.data_ptr())
    assert shim.ref_transformer_forward(garr, bt, p(x), t, p(txt), n_txt, p(pe), H, W, 1, p(out)) == 0
    ctx = Q.Context(0)
    model = Q.Model(ctx, g, blocks)
    ours = Q.forward(ctx, model, x, t, txt, pe[None])
    assert torch.equal(out, ours)
    ref = R.transformer_forward(garr, bt, x, t, txt, pe, H, W, sage=True)
    a, b = out.double().flatten(), ref.double().flatten()
    cos = float(a @ b / (a.norm() * b.norm()))
    assert cos >= 0.999, cos
    # odd latent sizes go through the shim's pad / crop (transformer.cu:266-290, 915-922)
    H2, W2 = 31, 29
    x2 = R.synth((1, 16, H2, W2), R.seed_for(5, "latent"), 1.0, dtype=torch.bfloat16)
    pe2 = torch.from_numpy(R.rope_table(H2, W2, n_txt)).cuda()
    out2 = torch.empty_like(x2)
    assert shim.ref_transformer_forward(garr, bt, p(x2), t, p(txt), n_txt, p(pe2), H2, W2, 1, p(out2)) == 0
    ref2 = R.transformer_forward(garr, bt, x2, t, txt, pe2, H2, W2, sage=True)
    a, b = out2.double().flatten(), ref2.double().flatten()
    assert float(a @ b / (a.norm() * b.norm())) >= 0.999
    model.close()
    ctx.close()


def test_shim_reports_sage_substitution(capfd):
    """use_sage_attention = false asks for the reference's materialised-softmax
    attention; the shim runs its SageAttention kernels instead and says so on
    stderr (once per process)."""
    if not (R.available() and os.path.exists(SHIM)):
        pytest.skip("reference / shim test build missing")
    torch.cuda.set_device(0)
    shim = ctypes.CDLL(SHIM)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    shim.ref_transformer_forward.argtypes = [vp, vp, vp, f, vp, i, vp, i, i, i, vp]
    shim.ref_transformer_forward.restype = i
    g, blocks = R.make_table(60, distinct=1)
    garr, _, bt = R.table_pointers(g, blocks)
    H, W, n_txt, t = 16, 16, 12, 650.0
    x = R.synth((1, 16, H, W), R.seed_for(6, "latent"), 1.0, dtype=torch.bfloat16)
    txt = R.synth((1, n_txt, 3584), R.seed_for(6, "context"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(R.rope_table(H, W, n_txt)).cuda()
    p = lambda t_: ctypes.c_void_p(t_.data_ptr())
    a, b = torch.empty_like(x), torch.empty_like(x)
    assert shim.ref_transformer_forward(garr, bt, p(x), t, p(txt), n_txt, p(pe), H, W, 1, p(a)) == 0
    capfd.readouterr()
    assert shim.ref_transformer_forward(garr, bt, p(x), t, p(txt), n_txt, p(pe), H, W, 0, p(b)) == 0
    assert shim.ref_transformer_forward(garr, bt, p(x), t, p(txt), n_txt, p(pe), H, W, 0, p(b)) == 0
    err = capfd.readouterr().err
    assert err.count("use_sage_attention = false requested") == 1, err
    assert torch.equal(a, b)
    # a new weights object (other tensors) in the same process: the shim
    # rebuilds its model instead of reusing the one of the test above
    ctx = Q.Context(0)
    model = Q.Model(ctx, g, blocks)
    assert torch.equal(a, Q.forward(ctx, model, x, t, txt, pe[None]))
    model.close()
    ctx.close()
