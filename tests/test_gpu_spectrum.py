"""Spectrum step skipping on the GPU: the forecaster (qi_spectrum_*) against
the reference's own spectrum_predict (oracle/_ref, cuda_kernels.cu:6268-6333)
and the float64 oracle; the forward's hidden-state capture and the output
head (qi_spectrum_output) against qi_forward itself (bit for bit: same
kernels) and against the reference's transformer_spectrum_output
(transformer.cu:939-1028); and both through the drop-in shim, as main.cu's
--spectrum schedule calls them (main.cu:660-683, 761-773, 877-879).

Bars: the forecaster's prediction within 1e-5 (oracle) / 1e-4 (reference's
FP32 solve) of the largest predicted value; the output head, which ends in a
BF16 GEMM and BF16 output, within cosine 0.9999 and max-rel 2e-2 of the
reference's on the same hidden state."""
import ctypes
import os

import numpy as np
import pytest
import torch

import qi_oracle as O
import qi_ref as R
import qib200 as Q

pytestmark = pytest.mark.gpu

SHIM = os.path.join(os.path.dirname(R.LIB_PATH), "libshimtest.so")
# Against the reference: order 4 (the reference fits T_0..T_4 whatever order it
# is given; below 4 its buffers are too small, so it is never run there)
CASES = [
    ([5, 6], 7, 4, 0.1, 1.0),
    ([5, 7, 9, 11, 13, 15], 16, 4, 0.1, 1.0),
    ([0, 1, 2, 3, 4, 5, 7, 9, 11, 13, 15, 17], 18, 4, 0.1, 0.5),
    (list(range(5, 45, 2)), 46, 4, 0.01, 0.75),
    ([10, 12, 14, 16, 18, 20, 22, 24], 23, 4, 1.0, 0.0),
]
# The library at other orders, against the oracle only
ORDER_CASES = [(list(range(5, 45, 2)), 46, 6, 0.01, 0.75), ([10, 12, 14, 16, 18, 20, 22, 24], 23, 3, 1.0, 0.25),
               ([3, 4, 5, 6, 7], 9, 0, 0.1, 1.0)]
F = 64 * 3072  # 64 image tokens x 3072


def metrics(a, b):
    a, b = a.double().flatten(), b.double().flatten()
    cos = float(a @ b / (a.norm() * b.norm() + 1e-300))
    return cos, float((a - b).abs().max() / (b.abs().max() + 1e-300))


@pytest.fixture(scope="module", autouse=True)
def _device():
    torch.cuda.set_device(0)
    if not R.available():
        pytest.skip("reference build oracle/_ref/libqiref.so missing")
    yield
    torch.cuda.synchronize()


@pytest.mark.parametrize("steps,target,order,lam,blend", CASES)
def test_predict_matches_reference_and_oracle(steps, target, order, lam, blend):
    K = len(steps)
    hist = R.synth((K, F), R.seed_for(32, f"spectrum_{K}_{order}"), 1.0)
    sp = Q.Spectrum(F, max_history=K, order=order, lam=lam)
    for k in range(K):
        sp.update(hist[k], steps[k])
    assert sp.history() == K
    ours = sp.predict(target, blend, like=hist[0])
    ref = R.spectrum_predict(hist, steps, target, blend, order, lam)
    ora = torch.from_numpy(O.spectrum_predict(hist.cpu().double().numpy(), steps, target,
                                              float(np.float32(blend)), order, float(np.float32(lam))))
    scale = float(ora.abs().max())
    assert float((ours.cpu().double() - ora).abs().max()) <= 1e-5 * scale
    assert float((ours.double() - ref.double()).abs().max()) <= 1e-4 * scale
    sp.close()


@pytest.mark.parametrize("steps,target,order,lam,blend", ORDER_CASES)
def test_predict_other_orders_match_oracle(steps, target, order, lam, blend):
    K = len(steps)
    hist = R.synth((K, F), R.seed_for(36, f"order_{K}_{order}"), 1.0)
    sp = Q.Spectrum(F, max_history=K, order=order, lam=lam)
    for k in range(K):
        sp.update(hist[k], steps[k])
    ours = sp.predict(target, blend, like=hist[0])
    ora = torch.from_numpy(O.spectrum_predict(hist.cpu().double().numpy(), steps, target,
                                              float(np.float32(blend)), order, float(np.float32(lam))))
    assert float((ours.cpu().double() - ora).abs().max()) <= 1e-5 * float(ora.abs().max())
    sp.close()


def test_reference_fits_order_4_whatever_it_is_given():
    """Documents the reference's behaviour: spectrum_init does not keep its
    max_order argument, so asked for order 6 the reference returns the order-4
    prediction (run only above 4, where its buffers are large enough)."""
    steps, target = list(range(5, 45, 2)), 46
    hist = R.synth((len(steps), F), R.seed_for(37, "order6"), 1.0)
    ref6 = R.spectrum_predict(hist, steps, target, 0.75, 6, 0.01)
    sp = Q.Spectrum(F, max_history=len(steps), order=4, lam=0.01)
    for k, s in enumerate(steps):
        sp.update(hist[k], s)
    ours4 = sp.predict(target, 0.75, like=hist[0])
    assert float((ours4 - ref6).abs().max()) <= 1e-4 * float(ref6.abs().max())
    sp.close()


def test_history_keeps_the_latest_states():
    steps = list(range(10, 26, 2))  # 8 states into a history of 5
    hist = R.synth((len(steps), F), R.seed_for(33, "ring"), 1.0)
    sp = Q.Spectrum(F, max_history=5, order=4, lam=0.1)
    for k, s in enumerate(steps):
        sp.update(hist[k], s)
    assert sp.history() == 5
    ours = sp.predict(25, 0.5, like=hist[0])
    ref = R.spectrum_predict(hist[-5:].contiguous(), steps[-5:], 25, 0.5, 4, 0.1)
    assert float((ours - ref).abs().max()) <= 1e-4 * float(ref.abs().max())
    with pytest.raises(Q.QIError):
        sp.update(hist[0], 24)  # steps must increase
    sp.reset()
    assert sp.history() == 0
    with pytest.raises(Q.QIError):
        sp.predict(26, like=hist[0])
    sp.close()


def _setup(H, W, n_txt, seed):
    g, blocks = R.make_table(60, distinct=1)
    garr, _, bt = R.table_pointers(g, blocks)
    x = R.synth((1, 16, H, W), R.seed_for(seed, "latent"), 1.0, dtype=torch.bfloat16)
    txt = R.synth((1, n_txt, 3584), R.seed_for(seed, "context"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(R.rope_table(H, W, n_txt)).cuda()
    return g, blocks, garr, bt, x, txt, pe


def test_capture_and_output_head():
    H, W, n_txt, t = 16, 16, 12, 640.0
    g, blocks, garr, bt, x, txt, pe = _setup(H, W, n_txt, 34)
    ctx = Q.Context(0)
    model = Q.Model(ctx, g, blocks)
    hidden = torch.empty((H // 2) * (W // 2), 3072, device="cuda")
    ctx.set_hidden_capture(hidden)
    out = Q.forward(ctx, model, x, t, txt, pe[None])
    ctx.set_hidden_capture(None)
    # the head on the captured state is the forward's own tail
    head = Q.spectrum_output(ctx, model, hidden, t, H, W)
    assert torch.equal(head, out)
    # against the reference: its captured state, and its head on the same state
    ref_out, ref_hidden = R.transformer_forward_capture(garr, bt, x, t, txt, pe, H, W, sage=True)
    cos, _ = metrics(hidden, ref_hidden)
    assert cos >= 0.999, cos
    ours = Q.spectrum_output(ctx, model, ref_hidden, t, H, W)
    ref = R.transformer_spectrum_output(garr, bt, ref_hidden, t, H, W)
    cos, maxrel = metrics(ours, ref)
    assert cos >= 0.9999 and maxrel <= 2e-2, (cos, maxrel)
    model.close()
    ctx.close()


def test_spectrum_through_the_shim():
    if not os.path.exists(SHIM):
        pytest.skip("shim test build missing")
    shim = ctypes.CDLL(SHIM)
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    shim.ref_transformer_forward_capture.argtypes = [vp, vp, vp, f, vp, i, vp, i, i, i, vp, vp]
    shim.ref_transformer_forward_capture.restype = i
    shim.ref_transformer_spectrum_output.argtypes = [vp, vp, vp, f, i, i, vp]
    shim.ref_transformer_spectrum_output.restype = i
    p = lambda t_: ctypes.c_void_p(t_.data_ptr())
    H, W, n_txt, t = 16, 16, 12, 610.0
    g, blocks, garr, bt, x, txt, pe = _setup(H, W, n_txt, 35)
    out = torch.empty_like(x)
    hidden = torch.empty((H // 2) * (W // 2), 3072, device="cuda")
    assert shim.ref_transformer_forward_capture(garr, bt, p(x), t, p(txt), n_txt, p(pe), H, W, 1, p(out),
                                                p(hidden)) == 0
    head = torch.empty_like(x)
    assert shim.ref_transformer_spectrum_output(garr, bt, p(hidden), t, H, W, p(head)) == 0
    assert torch.equal(head, out)
    ctx = Q.Context(0)
    model = Q.Model(ctx, g, blocks)
    assert torch.equal(Q.spectrum_output(ctx, model, hidden, t, H, W), head)
    # odd latent sizes: the shim pads to the patch size and crops, as the reference does
    H2, W2 = 15, 17
    n2 = ((H2 + 1) // 2) * ((W2 + 1) // 2)
    hid2 = R.synth((n2, 3072), R.seed_for(35, "hidden"), 1.0)
    ours2 = torch.empty(1, 16, H2, W2, dtype=torch.bfloat16, device="cuda")
    assert shim.ref_transformer_spectrum_output(garr, bt, p(hid2), t, H2, W2, p(ours2)) == 0
    ref2 = R.transformer_spectrum_output(garr, bt, hid2, t, H2, W2)
    cos, maxrel = metrics(ours2, ref2)
    assert cos >= 0.9999 and maxrel <= 2e-2, (cos, maxrel)
    model.close()
    ctx.close()
