"""qi_linear_i8_f32in_noalloc (the allocation-free FP32-input W8A8 linear,
scratch in a fixed device array) against qi_linear_i8_f32in, through the C
ABI.  Named to be collected last, so it runs both after every other test and,
when given alone, in a fresh process."""
import ctypes

import pytest
import torch

import qib200 as Q

pytestmark = pytest.mark.gpu

QI_ERR_ARG = 1
QI_ERR_UNSUPPORTED = 5
QI_ERR_DEVICE = 7
MAX_ROWS = 4096
MAX_CODES = 4 * 1024 * 1024


def metrics(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    cos = float(a @ b / (a.norm() * b.norm()))
    maxrel = float((a - b).abs().max() / b.abs().max())
    return cos, maxrel


def case(M, K, N, tag):
    x = Q.synth((M, K), Q.seed_for(41, f"x_{tag}"), 1.0)
    w = Q.synth((N, K), Q.seed_for(41, f"w_{tag}"), 0.02, dtype=torch.bfloat16)
    b = Q.synth((N,), Q.seed_for(41, f"b_{tag}"), 0.02, dtype=torch.bfloat16)
    wc, ws = Q.quantize_weight(w)
    return x, wc, ws, b


def noalloc(x, wc, ws, b, gelu, out):
    M, K = x.shape
    N = wc.shape[0]
    return Q.lib().qi_linear_i8_f32in_noalloc(Q._p(x), M, K, Q._p(wc), Q._p(ws), N, Q._p(b), int(gelu), Q._p(out),
                                              Q._stream())


def test_noalloc_matches_existing_entry_two_calls_in_a_row():
    torch.cuda.set_device(0)
    shapes = [(77, 3072, 3072, False), (300, 12288, 3072, True), (1365, 3072, 3072, True), (1, 3072, 3072, False)]
    cases = [case(M, K, N, f"{M}_{K}_{N}") for M, K, N, _ in shapes]
    expected = [Q.linear_i8_f32in(x, wc, ws, b, g) for (x, wc, ws, b), (_, _, _, g) in zip(cases, shapes)]
    outs = [torch.full_like(e, float("nan")) for e in expected]
    n_first = Q.lib().qi_alloc_count()  # the first calls, with their set-up, allocate nothing either
    # two calls in a row on one stream, no synchronisation between them
    for pair in ((0, 1), (2, 3)):
        for i in pair:
            x, wc, ws, b = cases[i]
            Q.check(noalloc(x, wc, ws, b, shapes[i][3], outs[i]))
        torch.cuda.synchronize()
    assert Q.lib().qi_alloc_count() == n_first
    for o, e in zip(outs, expected):
        cos, maxrel = metrics(o, e)
        assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)
    # the library counts every CUDA allocation it makes: none in these calls
    # (the first one above included); the device's free memory is a second,
    # coarser signal
    again = [torch.full_like(e, float("nan")) for e in expected[:2]]
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    n0 = Q.lib().qi_alloc_count()
    for i in (0, 1):
        x, wc, ws, b = cases[i]
        Q.check(noalloc(x, wc, ws, b, shapes[i][3], again[i]))
    torch.cuda.synchronize()
    assert Q.lib().qi_alloc_count() == n0
    assert torch.cuda.mem_get_info()[0] == free0
    for a, o in zip(again, outs[:2]):
        assert torch.equal(a, o)
    assert Q.lib().qi_linear_i8_f32in_noalloc_check() == 0


def test_noalloc_rejects_requests_beyond_its_scratch():
    torch.cuda.set_device(0)
    for M, K in ((MAX_ROWS + 1, 256), (MAX_CODES // 12288 + 1, 12288)):
        x, wc, ws, b = case(M, K, 64, f"big_{M}_{K}")
        out = torch.full((M, 64), 7.0, device="cuda")
        assert noalloc(x, wc, ws, b, False, out) == QI_ERR_UNSUPPORTED
        torch.cuda.synchronize()
        assert bool((out == 7.0).all())
    null = ctypes.c_void_p(0)
    assert Q.lib().qi_linear_i8_f32in_noalloc(null, 4, 256, null, null, 64, null, 0, null, null) == QI_ERR_ARG


def test_noalloc_reports_a_timed_out_wait():
    """A GEMM wait that gives up leaves its mark in the scratch's error word;
    qi_linear_i8_f32in_noalloc_check reports it once and clears it, and the
    entry keeps working afterwards."""
    torch.cuda.set_device(0)
    L = Q.lib()
    assert L.qi_linear_i8_f32in_noalloc_check() == 0
    n0 = L.qi_alloc_count()
    Q.check(L.qi_linear_i8_f32in_noalloc_selftest(2000, Q._stream()))
    assert L.qi_linear_i8_f32in_noalloc_check() == QI_ERR_DEVICE
    assert L.qi_linear_i8_f32in_noalloc_check() == 0
    x, wc, ws, b = case(64, 3072, 3072, "after_timeout")
    out = torch.empty(64, 3072, device="cuda")
    Q.check(noalloc(x, wc, ws, b, False, out))
    assert L.qi_linear_i8_f32in_noalloc_check() == 0
    assert L.qi_alloc_count() == n0
    cos, maxrel = metrics(out, Q.linear_i8_f32in(x, wc, ws, b, False))
    assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)
