"""Op-level parity of the CUDA kernels (called through the C ABI) against the
reference's own CUDA build (oracle/_ref/libqiref.so) on identical device
inputs, and against exact host/torch arithmetic.

Bars: INT8 codes and scales bit-exact; INT32 accumulators exact; floating
point outputs within the stated tolerances (cosine similarity and normwise
max relative error max|a-b| / max|b|)."""
import numpy as np
import pytest
import torch

import qib200 as Q
import qi_oracle as O
import qi_ref as R

pytestmark = pytest.mark.gpu


def metrics(a, b):
    a = a.double().flatten()
    b = b.double().flatten()
    cos = float(a @ b / (a.norm() * b.norm() + 1e-300))
    maxrel = float((a - b).abs().max() / (b.abs().max() + 1e-300))
    return cos, maxrel


@pytest.fixture(scope="module", autouse=True)
def _device():
    torch.cuda.set_device(0)
    if not R.available():
        pytest.skip("reference build oracle/_ref/libqiref.so missing")
    yield
    torch.cuda.synchronize()


# ------------------------------------------------------------------ generator
@pytest.mark.parametrize("dtype,offset", [(torch.float32, 0.0), (torch.bfloat16, 0.0), (torch.bfloat16, 1.0)])
def test_synthetic_generator_identical_everywhere(dtype, offset):
    seed = Q.seed_for(3, "generator")
    assert seed == R.seed_for(3, "generator") == O.seed_for(3, "generator")
    a = Q.synth((1000, 37), seed, 0.02, offset, dtype=dtype)
    b = R.synth((1000, 37), seed, 0.02, offset, dtype=dtype)
    assert torch.equal(a.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       b.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
    if dtype == torch.bfloat16:
        c = O.gen_bf16(seed, (1000, 37), 0.02, offset)
        np.testing.assert_array_equal(a.view(torch.int16).cpu().numpy().view(np.uint16), c)
    else:
        np.testing.assert_array_equal(a.cpu().numpy(), O.gen_f32(seed, (1000, 37), 0.02, offset))


# ------------------------------------------------------------------ quantizers
@pytest.mark.parametrize("N,K", [(16, 3072), (8, 12288), (16, 256), (4, 64), (4, 3584), (3072, 3072), (1, 128)])
def test_weight_quantizer_bitexact(N, K):
    w = Q.synth((N, K), Q.seed_for(12, f"w_{N}_{K}"), 0.02, dtype=torch.bfloat16)
    c, s = Q.quantize_weight(w)
    rc, rs = R.quantize_weight(w)
    assert torch.equal(c, rc)
    assert torch.equal(s.view(torch.int32), rs.view(torch.int32))


def _act(M, K, seed, scale=1.0):
    x = Q.synth((M, K), seed, scale)
    if M > 0:
        x[0] = 0.0
    if M > 1:
        x[1, 7] *= 1000.0
    if M > 2:
        x[2] = 1e-39  # subnormal row: flushed to zero like the reference (fast math)
    if M > 3:
        x[3, 5] = float("nan")  # NaN: the reference's max ignores it, its code is 0
    if M > 4:
        x[4, 9] = float("inf")  # infinite element (and the NaNs the transform makes of it)
    if M > 5:
        x[5] = 0.0
        x[5, 3] = 1e-36  # tiny maximum: 127 / max overflows to infinity
    if M > 6:
        x[6] = -0.0
    return x


@pytest.mark.parametrize("M,K,B", [(8, 3072, 1024), (4, 12288, 4096), (3, 256, 256), (5, 3584, 512),
                                   (1, 3072, 1024), (300, 3072, 1024), (129, 12288, 4096), (7, 3072, 1),
                                   (6, 3072, 512), (2, 12288, 1024)])
def test_activation_quantizer_bitexact(M, K, B):
    x = _act(M, K, Q.seed_for(11, f"act_{M}_{K}"))
    c, s = Q.fwht_quantize(x, B)
    rc, rs = R.fwht_quantize(x, B)
    assert torch.equal(c, rc)
    assert torch.equal(s.view(torch.int32), rs.view(torch.int32))


# ------------------------------------------------------------------ GEMM
# the last three shapes (M >= 512, K >= 8192) run on CTA pairs (256-row tiles),
# with M not a multiple of 256 and N not a multiple of the 256-column tile
@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (100, 256, 3072), (128, 3072, 3072), (300, 96, 3072),
                                   (1000, 9216, 3072), (257, 3072, 12288), (64, 512, 64), (513, 12288, 3072),
                                   (1000, 3072, 12288), (700, 544, 8192), (512, 256, 8192)])
def test_gemm_int32_accumulators_exact(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-128, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
    ones_m = torch.ones(M, device="cuda")
    ones_n = torch.ones(N, device="cuda")
    out = Q.linear_i8(a, ones_m, w, ones_n)
    exact = (a.double() @ w.double().T).float()  # |acc| < 2^31 < 2^53: exact, then RN to float
    assert torch.equal(out, exact)


@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("M,N,K", [(77, 3072, 3072), (512, 12288, 3072), (300, 3072, 12288)])
def test_linear_dequant_matches_reference(M, N, K, gelu):
    x = Q.synth((M, K), Q.seed_for(21, f"x_{M}_{N}_{K}"), 1.0)
    w = Q.synth((N, K), Q.seed_for(21, f"w_{M}_{N}_{K}"), 0.02, dtype=torch.bfloat16)
    b = Q.synth((N,), Q.seed_for(21, f"b_{M}_{N}_{K}"), 0.02, dtype=torch.bfloat16)
    wc, ws = Q.quantize_weight(w)
    ac, asc = Q.fwht_quantize(x)
    ours = Q.linear_i8(ac, asc, wc, ws, b, Q.EPI_GELU if gelu else Q.EPI_STORE)
    ref = R.linear_int8_preq(ac, asc, wc, ws, b, gelu)
    cos, maxrel = metrics(ours, ref)
    assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)
    # full FP32-input path (FWHT + quantize + GEMM + dequant), incl. M == 1
    ref2 = R.linear_int8(x, wc, ws, b, gelu)
    ours2 = Q.linear_i8_f32in(x, wc, ws, b, gelu)
    cos, maxrel = metrics(ours2, ref2)
    assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)
    if not gelu:
        r1 = R.linear_int8(x[:1].contiguous(), wc, ws, b, False)
        o1 = Q.linear_i8_f32in(x[:1].contiguous(), wc, ws, b, False)
        cos, maxrel = metrics(o1, r1)
        assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)


@pytest.mark.parametrize("M,N,K", [(200, 3072, 3072), (900, 3072, 12288)])  # second: CTA pairs
def test_linear_residual_epilogue(M, N, K):
    x = Q.synth((M, K), Q.seed_for(22, f"x{K}"), 1.0)
    w = Q.synth((N, K), Q.seed_for(22, f"w{K}"), 0.02, dtype=torch.bfloat16)
    b = Q.synth((N,), Q.seed_for(22, f"b{K}"), 0.02, dtype=torch.bfloat16)
    gate = Q.synth((N,), Q.seed_for(22, f"g{K}"), 0.5)
    resid = Q.synth((M, N), Q.seed_for(22, f"r{K}"), 3.0)
    wc, ws = Q.quantize_weight(w)
    ac, asc = Q.fwht_quantize(x)
    y = R.linear_int8_preq(ac, asc, wc, ws, b, False)
    expect = resid + gate[None, :] * y  # gate_add_fp32f (cuda_kernels.cu:2181)
    out = resid.clone()
    Q.linear_i8(ac, asc, wc, ws, b, Q.EPI_RESIDUAL, gate, out=out)
    cos, maxrel = metrics(out, expect)
    assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)


# ------------------------------------------------------------------ Sage
@pytest.mark.parametrize("BH,S", [(2, 200), (1, 77), (2, 384), (48, 1088), (3, 4352), (1, 1), (64, 257), (200, 131)])
def test_sage_quantizers_bitexact(BH, S):
    q = Q.synth((BH, S, 128), Q.seed_for(13, f"q_{BH}_{S}"), 1.0).half()
    k = Q.synth((BH, S, 128), Q.seed_for(13, f"k_{BH}_{S}"), 1.0).half()
    ours = Q.sage_quantize(q, k)
    ref = R.sage_quantize(q, k)
    names = ["kmean", "qc", "qs", "kc", "ks"]
    for n, a, b in zip(names, ours, ref):
        if a.dtype == torch.float32:
            assert torch.equal(a.view(torch.int32), b.view(torch.int32)), n
        else:
            assert torch.equal(a, b), n


# (2, 16896): the joint sequence of a 2048x2048 image (16384 image + 512 text tokens)
@pytest.mark.parametrize("BH,S", [(2, 200), (1, 77), (2, 384), (4, 1088), (2, 4352), (1, 129), (1, 1), (2, 16896)])
def test_sage_attention_matches_reference_and_exact(BH, S):
    q = Q.synth((BH, S, 128), Q.seed_for(14, f"q_{BH}_{S}"), 1.0).half()
    k = Q.synth((BH, S, 128), Q.seed_for(14, f"k_{BH}_{S}"), 1.0).half()
    v = Q.synth((BH, S, 128), Q.seed_for(14, f"v_{BH}_{S}"), 1.0).half()
    scale = 1.0 / np.sqrt(128.0)
    ours = Q.sage_attention(q, k, v, scale)
    ref = R.sage_attention(q, k, v, scale)
    cos, maxrel = metrics(ours, ref)
    assert cos > 0.9999 and maxrel < 1e-2, (cos, maxrel)
    exact = torch.softmax((q.float() @ k.float().transpose(1, 2)) * scale, dim=-1) @ v.float()
    cos_e, maxrel_e = metrics(ours, exact)
    cos_r, maxrel_r = metrics(ref, exact)
    assert cos_e > 0.999 and maxrel_e < 2e-2, (cos_e, maxrel_e)
    assert cos_e >= cos_r - 1e-4, (cos_e, cos_r)


def test_sage_attention_large_logits():
    # Q/K scaled up so rows have a dominant key: exercises the online rescale.
    BH, S = 2, 1000
    q = (Q.synth((BH, S, 128), Q.seed_for(15, "q"), 4.0)).half()
    k = (Q.synth((BH, S, 128), Q.seed_for(15, "k"), 4.0)).half()
    v = Q.synth((BH, S, 128), Q.seed_for(15, "v"), 1.0).half()
    scale = 1.0 / np.sqrt(128.0)
    ours = Q.sage_attention(q, k, v, scale)
    ref = R.sage_attention(q, k, v, scale)
    cos, maxrel = metrics(ours, ref)
    assert cos > 0.999 and maxrel < 2e-2, (cos, maxrel)


@pytest.mark.parametrize("zero", ["q", "k", "v"])
def test_sage_attention_degenerate_heads(zero):
    """An all-zero Q (or K) head gives uniform attention over the valid keys
    (tiny scales must not let masked keys in); a zero V head gives zeros."""
    BH, S = 3, 300  # S not a multiple of the 128-key block
    q = Q.synth((BH, S, 128), Q.seed_for(16, "q"), 1.0).half()
    k = Q.synth((BH, S, 128), Q.seed_for(16, "k"), 1.0).half()
    v = Q.synth((BH, S, 128), Q.seed_for(16, "v"), 1.0).half()
    {"q": q, "k": k, "v": v}[zero][1].zero_()
    scale = 1.0 / np.sqrt(128.0)
    ours = Q.sage_attention(q, k, v, scale)
    ref = R.sage_attention(q, k, v, scale)
    cos, maxrel = metrics(ours, ref)
    assert cos > 0.9999 and maxrel < 1e-2, (cos, maxrel)
    if zero == "v":
        assert torch.equal(ours[1], torch.zeros_like(ours[1]))
    else:
        uniform = v[1].float().mean(0, keepdim=True).expand(S, 128)
        assert (ours[1] - uniform).abs().max() < 2e-3


# ------------------------------------------------------------------ norms
def test_layer_norm_modulate_matches_reference():
    x = Q.synth((333, 3072), Q.seed_for(16, "x"), 2.0) + 0.5
    sh = Q.synth((3072,), Q.seed_for(16, "sh"), 0.1)
    sc = Q.synth((3072,), Q.seed_for(16, "sc"), 0.1)
    cos, maxrel = metrics(Q.layer_norm_modulate(x, sh, sc), R.layer_norm_modulate(x, sh, sc))
    assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)


def test_rms_norm_matches_reference():
    x = Q.synth((24 * 100, 128), Q.seed_for(17, "x"), 3.0)
    w = Q.synth((128,), Q.seed_for(17, "w"), 0.02, 1.0, dtype=torch.bfloat16)
    cos, maxrel = metrics(Q.rms_norm(x, w), R.rms_norm(x, w))
    assert cos > 0.999999 and maxrel < 1e-5, (cos, maxrel)


@pytest.mark.parametrize("h,w,n_txt", [(8, 8, 8), (166, 166, 256), (256, 256, 512), (7, 9, 5)])
def test_rope_table_bitexact(h, w, n_txt):
    np.testing.assert_array_equal(Q.rope_table(h, w, n_txt), R.rope_table(h, w, n_txt))
