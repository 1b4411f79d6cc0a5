"""CPU oracle self-checks (no GPU): the generator, the Walsh-Hadamard
quantizers, the exact INT8 GEMM, the Sage emulation against exact attention,
and agreement of the oracle's quantization-emulating and FP32 modes."""
import numpy as np
import pytest

import qi_oracle as O


def test_generator_deterministic_and_unit_variance():
    a = O.gen_f32(7, (1 << 18,))
    b = O.gen_f32(7, (1 << 18,))
    np.testing.assert_array_equal(a, b)
    assert abs(float(a.mean())) < 0.01 and abs(float(a.std()) - 1.0) < 0.01
    assert float(np.abs(a).max()) <= 3.47
    c = O.gen_f32(8, (1 << 18,))
    assert not np.array_equal(a, c)
    w = O.bf16_to_f32(O.gen_bf16(9, (4096,), 0.02, 1.0))
    assert abs(float(w.mean()) - 1.0) < 0.002


def test_seed_for_distinguishes_names():
    s = {O.seed_for(0, f"transformer_blocks.{i}.attn.to_q.weight") for i in range(60)}
    assert len(s) == 60
    assert O.seed_for(0, "x") != O.seed_for(1, "x")


@pytest.mark.parametrize("K,B", [(3072, 1024), (12288, 4096), (256, 256), (3584, 512), (64, 64)])
def test_fwht_is_orthogonal_involution(K, B):
    x = O.gen_f32(1, (5, K))
    y = O.fwht_rows(x, B)
    np.testing.assert_allclose(np.linalg.norm(y, axis=1), np.linalg.norm(x, axis=1), rtol=1e-5)
    np.testing.assert_allclose(O.fwht_rows(y, B), x, atol=1e-5)


def test_fwht_matches_hadamard_matrix():
    B = 16
    Hm = np.array([[1.0]])
    while Hm.shape[0] < B:
        Hm = np.block([[Hm, Hm], [Hm, -Hm]])
    x = O.gen_f32(2, (3, 2 * B))
    y = O.fwht_rows(x, B)
    ref = np.concatenate([x[:, :B] @ Hm.T, x[:, B:] @ Hm.T], axis=1) / np.sqrt(B)
    np.testing.assert_allclose(y, ref, atol=1e-5)


def test_activation_quantizer_properties():
    x = O.gen_f32(3, (6, 3072))
    x[0] = 0.0
    x[1, 9] = 500.0
    c, s = O.fwht_quant(x, 1024)
    assert c.dtype == np.int8 and s.dtype == np.float32
    assert s[0] == 0.0 and not c[0].any()
    assert (np.abs(c[1:]).max(axis=1) == 127).all()
    deq = c.astype(np.float32) * s[:, None]
    rot = O.fwht_rows(x, 1024)
    assert np.abs(deq - rot).max() <= s.max() * 0.5 + 1e-6


def test_weight_quantizer_matches_explicit_steps():
    w = O.gen_bf16(4, (8, 3072), 0.02)
    c, s = O.quant_weight(w)
    rot = O.fwht_rows(O.bf16_to_f32(w), 1024)
    mx = np.abs(rot).max(axis=1)
    np.testing.assert_array_equal(s, (mx / np.float32(127.0)).astype(np.float32))
    q = np.clip(np.rint(rot * (np.float32(127.0) / mx)[:, None]), -128, 127)
    np.testing.assert_array_equal(c, q.astype(np.int8))


def test_int8_gemm_exact():
    rng = np.random.default_rng(0)
    a = rng.integers(-128, 128, (37, 3072), dtype=np.int8)
    b = rng.integers(-128, 128, (70, 3072), dtype=np.int8)
    np.testing.assert_array_equal(O.gemm_i8(a, b), a.astype(np.int64) @ b.astype(np.int64).T)


def test_f32_gemm_and_attention():
    a = O.gen_f32(5, (33, 300))
    b = O.gen_f32(6, (17, 300))
    np.testing.assert_allclose(O.gemm_f32(a, b), a.astype(np.float64) @ b.T.astype(np.float64), rtol=1e-4,
                               atol=1e-4)
    q, k, v = (O.gen_f32(s, (2, 300, 128)) for s in (7, 8, 9))
    sc = np.float32(1.0 / np.sqrt(128.0))
    e = O.attention_exact(q, k, v, sc)
    f = O.attention_f32(q, k, v, sc)
    np.testing.assert_allclose(f, e, atol=2e-5)


@pytest.mark.parametrize("H,S", [(2, 200), (1, 77), (2, 333)])
def test_sage_emulation_close_to_exact(H, S):
    q, k, v = (O.f32_to_f16(O.gen_f32(s, (H, S, 128))).astype(np.float32) for s in (11, 12, 13))
    sc = np.float32(1.0 / np.sqrt(128.0))
    a = O.sage_attention(q, k, v, sc)
    e = O.attention_exact(q, k, v, sc)
    cos, maxrel = O.metrics(a, e)
    assert cos > 0.999 and maxrel < 2e-2, (cos, maxrel)


def test_sage_quantizer_scale_layout():
    H, S = 1, 200
    q = O.f32_to_f16(O.gen_f32(14, (H, S, 128))).astype(np.float32)
    k = q.copy()
    km, qc, qs, kc, ks = O.sage_quantize(q, k)
    assert qs.shape == (1, 64) and ks.shape == (1, 16)
    np.testing.assert_allclose(km[0], k[0].mean(axis=0), rtol=1e-4, atol=1e-6)
    # group g of Q covers tokens base + {0, 8, 16, 24}
    g = 37
    base = (g // 32) * 128 + ((g % 32) // 8) * 32 + g % 8
    toks = [t for t in (base, base + 8, base + 16, base + 24) if t < S]
    amax = max(1e-7, float(np.abs(q[0, toks]).max()))
    assert np.isclose(qs[0, g], amax / 127.0 + 1e-7, rtol=1e-6)


def test_quant_mode_agrees_with_fp32_mode_one_block():
    W = O.Weights(1, base_seed=0)
    H = Wd = 8
    n_txt = 8
    x = O.gen_bf16(O.seed_for(1, "latent"), (1, 16, H, Wd), 1.0)
    txt = O.gen_bf16(O.seed_for(1, "context"), (n_txt, 3584), 1.0)
    pe = O.rope_table(H, Wd, n_txt)
    a = O.forward(W, x, 500.0, txt, pe, mode="quant")
    b = O.forward(W, x, 500.0, txt, pe, mode="fp32")
    cos, maxrel = O.metrics(a, b)
    assert cos > 0.998 and maxrel < 0.1, (cos, maxrel)
