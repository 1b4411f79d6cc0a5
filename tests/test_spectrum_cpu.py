"""Spectrum forecasting, host side (no GPU): the library's prediction weights
(qi_spectrum_weights, the part of qi_spectrum_predict that runs on the host)
applied to a history must give the oracle's restatement of the reference's
spectrum_predict (oracle/qi_oracle.py, cuda_kernels.cu:6268-6333), and the
argument checks must reject what the reference cannot fit."""
import numpy as np
import pytest

import qi_oracle as O
import qib200 as Q

CASES = [
    # steps, target, order, lambda, blend
    ([5, 6], 7, 4, 0.1, 1.0),
    ([5, 7, 9, 11, 13, 15], 16, 4, 0.1, 1.0),
    ([0, 1, 2, 3, 4, 5, 7, 9, 11, 13, 15, 17], 18, 4, 0.1, 0.5),
    (list(range(5, 45, 2)), 46, 6, 0.01, 0.75),
    ([10, 12, 14, 16, 18, 20, 22, 24], 23, 3, 1.0, 0.0),
    ([3, 4, 5, 6, 7], 9, 0, 0.1, 1.0),
    ([1, 3], 2, 1, 0.5, 0.3),
]


@pytest.mark.parametrize("steps,target,order,lam,blend", CASES)
def test_weights_reproduce_the_oracle(steps, target, order, lam, blend):
    rng = np.random.default_rng(len(steps) * 131 + order)
    hist = rng.standard_normal((len(steps), 257))
    w = Q.spectrum_weights(steps, order, lam, target, blend)
    ours = w @ hist
    # blend and lambda cross the C ABI as float (as in the reference's API)
    ref = O.spectrum_predict(hist, steps, target, float(np.float32(blend)), order, float(np.float32(lam)))
    assert np.abs(ours - ref).max() <= 1e-9 * max(1.0, np.abs(ref).max())


def test_weights_are_linear_in_blend_and_sum_to_one():
    # both parts reproduce a constant history exactly when lambda -> 0
    steps = [2, 4, 6, 8, 10]
    w1 = Q.spectrum_weights(steps, 2, 1e-9, 11, 1.0)
    w0 = Q.spectrum_weights(steps, 2, 1e-9, 11, 0.0)
    wh = Q.spectrum_weights(steps, 2, 1e-9, 11, 0.5)
    assert abs(w1.sum() - 1.0) < 1e-6 and abs(w0.sum() - 1.0) < 1e-12
    np.testing.assert_allclose(wh, 0.5 * (w0 + w1), rtol=0, atol=1e-12)


@pytest.mark.parametrize("steps,order", [([5], 4), ([5, 5], 4), ([7, 6], 4), ([1, 2], 17), ([1, 2], -1)])
def test_weights_reject_what_cannot_be_fitted(steps, order):
    with pytest.raises(Q.QIError):
        Q.spectrum_weights(steps, order, 0.1, 9, 1.0)


def test_create_rejects_bad_shapes():
    for args in ((0, 10, 4, 0.1), (6, 10, 4, 0.1), (4096, 1, 4, 0.1), (4096, 129, 4, 0.1), (4096, 10, 4, -1.0)):
        with pytest.raises(Q.QIError):
            Q.Spectrum(*args)
