"""Failure detection without a GPU fault: a kernel wait that nothing satisfies
gives up after its limit and reports QI_ERR_DEVICE through the context's error
word; the context stays usable (a following kernel runs and checks clean)."""
import pytest
import torch

import qib200 as Q

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_error_and_context_survives():
    torch.cuda.set_device(0)
    ctx = Q.Context(0)
    ctx.check()
    Q.check(Q.lib().qi_selftest_wait_timeout(ctx.h, 20000, Q._stream()))
    torch.cuda.synchronize()
    with pytest.raises(Q.QIError, match="timed out"):
        ctx.check()
    ctx.check()  # the error word was read and cleared
    x = Q.synth((4, 3072), Q.seed_for(1, "after"), 1.0)
    c, s = Q.fwht_quantize(x)
    torch.cuda.synchronize()
    assert s.abs().min() > 0
    ctx.close()


def test_invalid_arguments_return_status_not_exit():
    torch.cuda.set_device(0)
    ctx = Q.Context(0)
    with pytest.raises(Q.QIError):
        Q.check(Q.lib().qi_selftest_wait_timeout(ctx.h, 0, Q._stream()))
    a = torch.zeros(8, 100, dtype=torch.int8, device="cuda")  # K % 16 != 0
    s = torch.ones(8, device="cuda")
    with pytest.raises(Q.QIError, match="invalid argument"):
        Q.linear_i8(a, s, torch.zeros(32, 100, dtype=torch.int8, device="cuda"), torch.ones(32, device="cuda"))
    ctx.check()
    ctx.close()
