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


def test_group_member_that_never_joins_times_out():
    """A head-parallel group of two where the second rank never joins: the
    non-blocking communicator's initialisation misses the deadline, is
    aborted, and qi_ctx_set_comm returns QI_ERR_NCCL instead of blocking;
    multi-GPU calls then fail with the same status until the context forms a
    group again, and with nranks = 1 it runs single-GPU forwards as before.
    (Only host-side bootstrap waits for the missing rank; no kernel runs.)"""
    import os
    import time
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(0)
    ctx = Q.Context(0)
    ctx.set_comm_timeout(1500)
    uid = Q.comm_unique_id()
    t0 = time.monotonic()
    with pytest.raises(Q.QIError, match="collective failed"):
        ctx.set_comm(uid, 0, 2)
    assert time.monotonic() - t0 < 30.0
    g, blocks = Q.make_weight_table(1, base_seed=3)
    model = Q.Model(ctx, g, blocks)
    x = Q.synth((1, 16, 8, 8), Q.seed_for(3, "x"), 1.0, dtype=torch.bfloat16)
    txt = Q.synth((1, 8, 3584), Q.seed_for(3, "c"), 1.0, dtype=torch.bfloat16)
    pe = torch.from_numpy(Q.rope_table(8, 8, 8)).cuda()[None]
    with pytest.raises(Q.QIError, match="collective failed"):
        Q.forward(ctx, model, x, 500.0, txt, pe)
    ctx.set_comm(None, 0, 1)
    y = Q.forward(ctx, model, x, 500.0, txt, pe)
    ctx.sync(5000)
    assert torch.isfinite(y.float()).all()
    model.close()
    ctx.close()
