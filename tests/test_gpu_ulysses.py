"""Head-parallel (Ulysses) forward on 2, 4 and 8 GPUs (12, 6 and 3 heads per
GPU) against the single-GPU forward.

Every per-token computation (linears, norms, quantizers) and every per-head
computation (K mean, Sage quantization, attention over the full joint
sequence) is the same arithmetic in both, so the outputs must be equal bit
for bit.  Uneven splits (odd token counts) and nb = 2 are covered, for both
exchange paths: stores into peer memory with flag barriers, and NCCL
all-to-alls.  Needs P GPUs; skipped otherwise."""
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _gpus():
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _worker(rank, P, H, W, n_txt, nb, blocks, exchange, uid_q, out_q):
    try:
        import os

        import numpy as np
        os.environ["QI_PEER_EXCHANGE"] = "1" if exchange == "peer" else "0"

        import qib200 as Q
        import qi_oracle as O
        torch.cuda.set_device(rank)
        g, bt = Q.make_weight_table(blocks, base_seed=0)
        ctx = Q.Context(rank)
        model = Q.Model(ctx, g, bt)
        if rank == 0:
            uid = Q.comm_unique_id()
            for _ in range(P - 1):
                uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=120)
        ctx.set_comm(uid, rank, P)
        xs = np.concatenate([O.gen_bf16(O.seed_for(3 + b, "latent"), (1, 16, H, W), 1.0) for b in range(nb)])
        ts = np.concatenate([O.gen_bf16(O.seed_for(3 + b, "context"), (n_txt, 3584), 1.0) for b in range(nb)])
        pe1 = O.rope_table(H, W, n_txt)
        x = torch.from_numpy(xs.view(np.int16)).cuda().view(torch.bfloat16)
        txt = torch.from_numpy(ts.view(np.int16)).cuda().view(torch.bfloat16).view(nb, n_txt, 3584)
        pe = torch.from_numpy(np.stack([pe1] * nb)).cuda()
        y = Q.forward(ctx, model, x, 700.0, txt, pe)
        torch.cuda.synchronize()
        ctx.check()
        # the same forward on one GPU, in a context without a group
        ctx1 = Q.Context(rank)
        y1 = Q.forward(ctx1, model, x, 700.0, txt, pe)
        torch.cuda.synchronize()
        ctx1.check()
        same = bool(torch.equal(y.view(torch.int16), y1.view(torch.int16)))
        diff = float((y.float() - y1.float()).abs().max())
        model.close()
        ctx1.close()
        ctx.close()
        out_q.put((rank, "ok" if same else f"outputs differ: max |diff| {diff}"))
    except BaseException as e:
        out_q.put((rank, repr(e)))


@pytest.mark.parametrize("exchange", ["peer", "nccl"])
@pytest.mark.parametrize("P,H,W,n_txt,nb", [(2, 66, 66, 77, 1), (2, 32, 48, 30, 2), (4, 66, 66, 77, 2),
                                             (8, 64, 64, 64, 1), (8, 66, 70, 37, 2)])
def test_head_parallel_forward_equals_single_gpu(P, H, W, n_txt, nb, exchange):
    if _gpus() < P:
        pytest.skip(f"needs {P} GPUs")
    blocks = 2
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, P, H, W, n_txt, nb, blocks, exchange, uid_q, out_q))
             for r in range(P)]
    for p in procs:
        p.start()
    results = dict(out_q.get(timeout=600) for _ in range(P))
    for p in procs:
        p.join(timeout=120)
    assert all(v == "ok" for v in results.values()), results
