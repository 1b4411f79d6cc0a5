"""Multi-rank host logic on CPU: gloo ranks, world size 2, no GPU.

* The rank layout of bench.py (topology.py): CFG halves and Ulysses groups.
* The two all-to-all exchanges of a head-parallel block, with the per-peer
  offsets and sizes from the library itself (qi_exchange_plan through the C
  ABI), driven through real gloo all-to-alls.  The packing and unpacking
  index maps of the CUDA kernels (qkv_post's send layout, the attention
  epilogue's per-destination output, the two gather kernels) are restated in
  Python; every 256-byte FP16 row is modelled as 64 int32 whose first four
  carry (batch/which, head, joint position, source rank), so each received
  row proves where it came from.
* The CFG pair exchange of the velocities.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import qib200 as Q
import topology as T

ROW = 64  # int32 per FP16 row of 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _owner(pos, n_txt, tlo, ilo, P):
    """Rank owning joint position `pos` and its local position there (the
    loop of the gather kernels and the attention epilogue)."""
    src = 0
    if pos < n_txt:
        while src + 1 < P and tlo[src + 1] <= pos:
            src += 1
        return src, pos - tlo[src]
    gi = pos - n_txt
    while src + 1 < P and ilo[src + 1] <= gi:
        src += 1
    return src, (tlo[src + 1] - tlo[src]) + gi - ilo[src]


def _local_to_joint(rank, lp, n_txt, tlo, ilo):
    nt = tlo[rank + 1] - tlo[rank]
    return tlo[rank] + lp if lp < nt else n_txt + ilo[rank] + lp - nt


def _a2a(send, sbytes, rbytes):
    recv = torch.empty(sum(rbytes) // 4, dtype=torch.int32)
    dist.all_to_all_single(recv, torch.from_numpy(send), output_split_sizes=[b // 4 for b in rbytes],
                           input_split_sizes=[b // 4 for b in sbytes])
    return recv.numpy()


def _exchange_worker(rank, world, port, nb, n_txt, n_img, out):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        P = world
        tlo, ilo = T.shard_map(P, n_txt, n_img)
        Hl = 24 // P
        L = [(tlo[r + 1] - tlo[r]) + (ilo[r + 1] - ilo[r]) for r in range(P)]
        Lr = L[rank]

        # ---- exchange 0: Q/K/V, packed by qkv_post as [dest][3][nb][Hl][L(rank)][128]
        so, sb, ro, rb = Q.exchange_plan(0, nb, n_txt, n_img, P, rank)
        assert all(so[q] == q * 3 * nb * Hl * Lr * 256 for q in range(P))
        send = np.zeros(sum(sb) // 4, np.int32)
        for dest in range(P):
            for which in range(3):
                for b in range(nb):
                    for hh in range(Hl):
                        for lp in range(Lr):
                            row = (((dest * 3 + which) * nb + b) * Hl + hh) * Lr + lp
                            pos = _local_to_joint(rank, lp, n_txt, tlo, ilo)
                            send[row * ROW:row * ROW + 4] = [which * nb + b, dest * Hl + hh, pos, rank]
        recv = _a2a(send, sb, rb)
        # ulysses_gather_qkv: [src][3][nb][Hl][L(src)] -> [3][nb*Hl][S] in joint order
        S = n_txt + n_img
        for which in range(3):
            for b in range(nb):
                for hh in range(Hl):
                    for pos in range(S):
                        src, lp = _owner(pos, n_txt, tlo, ilo, P)
                        off = sum(3 * nb * Hl * L[q] for q in range(src))
                        assert off * 256 == ro[src]
                        in_row = off + ((which * nb + b) * Hl + hh) * L[src] + lp
                        got = list(recv[in_row * ROW:in_row * ROW + 4])
                        assert got == [which * nb + b, rank * Hl + hh, pos, src], (got, which, b, hh, pos)

        # ---- exchange 1: attention output of this rank's heads, [dest][nb][L(dest)][Hl][128]
        so, sb, ro, rb = Q.exchange_plan(1, nb, n_txt, n_img, P, rank)
        send = np.zeros(sum(sb) // 4, np.int32)
        for b in range(nb):
            for hh in range(Hl):
                for pos in range(S):
                    dest, lp = _owner(pos, n_txt, tlo, ilo, P)
                    off = sum(nb * L[q] * Hl for q in range(dest))
                    assert off * 256 == so[dest]
                    row = off + (b * L[dest] + lp) * Hl + hh
                    send[row * ROW:row * ROW + 4] = [b, rank * Hl + hh, pos, rank]
        recv = _a2a(send, sb, rb)
        # ulysses_gather_o: [src][nb][L(rank)][Hl] -> rows [nb*ni image; nb*nt text] x 24 heads
        nt, ni = tlo[rank + 1] - tlo[rank], ilo[rank + 1] - ilo[rank]
        for orow in range(nb * (ni + nt)):
            if orow < nb * ni:
                b, lp = orow // ni, nt + orow % ni
            else:
                b, lp = (orow - nb * ni) // nt, (orow - nb * ni) % nt
            pos = _local_to_joint(rank, lp, n_txt, tlo, ilo)
            for h in range(24):
                src, hh = h // Hl, h % Hl
                in_row = ((src * nb + b) * Lr + lp) * Hl + hh
                got = list(recv[in_row * ROW:in_row * ROW + 4])
                assert got == [b, h, pos, src], (got, orow, h)
        out.put((rank, "ok"))
    except BaseException as e:  # report to the parent instead of hanging it
        out.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _cfg_worker(rank, world, port, out):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        r = T.roles(rank, world)
        pair = dist.new_group(r["cfg_pair"])
        v = torch.full((16,), float(r["half"] + 1))  # this half's velocity
        g = torch.empty(2 * 16)
        dist.all_gather_into_tensor(g, v, group=pair)
        g = g.view(2, 16)
        assert torch.equal(g[0], torch.full((16,), 1.0)) and torch.equal(g[1], torch.full((16,), 2.0))
        out.put((rank, "ok"))
    except BaseException as e:
        out.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _run(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in results.values()), results


@pytest.mark.parametrize("nb,n_txt,n_img", [(1, 10, 37), (2, 5, 16)])
def test_head_parallel_exchanges_world2(nb, n_txt, n_img):
    _run(_exchange_worker, 2, nb, n_txt, n_img)


def test_cfg_pair_exchange_world2():
    _run(_cfg_worker, 2)


def test_rank_layout():
    assert T.layout(1) == (False, 1)
    assert T.layout(2) == (True, 1)
    assert T.layout(4) == (True, 2)
    assert T.layout(8) == (True, 4)
    with pytest.raises(ValueError):
        T.layout(6 * 2 + 1)
    for world in (2, 4, 8):
        rs = [T.roles(r, world) for r in range(world)]
        # every rank in exactly one Ulysses group and one CFG pair
        groups = {tuple(x["ulysses_group"]) for x in rs}
        assert sorted(r for g in groups for r in g) == list(range(world))
        pairs = {tuple(x["cfg_pair"]) for x in rs}
        assert sorted(r for p in pairs for r in p) == list(range(world))
        for r, x in enumerate(rs):
            assert r in x["ulysses_group"] and r in x["cfg_pair"]
            assert x["ulysses_group"][x["urank"]] == r
            assert x["cfg_pair"][x["half"]] == r


def test_exchange_plan_sizes_match_shard_map():
    for P in (2, 3, 4, 6, 8):
        tlo, ilo = T.shard_map(P, 256, 6889)
        L = [(tlo[r + 1] - tlo[r]) + (ilo[r + 1] - ilo[r]) for r in range(P)]
        assert sum(L) == 256 + 6889
        for r in range(P):
            so, sb, ro, rb = Q.exchange_plan(0, 1, 256, 6889, P, r)
            assert sb == [3 * (24 // P) * L[r] * 256] * P
            assert rb == [3 * (24 // P) * L[q] * 256 for q in range(P)]
            so, sb, ro, rb = Q.exchange_plan(1, 1, 256, 6889, P, r)
            assert sb == [(24 // P) * L[q] * 256 for q in range(P)]
            assert rb == [(24 // P) * L[r] * 256] * P


# ------------------------------------------------------------------ failure detection
# Host-side: a rank that never reports a step, or leaves between steps, is
# found by every other rank through the store before it launches the next
# step's collectives (topology.StepMonitor).  The failures are made on the
# host (a rank that stops reporting or exits); no device is involved.
def _monitor_worker(rank, world, port, mode, out):
    import time
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
        store = dist.distributed_c10d._get_default_store()
        mon = T.StepMonitor(store, rank, world, timeout_s=2.0, prefix=f"t_{mode}")
        t0 = time.monotonic()
        for step in range(4):
            mon.check(step)
            t = torch.full((4,), float(rank + step))
            dist.all_reduce(t)  # the step's collective: every rank reaches it only after the check
            assert t[0].item() == sum(r + step for r in range(world))
            if mode == "silent" and rank == world - 1 and step == 1:
                time.sleep(6.0)  # never reports step 1; alive, but stuck on the host
                out.put((rank, "ok"))
                return
            if mode == "leave" and rank == world - 1 and step == 1:
                mon.leave()
                out.put((rank, "ok"))
                return  # leaves between steps, nothing in flight
            mon.finished(step)
        out.put((rank, "ok" if mode == "none" else "no failure seen"))
    except T.RankFailure as e:
        dt = time.monotonic() - t0
        expect = e.step == 2 and e.missing == [world - 1] and (mode == "silent" or e.left == [world - 1])
        out.put((rank, "ok" if expect and dt < 10.0 else f"wrong failure {e} after {dt:.1f} s"))
    except BaseException as e:
        out.put((rank, repr(e)))
    finally:
        if dist.is_initialized() and mode == "none":
            dist.destroy_process_group()


@pytest.mark.parametrize("mode,world", [("none", 2), ("silent", 2), ("leave", 2), ("leave", 3)])
def test_step_monitor_finds_failed_rank(mode, world):
    _run(_monitor_worker, world, mode)
