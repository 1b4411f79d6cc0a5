"""Rank layout of a multi-GPU denoising job (one process per GPU).

The reference runs cond and uncond one after the other on one GPU
(main.cu:761-773).  Here the two CFG halves go to two groups of ranks, and
each half may itself be split head-parallel (Ulysses) over P ranks:

    world 1: one rank runs both halves batched (nb = 2)
    world 2: CFG split, P = 1
    world 4: CFG split x P = 2
    world 8: CFG split x P = 4

Rank r belongs to CFG half r // P and is rank r % P of that half's Ulysses
group; ranks r and r +- P (same Ulysses rank, other half) exchange their
halves' velocities before the Euler step.
"""


def layout(world):
    """(cfg_split, P) for `world` ranks."""
    if world == 1:
        return False, 1
    if world % 2 or world // 2 > 8 or 24 % (world // 2):
        raise ValueError(f"unsupported world size {world}: 1, or 2 x P with P dividing 24, P <= 8")
    return True, world // 2


def roles(rank, world):
    """Role of `rank`: dict with the CFG half it computes (None when both are
    batched on one rank), its Ulysses rank and group size, the global ranks of
    its Ulysses group and of its CFG pair."""
    cfg_split, P = layout(world)
    if not cfg_split:
        return {"half": None, "urank": 0, "P": 1, "ulysses_group": [0], "cfg_pair": [0]}
    half, urank = rank // P, rank % P
    return {"half": half, "urank": urank, "P": P,
            "ulysses_group": [half * P + u for u in range(P)],
            "cfg_pair": [urank, P + urank]}


def shard_map(P, n_txt, n_img):
    """Token ranges per Ulysses rank: lists txt_lo, img_lo of length P + 1
    (the same even split the library uses)."""
    return [r * n_txt // P for r in range(P + 1)], [r * n_img // P for r in range(P + 1)]


class RankFailure(RuntimeError):
    """Ranks of the job that did not finish a step in time, or left."""

    def __init__(self, step, missing, left):
        self.step, self.missing, self.left = step, sorted(missing), sorted(left)
        super().__init__(f"step {step}: rank(s) {self.missing} did not finish step {step - 1} in time"
                         + (f"; rank(s) {self.left} left the job" if self.left else ""))


class StepMonitor:
    """Liveness of the ranks of a job between steps, on the host.

    Before a rank launches step k (and with it the collectives that wait for
    every peer), it checks through the process group's key-value store that
    every rank has finished step k - 1.  A rank that left (announced with
    leave(), or simply gone) or stopped reporting is found within
    `timeout_s` on every other rank, which then raise RankFailure instead of
    launching a collective that would wait for it.  The library's own
    collectives have a deadline too (qi_ctx_set_comm_timeout); this check
    keeps a whole job from reaching one."""

    def __init__(self, store, rank, world, timeout_s=10.0, prefix="qi_step"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = float(timeout_s), prefix

    def _key(self, step, rank):
        return f"{self.prefix}/{step}/{rank}"

    def finished(self, step):
        """This rank has finished `step` (its collectives included)."""
        self.store.set(self._key(step, self.rank), "1")

    def leave(self):
        """This rank leaves the job between steps."""
        self.store.set(f"{self.prefix}/left/{self.rank}", "1")

    def check(self, step):
        """Raises RankFailure unless every rank finished step - 1 within the
        timeout.  Step 0 needs nothing."""
        if step == 0:
            return
        import datetime
        import time
        keys = [self._key(step - 1, r) for r in range(self.world)]
        deadline = time.monotonic() + self.timeout_s
        while True:
            missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
            left = [r for r in range(self.world) if self.store.check([f"{self.prefix}/left/{r}"])]
            if not missing:
                return
            gone = set(left) & set(missing)
            if gone:  # known to have left: no need to wait out the deadline for it
                raise RankFailure(step, gone, left)
            if time.monotonic() > deadline:
                raise RankFailure(step, missing, left)
            try:
                self.store.wait([keys[missing[0]]], datetime.timedelta(milliseconds=50))
            except Exception:
                pass
