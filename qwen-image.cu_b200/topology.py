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
