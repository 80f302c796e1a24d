"""A model of the P2P exchange protocol of b2_exchange_merge /
b2_decode_step_exchange (csrc/b2_attn.cu, xchg_merge), checked under random
interleavings of the ranks.

Each rank, per step e: (1) writes its words, tagged e + 1, into slot e % 2 of
every rank's area; (2) polls its own area until every rank's word in that slot
carries tag e + 1, then reads them; the next step's writes follow the reads in
stream order.  The claims: no read ever sees a word of another step (with two
slots a rank is at most one step ahead of any other), and no rank waits
forever.  With one slot the same model loses words - the negative control
that shows the second slot is needed.
"""
import random

import pytest


def run(world: int, steps: int, slots: int, seed: int) -> bool:
    """True if every read saw the expected step's words and all ranks finished."""
    rng = random.Random(seed)
    area = [[[0] * world for _ in range(slots)] for _ in range(world)]   # area[owner][slot][writer] = tag
    step = [0] * world
    phase = ["write"] * world            # write -> read -> (next step) write
    pending = [list(range(world)) for _ in range(world)]   # destinations still to write this step
    ok = True
    for _ in range(100000):
        if all(s == steps for s in step):
            return ok
        r = rng.randrange(world)
        if step[r] == steps:
            continue
        e, slot = step[r], step[r] % slots
        if phase[r] == "write":
            # the stores reach the destinations one at a time, in any order
            dst = pending[r].pop(rng.randrange(len(pending[r])))
            area[dst][slot][r] = e + 1
            if not pending[r]:
                phase[r] = "read"
        else:
            tags = area[r][slot]
            if all(t == e + 1 for t in tags):
                step[r] += 1
                phase[r] = "write"
                pending[r] = list(range(world))
            elif any(t > e + 1 for t in tags):
                ok = False     # a word of a later step overwrote this step's before it was read
                step[r] += 1
                phase[r] = "write"
                pending[r] = list(range(world))
    return False               # no progress: a rank waits forever


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_two_slots_never_lose_a_word(world):
    for seed in range(200):
        assert run(world, steps=12, slots=2, seed=seed), f"world {world}, schedule {seed}"


def test_one_slot_loses_words():
    assert not all(run(2, steps=12, slots=1, seed=s) for s in range(200))
