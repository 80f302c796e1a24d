"""A CPU model of one CTA of the fused decode step's barrier protocol
(csrc/b2_attn.cu: step_producer, step_consumer, step_epilogue, publish,
step_merger), checked under random schedules.

Roles: the producer warp fills a ring of 4 stages (a stage = one block's K
and V tiles plus its StageMeta) item after item, ends with a marker on the
next stage and waits for its last copy on every other stage.  An item's
first block is issued with an expected transfer but no arrival; the
producer arrives on that stage only after the item's q is in the stage's
meta, so the phase completes when both the copy has landed and q is there; four consumer warps take every stage, run an epilogue at the
last block of an item (a barrier of the four warps, `ebar`, around a
reduction array double-buffered by epilogue parity) and, for items of a
sequence split over several CTAs, publish the item to the merger warp
through one of 4 slots (`pub`: every consumer arrives after its partial-state
stores; `pfree`: the merger has read the slot).  After the last stage they
publish an end marker.

As in the prefill model, every wait for the k-th completion of a barrier is
checked to find exactly k or k + 1 completed phases (the only range in which
a parity wait is exact), and the hazards the barriers guard are checked: a
stage and its meta are refilled only after all four warps are done with
them, a reduction buffer is written only after every warp has read its
previous contents, a slot's item info is overwritten only after the merger
has read it, and every role finishes.
"""
import random

import pytest

STAGES = 4
SLOTS = 4
WARPS = 4


class Barrier:
    def __init__(self, name, count):
        self.name, self.count, self.arrived, self.done = name, count, 0, 0

    def arrive(self):
        self.arrived += 1
        assert self.arrived <= self.count, f"{self.name}: too many arrivals"
        if self.arrived == self.count:
            self.arrived, self.done = 0, self.done + 1


class StepCTA:
    def __init__(self, items, seed, early_arrive=False):
        """items: list of (blocks, publishes) in the order the producer takes them.
        early_arrive: the first block's arrival comes with its copy (a wrong
        protocol, for the negative control)."""
        self.rng = random.Random(seed)
        self.early_arrive = early_arrive
        self.items = items
        self.bar = {}
        for s in range(STAGES):
            self.bar[f"full{s}"] = Barrier(f"full{s}", 1)
            self.bar[f"empty{s}"] = Barrier(f"empty{s}", WARPS)
        for i in range(SLOTS):
            self.bar[f"pub{i}"] = Barrier(f"pub{i}", WARPS)      # 128 threads, counted per warp
            self.bar[f"pfree{i}"] = Barrier(f"pfree{i}", 1)
        self.bar["ebar"] = Barrier("ebar", WARPS)
        self.stage = [None] * STAGES          # (item, block) a stage holds, or "end"
        self.stage_readers = [set() for _ in range(STAGES)]
        self.red_writer = [None, None]        # epilogue index whose values a buffer holds
        self.red_readers = [set(), set()]
        self.slot = [None] * SLOTS            # item published in a slot
        self.slot_unread = [False] * SLOTS
        self.merged = []
        self.tma = []
        self.first = {}                       # stage -> [copy landed, producer arrived] of a first block
        self.q_ready = [True] * STAGES        # the stage's meta holds its item's q (first blocks)

    def producer(self):
        issued = 0
        for it, (nblk, _) in enumerate(self.items):
            for jj in range(nblk):
                s = issued % STAGES
                if issued >= STAGES:
                    yield ("wait", f"empty{s}", issued // STAGES - 1)
                assert not self.stage_readers[s], f"stage {s} refilled while warps still read it"
                self.stage[s] = None                          # meta written, copy in flight
                if jj == 0:
                    self.q_ready[s] = False
                    if not self.early_arrive:
                        self.first[s] = [False, False]        # expect_tx only: no arrival yet
                self.tma.append((s, (it, jj)))
                if jj == 0:
                    yield ("work", None, None)                # the q/k work, with the copy in flight
                    self.q_ready[s] = True                    # q into the stage's meta, then arrive
                    if not self.early_arrive:
                        self.first[s][1] = True
                        if self.first[s][0]:
                            del self.first[s]
                            self.bar[f"full{s}"].arrive()
                issued += 1
        s = issued % STAGES
        if issued >= STAGES:
            yield ("wait", f"empty{s}", issued // STAGES - 1)
        assert not self.stage_readers[s]
        self.stage[s] = "end"
        self.stage_readers[s] = set(range(WARPS))
        self.bar[f"full{s}"].arrive()                         # the end marker: a plain arrival
        marker = s
        # drain: the last copy issued on every other stage has landed before
        # the producer leaves (the marker's stage: released above)
        for st in range(min(STAGES, issued)):
            if st != marker:
                yield ("wait", f"full{st}", (issued - 1 - st) // STAGES)

    def consumer(self, w):
        ephase, epilogues, pubs = 0, 0, 0
        it_no = 0
        for k in range(10 ** 6):
            s = k % STAGES
            yield ("wait", f"full{s}", k // STAGES)
            got = self.stage[s]
            assert got is not None, f"warp {w} read stage {s} before its copy landed"
            assert self.q_ready[s], f"warp {w} read stage {s} before its q was in the meta"
            if got == "end":
                self.stage_readers[s].discard(w)
                break
            item, jj = got
            self.stage_readers[s].discard(w)
            self.bar[f"empty{s}"].arrive()
            nblk, publishes = self.items[item]
            if jj == nblk - 1:
                rbuf = epilogues & 1
                # write this warp's share of red[rbuf]: everyone must have read the old contents
                assert not self.red_readers[rbuf] or self.red_writer[rbuf] == epilogues, \
                    f"red[{rbuf}] overwritten while a warp still reads epilogue {self.red_writer[rbuf]}"
                if self.red_writer[rbuf] != epilogues:
                    self.red_writer[rbuf] = epilogues
                    self.red_readers[rbuf] = set(range(WARPS))
                self.bar["ebar"].arrive()
                yield ("wait", "ebar", ephase)
                ephase += 1
                self.red_readers[rbuf].discard(w)              # merged after the barrier
                epilogues += 1
                if publishes:
                    slot = pubs % SLOTS
                    if pubs >= SLOTS:
                        yield ("wait", f"pfree{slot}", pubs // SLOTS - 1)
                    if w == 0:
                        assert not self.slot_unread[slot], f"slot {slot} overwritten before the merger read it"
                        self.slot[slot] = item
                        self.slot_unread[slot] = True
                    self.bar[f"pub{slot}"].arrive()
                    pubs += 1
                it_no += 1
        slot = pubs % SLOTS
        if pubs >= SLOTS:
            yield ("wait", f"pfree{slot}", pubs // SLOTS - 1)
        if w == 0:
            assert not self.slot_unread[slot]
            self.slot[slot] = -1
            self.slot_unread[slot] = True
        self.bar[f"pub{slot}"].arrive()

    def merger(self):
        for k in range(10 ** 6):
            slot = k % SLOTS
            yield ("wait", f"pub{slot}", k // SLOTS)
            assert self.slot_unread[slot]
            item = self.slot[slot]
            self.slot_unread[slot] = False
            self.bar[f"pfree{slot}"].arrive()
            if item == -1:
                return
            self.merged.append(item)

    def run(self):
        roles = {"producer": self.producer(), "merger": self.merger()}
        for w in range(WARPS):
            roles[f"c{w}"] = self.consumer(w)
        pending = dict.fromkeys(roles)
        for _ in range(10 ** 6):
            choices = [("role", n) for n, g in roles.items()
                       if g is not None and (pending[n] is None or pending[n][0] == "work"
                                             or self.bar[pending[n][1]].done > pending[n][2])]
            choices += [("tma", i) for i in range(len(self.tma))]
            if not choices:
                live = [n for n, g in roles.items() if g is not None]
                assert not live, f"deadlock: {[(n, pending[n]) for n in live]}"
                break
            kind, arg = self.rng.choice(choices)
            if kind == "tma":
                s, what = self.tma.pop(arg)
                self.stage[s] = what
                self.stage_readers[s] = set(range(WARPS))
                if s in self.first:                            # a first block: the arrival completes it
                    self.first[s][0] = True
                    if self.first[s][1]:
                        del self.first[s]
                        self.bar[f"full{s}"].arrive()
                else:
                    self.bar[f"full{s}"].arrive()
                continue
            p = pending[arg]
            if p is not None and p[0] == "wait":
                d = self.bar[p[1]].done
                assert d <= p[2] + 1, f"{arg}: wait for completion {p[2]} of {p[1]} with {d} done: lapped"
            try:
                nxt = next(roles[arg])
                if nxt[0] == "wait":
                    d = self.bar[nxt[1]].done
                    assert d >= nxt[2], f"{arg}: wait for completion {nxt[2]} of {nxt[1]} with {d} done: passes early"
                pending[arg] = nxt
            except StopIteration:
                roles[arg], pending[arg] = None, None
        assert self.merged == [i for i, (_, pub) in enumerate(self.items) if pub]


@pytest.mark.parametrize("seed", range(150))
def test_step_barriers_hold_under_random_schedules(seed):
    rng = random.Random(seed)
    items = [(rng.randint(1, 6), rng.random() < 0.6) for _ in range(rng.randint(0, 12))]
    StepCTA(items, seed).run()


def test_an_arrival_before_q_is_caught():
    """Negative control: if the first block's phase completed with its copy
    alone (q written afterwards), a consumer could read the meta before q;
    the model reports it under some schedule."""
    caught = 0
    for seed in range(200):
        try:
            StepCTA([(2, False), (1, True), (3, False)], seed, early_arrive=True).run()
        except AssertionError as e:
            assert "before its q" in str(e), e
            caught += 1
    assert caught > 0
