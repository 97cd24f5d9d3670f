"""Model check (CPU) of the tensor-parallel exchange protocol of the fused
all-reduce (go-infer_b200/csrc/tp.cuh, the kYPush epilogue of gemv.cu).

Each rank, for exchange k = 0, 1, 2, ...: stores its partial as one tagged
8-byte word (value, k) into slot `rank` of area k & 1 of every rank's region
(remote stores may stay in flight for any time; stores from one writer to
one address land in order), then waits for tag k in every slot of its own
area k & 1, reads the values and only then starts exchange k + 1.  Claim: a
read never returns another exchange's value — an area is rewritten (k + 2)
only after its reader has finished exchange k, because the writer needs the
reader's push of k + 1 to get that far.  The model runs random schedules of
world 2-8 ranks and checks every read; a variant with a single area (no
alternation) must fail, showing the check has teeth.
"""
import random

import pytest


def run_schedule(world, n_exchanges, seed, areas=2):
    rng = random.Random(seed)
    # region[r][area][slot] = (tag, value); tags start at a value no exchange uses
    region = [[[(-1, None)] * world for _ in range(areas)] for _ in range(world)]
    inflight = []  # (dest rank, area, slot, tag, value), per-writer order kept below
    state = [{"k": 0, "phase": "push", "pushed": 0, "got": {}} for _ in range(world)]
    reads = []

    def value(r, k):
        return f"r{r}k{k}"

    def stuck():  # nothing in flight and every unfinished rank waits for a tag that is not there
        if inflight:
            return False
        for r, s in enumerate(state):
            if s["k"] >= n_exchanges:
                continue
            if s["phase"] == "push":
                return False
            a = s["k"] % areas
            if all(slot in s["got"] or region[r][a][slot][0] == s["k"] for slot in range(world)):
                return False
        return True

    while any(s["k"] < n_exchanges for s in state):
        assert not stuck(), "deadlock: a reader waits for a tag that was overwritten"
        # pick an action: a rank's step or the landing of an in-flight store
        choices = [("rank", r) for r in range(world) if state[r]["k"] < n_exchanges]
        if inflight:
            choices += [("land", None)] * len(choices)
        kind, r = rng.choice(choices)
        if kind == "land":
            # land the oldest in-flight store of a random writer (per-writer order)
            writers = sorted({w for (_d, _a, w, _t, _v) in inflight})
            w = rng.choice(writers)
            i = next(i for i, st in enumerate(inflight) if st[2] == w)
            d, a, slot, tag, val = inflight.pop(i)
            region[d][a][slot] = (tag, val)
            continue
        s = state[r]
        k, a = s["k"], s["k"] % areas
        if s["phase"] == "push":
            d = s["pushed"]
            inflight.append((d, a, r, k, value(r, k)))  # one 8-byte store: tag and value together
            s["pushed"] += 1
            if s["pushed"] == world:
                s["phase"], s["got"] = "wait", {}
        else:
            for slot in range(world):
                if slot in s["got"]:
                    continue
                tag, val = region[r][a][slot]
                if tag == k:
                    s["got"][slot] = val
            if len(s["got"]) == world:
                reads.append((r, k, [s["got"][i] for i in range(world)]))
                s["k"], s["phase"], s["pushed"] = k + 1, "push", 0
    return reads


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_tagged_exchange_never_reads_another_exchange(world):
    for seed in range(150 if world < 8 else 40):
        for r, k, vals in run_schedule(world, 6, seed):
            assert vals == [f"r{i}k{k}" for i in range(world)], (seed, r, k, vals)


def test_single_area_can_deadlock_or_mix():
    # Without alternating areas a fast rank can overwrite a slot before a
    # slow reader saw it: some schedule must then stall (the reader waits
    # for a tag that was overwritten), which the model reports.
    bad = 0
    for seed in range(200):
        try:
            run_schedule(2, 6, seed, areas=1)
        except AssertionError:
            bad += 1
    assert bad > 0
