"""A model of the mbarrier protocol of the narrow fused kernel
(tensor-bridge_b200/csrc/fused_tmem_kernel.cuh), run under random schedules.

Each role replays, in order, the waits and arrivals the kernel issues: the raw-A
producer (SPR raw stages per round of four k-blocks), the B producer (one
arrival with the round's bytes on rdy), the MMA issuer (one rdy wait and one
fre commit per round; commits land later, like MMA completion), the epilogue
and the sixteen decode warps (slice j decodes k-block j of every round and
reads raw stage position j // RSK).  TMA completions also land later.  A wait
is modelled the way the hardware answers a parity wait -- it passes when the
barrier's current phase parity differs from the waited one -- and the model
fails when that answer differs from the intended one (the phase completed or
not), when an arrival lands in a phase other than the one it is meant for, or
when no role can move.  The ring depths are the ones the launcher picks for
each format and tile width, plus small rings."""
import random

import pytest

SMEM_BUDGET = 224 * 1024
DK = 4


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.c, self.pending = name, count, 0, 0

    def arrive(self, k, who):
        assert k == self.c, f"{who}: arrival meant for phase {k} of {self.name} lands in phase {self.c}"
        self.pending += 1
        if self.pending == self.count:
            self.pending, self.c = 0, self.c + 1


def run(units, RSK, SR, NRND, seed):
    """units: k-blocks per work unit of this CTA, in order."""
    SPR = DK // RSK
    rng = random.Random(seed)
    raw_full = [Bar(f"raw_full{i}", 2) for i in range(SR)]  # producer arrive + TMA bytes
    raw_empty = [Bar(f"raw_empty{i}", 4 * RSK) for i in range(SR)]
    rdy = [Bar(f"rdy{i}", 16 + 2) for i in range(NRND)]  # 16 decode warps + B arrive + B bytes
    fre = [Bar(f"fre{i}", 1) for i in range(NRND)]
    acc_full = [Bar(f"acc_full{i}", 1) for i in range(2)]
    acc_empty = [Bar(f"acc_empty{i}", 1) for i in range(2)]
    later = []
    rounds = [(nkb + DK - 1) // DK for nkb in units]

    def raw_producer():
        st = 0
        for nr in rounds:
            for _ in range(nr * SPR):
                rs, fill = st % SR, st // SR
                if fill:
                    yield ("wait", raw_empty[rs], fill - 1)
                yield ("arrive", raw_full[rs], fill)
                yield ("later", raw_full[rs], fill)
                st += 1

    def b_producer():
        r = 0
        for nr in rounds:
            for _ in range(nr):
                slot, use = r % NRND, r // NRND
                if use:
                    yield ("wait", fre[slot], use - 1)
                yield ("arrive", rdy[slot], use)
                yield ("later", rdy[slot], use)
                r += 1

    def mma():
        r = 0
        for ui, nr in enumerate(rounds):
            acc, k = ui & 1, ui >> 1
            if k:
                yield ("wait", acc_empty[acc], k - 1)
            for _ in range(nr):
                slot, use = r % NRND, r // NRND
                yield ("wait", rdy[slot], use)
                yield ("later", fre[slot], use)
                r += 1
            yield ("later", acc_full[acc], k)

    def epilogue():
        for ui, _ in enumerate(rounds):
            acc, k = ui & 1, ui >> 1
            yield ("wait", acc_full[acc], k)
            yield ("arrive", acc_empty[acc], k)

    def decode(j):
        r = 0
        for nr in rounds:
            for _ in range(nr):
                st = r * SPR + j // RSK
                rs, fill = st % SR, st // SR
                slot, use = r % NRND, r // NRND
                yield ("wait", raw_full[rs], fill)
                if use:
                    yield ("wait", fre[slot], use - 1)
                yield ("arrive", raw_empty[rs], fill)
                yield ("arrive", rdy[slot], use)
                r += 1

    roles = {"raw producer": raw_producer(), "B producer": b_producer(), "MMA": mma(), "epilogue": epilogue()}
    for q in range(4):
        for j in range(4):
            roles[f"decode q{q} s{j}"] = decode(j)
    cur = {n: next(g, None) for n, g in roles.items()}
    while True:
        live = [n for n, op in cur.items() if op is not None]
        if not live and not later:
            return
        ready = []
        for n in live:
            op = cur[n]
            if op[0] == "wait":
                bar, k = op[1], op[2]
                hw = (bar.c & 1) != (k & 1)
                assert hw == (bar.c >= k + 1), f"{n}: wait for phase {k} of {bar.name} at phase {bar.c}"
                if hw:
                    ready.append(n)
            else:
                ready.append(n)
        choices = ready + (["completion"] if later else [])
        assert choices, "no role can move: " + ", ".join(f"{n} waits {cur[n][1].name}" for n in live)
        pick = rng.choice(choices)
        if pick == "completion":
            bar, k, who = later.pop(rng.randrange(len(later)))
            bar.arrive(k, who)
            continue
        op = cur[pick]
        if op[0] == "arrive":
            op[1].arrive(op[2], pick)
        elif op[0] == "later":
            later.append((op[1], op[2], pick))
        cur[pick] = next(roles[pick], None)


ROW_BYTES = {"E2M1": 32, "E4M3": 64, "BF16": 128, "TF32": 256}


def launcher_rings(fmt, bn):
    """RSK, SR and NRND as the launcher (PickTmem) and TmemCfg choose them."""
    row = ROW_BYTES[fmt]
    rsk = 4 if row <= 64 else 2 if row == 128 else 1
    spr = DK // rsk
    nrnd = 3 if bn <= 32 else 2
    stage = rsk * row * 128
    sr = min(12, (SMEM_BUDGET - 1024 - nrnd * 4 * bn * 128) // stage)
    sr = sr // spr * spr
    return rsk, sr, nrnd


UNITS = [[64], [20, 28, 64, 12], [13, 9], [66, 10], [1, 2, 3, 5]]


@pytest.mark.parametrize("fmt", list(ROW_BYTES))
@pytest.mark.parametrize("bn", [16, 32, 64])
def test_launcher_rings(fmt, bn):
    rsk, sr, nrnd = launcher_rings(fmt, bn)
    assert sr >= DK // rsk and sr % (DK // rsk) == 0
    for i, units in enumerate(UNITS):
        run(units, rsk, sr, nrnd, seed=i)


@pytest.mark.parametrize("rsk,sr,nrnd", [(4, 1, 2), (4, 2, 3), (2, 2, 2), (2, 4, 3), (1, 4, 2), (1, 8, 3)])
def test_small_rings(rsk, sr, nrnd):
    for i, units in enumerate(UNITS):
        run(units, rsk, sr, nrnd, seed=10 + i)


def test_model_flags_mixed_slot_positions():
    """A raw ring whose depth is not a multiple of the stages per round puts
    different stage positions -- read by different warps -- into one slot, so
    a warp can wait on a slot that has been refilled twice since it last read
    it; the model catches the stale parity."""
    failures = 0
    for seed in range(20):
        try:
            run([64], 2, 3, 3, seed=seed)
        except AssertionError:
            failures += 1
    assert failures > 0
