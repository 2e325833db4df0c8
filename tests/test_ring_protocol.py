"""A model of the barrier protocol of the narrow fused kernel
(tensor-bridge_b200/csrc/fused_tmem_kernel.cuh), run under random schedules.

Each role replays, in order, the waits and arrivals the kernel issues: the raw-A
producer (SPR raw stages per round of four k-blocks, at most `inflight` stages
in flight), the B producer (one arrival with the round's bytes on rdy), the MMA
issuer (one rdy wait and one fre commit per round; commits land later, like MMA
completion), the epilogue and the sixteen decode warps (slice j decodes
k-block j of every round and reads raw stage position j // RSK).  With a raw
ring of at least two rounds a sync warp does the decode warps' mbarrier waits
one round ahead and their arrivals, and hands rounds over through two pairs of
named barriers; otherwise each decode warp waits and arrives itself.  TMA
completions also land later.  An mbarrier wait is modelled the way the
hardware answers a parity wait -- it passes when the barrier's current phase
parity differs from the waited one -- and the model fails when that answer
differs from the intended one (the phase completed or not), when an arrival
lands in a phase other than the one it is meant for, when one generation of a
named barrier collects arrivals meant for different rounds, or when no role
can move.  The ring depths are the ones the launcher picks for each format and
tile width, plus small rings."""
import random

import pytest

SMEM_BUDGET = 224 * 1024
DK = 4


class NamedBar:
    """A hardware named barrier: a generation completes after `count` arrivals;
    bar.sync arrives and waits for the generation it arrived in."""

    def __init__(self, name, count):
        self.name, self.count, self.gen, self.tags = name, count, 0, []

    def arrive(self, tag, who):
        if self.tags:
            assert self.tags[0] == tag, f"{who}: arrival for round {tag} in a generation of {self.name} for round {self.tags[0]}"
        self.tags.append(tag)
        gen = self.gen
        if len(self.tags) == self.count:
            self.tags, self.gen = [], self.gen + 1
        return gen


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.c, self.pending = name, count, 0, 0

    def arrive(self, k, who):
        assert k == self.c, f"{who}: arrival meant for phase {k} of {self.name} lands in phase {self.c}"
        self.pending += 1
        if self.pending == self.count:
            self.pending, self.c = 0, self.c + 1


def run(units, RSK, SR, NRND, seed, syncw=None, inflight=2):
    """units: k-blocks per work unit of this CTA, in order; inflight: raw
    stages the producer keeps in flight (fewer than SR, as in TmemCfg: the
    stage it waits for must not have been refilled; 0 = no bound)."""
    SPR = DK // RSK
    inflight = min(inflight, SR - 1)
    if syncw is None:
        syncw = SR >= 2 * SPR
    rng = random.Random(seed)
    raw_full = [Bar(f"raw_full{i}", 2) for i in range(SR)]  # producer arrive + TMA bytes
    raw_empty = [Bar(f"raw_empty{i}", 1 if syncw else 4 * RSK) for i in range(SR)]
    rdy = [Bar(f"rdy{i}", (1 if syncw else 16) + 2) for i in range(NRND)]  # decode side + B arrive + B bytes
    start = [NamedBar(f"START{i}", 17) for i in range(2)]
    done = [NamedBar(f"DONE{i}", 17) for i in range(2)]
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
                if inflight and st >= inflight:  # at most `inflight` stages in flight
                    old = st - inflight
                    yield ("wait", raw_full[old % SR], old // SR)
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
                if syncw:
                    yield ("nsync", start[r & 1], r)
                    yield ("narrive", done[r & 1], r)
                else:
                    st = r * SPR + j // RSK
                    rs, fill = st % SR, st // SR
                    slot, use = r % NRND, r // NRND
                    yield ("wait", raw_full[rs], fill)
                    if use:
                        yield ("wait", fre[slot], use - 1)
                    yield ("arrive", raw_empty[rs], fill)
                    yield ("arrive", rdy[slot], use)
                r += 1

    def sync_warp():
        nr = sum(rounds)

        def ready(r):
            for pos in range(SPR):
                st = r * SPR + pos
                yield ("wait", raw_full[st % SR], st // SR)
            if r // NRND:
                yield ("wait", fre[r % NRND], r // NRND - 1)

        if nr:
            yield from ready(0)
            yield ("narrive", start[0], 0)
        for r in range(nr):
            if r + 1 < nr:
                yield from ready(r + 1)
                yield ("narrive", start[(r + 1) & 1], r + 1)
            yield ("nsync", done[r & 1], r)
            for pos in range(SPR):
                st = r * SPR + pos
                yield ("arrive", raw_empty[st % SR], st // SR)
            yield ("arrive", rdy[r % NRND], r // NRND)

    roles = {"raw producer": raw_producer(), "B producer": b_producer(), "MMA": mma(), "epilogue": epilogue()}
    if syncw:
        roles["sync warp"] = sync_warp()
    for q in range(4):
        for j in range(4):
            roles[f"decode q{q} s{j}"] = decode(j)
    cur = {n: next(g, None) for n, g in roles.items()}
    parked = {}  # role -> (named barrier, generation it waits for)
    while True:
        live = [n for n, op in cur.items() if op is not None]
        if not live and not later:
            assert not any(b.tags for b in start + done), "named barrier left with arrivals"
            return
        ready = []
        for n in live:
            op = cur[n]
            if n in parked:
                nb, g = parked[n]
                if nb.gen > g:
                    del parked[n]
                    cur[n] = next(roles[n], None)
                    ready.append(None)  # progress was made
                continue
            if op[0] == "wait":
                bar, k = op[1], op[2]
                hw = (bar.c & 1) != (k & 1)
                assert hw == (bar.c >= k + 1), f"{n}: wait for phase {k} of {bar.name} at phase {bar.c}"
                if hw:
                    ready.append(n)
            else:
                ready.append(n)
        if None in ready:
            continue
        choices = ready + (["completion"] if later else [])
        assert choices, "no role can move: " + ", ".join(f"{n} waits {cur[n][1].name}" for n in live)
        choices = [c for c in choices if c not in parked]
        if not choices:
            continue
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
        elif op[0] == "narrive":
            op[1].arrive(op[2], pick)
        elif op[0] == "nsync":
            parked[pick] = (op[1], op[1].arrive(op[2], pick))
            continue
        cur[pick] = next(roles[pick], None)


ROW_BYTES = {"E2M1": 32, "E4M3": 64, "BF16": 128, "TF32": 256}


def launcher_rings(fmt, bn):
    """RSK, SR, NRND and stages in flight as the launcher (PickTmem) and
    TmemCfg choose them."""
    row = ROW_BYTES[fmt]
    rsk = 4 if row <= 64 else 2 if row == 128 else 1
    spr = DK // rsk
    nrnd = 3 if bn <= 32 else 2
    stage = rsk * row * 128
    sr = min(12, (SMEM_BUDGET - 1024 - nrnd * 4 * bn * 128) // stage)
    sr = sr // spr * spr
    inflight = max(1, 96 * 1024 // stage)
    return rsk, sr, nrnd, inflight


UNITS = [[64], [20, 28, 64, 12], [13, 9], [66, 10], [1, 2, 3, 5]]


@pytest.mark.parametrize("fmt", list(ROW_BYTES))
@pytest.mark.parametrize("bn", [16, 32, 64])
def test_launcher_rings(fmt, bn):
    rsk, sr, nrnd, inflight = launcher_rings(fmt, bn)
    assert sr >= DK // rsk and sr % (DK // rsk) == 0
    for i, units in enumerate(UNITS):
        run(units, rsk, sr, nrnd, seed=i, inflight=inflight)


@pytest.mark.parametrize("rsk,sr,nrnd", [(4, 1, 2), (4, 2, 3), (2, 2, 2), (2, 4, 3), (1, 4, 2), (1, 8, 3)])
def test_small_rings(rsk, sr, nrnd):
    for i, units in enumerate(UNITS):
        for inflight in (1, 3, 8):
            run(units, rsk, sr, nrnd, seed=10 + i, inflight=inflight)


@pytest.mark.parametrize("rsk,sr,nrnd", [(4, 2, 2), (4, 3, 3), (2, 4, 2), (1, 8, 3)])
def test_per_warp_protocol_on_deep_rings(rsk, sr, nrnd):
    """The per-warp protocol (used for TF32) is also sound on rings deep
    enough for the sync warp."""
    for i, units in enumerate(UNITS):
        run(units, rsk, sr, nrnd, seed=20 + i, syncw=False)


def test_model_flags_sync_warp_on_one_round_ring():
    """The sync warp waits for round r + 1's raw stages before it releases
    round r's: with a ring of a single round that is a deadlock, which is why
    such rings use the per-warp protocol."""
    with pytest.raises(AssertionError, match="no role can move"):
        run([64], 4, 1, 3, seed=0, syncw=True, inflight=0)


def test_model_flags_inflight_bound_beyond_ring():
    """Waiting for the stage INFLIGHT back when INFLIGHT >= SR reads a slot
    that has already been refilled: the model catches the stale parity."""
    import inspect
    src = inspect.getsource(run).replace("    inflight = min(inflight, SR - 1)\n", "")
    src = src.replace("def run(", "def run_unclamped(")
    ns = dict(globals())
    exec(src, ns)
    with pytest.raises(AssertionError):
        for seed in range(10):
            ns["run_unclamped"]([64], 4, 2, 3, seed=seed, inflight=3)


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
