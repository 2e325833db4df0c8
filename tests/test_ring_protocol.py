"""A model of the mbarrier protocol of the narrow fused kernel
(tensor-bridge_b200/csrc/fused_tmem_kernel.cuh), run under random schedules.

Each role replays, in order, the waits and arrivals the kernel issues: the raw-A
producer, the B producer, the MMA issuer (rounds of four k-blocks; its commits
land later, like MMA completion), the epilogue and the sixteen decode warps
(every warp walks every raw stage; the owner slice of a k-block is its CTA-wide
index mod 4).  TMA completions also land later.  A wait is modelled the way the
hardware answers a parity wait -- it passes when the barrier's current phase
parity differs from the waited one -- and the model fails when that answer
differs from the intended one (the phase completed or not), when an arrival
lands in a phase other than the one it is meant for, or when no role can move.
The ring depths are the ones the launcher picks for each format and tile width,
plus small rings."""
import random

import pytest

SMEM_BUDGET = 224 * 1024


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.c, self.pending = name, count, 0, 0

    def arrive(self, k, who):
        assert k == self.c, f"{who}: arrival meant for phase {k} of {self.name} lands in phase {self.c}"
        self.pending += 1
        if self.pending == self.count:
            self.pending, self.c = 0, self.c + 1


def run(units, RK, SR, SB, TS, seed, DK=4, NS=4):
    rng = random.Random(seed)
    raw_full = [Bar(f"raw_full{i}", 2) for i in range(SR)]  # producer arrive + TMA bytes
    raw_empty = [Bar(f"raw_empty{i}", 4 * NS) for i in range(SR)]
    b_full = [Bar(f"b_full{i}", 2) for i in range(SB)]
    b_empty = [Bar(f"b_empty{i}", 1) for i in range(SB)]
    t_full = [Bar(f"t_full{i}", 4) for i in range(TS)]
    t_empty = [Bar(f"t_empty{i}", 1) for i in range(TS)]
    acc_full = [Bar(f"acc_full{i}", 1) for i in range(2)]
    acc_empty = [Bar(f"acc_empty{i}", 1) for i in range(2)]
    later = []

    def raw_producer():
        use, s = [0] * SR, 0
        for nkb in units:
            for _ in range(0, nkb, RK):
                if use[s]:
                    yield ("wait", raw_empty[s], use[s] - 1)
                yield ("arrive", raw_full[s], use[s])
                yield ("later", raw_full[s], use[s])
                use[s] += 1
                s = (s + 1) % SR

    def b_producer():
        use, s = [0] * SB, 0
        for nkb in units:
            for _ in range(nkb):
                if use[s]:
                    yield ("wait", b_empty[s], use[s] - 1)
                yield ("arrive", b_full[s], use[s])
                yield ("later", b_full[s], use[s])
                use[s] += 1
                s = (s + 1) % SB

    def mma():
        buse, tuse, bs, ts = [0] * SB, [0] * TS, 0, 0
        for ui, nkb in enumerate(units):
            acc, k = ui & 1, ui >> 1
            if k:
                yield ("wait", acc_empty[acc], k - 1)
            for kb in range(0, nkb, DK):
                done = []
                for _ in range(min(DK, nkb - kb)):
                    yield ("wait", b_full[bs], buse[bs])
                    yield ("wait", t_full[ts], tuse[ts])
                    done.append((bs, buse[bs], ts, tuse[ts]))
                    buse[bs] += 1
                    tuse[ts] += 1
                    bs, ts = (bs + 1) % SB, (ts + 1) % TS
                for b, bk, t, tk in done:
                    yield ("later", t_empty[t], tk)
                    yield ("later", b_empty[b], bk)
            yield ("later", acc_full[acc], k)

    def epilogue():
        for ui, _ in enumerate(units):
            acc, k = ui & 1, ui >> 1
            yield ("wait", acc_full[acc], k)
            yield ("arrive", acc_empty[acc], k)

    def decode(j):
        ruse, tuse, rs, ts, t = [0] * SR, [0] * TS, 0, 0, 0
        for nkb in units:
            for kb in range(0, nkb, RK):
                nk = min(RK, nkb - kb)
                yield ("wait", raw_full[rs], ruse[rs])
                sub = (j - t) & 3
                if sub < nk:
                    tk = (ts + sub) % TS
                    if tuse[tk]:
                        yield ("wait", t_empty[tk], tuse[tk] - 1)
                    yield ("arrive", raw_empty[rs], ruse[rs])
                    yield ("arrive", t_full[tk], tuse[tk])
                else:
                    yield ("arrive", raw_empty[rs], ruse[rs])
                for d in range(nk):
                    tuse[(ts + d) % TS] += 1
                ruse[rs] += 1
                t, ts, rs = t + nk, (ts + nk) % TS, (rs + 1) % SR

    roles = {"raw producer": raw_producer(), "B producer": b_producer(), "MMA": mma(), "epilogue": epilogue()}
    for q in range(4):
        for j in range(NS):
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


def launcher_rings(fmt_rk, stage_bytes, bn):
    """SB, SR and TS as the launcher and TmemCfg choose them."""
    sb = 16 if bn <= 16 else 8
    sr = min(12, (SMEM_BUDGET - 1024 - sb * bn * 128) // stage_bytes)
    nacc = 4 if bn <= 16 else 2
    ts = min(12, (512 - 2 * nacc * bn) // 32)
    return sr, sb, ts


FORMATS = {"E2M1": (4, 16384), "E4M3": (2, 16384), "BF16": (1, 16384), "TF32": (1, 32768)}
UNITS = [[64], [5, 7, 16, 3], [13, 9], [66, 10]]


@pytest.mark.parametrize("fmt", list(FORMATS))
@pytest.mark.parametrize("bn", [16, 64])
def test_launcher_rings(fmt, bn):
    rk, stage = FORMATS[fmt]
    sr, sb, ts = launcher_rings(rk, stage, bn)
    for i, units in enumerate(UNITS):
        run(units, rk, sr, sb, ts, seed=i)


@pytest.mark.parametrize("rk,sr,sb", [(1, 5, 4), (2, 3, 4), (4, 4, 4), (1, 4, 8)])
def test_small_rings(rk, sr, sb):
    for i, units in enumerate(UNITS):
        run(units, rk, sr, sb, 8, seed=10 + i)


def test_model_flags_partial_raw_waits():
    """The earlier scheme -- each decode warp waiting only for the raw stages
    it reads -- is caught: with one k-block per stage and five stages a warp's
    parity wait can pass on the previous phase."""
    import inspect
    src = inspect.getsource(run)
    old = src.replace('raw_empty = [Bar(f"raw_empty{i}", 4 * NS) for i in range(SR)]',
                      'raw_empty = [Bar(f"raw_empty{i}", 4 * RK) for i in range(SR)]')
    old = old.replace('''                yield ("wait", raw_full[rs], ruse[rs])
                sub = (j - t) & 3''', '''                sub = (j - t) & 3
                if sub < nk:
                    yield ("wait", raw_full[rs], ruse[rs])''')
    old = old.replace('''                else:
                    yield ("arrive", raw_empty[rs], ruse[rs])''', '')
    old = old.replace("def run(", "def run_old(")
    ns = dict(globals())
    exec(old, ns)
    failures = 0
    for seed in range(5):
        try:
            ns["run_old"]([64], 1, 5, 16, 12, seed=seed)
        except AssertionError:
            failures += 1
    assert failures > 0
