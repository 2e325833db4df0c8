"""A model of the barrier protocol of the fused decode + GEMM kernel on SM
pairs (tensor-bridge_b200/csrc/fused_pair_kernel.cuh), run under random
schedules.

Both CTAs of a cluster replay, in order, the waits and arrivals their roles
issue: the B producer (the leader's arms the leader's full barrier; each CTA's
TMA bytes land on it later), the raw-A producer (its own raw ring), the decode
warps (wait for the raw stage and for the operand slots of a round in their
own CTA; per k-block the leader's warps arrive on the leader's full barrier
and the second CTA's warps issue a signal copy whose bytes land there later;
free the raw stage after its last k-block), the leader's MMA issuer (one full
wait per k-block; in a tile's first k-block a wait for each 256-column half's
accumulator to be drained right before that half's MMAs; a multicast commit
that lands later on the empty barrier of both CTAs, and per tile one on both
accumulator-full barriers) and the epilogue warps (wait on their own CTA's
accumulator-full barrier, then arrive on the leader's accumulator-empty
barrier of each half as they drain it).  Byte completions (TMA, signal
copies) are modelled as extra arrivals that land later.  The model fails when
an arrival lands in a phase other than the one it is meant for, when a parity
wait would pass (or block) against the intended answer, or when no role can
move.  Ring depths are the ones the launcher picks per format, plus small
rings."""
import inspect
import random

import pytest

from test_ring_protocol import Bar, library_ring_lines

ND = 2  # decode warps per CTA in the model (the kernel has 8 or 16)
NE = 2  # epilogue warps per CTA in the model (the kernel has 4)


def run(num_kb, units, RK, S, SA, DK, seed):
    assert RK % DK == 0 and DK <= S - 1
    rng = random.Random(seed)
    # leader's full barrier: producer arrival, both CTAs' B bytes, the leader's
    # decode warps' arrivals and the second CTA's signal copies
    full = [Bar(f"full{s}", 1 + 2 + 2 * ND) for s in range(S)]
    empty = [[Bar(f"empty{c}.{s}", 1) for s in range(S)] for c in range(2)]
    a_full = [[Bar(f"a_full{c}.{s}", 2) for s in range(SA)] for c in range(2)]
    a_empty = [[Bar(f"a_empty{c}.{s}", ND) for s in range(SA)] for c in range(2)]
    acc_full = [Bar(f"acc_full{c}", 1) for c in range(2)]
    acc_empty = [Bar(f"acc_empty{h}", 2 * NE) for h in range(2)]  # per half
    later = []

    def b_producer(c):
        g = 0
        for _ in range(units):
            for _ in range(num_kb):
                s, use = g % S, g // S
                if use:
                    yield ("wait", empty[c][s], use - 1)
                if c == 0:
                    yield ("arrive", full[s], use)
                yield ("later", full[s], use)
                g += 1

    def raw_producer(c):
        g = 0
        for _ in range(units):
            for _ in range(0, num_kb, RK):
                s, use = g % SA, g // SA
                if use:
                    yield ("wait", a_empty[c][s], use - 1)
                yield ("arrive", a_full[c][s], use)
                yield ("later", a_full[c][s], use)
                g += 1

    def decode(c):
        ga = gd = 0  # raw stages, operand slots
        for _ in range(units):
            for kb in range(0, num_kb, DK):
                cnt = min(DK, num_kb - kb)
                sub0 = kb % RK
                if sub0 == 0:
                    yield ("wait", a_full[c][ga % SA], ga // SA)
                for d in range(cnt):
                    g = gd + d
                    if g // S:
                        yield ("wait", empty[c][g % S], g // S - 1)
                for d in range(cnt):
                    g = gd + d
                    yield ("arrive" if c == 0 else "later", full[g % S], g // S)
                if sub0 + cnt == RK or kb + cnt == num_kb:
                    yield ("arrive", a_empty[c][ga % SA], ga // SA)
                    ga += 1
                gd += cnt

    def mma():
        g = 0
        for t in range(units):
            for kb in range(num_kb):
                yield ("wait", full[g % S], g // S)
                for h in range(2):
                    if kb == 0 and t:
                        yield ("wait", acc_empty[h], t - 1)
                yield ("later", empty[0][g % S], g // S)
                yield ("later", empty[1][g % S], g // S)
                g += 1
            yield ("later", acc_full[0], t)
            yield ("later", acc_full[1], t)

    def epilogue(c):
        for t in range(units):
            yield ("wait", acc_full[c], t)
            for h in range(2):
                yield ("arrive", acc_empty[h], t)

    roles = {"MMA": mma()}
    for c in range(2):
        roles[f"B producer {c}"] = b_producer(c)
        roles[f"raw producer {c}"] = raw_producer(c)
        for j in range(ND):
            roles[f"decode {c}.{j}"] = decode(c)
        for q in range(NE):
            roles[f"epilogue {c}.{q}"] = epilogue(c)
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


SMEM_BUDGET = 224 * 1024
RAW = {"E2M1": (4, 16384), "E4M3": (2, 16384), "BF16": (1, 16384), "TF32": (1, 32768)}


def launcher_rings(fmt):
    """RK, S, SA and DK as the launcher (PickFusedPair) chooses them."""
    rk, stage = RAW[fmt]
    s = 3 if fmt == "TF32" else 4
    sa = min(8, (SMEM_BUDGET - s * 3 * 128 * 128) // stage)
    dk = min(rk, 2)
    return rk, s, sa, dk


@pytest.mark.parametrize("fmt", list(RAW))
@pytest.mark.parametrize("num_kb,units", [(1, 3), (5, 4), (9, 5), (16, 2)])
def test_launcher_rings(fmt, num_kb, units):
    rk, s, sa, dk = launcher_rings(fmt)
    assert sa >= 2
    for seed in range(3):
        run(num_kb, units, rk, s, sa, dk, seed=seed)


def test_model_rings_are_the_librarys():
    """The Python copy of the launcher's ring rules (launcher_rings) gives the
    library's own choices (tests/ring_cfg_probe.cu)."""
    lines = library_ring_lines()
    if lines is None:
        pytest.skip("nvcc not available")
    pairs = {f[1]: tuple(int(v) for v in f[2:]) for f in lines if f[0] == "PAIR"}
    assert set(pairs) == set(RAW)
    for fmt, cfg in pairs.items():
        assert launcher_rings(fmt) == cfg, fmt


@pytest.mark.parametrize("rk,s,sa,dk", [(4, 2, 2, 1), (4, 3, 2, 2), (2, 3, 3, 2), (1, 2, 2, 1), (4, 5, 2, 4)])
def test_small_rings(rk, s, sa, dk):
    for i, (num_kb, units) in enumerate([(3, 3), (7, 4), (13, 2)]):
        run(num_kb, units, rk, s, sa, dk, seed=40 + i)


def test_model_flags_missing_peer_wait():
    """A decode warp of the second CTA that writes an operand slot without
    waiting for the pair's MMAs to release it lands its signal on the
    leader's full barrier in the wrong phase: the model catches it."""
    src = inspect.getsource(run)
    src = src.replace("                    if g // S:\n                        yield (\"wait\", empty[c][g % S], g // S - 1)\n",
                      "                    if g // S and c == 0:\n                        yield (\"wait\", empty[c][g % S], g // S - 1)\n")
    assert "and c == 0" in src
    src = src.replace("def run(", "def run_unsafe(")
    ns = dict(globals())
    exec(src, ns)
    failures = 0
    for seed in range(20):
        try:
            ns["run_unsafe"](9, 3, 2, 3, 3, 2, seed=seed)
        except AssertionError:
            failures += 1
    assert failures > 0
