"""A model of the barrier protocol of the narrow fused kernel
(tensor-bridge_b200/csrc/fused_tmem_kernel.cuh), run under random schedules.

Each role replays, in order, the waits and arrivals the kernel issues: the raw-A
producer (SPR raw stages per round of four k-blocks, at most `inflight` stages
in flight), the B producer (a ring of NBR round slots of its own: b_empty
wait, one arrival with the round's bytes on b_full), the MMA issuer (b_full
and rdy waits, one fre and one b_empty commit per round; commits land later,
like MMA completion), the epilogue and the decode warps.  In group mode (a raw
ring of at least NRND rounds) NG groups of eight decode warps take whole
rounds in turn: each warp of group g waits for the round's TMEM slot (fre),
then for its raw stages, and arrives on raw_empty and rdy.  In per-warp mode sixteen decode warps each
decode one k-block of every round (slice j reads raw stage position j // RSK)
and wait and arrive themselves.  TMA completions also land later.  An mbarrier
wait is modelled the way the hardware answers a parity wait -- it passes when
the barrier's current phase parity differs from the waited one -- and the
model fails when that answer differs from the intended one (the phase
completed or not), when an arrival lands in a phase other than the one it is
meant for, or when no role can move.  The ring depths are the ones the
launcher picks for each format and tile width, plus small rings."""
import functools
import os
import random
import shutil
import subprocess
import tempfile

import pytest

SMEM_BUDGET = 224 * 1024
DK = 4
GW = 8  # decode warps per group


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.c, self.pending = name, count, 0, 0

    def arrive(self, k, who):
        assert k == self.c, f"{who}: arrival meant for phase {k} of {self.name} lands in phase {self.c}"
        self.pending += 1
        if self.pending == self.count:
            self.pending, self.c = 0, self.c + 1


def run(units, RSK, SR, NRND, seed, mode=None, ng=None, inflight=2, raw_first=False, nbr=2):
    """units: k-blocks per work unit of this CTA, in order; inflight: raw
    stages the producer keeps in flight (fewer than SR, as in TmemCfg: the
    stage it waits for must not have been refilled; 0 = no bound).  mode:
    "groups" or "warps" (default: as TmemCfg picks); ng: decode groups in
    group mode (default NRND); raw_first: a group waits for its raw stages
    before its TMEM slot (the order the kernel does not use)."""
    SPR = DK // RSK
    inflight = min(inflight, SR - 1)
    if mode is None:
        mode = "groups" if SR // SPR >= NRND else "warps"
    ng = NRND if ng is None else ng
    rng = random.Random(seed)
    raw_full = [Bar(f"raw_full{i}", 2) for i in range(SR)]  # producer arrive + TMA bytes
    raw_empty = [Bar(f"raw_empty{i}", GW if mode == "groups" else 4 * RSK) for i in range(SR)]
    rdy = [Bar(f"rdy{i}", GW if mode == "groups" else 16) for i in range(NRND)]  # decode warps
    fre = [Bar(f"fre{i}", 1) for i in range(NRND)]
    b_full = [Bar(f"b_full{i}", 2) for i in range(nbr)]  # B arrive + B bytes
    b_empty = [Bar(f"b_empty{i}", 1) for i in range(nbr)]
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
                bs, buse = r % nbr, r // nbr
                if buse:
                    yield ("wait", b_empty[bs], buse - 1)
                yield ("arrive", b_full[bs], buse)
                yield ("later", b_full[bs], buse)
                r += 1

    def mma():
        r = 0
        for ui, nr in enumerate(rounds):
            acc, k = ui & 1, ui >> 1
            if k:
                yield ("wait", acc_empty[acc], k - 1)
            for _ in range(nr):
                slot, use = r % NRND, r // NRND
                bs, buse = r % nbr, r // nbr
                yield ("wait", b_full[bs], buse)
                yield ("wait", rdy[slot], use)
                yield ("later", fre[slot], use)
                yield ("later", b_empty[bs], buse)
                r += 1
            yield ("later", acc_full[acc], k)

    def epilogue():
        for ui, _ in enumerate(rounds):
            acc, k = ui & 1, ui >> 1
            yield ("wait", acc_full[acc], k)
            yield ("arrive", acc_empty[acc], k)

    def group_warp(g):
        r = 0
        for nr in rounds:
            for _ in range(nr):
                if r % ng == g:
                    slot, use = r % NRND, r // NRND
                    stages = [r * SPR + pos for pos in range(SPR)]
                    raw_waits = [("wait", raw_full[st % SR], st // SR) for st in stages]
                    slot_wait = [("wait", fre[slot], use - 1)] if use else []
                    for op in (raw_waits + slot_wait if raw_first else slot_wait + raw_waits):
                        yield op
                    for st in stages:
                        yield ("arrive", raw_empty[st % SR], st // SR)
                    yield ("arrive", rdy[slot], use)
                r += 1

    def slice_warp(j):
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
        if mode == "groups":
            for g in range(ng):
                for h in range(GW // 4):
                    roles[f"decode q{q} h{h} g{g}"] = group_warp(g)
        else:
            for j in range(4):
                roles[f"decode q{q} s{j}"] = slice_warp(j)
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
    """RSK, SR, NRND, stages in flight and B ring slots as the launcher
    (PickTmem) and TmemCfg choose them."""
    row = ROW_BYTES[fmt]
    rsk = 4 if row <= 64 else 2 if row == 128 else 1
    spr = DK // rsk
    nrnd = 3 if bn <= 32 else 2
    stage = rsk * row * 128
    bround = DK * bn * 128
    avail = SMEM_BUDGET - 1024
    nbr_t = max(2, min(8, 65536 // bround))
    nbr_g = (avail - nrnd * spr * stage) // bround
    nbr = nbr_g if 2 <= nbr_g < nbr_t else nbr_t
    sr = min(12, (avail - nbr * bround) // stage)
    sr = sr // spr * spr
    cap = 65536 // stage if stage <= 16384 else sr - 1
    inflight = min(sr - 1, cap)
    return rsk, sr, nrnd, inflight, nbr


UNITS = [[64], [20, 28, 64, 12], [13, 9], [66, 10], [1, 2, 3, 5]]


@functools.lru_cache(maxsize=1)
def library_ring_lines():
    """The ring configurations the library itself picks, as printed by
    tests/ring_cfg_probe.cu (host code built with nvcc; no GPU needed):
    {(kind, format, ...): values}.  None without nvcc."""
    if shutil.which("nvcc") is None:
        return None
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "ring_cfg_probe")
        subprocess.run(["nvcc", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
                        "-I" + os.path.join(root, "include"), "-I" + os.path.join(root, "tensor-bridge_b200", "csrc"),
                        os.path.join(root, "tests", "ring_cfg_probe.cu"), "-o", exe],
                       check=True, capture_output=True, timeout=600)
        out = subprocess.run([exe], check=True, capture_output=True, text=True, timeout=60).stdout
    return [line.split() for line in out.splitlines() if line.strip()]


@pytest.fixture(scope="module")
def library_rings():
    lines = library_ring_lines()
    if lines is None:
        pytest.skip("nvcc not available")
    return {(f[1], int(f[2])): tuple(int(v) for v in f[3:]) for f in lines if f[0] == "TMEM"}


def test_model_rings_are_the_librarys(library_rings):
    """The Python copy of the launcher's ring rules (launcher_rings) gives the
    library's own choices, so the protocol model runs the rings the kernel
    runs."""
    assert library_rings
    for (fmt, bn), (rsk, sr, nrnd, nbr, inflight, groups) in library_rings.items():
        m_rsk, m_sr, m_nrnd, m_inflight, m_nbr = launcher_rings(fmt, bn)
        assert (m_rsk, m_sr, m_nrnd, m_nbr, m_inflight) == (rsk, sr, nrnd, nbr, inflight), (fmt, bn)
        assert groups == (1 if m_sr // (DK // m_rsk) >= m_nrnd else 0), (fmt, bn)


@pytest.mark.parametrize("fmt", list(ROW_BYTES))
@pytest.mark.parametrize("bn", [16, 32, 64])
def test_launcher_rings(fmt, bn):
    rsk, sr, nrnd, inflight, nbr = launcher_rings(fmt, bn)
    assert sr >= DK // rsk and sr % (DK // rsk) == 0
    for i, units in enumerate(UNITS):
        run(units, rsk, sr, nrnd, seed=i, inflight=inflight, nbr=nbr)


@pytest.mark.parametrize("rsk,sr,nrnd", [(4, 1, 2), (4, 2, 3), (2, 2, 2), (2, 4, 3), (1, 4, 2), (1, 8, 3)])
def test_small_rings(rsk, sr, nrnd):
    for i, units in enumerate(UNITS):
        for inflight in (1, 3, 8):
            run(units, rsk, sr, nrnd, seed=10 + i, inflight=inflight)


@pytest.mark.parametrize("rsk,sr,nrnd", [(4, 2, 2), (4, 3, 3), (2, 4, 2), (1, 8, 3)])
def test_per_warp_protocol_on_deep_rings(rsk, sr, nrnd):
    """The per-warp protocol (used for TF32) is also sound on rings deep
    enough for the groups."""
    for i, units in enumerate(UNITS):
        run(units, rsk, sr, nrnd, seed=20 + i, mode="warps")


def _fails(**kw):
    failures = 0
    for seed in range(40):
        for units in UNITS:
            try:
                run(units, seed=seed, **kw)
            except AssertionError:
                failures += 1
    return failures


def test_model_flags_more_groups_than_round_slots():
    """With more decode groups than TMEM round slots a group can reach round
    r while the MMAs of round r - 2 NRND have not run: its parity wait on the
    slot passes on a stale phase.  The kernel uses NG = NRND."""
    assert _fails(RSK=4, SR=6, NRND=2, mode="groups", ng=3, inflight=0) > 0


def test_model_flags_raw_ring_shorter_than_round_slots():
    """With a raw ring of fewer than NRND rounds the slot wait no longer
    implies that the previous fill of each raw stage has landed: the raw wait
    can pass on a stale phase.  The kernel uses group mode only when the ring
    holds NRND rounds."""
    assert _fails(RSK=4, SR=2, NRND=3, mode="groups", inflight=0) > 0


def test_model_flags_raw_wait_before_slot_wait():
    """Waiting for the raw stages before the round's TMEM slot loses the
    guarantee when the ring depth is not a multiple of the group count (the
    group did not itself wait on the slot's previous fill): it can see a raw
    slot two fills behind.  Slot first, the same ring is sound."""
    assert _fails(RSK=4, SR=4, NRND=3, mode="groups", inflight=0, raw_first=True) > 0
    assert _fails(RSK=4, SR=4, NRND=3, mode="groups", inflight=0) == 0


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
