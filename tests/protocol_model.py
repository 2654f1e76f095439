"""A model of the decode GEMM's barrier protocol (nano-vllm-cpp26_b200/csrc/
gemm_decode_tc.cu, one CTA), run under random interleavings on the CPU.

Roles are generators over the CTA's units in the kernel's order: the producer
(refills ring slot g % S once the MMAs of unit g - S completed), two converter
groups (alternate units; a unit needs its TMA data and the MMAs of unit
g - ABUFS, which last read its A buffer; group 0 also folds every chunk two
units after it ends), and the MMA issuers (a unit needs its conversion, the
first unit of a chunk also its accumulator folded two chunks back). TMA copies
land and an issuer's MMAs complete at random later times, the MMAs of one
issuer in issue order. A wait on parity P passes when the barrier's completed
phase count C has C & 1 != P, the mbarrier rule; the model records a wait that
passes without its own phase completed (C != wanted + 1) and a state in which
nothing can move."""
import random


class Bar:
    def __init__(self, name, counter):
        self.name, self.C, self.counter = name, 0, counter

    def arrive(self):
        self.counter[0] += 1
        self.C += 1


def segments(nu, spt, stage0):
    """(index within its tile's segment, segment length) of every unit"""
    out, stage, j, ln = [], stage0, 0, 0
    for g in range(nu):
        if g == 0 or stage == 0:
            j, ln = 0, min(spt - stage, nu - g)
        out.append((j, ln))
        j += 1
        stage = 0 if stage + 1 == spt else stage + 1
    return out


def rule_by_unit(g, rel, ln, issuers, chunk):
    """the kernel's rule: unit g to issuer g % issuers; chunks are windows of
    issuers * chunk units of the segment"""
    w = rel % (issuers * chunk)
    return g % issuers, w < issuers, w >= issuers * (chunk - 1) or rel + issuers >= ln


def rule_by_segment(g, rel, ln, issuers, chunk):
    """an earlier rule: the unit's position in its segment picks the issuer"""
    ji = rel // issuers
    return rel % issuers, ji % chunk == 0, ji % chunk == chunk - 1 or rel + issuers >= ln


def simulate(nu, spt, stage0, rule=rule_by_unit, issuers=2, stages=8, abufs=4, chunk=4, lag=2,
             seed=0):
    rng = random.Random(seed)
    sch = segments(nu, spt, stage0)
    counter = [0]
    full = [Bar(f"full{i}", counter) for i in range(stages)]
    conv = [Bar(f"conv{i}", counter) for i in range(stages)]
    empty = [Bar(f"empty{i}", counter) for i in range(stages)]
    dfull = [[Bar(f"dfull{i}.{b}", counter) for b in range(2)] for i in range(issuers)]
    dfree = [[Bar(f"dfree{i}.{b}", counter) for b in range(2)] for i in range(issuers)]
    events, now, errors = [], [0], []
    queued = [[] for _ in range(issuers)]

    def later(fn, lo, hi):
        events.append((now[0] + rng.randint(lo, hi), fn))

    def wait(bar, c):
        while (bar.C & 1) == (c & 1):
            yield "wait"
        if bar.C != c + 1:
            errors.append(f"{bar.name}: passed for completion {c} at {bar.C}")

    def producer():
        for g in range(nu):
            if g >= stages:
                yield from wait(empty[g % stages], g // stages - 1)
            later(lambda s=g % stages: full[s].arrive(), 5, 200)
            yield "run"

    def complete(me):
        for b in queued[me].pop(0):
            b.arrive()

    def issuer(me):
        q = 0
        for g in range(nu):
            rel, ln = sch[g]
            who, first, last = rule(g, rel, ln, issuers, chunk)
            if who != me:
                continue
            yield from wait(conv[g % stages], g // stages)
            if first and q >= 2:
                yield from wait(dfree[me][q & 1], (q >> 1) - 1)
            commits = [empty[g % stages]]
            if last:
                commits.append(dfull[me][q & 1])
                q += 1
            queued[me].append(commits)
            later(lambda me=me: complete(me), 1, 60)
            yield "run"

    def converters(grp):
        folded = [0] * issuers
        pending = []

        def fold(i):
            yield from wait(dfull[i][folded[i] & 1], folded[i] >> 1)
            dfree[i][folded[i] & 1].arrive()
            folded[i] += 1

        for g in range(nu):
            rel, ln = sch[g]
            who, _, last = rule(g, rel, ln, issuers, chunk)
            if g % 2 == grp:
                yield from wait(full[g % stages], g // stages)
                if g >= abufs:
                    h = g - abufs
                    yield from wait(empty[h % stages], h // stages)
                yield "run"
                conv[g % stages].arrive()
            if grp != 0:
                continue
            while pending and pending[0][0] + lag <= g:
                yield from fold(pending.pop(0)[1])
            if len(pending) > 1:
                errors.append("fold queue over capacity")
            if last:
                pending.append((g, who))
        for _, i in pending:
            yield from fold(i)

    roles = [producer(), converters(0), converters(1)] + [issuer(i) for i in range(issuers)]
    alive = list(range(len(roles)))
    for _ in range(2_000_000):
        if not alive and not events:
            return errors
        events.sort(key=lambda e: e[0])
        moved = False
        while events and events[0][0] <= now[0]:
            events.pop(0)[1]()
            moved = True
        before = counter[0]
        order = alive[:]
        rng.shuffle(order)
        for r in order:
            try:
                if next(roles[r]) == "run":
                    moved = True
            except StopIteration:
                alive.remove(r)
                moved = True
        moved = moved or counter[0] != before
        if not moved:
            if not events:
                return errors + ["deadlock"]
            now[0] = min(e[0] for e in events)
        else:
            now[0] += 1
    return errors + ["no end"]


def cta_ranges(k, n, batch, sms=148, min_units=8, tile_n=128, stage_k=32):
    """(units, spt, first unit) of every CTA of the kernel's stream-K plan"""
    tiles = ((n + tile_n - 1) // tile_n) * batch
    spt = (k + stage_k - 1) // stage_k
    units = tiles * spt
    ctas = max(1, min(sms, units // min_units))
    for c in range(ctas):
        u0 = c * units // ctas
        yield (c + 1) * units // ctas - u0, spt, u0
