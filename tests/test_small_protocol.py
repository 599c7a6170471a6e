"""CPU model of the synchronisation protocol of the small-batch decoder (k_small_decode in
sigcomp_b200/csrc/sc_mlp_small.cuh), run under randomised interleavings.

One cluster of C CTAs (C = 4 here; the protocol does not depend on C) decodes tiles one after the
other.  Roles per CTA, with the kernel's unit walk (tile, step, layer), counters and parity
formulas: the TMA producer, the MMA issuer and the epilogue (its four warps, with the bounded
slice counter and the one thread that sends the slice; rank 0's epilogue also runs the coder step).

Barriers per CTA: full0/empty0 (layer-0 stages), full1/empty1 (weight stages), acc_full,
acc_empty (4 warps), xbar[2] (one local expect-tx arrival plus the C-1 peers' bulk copies),
lbar (rank 0: the same for the logit slices), rbar (4 arrivals from rank 0's warps).  TMA loads
and bulk copies complete asynchronously; MMAs complete in issue order, and a commit arrives once
every MMA issued before it has completed.

Shared memory is modelled by the regions the kernel overlays (in KB): B0 [0, 64), B1 [64, 128),
layer-0 stage s at [64 + 24 s, 88 + 24 s), weight stage s at [128 + 8 s, 136 + 8 s).  The model
checks the kernel's ordering claims directly:

- an MMA of layer L >= 1 reads B[(L-1) & 1] holding every CTA's slice of layer L-1 of its step;
- no write (a TMA load, a bulk copy landing, an epilogue store) touches a region that an MMA still
  in flight reads, or a buffer whose contents are still to be read;
- layer 0 reads, for window position k, the ring slot holding the token of step `step - W + k`,
  and rank 0 never overwrites a ring slot that a load in flight is reading;
- the coder reads all C logit slices of its step;
- every parity wait is within one phase of its target (so consecutive exchanges never mix), no
  barrier receives more arrivals than its count, and every role finishes.
"""

import random

import pytest

NL = 9
C = 4                 # CTAs per cluster in the model
W = 8                 # window positions = layer-0 K blocks (64 in the kernel)
S0, S1 = 6, 10        # layer-0 stages, weight stages
HID_KB = 4            # K blocks of a hidden or last layer


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.pending, self.tx, self.completed = name, count, count, 0, 0

    def arrive(self, n=1):
        self.pending -= n
        assert self.pending >= 0, f"{self.name}: more arrivals than its count in phase {self.completed}"
        self._check()

    def expect_tx(self, b):
        self.tx += b

    def complete_tx(self, b):
        self.tx -= b
        self._check()

    def _check(self):
        if self.pending == 0 and self.tx == 0:
            self.completed += 1
            self.pending = self.count


def parity_wait(bar, parity, target):
    """try_wait.parity, asserting that the barrier is within one phase of `target` (the completed
    phases the waiter needs)."""
    while True:
        c = bar.completed
        assert target - 1 <= c <= target, f"{bar.name}: waiter targets phase {target}, barrier at {c}"
        if (c & 1) != parity:
            return
        yield


def regions_overlap(a, b):
    return a[0] < b[1] and b[0] < a[1]


B_REG = [(0, 64), (64, 128)]
ST0 = [(64 + 24 * s, 88 + 24 * s) for s in range(S0)]
ST1 = [(128 + 8 * s, 136 + 8 * s) for s in range(S1)]


def units(tiles):
    for tile, steps in enumerate(tiles):
        for step in range(steps):
            for L in range(NL):
                yield tile, step, L


def simulate(tiles, seed, plant=None):
    """Run one cluster over `tiles` (the step count of each tile, decoded one after the other).
    `plant` injects one protocol mistake (tests of the model itself): 'one_xbar' (every exchange
    on the same barrier), 'no_switch_wait' (the producer refills the other stage ring without
    waiting for the one it leaves), 'early_ring' (layer 0 loads its newest window block without
    waiting for rank 0's release)."""
    rng = random.Random(seed)
    full0 = [[Bar(f"full0[{s}]/{c}", 1) for s in range(S0)] for c in range(C)]
    empty0 = [[Bar(f"empty0[{s}]/{c}", 1) for s in range(S0)] for c in range(C)]
    full1 = [[Bar(f"full1[{s}]/{c}", 1) for s in range(S1)] for c in range(C)]
    empty1 = [[Bar(f"empty1[{s}]/{c}", 1) for s in range(S1)] for c in range(C)]
    acc_full = [Bar(f"acc_full/{c}", 1) for c in range(C)]
    acc_empty = [Bar(f"acc_empty/{c}", 4) for c in range(C)]
    xbar = [[Bar(f"xbar[{b}]/{c}", 1) for b in range(2)] for c in range(C)]
    lbar = Bar("lbar/0", 1)
    rbar = [Bar(f"rbar/{c}", 4) for c in range(C)]
    # bufs[c][b][o]: unit (tile, step, layer) of owner o's slice in CTA c's buffer B[b]
    bufs = [[[None] * C for _ in range(2)] for _ in range(C)]
    # live[c][b]: what B[b] of CTA c holds until it is read (a layer's slices, the logits, or a
    # CTA's staged logit slice until its copy has left); None when it may be overwritten
    live = [[None, None] for _ in range(C)]
    ring = [None] * W                        # (tile, step) of the token each ring slot holds
    loads = []                               # TMA loads in flight: (cta, region, bar, bytes, ring slot)
    copies = []                              # bulk copies in flight
    mmas = [[] for _ in range(C)]            # per CTA, in issue order: (kind, what)
    logit_units = [None] * C                 # rank 0: unit of each CTA's logit slice in its B0
    decoded = []

    def in_flight_reads(c):
        return [r for kind, what in mmas[c] if kind == "mma" for r in what]

    def check_write(c, region, what, unit=None):
        for r in in_flight_reads(c):
            assert not regions_overlap(r, region), f"{what} lands in CTA {c} on a region an MMA still reads"
        for b in range(2):
            if regions_overlap(B_REG[b], region) and live[c][b] is not None:
                assert live[c][b] == unit, f"{what} overwrites B{b} of CTA {c} holding {live[c][b]}"

    def put_slice(c, b, owner, unit):
        check_write(c, B_REG[b], f"slice {unit} from CTA {owner}", ("layer",) + unit)
        live[c][b] = ("layer",) + unit
        bufs[c][b][owner] = unit

    def producer(c):
        it0 = it1 = rw = 0
        last_ring, first = -1, True
        for tile, step, L in units(tiles):
            rg = 0 if L == 0 else 1
            if rg != last_ring and last_ring >= 0 and plant != "no_switch_wait":
                i = (it1 if last_ring else it0) - 1
                if last_ring:
                    yield from parity_wait(empty1[c][i % S1], (i // S1) & 1, i // S1 + 1)
                else:
                    yield from parity_wait(empty0[c][i % S0], (i // S0) & 1, i // S0 + 1)
            last_ring = rg
            if L == 0:
                for kb in range(W):
                    s, u = it0 % S0, it0 // S0
                    yield from parity_wait(empty0[c][s], (u & 1) ^ 1, u)
                    check_write(c, ST0[s], "a layer-0 stage load")
                    full0[c][s].expect_tx(24)
                    full0[c][s].arrive()
                    loads.append((c, ST0[s], full0[c][s], 8, None))          # this CTA's weight slice
                    it0 += 1
                    if kb == W - 1:
                        # every layer 0 but the cluster's first consumes one release of rank 0
                        if not first and plant != "early_ring":
                            yield from parity_wait(rbar[c], rw & 1, rw + 1)
                        rw += 0 if first else 1
                        first = False
                    tau = step - W + kb
                    if tau >= 0:
                        assert ring[tau % W] == (tile, tau), \
                            f"step {step} loads window position {kb} from a slot holding {ring[tau % W]}"
                    loads.append((c, ST0[s], full0[c][s], 16, tau % W if tau >= 0 else None))
                    yield
            else:
                for kb in range(HID_KB):
                    s, u = it1 % S1, it1 // S1
                    yield from parity_wait(empty1[c][s], (u & 1) ^ 1, u)
                    check_write(c, ST1[s], "a weight stage load")
                    full1[c][s].expect_tx(8)
                    full1[c][s].arrive()
                    loads.append((c, ST1[s], full1[c][s], 8, None))
                    it1 += 1
                    yield

    def mma(c):
        it0 = it1 = uu = xm = 0
        for tile, step, L in units(tiles):
            yield from parity_wait(acc_empty[c], (uu & 1) ^ 1, uu)
            if L != 0:
                if plant == "one_xbar":
                    yield from parity_wait(xbar[c][0], xm & 1, xm + 1)
                else:
                    yield from parity_wait(xbar[c][xm & 1], (xm >> 1) & 1, (xm >> 1) + 1)
                xm += 1
                b = (L - 1) & 1
                assert all(bufs[c][b][o] == (tile, step, L - 1) for o in range(C)), \
                    f"CTA {c} layer {L} of step {step} reads B{b} before every slice of layer {L - 1} is in"
                for kb in range(HID_KB):
                    i = it1 + kb
                    yield from parity_wait(full1[c][i % S1], (i // S1) & 1, i // S1 + 1)
                mmas[c].append(("mma", [B_REG[b]] + [ST1[(it1 + kb) % S1] for kb in range(HID_KB)]))
                mmas[c].append(("consume", b))
                mmas[c].append(("commit", acc_full[c]))
                for kb in range(HID_KB):
                    mmas[c].append(("commit", empty1[c][(it1 + kb) % S1]))
                it1 += HID_KB
            else:
                for kb in range(W):
                    s = it0 % S0
                    yield from parity_wait(full0[c][s], (it0 // S0) & 1, it0 // S0 + 1)
                    mmas[c].append(("mma", [ST0[s]]))
                    mmas[c].append(("commit", empty0[c][s]))
                    it0 += 1
                    yield
                mmas[c].append(("commit", acc_full[c]))
            uu += 1
            yield

    def epilogue(c):
        ue = lw = xe = 0
        for tile, step, L in units(tiles):
            yield from parity_wait(acc_full[c], ue & 1, ue + 1)
            ue += 1
            acc_empty[c].arrive(4)                  # the four warps release the accumulator
            if L != NL - 1:
                b = L & 1
                for cp in copies:                   # this CTA's earlier slice must have left
                    assert not (cp[0] == "slice" and cp[2] == c and cp[3] == b), \
                        f"CTA {c} overwrites its slice in B{b} while a copy of it is in flight"
                put_slice(c, b, c, (tile, step, L))
                yield
                xb = xbar[c][0 if plant == "one_xbar" else xe & 1]
                xb.expect_tx(8 * (C - 1))
                xb.arrive()
                for d in range(C):
                    if d != c:
                        copies.append(("slice", d, c, b, (tile, step, L), xbar[d][0 if plant == "one_xbar" else xe & 1]))
                xe += 1
                continue
            if c != 0:
                check_write(c, B_REG[0], "a logit slice staged", ("stage", tile, step))
                live[c][0] = ("stage", tile, step)
                copies.append(("logits", 0, c, 0, (tile, step), lbar))
                yield
                continue
            check_write(0, B_REG[0], "rank 0's logit slice", ("logits", tile, step))
            live[0][0] = ("logits", tile, step)
            logit_units[0] = (tile, step)
            yield
            lbar.expect_tx(4 * (C - 1))
            lbar.arrive()
            yield from parity_wait(lbar, lw & 1, lw + 1)
            lw += 1
            assert all(u == (tile, step) for u in logit_units), f"the coder of step {step} reads a stale logit slice"
            live[0][0] = None                       # read into TMEM
            slot = step % W
            assert not [ld for ld in loads if ld[4] == slot], "rank 0 overwrites a ring slot a load still reads"
            ring[slot] = (tile, step)
            decoded.append((tile, step))
            yield
            for d in range(C):
                rbar[d].arrive(4)
            yield

    def land():
        """Complete one asynchronous operation: a load, a bulk copy, or a CTA's oldest MMA entry."""
        kinds = (["load"] if loads else []) + (["copy"] if copies else []) + \
                (["mma"] if any(mmas) else [])
        kind = rng.choice(kinds)
        if kind == "load":
            c, region, bar, nbytes, slot = loads.pop(rng.randrange(len(loads)))
            bar.complete_tx(nbytes)
        elif kind == "copy":
            what, d, owner, b, unit, bar = copies.pop(rng.randrange(len(copies)))
            if what == "slice":
                put_slice(d, b, owner, unit)
                bar.complete_tx(8)
            else:
                check_write(0, B_REG[0], f"the logit slice of CTA {owner}", ("logits",) + unit)
                live[0][0] = ("logits",) + unit
                logit_units[owner] = unit
                live[owner][0] = None               # the staged source has left
                bar.complete_tx(4)
        else:
            c = rng.choice([c for c in range(C) if mmas[c]])
            kind, what = mmas[c].pop(0)
            if kind == "commit":
                what.arrive()
            elif kind == "consume":
                live[c][what] = None

    alive = [g(c) for c in range(C) for g in (producer, mma, epilogue)]
    turns = 0
    while alive or loads or copies or any(mmas):
        turns += 1
        assert turns < 3_000_000, "deadlock: no role can make progress"
        if alive and (rng.random() < 0.55 or not (loads or copies or any(mmas))):
            g = rng.choice(alive)
            try:
                next(g)
            except StopIteration:
                alive.remove(g)
        else:
            land()
    assert decoded == [(t, s) for t, n in enumerate(tiles) for s in range(n)]


@pytest.mark.parametrize("tiles", [[3], [W + 3], [2, W + 2, 1]])
@pytest.mark.parametrize("seed", range(6))
def test_small_decoder_protocol(tiles, seed):
    simulate(tiles, seed)


@pytest.mark.parametrize("plant,message", [
    ("one_xbar", "within one phase|reads B|waiter targets"),
    ("no_switch_wait", "MMA still reads|overwrites"),
    ("early_ring", "slot"),
])
def test_the_model_catches_planted_protocol_mistakes(plant, message):
    import re
    caught = 0
    for seed in range(40):
        try:
            simulate([W + 3], seed, plant=plant)
        except AssertionError as e:
            assert re.search(message, str(e)), str(e)
            caught += 1
    assert caught > 0, f"no seed exposed the planted mistake {plant!r}"
