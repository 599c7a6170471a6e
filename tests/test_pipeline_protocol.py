"""CPU model of the synchronisation protocol of the fused pair kernels (k_fused2 in
sigcomp_b200/csrc/sc_mlp_fused2.cuh), run under randomised interleavings.

Roles of one SM pair, with the kernel's unit walk (for_each_unit2), counters and parity formulas:
two TMA producers (one per CTA), the MMA issuer (leader CTA), 2 x 12 epilogue warps, and for
compression 2 x 2 layer-0 builder warps.  Barriers: full[s] (leader; the leader's expect-tx arrival
plus both CTAs' transaction bytes), empty[s] (per CTA, MMA commit multicast), acc_full[b] (per CTA,
commit), acc_empty[b] (leader, 24 arrivals), g_full[b] (leader, 4 builder arrivals), g_empty[b] (per
CTA, commit), and the monotonic act_cnt[slot] counters (per CTA).  TMA transactions and MMA commits
complete asynchronously, commits in issue order.

An mbarrier parity wait is only sound while the barrier is at most one phase away from the phase the
waiter targets: further behind, the parity test passes early; further ahead, it never passes.  Every
wait here asserts that, so an ordering that lets a waiter fall two phases behind fails the test
instead of corrupting a run on the GPU.  The model also checks that no barrier ever receives more
arrivals than its count, and that every role finishes (no deadlock)."""

import random

import pytest

NL = 9
KB = 128
EPI_WARPS = 12
STAGES = 4
TM = 128


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
    """Wait as the kernel does (try_wait.parity), asserting that the barrier is within one phase of
    `target` (the number of completed phases the waiter needs)."""
    while True:
        c = bar.completed
        assert target - 1 <= c <= target, f"{bar.name}: waiter targets phase {target}, barrier at {c}"
        if (c & 1) != parity:
            return
        yield


def units(decode, n_tiles, maxlen):
    """for_each_unit2 for pair 0 of a one-pair grid: (grp, tt, pt, step, L, nh)."""
    ktd = 6 if decode else 5
    n_pt = (n_tiles + 1) // 2
    for g0, grp in zip(range(0, n_pt, ktd), range(10 ** 9)):
        gn = min(ktd, n_pt - g0)
        ml = [maxlen[g0 + tt] if decode else 1 for tt in range(gn)]
        for step in range(max(ml)):
            for L in range(NL):
                for tt in range(gn):
                    if decode and ml[tt] <= step:
                        continue
                    for nh in range(2 if L < NL - 1 else 1):
                        yield grp, tt, g0 + tt, step, L, nh


def simulate(decode, n_tiles, maxlen=None, l0_kblocks=8, seed=0, plant=None, slots=False):
    """Run one pair's roles to completion.  `plant` injects one protocol mistake into the model
    (tests of the model itself): 'counter' (a producer waits for one layer less), 'warp' (one
    epilogue warp missing) or 'stages' (the MMA cycles over one stage less than the producer).
    With `slots`, the operand buffers are a ring of 16 KB slots with a barrier pair per slot: a
    dual layer-0 K block takes three slots, every other K block two (12 slots for the decoder's
    192 KB, 8 for compression's 128 KB); each role tracks a slot's phase per slot."""
    rng = random.Random(seed)
    in_dim = [l0_kblocks * KB] + [512] * (NL - 1)
    nbuf = (12 if decode else 8) if slots else STAGES
    full = [Bar(f"full{s}", 1) for s in range(nbuf)]
    empty = [[Bar(f"empty{s}/cta{r}", 1) for s in range(nbuf)] for r in range(2)]

    def kblock_bufs(L, pos, it, n_ring):
        """The buffers (stage, or slots) of a K block and how far the position advances."""
        if not slots:
            return [it % n_ring], 1
        n = 3 if (decode and L == 0) else 2
        return [(pos + i) % n_ring for i in range(n)], n
    acc_full = [[Bar(f"acc_full{b}/cta{r}", 1) for b in range(2)] for r in range(2)]
    acc_empty = [Bar(f"acc_empty{b}", 2 * EPI_WARPS) for b in range(2)]
    g_full = [Bar(f"g_full{b}", 4) for b in range(2)]
    g_empty = [[Bar(f"g_empty{b}/cta{r}", 1) for b in range(2)] for r in range(2)]
    act = [[0] * 8 for _ in range(2)]
    done = {}                        # (rank, grp, tt, step, L) -> epilogue warps finished with that layer
    tma, commits = [], []            # in flight: (bar, bytes) / lists of barriers to arrive on

    def counter_wait(rank, tt, target):
        while act[rank][tt] < target:
            yield

    def producer(rank):
        it = pos = 0
        uses = [0] * nbuf                             # per buffer: times filled so far
        for grp, tt, pt, step, L, nh in units(decode, n_tiles, maxlen):
            if decode and L == 0 and nh == 1:
                continue                              # loaded with half 0
            nkb = in_dim[L] // KB
            if nh == 0 and (L >= 1 or (decode and step > 0)):
                k = (step if decode else grp) * NL + L - 1
                yield from counter_wait(rank, tt, EPI_WARPS * (k if plant == "counter" else k + 1))
            # the data this unit loads is complete: every epilogue warp of this CTA has written the
            # tile's previous layer (decode layer 0: the previous step's token, appended to the ring)
            if L >= 1:
                assert done.get((rank, grp, tt, step, L - 1), 0) == EPI_WARPS, "layer loaded before it was written"
            elif decode and step > 0:
                assert done.get((rank, grp, tt, step - 1, NL - 1), 0) == EPI_WARPS, "ring block loaded early"

            kstep = 2 if (not decode and L == 0) else 1
            for kb in range(0, nkb, kstep):
                bufs, adv = kblock_bufs(L, pos, it, nbuf)
                for j in bufs:
                    u = uses[j]
                    yield from parity_wait(empty[rank][j], (u & 1) ^ 1, u)
                    uses[j] += 1
                s = bufs[0]
                dual = decode and L == 0
                a_tma = decode or L != 0
                nbytes = 2 * ((2 if dual else 1) * 16 + (16 if a_tma else 16))
                if rank == 0:
                    full[s].expect_tx(nbytes)
                    full[s].arrive()
                tma.append((full[s], nbytes // 2))    # this CTA's share completes on the leader
                it += 1
                pos += adv
                yield

    def mma():
        it = uu = li = pos = 0
        firsts = [0] * nbuf                           # per buffer: K blocks it has led so far
        for grp, tt, pt, step, L, nh in units(decode, n_tiles, maxlen):
            if decode and L == 0 and nh == 1:
                continue
            dual = decode and L == 0
            nkb = in_dim[L] // KB
            ab = uu & 1
            yield from parity_wait(acc_empty[ab], ((uu >> 1) & 1) ^ 1, uu >> 1)
            if dual:
                yield from parity_wait(acc_empty[ab ^ 1], (((uu + 1) >> 1) & 1) ^ 1, (uu + 1) >> 1)
            gb = li & 1
            if not decode and L == 0 and nh == 0:
                yield from parity_wait(g_full[gb], (li >> 1) & 1, (li >> 1) + 1)
            kstep = 2 if (not decode and L == 0) else 1
            for kb in range(0, nkb, kstep):
                bufs, adv = kblock_bufs(L, pos, it, nbuf - 1 if plant == "stages" else nbuf)
                s = bufs[0]
                f = firsts[s]
                yield from parity_wait(full[s], f & 1, f + 1)
                firsts[s] += 1
                for j in bufs:                        # one commit per buffer, in order
                    commits.append([empty[0][j], empty[1][j]])
                it += 1
                pos += adv
                yield
            commits.append([acc_full[0][ab], acc_full[1][ab]])
            if dual:
                commits.append([acc_full[0][ab ^ 1], acc_full[1][ab ^ 1]])
            uu += 2 if dual else 1
            if not decode and L == 0 and nh == 1:
                commits.append([g_empty[0][gb], g_empty[1][gb]])
                li += 1

    def epilogue(rank):
        uu = 0
        for grp, tt, pt, step, L, nh in units(decode, n_tiles, maxlen):
            ab = uu & 1
            yield from parity_wait(acc_full[rank][ab], (uu >> 1) & 1, (uu >> 1) + 1)
            uu += 1
            yield                                     # tcgen05.ld, requantise, store
            acc_empty[ab].arrive()
            if L == NL - 1 or nh == 1:
                key = (rank, grp, tt, step, L)
                done[key] = done.get(key, 0) + 1
                act[rank][tt] += 1

    def builder(rank):
        li = 0
        for grp, tt, pt, step, L, nh in units(decode, n_tiles, maxlen):
            if L != 0 or nh != 0:
                continue
            gb = li & 1
            yield from parity_wait(g_empty[rank][gb], ((li >> 1) & 1) ^ 1, li >> 1)
            li += 1
            yield                                     # fill the sliding buffer
            g_full[gb].arrive()

    roles = [producer(0), producer(1), mma()]
    roles += [epilogue(r) for r in range(2) for _ in range(EPI_WARPS)][:-1 if plant == "warp" else None]
    if not decode:
        roles += [builder(r) for r in range(2) for _ in range(2)]
    live = list(range(len(roles)))
    idle = 0
    while live or tma or commits:
        choice = rng.random()
        if tma and choice < 0.15:
            bar, b = tma.pop(rng.randrange(len(tma)))
            bar.complete_tx(b)
            idle = 0
            continue
        if commits and choice < 0.3:
            for bar in commits.pop(0):                # MMA completions are in issue order
                bar.arrive()
            idle = 0
            continue
        if not live:
            continue
        i = rng.choice(live)
        try:
            next(roles[i])
        except StopIteration:
            live.remove(i)
        idle += 1
        assert idle < 200000, "no progress: deadlock"
    for b in full + acc_empty + g_full:
        assert b.pending == b.count and b.tx == 0, f"{b.name} left mid-phase"


@pytest.mark.parametrize("seed", range(3))
@pytest.mark.parametrize("n_tiles,maxlen", [(1, [3]), (4, [3, 3, 2, 1]), (12, [2] * 12), (11, [3, 3, 3, 2, 2, 2, 2, 1, 1, 1, 1])])
def test_decoder_protocol(n_tiles, maxlen, seed):
    simulate(True, n_tiles, maxlen, seed=seed)


@pytest.mark.parametrize("seed", range(3))
@pytest.mark.parametrize("n_tiles", [1, 2, 9, 10, 23])
def test_compress_protocol(n_tiles, seed):
    simulate(False, n_tiles, seed=seed)


@pytest.mark.parametrize("seed", range(3))
@pytest.mark.parametrize("decode,n_tiles,maxlen", [(True, 4, [3, 3, 2, 1]), (True, 12, [2] * 12),
                                                  (True, 11, [3, 3, 3, 2, 2, 2, 2, 1, 1, 1, 1]), (False, 23, None)])
def test_slot_ring_protocol(decode, n_tiles, maxlen, seed):
    """The 16 KB slot ring (a deeper prefetch for hidden layers) keeps every invariant."""
    simulate(decode, n_tiles, maxlen, seed=seed, slots=True)


@pytest.mark.parametrize("slots", [False, True])
@pytest.mark.parametrize("plant,messages", [("counter", ("loaded before it was written",)),
                                            ("warp", ("deadlock",)),
                                            ("stages", ("waiter targets phase", "deadlock"))])
def test_the_model_catches_planted_protocol_mistakes(plant, messages, slots):
    """Each planted mistake fails the model under some interleaving, for the expected reason."""
    errors = []
    for seed in range(4):
        for decode, n_tiles, maxlen in [(True, 4, [3, 3, 2, 1]), (True, 12, [2] * 12), (False, 10, None)]:
            try:
                simulate(decode, n_tiles, maxlen, seed=seed, plant=plant, slots=slots)
            except AssertionError as e:
                errors.append(str(e))
    assert errors and all(any(m in e for m in messages) for e in errors), errors[:3]
