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
arrivals than its count, and that every role finishes (no deadlock).

In the decoder, the two 256-column halves of each layer between the first and the last share their
stages: the producer loads a K block's activations and both weight halves once (with half 0), the
MMA issuer's half 0 waits for each stage and keeps it, and half 1 reads the same stages again and
releases them.

Both kernels' layers after the first also take their bias through a bias tile: one 16 KB buffer per
CTA, loaded by the producer after the K blocks of a layer's first unit in each step or tile group (bt_full on the
leader, bt_empty per CTA), read by one bias MMA at the end of every unit of the layer, and released
by a commit after the layer's last one.  The model checks that every bias MMA sees its own layer's
tile and that no tile lands while a bias MMA of the previous one is pending.

The decoder's unit walk is the kernel's one-launch schedule: each of six lanes runs a queue of
pair-tiles back to back (longest first, to the least-loaded lane), cut into segments at every
step where a lane changes tile, as `build_decode_schedule` in sc_mlp_tc.cu does for one pair.

Abort path: with `abort` set, one role gives up at a chosen wait, as a kernel role does when its
bounded wait times out.  Every other wait is then bounded too (a budget of scheduler turns), so
the roles that depend on the one that stopped also give up.  Each role then runs the kernel's
drain: a producer waits (bounded) on the full (leader) or empty (peer) phases of the last stages
it issued and then idles; the MMA issuer commits to the drain barrier after its last MMA, and
TMEM is freed only once that barrier completes.  The model checks that when the CTAs end, no
copy is still landing in shared memory and no MMA or commit is still in flight."""

import random

import pytest


class Timeout(Exception):
    """A bounded wait gave up (the kernel's wait returned false)."""

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


def parity_wait(bar, parity, target, budget=None):
    """Wait as the kernel does (try_wait.parity), asserting that the barrier is within one phase of
    `target` (the number of completed phases the waiter needs).  With a budget, give up (raise
    Timeout) after that many unsatisfied turns, as the kernel's bounded waits do."""
    turns = 0
    while True:
        c = bar.completed
        assert target - 1 <= c <= target, f"{bar.name}: waiter targets phase {target}, barrier at {c}"
        if (c & 1) != parity:
            return
        turns += 1
        if budget is not None and turns > budget:
            raise Timeout(bar.name)
        yield


def decode_schedule(maxlen, lanes=6):
    """One pair's lanes and segments: (s0, s1, [(pt, start) or None per lane]) in step order."""
    queues, load = [[] for _ in range(lanes)], [0] * lanes
    for pt in range(len(maxlen)):
        t = min(range(lanes), key=lambda i: (load[i], i))
        queues[t].append(pt)
        load[t] += maxlen[pt]
    segs, idx, start, gs = [], [0] * lanes, [0] * lanes, 0
    while True:
        ends = [start[t] + maxlen[queues[t][idx[t]]] for t in range(lanes) if idx[t] < len(queues[t])]
        if not ends:
            return segs
        nxt = min(ends)
        segs.append((gs, nxt, [(queues[t][idx[t]], start[t]) if idx[t] < len(queues[t]) else None
                               for t in range(lanes)]))
        for t in range(lanes):
            if idx[t] < len(queues[t]) and start[t] + maxlen[queues[t][idx[t]]] == nxt:
                idx[t] += 1
                start[t] = nxt
        gs = nxt


def units(decode, n_tiles, maxlen):
    """for_each_unit2 for pair 0 of a one-pair grid: (gs, tt, pt, step, L, nh), gs the global step
    (decode) or the tile group (compress)."""
    n_pt = (n_tiles + 1) // 2
    if decode:
        for s0, s1, lanes in decode_schedule(maxlen[:n_pt]):
            for gs in range(s0, s1):
                for L in range(NL):
                    for tt, cur in enumerate(lanes):
                        if cur is None:
                            continue
                        pt, start = cur
                        for nh in range(2 if L < NL - 1 else 1):
                            yield gs, tt, pt, gs - start, L, nh
        return
    ktd = 5
    for g0, grp in zip(range(0, n_pt, ktd), range(10 ** 9)):
        gn = min(ktd, n_pt - g0)
        for L in range(NL):
            for tt in range(gn):
                for nh in range(2 if L < NL - 1 else 1):
                    yield grp, tt, g0 + tt, 0, L, nh


def units_fl(decode, n_tiles, maxlen):
    """units() with the kernel's fl flags: bit 0 the first unit of its (step or group, layer), bit 1
    the last."""
    us = list(units(decode, n_tiles, maxlen))
    out = []
    for i, u in enumerate(us):
        key = (u[0], u[4])
        first = i == 0 or (us[i - 1][0], us[i - 1][4]) != key
        last = i == len(us) - 1 or (us[i + 1][0], us[i + 1][4]) != key
        out.append(u + ((1 if first else 0) | (2 if last else 0),))
    return out


class Done:
    """A commit entry that records the completion of an MMA (no barrier)."""

    def __init__(self, fn):
        self.fn = fn

    def arrive(self):
        self.fn()


def simulate(decode, n_tiles, maxlen=None, l0_kblocks=8, seed=0, plant=None, slots=False, abort=None):
    """Run one pair's roles to completion.  `plant` injects one protocol mistake into the model
    (tests of the model itself): 'counter' (a producer waits for one layer less), 'warp' (one
    epilogue warp missing) or 'stages' (the MMA cycles over one stage less than the producer).
    `abort` = (role, n): that role ('producer0', 'producer1', 'mma', 'epilogue0', 'epilogue1')
    gives up at its n-th wait.
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
    drain = [Bar(f"drain/cta{r}", 1) for r in range(2)]
    # stage ring: the bias tile of layers >= 1, loaded once per step (or tile group) and layer into
    # one buffer per CTA; bt_full on the leader (expect-tx + both CTAs' bytes), bt_empty per CTA (commit)
    tiles = not slots
    bt_full = Bar("bt_full", 1)
    bt_empty = [Bar(f"bt_empty/cta{r}", 1) for r in range(2)]
    tile_in = [None, None]                          # per CTA: the (step, layer) whose tile has landed
    tile_reads = {}                                 # (step, layer) -> bias MMAs issued, not completed
    act = [[0] * 8 for _ in range(2)]
    done = {}                        # (rank, gs, tt, L) -> epilogue warps finished with that layer
    tma, commits = [], []            # in flight: (bar, bytes) / lists of barriers to arrive on
    budget = 3000 if abort else None
    waits = {}                       # role name -> waits started (for the planted abort)

    def planted(role):
        waits[role] = waits.get(role, 0) + 1
        if abort and abort[0] == role and waits[role] == abort[1]:
            raise Timeout(f"planted at {role}")

    def pwait(role, bar, parity, target):
        planted(role)
        yield from parity_wait(bar, parity, target, budget)

    def counter_wait(rank, tt, target):
        planted(f"producer{rank}")
        turns = 0
        while act[rank][tt] < target:
            turns += 1
            if budget is not None and turns > budget:
                raise Timeout("act_cnt")
            yield

    def idle(turns):
        for _ in range(turns):
            yield

    def producer(rank):
        it = pos = 0
        uses = [0] * nbuf                             # per buffer: times filled so far
        led = [0] * nbuf                              # per buffer: K blocks it has led (full phases)
        issued = []                                   # per K block: (first buffer, its K block number, its fill number)
        nbt = 0                                       # bias tiles loaded
        try:
            for gs, tt, pt, step, L, nh, fl in units_fl(decode, n_tiles, maxlen):
                if decode and nh == 1 and (L == 0 or not slots):
                    continue                          # loaded with half 0 (shared stages)
                nkb = in_dim[L] // KB
                if nh == 0 and (L >= 1 or (decode and step > 0)):
                    k = gs * NL + L - 1
                    yield from counter_wait(rank, tt, EPI_WARPS * (k if plant == "counter" else k + 1))
                # the data this unit loads is complete: every epilogue warp of this CTA has written the
                # tile's previous layer (decode layer 0: the previous step's token, appended to the ring)
                if L >= 1:
                    assert done.get((rank, gs, tt, L - 1), 0) == EPI_WARPS, "layer loaded before it was written"
                elif decode and step > 0:
                    assert done.get((rank, gs - 1, tt, NL - 1), 0) == EPI_WARPS, "ring block loaded early"

                kstep = 2 if (not decode and L == 0) else 1
                for kb in range(0, nkb, kstep):
                    bufs, adv = kblock_bufs(L, pos, it, nbuf)
                    for j in bufs:
                        u = uses[j]
                        yield from pwait(f"producer{rank}", empty[rank][j], (u & 1) ^ 1, u)
                        uses[j] += 1
                    s = bufs[0]
                    dual = decode and L == 0
                    # decode without slots: the two halves of a layer >= 1 share each stage
                    both = dual or (decode and not slots and L < NL - 1)
                    a_tma = decode or L != 0
                    nbytes = 2 * ((2 if both else 1) * 16 + (16 if a_tma else 16))
                    if rank == 0:
                        full[s].expect_tx(nbytes)
                        full[s].arrive()
                    tma.append((full[s], nbytes // 2, rank))  # this CTA's share completes on the leader
                    issued.append((s, led[s], uses[s] - 1))
                    led[s] += 1
                    it += 1
                    pos += adv
                    yield
                if tiles and L >= 1 and fl & 1:
                    # the layer's bias tile, after the unit's K blocks, once the buffer is free
                    yield from pwait(f"producer{rank}", bt_empty[rank], (nbt & 1) ^ 1, nbt)
                    if rank == 0:
                        bt_full.expect_tx(32)
                        bt_full.arrive()

                    def land(key=(gs, L), r=rank):
                        for old_key, n in tile_reads.items():
                            assert old_key == key or n == 0, "bias tile overwritten under a pending bias MMA"
                        tile_in[r] = key
                    tma.append((bt_full, 16, rank, land))
                    nbt += 1
                    yield
        except Timeout:
            if plant == "no_drain":
                assert not [t for t in tma if t[2] == rank], \
                    "a CTA ends with copies still landing in its shared memory"
                return
            # drain: the last stages this CTA issued, on the leader's full or its own empty barrier
            for s, f, u in issued[-nbuf:]:
                try:
                    if rank == 0:
                        yield from parity_wait(full[s], f & 1, f + 1, 500)
                    else:
                        yield from parity_wait(empty[rank][s], u & 1, u + 1, 500)
                except Timeout:
                    pass
            if nbt:
                try:
                    if rank == 0:
                        yield from parity_wait(bt_full, (nbt - 1) & 1, nbt, 500)
                    else:
                        yield from parity_wait(bt_empty[rank], (nbt - 1) & 1, nbt, 500)
                except Timeout:
                    pass
            yield from idle(400)
            # the producer is the only role that issues copies into this CTA's shared memory
            assert not [t for t in tma if t[2] == rank], "a CTA ends with copies still landing in its shared memory"

    def mma():
        it = uu = li = pos = 0
        it_shared = 0                                 # first stage of the current shared layer
        firsts = [0] * nbuf                           # per buffer: K blocks it has led so far
        nbt = 0                                       # bias tiles used
        try:
            for gs, tt, pt, step, L, nh, fl in units_fl(decode, n_tiles, maxlen):
                if decode and L == 0 and nh == 1:
                    continue
                dual = decode and L == 0
                nkb = in_dim[L] // KB
                ab = uu & 1
                yield from pwait("mma", acc_empty[ab], ((uu >> 1) & 1) ^ 1, uu >> 1)
                if dual:
                    yield from pwait("mma", acc_empty[ab ^ 1], (((uu + 1) >> 1) & 1) ^ 1, (uu + 1) >> 1)
                gb = li & 1
                if not decode and L == 0 and nh == 0:
                    yield from pwait("mma", g_full[gb], (li >> 1) & 1, (li >> 1) + 1)
                kstep = 2 if (not decode and L == 0) else 1
                # decode without slots, layers 0 < L < NL-1: half 0 waits for each stage and keeps
                # it, half 1 reads the same stages again and releases them
                sh = decode and not slots and 0 < L < NL - 1
                if sh and nh == 0:
                    it_shared = it
                if sh and nh == 1:
                    n_ring = nbuf - 1 if plant == "stages" else nbuf
                    for kb in range(nkb):
                        j = (it_shared + kb) % n_ring
                        commits.append([empty[0][j], empty[1][j]])
                        yield
                for kb in range(0, nkb if not (sh and nh == 1) else 0, kstep):
                    bufs, adv = kblock_bufs(L, pos, it, nbuf - 1 if plant == "stages" else nbuf)
                    s = bufs[0]
                    f = firsts[s]
                    yield from pwait("mma", full[s], f & 1, f + 1)
                    firsts[s] += 1
                    if not (sh and nh == 0):
                        for j in bufs:                # one commit per buffer, in order
                            commits.append([empty[0][j], empty[1][j]])
                    it += 1
                    pos += adv
                    yield
                if tiles and L >= 1:
                    # the bias MMA after the K blocks; the tile is released after the layer's last
                    if fl & 1:
                        yield from pwait("mma", bt_full, nbt & 1, nbt + 1)
                        nbt += 1
                    key = (gs, L)
                    assert tile_in == [key, key], "bias MMA before its layer's tile landed"
                    tile_reads[key] = tile_reads.get(key, 0) + 1

                    def read_done(key=key):
                        tile_reads[key] -= 1
                    commits.append([Done(read_done)])
                    if fl & (1 if plant == "tile" else 2):
                        commits.append([bt_empty[0], bt_empty[1]])
                commits.append([acc_full[0][ab], acc_full[1][ab]])
                if dual:
                    commits.append([acc_full[0][ab ^ 1], acc_full[1][ab ^ 1]])
                uu += 2 if dual else 1
                if not decode and L == 0 and nh == 1:
                    commits.append([g_empty[0][gb], g_empty[1][gb]])
                    li += 1
        except Timeout:
            pass
        commits.append([drain[0], drain[1]])          # after every MMA and commit above

    def epilogue(rank, first):
        uu = 0
        name = f"epilogue{rank}" if first else f"epilogue{rank}x"
        try:
            for gs, tt, pt, step, L, nh in units(decode, n_tiles, maxlen):
                ab = uu & 1
                yield from pwait(name, acc_full[rank][ab], (uu >> 1) & 1, (uu >> 1) + 1)
                uu += 1
                yield                                 # tcgen05.ld, requantise, store
                acc_empty[ab].arrive()
                if L == NL - 1 or nh == 1:
                    key = (rank, gs, tt, L)
                    done[key] = done.get(key, 0) + 1
                    act[rank][tt] += 1
        except Timeout:
            pass

    def builder(rank):
        li = 0
        try:
            for gs, tt, pt, step, L, nh in units(decode, n_tiles, maxlen):
                if L != 0 or nh != 0:
                    continue
                gb = li & 1
                yield from pwait(f"builder{rank}", g_empty[rank][gb], ((li >> 1) & 1) ^ 1, li >> 1)
                li += 1
                yield                                 # fill the sliding buffer
                g_full[gb].arrive()
        except Timeout:
            pass

    def teardown(rank):
        # warp 1: TMEM is freed only once the drain barrier completes (bounded wait)
        try:
            if plant != "no_drain":
                yield from parity_wait(drain[rank], 0, 1, budget)
        except Timeout:
            pass
        freed[rank] = True
        assert not commits, "TMEM freed with MMAs or commits still in flight"

    freed = [False, False]
    roles = [producer(0), producer(1), mma()]
    roles += [epilogue(r, i == 0) for r in range(2) for i in range(EPI_WARPS)][:-1 if plant == "warp" else None]
    if not decode:
        roles += [builder(r) for r in range(2) for _ in range(2)]
    n_work = len(roles)
    roles += [teardown(0), teardown(1)]
    live = list(range(len(roles)))
    stalled = 0
    while live:
        choice = rng.random()
        if tma and choice < 0.15:
            entry = tma.pop(rng.randrange(len(tma)))
            if len(entry) > 3:
                entry[3]()                            # the copy's data is in shared memory
            entry[0].complete_tx(entry[1])
            stalled = 0
            continue
        if commits and choice < 0.3:
            for bar in commits.pop(0):                # MMA completions are in issue order
                bar.arrive()
            stalled = 0
            continue
        # the teardown runs after every role of the pair has finished (__syncthreads and the
        # cluster barrier before the TMEM release)
        ready = [i for i in live if i < n_work] or live
        i = rng.choice(ready)
        try:
            next(roles[i])
        except StopIteration:
            live.remove(i)
            if i >= n_work:
                continue
            if not [j for j in live if j < n_work]:
                # every role has finished: the CTAs end once the teardown is done
                assert not tma, "a CTA ends with copies still landing in its shared memory"
        stalled += 1
        assert stalled < (2000000 if abort else 200000), "no progress: deadlock"
    assert freed == [True, True] and not commits and not tma
    if abort:
        assert waits.get(abort[0], 0) >= abort[1], "the planted abort was never reached"
    if not abort:
        for b in full + acc_empty + g_full + [bt_full]:
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


def test_the_model_catches_an_early_bias_tile_release():
    """Releasing the bias tile after a layer's first bias MMA instead of its last lets the next
    layer's tile land while bias MMAs still read the buffer."""
    errors = []
    for seed in range(6):
        for n_tiles, maxlen in [(4, [3, 3, 2, 1]), (12, [2] * 12)]:
            try:
                simulate(True, n_tiles, maxlen, seed=seed, plant="tile")
            except AssertionError as e:
                errors.append(str(e))
    assert errors and all("bias" in e or "waiter targets phase" in e or "deadlock" in e for e in errors), errors[:3]


@pytest.mark.parametrize("seed", range(2))
@pytest.mark.parametrize("role,n", [("producer0", 3), ("producer1", 3), ("producer0", 40), ("producer1", 41),
                                    ("mma", 2), ("mma", 30), ("epilogue0", 5), ("epilogue1", 25)])
@pytest.mark.parametrize("decode,n_tiles,maxlen", [(True, 4, [3, 3, 2, 1]), (False, 10, None)])
def test_abort_path_drains_before_the_ctas_end(decode, n_tiles, maxlen, role, n, seed):
    """A role that gives up mid-run: every other role ends through its bounded waits, the
    producers' copies land and every MMA completes before TMEM is freed and the CTAs end."""
    simulate(decode, n_tiles, maxlen, seed=seed, abort=(role, n))


def test_the_model_catches_a_missing_drain():
    """Without the producer's drain, a producer that gives up leaves its last copies landing in
    shared memory after it has finished."""
    errors = []
    for seed in range(4):
        for role, n in (("producer0", 3), ("producer1", 41)):
            try:
                simulate(True, 4, [3, 3, 2, 1], seed=seed, abort=(role, n), plant="no_drain")
            except AssertionError as e:
                errors.append(str(e))
    assert errors and all("copies still landing" in e for e in errors), errors[:3]
