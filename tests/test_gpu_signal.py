"""GPU signal transform (sc_split_signal_device / sc_reassemble_signal_device)
against the host restatement of SigComp's _split_signal / _reassemble_signal
(sigcomp/main.py:129-171, 504-546), which is itself pinned to reference outputs
(tests/golden/signal.npz).  Integer work: bit-exact."""

import numpy as np
import pytest

from oracle import signal
from sigcomp_b200 import synthetic

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def codec():
    from sigcomp_b200.codec import B200Compression
    from sigcomp_b200.model import random_model
    return B200Compression(chunk_len=2048, gpu=0, model=random_model(3))


def _reads():
    rng = np.random.default_rng(17)
    reads = [synthetic.synth_read(rng, n) for n in (1, 2, 3, 100, 4095, 4096, 4097, 8193, 40000)]
    reads.append(np.asarray(np.arange(300) * 400 - 30000, dtype=np.int16))      # every delta large
    reads.append(np.full(5000, 123, dtype=np.int16))                              # no large delta
    reads.append(np.asarray([32767, -32768, 32767, 0, -1, 0, 255, -255], dtype=np.int16))   # int16 wraps
    big = synthetic.synth_read(rng, 70000).astype(np.int32)
    big[::997] += 9000                                                              # sparse large deltas
    reads.append(np.clip(big, -32768, 32767).astype(np.int16))
    return reads


def _host_split(read, lsb):
    if lsb:
        read = signal.lossy_encode(signal.reduce_lsb(read, lsb), lsb)
    return signal.split_signal(read)


@pytest.mark.parametrize("lsb", [0, 3])
def test_split_matches_host(codec, lsb):
    reads = _reads()
    got = codec.split_signals(reads, lsb=lsb)
    for r, g in zip(reads, got):
        want = _host_split(r, lsb)
        assert g[0] == want[0]
        for a, b in zip(g[1:], want[1:]):
            assert a.dtype == b.dtype and np.array_equal(a, b)


def test_split_matches_reference_golden(codec, golden):
    z = np.load(golden / "signal.npz")
    i = 0
    while f"sig{i}" in z:
        g = codec.split_signals([z[f"sig{i}"]])[0]
        assert g[0] == int(z[f"sig0_{i}"][0])
        assert np.array_equal(g[1], z[f"small{i}"]) and np.array_equal(g[2], z[f"large{i}"])
        assert np.array_equal(g[3], z[f"pos{i}"])
        i += 1
    assert i > 0


@pytest.mark.parametrize("lsb", [0, 3])
def test_reassemble_round_trip(codec, lsb):
    reads = _reads()
    splits = codec.split_signals(reads, lsb=lsb)
    back = codec.reassemble_signals(splits, [len(r) for r in reads], lsb=lsb)
    for r, b, sp in zip(reads, back, splits):
        want = r if lsb == 0 else signal.lossy_decode(signal.lossy_encode(signal.reduce_lsb(r, lsb), lsb), lsb)
        assert np.array_equal(b, want)
        host = signal.reassemble_signal(sp[0], len(r), sp[1], sp[2], sp[3])
        if lsb:
            host = signal.lossy_decode(host, lsb)
        assert np.array_equal(b, host)


def test_reassemble_rejects_mismatched_streams(codec):
    reads = _reads()[4:6]
    splits = codec.split_signals(reads)
    bad = [(splits[0][0], splits[0][1][:-1], splits[0][2], splits[0][3]), splits[1]]
    with pytest.raises(ValueError):
        codec.reassemble_signals(bad, [len(r) for r in reads])
    # a large position beyond the read
    far = [(splits[1][0], splits[1][1][:-1], np.asarray([0], np.uint16), np.asarray([10 ** 6], np.uint32))]
    with pytest.raises(ValueError):
        codec.reassemble_signals(far, [len(reads[1])])


def test_split_rejects_empty_read(codec):
    with pytest.raises(ValueError):
        codec.split_signals([np.zeros(3, np.int16), np.zeros(0, np.int16)])


def test_split_config2_batch_round_trip(codec):
    reads = synthetic.make_reads("r10_lognormal", seed=9, count=200)
    splits = codec.split_signals(reads)
    for r, sp in zip(reads[:20], splits[:20]):
        want = signal.split_signal(r)
        assert sp[0] == want[0] and all(np.array_equal(a, b) for a, b in zip(sp[1:], want[1:]))
    back = codec.reassemble_signals(splits, [len(r) for r in reads])
    assert all(np.array_equal(a, b) for a, b in zip(back, reads))
