"""Property tests (hypothesis) of the host-side restatements around the codec: the signal split
and its inverse, the read-record region, and the chunking of token streams.  The golden vectors
pin these to the reference on fixed inputs; here they hold on generated ones (CPU only)."""

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st
from hypothesis.extra import numpy as hnp

import bench
from oracle import signal
from sigcomp_b200.records import REC_FMT, pack_records, parse_records

int16_reads = hnp.arrays(np.int16, st.integers(1, 400),
                         elements=st.one_of(st.integers(-32768, 32767), st.sampled_from([-32768, 32767, 0, 255, 256])))


@settings(max_examples=200, deadline=None)
@given(int16_reads)
def test_split_then_reassemble_is_the_identity(read):
    sig0, small, large, pos = signal.split_signal(read)
    assert small.dtype == np.uint8 and len(small) + len(large) == len(read) - 1
    assert np.all(large >= 0)
    back = signal.reassemble_signal(sig0, len(read), small, large, pos)
    assert np.array_equal(back, read)


@settings(max_examples=100, deadline=None)
@given(int16_reads, st.integers(1, 8))
def test_lossy_split_round_trip_is_the_lossy_signal(read, lsb):
    coded = signal.lossy_encode(signal.reduce_lsb(read, lsb), lsb)
    sig0, small, large, pos = signal.split_signal(coded)
    back = signal.lossy_decode(signal.reassemble_signal(sig0, len(read), small, large, pos), lsb)
    assert np.array_equal(back, bench.lossy_round_trip(read, lsb))


records = st.lists(st.tuples(st.binary(min_size=REC_FMT.size, max_size=REC_FMT.size),
                             st.integers(-32768, 32767), st.integers(1, 2 ** 32 - 1), st.integers(0, 2 ** 32 - 1),
                             st.binary(max_size=64), st.binary(max_size=16), st.binary(max_size=16)),
                   max_size=12)


@settings(max_examples=150, deadline=None)
@given(records)
def test_record_region_round_trip(recs):
    cols = list(zip(*recs)) if recs else [[]] * 7
    region, offsets = pack_records(*[list(c) for c in cols])
    assert offsets[0] == 0 and offsets[-1] == len(region) and np.all(np.diff(offsets) > 0)
    parsed = parse_records(region)
    assert len(parsed) == len(recs)
    for r, (rec, sig0, n, c_small, s, l, p) in zip(parsed, recs):
        # random records hold NaN doubles too: compare field by field, NaN matching NaN
        assert all(a == b or (a != a and b != b) for a, b in zip(r["rec"], REC_FMT.unpack(rec)))
        assert (r["sig0"], r["N"], r["c_small"]) == (sig0, n, c_small)
        assert (r["s_bytes"], r["l_bytes"], r["p_bytes"]) == (s, l, p)


@settings(max_examples=200, deadline=None)
@given(st.lists(st.integers(0, 9000), max_size=40), st.integers(1, 4096))
def test_chunk_offsets_cut_reads_into_chunk_len_pieces(lengths, chunk_len):
    tok_off = np.zeros(len(lengths) + 1, np.int64)
    np.cumsum(lengths, out=tok_off[1:])
    got = bench.chunk_offsets(tok_off, chunk_len).tolist()
    want = [s for r in range(len(lengths)) for s in range(int(tok_off[r]), int(tok_off[r + 1]), chunk_len)]
    assert got == want + [int(tok_off[-1])]
