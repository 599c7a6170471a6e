"""The pipelined archive loops (sigcomp_b200.archive) on the CPU, with the CPU oracle in place of the
device calls: byte-identical records against the reference's archive region, order and offsets,
overlap of coding with writing, and errors from every stage."""

import io
import threading

import numpy as np
import pytest

from oracle_backed import OracleBacked
from sigcomp_b200 import synthetic
from sigcomp_b200.archive import RecordWriter, compress_reads, decompress_records, prefetch
from sigcomp_b200.records import REC_FMT, parse_records

from test_archive import _archive


def empty_rice(values, fallback_bits):
    """SigComp's _rice_compress for the only case these reads reach: no large values (one zero
    byte, main.py:176-177)."""
    if len(values):
        raise ValueError("this test coder handles empty arrays only")
    return b"\x00"


def empty_rice_decode(buf, count, fallback_bits):
    if count:
        raise ValueError("this test coder handles empty arrays only")
    return np.zeros(0, np.uint32)


def raw_rice(values, fallback_bits):
    """A stand-in blob format for large values (little-endian u32), not SigComp's rice format:
    it only carries the values through the pipeline so that their plumbing is checked."""
    return np.asarray(values, dtype="<u4").tobytes()


def raw_rice_decode(buf, count, fallback_bits):
    return np.frombuffer(buf, dtype="<u4")[:count]


def _batches(recs, reads, sizes):
    out, i = [], 0
    for k in sizes:
        out.append((recs[i:i + k], reads[i:i + k]))
        i += k
    return out


@pytest.mark.parametrize("name", ["lossless", "lossy"])
def test_pipeline_writes_reference_region(golden, name, request):
    model = request.getfixturevalue(f"{name}_model")
    reads, recs, region_ref, decoded_ref, lsb = _archive(golden, name)
    codec = OracleBacked(model)
    out = io.BytesIO()
    ids, offsets = compress_reads(codec, _batches(recs, reads, [4, 4, 3]), out, empty_rice, lsb=lsb,
                                  data_start=100)
    assert out.getvalue() == region_ref
    assert ids == [r[:16] for r in recs]
    # offsets: where each record starts, counted from the archive position of the first record
    sizes = [len(r) for r in _record_bytes(region_ref)]
    assert offsets.tolist() == (100 + np.concatenate([[0], np.cumsum(sizes)[:-1]])).tolist()
    # back, one region per batch of three records
    cut = [0, *np.cumsum(sizes).tolist()]
    regions = [region_ref[cut[i]:cut[min(i + 3, len(sizes))]] for i in range(0, len(sizes), 3)]
    got_recs, got = [], []
    for r, sig in decompress_records(codec, regions, empty_rice_decode, lsb=lsb):
        got_recs += r
        got += sig
    assert [REC_FMT.pack(*r) for r in got_recs] == recs
    assert all(np.array_equal(a, b) for a, b in zip(got, decoded_ref)) and len(got) == len(decoded_ref)


def _record_bytes(region):
    parsed = parse_records(region)
    out, pos = [], 0
    for p in parsed:
        n = REC_FMT.size + 10 + 12 + len(p["s_bytes"]) + len(p["l_bytes"]) + len(p["p_bytes"])
        out.append(region[pos:pos + n])
        pos += n
    assert pos == len(region)
    return out


def test_pipeline_carries_large_values(lossless_model):
    rng = np.random.default_rng(3)
    reads = [synthetic.synth_read(rng, n, synthetic.RNA004) for n in (5000, 1, 2, 300, 2100)]
    assert sum(int(np.count_nonzero(np.abs(np.diff(r.astype(np.int32))) > 127)) for r in reads) > 0
    recs = [bytes([i]) * REC_FMT.size for i in range(len(reads))]
    codec = OracleBacked(lossless_model)
    out = io.BytesIO()
    compress_reads(codec, _batches(recs, reads, [2, 3]), out, raw_rice)
    got = [s for _, sig in decompress_records(codec, [out.getvalue()], raw_rice_decode) for s in sig]
    assert all(np.array_equal(a, b) for a, b in zip(got, reads)) and len(got) == len(reads)


class _Gate:
    """Coding of batch 1 and writing of batch 0 wait for each other: the loop finishes only if the
    writer thread writes batch 0 while the calling thread codes batch 1."""

    def __init__(self, codec):
        self.codec = codec
        self.coding1, self.writing0 = threading.Event(), threading.Event()
        self.calls = 0
        self.writes = []

    def split_signals(self, reads, lsb=0):
        return self.codec.split_signals(reads, lsb)

    def batch_inference_reads(self, **kw):
        self.calls += 1
        if self.calls == 2:
            self.coding1.set()
            if not self.writing0.wait(10):
                raise AssertionError("batch 1 was coded before batch 0 was being written")
        return self.codec.batch_inference_reads(**kw)

    def write(self, data):
        if not self.writes:
            self.writing0.set()
            if not self.coding1.wait(10):
                raise AssertionError("batch 0 was written before batch 1 was being coded")
        self.writes.append(bytes(data))


def test_pipeline_overlaps_coding_and_writing(lossless_model):
    rng = np.random.default_rng(4)
    reads = [np.clip(np.cumsum(rng.integers(-20, 21, size=n)), -3000, 3000).astype(np.int16)
             for n in (900, 700, 800, 50)]
    recs = [bytes([i]) * REC_FMT.size for i in range(4)]
    gate = _Gate(OracleBacked(lossless_model))
    compress_reads(gate, _batches(recs, reads, [2, 1, 1]), gate, empty_rice)
    assert len(gate.writes) == 3


def test_pipeline_errors_reach_the_caller(lossless_model):
    rng = np.random.default_rng(5)
    reads = [synthetic.synth_read(rng, 3000, synthetic.RNA004) for _ in range(3)]
    recs = [b"\x01" * REC_FMT.size] * 3
    codec = OracleBacked(lossless_model)
    # the writer thread's rice coder fails: large values with the empty-only coder
    with pytest.raises(ValueError, match="empty arrays only"):
        compress_reads(codec, _batches(recs, reads, [1, 1, 1]), io.BytesIO(), empty_rice)

    # the batch source fails part-way
    def source():
        yield recs[:1], reads[:1]
        raise OSError("POD5 read failed")
    with pytest.raises(OSError, match="POD5 read failed"):
        compress_reads(codec, source(), io.BytesIO(), raw_rice)

    # a record that is not a REC_FMT record
    with pytest.raises(ValueError, match="REC_FMT"):
        compress_reads(codec, [([b"short"], reads[:1])], io.BytesIO(), raw_rice)

    # a truncated region
    out = io.BytesIO()
    compress_reads(codec, _batches(recs, reads, [3]), out, raw_rice)
    with pytest.raises(ValueError, match="truncated"):
        list(decompress_records(codec, [out.getvalue()[:-1]], raw_rice_decode))


def test_prefetch_order_and_early_exit():
    assert list(prefetch(range(50), depth=3)) == list(range(50))
    seen = []
    for x in prefetch(iter(range(1000)), depth=2):
        seen.append(x)
        if x == 5:
            break
    assert seen == list(range(6))
    with pytest.raises(ValueError):
        list(prefetch([1], depth=0))


def test_writer_rejects_use_after_close():
    w = RecordWriter(io.BytesIO(), raw_rice)
    ids, offsets = w.close()
    assert ids == [] and len(offsets) == 0
    with pytest.raises(ValueError, match="closed"):
        w.submit([], [], [], [])
