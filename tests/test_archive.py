"""Whole read records of the archive, both ways, against the reference's own archive bytes.

``tests/golden/archive.npz`` holds int16 reads taken by SigComp's compress path to the record region
(lossy transform, ``_split_signal``, ``batch_inference_reads``, ``_rice_compress``,
``_write_read_payload``; main.py:844-931) and that region taken back to signals (main.py:1142-1165),
for the lossless and the lossy model.  Every delta of these reads fits a token, so both rice blobs
are SigComp's empty encoding: rice coding itself stays in SigComp (fast_rice), outside this library.

The GPU test runs the path a SigComp user gets from this library (split on the GPU, the codec's
``batch_inference_reads``, :func:`pack_records`, then back); the CPU test runs the same host code
with the CPU oracle in place of the device calls.
"""

import numpy as np
import pytest

from oracle import signal
from oracle_backed import OracleBacked
from sigcomp_b200.records import REC_FMT, pack_records, parse_records

# SigComp's _rice_compress of an empty array: one zero byte (main.py:176-177)
EMPTY_RICE = b"\x00"


def _archive(golden, name):
    z = np.load(golden / "archive.npz")
    o = z["read_offsets"]
    reads = [z[f"{name}_reads"][o[i]:o[i + 1]] for i in range(len(o) - 1)]
    decoded = [z[f"{name}_decoded"][o[i]:o[i + 1]] for i in range(len(o) - 1)]
    rec = z[f"{name}_rec"].tobytes()
    recs = [rec[i * REC_FMT.size:(i + 1) * REC_FMT.size] for i in range(len(reads))]
    return reads, recs, z[f"{name}_region"].tobytes(), decoded, int(z[f"{name}_lsb"][0])


def _region(codec, reads, recs, splits):
    assert all(len(s[2]) == 0 and len(s[3]) == 0 for s in splits)
    framed = codec.batch_inference_reads(list_of_reads=[s[1] for s in splits], batch_size=1024)
    region, offsets = pack_records(recs, [s[0] for s in splits], [len(r) for r in reads],
                                   [len(s[1]) for s in splits], framed, [EMPTY_RICE] * len(reads),
                                   [EMPTY_RICE] * len(reads))
    assert offsets[-1] == len(region)
    return region


def _parsed_splits(codec, region):
    parsed = parse_records(region)
    assert all(p["c_large"] == 0 and p["l_bytes"] == EMPTY_RICE and p["p_bytes"] == EMPTY_RICE for p in parsed)
    small = codec.batch_inference_reads(list_of_compressed_reads=[p["s_bytes"] for p in parsed],
                                        list_of_lengths=[p["c_small"] for p in parsed], batch_size=4096)
    empty16, empty32 = np.zeros(0, np.uint16), np.zeros(0, np.uint32)
    return parsed, [(p["sig0"], s, empty16, empty32) for p, s in zip(parsed, small)]


@pytest.mark.parametrize("name", ["lossless", "lossy"])
def test_archive_region_oracle_on_cpu(golden, name, request):
    model = request.getfixturevalue(f"{name}_model")
    reads, recs, region_ref, decoded_ref, lsb = _archive(golden, name)
    codec = OracleBacked(model)
    region = _region(codec, reads, recs, signal.reads_to_tokens(reads, lsb))
    assert region == region_ref
    parsed, splits = _parsed_splits(codec, region)
    back = [signal.reassemble_signal(s[0], p["N"], s[1], s[2], s[3]) for p, s in zip(parsed, splits)]
    if lsb:
        back = [signal.lossy_decode(b, lsb) for b in back]
    assert all(np.array_equal(a, b) for a, b in zip(back, decoded_ref))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["lossless", "lossy"])
def test_archive_region_matches_reference(golden, name, request):
    from sigcomp_b200.codec import B200Compression
    model = request.getfixturevalue(f"{name}_model")
    reads, recs, region_ref, decoded_ref, lsb = _archive(golden, name)
    codec = B200Compression(chunk_len=2048, gpu=0, model=model)
    try:
        region = _region(codec, reads, recs, codec.split_signals(reads, lsb=lsb))
        assert region == region_ref
        parsed, splits = _parsed_splits(codec, region)
        back = codec.reassemble_signals(splits, [p["N"] for p in parsed], lsb=lsb)
        assert all(np.array_equal(a, b) for a, b in zip(back, decoded_ref))
    finally:
        codec.close()


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["lossless", "lossy"])
def test_archive_pipeline_matches_reference(golden, name, request):
    """The pipelined loops (reading, coding and writing overlapped) give the same records."""
    import io
    from sigcomp_b200.archive import compress_reads, decompress_records
    from sigcomp_b200.codec import B200Compression
    model = request.getfixturevalue(f"{name}_model")
    reads, recs, region_ref, decoded_ref, lsb = _archive(golden, name)
    codec = B200Compression(chunk_len=2048, gpu=0, model=model)
    try:
        out = io.BytesIO()
        batches = [(recs[i:i + 4], reads[i:i + 4]) for i in range(0, len(reads), 4)]
        ids, _ = compress_reads(codec, batches, out, lambda v, fallback_bits: EMPTY_RICE, lsb=lsb)
        assert out.getvalue() == region_ref and ids == [r[:16] for r in recs]
        got = [s for _, sig in decompress_records(codec, [region_ref], lambda b, c, fallback_bits: np.zeros(0, np.uint32),
                                                   lsb=lsb) for s in sig]
        assert len(got) == len(decoded_ref) and all(np.array_equal(a, b) for a, b in zip(got, decoded_ref))
    finally:
        codec.close()
