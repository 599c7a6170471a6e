"""Read records of a SigComp archive, packed for a whole batch at once.

A SIG2 archive is a header followed by one record per read
(sigcomp/main.py:549-590, written by ``_write_read_payload``):

    REC_FMT  '<16sddBBdIIIQ'   the POD5 per-read record (read id, ...)
    SPLIT    '<hII'            sig0, N (samples), c_small (tokens)
    u32 + bytes                compressed tokens (the codec's framed streams)
    u32 + bytes                rice-coded large values
    u32 + bytes                rice-coded large-value positions

and an optional SIDX index of ``'<16sQ'`` (read id, record offset) entries
(sigcomp/archive_shards.py:22, 290-300).  The struct layouts are the archive
format and are kept exactly.

:func:`pack_records` builds the record region of a batch in one buffer (record
offsets come from one exclusive scan of the record sizes), :func:`parse_records`
reads it back, and :func:`write_region_at` writes a region at a given offset of
an archive file (``os.pwrite``), which is how the ranks of a sharded job write
their records into one archive without a merge copy: each rank's region starts
at the exclusive scan of the shard sizes (:mod:`sigcomp_b200.sharding`).
"""

import os
import struct

import numpy as np

REC_FMT = struct.Struct("<16sddBBdIIIQ")
SPLIT_HDR_FMT = struct.Struct("<hII")
U32 = struct.Struct("<I")
IDX_MAGIC = b"SIDX"
INDEX_ENTRY = struct.Struct("<16sQ")


def record_sizes(s_bytes, l_bytes, p_bytes):
    """Size of every record: fixed parts plus the three blobs."""
    fixed = REC_FMT.size + SPLIT_HDR_FMT.size + 3 * U32.size
    return fixed + np.asarray([len(a) + len(b) + len(c) for a, b, c in zip(s_bytes, l_bytes, p_bytes)],
                              dtype=np.int64)


def pack_records(rec_bytes, sig0, n, c_small, s_bytes, l_bytes, p_bytes):
    """The record region of a batch: (bytes, int64 offsets[n_reads + 1]).

    ``rec_bytes[i]`` is the packed REC_FMT record of read i; the other
    arguments are per-read values / blobs as ``_write_read_payload`` takes them.
    """
    count = len(rec_bytes)
    if not (len(sig0) == len(n) == len(c_small) == len(s_bytes) == len(l_bytes) == len(p_bytes) == count):
        raise ValueError("record fields differ in length")
    sizes = record_sizes(s_bytes, l_bytes, p_bytes)
    offsets = np.zeros(count + 1, dtype=np.int64)
    np.cumsum(sizes, out=offsets[1:])
    buf = bytearray(int(offsets[-1]))
    for i in range(count):
        rec = rec_bytes[i]
        if len(rec) != REC_FMT.size:
            raise ValueError(f"record {i} is not a {REC_FMT.size}-byte REC_FMT record")
        pos = int(offsets[i])
        buf[pos:pos + REC_FMT.size] = rec
        pos += REC_FMT.size
        SPLIT_HDR_FMT.pack_into(buf, pos, int(sig0[i]), int(n[i]), int(c_small[i]))
        pos += SPLIT_HDR_FMT.size
        for blob in (s_bytes[i], l_bytes[i], p_bytes[i]):
            U32.pack_into(buf, pos, len(blob))
            pos += U32.size
            buf[pos:pos + len(blob)] = blob
            pos += len(blob)
    return bytes(buf), offsets


def parse_records(buf):
    """Inverse of :func:`pack_records`: one dict per record, as ``_parse_read_payload`` returns
    (``rec`` is the unpacked REC_FMT tuple)."""
    mv = memoryview(buf)
    out, pos, end = [], 0, len(buf)
    while pos < end:
        if end - pos < REC_FMT.size + SPLIT_HDR_FMT.size:
            raise ValueError("truncated record")
        rec = REC_FMT.unpack_from(mv, pos)
        pos += REC_FMT.size
        sig0, n, c_small = SPLIT_HDR_FMT.unpack_from(mv, pos)
        pos += SPLIT_HDR_FMT.size
        blobs = []
        for _ in range(3):
            if end - pos < U32.size:
                raise ValueError("truncated record")
            (length,) = U32.unpack_from(mv, pos)
            pos += U32.size
            if end - pos < length:
                raise ValueError("truncated record")
            blobs.append(bytes(mv[pos:pos + length]))
            pos += length
        out.append({"rec": rec, "sig0": sig0, "N": n, "c_small": c_small, "c_large": n - 1 - c_small,
                    "s_bytes": blobs[0], "l_bytes": blobs[1], "p_bytes": blobs[2]})
    return out


def index_bytes(read_ids, record_offsets, data_start=0):
    """SIDX index of a record region: magic, count, then (read id, absolute offset) entries."""
    if len(read_ids) > 0xFFFFFFFF:
        raise ValueError("SIDX supports at most 2**32-1 reads")
    parts = [IDX_MAGIC + U32.pack(len(read_ids))]
    parts += [INDEX_ENTRY.pack(rid, int(data_start) + int(off)) for rid, off in zip(read_ids, record_offsets)]
    return b"".join(parts)


def write_region_at(path, offset, data):
    """Write ``data`` at byte ``offset`` of ``path`` (created if missing), without
    touching the rest of the file: each rank of a sharded job writes its own region."""
    fd = os.open(path, os.O_WRONLY | os.O_CREAT, 0o644)
    try:
        mv = memoryview(data)
        done = 0
        while done < len(mv):
            done += os.pwrite(fd, mv[done:], int(offset) + done)
    finally:
        os.close(fd)
