"""Pipelined archive record I/O around the codec: the batch loops of SigComp's compress and
decompress commands, with the host's work overlapped with the GPU's.

SigComp's compress loop (sigcomp/main.py:844-931, ``flush_compress_batch``) splits a batch of
reads, codes it, rice-codes the large values, writes every record and only then reads the next
batch; its decompress loop (main.py:1142-1190) parses, decodes and reassembles the same way.  The
GPU idles while the host reads, packs and writes, and the host idles while the GPU codes.  Here
the three stages of each direction run at once, over bounded queues of whole batches:

compress (:func:`compress_reads`)
  1. a prefetch thread drains the caller's batch source (SigComp's POD5 reader), so reading
     batch i+1 overlaps coding batch i;
  2. the calling thread splits the batch on the GPU and runs the neural coder
     (``split_signals`` + ``batch_inference_reads``); the CUDA library and torch release the GIL
     while the device works;
  3. a writer thread (:class:`RecordWriter`) rice-codes the large values and position deltas
     with the caller's coder, packs the batch's records into one buffer
     (:func:`~sigcomp_b200.records.pack_records`) and writes it, while the codec works on the
     next batch.

decompress (:func:`decompress_records`)
  1. a prefetch thread parses the next region's records and rice-decodes their large values;
  2. the calling thread decodes the neural streams and reassembles the signals on the GPU.

Rice coding itself stays in SigComp (``_rice_compress`` / ``_rice_decompress``, main.py:174-186,
which call fast_rice): the caller passes those two functions in.  The records come out in batch
order and byte-identical to SigComp's ``_write_read_payload``; the writer also returns each
record's offset for the SIDX index (:func:`~sigcomp_b200.records.index_bytes`).
"""

import queue
import threading

import numpy as np

from .records import REC_FMT, pack_records, parse_records

_DONE = object()
# how long a stage waits on a full or empty queue before it looks again whether the other side
# has stopped (seconds); no wait is unbounded
_POLL = 0.1


class _Failure:
    def __init__(self, exc):
        self.exc = exc


def prefetch(iterable, depth=2):
    """Iterate over ``iterable`` on a background thread, at most ``depth`` items ahead.

    An exception raised by the source is raised again here, at the item where it happened.
    Leaving the loop early (break, or an error in the caller) stops the thread after the item it
    is producing.
    """
    if depth < 1:
        raise ValueError("depth must be positive")
    q = queue.Queue(maxsize=depth)
    stop = threading.Event()

    def put(item):
        while not stop.is_set():
            try:
                q.put(item, timeout=_POLL)
                return True
            except queue.Full:
                continue
        return False

    def run():
        try:
            for item in iterable:
                if not put(item):
                    return
        except BaseException as e:          # handed to the consumer
            put(_Failure(e))
            return
        put(_DONE)

    t = threading.Thread(target=run, name="sigcomp-prefetch", daemon=True)
    t.start()
    try:
        while True:
            try:
                item = q.get(timeout=_POLL)
            except queue.Empty:
                if not t.is_alive() and q.empty():
                    raise RuntimeError("the prefetch thread ended without finishing the source")
                continue
            if item is _DONE:
                return
            if isinstance(item, _Failure):
                raise item.exc
            yield item
    finally:
        stop.set()
        t.join()


class RecordWriter:
    """Writer thread for the record region of an archive.

    :meth:`submit` hands over one coded batch; the thread rice-codes its large values and position
    deltas (``rice_compress(values, fallback_bits=16 / 32)``, SigComp's ``_rice_compress``), packs
    its records and writes them to ``out`` (any object with ``write(bytes)``), in submission order.
    At most ``depth`` batches wait; a further :meth:`submit` blocks until one is written.
    :meth:`close` writes what is pending and returns ``(read_ids, record_offsets)``, the offsets
    counted from ``data_start`` (the position of the first record in the archive).  An error on the
    thread is raised by the next :meth:`submit` or by :meth:`close`.
    """

    def __init__(self, out, rice_compress, depth=2, data_start=0):
        if depth < 1:
            raise ValueError("depth must be positive")
        self._out = out
        self._rice = rice_compress
        self._q = queue.Queue(maxsize=depth)
        self._error = None
        self._stopped = threading.Event()
        self._pos = int(data_start)
        self._ids, self._offsets = [], []
        self._closed = False
        self._thread = threading.Thread(target=self._run, name="sigcomp-record-writer", daemon=True)
        self._thread.start()

    def _run(self):
        try:
            while True:
                item = self._q.get()
                if item is _DONE:
                    return
                recs, splits, n_samples, framed = item
                l_bytes = [self._rice(s[2], fallback_bits=16) for s in splits]
                p_bytes = [self._rice(s[3], fallback_bits=32) for s in splits]
                region, offsets = pack_records(recs, [s[0] for s in splits], n_samples,
                                               [len(s[1]) for s in splits], framed, l_bytes, p_bytes)
                self._out.write(region)
                self._ids.extend(r[:16] for r in recs)
                self._offsets.extend((self._pos + offsets[:-1]).tolist())
                self._pos += len(region)
        except BaseException as e:
            self._error = e
        finally:
            self._stopped.set()

    def _raise_if_failed(self):
        if self._error is not None:
            raise self._error

    def submit(self, recs, splits, n_samples, framed):
        """Queue one batch: the REC_FMT records, ``split_signals`` output, the reads' sample
        counts and the framed neural streams of its reads."""
        if self._closed:
            raise ValueError("the writer is closed")
        if not (len(recs) == len(splits) == len(n_samples) == len(framed)):
            raise ValueError("batch fields differ in length")
        if any(len(r) != REC_FMT.size for r in recs):
            raise ValueError(f"records must be {REC_FMT.size}-byte REC_FMT records")
        item = (list(recs), list(splits), [int(n) for n in n_samples], list(framed))
        while True:
            self._raise_if_failed()
            if self._stopped.is_set():
                raise RuntimeError("the record writer stopped")
            try:
                self._q.put(item, timeout=_POLL)
                return
            except queue.Full:
                continue

    def close(self):
        """Write every queued batch, stop the thread and return ``(read_ids, record_offsets)``."""
        if not self._closed:
            self._closed = True
            while not self._stopped.is_set():
                try:
                    self._q.put(_DONE, timeout=_POLL)
                    break
                except queue.Full:
                    continue
            self._thread.join()
        self._raise_if_failed()
        return list(self._ids), np.asarray(self._offsets, dtype=np.int64)

    def abort(self):
        """Stop without waiting for queued batches to be written (after an error elsewhere)."""
        self._closed = True
        while True:
            try:
                self._q.get_nowait()
            except queue.Empty:
                break
        try:
            self._q.put_nowait(_DONE)
        except queue.Full:
            pass
        self._thread.join()


def compress_reads(codec, batches, out, rice_compress, lsb=0, depth=2, batch_size=1024, data_start=0):
    """Compress batches of reads into archive records written to ``out``.

    ``batches`` yields ``(records, reads)``: the reads' packed REC_FMT records (bytes) and their
    int16 samples.  ``codec`` is a :class:`~sigcomp_b200.codec.B200Compression`;
    ``rice_compress`` is SigComp's ``_rice_compress``.  Returns ``(read_ids, record_offsets)`` for
    the SIDX index, the offsets counted from ``data_start``.
    """
    writer = RecordWriter(out, rice_compress, depth=depth, data_start=data_start)
    try:
        for recs, reads in prefetch(batches, depth):
            reads = list(reads)
            if not reads:
                continue
            splits = codec.split_signals(reads, lsb=lsb)
            framed = codec.batch_inference_reads(list_of_reads=[s[1] for s in splits], batch_size=batch_size)
            writer.submit(recs, splits, [len(r) for r in reads], framed)
    except BaseException:
        writer.abort()
        raise
    return writer.close()


def _parse_region(region, rice_decompress):
    """Records of one region with their large values and position deltas rice-decoded."""
    parsed = parse_records(region)
    for p in parsed:
        c = p["c_large"]
        if c < 0:
            raise ValueError("record holds more tokens than samples")
        p["large"] = np.asarray(rice_decompress(p["l_bytes"], c, fallback_bits=16)).astype(np.uint16)
        p["pos"] = np.asarray(rice_decompress(p["p_bytes"], c, fallback_bits=32)).astype(np.uint32)
        if len(p["large"]) != c or len(p["pos"]) != c:
            raise ValueError("rice-decoded large values do not match the record's count")
    return parsed


def decompress_records(codec, regions, rice_decompress, lsb=0, depth=2, batch_size=4096):
    """Decode archive record regions back to signals, one batch per region.

    ``regions`` yields byte strings of whole records (one batch each); ``rice_decompress`` is
    SigComp's ``_rice_decompress``.  Yields ``(records, signals)`` per region: the unpacked REC_FMT
    tuples and the int16 signals (lossy-decoded when ``lsb`` > 0).
    """
    parsed_batches = prefetch((_parse_region(r, rice_decompress) for r in regions), depth)
    try:
        for parsed in parsed_batches:
            if not parsed:
                continue
            small = codec.batch_inference_reads(list_of_compressed_reads=[p["s_bytes"] for p in parsed],
                                                list_of_lengths=[p["c_small"] for p in parsed], batch_size=batch_size)
            splits = [(p["sig0"], s, p["large"], p["pos"]) for p, s in zip(parsed, small)]
            signals = codec.reassemble_signals(splits, [p["N"] for p in parsed], lsb=lsb)
            yield [p["rec"] for p in parsed], signals
    finally:
        parsed_batches.close()
