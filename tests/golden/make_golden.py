"""Generate the golden fixtures in tests/golden/ by running the SigComp reference.

Run where the reference tree is available (it is not needed afterwards):

    NUMBA_CACHE_DIR=/tmp/nbcache python tests/golden/make_golden.py --reference <sigcomp checkout>

The reference is imported from its own tree (never copied).  Its CPU codec
(``sigcomp.cpu_compression.CPUQuantMLPCompression``, int_mm + Numba backends)
and its Python-backend range coder produce every expected output below.
``sigcomp.main`` imports ``pod5``, ``numcodecs`` and ``fast_rice`` at module
level; empty stand-in modules satisfy those imports (none of them is used by
the functions called here).

Fixtures written:
  models.json      - digests / scalars of the integer models derived by the reference loader
  mlp_<model>.npz  - context windows and the int8 logits the reference MLP gives for them
  coder.npz        - logits + symbols -> range-coded streams (python and numba coders)
  streams_<model>.npz - synthetic reads -> tokens -> reference compress_chunks streams
  signal.npz       - reference _split_signal / lossy transform outputs
  sharding.json    - sample counts -> read ranges of the reference multi-GPU partition
                     (sigcomp/read_assignment.py); `--only sharding` rewrites just this file
  streams_rna.npz  - RNA004-like reads (configuration 3 generator) through the reference CPU codec
                     with the lossless model; `--only rna` rewrites just this file
  records.npz      - read records written by the reference's _write_read_payload and the SIDX
                     index entries (sigcomp/main.py:549-590, archive_shards.py:22);
                     `--only records` rewrites just this file
  archive.npz      - int16 reads -> the reference's whole compress path to the record region, and
                     that region back to signals (main.py:844-931, 1142-1165), lossless and lossy;
                     `--only archive` rewrites just this file
"""

import argparse
import hashlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def _import_reference(path):
    for name in ("pod5", "numcodecs", "fast_rice"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.path.insert(0, str(path))
    import sigcomp.cpu_compression as cc
    import sigcomp.cpu_entropy_coding as ce
    import sigcomp.cpu_int_inference as ci
    import sigcomp.main as sm
    return cc, ce, ci, sm


def _digest(arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _model_arrays(decoder, lut):
    emb = decoder.embedding.weight_q.numpy()
    ws = [l.weight_q.numpy() for l in decoder.mlp]
    bs = [l.bias_q.numpy() for l in decoder.mlp]
    m0 = np.asarray([l.M0 for l in decoder.mlp], dtype=np.int64)
    sh = np.asarray([l.shift for l in decoder.mlp], dtype=np.int32)
    relu = np.asarray([1 if l.has_relu else 0 for l in decoder.mlp], dtype=np.uint8)
    return [emb, *ws, *bs, m0, sh, relu, np.asarray(lut, dtype=np.int64)], m0, sh, relu


def _coder_cases(ce, rng):
    """Logit/symbol streams that cover peaked, flat and carry-heavy coding."""
    cases = []
    lengths = [1, 2, 7, 64, 300, 600, 1024, 2048, 512, 700]
    for i, T in enumerate(lengths):
        kind = i % 5
        if kind == 0:      # peaked, symbols drawn near the peak
            base = rng.integers(-128, 0, size=(T, 256))
            peak = rng.integers(0, 256, size=T)
            base[np.arange(T), peak] = 127
            sym = np.where(rng.random(T) < 0.8, peak, rng.integers(0, 256, size=T))
        elif kind == 1:    # nearly flat logits, uniform symbols (carry-heavy)
            base = rng.integers(100, 128, size=(T, 256))
            sym = rng.integers(0, 256, size=T)
        elif kind == 2:    # flat logits, symbols at the top of the alphabet push lower up
            base = np.full((T, 256), 5)
            sym = np.where(rng.random(T) < 0.9, 255, rng.integers(0, 256, size=T))
        elif kind == 3:    # extreme: very improbable symbols (max 24 bits/symbol)
            base = np.full((T, 256), -128)
            base[:, 0] = 127
            sym = rng.integers(1, 256, size=T)
        else:              # random logits
            base = rng.integers(-128, 128, size=(T, 256))
            sym = rng.integers(0, 256, size=T)
        cases.append((base.astype(np.int8), sym.astype(np.int64)))
    return cases


def _encode_reference(ce, lut, logits, symbols, backend):
    T = len(symbols)
    enc = ce.CpuRangeStepEncoder(1, 2048 + 32, backend=backend, parallel="serial")
    saw_inversion = False
    valid = np.asarray([T], dtype=np.int64)
    for t in range(T):
        enc.encode_step_int8(logits[t:t + 1], lut, symbols[t:t + 1], valid, t)
        saw_inversion |= bool(enc.num_inverted[0] > 0)
    return enc.get_compressed()[0], saw_inversion


def _record_cases(path):
    """A batch of read records through the reference writer, parser and index entry format."""
    import io
    cc, ce, ci, sm = _import_reference(path)
    import sigcomp.archive_shards as ash
    rng = np.random.default_rng(11)
    recs, meta, blobs = [], [], []
    buf = io.BytesIO()
    for i in range(40):
        rec = sm.REC_FMT.pack(rng.bytes(16), float(rng.random()), float(rng.normal()), int(rng.integers(0, 256)),
                              int(rng.integers(0, 256)), float(rng.random() * 5000), int(rng.integers(0, 2 ** 32)),
                              int(rng.integers(0, 2 ** 32)), int(rng.integers(0, 2 ** 32)), int(rng.integers(0, 2 ** 62)))
        n = int(rng.integers(1, 100000))
        c_small = int(rng.integers(0, n))
        sizes = [0 if i % 7 == 0 else int(rng.integers(0, 400)) for _ in range(3)]
        s_b, l_b, p_b = (rng.bytes(k) for k in sizes)
        sig0 = int(rng.integers(-32768, 32768))
        sm._write_read_payload(buf, rec, sig0, n, c_small, s_b, l_b, p_b)
        recs.append(rec)
        meta.append((sig0, n, c_small))
        blobs.append((s_b, l_b, p_b))
    region = buf.getvalue()
    # parse back with the reference reader
    rd = io.BytesIO(region)
    parsed = []
    while True:
        item = sm._parse_read_payload(rd)
        if item is None:
            break
        info, split = item
        parsed.append((split["sig0"], split["N"], split["c_small"], split["c_large"]))
    assert len(parsed) == 40
    ids = [r[:16] for r in recs]
    offsets = np.cumsum([0] + [len(r) + sm.SPLIT_HDR_FMT.size + 12 + sum(len(x) for x in b)
                               for r, b in zip(recs, blobs)])[:-1]
    index = ash.IDX_MAGIC + sm.U32.pack(40) + b"".join(ash.INDEX_ENTRY.pack(i_, 1000 + int(o)) for i_, o in zip(ids, offsets))

    def cat(parts):
        return np.frombuffer(b"".join(parts), dtype=np.uint8), np.cumsum([0] + [len(p_) for p_ in parts]).astype(np.int64)

    rec_flat, rec_off = cat(recs)
    s_flat, s_off = cat([b[0] for b in blobs])
    l_flat, l_off = cat([b[1] for b in blobs])
    p_flat, p_off = cat([b[2] for b in blobs])
    np.savez_compressed(HERE / "records.npz", region=np.frombuffer(region, dtype=np.uint8),
                        rec=rec_flat, rec_off=rec_off, meta=np.asarray(meta, dtype=np.int64),
                        s=s_flat, s_off=s_off, l=l_flat, l_off=l_off, p=p_flat, p_off=p_off,
                        parsed=np.asarray(parsed, dtype=np.int64), index=np.frombuffer(index, dtype=np.uint8),
                        index_base=np.asarray([1000]))


def _rna_streams(path):
    """Configuration-3-like reads (levels N(800, 90), dwell 30, noise 20: more large deltas) through
    the reference CPU codec with the lossless model (no RNA004 model is bundled)."""
    cc, ce, ci, sm = _import_reference(path)
    sys.path.insert(0, str(REPO))
    from sigcomp_b200 import synthetic
    model_dir = Path(path) / "sigcomp" / "pretrained_models"
    codec = cc.CPUQuantMLPCompression(chunk_len=2048, model_path=str(model_dir / "lossless.pth"),
                                      inference_backend="int_mm", epilogue="numba", inference_batch_size=4096)
    rng = np.random.default_rng(33)
    reads = [synthetic.synth_read(rng, n, synthetic.RNA004) for n in (6000, 2500, 700, 2)]
    token_reads = [sm._split_signal(s)[1] for s in reads]
    chunks = []
    for tr in token_reads:
        chunks.extend(tr[i:i + 2048] for i in range(0, len(tr), 2048))
    streams = codec.compress_chunks(chunks, max_batch_size=1024)
    lengths = [len(c) for c in chunks]
    back = codec.decompress_chunks(streams, lengths, max_batch_size=4096)
    assert all(np.array_equal(a, b) for a, b in zip(back, chunks))
    framed = codec.batch_inference_reads(list_of_reads=token_reads, batch_size=1024)
    tok = np.concatenate([np.asarray(c, np.uint8) for c in chunks])
    np.savez_compressed(
        HERE / "streams_rna.npz", tokens=tok, offsets=np.cumsum([0] + lengths).astype(np.int64),
        words=np.frombuffer(b"".join(streams), dtype="<u4"),
        word_offsets=np.cumsum([0] + [len(x) // 4 for x in streams]).astype(np.int64),
        read_tokens=np.concatenate(token_reads),
        read_offsets=np.cumsum([0] + [len(t) for t in token_reads]).astype(np.int64),
        framed=np.frombuffer(b"".join(framed), dtype=np.uint8),
        framed_offsets=np.cumsum([0] + [len(f) for f in framed]).astype(np.int64))
    print("rna chunks", len(chunks), "tokens", len(tok), "words", sum(len(x) for x in streams) // 4)


def _archive_cases(path):
    """Whole read records of the archive's record region, both ways, from the reference's own code.

    Compress (main.py:844-931): the lossy transform when lsb > 0, ``_split_signal``, the CPU codec's
    ``batch_inference_reads``, ``_rice_compress`` of the large values and position deltas, and
    ``_write_read_payload``.  Decompress (main.py:1142-1165): ``_parse_read_payload``,
    ``batch_inference_reads`` on the framed streams, ``_reassemble_signal`` and the lossy decode.
    Every delta of these reads fits a token (|delta| <= 127), so both rice blobs are the reference's
    empty encoding (one zero byte, main.py:176-177) and fast_rice is never called.
    """
    import io
    cc, ce, ci, sm = _import_reference(path)
    model_dir = Path(path) / "sigcomp" / "pretrained_models"
    rng = np.random.default_rng(44)
    lengths = [9000, 4100, 2050, 2049, 2048, 700, 66, 65, 3, 2, 1]
    out = {}
    for name, lsb in (("lossless", 0), ("lossy", 3)):
        codec = cc.CPUQuantMLPCompression(chunk_len=2048, model_path=str(model_dir / f"{name}.pth"),
                                          inference_backend="int_mm", epilogue="numba", inference_batch_size=4096)
        reads = []
        for n in lengths:
            d = np.clip(np.rint(rng.normal(0.0, 30.0, size=n - 1)), -127, 127).astype(np.int64)
            reads.append((int(rng.integers(300, 700)) + np.concatenate([[0], np.cumsum(d)])).astype(np.int16))
        recs = [sm.REC_FMT.pack(rng.bytes(16), float(rng.random()), float(rng.normal()), int(rng.integers(0, 256)),
                                int(rng.integers(0, 256)), float(rng.random() * 5000), int(rng.integers(0, 2 ** 32)),
                                int(rng.integers(0, 2 ** 32)), int(rng.integers(0, 2 ** 32)),
                                int(rng.integers(0, 2 ** 62))) for _ in reads]
        splits, small = [], []
        for sig in reads:
            if lsb > 0:
                sig = sm._lossy_encode(sm._reduce_lsb(sig, lsb), lsb)
            s = sm._split_signal(sig)
            assert len(s[2]) == 0, "every delta fits a token"
            splits.append(s)
            small.append(s[1])
        framed = codec.batch_inference_reads(list_of_reads=small, batch_size=1024, use_tqdm=False)
        buf = io.BytesIO()
        for rec, sig, (sig0, sv, l_adj, pos), s_bytes in zip(recs, reads, splits, framed):
            sm._write_read_payload(buf, rec, sig0, len(sig), len(sv), s_bytes,
                                   sm._rice_compress(l_adj, fallback_bits=16), sm._rice_compress(pos, fallback_bits=32))
        region = buf.getvalue()
        # back through the reference's reader and decoder
        rd = io.BytesIO(region)
        parsed = []
        while (item := sm._parse_read_payload(rd)) is not None:
            parsed.append(item)
        decoded_small = codec.batch_inference_reads(list_of_compressed_reads=[p[1]["s_bytes"] for p in parsed],
                                                    list_of_lengths=[p[1]["c_small"] for p in parsed],
                                                    batch_size=4096, use_tqdm=False)
        decoded = []
        for (_, split), sv in zip(parsed, decoded_small):
            sig = sm._reassemble_signal(split["sig0"], split["N"], sv, split["c_large"], split["l_bytes"],
                                        split["p_bytes"])
            decoded.append(sm._lossy_decode(sig, lsb) if lsb > 0 else sig)
        out[f"{name}_lsb"] = np.asarray([lsb])
        out[f"{name}_reads"] = np.concatenate(reads)
        out[f"{name}_decoded"] = np.concatenate(decoded).astype(np.int16)
        out[f"{name}_rec"] = np.frombuffer(b"".join(recs), dtype=np.uint8)
        out[f"{name}_region"] = np.frombuffer(region, dtype=np.uint8)
        print("archive", name, "reads", len(reads), "region bytes", len(region))
    out["read_offsets"] = np.cumsum([0] + lengths).astype(np.int64)
    np.savez_compressed(HERE / "archive.npz", **out)


def _sharding_cases(path):
    """Read ranges of sample_balanced_ranges for edge cases and synthetic read sets."""
    sys.path.insert(0, str(path))
    from sigcomp.read_assignment import sample_balanced_ranges
    rng = np.random.default_rng(7)
    inputs = [
        ([], 4), ([5], 1), ([5], 8), ([0, 0, 0, 0, 0], 2), ([0, 0, 0, 0, 0, 0, 0], 3),
        ([1, 1, 1, 1], 4), ([10, 1, 1, 1], 2), ([1, 1, 1, 10], 2), ([3, 3], 2), ([4, 2, 2], 2),
        ([1000000, 1, 1, 1, 1, 1], 3), ([2 ** 62, 2 ** 62 - 1, 1, 7, 2 ** 62], 3), ([0, 9, 0, 9, 0], 4),
    ]
    for workers in (1, 2, 3, 4, 7, 8):
        counts = np.clip(np.rint(rng.lognormal(np.log(30000), 0.8, size=500)), 2000, 1000000)
        inputs.append(([int(c) for c in counts], workers))
        counts = rng.integers(0, 5, size=37)
        inputs.append(([int(c) for c in counts], workers))
    cases = []
    for counts, workers in inputs:
        ranges = sample_balanced_ranges(counts, workers)
        cases.append({"counts": counts, "workers": workers,
                      "ranges": [[r.start, r.stop, r.num_samples] for r in ranges]})
    errors = []
    for counts, workers in (([1, 2], 0), ([1, -1], 2), ([2 ** 64 - 1, 1], 2)):
        try:
            sample_balanced_ranges(counts, workers)
            errors.append({"counts": counts, "workers": workers, "error": None})
        except ValueError as e:
            errors.append({"counts": counts, "workers": workers, "error": str(e)})
    (HERE / "sharding.json").write_text(json.dumps({"cases": cases, "errors": errors}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SIGCOMP_REFERENCE", str(REPO / "baseline" / "_ref")),
                    help="root of the SigComp source tree (holding sigcomp/); default: $SIGCOMP_REFERENCE, "
                         "else the offline install under baseline/_ref")
    ap.add_argument("--only", choices=["sharding", "records", "rna", "archive"], default=None)
    args = ap.parse_args()
    os.environ.setdefault("NUMBA_CACHE_DIR", "/tmp/nbcache")
    if args.only in (None, "sharding"):
        _sharding_cases(Path(args.reference))
    if args.only in (None, "records"):
        _record_cases(Path(args.reference))
    if args.only in (None, "rna"):
        _rna_streams(Path(args.reference))
    if args.only in (None, "archive"):
        _archive_cases(Path(args.reference))
    if args.only is not None:
        return
    cc, ce, ci, sm = _import_reference(Path(args.reference))
    sys.path.insert(0, str(REPO))
    from sigcomp_b200 import synthetic

    rng = np.random.default_rng(20260101)
    models = {}
    model_dir = Path(args.reference) / "sigcomp" / "pretrained_models"

    # 1. integer models and MLP rows
    for name in ("lossless", "lossy"):
        dec = ci.load_cpu_decoder(str(model_dir / f"{name}.pth"), backend="int_mm", epilogue="numba")
        dec_np = ci.load_cpu_decoder(str(model_dir / f"{name}.pth"), backend="numpy", epilogue="torch")
        lut = ce.build_integer_exp_lut(float(dec.output_scale))
        arrays, m0, sh, relu = _model_arrays(dec, lut)
        models[name] = {
            "digest": _digest(arrays), "multipliers": m0.tolist(), "shifts": sh.tolist(),
            "relu": relu.tolist(), "output_scale": float(dec.output_scale),
            "exp_lut": [int(x) for x in lut],
        }
        # windows: chunk starts (SOS padded), random tokens, small-token-heavy, extremes
        rows = []
        for r in range(64):
            w = np.full(64, 256, dtype=np.int64)
            kind = r % 4
            start = rng.integers(0, 65)
            if kind == 0:
                w[start:] = rng.integers(0, 256, size=64 - start)
            elif kind == 1:
                w[:] = np.minimum(np.abs(rng.normal(0, 20, size=64)).astype(np.int64), 255)
            elif kind == 2:
                w[start:] = rng.integers(0, 40, size=64 - start)
            else:
                w[:] = rng.choice([0, 255, 256], size=64)
            rows.append(w)
        win = np.stack(rows)
        import torch
        with torch.inference_mode():
            logits = dec._ar_step(torch.from_numpy(win))[:, 0].numpy().copy()
            logits_np = dec_np._ar_step(torch.from_numpy(win))[:, 0].numpy().copy()
        assert np.array_equal(logits, logits_np), "reference int_mm and numpy backends disagree"
        np.savez_compressed(HERE / f"mlp_{name}.npz", windows=win.astype(np.int16), logits=logits)

    (HERE / "models.json").write_text(json.dumps(models, indent=1))

    # 2. range coder, python and numba backends
    lut = np.asarray(models["lossless"]["exp_lut"], dtype=np.int64)
    cases = _coder_cases(ce, rng)
    logits_all, sym_all, off, streams, inv = [], [], [0], [], []
    for lg, sy in cases:
        s_py, inv_py = _encode_reference(ce, lut, lg, sy, "python")
        s_nb, _ = _encode_reference(ce, lut, lg, sy, "numba")
        assert s_py == s_nb, "reference python and numba coders disagree"
        # the reference decoder must invert it
        dec = ce.CpuRangeDecoder([s_py], backend="python", parallel="serial")
        got = [int(dec.decode_step_int8(lg[t:t + 1], lut, np.asarray([len(sy)]), t)[0]) for t in range(len(sy))]
        assert got == [int(x) for x in sy]
        logits_all.append(lg)
        sym_all.append(sy)
        off.append(off[-1] + len(sy))
        streams.append(s_py)
        inv.append(inv_py)
    word_off = np.cumsum([0] + [len(s) // 4 for s in streams])
    np.savez_compressed(
        HERE / "coder.npz", lut=lut, logits=np.concatenate(logits_all),
        symbols=np.concatenate(sym_all).astype(np.uint8), offsets=np.asarray(off, dtype=np.int64),
        words=np.frombuffer(b"".join(streams), dtype="<u4"), word_offsets=word_off.astype(np.int64),
        inversions=np.asarray(inv, dtype=np.uint8))
    print("coder cases with an inversion (carry) pending:", int(np.sum(inv)), "of", len(inv))

    # 3. signal transform
    sigs = [synthetic.synth_read(rng, 5000), synthetic.synth_read(rng, 1, synthetic.R10),
            np.asarray([0, 32767, -32768, 0, 300, -300, 5, 5, 5, 1000], dtype=np.int16),
            np.asarray([7, 7], dtype=np.int16)]
    sig_fx = {}
    for i, s in enumerate(sigs):
        sig0, small, large, pos = sm._split_signal(s)
        lossy = sm._lossy_encode(sm._reduce_lsb(s, 3), 3)
        sig_fx[f"sig{i}"] = s
        sig_fx[f"sig0_{i}"] = np.asarray([sig0])
        sig_fx[f"small{i}"] = small
        sig_fx[f"large{i}"] = large
        sig_fx[f"pos{i}"] = pos
        sig_fx[f"lossy{i}"] = lossy
        sig_fx[f"lossy_dec{i}"] = sm._lossy_decode(lossy, 3)
    np.savez_compressed(HERE / "signal.npz", **sig_fx)

    # 4. end-to-end chunk streams through the reference CPU codec
    for name, lsb in (("lossless", 0), ("lossy", 3)):
        codec = cc.CPUQuantMLPCompression(chunk_len=2048, model_path=str(model_dir / f"{name}.pth"),
                                          inference_backend="int_mm", epilogue="numba",
                                          inference_batch_size=4096)
        reads = [synthetic.synth_read(rng, n) for n in (4097, 2049, 30)]
        # a read with no small tokens: every delta is large
        reads.append(np.asarray(np.arange(12) * 400 - 2000, dtype=np.int16))
        token_reads = []
        for s in reads:
            if lsb:
                s = sm._lossy_encode(sm._reduce_lsb(s, lsb), lsb)
            token_reads.append(sm._split_signal(s)[1])
        chunks = []
        for tr in token_reads:
            chunks.extend(tr[i:i + 2048] for i in range(0, len(tr), 2048))
        # explicit edge chunks: empty, a single token, exactly chunk_len
        chunks += [np.empty(0, np.uint8), np.asarray([3], np.uint8),
                   rng.integers(0, 40, size=2048).astype(np.uint8)]
        streams = codec.compress_chunks(chunks, max_batch_size=1024)
        lengths = [len(c) for c in chunks]
        back = codec.decompress_chunks(streams, lengths, max_batch_size=4096)
        assert all(np.array_equal(a, b) for a, b in zip(back, chunks))
        framed = codec.batch_inference_reads(list_of_reads=token_reads, batch_size=1024)
        tok = np.concatenate([np.asarray(c, np.uint8) for c in chunks])
        np.savez_compressed(
            HERE / f"streams_{name}.npz", tokens=tok,
            offsets=np.cumsum([0] + lengths).astype(np.int64),
            words=np.frombuffer(b"".join(streams), dtype="<u4"),
            word_offsets=np.cumsum([0] + [len(s) // 4 for s in streams]).astype(np.int64),
            read_tokens=np.concatenate(token_reads),
            read_offsets=np.cumsum([0] + [len(t) for t in token_reads]).astype(np.int64),
            framed=np.frombuffer(b"".join(framed), dtype=np.uint8),
            framed_offsets=np.cumsum([0] + [len(f) for f in framed]).astype(np.int64))
        print(name, "chunks", len(chunks), "tokens", len(tok), "words", sum(len(s) for s in streams) // 4)


if __name__ == "__main__":
    main()
