"""The GPU range coder alone (sc_encode_logits_device / sc_decode_logits_device, the counterparts
of the reference's GpuRangeStepEncoder and GpuRangeDecoder) on given logits, against:

- the reference's carry-heavy golden streams (tests/golden/coder.npz: ten streams from the
  reference CPU coder, eight of them through carry episodes, one a run of ten inverted words);
- seeded short streams that the oracle shows ending in the seal's extra zero word
  (cpu_entropy_coding.py:206-227).

All streams are coded in one call (one thread per stream) and decoded in one call (one warp per
stream).  The test asserts that the set covers every carry path of _encode_one and _seal
(cpu_entropy_coding.py:121-161, 206-227): carry episodes, runs of more than one inverted word,
inverted words flushed by the seal, and the seal's extra zero word.  Bit-exact."""

import ctypes

import numpy as np
import pytest

from oracle.oracle import OracleModel

pytestmark = pytest.mark.gpu

CAP = 2048 + 32


def _cases(golden, om):
    """[(logits, symbols, expected stream bytes, coverage)]"""
    z = np.load(golden / "coder.npz")
    off, woff = z["offsets"], z["word_offsets"]
    out = []
    for i in range(len(off) - 1):
        lg, sy = z["logits"][off[i]:off[i + 1]], z["symbols"][off[i]:off[i + 1]]
        ref = z["words"][woff[i]:woff[i + 1]].astype("<u4").tobytes()
        _, cov = om.encode_logits_coverage(lg, sy, CAP)
        out.append((lg, sy, ref, cov))
    # short random streams whose seal emits the extra zero word (found by a seeded search)
    zero = 0
    for seed in range(5000):
        rng = np.random.default_rng(seed)
        t = int(rng.integers(1, 6))
        lg = rng.integers(-128, 128, size=(t, 256)).astype(np.int8)
        sy = rng.integers(0, 256, size=t).astype(np.uint8)
        ref, cov = om.encode_logits_coverage(lg, sy, CAP)
        if cov["seal_zero"]:
            out.append((lg, sy, ref, cov))
            zero += 1
            if zero == 6:
                break
    return out


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def test_gpu_coder_matches_golden_carry_streams(golden, lossless_model):
    import torch
    from sigcomp_b200 import _lib
    from sigcomp_b200.codec import B200Compression
    om = OracleModel(lossless_model)
    cases = _cases(golden, om)
    cov = [c[3] for c in cases]
    assert sum(c["episodes"] for c in cov) > 0, "no carry episode covered"
    assert max(c["longest"] for c in cov) >= 2, "no run of several inverted words covered"
    assert any(c["seal_flush"] for c in cov), "no seal that flushes inverted words covered"
    assert any(c["seal_zero"] for c in cov), "no seal with the extra zero word covered"

    codec = B200Compression(chunk_len=2048, gpu=0, model=lossless_model)
    L, h, vp = codec._lib, codec.handle, ctypes.c_void_p
    st = vp(torch.cuda.current_stream().cuda_stream)
    lens = [len(c[1]) for c in cases]
    off = np.zeros(len(cases) + 1, np.int64)
    off[1:] = np.cumsum(lens)
    logits = _dev(np.concatenate([c[0] for c in cases]))
    symbols = _dev(np.concatenate([c[1] for c in cases]))
    d_off = _dev(off)
    cap = int(off[-1]) + 2 * len(cases) + 16
    words = torch.zeros(cap, dtype=torch.int32, device="cuda")
    woff = torch.zeros(len(cases) + 1, dtype=torch.int64, device="cuda")
    errs = torch.zeros(len(cases), dtype=torch.uint8, device="cuda")
    rc = L.sc_encode_logits_device(h, vp(logits.data_ptr()), vp(symbols.data_ptr()), vp(d_off.data_ptr()),
                                   len(cases), vp(words.data_ptr()), cap, vp(woff.data_ptr()),
                                   vp(errs.data_ptr()), st)
    _lib.check(rc, "sc_encode_logits_device")
    w, wo = words.cpu().numpy().view(np.uint32), woff.cpu().numpy()
    for i, c in enumerate(cases):
        assert w[wo[i]:wo[i + 1]].astype("<u4").tobytes() == c[2], f"stream {i} ({c[3]})"

    out = torch.full((int(off[-1]),), 7, dtype=torch.uint8, device="cuda")
    rc = L.sc_decode_logits_device(h, vp(logits.data_ptr()), vp(d_off.data_ptr()), vp(words.data_ptr()),
                                   vp(woff.data_ptr()), len(cases), vp(out.data_ptr()), vp(errs.data_ptr()), st)
    _lib.check(rc, "sc_decode_logits_device")
    assert np.array_equal(out.cpu().numpy(), np.concatenate([c[1] for c in cases]))
    assert not errs.cpu().numpy().any()
    codec.close()


def test_gpu_decoder_on_corrupted_streams_matches_oracle(golden, lossless_model):
    """200 copies of a golden stream, each with one bit flipped, decoded in one call: every
    stream either ends in the reference's error (cpu_entropy_coding.py:244-248) exactly where
    the oracle's decoder raises it, or decodes the same symbols as the oracle."""
    import torch
    from sigcomp_b200 import _lib
    from sigcomp_b200.codec import B200Compression
    z = np.load(golden / "coder.npz")
    off, woff = z["offsets"], z["word_offsets"]
    i = 9
    lg = z["logits"][off[i]:off[i + 1]]
    base = z["words"][woff[i]:woff[i + 1]]
    om = OracleModel(lossless_model)
    streams, want_err, want_sym = [], [], []
    for seed in range(200):
        rng = np.random.default_rng(seed)
        w = base.copy()
        w[rng.integers(0, len(w))] ^= np.uint32(1 << int(rng.integers(0, 32)))
        streams.append(w)
        try:
            want_sym.append(om.decode_logits(w.astype("<u4").tobytes(), lg).astype(np.uint8))
            want_err.append(0)
        except ValueError:
            want_sym.append(None)
            want_err.append(1)
    assert 0 < sum(want_err) < len(streams), "the set must hold both outcomes"
    n, T = len(streams), len(lg)
    codec = B200Compression(chunk_len=2048, gpu=0, model=lossless_model)
    L, h, vp = codec._lib, codec.handle, ctypes.c_void_p
    st = vp(torch.cuda.current_stream().cuda_stream)
    d_lg = _dev(np.tile(lg, (n, 1)))
    d_off = _dev(np.arange(n + 1, dtype=np.int64) * T)
    d_w = _dev(np.concatenate(streams).view(np.int32))
    d_wo = _dev(np.arange(n + 1, dtype=np.int64) * len(base))
    out = torch.zeros(n * T, dtype=torch.uint8, device="cuda")
    errs = torch.zeros(n, dtype=torch.uint8, device="cuda")
    rc = L.sc_decode_logits_device(h, vp(d_lg.data_ptr()), vp(d_off.data_ptr()), vp(d_w.data_ptr()),
                                   vp(d_wo.data_ptr()), n, vp(out.data_ptr()), vp(errs.data_ptr()), st)
    assert rc == _lib.SC_ERR_CORRUPT_STREAM
    assert f"in stream {want_err.index(1)}".encode() in L.sc_last_error()
    got_err, got = errs.cpu().numpy(), out.cpu().numpy().reshape(n, T)
    assert got_err.tolist() == want_err
    for c in range(n):
        if not want_err[c]:
            assert np.array_equal(got[c], want_sym[c]), c
    codec.close()
