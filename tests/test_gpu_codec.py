"""GPU parity: the CUDA codec (through the C ABI) against the CPU oracle and the
golden streams of the SigComp reference.  Bit-exact everywhere."""

import ctypes

import numpy as np
import pytest

from oracle.oracle import OracleModel

pytestmark = pytest.mark.gpu

PATHS = ["tcgen05", "cuda_cores"]
# every MLP implementation the library ships: fused on SM pairs, the small-batch decoder
# (clusters of eight SMs per tile), fused on single SMs, one launch per layer, CUDA cores
ALL_PATHS = ["tcgen05", "tcgen05_small", "tcgen05_fused1", "tcgen05_layers", "cuda_cores"]


def _chunks(z, tok="tokens", off="offsets"):
    o = z[off]
    return [z[tok][o[i]:o[i + 1]] for i in range(len(o) - 1)]


def _streams(z):
    o = z["word_offsets"]
    return [z["words"][o[i]:o[i + 1]].astype("<u4").tobytes() for i in range(len(o) - 1)]


_CODECS = {}


def _codec(model, path="auto", chunk_len=2048):
    from sigcomp_b200.codec import B200Compression
    key = (model.name, id(model), chunk_len)
    if key not in _CODECS:
        _CODECS[key] = B200Compression(chunk_len=chunk_len, gpu=0, model=model)
    c = _CODECS[key]
    if path.startswith("tcgen05") and not _tc_available(c):
        pytest.skip("tcgen05 path not built for this geometry")
    c.set_mlp_path(path)
    return c


def _tc_available(codec):
    from sigcomp_b200 import _lib
    rc = codec._lib.sc_model_set_mlp_path(codec.handle, 1)
    codec._lib.sc_model_set_mlp_path(codec.handle, 0)
    return rc == _lib.SC_OK


def _gpu_logits(codec, windows):
    import torch
    w = torch.from_numpy(np.ascontiguousarray(windows, dtype=np.int16)).cuda()
    out = torch.empty((len(windows), 256), dtype=torch.int8, device="cuda")
    from sigcomp_b200 import _lib
    rc = codec._lib.sc_mlp_logits_device(codec.handle, ctypes.c_void_p(w.data_ptr()), len(windows),
                                         ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc)
    return out.cpu().numpy()


@pytest.mark.parametrize("name", ["lossless", "lossy"])
@pytest.mark.parametrize("path", PATHS)
def test_mlp_logits_match_reference_golden(golden, name, path, request):
    model = request.getfixturevalue(f"{name}_model")
    z = np.load(golden / f"mlp_{name}.npz")
    assert np.array_equal(_gpu_logits(_codec(model, path), z["windows"]), z["logits"])


@pytest.mark.parametrize("path", PATHS)
@pytest.mark.parametrize("rows", [1, 127, 128, 129, 1000, 4099])
def test_mlp_logits_random_model_match_oracle(path, rows):
    from sigcomp_b200.model import random_model
    model = random_model(11)
    rng = np.random.default_rng(rows)
    win = rng.integers(0, 257, size=(rows, 64)).astype(np.int16)
    win[: rows // 3, : 20] = 256
    got = _gpu_logits(_codec(model, path), win)
    want = OracleModel(model).mlp(win)
    assert np.array_equal(got, want)
    # the random model must exercise both clamps of the final layer
    assert (want == 127).any() or (want == -128).any() or rows < 128


@pytest.mark.parametrize("name", ["lossless", "lossy", "rna"])
@pytest.mark.parametrize("path", ALL_PATHS)
def test_streams_match_reference_golden(golden, name, path, request):
    # "rna": configuration-3-like reads coded with the lossless model
    model = request.getfixturevalue(f"{'lossless' if name == 'rna' else name}_model")
    z = np.load(golden / f"streams_{name}.npz")
    chunks, ref = _chunks(z), _streams(z)
    codec = _codec(model, path)
    assert codec.compress_chunks(chunks) == ref
    back = codec.decompress_chunks(ref, [len(c) for c in chunks])
    assert all(np.array_equal(a, b) for a, b in zip(back, chunks))


@pytest.mark.parametrize("name", ["lossless", "lossy", "rna"])
def test_read_framing_matches_reference_golden(golden, name, request):
    model = request.getfixturevalue(f"{'lossless' if name == 'rna' else name}_model")
    z = np.load(golden / f"streams_{name}.npz")
    reads = _chunks(z, "read_tokens", "read_offsets")
    framed_ref = [z["framed"][z["framed_offsets"][i]:z["framed_offsets"][i + 1]].tobytes()
                  for i in range(len(reads))]
    codec = _codec(model)
    framed = codec.batch_inference_reads(list_of_reads=reads, batch_size=20480)
    assert framed == framed_ref
    back = codec.batch_inference_reads(list_of_compressed_reads=framed,
                                       list_of_lengths=[len(r) for r in reads], batch_size=20480)
    assert all(np.array_equal(a, b) for a, b in zip(back, reads))


def test_edge_chunks(lossless_model):
    codec = _codec(lossless_model)
    rng = np.random.default_rng(5)
    chunks = [np.empty(0, np.uint8), np.asarray([0], np.uint8), np.asarray([255], np.uint8),
              rng.integers(0, 256, size=2048).astype(np.uint8), np.full(2048, 255, np.uint8),
              np.zeros(2048, np.uint8), rng.integers(0, 3, size=65).astype(np.uint8), np.empty(0, np.uint8)]
    streams = codec.compress_chunks(chunks)
    assert streams[0] == b"" and streams[-1] == b""
    assert streams == OracleModel(lossless_model).compress_chunks(chunks)
    back = codec.decompress_chunks(streams, [len(c) for c in chunks])
    assert all(np.array_equal(a, b) for a, b in zip(back, chunks))
    assert codec.compress_chunks([]) == []
    assert codec.decompress_chunks([], []) == []



@pytest.mark.parametrize("chunk_len", [1, 63, 64, 65, 129, 300, 4096, 65535])
def test_chunk_lengths_match_oracle(lossless_model, chunk_len):
    """chunk_len is a codec parameter (1..65535, the '<H' frame): windows shorter than 64, tiles
    of 128 rows cut at chunk ends and the longest decoder launches all stay bit-exact, with full,
    short and empty chunks in one batch."""
    codec = _codec(lossless_model, chunk_len=chunk_len)
    rng = np.random.default_rng(chunk_len)
    chunks = [rng.integers(0, 40, size=chunk_len).astype(np.uint8) for _ in range(1 if chunk_len > 5000 else 3)]
    chunks += [rng.integers(0, 256, size=max(chunk_len // 3, 1)).astype(np.uint8), np.empty(0, np.uint8)]
    streams = codec.compress_chunks(chunks)
    assert streams == OracleModel(lossless_model).compress_chunks(chunks, chunk_len=chunk_len)
    back = codec.decompress_chunks(streams, [len(c) for c in chunks])
    assert all(np.array_equal(a, b) for a, b in zip(back, chunks))

def test_reads_without_small_tokens(lossless_model):
    codec = _codec(lossless_model)
    reads = [np.empty(0, np.uint8), np.asarray([7, 9], np.uint8), np.empty(0, np.uint8)]
    framed = codec.batch_inference_reads(list_of_reads=reads)
    assert framed[0] == b"" and framed[2] == b""
    back = codec.batch_inference_reads(list_of_compressed_reads=framed, list_of_lengths=[0, 2, 0])
    assert [list(x) for x in back] == [[], [7, 9], []]


def test_corrupt_stream_raises(lossless_model):
    codec = _codec(lossless_model)
    bad = np.asarray([0xFFFFFFFF, 0xFFFFFFFF], dtype="<u4").tobytes()   # quantile >= 2^24 at step 0
    good = codec.compress_chunks([np.arange(50, dtype=np.uint8)])[0]
    with pytest.raises(ValueError, match="invalid range stream"):
        codec.decompress_chunks([good, bad], [50, 10])
    with pytest.raises(ValueError, match="invalid range stream"):
        OracleModel(lossless_model).decompress_chunks([good, bad], [50, 10])
    # the model handle stays usable after a stream error
    assert np.array_equal(codec.decompress_chunks([good], [50])[0], np.arange(50, dtype=np.uint8))



def test_capi_rejects_bad_arguments(lossless_model):
    """The host-buffer entry points validate sizes and pointers before any device work and
    report SC_ERR_INVALID_ARGUMENT with a message; the handle stays usable."""
    from sigcomp_b200 import _lib
    codec = _codec(lossless_model)
    lib, h = codec._lib, codec.handle
    ptr = lambda a: ctypes.c_void_p(a.ctypes.data)
    tok = np.arange(10, dtype=np.uint8)
    words = np.zeros(64, np.uint32)
    woff = np.zeros(3, np.int64)

    def compress(tokens, off):
        return lib.sc_compress_chunks(h, tokens, ptr(off), len(off) - 1, ptr(words), len(words), ptr(woff),
                                      None, None)

    cases = [
        (None, np.asarray([0, 10], np.int64)),                       # tokens missing
        (ptr(tok), np.asarray([1, 10], np.int64)),                   # offsets[0] != 0
        (ptr(tok), np.asarray([0, 6, 4], np.int64)),                 # decreasing offsets
    ]
    for tokens, off in cases:
        assert compress(tokens, off) == _lib.SC_ERR_INVALID_ARGUMENT
        assert lib.sc_last_error()
    long_tok = np.zeros(2049, np.uint8)
    assert compress(ptr(long_tok), np.asarray([0, 2049], np.int64)) == _lib.SC_ERR_INVALID_ARGUMENT
    assert b"chunk_len" in lib.sc_last_error()

    out = np.zeros(16, np.uint8)

    def decompress(w, off, lengths):
        return lib.sc_decompress_chunks(h, w, ptr(off), ptr(lengths), len(lengths), ptr(out), None, None)

    lens = np.asarray([10], np.int64)
    assert decompress(None, np.asarray([0, 4], np.int64), lens) == _lib.SC_ERR_INVALID_ARGUMENT
    assert decompress(ptr(words), np.asarray([1, 4], np.int64), lens) == _lib.SC_ERR_INVALID_ARGUMENT
    assert decompress(ptr(words), np.asarray([0, 0], np.int64), lens) == _lib.SC_ERR_INVALID_ARGUMENT
    assert decompress(ptr(words), np.asarray([0, 4], np.int64), np.asarray([2049], np.int64)) == \
        _lib.SC_ERR_INVALID_ARGUMENT
    # still usable
    streams = codec.compress_chunks([tok])
    assert np.array_equal(codec.decompress_chunks(streams, [10])[0], tok)

def test_truncated_and_mismatched_streams_match_oracle(lossless_model):
    codec = _codec(lossless_model)
    om = OracleModel(lossless_model)
    rng = np.random.default_rng(9)
    chunks = [rng.integers(0, 30, size=n).astype(np.uint8) for n in (300, 1000, 2048)]
    streams = codec.compress_chunks(chunks)
    cases = [s[: 4 * max(1, len(s) // 8)] for s in streams]          # truncated streams
    cases += [s[::-1][: len(s) - len(s) % 4] or s for s in streams]  # scrambled bytes
    lengths = [len(c) for c in chunks] * 2
    for data, n in zip(cases, lengths):
        try:
            want = om.decompress_chunks([data], [n])[0]
        except ValueError:
            with pytest.raises(ValueError):
                codec.decompress_chunks([data], [n])
            continue
        assert np.array_equal(codec.decompress_chunks([data], [n])[0], want)


@pytest.mark.parametrize("path", ALL_PATHS)
def test_random_model_streams_match_oracle(path):
    from sigcomp_b200.model import random_model
    model = random_model(3)
    rng = np.random.default_rng(3)
    chunks = [rng.integers(0, 256, size=n).astype(np.uint8) for n in (1, 17, 128, 129, 2048, 700)]
    codec = _codec(model, path)
    om = OracleModel(model)
    streams = codec.compress_chunks(chunks)
    assert streams == om.compress_chunks(chunks)
    back = codec.decompress_chunks(streams, [len(c) for c in chunks])
    assert all(np.array_equal(a, b) for a, b in zip(back, chunks))


def test_decoder_bias_outside_the_tile_range():
    """The pair decoder adds the bias of layers after the first with an MMA against a bias tile of
    int8 digits, which reaches |b| <= 258,127; a layer with a bias beyond that keeps its bias in the
    epilogue.  A model mixing both kinds of layer must still decode the oracle's streams."""
    from sigcomp_b200.model import random_model
    model = random_model(7)
    for layer in (2, len(model.biases) - 1):
        b = np.asarray(model.biases[layer]).copy()
        b[::37] = np.where(b[::37] >= 0, 300_000, -300_000)
        model.biases[layer] = b
    rng = np.random.default_rng(7)
    chunks = [rng.integers(0, 256, size=n).astype(np.uint8) for n in (1, 300, 2048, 1500, 64)]
    om = OracleModel(model)
    streams = om.compress_chunks(chunks)
    for path in ALL_PATHS:
        codec = _codec(model, path)
        assert codec.compress_chunks(chunks) == streams, path
        back = codec.decompress_chunks(streams, [len(c) for c in chunks])
        assert all(np.array_equal(a, c) for a, c in zip(back, chunks)), path


def test_synthetic_reads_match_oracle(lossless_model):
    from oracle import signal
    from sigcomp_b200 import synthetic
    reads = synthetic.make_reads("r10_config1", seed=1, count=2)
    toks = [signal.split_signal(r)[1] for r in reads]
    chunks = []
    for t in toks:
        chunks += [t[i:i + 2048] for i in range(0, len(t), 2048)]
    codec = _codec(lossless_model)
    streams = codec.compress_chunks(chunks)
    assert streams == OracleModel(lossless_model).compress_chunks(chunks, backend="int_mm")


def test_large_round_trip_properties(lossless_model):
    """Config-2-shaped reads at a size the oracle cannot check directly: round trip
    identity, determinism, and agreement of the two MLP paths."""
    from oracle import signal
    from sigcomp_b200 import synthetic
    reads = synthetic.make_reads("r10_lognormal", seed=2, count=60)
    toks = [signal.split_signal(r)[1] for r in reads]
    codec = _codec(lossless_model)
    lengths = [len(t) for t in toks]
    framed = codec.batch_inference_reads(list_of_reads=toks, batch_size=20480)
    assert framed == codec.batch_inference_reads(list_of_reads=toks, batch_size=20480)
    back = codec.batch_inference_reads(list_of_compressed_reads=framed, list_of_lengths=lengths)
    assert all(np.array_equal(a, b) for a, b in zip(back, toks))
    if _tc_available(codec):
        for path in ("cuda_cores", "tcgen05_layers", "tcgen05_fused1"):
            codec.set_mlp_path(path)
            assert codec.batch_inference_reads(list_of_reads=toks[:8]) == framed[:8], path
        codec.set_mlp_path("auto")
    bits = 8 * sum(len(f) for f in framed) / sum(lengths)
    assert 4.0 < bits < 8.0


def test_decoder_runs_several_tiles_per_lane(lossless_model):
    """More chunks than the SM pairs' lanes hold at once (74 pairs x 6 lanes x 256 rows): one
    persistent launch decodes them all, each lane taking its next pair-tile when the previous
    one ends, with chunk lengths varying inside and across tiles.  Streams against the oracle
    on a sample, every chunk by round trip."""
    from oracle import signal
    from sigcomp_b200 import _lib, synthetic
    L = 64
    reads = synthetic.make_reads("r10_lognormal", seed=9, count=300)
    toks = np.concatenate([signal.split_signal(r)[1] for r in reads])
    rng = np.random.default_rng(3)
    lens = rng.integers(0, L + 1, size=160000)
    lens[rng.random(len(lens)) < 0.5] = L                 # half of them full, like real batches
    off = np.zeros(len(lens) + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    assert off[-1] <= len(toks)
    tokens = toks[:off[-1]]
    codec = _codec(lossless_model, chunk_len=L)
    words, woff = codec.compress_flat(tokens, off)
    sample = list(range(0, len(lens), 997))
    chunks = [tokens[off[i]:off[i + 1]] for i in sample]
    ref = OracleModel(lossless_model).compress_chunks(chunks, chunk_len=L, backend="int_mm")
    assert [words[woff[i]:woff[i + 1]].astype("<u4").tobytes() for i in sample] == ref
    launches = _lib.kernel_launches()
    back = codec.decompress_flat(words, woff, lens)
    assert np.array_equal(back, tokens)
    # the persistent decoder is one launch (plus the start-of-sequence block and the
    # decoder-state set-up), whatever the number of chunks
    assert _lib.kernel_launches() - launches <= 4


@pytest.mark.parametrize("layer", [0, 1, 8])
@pytest.mark.parametrize("rows", [1, 127, 1000])
def test_single_layer_matches_oracle(lossless_model, layer, rows):
    """sc_linear_layer_device (one tcgen05 layer: the reference's bit_exact_linear_kernel,
    quant_mlp_export.py:21-76) against the oracle's layer (cpu_int_inference.py:206-256)."""
    import torch
    from sigcomp_b200 import _lib
    codec = _codec(lossless_model)
    K = int(lossless_model.weights[layer].shape[1])
    N = int(lossless_model.weights[layer].shape[0])
    x = np.random.default_rng(rows + layer).integers(-128, 128, size=(rows, K)).astype(np.int8)
    xd = torch.from_numpy(x).cuda()
    y = torch.zeros((rows, N), dtype=torch.int8, device="cuda")
    rc = codec._lib.sc_linear_layer_device(codec.handle, layer, ctypes.c_void_p(xd.data_ptr()), rows,
                                           ctypes.c_void_p(y.data_ptr()),
                                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "sc_linear_layer_device")
    assert np.array_equal(y.cpu().numpy(), OracleModel(lossless_model).linear(x, layer))


def _mixed_chunks(n, L, seed):
    from oracle import signal
    from sigcomp_b200 import synthetic
    reads = synthetic.make_reads("r10_lognormal", seed=seed, count=max(4, n * L // 20000 + 2))
    toks = np.concatenate([signal.split_signal(r)[1] for r in reads])
    rng = np.random.default_rng(seed)
    lens = rng.integers(0, L + 1, size=n)
    lens[rng.random(n) < 0.4] = L
    off = np.zeros(n + 1, np.int64)
    np.cumsum(lens, out=off[1:])
    assert off[-1] <= len(toks)
    return toks[:off[-1]], off, lens


@pytest.mark.parametrize("n,L", [(700, 256), (5000, 64)])
def test_small_batch_decoder_matches_pairs(lossless_model, n, L):
    """Small batches decode on a cluster of eight SMs per 128-row tile: path 0 picks it for at
    most SMs / 8 tiles, path 5 forces it (5,000 chunks: 40 tiles over the clusters, each cluster
    taking several tiles in turn).  Against the pair kernel (path 1) and the input, with lengths
    mixed inside and across tiles, empty chunks included; streams against the oracle on a sample."""
    tokens, off, lens = _mixed_chunks(n, L, seed=n)
    codec = _codec(lossless_model, chunk_len=L)
    words, woff = codec.compress_flat(tokens, off)
    sample = list(range(0, n, 97))
    ref = OracleModel(lossless_model).compress_chunks([tokens[off[i]:off[i + 1]] for i in sample], chunk_len=L,
                                                      backend="int_mm")
    assert [words[woff[i]:woff[i + 1]].astype("<u4").tobytes() for i in sample] == ref
    try:
        for path in ("tcgen05_small", "tcgen05", "auto"):
            codec.set_mlp_path(path)
            assert np.array_equal(codec.decompress_flat(words, woff, lens), tokens), path
    finally:
        codec.set_mlp_path("auto")


def test_small_batch_decoder_corrupt_streams(lossless_model):
    """Damaged streams on the small-batch decoder end in the same per-chunk errors as on the pair
    kernel: the reference's invalid-stream condition stops a chunk's decoding, the other chunks
    of its tile decode on."""
    from sigcomp_b200 import _lib
    tokens, off, lens = _mixed_chunks(300, 256, seed=11)
    codec = _codec(lossless_model, chunk_len=256)
    words, woff = codec.compress_flat(tokens, off)
    rng = np.random.default_rng(12)
    bad = words.copy()
    hit = rng.choice(len(bad), size=60, replace=False)
    bad[hit] ^= rng.integers(1, 2 ** 32, size=60, dtype=np.uint64).astype(np.uint32)
    got = {}
    try:
        for path in ("tcgen05_small", "tcgen05"):
            codec.set_mlp_path(path)
            out = np.zeros(max(int(lens.sum()), 1), np.uint8)
            err = np.zeros(len(lens), np.uint8)
            rc = codec._lib.sc_decompress_chunks(codec.handle, _lib_ptr(bad), _lib_ptr(woff), _lib_ptr(lens), len(lens),
                                                 _lib_ptr(out), _lib_ptr(err), None)
            got[path] = (rc, out.copy(), err.copy())
    finally:
        codec.set_mlp_path("auto")
    rc_s, out_s, err_s = got["tcgen05_small"]
    rc_p, out_p, err_p = got["tcgen05"]
    assert rc_s == rc_p
    assert np.array_equal(err_s, err_p) and err_s.any()
    # chunks without an error decode identically
    for i in np.flatnonzero(err_s == 0):
        assert np.array_equal(out_s[off[i]:off[i + 1]], out_p[off[i]:off[i + 1]])


def _lib_ptr(a):
    return ctypes.c_void_p(a.ctypes.data)
