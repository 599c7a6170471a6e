"""Host-side logic that needs no GPU: C-ABI exports, signal transform, synthetic
data, framing validation and error mapping."""

import re
import ctypes
import struct

import numpy as np
import pytest

from oracle import signal
from sigcomp_b200 import _lib, synthetic
from conftest import REPO
from oracle_backed import OracleBacked


def _declared_symbols():
    names = set()
    for h in (REPO / "include").glob("*.h"):
        names |= set(re.findall(r"^SC_API[^(]*?\b(sc_\w+)\s*\(", h.read_text(), flags=re.M))
    return names


def test_library_exports_every_declared_symbol():
    declared = _declared_symbols()
    assert {"sc_model_create", "sc_compress_chunks", "sc_decompress_chunks", "sc_last_error"} <= declared
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in sorted(declared):
        assert hasattr(lib, name), name
    assert set(_lib.EXPORTS) <= declared
    L = _lib.load()
    assert L.sc_version().decode().startswith("sigcomp_b200")


def test_status_codes_map_to_reference_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.SC_ERR_INVALID_ARGUMENT)
    with pytest.raises(ValueError):
        _lib.check(_lib.SC_ERR_CORRUPT_STREAM)
    with pytest.raises(OverflowError):
        _lib.check(_lib.SC_ERR_CAPACITY)
    with pytest.raises(_lib.CodecError):
        _lib.check(_lib.SC_ERR_CUDA)
    _lib.check(_lib.SC_OK)


def test_model_create_without_gpu_fails_cleanly(lossless_model):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from sigcomp_b200.codec import B200Compression
    with pytest.raises((_lib.CodecError, ValueError)):
        B200Compression(chunk_len=2048, model=lossless_model)


def test_split_signal_matches_reference(golden):
    z = np.load(golden / "signal.npz")
    i = 0
    while f"sig{i}" in z.files:
        sig0, small, large, pos = signal.split_signal(z[f"sig{i}"])
        assert sig0 == int(z[f"sig0_{i}"][0])
        assert np.array_equal(small, z[f"small{i}"]) and small.dtype == np.uint8
        assert np.array_equal(large, z[f"large{i}"])
        assert np.array_equal(pos, z[f"pos{i}"])
        lossy = signal.lossy_encode(signal.reduce_lsb(z[f"sig{i}"], 3), 3)
        assert np.array_equal(lossy, z[f"lossy{i}"])
        assert np.array_equal(signal.lossy_decode(lossy, 3), z[f"lossy_dec{i}"])
        n = len(z[f"sig{i}"])
        back = signal.reassemble_signal(sig0, n, small, large, pos)
        assert np.array_equal(back, z[f"sig{i}"])
        i += 1
    assert i >= 3


def test_synthetic_reads_are_seeded():
    a = synthetic.make_reads("r10_lognormal", seed=3, count=5)
    b = synthetic.make_reads("r10_lognormal", seed=3, count=5)
    assert all(np.array_equal(x, y) for x, y in zip(a, b))
    assert all(2000 <= len(x) <= 1_000_000 for x in a)
    c = synthetic.make_reads("r10_config1", seed=0, count=2)
    assert [len(x) for x in c] == [20000, 20000]
    x = c[0].astype(np.float64)
    assert 350 < x.mean() < 650
    toks = signal.split_signal(c[0])[1]
    assert len(toks) > 0.95 * (len(c[0]) - 1)       # deltas are overwhelmingly small


class _FramingOnly:
    """Exercises the framing validation of B200Compression without a device."""

    def __new__(cls):
        from sigcomp_b200.codec import B200Compression
        obj = object.__new__(B200Compression)
        obj.chunk_len = 4
        obj.window_size = 64
        obj.SOS_token = 256
        return obj


def test_framing_validation_errors():
    codec = _FramingOnly()
    with pytest.raises(ValueError, match="batch_size"):
        codec.batch_inference_reads(list_of_reads=[np.zeros(3, np.uint8)], batch_size=0)
    with pytest.raises(ValueError, match="integers in"):
        codec.batch_inference_reads(list_of_reads=[np.asarray([1, 300])])
    with pytest.raises(ValueError, match="one-dimensional"):
        codec.batch_inference_reads(list_of_reads=[np.zeros((2, 2), np.uint8)])
    with pytest.raises(ValueError, match="required"):
        codec.batch_inference_reads(list_of_compressed_reads=[b""])
    with pytest.raises(ValueError, match="counts differ"):
        codec.batch_inference_reads(list_of_compressed_reads=[b""], list_of_lengths=[1, 2])
    with pytest.raises(ValueError, match="Truncated"):
        codec.batch_inference_reads(list_of_compressed_reads=[b"\x04"], list_of_lengths=[3])
    with pytest.raises(ValueError, match="Invalid or truncated"):
        codec.batch_inference_reads(list_of_compressed_reads=[b"\x03\x00abc"], list_of_lengths=[3])
    with pytest.raises(ValueError, match="Trailing"):
        codec.batch_inference_reads(list_of_compressed_reads=[b"\x04\x00abcdxx"], list_of_lengths=[3])
    with pytest.raises(ValueError, match="nonnegative"):
        codec.batch_inference_reads(list_of_compressed_reads=[b""], list_of_lengths=[-1])
    # empty reads need no device work
    assert [len(x) for x in codec.batch_inference_reads(list_of_compressed_reads=[b"", b""],
                                                        list_of_lengths=[0, 0])] == [0, 0]
    with pytest.raises(ValueError, match="chunk_len"):
        codec.decompress_chunks([b"abcd"], [5])
    with pytest.raises(ValueError, match="token length"):
        codec.decompress_chunks([b""], [3])
    with pytest.raises(ValueError, match="token length"):
        codec.decompress_chunks([b"abcd"], [0])
    with pytest.raises(ValueError, match="counts differ"):
        codec.decompress_chunks([b"abcd"], [1, 2])
    with pytest.raises(ValueError, match="exceeds chunk_len"):
        codec.compress_chunks([np.zeros(5, np.uint8)])


@pytest.mark.parametrize("name", ["lossless", "lossy", "rna"])
def test_read_framing_matches_reference_golden_on_cpu(golden, name, request):
    """batch_inference_reads' chunking and '<H' framing reproduce the reference's framed reads
    (ReadFramingMixin, cpu_compression.py:28-84) and parse them back."""
    model = request.getfixturevalue(f"{'lossless' if name == 'rna' else name}_model")
    z = np.load(golden / f"streams_{name}.npz")
    o = z["read_offsets"]
    reads = [z["read_tokens"][o[i]:o[i + 1]] for i in range(len(o) - 1)]
    fo = z["framed_offsets"]
    framed_ref = [z["framed"][fo[i]:fo[i + 1]].tobytes() for i in range(len(reads))]
    codec = OracleBacked(model)
    assert codec.batch_inference_reads(list_of_reads=reads) == framed_ref
    back = codec.batch_inference_reads(list_of_compressed_reads=framed_ref, list_of_lengths=[len(r) for r in reads])
    assert all(np.array_equal(a, b) for a, b in zip(back, reads))


def test_build_refuses_spills_in_the_fused_kernels():
    """The build fails if ptxas spills registers in a kernel whose tcgen05.ld results are in flight
    in registers; other kernels may spill."""
    from sigcomp_b200.build_ext import spilling_kernels
    log = "\n".join([
        "ptxas info    : Function properties for _ZN2sc12_GLOBAL__N_18k_fused2ILb1EEEvNS_12Fused2ParamsE",
        "    48 bytes stack frame, 36 bytes spill stores, 44 bytes spill loads",
        "ptxas info    : Used 128 registers, used 1 barriers, 48 bytes cumulative stack size",
        "ptxas info    : Function properties for _ZN2sc12_GLOBAL__N_18k_fused2ILb0EEEvNS_12Fused2ParamsE",
        "    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads",
        "ptxas info    : Function properties for _ZN2sc7k_layerEv",
        "    0 bytes stack frame, 8 bytes spill stores, 8 bytes spill loads",
    ])
    assert spilling_kernels(log) == [("_ZN2sc12_GLOBAL__N_18k_fused2ILb1EEEvNS_12Fused2ParamsE", 36, 44)]
    assert spilling_kernels(log.replace("36 bytes spill stores, 44", "0 bytes spill stores, 0")) == []


def test_frame_helpers_round_trip_and_error_order():
    """sc_frame_reads / sc_unframe_reads (the C passes of batch_inference_reads' framing) on
    random streams, and the reference's error order: reads are checked one after the other, so
    the first malformed read decides the message (cpu_compression.py:58-80)."""
    import ctypes
    L = _lib.load()
    rng = np.random.default_rng(12)
    n_reads, chunk_len = 50, 7
    lengths = rng.integers(0, 40, size=n_reads)
    nchunks = (lengths + chunk_len - 1) // chunk_len
    read_chunks = np.zeros(n_reads + 1, np.int64)
    np.cumsum(nchunks, out=read_chunks[1:])
    nwords = rng.integers(1, 20, size=int(read_chunks[-1]))
    woff = np.zeros(len(nwords) + 1, np.int64)
    np.cumsum(nwords, out=woff[1:])
    words = rng.integers(0, 2 ** 32, size=int(woff[-1]), dtype=np.uint64).astype(np.uint32)
    out = np.empty(4 * len(words) + 2 * len(nwords), np.uint8)
    out_off = np.zeros(n_reads + 1, np.int64)
    vp = ctypes.c_void_p
    assert L.sc_frame_reads(vp(words.ctypes.data), vp(woff.ctypes.data), vp(read_chunks.ctypes.data), n_reads,
                            vp(out.ctypes.data), len(out), vp(out_off.ctypes.data)) == _lib.SC_OK
    framed = [out[out_off[r]:out_off[r + 1]].tobytes() for r in range(n_reads)]
    for r in range(n_reads):           # the reference's frame: '<H' byte count, then the stream
        want = b"".join(struct.pack("<H", 4 * int(nwords[c])) + words[woff[c]:woff[c + 1]].astype("<u4").tobytes()
                        for c in range(read_chunks[r], read_chunks[r + 1]))
        assert framed[r] == want

    def unframe(reads, lens):
        lens = np.asarray(lens, np.int64)
        nb = np.asarray([len(d) for d in reads], np.int64)
        cap_c = int(((np.maximum(lens, 0) + chunk_len - 1) // chunk_len).sum())
        w = np.empty(max(int(nb.sum()) // 4, 1), np.uint32)
        wo = np.zeros(cap_c + 1, np.int64)
        cl = np.zeros(max(cap_c, 1), np.int64)
        rc_ = np.zeros(len(reads) + 1, np.int64)
        bad = np.zeros(1, np.int64)
        ptrs = (ctypes.c_char_p * max(len(reads), 1))(*reads)
        rc = L.sc_unframe_reads(ctypes.cast(ptrs, vp), vp(nb.ctypes.data), vp(lens.ctypes.data), len(reads),
                                chunk_len, vp(w.ctypes.data), len(w), vp(wo.ctypes.data), vp(cl.ctypes.data), cap_c,
                                vp(rc_.ctypes.data), vp(bad.ctypes.data))
        return rc, int(bad[0]), w, wo, cl, rc_

    rc, bad, w, wo, cl, rc_ = unframe(framed, lengths)
    assert rc == _lib.SC_OK and bad == -1
    assert np.array_equal(rc_, read_chunks) and np.array_equal(wo, woff)
    assert np.array_equal(w[:len(words)], words)
    assert cl.tolist()[:len(nwords)] == [min(chunk_len, int(lengths[r]) - chunk_len * (c - read_chunks[r]))
                                         for r in range(n_reads) for c in range(read_chunks[r], read_chunks[r + 1])]
    # the first malformed read decides: a truncated read 3 before a trailing-data read 7
    reads = list(framed)
    k3 = next(r for r in range(3, n_reads) if lengths[r] > 0)
    k7 = next(r for r in range(k3 + 1, n_reads) if lengths[r] > 0)
    reads[k3] = reads[k3][:-1]
    reads[k7] = reads[k7] + b"\x00"
    rc, bad, *_ = unframe(reads, lengths)
    assert rc == _lib.SC_ERR_INVALID_ARGUMENT and bad == k3
    assert b"Invalid or truncated" in L.sc_last_error()
    reads = list(framed)
    reads[k7] = reads[k7] + b"\x00"
    rc, bad, *_ = unframe(reads, lengths)
    assert bad == k7 and b"Trailing" in L.sc_last_error()
