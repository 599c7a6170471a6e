"""The allocation-free logits entry point, sc_mlp_logits_device_noalloc.

It serves callers that cannot call cudaMalloc (a host framework that has
reserved the GPU's memory for its own pool, or a latency-critical caller that
cannot accept cudaMalloc's device-wide synchronisation).  Its activations live
in one fixed device array that every call shares, so the test calls it twice
in a row, on batches of different sizes, and checks both against the
allocating entry point, sc_mlp_logits_device, and against the CPU oracle's
integer MLP (a C restatement of the reference's bit-exact layers), so an error
shared by the two CUDA paths still fails.  Logits are int8 and must match
exactly.

The file name makes pytest collect it last; it also passes alone in a fresh
process.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _logits(codec, windows, entry):
    import torch
    from sigcomp_b200 import _lib
    w = torch.from_numpy(np.ascontiguousarray(windows, dtype=np.int16)).cuda()
    out = torch.full((len(windows), 256), 99, dtype=torch.int8, device="cuda")
    fn = getattr(codec._lib, entry)
    rc = fn(codec.handle, ctypes.c_void_p(w.data_ptr()), len(windows), ctypes.c_void_p(out.data_ptr()),
            _stream())
    _lib.check(rc, entry)
    return out.cpu().numpy()


@pytest.fixture(scope="module")
def codec():
    from sigcomp_b200.codec import B200Compression
    from sigcomp_b200.model import random_model
    return B200Compression(chunk_len=2048, gpu=0, model=random_model(11))


@pytest.fixture(scope="module")
def oracle_model():
    from oracle.oracle import OracleModel
    from sigcomp_b200.model import random_model
    return OracleModel(random_model(11))


def _windows(rows, seed):
    rng = np.random.default_rng(seed)
    win = rng.integers(0, 257, size=(rows, 64)).astype(np.int16)
    win[: rows // 4, : 16] = 256          # start-of-sequence padding, as at a chunk's head
    return win


def test_no_alloc_logits_match_allocating_entry_point_twice(codec, oracle_model):
    from sigcomp_b200 import _lib
    limit = 4096                          # SC_NOALLOC_MAX_ROWS
    # first call fills the whole scratch, the second (smaller) one runs over its leftovers
    for rows, seed in ((limit, 1), (777, 2)):
        win = _windows(rows, seed)
        want = _logits(codec, win, "sc_mlp_logits_device")
        got = _logits(codec, win, "sc_mlp_logits_device_noalloc")
        assert np.array_equal(got, want), f"rows={rows}"
        if rows == 777:
            assert np.array_equal(got, oracle_model.mlp(win)), "no-alloc logits differ from the CPU oracle"
    assert (want == 127).any() or (want == -128).any()
    # above the fixed limit the call is refused, and a later call still works
    import torch
    w = torch.zeros((limit + 1, 64), dtype=torch.int16, device="cuda")
    out = torch.empty((limit + 1, 256), dtype=torch.int8, device="cuda")
    rc = codec._lib.sc_mlp_logits_device_noalloc(codec.handle, ctypes.c_void_p(w.data_ptr()), limit + 1,
                                                 ctypes.c_void_p(out.data_ptr()), _stream())
    assert rc == _lib.SC_ERR_INVALID_ARGUMENT
    assert b"scratch limit" in codec._lib.sc_last_error()
    win = _windows(5, 3)
    got = _logits(codec, win, "sc_mlp_logits_device_noalloc")
    assert np.array_equal(got, _logits(codec, win, "sc_mlp_logits_device"))
    assert np.array_equal(got, oracle_model.mlp(win))
