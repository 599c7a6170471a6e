"""Failure detection on the GPU without a GPU fault: every device-side wait of
the library is bounded, and a wait that runs out is reported as an error status
while the context stays usable (the self test waits on a barrier and a counter
that nothing signals)."""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_device_wait_timeout_is_reported_and_context_stays_usable():
    from sigcomp_b200 import _lib
    from sigcomp_b200.codec import B200Compression
    from sigcomp_b200.model import random_model
    codec = B200Compression(chunk_len=2048, gpu=0, model=random_model(5))
    rc = codec._lib.sc_selftest_wait_timeout(codec.handle, None)
    assert rc == _lib.SC_ERR_CUDA
    assert b"timed out" in codec._lib.sc_last_error()
    # the error flag was consumed and the device still works
    rng = np.random.default_rng(0)
    chunks = [rng.integers(0, 30, size=n).astype(np.uint8) for n in (5, 300, 2048)]
    streams = codec.compress_chunks(chunks)
    back = codec.decompress_chunks(streams, [len(c) for c in chunks])
    assert all(np.array_equal(a, b) for a, b in zip(back, chunks))
    codec.close()
