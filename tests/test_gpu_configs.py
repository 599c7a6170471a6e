"""BASELINE configurations 3 and 4 on the GPU at 200 reads each, against the CPU oracle.

- configuration 3: RNA004-like reads (rna_lognormal generator: median 15,000 samples, levels
  N(800, 90), dwell 30, noise 20) coded with the lossless model (no RNA004 model is bundled);
- configuration 4: configuration-2 reads in the lossy mode (lossy model, lsb_eliminate 3).

Each read goes through the GPU split (after the lossy step), the fused compress kernel, the
persistent decoder and the GPU reassembly.  The split must equal the oracle's restatement of
_split_signal (main.py:504-521), the chunk streams the oracle's (cpu_compression.py:178-257 with
the int_mm MLP, the reference's default CPU backend), and the round trip SigComp's lossy output
(main.py:158-171, 1162-1164).  Integer work: bit-exact."""

import numpy as np
import pytest

from oracle import signal
from oracle.oracle import OracleModel

pytestmark = pytest.mark.gpu

READS = 200


@pytest.mark.parametrize("generator,model_name,lsb", [("rna_lognormal", "lossless", 0),
                                                      ("r10_lognormal", "lossy", 3)],
                         ids=["config3", "config4"])
def test_configuration_reads_match_oracle(generator, model_name, lsb, request):
    from sigcomp_b200 import synthetic
    from sigcomp_b200.codec import B200Compression
    model = request.getfixturevalue(f"{model_name}_model")
    reads = synthetic.make_reads(generator, seed=77, count=READS)
    codec = B200Compression(chunk_len=2048, gpu=0, model=model)
    splits = codec.split_signals(reads, lsb=lsb)
    want = signal.reads_to_tokens(reads, lsb)
    for got, exp in zip(splits, want):
        assert got[0] == exp[0] and all(np.array_equal(a, b) for a, b in zip(got[1:], exp[1:]))
    chunks = [sp[1][i:i + 2048] for sp in splits for i in range(0, len(sp[1]), 2048)]
    assert len(chunks) > 2 * READS
    streams = codec.compress_chunks(chunks)
    assert streams == OracleModel(model).compress_chunks(chunks, backend="int_mm")
    back = codec.decompress_chunks(streams, [len(c) for c in chunks])
    assert all(np.array_equal(a, b) for a, b in zip(back, chunks))
    rebuilt = codec.reassemble_signals(splits, [len(r) for r in reads], lsb=lsb)
    for r, y in zip(reads, rebuilt):
        x = signal.lossy_decode(signal.lossy_encode(signal.reduce_lsb(r, lsb), lsb), lsb) if lsb else r
        assert np.array_equal(y, x)
    codec.close()
