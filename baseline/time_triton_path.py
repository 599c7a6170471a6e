"""Time SigComp's own GPU path (Triton) on the same kind of input as bench.py, as the GPU bar.

The reference is installed offline into baseline/_ref (git-ignored; it travels with the working
tree):

    python -m pip install --no-index --no-build-isolation --no-deps --find-links /opt/wheelhouse \\
        --target baseline/_ref <SigComp source tree>

This runs the reference's stock `QuantMLPCompression.compress_chunks` / `decompress_chunks`
(sigcomp/quant_mlp_export.py:271-377: nine Triton linear launches plus a coder-step kernel per token
step, driven from Python) on chunks of the configuration-2 generator. The batch is the reference
CLI's default GPU batch, 20,480 chunks (sigcomp/main.py:1855). A warm-up at the same batch size, with
2-token chunks, does Triton's compilation and autotuning first. Every phase prints its time as soon as
it ends. The last phase checks the reference's streams against this library's on the same chunks.

    python baseline/time_triton_path.py [--chunks 20480] [--chunk-len 2048]
"""

import argparse
import sys
import time
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent


def log(msg):
    print(f"[{time.strftime('%H:%M:%S')}] {msg}", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--chunks", type=int, default=20480)
    ap.add_argument("--chunk-len", type=int, default=2048)
    args = ap.parse_args()

    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(HERE / "_ref"))
    # import-only stand-ins for the reference's I/O dependencies, which the codec path never calls
    for mod in ("pod5", "numcodecs", "fast_rice"):
        sys.modules.setdefault(mod, types.ModuleType(mod))
    import torch
    from sigcomp.quant_mlp_export import QuantMLPCompression
    from sigcomp_b200 import signal, synthetic

    L, B = args.chunk_len, args.chunks
    chunks = []
    seed = 0
    while len(chunks) < B:
        for r in synthetic.make_reads("r10_lognormal", seed=seed, count=400):
            tok = signal.split_signal(r)[1]
            chunks += [tok[i:i + L] for i in range(0, len(tok), L)]
        seed += 1
    chunks = chunks[:B]
    n_tok = sum(len(c) for c in chunks)
    log(f"{B} chunks, {n_tok} tokens (configuration-2 generator)")

    ref = QuantMLPCompression(chunk_len=L, gpu=0)
    log("reference model loaded")
    warm = [c[:2] for c in chunks]
    s = ref.compress_chunks(warm, max_batch_size=B)
    ref.decompress_chunks(s, [len(c) for c in warm], max_batch_size=B)
    torch.cuda.synchronize()
    log("warm-up (Triton compile + autotune at this batch) done")

    t0 = time.perf_counter()
    streams = ref.compress_chunks(chunks, max_batch_size=B)
    torch.cuda.synchronize()
    t_c = time.perf_counter() - t0
    log(f"reference compress: {t_c:.3f} s, {n_tok / t_c / 1e6:.3f} Mtokens/s")
    t0 = time.perf_counter()
    back = ref.decompress_chunks(streams, [len(c) for c in chunks], max_batch_size=B)
    torch.cuda.synchronize()
    t_d = time.perf_counter() - t0
    log(f"reference decompress: {t_d:.3f} s, {n_tok / t_d / 1e6:.3f} Mtokens/s")
    ok = all(np.array_equal(a, b) for a, b in zip(back, chunks))
    log(f"reference round trip: {n_tok / (t_c + t_d) / 1e6:.3f} Mtokens/s, exact {ok}")

    from sigcomp_b200.codec import B200Compression
    ours = B200Compression(chunk_len=L, gpu=0)
    mine = ours.compress_chunks(chunks)
    log(f"streams equal to sigcomp_b200's: {mine == streams}")


if __name__ == "__main__":
    main()
