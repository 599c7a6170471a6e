"""Isolated INT8 layer sweep: the tcgen05 layer kernel alone at the model's layer shapes.

BASELINE configuration 5 includes "an isolated INT8 MLP layer sweep at the bundled model's layer
widths with 4K-1M context rows per launch, for tensor-pipe roofline".  This times one launch of
the layer kernel (``sc_linear_layer_device``: int8 x int8 -> int32 in TMEM, bias + exact
requantisation + ReLU in the epilogue) at each row count M for the three shapes of the model,
(N, K) = (512, 8192) layer 0, (512, 512) the hidden layers and (256, 512) the last layer, with
the library's own CUDA-event timing around the launch, and times ``torch._int_mm`` (cuBLASLt,
int32 output, no epilogue) on the same shapes as the measured ceiling.  The reference's
counterpart is bit_exact_linear_kernel (sigcomp/quant_mlp_export.py:21-76).  The layer's output
is checked against int32 products requantised like the reference on the smallest M.

Usage (one GPU): ``python -m sigcomp_b200.layer_sweep [--rows 4096,16384,65536,262144,1048576]``
"""

import argparse
import ctypes

import numpy as np

from . import _lib
from .codec import B200Compression
from .model import load_model

SHAPES = ((0, "layer 0 (N=512, K=8192)"), (1, "hidden (N=512, K=512)"), (8, "last (N=256, K=512)"))
KINDS = {0: "layer0", 1: "hidden", 8: "last_layer"}


def _requant_ref(acc, model, layer):
    """_requantize (cpu_int_kernels.py:5-14) on int32 products, in int64 numpy."""
    biased = (acc.astype(np.int64) + model.biases[layer].astype(np.int64))
    biased = ((biased + 2 ** 31) % 2 ** 32) - 2 ** 31                      # int32 wrap
    m0, sh = int(model.multipliers[layer]), int(model.shifts[layer])
    y = (biased * m0) >> sh
    lo = 0 if model.relu[layer] else -128
    return np.clip(y, lo, 127).astype(np.int8)


def sweep(rows_list, repeats=5, gpu=0):
    import torch
    model = load_model(name="lossless")
    codec = B200Compression(chunk_len=2048, gpu=gpu, model=model)
    lib, h = codec._lib, codec.handle
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = []
    for layer, name in SHAPES:
        w = torch.from_numpy(np.ascontiguousarray(model.weights[layer])).cuda()
        N, K = w.shape
        for M in rows_list:
            x = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda")
            y = torch.empty((M, N), dtype=torch.int8, device="cuda")
            call = lambda: _lib.check(lib.sc_linear_layer_device(h, layer, ctypes.c_void_p(x.data_ptr()), M,
                                                                 ctypes.c_void_p(y.data_ptr()), st))
            call()
            if M == rows_list[0]:
                acc = torch._int_mm(x, w.t()).cpu().numpy()
                assert np.array_equal(y.cpu().numpy(), _requant_ref(acc, model, layer)), f"layer {layer} M={M}"
            _lib.profile_enable(h, True)
            for _ in range(repeats):
                call()
            ms, n, _ = _lib.profile_read(h)[KINDS[layer]]
            _lib.profile_enable(h, False)
            t_layer = ms / n
            best = 1e9
            for _ in range(repeats + 2):
                a, b = torch.cuda.Event(True), torch.cuda.Event(True)
                a.record()
                torch._int_mm(x, w.t())
                b.record()
                torch.cuda.synchronize()
                best = min(best, a.elapsed_time(b))
            ops = 2.0 * M * N * K
            out.append((name, M, t_layer, ops / (t_layer * 1e-3) / 1e12, best, ops / (best * 1e-3) / 1e12))
            del x, y
        del w
    codec.close()
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--rows", default="4096,16384,65536,262144,1048576")
    ap.add_argument("--repeats", type=int, default=5)
    args = ap.parse_args(argv)
    rows = [int(r) for r in args.rows.split(",")]
    res = sweep(rows, args.repeats)
    print(f"{'shape':28s} {'M':>9s} {'layer ms':>10s} {'layer TOP/s':>12s} {'_int_mm ms':>11s} {'_int_mm TOP/s':>14s}"
          f" {'of 4.5 POPS':>11s}")
    for name, M, tl, al, tm, am in res:
        print(f"{name:28s} {M:9d} {tl:10.4f} {al:12.1f} {tm:11.4f} {am:14.1f} {al / 4500:11.3f}")


if __name__ == "__main__":
    main()
