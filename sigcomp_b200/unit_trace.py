"""Pipeline trace of the fused pair kernels: where the producer, MMA issuer and epilogue wait.

With ``sc_trace_enable`` the fused kernels record, for the first SM pair, three events per role
and unit (begin, dependency satisfied, end: include/sigcomp_b200.h).  This module runs one
compress and one decompress of a configuration-2 batch with tracing on and summarises CTA 0's
records per role and unit class (layer 0, hidden layers, last layer):

- wait: begin -> dependency satisfied (MMA: both accumulator buffers free; producer: the tile's
  previous layer written; epilogue: the unit's accumulator full);
- work: dependency satisfied -> end (MMA: every K block issued; producer: every K block
  loaded; epilogue: the unit requantised / decoded);
- MMA issue-busy: the share of the traced span in which the MMA issuer is inside a unit's work.

Usage (one GPU): ``python -m sigcomp_b200.unit_trace --reads 6000``.  Enough reads must be given
for the first pair to hold several tiles (the decoder's steady state); the trace buffer keeps the
first ``--records`` events of each CTA.
"""

import argparse
import collections
import ctypes

import numpy as np

from .codec import B200Compression
from .model import load_model
from .synthetic import make_reads

# role 3: the compress kernel's layer-0 builders, or the small-batch decoder's coder step (rank 0)
ROLES = {0: "producer", 1: "mma", 2: "epilogue", 3: "build/coder"}


def decode_records(rec):
    t = rec[:, 0].astype(np.int64)
    t -= t.min()
    w = rec[:, 1]
    return {
        "t": t,
        "role": (w & 15).astype(int),
        "event": ((w >> 4) & 15).astype(int),
        "layer": ((w >> 8) & 15).astype(int),
        "half": ((w >> 12) & 15).astype(int),
        "slot": ((w >> 16) & 0xFFFF).astype(int),
        "step": (w >> 32).astype(int),
    }


def summarise(rec, num_layers):
    """Rows (role, class, units, mean wait us, mean work us, total wait ms, total work ms) and the
    MMA issue-busy fraction."""
    ev = decode_records(rec)
    # A key can recur (compression runs every tile group of a slot with step 0, and the records
    # carry no group): in time order, a begin event opens a new occurrence of its key.
    units = collections.defaultdict(list)
    for i in np.argsort(ev["t"], kind="stable"):
        e = ev["event"][i]
        if e > 2:
            continue                  # per-K-block events
        key = (ev["role"][i], ev["step"][i], ev["layer"][i], ev["slot"][i], ev["half"][i])
        if e == 0:
            units[key].append({0: ev["t"][i]})
        elif units[key]:
            units[key][-1][e] = ev["t"][i]
    stats = collections.defaultdict(lambda: [0, 0, 0])
    busy = []
    for (role, _, layer, _, _), e in ((k, o) for k, occ in units.items() for o in occ):
        if not all(k in e for k in (0, 1, 2)):
            continue
        cls = "L0" if layer == 0 else ("last" if layer == num_layers - 1 else "hidden")
        s = stats[(ROLES.get(role, str(role)), cls)]
        s[0] += 1
        s[1] += e[1] - e[0]
        s[2] += e[2] - e[1]
        if role == 1:
            busy.append((e[1], e[2]))
    rows = [(r, c, n, w / n / 1e3, k / n / 1e3, w / 1e6, k / 1e6) for (r, c), (n, w, k) in sorted(stats.items())]
    frac = None
    if busy:
        busy.sort()
        span = busy[-1][1] - busy[0][0]
        frac = sum(b - a for a, b in busy) / span if span > 0 else None
    return rows, frac, int(ev["step"].max()) + 1, float(ev["t"].max()) / 1e3


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reads", type=int, default=6000, help="configuration-2 reads to code")
    ap.add_argument("--config1", action="store_true",
                    help="code configuration 1 instead (64 reads x 20,000 samples): its decode runs on the "
                         "small-batch decoder, one cluster of eight SMs per 128 chunks")
    ap.add_argument("--chunk-len", type=int, default=2048)
    ap.add_argument("--records", type=int, default=400000, help="trace records kept per CTA")
    ap.add_argument("--gpu", type=int, default=0)
    ap.add_argument("--mlp-path", default="auto", help="decoder to trace (see B200Compression.set_mlp_path)")
    ap.add_argument("--dump", default=None, help="also save the raw records (npz: compress, decode)")
    args = ap.parse_args(argv)

    model = load_model(name="lossless")
    reads = (make_reads("r10_config1", seed=5) if args.config1
             else make_reads("r10_lognormal", seed=5, count=args.reads))
    L = args.chunk_len
    codec = B200Compression(chunk_len=L, gpu=args.gpu, model=model)
    if args.mlp_path != "auto":
        codec.set_mlp_path(args.mlp_path)
    chunks = []
    for sp in codec.split_signals(reads):            # _split_signal on the GPU
        tok = sp[1]
        chunks += [tok[i:i + L] for i in range(0, len(tok), L)]
    off = np.zeros(len(chunks) + 1, np.int64)
    off[1:] = np.cumsum([len(c) for c in chunks])
    tokens = np.concatenate(chunks)
    lib = codec._lib
    buf = np.zeros((args.records, 2), np.uint64)

    def traced(run):
        if lib.sc_trace_enable(codec.handle, args.records) != 0:
            raise RuntimeError(lib.sc_last_error().decode())
        out = run()
        n = lib.sc_trace_read(codec.handle, 0, ctypes.c_void_p(buf.ctypes.data), args.records)
        lib.sc_trace_enable(codec.handle, 0)
        if n < 0:
            raise RuntimeError(lib.sc_last_error().decode())
        return out, buf[:n].copy()

    (words, woff), rec_c = traced(lambda: codec.compress_flat(tokens, off))
    _, rec_d = traced(lambda: codec.decompress_flat(words, woff, np.diff(off)))
    if args.dump:
        np.savez_compressed(args.dump, compress=rec_c, decode=rec_d)
    what = "configuration 1, 64 reads" if args.config1 else f"configuration-2 generator, {args.reads} reads"
    print(f"{what}, {len(chunks)} chunks of <= {L} tokens, {int(off[-1])} tokens; CTA 0 of the first SM pair "
          f"(of the first cluster for the small-batch decoder)")
    dec = "decode k_small_decode" if args.config1 else "decode k_fused2<1>"
    for name, rec in (("compress k_fused2<0>", rec_c), (dec, rec_d)):
        rows, frac, steps, span_us = summarise(rec, model.num_layers)
        print(f"\n== {name}: {len(rec)} records over {span_us:.1f} us, steps seen {steps} "
              f"({span_us / max(steps, 1):.1f} us per step)")
        print(f"  {'role':9s} {'units':6s} {'n':>7s} {'wait us':>9s} {'work us':>9s} {'wait ms':>9s} {'work ms':>9s}")
        for r, c, n, w, k, tw, tk in rows:
            print(f"  {r:9s} {c:6s} {n:7d} {w:9.2f} {k:9.2f} {tw:9.2f} {tk:9.2f}")
        if frac is not None:
            print(f"  MMA issue-busy {100 * frac:.1f} % of the traced span")
    codec.close()


if __name__ == "__main__":
    main()
