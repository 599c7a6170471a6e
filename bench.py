#!/usr/bin/env python
"""Benchmark of the SigComp neural codec hot path on B200.

Metric: compress & decompress Msamples/s at 1/2/4/8 B200, with
bits/sample, bit-exact.  A step is one compress + decompress round trip of a
rank's share of a job of synthetic int16 reads with the bundled model and
chunk_len 2048, the SigComp per-read path on the device, one sub-batch of reads
at a time (SigComp too codes a shard in batches):

  compress    split every read (sc_split_signal_device: delta / zig-zag / split of
              main.py:504-521) -> chunk the token streams -> sc_compress_chunks_device
  decompress  sc_decompress_chunks_device -> sc_reassemble_signal_device -> int16 reads

The job is sharded as SigComp's multi-GPU driver shards it: contiguous read ranges
balanced by sample count (sharding.sample_balanced_ranges, read_assignment.py:14-49),
every rank coding its range alone; the only collective is the all-gather of every
rank's stream byte count that lays out the archive (sharding.exchange_shard_bytes).
Configuration 2 (the default) is weak scaling: the job holds 20,000 reads per GPU.
Configuration 5 is strong scaling: one 200,000-read job (~11 G samples) over N GPUs.

  value      whole-job round-trip Msamples/s with the reads resident in HBM
  e2e        the same with every step's reads copied in from pinned host memory,
             the compressed record streams (words, large values, positions, offsets)
             copied out and back in, and the decoded reads copied out
  roofline   the dominant kernel (the persistent autoregressive decoder, all nine
             tcgen05 int8 layers + frequency search + range decoding in one launch)
             against the int8 tensor throughput measured in the same run with
             torch._int_mm; roofline_compress does the same for the fused compress
             kernel
  cpu_baseline  the CPU port of the reference codec (numpy split + int_mm GEMMs + C
             coder, oracle/) on a bounded sample, rank 0 at N=1

`--impl reference` times that CPU port alone on the host cores.  `--workload` picks
another BASELINE configuration (config1: the 64-read CPU case, config3: RNA004-like
reads, config4: the lossy mode with lsb_eliminate 3, config5: the 200,000-read
strong-scaling job); configuration 2 is the default.
"""

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "compress & decompress Msamples/s at 1/2/4/8 B200; bits/sample (bit-exact)"
UNIT = "Msamples/s"
CHUNK_LEN = 2048
L2_BYTES = 126 * 1024 * 1024           # B200 L2
# int8 MLP work per coded token: 2 x (8192*512 + 7*512*512 + 512*256) multiply-adds
OPS_PER_TOKEN = 2 * (8192 * 512 + 7 * 512 * 512 + 512 * 256)
# BASELINE.json configurations: (generator, reads, model, lossy lsb, description, scaling).  `reads`
# is per GPU for weak scaling and the whole job for strong scaling.  Configuration 2 is the headline;
# 1 is the CPU-runnable case, 3 the RNA004-like set (no RNA004 model is bundled: the lossless
# R10.4.1 model codes it), 4 the lossy mode on configuration 2's reads, 5 the multi-GPU job.
WORKLOADS = {
    "config1": ("r10_config1", 64, "lossless", 0,
                "r10_config1 (64 reads x 20,000 samples, levels N(500,60), dwell 12, noise 12), lossless model",
                "weak"),
    "config2": ("r10_lognormal", 20000, "lossless", 0,
                "r10_lognormal (configuration 2 generator: lognormal lengths median 30,000, levels N(500,60), "
                "dwell 12, noise 12), lossless model", "weak"),
    "config3": ("rna_lognormal", 10000, "lossless", 0,
                "rna_lognormal (configuration 3 generator: lognormal lengths median 15,000, levels N(800,90), "
                "dwell 30, noise 20), lossless R10.4.1 model (no RNA004 model is bundled)", "weak"),
    "config4": ("r10_lognormal", 20000, "lossy", 3,
                "r10_lognormal (configuration 2 reads), lossy model, lsb_eliminate 3", "weak"),
    "config5": ("r10_lognormal_large", 200000, "lossless", 0,
                "r10_lognormal_large (configuration 5: 200,000 reads, lognormal lengths median 40,000, "
                "levels N(500,60), dwell 12, noise 12), lossless model, one job sharded by read", "strong"),
}
JOB_SEED = 1000             # seed of every job's read lengths and, with the read index, of its samples
SUB_SAMPLES = 1_500_000_000  # samples per sub-batch of a rank's reads (bounds the device buffers)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config2",
                    help="BASELINE configuration (config2, the headline, by default)")
    ap.add_argument("--reads", type=int, default=None,
                    help="reads per GPU (weak scaling) or of the whole job (strong scaling); default: the "
                         "configuration's")
    ap.add_argument("--scaling", choices=["weak", "strong"], default=None,
                    help="override the configuration's scaling mode")
    ap.add_argument("--sub-samples", type=int, default=SUB_SAMPLES,
                    help="samples per sub-batch of a rank's reads")
    ap.add_argument("--gen-workers", type=int, default=None,
                    help="host processes generating the synthetic reads (default: the host's cores / ranks)")
    ap.add_argument("--cpu-reads", type=int, default=32,
                    help="reads in the CPU baseline sample (about 1.6 M samples: 10-20 s of CPU work per "
                         "warm-up + round trip)")
    ap.add_argument("--parity-reads", type=int, default=200,
                    help="reads whose GPU streams the CPU-baseline leg compares with the oracle's (compress "
                         "only, int_mm MLP: a few seconds of CPU work per 100 reads)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--mlp-path", default="auto",
                    choices=["auto", "tcgen05", "tcgen05_small"],
                    help="decoder to run: auto (the library's choice), tcgen05 (the pair kernel for every "
                         "batch), tcgen05_small (the small-batch clusters for every batch)")
    ap.add_argument("--no-plugin", action="store_true",
                    help="skip e2e_plugin (the read-level codec interface with host bytes in and out)")
    ap.add_argument("--chunk-len", type=int, default=CHUNK_LEN,
                    help="tokens per chunk (2048 in every configuration; smaller values give short "
                         "decoder launches for profiling)")
    args = ap.parse_args()
    gen, count, model, lsb, desc, scaling = WORKLOADS[args.workload]
    args.generator, args.model, args.lsb, args.workload_desc = gen, model, lsb, desc
    args.scaling = args.scaling or scaling
    if args.reads is None:
        args.reads = count
    return args


def lossy_round_trip(x, lsb):
    """What SigComp's lossy mode returns for int16 samples x: _lossy_decode(_lossy_encode(
    _reduce_lsb(x, lsb), lsb), lsb) (main.py:158-171, 1162-1164).  _reduce_lsb rounds x to a
    multiple of 2**lsb in int32 and wraps it to int16; the shift down and back up then returns
    that value unchanged."""
    if lsb == 0:
        return x
    v = np.asarray(x).astype(np.int32)
    step = 1 << lsb
    return ((v & ~(step - 1)) + ((v >> (lsb - 1)) & 1) * step).astype(np.int16)


def job_plan(generator, reads, scaling, world):
    """The job's read lengths and every rank's read range: the job holds `reads` reads per rank
    (weak) or `reads` in all (strong), cut by sample count as SigComp's multi-GPU driver cuts it."""
    from sigcomp_b200 import sharding, synthetic
    n_job = reads * world if scaling == "weak" else reads
    lengths = synthetic.job_lengths(generator, JOB_SEED, n_job)
    plans = sharding.sample_balanced_ranges(lengths, world)
    plans = list(plans) + [sharding.SampleRange(n_job, n_job, 0)] * (world - len(plans))
    return lengths, plans


def _gen_part(args):
    generator, lengths, start, stop = args
    from sigcomp_b200 import synthetic
    return synthetic.job_reads(generator, JOB_SEED, lengths, start, stop)


def generate_reads(generator, lengths, start, stop, workers):
    """Reads [start, stop) of the job, generated by `workers` host processes (spawned: this runs
    before the first CUDA call of the process, and forked children of a CUDA process can hang)."""
    if workers <= 1 or stop - start < 64:
        return _gen_part((generator, lengths, start, stop))
    import concurrent.futures
    import multiprocessing
    step = max(16, (stop - start) // (4 * workers))
    parts = [(generator, lengths, a, min(stop, a + step)) for a in range(start, stop, step)]
    with concurrent.futures.ProcessPoolExecutor(workers, mp_context=multiprocessing.get_context("spawn")) as ex:
        out = []
        for r in ex.map(_gen_part, parts):
            out += r
    return out


def sub_batches(lengths, limit):
    """Contiguous read ranges [a, b) of a rank's reads holding at most `limit` samples each (at
    least one read each)."""
    out, a, acc = [], 0, 0
    for i, n in enumerate(lengths):
        if i > a and acc + int(n) > limit:
            out.append((a, i))
            a, acc = i, 0
        acc += int(n)
    if len(lengths):
        out.append((a, len(lengths)))
    return out


def chunk_offsets(tok_off, chunk_len):
    """Chunk boundaries of per-read token streams (SigComp cuts each read's tokens
    into chunk_len pieces, cpu_compression.py:28-50): int64 offsets into the tokens."""
    ntok = np.diff(tok_off)
    nch = (ntok + chunk_len - 1) // chunk_len
    first = np.repeat(tok_off[:-1], nch)
    within = np.arange(int(nch.sum()), dtype=np.int64) - np.repeat(np.cumsum(nch) - nch, nch)
    starts = first + within * chunk_len
    return np.append(starts, tok_off[-1]).astype(np.int64)


def smi_gpu_id(local, env=None, props=None):
    """The nvidia-smi --id of CUDA device `local`.  CUDA ordinals and nvidia-smi indices can
    differ (CUDA_VISIBLE_DEVICES, device order), so the GPU is named by its PCI address
    (domain:bus:device.function, as nvidia-smi prints it); without device properties, a
    CUDA_VISIBLE_DEVICES list (indices or UUIDs, both accepted by --id) maps the ordinal."""
    if props is None:
        try:
            import torch
            if torch.cuda.is_available():
                props = torch.cuda.get_device_properties(local)
        except Exception:
            props = None
    if props is not None:
        return f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
    env = os.environ if env is None else env
    vis = [v.strip() for v in env.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    return vis[local] if local < len(vis) else str(local)


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={smi_gpu_id(self.index)}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        busy = [x for x in sm if x > 0.5 * mx] or sm
        return {"sm_mhz": float(np.median(busy)), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def int8_peak_tops():
    """Achievable dense int8 throughput on this GPU: torch._int_mm 8192^3, best of 10."""
    import torch
    a = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    b = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device="cuda")
    for _ in range(3):
        torch._int_mm(a, b.t())
    best = 1e9
    for _ in range(10):
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        s.record()
        torch._int_mm(a, b.t())
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    return 2 * 8192 ** 3 / (best * 1e-3) / 1e12


def cpu_round_trip(reads, chunk_len, steps=1, warmup=1, lsb=0, model="lossless"):
    """The reference path ported to the CPU: numpy split / reassembly (sigcomp_b200.signal,
    pinned to the reference's outputs) around the oracle codec (int_mm GEMMs + C coder)."""
    import torch
    from oracle import signal
    from oracle.oracle import OracleModel
    from sigcomp_b200.model import load_model
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    om = OracleModel(load_model(name=model))
    samples = int(sum(len(r) for r in reads))
    want = [lossy_round_trip(r, lsb) for r in reads]
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        splits = [signal.split_signal(signal.lossy_encode(signal.reduce_lsb(r, lsb), lsb) if lsb else r)
                  for r in reads]
        chunks = [sp[1][j:j + chunk_len] for sp in splits for j in range(0, len(sp[1]), chunk_len)]
        streams = om.compress_chunks(chunks, chunk_len=chunk_len, backend="int_mm")
        t1 = time.perf_counter()
        back = om.decompress_chunks(streams, [len(c) for c in chunks], chunk_len=chunk_len, backend="int_mm")
        pos, out = 0, []
        for r, sp in zip(reads, splits):
            k = (len(sp[1]) + chunk_len - 1) // chunk_len
            tok = np.concatenate(back[pos:pos + k]) if k else np.zeros(0, np.uint8)
            pos += k
            sig = signal.reassemble_signal(sp[0], len(r), tok, sp[2], sp[3])
            out.append(signal.lossy_decode(sig, lsb) if lsb else sig)
        t2 = time.perf_counter()
        if i >= warmup:
            times.append((t1 - t0, t2 - t1))
        assert all(np.array_equal(a, b) for a, b in zip(out, want))
    tc = sum(t[0] for t in times) / len(times)
    td = sum(t[1] for t in times) / len(times)
    return {"value": samples / (tc + td) / 1e6, "compress": samples / tc / 1e6, "decompress": samples / td / 1e6,
            "cores": cores, "seconds_per_step": tc + td, "samples": samples}


def parity_vs_oracle(pl, reads, n_reads, chunk_len, lsb, model):
    """Compare the GPU streams of the first `n_reads` reads of the rank's first sub-batch
    (compressed again after the timed region) with the oracle's streams for the same reads: the oracle's split
    (main.py:504-521) and its compress_chunks with the int_mm MLP (cpu_compression.py:178-257),
    both pinned to the reference's outputs by the golden tests."""
    from oracle import signal
    from oracle.oracle import OracleModel
    from sigcomp_b200.model import load_model
    n = min(n_reads, len(reads), pl.subs[0][1] - pl.subs[0][0])
    pl.compress(0)                       # the first sub-batch holds the first reads
    tok_off = pl.tok_off[:n + 1].cpu().numpy()
    ntok = np.diff(tok_off)
    k = int(((ntok + chunk_len - 1) // chunk_len).sum())
    woff = pl.woff[:k + 1].cpu().numpy()
    words = pl.words[:int(woff[k])].cpu().numpy().view(np.uint32)
    gpu = [words[woff[i]:woff[i + 1]].astype("<u4").tobytes() for i in range(k)]
    splits = signal.reads_to_tokens(reads[:n], lsb)
    chunks = [sp[1][j:j + chunk_len] for sp in splits for j in range(0, len(sp[1]), chunk_len)]
    t0 = time.perf_counter()
    ref = OracleModel(load_model(name=model)).compress_chunks(chunks, chunk_len=chunk_len, backend="int_mm")
    dt = time.perf_counter() - t0
    mismatch = next((i for i, (a, b) in enumerate(zip(gpu, ref)) if a != b), None)
    equal = len(chunks) == k and mismatch is None
    return {"reads": n, "chunks": k, "tokens": int(ntok.sum()), "equal": bool(equal),
            "first_mismatch": mismatch, "oracle_seconds": round(dt, 2),
            "what": "GPU chunk streams of the timed batch's first reads vs the CPU oracle's (oracle/: C coder "
                    "+ int_mm MLP, pinned to the reference's golden streams); decoded reads are checked "
                    "separately against the input (bit_exact_round_trip)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    n_reads = args.cpu_reads
    lengths, _ = job_plan(args.generator, n_reads, "strong", 1)
    reads = generate_reads(args.generator, lengths, 0, n_reads, 1)
    r = cpu_round_trip(reads, args.chunk_len, steps=args.steps, warmup=args.warmup, lsb=args.lsb, model=args.model)
    sample = f"the first {n_reads} reads ({r['samples']} samples) of the {args.workload} job per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["value"], 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["seconds_per_step"] * 1e3, 1), "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"{args.workload_desc}, chunk_len {args.chunk_len}", "reads_per_step": n_reads,
                   "samples_per_step": r["samples"]},
        "compress_msps": round(r["compress"], 4), "decompress_msps": round(r["decompress"], 4),
        "cpu_baseline": {"value": round(r["value"], 4), "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(r["value"], 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


class Pipeline:
    """Device buffers and the C-ABI calls of one rank's round trips.  The rank's reads (x) and
    the decoded reads (y) stay resident; the split, token, stream and offset buffers are sized
    for the largest sub-batch and reused by every sub-batch."""

    def __init__(self, codec, read_lengths, subs, chunk_len, lsb=0):
        import ctypes
        import torch
        self.torch, self.vp = torch, ctypes.c_void_p
        self.L, self.h = codec._lib, codec.handle
        self.chunk_len, self.lsb = chunk_len, lsb
        dev = torch.device("cuda", torch.cuda.current_device())
        lengths = np.asarray(read_lengths, dtype=np.int64)
        self.soff_h = np.zeros(len(lengths) + 1, np.int64)
        np.cumsum(lengths, out=self.soff_h[1:])
        self.S = int(self.soff_h[-1])
        self.subs = subs
        # every sub-batch's sample offsets relative to its first sample, back to back
        rel, self.rel_at = [], []
        for a, b in subs:
            self.rel_at.append(sum(len(r) for r in rel))
            rel.append(self.soff_h[a:b + 1] - self.soff_h[a])
        self.soff_rel_h = np.concatenate(rel) if rel else np.zeros(1, np.int64)
        max_reads = max((b - a for a, b in subs), default=1)
        max_samples = max((int(self.soff_h[b] - self.soff_h[a]) for a, b in subs), default=1)
        cap = max(max_samples - 1, 1)

        def e(n, dt):
            return torch.empty(max(int(n), 1), dtype=dt, device=dev)

        self.x, self.y = e(self.S, torch.int16), e(self.S, torch.int16)
        self.soff_rel = e(len(self.soff_rel_h), torch.int64)
        self.soff_rel.copy_(torch.from_numpy(self.soff_rel_h))
        self.sig0 = e(max_reads, torch.int16)
        self.tok, self.tok2 = e(cap, torch.uint8), e(cap, torch.uint8)
        self.tok_off, self.large_off = e(max_reads + 1, torch.int64), e(max_reads + 1, torch.int64)
        self.large, self.pos = e(cap, torch.int16), e(cap, torch.int32)
        max_chunks = cap // chunk_len + max_reads + 1        # every read adds at most one partial chunk
        self.word_cap = cap + 2 * max_chunks + 1
        self.words = e(self.word_cap, torch.int32)
        self.choff = e(max_chunks + 1, torch.int64)
        self.chlen = e(max_chunks, torch.int64)
        self.woff = e(max_chunks + 1, torch.int64)
        self.stream = torch.cuda.current_stream()
        self.n_chunks = 0
        self.chlen_h = np.zeros(0, np.int64)
        self.cur = None

    def p(self, t, elem_offset=0):
        return self.vp(t.data_ptr() + elem_offset * t.element_size())

    def sub(self, i):
        """(reads, first sample, samples, offset of its relative sample offsets) of sub-batch i."""
        a, b = self.subs[i]
        return b - a, int(self.soff_h[a]), int(self.soff_h[b] - self.soff_h[a]), self.rel_at[i]

    def compress(self, i):
        from sigcomp_b200 import _lib
        L, h, p, sp = self.L, self.h, self.p, self.vp(self.stream.cuda_stream)
        R, s0, _, ro = self.sub(i)
        self.cur = i
        _lib.check(L.sc_split_signal_device(h, p(self.x, s0), p(self.soff_rel, ro), R, self.lsb, p(self.sig0),
                                            p(self.tok), p(self.tok_off), p(self.large), p(self.pos),
                                            p(self.large_off), sp))
        # chunk boundaries of the per-read token streams (host, from the R + 1 token offsets)
        choff = chunk_offsets(self.tok_off[:R + 1].cpu().numpy(), self.chunk_len)
        n = len(choff) - 1
        self.n_chunks = n
        self.chlen_h = np.ascontiguousarray(np.diff(choff), dtype=np.int64)
        self.choff[:n + 1].copy_(self.torch.from_numpy(choff))
        self.chlen[:n].copy_(self.torch.from_numpy(self.chlen_h))
        _lib.check(L.sc_compress_chunks_device(h, p(self.tok), p(self.choff), n, p(self.words), self.word_cap,
                                               p(self.woff), None, sp))

    def decompress(self, i):
        from sigcomp_b200 import _lib
        L, h, p, sp = self.L, self.h, self.p, self.vp(self.stream.cuda_stream)
        R, s0, _, ro = self.sub(i)
        _lib.check(L.sc_decompress_chunks_device(h, p(self.words), p(self.woff), p(self.chlen),
                                                 self.vp(self.chlen_h.ctypes.data), self.n_chunks, p(self.tok2),
                                                 None, sp))
        _lib.check(L.sc_reassemble_signal_device(h, p(self.sig0), p(self.soff_rel, ro), R, self.lsb, p(self.tok2),
                                                 p(self.tok_off), p(self.large), p(self.pos), p(self.large_off),
                                                 p(self.y, s0), sp))

    def counts(self):
        """(tokens, large deltas, chunks, words) of the sub-batch last compressed."""
        R = self.sub(self.cur)[0]
        return (int(self.tok_off[R].item()), int(self.large_off[R].item()), self.n_chunks,
                int(self.woff[self.n_chunks].item()))


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    # this rank's reads, generated before the first CUDA call (by spawned helper processes)
    lengths, plans = job_plan(args.generator, args.reads, args.scaling, world)
    plan = plans[rank]
    workers = args.gen_workers or max(1, min(16, (os.cpu_count() or 1) // max(world, 1)))
    reads = generate_reads(args.generator, lengths, plan.start, plan.stop, workers)
    samples_np = np.concatenate(reads) if reads else np.zeros(0, np.int16)
    n_reads, n_samples = len(reads), len(samples_np)
    subs = sub_batches(lengths[plan.start:plan.stop], args.sub_samples)

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from sigcomp_b200 import _lib, sharding
    from sigcomp_b200.codec import B200Compression
    from sigcomp_b200.model import load_model

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    codec = B200Compression(chunk_len=args.chunk_len, gpu=local, model=load_model(name=args.model))
    if args.mlp_path != "auto":
        codec.set_mlp_path(args.mlp_path)
    pl = Pipeline(codec, lengths[plan.start:plan.stop], subs, args.chunk_len, args.lsb)
    pl.x[:n_samples].copy_(torch.from_numpy(samples_np))
    # what the round trip must return: the reads themselves, or SigComp's lossy output
    want = pl.x if args.lsb == 0 else torch.from_numpy(lossy_round_trip(samples_np, args.lsb)).cuda()
    state = {"bytes": 0, "tokens": 0, "large": 0, "chunks": 0}

    def exchange():
        # archive layout: every rank learns every shard's stream size (one int64 per rank)
        return sharding.exchange_shard_bytes(state["bytes"], device=torch.device("cuda", local)) \
            if world > 1 else [state["bytes"]]

    def step(timers=None):
        state.update(bytes=0, tokens=0, large=0, chunks=0)
        for i in range(len(subs)):
            if timers:
                timers[0].append(torch.cuda.Event(enable_timing=True))
                timers[0][-1].record()
            pl.compress(i)
            tok, large, chunks, words = pl.counts()
            # bits: framed neural streams (2-byte frame per chunk + words)
            state["bytes"] += 4 * words + 2 * chunks
            state["tokens"] += tok
            state["large"] += large
            state["chunks"] += chunks
            if timers:
                timers[1].append(torch.cuda.Event(enable_timing=True))
                timers[1][-1].record()
            pl.decompress(i)
            if timers:
                timers[2].append(torch.cuda.Event(enable_timing=True))
                timers[2][-1].record()
        return exchange()

    def sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ok = bool(torch.equal(pl.y[:n_samples], want[:n_samples]))
    n_tok, n_large, n_chunks, stream_bytes = state["tokens"], state["large"], state["chunks"], state["bytes"]

    # timed region (device-resident), with per-phase events and per-kernel profiling
    _lib.profile_enable(codec.handle, True)
    launches0 = _lib.kernel_launches()
    clocks = ClockSampler(local)
    clocks.start()
    sync()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    timers = ([], [], [])
    shard_bytes = None
    for _ in range(args.steps):
        shard_bytes = step(timers)
    ev[1].record()
    sync()
    clk = clocks.stop()
    elapsed_ms = ev[0].elapsed_time(ev[1])
    t_comp = sum(a.elapsed_time(b) for a, b in zip(timers[0], timers[1]))
    t_dec = sum(b.elapsed_time(c) for b, c in zip(timers[1], timers[2]))
    launches = _lib.kernel_launches() - launches0
    prof = _lib.profile_read(codec.handle)
    _lib.profile_enable(codec.handle, False)
    ok = ok and bool(torch.equal(pl.y[:n_samples], want[:n_samples]))

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    elapsed_max = max_over_ranks(elapsed_ms)
    elapsed_min = -max_over_ranks(-elapsed_ms)
    t_comp_max = max_over_ranks(t_comp)
    t_dec_max = max_over_ranks(t_dec)
    total_samples = sum_over_ranks(n_samples)
    total_stream = sum_over_ranks(stream_bytes)
    total_tokens = sum_over_ranks(n_tok)
    total_large = sum_over_ranks(n_large)
    all_ok = sum_over_ranks(0.0 if ok else 1.0) == 0
    layout_ok = shard_bytes is not None and int(sum(shard_bytes)) == int(total_stream)

    # ---- e2e: reads from pinned host memory, record streams out and back, reads out ------
    e2e = None
    if not args.no_e2e:
        def pinned(n, dt):
            return torch.empty(max(int(n), 1), dtype=dt).pin_memory()

        # host buffers: the rank's reads in and out, and one sub-batch's record streams
        h_x = torch.from_numpy(samples_np).pin_memory() if n_samples else pinned(1, torch.int16)
        h_soff = torch.from_numpy(pl.soff_rel_h).pin_memory()
        h_y = pinned(n_samples, torch.int16)
        cap = pl.word_cap
        h_words, h_woff = pinned(cap, torch.int32), pinned(pl.woff.numel(), torch.int64)
        h_large, h_pos = pinned(pl.large.numel(), torch.int16), pinned(pl.pos.numel(), torch.int32)
        h_sig0 = pinned(pl.sig0.numel(), torch.int16)
        h_tokoff, h_loff = pinned(pl.tok_off.numel(), torch.int64), pinned(pl.large_off.numel(), torch.int64)
        moved = {"h2d": 0, "d2h": 0}

        def copy(dst, src, n, kind, dst_at=0, src_at=0):
            dst[dst_at:dst_at + n].copy_(src[src_at:src_at + n], non_blocking=True)
            moved[kind] += n * src.element_size()

        def host_step():
            copy(pl.soff_rel, h_soff, h_soff.numel(), "h2d")
            for i in range(len(subs)):
                R, s0, ns, _ = pl.sub(i)
                copy(pl.x, h_x, ns, "h2d", s0, s0)
                pl.compress(i)
                _, nl, nc, nw = pl.counts()
                # the record streams of the archive: words + offsets, large values, positions, sig0, offsets
                streams = ((h_words, pl.words, nw), (h_woff, pl.woff, nc + 1), (h_large, pl.large, nl),
                           (h_pos, pl.pos, nl), (h_sig0, pl.sig0, R), (h_tokoff, pl.tok_off, R + 1),
                           (h_loff, pl.large_off, R + 1))
                for hb, db, n in streams:
                    copy(hb, db, n, "d2h")
                torch.cuda.current_stream().synchronize()
                for hb, db, n in streams:
                    copy(db, hb, n, "h2d")
                pl.decompress(i)
                copy(h_y, pl.y, ns, "d2h", s0, s0)
            torch.cuda.current_stream().synchronize()
            exchange()

        host_step()
        sync()
        moved = {"h2d": 0, "d2h": 0}
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            host_step()
        e1.record()
        sync()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
        ok_e2e = bool(np.array_equal(h_y.numpy()[:n_samples], want[:n_samples].cpu().numpy()))
        all_ok = all_ok and sum_over_ranks(0.0 if ok_e2e else 1.0) == 0
        e2e = {"value": round(total_samples * args.steps / (e2e_ms * 1e-3) / 1e6, 3), "unit": UNIT,
               "h2d_bytes_per_step": int(moved["h2d"] // args.steps),
               "d2h_bytes_per_step": int(moved["d2h"] // args.steps),
               "entry_points": "sc_split_signal_device + sc_compress_chunks_device | "
                               "sc_decompress_chunks_device + sc_reassemble_signal_device; every step's reads "
                               "and record streams through pinned host memory"}

    # ---- e2e_plugin: SigComp's own integration route, GPUCompression.batch_inference_reads with
    # host token streams in and framed host bytes out, then the framed bytes back to tokens
    # (cpu_compression.py:28-84; callers main.py:873, 1150), one call per sub-batch as SigComp's
    # flush loops call it per batch.  The token streams come from the split of the same reads
    # (the caller's _split_signal), made before the timed region.
    e2e_plugin = None
    if not args.no_plugin:
        toks = []
        for i in range(len(subs)):
            a_, b_ = subs[i]
            toks.append([sp[1] for sp in codec.split_signals(reads[a_:b_], lsb=args.lsb)])
        samples_sub = [int(pl.soff_h[b_] - pl.soff_h[a_]) for a_, b_ in subs]

        def plugin_step():
            out, nbytes = [], 0
            for t in toks:
                framed = codec.batch_inference_reads(list_of_reads=t, batch_size=20480)
                nbytes += sum(len(f) for f in framed)
                out.append(codec.batch_inference_reads(list_of_compressed_reads=framed,
                                                       list_of_lengths=[len(x) for x in t], batch_size=20480))
            return out, nbytes

        plugin_step()                       # warm-up: the model's buffers grow to this batch
        sync()
        t0 = time.perf_counter()
        p_back, p_bytes = plugin_step()
        torch.cuda.synchronize()
        p_s = max_over_ranks(time.perf_counter() - t0)
        p_ok = all(np.array_equal(x, y) for bt, t in zip(p_back, toks) for x, y in zip(bt, t))
        del p_back
        all_ok = all_ok and sum_over_ranks(0.0 if p_ok else 1.0) == 0
        tok_bytes = sum(sum(len(x) for x in t) for t in toks)
        e2e_plugin = {
            "value": round(total_samples / p_s / 1e6, 3), "unit": UNIT, "steps": 1,
            "seconds_per_step": round(p_s, 3), "frac_of_value": None,
            "host_bytes_in_per_step": int(sum_over_ranks(tok_bytes + p_bytes)),
            "host_bytes_out_per_step": int(sum_over_ranks(p_bytes + tok_bytes)),
            "route": "GPUCompression.batch_inference_reads(list_of_reads=...) then "
                     "(list_of_compressed_reads=..., list_of_lengths=...), host numpy tokens in, framed bytes "
                     "out and back, one call pair per sub-batch; wall clock, max over ranks (host work included)",
        }

    # ---- roofline of the fused kernels ------------------------------------------
    roofline = roofline_c = None
    if rank == 0:
        peak = int8_peak_tops()
        all_ms = sum(v[0] for v in prof.values())
        traffic_file = REPO / "profiles" / "fused_traffic.json"
        traffic_per_token = json.loads(traffic_file.read_text()) if traffic_file.exists() else {}

        def fused_roofline(kind, name):
            ms, n, toks = prof[kind]
            if ms <= 0 or n == 0:
                return None
            achieved = toks * OPS_PER_TOKEN / (ms * 1e-3) / 1e12
            tpt = traffic_per_token.get(kind)
            return {
                "kernel": name, "bound": "tensor", "achieved": round(achieved, 1), "peak": round(peak, 1),
                "unit": "TOP/s (int8)", "frac": round(achieved / peak, 4) if peak else None,
                "traffic": round(tpt * toks / n) if tpt else None,
                "peak_source": "torch._int_mm int8 8192^3 best of 10, measured in this run (MEASURED_PEAKS.json "
                               "has no int8 figure); datasheet dense int8 is 4500 TOP/s",
                "frac_of_datasheet": round(achieved / 4500.0, 4),
                "ops_per_token": OPS_PER_TOKEN, "tokens_per_launch": int(toks / n),
                "ops_per_launch": int(OPS_PER_TOKEN * toks / n), "launches": n,
                "avg_launch_ms": round(ms / n, 3),
                "share_of_gpu_time": round(ms / all_ms, 4) if all_ms else None,
            }

        roofline = fused_roofline("fused_decode", "k_fused2<1>: persistent autoregressive decoder on SM pairs "
                                                  "(9 tcgen05 int8 layers + frequency search + range decode)")
        if roofline is None:
            # a batch of at most SMs / 8 tiles of 128 chunks decodes on the small-batch clusters
            roofline = fused_roofline("small_decode", "k_small_decode: small-batch autoregressive decoder, a "
                                                      "cluster of 8 SMs per 128 chunks (9 tcgen05 int8 layers "
                                                      "split 8 ways + frequency search + range decode)")
        roofline_c = fused_roofline("fused_compress", "k_fused2<0>: fused compress on SM pairs (9 tcgen05 int8 "
                                                      "layers + (cum, freq) selection)")
        # the signal transform on either side of the codec: HBM-bound byte work, 3 algorithmic bytes
        # per sample each way (split: 2 B sample in, 1 B token out; reassembly: the reverse; the
        # large values, about 1 % of deltas, are left out)
        hbm = None
        peaks_file = REPO / "MEASURED_PEAKS.json"
        if peaks_file.exists():
            hbm = json.loads(peaks_file.read_text()).get("hbm_gbs")
        signal = {}
        for kind in ("split", "reassemble"):
            ms, n, samples = prof.get(kind, (0.0, 0, 0))
            if ms > 0 and n:
                gbs = 3 * samples / (ms * 1e-3) / 1e9
                signal[kind] = {"launch_ms": round(ms / n, 3), "samples_per_launch": int(samples / n),
                                "achieved_gbs": round(gbs, 1),
                                "frac_of_hbm": round(gbs / hbm, 4) if hbm else None}
        if roofline is not None:
            roofline["signal_kernels"] = signal or None
            roofline["kernel_ms"] = {k: round(v[0], 2) for k, v in prof.items()}
            roofline["kernel_launches"] = {k: v[1] for k, v in prof.items()}

    cpu = parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if args.parity_reads > 0:
            parity = parity_vs_oracle(pl, reads, args.parity_reads, args.chunk_len, args.lsb, args.model)
        n = min(args.cpu_reads, len(reads))
        r = cpu_round_trip(reads[:n], args.chunk_len, steps=1, warmup=1, lsb=args.lsb, model=args.model)
        cpu = {"value": round(r["value"], 4), "unit": UNIT, "cores": r["cores"], "kind": "port",
               "sample": f"first {n} reads of the same job ({r['samples']} samples), one round trip after one "
                         "warm-up",
               "compress_msps": round(r["compress"], 4), "decompress_msps": round(r["decompress"], 4)}

    if rank == 0:
        value = total_samples * args.steps / (elapsed_max * 1e-3) / 1e6
        job_reads = args.reads * world if args.scaling == "weak" else args.reads
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_max / args.steps, 2), "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{args.workload_desc}, chunk_len {args.chunk_len}",
                       "job_reads": job_reads, "job_samples": int(total_samples),
                       "reads_per_gpu": n_reads, "samples_per_gpu": n_samples, "tokens_per_gpu": n_tok,
                       "chunks_per_gpu": n_chunks, "sub_batches_per_gpu": len(subs),
                       "parallelism": f"reads sharded over {world} GPU(s) by sample count "
                                      "(sharding.sample_balanced_ranges); shard byte counts all-gathered once per "
                                      "step (sharding.exchange_shard_bytes)",
                       "step": "split -> compress -> decompress -> reassemble of every sub-batch, int16 reads in "
                               "and out",
                       "l2": (f"inputs larger than L2 ({2 * n_samples / 1e9:.2f} GB of samples, "
                              f"{n_tok / 1e9:.2f} GB of tokens per GPU); no flush needed"
                              if 2 * n_samples > L2_BYTES else
                              f"inputs ({2 * n_samples / 1e6:.1f} MB of samples per GPU) fit in L2 and are "
                              "not flushed between steps")},
            "compress_msps": round(total_samples * args.steps / (t_comp_max * 1e-3) / 1e6, 3),
            "decompress_msps": round(total_samples * args.steps / (t_dec_max * 1e-3) / 1e6, 3),
            "rank_balance": round(elapsed_min / elapsed_max, 4) if elapsed_max else None,
            "bits_per_sample_neural": round(8 * total_stream / total_samples, 4),
            "bits_per_small_token": round(8 * total_stream / total_tokens, 4),
            "large_delta_fraction": round(total_large / max(total_samples, 1), 5),
            "bit_exact_round_trip": all_ok,
            "archive_layout_consistent": layout_ok,
            "parity_vs_oracle": parity,
            "gpu_launches": int(launches),
            "clocks": clk, "roofline": roofline, "roofline_compress": roofline_c, "cpu_baseline": cpu,
            "e2e": e2e,
            "e2e_plugin": e2e_plugin,
        }
        if e2e_plugin is not None:
            e2e_plugin["frac_of_value"] = round(e2e_plugin["value"] / value, 4)
        print(json.dumps(line), flush=True)
    codec.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if all_ok and (parity is None or parity["equal"]) else 1


if __name__ == "__main__":
    sys.exit(main())
