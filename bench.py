#!/usr/bin/env python
"""Benchmark of the SigComp neural codec hot path on B200.

Metric: compress & decompress Msamples/s at 1/2/4/8 B200, with
bits/sample, bit-exact.  A step is one compress + decompress round trip of a
batch of synthetic reads drawn from the configuration-2 generator (R10.4.1-like,
lognormal lengths, median 30,000 samples) with the bundled lossless model and
chunk_len 2048.  Each rank holds its own batch (weak scaling, reads sharded by
rank, no collective on the data path); after each compress the ranks exchange
their stream byte counts (all-gather of one int64), which is how a sharded run
lays out the archive.

  value      whole-job round-trip Msamples/s with tokens resident in HBM
             (device entry points sc_compress_chunks_device / sc_decompress_chunks_device)
  e2e        the same through the host entry points (sc_compress_chunks /
             sc_decompress_chunks) from pinned host memory, copies timed
  roofline   the dominant kernel (the persistent autoregressive decoder, all nine
             tcgen05 int8 layers + frequency search + range decoding in one launch)
             against the int8 tensor throughput measured in the same run with
             torch._int_mm; roofline_compress does the same for the fused compress
             kernel
  cpu_baseline  the CPU port of the reference codec (int_mm + C coder, oracle/)
             on a bounded sample, rank 0 at N=1

`--impl reference` times that CPU port alone on the host cores.
"""

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "compress & decompress Msamples/s at 1/2/4/8 B200; bits/sample (bit-exact)"
UNIT = "Msamples/s"
CHUNK_LEN = 2048
# int8 MLP work per coded token: 2 x (8192*512 + 7*512*512 + 512*256) multiply-adds
OPS_PER_TOKEN = 2 * (8192 * 512 + 7 * 512 * 512 + 512 * 256)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--reads", type=int, default=20000,
                    help="reads per GPU per step (configuration 2 is 20,000 reads)")
    ap.add_argument("--cpu-reads", type=int, default=12, help="reads in the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--chunk-len", type=int, default=CHUNK_LEN,
                    help="tokens per chunk (2048 in every configuration; smaller values give short "
                         "decoder launches for profiling)")
    return ap.parse_args()


def make_batch(rank, n_reads, chunk_len=CHUNK_LEN):
    """Token chunks of one rank's batch: (samples, tokens, offsets, per-read token counts)."""
    from sigcomp_b200 import signal, synthetic
    reads = synthetic.make_reads("r10_lognormal", seed=1000 + rank, count=n_reads)
    samples = int(sum(len(r) for r in reads))
    toks = [signal.split_signal(r)[1] for r in reads]
    lengths = []
    for t in toks:
        lengths += [min(chunk_len, len(t) - i) for i in range(0, len(t), chunk_len)]
    offsets = np.zeros(len(lengths) + 1, dtype=np.int64)
    np.cumsum(lengths, out=offsets[1:])
    tokens = np.concatenate(toks).astype(np.uint8)
    return samples, tokens, offsets, np.asarray([len(t) for t in toks])


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
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
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


def cpu_round_trip(tokens, offsets, samples, steps=1, warmup=1):
    """The reference codec ported to the CPU (oracle/, int_mm GEMMs + C coder)."""
    import torch
    from oracle.oracle import OracleModel
    from sigcomp_b200.model import load_model
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    om = OracleModel(load_model(name="lossless"))
    chunks = [tokens[offsets[i]:offsets[i + 1]] for i in range(len(offsets) - 1)]
    lengths = [len(c) for c in chunks]
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        streams = om.compress_chunks(chunks, chunk_len=CHUNK_LEN, backend="int_mm")
        t1 = time.perf_counter()
        back = om.decompress_chunks(streams, lengths, chunk_len=CHUNK_LEN, backend="int_mm")
        t2 = time.perf_counter()
        if i >= warmup:
            times.append((t1 - t0, t2 - t1))
        assert all(np.array_equal(a, b) for a, b in zip(back, chunks))
    tc = sum(t[0] for t in times) / len(times)
    td = sum(t[1] for t in times) / len(times)
    return {"value": samples / (tc + td) / 1e6, "compress": samples / tc / 1e6, "decompress": samples / td / 1e6,
            "cores": cores, "seconds_per_step": tc + td}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    n_reads = args.cpu_reads
    samples, tokens, offsets, _ = make_batch(0, n_reads)
    r = cpu_round_trip(tokens, offsets, samples, steps=args.steps, warmup=args.warmup)
    sample = (f"{n_reads} reads ({samples} samples, {len(offsets) - 1} chunks) of the configuration-2 "
              "generator per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(r["value"], 4), "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(r["seconds_per_step"] * 1e3, 1), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": "r10_lognormal (configuration 2 generator), lossless model, chunk_len 2048",
                   "reads_per_step": n_reads, "samples_per_step": samples},
        "compress_msps": round(r["compress"], 4), "decompress_msps": round(r["decompress"], 4),
        "cpu_baseline": {"value": round(r["value"], 4), "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(r["value"], 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)

    import ctypes
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from sigcomp_b200 import _lib
    from sigcomp_b200.codec import B200Compression
    from sigcomp_b200.model import load_model

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    samples, tokens, offsets, read_tokens = make_batch(rank, args.reads, args.chunk_len)
    n_chunks = len(offsets) - 1
    n_tok = int(offsets[-1])
    lengths = np.diff(offsets)
    codec = B200Compression(chunk_len=args.chunk_len, gpu=local, model=load_model(name="lossless"))
    L = codec._lib
    h = codec.handle
    vp = ctypes.c_void_p
    stream = torch.cuda.current_stream()
    sp = vp(stream.cuda_stream)

    # device-resident inputs and outputs
    d_tok = torch.from_numpy(tokens).cuda()
    d_off = torch.from_numpy(offsets).cuda()
    d_len = torch.from_numpy(lengths.astype(np.int64)).cuda()
    cap = n_tok + 2 * n_chunks + 1
    d_words = torch.empty(cap, dtype=torch.int32, device="cuda")
    d_woff = torch.empty(n_chunks + 1, dtype=torch.int64, device="cuda")
    d_back = torch.empty(max(n_tok, 1), dtype=torch.uint8, device="cuda")
    lengths_h = np.ascontiguousarray(lengths, dtype=np.int64)
    counts = torch.zeros(world, dtype=torch.int64, device="cuda")

    def step():
        _lib.check(L.sc_compress_chunks_device(h, vp(d_tok.data_ptr()), vp(d_off.data_ptr()), n_chunks,
                                               vp(d_words.data_ptr()), cap, vp(d_woff.data_ptr()), None, sp))
        if world > 1:   # archive layout: every rank learns every shard's stream size
            dist.all_gather_into_tensor(counts, d_woff[-1:].contiguous())
        _lib.check(L.sc_decompress_chunks_device(h, vp(d_words.data_ptr()), vp(d_woff.data_ptr()),
                                                 vp(d_len.data_ptr()), vp(lengths_h.ctypes.data), n_chunks,
                                                 vp(d_back.data_ptr()), None, sp))

    def sync():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ok = bool(torch.equal(d_back[:n_tok], d_tok))
    n_words = int(d_woff[-1].item())
    # bits: framed neural streams (2-byte frame per chunk + words) over the samples
    stream_bytes = 4 * n_words + 2 * n_chunks

    # timed region (device-resident), with per-phase events and per-kernel profiling
    _lib.profile_enable(h, True)
    launches0 = _lib.kernel_launches()
    clocks = ClockSampler(local)
    clocks.start()
    sync()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record()
    t_comp = t_dec = 0.0
    for _ in range(args.steps):
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record()
        _lib.check(L.sc_compress_chunks_device(h, vp(d_tok.data_ptr()), vp(d_off.data_ptr()), n_chunks,
                                               vp(d_words.data_ptr()), cap, vp(d_woff.data_ptr()), None, sp))
        if world > 1:
            dist.all_gather_into_tensor(counts, d_woff[-1:].contiguous())
        b.record()
        _lib.check(L.sc_decompress_chunks_device(h, vp(d_words.data_ptr()), vp(d_woff.data_ptr()),
                                                 vp(d_len.data_ptr()), vp(lengths_h.ctypes.data), n_chunks,
                                                 vp(d_back.data_ptr()), None, sp))
        c.record()
        torch.cuda.synchronize()
        t_comp += a.elapsed_time(b)
        t_dec += b.elapsed_time(c)
    ev[1].record()
    sync()
    clk = clocks.stop()
    elapsed_ms = ev[0].elapsed_time(ev[1])
    launches = _lib.kernel_launches() - launches0
    prof = _lib.profile_read(h)
    _lib.profile_enable(h, False)
    ok = ok and bool(torch.equal(d_back[:n_tok], d_tok))

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
    t_comp_max = max_over_ranks(t_comp)
    t_dec_max = max_over_ranks(t_dec)
    total_samples = sum_over_ranks(samples)
    total_stream = sum_over_ranks(stream_bytes)
    total_tokens = sum_over_ranks(n_tok)
    all_ok = sum_over_ranks(0.0 if ok else 1.0) == 0

    # ---- e2e through the host entry points (pinned host buffers) -------------
    e2e = None
    if not args.no_e2e:
        pin_tok = torch.from_numpy(tokens).pin_memory().numpy()
        pin_off = torch.from_numpy(offsets).pin_memory().numpy()
        pin_words = torch.empty(cap, dtype=torch.int32).pin_memory().numpy().view(np.uint32)
        pin_woff = torch.empty(n_chunks + 1, dtype=torch.int64).pin_memory().numpy()
        pin_len = torch.from_numpy(lengths.astype(np.int64)).pin_memory().numpy()
        pin_back = torch.empty(max(n_tok, 1), dtype=torch.uint8).pin_memory().numpy()

        def host_step():
            _lib.check(L.sc_compress_chunks(h, vp(pin_tok.ctypes.data), vp(pin_off.ctypes.data), n_chunks,
                                            vp(pin_words.ctypes.data), cap, vp(pin_woff.ctypes.data), None, sp))
            if world > 1:
                counts_h = torch.tensor([int(pin_woff[-1])], dtype=torch.int64, device="cuda")
                dist.all_gather_into_tensor(counts, counts_h)
            _lib.check(L.sc_decompress_chunks(h, vp(pin_words.ctypes.data), vp(pin_woff.ctypes.data),
                                              vp(pin_len.ctypes.data), n_chunks, vp(pin_back.ctypes.data), None, sp))

        host_step()
        sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            host_step()
        e1.record()
        sync()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
        ok_e2e = bool(np.array_equal(pin_back[:n_tok], tokens))
        all_ok = all_ok and sum_over_ranks(0.0 if ok_e2e else 1.0) == 0
        nw = int(pin_woff[-1])
        h2d = tokens.nbytes + offsets.nbytes + 4 * nw + pin_woff.nbytes + pin_len.nbytes
        d2h = 4 * nw + pin_woff.nbytes + n_chunks + n_tok + n_chunks
        e2e = {"value": round(total_samples * args.steps / (e2e_ms * 1e-3) / 1e6, 3), "unit": UNIT,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "entry_points": "sc_compress_chunks + sc_decompress_chunks (host buffers, pinned)"}

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
        roofline_c = fused_roofline("fused_compress", "k_fused2<0>: fused compress on SM pairs (9 tcgen05 int8 layers "
                                              "+ (cum, freq) selection)")
        if roofline is not None:
            roofline["kernel_ms"] = {k: round(v[0], 2) for k, v in prof.items()}
            roofline["kernel_launches"] = {k: v[1] for k, v in prof.items()}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        n = min(args.cpu_reads, args.reads)
        cs, ctok, coff, _ = make_batch(rank, n)
        r = cpu_round_trip(ctok, coff, cs, steps=1, warmup=1)
        cpu = {"value": round(r["value"], 4), "unit": UNIT, "cores": r["cores"], "kind": "port",
               "sample": f"first {n} reads of the same batch ({cs} samples), one round trip after one warm-up",
               "compress_msps": round(r["compress"], 4), "decompress_msps": round(r["decompress"], 4)}

    if rank == 0:
        value = total_samples * args.steps / (elapsed_max * 1e-3) / 1e6
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(elapsed_max / args.steps, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": {"workload": "r10_lognormal (configuration 2 generator: lognormal lengths median 30,000, "
                                   "levels N(500,60), dwell 12, noise 12), lossless model, "
                                   f"chunk_len {args.chunk_len}",
                       "reads_per_gpu": args.reads, "samples_per_gpu": samples, "tokens_per_gpu": n_tok,
                       "chunks_per_gpu": n_chunks, "parallelism": f"reads sharded over {world} GPU(s)",
                       "l2": "inputs larger than L2 (tokens per GPU > 126 MB; activations stream through HBM)"},
            "compress_msps": round(total_samples * args.steps / (t_comp_max * 1e-3) / 1e6, 3),
            "decompress_msps": round(total_samples * args.steps / (t_dec_max * 1e-3) / 1e6, 3),
            "bits_per_sample_neural": round(8 * total_stream / total_samples, 4),
            "bits_per_small_token": round(8 * total_stream / total_tokens, 4),
            "bit_exact_round_trip": all_ok,
            "gpu_launches": int(launches),
            "clocks": clk, "roofline": roofline, "roofline_compress": roofline_c, "cpu_baseline": cpu,
            "e2e": e2e,
        }
        print(json.dumps(line), flush=True)
    codec.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0 if all_ok else 1


if __name__ == "__main__":
    sys.exit(main())
