"""Per-read sharding of a compression job over the GPUs of one node.

Reads are independent, so a job over N GPUs gives each rank one contiguous
range of reads, balanced by sample count, and compresses it alone.  The only
exchange is the size of every rank's output: an all-gather of one int64 per
rank, from which each rank knows where its records start in the merged
archive.  Concatenating the shards in rank order reproduces the single-GPU
record region byte for byte, because read order is preserved.

* :func:`sample_balanced_ranges` - the partition of SigComp's multi-GPU driver
  (sigcomp/read_assignment.py:14-49, called at sigcomp/multi_gpu.py:309):
  boundary ``i`` of ``parts`` sits at the prefix-sum index closest to
  ``total * i / parts``, ties going to the later index, with every part
  holding at least one read.
* :func:`exchange_shard_bytes` / :func:`shard_offsets` - the byte-count
  exchange and the exclusive scan that lays the shards out.
* :func:`compress_shard` - one rank's share of a sharded compression.
"""

from dataclasses import dataclass
import operator

import numpy as np


@dataclass(frozen=True)
class SampleRange:
    """Reads ``[start, stop)`` holding ``num_samples`` samples."""
    start: int
    stop: int
    num_samples: int


def sample_balanced_ranges(sample_counts, workers):
    """Split reads into at most ``workers`` contiguous ranges of near-equal sample count.

    Same result as sigcomp/read_assignment.py:14-49 for every input, errors
    included: ``workers`` must be positive, counts nonnegative integers whose
    total fits in uint64; an empty input gives ``()``.
    """
    workers = operator.index(workers)
    if workers < 1:
        raise ValueError('workers must be positive')
    counts = []
    total = 0
    for v in sample_counts:                             # validate in input order
        v = operator.index(v)
        if v < 0:
            raise ValueError('Sample counts must be nonnegative integers')
        total += v
        if total > 0xFFFFFFFFFFFFFFFF:
            raise ValueError('Total sample count exceeds uint64 capacity')
        counts.append(v)
    n = len(counts)
    if n == 0:
        return ()
    # exact prefix sums: numpy for the common case, Python integers near the uint64 limit
    if total < 2 ** 62:
        prefix = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(np.asarray(counts, dtype=np.int64), out=prefix[1:])
    else:
        prefix = np.zeros(n + 1, dtype=object)
        np.cumsum(np.asarray(counts, dtype=object), out=prefix[1:])
    parts = min(n, workers)
    bounds = [0]
    for i in range(1, parts):
        lo, hi = bounds[-1] + 1, n - (parts - i)       # every part keeps at least one read
        if total == 0:
            q, r = divmod(n, parts)
            b = i * q + min(i, r)
        else:
            goal = total * i                            # compare prefix * parts against goal exactly
            target = -(-goal // parts)                  # ceil(goal / parts)
            right = lo + int(np.searchsorted(prefix[lo:hi + 1], target, side='left'))
            right = min(right, hi)
            left = max(lo, right - 1)
            d_right = abs(int(prefix[right]) * parts - goal)
            d_left = abs(int(prefix[left]) * parts - goal)
            b = left if d_left < d_right else right     # ties: the later boundary
        bounds.append(b)
    bounds.append(n)
    return tuple(SampleRange(a, b, int(prefix[b]) - int(prefix[a])) for a, b in zip(bounds, bounds[1:]))


def shard_offsets(byte_counts, base=0):
    """Start offset of every shard in the merged record region, and its end."""
    starts = []
    pos = int(base)
    for b in byte_counts:
        starts.append(pos)
        pos += int(b)
    return starts, pos


def exchange_shard_bytes(local_bytes, group=None, device=None):
    """All-gather one int64 per rank (the only collective of a sharded job).

    Works on any torch.distributed backend: NCCL with ``device`` a CUDA device,
    gloo on the CPU.  Without an initialised process group it returns
    ``[local_bytes]``.
    """
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [int(local_bytes)]
    world = dist.get_world_size(group)
    if device is None:
        device = torch.device('cuda', torch.cuda.current_device()) \
            if dist.get_backend(group) == 'nccl' else torch.device('cpu')
    mine = torch.tensor([int(local_bytes)], dtype=torch.int64, device=device)
    every = torch.empty(world, dtype=torch.int64, device=device)
    dist.all_gather_into_tensor(every, mine, group=group)
    return [int(v) for v in every.cpu().tolist()]


@dataclass
class Shard:
    """One rank's part of a sharded compression."""
    reads: SampleRange
    records: list          # compressed record bytes of reads [reads.start, reads.stop)
    byte_offset: int       # where this shard's first record starts in the merged region
    total_bytes: int       # size of the merged region over all ranks
    rank_bytes: list       # every rank's shard size, in rank order


def compress_shard(codec, reads, *, rank=0, world=1, sample_counts=None, group=None, device=None,
                   batch_size=64):
    """Compress this rank's contiguous, sample-balanced share of ``reads``.

    ``reads`` is every read of the job (a list of uint8 token arrays, the
    ``list_of_reads`` of ``batch_inference_reads``); each rank must pass the
    same list.  ``sample_counts`` (default: token counts) are the raw signal
    lengths the partition balances, as SigComp balances POD5 sample counts.
    Ranks beyond the number of reads get an empty range.  All ranks take part
    in the byte-count exchange.
    """
    if sample_counts is None:
        sample_counts = [len(r) for r in reads]
    plans = sample_balanced_ranges(sample_counts, world)
    plan = plans[rank] if rank < len(plans) else SampleRange(len(reads), len(reads), 0)
    mine = list(reads[plan.start:plan.stop])
    records = codec.batch_inference_reads(list_of_reads=mine, batch_size=batch_size) if mine else []
    local = sum(len(r) for r in records)
    sizes = exchange_shard_bytes(local, group=group, device=device) if world > 1 else [local]
    starts, total = shard_offsets(sizes)
    return Shard(plan, records, starts[rank], total, sizes)
