"""Seeded synthetic nanopore-like reads.

There is no public dataset on the build machines, so every benchmark and
parity case draws its reads from this generator.  A read is a
piecewise-constant level trace (levels ~ N(mu, sigma) ADC units, geometric
dwell times) plus additive Gaussian noise, rounded to int16.  The read-length
distributions follow the benchmark configurations of the SigComp evaluation:

* ``r10_config1``: 64 reads x 20,000 samples, levels N(500, 60), dwell 12,
  noise 12 (the CPU-runnable case).
* ``r10_lognormal``: lognormal lengths (median 30,000, sigma_log 0.8, clipped to
  [2,000, 1,000,000]) with the same level/dwell/noise parameters.
* ``rna_lognormal``: levels N(800, 90), dwell 30, noise 20, lognormal lengths
  (median 15,000, sigma_log 0.9).
* ``r10_lognormal_large``: configuration 5's 200,000 reads, lognormal lengths (median
  40,000, sigma_log 0.8), R10 levels.

``job_lengths`` / ``job_reads`` draw the same distributions for the sharded benchmark jobs,
with one generator per read so that every rank makes only its own reads.
"""

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class ReadModel:
    level_mean: float = 500.0
    level_sd: float = 60.0
    dwell_mean: float = 12.0
    noise_sd: float = 12.0


R10 = ReadModel()
RNA004 = ReadModel(level_mean=800.0, level_sd=90.0, dwell_mean=30.0, noise_sd=20.0)


def synth_read(rng, n, model=R10):
    """One int16 read of ``n`` samples drawn from ``rng``."""
    n = int(n)
    if n <= 0:
        return np.empty(0, dtype=np.int16)
    p = 1.0 / float(model.dwell_mean)
    segments = []
    covered = 0
    while covered < n:
        batch = max(16, int((n - covered) * p * 1.5) + 16)
        dwell = rng.geometric(p, size=batch)
        segments.append(dwell)
        covered += int(dwell.sum())
    dwell = np.concatenate(segments)
    stops = np.cumsum(dwell)
    count = int(np.searchsorted(stops, n, side="left")) + 1
    dwell = dwell[:count]
    levels = rng.normal(model.level_mean, model.level_sd, size=count)
    trace = np.repeat(levels, dwell)[:n]
    trace = trace + rng.normal(0.0, model.noise_sd, size=n)
    return np.clip(np.rint(trace), -32768, 32767).astype(np.int16)


def lognormal_lengths(rng, count, median, sigma_log, lo=2000, hi=1_000_000):
    lengths = rng.lognormal(np.log(median), sigma_log, size=int(count))
    return np.clip(np.rint(lengths), lo, hi).astype(np.int64)


# Read sets of the sharded benchmark jobs: lengths drawn first from one generator (cheap for
# any count), samples of read i from their own generator seeded by (seed, i), so that a rank
# can make exactly its share of a job without the reads before it.
JOB_SETS = {
    "r10_config1": (64, None, R10),
    "r10_lognormal": (20000, (30000, 0.8), R10),
    "r10_lognormal_large": (200000, (40000, 0.8), R10),      # configuration 5: ~8 G samples
    "rna_lognormal": (10000, (15000, 0.9), RNA004),
}


def job_lengths(config, seed, count):
    """Sample counts of the first ``count`` reads of a sharded job (``count`` may exceed the
    configuration's read count: the lengths continue from the same distribution)."""
    base, dist, _ = JOB_SETS[config]
    if dist is None:
        return np.full(int(count), 20000, dtype=np.int64)
    rng = np.random.default_rng(seed)
    return lognormal_lengths(rng, int(count), dist[0], dist[1])


def job_reads(config, seed, lengths, start, stop):
    """Reads ``[start, stop)`` of a sharded job whose read lengths are ``lengths``."""
    model = JOB_SETS[config][2]
    return [synth_read(np.random.default_rng([int(seed), i]), lengths[i], model) for i in range(start, stop)]


def make_reads(config, seed=0, count=None):
    """Return a list of int16 reads for a named configuration.

    ``count`` truncates the read set (the lengths of the first ``count`` reads
    are the same as in the full set, because lengths are drawn first).
    """
    rng = np.random.default_rng(seed)
    if config == "r10_config1":
        total = 64
        lengths = np.full(total, 20000, dtype=np.int64)
        model = R10
    elif config == "r10_lognormal":
        total = 20000
        lengths = lognormal_lengths(rng, total, 30000, 0.8)
        model = R10
    elif config == "r10_lognormal_large":
        total = 200000
        lengths = lognormal_lengths(rng, total, 40000, 0.8)
        model = R10
    elif config == "rna_lognormal":
        total = 10000
        lengths = lognormal_lengths(rng, total, 15000, 0.9)
        model = RNA004
    else:
        raise ValueError(f"unknown synthetic configuration {config!r}")
    if count is not None:
        lengths = lengths[:int(count)]
    return [synth_read(rng, n, model) for n in lengths]
