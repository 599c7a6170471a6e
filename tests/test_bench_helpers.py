"""Host logic of bench.py: chunking of per-read token streams and the
configuration table (CPU only)."""

import numpy as np

import bench


def test_chunk_offsets_cut_each_read_into_chunk_len_pieces():
    tok_off = np.array([0, 5000, 5000, 9000, 13097], dtype=np.int64)
    got = bench.chunk_offsets(tok_off, 2048)
    assert got.tolist() == [0, 2048, 4096, 5000, 7048, 9000, 11048, 13096, 13097]


def test_chunk_offsets_match_sigcomp_framing():
    # ReadFramingMixin cuts every read's tokens into chunk_len pieces (cpu_compression.py:28-50)
    rng = np.random.default_rng(4)
    lens = rng.integers(0, 9000, size=50)
    tok_off = np.zeros(51, dtype=np.int64)
    np.cumsum(lens, out=tok_off[1:])
    want = []
    for r in range(50):
        want += list(range(int(tok_off[r]), int(tok_off[r + 1]), 1024))
    want.append(int(tok_off[-1]))
    assert bench.chunk_offsets(tok_off, 1024).tolist() == want


def test_chunk_offsets_empty():
    assert bench.chunk_offsets(np.array([0], dtype=np.int64), 2048).tolist() == [0]


def test_workloads_cover_baseline_configurations():
    assert set(bench.WORKLOADS) == {"config1", "config2", "config3", "config4", "config5"}
    assert bench.WORKLOADS["config2"][:4] == ("r10_lognormal", 20000, "lossless", 0)
    assert bench.WORKLOADS["config2"][5] == "weak"
    assert bench.WORKLOADS["config4"][2:4] == ("lossy", 3)
    assert bench.WORKLOADS["config5"][:2] == ("r10_lognormal_large", 200000)
    assert bench.WORKLOADS["config5"][5] == "strong"


def test_job_plan_shards_one_job_by_sample_count():
    from sigcomp_b200 import sharding
    # weak: the job grows with the ranks, each rank's range balanced by sample count
    lengths, plans = bench.job_plan("r10_lognormal", 1000, "weak", 4)
    assert len(lengths) == 4000 and len(plans) == 4
    assert plans[0].start == 0 and plans[-1].stop == 4000
    assert all(a.stop == b.start for a, b in zip(plans, plans[1:]))
    assert tuple(plans) == sharding.sample_balanced_ranges(lengths, 4)
    share = [p.num_samples / lengths.sum() for p in plans]
    assert max(share) - min(share) < 0.01
    # strong: one job of fixed size over every rank count; a prefix of the configuration-5 lengths
    l1, p1 = bench.job_plan("r10_lognormal_large", 5000, "strong", 1)
    l8, p8 = bench.job_plan("r10_lognormal_large", 5000, "strong", 8)
    assert np.array_equal(l1, l8) and len(p8) == 8 and p1[0].num_samples == sum(p.num_samples for p in p8)


def test_sub_batches_bound_the_samples():
    lengths = np.array([5, 5, 5, 20, 1, 1, 30, 2], np.int64)
    subs = bench.sub_batches(lengths, 12)
    assert subs == [(0, 2), (2, 3), (3, 4), (4, 6), (6, 7), (7, 8)]
    assert bench.sub_batches(lengths, 10 ** 9) == [(0, 8)]
    assert bench.sub_batches(np.zeros(0, np.int64), 10) == []


def test_generated_reads_do_not_depend_on_the_workers():
    lengths, _ = bench.job_plan("r10_lognormal", 80, "strong", 1)
    a = bench.generate_reads("r10_lognormal", lengths, 10, 80, 1)
    b = bench.generate_reads("r10_lognormal", lengths, 10, 80, 2)
    assert len(a) == 70 and all(np.array_equal(x, y) for x, y in zip(a, b))
    assert [len(x) for x in a] == lengths[10:80].tolist()


def test_lossy_round_trip_matches_signal_module():
    from oracle import signal
    x = np.asarray([0, 1, 7, 8, 9, -5, 32767, -32768, 1234], dtype=np.int16)
    assert np.array_equal(bench.lossy_round_trip(x, 0), x)
    y = bench.lossy_round_trip(x, 3)
    assert np.array_equal(y, signal.lossy_decode(signal.lossy_encode(signal.reduce_lsb(x, 3), 3), 3))
    assert np.all(np.abs(y.astype(np.int32) - x.astype(np.int32))[:6] <= 4)
    z = np.random.default_rng(9).integers(-32768, 32768, size=20000).astype(np.int16)
    for lsb in range(1, 9):
        assert np.array_equal(bench.lossy_round_trip(z, lsb),
                              signal.lossy_decode(signal.lossy_encode(signal.reduce_lsb(z, lsb), lsb), lsb))


def test_clock_sampler_names_the_gpu_by_pci_address():
    class Props:
        pci_domain_id, pci_bus_id, pci_device_id = 0, 0x1B, 0
    assert bench.smi_gpu_id(3, {"CUDA_VISIBLE_DEVICES": "5"}, Props()) == "00000000:1B:00.0"


def test_clock_sampler_maps_visible_devices(monkeypatch):
    import torch
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)      # no device properties
    assert bench.smi_gpu_id(0, {}) == "0"
    assert bench.smi_gpu_id(3, {}) == "3"
    assert bench.smi_gpu_id(0, {"CUDA_VISIBLE_DEVICES": "4,5"}) == "4"
    assert bench.smi_gpu_id(1, {"CUDA_VISIBLE_DEVICES": " 4, 5 "}) == "5"
    assert bench.smi_gpu_id(0, {"CUDA_VISIBLE_DEVICES": "GPU-1234abcd"}) == "GPU-1234abcd"
