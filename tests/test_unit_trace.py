"""The unit-trace summary (host side of the fused kernels' pipeline instrumentation)."""
import numpy as np

from sigcomp_b200.unit_trace import decode_records, summarise


def rec(t, role, ev, layer, half, slot, step):
    return [t, role | ev << 4 | layer << 8 | half << 12 | slot << 16 | step << 32]


def test_record_fields_round_trip():
    r = np.array([rec(5, 2, 1, 7, 1, 4, 1234)], dtype=np.uint64)
    ev = decode_records(r)
    assert (ev["role"][0], ev["event"][0], ev["layer"][0], ev["half"][0], ev["slot"][0], ev["step"][0]) == \
        (2, 1, 7, 1, 4, 1234)


def test_summary_of_waits_and_work():
    r = np.array([
        rec(0, 1, 0, 0, 0, 0, 0), rec(10_000, 1, 1, 0, 0, 0, 0), rec(50_000, 1, 2, 0, 0, 0, 0),
        rec(50_000, 1, 3, 0, 0, 0, 0),                                  # per-K-block event: ignored
        rec(50_000, 1, 0, 8, 0, 0, 0), rec(52_000, 1, 1, 8, 0, 0, 0), rec(60_000, 1, 2, 8, 0, 0, 0),
        rec(1_000, 0, 0, 3, 1, 2, 0), rec(1_500, 0, 1, 3, 1, 2, 0),    # incomplete unit: ignored
    ], dtype=np.uint64)
    rows, frac, steps, span_us = summarise(r, 9)
    assert [(a, b, n) for a, b, n, *_ in rows] == [("mma", "L0", 1), ("mma", "last", 1)]
    assert rows[0][3] == 10.0 and rows[0][4] == 40.0           # wait / work in us
    assert rows[1][3] == 2.0 and rows[1][4] == 8.0
    assert abs(frac - 48 / 50) < 1e-12                          # 40 + 8 us busy of 50 us (10 .. 60)
    assert steps == 1 and span_us == 60.0


def test_recurring_keys_are_separate_units():
    # compression runs every tile group with step 0: the same key recurs, one unit per begin event
    r = np.array([
        rec(0, 2, 0, 3, 0, 1, 0), rec(1_000, 2, 1, 3, 0, 1, 0), rec(3_000, 2, 2, 3, 0, 1, 0),
        rec(10_000, 2, 0, 3, 0, 1, 0), rec(14_000, 2, 1, 3, 0, 1, 0), rec(15_000, 2, 2, 3, 0, 1, 0),
    ], dtype=np.uint64)
    rows, _, _, _ = summarise(r, 9)
    assert len(rows) == 1
    role, cls, n, wait_us, work_us, _, _ = rows[0]
    assert (role, cls, n) == ("epilogue", "hidden", 2)
    assert wait_us == 2.5 and work_us == 1.5                   # (1 + 4) / 2 and (2 + 1) / 2
