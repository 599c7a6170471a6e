"""Host restatement of SigComp's signal transform on either side of the neural codec.

Test infrastructure, like the rest of ``oracle/``: the tests, ``smoke()`` and the
CPU-baseline leg of ``bench.py`` use it as the checker of the GPU signal kernels
(``sc_split_signal_device`` / ``sc_reassemble_signal_device``) and to turn int16
reads into token streams on the CPU.  The product package never imports it.
The functions follow ``sigcomp/main.py``:

* ``delta_zigzag_encode``  - ``_diff_encode`` + ``_zigzag_encode`` (main.py:129-155)
* ``reduce_lsb`` / ``lossy_encode`` / ``lossy_decode`` - main.py:158-171
* ``split_signal``         - ``_split_signal`` (main.py:504-521)
* ``reassemble_signal``    - ``_reassemble_signal`` (main.py:524-546) with the
  large values and positions passed decoded (the reference rice-codes them with
  the third-party ``fast_rice`` package, which is outside the codec).
"""

import numpy as np


def delta_zigzag_encode(signal):
    signal = np.asarray(signal, dtype=np.int16)
    delta = np.diff(signal).astype(np.int16)          # wraps like int16 arithmetic
    v = delta.astype(np.int32)
    return ((v << 1) ^ (v >> 31)).astype(np.uint16)


def delta_zigzag_decode(sig0, zz):
    v = np.asarray(zz).astype(np.uint32)
    delta = ((v >> 1) ^ -(v & 1)).astype(np.int16)
    out = np.empty(len(delta) + 1, dtype=np.int16)
    out[0] = sig0
    out[1:] = sig0 + np.cumsum(delta).astype(np.int16)
    return out


def reduce_lsb(signal, bit):
    v = np.asarray(signal).astype(np.int32)
    step = 1 << bit
    rounding = ((v >> (bit - 1)) & 1) * step
    upper = v & (~(step - 1))
    return (upper + rounding).astype(np.int16)


def lossy_encode(signal, bit):
    return (np.asarray(signal).astype(np.int32) >> bit).astype(np.int16)


def lossy_decode(signal, bit):
    return (np.asarray(signal).astype(np.int32) << bit).astype(np.int16)


def split_signal(sig):
    """Return ``(sig0, small_tokens uint8, large_values_minus_256 uint16, large_pos_deltas uint32)``."""
    sig = np.asarray(sig, dtype=np.int16)
    zz = delta_zigzag_encode(sig)
    is_large = zz >= 256
    small = zz[~is_large].astype(np.uint8)
    large_vals = zz[is_large].astype(np.uint16)
    large_pos = np.flatnonzero(is_large).astype(np.uint32)
    if len(large_pos):
        deltas = np.empty_like(large_pos)
        deltas[0] = large_pos[0]
        if len(large_pos) > 1:
            deltas[1:] = np.diff(large_pos) - 1
    else:
        deltas = np.empty(0, dtype=np.uint32)
    return int(sig[0]), small, (large_vals - 256).astype(np.uint16), deltas


def reassemble_signal(sig0, n, small, large_vals_minus_256, large_pos_deltas):
    large_vals = np.asarray(large_vals_minus_256).astype(np.uint16) + 256
    deltas = np.asarray(large_pos_deltas, dtype=np.uint32).copy()
    if len(deltas) > 1:
        deltas[1:] += 1
    pos = np.cumsum(deltas).astype(np.int64) if len(deltas) else np.empty(0, np.int64)
    zz = np.zeros(n - 1, dtype=np.uint16)
    mask = np.ones(n - 1, dtype=bool)
    if len(pos):
        zz[pos] = large_vals
        mask[pos] = False
    zz[mask] = small
    return delta_zigzag_decode(sig0, zz)


def reads_to_tokens(reads, lsb=0):
    """Apply the lossy transform (when ``lsb`` > 0) and split every read."""
    out = []
    for sig in reads:
        if lsb > 0:
            sig = lossy_encode(reduce_lsb(sig, lsb), lsb)
        out.append(split_signal(sig))
    return out
