"""The B200 codec object: a drop-in for SigComp's ``GPUCompression``.

SigComp's ``_load_model`` (sigcomp/main.py:189-225) returns, for
``--device cuda``, a ``GPUCompression(ReadFramingMixin, QuantMLPCompression)``
object.  :class:`B200Compression` has the same constructor arguments,
attributes (``chunk_len``, ``window_size``, ``SOS_token``, ``device``) and
methods:

* ``batch_inference_reads`` - read framing of ``ReadFramingMixin``
  (sigcomp/cpu_compression.py:28-84), same validation and error messages;
* ``compress_chunks`` / ``decompress_chunks`` - chunk codec with the byte-exact
  semantics of the reference CPU backend (cpu_compression.py:178-332).

All device work goes through the C ABI of ``libsigcomp_b200.so``.  There is no
CPU fallback: without a B200 the constructor raises.
"""

import ctypes
import struct

import numpy as np

from . import _lib
from .model import IntModel, load_model

_CHUNK_LENGTH = struct.Struct("<H")


def _symbols(values):
    """Validate one token sequence (cpu_compression.py:18-25)."""
    values = np.asarray(values)
    if values.ndim != 1:
        raise ValueError("Each token sequence must be one-dimensional")
    if values.size and (values.dtype.kind not in "iu" or np.any(values < 0) or np.any(values > 255)):
        raise ValueError("Signal tokens must be integers in [0, 255]")
    return np.ascontiguousarray(values, dtype=np.uint8)


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


class B200Compression:
    DEFAULT_DIM = 256
    DEFAULT_NUM_DEC_LAYERS = 8
    DEFAULT_WINDOW_SIZE = 64

    def __init__(self, chunk_len=1024, gpu=0, model_path=None, dim=None, num_dec_layers=None,
                 window_size=None, *, model=None, mlp_path="auto"):
        if chunk_len < 1 or chunk_len > 65535:
            raise ValueError("chunk_len must be in [1, 65535]")
        if model is None:
            model = load_model(model_path, dim=dim or self.DEFAULT_DIM,
                               num_dec_layers=num_dec_layers if num_dec_layers is not None
                               else self.DEFAULT_NUM_DEC_LAYERS,
                               window_size=window_size or self.DEFAULT_WINDOW_SIZE)
        if not isinstance(model, IntModel):
            raise TypeError("model must be an IntModel")
        self.model = model
        self.chunk_len = int(chunk_len)
        self.window_size = int(model.window_size)
        self.SOS_token = 256
        self.gpu = int(gpu)
        self.device = f"cuda:{self.gpu}"
        self._lib = _lib.load()
        self._handle = ctypes.c_void_p()
        self._create(model)
        self.set_mlp_path(mlp_path)

    # -- model handle -----------------------------------------------------------
    def _create(self, m):
        emb = np.ascontiguousarray(m.embedding, dtype=np.int8)
        ws = [np.ascontiguousarray(w, dtype=np.int8) for w in m.weights]
        bs = [np.ascontiguousarray(b, dtype=np.int32) for b in m.biases]
        in_dims = np.asarray([w.shape[1] for w in ws], dtype=np.int32)
        out_dims = np.asarray([w.shape[0] for w in ws], dtype=np.int32)
        w_ptrs = (ctypes.c_void_p * len(ws))(*[w.ctypes.data for w in ws])
        b_ptrs = (ctypes.c_void_p * len(bs))(*[b.ctypes.data for b in bs])
        mults = np.ascontiguousarray(m.multipliers, dtype=np.int64)
        shifts = np.ascontiguousarray(m.shifts, dtype=np.int32)
        relu = np.ascontiguousarray(m.relu, dtype=np.uint8)
        lut = np.ascontiguousarray(m.exp_lut, dtype=np.int64)
        rc = self._lib.sc_model_create(
            self.gpu, self.window_size, emb.shape[1], len(ws), _ptr(emb), _ptr(in_dims), _ptr(out_dims),
            ctypes.cast(w_ptrs, ctypes.c_void_p), ctypes.cast(b_ptrs, ctypes.c_void_p), _ptr(mults),
            _ptr(shifts), _ptr(relu), _ptr(lut), self.chunk_len, ctypes.byref(self._handle))
        _lib.check(rc, "sc_model_create")

    def set_mlp_path(self, path):
        code = {"auto": 0, "tcgen05": 1, "cuda_cores": 2, "tcgen05_layers": 3, "tcgen05_fused1": 4,
                "tcgen05_small": 5}[path]
        _lib.check(self._lib.sc_model_set_mlp_path(self._handle, code), "sc_model_set_mlp_path")
        self.mlp_path = path

    def close(self):
        if getattr(self, "_handle", None) is not None and self._handle.value:
            self._lib.sc_model_destroy(self._handle)
            self._handle = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._handle

    # -- flat (vectorised) entry points ----------------------------------------
    def compress_flat(self, tokens, offsets, stream=None):
        """tokens uint8[T], offsets int64[n+1] -> (words uint32[W], word_offsets int64[n+1])."""
        tokens = np.ascontiguousarray(tokens, dtype=np.uint8)
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        n = len(offsets) - 1
        lengths = np.diff(offsets)
        cap = int(lengths.sum() + 2 * n) + 1
        words = np.empty(cap, dtype=np.uint32)
        word_offsets = np.zeros(n + 1, dtype=np.int64)
        if n == 0:
            return words[:0], word_offsets
        rc = self._lib.sc_compress_chunks(self._handle, _ptr(tokens), _ptr(offsets), n, _ptr(words), cap,
                                          _ptr(word_offsets), None, stream)
        _lib.check(rc, "sc_compress_chunks")
        return words[:int(word_offsets[-1])], word_offsets

    def decompress_flat(self, words, word_offsets, lengths, stream=None):
        """words uint32[W], word_offsets int64[n+1], lengths int64[n] -> tokens uint8[sum(lengths)]."""
        words = np.ascontiguousarray(words, dtype=np.uint32)
        word_offsets = np.ascontiguousarray(word_offsets, dtype=np.int64)
        lengths = np.ascontiguousarray(lengths, dtype=np.int64)
        n = len(lengths)
        out = np.empty(max(int(lengths.sum()), 1), dtype=np.uint8)
        if n == 0:
            return out[:0]
        if len(words) == 0:
            words = np.zeros(1, dtype=np.uint32)
        rc = self._lib.sc_decompress_chunks(self._handle, _ptr(words), _ptr(word_offsets), _ptr(lengths), n,
                                            _ptr(out), None, stream)
        _lib.check(rc, "sc_decompress_chunks")
        return out[:int(lengths.sum())]

    # -- signal transform on the device (main.py:504-546) ----------------------
    def split_signals(self, reads, lsb=0):
        """``_split_signal`` of every int16 read on the GPU (after the lossy step when lsb > 0).

        Returns one ``(sig0, tokens uint8, large uint16 minus 256, position deltas uint32)``
        per read, like ``sigcomp.main._split_signal``.
        """
        import torch
        reads = [np.ascontiguousarray(r, dtype=np.int16) for r in reads]
        if any(len(r) == 0 for r in reads):
            raise ValueError("Every read must hold at least one sample")
        n = len(reads)
        if n == 0:
            return []
        off = np.zeros(n + 1, dtype=np.int64)
        np.cumsum([len(r) for r in reads], out=off[1:])
        dev = torch.device(self.device)
        x = torch.from_numpy(np.concatenate(reads)).to(dev)
        d_off = torch.from_numpy(off).to(dev)
        cap = max(int(off[-1]) - n, 1)
        sig0 = torch.empty(n, dtype=torch.int16, device=dev)
        tok = torch.empty(cap, dtype=torch.uint8, device=dev)
        tok_off = torch.empty(n + 1, dtype=torch.int64, device=dev)
        large = torch.empty(cap, dtype=torch.int16, device=dev)
        pos = torch.empty(cap, dtype=torch.int32, device=dev)
        large_off = torch.empty(n + 1, dtype=torch.int64, device=dev)
        vp = ctypes.c_void_p
        rc = self._lib.sc_split_signal_device(
            self._handle, vp(x.data_ptr()), vp(d_off.data_ptr()), n, int(lsb), vp(sig0.data_ptr()),
            vp(tok.data_ptr()), vp(tok_off.data_ptr()), vp(large.data_ptr()), vp(pos.data_ptr()),
            vp(large_off.data_ptr()), vp(torch.cuda.current_stream(dev).cuda_stream))
        _lib.check(rc, "sc_split_signal_device")
        s0, to, lo = sig0.cpu().numpy(), tok_off.cpu().numpy(), large_off.cpu().numpy()
        t, lv, lp = tok.cpu().numpy(), large.cpu().numpy().view(np.uint16), pos.cpu().numpy().view(np.uint32)
        return [(int(s0[i]), t[to[i]:to[i + 1]].copy(), lv[lo[i]:lo[i + 1]].copy(), lp[lo[i]:lo[i + 1]].copy())
                for i in range(n)]

    def reassemble_signals(self, splits, lengths, lsb=0):
        """Inverse of :meth:`split_signals`: ``_reassemble_signal`` (then ``_lossy_decode``) on the GPU."""
        import torch
        n = len(splits)
        if n != len(lengths):
            raise ValueError("splits and lengths differ in length")
        if n == 0:
            return []
        lengths = np.asarray(lengths, dtype=np.int64)
        if np.any(lengths < 1):
            raise ValueError("Every read must hold at least one sample")
        off = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(lengths, out=off[1:])
        to = np.zeros(n + 1, dtype=np.int64)
        np.cumsum([len(sp[1]) for sp in splits], out=to[1:])
        lo = np.zeros(n + 1, dtype=np.int64)
        np.cumsum([len(sp[2]) for sp in splits], out=lo[1:])
        if any(len(sp[2]) != len(sp[3]) for sp in splits):
            raise ValueError("large values and position deltas differ in length")
        dev = torch.device(self.device)

        def cat(parts, dtype, view):
            a = np.concatenate([np.asarray(p_, dtype=dtype) for p_ in parts]) if parts else np.zeros(0, dtype)
            a = a if len(a) else np.zeros(1, dtype)
            return torch.from_numpy(a.view(view)).to(dev)

        sig0 = torch.from_numpy(np.asarray([sp[0] for sp in splits], dtype=np.int16)).to(dev)
        tok = cat([sp[1] for sp in splits], np.uint8, np.uint8)
        large = cat([sp[2] for sp in splits], np.uint16, np.int16)
        pos = cat([sp[3] for sp in splits], np.uint32, np.int32)
        d_off, d_to, d_lo = (torch.from_numpy(a).to(dev) for a in (off, to, lo))
        out = torch.empty(int(off[-1]), dtype=torch.int16, device=dev)
        vp = ctypes.c_void_p
        rc = self._lib.sc_reassemble_signal_device(
            self._handle, vp(sig0.data_ptr()), vp(d_off.data_ptr()), n, int(lsb), vp(tok.data_ptr()),
            vp(d_to.data_ptr()), vp(large.data_ptr()), vp(pos.data_ptr()), vp(d_lo.data_ptr()),
            vp(out.data_ptr()), vp(torch.cuda.current_stream(dev).cuda_stream))
        _lib.check(rc, "sc_reassemble_signal_device")
        o = out.cpu().numpy()
        return [o[off[i]:off[i + 1]].copy() for i in range(n)]

    # -- chunk level (QuantMLPCompression interface) ---------------------------
    def compress_chunks(self, chunks, max_batch_size=64, use_perfect=False, use_tqdm=False):
        if max_batch_size < 1:
            raise ValueError("max_batch_size must be positive")
        batch = [_symbols(c) for c in chunks]
        lengths = np.asarray([len(c) for c in batch], dtype=np.int64)
        if np.any(lengths > self.chunk_len):
            raise ValueError("A token chunk exceeds chunk_len")
        if not len(batch):
            return []
        offsets = np.zeros(len(batch) + 1, dtype=np.int64)
        np.cumsum(lengths, out=offsets[1:])
        tokens = np.concatenate(batch) if offsets[-1] else np.zeros(0, np.uint8)
        words, woff = self.compress_flat(tokens, offsets)
        raw = words.astype("<u4", copy=False).view(np.uint8)
        return [raw[4 * woff[c]:4 * woff[c + 1]].tobytes() for c in range(len(batch))]

    def decompress_chunks(self, compressed_bytes_list, valid_lengths, max_batch_size=64, use_perfect=False,
                          use_tqdm=False):
        if max_batch_size < 1:
            raise ValueError("max_batch_size must be positive")
        if len(compressed_bytes_list) != len(valid_lengths):
            raise ValueError("Compressed chunk and length counts differ")
        if any(int(n) != n or n < 0 or n > self.chunk_len for n in valid_lengths):
            raise ValueError("Chunk lengths must be integers in [0, chunk_len]")
        for data, length in zip(compressed_bytes_list, valid_lengths):
            if (length and (not data or len(data) % 4)) or (not length and data):
                raise ValueError("Invalid range-coded chunk for its token length")
        n = len(compressed_bytes_list)
        if n == 0:
            return []
        lengths = np.asarray([int(x) for x in valid_lengths], dtype=np.int64)
        nbytes = np.asarray([len(d) for d in compressed_bytes_list], dtype=np.int64)
        woff = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(nbytes // 4, out=woff[1:])
        blob = b"".join(bytes(d) for d in compressed_bytes_list)
        words = np.frombuffer(blob, dtype="<u4").astype(np.uint32, copy=False)
        tokens = self.decompress_flat(words, woff, lengths)
        toff = np.zeros(n + 1, dtype=np.int64)
        np.cumsum(lengths, out=toff[1:])
        return [tokens[toff[c]:toff[c + 1]].copy() for c in range(n)]

    # -- read level (ReadFramingMixin interface) -------------------------------
    def batch_inference_reads(self, list_of_reads=None, list_of_compressed_reads=None, list_of_lengths=None,
                              batch_size=64, use_tqdm=False, prob_quant=0):
        if batch_size < 1:
            raise ValueError("batch_size must be positive")
        L = self.chunk_len
        if list_of_reads is not None:
            reads = [_symbols(r) for r in list_of_reads]
            rlen = np.asarray([len(r) for r in reads], dtype=np.int64)
            nchunks = (rlen + L - 1) // L
            n = int(nchunks.sum())
            tokens = np.concatenate(reads) if rlen.sum() else np.zeros(0, np.uint8)
            # chunk boundaries: every read split into chunk_len pieces
            read_start = np.zeros(len(reads) + 1, dtype=np.int64)
            np.cumsum(rlen, out=read_start[1:])
            chunk_read = np.repeat(np.arange(len(reads)), nchunks)
            first_chunk = np.zeros(len(reads) + 1, dtype=np.int64)
            np.cumsum(nchunks, out=first_chunk[1:])
            k = np.arange(n) - first_chunk[chunk_read]
            starts = read_start[chunk_read] + k * L
            ends = np.minimum(starts + L, read_start[chunk_read + 1])
            offsets = np.zeros(n + 1, dtype=np.int64)
            if n:
                offsets[:-1] = starts
                offsets[-1] = ends[-1]
            words, woff = self.compress_flat(tokens, offsets) if n else (np.zeros(0, np.uint32), offsets[:1])
            # frames of every read in one pass (sc_frame_reads: the reference's checks, in C)
            words = np.ascontiguousarray(words, dtype=np.uint32)
            if not len(words):
                words = np.zeros(1, np.uint32)
            cap = 4 * int(woff[-1]) + 2 * n
            out = np.empty(max(cap, 1), dtype=np.uint8)
            out_off = np.zeros(len(reads) + 1, dtype=np.int64)
            first_chunk = np.ascontiguousarray(first_chunk, dtype=np.int64)
            rc = _lib.load().sc_frame_reads(_ptr(words), _ptr(woff), _ptr(first_chunk), len(reads), _ptr(out), len(out),
                                          _ptr(out_off))
            _lib.check(rc, "sc_frame_reads")
            return [out[out_off[r]:out_off[r + 1]].tobytes() for r in range(len(reads))]

        if list_of_compressed_reads is None or list_of_lengths is None:
            raise ValueError("Compressed reads and token lengths are required")
        if len(list_of_compressed_reads) != len(list_of_lengths):
            raise ValueError("Compressed read and token length counts differ")
        # reads are checked in order, as the reference does: the first bad token length stops the
        # parse there, after the reads before it have been checked
        n_reads = len(list_of_lengths)
        good = n_reads
        for i, length in enumerate(list_of_lengths):
            if int(length) != length or length < 0:
                good = i
                break
        data = [d if isinstance(d, bytes) else bytes(d) for d in list_of_compressed_reads[:good]]
        lens = np.asarray([int(x) for x in list_of_lengths[:good]], dtype=np.int64)
        nbytes = np.asarray([len(d) for d in data], dtype=np.int64)
        chunks_cap = int(((lens + L - 1) // L).sum())
        words_cap = int(nbytes.sum()) // 4
        words = np.empty(max(words_cap, 1), dtype=np.uint32)
        woff = np.zeros(chunks_cap + 1, dtype=np.int64)
        clen = np.zeros(max(chunks_cap, 1), dtype=np.int64)
        read_chunks = np.zeros(good + 1, dtype=np.int64)
        bad = np.full(1, -1, dtype=np.int64)
        ptrs = (ctypes.c_char_p * max(good, 1))(*data) if good else (ctypes.c_char_p * 1)()
        rc = _lib.load().sc_unframe_reads(ctypes.cast(ptrs, ctypes.c_void_p), _ptr(nbytes), _ptr(lens), good, L,
                                        _ptr(words), len(words), _ptr(woff), _ptr(clen), chunks_cap,
                                        _ptr(read_chunks), _ptr(bad))
        _lib.check(rc, "sc_unframe_reads")
        if good < n_reads:
            raise ValueError("Token lengths must be nonnegative integers")
        n = int(read_chunks[-1])
        if n == 0:
            return [np.empty(0, dtype=np.uint8) for _ in range(n_reads)]
        tokens = self.decompress_flat(words[:int(woff[n])], woff[:n + 1], clen[:n])
        toff = np.zeros(n_reads + 1, dtype=np.int64)
        np.cumsum(lens, out=toff[1:])
        return [tokens[toff[r]:toff[r + 1]].copy() for r in range(n_reads)]


# The name SigComp's _load_model builds for --device cuda.
GPUCompression = B200Compression
