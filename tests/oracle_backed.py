"""Test double shared by the CPU tests: B200Compression's host-side framing with the CPU
oracle in place of its device calls."""

import numpy as np

from oracle import signal


class OracleBacked:
    """B200Compression's host framing with the CPU oracle in place of the device calls
    (compress_flat / decompress_flat, and the signal split / reassembly), so that the host code
    around them is checked on the CPU."""

    def __new__(cls, model, chunk_len=2048):
        from sigcomp_b200.codec import B200Compression
        from oracle.oracle import OracleModel
        obj = object.__new__(B200Compression)
        obj.chunk_len, obj.window_size, obj.SOS_token = chunk_len, 64, 256
        om = OracleModel(model)

        def compress_flat(tokens, offsets, stream=None):
            chunks = [tokens[offsets[i]:offsets[i + 1]] for i in range(len(offsets) - 1)]
            words = [np.frombuffer(s, "<u4") for s in om.compress_chunks(chunks, chunk_len, backend="int_mm")]
            woff = np.zeros(len(words) + 1, np.int64)
            np.cumsum([len(w) for w in words], out=woff[1:])
            return np.concatenate(words + [np.zeros(0, "<u4")]).astype(np.uint32), woff

        def decompress_flat(words, word_offsets, lengths, stream=None):
            streams = [words[word_offsets[i]:word_offsets[i + 1]].astype("<u4").tobytes()
                       for i in range(len(lengths))]
            out = om.decompress_chunks(streams, [int(x) for x in lengths], chunk_len, backend="int_mm")
            return np.concatenate(out + [np.zeros(0, np.uint8)])

        def split_signals(reads, lsb=0):
            return signal.reads_to_tokens(reads, lsb)

        def reassemble_signals(splits, lengths, lsb=0):
            out = [signal.reassemble_signal(s[0], int(n), s[1], s[2], s[3]) for s, n in zip(splits, lengths)]
            return [signal.lossy_decode(o, lsb) for o in out] if lsb else out

        obj.compress_flat, obj.decompress_flat = compress_flat, decompress_flat
        obj.split_signals, obj.reassemble_signals = split_signals, reassemble_signals
        return obj
