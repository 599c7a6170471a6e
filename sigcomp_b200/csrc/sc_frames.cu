// SIG2 read framing on the host, for the read-level codec interface
// (ReadFramingMixin.batch_inference_reads, sigcomp/cpu_compression.py:28-84).
//
// A compressed read is its chunks' range-coder streams one after the other, each
// preceded by its byte count as a little-endian uint16.  The reference builds and
// parses these frames in Python loops; these functions do the same passes in C
// with the reference's checks and messages, so that a batch of 400 k chunks costs
// a memory copy rather than 400 k interpreter iterations.  No device work.
#include <cstring>

#include "../../include/sigcomp_b200.h"
#include "sc_internal.h"

using sc::set_error;

extern "C" {

int sc_frame_reads(const uint32_t *words, const int64_t *word_offsets, const int64_t *read_chunks, int64_t n_reads,
                   uint8_t *out, int64_t out_capacity, int64_t *out_offsets)
{
    if (n_reads < 0 || !read_chunks || !out_offsets || (n_reads > 0 && (!word_offsets || !out))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    out_offsets[0] = 0;
    for (int64_t r = 0; r < n_reads; ++r) {
        int64_t bytes = 0;
        for (int64_t c = read_chunks[r]; c < read_chunks[r + 1]; ++c) {
            const int64_t nb = 4 * (word_offsets[c + 1] - word_offsets[c]);
            if (nb > 65535) {
                set_error("Compressed chunk exceeds the SIG2 uint16 frame; compress with a smaller --chunk-len");
                return SC_ERR_INVALID_ARGUMENT;
            }
            bytes += 2 + nb;
        }
        out_offsets[r + 1] = out_offsets[r] + bytes;
    }
    if (out_offsets[n_reads] > out_capacity) {
        set_error("framed output capacity %lld is too small", (long long)out_capacity);
        return SC_ERR_CAPACITY;
    }
    for (int64_t r = 0; r < n_reads; ++r) {
        uint8_t *p = out + out_offsets[r];
        for (int64_t c = read_chunks[r]; c < read_chunks[r + 1]; ++c) {
            const int64_t nb = 4 * (word_offsets[c + 1] - word_offsets[c]);
            p[0] = (uint8_t)(nb & 0xFF);
            p[1] = (uint8_t)(nb >> 8);
            if (nb) memcpy(p + 2, words + word_offsets[c], (size_t)nb);   // little-endian words
            p += 2 + nb;
        }
    }
    return SC_OK;
}

int sc_unframe_reads(const uint8_t *const *reads, const int64_t *read_bytes, const int64_t *token_lengths,
                     int64_t n_reads, int32_t chunk_len, uint32_t *words, int64_t words_capacity,
                     int64_t *word_offsets, int64_t *chunk_lengths, int64_t chunks_capacity, int64_t *read_chunks,
                     int64_t *bad_read)
{
    if (n_reads < 0 || chunk_len < 1 || !read_chunks || !word_offsets || !bad_read ||
        (n_reads > 0 && (!reads || !read_bytes || !token_lengths))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    *bad_read = -1;
    int64_t c = 0, w = 0;
    read_chunks[0] = 0;
    word_offsets[0] = 0;
    for (int64_t r = 0; r < n_reads; ++r) {
        const uint8_t *data = reads[r];
        const int64_t len = read_bytes[r];
        int64_t remaining = token_lengths[r], pos = 0;
        if (remaining < 0) {
            *bad_read = r;
            set_error("Token lengths must be nonnegative integers");
            return SC_ERR_INVALID_ARGUMENT;
        }
        while (remaining) {
            if (pos + 2 > len) {
                *bad_read = r;
                set_error("Truncated SIG2 chunk length");
                return SC_ERR_INVALID_ARGUMENT;
            }
            const int64_t size = (int64_t)data[pos] | ((int64_t)data[pos + 1] << 8);
            pos += 2;
            if (size == 0 || size % 4 || pos + size > len) {
                *bad_read = r;
                set_error("Invalid or truncated SIG2 range-coded chunk");
                return SC_ERR_INVALID_ARGUMENT;
            }
            const int64_t count = remaining < chunk_len ? remaining : chunk_len;
            if (c >= chunks_capacity || w + size / 4 > words_capacity) {
                set_error("unframed output capacity is too small");
                return SC_ERR_CAPACITY;
            }
            memcpy(words + w, data + pos, (size_t)size);
            w += size / 4;
            chunk_lengths[c] = count;
            ++c;
            word_offsets[c] = w;
            pos += size;
            remaining -= count;
        }
        if (pos != len) {
            *bad_read = r;
            set_error("Trailing SIG2 chunk data disagrees with token length");
            return SC_ERR_INVALID_ARGUMENT;
        }
        read_chunks[r + 1] = c;
    }
    return SC_OK;
}

}  // extern "C"
