/*
 * sigcomp_b200 - C ABI of the B200 neural codec for SigComp.
 *
 * These entry points replace the device half of SigComp's codec object, the
 * object `_load_model` returns for `--device cuda` (sigcomp/main.py:189-225):
 *   - GPUCompression.compress_chunks   (sigcomp/quant_mlp_export.py:271-323)
 *   - GPUCompression.decompress_chunks (sigcomp/quant_mlp_export.py:325-377)
 * with the byte-exact semantics of the reference CPU codec
 * (sigcomp/cpu_compression.py:178-332, sigcomp/cpu_entropy_coding.py).
 *
 * Conventions
 *   - Plain pointers and sizes; no framework types.  "host" entry points take
 *     host memory (pageable or pinned) and do the copies; "_device" entry points
 *     take device pointers already resident on the model's GPU.
 *   - `stream` is a cudaStream_t passed as void*; NULL selects the default stream.
 *     Every entry point returns after its work on `stream` has completed.
 *   - Return value: SC_OK or an SC_ERR_* code; sc_last_error() gives the message
 *     (thread-local, valid until the next call on the same thread).
 *   - A chunk is at most `chunk_len` tokens (uint8, the SigComp "small" symbols).
 *     A chunk's stream is a sequence of little-endian uint32 words.
 *   - One model handle may be used by one host thread at a time.
 */
#ifndef SIGCOMP_B200_H
#define SIGCOMP_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define SC_API __attribute__((visibility("default")))
#else
#define SC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SC_OK                   0
#define SC_ERR_INVALID_ARGUMENT 1  /* reference: ValueError (bad tokens, lengths, frames) */
#define SC_ERR_CAPACITY         2  /* reference: OverflowError (coder output capacity) */
#define SC_ERR_CORRUPT_STREAM   3  /* reference: ValueError("invalid range stream or mismatching entropy model") */
#define SC_ERR_CUDA             4  /* CUDA runtime failure */
#define SC_ERR_UNSUPPORTED      5  /* model geometry or device not supported */
#define SC_ERR_OUT_OF_MEMORY    6

typedef struct sc_model sc_model;

/* Library version string. */
SC_API const char *sc_version(void);

/* Message of the last failure on this thread ("" if none). */
SC_API const char *sc_last_error(void);

/* Number of kernels this library has launched in this process (all models). */
SC_API int64_t sc_kernel_launches(void);

/*
 * Upload an integer entropy model to `device` and return a handle.
 * Replaces the device model built by QuantMLPCompression.__init__
 * (sigcomp/quant_mlp_export.py:215-269; integer parameters as derived by
 * load_cpu_decoder, sigcomp/cpu_int_inference.py:395-445).
 *
 *   embedding   int8  [257][emb_dim]            quantised embedding table
 *   in_dims/out_dims [num_layers]               layer l is out_dims[l] x in_dims[l]
 *   weights[l]  int8  [out_dims[l]][in_dims[l]] row-major
 *   biases[l]   int32 [out_dims[l]]
 *   multipliers int64 [num_layers]  M0 in [0, 2^31]
 *   shifts      int32 [num_layers]  in [0, 63]
 *   relu        uint8 [num_layers]
 *   exp_lut     int64 [256]         build_integer_exp_lut(output_scale)
 *   chunk_len   maximum tokens per chunk (SigComp -L/--chunk-len)
 * Requirements: in_dims[0] == window * emb_dim, out_dims[last] == 256.
 */
SC_API int sc_model_create(int device, int32_t window, int32_t emb_dim, int32_t num_layers,
                    const int8_t *embedding, const int32_t *in_dims, const int32_t *out_dims,
                    const int8_t *const *weights, const int32_t *const *biases,
                    const int64_t *multipliers, const int32_t *shifts, const uint8_t *relu,
                    const int64_t *exp_lut, int32_t chunk_len, sc_model **out);

/* Release the model and every device buffer it owns. */
SC_API int sc_model_destroy(sc_model *model);

/* Select the MLP implementation: 0 = automatic (the tcgen05 kernels: fused persistent
 * kernels on SM pairs for compress/decompress, the tcgen05 layer kernels for
 * sc_mlp_logits_device; a model they cannot run is refused with SC_ERR_UNSUPPORTED),
 * 1 = tcgen05 fused persistent kernels on SM pairs (cta_group::2), 2 = CUDA-core
 * kernels, 3 = tcgen05 one launch per layer, 4 = tcgen05 fused on single SMs,
 * 5 = as 1, with every decode on the small-batch decoder (a cluster of eight SMs per
 * 128 chunks), which path 0 picks for batches of at most (SMs / 8) * 128 chunks and
 * path 1 never.
 * Paths 2-5 are cross-checks of the same arithmetic, run only when selected here. */
SC_API int sc_model_set_mlp_path(sc_model *model, int32_t path);

/*
 * Compress chunks (host memory).  Replaces compress_chunks
 * (sigcomp/quant_mlp_export.py:271-323; semantics of cpu_compression.py:178-257).
 *   tokens         uint8 [token_offsets[n_chunks]]   concatenated chunks
 *   token_offsets  int64 [n_chunks + 1]              chunk c = tokens[off[c] .. off[c+1])
 *   words          uint32 [words_capacity]           output streams, concatenated
 *   words_capacity >= sum over chunks of (length + 2) always suffices
 *   word_offsets   int64 [n_chunks + 1]              output: stream c = words[wo[c] .. wo[c+1])
 *   chunk_errors   uint8 [n_chunks] or NULL          output: 1 = coder capacity exceeded
 * Empty chunks produce empty streams.
 */
SC_API int sc_compress_chunks(sc_model *model, const uint8_t *tokens, const int64_t *token_offsets,
                       int64_t n_chunks, uint32_t *words, int64_t words_capacity,
                       int64_t *word_offsets, uint8_t *chunk_errors, void *stream);

/* Same as sc_compress_chunks with every array in device memory of the model's GPU. */
SC_API int sc_compress_chunks_device(sc_model *model, const uint8_t *tokens, const int64_t *token_offsets,
                              int64_t n_chunks, uint32_t *words, int64_t words_capacity,
                              int64_t *word_offsets, uint8_t *chunk_errors, void *stream);

/*
 * Decompress chunks (host memory).  Replaces decompress_chunks
 * (sigcomp/quant_mlp_export.py:325-377; semantics of cpu_compression.py:259-332).
 *   words          uint32 [word_offsets[n_chunks]]
 *   word_offsets   int64 [n_chunks + 1]
 *   lengths        int64 [n_chunks]      tokens to decode per chunk, each in [0, chunk_len]
 *   tokens         uint8 [sum(lengths)]  output, concatenated in chunk order
 *   chunk_errors   uint8 [n_chunks] or NULL   output: 1 = invalid stream
 * A chunk with length 0 must have an empty stream and vice versa, and every
 * nonempty stream is decoded against its own word range only.
 */
SC_API int sc_decompress_chunks(sc_model *model, const uint32_t *words, const int64_t *word_offsets,
                         const int64_t *lengths, int64_t n_chunks, uint8_t *tokens,
                         uint8_t *chunk_errors, void *stream);

/* Same as sc_decompress_chunks with words/word_offsets/lengths/tokens/chunk_errors
 * in device memory.  `lengths_host` (host copy of lengths) must also be given. */
SC_API int sc_decompress_chunks_device(sc_model *model, const uint32_t *words, const int64_t *word_offsets,
                                const int64_t *lengths, const int64_t *lengths_host, int64_t n_chunks,
                                uint8_t *tokens, uint8_t *chunk_errors, void *stream);

/*
 * The integer MLP alone on device memory: windows int16 [rows][window] (token
 * ids in [0, 256]) -> logits int8 [rows][256].  Replaces the batched
 * `_ar_step` of the GPU decoder (sigcomp/quant_mlp_export.py:125-130).
 */
SC_API int sc_mlp_logits_device(sc_model *model, const int16_t *windows, int64_t rows, int8_t *logits,
                         void *stream);

/*
 * One integer linear layer of the model alone, on device memory:
 *   y[rows][out_dims[layer]] = requant(x[rows][in_dims[layer]] * W^T + b)
 * with the layer's bias, M0/shift and ReLU (cpu_int_kernels.py:5-14), computed by the
 * tcgen05 layer kernel.  Replaces the reference's per-layer GPU kernel,
 * bit_exact_linear_kernel (sigcomp/quant_mlp_export.py:21-76), and
 * CPUBitExactInt8Linear.forward (sigcomp/cpu_int_inference.py:206-256).  For layer 0, x
 * holds the gathered context windows (x[r][p * emb_dim + c] = E[token_p][c]).  x must be
 * 16-byte aligned.
 */
SC_API int sc_linear_layer_device(sc_model *model, int32_t layer, const int8_t *x, int64_t rows, int8_t *y,
                                  void *stream);

/*
 * The range coder alone on given int8 logits (no MLP), in device memory.  Replaces the
 * reference's step encoder, GpuRangeStepEncoder (sigcomp/gpu_entropy_coding.py:255-303:
 * encode_step_int8 at every step, then seal and get_compressed), with the byte-exact
 * semantics of the CPU coder (sigcomp/cpu_entropy_coding.py:90-227: _frequencies,
 * _encode_one, _seal).
 *   logits         int8  [offsets[n_streams]][256]   the model's logits of every coded step
 *   symbols        uint8 [offsets[n_streams]]        the symbols to code
 *   offsets        int64 [n_streams + 1]             stream c codes rows offsets[c] .. offsets[c+1]
 *                                                    (each at most the model's chunk_len)
 *   words, words_capacity, word_offsets, stream_errors   as in sc_compress_chunks
 */
SC_API int sc_encode_logits_device(sc_model *model, const int8_t *logits, const uint8_t *symbols,
                                   const int64_t *offsets, int64_t n_streams, uint32_t *words,
                                   int64_t words_capacity, int64_t *word_offsets, uint8_t *stream_errors,
                                   void *stream);

/*
 * Inverse: decode offsets[c+1] - offsets[c] symbols of stream c, step t using logits row
 * offsets[c] + t.  Replaces GpuRangeDecoder (sigcomp/gpu_entropy_coding.py:400-454,
 * decode_step_int8 at every step; semantics of CpuRangeDecoder and _decode_partition,
 * cpu_entropy_coding.py:230-266, 451-481).  Device memory; stream_errors as in
 * sc_decompress_chunks (SC_ERR_CORRUPT_STREAM names the first invalid stream).
 */
SC_API int sc_decode_logits_device(sc_model *model, const int8_t *logits, const int64_t *offsets,
                                   const uint32_t *words, const int64_t *word_offsets, int64_t n_streams,
                                   uint8_t *symbols, uint8_t *stream_errors, void *stream);

/*
 * SIG2 read framing on the host (no device work), for the read-level interface
 * ReadFramingMixin.batch_inference_reads (sigcomp/cpu_compression.py:28-84): a
 * compressed read is its chunks' streams in order, each preceded by its byte
 * count as a little-endian uint16.
 *
 * sc_frame_reads: read r holds chunks read_chunks[r] .. read_chunks[r+1] of the
 * streams in `words` / `word_offsets` (as written by sc_compress_chunks); its
 * framed bytes go to out[out_offsets[r] .. out_offsets[r+1]) (out_offsets has
 * n_reads + 1 entries).  A stream above 65535 bytes returns
 * SC_ERR_INVALID_ARGUMENT with the reference's message; too small an
 * out_capacity returns SC_ERR_CAPACITY.
 */
SC_API int sc_frame_reads(const uint32_t *words, const int64_t *word_offsets, const int64_t *read_chunks,
                          int64_t n_reads, uint8_t *out, int64_t out_capacity, int64_t *out_offsets);

/*
 * sc_unframe_reads: the inverse, with the reference's checks and messages in
 * read order.  Read r is reads[r][0 .. read_bytes[r]) holding token_lengths[r]
 * tokens in chunks of chunk_len; its streams are appended to `words` (chunk c =
 * words[word_offsets[c] .. word_offsets[c+1]), chunk_lengths[c] tokens) and its
 * chunks are read_chunks[r] .. read_chunks[r+1].  On a malformed read, returns
 * SC_ERR_INVALID_ARGUMENT ("Truncated SIG2 chunk length", "Invalid or truncated
 * SIG2 range-coded chunk", "Trailing SIG2 chunk data disagrees with token
 * length", "Token lengths must be nonnegative integers") with *bad_read = r.
 */
SC_API int sc_unframe_reads(const uint8_t *const *reads, const int64_t *read_bytes, const int64_t *token_lengths,
                            int64_t n_reads, int32_t chunk_len, uint32_t *words, int64_t words_capacity,
                            int64_t *word_offsets, int64_t *chunk_lengths, int64_t chunks_capacity,
                            int64_t *read_chunks, int64_t *bad_read);

/*
 * SigComp's signal split on the device: _split_signal (sigcomp/main.py:504-521)
 * of every read, after the lossy step _lossy_encode(_reduce_lsb(read, lsb), lsb)
 * (main.py:158-171) when lsb > 0.  Every array is in device memory.
 *   samples        int16 [sample_offsets[n_reads]]   reads, concatenated (each >= 1 sample)
 *   sample_offsets int64 [n_reads + 1]
 *   lsb            0 (lossless) .. 15
 * Outputs (capacity of tokens/large/large_pos: sample_offsets[n_reads] - n_reads):
 *   sig0           int16  [n_reads]        first sample of each read (after the lossy step)
 *   tokens         uint8  []               zig-zag deltas below 256, read after read: the
 *                                          codec's input (main.py:862-873)
 *   token_offsets  int64  [n_reads + 1]
 *   large          uint16 []               the other deltas, minus 256
 *   large_pos      uint32 []               their position deltas (first position, then gaps - 1)
 *   large_offsets  int64  [n_reads + 1]
 * An empty read returns SC_ERR_INVALID_ARGUMENT (the reference fails on sig[0]).
 */
SC_API int sc_split_signal_device(sc_model *model, const int16_t *samples, const int64_t *sample_offsets,
                                  int64_t n_reads, int32_t lsb, int16_t *sig0, uint8_t *tokens,
                                  int64_t *token_offsets, uint16_t *large, uint32_t *large_pos,
                                  int64_t *large_offsets, void *stream);

/*
 * Inverse on the device: _reassemble_signal (sigcomp/main.py:524-546) with the
 * large values and position deltas given decoded, then _lossy_decode
 * (main.py:170-171) when lsb > 0.  Same array layout as sc_split_signal_device;
 * samples (output) has sample_offsets[n_reads] entries.  Streams that do not
 * describe reads of the given lengths return SC_ERR_INVALID_ARGUMENT.
 */
SC_API int sc_reassemble_signal_device(sc_model *model, const int16_t *sig0, const int64_t *sample_offsets,
                                       int64_t n_reads, int32_t lsb, const uint8_t *tokens,
                                       const int64_t *token_offsets, const uint16_t *large,
                                       const uint32_t *large_pos, const int64_t *large_offsets,
                                       int16_t *samples, void *stream);

/*
 * Failure-detection self test (no counterpart in the reference, which has no
 * device-side waits).  Every device-side wait in this library is bounded: after
 * its time limit (2 s) the kernel records the timeout in a device error flag and
 * returns, and the API call reports SC_ERR_CUDA ("a device-side wait timed out").
 * This call runs one small kernel whose waits nothing will satisfy, so it returns
 * SC_ERR_CUDA with that message after about 4 s; the device stays usable.
 */
SC_API int sc_selftest_wait_timeout(sc_model *model, void *stream);

/*
 * sc_mlp_logits_device without any device allocation.  No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc, such as a host
 * framework that has reserved the GPU's memory for its own pool, or a
 * latency-critical caller that cannot accept the device-wide synchronisation
 * of cudaMalloc/cudaFree.  Same arguments and the same logits as
 * sc_mlp_logits_device (computed by the CUDA-core layer kernels).
 *
 * Its intermediate activations live in a fixed device array of
 * 2 x SC_NOALLOC_MAX_ROWS x SC_NOALLOC_MAX_WIDTH bytes (4 MiB), held on every
 * GPU that loads the library until the process exits.  rows above
 * SC_NOALLOC_MAX_ROWS return SC_ERR_INVALID_ARGUMENT; a model with a hidden
 * layer wider than SC_NOALLOC_MAX_WIDTH returns SC_ERR_UNSUPPORTED.
 * The first call on a device looks up the array's device address (a one-time
 * set-up); make that first call before any stream capture.  All calls share
 * the array: calls whose work overlaps on the GPU (other streams, threads or
 * models on the same device) race and must be serialised by the caller.
 */
#define SC_NOALLOC_MAX_ROWS  4096
#define SC_NOALLOC_MAX_WIDTH 512
SC_API int sc_mlp_logits_device_noalloc(sc_model *model, const int16_t *windows, int64_t rows,
                                        int8_t *logits, void *stream);

/*
 * Per-launch CUDA-event timing (no counterpart in the reference; instrumentation
 * for the benchmark's roofline).  sc_profile_enable(m, 1) resets the counters and
 * starts recording an event pair around every launch on its own stream;
 * sc_profile_read returns, for one kernel class, the summed device time, the
 * number of launches and the work units (rows or chunks) they processed.
 * Kernel classes: 0 context windows, 1 MLP layer 0, 2 hidden layers, 3 last
 * layer, 4 frequency/symbol selection, 5 range encoder, 6 stream compaction,
 * 7 decoder step, 8 fused compress kernel (all layers + selection; work = rows),
 * 9 fused persistent decoder on SM pairs (work = decoded tokens), 10 small-batch
 * decoder on clusters of eight SMs (work = decoded tokens), 11 signal split and
 * 12 signal reassembly (work = samples).
 */
SC_API int sc_profile_enable(sc_model *model, int32_t enable);
SC_API int sc_profile_read(sc_model *model, int32_t kind, double *total_ms, int64_t *launches, int64_t *work);

/*
 * Unit trace of the fused kernels (no counterpart in the reference; pipeline
 * instrumentation).  With records_per_cta > 0 every later fused launch records,
 * for the first SM pair, one 16-byte event per role and unit: word 0 is the GPU
 * %globaltimer (ns), word 1 packs role | event << 4 | layer << 8 | half << 12 |
 * slot << 16 | step << 32 (roles 0 producer, 1 MMA, 2 epilogue, 3 layer-0
 * builders; events 0 begin, 1 dependency satisfied, 2 end).  0 disables.
 * The records of a CTA are split evenly over the four roles (each role keeps
 * at most records_per_cta / 4).  sc_trace_read copies up to `capacity` records
 * of CTA 0 or 1 of the most recent launch, role after role, and returns their
 * number (-1 on error).
 */
SC_API int sc_trace_enable(sc_model *model, int32_t records_per_cta);
SC_API int64_t sc_trace_read(sc_model *model, int32_t cta, uint64_t *records, int64_t capacity);

#ifdef __cplusplus
}
#endif

#endif /* SIGCOMP_B200_H */
