/*
 * CPU oracle for the SigComp neural codec hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is a plain-C restatement of the
 * reference's CPU codec, used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py as the checker.  The product (sigcomp_b200/)
 * never links or calls it.
 *
 * Parity is pinned: tests/golden/ holds streams, logits and exported model
 * digests produced by running the reference's own CPU codec
 * (sigcomp/cpu_compression.py, cpu_entropy_coding.py, cpu_int_inference.py),
 * and tests/test_oracle_golden.py checks this file against them.
 *
 * Reference functions restated here (paths relative to the SigComp tree):
 *   sco_frequencies     - _frequencies          sigcomp/cpu_entropy_coding.py:90-110
 *   sco_encode_symbol   - _encode_one           sigcomp/cpu_entropy_coding.py:121-161
 *   sco_seal            - _seal                 sigcomp/cpu_entropy_coding.py:206-227
 *   sco_decoder_init    - CpuRangeDecoder.__init__ sigcomp/cpu_entropy_coding.py:451-481
 *   sco_decode_symbol   - _decode_partition     sigcomp/cpu_entropy_coding.py:230-266
 *   sco_requantize      - _requantize           sigcomp/cpu_int_kernels.py:5-14
 *   sco_mlp_rows        - _embedding_window_row + CPUBitExactInt8Linear.forward
 *                         sigcomp/cpu_int_kernels.py:107-121, cpu_int_inference.py:206-256
 *   sco_compress_chunks - CPUQuantMLPCompression.compress_chunks  cpu_compression.py:178-257
 *   sco_decompress_chunks - CPUQuantMLPCompression.decompress_chunks cpu_compression.py:259-332
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define SCO_VOCAB 256
#define SCO_SOS 256
#define SCO_TOTAL ((int64_t)1 << 24)
#define SCO_RENORM ((uint64_t)1 << 32)

typedef struct {
    int window;          /* context window (64) */
    int emb_dim;         /* embedding width (128) */
    int num_layers;      /* linear layers (9) */
    const int8_t *embedding;      /* [257][emb_dim] */
    const int32_t *in_dims;       /* [num_layers] */
    const int32_t *out_dims;      /* [num_layers] */
    const int8_t *const *weights; /* [num_layers] -> [out][in] */
    const int32_t *const *biases; /* [num_layers] -> [out] */
    const int64_t *multipliers;   /* [num_layers] */
    const int32_t *shifts;        /* [num_layers] */
    const uint8_t *relu;          /* [num_layers] */
    const int64_t *exp_lut;       /* [256] */
} sco_model;

/* ---- entropy model: logits -> 24-bit frequency table ---------------------- */

void sco_frequencies(const int8_t *logits, const int64_t *lut, int64_t *freqs)
{
    int maximum = -128;
    for (int v = 0; v < SCO_VOCAB; ++v)
        if (logits[v] > maximum) maximum = logits[v];
    int64_t total = 0;
    for (int v = 0; v < SCO_VOCAB; ++v) {
        freqs[v] = lut[maximum - logits[v]];
        total += freqs[v];
    }
    int64_t total_freq = 0, max_freq = 0;
    int max_index = 0;
    for (int v = 0; v < SCO_VOCAB; ++v) {
        int64_t f = (freqs[v] * SCO_TOTAL) / total;
        if (f < 1) f = 1;
        freqs[v] = f;
        total_freq += f;
        if (f > max_freq) { max_freq = f; max_index = v; }
    }
    freqs[max_index] -= total_freq - SCO_TOTAL;
}

/* ---- range encoder --------------------------------------------------------- */

typedef struct {
    uint64_t lower, range;
    int64_t inverted;
    uint32_t first;
    int64_t position;
    /* coverage counters for the tests (no effect on the output): carry episodes (inverted
       set to 1), the longest run of inverted words, whether the seal flushed inverted words
       and whether it emitted the extra zero word */
    int64_t cov_episodes, cov_longest;
    int cov_seal_flush, cov_seal_zero;
} sco_encoder;

void sco_encoder_init(sco_encoder *e)
{
    e->lower = 0; e->range = ~(uint64_t)0; e->inverted = 0; e->first = 0; e->position = 0;
    e->cov_episodes = 0; e->cov_longest = 0; e->cov_seal_flush = 0; e->cov_seal_zero = 0;
}

/* returns 0 on success, 1 when the output capacity would be exceeded */
int sco_encode_symbol(sco_encoder *e, const int64_t *freqs, int symbol,
                      uint32_t *out, int64_t capacity)
{
    uint64_t cumulative = 0;
    for (int v = 0; v < symbol; ++v) cumulative += (uint64_t)freqs[v];
    uint64_t scale = e->range >> 24;
    uint64_t new_range = scale * (uint64_t)freqs[symbol];
    uint64_t new_lower = e->lower + scale * cumulative;
    if (e->inverted > 0 && new_lower + new_range > new_lower) {
        uint64_t emit_first, emit_rest;
        if (new_lower < e->lower) { emit_first = (uint64_t)e->first + 1; emit_rest = 0; }
        else { emit_first = e->first; emit_rest = 0xFFFFFFFFull; }
        if (e->position + e->inverted > capacity) return 1;
        out[e->position++] = (uint32_t)emit_first;
        for (int64_t i = 0; i < e->inverted - 1; ++i) out[e->position++] = (uint32_t)emit_rest;
        e->inverted = 0;
    }
    e->lower = new_lower;
    e->range = new_range;
    if (e->range < SCO_RENORM) {
        e->range <<= 32;
        uint32_t lower_word = (uint32_t)(e->lower >> 32);
        e->lower <<= 32;
        if (e->inverted > 0) {
            e->inverted += 1;
        } else if (e->lower + e->range > e->lower) {
            if (e->position >= capacity) return 1;
            out[e->position++] = lower_word;
        } else {
            e->inverted = 1;
            e->first = lower_word;
            e->cov_episodes += 1;
        }
        if (e->inverted > e->cov_longest) e->cov_longest = e->inverted;
    }
    return 0;
}

/* returns 0 on success, 1 on capacity overflow */
int sco_seal(sco_encoder *e, uint32_t *out, int64_t capacity)
{
    if (e->range != ~(uint64_t)0) {
        uint64_t point = e->lower + 0xFFFFFFFFull;
        if (e->inverted > 0) {
            uint64_t emit_first, emit_rest;
            e->cov_seal_flush = 1;
            if (point < e->lower) { emit_first = (uint64_t)e->first + 1; emit_rest = 0; }
            else { emit_first = e->first; emit_rest = 0xFFFFFFFFull; }
            if (e->position >= capacity) return 1;
            out[e->position++] = (uint32_t)emit_first;
            for (int64_t i = 0; i < e->inverted - 1; ++i) {
                if (e->position >= capacity) return 1;
                out[e->position++] = (uint32_t)emit_rest;
            }
        }
        uint64_t point_word = point >> 32;
        if (e->position >= capacity) return 1;
        out[e->position++] = (uint32_t)point_word;
        uint64_t upper_word = (e->lower + e->range) >> 32;
        if (upper_word == point_word) {
            if (e->position >= capacity) return 1;
            out[e->position++] = 0;
            e->cov_seal_zero = 1;
        }
    }
    return 0;
}

/* Encode one chunk from precomputed logits [T][256].  Returns 0 / 1 (capacity). */
int sco_encode_chunk(const int8_t *logits, const uint8_t *symbols, int64_t T,
                     const int64_t *lut, uint32_t *out, int64_t capacity, int64_t *nwords)
{
    sco_encoder e;
    int64_t freqs[SCO_VOCAB];
    sco_encoder_init(&e);
    for (int64_t t = 0; t < T; ++t) {
        sco_frequencies(logits + t * SCO_VOCAB, lut, freqs);
        if (sco_encode_symbol(&e, freqs, symbols[t], out, capacity)) { *nwords = e.position; return 1; }
    }
    int rc = sco_seal(&e, out, capacity);
    *nwords = e.position;
    return rc;
}

/* sco_encode_chunk that also reports which carry paths the stream took:
   cov[0] carry episodes, cov[1] longest inverted run, cov[2] seal flushed inverted words,
   cov[3] seal emitted the extra zero word. */
int sco_encode_chunk_coverage(const int8_t *logits, const uint8_t *symbols, int64_t T, const int64_t *lut,
                              uint32_t *out, int64_t capacity, int64_t *nwords, int64_t *cov)
{
    sco_encoder e;
    int64_t freqs[SCO_VOCAB];
    int rc = 0;
    sco_encoder_init(&e);
    for (int64_t t = 0; t < T && !rc; ++t) {
        sco_frequencies(logits + t * SCO_VOCAB, lut, freqs);
        rc = sco_encode_symbol(&e, freqs, symbols[t], out, capacity);
    }
    if (!rc) rc = sco_seal(&e, out, capacity);
    *nwords = e.position;
    cov[0] = e.cov_episodes;
    cov[1] = e.cov_longest;
    cov[2] = e.cov_seal_flush;
    cov[3] = e.cov_seal_zero;
    return rc;
}

/* ---- range decoder --------------------------------------------------------- */

typedef struct {
    uint64_t lower, range, point;
    int64_t read_pos, end_pos;
    const uint32_t *words;
} sco_decoder;

void sco_decoder_init(sco_decoder *d, const uint32_t *words, int64_t n)
{
    uint64_t point = 0;
    int64_t take = n < 2 ? n : 2;
    for (int64_t i = 0; i < take; ++i) point = (point << 32) | words[i];
    if (n == 1) point <<= 32;
    d->point = point;
    d->lower = 0;
    d->range = ~(uint64_t)0;
    d->read_pos = take;
    d->end_pos = n;
    d->words = words;
}

/* returns 0 ok, 1 invalid stream; *symbol receives the decoded symbol (256 on error) */
int sco_decode_symbol(sco_decoder *d, const int8_t *logits, const int64_t *lut, int *symbol)
{
    int64_t freqs[SCO_VOCAB];
    uint64_t scale = d->range >> 24;
    if (scale == 0) { *symbol = SCO_SOS; return 1; }
    uint64_t quantile = (d->point - d->lower) / scale;
    if (quantile >= (uint64_t)SCO_TOTAL) { *symbol = SCO_SOS; return 1; }
    sco_frequencies(logits, lut, freqs);
    uint64_t cumulative = 0;
    int s = 0;
    while (s < SCO_VOCAB - 1 && cumulative + (uint64_t)freqs[s] <= quantile) {
        cumulative += (uint64_t)freqs[s];
        ++s;
    }
    d->lower += scale * cumulative;
    d->range = scale * (uint64_t)freqs[s];
    if (d->range < SCO_RENORM) {
        d->lower <<= 32;
        d->range <<= 32;
        d->point <<= 32;
        if (d->read_pos < d->end_pos) d->point |= d->words[d->read_pos];
        d->read_pos += 1;
    }
    *symbol = s;
    return 0;
}

/* ---- integer MLP ----------------------------------------------------------- */

static inline int8_t sco_requantize(int32_t acc, int32_t bias, int64_t m0, int shift, int relu)
{
    int32_t biased = (int32_t)(uint32_t)((uint32_t)acc + (uint32_t)bias);   /* int32 wrap */
    int64_t prod = (int64_t)biased * m0;
    /* arithmetic shift == floor division by 2**shift */
    int64_t scaled = prod >= 0 ? (prod >> shift) : ~((~prod) >> shift);
    int64_t lo = relu ? 0 : -128;
    if (scaled < lo) scaled = lo;
    if (scaled > 127) scaled = 127;
    return (int8_t)scaled;
}

int8_t sco_requantize_one(int32_t acc, int32_t bias, int64_t m0, int32_t shift, int32_t relu)
{
    return sco_requantize(acc, bias, m0, shift, relu);
}

static int sco_max_width(const sco_model *m)
{
    int w = m->window * m->emb_dim;
    for (int l = 0; l < m->num_layers; ++l)
        if (m->out_dims[l] > w) w = m->out_dims[l];
    return w;
}

/* One row: window tokens (int16, values in [0, 256]) -> int8 logits. */
static void sco_mlp_row(const sco_model *m, const int16_t *window, int8_t *x, int8_t *y, int8_t *logits)
{
    const int E = m->emb_dim;
    for (int p = 0; p < m->window; ++p)
        memcpy(x + (size_t)p * E, m->embedding + (size_t)window[p] * E, (size_t)E);
    for (int l = 0; l < m->num_layers; ++l) {
        const int K = m->in_dims[l], N = m->out_dims[l];
        const int8_t *W = m->weights[l];
        int8_t *dst = (l == m->num_layers - 1) ? logits : y;
        for (int n = 0; n < N; ++n) {
            const int8_t *w = W + (size_t)n * K;
            int32_t acc = 0;
            for (int k = 0; k < K; ++k) acc += (int32_t)x[k] * (int32_t)w[k];
            dst[n] = sco_requantize(acc, m->biases[l][n], m->multipliers[l], m->shifts[l], m->relu[l]);
        }
        if (dst == y) { int8_t *t = x; x = y; y = t; }
    }
}

/* rows x window tokens -> rows x out logits.  Returns 1 if a token is outside [0, 256]. */
int sco_mlp_rows(const sco_model *m, const int16_t *windows, int64_t rows, int8_t *logits)
{
    const int W = sco_max_width(m);
    const int out = m->out_dims[m->num_layers - 1];
    int bad = 0;
    for (int64_t r = 0; r < rows * m->window; ++r)
        if (windows[r] < 0 || windows[r] > SCO_SOS) bad = 1;
    if (bad) return 1;
#pragma omp parallel
    {
        int8_t *x = (int8_t *)malloc((size_t)W), *y = (int8_t *)malloc((size_t)W);
#pragma omp for schedule(dynamic, 16)
        for (int64_t r = 0; r < rows; ++r)
            sco_mlp_row(m, windows + r * m->window, x, y, logits + r * out);
        free(x); free(y);
    }
    return 0;
}

/* Linear epilogue on a precomputed int32 accumulator (for the int_mm baseline).
 * With m0 < 2^31 and shift >= 32 (the exported models' case) the product's floor
 * division runs on 32-bit lanes: floor(p / 2^s) = floor(floor(p / 2^32) / 2^(s-32)),
 * and floor(p / 2^32) is the high word of the 64-bit product; otherwise every
 * element takes sco_requantize.  Both give sco_requantize's value. */
void sco_epilogue(const int32_t *acc, int64_t rows, int32_t n, const int32_t *bias,
                  int64_t m0, int32_t shift, int32_t relu, int8_t *out)
{
    if (m0 >= 0 && m0 < ((int64_t)1 << 31) && shift >= 32 && shift <= 63) {
        const int32_t m = (int32_t)m0, sh = shift - 32, lo = relu ? 0 : -128;
#pragma omp parallel for schedule(static)
        for (int64_t r = 0; r < rows; ++r) {
            const int32_t *a = acc + r * n;
            int8_t *o = out + r * n;
            for (int32_t c = 0; c < n; ++c) {
                const int32_t b = (int32_t)((uint32_t)a[c] + (uint32_t)bias[c]);   /* int32 wrap */
                const int32_t hi = (int32_t)(((int64_t)b * m) >> 32);
                int32_t v = hi >> sh;
                v = v < lo ? lo : v;
                v = v > 127 ? 127 : v;
                o[c] = (int8_t)v;
            }
        }
        return;
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int32_t c = 0; c < n; ++c)
            out[r * n + c] = sco_requantize(acc[r * n + c], bias[c], m0, shift, relu);
}

/* Teacher-forced windows for the rows of a set of chunks: rows are chunk-major,
 * row (c, t) holds tokens t-window..t-1 of chunk c, SOS before the chunk start. */
void sco_build_windows(const uint8_t *tokens, const int64_t *offsets, int64_t n_chunks,
                       int32_t window, int16_t *windows)
{
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t c = 0; c < n_chunks; ++c) {
        const int64_t begin = offsets[c], len = offsets[c + 1] - offsets[c];
        for (int64_t t = 0; t < len; ++t) {
            int16_t *w = windows + (begin + t) * window;
            for (int p = 0; p < window; ++p) {
                int64_t s = t - window + p;
                w[p] = s < 0 ? SCO_SOS : tokens[begin + s];
            }
        }
    }
}

/* Range-encode every chunk from its rows of logits.  words_out holds
 * `capacity` words per chunk; nwords[c] receives the stream length.
 * errors[c] = 1 on capacity overflow.  Returns the number of failed chunks. */
int64_t sco_encode_chunks(const int8_t *logits, const uint8_t *tokens, const int64_t *offsets,
                          int64_t n_chunks, const int64_t *lut, uint32_t *words_out,
                          int64_t capacity, int64_t *nwords, uint8_t *errors)
{
    int64_t failed = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(+:failed)
    for (int64_t c = 0; c < n_chunks; ++c) {
        const int64_t begin = offsets[c], len = offsets[c + 1] - offsets[c];
        if (len == 0) { nwords[c] = 0; errors[c] = 0; continue; }
        int rc = sco_encode_chunk(logits + begin * SCO_VOCAB, tokens + begin, len, lut,
                                  words_out + c * capacity, capacity, &nwords[c]);
        errors[c] = (uint8_t)rc;
        failed += rc;
    }
    return failed;
}

/* Full teacher-forced compression of chunks (MLP + coder), chunk-parallel. */
int64_t sco_compress_chunks(const sco_model *m, const uint8_t *tokens, const int64_t *offsets,
                            int64_t n_chunks, uint32_t *words_out, int64_t capacity,
                            int64_t *nwords, uint8_t *errors)
{
    const int64_t rows = offsets[n_chunks];
    int16_t *windows = (int16_t *)malloc((size_t)(rows > 0 ? rows : 1) * m->window * sizeof(int16_t));
    int8_t *logits = (int8_t *)malloc((size_t)(rows > 0 ? rows : 1) * SCO_VOCAB);
    sco_build_windows(tokens, offsets, n_chunks, m->window, windows);
    sco_mlp_rows(m, windows, rows, logits);
    int64_t failed = sco_encode_chunks(logits, tokens, offsets, n_chunks, m->exp_lut,
                                       words_out, capacity, nwords, errors);
    free(windows);
    free(logits);
    return failed;
}

/* Autoregressive decompression.  words/word_offsets hold each chunk's stream;
 * lengths[c] tokens are decoded into tokens_out at token_offsets[c].
 * errors[c] = 1 marks an invalid stream.  Returns the number of failed chunks. */
int64_t sco_decompress_chunks(const sco_model *m, const uint32_t *words, const int64_t *word_offsets,
                              const int64_t *lengths, int64_t n_chunks, const int64_t *token_offsets,
                              uint8_t *tokens_out, uint8_t *errors)
{
    const int W = sco_max_width(m);
    int64_t failed = 0;
#pragma omp parallel reduction(+:failed)
    {
        int8_t *x = (int8_t *)malloc((size_t)W), *y = (int8_t *)malloc((size_t)W);
        int8_t logits[SCO_VOCAB];
        int16_t *window = (int16_t *)malloc(sizeof(int16_t) * (size_t)m->window);
#pragma omp for schedule(dynamic, 1)
        for (int64_t c = 0; c < n_chunks; ++c) {
            sco_decoder d;
            const int64_t len = lengths[c];
            uint8_t *dst = tokens_out + token_offsets[c];
            errors[c] = 0;
            sco_decoder_init(&d, words + word_offsets[c], word_offsets[c + 1] - word_offsets[c]);
            for (int64_t t = 0; t < len; ++t) {
                for (int p = 0; p < m->window; ++p) {
                    int64_t s = t - m->window + p;
                    window[p] = s < 0 ? SCO_SOS : dst[s];
                }
                sco_mlp_row(m, window, x, y, logits);
                int sym;
                if (sco_decode_symbol(&d, logits, m->exp_lut, &sym)) { errors[c] = 1; break; }
                dst[t] = (uint8_t)sym;
            }
            failed += errors[c];
        }
        free(x); free(y); free(window);
    }
    return failed;
}

/* Decode one chunk from precomputed logits (used to test the decoder alone). */
int sco_decode_chunk_logits(const uint32_t *words, int64_t n, const int8_t *logits, int64_t T,
                            const int64_t *lut, int32_t *symbols)
{
    sco_decoder d;
    sco_decoder_init(&d, words, n);
    for (int64_t t = 0; t < T; ++t) {
        int s;
        if (sco_decode_symbol(&d, logits + t * SCO_VOCAB, lut, &s)) { symbols[t] = s; return 1; }
        symbols[t] = s;
    }
    return 0;
}

/* ---- batched autoregressive decoding (for the int_mm CPU baseline) -------
 * Mirrors the loop of decompress_chunks (cpu_compression.py:310-323): the MLP
 * of all active chunks runs as one batch per step, then every chunk decodes
 * one symbol. */

void *sco_dec_batch_create(const uint32_t *words, const int64_t *word_offsets, int64_t n)
{
    sco_decoder *d = (sco_decoder *)malloc(sizeof(sco_decoder) * (size_t)(n > 0 ? n : 1));
    for (int64_t c = 0; c < n; ++c)
        sco_decoder_init(&d[c], words + word_offsets[c], word_offsets[c + 1] - word_offsets[c]);
    return d;
}

void sco_dec_batch_free(void *h) { free(h); }

void sco_dec_batch_windows(const uint8_t *tokens, const int64_t *tok_off, const int64_t *idx, int64_t n_act,
                           int64_t t, int32_t window, int16_t *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n_act; ++i) {
        const uint8_t *src = tokens + tok_off[idx[i]];
        for (int p = 0; p < window; ++p) {
            int64_t s = t - window + p;
            out[i * window + p] = s < 0 ? SCO_SOS : src[s];
        }
    }
}

/* returns the number of chunks that failed at this step */
int64_t sco_dec_batch_step(void *h, const int8_t *logits, const int64_t *idx, int64_t n_act, const int64_t *lut,
                           uint8_t *tokens, const int64_t *tok_off, int64_t t, uint8_t *errors)
{
    sco_decoder *d = (sco_decoder *)h;
    int64_t failed = 0;
#pragma omp parallel for schedule(static) reduction(+:failed)
    for (int64_t i = 0; i < n_act; ++i) {
        const int64_t c = idx[i];
        int s;
        if (sco_decode_symbol(&d[c], logits + i * SCO_VOCAB, lut, &s)) {
            errors[c] = 1;
            failed += 1;
            continue;
        }
        tokens[tok_off[c] + t] = (uint8_t)s;
    }
    return failed;
}

/* Embedding gather of context windows: x[r][p*E + c] = E[win[r][p]][c]
 * (_embedding_window_row, sigcomp/cpu_int_kernels.py:107-121). Returns 1 on an
 * out-of-vocabulary token. */
int sco_gather_windows(const sco_model *m, const int16_t *windows, int64_t rows, int8_t *x)
{
    const int E = m->emb_dim, W = m->window;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(|:bad)
    for (int64_t r = 0; r < rows; ++r) {
        for (int p = 0; p < W; ++p) {
            const int tok = windows[r * W + p];
            if (tok < 0 || tok > SCO_SOS) { bad = 1; continue; }
            if (E == 128)          /* the exported models' width: a fixed-size copy */
                memcpy(x + (r * W + p) * 128, m->embedding + (size_t)tok * 128, 128);
            else
                memcpy(x + (r * W + p) * E, m->embedding + (size_t)tok * E, (size_t)E);
        }
    }
    return bad;
}
