// Chunk compression / decompression on the GPU.
//
// compress (teacher forced, cpu_compression.py:178-257):
//   windows -> integer MLP -> per-row (cum, freq) of the coded symbol
//   -> one sequential range encoder per chunk (thread per chunk) -> seal
//   -> word counts -> scan -> compaction into the caller's buffer.
// decompress (autoregressive, cpu_compression.py:259-332):
//   chunks ordered by length (descending) so the chunks still decoding at
//   step t are a prefix; per step: windows of the prefix -> MLP -> one warp per
//   chunk decodes a symbol and appends it to the chunk's output tokens.
#include <algorithm>
#include <cub/device/device_scan.cuh>

#include "sc_internal.h"

namespace sc {
namespace {

// --- compress --------------------------------------------------------------

// windows for the rows of chunks [c0, c1); row r = token_offsets[c] - row_base + t
__global__ void k_windows_compress(const uint8_t *__restrict__ tokens, const int64_t *__restrict__ off,
                                   int64_t c0, int64_t row_base, int window, int16_t *__restrict__ win)
{
    const int64_t c = c0 + blockIdx.x;
    const int64_t begin = off[c], len = off[c + 1] - begin;
    for (int64_t t = (int64_t)blockIdx.y * blockDim.x + threadIdx.x; t < len; t += (int64_t)gridDim.y * blockDim.x) {
        int16_t *w = win + (begin - row_base + t) * window;
        for (int p = 0; p < window; ++p) {
            const int64_t s = t - window + p;
            w[p] = s < 0 ? (int16_t)SC_SOS : (int16_t)tokens[begin + s];
        }
    }
}

// one warp per row: exact frequency table, then (cum, freq) of the coded symbol
__global__ void __launch_bounds__(256) k_cdf_select(const int8_t *__restrict__ logits,
                                                    const uint8_t *__restrict__ symbols,
                                                    const uint64_t *__restrict__ lut, int64_t rows,
                                                    uint2 *__restrict__ pairs)
{
    __shared__ uint64_t lut_s[SC_VOCAB];
    for (int i = threadIdx.x; i < SC_VOCAB; i += blockDim.x) lut_s[i] = lut[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const uint2 raw = *reinterpret_cast<const uint2 *>(logits + r * SC_VOCAB + lane * 8);
        int8_t x[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            x[j] = (int8_t)(raw.x >> (8 * j));
            x[4 + j] = (int8_t)(raw.y >> (8 * j));
        }
        uint32_t f[8];
        warp_frequencies(x, lut_s, f);
        const int sym = symbols[r];
        uint32_t part = 0, fs = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int v = lane * 8 + j;
            part += v < sym ? f[j] : 0u;
            fs = v == sym ? f[j] : fs;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            part += __shfl_xor_sync(0xffffffffu, part, o);
            fs += __shfl_xor_sync(0xffffffffu, fs, o);
        }
        if (lane == 0) pairs[r] = make_uint2(part, fs);
    }
}

// one thread per chunk: sequential range coding of the chunk's rows, then seal.
// The (cum, freq) pairs are fetched 16 at a time so one memory latency covers
// 16 symbol steps.
__global__ void k_encode(const uint2 *__restrict__ pairs, const int64_t *__restrict__ off, int64_t c0,
                         int64_t n, int64_t row_base, uint32_t *__restrict__ stage, int64_t cap,
                         int64_t *__restrict__ nwords, uint8_t *__restrict__ errors)
{
    constexpr int PF = 16;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t c = c0 + i;
    const int64_t begin = off[c] - row_base, len = off[c + 1] - off[c];
    uint32_t *out = stage + i * cap;
    EncState e;
    enc_init(e);
    int err = 0;
    for (int64_t t0 = 0; t0 < len && !err; t0 += PF) {
        uint2 pv[PF];
#pragma unroll
        for (int k = 0; k < PF; ++k) pv[k] = t0 + k < len ? pairs[begin + t0 + k] : make_uint2(0, 0);
#pragma unroll
        for (int k = 0; k < PF; ++k)
            if (t0 + k < len && !err) err = enc_symbol(e, pv[k].x, pv[k].y, out, cap);
    }
    if (!err) err = enc_seal(e, out, cap);
    nwords[i] = e.pos;
    errors[i] = (uint8_t)err;
}

// word_offsets[c0+1+i] = word_offsets[c0] + incl[i]; copy chunk words to place
__global__ void k_compact(const uint32_t *__restrict__ stage, int64_t cap, const int64_t *__restrict__ nwords,
                          const int64_t *__restrict__ incl, int64_t n, int64_t c0, int64_t *__restrict__ word_offsets,
                          uint32_t *__restrict__ words, int64_t words_capacity, int *__restrict__ overflow)
{
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= n) return;
    const int64_t base = word_offsets[c0];
    const int64_t end = base + incl[warp];
    const int64_t cnt = nwords[warp];
    const int64_t dst = end - cnt;
    if (lane == 0) word_offsets[c0 + 1 + warp] = end;
    if (end > words_capacity) {
        if (lane == 0) atomicExch(overflow, 1);
        return;
    }
    const uint32_t *src = stage + warp * cap;
    for (int64_t k = lane; k < cnt; k += 32) words[dst + k] = src[k];
}

__global__ void k_set_i64(int64_t *p, int64_t v) { *p = v; }

// --- decompress ------------------------------------------------------------

__global__ void k_dec_init(const uint32_t *__restrict__ words, const int64_t *__restrict__ word_offsets,
                           const int64_t *__restrict__ lengths, const int64_t *__restrict__ order, int64_t n,
                           DecState *__restrict__ st, uint8_t *__restrict__ errors, int *__restrict__ bad)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t c = order[i];
    const int64_t b = word_offsets[c], e = word_offsets[c + 1];
    errors[c] = 0;
    // an empty stream must go with an empty chunk and vice versa (cpu_compression.py:288-290)
    if ((lengths[c] > 0) != (e > b) || e < b) atomicExch(bad, 1);
    DecState d;
    dec_init(d, words, b, e);
    st[i] = d;
}

__global__ void k_windows_decode(const uint8_t *__restrict__ tokens, const int64_t *__restrict__ tok_off,
                                 const int64_t *__restrict__ order, int64_t n_act, int64_t t, int window,
                                 int16_t *__restrict__ win)
{
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_act * window) return;
    const int64_t i = idx / window;
    const int p = (int)(idx - i * window);
    const int64_t s = t - window + p;
    win[idx] = s < 0 ? (int16_t)SC_SOS : (int16_t)tokens[tok_off[order[i]] + s];
}

// One range-decoder step of one chunk by a whole warp (_decode_partition,
// cpu_entropy_coding.py:230-266): the exact frequency table of the row's 256 logits, the
// symbol whose interval holds the quotient, and the state update with renormalisation.
// Every lane holds the same state and ends with the same symbol.  Returns false (state
// untouched) for a stream that does not fit the model: zero scale or quotient >= 2^24.
__device__ __forceinline__ bool warp_decode_step(const int8_t *__restrict__ row, const uint64_t *lut_s,
                                                 const uint32_t *__restrict__ words, DecState &d, int &sym)
{
    const int lane = threadIdx.x & 31;
    const uint64_t scale = d.range >> SC_PRECISION;
    const uint64_t q = scale ? (d.point - d.lower) / scale : ~0ull;
    if (scale == 0 || q >= (uint64_t)SC_TOTAL) return false;
    const uint2 raw = *reinterpret_cast<const uint2 *>(row + lane * 8);
    int8_t x[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        x[j] = (int8_t)(raw.x >> (8 * j));
        x[4 + j] = (int8_t)(raw.y >> (8 * j));
    }
    uint32_t f[8];
    warp_frequencies(x, lut_s, f);
    uint32_t lsum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) lsum += f[j];
    // exclusive prefix over lanes
    uint32_t incl = lsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    uint32_t cum = incl - lsum;
    // symbol = (number of symbols whose exclusive cdf <= q) - 1
    int cnt = 0;
    uint32_t my_cum = 0, my_f = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if ((uint64_t)cum <= q) {
            ++cnt;
            my_cum = cum;
            my_f = f[j];
        }
        cum += f[j];
    }
    int total = cnt;
#pragma unroll
    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    sym = total - 1;
    const int owner = sym >> 3;
    const uint32_t s_cum = __shfl_sync(0xffffffffu, my_cum, owner);
    const uint32_t s_f = __shfl_sync(0xffffffffu, my_f, owner);
    d.lower += scale * (uint64_t)s_cum;
    d.range = scale * (uint64_t)s_f;
    if (d.range < (1ull << 32)) {
        d.lower <<= 32;
        d.range <<= 32;
        d.point <<= 32;
        if (d.read_pos < d.end_pos) d.point |= words[d.read_pos];
        d.read_pos += 1;
    }
    return true;
}

__global__ void __launch_bounds__(256) k_decode_step(const int8_t *__restrict__ logits, const uint64_t *__restrict__ lut,
                                                     const uint32_t *__restrict__ words,
                                                     const int64_t *__restrict__ order,
                                                     const int64_t *__restrict__ tok_off, int64_t n_act, int64_t t,
                                                     DecState *__restrict__ st, uint8_t *__restrict__ tokens,
                                                     uint8_t *__restrict__ errors)
{
    __shared__ uint64_t lut_s[SC_VOCAB];
    for (int i = threadIdx.x; i < SC_VOCAB; i += blockDim.x) lut_s[i] = lut[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (i >= n_act) return;
    const int64_t c = order[i];
    if (errors[c]) return;
    DecState d = st[i];
    int sym;
    if (!warp_decode_step(logits + i * SC_VOCAB, lut_s, words, d, sym)) {
        if (lane == 0) errors[c] = 1;
        return;
    }
    if (lane == 0) {
        st[i] = d;
        tokens[tok_off[c] + t] = (uint8_t)sym;
    }
}

// The range decoder alone on given logits: one warp per stream, all of its steps in turn;
// step t of stream c takes logits row off[c] + t and writes symbols[off[c] + t].
__global__ void __launch_bounds__(256) k_decode_logits(const int8_t *__restrict__ logits,
                                                       const int64_t *__restrict__ off,
                                                       const uint32_t *__restrict__ words,
                                                       const int64_t *__restrict__ word_off, int64_t n,
                                                       const uint64_t *__restrict__ lut,
                                                       uint8_t *__restrict__ symbols, uint8_t *__restrict__ errors)
{
    __shared__ uint64_t lut_s[SC_VOCAB];
    for (int i = threadIdx.x; i < SC_VOCAB; i += blockDim.x) lut_s[i] = lut[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t c = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (c >= n) return;
    const int64_t b = off[c], len = off[c + 1] - b;
    DecState d;
    dec_init(d, words, word_off[c], word_off[c + 1]);
    uint8_t err = 0;
    for (int64_t t = 0; t < len; ++t) {
        int sym;
        if (!warp_decode_step(logits + (b + t) * SC_VOCAB, lut_s, words, d, sym)) {
            err = 1;
            break;
        }
        if (lane == 0) symbols[b + t] = (uint8_t)sym;
    }
    if (lane == 0) errors[c] = err;
}

inline unsigned blocks_for(int64_t n, int per) { return (unsigned)((n + per - 1) / per); }

}  // namespace

static bool use_tc(const sc_model *m) { return m->tc_ok && m->mlp_path != 2; }

void run_mlp(sc_model *m, const int16_t *windows, int64_t rows, int8_t *logits, cudaStream_t s)
{
    if (use_tc(m)) {
        L0Source src{};
        src.kind = 1;
        src.windows = windows;
        mlp_tc(m, src, rows, 0, logits, s);
    } else {
        mlp_simple(m, windows, rows, logits, s);
    }
}

// Maximum MLP rows per pass (bounds the activation workspaces).
static int64_t max_rows_per_pass(const sc_model *m) { return (int64_t)1 << 20; }

int compress_device(sc_model *m, const uint8_t *tokens, const int64_t *off_d, const int64_t *off_h, int64_t n,
                    uint32_t *words, int64_t words_capacity, int64_t *word_offsets, uint8_t *errors_d,
                    cudaStream_t s)
{
    const int64_t cap = (int64_t)m->chunk_len + 32;
    const int64_t max_rows = max_rows_per_pass(m);
    k_set_i64<<<1, 1, 0, s>>>(word_offsets, 0);
    count_launch();
    int *overflow = (int *)m->ws_misc.get(64, s);
    SC_CUDA(cudaMemsetAsync(overflow, 0, sizeof(int), s));
    std::vector<int32_t> tile_c, tile_t;
    int64_t c0 = 0;
    while (c0 < n) {
        // group of chunks whose rows fit one pass (a chunk never exceeds chunk_len rows)
        // one group for the fused kernels (they need no per-row intermediate beyond the
        // 8-byte (cum, freq) pair); otherwise groups whose rows fit the activation buffers
        const bool fused_path = use_tc(m) && fused_supported(m);
        const int64_t row_limit = fused_path ? ((int64_t)1 << 28) : max_rows;
        const int64_t chunk_limit = fused_path ? ((int64_t)1 << 20) : n;
        int64_t c1 = c0;
        while (c1 < n && (c1 == c0 || (off_h[c1 + 1] - off_h[c0] <= row_limit && c1 - c0 < chunk_limit))) ++c1;
        const int64_t gn = c1 - c0;
        const int64_t row_base = off_h[c0], rows = off_h[c1] - off_h[c0];
        int64_t max_len = 0;
        for (int64_t c = c0; c < c1; ++c) max_len = std::max(max_len, off_h[c + 1] - off_h[c]);
        int64_t *nw = (int64_t *)m->ws_nwords.get(sizeof(int64_t) * gn * 2, s);
        int64_t *incl = nw + gn;
        uint8_t *err = errors_d + c0;
        uint32_t *stage = (uint32_t *)m->ws_stage.get(sizeof(uint32_t) * gn * cap, s);
        uint2 *pairs = (uint2 *)m->ws_pairs.get(sizeof(uint2) * std::max<int64_t>(rows, 1), s);
        if (rows > 0) {
            const bool fused = use_tc(m) && fused_supported(m);
            int8_t *logits = fused ? nullptr : (int8_t *)m->ws_logits.get((size_t)rows * SC_VOCAB, s);
            if (use_tc(m)) {
                // 128-row tiles that never cross a chunk: layer 0 slides over each chunk's tokens
                tile_c.clear();
                tile_t.clear();
                for (int64_t c = c0; c < c1; ++c)
                    for (int64_t t0 = 0; t0 < off_h[c + 1] - off_h[c]; t0 += 128) {
                        tile_c.push_back((int32_t)c);
                        tile_t.push_back((int32_t)t0);
                    }
                const int64_t nt = (int64_t)tile_c.size();
                int32_t *d_tiles = (int32_t *)m->ws_windows.get(sizeof(int32_t) * 2 * nt, s);
                SC_CUDA(cudaMemcpyAsync(d_tiles, tile_c.data(), sizeof(int32_t) * nt, cudaMemcpyHostToDevice, s));
                SC_CUDA(cudaMemcpyAsync(d_tiles + nt, tile_t.data(), sizeof(int32_t) * nt, cudaMemcpyHostToDevice, s));
                if (fused) {
                    // all layers + (cum, freq) selection in one persistent launch
                    fused_compress(m, d_tiles, d_tiles + nt, nt, tokens, off_d, row_base, rows, pairs, s);
                } else {
                    L0Source src{};
                    src.kind = 3;
                    src.tokens = tokens;
                    src.tok_off = off_d;
                    src.tile_chunk = d_tiles;
                    src.tile_t0 = d_tiles + nt;
                    src.row_base = row_base;
                    mlp_tc(m, src, rows, nt, logits, s);
                }
                SC_CUDA(cudaStreamSynchronize(s));   // tile lists are reused by the next group
            } else {
                int16_t *win = (int16_t *)m->ws_windows.get(sizeof(int16_t) * rows * m->window, s);
                dim3 g((unsigned)gn, (unsigned)std::max<int64_t>(1, std::min<int64_t>((max_len + 127) / 128, 16)));
                {
                    ProfScope ps0(m->prof, KK_WINDOWS, s, rows);
                    k_windows_compress<<<g, 128, 0, s>>>(tokens, off_d, c0, row_base, m->window, win);
                    SC_LAUNCH_CHECK();
                    count_launch();
                }
                mlp_simple(m, win, rows, logits, s);
            }
            if (!fused) {
            ProfScope ps1(m->prof, KK_CDF, s, rows);
            k_cdf_select<<<(unsigned)std::min<int64_t>(blocks_for(rows, 8), 148 * 16), 256, 0, s>>>(
                logits, tokens + row_base, m->lut, rows, pairs);
            SC_LAUNCH_CHECK();
            count_launch();
            }
        }
        {
        ProfScope ps2(m->prof, KK_ENCODE, s, rows);
        k_encode<<<blocks_for(gn, 128), 128, 0, s>>>(pairs, off_d, c0, gn, row_base, stage, cap, nw, err);
        SC_LAUNCH_CHECK();
        count_launch();
        }
        ProfScope ps3(m->prof, KK_COMPACT, s, gn);
        size_t tmp_bytes = 0;
        SC_CUDA(cub::DeviceScan::InclusiveSum(nullptr, tmp_bytes, nw, incl, (int)gn, s));
        void *tmp = m->ws_scan.get(tmp_bytes, s);
        SC_CUDA(cub::DeviceScan::InclusiveSum(tmp, tmp_bytes, nw, incl, (int)gn, s));
        count_launch();
        k_compact<<<blocks_for(gn * 32, 256), 256, 0, s>>>(stage, cap, nw, incl, gn, c0, word_offsets, words,
                                                          words_capacity, overflow);
        SC_LAUNCH_CHECK();
        count_launch();
        c0 = c1;
    }
    int h_overflow = 0;
    SC_CUDA(cudaMemcpyAsync(&h_overflow, overflow, sizeof(int), cudaMemcpyDeviceToHost, s));
    SC_CUDA(cudaStreamSynchronize(s));
    if (h_overflow) {
        set_error("output words capacity %lld is too small", (long long)words_capacity);
        return 2;
    }
    return 0;
}

int decompress_device(sc_model *m, const uint32_t *words, const int64_t *word_offsets, const int64_t *lengths_d,
                      const int64_t *lengths_h, int64_t n, uint8_t *tokens, uint8_t *errors_d, cudaStream_t s)
{
    if (n <= 0) return 0;
    // order chunks by length, descending (counting sort; lengths are in [0, chunk_len])
    std::vector<int64_t> count(m->chunk_len + 2, 0);
    for (int64_t c = 0; c < n; ++c) count[lengths_h[c]]++;
    std::vector<int64_t> start(m->chunk_len + 2, 0);
    int64_t acc = 0;
    for (int64_t L = m->chunk_len; L >= 0; --L) { start[L] = acc; acc += count[L]; }
    std::vector<int64_t> order(n), sorted_len(n), tok_off(n + 1, 0);
    for (int64_t c = 0; c < n; ++c) {
        const int64_t k = start[lengths_h[c]]++;
        order[k] = c;
        sorted_len[k] = lengths_h[c];
        tok_off[c + 1] = tok_off[c] + lengths_h[c];
    }
    int64_t *order_d = (int64_t *)m->ws_order.get(sizeof(int64_t) * (2 * n + 1), s);
    int64_t *tok_off_d = order_d + n;
    SC_CUDA(cudaMemcpyAsync(order_d, order.data(), sizeof(int64_t) * n, cudaMemcpyHostToDevice, s));
    SC_CUDA(cudaMemcpyAsync(tok_off_d, tok_off.data(), sizeof(int64_t) * (n + 1), cudaMemcpyHostToDevice, s));
    DecState *st = (DecState *)m->ws_state.get(sizeof(DecState) * n, s);
    int *bad = (int *)m->ws_misc.get(64, s);
    SC_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), s));
    k_dec_init<<<blocks_for(n, 256), 256, 0, s>>>(words, word_offsets, lengths_d, order_d, n, st, errors_d, bad);
    SC_LAUNCH_CHECK();
    count_launch();
    int h_bad = 0;
    SC_CUDA(cudaMemcpyAsync(&h_bad, bad, sizeof(int), cudaMemcpyDeviceToHost, s));
    SC_CUDA(cudaStreamSynchronize(s));
    if (h_bad) {
        set_error("Invalid range-coded chunk for its token length");
        return 1;
    }
    if (use_tc(m) && fused_supported(m)) {
        // persistent decoding of every nonempty chunk (empty ones sort last)
        int64_t n_live = n;
        while (n_live > 0 && sorted_len[n_live - 1] == 0) --n_live;
        fused_decode(m, order_d, n_live, sorted_len.data(), lengths_d, st, words, tokens, tok_off_d, errors_d, s);
        SC_CUDA(cudaStreamSynchronize(s));
        return 0;
    }
    const int64_t max_rows = max_rows_per_pass(m);
    // process the ordered chunks in groups of at most max_rows concurrent chunks
    for (int64_t g0 = 0; g0 < n; g0 += max_rows) {
        const int64_t g1 = std::min(n, g0 + max_rows);
        const int64_t gmax = sorted_len[g0];
        int16_t *win = use_tc(m) ? nullptr
                                 : (int16_t *)m->ws_windows.get(sizeof(int16_t) * (g1 - g0) * m->window, s);
        int8_t *logits = (int8_t *)m->ws_logits.get((size_t)(g1 - g0) * SC_VOCAB, s);
        int64_t n_act = g1 - g0;
        for (int64_t t = 0; t < gmax; ++t) {
            while (n_act > 0 && sorted_len[g0 + n_act - 1] <= t) --n_act;
            if (use_tc(m)) {
                L0Source src{};
                src.kind = 2;
                src.tokens = tokens;
                src.order = order_d + g0;
                src.tok_off = tok_off_d;
                src.t = t;
                mlp_tc(m, src, n_act, 0, logits, s);
            } else {
                {
                    ProfScope ps4(m->prof, KK_WINDOWS, s, n_act);
                    k_windows_decode<<<blocks_for(n_act * m->window, 256), 256, 0, s>>>(
                        tokens, tok_off_d, order_d + g0, n_act, t, m->window, win);
                    SC_LAUNCH_CHECK();
                    count_launch();
                }
                mlp_simple(m, win, n_act, logits, s);
            }
            ProfScope ps5(m->prof, KK_DECODE, s, n_act);
            k_decode_step<<<blocks_for(n_act, 8), 256, 0, s>>>(logits, m->lut, words, order_d + g0, tok_off_d,
                                                               n_act, t, st + g0, tokens, errors_d);
            SC_LAUNCH_CHECK();
            count_launch();
        }
    }
    SC_CUDA(cudaStreamSynchronize(s));
    return 0;
}

// The range encoder alone on given logits (k_cdf_select -> k_encode -> scan -> k_compact):
// stream c codes symbols[off[c] .. off[c+1]) with the frequencies of the same logits rows.
int encode_logits_device(sc_model *m, const int8_t *logits, const uint8_t *symbols, const int64_t *off_d,
                         const int64_t *off_h, int64_t n, uint32_t *words, int64_t words_capacity,
                         int64_t *word_offsets, uint8_t *errors_d, cudaStream_t s)
{
    const int64_t cap = (int64_t)m->chunk_len + 32;
    const int64_t rows = off_h[n];
    k_set_i64<<<1, 1, 0, s>>>(word_offsets, 0);
    SC_LAUNCH_CHECK();
    count_launch();
    int *overflow = (int *)m->ws_misc.get(64, s);
    SC_CUDA(cudaMemsetAsync(overflow, 0, sizeof(int), s));
    int64_t *nw = (int64_t *)m->ws_nwords.get(sizeof(int64_t) * n * 2, s);
    int64_t *incl = nw + n;
    uint32_t *stage = (uint32_t *)m->ws_stage.get(sizeof(uint32_t) * n * cap, s);
    uint2 *pairs = (uint2 *)m->ws_pairs.get(sizeof(uint2) * std::max<int64_t>(rows, 1), s);
    if (rows > 0) {
        k_cdf_select<<<(unsigned)std::min<int64_t>(blocks_for(rows, 8), 148 * 16), 256, 0, s>>>(logits, symbols,
                                                                                                 m->lut, rows, pairs);
        SC_LAUNCH_CHECK();
        count_launch();
    }
    k_encode<<<blocks_for(n, 128), 128, 0, s>>>(pairs, off_d, 0, n, 0, stage, cap, nw, errors_d);
    SC_LAUNCH_CHECK();
    count_launch();
    size_t tmp_bytes = 0;
    SC_CUDA(cub::DeviceScan::InclusiveSum(nullptr, tmp_bytes, nw, incl, (int)n, s));
    void *tmp = m->ws_scan.get(tmp_bytes, s);
    SC_CUDA(cub::DeviceScan::InclusiveSum(tmp, tmp_bytes, nw, incl, (int)n, s));
    count_launch();
    k_compact<<<blocks_for(n * 32, 256), 256, 0, s>>>(stage, cap, nw, incl, n, 0, word_offsets, words,
                                                      words_capacity, overflow);
    SC_LAUNCH_CHECK();
    count_launch();
    int h_overflow = 0;
    SC_CUDA(cudaMemcpyAsync(&h_overflow, overflow, sizeof(int), cudaMemcpyDeviceToHost, s));
    SC_CUDA(cudaStreamSynchronize(s));
    if (h_overflow) {
        set_error("output words capacity %lld is too small", (long long)words_capacity);
        return 2;
    }
    return 0;
}

// The range decoder alone on given logits (k_decode_logits).
void decode_logits_device(sc_model *m, const int8_t *logits, const int64_t *off_d, int64_t n, const uint32_t *words,
                          const int64_t *word_offsets, uint8_t *symbols, uint8_t *errors_d, cudaStream_t s)
{
    k_decode_logits<<<blocks_for(n, 8), 256, 0, s>>>(logits, off_d, words, word_offsets, n, m->lut, symbols,
                                                     errors_d);
    SC_LAUNCH_CHECK();
    count_launch();
    SC_CUDA(cudaStreamSynchronize(s));
}

}  // namespace sc
