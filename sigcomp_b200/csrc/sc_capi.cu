// extern "C" boundary of libsigcomp_b200 (declared in include/sigcomp_b200.h).
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstring>
#include <memory>
#include <new>

#include "../../include/sigcomp_b200.h"
#include "sc_internal.h"

namespace sc {

static thread_local char g_err[512] = "";
static std::atomic<int64_t> g_launches{0};

void set_error(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void count_launch(int64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int compress_device(sc_model *m, const uint8_t *tokens, const int64_t *off_d, const int64_t *off_h, int64_t n,
                    uint32_t *words, int64_t words_capacity, int64_t *word_offsets, uint8_t *errors_d,
                    cudaStream_t s);
int decompress_device(sc_model *m, const uint32_t *words, const int64_t *word_offsets, const int64_t *lengths_d,
                      const int64_t *lengths_h, int64_t n, uint8_t *tokens, uint8_t *errors_d, cudaStream_t s);
void run_mlp(sc_model *m, const int16_t *windows, int64_t rows, int8_t *logits, cudaStream_t s);
int split_signal_device(sc_model *m, const int16_t *samples, const int64_t *off_d, const int64_t *off_h,
                        int64_t n_reads, int lsb, int16_t *sig0, uint8_t *small, int64_t *small_off,
                        uint16_t *large, uint32_t *large_pos, int64_t *large_off, cudaStream_t s);
int wait_selftest(cudaStream_t s, int *done_d);
int encode_logits_device(sc_model *m, const int8_t *logits, const uint8_t *symbols, const int64_t *off_d,
                         const int64_t *off_h, int64_t n, uint32_t *words, int64_t words_capacity,
                         int64_t *word_offsets, uint8_t *errors_d, cudaStream_t s);
void decode_logits_device(sc_model *m, const int8_t *logits, const int64_t *off_d, int64_t n, const uint32_t *words,
                          const int64_t *word_offsets, uint8_t *symbols, uint8_t *errors_d, cudaStream_t s);
int reassemble_signal_device(sc_model *m, const int16_t *sig0, const int64_t *off_d, const int64_t *off_h,
                             int64_t n_reads, int lsb,
                             const uint8_t *small, const int64_t *small_off, const uint16_t *large,
                             const uint32_t *large_pos, const int64_t *large_off, int16_t *samples,
                             cudaStream_t s);

namespace {

// Makes the model's device current for one call and restores the caller's device after it.
// `err` records a failed switch; guarded() turns it into an error before any launch, so a call
// never runs on another device with this model's pointers.
struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) err = cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int map_cuda(const CudaError &e)
{
    set_error("CUDA error %s (%s) in %s", cudaGetErrorName(e.code), cudaGetErrorString(e.code), e.where.c_str());
    return e.code == cudaErrorMemoryAllocation ? SC_ERR_OUT_OF_MEMORY : SC_ERR_CUDA;
}

template <typename F>
int guarded(sc_model *m, F &&f)
{
    try {
        DeviceGuard g(m->device);
        SC_CUDA(g.err);
        int rc = f();
        if (m->prof.on) {
            SC_CUDA(cudaDeviceSynchronize());
            m->prof.collect();
        }
        if (read_device_error(1)) {
            set_error("a device-side wait timed out (kernel gave up after its time limit)");
            return SC_ERR_CUDA;
        }
        return rc;
    } catch (const CudaError &e) {
        return map_cuda(e);
    } catch (const std::bad_alloc &) {
        set_error("host out of memory");
        return SC_ERR_OUT_OF_MEMORY;
    } catch (...) {
        set_error("internal error");
        return SC_ERR_CUDA;
    }
}

// validate chunk offsets on the host; returns SC_OK or sets the error
int check_offsets(const sc_model *m, const int64_t *off, int64_t n)
{
    if (off[0] != 0) {
        set_error("token_offsets[0] must be 0");
        return SC_ERR_INVALID_ARGUMENT;
    }
    for (int64_t c = 0; c < n; ++c) {
        const int64_t len = off[c + 1] - off[c];
        if (len < 0) {
            set_error("token_offsets must be nondecreasing");
            return SC_ERR_INVALID_ARGUMENT;
        }
        if (len > m->chunk_len) {
            set_error("A token chunk exceeds chunk_len");
            return SC_ERR_INVALID_ARGUMENT;
        }
    }
    return SC_OK;
}

// Automatic selection (path 0) runs only the tcgen05 kernels: the fused pair kernels for
// compress/decompress and the tcgen05 layer kernels for the logits entry point.  A model
// whose geometry they do not cover is refused with SC_ERR_UNSUPPORTED instead of being run
// on another implementation; the other implementations run only when a caller selects them
// with sc_model_set_mlp_path (cross-checks in the tests).
int check_auto_path(const sc_model *m, bool fused)
{
    if (m->mlp_path != 0) return SC_OK;
    if (!m->tc_ok || (fused && !fused_supported(m))) {
        set_error("model geometry not supported by the tcgen05 kernels (window 64, emb_dim 128, layer widths "
                  "multiples of 256 up to 512, at most 9 layers)");
        return SC_ERR_UNSUPPORTED;
    }
    return SC_OK;
}

int first_error(const uint8_t *errs, int64_t n)
{
    for (int64_t c = 0; c < n; ++c)
        if (errs[c]) return (int)c;
    return -1;
}

}  // namespace
}  // namespace sc

using namespace sc;

extern "C" {

const char *sc_version(void) { return "sigcomp_b200 0.1.0 (sm_100a)"; }

const char *sc_last_error(void) { return g_err; }

int64_t sc_kernel_launches(void) { return g_launches.load(); }

int sc_model_create(int device, int32_t window, int32_t emb_dim, int32_t num_layers, const int8_t *embedding,
                    const int32_t *in_dims, const int32_t *out_dims, const int8_t *const *weights,
                    const int32_t *const *biases, const int64_t *multipliers, const int32_t *shifts,
                    const uint8_t *relu, const int64_t *exp_lut, int32_t chunk_len, sc_model **out)
{
    g_err[0] = 0;
    if (!out || !embedding || !in_dims || !out_dims || !weights || !biases || !multipliers || !shifts || !relu ||
        !exp_lut) {
        set_error("null argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    if (window < 1 || emb_dim < 16 || emb_dim % 16 || num_layers < 1 || chunk_len < 1 || chunk_len > 65535) {
        set_error("unsupported geometry: window=%d emb_dim=%d layers=%d chunk_len=%d", window, emb_dim, num_layers,
                  chunk_len);
        return SC_ERR_UNSUPPORTED;
    }
    if (in_dims[0] != window * emb_dim || out_dims[num_layers - 1] != SC_VOCAB) {
        set_error("layer 0 must take window*emb_dim inputs and the last layer must emit 256 logits");
        return SC_ERR_INVALID_ARGUMENT;
    }
    for (int l = 0; l < num_layers; ++l) {
        if (in_dims[l] % 64 || out_dims[l] % 64 || (l > 0 && in_dims[l] != out_dims[l - 1])) {
            set_error("unsupported layer %d shape %dx%d", l, out_dims[l], in_dims[l]);
            return SC_ERR_UNSUPPORTED;
        }
        if (multipliers[l] < 0 || multipliers[l] > (1ll << 31) || shifts[l] < 0 || shifts[l] > 63) {
            set_error("layer %d multiplier/shift out of range", l);
            return SC_ERR_INVALID_ARGUMENT;
        }
    }
    // exact-division preconditions: lut[0] = 2^38 and 0 <= lut[i] <= 2^38
    if (exp_lut[0] != (int64_t)SC_LUT_ONE) {
        set_error("exp_lut[0] must be 2**38 (build_integer_exp_lut)");
        return SC_ERR_INVALID_ARGUMENT;
    }
    for (int i = 0; i < SC_VOCAB; ++i)
        if (exp_lut[i] < 0 || exp_lut[i] > (int64_t)SC_LUT_ONE) {
            set_error("exp_lut must be nonnegative and at most 2**38");
            return SC_ERR_INVALID_ARGUMENT;
        }
    std::unique_ptr<sc_model> m(new (std::nothrow) sc_model());
    if (!m) {
        set_error("host out of memory");
        return SC_ERR_OUT_OF_MEMORY;
    }
    m->device = device;
    m->window = window;
    m->emb_dim = emb_dim;
    m->num_layers = num_layers;
    m->chunk_len = chunk_len;
    int rc = guarded(m.get(), [&]() -> int {
        int ndev = 0;
        SC_CUDA(cudaGetDeviceCount(&ndev));
        if (device < 0 || device >= ndev) {
            set_error("device %d not present (%d devices)", device, ndev);
            return SC_ERR_INVALID_ARGUMENT;
        }
        cudaDeviceProp prop;
        SC_CUDA(cudaGetDeviceProperties(&prop, device));
        if (prop.major != 10) {
            set_error("sigcomp_b200 requires an sm_100 (B200) GPU, found sm_%d%d", prop.major, prop.minor);
            return SC_ERR_UNSUPPORTED;
        }
        const size_t eb = (size_t)(SC_SOS + 1) * emb_dim;
        SC_CUDA(cudaMalloc(&m->emb, eb));
        SC_CUDA(cudaMemcpy(m->emb, embedding, eb, cudaMemcpyHostToDevice));
        SC_CUDA(cudaMalloc(&m->lut, sizeof(uint64_t) * SC_VOCAB));
        SC_CUDA(cudaMemcpy(m->lut, exp_lut, sizeof(uint64_t) * SC_VOCAB, cudaMemcpyHostToDevice));
        m->layers.resize(num_layers);
        for (int l = 0; l < num_layers; ++l) {
            LayerDev &L = m->layers[l];
            L.in_dim = in_dims[l];
            L.out_dim = out_dims[l];
            L.rq = make_requant(multipliers[l], shifts[l], relu[l]);
            const size_t wb = (size_t)L.in_dim * L.out_dim;
            SC_CUDA(cudaMalloc(&L.w, wb));
            SC_CUDA(cudaMemcpy(L.w, weights[l], wb, cudaMemcpyHostToDevice));
            SC_CUDA(cudaMalloc(&L.bias, sizeof(int32_t) * L.out_dim));
            SC_CUDA(cudaMemcpy(L.bias, biases[l], sizeof(int32_t) * L.out_dim, cudaMemcpyHostToDevice));
            // the pair kernels add the bias of layers >= 1 with an MMA (fast requantisation only)
            const std::vector<int8_t> bt = l > 0 && L.rq.hi_path ? bias_tile(biases[l], L.out_dim)
                                                                   : std::vector<int8_t>();
            if (!bt.empty()) {
                SC_CUDA(cudaMalloc(&L.bdig, bt.size()));
                SC_CUDA(cudaMemcpy(L.bdig, bt.data(), bt.size(), cudaMemcpyHostToDevice));
            }
        }
        m->tc_ok = mlp_tc_supported(m.get());
        if (m->tc_ok) mlp_tc_prepare(m.get());
        SC_CUDA(cudaDeviceSynchronize());
        return SC_OK;
    });
    if (rc != SC_OK) {
        sc_model_destroy(m.release());
        return rc;
    }
    *out = m.release();
    return SC_OK;
}

int sc_model_destroy(sc_model *m)
{
    if (!m) return SC_OK;
    {
        DeviceGuard g(m->device);
        cudaDeviceSynchronize();
        cudaFree(m->emb);
        cudaFree(m->lut);
        cudaFree(m->trace_buf);
        cudaFree(m->trace_count);
        for (auto &L : m->layers) {
            cudaFree(L.w);
            cudaFree(L.w_tc);
            cudaFree(L.bias);
            cudaFree(L.bdig);
        }
        for (DevBuf *b : {&m->ws_windows, &m->ws_act0, &m->ws_act1, &m->ws_logits, &m->ws_pairs, &m->ws_stage,
                          &m->ws_nwords, &m->ws_err, &m->ws_scan, &m->ws_tmp, &m->ws_order, &m->ws_state,
                          &m->ws_tok_off, &m->ws_misc, &m->ws_ering, &m->ws_sched})
            b->release();
    }
    delete m;
    return SC_OK;
}

int sc_model_set_mlp_path(sc_model *m, int32_t path)
{
    if (!m || path < 0 || path > 5) {
        set_error("invalid model or path");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if ((path == 1 || path >= 3) && !m->tc_ok) {
        set_error("tcgen05 MLP path is not available for this model geometry");
        return SC_ERR_UNSUPPORTED;
    }
    m->mlp_path = path;
    return SC_OK;
}

int sc_compress_chunks(sc_model *m, const uint8_t *tokens, const int64_t *token_offsets, int64_t n_chunks,
                       uint32_t *words, int64_t words_capacity, int64_t *word_offsets, uint8_t *chunk_errors,
                       void *stream)
{
    g_err[0] = 0;
    if (!m || n_chunks < 0 || (n_chunks > 0 && (!token_offsets || !words || !word_offsets))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (n_chunks == 0) {
        if (word_offsets) word_offsets[0] = 0;
        return SC_OK;
    }
    int rc = check_offsets(m, token_offsets, n_chunks);
    if (rc) return rc;
    if ((rc = check_auto_path(m, true))) return rc;
    if (token_offsets[n_chunks] > 0 && !tokens) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        const int64_t n_tok = token_offsets[n_chunks];
        uint8_t *d_tok = (uint8_t *)m->ws_tmp.get((size_t)std::max<int64_t>(n_tok, 1) + 16, s);
        int64_t *d_off = (int64_t *)m->ws_tok_off.get(sizeof(int64_t) * (2 * (n_chunks + 1)), s);
        int64_t *d_woff = d_off + n_chunks + 1;
        uint32_t *d_words = (uint32_t *)m->ws_err.get(sizeof(uint32_t) * std::max<int64_t>(words_capacity, 1) + n_chunks + 16, s);
        uint8_t *d_err = (uint8_t *)(d_words + std::max<int64_t>(words_capacity, 1));
        if (n_tok) SC_CUDA(cudaMemcpyAsync(d_tok, tokens, (size_t)n_tok, cudaMemcpyHostToDevice, s));
        SC_CUDA(cudaMemcpyAsync(d_off, token_offsets, sizeof(int64_t) * (n_chunks + 1), cudaMemcpyHostToDevice, s));
        int r = compress_device(m, d_tok, d_off, token_offsets, n_chunks, d_words, words_capacity, d_woff, d_err, s);
        if (r == 2) return SC_ERR_CAPACITY;
        SC_CUDA(cudaMemcpyAsync(word_offsets, d_woff, sizeof(int64_t) * (n_chunks + 1), cudaMemcpyDeviceToHost, s));
        std::vector<uint8_t> errs(n_chunks);
        SC_CUDA(cudaMemcpyAsync(errs.data(), d_err, (size_t)n_chunks, cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        const int64_t total = word_offsets[n_chunks];
        if (total) SC_CUDA(cudaMemcpyAsync(words, d_words, sizeof(uint32_t) * total, cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        if (chunk_errors) memcpy(chunk_errors, errs.data(), (size_t)n_chunks);
        const int bad = first_error(errs.data(), n_chunks);
        if (bad >= 0) {
            set_error("range-coder output capacity exceeded in stream %d; increase max_words", bad);
            return SC_ERR_CAPACITY;
        }
        return SC_OK;
    });
}

int sc_compress_chunks_device(sc_model *m, const uint8_t *tokens, const int64_t *token_offsets, int64_t n_chunks,
                              uint32_t *words, int64_t words_capacity, int64_t *word_offsets, uint8_t *chunk_errors,
                              void *stream)
{
    g_err[0] = 0;
    if (!m || n_chunks < 0 || (n_chunks > 0 && (!token_offsets || !words || !word_offsets))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (int rc = check_auto_path(m, true)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        std::vector<int64_t> off_h(n_chunks + 1);
        SC_CUDA(cudaMemcpyAsync(off_h.data(), token_offsets, sizeof(int64_t) * (n_chunks + 1), cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        int rc = check_offsets(m, off_h.data(), n_chunks);
        if (rc) return rc;
        uint8_t *d_err = chunk_errors ? chunk_errors : (uint8_t *)m->ws_tmp.get((size_t)n_chunks + 16, s);
        int r = compress_device(m, tokens, token_offsets, off_h.data(), n_chunks, words, words_capacity,
                                word_offsets, d_err, s);
        if (r == 2) return SC_ERR_CAPACITY;
        std::vector<uint8_t> errs(n_chunks);
        if (n_chunks) SC_CUDA(cudaMemcpyAsync(errs.data(), d_err, (size_t)n_chunks, cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        const int bad = first_error(errs.data(), n_chunks);
        if (bad >= 0) {
            set_error("range-coder output capacity exceeded in stream %d; increase max_words", bad);
            return SC_ERR_CAPACITY;
        }
        return SC_OK;
    });
}

int sc_decompress_chunks(sc_model *m, const uint32_t *words, const int64_t *word_offsets, const int64_t *lengths,
                         int64_t n_chunks, uint8_t *tokens, uint8_t *chunk_errors, void *stream)
{
    g_err[0] = 0;
    if (!m || n_chunks < 0 || (n_chunks > 0 && (!word_offsets || !lengths))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (n_chunks == 0) return SC_OK;
    int64_t n_tok = 0;
    if (word_offsets[0] != 0) {
        set_error("word_offsets[0] must be 0");
        return SC_ERR_INVALID_ARGUMENT;
    }
    for (int64_t c = 0; c < n_chunks; ++c) {
        if (lengths[c] < 0 || lengths[c] > m->chunk_len) {
            set_error("Chunk lengths must be integers in [0, chunk_len]");
            return SC_ERR_INVALID_ARGUMENT;
        }
        const int64_t nw = word_offsets[c + 1] - word_offsets[c];
        if (nw < 0 || (lengths[c] > 0) != (nw > 0)) {
            set_error("Invalid range-coded chunk for its token length");
            return SC_ERR_INVALID_ARGUMENT;
        }
        n_tok += lengths[c];
    }
    if ((n_tok > 0 && !tokens) || (word_offsets[n_chunks] > 0 && !words)) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (int rc = check_auto_path(m, true)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        const int64_t n_words = word_offsets[n_chunks];
        uint32_t *d_words = (uint32_t *)m->ws_tmp.get(sizeof(uint32_t) * std::max<int64_t>(n_words, 1), s);
        int64_t *d_woff = (int64_t *)m->ws_tok_off.get(sizeof(int64_t) * (2 * n_chunks + 1), s);
        int64_t *d_len = d_woff + n_chunks + 1;
        uint8_t *d_tok = (uint8_t *)m->ws_err.get((size_t)std::max<int64_t>(n_tok, 1) + n_chunks + 16, s);
        uint8_t *d_err = d_tok + std::max<int64_t>(n_tok, 1);
        if (n_words) SC_CUDA(cudaMemcpyAsync(d_words, words, sizeof(uint32_t) * n_words, cudaMemcpyHostToDevice, s));
        SC_CUDA(cudaMemcpyAsync(d_woff, word_offsets, sizeof(int64_t) * (n_chunks + 1), cudaMemcpyHostToDevice, s));
        SC_CUDA(cudaMemcpyAsync(d_len, lengths, sizeof(int64_t) * n_chunks, cudaMemcpyHostToDevice, s));
        int r = decompress_device(m, d_words, d_woff, d_len, lengths, n_chunks, d_tok, d_err, s);
        if (r == 1) return SC_ERR_INVALID_ARGUMENT;
        std::vector<uint8_t> errs(n_chunks);
        SC_CUDA(cudaMemcpyAsync(errs.data(), d_err, (size_t)n_chunks, cudaMemcpyDeviceToHost, s));
        if (n_tok) SC_CUDA(cudaMemcpyAsync(tokens, d_tok, (size_t)n_tok, cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        if (chunk_errors) memcpy(chunk_errors, errs.data(), (size_t)n_chunks);
        const int bad = first_error(errs.data(), n_chunks);
        if (bad >= 0) {
            set_error("invalid range stream or mismatching entropy model in stream %d", bad);
            return SC_ERR_CORRUPT_STREAM;
        }
        return SC_OK;
    });
}

int sc_decompress_chunks_device(sc_model *m, const uint32_t *words, const int64_t *word_offsets,
                                const int64_t *lengths, const int64_t *lengths_host, int64_t n_chunks,
                                uint8_t *tokens, uint8_t *chunk_errors, void *stream)
{
    g_err[0] = 0;
    if (!m || n_chunks < 0 || (n_chunks > 0 && (!word_offsets || !lengths || !lengths_host))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (n_chunks == 0) return SC_OK;
    for (int64_t c = 0; c < n_chunks; ++c)
        if (lengths_host[c] < 0 || lengths_host[c] > m->chunk_len) {
            set_error("Chunk lengths must be integers in [0, chunk_len]");
            return SC_ERR_INVALID_ARGUMENT;
        }
    if (int rc = check_auto_path(m, true)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        uint8_t *d_err = chunk_errors ? chunk_errors : (uint8_t *)m->ws_err.get((size_t)n_chunks + 16, s);
        int r = decompress_device(m, words, word_offsets, lengths, lengths_host, n_chunks, tokens, d_err, s);
        if (r == 1) return SC_ERR_INVALID_ARGUMENT;
        std::vector<uint8_t> errs(n_chunks);
        SC_CUDA(cudaMemcpyAsync(errs.data(), d_err, (size_t)n_chunks, cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        const int bad = first_error(errs.data(), n_chunks);
        if (bad >= 0) {
            set_error("invalid range stream or mismatching entropy model in stream %d", bad);
            return SC_ERR_CORRUPT_STREAM;
        }
        return SC_OK;
    });
}

int sc_profile_enable(sc_model *m, int32_t enable)
{
    if (!m) {
        set_error("invalid model");
        return SC_ERR_INVALID_ARGUMENT;
    }
    m->prof.on = enable != 0;
    m->prof.reset();
    return SC_OK;
}

int sc_profile_read(sc_model *m, int32_t kind, double *total_ms, int64_t *launches, int64_t *work)
{
    if (!m || kind < 0 || kind >= KK_KINDS) {
        set_error("invalid model or kernel kind");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (total_ms) *total_ms = m->prof.ms[kind];
    if (launches) *launches = m->prof.launches[kind];
    if (work) *work = m->prof.work[kind];
    return SC_OK;
}

int sc_trace_enable(sc_model *m, int32_t records_per_cta)
{
    if (!m || records_per_cta < 0) {
        set_error("invalid model or record count");
        return SC_ERR_INVALID_ARGUMENT;
    }
    return guarded(m, [&]() -> int {
        cudaFree(m->trace_buf);
        cudaFree(m->trace_count);
        m->trace_buf = nullptr;
        m->trace_count = nullptr;
        m->trace_cap = 0;
        if (records_per_cta > 0) {
            SC_CUDA(cudaMalloc(&m->trace_buf, sizeof(unsigned long long) * 2 * 2 * (size_t)records_per_cta));
            SC_CUDA(cudaMalloc(&m->trace_count, 8 * sizeof(unsigned int)));
            SC_CUDA(cudaMemset(m->trace_count, 0, 8 * sizeof(unsigned int)));
            m->trace_cap = records_per_cta;
        }
        return SC_OK;
    });
}

int64_t sc_trace_read(sc_model *m, int32_t cta, uint64_t *records, int64_t capacity)
{
    if (!m || cta < 0 || cta > 1 || !m->trace_buf) return 0;
    int64_t n = 0;
    int rc = guarded(m, [&]() -> int {
        // per role, the records it wrote (a role's region holds trace_cap / 4 of them)
        unsigned int cnt[8] = {};
        SC_CUDA(cudaMemcpy(cnt, m->trace_count, sizeof(cnt), cudaMemcpyDeviceToHost));
        const int64_t per_role = m->trace_cap / 4;
        for (int role = 0; role < 4 && n < capacity; ++role) {
            const int64_t k = std::min<int64_t>(std::min<int64_t>(cnt[cta * 4 + role], per_role), capacity - n);
            if (k > 0)
                SC_CUDA(cudaMemcpy(records + 2 * n, m->trace_buf + ((size_t)cta * 4 + role) * per_role * 2,
                                   sizeof(uint64_t) * 2 * k, cudaMemcpyDeviceToHost));
            n += k;
        }
        return SC_OK;
    });
    return rc == SC_OK ? n : -1;
}

int sc_selftest_wait_timeout(sc_model *m, void *stream)
{
    g_err[0] = 0;
    if (!m) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        int *done = (int *)m->ws_misc.get(64, s);
        SC_CUDA(cudaMemsetAsync(done, 0, sizeof(int), s));
        const int r = wait_selftest(s, done);
        if (r != 4) {                    // the kernel must end, with both waits timed out
            set_error("wait self test: unexpected result %d", r);
            return SC_ERR_CUDA;
        }
        return SC_OK;                    // guarded() reports the recorded timeout
    });
}

// read offsets of a signal call: nondecreasing, every read at least one sample
static int check_read_offsets(const int64_t *off, int64_t n)
{
    if (off[0] != 0) {
        set_error("sample_offsets[0] must be 0");
        return SC_ERR_INVALID_ARGUMENT;
    }
    for (int64_t r = 0; r < n; ++r)
        if (off[r + 1] - off[r] < 1) {
            set_error("read %lld has no samples", (long long)r);
            return SC_ERR_INVALID_ARGUMENT;
        }
    return SC_OK;
}

int sc_split_signal_device(sc_model *m, const int16_t *samples, const int64_t *sample_offsets, int64_t n_reads,
                           int32_t lsb, int16_t *sig0, uint8_t *tokens, int64_t *token_offsets, uint16_t *large,
                           uint32_t *large_pos, int64_t *large_offsets, void *stream)
{
    g_err[0] = 0;
    if (!m || n_reads < 0 || lsb < 0 || lsb > 15 || !sample_offsets || !token_offsets || !large_offsets ||
        (n_reads > 0 && (!samples || !sig0 || !tokens || !large || !large_pos))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        std::vector<int64_t> off_h(n_reads + 1);
        SC_CUDA(cudaMemcpyAsync(off_h.data(), sample_offsets, sizeof(int64_t) * (n_reads + 1),
                                cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        int rc = check_read_offsets(off_h.data(), n_reads);
        if (rc) return rc;
        split_signal_device(m, samples, sample_offsets, off_h.data(), n_reads, lsb, sig0, tokens, token_offsets,
                            large, large_pos, large_offsets, s);
        SC_CUDA(cudaStreamSynchronize(s));
        return SC_OK;
    });
}

int sc_reassemble_signal_device(sc_model *m, const int16_t *sig0, const int64_t *sample_offsets, int64_t n_reads,
                                int32_t lsb, const uint8_t *tokens, const int64_t *token_offsets,
                                const uint16_t *large, const uint32_t *large_pos, const int64_t *large_offsets,
                                int16_t *samples, void *stream)
{
    g_err[0] = 0;
    if (!m || n_reads < 0 || lsb < 0 || lsb > 15 || !sample_offsets || !token_offsets || !large_offsets ||
        (n_reads > 0 && (!sig0 || !samples))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        std::vector<int64_t> off_h(n_reads + 1);
        SC_CUDA(cudaMemcpyAsync(off_h.data(), sample_offsets, sizeof(int64_t) * (n_reads + 1),
                                cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        int rc = check_read_offsets(off_h.data(), n_reads);
        if (rc) return rc;
        if (reassemble_signal_device(m, sig0, sample_offsets, off_h.data(), n_reads, lsb, tokens, token_offsets,
                                     large, large_pos,
                                     large_offsets, samples, s)) {
            set_error("token and large-value streams do not match the read lengths");
            return SC_ERR_INVALID_ARGUMENT;
        }
        return SC_OK;
    });
}

int sc_mlp_logits_device(sc_model *m, const int16_t *windows, int64_t rows, int8_t *logits, void *stream)
{
    g_err[0] = 0;
    if (!m || rows < 0 || (rows > 0 && (!windows || !logits))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (int rc = check_auto_path(m, false)) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        run_mlp(m, windows, rows, logits, s);
        SC_CUDA(cudaStreamSynchronize(s));
        return SC_OK;
    });
}

int sc_encode_logits_device(sc_model *m, const int8_t *logits, const uint8_t *symbols, const int64_t *offsets,
                            int64_t n_streams, uint32_t *words, int64_t words_capacity, int64_t *word_offsets,
                            uint8_t *stream_errors, void *stream)
{
    g_err[0] = 0;
    if (!m || n_streams < 0 || (n_streams > 0 && (!offsets || !words || !word_offsets))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        std::vector<int64_t> off_h(n_streams + 1);
        SC_CUDA(cudaMemcpyAsync(off_h.data(), offsets, sizeof(int64_t) * (n_streams + 1), cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        int rc = check_offsets(m, off_h.data(), n_streams);
        if (rc) return rc;
        if (off_h[n_streams] > 0 && (!logits || !symbols)) {
            set_error("invalid argument");
            return SC_ERR_INVALID_ARGUMENT;
        }
        if (n_streams == 0) {
            const int64_t zero = 0;
            SC_CUDA(cudaMemcpyAsync(word_offsets, &zero, sizeof(zero), cudaMemcpyHostToDevice, s));
            SC_CUDA(cudaStreamSynchronize(s));
            return SC_OK;
        }
        uint8_t *d_err = stream_errors ? stream_errors : (uint8_t *)m->ws_tmp.get((size_t)n_streams + 16, s);
        int r = encode_logits_device(m, logits, symbols, offsets, off_h.data(), n_streams, words, words_capacity,
                                     word_offsets, d_err, s);
        if (r == 2) return SC_ERR_CAPACITY;
        std::vector<uint8_t> errs(n_streams);
        SC_CUDA(cudaMemcpyAsync(errs.data(), d_err, (size_t)n_streams, cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        const int bad = first_error(errs.data(), n_streams);
        if (bad >= 0) {
            set_error("range-coder output capacity exceeded in stream %d; increase max_words", bad);
            return SC_ERR_CAPACITY;
        }
        return SC_OK;
    });
}

int sc_decode_logits_device(sc_model *m, const int8_t *logits, const int64_t *offsets, const uint32_t *words,
                            const int64_t *word_offsets, int64_t n_streams, uint8_t *symbols,
                            uint8_t *stream_errors, void *stream)
{
    g_err[0] = 0;
    if (!m || n_streams < 0 || (n_streams > 0 && (!offsets || !word_offsets))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (n_streams == 0) return SC_OK;
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        std::vector<int64_t> off_h(n_streams + 1), woff_h(n_streams + 1);
        SC_CUDA(cudaMemcpyAsync(off_h.data(), offsets, sizeof(int64_t) * (n_streams + 1), cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaMemcpyAsync(woff_h.data(), word_offsets, sizeof(int64_t) * (n_streams + 1),
                                cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        if (off_h[0] != 0) {
            set_error("offsets[0] must be 0");
            return SC_ERR_INVALID_ARGUMENT;
        }
        for (int64_t c = 0; c < n_streams; ++c) {
            const int64_t len = off_h[c + 1] - off_h[c], nw = woff_h[c + 1] - woff_h[c];
            if (len < 0 || nw < 0 || (len > 0) != (nw > 0)) {
                set_error("Invalid range-coded chunk for its token length");
                return SC_ERR_INVALID_ARGUMENT;
            }
        }
        if ((off_h[n_streams] > 0 && (!logits || !symbols)) || (woff_h[n_streams] > 0 && !words)) {
            set_error("invalid argument");
            return SC_ERR_INVALID_ARGUMENT;
        }
        uint8_t *d_err = stream_errors ? stream_errors : (uint8_t *)m->ws_tmp.get((size_t)n_streams + 16, s);
        decode_logits_device(m, logits, offsets, n_streams, words, word_offsets, symbols, d_err, s);
        std::vector<uint8_t> errs(n_streams);
        SC_CUDA(cudaMemcpyAsync(errs.data(), d_err, (size_t)n_streams, cudaMemcpyDeviceToHost, s));
        SC_CUDA(cudaStreamSynchronize(s));
        const int bad = first_error(errs.data(), n_streams);
        if (bad >= 0) {
            set_error("invalid range stream or mismatching entropy model in stream %d", bad);
            return SC_ERR_CORRUPT_STREAM;
        }
        return SC_OK;
    });
}

int sc_linear_layer_device(sc_model *m, int32_t layer, const int8_t *x, int64_t rows, int8_t *y, void *stream)
{
    g_err[0] = 0;
    if (!m || layer < 0 || layer >= m->num_layers || rows < 0 || (rows > 0 && (!x || !y))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (!m->tc_ok) {
        set_error("model geometry not supported by the tcgen05 kernels");
        return SC_ERR_UNSUPPORTED;
    }
    if (((uintptr_t)x & 15) != 0) {
        set_error("x must be 16-byte aligned");
        return SC_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    return guarded(m, [&]() -> int {
        linear_tc(m, layer, x, rows, y, s);
        SC_CUDA(cudaStreamSynchronize(s));
        return SC_OK;
    });
}

}  // extern "C"
