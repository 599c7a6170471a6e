// Internal declarations shared by the sigcomp_b200 translation units.
#pragma once

#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>
#include <cuda.h>
#include <cuda_runtime.h>

#include "sc_common.cuh"

struct sc_model;

namespace sc {

// Thread-local error message used by sc_last_error().
void set_error(const char *fmt, ...);
void count_launch(int64_t n = 1);

struct CudaError {
    cudaError_t code;
    std::string where;
};

#define SC_CUDA(call)                                                              \
    do {                                                                           \
        cudaError_t _e = (call);                                                   \
        if (_e != cudaSuccess) throw ::sc::CudaError{_e, std::string(#call) + " at " + \
                                                     __FILE__ + ":" + std::to_string(__LINE__)}; \
    } while (0)

#define SC_LAUNCH_CHECK() SC_CUDA(cudaGetLastError())

// A grow-only device buffer owned by a model.
struct DevBuf {
    void *ptr = nullptr;
    size_t bytes = 0;
    void *get(size_t need, cudaStream_t s) {
        if (need <= bytes) return ptr;
        if (ptr) {
            SC_CUDA(cudaStreamSynchronize(s));
            SC_CUDA(cudaFree(ptr));
            ptr = nullptr;
            bytes = 0;
        }
        size_t cap = need < 4096 ? 4096 : need;
        SC_CUDA(cudaMalloc(&ptr, cap));
        bytes = cap;
        return ptr;
    }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        bytes = 0;
    }
};

// Kernel classes timed by the optional per-launch profiler (sc_profile_*).
enum KernelKind {
    KK_WINDOWS = 0, KK_LAYER0 = 1, KK_HIDDEN = 2, KK_LAST = 3, KK_CDF = 4, KK_ENCODE = 5,
    KK_COMPACT = 6, KK_DECODE = 7, KK_FUSED_COMPRESS = 8, KK_FUSED_DECODE = 9, KK_SMALL_DECODE = 10,
    KK_SPLIT = 11, KK_REASSEMBLE = 12, KK_KINDS = 13
};

// CUDA-event timing of individual launches on their own stream.  Disabled by
// default; when enabled every timed launch records an event pair, and the pairs
// are resolved after the API call has synchronised its stream.
struct Profiler {
    bool on = false;
    struct Rec {
        int kind;
        cudaEvent_t a, b;
        int64_t work;
    };
    std::vector<Rec> pending;
    std::vector<cudaEvent_t> pool;
    double ms[KK_KINDS] = {};
    int64_t launches[KK_KINDS] = {};
    int64_t work[KK_KINDS] = {};
    cudaEvent_t ev() {
        if (pool.empty()) {
            cudaEvent_t e;
            SC_CUDA(cudaEventCreate(&e));
            return e;
        }
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    void reset() {
        for (int k = 0; k < KK_KINDS; ++k) { ms[k] = 0; launches[k] = 0; work[k] = 0; }
    }
    void collect() {
        for (auto &r : pending) {
            float t = 0;
            SC_CUDA(cudaEventElapsedTime(&t, r.a, r.b));
            ms[r.kind] += t;
            launches[r.kind] += 1;
            work[r.kind] += r.work;
            pool.push_back(r.a);
            pool.push_back(r.b);
        }
        pending.clear();
    }
    ~Profiler() {
        for (auto e : pool) cudaEventDestroy(e);
        for (auto &r : pending) { cudaEventDestroy(r.a); cudaEventDestroy(r.b); }
    }
};

struct ProfScope {
    Profiler &p;
    cudaStream_t s;
    bool on;
    Profiler::Rec rec;
    ProfScope(Profiler &prof, int kind, cudaStream_t stream, int64_t work) : p(prof), s(stream), on(prof.on) {
        if (!on) return;
        rec.kind = kind;
        rec.work = work;
        rec.a = p.ev();
        rec.b = p.ev();
        SC_CUDA(cudaEventRecord(rec.a, s));
    }
    ~ProfScope() {
        if (!on) return;
        cudaEventRecord(rec.b, s);
        p.pending.push_back(rec);
    }
};

struct LayerDev {
    int32_t in_dim, out_dim;
    int8_t *w = nullptr;        // [out][in] row-major (CUDA-core path)
    int8_t *w_tc = nullptr;     // tensor-core operand layout (tcgen05 path), or null
    int32_t *bias = nullptr;    // [out]
    // bias tile of the pair kernels, [256][128] int8 (null when the bias stays in the epilogue):
    // row n holds, for each 256-column half h, 32 int8 digits of bias[h * 256 + n] in bytes
    // 64h .. 64h + 31 and the multipliers 16 x 127, 16 x 1 in bytes 64h + 32 .. 64h + 63
    int8_t *bdig = nullptr;
    Requant rq;
};

// Bias tile of one layer (see LayerDev::bdig), or an empty vector when the layer cannot use one:
// a width other than 256 or 512, or a bias outside the range the digits reach (|b| <= 258,127).
std::vector<int8_t> bias_tile(const int32_t *bias, int out_dim);

// Launch the CUDA-core MLP: windows int16 [rows][window] -> logits int8 [rows][256].
void mlp_simple(sc_model *m, const int16_t *windows, int64_t rows, int8_t *logits, cudaStream_t s);

// Where the rows of MLP layer 0 take their context windows from (tcgen05 path).
struct L0Source {
    int kind;                    // 1 explicit windows, 2 decode rows, 3 compress tiles
    const int16_t *windows;      // kind 1: [rows][64]
    const uint8_t *tokens;       // kind 2: decoded tokens; kind 3: the batch's tokens
    const int64_t *order;        // kind 2: active row -> chunk
    const int64_t *tok_off;      // kind 2: chunk -> first token; kind 3: token offsets of the chunks
    int64_t t;                   // kind 2: decode step
    const int32_t *tile_chunk;   // kind 3: chunk of each 128-row tile
    const int32_t *tile_t0;      // kind 3: first position of each tile
    int64_t row_base;            // kind 3: output row = tok_off[c] - row_base + t
};

// The tcgen05 MLP: layer 0 reads its windows as `src` describes, the other
// layers stream activations through HBM; `l0_tiles` is the tile count of
// compress tile lists (kind 3).
bool mlp_tc_supported(const sc_model *m);
void mlp_tc(sc_model *m, const L0Source &src, int64_t rows, int64_t l0_tiles, int8_t *logits, cudaStream_t s);
void mlp_tc_prepare(sc_model *m);
// One layer alone on explicit int8 activations [rows][in_dim] -> [rows][out_dim].
void linear_tc(sc_model *m, int layer, const int8_t *x, int64_t rows, int8_t *y, cudaStream_t s);

// Fused persistent kernels (all layers + coder step in one launch).
bool fused_supported(const sc_model *m);
void fused_compress(sc_model *m, const int32_t *tile_chunk, const int32_t *tile_t0, int64_t n_tiles,
                    const uint8_t *tokens, const int64_t *tok_off, int64_t row_base, int64_t rows, uint2 *pairs,
                    cudaStream_t s);
// Decode the chunks order[0 .. n_rows), sorted by length (descending, all nonzero; their
// lengths on the host in sorted_len), with every layer and the decoder step in persistent
// kernels: one launch on SM pairs, or, for a batch of at most num_sms / 8 tiles of 128 rows (or
// with mlp_path 5), one launch with a cluster of eight CTAs per tile; or launches of at most the
// single-SM kernels' capacity.
void fused_decode(sc_model *m, const int64_t *order, int64_t n_rows, const int64_t *sorted_len,
                  const int64_t *lengths, DecState *state, const uint32_t *words, uint8_t *tokens_out,
                  const int64_t *out_off, uint8_t *errors, cudaStream_t s);

// Value of the device error flag set by timed-out waits (optionally cleared).
int read_device_error(int clear);

}  // namespace sc

struct sc_model {
    int device = 0;
    int32_t window = 64, emb_dim = 128, num_layers = 0, chunk_len = 2048;
    // 0 auto, 1 tcgen05 (fused, CTA pairs), 2 CUDA cores, 3 tcgen05 layer by layer,
    // 4 tcgen05 fused on single CTAs, 5 as 1 with every decode on the small-batch clusters
    // (0 decodes batches of at most num_sms / 8 tiles there, 1 never)
    int32_t mlp_path = 0;
    int num_sms = 148;
    bool tc_ok = false;
    int8_t *emb = nullptr;     // [257][emb_dim]
    uint64_t *lut = nullptr;   // [256]
    std::vector<sc::LayerDev> layers;
    std::vector<CUtensorMap> tc_wmaps;   // weight tensor maps of the tcgen05 path (box 256 rows)
    std::vector<CUtensorMap> tc_wmaps2;  // weight tensor maps for CTA pairs (box 128 rows)
    std::vector<CUtensorMap> tc_bmaps2;  // bias tile maps for CTA pairs (box 128 rows; unset without a tile)
    std::vector<CUtensorMap> small_wmaps;  // small-batch decoder: box out_dim / 8 rows
    sc::Profiler prof;
    // unit trace of the first SM pair of the fused kernels (sc_trace_enable)
    unsigned long long *trace_buf = nullptr;
    unsigned int *trace_count = nullptr;
    int trace_cap = 0;
    // workspaces
    sc::DevBuf ws_windows, ws_act0, ws_act1, ws_logits, ws_pairs, ws_stage, ws_nwords,
        ws_err, ws_scan, ws_tmp, ws_order, ws_state, ws_tok_off, ws_misc, ws_ering, ws_sched;
};
