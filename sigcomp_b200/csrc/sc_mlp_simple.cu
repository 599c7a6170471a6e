// CUDA-core integer MLP (dp4a), the cross-check for the tensor-core path.
//
// One launch per linear layer: y = requant(x * W^T + b) with the exact
// epilogue of _requantize (sigcomp/cpu_int_kernels.py:5-14).  Layer 0 gathers
// its input rows from the embedding table through the context windows,
// x[row, p*E + c] = E_q[window[row, p], c] (sigcomp/cpu_int_kernels.py:107-121).
#include <mutex>

#include "sc_internal.h"
#include "../../include/sigcomp_b200.h"

namespace sc {
namespace {

constexpr int BM = 64, BN = 64, BK = 64, PAD = 16;   // row stride 80 B keeps 16-byte stores aligned

template <bool GATHER>
__global__ void __launch_bounds__(256) k_linear_dp4a(
    const int8_t *__restrict__ x, const int16_t *__restrict__ windows, const int8_t *__restrict__ emb,
    int emb_dim, int window, const int8_t *__restrict__ w, const int32_t *__restrict__ bias, Requant rq,
    int8_t *__restrict__ y, int64_t M, int N, int K)
{
    __shared__ __align__(16) int8_t As[BM][BK + PAD];
    __shared__ __align__(16) int8_t Bs[BN][BK + PAD];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t row0 = (int64_t)blockIdx.y * BM;
    const int col0 = blockIdx.x * BN;
    int32_t acc[4][4] = {};
    // loader mapping: 256 threads x 16 bytes = one 64x64 tile
    const int lr = tid >> 2, lk = (tid & 3) * 16;
    for (int k0 = 0; k0 < K; k0 += BK) {
        {
            const int64_t r = row0 + lr;
            int4 v = make_int4(0, 0, 0, 0);
            if (r < M) {
                if (GATHER) {
                    const int k = k0 + lk;
                    const int p = k / emb_dim, c = k - p * emb_dim;
                    const int tok = windows[r * window + p];
                    v = *reinterpret_cast<const int4 *>(emb + (int64_t)tok * emb_dim + c);
                } else {
                    v = *reinterpret_cast<const int4 *>(x + r * K + k0 + lk);
                }
            }
            *reinterpret_cast<int4 *>(&As[lr][lk]) = v;
            const int n = col0 + lr;
            int4 u = make_int4(0, 0, 0, 0);
            if (n < N) u = *reinterpret_cast<const int4 *>(w + (int64_t)n * K + k0 + lk);
            *reinterpret_cast<int4 *>(&Bs[lr][lk]) = u;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < BK; kk += 4) {
            int a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const int *>(&As[ty + 16 * i][kk]);
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const int *>(&Bs[tx + 16 * j][kk]);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = __dp4a(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t r = row0 + ty + 16 * i;
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = col0 + tx + 16 * j;
            if (n < N) y[r * N + n] = (int8_t)requant(acc[i][j], bias[n], rq);
        }
    }
}

}  // namespace

void mlp_simple(sc_model *m, const int16_t *windows, int64_t rows, int8_t *logits, cudaStream_t s)
{
    if (rows <= 0) return;
    int max_w = 0;
    for (auto &L : m->layers) max_w = L.out_dim > max_w ? L.out_dim : max_w;
    int8_t *bufs[2] = {
        (int8_t *)m->ws_act0.get((size_t)rows * max_w, s),
        (int8_t *)m->ws_act1.get((size_t)rows * max_w, s),
    };
    const int8_t *x = nullptr;
    for (int l = 0; l < m->num_layers; ++l) {
        const LayerDev &L = m->layers[l];
        int8_t *y = (l == m->num_layers - 1) ? logits : bufs[l & 1];
        dim3 grid((L.out_dim + BN - 1) / BN, (unsigned)((rows + BM - 1) / BM));
        ProfScope ps(m->prof, l == 0 ? KK_LAYER0 : (l == m->num_layers - 1 ? KK_LAST : KK_HIDDEN), s, rows);
        if (l == 0)
            k_linear_dp4a<true><<<grid, 256, 0, s>>>(nullptr, windows, m->emb, m->emb_dim, m->window, L.w,
                                                     L.bias, L.rq, y, rows, L.out_dim, L.in_dim);
        else
            k_linear_dp4a<false><<<grid, 256, 0, s>>>(x, nullptr, nullptr, 0, 0, L.w, L.bias, L.rq, y, rows,
                                                      L.out_dim, L.in_dim);
        SC_LAUNCH_CHECK();
        count_launch();
        x = y;
    }
}

}  // namespace sc

// ---------------------------------------------------------------------------
// Allocation-free MLP logits (sc_mlp_logits_device_noalloc).
//
// Some callers cannot call cudaMalloc: a host framework that has reserved the
// GPU's memory for its own pool (a serving engine's caching allocator) makes a
// library's own cudaMalloc fail or fragment that pool, and a latency-critical
// caller cannot accept the implicit device synchronisation of cudaMalloc and
// cudaFree.  sc_mlp_logits_device grows per-model activation buffers on first
// use; this variant runs the same CUDA-core layer kernels with the two
// ping-pong activation buffers in a fixed, file-scope device array instead.
//
// The array is loaded with the library and held on every GPU that loads it
// until the process exits.  All calls share it and it keeps the last call's
// contents; every layer overwrites all the rows it later reads, so nothing in
// it needs clearing.  Calls whose work overlaps on the GPU (two streams, two
// threads, two models on one device) race on the array.
// ---------------------------------------------------------------------------
namespace sc {
namespace {

constexpr int64_t kNoAllocMaxRows = SC_NOALLOC_MAX_ROWS;
constexpr int kNoAllocMaxWidth = SC_NOALLOC_MAX_WIDTH;
constexpr size_t kNoAllocBufBytes = (size_t)kNoAllocMaxRows * kNoAllocMaxWidth;

static __device__ __align__(256) int8_t g_noalloc_scratch[2 * kNoAllocBufBytes];

// Device address of g_noalloc_scratch per device ordinal.  In host code the
// array's name is a host-side stand-in, so the address must come from
// cudaGetSymbolAddress, called once per device with that device current.
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
int8_t *g_noalloc_ptr[kMaxDevices] = {};

int8_t *noalloc_scratch(int device)
{
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void *p = nullptr;
        SC_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_ptr[device] = (int8_t *)p;
    }
    return g_noalloc_ptr[device];
}

}  // namespace

}  // namespace sc

extern "C" SC_API int sc_mlp_logits_device_noalloc(sc_model *m, const int16_t *windows, int64_t rows,
                                                   int8_t *logits, void *stream)
{
    using namespace sc;
    set_error("%s", "");
    if (!m || rows < 0 || (rows > 0 && (!windows || !logits))) {
        set_error("invalid argument");
        return SC_ERR_INVALID_ARGUMENT;
    }
    if (rows > kNoAllocMaxRows) {
        set_error("sc_mlp_logits_device_noalloc: %lld rows exceed its fixed scratch limit of %lld rows "
                  "(split the batch, or use sc_mlp_logits_device)",
                  (long long)rows, (long long)kNoAllocMaxRows);
        return SC_ERR_INVALID_ARGUMENT;
    }
    for (int l = 0; l + 1 < m->num_layers; ++l)
        if (m->layers[l].out_dim > kNoAllocMaxWidth) {
            set_error("sc_mlp_logits_device_noalloc: layer %d is %d wide, above the scratch width of %d", l,
                      m->layers[l].out_dim, kNoAllocMaxWidth);
            return SC_ERR_UNSUPPORTED;
        }
    if (m->device < 0 || m->device >= kMaxDevices) {
        set_error("sc_mlp_logits_device_noalloc: device %d out of range", m->device);
        return SC_ERR_UNSUPPORTED;
    }
    cudaStream_t s = (cudaStream_t)stream;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != m->device) {
        // the scratch address and the weights belong to the model's device: never launch elsewhere
        const cudaError_t e = cudaSetDevice(m->device);
        if (e != cudaSuccess) {
            set_error("CUDA error %s (%s) selecting device %d", cudaGetErrorName(e), cudaGetErrorString(e),
                      m->device);
            return SC_ERR_CUDA;
        }
    }
    int rc = SC_OK;
    try {
        if (rows > 0) {
            int8_t *base = noalloc_scratch(m->device);
            int8_t *bufs[2] = {base, base + kNoAllocBufBytes};
            const int8_t *x = nullptr;
            for (int l = 0; l < m->num_layers; ++l) {
                const LayerDev &L = m->layers[l];
                int8_t *y = (l == m->num_layers - 1) ? logits : bufs[l & 1];
                dim3 grid((L.out_dim + BN - 1) / BN, (unsigned)((rows + BM - 1) / BM));
                if (l == 0)
                    k_linear_dp4a<true><<<grid, 256, 0, s>>>(nullptr, windows, m->emb, m->emb_dim, m->window,
                                                             L.w, L.bias, L.rq, y, rows, L.out_dim, L.in_dim);
                else
                    k_linear_dp4a<false><<<grid, 256, 0, s>>>(x, nullptr, nullptr, 0, 0, L.w, L.bias, L.rq, y,
                                                              rows, L.out_dim, L.in_dim);
                SC_LAUNCH_CHECK();
                count_launch();
                x = y;
            }
        }
        SC_CUDA(cudaStreamSynchronize(s));
    } catch (const CudaError &e) {
        set_error("CUDA error %s (%s) in %s", cudaGetErrorName(e.code), cudaGetErrorString(e.code),
                  e.where.c_str());
        rc = SC_ERR_CUDA;
    } catch (...) {
        // nothing may cross the C boundary (the scratch lookup takes a lock, which can throw)
        set_error("sc_mlp_logits_device_noalloc: internal error");
        rc = SC_ERR_CUDA;
    }
    if (prev >= 0 && prev != m->device) cudaSetDevice(prev);
    return rc;
}
