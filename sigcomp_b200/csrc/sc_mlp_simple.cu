// CUDA-core integer MLP (dp4a), the cross-check for the tensor-core path.
//
// One launch per linear layer: y = requant(x * W^T + b) with the exact
// epilogue of _requantize (sigcomp/cpu_int_kernels.py:5-14).  Layer 0 gathers
// its input rows from the embedding table through the context windows,
// x[row, p*E + c] = E_q[window[row, p], c] (sigcomp/cpu_int_kernels.py:107-121).
#include "sc_internal.h"

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
