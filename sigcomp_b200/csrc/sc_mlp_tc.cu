// tcgen05 tensor-core integer MLP for sm_100a.
//
// One launch per linear layer, y = requant(x * W^T + b), computed exactly:
// int8 x int8 products accumulate in int32 in tensor memory (TMEM) and the
// epilogue applies _requantize (sigcomp/cpu_int_kernels.py:5-14).
//
// Tile: 128 rows x 256 output columns per CTA, K streamed in 128-byte blocks
// through a multi-stage shared-memory ring:
//   warp 0        TMA producer: weight tile (256 x 128 B) and, for hidden
//                 layers, the activation tile (128 x 128 B)
//   warp 1        TMEM allocation; one lane issues tcgen05.mma (M=128, N=256,
//                 K=32, four per K block) and commits stage releases
//   warps 2-3     layer 0 only: build the activation tile from the embedding
//                 table held in shared memory (x[r, p*128 + c] = E_q[win[r, p], c],
//                 sigcomp/cpu_int_kernels.py:107-121), 128B-swizzled
//   warps 4-7     epilogue: TMEM -> registers -> requantise -> int8 rows
// Operands use the K-major 128-byte-swizzle layout written by TMA.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <array>
#include <climits>
#include <queue>

#include "sc_internal.h"
#include "sc_tc.cuh"

namespace sc {
namespace {

using namespace tc;

constexpr int TM = 128;          // rows per tile
constexpr int TN = 256;          // output columns per unit (one TMEM accumulator)
constexpr int KB = 128;          // bytes of K per stage
constexpr int A_BYTES = TM * KB;             // 16 KB
constexpr int B_BYTES = TN * KB;             // 32 KB
constexpr int EMB_ROWS = 257;
constexpr int EMB_DIM = 128;
constexpr int EMB_BYTES = EMB_ROWS * EMB_DIM;
constexpr int WIN = 64;                      // context window of the tensor-core path
constexpr int WS = WIN + 2;                  // window-token row stride (uint16): avoids bank conflicts
constexpr int G_ROWS = TM + WIN;             // sliding-window embedding rows per tile
constexpr int G_BYTES = G_ROWS * KB;         // 24 KB
constexpr int MAX_N = 512;

// A operand sources
enum { A_TMA = 0, A_GATHER = 1, A_SLIDE = 3 };

template <int MODE>
struct Cfg {
    static constexpr int STAGES = MODE == A_GATHER ? 3 : 4;
    static constexpr int STAGE_BYTES = (MODE == A_SLIDE ? 0 : A_BYTES) + B_BYTES;
    static constexpr int OFF_EXTRA = STAGES * STAGE_BYTES;
    // A_GATHER: embedding table + window tokens; A_SLIDE: two sliding buffers
    static constexpr int EXTRA = MODE == A_GATHER ? (33 * 1024 + TM * WS * 2)
                               : MODE == A_SLIDE ? 2 * G_BYTES : 0;
    static constexpr int OFF_BIAS = OFF_EXTRA + EXTRA;
    static constexpr int OFF_BAR = OFF_BIAS + MAX_N * 4;
    static constexpr int NBAR = 2 * STAGES + 8;
    static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
    static constexpr int SMEM = OFF_TMEM + 16 + 1024;   // + alignment slack
};

}  // namespace

namespace {

__device__ __forceinline__ void mma_k_block(uint32_t d, uint32_t a_addr, uint32_t b_addr, bool first) {
    constexpr uint32_t idesc = idesc_i8(TM, TN);
#pragma unroll
    for (int k = 0; k < KB / 32; ++k)
        mma_i8(d, smem_desc_sw128(a_addr + 32 * k), smem_desc_sw128(b_addr + 32 * k), idesc,
               (!first || k) ? 1u : 0u);
}

// Persistent layer kernel: every CTA walks row tiles blockIdx.x, +gridDim.x, ...
// and for each tile the N/256 output halves ("units").  Two TMEM accumulators
// (2 x 256 columns) let the epilogue of one unit overlap the MMAs of the next.
//   warp 0      TMA producer (weights; activations in A_TMA mode)
//   warp 1      TMEM owner; lane 0 issues tcgen05.mma and commits
//   warps 2-5   epilogue (TMEM lane quarters 2,3,0,1)
//   warps 6-7   A_GATHER: build activation stages from the embedding table;
//               A_SLIDE: build the per-tile sliding embedding buffer
template <int MODE>
__global__ void __launch_bounds__(256, 1) k_layer(
    const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, const L0Source src,
    const int8_t *__restrict__ emb, const int32_t *__restrict__ bias, Requant rq, int8_t *__restrict__ y,
    int64_t M, int N, int K, int n_tiles)
{
    using C = Cfg<MODE>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint64_t *full = bars, *empty = bars + C::STAGES;
    uint64_t *acc_full = bars + 2 * C::STAGES, *acc_empty = acc_full + 2;
    uint64_t *g_full = acc_empty + 2, *g_empty = g_full + 2;
    uint32_t *tmem_slot = (uint32_t *)(smem + C::OFF_TMEM);
    int32_t *bias_s = (int32_t *)(smem + C::OFF_BIAS);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NH = N / TN;
    const int nkb = K / KB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], MODE == A_GATHER ? 1 + 2 : 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
            mbar_init(&g_full[b], 2);
            mbar_init(&g_empty[b], 1);
        }
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
        if (MODE == A_TMA) prefetch_tmap(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * TN);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < N; i += blockDim.x) bias_s[i] = bias[i];
    if (MODE == A_GATHER) {
        const int4 *srcv = reinterpret_cast<const int4 *>(emb);
        int4 *dst = reinterpret_cast<int4 *>(smem + C::OFF_EXTRA);
        for (int i = threadIdx.x; i < EMB_BYTES / 16; i += blockDim.x) dst[i] = srcv[i];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x)
                for (int nh = 0; nh < NH && ok; ++nh)
                    for (int kb = 0; kb < nkb; ++kb, ++it) {
                        const int s = it % C::STAGES;
                        if (!(ok = mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1))) break;
                        uint8_t *st = smem + s * C::STAGE_BYTES;
                        if (MODE == A_TMA) {
                            mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
                            tma_load_2d(st, &tmap_x, &full[s], kb * KB, tile * TM);
                            tma_load_2d(st + A_BYTES, &tmap_w, &full[s], kb * KB, nh * TN);
                        } else {
                            mbar_arrive_expect_tx(&full[s], B_BYTES);
                            tma_load_2d(st + (MODE == A_SLIDE ? 0 : A_BYTES), &tmap_w, &full[s], kb * KB, nh * TN);
                        }
                    }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            uint32_t it = 0, uu = 0, li = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, ++li) {
                const int gb = li & 1;
                if (MODE == A_SLIDE && !(ok = mbar_wait(&g_full[gb], (li >> 1) & 1))) break;
                tc_fence_after();
                for (int nh = 0; nh < NH && ok; ++nh, ++uu) {
                    const int ab = uu & 1;
                    if (!(ok = mbar_wait(&acc_empty[ab], ((uu >> 1) & 1) ^ 1))) break;
                    tc_fence_after();
                    const uint32_t d = tmem_base + ab * TN;
                    for (int kb = 0; kb < nkb; ++kb, ++it) {
                        const int s = it % C::STAGES;
                        if (!(ok = mbar_wait(&full[s], (it / C::STAGES) & 1))) break;
                        tc_fence_after();
                        const uint32_t st = smem_u32(smem + s * C::STAGE_BYTES);
                        uint32_t a_addr, b_addr;
                        if (MODE == A_SLIDE) {
                            // K block kb is window position kb: rows kb .. kb+127 of the sliding buffer
                            a_addr = smem_u32(smem + C::OFF_EXTRA + gb * G_BYTES) + kb * KB;
                            b_addr = st;
                        } else {
                            a_addr = st;
                            b_addr = st + A_BYTES;
                        }
                        mma_k_block(d, a_addr, b_addr, kb == 0);
                        mma_commit(&empty[s]);
                    }
                    mma_commit(&acc_full[ab]);
                }
                if (MODE == A_SLIDE) mma_commit(&g_empty[gb]);
            }
        }
    } else if (warp >= 2 && warp <= 5) {
        // ---- epilogue: TMEM -> requantise -> int8 rows
        const int q = warp & 3;
        const int r = q * 32 + lane;
        uint32_t uu = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            int64_t row;
            bool valid;
            if (MODE == A_SLIDE) {
                const int c = src.tile_chunk[tile];
                const int t0 = src.tile_t0[tile];
                const int64_t len = src.tok_off[c + 1] - src.tok_off[c];
                valid = t0 + r < len;
                row = src.tok_off[c] - src.row_base + t0 + r;
            } else {
                row = (int64_t)tile * TM + r;
                valid = row < M;
            }
            for (int nh = 0; nh < NH; ++nh, ++uu) {
                const int ab = uu & 1;
                ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (uu >> 1) & 1));
                if (!ok) break;
                tc_fence_after();
                const uint32_t taddr = tmem_base + ab * TN + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
                for (int c = 0; c < TN / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c * 32, v);
                    tmem_ld_wait();
                    uint32_t packed[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        uint32_t p = 0;
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int col = nh * TN + c * 32 + i * 4 + b;
                            const int32_t o = requant((int32_t)v[i * 4 + b], bias_s[col], rq);
                            p |= ((uint32_t)(o & 0xFF)) << (8 * b);
                        }
                        packed[i] = p;
                    }
                    if (valid) {
                        uint4 *dst = reinterpret_cast<uint4 *>(y + row * N + nh * TN + c * 32);
                        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[ab]);
            }
        }
    } else if (MODE == A_GATHER) {
        // ---- warps 6-7: activation stages from the embedding table; warp 6 builds
        // rows 0-63, warp 7 rows 64-127, each from its own window tokens
        const int wb = (warp - 6) * 64;
        const uint8_t *emb_s = smem + C::OFF_EXTRA;
        uint16_t *win_s = (uint16_t *)(smem + C::OFF_EXTRA + 33 * 1024);
        const int j = lane & 7, sub = lane >> 3;
        uint32_t it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
            // window tokens of this warp's 64 rows: lane handles rows wb+lane and wb+lane+32
            __syncwarp();
            for (int h = 0; h < 2; ++h) {
                const int r = wb + lane + 32 * h;
                const int64_t row = (int64_t)tile * TM + r;
                uint16_t *dst = win_s + r * WS;
                if (row >= M) {
                    for (int p = 0; p < WIN; ++p) dst[p] = SC_SOS;
                } else if (src.kind == 1) {
                    const int4 *w = reinterpret_cast<const int4 *>(src.windows + row * WIN);
#pragma unroll
                    for (int v = 0; v < WIN / 8; ++v) {
                        const int4 x = w[v];
                        const uint32_t xs[4] = {(uint32_t)x.x, (uint32_t)x.y, (uint32_t)x.z, (uint32_t)x.w};
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            dst[v * 8 + 2 * e] = (uint16_t)(xs[e] & 0xFFFF);
                            dst[v * 8 + 2 * e + 1] = (uint16_t)(xs[e] >> 16);
                        }
                    }
                } else {
                    const int64_t b0 = src.tok_off[src.order[row]];
#pragma unroll 16
                    for (int p = 0; p < WIN; ++p) {
                        const int64_t pos = src.t - WIN + p;
                        dst[p] = pos >= 0 ? (uint16_t)src.tokens[b0 + pos] : (uint16_t)SC_SOS;
                    }
                }
            }
            __syncwarp();
            for (int nh = 0; nh < NH && ok; ++nh)
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1));
                    if (!ok) break;
                    uint8_t *a_st = smem + s * C::STAGE_BYTES;
#pragma unroll 4
                    for (int rr = sub; rr < 64; rr += 4) {
                        const int r = wb + rr;
                        const int tok = win_s[r * WS + kb];
                        const int4 v = *reinterpret_cast<const int4 *>(emb_s + tok * EMB_DIM + j * 16);
                        *reinterpret_cast<int4 *>(a_st + sw128_offset(r, j)) = v;
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[s]);
                }
        }
    } else if (MODE == A_SLIDE) {
        // ---- warps 6-7: sliding embedding buffer of the tile: row s holds
        // E_q[token at position t0 - 64 + s] (SOS before the chunk start), so the
        // activation of K block p is rows p .. p+127 of the buffer
        const int tw = threadIdx.x - 192;        // 0..63
        const int j = tw & 7, r0 = tw >> 3;
        uint32_t li = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++li) {
            const int gb = li & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&g_empty[gb], ((li >> 1) & 1) ^ 1))) break;
            uint8_t *g = smem + C::OFF_EXTRA + gb * G_BYTES;
            const int c = src.tile_chunk[tile];
            const int t0 = src.tile_t0[tile];
            const int64_t begin = src.tok_off[c];
            const int64_t len = src.tok_off[c + 1] - begin;
#pragma unroll 4
            for (int sr = r0; sr < G_ROWS; sr += 8) {
                const int64_t pos = (int64_t)t0 - WIN + sr;
                const int tok = pos < 0 ? SC_SOS : (pos < len ? src.tokens[begin + pos] : 0);
                const int4 v = *reinterpret_cast<const int4 *>(emb + tok * EMB_DIM + j * 16);
                *reinterpret_cast<int4 *>(g + sw128_offset(sr, j)) = v;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&g_full[gb]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 2 * TN);
    }
}

}  // namespace
}  // namespace sc

#include "sc_mlp_fused.cuh"
#include "sc_mlp_fused2.cuh"
#include "sc_mlp_small.cuh"

namespace sc {
namespace {

// ---- host side ------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        SC_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !p) throw CudaError{cudaErrorNotSupported, "cuTensorMapEncodeTiled"};
        fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    return fn;
}

// 2-D int8 tensor [rows][cols] (row pitch `pitch` bytes), box = box_rows x 128 bytes, 128B swizzle
CUtensorMap make_tmap(const void *base, uint64_t cols, uint64_t rows, uint64_t pitch, uint32_t box_rows)
{
    CUtensorMap m;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {(cuuint32_t)KB, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError{cudaErrorInvalidValue, "cuTensorMapEncodeTiled failed"};
    return m;
}

}  // namespace

std::vector<int8_t> bias_tile(const int32_t *bias, int out_dim)
{
    if (out_dim != TN && out_dim != 2 * TN) return {};
    // bias[c] = 127 * (d_0 + ... + d_15) + d_16 with every digit in [-127, 127] and |d_16| <= 63
    std::vector<int8_t> t((size_t)TN * KB, 0);
    for (int n = 0; n < TN; ++n) {
        int8_t *row = t.data() + (size_t)n * KB;
        for (int h = 0; h < 2; ++h) {
            int8_t *q = row + 64 * h;
            for (int j = 32; j < 48; ++j) q[j] = 127;
            for (int j = 48; j < 64; ++j) q[j] = 1;
            if (h * TN >= out_dim) continue;
            const int64_t b = bias[h * TN + n];
            int64_t hi = b >= 0 ? (b + 63) / 127 : -((-b + 63) / 127);
            const int64_t lo = b - 127 * hi;
            if (hi > 16 * 127 || hi < -16 * 127) return {};
            for (int j = 0; j < 16; ++j) {
                const int64_t d = hi > 127 ? 127 : (hi < -127 ? -127 : hi);
                q[j] = (int8_t)d;
                hi -= d;
            }
            q[16] = (int8_t)lo;
        }
    }
    return t;
}

bool mlp_tc_supported(const sc_model *m)
{
    if (m->emb_dim != EMB_DIM || m->window != WIN || m->layers[0].in_dim != WIN * EMB_DIM) return false;
    for (auto &L : m->layers)
        if (L.in_dim % KB || L.out_dim % TN || L.out_dim > MAX_N) return false;
    return true;
}

template <int MODE>
static void set_smem_attr()
{
    SC_CUDA(cudaFuncSetAttribute(k_layer<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<MODE>::SMEM));
}

void mlp_tc_prepare(sc_model *m)
{
    auto &maps = m->tc_wmaps;
    maps.clear();
    for (auto &L : m->layers) maps.push_back(make_tmap(L.w, L.in_dim, L.out_dim, L.in_dim, TN));
    set_smem_attr<A_TMA>();
    set_smem_attr<A_GATHER>();
    set_smem_attr<A_SLIDE>();
    SC_CUDA(cudaFuncSetAttribute(k_fused<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, FCfg<true>::SMEM));
    SC_CUDA(cudaFuncSetAttribute(k_fused2<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, F2Cfg<true>::SMEM));
    SC_CUDA(cudaFuncSetAttribute(k_fused2<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, F2Cfg<false>::SMEM));
    SC_CUDA(cudaFuncSetAttribute(k_fused2<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, F2Cfg<true>::SMEM));
    SC_CUDA(cudaFuncSetAttribute(k_fused2<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, F2Cfg<false>::SMEM));
    auto &maps2 = m->tc_wmaps2;
    maps2.clear();
    for (auto &L : m->layers) maps2.push_back(make_tmap(L.w, L.in_dim, L.out_dim, L.in_dim, TN / 2));
    auto &bmaps = m->tc_bmaps2;
    bmaps.assign(m->layers.size(), CUtensorMap{});
    for (size_t l = 0; l < m->layers.size(); ++l)
        if (m->layers[l].bdig) bmaps[l] = make_tmap(m->layers[l].bdig, KB, TN, KB, TN / 2);
    SC_CUDA(cudaFuncSetAttribute(k_fused<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, FCfg<false>::SMEM));
    SC_CUDA(cudaFuncSetAttribute(k_small_decode<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SmallCfg::SMEM));
    SC_CUDA(cudaFuncSetAttribute(k_small_decode<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SmallCfg::SMEM));
    auto &maps3 = m->small_wmaps;
    maps3.clear();
    for (auto &L : m->layers)
        maps3.push_back(make_tmap(L.w, L.in_dim, L.out_dim, L.in_dim, (uint32_t)(L.out_dim / SMALL_C)));
    SC_CUDA(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, m->device));
}

void mlp_tc(sc_model *m, const L0Source &src, int64_t rows, int64_t l0_tiles, int8_t *logits, cudaStream_t s)
{
    if (rows <= 0) return;
    auto &maps = m->tc_wmaps;
    int max_w = 0;
    for (auto &L : m->layers) max_w = L.out_dim > max_w ? L.out_dim : max_w;
    int8_t *bufs[2] = {
        (int8_t *)m->ws_act0.get((size_t)rows * max_w, s),
        (int8_t *)m->ws_act1.get((size_t)rows * max_w, s),
    };
    const int64_t row_tiles = (rows + TM - 1) / TM;
    const int8_t *x = nullptr;
    for (int l = 0; l < m->num_layers; ++l) {
        const LayerDev &L = m->layers[l];
        int8_t *yb = (l == m->num_layers - 1) ? logits : bufs[l & 1];
        ProfScope ps(m->prof, l == 0 ? KK_LAYER0 : (l == m->num_layers - 1 ? KK_LAST : KK_HIDDEN), s, rows);
        if (l == 0) {
            const int64_t nt = src.kind == 3 ? l0_tiles : row_tiles;
            const unsigned grid = (unsigned)std::min<int64_t>(nt, m->num_sms);
            if (src.kind == 3)
                k_layer<A_SLIDE><<<grid, 256, Cfg<A_SLIDE>::SMEM, s>>>(maps[0], maps[0], src, m->emb, L.bias, L.rq,
                                                                      yb, rows, L.out_dim, L.in_dim, (int)nt);
            else
                k_layer<A_GATHER><<<grid, 256, Cfg<A_GATHER>::SMEM, s>>>(maps[0], maps[0], src, m->emb, L.bias, L.rq,
                                                                        yb, rows, L.out_dim, L.in_dim, (int)nt);
        } else {
            CUtensorMap xm = make_tmap(x, L.in_dim, rows, L.in_dim, TM);
            const unsigned grid = (unsigned)std::min<int64_t>(row_tiles, m->num_sms);
            k_layer<A_TMA><<<grid, 256, Cfg<A_TMA>::SMEM, s>>>(maps[l], xm, src, m->emb, L.bias, L.rq, yb, rows,
                                                              L.out_dim, L.in_dim, (int)row_tiles);
        }
        SC_LAUNCH_CHECK();
        count_launch();
        x = yb;
    }
}

// One integer linear layer alone, y = requant(x * W_l^T + b_l), on explicit int8 activations
// x [rows][in_dim] (layer 0 included: x is then the gathered window rows), with the tcgen05
// layer kernel: the layer of the reference's bit_exact_linear_kernel (quant_mlp_export.py:21-76).
void linear_tc(sc_model *m, int layer, const int8_t *x, int64_t rows, int8_t *y, cudaStream_t s)
{
    if (rows <= 0) return;
    const LayerDev &L = m->layers[layer];
    const int kind = layer == 0 ? KK_LAYER0 : (layer == m->num_layers - 1 ? KK_LAST : KK_HIDDEN);
    ProfScope ps(m->prof, kind, s, rows);
    const int64_t row_tiles = (rows + TM - 1) / TM;
    CUtensorMap xm = make_tmap(x, L.in_dim, rows, L.in_dim, TM);
    const unsigned grid = (unsigned)std::min<int64_t>(row_tiles, m->num_sms);
    L0Source src{};
    k_layer<A_TMA><<<grid, 256, Cfg<A_TMA>::SMEM, s>>>(m->tc_wmaps[layer], xm, src, m->emb, L.bias, L.rq, y, rows,
                                                      L.out_dim, L.in_dim, (int)row_tiles);
    SC_LAUNCH_CHECK();
    count_launch();
}

// Shared parameters of the fused kernels; activation buffers are sized for
// grid * KT tiles of 128 rows.
static void fused_common(sc_model *m, FusedParams &p, int grid, cudaStream_t s)
{
    const int64_t rows = (int64_t)grid * KT * TM;
    int8_t *a0 = (int8_t *)m->ws_act0.get((size_t)rows * MAX_N, s);
    int8_t *a1 = (int8_t *)m->ws_act1.get((size_t)rows * MAX_N, s);
    p.act_ptr[0] = a0;
    p.act_ptr[1] = a1;
    p.act[0] = make_tmap(a0, MAX_N, rows, MAX_N, TM);
    p.act[1] = make_tmap(a1, MAX_N, rows, MAX_N, TM);
    p.num_layers = m->num_layers;
    for (int l = 0; l < m->num_layers; ++l) {
        p.w[l] = m->tc_wmaps[l];
        p.bias[l] = m->layers[l].bias;
        p.rq[l] = m->layers[l].rq;
        p.in_dim[l] = m->layers[l].in_dim;
        p.out_dim[l] = m->layers[l].out_dim;
    }
    p.emb = m->emb;
    p.lut = m->lut;
}

bool fused_supported(const sc_model *m) { return m->tc_ok && m->num_layers <= FMAX_LAYERS && m->mlp_path != 3; }

static bool use_pairs(const sc_model *m) { return m->mlp_path != 4 && m->num_sms >= 2; }


static void fused2_common(sc_model *m, Fused2Params &p, int grid, cudaStream_t s)
{
    const int64_t rows = (int64_t)grid * KT2 * TM;      // enough for either kernel's slots
    int8_t *a0 = (int8_t *)m->ws_act0.get((size_t)rows * MAX_N, s);
    int8_t *a1 = (int8_t *)m->ws_act1.get((size_t)rows * MAX_N, s);
    p.act_ptr[0] = a0;
    p.act_ptr[1] = a1;
    p.act[0] = make_tmap(a0, MAX_N, rows, MAX_N, TM);
    p.act[1] = make_tmap(a1, MAX_N, rows, MAX_N, TM);
    p.num_layers = m->num_layers;
    p.bias_mma = 0;
    for (int l = 0; l < m->num_layers; ++l) {
        p.w[l] = m->tc_wmaps2[l];
        if (m->layers[l].bdig) {
            p.bt[l] = m->tc_bmaps2[l];
            p.bias_mma |= 1u << l;
        }
        p.bias[l] = m->layers[l].bias;
        p.rq[l] = m->layers[l].rq;
        p.in_dim[l] = m->layers[l].in_dim;
        p.out_dim[l] = m->layers[l].out_dim;
    }
    p.emb = m->emb;
    p.lut = m->lut;
    if (m->trace_cap > 0) {
        SC_CUDA(cudaMemsetAsync(m->trace_count, 0, 8 * sizeof(unsigned int), s));
        p.trace = m->trace_buf;
        p.trace_count = m->trace_count;
        p.trace_cap = m->trace_cap;
    }
}

template <bool DECODE>
static void launch_pairs(const Fused2Params &p, int grid, cudaStream_t s)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(FUSED2_THREADS);
    cfg.dynamicSmemBytes = F2Cfg<DECODE>::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.trace != nullptr) SC_CUDA(cudaLaunchKernelEx(&cfg, k_fused2<DECODE, true>, p));
    else SC_CUDA(cudaLaunchKernelEx(&cfg, k_fused2<DECODE, false>, p));
}

void fused_compress(sc_model *m, const int32_t *tile_chunk, const int32_t *tile_t0, int64_t n_tiles,
                    const uint8_t *tokens, const int64_t *tok_off, int64_t row_base, int64_t rows, uint2 *pairs,
                    cudaStream_t s)
{
    if (n_tiles <= 0) return;
    ProfScope ps(m->prof, KK_FUSED_COMPRESS, s, rows);
    if (use_pairs(m)) {
        const int64_t n_pt = (n_tiles + 1) / 2;
        const int grid = 2 * (int)std::min<int64_t>(n_pt, m->num_sms / 2);
        Fused2Params p{};
        fused2_common(m, p, grid, s);
        p.n_tiles = (int)n_tiles;
        p.tile_chunk = tile_chunk;
        p.tile_t0 = tile_t0;
        p.tok_off = tok_off;
        p.tokens = tokens;
        p.row_base = row_base;
        p.pairs = pairs;
        launch_pairs<false>(p, grid, s);
    } else {
        const int grid = (int)std::min<int64_t>(n_tiles, m->num_sms);
        FusedParams p{};
        fused_common(m, p, grid, s);
        p.n_tiles = (int)n_tiles;
        p.tile_chunk = tile_chunk;
        p.tile_t0 = tile_t0;
        p.tok_off = tok_off;
        p.tokens = tokens;
        p.row_base = row_base;
        p.pairs = pairs;
        k_fused<false><<<grid, 256, FCfg<false>::SMEM, s>>>(p);
    }
    SC_LAUNCH_CHECK();
    count_launch();
}

// The start-of-sequence block of the decoder's embedding ring: 128 copies of E[SOS].
__global__ void k_sos_block(int8_t *dst, const int8_t *emb)
{
    reinterpret_cast<int4 *>(dst)[threadIdx.x] =
        reinterpret_cast<const int4 *>(emb + (size_t)SC_SOS * EMB_DIM)[threadIdx.x & (EMB_DIM / 16 - 1)];
}

// The decoder schedule of one launch on SM pairs (see DecSeg).  Pair-tile i holds rows
// 256 i .. 256 i + 255 of the length-sorted order and lasts as many steps as its first row.
// Pair-tiles go, longest first, to the pair with the least total steps so far (ties: the
// lowest pair) and, within it, to the lane with the fewest steps (ties: the lowest lane), so
// pairs finish together and each keeps its six lanes busy for as long as it can.  Each pair's
// timeline is then cut at every step where a lane changes pair-tile.
struct DecSchedule {
    std::vector<DecSeg> segs;
    std::vector<int32_t> pair_seg;
};

static DecSchedule build_decode_schedule(const std::vector<int32_t> &pt_len, int pairs)
{
    const int n_pt = (int)pt_len.size();
    std::vector<int64_t> pair_load(pairs, 0);
    std::vector<std::array<int64_t, KT2>> lane_load(pairs);
    std::vector<std::array<std::vector<int32_t>, KT2>> queue(pairs);
    for (auto &l : lane_load) l.fill(0);
    // min-heap on (steps so far, pair)
    std::priority_queue<std::pair<int64_t, int>, std::vector<std::pair<int64_t, int>>, std::greater<>> heap;
    for (int i = 0; i < pairs; ++i) heap.push({0, i});
    for (int pt = 0; pt < n_pt; ++pt) {
        const auto top = heap.top();
        heap.pop();
        const int pr = top.second;
        int lane = 0;
        for (int t = 1; t < KT2; ++t)
            if (lane_load[pr][t] < lane_load[pr][lane]) lane = t;
        queue[pr][lane].push_back(pt);
        lane_load[pr][lane] += pt_len[pt];
        pair_load[pr] += pt_len[pt];
        heap.push({pair_load[pr], pr});
    }
    DecSchedule out;
    out.pair_seg.push_back(0);
    for (int pr = 0; pr < pairs; ++pr) {
        int idx[KT2] = {};
        int32_t start[KT2] = {};
        int32_t gs = 0;
        while (true) {
            int32_t next = INT32_MAX;
            for (int t = 0; t < KT2; ++t)
                if (idx[t] < (int)queue[pr][t].size())
                    next = std::min(next, start[t] + pt_len[queue[pr][t][idx[t]]]);
            if (next == INT32_MAX) break;
            DecSeg sg;
            sg.s0 = gs;
            sg.s1 = next;
            for (int t = 0; t < KT2; ++t) {
                const bool on = idx[t] < (int)queue[pr][t].size();
                sg.pt[t] = on ? queue[pr][t][idx[t]] : -1;
                sg.start[t] = on ? start[t] : 0;
            }
            out.segs.push_back(sg);
            for (int t = 0; t < KT2; ++t)
                if (idx[t] < (int)queue[pr][t].size() && start[t] + pt_len[queue[pr][t][idx[t]]] == next) {
                    ++idx[t];
                    start[t] = next;
                }
            gs = next;
        }
        out.pair_seg.push_back((int32_t)out.segs.size());
    }
    return out;
}

// Small-batch decoding (sc_mlp_small.cuh): one cluster of SMALL_C CTAs per tile of 128 rows, as
// many clusters as tiles up to one per SMALL_C SMs (further tiles run after those, in order).
static void small_decode(sc_model *m, const int64_t *order, int64_t n_rows, const int64_t *sorted_len,
                         const int64_t *lengths, DecState *state, const uint32_t *words, uint8_t *tokens_out,
                         const int64_t *out_off, uint8_t *errors, cudaStream_t s)
{
    const int64_t n_tiles = (n_rows + TM - 1) / TM;
    if (n_tiles > INT32_MAX / SMALL_C) throw CudaError{cudaErrorInvalidValue, "small_decode: too many rows"};
    const int clusters = (int)std::min<int64_t>(n_tiles, std::max(1, m->num_sms / SMALL_C));
    std::vector<int32_t> steps(n_tiles);
    int64_t work = 0;
    for (int64_t t = 0; t < n_tiles; ++t) steps[t] = (int32_t)sorted_len[t * TM];
    for (int64_t j = 0; j < n_rows; ++j) work += sorted_len[j];
    int32_t *d_steps = (int32_t *)m->ws_sched.get(sizeof(int32_t) * n_tiles, s);
    SC_CUDA(cudaMemcpyAsync(d_steps, steps.data(), sizeof(int32_t) * n_tiles, cudaMemcpyHostToDevice, s));
    ProfScope ps(m->prof, KK_SMALL_DECODE, s, work);
    SmallParams p{};
    // embedding ring: [clusters][WIN] blocks of 128 rows x 128 B, then the SOS block
    const int64_t ring_rows = (int64_t)clusters * TM * WIN;
    int8_t *ring = (int8_t *)m->ws_ering.get((size_t)(ring_rows + TM) * KB, s);
    k_sos_block<<<1, TM * KB / 16, 0, s>>>(ring + ring_rows * KB, m->emb);
    SC_LAUNCH_CHECK();
    count_launch();
    p.ering = make_tmap(ring, KB, ring_rows + TM, KB, TM);
    p.ering_ptr = ring;
    p.ering_sos_row = ring_rows;
    p.num_layers = m->num_layers;
    for (int l = 0; l < m->num_layers; ++l) {
        p.w[l] = m->small_wmaps[l];
        p.bias[l] = m->layers[l].bias;
        p.rq[l] = m->layers[l].rq;
        p.in_dim[l] = m->layers[l].in_dim;
        p.out_dim[l] = m->layers[l].out_dim;
    }
    p.lut = m->lut;
    p.emb = m->emb;
    p.n_tiles = (int)n_tiles;
    p.tile_steps = d_steps;
    p.order = order;
    p.n_rows = n_rows;
    p.lengths = lengths;
    p.state = state;
    p.words = words;
    p.tokens_out = tokens_out;
    p.out_off = out_off;
    p.errors = errors;
    if (m->trace_cap > 0) {
        SC_CUDA(cudaMemsetAsync(m->trace_count, 0, 8 * sizeof(unsigned int), s));
        p.trace = m->trace_buf;
        p.trace_count = m->trace_count;
        p.trace_cap = m->trace_cap;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(clusters * SMALL_C));
    cfg.blockDim = dim3(SMALL_THREADS);
    cfg.dynamicSmemBytes = SmallCfg::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SMALL_C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (p.trace != nullptr) SC_CUDA(cudaLaunchKernelEx(&cfg, k_small_decode<true>, p));
    else SC_CUDA(cudaLaunchKernelEx(&cfg, k_small_decode<false>, p));
    SC_LAUNCH_CHECK();
    count_launch();
}

void fused_decode(sc_model *m, const int64_t *order, int64_t n_rows, const int64_t *sorted_len,
                  const int64_t *lengths, DecState *state, const uint32_t *words, uint8_t *tokens_out,
                  const int64_t *out_off, uint8_t *errors, cudaStream_t s)
{
    if (n_rows <= 0) return;
    const int64_t n_tiles = (n_rows + TM - 1) / TM;
    if (use_pairs(m) && (m->mlp_path == 5 || (m->mlp_path == 0 && n_tiles * SMALL_C <= m->num_sms))) {
        // too few tiles to fill the SM pairs' lanes: each tile on a cluster of eight SMs
        // (path 1 keeps every batch on the pairs, path 5 puts every batch here: cross-checks)
        small_decode(m, order, n_rows, sorted_len, lengths, state, words, tokens_out, out_off, errors, s);
        return;
    }
    if (use_pairs(m)) {
        // one launch for the whole batch: every pair-tile is queued on a lane of some SM pair
        const int64_t n_pt = (n_tiles + 1) / 2;
        if (n_pt > INT32_MAX / 2) throw CudaError{cudaErrorInvalidValue, "fused_decode: too many rows"};
        std::vector<int32_t> pt_len(n_pt);
        int64_t work = 0;
        for (int64_t i = 0; i < n_pt; ++i) pt_len[i] = (int32_t)sorted_len[i * 2 * TM];
        for (int64_t j = 0; j < n_rows; ++j) work += sorted_len[j];
        const int pairs = (int)std::min<int64_t>(n_pt, m->num_sms / 2);
        const int grid = 2 * pairs;
        const DecSchedule sched = build_decode_schedule(pt_len, pairs);
        const size_t seg_bytes = sizeof(DecSeg) * sched.segs.size();
        uint8_t *sd = (uint8_t *)m->ws_sched.get(seg_bytes + sizeof(int32_t) * sched.pair_seg.size(), s);
        SC_CUDA(cudaMemcpyAsync(sd, sched.segs.data(), seg_bytes, cudaMemcpyHostToDevice, s));
        SC_CUDA(cudaMemcpyAsync(sd + seg_bytes, sched.pair_seg.data(), sizeof(int32_t) * sched.pair_seg.size(),
                                cudaMemcpyHostToDevice, s));
        ProfScope ps(m->prof, KK_FUSED_DECODE, s, work);
        Fused2Params p{};
        fused2_common(m, p, grid, s);
        // embedding ring: [grid][kt2][WIN] blocks of 128 rows x 128 B, then the SOS block
        const int64_t ring_rows = (int64_t)grid * kt2<true>() * WIN * TM;
        int8_t *ring = (int8_t *)m->ws_ering.get((size_t)(ring_rows + TM) * KB, s);
        k_sos_block<<<1, TM * KB / 16, 0, s>>>(ring + ring_rows * KB, m->emb);
        SC_LAUNCH_CHECK();
        count_launch();
        p.ering = make_tmap(ring, KB, ring_rows + TM, KB, TM);
        p.ering_ptr = ring;
        p.ering_sos_row = ring_rows;
        p.n_tiles = (int)n_tiles;
        p.order = order;
        p.n_rows = n_rows;
        p.segs = reinterpret_cast<const DecSeg *>(sd);
        p.pair_seg = reinterpret_cast<const int32_t *>(sd + seg_bytes);
        p.lengths = lengths;
        p.state = state;
        p.words = words;
        p.tokens_out = tokens_out;
        p.out_off = out_off;
        p.errors = errors;
        launch_pairs<true>(p, grid, s);
        SC_LAUNCH_CHECK();
        count_launch();
        return;
    }
    // single-SM kernels (a cross-check path): launches of at most grid * KT tiles, chunks split
    // evenly over as few launches as that capacity allows
    const int64_t cap = (int64_t)m->num_sms * KT * TM;
    const int64_t launches = (n_rows + cap - 1) / cap;
    const int64_t per = (n_rows + launches - 1) / launches;
    std::vector<int32_t> maxlen;
    for (int64_t g0 = 0; g0 < n_rows; g0 += per) {
        const int64_t g1 = std::min(n_rows, g0 + per);
        maxlen.clear();
        int64_t work = 0;
        for (int64_t j = g0; j < g1; j += TM) maxlen.push_back((int32_t)sorted_len[j]);
        for (int64_t j = g0; j < g1; ++j) work += sorted_len[j];
        int32_t *d_maxlen = (int32_t *)m->ws_sched.get(sizeof(int32_t) * maxlen.size(), s);
        SC_CUDA(cudaMemcpyAsync(d_maxlen, maxlen.data(), sizeof(int32_t) * maxlen.size(), cudaMemcpyHostToDevice, s));
        const int64_t g_tiles = (g1 - g0 + TM - 1) / TM;
        ProfScope ps(m->prof, KK_FUSED_DECODE, s, work);
        const int grid = (int)std::min<int64_t>(g_tiles, m->num_sms);
        FusedParams p{};
        fused_common(m, p, grid, s);
        p.n_tiles = (int)g_tiles;
        p.order = order + g0;
        p.n_rows = g1 - g0;
        p.tile_maxlen = d_maxlen;
        p.lengths = lengths;
        p.state = state + g0;
        p.words = words;
        p.tokens_out = tokens_out;
        p.out_off = out_off;
        p.errors = errors;
        k_fused<true><<<grid, 256, FCfg<true>::SMEM, s>>>(p);
        SC_LAUNCH_CHECK();
        count_launch();
        SC_CUDA(cudaStreamSynchronize(s));       // tile lengths are rebuilt for the next launch
    }
}

namespace {

// Failure-detection self test: one warp waits on an mbarrier and on a shared-memory
// counter that nothing signals.  Both waits give up after their time limit, record
// the timeout in the device error flag and return, so the kernel ends normally.
__global__ void k_wait_selftest(int *done)
{
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t cnt;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        cnt = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const bool a = mbar_wait(&bar, 0);          // no arrival ever comes
        const bool b = counter_wait(&cnt, 1);       // no increment ever comes
        *done = (a ? 1 : 0) | (b ? 2 : 0) | 4;
    }
}

}  // namespace

int wait_selftest(cudaStream_t s, int *done_d)
{
    k_wait_selftest<<<1, 32, 0, s>>>(done_d);
    SC_LAUNCH_CHECK();
    count_launch();
    int done = 0;
    SC_CUDA(cudaMemcpyAsync(&done, done_d, sizeof(int), cudaMemcpyDeviceToHost, s));
    SC_CUDA(cudaStreamSynchronize(s));
    return done;
}

int read_device_error(int clear)
{
    int v = 0;
    SC_CUDA(cudaMemcpyFromSymbol(&v, tc::g_device_error, sizeof(int)));
    if (clear && v) {
        int z = 0;
        SC_CUDA(cudaMemcpyToSymbol(tc::g_device_error, &z, sizeof(int)));
    }
    return v;
}

}  // namespace sc
