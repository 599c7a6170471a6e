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

#include "sc_internal.h"
#include "sc_tc.cuh"

namespace sc {
namespace {

using namespace tc;

constexpr int TM = 128;          // rows per tile
constexpr int TN = 256;          // output columns per tile
constexpr int KB = 128;          // bytes of K per stage
constexpr int A_BYTES = TM * KB;             // 16 KB
constexpr int B_BYTES = TN * KB;             // 32 KB
constexpr int EMB_ROWS = 257;
constexpr int EMB_DIM = 128;
constexpr int EMB_BYTES = EMB_ROWS * EMB_DIM;

template <bool GATHER>
struct Cfg {
    static constexpr int STAGES = GATHER ? 3 : 4;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int OFF_EMB = STAGES * STAGE_BYTES;
    static constexpr int OFF_BIAS = OFF_EMB + (GATHER ? ((EMB_BYTES + 1023) / 1024) * 1024 : 0);
    static constexpr int OFF_BAR = OFF_BIAS + TN * 4;
    static constexpr int OFF_TMEM = OFF_BAR + (2 * STAGES + 2) * 8;
    static constexpr int SMEM = OFF_TMEM + 16 + 1024;   // + alignment slack
};

template <bool GATHER>
__global__ void __launch_bounds__(256, 1) k_linear_tc(
    const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
    const int16_t *__restrict__ windows, int window, const int8_t *__restrict__ emb,
    const int32_t *__restrict__ bias, Requant rq, int8_t *__restrict__ y, int64_t M, int N, int K)
{
    using C = Cfg<GATHER>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = (uint64_t *)(smem + C::OFF_BAR);
    uint64_t *empty = full + C::STAGES;
    uint64_t *acc_full = empty + C::STAGES;
    uint32_t *tmem_slot = (uint32_t *)(smem + C::OFF_TMEM);
    int32_t *bias_s = (int32_t *)(smem + C::OFF_BIAS);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m0 = (int64_t)blockIdx.x * TM;
    const int n0 = blockIdx.y * TN;
    const int nkb = K / KB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], GATHER ? 1 + 64 : 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
        if (!GATHER) prefetch_tmap(&tmap_x);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, TN);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < TN; i += blockDim.x) bias_s[i] = bias[n0 + i];
    if (GATHER) {
        const int4 *src = reinterpret_cast<const int4 *>(emb);
        int4 *dst = reinterpret_cast<int4 *>(smem + C::OFF_EMB);
        for (int i = threadIdx.x; i < EMB_BYTES / 16; i += blockDim.x) dst[i] = src[i];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_acc = *tmem_slot;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % C::STAGES;
            const uint32_t ph = (kb / C::STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1)) break;
            uint8_t *a_st = smem + s * C::STAGE_BYTES;
            uint8_t *b_st = a_st + A_BYTES;
            mbar_arrive_expect_tx(&full[s], GATHER ? B_BYTES : B_BYTES + A_BYTES);
            tma_load_2d(b_st, &tmap_w, &full[s], kb * KB, n0);
            if (!GATHER) tma_load_2d(a_st, &tmap_x, &full[s], kb * KB, (int32_t)m0);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        constexpr uint32_t idesc = idesc_i8(TM, TN);
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % C::STAGES;
            const uint32_t ph = (kb / C::STAGES) & 1;
            if (!mbar_wait(&full[s], ph)) { ok = false; break; }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(smem + s * C::STAGE_BYTES);
            const uint32_t b_addr = a_addr + A_BYTES;
#pragma unroll
            for (int k = 0; k < KB / 32; ++k)
                mma_i8(tmem_acc, smem_desc_sw128(a_addr + 32 * k), smem_desc_sw128(b_addr + 32 * k), idesc,
                       (kb | k) != 0);
            mma_commit(&empty[s]);
        }
        mma_commit(acc_full);
        (void)ok;
    } else if (GATHER && (warp == 2 || warp == 3)) {
        // ---- activation-tile builders for layer 0
        const int t = threadIdx.x - 64;       // 0..63
        const int j = t & 7;                  // 16-byte chunk of the 128-byte row
        const int r0 = t >> 3;                // first row, then every 8th
        const uint8_t *emb_s = smem + C::OFF_EMB;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % C::STAGES;
            const uint32_t ph = (kb / C::STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1)) break;
            uint8_t *a_st = smem + s * C::STAGE_BYTES;
#pragma unroll 4
            for (int r = r0; r < TM; r += 8) {
                const int64_t row = m0 + r;
                const int tok = row < M ? windows[row * window + kb] : 256;
                const int4 v = *reinterpret_cast<const int4 *>(emb_s + tok * EMB_DIM + j * 16);
                *reinterpret_cast<int4 *>(a_st + sw128_offset(r, j)) = v;
            }
            fence_proxy_async_smem();
            mbar_arrive(&full[s]);
        }
    } else if (warp >= 4) {
        // ---- epilogue
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const int64_t row = m0 + r;
        const bool ok = __all_sync(0xffffffffu, mbar_wait(acc_full, 0));
        if (ok) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < TN / 32; ++c) {
                uint32_t v[32];
                tmem_ld32(tmem_acc + ((uint32_t)(q * 32) << 16) + c * 32, v);
                tmem_ld_wait();
                uint32_t packed[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    uint32_t p = 0;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const int col = c * 32 + i * 4 + b;
                        const int32_t o = requant((int32_t)v[i * 4 + b], bias_s[col], rq);
                        p |= ((uint32_t)(o & 0xFF)) << (8 * b);
                    }
                    packed[i] = p;
                }
                if (row < M) {
                    uint4 *dst = reinterpret_cast<uint4 *>(y + row * N + n0 + c * 32);
                    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_acc, TN);
    }
}

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

bool mlp_tc_supported(const sc_model *m)
{
    if (m->emb_dim != EMB_DIM || m->window * EMB_DIM != m->layers[0].in_dim) return false;
    for (auto &L : m->layers)
        if (L.in_dim % KB || L.out_dim % TN) return false;
    return true;
}

void mlp_tc_prepare(sc_model *m)
{
    auto &maps = m->tc_wmaps;
    maps.clear();
    for (auto &L : m->layers) maps.push_back(make_tmap(L.w, L.in_dim, L.out_dim, L.in_dim, TN));
    static bool attr = false;
    if (!attr) {
        SC_CUDA(cudaFuncSetAttribute(k_linear_tc<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<true>::SMEM));
        SC_CUDA(cudaFuncSetAttribute(k_linear_tc<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<false>::SMEM));
        attr = true;
    }
}

void mlp_tc(sc_model *m, const int16_t *windows, int64_t rows, int8_t *logits, cudaStream_t s)
{
    if (rows <= 0) return;
    auto &maps = m->tc_wmaps;
    int max_w = 0;
    for (auto &L : m->layers) max_w = L.out_dim > max_w ? L.out_dim : max_w;
    int8_t *bufs[2] = {
        (int8_t *)m->ws_act0.get((size_t)rows * max_w, s),
        (int8_t *)m->ws_act1.get((size_t)rows * max_w, s),
    };
    const int8_t *x = nullptr;
    for (int l = 0; l < m->num_layers; ++l) {
        const LayerDev &L = m->layers[l];
        int8_t *yb = (l == m->num_layers - 1) ? logits : bufs[l & 1];
        dim3 grid((unsigned)((rows + TM - 1) / TM), L.out_dim / TN);
        ProfScope ps(m->prof, l == 0 ? KK_LAYER0 : (l == m->num_layers - 1 ? KK_LAST : KK_HIDDEN), s, rows);
        if (l == 0) {
            k_linear_tc<true><<<grid, 256, Cfg<true>::SMEM, s>>>(maps[0], maps[0], windows, m->window, m->emb, L.bias,
                                                               L.rq, yb, rows, L.out_dim, L.in_dim);
        } else {
            CUtensorMap xm = make_tmap(x, L.in_dim, rows, L.in_dim, TM);
            k_linear_tc<false><<<grid, 256, Cfg<false>::SMEM, s>>>(maps[l], xm, nullptr, 0, nullptr, L.bias, L.rq,
                                                                 yb, rows, L.out_dim, L.in_dim);
        }
        SC_LAUNCH_CHECK();
        count_launch();
        x = yb;
    }
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
