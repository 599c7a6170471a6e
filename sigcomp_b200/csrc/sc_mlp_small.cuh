// Small-batch decoder: one 128-row tile per cluster of SMALL_C CTAs (tcgen05 cta_group::1).
//
// The pair kernel (sc_mlp_fused2.cuh) gives each tile of 128 rows one SM and hides the latency of
// a step's nine dependent layers behind the other tiles of its SM.  A batch of a few hundred
// chunks has too few tiles for that: three SM pairs would run one tile each, one step every
// ~110 us.  Here every tile runs on a cluster of eight CTAs instead, each computing 1/8 of every
// layer's outputs (N = 64 of 512, 32 of the last layer's 256), so a step's work is spread over
// eight SMs, and a layer's output slices are exchanged in distributed shared memory:
//   - every CTA holds the tile's activations in two resident buffers (B0, B1: 128 rows x 512 B,
//     four 128-byte-swizzled K blocks, the MMA's A operand layout); layer L >= 1 reads
//     B[(L-1) & 1], and the epilogue of layer L < 8 writes its 64-column slice into B[L & 1] of
//     every CTA of the cluster (st.shared::cluster), then arrives on an `xbar` mbarrier of every
//     CTA, on which that CTA's MMA issuer waits before the next layer;
//   - consecutive exchanges alternate between two barriers: a warp makes its eight arrivals for
//     exchange k before its CTA can start on exchange k+1, but another CTA's barrier may not have
//     seen them all yet, and an arrival for k+1 must never count toward k there; one for k+2
//     cannot come before every CTA has seen all of k+1, hence all of k;
//   - the producer streams only weights for layers >= 1 (8 KB per K block, a ring that runs up
//     to 2.5 layers ahead); layer 0's A operand, the 64-token window, comes by TMA from the
//     cluster's embedding ring in global memory through 24 KB stages that overlay B1, which is
//     free during layer 0 (the producer switches between the two stage rings only after the one
//     it leaves is consumed: every MMA that read it, and hence layer 8's reads of B1, completed);
//   - the last layer's logit slices are gathered in rank 0's B0, free by then (`lbar`); rank 0's
//     epilogue runs the coder step of every row (the pair kernel's frequency pass, search and
//     range-decoder update), appends the decoded tokens' embedding rows to the ring and releases
//     the next step in every CTA (`rbar`).
// Layer 0 of step s reads window positions 0..62 from ring slots written at earlier steps, so its
// loads and MMAs start while rank 0 is still decoding step s-1 (its coder scratch and the
// accumulator are separate TMEM columns); only position 63, the token being decoded, waits for
// rbar.  Every buffer is written only after a signal that proves its previous contents consumed
// in every CTA: a CTA writes B[L & 1] at layer L after its own layer-L MMAs, which waited for
// every CTA's layer L-1 slices, each sent after that CTA's layer L-1 MMAs (the last readers of
// B[L & 1]) completed; layer 0's writes to B0 come after rbar of the previous step, which rank 0
// sends after the coder has read the logits out of its B0.  No TMA load uses cluster multicast;
// every wait is bounded.
#pragma once

namespace sc {

constexpr int SMALL_C = 8;                           // CTAs per tile
constexpr int SMALL_NS = MAX_N / SMALL_C;            // 64 output columns per CTA (hidden layers)
constexpr int SMALL_B = TM * MAX_N;                  // 64 KB: one resident activation buffer
constexpr int SMALL_ST0 = A_BYTES + SMALL_NS * KB;   // 24 KB: a layer-0 stage (ring block + weights)
constexpr int SMALL_STAGES0 = 6;                     // layer-0 stages, over B1 and beyond
constexpr int SMALL_ST1 = SMALL_NS * KB;             // 8 KB: a weight slice of one K block
constexpr int SMALL_STAGES1 = 10;                    // weight stages of layers >= 1
constexpr int SMALL_THREADS = 32 * 6;                // producer, MMA, four epilogue warps
// TMEM: columns 0..255 are rank 0's coder scratch (packed logits, cached frequencies), the
// accumulator (64 columns) lives after them, so a step's layer 0 can run during the coder step
constexpr int SMALL_TMEM_COLS = 512;
constexpr int SMALL_ACC_COL = 256;

struct SmallParams {
    CUtensorMap w[FMAX_LAYERS];       // weights, box (out_dim / SMALL_C) rows x 128 B
    CUtensorMap ering;                // embedding ring, box 128 rows x 128 B
    int8_t *ering_ptr;                // [clusters][WIN][128][128], then the start-of-sequence block
    int64_t ering_sos_row;
    const int32_t *bias[FMAX_LAYERS];
    Requant rq[FMAX_LAYERS];
    int in_dim[FMAX_LAYERS];
    int out_dim[FMAX_LAYERS];
    int num_layers;
    const uint64_t *lut;
    const int8_t *emb;
    int n_tiles;                      // tiles of 128 rows of `order`; cluster k runs tiles k, k + n_clusters, ...
    const int32_t *tile_steps;        // steps of each tile: the length of its longest chunk
    const int64_t *order;
    int64_t n_rows;
    const int64_t *lengths;
    DecState *state;
    const uint32_t *words;
    uint8_t *tokens_out;
    const int64_t *out_off;
    uint8_t *errors;
    // optional unit trace of CTAs 0 and 1 (ranks 0 and 1 of the first cluster), laid out as the
    // pair kernels' trace: [2][4 roles][trace_cap / 4][2]
    unsigned long long *trace;
    unsigned int *trace_count;
    int trace_cap;
};

// Trace record (role 0 producer, 1 MMA, 2 epilogue, 3 rank 0's coder step; events 0 begin,
// 1 dependency satisfied, 2 end), written by one thread per role into its own region; compiled
// out of the untraced kernel.
template <bool TRACE>
__device__ __forceinline__ void small_trace(const SmallParams &p, unsigned int &n, int role, int ev, int L, int step)
{
    if constexpr (TRACE) {
        if (blockIdx.x >= 2 || n >= (unsigned int)p.trace_cap / 4) return;
        unsigned long long *r = p.trace + (((size_t)blockIdx.x * 4 + role) * (p.trace_cap / 4) + n++) * 2;
        r[0] = globaltimer_ns();
        r[1] = (unsigned long long)role | ((unsigned long long)ev << 4) | ((unsigned long long)L << 8) |
               ((unsigned long long)step << 32);
    }
}

struct SmallCfg {
    static constexpr int OFF_B0 = 0;
    static constexpr int OFF_B1 = SMALL_B;                               // 64 KB
    static constexpr int OFF_RING0 = OFF_B1;                             // layer-0 stages over B1...
    static constexpr int OFF_RING1 = OFF_B1 + SMALL_B;                   // ...weight stages after it
    static constexpr int END_RINGS = OFF_RING0 + SMALL_STAGES0 * SMALL_ST0;   // 208 KB
    static_assert(OFF_RING1 + SMALL_STAGES1 * SMALL_ST1 <= END_RINGS, "weight stages inside the ring area");
    static constexpr int OFF_BIAS = END_RINGS;                           // this CTA's bias slices
    static constexpr int OFF_LUT = OFF_BIAS + FMAX_LAYERS * SMALL_NS * 4;
    static constexpr int OFF_BAR = OFF_LUT + 256 * 8;
    // full/empty of both rings, acc_full, acc_empty, xbar[2], lbar, rbar, drain
    static constexpr int NBAR = 2 * SMALL_STAGES0 + 2 * SMALL_STAGES1 + 7;
    static constexpr int OFF_CNT = OFF_BAR + NBAR * 8;                   // epilogue warps' slice counter
    static constexpr int OFF_TMEM = OFF_CNT + 16;
    static constexpr int SMEM = OFF_TMEM + 16 + 1024;
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Walk this cluster's (tile, step, layer) units in the order every role of every CTA follows.
template <typename F>
__device__ __forceinline__ void for_each_small_unit(const SmallParams &p, F &&f)
{
    const int n_clusters = gridDim.x / SMALL_C;
    for (int tile = blockIdx.x / SMALL_C; tile < p.n_tiles; tile += n_clusters) {
        const int steps = p.tile_steps[tile];
        for (int step = 0; step < steps; ++step)
            for (int L = 0; L < p.num_layers; ++L)
                if (!f(tile, step, L)) return;
    }
}

// Bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory to the shared memory of a
// CTA of the cluster, completing on an mbarrier of that CTA (both shared::cluster addresses): the
// copy engine moves a whole slice with one instruction, where per-thread remote stores would each
// pay the cluster network's round trip.
__device__ __forceinline__ void bulk_copy_to_cluster(uint32_t dst_cluster, const void *src, uint32_t bytes,
                                                     uint32_t bar_cluster)
{
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst_cluster), "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
                 : "memory");
}

// K-major operand without swizzle: 8-row x 16-byte core matrices of 128 contiguous bytes, the
// core matrices of one 16-byte K chunk stacked over the rows at `sbo` bytes, consecutive K chunks
// `lbo` bytes apart.  The resident activation buffers use lbo = 2048 (a K chunk of all 128 rows)
// and sbo = 128, so byte k of row r sits at (k / 16) * 2048 + r * 16 + k % 16 and a CTA's 64
// columns are one contiguous 8 KB block.
__device__ __forceinline__ uint64_t smem_desc_noswz(uint32_t smem_addr, uint32_t lbo, uint32_t sbo)
{
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFF) >> 4);       // start address  [0,14)
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;         // leading byte offset: next K core matrix
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;         // stride byte offset: next 8 rows
    d |= (uint64_t)1 << 46;                             // descriptor version (sm_100)
    return d;                                           // swizzle mode 0: none
}

constexpr int SMALL_KCHUNK = TM * 16;                // 2 KB: one 16-byte K chunk of all 128 rows

template <bool TRACE>
__global__ void __launch_bounds__(SMALL_THREADS, 1) k_small_decode(const __grid_constant__ SmallParams p)
{
    using C = SmallCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint64_t *full0 = bars, *empty0 = full0 + SMALL_STAGES0;       // layer-0 stages
    uint64_t *full1 = empty0 + SMALL_STAGES0, *empty1 = full1 + SMALL_STAGES1;   // weight stages
    uint64_t *acc_full = empty1 + SMALL_STAGES1, *acc_empty = acc_full + 1;
    uint64_t *xbar = acc_empty + 1;   // [2]: every CTA's slice of a layer's output is in this CTA's buffer
    uint64_t *lbar = xbar + 2;        // rank 0: every CTA's last-layer logit slice is in its B0
    uint64_t *rbar = lbar + 1;        // rank 0 appended the step's tokens to the ring
    uint64_t *drain = rbar + 1;       // the MMA issuer's last commit: TMEM is freed after it
    uint32_t *tmem_slot = (uint32_t *)(smem + C::OFF_TMEM);
    // +1 per epilogue warp once its rows of a unit's output slice are in this CTA's shared memory
    uint32_t *slice_cnt = (uint32_t *)(smem + C::OFF_CNT);
    int32_t *bias_s = (int32_t *)(smem + C::OFF_BIAS);
    uint64_t *lut_s = (uint64_t *)(smem + C::OFF_LUT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NL = p.num_layers;
    const uint32_t rank = cluster_ctarank();
    const int ring_block0 = (blockIdx.x / SMALL_C) * WIN;   // this cluster's first embedding-ring block

    if (threadIdx.x == 0) {
        for (int s = 0; s < SMALL_STAGES0; ++s) {
            mbar_init(&full0[s], 1);
            mbar_init(&empty0[s], 1);
        }
        for (int s = 0; s < SMALL_STAGES1; ++s) {
            mbar_init(&full1[s], 1);
            mbar_init(&empty1[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 4);
        // the exchanges: one local arrival (with the bytes the seven peers' copies bring)
        mbar_init(&xbar[0], 1);
        mbar_init(&xbar[1], 1);
        mbar_init(lbar, 1);
        mbar_init(rbar, 4);                            // rank 0's epilogue warps
        mbar_init(drain, 1);
        *slice_cnt = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, SMALL_TMEM_COLS);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < SC_VOCAB; i += blockDim.x) lut_s[i] = p.lut[i];
    for (int l = 0; l < NL; ++l) {
        const int ns = p.out_dim[l] / SMALL_C;
        for (int i = threadIdx.x; i < ns; i += blockDim.x) bias_s[l * SMALL_NS + i] = p.bias[l][(int)rank * ns + i];
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();                   // every CTA's barriers exist before any remote arrival or store
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer: layer 0's window blocks and weights, the other layers' weights
            uint32_t it0 = 0, it1 = 0, rw = 0;           // blocks issued per stage ring, rbar waits
            int last_ring = -1;
            unsigned int tn = 0;
            bool aborted = false, first = true;
            const uint64_t ring_policy = l2_policy_evict_first();
            for_each_small_unit(p, [&](int tile, int step, int L) -> bool {
                const int nkb = p.in_dim[L] / KB;
                const int ns = p.out_dim[L] / SMALL_C;
                const int rg = L == 0 ? 0 : 1;
                small_trace<TRACE>(p, tn, 0, 0, L, step);
                if (rg != last_ring && last_ring >= 0) {
                    // the two rings share memory: the one left behind is consumed (its last
                    // block's MMAs completed, and MMAs complete in order) before the other refills it
                    const uint32_t i = (last_ring ? it1 : it0) - 1;
                    const bool ok = last_ring ? mbar_wait_cluster(&empty1[i % SMALL_STAGES1], (i / SMALL_STAGES1) & 1)
                                              : mbar_wait_cluster(&empty0[i % SMALL_STAGES0], (i / SMALL_STAGES0) & 1);
                    if (!ok) return !(aborted = true);
                }
                last_ring = rg;
                if (L == 0) {
                    for (int kb = 0; kb < nkb; ++kb) {
                        const int s = it0 % SMALL_STAGES0;
                        if (!mbar_wait_cluster(&empty0[s], ((it0 / SMALL_STAGES0) & 1) ^ 1)) return !(aborted = true);
                        uint8_t *st = smem + C::OFF_RING0 + s * SMALL_ST0;
                        mbar_arrive_expect_tx(&full0[s], A_BYTES + ns * KB);
                        tma_load_2d(st + A_BYTES, &p.w[0], &full0[s], kb * KB, (int)rank * ns);
                        ++it0;
                        if (kb == nkb - 1) {
                            // window positions 0..62 hold tokens of earlier steps, already in the
                            // ring; the last one is the token rank 0 is decoding now.  Rank 0
                            // releases every step, a tile's last one too: every layer 0 but the
                            // cluster's very first consumes one release.
                            if (!first && !mbar_wait_cluster(rbar, rw & 1)) return !(aborted = true);
                            rw += first ? 0 : 1;
                            first = false;
                            small_trace<TRACE>(p, tn, 0, 1, L, step);
                        }
                        // window position kb holds token step - 64 + kb (start-of-sequence before 0)
                        const int tau = step - WIN + kb;
                        const int row = tau < 0 ? (int)p.ering_sos_row : (ring_block0 + (tau & (WIN - 1))) * TM;
                        tma_load_2d_hint(st, &p.ering, &full0[s], 0, row, ring_policy);
                    }
                } else {
                    small_trace<TRACE>(p, tn, 0, 1, L, step);
                    for (int kb = 0; kb < nkb; ++kb) {
                        const int s = it1 % SMALL_STAGES1;
                        if (!mbar_wait_cluster(&empty1[s], ((it1 / SMALL_STAGES1) & 1) ^ 1)) return !(aborted = true);
                        uint8_t *st = smem + C::OFF_RING1 + s * SMALL_ST1;
                        mbar_arrive_expect_tx(&full1[s], ns * KB);
                        tma_load_2d(st, &p.w[L], &full1[s], kb * KB, (int)rank * ns);
                        ++it1;
                    }
                }
                small_trace<TRACE>(p, tn, 0, 2, L, step);
                return true;
            });
            if (TRACE && blockIdx.x < 2) p.trace_count[blockIdx.x * 4 + 0] = tn;
            if (aborted) {
                // loads already issued may still be landing in shared memory: wait (bounded) for the
                // full phases of each ring's last stages, then give stragglers time before the CTA ends
                for (uint32_t i = it0 > (uint32_t)SMALL_STAGES0 ? it0 - SMALL_STAGES0 : 0; i < it0; ++i)
                    mbar_wait_cluster_drain(&full0[i % SMALL_STAGES0], (i / SMALL_STAGES0) & 1);
                for (uint32_t i = it1 > (uint32_t)SMALL_STAGES1 ? it1 - SMALL_STAGES1 : 0; i < it1; ++i)
                    mbar_wait_cluster_drain(&full1[i % SMALL_STAGES1], (i / SMALL_STAGES1) & 1);
                spin_ns(100000);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: D[128 x ns] = A[128 x K] * W_slice[ns x K]^T, one accumulator
            uint32_t it0 = 0, it1 = 0, uu = 0, xm = 0;
            unsigned int tn = 0;
            const uint32_t d = tmem_base + SMALL_ACC_COL;
            for_each_small_unit(p, [&](int tile, int step, int L) -> bool {
                const int nkb = p.in_dim[L] / KB;
                const uint32_t idesc = idesc_i8(TM, p.out_dim[L] / SMALL_C);
                small_trace<TRACE>(p, tn, 1, 0, L, step);
                if (!mbar_wait_cluster(acc_empty, (uu & 1) ^ 1)) return false;
                if (L != 0) {
                    // every CTA's slice of layer L-1's output is in this CTA's buffer
                    if (!mbar_wait_cluster(&xbar[xm & 1], (xm >> 1) & 1)) return false;
                    ++xm;
                }
                small_trace<TRACE>(p, tn, 1, 1, L, step);
                tc_fence_after();
                if (L == 0) {
                    for (int kb = 0; kb < nkb; ++kb, ++it0) {
                        const int s = it0 % SMALL_STAGES0;
                        if (!mbar_wait_cluster(&full0[s], (it0 / SMALL_STAGES0) & 1)) return false;
                        tc_fence_after();
                        const uint32_t st = smem_u32(smem + C::OFF_RING0 + s * SMALL_ST0);
#pragma unroll
                        for (int k = 0; k < KB / 32; ++k)
                            mma_i8(d, smem_desc_sw128(st + 32 * k), smem_desc_sw128(st + A_BYTES + 32 * k), idesc,
                                   (kb || k) ? 1u : 0u);
                        mma_commit(&empty0[s]);
                    }
                } else {
                    // K block kb of the resident buffer: K chunks 8 kb .. 8 kb + 7, two per MMA.
                    // The weights are streamed well ahead: wait for all of the layer's blocks, then
                    // issue its MMAs back to back (a commit between them costs more than an N=64
                    // MMA) and release the accumulator before the stages.
                    const uint32_t a = smem_u32(smem + (((L - 1) & 1) ? C::OFF_B1 : C::OFF_B0));
                    for (int kb = 0; kb < nkb; ++kb) {
                        const uint32_t i = it1 + kb;
                        if (!mbar_wait_cluster(&full1[i % SMALL_STAGES1], (i / SMALL_STAGES1) & 1)) return false;
                    }
                    tc_fence_after();
                    for (int kb = 0; kb < nkb; ++kb) {
                        const uint32_t b = smem_u32(smem + C::OFF_RING1 + ((it1 + kb) % SMALL_STAGES1) * SMALL_ST1);
#pragma unroll
                        for (int k = 0; k < KB / 32; ++k)
                            mma_i8(d, smem_desc_noswz(a + (kb * 8 + 2 * k) * SMALL_KCHUNK, SMALL_KCHUNK, 128),
                                   smem_desc_sw128(b + 32 * k), idesc, (kb || k) ? 1u : 0u);
                    }
                    mma_commit(acc_full);
                    for (int kb = 0; kb < nkb; ++kb) mma_commit(&empty1[(it1 + kb) % SMALL_STAGES1]);
                    it1 += nkb;
                    ++uu;
                    small_trace<TRACE>(p, tn, 1, 2, L, step);
                    return true;
                }
                mma_commit(acc_full);
                ++uu;
                small_trace<TRACE>(p, tn, 1, 2, L, step);
                return true;
            });
            if (TRACE && blockIdx.x < 2) p.trace_count[blockIdx.x * 4 + 1] = tn;
            mma_commit(drain);
        }
        __syncwarp();
    } else {
        // ---- epilogue warps: TMEM lane quarter q holds rows q*32 .. q*32+31 of the tile
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16);   // coder scratch (rank 0)
        const uint32_t tacc = taddr + SMALL_ACC_COL;                       // accumulator
        uint32_t ue = 0, lw = 0, xe = 0;
        unsigned int tn2 = 0, tn3 = 0;
        const bool tr = warp == 2 && lane == 0;
        for_each_small_unit(p, [&](int tile, int step, int L) -> bool {
            const int ns = p.out_dim[L] / SMALL_C;
            const int32_t *bias = bias_s + L * SMALL_NS;
            const Requant rq = p.rq[L];
            const bool rq_fast = rq.hi_path != 0;
            const int32_t rq_m0 = (int32_t)rq.m0, rq_hs = rq.hi_shift, rq_one = rq.one;
            const uint32_t rq_relu = rq.lo == 0 ? 0xFFFFFFFFu : 0u;
            const bool last = L == NL - 1;
            // rank 0 decodes: this row's coder state, fetched before the logits are ready
            const int64_t drow = (int64_t)tile * TM + r;
            bool dlive = false;
            int64_t dc = 0;
            DecState ds{};
            uint64_t dscale = 0, dq = 0;
            if (last && rank == 0 && drow < p.n_rows) {
                dc = p.order[drow];
                dlive = step < p.lengths[dc] && !p.errors[dc];
                if (dlive) {
                    ds = p.state[drow];
                    dscale = ds.range >> SC_PRECISION;
                    dq = dscale ? (ds.point - ds.lower) / dscale : ~0ull;
                    if (dq >= (uint64_t)SC_TOTAL) {      // invalid stream (cpu_entropy_coding.py:244-248)
                        p.errors[dc] = 1;
                        dlive = false;
                    }
                }
            }
            if (tr) small_trace<TRACE>(p, tn2, 2, 0, L, step);
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(acc_full, ue & 1))) return false;
            ++ue;
            if (tr) small_trace<TRACE>(p, tn2, 2, 1, L, step);
            tc_fence_after();
            // requantise this CTA's ns columns of the row: 32 (the last layer) or 64, in two halves
            auto requant32 = [&](int h, uint32_t (&out)[8]) {
                uint32_t va[32];
                tmem_ld32(tacc + h * 32, va);
                tmem_ld_wait();
                const int4 *bv = reinterpret_cast<const int4 *>(bias + h * 32);
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    out[i] = rq_fast ? requant4_hi(&va[4 * i], bv[i], rq_m0, rq_hs, rq_relu, rq_one)
                                     : requant4(&va[4 * i], bv[i], rq);
            };
            uint32_t lo[8], hi[8];
            requant32(0, lo);
            if (ns > 32) requant32(1, hi);
            // the accumulator is read: the next layer's MMA may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty);
            // This CTA's ns columns of the row: for a hidden layer, K chunks kc0 .. kc0 + 3 of the
            // next layer's A operand, written into this CTA's buffer and copied from there into
            // the same place of every other CTA's; for the last layer, 32 logits of the row for
            // rank 0, staged at [rank][row] (4 KB per CTA) in this CTA's B0 (free at this point).
            const uint32_t slice_bytes = (uint32_t)(ns / 16) * SMALL_KCHUNK;
            uint8_t *slice;
            if (!last) {
                const int kc0 = (int)rank * ns / 16;
                slice = smem + ((L & 1) ? C::OFF_B1 : C::OFF_B0) + kc0 * SMALL_KCHUNK;
                *reinterpret_cast<uint4 *>(slice + 0 * SMALL_KCHUNK + r * 16) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<uint4 *>(slice + 1 * SMALL_KCHUNK + r * 16) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                if (ns > 32) {
                    *reinterpret_cast<uint4 *>(slice + 2 * SMALL_KCHUNK + r * 16) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    *reinterpret_cast<uint4 *>(slice + 3 * SMALL_KCHUNK + r * 16) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                }
            } else {
                slice = smem + C::OFF_B0 + (int)rank * (TM * 32);
                *reinterpret_cast<uint4 *>(slice + r * 32) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<uint4 *>(slice + r * 32 + 16) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
            }
            fence_proxy_async_smem();                // read by the copy engine and the tensor core
            __syncwarp();
            if (lane == 0) counter_add_release(slice_cnt, 1);
            if (warp == 2) {
                // one thread sends the whole slice once every warp's rows are in it (the outcome of
                // its bounded wait goes to the whole warp, which leaves the walk together)
                bool ok = true;
                if (lane == 0) {
                    ok = counter_wait(slice_cnt, 4 * ue);
                    if (ok && !last) {
                        uint64_t *xb = &xbar[xe & 1];
                        mbar_arrive_expect_tx(xb, (SMALL_C - 1) * slice_bytes);
                        for (int c = 1; c < SMALL_C; ++c) {
                            const uint32_t dst = (rank + (uint32_t)c) % SMALL_C;
                            bulk_copy_to_cluster(map_to_rank(slice, dst), slice, slice_bytes, map_to_rank(xb, dst));
                        }
                    } else if (ok && rank == 0) {
                        mbar_arrive_expect_tx(lbar, (SMALL_C - 1) * (TM * 32));
                    } else if (ok) {
                        bulk_copy_to_cluster(map_to_rank(slice, 0), slice, TM * 32, map_to_rank(lbar, 0));
                    }
                }
                if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) return false;
            }
            if (tr) small_trace<TRACE>(p, tn2, 2, 2, L, step);
            if (!last) {
                ++xe;
                return true;
            }
            if (rank != 0) return true;
            // ---- rank 0: the coder step of every row of the tile, from all 256 logits
            if (tr) small_trace<TRACE>(p, tn3, 3, 0, L, step);
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(lbar, lw & 1))) return false;
            ++lw;
            if (tr) small_trace<TRACE>(p, tn3, 3, 1, L, step);
            int mlogit = -128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                // logits 32c .. 32c + 31 of the row, from CTA c's slice
                const uint4 a = *reinterpret_cast<const uint4 *>(smem + C::OFF_B0 + c * (TM * 32) + r * 32);
                const uint4 b = *reinterpret_cast<const uint4 *>(smem + C::OFF_B0 + c * (TM * 32) + r * 32 + 16);
                const uint32_t w8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
                for (int i = 0; i < 8; ++i)
#pragma unroll
                    for (int bb = 0; bb < 4; ++bb) mlogit = max(mlogit, pk_get(w8[i], bb));
                tmem_st8(taddr + c * 8, w8);
            }
            tmem_st_wait();
            int amax, sym;
            RowDivisor dv;
            uint32_t fix, cum, f;
            row_stats<true>(taddr, lut_s, mlogit, dv, fix, amax, -1, cum, f);
            row_find_cached(taddr, lut_s, mlogit, dv, fix, amax, dlive ? (uint32_t)dq : 0u, sym, cum, f);
            if (dlive) {
                DecState s = ds;
                s.lower += dscale * (uint64_t)cum;
                s.range = dscale * (uint64_t)f;
                if (s.range < (1ull << 32)) {
                    s.lower <<= 32;
                    s.range <<= 32;
                    s.point <<= 32;
                    if (s.read_pos < s.end_pos) s.point |= p.words[s.read_pos];
                    s.read_pos += 1;
                }
                p.state[drow] = s;
                p.tokens_out[p.out_off[dc] + step] = (uint8_t)sym;
                // append the token's embedding row to this row's window ring
                const uint4 *e = reinterpret_cast<const uint4 *>(p.emb + sym * EMB_DIM);
                uint8_t *dst = reinterpret_cast<uint8_t *>(
                    p.ering_ptr + (((size_t)ring_block0 + (step & (WIN - 1))) * TM + r) * KB);
                const uint64_t pol = l2_policy_evict_first();
#pragma unroll
                for (int i = 0; i < KB / 32; ++i) {
                    const uint4 a = e[2 * i], b = e[2 * i + 1];
                    const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                    st_global_v8_hint(dst + 32 * i, v, pol);
                }
            }
            fence_proxy_async_global();              // the ring block is read by TMA next step
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                for (int c = 0; c < SMALL_C; ++c) mbar_arrive_cluster(map_to_rank(rbar, (uint32_t)c));
            if (tr) small_trace<TRACE>(p, tn3, 3, 2, L, step);
            return true;
        });
        if (TRACE && tr && blockIdx.x < 2) {
            p.trace_count[blockIdx.x * 4 + 2] = tn2;
            p.trace_count[blockIdx.x * 4 + 3] = tn3;
        }
    }
    // teardown: TMEM is freed only after every MMA issued above has completed; every CTA of the
    // cluster stays until every thread of the cluster has finished its walk.  In a normal run
    // every bulk copy into this CTA was waited for (the exchange barriers) before its data was
    // used; after a timeout (which sets the device error flag before the cluster barrier) a copy
    // a peer issued before giving up may still be landing here, so the CTA then waits before it
    // ends.
    tc_fence_before();
    __syncthreads();
    if (warp == 1) mbar_wait_cluster_drain(drain, 0);
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (*(volatile int *)&g_device_error != 0) spin_ns(200000);
    if (warp == 1) tmem_dealloc(tmem_base, SMALL_TMEM_COLS);
}

}  // namespace sc
