// Small-batch decoder: one 128-row tile per cluster of SMALL_C CTAs (tcgen05 cta_group::1).
//
// The pair kernel (sc_mlp_fused2.cuh) gives each tile of 128 rows one SM and hides the latency of
// a step's nine dependent layers behind the other tiles of its SM.  A batch of a few hundred
// chunks has too few tiles for that: three SM pairs would run one tile each, one step every
// ~110 us.  Here every tile runs on a cluster of eight CTAs instead, each computing 1/8 of every
// layer's outputs (N = 64 of 512, 32 of the last layer's 256), so a step's MMA work is spread over
// eight SMs:
//   - every CTA loads the full A operand of a layer (the embedding ring for layer 0, the previous
//     layer's activations otherwise) and its own N-slice of the weights, by TMA;
//   - its epilogue writes its slice of the layer's output to the cluster's activation rows in
//     global memory (L2) and arrives on an `xbar` mbarrier of every CTA of the cluster, whose
//     producers wait for all eight slices before loading the next layer.  Consecutive exchanges
//     alternate between two barriers: a warp makes its eight arrivals for exchange k before its
//     CTA can start on exchange k+1, but another CTA's barrier may not have seen them all yet,
//     and an arrival for k+1 must never count toward k there; one for k+2 cannot come before
//     every CTA has seen all of k+1, hence all of k;
//   - the last layer's logit slices are gathered the same way in rank 0 (`lbar`), whose
//     epilogue runs the coder step of every row (the pair kernel's frequency pass, search and
//     range-decoder update), appends the decoded tokens' embedding rows to the ring and releases
//     the next step in every CTA (`rbar`).
// Layer 0 of step s reads window positions 0..62 from ring slots written at earlier steps, so its
// loads and MMAs start while rank 0 is still decoding step s-1 (its coder scratch and the
// accumulator are separate TMEM columns); only position 63, the token being decoded, waits for
// rank 0's release (rbar).  Every buffer is reused only after a signal that proves its previous
// contents were consumed in every CTA: layer 0's MMAs of step s, hence its epilogue and all that
// follows, come after rbar of step s-1, which rank 0 sends only after every CTA sent its
// last-layer slice of step s-1, i.e. after all their loads of step s-1 completed; the ring slot
// rank 0 writes at step s-1 held the token that layer 0 of step s-1 read first, in every CTA.
// No TMA load uses cluster multicast; every wait is bounded.
#pragma once

namespace sc {

constexpr int SMALL_C = 8;                           // CTAs per tile
constexpr int SMALL_STAGES = 8;
constexpr int SMALL_B_MAX = (MAX_N / SMALL_C) * KB;  // 8 KB: a 64-row weight slice of one K block
constexpr int SMALL_STAGE = A_BYTES + SMALL_B_MAX;   // 24 KB
constexpr int SMALL_THREADS = 32 * 6;                // producer, MMA, four epilogue warps
// TMEM: columns 0..255 are rank 0's coder scratch (packed logits, cached frequencies), the
// accumulator (64 columns) lives after them, so a step's layer 0 can run during the coder step
constexpr int SMALL_TMEM_COLS = 512;
constexpr int SMALL_ACC_COL = 256;

struct SmallParams {
    CUtensorMap w[FMAX_LAYERS];       // weights, box (out_dim / SMALL_C) rows x 128 B
    CUtensorMap act[2];               // activation ping-pong [clusters * 128][512], box 128 x 128 B
    CUtensorMap ering;                // embedding ring, box 128 rows x 128 B
    int8_t *act_ptr[2];
    int8_t *logits;                   // [clusters * 128][256]: the last layer's requantised logits
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
    static constexpr int OFF_BIAS = SMALL_STAGES * SMALL_STAGE;          // 192 KB
    static constexpr int OFF_LUT = OFF_BIAS + FMAX_LAYERS * MAX_N * 4;
    static constexpr int OFF_BAR = OFF_LUT + 256 * 8;
    // full/empty per stage, acc_full, acc_empty, xbar[2], lbar, rbar, drain
    static constexpr int NBAR = 2 * SMALL_STAGES + 7;
    static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
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

template <bool TRACE>
__global__ void __launch_bounds__(SMALL_THREADS, 1) k_small_decode(const __grid_constant__ SmallParams p)
{
    using C = SmallCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint64_t *full = bars, *empty = bars + SMALL_STAGES;
    uint64_t *acc_full = bars + 2 * SMALL_STAGES, *acc_empty = acc_full + 1;
    uint64_t *xbar = acc_empty + 1;   // [2]: all CTAs' slices of a layer's output are in L2
    uint64_t *lbar = xbar + 2;        // rank 0: all CTAs' last-layer logit slices are in L2
    uint64_t *rbar = lbar + 1;        // rank 0 appended the step's tokens to the ring
    uint64_t *drain = rbar + 1;       // the MMA issuer's last commit: TMEM is freed after it
    uint32_t *tmem_slot = (uint32_t *)(smem + C::OFF_TMEM);
    int32_t *bias_s = (int32_t *)(smem + C::OFF_BIAS);
    uint64_t *lut_s = (uint64_t *)(smem + C::OFF_LUT);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NL = p.num_layers;
    const uint32_t rank = cluster_ctarank();
    const int row0 = (blockIdx.x / SMALL_C) * TM;     // this cluster's activation / logit / ring rows

    if (threadIdx.x == 0) {
        for (int s = 0; s < SMALL_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 4);
        mbar_init(&xbar[0], 4 * SMALL_C);              // four epilogue warps of every CTA
        mbar_init(&xbar[1], 4 * SMALL_C);
        mbar_init(lbar, 4 * SMALL_C);
        mbar_init(rbar, 4);                            // rank 0's epilogue warps
        mbar_init(drain, 1);
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, SMALL_TMEM_COLS);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < SC_VOCAB; i += blockDim.x) lut_s[i] = p.lut[i];
    for (int l = 0; l < NL; ++l)
        for (int i = threadIdx.x; i < p.out_dim[l]; i += blockDim.x) bias_s[l * MAX_N + i] = p.bias[l][i];
    tc_fence_before();
    __syncthreads();
    cluster_sync();                   // every CTA's barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer: the full A operand and this CTA's N-slice of the weights
            uint32_t it = 0, xw = 0, rw = 0;
            unsigned int tn = 0;
            bool aborted = false, first = true;
            const uint64_t ring_policy = l2_policy_evict_first();
            for_each_small_unit(p, [&](int tile, int step, int L) -> bool {
                const int nkb = p.in_dim[L] / KB;
                const int ns = p.out_dim[L] / SMALL_C;
                const uint32_t tx = A_BYTES + ns * KB;
                const int pre = nkb < SMALL_STAGES ? nkb : SMALL_STAGES;
                small_trace<TRACE>(p, tn, 0, 0, L, step);
                auto a_load = [&](int kb, uint8_t *st, uint64_t *bar) {
                    if (L != 0) {
                        tma_load_2d(st, &p.act[(L - 1) & 1], bar, kb * KB, row0);
                    } else {
                        // window position kb holds token step - 64 + kb (start-of-sequence before 0)
                        const int tau = step - WIN + kb;
                        const int row = tau < 0 ? (int)p.ering_sos_row : (row0 / TM * WIN + (tau & (WIN - 1))) * TM;
                        tma_load_2d_hint(st, &p.ering, bar, 0, row, ring_policy);
                    }
                };
                auto acquire = [&](int kb) -> uint8_t * {       // stage of K block kb, with its weights
                    const uint32_t i = it + kb;
                    const int s = i % SMALL_STAGES;
                    if (!mbar_wait_cluster(&empty[s], ((i / SMALL_STAGES) & 1) ^ 1)) return nullptr;
                    uint8_t *st = smem + s * SMALL_STAGE;
                    mbar_arrive_expect_tx(&full[s], tx);
                    tma_load_2d(st + A_BYTES, &p.w[L], &full[s], kb * KB, (int)rank * ns);
                    return st;
                };
                auto bar_of = [&](int kb) { return &full[(it + kb) % SMALL_STAGES]; };
                if (L == 0) {
                    // window positions 0..62 hold tokens decoded at earlier steps, already in the
                    // ring: only the last one (the token rank 0 is decoding now) waits for its
                    // release, so this layer's loads and MMAs overlap the previous step's coder
                    for (int kb = 0; kb < nkb; ++kb) {
                        uint8_t *st = acquire(kb);
                        if (st == nullptr) {
                            it += kb;
                            return !(aborted = true);
                        }
                        if (kb == nkb - 1) {
                            // rank 0 releases every step, a tile's last one too: every layer 0 but
                            // the cluster's very first consumes one release
                            if (!first && !mbar_wait_cluster(rbar, rw & 1)) {
                                it += kb + 1;
                                return !(aborted = true);
                            }
                            rw += first ? 0 : 1;
                            first = false;
                            small_trace<TRACE>(p, tn, 0, 1, L, step);
                        }
                        a_load(kb, st, bar_of(kb));
                    }
                } else {
                    // the weights of the first stages go out before the operand is ready
                    uint8_t *sts[SMALL_STAGES];
                    for (int kb = 0; kb < pre; ++kb) {
                        sts[kb] = acquire(kb);
                        if (sts[kb] == nullptr) {
                            it += kb;
                            return !(aborted = true);
                        }
                    }
                    if (!mbar_wait_cluster(&xbar[xw & 1], (xw >> 1) & 1)) {
                        it += pre;
                        return !(aborted = true);
                    }
                    ++xw;
                    small_trace<TRACE>(p, tn, 0, 1, L, step);
                    for (int kb = 0; kb < pre; ++kb) a_load(kb, sts[kb], bar_of(kb));
                    for (int kb = pre; kb < nkb; ++kb) {
                        uint8_t *st = acquire(kb);
                        if (st == nullptr) {
                            it += kb;
                            return !(aborted = true);
                        }
                        a_load(kb, st, bar_of(kb));
                    }
                }
                it += nkb;
                small_trace<TRACE>(p, tn, 0, 2, L, step);
                return true;
            });
            if (TRACE && blockIdx.x < 2) p.trace_count[blockIdx.x * 4 + 0] = tn;
            if (aborted) {
                // loads already issued may still be landing in shared memory: wait (bounded) for the
                // full phases of the last stages, then give stragglers time before the CTA ends
                for (uint32_t i = it > (uint32_t)SMALL_STAGES ? it - SMALL_STAGES : 0; i < it; ++i)
                    mbar_wait_cluster_drain(&full[i % SMALL_STAGES], (i / SMALL_STAGES) & 1);
                spin_ns(100000);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: D[128 x ns] = A[128 x K] * W_slice[ns x K]^T, one accumulator
            uint32_t it = 0, uu = 0;
            unsigned int tn = 0;
            for_each_small_unit(p, [&](int tile, int step, int L) -> bool {
                const int nkb = p.in_dim[L] / KB;
                const int ns = p.out_dim[L] / SMALL_C;
                const uint32_t idesc = idesc_i8(TM, ns);
                small_trace<TRACE>(p, tn, 1, 0, L, step);
                if (!mbar_wait_cluster(acc_empty, (uu & 1) ^ 1)) return false;
                small_trace<TRACE>(p, tn, 1, 1, L, step);
                tc_fence_after();
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % SMALL_STAGES;
                    if (!mbar_wait_cluster(&full[s], (it / SMALL_STAGES) & 1)) return false;
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + s * SMALL_STAGE);
#pragma unroll
                    for (int k = 0; k < KB / 32; ++k)
                        mma_i8(tmem_base + SMALL_ACC_COL, smem_desc_sw128(st + 32 * k),
                               smem_desc_sw128(st + A_BYTES + 32 * k), idesc,
                               (kb || k) ? 1u : 0u);
                    mma_commit(&empty[s]);
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
            const int32_t *bias = bias_s + L * MAX_N + (int)rank * ns;
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
            if (!last) {
                int8_t *dst = p.act_ptr[L & 1] + (size_t)(row0 + r) * MAX_N + (int)rank * ns;
                st_global_v8(dst, lo);
                if (ns > 32) st_global_v8(dst + 32, hi);
                fence_proxy_async_global();          // read next by other CTAs' TMA
                __syncwarp();
                if (lane == 0)
                    for (int c = 0; c < SMALL_C; ++c) mbar_arrive_cluster(map_to_rank(&xbar[xe & 1], (uint32_t)c));
                ++xe;
                if (tr) small_trace<TRACE>(p, tn2, 2, 2, L, step);
                return true;
            }
            st_global_v8(p.logits + (size_t)(row0 + r) * SC_VOCAB + (int)rank * ns, lo);
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(map_to_rank(lbar, 0));
            if (tr) small_trace<TRACE>(p, tn2, 2, 2, L, step);
            if (rank != 0) return true;
            // ---- rank 0: the coder step of every row of the tile, from all 256 logits
            if (tr) small_trace<TRACE>(p, tn3, 3, 0, L, step);
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(lbar, lw & 1))) return false;
            ++lw;
            if (tr) small_trace<TRACE>(p, tn3, 3, 1, L, step);
            int mlogit = -128;
            {
                // all sixteen loads in flight at once (L2: the slices come from eight SMs)
                const uint4 *src = reinterpret_cast<const uint4 *>(p.logits + (size_t)(row0 + r) * SC_VOCAB);
                uint4 v[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = __ldcg(src + i);
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint32_t w8[8] = {v[2 * c].x, v[2 * c].y, v[2 * c].z, v[2 * c].w,
                                            v[2 * c + 1].x, v[2 * c + 1].y, v[2 * c + 1].z, v[2 * c + 1].w};
#pragma unroll
                    for (int i = 0; i < 8; ++i)
#pragma unroll
                        for (int bb = 0; bb < 4; ++bb) mlogit = max(mlogit, pk_get(w8[i], bb));
                    tmem_st8(taddr + c * 8, w8);
                }
                tmem_st_wait();
            }
            int amax, sym;
            RowDivisor d;
            uint32_t fix, cum, f;
            row_stats<true>(taddr, lut_s, mlogit, d, fix, amax, -1, cum, f);
            row_find_cached(taddr, lut_s, mlogit, d, fix, amax, dlive ? (uint32_t)dq : 0u, sym, cum, f);
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
                    p.ering_ptr + (((size_t)(row0 / TM) * WIN + (step & (WIN - 1))) * TM + r) * KB);
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
    // cluster stays until all remote arrivals are done
    tc_fence_before();
    __syncthreads();
    if (warp == 1) mbar_wait_cluster_drain(drain, 0);
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, SMALL_TMEM_COLS);
}

}  // namespace sc
