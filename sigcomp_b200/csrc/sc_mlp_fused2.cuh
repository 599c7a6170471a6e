// Fused persistent MLP kernels on CTA pairs (tcgen05 cta_group::2).
//
// Same schedule and fused epilogues as the single-CTA kernels in
// sc_mlp_fused.cuh, with every MMA spanning an SM pair: M = 256 rows (128 per
// CTA), N = 256, so each SM loads only half of every weight tile and issues no
// MMA of its own.  Included by sc_mlp_tc.cu (same translation unit as the
// device error flag).
//
// Per pair:
//   - both CTAs TMA-load their own activation rows and their half of the
//     weight tile into the same shared-memory offsets, completing on the
//     leader CTA's (rank 0) `full` barrier;
//   - the leader issues the pair MMA and multicasts its commits to the
//     `empty`, `acc_full` and `g_empty` barriers of both CTAs;
//   - each CTA's epilogue warps read their own 128 TMEM lanes and arrive on the
//     leader's `acc_empty` (remote arrive for the peer);
//   - compress: layer-0 builders fill sliding embedding buffers of their own
//     CTA's rows and arrive on the leader's barriers;
//   - decode: layer 0 reads its operand by TMA from a per-tile embedding ring
//     in global memory (the embedding rows of the last 64 tokens of every row,
//     one 128-row x 128-byte block per window position); the last-layer
//     epilogue appends each decoded token's embedding row, so a step writes
//     one block per tile instead of building all 64.
//   - the layers after the first add their bias with one K = 32 MMA against
//     a resident bias tile (loaded once per layer and step or tile group), so
//     their epilogues requantise without loading or adding a bias.
// No TMA load uses cluster multicast.
#pragma once

#include <type_traits>

namespace sc {

// pair-tiles in flight per CTA pair: six for the decoder (more units to overlap its
// long last-layer epilogues), five for compression (smaller activation buffers in L2)
constexpr int KT2 = 6;                // the larger of the two: sizes per-slot arrays
template <bool DECODE> constexpr int kt2() { return DECODE ? 6 : 5; }

// Decoder schedule.  Every SM pair runs KT2 tile lanes (slots); a lane decodes its queue of
// pair-tiles back to back, the next pair-tile starting at the global step after the previous
// one's last.  The host cuts each pair's timeline into segments over which no lane changes
// pair-tile, so one launch decodes any number of chunks.
struct DecSeg {
    int32_t s0, s1;                   // global steps [s0, s1) of this pair
    int32_t pt[KT2];                  // pair-tile of each lane, -1 while the lane is idle
    int32_t start[KT2];               // global step of that pair-tile's step 0
};

struct Fused2Params {
    CUtensorMap w[FMAX_LAYERS];       // weights, box 128 rows x 128 B (half of a 256-row unit)
    // bias tiles of layers >= 1 (box 128 rows x 128 B, one per CTA of the pair).  Row i
    // of CTA r's tile serves output column h * 256 + r * 128 + i of half h: bytes 64h .. 64h + 31
    // hold 32 int8 digits of that column's bias and bytes 64h + 32 .. 64h + 63 the constants
    // 16 x 127, 16 x 1.  One K = 32 MMA with the constants as A (the same in every row) and the
    // digits as B adds the bias to the accumulator after a unit's K blocks.
    CUtensorMap bt[FMAX_LAYERS];
    uint32_t bias_mma;                // bit L: layer L's bias enters through its bias tile
    CUtensorMap act[2];               // activation ping-pong, box 128 x 128 B
    int8_t *act_ptr[2];
    const int32_t *bias[FMAX_LAYERS];
    Requant rq[FMAX_LAYERS];
    int in_dim[FMAX_LAYERS];
    int out_dim[FMAX_LAYERS];
    int num_layers;
    const int8_t *emb;
    const uint64_t *lut;
    int n_tiles;
    // optional unit trace of the first CTA pair (null when tracing is off): per CTA, one region
    // of trace_cap / 4 records for each of the roles 0-3
    unsigned long long *trace;        // [2][4][trace_cap / 4][2]
    unsigned int *trace_count;        // [2][4]: records each role wrote
    int trace_cap;
    // compress
    const int32_t *tile_chunk;
    const int32_t *tile_t0;
    const int64_t *tok_off;
    const uint8_t *tokens;
    int64_t row_base;
    uint2 *pairs;
    // decode
    CUtensorMap ering;                // embedding ring, box 128 rows x 128 B
    int8_t *ering_ptr;                // [grid][kt2][WIN][TM][128], then the start-of-sequence block
    int64_t ering_sos_row;            // first row of the start-of-sequence block
    const int64_t *order;
    int64_t n_rows;
    const DecSeg *segs;               // this launch's segments, pair after pair
    const int32_t *pair_seg;          // [pairs + 1]: segments of pair i are segs[pair_seg[i] .. pair_seg[i+1])
    const int64_t *lengths;
    DecState *state;
    const uint32_t *words;
    uint8_t *tokens_out;
    const int64_t *out_off;
    uint8_t *errors;
};

namespace {

constexpr int B_HALF = (TN / 2) * KB;          // 16 KB: this CTA's half of a weight K block
constexpr int EPI_PER_Q = 3;                    // epilogue warps per TMEM lane quarter
constexpr int EPI_WARPS = 4 * EPI_PER_Q;        // epilogue warps per CTA
constexpr int BUILD_WARPS = 2;                  // compress: the last two warps fill the sliding buffers
constexpr int FUSED2_THREADS = 32 * (2 + EPI_WARPS + BUILD_WARPS);
constexpr int BIAS_MAX = FMAX_LAYERS * MAX_N;   // int32 entries

template <bool DECODE>
struct F2Cfg {
    // decode: layer 0 is one pass over K for both 256-column halves (two accumulators),
    // so a stage holds the ring block and both weight halves: the block is read from
    // the ring once per step instead of twice.  The two halves of the other 512-wide
    // layers share their stages the same way, one unit after the other: a stage holds a
    // K block of the activations and of both weight halves, half 0 keeps it and half 1
    // releases it, so each activation K block is loaded once per layer, not twice.
    static constexpr int STAGES = 4;
    static constexpr int STAGE_BYTES = A_BYTES + (DECODE ? 2 : 1) * B_HALF;   // 48 KB / 32 KB
    static constexpr int OFF_X = STAGES * STAGE_BYTES;                    // 192 KB / 128 KB
    static constexpr int X_BYTES = DECODE ? 0 : 2 * G_BYTES;
    // the current layer's bias tile (16 KB); the decoder's SMEM bias table holds layer 0 only
    static constexpr int OFF_BT = OFF_X + X_BYTES;
    static constexpr int BT_BYTES = TM * KB;
    static constexpr int OFF_BIAS = OFF_BT + BT_BYTES;
    static constexpr int BIAS_ENTRIES = DECODE ? MAX_N : BIAS_MAX;
    static constexpr int OFF_LUT = OFF_BIAS + BIAS_ENTRIES * 4;
    static constexpr int OFF_BAR = OFF_LUT + 256 * 8;
    static constexpr int NBAR = 2 * STAGES + 11;    // ... + the teardown drain barrier + bias tile pair
    static constexpr int OFF_CNT = OFF_BAR + NBAR * 8;
    static constexpr int OFF_TMEM = OFF_CNT + 8 * 4;
    static constexpr int SMEM = OFF_TMEM + 16 + 1024;
    static_assert(SMEM <= 232448, "shared memory per CTA");
};

// Trace record of one role event for a unit (first CTA pair only):
// word 0 = %globaltimer, word 1 = role | event << 4 | L << 8 | nh << 12 | tt << 16 | step << 32.
// roles: 0 producer, 1 MMA, 2 epilogue (warp 2), 3 compress layer-0 builders
// Each role traces from one thread into its own region of the trace buffer.  The producer and
// MMA threads count their records in a register (`n`), so a record costs them two stores and no
// global atomic on their critical path; the epilogue's tracing lane counts with an atomic on its
// role's global counter, which needs no register for the count across its unit loop.
__device__ __forceinline__ void trace_put(const Fused2Params &p, int role, unsigned int i, int ev, int L, int nh,
                                          int tt, int step)
{
    if (i >= (unsigned int)p.trace_cap / 4) return;
    unsigned long long *r = p.trace + (((size_t)blockIdx.x * 4 + role) * (p.trace_cap / 4) + i) * 2;
    r[0] = globaltimer_ns();
    r[1] = (unsigned long long)role | ((unsigned long long)ev << 4) | ((unsigned long long)L << 8) |
           ((unsigned long long)nh << 12) | ((unsigned long long)tt << 16) | ((unsigned long long)step << 32);
}

// Both are compiled out of the untraced kernels (TRACE false), which are the ones a normal
// call launches: the trace code would otherwise cost registers in every kernel.
template <bool TRACE>
__device__ __forceinline__ void trace_ev(const Fused2Params &p, unsigned int &n, int role, int ev, int L, int nh,
                                         int tt, int step)
{
    if constexpr (TRACE) {
        if (blockIdx.x >= 2) return;
        trace_put(p, role, n++, ev, L, nh, tt, step);
    }
}

template <bool TRACE>
__device__ __forceinline__ void trace_ev_atomic(const Fused2Params &p, int role, int ev, int L, int nh, int tt,
                                                int step)
{
    if constexpr (TRACE) {
        if (blockIdx.x >= 2) return;
        trace_put(p, role, atomicAdd(p.trace_count + blockIdx.x * 4 + role, 1u), ev, L, nh, tt, step);
    }
}

// Row frequency statistics (_frequencies, cpu_entropy_coding.py:90-110) from the
// packed logits in TMEM (64 words from taddr) with the maximum logit m known:
// row divisor, fix-up amount, first index of the maximum frequency and, for
// sym >= 0, the exclusive cumulative frequency and frequency of sym.
// With CACHE_F, the frequencies of symbols 0..191 (before the fix-up) are also
// stored in TMEM columns 64..255 of the same accumulator (read already), where
// row_find_cached picks them up instead of recomputing them.
template <bool CACHE_F = false>
__device__ __forceinline__ void row_stats(uint32_t taddr, const uint64_t *lut_s, int m, RowDivisor &d, uint32_t &fix,
                                          int &amax, int sym, uint32_t &sym_cum, uint32_t &sym_f)
{
    uint64_t T0 = 0, T1 = 0;                         // two chains of 64-bit adds
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        uint32_t w[16];
        tmem_ld16(taddr + g * 16, w);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; i += 2)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                T0 += lut_s[m - pk_get(w[i], b)];
                T1 += lut_s[m - pk_get(w[i + 1], b)];
            }
    }
    d = make_row_divisor(T0 + T1);
    uint32_t total = 0, best = 0, below = 0, fsym = 0;
    amax = 0;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        uint32_t w[16];
        tmem_ld16(taddr + g * 16, w);
        tmem_ld_wait();
        uint32_t f8[8];
#pragma unroll
        for (int i = 0; i < 16; ++i)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int v = g * 64 + 4 * i + b;
                uint32_t f = div_freq(lut_s[m - pk_get(w[i], b)], d);
                f = f < 1u ? 1u : f;
                total += f;
                if (f > best) { best = f; amax = v; }
                below += v < sym ? f : 0u;
                fsym = v == sym ? f : fsym;
                if (CACHE_F) {
                    f8[(4 * i + b) & 7] = f;
                    if (((4 * i + b) & 7) == 7 && g < 3) tmem_st8(taddr + 64 + g * 64 + 4 * i + b - 7, f8);
                }
            }
    }
    if (CACHE_F) tmem_st_wait();
    fix = total - SC_TOTAL;          // modulo 2^32; subtracting it from f[amax] is exact
    sym_cum = below - (amax < sym ? fix : 0u);
    sym_f = fsym - (amax == sym ? fix : 0u);
}

// The symbol whose fixed-up cumulative interval holds q: the first v with cum_v + f_v > q,
// with the frequencies of symbols 0..191 read back from TMEM (row_stats<true>) and those
// of 192..255 recomputed.  The warp scans groups while any lane is still searching (the
// TMEM loads are warp-collective).
__device__ __forceinline__ void row_find_cached(uint32_t taddr, const uint64_t *lut_s, int m, const RowDivisor &d,
                                                uint32_t fix, int amax, uint32_t q, int &sym, uint32_t &sym_cum,
                                                uint32_t &sym_f)
{
    uint32_t cum = 0;
    bool found = false;
    sym = SC_VOCAB - 1;
    sym_cum = 0;
    sym_f = 0;
#pragma unroll 1
    for (int g = 0; g < 4; ++g) {
        if (!__any_sync(0xffffffffu, !found)) break;
        if (g < 3) {
#pragma unroll 1
            for (int c4 = 0; c4 < 4; ++c4) {
                uint32_t fv[16];
                tmem_ld16(taddr + 64 + g * 64 + c4 * 16, fv);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int v = g * 64 + c4 * 16 + j;
                    const uint32_t f = fv[j] - (v == amax ? fix : 0u);
                    if (!found && cum + f > q) {
                        found = true;
                        sym = v;
                        sym_cum = cum;
                        sym_f = f;
                    }
                    cum += f;
                }
            }
        } else {
            uint32_t w[16];
            tmem_ld16(taddr + g * 16, w);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int v = g * 64 + 4 * i + b;
                    uint32_t f = div_freq(lut_s[m - pk_get(w[i], b)], d);
                    f = f < 1u ? 1u : f;
                    f -= v == amax ? fix : 0u;
                    if (!found && cum + f > q) {
                        found = true;
                        sym = v;
                        sym_cum = cum;
                        sym_f = f;
                    }
                    cum += f;
                }
        }
    }
}

// Walk this pair's units in the fixed order both CTAs and every role follow, calling
// f(gs, tt, pt, step, L, nh, fl) for each unit: layer L, output half nh, of pair-tile pt in slot tt
// at that tile's step `step`.  Pair-tile pt covers tiles 2*pt (rank 0) and 2*pt+1 (rank 1).
// fl bit 0: the first unit of layer L in this step (or group), bit 1: the last.
//   decode: gs is the pair's global step; every slot's lane runs its pair-tiles back to back,
//           so slot tt's units of global step gs are its (gs * NL + L)-th layer completion
//   compress: gs is the group of up to kt2() tiles; every tile takes one step
template <bool DECODE, typename F>
__device__ __forceinline__ void for_each_unit2(const Fused2Params &p, F &&f)
{
    const int NP = gridDim.x / 2;
    const int pair = blockIdx.x / 2;
    const int NL = p.num_layers;
    if (DECODE) {
        for (int sg = p.pair_seg[pair]; sg < p.pair_seg[pair + 1]; ++sg) {
            const DecSeg *S = p.segs + sg;
            const int s1 = S->s1;
            int first_tt = KT2, last_tt = -1;      // the segment's first and last busy lanes
            for (int tt = 0; tt < KT2; ++tt)
                if (S->pt[tt] >= 0) {
                    first_tt = min(first_tt, tt);
                    last_tt = tt;
                }
            for (int gs = S->s0; gs < s1; ++gs)
                for (int L = 0; L < NL; ++L)
#pragma unroll 1
                    for (int tt = 0; tt < KT2; ++tt) {
                        const int pt = S->pt[tt];
                        if (pt < 0) continue;
                        const int step = gs - S->start[tt];
                        const int NH = p.out_dim[L] / TN;
                        for (int nh = 0; nh < NH; ++nh) {
                            const int fl = (tt == first_tt && nh == 0 ? 1 : 0) | (tt == last_tt && nh == NH - 1 ? 2 : 0);
                            if (!f(gs, tt, pt, step, L, nh, fl)) return;
                        }
                    }
        }
        return;
    }
    const int n_pt = (p.n_tiles + 1) / 2;
    const int my_pt = n_pt > pair ? (n_pt - 1 - pair) / NP + 1 : 0;
    constexpr int KTD = kt2<DECODE>();
    for (int g0 = 0, grp = 0; g0 < my_pt; g0 += KTD, ++grp) {
        const int gn = min(KTD, my_pt - g0);
        for (int L = 0; L < NL; ++L)
#pragma unroll 1
            for (int tt = 0; tt < gn; ++tt) {
                const int pt = pair + (g0 + tt) * NP;
                const int NH = p.out_dim[L] / TN;
                for (int nh = 0; nh < NH; ++nh) {
                    const int fl = (tt == 0 && nh == 0 ? 1 : 0) | (tt == gn - 1 && nh == NH - 1 ? 2 : 0);
                    if (!f(grp, tt, pt, 0, L, nh, fl)) return;
                }
            }
    }
}

__device__ __forceinline__ void mma_k_block_pair(uint32_t d, uint32_t a_addr, uint32_t b_addr, bool first) {
    constexpr uint32_t idesc = idesc_i8(2 * TM, TN);
#pragma unroll
    for (int k = 0; k < KB / 32; ++k)
        mma_i8_pair(d, smem_desc_sw128(a_addr + 32 * k), smem_desc_sw128(b_addr + 32 * k), idesc,
                    (!first || k) ? 1u : 0u);
}

// TRACE: the instrumented build of the kernel (sc_trace_enable), with the unit trace of the
// first SM pair; normal calls launch the build without it.
template <bool DECODE, bool TRACE>
__global__ void __launch_bounds__(FUSED2_THREADS, 1) k_fused2(const __grid_constant__ Fused2Params p)
{
    using C = F2Cfg<DECODE>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint64_t *full = bars, *empty = bars + C::STAGES;
    uint64_t *acc_full = bars + 2 * C::STAGES, *acc_empty = acc_full + 2;
    uint64_t *g_full = acc_empty + 2, *g_empty = g_full + 2;
    // drain: the MMA issuer's last commit (both CTAs); TMEM is freed only after it
    uint64_t *drain = g_empty + 2;
    // bias tile loaded (leader: expect-tx + both CTAs' bytes) / free again (MMA commit)
    uint64_t *bt_full = drain + 1, *bt_empty = drain + 2;
    uint8_t *btile = smem + C::OFF_BT;
    // act_cnt[tt]: +1 per epilogue warp of this CTA when its tile of slot tt finishes a
    // layer; completion number k is reached at act_cnt[tt] >= EPI_WARPS * (k + 1)
    uint32_t *act_cnt = (uint32_t *)(smem + C::OFF_CNT);
    uint32_t *tmem_slot = (uint32_t *)(smem + C::OFF_TMEM);
    int32_t *bias_s = (int32_t *)(smem + C::OFF_BIAS);
    uint64_t *lut_s = (uint64_t *)(smem + C::OFF_LUT);
    uint8_t *xbuf = smem + C::OFF_X;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NL = p.num_layers;
    const uint32_t rank = cluster_ctarank();

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);                    // leader producer (+ transaction bytes)
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 2 * EPI_WARPS);
            mbar_init(&g_full[b], 4);
            mbar_init(&g_empty[b], 1);
        }
        mbar_init(drain, 1);
        mbar_init(bt_full, 1);
        mbar_init(bt_empty, 1);
        for (int tt = 0; tt < 8; ++tt) act_cnt[tt] = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, 2 * TN);
        tmem_relinquish_pair();
    }
    for (int i = threadIdx.x; i < SC_VOCAB; i += blockDim.x) lut_s[i] = p.lut[i];
    for (int l = 0; l < (DECODE ? 1 : NL); ++l)
        for (int i = threadIdx.x; i < p.out_dim[l]; i += blockDim.x) bias_s[l * MAX_N + i] = p.bias[l][i];
    tc_fence_before();
    __syncthreads();
    cluster_sync();                       // both CTAs' barriers exist before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int slot_row0 = blockIdx.x * kt2<DECODE>() * TM;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer (both CTAs): own activation rows + own half of the weights
            uint32_t it = 0;
            uint32_t nbt = 0;                          // bias tiles loaded
            unsigned int tn = 0;                       // trace records written
            bool aborted = false;
            // the embedding ring (hundreds of MB) streams from DRAM: keep it from evicting
            // the weights and activations that live in L2
            const uint64_t ring_policy = l2_policy_evict_first();
            for_each_unit2<DECODE>(p, [&](int gs, int tt, int pt, int step, int L, int nh, int fl) -> bool {
                // decode: half 1 of a layer is loaded with half 0 (layer 0: one dual pass; the
                // other layers: the two halves share their activation K blocks)
                const int nkb = p.in_dim[L] / KB;
                if (DECODE && nh == 1 && (L == 0 || nkb <= C::STAGES)) return true;
                trace_ev<TRACE>(p, tn, 0, 0, L, nh, tt, gs);
                if (nh == 0 && (L >= 1 || (DECODE && step > 0))) {
                    // layer L-1 of this tile is written (decode layer 0: the previous step's
                    // last layer appended its token to the embedding ring)
                    const uint32_t k = (uint32_t)(gs * NL + L - 1);
                    if (!counter_wait(&act_cnt[tt], EPI_WARPS * (k + 1))) return !(aborted = true);
                }
                trace_ev<TRACE>(p, tn, 0, 1, L, nh, tt, gs);
                const int ring0 = (blockIdx.x * kt2<DECODE>() + tt) * WIN * TM;
                // compress layer 0 reads A from the sliding buffer: its stages carry the
                // weights of two K blocks (the second in the unused activation half)
                const int kstep = (!DECODE && L == 0) ? 2 : 1;
                for (int kb = 0; kb < nkb; kb += kstep, ++it) {
                    const int s = it % C::STAGES;
                    if (!mbar_wait_cluster(&empty[s], ((it / C::STAGES) & 1) ^ 1)) return !(aborted = true);
                    uint8_t *st = smem + s * C::STAGE_BYTES;
                    const uint32_t fb = map_to_rank(&full[s], 0);
                    const bool a_tma = DECODE || L != 0;
                    // decode: layer 0 and the two-half layers load both weight halves per K block
                    const bool both = DECODE && (L == 0 || (p.out_dim[L] == 2 * TN && nkb <= C::STAGES));
                    if (rank == 0)
                        mbar_arrive_expect_tx(&full[s], 2 * ((both ? 2 : 1) * B_HALF + (a_tma ? A_BYTES : B_HALF)));
                    if (kstep == 2) {
                        tma_load_2d_pair(st, &p.w[L], fb, (kb + 1) * KB, nh * TN + (int)rank * (TN / 2));
                    } else if (L != 0) {
                        tma_load_2d_pair(st, &p.act[(L - 1) & 1], fb, kb * KB, slot_row0 + tt * TM);
                        if (both) tma_load_2d_pair(st + A_BYTES + B_HALF, &p.w[L], fb, kb * KB, TN + (int)rank * (TN / 2));
                    } else if (DECODE) {
                        // window position kb holds token step - 64 + kb (start-of-sequence before 0)
                        const int tau = step - WIN + kb;
                        const int row = tau < 0 ? (int)p.ering_sos_row : ring0 + (tau & (WIN - 1)) * TM;
                        tma_load_2d_pair_hint(st, &p.ering, fb, 0, row, ring_policy);
                        tma_load_2d_pair(st + A_BYTES + B_HALF, &p.w[L], fb, kb * KB, TN + (int)rank * (TN / 2));
                    }
                    tma_load_2d_pair(st + A_BYTES, &p.w[L], fb, kb * KB, nh * TN + (int)rank * (TN / 2));
                }
                if (L != 0 && (fl & 1) && ((p.bias_mma >> L) & 1u)) {
                    // the layer's bias tile, once per layer and step (or group), after the first unit's K
                    // blocks and once the previous layer's last bias MMA has read the buffer
                    if (!mbar_wait_cluster(bt_empty, (nbt & 1) ^ 1)) return !(aborted = true);
                    if (rank == 0) mbar_arrive_expect_tx(bt_full, 2 * C::BT_BYTES);
                    tma_load_2d_pair(btile, &p.bt[L], map_to_rank(bt_full, 0), 0, (int)rank * TM);
                    ++nbt;
                }
                trace_ev<TRACE>(p, tn, 0, 2, L, nh, tt, gs);
                return true;
            });
            if (TRACE && blockIdx.x < 2) p.trace_count[blockIdx.x * 4 + 0] = tn;
            if (aborted) {
                // Abort path: loads this CTA issued may still be landing in its shared memory.
                // They complete on the leader's full barrier, and a stage is released (empty)
                // only after the MMA that read it, so the leader waits for the full phases and
                // the peer for the empty phases of the last STAGES stages it issued (bounded),
                // then both give copies that no barrier reports on time to land.
                for (uint32_t i = it > (uint32_t)C::STAGES ? it - C::STAGES : 0; i < it; ++i) {
                    const int s = i % C::STAGES;
                    const uint32_t ph = (i / C::STAGES) & 1;
                    if (rank == 0) mbar_wait_cluster_drain(&full[s], ph);
                    else mbar_wait_cluster_drain(&empty[s], ph);
                }
                // the last bias tile, the same way
                if (nbt > 0) {
                    if (rank == 0) mbar_wait_cluster_drain(bt_full, (nbt - 1) & 1);
                    else mbar_wait_cluster_drain(bt_empty, (nbt - 1) & 1);
                }
                spin_ns(100000);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---- MMA issuer (leader CTA only)
            uint32_t it = 0, uu = 0, li = 0;
            uint32_t it_shared = 0;                    // decode: first stage of the current two-half layer
            uint32_t nbt = 0;                          // bias tiles used
            unsigned int tn = 0;                       // trace records written
            for_each_unit2<DECODE>(p, [&](int gs, int tt, int pt, int step, int L, int nh, int fl) -> bool {
                // decoding layer 0: half 1 accumulates in the other buffer during half 0's pass
                if (DECODE && L == 0 && nh == 1) return true;
                const bool dual = DECODE && L == 0;
                const int nkb = p.in_dim[L] / KB;
                // decoding a two-half layer >= 1: half 0 reads each stage after its wait and keeps
                // it; half 1 reads the same stages again (its own weight half) and releases them
                const bool sh = DECODE && L != 0 && p.out_dim[L] == 2 * TN && nkb <= C::STAGES;
                const bool shared0 = sh && nh == 0, shared1 = sh && nh == 1;
                const int ab = uu & 1;
                trace_ev<TRACE>(p, tn, 1, 0, L, nh, tt, gs);
                if (!mbar_wait_cluster(&acc_empty[ab], ((uu >> 1) & 1) ^ 1)) return false;
                if (dual && !mbar_wait_cluster(&acc_empty[ab ^ 1], (((uu + 1) >> 1) & 1) ^ 1)) return false;
                trace_ev<TRACE>(p, tn, 1, 1, L, nh, tt, gs);
                const int gb = li & 1;
                if (!DECODE && L == 0 && nh == 0 && !mbar_wait_cluster(&g_full[gb], (li >> 1) & 1)) return false;
                tc_fence_after();
                const uint32_t d = tmem_base + ab * TN;
                const int kstep = (!DECODE && L == 0) ? 2 : 1;
                // bias tile: after the K blocks one K = 32 MMA adds the bias to the accumulator
                // (integer sums: the order does not matter), so the tile has the unit's K blocks
                // to arrive; it is released after the layer's last bias MMA
                const bool bmma = L != 0 && ((p.bias_mma >> L) & 1u);
                if (shared0) it_shared = it;
                if (shared1) {
                    for (int kb = 0; kb < nkb; ++kb) {
                        const int s = (it_shared + kb) % C::STAGES;
                        const uint32_t st = smem_u32(smem + s * C::STAGE_BYTES);
                        mma_k_block_pair(d, st, st + A_BYTES + B_HALF, kb == 0);
                        mma_commit_pair(&empty[s], 0x3);
                    }
                }
                for (int kb = 0; kb < nkb && !shared1; kb += kstep, ++it) {
                    const int s = it % C::STAGES;
                    if (!mbar_wait_cluster(&full[s], (it / C::STAGES) & 1)) return false;
                    if (L == 0 && kb < 4) trace_ev<TRACE>(p, tn, 1, 3, L, kb, tt, gs);
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + s * C::STAGE_BYTES);
                    if (shared0) {
                        mma_k_block_pair(d, st, st + A_BYTES, kb == 0);
                        continue;                          // the stage stays for half 1
                    }
                    if (kstep == 2) {
                        const uint32_t g = smem_u32(xbuf + gb * G_BYTES);
                        mma_k_block_pair(d, g + kb * KB, st + A_BYTES, kb == 0);
                        mma_k_block_pair(d, g + (kb + 1) * KB, st, false);
                    } else {
                        mma_k_block_pair(d, st, st + A_BYTES, kb == 0);
                        if (dual) mma_k_block_pair(tmem_base + (ab ^ 1) * TN, st, st + A_BYTES + B_HALF, kb == 0);
                    }
                    mma_commit_pair(&empty[s], 0x3);
                }
                if (bmma) {
                    if ((fl & 1) && !mbar_wait_cluster(bt_full, (nbt++) & 1)) return false;
                    tc_fence_after();
                    const uint32_t b0 = smem_u32(btile) + 64 * nh;
                    mma_i8_pair(d, smem_desc_sw128(b0 + 32), smem_desc_sw128(b0), idesc_i8(2 * TM, TN), 1u);
                    if (fl & 2) mma_commit_pair(bt_empty, 0x3);
                }
                mma_commit_pair(&acc_full[ab], 0x3);
                if (dual) mma_commit_pair(&acc_full[ab ^ 1], 0x3);
                trace_ev<TRACE>(p, tn, 1, 2, L, nh, tt, gs);
                uu += dual ? 2 : 1;
                if (!DECODE && L == 0 && nh == p.out_dim[0] / TN - 1) {
                    mma_commit_pair(&g_empty[gb], 0x3);
                    ++li;
                }
                return true;
            });
            if (TRACE && blockIdx.x < 2) p.trace_count[blockIdx.x * 4 + 1] = tn;
            // completes (in both CTAs) once every MMA issued above, and every commit before
            // it, has completed: normal end or abort alike
            mma_commit_pair(drain, 0x3);
        }
        __syncwarp();
    } else if (warp >= 2 && warp < 2 + EPI_WARPS) {
        // ---- epilogue warps: TMEM lane quarter q; hidden layers split the eight
        // 32-column chunks of a unit between the EPI_PER_Q warps of a quarter.  The last
        // layer of a unit runs on one warp of the quarter, the warps taking turns: by tile
        // slot for decoding (so a row's coder state always stays with the warp that wrote
        // it), by unit for compression.
        const int q = warp & 3;
        const int part = (warp - 2) >> 2;
        const int r = q * 32 + lane;
        uint32_t uu = 0, lu = 0;
        for_each_unit2<DECODE>(p, [&](int gs, int tt, int pt, int step, int L, int nh, int fl) -> bool {
            const int ab = uu & 1;
            const bool tr = warp == 2 && lane == 0;
            if (tr) trace_ev_atomic<TRACE>(p, 2, 0, L, nh, tt, gs);
            bool mine = false;
            if (L == NL - 1) {
                mine = DECODE ? (tt % EPI_PER_Q == part) : ((int)(lu % EPI_PER_Q) == part);
                ++lu;
            }
            // decoding: this row's coder state and quotient, fetched before the logits are ready
            int64_t drow = 0, dc = 0;
            bool dlive = false;
            DecState ds{};
            uint64_t dscale = 0, dq = 0;
            if (DECODE && mine && L == NL - 1) {
                drow = (int64_t)(2 * pt + (int)rank) * TM + r;
                dlive = drow < p.n_rows;
                dc = dlive ? p.order[drow] : 0;
                dlive = dlive && step < p.lengths[dc] && !p.errors[dc];
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
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(&acc_full[ab], (uu >> 1) & 1))) return false;
            if (tr) trace_ev_atomic<TRACE>(p, 2, 1, L, nh, tt, gs);
            ++uu;
            tc_fence_after();
            const int NH = p.out_dim[L] / TN;
            if (L >= 1 && nh == NH - 1) {
                // every MMA that reads this tile's layer-L input has completed: its rows are
                // dead until layer L+1 overwrites them, so drop them from L2 instead of
                // letting them be written back to DRAM (each warp of the quarter takes every
                // third 128-byte line of its rows)
                const int8_t *in_row = p.act_ptr[(L - 1) & 1] + (size_t)(slot_row0 + tt * TM + r) * MAX_N;
                for (int ln = part; ln < p.in_dim[L] / 128; ln += EPI_PER_Q) discard_l2_line(in_row + ln * 128);
            }
            const uint32_t taddr = tmem_base + ab * TN + ((uint32_t)(q * 32) << 16);
            const Requant rq = p.rq[L];
            // fast-path parameters as scalars (uniform per unit)
            const bool rq_fast = rq.hi_path != 0;
            const int32_t rq_m0 = (int32_t)rq.m0, rq_hs = rq.hi_shift, rq_one = rq.one;
            const uint32_t rq_relu = rq.lo == 0 ? 0xFFFFFFFFu : 0u;
            // the layers after the first take their bias through their bias tiles (nb); without a
            // tile, compress reads it from SMEM and the decoder (which keeps only layer 0's bias
            // in SMEM) from global memory
            const int32_t *bias = (!DECODE || L == 0) ? bias_s + L * MAX_N : p.bias[L];
            const bool nb = L != 0 && ((p.bias_mma >> L) & 1u);
            const uint32_t acc_empty_leader = map_to_rank(&acc_empty[ab], 0);
            const int tile = 2 * pt + (int)rank;
            // hidden layers; NB: the accumulator holds the bias already (bias tile).  The
            // two forms are separate instantiations, so neither carries the other's registers.
            auto hidden_unit = [&](auto NB) -> bool {
                int8_t *dst_row = p.act_ptr[L & 1] + (size_t)(slot_row0 + tt * TM + r) * MAX_N + nh * TN;
                // requantise chunk c (32 columns) of this row and store it to the activations
                // with one 32-byte store
                auto store_chunk = [&](const uint32_t (&va)[32], int c) {
                    uint32_t packed[8];
                    if constexpr (decltype(NB)::value) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) packed[i] = requant4_hi_nb(&va[4 * i], rq_m0, rq_hs, rq_relu);
                    } else {
                        const int4 *bv = reinterpret_cast<const int4 *>(bias + nh * TN + c * 32);
                        if (rq_fast) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) packed[i] = requant4_hi(&va[4 * i], bv[i], rq_m0, rq_hs, rq_relu, rq_one);
                        } else {
#pragma unroll
                            for (int i = 0; i < 8; ++i) packed[i] = requant4(&va[4 * i], bv[i], rq);
                        }
                    }
                    st_global_v8(dst_row + c * 32, packed);
                };
                // chunks part, part + 3 and (parts 0 and 1) part + 6: each chunk's TMEM load is
                // issued before the previous chunk is requantised, and the accumulator is
                // released as soon as the last load has landed, before the last chunk's stores
                const int c0 = part, c1 = part + EPI_PER_Q, c2 = part + 2 * EPI_PER_Q;
                const bool three = c2 < TN / 32;                // warp-uniform
                uint32_t va[32], vb[32];
                tmem_ld32(taddr + c0 * 32, va);
                tmem_ld_wait();
                tmem_ld32(taddr + c1 * 32, vb);
                store_chunk(va, c0);
                tmem_ld_wait();
                if (three) tmem_ld32(taddr + c2 * 32, va);
                if (three) {
                    store_chunk(vb, c1);
                    tmem_ld_wait();
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster_relaxed(acc_empty_leader);
                if (three) store_chunk(va, c2);
                else store_chunk(vb, c1);
                if (nh == NH - 1) {
                    fence_proxy_async_global();
                    __syncwarp();
                    if (lane == 0) counter_add_release(&act_cnt[tt], 1);
                }
                if (tr) trace_ev_atomic<TRACE>(p, 2, 2, L, nh, tt, gs);
                return true;
            };
            if (L < NL - 1) {
                if (nb) return hidden_unit(std::true_type{});
                return hidden_unit(std::false_type{});
            }
            if (mine) {
                // last layer: requantise the 256 logits of this row, keep them packed in the
                // first 64 columns of the same accumulator (already read) and track the maximum
                int mlogit = -128;
#pragma unroll 1
                for (int c = 0; c < 8; ++c) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c * 32, v);
                    tmem_ld_wait();
                    const int4 *bv = reinterpret_cast<const int4 *>(bias + c * 32);
                    uint32_t w8[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        w8[i] = nb ? requant4_hi_nb(&v[4 * i], rq_m0, rq_hs, rq_relu)
                                   : rq_fast ? requant4_hi(&v[4 * i], bv[i], rq_m0, rq_hs, rq_relu, rq_one)
                                             : requant4(&v[4 * i], bv[i], rq);
#pragma unroll
                        for (int b = 0; b < 4; ++b) mlogit = max(mlogit, pk_get(w8[i], b));
                    }
                    tmem_st8(taddr + c * 8, w8);
                }
                tmem_st_wait();
                // warp-collective TMEM passes: every lane runs them, rows without work
                // compute on dummy inputs and store nothing
                if (!DECODE) {
                    const bool real_tile = tile < p.n_tiles;
                    const int c = real_tile ? p.tile_chunk[tile] : 0;
                    const int t0 = real_tile ? p.tile_t0[tile] : 0;
                    const int64_t begin = p.tok_off[c];
                    const bool valid = real_tile && t0 + r < p.tok_off[c + 1] - begin;
                    const int sym = valid ? p.tokens[begin + t0 + r] : 0;
                    int amax;
                    RowDivisor d;
                    uint32_t fix, cum, f;
                    row_stats(taddr, lut_s, mlogit, d, fix, amax, sym, cum, f);
                    if (valid) p.pairs[begin - p.row_base + t0 + r] = make_uint2(cum, f);
                } else {
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
                        // append the token's embedding row to this row's window ring; the ring is
                        // read back only 1 to 64 steps later, long after L2 would have to keep it,
                        // so the append goes out with the evict-first policy
                        const uint4 *e = reinterpret_cast<const uint4 *>(p.emb + sym * EMB_DIM);
                        uint8_t *dst = reinterpret_cast<uint8_t *>(
                            p.ering_ptr + (((size_t)(blockIdx.x * kt2<DECODE>() + tt) * WIN + (step & (WIN - 1))) * TM + r) * KB);
                        const uint64_t pol = l2_policy_evict_first();
#pragma unroll
                        for (int i = 0; i < KB / 32; ++i) {
                            const uint4 a = e[2 * i], b = e[2 * i + 1];
                            const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                            st_global_v8_hint(dst + 32 * i, v, pol);
                        }
                    }
                    fence_proxy_async_global();          // the ring block is read by TMA next step
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_cluster_relaxed(acc_empty_leader);
                counter_add_release(&act_cnt[tt], 1);
            }
            if (tr) trace_ev_atomic<TRACE>(p, 2, 2, L, nh, tt, gs);
            return true;
        });
    } else if (!DECODE) {
        // ---- last two warps (compress): sliding embedding buffer of this CTA's tile
        const int tw = threadIdx.x - 32 * (2 + EPI_WARPS);   // 0..63
        const int j = tw & 7, r0 = tw >> 3;
        uint32_t li = 0;
        for_each_unit2<DECODE>(p, [&](int gs, int tt, int pt, int step, int L, int nh, int fl) -> bool {
            if (L != 0 || nh != 0) return true;
            const int gb = li & 1;
            if (!__all_sync(0xffffffffu, mbar_wait_cluster(&g_empty[gb], ((li >> 1) & 1) ^ 1))) return false;
            ++li;
            uint8_t *g = xbuf + gb * G_BYTES;
            const int tile = 2 * pt + (int)rank;
            const bool real_tile = tile < p.n_tiles;
            const int c = real_tile ? p.tile_chunk[tile] : 0;
            const int t0 = real_tile ? p.tile_t0[tile] : 0;
            const int64_t begin = p.tok_off[c];
            const int64_t len = real_tile ? p.tok_off[c + 1] - begin : 0;
#pragma unroll 4
            for (int sr = r0; sr < G_ROWS; sr += 8) {
                const int64_t pos = (int64_t)t0 - WIN + sr;
                const int tok = pos < 0 ? SC_SOS : (pos < len ? p.tokens[begin + pos] : 0);
                const int4 v = *reinterpret_cast<const int4 *>(p.emb + tok * EMB_DIM + j * 16);
                *reinterpret_cast<int4 *>(g + sw128_offset(sr, j)) = v;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(map_to_rank(&g_full[gb], 0));
            return true;
        });
    }
    // Teardown.  Every MMA has completed once the drain barrier's phase 0 does (the issuer's
    // last commit, after all its MMAs and commits); only then is TMEM freed.  The wait is
    // bounded: on a timeout the device error flag is already set by the role that gave up.
    if (warp == 1) mbar_wait_cluster_drain(drain, 0);
    tc_fence_before();
    __syncthreads();
    cluster_sync();                       // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, 2 * TN);
    }
}

}  // namespace
}  // namespace sc
