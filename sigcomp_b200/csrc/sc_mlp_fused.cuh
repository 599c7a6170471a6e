// Fused persistent MLP kernels: all layers of the entropy model per 128-row
// tile in one launch, with the entropy-coder step fused into the last layer's
// epilogue.  Included by sc_mlp_tc.cu (same translation unit as the layer
// kernels and the device error flag).
//
// Each CTA owns up to KT tiles ("slots") and walks, for every step, every
// layer over all of its tiles in round-robin, so that while one tile's
// epilogue runs the tensor core is already busy with another tile:
//
//   for step:                       (decode: autoregressive steps; compress: 1)
//     for layer L:
//       for slot tt:                (tiles still active at this step)
//         for output half nh:       one 128x256 TMEM accumulator ("unit")
//
// Activations of slot tt live in two global ping-pong buffers (L2 resident,
// rows (blockIdx.x*KT + tt)*128 ...), written by the epilogue and read back by
// TMA for the next layer.  Per-slot monotonic counters (act_cnt) order an
// epilogue's global writes before the TMA reads of the next layer.
//
// Layer 0 operand A:
//   compress  sliding embedding buffer per tile (rows t0-64 .. t0+127 of the
//             chunk), K block p = rows p .. p+127 (no per-K-block gather)
//   decode    built per K block from the embedding table in shared memory and
//             a per-slot ring of the last 64 decoded tokens of every row
// Last layer epilogue (one thread per row, all 256 logits in registers):
//   compress  (cum, freq) of the row's symbol      (_frequencies + _encode_one's
//             inputs, sigcomp/cpu_entropy_coding.py:90-110, 121-131)
//   decode    one range-decoder step                (_decode_partition,
//             sigcomp/cpu_entropy_coding.py:230-266), token appended to the
//             output and to the slot's window ring
#pragma once

namespace sc {

constexpr int FMAX_LAYERS = 9;
constexpr int KT = 5;                 // tiles in flight per CTA

struct FusedParams {
    CUtensorMap w[FMAX_LAYERS];       // weights, box 256 x 128 B
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
    // compress
    const int32_t *tile_chunk;
    const int32_t *tile_t0;
    const int64_t *tok_off;
    const uint8_t *tokens;
    int64_t row_base;
    uint2 *pairs;
    // decode
    const int64_t *order;             // launch row -> chunk
    int64_t n_rows;
    const int32_t *tile_maxlen;       // steps of each tile (its first row's length)
    const int64_t *lengths;           // chunk -> tokens
    DecState *state;                  // launch row -> decoder state
    const uint32_t *words;
    uint8_t *tokens_out;
    const int64_t *out_off;           // chunk -> first output token
    uint8_t *errors;                  // chunk -> error flag
};

namespace {

template <bool DECODE>
struct FCfg {
    static constexpr int STAGES = 3;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;                 // 48 KB
    static constexpr int OFF_X = STAGES * STAGE_BYTES;                    // 144 KB
    static constexpr int EMB_PAD = 33 * 1024;
    static constexpr int RING_BYTES = TM * WIN;                           // 8 KB per slot
    static constexpr int X_BYTES = DECODE ? EMB_PAD + KT * RING_BYTES : 2 * G_BYTES;
    static constexpr int OFF_LUT = OFF_X + X_BYTES;
    static constexpr int OFF_BAR = OFF_LUT + 256 * 8;
    static constexpr int NBAR = 2 * STAGES + 4 + 4;
    static constexpr int OFF_CNT = OFF_BAR + NBAR * 8;               // act_cnt[KT]
    static constexpr int OFF_TMEM = OFF_CNT + 8 * 4;
    static constexpr int SMEM = OFF_TMEM + 16 + 1024;
};

__device__ __forceinline__ int pk_get(uint32_t w, int b) { return (int)(int8_t)(uint8_t)(w >> (8 * b)); }

// The row's 256 int8 logits are kept packed (4 per word) in TMEM columns
// taddr .. taddr+63 of the thread's lane; each pass streams them back 8 words
// (32 logits) at a time, which keeps the register footprint small.

// Frequency-table statistics of one row (_frequencies, cpu_entropy_coding.py:90-110):
// maximum logit, row divisor (sum of exp weights), the fix-up amount and the
// first index of the maximum frequency.  With sym >= 0 it also returns the
// exclusive cumulative frequency and the frequency of `sym`, fix-up applied.
__device__ __forceinline__ void row_freq_stats(uint32_t taddr, const uint64_t *lut_s, int &m, RowDivisor &d,
                                               uint32_t &fix, int &amax, int sym, uint32_t &sym_cum,
                                               uint32_t &sym_f)
{
    m = -128;
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
        uint32_t w[8];
        tmem_ld8(taddr + g * 8, w);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int b = 0; b < 4; ++b) m = max(m, pk_get(w[i], b));
    }
    uint64_t T = 0;
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
        uint32_t w[8];
        tmem_ld8(taddr + g * 8, w);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int b = 0; b < 4; ++b) T += lut_s[m - pk_get(w[i], b)];
    }
    d = make_row_divisor(T);
    uint32_t total = 0, best = 0, below = 0, fsym = 0;
    amax = 0;
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
        uint32_t w[8];
        tmem_ld8(taddr + g * 8, w);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int v = g * 32 + 4 * i + b;
                uint32_t f = div_freq(lut_s[m - pk_get(w[i], b)], d);
                f = f < 1u ? 1u : f;
                total += f;
                if (f > best) { best = f; amax = v; }
                below += v < sym ? f : 0u;
                fsym = v == sym ? f : fsym;
            }
    }
    fix = total - SC_TOTAL;          // modulo 2^32; subtracting it from f[amax] is exact
    sym_cum = below - (amax < sym ? fix : 0u);
    sym_f = fsym - (amax == sym ? fix : 0u);
}

// The symbol whose cumulative interval holds `q` (the largest v with cum_v <= q).
__device__ __forceinline__ void row_search(uint32_t taddr, const uint64_t *lut_s, int m, const RowDivisor &d,
                                           uint32_t fix, int amax, uint32_t q, int &sym, uint32_t &sym_cum,
                                           uint32_t &sym_f)
{
    uint32_t cum = 0;
    sym = 0;
    sym_cum = 0;
    sym_f = 0;
#pragma unroll 1
    for (int g = 0; g < 8; ++g) {
        uint32_t w[8];
        tmem_ld8(taddr + g * 8, w);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int v = g * 32 + 4 * i + b;
                uint32_t f = div_freq(lut_s[m - pk_get(w[i], b)], d);
                f = f < 1u ? 1u : f;
                f -= v == amax ? fix : 0u;
                if (cum <= q) { sym = v; sym_cum = cum; sym_f = f; }
                cum += f;
            }
    }
}

// Walk this CTA's units in the fixed order every role follows.  `f` returns
// false to stop (a timed-out wait).
template <bool DECODE, typename F>
__device__ __forceinline__ void for_each_unit(const FusedParams &p, F &&f)
{
    const int G = gridDim.x;
    const int my_tiles = p.n_tiles > (int)blockIdx.x ? (p.n_tiles - 1 - (int)blockIdx.x) / G + 1 : 0;
    const int NL = p.num_layers;
    for (int g0 = 0, grp = 0; g0 < my_tiles; g0 += KT, ++grp) {
        const int gn = min(KT, my_tiles - g0);
        int maxlen[KT];
        int steps = 1;
#pragma unroll
        for (int tt = 0; tt < KT; ++tt) {
            maxlen[tt] = 0;
            if (tt < gn) {
                maxlen[tt] = DECODE ? p.tile_maxlen[blockIdx.x + (g0 + tt) * G] : 1;
                steps = max(steps, maxlen[tt]);
            }
        }
        for (int step = 0; step < steps; ++step)
            for (int L = 0; L < NL; ++L)
#pragma unroll 1
                for (int tt = 0; tt < gn; ++tt) {
                    if (DECODE && maxlen[tt] <= step) continue;
                    const int tile = blockIdx.x + (g0 + tt) * G;
                    const int NH = p.out_dim[L] / TN;
                    for (int nh = 0; nh < NH; ++nh)
                        if (!f(grp, tt, tile, step, L, nh)) return;
                }
    }
}

__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

template <bool DECODE>
__global__ void __launch_bounds__(256, 1) k_fused(const __grid_constant__ FusedParams p)
{
    using C = FCfg<DECODE>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *bars = (uint64_t *)(smem + C::OFF_BAR);
    uint64_t *full = bars, *empty = bars + C::STAGES;
    uint64_t *acc_full = bars + 2 * C::STAGES, *acc_empty = acc_full + 2;
    uint64_t *g_full = acc_empty + 2, *g_empty = g_full + 2;
    // act_cnt[tt]: +1 per epilogue warp when slot tt finishes a layer, so layer
    // completion number k (0-based, counted over the slot's steps or groups) is
    // reached when act_cnt[tt] >= 4 * (k + 1)
    uint32_t *act_cnt = (uint32_t *)(smem + C::OFF_CNT);
    uint32_t *tmem_slot = (uint32_t *)(smem + C::OFF_TMEM);
    uint64_t *lut_s = (uint64_t *)(smem + C::OFF_LUT);
    uint8_t *xbuf = smem + C::OFF_X;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NL = p.num_layers;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], DECODE ? 1 + 2 : 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
            mbar_init(&g_full[b], 2);
            mbar_init(&g_empty[b], 1);
        }
        for (int tt = 0; tt < 8; ++tt) act_cnt[tt] = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, 2 * TN);
        tmem_relinquish();
    }
    for (int i = threadIdx.x; i < SC_VOCAB; i += blockDim.x) lut_s[i] = p.lut[i];
    if (DECODE) {
        const int4 *srcv = reinterpret_cast<const int4 *>(p.emb);
        int4 *dst = reinterpret_cast<int4 *>(xbuf);
        for (int i = threadIdx.x; i < EMB_BYTES / 16; i += blockDim.x) dst[i] = srcv[i];
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int slot_row0 = blockIdx.x * KT * TM;

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer: weights every unit; activations for layers >= 1
            uint32_t it = 0;
            for_each_unit<DECODE>(p, [&](int grp, int tt, int tile, int step, int L, int nh) -> bool {
                const int nkb = p.in_dim[L] / KB;
                if (L >= 1 && nh == 0) {
                    const uint32_t k = (uint32_t)((DECODE ? step : grp) * NL + L - 1);
                    if (!counter_wait(&act_cnt[tt], 4 * (k + 1))) return false;
                }
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    if (!mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1)) return false;
                    uint8_t *st = smem + s * C::STAGE_BYTES;
                    if (L == 0) {
                        mbar_arrive_expect_tx(&full[s], B_BYTES);
                    } else {
                        mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
                        tma_load_2d(st, &p.act[(L - 1) & 1], &full[s], kb * KB, slot_row0 + tt * TM);
                    }
                    tma_load_2d(st + A_BYTES, &p.w[L], &full[s], kb * KB, nh * TN);
                }
                return true;
            });
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            uint32_t it = 0, uu = 0, li = 0;
            for_each_unit<DECODE>(p, [&](int grp, int tt, int tile, int step, int L, int nh) -> bool {
                const int nkb = p.in_dim[L] / KB;
                const int ab = uu & 1;
                if (!mbar_wait(&acc_empty[ab], ((uu >> 1) & 1) ^ 1)) return false;
                const int gb = li & 1;
                if (!DECODE && L == 0 && nh == 0 && !mbar_wait(&g_full[gb], (li >> 1) & 1)) return false;
                tc_fence_after();
                const uint32_t d = tmem_base + ab * TN;
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % C::STAGES;
                    if (!mbar_wait(&full[s], (it / C::STAGES) & 1)) return false;
                    tc_fence_after();
                    const uint32_t st = smem_u32(smem + s * C::STAGE_BYTES);
                    const uint32_t a_addr =
                        (!DECODE && L == 0) ? smem_u32(xbuf + gb * G_BYTES) + kb * KB : st;
                    mma_k_block(d, a_addr, st + A_BYTES, kb == 0);
                    mma_commit(&empty[s]);
                }
                mma_commit(&acc_full[ab]);
                ++uu;
                if (!DECODE && L == 0 && nh == p.out_dim[0] / TN - 1) {
                    mma_commit(&g_empty[gb]);
                    ++li;
                }
                return true;
            });
        }
    } else if (warp >= 2 && warp <= 5) {
        // ---- epilogue warps: TMEM lane quarter q, row r of the tile
        const int q = warp & 3;
        const int r = q * 32 + lane;
        uint32_t uu = 0;
        for_each_unit<DECODE>(p, [&](int grp, int tt, int tile, int step, int L, int nh) -> bool {
            const int ab = uu & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (uu >> 1) & 1))) return false;
            ++uu;
            tc_fence_after();
            const uint32_t taddr = tmem_base + ab * TN + ((uint32_t)(q * 32) << 16);
            const Requant rq = p.rq[L];
            const int32_t *bias = p.bias[L];
            if (L < NL - 1) {
                int8_t *dst_row = p.act_ptr[L & 1] + (size_t)(slot_row0 + tt * TM + r) * MAX_N + nh * TN;
#pragma unroll 1
                for (int c = 0; c < TN / 32; ++c) {
                    uint32_t v[32];
                    tmem_ld32(taddr + c * 32, v);
                    tmem_ld_wait();
                    uint32_t packed[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        uint32_t w = 0;
#pragma unroll
                        for (int b = 0; b < 4; ++b) {
                            const int col = nh * TN + c * 32 + i * 4 + b;
                            const int32_t o = requant((int32_t)v[i * 4 + b], __ldg(bias + col), rq);
                            w |= ((uint32_t)(o & 0xFF)) << (8 * b);
                        }
                        packed[i] = w;
                    }
                    uint4 *dst = reinterpret_cast<uint4 *>(dst_row + c * 32);
                    dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                    dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[ab]);
                if (nh == p.out_dim[L] / TN - 1) {
                    fence_proxy_async_global();
                    __syncwarp();
                    if (lane == 0) counter_add_release(&act_cnt[tt], 1);
                }
                return true;
            }
            // last layer: requantise the 256 logits of this row and keep them packed
            // in the first 64 columns of the same accumulator (already read)
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {
                uint32_t v[32];
                tmem_ld32(taddr + c * 32, v);
                tmem_ld_wait();
                uint32_t w8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    uint32_t w = 0;
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const int col = c * 32 + i * 4 + b;
                        const int32_t o = requant((int32_t)v[i * 4 + b], __ldg(bias + col), rq);
                        w |= ((uint32_t)(o & 0xFF)) << (8 * b);
                    }
                    w8[i] = w;
                }
                tmem_st8(taddr + c * 8, w8);
            }
            tmem_st_wait();
            // the passes below issue warp-collective TMEM loads: every lane runs them,
            // lanes of rows without work compute on dummy inputs and store nothing
            if (!DECODE) {
                const int c = p.tile_chunk[tile];
                const int t0 = p.tile_t0[tile];
                const int64_t begin = p.tok_off[c];
                const bool valid = t0 + r < p.tok_off[c + 1] - begin;
                const int sym = valid ? p.tokens[begin + t0 + r] : 0;
                int m, amax;
                RowDivisor d;
                uint32_t fix, cum, f;
                row_freq_stats(taddr, lut_s, m, d, fix, amax, sym, cum, f);
                if (valid) p.pairs[begin - p.row_base + t0 + r] = make_uint2(cum, f);
            } else {
                const int64_t row = (int64_t)tile * TM + r;
                bool live = row < p.n_rows;
                const int64_t c = live ? p.order[row] : 0;
                live = live && step < p.lengths[c] && !p.errors[c];
                DecState s{};
                uint64_t scale = 0, qv = 0;
                if (live) {
                    s = p.state[row];
                    scale = s.range >> SC_PRECISION;
                    qv = scale ? (s.point - s.lower) / scale : ~0ull;
                    if (qv >= (uint64_t)SC_TOTAL) {      // invalid stream (cpu_entropy_coding.py:244-248)
                        p.errors[c] = 1;
                        live = false;
                    }
                }
                int m, amax, sym;
                RowDivisor d;
                uint32_t fix, cum, f;
                row_freq_stats(taddr, lut_s, m, d, fix, amax, -1, cum, f);
                row_search(taddr, lut_s, m, d, fix, amax, live ? (uint32_t)qv : 0u, sym, cum, f);
                if (live) {
                    s.lower += scale * (uint64_t)cum;
                    s.range = scale * (uint64_t)f;
                    if (s.range < (1ull << 32)) {
                        s.lower <<= 32;
                        s.range <<= 32;
                        s.point <<= 32;
                        if (s.read_pos < s.end_pos) s.point |= p.words[s.read_pos];
                        s.read_pos += 1;
                    }
                    p.state[row] = s;
                    p.tokens_out[p.out_off[c] + step] = (uint8_t)sym;
                    uint8_t *ring = xbuf + C::EMB_PAD + tt * C::RING_BYTES;
                    ring[r * WIN + (step & (WIN - 1))] = (uint8_t)sym;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&acc_empty[ab]);
                counter_add_release(&act_cnt[tt], 1);
            }
            return true;
        });
    } else if (DECODE) {
        // ---- warps 6-7: layer-0 activation stages from the embedding table and
        // the window rings (warp 6 rows 0-63, warp 7 rows 64-127)
        const int wb = (warp - 6) * 64;
        const int j = lane & 7, sub = lane >> 3;
        const uint8_t *emb_s = xbuf;
        uint32_t it = 0;
        // the builders take part in every ring iteration (their arrivals are part of
        // each stage's count), building the activation only for layer-0 stages; this
        // keeps their parity waits on `empty` at most one phase away
        for_each_unit<DECODE>(p, [&](int grp, int tt, int tile, int step, int L, int nh) -> bool {
            const int nkb = p.in_dim[L] / KB;
            if (L == 0 && nh == 0 && step > 0) {
                // the window ring holds step-1's token once the slot finished its last layer
                const uint32_t k = (uint32_t)(step * NL - 1);
                if (!__all_sync(0xffffffffu, counter_wait(&act_cnt[tt], 4 * (k + 1)))) return false;
            }
            const uint8_t *ring = xbuf + C::EMB_PAD + tt * C::RING_BYTES;
            for (int kb = 0; kb < nkb; ++kb, ++it) {
                const int s = it % C::STAGES;
                if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ((it / C::STAGES) & 1) ^ 1))) return false;
                if (L == 0) {
                    uint8_t *a_st = smem + s * C::STAGE_BYTES;
                    const int pos = step - WIN + kb;
#pragma unroll 4
                    for (int rr = sub; rr < 64; rr += 4) {
                        const int rrow = wb + rr;
                        const int tok = pos < 0 ? SC_SOS : ring[rrow * WIN + (pos & (WIN - 1))];
                        const int4 v = *reinterpret_cast<const int4 *>(emb_s + tok * EMB_DIM + j * 16);
                        *reinterpret_cast<int4 *>(a_st + sw128_offset(rrow, j)) = v;
                    }
                    fence_proxy_async_smem();
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[s]);
            }
            return true;
        });
    } else {
        // ---- warps 6-7 (compress): sliding embedding buffer of each tile
        const int tw = threadIdx.x - 192;        // 0..63
        const int j = tw & 7, r0 = tw >> 3;
        uint32_t li = 0;
        for_each_unit<DECODE>(p, [&](int grp, int tt, int tile, int step, int L, int nh) -> bool {
            if (L != 0 || nh != 0) return true;
            const int gb = li & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&g_empty[gb], ((li >> 1) & 1) ^ 1))) return false;
            ++li;
            uint8_t *g = xbuf + gb * G_BYTES;
            const int c = p.tile_chunk[tile];
            const int t0 = p.tile_t0[tile];
            const int64_t begin = p.tok_off[c];
            const int64_t len = p.tok_off[c + 1] - begin;
#pragma unroll 4
            for (int sr = r0; sr < G_ROWS; sr += 8) {
                const int64_t pos = (int64_t)t0 - WIN + sr;
                const int tok = pos < 0 ? SC_SOS : (pos < len ? p.tokens[begin + pos] : 0);
                const int4 v = *reinterpret_cast<const int4 *>(p.emb + tok * EMB_DIM + j * 16);
                *reinterpret_cast<int4 *>(g + sw128_offset(sr, j)) = v;
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&g_full[gb]);
            return true;
        });
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
