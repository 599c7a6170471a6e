// Shared device helpers of the sigcomp_b200 codec kernels.
//
// Exact integer semantics follow the reference CPU codec:
//   requantise  - _requantize            sigcomp/cpu_int_kernels.py:5-14
//   frequencies - _frequencies           sigcomp/cpu_entropy_coding.py:90-110
//   encoder     - _encode_one / _seal    sigcomp/cpu_entropy_coding.py:121-161, 206-227
//   decoder     - _decode_partition      sigcomp/cpu_entropy_coding.py:230-266
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define SC_VOCAB 256
#define SC_SOS 256
#define SC_PRECISION 24
#define SC_TOTAL (1u << 24)
#define SC_LUT_ONE (1ull << 38)

namespace sc {

// ---------------------------------------------------------------------------
// Requantisation: y = clamp(((int64)(int32)(acc + bias) * M0) >> shift, lo, 127)
// Arithmetic right shift of a signed product is floor division by 2^shift.
// ---------------------------------------------------------------------------
struct Requant {
    int64_t m0;      // in [0, 2^31]
    int32_t shift;   // in [0, 63]
    int32_t lo;      // 0 with ReLU, -128 without
    int32_t hi_path; // 1: m0 < 2^31 and shift >= 32 -> 32-bit mulhi form
    int32_t hi_shift;
    int32_t one;     // 1 (a run-time operand of the fast path's multiply-add)
};

__host__ __device__ inline Requant make_requant(int64_t m0, int32_t shift, int32_t relu) {
    Requant r;
    r.m0 = m0;
    r.shift = shift;
    r.lo = relu ? 0 : -128;
    r.hi_path = (m0 < (1ll << 31) && shift >= 32) ? 1 : 0;
    r.hi_shift = shift - 32;
    r.one = 1;
    return r;
}

__device__ __forceinline__ int32_t requant(int32_t acc, int32_t bias, const Requant &q) {
    const int32_t biased = (int32_t)((uint32_t)acc + (uint32_t)bias);   // int32 wrap
    int64_t scaled;
    if (q.hi_path) {
        // floor(biased * M0 / 2^32) is the high word of the signed 64-bit product;
        // a further arithmetic shift floors again: floor(floor(x / a) / b) = floor(x / ab).
        scaled = (int64_t)(__mulhi(biased, (int32_t)q.m0) >> q.hi_shift);
    } else {
        scaled = ((int64_t)biased * q.m0) >> q.shift;
    }
    scaled = scaled < q.lo ? q.lo : scaled;
    scaled = scaled > 127 ? 127 : scaled;
    return (int32_t)scaled;
}

// Four requantised outputs packed as int8 (lowest column in the lowest byte).
// Fast form for multipliers with the high-word path (M0 < 2^31, shift >= 32):
// the int32 wrap of acc + bias, the high word of the 64-bit product and an
// arithmetic shift give floor(biased * M0 / 2^shift); the lower bound (0 with
// ReLU, else -128) is applied with max, and cvt.pack.sat saturates to 127.
__device__ __forceinline__ uint32_t sat_pack4(int32_t r0, int32_t r1, int32_t r2, int32_t r3) {
    uint32_t hi, d;
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(r3), "r"(r2), "r"(0));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(r1), "r"(r0), "r"(hi));
    return d;
}

__device__ __forceinline__ int32_t requant_hi(uint32_t acc, int32_t bias, int32_t m0, int32_t hs, int32_t lo) {
    return max(__mulhi((int32_t)(acc + (uint32_t)bias), m0) >> hs, lo);
}

// requant4 with the fast-path parameters in registers (M0 < 2^31, shift >= 32),
// arranged to spread the work over the integer pipes: the bias is added by a
// multiply-add (`one` is 1 at run time), cvt.pack.sat clamps to [-128, 127],
// and the ReLU lower bound is applied to the four packed bytes at once
// (prmt replicates each byte's sign; relu_mask is all ones with ReLU, else 0).
__device__ __forceinline__ uint32_t requant4_hi(const uint32_t *acc, int4 bias, int32_t m0, int32_t hs,
                                                uint32_t relu_mask, int32_t one) {
    const int32_t v0 = __mulhi((int32_t)(acc[0] * (uint32_t)one + (uint32_t)bias.x), m0) >> hs;
    const int32_t v1 = __mulhi((int32_t)(acc[1] * (uint32_t)one + (uint32_t)bias.y), m0) >> hs;
    const int32_t v2 = __mulhi((int32_t)(acc[2] * (uint32_t)one + (uint32_t)bias.z), m0) >> hs;
    const int32_t v3 = __mulhi((int32_t)(acc[3] * (uint32_t)one + (uint32_t)bias.w), m0) >> hs;
    const uint32_t d = sat_pack4(v0, v1, v2, v3);
    uint32_t sgn;
    asm("prmt.b32 %0, %1, %1, 0xBA98;" : "=r"(sgn) : "r"(d));
    return d & ~(sgn & relu_mask);
}

// requant4_hi for an accumulator that already holds the bias (no bias load, no bias add)
__device__ __forceinline__ uint32_t requant4_hi_nb(const uint32_t *acc, int32_t m0, int32_t hs, uint32_t relu_mask) {
    const uint32_t d = sat_pack4(__mulhi((int32_t)acc[0], m0) >> hs, __mulhi((int32_t)acc[1], m0) >> hs,
                                 __mulhi((int32_t)acc[2], m0) >> hs, __mulhi((int32_t)acc[3], m0) >> hs);
    uint32_t sgn;
    asm("prmt.b32 %0, %1, %1, 0xBA98;" : "=r"(sgn) : "r"(d));
    return d & ~(sgn & relu_mask);
}

__device__ __forceinline__ uint32_t requant4(const uint32_t *acc, int4 bias, const Requant &q) {
    if (q.hi_path) {
        const int32_t m0 = (int32_t)q.m0, hs = q.hi_shift, lo = q.lo;
        return sat_pack4(requant_hi(acc[0], bias.x, m0, hs, lo), requant_hi(acc[1], bias.y, m0, hs, lo),
                         requant_hi(acc[2], bias.z, m0, hs, lo), requant_hi(acc[3], bias.w, m0, hs, lo));
    }
    const int32_t o0 = requant((int32_t)acc[0], bias.x, q), o1 = requant((int32_t)acc[1], bias.y, q);
    const int32_t o2 = requant((int32_t)acc[2], bias.z, q), o3 = requant((int32_t)acc[3], bias.w, q);
    return (uint32_t)(o0 & 0xFF) | ((uint32_t)(o1 & 0xFF) << 8) | ((uint32_t)(o2 & 0xFF) << 16) |
           ((uint32_t)(o3 & 0xFF) << 24);
}

// ---------------------------------------------------------------------------
// Exact floor(w * 2^24 / T) for one row with invariant divisor T.
// Preconditions (guaranteed by build_integer_exp_lut tables, lut[0] = 2^38,
// lut[i] <= 2^38): w <= 2^38 and 2^38 <= T <= 2^46.
// Method: invariant-divisor reciprocal (Granlund & Montgomery, "Division by
// Invariant Integers using Multiplication", 1994), specialised here:
//   R = floor(2^62 / T) <= 2^24;  q0 = floor(w * R / 2^38)  (w * R <= 2^62).
//   Since 2^62/T - 1 < R <= 2^62/T, q - 1 <= q0 <= q, one correction step
//   with the remainder w * 2^24 - q0 * T restores the exact quotient.
// ---------------------------------------------------------------------------
struct RowDivisor {
    uint64_t T;
    uint64_t R;
};

__device__ __forceinline__ RowDivisor make_row_divisor(uint64_t T) {
    RowDivisor d;
    d.T = T;
    d.R = (1ull << 62) / T;
    return d;
}

__device__ __forceinline__ uint32_t div_freq(uint64_t w, const RowDivisor &d) {
    // floor(w * R / 2^38) in 32-bit pieces: w = wh * 2^32 + wl (wh <= 64), R < 2^25, so
    // floor(w * R / 2^32) = wh * R + mulhi(wl, R) < 2^31 exactly; one more shift by 6.
    const uint32_t wl = (uint32_t)w, wh = (uint32_t)(w >> 32), R = (uint32_t)d.R;
    uint32_t q = (wh * R + __umulhi(wl, R)) >> 6;
    const uint64_t r = (w << 24) - (uint64_t)q * d.T;   // true remainder in [0, 2T), mod 2^64
    q += (r >= d.T) ? 1u : 0u;
    return q;
}

// ---------------------------------------------------------------------------
// Warp-cooperative frequency table of one row of 256 int8 logits.
// Lane l owns symbols 8l .. 8l+7.  On return f[j] is the final 24-bit
// frequency of symbol 8*lane + j (sum over the row is exactly 2^24).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void warp_frequencies(const int8_t x[8], const uint64_t *lut_s, uint32_t f[8]) {
    const int lane = threadIdx.x & 31;
    int m = x[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) m = max(m, (int)x[j]);
#pragma unroll
    for (int o = 16; o; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    uint64_t w[8];
    uint64_t s = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        w[j] = lut_s[m - x[j]];
        s += w[j];
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const RowDivisor d = make_row_divisor(s);
    uint32_t lsum = 0, lmax = 0;
    int lidx = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t q = div_freq(w[j], d);
        q = q < 1u ? 1u : q;
        f[j] = q;
        lsum += q;
        if (q > lmax) { lmax = q; lidx = j; }
    }
    uint32_t total = lsum;
#pragma unroll
    for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    // first index of the maximum: larger value wins, ties go to the lower symbol
    uint32_t bv = lmax;
    int bi = lane * 8 + lidx;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const uint32_t ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((bi >> 3) == lane) {
        const uint32_t excess = total - SC_TOTAL;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (j == (bi & 7)) f[j] -= excess;
    }
}

// ---------------------------------------------------------------------------
// Range encoder state and one symbol step (per thread).
// ---------------------------------------------------------------------------
struct EncState {
    uint64_t lower, range;
    int64_t inverted;
    uint32_t first;
    int64_t pos;
};

__device__ __forceinline__ void enc_init(EncState &e) {
    e.lower = 0; e.range = ~0ull; e.inverted = 0; e.first = 0; e.pos = 0;
}

// returns 1 when `cap` words would be exceeded
__device__ __forceinline__ int enc_symbol(EncState &e, uint32_t cum, uint32_t freq, uint32_t *out, int64_t cap) {
    const uint64_t scale = e.range >> SC_PRECISION;
    const uint64_t new_range = scale * (uint64_t)freq;
    const uint64_t new_lower = e.lower + scale * (uint64_t)cum;
    if (e.inverted > 0 && new_lower + new_range > new_lower) {
        uint32_t emit_first, emit_rest;
        if (new_lower < e.lower) { emit_first = e.first + 1u; emit_rest = 0u; }
        else { emit_first = e.first; emit_rest = 0xFFFFFFFFu; }
        if (e.pos + e.inverted > cap) return 1;
        out[e.pos++] = emit_first;
        for (int64_t i = 0; i < e.inverted - 1; ++i) out[e.pos++] = emit_rest;
        e.inverted = 0;
    }
    e.lower = new_lower;
    e.range = new_range;
    if (e.range < (1ull << 32)) {
        e.range <<= 32;
        const uint32_t lower_word = (uint32_t)(e.lower >> 32);
        e.lower <<= 32;
        if (e.inverted > 0) {
            e.inverted += 1;
        } else if (e.lower + e.range > e.lower) {
            if (e.pos >= cap) return 1;
            out[e.pos++] = lower_word;
        } else {
            e.inverted = 1;
            e.first = lower_word;
        }
    }
    return 0;
}

__device__ __forceinline__ int enc_seal(EncState &e, uint32_t *out, int64_t cap) {
    if (e.range != ~0ull) {
        const uint64_t point = e.lower + 0xFFFFFFFFull;
        if (e.inverted > 0) {
            uint32_t emit_first, emit_rest;
            if (point < e.lower) { emit_first = e.first + 1u; emit_rest = 0u; }
            else { emit_first = e.first; emit_rest = 0xFFFFFFFFu; }
            if (e.pos + e.inverted > cap) return 1;
            out[e.pos++] = emit_first;
            for (int64_t i = 0; i < e.inverted - 1; ++i) out[e.pos++] = emit_rest;
        }
        const uint64_t point_word = point >> 32;
        if (e.pos >= cap) return 1;
        out[e.pos++] = (uint32_t)point_word;
        if (((e.lower + e.range) >> 32) == point_word) {
            if (e.pos >= cap) return 1;
            out[e.pos++] = 0u;
        }
    }
    return 0;
}

// ---------------------------------------------------------------------------
// Range decoder state.
// ---------------------------------------------------------------------------
struct DecState {
    uint64_t lower, range, point;
    int64_t read_pos, end_pos;   // absolute word indices
};

__device__ __forceinline__ void dec_init(DecState &d, const uint32_t *words, int64_t begin, int64_t end) {
    const int64_t n = end - begin;
    uint64_t point = 0;
    const int64_t take = n < 2 ? n : 2;
    for (int64_t i = 0; i < take; ++i) point = (point << 32) | words[begin + i];
    if (n == 1) point <<= 32;
    d.point = point;
    d.lower = 0;
    d.range = ~0ull;
    d.read_pos = begin + take;
    d.end_pos = end;
}

}  // namespace sc
