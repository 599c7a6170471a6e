// Signal transform on the device, on either side of the neural codec.
//
// split (sigcomp/main.py:504-521, after the optional lossy step of main.py:158-171):
//   int16 read -> first sample, zig-zag deltas (main.py:129-155) -> deltas < 256 as
//   uint8 tokens (the codec's input), the others as (value - 256, position delta).
// reassemble (main.py:524-546, with the large values and positions already decoded):
//   tokens + large values/positions -> zig-zag deltas -> int16 read (-> lossy decode).
//
// One CTA per read walks the read in tiles of 2048 samples.  Every thread loads eight consecutive
// samples with one 16-byte load (tiles start at a multiple of eight samples, so the loads are
// aligned and a warp reads 512 contiguous bytes), block-wide scans give every token and large value
// its output index, and a tile's tokens are staged in shared memory so that they leave in
// consecutive bytes; reassembly stages a tile's tokens and samples the same way.  Reads are
// independent, so the grid is simply one CTA per read.
#include <algorithm>
#include <vector>
#include <cub/block/block_scan.cuh>
#include <cub/block/block_reduce.cuh>
#include <cub/device/device_scan.cuh>

#include "sc_internal.h"

namespace sc {
namespace {

constexpr int ST = 256;              // threads per CTA
constexpr int VEC = 8;               // samples per thread per tile (one 16-byte load)
constexpr int TILE = ST * VEC;       // samples per tile
constexpr int SPT = 16;              // reassembly: deltas per thread per block
constexpr int SBLK = ST * SPT;       // reassembly: deltas per block

__device__ __forceinline__ int64_t cmin64(int64_t a, int64_t b) { return a < b ? a : b; }

// lossy step applied to every sample before the split (lsb = 0: none)
__device__ __forceinline__ int32_t lossy_in(int16_t x, int lsb)
{
    if (lsb == 0) return x;
    const int32_t v = x, step = 1 << lsb;
    const int32_t rounding = ((v >> (lsb - 1)) & 1) * step;       // _reduce_lsb
    const int16_t reduced = (int16_t)((v & ~(step - 1)) + rounding);
    return (int16_t)((int32_t)reduced >> lsb);                      // _lossy_encode
}

__device__ __forceinline__ uint32_t zigzag16(int32_t cur, int32_t prev)
{
    const int32_t d = (int16_t)(cur - prev);                       // int16 wrap of the difference
    return (uint32_t)((d << 1) ^ (d >> 31)) & 0xFFFFu;
}

// Samples a .. a + 7 (a a multiple of 8) into v: one aligned 16-byte load, or element loads for a
// group that reaches past the end of the sample array (`total` samples).
__device__ __forceinline__ void load8(const int16_t *__restrict__ x, int64_t a, int64_t total, int16_t (&v)[VEC])
{
    if (a + VEC <= total) {
        const uint4 u = *reinterpret_cast<const uint4 *>(x + a);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[2 * k] = (int16_t)(w[k] & 0xFFFFu);
            v[2 * k + 1] = (int16_t)(w[k] >> 16);
        }
    } else {
#pragma unroll
        for (int k = 0; k < VEC; ++k) v[k] = a + k < total ? x[a + k] : (int16_t)0;
    }
}

// Zig-zag deltas of the samples a .. a + 7 of read [o, o + n): delta i - o - 1 pairs sample i with
// sample i - 1; zz[k] is valid when `valid` has bit k (o < a + k < o + n).
__device__ __forceinline__ uint32_t group_deltas(const int16_t *__restrict__ x, int64_t a, int64_t o, int64_t n,
                                                 int64_t total, int lsb, uint32_t (&zz)[VEC])
{
    int16_t v[VEC];
    load8(x, a, total, v);
    int32_t prev = a > o ? lossy_in(x[a - 1], lsb) : 0;
    uint32_t valid = 0;
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        const int64_t i = a + k;
        const int32_t cur = lossy_in(v[k], lsb);
        zz[k] = zigzag16(cur, prev);
        if (i > o && i < o + n) valid |= 1u << k;
        prev = cur;
    }
    return valid;
}

struct SplitAgg {
    int64_t small, large;
    int64_t last;                     // delta index of the last large value so far (-1: none)
};

struct SplitOp {
    __device__ __forceinline__ SplitAgg operator()(const SplitAgg &a, const SplitAgg &b) const
    {
        return SplitAgg{a.small + b.small, a.large + b.large, b.last > a.last ? b.last : a.last};
    }
};

// per read: number of small and large deltas
__global__ void __launch_bounds__(ST) k_split_count(const int16_t *__restrict__ x, const int64_t *__restrict__ off,
                                                     int64_t total, int lsb, int64_t *__restrict__ n_small,
                                                     int64_t *__restrict__ n_large)
{
    using Reduce = cub::BlockReduce<int, ST>;
    __shared__ typename Reduce::TempStorage tmp;
    const int64_t r = blockIdx.x;
    const int64_t o = off[r], n = off[r + 1] - o;
    int64_t large = 0;
    for (int64_t base = o & ~(int64_t)(VEC - 1); base < o + n; base += TILE) {
        const int64_t a = base + (int64_t)threadIdx.x * VEC;
        int cnt = 0;
        if (a < o + n) {
            uint32_t zz[VEC];
            const uint32_t valid = group_deltas(x, a, o, n, total, lsb, zz);
#pragma unroll
            for (int k = 0; k < VEC; ++k) cnt += ((valid >> k) & 1u) && zz[k] >= 256u;
        }
        const int tot = Reduce(tmp).Sum(cnt);
        __syncthreads();
        large += tot;
    }
    if (threadIdx.x == 0) {
        n_large[r] = large;
        n_small[r] = (n > 1 ? n - 1 : 0) - large;
    }
}

// per read: first sample, tokens, large values and position deltas at their output offsets
__global__ void __launch_bounds__(ST) k_split_write(const int16_t *__restrict__ x, const int64_t *__restrict__ off,
                                                     int64_t total, int lsb, const int64_t *__restrict__ small_off,
                                                     const int64_t *__restrict__ large_off, int16_t *__restrict__ sig0,
                                                     uint8_t *__restrict__ small, uint16_t *__restrict__ large,
                                                     uint32_t *__restrict__ large_pos)
{
    using Scan = cub::BlockScan<SplitAgg, ST>;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ uint8_t stok[TILE];         // the tile's tokens, compacted
    const int64_t r = blockIdx.x;
    const int64_t o = off[r], n = off[r + 1] - o;
    if (threadIdx.x == 0) sig0[r] = (int16_t)lossy_in(x[o], lsb);
    const int64_t sbase = small_off[r], lbase = large_off[r];
    SplitAgg run{0, 0, -1};                // totals of the earlier tiles (block-uniform)
    for (int64_t base = o & ~(int64_t)(VEC - 1); base < o + n; base += TILE) {
        const int64_t a = base + (int64_t)threadIdx.x * VEC;
        uint32_t zz[VEC];
        uint32_t valid = 0;
        SplitAgg mine{0, 0, -1};
        if (a < o + n) {
            valid = group_deltas(x, a, o, n, total, lsb, zz);
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                if (!((valid >> k) & 1u)) continue;
                if (zz[k] >= 256u) {
                    mine.large += 1;
                    mine.last = a + k - o - 1;
                } else {
                    mine.small += 1;
                }
            }
        }
        SplitAgg before, agg;
        Scan(tmp).ExclusiveScan(mine, before, SplitAgg{0, 0, -1}, SplitOp(), agg);
        int64_t si = before.small, li = lbase + run.large + before.large;
        int64_t last = before.last >= 0 ? before.last : run.last;
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            if (!((valid >> k) & 1u)) continue;
            const int64_t z = a + k - o - 1;
            if (zz[k] >= 256u) {
                large[li] = (uint16_t)(zz[k] - 256u);
                large_pos[li] = (uint32_t)(last >= 0 ? z - last - 1 : z);
                last = z;
                ++li;
            } else {
                stok[si++] = (uint8_t)zz[k];
            }
        }
        __syncthreads();
        // the tile's tokens leave in consecutive bytes
        uint8_t *dst = small + sbase + run.small;
        for (int64_t i = threadIdx.x; i < agg.small; i += ST) dst[i] = stok[i];
        run = SplitOp()(run, agg);
        __syncthreads();
    }
}

// per read: rebuild the zig-zag deltas from tokens and large values, then the samples
__global__ void __launch_bounds__(ST) k_reassemble(const int16_t *__restrict__ sig0, const int64_t *__restrict__ off,
                                                    int lsb, const uint8_t *__restrict__ small,
                                                    const int64_t *__restrict__ small_off,
                                                    const uint16_t *__restrict__ large,
                                                    const uint32_t *__restrict__ large_pos,
                                                    const int64_t *__restrict__ large_off, int16_t *__restrict__ out,
                                                    int *__restrict__ bad)
{
    using ScanI = cub::BlockScan<int64_t, ST>;
    using ScanS = cub::BlockScan<int32_t, ST>;
    __shared__ union {
        typename ScanI::TempStorage i;
        typename ScanS::TempStorage s;
    } tmp;
    __shared__ int64_t lpos[ST];          // positions of the current batch of large values
    __shared__ uint16_t lval[ST];
    __shared__ uint32_t mark[SBLK / 32];   // large deltas of the current block (bitmap)
    __shared__ uint16_t zl[SBLK];          // their zig-zag values
    __shared__ uint8_t tok[SBLK];          // the block's tokens, loaded in consecutive bytes
    __shared__ int16_t outs[SBLK];         // the block's samples, stored in consecutive elements
    const int64_t r = blockIdx.x;
    const int64_t o = off[r], n = off[r + 1] - o, nz = n - 1;
    const int64_t s0 = small_off[r], ns = small_off[r + 1] - s0;
    const int64_t l0 = large_off[r], nl = large_off[r + 1] - l0;
    if (ns < 0 || nl < 0 || ns + nl != nz) {   // the streams do not describe this read
        if (threadIdx.x == 0) atomicExch(bad, 1);
        return;
    }
    const int32_t first = sig0[r];
    if (threadIdx.x == 0) out[o] = (int16_t)(lsb ? (int32_t)first << lsb : first);
    // large values are placed batch by batch: positions are the running sum of (delta + 1) - 1
    int64_t lb = 0, lcount = 0, lnext = 0;   // batch start, batch size, next to place (block-uniform)
    int64_t carry = -1;                      // position of the last large value of the previous batch
    int64_t smalls_before = 0;               // tokens used by earlier blocks
    int32_t run = (int16_t)first;            // running sample value
    for (int64_t z0 = 0; z0 < nz; z0 += SBLK) {
        const int64_t z1 = cmin64(z0 + SBLK, nz);
        for (int i = threadIdx.x; i < SBLK / 32; i += ST) mark[i] = 0u;
        __syncthreads();
        while (true) {
            if (lnext == lb + lcount) {
                if (lb + lcount >= nl) break;
                lb += lcount;
                lcount = cmin64(ST, nl - lb);
                const int64_t step = threadIdx.x < lcount ? (int64_t)large_pos[l0 + lb + threadIdx.x] + 1 : 0;
                int64_t incl, total;
                ScanI(tmp.i).InclusiveSum(step, incl, total);
                if (threadIdx.x < lcount) {
                    lpos[threadIdx.x] = carry + incl;
                    lval[threadIdx.x] = large[l0 + lb + threadIdx.x];
                }
                carry += total;
                __syncthreads();
            }
            // the unplaced large values of the batch that fall before z1 form a prefix
            const int q = (int)(lnext - lb) + (int)threadIdx.x;
            const bool place = q < lcount && lpos[q] < z1;
            if (place) {
                const int b = (int)(lpos[q] - z0);
                atomicOr(&mark[b >> 5], 1u << (b & 31));
                zl[b] = (uint16_t)(lval[q] + 256u);
            }
            const int placed = __syncthreads_count(place);
            lnext += placed;
            if (lnext < lb + lcount) break;       // the next large value belongs to a later block
        }
        // tokens: each thread owns SPT consecutive deltas of the block
        const int64_t zb = z0 + (int64_t)threadIdx.x * SPT;
        const int m = zb < z1 ? (int)cmin64(SPT, z1 - zb) : 0;
        uint32_t lm = 0;                           // large flags of this thread's deltas
        for (int k = 0; k < m; ++k) {
            const int b = (int)(zb + k - z0);
            lm |= ((mark[b >> 5] >> (b & 31)) & 1u) << k;
        }
        const int32_t nsm = m - __popc(lm);
        int32_t sm_before, sm_total;
        ScanS(tmp.s).ExclusiveSum(nsm, sm_before, sm_total);
        for (int i = threadIdx.x; i < sm_total; i += ST) {
            const int64_t t = smalls_before + i;
            tok[i] = t < ns ? small[s0 + t] : (uint8_t)0;   // short token stream: flagged below
        }
        __syncthreads();
        int32_t dv[SPT];
        int32_t dsum = 0;
        int si = sm_before;
#pragma unroll
        for (int k = 0; k < SPT; ++k) {
            dv[k] = 0;
            if (k < m) {
                uint32_t v;
                if ((lm >> k) & 1u) {
                    v = zl[(int)(zb + k - z0)];
                } else {
                    v = tok[si++];
                }
                dv[k] = (int16_t)(int32_t)((v >> 1) ^ (0u - (v & 1u)));   // zig-zag decode
                dsum += dv[k];
            }
        }
        int32_t before, total;
        ScanS(tmp.s).ExclusiveSum(dsum, before, total);
        __syncthreads();
        int32_t acc = run + before;
#pragma unroll
        for (int k = 0; k < SPT; ++k) {
            if (k < m) {
                acc += dv[k];
                const int16_t sample = (int16_t)acc;
                outs[(int)(zb + k - z0)] = (int16_t)(lsb ? (int32_t)sample << lsb : sample);
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < (int)(z1 - z0); i += ST) out[o + z0 + 1 + i] = outs[i];
        run = (int16_t)(run + total);
        smalls_before += sm_total;
    }
    if (threadIdx.x == 0 && lnext != nl) atomicExch(bad, 1);   // large positions beyond the read
}

}  // namespace

int split_signal_device(sc_model *m, const int16_t *samples, const int64_t *off_d, const int64_t *off_h,
                        int64_t n_reads, int lsb, int16_t *sig0, uint8_t *small, int64_t *small_off,
                        uint16_t *large, uint32_t *large_pos, int64_t *large_off, cudaStream_t s)
{
    if (n_reads <= 0) {
        SC_CUDA(cudaMemsetAsync(small_off, 0, sizeof(int64_t), s));
        SC_CUDA(cudaMemsetAsync(large_off, 0, sizeof(int64_t), s));
        return 0;
    }
    const int64_t total = off_h[n_reads];
    ProfScope ps(m->prof, KK_SPLIT, s, total - off_h[0]);
    int64_t *cnt = (int64_t *)m->ws_misc.get(sizeof(int64_t) * 2 * (n_reads + 1), s);
    int64_t *ns = cnt, *nl = cnt + n_reads + 1;
    k_split_count<<<(unsigned)n_reads, ST, 0, s>>>(samples, off_d, total, lsb, ns, nl);
    SC_LAUNCH_CHECK();
    count_launch();
    // offsets[0] = 0, offsets[r + 1] = inclusive sums of the counts
    SC_CUDA(cudaMemsetAsync(small_off, 0, sizeof(int64_t), s));
    SC_CUDA(cudaMemsetAsync(large_off, 0, sizeof(int64_t), s));
    size_t tb = 0;
    SC_CUDA(cub::DeviceScan::InclusiveSum(nullptr, tb, ns, small_off + 1, (int)n_reads, s));
    void *tmp = m->ws_scan.get(tb, s);
    SC_CUDA(cub::DeviceScan::InclusiveSum(tmp, tb, ns, small_off + 1, (int)n_reads, s));
    SC_CUDA(cub::DeviceScan::InclusiveSum(tmp, tb, nl, large_off + 1, (int)n_reads, s));
    count_launch(2);
    k_split_write<<<(unsigned)n_reads, ST, 0, s>>>(samples, off_d, total, lsb, small_off, large_off, sig0, small,
                                                   large, large_pos);
    SC_LAUNCH_CHECK();
    count_launch();
    return 0;
}

int reassemble_signal_device(sc_model *m, const int16_t *sig0, const int64_t *off_d, const int64_t *off_h,
                             int64_t n_reads, int lsb,
                             const uint8_t *small, const int64_t *small_off, const uint16_t *large,
                             const uint32_t *large_pos, const int64_t *large_off, int16_t *samples,
                             cudaStream_t s)
{
    if (n_reads <= 0) return 0;
    int *bad = (int *)m->ws_err.get(64, s);
    SC_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), s));
    {
        ProfScope ps(m->prof, KK_REASSEMBLE, s, off_h[n_reads] - off_h[0]);
        k_reassemble<<<(unsigned)n_reads, ST, 0, s>>>(sig0, off_d, lsb, small, small_off, large, large_pos, large_off,
                                                      samples, bad);
        SC_LAUNCH_CHECK();
        count_launch();
    }
    int h_bad = 0;
    SC_CUDA(cudaMemcpyAsync(&h_bad, bad, sizeof(int), cudaMemcpyDeviceToHost, s));
    SC_CUDA(cudaStreamSynchronize(s));
    return h_bad ? 1 : 0;
}

}  // namespace sc
