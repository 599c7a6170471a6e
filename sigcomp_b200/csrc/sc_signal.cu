// Signal transform on the device, on either side of the neural codec.
//
// split (sigcomp/main.py:504-521, after the optional lossy step of main.py:158-171):
//   int16 read -> first sample, zig-zag deltas (main.py:129-155) -> deltas < 256 as
//   uint8 tokens (the codec's input), the others as (value - 256, position delta).
// reassemble (main.py:524-546, with the large values and positions already decoded):
//   tokens + large values/positions -> zig-zag deltas -> int16 read (-> lossy decode).
//
// One CTA per read walks the read in blocks of 4096 deltas; block-wide scans with a
// running prefix give every token and large value its output index.  Reads are
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
constexpr int SPT = 16;              // deltas per thread per block
constexpr int SBLK = ST * SPT;       // deltas per block

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

struct RunningPrefix {
    SplitAgg total;
    __device__ SplitAgg operator()(const SplitAgg &block_total)
    {
        const SplitAgg old = total;
        total = SplitOp()(total, block_total);
        return old;
    }
};

// per read: number of small and large deltas
__global__ void __launch_bounds__(ST) k_split_count(const int16_t *__restrict__ x, const int64_t *__restrict__ off,
                                                     int lsb, int64_t *__restrict__ n_small,
                                                     int64_t *__restrict__ n_large)
{
    using Reduce = cub::BlockReduce<int, ST>;
    __shared__ typename Reduce::TempStorage tmp;
    const int64_t r = blockIdx.x;
    const int64_t o = off[r], nz = off[r + 1] - o - 1;
    int64_t large = 0;
    for (int64_t z0 = 0; z0 < nz; z0 += SBLK) {
        int cnt = 0;
        const int64_t zb = z0 + (int64_t)threadIdx.x * SPT;
        if (zb < nz) {
            int32_t prev = lossy_in(x[o + zb], lsb);
            const int m = (int)cmin64(SPT, nz - zb);
            for (int k = 0; k < m; ++k) {
                const int32_t cur = lossy_in(x[o + zb + k + 1], lsb);
                cnt += zigzag16(cur, prev) >= 256u;
                prev = cur;
            }
        }
        const int tot = Reduce(tmp).Sum(cnt);
        __syncthreads();
        large += tot;
    }
    if (threadIdx.x == 0) {
        n_large[r] = large;
        n_small[r] = (nz > 0 ? nz : 0) - large;
    }
}

// per read: first sample, tokens, large values and position deltas at their output offsets
__global__ void __launch_bounds__(ST) k_split_write(const int16_t *__restrict__ x, const int64_t *__restrict__ off,
                                                     int lsb, const int64_t *__restrict__ small_off,
                                                     const int64_t *__restrict__ large_off, int16_t *__restrict__ sig0,
                                                     uint8_t *__restrict__ small, uint16_t *__restrict__ large,
                                                     uint32_t *__restrict__ large_pos)
{
    using Scan = cub::BlockScan<SplitAgg, ST>;
    __shared__ typename Scan::TempStorage tmp;
    const int64_t r = blockIdx.x;
    const int64_t o = off[r], nz = off[r + 1] - o - 1;
    if (threadIdx.x == 0) sig0[r] = (int16_t)lossy_in(x[o], lsb);
    const int64_t sbase = small_off[r], lbase = large_off[r];
    RunningPrefix run{SplitAgg{0, 0, -1}};
    for (int64_t z0 = 0; z0 < nz; z0 += SBLK) {
        const int64_t zb = z0 + (int64_t)threadIdx.x * SPT;
        const int m = zb < nz ? (int)cmin64(SPT, nz - zb) : 0;
        uint32_t zz[SPT];
        SplitAgg mine{0, 0, -1};
        if (m > 0) {
            int32_t prev = lossy_in(x[o + zb], lsb);
#pragma unroll
            for (int k = 0; k < SPT; ++k) {
                if (k < m) {
                    const int32_t cur = lossy_in(x[o + zb + k + 1], lsb);
                    zz[k] = zigzag16(cur, prev);
                    prev = cur;
                    if (zz[k] >= 256u) {
                        mine.large += 1;
                        mine.last = zb + k;
                    } else {
                        mine.small += 1;
                    }
                }
            }
        }
        SplitAgg before;
        Scan(tmp).ExclusiveScan(mine, before, SplitOp(), run);
        __syncthreads();
        int64_t si = sbase + before.small, li = lbase + before.large, last = before.last;
#pragma unroll
        for (int k = 0; k < SPT; ++k) {
            if (k < m) {
                const int64_t z = zb + k;
                if (zz[k] >= 256u) {
                    large[li] = (uint16_t)(zz[k] - 256u);
                    large_pos[li] = (uint32_t)(last >= 0 ? z - last - 1 : z);
                    last = z;
                    ++li;
                } else {
                    small[si++] = (uint8_t)zz[k];
                }
            }
        }
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
        __syncthreads();
        int32_t dv[SPT];
        int32_t dsum = 0;
        int64_t si = smalls_before + sm_before;
#pragma unroll
        for (int k = 0; k < SPT; ++k) {
            dv[k] = 0;
            if (k < m) {
                uint32_t v;
                if ((lm >> k) & 1u) {
                    v = zl[(int)(zb + k - z0)];
                } else {
                    v = si < ns ? small[s0 + si] : 0u;   // short token stream: flagged below
                    ++si;
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
                out[o + zb + k + 1] = (int16_t)(lsb ? (int32_t)sample << lsb : sample);
            }
        }
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
    int64_t *cnt = (int64_t *)m->ws_misc.get(sizeof(int64_t) * 2 * (n_reads + 1), s);
    int64_t *ns = cnt, *nl = cnt + n_reads + 1;
    k_split_count<<<(unsigned)n_reads, ST, 0, s>>>(samples, off_d, lsb, ns, nl);
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
    k_split_write<<<(unsigned)n_reads, ST, 0, s>>>(samples, off_d, lsb, small_off, large_off, sig0, small, large,
                                                   large_pos);
    SC_LAUNCH_CHECK();
    count_launch();
    return 0;
}

int reassemble_signal_device(sc_model *m, const int16_t *sig0, const int64_t *off_d, int64_t n_reads, int lsb,
                             const uint8_t *small, const int64_t *small_off, const uint16_t *large,
                             const uint32_t *large_pos, const int64_t *large_off, int16_t *samples,
                             cudaStream_t s)
{
    if (n_reads <= 0) return 0;
    int *bad = (int *)m->ws_err.get(64, s);
    SC_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), s));
    k_reassemble<<<(unsigned)n_reads, ST, 0, s>>>(sig0, off_d, lsb, small, small_off, large, large_pos, large_off,
                                                  samples, bad);
    SC_LAUNCH_CHECK();
    count_launch();
    int h_bad = 0;
    SC_CUDA(cudaMemcpyAsync(&h_bad, bad, sizeof(int), cudaMemcpyDeviceToHost, s));
    SC_CUDA(cudaStreamSynchronize(s));
    return h_bad ? 1 : 0;
}

}  // namespace sc
