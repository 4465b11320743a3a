// fft_exact.cuh -- the reference radix-2 FFT (fft.cpp:36-99) on the GPU with the
// reference build's rounding, so that spectra and inverse transforms are bit-identical
// to the CPU runtime's.
//
// The reference FFT is iterative Cooley-Tukey on a bit-reversed copy.  What fixes its
// rounding is (a) the order of stages and butterflies, which is a tree and therefore
// independent of how the butterflies of one stage are scheduled, (b) the twiddle of
// butterfly k at stage len, which is the k-th value of the recurrence w *= wlen
// (host-built table, nfx_lut.h), and (c) the expression shape of each complex product
// in the reference's GCC -O3 -mfma build:
//   forward butterfly  v = a*w:  re = ar*wr - ai*wi,         im = ai*wr + ar*wi
//   inverse butterfly  v = a*w:  re = fma(ar, wr, -(ai*wi)), im = fma(ar, wi, ai*wr)
// All arithmetic below uses the _rn intrinsics, which nvcc never contracts.
#pragma once

#include <cuda_runtime.h>

namespace nfx {

__device__ __forceinline__ int bit_reverse(int i, int log2n) {
    return log2n == 0 ? 0 : static_cast<int>(__brev(static_cast<unsigned>(i)) >> (32 - log2n));
}

// In-place transform of one row of n complex values in shared memory, already in
// bit-reversed order, by one warp.  `tw` is the stage-concatenated twiddle table
// (n - 1 entries).  INV selects the inverse butterflies (the caller applies the 1/n).
template <bool INV>
__device__ __forceinline__ void warp_fft_row(float2* a, int n, const float2* __restrict__ tw,
                                             int lane) {
    for (int half = 1; half < n; half <<= 1) {
        const float2* t = tw + (half - 1);
        for (int b = lane; b < n / 2; b += 32) {
            const int k = b & (half - 1);
            const int i0 = (b - k) * 2 + k;
            const int i1 = i0 + half;
            const float2 w = __ldg(t + k);
            const float2 u = a[i0];
            const float2 x = a[i1];
            float2 v;
            if (INV) {
                v.x = __fmaf_rn(x.x, w.x, -__fmul_rn(x.y, w.y));
                v.y = __fmaf_rn(x.x, w.y, __fmul_rn(x.y, w.x));
            } else {
                v.x = __fsub_rn(__fmul_rn(x.x, w.x), __fmul_rn(x.y, w.y));
                v.y = __fadd_rn(__fmul_rn(x.y, w.x), __fmul_rn(x.x, w.y));
            }
            a[i0] = make_float2(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y));
            a[i1] = make_float2(__fsub_rn(u.x, v.x), __fsub_rn(u.y, v.y));
        }
        __syncwarp();
    }
}

// The same transform when only the first `need` outputs are read.  A later stage reads,
// of each group of 2*half entries, only the first min(2*half, need) (by induction from
// the last stage), so a butterfly output is computed only when its position in its
// group is below that bound; every output computed is the one warp_fft_row computes.
template <bool INV>
__device__ __forceinline__ void warp_fft_row_first(float2* a, int n, const float2* __restrict__ tw,
                                                   int lane, int need) {
    for (int half = 1; half < n; half <<= 1) {
        const float2* t = tw + (half - 1);
        const int nd = need < 2 * half ? need : 2 * half;
        const int kk = nd < half ? nd : half;        // butterflies per group
        // lanes over (group, k) with k padded to a power of two (at most half)
        const int lg = kk <= 1 ? 0 : 32 - __clz(kk - 1);
        const int groups = n / (2 * half);
        for (int idx = lane; idx < (groups << lg); idx += 32) {
            const int k = idx & ((1 << lg) - 1);
            if (k >= kk) continue;
            const int i0 = ((idx >> lg) * 2 * half) + k;
            const int i1 = i0 + half;
            const float2 w = __ldg(t + k);
            const float2 u = a[i0];
            const float2 x = a[i1];
            float2 v;
            if (INV) {
                v.x = __fmaf_rn(x.x, w.x, -__fmul_rn(x.y, w.y));
                v.y = __fmaf_rn(x.x, w.y, __fmul_rn(x.y, w.x));
            } else {
                v.x = __fsub_rn(__fmul_rn(x.x, w.x), __fmul_rn(x.y, w.y));
                v.y = __fadd_rn(__fmul_rn(x.y, w.x), __fmul_rn(x.x, w.y));
            }
            a[i0] = make_float2(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y));
            if (k + half < nd) a[i1] = make_float2(__fsub_rn(u.x, v.x), __fsub_rn(u.y, v.y));
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// n = 1024 in registers: the butterflies and twiddles of warp_fft_row (so the same
// results, bit for bit), with the row held as 32 complex values per lane.  Stages with
// half <= 16 pair entries of one 32-entry block (lane l holds entries 32 l + j), stages
// with half >= 32 pair entries 32 apart (lane l holds entries 32 j + l); the row passes
// through shared memory at the start, once between the two layouts and at the end,
// instead of once per stage.  The shared-memory row is kept in the swizzled order
// fft1024_pos(i) = i ^ ((i >> 5) & 31), under which both layouts are read and written
// without bank conflicts; callers index the row through fft1024_pos.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int fft1024_pos(int i) { return i ^ ((i >> 5) & 31); }

template <bool INV>
__device__ __forceinline__ void fft_butterfly(float2& u, float2& x, float2 w) {
    float2 v;
    if (INV) {
        v.x = __fmaf_rn(x.x, w.x, -__fmul_rn(x.y, w.y));
        v.y = __fmaf_rn(x.x, w.y, __fmul_rn(x.y, w.x));
    } else {
        v.x = __fsub_rn(__fmul_rn(x.x, w.x), __fmul_rn(x.y, w.y));
        v.y = __fadd_rn(__fmul_rn(x.y, w.x), __fmul_rn(x.x, w.y));
    }
    const float2 a0 = make_float2(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y));
    x = make_float2(__fsub_rn(u.x, v.x), __fsub_rn(u.y, v.y));
    u = a0;
}

template <bool INV>
__device__ __forceinline__ void warp_fft1024(float2* a, const float2* __restrict__ tw, int lane) {
    float2 v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = a[fft1024_pos(32 * lane + j)];
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int half = 1 << s;
#pragma unroll
        for (int j0 = 0; j0 < 32; ++j0)
            if ((j0 & half) == 0) fft_butterfly<INV>(v[j0], v[j0 + half], __ldg(tw + (half - 1) + (j0 & (half - 1))));
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) a[fft1024_pos(32 * lane + j)] = v[j];
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = a[fft1024_pos(32 * j + lane)];
#pragma unroll
    for (int s = 0; s < 5; ++s) {
        const int h = 1 << s, half = 32 << s;
#pragma unroll
        for (int j0 = 0; j0 < 32; ++j0)
            if ((j0 & h) == 0)
                fft_butterfly<INV>(v[j0], v[j0 + h], __ldg(tw + (half - 1) + 32 * (j0 & (h - 1)) + lane));
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) a[fft1024_pos(32 * j + lane)] = v[j];
    __syncwarp();
}

// ---------------------------------------------------------------------------
// n = 128 in registers, four complex values per lane: the butterflies and twiddles of
// warp_fft_row (bit for bit).  In: v[m] = a[4 lane + m] of the bit-reversed row, so the
// stages with half <= 2 pair a lane's own entries and those with half = 4, 8, 16 pair
// entry m of lanes l and l ^ (half / 4) (exchanged by shuffles; both lanes evaluate the
// butterfly and keep their output).  One pass through `scratch` (128 float2, the warp's
// own; swizzled by fft128_pos so that neither layout has bank conflicts) turns the row
// into v[j] = a[lane + 32 j] for the stages with half = 32 and 64.  Out: v[j] = the
// transform's entry lane + 32 j.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int fft128_pos(int i) { return i ^ ((i >> 4) & 3); }

// entry of the natural-order row that lands at bit-reversed position 4 lane + m
__device__ __forceinline__ int fft128_src(int lane, int m) {
    return static_cast<int>(__brev(static_cast<unsigned>(lane)) >> 27) + 32 * (((m & 1) << 1) | (m >> 1));
}

template <bool INV>
__device__ __forceinline__ void warp_fft128_regs(float2 (&v)[4], float2* scratch, const float2* __restrict__ tw,
                                                 int lane) {
    const float2 w0 = __ldg(tw);
    fft_butterfly<INV>(v[0], v[1], w0);
    fft_butterfly<INV>(v[2], v[3], w0);
    fft_butterfly<INV>(v[0], v[2], __ldg(tw + 1));
    fft_butterfly<INV>(v[1], v[3], __ldg(tw + 2));
#pragma unroll
    for (int s = 1; s <= 4; s <<= 1) {
        const int half = 4 * s;
        const bool hi = (lane & s) != 0;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const float2 w = __ldg(tw + (half - 1) + ((4 * lane + m) & (half - 1)));
            const float2 p = make_float2(__shfl_xor_sync(0xffffffffu, v[m].x, s),
                                         __shfl_xor_sync(0xffffffffu, v[m].y, s));
            float2 u = hi ? p : v[m];
            float2 x = hi ? v[m] : p;
            fft_butterfly<INV>(u, x, w);
            v[m] = hi ? x : u;
        }
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) scratch[fft128_pos(4 * lane + m)] = v[m];
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = scratch[fft128_pos(lane + 32 * j)];
    __syncwarp();
    const float2 w32 = __ldg(tw + 31 + lane);
    fft_butterfly<INV>(v[0], v[1], w32);
    fft_butterfly<INV>(v[2], v[3], w32);
    fft_butterfly<INV>(v[0], v[2], __ldg(tw + 63 + lane));
    fft_butterfly<INV>(v[1], v[3], __ldg(tw + 95 + lane));
}

// n = 64 in registers, two complex values per lane, in the manner of warp_fft128_regs:
// in v[m] = a[2 lane + m] of the bit-reversed row (half = 1 within the lane, half = 2 ..
// 16 by shuffles with lane l ^ (half / 2)), one swizzled pass through `scratch` (64
// float2), half = 32 on v[j] = a[lane + 32 j].  Out: v[j] = the entry lane + 32 j.
__device__ __forceinline__ int fft64_pos(int i) { return i ^ ((i >> 4) & 1); }

// entry of the natural-order row that lands at bit-reversed position 2 lane + m
__device__ __forceinline__ int fft64_src(int lane, int m) {
    return static_cast<int>(__brev(static_cast<unsigned>(lane)) >> 27) + 32 * m;
}

template <bool INV>
__device__ __forceinline__ void warp_fft64_regs(float2 (&v)[2], float2* scratch, const float2* __restrict__ tw,
                                                int lane) {
    fft_butterfly<INV>(v[0], v[1], __ldg(tw));
#pragma unroll
    for (int s = 1; s <= 8; s <<= 1) {
        const int half = 2 * s;
        const bool hi = (lane & s) != 0;
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const float2 w = __ldg(tw + (half - 1) + ((2 * lane + m) & (half - 1)));
            const float2 p = make_float2(__shfl_xor_sync(0xffffffffu, v[m].x, s),
                                         __shfl_xor_sync(0xffffffffu, v[m].y, s));
            float2 u = hi ? p : v[m];
            float2 x = hi ? v[m] : p;
            fft_butterfly<INV>(u, x, w);
            v[m] = hi ? x : u;
        }
    }
#pragma unroll
    for (int m = 0; m < 2; ++m) scratch[fft64_pos(2 * lane + m)] = v[m];
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 2; ++j) v[j] = scratch[fft64_pos(lane + 32 * j)];
    __syncwarp();
    fft_butterfly<INV>(v[0], v[1], __ldg(tw + 31 + lane));
}

}  // namespace nfx
