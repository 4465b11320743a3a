// fno3d.cu -- FNO3d executor (sm_100a): the reference FNO3d::Forward
// (cpp/src/fno.cpp:1096-1281) with the reference's rounding, and its E4M3 variant.
//
// Activations are channel-first (b, c, h, w, d) as the reference's h_perm: fp32 on the
// FP32 path, one E4M3 byte per element (the reference encoder, fp8_e4m3.h:106-221) on
// the FP8 path.  One layer is
//
//   fwd3d_a   per (b, c, h) plane: the D-axis rFFT of every (h, w) line and the W-axis
//             transforms of the kept kd columns (fft.cpp:151-176)
//   fwd3d_b   per (b, c): the H-axis transforms of the kept (kw, kd) lines
//             (fft.cpp:177-194) -> truncated spectrum Xs
//   mix3d     per (b, group of output channels): the contraction (fno.cpp:1049-1077),
//             then the H-axis inverse of each kept (kw, kd) line (fft.cpp:196-214)
//   inv3d     per (b, o, h): the W-axis inverse of the kept kd columns and the D-axis
//             Irfft of every (h, w) line (fft.cpp:215-243) -> x1
//   local3d   per point: the local Linear (FP32: the reference dot-product rounding;
//             FP8: exact E4M3 products summed in k order), fake-quant, x1 + x2, the
//             activation, and the next activation (fp32 or E4M3 code)
//
// lift3d and proj3d close the network.  The only approximate operation is CUDA's tanhf
// inside GELU.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "fft_exact.cuh"
#include "fno3d.h"
#include "nfx_internal.h"
#include "numerics.cuh"
#include "sm100.cuh"

namespace nfx {
namespace {

__device__ __forceinline__ float act_f(float z, int act) {
    return act == 1 ? relu_ref(z) : gelu_tanh(z);
}

__device__ __forceinline__ float inv_of(float s) { return s == 0.0f ? 1.0f : __fdiv_rn(1.0f, s); }

// the value of an activation element: fp32, or an E4M3 code times its scale
__device__ __forceinline__ float value_at(const void* h, int64_t i, int fp8, float s) {
    if (fp8) return __fmul_rn(e4m3_decode_ref(static_cast<const uint8_t*>(h)[i]), s);
    return static_cast<const float*>(h)[i];
}

__global__ void __launch_bounds__(256) lift3d_kernel(Fno3dPlan p) {
    const int64_t P = static_cast<int64_t>(p.Hp) * p.Wp * p.Dp;
    const int64_t total = static_cast<int64_t>(p.B) * p.C * P;
    const int nu = linear_unfused_len(p.in_ch);
    const float inv = inv_of(p.s_lift);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t pt = t % P;
        const int64_t bc = t / P;
        const int c = static_cast<int>(bc % p.C);
        const int64_t b = bc / p.C;
        const int dd = static_cast<int>(pt % p.Dp);
        const int ww = static_cast<int>((pt / p.Dp) % p.Wp);
        const int hh = static_cast<int>(pt / (static_cast<int64_t>(p.Dp) * p.Wp));
        float v = 0.0f;
        if (hh < p.H && ww < p.W && dd < p.D) {
            const float* xr = p.x + (((b * p.H + hh) * p.W + ww) * p.D + dd) * p.in_ch;
            v = __ldg(p.lift_b + c);
            for (int k = 0; k < p.in_ch; ++k)
                v = linear_step(v, __ldg(xr + k), __ldg(p.lift_w + c * p.in_ch + k), k >= nu);
        }
        if (p.fp8) static_cast<uint8_t*>(p.h[0])[t] = static_cast<uint8_t>(e4m3_code(v, inv));
        else static_cast<float*>(p.h[0])[t] = v;
    }
}

// grid (Hp, C, B); smem rowbuf [8][Dp] float2, colbuf [MD][Wp] float2 (bit-reversed in w)
__global__ void __launch_bounds__(256) fwd3d_a_kernel(Fno3dPlan p, const void* hin, float s_in) {
    extern __shared__ float2 sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hh = blockIdx.x, c = blockIdx.y, b = blockIdx.z;
    const int lgD = 31 - __clz(p.Dp), lgW = 31 - __clz(p.Wp);
    float2* row = sm + warp * p.Dp;
    float2* col = sm + 8 * p.Dp;
    const int64_t base = ((static_cast<int64_t>(b) * p.C + c) * p.Hp + hh) * p.Wp * p.Dp;
    for (int w = warp; w < p.Wp; w += 8) {
        for (int d = lane; d < p.Dp; d += 32)
            row[bit_reverse(d, lgD)] = make_float2(value_at(hin, base + static_cast<int64_t>(w) * p.Dp + d, p.fp8, s_in), 0.0f);
        __syncwarp();
        warp_fft_row<false>(row, p.Dp, p.tw[4], lane);
        const int wr = bit_reverse(w, lgW);
        for (int kd = lane; kd < p.MD; kd += 32) col[kd * p.Wp + wr] = row[kd];
        __syncwarp();
    }
    __syncthreads();
    float2* A = p.A + ((static_cast<int64_t>(b) * p.C + c) * p.Hp + hh) * p.MW * p.MD;
    for (int kd = warp; kd < p.MD; kd += 8) {
        warp_fft_row<false>(col + kd * p.Wp, p.Wp, p.tw[2], lane);
        for (int kw = lane; kw < p.MW; kw += 32) A[kw * p.MD + kd] = col[kd * p.Wp + kw];
    }
}

// grid (C, B); smem [8][Hp] float2
__global__ void __launch_bounds__(256) fwd3d_b_kernel(Fno3dPlan p) {
    extern __shared__ float2 sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x, b = blockIdx.y;
    const int lgH = 31 - __clz(p.Hp);
    const int KK = p.MW * p.MD;
    float2* line = sm + warp * p.Hp;
    const float2* A = p.A + (static_cast<int64_t>(b) * p.C + c) * p.Hp * KK;
    float2* X = p.Xs + (static_cast<int64_t>(b) * p.C + c) * p.MH * KK;
    for (int q = warp; q < KK; q += 8) {
        for (int h = lane; h < p.Hp; h += 32) line[bit_reverse(h, lgH)] = A[static_cast<int64_t>(h) * KK + q];
        __syncwarp();
        warp_fft_row<false>(line, p.Hp, p.tw[0], lane);
        for (int kh = lane; kh < p.MH; kh += 32) X[kh * KK + q] = line[kh];
        __syncwarp();
    }
}

// grid (C / G, B); smem sY [G][M] float2, lines [8][Hp] float2
__global__ void __launch_bounds__(256) mix3d_kernel(Fno3dPlan p, const float* __restrict__ wr,
                                                    const float* __restrict__ wi, int G) {
    extern __shared__ float2 sm[];
    const int KK = p.MW * p.MD, M = p.MH * KK, C = p.C;
    float2* sY = sm;
    float2* lines = sm + G * M;
    const int b = blockIdx.y, o0 = blockIdx.x * G;
    for (int t = threadIdx.x; t < G * M; t += blockDim.x) {
        const int r = t / M, md = t - (t / M) * M;
        const int o = o0 + r;
        float sr = 0.0f, si = 0.0f;
        const float2* xb = p.Xs + static_cast<int64_t>(b) * C * M + md;
        for (int c = 0; c < C; ++c) {
            const float2 hv = xb[static_cast<int64_t>(c) * M];
            const int64_t k = (static_cast<int64_t>(c) * C + o) * M + md;
            const float a = __ldg(wr + k), bi = __ldg(wi + k);
            sr = __fadd_rn(sr, __fmaf_rn(hv.x, a, -__fmul_rn(hv.y, bi)));
            si = __fadd_rn(si, __fmaf_rn(hv.x, bi, __fmul_rn(hv.y, a)));
        }
        sY[t] = make_float2(sr, si);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lgH = 31 - __clz(p.Hp);
    const float invH = __fdiv_rn(1.0f, static_cast<float>(p.Hp));
    float2* line = lines + warp * p.Hp;
    for (int q = warp; q < G * KK; q += 8) {
        const int r = q / KK, kk = q - (q / KK) * KK;
        for (int h = lane; h < p.Hp; h += 32)
            line[bit_reverse(h, lgH)] = h < p.MH ? sY[r * M + h * KK + kk] : make_float2(0.0f, 0.0f);
        __syncwarp();
        warp_fft_row<true>(line, p.Hp, p.tw[1], lane);
        float2* dst = p.colinv + (static_cast<int64_t>(b) * C + o0 + r) * p.Hp * KK + kk;
        for (int h = lane; h < p.Hp; h += 32) {
            const float2 v = line[h];
            dst[static_cast<int64_t>(h) * KK] = make_float2(__fmul_rn(v.x, invH), __fmul_rn(v.y, invH));
        }
        __syncwarp();
    }
}

// grid (Hp, C, B); smem tmp [MD][Wp] float2, lines [8][max(Wp, Dp)] float2
__global__ void __launch_bounds__(256) inv3d_kernel(Fno3dPlan p) {
    extern __shared__ float2 sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hh = blockIdx.x, o = blockIdx.y, b = blockIdx.z;
    const int KK = p.MW * p.MD;
    const int lgW = 31 - __clz(p.Wp), lgD = 31 - __clz(p.Dp);
    const int LN = p.Wp > p.Dp ? p.Wp : p.Dp;
    float2* tmp = sm;
    float2* line = sm + p.MD * p.Wp + warp * LN;
    const float2* ci = p.colinv + ((static_cast<int64_t>(b) * p.C + o) * p.Hp + hh) * KK;
    const float invW = __fdiv_rn(1.0f, static_cast<float>(p.Wp));
    for (int kd = warp; kd < p.MD; kd += 8) {
        for (int w = lane; w < p.Wp; w += 32)
            line[bit_reverse(w, lgW)] = w < p.MW ? ci[w * p.MD + kd] : make_float2(0.0f, 0.0f);
        __syncwarp();
        warp_fft_row<true>(line, p.Wp, p.tw[3], lane);
        for (int w = lane; w < p.Wp; w += 32) {
            const float2 v = line[w];
            tmp[kd * p.Wp + w] = make_float2(__fmul_rn(v.x, invW), __fmul_rn(v.y, invW));
        }
        __syncwarp();
    }
    __syncthreads();
    const int half = p.Dp / 2 + 1;
    const float invD = __fdiv_rn(1.0f, static_cast<float>(p.Dp));
    float* x1 = p.x1 + ((static_cast<int64_t>(b) * p.C + o) * p.Hp + hh) * p.Wp * p.Dp;
    for (int w = warp; w < p.Wp; w += 8) {
        for (int j = lane; j < p.Dp; j += 32) {
            float2 v;
            if (j < half) {
                v = j < p.MD ? tmp[j * p.Wp + w] : make_float2(0.0f, 0.0f);
            } else {
                const int i = p.Dp - j;
                const float2 u = i < p.MD ? tmp[i * p.Wp + w] : make_float2(0.0f, 0.0f);
                v = make_float2(u.x, -u.y);
            }
            line[bit_reverse(j, lgD)] = v;
        }
        __syncwarp();
        warp_fft_row<true>(line, p.Dp, p.tw[5], lane);
        for (int d = lane; d < p.Dp; d += 32) x1[static_cast<int64_t>(w) * p.Dp + d] = __fmul_rn(line[d].x, invD);
        __syncwarp();
    }
}

// local layer + epilogue, one point per thread; smem weights [C][C]
template <int C>
__global__ void __launch_bounds__(128) local3d_kernel(Fno3dPlan p, Fno3dLayer L, const void* hin, void* hout) {
    __shared__ float4 sW4[C * C / 4];  // transposed [k][o]: 16-byte broadcast loads over o
    __shared__ float sB[C];
    float* sW = reinterpret_cast<float*>(sW4);
    const float* wsrc = p.fp8 ? L.loc_q : L.loc_w;
    for (int i = threadIdx.x; i < C * C; i += blockDim.x) sW[(i % C) * C + i / C] = wsrc[i];
    for (int i = threadIdx.x; i < C; i += blockDim.x) sB[i] = L.loc_b[i];
    __syncthreads();
    const int64_t P = static_cast<int64_t>(p.Hp) * p.Wp * p.Dp;
    const int64_t total = static_cast<int64_t>(p.B) * P;
    constexpr int nu = linear_unfused_len(C);
    const float sc = __fmul_rn(L.s_in, L.s_w);
    const float inv_out = inv_of(L.s_out);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = t / P, pt = t - (t / P) * P;
        const int64_t base = b * C * P + pt;
        float acc[C];
        if (p.fp8) {
#pragma unroll
            for (int o = 0; o < C; ++o) acc[o] = 0.0f;
            for (int k = 0; k < C; ++k) {
                const float a = e4m3_decode_ref(static_cast<const uint8_t*>(hin)[base + k * P]);
#pragma unroll
                for (int o4 = 0; o4 < C / 4; ++o4) {
                    const float4 w = sW4[k * (C / 4) + o4];
                    acc[4 * o4 + 0] = __fadd_rn(acc[4 * o4 + 0], __fmul_rn(a, w.x));
                    acc[4 * o4 + 1] = __fadd_rn(acc[4 * o4 + 1], __fmul_rn(a, w.y));
                    acc[4 * o4 + 2] = __fadd_rn(acc[4 * o4 + 2], __fmul_rn(a, w.z));
                    acc[4 * o4 + 3] = __fadd_rn(acc[4 * o4 + 3], __fmul_rn(a, w.w));
                }
            }
        } else {
#pragma unroll
            for (int o = 0; o < C; ++o) acc[o] = sB[o];
            for (int k = 0; k < C; ++k) {
                const float a = static_cast<const float*>(hin)[base + k * P];
                const bool fused = k >= nu;
#pragma unroll
                for (int o4 = 0; o4 < C / 4; ++o4) {
                    const float4 w = sW4[k * (C / 4) + o4];
                    acc[4 * o4 + 0] = linear_step(acc[4 * o4 + 0], a, w.x, fused);
                    acc[4 * o4 + 1] = linear_step(acc[4 * o4 + 1], a, w.y, fused);
                    acc[4 * o4 + 2] = linear_step(acc[4 * o4 + 2], a, w.z, fused);
                    acc[4 * o4 + 3] = linear_step(acc[4 * o4 + 3], a, w.w, fused);
                }
            }
        }
#pragma unroll
        for (int o = 0; o < C; ++o) {
            float x2 = acc[o];
            if (p.fp8) x2 = fp8_fake_quant(__fadd_rn(__fmul_rn(x2, sc), sB[o]), L.s_out, inv_out);
            const float z = act_f(__fadd_rn(p.x1[base + o * P], x2), p.act);
            if (p.fp8) static_cast<uint8_t*>(hout)[base + o * P] = static_cast<uint8_t>(e4m3_code(z, inv_out));
            else static_cast<float*>(hout)[base + o * P] = z;
        }
    }
}

// ---------------------------------------------------------------------------
// local3d_tc: the FP8 local layer on tensor cores (C = 32 or 64, tiles of 128 points
// of one sample).  The layer input codes are channel-first (b, c, point), so a tile is
// the MMA's A operand in MN-major layout: two TMA boxes of [C channels][64 points], one
// per 64-point M atom (64-byte swizzle).  The weights are the E4M3 codes of the decoded
// weights, a K-major [C out][C in] tile.  D = A W^T by tcgen05.mma.kind::f8f6f4 (E4M3 x
// E4M3, fp32 accumulation) into one of four TMEM stages; the products are exact, the
// tensor core's summation order is its own, so D may differ from the CUDA-core
// kernel's k-order sum in the last bits (within the FP8 path's 1e-3 tolerance).
//   warp 0      TMA producer (ring of A tiles)
//   warp 1      MMA issuer
//   warps 2-17  epilogue: four groups of four warps (one per TMEM lane quadrant) take
//               turns over the tiles; per element dequantise + bias, E4M3 fake-quant,
//               x1 + x2, the activation, the output code (as local3d_kernel).
// ---------------------------------------------------------------------------
template <int C>
struct L3Cfg {
    static constexpr int kGroups = 4;
    static constexpr int kEpiWarps = 4 * kGroups;
    static constexpr int kThreads = 32 * (2 + kEpiWarps);
    static constexpr int kStages = 6;
    static constexpr int kABytes = 128 * C;             // two [C][64] boxes
    static constexpr int kAccStages = kGroups;
    static constexpr int kTmemCols = kAccStages * C <= 128 ? 128 : 256;
    static constexpr int kOffA = 0;
    static constexpr int kOffW = kOffA + kStages * kABytes;
    static constexpr int kOffBias = kOffW + ((C * C + 1023) / 1024) * 1024;
    static constexpr int kOffBars = kOffBias + C * 4;
    static constexpr int kNumBars = 2 * kStages + 2 * kAccStages;
    static constexpr int kSmemBytes = kOffBars + 8 * kNumBars + 16 + 1024;
};

template <int C>
__global__ void __launch_bounds__(L3Cfg<C>::kThreads, 1)
local3d_tc_kernel(const __grid_constant__ CUtensorMap tmIn, const Fno3dPlan p, const Fno3dLayer L,
                  uint8_t* __restrict__ hout, unsigned* err) {
    using F = L3Cfg<C>;
    static_assert(C == 32 || C == 64, "K = C must be a multiple of 32");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem + F::kOffA;
    uint8_t* sW = smem + F::kOffW;
    float* sBias = reinterpret_cast<float*>(smem + F::kOffBias);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + F::kOffBars);
    uint64_t* empty = full + F::kStages;
    uint64_t* accFull = empty + F::kStages;
    uint64_t* accEmpty = accFull + F::kAccStages;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(accEmpty + F::kAccStages);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t Pp = static_cast<int64_t>(p.Hp) * p.Wp * p.Dp;
    const int tiles_per_sample = static_cast<int>(Pp / 128);
    const int num_tiles = p.B * tiles_per_sample;
    const int t_begin = static_cast<int>(static_cast<int64_t>(num_tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(num_tiles) * (blockIdx.x + 1) / gridDim.x);

    {
        // weights: E4M3 codes of the decoded weights, K-major rows of C bytes, swizzled
        for (int i = threadIdx.x; i < C * C; i += F::kThreads) {
            const int o = i / C, k = i % C;
            sW[swz_offset(o * C + k, C)] = static_cast<uint8_t>(e4m3_encode_ref(L.loc_q[i]));
        }
        for (int o = threadIdx.x; o < C; o += F::kThreads) sBias[o] = L.loc_b[o];
        if (threadIdx.x == 0) {
            for (int s = 0; s < F::kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < F::kAccStages; ++s) {
                mbar_init(&accFull[s], 1);
                mbar_init(&accEmpty[s], 4);
            }
            *sAbort = 0;
            fence_mbar_init();
        }
        if (warp == 1) tmem_alloc(sTmem, F::kTmemCols);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    const uint32_t tmem_base = *sTmem;

    if (warp == 0) {
        if (elect_one()) {
            prefetch_tmap(&tmIn);
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % F::kStages;
                const uint32_t ph = (it / F::kStages) & 1;
                if (!mbar_wait_backoff(&empty[s], ph ^ 1, sAbort, 1024)) {
                    *sAbort = 1;
                    atomicOr(err, kErrWaitSlotFree);
                    break;
                }
                const int b = tile / tiles_per_sample;
                const int p0 = (tile - b * tiles_per_sample) * 128;
                mbar_arrive_expect_tx(&full[s], F::kABytes);
                tma_load_2d(sA + s * F::kABytes, &tmIn, &full[s], p0, b * C);
                tma_load_2d(sA + s * F::kABytes + F::kABytes / 2, &tmIn, &full[s], p0 + 64, b * C);
            }
            for (int j = (it > F::kStages ? it - F::kStages : 0); j < it; ++j)
                if (!mbar_wait_drain(&full[j % F::kStages], (j / F::kStages) & 1)) {
                    atomicOr(err, kErrWaitDrain);
                    break;
                }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idesc = idesc_e4m3(C) | (1u << 15);  // A MN-major
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % F::kStages;
                const uint32_t ph = (it / F::kStages) & 1;
                const int a = it % F::kAccStages;
                const uint32_t aph = (it / F::kAccStages) & 1;
                if (!mbar_wait_backoff(&accEmpty[a], aph ^ 1, sAbort, 128) ||
                    !mbar_wait_backoff(&full[s], ph, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(err, kErrWaitTmaFull);
                    break;
                }
                tc_fence_after();
                const uint32_t aBase = smem_u32(sA + s * F::kABytes);
#pragma unroll
                for (int kk = 0; kk < C / 32; ++kk)
                    mma_f8(tmem_base + a * C, umma_desc_mn_sw64(aBase + kk * 2048, F::kABytes / 2, 512),
                           umma_desc(smem_u32(sW) + kk * 32, C), idesc, kk > 0 ? 1u : 0u);
                mma_commit(&empty[s]);
                mma_commit(&accFull[a]);
            }
            if (it > 0) {
                const int j = it - 1;
                if (!mbar_wait_drain(&accFull[j % F::kAccStages], (j / F::kAccStages) & 1))
                    atomicOr(err, kErrWaitDrain);
            }
        }
        __syncwarp();
    } else {
        const int ew = warp - 2;
        const int quad = warp & 3;
        const int grp = ew >> 2;
        const float sc = __fmul_rn(L.s_in, L.s_w);
        const float inv_out = inv_of(L.s_out);
        for (int it = grp; t_begin + it < t_end; it += F::kGroups) {
            const int tile = t_begin + it;
            const uint32_t aph = (it / F::kAccStages) & 1;
            if (!mbar_wait(&accFull[grp], aph, sAbort)) {
                *sAbort = 1;
                atomicOr(err, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            const int b = tile / tiles_per_sample;
            const int64_t pt = static_cast<int64_t>(tile - b * tiles_per_sample) * 128 + quad * 32 + lane;
            const int64_t base = static_cast<int64_t>(b) * C * Pp + pt;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + grp * C;
#pragma unroll 1
            for (int h = 0; h < C / 32; ++h) {
                uint32_t acc[32];
                float x1v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) x1v[j] = __ldg(p.x1 + base + static_cast<int64_t>(32 * h + j) * Pp);
                tmem_ld32(tbase + 32 * h, acc);
                tmem_wait_ld();
                if (h == C / 32 - 1) {
                    // the accumulator stage is free once every TMEM read of it is done
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&accEmpty[grp]);
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int o = 32 * h + j;
                    const float x2 = fp8_fake_quant(__fadd_rn(__fmul_rn(__uint_as_float(acc[j]), sc), sBias[o]),
                                                    L.s_out, inv_out);
                    const float z = act_f(__fadd_rn(x1v[j], x2), p.act);
                    hout[base + static_cast<int64_t>(o) * Pp] = static_cast<uint8_t>(e4m3_code(z, inv_out));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, F::kTmemCols);
    }
}

// projection, one unpadded point per thread
template <int C>
__global__ void __launch_bounds__(128) proj3d_kernel(Fno3dPlan p, const void* hin, float s_in) {
    __shared__ float sQ[C * C];
    const float* qsrc = p.fp8 ? p.pq_q : p.pq_w;
    for (int i = threadIdx.x; i < C * C; i += blockDim.x) sQ[i] = qsrc[i];
    __syncthreads();
    const int64_t Pp = static_cast<int64_t>(p.Hp) * p.Wp * p.Dp;
    const int64_t P = static_cast<int64_t>(p.H) * p.W * p.D;
    const int64_t total = static_cast<int64_t>(p.B) * P;
    constexpr int nu = linear_unfused_len(C);
    const float sc = __fmul_rn(s_in, p.s_pq_w);
    const float inv_pq = inv_of(p.s_pq), inv_po = inv_of(p.s_po);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = t / P, pt = t - (t / P) * P;
        const int dd = static_cast<int>(pt % p.D);
        const int ww = static_cast<int>((pt / p.D) % p.W);
        const int hh = static_cast<int>(pt / (static_cast<int64_t>(p.D) * p.W));
        const int64_t base = b * C * Pp + (static_cast<int64_t>(hh) * p.Wp + ww) * p.Dp + dd;
        float a[C];
#pragma unroll
        for (int k = 0; k < C; ++k) {
            if (p.fp8) a[k] = e4m3_decode_ref(static_cast<const uint8_t*>(hin)[base + k * Pp]);
            else a[k] = static_cast<const float*>(hin)[base + k * Pp];
        }
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = j < p.out_ch ? __ldg(p.po_b + j) : 0.0f;
        for (int c = 0; c < C; ++c) {
            float q;
            if (p.fp8) {
                q = 0.0f;
#pragma unroll
                for (int k = 0; k < C; ++k) q = __fadd_rn(q, __fmul_rn(a[k], sQ[c * C + k]));
                q = fp8_fake_quant(__fadd_rn(__fmul_rn(q, sc), __ldg(p.pq_b + c)), p.s_pq, inv_pq);
            } else {
                q = __ldg(p.pq_b + c);
#pragma unroll
                for (int k = 0; k < C; ++k) q = linear_step(q, a[k], sQ[c * C + k], k >= nu);
            }
            q = act_f(q, p.act);
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < p.out_ch)
                    acc[j] = linear_step(acc[j], q, __ldg(p.po_w + static_cast<int64_t>(j) * C + c), c >= nu);
        }
        float* yr = p.y + t * p.out_ch;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j < p.out_ch) yr[j] = p.fp8 ? fp8_fake_quant(acc[j], p.s_po, inv_po) : acc[j];
    }
}

int mix_group(int C) {
    for (int G = 8; G > 1; G >>= 1)
        if (C % G == 0) return G;
    return 1;
}

template <int C>
cudaError_t run_c(const Fno3dPlan& p, cudaStream_t st) {
    const int sms = device_sm_count();
    const int64_t Pp = static_cast<int64_t>(p.Hp) * p.Wp * p.Dp;
    cudaError_t e;
    auto timed = [&](const char* name, auto&& fn) -> cudaError_t {
        if (p.timer) p.timer->begin(name, st);
        fn();
        if (p.timer) p.timer->end(st);
        return cudaGetLastError();
    };
    const int64_t tl = static_cast<int64_t>(p.B) * p.C * Pp;
    if ((e = timed("fno3d_lift", [&] {
             lift3d_kernel<<<static_cast<int>(std::min<int64_t>((tl + 255) / 256, sms * 32)), 256, 0, st>>>(p);
         })) != cudaSuccess)
        return e;
    const int KK = p.MW * p.MD, M = p.MH * KK, G = mix_group(p.C);
    const int LN = std::max(p.Wp, p.Dp);
    const size_t sa = (8 * static_cast<size_t>(p.Dp) + static_cast<size_t>(p.MD) * p.Wp) * sizeof(float2);
    const size_t sb = 8 * static_cast<size_t>(p.Hp) * sizeof(float2);
    const size_t sx = (static_cast<size_t>(G) * M + 8 * static_cast<size_t>(p.Hp)) * sizeof(float2);
    const size_t si = (static_cast<size_t>(p.MD) * p.Wp + 8 * static_cast<size_t>(LN)) * sizeof(float2);
    if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(fwd3d_a_kernel), static_cast<int>(sa))) != cudaSuccess ||
        (e = set_max_dynamic_smem(reinterpret_cast<const void*>(fwd3d_b_kernel), static_cast<int>(sb))) != cudaSuccess ||
        (e = set_max_dynamic_smem(reinterpret_cast<const void*>(mix3d_kernel), static_cast<int>(sx))) != cudaSuccess ||
        (e = set_max_dynamic_smem(reinterpret_cast<const void*>(inv3d_kernel), static_cast<int>(si))) != cudaSuccess)
        return e;
    const int64_t tp = static_cast<int64_t>(p.B) * Pp;
    const int lgrid = static_cast<int>(std::min<int64_t>((tp + 127) / 128, sms * 16));
    for (int i = 0; i < p.L; ++i) {
        const Fno3dLayer& L = p.layer[i];
        const void* hin = p.h[i & 1];
        void* hout = p.h[(i + 1) & 1];
        if ((e = timed("fno3d_fwd", [&] {
                 fwd3d_a_kernel<<<dim3(p.Hp, p.C, p.B), 256, sa, st>>>(p, hin, L.s_in);
                 fwd3d_b_kernel<<<dim3(p.C, p.B), 256, sb, st>>>(p);
             })) != cudaSuccess)
            return e;
        if ((e = timed("fno3d_mix", [&] {
                 mix3d_kernel<<<dim3(p.C / G, p.B), 256, sx, st>>>(p, L.wr, L.wi, G);
             })) != cudaSuccess)
            return e;
        if ((e = timed("fno3d_inv", [&] { inv3d_kernel<<<dim3(p.Hp, p.C, p.B), 256, si, st>>>(p); })) != cudaSuccess)
            return e;
        bool tc = false;
        if constexpr (C == 32 || C == 64) {
            // FP8: the local layer on tensor cores when a sample is whole 128-point tiles
            if (p.fp8 && Pp % 128 == 0) {
                using F = L3Cfg<C>;
                CUtensorMap tm;
                unsigned* err = device_error_word();
                if (!err) return cudaErrorMemoryAllocation;
                if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, hin, static_cast<uint64_t>(Pp),
                               static_cast<uint64_t>(p.B) * C, static_cast<uint64_t>(Pp), 64, C, 64))
                    return cudaErrorInvalidValue;
                auto k = local3d_tc_kernel<C>;
                if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(k), F::kSmemBytes)) != cudaSuccess)
                    return e;
                const int64_t tiles = static_cast<int64_t>(p.B) * (Pp / 128);
                const int grid = static_cast<int>(std::min<int64_t>(tiles, sms));
                if ((e = timed("fno3d_local", [&] {
                         k<<<grid, F::kThreads, F::kSmemBytes, st>>>(tm, p, L, static_cast<uint8_t*>(hout), err);
                     })) != cudaSuccess)
                    return e;
                tc = true;
            }
        }
        if (!tc &&
            (e = timed("fno3d_local", [&] { local3d_kernel<C><<<lgrid, 128, 0, st>>>(p, L, hin, hout); })) !=
                cudaSuccess)
            return e;
    }
    const int64_t tq = static_cast<int64_t>(p.B) * p.H * p.W * p.D;
    const float s_last = p.L > 0 ? p.layer[p.L - 1].s_out : p.s_lift;
    return timed("fno3d_proj", [&] {
        proj3d_kernel<C><<<static_cast<int>(std::min<int64_t>((tq + 127) / 128, sms * 16)), 128, 0, st>>>(
            p, p.h[p.L & 1], s_last);
    });
}

}  // namespace

const char* fno3d_unsupported(int C, int Hp, int Wp, int Dp, int MH, int MW, int MD, int out_ch) {
    if (C != 8 && C != 16 && C != 32 && C != 64) return "FNO3d GPU executor: width must be 8, 16, 32 or 64";
    if (out_ch < 1 || out_ch > 16) return "FNO3d GPU executor: out_channels must be in [1, 16]";
    if (Hp > 1024 || Wp > 1024 || Dp > 1024) return "FNO3d GPU executor: padded grid sides <= 1024";
    const size_t G = static_cast<size_t>(mix_group(C));
    if ((G * MH * MW * MD + 8 * static_cast<size_t>(Hp)) * sizeof(float2) > 200 * 1024 ||
        (static_cast<size_t>(MD) * Wp + 8 * static_cast<size_t>(std::max(Wp, Dp))) * sizeof(float2) > 200 * 1024 ||
        (8 * static_cast<size_t>(Dp) + static_cast<size_t>(MD) * Wp) * sizeof(float2) > 200 * 1024)
        return "FNO3d GPU executor: too many modes for the shared-memory transforms";
    return nullptr;
}

cudaError_t fno3d_run(const Fno3dPlan& p, cudaStream_t st) {
    if (p.B == 0) return cudaSuccess;
    switch (p.C) {
        case 8: return run_c<8>(p, st);
        case 16: return run_c<16>(p, st);
        case 32: return run_c<32>(p, st);
        default: return run_c<64>(p, st);
    }
}

}  // namespace nfx
