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
#include <cmath>
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
    if (fp8) return __fmul_rn(e4m3_decode_fast(static_cast<const uint8_t*>(h)[i]), s);
    return static_cast<const float*>(h)[i];
}

// one padded point per thread, every channel (the padded sides are powers of two, so
// the point index splits by shifts; the input row is read once into L1)
__global__ void __launch_bounds__(256) lift3d_kernel(Fno3dPlan p) {
    const int lgD = 31 - __clz(p.Dp), lgW = 31 - __clz(p.Wp);
    const int lgP = lgD + lgW + (31 - __clz(p.Hp));
    const int64_t total = static_cast<int64_t>(p.B) << lgP;
    const int nu = linear_unfused_len(p.in_ch);
    const float inv = inv_of(p.s_lift);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = t >> lgP;
        const int pt = static_cast<int>(t - (b << lgP));
        const int dd = pt & (p.Dp - 1), ww = (pt >> lgD) & (p.Wp - 1), hh = pt >> (lgD + lgW);
        const bool inside = hh < p.H && ww < p.W && dd < p.D;
        const float* xr = p.x + (((b * p.H + hh) * p.W + ww) * p.D + dd) * p.in_ch;
        // the first 8 input features in registers, the rest (wider inputs) from L1
        constexpr int kReg = 8;
        const int nreg = p.in_ch < kReg ? p.in_ch : kReg;
        float xv[kReg];
#pragma unroll
        for (int k = 0; k < kReg; ++k) xv[k] = (inside && k < nreg) ? __ldg(xr + k) : 0.0f;
        uint8_t* h8 = static_cast<uint8_t*>(p.h[0]) + (b * p.C << lgP) + pt;
        float* h32 = static_cast<float*>(p.h[0]) + (b * p.C << lgP) + pt;
        for (int c = 0; c < p.C; ++c) {
            float v = 0.0f;
            if (inside) {
                const float* wc = p.lift_w + c * p.in_ch;
                v = __ldg(p.lift_b + c);
#pragma unroll
                for (int k = 0; k < kReg; ++k)
                    if (k < nreg) v = linear_step(v, xv[k], __ldg(wc + k), k >= nu);
                for (int k = kReg; k < p.in_ch; ++k) v = linear_step(v, __ldg(xr + k), __ldg(wc + k), k >= nu);
            }
            if (p.fp8) h8[static_cast<int64_t>(c) << lgP] = static_cast<uint8_t>(e4m3_code(v, inv));
            else h32[static_cast<int64_t>(c) << lgP] = v;
        }
    }
}

// Four consecutive padded points of one D row per thread (Dp a multiple of 4, IN <= 8
// input features, a compile-time count so every Linear step is unrolled with its
// rounding fixed): each weight is read once per four points, and a channel's four
// outputs leave in one 32-bit (E4M3 codes) or 128-bit (fp32) store.
template <int IN>
__global__ void __launch_bounds__(256) lift3d_x4_kernel(Fno3dPlan p) {
    const int lgD = 31 - __clz(p.Dp), lgW = 31 - __clz(p.Wp);
    const int lgP = lgD + lgW + (31 - __clz(p.Hp));
    const int64_t total = static_cast<int64_t>(p.B) << (lgP - 2);
    constexpr int nu = linear_unfused_len(IN);
    const float inv = inv_of(p.s_lift);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = t >> (lgP - 2);
        const int pt = static_cast<int>(t - (b << (lgP - 2))) << 2;
        const int dd = pt & (p.Dp - 1), ww = (pt >> lgD) & (p.Wp - 1), hh = pt >> (lgD + lgW);
        const bool row_in = hh < p.H && ww < p.W;
        bool in[4];
        float xv[4][IN];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            in[i] = row_in && dd + i < p.D;
            const float* xr = p.x + ((((b * p.H + hh) * p.W + ww) * p.D) + (in[i] ? dd + i : 0)) * IN;
#pragma unroll
            for (int k = 0; k < IN; ++k) xv[i][k] = in[i] ? __ldg(xr + k) : 0.0f;
        }
        uint8_t* h8 = static_cast<uint8_t*>(p.h[0]) + (b * p.C << lgP) + pt;
        float* h32 = static_cast<float*>(p.h[0]) + (b * p.C << lgP) + pt;
#pragma unroll 2
        for (int c = 0; c < p.C; ++c) {
            const float* wc = p.lift_w + c * IN;
            const float bc = __ldg(p.lift_b + c);
            float wk[IN];
#pragma unroll
            for (int k = 0; k < IN; ++k) wk[k] = __ldg(wc + k);
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float a = bc;
#pragma unroll
                for (int k = 0; k < IN; ++k) a = linear_step(a, xv[i][k], wk[k], k >= nu);
                v[i] = in[i] ? a : 0.0f;
            }
            if (p.fp8)
                *reinterpret_cast<uint32_t*>(h8 + (static_cast<int64_t>(c) << lgP)) =
                    e4m3_code(v[0], inv) | (e4m3_code(v[1], inv) << 8) | (e4m3_code(v[2], inv) << 16) |
                    (e4m3_code(v[3], inv) << 24);
            else
                *reinterpret_cast<float4*>(h32 + (static_cast<int64_t>(c) << lgP)) = make_float4(v[0], v[1], v[2], v[3]);
        }
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
    if (p.Dp == 64) {
        // D rows in registers (warp_fft64_regs): mode kd is entry lane + 32 j
        for (int w = warp; w < p.Wp; w += 8) {
            float2 v[2];
#pragma unroll
            for (int m = 0; m < 2; ++m)
                v[m] = make_float2(value_at(hin, base + static_cast<int64_t>(w) * 64 + fft64_src(lane, m), p.fp8, s_in), 0.0f);
            warp_fft64_regs<false>(v, row, p.tw[4], lane);
            const int wr = bit_reverse(w, lgW);
#pragma unroll
            for (int j = 0; j < 2; ++j)
                if (lane + 32 * j < p.MD) col[(lane + 32 * j) * p.Wp + wr] = v[j];
        }
    } else {
        for (int w = warp; w < p.Wp; w += 8) {
            for (int d = lane; d < p.Dp; d += 32)
                row[bit_reverse(d, lgD)] = make_float2(value_at(hin, base + static_cast<int64_t>(w) * p.Dp + d, p.fp8, s_in), 0.0f);
            __syncwarp();
            warp_fft_row<false>(row, p.Dp, p.tw[4], lane);
            const int wr = bit_reverse(w, lgW);
            for (int kd = lane; kd < p.MD; kd += 32) col[kd * p.Wp + wr] = row[kd];
            __syncwarp();
        }
    }
    __syncthreads();
    float2* A = p.A + ((static_cast<int64_t>(b) * p.C + c) * p.Hp + hh) * p.MW * p.MD;
    if (p.Wp == 64 && p.Dp >= 64) {  // the warp's row buffer (Dp entries) is the scratch
        for (int kd = warp; kd < p.MD; kd += 8) {
            float2 v[2];
#pragma unroll
            for (int m = 0; m < 2; ++m) v[m] = col[kd * 64 + 2 * lane + m];  // bit-reversed row
            warp_fft64_regs<false>(v, row, p.tw[2], lane);
#pragma unroll
            for (int j = 0; j < 2; ++j)
                if (lane + 32 * j < p.MW) A[(lane + 32 * j) * p.MD + kd] = v[j];
        }
        return;
    }
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
    if (p.Hp == 64) {
        for (int q = warp; q < KK; q += 8) {
            float2 v[2];
#pragma unroll
            for (int m = 0; m < 2; ++m) v[m] = A[static_cast<int64_t>(fft64_src(lane, m)) * KK + q];
            warp_fft64_regs<false>(v, line, p.tw[0], lane);
#pragma unroll
            for (int j = 0; j < 2; ++j)
                if (lane + 32 * j < p.MH) X[(lane + 32 * j) * KK + q] = v[j];
        }
        return;
    }
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
    if (p.Hp == 64) {
        for (int q = warp; q < G * KK; q += 8) {
            const int r = q / KK, kk = q - (q / KK) * KK;
            float2 v[2];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int h = fft64_src(lane, m);
                v[m] = h < p.MH ? sY[r * M + h * KK + kk] : make_float2(0.0f, 0.0f);
            }
            warp_fft64_regs<true>(v, line, p.tw[1], lane);
            float2* dst = p.colinv + (static_cast<int64_t>(b) * C + o0 + r) * p.Hp * KK + kk;
#pragma unroll
            for (int j = 0; j < 2; ++j)
                dst[static_cast<int64_t>(lane + 32 * j) * KK] =
                    make_float2(__fmul_rn(v[j].x, invH), __fmul_rn(v[j].y, invH));
        }
        return;
    }
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
    if (p.Wp == 64) {
        for (int kd = warp; kd < p.MD; kd += 8) {
            float2 v[2];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int w = fft64_src(lane, m);
                v[m] = w < p.MW ? ci[w * p.MD + kd] : make_float2(0.0f, 0.0f);
            }
            warp_fft64_regs<true>(v, line, p.tw[3], lane);
#pragma unroll
            for (int j = 0; j < 2; ++j)
                tmp[kd * 64 + lane + 32 * j] = make_float2(__fmul_rn(v[j].x, invW), __fmul_rn(v[j].y, invW));
        }
    } else {
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
    }
    __syncthreads();
    const int half = p.Dp / 2 + 1;
    const float invD = __fdiv_rn(1.0f, static_cast<float>(p.Dp));
    float* x1 = p.x1 + ((static_cast<int64_t>(b) * p.C + o) * p.Hp + hh) * p.Wp * p.Dp;
    if (p.Dp == 64) {
        // D lines in registers (warp_fft64_regs): point d is entry lane + 32 j
        for (int w = warp; w < p.Wp; w += 8) {
            float2 v[2];
#pragma unroll
            for (int m = 0; m < 2; ++m) {
                const int j = fft64_src(lane, m);
                if (j < half) {
                    v[m] = j < p.MD ? tmp[j * p.Wp + w] : make_float2(0.0f, 0.0f);
                } else {
                    const int i = 64 - j;
                    const float2 u = i < p.MD ? tmp[i * p.Wp + w] : make_float2(0.0f, 0.0f);
                    v[m] = make_float2(u.x, -u.y);
                }
            }
            warp_fft64_regs<true>(v, line, p.tw[5], lane);
#pragma unroll
            for (int j = 0; j < 2; ++j) x1[static_cast<int64_t>(w) * 64 + lane + 32 * j] = __fmul_rn(v[j].x, invD);
        }
        return;
    }
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

// ---------------------------------------------------------------------------
// Direct truncated DFTs of the D and W passes (fno3d_direct_dft: the FP8 variant at
// widths 32 / 64).  Only the kept modes are formed, each output one fp32 sum over its
// line against the correctly rounded tables of fno3d_dft_tables:
//   forward  Y[w][kd] = sum_d x[w][d] e^{-2 pi i kd d / Dp}              (real input)
//            A[kw][kd] = s_in * sum_w Y[w][kd] e^{-2 pi i kw w / Wp}
//   inverse  u[w][j]  = f_j sum_kw ci[kw][j] e^{+2 pi i kw w / Wp},
//            f_j = (j = 0 or j = Dp/2 ? 1 : 2) / (Wp Dp)   (exact powers of two)
//            x1[w][d] = sum_j Re(u[w][j] e^{+2 pi i j d / Dp})
// The inverse is the Hermitian D-axis Irfft of the reference (a kept mode j in
// 1 .. Dp/2 - 1 stands for itself and its conjugate at Dp - j), so x1 is the radix-2
// passes' result up to fp32 rounding.
// ---------------------------------------------------------------------------
struct DftDims {
    int MD4, MW2;   // kept modes rounded up to 4 (kd) and 2 (kw); table columns
    int XS, YS;     // row strides (floats): decoded plane, D-pass output
    int TWS, TWI;   // row strides (floats) of the W table: forward, inverse
    int UJ;         // row stride (floats) of the inverse D-pass input u
    int NPf, NPi;   // planes per CTA pass: forward, inverse
};

constexpr int kDftThreads = 128;
constexpr int kDftPre = 4;  // uint4 of codes a thread prefetches per forward pass

DftDims dft_dims(int Wp, int Dp, int MW, int MD) {
    DftDims g;
    g.MD4 = (MD + 3) / 4 * 4;
    g.MW2 = (MW + 1) / 2 * 2;
    g.XS = Dp + 4;
    g.YS = 2 * g.MD4 + 4;
    g.TWS = 2 * g.MW2 + 4;
    g.TWI = 2 * g.MW2 + 2;
    g.UJ = 2 * g.MD4 + 2;
    const int items_f = (Wp / 2) * (g.MD4 / 4), items_i = (Wp / 8) * (Dp / 4);
    g.NPf = std::max(1, kDftThreads / std::max(1, items_f));
    while (g.NPf > 1 && g.NPf * Wp * Dp > kDftPre * kDftThreads * 16) g.NPf >>= 1;
    g.NPi = std::max(1, kDftThreads / std::max(1, items_i));
    return g;
}

size_t dft_fwd_smem(const DftDims& g, int Wp, int Dp) {
    return sizeof(float) * (static_cast<size_t>(2) * Dp * g.MD4 + static_cast<size_t>(Wp) * g.TWS +
                            static_cast<size_t>(g.NPf) * Wp * (g.XS + g.YS));
}

size_t dft_inv_smem(const DftDims& g, int Wp, int Dp, int MW) {
    return sizeof(float) * (static_cast<size_t>(2) * g.MD4 * Dp + static_cast<size_t>(Wp) * g.TWI +
                            static_cast<size_t>(g.NPi) * (static_cast<size_t>(MW) * 2 * g.MD4 +
                                                          static_cast<size_t>(Wp) * g.UJ));
}

// W pass of the direct forward DFT for the NP planes q0 .. q0 + NP - 1 held in sY
// ([NP][Wp][ys] floats, (re, im) per kd): A[q][kw][kd] = s_in * sum_w Y[w][kd] e^{-2 pi i
// kw w / Wp}, 2 x 2 output modes per thread, w split over 8 consecutive lanes and
// summed by shuffles.  Every thread of the CTA takes part (the shuffles are warp-wide).
__device__ __forceinline__ void dft_w_pass(const Fno3dPlan& p, int MD4, int MW2, const float* sY, int ys,
                                           const float* tW, int tws, int NP, int64_t q0, int64_t nplanes,
                                           float s_in) {
    const int T = blockDim.x, tid = threadIdx.x, Wp = p.Wp;
    const int items2 = (MW2 / 2) * (MD4 / 2) * 8;
    for (int base = 0; base < NP * items2; base += T) {
        const int it = base + tid;
        const bool live = it < NP * items2;
        const int pl = live ? it / items2 : 0, r = it - pl * items2;
        const int s = r & 7, blk = r >> 3;
        const int kwp = blk / (MD4 / 2), kdp = blk - kwp * (MD4 / 2);
        // (re, im) of output (kw = 2 kwp + a, kd = 2 kdp + c) at 2 a + c, each lane of the
        // f32x2 products the scalar fmaf chain re += yr tc, re += yi (-ts); im += yr ts,
        // im += yi tc
        float2 o2[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) o2[k] = make_float2(0.0f, 0.0f);
        if (live) {
            for (int w = s; w < Wp; w += 8) {
                const float4 y = *reinterpret_cast<const float4*>(sY + (pl * Wp + w) * ys + 4 * kdp);
                const float4 t = *reinterpret_cast<const float4*>(tW + w * tws + 4 * kwp);
                const float yr[2] = {y.x, y.z}, yi[2] = {y.y, y.w};
                const float tc[2] = {t.x, t.z}, ts[2] = {t.y, t.w};
#pragma unroll
                for (int a = 0; a < 2; ++a)
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        float2& q = o2[2 * a + c];
                        q = fma2_rn(make_float2(yr[c], yr[c]), make_float2(tc[a], ts[a]), q);
                        q = fma2_rn(make_float2(yi[c], yi[c]), make_float2(-ts[a], tc[a]), q);
                    }
            }
        }
        float o[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            o[2 * k] = o2[k].x;
            o[2 * k + 1] = o2[k].y;
        }
#pragma unroll
        for (int m = 1; m < 8; m <<= 1)
#pragma unroll
            for (int k = 0; k < 8; ++k) o[k] = __fadd_rn(o[k], __shfl_xor_sync(0xffffffffu, o[k], m));
        const int64_t q = q0 + pl;
        if (live && s == 0 && q < nplanes) {
            float2* A = p.A + q * p.MW * p.MD;
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int kw = 2 * kwp + a, kd = 2 * kdp + c;
                    if (kw < p.MW && kd < p.MD)
                        A[kw * p.MD + kd] =
                            make_float2(__fmul_rn(o[4 * a + 2 * c], s_in), __fmul_rn(o[4 * a + 2 * c + 1], s_in));
                }
        }
    }
}

// Persistent over the B * C * Hp (b, c, h) planes, NPf planes per pass.
// smem floats: tD [Dp][MD4] float2 | tW [Wp][TWS] | x [NPf][Wp][XS] | Y [NPf][Wp][YS]
__global__ void __launch_bounds__(kDftThreads) fwd3d_dft_kernel(Fno3dPlan p, DftDims g,
                                                                const uint8_t* __restrict__ hin, float s_in) {
    extern __shared__ float4 sm4[];
    float* sm = reinterpret_cast<float*>(sm4);
    const int T = kDftThreads, tid = threadIdx.x;
    const int Wp = p.Wp, Dp = p.Dp, MD4 = g.MD4, NP = g.NPf, half = Wp / 2;
    float* tD = sm;
    float* tW = tD + 2 * Dp * MD4;
    float* sx = tW + Wp * g.TWS;
    float* sY = sx + NP * Wp * g.XS;
    for (int i = tid; i < 2 * Dp * MD4; i += T) tD[i] = __ldg(p.dft + i);
    {
        const float* gW = p.dft + 2 * Dp * MD4;
        const int rw = 2 * g.MW2;
        for (int i = tid; i < Wp * rw; i += T) tW[(i / rw) * g.TWS + i % rw] = __ldg(gW + i);
    }
    const int64_t nplanes = static_cast<int64_t>(p.B) * p.C * p.Hp;
    const int v16 = Wp * Dp / 16;  // uint4 of codes per plane
    const int nv = NP * v16;
    const int64_t npass = (nplanes + NP - 1) / NP;
    uint4 pre[kDftPre];
    auto fetch = [&](int64_t pass) {
        const int64_t q0 = pass * NP;
        const uint4* src = reinterpret_cast<const uint4*>(hin) + q0 * v16;
        const int64_t lim = (nplanes - q0) * v16;
#pragma unroll
        for (int r = 0; r < kDftPre; ++r) {
            const int i = tid + r * T;
            pre[r] = (i < nv && i < lim) ? __ldg(src + i) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    int64_t pass = blockIdx.x;
    if (pass < npass) fetch(pass);
    const int items1 = half * (MD4 / 4);
    for (; pass < npass; pass += gridDim.x) {
        __syncthreads();  // the previous pass is done with x and Y
#pragma unroll
        for (int r = 0; r < kDftPre; ++r) {
            const int i = tid + r * T;
            if (i < nv) {
                const int pl = i / v16, e = (i - pl * v16) * 16;
                const int w = e / Dp, d = e - w * Dp;
                float* dst = sx + (pl * Wp + w) * g.XS + d;
                const uint32_t wd[4] = {pre[r].x, pre[r].y, pre[r].z, pre[r].w};
#pragma unroll
                for (int m = 0; m < 4; ++m)
                    *reinterpret_cast<float4*>(dst + 4 * m) =
                        make_float4(e4m3_decode_fast(wd[m] & 0xFFu), e4m3_decode_fast((wd[m] >> 8) & 0xFFu),
                                    e4m3_decode_fast((wd[m] >> 16) & 0xFFu), e4m3_decode_fast(wd[m] >> 24));
            }
        }
        if (pass + gridDim.x < npass) fetch(pass + gridDim.x);
        __syncthreads();
        // D pass: rows rp and rp + Wp/2, kept modes 4 kq .. 4 kq + 3
        for (int it = tid; it < NP * items1; it += T) {
            const int pl = it / items1, r = it - pl * items1;
            const int rp = r % half, kq = r / half;
            const float* x0 = sx + (pl * Wp + rp) * g.XS;
            const float* x1p = x0 + half * g.XS;
            const float* tk = tD + 8 * kq;
            float a0[8], a1[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) a0[k] = a1[k] = 0.0f;
#pragma unroll 2
            for (int d = 0; d < Dp; d += 4) {
                const float4 u = *reinterpret_cast<const float4*>(x0 + d);
                const float4 v = *reinterpret_cast<const float4*>(x1p + d);
                const float uu[4] = {u.x, u.y, u.z, u.w}, vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 t0 = *reinterpret_cast<const float4*>(tk + (d + q) * 2 * MD4);
                    const float4 t1 = *reinterpret_cast<const float4*>(tk + (d + q) * 2 * MD4 + 4);
                    const float tt[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        a0[k] = __fmaf_rn(uu[q], tt[k], a0[k]);
                        a1[k] = __fmaf_rn(vv[q], tt[k], a1[k]);
                    }
                }
            }
            float* y0 = sY + (pl * Wp + rp) * g.YS + 8 * kq;
            float* y1 = y0 + half * g.YS;
            *reinterpret_cast<float4*>(y0) = make_float4(a0[0], a0[1], a0[2], a0[3]);
            *reinterpret_cast<float4*>(y0 + 4) = make_float4(a0[4], a0[5], a0[6], a0[7]);
            *reinterpret_cast<float4*>(y1) = make_float4(a1[0], a1[1], a1[2], a1[3]);
            *reinterpret_cast<float4*>(y1 + 4) = make_float4(a1[4], a1[5], a1[6], a1[7]);
        }
        __syncthreads();
        dft_w_pass(p, MD4, g.MW2, sY, g.YS, tW, g.TWS, NP, pass * NP, nplanes, s_in);
    }
}

// ---------------------------------------------------------------------------
// fwd3d_tc: the direct forward DFT with its D pass on tensor cores (fno3d_direct_dft
// geometries with Wp dividing 128, Dp = 64 or 128 and at most 16 kept kd modes).  A
// tile is 128 D rows (128 / Wp planes).  E4M3 values are exact in f16
// (cvt.rn.f16x2.e4m3x2 converts two codes per instruction), so the D pass
//   Y[row][n] = sum_d x[row][d] T[n][d],   T[2 kd] = cos(2 pi kd d / Dp), T[2 kd + 1] = -sin
// is one kind::f16 MMA chain (M = 128, N = 16 or 32, K = Dp, fp32 accumulation) with T
// split into two f16 terms, hi = f16(T) and lo = f16(T - hi), whose sum holds T to
// about 2^-22 relative (each product exact in fp32).  The W pass runs on CUDA cores
// from shared memory (dft_w_pass).  128 threads: all convert the tile's codes into
// the 128-byte-swizzled K-major A tile, thread 0 issues the MMAs, warp q reads TMEM
// lanes 32 q .. 32 q + 31 (its rows of Y).
// ---------------------------------------------------------------------------
struct FtcDims {
    int N;       // MMA N: 16 or 32 (2 MD4 rounded up)
    int YS;      // sY row stride (floats)
    int NPt;     // planes per tile (128 / Wp)
    int offB, offY, offW, offBar, smem;  // byte offsets in the 1024-aligned dynamic smem, its size
};

bool fwd_tc_ok(int Wp, int Dp, int MD) {
    return Wp <= 128 && 128 % Wp == 0 && (Dp == 64 || Dp == 128) && MD <= 16;
}

FtcDims ftc_dims(const DftDims& g, int Wp, int Dp) {
    FtcDims f;
    f.N = 2 * g.MD4 <= 16 ? 16 : 32;
    f.YS = f.N + 4;
    f.NPt = 128 / Wp;
    f.offB = Dp * 256;                             // A: 128 rows x Dp f16
    f.offY = f.offB + 2 * (Dp / 64) * f.N * 128;   // B: two f16 terms of T
    f.offW = f.offY + 128 * f.YS * 4;
    f.offBar = (f.offW + Wp * g.TWS * 4 + 15) & ~15;
    f.smem = f.offBar + 16 + 1024;                 // barrier, TMEM slot, abort flag; alignment slack
    return f;
}

// two E4M3 codes (low and high byte of v) -> f16x2 (low half from the low byte); exact
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t v) {
    uint32_t r;
    const unsigned short in = static_cast<unsigned short>(v & 0xFFFFu);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(in));
    return r;
}

__device__ __forceinline__ unsigned short f16_bits_rn(float x) {
    unsigned short r;
    asm("cvt.rn.f16.f32 %0, %1;" : "=h"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ float f16_bits_to_f32(unsigned short h) {
    float r;
    asm("cvt.f32.f16 %0, %1;" : "=f"(r) : "h"(h));
    return r;
}

__global__ void __launch_bounds__(128) fwd3d_tc_kernel(Fno3dPlan p, DftDims g, FtcDims f,
                                                       const uint8_t* __restrict__ hin, float s_in,
                                                       unsigned* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem;
    uint8_t* sB = smem + f.offB;
    float* sY = reinterpret_cast<float*>(smem + f.offY);
    float* tW = reinterpret_cast<float*>(smem + f.offW);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + f.offBar);
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int Wp = p.Wp, Dp = p.Dp, MD4 = g.MD4, N = f.N;
    const int nkc = Dp / 64;  // 128-byte K chunks (64 f16) of a row

    {
        // T as two f16 terms, K-major 128-byte swizzled: term t, chunk kc, row n
        for (int i = tid; i < N * Dp; i += 128) {
            const int n = i / Dp, d = i - n * Dp;
            const float v = n / 2 < MD4 ? __ldg(p.dft + (d * MD4 + n / 2) * 2 + (n & 1)) : 0.0f;
            const unsigned short hi = f16_bits_rn(v);
            const unsigned short lo = f16_bits_rn(__fsub_rn(v, f16_bits_to_f32(hi)));
            const uint32_t o = swz_offset(static_cast<uint32_t>(n * 128 + (d & 63) * 2), 128);
            const int kc = d >> 6;
            *reinterpret_cast<unsigned short*>(sB + (0 * nkc + kc) * N * 128 + o) = hi;
            *reinterpret_cast<unsigned short*>(sB + (1 * nkc + kc) * N * 128 + o) = lo;
        }
        const float* gW = p.dft + 2 * Dp * MD4;
        const int rw = 2 * g.MW2;
        for (int i = tid; i < Wp * rw; i += 128) tW[(i / rw) * g.TWS + i % rw] = __ldg(gW + i);
        if (tid == 0) {
            mbar_init(bar, 1);
            *sAbort = 0;
            fence_mbar_init();
        }
        if (warp == 0) tmem_alloc(sTmem, 32);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    const uint32_t tmem = *sTmem;
    const int64_t nplanes = static_cast<int64_t>(p.B) * p.C * p.Hp;
    const int64_t ntiles = nplanes / f.NPt;  // B C Hp Wp rows, a multiple of 128
    const int rv = Dp / 16;                  // uint4 of codes per row = per thread per tile
    constexpr int kMaxPre = 8;
    uint4 pre[kMaxPre];
    auto fetch = [&](int64_t tile) {
        const uint4* src = reinterpret_cast<const uint4*>(hin) + tile * 128 * rv;
#pragma unroll
        for (int r = 0; r < kMaxPre; ++r)
            if (r < rv) pre[r] = __ldg(src + tid + r * 128);
    };
    const uint32_t idesc = N == 16 ? idesc_f16(16) : idesc_f16(32);
    int64_t tile = blockIdx.x;
    if (tile < ntiles) fetch(tile);
    uint32_t phase = 0;
    for (; tile < ntiles; tile += gridDim.x) {
        // uint4 i of the tile: codes 16 (i % rv) .. + 15 of row i / rv -> two 16-byte f16 chunks
#pragma unroll
        for (int r = 0; r < kMaxPre; ++r) {
            if (r < rv) {
                const int i = tid + r * 128;
                const int row = i / rv, k0 = (i - row * rv) * 16;
                uint8_t* chunk = sA + (k0 >> 6) * (128 * 128);
                const uint32_t o0 = swz_offset(static_cast<uint32_t>(row * 128 + (k0 & 63) * 2), 128);
                const uint32_t o1 = swz_offset(static_cast<uint32_t>(row * 128 + (k0 & 63) * 2 + 16), 128);
                *reinterpret_cast<uint4*>(chunk + o0) =
                    make_uint4(e4m3x2_to_f16x2(pre[r].x), e4m3x2_to_f16x2(pre[r].x >> 16),
                               e4m3x2_to_f16x2(pre[r].y), e4m3x2_to_f16x2(pre[r].y >> 16));
                *reinterpret_cast<uint4*>(chunk + o1) =
                    make_uint4(e4m3x2_to_f16x2(pre[r].z), e4m3x2_to_f16x2(pre[r].z >> 16),
                               e4m3x2_to_f16x2(pre[r].w), e4m3x2_to_f16x2(pre[r].w >> 16));
            }
        }
        if (tile + gridDim.x < ntiles) fetch(tile + gridDim.x);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            for (int t = 0; t < 2; ++t)
                for (int kc = 0; kc < nkc; ++kc)
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        mma_f16(tmem, umma_desc(smem_u32(sA) + kc * 16384 + ks * 32, 128),
                                umma_desc(smem_u32(sB) + (t * nkc + kc) * N * 128 + ks * 32, 128), idesc,
                                (t | kc | ks) != 0 ? 1u : 0u);
            mma_commit(bar);
        }
        const bool ok = mbar_wait(bar, phase, sAbort);
        phase ^= 1u;
        if (!ok) {
            *sAbort = 1;
            atomicOr(err, kErrWaitAccFull);
        } else {
            tc_fence_after();
            const uint32_t taddr = tmem + (static_cast<uint32_t>(warp * 32) << 16);
            float* yrow = sY + (warp * 32 + lane) * f.YS;
            if (N == 16) {
                uint32_t v[16];
                tmem_ld16(taddr, v);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; j += 4)
                    *reinterpret_cast<uint4*>(yrow + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
                uint32_t v[32];
                tmem_ld32(taddr, v);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<uint4*>(yrow + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            }
        }
        tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
        dft_w_pass(p, MD4, g.MW2, sY, f.YS, tW, g.TWS, f.NPt, tile * f.NPt, nplanes, s_in);
    }
    tc_fence_before();
    __syncthreads();
    // an MMA chain whose completion wait gave up may still be running: let it finish
    // before its TMEM is released
    if (*sAbort && tid == 0 && !mbar_wait_drain(bar, phase ^ 1u)) atomicOr(err, kErrWaitDrain);
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
}

// Persistent over the B * C * Hp (b, o, h) planes of colinv, NPi planes per pass.
// smem floats: iC [MD4][Dp] | iS [MD4][Dp] | tW [Wp][TWI] | ci [NPi][MW][2 MD4] | u [NPi][Wp][UJ]
__global__ void __launch_bounds__(kDftThreads) inv3d_dft_kernel(Fno3dPlan p, DftDims g) {
    extern __shared__ float4 sm4[];
    float* sm = reinterpret_cast<float*>(sm4);
    const int T = kDftThreads, tid = threadIdx.x;
    const int Wp = p.Wp, Dp = p.Dp, MW = p.MW, MD = p.MD, MD4 = g.MD4, NP = g.NPi;
    float* iCS = sm;
    float* tW = iCS + 2 * MD4 * Dp;
    float* sci = tW + Wp * g.TWI;
    float* su = sci + NP * MW * 2 * MD4;
    {
        const float* gW = p.dft + 2 * Dp * MD4;
        const float* gI = gW + 2 * Wp * g.MW2;
        for (int i = tid; i < 2 * MD4 * Dp; i += T) iCS[i] = __ldg(gI + i);
        const int rw = 2 * g.MW2;
        for (int i = tid; i < Wp * rw; i += T) tW[(i / rw) * g.TWI + i % rw] = __ldg(gW + i);
    }
    const float* iS = iCS + MD4 * Dp;
    const int64_t nplanes = static_cast<int64_t>(p.B) * p.C * p.Hp;
    const int KK = MW * MD;
    const int64_t npass = (nplanes + NP - 1) / NP;
    const float unit = __fdiv_rn(1.0f, static_cast<float>(Wp) * static_cast<float>(Dp));
    const int items1 = Wp * (MD4 / 2);
    const int items2 = (Wp / 8) * (Dp / 4);
    for (int64_t pass = blockIdx.x; pass < npass; pass += gridDim.x) {
        const int64_t q0 = pass * NP;
        __syncthreads();  // the previous pass is done with ci and u
        for (int i = tid; i < NP * MW * MD4; i += T) {
            const int pl = i / (MW * MD4), r = i - pl * (MW * MD4);
            const int kw = r / MD4, kd = r - kw * MD4;
            float2 v = make_float2(0.0f, 0.0f);
            if (kd < MD && q0 + pl < nplanes) v = p.colinv[(q0 + pl) * KK + kw * MD + kd];
            *reinterpret_cast<float2*>(sci + (pl * MW + kw) * 2 * MD4 + 2 * kd) = v;
        }
        __syncthreads();
        // W inverse of the kept kd columns (two per thread), scaled by f_j
        for (int it = tid; it < NP * items1; it += T) {
            const int pl = it / items1, r = it - pl * items1;
            const int w = r % Wp, jp = r / Wp;
            float ar0 = 0.0f, ai0 = 0.0f, ar1 = 0.0f, ai1 = 0.0f;
            for (int kw = 0; kw < MW; ++kw) {
                const float4 c = *reinterpret_cast<const float4*>(sci + (pl * MW + kw) * 2 * MD4 + 4 * jp);
                const float2 t = *reinterpret_cast<const float2*>(tW + w * g.TWI + 2 * kw);
                // (cr + i ci)(tc - i ts), (tc, ts) = e^{-2 pi i kw w / Wp}
                ar0 = __fmaf_rn(c.x, t.x, ar0);
                ar0 = __fmaf_rn(c.y, t.y, ar0);
                ai0 = __fmaf_rn(c.y, t.x, ai0);
                ai0 = __fmaf_rn(-c.x, t.y, ai0);
                ar1 = __fmaf_rn(c.z, t.x, ar1);
                ar1 = __fmaf_rn(c.w, t.y, ar1);
                ai1 = __fmaf_rn(c.w, t.x, ai1);
                ai1 = __fmaf_rn(-c.z, t.y, ai1);
            }
            const int j0 = 2 * jp, j1 = j0 + 1;
            const float f0 = (j0 == 0 || 2 * j0 == Dp) ? unit : __fmul_rn(2.0f, unit);
            const float f1 = (2 * j1 == Dp) ? unit : __fmul_rn(2.0f, unit);
            // stored as (f Re, -f Im): x1 = sum_j u.x cos + u.y sin (UJ is even, not a multiple of 4)
            float2* ud = reinterpret_cast<float2*>(su + (pl * Wp + w) * g.UJ + 4 * jp);
            ud[0] = make_float2(__fmul_rn(ar0, f0), -__fmul_rn(ai0, f0));
            ud[1] = make_float2(__fmul_rn(ar1, f1), -__fmul_rn(ai1, f1));
        }
        __syncthreads();
        // D inverse: 8 rows x 4 consecutive points per thread
        for (int it = tid; it < NP * items2; it += T) {
            const int pl = it / items2, r = it - pl * items2;
            const int dq = r % (Dp / 4), rg = r / (Dp / 4);
            const float* ur = su + (pl * Wp + rg * 8) * g.UJ;
            // acc[i][h] holds points 4 dq + 2 h, + 1 of row i (f32x2 lanes, each the
            // scalar fmaf chain)
            float2 acc[8][2];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = make_float2(0.0f, 0.0f);
            for (int j = 0; j < MD; ++j) {
                const float4 c4 = *reinterpret_cast<const float4*>(iCS + j * Dp + 4 * dq);
                const float4 s4 = *reinterpret_cast<const float4*>(iS + j * Dp + 4 * dq);
                const float2 c01 = make_float2(c4.x, c4.y), c23 = make_float2(c4.z, c4.w);
                const float2 s01 = make_float2(s4.x, s4.y), s23 = make_float2(s4.z, s4.w);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float2 u = *reinterpret_cast<const float2*>(ur + i * g.UJ + 2 * j);
                    const float2 ux = make_float2(u.x, u.x), uy = make_float2(u.y, u.y);
                    acc[i][0] = fma2_rn(uy, s01, fma2_rn(ux, c01, acc[i][0]));
                    acc[i][1] = fma2_rn(uy, s23, fma2_rn(ux, c23, acc[i][1]));
                }
            }
            const int64_t q = q0 + pl;
            if (q < nplanes) {
                float* x1 = p.x1 + (q * Wp + rg * 8) * Dp + 4 * dq;
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    *reinterpret_cast<float4*>(x1 + static_cast<int64_t>(i) * Dp) =
                        make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
            }
        }
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
                const float a = e4m3_decode_fast(static_cast<const uint8_t*>(hin)[base + k * P]);
#pragma unroll
                for (int o4 = 0; o4 < C / 4; ++o4) {
                    const float4 w = sW4[k * (C / 4) + o4];
                    // two rounded products per f32x2 instruction, each sum a scalar add
                    const float2 m0 = mul2_rn(make_float2(a, a), make_float2(w.x, w.y));
                    const float2 m1 = mul2_rn(make_float2(a, a), make_float2(w.z, w.w));
                    acc[4 * o4 + 0] = __fadd_rn(acc[4 * o4 + 0], m0.x);
                    acc[4 * o4 + 1] = __fadd_rn(acc[4 * o4 + 1], m0.y);
                    acc[4 * o4 + 2] = __fadd_rn(acc[4 * o4 + 2], m1.x);
                    acc[4 * o4 + 3] = __fadd_rn(acc[4 * o4 + 3], m1.y);
                }
            }
        } else {
#pragma unroll
            for (int o = 0; o < C; ++o) acc[o] = sB[o];
            // the inputs of eight channels loaded before their products (the loads of
            // a group are in flight together)
            constexpr int KB = C % 8 == 0 ? 8 : 1;
            for (int k0 = 0; k0 < C; k0 += KB) {
                float av[KB];
#pragma unroll
                for (int kk = 0; kk < KB; ++kk) av[kk] = static_cast<const float*>(hin)[base + (k0 + kk) * P];
#pragma unroll
                for (int kk = 0; kk < KB; ++kk) {
                    const int k = k0 + kk;
                    const float a = av[kk];
                    const bool fused = k >= nu;
#pragma unroll
                    for (int o4 = 0; o4 < C / 4; ++o4) {
                        const float4 w = sW4[k * (C / 4) + o4];
                        if (nu >= C) {
                            // every product unfused: two per f32x2 instruction
                            const float2 m0 = mul2_rn(make_float2(a, a), make_float2(w.x, w.y));
                            const float2 m1 = mul2_rn(make_float2(a, a), make_float2(w.z, w.w));
                            acc[4 * o4 + 0] = __fadd_rn(acc[4 * o4 + 0], m0.x);
                            acc[4 * o4 + 1] = __fadd_rn(acc[4 * o4 + 1], m0.y);
                            acc[4 * o4 + 2] = __fadd_rn(acc[4 * o4 + 2], m1.x);
                            acc[4 * o4 + 3] = __fadd_rn(acc[4 * o4 + 3], m1.y);
                        } else {
                            acc[4 * o4 + 0] = linear_step(acc[4 * o4 + 0], a, w.x, fused);
                            acc[4 * o4 + 1] = linear_step(acc[4 * o4 + 1], a, w.y, fused);
                            acc[4 * o4 + 2] = linear_step(acc[4 * o4 + 2], a, w.z, fused);
                            acc[4 * o4 + 3] = linear_step(acc[4 * o4 + 3], a, w.w, fused);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int o = 0; o < C; ++o) {
            float x2 = acc[o];
            if (p.fp8) x2 = fp8_fake_quant_inner(__fadd_rn(__fmul_rn(x2, sc), sB[o]), L.s_out, inv_out);
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
    static constexpr int kOffPo = kOffBias + C * 4;         // projection: proj_out (16 x C) + bias
    static constexpr int kOffBars = kOffPo + (16 * C + 16) * 4;
    static constexpr int kNumBars = 2 * kStages + 2 * kAccStages;
    static constexpr int kSmemBytes = kOffBars + 8 * kNumBars + 16 + 1024;
};

// PROJ: the same tiles and MMA for the projection (proj3d_kernel's FP8 arithmetic):
// weights proj_q, per point q_c = fake-quant(D_c s + b_c), the activation, then
// proj_out summed over c in order (Linear rounding) and fake-quantised into y at the
// unpadded points.  `s_in` is the scale of the input codes.
template <int C, bool PROJ>
__global__ void __launch_bounds__(L3Cfg<C>::kThreads, 1)
local3d_tc_kernel(const __grid_constant__ CUtensorMap tmIn, const Fno3dPlan p, const Fno3dLayer L, float s_in,
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
            sW[swz_offset(o * C + k, C)] = static_cast<uint8_t>(e4m3_encode_ref(PROJ ? p.pq_q[i] : L.loc_q[i]));
        }
        for (int o = threadIdx.x; o < C; o += F::kThreads) sBias[o] = PROJ ? p.pq_b[o] : L.loc_b[o];
        if constexpr (PROJ) {
            float* sPo = reinterpret_cast<float*>(smem + F::kOffPo);
            for (int i = threadIdx.x; i < p.out_ch * C; i += F::kThreads) sPo[i] = p.po_w[i];
            for (int i = threadIdx.x; i < p.out_ch; i += F::kThreads) sPo[16 * C + i] = p.po_b[i];
        }
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
        const float sc = __fmul_rn(s_in, PROJ ? p.s_pq_w : L.s_w);
        const float s_out = PROJ ? p.s_pq : L.s_out;
        const float inv_out = inv_of(s_out);
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
            if constexpr (PROJ) {
                const float* sPo = reinterpret_cast<const float*>(smem + F::kOffPo);
                constexpr int nu = linear_unfused_len(C);
                float yo[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) yo[j] = j < p.out_ch ? sPo[16 * C + j] : 0.0f;
#pragma unroll 1
                for (int h = 0; h < C / 32; ++h) {
                    uint32_t acc[32];
                    tmem_ld32(tbase + 32 * h, acc);
                    tmem_wait_ld();
                    if (h == C / 32 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&accEmpty[grp]);
                    }
                    if (p.out_ch == 1) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int c = 32 * h + j;
                            const float q = fp8_fake_quant_inner(__fadd_rn(__fmul_rn(__uint_as_float(acc[j]), sc), sBias[c]),
                                                           s_out, inv_out);
                            yo[0] = linear_step(yo[0], act_f(q, p.act), sPo[c], c >= nu);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int c = 32 * h + j;
                            const float q = fp8_fake_quant_inner(__fadd_rn(__fmul_rn(__uint_as_float(acc[j]), sc), sBias[c]),
                                                           s_out, inv_out);
                            const float g = act_f(q, p.act);
#pragma unroll
                            for (int o = 0; o < 16; ++o)
                                if (o < p.out_ch) yo[o] = linear_step(yo[o], g, sPo[o * C + c], c >= nu);
                        }
                    }
                }
                // the padded grid's points outside the input grid carry no output
                const int lgD = 31 - __clz(p.Dp), lgW = 31 - __clz(p.Wp);
                const int ip = static_cast<int>(pt);
                const int dd = ip & (p.Dp - 1), ww = (ip >> lgD) & (p.Wp - 1), hh = ip >> (lgD + lgW);
                if (hh < p.H && ww < p.W && dd < p.D) {
                    const float inv_po = inv_of(p.s_po);
                    float* yr = p.y + (((static_cast<int64_t>(b) * p.H + hh) * p.W + ww) * p.D + dd) * p.out_ch;
#pragma unroll
                    for (int o = 0; o < 16; ++o)
                        if (o < p.out_ch) yr[o] = fp8_fake_quant(yo[o], p.s_po, inv_po);
                }
                continue;
            }
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
                    const float x2 = fp8_fake_quant_inner(__fadd_rn(__fmul_rn(__uint_as_float(acc[j]), sc), sBias[o]),
                                                    s_out, inv_out);
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

// x = hi + lo with hi holding the upper tf32 bits (rounded half away in magnitude) and
// lo the exact remainder, which a tf32 MMA reads to about 2^-11 of itself
__device__ __forceinline__ void split_tf32_x3(float x, float& hi, float& lo) {
    hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
    lo = __fsub_rn(x, hi);
}

// ---------------------------------------------------------------------------
// layer3d_tc: one whole FP8 layer after the spectral mix -- the W and D inverse
// transforms fused into the tensor-core local layer (fno3d_fused_layer geometries:
// widths 32 / 64, Dp = 64 or 128, at most 8 kept kw and kd modes), so the spectral
// branch x1 never leaves the chip.  A 128-point tile is R = 128 / Dp rows w of one
// (b, h) plane.  With
//   U[o][r][2 kd]     =  f_kd Re s,  U[o][r][2 kd + 1] = -f_kd Im s,
//   s = sum_kw colinv[b][o][h][kw][kd] e^{+2 pi i kw (w0 + r) / Wp},
//   f_kd = (kd = 0 or 2 kd = Dp ? 1 : 2) / (Wp Dp),
//   Binv[p][16 r' + 2 kd] = [r' = p / Dp] cos(2 pi kd d / Dp), ... + 1 = ... sin,
// x1[p][o] = sum_k Binv[p][k] U[o][k] over K = 32 (16 per row slot, zeros for absent
// rows and modes) is a kind::tf32 MMA, 3xTF32 (hi.hi + lo.hi + hi.lo, each operand
// split into tf32 hi and the remainder lo).  It lands beside the local layer's
// accumulator, and the epilogue reads both from TMEM.
//   warp 0       TMA producer of the layer-input code tiles
//   warp 1       MMA issuer: the E4M3 local GEMM and the x1 MMAs per tile
//   warps 2..    T builders (4 threads per output channel, 2 kd modes each): U of each
//                tile from the plane's colinv entries, held in registers while (b, h)
//                stays the same; four U buffers
//   then         epilogue: three groups of four warps (one per TMEM lane quadrant)
//                take turns over the tiles; per element as local3d_tc with x1 from TMEM
// ---------------------------------------------------------------------------
template <int C>
struct X3Cfg {
    static constexpr int kTb0 = 2;
    static constexpr int kTbWarps = C / 8;                 // 4 C threads
    static constexpr int kEpi0 = kTb0 + kTbWarps;
    static constexpr int kGroups = 3;
    static constexpr int kEpiWarps = 4 * kGroups;
    static constexpr int kThreads = 32 * (kEpi0 + kEpiWarps);
    static constexpr int kStages = 6;
    static constexpr int kABytes = 128 * C;               // two [C][64] boxes
    static constexpr int kAccStages = kGroups;
    static constexpr int kAccCols = 2 * C;                // local accumulator, then x1
    static constexpr int kTmemCols = kAccStages * kAccCols <= 256 ? 256 : 512;
    static constexpr int kTBufs = 4;
    static constexpr int kBinvBlk = 128 * 128;            // [128 points][32 fp32], 128-byte swizzle
    static constexpr int kUBlk = C * 128;                 // [C][32 fp32]
    static constexpr int kOffA = 0;
    static constexpr int kOffW = kOffA + kStages * kABytes;
    static constexpr int kOffBinv = kOffW + ((C * C + 1023) / 1024) * 1024;
    static constexpr int kOffU = kOffBinv + 2 * kBinvBlk;                 // hi, lo
    static constexpr int kOffBias = kOffU + kTBufs * 2 * kUBlk;           // hi, lo per buffer
    static constexpr int kOffTw = kOffBias + C * 4;                       // [Wp][8] float2 (Wp <= 128)
    static constexpr int kOffBars = kOffTw + 128 * 8 * 8;
    static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 2 * kTBufs;
    static constexpr int kSmemBytes = kOffBars + 8 * kNumBars + 16 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "smem");
};

bool fno3d_fused_layer_ok(int C, int Wp, int Dp, int MW, int MD) {
    return (C == 32 || C == 64) && (Dp == 64 || Dp == 128) && Wp <= 128 && MW <= 8 && MD <= 8;
}

template <int C>
__global__ void __launch_bounds__(X3Cfg<C>::kThreads, 1)
layer3d_tc_kernel(const __grid_constant__ CUtensorMap tmIn, const Fno3dPlan p, const Fno3dLayer L, DftDims g,
                  uint8_t* __restrict__ hout, unsigned* err) {
    using F = X3Cfg<C>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem + F::kOffA;
    uint8_t* sW = smem + F::kOffW;
    uint8_t* sBinv = smem + F::kOffBinv;
    uint8_t* sU = smem + F::kOffU;
    float* sBias = reinterpret_cast<float*>(smem + F::kOffBias);
    float2* sTw = reinterpret_cast<float2*>(smem + F::kOffTw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + F::kOffBars);
    uint64_t* empty = full + F::kStages;
    uint64_t* accFull = empty + F::kStages;
    uint64_t* accEmpty = accFull + F::kAccStages;
    uint64_t* tReady = accEmpty + F::kAccStages;
    uint64_t* tFree = tReady + F::kTBufs;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(tFree + F::kTBufs);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int Wp = p.Wp, Dp = p.Dp, MW = p.MW, MD = p.MD;
    const int64_t Pp = static_cast<int64_t>(p.Hp) * Wp * Dp;
    const int tiles_per_sample = static_cast<int>(Pp / 128);
    const int num_tiles = p.B * tiles_per_sample;
    const int t_begin = static_cast<int>(static_cast<int64_t>(num_tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(num_tiles) * (blockIdx.x + 1) / gridDim.x);

    {
        for (int i = threadIdx.x; i < C * C; i += F::kThreads) {
            const int o = i / C, k = i % C;
            sW[swz_offset(o * C + k, C)] = static_cast<uint8_t>(e4m3_encode_ref(L.loc_q[i]));
        }
        for (int o = threadIdx.x; o < C; o += F::kThreads) sBias[o] = L.loc_b[o];
        // W twiddles e^{-2 pi i kw w / Wp} (the DFT table's [Wp][MW2] block), kw < 8
        {
            const float2* gW = reinterpret_cast<const float2*>(p.dft + 2 * Dp * g.MD4);
            for (int i = threadIdx.x; i < Wp * 8; i += F::kThreads) {
                const int w = i >> 3, kw = i & 7;
                sTw[i] = kw < MW ? gW[w * g.MW2 + kw] : make_float2(0.0f, 0.0f);
            }
        }
        // Binv hi / lo: point p = r' Dp + d, column 16 r' + 2 kd (+1)
        {
            const float* iC = p.dft + 2 * Dp * g.MD4 + 2 * Wp * g.MW2;
            const float* iS = iC + g.MD4 * Dp;
            for (int i = threadIdx.x; i < 128 * 32; i += F::kThreads) {
                const int pt = i >> 5, k = i & 31;
                const int r = k >> 4, j = k & 15, kd = j >> 1;
                float v = 0.0f;
                if (r == pt / Dp && kd < MD) v = (j & 1) ? iS[kd * Dp + pt % Dp] : iC[kd * Dp + pt % Dp];
                float hi, lo;
                split_tf32_x3(v, hi, lo);
                const uint32_t o = swz_offset(static_cast<uint32_t>(pt * 128 + k * 4), 128);
                *reinterpret_cast<float*>(sBinv + o) = hi;
                *reinterpret_cast<float*>(sBinv + F::kBinvBlk + o) = lo;
            }
        }
        // U buffers start zero: the builders write only present rows and modes
        for (int i = threadIdx.x; i < F::kTBufs * 2 * F::kUBlk / 16; i += F::kThreads)
            reinterpret_cast<uint4*>(sU)[i] = make_uint4(0u, 0u, 0u, 0u);
        if (threadIdx.x == 0) {
            for (int s = 0; s < F::kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < F::kAccStages; ++s) {
                mbar_init(&accFull[s], 1);
                mbar_init(&accEmpty[s], 4);
            }
            for (int b = 0; b < F::kTBufs; ++b) {
                mbar_init(&tReady[b], F::kTbWarps * 32);
                mbar_init(&tFree[b], 1);
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
            constexpr uint32_t idesc8 = idesc_e4m3(C) | (1u << 15);  // A MN-major
            constexpr uint32_t idesc32 = idesc_tf32(C);
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % F::kStages;
                const uint32_t ph = (it / F::kStages) & 1;
                const int a = it % F::kAccStages;
                const uint32_t aph = (it / F::kAccStages) & 1;
                const int tb = it % F::kTBufs;
                if (!mbar_wait_backoff(&accEmpty[a], aph ^ 1, sAbort, 128) ||
                    !mbar_wait_backoff(&full[s], ph, sAbort, 128) ||
                    !mbar_wait_backoff(&tReady[tb], (it / F::kTBufs) & 1, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(err, kErrWaitTmaFull);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + a * F::kAccCols;
                const uint32_t aBase = smem_u32(sA + s * F::kABytes);
#pragma unroll
                for (int kk = 0; kk < C / 32; ++kk)
                    mma_f8(d, umma_desc_mn_sw64(aBase + kk * 2048, F::kABytes / 2, 512),
                           umma_desc(smem_u32(sW) + kk * 32, C), idesc8, kk > 0 ? 1u : 0u);
                const uint32_t bhi = smem_u32(sBinv), blo = bhi + F::kBinvBlk;
                const uint32_t uhi = smem_u32(sU) + tb * 2 * F::kUBlk, ulo = uhi + F::kUBlk;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_tf32(d + C, umma_desc(bhi + kk * 32, 128), umma_desc(uhi + kk * 32, 128), idesc32,
                             kk > 0 ? 1u : 0u);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_tf32(d + C, umma_desc(blo + kk * 32, 128), umma_desc(uhi + kk * 32, 128), idesc32, 1u);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_tf32(d + C, umma_desc(bhi + kk * 32, 128), umma_desc(ulo + kk * 32, 128), idesc32, 1u);
                mma_commit(&empty[s]);
                mma_commit(&accFull[a]);
                mma_commit(&tFree[tb]);
            }
            if (it > 0) {
                const int j = it - 1;
                if (!mbar_wait_drain(&accFull[j % F::kAccStages], (j / F::kAccStages) & 1))
                    atomicOr(err, kErrWaitDrain);
            }
        }
        __syncwarp();
    } else if (warp < F::kEpi0) {
        // ---------------- T builders: thread (o, q) owns kd = 2q, 2q + 1 of channel o
        const int ctid = (warp - F::kTb0) * 32 + lane;
        const int o = ctid % C, q = ctid / C;
        const int R = 128 / Dp;
        const float unit = __fdiv_rn(1.0f, static_cast<float>(Wp) * static_cast<float>(Dp));
        float f[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int kd = 2 * q + e;
            f[e] = (kd == 0 || 2 * kd == Dp) ? unit : __fmul_rn(2.0f, unit);
        }
        float2 ci[8][2];
        int cached = -1;
        int it = 0;
        for (int tile = t_begin; tile < t_end; ++tile, ++it) {
            const int b = tile / tiles_per_sample;
            const int pt0 = (tile - b * tiles_per_sample) * 128;
            const int h = pt0 / (Wp * Dp);
            const int w0 = (pt0 / Dp) % Wp;
            const int plane = b * p.Hp + h;
            if (plane != cached) {
                const float2* src = p.colinv + ((static_cast<int64_t>(b) * C + o) * p.Hp + h) * (MW * MD);
#pragma unroll
                for (int kw = 0; kw < 8; ++kw)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int kd = 2 * q + e;
                        ci[kw][e] = (kw < MW && kd < MD) ? __ldg(src + kw * MD + kd) : make_float2(0.0f, 0.0f);
                    }
                cached = plane;
            }
            const int tb = it % F::kTBufs;
            if (!mbar_wait_backoff(&tFree[tb], ((it / F::kTBufs) & 1) ^ 1, sAbort, 256)) {
                *sAbort = 1;
                atomicOr(err, kErrWaitSlotFree);
                break;
            }
            uint8_t* uhi = sU + tb * 2 * F::kUBlk;
            for (int r = 0; r < R; ++r) {
                const float2* tw = sTw + (w0 + r) * 8;
                float sr[2] = {0.0f, 0.0f}, si[2] = {0.0f, 0.0f};
#pragma unroll
                for (int kw = 0; kw < 8; ++kw) {
                    const float2 t = tw[kw];  // e^{-i theta}; e^{+i theta} = (t.x, -t.y)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        sr[e] = __fmaf_rn(ci[kw][e].x, t.x, sr[e]);
                        sr[e] = __fmaf_rn(ci[kw][e].y, t.y, sr[e]);
                        si[e] = __fmaf_rn(ci[kw][e].y, t.x, si[e]);
                        si[e] = __fmaf_rn(-ci[kw][e].x, t.y, si[e]);
                    }
                }
                float v[4] = {__fmul_rn(sr[0], f[0]), -__fmul_rn(si[0], f[0]), __fmul_rn(sr[1], f[1]),
                              -__fmul_rn(si[1], f[1])};
                float hi[4], lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) split_tf32_x3(v[e], hi[e], lo[e]);
                const uint32_t off = swz_offset(static_cast<uint32_t>(o * 128 + (16 * r + 4 * q) * 4), 128);
                *reinterpret_cast<float4*>(uhi + off) = make_float4(hi[0], hi[1], hi[2], hi[3]);
                *reinterpret_cast<float4*>(uhi + F::kUBlk + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
            }
            fence_proxy_async_smem();
            mbar_arrive(&tReady[tb]);
        }
    } else {
        const int ew = warp - F::kEpi0;
        const int quad = warp & 3;
        const int grp = ew >> 2;
        const float sc = __fmul_rn(L.s_in, L.s_w);
        const float inv_out = inv_of(L.s_out);
        for (int it = grp; t_begin + it < t_end; it += F::kGroups) {
            const int tile = t_begin + it;
            const int a = it % F::kAccStages;
            const uint32_t aph = (it / F::kAccStages) & 1;
            if (!mbar_wait(&accFull[a], aph, sAbort)) {
                *sAbort = 1;
                atomicOr(err, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            const int b = tile / tiles_per_sample;
            const int64_t pt = static_cast<int64_t>(tile - b * tiles_per_sample) * 128 + quad * 32 + lane;
            const int64_t base = static_cast<int64_t>(b) * C * Pp + pt;
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + a * F::kAccCols;
#pragma unroll 1
            for (int hc = 0; hc < C / 32; ++hc) {
                uint32_t acc[32], x1r[32];
                tmem_ld32(tbase + 32 * hc, acc);
                tmem_ld32(tbase + C + 32 * hc, x1r);
                tmem_wait_ld();
                if (hc == C / 32 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&accEmpty[a]);
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int oc = 32 * hc + j;
                    const float x2 = fp8_fake_quant_inner(__fadd_rn(__fmul_rn(__uint_as_float(acc[j]), sc), sBias[oc]),
                                                    L.s_out, inv_out);
                    const float z = act_f(__fadd_rn(__uint_as_float(x1r[j]), x2), p.act);
                    hout[base + static_cast<int64_t>(oc) * Pp] = static_cast<uint8_t>(e4m3_code(z, inv_out));
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
    __shared__ float4 sQ4[C * C / 4];  // [c][k]: 16-byte broadcast loads over k
    const float* qsrc = p.fp8 ? p.pq_q : p.pq_w;
    float* sQ = reinterpret_cast<float*>(sQ4);
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
            if (p.fp8) a[k] = e4m3_decode_fast(static_cast<const uint8_t*>(hin)[base + k * Pp]);
            else a[k] = static_cast<const float*>(hin)[base + k * Pp];
        }
        float qv[C];
#pragma unroll
        for (int c = 0; c < C; ++c) {
            float q = p.fp8 ? 0.0f : __ldg(p.pq_b + c);
#pragma unroll
            for (int k4 = 0; k4 < C / 4; ++k4) {
                const float4 w = sQ4[c * (C / 4) + k4];
                const float ww4[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int k = 4 * k4 + m;
                    q = p.fp8 ? __fadd_rn(q, __fmul_rn(a[k], ww4[m])) : linear_step(q, a[k], ww4[m], k >= nu);
                }
            }
            if (p.fp8) q = fp8_fake_quant_inner(__fadd_rn(__fmul_rn(q, sc), __ldg(p.pq_b + c)), p.s_pq, inv_pq);
            qv[c] = act_f(q, p.act);
        }
        float* yr = p.y + t * p.out_ch;
        for (int j = 0; j < p.out_ch; ++j) {
            float acc = __ldg(p.po_b + j);
            const float* wj = p.po_w + static_cast<int64_t>(j) * C;
#pragma unroll
            for (int c = 0; c < C; ++c) acc = linear_step(acc, qv[c], __ldg(wj + c), c >= nu);
            yr[j] = p.fp8 ? fp8_fake_quant(acc, p.s_po, inv_po) : acc;
        }
    }
}

// output channels per mix3d CTA: at most 8, fewer while the grid would leave SMs idle
int mix_group(int C, int64_t B = 0, int sms = 0) {
    int G = 1;
    for (int g = 8; g > 1; g >>= 1)
        if (C % g == 0) {
            G = g;
            break;
        }
    while (G > 1 && static_cast<int64_t>(C / G) * B < 2 * static_cast<int64_t>(sms)) G >>= 1;
    return G;
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
    const bool lift4 = p.Dp % 4 == 0 && p.in_ch >= 1 && p.in_ch <= 8;
    const int64_t tl = static_cast<int64_t>(p.B) * Pp / (lift4 ? 4 : 1);
    if ((e = timed("fno3d_lift", [&] {
             const int grid = static_cast<int>(std::min<int64_t>((tl + 255) / 256, sms * 16));
             if (lift4) {
                 switch (p.in_ch) {
                     case 1: lift3d_x4_kernel<1><<<grid, 256, 0, st>>>(p); break;
                     case 2: lift3d_x4_kernel<2><<<grid, 256, 0, st>>>(p); break;
                     case 3: lift3d_x4_kernel<3><<<grid, 256, 0, st>>>(p); break;
                     case 4: lift3d_x4_kernel<4><<<grid, 256, 0, st>>>(p); break;
                     case 5: lift3d_x4_kernel<5><<<grid, 256, 0, st>>>(p); break;
                     case 6: lift3d_x4_kernel<6><<<grid, 256, 0, st>>>(p); break;
                     case 7: lift3d_x4_kernel<7><<<grid, 256, 0, st>>>(p); break;
                     default: lift3d_x4_kernel<8><<<grid, 256, 0, st>>>(p); break;
                 }
             }
             else lift3d_kernel<<<grid, 256, 0, st>>>(p);
         })) != cudaSuccess)
        return e;
    const int KK = p.MW * p.MD, M = p.MH * KK, G = mix_group(p.C, p.B, sms);
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
    const bool direct = p.dft != nullptr;
    const DftDims g = dft_dims(p.Wp, p.Dp, p.MW, p.MD);
    const size_t sdf = dft_fwd_smem(g, p.Wp, p.Dp), sdi = dft_inv_smem(g, p.Wp, p.Dp, p.MW);
    int gdf = 0, gdi = 0;
    const bool ftc = direct && fwd_tc_ok(p.Wp, p.Dp, p.MD);
    const bool fused = direct && fno3d_fused_layer_ok(p.C, p.Wp, p.Dp, p.MW, p.MD);
    const FtcDims fd = ftc_dims(g, p.Wp, p.Dp);
    unsigned* err = device_error_word();
    if (ftc && !err) return cudaErrorMemoryAllocation;
    if (direct) {
        if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(fwd3d_dft_kernel), static_cast<int>(sdf))) !=
                cudaSuccess ||
            (e = set_max_dynamic_smem(reinterpret_cast<const void*>(inv3d_dft_kernel), static_cast<int>(sdi))) !=
                cudaSuccess)
            return e;
        int of = 0, oi = 0;
        if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&of, fwd3d_dft_kernel, kDftThreads, sdf)) !=
                cudaSuccess ||
            (e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&oi, inv3d_dft_kernel, kDftThreads, sdi)) !=
                cudaSuccess)
            return e;
        const int64_t planes = static_cast<int64_t>(p.B) * p.C * p.Hp;
        gdf = static_cast<int>(std::min<int64_t>((planes + g.NPf - 1) / g.NPf, static_cast<int64_t>(sms) * std::max(1, of)));
        if (ftc) {
            if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(fwd3d_tc_kernel), fd.smem)) != cudaSuccess)
                return e;
            // CTAs per SM from the shared memory (227 KB per SM; TMEM: 32 columns each)
            const int per_sm = std::max(1, std::min(8, (227 * 1024) / (fd.smem + 1024)));
            gdf = static_cast<int>(std::min<int64_t>(planes / fd.NPt, static_cast<int64_t>(sms) * per_sm));
        }
        gdi = static_cast<int>(std::min<int64_t>((planes + g.NPi - 1) / g.NPi, static_cast<int64_t>(sms) * std::max(1, oi)));
    }
    const int64_t tp = static_cast<int64_t>(p.B) * Pp;
    const int lgrid = static_cast<int>(std::min<int64_t>((tp + 127) / 128, sms * 16));
    const size_t tap_bytes = static_cast<size_t>(p.B) * C * Pp;
    for (int i = 0; i <= p.L; ++i) {
        if (p.tap_codes && p.fp8 &&
            (e = cudaMemcpyAsync(p.tap_codes + static_cast<size_t>(i) * tap_bytes, p.h[i & 1], tap_bytes,
                                 cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
            return e;
        if (i == p.L) break;
        const Fno3dLayer& L = p.layer[i];
        const void* hin = p.h[i & 1];
        void* hout = p.h[(i + 1) & 1];
        if ((e = timed("fno3d_fwd", [&] {
                 if (ftc)
                     fwd3d_tc_kernel<<<gdf, 128, fd.smem, st>>>(p, g, fd, static_cast<const uint8_t*>(hin), L.s_in, err);
                 else if (direct)
                     fwd3d_dft_kernel<<<gdf, kDftThreads, sdf, st>>>(p, g, static_cast<const uint8_t*>(hin), L.s_in);
                 else
                     fwd3d_a_kernel<<<dim3(p.Hp, p.C, p.B), 256, sa, st>>>(p, hin, L.s_in);
                 fwd3d_b_kernel<<<dim3(p.C, p.B), 256, sb, st>>>(p);
             })) != cudaSuccess)
            return e;
        if ((e = timed("fno3d_mix", [&] {
                 mix3d_kernel<<<dim3(p.C / G, p.B), 256, sx, st>>>(p, L.wr, L.wi, G);
             })) != cudaSuccess)
            return e;
        bool tc = false;
        if constexpr (C == 32 || C == 64) {
            // FP8, direct DFT geometries: inverse transforms fused into the local layer
            if (fused) {
                using F = X3Cfg<C>;
                CUtensorMap tm;
                if (!err) return cudaErrorMemoryAllocation;
                if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, hin, static_cast<uint64_t>(Pp),
                               static_cast<uint64_t>(p.B) * C, static_cast<uint64_t>(Pp), 64, C, 64))
                    return cudaErrorInvalidValue;
                auto k = layer3d_tc_kernel<C>;
                if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(k), F::kSmemBytes)) != cudaSuccess)
                    return e;
                const int64_t tiles = static_cast<int64_t>(p.B) * (Pp / 128);
                const int grid = static_cast<int>(std::min<int64_t>(tiles, sms));
                if ((e = timed("fno3d_local", [&] {
                         k<<<grid, F::kThreads, F::kSmemBytes, st>>>(tm, p, L, g, static_cast<uint8_t*>(hout), err);
                     })) != cudaSuccess)
                    return e;
                continue;
            }
        }
        if ((e = timed("fno3d_inv", [&] {
                 if (direct) inv3d_dft_kernel<<<gdi, kDftThreads, sdi, st>>>(p, g);
                 else inv3d_kernel<<<dim3(p.Hp, p.C, p.B), 256, si, st>>>(p);
             })) != cudaSuccess)
            return e;
        if constexpr (C == 32 || C == 64) {
            // FP8: the local layer on tensor cores when a sample is whole 128-point tiles
            if (p.fp8 && Pp % 128 == 0) {
                using F = L3Cfg<C>;
                CUtensorMap tm;
                if (!err) return cudaErrorMemoryAllocation;
                if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, hin, static_cast<uint64_t>(Pp),
                               static_cast<uint64_t>(p.B) * C, static_cast<uint64_t>(Pp), 64, C, 64))
                    return cudaErrorInvalidValue;
                auto k = local3d_tc_kernel<C, false>;
                if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(k), F::kSmemBytes)) != cudaSuccess)
                    return e;
                const int64_t tiles = static_cast<int64_t>(p.B) * (Pp / 128);
                const int grid = static_cast<int>(std::min<int64_t>(tiles, sms));
                if ((e = timed("fno3d_local", [&] {
                         k<<<grid, F::kThreads, F::kSmemBytes, st>>>(tm, p, L, L.s_in, static_cast<uint8_t*>(hout),
                                                                     err);
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
    if constexpr (C == 32 || C == 64) {
        // FP8: the projection on tensor cores (the local layer's tiles and MMA)
        if (p.fp8 && Pp % 128 == 0) {
            using F = L3Cfg<C>;
            CUtensorMap tm;
            if (!err) return cudaErrorMemoryAllocation;
            if (!encode_2d(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.h[p.L & 1], static_cast<uint64_t>(Pp),
                           static_cast<uint64_t>(p.B) * C, static_cast<uint64_t>(Pp), 64, C, 64))
                return cudaErrorInvalidValue;
            auto k = local3d_tc_kernel<C, true>;
            if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(k), F::kSmemBytes)) != cudaSuccess) return e;
            const int64_t tiles = static_cast<int64_t>(p.B) * (Pp / 128);
            const int grid = static_cast<int>(std::min<int64_t>(tiles, sms));
            return timed("fno3d_proj", [&] {
                k<<<grid, F::kThreads, F::kSmemBytes, st>>>(tm, p, p.layer[0], s_last, nullptr, err);
            });
        }
    }
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

bool fno3d_direct_dft(int C, int fp8, int Wp, int Dp, int MW, int MD) {
    if (!fp8 || (C != 32 && C != 64)) return false;
    if (Dp % 16 != 0 || Wp % 8 != 0 || static_cast<int64_t>(Wp) * Dp > kDftPre * kDftThreads * 16) return false;
    const DftDims g = dft_dims(Wp, Dp, MW, MD);
    return dft_fwd_smem(g, Wp, Dp) <= 200 * 1024 && dft_inv_smem(g, Wp, Dp, MW) <= 200 * 1024;
}

std::vector<float> fno3d_dft_tables(int Wp, int Dp, int MW, int MD) {
    const DftDims g = dft_dims(Wp, Dp, MW, MD);
    const double two_pi = 6.283185307179586476925286766559;
    std::vector<float> t(2 * static_cast<size_t>(Dp) * g.MD4 + 2 * static_cast<size_t>(Wp) * g.MW2 +
                             2 * static_cast<size_t>(g.MD4) * Dp,
                         0.0f);
    float* fD = t.data();
    float* fW = fD + 2 * static_cast<size_t>(Dp) * g.MD4;
    float* iC = fW + 2 * static_cast<size_t>(Wp) * g.MW2;
    float* iS = iC + static_cast<size_t>(g.MD4) * Dp;
    for (int d = 0; d < Dp; ++d)
        for (int k = 0; k < MD; ++k) {
            const double a = two_pi * static_cast<double>((static_cast<int64_t>(k) * d) % Dp) / Dp;
            fD[2 * (static_cast<size_t>(d) * g.MD4 + k)] = static_cast<float>(std::cos(a));
            fD[2 * (static_cast<size_t>(d) * g.MD4 + k) + 1] = static_cast<float>(-std::sin(a));
            iC[static_cast<size_t>(k) * Dp + d] = static_cast<float>(std::cos(a));
            iS[static_cast<size_t>(k) * Dp + d] = static_cast<float>(std::sin(a));
        }
    for (int w = 0; w < Wp; ++w)
        for (int k = 0; k < MW; ++k) {
            const double a = two_pi * static_cast<double>((static_cast<int64_t>(k) * w) % Wp) / Wp;
            fW[2 * (static_cast<size_t>(w) * g.MW2 + k)] = static_cast<float>(std::cos(a));
            fW[2 * (static_cast<size_t>(w) * g.MW2 + k) + 1] = static_cast<float>(-std::sin(a));
        }
    return t;
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
