// fno1d.cu -- FNO1d executor (sm_100a): the reference FNO1d::Forward
// (cpp/src/fno.cpp:408-706) with the reference's rounding.
//
// Activations between layers stay channel-last (b, p, c) in HBM, as int8 codes when the
// next layer snaps its input with per-tensor qparams (the snap is then exact and free:
// the previous layer's epilogue emits the code through the host-built z -> code table)
// and as fp32 otherwise.  One layer is
//
//   fft1d_fwd   per (b, c) row: the reference radix-2 rFFT (fft.cpp:73-84) of the
//               layer input, bit-identical, truncated to `modes` bins -> Xs (b, c, m)
//   [gemm_i8]   INT8 path only: tcgen05 LinearForwardBatched of the input codes
//               (fno.cpp:125-159) -> x2raw (b*N, C); widths the GEMM does not tile
//               (not 32/64/128/256) compute the same integers inside layer1d
//   layer1d     per (b, group of G output channels): the spectral contraction
//               (fno.cpp:181-196), the inverse transform (fft.cpp:86-99) of each
//               output row, the local Linear (FP32 dot product, or x2raw + bias), the
//               output fake-quant, x1 + x2 and the activation -> next activation
//
// lift1d (fno.cpp:438-466) and proj1d (fno.cpp:683-702) close the network.  The only
// operation that is not bit-identical to the reference is tanhf inside GELU where its
// result is consumed as fp32 (CUDA's tanhf vs glibc's differ by at most a few ulps);
// wherever GELU feeds a per-tensor snap the exact table is used instead.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "fft_exact.cuh"
#include "fno1d.h"
#include "nfx_internal.h"
#include "numerics.cuh"

namespace nfx {
namespace {

__device__ __forceinline__ float act_f(float z, int act) {
    return act == 1 ? relu_ref(z) : gelu_tanh(z);
}

// value of activation element idx: a code snapped back, (q - zp) * s, or the fp32 value
__device__ __forceinline__ float act_value(const void* h, int64_t idx, int codes, float s,
                                           float zpf) {
    if (codes)
        return __fmul_rn(__fsub_rn(static_cast<float>(static_cast<const int8_t*>(h)[idx]), zpf), s);
    return static_cast<const float*>(h)[idx];
}

// ---------------------------------------------------------------------------
// lift: h[b, p, c] = Linear from lift_b[c] over x[b, p, :] (fno.cpp:51-80); zero in
// the padded tail (fno.cpp:450-466); then the layer-0 snap as a code, when it exists.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) lift1d_kernel(const float* __restrict__ x, int n, int N,
                                                     int C, int in_ch, int64_t total,
                                                     const float* __restrict__ w,
                                                     const float* __restrict__ bias, int codes,
                                                     float s, int zp, void* out) {
    const float zpf = static_cast<float>(zp);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int c = static_cast<int>(t % C);
        const int64_t bp = t / C;
        const int p = static_cast<int>(bp % N);
        const int64_t b = bp / N;
        float acc = 0.0f;
        if (p < n) {
            acc = __ldg(bias + c);
            const float* xr = x + (b * n + p) * in_ch;
            const int nu = linear_unfused_len(in_ch);
            for (int k = 0; k < in_ch; ++k)
                acc = linear_step(acc, __ldg(xr + k), __ldg(w + c * in_ch + k), k >= nu);
        }
        if (codes)
            static_cast<int8_t*>(out)[t] = static_cast<int8_t>(static_cast<int>(fq_code(acc, s, zpf)));
        else
            static_cast<float*>(out)[t] = acc;
    }
}

// ---------------------------------------------------------------------------
// forward transform: grid (C / R, B), R warps, one row (b, c) per warp.
// Dynamic shared memory R * N float2.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fft1d_fwd_kernel(const void* __restrict__ h, int codes,
                                                        float s, int zp, int N, int log2N, int C,
                                                        int modes,
                                                        const float2* __restrict__ tw,
                                                        float2* __restrict__ Xs) {
    extern __shared__ float2 sa[];
    const int R = blockDim.x >> 5;
    const int b = blockIdx.y, c0 = blockIdx.x * R;
    const float zpf = static_cast<float>(zp);
    for (int t = threadIdx.x; t < N * R; t += blockDim.x) {
        const int p = t / R, r = t - (t / R) * R;
        const float v = act_value(h, (static_cast<int64_t>(b) * N + p) * C + c0 + r, codes, s, zpf);
        const int q = bit_reverse(p, log2N);
        sa[r * N + (N == 1024 ? fft1024_pos(q) : q)] = make_float2(v, 0.0f);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float2* row = sa + warp * N;
    if (N == 1024) {
        warp_fft1024<false>(row, tw, lane);
        for (int m = lane; m < modes; m += 32)
            Xs[(static_cast<int64_t>(b) * C + c0 + warp) * modes + m] = row[fft1024_pos(m)];
        return;
    }
    warp_fft_row_first<false>(row, N, tw, lane, modes);
    for (int m = lane; m < modes; m += 32)
        Xs[(static_cast<int64_t>(b) * C + c0 + warp) * modes + m] = row[m];
}

// ---------------------------------------------------------------------------
// layer: grid (C / G, B), 256 threads.  Dynamic shared memory:
//   sRow [G][N] float2 (inverse transforms, then x1), sY [G][modes] float2,
//   sW [G][C] float (local weights of the group, FP32 path)
// ---------------------------------------------------------------------------
struct Layer1dArgs {
    const void* h_in;
    void* h_out;
    const float2* Xs;
    const float* x2raw;
    const float2* tw_inv;
    Fno1dLayer L;
    int N, log2N, C, G, modes, act;
};

__global__ void __launch_bounds__(256, 2) layer1d_kernel(Layer1dArgs a) {
    extern __shared__ float2 smem[];
    const int G = a.G, N = a.N, C = a.C, modes = a.modes;
    float2* sRow = smem;
    float2* sY = sRow + static_cast<size_t>(G) * N;
    float* sW = reinterpret_cast<float*>(sY + static_cast<size_t>(G) * modes);
    const int b = blockIdx.y, o0 = blockIdx.x * G;
    const Fno1dLayer& L = a.L;

    // spectral contraction (fno.cpp:181-196), sum over input channels in order:
    //   re += fma(hr, wr, -(hi*wi)),  im += fma(hr, wi, hi*wr)
    for (int t = threadIdx.x; t < G * modes; t += blockDim.x) {
        const int r = t / modes, m = t - (t / modes) * modes;
        const int o = o0 + r;
        float sr = 0.0f, si = 0.0f;
        const float2* xb = a.Xs + static_cast<int64_t>(b) * C * modes + m;
        for (int c = 0; c < C; ++c) {
            const float2 hv = xb[static_cast<int64_t>(c) * modes];
            const int64_t wi = (static_cast<int64_t>(c) * C + o) * modes + m;
            const float wr = __ldg(L.wr + wi), wim = __ldg(L.wi + wi);
            sr = __fadd_rn(sr, __fmaf_rn(hv.x, wr, -__fmul_rn(hv.y, wim)));
            si = __fadd_rn(si, __fmaf_rn(hv.x, wim, __fmul_rn(hv.y, wr)));
        }
        sY[r * modes + m] = make_float2(sr, si);
    }
    if (!L.use_int8)
        for (int t = threadIdx.x; t < G * C; t += blockDim.x) sW[t] = __ldg(L.loc_w + static_cast<int64_t>(o0) * C + t);
    __syncthreads();

    // inverse transform of each output row (Irfft, fft.cpp:86-99): bins [0, half) from
    // the contraction (zero past `modes`), the upper half mirrored as conjugates
    const int half = N / 2 + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < G; r += blockDim.x >> 5) {
        float2* row = sRow + static_cast<size_t>(r) * N;
        for (int j = lane; j < N; j += 32) {
            float2 v;
            if (j < half) {
                v = j < modes ? sY[r * modes + j] : make_float2(0.0f, 0.0f);
            } else {
                const int i = N - j;
                const float2 u = i < modes ? sY[r * modes + i] : make_float2(0.0f, 0.0f);
                v = make_float2(u.x, -u.y);
            }
            const int q = bit_reverse(j, a.log2N);
            row[N == 1024 ? fft1024_pos(q) : q] = v;
        }
        __syncwarp();
        if (N == 1024) warp_fft1024<true>(row, a.tw_inv, lane);
        else warp_fft_row<true>(row, N, a.tw_inv, lane);
    }
    __syncthreads();

    // local layer + epilogue, one point per thread iteration
    const float inv_n = __fdiv_rn(1.0f, static_cast<float>(N));
    const float zpf_in = static_cast<float>(L.in_zp);
    const float zpf_fq = static_cast<float>(L.fq_zp);
    const float zpf_out = static_cast<float>(L.out_zp);
    for (int p = threadIdx.x; p < N; p += blockDim.x) {
        const int64_t row = static_cast<int64_t>(b) * N + p;
        float x2[8];
        if (L.use_int8 && a.x2raw) {
#pragma unroll
            for (int r = 0; r < 8; ++r)
                if (r < G) x2[r] = __fadd_rn(a.x2raw[row * C + o0 + r], __ldg(L.loc_b + o0 + r));
        } else if (L.use_int8) {
            // widths the tcgen05 GEMM does not tile: the same LinearForwardBatched
            // arithmetic on CUDA cores (int32 dot products, the reference epilogue)
            const int8_t* arow = static_cast<const int8_t*>(a.h_in) + row * C;
            int raw[8];
            int sum_a = 0;
#pragma unroll
            for (int r = 0; r < 8; ++r) raw[r] = 0;
            for (int k = 0; k < C; ++k) {
                const int av = arow[k];
                sum_a += av;
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < G) raw[r] += av * static_cast<int>(__ldg(L.Wq + static_cast<int64_t>(o0 + r) * C + k));
            }
#pragma unroll
            for (int r = 0; r < 8; ++r) {
                if (r >= G) break;
                const int o = o0 + r;
                const int zw = __ldg(L.zp_w + o);
                const float sWsA = __fmul_rn(__ldg(L.scale_w + o), L.in_s);
                const float y = dequant_ref(raw[r], zw, C * L.in_zp - 2 * sum_a, L.in_zp * __ldg(L.sum_w + o), sWsA);
                x2[r] = __fadd_rn(y, __ldg(L.loc_b + o));
            }
        } else {
#pragma unroll
            for (int r = 0; r < 8; ++r)
                if (r < G) x2[r] = __ldg(L.loc_b + o0 + r);
            const int nu = linear_unfused_len(C);
            for (int k = 0; k < C; ++k) {
                const float hv = act_value(a.h_in, row * C + k, L.in_codes, L.in_s, zpf_in);
#pragma unroll
                for (int r = 0; r < 8; ++r)
                    if (r < G) x2[r] = linear_step(x2[r], hv, sW[r * C + k], k >= nu);
            }
        }
#pragma unroll
        for (int r = 0; r < 8; ++r) {
            if (r >= G) break;
            const int o = o0 + r;
            float v = x2[r];
            if (L.fq_kind == 1) {
                v = fake_quant(v, L.fq_s, zpf_fq);
            } else if (L.fq_kind == 2) {
                const int64_t qi = static_cast<int64_t>(o) * N + p;
                v = fake_quant(v, __ldg(L.pt_s + qi), static_cast<float>(__ldg(L.pt_zp + qi)));
            } else if (L.fq_kind == 3) {
                v = fp8_log2_snap(v, L.fq_s);
            }
            const float x1 = __fmul_rn(sRow[static_cast<size_t>(r) * N + (N == 1024 ? fft1024_pos(p) : p)].x, inv_n);
            const float z = __fadd_rn(x1, v);
            if (L.out_codes) {
                const int q = L.lut_cells > 0
                                  ? code_from_lut(z, L.code_lut, L.lut_cells, L.lut_zlo, L.lut_inv_delta)
                                  : static_cast<int>(fq_code(act_f(z, a.act), L.out_s, zpf_out));
                static_cast<int8_t*>(a.h_out)[row * C + o] = static_cast<int8_t>(q);
            } else {
                static_cast<float*>(a.h_out)[row * C + o] = act_f(z, a.act);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Split layer (widths 16, 32 and 64 with the FP32 local Linear): inv1d_kernel runs the
// contraction and the inverse transform per (b, group of R output rows), as
// layer1d_kernel does, and writes x1 = Irfft(...) / N channel-first (b, c, p);
// local1d_kernel then takes one point per thread and all C output channels -- the
// local Linear (FP32 with the reference's rounding, from an input row read as 16-byte
// vectors, the weights as [k][o] 16-byte broadcasts; the INT8 GEMM's output + bias is
// also handled), the output fake-quant, x1 + x2, the activation -- and
// writes the point's next activation as one contiguous run.  Every element sees the
// operations layer1d_kernel applies, in the same order; the input row is read once per
// point instead of once per output-channel group.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 2) inv1d_kernel(Layer1dArgs a, float* __restrict__ x1f) {
    extern __shared__ float2 smem[];
    const int G = a.G, N = a.N, C = a.C, modes = a.modes;
    float2* sRow = smem;
    float2* sY = sRow + static_cast<size_t>(G) * N;
    const int b = blockIdx.y, o0 = blockIdx.x * G;
    const Fno1dLayer& L = a.L;
    for (int t = threadIdx.x; t < G * modes; t += blockDim.x) {
        const int r = t / modes, m = t - (t / modes) * modes;
        const int o = o0 + r;
        float sr = 0.0f, si = 0.0f;
        const float2* xb = a.Xs + static_cast<int64_t>(b) * C * modes + m;
        for (int c = 0; c < C; ++c) {
            const float2 hv = xb[static_cast<int64_t>(c) * modes];
            const int64_t wi = (static_cast<int64_t>(c) * C + o) * modes + m;
            const float wr = __ldg(L.wr + wi), wim = __ldg(L.wi + wi);
            sr = __fadd_rn(sr, __fmaf_rn(hv.x, wr, -__fmul_rn(hv.y, wim)));
            si = __fadd_rn(si, __fmaf_rn(hv.x, wim, __fmul_rn(hv.y, wr)));
        }
        sY[r * modes + m] = make_float2(sr, si);
    }
    __syncthreads();
    const int half = N / 2 + 1;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float inv_n = __fdiv_rn(1.0f, static_cast<float>(N));
    for (int r = warp; r < G; r += blockDim.x >> 5) {
        float2* row = sRow + static_cast<size_t>(r) * N;
        for (int j = lane; j < N; j += 32) {
            float2 v;
            if (j < half) {
                v = j < modes ? sY[r * modes + j] : make_float2(0.0f, 0.0f);
            } else {
                const int i = N - j;
                const float2 u = i < modes ? sY[r * modes + i] : make_float2(0.0f, 0.0f);
                v = make_float2(u.x, -u.y);
            }
            const int q = bit_reverse(j, a.log2N);
            row[N == 1024 ? fft1024_pos(q) : q] = v;
        }
        __syncwarp();
        if (N == 1024) warp_fft1024<true>(row, a.tw_inv, lane);
        else warp_fft_row<true>(row, N, a.tw_inv, lane);
        float* dst = x1f + (static_cast<int64_t>(b) * C + o0 + r) * N;
        for (int p = lane; p < N; p += 32) dst[p] = __fmul_rn(row[N == 1024 ? fft1024_pos(p) : p].x, inv_n);
    }
}

template <int C>
__global__ void __launch_bounds__(128) local1d_kernel(Layer1dArgs a, const float* __restrict__ x1f,
                                                      int64_t total) {
    __shared__ float4 sW4[C * C / 4];  // [k][o]
    __shared__ float sB[C];
    float* sW = reinterpret_cast<float*>(sW4);
    const Fno1dLayer& L = a.L;
    const bool f32 = !L.use_int8;
    if (f32)
        for (int i = threadIdx.x; i < C * C; i += blockDim.x) sW[(i % C) * C + i / C] = __ldg(L.loc_w + i);
    for (int i = threadIdx.x; i < C; i += blockDim.x) sB[i] = __ldg(L.loc_b + i);
    __syncthreads();
    const int N = a.N, lgN = a.log2N;
    constexpr int nu = linear_unfused_len(C);
    const float zpf_in = static_cast<float>(L.in_zp);
    const float zpf_fq = static_cast<float>(L.fq_zp);
    const float zpf_out = static_cast<float>(L.out_zp);
    for (int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; row < total;
         row += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = row >> lgN;
        const int p = static_cast<int>(row - (b << lgN));
        float acc[C];
        if (f32) {
#pragma unroll
            for (int o = 0; o < C; ++o) acc[o] = sB[o];
            // four input features per pass (a compact loop body keeps the code in the
            // instruction cache)
#pragma unroll 1
            for (int k4 = 0; k4 < C / 4; ++k4) {
                float hv[4];
                if (L.in_codes) {
                    const uint32_t w4 = *reinterpret_cast<const uint32_t*>(static_cast<const int8_t*>(a.h_in) + row * C + 4 * k4);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int8_t code = static_cast<int8_t>((w4 >> (8 * j)) & 0xFFu);
                        hv[j] = __fmul_rn(__fsub_rn(static_cast<float>(code), zpf_in), L.in_s);
                    }
                } else {
                    const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(a.h_in) + row * C + 4 * k4);
                    hv[0] = v.x;
                    hv[1] = v.y;
                    hv[2] = v.z;
                    hv[3] = v.w;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int k = 4 * k4 + j;
                    const bool fused = k >= nu;
#pragma unroll
                    for (int o4 = 0; o4 < C / 4; ++o4) {
                        const float4 w = sW4[k * (C / 4) + o4];
                        if (nu >= C) {
                            // every product unfused (C a multiple of 8): two rounded
                            // products per f32x2 instruction, each sum a scalar add
                            const float2 m0 = mul2_rn(make_float2(hv[j], hv[j]), make_float2(w.x, w.y));
                            const float2 m1 = mul2_rn(make_float2(hv[j], hv[j]), make_float2(w.z, w.w));
                            acc[4 * o4 + 0] = __fadd_rn(acc[4 * o4 + 0], m0.x);
                            acc[4 * o4 + 1] = __fadd_rn(acc[4 * o4 + 1], m0.y);
                            acc[4 * o4 + 2] = __fadd_rn(acc[4 * o4 + 2], m1.x);
                            acc[4 * o4 + 3] = __fadd_rn(acc[4 * o4 + 3], m1.y);
                        } else {
                            acc[4 * o4 + 0] = linear_step(acc[4 * o4 + 0], hv[j], w.x, fused);
                            acc[4 * o4 + 1] = linear_step(acc[4 * o4 + 1], hv[j], w.y, fused);
                            acc[4 * o4 + 2] = linear_step(acc[4 * o4 + 2], hv[j], w.z, fused);
                            acc[4 * o4 + 3] = linear_step(acc[4 * o4 + 3], hv[j], w.w, fused);
                        }
                    }
                }
            }
        } else {
            const float4* xr = reinterpret_cast<const float4*>(a.x2raw + row * C);
#pragma unroll
            for (int o4 = 0; o4 < C / 4; ++o4) {
                const float4 v = xr[o4];
                acc[4 * o4 + 0] = __fadd_rn(v.x, sB[4 * o4 + 0]);
                acc[4 * o4 + 1] = __fadd_rn(v.y, sB[4 * o4 + 1]);
                acc[4 * o4 + 2] = __fadd_rn(v.z, sB[4 * o4 + 2]);
                acc[4 * o4 + 3] = __fadd_rn(v.w, sB[4 * o4 + 3]);
            }
        }
        const float* x1p = x1f + b * C * N + p;
#pragma unroll
        for (int o4 = 0; o4 < C / 4; ++o4) {
            float out[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int o = 4 * o4 + j;
                float v = acc[o];
                if (L.fq_kind == 1) {
                    v = fake_quant(v, L.fq_s, zpf_fq);
                } else if (L.fq_kind == 2) {
                    const int64_t qi = static_cast<int64_t>(o) * N + p;
                    v = fake_quant(v, __ldg(L.pt_s + qi), static_cast<float>(__ldg(L.pt_zp + qi)));
                } else if (L.fq_kind == 3) {
                    v = fp8_log2_snap(v, L.fq_s);
                }
                const float z = __fadd_rn(x1p[static_cast<int64_t>(o) * N], v);
                if (L.out_codes)
                    out[j] = __int_as_float(L.lut_cells > 0
                                                ? code_from_lut(z, L.code_lut, L.lut_cells, L.lut_zlo, L.lut_inv_delta)
                                                : static_cast<int>(fq_code(act_f(z, a.act), L.out_s, zpf_out)));
                else
                    out[j] = act_f(z, a.act);
            }
            if (L.out_codes) {
                const uint32_t pk = (static_cast<uint32_t>(__float_as_int(out[0])) & 0xFFu) |
                                    ((static_cast<uint32_t>(__float_as_int(out[1])) & 0xFFu) << 8) |
                                    ((static_cast<uint32_t>(__float_as_int(out[2])) & 0xFFu) << 16) |
                                    ((static_cast<uint32_t>(__float_as_int(out[3])) & 0xFFu) << 24);
                reinterpret_cast<uint32_t*>(static_cast<int8_t*>(a.h_out) + row * C)[o4] = pk;
            } else {
                reinterpret_cast<float4*>(static_cast<float*>(a.h_out) + row * C)[o4] =
                    make_float4(out[0], out[1], out[2], out[3]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// projection for widths up to 128, over tiles of kProjTP points (the same arithmetic as
// proj1d_kernel below, element for element):
//   phase 1  the tile's activation rows -> sH [TP][C], proj_q transposed -> sWt [C][C]
//   phase 2  q[p][c]: thread (c, point group) runs the proj_q dot products of eight
//            points at a time (independent chains; the point's features are warp-
//            uniform broadcasts, the weight column one conflict-free load per k for
//            all eight), then the activation -> sQ [TP][C + 1]
//   phase 3  one thread per point: the proj_out sums over c in order
// ---------------------------------------------------------------------------
constexpr int kProjTP = 64;
constexpr int kProjThreads = 128;
constexpr int kProjILP = 8;   // points per thread and pass (independent dot products)

size_t proj1d_tiled_smem(int C) {
    return (static_cast<size_t>(kProjTP) * C + static_cast<size_t>(C) * C +
            static_cast<size_t>(kProjTP) * (C + 1)) * sizeof(float);
}

__global__ void __launch_bounds__(kProjThreads) proj1d_tiled_kernel(
    const float* __restrict__ h, int n, int N, int C, int out_ch, int64_t total,
    const float* __restrict__ pq_w, const float* __restrict__ pq_b, const float* __restrict__ po_w,
    const float* __restrict__ po_b, int act, float* __restrict__ y) {
    extern __shared__ float sh[];
    float* sH = sh;                                   // [TP][C]
    float* sWt = sH + static_cast<size_t>(kProjTP) * C;  // [C][C]: sWt[k * C + c] = pq_w[c][k]
    float* sQ = sWt + static_cast<size_t>(C) * C;     // [TP][C + 1]
    const int tid = threadIdx.x;
    for (int t = tid; t < C * C; t += kProjThreads) {
        const int c = t / C, k = t - (t / C) * C;
        sWt[k * C + c] = __ldg(pq_w + t);
    }
    const int nu = linear_unfused_len(C);
    const int G = C <= kProjThreads ? kProjThreads / C : 1;  // point groups
    for (int64_t t0 = static_cast<int64_t>(blockIdx.x) * kProjTP; t0 < total;
         t0 += static_cast<int64_t>(gridDim.x) * kProjTP) {
        const int np = static_cast<int>(total - t0 < kProjTP ? total - t0 : kProjTP);
        __syncthreads();  // the previous tile's sH / sQ are no longer read
        for (int e = tid; e < np * C; e += kProjThreads) {
            const int r = e / C, k = e - (e / C) * C;
            const int64_t t = t0 + r;
            const int64_t b = t / n;
            const int pp = static_cast<int>(t - b * n);
            sH[r * C + k] = h[(b * N + pp) * C + k];
        }
        __syncthreads();
        for (int item = tid; item < C * G; item += kProjThreads) {
            const int c = item % C, g = item / C;
            const float bias = __ldg(pq_b + c);
            for (int r0 = g * kProjILP; r0 < np; r0 += kProjILP * G) {
                float q[kProjILP];
                const float* hr[kProjILP];
#pragma unroll
                for (int u = 0; u < kProjILP; ++u) {
                    q[u] = bias;
                    hr[u] = sH + (r0 + u < np ? r0 + u : r0) * C;
                }
                int k = 0;
                for (; k < nu; ++k) {
                    const float wv = sWt[k * C + c];
#pragma unroll
                    for (int u = 0; u < kProjILP; ++u) q[u] = __fadd_rn(q[u], __fmul_rn(hr[u][k], wv));
                }
                for (; k < C; ++k) {
                    const float wv = sWt[k * C + c];
#pragma unroll
                    for (int u = 0; u < kProjILP; ++u) q[u] = __fmaf_rn(hr[u][k], wv, q[u]);
                }
#pragma unroll
                for (int u = 0; u < kProjILP; ++u)
                    if (r0 + u < np) sQ[(r0 + u) * (C + 1) + c] = act_f(q[u], act);
            }
        }
        __syncthreads();
        if (tid < np) {
            const float* qr = sQ + tid * (C + 1);
            float acc[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = j < out_ch ? __ldg(po_b + j) : 0.0f;
            for (int c = 0; c < C; ++c) {
                const float qv = qr[c];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (j < out_ch)
                        acc[j] = linear_step(acc[j], qv, __ldg(po_w + static_cast<int64_t>(j) * C + c), c >= nu);
            }
            float* yr = y + (t0 + tid) * out_ch;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < out_ch) yr[j] = acc[j];
        }
    }
}

// The same tiled projection with the width and the output-channel count as template
// parameters (C in {16, 32, 64, 128}, 1 <= OUT <= 4): the rows are staged one warp per
// row (the sample index divided out once per row), the dot products' rounding split is
// a compile-time constant, and the proj_out sums run over exactly OUT accumulators with
// the weights in shared memory.  Element for element the arithmetic of
// proj1d_tiled_kernel.
template <int C, int OUT>
__global__ void __launch_bounds__(kProjThreads) proj1d_tiled_t_kernel(
    const float* __restrict__ h, int n, int N, int64_t total, const float* __restrict__ pq_w,
    const float* __restrict__ pq_b, const float* __restrict__ po_w, const float* __restrict__ po_b, int act,
    float* __restrict__ y) {
    extern __shared__ float sh[];
    float* sH = sh;                                 // [TP][C]
    float* sWt = sH + kProjTP * C;                  // [C][C]: sWt[k * C + c] = pq_w[c][k]
    float* sQ = sWt + C * C;                        // [TP][C + 1]
    __shared__ float sPo[OUT * C];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int t = tid; t < C * C; t += kProjThreads) sWt[(t % C) * C + t / C] = __ldg(pq_w + t);
    for (int t = tid; t < OUT * C; t += kProjThreads) sPo[t] = __ldg(po_w + t);
    constexpr int nu = linear_unfused_len(C);
    constexpr int G = C <= kProjThreads ? kProjThreads / C : 1;  // point groups
    for (int64_t t0 = static_cast<int64_t>(blockIdx.x) * kProjTP; t0 < total;
         t0 += static_cast<int64_t>(gridDim.x) * kProjTP) {
        const int np = static_cast<int>(total - t0 < kProjTP ? total - t0 : kProjTP);
        __syncthreads();  // the previous tile's sH / sQ are no longer read
        for (int r = warp; r < np; r += kProjThreads / 32) {
            const int64_t t = t0 + r;
            const int64_t b = t / n;
            const int pp = static_cast<int>(t - b * n);
            const float* src = h + (b * N + pp) * C;
#pragma unroll
            for (int k = lane; k < C; k += 32) sH[r * C + k] = src[k];
        }
        __syncthreads();
        for (int item = tid; item < C * G; item += kProjThreads) {
            const int c = item % C, g = item / C;
            const float bias = __ldg(pq_b + c);
            for (int r0 = g * kProjILP; r0 < np; r0 += kProjILP * G) {
                float q[kProjILP];
                const float* hr[kProjILP];
#pragma unroll
                for (int u = 0; u < kProjILP; ++u) {
                    q[u] = bias;
                    hr[u] = sH + (r0 + u < np ? r0 + u : r0) * C;
                }
#pragma unroll 8
                for (int k = 0; k < nu; ++k) {
                    const float wv = sWt[k * C + c];
#pragma unroll
                    for (int u = 0; u < kProjILP; ++u) q[u] = __fadd_rn(q[u], __fmul_rn(hr[u][k], wv));
                }
#pragma unroll 8
                for (int k = nu; k < C; ++k) {
                    const float wv = sWt[k * C + c];
#pragma unroll
                    for (int u = 0; u < kProjILP; ++u) q[u] = __fmaf_rn(hr[u][k], wv, q[u]);
                }
#pragma unroll
                for (int u = 0; u < kProjILP; ++u)
                    if (r0 + u < np) sQ[(r0 + u) * (C + 1) + c] = act_f(q[u], act);
            }
        }
        __syncthreads();
        if (tid < np) {
            const float* qr = sQ + tid * (C + 1);
            float acc[OUT];
#pragma unroll
            for (int j = 0; j < OUT; ++j) acc[j] = __ldg(po_b + j);
#pragma unroll 8
            for (int c = 0; c < C; ++c) {
                const float qv = qr[c];
#pragma unroll
                for (int j = 0; j < OUT; ++j) acc[j] = linear_step(acc[j], qv, sPo[j * C + c], c >= nu);
            }
            float* yr = y + (t0 + tid) * OUT;
#pragma unroll
            for (int j = 0; j < OUT; ++j) yr[j] = acc[j];
        }
    }
}

// ---------------------------------------------------------------------------
// projection (fno.cpp:683-702): q = Linear(h, proj_q) -> act -> y = Linear(q, proj_out),
// both the reference's sequential dot product from the bias (linear_step), the proj_out
// sum interleaved with the production of q[c] in increasing c (the same operation
// sequence per output).  One point per
// thread; the point's activation row is staged in shared memory [threads][C + 1].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) proj1d_kernel(const float* __restrict__ h, int n, int N,
                                                     int C, int out_ch, int64_t total,
                                                     const float* __restrict__ pq_w,
                                                     const float* __restrict__ pq_b,
                                                     const float* __restrict__ po_w,
                                                     const float* __restrict__ po_b, int act,
                                                     float* __restrict__ y) {
    extern __shared__ float sh[];
    float* mine = sh + static_cast<size_t>(threadIdx.x) * (C + 1);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = t / n;
        const int p = static_cast<int>(t - b * n);
        const float* hr = h + (b * N + p) * C;
        for (int k = 0; k < C; ++k) mine[k] = hr[k];
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = j < out_ch ? __ldg(po_b + j) : 0.0f;
        const int nu = linear_unfused_len(C);
        for (int c = 0; c < C; ++c) {
            float q = __ldg(pq_b + c);
            const float* wr = pq_w + static_cast<int64_t>(c) * C;
            for (int k = 0; k < C; ++k) q = linear_step(q, mine[k], __ldg(wr + k), k >= nu);
            q = act_f(q, act);
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < out_ch)
                    acc[j] = linear_step(acc[j], q, __ldg(po_w + static_cast<int64_t>(j) * C + c), c >= nu);
        }
        float* yr = y + t * out_ch;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j < out_ch) yr[j] = acc[j];
    }
}

int ilog2(int v) {
    int l = 0;
    while ((1 << l) < v) ++l;
    return l;
}

// rows per CTA: the largest of 8, 4, 2, 1 that divides C with R * N float2 <= 64 KB
int rows_per_cta(int C, int N) {
    for (int R = 8; R > 1; R >>= 1)
        if (C % R == 0 && static_cast<size_t>(R) * N * sizeof(float2) <= 65536) return R;
    return 1;
}

}  // namespace

cudaError_t fno1d_run(const Fno1dPlan& pl, cudaStream_t st) {
    if (pl.B == 0) return cudaSuccess;
    const int N = pl.N, C = pl.C, log2N = ilog2(N);
    const int sms = device_sm_count();
    const int R = rows_per_cta(C, N);
    cudaError_t e;
    {
        const int64_t total = static_cast<int64_t>(pl.B) * N * C;
        const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, sms * 16));
        const Fno1dLayer& L0 = pl.layer[0];
        if (pl.timer) pl.timer->begin("fno1d_lift", st);
        lift1d_kernel<<<grid, 256, 0, st>>>(pl.x, pl.n, N, C, pl.in_ch, total, pl.lift_w, pl.lift_b,
                                            L0.in_codes, L0.in_s, L0.in_zp, pl.h[0]);
        if (pl.timer) pl.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    const size_t fwd_smem = static_cast<size_t>(R) * N * sizeof(float2);
    if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(fft1d_fwd_kernel),
                                  static_cast<int>(fwd_smem))) != cudaSuccess)
        return e;
    const size_t layer_smem = static_cast<size_t>(R) * N * sizeof(float2) +
                              static_cast<size_t>(R) * pl.modes * sizeof(float2) +
                              static_cast<size_t>(R) * C * sizeof(float);
    if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(layer1d_kernel),
                                  static_cast<int>(layer_smem))) != cudaSuccess)
        return e;
    for (int i = 0; i < pl.L; ++i) {
        const Fno1dLayer& L = pl.layer[i];
        const void* hin = pl.h[i & 1];
        void* hout = pl.h[(i + 1) & 1];
        if (pl.timer) pl.timer->begin("fno1d_fft_fwd", st);
        fft1d_fwd_kernel<<<dim3(C / R, pl.B), 32 * R, fwd_smem, st>>>(
            hin, L.in_codes, L.in_s, L.in_zp, N, log2N, C, pl.modes, pl.tw_fwd, pl.Xs);
        if (pl.timer) pl.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        if (L.use_int8 && gemm_i8_supported(C, C)) {
            GemmArgs g{};
            g.A = static_cast<const int8_t*>(hin);
            g.scale_a_t = L.in_s;
            g.zp_a_t = L.in_zp;
            g.W = L.Wq;
            g.scale_w = L.scale_w;
            g.zp_w = L.zp_w;
            g.sum_w = L.sum_w;
            g.bias = nullptr;
            g.act = 0;
            g.C = pl.x2raw;
            g.M = pl.B * N;
            g.err = pl.err;
            if (pl.timer) pl.timer->begin("fno1d_gemm_i8", st);
            e = gemm_i8_launch(g, C, C, st);
            if (pl.timer) pl.timer->end(st);
            if (e != cudaSuccess) return e;
        }
        // the FP32 local layer splits off (its per-point dot products dominate); with the
        // INT8 GEMM the local term is a read of x2raw and the fused kernel is faster
        const bool split = (C == 16 || C == 32 || C == 64) && !L.use_int8 && pl.x1f != nullptr;
        Layer1dArgs a;
        a.h_in = hin;
        a.h_out = hout;
        a.Xs = pl.Xs;
        a.x2raw = gemm_i8_supported(C, C) ? pl.x2raw : nullptr;
        a.tw_inv = pl.tw_inv;
        a.L = L;
        a.N = N;
        a.log2N = log2N;
        a.C = C;
        a.G = R;
        a.modes = pl.modes;
        a.act = pl.act;
        if (split) {
            const size_t inv_smem = static_cast<size_t>(R) * N * sizeof(float2) +
                                    static_cast<size_t>(R) * pl.modes * sizeof(float2);
            if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(inv1d_kernel),
                                          static_cast<int>(inv_smem))) != cudaSuccess)
                return e;
            if (pl.timer) pl.timer->begin("fno1d_inv", st);
            inv1d_kernel<<<dim3(C / R, pl.B), 32 * R, inv_smem, st>>>(a, pl.x1f);
            if (pl.timer) pl.timer->end(st);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            const int64_t total = static_cast<int64_t>(pl.B) * N;
            const int grid = static_cast<int>(std::min<int64_t>((total + 127) / 128, sms * 8));
            if (pl.timer) pl.timer->begin("fno1d_layer", st);
            if (C == 16) local1d_kernel<16><<<grid, 128, 0, st>>>(a, pl.x1f, total);
            else if (C == 32) local1d_kernel<32><<<grid, 128, 0, st>>>(a, pl.x1f, total);
            else local1d_kernel<64><<<grid, 128, 0, st>>>(a, pl.x1f, total);
            if (pl.timer) pl.timer->end(st);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            continue;
        }
        if (pl.timer) pl.timer->begin("fno1d_layer", st);
        layer1d_kernel<<<dim3(C / R, pl.B), 256, layer_smem, st>>>(a);
        if (pl.timer) pl.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    if (C <= 128) {
        const int64_t total = static_cast<int64_t>(pl.B) * pl.n;
        const size_t smem = proj1d_tiled_smem(C);
        if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(proj1d_tiled_kernel),
                                      static_cast<int>(smem))) != cudaSuccess)
            return e;
        const int per_sm = smem <= 56 * 1024 ? 4 : (smem <= 112 * 1024 ? 2 : 1);
        const int grid = static_cast<int>(std::min<int64_t>((total + kProjTP - 1) / kProjTP, sms * per_sm * 2));
        if (pl.timer) pl.timer->begin("fno1d_proj", st);
        const float* hl = static_cast<const float*>(pl.h[pl.L & 1]);
        bool done = false;
#define NFX_PROJ1D(CC, OO)                                                                                 \
    if (!done && C == CC && pl.out_ch == OO) {                                                             \
        if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(proj1d_tiled_t_kernel<CC, OO>),         \
                                      static_cast<int>(smem))) != cudaSuccess)                             \
            return e;                                                                                      \
        proj1d_tiled_t_kernel<CC, OO><<<grid, kProjThreads, smem, st>>>(hl, pl.n, N, total, pl.pq_w, pl.pq_b, \
                                                                        pl.po_w, pl.po_b, pl.act, pl.y);    \
        done = true;                                                                                       \
    }
        NFX_PROJ1D(16, 1) NFX_PROJ1D(32, 1) NFX_PROJ1D(64, 1) NFX_PROJ1D(128, 1)
        NFX_PROJ1D(16, 2) NFX_PROJ1D(32, 2) NFX_PROJ1D(64, 2) NFX_PROJ1D(128, 2)
        NFX_PROJ1D(16, 3) NFX_PROJ1D(32, 3) NFX_PROJ1D(64, 3) NFX_PROJ1D(128, 3)
        NFX_PROJ1D(16, 4) NFX_PROJ1D(32, 4) NFX_PROJ1D(64, 4) NFX_PROJ1D(128, 4)
#undef NFX_PROJ1D
        if (!done)
            proj1d_tiled_kernel<<<grid, kProjThreads, smem, st>>>(hl, pl.n, N, C, pl.out_ch, total, pl.pq_w, pl.pq_b,
                                                                  pl.po_w, pl.po_b, pl.act, pl.y);
        if (pl.timer) pl.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    } else {
        const int64_t total = static_cast<int64_t>(pl.B) * pl.n;
        const int threads = C > 128 ? 64 : 128;
        const size_t smem = static_cast<size_t>(threads) * (C + 1) * sizeof(float);
        if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(proj1d_kernel),
                                      static_cast<int>(smem))) != cudaSuccess)
            return e;
        const int grid = static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, sms * 8));
        if (pl.timer) pl.timer->begin("fno1d_proj", st);
        proj1d_kernel<<<grid, threads, smem, st>>>(static_cast<const float*>(pl.h[pl.L & 1]), pl.n, N, C,
                                                   pl.out_ch, total, pl.pq_w, pl.pq_b, pl.po_w,
                                                   pl.po_b, pl.act, pl.y);
        if (pl.timer) pl.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace nfx
