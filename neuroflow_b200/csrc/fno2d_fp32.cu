// fno2d_fp32.cu -- FNO2d FP32 fake-quant executor (sm_100a): the reference
// FNO2d::Forward (cpp/src/fno.cpp:777-995) as InferenceRuntime::Run executes it when
// EnableInt8Gemm is not in effect, with the reference's rounding.
//
// Activations are fp32, channel-first (b, c, h, w), as the reference's h_perm: rows
// of a channel are contiguous for the transforms, and a warp of consecutive points
// reads one channel coalesced for the local layer.  One layer is
//
//   fwd2d    per (b, c): the reference Rfft2 (fft.cpp:101-124) restricted to what the
//            truncation keeps -- every row transform (all of them feed the kept
//            columns), then the column transforms of the MW kept columns -> Xs
//   mix2d    per (b, group of output channels): the per-mode contraction
//            (fno.cpp:740-764), then the column pass of Irfft2 (fft.cpp:126-149) for
//            the MW nonzero columns -> colinv (b, o, h, kw)
//   layer2d  per (b, row): the row pass of Irfft2 for every output channel (x1), the
//            local Linear of the row's points, locs.i.output fake-quant, x1 + x2 and
//            the activation -> next activation
//
// Every product, sum and transform follows the reference's expression shapes
// (fft_exact.cuh, linear_step); the only approximate operation is CUDA's tanhf inside
// GELU.  Columns of Irfft2 that the truncation leaves all-zero are taken as +0.
//
// With the INT8 composition (Fno2dI8Linear / Fno2dSnap in fno2d.h) the lift and every
// layer but the last store their output snapped for the next layer, layer2d takes the
// local Linear over the input's int8 codes, and proj2d does the same for proj_q.  The
// snaps after an activation come from the host's exact z -> code tables, so GELU stays
// exact there too.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <type_traits>

#include "fft_exact.cuh"
#include "fno2d.h"
#include "nfx_internal.h"
#include "numerics.cuh"

namespace nfx {
namespace {

constexpr int kChunk = 16;  // output channels per inverse-row chunk in layer2d
constexpr int kMaxWp = 512;

__device__ __forceinline__ float act_f(float z, int act) {
    return act == 1 ? relu_ref(z) : gelu_tanh(z);
}

// Calibration observer of one thread: the range of the values it saw, merged across
// the warp and into the tensor's global keys at the end of the kernel.
struct Obs {
    float lo = INFINITY, hi = -INFINITY;
    bool nan = false;
    __device__ __forceinline__ void see(float v) {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
        nan = nan || (v != v);
    }
    // whole warp
    __device__ __forceinline__ void flush(unsigned* obs, int i) {
        for (int o = 16; o > 0; o >>= 1) {
            lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
            hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
        }
        const bool any_nan = __any_sync(0xffffffffu, nan);
        if ((threadIdx.x & 31) == 0) {
            if (lo <= hi) {
                atomicMin(obs + i, float_order_key(lo));
                atomicMax(obs + kFno2dObsMax + i, float_order_key(hi));
            }
            if (any_nan) atomicOr(obs + 2 * kFno2dObsMax + i, 1u);
        }
    }
};

int ilog2(int v) {
    int l = 0;
    while ((1 << l) < v) ++l;
    return l;
}

// lift (fno.cpp:848-865): Linear, lift.output fake-quant, permute to channel-first,
// zero padding
__global__ void __launch_bounds__(256) lift2d_f32_kernel(Fno2dF32Plan p) {
    const int64_t total = static_cast<int64_t>(p.B) * p.C * p.Hp * p.Wp;
    const int nu = linear_unfused_len(p.in_ch);
    Obs ob;
    // Hp and Wp are powers of two (radix-2 transforms): the point's coordinates by
    // shifts and masks, and one 32-bit division by C
    const int lgW = 31 - __clz(p.Wp), lgH = 31 - __clz(p.Hp);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int ww = static_cast<int>(t & (p.Wp - 1));
        const int hh = static_cast<int>((t >> lgW) & (p.Hp - 1));
        const int64_t bc = t >> (lgW + lgH);
        int c;
        int64_t b;
        if (bc <= 0x7fffffff) {
            const unsigned q = static_cast<unsigned>(bc) / static_cast<unsigned>(p.C);
            b = q;
            c = static_cast<int>(static_cast<unsigned>(bc) - q * static_cast<unsigned>(p.C));
        } else {
            b = bc / p.C;
            c = static_cast<int>(bc - b * p.C);
        }
        float v = 0.0f;
        if (hh < p.H && ww < p.W) {
            const float* xr = p.x + ((b * p.H + hh) * p.W + ww) * p.in_ch;
            v = __ldg(p.lift_b + c);
            for (int k = 0; k < p.in_ch; ++k)
                v = linear_step(v, __ldg(xr + k), __ldg(p.lift_w + c * p.in_ch + k), k >= nu);
            if (p.obs) {
                ob.see(v);
                if (p.obs_vals[0]) p.obs_vals[0][((b * p.H + hh) * p.W + ww) * p.C + c] = v;
            }
            v = apply_fq(v, p.fq_lift);
        }
        // layer 0's input snap (padding zeros included, as the reference pads first)
        if (p.snap_lift.kind == 1) v = fake_quant(v, p.snap_lift.scale, static_cast<float>(p.snap_lift.zp));
        p.h[0][t] = v;
    }
    if (p.obs) ob.flush(p.obs, 0);
}

// forward truncated Rfft2 of one (b, c) plane; 256 threads; shared memory
// rowbuf [8][Wp] float2, colbuf [MW][Hp] float2 (columns stored bit-reversed)
__global__ void __launch_bounds__(256) fwd2d_kernel(const float* __restrict__ hin, int Hp, int Wp,
                                                    int C, int MH, int MW,
                                                    const float2* __restrict__ twf_w,
                                                    const float2* __restrict__ twf_h,
                                                    float2* __restrict__ Xs) {
    extern __shared__ float2 sm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x, b = blockIdx.y;
    const int lgW = 31 - __clz(Wp), lgH = 31 - __clz(Hp);
    float2* row = sm + warp * Wp;
    float2* col = sm + 8 * Wp;
    const float* plane = hin + (static_cast<int64_t>(b) * C + c) * Hp * Wp;
    if (Wp == 128) {
        // rows in registers (warp_fft128_regs); the kept modes kw < MW are entries
        // lane + 32 j of the result
        for (int r = warp; r < Hp; r += 8) {
            const float* src = plane + static_cast<int64_t>(r) * 128;
            float2 v[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) v[m] = make_float2(src[fft128_src(lane, m)], 0.0f);
            warp_fft128_regs<false>(v, row, twf_w, lane);
            const int rr = bit_reverse(r, lgH);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (lane + 32 * j < MW) col[(lane + 32 * j) * Hp + rr] = v[j];
        }
    } else {
        for (int r = warp; r < Hp; r += 8) {
            for (int j = lane; j < Wp; j += 32) row[bit_reverse(j, lgW)] = make_float2(plane[static_cast<int64_t>(r) * Wp + j], 0.0f);
            __syncwarp();
            warp_fft_row_first<false>(row, Wp, twf_w, lane, MW);
            const int rr = bit_reverse(r, lgH);
            for (int kw = lane; kw < MW; kw += 32) col[kw * Hp + rr] = row[kw];
            __syncwarp();
        }
    }
    __syncthreads();
    if (Hp == 128 && Wp >= 128) {  // the warp's row buffer (Wp entries) is the scratch
        for (int kw = warp; kw < MW; kw += 8) {
            float2 v[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) v[m] = col[kw * 128 + 4 * lane + m];  // bit-reversed column
            warp_fft128_regs<false>(v, row, twf_h, lane);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (lane + 32 * j < MH) Xs[((static_cast<int64_t>(b) * C + c) * MH + lane + 32 * j) * MW + kw] = v[j];
        }
        return;
    }
    for (int kw = warp; kw < MW; kw += 8) {
        warp_fft_row_first<false>(col + kw * Hp, Hp, twf_h, lane, MH);
        for (int kh = lane; kh < MH; kh += 32)
            Xs[((static_cast<int64_t>(b) * C + c) * MH + kh) * MW + kw] = col[kw * Hp + kh];
    }
}

// contraction + column inverse; grid (C / G, B), 256 threads; shared memory
// sY [G][MH*MW] float2, colb [8][Hp] float2
__global__ void __launch_bounds__(256) mix2d_kernel(const float2* __restrict__ Xs,
                                                    const float* __restrict__ wr,
                                                    const float* __restrict__ wi, int Hp, int C,
                                                    int MH, int MW, int G,
                                                    const float2* __restrict__ twi_h,
                                                    float2* __restrict__ colinv) {
    extern __shared__ float2 sm[];
    const int M = MH * MW;
    float2* sY = sm;
    float2* colb = sm + G * M;
    const int b = blockIdx.y, o0 = blockIdx.x * G;
    for (int t = threadIdx.x; t < G * M; t += blockDim.x) {
        const int r = t / M, md = t - (t / M) * M;
        const int o = o0 + r;
        float sr = 0.0f, si = 0.0f;
        const float2* xb = Xs + static_cast<int64_t>(b) * C * M + md;
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
    const int lgH = 31 - __clz(Hp);
    const float invH = __fdiv_rn(1.0f, static_cast<float>(Hp));
    float2* cb = colb + warp * Hp;
    if (Hp == 128) {
        for (int q = warp; q < G * MW; q += 8) {
            const int r = q / MW, kw = q - (q / MW) * MW;
            float2 v[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const int i = fft128_src(lane, m);
                v[m] = i < MH ? sY[r * M + i * MW + kw] : make_float2(0.0f, 0.0f);
            }
            warp_fft128_regs<true>(v, cb, twi_h, lane);
            float2* dst = colinv + ((static_cast<int64_t>(b) * C + o0 + r) * Hp) * MW + kw;
#pragma unroll
            for (int j = 0; j < 4; ++j)
                dst[static_cast<int64_t>(lane + 32 * j) * MW] =
                    make_float2(__fmul_rn(v[j].x, invH), __fmul_rn(v[j].y, invH));
        }
        return;
    }
    for (int q = warp; q < G * MW; q += 8) {
        const int r = q / MW, kw = q - (q / MW) * MW;
        for (int i = lane; i < Hp; i += 32)
            cb[bit_reverse(i, lgH)] = i < MH ? sY[r * M + i * MW + kw] : make_float2(0.0f, 0.0f);
        __syncwarp();
        warp_fft_row<true>(cb, Hp, twi_h, lane);
        float2* dst = colinv + ((static_cast<int64_t>(b) * C + o0 + r) * Hp) * MW + kw;
        for (int i = lane; i < Hp; i += 32) {
            const float2 v = cb[i];
            dst[static_cast<int64_t>(i) * MW] = make_float2(__fmul_rn(v.x, invH), __fmul_rn(v.y, invH));
        }
        __syncwarp();
    }
}

// row inverse + local layer + epilogue for one row of one sample; grid (Hp, B), 256
// threads; shared memory sH [C][Wp] float, sX1 [kChunk][Wp] float2, sSum [Wp] float
struct Layer2dArgs {
    const float* hin;
    float* hout;
    const float2* colinv;
    const float2* twi_w;
    const float* loc_w;
    const float* loc_b;
    FqParam fq;
    Fno2dI8Linear i8;     // wz nullptr: FP32 Linear
    Fno2dSnap snap;       // output snap (kind 0: the activation's value)
    int Hp, Wp, C, MW, act;
    unsigned* obs;        // calibration observers (Fno2dF32Plan::obs), tensor obs_i
    float* obs_vals;
    int obs_i;
};

// OBS: calibration observers compiled in; I8: the INT8 composition (int8 Linear and /
// or the output snap) compiled in.  The plain FP32 network runs the <false, false>
// instantiation, with neither in its loops.
// NJ = max(1, Wp / 32): the groups of 32 points a lane covers, a compile-time count so
// the local Linear's loops carry no idle iterations.
template <bool OBS, bool I8, int NJ>
__global__ void __launch_bounds__(256) layer2d_kernel(Layer2dArgs a) {
    extern __shared__ float2 sm[];
    const int Wp = a.Wp, C = a.C, Hp = a.Hp;
    float* sH = reinterpret_cast<float*>(sm);
    float2* sX1 = sm + (static_cast<size_t>(C) * Wp + 1) / 2;
    float* sSum = reinterpret_cast<float*>(sX1 + static_cast<size_t>(kChunk) * Wp);
    const int hh = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lgW = 31 - __clz(Wp);
    const int half = Wp / 2 + 1;
    const bool i8 = I8 && a.i8.wz != nullptr;
    const float zp_in = static_cast<float>(a.i8.zp_in);
    if (Wp % 4 == 0) {
        // 16-byte loads, four in flight per thread
#pragma unroll 4
        for (int t4 = threadIdx.x; t4 < C * Wp / 4; t4 += blockDim.x) {
            const int t = 4 * t4;
            const int k = t / Wp, w = t - (t / Wp) * Wp;
            const float4 v = *reinterpret_cast<const float4*>(a.hin + ((static_cast<int64_t>(b) * C + k) * Hp + hh) * Wp + w);
            // INT8: QuantiseActivation's code (int8_gemm.cpp:507-520) of the snapped input
            *reinterpret_cast<float4*>(sH + t) =
                i8 ? make_float4(fq_code(v.x, a.i8.s_in, zp_in), fq_code(v.y, a.i8.s_in, zp_in),
                                 fq_code(v.z, a.i8.s_in, zp_in), fq_code(v.w, a.i8.s_in, zp_in))
                   : v;
        }
    } else {
        for (int t = threadIdx.x; t < C * Wp; t += blockDim.x) {
            const int k = t / Wp, w = t - (t / Wp) * Wp;
            const float v = a.hin[((static_cast<int64_t>(b) * C + k) * Hp + hh) * Wp + w];
            sH[t] = i8 ? fq_code(v, a.i8.s_in, zp_in) : v;
        }
    }
    if (i8) {
        // sum_a of each point (exact: |sum| <= 128 C)
        __syncthreads();
        for (int w = threadIdx.x; w < Wp; w += blockDim.x) {
            float sa = 0.0f;
            for (int k = 0; k < C; ++k) sa = __fadd_rn(sa, sH[static_cast<size_t>(k) * Wp + w]);
            sSum[w] = sa;
        }
    }
    const float invW = __fdiv_rn(1.0f, static_cast<float>(Wp));
    const int nu = linear_unfused_len(C);
    Obs ob;
    constexpr int R = kChunk / 8;
    // at Wp = 128 no chunk-wide barrier follows the row pass: the layer input (and
    // sSum) must be visible before the first local Linear
    if constexpr (NJ == 4) __syncthreads();
    for (int o0 = 0; o0 < C; o0 += kChunk) {
        // row pass of Irfft2 (fft.cpp:86-99) for kChunk output channels.  At Wp = 128
        // (NJ = 4) each warp transforms the rows of its own R output channels in
        // registers: entry lane + 32 j of the result is the x1 of point lane + 32 j,
        // the point this lane takes in the local Linear below.
        float x1v[R][NJ];
        if constexpr (NJ == 4) {
#pragma unroll
            for (int rr = 0; rr < R; ++rr) {
                const int r = warp * R + rr;
                if (o0 + r >= C) break;
                const float2* ci = a.colinv + ((static_cast<int64_t>(b) * C + o0 + r) * Hp + hh) * a.MW;
                float2 v[4];
#pragma unroll
                for (int m = 0; m < 4; ++m) {
                    const int j = fft128_src(lane, m);
                    if (j < half) {
                        v[m] = j < a.MW ? ci[j] : make_float2(0.0f, 0.0f);
                    } else {
                        const int i = 128 - j;
                        const float2 u = i < a.MW ? ci[i] : make_float2(0.0f, 0.0f);
                        v[m] = make_float2(u.x, -u.y);
                    }
                }
                warp_fft128_regs<true>(v, sX1 + static_cast<size_t>(warp) * 128, a.twi_w, lane);
#pragma unroll
                for (int j = 0; j < 4; ++j) x1v[rr][j] = v[j].x;
            }
        } else {
            for (int r = warp; r < kChunk && o0 + r < C; r += 8) {
                float2* row = sX1 + static_cast<size_t>(r) * Wp;
                const float2* ci = a.colinv + ((static_cast<int64_t>(b) * C + o0 + r) * Hp + hh) * a.MW;
                for (int j = lane; j < Wp; j += 32) {
                    float2 v;
                    if (j < half) {
                        v = j < a.MW ? ci[j] : make_float2(0.0f, 0.0f);
                    } else {
                        const int i = Wp - j;
                        const float2 u = i < a.MW ? ci[i] : make_float2(0.0f, 0.0f);
                        v = make_float2(u.x, -u.y);
                    }
                    row[bit_reverse(j, lgW)] = v;
                }
                __syncwarp();
                warp_fft_row<true>(row, Wp, a.twi_w, lane);
            }
            __syncthreads();
        }
        // local Linear of the row's points for this chunk: warp -> R output channels,
        // lane -> points lane + 32 j; one shared-memory load of a point's input feeds
        // all R channels (each channel's sum keeps the k order)
        float acc[R][NJ];
        const float* wrow[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
            const int o = min(o0 + warp * R + rr, C - 1);
            wrow[rr] = (i8 ? a.i8.wz : a.loc_w) + static_cast<int64_t>(o) * C;
            const float bias = i8 ? 0.0f : __ldg(a.loc_b + o);
#pragma unroll
            for (int j = 0; j < NJ; ++j) acc[rr][j] = bias;
        }
        if (i8) {
            // exact integer dot product of codes and (w - zp_w)
            for (int k = 0; k < C; ++k) {
                const float* hk = sH + static_cast<size_t>(k) * Wp;
                float hv[NJ];
#pragma unroll
                for (int j = 0; j < NJ; ++j) hv[j] = (NJ > 1 || lane < Wp) ? hk[lane + 32 * j] : 0.0f;
#pragma unroll
                for (int rr = 0; rr < R; ++rr) {
                    const float wv = __ldg(wrow[rr] + k);
#pragma unroll
                    for (int j = 0; j < NJ; ++j) acc[rr][j] = __fmaf_rn(hv[j], wv, acc[rr][j]);
                }
            }
        } else {
            // the reference's unfused products (k < nu) and fused tail as two loops, so
            // neither carries the other's form
            auto steps = [&](auto fused, int k0, int k1) {
                for (int k = k0; k < k1; ++k) {
                    const float* hk = sH + static_cast<size_t>(k) * Wp;
                    float hv[NJ];
#pragma unroll
                    for (int j = 0; j < NJ; ++j) hv[j] = (NJ > 1 || lane < Wp) ? hk[lane + 32 * j] : 0.0f;
#pragma unroll
                    for (int rr = 0; rr < R; ++rr) {
                        const float wv = __ldg(wrow[rr] + k);
                        if constexpr (!decltype(fused)::value && NJ % 2 == 0) {
                            // two rounded products per f32x2 instruction, each sum a
                            // scalar rounded add
#pragma unroll
                            for (int j = 0; j < NJ; j += 2) {
                                const float2 m = mul2_rn(make_float2(hv[j], hv[j + 1]), make_float2(wv, wv));
                                acc[rr][j] = __fadd_rn(acc[rr][j], m.x);
                                acc[rr][j + 1] = __fadd_rn(acc[rr][j + 1], m.y);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < NJ; ++j)
                                acc[rr][j] = linear_step(acc[rr][j], hv[j], wv, decltype(fused)::value);
                        }
                    }
                }
            };
            steps(std::false_type{}, 0, nu);
            steps(std::true_type{}, nu, C);
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
            const int r = warp * R + rr;
            const int o = o0 + r;
            if (o >= C) break;
            if (i8) {
                // the epilogue of the integer sums
                const float bias = __ldg(a.loc_b + o);
                const int4 cc = __ldg(a.i8.cols + o);
#pragma unroll
                for (int j = 0; j < NJ; ++j)
                    if (NJ > 1 || lane < Wp) {
                        const int v = __float2int_rn(acc[rr][j]) - cc.y * __float2int_rn(sSum[lane + 32 * j]) + cc.z;
                        const float y = __fadd_rn(__fmul_rn(__int_as_float(cc.x), __int2float_rn(v)), 0.0f);
                        acc[rr][j] = __fadd_rn(y, bias);
                    }
            }
            float* dst = a.hout + ((static_cast<int64_t>(b) * C + o) * Hp + hh) * Wp;
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                const int w = lane + 32 * j;
                if (NJ > 1 || w < Wp) {
                    if (OBS) {
                        ob.see(acc[rr][j]);
                        if (a.obs_vals) a.obs_vals[((static_cast<int64_t>(b) * Hp + hh) * Wp + w) * C + o] = acc[rr][j];
                    }
                    const float x2 = apply_fq(acc[rr][j], a.fq);
                    const float x1 = __fmul_rn(NJ == 4 ? x1v[rr][j] : sX1[static_cast<size_t>(r) * Wp + w].x, invW);
                    const float z = __fadd_rn(x1, x2);
                    if (I8 && a.snap.fq.kind == 1) {
                        const float zpo = static_cast<float>(a.snap.fq.zp);
                        const float q = a.snap.code_lut
                                            ? static_cast<float>(code_from_lut(z, a.snap.code_lut, a.snap.lut_cells,
                                                                               a.snap.lut_zlo, a.snap.lut_inv_delta))
                                            : fq_code(act_f(z, a.act), a.snap.fq.scale, zpo);
                        dst[w] = __fmul_rn(__fsub_rn(q, zpo), a.snap.fq.scale);
                    } else {
                        dst[w] = act_f(z, a.act);
                    }
                }
            }
        }
        // the next chunk's row pass rewrites sX1 (at Wp = 128 each warp only its own
        // scratch row)
        if constexpr (NJ != 4) __syncthreads();
    }
    if (OBS) ob.flush(a.obs, a.obs_i);
}

template <bool OBS, bool I8>
void (*layer2d_pick(int Wp))(Layer2dArgs) {
    switch (Wp >= 32 ? Wp / 32 : 1) {
        case 1: return layer2d_kernel<OBS, I8, 1>;
        case 2: return layer2d_kernel<OBS, I8, 2>;
        case 4: return layer2d_kernel<OBS, I8, 4>;
        case 8: return layer2d_kernel<OBS, I8, 8>;
        default: return layer2d_kernel<OBS, I8, 16>;
    }
}

// projection (fno.cpp:966-993): one unpadded point per thread, its channel column
// staged in shared memory [threads][C + 1]
template <bool OBS, bool I8>
__global__ void __launch_bounds__(128) proj2d_f32_kernel(Fno2dF32Plan p, const float* __restrict__ h) {
    extern __shared__ float sh[];
    float* mine = sh + static_cast<size_t>(threadIdx.x) * (p.C + 1);
    const int64_t total = static_cast<int64_t>(p.B) * p.H * p.W;
    const int C = p.C;
    const int nu = linear_unfused_len(C);
    Obs obq, obo;
    const int iq = p.L + 1, io = p.L + 2;
    const bool pq8 = I8 && p.pq_i8.wz != nullptr;
    const float zp_in = static_cast<float>(p.pq_i8.zp_in);
    const float zp_pq = static_cast<float>(p.fq_pq.zp);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int ww = static_cast<int>(t % p.W);
        const int64_t r = t / p.W;
        const int hh = static_cast<int>(r % p.H);
        const int64_t b = r / p.H;
        for (int k = 0; k < C; ++k) mine[k] = h[((b * C + k) * p.Hp + hh) * p.Wp + ww];
        // INT8 proj_q: the point's codes and their sum (int8_gemm.cpp:507-520, :567)
        float sum_a = 0.0f;
        if (pq8) {
            for (int k = 0; k < C; ++k) {
                mine[k] = fq_code(mine[k], p.pq_i8.s_in, zp_in);
                sum_a = __fadd_rn(sum_a, mine[k]);
            }
        }
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = j < p.out_ch ? __ldg(p.po_b + j) : 0.0f;
        for (int c = 0; c < C; ++c) {
            float q;
            if (pq8) {
                float s = 0.0f;
                const float* wr = p.pq_i8.wz + static_cast<int64_t>(c) * C;
                for (int k = 0; k < C; ++k) s = __fmaf_rn(mine[k], __ldg(wr + k), s);
                const int4 cc = __ldg(p.pq_i8.cols + c);
                const int v = __float2int_rn(s) - cc.y * __float2int_rn(sum_a) + cc.z;
                q = __fadd_rn(__fadd_rn(__fmul_rn(__int_as_float(cc.x), __int2float_rn(v)), 0.0f),
                              __ldg(p.pq_b + c));
            } else {
                q = __ldg(p.pq_b + c);
                const float* wr = p.pq_w + static_cast<int64_t>(c) * C;
                for (int k = 0; k < C; ++k) q = linear_step(q, mine[k], __ldg(wr + k), k >= nu);
            }
            if (OBS) {
                obq.see(q);
                if (p.obs_vals[iq]) p.obs_vals[iq][t * C + c] = q;
            }
            if (I8 && p.pq_act_table && p.fq_pq.kind == 1)
                q = __ldg(p.pq_act_table + static_cast<int>(fq_code(q, p.fq_pq.scale, zp_pq)) + 128);
            else
                q = act_f(apply_fq(q, p.fq_pq), p.act);
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < p.out_ch)
                    acc[j] = linear_step(acc[j], q, __ldg(p.po_w + static_cast<int64_t>(j) * C + c), c >= nu);
        }
        float* yr = p.y + t * p.out_ch;
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (j < p.out_ch) {
                if (OBS) {
                    obo.see(acc[j]);
                    if (p.obs_vals[io]) p.obs_vals[io][t * p.out_ch + j] = acc[j];
                }
                yr[j] = apply_fq(acc[j], p.fq_po);
            }
    }
    if (OBS) {
        obq.flush(p.obs, iq);
        obo.flush(p.obs, io);
    }
}

// The plain FP32 projection (no observers, no INT8 composition) for widths 32 and 64
// with 1 to 4 output channels: the point's C inputs in registers (coalesced channel
// loads), proj_q rows as 16-byte broadcasts from shared memory, exactly OUT proj_out
// sums.  Element for element proj2d_f32_kernel<false, false>'s arithmetic.
template <int C, int OUT>
__global__ void __launch_bounds__(128) proj2d_f32_fast_kernel(Fno2dF32Plan p, const float* __restrict__ h) {
    __shared__ float4 sW4[C * C / 4];   // proj_q, [c][k]
    __shared__ float sPo[OUT * C];
    __shared__ float sB[C];
    for (int i = threadIdx.x; i < C * C; i += blockDim.x) reinterpret_cast<float*>(sW4)[i] = __ldg(p.pq_w + i);
    for (int i = threadIdx.x; i < OUT * C; i += blockDim.x) sPo[i] = __ldg(p.po_w + i);
    for (int i = threadIdx.x; i < C; i += blockDim.x) sB[i] = __ldg(p.pq_b + i);
    __syncthreads();
    const int64_t total = static_cast<int64_t>(p.B) * p.H * p.W;
    constexpr int nu = linear_unfused_len(C);
    const int64_t plane = static_cast<int64_t>(p.Hp) * p.Wp;
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int ww = static_cast<int>(t % p.W);
        const int64_t r = t / p.W;
        const int hh = static_cast<int>(r % p.H);
        const int64_t b = r / p.H;
        const float* src = h + b * C * plane + static_cast<int64_t>(hh) * p.Wp + ww;
        float x[C];
#pragma unroll
        for (int k = 0; k < C; ++k) x[k] = src[k * plane];
        float acc[OUT];
#pragma unroll
        for (int j = 0; j < OUT; ++j) acc[j] = __ldg(p.po_b + j);
#pragma unroll 1
        for (int c = 0; c < C; ++c) {
            float q = sB[c];
#pragma unroll
            for (int k4 = 0; k4 < C / 4; ++k4) {
                const float4 w = sW4[c * (C / 4) + k4];
                q = linear_step(q, x[4 * k4 + 0], w.x, 4 * k4 + 0 >= nu);
                q = linear_step(q, x[4 * k4 + 1], w.y, 4 * k4 + 1 >= nu);
                q = linear_step(q, x[4 * k4 + 2], w.z, 4 * k4 + 2 >= nu);
                q = linear_step(q, x[4 * k4 + 3], w.w, 4 * k4 + 3 >= nu);
            }
            q = act_f(apply_fq(q, p.fq_pq), p.act);
#pragma unroll
            for (int j = 0; j < OUT; ++j) acc[j] = linear_step(acc[j], q, sPo[j * C + c], c >= nu);
        }
        float* yr = p.y + t * OUT;
#pragma unroll
        for (int j = 0; j < OUT; ++j) yr[j] = apply_fq(acc[j], p.fq_po);
    }
}

template <int C>
void (*proj2d_fast_pick(int out_ch))(Fno2dF32Plan, const float*) {
    switch (out_ch) {
        case 1: return proj2d_f32_fast_kernel<C, 1>;
        case 2: return proj2d_f32_fast_kernel<C, 2>;
        case 3: return proj2d_f32_fast_kernel<C, 3>;
        case 4: return proj2d_f32_fast_kernel<C, 4>;
        default: return nullptr;
    }
}

size_t fwd_smem(int Hp, int Wp, int MW) {
    return (8 * static_cast<size_t>(Wp) + static_cast<size_t>(MW) * Hp) * sizeof(float2);
}
size_t layer_smem(int C, int Wp) {
    return ((static_cast<size_t>(C) * Wp + 1) / 2 + static_cast<size_t>(kChunk) * Wp) * sizeof(float2) +
           static_cast<size_t>(Wp) * sizeof(float);
}
int mix_group(int C) {
    for (int G = 8; G > 1; G >>= 1)
        if (C % G == 0) return G;
    return 1;
}

}  // namespace

const char* fno2d_f32_unsupported(int C, int MH, int MW, int Hp, int Wp, int out_ch) {
    if (C < 1 || C > 256) return "FNO2d GPU executor: width must be in [1, 256]";
    if (out_ch < 1 || out_ch > 16) return "FNO2d GPU executor: out_channels must be in [1, 16]";
    if (Wp > kMaxWp || Hp > 4096) return "FNO2d GPU executor: padded W <= 512 and H <= 4096";
    if (fwd_smem(Hp, Wp, MW) > 200 * 1024 || layer_smem(C, Wp) > 200 * 1024)
        return "FNO2d GPU executor: grid too large for the shared-memory transforms";
    if (static_cast<size_t>(mix_group(C)) * MH * MW * sizeof(float2) + 8 * static_cast<size_t>(Hp) * sizeof(float2) >
        200 * 1024)
        return "FNO2d GPU executor: too many modes";
    return nullptr;
}

cudaError_t fno2d_f32_run(const Fno2dF32Plan& p, cudaStream_t st) {
    if (p.B == 0) return cudaSuccess;
    const int sms = device_sm_count();
    cudaError_t e;
    {
        const int64_t total = static_cast<int64_t>(p.B) * p.C * p.Hp * p.Wp;
        const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, sms * 32));
        if (p.timer) p.timer->begin("fno2d_f32_lift", st);
        lift2d_f32_kernel<<<grid, 256, 0, st>>>(p);
        if (p.timer) p.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    const size_t sf = fwd_smem(p.Hp, p.Wp, p.MW);
    const int G = mix_group(p.C);
    const size_t sx = (static_cast<size_t>(G) * p.MH * p.MW + 8 * static_cast<size_t>(p.Hp)) * sizeof(float2);
    const size_t sl = layer_smem(p.C, p.Wp);
    if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(fwd2d_kernel), static_cast<int>(sf))) != cudaSuccess ||
        (e = set_max_dynamic_smem(reinterpret_cast<const void*>(mix2d_kernel), static_cast<int>(sx))) != cudaSuccess)
        return e;
    // the instantiation of the layer and projection kernels: observers, INT8 composition
    const bool obs = p.obs != nullptr;
    bool i8 = p.pq_i8.wz != nullptr || p.pq_act_table != nullptr;
    for (int i = 0; i < p.L; ++i) i8 = i8 || p.layer[i].i8.wz != nullptr || p.layer[i].snap.fq.kind != 0;
    auto layer_k = obs ? (i8 ? layer2d_pick<true, true>(p.Wp) : layer2d_pick<true, false>(p.Wp))
                       : (i8 ? layer2d_pick<false, true>(p.Wp) : layer2d_pick<false, false>(p.Wp));
    auto proj_k = obs ? (i8 ? proj2d_f32_kernel<true, true> : proj2d_f32_kernel<true, false>)
                      : (i8 ? proj2d_f32_kernel<false, true> : proj2d_f32_kernel<false, false>);
    if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(layer_k), static_cast<int>(sl))) != cudaSuccess)
        return e;
    for (int i = 0; i < p.L; ++i) {
        const float* hin = p.h[i & 1];
        float* hout = p.h[(i + 1) & 1];
        const Fno2dF32Layer& L = p.layer[i];
        if (p.timer) p.timer->begin("fno2d_f32_fwd", st);
        fwd2d_kernel<<<dim3(p.C, p.B), 256, sf, st>>>(hin, p.Hp, p.Wp, p.C, p.MH, p.MW, p.twf_w, p.twf_h, p.Xs);
        if (p.timer) p.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        if (p.timer) p.timer->begin("fno2d_f32_mix", st);
        mix2d_kernel<<<dim3(p.C / G, p.B), 256, sx, st>>>(p.Xs, L.wr, L.wi, p.Hp, p.C, p.MH, p.MW, G, p.twi_h,
                                                         p.colinv);
        if (p.timer) p.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        Layer2dArgs a;
        a.hin = hin;
        a.hout = hout;
        a.colinv = p.colinv;
        a.twi_w = p.twi_w;
        a.loc_w = L.loc_w;
        a.loc_b = L.loc_b;
        a.fq = L.fq;
        a.i8 = L.i8;
        a.snap = L.snap;
        a.obs = p.obs;
        a.obs_vals = p.obs ? p.obs_vals[1 + i] : nullptr;
        a.obs_i = 1 + i;
        a.Hp = p.Hp;
        a.Wp = p.Wp;
        a.C = p.C;
        a.MW = p.MW;
        a.act = p.act;
        if (p.timer) p.timer->begin("fno2d_f32_layer", st);
        layer_k<<<dim3(p.Hp, p.B), 256, sl, st>>>(a);
        if (p.timer) p.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    {
        const int64_t total = static_cast<int64_t>(p.B) * p.H * p.W;
        const int threads = p.C > 128 ? 64 : 128;
        const size_t smem = static_cast<size_t>(threads) * (p.C + 1) * sizeof(float);
        if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(proj_k), static_cast<int>(smem))) !=
            cudaSuccess)
            return e;
        const int grid = static_cast<int>(std::min<int64_t>((total + threads - 1) / threads, sms * 8));
        void (*fast)(Fno2dF32Plan, const float*) = nullptr;
        if (!obs && !i8) fast = p.C == 64 ? proj2d_fast_pick<64>(p.out_ch) : p.C == 32 ? proj2d_fast_pick<32>(p.out_ch) : nullptr;
        if (p.timer) p.timer->begin("fno2d_f32_proj", st);
        if (fast)
            fast<<<grid, 128, 0, st>>>(p, p.h[p.L & 1]);
        else
            proj_k<<<grid, threads, smem, st>>>(p, p.h[p.L & 1]);
        if (p.timer) p.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace nfx
