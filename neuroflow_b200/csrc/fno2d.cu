// fno2d.cu -- FNO2d INT8 layer executor kernels (sm_100a).
//
// Activations between layers live in HBM only as int8 codes, channel-last
// (b, h, w, c), quantised with the layer-input qparams (the reference FNO1d INT8
// convention, cpp/src/fno.cpp:475-549, applied to FNO2d's structure,
// cpp/src/fno.cpp:777-995).  One layer is three kernels:
//
//   spec_fwd   codes -> per-row-block partial spectra of the truncated 2D rFFT
//              (rows: W-axis DFT restricted to kw < MW; then the H-axis DFT
//              restricted to kh < MH, accumulated over the block's rows).
//   spec_mix   sum of the partials, then the per-mode complex (in x out) contraction
//              (fno.cpp:740-764) on tensor cores (3xTF32) -> Y (b, kh, kw, o).
//   layer      tcgen05 kind::i8 GEMM of the local 1x1 layer (codes x locs.i codes),
//              fused with: inverse truncated 2D transform of Y evaluated at the
//              tile's points (x1), the LinearForwardBatched dequant epilogue + bias,
//              locs.i.output fake-quant (x2), x1 + x2, activation, and quantisation
//              to the next layer's codes (16-byte stores; TMA stores in the W != 128 kernel).
//
// lift (K = in_ch, CUDA cores) and the projection (tcgen05 GEMM for proj_q, the
// out_ch-wide proj_out dot product in the epilogue) close the network.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>
#include <utility>

#include "fno2d.h"
#include "nfx_internal.h"
#include "numerics.cuh"
#include "sm100.cuh"

namespace nfx {
namespace {

constexpr int pow2ceil(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
}

__device__ __forceinline__ float activation(float z, int act) {
    return act == 1 ? relu_ref(z) : gelu_tanh(z);
}

// ---------------------------------------------------------------------------
// Division-free code of v under (s, zp) with the fast-path test of fq_code_fast
// (numerics.cuh), in the form the epilogues pack directly:
//   r = v * (1/s);  t = r + (1.5 * 2^23 + zp)
// rounds r to an integer in t's last place (t has unit spacing for |r| < 2^22), so
// k = t - (1.5 * 2^23 + zp) = rint(r) exactly, and t clamped to 1.5 * 2^23 +
// [-128, 127] carries the clamped code clamp(rint(r) + zp) as its low byte (and as
// bits(t) - 0x4B400000).  `bad` is set where the element needs the exact division:
// r within 2^-14 of a half-integer (where rint and std::round may differ too), or NaN.
// ---------------------------------------------------------------------------
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
__device__ __forceinline__ float fast_code_t(float v, float inv_s, float magic_zp, bool& bad) {
    const float r = __fmul_rn(v, inv_s);
    const float t = __fadd_rn(r, magic_zp);
    const float k = __fsub_rn(t, magic_zp);
    bad = !(fabsf(__fsub_rn(r, k)) < kFastRoundLimit);
    return fminf(fmaxf(t, kMagic - 128.0f), kMagic + 127.0f);
}

// ---------------------------------------------------------------------------
// lift: x (M, in_ch) fp32 -> codes (M, C) with the lift.output qparams.
// fno.cpp:848-853 (Linear + fake-quant), fno.cpp:51-80 (the dot product from the bias).
// One thread per point and all C channels: the weights and biases are constant-bank
// operands (compile-time offsets), so a thread holds only its inputs and packed codes
// and the kernel runs at full occupancy.  The fast-path test keeps the largest
// |r - rint(r)| of the point (NaN-propagating max); a point with a near-half-integer
// quotient, or a NaN, recomputes its channels with the exact division.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

template <int C, int IN>
__global__ void __launch_bounds__(256) lift_kernel(const float* __restrict__ x, int64_t M,
                                                   const __grid_constant__ LiftCols lc, float s, int zp,
                                                   float inv_s, int8_t* __restrict__ codes) {
    static_assert(C % 16 == 0 && C <= kFno2dColMax && IN <= kFno2dLiftInMax, "lift layout");
    constexpr int nu = linear_unfused_len(IN);
    const float magic_zp = kMagic + static_cast<float>(zp);
    const float zpf = static_cast<float>(zp);
    grid_dep_wait();   // x and the codes buffer may still be in use by the previous kernel
    grid_dep_launch();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t m = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; m < M; m += stride) {
        float xv[IN];
#pragma unroll
        for (int k = 0; k < IN; ++k) xv[k] = __ldg(x + m * IN + k);
        uint32_t words[C / 4];
        float dmax[C / 4];    // per packed word of 4 channels
#pragma unroll
        for (int o = 0; o < C; ++o) {
            float acc = lc.b[o];
#pragma unroll
            for (int k = 0; k < IN; ++k) acc = linear_step(acc, xv[k], lc.w[o][k], k >= nu);
            const float r = __fmul_rn(acc, inv_s);
            const float t = __fadd_rn(r, magic_zp);
            const float d = fabsf(__fsub_rn(r, __fsub_rn(t, magic_zp)));
            dmax[o >> 2] = (o & 3) == 0 ? d : fmax_nan(dmax[o >> 2], d);
            const float tc = fminf(fmaxf(t, kMagic - 128.0f), kMagic + 127.0f);
            const uint32_t sel = (0x3210u & ~(0xFu << (4 * (o & 3)))) | (4u << (4 * (o & 3)));
            words[o >> 2] = __byte_perm((o & 3) == 0 ? 0u : words[o >> 2], __float_as_uint(tc), sel);
        }
#pragma unroll
        for (int g = 0; g < C / 4; ++g) {
            if (dmax[g] < kFastRoundLimit) continue;
            // rare: a quotient next to a half-integer, huge or NaN in this group
#pragma unroll 1
            for (int o = 4 * g; o < 4 * g + 4; ++o) {
                float a = lc.b[o];
                for (int k = 0; k < IN; ++k) a = linear_step(a, xv[k], lc.w[o][k], k >= nu);
                const float r = __fmul_rn(a, inv_s);
                if (fabsf(__fsub_rn(r, rintf(r))) < kFastRoundLimit) continue;
                const uint32_t byte = static_cast<uint32_t>(static_cast<int>(fq_code(a, s, zpf))) & 0xFFu;
                uint32_t& w = words[o >> 2];
                w = (w & ~(0xFFu << (8 * (o & 3)))) | (byte << (8 * (o & 3)));
            }
        }
        uint4* dst = reinterpret_cast<uint4*>(codes + m * C);
#pragma unroll
        for (int q = 0; q < C / 16; ++q)
            dst[q] = make_uint4(words[4 * q], words[4 * q + 1], words[4 * q + 2], words[4 * q + 3]);
    }
}

// ---------------------------------------------------------------------------
// spec_fwd: grid (H / HB, B), C*MW threads.  Thread (c, kw) = (tid % C, tid / C)
// accumulates  X[kh][kw][c] += F[h][kw][c] * e^{-2 pi i kh h / H}  over the block's
// rows, with F[h][kw][c] = sum_w x[h][w][c] e^{-2 pi i kw w / W} and
// x = (code - zp) * s, the snapped activation (fno.cpp:497-505).
// ---------------------------------------------------------------------------
template <int C, int MH, int MW>
__global__ void __launch_bounds__(C * MW) spec_fwd_kernel(const int8_t* __restrict__ codes, int H,
                                                          int W, int HB, float s, int zp,
                                                          const float2* __restrict__ twf_w,
                                                          const float2* __restrict__ twf_h,
                                                          float2* __restrict__ xpart) {
    constexpr int kThr = C * MW;
    extern __shared__ float smem_f[];
    float* sx = smem_f;                                          // [W][C]
    float2* stw = reinterpret_cast<float2*>(smem_f + W * C);     // [MW][W]
    const int hb = blockIdx.x, b = blockIdx.y;
    const int nHB = gridDim.x;
    for (int i = threadIdx.x; i < MW * W; i += kThr) stw[i] = twf_w[i];
    const int c = threadIdx.x % C, kw = threadIdx.x / C;
    float2 acc[MH];
#pragma unroll
    for (int kh = 0; kh < MH; ++kh) acc[kh] = make_float2(0.f, 0.f);
    const float zpf = static_cast<float>(zp);
    const int8_t* src_b = codes + static_cast<int64_t>(b) * H * W * C;
    for (int r = 0; r < HB; ++r) {
        const int h = hb * HB + r;
        __syncthreads();
        const int4* row = reinterpret_cast<const int4*>(src_b + static_cast<int64_t>(h) * W * C);
        for (int i = threadIdx.x; i < W * C / 16; i += kThr) {
            int4 v = row[i];
            const int8_t* q = reinterpret_cast<const int8_t*>(&v);
#pragma unroll
            for (int j = 0; j < 16; ++j)
                sx[i * 16 + j] = __fmul_rn(__fsub_rn(static_cast<float>(q[j]), zpf), s);
        }
        __syncthreads();
        float fr = 0.f, fi = 0.f;
        const float2* t = stw + kw * W;
        for (int w = 0; w < W; ++w) {
            const float xv = sx[w * C + c];
            const float2 tw = t[w];
            fr = fmaf(xv, tw.x, fr);
            fi = fmaf(xv, tw.y, fi);
        }
        const float2* eh = twf_h + h * MH;
#pragma unroll
        for (int kh = 0; kh < MH; ++kh) {
            const float2 e = __ldg(eh + kh);
            acc[kh].x = fmaf(fr, e.x, fmaf(-fi, e.y, acc[kh].x));
            acc[kh].y = fmaf(fr, e.y, fmaf(fi, e.x, acc[kh].y));
        }
    }
    // xpart[b][hb][kh][kw][c]
    float2* dst = xpart + (static_cast<int64_t>(b) * nHB + hb) * (MH * MW * C);
#pragma unroll
    for (int kh = 0; kh < MH; ++kh) dst[(kh * MW + kw) * C + c] = acc[kh];
}

// ---------------------------------------------------------------------------
// spec_mix_tc: the per-mode contraction on tensor cores (C == 64).  For mode m and a
// tile of 128 samples, with x the sum of the row-block partials (fixed order) as the
// real row [re, im] per input channel, y = x Wr where Wr is the real (2C x 2C) form of
// the complex weights (fno.cpp:740-764):
//   D[b][n] = sum_k X[b][k] Wr[k][n]     (tcgen05 kind::tf32, 3xTF32: hi.hi + lo.hi + hi.lo)
// in four K chunks of 32 floats (one 128-byte swizzle atom); the weights' tf32 halves
// are prepared on the host and loaded by TMA, the activations are summed and split by
// all threads.  Accumulator: 128 lanes (samples) x 128 columns (2 out + re/im).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void split_tf32_m(float x, float& hi, float& lo) {
    hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
    lo = __fsub_rn(x, hi);
}

constexpr int kMixTcThreads = 256;
// PRE: every K chunk's weight tiles resident at once (one weight buffer pair per
// chunk, 160 KB; used when one sample tile per mode leaves CTAs one per SM), all
// requested before the kernel waits for its predecessor; otherwise one buffer pair,
// chunk c's weights requested once chunk c - 1's MMAs have read theirs (66 KB, several
// CTAs per SM).
template <int C, bool PRE>
struct MixCfg {
    static constexpr int kK = 2 * C;                 // 128 floats per row
    static constexpr int kChunk = 32;                // floats per K chunk
    static constexpr int kChunks = kK / kChunk;
    static constexpr int kTile = 128 * 128;          // [128 rows][32 floats], SW128
    static constexpr int kBufs = PRE ? kChunks : 1;  // weight buffer pairs (hi, lo)
    static constexpr int kOffAhi = 0;
    static constexpr int kOffAlo = kTile;
    static constexpr int kOffB = 2 * kTile;
    static constexpr int kOffBars = kOffB + 2 * kBufs * kTile;
    static constexpr int kSmemBytes = kOffBars + 8 * (kBufs + 1) + 16 + 1024;
    static_assert(C == 64, "one 128-column accumulator");
};

template <int C, int MH, int MW, bool PRE>
__global__ void __launch_bounds__(kMixTcThreads) spec_mix_tc_kernel(const __grid_constant__ CUtensorMap tmWhi,
                                                                    const __grid_constant__ CUtensorMap tmWlo,
                                                                    const float2* __restrict__ xpart, int nHB,
                                                                    int B, float2* __restrict__ Y,
                                                                    unsigned* err) {
    using F = MixCfg<C, PRE>;
    constexpr int M = MH * MW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sAhi = smem + F::kOffAhi;
    uint8_t* sAlo = smem + F::kOffAlo;
    uint8_t* sB = smem + F::kOffB;                   // pair q: hi at tile 2q, lo at 2q + 1
    uint64_t* bFull = reinterpret_cast<uint64_t*>(smem + F::kOffBars);   // [kBufs]
    uint64_t* mmaDone = bFull + F::kBufs;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(mmaDone + 1);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = blockIdx.x;
    const int b0 = blockIdx.y * 128;

    // weight chunk c into buffer pair c % kBufs (the weights are read-only and written by
    // no kernel of the forward, so they may be requested before the predecessor ends)
    auto load_w = [&](int c) {
        const int q = c % F::kBufs;
        mbar_arrive_expect_tx(&bFull[q], 2 * F::kTile);
        tma_load_2d(sB + 2 * q * F::kTile, &tmWhi, &bFull[q], c * F::kChunk, m * F::kK);
        tma_load_2d(sB + (2 * q + 1) * F::kTile, &tmWlo, &bFull[q], c * F::kChunk, m * F::kK);
    };
    if (threadIdx.x == 0) {
        for (int q = 0; q < F::kBufs; ++q) mbar_init(&bFull[q], 1);
        mbar_init(mmaDone, 1);
        *sAbort = 0;
        fence_mbar_init();
        prefetch_tmap(&tmWhi);
        prefetch_tmap(&tmWlo);
        for (int c = 0; c < F::kBufs; ++c) load_w(c);
    }
    if (warp == 0) tmem_alloc(sTmem, 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *sTmem;
    // the prologue above touched only this CTA's state and read-only tables
    grid_dep_wait();
    grid_dep_launch();
    constexpr uint32_t idesc = idesc_tf32(128);
    bool ok = true;
    int issued = F::kBufs;   // weight chunk loads issued

    // A chunk c: rows = samples, columns k = 2 i + re/im for i in [16 c, 16 c + 16); the
    // partials of chunk c + 1 are loaded while the MMAs of chunk c run
    constexpr int kPer = 128 * 16 / kMixTcThreads;   // (row, channel) pairs per thread
    float2 u[kPer][4];
    auto load_chunk = [&](int c) {
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            const int idx = threadIdx.x + kMixTcThreads * q;
            const int r = idx >> 4, i = 16 * c + (idx & 15);
            const int b = b0 + r < B ? b0 + r : B - 1;
            const float2* src = xpart + (static_cast<int64_t>(b) * nHB * M + m) * C + i;
            if (nHB == 4) {
#pragma unroll
                for (int hb = 0; hb < 4; ++hb) u[q][hb] = __ldg(src + static_cast<int64_t>(hb) * M * C);
            } else {
                u[q][0] = __ldg(src);
                for (int hb = 1; hb < nHB; ++hb) {
                    const float2 w = __ldg(src + static_cast<int64_t>(hb) * M * C);
                    u[q][0].x += w.x;
                    u[q][0].y += w.y;
                }
            }
        }
    };
    load_chunk(0);
    for (int c = 0; c < F::kChunks && ok; ++c) {
        if (c > 0 && !mbar_wait(mmaDone, (c - 1) & 1, sAbort)) {
            ok = false;
            break;
        }
        if (!PRE && c > 0) {
            if (threadIdx.x == 0) load_w(c);
            ++issued;
        }
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            const int idx = threadIdx.x + kMixTcThreads * q;
            const int r = idx >> 4, il = idx & 15;
            float2 v = u[q][0];
            if (nHB == 4) {
#pragma unroll
                for (int hb = 1; hb < 4; ++hb) {
                    v.x += u[q][hb].x;
                    v.y += u[q][hb].y;
                }
            }
            if (b0 + r >= B) v = make_float2(0.f, 0.f);
            float hr, lr, hi, li;
            split_tf32_m(v.x, hr, lr);
            split_tf32_m(v.y, hi, li);
            const uint32_t off = swz_offset(r * 128 + il * 8, 128);
            *reinterpret_cast<float2*>(sAhi + off) = make_float2(hr, hi);
            *reinterpret_cast<float2*>(sAlo + off) = make_float2(lr, li);
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
            const int q = c % F::kBufs;
            if (!mbar_wait(&bFull[q], (c / F::kBufs) & 1, sAbort)) {
                *sAbort = 1;
                atomicOr(err, kErrWaitTmaFull);
            } else {
                tc_fence_after();
                const uint32_t ahi = smem_u32(sAhi), alo = smem_u32(sAlo);
                const uint32_t bhi = smem_u32(sB + 2 * q * F::kTile), blo = bhi + F::kTile;
#pragma unroll
                for (int kk = 0; kk < F::kChunk / 8; ++kk) {
                    mma_tf32(tmem_base, umma_desc(ahi + kk * 32, 128), umma_desc(bhi + kk * 32, 128), idesc,
                             (c > 0 || kk > 0) ? 1u : 0u);
                    mma_tf32(tmem_base, umma_desc(alo + kk * 32, 128), umma_desc(bhi + kk * 32, 128), idesc, 1u);
                    mma_tf32(tmem_base, umma_desc(ahi + kk * 32, 128), umma_desc(blo + kk * 32, 128), idesc, 1u);
                }
                mma_commit(mmaDone);
            }
        }
        if (c + 1 < F::kChunks) load_chunk(c + 1);
        if (*sAbort) ok = false;
    }
    // the last chunk's MMAs
    if (ok && !mbar_wait(mmaDone, (F::kChunks - 1) & 1, sAbort)) ok = false;
    if (!ok) {
        if (threadIdx.x == 0) {
            atomicOr(err, kErrWaitAccFull);
            // the TMA loads already issued land before the CTA leaves
            if (PRE) {
                for (int q = 0; q < F::kBufs; ++q) mbar_wait_drain(&bFull[q], 0);
            } else {
                mbar_wait_drain(bFull, (issued - 1) & 1);
            }
        }
    } else if (warp < 4) {
        tc_fence_after();
        const int r = warp * 32 + lane;
        const int b = b0 + r;
        const uint32_t tb = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint32_t v[64];
            tmem_ld32(tb + h * 64, *reinterpret_cast<uint32_t(*)[32]>(v));
            tmem_ld32(tb + h * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
            tmem_wait_ld();
            asm volatile("" ::: "memory");
            if (b < B) {
                float4* dst = reinterpret_cast<float4*>(Y + (static_cast<int64_t>(b) * M + m) * C) + h * 16;
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    dst[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                         __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 128);
    }
}

// ---------------------------------------------------------------------------
// layer / projection: tcgen05 GEMM over 128-point tiles with fused epilogues.
//
// TMEM per accumulator stage: [0, C) int32 local-layer accumulator, [C, C+16)
// int32 sum_a (ones block), and with TCX [kX1Col, kX1Col + C) the fp32 spectral
// branch x1, produced by 3xTF32 tcgen05 MMAs:
//   x1[p][o] = sum_j Binv[p][j] * T[o][j],  j = 2 kw + {re, im},
//   Binv[p][2kw] = f cos(2 pi kw w/W)/W,  Binv[p][2kw+1] = -f sin(2 pi kw w/W)/W,
//   T[o][2kw] + i T[o][2kw+1] = sum_kh Y[kh][kw][o] e^{2 pi i kh h/H}/H,
// with each fp32 operand split into a tf32 "hi" part and the remainder "lo" and the
// product accumulated as hi*hi + lo*hi + hi*lo (error ~2^-21 relative).  TCX needs the
// tile to be one grid row (W == 128); narrower grids evaluate x1 on CUDA cores.
// ---------------------------------------------------------------------------
constexpr int kEpiWarp0 = 4;  // warp 0 TMA, warp 1 MMA/TMEM, epilogue warps from 4
constexpr int kLutMaxCells = kFno2dLutCells;

template <int C, int MH, int MW, bool PROJ, bool TCX>
struct LCfg {
    // 16 epilogue warps: 4 per TMEM lane quadrant, each owning C/4 columns
    static constexpr int kEpiWarps = 16;
    static constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
    static constexpr int kABytes = 128 * C;
    static constexpr int kStages = 3;
    static constexpr int kOnesCol = C;
    static constexpr int kX1Col = ((C + 16 + 31) / 32) * 32;
    static constexpr int kAccCols = TCX ? kX1Col + C : kX1Col;
    static constexpr int kAccStages = 2;
    static constexpr int kTmemCols = pow2ceil(kAccStages * kAccCols);
    static constexpr int kCols = C / 4;                   // columns per epilogue warp
    static constexpr int kCh = kCols;                     // columns per TMEM load
    static_assert(kCols == 16, "the epilogue is laid out for width 64");
    static constexpr int kRmax = 4;                       // rows per tile (W >= 32)
    static constexpr int kKx = 32;                        // padded K of the x1 MMA (fp32)
    static_assert(!TCX || 2 * MW <= kKx, "x1 MMA K");
    static constexpr int up1k(int v) { return (v + 1023) / 1024 * 1024; }
    static constexpr int kOffW = 0;
    static constexpr int kOffOnes = up1k(C * C);
    static constexpr int kOffA = kOffOnes + 1024;
    static constexpr int kOffStage = kOffA + kStages * kABytes;
    static constexpr int kOffY = kOffStage + (PROJ ? 0 : kEpiWarps * 2 * 512);
    // layer: cached spectrum Y of the current sample; projection: 2 x [128][C+1] activations
    static constexpr int kYBytes = PROJ ? 2 * 128 * (C + 1) * 4 : MH * MW * C * 8;
    static constexpr int kOffBinv = up1k(kOffY + kYBytes);
    static constexpr int kBinvBytes = TCX ? 2 * 128 * kKx * 4 : 0;        // hi, lo
    static constexpr int kOffTop = kOffBinv + kBinvBytes;
    static constexpr int kTopBytes = TCX ? 2 * 2 * C * kKx * 4 : 0;       // 2 buffers x (hi, lo)
    static constexpr int kOffT = kOffTop + kTopBytes;
    static constexpr int kTBytes = (PROJ || TCX) ? 0 : kRmax * MW * C * 8;
    static constexpr int kOffTw = kOffT + kTBytes;
    static constexpr int kTwBytes = (PROJ || TCX) ? 0 : MW * 128 * 8;
    static constexpr int kOffLut = kOffTw + kTwBytes;
    static constexpr int kLutBytes = PROJ ? 256 * 4 : kLutMaxCells * 8;   // code cells / act table
    static constexpr int kOffCol = kOffLut + kLutBytes;
    static constexpr int kColBytes = C * 16 + 4 * C * 4 + 16;           // params, proj_out w, b
    static constexpr int kOffBars = kOffCol + kColBytes;
    static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 2 + 1;
    static constexpr int kSmemBytes = kOffBars + 8 * kNumBars + 16 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "smem");
};

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
    hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
    lo = __fsub_rn(x, hi);
}

template <int C, int MH, int MW, bool PROJ, bool TCX>
__global__ void __launch_bounds__(LCfg<C, MH, MW, PROJ, TCX>::kThreads, 1)
layer_kernel(const __grid_constant__ CUtensorMap tmIn, const __grid_constant__ CUtensorMap tmOut,
             const LayerArgs p) {
    using L = LCfg<C, MH, MW, PROJ, TCX>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, derived by indexing the shared array so that the
    // compiler keeps shared-memory (not generic) loads and stores through it
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sW = smem + L::kOffW;
    uint8_t* sOnes = smem + L::kOffOnes;
    uint8_t* sA = smem + L::kOffA;
    uint8_t* sStage = smem + L::kOffStage;
    float2* sY = reinterpret_cast<float2*>(smem + L::kOffY);
    uint8_t* sBinv = smem + L::kOffBinv;
    uint8_t* sTop = smem + L::kOffTop;
    float2* sT = reinterpret_cast<float2*>(smem + L::kOffT);
    float2* sTw = reinterpret_cast<float2*>(smem + L::kOffTw);
    int2* sLut = reinterpret_cast<int2*>(smem + L::kOffLut);
    float* sAct = reinterpret_cast<float*>(smem + L::kOffLut);
    float* sG = reinterpret_cast<float*>(smem + L::kOffY);       // PROJ: [2][128][C+1]
    float4* sCol = reinterpret_cast<float4*>(smem + L::kOffCol);  // {sW*s_in, zp_w, zp_in*sum_w, bias}
    float* sWout = reinterpret_cast<float*>(sCol + C);            // [out_ch][C] (PROJ)
    float* sBout = sWout + 4 * C;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBars);
    uint64_t* empty = full + L::kStages;
    uint64_t* accFull = empty + L::kStages;
    uint64_t* accEmpty = accFull + L::kAccStages;
    uint64_t* tReady = accEmpty + L::kAccStages;
    uint64_t* epiBar = tReady + 2;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(epiBar + 1);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = static_cast<int>((p.M + 127) / 128);
    const int t_begin = static_cast<int>(static_cast<int64_t>(num_tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(num_tiles) * (blockIdx.x + 1) / gridDim.x);
    const bool use_lut = !PROJ && p.lut_cells > 0;
    const bool use_act = PROJ && p.act_table != nullptr && p.fq_out.kind == 1;

    // ---- set-up
    {
        constexpr int kChunks = C / 16;
        for (int idx = threadIdx.x; idx < C * kChunks; idx += L::kThreads) {
            const int o = idx / kChunks, c = idx % kChunks;
            const uint4 v = *reinterpret_cast<const uint4*>(p.Wq + o * C + c * 16);
            *reinterpret_cast<uint4*>(sW + swz_offset(o * C + c * 16, C)) = v;
        }
        for (int idx = threadIdx.x; idx < 1024 / 16; idx += L::kThreads) {
            const uint32_t one = (idx * 16 < C) ? 0x01010101u : 0u;  // row 0 = ones
            *reinterpret_cast<uint4*>(sOnes + idx * 16) = make_uint4(one, one, one, one);
        }
        for (int o = threadIdx.x; o < C; o += L::kThreads)
            sCol[o] = make_float4(__fmul_rn(p.scale_w[o], p.s_in), __int_as_float(p.zp_w[o]),
                                  __int_as_float(p.zp_in * p.sum_w[o]), p.bias[o]);
        if (PROJ) {
            for (int i = threadIdx.x; i < p.out_ch * C; i += L::kThreads) sWout[i] = p.w_out[i];
            for (int i = threadIdx.x; i < p.out_ch; i += L::kThreads) sBout[i] = p.b_out[i];
            if (use_act)
                for (int i = threadIdx.x; i < 256; i += L::kThreads) sAct[i] = p.act_table[i];
        } else {
            if (use_lut)
                for (int i = threadIdx.x; i < p.lut_cells; i += L::kThreads) sLut[i] = p.code_lut[i];
            if constexpr (TCX) {
                // Binv (A operand, 128 points x 32, SW128 K-major), hi and lo
                for (int idx = threadIdx.x; idx < 128 * L::kKx; idx += L::kThreads) {
                    const int w = idx / L::kKx, j = idx % L::kKx;
                    float v = 0.0f;
                    if (j < 2 * MW) {
                        const float2 t = p.twi_w[(j >> 1) * p.W + w];
                        v = (j & 1) ? -t.y : t.x;
                    }
                    float hi, lo;
                    split_tf32(v, hi, lo);
                    const uint32_t off = swz_offset(w * 128 + j * 4, 128);
                    *reinterpret_cast<float*>(sBinv + off) = hi;
                    *reinterpret_cast<float*>(sBinv + 128 * 128 + off) = lo;
                }
                // T operand buffers: zero (the K padding columns stay zero)
                for (int idx = threadIdx.x; idx < L::kTopBytes / 16; idx += L::kThreads)
                    reinterpret_cast<uint4*>(sTop)[idx] = make_uint4(0, 0, 0, 0);
            } else {
                for (int i = threadIdx.x; i < MW * p.W; i += L::kThreads) sTw[i] = p.twi_w[i];
            }
        }
        if (threadIdx.x == 0) {
            for (int s = 0; s < L::kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < L::kAccStages; ++s) {
                mbar_init(&accFull[s], 1);
                mbar_init(&accEmpty[s], L::kEpiWarps);
            }
            mbar_init(&tReady[0], L::kEpiWarps * 32);
            mbar_init(&tReady[1], L::kEpiWarps * 32);
            mbar_init(epiBar, L::kEpiWarps * 32);
            *sAbort = 0;
            fence_mbar_init();
        }
        if (warp == 1) tmem_alloc(sTmem, L::kTmemCols);
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
                const int s = it % L::kStages;
                const uint32_t ph = (it / L::kStages) & 1;
                if (!mbar_wait_backoff(&empty[s], ph ^ 1, sAbort, 1024)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitSlotFree);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], L::kABytes);
                tma_load_2d(sA + s * L::kABytes, &tmIn, &full[s], 0, tile * 128);
            }
            for (int j = (it > L::kStages ? it - L::kStages : 0); j < it; ++j)
                if (!mbar_wait_backoff(&full[j % L::kStages], (j / L::kStages) & 1, sAbort, 1024)) break;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one()) {
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % L::kStages;
                const uint32_t ph = (it / L::kStages) & 1;
                const int a = it % L::kAccStages;
                const uint32_t aph = (it / L::kAccStages) & 1;
                if (!mbar_wait_backoff(&accEmpty[a], aph ^ 1, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitAccFree);
                    break;
                }
                if (!mbar_wait_backoff(&full[s], ph, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitTmaFull);
                    break;
                }
                if constexpr (TCX && !PROJ) {
                    if (!mbar_wait_backoff(&tReady[it & 1], (it >> 1) & 1, sAbort, 128)) {
                        *sAbort = 1;
                        atomicOr(p.err, kErrWaitDrain);
                        break;
                    }
                }
                tc_fence_after();
                const uint32_t d = tmem_base + a * L::kAccCols;
                const uint32_t aBase = smem_u32(sA + s * L::kABytes);
#pragma unroll
                for (int kk = 0; kk < C / 32; ++kk) {
                    const uint64_t ad = umma_desc(aBase + kk * 32, C);
                    const uint64_t wd = umma_desc(smem_u32(sW) + kk * 32, C);
                    const uint64_t od = umma_desc(smem_u32(sOnes) + kk * 32, C);
                    mma_i8(d, ad, wd, idesc_i8(C), kk > 0 ? 1u : 0u);
                    mma_i8(d + L::kOnesCol, ad, od, idesc_i8(16), kk > 0 ? 1u : 0u);
                }
                if constexpr (TCX && !PROJ) {
                    const uint32_t dx = d + L::kX1Col;
                    const uint32_t bhi = smem_u32(sBinv), blo = bhi + 128 * 128;
                    const uint32_t thi = smem_u32(sTop) + (it & 1) * (2 * C * 128);
                    const uint32_t tlo = thi + C * 128;
                    constexpr uint32_t idx1 = idesc_tf32(C);
#pragma unroll
                    for (int kk = 0; kk < L::kKx / 8; ++kk)
                        mma_tf32(dx, umma_desc(bhi + kk * 32, 128), umma_desc(thi + kk * 32, 128),
                                 idx1, kk > 0 ? 1u : 0u);
#pragma unroll
                    for (int kk = 0; kk < L::kKx / 8; ++kk)
                        mma_tf32(dx, umma_desc(blo + kk * 32, 128), umma_desc(thi + kk * 32, 128),
                                 idx1, 1u);
#pragma unroll
                    for (int kk = 0; kk < L::kKx / 8; ++kk)
                        mma_tf32(dx, umma_desc(bhi + kk * 32, 128), umma_desc(tlo + kk * 32, 128),
                                 idx1, 1u);
                }
                mma_commit(&empty[s]);
                mma_commit(&accFull[a]);
            }
            if (it > 0) {
                const int j = it - 1;
                mbar_wait_backoff(&accFull[j % L::kAccStages], (j / L::kAccStages) & 1, sAbort, 1024);
            }
        }
        __syncwarp();
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + L::kEpiWarps) {
        const int ew = warp - kEpiWarp0;
        const int etid = ew * 32 + lane;
        constexpr int kEpiThreads = L::kEpiWarps * 32;
        const int quad = warp & 3;
        const int col0 = (ew >> 2) * L::kCols;  // this warp's 16 columns
        const int row = quad * 32 + lane;  // row of the 128-point tile
        const int P = p.H * p.W;
        const int R = 128 / p.W > 0 ? 128 / p.W : 1;
        const float s_out = p.fq_out.scale, inv_out = p.fq_out.inv_scale;
        const float zpo = static_cast<float>(p.fq_out.zp);
        const float klo = -128.0f - zpo, khi = 127.0f - zpo;         // code offsets' range
        const float lut_c = __fmul_rn(-p.lut_zlo, p.lut_inv_delta);  // table index offset
        int cached_b = -1;
        int it = 0, nstore = 0;
        uint32_t nsync = 0;
        // all epilogue threads meet here; bounded, so a missing peer turns into an abort
        auto epi_sync = [&]() -> bool {
            mbar_arrive(epiBar);
            const bool ok = mbar_wait(epiBar, nsync & 1u, sAbort);
            ++nsync;
            return ok;
        };
        bool epi_ok = true;
        // reload the cached spectrum when tile `tile` belongs to another sample
        auto ensure_y = [&](int tile) -> bool {
            const int b = static_cast<int>(static_cast<int64_t>(tile) * 128 / P);
            if (b == cached_b) return true;
            if (!epi_sync()) return false;
            const float4* src = reinterpret_cast<const float4*>(p.Y + static_cast<int64_t>(b) * MH * MW * C);
            float4* dst = reinterpret_cast<float4*>(sY);
            for (int i = etid; i < MH * MW * C / 2; i += kEpiThreads) dst[i] = src[i];
            cached_b = b;
            return epi_sync();
        };
        // TCX: T of tile `tile` into operand buffer `buf` (hi/lo tf32 split, SW128 rows o)
        auto compute_top = [&](int tile, int buf) {
            const int64_t g0 = static_cast<int64_t>(tile) * 128;
            const int h = static_cast<int>((g0 % P) / p.W);
            float2 eh[MH];
#pragma unroll
            for (int kh = 0; kh < MH; ++kh) eh[kh] = __ldg(p.twi_h + h * MH + kh);
            uint8_t* thi = sTop + buf * (2 * C * 128);
            uint8_t* tlo = thi + C * 128;
            for (int idx = etid; idx < MW * C; idx += kEpiThreads) {
                const int kw = idx / C, o = idx % C;
                float tr = 0.f, ti = 0.f;
#pragma unroll
                for (int kh = 0; kh < MH; ++kh) {
                    const float2 y = sY[(kh * MW + kw) * C + o];
                    tr = fmaf(y.x, eh[kh].x, fmaf(-y.y, eh[kh].y, tr));
                    ti = fmaf(y.x, eh[kh].y, fmaf(y.y, eh[kh].x, ti));
                }
                float h0, l0, h1, l1;
                split_tf32(tr, h0, l0);
                split_tf32(ti, h1, l1);
                const uint32_t o0 = swz_offset(o * 128 + (2 * kw) * 4, 128);
                const uint32_t o1 = swz_offset(o * 128 + (2 * kw + 1) * 4, 128);
                *reinterpret_cast<float*>(thi + o0) = h0;
                *reinterpret_cast<float*>(thi + o1) = h1;
                *reinterpret_cast<float*>(tlo + o0) = l0;
                *reinterpret_cast<float*>(tlo + o1) = l1;
            }
            fence_proxy_async_smem();
            mbar_arrive(&tReady[buf]);
        };
        if constexpr (TCX && !PROJ) {
            if (t_begin < t_end) {
                if (!ensure_y(t_begin)) epi_ok = false;
                else compute_top(t_begin, 0);
            }
        }
        for (int tile = t_begin; tile < t_end && epi_ok; ++tile, ++it) {
            const int64_t g0 = static_cast<int64_t>(tile) * 128;
            const int p0 = static_cast<int>(g0 % P);
            if constexpr (!PROJ) {
                if constexpr (TCX) {
                    if (tile + 1 < t_end) {
                        if (!ensure_y(tile + 1)) {
                            epi_ok = false;
                            break;
                        }
                        compute_top(tile + 1, (it + 1) & 1);
                    }
                } else {
                    // inverse transform along H for this tile's rows: T[r][kw][o]
                    if (!ensure_y(tile)) {
                        epi_ok = false;
                        break;
                    }
                    const int h0 = p0 / p.W;
                    for (int idx = etid; idx < R * MW * C; idx += kEpiThreads) {
                        const int r = idx / (MW * C), rem = idx % (MW * C);
                        const int kw = rem / C, o = rem % C;
                        const float2* eh = p.twi_h + (h0 + r) * MH;
                        float tr = 0.f, ti = 0.f;
#pragma unroll
                        for (int kh = 0; kh < MH; ++kh) {
                            const float2 y = sY[(kh * MW + kw) * C + o];
                            const float2 e = __ldg(eh + kh);
                            tr = fmaf(y.x, e.x, fmaf(-y.y, e.y, tr));
                            ti = fmaf(y.x, e.y, fmaf(y.y, e.x, ti));
                        }
                        sT[idx] = make_float2(tr, ti);
                    }
                    if (!epi_sync()) {
                        epi_ok = false;
                        break;
                    }
                }
            }
            const int a = it % L::kAccStages;
            const uint32_t aph = (it / L::kAccStages) & 1;
            if (!mbar_wait(&accFull[a], aph, sAbort)) {
                *sAbort = 1;
                atomicOr(p.err, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + a * L::kAccCols;
            uint32_t sum_u;
            tmem_ld1(tbase + L::kOnesCol, sum_u);
            tmem_wait_ld();
            const int rconst = C * p.zp_in - 2 * static_cast<int>(sum_u);
            // this point's position inside the tile's rows and its W twiddles (CUDA-core x1)
            const int pr = (p0 % p.W + row) / p.W;
            const int pw = (p0 + row) % p.W;
            float2 ew_reg[MW];
            if constexpr (!PROJ && !TCX) {
#pragma unroll
                for (int kw = 0; kw < MW; ++kw) ew_reg[kw] = sTw[kw * p.W + pw];
            }
            float acc_out[4];
            if constexpr (PROJ) {
#pragma unroll
                for (int j = 0; j < 4; ++j) acc_out[j] = j < p.out_ch ? sBout[j] : 0.0f;
            }
#pragma unroll 1
            for (int c0 = col0; c0 < col0 + L::kCols; c0 += L::kCh) {
                uint32_t raw[32];
                uint32_t x1r[32];
                tmem_ld16(tbase + c0, raw);
                if constexpr (TCX && !PROJ) tmem_ld16(tbase + L::kX1Col + c0, x1r);
                tmem_wait_ld();
                const bool last_chunk = c0 + L::kCh >= col0 + L::kCols;
                // The fast, branch-free pass over the chunk; elements whose fake-quant
                // quotient lies next to a half-integer are fixed afterwards with the
                // exact division (their accumulators are re-read from TMEM).
                uint32_t bad = 0;
                if constexpr (PROJ) {
                    float g[32];
#pragma unroll
                    for (int j = 0; j < L::kCh; ++j) {
                        const float4 cp = sCol[c0 + j];
                        const int vint = static_cast<int>(raw[j]) + __float_as_int(cp.y) * rconst -
                                         __float_as_int(cp.z);
                        const float v = __fadd_rn(__fmul_rn(cp.x, __int2float_rn(vint)), cp.w);
                        if (use_act) {
                            bool b;
                            const float q = fq_code_try(v, inv_out, zpo, b);
                            bad |= static_cast<uint32_t>(b) << j;
                            g[j] = sAct[static_cast<int>(q) + 128];
                        } else {
                            g[j] = activation(apply_fq(v, p.fq_out), p.act);
                        }
                    }
                    uint32_t any = __reduce_or_sync(0xffffffffu, bad);
                    while (any) {
                        const int j = __ffs(any) - 1;
                        any &= any - 1;
                        uint32_t rj;
                        tmem_ld1(tbase + c0 + j, rj);
                        tmem_wait_ld();
                        if (bad & (1u << j)) {
                            const float4 cp = sCol[c0 + j];
                            const int vint = static_cast<int>(rj) + __float_as_int(cp.y) * rconst -
                                             __float_as_int(cp.z);
                            const float v = __fadd_rn(__fmul_rn(cp.x, __int2float_rn(vint)), cp.w);
                            const float gj = sAct[static_cast<int>(fq_code(v, s_out, zpo)) + 128];
#pragma unroll
                            for (int k = 0; k < 32; ++k)
                                if (k == j) g[k] = gj;
                        }
                    }
                    if (last_chunk) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&accEmpty[a]);
                    }
                    float* grow = sG + (it & 1) * (128 * (C + 1)) + row * (C + 1) + c0;
#pragma unroll
                    for (int j = 0; j < L::kCh; ++j) grow[j] = g[j];
                } else {
                    // x1 of element j (tensor-core result, or CUDA-core inverse W-DFT)
                    auto x1_of = [&](int j, uint32_t xbits) -> float {
                        if constexpr (TCX) {
                            return __uint_as_float(xbits);
                        } else {
                            const float2* trow = sT + (pr * MW) * C + c0 + j;
                            float x1 = 0.f;
#pragma unroll
                            for (int kw = 0; kw < MW; ++kw) {
                                const float2 t = trow[kw * C];
                                x1 = fmaf(t.x, ew_reg[kw].x, fmaf(-t.y, ew_reg[kw].y, x1));
                            }
                            return x1;
                        }
                    };
                    auto code_of = [&](float z) -> int {
                        if (use_lut) {
                            const bool s0 = z < p.lut_split && p.lut_two;
                            const int2 cell = lut_cell(z, sLut, p.lut_cells, s0 ? p.lut_inv0 : (p.lut_two ? p.lut_inv1 : p.lut_inv_delta),
                                                       s0 ? p.lut_c0 : (p.lut_two ? p.lut_c1 : lut_c));
                            const int w = z >= __int_as_float(cell.x) ? (cell.y >> 8) : cell.y;
                            return static_cast<int>(static_cast<int8_t>(w & 0xFF));
                        }
                        return static_cast<int>(fq_code(activation(z, p.act), s_out, zpo));
                    };
                    // Per element: dequantise + bias, the fast fake-quant offset k (x2 =
                    // k * s exactly), z = x1 + x2, and the next code, inserted into the
                    // packed word with one byte permute: the table cell's bytes hold the
                    // codes below / from its breakpoint, the selector picks one.
                    uint32_t packed[8];
                    auto chunk = [&](auto lut_tag) {
#pragma unroll
                        for (int j = 0; j < L::kCh; ++j) {
                            const float x1 = x1_of(j, x1r[j]);
                            const float4 cp = sCol[c0 + j];
                            const int vint = static_cast<int>(raw[j]) + __float_as_int(cp.y) * rconst -
                                             __float_as_int(cp.z);
                            const float v = __fadd_rn(__fmul_rn(cp.x, __int2float_rn(vint)), cp.w);
                            bool b;
                            const float kq = fq_offset_try(v, inv_out, klo, khi, b);
                            bad |= static_cast<uint32_t>(b) << j;
                            const float z = __fadd_rn(x1, __fmul_rn(kq, s_out));
                            const uint32_t prev = (j & 3) == 0 ? 0u : packed[j >> 2];
                            const uint32_t sel_lo = (0x3210u & ~(0xFu << (4 * (j & 3)))) | (4u << (4 * (j & 3)));
                            if constexpr (decltype(lut_tag)::value != 0) {
                                int2 cell;
                                if constexpr (decltype(lut_tag)::value == 2) {
                                    const bool s0 = z < p.lut_split;
                                    cell = lut_cell(z, sLut, p.lut_cells, s0 ? p.lut_inv0 : p.lut_inv1,
                                                    s0 ? p.lut_c0 : p.lut_c1);
                                } else {
                                    cell = lut_cell(z, sLut, p.lut_cells, p.lut_inv_delta, lut_c);
                                }
                                const uint32_t sel = z >= __int_as_float(cell.x) ? sel_lo + (1u << (4 * (j & 3))) : sel_lo;
                                packed[j >> 2] = __byte_perm(prev, static_cast<uint32_t>(cell.y), sel);
                            } else {
                                packed[j >> 2] = __byte_perm(prev, static_cast<uint32_t>(code_of(z)), sel_lo);
                            }
                        }
                    };
                    if (use_lut && p.lut_two) chunk(std::integral_constant<int, 2>{});
                    else if (use_lut) chunk(std::integral_constant<int, 1>{});
                    else chunk(std::integral_constant<int, 0>{});
                    uint8_t* buf = sStage + (ew * 2 + (nstore & 1)) * 512;
                    if (nstore >= 2) {
                        if (lane == 0) tma_store_wait_read<1>();
                        __syncwarp();
                    }
                    constexpr int kRow = L::kCh;  // bytes per row of this warp's half tile
#pragma unroll
                    for (int j16 = 0; j16 < kRow / 16; ++j16) {
                        const uint32_t off = (kRow == 32) ? swz_offset(lane * 32 + j16 * 16, 32)
                                                          : static_cast<uint32_t>(lane * 16);
                        *reinterpret_cast<uint4*>(buf + off) =
                            make_uint4(packed[4 * j16], packed[4 * j16 + 1], packed[4 * j16 + 2],
                                       packed[4 * j16 + 3]);
                    }
                    uint32_t any = __reduce_or_sync(0xffffffffu, bad);
                    while (any) {
                        const int j = __ffs(any) - 1;
                        any &= any - 1;
                        uint32_t rj, xj = 0;
                        tmem_ld1(tbase + c0 + j, rj);
                        if constexpr (TCX) tmem_ld1(tbase + L::kX1Col + c0 + j, xj);
                        tmem_wait_ld();
                        if (bad & (1u << j)) {
                            const float4 cp = sCol[c0 + j];
                            const int vint = static_cast<int>(rj) + __float_as_int(cp.y) * rconst -
                                             __float_as_int(cp.z);
                            const float v = __fadd_rn(__fmul_rn(cp.x, __int2float_rn(vint)), cp.w);
                            const float x2 = __fmul_rn(__fsub_rn(fq_code(v, s_out, zpo), zpo), s_out);
                            const int code = code_of(__fadd_rn(x1_of(j, xj), x2));
                            const uint32_t off = (kRow == 32)
                                                     ? swz_offset(lane * 32 + (j >> 4) * 16, 32) + (j & 15)
                                                     : static_cast<uint32_t>(lane * 16 + j);
                            buf[off] = static_cast<uint8_t>(code & 0xFF);
                        }
                    }
                    if (last_chunk) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&accEmpty[a]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmOut, buf, c0, static_cast<int>(g0) + quad * 32);
                        tma_store_commit();
                    }
                    ++nstore;
                }
            }
            if constexpr (PROJ) {
                // the 64 activations of every row are in shared memory; the first warp of
                // each lane quadrant runs the reference's sequential proj_out dot product
                if (!epi_sync()) {
                    epi_ok = false;
                    break;
                }
                if (ew >= 4) continue;
                const float* grow = sG + (it & 1) * (128 * (C + 1)) + row * (C + 1);
#pragma unroll
                for (int o = 0; o < C; ++o) {
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj)
                        if (jj < p.out_ch)
                            acc_out[jj] = linear_step(acc_out[jj], grow[o], sWout[jj * C + o],
                                                      o >= linear_unfused_len(C));
                }
                const int64_t m = g0 + row;
                if (m < p.M) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (j >= p.out_ch) break;
                        float yv = acc_out[j];
                        if (p.fq_final.kind == 1) {
                            const float zf = static_cast<float>(p.fq_final.zp);
                            const float q = fq_code_fast(yv, p.fq_final.scale, p.fq_final.inv_scale, zf);
                            yv = __fmul_rn(__fsub_rn(q, zf), p.fq_final.scale);
                        } else {
                            yv = apply_fq(yv, p.fq_final);
                        }
                        p.y[m * p.out_ch + j] = yv;
                    }
                }
            } else if constexpr (!TCX) {
                // every epilogue thread is done with sT before the next tile rewrites it
                if (!epi_sync()) {
                    epi_ok = false;
                    break;
                }
            }
        }
        if (!epi_ok) {
            *sAbort = 1;
            atomicOr(p.err, kErrWaitDrain);
        }
        if (lane == 0) tma_store_wait_all<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

// Wait for this thread's outstanding tcgen05.ld; naming the destination registers
// keeps their uses after the wait.
__device__ __forceinline__ void tmem_wait_ld16(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// ---------------------------------------------------------------------------
// layer_tc: the local layer + spectral branch of one FNO2d layer on W == 128 grids
// (one 128-point tile = one grid row), with the work split over warp roles:
//   warp 0       TMA producer of the layer-input codes (ring of kStages tiles)
//   warp 1       MMA issuer and TMEM owner: per tile the int8 local GEMM, the ones
//                block (sum_a) and the 3xTF32 inverse W-transform x1 = Binv T
//   warps 2-7    T builders: the H-direction inverse
//                transform T[o][kw] of the tile's rows from the cached spectrum Y,
//                four rows per pass (tile_row's groups), split into tf32 hi/lo
//                halves, four T buffers
//   warps 8-23   epilogue: two groups of 8 warps take turns over the tiles; in a
//                group, 2 warps per TMEM lane quadrant, 32 columns each.  Per
//                element: dequantise + bias (one 16-byte constant load per field
//                and four columns), the fast fake-quant offset k, z = x1 + k s, the
//                next code from the table, the products two columns per f32x2
//                instruction; 16 packed codes per thread and chunk go out as one
//                16-byte store.
// Four accumulator stages (all 512 TMEM columns): each epilogue group alternates
// between two stages, so the MMA of tile t + 4 has a whole group tile period to land
// after its group released tile t; a group waits on a stage only after it drained the
// stage's previous tile itself, so parity waits stay exact.
// ---------------------------------------------------------------------------
template <int C, int MH, int MW>
struct TCfg {
    static constexpr int kTBuild0 = 2;                  // first T-builder warp
    static constexpr int kTBuildWarps = 6;
    static constexpr int kEpi0 = kTBuild0 + kTBuildWarps;  // quadrant = warp & 3
    static constexpr int kEpiWarps = 16;
    static constexpr int kThreads = 32 * (kEpi0 + kEpiWarps);
    static constexpr int kABytes = 128 * C;
    static constexpr int kStages = 3;
    static constexpr int kX1Col = C;
    static constexpr int kAccCols = kX1Col + C;
    static constexpr int kAccStages = 4;
    static constexpr int kTmemCols = pow2ceil(kAccStages * kAccCols);
    // x1 MMA operands: K = 2 MW = 24 (kw, re/im) in three K-blocks of 8 fp32, each a
    // 32-byte-row SW32 tile (Binv: 128 points x 8, T: C outputs x 8)
    static constexpr int kKb = 3;
    static_assert(2 * MW == 8 * kKb, "x1 MMA K");
    static constexpr int kBinvBlk = 128 * 32;
    static constexpr int kTBlk = C * 32;
    static constexpr int kTBufs = 4;                    // T operand buffers (two tile pairs)
    static_assert(C == 64, "the epilogue is laid out for width 64");
    static constexpr int up1k(int v) { return (v + 1023) / 1024 * 1024; }
    static constexpr int kOffW = 0;
    static constexpr int kOffZ = up1k(C * C);                           // [3][C][32] int8
    static constexpr int kOffA = kOffZ + up1k(3 * C * 32);
    static constexpr int kOffY = kOffA + kStages * kABytes;
    static constexpr int kYBytes = MH * MW * C * 8;
    static constexpr int kOffBinv = up1k(kOffY + kYBytes);
    static constexpr int kBinvBytes = 2 * kKb * kBinvBlk;               // hi, lo
    static constexpr int kOffTop = kOffBinv + kBinvBytes;
    static constexpr int kTBuf = 2 * kKb * kTBlk;                       // hi, lo of one T
    static constexpr int kTopBytes = kTBufs * kTBuf;
    static constexpr int kOffLut = kOffTop + kTopBytes;
    static constexpr int kLutBytes = kFno2dLutCellsTc * 8;
    static constexpr int kOffCol = kOffLut + kLutBytes;                // float4 [C]
    static constexpr int kOffBars = kOffCol + C * 16;
    static constexpr int kNumBars = 2 * kStages + 2 * kAccStages + 2 * kTBufs;
    static constexpr int kSmemBytes = kOffBars + 8 * kNumBars + 16 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "smem");
};

__device__ __forceinline__ void tmem_wait_ld_33(uint32_t (&a)[16], uint32_t (&b)[16], uint32_t& c) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]),
                   "+r"(a[6]), "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]),
                   "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]), "+r"(b[0]), "+r"(b[1]),
                   "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]),
                   "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]),
                   "+r"(b[14]), "+r"(b[15]), "+r"(c)
                 :
                 : "memory");
}

// Table cell of z in the saturating form: u = sat(fma(z, alpha, beta)) (NaN -> 0),
// idx = rint(u * nm1) read from the bits of fma(u, nm1, 1.5 * 2^23).
__device__ __forceinline__ int2 lut_cell_sat(float z, const int2* lut, float alpha, float beta,
                                             float nm1) {
    const float u = __saturatef(__fmaf_rn(z, alpha, beta));
    const float x = __fmaf_rn(u, nm1, kMagic);
    return lut[__float_as_int(x) - 0x4B400000];
}

template <int C, int MH, int MW, bool TWO>
__global__ void __launch_bounds__(TCfg<C, MH, MW>::kThreads, 1)
layer_tc_kernel(const __grid_constant__ CUtensorMap tmIn,
                const LayerArgs p, const __grid_constant__ LayerCols cols) {
    using L = TCfg<C, MH, MW>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sW = smem + L::kOffW;
    uint8_t* sZ = smem + L::kOffZ;
    uint8_t* sA = smem + L::kOffA;
    float2* sY = reinterpret_cast<float2*>(smem + L::kOffY);
    uint8_t* sBinv = smem + L::kOffBinv;
    uint8_t* sTop = smem + L::kOffTop;
    int2* sLut = reinterpret_cast<int2*>(smem + L::kOffLut);
    float4* sCol = reinterpret_cast<float4*>(smem + L::kOffCol);  // {a, zp, nk, b} per column
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBars);
    uint64_t* empty = full + L::kStages;
    uint64_t* accFull = empty + L::kStages;
    uint64_t* accEmpty = accFull + L::kAccStages;
    uint64_t* tReady = accEmpty + L::kAccStages;
    uint64_t* tFree = tReady + L::kTBufs;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(tFree + L::kTBufs);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = static_cast<int>((p.M + 127) / 128);
    const int t_begin = static_cast<int>(static_cast<int64_t>(num_tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(num_tiles) * (blockIdx.x + 1) / gridDim.x);
    // Logical tile L (the CTA loop order) -> grid row (one 128-point tile is one row,
    // W == 128).  Within a sample the logical tiles come in groups of four, group g >= 1
    // being the rows g, g + H/2, H - g and H/2 - g (whose H-direction twiddles are those
    // of row g times (-1)^kh and/or conjugated), group 0 the rows 0, H/2, H/4, 3H/4.
    auto tile_row = [&](int Lt) -> int {
        const int b = Lt / p.H;
        const int r = Lt - b * p.H;
        const int g = r >> 2, k = r & 3;
        const int h2 = p.H >> 1;
        const int row = g == 0 ? (k & 1) * h2 + (k >> 1) * (p.H >> 2)
                               : (k < 2 ? g : (k == 2 ? p.H - g : h2 - g)) + (k == 1 ? h2 : 0);
        return b * p.H + row;
    };

    // ---- set-up
    {
        constexpr int kChunks = C / 16;
        for (int idx = threadIdx.x; idx < C * kChunks; idx += L::kThreads) {
            const int o = idx / kChunks, c = idx % kChunks;
            const uint4 v = *reinterpret_cast<const uint4*>(p.Wq + o * C + c * 16);
            *reinterpret_cast<uint4*>(sW + swz_offset(o * C + c * 16, C)) = v;
        }
        // Z blocks: one value per row, so the 32-byte swizzle leaves them unchanged
        for (int idx = threadIdx.x; idx < 3 * C * 32 / 16; idx += L::kThreads)
            reinterpret_cast<uint4*>(sZ)[idx] = reinterpret_cast<const uint4*>(p.zrows)[idx];
        for (int i = threadIdx.x; i < p.lut_cells; i += L::kThreads) sLut[i] = p.code_lut[i];
        for (int o = threadIdx.x; o < C; o += L::kThreads)
            sCol[o] = cols.v[o];
        // Binv (A operand of the x1 MMA, 128 points x 24 in three SW32 K-blocks), hi, lo
        for (int idx = threadIdx.x; idx < 128 * 2 * MW; idx += L::kThreads) {
            const int w = idx / (2 * MW), j = idx % (2 * MW);
            const float2 t = p.twi_w[(j >> 1) * p.W + w];
            const float v = (j & 1) ? -t.y : t.x;
            float hi, lo;
            split_tf32(v, hi, lo);
            const uint32_t off = (j >> 3) * L::kBinvBlk + swz_offset(w * 32 + (j & 7) * 4, 32);
            *reinterpret_cast<float*>(sBinv + off) = hi;
            *reinterpret_cast<float*>(sBinv + L::kKb * L::kBinvBlk + off) = lo;
        }
        if (threadIdx.x == 0) {
            for (int s = 0; s < L::kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < L::kAccStages; ++s) {
                mbar_init(&accFull[s], 1);
                mbar_init(&accEmpty[s], L::kEpiWarps / 2);
            }
            for (int b = 0; b < L::kTBufs; ++b) {
                mbar_init(&tReady[b], L::kTBuildWarps * 32);
                mbar_init(&tFree[b], 1);
            }
            *sAbort = 0;
            fence_mbar_init();
        }
        if (warp == 1) tmem_alloc(sTmem, L::kTmemCols);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    const uint32_t tmem_base = *sTmem;
    // the prologue above touched only this CTA's state and read-only tables
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (elect_one()) {
            prefetch_tmap(&tmIn);
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % L::kStages;
                const uint32_t ph = (it / L::kStages) & 1;
                if (!mbar_wait_backoff(&empty[s], ph ^ 1, sAbort, 1024)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitSlotFree);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], L::kABytes);
                tma_load_2d(sA + s * L::kABytes, &tmIn, &full[s], 0, tile_row(tile) * 128);
            }
            for (int j = (it > L::kStages ? it - L::kStages : 0); j < it; ++j)
                if (!mbar_wait_backoff(&full[j % L::kStages], (j / L::kStages) & 1, sAbort, 1024)) break;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one()) {
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % L::kStages;
                const uint32_t ph = (it / L::kStages) & 1;
                const int a = it % L::kAccStages;
                const uint32_t aph = (it / L::kAccStages) & 1;
                const int b = it % L::kTBufs;
                if (!mbar_wait_backoff(&accEmpty[a], aph ^ 1, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitAccFree);
                    break;
                }
                if (!mbar_wait_backoff(&full[s], ph, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitTmaFull);
                    break;
                }
                if (!mbar_wait_backoff(&tReady[b], (it / L::kTBufs) & 1, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitDrain);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + a * L::kAccCols;
                const uint32_t aBase = smem_u32(sA + s * L::kABytes);
#pragma unroll
                for (int kk = 0; kk < C / 32; ++kk) {
                    const uint64_t ad = umma_desc(aBase + kk * 32, C);
                    const uint64_t wd = umma_desc(smem_u32(sW) + kk * 32, C);
                    mma_i8(d, ad, wd, idesc_i8(C), kk > 0 ? 1u : 0u);
                    // + sum_k a_k z_q: the same 32-column Z block serves both K halves
                    for (int q = 0; q < p.nz; ++q)
                        mma_i8(d, ad, umma_desc(smem_u32(sZ) + q * C * 32, 32), idesc_i8(C), 1u);
                }
                {
                    const uint32_t dx = d + L::kX1Col;
                    const uint32_t bhi = smem_u32(sBinv), blo = bhi + L::kKb * L::kBinvBlk;
                    const uint32_t thi = smem_u32(sTop) + b * L::kTBuf;
                    const uint32_t tlo = thi + L::kKb * L::kTBlk;
                    constexpr uint32_t idx1 = idesc_tf32(C);
#pragma unroll
                    for (int kk = 0; kk < L::kKb; ++kk)
                        mma_tf32(dx, umma_desc(bhi + kk * L::kBinvBlk, 32), umma_desc(thi + kk * L::kTBlk, 32),
                                 idx1, kk > 0 ? 1u : 0u);
#pragma unroll
                    for (int kk = 0; kk < L::kKb; ++kk)
                        mma_tf32(dx, umma_desc(blo + kk * L::kBinvBlk, 32), umma_desc(thi + kk * L::kTBlk, 32),
                                 idx1, 1u);
#pragma unroll
                    for (int kk = 0; kk < L::kKb; ++kk)
                        mma_tf32(dx, umma_desc(bhi + kk * L::kBinvBlk, 32), umma_desc(tlo + kk * L::kTBlk, 32),
                                 idx1, 1u);
                }
                mma_commit(&empty[s]);
                mma_commit(&accFull[a]);
                mma_commit(&tFree[b]);
            }
            if (it > 0) {
                const int j = it - 1;
                mbar_wait_backoff(&accFull[j % L::kAccStages], (j / L::kAccStages) & 1, sAbort, 1024);
            }
        }
        __syncwarp();
    } else if (warp >= L::kTBuild0 && warp < L::kEpi0) {
        // ---------------- T builders
        // One pass over the cached spectrum per group of four logical tiles (tile_row):
        // with e = e(g, kh) the twiddle of row g, the rows g + H/2, H - g and H/2 - g have
        // twiddles (-1)^kh e, conj(e) and (-1)^kh conj(e).  Per parity class of kh (E, O)
        // the four sums Rc = sum Yr c, Is = sum Yi s, Rs = sum Yr s, Ic = sum Yi c give
        //   T(g)       = (Rc - Is) + i (Rs + Ic)   summed E + O,
        //   T(g + H/2) = the same, E - O,
        //   T(H - g)   = (Rc + Is) + i (Ic - Rs)   summed E + O,
        //   T(H/2 - g) = the same, E - O.
        // Group 0 takes two passes: g = 0 for rows 0, H/2 and g = H/4 for H/4, 3H/4.
        const int ctid = (warp - L::kTBuild0) * 32 + lane;
        constexpr int kBT = L::kTBuildWarps * 32;
        constexpr int kPer = MW * C / kBT;                   // (kw, o) pairs per thread
        static_assert(MW * C % kBT == 0, "T builder layout");
        static_assert(MH % 2 == 0, "parity classes");
        const int o = ctid % C;
        int cached_b = -1;
        bool ok = true;
        for (int L0 = t_begin & ~3; L0 < t_end && ok; L0 += 4) {
            const int first = L0 > t_begin ? L0 : t_begin;
            const int last = L0 + 4 < t_end ? L0 + 4 : t_end;
            const int smp = L0 / p.H;
            const int g = (L0 - smp * p.H) >> 2;
            if (smp != cached_b) {
                // each builder caches exactly the spectrum entries it reads below, so the
                // reload needs no barrier among the builders
                const float2* src = p.Y + static_cast<int64_t>(smp) * MH * MW * C;
#pragma unroll 1
                for (int r = 0; r < kPer; ++r) {
                    const int kw = (ctid + kBT * r) / C;
#pragma unroll
                    for (int kh = 0; kh < MH; ++kh)
                        sY[(kh * MW + kw) * C + o] = __ldg(src + (kh * MW + kw) * C + o);
                }
                cached_b = smp;
            }
            for (int pass = 0; pass < (g == 0 ? 2 : 1) && ok; ++pass) {
                const int h = g == 0 ? pass * (p.H >> 2) : g;
                const int m0 = g == 0 ? 2 * pass : 0, m1 = g == 0 ? m0 + 2 : 4;  // members
                if (L0 + m1 <= first || L0 + m0 >= last) continue;
                float acc[kPer][8];  // per pair: E {Rc, Is, Rs, Ic}, O {Rc, Is, Rs, Ic}
#pragma unroll
                for (int r = 0; r < kPer; ++r)
#pragma unroll
                    for (int q = 0; q < 8; ++q) acc[r][q] = 0.0f;
#pragma unroll
                for (int kh = 0; kh < MH; ++kh) {
                    const float2 e = __ldg(p.twi_h + h * MH + kh);
                    const float2 es = make_float2(e.y, e.x);
#pragma unroll
                    for (int r = 0; r < kPer; ++r) {
                        const int kw = (ctid + kBT * r) / C;
                        const float2 y = sY[(kh * MW + kw) * C + o];
                        float* a = acc[r] + (kh & 1) * 4;
                        const float2 a01 = fma2_rn(y, e, make_float2(a[0], a[1]));
                        const float2 a23 = fma2_rn(y, es, make_float2(a[2], a[3]));
                        a[0] = a01.x;
                        a[1] = a01.y;
                        a[2] = a23.x;
                        a[3] = a23.y;
                    }
                }
                for (int k = m0; k < m1; ++k) {
                    const int Lk = L0 + k;
                    if (Lk < first || Lk >= last) continue;
                    const int itk = Lk - t_begin;
                    const int bq = itk % L::kTBufs;
                    if (!mbar_wait_backoff(&tFree[bq], ((itk / L::kTBufs) & 1) ^ 1, sAbort, 256)) {
                        *sAbort = 1;
                        atomicOr(p.err, kErrWaitDrain);
                        ok = false;
                        break;
                    }
                    const bool conj = g != 0 && k >= 2;     // rows H - g, H/2 - g
                    const bool minus = (k & 1) != 0;        // E - O
                    uint8_t* tb = sTop + bq * L::kTBuf;
#pragma unroll
                    for (int r = 0; r < kPer; ++r) {
                        const int kw = (ctid + kBT * r) / C;
                        const float* E = acc[r];
                        const float* O = acc[r] + 4;
                        const float er = conj ? E[0] + E[1] : E[0] - E[1];
                        const float ei = conj ? E[3] - E[2] : E[2] + E[3];
                        const float orr = conj ? O[0] + O[1] : O[0] - O[1];
                        const float oi = conj ? O[3] - O[2] : O[2] + O[3];
                        // element (o, j = 2 kw + re/im): K-block j / 8, column j % 8
                        const uint32_t off = (kw >> 2) * L::kTBlk + swz_offset(o * 32 + (2 * kw & 7) * 4, 32);
                        constexpr int kLo = L::kKb * L::kTBlk;
                        float h0, l0, h1, l1;
                        split_tf32(minus ? __fsub_rn(er, orr) : __fadd_rn(er, orr), h0, l0);
                        split_tf32(minus ? __fsub_rn(ei, oi) : __fadd_rn(ei, oi), h1, l1);
                        *reinterpret_cast<float2*>(tb + off) = make_float2(h0, h1);
                        *reinterpret_cast<float2*>(tb + kLo + off) = make_float2(l0, l1);
                    }
                    fence_proxy_async_smem();
                    mbar_arrive(&tReady[bq]);
                }
            }
        }
    } else if (warp >= L::kEpi0 && warp < L::kEpi0 + L::kEpiWarps) {
        // ---------------- epilogue
        const int ew = warp - L::kEpi0;
        const int quad = warp & 3;
        const int grp = ew >> 3;                 // two groups take turns over the tiles
        const int cw = ((ew >> 2) & 1) * 32;     // this warp's columns cw .. cw + 31
        const float s_out = p.fq_out.scale, inv_out = p.fq_out.inv_scale;
        const float zpo = static_cast<float>(p.fq_out.zp);
        const float klo = -128.0f - zpo, khi = 127.0f - zpo;
        for (int it = grp; t_begin + it < t_end; it += 2) {
            const int tile = t_begin + it;
            const int a = it % L::kAccStages;
            const uint32_t aph = (it / L::kAccStages) & 1;
            if (!mbar_wait(&accFull[a], aph, sAbort)) {
                *sAbort = 1;
                atomicOr(p.err, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + a * L::kAccCols;
            uint4* dst = reinterpret_cast<uint4*>(p.codes_out +
                                                  (static_cast<int64_t>(tile_row(tile)) * 128 + quad * 32 + lane) * C + cw);
#pragma unroll 1
            for (int ch = 0; ch < 2; ++ch) {
            const int c0 = cw + 16 * ch;
            uint32_t raw[16], x1r[16], none = 0;
            tmem_ld16_async(tbase + c0, raw);
            tmem_ld16_async(tbase + L::kX1Col + c0, x1r);
            tmem_wait_ld_33(raw, x1r, none);
            // Per element: dequantise + bias, the fast fake-quant offset k (x2 = k s), z =
            // x1 + x2 and the next code from the table cell (breakpoint t, codes below /
            // from t), inserted into the packed word with one byte permute.
            uint32_t packed[4];
            // per packed word, the largest |r - rint(r)| of its four elements (r is finite:
            // v comes from an integer accumulator)
            float dmax[4];
            float zz[16];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                // the products of two columns per f32x2 instruction; every sum stays a
                // scalar add (a packed add of a packed product would be fused)
                const float4 A4 = reinterpret_cast<const float4*>(cols.a)[(c0 >> 2) + (j >> 2)];
                const int4 N4 = reinterpret_cast<const int4*>(cols.nk)[(c0 >> 2) + (j >> 2)];
                const float4 B4 = reinterpret_cast<const float4*>(cols.b)[(c0 >> 2) + (j >> 2)];
                const bool lo = (j & 2) == 0;
                const float2 ca = lo ? make_float2(A4.x, A4.y) : make_float2(A4.z, A4.w);
                const float2 cb = lo ? make_float2(B4.x, B4.y) : make_float2(B4.z, B4.w);
                const int n0 = lo ? N4.x : N4.z, n1 = lo ? N4.y : N4.w;
                const float2 f = make_float2(__int2float_rn(static_cast<int>(raw[j]) + n0),
                                             __int2float_rn(static_cast<int>(raw[j + 1]) + n1));
                const float2 m = mul2_rn(ca, f);
                const float2 v = make_float2(__fadd_rn(m.x, cb.x), __fadd_rn(m.y, cb.y));
                const float2 r = mul2_rn(v, make_float2(inv_out, inv_out));
                const float k0 = rintf(r.x), k1 = rintf(r.y);
                const float dm = fmaxf(fabsf(__fsub_rn(r.x, k0)), fabsf(__fsub_rn(r.y, k1)));
                dmax[j >> 2] = lo ? dm : fmaxf(dmax[j >> 2], dm);
                const float2 x2 = mul2_rn(make_float2(fminf(fmaxf(k0, klo), khi), fminf(fmaxf(k1, klo), khi)),
                                          make_float2(s_out, s_out));
                zz[j] = __fadd_rn(__uint_as_float(x1r[j]), x2.x);
                zz[j + 1] = __fadd_rn(__uint_as_float(x1r[j + 1]), x2.y);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                int2 cell[8];
#pragma unroll
                for (int q = 0; q < 8; q += 2) {
                    const float z0 = zz[8 * h + q], z1 = zz[8 * h + q + 1];
                    float u0, u1;
                    if constexpr (TWO) {
                        const bool s0 = z0 < p.lut_split, s1 = z1 < p.lut_split;
                        u0 = __saturatef(__fmaf_rn(z0, s0 ? p.lut_alpha0 : p.lut_alpha1, s0 ? p.lut_beta0 : p.lut_beta1));
                        u1 = __saturatef(__fmaf_rn(z1, s1 ? p.lut_alpha0 : p.lut_alpha1, s1 ? p.lut_beta0 : p.lut_beta1));
                    } else {
                        u0 = __saturatef(__fmaf_rn(z0, p.lut_alpha1, p.lut_beta1));
                        u1 = __saturatef(__fmaf_rn(z1, p.lut_alpha1, p.lut_beta1));
                    }
                    const float2 x = fma2_rn(make_float2(u0, u1), make_float2(p.lut_nm1, p.lut_nm1),
                                             make_float2(kMagic, kMagic));
                    cell[q] = sLut[__float_as_int(x.x) - 0x4B400000];
                    cell[q + 1] = sLut[__float_as_int(x.y) - 0x4B400000];
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const int j = 8 * h + q;
                    const float z = zz[j];
                    const uint32_t sel_lo = (0x3210u & ~(0xFu << (4 * (j & 3)))) | (4u << (4 * (j & 3)));
                    const uint32_t sel = z >= __int_as_float(cell[q].x) ? sel_lo + (1u << (4 * (j & 3))) : sel_lo;
                    const uint32_t prev = (j & 3) == 0 ? 0u : packed[j >> 2];
                    packed[j >> 2] = __byte_perm(prev, static_cast<uint32_t>(cell[q].y), sel);
                }
            }
            // rare: a word holding an element whose quotient lies next to a half-integer;
            // its four accumulators are read again from TMEM and those elements take the
            // exact division
            const uint32_t badw = (dmax[0] < kFastRoundLimit ? 0u : 1u) | (dmax[1] < kFastRoundLimit ? 0u : 2u) |
                                  (dmax[2] < kFastRoundLimit ? 0u : 4u) | (dmax[3] < kFastRoundLimit ? 0u : 8u);
            uint32_t any = __reduce_or_sync(0xffffffffu, badw);
            while (any) {
                const int w4 = __ffs(any) - 1;
                any &= any - 1;
                uint32_t rj[4], xj[4];
                tmem_ld4(tbase + c0 + 4 * w4, rj);
                tmem_ld4(tbase + L::kX1Col + c0 + 4 * w4, xj);
                tmem_wait_ld();
                asm volatile("" : "+r"(rj[0]), "+r"(rj[1]), "+r"(rj[2]), "+r"(rj[3]), "+r"(xj[0]),
                                  "+r"(xj[1]), "+r"(xj[2]), "+r"(xj[3]));  // uses stay after the wait
                if (badw & (1u << w4)) {
                    uint32_t w = w4 == 0 ? packed[0] : (w4 == 1 ? packed[1] : (w4 == 2 ? packed[2] : packed[3]));
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const float4 cp = sCol[c0 + 4 * w4 + jj];
                        const int vint = static_cast<int>(rj[jj]) + __float_as_int(cp.z);
                        const float v = __fadd_rn(__fmul_rn(cp.x, __int2float_rn(vint)), cp.w);
                        const float r = __fmul_rn(v, inv_out);
                        if (fabsf(__fsub_rn(r, rintf(r))) < kFastRoundLimit) continue;
                        const float x2 = __fmul_rn(__fsub_rn(fq_code(v, s_out, zpo), zpo), s_out);
                        const float z = __fadd_rn(__uint_as_float(xj[jj]), x2);
                        const bool s0 = TWO && z < p.lut_split;
                        const int2 cell = lut_cell_sat(z, sLut, s0 ? p.lut_alpha0 : p.lut_alpha1,
                                                       s0 ? p.lut_beta0 : p.lut_beta1, p.lut_nm1);
                        const uint32_t code = (z >= __int_as_float(cell.x) ? (cell.y >> 8) : cell.y) & 0xFFu;
                        w = (w & ~(0xFFu << (8 * jj))) | (code << (8 * jj));
                    }
                    if (w4 == 0) packed[0] = w;
                    else if (w4 == 1) packed[1] = w;
                    else if (w4 == 2) packed[2] = w;
                    else packed[3] = w;
                }
            }
            dst[ch] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accEmpty[a]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// proj: the projection (fno.cpp:972-993) over 128-point tiles.
//   q = LinearForwardBatched(codes, proj_q) + bias   (tcgen05 kind::i8, as the layers)
//   g = act(fake_quant(q, proj_q.output))            (the 256-entry activation table)
//   y = fake_quant(proj_out(g), proj_out.output)     (the reference's sequential
//                                                      out_ch-wide dot product)
// The proj_out dot product runs over a point's 64 activations in order, so one thread
// owns a point and all its columns.  Four epilogue warp groups (one warp per TMEM lane
// quadrant each) take turns over the CTA's tiles; group g drains accumulator stage g,
// so four tiles are in flight and no activation leaves the registers.
// ---------------------------------------------------------------------------
template <int C>
struct PCfg {
    static constexpr int kGroups = 4;
    static constexpr int kEpiWarps = 4 * kGroups;
    static constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
    static constexpr int kABytes = 128 * C;
    static constexpr int kStages = 4;
    static constexpr int kOnesCol = C;
    static constexpr int kAccCols = ((C + 16 + 31) / 32) * 32;
    static constexpr int kAccStages = kGroups;
    static constexpr int kTmemCols = pow2ceil(kAccStages * kAccCols);
    static_assert(kTmemCols <= 512, "TMEM");
    static constexpr int up1k(int v) { return (v + 1023) / 1024 * 1024; }
    static constexpr int kOffW = 0;
    static constexpr int kOffOnes = up1k(C * C);
    static constexpr int kOffA = kOffOnes + 1024;
    static constexpr int kOffCol = kOffA + kStages * kABytes;          // float4 [C]
    static constexpr int kOffAct = kOffCol + C * 16;                    // float [256]
    static constexpr int kOffWout = kOffAct + 256 * 4;                  // float [4][C], [4]
    static constexpr int kOffBars = kOffWout + 4 * C * 4 + 16;
    static constexpr int kNumBars = 2 * kStages + 2 * kAccStages;
    static constexpr int kSmemBytes = kOffBars + 8 * kNumBars + 16 + 1024;
    static_assert(kSmemBytes <= 227 * 1024, "smem");
};

// The activation-table value of v through the exact fake-quant division (the rare
// path of proj_kernel's fast code test), out of line.
__device__ __noinline__ float proj_exact_g(float v, float s_out, float zpo, const float* sAct) {
    return sAct[static_cast<int>(fq_code(v, s_out, zpo)) + 128];
}

template <int C, int OUT>
__global__ void __launch_bounds__(PCfg<C>::kThreads, 1)
proj_kernel(const __grid_constant__ CUtensorMap tmIn, const LayerArgs p,
            const __grid_constant__ ProjCols cols) {
    using L = PCfg<C>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sW = smem + L::kOffW;
    uint8_t* sOnes = smem + L::kOffOnes;
    uint8_t* sA = smem + L::kOffA;
    float4* sCol = reinterpret_cast<float4*>(smem + L::kOffCol);  // {sW*s_in, zp_w, zp_in*sum_w, bias}
    float* sAct = reinterpret_cast<float*>(smem + L::kOffAct);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kOffBars);
    uint64_t* empty = full + L::kStages;
    uint64_t* accFull = empty + L::kStages;
    uint64_t* accEmpty = accFull + L::kAccStages;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(accEmpty + L::kAccStages);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = static_cast<int>((p.M + 127) / 128);
    const int t_begin = static_cast<int>(static_cast<int64_t>(num_tiles) * blockIdx.x / gridDim.x);
    const int t_end = static_cast<int>(static_cast<int64_t>(num_tiles) * (blockIdx.x + 1) / gridDim.x);
    const bool use_act = p.act_table != nullptr && p.fq_out.kind == 1;

    {
        constexpr int kChunks = C / 16;
        for (int idx = threadIdx.x; idx < C * kChunks; idx += L::kThreads) {
            const int o = idx / kChunks, c = idx % kChunks;
            const uint4 v = *reinterpret_cast<const uint4*>(p.Wq + o * C + c * 16);
            *reinterpret_cast<uint4*>(sW + swz_offset(o * C + c * 16, C)) = v;
        }
        for (int idx = threadIdx.x; idx < 1024 / 16; idx += L::kThreads) {
            const uint32_t one = (idx * 16 < C) ? 0x01010101u : 0u;  // row 0 = ones
            *reinterpret_cast<uint4*>(sOnes + idx * 16) = make_uint4(one, one, one, one);
        }
        for (int o = threadIdx.x; o < C; o += L::kThreads)
            sCol[o] = make_float4(__fmul_rn(p.scale_w[o], p.s_in), __int_as_float(p.zp_w[o]),
                                  __int_as_float(p.zp_in * p.sum_w[o]), p.bias[o]);
        if (use_act)
            for (int i = threadIdx.x; i < 256; i += L::kThreads) sAct[i] = p.act_table[i];
        if (threadIdx.x == 0) {
            for (int s = 0; s < L::kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < L::kAccStages; ++s) {
                mbar_init(&accFull[s], 1);
                mbar_init(&accEmpty[s], 4);  // the group's four warps
            }
            *sAbort = 0;
            fence_mbar_init();
        }
        if (warp == 1) tmem_alloc(sTmem, L::kTmemCols);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    const uint32_t tmem_base = *sTmem;
    // the prologue above touched only this CTA's state and read-only tables
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (elect_one()) {
            prefetch_tmap(&tmIn);
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % L::kStages;
                const uint32_t ph = (it / L::kStages) & 1;
                if (!mbar_wait_backoff(&empty[s], ph ^ 1, sAbort, 1024)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitSlotFree);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], L::kABytes);
                tma_load_2d(sA + s * L::kABytes, &tmIn, &full[s], 0, tile * 128);
            }
            for (int j = (it > L::kStages ? it - L::kStages : 0); j < it; ++j)
                if (!mbar_wait_backoff(&full[j % L::kStages], (j / L::kStages) & 1, sAbort, 1024)) break;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (elect_one()) {
            int it = 0;
            for (int tile = t_begin; tile < t_end; ++tile, ++it) {
                const int s = it % L::kStages;
                const uint32_t ph = (it / L::kStages) & 1;
                const int a = it % L::kAccStages;
                const uint32_t aph = (it / L::kAccStages) & 1;
                if (!mbar_wait_backoff(&accEmpty[a], aph ^ 1, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitAccFree);
                    break;
                }
                if (!mbar_wait_backoff(&full[s], ph, sAbort, 128)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitTmaFull);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + a * L::kAccCols;
                const uint32_t aBase = smem_u32(sA + s * L::kABytes);
#pragma unroll
                for (int kk = 0; kk < C / 32; ++kk) {
                    const uint64_t ad = umma_desc(aBase + kk * 32, C);
                    const uint64_t wd = umma_desc(smem_u32(sW) + kk * 32, C);
                    const uint64_t od = umma_desc(smem_u32(sOnes) + kk * 32, C);
                    mma_i8(d, ad, wd, idesc_i8(C), kk > 0 ? 1u : 0u);
                    mma_i8(d + L::kOnesCol, ad, od, idesc_i8(16), kk > 0 ? 1u : 0u);
                }
                mma_commit(&empty[s]);
                mma_commit(&accFull[a]);
            }
            if (it > 0) {
                const int j = it - 1;
                mbar_wait_backoff(&accFull[j % L::kAccStages], (j / L::kAccStages) & 1, sAbort, 1024);
            }
        }
        __syncwarp();
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + L::kEpiWarps) {
        const int ew = warp - kEpiWarp0;
        const int quad = warp & 3;
        const int grp = ew >> 2;
        const int row = quad * 32 + lane;
        const float s_out = p.fq_out.scale, inv_out = p.fq_out.inv_scale;
        const float zpo = static_cast<float>(p.fq_out.zp);
        const float magic_zp = kMagic + zpo;
        constexpr int nu = linear_unfused_len(C);
        for (int it = grp; t_begin + it < t_end; it += L::kGroups) {
            const int tile = t_begin + it;
            const uint32_t aph = (it / L::kGroups) & 1;
            if (!mbar_wait(&accFull[grp], aph, sAbort)) {
                *sAbort = 1;
                atomicOr(p.err, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + grp * L::kAccCols;
            uint32_t raw[2][16];
            uint32_t sum_u;
            tmem_ld1(tbase + L::kOnesCol, sum_u);
            tmem_ld16_async(tbase, raw[0]);
            tmem_wait_ld16(raw[0]);
            asm volatile("" : "+r"(sum_u));  // sum_u is used after the wait above
            const int rconst = C * p.zp_in - 2 * static_cast<int>(sum_u);
            float acc_out[OUT];
#pragma unroll
            for (int j = 0; j < OUT; ++j) acc_out[j] = cols.bout[j];
#pragma unroll
            for (int c = 0; c < C / 16; ++c) {
                uint32_t (&cur)[16] = raw[c & 1];
                if (c + 1 < C / 16) tmem_ld16_async(tbase + (c + 1) * 16, raw[(c + 1) & 1]);
                float g[16];
                float vv[16];
                float dmax = 0.0f;   // largest |r - rint(r)| of the chunk (v is finite)
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float4 cp = cols.v[c * 16 + j];  // constant-bank operands
                    const int vint = static_cast<int>(cur[j]) + __float_as_int(cp.y) * rconst +
                                     __float_as_int(cp.z);
                    const float v = __fadd_rn(__fmul_rn(cp.x, __int2float_rn(vint)), cp.w);
                    vv[j] = v;
                    if (use_act) {
                        const float r = __fmul_rn(v, inv_out);
                        const float t = __fadd_rn(r, magic_zp);
                        dmax = fmaxf(dmax, fabsf(__fsub_rn(r, __fsub_rn(t, magic_zp))));
                        const float tc = fminf(fmaxf(t, kMagic - 128.0f), kMagic + 127.0f);
                        g[j] = sAct[__float_as_int(tc) - (0x4B400000 - 128)];
                    } else {
                        g[j] = activation(apply_fq(v, p.fq_out), p.act);
                    }
                }
                if (use_act && !(dmax < kFastRoundLimit)) {
                    // rare: the chunk holds a quotient next to a half-integer; those
                    // elements take the exact division (out of line)
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float r = __fmul_rn(vv[j], inv_out);
                        if (!(fabsf(__fsub_rn(r, rintf(r))) < kFastRoundLimit))
                            g[j] = proj_exact_g(vv[j], s_out, zpo, sAct);
                    }
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int o = c * 16 + j;
#pragma unroll
                    for (int jj = 0; jj < OUT; ++jj)
                        acc_out[jj] = linear_step(acc_out[jj], g[j], cols.wout[jj][o], o >= nu);
                }
                if (c + 1 < C / 16) tmem_wait_ld16(raw[(c + 1) & 1]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accEmpty[grp]);
            const int64_t m = static_cast<int64_t>(tile) * 128 + row;
            if (m < p.M) {
#pragma unroll
                for (int j = 0; j < OUT; ++j) {
                    float yv = acc_out[j];
                    if (p.fq_final.kind == 1) {
                        const float zf = static_cast<float>(p.fq_final.zp);
                        const float q = fq_code_fast(yv, p.fq_final.scale, p.fq_final.inv_scale, zf);
                        yv = __fmul_rn(__fsub_rn(q, zf), p.fq_final.scale);
                    } else {
                        yv = apply_fq(yv, p.fq_final);
                    }
                    p.y[m * OUT + j] = yv;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// spec_fwd_tc2: the forward transform of a layer on tensor cores (W == 128).
//
// Row DFT (along W) as an exact integer GEMM: for a pair of grid rows,
//   D_l[(r, c)][n] = sum_w code[h+r][w][c] * Blimb_l[n][w]      (tcgen05 kind::i8)
// where the DFT basis B[j][w] (cos / -sin of 2 pi kw w / W, j = 2 kw + {0, 1}) is
// scaled by 2^27, rounded to an integer and split into four balanced base-256
// digits Blimb_0..3.  The codes are the MMA's A operand in MN-major layout (two
// TMA-loaded [w][c] tiles, one per row, as the two 64-wide M atoms); the digit
// matrices are the K-major B operand.  Recombined in fp32 (exact digit partials and
// power-of-two weights; four rounded multiply-adds),
//   F[h][j][c] = s * (sum_l D_l 256^(3-l) - zp * sum_w Bint[j][w]) / 2^27
// is the row DFT of the snapped activation (code - zp) * s.  The H-axis DFT
//   X[kh][kw][c] += F[h][kw][c] * e^{-2 pi i kh h / H}
// is a second (3xTF32) MMA over groups of four rows, described below.
// A work unit is (sample, block of HB rows); CTAs loop over units.
// ---------------------------------------------------------------------------
constexpr int kFwdEpiWarps = 12;  // 3 per TMEM lane quadrant
constexpr int kFwdThreads = 32 * (4 + kFwdEpiWarps);

// MN-major descriptor: SW64 atoms of 64 bytes along M, `lbo` between M atoms,
// `sbo` between groups of 8 K rows.
__device__ __forceinline__ uint64_t umma_desc_mn64(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           (static_cast<uint64_t>(4u) << 61);
}

// ---------------------------------------------------------------------------
// The drain warps recombine each row pair's digit accumulators to fp32 F and write
// it, split into tf32 hi and lo halves, as the A operand of the H-axis MMA, which
// accumulates in TMEM:
//   X[(kw, c)][(kh, ri)] += sum_{(h, f)} F[h][kw][c][f] * E[(kh, ri)][(h, f)]
// over groups of four rows (K = 4 rows x {re, im} = 8), with E the complex twiddle
// e^{-2 pi i kh h / H} written as a real 2x2 block per (kh, h) (3xTF32 products).
// M = (kw, c) is 768 = six 128-lane blocks, N = (kh, ri) = 24 padded to 32.  At the
// end of a unit the drain warps read X from TMEM and write the unit's partial
// spectrum.
// ---------------------------------------------------------------------------
template <int C, int MH, int MW>
struct F2Cfg {
    static constexpr int kTile = 128 * C;                   // one grid row of codes
    static constexpr int kStages = 6;                       // row-pair ring
    static constexpr int kStageBytes = 2 * kTile;
    static constexpr int kN = 32;                           // basis rows per digit in p.limbs
    static constexpr int kN1 = 4 * 2 * MW;                  // row-DFT MMA N: 4 digits x 24
    static constexpr int kLimbBytes = kN1 * 128;            // [96][128] int8, SW128
    static constexpr int kD1Stages = 3;                     // row-DFT accumulator stages
    static constexpr int kMBlocks = (MW * C) / 128;         // M blocks of the H-DFT MMA
    static constexpr int kA2Block = 128 * 32;               // [128 m][8 k] fp32, SW32
    static constexpr int kA2Bytes = kMBlocks * kA2Block;    // one of hi / lo
    static constexpr int kB2Bytes = 32 * 32;                // [32 n][8 k] fp32, SW32
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kStages * kStageBytes;
    static constexpr int kOffA2 = kOffB + ((kLimbBytes + 1023) / 1024) * 1024;  // 2 x (hi, lo)
    static constexpr int kOffB2 = kOffA2 + 2 * 2 * kA2Bytes; // 2 buffers x (hi, lo)
    static constexpr int kOffBars = kOffB2 + 2 * 2 * kB2Bytes;
    static constexpr int kNumBars = 2 * kStages + 2 * kD1Stages + 2 + 2 + 2;
    static constexpr int kOffCzp = kOffBars + 8 * kNumBars + 16;  // 2*MW floats
    static constexpr int kSmemBytes = kOffCzp + 4 * 2 * MW + 1024;
    // TMEM: row-DFT stage a at columns [128 a, 128 a + 96); the six 32-column X blocks
    // fill the gaps [128 a + 96, 128 a + 128) and [384, 480)
    static constexpr int kTmemCols = 512;
    __device__ static constexpr uint32_t x_col(int mb) {
        return mb < 3 ? static_cast<uint32_t>(mb * 128 + 96) : static_cast<uint32_t>(384 + (mb - 3) * 32);
    }
    static_assert(kSmemBytes <= 227 * 1024, "smem");
    static_assert(2 * MW <= 24 && MH * 2 <= 32, "basis rows");
    static_assert((MW * C) % 128 == 0 && kMBlocks == 6, "H-DFT MMA blocks");
    static_assert(kN1 % 16 == 0 && kN1 <= 96, "row-DFT MMA N");
    static_assert(2 * MW == 24, "drain layout: 8 basis columns per warp third");
};

template <int C, int MH, int MW>
__global__ void __launch_bounds__(kFwdThreads, 1)
spec_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tmCodes, const SpecFwdArgs p) {
    using F = F2Cfg<C, MH, MW>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem + F::kOffA;
    uint8_t* sB = smem + F::kOffB;
    uint8_t* sA2 = smem + F::kOffA2;
    uint8_t* sB2 = smem + F::kOffB2;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + F::kOffBars);
    uint64_t* empty = full + F::kStages;
    uint64_t* d1Full = empty + F::kStages;
    uint64_t* d1Empty = d1Full + F::kD1Stages;
    uint64_t* a2Ready = d1Empty + F::kD1Stages;
    uint64_t* a2Free = a2Ready + 2;
    uint64_t* xFull = a2Free + 2;
    uint64_t* xEmpty = xFull + 1;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(xFull + 2);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
    float* sCzp = reinterpret_cast<float*>(smem + F::kOffCzp);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int pairs_per_unit = p.HB / 2;      // even (HB is a multiple of 4)
    const int groups_per_unit = pairs_per_unit / 2;
    const int nHB = p.H / p.HB;
    const int num_units = p.B * nHB;
    const int my_units = (num_units - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                         static_cast<int>(gridDim.x);
    const int total = my_units * pairs_per_unit;   // row pairs of this CTA

    {
        // the four digit matrices stacked into one B operand: row l*24 + j = digit l of
        // basis row j (K-major, 128-byte swizzle)
        for (int idx = threadIdx.x; idx < F::kN1 * 8; idx += kFwdThreads) {
            const int row = idx / 8, ch = idx % 8;
            const int l = row / (2 * MW), n = row % (2 * MW);
            const uint4 v = *reinterpret_cast<const uint4*>(p.limbs + (l * F::kN + n) * 128 + ch * 16);
            *reinterpret_cast<uint4*>(sB + swz_offset(row * 128 + ch * 16, 128)) = v;
        }
        // B2 rows n >= 2*MH stay zero
        for (int idx = threadIdx.x; idx < 2 * 2 * F::kB2Bytes / 16; idx += kFwdThreads)
            reinterpret_cast<uint4*>(sB2)[idx] = make_uint4(0, 0, 0, 0);
        // the zero-point term of basis column t: -zp * sum_w Bint[t][w] / 2^27
        if (threadIdx.x < 2 * MW)
            sCzp[threadIdx.x] = static_cast<float>(
                -static_cast<double>(static_cast<long long>(p.zp) * p.sum_b[threadIdx.x]) *
                7.450580596923828125e-9);
        if (threadIdx.x == 0) {
            for (int s = 0; s < F::kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < F::kD1Stages; ++s) {
                mbar_init(&d1Full[s], 1);
                mbar_init(&d1Empty[s], 4);                // the drain group of this stage
            }
            for (int s = 0; s < 2; ++s) {
                mbar_init(&a2Ready[s], 2 * 128);          // two pairs, one drain group each
                mbar_init(&a2Free[s], 1);
            }
            mbar_init(xFull, 1);
            mbar_init(xEmpty, 4);                         // the group that drains X
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
    // the prologue above touched only this CTA's state and read-only tables
    grid_dep_wait();
    grid_dep_launch();

    if (warp == 0) {
        if (elect_one()) {
            prefetch_tmap(&tmCodes);
            int it = 0;
            for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
                const int b = u / nHB, hb = u % nHB;
                for (int k = 0; k < pairs_per_unit; ++k, ++it) {
                    const int s = it % F::kStages;
                    const uint32_t ph = (it / F::kStages) & 1;
                    if (!mbar_wait_backoff(&empty[s], ph ^ 1, sAbort, 1024)) {
                        *sAbort = 1;
                        atomicOr(p.err, kErrWaitSlotFree);
                        goto producer_done2;
                    }
                    mbar_arrive_expect_tx(&full[s], F::kStageBytes);
                    const int row = b * p.H + hb * p.HB + 2 * k;
                    tma_load_2d(sA + s * F::kStageBytes, &tmCodes, &full[s], 0, row * 128);
                    tma_load_2d(sA + s * F::kStageBytes + F::kTile, &tmCodes, &full[s], 0, (row + 1) * 128);
                }
            }
        producer_done2:
            for (int j = (it > F::kStages ? it - F::kStages : 0); j < it; ++j)
                if (!mbar_wait_backoff(&full[j % F::kStages], (j / F::kStages) & 1, sAbort, 1024)) break;
        }
        __syncwarp();
    } else if (warp == 1) {
        // row DFTs: one N = 96 int8 MMA chain per row pair into its D1 stage
        if (elect_one()) {
            constexpr uint32_t idesc1 = idesc_i8(F::kN1) | (1u << 15);  // A MN-major
            for (int it = 0; it < total; ++it) {
                const int s = it % F::kStages;
                const uint32_t ph = (it / F::kStages) & 1;
                const int a = it % F::kD1Stages;
                const uint32_t aph = (it / F::kD1Stages) & 1;
                if (!mbar_wait(&d1Empty[a], aph ^ 1, sAbort) ||
                    !mbar_wait(&full[s], ph, sAbort)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitAccFree);
                    break;
                }
                tc_fence_after();
                const uint32_t aBase = smem_u32(sA + s * F::kStageBytes);
                const uint32_t d = tmem_base + a * 128;
                const uint32_t bBase = smem_u32(sB);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma_i8(d, umma_desc_mn64(aBase + kk * 2048, F::kTile, 512),
                           umma_desc(bBase + kk * 32, 128), idesc1, kk > 0 ? 1u : 0u);
                mma_commit(&empty[s]);
                mma_commit(&d1Full[a]);
            }
        }
        __syncwarp();
    } else if (warp == 2) {
        // H-DFTs: per group of four rows (row pairs 2g, 2g+1), 3xTF32 into the X blocks;
        // a second issuing thread, so the row DFTs never queue behind these waits
        if (elect_one()) {
            constexpr uint32_t idesc2 = idesc_tf32(32);
            const int ngroups = total / 2;
            bool ok = true;
            for (int gh = 0; gh < ngroups; ++gh) {
                const bool first = (gh % groups_per_unit) == 0;
                if (!mbar_wait_backoff(&a2Ready[gh & 1], (gh >> 1) & 1, sAbort, 128) ||
                    (first && !mbar_wait_backoff(xEmpty, ((gh / groups_per_unit) & 1) ^ 1, sAbort, 128))) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitDrain);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t ahi = smem_u32(sA2) + (gh & 1) * 2 * F::kA2Bytes;
                const uint32_t alo = ahi + F::kA2Bytes;
                const uint32_t bhi = smem_u32(sB2) + (gh & 1) * 2 * F::kB2Bytes;
                const uint32_t blo = bhi + F::kB2Bytes;
#pragma unroll
                for (int mb = 0; mb < F::kMBlocks; ++mb) {
                    const uint32_t d = tmem_base + F::x_col(mb);
                    const uint32_t ao = mb * F::kA2Block;
                    mma_tf32(d, umma_desc(ahi + ao, 32), umma_desc(bhi, 32), idesc2, first ? 0u : 1u);
                    mma_tf32(d, umma_desc(alo + ao, 32), umma_desc(bhi, 32), idesc2, 1u);
                    mma_tf32(d, umma_desc(ahi + ao, 32), umma_desc(blo, 32), idesc2, 1u);
                }
                mma_commit(&a2Free[gh & 1]);
                if ((gh % groups_per_unit) == groups_per_unit - 1) mma_commit(xFull);
            }
            if (ok && total > 0) mbar_wait_backoff(xFull, (my_units - 1) & 1, sAbort, 1024);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // Three drain groups of four warps (one per TMEM lane quadrant) take turns over
        // the row pairs (group g drains row-DFT stage g), so three pairs' TMEM reads,
        // recombination and operand stores overlap.  Each thread recombines all 24
        // basis columns of its lane (r, c).
        const int ew = warp - 4;            // 0..11
        const int grp = ew >> 2;            // 0..2
        const int gtid = (ew & 3) * 32 + lane;  // 0..127 within the group
        const int quad = warp & 3;
        const int m = quad * 32 + lane;     // TMEM lane = (r, c)
        const int r = m / C, c = m % C;
        // digit l of basis columns 8 part .. 8 part + 7 of this thread's lane
        auto ld_part = [&](uint32_t tb, int part, uint32_t (&d)[4][8]) {
#pragma unroll
            for (int l = 0; l < 4; ++l)
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x8.b32 "
                    "{%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                    : "=r"(d[l][0]), "=r"(d[l][1]), "=r"(d[l][2]), "=r"(d[l][3]), "=r"(d[l][4]),
                      "=r"(d[l][5]), "=r"(d[l][6]), "=r"(d[l][7])
                    : "r"(tb + l * 2 * MW + 8 * part)
                    : "memory");
        };
        // keeps every use of d after the tcgen05.wait::ld that precedes it
        auto pin = [](uint32_t (&d)[4][8]) {
#pragma unroll
            for (int l = 0; l < 4; ++l)
                asm volatile("" : "+r"(d[l][0]), "+r"(d[l][1]), "+r"(d[l][2]), "+r"(d[l][3]),
                                  "+r"(d[l][4]), "+r"(d[l][5]), "+r"(d[l][6]), "+r"(d[l][7]));
        };
        // digits -> fp32 F of 8 basis columns (4 kw x re/im), stored as tf32 hi / lo
        auto recombine = [&](int part, const uint32_t (&d)[4][8], uint8_t* ahi, uint8_t* alo, int hl) {
#pragma unroll
            for (int t2 = 0; t2 < 4; ++t2) {
                float fv[2];
#pragma unroll
                for (int f = 0; f < 2; ++f) {
                    const int t = 2 * t2 + f;
                    float u = __fmaf_rn(__int2float_rn(static_cast<int>(d[3][t])), 0x1p-27f, sCzp[8 * part + t]);
                    u = __fmaf_rn(__int2float_rn(static_cast<int>(d[2][t])), 0x1p-19f, u);
                    u = __fmaf_rn(__int2float_rn(static_cast<int>(d[1][t])), 0x1p-11f, u);
                    u = __fmaf_rn(__int2float_rn(static_cast<int>(d[0][t])), 0x1p-3f, u);
                    fv[f] = __fmul_rn(u, p.s);
                }
                const int kw = 4 * part + t2;
                const int mb = kw >> 1;
                const int ml = (kw & 1) * C + c;
                float h0, l0, h1, l1;
                split_tf32(fv[0], h0, l0);
                split_tf32(fv[1], h1, l1);
                const uint32_t off = mb * F::kA2Block + swz_offset(ml * 32 + hl * 8, 32);
                *reinterpret_cast<float2*>(ahi + off) = make_float2(h0, h1);
                *reinterpret_cast<float2*>(alo + off) = make_float2(l0, l1);
            }
        };
        bool ok = true;
        for (int it = grp; it < total && ok; it += F::kD1Stages) {
            const int g = it >> 1;
            const int pig = it & 1;                        // pair in group of four rows
            const int a = grp;                             // = it % kD1Stages
            // twiddles of the group's E entries (two per thread of the group draining
            // the first pair), loaded before the waits
            float2 ev[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            if (pig == 0) {
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {
                    const int idx = gtid + 128 * e2;
                    const int kh = idx >> 4, hh = (idx & 7) >> 1;
                    if (kh < MH) {
                        const int unit = blockIdx.x + (it / pairs_per_unit) * gridDim.x;
                        const int h = (unit % nHB) * p.HB + 2 * (it % pairs_per_unit) + hh;
                        ev[e2] = __ldg(p.twf_h + h * MH + kh);
                    }
                }
            }
            if (!mbar_wait(&d1Full[a], (it / F::kD1Stages) & 1, sAbort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint8_t* ahi = sA2 + (g & 1) * 2 * F::kA2Bytes;
            uint8_t* alo = ahi + F::kA2Bytes;
            const int hl = 2 * pig + r;                    // row within the group
            const uint32_t tb = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + a * 128;
            uint32_t dA[4][8], dB[4][8];
            ld_part(tb, 0, dA);
            ld_part(tb, 1, dB);
            // the A2 buffer is free once the H-DFT of two groups back has completed
            const bool free_ok = mbar_wait(&a2Free[g & 1], ((g >> 1) & 1) ^ 1, sAbort);
            tmem_wait_ld();
            pin(dA);
            pin(dB);
            if (!free_ok) {
                ok = false;
                break;
            }
            recombine(0, dA, ahi, alo, hl);
            ld_part(tb, 2, dA);
            recombine(1, dB, ahi, alo, hl);
            tmem_wait_ld();
            pin(dA);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d1Empty[a]);
            recombine(2, dA, ahi, alo, hl);
            if (pig == 0) {
                // E of the group's four rows -> B2 (rows n = (kh, ri), k = (h, f))
#pragma unroll
                for (int e2 = 0; e2 < 2; ++e2) {
                    const int idx = gtid + 128 * e2;
                    const int n = idx >> 3, k = idx & 7;
                    const int kh = n >> 1, ri = n & 1, f = k & 1;
                    const float2 e = ev[e2];
                    float v = 0.0f;
                    if (kh < MH) v = ri == 0 ? (f == 0 ? e.x : -e.y) : (f == 0 ? e.y : e.x);
                    float hi, lo;
                    split_tf32(v, hi, lo);
                    uint8_t* bhi = sB2 + (g & 1) * 2 * F::kB2Bytes;
                    const uint32_t off = swz_offset(n * 32 + k * 4, 32);
                    *reinterpret_cast<float*>(bhi + off) = hi;
                    *reinterpret_cast<float*>(bhi + F::kB2Bytes + off) = lo;
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(&a2Ready[g & 1]);
            if (pig == 1 && (g % groups_per_unit) == groups_per_unit - 1) {
                // unit complete: X -> partial spectrum of (sample, row block)
                const int u_local = it / pairs_per_unit;
                if (!mbar_wait(xFull, u_local & 1, sAbort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int unit = blockIdx.x + u_local * gridDim.x;
                const int b = unit / nHB, hb = unit % nHB;
                float2* dst = p.xpart + (static_cast<int64_t>(b) * nHB + hb) * (MH * MW * C);
#pragma unroll 1
                for (int mb = 0; mb < F::kMBlocks; ++mb) {
                    uint32_t x[24];
                    const uint32_t xa = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + F::x_col(mb);
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                        : "=r"(x[0]), "=r"(x[1]), "=r"(x[2]), "=r"(x[3]), "=r"(x[4]), "=r"(x[5]),
                          "=r"(x[6]), "=r"(x[7]), "=r"(x[8]), "=r"(x[9]), "=r"(x[10]), "=r"(x[11]),
                          "=r"(x[12]), "=r"(x[13]), "=r"(x[14]), "=r"(x[15])
                        : "r"(xa));
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x8.b32 "
                        "{%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                        : "=r"(x[16]), "=r"(x[17]), "=r"(x[18]), "=r"(x[19]), "=r"(x[20]),
                          "=r"(x[21]), "=r"(x[22]), "=r"(x[23])
                        : "r"(xa + 16));
                    tmem_wait_ld();
                    const int kw = 2 * mb + (m >> 6), cc = m & 63;
#pragma unroll
                    for (int kh = 0; kh < MH; ++kh)
                        dst[(kh * MW + kw) * C + cc] =
                            make_float2(__uint_as_float(x[2 * kh]), __uint_as_float(x[2 * kh + 1]));
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(xEmpty);
            }
        }
        if (!ok) {
            *sAbort = 1;
            atomicOr(p.err, kErrWaitAccFull);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, F::kTmemCols);
    }
}

// Launch with programmatic stream serialization (see grid_dep_wait in sm100.cuh).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename Kern>
cudaError_t set_smem(Kern k, int bytes) {
    return set_max_dynamic_smem(reinterpret_cast<const void*>(k), bytes);
}

template <int C, int MH, int MW>
cudaError_t run_layers(const Fno2dPlan& pl, cudaStream_t st) {
    cudaError_t e;
    // the forward's launches follow each other on `st` with nothing between them
    TimerChain chained(pl.timer);
    const int64_t M = static_cast<int64_t>(pl.B) * pl.H * pl.W;
    // lift
    {
        const int64_t blocks64 = (M + 255) / 256;
        const int grid = static_cast<int>(blocks64 < 148 * 8 ? blocks64 : 148 * 8);
        if (pl.timer) pl.timer->begin("fno2d_lift", st);
        switch (pl.in_ch) {
#define NFX_LIFT(n)                                                                            \
    case n:                                                                                    \
        e = launch_pdl(lift_kernel<C, n>, dim3(grid), dim3(256), 0, st, pl.x, M, pl.lift_cols,   \
                       pl.lift_s, pl.lift_zp, pl.lift_inv_s, pl.codes[0]);                       \
        break;
            NFX_LIFT(1) NFX_LIFT(2) NFX_LIFT(3) NFX_LIFT(4) NFX_LIFT(5) NFX_LIFT(6) NFX_LIFT(7)
            NFX_LIFT(8)
#undef NFX_LIFT
            default: return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
        if (pl.timer) pl.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        if (pl.tap_codes &&
            (e = cudaMemcpyAsync(pl.tap_codes, pl.codes[0], static_cast<size_t>(M) * C,
                                 cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
            return e;
    }
    const int sms = device_sm_count();
    const int num_tiles = static_cast<int>((M + 127) / 128);
    const int grid_l = num_tiles < sms ? num_tiles : sms;
    int cur = 0;
    for (int i = 0; i < pl.L; ++i) {
        const int nHB = pl.H / pl.HB;
        const int sm_fwd = (pl.W * C + MW * pl.W * 2) * 4;
        if (pl.W == 128 && pl.fwd_limbs && (pl.HB % 4) == 0) {
            using FC = F2Cfg<C, MH, MW>;
            auto k = spec_fwd_tc2_kernel<C, MH, MW>;
            if ((e = set_smem(k, FC::kSmemBytes)) != cudaSuccess) return e;
            CUtensorMap tc;
            if (!encode_2d(&tc, CU_TENSOR_MAP_DATA_TYPE_UINT8, pl.codes[cur], C, M, C, C, 128, C))
                return cudaErrorInvalidValue;
            SpecFwdArgs fa{pl.fwd_limbs, pl.fwd_sum_b, pl.twf_h, pl.xpart, pl.layer[i].s_in,
                           pl.layer[i].zp_in, pl.B, pl.H, pl.HB, pl.err};
            const int units = pl.B * nHB;
            if (pl.timer) pl.timer->begin("fno2d_spec_fwd", st);
            e = launch_pdl(k, dim3(units < sms ? units : sms), dim3(kFwdThreads), FC::kSmemBytes, st, tc, fa);
            if (e != cudaSuccess) return e;
            if (pl.timer) pl.timer->end(st);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        } else {
            auto k = spec_fwd_kernel<C, MH, MW>;
            if ((e = set_smem(k, sm_fwd)) != cudaSuccess) return e;
            if (pl.timer) pl.timer->begin("fno2d_spec_fwd", st);
            k<<<dim3(nHB, pl.B), C * MW, sm_fwd, st>>>(pl.codes[cur], pl.H, pl.W, pl.HB,
                                                    pl.layer[i].s_in, pl.layer[i].zp_in,
                                                    pl.twf_w, pl.twf_h, pl.xpart);
            if (pl.timer) pl.timer->end(st);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        }
        {
            if (pl.layer[i].wmix_hi == nullptr || pl.layer[i].wmix_lo == nullptr) return cudaErrorInvalidValue;
            using FM = MixCfg<C, false>;
            // every chunk's weights resident when one sample tile per mode gives one CTA
            // per SM anyway
            const bool pre = (pl.B + 127) / 128 == 1;
            auto k = pre ? spec_mix_tc_kernel<C, MH, MW, true> : spec_mix_tc_kernel<C, MH, MW, false>;
            const int mix_smem = pre ? MixCfg<C, true>::kSmemBytes : FM::kSmemBytes;
            if ((e = set_smem(k, mix_smem)) != cudaSuccess) return e;
            CUtensorMap thi, tlo;
            const uint64_t rows = static_cast<uint64_t>(MH) * MW * FM::kK;
            if (!encode_2d(&thi, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pl.layer[i].wmix_hi, FM::kK, rows,
                           FM::kK * 4, FM::kChunk, FM::kK, 128) ||
                !encode_2d(&tlo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, pl.layer[i].wmix_lo, FM::kK, rows,
                           FM::kK * 4, FM::kChunk, FM::kK, 128))
                return cudaErrorInvalidValue;
            if (pl.timer) pl.timer->begin("fno2d_spec_mix", st);
            e = launch_pdl(k, dim3(MH * MW, (pl.B + 127) / 128), dim3(kMixTcThreads), mix_smem, st,
                           thi, tlo, static_cast<const float2*>(pl.xpart), nHB, pl.B, pl.Y, pl.err);
            if (e != cudaSuccess) return e;
            if (pl.timer) pl.timer->end(st);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        }
        {
            LayerArgs a = pl.W == 128 ? pl.layer[i].args_tc : pl.layer[i].args;
            a.M = M;
            a.H = pl.H;
            a.W = pl.W;
            a.Y = pl.Y;
            a.twi_w = pl.twi_w;
            a.twi_h = pl.twi_h;
            a.err = pl.err;
            CUtensorMap tin, tout;
            if (!encode_2d(&tin, CU_TENSOR_MAP_DATA_TYPE_UINT8, pl.codes[cur], C, M, C, C, 128, C) ||
                !encode_2d(&tout, CU_TENSOR_MAP_DATA_TYPE_UINT8, pl.codes[cur ^ 1], C, M, C, C / 4,
                           32, 0))
                return cudaErrorInvalidValue;
            if (pl.timer) pl.timer->begin("fno2d_layer", st);
            if (pl.W == 128 && a.lut_cells > 0 && a.lut_cells <= kFno2dLutCellsTc) {
                using TC = TCfg<C, MH, MW>;
                if (!encode_2d(&tout, CU_TENSOR_MAP_DATA_TYPE_UINT8, pl.codes[cur ^ 1], C, M, C, C / 2, 32, 0))
                    return cudaErrorInvalidValue;
                a.codes_out = pl.codes[cur ^ 1];
                auto k = a.lut_two ? layer_tc_kernel<C, MH, MW, true> : layer_tc_kernel<C, MH, MW, false>;
                if ((e = set_smem(k, TC::kSmemBytes)) != cudaSuccess) return e;
                e = launch_pdl(k, dim3(grid_l), dim3(TC::kThreads), TC::kSmemBytes, st, tin, a,
                               pl.layer[i].cols);
                if (e != cudaSuccess) return e;
            } else if (pl.W == 128) {
                using LC = LCfg<C, MH, MW, false, true>;
                auto k = layer_kernel<C, MH, MW, false, true>;
                if ((e = set_smem(k, LC::kSmemBytes)) != cudaSuccess) return e;
                k<<<grid_l, LC::kThreads, LC::kSmemBytes, st>>>(tin, tout, a);
            } else {
                using LC = LCfg<C, MH, MW, false, false>;
                auto k = layer_kernel<C, MH, MW, false, false>;
                if ((e = set_smem(k, LC::kSmemBytes)) != cudaSuccess) return e;
                k<<<grid_l, LC::kThreads, LC::kSmemBytes, st>>>(tin, tout, a);
            }
            if (pl.timer) pl.timer->end(st);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        }
        cur ^= 1;
        if (pl.tap_codes &&
            (e = cudaMemcpyAsync(pl.tap_codes + static_cast<size_t>(i + 1) * M * C, pl.codes[cur],
                                 static_cast<size_t>(M) * C, cudaMemcpyDeviceToDevice, st)) != cudaSuccess)
            return e;
    }
    {
        using PC = PCfg<C>;
        auto k = pl.proj.out_ch == 1 ? proj_kernel<C, 1>
                 : pl.proj.out_ch == 2 ? proj_kernel<C, 2>
                 : pl.proj.out_ch == 3 ? proj_kernel<C, 3> : proj_kernel<C, 4>;
        if ((e = set_smem(k, PC::kSmemBytes)) != cudaSuccess) return e;
        CUtensorMap tin;
        if (!encode_2d(&tin, CU_TENSOR_MAP_DATA_TYPE_UINT8, pl.codes[cur], C, M, C, C, 128, C))
            return cudaErrorInvalidValue;
        LayerArgs a = pl.proj;
        a.M = M;
        a.H = pl.H;
        a.W = pl.W;
        a.err = pl.err;
        a.y = pl.y;
        if (pl.timer) pl.timer->begin("fno2d_proj", st);
        e = launch_pdl(k, dim3(grid_l), dim3(PC::kThreads), PC::kSmemBytes, st, tin, a, pl.proj_cols);
        if (e != cudaSuccess) return e;
        if (pl.timer) pl.timer->end(st);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace

bool fno2d_supported(int C, int MH, int MW) {
    return C == 64 && MH == 12 && MW == 12;
}

cudaError_t fno2d_run(const Fno2dPlan& pl, cudaStream_t st) {
    if (pl.C == 64 && pl.MH == 12 && pl.MW == 12) return run_layers<64, 12, 12>(pl, st);
    return cudaErrorInvalidValue;
}

}  // namespace nfx
