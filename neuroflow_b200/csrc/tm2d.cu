// tm2d.cu -- TokenMixer2D executor (sm_100a): the reference TokenMixer2D::Forward
// (cpp/src/fno.cpp:1756-1956) with the reference's loop order and rounding, and the
// INT8 per-token variant of its q/k/v/o/ffn layers on the tcgen05 GEMM.
//
//   pool        mean over the pp points of each patch (fno.cpp:1803-1816)
//   linear_f32  every FP32 Linear (fno.cpp:51-80): register-tiled CUDA-core GEMM whose
//               outputs accumulate over k in order with the reference build's
//               vector-block / fused-tail rounding (linear_step); bias first,
//               activation or residual add in the epilogue; the unslice Linear reads
//               its (x, token) concatenation directly
//   layer_norm  LayerNormLastDim (fno.cpp:1418-1438), one row per lane
//   attention   per (b, head, 128 queries), one query per thread, K/V streamed through
//               shared memory: scores with the reference's dot-product rounding, the
//               softmax of fno.cpp:1441-1456 (max, exp, sequential sum, 1/sum), and
//               the attention-times-V sum in key order (4-wide unfused blocks, fused
//               tail); three passes over the keys instead of a materialised n x n matrix
//   row_quant   INT8 path: per-row qparams (the compute_tensor_qparams rule in double)
//               and the activation codes (QuantiseActivation, int8_gemm.cpp:507-520)
//   attention_online  INT8 path: one pass over the keys with an online softmax and
//               fused multiply-adds (fp32-accurate, not the reference's order)
//   attention_tc  head dim 32, both paths: the same attention on tensor cores (3xTF32
//               tcgen05 MMAs, TMEM accumulators, online softmax); fp32-accurate, not the
//               reference's summation order -- the FP32 network stays within rtol 1e-5
//               of the reference's
//
// Approximate operations: CUDA's expf in the softmax and tanhf in GELU (a few ulps
// from glibc's); everything else is bit-identical to the reference arithmetic.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <type_traits>

#include "nfx_internal.h"
#include "numerics.cuh"
#include "sm100.cuh"
#include "tm2d.h"

namespace nfx {
namespace {

__device__ __forceinline__ float act_f(float z, int act) {
    return act == 1 ? relu_ref(z) : gelu_tanh(z);
}

// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) pool_kernel(const float* __restrict__ x, int64_t total,
                                                   int in_d, int NP, int pp,
                                                   float* __restrict__ pooled) {
    const float ppf = static_cast<float>(pp);
    for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
         t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int d = static_cast<int>(t % in_d);
        const int64_t bp = t / in_d;              // b * NP + patch
        const int64_t b = bp / NP, pi = bp % NP;
        const float* src = x + ((b * NP + pi) * pp) * in_d + d;
        float acc = 0.0f;
        for (int q = 0; q < pp; ++q) acc = __fadd_rn(acc, __fdiv_rn(src[static_cast<int64_t>(q) * in_d], ppf));
        pooled[t] = acc;
    }
}

// ---------------------------------------------------------------------------
// FP32 Linear: C[m, n] = epi(b[n] + sum_k A[m, k] W[n, k]); 64x64 tile, 256 threads,
// 4x4 outputs per thread, K staged 32 at a time.  A source 1 is the unslice
// concatenation: row m = (b, point p) -> [x[b, p, 0:in_d], tok[b, p / pp, 0:L]].
// epi: act (0 none, 1 GELU, 2 ReLU) then, when R is set, R[m, n] + value.
// ---------------------------------------------------------------------------
struct LinArgs {
    const float* A;
    int src;              // 0 plain, 1 unslice concat
    const float* x;       // concat source
    const float* tok;
    int in_d, L, pp, npts;
    const float* W;
    const float* bias;
    const float* R;
    float* C;
    int64_t M;
    int N, K, act;
};

constexpr int kBM = 64, kBN = 64, kBK = 32;

__device__ __forceinline__ float lin_a(const LinArgs& a, int64_t m, int k) {
    if (a.src == 0) return a.A[m * a.K + k];
    const int64_t b = m / a.npts, p = m % a.npts;
    if (k < a.in_d) return a.x[m * a.in_d + k];
    return a.tok[(b * (a.npts / a.pp) + p / a.pp) * a.L + (k - a.in_d)];
}

__global__ void __launch_bounds__(256) linear_f32_kernel(LinArgs a) {
    __shared__ float As[kBK][kBM + 4];
    __shared__ float Ws[kBK][kBN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kBM;
    const int n0 = blockIdx.x * kBN;
    const int nu = linear_unfused_len(a.K);
    float acc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        const float bv = (a.bias && n < a.N) ? __ldg(a.bias + n) : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][j] = bv;
    }
    for (int k0 = 0; k0 < a.K; k0 += kBK) {
        for (int t = threadIdx.x; t < kBM * kBK; t += 256) {
            const int mm = t / kBK, kk = t % kBK;
            const int64_t m = m0 + mm;
            const int k = k0 + kk;
            As[kk][mm] = (m < a.M && k < a.K) ? lin_a(a, m, k) : 0.0f;
        }
        for (int t = threadIdx.x; t < kBN * kBK; t += 256) {
            const int nn = t / kBK, kk = t % kBK;
            const int n = n0 + nn, k = k0 + kk;
            Ws[kk][nn] = (n < a.N && k < a.K) ? __ldg(a.W + static_cast<int64_t>(n) * a.K + k) : 0.0f;
        }
        __syncthreads();
        const int kend = min(kBK, a.K - k0);
        // the reference's unfused products (k < nu) and fused tail as separate loops
        auto steps = [&](auto fused, int kb, int ke) {
            for (int kk = kb; kk < ke; ++kk) {
                float av[4], wv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
                for (int j = 0; j < 4; ++j) wv[j] = Ws[kk][tx * 4 + j];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if constexpr (!decltype(fused)::value) {
                        // two rounded products per f32x2 instruction, each sum a scalar
                        // rounded add
#pragma unroll
                        for (int j = 0; j < 4; j += 2) {
                            const float2 m = mul2_rn(make_float2(av[i], av[i]), make_float2(wv[j], wv[j + 1]));
                            acc[i][j] = __fadd_rn(acc[i][j], m.x);
                            acc[i][j + 1] = __fadd_rn(acc[i][j + 1], m.y);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(av[i], wv[j], acc[i][j]);
                    }
                }
            }
        };
        const int ksplit = min(kend, max(0, nu - k0));
        steps(std::false_type{}, 0, ksplit);
        steps(std::true_type{}, ksplit, kend);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t m = m0 + ty * 4 + i;
        if (m >= a.M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n >= a.N) continue;
            float v = acc[i][j];
            if (a.act == 1) v = gelu_tanh(v);
            else if (a.act == 2) v = relu_ref(v);
            if (a.R) v = __fadd_rn(a.R[m * a.N + n], v);
            a.C[m * a.N + n] = v;
        }
    }
}

// ---------------------------------------------------------------------------
// LayerNorm: 32 rows per warp staged in shared memory [32][d + 1], one row per lane
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) layer_norm_kernel(const float* __restrict__ x, int64_t rows,
                                                         int d, const float* __restrict__ g,
                                                         const float* __restrict__ bta,
                                                         float* __restrict__ y) {
    extern __shared__ float sr[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* mine = sr + static_cast<size_t>(warp) * 32 * (d + 1);
    const int64_t r0 = (static_cast<int64_t>(blockIdx.x) * 4 + warp) * 32;
    for (int i = lane; i < 32 * d; i += 32) {
        const int rr = i / d, c = i % d;
        mine[rr * (d + 1) + c] = r0 + rr < rows ? x[(r0 + rr) * d + c] : 0.0f;
    }
    __syncwarp();
    const int64_t r = r0 + lane;
    if (r < rows) {
        const float* xr = mine + lane * (d + 1);
        float mean = 0.0f;
        for (int i = 0; i < d; ++i) mean = __fadd_rn(mean, xr[i]);
        mean = __fdiv_rn(mean, static_cast<float>(d));
        const int nu = linear_unfused_len(d);
        float var = 0.0f;
        for (int i = 0; i < d; ++i) {
            const float df = __fsub_rn(xr[i], mean);
            var = linear_step(var, df, df, i >= nu);
        }
        var = __fdiv_rn(var, static_cast<float>(d));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
        for (int i = 0; i < d; ++i)
            mine[lane * (d + 1) + i] = __fmaf_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), __ldg(g + i), __ldg(bta + i));
    }
    __syncwarp();
    for (int i = lane; i < 32 * d; i += 32) {
        const int rr = i / d, c = i % d;
        if (r0 + rr < rows) y[(r0 + rr) * d + c] = mine[rr * (d + 1) + c];
    }
}

// ---------------------------------------------------------------------------
// attention: grid (ceil(NP / 128), heads, B), 128 threads, one query each.
// Q/K/V rows are (b * NP + token) * L + head * HD.
// ---------------------------------------------------------------------------
constexpr int kQ = 128;

template <int HD>
__global__ void __launch_bounds__(kQ) attention_kernel(const float* __restrict__ Q,
                                                       const float* __restrict__ K,
                                                       const float* __restrict__ V, int NP, int L,
                                                       float scale, float* __restrict__ out) {
    constexpr int kKeys = HD <= 32 ? 128 : 64;  // 32 KB of K and V per chunk
    __shared__ float4 sK[kKeys][HD / 4];  // 16-byte broadcast loads in the inner loops
    __shared__ float4 sV[kKeys][HD / 4];
    const int b = blockIdx.z, head = blockIdx.y;
    const int i = blockIdx.x * kQ + threadIdx.x;
    const bool live = i < NP;
    const int64_t base = static_cast<int64_t>(b) * NP * L + head * HD;
    float q[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) q[d] = live ? Q[base + static_cast<int64_t>(i) * L + d] : 0.0f;
    constexpr int nu = linear_unfused_len(HD);
    auto score = [&](int jj) {
        float s = 0.0f;
#pragma unroll
        for (int d4 = 0; d4 < HD / 4; ++d4) {
            const float4 k4 = sK[jj][d4];
            s = linear_step(s, q[4 * d4 + 0], k4.x, 4 * d4 + 0 >= nu);
            s = linear_step(s, q[4 * d4 + 1], k4.y, 4 * d4 + 1 >= nu);
            s = linear_step(s, q[4 * d4 + 2], k4.z, 4 * d4 + 2 >= nu);
            s = linear_step(s, q[4 * d4 + 3], k4.w, 4 * d4 + 3 >= nu);
        }
        return __fmul_rn(s, scale);
    };
    auto load = [&](float4 (*dst)[HD / 4], const float* src, int j0) {
        float* flat = reinterpret_cast<float*>(dst);
        for (int t = threadIdx.x; t < kKeys * HD; t += kQ) {
            const int jj = t / HD, d = t % HD;
            flat[t] = j0 + jj < NP ? src[base + static_cast<int64_t>(j0 + jj) * L + d] : 0.0f;
        }
    };
    // pass 1: row max (fno.cpp:1444-1447)
    float mx = 0.0f;
    for (int j0 = 0; j0 < NP; j0 += kKeys) {
        load(sK, K, j0);
        __syncthreads();
        const int n = min(kKeys, NP - j0);
#pragma unroll 2
        for (int jj = 0; jj < n; ++jj) {
            const float s = score(jj);
            if (j0 + jj == 0) mx = s;
            else if (s > mx) mx = s;
        }
        __syncthreads();
    }
    // pass 2: sum of exp(s - max) in key order (fno.cpp:1448-1452)
    float sum = 0.0f;
    for (int j0 = 0; j0 < NP; j0 += kKeys) {
        load(sK, K, j0);
        __syncthreads();
        const int n = min(kKeys, NP - j0);
#pragma unroll 2
        for (int jj = 0; jj < n; ++jj) sum = __fadd_rn(sum, expf(__fsub_rn(score(jj), mx)));
        __syncthreads();
    }
    const float inv = __fdiv_rn(1.0f, sum);
    // pass 3: (e * inv) times V, summed in key order (fno.cpp:1919-1929)
    float acc[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) acc[d] = 0.0f;
    const int av_vec = (NP / 4) * 4;
    for (int j0 = 0; j0 < NP; j0 += kKeys) {
        load(sK, K, j0);
        load(sV, V, j0);
        __syncthreads();
        const int n = min(kKeys, NP - j0);
        for (int jj = 0; jj < n; ++jj) {
            const float p = __fmul_rn(expf(__fsub_rn(score(jj), mx)), inv);
            const bool fused = j0 + jj >= av_vec;
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; ++d4) {
                const float4 v4 = sV[jj][d4];
                acc[4 * d4 + 0] = linear_step(acc[4 * d4 + 0], p, v4.x, fused);
                acc[4 * d4 + 1] = linear_step(acc[4 * d4 + 1], p, v4.y, fused);
                acc[4 * d4 + 2] = linear_step(acc[4 * d4 + 2], p, v4.z, fused);
                acc[4 * d4 + 3] = linear_step(acc[4 * d4 + 3], p, v4.w, fused);
            }
        }
        __syncthreads();
    }
    if (live) {
#pragma unroll
        for (int d = 0; d < HD; ++d) out[base + static_cast<int64_t>(i) * L + d] = acc[d];
    }
}

// ---------------------------------------------------------------------------
// attention of the INT8 variant (no reference counterpart): one pass over the keys
// with an online softmax (running max, rescaled sum and accumulator), fused
// multiply-adds.  Same grid and shared-memory staging as attention_kernel; the result
// equals the reference-order attention to fp32 rounding, not bit for bit.
// ---------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(kQ) attention_online_kernel(const float* __restrict__ Q,
                                                              const float* __restrict__ K,
                                                              const float* __restrict__ V, int NP,
                                                              int L, float scale,
                                                              float* __restrict__ out) {
    constexpr int kKeys = HD <= 32 ? 128 : 64;
    __shared__ float4 sK[kKeys][HD / 4];
    __shared__ float4 sV[kKeys][HD / 4];
    const int b = blockIdx.z, head = blockIdx.y;
    const int i = blockIdx.x * kQ + threadIdx.x;
    const bool live = i < NP;
    const int64_t base = static_cast<int64_t>(b) * NP * L + head * HD;
    float q[HD], acc[HD];
#pragma unroll
    for (int d = 0; d < HD; ++d) {
        q[d] = live ? Q[base + static_cast<int64_t>(i) * L + d] : 0.0f;
        acc[d] = 0.0f;
    }
    float mx = -INFINITY, l = 0.0f;
    for (int j0 = 0; j0 < NP; j0 += kKeys) {
        float* fk = reinterpret_cast<float*>(sK);
        float* fv = reinterpret_cast<float*>(sV);
        for (int t = threadIdx.x; t < kKeys * HD; t += kQ) {
            const int jj = t / HD, d = t % HD;
            const bool in = j0 + jj < NP;
            fk[t] = in ? K[base + static_cast<int64_t>(j0 + jj) * L + d] : 0.0f;
            fv[t] = in ? V[base + static_cast<int64_t>(j0 + jj) * L + d] : 0.0f;
        }
        __syncthreads();
        const int n = min(kKeys, NP - j0);
        for (int jj = 0; jj < n; ++jj) {
            float sc = 0.0f;
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; ++d4) {
                const float4 k4 = sK[jj][d4];
                sc = fmaf(q[4 * d4], k4.x, sc);
                sc = fmaf(q[4 * d4 + 1], k4.y, sc);
                sc = fmaf(q[4 * d4 + 2], k4.z, sc);
                sc = fmaf(q[4 * d4 + 3], k4.w, sc);
            }
            sc *= scale;
            if (sc > mx) {
                const float c = expf(mx - sc);
                l *= c;
#pragma unroll
                for (int d = 0; d < HD; ++d) acc[d] *= c;
                mx = sc;
            }
            const float pj = expf(sc - mx);
            l += pj;
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; ++d4) {
                const float4 v4 = sV[jj][d4];
                acc[4 * d4] = fmaf(pj, v4.x, acc[4 * d4]);
                acc[4 * d4 + 1] = fmaf(pj, v4.y, acc[4 * d4 + 1]);
                acc[4 * d4 + 2] = fmaf(pj, v4.z, acc[4 * d4 + 2]);
                acc[4 * d4 + 3] = fmaf(pj, v4.w, acc[4 * d4 + 3]);
            }
        }
        __syncthreads();
    }
    if (live) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int d = 0; d < HD; ++d) out[base + static_cast<int64_t>(i) * L + d] = acc[d] * inv;
    }
}

// ---------------------------------------------------------------------------
// INT8 path: per-row qparams + codes.  32 rows per warp staged [32][K + 1].
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) row_quant_kernel(const float* __restrict__ A, int64_t rows,
                                                        int K, int8_t* __restrict__ codes,
                                                        float* __restrict__ row_s,
                                                        int32_t* __restrict__ row_zp) {
    extern __shared__ float sr[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* mine = sr + static_cast<size_t>(warp) * 32 * (K + 1);
    const int64_t r0 = (static_cast<int64_t>(blockIdx.x) * 4 + warp) * 32;
    for (int i = lane; i < 32 * K; i += 32) {
        const int rr = i / K, c = i % K;
        mine[rr * (K + 1) + c] = r0 + rr < rows ? A[(r0 + rr) * K + c] : 0.0f;
    }
    __syncwarp();
    const int64_t r = r0 + lane;
    float s = 1.0f;
    int zp = 0;
    if (r < rows) {
        const float* xr = mine + lane * (K + 1);
        float mn = xr[0], mx = xr[0];
        for (int i = 1; i < K; ++i) {
            if (xr[i] < mn) mn = xr[i];
            if (xr[i] > mx) mx = xr[i];
        }
        if (!(mx == mn || mn != mn || mx != mx)) {
            double sc = (static_cast<double>(mx) - static_cast<double>(mn)) / 255.0;
            const double raw = rint(-128.0 - static_cast<double>(mn) / sc);
            const double z = raw < -128.0 ? -128.0 : (raw > 127.0 ? 127.0 : raw);
            if (z != raw) sc = z == -128.0 ? static_cast<double>(mx) / 255.0 : -static_cast<double>(mn) / 255.0;
            s = static_cast<float>(sc);
            zp = static_cast<int>(z);
        }
        row_s[r] = s;
        row_zp[r] = zp;
    }
    // codes: each lane quantises its own row (QuantiseActivation)
    __syncwarp();
    const float my_s = s;
    const int my_zp = zp;
    for (int rr = 0; rr < 32; ++rr) {
        const float srow = __shfl_sync(0xffffffffu, my_s, rr);
        const int zrow = __shfl_sync(0xffffffffu, my_zp, rr);
        if (r0 + rr >= rows) break;
        for (int c = lane; c < K; c += 32)
            codes[(r0 + rr) * K + c] = static_cast<int8_t>(quantise_i8(mine[rr * (K + 1) + c], srow, zrow));
    }
}

__global__ void __launch_bounds__(256) add_kernel(float* __restrict__ t, const float* __restrict__ u,
                                                  int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        t[i] = __fadd_rn(t[i], u[i]);
}

cudaError_t linear(const LinArgs& a, cudaStream_t st) {
    const dim3 grid((a.N + kBN - 1) / kBN, static_cast<unsigned>((a.M + kBM - 1) / kBM));
    linear_f32_kernel<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

LinArgs lin(const float* A, int64_t M, int K, const float* W, const float* b, int N, float* C,
            int act = 0, const float* R = nullptr) {
    LinArgs a{};
    a.A = A;
    a.src = 0;
    a.W = W;
    a.bias = b;
    a.R = R;
    a.C = C;
    a.M = M;
    a.N = N;
    a.K = K;
    a.act = act;
    return a;
}

// ---------------------------------------------------------------------------
// attention_tc (head dim 32): softmax(Q K^T * scale) V on tensor cores in 3xTF32, one
// CTA per (128 queries, head, sample), keys in tiles of 64 (a flash-attention
// schedule: no n x n matrix).  Every operand x is held as the tf32 pair
// hi = x with its 13 low mantissa bits cleared and lo = x - hi (split_qkv_kernel for
// Q, K, V; the softmax warps for P), and each product as hi*hi + lo*hi + hi*lo
// (about 2^-21 relative error).
//   warp 0      TMA: the Q pair once, then K and V pairs of each key tile (ring of 2)
//   warp 1      MMA issuer: S_j = Q K_j^T into one of two TMEM buffers (64 columns),
//               O_j = P_j V_j into one of two TMEM buffers (32 columns)
//   warps 2-5   softmax, one query row per thread (TMEM lane): the row max, the
//               exponentials exp2((s - m) scale log2 e), the running sum, P_j written
//               to shared memory as the A operand, and O accumulated in registers with
//               the online rescaling; O / sum is written at the end
//   warps 6-7   V_j transposed into the K-major B operand (two buffers; an MN-major tf32
//               operand would need the 32-byte-atom swizzle)
// The result equals softmax attention to fp32 accuracy but not in the reference's
// summation order (fno.cpp:1441-1456, 1919-1929), which attention_kernel keeps.
// ---------------------------------------------------------------------------
struct AttnCfg {
    static constexpr int kQT = 128;                  // queries per CTA
    static constexpr int kKT = 64;                   // keys per tile
    static constexpr int kQBytes = kQT * 128;        // [128 rows][32 f32], SW128
    static constexpr int kKVBytes = kKT * 128;       // [64 rows][32 f32], SW128
    static constexpr int kStages = 2;
    static constexpr int kStageBytes = 4 * kKVBytes; // K hi, K lo, V hi, V lo
    static constexpr int kPBlk = kQT * 128;          // [128 rows][32 keys] f32, SW128
    static constexpr int kPBytes = 2 * kPBlk;        // 64 keys = two K blocks
    static constexpr int kOffQ = 0;                  // Q hi, Q lo
    static constexpr int kOffKV = 2 * kQBytes;
    static constexpr int kOffP = kOffKV + kStages * kStageBytes;  // P hi, P lo
    static constexpr int kVtBlk = 32 * 128;          // V^T [32 dims][32 keys] f32, SW128
    static constexpr int kVtBytes = 2 * kVtBlk;      // 64 keys
    static constexpr int kOffVt = kOffP + 2 * kPBytes;             // 2 x (V^T hi, V^T lo)
    static constexpr int kOffBars = kOffVt + 4 * kVtBytes;
    static constexpr int kSmemBytes = kOffBars + 256 + 1024;
    static constexpr int kThreads = 256;
    static constexpr int kTmemCols = 256;            // S 2 x 64 at 0, O 2 x 32 at 128
};

// hi / lo tf32 pairs of q, k and v (T rows x L): hi keeps the top 10 mantissa bits
__global__ void __launch_bounds__(256) split_qkv_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                        const float* __restrict__ v, int64_t n,
                                                        float* __restrict__ out) {
    const float* src[3] = {q, k, v};
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
#pragma unroll
        for (int t = 0; t < 3; ++t) {
            const float x = src[t][i];
            const float hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
            out[(2 * t) * n + i] = hi;
            out[(2 * t + 1) * n + i] = __fsub_rn(x, hi);
        }
    }
}

__global__ void __launch_bounds__(AttnCfg::kThreads, 1)
attention_tc_kernel(const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                    const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                    const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl, int NP,
                    int L, float scale, float* __restrict__ out, unsigned* err) {
    using F = AttnCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sQ = smem + F::kOffQ;
    uint8_t* sKV = smem + F::kOffKV;
    uint8_t* sP = smem + F::kOffP;
    uint8_t* sVt = smem + F::kOffVt;
    uint64_t* qFull = reinterpret_cast<uint64_t*>(smem + F::kOffBars);
    uint64_t* kvFull = qFull + 1;
    uint64_t* kvEmpty = kvFull + F::kStages;
    uint64_t* sFull = kvEmpty + F::kStages;
    uint64_t* sFree = sFull + 2;
    uint64_t* pReady = sFree + 2;
    uint64_t* oFull = pReady + 1;
    uint64_t* oFree = oFull + 2;
    uint64_t* vtReady = oFree + 2;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(vtReady + 2);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.z, head = blockIdx.y, q0 = blockIdx.x * F::kQT;
    const int row0 = b * NP;
    const int nt = (NP + F::kKT - 1) / F::kKT;

    if (threadIdx.x == 0) {
        mbar_init(qFull, 1);
        for (int s = 0; s < F::kStages; ++s) {
            mbar_init(&kvFull[s], 1);
            mbar_init(&kvEmpty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sFull[s], 1);
            mbar_init(&sFree[s], 4);
            mbar_init(&oFull[s], 1);
            mbar_init(&oFree[s], 4);
            mbar_init(&vtReady[s], 2);
        }
        mbar_init(pReady, 4);
        *sAbort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(sTmem, F::kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *sTmem;

    if (warp == 0) {
        if (elect_one()) {
            prefetch_tmap(&tmQh);
            prefetch_tmap(&tmKh);
            mbar_arrive_expect_tx(qFull, 2 * F::kQBytes);
            tma_load_2d(sQ, &tmQh, qFull, head * 32, row0 + q0);
            tma_load_2d(sQ + F::kQBytes, &tmQl, qFull, head * 32, row0 + q0);
            int j = 0;
            for (; j < nt; ++j) {
                const int s = j % F::kStages;
                if (!mbar_wait_backoff(&kvEmpty[s], ((j / F::kStages) & 1) ^ 1, sAbort, 512)) {
                    *sAbort = 1;
                    atomicOr(err, kErrWaitSlotFree);
                    break;
                }
                uint8_t* st = sKV + s * F::kStageBytes;
                const int y = row0 + j * F::kKT;
                mbar_arrive_expect_tx(&kvFull[s], F::kStageBytes);
                tma_load_2d(st, &tmKh, &kvFull[s], head * 32, y);
                tma_load_2d(st + F::kKVBytes, &tmKl, &kvFull[s], head * 32, y);
                tma_load_2d(st + 2 * F::kKVBytes, &tmVh, &kvFull[s], head * 32, y);
                tma_load_2d(st + 3 * F::kKVBytes, &tmVl, &kvFull[s], head * 32, y);
            }
            // every load issued lands before the CTA leaves
            if (!mbar_wait_drain(qFull, 0)) atomicOr(err, kErrWaitDrain);
            for (int i = (j > F::kStages ? j - F::kStages : 0); i < j; ++i)
                if (!mbar_wait_drain(&kvFull[i % F::kStages], (i / F::kStages) & 1)) {
                    atomicOr(err, kErrWaitDrain);
                    break;
                }
        }
        __syncwarp();
    }
    else if (warp == 1) {
        if (elect_one()) {
            constexpr uint32_t idS = idesc_tf32(F::kKT);          // A, B K-major
            constexpr uint32_t idO = idesc_tf32(32);                // B = V^T, K-major
            const uint32_t qh = smem_u32(sQ), ql = qh + F::kQBytes;
            const uint32_t ph = smem_u32(sP), pl = ph + F::kPBytes;
            bool ok = mbar_wait(qFull, 0, sAbort);
            uint64_t* last_bar = nullptr;   // the barrier of the last commit issued
            uint32_t last_ph = 0;
            auto s_issue = [&](int j) -> bool {
                const int s = j % F::kStages, bs = j & 1;
                if (!mbar_wait(&kvFull[s], (j / F::kStages) & 1, sAbort) ||
                    !mbar_wait(&sFree[bs], ((j >> 1) & 1) ^ 1, sAbort))
                    return false;
                tc_fence_after();
                const uint32_t kh = smem_u32(sKV + s * F::kStageBytes), kl = kh + F::kKVBytes;
                const uint32_t d = tmem_base + bs * F::kKT;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t a = umma_desc(qh + kk * 32, 128), al = umma_desc(ql + kk * 32, 128);
                    const uint64_t bh = umma_desc(kh + kk * 32, 128), bl = umma_desc(kl + kk * 32, 128);
                    mma_tf32(d, a, bh, idS, kk > 0 ? 1u : 0u);
                    mma_tf32(d, al, bh, idS, 1u);
                    mma_tf32(d, a, bl, idS, 1u);
                }
                mma_commit(&sFull[bs]);
                last_bar = &sFull[bs];
                last_ph = (j >> 1) & 1;
                return true;
            };
            auto pv_issue = [&](int j) -> bool {
                const int s = j % F::kStages, bs = j & 1;
                if (!mbar_wait(pReady, j & 1, sAbort) || !mbar_wait(&vtReady[bs], (j >> 1) & 1, sAbort) ||
                    !mbar_wait(&oFree[bs], ((j >> 1) & 1) ^ 1, sAbort))
                    return false;
                tc_fence_after();
                const uint32_t vh = smem_u32(sVt + bs * 2 * F::kVtBytes), vl = vh + F::kVtBytes;
                const uint32_t d = tmem_base + 128 + bs * 32;
#pragma unroll
                for (int kk = 0; kk < F::kKT / 8; ++kk) {
                    const uint32_t po = (kk >> 2) * F::kPBlk + (kk & 3) * 32;
                    const uint32_t vo = (kk >> 2) * F::kVtBlk + (kk & 3) * 32;
                    const uint64_t a = umma_desc(ph + po, 128), al = umma_desc(pl + po, 128);
                    const uint64_t bh = umma_desc(vh + vo, 128), bl = umma_desc(vl + vo, 128);
                    mma_tf32(d, a, bh, idO, kk > 0 ? 1u : 0u);
                    mma_tf32(d, al, bh, idO, 1u);
                    mma_tf32(d, a, bl, idO, 1u);
                }
                mma_commit(&oFull[bs]);
                mma_commit(&kvEmpty[s]);
                last_bar = &oFull[bs];
                last_ph = (j >> 1) & 1;
                return true;
            };
            if (ok) ok = s_issue(0);
            if (ok && nt > 1) ok = s_issue(1);
            for (int j = 0; j < nt && ok; ++j) {
                ok = pv_issue(j);
                if (ok && j + 2 < nt) ok = s_issue(j + 2);
            }
            if (!ok) {
                *sAbort = 1;
                atomicOr(err, kErrWaitAccFree);
            }
            // the MMAs issued so far (in order) complete before TMEM is released
            if (last_bar && !mbar_wait_drain(last_bar, last_ph)) atomicOr(err, kErrWaitDrain);
        }
        __syncwarp();
    } else if (warp >= 6) {
        // V_j -> V^T buffer j % 2 once PV_{j-2} (the buffer's previous reader) is done:
        // thread (warp, lane) moves dim `lane` of 32 keys
        const int k0 = (warp - 6) * 32;
        for (int j = 0; j < nt; ++j) {
            const int s = j % F::kStages, bs = j & 1;
            if (!mbar_wait(&kvFull[s], (j / F::kStages) & 1, sAbort) ||
                (j >= 2 && !mbar_wait(&oFull[bs], ((j - 2) >> 1) & 1, sAbort))) {
                *sAbort = 1;
                atomicOr(err, kErrWaitDrain);
                break;
            }
            const uint8_t* vsrc = sKV + s * F::kStageBytes + 2 * F::kKVBytes;
            uint8_t* vdst = sVt + bs * 2 * F::kVtBytes;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
#pragma unroll 8
                for (int kq = 0; kq < 32; ++kq) {
                    const int key = k0 + kq;
                    const float x = *reinterpret_cast<const float*>(vsrc + h * F::kKVBytes +
                                                                    swz_offset(key * 128 + lane * 4, 128));
                    *reinterpret_cast<float*>(vdst + h * F::kVtBytes + (key >> 5) * F::kVtBlk +
                                              swz_offset(lane * 128 + (key & 31) * 4, 128)) = x;
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&vtReady[bs]);
        }
    } else {
        // softmax: one query row per thread
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const float c2 = __fmul_rn(scale, 1.4426950408889634f);
        const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
        float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
        float o[32];
#pragma unroll
        for (int d = 0; d < 32; ++d) o[d] = 0.0f;
        auto take_o = [&](int j) -> bool {
            const int bs = j & 1;
            if (!mbar_wait(&oFull[bs], (j >> 1) & 1, sAbort)) return false;
            tc_fence_after();
            uint32_t ot[32];
            tmem_ld32(tmem_base + lane_base + 128 + bs * 32, ot);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 32; ++d) o[d] = fmaf(o[d], alpha_prev, __uint_as_float(ot[d]));
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&oFree[bs]);
            return true;
        };
        bool ok = true;
        for (int j = 0; j < nt && ok; ++j) {
            const int bs = j & 1;
            if (!mbar_wait(&sFull[bs], (j >> 1) & 1, sAbort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t sv[64];
            tmem_ld32(tmem_base + lane_base + bs * F::kKT, *reinterpret_cast<uint32_t(*)[32]>(sv));
            tmem_ld32(tmem_base + lane_base + bs * F::kKT + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
            tmem_wait_ld();
            asm volatile("" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sFree[bs]);
            const int nk = min(F::kKT, NP - j * F::kKT);
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int cc = 0; cc < 64; ++cc)
                if (cc < nk) mx4[cc & 3] = fmaxf(mx4[cc & 3], __uint_as_float(sv[cc]));
            const float m_new = fmaxf(m, fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])));
            const float alpha = m == -INFINITY ? 0.0f : exp2f((m - m_new) * c2);
            // the exponentials of S_j first (they overlap the MMA of P_{j-1} V_{j-1})
            float sum4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int cc = 0; cc < 64; ++cc) {
                const float p = cc < nk ? exp2f((__uint_as_float(sv[cc]) - m_new) * c2) : 0.0f;
                sum4[cc & 3] += p;
                sv[cc] = __float_as_uint(p);
            }
            // P_{j-1} has been consumed once O_{j-1} is ready: take it, then write P_j
            if (j > 0 && !take_o(j - 1)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int blk = 0; blk < 2; ++blk) {
#pragma unroll
                for (int c4 = 0; c4 < 8; ++c4) {
                    float ph4[4], pl4[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float p = __uint_as_float(sv[blk * 32 + c4 * 4 + u]);
                        ph4[u] = __uint_as_float(__float_as_uint(p) & 0xFFFFE000u);
                        pl4[u] = p - ph4[u];
                    }
                    const uint32_t off = blk * F::kPBlk + swz_offset(r * 128 + c4 * 16, 128);
                    *reinterpret_cast<float4*>(sP + off) = make_float4(ph4[0], ph4[1], ph4[2], ph4[3]);
                    *reinterpret_cast<float4*>(sP + F::kPBytes + off) = make_float4(pl4[0], pl4[1], pl4[2], pl4[3]);
                }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(pReady);
            l = fmaf(l, alpha, (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
            m = m_new;
            alpha_prev = alpha;
        }
        if (ok) ok = take_o(nt - 1);
        if (!ok) {
            *sAbort = 1;
            atomicOr(err, kErrWaitAccFull);
        } else if (q0 + r < NP) {
            const float inv = __fdiv_rn(1.0f, l);
            float* dst = out + static_cast<int64_t>(row0 + q0 + r) * L + head * 32;
#pragma unroll
            for (int d4 = 0; d4 < 8; ++d4)
                reinterpret_cast<float4*>(dst)[d4] =
                    make_float4(o[4 * d4] * inv, o[4 * d4 + 1] * inv, o[4 * d4 + 2] * inv, o[4 * d4 + 3] * inv);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, F::kTmemCols);
    }
}

template <int HD>
cudaError_t attention(const Tm2dPlan& p, cudaStream_t st) {
    const dim3 grid((p.NP + kQ - 1) / kQ, p.heads, p.B);
    // fno.cpp:1799: 1.0f / std::sqrt((float)head_dim), IEEE on the host
    const float scale = 1.0f / std::sqrt(static_cast<float>(HD));
    if constexpr (HD == 32) {
        if (p.tc_attention && p.qkv_split) {
            using F = AttnCfg;
            const int64_t T = static_cast<int64_t>(p.B) * p.NP;
            const int64_t n = T * p.L;
            const int sms = device_sm_count();
            split_qkv_kernel<<<static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * sms)), 256, 0, st>>>(
                p.q, p.k, p.v, n, p.qkv_split);
            CUtensorMap m[6];
            for (int t = 0; t < 6; ++t) {
                const int rows = (t == 0 || t == 1) ? F::kQT : F::kKT;
                if (!encode_2d(&m[t], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.qkv_split + t * n, p.L, T,
                               static_cast<uint64_t>(p.L) * 4, 32, rows, 128))
                    return cudaErrorInvalidValue;
            }
            cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(attention_tc_kernel), F::kSmemBytes);
            if (e != cudaSuccess) return e;
            attention_tc_kernel<<<dim3((p.NP + F::kQT - 1) / F::kQT, p.heads, p.B), F::kThreads, F::kSmemBytes, st>>>(
                m[0], m[1], m[2], m[3], m[4], m[5], p.NP, p.L, scale, p.ho, p.err);
            return cudaGetLastError();
        }
    }
    if (p.int8) attention_online_kernel<HD><<<grid, kQ, 0, st>>>(p.q, p.k, p.v, p.NP, p.L, scale, p.ho);
    else attention_kernel<HD><<<grid, kQ, 0, st>>>(p.q, p.k, p.v, p.NP, p.L, scale, p.ho);
    return cudaGetLastError();
}

}  // namespace

const char* tm2d_unsupported(int L, int heads, int in_d, int out_d) {
    if (heads < 1 || L % heads) return "TokenMixer2D: latent_dim must be a multiple of n_heads";
    const int hd = L / heads;
    if (hd != 8 && hd != 16 && hd != 32 && hd != 64)
        return "TokenMixer2D GPU executor: head_dim must be 8, 16, 32 or 64";
    if (L > 512 || in_d < 1 || out_d < 1) return "TokenMixer2D GPU executor: latent_dim <= 512";
    return nullptr;
}

cudaError_t tm2d_run(const Tm2dPlan& p, cudaStream_t st) {
    if (p.B == 0) return cudaSuccess;
    const int sms = device_sm_count();
    const int npts = p.h * p.w;
    const int pp = npts / p.NP;
    const int64_t T = static_cast<int64_t>(p.B) * p.NP;
    const int L = p.L;
    cudaError_t e;
    auto timed = [&](const char* name, auto&& fn) -> cudaError_t {
        if (p.timer) p.timer->begin(name, st);
        const cudaError_t r = fn();
        if (p.timer) p.timer->end(st);
        return r;
    };
    auto grid1 = [&](int64_t n) { return static_cast<int>(std::min<int64_t>((n + 255) / 256, sms * 16)); };
    // patches and the slice embedding (fno.cpp:1803-1825)
    e = timed("tm2d_embed", [&] {
        pool_kernel<<<grid1(T * p.in_d), 256, 0, st>>>(p.x, T * p.in_d, p.in_d, p.NP, pp, p.pooled);
        cudaError_t r = cudaGetLastError();
        if (r != cudaSuccess) return r;
        return linear(lin(p.pooled, T, p.in_d, p.se_w, p.se_b, L, p.tok), st);
    });
    if (e != cudaSuccess) return e;
    const size_t ln_smem = 4 * 32 * static_cast<size_t>(L + 1) * sizeof(float);
    const size_t q2_smem = 4 * 32 * static_cast<size_t>(2 * L + 1) * sizeof(float);
    if ((e = set_max_dynamic_smem(reinterpret_cast<const void*>(layer_norm_kernel), static_cast<int>(ln_smem))) != cudaSuccess ||
        (e = set_max_dynamic_smem(reinterpret_cast<const void*>(row_quant_kernel), static_cast<int>(q2_smem))) != cudaSuccess)
        return e;
    const unsigned rows_grid = static_cast<unsigned>((T + 127) / 128);
    auto layer_norm = [&](const float* g, const float* b) {
        layer_norm_kernel<<<rows_grid, 128, ln_smem, st>>>(p.tok, T, L, g, b, p.ln);
        return cudaGetLastError();
    };
    // INT8 Linear: codes + per-row qparams of A, then the GEMM with bias and the
    // epilogue activation `act` (GemmArgs code: 0 none, 1 GELU, 2 ReLU)
    auto linear8 = [&](const float* A, int K, const Tm2dInt8Linear& q8, const float* bias, int N,
                       int act, float* C) -> cudaError_t {
        const size_t sm = 4 * 32 * static_cast<size_t>(K + 1) * sizeof(float);
        row_quant_kernel<<<rows_grid, 128, sm, st>>>(A, T, K, p.codes, p.row_s, p.row_zp);
        cudaError_t r = cudaGetLastError();
        if (r != cudaSuccess) return r;
        GemmArgs g{};
        g.A = p.codes;
        g.scale_a = p.row_s;
        g.zp_a = p.row_zp;
        g.W = q8.Wq;
        g.scale_w = q8.scale_w;
        g.zp_w = q8.zp_w;
        g.sum_w = q8.sum_w;
        g.bias = bias;
        g.act = act;
        g.C = C;
        g.M = static_cast<int>(T);
        g.err = p.err;
        return gemm_i8_launch(g, K, N, st);
    };
    for (int li = 0; li < p.layers; ++li) {
        const Tm2dBlock& B = p.blk[li];
        if ((e = timed("tm2d_layer_norm", [&] { return layer_norm(B.w[0], B.b[0]); })) != cudaSuccess) return e;
        e = timed(p.int8 ? "tm2d_qkv_int8" : "tm2d_qkv", [&]() -> cudaError_t {
            cudaError_t r;
            if (p.int8) {
                if ((r = linear8(p.ln, L, B.q8[1], B.b[1], L, 0, p.q)) != cudaSuccess) return r;
                if ((r = linear8(p.ln, L, B.q8[2], B.b[2], L, 0, p.k)) != cudaSuccess) return r;
                return linear8(p.ln, L, B.q8[3], B.b[3], L, 0, p.v);
            }
            if ((r = linear(lin(p.ln, T, L, B.w[1], B.b[1], L, p.q), st)) != cudaSuccess) return r;
            if ((r = linear(lin(p.ln, T, L, B.w[2], B.b[2], L, p.k), st)) != cudaSuccess) return r;
            return linear(lin(p.ln, T, L, B.w[3], B.b[3], L, p.v), st);
        });
        if (e != cudaSuccess) return e;
        e = timed("tm2d_attention", [&]() -> cudaError_t {
            switch (L / p.heads) {
                case 8: return attention<8>(p, st);
                case 16: return attention<16>(p, st);
                case 32: return attention<32>(p, st);
                default: return attention<64>(p, st);
            }
        });
        if (e != cudaSuccess) return e;
        e = timed(p.int8 ? "tm2d_o_int8" : "tm2d_o", [&]() -> cudaError_t {
            if (!p.int8) return linear(lin(p.ho, T, L, B.w[4], B.b[4], L, p.tok, 0, p.tok), st);
            cudaError_t r = linear8(p.ho, L, B.q8[4], B.b[4], L, 0, p.f1);
            if (r != cudaSuccess) return r;
            add_kernel<<<grid1(T * L), 256, 0, st>>>(p.tok, p.f1, T * L);
            return cudaGetLastError();
        });
        if (e != cudaSuccess) return e;
        if ((e = timed("tm2d_layer_norm", [&] { return layer_norm(B.w[5], B.b[5]); })) != cudaSuccess) return e;
        e = timed(p.int8 ? "tm2d_ffn_int8" : "tm2d_ffn", [&]() -> cudaError_t {
            const int act = p.act == 1 ? 2 : 1;
            cudaError_t r;
            if (!p.int8) {
                if ((r = linear(lin(p.ln, T, L, B.w[6], B.b[6], 2 * L, p.f0, act), st)) != cudaSuccess) return r;
                return linear(lin(p.f0, T, 2 * L, B.w[7], B.b[7], L, p.tok, 0, p.tok), st);
            }
            if ((r = linear8(p.ln, L, B.q8[6], B.b[6], 2 * L, act, p.f0)) != cudaSuccess) return r;
            if ((r = linear8(p.f0, 2 * L, B.q8[7], B.b[7], L, 0, p.f1)) != cudaSuccess) return r;
            add_kernel<<<grid1(T * L), 256, 0, st>>>(p.tok, p.f1, T * L);
            return cudaGetLastError();
        });
        if (e != cudaSuccess) return e;
    }
    // unslice + head (fno.cpp:1935-1954)
    e = timed("tm2d_decode", [&]() -> cudaError_t {
        const int64_t P = static_cast<int64_t>(p.B) * npts;
        LinArgs a = lin(nullptr, P, p.in_d + L, p.un_w, p.un_b, L, p.feat);
        a.src = 1;
        a.x = p.x;
        a.tok = p.tok;
        a.in_d = p.in_d;
        a.L = L;
        a.pp = pp;
        a.npts = npts;
        cudaError_t r = linear(a, st);
        if (r != cudaSuccess) return r;
        return linear(lin(p.feat, P, L, p.head_w, p.head_b, p.out_d, p.y), st);
    });
    return e;
}

}  // namespace nfx
