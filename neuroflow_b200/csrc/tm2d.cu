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
//
// Approximate operations: CUDA's expf in the softmax and tanhf in GELU (a few ulps
// from glibc's); everything else is bit-identical to the reference arithmetic.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>

#include "nfx_internal.h"
#include "numerics.cuh"
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
        for (int kk = 0; kk < kend; ++kk) {
            const bool fused = k0 + kk >= nu;
            float av[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[j] = Ws[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = linear_step(acc[i][j], av[i], wv[j], fused);
        }
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

template <int HD>
cudaError_t attention(const Tm2dPlan& p, cudaStream_t st) {
    const dim3 grid((p.NP + kQ - 1) / kQ, p.heads, p.B);
    // fno.cpp:1799: 1.0f / std::sqrt((float)head_dim), IEEE on the host
    const float scale = 1.0f / std::sqrt(static_cast<float>(HD));
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
