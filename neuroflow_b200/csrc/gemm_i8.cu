// gemm_i8.cu -- W8A8 INT8 GEMM with the reference dequant epilogue on tcgen05.
//
// Computes, for activation codes A (M x K, int8, row-major) and per-channel weight
// codes W (N x K, int8, PyTorch (out, in) layout):
//   raw[m, o] = sum_k A[m,k] * W[o,k]                      (tcgen05.mma kind::i8)
//   sum_a[m]  = sum_k A[m,k]                                (same MMA, a ones row)
//   y[m, o]   = LinearForwardBatched epilogue (int8_gemm.cpp:559-578) with the row's
//               (scale_A, zp_A), then + bias[o] (fno.cpp:541-548), then GELU
//               (fno.cpp:36-48, in the sigmoid form of gelu_fast) when requested.
// The int32 accumulator acc = raw - zp_w*sum_a is exactly the reference's.
//
// Structure (persistent, warp-specialised, one CTA per SM):
//   warp 0      TMA producer: A tiles (128 rows x K) into a kStages ring.
//   warp 1      TMEM owner + MMA issuer (one elected lane).
//   warps 4-19  epilogue: 4 warps per TMEM lane quadrant, N/4 columns each;
//               tcgen05.ld from TMEM, integer/float epilogue with the column
//               constants in one 16-byte shared load, swizzled staging in shared
//               memory, TMA store of fp32 tiles of 16 (or 8) columns.
// The weight tile (N x K, <= 64 KB) stays resident in shared memory for the CTA's
// lifetime; TMEM holds two accumulator stages when they fit so that the MMA of tile
// t+1 overlaps the epilogue of tile t.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "numerics.cuh"
#include "sm100.cuh"
#include "nfx_internal.h"

namespace nfx {
namespace {

constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 16;                           // 4 per TMEM lane quadrant
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);  // warps 2-3 idle

constexpr int pow2ceil(int v) {
    int p = 32;
    while (p < v) p <<= 1;
    return p;
}

template <int K, int N>
struct Cfg {
    static constexpr int kRowBytes = K >= 128 ? 128 : K;  // swizzle row width
    static constexpr int kKBlocks = K / kRowBytes;         // 2 only for K = 256
    static constexpr int kABytes = 128 * K;
    // A-tile ring: about 64 KB of loads in flight per SM (2 to 16 tiles)
    static constexpr int kStages = (65536 / kABytes) < 2 ? 2 : ((65536 / kABytes) > 16 ? 16 : 65536 / kABytes);
    // accumulator stage: N columns + a 16-column block for sum_a, rounded to 32 columns
    static constexpr int kAccCols = ((N + 16 + 31) / 32) * 32;
    // Epilogue warp groups (one warp per lane quadrant and column part each) take
    // turns over the CTA's tiles, group g always draining accumulator stage g: as
    // many groups as stages fit in TMEM (at most 4), so narrow tiles keep up to four
    // tiles in flight and every warp handles N / kSplit columns of its tiles.
    static constexpr int kGroups = (4 * kAccCols <= 512) ? 4 : ((2 * kAccCols <= 512) ? 2 : 1);
    static constexpr int kAccStages = kGroups;
    static constexpr int kSplit = 4 / kGroups;           // column parts per group
    static constexpr int kTmemCols = pow2ceil(kAccStages * kAccCols);
    static constexpr int kCols = N / kSplit;             // columns per epilogue warp
    static constexpr int kCh = kCols < 16 ? kCols : 16;  // columns per TMEM load / store box
    static constexpr int kStageBytes = 32 * kCh * 4;     // one staging buffer (32 rows)
    // shared memory map (offsets from a 1024-aligned base)
    static constexpr int kOffW = 0;
    static constexpr int kWBytes = ((N * K + 1023) / 1024) * 1024;
    static constexpr int kOffOnes = kOffW + kWBytes;
    static constexpr int kOnesBytes = ((16 * K + 1023) / 1024) * 1024;
    static constexpr int kOffA = kOffOnes + kOnesBytes;
    static constexpr int kOffStage = kOffA + kStages * kABytes;
    static constexpr int kOffParams = kOffStage + kEpiWarps * 2 * kStageBytes;
    static constexpr int kParamBytes = N * 16;
    static constexpr int kOffBars = kOffParams + kParamBytes;
    static constexpr int kBarBytes = 8 * (2 * kStages + 2 * kAccStages) + 16;
    static constexpr int kSmemBytes = kOffBars + kBarBytes + 1024;  // + alignment slack
    static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
    static_assert(N % 32 == 0 && N >= 32 && N <= 256, "N");
    static_assert(K % 32 == 0 && K >= 32 && K <= 256, "K");
};

template <int CH>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[CH]) {
    if constexpr (CH == 16) {
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
            "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
              "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
              "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
            : "r"(taddr));
    } else {
        static_assert(CH == 8, "chunk");
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
              "=r"(r[6]), "=r"(r[7])
            : "r"(taddr));
    }
}
template <int CH>
__device__ __forceinline__ void tmem_wait_cols(uint32_t (&r)[CH], uint32_t& x) {
    if constexpr (CH == 16) {
        asm volatile("tcgen05.wait::ld.sync.aligned;"
                     : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                       "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                       "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(x)
                     :
                     : "memory");
    } else {
        asm volatile("tcgen05.wait::ld.sync.aligned;"
                     : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                       "+r"(r[6]), "+r"(r[7]), "+r"(x)
                     :
                     : "memory");
    }
}

// GELU (fno.cpp:36-48) as z * sigmoid(2u) = z / (1 + 2^(-2 u log2 e)), u = c (z +
// 0.044715 z^3) with the reference's contraction of the cubic term.  This is the
// identity 0.5 (1 + tanh u) = 1 / (1 + e^(-2u)); the exponential is the hardware
// base-2 approximation (ex2.approx, relative error ~2^-22), so the result is within a
// few ulp of the exact GELU -- no cancellation for u << 0, unlike 1 + tanh(u).
__device__ __forceinline__ float gelu_fast(float z) {
    const float c2 = -2.0f * 0.7978845608028654f * 1.4426950408889634f;  // -2 sqrt(2/pi) log2(e)
    const float t = __fmul_rn(__fmul_rn(0.044715f, z), z);
    const float inner = __fmaf_rn(z, t, z);
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(c2, inner)));
    return __fdividef(z, __fadd_rn(1.0f, e));
}

template <int K, int N>
__global__ void __launch_bounds__(kThreads, 1)
gemm_i8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmC,
               const GemmArgs p) {
    using C = Cfg<K, N>;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, derived by indexing the shared array so that the
    // compiler keeps shared-memory (not generic) loads and stores through it
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sW = smem + C::kOffW;
    uint8_t* sOnes = smem + C::kOffOnes;
    uint8_t* sA = smem + C::kOffA;
    uint8_t* sStage = smem + C::kOffStage;
    float4* sCol = reinterpret_cast<float4*>(smem + C::kOffParams);  // {sW, zp_w, sum_w, bias}
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBars);
    uint64_t* empty = full + C::kStages;
    uint64_t* accFull = empty + C::kStages;
    uint64_t* accEmpty = accFull + C::kAccStages;
    uint32_t* sTmem = reinterpret_cast<uint32_t*>(accEmpty + C::kAccStages);
    volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = (p.M + 127) / 128;
    const uint64_t budget = p.wait_ns ? p.wait_ns : kWaitNs;

    // ---- one-time set-up: weights (swizzled), ones block, column params, barriers
    {
        constexpr int kChunksPerRow = K / 16;
        for (int idx = threadIdx.x; idx < N * kChunksPerRow; idx += kThreads) {
            const int o = idx / kChunksPerRow, c = idx % kChunksPerRow;
            const int kb = (c * 16) / C::kRowBytes, off = (c * 16) % C::kRowBytes;
            const uint4 v = *reinterpret_cast<const uint4*>(p.W + static_cast<size_t>(o) * K + c * 16);
            *reinterpret_cast<uint4*>(sW + kb * N * C::kRowBytes +
                                      swz_offset(o * C::kRowBytes + off, C::kRowBytes)) = v;
        }
        for (int idx = threadIdx.x; idx < C::kOnesBytes / 16; idx += kThreads) {
            // rows of 16 x kRowBytes per K block; row 0 of every block is all ones.
            const int blk_bytes = 16 * C::kRowBytes;
            const int in_blk = (idx * 16) % blk_bytes;
            const bool row0 = (idx * 16) < C::kKBlocks * blk_bytes && in_blk < C::kRowBytes;
            const uint32_t one = row0 ? 0x01010101u : 0u;
            *reinterpret_cast<uint4*>(sOnes + idx * 16) = make_uint4(one, one, one, one);
        }
        for (int o = threadIdx.x; o < N; o += kThreads) {
            // (y + 0.0f) + b equals y + b' with b' = b except that a bias of -0.0
            // becomes +0.0 (the only value for which the "+ 0.0f" of the reference
            // epilogue is observable after the bias add); no bias means b' = +0.0.
            float b = p.bias ? p.bias[o] : 0.0f;
            if (b == 0.0f) b = 0.0f;
            sCol[o] = make_float4(p.scale_w[o], __int_as_float(p.zp_w[o]), __int_as_float(p.sum_w[o]), b);
        }
        if (threadIdx.x == 0) {
            for (int s = 0; s < C::kStages; ++s) {
                mbar_init(&full[s], 1);
                mbar_init(&empty[s], 1);
            }
            for (int s = 0; s < C::kAccStages; ++s) {
                mbar_init(&accFull[s], 1);
                mbar_init(&accEmpty[s], 4 * C::kSplit);
            }
            *sAbort = 0;
            fence_mbar_init();
        }
        if (warp == 1) tmem_alloc(sTmem, C::kTmemCols);
        fence_proxy_async_smem();  // weights/ones written by the generic proxy, read by MMA
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }
    const uint32_t tmem_base = *sTmem;

    if (warp == 0) {
        // ---------------- TMA producer
        if (elect_one()) {
            prefetch_tmap(&tmA);
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
                const int s = it % C::kStages;
                const uint32_t ph = (it / C::kStages) & 1;
                if (!mbar_wait_backoff(&empty[s], ph ^ 1, sAbort, 1024, 32, budget)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitSlotFree);
                    break;
                }
                mbar_arrive_expect_tx(&full[s], C::kABytes);
                for (int kb = 0; kb < C::kKBlocks; ++kb)
                    tma_load_2d(sA + s * C::kABytes + kb * 128 * C::kRowBytes, &tmA, &full[s],
                                kb * C::kRowBytes, tile * 128);
            }
            // Drain: every load this thread issued must land before the CTA exits, also
            // after an abort (the loads complete by themselves).
            const int issued = it;
            for (int j = (issued > C::kStages ? issued - C::kStages : 0); j < issued; ++j) {
                if (!mbar_wait_drain(&full[j % C::kStages], (j / C::kStages) & 1)) {
                    atomicOr(p.err, kErrWaitDrain);
                    break;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (elect_one()) {
            int it = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
                const int s = it % C::kStages;
                const uint32_t ph = (it / C::kStages) & 1;
                const int a = it % C::kAccStages;
                const uint32_t aph = (it / C::kAccStages) & 1;
                if (!mbar_wait_backoff(&accEmpty[a], aph ^ 1, sAbort, 128, 32, budget)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitAccFree);
                    break;
                }
                if (!mbar_wait_backoff(&full[s], ph, sAbort, 128, 32, budget)) {
                    *sAbort = 1;
                    atomicOr(p.err, kErrWaitTmaFull);
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + a * C::kAccCols;
                const uint32_t aBase = smem_u32(sA + s * C::kABytes);
                const uint32_t wBase = smem_u32(sW);
                const uint32_t oBase = smem_u32(sOnes);
#pragma unroll
                for (int kk = 0; kk < K / 32; ++kk) {
                    const int kb = (kk * 32) / C::kRowBytes, off = (kk * 32) % C::kRowBytes;
                    const uint64_t ad = umma_desc(aBase + kb * 128 * C::kRowBytes + off, C::kRowBytes);
                    const uint64_t wd = umma_desc(wBase + kb * N * C::kRowBytes + off, C::kRowBytes);
                    const uint64_t od = umma_desc(oBase + kb * 16 * C::kRowBytes + off, C::kRowBytes);
                    mma_i8(d, ad, wd, idesc_i8(N), kk > 0 ? 1u : 0u);
                    mma_i8(d + N, ad, od, idesc_i8(16), kk > 0 ? 1u : 0u);
                }
                mma_commit(&empty[s]);
                mma_commit(&accFull[a]);
            }
            // Drain: the last commit must complete before TMEM is released, also after
            // an abort (the MMAs issued so far complete by themselves, in order).
            if (it > 0) {
                const int j = it - 1;
                if (!mbar_wait_drain(&accFull[j % C::kAccStages], (j / C::kAccStages) & 1))
                    atomicOr(p.err, kErrWaitDrain);
            }
        }
        __syncwarp();
    } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kEpiWarps) {
        // ---------------- epilogue: 4 warps per lane quadrant, N/4 columns each
        const int ew = warp - kEpiWarp0;
        const int quad = warp & 3;               // TMEM lanes 32*quad .. +31
        const int grp = (ew >> 2) / C::kSplit;   // tiles it = grp (mod kGroups)
        const int col0 = ((ew >> 2) % C::kSplit) * C::kCols;  // this warp's column range
        uint8_t* myStage = sStage + ew * 2 * C::kStageBytes;
        const bool per_row = p.scale_a != nullptr;
        // the row's (scale_A, zp_A) of the next tile are loaded one tile ahead
        auto row_params = [&](int tile, float& sa, int& za) {
            const int m = tile * 128 + quad * 32 + lane;
            sa = p.scale_a_t;
            za = p.zp_a_t;
            if (per_row && tile < num_tiles && m < p.M) {
                sa = __ldg(p.scale_a + m);
                za = __ldg(p.zp_a + m);
            }
        };
        float sA_next;
        int zA_next;
        const int tstride = C::kGroups * gridDim.x;
        row_params(blockIdx.x + grp * gridDim.x, sA_next, zA_next);
        int nstore = 0;
        for (int it = grp, tile = blockIdx.x + grp * gridDim.x; tile < num_tiles;
             it += C::kGroups, tile += tstride) {
            const float sAr = sA_next;
            const int zA = zA_next;
            row_params(tile + tstride, sA_next, zA_next);
            const int a = it % C::kAccStages;
            const uint32_t aph = (it / C::kAccStages) & 1;
            if (!mbar_wait(&accFull[a], aph, sAbort, budget)) {
                *sAbort = 1;
                atomicOr(p.err, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + a * C::kAccCols;
            uint32_t sum_u;
            tmem_ld1(tbase + N, sum_u);
            const int nzA = -zA;
#pragma unroll 1
            for (int c0 = col0; c0 < col0 + C::kCols; c0 += C::kCh) {
                uint32_t raw[C::kCh];
                tmem_ld_cols<C::kCh>(tbase + c0, raw);
                tmem_wait_cols<C::kCh>(raw, sum_u);
                if (c0 + C::kCh >= col0 + C::kCols) {
                    // last TMEM read of this accumulator stage by this warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&accEmpty[a]);
                }
                const int rconst = K * zA - 2 * static_cast<int>(sum_u);
                float y[C::kCh];
#pragma unroll
                for (int j = 0; j < C::kCh; ++j) {
                    const float4 cp = sCol[c0 + j];
                    // LinearForwardBatched (int8_gemm.cpp:574-577): v = acc - zp_w*sum_a -
                    // zp_A*sum_w + K*zp_w*zp_A with acc = raw - zp_w*sum_a
                    const int v = static_cast<int>(raw[j]) + __float_as_int(cp.y) * rconst +
                                  nzA * __float_as_int(cp.z);
                    float t = __fmul_rn(__fmul_rn(cp.x, sAr), __int2float_rn(v));
                    t = __fadd_rn(t, cp.w);
                    if (p.act == 1) t = gelu_fast(t);
                    else if (p.act == 2) t = relu_ref(t);
                    y[j] = t;
                }
                // staging buffer (double-buffered per warp); make sure the TMA store
                // that last used it has finished reading.
                uint8_t* buf = myStage + (nstore & 1) * C::kStageBytes;
                if (nstore >= 2) {
                    if (lane == 0) tma_store_wait_read<1>();
                    __syncwarp();
                }
                constexpr int kRow = C::kCh * 4;
#pragma unroll
                for (int j4 = 0; j4 < C::kCh / 4; ++j4) {
                    const uint32_t off = swz_offset(lane * kRow + j4 * 16, kRow);
                    *reinterpret_cast<float4*>(buf + off) =
                        make_float4(y[4 * j4], y[4 * j4 + 1], y[4 * j4 + 2], y[4 * j4 + 3]);
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tmC, buf, c0, tile * 128 + quad * 32);
                    tma_store_commit();
                }
                ++nstore;
            }
        }
        if (lane == 0) tma_store_wait_all<0>();
        __syncwarp();
    }

    // ---- teardown
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}

template <int K, int N>
cudaError_t launch(const GemmArgs& p, const CUtensorMap& tmA, int num_sms, cudaStream_t stream) {
    using C = Cfg<K, N>;
    // output tiles of kCh columns x 32 rows, swizzled like the staging buffers
    CUtensorMap tmC;
    if (!encode_2d(&tmC, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.C, N, p.M, static_cast<uint64_t>(N) * 4,
                   C::kCh, 32, C::kCh * 4))
        return cudaErrorInvalidValue;
    auto kern = gemm_i8_kernel<K, N>;
    cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(kern), C::kSmemBytes);
    if (e != cudaSuccess) return e;
    const int tiles = (p.M + 127) / 128;
    const int grid = tiles < num_sms ? tiles : num_sms;
    kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tmA, tmC, p);
    return cudaGetLastError();
}

template <int K>
cudaError_t dispatch_n(int N, const GemmArgs& p, const CUtensorMap& a, int sms, cudaStream_t s) {
    switch (N) {
        case 32: return launch<K, 32>(p, a, sms, s);
        case 64: return launch<K, 64>(p, a, sms, s);
        case 128: return launch<K, 128>(p, a, sms, s);
        case 256: return launch<K, 256>(p, a, sms, s);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

bool gemm_i8_supported(int K, int N) {
    auto ok = [](int v) { return v == 32 || v == 64 || v == 128 || v == 256; };
    return ok(K) && ok(N);
}

cudaError_t gemm_i8_launch(const GemmArgs& p_in, int K, int N, cudaStream_t stream) {
    GemmArgs p = p_in;
    p.wait_ns = debug_wait_budget_ns();
    const int row_bytes = K >= 128 ? 128 : K;
    CUtensorMap tmA;
    if (!encode_2d(&tmA, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.A, K, p.M, K, row_bytes, 128, row_bytes))
        return cudaErrorInvalidValue;
    const int sms = device_sm_count();
    switch (K) {
        case 32: return dispatch_n<32>(N, p, tmA, sms, stream);
        case 64: return dispatch_n<64>(N, p, tmA, sms, stream);
        case 128: return dispatch_n<128>(N, p, tmA, sms, stream);
        case 256: return dispatch_n<256>(N, p, tmA, sms, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace nfx
