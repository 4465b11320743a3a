// tm2d.h -- host/device interface of the TokenMixer2D executor (tm2d.cu).
//
// FP32 path: the reference TokenMixer2D::Forward (cpp/src/fno.cpp:1756-1956), as
// InferenceRuntime::RunTokenMixer2D runs it.  INT8 path (EnableInt8Gemm, no reference
// counterpart: the reference runtime ignores NIRQ for this op): q, k, v, o, ffn0 and
// ffn1 run through the tcgen05 INT8 GEMM with per-token (per-row) activation qparams
// computed on the fly and per-channel weight codes; everything else as the FP32 path.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "nfx_internal.h"

namespace nfx {

constexpr int kTm2dMaxLayers = 8;

struct Tm2dInt8Linear {
    const int8_t* Wq;       // (N, K) codes
    const float* scale_w;   // (N,)
    const int32_t* zp_w;
    const int32_t* sum_w;
};

struct Tm2dBlock {
    const float* w[8];      // ln1, q, k, v, o, ln2, ffn0, ffn1 (weight)
    const float* b[8];      // (bias)
    Tm2dInt8Linear q8[8];   // INT8 path: slots 1, 2, 3, 4, 6, 7
};

struct Tm2dPlan {
    int B, in_d, out_d, L, h, w, NP, heads, layers, act, int8;
    const float* x;         // (B, h, w, in_d)
    float* y;               // (B, h, w, out_d)
    const float* se_w;      // slice_embed.proj (L, in_d)
    const float* se_b;
    const float* un_w;      // unslice.proj (L, in_d + L)
    const float* un_b;
    const float* head_w;    // (out_d, L)
    const float* head_b;
    Tm2dBlock blk[kTm2dMaxLayers];
    // scratch (device)
    float* pooled;          // (B*NP, in_d)
    float* tok;             // (B*NP, L)
    float* ln;              // (B*NP, L)
    float* q;               // (B*NP, L) x3 (q, k, v)
    float* k;
    float* v;
    float* ho;              // (B*NP, L)
    float* f0;              // (B*NP, 2L)
    float* f1;              // (B*NP, L)
    float* feat;            // (B*h*w, L)
    float* qkv_split;       // (6, B*NP, L): tf32 hi / lo pairs of q, k, v (tensor-core attention)
    int tc_attention;       // 1: attention on tensor cores (head dim 32), else on CUDA cores
    int8_t* codes;          // INT8 path: (B*NP, 2L) activation codes
    float* row_s;           // (B*NP,) per-row scales
    int32_t* row_zp;
    unsigned* err;
    KernelTimer* timer;
};

const char* tm2d_unsupported(int L, int heads, int in_d, int out_d);
cudaError_t tm2d_run(const Tm2dPlan& plan, cudaStream_t stream);

}  // namespace nfx
