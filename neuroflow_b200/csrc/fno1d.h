// fno1d.h -- host/device interface of the FNO1d executor (fno1d.cu).
//
// The executor reproduces the reference FNO1d::Forward (cpp/src/fno.cpp:408-706) after
// InferenceRuntime::Create (load-time weight fake-quant) and, optionally,
// EnableInt8Gemm (fno.cpp:360-406): every branch the reference takes per layer -- the
// per-tensor input snap, INT8 LinearForwardBatched or FP32 Linear for the local layer,
// the FP8 / per-token / per-tensor output fake-quant -- is decided on the host from
// the IR exactly as the reference decides it, and run on the GPU.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "nfx_internal.h"

namespace nfx {

constexpr int kFno1dMaxLayers = 8;

struct Fno1dLayer {
    const float* wr;        // (C, C, modes) spectral weights, real (fake-quantised at load)
    const float* wi;        // imaginary
    const float* loc_w;     // (C, C) fp32, (out, in)
    const float* loc_b;     // (C,)
    // layer-input snap (fno.cpp:488-508): the input buffer holds int8 codes when set
    int in_codes;
    float in_s;
    int in_zp;
    // INT8 local layer (LinearDispatchTryInt8, fno.cpp:125-159); needs in_codes
    int use_int8;
    const int8_t* Wq;
    const float* scale_w;
    const int32_t* zp_w;
    const int32_t* sum_w;
    // output fake-quant of locs.i.output (fno.cpp:572-654):
    // 0 none, 1 per-tensor INT8, 2 per-token, 3 FP8 log2 snap
    int fq_kind;
    float fq_s;
    int fq_zp;
    const float* pt_s;      // per-token scales, read at index c*N + p (the reference's flat index)
    const int32_t* pt_zp;
    // output of the layer: next-layer codes (out_codes = 1, snapped with out_s/out_zp)
    // or the fp32 activation
    int out_codes;
    float out_s;
    int out_zp;
    const int2* code_lut;   // exact z -> code table (nullptr: evaluate directly)
    int lut_cells;
    float lut_zlo, lut_inv_delta;
};

struct Fno1dPlan {
    int B, n, N, C, in_ch, out_ch, modes, L, act;  // N = padded length (power of two)
    const float* x;          // (B, n, in_ch)
    float* y;                // (B, n, out_ch)
    const float* lift_w;     // (C, in_ch)
    const float* lift_b;
    const float* pq_w;       // (C, C)
    const float* pq_b;
    const float* po_w;       // (out_ch, C)
    const float* po_b;
    Fno1dLayer layer[kFno1dMaxLayers];
    const float2* tw_fwd;    // recurrence twiddles for length N (nfx_lut.h)
    const float2* tw_inv;
    void* h[2];              // ping-pong activations (B, N, C): int8 codes or fp32
    float2* Xs;              // (B, C, modes) truncated spectra
    float* x2raw;            // (B*N, C) INT8 GEMM output (dequantised, before the bias)
    float* x1f;              // (B, C, N) spectral branch of the split layer, or null
    unsigned* err;
    KernelTimer* timer;
};

// Largest supported padded length and width.
constexpr int kFno1dMaxN = 8192;
constexpr int kFno1dMaxC = 256;
cudaError_t fno1d_run(const Fno1dPlan& plan, cudaStream_t stream);

}  // namespace nfx
