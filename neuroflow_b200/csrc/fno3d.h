// fno3d.h -- host/device interface of the FNO3d executor (fno3d.cu).
//
// FP32 path: the reference FNO3d::Forward (cpp/src/fno.cpp:1096-1281), as
// InferenceRuntime::Run executes it (no quantisation: the runtime builds FNO3d without
// its NIRQ block).  FP8 path (nfx_runtime_enable_fp8, no reference counterpart): the
// E4M3 variant -- per-tensor E4M3 weights, E4M3 activation codes between layers with
// the ".output" scales, E4M3 fake-quant at FNO2d's output boundaries.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "nfx_internal.h"

namespace nfx {

constexpr int kFno3dMaxLayers = 8;

struct Fno3dLayer {
    const float* wr;       // (C, C, MH, MW, MD) spectral weights
    const float* wi;
    const float* loc_w;    // (C, C) fp32 (FP32 path)
    const float* loc_q;    // (C, C) decoded E4M3 weights (FP8 path)
    const float* loc_b;
    float s_in;            // FP8: scale of the layer-input codes
    float s_w;             // FP8: weight scale
    float s_out;           // FP8: locs.i.output scale (x2 fake-quant and the output codes)
};

struct Fno3dPlan {
    int B, H, W, D, Hp, Wp, Dp, C, MH, MW, MD, L, in_ch, out_ch, act, fp8;
    const float* x;        // (B, H, W, D, in_ch)
    float* y;              // (B, H, W, D, out_ch)
    const float* lift_w;   // (C, in_ch) (FP8: fake-quantised)
    const float* lift_b;
    float s_lift;          // FP8: lift.output scale
    Fno3dLayer layer[kFno3dMaxLayers];
    const float* pq_w;     // (C, C) fp32
    const float* pq_q;     // decoded E4M3 proj_q weights
    const float* pq_b;
    float s_pq_w, s_pq;    // FP8: proj_q weight scale, proj_q.output scale
    const float* po_w;     // (out_ch, C) (FP8: fake-quantised)
    const float* po_b;
    float s_po;            // FP8: proj_out.output scale
    const float2* tw[6];   // recurrence twiddles: fwd/inv for Hp, Wp, Dp
    void* h[2];            // activations (B, C, Hp, Wp, Dp): fp32, or E4M3 bytes (FP8)
    float2* A;             // (B, C, Hp, MW, MD) after the D and W passes
    float2* Xs;            // (B, C, MH, MW, MD)
    float2* colinv;        // (B, C, Hp, MW, MD) after the H inverse pass
    float* x1;             // (B, C, Hp, Wp, Dp) spectral branch output
    const float* dft;      // direct-DFT tables (fno3d_dft_tables), or null: radix-2 passes
    KernelTimer* timer;
    // FP8 parity taps (nullptr: off): the E4M3 codes of every layer input -- the lift's
    // output, then each layer's output -- copied as L + 1 consecutive (B, C, Hp, Wp, Dp)
    // blocks after the kernel that wrote them
    uint8_t* tap_codes;
};

// The FP8 variant at widths 32 and 64 (whose tensor-core local layer already holds it
// to 1e-3 relative L2 rather than bit-exactness) runs the D and W passes as direct
// truncated DFTs on CUDA cores instead of the reference's radix-2 transforms: only
// the kept modes are formed, every output a plain fp32 sum over one line.  The values
// are the same transform's up to fp32 rounding.  True when that path applies.
bool fno3d_direct_dft(int C, int fp8, int Wp, int Dp, int MW, int MD);
// Its tables, correctly rounded from double (floats; MD4 = MD rounded up to 4, MW2 = MW
// rounded up to 2, columns past MD / MW zero):
//   [Dp][MD4] float2  e^{-2 pi i kd d / Dp}
//   [Wp][MW2] float2  e^{-2 pi i kw w / Wp}
//   [MD4][Dp]         cos(2 pi j d / Dp), then [MD4][Dp] sin(2 pi j d / Dp)
std::vector<float> fno3d_dft_tables(int Wp, int Dp, int MW, int MD);

const char* fno3d_unsupported(int C, int Hp, int Wp, int Dp, int MH, int MW, int MD, int out_ch);
cudaError_t fno3d_run(const Fno3dPlan& plan, cudaStream_t stream);

}  // namespace nfx
