// fno2d.h -- host/device interface of the FNO2d INT8 executor (fno2d.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "nfx_internal.h"

namespace nfx {

// Arguments of one tcgen05 layer launch (local 1x1 layer or the projection).
struct LayerArgs {
    // GEMM operands: weight codes (C, C), per-channel params
    const int8_t* Wq;
    const float* scale_w;
    const int32_t* zp_w;
    const int32_t* sum_w;
    const float* bias;
    // -2 zp_w split into nz int8 parts, each as a (C rows, 32 columns) K-major block of
    // one repeated value per row: the layer's MMA adds A x Z_p, so the accumulator holds
    // sum_k a_k (w_k - 2 zp_w) and the epilogue needs only a per-column constant
    const int8_t* zrows;  // [3][C][32]
    int8_t* codes_out;    // layer_tc: the (M, C) output codes
    int nz;
    float s_in;       // input activation qparams (the layer-input key)
    int zp_in;
    FqParam fq_out;   // locs.i.output (layer) / proj_q.output (projection)
    FqParam fq_final; // proj_out.output (projection only)
    int act;          // 0 GELU (tanh form), 1 ReLU
    // spectral branch (layer only)
    const float2* Y;      // (B, MH*MW, C) mixed spectrum
    const float2* twi_w;  // (MW, W)  f_kw * e^{+2 pi i kw w / W} / W
    const float2* twi_h;  // (H, MH)  e^{+2 pi i kh h / H} / H
    // z -> next-layer code table (layer; lut_cells == 0: evaluate directly)
    const int2* code_lut;  // CodeCell[lut_cells] {breakpoint, base | d << 8}
    int lut_cells;
    float lut_zlo, lut_inv_delta;
    // two-segment tables (lut_two != 0): cell index z < lut_split ? fma(z, inv0, c0)
    // : fma(z, inv1, c1) (CodeLut in nfx_lut.h)
    int lut_two;
    float lut_split, lut_inv0, lut_c0, lut_inv1, lut_c1;
    // the same index in saturating form (CodeLut::alpha0 .. nm1 in nfx_lut.h)
    float lut_alpha0, lut_beta0, lut_alpha1, lut_beta1, lut_nm1;
    // activation of the 256 fake-quantised proj_q values (projection; nullptr: direct)
    const float* act_table;
    // projection only
    const float* w_out;   // (out_ch, C) proj_out weight (fake-quantised at load)
    const float* b_out;   // (out_ch,)
    int out_ch;
    float* y;             // (M, out_ch)
    // geometry
    int64_t M;
    int H, W;
    unsigned* err;
};

// Arguments of the tensor-core forward transform (spec_fwd_tc_kernel, W == 128).
struct SpecFwdArgs {
    const int8_t* limbs;      // [4][32][128] int8: base-256 digits of the scaled DFT basis
    const long long* sum_b;   // [2*MW] sum over w of the scaled basis (for the zero point)
    const float2* twf_h;      // (H, MH)
    float2* xpart;            // (B, H/HB, MH*MW, C)
    float s;                  // layer-input scale and zero point
    int zp;
    int B, H, HB;
    unsigned* err;
};

// Per-output-channel constants of a local layer's epilogue, passed by value so that
// the kernel reads them through the constant cache (off the shared-memory pipe).  The
// reference's integer (int8_gemm.cpp:574-577, fno.cpp:541-548) is
//   acc - zp_w sum_a - zp_in sum_w + K zp_w zp_in,  acc = sum_k a_k (w_k - zp_w),
// i.e. sum_k a_k (w_k - 2 zp_w) + nk' with nk' = zp_in (K zp_w - sum_w); the MMA
// produces the first term (the Z blocks of LayerArgs), so
//   v = a[o] * float(raw' + nk'[o]) + b[o],  a = scale_w * s_in,
// stored as float4 {a, bits(zp_w), bits(nk'), b}, and again per field (a, nk', b),
// so that one 16-byte constant load brings one field of four columns.
constexpr int kFno2dColMax = 64;
struct LayerCols {
    float4 v[kFno2dColMax];
    float a[kFno2dColMax];
    int nk[kFno2dColMax];
    float b[kFno2dColMax];
};
// The projection's constants: proj_q's epilogue columns as above, and proj_out's
// weights and biases (out_ch <= 4), read as constant-bank operands.
struct ProjCols {
    float4 v[kFno2dColMax];
    float wout[4][kFno2dColMax];
    float bout[4];
};

// The lift's weights (C, in_ch <= 8) and biases, read as constant-bank operands.
constexpr int kFno2dLiftInMax = 8;
struct LiftCols {
    float w[kFno2dColMax][kFno2dLiftInMax];
    float b[kFno2dColMax];
};

// Code-table capacities (cells of 8 bytes in shared memory): the W == 128 layer
// kernel has room for a one-segment table of up to kFno2dLutCellsTc cells; the general
// layer kernel for up to kFno2dLutCells (two segments when one does not fit).
constexpr int kFno2dLutCells = 3072;
constexpr int kFno2dLutCellsTc = 5632;

struct Fno2dLayerPlan {
    float s_in;
    int zp_in;
    const float2* wspec;  // (MH*MW, C, C) complex, [mode][in][out]
    // The same weights as one real (2C x 2C) matrix per mode for the tensor-core
    // contraction, transposed (row n = 2 out + re/im, column k = 2 in + re/im) and split
    // into tf32 high and low parts: (MH*MW*2C, 2C) each; null when C != 64.
    const float* wmix_hi;
    const float* wmix_lo;
    LayerArgs args;
    LayerArgs args_tc;    // the same with the W == 128 kernel's code table
    LayerCols cols;
};

constexpr int kFno2dMaxLayers = 8;

// Everything one forward pass needs (device pointers).
struct Fno2dPlan {
    int B, H, W, C, MH, MW, L, in_ch, HB;
    const float* x;        // (B, H, W, in_ch)
    float* y;              // (B, H, W, out_ch)
    const float* lift_w;   // (C, in_ch)
    const float* lift_b;   // (C,)
    float lift_s;
    int lift_zp;
    float lift_inv_s;
    LiftCols lift_cols;    // the same weights and biases as constant-bank operands
    int8_t* codes[2];      // ping-pong (B*H*W, C)
    float2* xpart;         // (B, H/HB, MH*MW, C)
    float2* Y;             // (B, MH*MW, C)
    const float2* twf_w;   // (MW, W)  e^{-2 pi i kw w / W}
    const int8_t* fwd_limbs;    // tensor-core forward basis (W == 128), see SpecFwdArgs
    const long long* fwd_sum_b;
    const float2* twf_h;   // (H, MH)  e^{-2 pi i kh h / H}
    const float2* twi_w;
    const float2* twi_h;
    Fno2dLayerPlan layer[kFno2dMaxLayers];
    LayerArgs proj;
    ProjCols proj_cols;    // proj_q epilogue and proj_out constants
    unsigned* err;
    KernelTimer* timer;    // nullptr unless profiling is enabled
    // parity taps (nullptr: off): the int8 codes of every layer input -- the lift's
    // output, then each layer's output, the last one being the projection's input --
    // copied as L + 1 consecutive (B*H*W, C) blocks after the kernel that wrote them
    int8_t* tap_codes;
};

// Row blocks per sample of the forward transform's partial spectra (B x this many
// partials of MH*MW*C complex values are written by spec_fwd and summed by spec_mix).
inline int fno2d_row_blocks(int H) { return H < 4 ? H : 4; }

bool fno2d_supported(int C, int MH, int MW);

// The forward transform runs on tensor cores (spec_fwd_tc2_kernel) for W = 128 rows
// with at most 12 kept W-modes, from the basis digits below; elsewhere on CUDA cores.
inline bool fno2d_tc_forward(int W, int MW) { return W == 128 && 2 * MW <= 24; }
constexpr int kFno2dLimbBytes = 4 * 32 * 128;   // [4][32][128] int8 basis digits

// Host-side transform tables of the INT8 executor for an H x W grid (nfx_runtime.cpp):
// fw, iw (MW, W) and fh, ih (H, MH) complex as float pairs (layouts of Fno2dPlan's
// twf_w, twi_w, twf_h, twi_h), and, when fno2d_tc_forward(W, MW) and limbs / sum_b are
// not null, the tensor-core forward basis (SpecFwdArgs::limbs, sum_b [2 MW]).
void fno2d_tables(int H, int W, int MH, int MW, float* fw, float* fh, float* iw, float* ih,
                  int8_t* limbs, long long* sum_b);
cudaError_t fno2d_run(const Fno2dPlan& plan, cudaStream_t stream);

// ---------------------------------------------------------------------------
// FP32 fake-quant executor (fno2d_fp32.cu): the reference FNO2d::Forward
// (fno.cpp:777-995) as the runtime runs it without EnableInt8Gemm.  Activations are
// fp32 channel-first (b, c, h, w) like the reference's h_perm.
//
// The same kernels also run the INT8 composition (EnableInt8Gemm) on geometries the
// width-64 executor above does not take: the layer inputs snapped with the previous
// ".output" qparams, and the 1x1 layers through LinearForwardBatched on int8 codes
// (Fno2dI8Linear).  The snapped activations stay fp32 values (q - zp) * s.
// ---------------------------------------------------------------------------

// One 1x1 layer through LinearForwardBatched (int8_gemm.cpp:530-580) with the
// QuantiseWeight2D codes (fno.cpp:325-358): the input is quantised with (s_in, zp_in),
// acc = sum_k a_k (w_ok - zp_w[o]) is exact in fp32 (|acc| < 2^24 for C <= 256), and
//   y = (scale_w[o] * s_in) * float(acc - zp_w[o] sum_a - zp_in sum_w[o] + C zp_w[o] zp_in)
// then y + 0.0f and + bias[o] as two roundings.
struct Fno2dI8Linear {
    const float* wz;      // (C, C) w_ok - zp_w[o] as floats (nullptr: the FP32 Linear runs)
    const int4* cols;     // per output channel {float bits of scale_w * s_in, zp_w,
                          //  C zp_w zp_in - zp_in sum_w, 0}
    float s_in;
    int zp_in;
};

// Snap of a layer's output for its consumer (apply_input_fq of the INT8 composition):
// kind 1 stores (code - zp) * s, the code from the exact z -> code table when present.
struct Fno2dSnap {
    FqParam fq;
    const int2* code_lut; // one-segment table (nfx_lut.h); nullptr: evaluate directly
    int lut_cells;
    float lut_zlo, lut_inv_delta;
};

struct Fno2dF32Layer {
    const float* wr;      // (C, C, MH, MW) spectral weights (fake-quantised at load)
    const float* wi;
    const float* loc_w;   // (C, C)
    const float* loc_b;
    FqParam fq;           // locs.i.output
    Fno2dI8Linear i8;     // INT8 composition: the local Linear (wz nullptr: FP32)
    Fno2dSnap snap;       // INT8 composition: snap of this layer's output (kind 0: none)
};

struct Fno2dF32Plan {
    int B, H, W, Hp, Wp, C, MH, MW, L, in_ch, out_ch, act;
    const float* x;       // (B, H, W, in_ch)
    float* y;             // (B, H, W, out_ch)
    const float* lift_w;
    const float* lift_b;
    FqParam fq_lift;
    Fno2dF32Layer layer[kFno2dMaxLayers];
    const float* pq_w;
    const float* pq_b;
    FqParam fq_pq;
    const float* po_w;
    const float* po_b;
    FqParam fq_po;
    // INT8 composition: the lift output's snap (layer 0's input), proj_q through
    // LinearForwardBatched, and act(proj_q.output fake-quant) from a 256-entry table
    // (build_act_table; nullptr: evaluated)
    FqParam snap_lift;
    Fno2dI8Linear pq_i8;
    const float* pq_act_table;
    const float2* twf_w;  // recurrence twiddles (nfx_lut.h) for Wp and Hp
    const float2* twi_w;
    const float2* twf_h;
    const float2* twi_h;
    float* h[2];          // (B, C, Hp, Wp)
    float2* Xs;           // (B, C, MH, MW) truncated spectra
    float2* colinv;       // (B, C, Hp, MW) column-inverse transforms
    KernelTimer* timer;
    // Calibration observers (nullptr: off).  Observed tensor i -- 0 lift, 1 + l locs.l,
    // L + 1 proj_q, L + 2 proj_out, the Linear outputs before their fake-quant -- updates
    // obs[i] (ordered-float key of the minimum), obs[kFno2dObsMax + i] (key of the
    // maximum), obs[2 kFno2dObsMax + i] (nonzero after a NaN), and, when obs_vals[i] is
    // set, stores every value at its channel-last element index in obs_vals[i].
    unsigned* obs;
    float* obs_vals[16];
};
constexpr int kFno2dObsMax = 16;

// Geometry limits of the FP32 executor; returns nullptr or the reason it is unsupported.
const char* fno2d_f32_unsupported(int C, int MH, int MW, int Hp, int Wp, int out_ch);
cudaError_t fno2d_f32_run(const Fno2dF32Plan& plan, cudaStream_t stream);

}  // namespace nfx
