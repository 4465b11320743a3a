// nfx_lut.h -- host-built tables that let the GPU epilogues reproduce the reference's
// float activation + quantisation exactly without evaluating them per element.
//
// 1. Code table.  The next layer's input code is
//        code(z) = fq_code(act(z), s, zp)
//    with act the reference GELU (fno.cpp:36-48, glibc tanhf) or ReLU and fq_code the
//    reference float quantiser (fno.cpp:497-505).  code(z) is a step function of the
//    float z = x1 + x2.  The table splits z into uniform cells; each cell stores the
//    code at its (slightly extended) left edge, the code after its breakpoint and at
//    most one breakpoint inside, found exactly by bisection over consecutive float
//    values using the host's reference-equivalent arithmetic.  The GPU evaluates
//        code = z >= t ? hi : lo
//    for the cell of z (index fma(z, inv_delta, -zlo * inv_delta)).  Where float
//    rounding makes code(z) flip back and forth within a few ulps of a breakpoint, the
//    table keeps one breakpoint of that window.
// 2. Activation table.  The projection applies the activation to a fake-quantised
//    value, which takes one of 256 values (k - zp)*s; the table holds the reference
//    activation of each.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

namespace nfx {

struct CodeCell {
    float t;        // breakpoint (+inf when unused)
    int32_t packed; // code below t (byte 0) | code from t on (byte 1)
};

struct CodeLut {
    float zlo = 0.f;        // one-segment tables: index fma(z, inv_delta, -zlo * inv_delta)
    float inv_delta = 0.f;  // (0 for a two-segment table)
    // General index: z < zsplit ? fma(z, inv0, c0) : fma(z, inv1, c1), truncated and
    // clamped to the cells.  One-segment tables have zsplit = -inf and (inv1, c1) equal
    // to the form above; two-segment tables give the sides of the split their own cell
    // size (the negative branch of GELU needs far coarser cells than the positive one).
    float zsplit = 0.f;
    float inv0 = 0.f, c0 = 0.f, inv1 = 0.f, c1 = 0.f;
    // Saturating form of the same index (lut_index_sat): u = sat(fma(z, alpha, beta)),
    // idx = rint(u * nm1), with (alpha, beta) of the segment; nm1 = cells - 1.
    float alpha0 = 0.f, beta0 = 0.f, alpha1 = 0.f, beta1 = 0.f, nm1 = 0.f;
    std::vector<CodeCell> cells;
};

// The saturating index of z (the device's lut_index_sat, evaluated on the host).
int lut_index_sat(float z, const CodeLut& L);

// Reference activation (act 0: GELU tanh form, act 1: ReLU) in float.
float act_ref(float z, int act);
// Reference float quantiser: clamp(round(v / s) + zp) as a float in [-128, 127].
float fq_code_ref(float v, float s, float zp);

// Build the z -> code table for (s, zp, act).  Returns false (with a reason) if no
// table with at most `max_cells` cells and one breakpoint per cell exists (with
// `allow_split`, two segments of different cell sizes are tried after one).
bool build_code_lut(float s, int zp, int act, int max_cells, CodeLut& out, std::string& why,
                    bool allow_split = false);

// act_ref((k - zp) * s) for k = -128..127 (index k + 128).
std::vector<float> build_act_table(float s, int zp, int act);

// 3. FFT twiddles.  The reference radix-2 FFT (fft.cpp:49-69) does not evaluate
//    e^{-+2 pi i k/len}; it starts each butterfly group at w = 1 and updates
//    w *= wlen after every butterfly, with wlen = (cosf(ang), sinf(ang)),
//    ang = (-+2.0f * (float)M_PI) / (float)len, and the product in the fused form
//    the reference build emits (re = fma(wr, lr, -(wi*li)), im = fma(wr, li, wi*lr)).
//    The table holds those rounded values, stage after stage: entry (len/2 - 1 + k)
//    is the w of butterfly k at stage len, for len = 2, 4, ..., n (n - 1 entries,
//    interleaved re, im).
std::vector<float> build_fft_twiddles(int n, bool inverse);

// 4. E4M3 (fp8_e4m3.h:106-334), host side: the reference encoder (with its subnormal
//    clamp), decoder, and the per-tensor fake-quant of a weight tensor.  `xq` receives
//    the decoded E4M3 values, `out` the fake-quantised ones (either may be null).
uint8_t e4m3_encode(float v);
float e4m3_decode(uint8_t b);
void e4m3_fake_quant(const float* in, float scale, float* xq, float* out, size_t n);

}  // namespace nfx
