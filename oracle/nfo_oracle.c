/*
 * nfo_oracle.c -- CPU restatement of the NeuroFlow reference arithmetic for the
 * quantized neural-operator inference path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA path in
 * neuroflow_b200/csrc.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg may load it.  It is never linked into the product library.
 *
 * Every function below restates one piece of the reference C++ runtime
 * (cpp/src/*.cpp of AITree69/neuroflow) and names the file:line it follows.  The
 * expression shapes are kept identical to the reference so that, compiled with the
 * same compiler and the same flags as the reference build (-O3 -mavx2 -mfma, GCC's
 * default floating-point contraction), the results are bit-identical.  That claim is
 * checked by tests/test_oracle_pin.py against the reference sources compiled from
 * their original location (oracle/Makefile, target `ref`).
 *
 * Two FNO2d modes exist:
 *   mode 0  "fake-quant fp32": the reference FNO2d::Forward (cpp/src/fno.cpp:777-995)
 *           with the runtime's load-time weight fake-quant (cpp/src/fno.cpp:217-290).
 *           Pinned bit-exact against the reference runtime.
 *   mode 1  "int8": the reference has no INT8 GEMM for FNO2d.  This mode applies the
 *           reference FNO1d INT8 convention (cpp/src/fno.cpp:125-159, :360-406,
 *           :475-549) to FNO2d's layer structure: the layer input is snapped with the
 *           previous layer's ".output" qparams, the 1x1 layers (locs.i, proj_q) run
 *           through LinearForwardBatched (cpp/src/int8_gemm.cpp:530-580) with the
 *           per-channel weight codes of QuantiseWeight2D (cpp/src/fno.cpp:325-358),
 *           and the FNO2d output fake-quant boundaries are kept.  Each piece is pinned
 *           separately; the composition has no reference counterpart.
 */
#include <complex.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

#define NFO_MAX_LAYERS 8

/* ------------------------------------------------------------------------- */
/* Quantisation primitives                                                    */
/* ------------------------------------------------------------------------- */

/* int8_gemm.cpp:507-520 QuantiseActivation: q = (int)round(v/s) + zp, clamp. */
void nfo_quantise_activation(const float* A, int8_t* A_q, int64_t n, float scale_A,
                             int32_t zp_A) {
    for (int64_t i = 0; i < n; ++i) {
        int32_t q = (int32_t)(roundf(A[i] / scale_A)) + zp_A;
        if (q < -128) q = -128;
        if (q > 127) q = 127;
        A_q[i] = (int8_t)q;
    }
}

/* fno.cpp:830-842 (and :497-505, :629-640): float fake-quant round trip. */
void nfo_fake_quant(float* data, int64_t numel, float scale, int32_t zero_point) {
    const float zp = (float)zero_point;
    for (int64_t k = 0; k < numel; ++k) {
        float v = data[k];
        float q = roundf(v / scale) + zp;
        if (q < -128.0f) q = -128.0f;
        if (q > 127.0f) q = 127.0f;
        data[k] = (q - zp) * scale;
    }
}

/* fno.cpp:813-828 FNO2d FP8 branch of apply_fake_quant: a log2 snap.  The exponent
 * passed to std::ldexp is a float converted to int (truncation toward zero), which
 * is what the reference computes. */
void nfo_fake_quant_fp8_log2(float* data, int64_t numel, float scale) {
    if (!(scale > 0.0f)) return;
    for (int64_t k = 0; k < numel; ++k) {
        const float v = data[k] / scale;
        const float abs_v = fabsf(v);
        const float sign = v < 0.0f ? -1.0f : 1.0f;
        const float quant_v = (abs_v < 0.015625f)
            ? abs_v
            : ldexpf(1.0f, (int)(roundf(log2f(abs_v) * 8.0f) / 8.0f));
        const float clamped = fminf(quant_v, 448.0f);
        data[k] = sign * clamped * scale;
    }
}

/* fno.cpp:236-241 fake_quant_pt (per element, zp given as float). */
static inline float fake_quant_pt(float v, float s, float zp) {
    float q = roundf(v / s) + zp;
    if (q < -128.0f) q = -128.0f;
    if (q > 127.0f) q = 127.0f;
    return (q - zp) * s;
}

/* fno.cpp:217-290 DequantiseWeight.  Per-channel qparams are applied for 2-D tensors
 * with axis 0 and 3-D tensors with axis 1; any other layout falls through to the
 * per-tensor qparams when those exist.  Returns 1 if the tensor was modified. */
int nfo_dequantise_weight(float* t, const int64_t* shape, int ndim,
                          const float* pc_scales, const int32_t* pc_zps, int64_t pc_n,
                          int pc_axis, int has_pc, float pt_scale, int32_t pt_zp,
                          int has_pt) {
    if (has_pc) {
        if (ndim == 2 && pc_axis == 0) {
            for (int64_t c = 0; c < pc_n; ++c) {
                const float s = pc_scales[c];
                const float zp = (float)pc_zps[c];
                for (int64_t i = 0; i < shape[1]; ++i) {
                    const int64_t off = c * shape[1] + i;
                    t[off] = fake_quant_pt(t[off], s, zp);
                }
            }
            return 1;
        } else if (ndim == 3 && pc_axis == 1) {
            const int64_t in_dim = shape[0], out_dim = shape[1], modes_dim = shape[2];
            for (int64_t i = 0; i < in_dim; ++i)
                for (int64_t c = 0; c < out_dim; ++c) {
                    const float s = pc_scales[c];
                    const float zp = (float)pc_zps[c];
                    for (int64_t k = 0; k < modes_dim; ++k) {
                        const int64_t off = i * (out_dim * modes_dim) + c * modes_dim + k;
                        t[off] = fake_quant_pt(t[off], s, zp);
                    }
                }
            return 1;
        }
    }
    if (has_pt) {
        const float s = pt_scale;
        const float zp = (float)pt_zp;
        int64_t numel = 1;
        for (int d = 0; d < ndim; ++d) numel *= shape[d];
        for (int64_t i = 0; i < numel; ++i) t[i] = fake_quant_pt(t[i], s, zp);
        return 1;
    }
    return 0;
}

/* fno.cpp:325-358 QuantiseWeight2D: per-output-row codes and the cached
 * sum_W_per_row[o] = sum_i (W_q[o,i] - zp[o]). */
void nfo_quantise_weight_2d(const float* W, int n_out, int k, const float* scales,
                            const int32_t* zps, int8_t* W_q, int32_t* sum_w) {
    for (int64_t c = 0; c < n_out; ++c) {
        const float s = scales[c];
        const float zp = (float)zps[c];
        int32_t row_sum = 0;
        for (int64_t i = 0; i < k; ++i) {
            const int64_t off = c * k + i;
            float q = roundf(W[off] / s) + zp;
            if (q < -128.0f) q = -128.0f;
            if (q > 127.0f) q = 127.0f;
            const int8_t q8 = (int8_t)q;
            W_q[off] = q8;
            row_sum += (int32_t)q8 - zps[c];
        }
        sum_w[c] = row_sum;
    }
}

/* int8_gemm.cpp:479-496 PrecomputeSumW. */
void nfo_precompute_sum_w(const int8_t* W_q, const int32_t* zp_w, int in_f, int out_f,
                          int32_t* out) {
    for (int o = 0; o < out_f; ++o) {
        int32_t acc = 0;
        const int8_t* w_row = W_q + (int64_t)o * in_f;
        for (int i = 0; i < in_f; ++i) acc += (int32_t)w_row[i] - zp_w[o];
        out[o] = acc;
    }
}

/* int8_gemm.cpp:530-580 LinearForwardBatched: bulk quantise, per-row Sum a, scalar
 * int32 GEMM with acc = sum a*(w - zp_w), and the reference epilogue
 *   y = sW*sA*float(acc - zp_w*sum_a - zp_A*sum_w + (int64)K*zp_w*zp_A)
 * followed by y + (bias or 0).  The optional acc_out / codes_out taps expose the
 * int32 accumulator and the int8 activation codes for bit-exact checks. */
void nfo_linear_forward_batched(const int8_t* W_q, const float* scale_W,
                                const int32_t* zp_W, const int32_t* sum_W,
                                const float* bias, int in_f, int out_f, float scale_A,
                                int32_t zp_A, int bsz, const float* A, float* C,
                                int32_t* acc_out, int8_t* codes_out) {
    if (bsz <= 0) return;
    int8_t* A_q = codes_out ? codes_out : (int8_t*)malloc((size_t)bsz * in_f);
    nfo_quantise_activation(A, A_q, (int64_t)bsz * in_f, scale_A, zp_A);
    for (int r = 0; r < bsz; ++r) {
        const int8_t* a_row = A_q + (int64_t)r * in_f;
        int32_t sum_a = 0;
        for (int i = 0; i < in_f; ++i) sum_a += a_row[i];
        float* c_row = C + (int64_t)r * out_f;
        for (int o = 0; o < out_f; ++o) {
            const int8_t* w_row = W_q + (int64_t)o * in_f;
            const int32_t zp_w_o = zp_W[o];
            int32_t acc = 0;
            for (int i = 0; i < in_f; ++i)
                acc += (int32_t)a_row[i] * ((int32_t)w_row[i] - zp_w_o);
            if (acc_out) acc_out[(int64_t)r * out_f + o] = acc;
            const int32_t sum_w = sum_W ? sum_W[o] : 0;
            const float y = scale_W[o] * scale_A *
                (float)(acc - zp_w_o * sum_a - zp_A * sum_w + (int64_t)in_f * zp_w_o * zp_A);
            c_row[o] = y + (bias ? bias[o] : 0.0f);
        }
    }
    if (!codes_out) free(A_q);
}

/* fno.cpp:36-48 ApplyActivation: GELU (tanh approximation) or ReLU. */
void nfo_apply_activation(float* data, int64_t n, int relu) {
    if (relu) {
        for (int64_t i = 0; i < n; ++i)
            if (data[i] < 0.0f) data[i] = 0.0f;
    } else {
        /* the reference build contracts z + 0.044715f*z*z*z into one fma */
        const float c = sqrtf(2.0f / (float)M_PI);
        for (int64_t i = 0; i < n; ++i) {
            float z = data[i];
            const float inner = fmaf(0.044715f * z * z, z, z);
            data[i] = 0.5f * z * (1.0f + tanhf(c * inner));
        }
    }
}

/* Per-token INT8 GEMM used by the standalone GEMM sweep: activation codes with one
 * (scale, zero point) per row, per-channel weight codes, and the reference epilogue
 * of int8_gemm.cpp:574-577 evaluated with the row's own (scale_A, zp_A); then
 * bias (fno.cpp:541-548 adds it as a separate float add) and optional GELU
 * (fno.cpp:36-48).  The per-row form has no reference entry point; its arithmetic is
 * the reference formula with scale_A/zp_A indexed by row. */
void nfo_int8_gemm_rows(const int8_t* A_q, const float* scale_A, const int32_t* zp_A,
                        int M, int K, const int8_t* W_q, const float* scale_W,
                        const int32_t* zp_W, const int32_t* sum_W, int N,
                        const float* bias, int gelu, float* C, int32_t* acc_out) {
    const float c = sqrtf(2.0f / (float)M_PI);
    for (int64_t r = 0; r < M; ++r) {
        const int8_t* a_row = A_q + r * K;
        int32_t sum_a = 0;
        for (int i = 0; i < K; ++i) sum_a += a_row[i];
        const float sA = scale_A[r];
        const int32_t zA = zp_A[r];
        for (int o = 0; o < N; ++o) {
            const int8_t* w_row = W_q + (int64_t)o * K;
            const int32_t zp_w_o = zp_W[o];
            int32_t acc = 0;
            for (int i = 0; i < K; ++i) acc += (int32_t)a_row[i] * ((int32_t)w_row[i] - zp_w_o);
            if (acc_out) acc_out[r * N + o] = acc;
            const float y = scale_W[o] * sA *
                (float)(acc - zp_w_o * sum_a - zA * sum_W[o] + (int64_t)K * zp_w_o * zA);
            float out = y + 0.0f;
            if (bias) out = out + bias[o];
            if (gelu) {
                float z = out;
                out = 0.5f * z * (1.0f + tanhf(c * fmaf(0.044715f * z * z, z, z)));
            }
            C[r * N + o] = out;
        }
    }
}

/* fno.cpp:51-80 Linear, the hand-rolled loop (the reference is built without Eigen).
 * The reference build (GCC -O3, cpp/CMakeLists.txt:78 flags with AVX-512) vectorises
 * the dot product as 16-wide blocks of products that are then added to the
 * accumulator one by one in order (unfused), one 8-wide block when at least 8 terms
 * remain, and a scalar tail of fused multiply-adds for the last k mod 8 terms.  The
 * sum order is the plain sequential one throughout; only the fusion changes. */
int nfo_linear_unfused_len(int k) {
    const int a = (k / 16) * 16;
    return (k - a >= 8) ? a + 8 : a;
}

void nfo_linear(const float* x, const float* W, const float* b, int bsz, int k, int n,
                float* y) {
    for (int i = 0; i < bsz; ++i) {
        const float* xi = x + (int64_t)i * k;
        float* yi = y + (int64_t)i * n;
        for (int j = 0; j < n; ++j) {
            float acc = b ? b[j] : 0.0f;
            const float* wj = W + (int64_t)j * k;
            const int vec = nfo_linear_unfused_len(k);
            int p = 0;
            for (; p < vec; ++p) acc = acc + xi[p] * wj[p];
            for (; p < k; ++p) acc = fmaf(xi[p], wj[p], acc);
            yi[j] = acc;
        }
    }
}

/* ------------------------------------------------------------------------- */
/* FFT: radix-2 Cooley-Tukey with the twiddle recurrence w *= wlen             */
/* ------------------------------------------------------------------------- */

/* fft.cpp:36-46 bit reversal. */
static void bit_reverse(float complex* a, int n) {
    int j = 0;
    for (int i = 1; i < n; ++i) {
        int bit = n >> 1;
        for (; j & bit; bit >>= 1) j ^= bit;
        j ^= bit;
        if (i < j) {
            float complex t = a[i];
            a[i] = a[j];
            a[j] = t;
        }
    }
}

/* Complex products as the reference build evaluates them.  With -O3 -mavx2 -mfma
 * (with or without the -mavx512* flags) GCC emits two code paths for
 * ComplexFftInPlace (fft.cpp:49-69):
 *   forward butterfly  v = a*w : packed multiplies + addsub, no fusion
 *                                re = ar*wr - ai*wi,  im = ai*wr + ar*wi
 *   inverse butterfly  v = a*w : re = fma(ar, wr, -(ai*wi)),  im = fma(ar, wi, ai*wr)
 *   twiddle update  w *= wlen  : same fused form as the inverse butterfly.
 * The helpers below spell those forms out so that the restatement does not depend
 * on the C compiler's own contraction choices. */
__attribute__((optimize("fp-contract=off")))
static float complex cmul_plain(float complex a, float complex b) {
    const float ar = crealf(a), ai = cimagf(a), br = crealf(b), bi = cimagf(b);
    const float p0 = ar * br, p1 = ai * bi, p2 = ai * br, p3 = ar * bi;
    return CMPLXF(p0 - p1, p2 + p3);
}

__attribute__((optimize("fp-contract=off")))
static float complex cmul_fused(float complex a, float complex b) {
    const float ar = crealf(a), ai = cimagf(a), br = crealf(b), bi = cimagf(b);
    const float p1 = ai * bi, p2 = ai * br;
    return CMPLXF(fmaf(ar, br, -p1), fmaf(ar, bi, p2));
}

/* fft.cpp:49-69 in-place complex FFT; the inverse scales by 1/n. */
static void complex_fft(float complex* a, int n, int inverse) {
    bit_reverse(a, n);
    for (int len = 2; len <= n; len <<= 1) {
        const float ang = (inverse ? 2.0f : -2.0f) * (float)M_PI / (float)len;
        const float complex wlen = CMPLXF(cosf(ang), sinf(ang));
        for (int i = 0; i < n; i += len) {
            float complex w = CMPLXF(1.0f, 0.0f);
            for (int k = 0; k < len / 2; ++k) {
                float complex u = a[i + k];
                float complex v = inverse ? cmul_fused(a[i + k + len / 2], w)
                                          : cmul_plain(a[i + k + len / 2], w);
                a[i + k] = u + v;
                a[i + k + len / 2] = u - v;
                w = cmul_fused(w, wlen);
            }
        }
    }
    if (inverse) {
        const float inv = 1.0f / (float)n;
        for (int i = 0; i < n; ++i) a[i] *= inv;
    }
}

/* fft.cpp:73-84 Rfft: out has n/2+1 interleaved complex values. */
void nfo_rfft(const float* x, int n, float* out_complex) {
    float complex* buf = (float complex*)malloc(sizeof(float complex) * n);
    for (int i = 0; i < n; ++i) buf[i] = CMPLXF(x[i], 0.0f);
    complex_fft(buf, n, 0);
    const int half = n / 2 + 1;
    for (int i = 0; i < half; ++i) {
        out_complex[2 * i] = crealf(buf[i]);
        out_complex[2 * i + 1] = cimagf(buf[i]);
    }
    free(buf);
}

/* fft.cpp:86-99 Irfft: mirror conjugates of bins 1..n/2-1, complex inverse, real part. */
void nfo_irfft(const float* x_complex, int n, float* out) {
    float complex* buf = (float complex*)malloc(sizeof(float complex) * n);
    const int half = n / 2 + 1;
    for (int i = 0; i < half; ++i) buf[i] = CMPLXF(x_complex[2 * i], x_complex[2 * i + 1]);
    for (int i = 1; i < n - half + 1; ++i) buf[n - i] = conjf(buf[i]);
    complex_fft(buf, n, 1);
    for (int i = 0; i < n; ++i) out[i] = crealf(buf[i]);
    free(buf);
}

/* fft.cpp:101-124 Rfft2: row rfft, then column complex FFT over the W/2+1 columns. */
void nfo_rfft2(const float* x, int H, int W, float* out_complex) {
    const int half_w = W / 2 + 1;
    float complex* scratch = (float complex*)malloc(sizeof(float complex) * (size_t)H * half_w);
    for (int i = 0; i < H; ++i)
        nfo_rfft(x + (int64_t)i * W, W, (float*)(scratch + (int64_t)i * half_w));
    float complex* col = (float complex*)malloc(sizeof(float complex) * H);
    for (int j = 0; j < half_w; ++j) {
        for (int i = 0; i < H; ++i) col[i] = scratch[(int64_t)i * half_w + j];
        complex_fft(col, H, 0);
        for (int i = 0; i < H; ++i) {
            out_complex[((int64_t)i * half_w + j) * 2] = crealf(col[i]);
            out_complex[((int64_t)i * half_w + j) * 2 + 1] = cimagf(col[i]);
        }
    }
    free(col);
    free(scratch);
}

/* fft.cpp:126-149 Irfft2: column inverse complex FFT, then row irfft. */
void nfo_irfft2(const float* x_complex, int H, int W, float* out) {
    const int half_w = W / 2 + 1;
    float complex* col = (float complex*)malloc(sizeof(float complex) * H);
    float complex* scratch = (float complex*)malloc(sizeof(float complex) * (size_t)H * half_w);
    for (int j = 0; j < half_w; ++j) {
        for (int i = 0; i < H; ++i)
            col[i] = CMPLXF(x_complex[((int64_t)i * half_w + j) * 2],
                            x_complex[((int64_t)i * half_w + j) * 2 + 1]);
        complex_fft(col, H, 1);
        for (int i = 0; i < H; ++i) scratch[(int64_t)i * half_w + j] = col[i];
    }
    for (int i = 0; i < H; ++i)
        nfo_irfft((const float*)(scratch + (int64_t)i * half_w), W, out + (int64_t)i * W);
    free(scratch);
    free(col);
}

/* fft.cpp:151-194 Rfft3: D-axis rfft, W-axis cfft, H-axis cfft. */
void nfo_rfft3(const float* x, int H, int W, int D, float* out_complex) {
    const int half_d = D / 2 + 1;
    const size_t tot = (size_t)H * W * half_d;
    float complex* scratch = (float complex*)malloc(sizeof(float complex) * tot);
    for (int i = 0; i < H; ++i)
        for (int j = 0; j < W; ++j)
            nfo_rfft(x + ((int64_t)i * W + j) * D, D,
                     (float*)(scratch + ((int64_t)i * W + j) * half_d));
    float complex* col_w = (float complex*)malloc(sizeof(float complex) * W);
    for (int i = 0; i < H; ++i)
        for (int k = 0; k < half_d; ++k) {
            for (int j = 0; j < W; ++j) col_w[j] = scratch[((int64_t)i * W + j) * half_d + k];
            complex_fft(col_w, W, 0);
            for (int j = 0; j < W; ++j) scratch[((int64_t)i * W + j) * half_d + k] = col_w[j];
        }
    float complex* col_h = (float complex*)malloc(sizeof(float complex) * H);
    for (int j = 0; j < W; ++j)
        for (int k = 0; k < half_d; ++k) {
            for (int i = 0; i < H; ++i) col_h[i] = scratch[((int64_t)i * W + j) * half_d + k];
            complex_fft(col_h, H, 0);
            for (int i = 0; i < H; ++i) {
                out_complex[(((int64_t)i * W + j) * half_d + k) * 2] = crealf(col_h[i]);
                out_complex[(((int64_t)i * W + j) * half_d + k) * 2 + 1] = cimagf(col_h[i]);
            }
        }
    free(col_h);
    free(col_w);
    free(scratch);
}

/* fft.cpp:196-243 Irfft3: H-axis inverse, W-axis inverse, D-axis irfft. */
void nfo_irfft3(const float* x_complex, int H, int W, int D, float* out) {
    const int half_d = D / 2 + 1;
    const size_t tot = (size_t)H * W * half_d;
    float complex* col_h = (float complex*)malloc(sizeof(float complex) * H);
    float complex* scratch = (float complex*)malloc(sizeof(float complex) * tot);
    for (int j = 0; j < W; ++j)
        for (int k = 0; k < half_d; ++k) {
            for (int i = 0; i < H; ++i)
                col_h[i] = CMPLXF(x_complex[(((int64_t)i * W + j) * half_d + k) * 2],
                                  x_complex[(((int64_t)i * W + j) * half_d + k) * 2 + 1]);
            complex_fft(col_h, H, 1);
            for (int i = 0; i < H; ++i) scratch[((int64_t)i * W + j) * half_d + k] = col_h[i];
        }
    float complex* col_w = (float complex*)malloc(sizeof(float complex) * W);
    for (int i = 0; i < H; ++i)
        for (int k = 0; k < half_d; ++k) {
            for (int j = 0; j < W; ++j) col_w[j] = scratch[((int64_t)i * W + j) * half_d + k];
            complex_fft(col_w, W, 1);
            for (int j = 0; j < W; ++j) scratch[((int64_t)i * W + j) * half_d + k] = col_w[j];
        }
    for (int i = 0; i < H; ++i)
        for (int j = 0; j < W; ++j)
            nfo_irfft((const float*)(scratch + ((int64_t)i * W + j) * half_d), D,
                      out + ((int64_t)i * W + j) * D);
    free(col_w);
    free(scratch);
    free(col_h);
}

/* ------------------------------------------------------------------------- */
/* Spectral convolutions                                                      */
/* ------------------------------------------------------------------------- */

/* fno.cpp:164-207 SpectralConv1d on h (b, w, n). */
void nfo_spectral_conv1d(const float* h, int bsz, int w, int n, int modes,
                         const float* w_real, const float* w_imag, float* out) {
    const int half = n / 2 + 1;
    float* Hs = (float*)malloc(sizeof(float) * (size_t)w * half * 2);
    float* Out_ft = (float*)malloc(sizeof(float) * (size_t)w * half * 2);
    float* time_scratch = (float*)malloc(sizeof(float) * n);
    for (int bi = 0; bi < bsz; ++bi) {
        memset(Out_ft, 0, sizeof(float) * (size_t)w * half * 2);
        for (int wi = 0; wi < w; ++wi)
            nfo_rfft(h + (int64_t)bi * w * n + (int64_t)wi * n, n, Hs + (int64_t)wi * half * 2);
        for (int mi = 0; mi < modes; ++mi)
            for (int wo = 0; wo < w; ++wo) {
                float sum_re = 0.0f, sum_im = 0.0f;
                for (int wi2 = 0; wi2 < w; ++wi2) {
                    float hr = Hs[wi2 * half * 2 + 2 * mi];
                    float hi = Hs[wi2 * half * 2 + 2 * mi + 1];
                    float wr = w_real[((wi2 * w) + wo) * modes + mi];
                    float wi3 = w_imag[((wi2 * w) + wo) * modes + mi];
                    sum_re = sum_re + fmaf(hr, wr, -(hi * wi3));
                    sum_im = sum_im + fmaf(hr, wi3, hi * wr);
                }
                Out_ft[wo * half * 2 + 2 * mi] = sum_re;
                Out_ft[wo * half * 2 + 2 * mi + 1] = sum_im;
            }
        for (int wo = 0; wo < w; ++wo) {
            nfo_irfft(Out_ft + (int64_t)wo * half * 2, n, time_scratch);
            memcpy(out + (int64_t)bi * w * n + (int64_t)wo * n, time_scratch, sizeof(float) * n);
        }
    }
    free(time_scratch);
    free(Out_ft);
    free(Hs);
}

/* fno.cpp:717-771 SpectralConv2d on h (b, w, H, W). */
void nfo_spectral_conv2d(const float* h, int bsz, int w, int H, int W, int modes_h,
                         int modes_w, const float* w_real, const float* w_imag, float* out) {
    const int half_w = W / 2 + 1;
    const size_t spec = (size_t)w * H * half_w * 2;
    float* H_spec = (float*)malloc(sizeof(float) * spec);
    float* Out_ft = (float*)malloc(sizeof(float) * spec);
    for (int bi = 0; bi < bsz; ++bi) {
        memset(Out_ft, 0, sizeof(float) * spec);
        for (int wi = 0; wi < w; ++wi)
            nfo_rfft2(h + ((int64_t)bi * w + wi) * H * W, H, W,
                      H_spec + ((int64_t)wi * H) * half_w * 2);
        for (int mi = 0; mi < modes_h; ++mi)
            for (int mj = 0; mj < modes_w; ++mj)
                for (int wo = 0; wo < w; ++wo) {
                    float sum_re = 0.0f, sum_im = 0.0f;
                    for (int wi = 0; wi < w; ++wi) {
                        const float* H_wi = H_spec + (((int64_t)wi * H + mi) * half_w + mj) * 2;
                        float hr = H_wi[0];
                        float hi = H_wi[1];
                        const float* w_wi =
                            w_real + ((((int64_t)wi * w) + wo) * modes_h + mi) * modes_w + mj;
                        const float* wi_wi =
                            w_imag + ((((int64_t)wi * w) + wo) * modes_h + mi) * modes_w + mj;
                        float wr = w_wi[0];
                        float wii = wi_wi[0];
                        sum_re = sum_re + fmaf(hr, wr, -(hi * wii));
                        sum_im = sum_im + fmaf(hr, wii, hi * wr);
                    }
                    float* Out_wo = Out_ft + (((int64_t)wo * H + mi) * half_w + mj) * 2;
                    Out_wo[0] = sum_re;
                    Out_wo[1] = sum_im;
                }
        for (int wo = 0; wo < w; ++wo)
            nfo_irfft2(Out_ft + (int64_t)wo * H * half_w * 2, H, W,
                       out + (((int64_t)bi * w + wo) * H) * W);
    }
    free(Out_ft);
    free(H_spec);
}

/* ------------------------------------------------------------------------- */
/* FNO2d forward                                                              */
/* ------------------------------------------------------------------------- */

/* Weight qparams attached to one weight tensor (per-channel and/or per-tensor). */
typedef struct {
    const float* pc_scales;
    const int32_t* pc_zps;
    int64_t pc_n;
    int32_t pc_axis;
    int32_t has_pc;
    float pt_scale;
    int32_t pt_zp;
    int32_t has_pt;
} nfo_wq;

/* Activation qparams for one ".output" key: INT8 per-tensor and/or FP8 scale. */
typedef struct {
    float scale;
    int32_t zp;
    int32_t has;
    float fp8_scale;
    int32_t has_fp8;
} nfo_aq;

typedef struct {
    int32_t in_ch, out_ch, width, modes_h, modes_w, n_layers, pad_factor, relu;
    int32_t quant_enabled;
    const float* lift_w;
    const float* lift_b;
    const float* proj_q_w;
    const float* proj_q_b;
    const float* proj_out_w;
    const float* proj_out_b;
    const float* spec_wr[NFO_MAX_LAYERS];
    const float* spec_wi[NFO_MAX_LAYERS];
    const float* loc_w[NFO_MAX_LAYERS];
    const float* loc_b[NFO_MAX_LAYERS];
    nfo_wq q_lift_w, q_lift_b, q_proj_q_w, q_proj_q_b, q_proj_out_w, q_proj_out_b;
    nfo_wq q_spec_wr[NFO_MAX_LAYERS];
    nfo_wq q_spec_wi[NFO_MAX_LAYERS];
    nfo_wq q_loc_w[NFO_MAX_LAYERS];
    nfo_wq q_loc_b[NFO_MAX_LAYERS];
    nfo_aq a_lift, a_proj_q, a_proj_out;
    nfo_aq a_locs[NFO_MAX_LAYERS];
} nfo_fno2d;

static float* dup_floats(const float* src, int64_t n) {
    float* d = (float*)malloc(sizeof(float) * (size_t)(n > 0 ? n : 1));
    memcpy(d, src, sizeof(float) * (size_t)n);
    return d;
}

static void dq_weight(float* t, int64_t d0, int64_t d1, int64_t d2, int64_t d3, int ndim,
                      const nfo_wq* q) {
    int64_t shape[4] = {d0, d1, d2, d3};
    nfo_dequantise_weight(t, shape, ndim, q->pc_scales, q->pc_zps, q->pc_n, q->pc_axis,
                          q->has_pc, q->pt_scale, q->pt_zp, q->has_pt);
}

/* fno.cpp:810-844 apply_fake_quant: FP8 log2 snap takes precedence over INT8. */
static void apply_fq(float* data, int64_t numel, const nfo_aq* a, int quant_enabled) {
    if (!quant_enabled) return;
    if (a->has_fp8) {
        nfo_fake_quant_fp8_log2(data, numel, a->fp8_scale);
    } else if (a->has) {
        nfo_fake_quant(data, numel, a->scale, a->zp);
    }
}

/* The layer-input snap of the FNO1d INT8 convention (fno.cpp:475-508): INT8
 * per-tensor only (the FP8 table is not consulted for the input snap). */
static void apply_input_fq(float* data, int64_t numel, const nfo_aq* a, int quant_enabled) {
    if (quant_enabled && a->has) nfo_fake_quant(data, numel, a->scale, a->zp);
}

/* Optional per-layer taps for layer-wise parity checks (may be NULL):
 * codes_in[i]  : int8 codes of the layer-i input (channel-last), int8 mode only
 * x1_out[i]    : spectral branch output, channel-first (b, w, H, W)
 * h_out[i]     : layer-i output after the activation, channel-last (b, H, W, w)
 * Linear outputs before their fake-quant -- what calibrate()'s hooks observe
 * (neuroflow/quant/static_quant.py:656-668): lift_out (b, H, W, w), x2_out[i] the
 * local Linear of layer i (b, Hp, Wp, w), q_out proj_q (b, H, W, w); proj_out's is y. */
typedef struct {
    int8_t* codes_in[NFO_MAX_LAYERS + 1];
    float* x1_out[NFO_MAX_LAYERS];
    float* h_out[NFO_MAX_LAYERS];
    float* lift_out;
    float* x2_out[NFO_MAX_LAYERS];
    float* q_out;
} nfo_taps;

/* mode 0: fno.cpp:777-995 with the Create-time weight fake-quant (fno.cpp:997-1020).
 * mode 1: the INT8 composition described in the file header.
 * x (b, H, W, in_ch) -> y (b, H, W, out_ch).  Returns 0, or a StatusCode value on
 * a rejected shape (tensor.h:31-37). */
int nfo_fno2d_forward(const nfo_fno2d* m, int mode, const float* x, int bsz, int H0,
                      int W0, float* y, nfo_taps* taps) {
    const int w = m->width, mh = m->modes_h, mw = m->modes_w, L = m->n_layers;
    const int in_ch = m->in_ch, out_ch = m->out_ch;
    if (L > NFO_MAX_LAYERS) return 1;
    if (H0 <= 0 || W0 <= 0 || (H0 & (H0 - 1)) || (W0 & (W0 - 1))) return 1;

    /* Create-time weight copies + fake-quant (fno.cpp:997-1020). */
    float* lift_w = dup_floats(m->lift_w, (int64_t)w * in_ch);
    float* lift_b = dup_floats(m->lift_b, w);
    float* pq_w = dup_floats(m->proj_q_w, (int64_t)w * w);
    float* pq_b = dup_floats(m->proj_q_b, w);
    float* po_w = dup_floats(m->proj_out_w, (int64_t)out_ch * w);
    float* po_b = dup_floats(m->proj_out_b, out_ch);
    float* swr[NFO_MAX_LAYERS];
    float* swi[NFO_MAX_LAYERS];
    float* lw[NFO_MAX_LAYERS];
    float* lb[NFO_MAX_LAYERS];
    const int64_t nspec = (int64_t)w * w * mh * mw;
    for (int i = 0; i < L; ++i) {
        swr[i] = dup_floats(m->spec_wr[i], nspec);
        swi[i] = dup_floats(m->spec_wi[i], nspec);
        lw[i] = dup_floats(m->loc_w[i], (int64_t)w * w);
        lb[i] = dup_floats(m->loc_b[i], w);
    }
    if (m->quant_enabled) {
        dq_weight(lift_w, w, in_ch, 0, 0, 2, &m->q_lift_w);
        dq_weight(lift_b, w, 0, 0, 0, 1, &m->q_lift_b);
        dq_weight(pq_w, w, w, 0, 0, 2, &m->q_proj_q_w);
        dq_weight(pq_b, w, 0, 0, 0, 1, &m->q_proj_q_b);
        dq_weight(po_w, out_ch, w, 0, 0, 2, &m->q_proj_out_w);
        dq_weight(po_b, out_ch, 0, 0, 0, 1, &m->q_proj_out_b);
        for (int i = 0; i < L; ++i) {
            dq_weight(swr[i], w, w, mh, mw, 4, &m->q_spec_wr[i]);
            dq_weight(swi[i], w, w, mh, mw, 4, &m->q_spec_wi[i]);
            dq_weight(lw[i], w, w, 0, 0, 2, &m->q_loc_w[i]);
            dq_weight(lb[i], w, 0, 0, 0, 1, &m->q_loc_b[i]);
        }
    }

    /* INT8 caches (fno.cpp:325-406 applied to locs.i and proj_q). */
    int8_t* lq[NFO_MAX_LAYERS + 1];
    int32_t* lsum[NFO_MAX_LAYERS + 1];
    int use_int8[NFO_MAX_LAYERS + 1];
    for (int i = 0; i <= L; ++i) {
        const nfo_wq* q = (i < L) ? &m->q_loc_w[i] : &m->q_proj_q_w;
        const float* W = (i < L) ? lw[i] : pq_w;
        const nfo_aq* a_in = (i == 0) ? &m->a_lift : &m->a_locs[i - 1];
        use_int8[i] = (mode == 1) && q->has_pc && q->pc_axis == 0 && a_in->has &&
                      m->quant_enabled;
        lq[i] = NULL;
        lsum[i] = NULL;
        if (use_int8[i]) {
            lq[i] = (int8_t*)malloc((size_t)w * w);
            lsum[i] = (int32_t*)malloc(sizeof(int32_t) * w);
            nfo_quantise_weight_2d(W, w, w, q->pc_scales, q->pc_zps, lq[i], lsum[i]);
        }
    }

    int64_t H = H0, W = W0;
    const int64_t P = H * W;
    const int64_t M = (int64_t)bsz * P;

    float* h = (float*)calloc((size_t)(M * w), sizeof(float));        /* (b,H,W,w) */
    nfo_linear(x, lift_w, lift_b, (int)M, in_ch, w, h);
    if (taps && taps->lift_out) memcpy(taps->lift_out, h, sizeof(float) * M * w);
    apply_fq(h, M * w, &m->a_lift, m->quant_enabled);

    float* h_perm = (float*)calloc((size_t)(M * w), sizeof(float));   /* (b,w,H,W) */
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int wi = 0; wi < w; ++wi)
            for (int64_t hi = 0; hi < H; ++hi)
                for (int64_t wj = 0; wj < W; ++wj)
                    h_perm[((bi * w + wi) * H + hi) * W + wj] = h[((bi * H + hi) * W + wj) * w + wi];

    /* fno.cpp:867-892 padding */
    int64_t pad_h = 0, pad_w = 0;
    if (m->pad_factor > 1) {
        const int pf = m->pad_factor;
        pad_h = (pf - (H % pf)) % pf;
        pad_w = (pf - (W % pf)) % pf;
        if (pad_h > 0 || pad_w > 0) {
            const int64_t Hp = H + pad_h, Wp = W + pad_w;
            float* padded = (float*)calloc((size_t)(bsz * w * Hp * Wp), sizeof(float));
            for (int64_t bi = 0; bi < bsz; ++bi)
                for (int wi = 0; wi < w; ++wi)
                    for (int64_t hi = 0; hi < H; ++hi)
                        memcpy(padded + ((bi * w + wi) * Hp + hi) * Wp,
                               h_perm + ((bi * w + wi) * H + hi) * W, sizeof(float) * W);
            free(h_perm);
            h_perm = padded;
            H += pad_h;
            W += pad_w;
        }
    }
    const int64_t Mp = (int64_t)bsz * H * W;
    float* x1 = (float*)calloc((size_t)(Mp * w), sizeof(float));
    float* x2 = (float*)calloc((size_t)(Mp * w), sizeof(float));
    float* pin = (float*)calloc((size_t)(Mp * w), sizeof(float));
    float* pout = (float*)calloc((size_t)(Mp * w), sizeof(float));
    float* add = (float*)calloc((size_t)(Mp * w), sizeof(float));

    for (int i = 0; i < L; ++i) {
        const nfo_aq* a_in = (i == 0) ? &m->a_lift : &m->a_locs[i - 1];
        if (mode == 1) apply_input_fq(h_perm, Mp * w, a_in, m->quant_enabled);
        nfo_spectral_conv2d(h_perm, bsz, w, (int)H, (int)W, mh, mw, swr[i], swi[i], x1);
        if (taps && taps->x1_out[i]) memcpy(taps->x1_out[i], x1, sizeof(float) * Mp * w);
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int64_t hi = 0; hi < H; ++hi)
                for (int64_t wj = 0; wj < W; ++wj)
                    for (int wi = 0; wi < w; ++wi)
                        pin[((bi * H + hi) * W + wj) * w + wi] = h_perm[((bi * w + wi) * H + hi) * W + wj];
        if (use_int8[i]) {
            nfo_linear_forward_batched(lq[i], m->q_loc_w[i].pc_scales, m->q_loc_w[i].pc_zps,
                                       lsum[i], NULL, w, w, a_in->scale, a_in->zp, (int)Mp, pin,
                                       pout, NULL, taps ? taps->codes_in[i] : NULL);
            for (int64_t r = 0; r < Mp; ++r)
                for (int j = 0; j < w; ++j) pout[r * w + j] += lb[i][j];
        } else {
            nfo_linear(pin, lw[i], lb[i], (int)Mp, w, w, pout);
        }
        if (taps && taps->x2_out[i]) memcpy(taps->x2_out[i], pout, sizeof(float) * Mp * w);
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int wi = 0; wi < w; ++wi)
                for (int64_t hi = 0; hi < H; ++hi)
                    for (int64_t wj = 0; wj < W; ++wj)
                        x2[((bi * w + wi) * H + hi) * W + wj] = pout[((bi * H + hi) * W + wj) * w + wi];
        apply_fq(x2, Mp * w, &m->a_locs[i], m->quant_enabled);
        for (int64_t k = 0; k < Mp * w; ++k) add[k] = x1[k] + x2[k];
        nfo_apply_activation(add, Mp * w, m->relu);
        memcpy(h_perm, add, sizeof(float) * Mp * w);
        if (taps && taps->h_out[i]) {
            for (int64_t bi = 0; bi < bsz; ++bi)
                for (int64_t hi = 0; hi < H; ++hi)
                    for (int64_t wj = 0; wj < W; ++wj)
                        for (int wi = 0; wi < w; ++wi)
                            taps->h_out[i][((bi * H + hi) * W + wj) * w + wi] =
                                h_perm[((bi * w + wi) * H + hi) * W + wj];
        }
    }

    if (pad_h > 0 || pad_w > 0) {
        const int64_t oh = H - pad_h, ow = W - pad_w;
        float* trimmed = (float*)calloc((size_t)(bsz * w * oh * ow), sizeof(float));
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int wi = 0; wi < w; ++wi)
                for (int64_t hi = 0; hi < oh; ++hi)
                    memcpy(trimmed + ((bi * w + wi) * oh + hi) * ow,
                           h_perm + ((bi * w + wi) * H + hi) * W, sizeof(float) * ow);
        free(h_perm);
        h_perm = trimmed;
        H = oh;
        W = ow;
    }

    float* h_back = (float*)calloc((size_t)(M * w), sizeof(float));
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int64_t hi = 0; hi < H; ++hi)
            for (int64_t wj = 0; wj < W; ++wj)
                for (int wi = 0; wi < w; ++wi)
                    h_back[((bi * H + hi) * W + wj) * w + wi] = h_perm[((bi * w + wi) * H + hi) * W + wj];

    float* q = (float*)calloc((size_t)(M * w), sizeof(float));
    if (use_int8[L]) {
        const nfo_aq* a_in = (L == 0) ? &m->a_lift : &m->a_locs[L - 1];
        nfo_linear_forward_batched(lq[L], m->q_proj_q_w.pc_scales, m->q_proj_q_w.pc_zps,
                                   lsum[L], NULL, w, w, a_in->scale, a_in->zp, (int)M, h_back, q,
                                   NULL, taps ? taps->codes_in[L] : NULL);
        for (int64_t r = 0; r < M; ++r)
            for (int j = 0; j < w; ++j) q[r * w + j] += pq_b[j];
    } else {
        nfo_linear(h_back, pq_w, pq_b, (int)M, w, w, q);
    }
    if (taps && taps->q_out) memcpy(taps->q_out, q, sizeof(float) * M * w);
    apply_fq(q, M * w, &m->a_proj_q, m->quant_enabled);
    nfo_apply_activation(q, M * w, m->relu);
    nfo_linear(q, po_w, po_b, (int)M, w, out_ch, y);
    apply_fq(y, M * out_ch, &m->a_proj_out, m->quant_enabled);

    free(q);
    free(h_back);
    free(add);
    free(pout);
    free(pin);
    free(x2);
    free(x1);
    free(h_perm);
    free(h);
    for (int i = 0; i <= L; ++i) {
        free(lq[i]);
        free(lsum[i]);
    }
    for (int i = 0; i < L; ++i) {
        free(swr[i]);
        free(swi[i]);
        free(lw[i]);
        free(lb[i]);
    }
    free(lift_w);
    free(lift_b);
    free(pq_w);
    free(pq_b);
    free(po_w);
    free(po_b);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* FNO1d (fno.cpp:408-706)                                                    */
/* ------------------------------------------------------------------------- */

/* Activation qparams of one ".output" key as FNO1d consults them: the per-tensor
 * INT8 map, the per-token map (fno.cpp:606-628) and the FP8 map (fno.cpp:580-603). */
typedef struct {
    float scale;
    int32_t zp;
    int32_t has;
    float fp8_scale;
    int32_t has_fp8;
    const float* pt_scales;
    const int32_t* pt_zps;
    int64_t pt_n;
    int32_t pt_width;
    int32_t has_pt;
} nfo_aq1;

typedef struct {
    int32_t in_ch, out_ch, width, modes, n_layers, pad_factor, relu;
    int32_t quant_enabled;  /* the IR carried a NIRQ block (runtime.cpp:25-35) */
    int32_t int8_enabled;   /* InferenceRuntime::EnableInt8Gemm was called */
    const float* lift_w;
    const float* lift_b;
    const float* proj_q_w;
    const float* proj_q_b;
    const float* proj_out_w;
    const float* proj_out_b;
    const float* spec_wr[NFO_MAX_LAYERS];
    const float* spec_wi[NFO_MAX_LAYERS];
    const float* loc_w[NFO_MAX_LAYERS];
    const float* loc_b[NFO_MAX_LAYERS];
    nfo_wq q_lift_w, q_lift_b, q_proj_q_w, q_proj_q_b, q_proj_out_w, q_proj_out_b;
    nfo_wq q_spec_wr[NFO_MAX_LAYERS];
    nfo_wq q_spec_wi[NFO_MAX_LAYERS];
    nfo_wq q_loc_w[NFO_MAX_LAYERS];
    nfo_wq q_loc_b[NFO_MAX_LAYERS];
    nfo_aq1 a_lift;
    nfo_aq1 a_locs[NFO_MAX_LAYERS];
} nfo_fno1d;

/* FNO1d::Forward with the runtime's Create-time weight fake-quant (fno.cpp:293-315)
 * and, when int8_enabled, EnableInt8Gemm's per-channel weight codes (fno.cpp:360-406)
 * and the LinearDispatchTryInt8 rule (fno.cpp:125-159).  x (b, n, in_ch) ->
 * y (b, n, out_ch).  Returns 0 or the StatusCode of a rejected call. */
int nfo_fno1d_forward(const nfo_fno1d* m, const float* x, int bsz, int n0, float* y) {
    const int w = m->width, modes = m->modes, L = m->n_layers;
    const int in_ch = m->in_ch, out_ch = m->out_ch;
    if (L > NFO_MAX_LAYERS) return 1;
    if (n0 <= 0 || (n0 & (n0 - 1))) return 1;
    {   /* per-token tables must cover the (padded) flat index range they are read at */
        int64_t np = n0;
        if (m->pad_factor > 1 && n0 % m->pad_factor) np += m->pad_factor - n0 % m->pad_factor;
        for (int i = 0; i < L; ++i) {
            const nfo_aq1* a = &m->a_locs[i];
            if (m->quant_enabled && !a->has_fp8 && a->has_pt &&
                (a->pt_width > w || np * a->pt_width > a->pt_n))
                return 1;
        }
    }

    float* lift_w = dup_floats(m->lift_w, (int64_t)w * in_ch);
    float* lift_b = dup_floats(m->lift_b, w);
    float* pq_w = dup_floats(m->proj_q_w, (int64_t)w * w);
    float* pq_b = dup_floats(m->proj_q_b, w);
    float* po_w = dup_floats(m->proj_out_w, (int64_t)out_ch * w);
    float* po_b = dup_floats(m->proj_out_b, out_ch);
    float* swr[NFO_MAX_LAYERS];
    float* swi[NFO_MAX_LAYERS];
    float* lw[NFO_MAX_LAYERS];
    float* lb[NFO_MAX_LAYERS];
    const int64_t nspec = (int64_t)w * w * modes;
    for (int i = 0; i < L; ++i) {
        swr[i] = dup_floats(m->spec_wr[i], nspec);
        swi[i] = dup_floats(m->spec_wi[i], nspec);
        lw[i] = dup_floats(m->loc_w[i], (int64_t)w * w);
        lb[i] = dup_floats(m->loc_b[i], w);
    }
    if (m->quant_enabled) {
        dq_weight(lift_w, w, in_ch, 0, 0, 2, &m->q_lift_w);
        dq_weight(lift_b, w, 0, 0, 0, 1, &m->q_lift_b);
        dq_weight(pq_w, w, w, 0, 0, 2, &m->q_proj_q_w);
        dq_weight(pq_b, w, 0, 0, 0, 1, &m->q_proj_q_b);
        dq_weight(po_w, out_ch, w, 0, 0, 2, &m->q_proj_out_w);
        dq_weight(po_b, out_ch, 0, 0, 0, 1, &m->q_proj_out_b);
        for (int i = 0; i < L; ++i) {
            dq_weight(swr[i], w, w, modes, 0, 3, &m->q_spec_wr[i]);
            dq_weight(swi[i], w, w, modes, 0, 3, &m->q_spec_wi[i]);
            dq_weight(lw[i], w, w, 0, 0, 2, &m->q_loc_w[i]);
            dq_weight(lb[i], w, 0, 0, 0, 1, &m->q_loc_b[i]);
        }
    }
    /* EnableInt8Gemm cache for locs.i (lift/proj caches exist too but Forward never
     * dispatches them) and the per-layer dispatch decision. */
    int8_t* lq[NFO_MAX_LAYERS];
    int32_t* lsum[NFO_MAX_LAYERS];
    int use_int8[NFO_MAX_LAYERS];
    for (int i = 0; i < L; ++i) {
        const nfo_aq1* a_in = (i == 0) ? &m->a_lift : &m->a_locs[i - 1];
        const nfo_wq* q = &m->q_loc_w[i];
        lq[i] = NULL;
        lsum[i] = NULL;
        use_int8[i] = m->int8_enabled && m->quant_enabled && q->has_pc && q->pc_axis == 0 &&
                      !a_in->has_pt && !a_in->has_fp8 && a_in->has;
        if (use_int8[i]) {
            lq[i] = (int8_t*)malloc((size_t)w * w);
            lsum[i] = (int32_t*)malloc(sizeof(int32_t) * w);
            nfo_quantise_weight_2d(lw[i], w, w, q->pc_scales, q->pc_zps, lq[i], lsum[i]);
        }
    }

    int64_t n = n0;
    float* h = (float*)calloc((size_t)bsz * n * w, sizeof(float));
    nfo_linear(x, lift_w, lift_b, (int)(bsz * n), in_ch, w, h);
    float* h_perm = (float*)calloc((size_t)bsz * w * n, sizeof(float));
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int wi = 0; wi < w; ++wi)
            for (int64_t ni = 0; ni < n; ++ni)
                h_perm[(bi * w + wi) * n + ni] = h[(bi * n + ni) * w + wi];
    /* fno.cpp:450-466 padding */
    int64_t pad_len = 0;
    if (m->pad_factor > 1) {
        const int64_t r = n % m->pad_factor;
        pad_len = r == 0 ? 0 : m->pad_factor - r;
        if (pad_len > 0) {
            const int64_t np = n + pad_len;
            float* padded = (float*)calloc((size_t)bsz * w * np, sizeof(float));
            for (int64_t bi = 0; bi < bsz; ++bi)
                for (int wi = 0; wi < w; ++wi)
                    memcpy(padded + (bi * w + wi) * np, h_perm + (bi * w + wi) * n,
                           sizeof(float) * n);
            free(h_perm);
            h_perm = padded;
            n = np;
        }
    }
    const int64_t numel = (int64_t)bsz * w * n;
    float* x1 = (float*)calloc((size_t)numel, sizeof(float));
    float* x2 = (float*)calloc((size_t)numel, sizeof(float));
    float* pin = (float*)calloc((size_t)numel, sizeof(float));
    float* pout = (float*)calloc((size_t)numel, sizeof(float));
    float* add = (float*)calloc((size_t)numel, sizeof(float));

    for (int i = 0; i < L; ++i) {
        const nfo_aq1* a_in = (i == 0) ? &m->a_lift : &m->a_locs[i - 1];
        const nfo_aq1* a_out = &m->a_locs[i];
        /* fno.cpp:488-508 input snap (per-tensor map only) */
        if (m->quant_enabled && a_in->has) nfo_fake_quant(h_perm, numel, a_in->scale, a_in->zp);
        nfo_spectral_conv1d(h_perm, bsz, w, (int)n, modes, swr[i], swi[i], x1);
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int64_t ni = 0; ni < n; ++ni)
                for (int wi = 0; wi < w; ++wi)
                    pin[(bi * n + ni) * w + wi] = h_perm[(bi * w + wi) * n + ni];
        if (use_int8[i]) {
            nfo_linear_forward_batched(lq[i], m->q_loc_w[i].pc_scales, m->q_loc_w[i].pc_zps,
                                       lsum[i], NULL, w, w, a_in->scale, a_in->zp,
                                       (int)(bsz * n), pin, pout, NULL, NULL);
            for (int64_t r = 0; r < bsz * n; ++r)
                for (int j = 0; j < w; ++j) pout[r * w + j] += lb[i][j];
        } else {
            nfo_linear(pin, lw[i], lb[i], (int)(bsz * n), w, w, pout);
        }
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int wi = 0; wi < w; ++wi)
                for (int64_t ni = 0; ni < n; ++ni)
                    x2[(bi * w + wi) * n + ni] = pout[(bi * n + ni) * w + wi];
        if (m->quant_enabled) {
            if (a_out->has_fp8) {
                nfo_fake_quant_fp8_log2(x2, numel, a_out->fp8_scale);
            } else if (a_out->has_pt) {
                /* fno.cpp:606-628: the loop walks x2 with a flat (n, w_axis) index
                 * although x2 is (b, w, n) here, so element k of a sample takes
                 * scale k: element (channel c, position p) uses scales[c*n + p]. */
                const int64_t wa = a_out->pt_width;
                for (int64_t bi = 0; bi < bsz; ++bi)
                    for (int64_t ni = 0; ni < n; ++ni)
                        for (int64_t wi = 0; wi < wa; ++wi) {
                            const int64_t qi = ni * wa + wi;
                            const int64_t off = bi * n * wa + ni * wa + wi;
                            x2[off] = fake_quant_pt(x2[off], a_out->pt_scales[qi],
                                                    (float)a_out->pt_zps[qi]);
                        }
            } else if (a_out->has) {
                nfo_fake_quant(x2, (int64_t)bsz * n * w, a_out->scale, a_out->zp);
            }
        }
        for (int64_t k = 0; k < numel; ++k) add[k] = x1[k] + x2[k];
        nfo_apply_activation(add, numel, m->relu);
        memcpy(h_perm, add, sizeof(float) * numel);
    }
    if (pad_len > 0) {
        const int64_t orig = n - pad_len;
        float* trimmed = (float*)calloc((size_t)bsz * w * orig, sizeof(float));
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int wi = 0; wi < w; ++wi)
                memcpy(trimmed + (bi * w + wi) * orig, h_perm + (bi * w + wi) * n,
                       sizeof(float) * orig);
        free(h_perm);
        h_perm = trimmed;
        n = orig;
    }
    float* h_back = (float*)calloc((size_t)bsz * n * w, sizeof(float));
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int64_t ni = 0; ni < n; ++ni)
            for (int wi = 0; wi < w; ++wi)
                h_back[(bi * n + ni) * w + wi] = h_perm[(bi * w + wi) * n + ni];
    float* q = (float*)calloc((size_t)bsz * n * w, sizeof(float));
    nfo_linear(h_back, pq_w, pq_b, (int)(bsz * n), w, w, q);
    nfo_apply_activation(q, (int64_t)bsz * n * w, m->relu);
    nfo_linear(q, po_w, po_b, (int)(bsz * n), w, out_ch, y);

    free(q);
    free(h_back);
    free(add);
    free(pout);
    free(pin);
    free(x2);
    free(x1);
    free(h_perm);
    free(h);
    for (int i = 0; i < L; ++i) {
        free(lq[i]);
        free(lsum[i]);
        free(swr[i]);
        free(swi[i]);
        free(lw[i]);
        free(lb[i]);
    }
    free(lift_w);
    free(lift_b);
    free(pq_w);
    free(pq_b);
    free(po_w);
    free(po_b);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* TokenMixer2D (fno.cpp:1418-1456, :1756-1956)                               */
/* ------------------------------------------------------------------------- */

/* A sequential dot-product reduction as the reference build evaluates it (the rule of
 * nfo_linear): acc0 + sum_p a[p*sa] * b[p*sb]. */
static float dot_ref(float acc, const float* a, int64_t sa, const float* b, int64_t sb, int k) {
    const int vec = nfo_linear_unfused_len(k);
    int p = 0;
    for (; p < vec; ++p) acc = acc + a[p * sa] * b[p * sb];
    for (; p < k; ++p) acc = fmaf(a[p * sa], b[p * sb], acc);
    return acc;
}

/* fno.cpp:1418-1438 LayerNormLastDim: sequential mean, sequential sum of squared
 * deviations (vector-block rule), y = fma((x - mean) * inv, gamma, beta). */
void nfo_layer_norm(const float* x, int rows, int d, const float* gamma, const float* beta,
                    float* y) {
    const float eps = 1e-5f;
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (int64_t)r * d;
        float* yr = y + (int64_t)r * d;
        float mean = 0.0f;
        for (int i = 0; i < d; ++i) mean += xr[i];
        mean /= (float)d;
        const int vec = nfo_linear_unfused_len(d);
        float var = 0.0f;
        for (int i = 0; i < d; ++i) {
            const float diff = xr[i] - mean;
            var = i < vec ? var + diff * diff : fmaf(diff, diff, var);
        }
        var /= (float)d;
        const float inv = 1.0f / sqrtf(var + eps);
        for (int i = 0; i < d; ++i) yr[i] = fmaf((xr[i] - mean) * inv, gamma[i], beta[i]);
    }
}

/* Per-row (per-token) INT8 qparams of a row by the compute_tensor_qparams rule
 * (neuroflow/quant/static_quant.py:480-533, Python floats = double): scale =
 * (max - min) / 255, zp = clip(round_half_even(-128 - min / scale)), the clipped-zp
 * scale fix-up, then the scale rounded to float32. */
void nfo_row_qparams(const float* row, int n, float* scale_out, int32_t* zp_out) {
    float mn = row[0], mx = row[0];
    for (int i = 1; i < n; ++i) {
        if (row[i] < mn) mn = row[i];
        if (row[i] > mx) mx = row[i];
    }
    if (mx == mn || mn != mn || mx != mx) {
        *scale_out = 1.0f;
        *zp_out = 0;
        return;
    }
    double scale = ((double)mx - (double)mn) / 255.0;
    const double raw = nearbyint(-128.0 - (double)mn / scale);
    double zp = raw < -128.0 ? -128.0 : (raw > 127.0 ? 127.0 : raw);
    if (zp != raw) {
        if (zp == -128.0) scale = ((double)mx - 0.0) / 255.0;
        else scale = (0.0 - (double)mn) / 255.0;
    }
    *scale_out = (float)scale;
    *zp_out = (int32_t)zp;
}

typedef struct {
    int32_t in_dim, out_dim, latent, h, w, n_patches, n_heads, n_layers, relu;
    const float* se_w;    /* slice_embed.proj (latent, in_dim) */
    const float* se_b;
    const float* un_w;    /* unslice.proj (latent, in_dim + latent) */
    const float* un_b;
    const float* head_w;  /* (out_dim, latent) */
    const float* head_b;
    /* per block: ln1, q, k, v, o, ln2, ffn0, ffn1 (weight, bias) */
    const float* blk_w[NFO_MAX_LAYERS][8];
    const float* blk_b[NFO_MAX_LAYERS][8];
    /* INT8 variant: per-channel (axis 0) weight qparams of q, k, v, o, ffn0, ffn1
     * (block slots 1, 2, 3, 4, 6, 7) */
    const float* pc_s[NFO_MAX_LAYERS][8];
    const int32_t* pc_zp[NFO_MAX_LAYERS][8];
} nfo_tm2d;

/* One Linear of the INT8 variant: per-token dynamic activation qparams, per-channel
 * weight codes (QuantiseWeight2D), the LinearForwardBatched epilogue per row, then
 * + bias as a separate add and the optional GELU (nfo_int8_gemm_rows). */
static void tm2d_linear_int8(const float* A, int M, int K, const float* W, const float* b,
                             const float* pcs, const int32_t* pczp, int N, int gelu, float* C) {
    int8_t* Wq = (int8_t*)malloc((size_t)N * K);
    int32_t* sw = (int32_t*)malloc(sizeof(int32_t) * N);
    nfo_quantise_weight_2d(W, N, K, pcs, pczp, Wq, sw);
    int8_t* Aq = (int8_t*)malloc((size_t)M * K);
    float* sA = (float*)malloc(sizeof(float) * M);
    int32_t* zA = (int32_t*)malloc(sizeof(int32_t) * M);
    for (int r = 0; r < M; ++r) {
        nfo_row_qparams(A + (int64_t)r * K, K, &sA[r], &zA[r]);
        nfo_quantise_activation(A + (int64_t)r * K, Aq + (int64_t)r * K, K, sA[r], zA[r]);
    }
    nfo_int8_gemm_rows(Aq, sA, zA, M, K, Wq, pcs, pczp, sw, N, b, gelu, C, NULL);
    free(zA);
    free(sA);
    free(Aq);
    free(sw);
    free(Wq);
}

/* mode 0: TokenMixer2D::Forward (fno.cpp:1756-1956), FP32, the reference's loops and
 *         rounding (the AV sum uses the fused scalar form: its strided V operand keeps
 *         the reference build from vectorising it).
 * mode 1: the INT8 variant: q, k, v, o, ffn0, ffn1 through tm2d_linear_int8.
 * x (b, h, w, in_dim) -> y (b, h, w, out_dim).  Returns 0 or a StatusCode. */
int nfo_tm2d_forward(const nfo_tm2d* m, int mode, const float* x, int bsz, float* y) {
    const int in_d = m->in_dim, out_d = m->out_dim, L = m->latent, np_ = m->n_patches;
    const int nh = m->n_heads, nl = m->n_layers;
    if (np_ <= 0 || (m->h * m->w) % np_ != 0 || L % nh != 0 || nl < 1 || nl > NFO_MAX_LAYERS)
        return 1;
    const int hd = L / nh;
    const int n_points = m->h * m->w;
    const int pp = n_points / np_;
    const float scale = 1.0f / sqrtf((float)hd);
    const int64_t bnp = (int64_t)bsz * np_;
    float* xp = (float*)calloc((size_t)(bnp * in_d), sizeof(float));
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int pi = 0; pi < np_; ++pi)
            for (int q = 0; q < pp; ++q) {
                const float* src = x + ((bi * n_points) + (int64_t)pi * pp + q) * in_d;
                float* dst = xp + (bi * np_ + pi) * in_d;
                for (int d = 0; d < in_d; ++d) dst[d] += src[d] / (float)pp;
            }
    float* tok = (float*)malloc(sizeof(float) * (size_t)(bnp * L));
    nfo_linear(xp, m->se_w, m->se_b, (int)bnp, in_d, L, tok);
    float* ln = (float*)malloc(sizeof(float) * (size_t)(bnp * L));
    float* Q = (float*)malloc(sizeof(float) * (size_t)(bnp * L));
    float* Kb = (float*)malloc(sizeof(float) * (size_t)(bnp * L));
    float* V = (float*)malloc(sizeof(float) * (size_t)(bnp * L));
    float* ho = (float*)malloc(sizeof(float) * (size_t)(bnp * L));
    float* f0 = (float*)malloc(sizeof(float) * (size_t)(bnp * 2 * L));
    float* f1 = (float*)malloc(sizeof(float) * (size_t)(bnp * L));
    float* attn = (float*)malloc(sizeof(float) * (size_t)np_ * np_);
    for (int li = 0; li < nl; ++li) {
        const float* const* Wt = m->blk_w[li];
        const float* const* Bt = m->blk_b[li];
        nfo_layer_norm(tok, (int)bnp, L, Wt[0], Bt[0], ln);
        if (mode == 1) {
            tm2d_linear_int8(ln, (int)bnp, L, Wt[1], Bt[1], m->pc_s[li][1], m->pc_zp[li][1], L, 0, Q);
            tm2d_linear_int8(ln, (int)bnp, L, Wt[2], Bt[2], m->pc_s[li][2], m->pc_zp[li][2], L, 0, Kb);
            tm2d_linear_int8(ln, (int)bnp, L, Wt[3], Bt[3], m->pc_s[li][3], m->pc_zp[li][3], L, 0, V);
        } else {
            nfo_linear(ln, Wt[1], Bt[1], (int)bnp, L, L, Q);
            nfo_linear(ln, Wt[2], Bt[2], (int)bnp, L, L, Kb);
            nfo_linear(ln, Wt[3], Bt[3], (int)bnp, L, L, V);
        }
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int hi = 0; hi < nh; ++hi) {
                for (int i = 0; i < np_; ++i)
                    for (int j = 0; j < np_; ++j) {
                        const float* q = Q + ((bi * np_ + i) * nh + hi) * hd;
                        const float* k = Kb + ((bi * np_ + j) * nh + hi) * hd;
                        attn[(int64_t)i * np_ + j] = dot_ref(0.0f, q, 1, k, 1, hd) * scale;
                    }
                for (int i = 0; i < np_; ++i) {  /* fno.cpp:1441-1456 */
                    float* zr = attn + (int64_t)i * np_;
                    float mx = zr[0];
                    for (int j = 1; j < np_; ++j)
                        if (zr[j] > mx) mx = zr[j];
                    float sum = 0.0f;
                    for (int j = 0; j < np_; ++j) {
                        zr[j] = expf(zr[j] - mx);
                        sum += zr[j];
                    }
                    const float inv = 1.0f / sum;
                    for (int j = 0; j < np_; ++j) zr[j] *= inv;
                }
                const int av_vec = (np_ / 4) * 4;
                for (int i = 0; i < np_; ++i)
                    for (int dh = 0; dh < hd; ++dh) {
                        float acc = 0.0f;
                        for (int j = 0; j < np_; ++j) {
                            const float a = attn[(int64_t)i * np_ + j];
                            const float v = V[((bi * np_ + j) * nh + hi) * hd + dh];
                            acc = j < av_vec ? acc + a * v : fmaf(a, v, acc);
                        }
                        ho[((bi * np_ + i) * nh + hi) * hd + dh] = acc;
                    }
            }
        if (mode == 1)
            tm2d_linear_int8(ho, (int)bnp, L, Wt[4], Bt[4], m->pc_s[li][4], m->pc_zp[li][4], L, 0, f1);
        else
            nfo_linear(ho, Wt[4], Bt[4], (int)bnp, L, L, f1);
        for (int64_t i = 0; i < bnp * L; ++i) tok[i] += f1[i];
        nfo_layer_norm(tok, (int)bnp, L, Wt[5], Bt[5], ln);
        if (mode == 1) {
            tm2d_linear_int8(ln, (int)bnp, L, Wt[6], Bt[6], m->pc_s[li][6], m->pc_zp[li][6], 2 * L,
                             m->relu ? 0 : 1, f0);
            if (m->relu)
                for (int64_t i = 0; i < bnp * 2 * L; ++i) f0[i] = f0[i] < 0.0f ? 0.0f : f0[i];
            tm2d_linear_int8(f0, (int)bnp, 2 * L, Wt[7], Bt[7], m->pc_s[li][7], m->pc_zp[li][7], L, 0, f1);
        } else {
            nfo_linear(ln, Wt[6], Bt[6], (int)bnp, L, 2 * L, f0);
            nfo_apply_activation(f0, bnp * 2 * L, m->relu);
            nfo_linear(f0, Wt[7], Bt[7], (int)bnp, 2 * L, L, f1);
        }
        for (int64_t i = 0; i < bnp * L; ++i) tok[i] += f1[i];
    }
    /* unslice: concat (x, token of the point's patch) -> Linear -> head */
    const int ipl = in_d + L;
    float* cat = (float*)malloc(sizeof(float) * (size_t)ipl);
    float* feat = (float*)malloc(sizeof(float) * (size_t)L);
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int64_t ni = 0; ni < n_points; ++ni) {
            memcpy(cat, x + (bi * n_points + ni) * in_d, sizeof(float) * in_d);
            memcpy(cat + in_d, tok + (bi * np_ + ni / pp) * L, sizeof(float) * L);
            nfo_linear(cat, m->un_w, m->un_b, 1, ipl, L, feat);
            nfo_linear(feat, m->head_w, m->head_b, 1, L, out_d, y + (bi * n_points + ni) * out_d);
        }
    free(feat);
    free(cat);
    free(attn);
    free(f1);
    free(f0);
    free(ho);
    free(V);
    free(Kb);
    free(Q);
    free(ln);
    free(tok);
    free(xp);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* FP8 E4M3 (cpp/include/neuroflow/fp8_e4m3.h)                                */
/* ------------------------------------------------------------------------- */

/* fp8_e4m3.h:106-221 fp32_to_e4m3_bits.  NaN -> 0x7F; +-inf -> +-448; +-0 keeps its
 * sign.  Normal inputs: the 23-bit mantissa is rounded to 3 bits, half to even on the
 * 20 dropped bits, a carry bumps the exponent, and biased exponents above 15 saturate
 * to +-448.  Inputs whose biased exponent is below 1 take the subnormal branch:
 * round(|v| * 2^9) to nearest-even in double, clamped to [0, 7] -- the clamp keeps
 * values in [7.5, 8) * 2^-9 at 7 * 2^-9 where an IEEE-style encoder gives 2^-6. */
uint8_t nfo_fp32_to_e4m3(float v) {
    if (isnan(v)) return 0x7F;
    if (isinf(v)) return v < 0.0f ? 0xFE : 0x7E;
    uint32_t u;
    memcpy(&u, &v, 4);
    const uint32_t sign = u >> 31;
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a == 0) return (uint8_t)(sign << 7);
    const int e = (int)((a >> 23) & 0xFFu) - 127 + 7;
    if (e < 1) {
        float af;
        memcpy(&af, &a, 4);
        double r = nearbyint((double)af * 512.0);
        if (r < 0.0) r = 0.0;
        if (r > 7.0) r = 7.0;
        return (uint8_t)((sign << 7) | (uint32_t)r);
    }
    uint32_t m = (a >> 20) & 7u;
    const uint32_t rest = a & 0xFFFFFu;
    if (rest > 0x80000u || (rest == 0x80000u && (m & 1u))) m += 1;
    int ee = e;
    if (m & 8u) {
        m &= 7u;
        ee += 1;
    }
    if (ee > 15) return (uint8_t)((sign << 7) | 0x7Eu);
    return (uint8_t)((sign << 7) | ((uint32_t)ee << 3) | m);
}

/* fp8_e4m3.h:223-284 e4m3_bits_to_fp32. */
float nfo_e4m3_to_fp32(uint8_t b) {
    const uint32_t sign = (b >> 7) & 1u, ex = (b >> 3) & 0xFu, mt = b & 7u;
    float v;
    if (ex == 0xFu && mt == 7u) {
        const uint32_t q = 0x7FC00000u | (sign << 31);
        memcpy(&v, &q, 4);
        return v;
    }
    if (ex == 0) {
        if (mt == 0) return sign ? -0.0f : 0.0f;
        v = ldexpf((float)mt, -9);
        return sign ? -v : v;
    }
    const uint32_t u = (sign << 31) | ((ex + 120u) << 23) | (mt << 20);
    memcpy(&v, &u, 4);
    return v;
}

/* fp8_e4m3.h:312-334 per-tensor fake-quant: scale down by 1/scale, saturate to +-448,
 * encode, decode, scale up. */
void nfo_fp8_fake_quant(const float* in, float scale, float* out, int64_t n) {
    const float inv = scale == 0.0f ? 1.0f : 1.0f / scale;
    for (int64_t i = 0; i < n; ++i) {
        float xs = in[i] * inv;
        xs = xs > 448.0f ? 448.0f : (xs < -448.0f ? -448.0f : xs);
        out[i] = nfo_e4m3_to_fp32(nfo_fp32_to_e4m3(xs)) * scale;
    }
}

void nfo_fp32_to_e4m3_array(const float* in, uint8_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = nfo_fp32_to_e4m3(in[i]);
}

/* ------------------------------------------------------------------------- */
/* FNO3d (fno.cpp:1031-1281)                                                  */
/* ------------------------------------------------------------------------- */

/* fno.cpp:1031-1090 SpectralConv3d on h (b, w, H, W, D). */
void nfo_spectral_conv3d(const float* h, int bsz, int w, int H, int W, int D, int mh, int mw,
                         int md, const float* w_real, const float* w_imag, float* out) {
    const int half_d = D / 2 + 1;
    const size_t vol = (size_t)H * W * half_d * 2;
    float* Hs = (float*)malloc(sizeof(float) * vol * w);
    float* Of = (float*)malloc(sizeof(float) * vol * w);
    for (int bi = 0; bi < bsz; ++bi) {
        memset(Of, 0, sizeof(float) * vol * w);
        for (int wi = 0; wi < w; ++wi)
            nfo_rfft3(h + ((int64_t)bi * w + wi) * H * W * D, H, W, D, Hs + (size_t)wi * vol);
        for (int mi = 0; mi < mh; ++mi)
            for (int mj = 0; mj < mw; ++mj)
                for (int mk = 0; mk < md; ++mk)
                    for (int wo = 0; wo < w; ++wo) {
                        float sr = 0.0f, si = 0.0f;
                        for (int wi = 0; wi < w; ++wi) {
                            const float* hp = Hs + (size_t)wi * vol +
                                              ((((int64_t)mi * W + mj) * half_d + mk) * 2);
                            const int64_t k = ((((int64_t)wi * w + wo) * mh + mi) * mw + mj) * md + mk;
                            const float hr = hp[0], hi = hp[1], wr = w_real[k], wim = w_imag[k];
                            sr = sr + fmaf(hr, wr, -(hi * wim));
                            si = si + fmaf(hr, wim, hi * wr);
                        }
                        float* op = Of + (size_t)wo * vol + ((((int64_t)mi * W + mj) * half_d + mk) * 2);
                        op[0] = sr;
                        op[1] = si;
                    }
        for (int wo = 0; wo < w; ++wo)
            nfo_irfft3(Of + (size_t)wo * vol, H, W, D, out + ((int64_t)bi * w + wo) * H * W * D);
    }
    free(Of);
    free(Hs);
}

/* FNO3d model: weights as loaded; fp8 scales for the FP8 variant. */
typedef struct {
    int32_t in_ch, out_ch, width, modes_h, modes_w, modes_d, n_layers, pad_factor, relu;
    const float* lift_w;
    const float* lift_b;
    const float* proj_q_w;
    const float* proj_q_b;
    const float* proj_out_w;
    const float* proj_out_b;
    const float* spec_wr[NFO_MAX_LAYERS];
    const float* spec_wi[NFO_MAX_LAYERS];
    const float* loc_w[NFO_MAX_LAYERS];
    const float* loc_b[NFO_MAX_LAYERS];
    /* FP8 variant: per-tensor scales of the Linear weights and of the ".output" keys */
    float s_lift_w, s_proj_q_w, s_proj_out_w;
    float s_loc_w[NFO_MAX_LAYERS];
    float s_lift, s_proj_q, s_proj_out;
    float s_locs[NFO_MAX_LAYERS];
} nfo_fno3d;

/* E4M3 codes of in / scale as fp8_e4m3_per_tensor_fake_quant forms them: xq = the
 * decoded E4M3 value, snapped = xq * scale (the fake-quantised value). */
static void fp8_codes(const float* in, float scale, float* xq, float* snapped, int64_t n) {
    const float inv = scale == 0.0f ? 1.0f : 1.0f / scale;
    for (int64_t i = 0; i < n; ++i) {
        float xs = in[i] * inv;
        xs = xs > 448.0f ? 448.0f : (xs < -448.0f ? -448.0f : xs);
        const float q = nfo_e4m3_to_fp32(nfo_fp32_to_e4m3(xs));
        if (xq) xq[i] = q;
        if (snapped) snapped[i] = q * scale;
    }
}

/* the FP8 variant's local layer: exact products of E4M3 values summed in fp32 in k
 * order, y = acc * (s_in * s_w) + bias */
static void fp8_linear(const float* aq, const float* wq, const float* b, int64_t M, int K, int N,
                       float sc, float* y) {
    for (int64_t r = 0; r < M; ++r)
        for (int o = 0; o < N; ++o) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += aq[r * K + k] * wq[(int64_t)o * K + k];
            y[r * N + o] = acc * sc + b[o];
        }
}

/* mode 0: FNO3d::Forward (fno.cpp:1096-1281), FP32, no quantisation (the reference
 *         runtime builds FNO3d without its NIRQ block, runtime.cpp:51-54).
 * mode 1: the FP8 E4M3 variant (no reference counterpart): Linear weights
 *         fake-quantised to E4M3 per tensor at load (fp8_e4m3.h:312-334); the lift
 *         output and every layer output (after the activation) become E4M3 codes with
 *         the ".output" scale of the Linear that produced them (the FNO1d input-snap
 *         convention, fno.cpp:488-508); the local layers and proj_q multiply the
 *         E4M3 codes exactly and sum in fp32 in k order (fp8_linear);
 *         locs.i.output, proj_q.output and proj_out.output are E4M3 fake-quantised
 *         like FNO2d's boundaries (fno.cpp:810-844).
 * x (b, H, W, D, in_ch) -> y (b, H, W, D, out_ch). */
/* taps (mode 1, or NULL): the E4M3 values of every layer input -- the lift's output, then
 * each layer's output -- as L + 1 consecutive channel-first padded (B, C, Hp, Wp, Dp)
 * blocks */
static int fno3d_forward_impl(const nfo_fno3d* m, int mode, const float* x, int bsz, int H0, int W0, int D0,
                              float* y, float* taps) {
    const int w = m->width, mh = m->modes_h, mw = m->modes_w, md = m->modes_d, L = m->n_layers;
    const int in_ch = m->in_ch, out_ch = m->out_ch;
    if (L > NFO_MAX_LAYERS) return 1;
    const int pw[3] = {H0, W0, D0};
    for (int i = 0; i < 3; ++i)
        if (pw[i] <= 0 || (pw[i] & (pw[i] - 1))) return 1;
    float* lift_w = dup_floats(m->lift_w, (int64_t)w * in_ch);
    float* pq_w = dup_floats(m->proj_q_w, (int64_t)w * w);
    float* po_w = dup_floats(m->proj_out_w, (int64_t)out_ch * w);
    float* pq_q = (float*)malloc(sizeof(float) * (size_t)w * w);
    float* lw[NFO_MAX_LAYERS];
    float* lq[NFO_MAX_LAYERS];
    for (int i = 0; i < L; ++i) {
        lw[i] = dup_floats(m->loc_w[i], (int64_t)w * w);
        lq[i] = (float*)malloc(sizeof(float) * (size_t)w * w);
    }
    if (mode == 1) {
        fp8_codes(lift_w, m->s_lift_w, NULL, lift_w, (int64_t)w * in_ch);
        fp8_codes(pq_w, m->s_proj_q_w, pq_q, pq_w, (int64_t)w * w);
        fp8_codes(po_w, m->s_proj_out_w, NULL, po_w, (int64_t)out_ch * w);
        for (int i = 0; i < L; ++i) fp8_codes(lw[i], m->s_loc_w[i], lq[i], lw[i], (int64_t)w * w);
    }
    int64_t H = H0, W = W0, D = D0;
    const int64_t P = H * W * D, M = (int64_t)bsz * P;
    float* h = (float*)malloc(sizeof(float) * (size_t)(M * w));
    nfo_linear(x, lift_w, m->lift_b, (int)M, in_ch, w, h);
    float* hp = (float*)calloc((size_t)(M * w), sizeof(float));   /* channel-first values */
    float* xq = (float*)calloc((size_t)(M * w), sizeof(float));   /* channel-first E4M3 codes */
    if (mode == 1) fp8_codes(h, m->s_lift, NULL, h, M * w);
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int wi = 0; wi < w; ++wi)
            for (int64_t p = 0; p < P; ++p) hp[(bi * w + wi) * P + p] = h[(bi * P + p) * w + wi];
    if (mode == 1) fp8_codes(hp, m->s_lift, xq, NULL, M * w);  /* the codes of the snapped lift */
    int64_t pad[3] = {0, 0, 0};
    if (m->pad_factor > 1) {
        const int pf = m->pad_factor;
        const int64_t dims[3] = {H, W, D};
        for (int i = 0; i < 3; ++i) pad[i] = (pf - (dims[i] % pf)) % pf;
        if (pad[0] || pad[1] || pad[2]) {
            const int64_t Hp = H + pad[0], Wp = W + pad[1], Dp = D + pad[2];
            float* a = (float*)calloc((size_t)(bsz * w * Hp * Wp * Dp), sizeof(float));
            float* b = (float*)calloc((size_t)(bsz * w * Hp * Wp * Dp), sizeof(float));
            for (int64_t bw = 0; bw < (int64_t)bsz * w; ++bw)
                for (int64_t hi = 0; hi < H; ++hi)
                    for (int64_t wj = 0; wj < W; ++wj) {
                        memcpy(a + ((bw * Hp + hi) * Wp + wj) * Dp, hp + ((bw * H + hi) * W + wj) * D,
                               sizeof(float) * D);
                        memcpy(b + ((bw * Hp + hi) * Wp + wj) * Dp, xq + ((bw * H + hi) * W + wj) * D,
                               sizeof(float) * D);
                    }
            free(hp);
            free(xq);
            hp = a;
            xq = b;
            H = Hp;
            W = Wp;
            D = Dp;
        }
    }
    const int64_t Pp = H * W * D, Mp = (int64_t)bsz * Pp;
    if (taps && mode == 1) memcpy(taps, xq, sizeof(float) * (size_t)(Mp * w));
    float* x1 = (float*)malloc(sizeof(float) * (size_t)(Mp * w));
    float* pin = (float*)malloc(sizeof(float) * (size_t)(Mp * w));
    float* pout = (float*)malloc(sizeof(float) * (size_t)(Mp * w));
    for (int i = 0; i < L; ++i) {
        nfo_spectral_conv3d(hp, bsz, w, (int)H, (int)W, (int)D, mh, mw, md, m->spec_wr[i], m->spec_wi[i], x1);
        const float* src = mode == 1 ? xq : hp;
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int64_t p = 0; p < Pp; ++p)
                for (int wi = 0; wi < w; ++wi) pin[(bi * Pp + p) * w + wi] = src[(bi * w + wi) * Pp + p];
        if (mode == 1) {
            const float s_in = i == 0 ? m->s_lift : m->s_locs[i - 1];
            fp8_linear(pin, lq[i], m->loc_b[i], Mp, w, w, s_in * m->s_loc_w[i], pout);
            fp8_codes(pout, m->s_locs[i], NULL, pout, Mp * w);
        } else {
            nfo_linear(pin, lw[i], m->loc_b[i], (int)Mp, w, w, pout);
        }
        for (int64_t bi = 0; bi < bsz; ++bi)
            for (int wi = 0; wi < w; ++wi)
                for (int64_t p = 0; p < Pp; ++p) {
                    const int64_t k = (bi * w + wi) * Pp + p;
                    hp[k] = x1[k] + pout[(bi * Pp + p) * w + wi];
                }
        nfo_apply_activation(hp, Mp * w, m->relu);
        if (mode == 1) fp8_codes(hp, m->s_locs[i], xq, hp, Mp * w);
        if (taps && mode == 1) memcpy(taps + (size_t)(i + 1) * (size_t)(Mp * w), xq, sizeof(float) * (size_t)(Mp * w));
    }
    if (pad[0] || pad[1] || pad[2]) {
        const int64_t oh = H - pad[0], ow = W - pad[1], od = D - pad[2];
        float* a = (float*)malloc(sizeof(float) * (size_t)(bsz * w * oh * ow * od));
        float* b = (float*)malloc(sizeof(float) * (size_t)(bsz * w * oh * ow * od));
        for (int64_t bw = 0; bw < (int64_t)bsz * w; ++bw)
            for (int64_t hi = 0; hi < oh; ++hi)
                for (int64_t wj = 0; wj < ow; ++wj) {
                    memcpy(a + ((bw * oh + hi) * ow + wj) * od, hp + ((bw * H + hi) * W + wj) * D,
                           sizeof(float) * od);
                    memcpy(b + ((bw * oh + hi) * ow + wj) * od, xq + ((bw * H + hi) * W + wj) * D,
                           sizeof(float) * od);
                }
        free(hp);
        free(xq);
        hp = a;
        xq = b;
        H = oh;
        W = ow;
        D = od;
    }
    float* hb = (float*)malloc(sizeof(float) * (size_t)(M * w));
    const float* src = mode == 1 ? xq : hp;
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int64_t p = 0; p < P; ++p)
            for (int wi = 0; wi < w; ++wi) hb[(bi * P + p) * w + wi] = src[(bi * w + wi) * P + p];
    float* q = (float*)malloc(sizeof(float) * (size_t)(M * w));
    if (mode == 1) {
        const float s_in = L == 0 ? m->s_lift : m->s_locs[L - 1];
        fp8_linear(hb, pq_q, m->proj_q_b, M, w, w, s_in * m->s_proj_q_w, q);
        fp8_codes(q, m->s_proj_q, NULL, q, M * w);
    } else {
        nfo_linear(hb, pq_w, m->proj_q_b, (int)M, w, w, q);
    }
    nfo_apply_activation(q, M * w, m->relu);
    nfo_linear(q, po_w, m->proj_out_b, (int)M, w, out_ch, y);
    if (mode == 1) fp8_codes(y, m->s_proj_out, NULL, y, M * out_ch);
    free(q);
    free(hb);
    free(pout);
    free(pin);
    free(x1);
    free(xq);
    free(hp);
    free(h);
    for (int i = 0; i < L; ++i) {
        free(lw[i]);
        free(lq[i]);
    }
    free(pq_q);
    free(po_w);
    free(pq_w);
    free(lift_w);
    return 0;
}

int nfo_fno3d_forward(const nfo_fno3d* m, int mode, const float* x, int bsz, int H0, int W0, int D0,
                      float* y) {
    return fno3d_forward_impl(m, mode, x, bsz, H0, W0, D0, y, NULL);
}

int nfo_fno3d_forward_taps(const nfo_fno3d* m, int mode, const float* x, int bsz, int H0, int W0, int D0,
                           float* y, float* taps) {
    return fno3d_forward_impl(m, mode, x, bsz, H0, W0, D0, y, taps);
}

/* ------------------------------------------------------------------------- */
/* DeepONet (fno.cpp:1289-1406)                                               */
/* ------------------------------------------------------------------------- */

#define NFO_MAX_MLP 8

/* Weights as loaded (ir_loader.h:514-547): branch/trunk layers (out, in) + bias, and
 * the output bias (out_ch).  Hidden widths come from the second-to-last layer. */
typedef struct {
    int32_t in_branch, in_trunk, latent, out_ch, n_branch, n_trunk, hidden_branch, hidden_trunk, relu;
    const float* bw[NFO_MAX_MLP];
    const float* bb[NFO_MAX_MLP];
    const float* tw[NFO_MAX_MLP];
    const float* tb[NFO_MAX_MLP];
    const float* bias;
} nfo_deeponet;

/* One MLP as DeepONet::Forward runs it: Linear per layer, activation after every
 * layer but the last (fno.cpp:1325-1343, :1368-1385). Returns the final rows. */
static float* deeponet_mlp(const float* x, int64_t rows, int in0, int n, int hidden, int last,
                           const float* const* W, const float* const* b, int relu) {
    float* cur = dup_floats(x, rows * in0);
    int in = in0;
    for (int i = 0; i < n; ++i) {
        const int out = (i == n - 1) ? last : hidden;
        float* next = (float*)calloc((size_t)(rows * out), sizeof(float));
        nfo_linear(cur, W[i], b[i], (int)rows, in, out, next);
        if (i < n - 1) nfo_apply_activation(next, rows * out, relu);
        free(cur);
        cur = next;
        in = out;
    }
    return cur;
}

/* u (b, n_sensor, in_branch), y (b, n_query, in_trunk) -> out (b, n_query, out_ch).
 * The sensor mean is a sequential sum divided by n_sensor (fno.cpp:1352-1361); the
 * branch/trunk dot product (fno.cpp:1388-1398) is reduced in order and vectorised by
 * the reference build like Linear: products of the first nfo_linear_unfused_len(latent)
 * terms rounded then added, the rest fused; then + bias. */
int nfo_deeponet_forward(const nfo_deeponet* m, const float* u, int bsz, int n_sensor,
                         const float* y, int n_query, float* out) {
    if (m->n_branch < 1 || m->n_trunk < 1 || m->n_branch > NFO_MAX_MLP || m->n_trunk > NFO_MAX_MLP)
        return 3;
    const int oc = m->out_ch, lat = m->latent;
    const int64_t rb = (int64_t)bsz * n_sensor, rt = (int64_t)bsz * n_query;
    float* bf = deeponet_mlp(u, rb, m->in_branch, m->n_branch, m->hidden_branch, oc * lat,
                             m->bw, m->bb, m->relu);
    float* bo = (float*)calloc((size_t)bsz * oc * lat, sizeof(float));
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int ci = 0; ci < oc; ++ci)
            for (int k = 0; k < lat; ++k) {
                float acc = 0.0f;
                for (int64_t si = 0; si < n_sensor; ++si)
                    acc = acc + bf[((bi * n_sensor + si) * oc + ci) * lat + k];
                bo[(bi * oc + ci) * lat + k] = acc / (float)n_sensor;
            }
    float* tf = deeponet_mlp(y, rt, m->in_trunk, m->n_trunk, m->hidden_trunk, lat, m->tw, m->tb,
                             m->relu);
    const int vec = nfo_linear_unfused_len(lat);
    for (int64_t bi = 0; bi < bsz; ++bi)
        for (int64_t i = 0; i < n_query; ++i)
            for (int ci = 0; ci < oc; ++ci) {
                const float* a = bo + (bi * oc + ci) * lat;
                const float* t = tf + (bi * n_query + i) * lat;
                float acc = 0.0f;
                int k = 0;
                for (; k < vec; ++k) acc = acc + a[k] * t[k];
                for (; k < lat; ++k) acc = fmaf(a[k], t[k], acc);
                out[(bi * n_query + i) * oc + ci] = acc + m->bias[ci];
            }
    free(tf);
    free(bo);
    free(bf);
    return 0;
}

/* ------------------------------------------------------------------------- */
/* GraphOp / GraphOp2D (fno.cpp:1653-1741, :1969-2060)                         */
/* ------------------------------------------------------------------------- */

/* Both ops run the same network on n_nodes = n_nodes (1D) or h*w (2D) nodes; the
 * adjacency is CSR (offsets n_nodes + 1, indices), deg_inv per node. */
typedef struct {
    int32_t in_dim, out_dim, n_nodes, hidden, n_layers, relu;
    const float* lift_w;
    const float* lift_b;
    const float* self_w[NFO_MAX_LAYERS];
    const float* self_b[NFO_MAX_LAYERS];
    const float* neigh_w[NFO_MAX_LAYERS];
    const float* neigh_b[NFO_MAX_LAYERS];
    const float* head_w;
    const float* head_b;
    const int32_t* adj_off;
    const int32_t* adj_idx;
    const float* deg_inv;
} nfo_graphop;

/* x (b, n_nodes, in_dim) -> y (b, n_nodes, out_dim).  Aggregation: per node and
 * batch, a sequential sum of the neighbours' rows in CSR order from 0, times deg_inv;
 * then Linear(h) + Linear(agg), the activation, and h += (fno.cpp:1698-1733). */
int nfo_graphop_forward(const nfo_graphop* m, const float* x, int bsz, float* y) {
    if (m->n_layers < 1 || m->n_layers > NFO_MAX_LAYERS) return 3;
    const int n = m->n_nodes, hd = m->hidden;
    const int64_t bnh = (int64_t)bsz * n;
    float* h = (float*)calloc((size_t)(bnh * hd), sizeof(float));
    float* agg = (float*)calloc((size_t)(bnh * hd), sizeof(float));
    float* hs = (float*)calloc((size_t)(bnh * hd), sizeof(float));
    float* hn = (float*)calloc((size_t)(bnh * hd), sizeof(float));
    nfo_linear(x, m->lift_w, m->lift_b, (int)bnh, m->in_dim, hd, h);
    for (int li = 0; li < m->n_layers; ++li) {
        memset(agg, 0, sizeof(float) * (size_t)(bnh * hd));
        for (int i = 0; i < n; ++i) {
            const int lo = m->adj_off[i], hi = m->adj_off[i + 1];
            const float di = m->deg_inv[i];
            for (int64_t bi = 0; bi < bsz; ++bi) {
                float* dst = agg + (bi * n + i) * hd;
                for (int k = lo; k < hi; ++k) {
                    const float* src = h + (bi * n + m->adj_idx[k]) * hd;
                    for (int d = 0; d < hd; ++d) dst[d] = dst[d] + src[d];
                }
                for (int d = 0; d < hd; ++d) dst[d] = dst[d] * di;
            }
        }
        nfo_linear(h, m->self_w[li], m->self_b[li], (int)bnh, hd, hd, hs);
        nfo_linear(agg, m->neigh_w[li], m->neigh_b[li], (int)bnh, hd, hd, hn);
        for (int64_t k = 0; k < bnh * hd; ++k) hs[k] = hs[k] + hn[k];
        nfo_apply_activation(hs, bnh * hd, m->relu);
        for (int64_t k = 0; k < bnh * hd; ++k) h[k] = h[k] + hs[k];
    }
    nfo_linear(h, m->head_w, m->head_b, (int)bnh, hd, m->out_dim, y);
    free(hn);
    free(hs);
    free(agg);
    free(h);
    return 0;
}
