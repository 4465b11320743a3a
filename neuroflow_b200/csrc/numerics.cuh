// numerics.cuh -- device restatements of the reference runtime's scalar arithmetic,
// written with explicit IEEE intrinsics so that nvcc cannot re-associate or contract
// them differently from the reference build (GCC -O3 -mfma, whose contraction choices
// are spelled out per function below).
#pragma once

#include <climits>
#include <cstdint>

#include "nfx_internal.h"

namespace nfx {

// int8_gemm.cpp:514-518 QuantiseActivation for one element:
//   q = (int32)std::round(v / s) + zp, clamped to [-128, 127].
// std::round is half-away-from-zero (CUDA roundf); the division is IEEE.  The
// float->int conversion follows x86 cvttss2si, which the reference executes: values
// outside int32 range and NaN become INT_MIN, and the following `+ zp` wraps.
__device__ __forceinline__ int quantise_i8(float v, float s, int zp) {
    const float r = roundf(__fdiv_rn(v, s));
    int q = (fabsf(r) < 2147483648.0f) ? __float2int_rz(r) : INT_MIN;
    q = static_cast<int>(static_cast<unsigned>(q) + static_cast<unsigned>(zp));
    return q < -128 ? -128 : (q > 127 ? 127 : q);
}

// fno.cpp:497-505 / :830-842: the float form of the same code,
//   q = std::round(v / s) + zp (float), clamped with ordered compares (NaN passes).
__device__ __forceinline__ float fq_code(float v, float s, float zp) {
    float q = __fadd_rn(roundf(__fdiv_rn(v, s)), zp);
    if (q < -128.0f) q = -128.0f;
    if (q > 127.0f) q = 127.0f;
    return q;
}

// The same code without a division on the common path.  r = v * fl(1/s) differs from
// v / s by at most |v/s| * 2^-23, and the reference's quotient fl(v / s) from v / s by
// at most |v/s| * 2^-24; for |v/s| < 2^8 the two are within 1.5 * 2^-15 of each other,
// so rounding r to the nearest integer gives the rounding of the reference's quotient
// whenever r is not within 2^-14 of a half-integer (there round-half-away and
// round-half-even agree too; r - rint(r) is exact).  For |v/s| >= 2^8 both roundings
// are at least 256 in magnitude and saturate the code (|k| > 255 for any zero point).
// Inputs next to a half-integer, and NaN, take the exact path.
constexpr float kFastRoundLimit = 0.49993896484375f;  // 0.5 - 2^-14
__device__ __forceinline__ float fq_code_fast(float v, float s, float inv_s, float zp) {
    const float r = __fmul_rn(v, inv_s);
    const float k = rintf(r);
    if (!(fabsf(__fsub_rn(r, k)) < kFastRoundLimit)) return fq_code(v, s, zp);
    float q = __fadd_rn(k, zp);
    q = fminf(fmaxf(q, -128.0f), 127.0f);
    return q;
}

// Branch-free form of the fast path for unrolled epilogues: returns the fast code and
// reports in `bad` whether the element needs the exact path (the caller fixes those
// elements afterwards, outside the unrolled loop).
__device__ __forceinline__ float fq_code_try(float v, float inv_s, float zp, bool& bad) {
    const float r = __fmul_rn(v, inv_s);
    const float k = rintf(r);
    bad = !(fabsf(__fsub_rn(r, k)) < kFastRoundLimit);
    return fminf(fmaxf(__fadd_rn(k, zp), -128.0f), 127.0f);
}

// The same test returning the snapped value's integer offset directly:
// (fq_code - zp) = clamp(k, -128 - zp, 127 - zp), exact because k is an integer-valued
// float below 2^24 on the fast path.  klo = -128 - zp, khi = 127 - zp.
__device__ __forceinline__ float fq_offset_try(float v, float inv_s, float klo, float khi, bool& bad) {
    const float r = __fmul_rn(v, inv_s);
    const float k = rintf(r);
    bad = !(fabsf(__fsub_rn(r, k)) < kFastRoundLimit);
    return fminf(fmaxf(k, klo), khi);
}

// Two independent fp32 operations in one instruction (the sm_100 f32x2 forms): IEEE
// round-to-nearest per lane, so each lane equals the scalar __fmul_rn / __fmaf_rn
// result bit for bit.  A product from mul2_rn must not feed a packed add or subtract:
// ptxas contracts mul.rn.f32x2 followed by add.rn.f32x2 into one fused f32x2 FMA
// despite the explicit rounding (found by comparing against the scalar forms); sums of
// packed products are therefore written as scalar __fadd_rn / __fsub_rn.
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
        "mul.rn.f32x2 z, x, y;\n\tmov.b64 {%0, %1}, z;\n\t}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    float2 r;
    asm("{\n\t.reg .b64 x, y, w, z;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
        "mov.b64 w, {%6, %7};\n\tfma.rn.f32x2 z, x, y, w;\n\tmov.b64 {%0, %1}, z;\n\t}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return r;
}

// fake-quant round trip: (q - zp) * s.
__device__ __forceinline__ float fake_quant(float v, float s, float zp) {
    return __fmul_rn(__fsub_rn(fq_code(v, s, zp), zp), s);
}

// fno.cpp:36-48 GELU (tanh form).  The reference build evaluates
//   z + 0.044715f*z*z*z   as   fma(z, (0.044715f*z)*z, z)
// and 0.5f*z*(1+t) as (0.5f*z)*(1+t).  tanhf is CUDA's (the reference uses glibc's;
// the two differ by at most a couple of ulps, which the parity tolerance states).
__device__ __forceinline__ float gelu_tanh(float z) {
    const float c = 0x1.988452p-1f;  // sqrtf(2.0f / (float)M_PI): both steps correctly rounded
    const float t = __fmul_rn(__fmul_rn(0.044715f, z), z);
    const float inner = __fmaf_rn(z, t, z);
    const float th = tanhf(__fmul_rn(c, inner));
    return __fmul_rn(__fmul_rn(0.5f, z), __fadd_rn(1.0f, th));
}

__device__ __forceinline__ float relu_ref(float z) { return z < 0.0f ? 0.0f : z; }

// fno.cpp:585-603 / :813-828 FP8 branch: log2 snap of v / scale.  The std::ldexp
// exponent is the float round(log2|u| * 8) / 8 truncated to int, as the reference
// computes it.  log2f is CUDA's (glibc's may differ by an ulp next to a breakpoint).
__device__ __forceinline__ float fp8_log2_snap(float v, float scale) {
    if (!(scale > 0.0f)) return v;
    const float u = __fdiv_rn(v, scale);
    const float a = fabsf(u);
    const float sign = u < 0.0f ? -1.0f : 1.0f;
    const float qv = (a < 0.015625f)
                         ? a
                         : ldexpf(1.0f, static_cast<int>(__fdiv_rn(
                                            roundf(__fmul_rn(log2f(a), 8.0f)), 8.0f)));
    return __fmul_rn(__fmul_rn(sign, fminf(qv, 448.0f)), scale);
}

// A float's bits mapped to an unsigned key with the same order (negative values
// reversed), so that atomicMin / atomicMax on keys are min / max on the floats.
__host__ __device__ __forceinline__ unsigned float_order_key(float v) {
#ifdef __CUDA_ARCH__
    const unsigned u = __float_as_uint(v);
#else
    unsigned u;
    memcpy(&u, &v, 4);
#endif
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ __forceinline__ float float_from_order_key(unsigned k) {
    const unsigned u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float v;
    memcpy(&v, &u, 4);
    return v;
#endif
}

// fp8_e4m3.h:106-221 fp32_to_e4m3_bits, the reference's encoder: NaN -> 0x7F, +-inf ->
// +-448, round-half-even of the mantissa to 3 bits with exponent carry and saturation
// to +-448; below the normal range round(|v| * 2^9) clamped to [0, 7] (so values in
// [7.5, 8) * 2^-9 stay at code 7 where the hardware cvt gives the smallest normal).
__device__ __forceinline__ uint32_t e4m3_encode_ref(float v) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t sign = u >> 31, a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7Fu;
    if (a == 0x7F800000u) return sign ? 0xFEu : 0x7Eu;
    if (a == 0) return sign << 7;
    const int e = static_cast<int>(a >> 23) - 120;
    if (e < 1) {
        const float r = fminf(fmaxf(rintf(__fmul_rn(__uint_as_float(a), 512.0f)), 0.0f), 7.0f);
        return (sign << 7) | static_cast<uint32_t>(r);
    }
    uint32_t m = (a >> 20) & 7u;
    const uint32_t rest = a & 0xFFFFFu;
    if (rest > 0x80000u || (rest == 0x80000u && (m & 1u))) ++m;
    int ee = e;
    if (m & 8u) {
        m &= 7u;
        ++ee;
    }
    if (ee > 15) return (sign << 7) | 0x7Eu;
    return (sign << 7) | (static_cast<uint32_t>(ee) << 3) | m;
}

// fp8_e4m3.h:223-284 e4m3_bits_to_fp32.
__device__ __forceinline__ float e4m3_decode_ref(uint32_t b) {
    const uint32_t sign = (b >> 7) & 1u, ex = (b >> 3) & 15u, mt = b & 7u;
    if (ex == 15u && mt == 7u) return __uint_as_float(0x7FC00000u | (sign << 31));
    if (ex == 0u) {
        const float v = __fmul_rn(static_cast<float>(mt), 0.001953125f);
        return sign ? -v : v;
    }
    return __uint_as_float((sign << 31) | ((ex + 120u) << 23) | (mt << 20));
}

// e4m3_encode_ref of v clamped to [-448, 448] (e4m3_code's saturation; NaN passes), by
// the hardware conversion.  cvt.rn.satfinite.e4m3x2.f32 rounds half-even to 3 mantissa
// bits like the reference and saturates finite values and infinities to +-448 itself;
// the two differ only where the reference's subnormal rule keeps |v| in [7.5, 8) *
// 2^-9 at code 7 (the conversion gives the smallest normal, code 8) and on NaN (the
// reference gives 0x7F for either sign); both are patched.  nfx_fp8_e4m3_selfcheck
// compares the two over every fp32 bit pattern.
__device__ __forceinline__ uint32_t e4m3_encode_fast(float v) {
#ifdef __CUDA_ARCH__
    unsigned short r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
    uint32_t c = r & 0xFFu;
    c = ((c & 0x7Fu) == 8u && fabsf(v) < 0.015625f) ? c - 1u : c;
    return v != v ? 0x7Fu : c;
#else
    return e4m3_encode_ref(v);
#endif
}

// e4m3_decode_ref by the hardware conversion (E4M3 -> f16 is exact, f16 -> f32 too);
// the NaN codes get the reference's bit pattern.
__device__ __forceinline__ float e4m3_decode_fast(uint32_t b) {
#ifdef __CUDA_ARCH__
    uint32_t h2;
    const unsigned short in = static_cast<unsigned short>(b & 0xFFu);
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(in));
    float f;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tcvt.f32.f16 %0, lo;\n\t}" : "=f"(f) : "r"(h2));
    return (b & 0x7Fu) == 0x7Fu ? __uint_as_float(0x7FC00000u | ((b & 0x80u) << 24)) : f;
#else
    return e4m3_decode_ref(b);
#endif
}

// fp8_fake_quant for a value whose result is only consumed on the way to another E4M3
// code (e4m3_code patches a NaN to the reference's 0x7F there): the same value for
// every non-NaN input, a NaN for a NaN, without the NaN bit-pattern fix-ups.
__device__ __forceinline__ float fp8_fake_quant_inner(float v, float scale, float inv) {
#ifdef __CUDA_ARCH__
    const float xs = __fmul_rn(v, inv);
    unsigned short r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(xs));
    r = ((r & 0x7Fu) == 8u && fabsf(xs) < 0.015625f) ? static_cast<unsigned short>(r - 1u) : r;
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(r));
    float f;
    asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tcvt.f32.f16 %0, lo;\n\t}" : "=f"(f) : "r"(h2));
    return __fmul_rn(f, scale);
#else
    float xs = __fmul_rn(v, inv);
    xs = xs > 448.0f ? 448.0f : (xs < -448.0f ? -448.0f : xs);
    return __fmul_rn(e4m3_decode_ref(e4m3_encode_ref(xs)), scale);
#endif
}

// fp8_e4m3.h:312-334: the E4M3 code of v under `inv` = 1/scale (scale 0 -> 1).
__device__ __forceinline__ uint32_t e4m3_code(float v, float inv) {
    return e4m3_encode_fast(__fmul_rn(v, inv));
}
// ... and the fake-quantised value
__device__ __forceinline__ float fp8_fake_quant(float v, float scale, float inv) {
    return __fmul_rn(e4m3_decode_fast(e4m3_code(v, inv)), scale);
}

// fno.cpp:810-844 apply_fake_quant for one element: FP8 first, else INT8 per-tensor.
__device__ __forceinline__ float apply_fq(float v, const FqParam& q) {
    if (q.kind == 1) return fake_quant(v, q.scale, static_cast<float>(q.zp));
    if (q.kind == 2) return fp8_log2_snap(v, q.scale);
    return v;
}

// fno.cpp:51-80 Linear (acc = b; acc += x[p]*w[p] for p = 0..k-1) as the reference
// build (GCC -O3 with the AVX-512 flags of cpp/CMakeLists.txt:78) evaluates it: the
// sum is sequential, but the first linear_unfused_len(k) products come from 16- and
// 8-wide vector multiplies and are added rounded; the scalar tail (k mod 8 terms) is
// fused.
__host__ __device__ constexpr int linear_unfused_len(int k) {
    return (k - (k / 16) * 16 >= 8) ? (k / 16) * 16 + 8 : (k / 16) * 16;
}
__device__ __forceinline__ float linear_step(float acc, float x, float w, bool fused) {
    return fused ? __fmaf_rn(x, w, acc) : __fadd_rn(acc, __fmul_rn(x, w));
}

// The next layer's code from z = x1 + x2 via the host-built exact table (nfx_lut.h).
// Cell index fma(z, inv_delta, c) with c = -zlo * inv_delta (the cells overlap their
// neighbours by far more than this index's rounding); the cell holds the breakpoint t
// and the codes below / from t as bytes lo | hi << 8.
__device__ __forceinline__ int2 lut_cell(float z, const int2* lut, int ncells, float inv_delta,
                                         float c) {
    int idx = __float2int_rz(__fmaf_rn(z, inv_delta, c));
    idx = idx < 0 ? 0 : (idx > ncells - 1 ? ncells - 1 : idx);
    return lut[idx];
}
__device__ __forceinline__ int code_from_lut(float z, const int2* lut, int ncells, float zlo,
                                             float inv_delta) {
    const int2 cell = lut_cell(z, lut, ncells, inv_delta, __fmul_rn(-zlo, inv_delta));
    const int w = z >= __int_as_float(cell.x) ? (cell.y >> 8) : cell.y;
    return static_cast<int>(static_cast<int8_t>(w & 0xFF));
}

// int8_gemm.cpp:574-577 epilogue of LinearForwardBatched for one output:
//   v = acc - zp_w*sum_a - zp_A*sum_w + K*zp_w*zp_A,  acc = sum a*(w - zp_w)
// Given raw = sum a*w (the tensor-core product) and sum_a, acc = raw - zp_w*sum_a, so
//   v = raw + zp_w*(K*zp_A - 2*sum_a) - zp_A*sum_w.
// Every term stays inside int32 for K <= 256, so int32 arithmetic gives the same
// value as the reference's int32/int64 mix.  y = (sW*sA)*float(v), then y + 0.0f.
__device__ __forceinline__ float dequant_ref(int raw, int zp_w, int rconst, int zpA_sumw,
                                             float sWsA) {
    const int v = raw + zp_w * rconst - zpA_sumw;
    return __fadd_rn(__fmul_rn(sWsA, __int2float_rn(v)), 0.0f);
}

}  // namespace nfx
