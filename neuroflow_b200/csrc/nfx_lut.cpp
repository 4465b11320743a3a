// nfx_lut.cpp -- construction of the exact activation/quantisation tables.
//
// This file is compiled for the host without FMA contraction (x86-64 baseline), so
// every float operation below rounds exactly where written.  The reference build
// (GCC -O3 -mfma) contracts one product of its GELU, z + 0.044715f*z*z*z, into
// fma(z, (0.044715f*z)*z, z); std::fma reproduces that.  tanh is the C library's
// tanhf, the function the reference calls.
#include "nfx_lut.h"

#include <cmath>
#include <cstring>
#include <limits>

namespace nfx {
namespace {

float next_up(float x) { return std::nextafter(x, std::numeric_limits<float>::infinity()); }

// order-preserving map of finite floats to integers, and back
int64_t f2o(float f) {
    int32_t i;
    std::memcpy(&i, &f, 4);
    return i >= 0 ? static_cast<int64_t>(i) : -static_cast<int64_t>(i & 0x7FFFFFFF);
}
float o2f(int64_t o) {
    int32_t i = o >= 0 ? static_cast<int32_t>(o) : static_cast<int32_t>((-o) | 0x80000000u);
    float f;
    std::memcpy(&f, &i, 4);
    return f;
}

struct Transition {
    float t;         // smallest float with the new code (bisection result)
    int before, after;
};

// Saturating index form: cell j of a segment covers [zlo + j delta, zlo + (j + 1) delta)
// (plus margins), i.e. idx = round((z - zlo) / delta - 0.5) + offset, evaluated as
// u = sat((z * inv + c) / (n - 1)) and idx = rint(u * (n - 1)) via the 1.5 * 2^23
// addend; the extra roundings move the index by far less than the cell margin.
void set_sat_params(CodeLut& L, double zlo0, double d0, double zlo1, double d1, int off1) {
    const double nm1 = static_cast<double>(L.cells.size()) - 1.0;
    L.nm1 = static_cast<float>(nm1);
    if (nm1 <= 0.0) {
        L.alpha0 = L.alpha1 = L.beta0 = L.beta1 = 0.0f;
        return;
    }
    L.alpha0 = static_cast<float>(1.0 / d0 / nm1);
    L.beta0 = static_cast<float>((-zlo0 / d0 - 0.5) / nm1);
    L.alpha1 = static_cast<float>(1.0 / d1 / nm1);
    L.beta1 = static_cast<float>((off1 - zlo1 / d1 - 0.5) / nm1);
}

}  // namespace

int lut_index_sat(float z, const CodeLut& L) {
    const bool s0 = z < L.zsplit;
    float u = std::fma(z, s0 ? L.alpha0 : L.alpha1, s0 ? L.beta0 : L.beta1);
    u = (u > 0.0f) ? (u < 1.0f ? u : 1.0f) : 0.0f;  // saturate; NaN -> 0
    const float x = std::fma(u, L.nm1, 12582912.0f);
    int32_t b;
    std::memcpy(&b, &x, 4);
    return b - 0x4B400000;
}

float act_ref(float z, int act) {
    if (act == 1) return z < 0.0f ? 0.0f : z;
    const float c = std::sqrt(2.0f / static_cast<float>(3.14159265358979323846));
    const float t = (0.044715f * z) * z;
    const float inner = std::fma(z, t, z);
    const float th = std::tanh(c * inner);
    return (0.5f * z) * (1.0f + th);
}

float fq_code_ref(float v, float s, float zp) {
    float q = std::round(v / s) + zp;
    if (q < -128.0f) q = -128.0f;
    if (q > 127.0f) q = 127.0f;
    return q;
}

std::vector<float> build_act_table(float s, int zp, int act) {
    std::vector<float> t(256);
    const float zpf = static_cast<float>(zp);
    for (int k = -128; k <= 127; ++k) t[k + 128] = act_ref((static_cast<float>(k) - zpf) * s, act);
    return t;
}

bool build_code_lut(float s, int zp, int act, int max_cells, CodeLut& out, std::string& why,
                    bool allow_split) {
    if (!(s > 0.0f) || !std::isfinite(s)) {
        why = "scale must be positive and finite";
        return false;
    }
    const float zpf = static_cast<float>(zp);
    auto code = [&](float z) { return static_cast<int>(fq_code_ref(act_ref(z, act), s, zpf)); };

    // scan range: the negative branch of GELU is bounded below by -0.17, so every
    // breakpoint with z < 0 lies above -64; on the positive side codes saturate by
    // z = (128 - zp) * s (act(z) <= z there).
    const float zmin = -64.0f;
    const float zmax = std::fmax(64.0f, (129.0f - zpf) * s * 1.01f);
    if (code(zmin) != code(-1.0e30f)) {
        why = "activation does not settle below z = -64";
        return false;
    }
    const double h = std::fmin(0.25, 0.5 * s) / 64.0;  // far below the breakpoint spacing
    std::vector<Transition> tr;
    float prev_z = zmin;
    int prev_c = code(zmin);
    const int64_t nsteps = static_cast<int64_t>(std::ceil((zmax - zmin) / h));
    for (int64_t i = 1; i <= nsteps; ++i) {
        const float z = i == nsteps ? zmax : static_cast<float>(zmin + h * i);
        const int c = code(z);
        if (c != prev_c) {
            // bisection over consecutive floats: smallest z' in (prev_z, z] with code != prev_c
            int64_t lo = f2o(prev_z), hi = f2o(z);
            while (hi - lo > 1) {
                const int64_t mid = lo + (hi - lo) / 2;
                if (code(o2f(mid)) == prev_c) lo = mid;
                else hi = mid;
            }
            tr.push_back({o2f(hi), prev_c, c});
        }
        prev_z = z;
        prev_c = c;
    }
    if (code(zmax) != code(1.0e30f)) {
        why = "activation does not saturate within the scan range";
        return false;
    }
    for (const auto& t : tr) {
        if (std::abs(t.after - t.before) != 1) {
            why = "code jumps by more than one step between scan points";
            return false;
        }
    }
    if (tr.empty()) {
        out.zlo = 0.0f;
        out.inv_delta = 1.0f;
        out.zsplit = -std::numeric_limits<float>::infinity();
        out.inv0 = out.inv1 = 1.0f;
        out.c0 = out.c1 = 0.0f;
        out.alpha0 = out.alpha1 = out.beta0 = out.beta1 = 0.0f;
        out.nm1 = 0.0f;
        out.cells.assign(1, CodeCell{std::numeric_limits<float>::infinity(),
                                     (code(0.0f) & 0xFF) | ((code(0.0f) & 0xFF) << 8)});
        return true;
    }
    // Cells of one segment: [zlo + delta j, zlo + delta (j + 1)) widened by a margin of
    // delta / 64 on both sides, at most one breakpoint each.  The last cell of the last
    // segment is open to +inf.
    auto fill = [&](double zlo, double delta, int ncells, bool open_end,
                    std::vector<CodeCell>& cells) -> bool {
        const double margin = delta / 64.0;
        size_t first = 0;  // first transition not left of the current cell's range
        for (int j = 0; j < ncells; ++j) {
            const double a = zlo + delta * j - margin;
            const double b = (open_end && j == ncells - 1) ? 1e30 : zlo + delta * (j + 1) + margin;
            while (first < tr.size() && tr[first].t < a) ++first;
            const int base = first == 0 ? tr.front().before : tr[first - 1].after;
            CodeCell c{std::numeric_limits<float>::infinity(), 0};
            int d = 0;
            int n = 0;
            for (size_t k = first; k < tr.size() && tr[k].t < b; ++k) {
                if (n == 1) return false;
                c.t = tr[k].t;
                d = tr[k].after - tr[k].before;
                ++n;
            }
            c.packed = (base & 0xFF) | (((base + d) & 0xFF) << 8);
            cells.push_back(c);
        }
        return true;
    };
    // Every z is checked against the device's lookup (lut_index in numerics.cuh).
    auto self_check = [&](const CodeLut& L) -> bool {
        const int n = static_cast<int>(L.cells.size());
        const double lo_z = tr.front().t, hi_z = tr.back().t;
        uint32_t st = 12345u;
        for (int k = 0; k < 40000; ++k) {
            st = st * 1664525u + 1013904223u;
            float z = static_cast<float>(lo_z - 1.0 + (hi_z - lo_z + 2.0) * (st >> 8) / 16777216.0);
            if (k & 1) {  // half of the points next to a breakpoint or the split
                const float t = (k & 2) ? L.zsplit : tr[(st >> 3) % tr.size()].t;
                if (std::isfinite(t)) {
                    int32_t b;
                    std::memcpy(&b, &t, 4);
                    b += static_cast<int32_t>((st >> 11) % 9) - 4;
                    std::memcpy(&z, &b, 4);
                }
            }
            const bool s0 = z < L.zsplit;
            const float fi = std::fma(z, s0 ? L.inv0 : L.inv1, s0 ? L.c0 : L.c1);
            int idx = static_cast<int>(fi);
            if (fi < 0.0f) idx = 0;
            if (idx > n - 1) idx = n - 1;
            const int idx_sat = lut_index_sat(z, L);
            const CodeCell& cc = L.cells[idx];
            const CodeCell& cs = L.cells[idx_sat];
            const int got = static_cast<int8_t>(((z >= cc.t) ? (cc.packed >> 8) : cc.packed) & 0xFF);
            const int got_sat = static_cast<int8_t>(((z >= cs.t) ? (cs.packed >> 8) : cs.packed) & 0xFF);
            const int want = code(z);
            if (got != want || got_sat != want) {
                // accept only the flip windows of a few ulps around a breakpoint
                bool near = false;
                for (const auto& t : tr)
                    if (std::fabs(static_cast<double>(z) - t.t) <= 64.0 * std::fabs(next_up(t.t) - t.t))
                        near = true;
                if (!near) return false;
            }
        }
        return true;
    };
    // Largest cell size 2^-k (2 <= k < 26) for which the transitions in [zlo, zhi) fall
    // at most one per cell; 0 if none.
    const double delta0 = std::fmin(0.25, 0.5 * s);
    auto cell_size = [&](double zlo_t, double zhi_t) -> double {
        double gap = 1e30;
        float prev = 0.0f;
        bool have = false;
        for (const auto& t : tr) {
            if (t.t < zlo_t || t.t >= zhi_t) continue;
            if (have) gap = std::fmin(gap, static_cast<double>(t.t) - prev);
            prev = t.t;
            have = true;
        }
        double d = 0.25;
        for (int k = 0; k < 24; ++k, d *= 0.5)
            if (d * (1.0 + 1.0 / 16.0) < gap) return d;
        return 0.0;
    };

    const double lo_z = tr.front().t, hi_z = tr.back().t;
    // one segment: index fma(z, inv_delta, -zlo * inv_delta)
    for (double delta = delta0; delta > delta0 / 1024.0; delta *= 0.5) {
        const double zlo = lo_z - 2.0 * delta;
        const int ncells = static_cast<int>(std::ceil((hi_z - zlo) / delta)) + 2;
        if (ncells > max_cells) break;
        std::vector<CodeCell> cells;
        if (!fill(zlo, delta, ncells, true, cells)) continue;
        CodeLut L;
        L.zlo = static_cast<float>(zlo);
        L.inv_delta = static_cast<float>(1.0 / delta);
        L.zsplit = -std::numeric_limits<float>::infinity();
        L.inv0 = L.inv1 = L.inv_delta;
        L.c0 = L.c1 = -L.zlo * L.inv_delta;
        L.cells = std::move(cells);
        set_sat_params(L, zlo, delta, zlo, delta, 0);
        if (!self_check(L)) {
            why = "code table self-check failed";
            return false;
        }
        out = std::move(L);
        return true;
    }
    if (!allow_split) {
        why = "code table would need more than the allowed number of cells";
        return false;
    }
    // two segments, split in the middle of a gap between consecutive breakpoints: the
    // dense and the sparse side of the activation get their own cell size.
    int best_cells = max_cells + 1;
    double best_split = 0.0, best_d0 = 0.0, best_d1 = 0.0;
    for (size_t i = 0; i + 1 < tr.size(); ++i) {
        const double zs = 0.5 * (static_cast<double>(tr[i].t) + tr[i + 1].t);
        const double d0 = cell_size(-1e30, zs), d1 = cell_size(zs, 1e30);
        if (d0 <= 0.0 || d1 <= 0.0) continue;
        const double g = std::fmin(zs - tr[i].t, tr[i + 1].t - zs);
        if (g < 4.0 * std::fmax(d0, d1)) continue;  // keep the split well away from breakpoints
        const int n0 = static_cast<int>(std::ceil((zs - (lo_z - 2.0 * d0)) / d0)) + 2;
        const int n1 = static_cast<int>(std::ceil((hi_z - (zs - 2.0 * d1)) / d1)) + 2;
        if (n0 + n1 < best_cells) {
            best_cells = n0 + n1;
            best_split = zs;
            best_d0 = d0;
            best_d1 = d1;
        }
    }
    if (best_cells > max_cells) {
        why = "code table would need more than the allowed number of cells";
        return false;
    }
    {
        const float zs = static_cast<float>(best_split);
        const double zlo0 = lo_z - 2.0 * best_d0;
        const int n0 = static_cast<int>(std::ceil((static_cast<double>(zs) - zlo0) / best_d0)) + 2;
        const double zlo1 = static_cast<double>(zs) - 2.0 * best_d1;
        const int n1 = static_cast<int>(std::ceil((hi_z - zlo1) / best_d1)) + 2;
        std::vector<CodeCell> cells;
        if (!fill(zlo0, best_d0, n0, false, cells) || !fill(zlo1, best_d1, n1, true, cells)) {
            why = "no cell size gives at most one breakpoint per cell";
            return false;
        }
        CodeLut L;
        L.zlo = static_cast<float>(zlo0);
        L.inv_delta = 0.0f;  // not a one-segment table
        L.zsplit = zs;
        L.inv0 = static_cast<float>(1.0 / best_d0);
        L.c0 = -static_cast<float>(zlo0) * L.inv0;
        L.inv1 = static_cast<float>(1.0 / best_d1);
        L.c1 = static_cast<float>(n0) - static_cast<float>(zlo1) * L.inv1;
        L.cells = std::move(cells);
        set_sat_params(L, zlo0, best_d0, zlo1, best_d1, n0);
        if (!self_check(L)) {
            why = "code table self-check failed";
            return false;
        }
        out = std::move(L);
        return true;
    }
}

uint8_t e4m3_encode(float v) {
    if (std::isnan(v)) return 0x7F;
    if (std::isinf(v)) return v < 0.0f ? 0xFE : 0x7E;
    uint32_t u;
    std::memcpy(&u, &v, 4);
    const uint32_t sign = u >> 31, a = u & 0x7FFFFFFFu;
    if (a == 0) return static_cast<uint8_t>(sign << 7);
    const int e = static_cast<int>((a >> 23) & 0xFFu) - 120;
    if (e < 1) {
        float af;
        std::memcpy(&af, &a, 4);
        double r = std::nearbyint(static_cast<double>(af) * 512.0);
        r = r < 0.0 ? 0.0 : (r > 7.0 ? 7.0 : r);
        return static_cast<uint8_t>((sign << 7) | static_cast<uint32_t>(r));
    }
    uint32_t m = (a >> 20) & 7u;
    const uint32_t rest = a & 0xFFFFFu;
    if (rest > 0x80000u || (rest == 0x80000u && (m & 1u))) ++m;
    int ee = e;
    if (m & 8u) {
        m &= 7u;
        ++ee;
    }
    if (ee > 15) return static_cast<uint8_t>((sign << 7) | 0x7Eu);
    return static_cast<uint8_t>((sign << 7) | (static_cast<uint32_t>(ee) << 3) | m);
}

float e4m3_decode(uint8_t b) {
    const uint32_t sign = (b >> 7) & 1u, ex = (b >> 3) & 15u, mt = b & 7u;
    float v;
    if (ex == 15u && mt == 7u) {
        const uint32_t q = 0x7FC00000u | (sign << 31);
        std::memcpy(&v, &q, 4);
        return v;
    }
    if (ex == 0u) {
        v = std::ldexp(static_cast<float>(mt), -9);
        return sign ? -v : v;
    }
    const uint32_t u = (sign << 31) | ((ex + 120u) << 23) | (mt << 20);
    std::memcpy(&v, &u, 4);
    return v;
}

void e4m3_fake_quant(const float* in, float scale, float* xq, float* out, size_t n) {
    const float inv = scale == 0.0f ? 1.0f : 1.0f / scale;
    for (size_t i = 0; i < n; ++i) {
        float xs = in[i] * inv;
        xs = xs > 448.0f ? 448.0f : (xs < -448.0f ? -448.0f : xs);
        const float q = e4m3_decode(e4m3_encode(xs));
        if (xq) xq[i] = q;
        if (out) out[i] = q * scale;
    }
}

std::vector<float> build_fft_twiddles(int n, bool inverse) {
    std::vector<float> t(2 * static_cast<size_t>(n > 1 ? n - 1 : 0));
    const float pi = static_cast<float>(3.14159265358979323846);
    for (int len = 2; len <= n; len <<= 1) {
        const float ang = (inverse ? 2.0f : -2.0f) * pi / static_cast<float>(len);
        const float lr = std::cos(ang), li = std::sin(ang);
        float wr = 1.0f, wi = 0.0f;
        for (int k = 0; k < len / 2; ++k) {
            const size_t e = static_cast<size_t>(len / 2 - 1 + k);
            t[2 * e] = wr;
            t[2 * e + 1] = wi;
            const float nr = std::fma(wr, lr, -(wi * li));
            const float ni = std::fma(wr, li, wi * lr);
            wr = nr;
            wi = ni;
        }
    }
    return t;
}

}  // namespace nfx
