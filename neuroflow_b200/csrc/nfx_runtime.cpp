// nfx_runtime.cpp -- the runtime handle behind nfx_runtime_* (include/nfx.h): the
// device-side counterpart of the reference InferenceRuntime (runtime.cpp:21-171).
//
// Create loads the IR on the host, applies the load-time weight fake-quant
// (fno.cpp:997-1020 -> DequantiseWeight), and uploads the weights once.
// EnableInt8Gemm builds the per-channel weight codes (QuantiseWeight2D) and enables
// the INT8 executor.  Run/RunDevice validate shapes like FNO2d::Forward
// (fno.cpp:778-794) and launch the executor on the handle's device.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/nfx.h"
#include "fno1d.h"
#include "fno2d.h"
#include "fno3d.h"
#include "nfx_internal.h"
#include "nfx_ir.h"
#include "nfx_copy_pool.h"
#include "mlp_ops.h"
#include "nfx_lut.h"
#include "tm2d.h"

namespace nfx {
int set_thread_error(int code, const std::string& msg);
}

namespace nfx {
void fno2d_tables(int H, int W, int MH, int MW, float* fw, float* fh, float* iw, float* ih,
                  int8_t* limbs, long long* sum_b) {
    const double two_pi = 6.283185307179586476925286766559;
    for (int k = 0; k < MW; ++k)
        for (int w = 0; w < W; ++w) {
            const double a = two_pi * static_cast<double>((static_cast<int64_t>(k) * w) % W) / W;
            const double f = (k == 0 || 2 * k == W) ? 1.0 : 2.0;
            fw[2 * (k * W + w)] = static_cast<float>(std::cos(a));
            fw[2 * (k * W + w) + 1] = static_cast<float>(-std::sin(a));
            iw[2 * (k * W + w)] = static_cast<float>(f * std::cos(a) / W);
            iw[2 * (k * W + w) + 1] = static_cast<float>(f * std::sin(a) / W);
        }
    for (int h = 0; h < H; ++h)
        for (int k = 0; k < MH; ++k) {
            const double a = two_pi * static_cast<double>((static_cast<int64_t>(k) * h) % H) / H;
            fh[2 * (h * MH + k)] = static_cast<float>(std::cos(a));
            fh[2 * (h * MH + k) + 1] = static_cast<float>(-std::sin(a));
            ih[2 * (h * MH + k)] = static_cast<float>(std::cos(a) / H);
            ih[2 * (h * MH + k) + 1] = static_cast<float>(std::sin(a) / H);
        }
    if (!limbs || !sum_b || !fno2d_tc_forward(W, MW)) return;
    // integer DFT basis of the tensor-core forward transform: the basis scaled by 2^27
    // and rounded, split into four balanced base-256 digits
    std::memset(limbs, 0, kFno2dLimbBytes);
    for (int j = 0; j < 2 * MW; ++j) {
        const int kw = j / 2, n = j;  // basis row j of every digit matrix
        sum_b[j] = 0;
        for (int w = 0; w < W; ++w) {
            const double a = two_pi * static_cast<double>((static_cast<int64_t>(kw) * w) % W) / W;
            const double v = (j & 1) ? -std::sin(a) : std::cos(a);
            long long r = std::llround(v * 134217728.0);
            sum_b[j] += r;
            int dig[4];
            for (int l = 3; l >= 1; --l) {
                const long long d = ((r + 128) & 255) - 128;
                dig[l] = static_cast<int>(d);
                r = (r - d) / 256;
            }
            dig[0] = static_cast<int>(r);
            for (int l = 0; l < 4; ++l) limbs[(l * 32 + n) * 128 + w] = static_cast<int8_t>(dig[l]);
        }
    }
}
}  // namespace nfx

namespace nfx {
// Event-pair timer: begin/end record events on the launch stream; read() waits for
// them and folds the elapsed times into per-kernel totals.
struct EventTimer : KernelTimer {
    struct Pending {
        std::string name;
        cudaEvent_t a, b;
        bool shared_a;   // a is the previous entry's b (chained launches)
    };
    bool chain_on = false;
    cudaEvent_t last_end = nullptr;
    cudaStream_t last_stream = nullptr;
    std::vector<Pending> pending;
    std::vector<cudaEvent_t> pool;
    std::vector<std::string> names;
    std::vector<int> launches;
    std::vector<double> total_ms;
    cudaEvent_t take() {
        if (!pool.empty()) {
            cudaEvent_t e = pool.back();
            pool.pop_back();
            return e;
        }
        cudaEvent_t e = nullptr;
        cudaEventCreate(&e);
        return e;
    }
    void begin(const char* name, cudaStream_t s) override {
        const bool share = chain_on && last_end != nullptr && last_stream == s;
        Pending p{name, share ? last_end : take(), take(), share};
        if (!share) cudaEventRecord(p.a, s);
        last_end = nullptr;
        pending.push_back(p);
    }
    void end(cudaStream_t s) override {
        if (pending.empty()) return;
        cudaEventRecord(pending.back().b, s);
        last_end = pending.back().b;
        last_stream = s;
    }
    void chain(bool on) override {
        chain_on = on;
        last_end = nullptr;
    }
    void collect() {
        for (auto& p : pending) {
            cudaEventSynchronize(p.b);
            float ms = 0.f;
            cudaEventElapsedTime(&ms, p.a, p.b);
            size_t i = 0;
            while (i < names.size() && names[i] != p.name) ++i;
            if (i == names.size()) {
                names.push_back(p.name);
                launches.push_back(0);
                total_ms.push_back(0.0);
            }
            launches[i] += 1;
            total_ms[i] += ms;
            if (!p.shared_a) pool.push_back(p.a);
            pool.push_back(p.b);
        }
        pending.clear();
        last_end = nullptr;
    }
    void reset() {
        collect();
        names.clear();
        launches.clear();
        total_ms.clear();
    }
    ~EventTimer() override {
        for (auto& p : pending) {
            if (!p.shared_a) cudaEventDestroy(p.a);
            cudaEventDestroy(p.b);
        }
        for (auto e : pool) cudaEventDestroy(e);
    }
};
}  // namespace nfx

struct nfx_runtime {
    int device = 0;
    nfx::IrModel model;
    std::string err;
    bool int8_enabled = false;
    cudaStream_t stream = nullptr;  // used by the synchronous host-buffer Run
    // host-buffer Run of a large batch: copies on their own streams, overlapped with
    // the compute of neighbouring batch chunks
    cudaStream_t s_h2d = nullptr, s_d2h = nullptr;
    cudaEvent_t ev_in[8] = {}, ev_out[8] = {}, ev_done[8] = {};
    // pageable caller buffers: pinned staging copies of x and y, filled and drained by
    // a pool of host copy threads while the GPU works on neighbouring chunks
    float* hx = nullptr;
    float* hy = nullptr;
    size_t hx_cap = 0, hy_cap = 0;
    std::unique_ptr<nfx::CopyPool> pool;
    std::vector<void*> allocs;      // weights and tables (freed at destroy)
    // FNO2d state
    nfx::Fno2dPlan plan{};
    int max_B = 0;                  // capacity of the activation buffers
    int buf_H = 0, buf_W = 0;
    void* act_bufs[4] = {nullptr, nullptr, nullptr, nullptr};
    float* dx = nullptr;            // host-Run staging (device side)
    float* dy = nullptr;
    size_t dx_cap = 0, dy_cap = 0;
    float2* tw[4] = {nullptr, nullptr, nullptr, nullptr};  // twf_w, twf_h, twi_w, twi_h
    int tw_H = 0, tw_W = 0;
    int8_t* fwd_limbs = nullptr;      // tensor-core forward basis digits (W == 128)
    long long* fwd_sum_b = nullptr;
    int8_t* tap_codes = nullptr;      // caller's parity-tap buffer (nfx_runtime_set_code_taps)
    int64_t tap_cap = 0;
    // GPU calibration (nfx_calibrate_*): range keys of every observed Linear output,
    // and, when values are kept, one device chunk per tensor and observed batch
    unsigned* calib_stats = nullptr;
    int calib_keep = 0;
    std::vector<std::vector<std::pair<float*, int64_t>>> calib_vals;
    // FNO2d FP32 (reference fake-quant) state; plan2i: the same kernels running the
    // INT8 composition where the width-64 executor does not apply (f2_fast false, or a
    // grid outside its range)
    nfx::Fno2dF32Plan plan2f{};
    nfx::Fno2dF32Plan plan2i{};
    bool f2_fast = false;
    void* f2_bufs[4] = {nullptr, nullptr, nullptr, nullptr};  // h0, h1, Xs, colinv
    int64_t f2_cap[4] = {0, 0, 0, 0};
    float2* f2_tw[4] = {nullptr, nullptr, nullptr, nullptr};   // fwd W, inv W, fwd H, inv H
    int f2_tw_H = 0, f2_tw_W = 0;
    // FNO3d state
    nfx::Fno3dPlan plan3{};
    bool fp8_enabled = false;
    void* f3_bufs[6] = {};           // h0, h1, A, Xs, colinv, x1
    int64_t f3_cap[6] = {};
    float2* f3_tw[6] = {};
    int f3_tw_dims[3] = {0, 0, 0};
    float* f3_dft = nullptr;         // direct-DFT tables of the FP8 width-32/64 variant
    int f3_dft_key[4] = {0, 0, 0, 0};
    // TokenMixer2D state
    nfx::Tm2dPlan plan_tm{};
    void* tm_bufs[13] = {};
    int64_t tm_cap_T = 0, tm_cap_P = 0;
    // DeepONet / GraphOp / GraphOp2D state (mlp_ops.h): the layer chains with their
    // device weights; `mo_why` is why Run refuses the model (empty: runnable)
    nfx::MlpArgs mo_branch{}, mo_trunk{}, mo_lift{}, mo_head{};
    nfx::GraphLayerArgs mo_blocks[nfx::kMlpMaxLayers] = {};
    const float* mo_bias = nullptr;
    int mo_nodes = 0, mo_layers = 0, mo_code = 0;
    std::string mo_why;
    void* mo_bufs[2] = {nullptr, nullptr};
    int64_t mo_cap[2] = {0, 0};
    // FNO1d state
    nfx::Fno1dPlan plan1{};
    int pt_n[nfx::kFno1dMaxLayers] = {};   // per-token table sizes (locs.i.output)
    int pt_w[nfx::kFno1dMaxLayers] = {};
    void* f1_bufs[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};  // h0, h1, Xs, x2raw, x1f
    int64_t f1_cap_BN = 0;                // B * N the buffers hold
    float2* f1_tw[2] = {nullptr, nullptr};
    int f1_tw_N = 0;
    std::unique_ptr<nfx::EventTimer> timer;  // per-kernel timing when enabled
};

namespace {

int rt_fail(nfx_runtime* rt, int code, const std::string& m) {
    if (rt) rt->err = m;
    return code;
}

bool cuda_ok(nfx_runtime* rt, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return true;
    rt->err = std::string(what) + ": " + cudaGetErrorString(e);
    return false;
}

template <typename T>
T* upload(nfx_runtime* rt, const T* host, size_t count) {
    void* p = nullptr;
    if (cudaMalloc(&p, count * sizeof(T) + 16) != cudaSuccess) return nullptr;
    rt->allocs.push_back(p);
    if (count && cudaMemcpy(p, host, count * sizeof(T), cudaMemcpyHostToDevice) != cudaSuccess)
        return nullptr;
    return static_cast<T*>(p);
}

nfx::FqParam fq_for(const nfx::IrModel& m, const std::string& key) {
    nfx::FqParam f{0, 1.0f, 0, 1.0f};
    if (!m.quant_enabled) return f;
    auto it8 = m.activation_fp8_qparams.find(key);
    if (it8 != m.activation_fp8_qparams.end()) {
        f.kind = 2;
        f.scale = it8->second;
        return f;
    }
    auto it = m.activation_qparams.find(key);
    if (it != m.activation_qparams.end()) {
        f.kind = 1;
        f.scale = it->second.scale;
        f.zp = it->second.zero_point;
        f.inv_scale = 1.0f / f.scale;
    }
    return f;
}

const float* wptr(nfx_runtime* rt, const std::string& name) {
    const auto& t = rt->model.weights.at(name);
    return upload(rt, t.data.data(), t.data.size());
}

// FNO2d config block (ir_loader.h:147-155)
struct F2 {
    int in_ch, out_ch, width, mh, mw, L, pad;
};
F2 fno2d_cfg(const nfx::IrModel& m) {
    return F2{m.cfg[0], m.cfg[1], m.cfg[2], m.cfg[3], m.cfg[4], m.cfg[5], m.cfg[6]};
}

// The FP32 fake-quant plan (fno2d_fp32.cu): weights as the reference holds them after
// Create, and the four ".output" fake-quant boundaries of FNO2d::Forward.
int fno2d_f32_create(nfx_runtime* rt) {
    auto& m = rt->model;
    const F2 c = fno2d_cfg(m);
    auto& pl = rt->plan2f;
    if (c.L > nfx::kFno2dMaxLayers || c.in_ch < 1) return NFX_OK;  // Run reports it
    pl.C = c.width;
    pl.MH = c.mh;
    pl.MW = c.mw;
    pl.L = c.L;
    pl.in_ch = c.in_ch;
    pl.out_ch = c.out_ch;
    pl.act = m.activation == "relu" ? 1 : 0;
    pl.lift_w = wptr(rt, "lift.weight");
    pl.lift_b = wptr(rt, "lift.bias");
    pl.pq_w = wptr(rt, "proj_q.weight");
    pl.pq_b = wptr(rt, "proj_q.bias");
    pl.po_w = wptr(rt, "proj_out.weight");
    pl.po_b = wptr(rt, "proj_out.bias");
    pl.fq_lift = fq_for(m, "lift.output");
    pl.fq_pq = fq_for(m, "proj_q.output");
    pl.fq_po = fq_for(m, "proj_out.output");
    if (!pl.lift_w || !pl.lift_b || !pl.pq_w || !pl.pq_b || !pl.po_w || !pl.po_b)
        return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    for (int i = 0; i < c.L; ++i) {
        const std::string s = std::to_string(i);
        auto& L = pl.layer[i];
        L.wr = wptr(rt, "specs." + s + ".weights_real");
        L.wi = wptr(rt, "specs." + s + ".weights_imag");
        L.loc_w = wptr(rt, "locs." + s + ".weight");
        L.loc_b = wptr(rt, "locs." + s + ".bias");
        L.fq = fq_for(m, "locs." + s + ".output");
        if (!L.wr || !L.wi || !L.loc_w || !L.loc_b) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    }
    return NFX_OK;
}

int fno2d_create(nfx_runtime* rt) {
    auto& m = rt->model;
    const F2 c = fno2d_cfg(m);
    if (m.quant_enabled) {
        for (const auto& name : m.weight_order) nfx::dequantise_weight(m.weights[name], m, name);
    }
    int s0 = fno2d_f32_create(rt);
    if (s0 != NFX_OK) return s0;
    if (!nfx::fno2d_supported(c.width, c.mh, c.mw)) return NFX_OK;  // INT8 path unavailable
    auto& pl = rt->plan;
    pl.C = c.width;
    pl.MH = c.mh;
    pl.MW = c.mw;
    pl.L = c.L;
    pl.in_ch = c.in_ch;
    pl.lift_w = wptr(rt, "lift.weight");
    pl.lift_b = wptr(rt, "lift.bias");
    if (!pl.lift_w || !pl.lift_b) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    for (int i = 0; i < c.L && i < nfx::kFno2dMaxLayers; ++i) {
        // spectral weights (in, out, mh, mw) real/imag -> [mode][in][out] complex
        const auto& wr = m.weights.at("specs." + std::to_string(i) + ".weights_real");
        const auto& wi = m.weights.at("specs." + std::to_string(i) + ".weights_imag");
        const int C = c.width, M = c.mh * c.mw;
        std::vector<float> packed(static_cast<size_t>(M) * C * C * 2);
        for (int in = 0; in < C; ++in)
            for (int o = 0; o < C; ++o)
                for (int md = 0; md < M; ++md) {
                    const size_t src = (static_cast<size_t>(in) * C + o) * M + md;
                    const size_t dst = ((static_cast<size_t>(md) * C + in) * C + o) * 2;
                    packed[dst] = wr.data[src];
                    packed[dst + 1] = wi.data[src];
                }
        pl.layer[i].wspec = reinterpret_cast<const float2*>(upload(rt, packed.data(), packed.size()));
        pl.layer[i].wmix_hi = nullptr;
        pl.layer[i].wmix_lo = nullptr;
        if (C == 64) {
            // per mode the real form of y = x W (x, y complex rows): row n = 2 o + ri_out,
            // column k = 2 in + ri_in; tf32 split as the device's split_tf32
            const int K = 2 * C;
            std::vector<float> hi(static_cast<size_t>(M) * K * K), lo(hi.size());
            auto split = [](float x, float& h, float& l) {
                uint32_t u;
                std::memcpy(&u, &x, 4);
                u = (u + 0x1000u) & 0xFFFFE000u;
                std::memcpy(&h, &u, 4);
                l = x - h;
            };
            for (int md = 0; md < M; ++md)
                for (int in = 0; in < C; ++in)
                    for (int o = 0; o < C; ++o) {
                        const size_t src = (static_cast<size_t>(in) * C + o) * M + md;
                        const float r = wr.data[src], im = wi.data[src];
                        const float v[2][2] = {{r, im}, {-im, r}};  // [ri_in][ri_out]
                        for (int a2 = 0; a2 < 2; ++a2)
                            for (int b2 = 0; b2 < 2; ++b2) {
                                const size_t d = (static_cast<size_t>(md) * K + 2 * o + b2) * K + 2 * in + a2;
                                split(v[a2][b2], hi[d], lo[d]);
                            }
                    }
            pl.layer[i].wmix_hi = upload(rt, hi.data(), hi.size());
            pl.layer[i].wmix_lo = upload(rt, lo.data(), lo.size());
            if (!pl.layer[i].wmix_hi || !pl.layer[i].wmix_lo) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
        }
        auto& a = pl.layer[i].args;
        a.bias = wptr(rt, "locs." + std::to_string(i) + ".bias");
        if (!pl.layer[i].wspec || !a.bias) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    }
    pl.proj.bias = wptr(rt, "proj_q.bias");
    pl.proj.w_out = wptr(rt, "proj_out.weight");
    pl.proj.b_out = wptr(rt, "proj_out.bias");
    pl.proj.out_ch = c.out_ch;
    if (!pl.proj.bias || !pl.proj.w_out || !pl.proj.b_out)
        return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    return NFX_OK;
}

// The INT8 composition on the FP32 executor's kernels (plan2i), for any geometry that
// executor runs.  Per layer, as the composition defines it: the layer input is
// snapped with its key's per-tensor INT8 qparams when they exist (lift.output for
// layer 0, locs.{i-1}.output after), and locs.i / proj_q run LinearForwardBatched
// when the weight has per-channel axis-0 qparams and the input key per-tensor ones.
bool fno2d_i8_generic(nfx_runtime* rt) {
    auto& m = rt->model;
    const F2 c = fno2d_cfg(m);
    if (!rt->plan2f.lift_w) return false;
    nfx::Fno2dF32Plan pl = rt->plan2f;
    const int act = pl.act;
    auto in_qp = [&](int i, nfx::QP& q) {
        auto it = m.activation_qparams.find(i == 0 ? std::string("lift.output")
                                                   : "locs." + std::to_string(i - 1) + ".output");
        if (it == m.activation_qparams.end()) return false;
        q = it->second;
        return true;
    };
    auto fq1 = [](const nfx::QP& q) { return nfx::FqParam{1, q.scale, q.zero_point, 1.0f / q.scale}; };
    const nfx::FqParam none{0, 1.0f, 0, 1.0f};
    // i in [0, L]: layer i's local Linear, i == L proj_q
    auto linear = [&](int i, nfx::Fno2dI8Linear& out) -> bool {
        out = nfx::Fno2dI8Linear{nullptr, nullptr, 1.0f, 0};
        const std::string wname = i < c.L ? "locs." + std::to_string(i) + ".weight" : "proj_q.weight";
        nfx::QP in;
        auto pc = m.weight_per_channel_qparams.find(wname);
        if (pc == m.weight_per_channel_qparams.end() || !in_qp(i, in)) return true;  // FP32 Linear
        std::vector<int8_t> codes;
        std::vector<int32_t> sum_w;
        if (!nfx::quantise_weight_2d(m.weights.at(wname), pc->second, codes, sum_w)) return true;
        const int C = c.width;
        if (static_cast<int>(codes.size()) != C * C || static_cast<int>(pc->second.zero_points.size()) < C)
            return true;
        std::vector<float> wz(codes.size());
        std::vector<int32_t> cols(static_cast<size_t>(4) * C, 0);
        for (int o = 0; o < C; ++o) {
            const int32_t zpw = pc->second.zero_points[o];
            for (int k = 0; k < C; ++k)
                wz[static_cast<size_t>(o) * C + k] = static_cast<float>(codes[static_cast<size_t>(o) * C + k] - zpw);
            const float sws = pc->second.scales[o] * in.scale;
            std::memcpy(&cols[4 * o], &sws, 4);
            cols[4 * o + 1] = zpw;
            cols[4 * o + 2] = C * zpw * in.zero_point - in.zero_point * sum_w[o];
        }
        out.wz = upload(rt, wz.data(), wz.size());
        out.cols = reinterpret_cast<const int4*>(upload(rt, cols.data(), cols.size()));
        out.s_in = in.scale;
        out.zp_in = in.zero_point;
        return out.wz && out.cols;
    };
    auto snap = [&](const nfx::QP& q, nfx::Fno2dSnap& out) -> bool {
        out = nfx::Fno2dSnap{fq1(q), nullptr, 0, 0.0f, 0.0f};
        nfx::CodeLut lut;
        std::string why;
        if (nfx::build_code_lut(q.scale, q.zero_point, act, 1 << 15, lut, why)) {
            out.code_lut = reinterpret_cast<const int2*>(upload(rt, lut.cells.data(), lut.cells.size()));
            if (!out.code_lut) return false;
            out.lut_cells = static_cast<int>(lut.cells.size());
            out.lut_zlo = lut.zlo;
            out.lut_inv_delta = lut.inv_delta;
        }
        return true;
    };
    nfx::QP q;
    pl.snap_lift = in_qp(0, q) ? fq1(q) : none;
    for (int i = 0; i <= c.L; ++i) {
        nfx::Fno2dI8Linear& li = i < c.L ? pl.layer[i].i8 : pl.pq_i8;
        if (!linear(i, li)) return false;
    }
    for (int i = 0; i < c.L; ++i) {
        pl.layer[i].snap = nfx::Fno2dSnap{none, nullptr, 0, 0.0f, 0.0f};
        // the next layer's input snap; after the last layer only proj_q's own
        // quantisation, which the snapped value reproduces (the snap is idempotent)
        const bool want = i + 1 < c.L ? in_qp(i + 1, q) : (pl.pq_i8.wz != nullptr && in_qp(c.L, q));
        if (want && !snap(q, pl.layer[i].snap)) return false;
    }
    pl.pq_act_table = nullptr;
    if (pl.fq_pq.kind == 1) {
        const std::vector<float> t = nfx::build_act_table(pl.fq_pq.scale, pl.fq_pq.zp, act);
        pl.pq_act_table = upload(rt, t.data(), t.size());
        if (!pl.pq_act_table) return false;
    }
    rt->plan2i = pl;
    return true;
}

bool fno2d_i8_fast(nfx_runtime* rt);

// EnableInt8Gemm for FNO2d.  The INT8 composition runs on every geometry through
// plan2i; the width-64 executor (plan, f2_fast) takes it over when every locs.i and
// proj_q has per-channel (axis 0) weight qparams and every layer input key per-tensor
// INT8 activation qparams.
void fno2d_enable_int8(nfx_runtime* rt) {
    if (!rt->model.quant_enabled || !fno2d_i8_generic(rt)) return;
    rt->int8_enabled = true;
    rt->f2_fast = fno2d_i8_fast(rt);
}

bool fno2d_i8_fast(nfx_runtime* rt) {
    auto& m = rt->model;
    const F2 c = fno2d_cfg(m);
    if (!m.quant_enabled || !nfx::fno2d_supported(c.width, c.mh, c.mw) || c.L > nfx::kFno2dMaxLayers)
        return false;
    if (c.out_ch < 1 || c.out_ch > 4 || c.in_ch < 1 || c.in_ch > 8) return false;
    auto act_key = [](int i) { return i == 0 ? std::string("lift.output")
                                             : "locs." + std::to_string(i - 1) + ".output"; };
    for (int i = 0; i <= c.L; ++i) {
        if (!m.activation_qparams.count(act_key(i))) return false;
        if (m.activation_fp8_qparams.count(act_key(i))) return false;
    }
    auto& pl = rt->plan;
    for (int i = 0; i <= c.L; ++i) {
        const std::string wname = i < c.L ? "locs." + std::to_string(i) + ".weight" : "proj_q.weight";
        auto pc = m.weight_per_channel_qparams.find(wname);
        if (pc == m.weight_per_channel_qparams.end()) return false;
        std::vector<int8_t> codes;
        std::vector<int32_t> sum_w;
        if (!nfx::quantise_weight_2d(m.weights.at(wname), pc->second, codes, sum_w)) return false;
        if (static_cast<int>(codes.size()) != c.width * c.width) return false;
        nfx::LayerArgs& a = i < c.L ? pl.layer[i].args : pl.proj;
        a.Wq = upload(rt, codes.data(), codes.size());
        a.scale_w = upload(rt, pc->second.scales.data(), static_cast<size_t>(c.width));
        a.zp_w = upload(rt, pc->second.zero_points.data(), static_cast<size_t>(c.width));
        a.sum_w = upload(rt, sum_w.data(), sum_w.size());
        if (!a.Wq || !a.scale_w || !a.zp_w || !a.sum_w) return false;
        {
            // -2 zp_w (in [-254, 256]) as up to three int8 parts per output channel
            std::vector<int8_t> zr(static_cast<size_t>(3) * c.width * 32, 0);
            a.nz = 2;
            for (int o = 0; o < c.width; ++o) {
                const int v = -2 * pc->second.zero_points[o];
                const int z0 = std::min(127, std::max(-128, v));
                const int z1 = std::min(127, std::max(-128, v - z0));
                const int z2 = v - z0 - z1;
                if (z2 != 0) a.nz = 3;
                const int zp3[3] = {z0, z1, z2};
                for (int q = 0; q < 3; ++q)
                    for (int k = 0; k < 32; ++k)
                        zr[(static_cast<size_t>(q) * c.width + o) * 32 + k] = static_cast<int8_t>(zp3[q]);
            }
            a.zrows = upload(rt, zr.data(), zr.size());
            if (!a.zrows) return false;
        }
        const nfx::QP in = m.activation_qparams.at(act_key(i));
        a.s_in = in.scale;
        a.zp_in = in.zero_point;
        a.act = m.activation == "relu" ? 1 : 0;
        if (i < c.L) {
            pl.layer[i].s_in = in.scale;
            pl.layer[i].zp_in = in.zero_point;
            a.fq_out = fq_for(m, "locs." + std::to_string(i) + ".output");
            // exact z -> next-code table (falls back to direct evaluation when absent)
            nfx::CodeLut lut;
            std::string why;
            a.code_lut = nullptr;
            a.lut_cells = 0;
            a.lut_two = 0;
            if (nfx::build_code_lut(a.fq_out.scale, a.fq_out.zp, a.act, nfx::kFno2dLutCells, lut, why, true)) {
                a.code_lut = reinterpret_cast<const int2*>(upload(rt, lut.cells.data(), lut.cells.size()));
                if (a.code_lut) {
                    a.lut_cells = static_cast<int>(lut.cells.size());
                    a.lut_zlo = lut.zlo;
                    a.lut_inv_delta = lut.inv_delta;
                    a.lut_two = std::isfinite(lut.zsplit) ? 1 : 0;
                    a.lut_split = lut.zsplit;
                    a.lut_inv0 = lut.inv0;
                    a.lut_c0 = lut.c0;
                    a.lut_inv1 = lut.inv1;
                    a.lut_c1 = lut.c1;
                    a.lut_alpha0 = lut.alpha0;
                    a.lut_beta0 = lut.beta0;
                    a.lut_alpha1 = lut.alpha1;
                    a.lut_beta1 = lut.beta1;
                    a.lut_nm1 = lut.nm1;
                }
            }
            // the W == 128 kernel's table: one segment when up to kFno2dLutCellsTc cells do
            pl.layer[i].args_tc = a;
            if (a.lut_two) {
                nfx::CodeLut lut1;
                std::string why1;
                if (nfx::build_code_lut(a.fq_out.scale, a.fq_out.zp, a.act, nfx::kFno2dLutCellsTc, lut1,
                                        why1, false)) {
                    nfx::LayerArgs& t = pl.layer[i].args_tc;
                    t.code_lut = reinterpret_cast<const int2*>(upload(rt, lut1.cells.data(), lut1.cells.size()));
                    if (t.code_lut) {
                        t.lut_cells = static_cast<int>(lut1.cells.size());
                        t.lut_zlo = lut1.zlo;
                        t.lut_inv_delta = lut1.inv_delta;
                        t.lut_two = 0;
                        t.lut_split = lut1.zsplit;
                        t.lut_inv0 = lut1.inv0;
                        t.lut_c0 = lut1.c0;
                        t.lut_inv1 = lut1.inv1;
                        t.lut_c1 = lut1.c1;
                        t.lut_alpha0 = lut1.alpha0;
                        t.lut_beta0 = lut1.beta0;
                        t.lut_alpha1 = lut1.alpha1;
                        t.lut_beta1 = lut1.beta1;
                        t.lut_nm1 = lut1.nm1;
                    } else {
                        t = a;
                    }
                }
            }
            // epilogue constants (the device's former per-element shared loads)
            nfx::LayerCols& cols = pl.layer[i].cols;
            const std::vector<float>& bias = m.weights.at("locs." + std::to_string(i) + ".bias").data;
            for (int o = 0; o < c.width && o < nfx::kFno2dColMax; ++o) {
                const int32_t zp = pc->second.zero_points[o];
                const int32_t nk = in.zero_point * (c.width * zp - sum_w[o]);
                float zpf, nkf;
                std::memcpy(&zpf, &zp, 4);
                std::memcpy(&nkf, &nk, 4);
                cols.v[o] = make_float4(pc->second.scales[o] * in.scale, zpf, nkf, bias[o]);
                cols.a[o] = cols.v[o].x;
                cols.nk[o] = nk;
                cols.b[o] = bias[o];
            }
        } else {
            nfx::ProjCols& cols = pl.proj_cols;
            const std::vector<float>& wo = m.weights.at("proj_out.weight").data;  // (out_ch, C)
            const std::vector<float>& bo = m.weights.at("proj_out.bias").data;
            for (int j = 0; j < 4; ++j) {
                cols.bout[j] = j < c.out_ch ? bo[j] : 0.0f;
                for (int o = 0; o < nfx::kFno2dColMax; ++o)
                    cols.wout[j][o] = (j < c.out_ch && o < c.width) ? wo[static_cast<size_t>(j) * c.width + o] : 0.0f;
            }
            const std::vector<float>& bias = m.weights.at("proj_q.bias").data;
            for (int o = 0; o < c.width && o < nfx::kFno2dColMax; ++o) {
                const int32_t zp = pc->second.zero_points[o];
                const int32_t nk = -(in.zero_point * sum_w[o]);
                float zpf, nkf;
                std::memcpy(&zpf, &zp, 4);
                std::memcpy(&nkf, &nk, 4);
                cols.v[o] = make_float4(pc->second.scales[o] * in.scale, zpf, nkf, bias[o]);
            }
            a.fq_out = fq_for(m, "proj_q.output");
            a.fq_final = fq_for(m, "proj_out.output");
            a.act_table = nullptr;
            if (a.fq_out.kind == 1) {
                const std::vector<float> t = nfx::build_act_table(a.fq_out.scale, a.fq_out.zp, a.act);
                a.act_table = upload(rt, t.data(), t.size());
            }
        }
    }
    const nfx::QP lq = m.activation_qparams.at("lift.output");
    pl.lift_s = lq.scale;
    pl.lift_zp = lq.zero_point;
    pl.lift_inv_s = 1.0f / lq.scale;
    {
        const std::vector<float>& lw = m.weights.at("lift.weight").data;  // (C, in_ch)
        const std::vector<float>& lb = m.weights.at("lift.bias").data;
        pl.lift_cols = nfx::LiftCols{};
        for (int o = 0; o < c.width && o < nfx::kFno2dColMax; ++o) {
            pl.lift_cols.b[o] = lb[o];
            for (int k = 0; k < c.in_ch && k < nfx::kFno2dLiftInMax; ++k)
                pl.lift_cols.w[o][k] = lw[static_cast<size_t>(o) * c.in_ch + k];
        }
    }
    return true;
}

// Twiddle tables in double precision, rounded once to float (fno2d_tables).
int ensure_twiddles(nfx_runtime* rt, int H, int W) {
    if (rt->tw_H == H && rt->tw_W == W) return NFX_OK;
    const int MH = rt->plan.MH, MW = rt->plan.MW;
    std::vector<float> fw(2 * MW * W), fh(2 * H * MH), iw(2 * MW * W), ih(2 * H * MH);
    const bool tc = nfx::fno2d_tc_forward(W, MW);
    std::vector<int8_t> limbs(tc ? nfx::kFno2dLimbBytes : 0);
    std::vector<long long> sum_b(tc ? 2 * MW : 0);
    nfx::fno2d_tables(H, W, MH, MW, fw.data(), fh.data(), iw.data(), ih.data(),
                      tc ? limbs.data() : nullptr, tc ? sum_b.data() : nullptr);
    for (auto*& p : rt->tw) {
        if (p) cudaFree(p);
        p = nullptr;
    }
    const std::vector<float>* src[4] = {&fw, &fh, &iw, &ih};
    for (int i = 0; i < 4; ++i) {
        void* p = nullptr;
        if (!cuda_ok(rt, cudaMalloc(&p, src[i]->size() * 4), "cudaMalloc")) return NFX_INTERNAL;
        rt->tw[i] = static_cast<float2*>(p);
        if (!cuda_ok(rt, cudaMemcpy(p, src[i]->data(), src[i]->size() * 4, cudaMemcpyHostToDevice),
                     "cudaMemcpy"))
            return NFX_INTERNAL;
    }
    if (rt->fwd_limbs) cudaFree(rt->fwd_limbs);
    if (rt->fwd_sum_b) cudaFree(rt->fwd_sum_b);
    rt->fwd_limbs = nullptr;
    rt->fwd_sum_b = nullptr;
    if (tc) {
        void* p1 = nullptr;
        void* p2 = nullptr;
        if (!cuda_ok(rt, cudaMalloc(&p1, limbs.size()), "cudaMalloc") ||
            !cuda_ok(rt, cudaMalloc(&p2, sum_b.size() * sizeof(long long)), "cudaMalloc"))
            return NFX_INTERNAL;
        rt->fwd_limbs = static_cast<int8_t*>(p1);
        rt->fwd_sum_b = static_cast<long long*>(p2);
        if (!cuda_ok(rt, cudaMemcpy(p1, limbs.data(), limbs.size(), cudaMemcpyHostToDevice), "cudaMemcpy") ||
            !cuda_ok(rt, cudaMemcpy(p2, sum_b.data(), sum_b.size() * sizeof(long long),
                                    cudaMemcpyHostToDevice), "cudaMemcpy"))
            return NFX_INTERNAL;
    }
    rt->tw_H = H;
    rt->tw_W = W;
    return NFX_OK;
}

int ensure_buffers(nfx_runtime* rt, int B, int H, int W) {
    if (B <= rt->max_B && H == rt->buf_H && W == rt->buf_W) return NFX_OK;
    for (auto*& p : rt->act_bufs) {
        if (p) cudaFree(p);
        p = nullptr;
    }
    const auto& pl = rt->plan;
    const size_t M = static_cast<size_t>(B) * H * W;
    const int nHB = nfx::fno2d_row_blocks(H);
    const size_t sizes[4] = {M * pl.C, M * pl.C,
                             static_cast<size_t>(B) * nHB * pl.MH * pl.MW * pl.C * sizeof(float2),
                             static_cast<size_t>(B) * pl.MH * pl.MW * pl.C * sizeof(float2)};
    for (int i = 0; i < 4; ++i)
        if (!cuda_ok(rt, cudaMalloc(&rt->act_bufs[i], sizes[i] + 256), "cudaMalloc activations"))
            return NFX_INTERNAL;
    rt->max_B = B;
    rt->buf_H = H;
    rt->buf_W = W;
    return NFX_OK;
}

int check_fno2d_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    const F2 c = fno2d_cfg(rt->model);
    if (xr != 4) return rt_fail(rt, NFX_SHAPE_MISMATCH, "expected 4D input (batch, h, w, in_ch)");
    if (xs[3] != c.in_ch) return rt_fail(rt, NFX_SHAPE_MISMATCH, "input channels mismatch");
    if (yr != 4 || ys[0] != xs[0] || ys[1] != xs[1] || ys[2] != xs[2] || ys[3] != c.out_ch)
        return rt_fail(rt, NFX_SHAPE_MISMATCH, "output buffer shape mismatch");
    auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
    if (!pow2(xs[1]) || !pow2(xs[2]))
        return rt_fail(rt, NFX_INVALID_ARG, "FNO2d: H and W must each be a power of two");
    return NFX_OK;
}

int ensure_f2_buf(nfx_runtime* rt, int i, int64_t bytes) {
    if (bytes <= rt->f2_cap[i]) return NFX_OK;
    if (rt->f2_bufs[i]) cudaFree(rt->f2_bufs[i]);
    rt->f2_bufs[i] = nullptr;
    rt->f2_cap[i] = 0;
    if (!cuda_ok(rt, cudaMalloc(&rt->f2_bufs[i], static_cast<size_t>(bytes) + 256), "cudaMalloc activations"))
        return NFX_INTERNAL;
    rt->f2_cap[i] = bytes;
    return NFX_OK;
}

// FNO2d without EnableInt8Gemm: the reference's FP32 fake-quant network.  With `obs`
// (calibration), the Linear outputs are observed and no fake-quant is applied.  After
// EnableInt8Gemm the same kernels run the INT8 composition (plan2i).
int fno2d_f32_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st,
                     unsigned* obs = nullptr, float* const* obs_vals = nullptr) {
    const F2 c = fno2d_cfg(rt->model);
    auto& pl0 = rt->int8_enabled && !obs ? rt->plan2i : rt->plan2f;
    if (!pl0.lift_w)
        return rt_fail(rt, NFX_UNSUPPORTED_OP, "FNO2d GPU executor: needs <= 8 layers");
    const int B = static_cast<int>(xs[0]), H = static_cast<int>(xs[1]), W = static_cast<int>(xs[2]);
    int Hp = H, Wp = W;
    if (c.pad > 1) {
        Hp = H + (c.pad - H % c.pad) % c.pad;
        Wp = W + (c.pad - W % c.pad) % c.pad;
    }
    if ((Hp & (Hp - 1)) || (Wp & (Wp - 1)))
        return rt_fail(rt, NFX_INVALID_ARG, "FNO2d: padded H and W must be powers of two");
    if (c.mh > Hp || c.mw > Wp / 2 + 1)
        return rt_fail(rt, NFX_INVALID_ARG, "FNO2d: modes exceed the (padded) grid");
    if (const char* why = nfx::fno2d_f32_unsupported(c.width, c.mh, c.mw, Hp, Wp, c.out_ch))
        return rt_fail(rt, NFX_UNSUPPORTED_OP, why);
    if (B == 0) return NFX_OK;
    if (rt->f2_tw_H != Hp || rt->f2_tw_W != Wp) {
        const int lens[4] = {Wp, Wp, Hp, Hp};
        for (int i = 0; i < 4; ++i) {
            const std::vector<float> t = nfx::build_fft_twiddles(lens[i], (i & 1) == 1);
            if (rt->f2_tw[i]) cudaFree(rt->f2_tw[i]);
            rt->f2_tw[i] = nullptr;
            void* p = nullptr;
            if (!cuda_ok(rt, cudaMalloc(&p, t.size() * 4 + 16), "cudaMalloc twiddles")) return NFX_INTERNAL;
            rt->f2_tw[i] = static_cast<float2*>(p);
            if (!t.empty() && !cuda_ok(rt, cudaMemcpy(p, t.data(), t.size() * 4, cudaMemcpyHostToDevice),
                                       "cudaMemcpy twiddles"))
                return NFX_INTERNAL;
        }
        rt->f2_tw_H = Hp;
        rt->f2_tw_W = Wp;
    }
    const int64_t plane = static_cast<int64_t>(B) * c.width * Hp * Wp;
    int s = ensure_f2_buf(rt, 0, plane * 4);
    if (s == NFX_OK) s = ensure_f2_buf(rt, 1, plane * 4);
    if (s == NFX_OK) s = ensure_f2_buf(rt, 2, static_cast<int64_t>(B) * c.width * c.mh * c.mw * 8);
    if (s == NFX_OK) s = ensure_f2_buf(rt, 3, static_cast<int64_t>(B) * c.width * Hp * c.mw * 8);
    if (s != NFX_OK) return s;
    nfx::Fno2dF32Plan pl = pl0;
    pl.B = B;
    pl.H = H;
    pl.W = W;
    pl.Hp = Hp;
    pl.Wp = Wp;
    pl.x = dx;
    pl.y = dy;
    pl.twf_w = rt->f2_tw[0];
    pl.twi_w = rt->f2_tw[1];
    pl.twf_h = rt->f2_tw[2];
    pl.twi_h = rt->f2_tw[3];
    pl.h[0] = static_cast<float*>(rt->f2_bufs[0]);
    pl.h[1] = static_cast<float*>(rt->f2_bufs[1]);
    pl.Xs = static_cast<float2*>(rt->f2_bufs[2]);
    pl.colinv = static_cast<float2*>(rt->f2_bufs[3]);
    pl.timer = rt->timer.get();
    pl.obs = obs;
    for (int i = 0; i < nfx::kFno2dObsMax; ++i) pl.obs_vals[i] = obs && obs_vals ? obs_vals[i] : nullptr;
    if (obs) {
        pl.fq_lift.kind = 0;
        pl.fq_pq.kind = 0;
        pl.fq_po.kind = 0;
        for (int i = 0; i < pl.L && i < nfx::kFno2dMaxLayers; ++i) pl.layer[i].fq.kind = 0;
    }
    const cudaError_t e = nfx::fno2d_f32_run(pl, st);
    if (e != cudaSuccess)
        return rt_fail(rt, NFX_INTERNAL, std::string("FNO2d launch failed: ") + cudaGetErrorString(e));
    return NFX_OK;
}

int fno2d_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st) {
    const F2 c = fno2d_cfg(rt->model);
    if (!rt->int8_enabled) return fno2d_f32_launch(rt, dx, xs, dy, st);
    const int B = static_cast<int>(xs[0]), H = static_cast<int>(xs[1]), W = static_cast<int>(xs[2]);
    // the width-64 executor's range; elsewhere the composition runs on plan2i
    const bool fast = rt->f2_fast && W >= 32 && W <= 128 && H >= 8 && H <= 4096 && c.mh <= H &&
                      c.mw <= W / 2 + 1 && !(c.pad > 1 && ((H % c.pad) || (W % c.pad)));
    if (!fast) {
        if (rt->tap_codes)
            return rt_fail(rt, NFX_UNSUPPORTED_OP,
                           "code taps are written by the width-64 12x12 INT8 executor only");
        return fno2d_f32_launch(rt, dx, xs, dy, st);
    }
    if (B == 0) return NFX_OK;
    int s = ensure_twiddles(rt, H, W);
    if (s != NFX_OK) return s;
    s = ensure_buffers(rt, B, H, W);
    if (s != NFX_OK) return s;
    nfx::Fno2dPlan pl = rt->plan;
    pl.B = B;
    pl.H = H;
    pl.W = W;
    pl.HB = H / nfx::fno2d_row_blocks(H);
    pl.x = dx;
    pl.y = dy;
    pl.codes[0] = static_cast<int8_t*>(rt->act_bufs[0]);
    pl.codes[1] = static_cast<int8_t*>(rt->act_bufs[1]);
    pl.xpart = static_cast<float2*>(rt->act_bufs[2]);
    pl.Y = static_cast<float2*>(rt->act_bufs[3]);
    pl.twf_w = rt->tw[0];
    pl.twf_h = rt->tw[1];
    pl.twi_w = rt->tw[2];
    pl.twi_h = rt->tw[3];
    pl.fwd_limbs = rt->fwd_limbs;
    pl.fwd_sum_b = rt->fwd_sum_b;
    pl.err = nfx::device_error_word();
    if (!pl.err) return rt_fail(rt, NFX_INTERNAL, "no device error word");
    pl.timer = rt->timer.get();
    pl.tap_codes = nullptr;
    if (rt->tap_codes) {
        const int64_t need = static_cast<int64_t>(c.L + 1) * B * H * W * c.width;
        if (need > rt->tap_cap)
            return rt_fail(rt, NFX_INVALID_ARG, "code-tap buffer too small: needs " +
                                                    std::to_string(need) + " bytes");
        pl.tap_codes = rt->tap_codes;
    }
    const cudaError_t e = nfx::fno2d_run(pl, st);
    if (e != cudaSuccess)
        return rt_fail(rt, NFX_INTERNAL, std::string("FNO2d launch failed: ") + cudaGetErrorString(e));
    return NFX_OK;
}

// ---------------------------------------------------------------------------
// FNO1d (fno.cpp:408-706)
// ---------------------------------------------------------------------------
struct F1 {
    int in_ch, out_ch, width, modes, L, pad;
};
F1 fno1d_cfg(const nfx::IrModel& m) {
    return F1{m.cfg[0], m.cfg[1], m.cfg[2], m.cfg[3], m.cfg[4], m.cfg[5]};
}

std::string in_key(int i) {
    return i == 0 ? std::string("lift.output") : "locs." + std::to_string(i - 1) + ".output";
}

// Create: load-time weight fake-quant (fno.cpp:293-315), uploads, and the per-layer
// branch decisions of FNO1d::Forward that depend only on the IR.
int fno1d_create(nfx_runtime* rt) {
    auto& m = rt->model;
    const F1 c = fno1d_cfg(m);
    if (m.quant_enabled)
        for (const auto& name : m.weight_order) nfx::dequantise_weight(m.weights[name], m, name);
    if (c.L > nfx::kFno1dMaxLayers || c.width > nfx::kFno1dMaxC || c.width < 1 || c.out_ch > 16 ||
        c.out_ch < 1 || c.in_ch < 1 || c.modes < 0)
        return NFX_OK;  // Run reports UnsupportedOp
    auto& pl = rt->plan1;
    pl.C = c.width;
    pl.in_ch = c.in_ch;
    pl.out_ch = c.out_ch;
    pl.modes = c.modes;
    pl.L = c.L;
    pl.act = m.activation == "relu" ? 1 : 0;
    pl.lift_w = wptr(rt, "lift.weight");
    pl.lift_b = wptr(rt, "lift.bias");
    pl.pq_w = wptr(rt, "proj_q.weight");
    pl.pq_b = wptr(rt, "proj_q.bias");
    pl.po_w = wptr(rt, "proj_out.weight");
    pl.po_b = wptr(rt, "proj_out.bias");
    if (!pl.lift_w || !pl.lift_b || !pl.pq_w || !pl.pq_b || !pl.po_w || !pl.po_b)
        return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    const bool q = m.quant_enabled;
    for (int i = 0; i < c.L; ++i) {
        nfx::Fno1dLayer& L = pl.layer[i];
        L = nfx::Fno1dLayer{};
        const std::string s = std::to_string(i);
        L.wr = wptr(rt, "specs." + s + ".weights_real");
        L.wi = wptr(rt, "specs." + s + ".weights_imag");
        L.loc_w = wptr(rt, "locs." + s + ".weight");
        L.loc_b = wptr(rt, "locs." + s + ".bias");
        if (!L.wr || !L.wi || !L.loc_w || !L.loc_b) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
        // input snap: the per-tensor map only (fno.cpp:488-508)
        auto it = m.activation_qparams.find(in_key(i));
        if (q && it != m.activation_qparams.end()) {
            L.in_codes = 1;
            L.in_s = it->second.scale;
            L.in_zp = it->second.zero_point;
        }
        // output fake-quant: FP8, else per-token, else per-tensor (fno.cpp:572-654)
        const std::string ok = "locs." + s + ".output";
        if (q) {
            auto i8 = m.activation_fp8_qparams.find(ok);
            auto ipt = m.activation_per_token_qparams.find(ok);
            auto ipx = m.activation_qparams.find(ok);
            if (i8 != m.activation_fp8_qparams.end()) {
                L.fq_kind = 3;
                L.fq_s = i8->second;
            } else if (ipt != m.activation_per_token_qparams.end()) {
                L.fq_kind = 2;
                L.pt_s = upload(rt, ipt->second.scales.data(), ipt->second.scales.size());
                L.pt_zp = upload(rt, ipt->second.zero_points.data(), ipt->second.zero_points.size());
                if (!L.pt_s || !L.pt_zp) return rt_fail(rt, NFX_INTERNAL, "qparam upload failed");
                rt->pt_n[i] = static_cast<int>(std::min(ipt->second.scales.size(), ipt->second.zero_points.size()));
                rt->pt_w[i] = ipt->second.width;
            } else if (ipx != m.activation_qparams.end()) {
                L.fq_kind = 1;
                L.fq_s = ipx->second.scale;
                L.fq_zp = ipx->second.zero_point;
            }
        }
    }
    // each layer's output is the next layer's input: codes when that layer snaps
    for (int i = 0; i + 1 < c.L; ++i) {
        nfx::Fno1dLayer& L = pl.layer[i];
        const nfx::Fno1dLayer& Ln = pl.layer[i + 1];
        if (!Ln.in_codes) continue;
        L.out_codes = 1;
        L.out_s = Ln.in_s;
        L.out_zp = Ln.in_zp;
        nfx::CodeLut lut;
        std::string why;
        if (nfx::build_code_lut(L.out_s, L.out_zp, pl.act, 4096, lut, why)) {
            L.code_lut = reinterpret_cast<const int2*>(upload(rt, lut.cells.data(), lut.cells.size()));
            if (!L.code_lut) return rt_fail(rt, NFX_INTERNAL, "table upload failed");
            L.lut_cells = static_cast<int>(lut.cells.size());
            L.lut_zlo = lut.zlo;
            L.lut_inv_delta = lut.inv_delta;
        }
    }
    return NFX_OK;
}

// EnableInt8Gemm (runtime.cpp:155-166 -> fno.cpp:360-406): the flag is set whatever
// the IR holds; a layer dispatches through the INT8 GEMM when LinearDispatchTryInt8
// would (per-channel axis-0 weight codes, a per-tensor input qparam, no per-token or
// FP8 qparam for the input key).
void fno1d_enable_int8(nfx_runtime* rt) {
    auto& m = rt->model;
    const F1 c = fno1d_cfg(m);
    rt->int8_enabled = true;
    if (!m.quant_enabled || c.L > nfx::kFno1dMaxLayers) return;
    auto& pl = rt->plan1;
    if (!pl.lift_w) return;  // unsupported geometry; Run reports it
    for (int i = 0; i < c.L; ++i) {
        nfx::Fno1dLayer& L = pl.layer[i];
        const std::string k = in_key(i);
        if (m.activation_per_token_qparams.count(k) || m.activation_fp8_qparams.count(k)) continue;
        if (!m.activation_qparams.count(k)) continue;
        const std::string wname = "locs." + std::to_string(i) + ".weight";
        auto pc = m.weight_per_channel_qparams.find(wname);
        if (pc == m.weight_per_channel_qparams.end()) continue;
        std::vector<int8_t> codes;
        std::vector<int32_t> sum_w;
        if (!nfx::quantise_weight_2d(m.weights.at(wname), pc->second, codes, sum_w)) continue;
        L.Wq = upload(rt, codes.data(), codes.size());
        L.scale_w = upload(rt, pc->second.scales.data(), pc->second.scales.size());
        L.zp_w = upload(rt, pc->second.zero_points.data(), pc->second.zero_points.size());
        L.sum_w = upload(rt, sum_w.data(), sum_w.size());
        if (!L.Wq || !L.scale_w || !L.zp_w || !L.sum_w) continue;
        L.use_int8 = 1;
    }
}

int check_fno1d_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    const F1 c = fno1d_cfg(rt->model);
    if (xr != 3) return rt_fail(rt, NFX_SHAPE_MISMATCH, "expected 3D input (batch, n, in_ch)");
    if (xs[2] != c.in_ch) return rt_fail(rt, NFX_SHAPE_MISMATCH, "input channels mismatch");
    if (yr != 3 || ys[0] != xs[0] || ys[1] != xs[1] || ys[2] != c.out_ch)
        return rt_fail(rt, NFX_SHAPE_MISMATCH, "output buffer shape mismatch");
    if (!(xs[1] > 0 && (xs[1] & (xs[1] - 1)) == 0))
        return rt_fail(rt, NFX_INVALID_ARG, "Stage 1: input length n must be a power of two");
    return NFX_OK;
}

int fno1d_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st) {
    const F1 c = fno1d_cfg(rt->model);
    auto& pl0 = rt->plan1;
    if (!pl0.lift_w)
        return rt_fail(rt, NFX_UNSUPPORTED_OP,
                       "FNO1d GPU executor: needs width <= 256, out_channels <= 16, <= 8 layers");
    const int B = static_cast<int>(xs[0]), n = static_cast<int>(xs[1]);
    int N = n;
    if (c.pad > 1 && n % c.pad) N = n + (c.pad - n % c.pad);
    if (N & (N - 1))
        return rt_fail(rt, NFX_INVALID_ARG, "FNO1d: padded length must be a power of two");
    if (N > nfx::kFno1dMaxN)
        return rt_fail(rt, NFX_UNSUPPORTED_OP, "FNO1d GPU executor: padded length above 8192");
    if (c.modes > N / 2 + 1)
        return rt_fail(rt, NFX_INVALID_ARG, "FNO1d: modes exceed n/2 + 1");
    for (int i = 0; i < c.L; ++i) {
        const auto& L = pl0.layer[i];
        if (L.fq_kind == 2 && (rt->pt_w[i] != c.width || static_cast<int64_t>(rt->pt_n[i]) <
                                                            static_cast<int64_t>(N) * c.width))
            return rt_fail(rt, NFX_INVALID_ARG,
                           "FNO1d: per-token qparams of locs." + std::to_string(i) +
                               ".output do not cover (n, width)");
    }
    if (B == 0) return NFX_OK;
    // twiddles for N
    if (rt->f1_tw_N != N) {
        for (int inv = 0; inv < 2; ++inv) {
            const std::vector<float> t = nfx::build_fft_twiddles(N, inv == 1);
            if (rt->f1_tw[inv]) cudaFree(rt->f1_tw[inv]);
            rt->f1_tw[inv] = nullptr;
            void* p = nullptr;
            if (!cuda_ok(rt, cudaMalloc(&p, t.size() * 4 + 16), "cudaMalloc twiddles")) return NFX_INTERNAL;
            rt->f1_tw[inv] = static_cast<float2*>(p);
            if (!t.empty() && !cuda_ok(rt, cudaMemcpy(p, t.data(), t.size() * 4, cudaMemcpyHostToDevice),
                                       "cudaMemcpy twiddles"))
                return NFX_INTERNAL;
        }
        rt->f1_tw_N = N;
    }
    const int64_t BN = static_cast<int64_t>(B) * N;
    if (BN > rt->f1_cap_BN) {
        for (auto*& p : rt->f1_bufs) {
            if (p) cudaFree(p);
            p = nullptr;
        }
        const size_t sizes[5] = {static_cast<size_t>(BN) * c.width * 4, static_cast<size_t>(BN) * c.width * 4,
                                 static_cast<size_t>(B) * c.width * (c.modes > 0 ? c.modes : 1) * sizeof(float2),
                                 static_cast<size_t>(BN) * c.width * 4, static_cast<size_t>(BN) * c.width * 4};
        for (int i = 0; i < 5; ++i)
            if (!cuda_ok(rt, cudaMalloc(&rt->f1_bufs[i], sizes[i] + 256), "cudaMalloc activations"))
                return NFX_INTERNAL;
        rt->f1_cap_BN = BN;
    }
    nfx::Fno1dPlan pl = pl0;
    pl.B = B;
    pl.n = n;
    pl.N = N;
    pl.x = dx;
    pl.y = dy;
    pl.tw_fwd = rt->f1_tw[0];
    pl.tw_inv = rt->f1_tw[1];
    pl.h[0] = rt->f1_bufs[0];
    pl.h[1] = rt->f1_bufs[1];
    pl.Xs = static_cast<float2*>(rt->f1_bufs[2]);
    pl.x2raw = static_cast<float*>(rt->f1_bufs[3]);
    pl.x1f = static_cast<float*>(rt->f1_bufs[4]);
    if (c.L == 0) pl.layer[0] = nfx::Fno1dLayer{};
    pl.err = nfx::device_error_word();
    if (!pl.err) return rt_fail(rt, NFX_INTERNAL, "no device error word");
    pl.timer = rt->timer.get();
    const cudaError_t e = nfx::fno1d_run(pl, st);
    if (e != cudaSuccess)
        return rt_fail(rt, NFX_INTERNAL, std::string("FNO1d launch failed: ") + cudaGetErrorString(e));
    return NFX_OK;
}

// ---------------------------------------------------------------------------
// FNO3d (fno.cpp:1096-1281)
// ---------------------------------------------------------------------------
int fno3d_create(nfx_runtime* rt) {
    // the reference builds FNO3d from the raw weights without its NIRQ block
    // (runtime.cpp:51-54)
    auto& m = rt->model;
    auto& pl = rt->plan3;
    const int* c = m.cfg;
    pl.in_ch = c[0];
    pl.out_ch = c[1];
    pl.C = c[2];
    pl.MH = c[3];
    pl.MW = c[4];
    pl.MD = c[5];
    pl.L = c[6];
    pl.act = m.activation == "relu" ? 1 : 0;
    if (pl.L > nfx::kFno3dMaxLayers || pl.in_ch < 1) return NFX_OK;  // Run reports it
    pl.lift_w = wptr(rt, "lift.weight");
    pl.lift_b = wptr(rt, "lift.bias");
    pl.pq_w = wptr(rt, "proj_q.weight");
    pl.pq_b = wptr(rt, "proj_q.bias");
    pl.po_w = wptr(rt, "proj_out.weight");
    pl.po_b = wptr(rt, "proj_out.bias");
    if (!pl.lift_w || !pl.lift_b || !pl.pq_w || !pl.pq_b || !pl.po_w || !pl.po_b)
        return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    for (int i = 0; i < pl.L; ++i) {
        const std::string s = std::to_string(i);
        auto& L = pl.layer[i];
        L.wr = wptr(rt, "specs." + s + ".weights_real");
        L.wi = wptr(rt, "specs." + s + ".weights_imag");
        L.loc_w = wptr(rt, "locs." + s + ".weight");
        L.loc_b = wptr(rt, "locs." + s + ".bias");
        if (!L.wr || !L.wi || !L.loc_w || !L.loc_b) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    }
    return NFX_OK;
}

// FP8 E4M3 executor (no reference counterpart): needs an FP8 scale (NIRQ kind 3) for
// every Linear weight and every ".output" key.
void fno3d_enable_fp8(nfx_runtime* rt) {
    auto& m = rt->model;
    auto& pl = rt->plan3;
    if (!pl.lift_w || !m.quant_enabled) return;
    auto sc = [&](const std::string& k, float& out) {
        auto it = m.activation_fp8_qparams.find(k);
        if (it == m.activation_fp8_qparams.end()) return false;
        out = it->second;
        return true;
    };
    float s_lift_w, s_pq_w, s_po_w, s_lift, s_pq, s_po;
    std::vector<float> s_lw(pl.L), s_lo(pl.L);
    if (!sc("lift.weight", s_lift_w) || !sc("proj_q.weight", s_pq_w) || !sc("proj_out.weight", s_po_w) ||
        !sc("lift.output", s_lift) || !sc("proj_q.output", s_pq) || !sc("proj_out.output", s_po))
        return;
    for (int i = 0; i < pl.L; ++i)
        if (!sc("locs." + std::to_string(i) + ".weight", s_lw[i]) || !sc("locs." + std::to_string(i) + ".output", s_lo[i]))
            return;
    auto fq = [&](const std::string& name, float scale, bool want_xq, const float** fq_out, const float** xq_out) {
        const auto& t = m.weights.at(name);
        std::vector<float> xq(t.data.size()), v(t.data.size());
        nfx::e4m3_fake_quant(t.data.data(), scale, xq.data(), v.data(), t.data.size());
        if (fq_out) *fq_out = upload(rt, v.data(), v.size());
        if (want_xq) *xq_out = upload(rt, xq.data(), xq.size());
    };
    nfx::Fno3dPlan q = pl;
    fq("lift.weight", s_lift_w, false, &q.lift_w, nullptr);
    fq("proj_out.weight", s_po_w, false, &q.po_w, nullptr);
    fq("proj_q.weight", s_pq_w, true, nullptr, &q.pq_q);
    for (int i = 0; i < pl.L; ++i)
        fq("locs." + std::to_string(i) + ".weight", s_lw[i], true, nullptr, &q.layer[i].loc_q);
    if (!q.lift_w || !q.po_w || !q.pq_q) return;
    for (int i = 0; i < pl.L; ++i) {
        if (!q.layer[i].loc_q) return;
        q.layer[i].s_in = i == 0 ? s_lift : s_lo[i - 1];
        q.layer[i].s_w = s_lw[i];
        q.layer[i].s_out = s_lo[i];
    }
    q.s_lift = s_lift;
    q.s_pq_w = s_pq_w;
    q.s_pq = s_pq;
    q.s_po = s_po;
    q.fp8 = 1;
    pl = q;
    rt->fp8_enabled = true;
}

int check_fno3d_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    const auto& pl = rt->plan3;
    if (xr != 5) return rt_fail(rt, NFX_SHAPE_MISMATCH, "expected 5D input (batch, h, w, d, in_ch)");
    if (xs[4] != pl.in_ch) return rt_fail(rt, NFX_SHAPE_MISMATCH, "input channels mismatch");
    if (yr != 5 || ys[0] != xs[0] || ys[1] != xs[1] || ys[2] != xs[2] || ys[3] != xs[3] || ys[4] != pl.out_ch)
        return rt_fail(rt, NFX_SHAPE_MISMATCH, "output buffer shape mismatch");
    auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
    if (!pow2(xs[1]) || !pow2(xs[2]) || !pow2(xs[3]))
        return rt_fail(rt, NFX_INVALID_ARG, "FNO3d: H, W, and D must each be a power of two");
    return NFX_OK;
}

int fno3d_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st) {
    auto& pl0 = rt->plan3;
    if (!pl0.lift_w) return rt_fail(rt, NFX_UNSUPPORTED_OP, "FNO3d GPU executor: needs <= 8 layers");
    const int B = static_cast<int>(xs[0]);
    int dims[3] = {static_cast<int>(xs[1]), static_cast<int>(xs[2]), static_cast<int>(xs[3])};
    int pd[3] = {dims[0], dims[1], dims[2]};
    const int pf = rt->model.cfg[7];
    if (pf > 1)
        for (int i = 0; i < 3; ++i) pd[i] = dims[i] + (pf - dims[i] % pf) % pf;
    for (int i = 0; i < 3; ++i)
        if (pd[i] & (pd[i] - 1)) return rt_fail(rt, NFX_INVALID_ARG, "FNO3d: padded sides must be powers of two");
    if (pl0.MH > pd[0] || pl0.MW > pd[1] || pl0.MD > pd[2] / 2 + 1)
        return rt_fail(rt, NFX_INVALID_ARG, "FNO3d: modes exceed the (padded) grid");
    if (const char* why = nfx::fno3d_unsupported(pl0.C, pd[0], pd[1], pd[2], pl0.MH, pl0.MW, pl0.MD, pl0.out_ch))
        return rt_fail(rt, NFX_UNSUPPORTED_OP, why);
    if (B == 0) return NFX_OK;
    if (rt->f3_tw_dims[0] != pd[0] || rt->f3_tw_dims[1] != pd[1] || rt->f3_tw_dims[2] != pd[2]) {
        for (int i = 0; i < 6; ++i) {
            const std::vector<float> t = nfx::build_fft_twiddles(pd[i / 2], (i & 1) == 1);
            if (rt->f3_tw[i]) cudaFree(rt->f3_tw[i]);
            rt->f3_tw[i] = nullptr;
            void* p = nullptr;
            if (!cuda_ok(rt, cudaMalloc(&p, t.size() * 4 + 16), "cudaMalloc twiddles")) return NFX_INTERNAL;
            rt->f3_tw[i] = static_cast<float2*>(p);
            if (!t.empty() && !cuda_ok(rt, cudaMemcpy(p, t.data(), t.size() * 4, cudaMemcpyHostToDevice),
                                       "cudaMemcpy twiddles"))
                return NFX_INTERNAL;
        }
        for (int i = 0; i < 3; ++i) rt->f3_tw_dims[i] = pd[i];
    }
    const bool direct = nfx::fno3d_direct_dft(pl0.C, pl0.fp8, pd[1], pd[2], pl0.MW, pl0.MD);
    const int dkey[4] = {pd[1], pd[2], pl0.MW, pl0.MD};
    if (direct && !std::equal(dkey, dkey + 4, rt->f3_dft_key)) {
        const std::vector<float> t = nfx::fno3d_dft_tables(pd[1], pd[2], pl0.MW, pl0.MD);
        if (rt->f3_dft) cudaFree(rt->f3_dft);
        rt->f3_dft = nullptr;
        std::fill(rt->f3_dft_key, rt->f3_dft_key + 4, 0);
        void* p = nullptr;
        if (!cuda_ok(rt, cudaMalloc(&p, t.size() * 4), "cudaMalloc DFT tables")) return NFX_INTERNAL;
        rt->f3_dft = static_cast<float*>(p);
        if (!cuda_ok(rt, cudaMemcpy(p, t.data(), t.size() * 4, cudaMemcpyHostToDevice), "cudaMemcpy DFT tables"))
            return NFX_INTERNAL;
        std::copy(dkey, dkey + 4, rt->f3_dft_key);
    }
    const int64_t vol = static_cast<int64_t>(B) * pl0.C * pd[0] * pd[1] * pd[2];
    const int64_t kk = static_cast<int64_t>(B) * pl0.C * pl0.MW * pl0.MD;
    const int64_t sizes[6] = {vol * 4, vol * 4, kk * pd[0] * 8, kk * pl0.MH * 8, kk * pd[0] * 8, vol * 4};
    for (int i = 0; i < 6; ++i) {
        if (sizes[i] <= rt->f3_cap[i]) continue;
        if (rt->f3_bufs[i]) cudaFree(rt->f3_bufs[i]);
        rt->f3_bufs[i] = nullptr;
        rt->f3_cap[i] = 0;
        if (!cuda_ok(rt, cudaMalloc(&rt->f3_bufs[i], static_cast<size_t>(sizes[i]) + 256), "cudaMalloc activations"))
            return NFX_INTERNAL;
        rt->f3_cap[i] = sizes[i];
    }
    nfx::Fno3dPlan pl = pl0;
    pl.B = B;
    pl.H = dims[0];
    pl.W = dims[1];
    pl.D = dims[2];
    pl.Hp = pd[0];
    pl.Wp = pd[1];
    pl.Dp = pd[2];
    pl.x = dx;
    pl.y = dy;
    for (int i = 0; i < 6; ++i) pl.tw[i] = rt->f3_tw[i];
    pl.dft = direct ? rt->f3_dft : nullptr;
    pl.tap_codes = nullptr;
    if (rt->tap_codes) {
        if (!pl.fp8) return rt_fail(rt, NFX_UNSUPPORTED_OP, "FNO3d code taps exist for the FP8 variant only");
        const int64_t need = static_cast<int64_t>(pl.L + 1) * vol;
        if (need > rt->tap_cap) return rt_fail(rt, NFX_INVALID_ARG, "code tap buffer too small");
        pl.tap_codes = reinterpret_cast<uint8_t*>(rt->tap_codes);
    }
    pl.h[0] = rt->f3_bufs[0];
    pl.h[1] = rt->f3_bufs[1];
    pl.A = static_cast<float2*>(rt->f3_bufs[2]);
    pl.Xs = static_cast<float2*>(rt->f3_bufs[3]);
    pl.colinv = static_cast<float2*>(rt->f3_bufs[4]);
    pl.x1 = static_cast<float*>(rt->f3_bufs[5]);
    pl.timer = rt->timer.get();
    const cudaError_t e = nfx::fno3d_run(pl, st);
    if (e != cudaSuccess)
        return rt_fail(rt, NFX_INTERNAL, std::string("FNO3d launch failed: ") + cudaGetErrorString(e));
    return NFX_OK;
}

// ---------------------------------------------------------------------------
// TokenMixer2D (fno.cpp:1756-1956)
// ---------------------------------------------------------------------------
const char* kTmParts[8] = {"ln1", "q_proj", "k_proj", "v_proj", "o_proj", "ln2", "ffn0", "ffn1"};

int tm2d_create(nfx_runtime* rt) {
    // the reference runtime builds TokenMixer2D from the raw weights and ignores NIRQ
    // (runtime.cpp:61-64).  The 1D TokenMixer (fno.cpp:1460-1644) is the same network
    // on n_points points: it runs as a 1 x n_points grid.
    auto& m = rt->model;
    auto& pl = rt->plan_tm;
    const int* c = m.cfg;
    pl.in_d = c[0];
    pl.out_d = c[1];
    pl.L = c[2];
    if (m.op == "TokenMixer") {
        pl.h = 1;
        pl.w = c[3];
        pl.NP = c[4];
        pl.heads = c[5];
        pl.layers = c[6];
    } else {
        pl.h = c[3];
        pl.w = c[4];
        pl.NP = c[5];
        pl.heads = c[6];
        pl.layers = c[7];
    }
    pl.act = m.activation == "relu" ? 1 : 0;
    if (pl.layers < 1 || pl.layers > nfx::kTm2dMaxLayers) return NFX_OK;  // Run reports it
    pl.se_w = wptr(rt, "slice_embed.proj.weight");
    pl.se_b = wptr(rt, "slice_embed.proj.bias");
    pl.un_w = wptr(rt, "unslice.proj.weight");
    pl.un_b = wptr(rt, "unslice.proj.bias");
    pl.head_w = wptr(rt, "head.weight");
    pl.head_b = wptr(rt, "head.bias");
    if (!pl.se_w || !pl.se_b || !pl.un_w || !pl.un_b || !pl.head_w || !pl.head_b)
        return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    for (int i = 0; i < pl.layers; ++i)
        for (int j = 0; j < 8; ++j) {
            const std::string pre = "blocks." + std::to_string(i) + "." + kTmParts[j];
            pl.blk[i].w[j] = wptr(rt, pre + ".weight");
            pl.blk[i].b[j] = wptr(rt, pre + ".bias");
            if (!pl.blk[i].w[j] || !pl.blk[i].b[j]) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
        }
    return NFX_OK;
}

// EnableInt8Gemm for TokenMixer2D (no reference counterpart): q, k, v, o, ffn0, ffn1 of
// every block need per-channel (axis 0) weight qparams in NIRQ; the weight codes follow
// QuantiseWeight2D (fno.cpp:325-358) on the raw weights.
void tm2d_enable_int8(nfx_runtime* rt) {
    auto& m = rt->model;
    auto& pl = rt->plan_tm;
    if (!pl.se_w || !m.quant_enabled) return;
    const int slots[6] = {1, 2, 3, 4, 6, 7};
    for (int i = 0; i < pl.layers; ++i)
        for (int j : slots) {
            const std::string wn = "blocks." + std::to_string(i) + "." + kTmParts[j] + ".weight";
            auto pc = m.weight_per_channel_qparams.find(wn);
            if (pc == m.weight_per_channel_qparams.end()) return;
            const auto& t = m.weights.at(wn);
            if (!nfx::gemm_i8_supported(static_cast<int>(t.shape[1]), static_cast<int>(t.shape[0]))) return;
        }
    for (int i = 0; i < pl.layers; ++i)
        for (int j : slots) {
            const std::string wn = "blocks." + std::to_string(i) + "." + kTmParts[j] + ".weight";
            const auto& pc = m.weight_per_channel_qparams.at(wn);
            std::vector<int8_t> codes;
            std::vector<int32_t> sum_w;
            if (!nfx::quantise_weight_2d(m.weights.at(wn), pc, codes, sum_w)) return;
            auto& q = pl.blk[i].q8[j];
            q.Wq = upload(rt, codes.data(), codes.size());
            q.scale_w = upload(rt, pc.scales.data(), pc.scales.size());
            q.zp_w = upload(rt, pc.zero_points.data(), pc.zero_points.size());
            q.sum_w = upload(rt, sum_w.data(), sum_w.size());
            if (!q.Wq || !q.scale_w || !q.zp_w || !q.sum_w) return;
        }
    pl.int8 = 1;
    rt->int8_enabled = true;
}

int check_tm1d_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    // fno.cpp:1461-1497
    const auto& pl = rt->plan_tm;
    if (xr != 3) return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer: expected 3D x (batch, n_points, in_dim)");
    if (xs[2] != pl.in_d) return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer: input feature dim mismatch");
    if (xs[1] != pl.w) return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer: n_points mismatch");
    if (yr != 3 || ys[0] != xs[0] || ys[1] != xs[1] || ys[2] != pl.out_d)
        return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer: output buffer shape mismatch");
    if (pl.NP <= 0 || pl.w % pl.NP != 0)
        return rt_fail(rt, NFX_INVALID_ARG, "TokenMixer: n_points must be a multiple of n_patches");
    if (pl.heads <= 0 || pl.L % pl.heads != 0)
        return rt_fail(rt, NFX_INVALID_ARG, "TokenMixer: latent_dim must be a multiple of n_heads");
    if (pl.layers < 1) return rt_fail(rt, NFX_INVALID_ARG, "TokenMixer: n_layers must be >= 1");
    if (pl.layers > nfx::kTm2dMaxLayers || !pl.se_w)
        return rt_fail(rt, NFX_UNSUPPORTED_OP, "TokenMixer GPU executor: at most 8 blocks");
    if (const char* why = nfx::tm2d_unsupported(pl.L, pl.heads, pl.in_d, pl.out_d))
        return rt_fail(rt, NFX_UNSUPPORTED_OP, why);
    return NFX_OK;
}

int check_tm2d_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    if (rt->model.op == "TokenMixer") return check_tm1d_shapes(rt, xs, xr, ys, yr);
    const auto& pl = rt->plan_tm;
    if (xr != 4) return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer2D: expected 4D x (batch, h, w, in_dim)");
    if (xs[3] != pl.in_d) return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer2D: input feature dim mismatch");
    if (xs[1] != pl.h || xs[2] != pl.w) return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer2D: h / w mismatch");
    if (yr != 4 || ys[0] != xs[0] || ys[1] != xs[1] || ys[2] != xs[2] || ys[3] != pl.out_d)
        return rt_fail(rt, NFX_SHAPE_MISMATCH, "TokenMixer2D: output buffer shape mismatch");
    if (pl.NP <= 0 || (pl.h * pl.w) % pl.NP != 0)
        return rt_fail(rt, NFX_INVALID_ARG, "TokenMixer2D: h*w must be a multiple of n_patches");
    if (pl.heads <= 0 || pl.L % pl.heads != 0)
        return rt_fail(rt, NFX_INVALID_ARG, "TokenMixer2D: latent_dim must be a multiple of n_heads");
    if (pl.layers < 1) return rt_fail(rt, NFX_INVALID_ARG, "TokenMixer2D: n_layers must be >= 1");
    if (pl.layers > nfx::kTm2dMaxLayers || !pl.se_w)
        return rt_fail(rt, NFX_UNSUPPORTED_OP, "TokenMixer2D GPU executor: at most 8 blocks");
    if (const char* why = nfx::tm2d_unsupported(pl.L, pl.heads, pl.in_d, pl.out_d))
        return rt_fail(rt, NFX_UNSUPPORTED_OP, why);
    return NFX_OK;
}

int tm2d_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st) {
    auto& pl0 = rt->plan_tm;
    const int B = static_cast<int>(xs[0]);
    if (B == 0) return NFX_OK;
    const int64_t T = static_cast<int64_t>(B) * pl0.NP;
    const int64_t P = static_cast<int64_t>(B) * pl0.h * pl0.w;
    const int L = pl0.L;
    if (T > rt->tm_cap_T || P > rt->tm_cap_P) {
        for (auto*& p : rt->tm_bufs) {
            if (p) cudaFree(p);
            p = nullptr;
        }
        const int64_t sizes[13] = {T * pl0.in_d * 4, T * L * 4, T * L * 4, T * L * 4, T * L * 4, T * L * 4,
                                   T * L * 4, T * 2 * L * 4, T * L * 4, P * L * 4, T * 2 * L, T * 8,
                                   6 * T * L * 4};
        for (int i = 0; i < 13; ++i)
            if (!cuda_ok(rt, cudaMalloc(&rt->tm_bufs[i], static_cast<size_t>(sizes[i]) + 256), "cudaMalloc activations"))
                return NFX_INTERNAL;
        rt->tm_cap_T = T;
        rt->tm_cap_P = P;
    }
    nfx::Tm2dPlan pl = pl0;
    pl.B = B;
    pl.x = dx;
    pl.y = dy;
    float** f[10] = {&pl.pooled, &pl.tok, &pl.ln, &pl.q, &pl.k, &pl.v, &pl.ho, &pl.f0, &pl.f1, &pl.feat};
    for (int i = 0; i < 10; ++i) *f[i] = static_cast<float*>(rt->tm_bufs[i]);
    pl.codes = static_cast<int8_t*>(rt->tm_bufs[10]);
    pl.row_s = static_cast<float*>(rt->tm_bufs[11]);
    pl.row_zp = reinterpret_cast<int32_t*>(static_cast<char*>(rt->tm_bufs[11]) + T * 4);
    pl.qkv_split = static_cast<float*>(rt->tm_bufs[12]);
    // attention on tensor cores (3xTF32, fp32-accurate; head dim 32); the FP32 path's
    // outputs stay within rtol 1e-5 of the reference-order attention
    pl.tc_attention = 1;
    pl.err = nfx::device_error_word();
    if (!pl.err) return rt_fail(rt, NFX_INTERNAL, "no device error word");
    pl.timer = rt->timer.get();
    const cudaError_t e = nfx::tm2d_run(pl, st);
    if (e != cudaSuccess)
        return rt_fail(rt, NFX_INTERNAL, std::string("TokenMixer2D launch failed: ") + cudaGetErrorString(e));
    return NFX_OK;
}

// ---------------------------------------------------------------------------
// DeepONet (fno.cpp:1289-1406), GraphOp / GraphOp2D (fno.cpp:1653-1741, :1969-2060)
// ---------------------------------------------------------------------------

// A weight the reference indexes as (out, in) with the widths the loader derived;
// the reference reads past a tensor whose shape disagrees, the GPU runtime refuses it.
bool mo_layer(nfx_runtime* rt, const std::string& wname, const std::string& bname, int in, int out,
              nfx::MlpLayer& L) {
    const auto& w = rt->model.weights.at(wname);
    const auto& b = rt->model.weights.at(bname);
    if (w.numel() != static_cast<int64_t>(in) * out || b.numel() < out) {
        rt->mo_why = wname + " does not hold the (" + std::to_string(out) + ", " + std::to_string(in) +
                     ") weight the configuration implies";
        return false;
    }
    L.w = upload(rt, w.data.data(), w.data.size());
    L.b = upload(rt, b.data.data(), b.data.size());
    L.in = in;
    L.out = out;
    if (!L.w || !L.b) {
        rt->mo_why = "weight upload failed";
        return false;
    }
    return true;
}

int deeponet_create(nfx_runtime* rt) {
    auto& m = rt->model;
    const int* c = m.cfg;
    const int in_b = c[0], in_t = c[1], lat = c[2], oc = c[3], nb = c[4], nt = c[5];
    const int act = m.activation == "relu" ? 1 : 0;
    // hidden widths from the second-to-last layer of each net (ir_loader.h:536-547)
    auto hidden = [&](const char* net, int n) {
        if (n < 2) return 0;
        const auto& w = m.weights.at(std::string(net) + ".layers." + std::to_string(n - 2) + ".weight");
        return w.shape.empty() ? 0 : static_cast<int>(w.shape[0]);
    };
    if (nb < 1 || nt < 1 || nb > nfx::kMlpMaxLayers || nt > nfx::kMlpMaxLayers) {
        rt->mo_why = "DeepONet GPU executor: 1 to 8 layers per net";
        rt->mo_code = NFX_UNSUPPORTED_OP;
        return NFX_OK;
    }
    const int hb = hidden("branch", nb), ht = hidden("trunk", nt);
    struct Net {
        const char* name;
        int n, in0, hid, last;
        nfx::MlpArgs* args;
    } nets[2] = {{"branch", nb, in_b, hb, oc * lat, &rt->mo_branch}, {"trunk", nt, in_t, ht, lat, &rt->mo_trunk}};
    for (const Net& net : nets) {
        nfx::MlpArgs& a = *net.args;
        a = nfx::MlpArgs{};
        a.n_layers = net.n;
        a.act = act;
        for (int i = 0; i < net.n; ++i) {
            const std::string pre = std::string(net.name) + ".layers." + std::to_string(i);
            const int in = i == 0 ? net.in0 : net.hid, out = i == net.n - 1 ? net.last : net.hid;
            if (!mo_layer(rt, pre + ".weight", pre + ".bias", in, out, a.layer[i])) {
                rt->mo_code = NFX_UNSUPPORTED_OP;
                return rt->mo_why == "weight upload failed" ? rt_fail(rt, NFX_INTERNAL, rt->mo_why) : NFX_OK;
            }
        }
        if (nfx::mlp_max_dim(a) > nfx::kMlpMaxDim) {
            rt->mo_why = "DeepONet GPU executor: layer widths above 512";
            rt->mo_code = NFX_UNSUPPORTED_OP;
            return NFX_OK;
        }
    }
    const auto& bias = m.weights.at("bias.weight");
    if (bias.numel() < oc) {
        rt->mo_why = "bias.weight holds fewer than out_channels values";
        rt->mo_code = NFX_UNSUPPORTED_OP;
        return NFX_OK;
    }
    rt->mo_bias = upload(rt, bias.data.data(), bias.data.size());
    if (!rt->mo_bias) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    return NFX_OK;
}

int graphop_create(nfx_runtime* rt) {
    auto& m = rt->model;
    const int* c = m.cfg;
    const bool two = m.op == "GraphOp2D";
    const int in_d = c[0], out_d = c[1];
    const int nodes = two ? c[2] * c[3] : c[2];
    const int hd = two ? c[4] : c[3], L = two ? c[5] : c[4];
    const int act = m.activation == "relu" ? 1 : 0;
    rt->mo_nodes = nodes;
    rt->mo_layers = L;
    if (L < 1) return NFX_OK;  // Run reports it (fno.cpp:1675-1677)
    if (L > nfx::kMlpMaxLayers || hd < 1 || hd > nfx::kGraphMaxHidden || in_d > nfx::kMlpMaxDim ||
        out_d > nfx::kMlpMaxDim) {
        rt->mo_why = m.op + " GPU executor: at most 8 blocks and hidden_dim <= 256";
        rt->mo_code = NFX_UNSUPPORTED_OP;
        return NFX_OK;
    }
    auto fail = [&]() {
        rt->mo_code = NFX_UNSUPPORTED_OP;
        return rt->mo_why == "weight upload failed" ? rt_fail(rt, NFX_INTERNAL, rt->mo_why) : NFX_OK;
    };
    rt->mo_lift = nfx::MlpArgs{};
    rt->mo_lift.n_layers = 1;
    rt->mo_head = rt->mo_lift;
    if (!mo_layer(rt, "lift.weight", "lift.bias", in_d, hd, rt->mo_lift.layer[0]) ||
        !mo_layer(rt, "head.weight", "head.bias", hd, out_d, rt->mo_head.layer[0]))
        return fail();
    for (int i = 0; i < L; ++i) {
        const std::string pre = "blocks." + std::to_string(i) + ".";
        nfx::MlpLayer ls{}, ln{};
        if (!mo_layer(rt, pre + "lin_self.weight", pre + "lin_self.bias", hd, hd, ls) ||
            !mo_layer(rt, pre + "lin_neigh.weight", pre + "lin_neigh.bias", hd, hd, ln))
            return fail();
        nfx::GraphLayerArgs& g = rt->mo_blocks[i];
        g = nfx::GraphLayerArgs{};
        g.n_nodes = nodes;
        g.hidden = hd;
        g.act = act;
        g.ws = ls.w;
        g.bs = ls.b;
        g.wn = ln.w;
        g.bn = ln.b;
    }
    // CSR adjacency: float tensors converted as the loader does (ir_loader.h:421-431)
    const auto& off = m.weights.at("graph.adj_offsets").data;
    const auto& idx = m.weights.at("graph.adj_indices").data;
    const auto& dinv = m.weights.at("graph.deg_inv").data;
    std::vector<int32_t> o32(off.size()), i32(idx.size());
    for (size_t k = 0; k < off.size(); ++k) o32[k] = static_cast<int32_t>(off[k]);
    for (size_t k = 0; k < idx.size(); ++k) i32[k] = static_cast<int32_t>(idx[k]);
    if (static_cast<int>(o32.size()) == nodes + 1 && static_cast<int>(dinv.size()) == nodes) {
        // the reference reads outside h for an index or offset out of range; the GPU
        // runtime refuses such a graph
        bool ok = o32[0] == 0;
        for (int k = 0; k < nodes && ok; ++k) ok = o32[k] <= o32[k + 1];
        ok = ok && o32[nodes] <= static_cast<int32_t>(i32.size());
        for (size_t k = 0; k < i32.size() && ok; ++k) ok = i32[k] >= 0 && i32[k] < nodes;
        if (!ok) {
            rt->mo_why = m.op + ": adjacency offsets or indices out of range";
            rt->mo_code = NFX_INVALID_ARG;
            return NFX_OK;
        }
    }
    const int* doff = upload(rt, o32.data(), o32.size());
    const int* didx = upload(rt, i32.data(), std::max<size_t>(i32.size(), 1));
    const float* ddeg = upload(rt, dinv.data(), std::max<size_t>(dinv.size(), 1));
    if (!doff || !didx || !ddeg) return rt_fail(rt, NFX_INTERNAL, "weight upload failed");
    for (int i = 0; i < L; ++i) {
        rt->mo_blocks[i].adj_off = doff;
        rt->mo_blocks[i].adj_idx = didx;
        rt->mo_blocks[i].deg_inv = ddeg;
    }
    return NFX_OK;
}

int ensure_mo_buf(nfx_runtime* rt, int i, int64_t floats) {
    if (floats <= rt->mo_cap[i]) return NFX_OK;
    if (rt->mo_bufs[i]) cudaFree(rt->mo_bufs[i]);
    rt->mo_bufs[i] = nullptr;
    rt->mo_cap[i] = 0;
    if (!cuda_ok(rt, cudaMalloc(&rt->mo_bufs[i], static_cast<size_t>(floats) * 4 + 256), "cudaMalloc activations"))
        return NFX_INTERNAL;
    rt->mo_cap[i] = floats;
    return NFX_OK;
}

// fno.cpp:1289-1311 (the reference's checks and messages), and u, y with one batch
int check_deeponet_shapes(nfx_runtime* rt, const int64_t* us, int ur, const int64_t* ys, int yr,
                          const int64_t* os, int orank) {
    const int* c = rt->model.cfg;
    if (ur != 3) return rt_fail(rt, NFX_SHAPE_MISMATCH, "DeepONet: expected 3D u (batch, n_sensor, in_branch)");
    if (yr != 3) return rt_fail(rt, NFX_SHAPE_MISMATCH, "DeepONet: expected 3D y (batch, n_query, in_trunk)");
    if (us[2] != c[0]) return rt_fail(rt, NFX_SHAPE_MISMATCH, "DeepONet: input branch feature dim mismatch");
    if (ys[2] != c[1]) return rt_fail(rt, NFX_SHAPE_MISMATCH, "DeepONet: input trunk feature dim mismatch");
    if (orank != 3 || os[0] != us[0] || os[1] != ys[1] || os[2] != c[3])
        return rt_fail(rt, NFX_SHAPE_MISMATCH, "DeepONet: output buffer shape mismatch");
    // the reference reads y with u's batch size
    if (ys[0] != us[0]) return rt_fail(rt, NFX_SHAPE_MISMATCH, "DeepONet: u and y batch sizes differ");
    if (!rt->mo_why.empty()) return rt_fail(rt, rt->mo_code ? rt->mo_code : NFX_UNSUPPORTED_OP, rt->mo_why);
    return NFX_OK;
}

int deeponet_launch(nfx_runtime* rt, const float* du, const int64_t* us, const float* dy, const int64_t* ys,
                    float* dout, cudaStream_t st) {
    const int* c = rt->model.cfg;
    const int64_t B = us[0], ns = us[1], nq = ys[1];
    const int F = c[3] * c[2];
    if (B == 0 || nq == 0) return NFX_OK;
    int s = ensure_mo_buf(rt, 0, B * ns * F);
    if (s == NFX_OK) s = ensure_mo_buf(rt, 1, B * F);
    if (s != NFX_OK) return s;
    float* bflat = static_cast<float*>(rt->mo_bufs[0]);
    float* bmean = static_cast<float*>(rt->mo_bufs[1]);
    nfx::MlpArgs br = rt->mo_branch;
    br.x = du;
    br.rows = B * ns;
    br.y = bflat;
    nfx::MeanArgs mean{bflat, bmean, B, static_cast<int>(ns), F};
    nfx::MlpArgs tr = rt->mo_trunk;
    tr.x = dy;
    tr.rows = B * nq;
    tr.y = dout;
    tr.dot_branch = bmean;
    tr.dot_bias = rt->mo_bias;
    tr.dot_ch = c[3];
    tr.rows_per_group = nq;
    cudaError_t e = cudaSuccess;
    auto* tm = rt->timer.get();
    if (tm) tm->begin("deeponet_branch", st);
    if (ns > 0) e = nfx::mlp_rows(br, st);
    if (tm) tm->end(st);
    if (e == cudaSuccess) {
        if (tm) tm->begin("deeponet_mean", st);
        e = nfx::sensor_mean(mean, st);
        if (tm) tm->end(st);
    }
    if (e == cudaSuccess) {
        if (tm) tm->begin("deeponet_trunk_dot", st);
        e = nfx::mlp_rows(tr, st);
        if (tm) tm->end(st);
    }
    if (e != cudaSuccess)
        return rt_fail(rt, NFX_INTERNAL, std::string("DeepONet launch failed: ") + cudaGetErrorString(e));
    return NFX_OK;
}

// fno.cpp:1653-1687 (GraphOp) and :1969-2010 (GraphOp2D): checks and messages
int check_graphop_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    const auto& m = rt->model;
    const int* c = m.cfg;
    const bool two = m.op == "GraphOp2D";
    const std::string& op = m.op;
    if (two) {
        if (xr != 4) return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp2D: expected 4D x (batch, h, w, in_dim)");
        if (xs[3] != c[0]) return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp2D: input feature dim mismatch");
        if (xs[1] != c[2] || xs[2] != c[3]) return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp2D: h / w mismatch");
        if (yr != 4 || ys[0] != xs[0] || ys[1] != xs[1] || ys[2] != xs[2] || ys[3] != c[1])
            return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp2D: output buffer shape mismatch");
    } else {
        if (xr != 3) return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp: expected 3D x (batch, n_nodes, in_dim)");
        if (xs[2] != c[0]) return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp: input feature dim mismatch");
        if (xs[1] != c[2]) return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp: n_nodes mismatch");
        if (yr != 3 || ys[0] != xs[0] || ys[1] != xs[1] || ys[2] != c[1])
            return rt_fail(rt, NFX_SHAPE_MISMATCH, "GraphOp: output buffer shape mismatch");
    }
    if (rt->mo_layers < 1) return rt_fail(rt, NFX_INVALID_ARG, op + ": n_layers must be >= 1");
    const int nodes = rt->mo_nodes;
    if (static_cast<int>(m.weights.at("graph.adj_offsets").data.size()) != nodes + 1)
        return rt_fail(rt, NFX_INTERNAL, op + ": adj_offsets size mismatch");
    if (static_cast<int>(m.weights.at("graph.deg_inv").data.size()) != nodes)
        return rt_fail(rt, NFX_INTERNAL, op + ": deg_inv size mismatch");
    if (!rt->mo_why.empty()) return rt_fail(rt, rt->mo_code ? rt->mo_code : NFX_UNSUPPORTED_OP, rt->mo_why);
    return NFX_OK;
}

int graphop_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st) {
    const int64_t B = xs[0];
    if (B == 0) return NFX_OK;
    const int64_t rows = B * rt->mo_nodes;
    const int hd = rt->mo_blocks[0].hidden;
    int s = ensure_mo_buf(rt, 0, rows * hd);
    if (s == NFX_OK) s = ensure_mo_buf(rt, 1, rows * hd);
    if (s != NFX_OK) return s;
    float* h[2] = {static_cast<float*>(rt->mo_bufs[0]), static_cast<float*>(rt->mo_bufs[1])};
    auto* tm = rt->timer.get();
    nfx::MlpArgs lift = rt->mo_lift;
    lift.x = dx;
    lift.rows = rows;
    lift.y = h[0];
    if (tm) tm->begin("graphop_lift", st);
    cudaError_t e = nfx::mlp_rows(lift, st);
    if (tm) tm->end(st);
    for (int i = 0; i < rt->mo_layers && e == cudaSuccess; ++i) {
        nfx::GraphLayerArgs g = rt->mo_blocks[i];
        g.h = h[i & 1];
        g.out = h[(i + 1) & 1];
        g.rows = rows;
        if (tm) tm->begin("graphop_block", st);
        e = nfx::graph_layer(g, st);
        if (tm) tm->end(st);
    }
    if (e == cudaSuccess) {
        nfx::MlpArgs head = rt->mo_head;
        head.x = h[rt->mo_layers & 1];
        head.rows = rows;
        head.y = dy;
        if (tm) tm->begin("graphop_head", st);
        e = nfx::mlp_rows(head, st);
        if (tm) tm->end(st);
    }
    if (e != cudaSuccess)
        return rt_fail(rt, NFX_INTERNAL, rt->model.op + " launch failed: " + cudaGetErrorString(e));
    return NFX_OK;
}

// ---------------------------------------------------------------------------
// op dispatch of Run / RunDevice
// ---------------------------------------------------------------------------
int check_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    if (rt->model.op == "FNO2d") return check_fno2d_shapes(rt, xs, xr, ys, yr);
    if (rt->model.op == "FNO1d") return check_fno1d_shapes(rt, xs, xr, ys, yr);
    if (rt->model.op == "FNO3d") return check_fno3d_shapes(rt, xs, xr, ys, yr);
    // runtime.cpp:97-100: Run serves the FNO family only
    return rt_fail(rt, NFX_INTERNAL, "runtime does not support op: " + rt->model.op);
}

int launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st) {
    if (rt->model.op == "FNO1d") return fno1d_launch(rt, dx, xs, dy, st);
    if (rt->model.op == "FNO3d") return fno3d_launch(rt, dx, xs, dy, st);
    return fno2d_launch(rt, dx, xs, dy, st);
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

int64_t numel(const int64_t* s, int r) {
    int64_t n = 1;
    for (int i = 0; i < r; ++i) n *= s[i];
    return n;
}

// Page-locked (pinned or registered) host memory, which the copy engines read and
// write asynchronously; ordinary pageable memory is not.
bool host_pinned(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeHost || a.type == cudaMemoryTypeManaged;
}

// Host-buffer Run for pageable x / y: per chunk, the copy pool moves the chunk's input
// into pinned staging, the copy engine takes it to the device, the chunk computes, the
// output comes back to pinned staging and the pool moves it to y.  The host copies of
// chunk c + 1 overlap the device copies and compute of chunk c, and the output copies
// of chunk c overlap the compute of the chunks after it.
int staged_run(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank, float* y,
               size_t nx, size_t ny, const int64_t* nbs, const int64_t* b0s, int nchunk) {
    if (nx > rt->hx_cap) {
        if (rt->calib_stats) cudaFree(rt->calib_stats);
    for (auto& t : rt->calib_vals)
        for (auto& c : t) cudaFree(c.first);
    if (rt->hx) cudaFreeHost(rt->hx);
        rt->hx = nullptr;
        rt->hx_cap = 0;
        if (!cuda_ok(rt, cudaHostAlloc(&rt->hx, nx * 4, cudaHostAllocDefault), "pinned staging"))
            return NFX_INTERNAL;
        rt->hx_cap = nx;
    }
    if (ny > rt->hy_cap) {
        if (rt->hy) cudaFreeHost(rt->hy);
        rt->hy = nullptr;
        rt->hy_cap = 0;
        if (!cuda_ok(rt, cudaHostAlloc(&rt->hy, ny * 4, cudaHostAllocDefault), "pinned staging"))
            return NFX_INTERNAL;
        rt->hy_cap = ny;
    }
    if (!rt->pool) {
        const int hw = static_cast<int>(std::thread::hardware_concurrency());
        rt->pool.reset(new nfx::CopyPool(std::max(0, std::min(7, hw / 2 - 1))));
    }
    const int64_t B = x_shape[0];
    const size_t xs = nx / static_cast<size_t>(B), ys = ny / static_cast<size_t>(B);
    int rc = NFX_OK;
    int issued = 0, drained = 0;
    auto drain = [&](int c) {
        const size_t yo = static_cast<size_t>(b0s[c]) * ys, yn = static_cast<size_t>(nbs[c]) * ys;
        rt->pool->copy(y + yo, rt->hy + yo, yn * 4);
    };
    for (int c = 0; c < nchunk && rc == NFX_OK; ++c) {
        // outputs that have already arrived leave staging between the input copies
        while (drained < issued && cudaEventQuery(rt->ev_done[drained]) == cudaSuccess) drain(drained++);
        const size_t xo = static_cast<size_t>(b0s[c]) * xs, yo = static_cast<size_t>(b0s[c]) * ys;
        const size_t xn = static_cast<size_t>(nbs[c]) * xs, yn = static_cast<size_t>(nbs[c]) * ys;
        rt->pool->copy(rt->hx + xo, x + xo, xn * 4);
        std::vector<int64_t> shp(x_shape, x_shape + x_rank);
        shp[0] = nbs[c];
        if (!cuda_ok(rt, cudaMemcpyAsync(rt->dx + xo, rt->hx + xo, xn * 4, cudaMemcpyHostToDevice, rt->s_h2d),
                     "H2D") ||
            !cuda_ok(rt, cudaEventRecord(rt->ev_in[c], rt->s_h2d), "event") ||
            !cuda_ok(rt, cudaStreamWaitEvent(rt->stream, rt->ev_in[c], 0), "event wait")) {
            rc = NFX_INTERNAL;
            break;
        }
        rc = launch(rt, rt->dx + xo, shp.data(), rt->dy + yo, rt->stream);
        if (rc != NFX_OK) break;
        if (!cuda_ok(rt, cudaEventRecord(rt->ev_out[c], rt->stream), "event") ||
            !cuda_ok(rt, cudaStreamWaitEvent(rt->s_d2h, rt->ev_out[c], 0), "event wait") ||
            !cuda_ok(rt, cudaMemcpyAsync(rt->hy + yo, rt->dy + yo, yn * 4, cudaMemcpyDeviceToHost, rt->s_d2h),
                     "D2H") ||
            !cuda_ok(rt, cudaEventRecord(rt->ev_done[c], rt->s_d2h), "event")) {
            rc = NFX_INTERNAL;
            break;
        }
        issued = c + 1;
    }
    for (int c = drained; c < issued && rc == NFX_OK; ++c) {
        if (!cuda_ok(rt, cudaEventSynchronize(rt->ev_done[c]), "output copy")) {
            rc = NFX_INTERNAL;
            break;
        }
        drain(c);
    }
    // every queued copy and kernel ends before Run returns, also on the error path
    const bool synced = cuda_ok(rt, cudaStreamSynchronize(rt->s_h2d), "input copy") &&
                        cuda_ok(rt, cudaStreamSynchronize(rt->stream), "execution") &&
                        cuda_ok(rt, cudaStreamSynchronize(rt->s_d2h), "output copy");
    if (rc != NFX_OK) return rc;
    if (!synced) return NFX_INTERNAL;
    return nfx_runtime_check(rt);
}

}  // namespace

namespace nfx {

// Helpers of the allocation-free entry point (noalloc.cu).  They validate the call
// exactly as nfx_runtime_run_device does and copy the handle's weight plan, without
// touching the handle's on-demand buffers.
int runtime_device(const nfx_runtime* rt) { return rt->device; }

int runtime_fail(nfx_runtime* rt, int code, const char* msg) { return rt_fail(rt, code, msg); }

// Helpers of the multi-GPU entry points (nfx_multi.cpp).
int runtime_check_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr) {
    if (!xs || !ys) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    return check_shapes(rt, xs, xr, ys, yr);
}

int runtime_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st) {
    return launch(rt, dx, xs, dy, st);
}

cudaStream_t runtime_stream(nfx_runtime* rt) { return rt->stream; }

// The handle's device staging buffers, grown to hold nx input and ny output floats.
int runtime_staging(nfx_runtime* rt, size_t nx, size_t ny, float** dx, float** dy) {
    if (nx > rt->dx_cap) {
        if (rt->dx) cudaFree(rt->dx);
        rt->dx = nullptr;
        rt->dx_cap = 0;
        if (!cuda_ok(rt, cudaMalloc(&rt->dx, nx * 4), "cudaMalloc input")) return NFX_INTERNAL;
        rt->dx_cap = nx;
    }
    if (ny > rt->dy_cap) {
        if (rt->dy) cudaFree(rt->dy);
        rt->dy = nullptr;
        rt->dy_cap = 0;
        if (!cuda_ok(rt, cudaMalloc(&rt->dy, ny * 4), "cudaMalloc output")) return NFX_INTERNAL;
        rt->dy_cap = ny;
    }
    *dx = rt->dx;
    *dy = rt->dy;
    return NFX_OK;
}

int runtime_fail_str(nfx_runtime* rt, int code, const std::string& msg) { return rt_fail(rt, code, msg); }

// ---- calibration (nfx_calib.cu) --------------------------------------------------
// Observed tensors of an FNO2d handle: lift, locs.0 .. locs.L-1, proj_q, proj_out.
int calib_tensors(const nfx_runtime* rt) {
    if (rt->model.op != "FNO2d") return 0;
    return fno2d_cfg(rt->model).L + 3;
}

std::string calib_name(const nfx_runtime* rt, int i) {
    const int L = fno2d_cfg(rt->model).L;
    if (i == 0) return "lift.output";
    if (i <= L) return "locs." + std::to_string(i - 1) + ".output";
    return i == L + 1 ? "proj_q.output" : "proj_out.output";
}

unsigned*& calib_stats(nfx_runtime* rt) { return rt->calib_stats; }
int& calib_keep(nfx_runtime* rt) { return rt->calib_keep; }
std::vector<std::vector<std::pair<float*, int64_t>>>& calib_vals(nfx_runtime* rt) { return rt->calib_vals; }

// One calibration batch (host x): the FP32 network without fake-quant, observing every
// Linear output; with kept values, each tensor's values go to a new device chunk.
int calib_observe(nfx_runtime* rt, const float* x, const int64_t* xs, int xr) {
    if (rt->model.op != "FNO2d" || rt->int8_enabled)
        return rt_fail(rt, NFX_UNSUPPORTED_OP,
                       "calibration observes the FP32 FNO2d network: create the runtime without "
                       "EnableInt8Gemm");
    if (!rt->calib_stats) return rt_fail(rt, NFX_INVALID_ARG, "call nfx_calibrate_begin first");
    const F2 c = fno2d_cfg(rt->model);
    if (!xs || xr != 4) return rt_fail(rt, NFX_SHAPE_MISMATCH, "expected 4D input (batch, h, w, in_ch)");
    const int64_t ys[4] = {xs[0], xs[1], xs[2], c.out_ch};
    int s = check_fno2d_shapes(rt, xs, xr, ys, 4);
    if (s != NFX_OK) return s;
    const int64_t B = xs[0], H = xs[1], W = xs[2];
    if (B == 0) return NFX_OK;
    if (!x) return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    int64_t Hp = H, Wp = W;
    if (c.pad > 1) {
        Hp = H + (c.pad - H % c.pad) % c.pad;
        Wp = W + (c.pad - W % c.pad) % c.pad;
    }
    const size_t nx = static_cast<size_t>(B * H * W * c.in_ch), ny = static_cast<size_t>(B * H * W * c.out_ch);
    float* dx = nullptr;
    float* dy = nullptr;
    s = nfx::runtime_staging(rt, nx, ny, &dx, &dy);
    if (s != NFX_OK) return s;
    float* vals[kFno2dObsMax] = {};
    const int n = c.L + 3;
    if (rt->calib_keep) {
        for (int i = 0; i < n; ++i) {
            const int64_t cnt = i == 0 ? B * H * W * c.width
                                : i <= c.L ? B * Hp * Wp * c.width
                                : i == c.L + 1 ? B * H * W * c.width : B * H * W * c.out_ch;
            void* p = nullptr;
            if (!cuda_ok(rt, cudaMalloc(&p, static_cast<size_t>(cnt) * 4), "cudaMalloc calibration values"))
                return NFX_INTERNAL;
            vals[i] = static_cast<float*>(p);
            rt->calib_vals[i].push_back({vals[i], cnt});
        }
    }
    if (!cuda_ok(rt, cudaMemcpyAsync(dx, x, nx * 4, cudaMemcpyHostToDevice, rt->stream), "H2D")) return NFX_INTERNAL;
    s = fno2d_f32_launch(rt, dx, xs, dy, rt->stream, rt->calib_stats, vals);
    if (s != NFX_OK) return s;
    if (!cuda_ok(rt, cudaStreamSynchronize(rt->stream), "calibration batch")) return NFX_INTERNAL;
    return nfx_runtime_check(rt);
}

int fno2d_noalloc_plan(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                       float* y, const int64_t* y_shape, int y_rank, Fno2dPlan* plan) {
    if (!x_shape || !y_shape) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    if (rt->model.op != "FNO2d")
        return rt_fail(rt, NFX_UNSUPPORTED_OP, "the allocation-free entry point runs FNO2d");
    int s = check_fno2d_shapes(rt, x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return s;
    const F2 c = fno2d_cfg(rt->model);
    if (!rt->int8_enabled)
        return rt_fail(rt, NFX_UNSUPPORTED_OP,
                       "the allocation-free entry point runs the FNO2d INT8 path: call EnableInt8Gemm() first");
    if (!rt->f2_fast)
        return rt_fail(rt, NFX_UNSUPPORTED_OP,
                       "the allocation-free entry point runs the width-64 12x12 FNO2d INT8 executor");
    const int B = static_cast<int>(x_shape[0]), H = static_cast<int>(x_shape[1]),
              W = static_cast<int>(x_shape[2]);
    if (W < 32 || W > 128 || H < 8 || H > 4096 || c.mh > H || c.mw > W / 2 + 1)
        return rt_fail(rt, NFX_UNSUPPORTED_OP,
                       "FNO2d GPU executor: needs 32 <= W <= 128, H >= 8, modes within the grid");
    if (c.pad > 1 && ((H % c.pad) || (W % c.pad)))
        return rt_fail(rt, NFX_UNSUPPORTED_OP, "FNO2d GPU executor: padding is not supported");
    if (B > 0 && (!x || !y)) return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    *plan = rt->plan;
    plan->B = B;
    plan->H = H;
    plan->W = W;
    plan->HB = H / nfx::fno2d_row_blocks(H);
    plan->x = x;
    plan->y = y;
    plan->fwd_limbs = nullptr;  // the caller places the transform tables
    plan->fwd_sum_b = nullptr;
    plan->timer = nullptr;
    plan->tap_codes = nullptr;
    return NFX_OK;
}

}  // namespace nfx

extern "C" {

int nfx_runtime_create(const char* ir_path, int device, nfx_runtime** out) {
    if (!out) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_runtime_create: out is NULL");
    *out = nullptr;
    if (!ir_path) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_runtime_create: path is NULL");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_runtime_create: no such CUDA device");
    std::unique_ptr<nfx_runtime> rt(new nfx_runtime());
    rt->device = device;
    std::string msg;
    int s = nfx::load_ir(ir_path, rt->model, msg);
    if (s != NFX_OK) return nfx::set_thread_error(s, msg);
    const auto& op = rt->model.op;
    if (op != "FNO1d" && op != "FNO2d" && op != "FNO3d" && op != "DeepONet" && op != "TokenMixer" &&
        op != "GraphOp" && op != "TokenMixer2D" && op != "GraphOp2D")
        return nfx::set_thread_error(NFX_UNSUPPORTED_OP, "runtime does not support op: " + op);
    DeviceGuard g(device);
    if (cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking) != cudaSuccess)
        return nfx::set_thread_error(NFX_INTERNAL, "cudaStreamCreate failed");
    if (op == "FNO2d") {
        s = fno2d_create(rt.get());
        if (s != NFX_OK) return nfx::set_thread_error(s, rt->err);
    } else if (op == "FNO1d") {
        s = fno1d_create(rt.get());
        if (s != NFX_OK) return nfx::set_thread_error(s, rt->err);
    } else if (op == "FNO3d") {
        s = fno3d_create(rt.get());
        if (s != NFX_OK) return nfx::set_thread_error(s, rt->err);
    } else if (op == "TokenMixer2D" || op == "TokenMixer") {
        s = tm2d_create(rt.get());
        if (s != NFX_OK) return nfx::set_thread_error(s, rt->err);
    } else if (op == "DeepONet") {
        s = deeponet_create(rt.get());
        if (s != NFX_OK) return nfx::set_thread_error(s, rt->err);
    } else if (op == "GraphOp" || op == "GraphOp2D") {
        s = graphop_create(rt.get());
        if (s != NFX_OK) return nfx::set_thread_error(s, rt->err);
    }
    if (!nfx::device_error_word())
        return nfx::set_thread_error(NFX_INTERNAL, "cannot allocate the device error word");
    *out = rt.release();
    return NFX_OK;
}

int nfx_load_neuroir(const char* ir_path, char* op_out, int op_cap, int32_t* cfg_out8,
                     int* n_weights_out, int* quant_enabled_out) {
    if (!ir_path) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_load_neuroir: path is NULL");
    nfx::IrModel m;
    std::string msg;
    const int s = nfx::load_ir(ir_path, m, msg);
    if (s != NFX_OK) return nfx::set_thread_error(s, msg);
    if (op_out && op_cap > 0) {
        const size_t n = std::min(static_cast<size_t>(op_cap - 1), m.op.size());
        std::memcpy(op_out, m.op.data(), n);
        op_out[n] = 0;
    }
    if (cfg_out8)
        for (int i = 0; i < 8; ++i) cfg_out8[i] = m.cfg[i];
    if (n_weights_out) *n_weights_out = static_cast<int>(m.weight_order.size());
    if (quant_enabled_out) *quant_enabled_out = m.quant_enabled ? 1 : 0;
    return NFX_OK;
}

void nfx_runtime_destroy(nfx_runtime* rt) {
    if (!rt) return;
    DeviceGuard g(rt->device);
    cudaDeviceSynchronize();
    for (void* p : rt->allocs) cudaFree(p);
    for (void* p : rt->act_bufs)
        if (p) cudaFree(p);
    for (auto* p : rt->tw)
        if (p) cudaFree(p);
    for (void* p : rt->f1_bufs)
        if (p) cudaFree(p);
    for (void* p : rt->f2_bufs)
        if (p) cudaFree(p);
    for (void* p : rt->tm_bufs)
        if (p) cudaFree(p);
    for (void* p : rt->mo_bufs)
        if (p) cudaFree(p);
    for (void* p : rt->f3_bufs)
        if (p) cudaFree(p);
    for (auto* p : rt->f3_tw)
        if (p) cudaFree(p);
    if (rt->f3_dft) cudaFree(rt->f3_dft);
    for (auto* p : rt->f2_tw)
        if (p) cudaFree(p);
    for (auto* p : rt->f1_tw)
        if (p) cudaFree(p);
    if (rt->fwd_limbs) cudaFree(rt->fwd_limbs);
    if (rt->fwd_sum_b) cudaFree(rt->fwd_sum_b);
    if (rt->dx) cudaFree(rt->dx);
    if (rt->dy) cudaFree(rt->dy);
    if (rt->stream) cudaStreamDestroy(rt->stream);
    if (rt->s_h2d) cudaStreamDestroy(rt->s_h2d);
    if (rt->s_d2h) cudaStreamDestroy(rt->s_d2h);
    for (int i = 0; i < 8; ++i) {
        if (rt->ev_in[i]) cudaEventDestroy(rt->ev_in[i]);
        if (rt->ev_out[i]) cudaEventDestroy(rt->ev_out[i]);
        if (rt->ev_done[i]) cudaEventDestroy(rt->ev_done[i]);
    }
    if (rt->calib_stats) cudaFree(rt->calib_stats);
    for (auto& t : rt->calib_vals)
        for (auto& c : t) cudaFree(c.first);
    if (rt->hx) cudaFreeHost(rt->hx);
    if (rt->hy) cudaFreeHost(rt->hy);
    rt->pool.reset();
    rt->timer.reset();
    delete rt;
}

int nfx_runtime_profile_enable(nfx_runtime* rt, int enable) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    DeviceGuard g(rt->device);
    if (enable) {
        if (!rt->timer) rt->timer.reset(new nfx::EventTimer());
        rt->timer->reset();
    } else {
        rt->timer.reset();
    }
    return NFX_OK;
}

int nfx_runtime_profile_count(nfx_runtime* rt) {
    if (!rt || !rt->timer) return 0;
    DeviceGuard g(rt->device);
    rt->timer->collect();
    return static_cast<int>(rt->timer->names.size());
}

int nfx_runtime_profile_entry(nfx_runtime* rt, int i, const char** name, int* launches,
                              double* total_ms) {
    if (!rt || !rt->timer) return rt_fail(rt, NFX_INVALID_ARG, "profiling is not enabled");
    DeviceGuard g(rt->device);
    rt->timer->collect();
    if (i < 0 || i >= static_cast<int>(rt->timer->names.size()))
        return rt_fail(rt, NFX_INVALID_ARG, "profile entry out of range");
    if (name) *name = rt->timer->names[i].c_str();
    if (launches) *launches = rt->timer->launches[i];
    if (total_ms) *total_ms = rt->timer->total_ms[i];
    return NFX_OK;
}

const char* nfx_runtime_op(const nfx_runtime* rt) { return rt ? rt->model.op.c_str() : ""; }

void nfx_runtime_enable_int8_gemm(nfx_runtime* rt) {
    if (!rt) return;
    DeviceGuard g(rt->device);
    if (rt->model.op == "FNO2d") fno2d_enable_int8(rt);
    if (rt->model.op == "FNO1d") fno1d_enable_int8(rt);
    if (rt->model.op == "TokenMixer2D" || rt->model.op == "TokenMixer") tm2d_enable_int8(rt);
}

int nfx_runtime_is_int8_gemm_enabled(const nfx_runtime* rt) { return rt && rt->int8_enabled ? 1 : 0; }

const char* nfx_runtime_last_error(const nfx_runtime* rt) { return rt ? rt->err.c_str() : ""; }

int nfx_runtime_run_device(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                           float* y, const int64_t* y_shape, int y_rank, void* stream) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!x_shape || !y_shape) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    DeviceGuard g(rt->device);
    int s = check_shapes(rt, x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return s;
    if (numel(x_shape, x_rank) > 0 && (!x || !y)) return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    return launch(rt, x, x_shape, y, static_cast<cudaStream_t>(stream));
}

int nfx_runtime_set_code_taps(nfx_runtime* rt, int8_t* device_buffer, int64_t capacity_bytes) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (device_buffer && capacity_bytes <= 0) return rt_fail(rt, NFX_INVALID_ARG, "tap capacity must be > 0");
    rt->tap_codes = device_buffer;
    rt->tap_cap = device_buffer ? capacity_bytes : 0;
    return NFX_OK;
}

int nfx_runtime_check(nfx_runtime* rt) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    DeviceGuard g(rt->device);
    if (!cuda_ok(rt, cudaDeviceSynchronize(), "device error")) return NFX_INTERNAL;
    unsigned* w = nfx::device_error_word();
    unsigned v = 0;
    if (!w || !cuda_ok(rt, cudaMemcpy(&v, w, 4, cudaMemcpyDeviceToHost), "error word read"))
        return NFX_INTERNAL;
    if (v) {
        cudaMemset(w, 0, 4);
        return rt_fail(rt, NFX_INTERNAL,
                       "a kernel gave up waiting (device error flags 0x" + std::to_string(v) + ")");
    }
    return NFX_OK;
}

int nfx_runtime_run(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank, float* y,
                    const int64_t* y_shape, int y_rank) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!x_shape || !y_shape) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    DeviceGuard g(rt->device);
    int s = check_shapes(rt, x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return s;
    const size_t nx = static_cast<size_t>(numel(x_shape, x_rank));
    const size_t ny = static_cast<size_t>(numel(y_shape, y_rank));
    if (nx == 0) return NFX_OK;
    if (!x || !y) return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    if (nx > rt->dx_cap) {
        if (rt->dx) cudaFree(rt->dx);
        rt->dx = nullptr;
        if (!cuda_ok(rt, cudaMalloc(&rt->dx, nx * 4), "cudaMalloc input")) return NFX_INTERNAL;
        rt->dx_cap = nx;
    }
    if (ny > rt->dy_cap) {
        if (rt->dy) cudaFree(rt->dy);
        rt->dy = nullptr;
        if (!cuda_ok(rt, cudaMalloc(&rt->dy, ny * 4), "cudaMalloc output")) return NFX_INTERNAL;
        rt->dy_cap = ny;
    }
    // Samples are independent, so a large batch runs as several chunks: the input copy
    // of chunk c+1 and the output copy of chunk c-1 overlap the compute of chunk c (the
    // copy engines of both directions and the SMs work at once; with pinned host
    // buffers the copies are truly asynchronous).  Nothing hides the first chunk's
    // input copy and the last chunk's output copy, so both chunks are small (q / 2 and
    // q); the ones between are 2q, 4q, ... (an input copy must finish within the
    // previous chunk's compute, which takes about 2.5x as long per sample).  With q =
    // SMs / gcd(SMs, 4) samples the middle chunks fill whole rounds of the persistent
    // kernels' units (4 row blocks or 128 points per sample).
    const int64_t B = x_shape[0];
    int64_t nbs[8], b0s[8];
    int nchunk = 1;
    nbs[0] = B;
    {
        const int sms = nfx::device_sm_count();
        int g = 4, a = sms > 0 ? sms : 4;
        while (a % g) --g;  // gcd(sms, 4)
        const int64_t q = std::max<int64_t>(8, (sms > 0 ? sms : 32) / g);
        if (B >= 4 * q) {
            nchunk = 0;
            const int64_t first = (q + 1) / 2;
            nbs[nchunk++] = first;
            int64_t rem = B - first - q, step = 2 * q;
            while (rem > 0) {
                int64_t take = std::min(step, rem);
                if (rem - take < q / 2 || nchunk == 6) take = rem;
                nbs[nchunk++] = take;
                rem -= take;
                step *= 2;
            }
            nbs[nchunk++] = q;
        } else if (B >= 32) {
            nchunk = 2;
            nbs[0] = B / 2;
            nbs[1] = B - B / 2;
        }
        b0s[0] = 0;
        for (int c = 1; c < nchunk; ++c) b0s[c] = b0s[c - 1] + nbs[c - 1];
    }
    // Pageable (ordinary) caller memory cannot feed the copy engines asynchronously:
    // such buffers are staged through pinned copies (staged_run below).
    const bool staged = !host_pinned(x) || !host_pinned(y);
    if ((nchunk > 1 || staged) && !rt->s_h2d) {
        bool ok = cudaStreamCreateWithFlags(&rt->s_h2d, cudaStreamNonBlocking) == cudaSuccess &&
                  cudaStreamCreateWithFlags(&rt->s_d2h, cudaStreamNonBlocking) == cudaSuccess;
        for (int i = 0; i < 8 && ok; ++i)
            ok = cudaEventCreateWithFlags(&rt->ev_in[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&rt->ev_out[i], cudaEventDisableTiming) == cudaSuccess &&
                 cudaEventCreateWithFlags(&rt->ev_done[i], cudaEventDisableTiming) == cudaSuccess;
        if (!ok) return rt_fail(rt, NFX_INTERNAL, "creating the copy streams failed");
    }
    if (staged) return staged_run(rt, x, x_shape, x_rank, y, nx, ny, nbs, b0s, nchunk);
    if (nchunk == 1) {
        if (!cuda_ok(rt, cudaMemcpyAsync(rt->dx, x, nx * 4, cudaMemcpyHostToDevice, rt->stream), "H2D"))
            return NFX_INTERNAL;
        s = launch(rt, rt->dx, x_shape, rt->dy, rt->stream);
        if (s != NFX_OK) return s;
        if (!cuda_ok(rt, cudaMemcpyAsync(y, rt->dy, ny * 4, cudaMemcpyDeviceToHost, rt->stream), "D2H"))
            return NFX_INTERNAL;
        if (!cuda_ok(rt, cudaStreamSynchronize(rt->stream), "execution")) return NFX_INTERNAL;
        return nfx_runtime_check(rt);
    }
    const size_t xs = nx / static_cast<size_t>(B), ys = ny / static_cast<size_t>(B);
    for (int c = 0; c < nchunk; ++c) {
        const size_t off = static_cast<size_t>(b0s[c]) * xs;
        if (!cuda_ok(rt, cudaMemcpyAsync(rt->dx + off, x + off, static_cast<size_t>(nbs[c]) * xs * 4,
                                         cudaMemcpyHostToDevice, rt->s_h2d), "H2D") ||
            !cuda_ok(rt, cudaEventRecord(rt->ev_in[c], rt->s_h2d), "event"))
            return NFX_INTERNAL;
    }
    int rc = NFX_OK;
    for (int c = 0; c < nchunk && rc == NFX_OK; ++c) {
        std::vector<int64_t> shp(x_shape, x_shape + x_rank);
        shp[0] = nbs[c];
        const size_t xo = static_cast<size_t>(b0s[c]) * xs, yo = static_cast<size_t>(b0s[c]) * ys;
        if (!cuda_ok(rt, cudaStreamWaitEvent(rt->stream, rt->ev_in[c], 0), "event wait")) {
            rc = NFX_INTERNAL;
            break;
        }
        rc = launch(rt, rt->dx + xo, shp.data(), rt->dy + yo, rt->stream);
        if (rc != NFX_OK) break;
        if (!cuda_ok(rt, cudaEventRecord(rt->ev_out[c], rt->stream), "event") ||
            !cuda_ok(rt, cudaStreamWaitEvent(rt->s_d2h, rt->ev_out[c], 0), "event wait") ||
            !cuda_ok(rt, cudaMemcpyAsync(y + yo, rt->dy + yo, static_cast<size_t>(nbs[c]) * ys * 4,
                                         cudaMemcpyDeviceToHost, rt->s_d2h), "D2H"))
            rc = NFX_INTERNAL;
    }
    // every queued copy and kernel ends before Run returns, also on the error path
    const bool synced = cuda_ok(rt, cudaStreamSynchronize(rt->s_h2d), "input copy") &&
                        cuda_ok(rt, cudaStreamSynchronize(rt->stream), "execution") &&
                        cuda_ok(rt, cudaStreamSynchronize(rt->s_d2h), "output copy");
    if (rc != NFX_OK) return rc;
    if (!synced) return NFX_INTERNAL;
    return nfx_runtime_check(rt);
}

void nfx_runtime_enable_fp8(nfx_runtime* rt) {
    if (!rt) return;
    DeviceGuard g(rt->device);
    if (rt->model.op == "FNO3d") fno3d_enable_fp8(rt);
}

int nfx_runtime_is_fp8_enabled(const nfx_runtime* rt) { return rt && rt->fp8_enabled ? 1 : 0; }

}  // extern "C"

namespace {

// Single-input ops outside Run (RunTokenMixer2D, RunTokenMixer, RunGraphOp,
// RunGraphOp2D; runtime.cpp:115-153): the op's shape checks, then its launcher on
// device buffers, or through the runtime's device staging for host buffers.
using OpCheck = int (*)(nfx_runtime*, const int64_t*, int, const int64_t*, int);
using OpLaunch = int (*)(nfx_runtime*, const float*, const int64_t*, float*, cudaStream_t);

bool op_is(const nfx_runtime* rt, const char* a, const char* b = nullptr) {
    return rt->model.op == a || (b && rt->model.op == b);
}

int run_other_device(nfx_runtime* rt, const char* op, bool ok_op, OpCheck check, OpLaunch launch_fn,
                     const float* x, const int64_t* x_shape, int x_rank, float* y, const int64_t* y_shape,
                     int y_rank, void* stream) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!x_shape || !y_shape) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    DeviceGuard g(rt->device);
    if (!ok_op) return rt_fail(rt, NFX_INTERNAL, std::string(op) + " not initialized");
    int s = check(rt, x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return s;
    if (numel(x_shape, x_rank) > 0 && (!x || !y)) return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    return launch_fn(rt, x, x_shape, y, static_cast<cudaStream_t>(stream));
}

int ensure_staging(nfx_runtime* rt, size_t nx, size_t ny) {
    if (nx > rt->dx_cap) {
        if (rt->dx) cudaFree(rt->dx);
        rt->dx = nullptr;
        if (!cuda_ok(rt, cudaMalloc(&rt->dx, nx * 4), "cudaMalloc input")) return NFX_INTERNAL;
        rt->dx_cap = nx;
    }
    if (ny > rt->dy_cap) {
        if (rt->dy) cudaFree(rt->dy);
        rt->dy = nullptr;
        if (!cuda_ok(rt, cudaMalloc(&rt->dy, ny * 4), "cudaMalloc output")) return NFX_INTERNAL;
        rt->dy_cap = ny;
    }
    return NFX_OK;
}

int run_other_host(nfx_runtime* rt, const char* op, bool ok_op, OpCheck check, OpLaunch launch_fn,
                   const float* x, const int64_t* x_shape, int x_rank, float* y, const int64_t* y_shape,
                   int y_rank) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!x_shape || !y_shape) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    DeviceGuard g(rt->device);
    if (!ok_op) return rt_fail(rt, NFX_INTERNAL, std::string(op) + " not initialized");
    int s = check(rt, x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return s;
    const size_t nx = static_cast<size_t>(numel(x_shape, x_rank));
    const size_t ny = static_cast<size_t>(numel(y_shape, y_rank));
    if (nx == 0 || ny == 0) return NFX_OK;
    if (!x || !y) return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    s = ensure_staging(rt, nx, ny);
    if (s != NFX_OK) return s;
    if (!cuda_ok(rt, cudaMemcpyAsync(rt->dx, x, nx * 4, cudaMemcpyHostToDevice, rt->stream), "H2D"))
        return NFX_INTERNAL;
    s = launch_fn(rt, rt->dx, x_shape, rt->dy, rt->stream);
    if (s != NFX_OK) {
        cudaStreamSynchronize(rt->stream);
        return s;
    }
    if (!cuda_ok(rt, cudaMemcpyAsync(y, rt->dy, ny * 4, cudaMemcpyDeviceToHost, rt->stream), "D2H"))
        return NFX_INTERNAL;
    if (!cuda_ok(rt, cudaStreamSynchronize(rt->stream), "execution")) return NFX_INTERNAL;
    return nfx_runtime_check(rt);
}

}  // namespace

extern "C" {

int nfx_runtime_run_tokenmixer2d_device(nfx_runtime* rt, const float* x, const int64_t* x_shape,
                                        int x_rank, float* y, const int64_t* y_shape, int y_rank,
                                        void* stream) {
    return run_other_device(rt, "TokenMixer2D", rt && op_is(rt, "TokenMixer2D"), check_tm2d_shapes, tm2d_launch,
                            x, x_shape, x_rank, y, y_shape, y_rank, stream);
}

int nfx_runtime_run_tokenmixer2d(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                                 float* y, const int64_t* y_shape, int y_rank) {
    return run_other_host(rt, "TokenMixer2D", rt && op_is(rt, "TokenMixer2D"), check_tm2d_shapes, tm2d_launch, x,
                          x_shape, x_rank, y, y_shape, y_rank);
}

int nfx_runtime_run_tokenmixer_device(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                                      float* y, const int64_t* y_shape, int y_rank, void* stream) {
    return run_other_device(rt, "TokenMixer", rt && op_is(rt, "TokenMixer"), check_tm2d_shapes, tm2d_launch, x,
                            x_shape, x_rank, y, y_shape, y_rank, stream);
}

int nfx_runtime_run_tokenmixer(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank, float* y,
                               const int64_t* y_shape, int y_rank) {
    return run_other_host(rt, "TokenMixer", rt && op_is(rt, "TokenMixer"), check_tm2d_shapes, tm2d_launch, x,
                          x_shape, x_rank, y, y_shape, y_rank);
}

int nfx_runtime_run_graphop_device(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                                   float* y, const int64_t* y_shape, int y_rank, void* stream) {
    return run_other_device(rt, "GraphOp", rt && op_is(rt, "GraphOp"), check_graphop_shapes, graphop_launch, x,
                            x_shape, x_rank, y, y_shape, y_rank, stream);
}

int nfx_runtime_run_graphop(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank, float* y,
                            const int64_t* y_shape, int y_rank) {
    return run_other_host(rt, "GraphOp", rt && op_is(rt, "GraphOp"), check_graphop_shapes, graphop_launch, x,
                          x_shape, x_rank, y, y_shape, y_rank);
}

int nfx_runtime_run_graphop2d_device(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                                     float* y, const int64_t* y_shape, int y_rank, void* stream) {
    return run_other_device(rt, "GraphOp2D", rt && op_is(rt, "GraphOp2D"), check_graphop_shapes, graphop_launch,
                            x, x_shape, x_rank, y, y_shape, y_rank, stream);
}

int nfx_runtime_run_graphop2d(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank, float* y,
                              const int64_t* y_shape, int y_rank) {
    return run_other_host(rt, "GraphOp2D", rt && op_is(rt, "GraphOp2D"), check_graphop_shapes, graphop_launch, x,
                          x_shape, x_rank, y, y_shape, y_rank);
}

int nfx_runtime_run_deeponet_device(nfx_runtime* rt, const float* u, const int64_t* u_shape, int u_rank,
                                    const float* y, const int64_t* y_shape, int y_rank, float* out,
                                    const int64_t* out_shape, int out_rank, void* stream) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!u_shape || !y_shape || !out_shape) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    DeviceGuard g(rt->device);
    if (!op_is(rt, "DeepONet")) return rt_fail(rt, NFX_INTERNAL, "DeepONet not initialized");
    int s = check_deeponet_shapes(rt, u_shape, u_rank, y_shape, y_rank, out_shape, out_rank);
    if (s != NFX_OK) return s;
    if (numel(out_shape, out_rank) > 0 && (!y || !out || (numel(u_shape, u_rank) > 0 && !u)))
        return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    return deeponet_launch(rt, u, u_shape, y, y_shape, out, static_cast<cudaStream_t>(stream));
}

// runtime.cpp:103-113 RunDeepONet on host buffers: u and y staged one after the other
int nfx_runtime_run_deeponet(nfx_runtime* rt, const float* u, const int64_t* u_shape, int u_rank,
                             const float* y, const int64_t* y_shape, int y_rank, float* out,
                             const int64_t* out_shape, int out_rank) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!u_shape || !y_shape || !out_shape) return rt_fail(rt, NFX_INVALID_ARG, "null shape");
    DeviceGuard g(rt->device);
    if (!op_is(rt, "DeepONet")) return rt_fail(rt, NFX_INTERNAL, "DeepONet not initialized");
    int s = check_deeponet_shapes(rt, u_shape, u_rank, y_shape, y_rank, out_shape, out_rank);
    if (s != NFX_OK) return s;
    const size_t nu = static_cast<size_t>(numel(u_shape, u_rank));
    const size_t ny = static_cast<size_t>(numel(y_shape, y_rank));
    const size_t no = static_cast<size_t>(numel(out_shape, out_rank));
    if (no == 0) return NFX_OK;
    if (!y || !out || (nu > 0 && !u)) return rt_fail(rt, NFX_INVALID_ARG, "null buffer");
    s = ensure_staging(rt, nu + ny, no);
    if (s != NFX_OK) return s;
    float* du = rt->dx;
    float* dyq = rt->dx + nu;
    if ((nu > 0 && !cuda_ok(rt, cudaMemcpyAsync(du, u, nu * 4, cudaMemcpyHostToDevice, rt->stream), "H2D")) ||
        !cuda_ok(rt, cudaMemcpyAsync(dyq, y, ny * 4, cudaMemcpyHostToDevice, rt->stream), "H2D"))
        return NFX_INTERNAL;
    s = deeponet_launch(rt, du, u_shape, dyq, y_shape, rt->dy, rt->stream);
    if (s != NFX_OK) {
        cudaStreamSynchronize(rt->stream);
        return s;
    }
    if (!cuda_ok(rt, cudaMemcpyAsync(out, rt->dy, no * 4, cudaMemcpyDeviceToHost, rt->stream), "D2H"))
        return NFX_INTERNAL;
    if (!cuda_ok(rt, cudaStreamSynchronize(rt->stream), "execution")) return NFX_INTERNAL;
    return nfx_runtime_check(rt);
}

}  // extern "C"
