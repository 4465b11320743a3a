// ref_shim.cpp -- extern "C" entry points into the reference NeuroFlow C++ runtime,
// compiled from the reference's own sources where they lie (see oracle/Makefile).
//
// TEST INFRASTRUCTURE ONLY: this builds oracle/_ref/libnflow_ref.so, which the
// parity tests use to pin the CPU restatement in nfo_oracle.c and which bench.py's
// reference arm times on the host cores.  Nothing in the product links it.
//
// The reference keeps Linear / ApplyActivation / SpectralConv2d in an anonymous
// namespace inside cpp/src/fno.cpp, so that file is compiled as part of this
// translation unit (it is found through -I on the reference source directory); the
// wrappers below call those helpers unchanged.
#include "fno.cpp"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "neuroflow/fft.h"
#include "neuroflow/fp8_e4m3.h"
#include "neuroflow/int8_gemm.h"
#include "neuroflow/runtime.h"

namespace {
thread_local std::string g_last_error;

std::vector<int64_t> ToShape(const int64_t* s, int r) {
    return std::vector<int64_t>(s, s + r);
}
}  // namespace

extern "C" {

const char* ref_last_error() { return g_last_error.c_str(); }

// runtime.cpp:79-83 InferenceRuntime::Create
int ref_runtime_create(const char* path, void** out) {
    std::unique_ptr<nflow::InferenceRuntime> rt;
    auto s = nflow::InferenceRuntime::Create(path, rt);
    if (!s.ok()) {
        g_last_error = s.message();
        *out = nullptr;
        return static_cast<int>(s.code());
    }
    *out = rt.release();
    return 0;
}

void ref_runtime_destroy(void* h) { delete static_cast<nflow::InferenceRuntime*>(h); }

void ref_runtime_enable_int8(void* h) {
    static_cast<nflow::InferenceRuntime*>(h)->EnableInt8Gemm();
}

int ref_runtime_is_int8(void* h) {
    return static_cast<nflow::InferenceRuntime*>(h)->IsInt8GemmEnabled() ? 1 : 0;
}

// runtime.cpp:85-101 InferenceRuntime::Run (FNO1d / FNO2d / FNO3d)
int ref_runtime_run(void* h, const float* x, const int64_t* xs, int xr, float* y,
                    const int64_t* ys, int yr) {
    auto* rt = static_cast<nflow::InferenceRuntime*>(h);
    auto s = rt->Run(x, ToShape(xs, xr), y, ToShape(ys, yr));
    if (!s.ok()) g_last_error = s.message();
    return static_cast<int>(s.code());
}

// runtime.cpp:135-143 InferenceRuntime::RunTokenMixer2D
int ref_runtime_run_tokenmixer2d(void* h, const float* x, const int64_t* xs, int xr,
                                 float* y, const int64_t* ys, int yr) {
    auto* rt = static_cast<nflow::InferenceRuntime*>(h);
    auto s = rt->RunTokenMixer2D(x, ToShape(xs, xr), y, ToShape(ys, yr));
    if (!s.ok()) g_last_error = s.message();
    return static_cast<int>(s.code());
}

// runtime.cpp:103-113 InferenceRuntime::RunDeepONet
int ref_runtime_run_deeponet(void* h, const float* u, const int64_t* us, int ur, const float* y,
                             const int64_t* ys, int yr, float* out, const int64_t* os, int orank) {
    auto* rt = static_cast<nflow::InferenceRuntime*>(h);
    auto s = rt->RunDeepONet(u, ToShape(us, ur), y, ToShape(ys, yr), out, ToShape(os, orank));
    if (!s.ok()) g_last_error = s.message();
    return static_cast<int>(s.code());
}

// runtime.cpp:115-153 RunTokenMixer / RunGraphOp / RunGraphOp2D (kind 0, 1, 2)
int ref_runtime_run_other(void* h, int kind, const float* x, const int64_t* xs, int xr, float* y,
                          const int64_t* ys, int yr) {
    auto* rt = static_cast<nflow::InferenceRuntime*>(h);
    nflow::Status s = nflow::Status::Ok();
    if (kind == 0) s = rt->RunTokenMixer(x, ToShape(xs, xr), y, ToShape(ys, yr));
    else if (kind == 1) s = rt->RunGraphOp(x, ToShape(xs, xr), y, ToShape(ys, yr));
    else s = rt->RunGraphOp2D(x, ToShape(xs, xr), y, ToShape(ys, yr));
    if (!s.ok()) g_last_error = s.message();
    return static_cast<int>(s.code());
}

// fno.cpp:51-80
void ref_linear(const float* x, const float* W, const float* b, int bsz, int k, int n,
                float* y) {
    nflow::fno::Linear(x, W, b, bsz, k, n, y);
}

// fno.cpp:36-48
void ref_apply_activation(float* data, int64_t n, int relu) {
    nflow::fno::ApplyActivation(data, n, relu ? std::string("relu") : std::string("gelu"));
}

// fno.cpp:717-771
void ref_spectral_conv2d(const float* h, int bsz, int w, int H, int W, int mh, int mw,
                         const float* wr, const float* wi, float* out) {
    nflow::fno::SpectralConv2d(h, bsz, w, H, W, mh, mw, wr, wi, out);
}

// fno.cpp:164-207
void ref_spectral_conv1d(const float* h, int bsz, int w, int n, int modes,
                         const float* wr, const float* wi, float* out) {
    nflow::fno::SpectralConv1d(h, bsz, w, n, modes, wr, wi, out);
}

// fft.cpp
void ref_rfft(const float* x, int n, float* out) { nflow::fft::Rfft(x, n, out); }
void ref_irfft(const float* x, int n, float* out) { nflow::fft::Irfft(x, n, out); }
void ref_rfft2(const float* x, int H, int W, float* out) { nflow::fft::Rfft2(x, H, W, out); }
void ref_irfft2(const float* x, int H, int W, float* out) { nflow::fft::Irfft2(x, H, W, out); }
void ref_rfft3(const float* x, int H, int W, int D, float* out) {
    nflow::fft::Rfft3(x, H, W, D, out);
}
void ref_irfft3(const float* x, int H, int W, int D, float* out) {
    nflow::fft::Irfft3(x, H, W, D, out);
}

// fp8_e4m3.h:106-298 / :312-334 (header-only; the reference's own encoder and
// per-tensor fake-quant)
void ref_fp32_to_e4m3(const float* in, uint8_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = nflow::fp32_to_e4m3_bits(in[i]);
}
void ref_e4m3_to_fp32(const uint8_t* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = nflow::e4m3_bits_to_fp32(in[i]);
}
void ref_fp8_fake_quant(const float* in, float scale, float* out, int64_t n) {
    nflow::fp8_e4m3_per_tensor_fake_quant(in, scale, out, static_cast<size_t>(n));
}

// int8_gemm.cpp:507-520
void ref_quantise_activation(const float* A, int8_t* Aq, int bsz, int in_f, float s,
                             int32_t zp) {
    nflow::int8_gemm::QuantiseActivation(A, Aq, bsz, in_f, s, zp);
}

// int8_gemm.cpp:530-580
int ref_linear_forward_batched(const int8_t* Wq, const float* sW, const int32_t* zpW,
                               const int32_t* sumW, const float* bias, int in_f, int out_f,
                               float sA, int32_t zpA, int bsz, const float* A, float* C) {
    nflow::int8_gemm::Int8LinearParams p;
    p.W_int8 = Wq;
    p.scale_W = sW;
    p.zp_W = zpW;
    p.bias = bias;
    p.in_features = in_f;
    p.out_features = out_f;
    p.scale_A = sA;
    p.zp_A = zpA;
    p.sum_W_per_row = sumW;
    auto s = nflow::int8_gemm::LinearForwardBatched(p, bsz, A, C);
    return static_cast<int>(s.code());
}

// int8_gemm.cpp:479-496
void ref_precompute_sum_w(const int8_t* Wq, const int32_t* zpW, int in_f, int out_f,
                          int32_t* out) {
    const int32_t* p = nflow::int8_gemm::PrecomputeSumW(Wq, zpW, in_f, out_f);
    if (!p) return;
    std::copy(p, p + out_f, out);
    delete[] p;
}

// Host-core throughput of InferenceRuntime::Run: one runtime per thread on disjoint
// batch slices (Run is not thread-safe, so each thread owns its runtime).  `x` holds
// `bsz` samples of `sample_elems` floats; each thread runs its slice `reps` times.
// Returns the wall time in seconds, or a negative value on error.
double ref_bench_run(const char* path, int op_tokenmixer2d, int enable_int8, const float* x,
                     const int64_t* x_shape, int x_rank, const int64_t* y_shape, int nthreads,
                     int reps) {
    const int64_t bsz = x_shape[0];
    int64_t in_elems = 1, out_elems = 1;
    for (int i = 1; i < x_rank; ++i) in_elems *= x_shape[i];
    for (int i = 1; i < x_rank; ++i) out_elems *= y_shape[i];
    nthreads = std::max(1, std::min<int>(nthreads, static_cast<int>(bsz)));
    std::vector<std::unique_ptr<nflow::InferenceRuntime>> rts(nthreads);
    for (int t = 0; t < nthreads; ++t) {
        auto s = nflow::InferenceRuntime::Create(path, rts[t]);
        if (!s.ok()) {
            g_last_error = s.message();
            return -1.0;
        }
        if (enable_int8) rts[t]->EnableInt8Gemm();
    }
    std::atomic<int> failed{0};
    auto t0 = std::chrono::steady_clock::now();
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; ++t) {
        th.emplace_back([&, t]() {
            const int64_t lo = bsz * t / nthreads, hi = bsz * (t + 1) / nthreads;
            if (hi <= lo) return;
            std::vector<int64_t> xs(x_shape, x_shape + x_rank), ys(y_shape, y_shape + x_rank);
            xs[0] = ys[0] = hi - lo;
            std::vector<float> y(static_cast<size_t>((hi - lo) * out_elems));
            for (int r = 0; r < reps; ++r) {
                nflow::Status s = op_tokenmixer2d
                    ? rts[t]->RunTokenMixer2D(x + lo * in_elems, xs, y.data(), ys)
                    : rts[t]->Run(x + lo * in_elems, xs, y.data(), ys);
                if (!s.ok()) failed = 1;
            }
        });
    }
    for (auto& t : th) t.join();
    auto t1 = std::chrono::steady_clock::now();
    if (failed) return -2.0;
    return std::chrono::duration<double>(t1 - t0).count();
}

}  // extern "C"
