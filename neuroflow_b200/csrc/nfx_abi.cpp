// nfx_abi.cpp -- extern "C" entry points of the GEMM and error-reporting part of
// include/nfx.h.  (The runtime handle entry points live in nfx_runtime.cpp.)
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <string>

#include "../../include/nfx.h"
#include "nfx_internal.h"

namespace {
thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}
}  // namespace

namespace nfx {
int set_thread_error(int code, const std::string& msg) { return fail(code, msg); }

namespace {
std::atomic<unsigned long long> g_wait_budget_ns{0};
}
unsigned long long debug_wait_budget_ns() { return g_wait_budget_ns.load(std::memory_order_relaxed); }
}  // namespace nfx

extern "C" {

const char* nfx_last_error(void) { return g_err.c_str(); }

void nfx_debug_set_wait_budget_ns(unsigned long long ns) {
    nfx::g_wait_budget_ns.store(ns, std::memory_order_relaxed);
}

int nfx_int8_gemm(const int8_t* A, const float* scale_a, const int32_t* zp_a, float scale_a_t,
                  int32_t zp_a_t, int M, int K, const int8_t* W, const float* scale_w,
                  const int32_t* zp_w, const int32_t* sum_w, const float* bias, int N, int act,
                  float* C, void* stream) {
    if (M < 0) return fail(NFX_INVALID_ARG, "nfx_int8_gemm: M < 0");
    if (!nfx::gemm_i8_supported(K, N))
        return fail(NFX_INVALID_ARG, "nfx_int8_gemm: K and N must be 32, 64, 128 or 256");
    if (act < 0 || act > 2) return fail(NFX_INVALID_ARG, "nfx_int8_gemm: act must be 0, 1 or 2");
    if (M == 0) return NFX_OK;
    if (!A || !W || !scale_w || !zp_w || !sum_w || !C)
        return fail(NFX_INVALID_ARG, "nfx_int8_gemm: null pointer");
    if ((scale_a == nullptr) != (zp_a == nullptr))
        return fail(NFX_INVALID_ARG, "nfx_int8_gemm: scale_a and zp_a must both be set or NULL");
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(W) |
         reinterpret_cast<uintptr_t>(C)) & 15)
        return fail(NFX_INVALID_ARG, "nfx_int8_gemm: A, W and C must be 16-byte aligned");
    nfx::GemmArgs p{};
    p.A = A;
    p.scale_a = scale_a;
    p.zp_a = zp_a;
    p.scale_a_t = scale_a_t;
    p.zp_a_t = zp_a_t;
    p.W = W;
    p.scale_w = scale_w;
    p.zp_w = zp_w;
    p.sum_w = sum_w;
    p.bias = bias;
    p.act = act;
    p.C = C;
    p.M = M;
    p.err = nfx::device_error_word();
    if (!p.err) return fail(NFX_INTERNAL, "nfx_int8_gemm: cannot allocate the device error word");
    cudaError_t e = nfx::gemm_i8_launch(p, K, N, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess)
        return fail(NFX_INTERNAL, std::string("nfx_int8_gemm: launch failed: ") +
                                      cudaGetErrorString(e));
    return NFX_OK;
}

int nfx_device_errors(unsigned* flags_out) {
    unsigned* w = nfx::device_error_word();
    if (!w) return fail(NFX_INTERNAL, "nfx_device_errors: no device error word");
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess)
        return fail(NFX_INTERNAL, std::string("nfx_device_errors: ") + cudaGetErrorString(e));
    unsigned v = 0;
    e = cudaMemcpy(&v, w, sizeof(v), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(w, 0, sizeof(unsigned));
    if (e != cudaSuccess)
        return fail(NFX_INTERNAL, std::string("nfx_device_errors: ") + cudaGetErrorString(e));
    if (flags_out) *flags_out = v;
    return NFX_OK;
}

}  // extern "C"
