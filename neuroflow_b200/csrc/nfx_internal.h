// nfx_internal.h -- declarations shared by the CUDA translation units and the C-ABI
// layer (not part of the public interface; the public one is include/nfx.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace nfx {

// Fake-quant applied at an ".output" boundary: kind 0 none, 1 INT8 per-tensor,
// 2 the reference FNO2d FP8 log2 snap (fno.cpp:813-828).
struct FqParam {
    int kind;
    float scale;
    int zp;
    float inv_scale;  // 1/scale (IEEE), for the division-free fast path
};

// Arguments of the INT8 GEMM kernel (gemm_i8.cu).  Device pointers.
struct GemmArgs {
    const int8_t* A;          // (M, K) activation codes
    const float* scale_a;     // (M,) per-row scale, or nullptr -> scale_a_t
    const int32_t* zp_a;      // (M,) per-row zero point, or nullptr -> zp_a_t
    float scale_a_t;
    int zp_a_t;
    const int8_t* W;          // (N, K) weight codes, (out, in) layout
    const float* scale_w;     // (N,)
    const int32_t* zp_w;      // (N,)
    const int32_t* sum_w;     // (N,) sum_k (W[o,k] - zp_w[o])
    const float* bias;        // (N,) or nullptr
    int act;                  // 0 none, 1 GELU (tanh form), 2 ReLU
    float* C;                 // (M, N) fp32 output
    int M;
    unsigned* err;            // device error word
    // budget of the kernel's pipeline waits in ns (0: the default of 2 s); the drains
    // before teardown always use the default
    unsigned long long wait_ns;
};

// Test hook of the failure path (nfx_debug_set_wait_budget_ns): the pipeline-wait
// budget that gemm_i8_launch gives every GEMM launch (0: the default).
unsigned long long debug_wait_budget_ns();

bool gemm_i8_supported(int K, int N);
cudaError_t gemm_i8_launch(const GemmArgs& p, int K, int N, cudaStream_t stream);

// Optional per-kernel device timing (CUDA events on the launch stream).
struct KernelTimer {
    virtual void begin(const char* name, cudaStream_t s) = 0;
    virtual void end(cudaStream_t s) = 0;
    // chain(true): a begin() that directly follows an end() on the same stream (with
    // no other stream operation between them) reuses that end event, one event per
    // kernel boundary instead of two; chain(false) ends such a run of launches.
    virtual void chain(bool on) { (void)on; }
    virtual ~KernelTimer() = default;
};
// Keeps a timer chained for one scope (a run of back-to-back launches).
struct TimerChain {
    KernelTimer* t;
    explicit TimerChain(KernelTimer* timer) : t(timer) {
        if (t) t->chain(true);
    }
    ~TimerChain() {
        if (t) t->chain(false);
    }
};

// Host helpers (nfx_host.cpp)
int current_device();
int device_sm_count();
unsigned* device_error_word();  // per current device, allocated once
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device).
cudaError_t set_max_dynamic_smem(const void* kernel, int bytes);
// Encode a 2-D row-major tensor map (inner dimension first).  Returns false on error.
bool encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
               uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
               int swizzle_bytes);

}  // namespace nfx
