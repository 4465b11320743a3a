// nfx_host.cpp -- per-device host helpers: SM count, the device error word, and
// tensor-map encoding through the driver entry point (no link-time libcuda
// dependency).
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include "nfx_internal.h"

namespace nfx {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
int g_sms[kMaxDevices] = {0};
unsigned* g_err[kMaxDevices] = {nullptr};

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

EncodeTiledFn encode_fn() {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    return g_encode;
}
}  // namespace

int current_device() {
    int d = -1;
    if (cudaGetDevice(&d) != cudaSuccess) return -1;
    return d;
}

int device_sm_count() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return 1;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_sms[d] == 0) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, d);
        g_sms[d] = v > 0 ? v : 1;
    }
    return g_sms[d];
}

unsigned* device_error_word() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_err[d]) {
        void* p = nullptr;
        if (cudaMalloc(&p, 256) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, 256);
        cudaDeviceSynchronize();
        g_err[d] = static_cast<unsigned*>(p);
    }
    return g_err[d];
}

cudaError_t set_max_dynamic_smem(const void* kernel, int bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> done;
    const int d = current_device();
    std::lock_guard<std::mutex> lk(mu);
    auto key = std::make_pair(kernel, d);
    auto it = done.find(key);
    if (it != done.end() && it->second >= bytes) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) done[key] = bytes;
    return e;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner,
               uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
               int swizzle_bytes) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
    if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
    if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
    if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
    const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace nfx
