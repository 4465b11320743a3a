// nfx_fp8.cu -- FP8 E4M3 conversions of the reference's fp8_e4m3.h on the GPU:
// fp32_array_to_e4m3_bits (fp8_e4m3.h:286), e4m3_bits_to_fp32_array (:295)
// and fp8_e4m3_per_tensor_fake_quant (:312-334), with the reference's bit-level
// encoder (numerics.cuh: e4m3_encode_ref / e4m3_decode_ref).  Device-pointer entry
// points run on a caller stream; the host-pointer ones (the neuroflow_cpp helpers)
// stage through device memory and synchronise.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "../../include/nfx.h"
#include "nfx_internal.h"
#include "numerics.cuh"

namespace nfx {
int set_thread_error(int code, const std::string& msg);
}

namespace {

__global__ void e4m3_encode_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = static_cast<uint8_t>(nfx::e4m3_encode_ref(x[i]));
}

__global__ void e4m3_decode_kernel(const uint8_t* __restrict__ b, float* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = nfx::e4m3_decode_ref(b[i]);
}

__global__ void e4m3_fake_quant_kernel(const float* __restrict__ x, float scale, float inv,
                                       float* __restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = nfx::fp8_fake_quant(x[i], scale, inv);
}

// Every fp32 bit pattern through the hardware-conversion encoder (which saturates by
// itself) and, clamped as e4m3_code clamps, through the reference one, and through the
// executors' inner fake-quant against the reference round trip; every code through
// both decoders (bit patterns).
__global__ void e4m3_selfcheck_kernel(unsigned long long* bad) {
    unsigned long long n = 0;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < (1ull << 32); i += stride) {
        const float v = __uint_as_float(static_cast<uint32_t>(i));
        const float xs = v > 448.0f ? 448.0f : (v < -448.0f ? -448.0f : v);
        if (nfx::e4m3_encode_fast(v) != nfx::e4m3_encode_ref(xs)) ++n;
        // the executors' inner fake-quant: the reference value, any NaN for a NaN
        const float fq = nfx::fp8_fake_quant_inner(v, 1.0f, 1.0f);
        const float fr = nfx::e4m3_decode_ref(nfx::e4m3_encode_ref(xs));
        if (fr == fr ? __float_as_uint(fq) != __float_as_uint(fr) : fq == fq) ++n;
        if (i < 256 && __float_as_uint(nfx::e4m3_decode_fast(static_cast<uint32_t>(i))) !=
                           __float_as_uint(nfx::e4m3_decode_ref(static_cast<uint32_t>(i))))
            ++n;
    }
    if (n) atomicAdd(bad, n);
}

int grid_for(int64_t n) {
    const int64_t blocks = (n + 255) / 256;
    const int cap = 8 * nfx::device_sm_count();
    return static_cast<int>(blocks < cap ? (blocks > 0 ? blocks : 1) : cap);
}

// 1 / scale as the reference computes it (scale 0 -> 1)
float inv_scale(float scale) { return scale == 0.0f ? 1.0f : 1.0f / scale; }

int launch_fail(const char* what) {
    return nfx::set_thread_error(NFX_INTERNAL, std::string(what) + ": " +
                                                   cudaGetErrorString(cudaGetLastError()));
}

// Host-buffer call: copy in, run, copy out, synchronously on a private stream.
template <typename In, typename Out, typename Launch>
int host_call(const In* in, Out* out, int64_t n, Launch launch, const char* what) {
    if (n < 0) return nfx::set_thread_error(NFX_INVALID_ARG, std::string(what) + ": n < 0");
    if (n == 0) return NFX_OK;
    if (!in || !out) return nfx::set_thread_error(NFX_INVALID_ARG, std::string(what) + ": null buffer");
    void* din = nullptr;
    void* dout = nullptr;
    cudaStream_t st = nullptr;
    int rc = NFX_OK;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&din, static_cast<size_t>(n) * sizeof(In)) != cudaSuccess ||
        cudaMalloc(&dout, static_cast<size_t>(n) * sizeof(Out)) != cudaSuccess) {
        rc = nfx::set_thread_error(NFX_INTERNAL, std::string(what) + ": device allocation failed");
    } else if (cudaMemcpyAsync(din, in, static_cast<size_t>(n) * sizeof(In), cudaMemcpyHostToDevice, st) !=
               cudaSuccess) {
        rc = nfx::set_thread_error(NFX_INTERNAL, std::string(what) + ": input copy failed");
    } else {
        launch(static_cast<const In*>(din), static_cast<Out*>(dout), st);
        if (cudaGetLastError() != cudaSuccess) {
            rc = launch_fail(what);
        } else if (cudaMemcpyAsync(out, dout, static_cast<size_t>(n) * sizeof(Out), cudaMemcpyDeviceToHost,
                                   st) != cudaSuccess ||
                   cudaStreamSynchronize(st) != cudaSuccess) {
            rc = nfx::set_thread_error(NFX_INTERNAL, std::string(what) + ": execution failed");
        }
    }
    if (st) cudaStreamSynchronize(st);
    if (din) cudaFree(din);
    if (dout) cudaFree(dout);
    if (st) cudaStreamDestroy(st);
    return rc;
}

}  // namespace

extern "C" {

int nfx_fp8_e4m3_to_bits(const float* x, uint8_t* bits, int64_t n, void* stream) {
    if (n < 0) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_fp8_e4m3_to_bits: n < 0");
    if (n == 0) return NFX_OK;
    if (!x || !bits) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_fp8_e4m3_to_bits: null buffer");
    e4m3_encode_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, bits, n);
    return cudaGetLastError() == cudaSuccess ? NFX_OK : launch_fail("nfx_fp8_e4m3_to_bits");
}

int nfx_fp8_e4m3_from_bits(const uint8_t* bits, float* y, int64_t n, void* stream) {
    if (n < 0) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_fp8_e4m3_from_bits: n < 0");
    if (n == 0) return NFX_OK;
    if (!bits || !y) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_fp8_e4m3_from_bits: null buffer");
    e4m3_decode_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(bits, y, n);
    return cudaGetLastError() == cudaSuccess ? NFX_OK : launch_fail("nfx_fp8_e4m3_from_bits");
}

int nfx_fp8_e4m3_fake_quant(const float* x, float scale, float* y, int64_t n, void* stream) {
    if (n < 0) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_fp8_e4m3_fake_quant: n < 0");
    if (n == 0) return NFX_OK;
    if (!x || !y) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_fp8_e4m3_fake_quant: null buffer");
    e4m3_fake_quant_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, scale, inv_scale(scale),
                                                                                      y, n);
    return cudaGetLastError() == cudaSuccess ? NFX_OK : launch_fail("nfx_fp8_e4m3_fake_quant");
}

int nfx_fp8_e4m3_to_bits_host(const float* x, uint8_t* bits, int64_t n) {
    return host_call(x, bits, n, [n](const float* dx, uint8_t* db, cudaStream_t st) {
        e4m3_encode_kernel<<<grid_for(n), 256, 0, st>>>(dx, db, n);
    }, "nfx_fp8_e4m3_to_bits_host");
}

int nfx_fp8_e4m3_from_bits_host(const uint8_t* bits, float* y, int64_t n) {
    return host_call(bits, y, n, [n](const uint8_t* db, float* dy, cudaStream_t st) {
        e4m3_decode_kernel<<<grid_for(n), 256, 0, st>>>(db, dy, n);
    }, "nfx_fp8_e4m3_from_bits_host");
}

int nfx_fp8_e4m3_fake_quant_host(const float* x, float scale, float* y, int64_t n) {
    const float inv = inv_scale(scale);
    return host_call(x, y, n, [n, scale, inv](const float* dx, float* dy, cudaStream_t st) {
        e4m3_fake_quant_kernel<<<grid_for(n), 256, 0, st>>>(dx, scale, inv, dy, n);
    }, "nfx_fp8_e4m3_fake_quant_host");
}

int nfx_fp8_e4m3_selfcheck(unsigned long long* mismatches) {
    if (!mismatches) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_fp8_e4m3_selfcheck: null output");
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, sizeof(*d)) != cudaSuccess)
        return nfx::set_thread_error(NFX_INTERNAL, "nfx_fp8_e4m3_selfcheck: device allocation failed");
    int rc = NFX_OK;
    if (cudaMemset(d, 0, sizeof(*d)) != cudaSuccess) {
        rc = nfx::set_thread_error(NFX_INTERNAL, "nfx_fp8_e4m3_selfcheck: memset failed");
    } else {
        e4m3_selfcheck_kernel<<<8 * nfx::device_sm_count(), 256>>>(d);
        if (cudaGetLastError() != cudaSuccess)
            rc = launch_fail("nfx_fp8_e4m3_selfcheck");
        else if (cudaMemcpy(mismatches, d, sizeof(*d), cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = nfx::set_thread_error(NFX_INTERNAL, "nfx_fp8_e4m3_selfcheck: execution failed");
    }
    cudaFree(d);
    return rc;
}

}  // extern "C"
