// nfx_calib.cu -- activation calibration on the GPU (nfx_calibrate_*), the device-side
// counterpart of the reference's calibrate() / quantise_model()
// (neuroflow/quant/static_quant.py:609-741, :855-935).
//
// The reference runs the FP32 PyTorch model on a calibration set with forward hooks on
// every nn.Linear, keeps every output tensor on the host, and reduces them: min / max
// (compute_tensor_qparams, :480-533), or the (100 - p) / 2 and 100 - (100 - p) / 2
// percentiles of all values (:699-716), and abs-max / 448 for FP8 E4M3
// (compute_fp8_e4m3_qparams, :338-352).  Here the FP32 FNO2d executor runs the batches
// with observers in its kernels: each Linear output's range is reduced per warp and
// merged with atomics on order-preserving float keys; for percentiles the values are
// kept on the device and the two order statistics that numpy's linear interpolation
// needs are found by an exact radix select (four 8-bit passes over the value keys).
// The qparam formulas then run on the host in double precision, as the reference's
// Python does, and return float32 scales as NIRQ stores them.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "../../include/nfx.h"
#include "fno2d.h"
#include "nfx_internal.h"
#include "numerics.cuh"

namespace nfx {
int set_thread_error(int code, const std::string& msg);
int runtime_device(const nfx_runtime* rt);
int runtime_fail_str(nfx_runtime* rt, int code, const std::string& msg);
int calib_tensors(const nfx_runtime* rt);
std::string calib_name(const nfx_runtime* rt, int i);
unsigned*& calib_stats(nfx_runtime* rt);
int& calib_keep(nfx_runtime* rt);
std::vector<std::vector<std::pair<float*, int64_t>>>& calib_vals(nfx_runtime* rt);
int calib_observe(nfx_runtime* rt, const float* x, const int64_t* xs, int xr);
}  // namespace nfx

namespace {

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

// 256-bin histogram of the key digit at `shift` over the values whose higher digits
// equal `prefix` (under `mask`).
__global__ void __launch_bounds__(256) radix_hist_kernel(const float* __restrict__ v, int64_t n, unsigned prefix,
                                                         unsigned mask, int shift,
                                                         unsigned long long* __restrict__ hist) {
    __shared__ unsigned h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const unsigned k = nfx::float_order_key(v[i]);
        if ((k & mask) == prefix) atomicAdd(&h[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (h[threadIdx.x]) atomicAdd(&hist[threadIdx.x], static_cast<unsigned long long>(h[threadIdx.x]));
}

// The value of rank r (0-based, ascending) among the kept values of one tensor.
bool kth_value(const std::vector<std::pair<float*, int64_t>>& chunks, int64_t r, float& out,
               unsigned long long* dhist) {
    unsigned prefix = 0, mask = 0;
    const int sms = nfx::device_sm_count();
    for (int shift = 24; shift >= 0; shift -= 8) {
        if (cudaMemset(dhist, 0, 256 * sizeof(unsigned long long)) != cudaSuccess) return false;
        for (const auto& c : chunks) {
            const int64_t blocks = (c.second + 255) / 256;
            const int grid = static_cast<int>(blocks < 8 * sms ? (blocks > 0 ? blocks : 1) : 8 * sms);
            radix_hist_kernel<<<grid, 256>>>(c.first, c.second, prefix, mask, shift, dhist);
        }
        unsigned long long hist[256];
        if (cudaMemcpy(hist, dhist, sizeof(hist), cudaMemcpyDeviceToHost) != cudaSuccess) return false;
        int b = 0;
        while (b < 255 && static_cast<int64_t>(hist[b]) <= r) {
            r -= static_cast<int64_t>(hist[b]);
            ++b;
        }
        prefix |= static_cast<unsigned>(b) << shift;
        mask |= 255u << shift;
    }
    out = nfx::float_from_order_key(prefix);
    return true;
}

// numpy.percentile's default ("linear") method: virtual index (n - 1) q, then
// numpy's _lerp between the neighbouring order statistics, in double.
bool percentile(const std::vector<std::pair<float*, int64_t>>& chunks, int64_t n, double q, double& out,
                unsigned long long* dhist) {
    const double vi = static_cast<double>(n - 1) * (q / 100.0);
    const int64_t lo = static_cast<int64_t>(std::floor(vi));
    const double t = vi - static_cast<double>(lo);
    float a = 0.f, b = 0.f;
    if (!kth_value(chunks, lo, a, dhist)) return false;
    if (lo + 1 < n && t != 0.0) {
        if (!kth_value(chunks, lo + 1, b, dhist)) return false;
    } else {
        b = a;
    }
    const double da = a, db = b, diff = db - da;
    out = t >= 0.5 ? db - diff * (1.0 - t) : da + diff * t;
    return true;
}

}  // namespace

extern "C" {

int nfx_calibrate_begin(nfx_runtime* rt, int keep_values) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    const int n = nfx::calib_tensors(rt);
    if (n == 0) return nfx::runtime_fail_str(rt, NFX_UNSUPPORTED_OP, "calibration supports FNO2d models");
    DeviceGuard g(nfx::runtime_device(rt));
    nfx_calibrate_end(rt);
    void* p = nullptr;
    if (cudaMalloc(&p, 3 * nfx::kFno2dObsMax * sizeof(unsigned)) != cudaSuccess)
        return nfx::runtime_fail_str(rt, NFX_INTERNAL, "cudaMalloc calibration statistics");
    unsigned init[3 * nfx::kFno2dObsMax];
    for (int i = 0; i < nfx::kFno2dObsMax; ++i) {
        init[i] = 0xFFFFFFFFu;                    // min key
        init[nfx::kFno2dObsMax + i] = 0u;         // max key
        init[2 * nfx::kFno2dObsMax + i] = 0u;     // NaN seen
    }
    if (cudaMemcpy(p, init, sizeof(init), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(p);
        return nfx::runtime_fail_str(rt, NFX_INTERNAL, "initialising calibration statistics");
    }
    nfx::calib_stats(rt) = static_cast<unsigned*>(p);
    nfx::calib_keep(rt) = keep_values ? 1 : 0;
    nfx::calib_vals(rt).assign(n, {});
    return NFX_OK;
}

int nfx_calibrate_observe(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    DeviceGuard g(nfx::runtime_device(rt));
    return nfx::calib_observe(rt, x, x_shape, x_rank);
}

int nfx_calibrate_count(const nfx_runtime* rt) {
    return rt && nfx::calib_stats(const_cast<nfx_runtime*>(rt)) ? nfx::calib_tensors(rt) : 0;
}

int nfx_calibrate_result(nfx_runtime* rt, int index, double pct, char* name_out, int name_cap, float* scale_out,
                         int32_t* zp_out, float* fp8_scale_out, double* lo_out, double* hi_out) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    unsigned* stats = nfx::calib_stats(rt);
    if (!stats) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "call nfx_calibrate_begin first");
    const int n = nfx::calib_tensors(rt);
    if (index < 0 || index >= n) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "calibration index out of range");
    if (!(pct > 0.0 && pct <= 100.0)) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "percentile must be in (0, 100]");
    DeviceGuard g(nfx::runtime_device(rt));
    unsigned h[3 * nfx::kFno2dObsMax];
    if (cudaDeviceSynchronize() != cudaSuccess || cudaMemcpy(h, stats, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess)
        return nfx::runtime_fail_str(rt, NFX_INTERNAL, "reading calibration statistics");
    const std::string name = nfx::calib_name(rt, index);
    if (name_out && name_cap > 0) {
        const size_t k = name.size() < static_cast<size_t>(name_cap - 1) ? name.size() : static_cast<size_t>(name_cap - 1);
        std::memcpy(name_out, name.data(), k);
        name_out[k] = 0;
    }
    const bool nan = h[2 * nfx::kFno2dObsMax + index] != 0;
    const bool seen = h[index] <= h[nfx::kFno2dObsMax + index] && h[index] != 0xFFFFFFFFu;
    if (!seen) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "no calibration batch observed");
    const float tmin = nfx::float_from_order_key(h[index]);
    const float tmax = nfx::float_from_order_key(h[nfx::kFno2dObsMax + index]);
    constexpr double kQmin = -128.0, kQmax = 127.0, kSpan = kQmax - kQmin;
    double scale = 1.0, mins = tmin, maxs = tmax;
    int zp = 0;
    if (nan) {
        // a NaN range gives the no-op qparams (static_quant.py:515-519); the reference's
        // percentile branch has no rule for NaN (its int() of a NaN zero point raises)
        mins = maxs = NAN;
    } else if (pct >= 100.0) {
        // compute_tensor_qparams (static_quant.py:510-533)
        if (tmax != tmin) {
            scale = (static_cast<double>(tmax) - tmin) / kSpan;
            const double raw = std::nearbyint(kQmin - tmin / scale);
            zp = static_cast<int>(raw < kQmin ? kQmin : (raw > kQmax ? kQmax : raw));
            if (zp != raw) scale = zp == static_cast<int>(kQmin) ? (static_cast<double>(tmax) - 0.0) / kSpan
                                                                  : (0.0 - static_cast<double>(tmin)) / kSpan;
        }
    } else {
        // calibrate()'s percentile branch (static_quant.py:703-716)
        auto& chunks = nfx::calib_vals(rt)[index];
        if (!nfx::calib_keep(rt) || chunks.empty())
            return nfx::runtime_fail_str(rt, NFX_INVALID_ARG,
                                         "percentiles need the values: nfx_calibrate_begin(rt, 1)");
        int64_t total = 0;
        for (const auto& c : chunks) total += c.second;
        void* dh = nullptr;
        if (cudaMalloc(&dh, 256 * sizeof(unsigned long long)) != cudaSuccess)
            return nfx::runtime_fail_str(rt, NFX_INTERNAL, "cudaMalloc histogram");
        const double lo_p = (100.0 - pct) / 2.0, hi_p = 100.0 - lo_p;
        const bool ok = percentile(chunks, total, lo_p, mins, static_cast<unsigned long long*>(dh)) &&
                        percentile(chunks, total, hi_p, maxs, static_cast<unsigned long long*>(dh));
        cudaFree(dh);
        if (!ok || cudaGetLastError() != cudaSuccess)
            return nfx::runtime_fail_str(rt, NFX_INTERNAL, "percentile selection failed");
        const double spans = maxs - mins;
        scale = spans > 0 ? spans / kSpan : 1.0;
        const double raw = std::nearbyint(kQmin - mins / scale);
        zp = static_cast<int>(raw < kQmin ? kQmin : (raw > kQmax ? kQmax : raw));
        if (zp == static_cast<int>(kQmin) && maxs > 0) scale = maxs / kSpan;
        else if (zp == static_cast<int>(kQmax) && mins < 0) scale = -mins / kSpan;
    }
    // compute_fp8_e4m3_qparams (static_quant.py:338-352): abs-max of the tensor / 448
    float fp8 = 1.0f;
    if (!nan) {
        const float amax = std::fabs(tmin) > std::fabs(tmax) ? std::fabs(tmin) : std::fabs(tmax);
        if (amax != 0.0f) fp8 = static_cast<float>(static_cast<double>(amax) / 448.0);
    }
    if (scale_out) *scale_out = static_cast<float>(scale);
    if (zp_out) *zp_out = zp;
    if (fp8_scale_out) *fp8_scale_out = fp8;
    if (lo_out) *lo_out = mins;
    if (hi_out) *hi_out = maxs;
    return NFX_OK;
}

int nfx_calibrate_end(nfx_runtime* rt) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    DeviceGuard g(nfx::runtime_device(rt));
    cudaDeviceSynchronize();
    if (nfx::calib_stats(rt)) cudaFree(nfx::calib_stats(rt));
    nfx::calib_stats(rt) = nullptr;
    for (auto& t : nfx::calib_vals(rt))
        for (auto& c : t) cudaFree(c.first);
    nfx::calib_vals(rt).clear();
    return NFX_OK;
}

}  // extern "C"
