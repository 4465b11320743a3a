// noalloc.cu -- an FNO2d forward entry point that allocates nothing.
//
// Who needs it: callers that cannot call cudaMalloc at the moment they run
// inference -- a host process whose device memory is owned by another allocator
// (a framework's caching allocator, or a simulation code that reserves the device
// up front), a real-time loop that must not take an allocation's latency or
// failure mode, or an engine whose own rules forbid allocation after start-up.
// nfx_runtime_run_device normally keeps its scratch (int8 activation codes, partial
// and mixed spectra, transform tables, the device error word) in buffers it
// allocates on demand; this entry point keeps them in one fixed file-scope device
// array instead, whose size is set at compile time.
//
// The array holds kNoAllocScratchBytes (32 MiB) on every GPU where the entry point has
// run, until the process exits.  With CUDA's lazy module loading (the default) that
// memory is reserved when the first call on a device looks the array up, not when the
// library is loaded, so that first call belongs at start-up (it can fail for lack of
// memory if the device is already full) and before any stream capture.  All calls
// share the array, so calls that overlap on the GPU (two streams, two threads) race on
// it and must be serialised by the caller.  Each call clears the error word and
// rewrites the activation buffers before reading them; the transform tables are
// rewritten (synchronously, from static host tables) only when the grid differs from
// the previous call's on that device.
//
// Capacity: 256 B of header, the transform tables (49,152 B at 128 x 128 with 12 x 12
// modes, plus the 16,384 B of tensor-core basis digits and 192 B of digit sums at
// W = 128), and per sample 2 H W C bytes of codes + 4 x 12 x 12 x C x 8 bytes of
// partial spectra + 12 x 12 x C x 8 bytes of mixed spectrum: 2,465,792 B for a
// 128 x 128 sample at width 64, so 13 such samples fit and 14 are refused.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/nfx.h"
#include "fno2d.h"
#include "nfx_internal.h"

namespace nfx {
// Validation and weight plan of the runtime handle, without any allocation
// (nfx_runtime.cpp).
int fno2d_noalloc_plan(nfx_runtime* rt, const float* x, const int64_t* x_shape, int x_rank,
                       float* y, const int64_t* y_shape, int y_rank, Fno2dPlan* plan);
int runtime_device(const nfx_runtime* rt);
int runtime_fail(nfx_runtime* rt, int code, const char* msg);
}  // namespace nfx

namespace {

constexpr size_t kNoAllocScratchBytes = size_t{32} << 20;  // 32 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device ordinal.  In host code the array's
// name is only a host-side stand-in, so the address is looked up once per device
// with that device current, and passed to the kernels.
constexpr int kMaxDev = 64;
void* g_scratch_addr[kMaxDev] = {};
std::mutex g_scratch_mu;

// Host copies of the transform tables, built by the same code as the allocating
// path's (fno2d_tables), for grids up to kMaxH x kMaxW with 12 x 12 modes.
constexpr int kMaxH = 4096, kMaxW = 128, kModes = 12;
float g_fw[2 * kModes * kMaxW], g_iw[2 * kModes * kMaxW];
float g_fh[2 * kMaxH * kModes], g_ih[2 * kMaxH * kModes];
int8_t g_limbs[nfx::kFno2dLimbBytes];
long long g_sum_b[2 * kModes];
int g_tables_hw[kMaxDev][2] = {};   // grid whose tables each device's scratch holds

size_t up256(size_t v) { return (v + 255) & ~size_t{255}; }

}  // namespace

extern "C" int nfx_runtime_run_device_noalloc(nfx_runtime* rt, const float* x,
                                              const int64_t* x_shape, int x_rank, float* y,
                                              const int64_t* y_shape, int y_rank,
                                              void* stream) {
    if (!rt) return NFX_INVALID_ARG;
    const int dev = nfx::runtime_device(rt);
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
    struct Restore {
        int p, d;
        ~Restore() {
            if (p >= 0 && p != d) cudaSetDevice(p);
        }
    } restore{prev, dev};

    nfx::Fno2dPlan pl{};
    int s = nfx::fno2d_noalloc_plan(rt, x, x_shape, x_rank, y, y_shape, y_rank, &pl);
    if (s != NFX_OK) return s;
    if (pl.B == 0) return NFX_OK;

    // scratch layout: error word | 4 transform tables | basis digits + sums | codes x2 |
    // partial spectra | Y
    const size_t M = static_cast<size_t>(pl.B) * pl.H * pl.W;
    const int nHB = pl.H / pl.HB;
    const size_t modes = static_cast<size_t>(pl.MH) * pl.MW;
    const bool tc = nfx::fno2d_tc_forward(pl.W, pl.MW);
    if (pl.H > kMaxH || pl.W > kMaxW || pl.MH != kModes || pl.MW != kModes)
        return nfx::runtime_fail(rt, NFX_UNSUPPORTED_OP,
                                 "nfx_runtime_run_device_noalloc: grid or modes beyond its tables");
    const size_t n_fw = 2 * static_cast<size_t>(pl.MW) * pl.W, n_fh = 2 * static_cast<size_t>(pl.H) * pl.MH;
    size_t off = 256;
    const size_t o_fw = off; off += up256(sizeof(float) * n_fw);
    const size_t o_fh = off; off += up256(sizeof(float) * n_fh);
    const size_t o_iw = off; off += up256(sizeof(float) * n_fw);
    const size_t o_ih = off; off += up256(sizeof(float) * n_fh);
    const size_t o_lb = off; off += tc ? up256(nfx::kFno2dLimbBytes) : 0;
    const size_t o_sb = off; off += tc ? up256(sizeof(long long) * 2 * pl.MW) : 0;
    const size_t o_c0 = off; off += up256(M * pl.C);
    const size_t o_c1 = off; off += up256(M * pl.C);
    const size_t o_xp = off; off += up256(sizeof(float2) * pl.B * nHB * modes * pl.C);
    const size_t o_y = off;  off += up256(sizeof(float2) * pl.B * modes * pl.C);
    if (off > kNoAllocScratchBytes)
        return nfx::runtime_fail(rt, NFX_INVALID_ARG,
                                 "nfx_runtime_run_device_noalloc: this batch needs more than the "
                                 "32 MiB of fixed scratch (2,465,792 B per 128x128 sample at "
                                 "width 64: at most 13 such samples per call); split the batch");

    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_scratch_mu);
        if (dev < 0 || dev >= kMaxDev)
            return nfx::runtime_fail(rt, NFX_INTERNAL, "device ordinal out of range");
        if (!g_scratch_addr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p)
                return nfx::runtime_fail(rt, NFX_INTERNAL,
                                         "cudaGetSymbolAddress of the fixed scratch failed");
            g_scratch_addr[dev] = p;
        }
        base = g_scratch_addr[dev];
        unsigned char* b = static_cast<unsigned char*>(base);
        if (g_tables_hw[dev][0] != pl.H || g_tables_hw[dev][1] != pl.W) {
            // the previous call's work on this device has finished (every call
            // synchronises its stream before returning), so the tables can be replaced
            nfx::fno2d_tables(pl.H, pl.W, pl.MH, pl.MW, g_fw, g_fh, g_iw, g_ih, tc ? g_limbs : nullptr,
                              tc ? g_sum_b : nullptr);
            bool ok = cudaMemcpy(b + o_fw, g_fw, sizeof(float) * n_fw, cudaMemcpyHostToDevice) == cudaSuccess &&
                      cudaMemcpy(b + o_fh, g_fh, sizeof(float) * n_fh, cudaMemcpyHostToDevice) == cudaSuccess &&
                      cudaMemcpy(b + o_iw, g_iw, sizeof(float) * n_fw, cudaMemcpyHostToDevice) == cudaSuccess &&
                      cudaMemcpy(b + o_ih, g_ih, sizeof(float) * n_fh, cudaMemcpyHostToDevice) == cudaSuccess;
            if (ok && tc)
                ok = cudaMemcpy(b + o_lb, g_limbs, nfx::kFno2dLimbBytes, cudaMemcpyHostToDevice) == cudaSuccess &&
                     cudaMemcpy(b + o_sb, g_sum_b, sizeof(long long) * 2 * pl.MW,
                                cudaMemcpyHostToDevice) == cudaSuccess;
            if (!ok) {
                g_tables_hw[dev][0] = g_tables_hw[dev][1] = 0;
                return nfx::runtime_fail(rt, NFX_INTERNAL, "uploading the transform tables failed");
            }
            g_tables_hw[dev][0] = pl.H;
            g_tables_hw[dev][1] = pl.W;
        }
    }
    unsigned char* b = static_cast<unsigned char*>(base);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned* err = reinterpret_cast<unsigned*>(b);
    if (cudaMemsetAsync(err, 0, sizeof(unsigned), st) != cudaSuccess)
        return nfx::runtime_fail(rt, NFX_INTERNAL, "clearing the error word failed");
    pl.twf_w = reinterpret_cast<const float2*>(b + o_fw);
    pl.twf_h = reinterpret_cast<const float2*>(b + o_fh);
    pl.twi_w = reinterpret_cast<const float2*>(b + o_iw);
    pl.twi_h = reinterpret_cast<const float2*>(b + o_ih);
    pl.fwd_limbs = tc ? reinterpret_cast<const int8_t*>(b + o_lb) : nullptr;
    pl.fwd_sum_b = tc ? reinterpret_cast<const long long*>(b + o_sb) : nullptr;
    pl.codes[0] = reinterpret_cast<int8_t*>(b + o_c0);
    pl.codes[1] = reinterpret_cast<int8_t*>(b + o_c1);
    pl.xpart = reinterpret_cast<float2*>(b + o_xp);
    pl.Y = reinterpret_cast<float2*>(b + o_y);
    pl.err = err;
    pl.timer = nullptr;
    if (nfx::fno2d_run(pl, st) != cudaSuccess)
        return nfx::runtime_fail(rt, NFX_INTERNAL, "FNO2d launch failed");
    if (cudaStreamSynchronize(st) != cudaSuccess)
        return nfx::runtime_fail(rt, NFX_INTERNAL, "FNO2d execution failed");
    unsigned flags = 0;
    if (cudaMemcpy(&flags, err, sizeof(flags), cudaMemcpyDeviceToHost) != cudaSuccess)
        return nfx::runtime_fail(rt, NFX_INTERNAL, "reading the error word failed");
    if (flags)
        return nfx::runtime_fail(rt, NFX_INTERNAL, "a kernel gave up waiting (device timeout)");
    return NFX_OK;
}
