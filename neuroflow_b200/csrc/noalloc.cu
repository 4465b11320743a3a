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
// The array holds kNoAllocScratchBytes (32 MiB) on every GPU that loads the library,
// until the process exits.  All calls share it, so calls that overlap on the GPU
// (two streams, two threads) race on it and must be serialised by the caller.  Each
// call rewrites everything it reads before reading it, except the error word, which
// it clears first.
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

__global__ void noalloc_twiddles(float2* fw, float2* fh, float2* iw, float2* ih, int H, int W,
                                 int MH, int MW) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < MW * W) {
        const int k = i / W, w = i % W;
        const double a = 2.0 * static_cast<double>((static_cast<int64_t>(k) * w) % W) / W;
        double s, c;
        sincospi(a, &s, &c);
        const double f = (k == 0 || 2 * k == W) ? 1.0 : 2.0;
        fw[i] = make_float2(static_cast<float>(c), static_cast<float>(-s));
        iw[i] = make_float2(static_cast<float>(f * c / W), static_cast<float>(f * s / W));
    }
    if (i < H * MH) {
        const int h = i / MH, k = i % MH;
        const double a = 2.0 * static_cast<double>((static_cast<int64_t>(k) * h) % H) / H;
        double s, c;
        sincospi(a, &s, &c);
        fh[i] = make_float2(static_cast<float>(c), static_cast<float>(-s));
        ih[i] = make_float2(static_cast<float>(c / H), static_cast<float>(s / H));
    }
}

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

    // scratch layout: error word | 4 transform tables | codes x2 | partial spectra | Y
    const size_t M = static_cast<size_t>(pl.B) * pl.H * pl.W;
    const int nHB = pl.H / pl.HB;
    const size_t modes = static_cast<size_t>(pl.MH) * pl.MW;
    size_t off = 256;
    const size_t o_fw = off; off += up256(sizeof(float2) * pl.MW * pl.W);
    const size_t o_fh = off; off += up256(sizeof(float2) * pl.H * pl.MH);
    const size_t o_iw = off; off += up256(sizeof(float2) * pl.MW * pl.W);
    const size_t o_ih = off; off += up256(sizeof(float2) * pl.H * pl.MH);
    const size_t o_c0 = off; off += up256(M * pl.C);
    const size_t o_c1 = off; off += up256(M * pl.C);
    const size_t o_xp = off; off += up256(sizeof(float2) * pl.B * nHB * modes * pl.C);
    const size_t o_y = off;  off += up256(sizeof(float2) * pl.B * modes * pl.C);
    if (off > kNoAllocScratchBytes)
        return nfx::runtime_fail(rt, NFX_INVALID_ARG,
                                 "nfx_runtime_run_device_noalloc: this batch needs more than the "
                                 "32 MiB of fixed scratch (about 2.5 MB per 128x128 sample at "
                                 "width 64); split the batch");

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
    }
    unsigned char* b = static_cast<unsigned char*>(base);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    unsigned* err = reinterpret_cast<unsigned*>(b);
    if (cudaMemsetAsync(err, 0, sizeof(unsigned), st) != cudaSuccess)
        return nfx::runtime_fail(rt, NFX_INTERNAL, "clearing the error word failed");
    float2* fw = reinterpret_cast<float2*>(b + o_fw);
    float2* fh = reinterpret_cast<float2*>(b + o_fh);
    float2* iw = reinterpret_cast<float2*>(b + o_iw);
    float2* ih = reinterpret_cast<float2*>(b + o_ih);
    const int ntw = pl.MW * pl.W > pl.H * pl.MH ? pl.MW * pl.W : pl.H * pl.MH;
    noalloc_twiddles<<<(ntw + 255) / 256, 256, 0, st>>>(fw, fh, iw, ih, pl.H, pl.W, pl.MH, pl.MW);
    if (cudaGetLastError() != cudaSuccess)
        return nfx::runtime_fail(rt, NFX_INTERNAL, "transform-table launch failed");
    pl.twf_w = fw;
    pl.twf_h = fh;
    pl.twi_w = iw;
    pl.twi_h = ih;
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
