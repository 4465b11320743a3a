// nfx_multi.cpp -- inference partitioned by batch across the GPUs of one node.
//
// Samples are independent (no layer of FNO1d/2d/3d couples two samples), so a batch
// of B samples on G GPUs runs as G contiguous slices of ceil(B / G) samples, each on
// its own GPU with its own copy of the weights, and the only communication is moving
// inputs to and outputs from the GPU that owns the caller's buffers.  Two forms:
//
//  * nfx_group_*: one process drives G GPUs (the reference's API shape: one Create,
//    one Run over the whole batch).  With host buffers every GPU copies its own slice
//    in and out over its own PCIe link, one host thread per GPU; with device buffers on
//    the first GPU, NCCL point-to-point transfers scatter the input slices and gather
//    the outputs back over NVLink.
//  * nfx_runtime_run_sharded*: one process per GPU (torchrun-style).  Every rank passes
//    the whole batch, computes its slice, and NCCL gathers the outputs -- to every rank
//    (all-gather) or to one root.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or $NFX_NCCL_LIB) the first time
// one of these entry points needs it, so the single-GPU library does not depend on it;
// a process that already loaded NCCL (e.g. through torch) shares that copy.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/nfx.h"

namespace nfx {
int set_thread_error(int code, const std::string& msg);
int runtime_device(const nfx_runtime* rt);
int runtime_check_shapes(nfx_runtime* rt, const int64_t* xs, int xr, const int64_t* ys, int yr);
int runtime_launch(nfx_runtime* rt, const float* dx, const int64_t* xs, float* dy, cudaStream_t st);
cudaStream_t runtime_stream(nfx_runtime* rt);
int runtime_staging(nfx_runtime* rt, size_t nx, size_t ny, float** dx, float** dy);
int runtime_fail_str(nfx_runtime* rt, int code, const std::string& msg);
}  // namespace nfx

namespace {

// ---- NCCL, resolved at run time -------------------------------------------------
struct Nccl {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string why;
};

Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* env = std::getenv("NFX_NCCL_LIB");
        void* h = nullptr;
        if (env && *env) {
            h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
        } else {
            h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
            if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        }
        if (!h) {
            n.why = std::string("cannot load NCCL (libnccl.so.2): ") + (dlerror() ? dlerror() : "");
            return;
        }
        auto sym = [&](const char* name) { return dlsym(h, name); };
        n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(sym("ncclGetUniqueId"));
        n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(sym("ncclCommInitRank"));
        n.comm_init_all = reinterpret_cast<decltype(n.comm_init_all)>(sym("ncclCommInitAll"));
        n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(sym("ncclCommDestroy"));
        n.all_gather = reinterpret_cast<decltype(n.all_gather)>(sym("ncclAllGather"));
        n.send = reinterpret_cast<decltype(n.send)>(sym("ncclSend"));
        n.recv = reinterpret_cast<decltype(n.recv)>(sym("ncclRecv"));
        n.group_start = reinterpret_cast<decltype(n.group_start)>(sym("ncclGroupStart"));
        n.group_end = reinterpret_cast<decltype(n.group_end)>(sym("ncclGroupEnd"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(sym("ncclGetErrorString"));
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_init_all && n.comm_destroy &&
               n.all_gather && n.send && n.recv && n.group_start && n.group_end && n.error_string;
        if (!n.ok) n.why = "libnccl.so.2 lacks a required symbol";
    });
    return n;
}

std::string nccl_msg(const char* what, ncclResult_t r) {
    return std::string(what) + ": " + (nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

int64_t numel(const int64_t* s, int r) {
    int64_t n = 1;
    for (int i = 0; i < r; ++i) n *= s[i];
    return n;
}

// Contiguous slice of a batch: ceil(B / world) samples per rank, the last ranks
// possibly shorter or empty.
void slice_of(int64_t B, int world, int rank, int64_t* b0, int64_t* nb) {
    const int64_t per = world > 0 ? (B + world - 1) / world : B;
    const int64_t s = std::min<int64_t>(B, per * rank);
    *b0 = s;
    *nb = std::max<int64_t>(0, std::min<int64_t>(per, B - s));
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

// Gather of the fp32 output slices of every rank inside one full-batch buffer `y`
// (this rank's slice already written at its offset): to every rank (root < 0) or to
// `root` only.  Enqueued on `st`; the caller brackets nothing (group calls inside).
ncclResult_t gather_slices(float* y, int64_t B, int64_t per_sample, int world, int rank, int root,
                           ncclComm_t comm, cudaStream_t st) {
    Nccl& n = nccl();
    if (world == 1) return ncclSuccess;   // the one slice is the whole batch
    int64_t b0, nb;
    slice_of(B, world, rank, &b0, &nb);
    if (root < 0 && B % world == 0) {
        // equal slices: in-place all-gather (send buffer = this rank's part of y)
        return n.all_gather(y + b0 * per_sample, y, static_cast<size_t>(nb * per_sample), ncclFloat32,
                            comm, st);
    }
    ncclResult_t r = n.group_start();
    if (r != ncclSuccess) return r;
    for (int p = 0; p < world; ++p) {
        if (p == rank) continue;
        int64_t pb0, pnb;
        slice_of(B, world, p, &pb0, &pnb);
        const bool i_send = nb > 0 && (root < 0 || p == root);
        const bool i_recv = pnb > 0 && (root < 0 || rank == root);
        if (i_send && r == ncclSuccess)
            r = n.send(y + b0 * per_sample, static_cast<size_t>(nb * per_sample), ncclFloat32, p, comm, st);
        if (i_recv && r == ncclSuccess)
            r = n.recv(y + pb0 * per_sample, static_cast<size_t>(pnb * per_sample), ncclFloat32, p, comm, st);
    }
    const ncclResult_t r2 = n.group_end();
    return r != ncclSuccess ? r : r2;
}

}  // namespace

struct nfx_comm {
    ncclComm_t comm = nullptr;
    int world = 1, rank = 0, device = 0;
};

struct nfx_group {
    std::vector<nfx_runtime*> rts;
    std::vector<int> devices;
    std::vector<ncclComm_t> comms;     // created on first use by nfx_group_run_device
    std::vector<cudaStream_t> streams;
    std::vector<cudaEvent_t> events;
    std::string err;
};

namespace {
int group_fail(nfx_group* g, int code, const std::string& m) {
    g->err = m;
    return code;
}
}  // namespace

extern "C" {

void nfx_batch_slice(int64_t batch, int world, int rank, int64_t* first, int64_t* count) {
    int64_t b0 = 0, nb = 0;
    if (batch > 0 && world > 0 && rank >= 0 && rank < world) slice_of(batch, world, rank, &b0, &nb);
    if (first) *first = b0;
    if (count) *count = nb;
}

// ---- one process per GPU ----------------------------------------------------------

int nfx_comm_unique_id(unsigned char* id_out, int id_bytes) {
    Nccl& n = nccl();
    if (!n.ok) return nfx::set_thread_error(NFX_INTERNAL, n.why);
    if (!id_out || id_bytes < static_cast<int>(sizeof(ncclUniqueId)))
        return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_comm_unique_id: needs a 128-byte buffer");
    ncclUniqueId id;
    const ncclResult_t r = n.get_unique_id(&id);
    if (r != ncclSuccess) return nfx::set_thread_error(NFX_INTERNAL, nccl_msg("ncclGetUniqueId", r));
    std::memcpy(id_out, &id, sizeof(id));
    return NFX_OK;
}

int nfx_comm_create(const unsigned char* id, int id_bytes, int world, int rank, int device,
                    nfx_comm** out) {
    if (!out) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_comm_create: out is NULL");
    *out = nullptr;
    Nccl& n = nccl();
    if (!n.ok) return nfx::set_thread_error(NFX_INTERNAL, n.why);
    if (!id || id_bytes < static_cast<int>(sizeof(ncclUniqueId)))
        return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_comm_create: needs the 128-byte unique id");
    if (world < 1 || rank < 0 || rank >= world)
        return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_comm_create: rank out of range");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
        return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_comm_create: no such CUDA device");
    std::unique_ptr<nfx_comm> c(new nfx_comm());
    c->world = world;
    c->rank = rank;
    c->device = device;
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    DeviceGuard g(device);
    const ncclResult_t r = n.comm_init_rank(&c->comm, world, uid, rank);
    if (r != ncclSuccess) return nfx::set_thread_error(NFX_INTERNAL, nccl_msg("ncclCommInitRank", r));
    *out = c.release();
    return NFX_OK;
}

void nfx_comm_destroy(nfx_comm* c) {
    if (!c) return;
    if (c->comm) {
        DeviceGuard g(c->device);
        nccl().comm_destroy(c->comm);
    }
    delete c;
}

int nfx_runtime_run_sharded(nfx_runtime* rt, nfx_comm* comm, const float* x, const int64_t* x_shape,
                            int x_rank, float* y, const int64_t* y_shape, int y_rank, int root,
                            void* stream) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!comm) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "null communicator");
    if (comm->device != nfx::runtime_device(rt))
        return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "communicator and runtime are on different devices");
    if (root >= comm->world) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "root out of range");
    DeviceGuard g(comm->device);
    int s = nfx::runtime_check_shapes(rt, x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return s;
    const int64_t B = x_shape[0];
    if (B == 0) return NFX_OK;
    if (!x || !y) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "null buffer");
    const int64_t xs = numel(x_shape, x_rank) / B, ys = numel(y_shape, y_rank) / B;
    int64_t b0, nb;
    slice_of(B, comm->world, comm->rank, &b0, &nb);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (nb > 0) {
        std::vector<int64_t> shp(x_shape, x_shape + x_rank);
        shp[0] = nb;
        s = nfx::runtime_launch(rt, x + b0 * xs, shp.data(), y + b0 * ys, st);
        if (s != NFX_OK) return s;
    }
    const ncclResult_t r = gather_slices(y, B, ys, comm->world, comm->rank, root, comm->comm, st);
    if (r != ncclSuccess) return nfx::runtime_fail_str(rt, NFX_INTERNAL, nccl_msg("output gather", r));
    return NFX_OK;
}

int nfx_runtime_run_sharded_host(nfx_runtime* rt, nfx_comm* comm, const float* x,
                                 const int64_t* x_shape, int x_rank, float* y,
                                 const int64_t* y_shape, int y_rank, int root) {
    if (!rt) return nfx::set_thread_error(NFX_INVALID_ARG, "null runtime");
    if (!comm) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "null communicator");
    if (comm->device != nfx::runtime_device(rt))
        return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "communicator and runtime are on different devices");
    if (root >= comm->world) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "root out of range");
    DeviceGuard g(comm->device);
    int s = nfx::runtime_check_shapes(rt, x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return s;
    const int64_t B = x_shape[0];
    if (B == 0) return NFX_OK;
    if (!x || !y) return nfx::runtime_fail_str(rt, NFX_INVALID_ARG, "null buffer");
    const int64_t xs = numel(x_shape, x_rank) / B, ys = numel(y_shape, y_rank) / B;
    int64_t b0, nb;
    slice_of(B, comm->world, comm->rank, &b0, &nb);
    float* dx = nullptr;
    float* dy = nullptr;
    s = nfx::runtime_staging(rt, static_cast<size_t>(std::max<int64_t>(nb, 1) * xs),
                             static_cast<size_t>(B * ys), &dx, &dy);
    if (s != NFX_OK) return s;
    cudaStream_t st = nfx::runtime_stream(rt);
    if (nb > 0) {
        if (cudaMemcpyAsync(dx, x + b0 * xs, static_cast<size_t>(nb * xs) * 4, cudaMemcpyHostToDevice, st) !=
            cudaSuccess)
            return nfx::runtime_fail_str(rt, NFX_INTERNAL, "input copy failed");
        std::vector<int64_t> shp(x_shape, x_shape + x_rank);
        shp[0] = nb;
        s = nfx::runtime_launch(rt, dx, shp.data(), dy + b0 * ys, st);
        if (s != NFX_OK) {
            cudaStreamSynchronize(st);
            return s;
        }
    }
    const ncclResult_t r = gather_slices(dy, B, ys, comm->world, comm->rank, root, comm->comm, st);
    if (r != ncclSuccess) {
        cudaStreamSynchronize(st);
        return nfx::runtime_fail_str(rt, NFX_INTERNAL, nccl_msg("output gather", r));
    }
    if (root < 0 || root == comm->rank) {
        if (cudaMemcpyAsync(y, dy, static_cast<size_t>(B * ys) * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) {
            cudaStreamSynchronize(st);
            return nfx::runtime_fail_str(rt, NFX_INTERNAL, "output copy failed");
        }
    }
    if (cudaStreamSynchronize(st) != cudaSuccess)
        return nfx::runtime_fail_str(rt, NFX_INTERNAL, "sharded run failed");
    return nfx_runtime_check(rt);
}

// ---- one process, several GPUs --------------------------------------------------

int nfx_group_create(const char* ir_path, const int* devices, int n_devices, nfx_group** out) {
    if (!out) return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_group_create: out is NULL");
    *out = nullptr;
    if (!devices || n_devices < 1)
        return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_group_create: needs at least one device");
    for (int i = 0; i < n_devices; ++i)
        for (int j = 0; j < i; ++j)
            if (devices[i] == devices[j])
                return nfx::set_thread_error(NFX_INVALID_ARG, "nfx_group_create: a device is listed twice");
    std::unique_ptr<nfx_group> g(new nfx_group());
    for (int i = 0; i < n_devices; ++i) {
        nfx_runtime* rt = nullptr;
        const int s = nfx_runtime_create(ir_path, devices[i], &rt);
        if (s != NFX_OK) {
            for (auto* r : g->rts) nfx_runtime_destroy(r);
            return s;  // the thread error holds the member's message
        }
        g->rts.push_back(rt);
        g->devices.push_back(devices[i]);
    }
    *out = g.release();
    return NFX_OK;
}

void nfx_group_destroy(nfx_group* g) {
    if (!g) return;
    for (size_t i = 0; i < g->rts.size(); ++i) {
        DeviceGuard dg(g->devices[i]);
        cudaDeviceSynchronize();
        if (i < g->comms.size() && g->comms[i]) nccl().comm_destroy(g->comms[i]);
        if (i < g->streams.size() && g->streams[i]) cudaStreamDestroy(g->streams[i]);
        if (i < g->events.size() && g->events[i]) cudaEventDestroy(g->events[i]);
    }
    for (auto* r : g->rts) nfx_runtime_destroy(r);
    delete g;
}

int nfx_group_size(const nfx_group* g) { return g ? static_cast<int>(g->rts.size()) : 0; }

nfx_runtime* nfx_group_member(nfx_group* g, int i) {
    return (g && i >= 0 && i < static_cast<int>(g->rts.size())) ? g->rts[i] : nullptr;
}

const char* nfx_group_last_error(const nfx_group* g) { return g ? g->err.c_str() : ""; }

void nfx_group_enable_int8_gemm(nfx_group* g) {
    if (!g) return;
    for (auto* r : g->rts) nfx_runtime_enable_int8_gemm(r);
}

int nfx_group_is_int8_gemm_enabled(const nfx_group* g) {
    if (!g || g->rts.empty()) return 0;
    for (auto* r : g->rts)
        if (!nfx_runtime_is_int8_gemm_enabled(r)) return 0;
    return 1;
}

void nfx_group_enable_fp8(nfx_group* g) {
    if (!g) return;
    for (auto* r : g->rts) nfx_runtime_enable_fp8(r);
}

int nfx_group_run(nfx_group* g, const float* x, const int64_t* x_shape, int x_rank, float* y,
                  const int64_t* y_shape, int y_rank) {
    if (!g) return nfx::set_thread_error(NFX_INVALID_ARG, "null group");
    const int G = static_cast<int>(g->rts.size());
    int s = nfx::runtime_check_shapes(g->rts[0], x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return group_fail(g, s, nfx_runtime_last_error(g->rts[0]));
    const int64_t B = x_shape[0];
    if (B == 0) return NFX_OK;
    if (!x || !y) return group_fail(g, NFX_INVALID_ARG, "null buffer");
    const int64_t xs = numel(x_shape, x_rank) / B, ys = numel(y_shape, y_rank) / B;
    // every member runs the single-GPU host Run on its slice (copies overlapped with its
    // compute in chunks), one host thread per member
    std::vector<int> rc(G, NFX_OK);
    std::vector<std::thread> th;
    for (int m = 0; m < G; ++m) {
        int64_t b0, nb;
        slice_of(B, G, m, &b0, &nb);
        if (nb == 0) continue;
        th.emplace_back([&, m, b0, nb] {
            std::vector<int64_t> xsh(x_shape, x_shape + x_rank), ysh(y_shape, y_shape + y_rank);
            xsh[0] = nb;
            ysh[0] = nb;
            rc[m] = nfx_runtime_run(g->rts[m], x + b0 * xs, xsh.data(), x_rank, y + b0 * ys, ysh.data(),
                                    y_rank);
        });
    }
    for (auto& t : th) t.join();
    for (int m = 0; m < G; ++m)
        if (rc[m] != NFX_OK)
            return group_fail(g, rc[m], "device " + std::to_string(g->devices[m]) + ": " +
                                            nfx_runtime_last_error(g->rts[m]));
    return NFX_OK;
}

int nfx_group_run_device(nfx_group* g, const float* x, const int64_t* x_shape, int x_rank, float* y,
                         const int64_t* y_shape, int y_rank, void* stream) {
    if (!g) return nfx::set_thread_error(NFX_INVALID_ARG, "null group");
    const int G = static_cast<int>(g->rts.size());
    int s = nfx::runtime_check_shapes(g->rts[0], x_shape, x_rank, y_shape, y_rank);
    if (s != NFX_OK) return group_fail(g, s, nfx_runtime_last_error(g->rts[0]));
    const int64_t B = x_shape[0];
    if (B == 0) return NFX_OK;
    if (!x || !y) return group_fail(g, NFX_INVALID_ARG, "null buffer");
    const int64_t xs = numel(x_shape, x_rank) / B, ys = numel(y_shape, y_rank) / B;
    cudaStream_t caller = static_cast<cudaStream_t>(stream);
    if (G == 1) {
        DeviceGuard dg(g->devices[0]);
        s = nfx::runtime_launch(g->rts[0], x, x_shape, y, caller);
        return s == NFX_OK ? s : group_fail(g, s, nfx_runtime_last_error(g->rts[0]));
    }
    Nccl& n = nccl();
    if (!n.ok) return group_fail(g, NFX_INTERNAL, n.why);
    if (g->comms.empty()) {
        std::vector<ncclComm_t> comms(G, nullptr);
        const ncclResult_t r = n.comm_init_all(comms.data(), G, g->devices.data());
        if (r != ncclSuccess) return group_fail(g, NFX_INTERNAL, nccl_msg("ncclCommInitAll", r));
        g->comms = comms;
        g->streams.assign(G, nullptr);
        g->events.assign(G, nullptr);
        for (int m = 0; m < G; ++m) {
            DeviceGuard dg(g->devices[m]);
            if (cudaStreamCreateWithFlags(&g->streams[m], cudaStreamNonBlocking) != cudaSuccess ||
                cudaEventCreateWithFlags(&g->events[m], cudaEventDisableTiming) != cudaSuccess)
                return group_fail(g, NFX_INTERNAL, "creating the member streams failed");
        }
    }
    // member staging (members 1..G-1 hold their input and output slices)
    std::vector<int64_t> b0(G), nb(G);
    std::vector<float*> dx(G, nullptr), dy(G, nullptr);
    for (int m = 0; m < G; ++m) {
        slice_of(B, G, m, &b0[m], &nb[m]);
        if (m > 0 && nb[m] > 0) {
            DeviceGuard dg(g->devices[m]);
            s = nfx::runtime_staging(g->rts[m], static_cast<size_t>(nb[m] * xs), static_cast<size_t>(nb[m] * ys),
                                     &dx[m], &dy[m]);
            if (s != NFX_OK) return group_fail(g, s, nfx_runtime_last_error(g->rts[m]));
        }
    }
    // the members start after the work the caller queued before this call
    {
        DeviceGuard dg(g->devices[0]);
        if (cudaEventRecord(g->events[0], caller) != cudaSuccess)
            return group_fail(g, NFX_INTERNAL, "event record failed");
    }
    for (int m = 0; m < G; ++m) {
        DeviceGuard dg(g->devices[m]);
        if (cudaStreamWaitEvent(g->streams[m], g->events[0], 0) != cudaSuccess)
            return group_fail(g, NFX_INTERNAL, "event wait failed");
    }
    // scatter the input slices from the first device
    ncclResult_t r = n.group_start();
    for (int m = 1; m < G && r == ncclSuccess; ++m) {
        if (nb[m] == 0) continue;
        r = n.send(x + b0[m] * xs, static_cast<size_t>(nb[m] * xs), ncclFloat32, m, g->comms[0], g->streams[0]);
        if (r == ncclSuccess)
            r = n.recv(dx[m], static_cast<size_t>(nb[m] * xs), ncclFloat32, 0, g->comms[m], g->streams[m]);
    }
    ncclResult_t r2 = n.group_end();
    if (r != ncclSuccess || r2 != ncclSuccess)
        return group_fail(g, NFX_INTERNAL, nccl_msg("input scatter", r != ncclSuccess ? r : r2));
    // every member's forward on its own stream
    for (int m = 0; m < G; ++m) {
        if (nb[m] == 0) continue;
        DeviceGuard dg(g->devices[m]);
        std::vector<int64_t> shp(x_shape, x_shape + x_rank);
        shp[0] = nb[m];
        s = m == 0 ? nfx::runtime_launch(g->rts[0], x + b0[0] * xs, shp.data(), y + b0[0] * ys, g->streams[0])
                   : nfx::runtime_launch(g->rts[m], dx[m], shp.data(), dy[m], g->streams[m]);
        if (s != NFX_OK) return group_fail(g, s, nfx_runtime_last_error(g->rts[m]));
    }
    // gather the output slices into the caller's buffer
    r = n.group_start();
    for (int m = 1; m < G && r == ncclSuccess; ++m) {
        if (nb[m] == 0) continue;
        r = n.send(dy[m], static_cast<size_t>(nb[m] * ys), ncclFloat32, 0, g->comms[m], g->streams[m]);
        if (r == ncclSuccess)
            r = n.recv(y + b0[m] * ys, static_cast<size_t>(nb[m] * ys), ncclFloat32, m, g->comms[0], g->streams[0]);
    }
    r2 = n.group_end();
    if (r != ncclSuccess || r2 != ncclSuccess)
        return group_fail(g, NFX_INTERNAL, nccl_msg("output gather", r != ncclSuccess ? r : r2));
    // the caller's stream continues once the gathered outputs have arrived
    DeviceGuard dg(g->devices[0]);
    if (cudaEventRecord(g->events[0], g->streams[0]) != cudaSuccess ||
        cudaStreamWaitEvent(caller, g->events[0], 0) != cudaSuccess)
        return group_fail(g, NFX_INTERNAL, "event record failed");
    return NFX_OK;
}

int nfx_group_check(nfx_group* g) {
    if (!g) return nfx::set_thread_error(NFX_INVALID_ARG, "null group");
    for (size_t m = 0; m < g->rts.size(); ++m) {
        const int s = nfx_runtime_check(g->rts[m]);
        if (s != NFX_OK)
            return group_fail(g, s, "device " + std::to_string(g->devices[m]) + ": " +
                                        nfx_runtime_last_error(g->rts[m]));
    }
    return NFX_OK;
}

}  // extern "C"
