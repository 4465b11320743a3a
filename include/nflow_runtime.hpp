// nflow_runtime.hpp -- the reference's C++ inference interface, nflow::Status and
// nflow::InferenceRuntime (cpp/include/neuroflow/tensor.h:29-60,
// cpp/include/neuroflow/runtime.h:64-135), implemented header-only over the C-ABI of
// libnfx.so (nfx.h).  A C++ caller of the reference runtime (nflow_infer, the pybind
// module, an embedding application) switches to the B200 runtime by including this
// header instead of neuroflow/runtime.h and linking libnfx.so; the calls, return
// values and messages stay the same.
//
// Differences a caller can see: Create binds the runtime to CUDA device 0 (or the
// device given to CreateOnDevice); RunDeepONet refuses u and y of different batch
// sizes (ShapeMismatch), and GraphOp / GraphOp2D a graph whose indices leave the node
// range (InvalidArg), where the reference reads outside its buffers; and LoadNeuroIr
// fills a LoadedModelInfo (op, config block, weight count, NIRQ flag) rather than the
// reference's weight-holding LoadedModel.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "nfx.h"

namespace nflow {

// tensor.h:29-37
enum class StatusCode {
    Ok = 0,
    InvalidArg = 1,
    FileNotFound = 2,
    ParseError = 3,
    ShapeMismatch = 4,
    UnsupportedOp = 5,
    Internal = 99,
};

// tensor.h:39-60
class Status {
public:
    Status() = default;
    explicit Status(StatusCode code, std::string msg = "") : code_(code), msg_(std::move(msg)) {}

    bool ok() const { return code_ == StatusCode::Ok; }
    StatusCode code() const { return code_; }
    const std::string& message() const { return msg_; }

    static Status Ok() { return Status(StatusCode::Ok); }
    static Status InvalidArg(std::string m) { return Status(StatusCode::InvalidArg, std::move(m)); }
    static Status FileNotFound(std::string m) { return Status(StatusCode::FileNotFound, std::move(m)); }
    static Status ParseError(std::string m) { return Status(StatusCode::ParseError, std::move(m)); }
    static Status ShapeMismatch(std::string m) { return Status(StatusCode::ShapeMismatch, std::move(m)); }
    static Status UnsupportedOp(std::string m) { return Status(StatusCode::UnsupportedOp, std::move(m)); }
    static Status Internal(std::string m) { return Status(StatusCode::Internal, std::move(m)); }

private:
    StatusCode code_ = StatusCode::Ok;
    std::string msg_;
};

// What LoadNeuroIr (runtime.h:66) reports without building the model: the op, the
// 8-int config block of the IR header (unused slots 0), the number of weights, and
// whether a NIRQ quantisation block is present.
struct LoadedModelInfo {
    std::string op;
    int32_t cfg[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int n_weights = 0;
    bool quant_enabled = false;
};

namespace detail {
inline Status from_code(int code, const char* msg) {
    return code == NFX_OK ? Status::Ok() : Status(static_cast<StatusCode>(code), msg ? msg : "");
}
}  // namespace detail

inline Status LoadNeuroIr(const std::string& path, LoadedModelInfo& out) {
    char op[32] = {0};
    int nw = 0, q = 0;
    const int s = nfx_load_neuroir(path.c_str(), op, static_cast<int>(sizeof(op)), out.cfg, &nw, &q);
    if (s != NFX_OK) return detail::from_code(s, nfx_last_error());
    out.op = op;
    out.n_weights = nw;
    out.quant_enabled = q != 0;
    return Status::Ok();
}

// runtime.h:69-135: load once, run many.  Not thread-safe (one thread per runtime),
// like the reference.
class InferenceRuntime {
public:
    ~InferenceRuntime() {
        if (rt_) nfx_runtime_destroy(rt_);
    }
    InferenceRuntime(const InferenceRuntime&) = delete;
    InferenceRuntime& operator=(const InferenceRuntime&) = delete;

    static Status Create(const std::string& ir_path, std::unique_ptr<InferenceRuntime>& out) {
        return CreateOnDevice(ir_path, 0, out);
    }

    // Create on a chosen CUDA device (no counterpart in the reference).
    static Status CreateOnDevice(const std::string& ir_path, int device,
                                 std::unique_ptr<InferenceRuntime>& out) {
        nfx_runtime* h = nullptr;
        const int s = nfx_runtime_create(ir_path.c_str(), device, &h);
        if (s != NFX_OK) return detail::from_code(s, nfx_last_error());
        out.reset(new InferenceRuntime(h));
        return Status::Ok();
    }

    // x, y: host float32 row-major buffers (runtime.h:76-79)
    Status Run(const float* x, const std::vector<int64_t>& x_shape, float* y,
               const std::vector<int64_t>& y_shape) {
        return status(nfx_runtime_run(rt_, x, x_shape.data(), static_cast<int>(x_shape.size()), y,
                                      y_shape.data(), static_cast<int>(y_shape.size())));
    }

    Status RunTokenMixer2D(const float* x, const std::vector<int64_t>& x_shape, float* y,
                           const std::vector<int64_t>& y_shape) {
        return status(nfx_runtime_run_tokenmixer2d(rt_, x, x_shape.data(), static_cast<int>(x_shape.size()),
                                                   y, y_shape.data(), static_cast<int>(y_shape.size())));
    }

    // runtime.h:82-84
    Status RunDeepONet(const float* u, const std::vector<int64_t>& u_shape, const float* y,
                       const std::vector<int64_t>& y_shape, float* out, const std::vector<int64_t>& out_shape) {
        return status(nfx_runtime_run_deeponet(rt_, u, u_shape.data(), static_cast<int>(u_shape.size()), y,
                                               y_shape.data(), static_cast<int>(y_shape.size()), out,
                                               out_shape.data(), static_cast<int>(out_shape.size())));
    }
    // runtime.h:88-89
    Status RunTokenMixer(const float* x, const std::vector<int64_t>& x_shape, float* y,
                         const std::vector<int64_t>& y_shape) {
        return status(nfx_runtime_run_tokenmixer(rt_, x, x_shape.data(), static_cast<int>(x_shape.size()), y,
                                                 y_shape.data(), static_cast<int>(y_shape.size())));
    }
    // runtime.h:93-94
    Status RunGraphOp(const float* x, const std::vector<int64_t>& x_shape, float* y,
                      const std::vector<int64_t>& y_shape) {
        return status(nfx_runtime_run_graphop(rt_, x, x_shape.data(), static_cast<int>(x_shape.size()), y,
                                              y_shape.data(), static_cast<int>(y_shape.size())));
    }
    // runtime.h:103-104
    Status RunGraphOp2D(const float* x, const std::vector<int64_t>& x_shape, float* y,
                        const std::vector<int64_t>& y_shape) {
        return status(nfx_runtime_run_graphop2d(rt_, x, x_shape.data(), static_cast<int>(x_shape.size()), y,
                                                y_shape.data(), static_cast<int>(y_shape.size())));
    }

    const std::string& op() const { return op_; }

    void EnableInt8Gemm() { nfx_runtime_enable_int8_gemm(rt_); }
    bool IsInt8GemmEnabled() const { return nfx_runtime_is_int8_gemm_enabled(rt_) != 0; }

    // FNO3d FP8 E4M3 executor (no counterpart in the reference)
    void EnableFp8() { nfx_runtime_enable_fp8(rt_); }
    bool IsFp8Enabled() const { return nfx_runtime_is_fp8_enabled(rt_) != 0; }

    // The underlying C-ABI handle, for the device-buffer and multi-GPU entry points.
    nfx_runtime* handle() const { return rt_; }

private:
    explicit InferenceRuntime(nfx_runtime* h) : rt_(h), op_(nfx_runtime_op(h)) {}
    Status status(int s) const { return detail::from_code(s, nfx_runtime_last_error(rt_)); }

    nfx_runtime* rt_ = nullptr;
    std::string op_;
};

}  // namespace nflow
