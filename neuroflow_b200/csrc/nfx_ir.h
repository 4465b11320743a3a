// nfx_ir.h -- NeuroIR v0 binary (.nneuroir) + NIRQ block loader.
//
// Same byte format and the same acceptance rules as the reference loader
// (cpp/include/neuroflow/ir_loader.h:61-653): magic "NIR0", version 1..3, op code
// 1..8, a 7- or 8-int32 config block, activation byte, named float32 weights in the
// fixed per-op order (name-checked), and the optional trailing "NIRQ" block with
// per-tensor (kind 0), per-channel (1), per-token (2) and FP8 (3) entries.  Kind-0
// names ending in ".output" are activation qparams, the rest weight qparams
// (ir_loader.h:577-585).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace nfx {

struct HostTensor {
    std::vector<int64_t> shape;
    std::vector<float> data;
    int64_t numel() const {
        int64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }
};

struct QP {
    float scale = 1.0f;
    int32_t zero_point = 0;
};

struct PerChannelQP {
    std::vector<float> scales;
    std::vector<int32_t> zero_points;
    int32_t channel_axis = 0;
};

struct PerTokenQP {
    std::vector<float> scales;
    std::vector<int32_t> zero_points;
    int32_t width = 0;
};

struct IrModel {
    std::string op;
    int32_t cfg[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    std::string activation = "gelu";
    std::vector<std::string> weight_order;
    std::unordered_map<std::string, HostTensor> weights;
    bool quant_enabled = false;
    std::unordered_map<std::string, QP> weight_qparams;
    std::unordered_map<std::string, QP> activation_qparams;
    std::unordered_map<std::string, PerChannelQP> weight_per_channel_qparams;
    std::unordered_map<std::string, PerTokenQP> activation_per_token_qparams;
    std::unordered_map<std::string, float> activation_fp8_qparams;
};

// Returns a reference StatusCode (0 ok) and fills `msg` on error.
int load_ir(const std::string& path, IrModel& out, std::string& msg);

// fno.cpp:217-290 DequantiseWeight applied in place (load-time weight fake-quant).
bool dequantise_weight(HostTensor& t, const IrModel& m, const std::string& name);

// fno.cpp:325-358 QuantiseWeight2D: per-output-row codes and sum_W_per_row.
bool quantise_weight_2d(const HostTensor& t, const PerChannelQP& pcp, std::vector<int8_t>& codes,
                        std::vector<int32_t>& sum_w);

}  // namespace nfx
