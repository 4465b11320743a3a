// nfx_ir.cpp -- NeuroIR v0 + NIRQ loader and the load-time weight transforms.
#include "nfx_ir.h"

#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>

#include "../../include/nfx.h"

namespace nfx {
namespace {

struct Cursor {
    const uint8_t* p;
    size_t n;
    size_t off = 0;
    bool u8(uint8_t& v) {
        if (off + 1 > n) return false;
        v = p[off++];
        return true;
    }
    bool u16(uint16_t& v) {
        if (off + 2 > n) return false;
        std::memcpy(&v, p + off, 2);
        off += 2;
        return true;
    }
    bool i32(int32_t& v) {
        if (off + 4 > n) return false;
        std::memcpy(&v, p + off, 4);
        off += 4;
        return true;
    }
    bool u32(uint32_t& v) {
        if (off + 4 > n) return false;
        std::memcpy(&v, p + off, 4);
        off += 4;
        return true;
    }
};

// The fixed weight order per op (ir_loader.h:273-532).
std::vector<std::string> weight_names(const IrModel& m) {
    std::vector<std::string> w;
    const auto& c = m.cfg;
    if (m.op == "FNO1d" || m.op == "FNO2d" || m.op == "FNO3d") {
        const int L = m.op == "FNO1d" ? c[4] : (m.op == "FNO2d" ? c[5] : c[6]);
        w = {"lift.weight", "lift.bias"};
        for (int i = 0; i < L; ++i) {
            const std::string s = std::to_string(i);
            w.push_back("specs." + s + ".weights_real");
            w.push_back("specs." + s + ".weights_imag");
            w.push_back("locs." + s + ".weight");
            w.push_back("locs." + s + ".bias");
        }
        for (const char* n : {"proj_q.weight", "proj_q.bias", "proj_out.weight", "proj_out.bias"})
            w.push_back(n);
    } else if (m.op == "TokenMixer" || m.op == "TokenMixer2D") {
        const int L = m.op == "TokenMixer" ? c[6] : c[7];
        w = {"slice_embed.proj.weight", "slice_embed.proj.bias"};
        for (int i = 0; i < L; ++i) {
            const std::string pre = "blocks." + std::to_string(i) + ".";
            for (const char* part : {"ln1", "q_proj", "k_proj", "v_proj", "o_proj", "ln2", "ffn0", "ffn1"}) {
                w.push_back(pre + part + ".weight");
                w.push_back(pre + part + ".bias");
            }
        }
        for (const char* n : {"unslice.proj.weight", "unslice.proj.bias", "head.weight", "head.bias"})
            w.push_back(n);
    } else if (m.op == "GraphOp" || m.op == "GraphOp2D") {
        const int L = m.op == "GraphOp" ? c[4] : c[5];
        w = {"lift.weight", "lift.bias"};
        for (int i = 0; i < L; ++i) {
            const std::string pre = "blocks." + std::to_string(i) + ".";
            for (const char* part : {"lin_self.weight", "lin_self.bias", "lin_neigh.weight", "lin_neigh.bias"})
                w.push_back(pre + part);
        }
        for (const char* n : {"head.weight", "head.bias", "graph.adj_offsets", "graph.adj_indices", "graph.deg_inv"})
            w.push_back(n);
    } else if (m.op == "DeepONet") {
        for (int i = 0; i < c[4]; ++i) {
            w.push_back("branch.layers." + std::to_string(i) + ".weight");
            w.push_back("branch.layers." + std::to_string(i) + ".bias");
        }
        for (int i = 0; i < c[5]; ++i) {
            w.push_back("trunk.layers." + std::to_string(i) + ".weight");
            w.push_back("trunk.layers." + std::to_string(i) + ".bias");
        }
        w.push_back("bias.weight");
    }
    return w;
}

inline float fake_quant_pt(float v, float s, float zp) {
    float q = std::round(v / s) + zp;
    if (q < -128.0f) q = -128.0f;
    if (q > 127.0f) q = 127.0f;
    return (q - zp) * s;
}

}  // namespace

int load_ir(const std::string& path, IrModel& out, std::string& msg) {
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) {
        msg = "cannot open IR file: " + path;
        return NFX_FILE_NOT_FOUND;
    }
    std::ostringstream ss;
    ss << f.rdbuf();
    const std::string buf = ss.str();
    Cursor cur{reinterpret_cast<const uint8_t*>(buf.data()), buf.size()};
    auto parse_err = [&](const std::string& m) {
        msg = m;
        return NFX_PARSE_ERROR;
    };
    if (cur.n < 4 || std::memcmp(cur.p, "NIR0", 4) != 0) return parse_err("bad magic in IR file");
    cur.off = 4;
    uint16_t version = 0;
    if (!cur.u16(version)) return parse_err("truncated header");
    if (version != 1 && version != 2 && version != 3) return parse_err("unsupported IR binary version");
    uint8_t op_code = 0, reserved = 0;
    if (!cur.u8(op_code) || !cur.u8(reserved)) return parse_err("truncated header");
    static const char* kOps[] = {"", "FNO1d", "FNO2d", "FNO3d", "DeepONet",
                                 "TokenMixer", "GraphOp", "TokenMixer2D", "GraphOp2D"};
    if (op_code < 1 || op_code > 8) {
        msg = "unknown op_code";
        return NFX_UNSUPPORTED_OP;
    }
    out.op = kOps[op_code];
    const int cfg_len = (op_code == 3 || op_code == 5 || op_code == 6 || op_code == 7 || op_code == 8) ? 8 : 7;
    for (int i = 0; i < cfg_len; ++i)
        if (!cur.i32(out.cfg[i])) return parse_err("truncated config");
    uint8_t act = 0;
    if (!cur.u8(act)) return parse_err("truncated activation");
    out.activation = act == 1 ? "relu" : "gelu";
    cur.off += 3;
    uint32_t n_weights = 0;
    if (!cur.u32(n_weights)) return parse_err("truncated n_weights");

    for (const std::string& name : weight_names(out)) {
        uint8_t name_len = 0;
        if (!cur.u8(name_len)) return parse_err("truncated name_len");
        if (cur.off + name_len > cur.n) return parse_err("truncated name");
        std::string read_name(reinterpret_cast<const char*>(cur.p + cur.off), name_len);
        cur.off += name_len;
        if (read_name != name) return parse_err("weight name mismatch: " + read_name + " != " + name);
        uint8_t ndim = 0;
        if (!cur.u8(ndim)) return parse_err("truncated ndim");
        HostTensor t;
        t.shape.resize(ndim);
        for (int i = 0; i < ndim; ++i) {
            int32_t d = 0;
            if (!cur.i32(d)) return parse_err("truncated dim");
            t.shape[i] = d;
        }
        const int64_t numel = t.numel();
        if (numel < 0) return parse_err("truncated data");
        const size_t bytes = static_cast<size_t>(numel) * sizeof(float);
        if (cur.off + bytes > cur.n) return parse_err("truncated data");
        t.data.resize(static_cast<size_t>(numel));
        if (bytes) std::memcpy(t.data.data(), cur.p + cur.off, bytes);
        cur.off += bytes;
        out.weight_order.push_back(name);
        out.weights[name] = std::move(t);
    }

    if (cur.off + 4 <= cur.n && std::memcmp(cur.p + cur.off, "NIRQ", 4) == 0) {
        cur.off += 4;
        uint8_t flag = 0;
        if (!cur.u8(flag)) return parse_err("truncated quant_flag");
        if (flag != 1) return parse_err("unsupported quant_flag");
        out.quant_enabled = true;
        uint32_t nq = 0;
        if (!cur.u32(nq)) return parse_err("truncated n_qparams");
        for (uint32_t i = 0; i < nq; ++i) {
            uint8_t kind = 0, name_len = 0;
            if (!cur.u8(kind)) return parse_err("truncated qparam kind");
            if (!cur.u8(name_len)) return parse_err("truncated qparam name_len");
            if (cur.off + name_len > cur.n) return parse_err("truncated qparam name");
            std::string name(reinterpret_cast<const char*>(cur.p + cur.off), name_len);
            cur.off += name_len;
            if (kind == 0) {
                if (cur.off + 8 > cur.n) return parse_err("truncated qparam scale/zp");
                QP qp;
                std::memcpy(&qp.scale, cur.p + cur.off, 4);
                std::memcpy(&qp.zero_point, cur.p + cur.off + 4, 4);
                cur.off += 8;
                if (name.size() >= 7 && name.compare(name.size() - 7, 7, ".output") == 0)
                    out.activation_qparams[name] = qp;
                else
                    out.weight_qparams[name] = qp;
            } else if (kind == 1) {
                if (cur.off + 5 > cur.n) return parse_err("truncated per-channel header");
                uint32_t n_ch = 0;
                uint8_t axis = 0;
                std::memcpy(&n_ch, cur.p + cur.off, 4);
                std::memcpy(&axis, cur.p + cur.off + 4, 1);
                cur.off += 5;
                if (cur.off + static_cast<size_t>(n_ch) * 8 > cur.n)
                    return parse_err("truncated per-channel data");
                PerChannelQP pc;
                pc.channel_axis = axis;
                pc.scales.resize(n_ch);
                pc.zero_points.resize(n_ch);
                std::memcpy(pc.scales.data(), cur.p + cur.off, n_ch * 4);
                std::memcpy(pc.zero_points.data(), cur.p + cur.off + n_ch * 4, n_ch * 4);
                cur.off += static_cast<size_t>(n_ch) * 8;
                out.weight_per_channel_qparams[name] = std::move(pc);
            } else if (kind == 2) {
                if (cur.off + 8 > cur.n) return parse_err("truncated per-token header");
                uint32_t n_tok = 0, width = 0;
                std::memcpy(&n_tok, cur.p + cur.off, 4);
                std::memcpy(&width, cur.p + cur.off + 4, 4);
                cur.off += 8;
                if (cur.off + static_cast<size_t>(n_tok) * 8 > cur.n)
                    return parse_err("truncated per-token data");
                PerTokenQP pt;
                pt.width = static_cast<int32_t>(width);
                pt.scales.resize(n_tok);
                pt.zero_points.resize(n_tok);
                std::memcpy(pt.scales.data(), cur.p + cur.off, n_tok * 4);
                std::memcpy(pt.zero_points.data(), cur.p + cur.off + n_tok * 4, n_tok * 4);
                cur.off += static_cast<size_t>(n_tok) * 8;
                out.activation_per_token_qparams[name] = std::move(pt);
            } else if (kind == 3) {
                if (cur.off + 4 > cur.n) return parse_err("truncated fp8 scale");
                float s = 0.0f;
                std::memcpy(&s, cur.p + cur.off, 4);
                cur.off += 4;
                out.activation_fp8_qparams[name] = s;
            } else {
                return parse_err("unsupported qparam kind");
            }
        }
    }
    return NFX_OK;
}

bool dequantise_weight(HostTensor& t, const IrModel& m, const std::string& name) {
    auto pc = m.weight_per_channel_qparams.find(name);
    if (pc != m.weight_per_channel_qparams.end()) {
        const auto& q = pc->second;
        const int64_t n_ch = static_cast<int64_t>(q.scales.size());
        if (t.shape.size() == 2 && q.channel_axis == 0) {
            for (int64_t c = 0; c < n_ch; ++c) {
                const float s = q.scales[c];
                const float zp = static_cast<float>(q.zero_points[c]);
                for (int64_t i = 0; i < t.shape[1]; ++i) {
                    const int64_t off = c * t.shape[1] + i;
                    t.data[off] = fake_quant_pt(t.data[off], s, zp);
                }
            }
            return true;
        } else if (t.shape.size() == 3 && q.channel_axis == 1) {
            const int64_t in_dim = t.shape[0], out_dim = t.shape[1], modes = t.shape[2];
            for (int64_t i = 0; i < in_dim; ++i)
                for (int64_t c = 0; c < out_dim; ++c) {
                    const float s = q.scales[c];
                    const float zp = static_cast<float>(q.zero_points[c]);
                    for (int64_t k = 0; k < modes; ++k) {
                        const int64_t off = i * (out_dim * modes) + c * modes + k;
                        t.data[off] = fake_quant_pt(t.data[off], s, zp);
                    }
                }
            return true;
        }
    }
    auto pt = m.weight_qparams.find(name);
    if (pt != m.weight_qparams.end()) {
        const float s = pt->second.scale;
        const float zp = static_cast<float>(pt->second.zero_point);
        for (auto& v : t.data) v = fake_quant_pt(v, s, zp);
        return true;
    }
    return false;
}

bool quantise_weight_2d(const HostTensor& t, const PerChannelQP& pcp, std::vector<int8_t>& codes,
                        std::vector<int32_t>& sum_w) {
    if (t.shape.size() != 2 || pcp.channel_axis != 0) return false;
    const int64_t n = t.shape[0], k = t.shape[1];
    if (static_cast<int64_t>(pcp.scales.size()) < n) return false;
    codes.assign(static_cast<size_t>(n * k), 0);
    sum_w.assign(static_cast<size_t>(n), 0);
    for (int64_t c = 0; c < n; ++c) {
        const float s = pcp.scales[c];
        const float zp = static_cast<float>(pcp.zero_points[c]);
        int32_t row_sum = 0;
        for (int64_t i = 0; i < k; ++i) {
            float q = std::round(t.data[c * k + i] / s) + zp;
            if (q < -128.0f) q = -128.0f;
            if (q > 127.0f) q = 127.0f;
            const int8_t q8 = static_cast<int8_t>(q);
            codes[c * k + i] = q8;
            row_sum += static_cast<int32_t>(q8) - pcp.zero_points[c];
        }
        sum_w[c] = row_sum;
    }
    return true;
}

}  // namespace nfx
