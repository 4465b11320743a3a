// nflow_infer -- command-line front-end of libnfx.so with the reference CLI's flags
// (cpp/src/main.cpp:27-115): --model <file.nneuroir> --input <x.npy> --output <y.npy>.
// Written against nflow::InferenceRuntime (include/nflow_runtime.hpp), the reference's
// C++ interface over the C-ABI, as the reference CLI is written against its own.
// Extra flags: --int8 (EnableInt8Gemm), --fp8 (the FNO3d E4M3 executor), --device N.
// TokenMixer, GraphOp, TokenMixer2D and GraphOp2D models run through their own Run
// calls like the reference's `infer` (pybind_module.cpp:61-111); DeepONet, with two
// inputs, is refused as by the reference CLI.  Exit code 0 on success, 1 on any error,
// as the reference.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "nflow_runtime.hpp"

namespace {

// .npy v1/v2/v3 reader for little-endian float32 C-order arrays.
bool read_npy(const std::string& path, std::vector<int64_t>& shape, std::vector<float>& data,
              std::string& err) {
    std::ifstream f(path, std::ios::binary);
    if (!f) {
        err = "cannot open " + path;
        return false;
    }
    char magic[6];
    uint8_t ver[2];
    if (!f.read(magic, 6) || std::memcmp(magic, "\x93NUMPY", 6) != 0 ||
        !f.read(reinterpret_cast<char*>(ver), 2)) {
        err = "not a .npy file";
        return false;
    }
    uint32_t hlen = 0;
    if (ver[0] == 1) {
        uint16_t h16 = 0;
        f.read(reinterpret_cast<char*>(&h16), 2);
        hlen = h16;
    } else {
        f.read(reinterpret_cast<char*>(&hlen), 4);
    }
    std::string header(hlen, '\0');
    if (!f.read(&header[0], hlen)) {
        err = "truncated .npy header";
        return false;
    }
    auto value_of = [&](const std::string& key) -> std::string {
        const size_t k = header.find("'" + key + "'");
        if (k == std::string::npos) return "";
        size_t v = header.find(':', k);
        if (v == std::string::npos) return "";
        ++v;
        while (v < header.size() && header[v] == ' ') ++v;
        if (header[v] == '(') return header.substr(v, header.find(')', v) - v + 1);
        size_t e = v;
        while (e < header.size() && header[e] != ',' && header[e] != '}') ++e;
        return header.substr(v, e - v);
    };
    const std::string descr = value_of("descr");
    if (descr.find("<f4") == std::string::npos && descr.find("=f4") == std::string::npos) {
        err = "expected float32 little-endian data, got descr " + descr;
        return false;
    }
    if (value_of("fortran_order").find("False") == std::string::npos) {
        err = "fortran-ordered arrays are not supported";
        return false;
    }
    const std::string s = value_of("shape");
    shape.clear();
    int64_t n = 1;
    for (size_t i = 1; i < s.size(); ++i) {
        if (s[i] >= '0' && s[i] <= '9') {
            int64_t v = 0;
            while (i < s.size() && s[i] >= '0' && s[i] <= '9') v = v * 10 + (s[i++] - '0');
            shape.push_back(v);
            n *= v;
        }
    }
    data.resize(static_cast<size_t>(n));
    if (n && !f.read(reinterpret_cast<char*>(data.data()), n * 4)) {
        err = "truncated .npy data";
        return false;
    }
    return true;
}

bool write_npy(const std::string& path, const std::vector<int64_t>& shape, const std::vector<float>& data,
               std::string& err) {
    std::ostringstream h;
    h << "{'descr': '<f4', 'fortran_order': False, 'shape': (";
    for (size_t i = 0; i < shape.size(); ++i) h << shape[i] << (shape.size() == 1 || i + 1 < shape.size() ? ", " : "");
    h << "), }";
    std::string header = h.str();
    const size_t total = 10 + header.size() + 1;
    header.append((64 - total % 64) % 64, ' ');
    header.push_back('\n');
    std::ofstream f(path, std::ios::binary);
    if (!f) {
        err = "cannot open " + path + " for writing";
        return false;
    }
    const uint16_t hl = static_cast<uint16_t>(header.size());
    f.write("\x93NUMPY\x01\x00", 8);
    f.write(reinterpret_cast<const char*>(&hl), 2);
    f.write(header.data(), static_cast<std::streamsize>(header.size()));
    f.write(reinterpret_cast<const char*>(data.data()), static_cast<std::streamsize>(data.size() * 4));
    if (!f) {
        err = "write failed";
        return false;
    }
    return true;
}

void usage() {
    std::cout << "Usage: nflow_infer --model <file.nneuroir> --input <x.npy> --output <y.npy> "
                 "[--int8] [--fp8] [--device N]\n";
}

}  // namespace

int main(int argc, char** argv) {
    std::string model, input, output;
    bool int8 = false, fp8 = false;
    int device = 0;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (a == "--model" && i + 1 < argc) model = argv[++i];
        else if (a == "--input" && i + 1 < argc) input = argv[++i];
        else if (a == "--output" && i + 1 < argc) output = argv[++i];
        else if (a == "--device" && i + 1 < argc) device = std::atoi(argv[++i]);
        else if (a == "--int8") int8 = true;
        else if (a == "--fp8") fp8 = true;
        else if (a == "--help" || a == "-h") {
            usage();
            return 0;
        }
    }
    if (model.empty() || input.empty() || output.empty()) {
        usage();
        return 1;
    }
    nflow::LoadedModelInfo info;
    nflow::Status st = nflow::LoadNeuroIr(model, info);
    if (!st.ok()) {
        std::cerr << "model load failed: " << st.message() << std::endl;
        return 1;
    }
    const std::string& ops = info.op;
    int rank = 0;
    int64_t out_ch = 0;
    if (ops == "FNO1d") rank = 3, out_ch = info.cfg[1];
    else if (ops == "FNO2d") rank = 4, out_ch = info.cfg[1];
    else if (ops == "FNO3d") rank = 5, out_ch = info.cfg[1];
    else if (ops == "TokenMixer2D" || ops == "GraphOp2D") rank = 4, out_ch = info.cfg[1];
    else if (ops == "TokenMixer" || ops == "GraphOp") rank = 3, out_ch = info.cfg[1];
    else {
        std::cerr << "unsupported op in IR: " << ops << std::endl;
        return 1;
    }
    std::vector<int64_t> xs;
    std::vector<float> x;
    std::string err;
    if (!read_npy(input, xs, x, err)) {
        std::cerr << "input read failed: " << err << std::endl;
        return 1;
    }
    if (static_cast<int>(xs.size()) != rank) {
        std::cerr << "expected " << rank << "D input for " << ops << ", got rank " << xs.size() << std::endl;
        return 1;
    }
    std::unique_ptr<nflow::InferenceRuntime> rt;
    st = nflow::InferenceRuntime::CreateOnDevice(model, device, rt);
    if (!st.ok()) {
        std::cerr << "runtime create failed: " << st.message() << std::endl;
        return 1;
    }
    if (int8) rt->EnableInt8Gemm();
    if (fp8) rt->EnableFp8();
    std::vector<int64_t> ys = xs;
    ys.back() = out_ch;
    int64_t ny = 1;
    for (auto d : ys) ny *= d;
    std::vector<float> y(static_cast<size_t>(ny));
    if (ops == "TokenMixer2D") st = rt->RunTokenMixer2D(x.data(), xs, y.data(), ys);
    else if (ops == "TokenMixer") st = rt->RunTokenMixer(x.data(), xs, y.data(), ys);
    else if (ops == "GraphOp") st = rt->RunGraphOp(x.data(), xs, y.data(), ys);
    else if (ops == "GraphOp2D") st = rt->RunGraphOp2D(x.data(), xs, y.data(), ys);
    else st = rt->Run(x.data(), xs, y.data(), ys);
    if (!st.ok()) {
        std::cerr << "inference failed: " << st.message() << std::endl;
        return 1;
    }
    rt.reset();
    if (!write_npy(output, ys, y, err)) {
        std::cerr << "output write failed: " << err << std::endl;
        return 1;
    }
    std::cout << "ok: wrote " << output << " op=" << ops << " shape=(";
    for (size_t i = 0; i < ys.size(); ++i) std::cout << (i ? "," : "") << ys[i];
    std::cout << ")" << std::endl;
    return 0;
}
