// mlp_ops.h -- GPU executors of the reference's MLP-style operators (sm_100a):
// DeepONet::Forward (cpp/src/fno.cpp:1289-1406) and GraphOp / GraphOp2D::Forward
// (fno.cpp:1653-1741, :1969-2060), FP32 with the reference's rounding.
//
// All three are chains of the reference Linear (fno.cpp:51-80) over rows of a few dozen
// to a few hundred features, plus a per-row reduction (the sensor mean, the
// branch-trunk dot product, the neighbour aggregation).  Each row is one thread's work:
// its features sit in shared memory ([threads][dim + 1], conflict-free across lanes),
// every Linear output is the reference's in-order dot product (linear_step), and the
// weights are read as warp-uniform broadcast loads.  Rows are moved between global and
// shared memory cooperatively, so the global traffic stays coalesced.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace nfx {

constexpr int kMlpMaxLayers = 8;
constexpr int kMlpMaxDim = 512;      // widest row the shared-memory layout takes
constexpr int kGraphMaxHidden = 256;

struct MlpLayer {
    const float* w;  // (out, in), the reference's nn.Linear layout
    const float* b;  // (out)
    int in, out;
};

// Rows through a Linear chain, the activation after every layer but the last
// (DeepONet's MLPs, fno.cpp:1325-1343 and :1368-1385; GraphOp's lift and head are
// one-layer chains).  With `dot_branch`, the chain's last output row t of row r
// (latent wide) is not stored; instead
//   y[r, c] = dot(dot_branch[(r / rows_per_group) * dot_ch + c, :], t) + dot_bias[c]
// for c < dot_ch (DeepONet's output, fno.cpp:1388-1398), the dot product in the
// reference's order and fusion.
struct MlpArgs {
    const float* x;
    int64_t rows;
    float* y;
    int n_layers;
    MlpLayer layer[kMlpMaxLayers];
    int act;  // 1 ReLU, 0 GELU (tanh form)
    const float* dot_branch;
    const float* dot_bias;
    int dot_ch;
    int64_t rows_per_group;
};

// DeepONet branch mean (fno.cpp:1352-1361): out[g, f] = (sum_s in[g, s, f]) / n, the sum
// sequential over s.
struct MeanArgs {
    const float* in;  // (groups, n, F)
    float* out;       // (groups, F)
    int64_t groups;
    int n, F;
};

// One GraphOp block (fno.cpp:1698-1733) on rows (b, i) of h (b, n_nodes, hidden):
//   agg = deg_inv[i] * sum_{k in adj(i)} h[b, idx[k]]   (sequential over k from 0)
//   out = h + act(Linear_self(h) + Linear_neigh(agg))
struct GraphLayerArgs {
    const float* h;
    float* out;
    int64_t rows;
    int n_nodes, hidden, act;
    const int* adj_off;
    const int* adj_idx;
    const float* deg_inv;
    const float* ws;
    const float* bs;
    const float* wn;
    const float* bn;
};

int mlp_max_dim(const MlpArgs& a);
cudaError_t mlp_rows(const MlpArgs& a, cudaStream_t st);
cudaError_t sensor_mean(const MeanArgs& a, cudaStream_t st);
cudaError_t graph_layer(const GraphLayerArgs& a, cudaStream_t st);

}  // namespace nfx
