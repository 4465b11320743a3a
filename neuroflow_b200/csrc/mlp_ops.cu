// mlp_ops.cu -- row-MLP, sensor-mean and graph-block kernels for DeepONet and
// GraphOp / GraphOp2D (declarations and layout in mlp_ops.h).
#include "mlp_ops.h"

#include <algorithm>

#include "nfx_internal.h"
#include "numerics.cuh"

namespace nfx {
namespace {

__device__ __forceinline__ float act_f(float z, int act) { return act == 1 ? relu_ref(z) : gelu_tanh(z); }

// The reference Linear output j of one row: acc = b; acc += x[p] * w[p] in order, the
// first nu products rounded before the add, the rest fused (linear_step).
__device__ __forceinline__ float row_dot(const float* __restrict__ x, const float* __restrict__ w, int k,
                                         int nu, float acc) {
    int p = 0;
    for (; p < nu; ++p) acc = __fadd_rn(acc, __fmul_rn(x[p], __ldg(w + p)));
    for (; p < k; ++p) acc = __fmaf_rn(x[p], __ldg(w + p), acc);
    return acc;
}

// Smallest odd row stride above `dim` (odd strides keep the lanes' rows in distinct
// shared-memory banks).
int odd_stride(int dim) { return (dim + 1) | 1; }

// Rows per CTA for two [rows][stride] float buffers in at most 200 KB.
int rows_per_cta(int stride) {
    for (int t = 128; t >= 32; t >>= 1)
        if (2 * static_cast<size_t>(t) * stride * sizeof(float) <= 200 * 1024) return t;
    return 0;
}

__global__ void __launch_bounds__(128) mlp_rows_kernel(MlpArgs a, int stride) {
    extern __shared__ float sm[];
    const int T = blockDim.x, tid = threadIdx.x;
    float* cur = sm;
    float* nxt = sm + static_cast<size_t>(T) * stride;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * T;
    const int nr = static_cast<int>(a.rows - r0 < T ? a.rows - r0 : T);
    const int in0 = a.layer[0].in;
    for (int t = tid; t < nr * in0; t += T) {
        const int r = t / in0, c = t - r * in0;
        cur[r * stride + c] = a.x[r0 * in0 + t];
    }
    __syncthreads();
    const bool live = tid < nr;
    int width = in0;
    for (int l = 0; l < a.n_layers; ++l) {
        const MlpLayer L = a.layer[l];
        if (live) {
            const int nu = linear_unfused_len(L.in);
            const float* mine = cur + tid * stride;
            float* dst = nxt + tid * stride;
            const bool last = l == a.n_layers - 1;
            for (int j = 0; j < L.out; ++j) {
                float acc = row_dot(mine, L.w + static_cast<int64_t>(j) * L.in, L.in, nu, __ldg(L.b + j));
                dst[j] = last ? acc : act_f(acc, a.act);
            }
        }
        float* t = cur;
        cur = nxt;
        nxt = t;
        width = L.out;
    }
    if (a.dot_branch) {
        if (live) {
            const int lat = width;
            const int nu = linear_unfused_len(lat);
            const float* t = cur + tid * stride;
            float* dst = nxt + tid * stride;
            const int64_t g = (r0 + tid) / a.rows_per_group;
            for (int c = 0; c < a.dot_ch; ++c) {
                const float* br = a.dot_branch + (g * a.dot_ch + c) * lat;
                float acc = 0.0f;
                int k = 0;
                for (; k < nu; ++k) acc = __fadd_rn(acc, __fmul_rn(__ldg(br + k), t[k]));
                for (; k < lat; ++k) acc = __fmaf_rn(__ldg(br + k), t[k], acc);
                dst[c] = __fadd_rn(acc, __ldg(a.dot_bias + c));
            }
        }
        cur = nxt;
        width = a.dot_ch;
    }
    __syncthreads();
    for (int t = tid; t < nr * width; t += T) {
        const int r = t / width, c = t - r * width;
        a.y[r0 * width + t] = cur[r * stride + c];
    }
}

__global__ void __launch_bounds__(256) sensor_mean_kernel(MeanArgs a) {
    const int64_t total = a.groups * a.F;
    const float nf = static_cast<float>(a.n);
    for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t g = idx / a.F;
        const int f = static_cast<int>(idx - g * a.F);
        const float* p = a.in + g * a.n * a.F + f;
        float acc = 0.0f;
        for (int s = 0; s < a.n; ++s) acc = __fadd_rn(acc, __ldg(p + static_cast<int64_t>(s) * a.F));
        a.out[idx] = __fdiv_rn(acc, nf);
    }
}

__global__ void __launch_bounds__(128) graph_layer_kernel(GraphLayerArgs a, int stride) {
    extern __shared__ float sm[];
    const int T = blockDim.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, nwarps = T >> 5;
    float* hrow = sm;
    float* agg = sm + static_cast<size_t>(T) * stride;
    const int64_t r0 = static_cast<int64_t>(blockIdx.x) * T;
    const int nr = static_cast<int>(a.rows - r0 < T ? a.rows - r0 : T);
    const int hd = a.hidden, n = a.n_nodes;
    // neighbour sums, one warp per row, lanes over the features (coalesced rows)
    for (int r = warp; r < nr; r += nwarps) {
        const int64_t row = r0 + r;
        const int64_t b = row / n;
        const int i = static_cast<int>(row - b * n);
        const int lo = __ldg(a.adj_off + i), hi = __ldg(a.adj_off + i + 1);
        const float di = __ldg(a.deg_inv + i);
        const float* hb = a.h + b * n * hd;
        for (int d = lane; d < hd; d += 32) {
            float acc = 0.0f;
            for (int k = lo; k < hi; ++k)
                acc = __fadd_rn(acc, hb[static_cast<int64_t>(__ldg(a.adj_idx + k)) * hd + d]);
            agg[r * stride + d] = __fmul_rn(acc, di);
            hrow[r * stride + d] = hb[static_cast<int64_t>(i) * hd + d];
        }
    }
    __syncthreads();
    if (tid >= nr) return;
    const float* hr = hrow + tid * stride;
    const float* ar = agg + tid * stride;
    float* out = a.out + (r0 + tid) * hd;
    const int nu = linear_unfused_len(hd);
    for (int j = 0; j < hd; ++j) {
        const float s = row_dot(hr, a.ws + static_cast<int64_t>(j) * hd, hd, nu, __ldg(a.bs + j));
        const float q = row_dot(ar, a.wn + static_cast<int64_t>(j) * hd, hd, nu, __ldg(a.bn + j));
        out[j] = __fadd_rn(hr[j], act_f(__fadd_rn(s, q), a.act));
    }
}

}  // namespace

int mlp_max_dim(const MlpArgs& a) {
    int m = a.n_layers > 0 ? a.layer[0].in : 0;
    for (int l = 0; l < a.n_layers; ++l) m = std::max(m, a.layer[l].out);
    if (a.dot_branch) m = std::max(m, a.dot_ch);
    return m;
}

cudaError_t mlp_rows(const MlpArgs& a, cudaStream_t st) {
    if (a.rows == 0) return cudaSuccess;
    const int dim = mlp_max_dim(a);
    if (a.n_layers < 1 || a.n_layers > kMlpMaxLayers || dim > kMlpMaxDim) return cudaErrorInvalidValue;
    const int stride = odd_stride(dim);
    const int T = rows_per_cta(stride);
    const size_t smem = 2 * static_cast<size_t>(T) * stride * sizeof(float);
    cudaError_t e = set_max_dynamic_smem(reinterpret_cast<const void*>(mlp_rows_kernel), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int64_t grid = (a.rows + T - 1) / T;
    mlp_rows_kernel<<<static_cast<unsigned>(grid), T, smem, st>>>(a, stride);
    return cudaGetLastError();
}

cudaError_t sensor_mean(const MeanArgs& a, cudaStream_t st) {
    const int64_t total = a.groups * a.F;
    if (total == 0) return cudaSuccess;
    const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, device_sm_count() * 8));
    sensor_mean_kernel<<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t graph_layer(const GraphLayerArgs& a, cudaStream_t st) {
    if (a.rows == 0) return cudaSuccess;
    if (a.hidden < 1 || a.hidden > kGraphMaxHidden) return cudaErrorInvalidValue;
    const int stride = odd_stride(a.hidden);
    const int T = rows_per_cta(stride);
    const size_t smem = 2 * static_cast<size_t>(T) * stride * sizeof(float);
    cudaError_t e =
        set_max_dynamic_smem(reinterpret_cast<const void*>(graph_layer_kernel), static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const int64_t grid = (a.rows + T - 1) / T;
    graph_layer_kernel<<<static_cast<unsigned>(grid), T, smem, st>>>(a, stride);
    return cudaGetLastError();
}

}  // namespace nfx
