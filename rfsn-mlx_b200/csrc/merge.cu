// Log-sum-exp merge of attention results over disjoint key sets.
//
// For parts r = 0..P-1 with normalised outputs O_r and natural-log LSE_r of
// the same query rows, the exact result over the union of their keys is
//   O = sum_r exp(LSE_r - M) O_r / sum_r exp(LSE_r - M),  M = max_r LSE_r,
// the associative form of the global-max merge of attention_exact.py:141-164.
// Used after the cross-GPU gather of sharded decode. Parts are combined in
// rank order, so the result is deterministic.
#include <math_constants.h>

#include "params.cuh"

namespace rfsn {
namespace {

__global__ void lse_merge_kernel(const float* __restrict__ parts_out, const float* __restrict__ parts_lse, int n_parts,
                                 int rows, int head_dim, float* __restrict__ out, float* __restrict__ lse_out) {
    const int row = blockIdx.x;
    float M = -CUDART_INF_F;
    for (int r = 0; r < n_parts; ++r) M = fmaxf(M, parts_lse[(size_t)r * rows + row]);
    float W = 0.f;
    for (int r = 0; r < n_parts; ++r) {
        const float l = parts_lse[(size_t)r * rows + row];
        W += (M == -CUDART_INF_F) ? 0.f : expf(l - M);
    }
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float acc = 0.f;
        if (M != -CUDART_INF_F) {
            for (int r = 0; r < n_parts; ++r) {
                const float w = expf(parts_lse[(size_t)r * rows + row] - M);
                acc += w * parts_out[((size_t)r * rows + row) * head_dim + d];
            }
        }
        out[(size_t)row * head_dim + d] = W > 0.f ? acc / W : 0.f;
    }
    if (lse_out != nullptr && threadIdx.x == 0) lse_out[row] = W > 0.f ? M + logf(W) : -CUDART_INF_F;
}

}  // namespace

void preload_merge_kernels() {
    cudaFuncAttributes a;
    cudaFuncGetAttributes(&a, lse_merge_kernel);
}

rfsn_status lse_merge_launch(const float* parts_out, const float* parts_lse, int n_parts, int rows, int head_dim,
                             float* out, float* lse_out, cudaStream_t stream) {
    const int threads = head_dim >= 128 ? 128 : ((head_dim + 31) / 32) * 32;
    lse_merge_kernel<<<rows, threads, 0, stream>>>(parts_out, parts_lse, n_parts, rows, head_dim, out, lse_out);
    RFSN_CUDA(cudaGetLastError());
    note_launch();
    return RFSN_OK;
}

}  // namespace rfsn
