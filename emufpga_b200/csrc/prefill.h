// Launch interface of the prompt kernels (prefill.cu); the tensor-core
// product and the attention query mode are declared in kernels.h.
#pragma once
#include <cuda_runtime.h>

#include "kernels.h"
#include "moe.h"

namespace spm {

// Decode the embedding rows of tokens[0..T) into out (T x cols), exactly.
cudaError_t launch_embed_rows(uint32_t dtype, const uint8_t* tiles, const Packed& p, const uint32_t* tokens, int T,
                              float* out, cudaStream_t stream);
// RMSNorm of T rows of `width` values: y = (x * s) * gain.
cudaError_t launch_norm_rows(const float* x, const float* gain, float eps, int width, int T, float* y,
                             cudaStream_t stream);

struct QkArgs {
    float* q;                      // [T][heads * head_dim], normed and rotated in place
    const float *k, *v;            // [T][kv_heads * head_dim]
    float *kcache, *vcache;        // [client][layer][context][kv_width]
    uint16_t *kplanes, *vplanes;   // the rows as three bf16 parts (AttnParams), or nullptr
    const float2* rope;            // [context][head_dim / 2]
    const float *q_norm, *k_norm;  // QK-norm gains or nullptr (LLAMA)
    int32_t client, layer, layers, context, pos0;
    int32_t heads, kv_heads, head_dim, family;
    float eps;
};
// Row t at position pos0 + t: QK-norm, RoPE, and the KV cache append.
cudaError_t launch_qk_rope_append(const QkArgs& a, int T, cudaStream_t stream);

// Routing of T rows: sel/prob [T][K] in route order, norm [T] (sum of the
// selected probabilities), counts[e] += routes to expert e.
cudaError_t launch_route_rows(const float* logits, const float* bias, int T, int E, int K, int32_t* sel, float* prob,
                              float* norm, int32_t* counts, cudaStream_t stream);
// Places in the expert groups: list[place] = row, slot[row][j] = place.
cudaError_t launch_scatter_rows(const int32_t* sel, int T, int K, const int32_t* offsets, int32_t* cursor,
                                int32_t* list, int32_t* slot, cudaStream_t stream);
// x[t] += sum over row t's routes (ascending expert id) of (y[slot] * p) / norm.
cudaError_t launch_combine_rows(const int32_t* sel, const float* prob, const float* norm, const int32_t* slot,
                                const float* y, float* x, int T, int K, int width, cudaStream_t stream);

}  // namespace spm
