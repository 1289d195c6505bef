// Launch interface of the sm_100a kernels (kernels.cu).  Host orchestration in
// engine.cu calls these; every launcher enqueues on `stream` and returns the
// launch status without synchronising.
#pragma once
#include <cuda_runtime.h>

#include "common.h"

namespace spm {

enum Epilogue { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

// One matrix (or a gate/up pair) inside a GEMV launch.
struct GemvJob {
    const uint8_t* a;     // tile 0 of the matrix in the device image
    const uint8_t* b;     // tile 0 of the paired matrix (EPI_SWIGLU) or nullptr
    float* y;             // y[p * y_stride + row]
    const float* aux;     // residual for EPI_ADD (may alias y)
    uint32_t tile_begin;  // first global tile index of this job
    uint32_t rows;
    int32_t y_stride, aux_stride, epi;
};

struct GemvLaunch {
    GemvJob job[4];
    int32_t njobs;
    uint32_t total_tiles;
    uint32_t cols, tile_bytes, plane1, plane2, plane3;
    const float* x;       // x[p * x_stride + col]
    int32_t x_stride, n;
};

cudaError_t launch_gemv(uint32_t dtype, const GemvLaunch& L, int sms, cudaStream_t stream);

struct AttnParams {
    const float *q, *k, *v;        // [n][q_width], [n][kv_width]
    float* out;                    // [n][q_width]
    float *kcache, *vcache;        // [client][layer][context][kv_width]
    const int32_t* pos;            // [n] position of the token being decoded
    const float2* rope;            // [context][head_dim/2] (cos, sin)
    const float *q_norm, *k_norm;  // QK-norm gains or nullptr
    int32_t layer, layers, context, heads, kv_heads, head_dim, family;
    float eps;
};
cudaError_t launch_attention(const AttnParams& P, int n, cudaStream_t stream);

cudaError_t launch_rmsnorm(const float* x, const float* gain, float* out, int n, int width, float eps,
                           cudaStream_t stream);
// Gather-and-decode one packed row per client (embedding lookup).
cudaError_t launch_embed(uint32_t dtype, const uint8_t* tiles, const Packed& p, const uint32_t* tokens, int n,
                         float* out, cudaStream_t stream);
// Decode rows [row0, row0+rows) into out (rows x cols floats), exact.
cudaError_t launch_dequant(uint32_t dtype, const uint8_t* tiles, const Packed& p, uint64_t row0, uint64_t rows,
                           float* out, cudaStream_t stream);
// Greedy pick per client over logits [n][vocab]: largest value, last index on ties.
cudaError_t launch_argmax(const float* logits, int n, int vocab, uint32_t* out, cudaStream_t stream);
cudaError_t launch_advance(int32_t* pos, int n, cudaStream_t stream);

}  // namespace spm
