// Launch interface of the sm_100a kernels (kernels.cu).  Host orchestration in
// engine.cu calls these; every launcher enqueues on `stream` and returns the
// launch status without synchronising.
#pragma once
#include <cuda_runtime.h>

#include "common.h"

namespace spm {

struct MoePlan;

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
    // Fused RMSNorm of x when gain != nullptr: x_hat = (x * s_p) * gain, with
    // s_p = 1/sqrt(sum_k sumsq[k*8+p] / cols + eps) over the producer's parts.
    const float* gain;
    const float* sumsq;
    int32_t sumsq_parts;
    float eps;
    float* sumsq_out;     // EPI_ADD: per-CTA sum of squares of the rows written, [grid][8]
    int32_t* status;      // device error word: a bounded wait that gave up sets it
    int32_t slots;        // shared-memory ring slots, a multiple of the groups (set by gemv_geometry)
    int32_t group_warps;  // warps that share a tile (set by gemv_geometry)
    uint32_t xrec;        // bytes of one client's staged 32-value unit (set by launch_gemv)
    int32_t tc;           // tensor-core inner loop (integer codes, four or more clients; set by launch_gemv)
    int32_t tc2;          // K-quant tensor-core loop, codes as A, sixteen rows a slot (set by launch_gemv)
    int32_t c0;           // index of client 0 of this launch in the sum-of-squares arrays
    // Expert mode (plan != nullptr): one job over a [experts][rows][cols]
    // tensor; the grid is one wave of resident CTAs (at least expert_max),
    // and with nl active experts in the plan each expert's tiles split into
    // C = max(expert_chunks, grid / nl) chunks: CTA b streams chunk b % C of
    // active expert b / C; client slot p of the expert reads x row
    // plan->tok[a][p] (xmode 0) or a*8+p (xmode 1) and writes y row a*8+p.
    const MoePlan* plan;
    int32_t expert_max;     // active experts of this rank, at most
    int32_t expert_chunks;  // chunks per expert, at least (sizes the ring)
    uint32_t expert_tiles;
    int32_t xmode;
    // Expert parallel (world > 1, expert mode): experts e with e % world ==
    // rank are this GPU's; CTAs of other experts do no work.  When ep_peer_y
    // is set, each output row goes to the same place in every rank's buffer
    // (ep_peer_y[parity * world + p]) and the launch's last CTA, once every
    // CTA's stores are fenced, writes the flag value E = *ep_step * ep_layers +
    // ep_layer + 1 to ep_peer_flag[parity * world + p] for every rank p
    // (parity = E & 1; ep_done counts finished CTAs and returns to zero).
    int32_t world, rank;
    float* const* ep_peer_y;
    uint32_t* const* ep_peer_flag;
    uint32_t* ep_done;
    const uint32_t* ep_step;
    int32_t ep_layers, ep_layer;
    // Data-parallel attention (world > 1, dense launches of one job): with
    // ep_dense set, ep_peer_y holds every rank's output base (no parity; the
    // launch's rows go from client c0 on, job[0].y_stride apart) and each
    // output row goes to all of them; ep_peer_sumsq, when set, holds every rank's
    // sum-of-squares array and the per-CTA sums go to all of them too.  With
    // ep_wait_flags set the launch first waits (bounded by wait_ns, status 8)
    // until ep_wait_flags[(E & 1) * 64 + p] == E for every rank p, E as above.
    int32_t ep_dense;
    float* const* ep_peer_sumsq;
    const uint32_t* ep_wait_flags;
    uint64_t wait_ns;
};

// Grid, ring slots and dynamic shared memory of a streaming GEMV launch.
struct GemvGeometry {
    int grid, slots, warps, group_warps;
    size_t smem;
};
// `per`: tiles per CTA when the caller fixes the grid (expert mode), else 0.
GemvGeometry gemv_geometry(const GemvLaunch& L, bool dual, int sms, int per = 0);
// `pdl`: launch with programmatic stream serialization (prefetch of the
// weights overlaps the previous kernel; activations are read after it ends).
// `grid_out` receives the grid size (= sum-of-squares parts written by EPI_ADD).
cudaError_t launch_gemv(uint32_t dtype, GemvLaunch L, int sms, cudaStream_t stream, bool pdl, int* grid_out = nullptr);

// Many-position product on the tensor cores (prefill_gemm.cu):
// y[t * y_stride + f] (+= aux for EPI_ADD) = sum_k W[f][k] * x_t[k] for every
// row f of one packed matrix and t < tokens, where x_t is row x_index[t] (or
// t) of x; with x2 set the input is silu(x) * x2 (a SwiGLU pair) instead.
// cols must be a multiple of 64, x 16-byte aligned with x_stride % 4 == 0.
struct GemmArgs {
    const uint8_t* w;      // tile 0 of the packed matrix
    Packed pk;
    const float* x;
    const float* x2;
    const int32_t* x_index;
    int32_t x_stride, tokens;
    float* y;
    int32_t y_stride;
    const float* aux;      // residual for EPI_ADD (may alias y)
    int32_t aux_stride, epi;
    int32_t* status;       // device error word (code 7: a bounded wait gave up)
    // Grouped mode (groups != nullptr; routed experts): CTA row y takes group
    // groups[y] = {expert e, first place, count <= 128, 0}: the matrix is the
    // pk.rows rows starting e * w_stride bytes after w, its positions are
    // places first..first+count-1 (x row x_index[place], or place itself
    // without x_index) and its outputs go to y rows of those places.
    const int4* groups;
    int32_t ngroups;
    uint64_t w_stride;
};
cudaError_t launch_prefill_gemm(const GemmArgs& a, cudaStream_t stream);

// Positions per attention CTA, at most and at least; a (kv head, client) is
// split over ceil(context / chunk) CTAs whose softmax partials are combined,
// with the chunk halved from the maximum while the grid has fewer CTAs than
// the device has SMs.
constexpr int kAttnChunk = 256;
constexpr int kAttnMinChunk = 64;

struct AttnParams {
    const float *q, *k, *v;        // [n][q_width], [n][kv_width]
    float* out;                    // [n][q_width]
    float *kcache, *vcache;        // [client][layer][context][kv_width]
    // The same rows split exactly into three bf16 parts (hi, mid, lo; section
    // "attention on tensor cores" of kernels.cu), [client][layer][context]
    // [kv_heads][3][head_dim], or nullptr: written at every append when set,
    // read by the tensor-core kernel.
    uint16_t *kplanes, *vplanes;
    const int32_t* pos;            // [n] position of the token being decoded
    const float2* rope;            // [context][head_dim/2] (cos, sin)
    const float *q_norm, *k_norm;  // QK-norm gains or nullptr
    float* scratch;                // [n][kv_heads][chunks][group][head_dim + 2] partials
    int32_t* counters;             // [n][kv_heads], zero between launches
    int32_t layer, layers, context, heads, kv_heads, head_dim, family;
    float eps;
    int32_t chunk;                 // positions per CTA (set by launch_attention)
    int32_t* status;               // device error word: a bounded wait that gave up sets it (code 6)
    // Query mode (qpos != nullptr; prefill): row i of q is a query already
    // QK-normed and rotated, at position qpos[i], over the cache of client
    // cache_client, whose rows up to that position are already written; no
    // append.  Launched without programmatic dependent launch.  In decode
    // mode row i is client cache_client + i's (the cache's client index).
    const int32_t* qpos;
    int32_t cache_client;
    // Set by launch_attention: the chunks of a (kv head, client) form one
    // thread-block cluster and combine their partials through distributed
    // shared memory instead of the scratch and the last-CTA counter.
    int32_t cluster;
};
size_t attention_smem(const AttnParams& P);
cudaError_t launch_attention(const AttnParams& P, int n, cudaStream_t stream, bool pdl);
// Query mode over n query rows, one CTA per (kv head, query) covering the
// whole prefix (no split, no partials).
cudaError_t launch_attention_queries(const AttnParams& P, int n, cudaStream_t stream);

// Gather-and-decode one packed row per client (embedding lookup).
// Also writes sumsq_out[i*8 + c] = (i == c) ? sum of squares of row i : 0.
// Client c0 + i's row goes to out row i; sumsq_out[i*8 + c] = (c == c0 + i) ? ss : 0.
cudaError_t launch_embed(uint32_t dtype, const uint8_t* tiles, const Packed& p, const uint32_t* tokens, int n,
                         float* out, float* sumsq_out, cudaStream_t stream, bool pdl, int c0 = 0);
// Decode rows [row0, row0+rows) into out (rows x cols floats), exact.
cudaError_t launch_dequant(uint32_t dtype, const uint8_t* tiles, const Packed& p, uint64_t row0, uint64_t rows,
                           float* out, cudaStream_t stream);
// Greedy pick per client over logits [n][vocab]: largest value, last index on ties.
cudaError_t launch_argmax(const float* logits, int n, int vocab, uint32_t* out, cudaStream_t stream, bool pdl);
// positions += 1 for clients 0..n-1; the step counter (if any) += 1.
cudaError_t launch_advance(int32_t* pos, int n, uint32_t* step, cudaStream_t stream, bool pdl);

}  // namespace spm
