// Prompt (prefill) kernels besides the tensor-core product (prefill_gemm.cu)
// and the attention kernel's query mode (kernels.cu).  A prompt's T positions
// of one client go through a layer together:
//   embedding rows -> per layer [RMSNorm rows] [q, k, v products]
//   [QK-norm, RoPE, KV append] [attention over the cache, one query per row]
//   [o product + residual] [RMSNorm rows] then the feed-forward:
//   dense  : [gate, up products] [down product of silu(gate)*up + residual]
//   routed : [router product] [route rows] [group rows by expert]
//            [gate, up, down products per expert group] [combine rows].
// Each row computes what one decode step computes for that position (same
// equations and operation order per value; products and sums may round
// differently, as they do between the decode GEMV and the reference).
#include <cuda_runtime.h>

#include "dequant.cuh"
#include "prefill.h"

namespace spm {
namespace {
using namespace dev;

__device__ float block_sum256(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) red[w] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[32] = t;
    }
    __syncthreads();
    const float t = red[32];
    __syncthreads();
    return t;
}

// Row t of the embedding for token tokens[t] (exact decode, spm-batch/src/step.rs:27-30).
__global__ void __launch_bounds__(128) embed_rows_kernel(uint32_t dtype, const uint8_t* tiles, const Packed p,
                                                         const uint32_t* tokens, float* out) {
    const uint32_t U = uint32_t(p.cols >> 5);
    const uint64_t r = tokens[blockIdx.x];
    float* o = out + size_t(blockIdx.x) * p.cols;
    for (uint32_t u = threadIdx.x; u < U; u += blockDim.x) {
        float w[32];
        dequant_unit(dtype, tiles + (r / kTileRows) * p.tile_bytes, p, uint32_t(r % kTileRows), u, w);
#pragma unroll
        for (int l = 0; l < 32; l++) o[32 * size_t(u) + l] = w[l];
    }
}

// y = (x * s) * g, s = 1 / sqrt(sum x^2 / n + eps) per row
// (spm-smol-ops/src/norm.rs:12-21, spm-qwen3-slice/src/math.rs:1-10).
__global__ void __launch_bounds__(256) norm_rows_kernel(const float* x, const float* gain, float eps, int width,
                                                        float* y) {
    __shared__ float red[33];
    const float* xr = x + size_t(blockIdx.x) * width;
    float* yr = y + size_t(blockIdx.x) * width;
    float ss = 0.f;
    for (int c = threadIdx.x; c < width; c += blockDim.x) ss = fmaf(xr[c], xr[c], ss);
    ss = block_sum256(ss, red);
    const float count = float(width > 65535 ? 65535 : width);
    const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, count), eps)));
    for (int c = threadIdx.x; c < width; c += blockDim.x) yr[c] = __fmul_rn(__fmul_rn(xr[c], s), gain[c]);
}

__device__ __forceinline__ void rope_pair(float& x, float& y, float c, float s, bool llama) {
    if (llama) {  // spm-ops/src/attention.rs:29-30
        const float nx = __fmaf_rn(x, c, -__fmul_rn(y, s));
        const float ny = __fmaf_rn(x, s, __fmul_rn(y, c));
        x = nx;
        y = ny;
    } else {      // spm-qwen3-slice/src/attention.rs:20-23
        const float nx = __fsub_rn(__fmul_rn(x, c), __fmul_rn(y, s));
        const float ny = __fadd_rn(__fmul_rn(y, c), __fmul_rn(x, s));
        x = nx;
        y = ny;
    }
}

// Row t: QK-norm and RoPE at position pos0 + t of the row's q and k (q in
// place), then k and v into the client's cache at that position -- the
// decode attention kernel's preamble for one position
// (spm-qwen3-slice/src/attention.rs:27-34, spm-kv/src/cache.rs:49-58).
__global__ void __launch_bounds__(256) qk_rope_append_kernel(const QkArgs a) {
    extern __shared__ float qk[];  // q (qw) then k (kvw)
    __shared__ float red[33];
    const int t = blockIdx.x, qw = a.heads * a.head_dim, kvw = a.kv_heads * a.head_dim, hd = a.head_dim;
    const bool llama = a.family == SPM_FAMILY_LLAMA;
    float* q = qk;
    float* k = qk + qw;
    const float* qg = a.q + size_t(t) * qw;
    const float* kg = a.k + size_t(t) * kvw;
    for (int c = threadIdx.x; c < qw; c += blockDim.x) q[c] = qg[c];
    for (int c = threadIdx.x; c < kvw; c += blockDim.x) k[c] = kg[c];
    __syncthreads();
    if (a.family == SPM_FAMILY_OLMOE) {
        float sq = 0.f, sk = 0.f;
        for (int c = threadIdx.x; c < qw; c += blockDim.x) sq = fmaf(q[c], q[c], sq);
        for (int c = threadIdx.x; c < kvw; c += blockDim.x) sk = fmaf(k[c], k[c], sk);
        sq = block_sum256(sq, red);
        sk = block_sum256(sk, red);
        const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, float(qw)), a.eps)));
        const float sck = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sk, float(kvw)), a.eps)));
        for (int c = threadIdx.x; c < qw; c += blockDim.x) q[c] = __fmul_rn(__fmul_rn(q[c], scq), a.q_norm[c]);
        for (int c = threadIdx.x; c < kvw; c += blockDim.x) k[c] = __fmul_rn(__fmul_rn(k[c], sck), a.k_norm[c]);
        __syncthreads();
    } else if (!llama) {
        const int lane = threadIdx.x & 31;
        for (int h = threadIdx.x >> 5; h < a.heads + a.kv_heads; h += blockDim.x / 32) {
            float* x = h < a.heads ? q + h * hd : k + (h - a.heads) * hd;
            const float* g = h < a.heads ? a.q_norm : a.k_norm;
            float ss = 0.f;
            for (int c = lane; c < hd; c += 32) ss = fmaf(x[c], x[c], ss);
            ss = warp_sum(ss);
            const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(hd)), a.eps)));
            __syncwarp();
            for (int c = lane; c < hd; c += 32) x[c] = __fmul_rn(__fmul_rn(x[c], s), g[c]);
        }
        __syncthreads();
    }
    const int pos = a.pos0 + t, half = hd / 2;
    const float2* rt = a.rope + size_t(pos) * half;
    for (int e = threadIdx.x; e < (a.heads + a.kv_heads) * half; e += blockDim.x) {
        const int h = e / half, j = e % half;
        float* x = h < a.heads ? q + h * hd : k + (h - a.heads) * hd;
        const float2 cs = rt[j];
        rope_pair(x[j], x[j + half], cs.x, cs.y, llama);
    }
    __syncthreads();
    float* qo = a.q + size_t(t) * qw;
    for (int c = threadIdx.x; c < qw; c += blockDim.x) qo[c] = q[c];
    const size_t row = ((size_t(a.client) * a.layers + a.layer) * a.context + pos) * kvw;
    for (int c = threadIdx.x; c < kvw; c += blockDim.x) {
        const float vv = a.v[size_t(t) * kvw + c];
        a.kcache[row + c] = k[c];
        a.vcache[row + c] = vv;
        if (a.kplanes) {
            // head h's [3][hd] plane row
            const int h = c / hd, d = c % hd;
            store_planes(a.kplanes + (row + size_t(h) * hd) * 3, hd, d, k[c]);
            store_planes(a.vplanes + (row + size_t(h) * hd) * 3, hd, d, vv);
        }
    }
}

// f32::total_cmp order key (spm-granite-moe/src/math.rs:35-39 sorts by it).
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    return b ^ int32_t(uint32_t(b >> 31) >> 1);
}

// One warp per row: softmax over (logits + bias), top-K (largest first, the
// lower id among equals), the sum of the selected probabilities in route
// order -- the decode route kernel's arithmetic (spm-granite-moe/src/
// moe.rs:17-35, math.rs:23-39) -- and a count per selected expert.
__global__ void __launch_bounds__(256) route_rows_kernel(const float* logits, const float* bias, int T, int E, int K,
                                                         int32_t* sel, float* prob, float* norm, int32_t* counts) {
    __shared__ float pr[8][kMoeMaxExperts];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + w;
    if (t >= T) return;
    float* p = pr[w];
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) {
        const float v = bias ? logits[size_t(t) * E + e] + bias[e] : logits[size_t(t) * E + e];
        p[e] = v;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
    for (int e = lane; e < E; e += 32) {
        const float v = expf(p[e] - mx);
        p[e] = v;
        sum += v;
    }
    sum = warp_sum(sum);
    __syncwarp();
    for (int e = lane; e < E; e += 32) p[e] = __fdiv_rn(p[e], sum);
    __syncwarp();
    uint64_t taken[4] = {0, 0, 0, 0};
    float s = 0.f;
    for (int j = 0; j < K; j++) {
        int32_t bk = INT32_MIN;
        int bi = -1;
        for (int e = lane; e < E; e += 32) {
            if (taken[e >> 6] & (1ull << (e & 63))) continue;
            const int32_t k = total_key(p[e]);
            if (bi < 0 || k > bk) { bk = k; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const int32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ok > bk || (ok == bk && oi < bi))) { bk = ok; bi = oi; }
        }
        taken[bi >> 6] |= 1ull << (bi & 63);
        s += p[bi];  // in route order (layout.rs:289-293)
        if (lane == 0) {
            sel[size_t(t) * K + j] = bi;
            prob[size_t(t) * K + j] = p[bi];
            atomicAdd(&counts[bi], 1);
        }
    }
    if (lane == 0) norm[t] = s;
}

// Row t's route j gets a place in its expert's group: list[place] = t and
// slot[t][j] = place, places of expert e starting at offsets[e].
__global__ void scatter_rows_kernel(const int32_t* sel, int T, int K, const int32_t* offsets, int32_t* cursor,
                                    int32_t* list, int32_t* slot) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= T * K) return;
    const int e = sel[i];
    const int place = offsets[e] + atomicAdd(&cursor[e], 1);
    list[place] = i / K;
    slot[i] = place;
}

// x[t] += sum over row t's routes in ascending expert id of (y[slot] * p) / norm
// (spm-granite-moe/src/layout.rs:283-302; the decode combine's order).
__global__ void __launch_bounds__(256) combine_rows_kernel(const int32_t* sel, const float* prob, const float* norm,
                                                           const int32_t* slot, const float* y, float* x, int K,
                                                           int width) {
    const int t = blockIdx.y, col = blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= width) return;
    int ids[kMoeMaxUsed], js[kMoeMaxUsed];
    for (int j = 0; j < K; j++) ids[j] = sel[size_t(t) * K + j], js[j] = j;
    for (int a = 1; a < K; a++)
        for (int b = a; b > 0 && ids[b - 1] > ids[b]; b--) {
            const int ti = ids[b], tj = js[b];
            ids[b] = ids[b - 1], js[b] = js[b - 1];
            ids[b - 1] = ti, js[b - 1] = tj;
        }
    const float nrm = norm[t];
    float total = 0.f;
    for (int j = 0; j < K; j++) {
        const int r = js[j];
        const float v = y[size_t(slot[size_t(t) * K + r]) * width + col];
        total = total + __fdiv_rn(__fmul_rn(v, prob[size_t(t) * K + r]), nrm);
    }
    x[size_t(t) * width + col] = x[size_t(t) * width + col] + total;
}

}  // namespace

cudaError_t launch_embed_rows(uint32_t dtype, const uint8_t* tiles, const Packed& p, const uint32_t* tokens, int T,
                              float* out, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    embed_rows_kernel<<<T, 128, 0, s>>>(dtype, tiles, p, tokens, out);
    return cudaGetLastError();
}

cudaError_t launch_norm_rows(const float* x, const float* gain, float eps, int width, int T, float* y,
                             cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    norm_rows_kernel<<<T, 256, 0, s>>>(x, gain, eps, width, y);
    return cudaGetLastError();
}

cudaError_t launch_qk_rope_append(const QkArgs& a, int T, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    const size_t smem = size_t(a.heads + a.kv_heads) * a.head_dim * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(qk_rope_append_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(smem));
        if (e != cudaSuccess) return e;
    }
    qk_rope_append_kernel<<<T, 256, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_route_rows(const float* logits, const float* bias, int T, int E, int K, int32_t* sel, float* prob,
                              float* norm, int32_t* counts, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    if (E > kMoeMaxExperts || K > kMoeMaxUsed || K > E) return cudaErrorInvalidValue;
    route_rows_kernel<<<(T + 7) / 8, 256, 0, s>>>(logits, bias, T, E, K, sel, prob, norm, counts);
    return cudaGetLastError();
}

cudaError_t launch_scatter_rows(const int32_t* sel, int T, int K, const int32_t* offsets, int32_t* cursor,
                                int32_t* list, int32_t* slot, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    scatter_rows_kernel<<<(T * K + 255) / 256, 256, 0, s>>>(sel, T, K, offsets, cursor, list, slot);
    return cudaGetLastError();
}

cudaError_t launch_combine_rows(const int32_t* sel, const float* prob, const float* norm, const int32_t* slot,
                                const float* y, float* x, int T, int K, int width, cudaStream_t s) {
    if (T <= 0) return cudaSuccess;
    combine_rows_kernel<<<dim3((width + 255) / 256, T), 256, 0, s>>>(sel, prob, norm, slot, y, x, K, width);
    return cudaGetLastError();
}

}  // namespace spm
