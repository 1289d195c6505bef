// sm_100a kernels of the decode token loop besides the GEMV (gemv.cu):
// exact dequantization (parity hook and embedding lookup), attention over the
// device KV cache, greedy selection, position bookkeeping.
#include "device.cuh"

namespace spm {
namespace {
using namespace dev;

// ---------------------------------------------------------------- decode ----
// Exact dequantization of unit u of a packed row, in the reference's
// arithmetic order (spm-gguf/src/tensor.rs:103-210; ggml Q2_K):
// Q8_0 d*q;  Q6_K (d*sc)*(q-32);  Q5_K (d*sc)*q - dmin*m;  Q2_K (d*sc)*q - dmin*m.
__device__ void dequant_unit(uint32_t dtype, const uint8_t* tile, const Packed& p, uint32_t rt, uint32_t u,
                             float* out) {
    const uint32_t U = uint32_t(p.cols >> 5), B = uint32_t(p.cols >> 8);
    const size_t unit = size_t(rt) * U + u;
    switch (dtype) {
        case SPM_F32: {
            const float* w = reinterpret_cast<const float*>(tile) + size_t(rt) * p.cols + 32 * size_t(u);
            for (int i = 0; i < 32; i++) out[i] = w[i];
            break;
        }
        case SPM_Q8_0: {
            const float d = h2f(tile[p.plane[1] + unit * 2] | (tile[p.plane[1] + unit * 2 + 1] << 8));
            for (int i = 0; i < 32; i++) out[i] = __fmul_rn(d, float(int8_t(tile[unit * 32 + i])));
            break;
        }
        case SPM_Q6_K: {
            const uint8_t* ql = tile + unit * 16;
            const uint8_t* qh = tile + p.plane[1] + unit * 8;
            const uint8_t* sc = tile + p.plane[2] + unit * 2;
            const size_t bo = p.plane[3] + (size_t(rt) * B + (u >> 3)) * 2;
            const float d = h2f(tile[bo] | (tile[bo + 1] << 8));
            for (int l = 0; l < 32; l++) {
                const int i = l & 15, half = l >> 4, t = i >> 2, b = i & 3;
                const uint32_t lo = half ? (ql[i] >> 4) : (ql[i] & 15);
                const uint32_t hi = (qh[4 * half + b] >> (2 * t)) & 3;
                const float q = float(lo | (hi << 4));
                out[l] = __fmul_rn(__fmul_rn(d, float(int8_t(sc[half]))), __fsub_rn(q, 32.0f));
            }
            break;
        }
        case SPM_Q5_K: {
            const uint8_t* m = tile + (size_t(rt) * B + (u >> 3)) * 16;
            const uint8_t* qs = tile + p.plane[1] + unit * 16;
            const uint8_t* qhp = tile + p.plane[2] + unit * 4;
            const uint32_t qh = qhp[0] | (qhp[1] << 8) | (qhp[2] << 16) | (uint32_t(qhp[3]) << 24);
            const float d = h2f(m[0] | (m[1] << 8)), dmin = h2f(m[2] | (m[3] << 8));
            const uint8_t* s = m + 4;
            const int j = int(u & 7);
            int sc, mn;
            if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
            else { sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
            for (int l = 0; l < 32; l++) {
                const int i = l & 15;
                const uint32_t lo = (l >> 4) ? (qs[i] >> 4) : (qs[i] & 15);
                const float q = float(lo | (((qh >> l) & 1) << 4));
                out[l] = __fsub_rn(__fmul_rn(__fmul_rn(d, float(sc)), q), __fmul_rn(dmin, float(mn)));
            }
            break;
        }
        case SPM_Q2_K: {
            const uint8_t* qs = tile + unit * 8;
            const uint8_t* sc = tile + p.plane[1] + unit * 2;
            const size_t bo = p.plane[2] + (size_t(rt) * B + (u >> 3)) * 4;
            const float d = h2f(tile[bo] | (tile[bo + 1] << 8)), dmin = h2f(tile[bo + 2] | (tile[bo + 3] << 8));
            for (int l = 0; l < 32; l++) {
                const int h = l >> 4, i = l & 15, t = i >> 2, b = i & 3;
                const float q = float((qs[4 * h + b] >> (2 * t)) & 3);
                const float dl = __fmul_rn(d, float(sc[h] & 15)), ml = __fmul_rn(dmin, float(sc[h] >> 4));
                out[l] = __fsub_rn(__fmul_rn(dl, q), ml);
            }
            break;
        }
    }
}


__global__ void dequant_kernel(uint32_t dtype, const uint8_t* tiles, const Packed p, uint64_t row0, uint64_t rows,
                               float* out) {
    const uint32_t U = uint32_t(p.cols >> 5);
    const uint64_t total = rows * U;
    for (uint64_t i = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; i < total; i += uint64_t(gridDim.x) * blockDim.x) {
        const uint64_t r = row0 + i / U;
        const uint32_t u = uint32_t(i % U);
        dequant_unit(dtype, tiles + (r / kTileRows) * p.tile_bytes, p, uint32_t(r % kTileRows), u,
                     out + (i / U) * p.cols + 32 * size_t(u));
    }
}

// ------------------------------------------------------------ reductions ----
template <int NT>
__device__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) red[w] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[32] = t;
    }
    __syncthreads();
    const float t = red[32];
    __syncthreads();
    return t;
}

template <int NT>
__device__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) red[w] = v;
    __syncthreads();
    if (threadIdx.x < 32) {
        float t = threadIdx.x < NT / 32 ? red[threadIdx.x] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
        if (threadIdx.x == 0) red[32] = t;
    }
    __syncthreads();
    const float t = red[32];
    __syncthreads();
    return t;
}

// Embedding gather (spm-batch/src/step.rs:27-30): decode the token's row,
// exactly; also the row's sum of squares for the first layer's fused norm.
__global__ void __launch_bounds__(128) embed_kernel(uint32_t dtype, const uint8_t* tiles, const Packed p,
                                                    const uint32_t* tokens, float* out, float* sumsq) {
    __shared__ float red[33];
    pdl_wait();
    const uint32_t U = uint32_t(p.cols >> 5);
    const uint64_t r = tokens[blockIdx.x];
    float* o = out + size_t(blockIdx.x) * p.cols;
    float ss = 0.f;
    for (uint32_t u = threadIdx.x; u < U; u += blockDim.x) {
        float w[32];
        dequant_unit(dtype, tiles + (r / kTileRows) * p.tile_bytes, p, uint32_t(r % kTileRows), u, w);
#pragma unroll
        for (int l = 0; l < 32; l++) {
            o[32 * size_t(u) + l] = w[l];
            ss = fmaf(w[l], w[l], ss);
        }
    }
    ss = block_sum<128>(ss, red);
    pdl_trigger();
    if (threadIdx.x < 8) sumsq[blockIdx.x * 8 + threadIdx.x] = threadIdx.x == blockIdx.x ? ss : 0.f;
}

// Greedy selection: largest logit, LAST index among equals
// (spm-batch/examples/serve-demo.rs:74-79, max_by keeps the last maximum).
__global__ void __launch_bounds__(1024) argmax_kernel(const float* logits, int vocab, uint32_t* out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    pdl_wait();
    const float* row = logits + size_t(blockIdx.x) * vocab;
    float bv = -INFINITY;
    int bi = -1;
    for (int i = threadIdx.x; i < vocab; i += 1024) {
        const float v = row[i];
        if (bi < 0 || v >= bv) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi > bi))) { bv = ov; bi = oi; }
    }
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) { sv[w] = bv; si[w] = bi; }
    __syncthreads();
    pdl_trigger();
    if (w == 0) {
        bv = sv[lane];
        bi = si[lane];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi > bi))) { bv = ov; bi = oi; }
        }
        if (lane == 0) out[blockIdx.x] = uint32_t(bi < 0 ? 0 : bi);
    }
}

__global__ void advance_kernel(int32_t* pos, int n, uint32_t* step) {
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x < n) pos[threadIdx.x] += 1;
    if (step && threadIdx.x == 0) *step += 1;
}

// ------------------------------------------------------------- attention ----
// Grid (kv head, client, position chunk of P.chunk).  Every CTA applies the
// QK-norm and RoPE (host-computed cos/sin table) to its group's queries and
// the new key; the CTA whose chunk holds the new position appends k, v to the
// cache (spm-kv/src/cache.rs:49-58).  Each CTA scores its positions for all
// query heads of the group (keys staged in shared memory, shared by the
// group), forms its chunk's softmax partials (max, sum, unnormalised value
// sum), and the last CTA of a (kv head, client) to finish combines the chunks
// in chunk order.  The scores, the mask (diagonal included) and the GQA head
// mapping are the reference's:
//   LLAMA  : spm-kv/src/attend.rs:37-94   (dot * (1/sqrt hd))
//   others : spm-qwen3-slice/src/attention.rs:36-79 (dot / sqrt hd), with
//            per-head (Qwen3) or full-width (OLMoE) QK RMSNorm.
constexpr int kAttnThreads = 256;
constexpr int kSub = 64;  // positions staged per pass

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

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams P) {
    extern __shared__ __align__(16) float sm[];
    const int kvh = blockIdx.x, i = blockIdx.y, chunk = blockIdx.z, S = gridDim.z;
    const int hd = P.head_dim, group = P.heads / P.kv_heads;
    const int qw = P.heads * hd, kvw = P.kv_heads * hd, ld = hd + 4;
    const bool llama = P.family == SPM_FAMILY_LLAMA;
    float* qs = sm;                         // group * hd
    float* kn = qs + group * hd;            // hd (new key)
    float* vn = kn + hd;                    // hd (new value)
    float* kv = vn + hd;                    // kSub * ld (staged keys; values of later passes)
    float* vb = kv + kSub * ld;             // kSub * ld (values of the first pass)
    float* sc = vb + kSub * ld;             // group * kChunk scores
    float* red = sc + group * kAttnChunk;   // 64
    // The position and the cached rows before it come from earlier steps, so
    // the first pass's keys and values are fetched before waiting for the
    // kernel that produces this step's q, k, v.
    const int pos = P.pos[i];
    const int p0 = chunk * P.chunk;
    const int p1 = min(pos + 1, p0 + P.chunk);
    const size_t base = (size_t(i) * P.layers + P.layer) * P.context * size_t(kvw) + size_t(kvh) * hd;
    float* kc = P.kcache + base;
    float* vc = P.vcache + base;
    {
        const int pre = max(0, min(min(pos, p1), p0 + kSub) - p0);  // cached rows of the first pass
        for (int t = threadIdx.x; t < pre * (hd / 4); t += kAttnThreads) {
            const int p = t / (hd / 4), c4 = t % (hd / 4);
            *reinterpret_cast<float4*>(kv + p * ld + 4 * c4) = *reinterpret_cast<const float4*>(kc + size_t(p0 + p) * kvw + 4 * c4);
            *reinterpret_cast<float4*>(vb + p * ld + 4 * c4) = *reinterpret_cast<const float4*>(vc + size_t(p0 + p) * kvw + 4 * c4);
        }
    }
    pdl_wait();
    const float* qg = P.q + size_t(i) * qw + size_t(kvh) * group * hd;
    for (int t = threadIdx.x; t < group * hd; t += kAttnThreads) qs[t] = qg[t];
    for (int t = threadIdx.x; t < hd; t += kAttnThreads) {
        kn[t] = P.k[size_t(i) * kvw + size_t(kvh) * hd + t];
        vn[t] = P.v[size_t(i) * kvw + size_t(kvh) * hd + t];
    }
    __syncthreads();
    if (P.family == SPM_FAMILY_OLMOE) {
        float sq = 0.f, sk = 0.f;
        for (int t = threadIdx.x; t < qw; t += kAttnThreads) sq = fmaf(P.q[size_t(i) * qw + t], P.q[size_t(i) * qw + t], sq);
        for (int t = threadIdx.x; t < kvw; t += kAttnThreads) sk = fmaf(P.k[size_t(i) * kvw + t], P.k[size_t(i) * kvw + t], sk);
        sq = block_sum<kAttnThreads>(sq, red);
        sk = block_sum<kAttnThreads>(sk, red);
        const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, float(qw)), P.eps)));
        const float sck = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sk, float(kvw)), P.eps)));
        for (int t = threadIdx.x; t < group * hd; t += kAttnThreads)
            qs[t] = __fmul_rn(__fmul_rn(qs[t], scq), P.q_norm[kvh * group * hd + t]);
        for (int t = threadIdx.x; t < hd; t += kAttnThreads) kn[t] = __fmul_rn(__fmul_rn(kn[t], sck), P.k_norm[kvh * hd + t]);
        __syncthreads();
    } else if (!llama) {
        // per-head RMSNorm, one warp per head (spm-qwen3-slice/src/attention.rs:27-34)
        const int lane = threadIdx.x & 31;
        for (int h = threadIdx.x >> 5; h <= group; h += kAttnThreads / 32) {
            float* x = h < group ? qs + h * hd : kn;
            const float* g = h < group ? P.q_norm : P.k_norm;
            float ss = 0.f;
            for (int t = lane; t < hd; t += 32) ss = fmaf(x[t], x[t], ss);
            ss = warp_sum(ss);
            const float s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(hd)), P.eps)));
            __syncwarp();
            for (int t = lane; t < hd; t += 32) x[t] = __fmul_rn(__fmul_rn(x[t], s), g[t]);
        }
        __syncthreads();
    }
    const int half = hd / 2;
    const float2* rt = P.rope + size_t(pos) * half;
    for (int t = threadIdx.x; t < (group + 1) * half; t += kAttnThreads) {
        const int h = t / half, j = t % half;
        float* x = h < group ? qs + h * hd : kn;
        const float2 cs = rt[j];
        rope_pair(x[j], x[j + half], cs.x, cs.y, llama);
    }
    __syncthreads();
    if (pos >= p0 && pos < p0 + P.chunk)
        for (int t = threadIdx.x; t < hd; t += kAttnThreads) {
            kc[size_t(pos) * kvw + t] = kn[t];
            vc[size_t(pos) * kvw + t] = vn[t];
            if (pos < p0 + kSub) {  // the new row of the first pass
                kv[(pos - p0) * ld + t] = kn[t];
                vb[(pos - p0) * ld + t] = vn[t];
            }
        }
    __syncthreads();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(float(hd)));
    const float denom = __fsqrt_rn(float(hd));
    const int npos = max(0, p1 - p0);
    // ---- scores for this chunk, all heads of the group ----
    for (int b0 = 0; b0 < npos; b0 += kSub) {
        const int nb = min(kSub, npos - b0);
        if (b0 > 0) {  // the first pass was staged before the wait
            __syncthreads();
            for (int t = threadIdx.x; t < nb * (hd / 4); t += kAttnThreads) {
                const int p = t / (hd / 4), c4 = t % (hd / 4);
                const float4 v = *reinterpret_cast<const float4*>(kc + size_t(p0 + b0 + p) * kvw + 4 * c4);
                *reinterpret_cast<float4*>(kv + p * ld + 4 * c4) = v;
            }
            __syncthreads();
        }
        for (int t = threadIdx.x; t < nb * group; t += kAttnThreads) {
            const int p = t % nb, h = t / nb;
            const float* q = qs + h * hd;
            const float* k = kv + p * ld;
            float d = 0.f;
            for (int c = 0; c < hd; c += 4) {
                const float4 kk = *reinterpret_cast<const float4*>(k + c);
                d = fmaf(q[c], kk.x, d);
                d = fmaf(q[c + 1], kk.y, d);
                d = fmaf(q[c + 2], kk.z, d);
                d = fmaf(q[c + 3], kk.w, d);
            }
            sc[h * kAttnChunk + b0 + p] = llama ? __fmul_rn(d, scale) : __fdiv_rn(d, denom);
        }
        __syncthreads();
    }
    // ---- chunk softmax partials per head (one warp per head): m, l ----
    float* part = P.scratch + ((size_t(i) * P.kv_heads + kvh) * S + chunk) * group * (hd + 2);
    float* ml = red;  // [group][2]: max, sum of exp
    {
        const int lane = threadIdx.x & 31;
        for (int h = threadIdx.x >> 5; h < group; h += kAttnThreads / 32) {
            float mx = -INFINITY;
            for (int p = lane; p < npos; p += 32) mx = fmaxf(mx, sc[h * kAttnChunk + p]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            float tot = 0.f;
            for (int p = lane; p < npos; p += 32) {
                const float e = expf(sc[h * kAttnChunk + p] - mx);
                sc[h * kAttnChunk + p] = e;
                tot += e;
            }
            tot = warp_sum(tot);
            if (lane == 0) {
                ml[2 * h] = mx;
                ml[2 * h + 1] = tot;
            }
        }
    }
    __syncthreads();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // (head, dim) pairs t, t+256, ... (group*hd <= 1024)
    for (int b0 = 0; b0 < npos; b0 += kSub) {
        const int nb = min(kSub, npos - b0);
        const float* vv = b0 == 0 ? vb : kv;
        if (b0 > 0) {
            for (int t = threadIdx.x; t < nb * (hd / 4); t += kAttnThreads) {
                const int p = t / (hd / 4), c4 = t % (hd / 4);
                *reinterpret_cast<float4*>(kv + p * ld + 4 * c4) =
                    *reinterpret_cast<const float4*>(vc + size_t(p0 + b0 + p) * kvw + 4 * c4);
            }
            __syncthreads();
        }
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int t = threadIdx.x + r * kAttnThreads;
            if (t < group * hd) {
                const int h = t / hd, dd = t % hd;
                float a = acc[r];
                for (int p = 0; p < nb; p++) a = fmaf(sc[h * kAttnChunk + b0 + p], vv[p * ld + dd], a);
                acc[r] = a;
            }
        }
        __syncthreads();
    }
    if (S == 1) {
        // the whole prefix is in this CTA: finish here (no partials)
#pragma unroll
        for (int r = 0; r < 4; r++) {
            const int t = threadIdx.x + r * kAttnThreads;
            if (t < group * hd) {
                const int h = t / hd, dd = t % hd;
                P.out[size_t(i) * qw + (size_t(kvh) * group + h) * hd + dd] = __fdiv_rn(acc[r], ml[2 * h + 1]);
            }
        }
        pdl_trigger();
        return;
    }
#pragma unroll
    for (int r = 0; r < 4; r++) {
        const int t = threadIdx.x + r * kAttnThreads;
        if (t < group * hd) part[(t / hd) * (hd + 2) + (t % hd)] = acc[r];
    }
    if (threadIdx.x < group) {
        part[threadIdx.x * (hd + 2) + hd] = ml[2 * threadIdx.x];
        part[threadIdx.x * (hd + 2) + hd + 1] = ml[2 * threadIdx.x + 1];
    }
    // ---- the last chunk CTA of this (kv head, client) combines ----
    __shared__ int last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        int* ctr = P.counters + i * P.kv_heads + kvh;
        last = atomicAdd(ctr, 1) == S - 1;
        if (last) *ctr = 0;
    }
    __syncthreads();
    pdl_trigger();
    if (!last) return;
    __threadfence();
    const float* parts = P.scratch + (size_t(i) * P.kv_heads + kvh) * S * group * (hd + 2);
    for (int t = threadIdx.x; t < group * hd; t += kAttnThreads) {
        const int h = t / hd, dd = t % hd;
        float M = -INFINITY;
#pragma unroll 4
        for (int s = 0; s < S; s++) M = fmaxf(M, __ldcg(parts + (size_t(s) * group + h) * (hd + 2) + hd));
        // chunks in order; the loads of four chunks are in flight together
        float Lsum = 0.f, O = 0.f;
#pragma unroll 4
        for (int s = 0; s < S; s++) {
            const float* ps = parts + (size_t(s) * group + h) * (hd + 2);
            const float m = __ldcg(ps + hd), l = __ldcg(ps + hd + 1), o = __ldcg(ps + dd);
            const float w = m == -INFINITY ? 0.f : expf(m - M);
            Lsum = fmaf(l, w, Lsum);
            O = fmaf(o, w, O);
        }
        P.out[size_t(i) * qw + (size_t(kvh) * group + h) * hd + dd] = __fdiv_rn(O, Lsum);
    }
}

}  // namespace

size_t attention_smem(const AttnParams& P) {
    const int group = P.heads / P.kv_heads;
    return (size_t(group) * P.head_dim + 2 * P.head_dim + 2 * size_t(kSub) * (P.head_dim + 4) +
            size_t(group) * kAttnChunk + 64) * sizeof(float);
}

static cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                              void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_attention(const AttnParams& P, int n, cudaStream_t s, bool pdl) {
    const size_t smem = attention_smem(P);
    static int configured_for = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && configured_for != dev) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        if (e != cudaSuccess) return e;
        configured_for = dev;
    }
    static int sms[64] = {};
    if (dev < 64 && !sms[dev]) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    const int target = dev < 64 && sms[dev] ? sms[dev] : 148;
    int chunk = kAttnChunk;
    while (chunk > kAttnMinChunk && ((P.context + chunk - 1) / chunk) * P.kv_heads * n < target) chunk /= 2;
    const int chunks = (P.context + chunk - 1) / chunk;
    AttnParams p = P;
    p.chunk = chunk;
    void* args[] = {&p};
    return launch_pdl(reinterpret_cast<const void*>(attention_kernel), dim3(P.kv_heads, n, chunks),
                      dim3(kAttnThreads), smem, s, pdl, args);
}

cudaError_t launch_embed(uint32_t dtype, const uint8_t* tiles, const Packed& p, const uint32_t* tokens, int n,
                         float* out, float* sumsq, cudaStream_t s, bool pdl) {
    Packed pk = p;
    void* args[] = {&dtype, &tiles, &pk, &tokens, &out, &sumsq};
    return launch_pdl(reinterpret_cast<const void*>(embed_kernel), dim3(n), dim3(128), 0, s, pdl, args);
}

cudaError_t launch_dequant(uint32_t dtype, const uint8_t* tiles, const Packed& p, uint64_t row0, uint64_t rows,
                           float* out, cudaStream_t s) {
    const uint64_t units = rows * (p.cols / 32);
    uint64_t grid = (units + 255) / 256;
    if (grid > 65535) grid = 65535;
    if (grid == 0) return cudaSuccess;
    dequant_kernel<<<unsigned(grid), 256, 0, s>>>(dtype, tiles, p, row0, rows, out);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float* logits, int n, int vocab, uint32_t* out, cudaStream_t s, bool pdl) {
    void* args[] = {&logits, &vocab, &out};
    return launch_pdl(reinterpret_cast<const void*>(argmax_kernel), dim3(n), dim3(1024), 0, s, pdl, args);
}

cudaError_t launch_advance(int32_t* pos, int n, uint32_t* step, cudaStream_t s, bool pdl) {
    void* args[] = {&pos, &n, &step};
    return launch_pdl(reinterpret_cast<const void*>(advance_kernel), dim3(1), dim3(32), 0, s, pdl, args);
}

}  // namespace spm
