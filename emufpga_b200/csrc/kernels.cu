// sm_100a kernels of the decode token loop besides the GEMV (gemv.cu):
// exact dequantization (parity hook and embedding lookup), attention over the
// device KV cache, greedy selection, position bookkeeping.
#include <algorithm>

#include <cooperative_groups.h>

#include "dequant.cuh"

namespace spm {
namespace {
using namespace dev;

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
                                                    const uint32_t* tokens, float* out, float* sumsq, int c0) {
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
    if (threadIdx.x < 8) sumsq[blockIdx.x * 8 + threadIdx.x] = int(threadIdx.x) == c0 + int(blockIdx.x) ? ss : 0.f;
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
// cache (spm-kv/src/cache.rs:49-58).  The chunk's cached keys and values move
// through a two-stage shared-memory ring of kAttnTile positions with 16-byte
// asynchronous copies (every thread a share of the tile's rows, one copy group
// per tile); the first two tiles come from earlier steps and are requested
// before waiting for the kernel that produces this step's q, k, v.  Per tile every query head of the
// group scores the positions, the running softmax (max, sum) is updated and
// the unnormalised value sum rescaled and accumulated (online softmax); the
// last CTA of a (kv head, client) to finish combines the chunks' partials in
// chunk order.  The scores, the mask (diagonal included) and the GQA head
// mapping are the reference's:
//   LLAMA  : spm-kv/src/attend.rs:37-94   (dot * (1/sqrt hd))
//   others : spm-qwen3-slice/src/attention.rs:36-79 (dot / sqrt hd), with
//            per-head (Qwen3) or full-width (OLMoE) QK RMSNorm.
constexpr int kAttnThreads = 256;
constexpr int kAttnTile = 32;    // positions per staged tile
constexpr int kAttnStages = 2;

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

// The inputs of one (kv head, client): the group's queries into qs and, in
// decode mode, the new key and value into kn, vn, QK-normed and rotated (in
// query mode the queries are ready as they are); the CTA whose chunk
// [p0, p0 + P.chunk) holds the new position appends the key and value to the
// cache (spm-kv/src/cache.rs:49-58).  Waits for the kernel that produced q, k, v.
template <int NT>
__device__ void attn_prepare(const AttnParams& P, int i, int kvh, int pos, int p0, bool qmode, float* qs, float* kn,
                             float* vn, float* red, float* kc, float* vc, uint16_t* kp, uint16_t* vp) {
    const int hd = P.head_dim, group = P.heads / P.kv_heads;
    const int qw = P.heads * hd, kvw = P.kv_heads * hd;
    const bool llama = P.family == SPM_FAMILY_LLAMA;
    const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
    pdl_wait();
    const float* qg = P.q + size_t(i) * qw + size_t(kvh) * group * hd;
    for (int t = threadIdx.x; t < group * hd; t += NT) qs[t] = qg[t];
    if (!qmode)
        for (int t = threadIdx.x; t < hd; t += NT) {
            kn[t] = P.k[size_t(i) * kvw + size_t(kvh) * hd + t];
            vn[t] = P.v[size_t(i) * kvw + size_t(kvh) * hd + t];
        }
    __syncthreads();
    if (qmode) {
        // the query is normed and rotated, the cache rows are in place
    } else if (P.family == SPM_FAMILY_OLMOE) {
        float sq = 0.f, sk = 0.f;
        for (int t = threadIdx.x; t < qw; t += NT) sq = fmaf(P.q[size_t(i) * qw + t], P.q[size_t(i) * qw + t], sq);
        for (int t = threadIdx.x; t < kvw; t += NT) sk = fmaf(P.k[size_t(i) * kvw + t], P.k[size_t(i) * kvw + t], sk);
        sq = block_sum<NT>(sq, red);
        sk = block_sum<NT>(sk, red);
        const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, float(qw)), P.eps)));
        const float sck = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sk, float(kvw)), P.eps)));
        for (int t = threadIdx.x; t < group * hd; t += NT)
            qs[t] = __fmul_rn(__fmul_rn(qs[t], scq), P.q_norm[kvh * group * hd + t]);
        for (int t = threadIdx.x; t < hd; t += NT) kn[t] = __fmul_rn(__fmul_rn(kn[t], sck), P.k_norm[kvh * hd + t]);
        __syncthreads();
    } else if (!llama) {
        // per-head RMSNorm, one warp per head (spm-qwen3-slice/src/attention.rs:27-34)
        for (int h = warp; h <= group; h += NT / 32) {
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
    for (int t = threadIdx.x; !qmode && t < (group + 1) * half; t += NT) {
        const int h = t / half, j = t % half;
        float* x = h < group ? qs + h * hd : kn;
        const float2 cs = rt[j];
        rope_pair(x[j], x[j + half], cs.x, cs.y, llama);
    }
    __syncthreads();
    if (!qmode && pos >= p0 && pos < p0 + P.chunk)
        for (int t = threadIdx.x; t < hd; t += NT) {
            kc[size_t(pos) * kvw + t] = kn[t];
            vc[size_t(pos) * kvw + t] = vn[t];
            if (kp) {  // the plane rows of the same position
                store_planes(kp + size_t(pos) * kvw * 3, hd, t, kn[t]);
                store_planes(vp + size_t(pos) * kvw * 3, hd, t, vn[t]);
            }
        }
}

// Once every CTA of a (kv head, client) has written its chunk's partial to
// P.scratch (unnormalised value sums, then the max and the sum of
// exponentials of each head): the last one to finish combines the partials
// in chunk order into the output.
template <int NT>
__device__ void attn_combine(const AttnParams& P, int i, int kvh, int S) {
    const int hd = P.head_dim, group = P.heads / P.kv_heads, qw = P.heads * hd;
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
    for (int t = threadIdx.x; t < group * hd; t += NT) {
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

// The chunks of a (kv head, client) as one cluster of S CTAs (rank =
// chunk), each with its partial [group][hd + 2] in its own shared memory at
// `part`: once every partial is in place, CTA r combines the outputs
// r * per .. (r + 1) * per - 1, reading the partials from the other CTAs'
// shared memory in chunk order -- attn_combine's arithmetic, without the
// global round trip and the counter.  A second cluster barrier keeps every
// partial alive until all have been read.
template <int NT>
__device__ void attn_cluster_combine(const AttnParams& P, int i, int kvh, int S, int chunk, float* part) {
    namespace cg = cooperative_groups;
    const int hd = P.head_dim, group = P.heads / P.kv_heads, qw = P.heads * hd;
    cg::cluster_group cl = cg::this_cluster();
    cl.sync();
    pdl_trigger();
    const int per = (group * hd + S - 1) / S;
    for (int t = chunk * per + int(threadIdx.x); t < min(group * hd, (chunk + 1) * per); t += NT) {
        const int h = t / hd, dd = t % hd;
        float M = -INFINITY;
        for (int s = 0; s < S; s++) M = fmaxf(M, cl.map_shared_rank(part, s)[h * (hd + 2) + hd]);
        float Lsum = 0.f, O = 0.f;
        for (int s = 0; s < S; s++) {
            const float* ps = cl.map_shared_rank(part, s) + h * (hd + 2);
            const float m = ps[hd], l = ps[hd + 1], o = ps[dd];
            const float w = m == -INFINITY ? 0.f : expf(m - M);
            Lsum = fmaf(l, w, Lsum);
            O = fmaf(o, w, O);
        }
        P.out[size_t(i) * qw + (size_t(kvh) * group + h) * hd + dd] = __fdiv_rn(O, Lsum);
    }
    cl.sync();
}

// Shared memory of the attention kernel, in floats (mbarriers at the end).
struct AttnSmem {
    int qs, kn, vn, kt, vt, part, prob, stat, total;
    __host__ __device__ AttnSmem(int group, int hd) {
        const int ld = hd + 4;
        const int R = 8 / group;  // warps per head in the scores (group <= 8)
        qs = 0;
        kn = qs + group * hd;
        vn = kn + hd;
        kt = (vn + hd + 31) & ~31;                   // [stage][tile][ld]
        vt = kt + kAttnStages * kAttnTile * ld;
        part = vt + kAttnStages * kAttnTile * ld;    // [R][group][tile] partial dots
        prob = part + R * group * kAttnTile;          // [tile][group] probabilities
        stat = prob + kAttnTile * group;              // [group]: alpha, m, l (3 arrays) + 64 reduction
        total = stat + 3 * group + 64;
    }
};

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnParams P) {
    extern __shared__ __align__(128) float sm[];
    const int kvh = blockIdx.x, i = blockIdx.y, chunk = blockIdx.z, S = gridDim.z;
    const int hd = P.head_dim, group = P.heads / P.kv_heads;
    const int qw = P.heads * hd, kvw = P.kv_heads * hd, ld = hd + 4;
    const bool llama = P.family == SPM_FAMILY_LLAMA;
    const AttnSmem L(group, hd);
    float* qs = sm + L.qs;
    float* kn = sm + L.kn;
    float* vn = sm + L.vn;
    float* red = sm + L.stat + 3 * group;
    const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
    const bool qmode = P.qpos != nullptr;
    const int pos = qmode ? P.qpos[i] : P.pos[i];
    const int p0 = chunk * P.chunk;
    const int p1 = min(pos + 1, p0 + P.chunk);
    const int npos = max(0, p1 - p0), ntiles = (npos + kAttnTile - 1) / kAttnTile;
    const size_t cc = size_t(P.cache_client) + (qmode ? 0 : size_t(i));
    const size_t base = (cc * P.layers + P.layer) * P.context * size_t(kvw) + size_t(kvh) * hd;
    float* kc = P.kcache + base;
    float* vc = P.vcache + base;
    // every thread copies its share of tile j's key and value rows into stage
    // j % kAttnStages (16 bytes per copy), as one copy group
    // thread t copies 16-byte column c4 of rows r0, r0 + rstep, ... (hd / 4 divides 256)
    const int q4 = hd / 4, c4 = int(threadIdx.x) % q4, r0 = int(threadIdx.x) / q4, rstep = kAttnThreads / q4;
    auto request = [&](int j) {
        const int s = j % kAttnStages, t0 = p0 + j * kAttnTile, nr = min(kAttnTile, p1 - t0);
        for (int r = r0; r < nr; r += rstep) {
            const size_t g = size_t(t0 + r) * kvw + 4 * c4;
            const int o = (s * kAttnTile + r) * ld + 4 * c4;
            cp_async16(sm + L.kt + o, kc + g);
            cp_async16(sm + L.vt + o, vc + g);
        }
        cp_async_commit();
    };
    for (int j = 0; j < kAttnStages; j++) {
        if (j < ntiles) request(j);
        else cp_async_commit();  // empty group: the wait counts below stay uniform
    }
    uint16_t* kp = P.kplanes ? P.kplanes + base * 3 : nullptr;
    uint16_t* vp = P.vplanes ? P.vplanes + base * 3 : nullptr;
    attn_prepare<kAttnThreads>(P, i, kvh, pos, p0, qmode, qs, kn, vn, red, kc, vc, kp, vp);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(float(hd)));
    const float denom = __fsqrt_rn(float(hd));
    // scores: warp w takes head w % group (R = 8 / group warps per head, each
    // over hd / R dimensions), lane = position in the tile
    const int R = 8 / group;  // group <= 8 (the session checks)
    const int sh = warp % group, sr = warp / group;  // score head, dimension part
    const bool scorer = warp < group * R;
    const int dlen = hd / R, d0 = sr * dlen;
    // values: thread t owns dimension t % hd of the hpt consecutive heads
    // (t / hd) * hpt + k
    const int vd = int(threadIdx.x) % hd, vslot = int(threadIdx.x) / hd, vstep = kAttnThreads / hd;
    const int hpt = (group + vstep - 1) / vstep, h0 = vslot * hpt;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    float m_run = -INFINITY, l_run = 0.f;  // softmax state of head `warp` (warps < group)
    float* part = sm + L.part;
    float* prob = sm + L.prob;
    float* alpha = sm + L.stat;
    for (int j = 0; j < ntiles; j++) {
        const int s = j % kAttnStages, t0 = p0 + j * kAttnTile, nr = min(kAttnTile, p1 - t0);
        cp_async_wait<kAttnStages - 1>();  // this thread's copies of tile j have landed
        __syncthreads();                   // and every other thread's
        const float* kt = sm + L.kt + s * kAttnTile * ld;
        const float* vt = sm + L.vt + s * kAttnTile * ld;
        if (!qmode && pos >= t0 && pos < t0 + nr) {
            // the new row: the copy brought the cache's old contents
            __syncthreads();
            for (int t = threadIdx.x; t < hd; t += kAttnThreads) {
                sm[L.kt + (s * kAttnTile + pos - t0) * ld + t] = kn[t];
                sm[L.vt + (s * kAttnTile + pos - t0) * ld + t] = vn[t];
            }
            __syncthreads();
        }
        if (scorer) {
            float d = 0.f;
            if (lane < nr) {
                const float4* q = reinterpret_cast<const float4*>(qs + sh * hd + d0);
                const float4* k = reinterpret_cast<const float4*>(kt + lane * ld + d0);
#pragma unroll 8
                for (int c = 0; c < dlen / 4; c++) {
                    const float4 qq = q[c], kk = k[c];
                    d = fmaf(qq.x, kk.x, d);
                    d = fmaf(qq.y, kk.y, d);
                    d = fmaf(qq.z, kk.z, d);
                    d = fmaf(qq.w, kk.w, d);
                }
            }
            part[(sr * group + sh) * kAttnTile + lane] = d;
        }
        __syncthreads();
        if (warp < group) {
            // running softmax of head `warp`: lane = position
            float sc = -INFINITY;
            if (lane < nr) {
                float d = 0.f;
                for (int r = 0; r < R; r++) d += part[(r * group + warp) * kAttnTile + lane];
                sc = llama ? __fmul_rn(d, scale) : __fdiv_rn(d, denom);
            }
            float mx = sc;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_new = fmaxf(m_run, mx);
            const float a = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
            const float e = lane < nr ? expf(sc - m_new) : 0.f;
            l_run = fmaf(l_run, a, warp_sum(e));
            m_run = m_new;
            prob[lane * group + warp] = e;
            if (lane == 0) alpha[warp] = a;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (k < hpt && h0 + k < group) acc[k] *= alpha[h0 + k];
        if (hpt == 4 && h0 + 4 <= group) {
            // four heads: their probabilities of a position are one vector
            for (int p = 0; p < nr; p++) {
                const float v = vt[p * ld + vd];
                const float4 pr = *reinterpret_cast<const float4*>(prob + p * group + h0);
                acc[0] = fmaf(pr.x, v, acc[0]);
                acc[1] = fmaf(pr.y, v, acc[1]);
                acc[2] = fmaf(pr.z, v, acc[2]);
                acc[3] = fmaf(pr.w, v, acc[3]);
            }
        } else {
            for (int p = 0; p < nr; p++) {
                const float v = vt[p * ld + vd];
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if (k < hpt && h0 + k < group) acc[k] = fmaf(prob[p * group + h0 + k], v, acc[k]);
            }
        }
        __syncthreads();
        // stage s is free: request tile j + kAttnStages into it
        if (j + kAttnStages < ntiles) request(j + kAttnStages);
        else cp_async_commit();
    }
    cp_async_wait<0>();
    float* m_sh = sm + L.stat + group;  // [group] max, then [group] sum
    if (warp < group && lane == 0) {
        m_sh[warp] = m_run;
        m_sh[group + warp] = l_run;
    }
    __syncthreads();
    if (S == 1) {
        // the whole prefix is in this CTA: finish here (no partials)
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int h = h0 + k;
            if (k < hpt && h < group)
                P.out[size_t(i) * qw + (size_t(kvh) * group + h) * hd + vd] = __fdiv_rn(acc[k], m_sh[group + h]);
        }
        pdl_trigger();
        return;
    }
    // this chunk's partial: in the scratch, or (cluster) in the tile ring,
    // which the loop no longer uses
    float* outp = P.cluster ? sm + L.kt : P.scratch + ((size_t(i) * P.kv_heads + kvh) * S + chunk) * group * (hd + 2);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int h = h0 + k;
        if (k < hpt && h < group) outp[h * (hd + 2) + vd] = acc[k];
    }
    if (threadIdx.x < group) {
        outp[threadIdx.x * (hd + 2) + hd] = m_sh[threadIdx.x];
        outp[threadIdx.x * (hd + 2) + hd + 1] = m_sh[group + threadIdx.x];
    }
    if (!P.cluster) {
        attn_combine<kAttnThreads>(P, i, kvh, S);
        return;
    }
    attn_cluster_combine<kAttnThreads>(P, i, kvh, S, chunk, outp);
}

// ------------------------------------------------ attention on tensor cores ----
// Decode attention of the grouped-query models (4 to 8 query heads per kv
// head, head_dim 64 or 128) with the products on the tensor cores
// (mma.sync m16n8k16, bf16 operands, fp32 accumulation).  Every fp32 operand
// is split exactly into three bf16 parts by truncation, x = hi + mid + lo
// (8 + 8 + 8 significant bits), and a product takes the six part products
// hi*hi, hi*mid, mid*hi, hi*lo, mid*mid, lo*hi (the three left out are below
// 2^-32 of it), smallest first.  The cached keys and values are split once,
// when they are appended: the session keeps them as plane rows [3][hd] of
// bf16 beside the fp32 cache (6 bytes per value).  Per warp and 16 cached
// positions:
//   scores  S^T (16 positions x 8 heads) = K (16 x hd) . Q^T (hd x 8 heads)
//   softmax of each head over the positions: running max and sum, as in
//           attention_kernel (the reference's scores, scale and mask)
//   values  O^T (hd x 8 heads) += V^T (hd x 16) . P^T (16 x 8 heads)
// The key and value fragments come straight from the staged plane rows with
// ldmatrix (transposed for the values); the queries are split once per CTA
// and the probabilities per sub-tile, whose fragments become the B operand
// of the value product by a transpose of each 8 x 8 block (movmatrix);
// heads beyond the group are zero columns.  Grid (kv head, client, chunk)
// as attention_kernel, one CTA of eight warps per SM: warp w streams
// sub-tiles w, w + 8, ... of its chunk (16 positions each) through its own
// slot of bulk row copies, keys and values on separate barriers (the next
// sub-tile's keys go out once the scores have read this one's, its values
// once the value products have; later sub-tiles are asked into L2 at the
// start), the warps' softmax states are merged through shared memory, and
// the chunks' partials as in attention_kernel.
constexpr int kTcWarps = 8, kTcThreads = 32 * kTcWarps, kTcStages = 1, kTcSub = 16;

template <int HD>
struct AttnTcSmem {  // in bytes
    // a staged row is one position's [3][HD] bf16 planes; rows 16 bytes
    // apart beyond their size, so the 8 rows an ldmatrix reads fall on
    // distinct banks
    static constexpr int row = 3 * HD * 2 + 16;
    static constexpr int stage = 2 * kTcSub * row;  // keys, then values
    static constexpr int qs = 0, kn = 4 * 8 * HD, vn = kn + 4 * HD, red = vn + 4 * HD, ring = red + 4 * 64;
    static constexpr int total = ring + kTcWarps * kTcStages * stage;
    // after the loop the ring holds the warps' states: [warp][8 heads][HD + 2] floats
    static_assert(kTcWarps * 8 * (HD + 2) * 4 <= kTcWarps * kTcStages * stage, "warp states fit in the ring");
    static_assert(ring % 16 == 0 && row % 16 == 0, "bulk copy destinations 16-byte aligned");
};

// x0, x1 -> three bf16x2 words (hi, mid, lo), x0 in the low halves.
__device__ __forceinline__ void split3(float x0, float x1, uint32_t (&p)[3]) {
    const uint32_t b0 = __float_as_uint(x0), b1 = __float_as_uint(x1);
    const float r0 = __fsub_rn(x0, __uint_as_float(b0 & 0xffff0000u));
    const float r1 = __fsub_rn(x1, __uint_as_float(b1 & 0xffff0000u));
    const uint32_t c0 = __float_as_uint(r0), c1 = __float_as_uint(r1);
    const float l0 = __fsub_rn(r0, __uint_as_float(c0 & 0xffff0000u));
    const float l1 = __fsub_rn(r1, __uint_as_float(c1 & 0xffff0000u));
    p[0] = __byte_perm(b0, b1, 0x7632);
    p[1] = __byte_perm(c0, c1, 0x7632);
    p[2] = __byte_perm(__float_as_uint(l0), __float_as_uint(l1), 0x7632);
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d += A . B over the six part products, smallest first.
__device__ __forceinline__ void mma_split(float (&d)[4], const uint32_t (&a)[3][4], const uint32_t (&b)[3][2]) {
    mma_bf16(d, a[2], b[0][0], b[0][1]);  // lo  x hi
    mma_bf16(d, a[1], b[1][0], b[1][1]);  // mid x mid
    mma_bf16(d, a[0], b[2][0], b[2][1]);  // hi  x lo
    mma_bf16(d, a[1], b[0][0], b[0][1]);  // mid x hi
    mma_bf16(d, a[0], b[1][0], b[1][1]);  // hi  x mid
    mma_bf16(d, a[0], b[0][0], b[0][1]);  // hi  x hi
}

__device__ __forceinline__ uint32_t movtrans(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}

// Four 8 x 8 bf16 matrices from shared memory (lane l gives the address of
// row l % 8 of matrix l / 8), as the A fragment of m16n8k16; .trans
// transposes each matrix on the way.
__device__ __forceinline__ void ldsm_x4(uint32_t (&a)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&a)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3])
                 : "r"(addr));
}

template <int HD>
__global__ void __launch_bounds__(kTcThreads) attention_tc_kernel(const AttnParams P) {
    using L = AttnTcSmem<HD>;
    constexpr int KS = HD / 16;  // k-steps of the scores, m-tiles of the values
    constexpr int RW = 3 * HD;   // a plane row, in bf16
    extern __shared__ __align__(128) uint8_t smb[];
    __shared__ uint64_t kbar[kTcWarps], vbar[kTcWarps];  // this warp's key rows, value rows landed
    const int kvh = blockIdx.x, i = blockIdx.y, chunk = blockIdx.z, S = gridDim.z;
    const int group = P.heads / P.kv_heads, kvw = P.kv_heads * HD, qw = P.heads * HD;
    const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31), g = lane >> 2, t = lane & 3;
    const int pos = P.pos[i];
    const int p0 = chunk * P.chunk, p1 = min(pos + 1, p0 + P.chunk);
    const int npos = max(0, p1 - p0), nsub = (npos + kTcSub - 1) / kTcSub;
    const int mine = nsub > warp ? (nsub - warp + kTcWarps - 1) / kTcWarps : 0;  // this warp's sub-tiles
    const size_t cc = size_t(P.cache_client) + size_t(i);
    const size_t base = (cc * P.layers + P.layer) * P.context * size_t(kvw) + size_t(kvh) * HD;
    float* kc = P.kcache + base;
    float* vc = P.vcache + base;
    uint16_t* kp = P.kplanes + base * 3;  // position p's plane row at p * kvw * 3
    uint16_t* vp = P.vplanes + base * 3;
    uint8_t* ring = smb + L::ring + warp * kTcStages * L::stage;
    if (lane == 0) {
        mbar_init(&kbar[warp], 1);
        mbar_init(&vbar[warp], 1);
        mbar_fence_init();
    }
    __syncwarp();
    // the key (v = false) or value rows of sub-tile j of this warp, positions
    // s0 .. s0 + nr - 1, one row per lane; the keys of the next sub-tile are
    // requested once the scores have read this one's, the values once the
    // value products have
    auto issue = [&](int j, bool v) {
        const int s0 = p0 + (warp + kTcWarps * j) * kTcSub, nr = min(kTcSub, p1 - s0);
        uint64_t* bar = v ? &vbar[warp] : &kbar[warp];
        if (lane == 0) mbar_expect_tx(bar, uint32_t(nr) * RW * 2u);
        __syncwarp();
        if (lane < nr)
            bulk_g2s(ring + (v ? kTcSub + lane : lane) * L::row, (v ? vp : kp) + size_t(s0 + lane) * kvw * 3, RW * 2,
                     bar);
    };
    // the cached rows come from earlier steps: requested before the wait for
    // q, k, v, the first sub-tile into the ring and the warp's later ones
    // toward L2, so that their copies find them there
    if (mine > 0) {
        issue(0, false);
        issue(0, true);
    }
    for (int j = 1; j < mine; j++) {
        const int s0 = p0 + (warp + kTcWarps * j) * kTcSub, r = lane & 15;
        if (r < min(kTcSub, p1 - s0)) prefetch_l2((lane < 16 ? kp : vp) + size_t(s0 + r) * kvw * 3, RW * 2);
    }
    float* qs = reinterpret_cast<float*>(smb + L::qs);
    float* kn = reinterpret_cast<float*>(smb + L::kn);
    float* vn = reinterpret_cast<float*>(smb + L::vn);
    attn_prepare<kTcThreads>(P, i, kvh, pos, p0, false, qs, kn, vn, reinterpret_cast<float*>(smb + L::red), kc, vc,
                             kp, vp);
    const bool llama = P.family == SPM_FAMILY_LLAMA;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(float(HD)));
    const float denom = __fsqrt_rn(float(HD));
    // Q^T as the B operand: lane (g, t) holds head g's dims 2t, 2t+1 (+8) of each k-step
    uint32_t bq[KS][3][2];
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
        const bool on = g < group;
        const float* qr = qs + (on ? g : 0) * HD + ks * 16 + 2 * t;
        uint32_t lo[3], hi[3];
        split3(on ? qr[0] : 0.f, on ? qr[1] : 0.f, lo);
        split3(on ? qr[8] : 0.f, on ? qr[9] : 0.f, hi);
#pragma unroll
        for (int q = 0; q < 3; q++) {
            bq[ks][q][0] = lo[q];
            bq[ks][q][1] = hi[q];
        }
    }
    // ldmatrix addresses of this lane: keys (A = K, rows = positions) row
    // (l & 7) + 8 ((l >> 3) & 1), column 8 (l >> 4); values (A = V^T via
    // .trans, rows of the stage = positions) row (l & 7) + 8 (l >> 4),
    // column 8 ((l >> 3) & 1)
    const uint32_t k_off = uint32_t(((lane & 7) + 8 * ((lane >> 3) & 1)) * L::row + 16 * (lane >> 4));
    const uint32_t v_off = uint32_t((kTcSub + (lane & 7) + 8 * (lane >> 4)) * L::row + 16 * ((lane >> 3) & 1));
    // softmax state of heads 2t, 2t+1 (the sums per lane, added up at the end)
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o[KS][4];  // O^T m-tile mt: dims mt*16 + g (+8) x heads 2t, 2t+1
#pragma unroll
    for (int mt = 0; mt < KS; mt++) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    // copy phases issued and not yet waited for (-1: none): keys, values
    int kout = mine > 0 ? 0 : -1, vout = kout;
    bool ok = true;
    uint8_t* const kt = ring;
    for (int j = 0; j < mine; j++) {
        const int s0 = p0 + (warp + kTcWarps * j) * kTcSub, nr = min(kTcSub, p1 - s0);
        if (!mbar_wait(&kbar[warp], uint32_t(j) & 1u)) {
            flag(P.status, 6);
            ok = false;
            break;
        }
        kout = -1;
        if (nr < kTcSub)  // key rows past the chunk: zero (their scores are masked)
            for (int e = lane; e < (kTcSub - nr) * RW; e += 32)
                reinterpret_cast<uint16_t*>(kt + (nr + e / RW) * L::row)[e % RW] = 0;
        if (pos >= s0 && pos < s0 + nr)  // the new row: the copy brought the cache's old contents
            for (int c = lane; c < HD; c += 32)
                store_planes(reinterpret_cast<uint16_t*>(kt + (pos - s0) * L::row), HD, c, kn[c]);
        __syncwarp();
        const uint32_t ks_base = saddr(kt) + k_off, vs_base = saddr(kt) + v_off;
        // ---- scores: two accumulators over alternate k-steps ----
        float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < KS; ks++) {
            uint32_t a[3][4];
#pragma unroll
            for (int q = 0; q < 3; q++) ldsm_x4(a[q], ks_base + uint32_t(q * HD * 2 + ks * 32));
            if (ks & 1) mma_split(sb, a, bq[ks]);
            else mma_split(sa, a, bq[ks]);
        }
        __syncwarp();
        if (j + 1 < mine) {
            fence_proxy_async();  // the key rows' reads and writes before the copies that refill them
            issue(j + 1, false);
            kout = j + 1;
        }
        // ---- softmax: sc[0], sc[1] position g, heads 2t, 2t+1; sc[2], sc[3] position g + 8 ----
        float sc[4], pr[4], mx[2], alpha[2];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float d = sa[e] + sb[e];
            const bool valid = (e < 2 ? g : g + 8) < nr;
            sc[e] = !valid ? -INFINITY : llama ? __fmul_rn(d, scale) : __fdiv_rn(d, denom);
        }
        mx[0] = fmaxf(sc[0], sc[2]);
        mx[1] = fmaxf(sc[1], sc[3]);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], off));
            mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], off));
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const float m_new = fmaxf(m_run[h], mx[h]);
            alpha[h] = m_run[h] == -INFINITY ? 0.f : expf(m_run[h] - m_new);
            m_run[h] = m_new;
        }
#pragma unroll
        for (int e = 0; e < 4; e++) pr[e] = sc[e] == -INFINITY ? 0.f : expf(sc[e] - m_run[e & 1]);
#pragma unroll
        for (int h = 0; h < 2; h++) l_run[h] = fmaf(l_run[h], alpha[h], pr[h] + pr[h + 2]);
#pragma unroll
        for (int mt = 0; mt < KS; mt++) {
            o[mt][0] *= alpha[0];
            o[mt][1] *= alpha[1];
            o[mt][2] *= alpha[0];
            o[mt][3] *= alpha[1];
        }
        // ---- P^T as the B operand: positions 2t, 2t+1 (+8) of head g ----
        uint32_t bp[3][2];
        {
            uint32_t pa[3], pb[3];
            split3(pr[0], pr[1], pa);
            split3(pr[2], pr[3], pb);
#pragma unroll
            for (int q = 0; q < 3; q++) {
                bp[q][0] = movtrans(pa[q]);
                bp[q][1] = movtrans(pb[q]);
            }
        }
        if (!mbar_wait(&vbar[warp], uint32_t(j) & 1u)) {
            flag(P.status, 6);
            ok = false;
            break;
        }
        vout = -1;
        if (nr < kTcSub)  // value rows past the chunk: zero (probability 0, value finite)
            for (int e = lane; e < (kTcSub - nr) * RW; e += 32)
                reinterpret_cast<uint16_t*>(kt + (kTcSub + nr + e / RW) * L::row)[e % RW] = 0;
        if (pos >= s0 && pos < s0 + nr)
            for (int c = lane; c < HD; c += 32)
                store_planes(reinterpret_cast<uint16_t*>(kt + (kTcSub + pos - s0) * L::row), HD, c, vn[c]);
        __syncwarp();
        // ---- values: V^T m-tile mt (dims mt*16 ..) times P^T ----
#pragma unroll
        for (int mt = 0; mt < KS; mt++) {
            uint32_t a[3][4];
#pragma unroll
            for (int q = 0; q < 3; q++) ldsm_x4_trans(a[q], vs_base + uint32_t(q * HD * 2 + mt * 32));
            mma_split(o[mt], a, bp);
        }
        __syncwarp();
        if (j + 1 < mine) {
            fence_proxy_async();  // the value rows' reads and writes before the copies that refill them
            issue(j + 1, true);
            vout = j + 1;
        }
    }
    if (!ok) {
        // a wait gave up: the copies still in flight land before the CTA ends
        // (each phase waited for once more, bounded), and this warp adds nothing
        if (kout >= 0) mbar_wait(&kbar[warp], uint32_t(kout) & 1u);
        if (vout >= 0) mbar_wait(&vbar[warp], uint32_t(vout) & 1u);
        m_run[0] = m_run[1] = -INFINITY;
        l_run[0] = l_run[1] = 0.f;
#pragma unroll
        for (int mt = 0; mt < KS; mt++) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
    }
#pragma unroll
    for (int h = 0; h < 2; h++)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], off);
    __syncthreads();  // every warp is done with its ring: it holds the warps' states now
    {
        float* ws = reinterpret_cast<float*>(smb + L::ring) + warp * 8 * (HD + 2);
#pragma unroll
        for (int mt = 0; mt < KS; mt++) {
            ws[(2 * t) * (HD + 2) + mt * 16 + g] = o[mt][0];
            ws[(2 * t + 1) * (HD + 2) + mt * 16 + g] = o[mt][1];
            ws[(2 * t) * (HD + 2) + mt * 16 + g + 8] = o[mt][2];
            ws[(2 * t + 1) * (HD + 2) + mt * 16 + g + 8] = o[mt][3];
        }
        if (g == 0) {
            ws[(2 * t) * (HD + 2) + HD] = m_run[0];
            ws[(2 * t + 1) * (HD + 2) + HD] = m_run[1];
            ws[(2 * t) * (HD + 2) + HD + 1] = l_run[0];
            ws[(2 * t + 1) * (HD + 2) + HD + 1] = l_run[1];
        }
    }
    __syncthreads();
    // the warps' states merged in warp order: this chunk's partial (in the
    // scratch, or with a cluster in the ring after the warps' states), or
    // the output
    float* outp = P.cluster ? reinterpret_cast<float*>(smb + L::ring) + kTcWarps * 8 * (HD + 2)
                            : P.scratch + ((size_t(i) * P.kv_heads + kvh) * S + chunk) * group * (HD + 2);
    for (int e = threadIdx.x; e < group * HD; e += kTcThreads) {
        const int h = e / HD, d = e % HD;
        const float* st = reinterpret_cast<const float*>(smb + L::ring) + h * (HD + 2);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kTcWarps; w++) M = fmaxf(M, st[w * 8 * (HD + 2) + HD]);
        float Lsum = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kTcWarps; w++) {
            const float* ws = st + w * 8 * (HD + 2);
            const float m = ws[HD];
            const float wt = m == -INFINITY ? 0.f : expf(m - M);
            Lsum = fmaf(ws[HD + 1], wt, Lsum);
            O = fmaf(ws[d], wt, O);
        }
        if (S == 1) {
            P.out[size_t(i) * qw + (size_t(kvh) * group + h) * HD + d] = __fdiv_rn(O, Lsum);
        } else {
            outp[h * (HD + 2) + d] = O;
            if (d == 0) {
                outp[h * (HD + 2) + HD] = M;
                outp[h * (HD + 2) + HD + 1] = Lsum;
            }
        }
    }
    if (S == 1) {
        pdl_trigger();
        return;
    }
    if (P.cluster) {
        attn_cluster_combine<kTcThreads>(P, i, kvh, S, chunk, outp);
        return;
    }
    attn_combine<kTcThreads>(P, i, kvh, S);
}

}  // namespace

size_t attention_smem(const AttnParams& P) {
    const AttnSmem L(P.heads / P.kv_heads, P.head_dim);
    return size_t(L.total) * sizeof(float);
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

// An attention grid (kv head, client, chunk); with `cluster` the chunks of
// each (kv head, client) form one thread-block cluster (at most 8).
static cudaError_t launch_attention_grid(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                                         int cluster, void** args) {
    if (!cluster) return launch_pdl(fn, grid, block, smem, s, pdl, args);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = grid.z;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// The tensor-core kernel takes decode steps of 4 to 8 query heads per kv head
// and head_dim 64 or 128 with at least 16 (kv head, client) pairs.  (With
// fewer pairs -- Qwen3-8B with one client: 8 -- a step's attention is a
// latency chain of prologue, one sub-tile per warp and the chunk combine,
// and the 256-thread CUDA-core kernel measured shorter: 23 against 32 us
// per layer.)
static bool attention_tc_fits(const AttnParams& P, int n) {
    const int group = P.heads / P.kv_heads;
    return P.qpos == nullptr && P.kplanes && P.vplanes && group >= 4 && group <= 8 &&
           (P.head_dim == 64 || P.head_dim == 128) && P.kv_heads * n >= 16;
}

template <int HD>
static cudaError_t launch_attention_tc(const AttnParams& P, int n, int sms, cudaStream_t s, bool pdl) {
    const size_t smem = size_t(AttnTcSmem<HD>::total);
    static int configured_for = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_for != dev) {
        cudaError_t e = cudaFuncSetAttribute(attention_tc_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(smem));
        if (e != cudaSuccess) return e;
        configured_for = dev;
    }
    // one CTA per SM: about as many (kv head, client, chunk) CTAs as SMs,
    // chunks a multiple of the warps' 16 positions each (and of the 64 the
    // session's partials are sized for)
    constexpr int step = kTcWarps * kTcSub > kAttnMinChunk ? kTcWarps * kTcSub : kAttnMinChunk;
    const int pairs = P.kv_heads * n;
    const int want = std::max(1, sms / pairs);
    int chunk = (P.context + want - 1) / want;
    chunk = std::max(step, (chunk + step - 1) / step * step);
    const int chunks = (P.context + chunk - 1) / chunk;
    AttnParams p = P;
    p.chunk = chunk;
    // up to eight chunks of a pair form a cluster and combine on chip
    p.cluster = chunks > 1 && chunks <= 8 ? 1 : 0;
    void* args[] = {&p};
    return launch_attention_grid(reinterpret_cast<const void*>(attention_tc_kernel<HD>),
                                 dim3(P.kv_heads, n, chunks), dim3(kTcThreads), smem, s, pdl, p.cluster, args);
}

cudaError_t launch_attention(const AttnParams& P, int n, cudaStream_t s, bool pdl) {
    if (attention_tc_fits(P, n)) {
        static int tc_sms[64] = {};
        int d = 0;
        cudaGetDevice(&d);
        if (d < 64 && !tc_sms[d]) cudaDeviceGetAttribute(&tc_sms[d], cudaDevAttrMultiProcessorCount, d);
        const int sms = d < 64 && tc_sms[d] ? tc_sms[d] : 148;
        return P.head_dim == 128 ? launch_attention_tc<128>(P, n, sms, s, pdl) : launch_attention_tc<64>(P, n, sms, s, pdl);
    }
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
    while (chunk > kAttnMinChunk && ((P.context + chunk - 1) / chunk) * P.kv_heads * n < 3 * target) chunk /= 2;
    int chunks = (P.context + chunk - 1) / chunk;
    AttnParams p = P;
    p.cluster = 0;
    if (P.kv_heads * n < 16) {
        // Few (kv head, client) pairs (one client of Qwen3-8B: 8): the step's
        // attention is a latency chain, so each pair's prefix is split into
        // at most 8 chunks that form one cluster and combine on chip.
        int c8 = (P.context + 7) / 8;
        c8 = std::max(kAttnMinChunk, (c8 + kAttnMinChunk - 1) / kAttnMinChunk * kAttnMinChunk);
        const int s8 = (P.context + c8 - 1) / c8;
        if (s8 > 1) {
            chunk = c8;
            chunks = s8;
            p.cluster = 1;
        }
    }
    p.chunk = chunk;
    void* args[] = {&p};
    return launch_attention_grid(reinterpret_cast<const void*>(attention_kernel), dim3(P.kv_heads, n, chunks),
                                 dim3(kAttnThreads), smem, s, pdl, p.cluster, args);
}

cudaError_t launch_attention_queries(const AttnParams& P, int n, cudaStream_t s) {
    const size_t smem = attention_smem(P);
    static int configured_for = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && configured_for != dev) {
        cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        if (e != cudaSuccess) return e;
        configured_for = dev;
    }
    AttnParams p = P;
    p.cluster = 0;
    p.chunk = P.context;  // one CTA covers the whole prefix: S == 1, no partials
    void* args[] = {&p};
    return launch_pdl(reinterpret_cast<const void*>(attention_kernel), dim3(P.kv_heads, n, 1), dim3(kAttnThreads),
                      smem, s, false, args);
}

cudaError_t launch_embed(uint32_t dtype, const uint8_t* tiles, const Packed& p, const uint32_t* tokens, int n,
                         float* out, float* sumsq, cudaStream_t s, bool pdl, int c0) {
    Packed pk = p;
    void* args[] = {&dtype, &tiles, &pk, &tokens, &out, &sumsq, &c0};
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
