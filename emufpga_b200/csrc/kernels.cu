// sm_100a kernels of the decode token loop besides the GEMV (gemv.cu):
// exact dequantization (parity hook and embedding lookup), attention over the
// device KV cache, greedy selection, position bookkeeping.
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
    pdl_wait();
    const float* qg = P.q + size_t(i) * qw + size_t(kvh) * group * hd;
    for (int t = threadIdx.x; t < group * hd; t += kAttnThreads) qs[t] = qg[t];
    if (!qmode)
        for (int t = threadIdx.x; t < hd; t += kAttnThreads) {
            kn[t] = P.k[size_t(i) * kvw + size_t(kvh) * hd + t];
            vn[t] = P.v[size_t(i) * kvw + size_t(kvh) * hd + t];
        }
    __syncthreads();
    if (qmode) {
        // the query is normed and rotated, the cache rows are in place
    } else if (P.family == SPM_FAMILY_OLMOE) {
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
        for (int h = warp; h <= group; h += kAttnThreads / 32) {
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
    for (int t = threadIdx.x; !qmode && t < (group + 1) * half; t += kAttnThreads) {
        const int h = t / half, j = t % half;
        float* x = h < group ? qs + h * hd : kn;
        const float2 cs = rt[j];
        rope_pair(x[j], x[j + half], cs.x, cs.y, llama);
    }
    __syncthreads();
    if (!qmode && pos >= p0 && pos < p0 + P.chunk)
        for (int t = threadIdx.x; t < hd; t += kAttnThreads) {
            kc[size_t(pos) * kvw + t] = kn[t];
            vc[size_t(pos) * kvw + t] = vn[t];
        }
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
    float* outp = P.scratch + ((size_t(i) * P.kv_heads + kvh) * S + chunk) * group * (hd + 2);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int h = h0 + k;
        if (k < hpt && h < group) outp[h * (hd + 2) + vd] = acc[k];
    }
    if (threadIdx.x < group) {
        outp[threadIdx.x * (hd + 2) + hd] = m_sh[threadIdx.x];
        outp[threadIdx.x * (hd + 2) + hd + 1] = m_sh[group + threadIdx.x];
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
    while (chunk > kAttnMinChunk && ((P.context + chunk - 1) / chunk) * P.kv_heads * n < 3 * target) chunk /= 2;
    const int chunks = (P.context + chunk - 1) / chunk;
    AttnParams p = P;
    p.chunk = chunk;
    void* args[] = {&p};
    return launch_pdl(reinterpret_cast<const void*>(attention_kernel), dim3(P.kv_heads, n, chunks),
                      dim3(kAttnThreads), smem, s, pdl, args);
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
