// The streamed dequant-GEMV: y[p][r] = sum_c W[r][c] * x[p][c] for up to 8
// clients p off ONE pass over the packed weights (host_pack.cpp layout).
//
// Each CTA owns a contiguous run of 4-row tiles.  A producer warp streams the
// run into a shared-memory ring with cp.async.bulk (one bulk copy per tile,
// completion on an mbarrier), so the bytes in flight per SM do not depend on
// registers or occupancy.  Eight consumer warps in two groups work on every
// tile: a group takes two of its rows (or, for a gate/up pair, every row of
// one of the two matrices), its four warps split the row's 32-weight units,
// and partial sums are combined in shared memory in warp order.
//
// Per unit a lane turns four codes at a time into floats with one byte
// permute each and applies them to all clients' activations (staged once per
// CTA in shared memory) while they sit in registers -- the reference's "one
// weight, every position" schedule (spm-linear/src/resident.rs:120-137).
// The K-quant codes q (< 128) become f = 1 + q/128 exactly (q in the
// mantissa of 1.0), so that per 16- or 32-value sub-block
//     sum_c q_c x_c = 128 * sum_c f_c x_c - 128 * sum_c x_c
// with the activation sums precomputed once per CTA; Q8_0 codes become
// 2^23 + (q ^ 128) and are re-centred exactly.  Block scales are applied once
// per sub-block:
//     sum_c w_c x_c = (d*sc) * sum_c q_c x_c  [- (dmin*m) * sum_c x_c]
// which is the reference dot product regrouped.  The weights are the
// reference's bit for bit (the dequant kernel checks that); the fp32 sums are
// in a different order than the reference's FMA chain.
//
// Launched with programmatic dependent launch: the ring is filled while the
// previous kernel still runs (weights never depend on it), and the consumers
// read the activations only after griddepcontrol.wait.
#pragma once
#include "device.cuh"
#include "moe.h"

namespace spm {
namespace gemv {
using namespace dev;

constexpr int kGroupWarps = 4;                 // warps per consumer group
constexpr int kConsumers = 2 * kGroupWarps;    // consumer warps per CTA
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kMaxSlots = 16;
constexpr size_t kRingBytes = 96 * 1024;       // weight ring, at most
constexpr size_t kSmemMax = 212 * 1024;        // dynamic shared memory, at most (static use ~7 KB)
constexpr size_t kHalfSm = 104 * 1024;         // dynamic shared memory for two CTAs per SM
constexpr size_t kRingMin = 24 * 1024;         // weight ring, at least
constexpr int kAuxPrefetch = 1024;             // residual values prefetched per CTA, at most

// Activations of the clients in shared memory (normalised when the launch
// fuses an RMSNorm).  Unit u's 32 values are 8 chunks of 4; chunk t is stored
// at slot t ^ (u & 7) so that the lanes of a quarter-warp, reading chunk t of
// consecutive units, hit distinct banks.  xsum holds the sum of every 16
// consecutive values (K-quant re-centring).
__device__ __forceinline__ uint32_t xoff(uint32_t u, uint32_t chunk) {
    return (u * 8 + (chunk ^ (u & 7))) * 16;
}

template <int NC>
struct XIn {
    uint32_t xs, cstride;  // shared base of x, bytes per client
    uint32_t ss, sstride;  // shared base of the 16-value sums, bytes per client
    __device__ __forceinline__ void load(uint32_t u, int off, float4 (&o)[NC]) const {
        const uint32_t a = xs + xoff(u, uint32_t(off) >> 2);
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const uint4 v = lds128(a + c * cstride);
            o[c] = make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
        }
    }
    // sum of the 16 values starting at 32*u + 16*half, per client
    __device__ __forceinline__ void sums(uint32_t u, int half, float (&o)[NC]) const {
#pragma unroll
        for (int c = 0; c < NC; c++) o[c] = __uint_as_float(lds32(ss + c * sstride + (2 * u + half) * 4));
    }
};

template <int NC>
__device__ __forceinline__ void dot4(float (&s)[NC], float f0, float f1, float f2, float f3, const float4 (&x)[NC]) {
#pragma unroll
    for (int c = 0; c < NC; c++) {
        s[c] = fmaf(f0, x[c].x, s[c]);
        s[c] = fmaf(f1, x[c].y, s[c]);
        s[c] = fmaf(f2, x[c].z, s[c]);
        s[c] = fmaf(f3, x[c].w, s[c]);
    }
}

__device__ __forceinline__ uint32_t word(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

// 1 + (byte B of q & 127)/128 exactly, for q bytes with bit 7 set.
template <int B>
__device__ __forceinline__ float onef(uint32_t q) {
    return __uint_as_float(__byte_perm(q, 0x3F000000u, 0x7044u | (B << 8)));
}
// int8 -> float exactly: 2^23 + (b ^ 128) - (2^23 + 128).
__device__ __forceinline__ float i8f(uint32_t b) { return bytef<0>(b ^ 0x80u) - 8388736.0f; }

template <int VR, int NC>
__device__ __forceinline__ void zero(float (&s)[VR][NC]) {
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) s[v][c] = 0.f;
}

// Every unit function adds unit u of the rows `rows` (row indices inside the
// tile at shared address t) times the activations into acc[v][client].

// ------------------------------------------------------------------ Q8_0 --
template <int NC, int VR>
__device__ __forceinline__ void unit_q8_0(uint32_t t, const uint32_t (&rows)[VR], uint32_t u, const GemvLaunch& L,
                                          const XIn<NC>& X, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5;
    uint4 q0[VR], q1[VR];
    float d[VR];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint32_t unit = rows[v] * U + u;
        q0[v] = lds128(t + unit * 32);
        q1[v] = lds128(t + unit * 32 + 16);
        d[v] = h2f(lds16(t + L.plane1 + unit * 2));
    }
    float s[VR][NC];
    zero(s);
#pragma unroll
    for (int k = 0; k < 8; k++) {
        float4 x[NC];
        X.load(u, 4 * k, x);
#pragma unroll
        for (int v = 0; v < VR; v++) {
            const uint32_t w = (k < 4 ? word(q0[v], k) : word(q1[v], k - 4)) ^ 0x80808080u;
            const float c0 = 8388736.0f;  // 2^23 + 128: (u8 ^ 0x80) - 128 == int8
            dot4<NC>(s[v], bytef<0>(w) - c0, bytef<1>(w) - c0, bytef<2>(w) - c0, bytef<3>(w) - c0, x);
        }
    }
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) acc[v][c] = fmaf(d[v], s[v][c], acc[v][c]);
}

// ------------------------------------------------------------------ Q6_K --
template <int NC, int VR>
__device__ __forceinline__ void unit_q6_k(uint32_t t, const uint32_t (&rows)[VR], uint32_t u, const GemvLaunch& L,
                                          const XIn<NC>& X, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5, B = L.cols >> 8;
    uint4 ql[VR];
    uint2 qh[VR];
    float ds[VR][2];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint32_t unit = rows[v] * U + u;
        ql[v] = lds128(t + unit * 16);
        qh[v] = lds64(t + L.plane1 + unit * 8);
        const uint32_t sc = lds16(t + L.plane2 + unit * 2);
        const float d = h2f(lds16(t + L.plane3 + (rows[v] * B + (u >> 3)) * 2));
        ds[v][0] = d * i8f(sc & 0xffu);
        ds[v][1] = d * i8f(sc >> 8);
    }
#pragma unroll
    for (int run = 0; run < 2; run++) {
        float s[VR][NC], xs[NC];
        zero(s);
        X.sums(u, run, xs);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float4 x[NC];
            X.load(u, 16 * run + 4 * k, x);
#pragma unroll
            for (int v = 0; v < VR; v++) {
                const uint32_t w = word(ql[v], k);
                const uint32_t h = run ? qh[v].y : qh[v].x;
                const uint32_t hs = ((k < 2 ? h << (4 - 2 * k) : h >> (2 * k - 4)) & 0x30303030u) | 0x80808080u;
                const uint32_t q = ((run ? (w >> 4) : w) & 0x0F0F0F0Fu) | hs;
                dot4<NC>(s[v], onef<0>(q), onef<1>(q), onef<2>(q), onef<3>(q), x);
            }
        }
        // sum (q - 32) x = 128 sum f x - 160 sum x
#pragma unroll
        for (int v = 0; v < VR; v++)
#pragma unroll
            for (int c = 0; c < NC; c++) acc[v][c] = fmaf(ds[v][run], fmaf(s[v][c], 128.0f, -160.0f * xs[c]), acc[v][c]);
    }
}

// ------------------------------------------------------------------ Q5_K --
__device__ __forceinline__ uint32_t sbyte(const uint4& m, int k) {  // scales byte k (0..11)
    const uint32_t w = k < 4 ? m.y : k < 8 ? m.z : m.w;
    return (w >> (8 * (k & 3))) & 0xffu;
}

template <int NC, int VR>
__device__ __forceinline__ void unit_q5_k(uint32_t t, const uint32_t (&rows)[VR], uint32_t u, const GemvLaunch& L,
                                          const XIn<NC>& X, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5, B = L.cols >> 8;
    const int j = int(u & 7);
    uint4 qs[VR];
    uint32_t qh[VR];
    float ds[VR], dm[VR];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint32_t unit = rows[v] * U + u;
        const uint4 m = lds128(t + (rows[v] * B + (u >> 3)) * 16);
        qs[v] = lds128(t + L.plane1 + unit * 16);
        qh[v] = lds32(t + L.plane2 + unit * 4);
        uint32_t sc, mn;
        if (j < 4) {
            sc = sbyte(m, j) & 63;
            mn = sbyte(m, j + 4) & 63;
        } else {
            sc = (sbyte(m, j + 4) & 15) | ((sbyte(m, j - 4) >> 6) << 4);
            mn = (sbyte(m, j + 4) >> 4) | ((sbyte(m, j) >> 6) << 4);
        }
        ds[v] = h2f(m.x) * (bytef<0>(sc) - 8388608.0f);
        dm[v] = h2f(m.x >> 16) * (bytef<0>(mn) - 8388608.0f);
    }
    float s[VR][NC], xa[NC], xb[NC];
    zero(s);
    X.sums(u, 0, xa);
    X.sums(u, 1, xb);
#pragma unroll
    for (int run = 0; run < 2; run++) {
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float4 x[NC];
            X.load(u, 16 * run + 4 * k, x);
#pragma unroll
            for (int v = 0; v < VR; v++) {
                const uint32_t w = word(qs[v], k);
                const uint32_t sp =
                    (((((qh[v] >> (16 * run + 4 * k)) & 0xfu) * 0x02040810u) & 0x10101010u)) | 0x80808080u;
                const uint32_t q = ((run ? (w >> 4) : w) & 0x0F0F0F0Fu) | sp;
                dot4<NC>(s[v], onef<0>(q), onef<1>(q), onef<2>(q), onef<3>(q), x);
            }
        }
    }
    // sum w x = ds * (128 sum f x - 128 sum x) - dm * sum x
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const float xsum = xa[c] + xb[c];
            acc[v][c] = fmaf(-dm[v], xsum, fmaf(ds[v], fmaf(s[v][c], 128.0f, -128.0f * xsum), acc[v][c]));
        }
}

// ------------------------------------------------------------------ Q2_K --
template <int NC, int VR>
__device__ __forceinline__ void unit_q2_k(uint32_t t, const uint32_t (&rows)[VR], uint32_t u, const GemvLaunch& L,
                                          const XIn<NC>& X, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5, B = L.cols >> 8;
    uint2 qs[VR];
    uint32_t sc[VR];
    float d[VR], dmin[VR];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint32_t unit = rows[v] * U + u;
        qs[v] = lds64(t + unit * 8);
        sc[v] = lds16(t + L.plane1 + unit * 2);
        const uint32_t dd = lds32(t + L.plane2 + (rows[v] * B + (u >> 3)) * 4);
        d[v] = h2f(dd);
        dmin[v] = h2f(dd >> 16);
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float s[VR][NC], xs[NC];
        zero(s);
        X.sums(u, h, xs);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float4 x[NC];
            X.load(u, 16 * h + 4 * k, x);
#pragma unroll
            for (int v = 0; v < VR; v++) {
                const uint32_t q = (((h ? qs[v].y : qs[v].x) >> (2 * k)) & 0x03030303u) | 0x80808080u;
                dot4<NC>(s[v], onef<0>(q), onef<1>(q), onef<2>(q), onef<3>(q), x);
            }
        }
#pragma unroll
        for (int v = 0; v < VR; v++) {
            const uint32_t b = (sc[v] >> (8 * h)) & 0xffu;
            const float dl = d[v] * (bytef<0>(b & 15u) - 8388608.0f);
            const float ml = dmin[v] * (bytef<0>(b >> 4) - 8388608.0f);
#pragma unroll
            for (int c = 0; c < NC; c++)
                acc[v][c] = fmaf(-ml, xs[c], fmaf(dl, fmaf(s[v][c], 128.0f, -128.0f * xs[c]), acc[v][c]));
        }
    }
}

// ------------------------------------------------------------------- F32 --
template <int NC, int VR>
__device__ __forceinline__ void unit_f32(uint32_t t, const uint32_t (&rows)[VR], uint32_t u, const GemvLaunch& L,
                                         const XIn<NC>& X, float (&acc)[VR][NC]) {
#pragma unroll
    for (int k = 0; k < 8; k++) {
        float4 x[NC];
        X.load(u, 4 * k, x);
#pragma unroll
        for (int v = 0; v < VR; v++) {
            const uint4 w = lds128(t + (rows[v] * L.cols + 32 * u + 4 * k) * 4);
            dot4<NC>(acc[v], __uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w),
                     x);
        }
    }
}

template <int ENC, int NC, int VR>
__device__ __forceinline__ void unit_dot(uint32_t t, const uint32_t (&rows)[VR], uint32_t u, const GemvLaunch& L,
                                         const XIn<NC>& X, float (&acc)[VR][NC]) {
    if constexpr (ENC == SPM_Q8_0) unit_q8_0<NC, VR>(t, rows, u, L, X, acc);
    else if constexpr (ENC == SPM_Q6_K) unit_q6_k<NC, VR>(t, rows, u, L, X, acc);
    else if constexpr (ENC == SPM_Q5_K) unit_q5_k<NC, VR>(t, rows, u, L, X, acc);
    else if constexpr (ENC == SPM_Q2_K) unit_q2_k<NC, VR>(t, rows, u, L, X, acc);
    else unit_f32<NC, VR>(t, rows, u, L, X, acc);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return __fdiv_rn(g, 1.0f + expf(-g)) * u; }

__device__ __forceinline__ const GemvJob& pick(const GemvLaunch& L, uint32_t g) {
    if (L.njobs > 3 && g >= L.job[3].tile_begin) return L.job[3];
    if (L.njobs > 2 && g >= L.job[2].tile_begin) return L.job[2];
    if (L.njobs > 1 && g >= L.job[1].tile_begin) return L.job[1];
    return L.job[0];
}

// Rows of a pass per group: single matrix -> 2 of the tile's 4 rows per group
// (group g: rows g, g+2) in one pass; gate/up pair -> group g takes matrix g,
// VR rows per pass.
template <int NC, bool DUAL>
struct Shape {
    static constexpr int VR = DUAL ? (NC <= 4 ? 4 : 2) : 2;
    static constexpr int PASSES = DUAL ? kTileRows / VR : 1;
};

// A CTA owns tiles [t0, t1).  Warp 8 (producer) streams them through the
// ring; warps 0-7 (consumers) all pass every ring slot, so each full/empty
// barrier phase is awaited in order by every waiter.
template <int ENC, int NC, bool DUAL>
__global__ void __launch_bounds__(kThreads, 2) gemv_stream(const __grid_constant__ GemvLaunch L) {
    constexpr int VR = Shape<NC, DUAL>::VR, PASSES = Shape<NC, DUAL>::PASSES;
    constexpr bool kquant = ENC == SPM_Q6_K || ENC == SPM_Q5_K || ENC == SPM_Q2_K;
    extern __shared__ __align__(128) uint8_t ring[];
    __shared__ uint64_t full[kMaxSlots], empty[kMaxSlots];
    __shared__ float nscale[8];
    __shared__ float part[2][kConsumers][VR][NC];
    __shared__ float sqw[kConsumers][8];
    __shared__ float auxs[kAuxPrefetch];
    __shared__ int32_t xrows[NC], yrows[NC], srows[NC];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t t0, t1;
    uint32_t rbase = 0, rlim = 0xffffffffu;  // expert mode: rows of the expert's matrix
    int n_act = NC;  // clients of this CTA with data (expert mode: the expert's clients)
    if (L.plan) {
        // expert mode: the plan comes from the previous kernel
        pdl_wait();
        const int a = int(blockIdx.x) / L.expert_chunks, chunk = int(blockIdx.x) % L.expert_chunks;
        if (a >= L.plan->count) {
            pdl_trigger();
            return;
        }
        const uint32_t e = uint32_t(L.plan->expert[a]), Te = L.expert_tiles, C = uint32_t(L.expert_chunks);
        rbase = e * Te * kTileRows;
        rlim = Te * kTileRows;
        t0 = e * Te + uint32_t(uint64_t(Te) * chunk / C);
        t1 = e * Te + uint32_t(uint64_t(Te) * (chunk + 1) / C);
        n_act = L.plan->ntok[a];
        if (threadIdx.x < NC) {
            const int c = threadIdx.x;
            const int client = L.plan->tok[a][c < n_act ? c : 0];
            xrows[c] = L.xmode == 0 ? client : a * kMoeMaxClients + c;
            yrows[c] = a * kMoeMaxClients + c;
            srows[c] = client;
        }
    } else {
        const uint32_t T = L.total_tiles, G = gridDim.x;
        t0 = uint32_t(uint64_t(T) * blockIdx.x / G);
        t1 = uint32_t(uint64_t(T) * (blockIdx.x + 1) / G);
        if (threadIdx.x < NC) {
            xrows[threadIdx.x] = threadIdx.x;
            yrows[threadIdx.x] = threadIdx.x;
            srows[threadIdx.x] = L.c0 + threadIdx.x;
        }
    }
    const uint32_t nt = t1 - t0, NS = uint32_t(L.slots);
    const uint32_t slot_bytes = L.tile_bytes * (DUAL ? 2u : 1u);
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsumers) {
        // ---- producer: the weights of this CTA's tiles, in order ----
        if (lane == 0) {
            for (uint32_t i = 0; i < nt; i++) {
                const uint32_t s = i % NS;
                if (i >= NS && !mbar_wait(&empty[s], ((i / NS) - 1) & 1)) {
                    flag(L.status, 1);
                    break;
                }
                const uint32_t g = t0 + i;
                const GemvJob& J = pick(L, g);
                const size_t off = size_t(g - J.tile_begin) * L.tile_bytes;
                mbar_expect_tx(&full[s], slot_bytes);
                bulk_g2s(ring + size_t(s) * slot_bytes, J.a + off, L.tile_bytes, &full[s]);
                if (DUAL) bulk_g2s(ring + size_t(s) * slot_bytes + L.tile_bytes, J.b + off, L.tile_bytes, &full[s]);
                if (i + 1 == NS || i + 1 == nt) pdl_trigger();
            }
            if (nt == 0) pdl_trigger();
        }
        return;
    }

    // ---- consumers ----
    constexpr int CT = kConsumers * 32;
    const int ctid = threadIdx.x;
    pdl_wait();  // activations (and norm partials) come from the previous kernel
    const uint32_t U = L.cols >> 5;
    const uint32_t xbase = NS * slot_bytes;
    const uint32_t cstride = U * 128;
    const uint32_t sbase = xbase + NC * cstride, sstride = (L.cols >> 4) * 4;
    // raw activations into shared memory while the norm partials are summed
    // (16 lanes per client, fixed-order tree), then normalise in place
    const uint32_t k4 = L.cols >> 2;
    float ssum = 0.f;
    const int sc_c = ctid >> 4, sc_j = ctid & 15;
    if (L.gain && sc_c < NC)
        for (int p = sc_j; p < L.sumsq_parts; p += 16) ssum += L.sumsq[p * 8 + srows[sc_c]];
    for (uint32_t idx = ctid; idx < NC * k4; idx += CT) {
        const uint32_t c = idx / k4, col = 4 * (idx % k4);
        *reinterpret_cast<float4*>(ring + xbase + c * cstride + xoff(col >> 5, (col & 31) >> 2)) =
            int(c) < n_act ? ldx4(L.x + size_t(xrows[c]) * L.x_stride + col) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // the residual rows this CTA will add to (EPI_ADD), loaded with x
    const bool aux_pre = nt * kTileRows * NC <= uint32_t(kAuxPrefetch);
    if (aux_pre)
        for (uint32_t idx = ctid; idx < nt * kTileRows * NC; idx += CT) {
            const uint32_t i = idx / (kTileRows * NC), e = (idx / NC) % kTileRows, c = idx % NC;
            const GemvJob& J = pick(L, t0 + i);
            const uint32_t row = (t0 + i - J.tile_begin) * kTileRows + e;
            if (J.epi == EPI_ADD && row < J.rows) auxs[idx] = J.aux[size_t(yrows[c]) * J.aux_stride + row];
        }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
    if (L.gain && sc_c < NC && sc_j == 0)
        nscale[sc_c] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssum, float(L.cols)), L.eps)));
    bar_sync(1, CT);
    if (L.gain) {
        for (uint32_t idx = ctid; idx < NC * k4; idx += CT) {
            const uint32_t c = idx / k4, col = 4 * (idx % k4);
            float4* p = reinterpret_cast<float4*>(ring + xbase + c * cstride + xoff(col >> 5, (col & 31) >> 2));
            const float4 v = *p, g = ldx4(L.gain + col);
            const float sc = nscale[c];
            *p = make_float4(__fmul_rn(__fmul_rn(v.x, sc), g.x), __fmul_rn(__fmul_rn(v.y, sc), g.y),
                             __fmul_rn(__fmul_rn(v.z, sc), g.z), __fmul_rn(__fmul_rn(v.w, sc), g.w));
        }
        bar_sync(1, CT);
    }
    if constexpr (kquant) {
        // sums of every 16 consecutive activations, per client
        for (uint32_t idx = ctid; idx < NC * (L.cols >> 4); idx += CT) {
            const uint32_t c = idx / (L.cols >> 4), h = idx % (L.cols >> 4), u = h >> 1;
            const uint8_t* xc = ring + xbase + c * cstride;
            float sum = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float4 v = *reinterpret_cast<const float4*>(xc + xoff(u, (h & 1) * 4 + k));
                sum += (v.x + v.y) + (v.z + v.w);
            }
            *reinterpret_cast<float*>(ring + sbase + c * sstride + h * 4) = sum;
        }
        bar_sync(1, CT);
    }
    XIn<NC> X;
    X.xs = saddr(ring) + xbase;
    X.cstride = cstride;
    X.ss = saddr(ring) + sbase;
    X.sstride = sstride;
    float sqacc[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) sqacc[c] = 0.f;
    const uint32_t ring_s = saddr(ring);
    const int grp = warp / kGroupWarps, gw = warp % kGroupWarps;
    uint32_t buf = 0;
    for (uint32_t i = 0; i < nt; i++) {
        const uint32_t s = i % NS;
        if (!mbar_wait(&full[s], (i / NS) & 1)) {
            flag(L.status, 2);
            break;
        }
        const uint32_t g = t0 + i;
        const GemvJob& J = pick(L, g);
        const uint32_t tile = g - J.tile_begin;
        const uint32_t tbase = ring_s + s * slot_bytes + (DUAL && grp ? L.tile_bytes : 0);
#pragma unroll 1
        for (int pass = 0; pass < PASSES; pass++) {
            uint32_t rows[VR];
#pragma unroll
            for (int v = 0; v < VR; v++) rows[v] = DUAL ? uint32_t(pass * VR + v) : uint32_t(grp + 2 * v);
            float acc[VR][NC];
            zero(acc);
#pragma unroll 1
            for (uint32_t u = uint32_t(gw) * 32 + lane; u < U; u += kGroupWarps * 32)
                unit_dot<ENC, NC, VR>(tbase, rows, u, L, X, acc);
#pragma unroll
            for (int v = 0; v < VR; v++)
#pragma unroll
                for (int c = 0; c < NC; c++) acc[v][c] = warp_sum(acc[v][c]);
            if (lane == 0)
#pragma unroll
                for (int v = 0; v < VR; v++)
#pragma unroll
                    for (int c = 0; c < NC; c++) part[buf][warp][v][c] = acc[v][c];
            if (pass + 1 == PASSES) {  // this warp is done reading the slot
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            bar_sync(1, CT);
            // one warp finishes the rows; the others go on (partials are double-buffered)
            if (uint32_t(warp) == (i * PASSES + pass) % kConsumers) {
#pragma unroll
                for (int e = 0; e < (DUAL ? VR : 2 * VR); e++) {
                    // DUAL: row pass*VR+e from groups 0 (gate) and 1 (up);
                    // single: row e = g + 2v of group g = e % 2, v = e / 2
                    const int gsel = DUAL ? 0 : (e & 1), v = DUAL ? e : (e >> 1);
                    const uint32_t grow = tile * kTileRows + (DUAL ? uint32_t(pass * VR + e) : uint32_t(e));
                    const uint32_t row = grow - rbase;
                    if (grow >= J.rows || row >= rlim) continue;
#pragma unroll
                    for (int c = 0; c < NC; c++) {
                        float a = 0.f, b = 0.f;
#pragma unroll
                        for (int w = 0; w < kGroupWarps; w++) {
                            a += part[buf][gsel * kGroupWarps + w][v][c];
                            if (DUAL) b += part[buf][kGroupWarps + w][v][c];
                        }
                        float r = a;
                        if constexpr (DUAL) r = silu_mul(a, b);
                        if (lane == ((e * NC + c) & 31) && c < n_act) {
                            if (J.epi == EPI_ADD) {
                                const uint32_t e2 = DUAL ? uint32_t(pass * VR + e) : uint32_t(e);
                                r = (aux_pre ? auxs[(i * kTileRows + e2) * NC + c] : J.aux[size_t(yrows[c]) * J.aux_stride + row]) + r;
                            }
                            J.y[size_t(yrows[c]) * J.y_stride + row] = r;
                            sqacc[c] = fmaf(r, r, sqacc[c]);
                        }
                    }
                }
            }
            buf ^= 1;
        }
    }
    if (L.sumsq_out) {
        // per-CTA sum of squares of the rows written, reduced in a fixed order
#pragma unroll
        for (int c = 0; c < NC; c++) sqacc[c] = warp_sum(sqacc[c]);
        if (lane == 0)
#pragma unroll
            for (int c = 0; c < NC; c++) sqw[warp][c] = sqacc[c];
        bar_sync(1, CT);
        if (ctid < NC) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumers; w++) t += sqw[w][ctid];
            L.sumsq_out[blockIdx.x * 8 + L.c0 + ctid] = t;
        }
    }
}

template <int ENC, int NC, bool DUAL>
cudaError_t configure(int* occ, size_t smem) {
    auto kern = gemv_stream<ENC, NC, DUAL>;
    static unsigned configured = 0;  // bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemMax));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     int(cudaSharedmemCarveoutMaxShared));
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    if (occ) return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, kern, kThreads, smem);
    return cudaSuccess;
}

template <int ENC, int NC, bool DUAL>
cudaError_t launch_t(const GemvLaunch& L, int grid, size_t smem, cudaStream_t s, bool pdl) {
    cudaError_t e = configure<ENC, NC, DUAL>(nullptr, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_stream<ENC, NC, DUAL>, L);
}

// All instantiations for one block type (compiled in gemv_<type>.cu).
template <int ENC>
cudaError_t launch_enc(const GemvLaunch& L, bool dual, int grid, size_t smem, cudaStream_t s, bool pdl) {
#define SPM_NC(n) \
    case n: return dual ? launch_t<ENC, n, true>(L, grid, smem, s, pdl) : launch_t<ENC, n, false>(L, grid, smem, s, pdl);
    switch (L.n) {
        SPM_NC(1) SPM_NC(2) SPM_NC(3) SPM_NC(4) SPM_NC(5) SPM_NC(6) SPM_NC(7) SPM_NC(8)
        default: return cudaErrorInvalidValue;
    }
#undef SPM_NC
}

// Resident CTAs per SM of the kernel a launch would use.
template <int ENC>
int occupancy_enc(const GemvLaunch& L, bool dual, size_t smem) {
    int occ = 0;
    cudaError_t e = cudaErrorInvalidValue;
#define SPM_NC(n) \
    case n: e = dual ? configure<ENC, n, true>(&occ, smem) : configure<ENC, n, false>(&occ, smem); break;
    switch (L.n) {
        SPM_NC(1) SPM_NC(2) SPM_NC(3) SPM_NC(4) SPM_NC(5) SPM_NC(6) SPM_NC(7) SPM_NC(8)
        default: break;
    }
#undef SPM_NC
    return e == cudaSuccess && occ > 0 ? occ : 1;
}

}  // namespace gemv
}  // namespace spm
