// sm_100a kernels of the decode token loop.
//
// The GEMV is the hot path: it streams one packed weight matrix (host_pack.cpp
// layout) from HBM exactly once and applies every weight to all N clients'
// activations while it is in registers -- the reference's "one weight,
// every position" schedule (spm-linear/src/resident.rs:120-137) mapped onto
// warps.  Each thread owns one 32-weight unit per pass; codes become floats
// with a byte permute into the mantissa of 2^23 (exact), the 16- or
// 32-weight sub-block sums are taken against the activations, and the block
// scale is applied once per sub-block:
//     sum_c w_c x_c = (d*sc) * sum_c q_c x_c  [- (dmin*m) * sum_c x_c]
// which is the reference dot product regrouped (the weights themselves are
// decoded bit-exactly by the dequant kernel below; only the order of the
// fp32 additions differs from the reference FMA chain).
#include <cuda_fp16.h>

#include "kernels.h"

namespace spm {
namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ uint4 ldw4(const uint8_t* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}
__device__ __forceinline__ uint2 ldw2(const uint8_t* p) {
    uint2 r;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldw1(const uint8_t* p) {
    uint32_t r;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldu16(const uint8_t* p) {
    unsigned short r;
    asm("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ float4 ldx4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// Exact half -> float.
__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)(bits & 0xffff))); }

// 2^23 + (byte b of w), exactly; subtracting a constant recovers the code.
template <int B>
__device__ __forceinline__ float bytef(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | B));
}

template <int T>
__device__ __forceinline__ uint32_t word(const uint4& v) {
    return T == 0 ? v.x : T == 1 ? v.y : T == 2 ? v.z : v.w;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

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

// Row `rt` of the tile that virtual row v reads (paired gate/up launches read
// matrix b for v >= RR).
template <int RR>
__device__ __forceinline__ const uint8_t* vtile(const uint8_t* ta, const uint8_t* tb, int v) {
    return v < RR ? ta : tb;
}

// ---------------------------------------------------------------- Q8_0 ----
template <int NC, int VR, int RR>
__device__ __forceinline__ void unit_q8_0(const uint8_t* ta, const uint8_t* tb, int r0, uint32_t u,
                                          const GemvLaunch& L, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5;
    uint4 q0[VR], q1[VR];
    float d[VR];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint8_t* t = vtile<RR>(ta, tb, v);
        const size_t unit = size_t(r0 + v % RR) * U + u;
        q0[v] = ldw4(t + unit * 32);
        q1[v] = ldw4(t + unit * 32 + 16);
        d[v] = h2f(ldu16(t + L.plane1 + unit * 2));
    }
    const float* xb = L.x + 32 * size_t(u);
    float s[VR][NC];
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) s[v][c] = 0.f;
#pragma unroll
    for (int t = 0; t < 8; t++) {
        float4 x[NC];
#pragma unroll
        for (int c = 0; c < NC; c++) x[c] = ldx4(xb + size_t(c) * L.x_stride + 4 * t);
#pragma unroll
        for (int v = 0; v < VR; v++) {
            uint32_t w = (t < 4 ? (t == 0 ? q0[v].x : t == 1 ? q0[v].y : t == 2 ? q0[v].z : q0[v].w)
                                : (t == 4 ? q1[v].x : t == 5 ? q1[v].y : t == 6 ? q1[v].z : q1[v].w)) ^
                         0x80808080u;
            const float k = 8388736.0f;  // 2^23 + 128: (u8 ^ 0x80) - 128 == int8
            dot4<NC>(s[v], bytef<0>(w) - k, bytef<1>(w) - k, bytef<2>(w) - k, bytef<3>(w) - k, x);
        }
    }
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) acc[v][c] = fmaf(d[v], s[v][c], acc[v][c]);
}

// ---------------------------------------------------------------- Q6_K ----
template <int NC, int VR, int RR>
__device__ __forceinline__ void unit_q6_k(const uint8_t* ta, const uint8_t* tb, int r0, uint32_t u,
                                          const GemvLaunch& L, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5, B = L.cols >> 8;
    uint4 ql[VR];
    uint2 qh[VR];
    float dsa[VR], dsb[VR];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint8_t* t = vtile<RR>(ta, tb, v);
        const size_t row = size_t(r0 + v % RR), unit = row * U + u;
        ql[v] = ldw4(t + unit * 16);
        qh[v] = ldw2(t + L.plane1 + unit * 8);
        const uint32_t sc = ldu16(t + L.plane2 + unit * 2);
        const float d = h2f(ldu16(t + L.plane3 + (row * B + (u >> 3)) * 2));
        dsa[v] = d * float(int8_t(sc & 0xff));
        dsb[v] = d * float(int8_t(sc >> 8));
    }
    const float* xb = L.x + 32 * size_t(u);
    float sa[VR][NC], sb[VR][NC];
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) sa[v][c] = sb[v][c] = 0.f;
#pragma unroll
    for (int t = 0; t < 4; t++) {
        float4 xa[NC], xc[NC];
#pragma unroll
        for (int c = 0; c < NC; c++) {
            xa[c] = ldx4(xb + size_t(c) * L.x_stride + 4 * t);
            xc[c] = ldx4(xb + size_t(c) * L.x_stride + 16 + 4 * t);
        }
#pragma unroll
        for (int v = 0; v < VR; v++) {
            const uint32_t w = t == 0 ? ql[v].x : t == 1 ? ql[v].y : t == 2 ? ql[v].z : ql[v].w;
            const uint32_t ha = (t < 2 ? qh[v].x << (4 - 2 * t) : qh[v].x >> (2 * t - 4)) & 0x30303030u;
            const uint32_t hb = (t < 2 ? qh[v].y << (4 - 2 * t) : qh[v].y >> (2 * t - 4)) & 0x30303030u;
            const uint32_t qa = (w & 0x0F0F0F0Fu) | ha;
            const uint32_t qb = ((w >> 4) & 0x0F0F0F0Fu) | hb;
            const float k = 8388640.0f;  // 2^23 + 32
            dot4<NC>(sa[v], bytef<0>(qa) - k, bytef<1>(qa) - k, bytef<2>(qa) - k, bytef<3>(qa) - k, xa);
            dot4<NC>(sb[v], bytef<0>(qb) - k, bytef<1>(qb) - k, bytef<2>(qb) - k, bytef<3>(qb) - k, xc);
        }
    }
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) {
            acc[v][c] = fmaf(dsa[v], sa[v][c], acc[v][c]);
            acc[v][c] = fmaf(dsb[v], sb[v][c], acc[v][c]);
        }
}

// ---------------------------------------------------------------- Q5_K ----
__device__ __forceinline__ uint32_t sbyte(const uint4& m, int k) {  // scales byte k (0..11)
    const uint32_t w = k < 4 ? m.y : k < 8 ? m.z : m.w;
    return (w >> (8 * (k & 3))) & 0xffu;
}

template <int NC, int VR, int RR>
__device__ __forceinline__ void unit_q5_k(const uint8_t* ta, const uint8_t* tb, int r0, uint32_t u,
                                          const GemvLaunch& L, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5, B = L.cols >> 8;
    const int j = int(u & 7);
    uint4 qs[VR];
    uint32_t qh[VR];
    float ds[VR], dm[VR];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint8_t* t = vtile<RR>(ta, tb, v);
        const size_t row = size_t(r0 + v % RR), unit = row * U + u;
        const uint4 m = ldw4(t + (row * B + (u >> 3)) * 16);
        qs[v] = ldw4(t + L.plane1 + unit * 16);
        qh[v] = ldw1(t + L.plane2 + unit * 4);
        uint32_t sc, mn;
        if (j < 4) {
            sc = sbyte(m, j) & 63;
            mn = sbyte(m, j + 4) & 63;
        } else {
            sc = (sbyte(m, j + 4) & 15) | ((sbyte(m, j - 4) >> 6) << 4);
            mn = (sbyte(m, j + 4) >> 4) | ((sbyte(m, j) >> 6) << 4);
        }
        ds[v] = h2f(m.x) * float(sc);
        dm[v] = h2f(m.x >> 16) * float(mn);
    }
    const float* xb = L.x + 32 * size_t(u);
    float s[VR][NC], xs[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) xs[c] = 0.f;
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) s[v][c] = 0.f;
#pragma unroll
    for (int t = 0; t < 4; t++) {
        float4 xa[NC], xc[NC];
#pragma unroll
        for (int c = 0; c < NC; c++) {
            xa[c] = ldx4(xb + size_t(c) * L.x_stride + 4 * t);
            xc[c] = ldx4(xb + size_t(c) * L.x_stride + 16 + 4 * t);
            xs[c] += (xa[c].x + xa[c].y) + (xa[c].z + xa[c].w) + ((xc[c].x + xc[c].y) + (xc[c].z + xc[c].w));
        }
#pragma unroll
        for (int v = 0; v < VR; v++) {
            const uint32_t w = t == 0 ? qs[v].x : t == 1 ? qs[v].y : t == 2 ? qs[v].z : qs[v].w;
            const uint32_t spa = (((qh[v] >> (4 * t)) & 0xfu) * 0x02040810u) & 0x10101010u;
            const uint32_t spb = (((qh[v] >> (16 + 4 * t)) & 0xfu) * 0x02040810u) & 0x10101010u;
            const uint32_t qa = (w & 0x0F0F0F0Fu) | spa;
            const uint32_t qb = ((w >> 4) & 0x0F0F0F0Fu) | spb;
            const float k = 8388608.0f;
            dot4<NC>(s[v], bytef<0>(qa) - k, bytef<1>(qa) - k, bytef<2>(qa) - k, bytef<3>(qa) - k, xa);
            dot4<NC>(s[v], bytef<0>(qb) - k, bytef<1>(qb) - k, bytef<2>(qb) - k, bytef<3>(qb) - k, xc);
        }
    }
#pragma unroll
    for (int v = 0; v < VR; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) acc[v][c] = fmaf(-dm[v], xs[c], fmaf(ds[v], s[v][c], acc[v][c]));
}

// ---------------------------------------------------------------- Q2_K ----
template <int NC, int VR, int RR>
__device__ __forceinline__ void unit_q2_k(const uint8_t* ta, const uint8_t* tb, int r0, uint32_t u,
                                          const GemvLaunch& L, float (&acc)[VR][NC]) {
    const uint32_t U = L.cols >> 5, B = L.cols >> 8;
    uint2 qs[VR];
    float dl[VR][2], ml[VR][2];
#pragma unroll
    for (int v = 0; v < VR; v++) {
        const uint8_t* t = vtile<RR>(ta, tb, v);
        const size_t row = size_t(r0 + v % RR), unit = row * U + u;
        qs[v] = ldw2(t + unit * 8);
        const uint32_t sc = ldu16(t + L.plane1 + unit * 2);
        const uint32_t dd = ldw1(t + L.plane2 + (row * B + (u >> 3)) * 4);
        const float d = h2f(dd), dmin = h2f(dd >> 16);
        dl[v][0] = d * float(sc & 15);
        ml[v][0] = dmin * float((sc >> 4) & 15);
        dl[v][1] = d * float((sc >> 8) & 15);
        ml[v][1] = dmin * float((sc >> 12) & 15);
    }
    const float* xb = L.x + 32 * size_t(u);
#pragma unroll
    for (int h = 0; h < 2; h++) {
        float s[VR][NC], xs[NC];
#pragma unroll
        for (int c = 0; c < NC; c++) xs[c] = 0.f;
#pragma unroll
        for (int v = 0; v < VR; v++)
#pragma unroll
            for (int c = 0; c < NC; c++) s[v][c] = 0.f;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            float4 x[NC];
#pragma unroll
            for (int c = 0; c < NC; c++) {
                x[c] = ldx4(xb + size_t(c) * L.x_stride + 16 * h + 4 * t);
                xs[c] += (x[c].x + x[c].y) + (x[c].z + x[c].w);
            }
#pragma unroll
            for (int v = 0; v < VR; v++) {
                const uint32_t q = ((h == 0 ? qs[v].x : qs[v].y) >> (2 * t)) & 0x03030303u;
                const float k = 8388608.0f;
                dot4<NC>(s[v], bytef<0>(q) - k, bytef<1>(q) - k, bytef<2>(q) - k, bytef<3>(q) - k, x);
            }
        }
#pragma unroll
        for (int v = 0; v < VR; v++)
#pragma unroll
            for (int c = 0; c < NC; c++) acc[v][c] = fmaf(-ml[v][h], xs[c], fmaf(dl[v][h], s[v][c], acc[v][c]));
    }
}

// ----------------------------------------------------------------- F32 ----
template <int NC, int VR, int RR>
__device__ __forceinline__ void unit_f32(const uint8_t* ta, const uint8_t* tb, int r0, uint32_t u,
                                         const GemvLaunch& L, float (&acc)[VR][NC]) {
    const float* xb = L.x + 32 * size_t(u);
#pragma unroll
    for (int t = 0; t < 8; t++) {
        float4 x[NC];
#pragma unroll
        for (int c = 0; c < NC; c++) x[c] = ldx4(xb + size_t(c) * L.x_stride + 4 * t);
#pragma unroll
        for (int v = 0; v < VR; v++) {
            const uint8_t* tl = vtile<RR>(ta, tb, v);
            const uint4 w = ldw4(tl + (size_t(r0 + v % RR) * L.cols + 32 * size_t(u) + 4 * t) * 4);
            dot4<NC>(acc[v], __uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z),
                     __uint_as_float(w.w), x);
        }
    }
}

template <int ENC, int NC, int VR, int RR>
__device__ __forceinline__ void unit_dot(const uint8_t* ta, const uint8_t* tb, int r0, uint32_t u,
                                         const GemvLaunch& L, float (&acc)[VR][NC]) {
    if constexpr (ENC == SPM_Q8_0) unit_q8_0<NC, VR, RR>(ta, tb, r0, u, L, acc);
    else if constexpr (ENC == SPM_Q6_K) unit_q6_k<NC, VR, RR>(ta, tb, r0, u, L, acc);
    else if constexpr (ENC == SPM_Q5_K) unit_q5_k<NC, VR, RR>(ta, tb, r0, u, L, acc);
    else if constexpr (ENC == SPM_Q2_K) unit_q2_k<NC, VR, RR>(ta, tb, r0, u, L, acc);
    else unit_f32<NC, VR, RR>(ta, tb, r0, u, L, acc);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return __fdiv_rn(g, 1.0f + expf(-g)) * u; }

// A CTA of 8 warps takes 8/KS tiles at a time; KS warps share a tile, each
// summing every KS-th run of 32 units, and their partial sums are added in a
// fixed order (deterministic).
template <int ENC, int NC, int VR, bool DUAL, int KS>
__global__ void __launch_bounds__(kWarps * 32) gemv_kernel(const __grid_constant__ GemvLaunch L) {
    constexpr int RR = DUAL ? VR / 2 : VR;
    constexpr int TPC = kWarps / KS;  // tiles per CTA pass
    __shared__ float part[kWarps][VR][NC];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slot = warp / KS, ks = warp % KS;
    const uint32_t U = L.cols >> 5;
    for (uint32_t base = blockIdx.x * TPC; base < L.total_tiles; base += gridDim.x * TPC) {
        const uint32_t g = base + slot;
        const bool active = g < L.total_tiles;
        GemvJob J = L.job[0];
        if (L.njobs > 1 && g >= L.job[1].tile_begin) J = L.job[1];
        if (L.njobs > 2 && g >= L.job[2].tile_begin) J = L.job[2];
        if (L.njobs > 3 && g >= L.job[3].tile_begin) J = L.job[3];
        const uint32_t tile = g - J.tile_begin;
        const uint8_t* ta = J.a + size_t(tile) * L.tile_bytes;
        const uint8_t* tb = DUAL ? J.b + size_t(tile) * L.tile_bytes : nullptr;
#pragma unroll 1
        for (int r0 = 0; r0 < kTileRows; r0 += RR) {
            float acc[VR][NC];
#pragma unroll
            for (int v = 0; v < VR; v++)
#pragma unroll
                for (int c = 0; c < NC; c++) acc[v][c] = 0.f;
            if (active) {
#pragma unroll 1
                for (uint32_t u = uint32_t(ks) * 32 + lane; u < U; u += 32 * KS)
                    unit_dot<ENC, NC, VR, RR>(ta, tb, r0, u, L, acc);
            }
#pragma unroll
            for (int v = 0; v < VR; v++)
#pragma unroll
                for (int c = 0; c < NC; c++) acc[v][c] = warp_sum(acc[v][c]);
            if constexpr (KS > 1) {
                if (lane == 0) {
#pragma unroll
                    for (int v = 0; v < VR; v++)
#pragma unroll
                        for (int c = 0; c < NC; c++) part[warp][v][c] = acc[v][c];
                }
                __syncthreads();
                if (ks == 0) {
#pragma unroll
                    for (int v = 0; v < VR; v++)
#pragma unroll
                        for (int c = 0; c < NC; c++) {
                            float t = part[warp][v][c];
#pragma unroll
                            for (int k = 1; k < KS; k++) t += part[warp + k][v][c];
                            acc[v][c] = t;
                        }
                }
                __syncthreads();
            }
            if (active && ks == 0) {
#pragma unroll
                for (int v = 0; v < RR; v++) {
                    const uint32_t row = tile * kTileRows + r0 + v;
                    if (row >= J.rows) continue;
#pragma unroll
                    for (int c = 0; c < NC; c++) {
                        if (lane != ((v * NC + c) & 31)) continue;
                        float r = acc[v][c];
                        if constexpr (DUAL) r = silu_mul(acc[v][c], acc[v + RR][c]);
                        if (J.epi == EPI_ADD) r = J.aux[size_t(c) * J.aux_stride + row] + r;
                        J.y[size_t(c) * J.y_stride + row] = r;
                    }
                }
            }
        }
    }
}

template <int ENC, int NC, int VR, bool DUAL>
cudaError_t launch_ks(const GemvLaunch& L, int sms, cudaStream_t s) {
    // Enough warps in flight to cover HBM latency: split K when tiles are few.
    const uint32_t U = L.cols >> 5;
    int ks = 1;
    while (ks < 8 && uint64_t(L.total_tiles) * ks < uint64_t(sms) * 48 && U >= 64u * ks) ks *= 2;
    const uint32_t tpc = kWarps / ks;
    uint32_t grid = (L.total_tiles + tpc - 1) / tpc;
    const uint32_t cap = uint32_t(sms) * 16;
    if (grid > cap) grid = cap;
    if (grid == 0) return cudaSuccess;
    switch (ks) {
        case 1: gemv_kernel<ENC, NC, VR, DUAL, 1><<<grid, kWarps * 32, 0, s>>>(L); break;
        case 2: gemv_kernel<ENC, NC, VR, DUAL, 2><<<grid, kWarps * 32, 0, s>>>(L); break;
        case 4: gemv_kernel<ENC, NC, VR, DUAL, 4><<<grid, kWarps * 32, 0, s>>>(L); break;
        default: gemv_kernel<ENC, NC, VR, DUAL, 8><<<grid, kWarps * 32, 0, s>>>(L); break;
    }
    return cudaGetLastError();
}

template <int ENC, int NC>
cudaError_t launch_nc(const GemvLaunch& L, bool dual, int sms, cudaStream_t s) {
    constexpr int VR = NC <= 4 ? 4 : 2;
    if (dual) return launch_ks<ENC, NC, VR, true>(L, sms, s);
    return launch_ks<ENC, NC, VR, false>(L, sms, s);
}

template <int ENC>
cudaError_t launch_enc(const GemvLaunch& L, bool dual, int sms, cudaStream_t s) {
    switch (L.n) {
        case 1: return launch_nc<ENC, 1>(L, dual, sms, s);
        case 2: return launch_nc<ENC, 2>(L, dual, sms, s);
        case 3: return launch_nc<ENC, 3>(L, dual, sms, s);
        case 4: return launch_nc<ENC, 4>(L, dual, sms, s);
        case 5: return launch_nc<ENC, 5>(L, dual, sms, s);
        case 6: return launch_nc<ENC, 6>(L, dual, sms, s);
        case 7: return launch_nc<ENC, 7>(L, dual, sms, s);
        case 8: return launch_nc<ENC, 8>(L, dual, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

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

__global__ void embed_kernel(uint32_t dtype, const uint8_t* tiles, const Packed p, const uint32_t* tokens,
                             float* out) {
    const uint32_t U = uint32_t(p.cols >> 5);
    const uint64_t r = tokens[blockIdx.x];
    for (uint32_t u = threadIdx.x; u < U; u += blockDim.x)
        dequant_unit(dtype, tiles + (r / kTileRows) * p.tile_bytes, p, uint32_t(r % kTileRows), u,
                     out + size_t(blockIdx.x) * p.cols + 32 * size_t(u));
}

// ------------------------------------------------------------ reductions ----
template <int NT>
__device__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    if (threadIdx.x < 32) {
        t = threadIdx.x < NT / 32 ? red[threadIdx.x] : 0.f;
        t = warp_sum(t);
        if (threadIdx.x == 0) red[32] = t;
    }
    __syncthreads();
    t = red[32];
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

// RMSNorm: x * (1/sqrt(mean(x^2) + eps)) * g (spm-smol-ops/src/norm.rs:12-21,
// spm-qwen3-slice/src/math.rs:1-10; both round the same way).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* x, const float* g, float* out, int width, float eps) {
    __shared__ float red[33];
    const float* xr = x + size_t(blockIdx.x) * width;
    float ss = 0.f;
    for (int i = threadIdx.x; i < width; i += 256) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum<256>(ss, red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(width)), eps)));
    for (int i = threadIdx.x; i < width; i += 256)
        out[size_t(blockIdx.x) * width + i] = __fmul_rn(__fmul_rn(xr[i], scale), g[i]);
}

// Greedy selection: largest logit, LAST index among equals
// (spm-batch/examples/serve-demo.rs:74-79, max_by keeps the last maximum).
__global__ void __launch_bounds__(1024) argmax_kernel(const float* logits, int vocab, uint32_t* out) {
    __shared__ float sv[32];
    __shared__ int si[32];
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

__global__ void advance_kernel(int32_t* pos, int n) {
    if (threadIdx.x < n) pos[threadIdx.x] += 1;
}

// ------------------------------------------------------------- attention ----
// One CTA per (kv head, client): QK-norm, RoPE at the client's position from
// the host-computed table, KV append, then each query head of the group
// attends over positions 0..pos (the diagonal included).
//   LLAMA  : spm-kv/src/attend.rs:37-94   (dot*(1/sqrt hd), fma value chain)
//   others : spm-qwen3-slice/src/attention.rs:11-79 (dot/sqrt hd, mul+add values)
constexpr int kAttnThreads = 128;

__device__ __forceinline__ void rope_pair(float& x, float& y, float c, float s, bool llama) {
    if (llama) {  // spm-ops/src/attention.rs:249-251
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
    extern __shared__ float sm[];
    const int kvh = blockIdx.x, i = blockIdx.y;
    const int hd = P.head_dim, group = P.heads / P.kv_heads;
    const int qw = P.heads * hd, kvw = P.kv_heads * hd;
    const bool llama = P.family == SPM_FAMILY_LLAMA;
    float* qs = sm;                   // group * hd
    float* ks = qs + group * hd;      // hd
    float* scores = ks + hd;          // context
    float* red = scores + P.context;  // 33
    const int pos = P.pos[i];
    const float* qg = P.q + size_t(i) * qw + size_t(kvh) * group * hd;
    const float* kg = P.k + size_t(i) * kvw + size_t(kvh) * hd;
    const float* vg = P.v + size_t(i) * kvw + size_t(kvh) * hd;
    for (int t = threadIdx.x; t < group * hd; t += kAttnThreads) qs[t] = qg[t];
    for (int t = threadIdx.x; t < hd; t += kAttnThreads) ks[t] = kg[t];
    __syncthreads();
    // ---- QK-norm ----
    if (P.family == SPM_FAMILY_OLMOE) {
        // Full-width RMSNorm of the whole q and k projections.
        float sq = 0.f, sk = 0.f;
        for (int t = threadIdx.x; t < qw; t += kAttnThreads) sq = fmaf(P.q[size_t(i) * qw + t], P.q[size_t(i) * qw + t], sq);
        for (int t = threadIdx.x; t < kvw; t += kAttnThreads) sk = fmaf(P.k[size_t(i) * kvw + t], P.k[size_t(i) * kvw + t], sk);
        sq = block_sum<kAttnThreads>(sq, red);
        sk = block_sum<kAttnThreads>(sk, red);
        const float scq = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, float(qw)), P.eps)));
        const float sck = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sk, float(kvw)), P.eps)));
        for (int t = threadIdx.x; t < group * hd; t += kAttnThreads)
            qs[t] = __fmul_rn(__fmul_rn(qs[t], scq), P.q_norm[kvh * group * hd + t]);
        for (int t = threadIdx.x; t < hd; t += kAttnThreads)
            ks[t] = __fmul_rn(__fmul_rn(ks[t], sck), P.k_norm[kvh * hd + t]);
        __syncthreads();
    } else if (!llama) {
        // Per-head RMSNorm (spm-qwen3-slice/src/attention.rs:27-34).
        for (int h = 0; h <= group; h++) {
            float* x = h < group ? qs + h * hd : ks;
            const float* g = h < group ? P.q_norm : P.k_norm;
            float ss = 0.f;
            for (int t = threadIdx.x; t < hd; t += kAttnThreads) ss = fmaf(x[t], x[t], ss);
            ss = block_sum<kAttnThreads>(ss, red);
            const float sc = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, float(hd)), P.eps)));
            for (int t = threadIdx.x; t < hd; t += kAttnThreads) x[t] = __fmul_rn(__fmul_rn(x[t], sc), g[t]);
            __syncthreads();
        }
    }
    // ---- RoPE (half-split pairs i, i + hd/2) ----
    const int half = hd / 2;
    const float2* rt = P.rope + size_t(pos) * half;
    for (int t = threadIdx.x; t < (group + 1) * half; t += kAttnThreads) {
        const int h = t / half, j = t % half;
        float* x = h < group ? qs + h * hd : ks;
        const float2 cs = rt[j];
        rope_pair(x[j], x[j + half], cs.x, cs.y, llama);
    }
    __syncthreads();
    // ---- KV append (spm-kv/src/cache.rs:49-58) ----
    const size_t layer_base = (size_t(i) * P.layers + P.layer) * P.context * size_t(kvw) + size_t(kvh) * hd;
    float* kc = P.kcache + layer_base;
    float* vc = P.vcache + layer_base;
    for (int t = threadIdx.x; t < hd; t += kAttnThreads) {
        kc[size_t(pos) * kvw + t] = ks[t];
        vc[size_t(pos) * kvw + t] = vg[t];
    }
    __syncthreads();
    const int positions = pos + 1;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(float(hd)));
    const float denom = __fsqrt_rn(float(hd));
    for (int h = 0; h < group; h++) {
        const float* q = qs + h * hd;
        for (int p = warp; p < positions; p += kAttnThreads / 32) {
            const float* kp = kc + size_t(p) * kvw;
            float d = 0.f;
            for (int t = lane; t < hd; t += 32) d = fmaf(q[t], kp[t], d);
            d = warp_sum(d);
            if (lane == 0) scores[p] = llama ? __fmul_rn(d, scale) : __fdiv_rn(d, denom);
        }
        __syncthreads();
        float mx = -INFINITY;
        for (int p = threadIdx.x; p < positions; p += kAttnThreads) mx = fmaxf(mx, scores[p]);
        mx = block_max<kAttnThreads>(mx, red);
        float tot = 0.f;
        for (int p = threadIdx.x; p < positions; p += kAttnThreads) {
            const float e = expf(scores[p] - mx);
            scores[p] = e;
            tot += e;
        }
        tot = block_sum<kAttnThreads>(tot, red);
        for (int p = threadIdx.x; p < positions; p += kAttnThreads) scores[p] = __fdiv_rn(scores[p], tot);
        __syncthreads();
        float* o = P.out + size_t(i) * qw + (size_t(kvh) * group + h) * hd;
        for (int t = threadIdx.x; t < hd; t += kAttnThreads) {
            float a = 0.f;
            for (int p = 0; p < positions; p++) {
                const float v = vc[size_t(p) * kvw + t];
                a = llama ? __fmaf_rn(scores[p], v, a) : __fadd_rn(a, __fmul_rn(v, scores[p]));
            }
            o[t] = a;
        }
        __syncthreads();
    }
}

}  // namespace

cudaError_t launch_gemv(uint32_t dtype, const GemvLaunch& L, int sms, cudaStream_t s) {
    const bool dual = L.job[0].b != nullptr;
    switch (dtype) {
        case SPM_Q8_0: return launch_enc<SPM_Q8_0>(L, dual, sms, s);
        case SPM_Q6_K: return launch_enc<SPM_Q6_K>(L, dual, sms, s);
        case SPM_Q5_K: return launch_enc<SPM_Q5_K>(L, dual, sms, s);
        case SPM_Q2_K: return launch_enc<SPM_Q2_K>(L, dual, sms, s);
        case SPM_F32: return launch_enc<SPM_F32>(L, dual, sms, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_attention(const AttnParams& P, int n, cudaStream_t s) {
    const int group = P.heads / P.kv_heads;
    const size_t smem = (size_t(group) * P.head_dim + P.head_dim + P.context + 33) * sizeof(float);
    attention_kernel<<<dim3(P.kv_heads, n), kAttnThreads, smem, s>>>(P);
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const float* x, const float* g, float* out, int n, int width, float eps, cudaStream_t s) {
    rmsnorm_kernel<<<n, 256, 0, s>>>(x, g, out, width, eps);
    return cudaGetLastError();
}

cudaError_t launch_embed(uint32_t dtype, const uint8_t* tiles, const Packed& p, const uint32_t* tokens, int n,
                         float* out, cudaStream_t s) {
    embed_kernel<<<n, 128, 0, s>>>(dtype, tiles, p, tokens, out);
    return cudaGetLastError();
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

cudaError_t launch_argmax(const float* logits, int n, int vocab, uint32_t* out, cudaStream_t s) {
    argmax_kernel<<<n, 1024, 0, s>>>(logits, vocab, out);
    return cudaGetLastError();
}

cudaError_t launch_advance(int32_t* pos, int n, cudaStream_t s) {
    advance_kernel<<<1, 32, 0, s>>>(pos, n);
    return cudaGetLastError();
}

}  // namespace spm
