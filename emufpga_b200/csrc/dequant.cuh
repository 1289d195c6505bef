// Exact dequantization of one 32-weight unit of a packed matrix row, shared by
// the parity hook, the embedding gather and the tensor-core GEMM's producers.
#pragma once
#include "device.cuh"

namespace spm {
namespace dev {

// ---------------------------------------------------------------- decode ----
// Exact dequantization of unit u of a packed row, in the reference's
// arithmetic order (spm-gguf/src/tensor.rs:103-210; ggml Q2_K):
// Q8_0 d*q;  Q6_K (d*sc)*(q-32);  Q5_K (d*sc)*q - dmin*m;  Q2_K (d*sc)*q - dmin*m.
__device__ __forceinline__ void dequant_unit(uint32_t dtype, const uint8_t* tile, const Packed& p, uint32_t rt, uint32_t u,
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
            const uint8_t* m = tile + p.plane[3] + (size_t(rt) * B + (u >> 3)) * 4;
            const uint8_t* qs = tile + unit * 16;
            const uint8_t* qhp = tile + p.plane[1] + unit * 4;
            const uint32_t qh = qhp[0] | (qhp[1] << 8) | (qhp[2] << 16) | (uint32_t(qhp[3]) << 24);
            const float d = h2f(m[0] | (m[1] << 8)), dmin = h2f(m[2] | (m[3] << 8));
            const int sc = tile[p.plane[2] + unit * 2], mn = tile[p.plane[2] + unit * 2 + 1];
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


}  // namespace dev
}  // namespace spm
