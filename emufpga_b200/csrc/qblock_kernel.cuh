// GGML blocks of a .spm Q-profile stream (Q8_0, Q6_K, Q5_K), decoded one
// value at a time and applied in the reference's order: the FMA-chain GEMV of
// spm-granite-moe/src/layout.rs:208-242 (q6_operation) and
// gemma_smoke.rs:201-236 (stream_matrix).  See qblock.cu for the contract.
//
// The per-value decoders restate spm-gguf/src/tensor.rs (Q8_0 :193-210,
// Q6_K :103-139, Q5_K :144-188) with the same products in the same order, each
// rounded once: Q8_0 d*q; Q6_K (d*sc)*(q-32); Q5_K (d*sc)*q - dmin*m.  The
// helpers below are the IEEE-rounded intrinsics on the device and plain
// arithmetic on the host, where this header is also compiled to check the
// kernel body against the CPU oracle.
#pragma once
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define SPM_QB_HD __host__ __device__ __forceinline__
#else
#define SPM_QB_HD inline
#endif

namespace spm {

struct QBlockArgs {
    const uint8_t* blocks;  // the stream's blocks in source row-major order
    const float* x;         // positions x cols
    float* y;               // positions x rows
    uint64_t rows_pad;      // rows rounded up to 32 (thread mapping)
    uint32_t rows, cols;
    int32_t positions;
};

SPM_QB_HD float qb_float(uint32_t v) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(v);
#else
    float f;
    std::memcpy(&f, &v, 4);
    return f;
#endif
}

SPM_QB_HD float qb_mul(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}

SPM_QB_HD float qb_sub(float a, float b) {
#if defined(__CUDA_ARCH__)
    return __fsub_rn(a, b);
#else
    return a - b;
#endif
}

SPM_QB_HD float qb_fma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
    return __fmaf_rn(a, b, c);
#else
    return __builtin_fmaf(a, b, c);
#endif
}

SPM_QB_HD uint32_t qb_clz(uint32_t v) {
#if defined(__CUDA_ARCH__)
    return uint32_t(__clz(int(v)));
#else
    return uint32_t(__builtin_clz(v));
#endif
}

// IEEE half -> float, exact for every input including subnormals
// (spm-gguf/src/tensor.rs:82-98).
SPM_QB_HD float qb_half(uint16_t bits) {
    const uint32_t sign = uint32_t(bits & 0x8000u) << 16;
    const uint32_t exp = (bits >> 10) & 0x1fu, frac = bits & 0x3ffu;
    uint32_t out;
    if (exp == 0 && frac == 0) {
        out = sign;
    } else if (exp == 0) {
        const uint32_t shift = qb_clz(frac) - 21u;
        out = sign | ((113u - shift) << 23) | (((frac << shift) & 0x3ffu) << 13);
    } else if (exp == 31) {
        out = sign | 0x7f800000u | (frac << 13);
    } else {
        out = sign | ((exp + 112u) << 23) | (frac << 13);
    }
    return qb_float(out);
}

SPM_QB_HD uint16_t qb_le16(const uint8_t* p) { return uint16_t(p[0] | (p[1] << 8)); }

// Value i of a Q8_0 block (34 bytes: f16 d, 32 int8).
SPM_QB_HD float q8_0_value(const uint8_t* b, float d, uint32_t i) { return qb_mul(d, float(int8_t(b[2 + i]))); }

// Value i of a Q6_K block (210 bytes: ql[128], qh[64], int8 sc[16], f16 d).
SPM_QB_HD float q6_k_value(const uint8_t* b, float d, uint32_t i) {
    const uint32_t half = i >> 7, lane = (i >> 5) & 3, l = i & 31;
    const uint8_t ql = b[half * 64 + l + ((lane & 1) << 5)];
    const uint32_t nib = (lane & 2) ? uint32_t(ql >> 4) : uint32_t(ql & 15);
    const uint32_t hi = (uint32_t(b[128 + half * 32 + l]) >> (2 * lane)) & 3u;
    const float sc = float(int8_t(b[192 + half * 8 + (l >> 4) + lane * 2]));
    return qb_mul(qb_mul(d, sc), float(nib | (hi << 4)) - 32.0f);
}

// Value i of a Q5_K block (176 bytes: f16 d, f16 dmin, scales[12], qh[32],
// qs[128]); sub-block j = i / 32 takes its 6-bit scale and min from
// scale_min_q5 (tensor.rs:179-188).
SPM_QB_HD float q5_k_value(const uint8_t* b, float d, float dmin, uint32_t i) {
    const uint32_t j = i >> 5, group = i >> 6, lane = i & 31;
    const uint8_t* s = b + 4;
    uint32_t sc, m;
    if (j < 4) {
        sc = s[j] & 63u;
        m = s[j + 4] & 63u;
    } else {
        sc = (s[j + 4] & 0x0fu) | ((uint32_t(s[j - 4]) >> 6) << 4);
        m = (uint32_t(s[j + 4]) >> 4) | ((uint32_t(s[j]) >> 6) << 4);
    }
    const uint8_t packed = b[48 + group * 32 + lane];
    const uint32_t low = (j & 1) ? uint32_t(packed >> 4) : uint32_t(packed & 15);
    const uint32_t quant = low + (((uint32_t(b[16 + lane]) >> j) & 1u) ? 16u : 0u);
    return qb_sub(qb_mul(qb_mul(d, float(sc)), float(quant)), qb_mul(dmin, float(m)));
}

// Profiles by .spm encoding code: values and bytes per block.
template <int ENC> struct QBlock;
template <> struct QBlock<6> { static constexpr uint32_t values = 32, bytes = 34; };    // Q8_0
template <> struct QBlock<4> { static constexpr uint32_t values = 256, bytes = 210; };  // Q6_K
template <> struct QBlock<5> { static constexpr uint32_t values = 256, bytes = 176; };  // Q5_K

namespace {

constexpr int kQBlockThreads = 128;

// One thread owns one row and PPT positions and walks the row's values in
// stream order (position k = row * cols + col, so a row may start or end
// inside a block), decoding each value once and applying it to every
// position with a fused multiply-add, as the reference does.
template <int PPT, int ENC>
__global__ void __launch_bounds__(kQBlockThreads) qblock_chain_kernel(const QBlockArgs a) {
    constexpr uint32_t BV = QBlock<ENC>::values, BB = QBlock<ENC>::bytes;
    const uint64_t t = uint64_t(blockIdx.x) * kQBlockThreads + threadIdx.x;
    const uint64_t row = t % a.rows_pad;
    const uint64_t p0 = t / a.rows_pad * PPT;
    if (row >= a.rows || p0 >= uint64_t(a.positions)) return;
    const int np = min(PPT, a.positions - int(p0));
    const float* xb[PPT];
    float acc[PPT];
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        xb[k] = a.x + uint64_t(min(int(p0) + k, a.positions - 1)) * a.cols;
        acc[k] = 0.0f;
    }
    const uint64_t k0 = row * a.cols, k1 = k0 + a.cols;
    uint64_t k = k0;
    while (k < k1) {
        const uint64_t blk = k / BV;
        const uint8_t* b = a.blocks + blk * BB;
        const uint32_t first = uint32_t(k - blk * BV);
        const uint32_t last = uint32_t(min(uint64_t(BV), k1 - blk * BV));
        float d, dmin = 0.0f;
        if constexpr (ENC == 4)
            d = qb_half(qb_le16(b + 208));
        else
            d = qb_half(qb_le16(b));
        if constexpr (ENC == 5) dmin = qb_half(qb_le16(b + 2));
        for (uint32_t i = first; i < last; ++i) {
            float w;
            if constexpr (ENC == 6)
                w = q8_0_value(b, d, i);
            else if constexpr (ENC == 4)
                w = q6_k_value(b, d, i);
            else
                w = q5_k_value(b, d, dmin, i);
            const uint64_t col = blk * BV + i - k0;
#pragma unroll
            for (int p = 0; p < PPT; ++p) acc[p] = qb_fma(w, xb[p][col], acc[p]);
        }
        k = blk * BV + last;
    }
#pragma unroll
    for (int p = 0; p < PPT; ++p)
        if (p < np) a.y[(p0 + p) * a.rows + row] = acc[p];
}

}  // namespace
}  // namespace spm
