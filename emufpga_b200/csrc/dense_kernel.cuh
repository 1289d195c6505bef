// The dense .spm streamed GEMV kernel (see dense.cu for the contract).
#pragma once
#include <cstdint>

#ifndef SPM_DENSE_PREFETCH
#define SPM_DENSE_PREFETCH(p) asm volatile("prefetch.global.L1 [%0];" ::"l"(p))
#endif

namespace spm {

struct DenseArgs {
    const void* w;     // column-major, element (r, c) at c * rows_pad + r (f32 or bf16 bits)
    const float* x;    // positions x cols
    float* y;          // positions x rows
    uint64_t rows_pad;
    uint32_t rows, cols;
    int32_t positions;
};

namespace {

constexpr int kDenseThreads = 128;

template <bool BF16>
__device__ __forceinline__ float dense_weight(const void* w, uint64_t at) {
    if constexpr (BF16)
        return __uint_as_float(uint32_t(__ldg(static_cast<const uint16_t*>(w) + at)) << 16);
    else
        return __ldg(static_cast<const float*>(w) + at);
}

// One thread owns one row and PPT positions; for each of them it runs the
// reference's chain acc = fma(w[c], x[p][c], acc) over the columns in order.
template <int PPT, bool BF16>
__global__ void __launch_bounds__(kDenseThreads) dense_streamed_kernel(const DenseArgs a) {
    const uint64_t t = uint64_t(blockIdx.x) * kDenseThreads + threadIdx.x;
    const uint64_t row = t % a.rows_pad;
    const uint64_t p0 = t / a.rows_pad * PPT;
    if (row >= a.rows || p0 >= uint64_t(a.positions)) return;
    const int np = min(PPT, a.positions - int(p0));
    // positions past the last one (a partial block) repeat its loads; their
    // results are not stored
    const float* xb[PPT];
    float acc[PPT];
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
        xb[k] = a.x + uint64_t(min(int(p0) + k, a.positions - 1)) * a.cols;
        acc[k] = 0.0f;
    }
    // Columns go 16 at a time; the next 16 weights are loaded before these
    // are used, and each block of 16 activations before any is used.  Loads
    // of columns past the end are clamped to the last column and not applied.
    const uint64_t last = a.cols ? a.cols - 1 : 0;
    float wn[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) wn[j] = a.cols ? dense_weight<BF16>(a.w, min(uint64_t(j), last) * a.rows_pad + row) : 0.f;
    for (uint64_t c0 = 0; c0 < a.cols; c0 += 16) {
        float wv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) wv[j] = wn[j];
        if (c0 + 16 < a.cols) {
#pragma unroll
            for (int j = 0; j < 16; ++j) wn[j] = dense_weight<BF16>(a.w, min(c0 + 16 + j, last) * a.rows_pad + row);
        }
        if ((c0 & 31) == 0) {
            const uint64_t cp = min(c0 + 64, last);
#pragma unroll
            for (int k = 0; k < PPT; ++k) SPM_DENSE_PREFETCH(xb[k] + cp);
        }
        float xv[PPT][16];
#pragma unroll
        for (int k = 0; k < PPT; ++k)
#pragma unroll
            for (int j = 0; j < 16; ++j) xv[k][j] = __ldg(xb[k] + min(c0 + j, last));
        if (c0 + 16 <= a.cols) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
#pragma unroll
                for (int k = 0; k < PPT; ++k) acc[k] = __fmaf_rn(wv[j], xv[k][j], acc[k]);
        } else {
            const int n = int(a.cols - c0);  // the same for the whole warp
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (j < n) {
#pragma unroll
                    for (int k = 0; k < PPT; ++k) acc[k] = __fmaf_rn(wv[j], xv[k][j], acc[k]);
                }
        }
    }
#pragma unroll
    for (int k = 0; k < PPT; ++k)
        if (k < np) a.y[(p0 + k) * a.rows + row] = acc[k];
}

}  // namespace
}  // namespace spm
