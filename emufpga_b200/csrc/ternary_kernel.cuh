// The ternary GEMV kernel (see ternary.cu for the contract and the layout).
// Kept apart from the launch code so that the kernel body is one unit: its
// thread-to-(row, lanes) mapping, the group walk and the clamps that keep
// padding loads in bounds.
#pragma once
#include <cstdint>

// An L1 prefetch hint for one 128-byte line (a hook so that a host build of
// this kernel body can check the addresses instead).
#ifndef SPM_TERNARY_PREFETCH
#define SPM_TERNARY_PREFETCH(p) asm volatile("prefetch.global.L1 [%0];" ::"l"(p))
#endif

namespace spm {

struct TernaryArgs {
    const uint32_t* codes;
    const float* scales;
    const float* x;
    float* y;
    uint64_t rows_pad, col_words, x_cols;
    uint32_t rows, cols, group;
    uint32_t q, r;        // rows / group, rows % group: one column = q groups + r positions
    uint32_t last_group;  // groups - 1
    int32_t lanes;
};

namespace {

constexpr int kTernaryThreads = 128;
constexpr int kCodeAhead = 4;   // code words in flight per thread (64 columns)
constexpr uint32_t kAhead = 64; // columns between an activation/scale prefetch and its use

template <int LPT>
__global__ void __launch_bounds__(kTernaryThreads) ternary_gemv_kernel(const TernaryArgs a) {
    const uint64_t t = uint64_t(blockIdx.x) * kTernaryThreads + threadIdx.x;
    const uint64_t row = t % a.rows_pad;
    const uint64_t l0 = t / a.rows_pad * LPT;
    if (row >= a.rows || l0 >= uint64_t(a.lanes)) return;
    const int nl = min(LPT, a.lanes - int(l0));
    // lanes past the last one (a partial block) repeat its loads; their
    // results are not stored
    const float* xb[LPT];
    float acc[LPT];
#pragma unroll
    for (int k = 0; k < LPT; ++k) {
        xb[k] = a.x + uint64_t(min(int(l0) + k, a.lanes - 1)) * a.x_cols;
        acc[k] = 0.0f;
    }

    // Group and offset inside it of stream position col * rows + row, for
    // col = 0 here and advanced by `rows` positions per column below.
    uint32_t g = uint32_t(row / a.group);
    uint32_t rem = uint32_t(row % a.group);
    const uint32_t wrap = a.group - a.r;  // rem >= wrap: the step crosses one more group

    // Code words arrive kCodeAhead words before use, shifted through
    // registers; one 128-byte line of every lane's activations and of the
    // scales is prefetched kAhead columns before use, once per 32 columns
    // (addresses clamped into the buffers).  Each word's 16 scales and
    // 16 x LPT activations are loaded before any of them is used.
    const uint32_t* wp = a.codes + row;
    uint32_t ahead[kCodeAhead];
#pragma unroll
    for (int u = 0; u < kCodeAhead; ++u) ahead[u] = uint64_t(u) < a.col_words ? __ldg(wp + u * a.rows_pad) : 0u;
    for (uint64_t cw = 0; cw < a.col_words; ++cw) {
        const uint32_t w = ahead[0];
#pragma unroll
        for (int u = 0; u + 1 < kCodeAhead; ++u) ahead[u] = ahead[u + 1];
        ahead[kCodeAhead - 1] =
            cw + kCodeAhead < a.col_words ? __ldg(wp + (cw + kCodeAhead) * a.rows_pad) : 0u;
        const uint32_t c0 = uint32_t(cw * 16);
        if ((cw & 1) == 0) {
            const uint32_t cp = min(c0 + kAhead, a.cols - 1);
#pragma unroll
            for (int k = 0; k < LPT; ++k) SPM_TERNARY_PREFETCH(xb[k] + cp);
            const uint64_t ga = uint64_t(g) + uint64_t(kAhead) * (uint64_t(a.q) + 1);
            SPM_TERNARY_PREFETCH(a.scales + (ga < a.last_group ? ga : a.last_group));
        }
        float sc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            sc[j] = __ldg(a.scales + min(g, a.last_group));
            if (rem >= wrap) {
                rem -= wrap;
                g += a.q + 1;
            } else {
                rem += a.r;
                g += a.q;
            }
        }
        float xv[LPT][16];
#pragma unroll
        for (int k = 0; k < LPT; ++k)
#pragma unroll
            for (int j = 0; j < 16; ++j)
                // padding columns hold code 0; clamping keeps their loads in bounds
                xv[k][j] = __ldg(xb[k] + min(c0 + uint32_t(j), a.cols - 1));
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            // bit 0 of the code enables the accumulator; bit 1 negates the
            // term, and acc + (-t) is exactly acc - t in IEEE arithmetic
            const bool enable = (w >> (2 * j)) & 1u;
            const uint32_t sign = (w << (30 - 2 * j)) & 0x80000000u;
#pragma unroll
            for (int k = 0; k < LPT; ++k) {
                const float t = __int_as_float(__float_as_int(__fmul_rn(sc[j], xv[k][j])) ^ sign);
                const float sum = __fadd_rn(acc[k], t);
                acc[k] = enable ? sum : acc[k];
            }
        }
    }
#pragma unroll
    for (int k = 0; k < LPT; ++k)
        if (k < nl) a.y[(l0 + k) * a.rows + row] = acc[k];
}

}  // namespace
}  // namespace spm
