// The ternary GEMV kernel (see ternary.cu for the contract and the layout).
// Kept apart from the launch code so that the kernel body is one unit: its
// thread-to-(row, lanes) mapping, the group walk and the clamps that keep
// padding loads in bounds.
#pragma once
#include <cstdint>

namespace spm {
namespace {

constexpr int kTernaryThreads = 128;

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

    const uint32_t* wp = a.codes + row;
    uint32_t w = a.col_words ? __ldg(wp) : 0u;
    for (uint64_t cw = 0; cw < a.col_words; ++cw) {
        const uint32_t next = cw + 1 < a.col_words ? __ldg(wp + (cw + 1) * a.rows_pad) : 0u;
        const uint32_t c0 = uint32_t(cw * 16);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            // padding columns hold code 0; clamping keeps their loads in bounds
            const uint32_t c = min(c0 + uint32_t(j), a.cols - 1);
            const float s = __ldg(a.scales + min(g, a.last_group));
            const uint32_t code = (w >> (2 * j)) & 3u;
#pragma unroll
            for (int k = 0; k < LPT; ++k) {
                const float term = __fmul_rn(s, __ldg(xb[k] + c));
                if (code & 1u) acc[k] = (code & 2u) ? __fsub_rn(acc[k], term) : __fadd_rn(acc[k], term);
            }
            if (rem >= wrap) {
                rem -= wrap;
                g += a.q + 1;
            } else {
                rem += a.r;
                g += a.q;
            }
        }
        w = next;
    }
#pragma unroll
    for (int k = 0; k < LPT; ++k)
        if (k < nl) a.y[(l0 + k) * a.rows + row] = acc[k];
}

}  // namespace
}  // namespace spm
