// Shared by the kernels that keep one sequential f32 chain per output (the
// ternary GEMV and the dense .spm streamed GEMV): how many chains a thread
// carries.  More per thread share the weight loads; fewer spread the chains
// over more warps.  Take the most that still leaves about two warps per
// scheduler.
#pragma once
#include <cstdint>

namespace spm {

inline int chains_per_thread(uint64_t rows_pad, int chains, int sms, int most = 8) {
    const uint64_t target = 8ull * uint64_t(sms);
    for (int L : {8, 4, 2})
        if (L <= most && chains >= L && rows_pad / 32 * uint64_t((chains + L - 1) / L) >= target) return L;
    return 1;
}

}  // namespace spm
