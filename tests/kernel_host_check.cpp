// TEST INFRASTRUCTURE ONLY -- never part of libspmgpu.so.
//
// Compiles the bodies of the sequential-chain kernels (ternary_kernel.cuh,
// dense_kernel.cuh, qblock_kernel.cuh) for the host, with the CUDA builtins
// they use replaced by their IEEE host equivalents, and runs every thread of
// a launch one after another over exact-size buffers.  tests/
// test_kernel_host_check.py compares the results with the oracle bit for bit
// and builds this file under AddressSanitizer where available, so the
// kernels' thread mapping, group walk, clamps and order of operations are
// checked without a GPU.  It says nothing about the device's behaviour beyond
// that; the GPU tests do.
//
//   kernel_host_check ternary <spm> <x.bin> <lanes> <x_cols> <sms> <y.bin>
//   kernel_host_check dense   <spm> <index> <x.bin> <positions> <sms> <y.bin>
//   kernel_host_check qblock  <spm> <x.bin> <positions> <sms> <y.bin>
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

using std::min;
struct HostDim3 {
    unsigned x, y, z;
};
static HostDim3 blockIdx, threadIdx;
#define __global__
#define __device__
#define __forceinline__ inline
#define __launch_bounds__(n)
template <class T>
static inline T __ldg(const T* p) { return *p; }
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fsub_rn(float a, float b) { return a - b; }
static inline float __fmaf_rn(float a, float b, float c) { return std::fmaf(a, b, c); }
static inline float __uint_as_float(uint32_t v) { float f; std::memcpy(&f, &v, 4); return f; }
static inline float __int_as_float(uint32_t v) { float f; std::memcpy(&f, &v, 4); return f; }
static inline float __int_as_float(int v) { float f; std::memcpy(&f, &v, 4); return f; }
static inline int __float_as_int(float f) { int v; std::memcpy(&v, &f, 4); return v; }
// prefetch hints become reads, so an out-of-bounds address is caught
static volatile float g_sink;
#define SPM_TERNARY_PREFETCH(p) (g_sink = *(const float*)(p))
#define SPM_DENSE_PREFETCH(p) (g_sink = *(const float*)(p))

#include "../emufpga_b200/csrc/chain.h"
#include "../emufpga_b200/csrc/common.h"
#include "../emufpga_b200/csrc/dense_kernel.cuh"
#include "../emufpga_b200/csrc/qblock_kernel.cuh"
#include "../emufpga_b200/csrc/ternary_kernel.cuh"

using namespace spm;

static std::vector<uint8_t> slurp(const char* path) {
    std::ifstream f(path, std::ios::binary);
    return std::vector<uint8_t>((std::istreambuf_iterator<char>(f)), {});
}

template <class T>
static T* exact(const void* src, size_t n) {
    T* p = static_cast<T*>(std::malloc(n ? n * sizeof(T) : 1));
    if (n) std::memcpy(p, src, n * sizeof(T));
    return p;
}

template <class Args, class Kernel>
static void run_grid(uint64_t rows_pad, int chains, int per_thread, const Args& a, Kernel kernel, int threads) {
    const uint64_t total = rows_pad * uint64_t((chains + per_thread - 1) / per_thread);
    const uint64_t blocks = (total + threads - 1) / threads;
    for (uint64_t b = 0; b < blocks; ++b)
        for (int t = 0; t < threads; ++t) {
            blockIdx.x = unsigned(b);
            threadIdx.x = unsigned(t);
            kernel(a);
        }
}

static int ternary(char** argv) {
    const std::vector<uint8_t> spm = slurp(argv[0]);
    const std::vector<uint8_t> xb = slurp(argv[1]);
    const int lanes = std::atoi(argv[2]), sms = std::atoi(argv[4]);
    const uint64_t x_cols = std::strtoull(argv[3], nullptr, 10);
    const PackedStream ps = pack_ternary(spm.data(), spm.size(), 0);
    const StreamPlan& h = ps.plan;
    if (xb.size() / 4 != size_t(lanes) * x_cols) return 4;
    uint32_t* codes = exact<uint32_t>(ps.data.data(), h.col_words * h.rows_pad);
    float* scales = exact<float>(ps.data.data() + h.scale_off, h.groups);
    float* x = exact<float>(xb.data(), xb.size() / 4);
    float* y = static_cast<float*>(std::malloc(std::max<size_t>(1, size_t(lanes) * h.rows * 4)));
    TernaryArgs a{};
    a.codes = codes, a.scales = scales, a.x = x, a.y = y;
    a.rows_pad = h.rows_pad, a.col_words = h.col_words, a.x_cols = x_cols;
    a.rows = h.rows, a.cols = h.cols, a.group = h.group_size;
    a.q = h.rows / h.group_size, a.r = h.rows % h.group_size;
    a.last_group = h.groups ? uint32_t(h.groups - 1) : 0u, a.lanes = lanes;
    const int L = chains_per_thread(h.rows_pad, lanes, sms);
    if (lanes > 0 && h.rows > 0) {
        if (L == 8) run_grid(h.rows_pad, lanes, 8, a, ternary_gemv_kernel<8>, kTernaryThreads);
        else if (L == 4) run_grid(h.rows_pad, lanes, 4, a, ternary_gemv_kernel<4>, kTernaryThreads);
        else if (L == 2) run_grid(h.rows_pad, lanes, 2, a, ternary_gemv_kernel<2>, kTernaryThreads);
        else run_grid(h.rows_pad, lanes, 1, a, ternary_gemv_kernel<1>, kTernaryThreads);
    }
    std::ofstream(argv[5], std::ios::binary).write(reinterpret_cast<char*>(y), size_t(lanes) * h.rows * 4);
    std::printf("%d %llu\n", L, (unsigned long long)ps.reserved_codes);
    std::free(codes), std::free(scales), std::free(x), std::free(y);
    return 0;
}

template <bool B>
static void dense_ppt(int p, uint64_t rows_pad, int positions, const DenseArgs& a) {
    if (p == 4) run_grid(rows_pad, positions, 4, a, dense_streamed_kernel<4, B>, kDenseThreads);
    else if (p == 2) run_grid(rows_pad, positions, 2, a, dense_streamed_kernel<2, B>, kDenseThreads);
    else run_grid(rows_pad, positions, 1, a, dense_streamed_kernel<1, B>, kDenseThreads);
}

static int dense(char** argv) {
    const std::vector<uint8_t> spm = slurp(argv[0]);
    const int index = std::atoi(argv[1]);
    const std::vector<uint8_t> xb = slurp(argv[2]);
    const int positions = std::atoi(argv[3]), sms = std::atoi(argv[4]);
    const PackedStream ps = pack_dense(spm.data(), spm.size(), uint32_t(index));
    const StreamPlan& h = ps.plan;
    if (xb.size() / 4 != size_t(positions) * h.cols) return 4;
    uint8_t* w = exact<uint8_t>(ps.data.data(), ps.data.size());
    float* x = exact<float>(xb.data(), xb.size() / 4);
    float* y = static_cast<float*>(std::malloc(std::max<size_t>(1, size_t(positions) * h.rows * 4)));
    DenseArgs a{};
    a.w = w, a.x = x, a.y = y, a.rows_pad = h.rows_pad, a.rows = h.rows, a.cols = h.cols, a.positions = positions;
    const int ppt = chains_per_thread(h.rows_pad, positions, sms, 4);
    if (positions > 0 && h.rows > 0) {
        if (h.encoding == SPM_ENC_BF16) dense_ppt<true>(ppt, h.rows_pad, positions, a);
        else dense_ppt<false>(ppt, h.rows_pad, positions, a);
    }
    std::ofstream(argv[5], std::ios::binary).write(reinterpret_cast<char*>(y), size_t(positions) * h.rows * 4);
    std::printf("%d\n", ppt);
    std::free(w), std::free(x), std::free(y);
    return 0;
}

template <int E>
static void qblock_ppt(int p, uint64_t rows_pad, int positions, const QBlockArgs& a) {
    if (p == 4) run_grid(rows_pad, positions, 4, a, qblock_chain_kernel<4, E>, kQBlockThreads);
    else if (p == 2) run_grid(rows_pad, positions, 2, a, qblock_chain_kernel<2, E>, kQBlockThreads);
    else run_grid(rows_pad, positions, 1, a, qblock_chain_kernel<1, E>, kQBlockThreads);
}

static int qblock(char** argv) {
    const std::vector<uint8_t> spm = slurp(argv[0]);
    const std::vector<uint8_t> xb = slurp(argv[1]);
    const int positions = std::atoi(argv[2]), sms = std::atoi(argv[3]);
    const PackedStream ps = pack_qblocks(spm.data(), spm.size(), 0);
    const StreamPlan& h = ps.plan;
    if (xb.size() / 4 != size_t(positions) * h.cols) return 4;
    uint8_t* blk = exact<uint8_t>(ps.data.data(), ps.data.size());
    float* x = exact<float>(xb.data(), xb.size() / 4);
    float* y = static_cast<float*>(std::malloc(std::max<size_t>(1, size_t(positions) * h.rows * 4)));
    QBlockArgs a{};
    a.blocks = blk, a.x = x, a.y = y, a.rows_pad = h.rows_pad, a.rows = h.rows, a.cols = h.cols;
    a.positions = positions;
    const int ppt = chains_per_thread(h.rows_pad, positions, sms, 4);
    if (positions > 0 && h.rows > 0) {
        if (h.encoding == SPM_ENC_Q8_0) qblock_ppt<6>(ppt, h.rows_pad, positions, a);
        else if (h.encoding == SPM_ENC_Q6K) qblock_ppt<4>(ppt, h.rows_pad, positions, a);
        else qblock_ppt<5>(ppt, h.rows_pad, positions, a);
    }
    std::ofstream(argv[4], std::ios::binary).write(reinterpret_cast<char*>(y), size_t(positions) * h.rows * 4);
    std::printf("%d\n", ppt);
    std::free(blk), std::free(x), std::free(y);
    return 0;
}

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const std::string mode = argv[1];
    try {
        if (mode == "ternary" && argc == 8) return ternary(argv + 2);
        if (mode == "dense" && argc == 8) return dense(argv + 2);
        if (mode == "qblock" && argc == 7) return qblock(argv + 2);
    } catch (const Error& e) {
        std::fprintf(stderr, "refused: %d %s\n", e.code, e.msg.c_str());
        return 3;
    }
    return 2;
}
