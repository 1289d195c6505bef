// Ternary GEMV over a .spm stream (Encoding::Ternary2F32I32): the device form
// of spm_gemv_ref::run_gemv (spm-gemv-ref/src/gemv.rs:39-126,
// datapath.rs:19-55, spm-accum/src/bank.rs:56-66).
//
// The reference's result is defined by its order of operations: for every
// output row and lane, an f32 accumulator starts at +0 and, for the row's
// weights in stream order (columns ascending), adds or subtracts
// scale(group) * x[col] -- the product rounded once, then the sum rounded
// once -- and is left untouched by zero codes.  f32 addition is not
// associative, so a split over columns or a reduction tree would change the
// low bits; this kernel keeps one sequential chain per (row, lane) and
// spreads the work over rows and lanes instead.  Rounding is pinned with
// __fmul_rn / __fadd_rn, which the compiler never contracts; a subtraction
// is the addition of the negated product, which IEEE arithmetic defines to
// be the same operation.
//
// Layout in HBM (packed on the host by pack_ternary): for every 16 columns one
// 32-bit word per row, rows padded to a multiple of 32, so a warp of 32 rows
// reads 128 contiguous bytes per 16 columns; the scales follow.  Threads of a
// warp share their lanes, so activation loads are warp-uniform broadcasts.
//
// Roofline: HBM is not the bound.  Each (row, lane) chain is `cols` dependent
// adds, so a launch takes at least cols x the add latency, and the issue cost
// (a handful of instructions per weight and lane) spreads over rows x lanes
// chains.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <memory>

#include "abi.h"
#include "chain.h"
#include "chain_launch.h"

namespace spm {
namespace {

template <int LPT>
cudaError_t launch(const TernaryArgs& a, cudaStream_t stream) {
    const uint64_t threads = a.rows_pad * uint64_t((a.lanes + LPT - 1) / LPT);
    const uint64_t blocks = (threads + kTernaryThreads - 1) / kTernaryThreads;
    if (blocks > 0x7FFFFFFFull) return cudaErrorInvalidConfiguration;
    ternary_gemv_kernel<LPT><<<unsigned(blocks), kTernaryThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_ternary_gemv(const TernaryArgs& a, int sms, cudaStream_t stream) {
    switch (chains_per_thread(a.rows_pad, a.lanes, sms)) {
        case 8: return launch<8>(a, stream);
        case 4: return launch<4>(a, stream);
        case 2: return launch<2>(a, stream);
        default: return launch<1>(a, stream);
    }
}

}  // namespace spm

using namespace spm;

struct spm_ternary {
    uint32_t rows = 0, cols = 0, group_size = 0;
    uint64_t groups = 0, col_words = 0, rows_pad = 0;
    uint64_t payload_bytes = 0, reserved_codes = 0, device_bytes = 0;
    int device = 0, sms = 148;
    uint8_t* mem = nullptr;
    const uint32_t* codes = nullptr;
    const float* scales = nullptr;
    ~spm_ternary() { if (mem) cudaFree(mem); }
};

spm_status spm_ternary_upload(const uint8_t* spm, uint64_t len, int32_t index, int device, spm_ternary** out) {
    return guarded([&] {
        if (!out) fail(SPM_E_ARG, "null output");
        if (index < 0) fail(SPM_E_ARG, "stream index out of range");
        const PackedStream h = pack_ternary(spm, len, uint32_t(index));
        const StreamPlan& pl = h.plan;
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) fail(SPM_E_NO_DEVICE, "no CUDA device is visible");
        std::unique_ptr<spm_ternary> t(new spm_ternary());
        t->rows = pl.rows;
        t->cols = pl.cols;
        t->group_size = pl.group_size;
        t->groups = pl.groups;
        t->col_words = pl.col_words;
        t->rows_pad = pl.rows_pad;
        t->payload_bytes = pl.payload_bytes;
        t->reserved_codes = h.reserved_codes;
        t->device = device;
        CUDA_OK(cudaSetDevice(device));
        CUDA_OK(cudaDeviceGetAttribute(&t->sms, cudaDevAttrMultiProcessorCount, device));
        t->device_bytes = std::max<uint64_t>(pl.bytes, 256);
        CUDA_OK(cudaMalloc(&t->mem, t->device_bytes));
        if (pl.bytes) CUDA_OK(cudaMemcpy(t->mem, h.data.data(), pl.bytes, cudaMemcpyHostToDevice));
        t->codes = reinterpret_cast<const uint32_t*>(t->mem);
        t->scales = reinterpret_cast<const float*>(t->mem + pl.scale_off);
        *out = t.release();
    });
}

spm_status spm_ternary_free(spm_ternary* t) {
    return guarded([&] { delete t; });
}

spm_status spm_ternary_describe(const spm_ternary* t, spm_ternary_info* out) {
    return guarded([&] {
        if (!t || !out) fail(SPM_E_ARG, "null argument");
        *out = spm_ternary_info{};
        out->rows = t->rows;
        out->cols = t->cols;
        out->group_size = t->group_size;
        out->groups = t->groups;
        out->payload_bytes = t->payload_bytes;
        out->reserved_codes = t->reserved_codes;
        out->device_bytes = t->device_bytes;
    });
}

spm_status spm_ternary_gemv(const spm_ternary* t, const float* x_dev, int32_t lanes, uint64_t x_cols, float* y_dev,
                            void* cuda_stream) {
    return guarded([&] {
        if (!t) fail(SPM_E_ARG, "null matrix");
        if (lanes < 0) fail(SPM_E_ARG, "negative lane count");
        if (x_cols < t->cols) {
            char msg[96];
            std::snprintf(msg, sizeof msg, "need %u activations per lane, got %llu", t->cols,
                          (unsigned long long)x_cols);
            fail(SPM_E_ACTIVATION_LEN, msg);
        }
        if (lanes == 0 || t->rows == 0) return;
        if (!y_dev || (t->cols && !x_dev)) fail(SPM_E_ARG, "null activation or output pointer");
        CUDA_OK(cudaSetDevice(t->device));
        TernaryArgs a{};
        a.codes = t->codes;
        a.scales = t->scales;
        a.x = x_dev;
        a.y = y_dev;
        a.rows_pad = t->rows_pad;
        a.col_words = t->col_words;
        a.x_cols = x_cols;
        a.rows = t->rows;
        a.cols = t->cols;
        a.group = t->group_size;
        a.q = t->rows / t->group_size;
        a.r = t->rows % t->group_size;
        a.last_group = t->groups ? uint32_t(t->groups - 1) : 0u;
        a.lanes = lanes;
        const cudaError_t e = launch_ternary_gemv(a, t->sms, static_cast<cudaStream_t>(cuda_stream));
        if (e == cudaErrorInvalidConfiguration) fail(SPM_E_ARG, "too many rows x lanes for one launch");
        CUDA_OK(e);
    });
}
