// Dense .spm streams (Encoding::F32 / Bf16) on the device: spm_linear::streamed
// (spm-linear/src/stream.rs:31-125 with resident.rs:124-137).
//
// The reference's product is y[p][r] = fma(W[r][c], x[p][c], y[p][r]) over
// c ascending, starting from +0 -- one fused multiply-add per weight and
// position, in stream order.  The kernel (dense_kernel.cuh) keeps exactly that
// chain per (row, position), so results are bit-identical; a split over
// columns or a tree reduction would round differently.  The stream is packed
// column-major with rows padded to 32, so at every column a warp of 32 rows
// reads one contiguous 128-byte (f32) or 64-byte (bf16) segment, and the
// activation of that column is a warp-uniform load.  Each chain is `cols`
// dependent FMAs, which bounds a launch from below.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <memory>

#include "abi.h"
#include "chain.h"
#include "chain_launch.h"

namespace spm {
namespace {

template <int PPT, bool BF16>
cudaError_t launch_dense(const DenseArgs& a, cudaStream_t stream) {
    const uint64_t threads = a.rows_pad * uint64_t((a.positions + PPT - 1) / PPT);
    const uint64_t blocks = (threads + kDenseThreads - 1) / kDenseThreads;
    if (blocks > 0x7FFFFFFFull) return cudaErrorInvalidConfiguration;
    dense_streamed_kernel<PPT, BF16><<<unsigned(blocks), kDenseThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

template <bool BF16>
cudaError_t launch_dense_ppt(int ppt, const DenseArgs& a, cudaStream_t stream) {
    switch (ppt) {
        case 4: return launch_dense<4, BF16>(a, stream);
        case 2: return launch_dense<2, BF16>(a, stream);
        default: return launch_dense<1, BF16>(a, stream);
    }
}

}  // namespace

cudaError_t launch_dense_streamed(const DenseArgs& a, bool bf16, int sms, cudaStream_t stream) {
    // four positions per thread at most: eight would need more than 255
    // registers for the hoisted activations
    const int ppt = chains_per_thread(a.rows_pad, a.positions, sms, 4);
    return bf16 ? launch_dense_ppt<true>(ppt, a, stream) : launch_dense_ppt<false>(ppt, a, stream);
}

}  // namespace spm

using namespace spm;

struct spm_dense {
    uint32_t rows = 0, cols = 0, group_size = 0, encoding = 0;
    uint64_t rows_pad = 0, groups = 0, payload_bytes = 0, device_bytes = 0;
    int device = 0, sms = 148;
    void* mem = nullptr;
    ~spm_dense() { if (mem) cudaFree(mem); }
};

spm_status spm_dense_upload(const uint8_t* spm, uint64_t len, int32_t index, int device, spm_dense** out) {
    return guarded([&] {
        if (!out) fail(SPM_E_ARG, "null output");
        if (index < 0) fail(SPM_E_ARG, "stream index out of range");
        const PackedStream h = pack_dense(spm, len, uint32_t(index));
        const StreamPlan& pl = h.plan;
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) fail(SPM_E_NO_DEVICE, "no CUDA device is visible");
        std::unique_ptr<spm_dense> t(new spm_dense());
        t->rows = pl.rows;
        t->cols = pl.cols;
        t->group_size = pl.group_size;
        t->encoding = pl.encoding;
        t->rows_pad = pl.rows_pad;
        t->groups = pl.groups;
        t->payload_bytes = pl.payload_bytes;
        t->device = device;
        CUDA_OK(cudaSetDevice(device));
        CUDA_OK(cudaDeviceGetAttribute(&t->sms, cudaDevAttrMultiProcessorCount, device));
        t->device_bytes = std::max<uint64_t>(pl.bytes, 256);
        CUDA_OK(cudaMalloc(&t->mem, t->device_bytes));
        if (pl.bytes) CUDA_OK(cudaMemcpy(t->mem, h.data.data(), pl.bytes, cudaMemcpyHostToDevice));
        *out = t.release();
    });
}

spm_status spm_dense_free(spm_dense* t) {
    return guarded([&] { delete t; });
}

spm_status spm_dense_describe(const spm_dense* t, spm_dense_info* out) {
    return guarded([&] {
        if (!t || !out) fail(SPM_E_ARG, "null argument");
        *out = spm_dense_info{};
        out->rows = t->rows;
        out->cols = t->cols;
        out->group_size = t->group_size;
        out->encoding = t->encoding;
        out->groups = t->groups;
        out->payload_bytes = t->payload_bytes;
        out->device_bytes = t->device_bytes;
    });
}

spm_status spm_dense_streamed(const spm_dense* t, const float* x_dev, uint64_t x_len, int32_t positions,
                              float* y_dev, void* cuda_stream) {
    return guarded([&] {
        if (!t) fail(SPM_E_ARG, "null matrix");
        if (positions < 0) fail(SPM_E_ARG, "negative position count");
        const uint64_t need = uint64_t(positions) * t->cols;
        if (x_len < need) {
            char msg[96];
            std::snprintf(msg, sizeof msg, "need %llu activations, got %llu", (unsigned long long)need,
                          (unsigned long long)x_len);
            fail(SPM_E_ACTIVATION_LEN, msg);
        }
        if (positions == 0 || t->rows == 0) return;
        if (!y_dev || (t->cols && !x_dev)) fail(SPM_E_ARG, "null activation or output pointer");
        CUDA_OK(cudaSetDevice(t->device));
        DenseArgs a{};
        a.w = t->mem;
        a.x = x_dev;
        a.y = y_dev;
        a.rows_pad = t->rows_pad;
        a.rows = t->rows;
        a.cols = t->cols;
        a.positions = positions;
        const cudaError_t e = launch_dense_streamed(a, t->encoding == SPM_ENC_BF16, t->sms,
                                                    static_cast<cudaStream_t>(cuda_stream));
        if (e == cudaErrorInvalidConfiguration) fail(SPM_E_ARG, "too many rows x positions for one launch");
        CUDA_OK(e);
    });
}
