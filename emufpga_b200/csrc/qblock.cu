// Q-profile .spm streams (Encoding::Q8_0, Q6K, Q5K) on the device: the
// reference's block consumers q6_operation (spm-granite-moe/src/
// layout.rs:208-242) and stream_matrix (gemma_smoke.rs:201-236).
//
// Their product is out[p][row] = fma(w, x[p][col], out[p][row]) for every
// value of every block in source row-major order (value k is W[k / cols]
// [k % cols]), each block decoded by spm-gguf's decoders.  The kernel
// (qblock_kernel.cuh) keeps that chain per (row, position) and decodes each
// value with the same products in the same order, so results are
// bit-identical.  It is the parity form of these profiles: the fast decode
// GEMV for the same blocks is the GGUF path (gemv_stream), which sums in a
// different order.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <memory>

#include "abi.h"
#include "chain.h"
#include "chain_launch.h"

namespace spm {
namespace {

template <int PPT, int ENC>
cudaError_t launch_q(const QBlockArgs& a, cudaStream_t stream) {
    const uint64_t threads = a.rows_pad * uint64_t((a.positions + PPT - 1) / PPT);
    const uint64_t blocks = (threads + kQBlockThreads - 1) / kQBlockThreads;
    if (blocks > 0x7FFFFFFFull) return cudaErrorInvalidConfiguration;
    qblock_chain_kernel<PPT, ENC><<<unsigned(blocks), kQBlockThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

template <int ENC>
cudaError_t launch_q_ppt(int ppt, const QBlockArgs& a, cudaStream_t stream) {
    switch (ppt) {
        case 4: return launch_q<4, ENC>(a, stream);
        case 2: return launch_q<2, ENC>(a, stream);
        default: return launch_q<1, ENC>(a, stream);
    }
}

}  // namespace

cudaError_t launch_qblock_chain(const QBlockArgs& a, uint8_t encoding, int sms, cudaStream_t stream) {
    const int ppt = chains_per_thread(a.rows_pad, a.positions, sms, 4);
    switch (encoding) {
        case SPM_ENC_Q8_0: return launch_q_ppt<SPM_ENC_Q8_0>(ppt, a, stream);
        case SPM_ENC_Q6K: return launch_q_ppt<SPM_ENC_Q6K>(ppt, a, stream);
        case SPM_ENC_Q5K: return launch_q_ppt<SPM_ENC_Q5K>(ppt, a, stream);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace spm

using namespace spm;

struct spm_qblocks {
    uint32_t rows = 0, cols = 0, group_size = 0, encoding = 0;
    uint64_t groups = 0, payload_bytes = 0, device_bytes = 0;
    int device = 0, sms = 148;
    uint8_t* mem = nullptr;
    ~spm_qblocks() { if (mem) cudaFree(mem); }
};

spm_status spm_qblocks_upload(const uint8_t* spm, uint64_t len, int32_t index, int device, spm_qblocks** out) {
    return guarded([&] {
        if (!out) fail(SPM_E_ARG, "null output");
        if (index < 0) fail(SPM_E_ARG, "stream index out of range");
        const PackedStream h = pack_qblocks(spm, len, uint32_t(index));
        const StreamPlan& pl = h.plan;
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) fail(SPM_E_NO_DEVICE, "no CUDA device is visible");
        std::unique_ptr<spm_qblocks> t(new spm_qblocks());
        t->rows = pl.rows;
        t->cols = pl.cols;
        t->group_size = pl.group_size;
        t->encoding = pl.encoding;
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

spm_status spm_qblocks_free(spm_qblocks* t) {
    return guarded([&] { delete t; });
}

spm_status spm_qblocks_describe(const spm_qblocks* t, spm_dense_info* out) {
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

spm_status spm_qblocks_gemv(const spm_qblocks* t, const float* x_dev, uint64_t x_len, int32_t positions,
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
        QBlockArgs a{};
        a.blocks = t->mem;
        a.x = x_dev;
        a.y = y_dev;
        a.rows_pad = (uint64_t(t->rows) + 31) / 32 * 32;
        a.rows = t->rows;
        a.cols = t->cols;
        a.positions = positions;
        const cudaError_t e = launch_qblock_chain(a, uint8_t(t->encoding), t->sms,
                                                  static_cast<cudaStream_t>(cuda_stream));
        if (e == cudaErrorInvalidConfiguration) fail(SPM_E_ARG, "too many rows x positions for one launch");
        CUDA_OK(e);
    });
}
