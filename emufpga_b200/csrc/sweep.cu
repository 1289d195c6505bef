// Host-to-HBM streaming of a .spm file: the reference's file-backed weight
// stream (spm-stream-file/src/prefetch.rs: a worker reads ahead into a
// bounded buffer; spm-stream-groups/src/groups.rs: streams are consumed in
// file order and rewound between sweeps) with the device as the consumer.
//
// Every stream is packed once into pinned host memory, in the device layout
// of its kernel (dense.cu / ternary.cu).  The device holds only a ring of
// `device_bytes`: each spm_sweep_next runs the next stream out of the ring,
// and the streams after it are copied into the ring on a copy stream while it
// computes, as far ahead as the ring allows.  A region of the ring is reused
// only after the kernel that read it was enqueued, and the copy stream waits
// for that kernel: each occupant carries its own pair of events (copied,
// consumed), so waits never depend on which CUDA stream the caller uses.
// Prefetch runs cyclically into the next sweep's first streams, so back to
// back sweeps keep the copy engine busy across the rewind.
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <deque>
#include <memory>
#include <string>
#include <vector>

#include "abi.h"
#include "chain_launch.h"
#include "sweep_ring.h"

using namespace spm;

namespace {

bool block_profile(uint8_t enc) { return enc == SPM_ENC_Q8_0 || enc == SPM_ENC_Q6K || enc == SPM_ENC_Q5K; }

struct SweepStream {
    uint8_t kind = 0;             // the stream's .spm encoding
    uint32_t rows = 0, cols = 0, group = 0;
    uint64_t rows_pad = 0, col_words = 0, groups = 0;
    uint64_t host_off = 0, bytes = 0;  // packed bytes in the pinned image
    uint64_t scale_off = 0;            // ternary: scales inside the packed bytes
    uint64_t payload_bytes = 0;
};

uint64_t align256(uint64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

struct spm_sweep final : RingBackend {
    int device = 0, sms = 148;
    std::vector<SweepStream> streams;
    uint8_t* host = nullptr;
    uint64_t host_bytes = 0;
    uint8_t* ring_mem = nullptr;
    uint64_t cap = 0;
    cudaStream_t copy_stream = nullptr;
    std::unique_ptr<SweepRing> ring;
    std::vector<cudaEvent_t> copied, consumed;
    uint64_t bytes_copied = 0;
    // the launch in progress (set by spm_sweep_next around SweepRing::run)
    const float* x = nullptr;
    float* y = nullptr;
    int32_t positions = 0;
    cudaStream_t compute = nullptr;

    ~spm_sweep() override {
        if (copy_stream) cudaStreamSynchronize(copy_stream);
        for (cudaEvent_t e : consumed) cudaEventSynchronize(e);  // kernels that read the ring
        for (cudaEvent_t e : copied) cudaEventDestroy(e);
        for (cudaEvent_t e : consumed) cudaEventDestroy(e);
        if (copy_stream) cudaStreamDestroy(copy_stream);
        if (ring_mem) cudaFree(ring_mem);
        if (host) cudaFreeHost(host);
    }

    int create_events() override {
        cudaEvent_t a = nullptr, b = nullptr;
        CUDA_OK(cudaEventCreateWithFlags(&a, cudaEventDisableTiming));
        if (cudaEventCreateWithFlags(&b, cudaEventDisableTiming) != cudaSuccess) {
            cudaEventDestroy(a);
            fail(SPM_E_CUDA, "cudaEventCreateWithFlags failed");
        }
        copied.push_back(a);
        consumed.push_back(b);
        return int(copied.size()) - 1;
    }

    void wait_consumed(int ev) override { CUDA_OK(cudaStreamWaitEvent(copy_stream, consumed[ev], 0)); }

    void copy(uint32_t stream, uint64_t off, int ev) override {
        const SweepStream& st = streams[stream];
        if (st.bytes)
            CUDA_OK(cudaMemcpyAsync(ring_mem + off, host + st.host_off, st.bytes, cudaMemcpyHostToDevice,
                                    copy_stream));
        CUDA_OK(cudaEventRecord(copied[ev], copy_stream));
        bytes_copied += st.bytes;
    }

    void launch(uint32_t stream, uint64_t off, int ev) override {
        const SweepStream& st = streams[stream];
        CUDA_OK(cudaStreamWaitEvent(compute, copied[ev], 0));
        cudaError_t e = cudaSuccess;
        if (positions > 0 && st.rows > 0) {
            const uint8_t* base = ring_mem + off;
            if (st.kind == SPM_ENC_TERNARY) {
                TernaryArgs a{};
                a.codes = reinterpret_cast<const uint32_t*>(base);
                a.scales = reinterpret_cast<const float*>(base + st.scale_off);
                a.x = x;
                a.y = y;
                a.rows_pad = st.rows_pad;
                a.col_words = st.col_words;
                a.x_cols = st.cols;
                a.rows = st.rows;
                a.cols = st.cols;
                a.group = st.group;
                a.q = st.rows / st.group;
                a.r = st.rows % st.group;
                a.last_group = st.groups ? uint32_t(st.groups - 1) : 0u;
                a.lanes = positions;
                e = launch_ternary_gemv(a, sms, compute);
            } else if (block_profile(st.kind)) {
                QBlockArgs a{};
                a.blocks = base;
                a.x = x;
                a.y = y;
                a.rows_pad = st.rows_pad;
                a.rows = st.rows;
                a.cols = st.cols;
                a.positions = positions;
                e = launch_qblock_chain(a, st.kind, sms, compute);
            } else {
                DenseArgs a{};
                a.w = base;
                a.x = x;
                a.y = y;
                a.rows_pad = st.rows_pad;
                a.rows = st.rows;
                a.cols = st.cols;
                a.positions = positions;
                e = launch_dense_streamed(a, st.kind == SPM_ENC_BF16, sms, compute);
            }
        }
        if (e == cudaErrorInvalidConfiguration) fail(SPM_E_ARG, "too many rows x positions for one launch");
        CUDA_OK(e);
        CUDA_OK(cudaEventRecord(consumed[ev], compute));
    }
};

spm_status spm_sweep_open(const uint8_t* spm, uint64_t len, int device, uint64_t device_bytes, spm_sweep** out) {
    return guarded([&] {
        if (!out) fail(SPM_E_ARG, "null output");
        const SpmFile f = spm_file_parse(spm, len);
        std::unique_ptr<spm_sweep> s(new spm_sweep());
        // plan every stream first (host work, so refusals need no device);
        // each is packed later straight into the pinned image
        std::vector<StreamPlan> plans;
        uint64_t largest = 0;
        for (uint32_t i = 0; i < f.desc.size(); ++i) {
            const uint8_t enc = f.desc[i].encoding;
            const StreamPlan pl = enc == SPM_ENC_TERNARY ? plan_ternary(spm, len, i)
                                  : block_profile(enc)   ? plan_qblocks(spm, len, i)
                                                         : plan_dense(spm, len, i);
            SweepStream st;
            st.kind = enc;
            st.rows = pl.rows, st.cols = pl.cols, st.group = pl.group_size;
            st.rows_pad = pl.rows_pad, st.col_words = pl.col_words, st.groups = pl.groups;
            st.scale_off = pl.scale_off;
            st.bytes = pl.bytes;
            st.payload_bytes = pl.payload_bytes;
            st.host_off = s->host_bytes;
            s->host_bytes = align256(s->host_bytes + st.bytes);
            largest = std::max(largest, align256(st.bytes));
            s->streams.push_back(st);
            plans.push_back(pl);
        }
        if (s->streams.empty()) fail(SPM_E_ARG, "parameter stream declares no operations");
        if (device_bytes == 0) device_bytes = 2 * largest;
        if (device_bytes < largest) {
            char msg[128];
            std::snprintf(msg, sizeof msg, "device_bytes %llu cannot hold the largest stream (%llu bytes)",
                          (unsigned long long)device_bytes, (unsigned long long)largest);
            fail(SPM_E_ARG, msg);
        }
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) fail(SPM_E_NO_DEVICE, "no CUDA device is visible");
        s->device = device;
        CUDA_OK(cudaSetDevice(device));
        CUDA_OK(cudaDeviceGetAttribute(&s->sms, cudaDevAttrMultiProcessorCount, device));
        CUDA_OK(cudaHostAlloc(reinterpret_cast<void**>(&s->host), std::max<uint64_t>(s->host_bytes, 256),
                              cudaHostAllocDefault));
        for (uint32_t i = 0; i < s->streams.size(); ++i)
            if (plans[i].bytes) fill_stream(spm, plans[i], s->host + s->streams[i].host_off);
        s->cap = device_bytes / 256 * 256;
        CUDA_OK(cudaMalloc(reinterpret_cast<void**>(&s->ring_mem), s->cap));
        CUDA_OK(cudaStreamCreateWithFlags(&s->copy_stream, cudaStreamNonBlocking));
        std::vector<uint64_t> regions;
        for (const SweepStream& st : s->streams) regions.push_back(align256(st.bytes));
        s->ring.reset(new SweepRing(regions, s->cap));
        s->ring->prefetch(*s);  // start reading ahead, as the reference's worker does on open
        *out = s.release();
    });
}

spm_status spm_sweep_open_file(const char* path, int device, uint64_t device_bytes, spm_sweep** out) {
    // The file is mapped, not read into memory: packing reads it once, straight
    // into the pinned image, so the host holds one copy of the weights.
    int fd = -1;
    void* map = MAP_FAILED;
    uint64_t len = 0;
    const spm_status st = guarded([&] {
        if (!path) fail(SPM_E_ARG, "null path");
        fd = open(path, O_RDONLY);
        if (fd < 0) fail(SPM_E_STREAM, std::string("cannot open ") + path);
        struct stat sb;
        if (fstat(fd, &sb) != 0) fail(SPM_E_STREAM, std::string("cannot stat ") + path);
        len = uint64_t(sb.st_size);
        if (len) {
            map = mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0);
            if (map == MAP_FAILED) fail(SPM_E_STREAM, std::string("cannot map ") + path);
        }
    });
    spm_status rc = st;
    if (rc == SPM_OK) rc = spm_sweep_open(len ? static_cast<const uint8_t*>(map) : nullptr, len, device, device_bytes, out);
    if (map != MAP_FAILED) munmap(map, len);
    if (fd >= 0) close(fd);
    return rc;
}

spm_status spm_sweep_close(spm_sweep* s) {
    return guarded([&] {
        if (s) CUDA_OK(cudaSetDevice(s->device));
        delete s;
    });
}

spm_status spm_sweep_describe(const spm_sweep* s, spm_sweep_info* out) {
    return guarded([&] {
        if (!s || !out) fail(SPM_E_ARG, "null argument");
        *out = spm_sweep_info{};
        out->streams = int32_t(s->streams.size());
        out->position = int32_t(s->ring->position());
        out->host_bytes = s->host_bytes;
        out->device_bytes = s->cap;
        out->copies = s->ring->copies();
        out->bytes_copied = s->bytes_copied;
    });
}

spm_status spm_sweep_stream(const spm_sweep* s, int32_t index, uint32_t* rows, uint32_t* cols, uint32_t* encoding) {
    return guarded([&] {
        if (!s) fail(SPM_E_ARG, "null sweep");
        if (index < 0 || uint32_t(index) >= s->streams.size()) fail(SPM_E_ARG, "stream index out of range");
        const SweepStream& st = s->streams[index];
        if (rows) *rows = st.rows;
        if (cols) *cols = st.cols;
        if (encoding) *encoding = st.kind;
    });
}

spm_status spm_sweep_next(spm_sweep* s, const float* x_dev, uint64_t x_len, int32_t positions, float* y_dev,
                          void* cuda_stream, int32_t* stream_index) {
    return guarded([&] {
        if (!s) fail(SPM_E_ARG, "null sweep");
        const uint64_t n = s->streams.size();
        if (s->ring->position() >= n) fail(SPM_E_TRUNCATED, "the sweep has run every stream: rewind it");
        const SweepStream& st = s->streams[s->ring->position()];
        if (positions < 0) fail(SPM_E_ARG, "negative position count");
        const uint64_t need = uint64_t(positions) * st.cols;
        if (x_len < need) {
            char msg[96];
            std::snprintf(msg, sizeof msg, "need %llu activations, got %llu", (unsigned long long)need,
                          (unsigned long long)x_len);
            fail(SPM_E_ACTIVATION_LEN, msg);
        }
        if (positions > 0 && st.rows > 0 && (!y_dev || (st.cols && !x_dev)))
            fail(SPM_E_ARG, "null activation or output pointer");
        CUDA_OK(cudaSetDevice(s->device));
        s->x = x_dev;
        s->y = y_dev;
        s->positions = positions;
        s->compute = static_cast<cudaStream_t>(cuda_stream);
        const uint32_t index = s->ring->run(*s);
        if (stream_index) *stream_index = int32_t(index);
    });
}

spm_status spm_sweep_rewind(spm_sweep* s) {
    return guarded([&] {
        if (!s) fail(SPM_E_ARG, "null sweep");
        CUDA_OK(cudaSetDevice(s->device));
        s->ring->rewind(*s);
    });
}
