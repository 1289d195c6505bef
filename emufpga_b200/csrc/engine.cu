// Host orchestration and the C ABI (include/spmgpu.h).
//
// A model is the weight stream laid out in HBM in consumption order (the
// .order file's [rotating] list, then the [resident] quantized tensors), one
// packed matrix after another.  A session owns the per-client KV caches and
// scratch, and replays one CUDA graph per client count: a decode step reads
// every weight exactly once and serves all clients
// (spm-batch/src/step.rs:19-53).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <atomic>
#include <cmath>
#include <fstream>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <thread>

#include "abi.h"
#include "kernels.h"
#include "moe.h"
#include "prefill.h"

namespace spm {
const std::string& last_error();
}
using namespace spm;

// A packed matrix in the device image.
struct StreamDesc {
    std::string name;
    Packed pk;
    uint64_t experts = 1;       // >1: rows = experts * rows_per_expert
    bool rotating = false;      // swept every step (counted in weight bytes)
};

struct LayerIdx {
    int q = -1, k = -1, v = -1, o = -1, gate = -1, up = -1, down = -1;
    int router = -1, gate_exps = -1, up_exps = -1, down_exps = -1;
    int64_t attn_norm = -1, ffn_norm = -1, q_norm = -1, k_norm = -1, bias = -1;  // offsets in gains
};

struct spm_model {
    spm_model_cfg cfg{};
    int device = 0, sms = 148;
    int world = 1, rank = 0;  // expert parallel: this GPU holds experts e with e % world == rank
    uint8_t* image = nullptr;
    uint64_t image_bytes = 0;
    std::vector<StreamDesc> streams;
    std::vector<LayerIdx> layers;
    int embed = -1, head = -1;
    float* gains = nullptr;
    int64_t output_norm = -1;
    uint64_t weight_bytes = 0;
    ~spm_model() {
        if (image) cudaFree(image);
        if (gains) cudaFree(gains);
    }
    const uint8_t* tiles(int idx) const { return image + streams[idx].pk.offset; }
};

struct spm_weights {
    Packed pk;
    int device = 0, sms = 148;
    uint8_t* dev = nullptr;
    ~spm_weights() { if (dev) cudaFree(dev); }
};

// Upper bound on the CTAs of any GEMV launch (2 per SM) and so on the
// sum-of-squares parts one launch writes.
constexpr int kMaxParts = 2 * 1024;

struct spm_session {
    spm_model* m = nullptr;
    int max_clients = 0, context = 0;
    cudaStream_t stream = nullptr;
    float *kc = nullptr, *vc = nullptr;
    // the cache rows split into three bf16 planes, for the tensor-core
    // attention (models with 4-8 query heads per kv head, head_dim 64 or 128)
    uint16_t *kp = nullptr, *vp = nullptr;
    float *states = nullptr, *normed = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
    float *act = nullptr, *logits = nullptr;
    float2* rope = nullptr;
    int32_t* pos = nullptr;
    uint32_t *tokens = nullptr, *argmax = nullptr;
    uint32_t *h_tokens = nullptr, *h_argmax = nullptr;
    float* sumsq = nullptr;            // two [kMaxParts][8] partial sum-of-squares buffers
    // routed feed-forward: router logits, one plan per layer, expert activations / outputs
    float *moe_logits = nullptr, *moe_act = nullptr, *moe_out = nullptr;
    MoePlan* plans = nullptr;
    int moe_max_active = 0;
    float* attn_scratch = nullptr;
    int32_t* attn_counters = nullptr;
    uint32_t* route_counter = nullptr;  // CTAs of the router launch that have finished (zero between launches)
    int32_t* status = nullptr;         // device error word of bounded waits
    int32_t* h_status = nullptr;
    uint32_t* step = nullptr;          // steps taken (advance kernel); names the exchange rounds
    // Expert parallel exchange (model world > 1): one allocation, exported by
    // CUDA IPC, holding flags[2][64] (512 bytes) then two parity buffers of
    // expert output rows; every rank writes its experts' rows into every
    // rank's buffer and raises its flag there.
    uint8_t* ep_region = nullptr;
    size_t ep_xbytes = 0;              // bytes of one parity buffer
    uint32_t* ep_done = nullptr;       // CTA counter of the expert down launch
    float** ep_peer_y = nullptr;       // device [2][world]
    uint32_t** ep_peer_flag = nullptr; // device [2][world]
    std::vector<void*> ep_mapped;      // peers' regions opened by IPC
    // Data-parallel attention (world > 1): rank r runs the attention block
    // of its own clients; the area after the expert buffers in ep_region
    // holds the all-gather flags [2][64] and the greedy-pick flags [64]
    // (dp_flags), then this session's greedy picks, states and sums of
    // squares, which the other ranks write into.
    size_t dp_off = 0, dp_states_bytes = 0;
    uint32_t* dp_flags = nullptr;
    uint32_t* ep_done2 = nullptr;       // CTA counter of the o launch
    float** dp_peer_states = nullptr;   // device [world]: every rank's states
    float** dp_peer_sumsq = nullptr;    // device [world]: every rank's second sums-of-squares array
    uint32_t** dp_peer_flag = nullptr;  // device [2][world]: this rank's all-gather flag on every rank
    uint32_t** dp_peer_argmax = nullptr;  // device [world]
    uint32_t** dp_peer_gflag = nullptr;   // device [world]: every rank's greedy-pick flags
    bool ep_ready = false;
    uint64_t wait_ns = 1000000000ull;  // limit of the device waits on other ranks (spm_session_set_wait_limit)
    std::vector<int> lens;
    bool graphs = true, pdl = true;
    // GEMV launch profile (spm_session_set_profile): steps run eagerly and
    // every GEMV launch is bracketed by an event pair on the session stream;
    // a launch's algorithmic bytes are the quantized weight bytes it streams
    // (for expert launches counted from the step's plans once it has run).
    struct ProfLaunch {
        cudaEvent_t a, b;
        uint64_t bytes;
        int32_t kind, layer, stream;
    };
    bool prof = false;
    std::vector<ProfLaunch> prof_pending;
    // Prompt buffers (spm_prefill), allocated on first use for kPrefillRows rows.
    struct Prefill {
        int rows = 0;
        uint32_t* tokens = nullptr;
        int32_t* qpos = nullptr;
        float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
        float *g = nullptr, *u = nullptr;                          // dense feed-forward
        float *logits = nullptr, *prob = nullptr, *norm = nullptr, *ge = nullptr, *ue = nullptr, *ye = nullptr;
        int32_t *sel = nullptr, *counts = nullptr, *offsets = nullptr, *cursor = nullptr, *list = nullptr,
                *slot = nullptr;
        int4* groups = nullptr;                                    // routed: expert groups of <= 128 places
    } pf;
    std::vector<float> prof_ms;
    std::vector<uint64_t> prof_bytes;
    std::vector<int32_t> prof_kind;
    std::map<int, cudaGraphExec_t> exec;
    std::map<int, int> launches;
    std::vector<void*> allocs;
    ~spm_session() {
        for (auto& p : prof_pending) cudaEventDestroy(p.a), cudaEventDestroy(p.b);
        for (auto& kv : exec) cudaGraphExecDestroy(kv.second);
        for (void* p : ep_mapped) cudaIpcCloseMemHandle(p);
        for (void* p : allocs) cudaFree(p);
        if (h_tokens) cudaFreeHost(h_tokens);
        if (h_argmax) cudaFreeHost(h_argmax);
        if (h_status) cudaFreeHost(h_status);
        if (stream) cudaStreamDestroy(stream);
    }
    template <class T>
    T* alloc(size_t count) {
        void* p = nullptr;
        CUDA_OK(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)));
        CUDA_OK(cudaMemset(p, 0, std::max<size_t>(count, 1) * sizeof(T)));
        allocs.push_back(p);
        return static_cast<T*>(p);
    }
};

namespace {

bool is_moe(const spm_model_cfg& c) { return c.family == SPM_FAMILY_OLMOE || c.family == SPM_FAMILY_QWEN3MOE; }

uint32_t meta_u32(const Gguf& g, const std::string& key, uint32_t dflt) {
    auto* m = g.meta_find(key);
    return (m && m->has_int) ? uint32_t(m->u) : dflt;
}
float meta_f32(const Gguf& g, const std::string& key, float dflt) {
    auto* m = g.meta_find(key);
    return (m && m->has_float) ? float(m->f) : dflt;
}

// Model shape from GGUF metadata when the caller passes none.
spm_model_cfg cfg_from_gguf(const Gguf& g) {
    spm_model_cfg c{};
    auto* a = g.meta_find("general.architecture");
    if (!a) fail(SPM_E_STREAM, "GGUF has no general.architecture and no shape was given");
    const std::string arch = a->s;
    if (arch == "llama") c.family = SPM_FAMILY_LLAMA;
    else if (arch == "qwen3") c.family = SPM_FAMILY_QWEN3;
    else if (arch == "olmoe") c.family = SPM_FAMILY_OLMOE;
    else if (arch == "qwen3moe") c.family = SPM_FAMILY_QWEN3MOE;
    else fail(SPM_E_ARG, "unsupported architecture " + arch);
    c.layers = meta_u32(g, arch + ".block_count", 0);
    c.hidden = meta_u32(g, arch + ".embedding_length", 0);
    c.intermediate = meta_u32(g, arch + ".feed_forward_length", 0);
    c.heads = meta_u32(g, arch + ".attention.head_count", 0);
    c.kv_heads = meta_u32(g, arch + ".attention.head_count_kv", c.heads);
    c.head_dim = meta_u32(g, arch + ".attention.key_length", c.heads ? c.hidden / c.heads : 0);
    c.experts = meta_u32(g, arch + ".expert_count", 0);
    c.experts_used = meta_u32(g, arch + ".expert_used_count", 0);
    c.expert_ff = meta_u32(g, arch + ".expert_feed_forward_length", 0);
    c.rope_base = meta_f32(g, arch + ".rope.freq_base", 10000.0f);
    c.eps = meta_f32(g, arch + ".attention.layer_norm_rms_epsilon", 1e-5f);
    auto* te = g.find("token_embd.weight");
    if (!te || te->dims.size() < 2) fail(SPM_E_STREAM, "missing token_embd.weight");
    c.vocab = meta_u32(g, arch + ".vocab_size", uint32_t(te->dims[1]));
    c.tied = g.find("output.weight") ? 0 : 1;
    return c;
}

void check_cfg(const spm_model_cfg& c) {
    if (c.family < SPM_FAMILY_LLAMA || c.family > SPM_FAMILY_QWEN3MOE) fail(SPM_E_ARG, "unknown model family");
    if (!c.layers || !c.hidden || !c.heads || !c.kv_heads || !c.head_dim || !c.vocab)
        fail(SPM_E_ARG, "model shape has a zero dimension");
    if (c.heads % c.kv_heads) fail(SPM_E_ARG, "heads must group evenly over kv_heads");
    if (c.head_dim % 2 || c.head_dim > 1024) fail(SPM_E_ARG, "head_dim must be even and at most 1024");
    if (c.hidden % 32) fail(SPM_E_ARG, "hidden must be a multiple of 32");
    if (is_moe(c) && (!c.experts || !c.experts_used || c.experts_used > c.experts || !c.expert_ff))
        fail(SPM_E_ARG, "MoE shape needs experts, experts_used <= experts and expert_ff");
}

// Both directions, as spm-order/src/order.rs:64-83 (reorder).
void check_order(const Order& o, const Gguf& g) {
    std::set<std::string> wanted;
    for (auto* list : {&o.rotating, &o.resident})
        for (auto& n : *list) {
            if (!g.find(n)) fail(SPM_E_STREAM, n + ": named in the order file but not in the checkpoint");
            if (!wanted.insert(n).second) fail(SPM_E_STREAM, n + ": named twice in the order file");
        }
    for (auto& t : g.tensors)
        if (!wanted.count(t.name)) fail(SPM_E_STREAM, t.name + ": in the checkpoint but not named in the order file");
}

// Host-side description of a model: streams in consumption order with their
// packed shapes and offsets in the device image, the norm gains, and the
// per-layer stream and gain indices.  Built from a GGUF (describe) or read
// from a packed image file (read_image); no GPU involved.
struct ModelDesc {
    spm_model_cfg cfg{};
    std::vector<StreamDesc> streams;
    std::vector<float> gains;
    std::map<std::string, int> stream_of;
    std::map<std::string, std::pair<int64_t, uint64_t>> gain_of;  // offset in gains, length
    std::vector<LayerIdx> layers;
    int embed = -1, head = -1;
    int64_t output_norm = -1;
    uint64_t image_bytes = 0, weight_bytes = 0;
};

// Layer indices, shape and encoding checks, and the weight bytes of a sweep,
// from the stream and gain tables.
void index_layers(ModelDesc& d) {
    const spm_model_cfg& c = d.cfg;
    auto need_stream = [&](const std::string& n) {
        auto it = d.stream_of.find(n);
        if (it == d.stream_of.end()) fail(SPM_E_STREAM, "missing tensor " + n);
        return it->second;
    };
    auto need_gain = [&](const std::string& n, uint64_t count) {
        auto it = d.gain_of.find(n);
        if (it == d.gain_of.end()) fail(SPM_E_STREAM, "missing tensor " + n);
        if (it->second.second != count) fail(SPM_E_ARG, n + " has the wrong length");
        return it->second.first;
    };
    auto check_shape = [&](int idx, uint64_t rows, uint64_t cols) {
        const StreamDesc& s = d.streams[idx];
        if (s.pk.rows != rows || s.pk.cols != cols)
            fail(SPM_E_ARG, s.name + ": shape " + std::to_string(s.pk.rows) + "x" + std::to_string(s.pk.cols) +
                                " does not match the model (" + std::to_string(rows) + "x" + std::to_string(cols) + ")");
        return idx;
    };
    const uint64_t qw = uint64_t(c.heads) * c.head_dim, kvw = uint64_t(c.kv_heads) * c.head_dim;
    d.layers.assign(c.layers, LayerIdx{});
    for (uint32_t l = 0; l < c.layers; l++) {
        const std::string p = "blk." + std::to_string(l) + ".";
        LayerIdx& L = d.layers[l];
        L.q = check_shape(need_stream(p + "attn_q.weight"), qw, c.hidden);
        L.k = check_shape(need_stream(p + "attn_k.weight"), kvw, c.hidden);
        L.v = check_shape(need_stream(p + "attn_v.weight"), kvw, c.hidden);
        L.o = check_shape(need_stream(p + "attn_output.weight"), c.hidden, qw);
        L.attn_norm = need_gain(p + "attn_norm.weight", c.hidden);
        L.ffn_norm = need_gain(p + "ffn_norm.weight", c.hidden);
        if (c.family == SPM_FAMILY_OLMOE) {
            L.q_norm = need_gain(p + "attn_q_norm.weight", qw);
            L.k_norm = need_gain(p + "attn_k_norm.weight", kvw);
        } else if (c.family != SPM_FAMILY_LLAMA) {
            L.q_norm = need_gain(p + "attn_q_norm.weight", c.head_dim);
            L.k_norm = need_gain(p + "attn_k_norm.weight", c.head_dim);
        }
        if (is_moe(c)) {
            L.router = check_shape(need_stream(p + "ffn_gate_inp.weight"), c.experts, c.hidden);
            L.gate_exps = check_shape(need_stream(p + "ffn_gate_exps.weight"), uint64_t(c.experts) * c.expert_ff, c.hidden);
            L.up_exps = check_shape(need_stream(p + "ffn_up_exps.weight"), uint64_t(c.experts) * c.expert_ff, c.hidden);
            L.down_exps = check_shape(need_stream(p + "ffn_down_exps.weight"), uint64_t(c.experts) * c.hidden, c.expert_ff);
            if (d.gain_of.count(p + "exp_probs_b.bias")) L.bias = need_gain(p + "exp_probs_b.bias", c.experts);
        } else {
            L.gate = check_shape(need_stream(p + "ffn_gate.weight"), c.intermediate, c.hidden);
            L.up = check_shape(need_stream(p + "ffn_up.weight"), c.intermediate, c.hidden);
            L.down = check_shape(need_stream(p + "ffn_down.weight"), c.hidden, c.intermediate);
            if (d.streams[L.gate].pk.dtype != d.streams[L.up].pk.dtype)
                fail(SPM_E_ENCODING, p + "ffn_gate and ffn_up must share an encoding");
        }
        if (d.streams[L.q].pk.dtype != d.streams[L.k].pk.dtype || d.streams[L.q].pk.dtype != d.streams[L.v].pk.dtype)
            fail(SPM_E_ENCODING, p + "attn_q/k/v must share an encoding");
    }
    d.embed = check_shape(need_stream("token_embd.weight"), c.vocab, c.hidden);
    d.head = c.tied ? d.embed : check_shape(need_stream("output.weight"), c.vocab, c.hidden);
    d.output_norm = need_gain("output_norm.weight", c.hidden);
    if (d.streams[d.embed].pk.dtype == SPM_F32 && c.hidden % 32) fail(SPM_E_ARG, "bad embedding width");
    // StepReport::for_sweep (spm-batch/src/session.rs:105-120): descriptor
    // bytes of every matrix one step reads -- here the rotating streams plus
    // the LM head.  MoE steps read only the routed experts; their per-step
    // bytes are counted by the session.
    d.weight_bytes = 0;
    for (auto& s : d.streams)
        if (s.rotating && s.experts == 1) d.weight_bytes += s.pk.quant_bytes;
    if (!d.streams[d.head].rotating) d.weight_bytes += d.streams[d.head].pk.quant_bytes;
}

ModelDesc describe(const Gguf& g, const uint8_t* buf, const std::string* order_text, const spm_model_cfg* cfg) {
    ModelDesc d;
    d.cfg = cfg ? *cfg : cfg_from_gguf(g);
    check_cfg(d.cfg);
    Order order =
        parse_order(order_text ? *order_text : default_order(d.cfg, g.find("blk.0.exp_probs_b.bias") != nullptr));
    check_order(order, g);
    // Streams in consumption order; 1-D tensors are resident gains.
    uint64_t off = 0;
    auto add_names = [&](const std::vector<std::string>& names, bool rotating) {
        for (auto& n : names) {
            const GgufTensor* t = g.find(n);
            if (t->dims.size() == 1) {
                if (t->dtype != SPM_F32 && t->dtype != SPM_F16)
                    fail(SPM_E_ENCODING, n + ": 1-D tensors must be F32 or F16");
                d.gain_of[n] = {int64_t(d.gains.size()), t->dims[0]};
                std::vector<float> v(t->dims[0]);
                decode_blocks(t->dtype, buf + t->offset, t->len, v.data());
                d.gains.insert(d.gains.end(), v.begin(), v.end());
                while (d.gains.size() % 4) d.gains.push_back(0.f);
                continue;
            }
            StreamDesc s;
            s.name = n;
            s.rotating = rotating;
            uint64_t rows = 1;
            for (size_t k = 1; k < t->dims.size(); k++) rows *= t->dims[k];
            s.experts = t->dims.size() > 2 ? t->dims[2] : 1;
            s.pk = packed_shape(t->dtype, rows, t->dims[0]);
            s.pk.offset = off;
            off += (s.pk.tiles * s.pk.tile_bytes + 255) & ~uint64_t(255);
            d.stream_of[n] = int(d.streams.size());
            d.streams.push_back(s);
        }
    };
    add_names(order.rotating, true);
    add_names(order.resident, false);
    d.image_bytes = off;
    index_layers(d);
    return d;
}

// Pack stream i of a GGUF-described model into host memory (all experts, or
// with world > 1 only rank's, each at its own place).  Calls sink(offset in
// the image, bytes, size) for every packed run.
template <class Sink>
void pack_stream(const ModelDesc& d, const Gguf& g, const uint8_t* buf, size_t i, int world, int rank,
                 std::vector<uint8_t>& host, Sink&& sink) {
    const StreamDesc& s = d.streams[i];
    const GgufTensor* t = g.find(s.name);
    if (world > 1 && s.experts > 1) {
        // this rank's experts only; each is a whole run of tiles
        const uint64_t er = s.pk.rows / s.experts;
        Packed sub = packed_shape(s.pk.dtype, er, s.pk.cols);
        if (sub.tile_bytes != s.pk.tile_bytes || sub.tiles * s.experts != s.pk.tiles)
            fail(SPM_E_ARG, s.name + ": experts are not whole tiles");
        const uint64_t src = t->len / s.experts;
        host.resize(sub.tiles * sub.tile_bytes);
        for (uint64_t e = uint64_t(rank); e < s.experts; e += uint64_t(world)) {
            pack_matrix(sub, buf + t->offset + e * src, host.data());
            sink(s.pk.offset + e * host.size(), host.data(), host.size());
        }
        return;
    }
    host.resize(s.pk.tiles * s.pk.tile_bytes);
    pack_matrix(s.pk, buf + t->offset, host.data());
    sink(s.pk.offset, host.data(), host.size());
}

// Runs f(i, worker) for i < count on up to 16 host threads; the first error wins.
template <class F>
void parallel_streams(size_t count, F&& f) {
    std::atomic<size_t> next{0};
    std::vector<std::string> errs(std::max(1u, std::min(16u, std::thread::hardware_concurrency())));
    std::vector<int> codes(errs.size(), 0);
    auto worker = [&](size_t w) {
        try {
            for (;;) {
                const size_t i = next.fetch_add(1);
                if (i >= count) break;
                f(i, w);
            }
        } catch (const Error& e) {
            errs[w] = e.msg;
            codes[w] = e.code;
        }
    };
    std::vector<std::thread> pool;
    for (size_t w = 0; w < errs.size(); w++) pool.emplace_back(worker, w);
    for (auto& th : pool) th.join();
    for (size_t w = 0; w < errs.size(); w++)
        if (!errs[w].empty()) fail(codes[w], errs[w]);
}

// A model on `device` from its description: allocation, gains, and fill(m)
// to put the packed tiles in place.
template <class Fill>
spm_model* make_model(ModelDesc&& d, int device, int world, int rank, Fill&& fill) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) fail(SPM_E_NO_DEVICE, "no CUDA device is visible");
    if (device < 0 || device >= ndev) fail(SPM_E_ARG, "device index out of range");
    if (world < 1 || world > 8 || rank < 0 || rank >= world) fail(SPM_E_ARG, "expert parallel: 1 to 8 ranks");
    if (world > 1 && !is_moe(d.cfg)) fail(SPM_E_ARG, "expert parallel needs a routed (MoE) model");
    std::unique_ptr<spm_model> m(new spm_model());
    m->cfg = d.cfg;
    m->device = device;
    m->world = world;
    m->rank = rank;
    CUDA_OK(cudaSetDevice(device));
    CUDA_OK(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, device));
    m->streams = std::move(d.streams);
    m->layers = std::move(d.layers);
    m->embed = d.embed;
    m->head = d.head;
    m->output_norm = d.output_norm;
    m->image_bytes = d.image_bytes;
    m->weight_bytes = d.weight_bytes;
    CUDA_OK(cudaMalloc(&m->image, std::max<uint64_t>(m->image_bytes, 256)));
    fill(m.get());
    CUDA_OK(cudaMalloc(&m->gains, std::max<size_t>(d.gains.size(), 4) * sizeof(float)));
    CUDA_OK(cudaMemcpy(m->gains, d.gains.data(), d.gains.size() * sizeof(float), cudaMemcpyHostToDevice));
    return m.release();
}

spm_model* open_model(const uint8_t* buf, uint64_t len, const std::string* order_text, const spm_model_cfg* cfg,
                      int device, int world = 1, int rank = 0) {
    Gguf g = gguf_parse(buf, len);
    ModelDesc d = describe(g, buf, order_text, cfg);
    ModelDesc keep = d;  // stream table for packing after make_model takes d
    return make_model(std::move(d), device, world, rank, [&](spm_model* m) {
        // pack each matrix on the host (threads over matrices) and copy
        parallel_streams(keep.streams.size(), [&](size_t i, size_t) {
            if (cudaSetDevice(device) != cudaSuccess) fail(SPM_E_CUDA, "cudaSetDevice failed");
            std::vector<uint8_t> host;
            pack_stream(keep, g, buf, i, world, rank, host, [&](uint64_t off, const uint8_t* p, size_t n) {
                CUDA_OK(cudaMemcpy(m->image + off, p, n, cudaMemcpyHostToDevice));
            });
        });
    });
}

// A GGUF file mapped read-only: ranks that open the same file share its
// pages instead of each holding a copy.
struct Mapped {
    const uint8_t* p = nullptr;
    size_t n = 0;
    explicit Mapped(const char* path) {
        const int fd = open(path, O_RDONLY);
        if (fd < 0) fail(SPM_E_STREAM, std::string(path) + ": cannot open");
        struct stat st {};
        if (fstat(fd, &st) != 0 || st.st_size <= 0) {
            close(fd);
            fail(SPM_E_STREAM, std::string(path) + ": cannot read");
        }
        n = size_t(st.st_size);
        void* q = mmap(nullptr, n, PROT_READ, MAP_SHARED, fd, 0);
        close(fd);
        if (q == MAP_FAILED) fail(SPM_E_STREAM, std::string(path) + ": cannot map");
        p = static_cast<const uint8_t*>(q);
    }
    ~Mapped() {
        if (p) munmap(const_cast<uint8_t*>(p), n);
    }
};

// ---- packed device image files ----
// A model already packed for the device: the stream table, the norm gains,
// then the tiles exactly as they sit in HBM, so that opening it is one
// sequential read and upload.  The file is a .spm container (spm-header,
// spm-layout) extended with this library's tiled profiles.  Layout (little
// endian):
//   the 32-byte .spm header: magic, version 1.1, little-endian, stream count;
//   one 32-byte .spm descriptor per stream: rows, cols, group_size = values
//     per GGML block, encoding = kImageProfile + GGML type (this library's
//     tiled layout of that block type; .spm profiles 1-6 are the reference's,
//     so a stock .spm reader refuses these as unknown encodings),
//     lane_count = rows per tile;
//   "SPMIMG02", u64 data offset (4096-aligned), u64 image bytes, the
//   spm_model_cfg, u32 streams { u16 name length, name, u32 dtype, u64 rows,
//   cols, experts, u8 rotating, u64 tiles, tile bytes, u32 planes[4], u64
//   offset, quant bytes }, u32 gains { u16 name length, name, u64 offset,
//   length }, u64 floats, the floats; zeros up to the data offset; the image.
constexpr uint8_t kSpmMagic[8] = {0x89, 'S', 'P', 'M', 0x0D, 0x0A, 0x1A, 0x0A};
constexpr char kImageMagic[8] = {'S', 'P', 'M', 'I', 'M', 'G', '0', '2'};
constexpr uint8_t kImageProfile = 0x80;
constexpr uint64_t kImageAlign = 4096;

struct ImgWriter {
    std::vector<uint8_t> b;
    template <class T>
    void put(const T& v) {
        const uint8_t* p = reinterpret_cast<const uint8_t*>(&v);
        b.insert(b.end(), p, p + sizeof(T));
    }
    void str(const std::string& s) {
        put(uint16_t(s.size()));
        b.insert(b.end(), s.begin(), s.end());
    }
};

struct ImgReader {
    const uint8_t* p;
    uint64_t n, at = 0;
    template <class T>
    T get() {
        if (n - at < sizeof(T)) fail(SPM_E_TRUNCATED, "image header is truncated");
        T v;
        std::memcpy(&v, p + at, sizeof(T));
        at += sizeof(T);
        return v;
    }
    std::string str() {
        const uint16_t k = get<uint16_t>();
        if (n - at < k) fail(SPM_E_TRUNCATED, "image header is truncated");
        std::string s(reinterpret_cast<const char*>(p + at), k);
        at += k;
        return s;
    }
};

// The .spm descriptor of one packed stream.
void image_descriptor(ImgWriter& w, const StreamDesc& s) {
    uint64_t bv = 0, bb = 0;
    if (!type_layout(s.pk.dtype, &bv, &bb)) fail(SPM_E_ENCODING, s.name + ": no block layout");
    if (s.pk.rows > 0xFFFFFFFFull || s.pk.cols > 0xFFFFFFFFull) fail(SPM_E_ARG, s.name + ": too large for .spm");
    w.put(uint32_t(s.pk.rows));
    w.put(uint32_t(s.pk.cols));
    w.put(uint32_t(bv));
    w.put(uint8_t(kImageProfile + s.pk.dtype));
    w.put(uint8_t(0));
    w.put(uint16_t(kTileRows));
    for (int k = 0; k < 16; k++) w.put(uint8_t(0));
}

std::vector<uint8_t> image_header(const ModelDesc& d) {
    ImgWriter w;
    w.b.insert(w.b.end(), kSpmMagic, kSpmMagic + 8);  // .spm header (spm-header/src/lib.rs:3-25)
    w.put(uint16_t(1));
    w.put(uint16_t(1));
    w.put(uint32_t(0));  // little-endian, reserved
    w.put(uint32_t(d.streams.size()));
    for (int k = 0; k < 12; k++) w.put(uint8_t(0));
    for (const StreamDesc& s : d.streams) image_descriptor(w, s);
    w.b.insert(w.b.end(), kImageMagic, kImageMagic + 8);
    const size_t data_at = w.b.size();
    w.put(uint64_t(0));  // data offset, patched below
    w.put(d.image_bytes);
    w.put(d.cfg);
    w.put(uint32_t(d.streams.size()));
    for (const StreamDesc& s : d.streams) {
        w.str(s.name);
        w.put(s.pk.dtype);
        w.put(s.pk.rows);
        w.put(s.pk.cols);
        w.put(s.experts);
        w.put(uint8_t(s.rotating ? 1 : 0));
        w.put(s.pk.tiles);
        w.put(s.pk.tile_bytes);
        for (int k = 0; k < 4; k++) w.put(s.pk.plane[k]);
        w.put(s.pk.offset);
        w.put(s.pk.quant_bytes);
    }
    w.put(uint32_t(d.gain_of.size()));
    for (const auto& kv : d.gain_of) {
        w.str(kv.first);
        w.put(uint64_t(kv.second.first));
        w.put(kv.second.second);
    }
    w.put(uint64_t(d.gains.size()));
    for (float f : d.gains) w.put(f);
    const uint64_t data = (w.b.size() + kImageAlign - 1) / kImageAlign * kImageAlign;
    std::memcpy(w.b.data() + data_at, &data, 8);
    w.b.resize(data, 0);
    return w.b;
}

// The description and data offset of an image file held in memory.
ModelDesc read_image(const uint8_t* p, uint64_t n, uint64_t* data) {
    if (n < 32) fail(SPM_E_TRUNCATED, "image header is truncated");
    if (std::memcmp(p, kSpmMagic, 8) != 0) fail(SPM_E_STREAM, "not a packed image (bad magic)");
    uint16_t major;
    std::memcpy(&major, p + 8, 2);
    if (major != 1 || p[12] != 0) fail(SPM_E_STREAM, "not a packed image (version or byte order)");
    uint32_t nd;
    std::memcpy(&nd, p + 16, 4);
    if (nd > 1u << 20) fail(SPM_E_STREAM, "image stream count is not plausible");
    const uint64_t dir = 32 + 32 * uint64_t(nd);
    if (n < dir + 8) fail(SPM_E_TRUNCATED, "image header is truncated");
    if (std::memcmp(p + dir, kImageMagic, 8) != 0) fail(SPM_E_STREAM, "not a packed image (a .spm file of streams?)");
    ImgReader r{p, n, dir + 8};
    ModelDesc d;
    *data = r.get<uint64_t>();
    d.image_bytes = r.get<uint64_t>();
    d.cfg = r.get<spm_model_cfg>();
    check_cfg(d.cfg);
    const uint32_t ns = r.get<uint32_t>();
    if (ns != nd) fail(SPM_E_STREAM, "image directory and stream table disagree");
    for (uint32_t i = 0; i < ns; i++) {
        StreamDesc s;
        s.name = r.str();
        const uint32_t dtype = r.get<uint32_t>();
        const uint64_t rows = r.get<uint64_t>(), cols = r.get<uint64_t>();
        s.experts = r.get<uint64_t>();
        s.rotating = r.get<uint8_t>() != 0;
        Packed want = packed_shape(dtype, rows, cols);  // the layout this library packs
        Packed got = want;
        got.tiles = r.get<uint64_t>();
        got.tile_bytes = r.get<uint64_t>();
        for (int k = 0; k < 4; k++) got.plane[k] = r.get<uint32_t>();
        got.offset = r.get<uint64_t>();
        got.quant_bytes = r.get<uint64_t>();
        if (got.tiles != want.tiles || got.tile_bytes != want.tile_bytes || got.quant_bytes != want.quant_bytes ||
            std::memcmp(got.plane, want.plane, sizeof(want.plane)) != 0 || s.experts == 0 || rows % s.experts)
            fail(SPM_E_STREAM, s.name + ": packed layout does not match this library");
        if (got.offset > d.image_bytes || got.tiles * got.tile_bytes > d.image_bytes - got.offset)
            fail(SPM_E_STREAM, s.name + ": outside the image");
        s.pk = got;
        ImgWriter want_desc;  // the descriptor this stream must have in the directory
        image_descriptor(want_desc, s);
        if (std::memcmp(p + 32 + 32 * uint64_t(i), want_desc.b.data(), 32) != 0)
            fail(SPM_E_STREAM, s.name + ": directory entry does not match the stream");
        if (!d.stream_of.emplace(s.name, int(d.streams.size())).second) fail(SPM_E_STREAM, "duplicate stream " + s.name);
        d.streams.push_back(s);
    }
    const uint32_t ng = r.get<uint32_t>();
    std::vector<std::pair<std::string, std::pair<int64_t, uint64_t>>> gains;
    for (uint32_t i = 0; i < ng && i < (1u << 20); i++) {
        std::string name = r.str();
        const uint64_t off = r.get<uint64_t>(), len = r.get<uint64_t>();
        gains.push_back({name, {int64_t(off), len}});
    }
    const uint64_t nf = r.get<uint64_t>();
    if (nf > (n - r.at) / 4) fail(SPM_E_TRUNCATED, "image gains are truncated");
    d.gains.resize(nf);
    std::memcpy(d.gains.data(), p + r.at, nf * 4);
    r.at += nf * 4;
    for (auto& gk : gains) {
        if (gk.second.first < 0 || uint64_t(gk.second.first) > nf || gk.second.second > nf - uint64_t(gk.second.first))
            fail(SPM_E_STREAM, gk.first + ": gain outside the table");
        d.gain_of[gk.first] = gk.second;
    }
    if (*data < r.at || *data % kImageAlign || *data > n || d.image_bytes > n - *data)
        fail(SPM_E_TRUNCATED, "image data is truncated");
    index_layers(d);
    return d;
}

void write_image(const uint8_t* buf, uint64_t len, const std::string* order_text, const spm_model_cfg* cfg,
                 const char* path) {
    Gguf g = gguf_parse(buf, len);
    ModelDesc d = describe(g, buf, order_text, cfg);
    const std::vector<uint8_t> head = image_header(d);
    const int fd = open(path, O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) fail(SPM_E_STREAM, std::string(path) + ": cannot create");
    struct Closer {
        int fd;
        ~Closer() { close(fd); }
    } closer{fd};
    auto put = [&](uint64_t off, const uint8_t* p, size_t n) {
        while (n) {
            const ssize_t k = pwrite(fd, p, n, off_t(off));
            if (k <= 0) fail(SPM_E_STREAM, std::string(path) + ": write failed");
            p += k, n -= size_t(k), off += uint64_t(k);
        }
    };
    if (ftruncate(fd, off_t(head.size() + d.image_bytes)) != 0) fail(SPM_E_STREAM, std::string(path) + ": cannot size");
    put(0, head.data(), head.size());
    parallel_streams(d.streams.size(), [&](size_t i, size_t) {
        std::vector<uint8_t> host;
        pack_stream(d, g, buf, i, 1, 0, host, [&](uint64_t off, const uint8_t* p, size_t n) { put(head.size() + off, p, n); });
    });
}

std::string read_file(const char* path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) fail(SPM_E_STREAM, std::string(path) + ": cannot open");
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

// ---- one decode step ----
GemvLaunch gemv_base(const spm_model* m, int idx, const float* x, int n) {
    const Packed& p = m->streams[idx].pk;
    GemvLaunch L{};
    L.cols = uint32_t(p.cols);
    L.tile_bytes = uint32_t(p.tile_bytes);
    L.plane1 = p.plane[1];
    L.plane2 = p.plane[2];
    L.plane3 = p.plane[3];
    L.x = x;
    L.x_stride = int(p.cols);
    L.n = n;
    return L;
}

void add_job(GemvLaunch& L, const spm_model* m, int idx, const uint8_t* b, float* y, int y_stride, const float* aux,
             int aux_stride, int epi) {
    GemvJob& J = L.job[L.njobs++];
    const Packed& p = m->streams[idx].pk;
    J.a = m->tiles(idx);
    J.b = b;
    J.y = y;
    J.y_stride = y_stride;
    J.aux = aux;
    J.aux_stride = aux_stride;
    J.epi = epi;
    J.rows = uint32_t(p.rows);
    J.tile_begin = L.total_tiles;
    L.total_tiles += uint32_t(p.tiles);
}

// Launches a GEMV; returns its grid size (the number of sum-of-squares parts
// an EPI_ADD launch writes).
int run_gemv(const spm_model* m, GemvLaunch L, uint32_t dtype, cudaStream_t st, bool pdl) {
    int grid = 0;
    CUDA_OK(launch_gemv(dtype, L, m->sms, st, pdl, &grid));
    return grid;
}

// One decode step (spm-batch/src/step.rs:19-53), one kernel per streamed op:
//   embed -> per layer [norm+QKV] [attention] [O+residual] [norm+gate/up+SwiGLU]
//   [down+residual] -> [final norm + LM head] -> argmax -> positions += 1.
// The RMSNorms are fused into the GEMV that consumes them: the residual-add
// epilogues (and the embedding) write per-CTA sums of squares, which the next
// GEMV reduces in a fixed order before normalising its activations on load.
void enqueue_step(spm_session* s, int n) {
    spm_model* m = s->m;
    const spm_model_cfg& c = m->cfg;
    cudaStream_t st = s->stream;
    const bool pdl = s->pdl;
    const int d = int(c.hidden), qw = int(c.heads * c.head_dim), kvw = int(c.kv_heads * c.head_dim);
    const int ff = int(c.intermediate);
    const StreamDesc& E = m->streams[m->embed];
    float* part[2] = {s->sumsq, s->sumsq + kMaxParts * 8};
    // data-parallel attention: this rank's clients f0..f0+nl-1 run the
    // attention block; the routed feed-forward sees every client
    const bool dp = m->world > 1;
    const int nl = dp ? n / m->world : n, f0 = dp ? m->rank * nl : 0;
    // Every launch of the step goes through timed(): with the profile on, an
    // event pair brackets it (kind, layer, the stream it reads and its bytes
    // are kept for the record).
    auto timed = [&](int kind, int layer, int idx, uint64_t bytes, auto&& launch) {
        cudaEvent_t a = nullptr, b = nullptr;
        if (s->prof) {
            CUDA_OK(cudaEventCreate(&a));
            CUDA_OK(cudaEventCreate(&b));
            CUDA_OK(cudaEventRecord(a, st));
        }
        auto r = launch();
        if (s->prof) {
            CUDA_OK(cudaEventRecord(b, st));
            s->prof_pending.push_back({a, b, bytes, kind, layer, idx});
        }
        return r;
    };
    auto gemv = [&](const GemvLaunch& g, int idx, int kind, int layer, uint64_t bytes) {
        return timed(kind, layer, idx, bytes, [&] { return run_gemv(m, g, m->streams[idx].pk.dtype, st, pdl); });
    };
    auto qbytes = [&](int idx) { return m->streams[idx].pk.quant_bytes; };
    timed(SPM_KERNEL_OTHER, -1, -1, 0, [&] {
        CUDA_OK(launch_embed(E.pk.dtype, m->tiles(m->embed), E.pk, s->tokens + f0, nl, s->states + size_t(f0) * d,
                             part[0], st, false, f0));
        return 0;
    });
    int parts = nl;
    auto norm_in = [&](GemvLaunch& g, int64_t gain, int which) {
        g.gain = m->gains + gain;
        g.sumsq = part[which];
        g.sumsq_parts = parts;
        g.eps = c.eps;
    };
    for (uint32_t l = 0; l < c.layers; l++) {
        const LayerIdx& L = m->layers[l];
        GemvLaunch g = gemv_base(m, L.q, s->states + size_t(f0) * d, nl);
        g.status = s->status;
        g.c0 = f0;
        norm_in(g, L.attn_norm, 0);
        add_job(g, m, L.q, nullptr, s->q, qw, nullptr, 0, EPI_STORE);
        add_job(g, m, L.k, nullptr, s->k, kvw, nullptr, 0, EPI_STORE);
        add_job(g, m, L.v, nullptr, s->v, kvw, nullptr, 0, EPI_STORE);
        gemv(g, L.q, SPM_GEMV_DENSE, int(l), qbytes(L.q) + qbytes(L.k) + qbytes(L.v));
        AttnParams P{};
        P.q = s->q; P.k = s->k; P.v = s->v; P.out = s->attn;
        P.kcache = s->kc; P.vcache = s->vc; P.pos = s->pos + f0; P.rope = s->rope; P.cache_client = f0;
        P.kplanes = s->kp; P.vplanes = s->vp;
        P.scratch = s->attn_scratch; P.counters = s->attn_counters;
        P.q_norm = L.q_norm >= 0 ? m->gains + L.q_norm : nullptr;
        P.k_norm = L.k_norm >= 0 ? m->gains + L.k_norm : nullptr;
        P.layer = int(l); P.layers = int(c.layers); P.context = s->context;
        P.heads = int(c.heads); P.kv_heads = int(c.kv_heads); P.head_dim = int(c.head_dim);
        P.family = int(c.family); P.eps = c.eps; P.status = s->status;
        timed(SPM_KERNEL_ATTENTION, int(l), -1, 0, [&] {
            CUDA_OK(launch_attention(P, nl, st, pdl));
            return 0;
        });
        GemvLaunch go = gemv_base(m, L.o, s->attn, nl);
        go.status = s->status;
        go.sumsq_out = part[1];
        go.c0 = f0;
        if (dp) {
            // rows and sums of squares of this rank's clients to every rank,
            // then this rank's all-gather flag up on every rank
            if (!s->ep_ready) fail(SPM_E_ARG, "expert parallel session: call spm_session_ep_connect first");
            go.ep_dense = 1;
            go.world = m->world;
            go.rank = m->rank;
            go.ep_peer_y = s->dp_peer_states;
            go.ep_peer_sumsq = s->dp_peer_sumsq;
            go.ep_peer_flag = s->dp_peer_flag;
            go.ep_done = s->ep_done2;
            go.ep_step = s->step;
            go.ep_layers = int32_t(c.layers);
            go.ep_layer = int32_t(l);
        }
        add_job(go, m, L.o, nullptr, s->states + size_t(f0) * d, d, s->states + size_t(f0) * d, d, EPI_ADD);
        parts = gemv(go, L.o, SPM_GEMV_DENSE, int(l), qbytes(L.o));
        if (is_moe(c)) {
            // routed feed-forward (spm-granite-moe/src/layout.rs:188-333)
            const int E = int(c.experts), K = int(c.experts_used), eff = int(c.expert_ff);
            MoePlan* plan = s->plans + l;
            if (m->world == 1 && m->streams[L.router].pk.dtype == SPM_F32) {
                // one GPU: the router logits and the routing are one launch
                const Packed& rp = m->streams[L.router].pk;
                RouterArgs ra{};
                ra.x = s->states;
                ra.x_stride = d;
                ra.gain = m->gains + L.ffn_norm;
                ra.sumsq = part[1];
                ra.sumsq_parts = parts;
                ra.eps = c.eps;
                ra.w = reinterpret_cast<const float*>(m->tiles(L.router));
                ra.cols = int(rp.cols);
                ra.E = E;
                ra.K = K;
                ra.n = n;
                ra.bias = L.bias >= 0 ? m->gains + L.bias : nullptr;
                ra.logits = s->moe_logits;
                ra.plan = plan;
                ra.counter = s->route_counter;
                timed(SPM_KERNEL_ROUTE, int(l), -1, 0, [&] {
                    CUDA_OK(launch_router_route(ra, st, pdl));
                    return 0;
                });
            } else {
                GemvLaunch gr = gemv_base(m, L.router, s->states, n);
                gr.status = s->status;
                norm_in(gr, L.ffn_norm, 1);
                if (dp) {
                    // every rank's rows of this layer must be in place
                    gr.world = m->world;
                    gr.ep_wait_flags = s->dp_flags;
                    gr.ep_step = s->step;
                    gr.ep_layers = int32_t(c.layers);
                    gr.ep_layer = int32_t(l);
                    gr.wait_ns = s->wait_ns;
                }
                add_job(gr, m, L.router, nullptr, s->moe_logits, E, nullptr, 0, EPI_STORE);
                gemv(gr, L.router, SPM_GEMV_ROUTER, int(l), qbytes(L.router));
                timed(SPM_KERNEL_ROUTE, int(l), -1, 0, [&] {
                    CUDA_OK(launch_route(s->moe_logits, L.bias >= 0 ? m->gains + L.bias : nullptr, n, E, K, m->world, m->rank,
                                         plan, st, pdl));
                    return 0;
                });
            }
            // active experts of this rank, at most; the expert launches fill
            // the SMs once and split the active experts over them (at least
            // the chunks that would give every SM two CTAs with all possible
            // experts active, which bounds a CTA's tiles)
            const int local_max = std::min(s->moe_max_active, (E + m->world - 1) / m->world);
            const int chunks_gu = std::max(1, std::min(eff / kTileRows, (2 * m->sms + local_max - 1) / local_max));
            GemvLaunch ge = gemv_base(m, L.gate_exps, s->states, kMoeMaxClients);
            ge.status = s->status;
            ge.world = m->world;
            ge.rank = m->rank;
            norm_in(ge, L.ffn_norm, 1);
            add_job(ge, m, L.gate_exps, m->tiles(L.up_exps), s->moe_act, eff, nullptr, 0, EPI_SWIGLU);
            ge.plan = plan;
            ge.expert_max = local_max;
            ge.expert_chunks = chunks_gu;
            ge.expert_tiles = uint32_t(eff / kTileRows);
            ge.total_tiles = ge.expert_tiles;
            ge.xmode = 0;
            gemv(ge, L.gate_exps, SPM_GEMV_EXPERT_GATE_UP, int(l), 0);  // bytes from the plan
            const int chunks_d = std::max(1, std::min(d / kTileRows, (2 * m->sms + local_max - 1) / local_max));
            GemvLaunch gx = gemv_base(m, L.down_exps, s->moe_act, kMoeMaxClients);
            gx.status = s->status;
            gx.world = m->world;
            gx.rank = m->rank;
            MoeExchange ex{};
            const float* outs = s->moe_out;
            if (m->world > 1) {
                // rows go to every rank's buffer; the combine waits for all ranks
                if (!s->ep_ready) fail(SPM_E_ARG, "expert parallel session: call spm_session_ep_connect first");
                gx.ep_peer_y = s->ep_peer_y;
                gx.ep_peer_flag = s->ep_peer_flag;
                gx.ep_done = s->ep_done;
                gx.ep_step = s->step;
                gx.ep_layers = int32_t(c.layers);
                gx.ep_layer = int32_t(l);
                ex = MoeExchange{reinterpret_cast<const uint32_t*>(s->ep_region), s->step, m->world, int32_t(c.layers),
                                 int32_t(l), s->ep_xbytes / sizeof(float), s->status, s->wait_ns};
                outs = reinterpret_cast<const float*>(s->ep_region + 512);
            }
            add_job(gx, m, L.down_exps, nullptr, s->moe_out, d, nullptr, 0, EPI_STORE);
            gx.plan = plan;
            gx.expert_max = local_max;
            gx.expert_chunks = chunks_d;
            gx.expert_tiles = uint32_t(d / kTileRows);
            gx.total_tiles = gx.expert_tiles;
            gx.xmode = 1;
            gemv(gx, L.down_exps, SPM_GEMV_EXPERT_DOWN, int(l), 0);
            timed(SPM_KERNEL_COMBINE, int(l), -1, 0, [&] {
                CUDA_OK(launch_combine(plan, outs, d, s->states, d, nl, K, part[0], m->world > 1 ? &ex : nullptr, st, pdl,
                                       f0));
                return 0;
            });
            parts = combine_parts(d, nl);
            continue;
        }
        GemvLaunch gu = gemv_base(m, L.gate, s->states, n);
        gu.status = s->status;
        norm_in(gu, L.ffn_norm, 1);
        add_job(gu, m, L.gate, m->tiles(L.up), s->act, ff, nullptr, 0, EPI_SWIGLU);
        gemv(gu, L.gate, SPM_GEMV_DENSE, int(l), qbytes(L.gate) + qbytes(L.up));
        GemvLaunch gd = gemv_base(m, L.down, s->act, n);
        gd.status = s->status;
        gd.sumsq_out = part[0];
        add_job(gd, m, L.down, nullptr, s->states, d, s->states, d, EPI_ADD);
        parts = gemv(gd, L.down, SPM_GEMV_DENSE, int(l), qbytes(L.down));
    }
    GemvLaunch gh = gemv_base(m, m->head, s->states + size_t(f0) * d, nl);
    gh.status = s->status;
    gh.c0 = f0;
    norm_in(gh, m->output_norm, 0);
    add_job(gh, m, m->head, nullptr, s->logits + size_t(f0) * c.vocab, int(c.vocab), nullptr, 0, EPI_STORE);
    gemv(gh, m->head, SPM_GEMV_HEAD, -1, qbytes(m->head));
    timed(SPM_KERNEL_OTHER, -1, -1, 0, [&] {
        CUDA_OK(launch_argmax(s->logits + size_t(f0) * c.vocab, nl, int(c.vocab), s->argmax + f0, st, pdl));
        return 0;
    });
    if (dp)
        timed(SPM_KERNEL_OTHER, -1, -1, 0, [&] {
            CUDA_OK(launch_ep_gather(s->argmax, s->dp_peer_argmax, s->dp_peer_gflag, s->dp_flags + 128, s->step, f0,
                                     nl, m->world, m->rank, s->status, s->wait_ns, st, pdl));
            return 0;
        });
    timed(SPM_KERNEL_OTHER, -1, -1, 0, [&] {
        CUDA_OK(launch_advance(s->pos, n, s->step, st, pdl));
        return 0;
    });
}

// A bounded device wait that gave up leaves a code in the status word; the
// step's outputs are then not trustworthy.  The word is cleared after reporting.
void check_status(spm_session* s) {
    if (*s->h_status) {
        const int code = *s->h_status;
        *s->h_status = 0;
        cudaMemsetAsync(s->status, 0, sizeof(int32_t), s->stream);
        cudaStreamSynchronize(s->stream);
        fail(SPM_E_TIMEOUT, "a device wait gave up (code " + std::to_string(code) + ")");
    }
}

// After a profiled step: wait for it, count the expert launches' bytes from
// the step's plans (this rank's active experts times one expert's matrices),
// and move the launches' event times into the record.
void collect_profile(spm_session* s) {
    spm_model* m = s->m;
    CUDA_OK(cudaStreamSynchronize(s->stream));
    std::vector<MoePlan> plans;
    if (is_moe(m->cfg)) {
        plans.resize(m->cfg.layers);
        CUDA_OK(cudaMemcpy(plans.data(), s->plans, plans.size() * sizeof(MoePlan), cudaMemcpyDeviceToHost));
    }
    for (auto& p : s->prof_pending) {
        uint64_t bytes = p.bytes;
        if (p.kind == SPM_GEMV_EXPERT_GATE_UP || p.kind == SPM_GEMV_EXPERT_DOWN) {
            const StreamDesc& d = m->streams[p.stream];
            const uint64_t one = d.pk.quant_bytes / d.experts;
            bytes = uint64_t(plans[p.layer].nlocal) * one * (p.kind == SPM_GEMV_EXPERT_GATE_UP ? 2 : 1);
        }
        float ms = 0.f;
        CUDA_OK(cudaEventElapsedTime(&ms, p.a, p.b));
        cudaEventDestroy(p.a);
        cudaEventDestroy(p.b);
        s->prof_ms.push_back(ms);
        s->prof_bytes.push_back(bytes);
        s->prof_kind.push_back(p.kind);
    }
    s->prof_pending.clear();
}

// Client counts above 8 are not batched into one sweep by this build.
constexpr int kMaxBatch = 8;

void step(spm_session* s, int n) {
    if (n < 1 || n > s->max_clients) fail(SPM_E_ARG, "client count out of range");
    if (n > kMaxBatch) fail(SPM_E_ARG, "at most 8 clients share one sweep");
    if (n % s->m->world) fail(SPM_E_ARG, "expert parallel: the client count must be a multiple of the ranks");
    for (int i = 0; i < n; i++)
        if (s->lens[i] >= s->context) fail(SPM_E_CONTEXT, "context " + std::to_string(s->context) + " exhausted");
    if (s->graphs && !s->prof) {
        auto it = s->exec.find(n);
        if (it == s->exec.end()) {
            cudaGraph_t graph;
            CUDA_OK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
            try {
                enqueue_step(s, n);
            } catch (...) {
                cudaStreamEndCapture(s->stream, &graph);
                throw;
            }
            CUDA_OK(cudaStreamEndCapture(s->stream, &graph));
            size_t nodes = 0;
            CUDA_OK(cudaGraphGetNodes(graph, nullptr, &nodes));
            std::vector<cudaGraphNode_t> list(nodes);
            CUDA_OK(cudaGraphGetNodes(graph, list.data(), &nodes));
            int kernels = 0;
            for (auto nd : list) {
                cudaGraphNodeType t;
                CUDA_OK(cudaGraphNodeGetType(nd, &t));
                if (t == cudaGraphNodeTypeKernel) kernels++;
            }
            s->launches[n] = kernels;
            cudaGraphExec_t ge;
            CUDA_OK(cudaGraphInstantiate(&ge, graph, 0));
            cudaGraphDestroy(graph);
            it = s->exec.emplace(n, ge).first;
        }
        CUDA_OK(cudaGraphLaunch(it->second, s->stream));
    } else {
        enqueue_step(s, n);
        if (s->prof) collect_profile(s);
    }
    for (int i = 0; i < n; i++) s->lens[i]++;
}

// ---- prompts on the tensor cores ----
// Rows per prompt chunk; longer prompts run chunk after chunk (a chunk's
// attention reads the earlier chunks' keys and values from the cache).
constexpr int kPrefillRows = 1024;

void prefill_buffers(spm_session* s) {
    auto& P = s->pf;
    if (P.rows) return;
    const spm_model_cfg& c = s->m->cfg;
    const size_t T = kPrefillRows, d = c.hidden, qw = size_t(c.heads) * c.head_dim, kvw = size_t(c.kv_heads) * c.head_dim;
    P.tokens = s->alloc<uint32_t>(T);
    P.qpos = s->alloc<int32_t>(T);
    P.x = s->alloc<float>(T * d);
    P.xn = s->alloc<float>(T * d);
    P.q = s->alloc<float>(T * qw);
    P.k = s->alloc<float>(T * kvw);
    P.v = s->alloc<float>(T * kvw);
    P.attn = s->alloc<float>(T * qw);
    if (is_moe(c)) {
        const size_t E = c.experts, K = c.experts_used, R = T * K;
        P.logits = s->alloc<float>(T * E);
        P.sel = s->alloc<int32_t>(R);
        P.prob = s->alloc<float>(R);
        P.norm = s->alloc<float>(T);
        P.counts = s->alloc<int32_t>(E);
        P.offsets = s->alloc<int32_t>(E);
        P.cursor = s->alloc<int32_t>(E);
        P.list = s->alloc<int32_t>(R);
        P.slot = s->alloc<int32_t>(R);
        P.groups = s->alloc<int4>(R / 128 + E + 1);
        P.ge = s->alloc<float>(R * c.expert_ff);
        P.ue = s->alloc<float>(R * c.expert_ff);
        P.ye = s->alloc<float>(R * d);
    } else {
        P.g = s->alloc<float>(T * c.intermediate);
        P.u = s->alloc<float>(T * c.intermediate);
    }
    P.rows = int(T);
}

// y = x W^T for T rows on the tensor cores (plain or with residual / SwiGLU input).
void gemm_rows(spm_session* s, int idx, const float* x, const float* x2, int T, float* y, int epi) {
    spm_model* m = s->m;
    const Packed& p = m->streams[idx].pk;
    GemmArgs a{};
    a.w = m->tiles(idx);
    a.pk = p;
    a.x = x;
    a.x2 = x2;
    a.x_stride = int32_t(p.cols);
    a.tokens = T;
    a.y = y;
    a.y_stride = int32_t(p.rows);
    a.aux = y;
    a.aux_stride = int32_t(p.rows);
    a.epi = epi;
    a.status = s->status;
    CUDA_OK(launch_prefill_gemm(a, s->stream));
}

// One chunk of a prompt: T tokens of `client` at positions pos0.. (the
// decode step's layer schedule, every position of the chunk at once).
void prefill_chunk(spm_session* s, int client, const uint32_t* tokens, int T, int pos0) {
    spm_model* m = s->m;
    const spm_model_cfg& c = m->cfg;
    auto& P = s->pf;
    cudaStream_t st = s->stream;
    const int d = int(c.hidden);
    std::vector<int32_t> qpos(T);
    for (int t = 0; t < T; t++) qpos[t] = pos0 + t;
    CUDA_OK(cudaMemcpyAsync(P.tokens, tokens, size_t(T) * sizeof(uint32_t), cudaMemcpyHostToDevice, st));
    CUDA_OK(cudaMemcpyAsync(P.qpos, qpos.data(), size_t(T) * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    const StreamDesc& E = m->streams[m->embed];
    CUDA_OK(launch_embed_rows(E.pk.dtype, m->tiles(m->embed), E.pk, P.tokens, T, P.x, st));
    std::vector<int32_t> counts, offsets;
    std::vector<int4> groups;
    for (uint32_t l = 0; l < c.layers; l++) {
        const LayerIdx& L = m->layers[l];
        CUDA_OK(launch_norm_rows(P.x, m->gains + L.attn_norm, c.eps, d, T, P.xn, st));
        gemm_rows(s, L.q, P.xn, nullptr, T, P.q, EPI_STORE);
        gemm_rows(s, L.k, P.xn, nullptr, T, P.k, EPI_STORE);
        gemm_rows(s, L.v, P.xn, nullptr, T, P.v, EPI_STORE);
        QkArgs q{};
        q.q = P.q; q.k = P.k; q.v = P.v; q.kcache = s->kc; q.vcache = s->vc; q.rope = s->rope;
        q.kplanes = s->kp; q.vplanes = s->vp;
        q.q_norm = L.q_norm >= 0 ? m->gains + L.q_norm : nullptr;
        q.k_norm = L.k_norm >= 0 ? m->gains + L.k_norm : nullptr;
        q.client = client; q.layer = int(l); q.layers = int(c.layers); q.context = s->context; q.pos0 = pos0;
        q.heads = int(c.heads); q.kv_heads = int(c.kv_heads); q.head_dim = int(c.head_dim); q.family = int(c.family);
        q.eps = c.eps;
        CUDA_OK(launch_qk_rope_append(q, T, st));
        AttnParams A{};
        A.q = P.q; A.out = P.attn; A.kcache = s->kc; A.vcache = s->vc; A.rope = s->rope;
        A.layer = int(l); A.layers = int(c.layers); A.context = s->context;
        A.heads = int(c.heads); A.kv_heads = int(c.kv_heads); A.head_dim = int(c.head_dim);
        A.family = int(c.family); A.eps = c.eps; A.status = s->status;
        A.qpos = P.qpos; A.cache_client = client;
        CUDA_OK(launch_attention_queries(A, T, st));
        gemm_rows(s, L.o, P.attn, nullptr, T, P.x, EPI_ADD);
        CUDA_OK(launch_norm_rows(P.x, m->gains + L.ffn_norm, c.eps, d, T, P.xn, st));
        if (!is_moe(c)) {
            gemm_rows(s, L.gate, P.xn, nullptr, T, P.g, EPI_STORE);
            gemm_rows(s, L.up, P.xn, nullptr, T, P.u, EPI_STORE);
            gemm_rows(s, L.down, P.g, P.u, T, P.x, EPI_ADD);
            continue;
        }
        // routed feed-forward: route every row, group the rows by expert, run
        // each expert over its group, combine in ascending expert id
        const int Ex = int(c.experts), K = int(c.experts_used), eff = int(c.expert_ff);
        gemm_rows(s, L.router, P.xn, nullptr, T, P.logits, EPI_STORE);
        CUDA_OK(cudaMemsetAsync(P.counts, 0, size_t(Ex) * sizeof(int32_t), st));
        CUDA_OK(launch_route_rows(P.logits, L.bias >= 0 ? m->gains + L.bias : nullptr, T, Ex, K, P.sel, P.prob,
                                  P.norm, P.counts, st));
        counts.resize(Ex);
        CUDA_OK(cudaMemcpyAsync(counts.data(), P.counts, size_t(Ex) * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
        CUDA_OK(cudaStreamSynchronize(st));
        offsets.assign(Ex, 0);
        groups.clear();
        int run = 0;
        for (int e = 0; e < Ex; e++) {
            offsets[e] = run;
            for (int g0 = 0; g0 < counts[e]; g0 += 128) groups.push_back(make_int4(e, run + g0, std::min(128, counts[e] - g0), 0));
            run += counts[e];
        }
        if (run != T * K) fail(SPM_E_CUDA, "prefill routing lost rows");
        CUDA_OK(cudaMemcpyAsync(P.offsets, offsets.data(), size_t(Ex) * sizeof(int32_t), cudaMemcpyHostToDevice, st));
        CUDA_OK(cudaMemcpyAsync(P.groups, groups.data(), groups.size() * sizeof(int4), cudaMemcpyHostToDevice, st));
        CUDA_OK(cudaMemsetAsync(P.cursor, 0, size_t(Ex) * sizeof(int32_t), st));
        CUDA_OK(launch_scatter_rows(P.sel, T, K, P.offsets, P.cursor, P.list, P.slot, st));
        auto grouped = [&](int idx, const float* x, const float* x2, const int32_t* xi, float* y) {
            const StreamDesc& S = m->streams[idx];
            GemmArgs a{};
            a.w = m->tiles(idx);
            a.pk = packed_shape(S.pk.dtype, S.pk.rows / S.experts, S.pk.cols);  // one expert's matrix
            a.w_stride = a.pk.tiles * a.pk.tile_bytes;
            a.x = x;
            a.x2 = x2;
            a.x_index = xi;
            a.x_stride = int32_t(S.pk.cols);
            a.y = y;
            a.y_stride = int32_t(a.pk.rows);
            a.epi = EPI_STORE;
            a.status = s->status;
            a.groups = P.groups;
            a.ngroups = int32_t(groups.size());
            CUDA_OK(launch_prefill_gemm(a, st));
        };
        grouped(L.gate_exps, P.xn, nullptr, P.list, P.ge);
        grouped(L.up_exps, P.xn, nullptr, P.list, P.ue);
        grouped(L.down_exps, P.ge, P.ue, nullptr, P.ye);
        (void)eff;
        CUDA_OK(launch_combine_rows(P.sel, P.prob, P.norm, P.slot, P.ye, P.x, T, K, d, st));
    }
}

// Host-computed rotary table so that cos/sin are the oracle's glibc values:
// LLAMA spm-ops/src/attention.rs:20-27, others spm-qwen3-slice/src/attention.rs:11-19.
std::vector<float2> rope_table(const spm_model_cfg& c, int context) {
    const int half = int(c.head_dim / 2);
    std::vector<float2> t(size_t(context) * half);
    for (int pos = 0; pos < context; pos++)
        for (int i = 0; i < half; i++) {
            float theta;
            if (c.family == SPM_FAMILY_LLAMA) {
                const float width = float(c.head_dim), at = float(pos > 65535 ? 65535 : pos), index = float(i);
                theta = powf(c.rope_base, -2.0f * index / width) * at;
            } else {
                const float exponent = 2.0f * float(i) / float(c.head_dim);
                theta = float(pos) / powf(c.rope_base, exponent);
            }
            t[size_t(pos) * half + i] = make_float2(cosf(theta), sinf(theta));
        }
    return t;
}

}  // namespace

// ================================================================== C ABI ==
extern "C" {

const char* spm_last_error(void) { return spm::last_error().c_str(); }
const char* spm_version(void) { return "emufpga-b200 0.1 (sm_100a)"; }
void spm_free(void* p) { std::free(p); }

spm_status spm_synth_gguf(const spm_synth_spec* spec, uint8_t** out, uint64_t* len) {
    return guarded([&] {
        if (!spec || !out || !len) fail(SPM_E_ARG, "null argument");
        *out = synth_gguf(*spec, len);
    });
}

spm_status spm_gguf_probe(const uint8_t* buf, uint64_t len, uint64_t* tensors, uint64_t* data_offset) {
    return guarded([&] {
        if (!buf && len) fail(SPM_E_ARG, "null buffer");
        Gguf g = gguf_parse(buf, len);
        if (tensors) *tensors = g.tensors.size();
        if (data_offset) *data_offset = g.data_offset;
    });
}

spm_status spm_gguf_probe_file(const char* path, uint64_t* tensors, uint64_t* data_offset) {
    return guarded([&] {
        std::string s = read_file(path);
        Gguf g = gguf_parse(reinterpret_cast<const uint8_t*>(s.data()), s.size());
        if (tensors) *tensors = g.tensors.size();
        if (data_offset) *data_offset = g.data_offset;
    });
}

spm_status spm_gguf_find(const uint8_t* buf, uint64_t len, const char* name, uint32_t* dtype, uint64_t* dims4,
                         uint64_t* offset, uint64_t* nbytes) {
    return guarded([&] {
        Gguf g = gguf_parse(buf, len);
        const GgufTensor* t = g.find(name ? name : "");
        if (!t) fail(SPM_E_STREAM, std::string("no tensor named ") + (name ? name : ""));
        if (dtype) *dtype = t->dtype;
        if (dims4)
            for (int d = 0; d < 4; d++) dims4[d] = d < int(t->dims.size()) ? t->dims[d] : 1;
        if (offset) *offset = t->offset;
        if (nbytes) *nbytes = t->len;
    });
}

spm_status spm_decode_blocks(uint32_t dtype, const uint8_t* bytes, uint64_t nbytes, float* out) {
    return guarded([&] { decode_blocks(dtype, bytes, nbytes, out); });
}

spm_status spm_order_check(const char* text, const uint8_t* gguf, uint64_t len) {
    return guarded([&] { check_order(parse_order(text ? text : ""), gguf_parse(gguf, len)); });
}

spm_status spm_order_default(const spm_model_cfg* cfg, const uint8_t* gguf, uint64_t len, char** text) {
    return guarded([&] {
        bool bias = false;
        if (gguf) bias = gguf_parse(gguf, len).find("blk.0.exp_probs_b.bias") != nullptr;
        std::string s = default_order(*cfg, bias);
        *text = static_cast<char*>(std::malloc(s.size() + 1));
        std::memcpy(*text, s.c_str(), s.size() + 1);
    });
}

spm_status spm_model_open(const char* gguf_path, const char* order_path, const spm_model_cfg* cfg, int device,
                          spm_model** out) {
    return guarded([&] {
        Mapped img(gguf_path);
        std::string order;
        if (order_path) order = read_file(order_path);
        *out = open_model(img.p, img.n, order_path ? &order : nullptr, cfg, device);
    });
}

spm_status spm_model_open_memory(const uint8_t* gguf, uint64_t len, const char* order_text, const spm_model_cfg* cfg,
                                 int device, spm_model** out) {
    return guarded([&] {
        std::string order = order_text ? order_text : "";
        *out = open_model(gguf, len, order_text ? &order : nullptr, cfg, device);
    });
}

spm_status spm_model_open_ep(const char* gguf_path, const char* order_path, const spm_model_cfg* cfg, int device,
                             int32_t world, int32_t rank, spm_model** out) {
    return guarded([&] {
        Mapped img(gguf_path);
        std::string order;
        if (order_path) order = read_file(order_path);
        *out = open_model(img.p, img.n, order_path ? &order : nullptr, cfg, device, world, rank);
    });
}

spm_status spm_model_open_memory_ep(const uint8_t* gguf, uint64_t len, const char* order_text,
                                    const spm_model_cfg* cfg, int device, int32_t world, int32_t rank,
                                    spm_model** out) {
    return guarded([&] {
        std::string order = order_text ? order_text : "";
        *out = open_model(gguf, len, order_text ? &order : nullptr, cfg, device, world, rank);
    });
}

spm_status spm_pack_image(const uint8_t* gguf, uint64_t len, const char* order_text, const spm_model_cfg* cfg,
                          const char* path) {
    return guarded([&] {
        std::string order = order_text ? order_text : "";
        write_image(gguf, len, order_text ? &order : nullptr, cfg, path);
    });
}

spm_status spm_image_probe(const char* path, uint64_t* image_bytes, int32_t* streams) {
    return guarded([&] {
        Mapped f(path);
        uint64_t data = 0;
        ModelDesc d = read_image(f.p, f.n, &data);
        if (image_bytes) *image_bytes = d.image_bytes;
        if (streams) *streams = int32_t(d.streams.size());
    });
}

spm_status spm_model_open_image(const char* path, int device, spm_model** out) {
    return guarded([&] {
        Mapped f(path);
        uint64_t data = 0;
        ModelDesc d = read_image(f.p, f.n, &data);
        const uint64_t bytes = d.image_bytes;
        *out = make_model(std::move(d), device, 1, 0, [&](spm_model* m) {
            CUDA_OK(cudaMemcpy(m->image, f.p + data, bytes, cudaMemcpyHostToDevice));  // one sequential upload
        });
    });
}

spm_status spm_model_close(spm_model* m) {
    return guarded([&] {
        if (m) cudaSetDevice(m->device);
        delete m;
    });
}

spm_status spm_model_weight_bytes(const spm_model* m, uint64_t* bytes) {
    return guarded([&] { *bytes = m->weight_bytes; });
}

spm_status spm_model_stream_count(const spm_model* m, int32_t* streams) {
    return guarded([&] { *streams = int32_t(m->streams.size()); });
}

spm_status spm_model_stream_info(const spm_model* m, int32_t index, uint64_t* rows, uint64_t* cols, uint32_t* dtype,
                                 uint64_t* bytes) {
    return guarded([&] {
        if (index < 0 || index >= int32_t(m->streams.size())) fail(SPM_E_ARG, "stream index out of range");
        const Packed& p = m->streams[index].pk;
        if (rows) *rows = p.rows;
        if (cols) *cols = p.cols;
        if (dtype) *dtype = p.dtype;
        if (bytes) *bytes = p.quant_bytes;
    });
}

spm_status spm_model_stream_index(const spm_model* m, const char* name, int32_t* index) {
    return guarded([&] {
        for (size_t i = 0; i < m->streams.size(); i++)
            if (m->streams[i].name == name) { *index = int32_t(i); return; }
        fail(SPM_E_ARG, std::string("no stream named ") + name);
    });
}

spm_status spm_dequant_rows(const spm_model* m, int32_t index, uint64_t row0, uint64_t rows, float* out_host) {
    return guarded([&] {
        if (index < 0 || index >= int32_t(m->streams.size())) fail(SPM_E_ARG, "stream index out of range");
        const Packed& p = m->streams[index].pk;
        if (row0 > p.rows || rows > p.rows - row0) fail(SPM_E_ARG, "row range exceeds the matrix");
        CUDA_OK(cudaSetDevice(m->device));
        DeviceBuf out;
        CUDA_OK(cudaMalloc(&out.p, std::max<uint64_t>(rows * p.cols, 1) * sizeof(float)));
        CUDA_OK(launch_dequant(p.dtype, m->tiles(index), p, row0, rows, static_cast<float*>(out.p), nullptr));
        CUDA_OK(cudaMemcpy(out_host, out.p, rows * p.cols * sizeof(float), cudaMemcpyDeviceToHost));
    });
}

// Positions from which a product over one matrix runs on the tensor cores
// (prefill_gemm.cu) instead of streaming GEMVs of up to eight positions.
static constexpr int32_t kTensorPositions = 16;

// y = x W^T for `positions` rows of x on the tensor cores, when the shapes allow.
static bool tensor_product(const uint8_t* tiles, const Packed& p, const float* x, int32_t positions, float* y,
                    cudaStream_t st, int32_t* status) {
    if (positions < kTensorPositions || p.cols % 64 || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
    GemmArgs a{};
    a.w = tiles;
    a.pk = p;
    a.x = x;
    a.x_stride = int32_t(p.cols);
    a.tokens = positions;
    a.y = y;
    a.y_stride = int32_t(p.rows);
    a.epi = EPI_STORE;
    a.status = status;
    CUDA_OK(launch_prefill_gemm(a, st));
    return true;
}

spm_status spm_streamed(const spm_model* m, int32_t index, const float* x_dev, int32_t positions, float* y_dev,
                        void* cuda_stream) {
    return guarded([&] {
        if (index < 0 || index >= int32_t(m->streams.size())) fail(SPM_E_ARG, "stream index out of range");
        if (positions < 0) fail(SPM_E_ACTIVATION_LEN, "negative position count");
        if (positions > 0 && (!x_dev || !y_dev)) fail(SPM_E_ARG, "null activation or output pointer");
        CUDA_OK(cudaSetDevice(m->device));
        const Packed& p = m->streams[index].pk;
        if (tensor_product(m->tiles(index), p, x_dev, positions, y_dev, static_cast<cudaStream_t>(cuda_stream),
                           nullptr))
            return;
        for (int32_t p0 = 0; p0 < positions; p0 += kMaxBatch) {
            const int n = std::min(kMaxBatch, positions - p0);
            GemvLaunch L = gemv_base(m, index, x_dev + size_t(p0) * p.cols, n);
            add_job(L, m, index, nullptr, y_dev + size_t(p0) * p.rows, int(p.rows), nullptr, 0, EPI_STORE);
            run_gemv(m, L, p.dtype, static_cast<cudaStream_t>(cuda_stream), false);
        }
    });
}

spm_status spm_weights_upload(uint32_t dtype, uint64_t rows, uint64_t cols, const uint8_t* blocks, int device,
                              spm_weights** out) {
    return guarded([&] {
        std::unique_ptr<spm_weights> w(new spm_weights());
        w->pk = packed_shape(dtype, rows, cols);
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) fail(SPM_E_NO_DEVICE, "no CUDA device is visible");
        w->device = device;
        CUDA_OK(cudaSetDevice(device));
        CUDA_OK(cudaDeviceGetAttribute(&w->sms, cudaDevAttrMultiProcessorCount, device));
        std::vector<uint8_t> host(w->pk.tiles * w->pk.tile_bytes);
        pack_matrix(w->pk, blocks, host.data());
        CUDA_OK(cudaMalloc(&w->dev, host.size()));
        CUDA_OK(cudaMemcpy(w->dev, host.data(), host.size(), cudaMemcpyHostToDevice));
        *out = w.release();
    });
}

spm_status spm_weights_free(spm_weights* w) {
    return guarded([&] { delete w; });
}

spm_status spm_weights_gemv(const spm_weights* w, const float* x_dev, int32_t positions, float* y_dev,
                            void* cuda_stream) {
    return guarded([&] {
        if (positions < 0) fail(SPM_E_ACTIVATION_LEN, "negative position count");
        CUDA_OK(cudaSetDevice(w->device));
        const Packed& p = w->pk;
        if (tensor_product(w->dev, p, x_dev, positions, y_dev, static_cast<cudaStream_t>(cuda_stream), nullptr))
            return;
        for (int32_t p0 = 0; p0 < positions; p0 += kMaxBatch) {
            const int n = std::min(kMaxBatch, positions - p0);
            GemvLaunch L{};
            L.cols = uint32_t(p.cols);
            L.tile_bytes = uint32_t(p.tile_bytes);
            L.plane1 = p.plane[1];
            L.plane2 = p.plane[2];
            L.plane3 = p.plane[3];
            L.x = x_dev + size_t(p0) * p.cols;
            L.x_stride = int(p.cols);
            L.n = n;
            GemvJob& J = L.job[L.njobs++];
            J.a = w->dev;
            J.y = y_dev + size_t(p0) * p.rows;
            J.y_stride = int(p.rows);
            J.rows = uint32_t(p.rows);
            J.epi = EPI_STORE;
            L.total_tiles = uint32_t(p.tiles);
            CUDA_OK(launch_gemv(p.dtype, L, w->sms, static_cast<cudaStream_t>(cuda_stream), false));
        }
    });
}

spm_status spm_weights_dequant(const spm_weights* w, uint64_t row0, uint64_t rows, float* out_host) {
    return guarded([&] {
        const Packed& p = w->pk;
        if (row0 > p.rows || rows > p.rows - row0) fail(SPM_E_ARG, "row range exceeds the matrix");
        CUDA_OK(cudaSetDevice(w->device));
        DeviceBuf out;
        CUDA_OK(cudaMalloc(&out.p, std::max<uint64_t>(rows * p.cols, 1) * sizeof(float)));
        CUDA_OK(launch_dequant(p.dtype, w->dev, p, row0, rows, static_cast<float*>(out.p), nullptr));
        CUDA_OK(cudaMemcpy(out_host, out.p, rows * p.cols * sizeof(float), cudaMemcpyDeviceToHost));
    });
}

spm_status spm_session_create(spm_model* m, int32_t max_clients, int32_t max_context, spm_session** out) {
    return guarded([&] {
        if (max_clients < 1 || max_context < 1) fail(SPM_E_ARG, "clients and context must be positive");
        CUDA_OK(cudaSetDevice(m->device));
        std::unique_ptr<spm_session> s(new spm_session());
        s->m = m;
        s->max_clients = max_clients;
        s->context = max_context;
        const spm_model_cfg& c = m->cfg;
        const size_t n = size_t(max_clients), d = c.hidden, qw = size_t(c.heads) * c.head_dim;
        const size_t kvw = size_t(c.kv_heads) * c.head_dim;
        const size_t ff = std::max<size_t>(c.intermediate, c.expert_ff);
        CUDA_OK(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
        s->kc = s->alloc<float>(n * c.layers * size_t(max_context) * kvw);
        s->vc = s->alloc<float>(n * c.layers * size_t(max_context) * kvw);
        {
            const uint32_t grp = c.heads / c.kv_heads;
            if (grp >= 4 && grp <= 8 && (c.head_dim == 64 || c.head_dim == 128)) {
                s->kp = s->alloc<uint16_t>(3 * n * c.layers * size_t(max_context) * kvw);
                s->vp = s->alloc<uint16_t>(3 * n * c.layers * size_t(max_context) * kvw);
            }
        }
        s->normed = s->alloc<float>(n * d);
        s->q = s->alloc<float>(n * qw);
        s->k = s->alloc<float>(n * kvw);
        s->v = s->alloc<float>(n * kvw);
        s->attn = s->alloc<float>(n * qw);
        s->act = s->alloc<float>(n * ff);
        s->logits = s->alloc<float>(n * c.vocab);
        s->pos = s->alloc<int32_t>(n);
        s->tokens = s->alloc<uint32_t>(n);
        s->status = s->alloc<int32_t>(1);
        const size_t chunks = (size_t(max_context) + kAttnMinChunk - 1) / kAttnMinChunk;
        const size_t group = c.heads / c.kv_heads;
        // the attention kernel splits a score over 8 / group warps, four values at a time
        if (group > 8 || group * c.head_dim > 1024 || c.head_dim > 256 || c.head_dim % (4 * (8 / group)))
            fail(SPM_E_ARG, "attention supports at most 8 query heads and 1024 query values per kv head, "
                            "head_dim up to 256 and a multiple of 4 * (8 / group)");
        s->attn_scratch = s->alloc<float>(n * c.kv_heads * chunks * group * (c.head_dim + 2));
        s->attn_counters = s->alloc<int32_t>(n * c.kv_heads);
        if (is_moe(c)) {
            if (c.experts > uint32_t(kMoeMaxExperts) || c.experts_used > uint32_t(kMoeMaxUsed))
                fail(SPM_E_ARG, "at most 256 experts and 8 routed per token");
            if (c.expert_ff % kTileRows || c.hidden % kTileRows) fail(SPM_E_ARG, "expert rows must be whole tiles");
            s->moe_max_active = int(std::min<size_t>(c.experts, std::min<size_t>(n, kMoeMaxClients) * c.experts_used));
            s->moe_logits = s->alloc<float>(n * c.experts);
            s->route_counter = s->alloc<uint32_t>(1);
            s->plans = s->alloc<MoePlan>(c.layers);
            s->moe_act = s->alloc<float>(size_t(s->moe_max_active) * kMoeMaxClients * c.expert_ff);
            s->moe_out = s->alloc<float>(size_t(s->moe_max_active) * kMoeMaxClients * c.hidden);
            if (m->world > 1) {
                s->ep_xbytes = (size_t(s->moe_max_active) * kMoeMaxClients * c.hidden * sizeof(float) + 255) & ~size_t(255);
                // after the exchange: flags [2][64] + [64], greedy picks,
                // states, sums of squares (every rank writes into them)
                s->dp_off = 512 + 2 * s->ep_xbytes;
                const size_t pick_off = 1024, states_off = pick_off + ((n * sizeof(uint32_t) + 255) & ~size_t(255));
                s->dp_states_bytes = (n * d * sizeof(float) + 255) & ~size_t(255);
                const size_t sumsq_off = states_off + s->dp_states_bytes;
                const size_t dp_bytes = sumsq_off + 2 * size_t(kMaxParts) * 8 * sizeof(float);
                s->ep_region = s->alloc<uint8_t>(s->dp_off + dp_bytes);
                uint8_t* dp = s->ep_region + s->dp_off;
                s->dp_flags = reinterpret_cast<uint32_t*>(dp);
                s->argmax = reinterpret_cast<uint32_t*>(dp + pick_off);
                s->states = reinterpret_cast<float*>(dp + states_off);
                s->sumsq = reinterpret_cast<float*>(dp + sumsq_off);
                s->ep_done = s->alloc<uint32_t>(1);
                s->ep_done2 = s->alloc<uint32_t>(1);
                s->ep_peer_y = s->alloc<float*>(2 * size_t(m->world));
                s->ep_peer_flag = s->alloc<uint32_t*>(2 * size_t(m->world));
                s->dp_peer_states = s->alloc<float*>(m->world);
                s->dp_peer_sumsq = s->alloc<float*>(m->world);
                s->dp_peer_flag = s->alloc<uint32_t*>(2 * size_t(m->world));
                s->dp_peer_argmax = s->alloc<uint32_t*>(m->world);
                s->dp_peer_gflag = s->alloc<uint32_t*>(m->world);
            }
        }
        if (!s->states) {
            s->states = s->alloc<float>(n * d);
            s->argmax = s->alloc<uint32_t>(n);
            s->sumsq = s->alloc<float>(2 * size_t(kMaxParts) * 8);
        }
        s->step = s->alloc<uint32_t>(1);
        auto table = rope_table(c, max_context);
        s->rope = s->alloc<float2>(table.size());
        CUDA_OK(cudaMemcpy(s->rope, table.data(), table.size() * sizeof(float2), cudaMemcpyHostToDevice));
        CUDA_OK(cudaMallocHost(&s->h_tokens, n * sizeof(uint32_t)));
        CUDA_OK(cudaMallocHost(&s->h_argmax, n * sizeof(uint32_t)));
        CUDA_OK(cudaMallocHost(&s->h_status, sizeof(int32_t)));
        s->lens.assign(n, 0);
        *out = s.release();
    });
}

spm_status spm_session_destroy(spm_session* s) {
    return guarded([&] {
        if (s) cudaSetDevice(s->m->device);
        delete s;
    });
}

spm_status spm_client_reset(spm_session* s, int32_t client) {
    return guarded([&] {
        if (client < 0 || client >= s->max_clients) fail(SPM_E_ARG, "client index out of range");
        CUDA_OK(cudaSetDevice(s->m->device));
        CUDA_OK(cudaMemsetAsync(s->pos + client, 0, sizeof(int32_t), s->stream));
        CUDA_OK(cudaStreamSynchronize(s->stream));
        s->lens[client] = 0;
    });
}

spm_status spm_client_len(const spm_session* s, int32_t client, int32_t* len) {
    return guarded([&] {
        if (client < 0 || client >= s->max_clients) fail(SPM_E_ARG, "client index out of range");
        *len = s->lens[client];
    });
}

spm_status spm_decode_step(spm_session* s, const uint32_t* tokens, int32_t n, float* logits_host,
                           uint32_t* argmax_host) {
    return guarded([&] {
        if (n < 1 || n > s->max_clients) fail(SPM_E_ARG, "client count out of range");
        for (int i = 0; i < n; i++)
            if (tokens[i] >= s->m->cfg.vocab) fail(SPM_E_ARG, "token id out of range");
        CUDA_OK(cudaSetDevice(s->m->device));
        std::memcpy(s->h_tokens, tokens, size_t(n) * sizeof(uint32_t));
        CUDA_OK(cudaMemcpyAsync(s->tokens, s->h_tokens, size_t(n) * sizeof(uint32_t), cudaMemcpyHostToDevice, s->stream));
        step(s, n);
        if (argmax_host)
            CUDA_OK(cudaMemcpyAsync(s->h_argmax, s->argmax, size_t(n) * sizeof(uint32_t), cudaMemcpyDeviceToHost, s->stream));
        if (logits_host)
            CUDA_OK(cudaMemcpyAsync(logits_host, s->logits, size_t(n) * s->m->cfg.vocab * sizeof(float),
                                    cudaMemcpyDeviceToHost, s->stream));
        CUDA_OK(cudaMemcpyAsync(s->h_status, s->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s->stream));
        CUDA_OK(cudaStreamSynchronize(s->stream));
        check_status(s);
        if (argmax_host) std::memcpy(argmax_host, s->h_argmax, size_t(n) * sizeof(uint32_t));
    });
}

spm_status spm_decode_step_device(spm_session* s, const uint32_t* tokens_dev, int32_t n, float* logits_dev,
                                  uint32_t* argmax_dev) {
    return guarded([&] {
        if (n < 1 || n > s->max_clients) fail(SPM_E_ARG, "client count out of range");
        CUDA_OK(cudaSetDevice(s->m->device));
        if (tokens_dev != s->tokens)
            CUDA_OK(cudaMemcpyAsync(s->tokens, tokens_dev, size_t(n) * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s->stream));
        step(s, n);
        if (argmax_dev)
            CUDA_OK(cudaMemcpyAsync(argmax_dev, s->argmax, size_t(n) * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s->stream));
        if (logits_dev)
            CUDA_OK(cudaMemcpyAsync(logits_dev, s->logits, size_t(n) * s->m->cfg.vocab * sizeof(float),
                                    cudaMemcpyDeviceToDevice, s->stream));
    });
}

spm_status spm_prefill(spm_session* s, int32_t client, const uint32_t* tokens, int32_t len) {
    return guarded([&] {
        spm_model* m = s->m;
        if (client < 0 || client >= s->max_clients) fail(SPM_E_ARG, "client index out of range");
        if (len < 0 || (len > 0 && !tokens)) fail(SPM_E_ARG, "bad prompt");
        if (m->world > 1) fail(SPM_E_ARG, "prefill runs on single-GPU models");
        for (int32_t t = 0; t < len; t++)
            if (tokens[t] >= m->cfg.vocab) fail(SPM_E_ARG, "token id out of range");
        if (int64_t(s->lens[client]) + len > s->context)
            fail(SPM_E_CONTEXT, "context " + std::to_string(s->context) + " exhausted");
        if (m->streams[m->embed].pk.cols % 64) fail(SPM_E_ARG, "prefill needs hidden a multiple of 64");
        CUDA_OK(cudaSetDevice(m->device));
        prefill_buffers(s);
        for (int32_t t0 = 0; t0 < len; t0 += kPrefillRows) {
            const int T = std::min(kPrefillRows, len - t0);
            prefill_chunk(s, client, tokens + t0, T, s->lens[client]);
            s->lens[client] += T;
        }
        const int32_t pos = s->lens[client];
        CUDA_OK(cudaMemcpyAsync(s->pos + client, &pos, sizeof(int32_t), cudaMemcpyHostToDevice, s->stream));
        CUDA_OK(cudaMemcpyAsync(s->h_status, s->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s->stream));
        CUDA_OK(cudaStreamSynchronize(s->stream));
        check_status(s);
    });
}

spm_status spm_session_sync(spm_session* s) {
    return guarded([&] {
        CUDA_OK(cudaMemcpyAsync(s->h_status, s->status, sizeof(int32_t), cudaMemcpyDeviceToHost, s->stream));
        CUDA_OK(cudaStreamSynchronize(s->stream));
        check_status(s);
    });
}

spm_status spm_session_stream(const spm_session* s, void** cuda_stream) {
    return guarded([&] { *cuda_stream = s->stream; });
}

spm_status spm_session_set_graphs(spm_session* s, int32_t enable) {
    return guarded([&] { s->graphs = enable != 0; });
}

spm_status spm_session_routes(const spm_session* s, int32_t n, int32_t* routes_host) {
    return guarded([&] {
        const spm_model_cfg& c = s->m->cfg;
        if (!is_moe(c)) fail(SPM_E_ARG, "the model has no routed layers");
        if (n < 1 || n > s->max_clients || n > kMoeMaxClients) fail(SPM_E_ARG, "client count out of range");
        std::vector<MoePlan> plans(c.layers);
        CUDA_OK(cudaMemcpy(plans.data(), s->plans, c.layers * sizeof(MoePlan), cudaMemcpyDeviceToHost));
        for (uint32_t l = 0; l < c.layers; l++)
            for (int i = 0; i < n; i++)
                for (uint32_t j = 0; j < c.experts_used; j++)
                    routes_host[(size_t(l) * n + i) * c.experts_used + j] = plans[l].route[i][j];
    });
}

spm_status spm_session_route_gaps(const spm_session* s, int32_t n, float* gaps_host) {
    return guarded([&] {
        const spm_model_cfg& c = s->m->cfg;
        if (!is_moe(c)) fail(SPM_E_ARG, "the model has no routed layers");
        if (n < 1 || n > s->max_clients || n > kMoeMaxClients) fail(SPM_E_ARG, "client count out of range");
        std::vector<MoePlan> plans(c.layers);
        CUDA_OK(cudaMemcpy(plans.data(), s->plans, c.layers * sizeof(MoePlan), cudaMemcpyDeviceToHost));
        for (uint32_t l = 0; l < c.layers; l++)
            for (int i = 0; i < n; i++) gaps_host[size_t(l) * n + i] = plans[l].gap[i];
    });
}

spm_status spm_session_ep_handle(spm_session* s, void* handle) {
    return guarded([&] {
        if (s->m->world < 2) fail(SPM_E_ARG, "the model is not expert parallel");
        CUDA_OK(cudaSetDevice(s->m->device));
        cudaIpcMemHandle_t h;
        CUDA_OK(cudaIpcGetMemHandle(&h, s->ep_region));
        static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
        std::memcpy(handle, &h, sizeof(h));
    });
}

spm_status spm_session_ep_connect(spm_session* s, const void* handles) {
    return guarded([&] {
        const int world = s->m->world, rank = s->m->rank;
        if (world < 2) fail(SPM_E_ARG, "the model is not expert parallel");
        if (s->ep_ready) fail(SPM_E_ARG, "the session is already connected");
        CUDA_OK(cudaSetDevice(s->m->device));
        std::vector<uint8_t*> base(world);
        cudaIpcMemHandle_t own;
        CUDA_OK(cudaIpcGetMemHandle(&own, s->ep_region));
        for (int p = 0; p < world; p++) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t*>(handles) + size_t(p) * 64, sizeof(h));
            // this session's own handle (its own rank, or a rank slot a caller
            // points back at this buffer) maps its own region
            if (p == rank || std::memcmp(&h, &own, sizeof(h)) == 0) {
                base[p] = s->ep_region;
                continue;
            }
            void* q = nullptr;
            CUDA_OK(cudaIpcOpenMemHandle(&q, h, cudaIpcMemLazyEnablePeerAccess));
            s->ep_mapped.push_back(q);
            base[p] = static_cast<uint8_t*>(q);
        }
        std::vector<float*> y(2 * size_t(world));
        std::vector<uint32_t*> f(2 * size_t(world));
        for (int k = 0; k < 2; k++)
            for (int p = 0; p < world; p++) {
                y[k * world + p] = reinterpret_cast<float*>(base[p] + 512 + k * s->ep_xbytes);
                f[k * world + p] = reinterpret_cast<uint32_t*>(base[p]) + k * 64 + rank;
            }
        CUDA_OK(cudaMemcpy(s->ep_peer_y, y.data(), y.size() * sizeof(float*), cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(s->ep_peer_flag, f.data(), f.size() * sizeof(uint32_t*), cudaMemcpyHostToDevice));
        // data-parallel attention: the same offsets in every rank's region
        const uint8_t* own_base = s->ep_region;
        auto at = [&](int p, const void* own_ptr) {
            return base[p] + (static_cast<const uint8_t*>(own_ptr) - own_base);
        };
        std::vector<float*> st(world), sq(world);
        std::vector<uint32_t*> df(2 * size_t(world)), am(world), gf(world);
        for (int p = 0; p < world; p++) {
            st[p] = reinterpret_cast<float*>(at(p, s->states));
            sq[p] = reinterpret_cast<float*>(at(p, s->sumsq + kMaxParts * 8));
            am[p] = reinterpret_cast<uint32_t*>(at(p, s->argmax));
            gf[p] = reinterpret_cast<uint32_t*>(at(p, s->dp_flags + 128));
            for (int k = 0; k < 2; k++) df[k * world + p] = reinterpret_cast<uint32_t*>(at(p, s->dp_flags)) + k * 64 + rank;
        }
        CUDA_OK(cudaMemcpy(s->dp_peer_states, st.data(), st.size() * sizeof(float*), cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(s->dp_peer_sumsq, sq.data(), sq.size() * sizeof(float*), cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(s->dp_peer_flag, df.data(), df.size() * sizeof(uint32_t*), cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(s->dp_peer_argmax, am.data(), am.size() * sizeof(uint32_t*), cudaMemcpyHostToDevice));
        CUDA_OK(cudaMemcpy(s->dp_peer_gflag, gf.data(), gf.size() * sizeof(uint32_t*), cudaMemcpyHostToDevice));
        s->ep_ready = true;
    });
}

spm_status spm_session_set_wait_limit(spm_session* s, uint64_t nanoseconds) {
    return guarded([&] {
        if (nanoseconds == 0) fail(SPM_E_ARG, "the wait limit must be positive");
        CUDA_OK(cudaSetDevice(s->m->device));
        CUDA_OK(cudaStreamSynchronize(s->stream));
        s->wait_ns = nanoseconds;
        for (auto& kv : s->exec) cudaGraphExecDestroy(kv.second);  // captured steps hold the old limit
        s->exec.clear();
    });
}

spm_status spm_session_set_profile(spm_session* s, int32_t enable) {
    return guarded([&] {
        CUDA_OK(cudaSetDevice(s->m->device));
        CUDA_OK(cudaStreamSynchronize(s->stream));
        for (auto& p : s->prof_pending) cudaEventDestroy(p.a), cudaEventDestroy(p.b);
        s->prof_pending.clear();
        s->prof_ms.clear();
        s->prof_bytes.clear();
        s->prof_kind.clear();
        s->prof = enable != 0;
    });
}

spm_status spm_session_profile(const spm_session* s, int32_t max, float* ms, uint64_t* bytes, int32_t* kind,
                               int32_t* count) {
    return guarded([&] {
        const int32_t have = int32_t(s->prof_ms.size());
        if (count) *count = have;
        for (int32_t i = 0; i < std::min(max, have); i++) {
            if (ms) ms[i] = s->prof_ms[i];
            if (bytes) bytes[i] = s->prof_bytes[i];
            if (kind) kind[i] = s->prof_kind[i];
        }
    });
}

spm_status spm_session_launches_per_step(spm_session* s, int32_t n, int32_t* launches) {
    return guarded([&] {
        auto it = s->launches.find(n);
        if (it == s->launches.end()) fail(SPM_E_ARG, "no step has been captured at this client count");
        *launches = it->second;
    });
}

}  // extern "C"

// ---- dequantization into a static device buffer (no allocation) ----
//
// spm_dequant_rows allocates a device buffer for the decoded rows on every
// call.  Some callers cannot allocate device memory: a parity or monitoring
// hook that runs beside a serving session which has committed the rest of
// HBM to KV caches (an allocation there can fail), or one that must not add
// the device-wide synchronisation that cudaMalloc and cudaFree may imply to a
// device whose other streams are decoding.  spm_dequant_rows_static serves
// them: it decodes into a fixed buffer that is part of this library's device
// image, so it allocates nothing, at the price of a size limit and of one
// buffer per device shared by every call.
//
// kStaticDequantFloats bounds rows x cols of one call (4 MiB of floats); every
// GPU that loads the library holds the buffer until the process exits.  The
// buffer keeps the previous call's contents, but nothing in it needs to start
// at zero: the kernel writes every float that the call then copies out.
// Calls that overlap on the GPU (from two host threads, say) use the same
// buffer and race; serialise them.  Every call looks up the buffer's device
// address in the calling thread's current context (cheap once the module is
// loaded), so an address never outlives the context it belongs to.  The first
// call on a device loads this library's device code there; make that first
// call before any stream capture begins on that device.
constexpr uint64_t kStaticDequantFloats = uint64_t(1) << 20;
static __device__ __align__(256) float g_static_dequant[kStaticDequantFloats];

namespace {
// In host code the array's name is only a stand-in; its device address comes
// from the runtime, for the current device's context.
float* static_dequant_buffer() {
    float* ptr = nullptr;
    CUDA_OK(cudaGetSymbolAddress((void**)&ptr, g_static_dequant));
    return ptr;
}
}  // namespace

extern "C" {

spm_status spm_dequant_rows_static(const spm_model* m, int32_t index, uint64_t row0, uint64_t rows,
                                   float* out_host) {
    return guarded([&] {
        if (index < 0 || index >= int32_t(m->streams.size())) fail(SPM_E_ARG, "stream index out of range");
        const Packed& p = m->streams[index].pk;
        if (row0 > p.rows || rows > p.rows - row0) fail(SPM_E_ARG, "row range exceeds the matrix");
        if (rows > kStaticDequantFloats / std::max<uint64_t>(p.cols, 1))
            fail(SPM_E_ARG, "spm_dequant_rows_static: " + std::to_string(rows) + " rows x " + std::to_string(p.cols) +
                                " cols exceeds the static buffer of " + std::to_string(kStaticDequantFloats) +
                                " floats; request fewer rows per call");
        CUDA_OK(cudaSetDevice(m->device));
        float* buf = static_dequant_buffer();
        CUDA_OK(launch_dequant(p.dtype, m->tiles(index), p, row0, rows, buf, nullptr));
        CUDA_OK(cudaMemcpy(out_host, buf, rows * p.cols * sizeof(float), cudaMemcpyDeviceToHost));
    });
}

}  // extern "C"
