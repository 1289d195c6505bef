// Encoders (GGML Q8_0 / Q6_K / Q5_K / Q2_K blocks) and the synthetic GGUF
// writer.  The reference ships neither a GGUF writer nor a K-quant quantizer
// (its spm-quantize emits ternary only), so these are this library's own: any
// valid block encoding serves, because the oracle and the device path consume
// the same bytes.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cmath>
#include <thread>

#include "common.h"

namespace spm {

// ---- encoders: simple absmax / range quantizers, one row of blocks at a time ----
static int iround(float x) { return int(std::lrintf(x)); }
static int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

static void enc_q8_0(const float* x, uint8_t* b) {
    float amax = 0;
    for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(x[i]));
    float d = amax / 127.0f;
    uint16_t d16 = f32_to_f16(d);
    float dq = f16_to_f32(d16);
    b[0] = uint8_t(d16 & 0xff);
    b[1] = uint8_t(d16 >> 8);
    for (int i = 0; i < 32; i++) b[2 + i] = uint8_t(int8_t(dq > 0 ? clampi(iround(x[i] / dq), -127, 127) : 0));
}

static void enc_q6_k(const float* x, uint8_t* b) {
    float s[16], smax = 0;
    for (int j = 0; j < 16; j++) {
        float amax = 0;
        for (int i = 0; i < 16; i++) amax = std::max(amax, std::fabs(x[16 * j + i]));
        s[j] = amax / 31.0f;
        smax = std::max(smax, s[j]);
    }
    uint16_t d16 = f32_to_f16(smax / 127.0f);
    float d = f16_to_f32(d16);
    std::memset(b, 0, 210);
    int8_t sc[16];
    for (int j = 0; j < 16; j++) sc[j] = int8_t(d > 0 ? clampi(iround(s[j] / d), -128, 127) : 0);
    uint8_t q[256];
    for (int k = 0; k < 256; k++) {
        float e = d * float(sc[k / 16]);
        q[k] = uint8_t(e != 0 ? clampi(iround(x[k] / e), -32, 31) + 32 : 32);
    }
    // ggml layout: half n, l in 0..32: ql[64n+l] = q(l) | q(l+64)<<4,
    // ql[64n+32+l] = q(l+32) | q(l+96)<<4, qh[32n+l] = hi2 of q(l), q(l+32), q(l+64), q(l+96).
    for (int n = 0; n < 2; n++) {
        const uint8_t* qq = q + 128 * n;
        for (int l = 0; l < 32; l++) {
            b[64 * n + l] = uint8_t((qq[l] & 15) | ((qq[l + 64] & 15) << 4));
            b[64 * n + 32 + l] = uint8_t((qq[l + 32] & 15) | ((qq[l + 96] & 15) << 4));
            b[128 + 32 * n + l] = uint8_t((qq[l] >> 4) | ((qq[l + 32] >> 4) << 2) | ((qq[l + 64] >> 4) << 4) |
                                          ((qq[l + 96] >> 4) << 6));
        }
    }
    for (int j = 0; j < 16; j++) b[192 + j] = uint8_t(sc[j]);
    b[208] = uint8_t(d16 & 0xff);
    b[209] = uint8_t(d16 >> 8);
}

static void enc_q5_k(const float* x, uint8_t* b) {
    float scale[8], mins[8], smax = 0, mmax = 0;
    for (int j = 0; j < 8; j++) {
        float lo = 0, hi = 0;
        for (int i = 0; i < 32; i++) { lo = std::min(lo, x[32 * j + i]); hi = std::max(hi, x[32 * j + i]); }
        scale[j] = (hi - lo) / 31.0f;
        mins[j] = -lo;
        smax = std::max(smax, scale[j]);
        mmax = std::max(mmax, mins[j]);
    }
    uint16_t d16 = f32_to_f16(smax / 63.0f), m16 = f32_to_f16(mmax / 63.0f);
    float d = f16_to_f32(d16), dmin = f16_to_f32(m16);
    int sc[8], mn[8];
    for (int j = 0; j < 8; j++) {
        sc[j] = d > 0 ? clampi(iround(scale[j] / d), 0, 63) : 0;
        mn[j] = dmin > 0 ? clampi(iround(mins[j] / dmin), 0, 63) : 0;
    }
    std::memset(b, 0, 176);
    b[0] = uint8_t(d16 & 0xff); b[1] = uint8_t(d16 >> 8);
    b[2] = uint8_t(m16 & 0xff); b[3] = uint8_t(m16 >> 8);
    uint8_t* s = b + 4;
    for (int j = 0; j < 4; j++) {
        s[j] = uint8_t((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = uint8_t((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = uint8_t((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    uint8_t* qh = b + 16;
    uint8_t* qs = b + 48;
    for (int j = 0; j < 8; j++) {
        float e = d * float(sc[j]), off = dmin * float(mn[j]);
        for (int l = 0; l < 32; l++) {
            int q = e > 0 ? clampi(iround((x[32 * j + l] + off) / e), 0, 31) : 0;
            qs[(j / 2) * 32 + l] |= uint8_t((q & 15) << ((j & 1) * 4));
            qh[l] |= uint8_t(((q >> 4) & 1) << j);
        }
    }
}

static void enc_q2_k(const float* x, uint8_t* b) {
    float scale[16], mins[16], smax = 0, mmax = 0;
    for (int j = 0; j < 16; j++) {
        float lo = 0, hi = 0;
        for (int i = 0; i < 16; i++) { lo = std::min(lo, x[16 * j + i]); hi = std::max(hi, x[16 * j + i]); }
        scale[j] = (hi - lo) / 3.0f;
        mins[j] = -lo;
        smax = std::max(smax, scale[j]);
        mmax = std::max(mmax, mins[j]);
    }
    uint16_t d16 = f32_to_f16(smax / 15.0f), m16 = f32_to_f16(mmax / 15.0f);
    float d = f16_to_f32(d16), dmin = f16_to_f32(m16);
    std::memset(b, 0, 84);
    for (int j = 0; j < 16; j++) {
        int sc = d > 0 ? clampi(iround(scale[j] / d), 0, 15) : 0;
        int mn = dmin > 0 ? clampi(iround(mins[j] / dmin), 0, 15) : 0;
        b[j] = uint8_t(sc | (mn << 4));
        float e = d * float(sc), off = dmin * float(mn);
        // sub-block j covers weights 16j..16j+15 = (n, shift pair jj, part)
        for (int i = 0; i < 16; i++) {
            int k = 16 * j + i, n = k / 128, jj = (k % 128) / 32, l = k % 32;
            int q = e > 0 ? clampi(iround((x[k] + off) / e), 0, 3) : 0;
            b[16 + 32 * n + l] |= uint8_t(q << (2 * jj));
        }
    }
    b[80] = uint8_t(d16 & 0xff); b[81] = uint8_t(d16 >> 8);
    b[82] = uint8_t(m16 & 0xff); b[83] = uint8_t(m16 >> 8);
}

void quantize(uint32_t t, const float* src, uint64_t n, uint8_t* dst) {
    uint64_t bv, bb;
    if (!type_layout(t, &bv, &bb)) fail(SPM_E_ENCODING, "unsupported GGML dtype " + std::to_string(t));
    if (n % bv) fail(SPM_E_ARG, "value count is not a whole number of blocks");
    for (uint64_t i = 0; i < n / bv; i++) {
        const float* x = src + i * bv;
        uint8_t* b = dst + i * bb;
        switch (t) {
            case SPM_F32: std::memcpy(b, x, 4); break;
            case SPM_F16: { uint16_t h = f32_to_f16(x[0]); b[0] = uint8_t(h); b[1] = uint8_t(h >> 8); break; }
            case SPM_Q8_0: enc_q8_0(x, b); break;
            case SPM_Q6_K: enc_q6_k(x, b); break;
            case SPM_Q5_K: enc_q5_k(x, b); break;
            case SPM_Q2_K: enc_q2_k(x, b); break;
            default: fail(SPM_E_ENCODING, "no encoder for GGML dtype " + std::to_string(t));
        }
    }
}

// ---- seeded values: splitmix64 counters, Box-Muller pairs ----
static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
// Normal value `i` of stream `key`: pair i/2 of a Box-Muller transform whose
// uniforms come from mix64(key ^ pair).  Independent of thread layout.
// Each pair is transformed once and gives both of its values.
static void normals(uint64_t key, uint64_t first, uint64_t count, float sigma, float* out) {
    uint64_t k = 0;
    while (k < count) {
        const uint64_t i = first + k, pair = i >> 1;
        const uint64_t h = mix64(key ^ mix64(pair));
        const float u1 = (float(uint32_t(h >> 40)) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = float(uint32_t(h & 0xffffffu)) * (1.0f / 16777216.0f);
        const float r = std::sqrt(-2.0f * std::log(u1));
        const float a = 6.28318530718f * u2;
        if ((i & 1) == 0) {
            out[k++] = sigma * r * std::cos(a);
            if (k == count) break;
        }
        out[k++] = sigma * r * std::sin(a);
    }
}

namespace {
struct Plan {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t dtype;
    int kind;  // 0 weights N(0,sigma), 1 norm gain, 2 router bias
    uint32_t layer;
    uint64_t rel = 0, len = 0;
};

void put_u32(std::vector<uint8_t>& v, uint32_t x) { for (int i = 0; i < 4; i++) v.push_back(uint8_t(x >> (8 * i))); }
void put_u64(std::vector<uint8_t>& v, uint64_t x) { for (int i = 0; i < 8; i++) v.push_back(uint8_t(x >> (8 * i))); }
void put_str(std::vector<uint8_t>& v, const std::string& s) { put_u64(v, s.size()); v.insert(v.end(), s.begin(), s.end()); }
void kv_u32(std::vector<uint8_t>& v, const std::string& k, uint32_t x) { put_str(v, k); put_u32(v, 4); put_u32(v, x); }
void kv_f32(std::vector<uint8_t>& v, const std::string& k, float x) {
    put_str(v, k); put_u32(v, 6); uint32_t b; std::memcpy(&b, &x, 4); put_u32(v, b);
}
void kv_str(std::vector<uint8_t>& v, const std::string& k, const std::string& s) { put_str(v, k); put_u32(v, 8); put_str(v, s); }
}  // namespace

static const char* arch_name(uint32_t family) {
    switch (family) {
        case SPM_FAMILY_LLAMA: return "llama";
        case SPM_FAMILY_QWEN3: return "qwen3";
        case SPM_FAMILY_OLMOE: return "olmoe";
        case SPM_FAMILY_QWEN3MOE: return "qwen3moe";
        default: fail(SPM_E_ARG, "unknown model family");
    }
}

uint8_t* synth_gguf(const spm_synth_spec& sp, uint64_t* out_len) {
    const spm_model_cfg& c = sp.cfg;
    if (!c.layers || !c.hidden || !c.heads || !c.kv_heads || !c.head_dim || !c.vocab)
        fail(SPM_E_ARG, "model shape has a zero dimension");
    bool moe = c.family == SPM_FAMILY_OLMOE || c.family == SPM_FAMILY_QWEN3MOE;
    uint64_t qw = uint64_t(c.heads) * c.head_dim, kvw = uint64_t(c.kv_heads) * c.head_dim;
    std::vector<Plan> plan;
    auto add = [&](std::string name, std::vector<uint64_t> dims, uint32_t dt, int kind, uint32_t layer) {
        plan.push_back(Plan{std::move(name), std::move(dims), dt, kind, layer});
    };
    add("token_embd.weight", {c.hidden, c.vocab}, sp.embed_type, 0, 0);
    for (uint32_t l = 0; l < c.layers; l++) {
        std::string p = "blk." + std::to_string(l) + ".";
        add(p + "attn_norm.weight", {c.hidden}, SPM_F32, 1, l);
        add(p + "attn_q.weight", {c.hidden, qw}, sp.layer_type, 0, l);
        add(p + "attn_k.weight", {c.hidden, kvw}, sp.layer_type, 0, l);
        add(p + "attn_v.weight", {c.hidden, kvw}, sp.layer_type, 0, l);
        add(p + "attn_output.weight", {qw, c.hidden}, sp.layer_type, 0, l);
        if (c.family == SPM_FAMILY_OLMOE) {
            add(p + "attn_q_norm.weight", {qw}, SPM_F32, 1, l);
            add(p + "attn_k_norm.weight", {kvw}, SPM_F32, 1, l);
        } else if (c.family != SPM_FAMILY_LLAMA) {
            add(p + "attn_q_norm.weight", {c.head_dim}, SPM_F32, 1, l);
            add(p + "attn_k_norm.weight", {c.head_dim}, SPM_F32, 1, l);
        }
        add(p + "ffn_norm.weight", {c.hidden}, SPM_F32, 1, l);
        if (moe) {
            add(p + "ffn_gate_inp.weight", {c.hidden, c.experts}, SPM_F32, 0, l);
            if (sp.zipf_s > 0) add(p + "exp_probs_b.bias", {c.experts}, SPM_F32, 2, l);
            add(p + "ffn_gate_exps.weight", {c.hidden, c.expert_ff, c.experts}, sp.expert_type, 0, l);
            add(p + "ffn_up_exps.weight", {c.hidden, c.expert_ff, c.experts}, sp.expert_type, 0, l);
            add(p + "ffn_down_exps.weight", {c.expert_ff, c.hidden, c.experts}, sp.expert_type, 0, l);
        } else {
            add(p + "ffn_gate.weight", {c.hidden, c.intermediate}, sp.layer_type, 0, l);
            add(p + "ffn_up.weight", {c.hidden, c.intermediate}, sp.layer_type, 0, l);
            add(p + "ffn_down.weight", {c.intermediate, c.hidden}, sp.layer_type, 0, l);
        }
    }
    add("output_norm.weight", {c.hidden}, SPM_F32, 1, 0);
    if (!c.tied) add("output.weight", {c.hidden, c.vocab}, sp.head_type, 0, 0);

    const uint64_t align = 32;
    uint64_t rel = 0;
    for (auto& t : plan) {
        uint64_t bv, bb, elems = 1;
        for (auto d : t.dims) elems *= d;
        if (!type_layout(t.dtype, &bv, &bb)) fail(SPM_E_ENCODING, "unsupported dtype for " + t.name);
        if (t.dims[0] % bv) fail(SPM_E_ARG, t.name + ": row length is not a whole number of blocks");
        t.rel = rel;
        t.len = elems / bv * bb;
        rel = (rel + t.len + align - 1) & ~(align - 1);
    }
    std::vector<uint8_t> head;
    head.insert(head.end(), {'G', 'G', 'U', 'F'});
    put_u32(head, 3);
    put_u64(head, plan.size());
    std::string arch = arch_name(c.family);
    std::vector<uint8_t> kv;
    uint64_t nkv = 0;
    kv_str(kv, "general.architecture", arch); nkv++;
    kv_u32(kv, "general.alignment", uint32_t(align)); nkv++;
    kv_u32(kv, arch + ".block_count", c.layers); nkv++;
    kv_u32(kv, arch + ".embedding_length", c.hidden); nkv++;
    kv_u32(kv, arch + ".feed_forward_length", c.intermediate); nkv++;
    kv_u32(kv, arch + ".attention.head_count", c.heads); nkv++;
    kv_u32(kv, arch + ".attention.head_count_kv", c.kv_heads); nkv++;
    kv_u32(kv, arch + ".attention.key_length", c.head_dim); nkv++;
    kv_u32(kv, arch + ".vocab_size", c.vocab); nkv++;
    kv_f32(kv, arch + ".rope.freq_base", c.rope_base); nkv++;
    kv_f32(kv, arch + ".attention.layer_norm_rms_epsilon", c.eps); nkv++;
    if (moe) {
        kv_u32(kv, arch + ".expert_count", c.experts); nkv++;
        kv_u32(kv, arch + ".expert_used_count", c.experts_used); nkv++;
        kv_u32(kv, arch + ".expert_feed_forward_length", c.expert_ff); nkv++;
    }
    put_u64(head, nkv);
    head.insert(head.end(), kv.begin(), kv.end());
    for (auto& t : plan) {
        put_str(head, t.name);
        put_u32(head, uint32_t(t.dims.size()));
        for (auto d : t.dims) put_u64(head, d);
        put_u32(head, t.dtype);
        put_u64(head, t.rel);
    }
    uint64_t base = (head.size() + align - 1) & ~(align - 1);
    uint8_t* out = static_cast<uint8_t*>(std::calloc(1, base + rel));
    if (!out) fail(SPM_E_ARG, "cannot allocate the GGUF image");
    std::memcpy(out, head.data(), head.size());

    // Work items: (tensor, row range); each fills its rows independently.
    struct Item { size_t t; uint64_t r0, r1; };
    std::vector<Item> items;
    for (size_t i = 0; i < plan.size(); i++) {
        uint64_t rows = 1;
        for (size_t d = 1; d < plan[i].dims.size(); d++) rows *= plan[i].dims[d];
        uint64_t step = std::max<uint64_t>(1, (1u << 20) / plan[i].dims[0]);
        for (uint64_t r = 0; r < rows; r += step) items.push_back({i, r, std::min(rows, r + step)});
    }
    unsigned nt = sp.threads > 0 ? unsigned(sp.threads) : std::max(1u, std::thread::hardware_concurrency());
    std::atomic<size_t> next{0};
    std::vector<std::string> errs(nt);
    auto worker = [&](unsigned w) {
        std::vector<float> vals;
        try {
            for (;;) {
                size_t k = next.fetch_add(1);
                if (k >= items.size()) break;
                const Plan& t = plan[items[k].t];
                uint64_t cols = t.dims[0], bv, bb;
                type_layout(t.dtype, &bv, &bb);
                uint64_t n = (items[k].r1 - items[k].r0) * cols;
                vals.resize(n);
                uint64_t key = mix64(sp.seed ^ mix64(0x5eed0000ull + items[k].t));
                if (t.kind == 0) {
                    normals(key, items[k].r0 * cols, n, sp.sigma, vals.data());
                } else if (t.kind == 1) {
                    if (sp.gain_sigma > 0) {
                        normals(key, items[k].r0 * cols, n, sp.gain_sigma, vals.data());
                        for (auto& v : vals) v += 1.0f;
                    } else {
                        std::fill(vals.begin(), vals.end(), 1.0f);
                    }
                } else {
                    // Zipf(s) router bias: b_e = ln p_e, p_e ~ rank(e)^-s under a
                    // seeded permutation of ranks 1..E, one permutation per layer.
                    uint64_t E = cols;
                    std::vector<uint64_t> rank(E);
                    for (uint64_t e = 0; e < E; e++) rank[e] = e + 1;
                    uint64_t st = mix64(sp.seed ^ (0x21bfull << 32) ^ t.layer);
                    for (uint64_t e = E - 1; e > 0; e--) {
                        st = mix64(st);
                        std::swap(rank[e], rank[st % (e + 1)]);
                    }
                    double z = 0;
                    for (uint64_t e = 1; e <= E; e++) z += std::pow(double(e), -double(sp.zipf_s));
                    for (uint64_t e = 0; e < E; e++)
                        vals[e] = float(-double(sp.zipf_s) * std::log(double(rank[e])) - std::log(z));
                }
                uint8_t* dst = out + base + t.rel + items[k].r0 * (cols / bv) * bb;
                quantize(t.dtype, vals.data(), n, dst);
            }
        } catch (const Error& e) {
            errs[w] = e.msg;
        }
    };
    std::vector<std::thread> pool;
    for (unsigned w = 0; w < nt; w++) pool.emplace_back(worker, w);
    for (auto& th : pool) th.join();
    for (auto& e : errs)
        if (!e.empty()) { std::free(out); fail(SPM_E_ARG, e); }
    *out_len = base + rel;
    return out;
}

}  // namespace spm
