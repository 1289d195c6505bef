// Host-side format code: errors, GGML block geometry, the bounded GGUF parser,
// the block decoders and .order files.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <fstream>
#include <set>
#include <sstream>

#include "common.h"

namespace spm {

static thread_local std::string g_error;
void set_error(const std::string& msg) { g_error = msg; }
const std::string& last_error() { return g_error; }
[[noreturn]] void fail(spm_status code, const std::string& msg) { throw Error{code, msg}; }

bool type_layout(uint32_t t, uint64_t* bv, uint64_t* bb) {
    uint64_t v = 0, b = 0;
    switch (t) {
        case 0: v = 1; b = 4; break;
        case 1: case 30: v = 1; b = 2; break;
        case 2: v = 32; b = 18; break;
        case 3: v = 32; b = 20; break;
        case 6: v = 32; b = 22; break;
        case 7: v = 32; b = 24; break;
        case 8: v = 32; b = 34; break;
        case 9: v = 32; b = 40; break;
        case 10: v = 256; b = 84; break;
        case 11: v = 256; b = 110; break;
        case 12: v = 256; b = 144; break;
        case 13: v = 256; b = 176; break;
        case 14: v = 256; b = 210; break;
        case 15: v = 256; b = 292; break;
        case 16: v = 1; b = 8; break;
        default: return false;
    }
    if (bv) *bv = v;
    if (bb) *bb = b;
    return true;
}

// IEEE half -> float, exact for every input (spm-gguf/src/tensor.rs:82-98).
float f16_to_f32(uint16_t bits) {
    uint32_t sign = uint32_t(bits & 0x8000u) << 16;
    uint32_t exp = (bits >> 10) & 0x1fu, frac = bits & 0x3ffu, out;
    if (exp == 0 && frac == 0) out = sign;
    else if (exp == 0) {
        uint32_t shift = uint32_t(__builtin_clz(frac)) - 21u;
        out = sign | ((113u - shift) << 23) | (((frac << shift) & 0x3ffu) << 13);
    } else if (exp == 31) out = sign | 0x7f800000u | (frac << 13);
    else out = sign | ((exp + 112u) << 23) | (frac << 13);
    float f;
    std::memcpy(&f, &out, 4);
    return f;
}

// float -> half, round to nearest even (used only by the encoders).
uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mag = x & 0x7fffffffu;
    if (mag >= 0x7f800000u) return uint16_t(sign | (mag > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (mag >= 0x477ff000u) return uint16_t(sign | 0x7c00u);  // rounds to inf
    if (mag < 0x38800000u) {                                  // subnormal half
        if (mag < 0x33000000u) return uint16_t(sign);
        uint32_t e = mag >> 23, m = (mag & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126u - e;  // 14 + (127 - 1 - e) ... aligns to 2^-24 units
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return uint16_t(sign | q);
    }
    uint32_t e = (mag >> 23) - 112u, m = mag & 0x7fffffu;
    uint32_t q = (e << 10) | (m >> 13), rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return uint16_t(sign | q);
}

// ------------------------------------------------------------------
// GGUF: spm-gguf/src/parse.rs:31-182 and wire.rs:10-91, on a memory image.
// ------------------------------------------------------------------
static constexpr uint64_t kMaxMetadata = 1000000, kMaxTensors = 1000000;
static constexpr uint64_t kMaxString = 16ull << 20, kMaxArray = 2000000;
static constexpr uint32_t kMaxDims = 8;
static constexpr uint64_t kMaxHeaderBytes = 512ull << 20;

namespace {
struct Reader {
    const uint8_t* buf;
    uint64_t pos, len;
    const uint8_t* take(uint64_t n) {
        uint64_t end = pos + n;
        if (end < pos) fail(SPM_E_STREAM, "file position overflow");
        if (end > kMaxHeaderBytes) fail(SPM_E_STREAM, "GGUF header exceeds limit");
        if (end > len) fail(SPM_E_TRUNCATED, "unexpected end of GGUF");
        const uint8_t* p = buf + pos;
        pos = end;
        return p;
    }
    uint32_t u32() { uint32_t v; std::memcpy(&v, take(4), 4); return v; }
    uint64_t u64() { uint64_t v; std::memcpy(&v, take(8), 8); return v; }
    std::string str() {
        uint64_t n = u64();
        if (n > kMaxString) fail(SPM_E_STREAM, "string length " + std::to_string(n) + " exceeds limit");
        const uint8_t* p = take(n);
        return std::string(reinterpret_cast<const char*>(p), n);
    }
    void value(uint32_t ty, int depth, GgufMeta* m) {
        if (depth > 4) fail(SPM_E_STREAM, "metadata nesting exceeds limit");
        const uint8_t* p;
        switch (ty) {
            case 0: p = take(1); if (m) { m->has_int = true; m->u = p[0]; } return;
            case 1: p = take(1); if (m) { m->has_int = true; m->u = uint64_t(int64_t(int8_t(p[0]))); } return;
            case 2: p = take(2); if (m) { m->has_int = true; m->u = uint64_t(p[0] | (p[1] << 8)); } return;
            case 3: { p = take(2); int16_t v; std::memcpy(&v, p, 2); if (m) { m->has_int = true; m->u = uint64_t(int64_t(v)); } return; }
            case 4: { uint32_t v = u32(); if (m) { m->has_int = true; m->u = v; } return; }
            case 5: { uint32_t v = u32(); if (m) { m->has_int = true; m->u = uint64_t(int64_t(int32_t(v))); } return; }
            case 6: { float f; std::memcpy(&f, take(4), 4); if (m) { m->has_float = true; m->f = f; } return; }
            case 7: p = take(1); if (p[0] > 1) fail(SPM_E_STREAM, "invalid boolean metadata value");
                    if (m) { m->has_int = true; m->u = p[0]; } return;
            case 8: { std::string s = str(); if (m) m->s = s; return; }
            case 9: {
                uint32_t inner = u32();
                uint64_t n = u64();
                if (n > kMaxArray) fail(SPM_E_STREAM, "array length " + std::to_string(n) + " exceeds limit");
                for (uint64_t i = 0; i < n; i++) value(inner, depth + 1, nullptr);
                return;
            }
            case 10: { uint64_t v = u64(); if (m) { m->has_int = true; m->u = v; } return; }
            case 11: { uint64_t v = u64(); if (m) { m->has_int = true; m->u = v; } return; }
            case 12: { double d; std::memcpy(&d, take(8), 8); if (m) { m->has_float = true; m->f = d; } return; }
            default: fail(SPM_E_STREAM, "unknown metadata type " + std::to_string(ty));
        }
    }
};
}  // namespace

const GgufTensor* Gguf::find(const std::string& name) const {
    for (auto& t : tensors)
        if (t.name == name) return &t;
    return nullptr;
}
const GgufMeta* Gguf::meta_find(const std::string& key) const {
    for (auto& m : meta)
        if (m.key == key) return &m;
    return nullptr;
}

Gguf gguf_parse(const uint8_t* buf, uint64_t len) {
    Reader r{buf, 0, len};
    Gguf g;
    if (std::memcmp(r.take(4), "GGUF", 4) != 0) fail(SPM_E_STREAM, "invalid GGUF magic");
    g.version = r.u32();
    if (g.version != 3) fail(SPM_E_STREAM, "unsupported GGUF version " + std::to_string(g.version));
    uint64_t tensors = r.u64(), metadata = r.u64();
    if (tensors > kMaxTensors) fail(SPM_E_STREAM, "tensor count exceeds limit");
    if (metadata > kMaxMetadata) fail(SPM_E_STREAM, "metadata count exceeds limit");
    std::set<std::string> keys;
    for (uint64_t i = 0; i < metadata; i++) {
        GgufMeta m;
        m.key = r.str();
        m.type = r.u32();
        r.value(m.type, 0, &m);
        if (!keys.insert(m.key).second) fail(SPM_E_STREAM, "duplicate metadata key");
        g.meta.push_back(std::move(m));
    }
    std::set<std::string> names;
    std::vector<GgufTensor> raw;
    for (uint64_t i = 0; i < tensors; i++) {
        GgufTensor t;
        t.name = r.str();
        if (!names.insert(t.name).second) fail(SPM_E_STREAM, "duplicate tensor name " + t.name);
        uint32_t nd = r.u32();
        if (nd == 0 || nd > kMaxDims) fail(SPM_E_STREAM, "invalid dimension count " + std::to_string(nd));
        for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.u64());
        t.dtype = r.u32();
        t.offset = r.u64();
        raw.push_back(std::move(t));
    }
    uint64_t align = 32;
    if (auto* m = g.meta_find("general.alignment")) {
        if (m->has_int) align = m->u;
    }
    if (align == 0 || (align & (align - 1)) != 0) fail(SPM_E_STREAM, "invalid alignment");
    uint64_t base = (r.pos + align - 1) & ~(align - 1);
    if (base > len) fail(SPM_E_STREAM, "tensor data starts beyond file");
    g.data_offset = base;
    for (auto& t : raw) {
        if (t.offset % align != 0) fail(SPM_E_STREAM, "unaligned tensor " + t.name);
        uint64_t elems = 1;
        for (uint64_t d : t.dims) {
            if (d == 0) fail(SPM_E_STREAM, "tensor " + t.name + " has a zero dimension");
            if (elems > UINT64_MAX / d) fail(SPM_E_STREAM, "tensor element count overflow");
            elems *= d;
        }
        uint64_t bv, bb;
        if (!type_layout(t.dtype, &bv, &bb)) fail(SPM_E_ENCODING, "unsupported GGML dtype " + std::to_string(t.dtype));
        if (elems % bv != 0) fail(SPM_E_STREAM, "tensor " + t.name + " does not fill dtype blocks");
        if (elems / bv > UINT64_MAX / bb) fail(SPM_E_STREAM, "tensor byte length overflow");
        t.len = elems / bv * bb;
        uint64_t off = base + t.offset;
        if (off < base) fail(SPM_E_STREAM, "tensor offset overflow");
        if (off + t.len < off || off + t.len > len) fail(SPM_E_TRUNCATED, "tensor " + t.name + " extends beyond file");
        t.offset = off;
    }
    std::sort(raw.begin(), raw.end(), [](const GgufTensor& a, const GgufTensor& b) { return a.offset < b.offset; });
    for (size_t i = 1; i < raw.size(); i++)
        if (raw[i - 1].offset + raw[i - 1].len > raw[i].offset) fail(SPM_E_STREAM, "overlapping tensor ranges");
    g.tensors = std::move(raw);
    return g;
}

// ------------------------------------------------------------------
// Host block decoders (spm-gguf/src/tensor.rs:69-210; Q2_K from ggml's
// published block_q2_K).  Same arithmetic order as the device decoders.
// ------------------------------------------------------------------
static uint16_t rd16(const uint8_t* p) { return uint16_t(p[0] | (p[1] << 8)); }

void decode_blocks(uint32_t t, const uint8_t* b, uint64_t nbytes, float* out) {
    uint64_t bv, bb;
    if (!type_layout(t, &bv, &bb)) fail(SPM_E_ENCODING, "unsupported GGML dtype " + std::to_string(t));
    if (nbytes % bb != 0) fail(SPM_E_TRUNCATED, "byte length is not a whole number of blocks");
    uint64_t nb = nbytes / bb;
    for (uint64_t i = 0; i < nb; i++) {
        const uint8_t* blk = b + i * bb;
        float* o = out + i * bv;
        switch (t) {
            case SPM_F32: std::memcpy(o, blk, 4); break;
            case SPM_F16: o[0] = f16_to_f32(rd16(blk)); break;
            case SPM_Q8_0: {
                float d = f16_to_f32(rd16(blk));
                for (int k = 0; k < 32; k++) o[k] = d * float(int8_t(blk[2 + k]));
                break;
            }
            case SPM_Q6_K: {
                float d = f16_to_f32(rd16(blk + 208));
                for (int half = 0; half < 2; half++) {
                    const uint8_t* ql = blk + half * 64;
                    const uint8_t* qh = blk + 128 + half * 32;
                    const uint8_t* sc = blk + 192 + half * 8;
                    for (int l = 0; l < 32; l++) {
                        int is = l / 16;
                        int q[4] = {(ql[l] & 15) | ((qh[l] & 3) << 4), (ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4),
                                    (ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4), (ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)};
                        for (int g = 0; g < 4; g++)
                            o[half * 128 + l + 32 * g] = d * float(int8_t(sc[is + 2 * g])) * (float(q[g]) - 32.0f);
                    }
                }
                break;
            }
            case SPM_Q5_K: {
                float d = f16_to_f32(rd16(blk)), dmin = f16_to_f32(rd16(blk + 2));
                const uint8_t* s = blk + 4;
                const uint8_t* qh = blk + 16;
                const uint8_t* qs = blk + 48;
                for (int j = 0; j < 8; j++) {
                    int sc, m;
                    if (j < 4) { sc = s[j] & 63; m = s[j + 4] & 63; }
                    else { sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
                    for (int l = 0; l < 32; l++) {
                        int lo = (j & 1) ? (qs[(j / 2) * 32 + l] >> 4) : (qs[(j / 2) * 32 + l] & 15);
                        int q = lo + ((qh[l] >> j) & 1) * 16;
                        o[j * 32 + l] = d * float(sc) * float(q) - dmin * float(m);
                    }
                }
                break;
            }
            case SPM_Q2_K: {
                float d = f16_to_f32(rd16(blk + 80)), dmin = f16_to_f32(rd16(blk + 82));
                for (int k = 0; k < 256; k++) {
                    int n = k / 128, j = (k % 128) / 32, l = k % 32;
                    uint8_t sc = blk[8 * n + 2 * j + l / 16];
                    float dl = d * float(sc & 15), ml = dmin * float(sc >> 4);
                    o[k] = dl * float((blk[16 + 32 * n + l] >> (2 * j)) & 3) - ml;
                }
                break;
            }
            default: fail(SPM_E_ENCODING, "no decoder for GGML dtype " + std::to_string(t));
        }
    }
}

// ------------------------------------------------------------------
// .order files: spm-order/src/order.rs:28-52 (parse) and :64-83 (reorder).
// ------------------------------------------------------------------
Order parse_order(const std::string& text) {
    Order o;
    int section = -1;
    std::istringstream in(text);
    std::string line;
    int lineno = 0;
    while (std::getline(in, line)) {
        lineno++;
        size_t a = line.find_first_not_of(" \t\r"), z = line.find_last_not_of(" \t\r");
        if (a == std::string::npos) continue;
        line = line.substr(a, z - a + 1);
        if (line[0] == '#') continue;
        if (line == "[rotating]") section = 1;
        else if (line == "[resident]") section = 0;
        else if (section == 1) o.rotating.push_back(line);
        else if (section == 0) o.resident.push_back(line);
        else fail(SPM_E_STREAM, "line " + std::to_string(lineno) + ": name before any [rotating] or [resident] section");
    }
    return o;
}

std::string default_order(const spm_model_cfg& c, bool router_bias) {
    std::ostringstream o;
    bool moe = c.family == SPM_FAMILY_OLMOE || c.family == SPM_FAMILY_QWEN3MOE;
    o << "# consumption order: per layer q, k, v, o, then the feed-forward streams\n[rotating]\n";
    for (uint32_t l = 0; l < c.layers; l++) {
        for (const char* n : {"attn_q", "attn_k", "attn_v", "attn_output"}) o << "blk." << l << "." << n << ".weight\n";
        if (moe) {
            for (const char* n : {"ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"})
                o << "blk." << l << "." << n << ".weight\n";
        } else {
            for (const char* n : {"ffn_gate", "ffn_up", "ffn_down"}) o << "blk." << l << "." << n << ".weight\n";
        }
    }
    if (!c.tied) o << "output.weight\n";
    o << "[resident]\ntoken_embd.weight\n";
    for (uint32_t l = 0; l < c.layers; l++) {
        o << "blk." << l << ".attn_norm.weight\n" << "blk." << l << ".ffn_norm.weight\n";
        if (c.family != SPM_FAMILY_LLAMA)
            o << "blk." << l << ".attn_q_norm.weight\n" << "blk." << l << ".attn_k_norm.weight\n";
        if (moe && router_bias) o << "blk." << l << ".exp_probs_b.bias\n";
    }
    o << "output_norm.weight\n";
    return o.str();
}

}  // namespace spm
