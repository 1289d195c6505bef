// .spm files on the host: the fixed 32-byte header (spm-header/src/parse.rs:
// 10-62), the 32-byte stream descriptors (spm-layout/src/wire.rs:12-30,
// model.rs Encoding::bytes_for), the group order (spm-walk/src/cursor.rs,
// spm-layout/src/tiling.rs:37-51) and the group framing -- an f32 scale, then
// the group's payload (spm-file/src/read.rs:69-101).  Plus the device packing
// of a ternary stream (spm-codec/src/lib.rs: two bits per weight, LSB pair
// first, bit 0 = nonzero, bit 1 = negative).
#include <cstdio>

#include "abi.h"

namespace spm {

static uint16_t le16(const uint8_t* p) { return uint16_t(p[0] | (p[1] << 8)); }
static uint32_t le32(const uint8_t* p) {
    return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

static std::string fmt(const char* f, unsigned long long a, unsigned long long b = 0) {
    char buf[160];
    std::snprintf(buf, sizeof buf, f, a, b);
    return buf;
}

// Encoding::bytes_for: wire bytes of a group of `count` weights.
static unsigned __int128 bytes_for(uint8_t enc, uint64_t count) {
    using u128 = unsigned __int128;
    switch (enc) {
        case SPM_ENC_TERNARY: return (u128(count) + 3) / 4;
        case SPM_ENC_F32: return u128(count) * 4;
        case SPM_ENC_BF16: return u128(count) * 2;
        case SPM_ENC_Q6K: return (u128(count) + 255) / 256 * 210;
        case SPM_ENC_Q5K: return (u128(count) + 255) / 256 * 176;
        default: return (u128(count) + 31) / 32 * 34;
    }
}

SpmFile spm_file_parse(const uint8_t* b, uint64_t len) {
    static const uint8_t kMagic[8] = {0x89, 'S', 'P', 'M', 0x0D, 0x0A, 0x1A, 0x0A};
    if (!b && len) fail(SPM_E_ARG, "null .spm image");
    if (len < 32) fail(SPM_E_TRUNCATED, fmt("header truncated: %llu bytes available, need 32", len));
    if (std::memcmp(b, kMagic, 8) != 0) fail(SPM_E_STREAM, "bad magic: not a .spm file, or corrupted in transit");
    SpmFile f;
    f.major = le16(b + 8);
    if (f.major > 1) fail(SPM_E_STREAM, fmt("unsupported .spm major version %llu: this build reads up to 1", f.major));
    f.minor = le16(b + 10);
    if (b[12] != 0) fail(SPM_E_STREAM, fmt("unknown endianness discriminant %llu", b[12]));
    const uint32_t n = le32(b + 16);
    f.desc.reserve(std::min<uint64_t>(n, (len - 32) / 32));  // a hostile count allocates nothing
    uint64_t at = 32;
    for (uint32_t i = 0; i < n; ++i, at += 32) {
        const uint64_t avail = at <= len ? len - at : 0;
        if (avail < 32) fail(SPM_E_TRUNCATED, fmt("descriptor truncated: %llu bytes, need 32", avail));
        const uint8_t* p = b + at;
        SpmDesc d;
        d.group_size = le32(p + 8);
        if (d.group_size == 0) fail(SPM_E_STREAM, "group_size must be at least 1");
        if (p[12] < SPM_ENC_TERNARY || p[12] > SPM_ENC_Q8_0)
            fail(SPM_E_ENCODING, fmt("unknown .spm encoding profile %llu", p[12]));
        d.rows = le32(p);
        d.cols = le32(p + 4);
        d.encoding = p[12];
        d.lane_count = le16(p + 14);
        f.desc.push_back(d);
    }
    f.payload = at;
    return f;
}

// Wire size of one stream, and the truncation a forward reader would report.
struct StreamWire {
    uint64_t total, full, rem, groups;
    unsigned __int128 full_bytes, rem_bytes;  // one full group, the short one (scale included)
    unsigned __int128 bytes() const { return full_bytes * full + (rem ? rem_bytes : 0); }
};

static StreamWire wire_of(const SpmDesc& d) {
    StreamWire w;
    w.total = uint64_t(d.rows) * d.cols;
    w.full = w.total / d.group_size;
    w.rem = w.total % d.group_size;
    w.groups = w.full + (w.rem ? 1 : 0);
    w.full_bytes = 4 + bytes_for(d.encoding, d.group_size);
    w.rem_bytes = 4 + bytes_for(d.encoding, w.rem);
    return w;
}

[[noreturn]] static void truncated(const StreamWire& w, uint64_t avail) {
    // the first group a sequential reader cannot complete
    const unsigned __int128 k = avail / w.full_bytes;
    if (k < w.full)
        fail(SPM_E_TRUNCATED, fmt("payload truncated: group needs %llu bytes, %llu remain",
                                  (unsigned long long)w.full_bytes, (unsigned long long)(avail - k * w.full_bytes)));
    fail(SPM_E_TRUNCATED, fmt("payload truncated: group needs %llu bytes, %llu remain",
                              (unsigned long long)w.rem_bytes, (unsigned long long)(avail - w.full * w.full_bytes)));
}

SpmSpan spm_file_locate(const SpmFile& f, uint64_t len, uint32_t index) {
    if (index >= f.desc.size()) fail(SPM_E_ARG, "stream index out of range");
    uint64_t at = f.payload;
    SpmSpan span;
    for (uint32_t s = 0; s <= index; ++s) {
        const StreamWire w = wire_of(f.desc[s]);
        const uint64_t avail = len - at;
        if (w.bytes() > avail) truncated(w, avail);
        if (s == index) {
            span.offset = at;
            span.bytes = uint64_t(w.bytes());
            span.groups = w.groups;
        }
        at += uint64_t(w.bytes());
    }
    return span;
}

static const char* encoding_name(uint8_t enc) {  // Debug names of spm_layout::Encoding
    switch (enc) {
        case SPM_ENC_TERNARY: return "Ternary2F32I32";
        case SPM_ENC_F32: return "F32";
        case SPM_ENC_BF16: return "Bf16";
        case SPM_ENC_Q6K: return "Q6K";
        case SPM_ENC_Q5K: return "Q5K";
        default: return "Q8_0";
    }
}

static uint64_t align256(uint64_t v) { return (v + 255) / 256 * 256; }

StreamPlan plan_ternary(const uint8_t* buf, uint64_t len, uint32_t index) {
    const SpmFile f = spm_file_parse(buf, len);
    if (f.desc.empty()) fail(SPM_E_ARG, "parameter stream declares no operations");
    if (index >= f.desc.size()) fail(SPM_E_ARG, "stream index out of range");
    const SpmDesc& d = f.desc[index];
    if (d.encoding != SPM_ENC_TERNARY)
        fail(SPM_E_ENCODING, fmt("stream %llu is not ternary (encoding profile %llu)", index, d.encoding));
    const SpmSpan span = spm_file_locate(f, len, index);
    // The reference's scan pulls the first group after its stream before it
    // stops (spm-gemv-ref/src/gemv.rs:88-104), so that group must be whole.
    for (uint32_t s = index + 1; s < f.desc.size(); ++s) {
        const StreamWire w = wire_of(f.desc[s]);
        if (!w.groups) continue;
        const unsigned __int128 first = w.full ? w.full_bytes : w.rem_bytes;
        const uint64_t avail = len - (span.offset + span.bytes);
        if (first > avail)
            fail(SPM_E_TRUNCATED, fmt("payload truncated: group needs %llu bytes, %llu remain",
                                      (unsigned long long)first, avail));
        break;
    }
    if (span.groups > 0xFFFFFFFFull) fail(SPM_E_ARG, "a ternary stream may hold at most 2^32 - 1 scale groups");
    StreamPlan p;
    p.encoding = d.encoding;
    p.rows = d.rows;
    p.cols = d.cols;
    p.group_size = d.group_size;
    p.groups = span.groups;
    p.offset = span.offset;
    p.rows_pad = (uint64_t(d.rows) + 31) / 32 * 32;
    p.col_words = (uint64_t(d.cols) + 15) / 16;
    p.scale_off = align256(p.col_words * p.rows_pad * 4);
    p.bytes = p.scale_off + p.groups * 4;
    p.payload_bytes = span.bytes - 4 * span.groups;
    return p;
}

StreamPlan plan_dense(const uint8_t* buf, uint64_t len, uint32_t index) {
    const SpmFile f = spm_file_parse(buf, len);
    if (index >= f.desc.size()) fail(SPM_E_ARG, "stream index out of range");
    const SpmDesc& d = f.desc[index];
    // spm-codec-any/src/decode.rs:36-45: only the dense profiles decode to
    // weights; the others need a scale-aware engine (LinearError::Stream)
    if (d.encoding != SPM_ENC_F32 && d.encoding != SPM_ENC_BF16)
        fail(SPM_E_STREAM, std::string("parameter stream: ") + encoding_name(d.encoding) +
                               " needs a scale-aware engine");
    const SpmSpan span = spm_file_locate(f, len, index);
    StreamPlan p;
    p.encoding = d.encoding;
    p.rows = d.rows;
    p.cols = d.cols;
    p.group_size = d.group_size;
    p.groups = span.groups;
    p.offset = span.offset;
    p.rows_pad = (uint64_t(d.rows) + 31) / 32 * 32;
    p.bytes = p.rows_pad * d.cols * (d.encoding == SPM_ENC_F32 ? 4 : 2);
    p.payload_bytes = span.bytes - 4 * span.groups;
    return p;
}

StreamPlan plan_qblocks(const uint8_t* buf, uint64_t len, uint32_t index) {
    const SpmFile f = spm_file_parse(buf, len);
    if (index >= f.desc.size()) fail(SPM_E_ARG, "stream index out of range");
    const SpmDesc& d = f.desc[index];
    uint32_t bv = 0;
    switch (d.encoding) {
        case SPM_ENC_Q8_0: bv = 32; break;
        case SPM_ENC_Q6K: bv = 256; break;
        case SPM_ENC_Q5K: bv = 256; break;
        default:
            fail(SPM_E_STREAM, std::string("stream is ") + encoding_name(d.encoding) +
                                   ", not a block profile (Q8_0, Q6K or Q5K)");
    }
    const uint64_t total = uint64_t(d.rows) * d.cols;
    // every group must be exactly one block, the last one included
    if (d.group_size != bv || total % bv)
        fail(SPM_E_STREAM, std::string("unexpected packed group: ") + encoding_name(d.encoding) +
                               " streams hold one " + std::to_string(bv) + "-value block per group");
    const SpmSpan span = spm_file_locate(f, len, index);
    StreamPlan p;
    p.encoding = d.encoding;
    p.rows = d.rows;
    p.cols = d.cols;
    p.group_size = d.group_size;
    p.groups = span.groups;
    p.offset = span.offset;
    p.rows_pad = (uint64_t(d.rows) + 31) / 32 * 32;
    p.bytes = span.bytes - 4 * span.groups;
    p.payload_bytes = p.bytes;
    return p;
}

uint64_t fill_stream(const uint8_t* buf, const StreamPlan& pl, uint8_t* dst) {
    std::memset(dst, 0, pl.bytes);
    const uint64_t total = uint64_t(pl.rows) * pl.cols;
    const uint8_t* p = buf + pl.offset;
    uint64_t reserved = 0;
    if (pl.encoding == SPM_ENC_TERNARY) {
        uint32_t* codes = reinterpret_cast<uint32_t*>(dst);
        uint8_t* scales = dst + pl.scale_off;
        uint64_t r = 0, c = 0;  // (row, col) of the next weight: stream position c * rows + r
        for (uint64_t g = 0; g < pl.groups; ++g) {
            const uint64_t count = std::min<uint64_t>(pl.group_size, total - g * pl.group_size);
            std::memcpy(scales + 4 * g, p, 4);  // f32::from_le_bytes on a little-endian host
            const uint8_t* packed = p + 4;
            for (uint64_t local = 0; local < count; ++local) {
                const uint32_t code = (packed[local >> 2] >> ((local & 3) * 2)) & 3u;
                if (code) {
                    codes[(c >> 4) * pl.rows_pad + r] |= code << ((c & 15) * 2);
                    if (code == 2) ++reserved;
                }
                if (++r == pl.rows) {
                    r = 0;
                    ++c;
                }
            }
            p += 4 + uint64_t(bytes_for(SPM_ENC_TERNARY, count));
        }
    } else if (pl.encoding == SPM_ENC_F32 || pl.encoding == SPM_ENC_BF16) {
        const uint32_t es = pl.encoding == SPM_ENC_F32 ? 4 : 2;
        uint64_t r = 0, c = 0;
        for (uint64_t g = 0; g < pl.groups; ++g) {
            const uint64_t count = std::min<uint64_t>(pl.group_size, total - g * pl.group_size);
            const uint8_t* w = p + 4;  // the group scale is inert for the dense profiles
            for (uint64_t i = 0; i < count; ++i) {
                std::memcpy(dst + (c * pl.rows_pad + r) * es, w + i * es, es);
                if (++r == pl.rows) {
                    r = 0;
                    ++c;
                }
            }
            p += 4 + count * es;
        }
    } else {
        const uint64_t bb = pl.groups ? pl.bytes / pl.groups : 0;
        for (uint64_t g = 0; g < pl.groups; ++g, p += 4 + bb) std::memcpy(dst + g * bb, p + 4, bb);
    }
    return reserved;
}

static PackedStream pack(const uint8_t* buf, StreamPlan plan) {
    PackedStream out;
    out.plan = plan;
    out.data.resize(plan.bytes);
    out.reserved_codes = plan.bytes ? fill_stream(buf, plan, out.data.data()) : 0;
    return out;
}

PackedStream pack_ternary(const uint8_t* buf, uint64_t len, uint32_t index) {
    return pack(buf, plan_ternary(buf, len, index));
}

PackedStream pack_dense(const uint8_t* buf, uint64_t len, uint32_t index) {
    return pack(buf, plan_dense(buf, len, index));
}

PackedStream pack_qblocks(const uint8_t* buf, uint64_t len, uint32_t index) {
    return pack(buf, plan_qblocks(buf, len, index));
}

}  // namespace spm

using namespace spm;

spm_status spm_file_probe(const uint8_t* spm, uint64_t len, uint32_t* version_major, uint32_t* version_minor,
                          int32_t* streams) {
    return guarded([&] {
        const SpmFile f = spm_file_parse(spm, len);
        if (f.desc.size() > 0x7FFFFFFFu) fail(SPM_E_ARG, "too many streams");
        if (version_major) *version_major = f.major;
        if (version_minor) *version_minor = f.minor;
        if (streams) *streams = int32_t(f.desc.size());
    });
}

spm_status spm_file_stream(const uint8_t* spm, uint64_t len, int32_t index, spm_file_stream_info* out) {
    return guarded([&] {
        if (!out) fail(SPM_E_ARG, "null output");
        if (index < 0) fail(SPM_E_ARG, "stream index out of range");
        const SpmFile f = spm_file_parse(spm, len);
        const SpmSpan span = spm_file_locate(f, len, uint32_t(index));
        const SpmDesc& d = f.desc[index];
        *out = spm_file_stream_info{};
        out->rows = d.rows;
        out->cols = d.cols;
        out->group_size = d.group_size;
        out->encoding = d.encoding;
        out->lane_count = d.lane_count;
        out->groups = span.groups;
        out->offset = span.offset;
        out->bytes = span.bytes;
    });
}
