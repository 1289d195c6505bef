// Internal declarations shared by the host (.cpp) and device (.cu) halves of
// libspmgpu.so.  Nothing here crosses the C ABI (include/spmgpu.h does).
#pragma once
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/spmgpu.h"

namespace spm {

// ---- errors: a thread-local message behind spm_last_error() ----
void set_error(const std::string& msg);
struct Error {
    spm_status code;
    std::string msg;
};
[[noreturn]] void fail(spm_status code, const std::string& msg);

// ---- GGML block geometry (spm-gguf/src/parse.rs:26-45) ----
bool type_layout(uint32_t dtype, uint64_t* block_values, uint64_t* block_bytes);
float f16_to_f32(uint16_t bits);
uint16_t f32_to_f16(float f);

// ---- GGUF container ----
struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;  // ne[0] = innermost (cols)
    uint32_t dtype = 0;
    uint64_t offset = 0;         // absolute byte offset in the image
    uint64_t len = 0;            // byte length
};
struct GgufMeta {
    std::string key;
    uint32_t type = 0;
    bool has_int = false, has_float = false;
    uint64_t u = 0;
    double f = 0;
    std::string s;
};
struct Gguf {
    uint32_t version = 0;
    uint64_t data_offset = 0;
    std::vector<GgufMeta> meta;
    std::vector<GgufTensor> tensors;  // sorted by offset
    const GgufTensor* find(const std::string& name) const;
    const GgufMeta* meta_find(const std::string& key) const;
};
// Bounded parse of an in-memory image (limits of spm-gguf/src/lib.rs:11-16).
Gguf gguf_parse(const uint8_t* buf, uint64_t len);

// ---- host codecs ----
void decode_blocks(uint32_t dtype, const uint8_t* bytes, uint64_t nbytes, float* out);
// Quantize n values (n a multiple of the block size) into GGML blocks.
void quantize(uint32_t dtype, const float* src, uint64_t n, uint8_t* dst);

// ---- synthetic models ----
// Returns a malloc'd GGUF image (release with free) of *len bytes.
uint8_t* synth_gguf(const spm_synth_spec& spec, uint64_t* len);

// ---- .order files (spm-order/src/order.rs) ----
struct Order {
    std::vector<std::string> rotating, resident;
};
Order parse_order(const std::string& text);
std::string default_order(const spm_model_cfg& cfg, bool router_bias);

// ---- packed device layout of one quantized matrix ----
// Rows are grouped in tiles of kTileRows.  Inside a tile every plane is
// contiguous and 16-byte aligned; a plane holds one fixed-size record per
// 32-weight unit (or per 256-weight block) of every row of the tile.  The
// records keep exactly the GGML bytes, rearranged so that one thread owns one
// unit and extracts four codes per 32-bit word.
constexpr int kTileRows = 4;
struct Packed {
    uint32_t dtype = 0;
    uint64_t rows = 0, cols = 0;
    uint64_t tiles = 0, tile_bytes = 0;
    uint32_t plane[4] = {0, 0, 0, 0};  // plane offsets inside a tile
    uint64_t offset = 0;               // offset of tile 0 in the device image
    uint64_t quant_bytes = 0;          // GGML size: rows*cols/bv*bb
};
Packed packed_shape(uint32_t dtype, uint64_t rows, uint64_t cols);
// Repack GGML row-major blocks into `dst` (packed.tiles * tile_bytes bytes).
void pack_matrix(const Packed& p, const uint8_t* gguf_blocks, uint8_t* dst);

// ---- .spm files (spm-header, spm-layout, spm-file) ----
enum : uint8_t { SPM_ENC_TERNARY = 1, SPM_ENC_F32 = 2, SPM_ENC_BF16 = 3, SPM_ENC_Q6K = 4, SPM_ENC_Q5K = 5,
                 SPM_ENC_Q8_0 = 6 };
struct SpmDesc {
    uint32_t rows = 0, cols = 0, group_size = 0;
    uint8_t encoding = 0;
    uint16_t lane_count = 0;
};
struct SpmFile {
    uint16_t major = 0, minor = 0;
    std::vector<SpmDesc> desc;
    uint64_t payload = 0;  // offset of the first group
};
// Header and directory; throws like the reference's parse functions.
SpmFile spm_file_parse(const uint8_t* buf, uint64_t len);
// Placement of one stream's groups in the file.
struct SpmSpan {
    uint64_t offset = 0;   // first group
    uint64_t bytes = 0;    // scales plus payloads of all its groups
    uint64_t groups = 0;
};
// Walks the groups of streams 0..index in file order; throws SPM_E_TRUNCATED
// with the reference's PayloadTruncated message when the file ends inside one.
SpmSpan spm_file_locate(const SpmFile& f, uint64_t len, uint32_t index);

// The device form of one .spm stream, in two steps: plan_* validates the
// stream (the refusals of the matching upload call) and sizes its device
// form; fill_stream writes that form into memory the caller provides, so a
// caller can pack straight into pinned or device-bound buffers.
//   ternary: codes[w * rows_pad + r] holds the 2-bit codes of row r for
//     columns 16w..16w+15 (column 16w+j at bits 2j, 2j+1; padding holds
//     code 0), then at scale_off the f32 scale of every group;
//   dense (F32, Bf16): the group framing removed, column-major with rows
//     padded to 32 (zeros), element (r, c) at c * rows_pad + r, as f32 or the
//     raw bf16 bits;
//   block profiles (Q8_0, Q6K, Q5K): the GGML blocks back to back in source
//     row-major order (the reference's consumers take exactly one block per
//     group, spm-granite-moe/src/layout.rs:225-227, gemma_smoke.rs:219-221).
struct StreamPlan {
    uint8_t encoding = 0;
    uint32_t rows = 0, cols = 0, group_size = 0;
    uint64_t groups = 0, rows_pad = 0, col_words = 0;
    uint64_t offset = 0;         // the stream's first group in the file
    uint64_t bytes = 0;          // size of the device form
    uint64_t scale_off = 0;      // ternary: the scales inside the device form
    uint64_t payload_bytes = 0;  // weight bytes of the stream (scales excluded)
};
StreamPlan plan_ternary(const uint8_t* buf, uint64_t len, uint32_t index);
StreamPlan plan_dense(const uint8_t* buf, uint64_t len, uint32_t index);
StreamPlan plan_qblocks(const uint8_t* buf, uint64_t len, uint32_t index);
// Writes the device form (plan.bytes bytes at dst); returns the number of
// reserved 0b10 codes of a ternary stream (0 otherwise).
uint64_t fill_stream(const uint8_t* buf, const StreamPlan& plan, uint8_t* dst);

// A stream packed into host memory: its plan and device form.
struct PackedStream {
    StreamPlan plan;
    std::vector<uint8_t> data;
    uint64_t reserved_codes = 0;
};
PackedStream pack_ternary(const uint8_t* buf, uint64_t len, uint32_t index);
PackedStream pack_dense(const uint8_t* buf, uint64_t len, uint32_t index);
PackedStream pack_qblocks(const uint8_t* buf, uint64_t len, uint32_t index);

}  // namespace spm
