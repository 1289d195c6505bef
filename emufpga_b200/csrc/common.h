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

// A ternary stream repacked for the device.  codes[w * rows_pad + r] holds the
// 2-bit codes of row r for columns 16w..16w+15 (column 16w+j at bits 2j, 2j+1;
// padding rows and columns hold code 0); scales[g] is group g's scale.
struct TernaryHost {
    uint32_t rows = 0, cols = 0, group_size = 0;
    uint64_t groups = 0, col_words = 0, rows_pad = 0;
    uint64_t payload_bytes = 0;   // packed weight bytes of the stream (scales excluded)
    uint64_t reserved_codes = 0;  // 0b10 codes: no-ops for the datapath, as in the reference
    std::vector<uint32_t> codes;
    std::vector<float> scales;
};
TernaryHost pack_ternary(const uint8_t* buf, uint64_t len, uint32_t index);

// A dense (F32 or Bf16) stream repacked for the device: the group framing
// removed, column-major with rows padded to a multiple of 32 (zeros), element
// (r, c) at c * rows_pad + r, as f32 or as the raw bf16 bits.
struct DenseHost {
    uint32_t rows = 0, cols = 0, group_size = 0;
    uint8_t encoding = 0;
    uint64_t rows_pad = 0, groups = 0, payload_bytes = 0;
    std::vector<uint8_t> data;
};
DenseHost pack_dense(const uint8_t* buf, uint64_t len, uint32_t index);

// A Q-profile stream (Q8_0, Q6_K, Q5_K) with the group framing removed: its
// GGML blocks back to back in source row-major order.  The reference's
// consumers take exactly one block per group (spm-granite-moe/src/
// layout.rs:225-227, gemma_smoke.rs:219-221).
struct QBlockHost {
    uint32_t rows = 0, cols = 0, group_size = 0;
    uint8_t encoding = 0;
    uint64_t groups = 0;
    std::vector<uint8_t> blocks;
};
QBlockHost pack_qblocks(const uint8_t* buf, uint64_t len, uint32_t index);

}  // namespace spm
