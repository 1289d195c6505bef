// Repacking GGML row-major blocks into the device tile layout.
//
// One thread of the GEMV owns one 32-weight unit of a row.  Each plane below
// holds one fixed-size record per unit (or per 256-weight block), so a warp's
// loads of a plane are contiguous.  The records hold exactly the bits of the
// GGML block -- only their positions change -- so the bytes streamed per weight
// equal the GGUF bytes per weight, with one exception: Q5_K's twelve bytes of
// 6-bit scales and mins are stored unpacked, one byte each per unit (sixteen
// bytes per block, 180 instead of 176 per 256 weights), so that a unit's scale
// and min are one 2-byte load instead of a selection among twelve bytes that
// depends on the unit's place in the block.  Inside a unit, weights l and l+16 share a
// byte (low / high nibble) and the high bits of weights 4t..4t+3 sit in the
// same bit slot of four consecutive bytes: one shift and one mask then yield
// four codes, one per byte, ready for the byte-to-float conversion.
//
// Per tile of kTileRows rows (U = cols/32 units, B = cols/256 blocks per row):
//   Q8_0 : QS[TR][U][32]  D[TR][U][2]
//   Q6_K : QL[TR][U][16]  QH[TR][U][8]   SC[TR][U][2]  D[TR][B][2]
//   Q5_K : QS[TR][U][16]  QH[TR][U][4]   SM[TR][U][2] (scale, min)  DM[TR][B][4] (d, dmin)
//   Q2_K : QS[TR][U][8]   SC[TR][U][2]   DD[TR][B][4]  (d, dmin)
//   F32  : W[TR][cols][4]
#include "common.h"

namespace spm {

static uint64_t a16(uint64_t x) { return (x + 15) & ~uint64_t(15); }

Packed packed_shape(uint32_t dtype, uint64_t rows, uint64_t cols) {
    Packed p;
    p.dtype = dtype;
    p.rows = rows;
    p.cols = cols;
    uint64_t bv, bb;
    if (!type_layout(dtype, &bv, &bb)) fail(SPM_E_ENCODING, "unsupported GGML dtype " + std::to_string(dtype));
    if (rows == 0 || cols == 0) fail(SPM_E_ARG, "matrix has a zero dimension");
    p.quant_bytes = rows * (cols / bv) * bb;
    const uint64_t TR = kTileRows, U = cols / 32, B = cols / 256;
    switch (dtype) {
        case SPM_F32:
            if (cols % 32) fail(SPM_E_ARG, "F32 rows must be a multiple of 32 values");
            p.tile_bytes = TR * cols * 4;
            break;
        case SPM_Q8_0:
            if (cols % 32) fail(SPM_E_ARG, "Q8_0 rows must be whole blocks");
            p.plane[1] = uint32_t(TR * U * 32);
            p.tile_bytes = a16(p.plane[1] + TR * U * 2);
            break;
        case SPM_Q6_K:
            if (cols % 256) fail(SPM_E_ARG, "Q6_K rows must be whole blocks");
            p.plane[1] = uint32_t(TR * U * 16);
            p.plane[2] = uint32_t(p.plane[1] + TR * U * 8);
            p.plane[3] = uint32_t(a16(p.plane[2] + TR * U * 2));
            p.tile_bytes = a16(p.plane[3] + TR * B * 2);
            break;
        case SPM_Q5_K:
            if (cols % 256) fail(SPM_E_ARG, "Q5_K rows must be whole blocks");
            p.plane[1] = uint32_t(TR * U * 16);
            p.plane[2] = uint32_t(p.plane[1] + TR * U * 4);
            p.plane[3] = uint32_t(a16(p.plane[2] + TR * U * 2));
            p.tile_bytes = a16(p.plane[3] + TR * B * 4);
            break;
        case SPM_Q2_K:
            if (cols % 256) fail(SPM_E_ARG, "Q2_K rows must be whole blocks");
            p.plane[1] = uint32_t(TR * U * 8);
            p.plane[2] = uint32_t(p.plane[1] + TR * U * 2);
            p.tile_bytes = a16(p.plane[2] + TR * B * 4);
            break;
        default:
            fail(SPM_E_ENCODING, "the device path has no kernel for GGML dtype " + std::to_string(dtype));
    }
    p.tiles = (rows + TR - 1) / TR;
    return p;
}

// The 6-bit codes of Q6_K block `blk`, in weight order (ggml layout,
// spm-gguf/src/tensor.rs:116-136).
static void q6_codes(const uint8_t* blk, uint8_t* q) {
    for (int half = 0; half < 2; half++) {
        const uint8_t* ql = blk + half * 64;
        const uint8_t* qh = blk + 128 + half * 32;
        for (int l = 0; l < 32; l++) {
            q[half * 128 + l] = uint8_t((ql[l] & 15) | ((qh[l] & 3) << 4));
            q[half * 128 + l + 32] = uint8_t((ql[l + 32] & 15) | (((qh[l] >> 2) & 3) << 4));
            q[half * 128 + l + 64] = uint8_t((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4));
            q[half * 128 + l + 96] = uint8_t((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4));
        }
    }
}

// 5-bit codes of a Q5_K block in weight order (spm-gguf/src/tensor.rs:158-174).
static void q5_codes(const uint8_t* blk, uint8_t* q) {
    const uint8_t* qh = blk + 16;
    const uint8_t* qs = blk + 48;
    for (int j = 0; j < 8; j++)
        for (int l = 0; l < 32; l++) {
            uint8_t p = qs[(j / 2) * 32 + l];
            q[32 * j + l] = uint8_t(((j & 1) ? (p >> 4) : (p & 15)) | (((qh[l] >> j) & 1) << 4));
        }
}

// 2-bit codes of a Q2_K block in weight order (ggml block_q2_K).
static void q2_codes(const uint8_t* blk, uint8_t* q) {
    for (int k = 0; k < 256; k++) {
        int n = k / 128, jj = (k % 128) / 32, l = k % 32;
        q[k] = uint8_t((blk[16 + 32 * n + l] >> (2 * jj)) & 3);
    }
}

// Low nibbles of the 32 codes of one unit: byte i = q[i] | q[i+16] << 4.
static void put_nibbles(const uint8_t* q, uint8_t* dst) {
    for (int i = 0; i < 16; i++) dst[i] = uint8_t((q[i] & 15) | ((q[i + 16] & 15) << 4));
}

void pack_matrix(const Packed& p, const uint8_t* src, uint8_t* dst) {
    const uint64_t TR = kTileRows, K = p.cols, U = K / 32, B = K / 256;
    uint64_t bv, bb;
    type_layout(p.dtype, &bv, &bb);
    const uint64_t row_bytes = K / bv * bb;
    std::memset(dst, 0, p.tiles * p.tile_bytes);
    uint8_t q[256];
    for (uint64_t r = 0; r < p.rows; r++) {
        uint8_t* tile = dst + (r / TR) * p.tile_bytes;
        const uint64_t rt = r % TR;
        const uint8_t* row = src + r * row_bytes;
        switch (p.dtype) {
            case SPM_F32:
                std::memcpy(tile + rt * K * 4, row, K * 4);
                break;
            case SPM_Q8_0:
                for (uint64_t u = 0; u < U; u++) {
                    const uint8_t* blk = row + u * 34;
                    std::memcpy(tile + (rt * U + u) * 32, blk + 2, 32);
                    std::memcpy(tile + p.plane[1] + (rt * U + u) * 2, blk, 2);
                }
                break;
            case SPM_Q6_K:
                for (uint64_t b = 0; b < B; b++) {
                    const uint8_t* blk = row + b * 210;
                    q6_codes(blk, q);
                    for (int j = 0; j < 8; j++) {
                        uint64_t u = b * 8 + j;
                        const uint8_t* qq = q + 32 * j;
                        put_nibbles(qq, tile + (rt * U + u) * 16);
                        uint8_t* qh = tile + p.plane[1] + (rt * U + u) * 8;
                        for (int w = 0; w < 2; w++)
                            for (int t = 0; t < 4; t++)
                                for (int bi = 0; bi < 4; bi++)
                                    qh[4 * w + bi] |= uint8_t(((qq[16 * w + 4 * t + bi] >> 4) & 3) << (2 * t));
                        int n = j / 4, g = j % 4;
                        uint8_t* sc = tile + p.plane[2] + (rt * U + u) * 2;
                        sc[0] = blk[192 + 8 * n + 2 * g];
                        sc[1] = blk[192 + 8 * n + 2 * g + 1];
                    }
                    std::memcpy(tile + p.plane[3] + (rt * B + b) * 2, blk + 208, 2);
                }
                break;
            case SPM_Q5_K:
                for (uint64_t b = 0; b < B; b++) {
                    const uint8_t* blk = row + b * 176;
                    q5_codes(blk, q);
                    std::memcpy(tile + p.plane[3] + (rt * B + b) * 4, blk, 4);
                    const uint8_t* s = blk + 4;
                    for (int j = 0; j < 8; j++) {
                        uint64_t u = b * 8 + j;
                        const uint8_t* qq = q + 32 * j;
                        put_nibbles(qq, tile + (rt * U + u) * 16);
                        uint32_t hb = 0;
                        for (int l = 0; l < 32; l++) hb |= uint32_t((qq[l] >> 4) & 1) << l;
                        std::memcpy(tile + p.plane[1] + (rt * U + u) * 4, &hb, 4);
                        // sub-block j's 6-bit scale and min (spm-gguf/src/tensor.rs:141-156)
                        uint8_t* sm = tile + p.plane[2] + (rt * U + u) * 2;
                        if (j < 4) {
                            sm[0] = uint8_t(s[j] & 63);
                            sm[1] = uint8_t(s[j + 4] & 63);
                        } else {
                            sm[0] = uint8_t((s[j + 4] & 15) | ((s[j - 4] >> 6) << 4));
                            sm[1] = uint8_t((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
                        }
                    }
                }
                break;
            case SPM_Q2_K:
                for (uint64_t b = 0; b < B; b++) {
                    const uint8_t* blk = row + b * 84;
                    q2_codes(blk, q);
                    for (int j = 0; j < 8; j++) {
                        uint64_t u = b * 8 + j;
                        const uint8_t* qq = q + 32 * j;
                        uint8_t* qs = tile + (rt * U + u) * 8;
                        for (int w = 0; w < 2; w++)
                            for (int t = 0; t < 4; t++)
                                for (int bi = 0; bi < 4; bi++)
                                    qs[4 * w + bi] |= uint8_t((qq[16 * w + 4 * t + bi] & 3) << (2 * t));
                        int n = j / 4, jj = j % 4;
                        uint8_t* sc = tile + p.plane[1] + (rt * U + u) * 2;
                        sc[0] = blk[8 * n + 2 * jj];
                        sc[1] = blk[8 * n + 2 * jj + 1];
                    }
                    std::memcpy(tile + p.plane[2] + (rt * B + b) * 4, blk + 80, 4);
                }
                break;
        }
    }
}

}  // namespace spm
