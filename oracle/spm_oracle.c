/*
 * spm_oracle.c -- TEST INFRASTRUCTURE ONLY (see spm_oracle.h).
 *
 * CPU restatement of the emufpga decode token loop, used by tests/ as the
 * parity checker and by bench.py as the timed CPU baseline.  Build with
 * -ffp-contract=off (oracle/Makefile): every product and sum below must
 * round exactly where the Rust reference rounds.
 */
#include "spm_oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ */
/* Half floats: spm-gguf/src/tensor.rs:82-98 (exact, subnormals too).  */
/* ------------------------------------------------------------------ */
float or_f16_to_f32(uint16_t bits) {
    uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    uint32_t exp = (bits >> 10) & 0x1fu;
    uint32_t fraction = bits & 0x03ffu;
    uint32_t out;
    if (exp == 0 && fraction == 0) {
        out = sign;
    } else if (exp == 0) {
        uint32_t shift = (uint32_t)__builtin_clz(fraction) - 21u;
        uint32_t normalized = fraction << shift;
        uint32_t exponent = 113u - shift;
        out = sign | (exponent << 23) | ((normalized & 0x03ffu) << 13);
    } else if (exp == 31) {
        out = sign | 0x7f800000u | (fraction << 13);
    } else {
        out = sign | ((exp + 112u) << 23) | (fraction << 13);
    }
    float f;
    memcpy(&f, &out, 4);
    return f;
}

static uint16_t le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* GGML block geometry: spm-gguf/src/parse.rs:26-45. */
int or_type_layout(uint32_t t, uint64_t* bv, uint64_t* bb) {
    uint64_t v, b;
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
        default: return -1;
    }
    if (bv) *bv = v;
    if (bb) *bb = b;
    return 0;
}

/* Q8_0: spm-gguf/src/tensor.rs:193-210.  w = d * (float)(int8)q. */
__attribute__((target_clones("avx2", "default"))) static void dec_q8_0(const uint8_t* blk, float* out) {
    float d = or_f16_to_f32(le16(blk));
    for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)blk[2 + i];
}

/* Q6_K: spm-gguf/src/tensor.rs:103-139.  w = (d * sc) * (q - 32); the
 * product d * sc is formed once per 16 values (the same rounding as forming it
 * per value, which the reference writes). */
__attribute__((target_clones("avx2", "default"))) static void dec_q6_k(const uint8_t* blk, float* out) {
    const uint8_t* ql0 = blk;
    const uint8_t* qh0 = blk + 128;
    const uint8_t* sc0 = blk + 192;
    float d = or_f16_to_f32(le16(blk + 208));
    for (int half = 0; half < 2; half++) {
        const uint8_t* ql = ql0 + half * 64;
        const uint8_t* qh = qh0 + half * 32;
        const uint8_t* sc = sc0 + half * 8;
        float* o = out + half * 128;
        for (int lane = 0; lane < 4; lane++) {
            const uint8_t* qlo = ql + (lane & 1) * 32;
            const int lshift = (lane >> 1) * 4, hshift = lane * 2;
            for (int is = 0; is < 2; is++) {
                const float ds = d * (float)(int8_t)sc[is + lane * 2];
                for (int l = is * 16; l < is * 16 + 16; l++) {
                    const int q = ((qlo[l] >> lshift) & 0x0f) | (((qh[l] >> hshift) & 3) << 4);
                    o[l + lane * 32] = ds * ((float)q - 32.0f);
                }
            }
        }
    }
}

/* spm-gguf/src/tensor.rs:179-188. */
static void scale_min_q5(int index, const uint8_t* p, uint8_t* sc, uint8_t* m) {
    if (index < 4) {
        *sc = p[index] & 63;
        *m = p[index + 4] & 63;
    } else {
        *sc = (uint8_t)((p[index + 4] & 0x0f) | ((p[index - 4] >> 6) << 4));
        *m = (uint8_t)((p[index + 4] >> 4) | ((p[index] >> 6) << 4));
    }
}

/* Q5_K: spm-gguf/src/tensor.rs:144-177.  w = (d*sc)*q - dmin*m; the two
 * products d*sc and dmin*m are formed once per 32 values (the same roundings
 * as forming them per value). */
__attribute__((target_clones("avx2", "default"))) static void dec_q5_k(const uint8_t* blk, float* out) {
    float d = or_f16_to_f32(le16(blk));
    float dmin = or_f16_to_f32(le16(blk + 2));
    const uint8_t* scales = blk + 4;
    const uint8_t* qh = blk + 16;
    const uint8_t* qs = blk + 48;
    for (int group = 0; group < 4; group++) {
        for (int half = 0; half < 2; half++) {
            int index = group * 2 + half;
            uint8_t sc, mn;
            scale_min_q5(index, scales, &sc, &mn);
            const float ds = d * (float)sc, dm = dmin * (float)mn;
            float* o = out + index * 32;
            for (int lane = 0; lane < 32; lane++) {
                const int low = (qs[group * 32 + lane] >> (half * 4)) & 0x0f;
                const int quant = low + (((qh[lane] >> index) & 1) << 4);
                o[lane] = ds * (float)quant - dm;
            }
        }
    }
}

/* Q2_K: not in the reference (GGUF dtype 10 is only sized, parse.rs:36).
 * Follows ggml's published block_q2_K: scales[16] (low nibble scale, high
 * nibble min), qs[64] (four 2-bit planes per 32 bytes), d, dmin (fp16).
 * w = (d*(sc&15)) * q - (dmin*(sc>>4)).  Pinned against gguf-py 0.19.0. */
__attribute__((target_clones("avx2", "default"))) static void dec_q2_k(const uint8_t* blk, float* out) {
    const uint8_t* scales = blk;
    const uint8_t* qs = blk + 16;
    float d = or_f16_to_f32(le16(blk + 80));
    float dmin = or_f16_to_f32(le16(blk + 82));
    int is = 0, k = 0;
    for (int n = 0; n < 2; n++) {
        const uint8_t* q = qs + n * 32;
        for (int j = 0; j < 4; j++) {
            int shift = 2 * j;
            for (int part = 0; part < 2; part++) {
                uint8_t sc = scales[is++];
                float dl = d * (float)(sc & 0xf);
                float ml = dmin * (float)(sc >> 4);
                for (int l = 0; l < 16; l++) {
                    float qv = (float)((q[part * 16 + l] >> shift) & 3);
                    out[k++] = dl * qv - ml;
                }
            }
        }
    }
}

int or_decode(uint32_t t, const uint8_t* bytes, uint64_t nbytes, float* out) {
    uint64_t bv, bb;
    if (or_type_layout(t, &bv, &bb) != 0) return -2;
    if (nbytes % bb != 0) return -1;
    uint64_t nb = nbytes / bb;
    switch (t) {
        case OR_F32:
            for (uint64_t i = 0; i < nb; i++) memcpy(out + i, bytes + 4 * i, 4);
            return 0;
        case OR_F16:
            for (uint64_t i = 0; i < nb; i++) out[i] = or_f16_to_f32(le16(bytes + 2 * i));
            return 0;
        case OR_Q8_0:
            for (uint64_t i = 0; i < nb; i++) dec_q8_0(bytes + i * bb, out + i * bv);
            return 0;
        case OR_Q6_K:
            for (uint64_t i = 0; i < nb; i++) dec_q6_k(bytes + i * bb, out + i * bv);
            return 0;
        case OR_Q5_K:
            for (uint64_t i = 0; i < nb; i++) dec_q5_k(bytes + i * bb, out + i * bv);
            return 0;
        case OR_Q2_K:
            for (uint64_t i = 0; i < nb; i++) dec_q2_k(bytes + i * bb, out + i * bv);
            return 0;
        default:
            return -2;
    }
}

/* ------------------------------------------------------------------ */
/* GGUF: a bounded restatement of spm-gguf/src/parse.rs:31-182 and     */
/* wire.rs:10-91, reading from memory instead of a file.               */
/* ------------------------------------------------------------------ */
#define OR_MAX_METADATA 1000000ull
#define OR_MAX_TENSORS 1000000ull
#define OR_MAX_STRING (16ull * 1024 * 1024)
#define OR_MAX_ARRAY 2000000ull
#define OR_MAX_DIMS 8u
#define OR_MAX_HEADER_BYTES (512ull * 1024 * 1024)

typedef struct {
    char* name;
    uint64_t dims[OR_MAX_DIMS];
    uint32_t ndims, dtype;
    uint64_t offset, len;
} or_tensor;

struct or_gguf {
    uint64_t count;
    or_tensor* t;
    uint64_t alignment;
};

typedef struct {
    const uint8_t* buf;
    uint64_t pos, len;
    char* err;
    int errlen;
} parser;

static int perr(parser* p, const char* msg) {
    if (p->err && p->errlen > 0) snprintf(p->err, (size_t)p->errlen, "%s", msg);
    return -1;
}

static int take(parser* p, uint64_t n, const uint8_t** out) {
    uint64_t end = p->pos + n;
    if (end < p->pos) return perr(p, "file position overflow");
    if (end > OR_MAX_HEADER_BYTES) return perr(p, "GGUF header exceeds limit");
    if (end > p->len) return perr(p, "unexpected end of GGUF");
    *out = p->buf + p->pos;
    p->pos = end;
    return 0;
}
static int rd_u32(parser* p, uint32_t* v) {
    const uint8_t* b;
    if (take(p, 4, &b)) return -1;
    memcpy(v, b, 4);
    return 0;
}
static int rd_u64(parser* p, uint64_t* v) {
    const uint8_t* b;
    if (take(p, 8, &b)) return -1;
    memcpy(v, b, 8);
    return 0;
}
static int rd_string(parser* p, const uint8_t** s, uint64_t* n) {
    if (rd_u64(p, n)) return -1;
    if (*n > OR_MAX_STRING) return perr(p, "string length exceeds limit");
    return take(p, *n, s);
}

/* wire.rs:49-91.  `want_u64` receives integer values (for general.alignment). */
static int rd_value(parser* p, uint32_t ty, int depth, int* has_int, uint64_t* ival) {
    const uint8_t* b;
    uint64_t n;
    if (depth > 4) return perr(p, "metadata nesting exceeds limit");
    *has_int = 0;
    switch (ty) {
        case 0: case 1: if (take(p, 1, &b)) return -1; *has_int = ty == 0; *ival = b[0]; return 0;
        case 2: case 3: if (take(p, 2, &b)) return -1; *has_int = ty == 2; *ival = le16(b); return 0;
        case 4: case 5: { uint32_t v; if (rd_u32(p, &v)) return -1; *has_int = ty == 4; *ival = v; return 0; }
        case 6: return take(p, 4, &b);
        case 7: if (take(p, 1, &b)) return -1; if (b[0] > 1) return perr(p, "invalid boolean metadata value"); return 0;
        case 8: return rd_string(p, &b, &n);
        case 9: {
            uint32_t inner;
            if (rd_u32(p, &inner) || rd_u64(p, &n)) return -1;
            if (n > OR_MAX_ARRAY) return perr(p, "array length exceeds limit");
            for (uint64_t i = 0; i < n; i++) {
                int hi; uint64_t iv;
                if (rd_value(p, inner, depth + 1, &hi, &iv)) return -1;
            }
            return 0;
        }
        case 10: case 11: if (rd_u64(p, ival)) return -1; *has_int = ty == 10; return 0;
        case 12: return take(p, 8, &b);
        default: return perr(p, "unknown metadata type");
    }
}

static int cmp_offset(const void* a, const void* b) {
    const or_tensor* x = (const or_tensor*)a;
    const or_tensor* y = (const or_tensor*)b;
    return x->offset < y->offset ? -1 : x->offset > y->offset ? 1 : 0;
}

void or_gguf_free(or_gguf* g) {
    if (!g) return;
    for (uint64_t i = 0; i < g->count; i++) free(g->t[i].name);
    free(g->t);
    free(g);
}

int or_gguf_parse(const uint8_t* buf, uint64_t len, or_gguf** out, char* err, int errlen) {
    parser P = {buf, 0, len, err, errlen};
    parser* p = &P;
    const uint8_t* b;
    *out = NULL;
    if (take(p, 4, &b)) return -1;
    if (memcmp(b, "GGUF", 4) != 0) return perr(p, "invalid GGUF magic");
    uint32_t version;
    uint64_t tensors, metadata;
    if (rd_u32(p, &version)) return -1;
    if (version != 3) return perr(p, "unsupported GGUF version");
    if (rd_u64(p, &tensors) || rd_u64(p, &metadata)) return -1;
    if (tensors > OR_MAX_TENSORS) return perr(p, "tensor count exceeds limit");
    if (metadata > OR_MAX_METADATA) return perr(p, "metadata count exceeds limit");
    uint64_t align = 32;
    for (uint64_t i = 0; i < metadata; i++) {
        const uint8_t* key;
        uint64_t klen;
        uint32_t ty;
        int hi;
        uint64_t iv = 0;
        if (rd_string(p, &key, &klen) || rd_u32(p, &ty)) return -1;
        if (rd_value(p, ty, 0, &hi, &iv)) return -1;
        if (hi && klen == 17 && memcmp(key, "general.alignment", 17) == 0) align = iv;
    }
    or_gguf* g = (or_gguf*)calloc(1, sizeof(or_gguf));
    g->t = (or_tensor*)calloc(tensors ? tensors : 1, sizeof(or_tensor));
    g->alignment = align;
    for (uint64_t i = 0; i < tensors; i++) {
        const uint8_t* name;
        uint64_t nlen;
        if (rd_string(p, &name, &nlen)) goto fail;
        or_tensor* t = &g->t[i];
        t->name = (char*)malloc(nlen + 1);
        memcpy(t->name, name, nlen);
        t->name[nlen] = 0;
        g->count = i + 1;
        for (uint64_t j = 0; j < i; j++)
            if (strcmp(g->t[j].name, t->name) == 0) { perr(p, "duplicate tensor name"); goto fail; }
        if (rd_u32(p, &t->ndims)) goto fail;
        if (t->ndims == 0 || t->ndims > OR_MAX_DIMS) { perr(p, "invalid dimension count"); goto fail; }
        for (uint32_t d = 0; d < t->ndims; d++)
            if (rd_u64(p, &t->dims[d])) goto fail;
        if (rd_u32(p, &t->dtype) || rd_u64(p, &t->offset)) goto fail;
    }
    if (align == 0 || (align & (align - 1)) != 0) { perr(p, "invalid alignment"); goto fail; }
    uint64_t base = (p->pos + align - 1) & ~(align - 1);
    if (base > len) { perr(p, "tensor data starts beyond file"); goto fail; }
    for (uint64_t i = 0; i < tensors; i++) {
        or_tensor* t = &g->t[i];
        if (t->offset % align != 0) { perr(p, "unaligned tensor"); goto fail; }
        uint64_t elems = 1;
        for (uint32_t d = 0; d < t->ndims; d++) {
            if (t->dims[d] == 0) { perr(p, "tensor has a zero dimension"); goto fail; }
            if (elems > UINT64_MAX / t->dims[d]) { perr(p, "tensor element count overflow"); goto fail; }
            elems *= t->dims[d];
        }
        uint64_t bv, bb;
        if (or_type_layout(t->dtype, &bv, &bb)) { perr(p, "unsupported GGML dtype"); goto fail; }
        if (elems % bv != 0) { perr(p, "tensor does not fill dtype blocks"); goto fail; }
        uint64_t nblk = elems / bv;
        if (nblk > UINT64_MAX / bb) { perr(p, "tensor byte length overflow"); goto fail; }
        t->len = nblk * bb;
        uint64_t off = base + t->offset;
        if (off < base) { perr(p, "tensor offset overflow"); goto fail; }
        if (off + t->len < off || off + t->len > len) { perr(p, "tensor extends beyond file"); goto fail; }
        t->offset = off;
    }
    qsort(g->t, tensors, sizeof(or_tensor), cmp_offset);
    for (uint64_t i = 1; i < tensors; i++)
        if (g->t[i - 1].offset + g->t[i - 1].len > g->t[i].offset) { perr(p, "overlapping tensor ranges"); goto fail; }
    *out = g;
    return 0;
fail:
    or_gguf_free(g);
    return -1;
}

int or_gguf_find(const or_gguf* g, const char* name, uint32_t* dtype, uint64_t* dims4,
                 uint32_t* ndims, uint64_t* offset, uint64_t* nbytes) {
    for (uint64_t i = 0; i < g->count; i++) {
        if (strcmp(g->t[i].name, name) == 0) {
            if (dtype) *dtype = g->t[i].dtype;
            if (ndims) *ndims = g->t[i].ndims;
            if (dims4)
                for (int d = 0; d < 4; d++) dims4[d] = d < (int)g->t[i].ndims ? g->t[i].dims[d] : 1;
            if (offset) *offset = g->t[i].offset;
            if (nbytes) *nbytes = g->t[i].len;
            return 0;
        }
    }
    return -1;
}

uint64_t or_gguf_tensor_count(const or_gguf* g) { return g->count; }

/* ------------------------------------------------------------------ */
/* Streamed GEMV.                                                      */
/* ------------------------------------------------------------------ */
static int nthreads(int threads) {
#ifdef _OPENMP
    return threads > 0 ? threads : omp_get_max_threads();
#else
    (void)threads;
    return 1;
#endif
}

/* Each (position,row) accumulator is the reference's sequential chain
 * out = fma(w, x[col], out) over col ascending, starting from +0.0:
 * spm-linear/src/resident.rs:124-137 (apply_weight) and
 * spm-granite-moe/src/layout.rs:232-238 (q6_operation).  Rows are
 * independent, so spreading rows over threads leaves every bit unchanged.
 *
 * Speed without changing a bit: R rows x P positions chains advance together
 * column by column (each chain still adds its columns in ascending order from
 * +0.0), so the CPU overlaps independent chains instead of waiting on one;
 * fmaf is the correctly rounded fused multiply-add whether it runs as the FMA
 * instruction (the "fma" clone, chosen at load time where the CPU has it) or
 * as the libm call.  The plain-dot form (or_gemv_dot) keeps its separately
 * rounded multiply and add (-ffp-contract=off). */
#define OR_STEP_FMA(w, x, a) fmaf((w), (x), (a))
#define OR_STEP_DOT(w, x, a) ((a) + (x) * (w))
#define OR_CHAINS(NAME, R, P, STEP)                                                          \
    __attribute__((target_clones("fma", "default"))) static void NAME(                       \
        const float* w, uint64_t cols, const float* x, uint64_t xs, float* out) {            \
        float a[R][P];                                                                       \
        for (int r = 0; r < R; r++)                                                          \
            for (int p = 0; p < P; p++) a[r][p] = 0.0f;                                      \
        for (uint64_t c = 0; c < cols; c++) {                                                \
            float xv[P];                                                                     \
            _Pragma("GCC unroll 8") for (int p = 0; p < P; p++) xv[p] = x[(uint64_t)p * xs + c]; \
            _Pragma("GCC unroll 8") for (int r = 0; r < R; r++) {                            \
                const float wv = w[(uint64_t)r * cols + c];                                  \
                _Pragma("GCC unroll 8") for (int p = 0; p < P; p++) a[r][p] = STEP(wv, xv[p], a[r][p]); \
            }                                                                                \
        }                                                                                    \
        for (int r = 0; r < R; r++)                                                          \
            for (int p = 0; p < P; p++) out[r * P + p] = a[r][p];                            \
    }
OR_CHAINS(fma_8x1, 8, 1, OR_STEP_FMA)
OR_CHAINS(fma_4x2, 4, 2, OR_STEP_FMA)
OR_CHAINS(fma_3x3, 3, 3, OR_STEP_FMA)
OR_CHAINS(fma_2x4, 2, 4, OR_STEP_FMA)
OR_CHAINS(fma_1x1, 1, 1, OR_STEP_FMA)
OR_CHAINS(fma_1x2, 1, 2, OR_STEP_FMA)
OR_CHAINS(fma_1x3, 1, 3, OR_STEP_FMA)
OR_CHAINS(fma_1x4, 1, 4, OR_STEP_FMA)
OR_CHAINS(dot_8x1, 8, 1, OR_STEP_DOT)
OR_CHAINS(dot_4x2, 4, 2, OR_STEP_DOT)
OR_CHAINS(dot_3x3, 3, 3, OR_STEP_DOT)
OR_CHAINS(dot_2x4, 2, 4, OR_STEP_DOT)
OR_CHAINS(dot_1x1, 1, 1, OR_STEP_DOT)
OR_CHAINS(dot_1x2, 1, 2, OR_STEP_DOT)
OR_CHAINS(dot_1x3, 1, 3, OR_STEP_DOT)
OR_CHAINS(dot_1x4, 1, 4, OR_STEP_DOT)

typedef void (*or_chain_fn)(const float*, uint64_t, const float*, uint64_t, float*);
#define OR_ROW_BLOCK 8

/* Rows [r0, r0+nr) decoded in w (nr <= OR_ROW_BLOCK rows of cols values):
 * every (position, row) chain of them, into y[pos][row]. */
static void chains_block(const float* w, uint64_t r0, int nr, uint64_t rows, uint64_t cols, const float* x,
                         int positions, float* y, int fused) {
    static const or_chain_fn wide_fma[5] = {0, fma_8x1, fma_4x2, fma_3x3, fma_2x4};
    static const or_chain_fn wide_dot[5] = {0, dot_8x1, dot_4x2, dot_3x3, dot_2x4};
    static const or_chain_fn one_fma[5] = {0, fma_1x1, fma_1x2, fma_1x3, fma_1x4};
    static const or_chain_fn one_dot[5] = {0, dot_1x1, dot_1x2, dot_1x3, dot_1x4};
    static const int wide_rows[5] = {0, 8, 4, 3, 2};
    float out[8 * 4];
    for (int p0 = 0; p0 < positions; p0 += 4) {
        const int pc = positions - p0 < 4 ? positions - p0 : 4;
        const int R = wide_rows[pc];
        int r = 0;
        for (; r + R <= nr; r += R) {
            (fused ? wide_fma : wide_dot)[pc](w + (uint64_t)r * cols, cols, x + (uint64_t)p0 * cols, cols, out);
            for (int i = 0; i < R; i++)
                for (int p = 0; p < pc; p++) y[(uint64_t)(p0 + p) * rows + r0 + (uint64_t)(r + i)] = out[i * pc + p];
        }
        for (; r < nr; r++) {
            (fused ? one_fma : one_dot)[pc](w + (uint64_t)r * cols, cols, x + (uint64_t)p0 * cols, cols, out);
            for (int p = 0; p < pc; p++) y[(uint64_t)(p0 + p) * rows + r0 + (uint64_t)r] = out[p];
        }
    }
}

static int gemv_impl(uint32_t t, const uint8_t* blocks, uint64_t rows, uint64_t cols,
                     const float* x, int positions, float* y, int threads, int fused) {
    uint64_t bv, bb;
    if (or_type_layout(t, &bv, &bb)) return -2;
    if (cols % bv != 0) return -1;
    uint64_t row_bytes = cols / bv * bb;
    int nt = nthreads(threads);
    const int64_t nblocks = (int64_t)((rows + OR_ROW_BLOCK - 1) / OR_ROW_BLOCK);
#pragma omp parallel num_threads(nt) if (nt > 1)
    {
        float* w = (float*)malloc(OR_ROW_BLOCK * cols * sizeof(float) + 1);
#pragma omp for schedule(static)
        for (int64_t b = 0; b < nblocks; b++) {
            const uint64_t r0 = (uint64_t)b * OR_ROW_BLOCK;
            const int nr = (int)(rows - r0 < OR_ROW_BLOCK ? rows - r0 : OR_ROW_BLOCK);
            for (int i = 0; i < nr; i++)
                or_decode(t, blocks + (r0 + (uint64_t)i) * row_bytes, row_bytes, w + (uint64_t)i * cols);
            chains_block(w, r0, nr, rows, cols, x, positions, y, fused);
        }
        free(w);
    }
    return 0;
}

int or_gemv_fma(uint32_t t, const uint8_t* blocks, uint64_t rows, uint64_t cols, const float* x,
                int positions, float* y, int threads) {
    return gemv_impl(t, blocks, rows, cols, x, positions, y, threads, 1);
}

/* spm-batch/src/inner.rs:89-105 (finish) and spm-qwen3-slice/src/math.rs:12-20
 * (matvec): `zip(a, b).map(|(a, b)| a * b).sum()`, no fused multiply-add. */
int or_gemv_dot(uint32_t t, const uint8_t* blocks, uint64_t rows, uint64_t cols, const float* x,
                int positions, float* y, int threads) {
    return gemv_impl(t, blocks, rows, cols, x, positions, y, threads, 0);
}

/* ------------------------------------------------------------------ */
/* Elementwise ops.                                                    */
/* ------------------------------------------------------------------ */
/* spm-smol-ops/src/norm.rs:12-21: mean of squares, 1/sqrt(mean+eps), x*s*g. */
void or_scaled_rms_norm(float* values, const float* weight, float eps, int width, int rows) {
    for (int r = 0; r < rows; r++) {
        float* row = values + (size_t)r * width;
        float count = (float)(width > 65535 ? 65535 : width);
        float sum = 0.0f;
        for (int i = 0; i < width; i++) sum = sum + row[i] * row[i];
        float mean = sum / count;
        float scale = 1.0f / sqrtf(mean + eps);
        for (int i = 0; i < width; i++) row[i] = row[i] * scale * weight[i];
    }
}

/* spm-qwen3-slice/src/math.rs:1-10 (and spm-granite-moe math.rs:1-11). */
void or_rms_norm_slice(const float* input, const float* weight, int n, float eps, float* out) {
    float count = (float)n;
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum = sum + input[i] * input[i];
    float ms = sum / count;
    float scale = 1.0f / sqrtf(ms + eps);
    for (int i = 0; i < n; i++) out[i] = input[i] * scale * weight[i];
}

/* spm-ops/src/attention.rs:20-31: theta = base^(-2i/d) * pos, FMA rotation. */
void or_rope_smol(float* head, int dim, int position, float base) {
    float width = (float)dim;
    float at = (float)position;
    int half = dim / 2;
    for (int pair = 0; pair < half; pair++) {
        float index = (float)pair;
        float theta = powf(base, -2.0f * index / width) * at;
        float s = sinf(theta), c = cosf(theta);
        float x = head[pair], y = head[pair + half];
        head[pair] = fmaf(x, c, -(y * s));
        head[pair + half] = fmaf(x, s, y * c);
    }
}

/* spm-qwen3-slice/src/attention.rs:11-25: angle = pos / base^(2i/d), no FMA. */
void or_rope_slice(float* head, int dim, int position, float base) {
    int half = dim / 2;
    for (int index = 0; index < half; index++) {
        float index_f = (float)index;
        float width = (float)dim;
        float pos = (float)position;
        float exponent = 2.0f * index_f / width;
        float angle = pos / powf(base, exponent);
        float s = sinf(angle), c = cosf(angle);
        float left = head[index], right = head[index + half];
        head[index] = left * c - right * s;
        head[index + half] = right * c + left * s;
    }
}

/* spm-ops/src/nonlinear.rs:4-7. */
float or_silu(float x) { return x / (1.0f + expf(-x)); }

/* spm-kv/src/attend.rs:37-94 (attend_head + attend_cached).  keys/values are
 * positions x (kv_heads*head_dim). */
void or_attend_cached(const float* query, const float* keys, const float* values, int positions,
                      int heads, int kv_heads, int head_dim, float* out) {
    int group = heads / kv_heads, stride = kv_heads * head_dim;
    float* scores = (float*)malloc(sizeof(float) * (positions > 0 ? positions : 1));
    float scale = 1.0f / sqrtf((float)head_dim);
    for (int h = 0; h < heads; h++) {
        const float* q = query + h * head_dim;
        int offset = (h / group) * head_dim;
        float* o = out + h * head_dim;
        for (int p = 0; p < positions; p++) {
            const float* k = keys + (size_t)p * stride + offset;
            float dot = 0.0f;
            for (int i = 0; i < head_dim; i++) dot = dot + q[i] * k[i];
            scores[p] = dot * scale;
        }
        if (positions > 0) {
            float mx = scores[0];
            for (int p = 1; p < positions; p++) mx = fmaxf(mx, scores[p]);
            float total = 0.0f;
            for (int p = 0; p < positions; p++) {
                scores[p] = expf(scores[p] - mx);
                total = total + scores[p];
            }
            for (int p = 0; p < positions; p++) scores[p] = scores[p] / total;
        }
        for (int i = 0; i < head_dim; i++) o[i] = 0.0f;
        for (int p = 0; p < positions; p++) {
            const float* v = values + (size_t)p * stride + offset;
            for (int i = 0; i < head_dim; i++) o[i] = fmaf(scores[p], v[i], o[i]);
        }
    }
    free(scores);
}

/* spm-qwen3-slice/src/attention.rs:36-79 (softmax + causal_gqa) for the one
 * query at the end of the cached prefix.  The slice divides by the f32 literal
 * 11.313708 for head_dim 128, which is sqrtf(128). */
void or_attend_slice(const float* query, const float* keys, const float* values, int positions,
                     int heads, int kv_heads, int head_dim, float* out) {
    int stride = kv_heads * head_dim;
    float* scores = (float*)malloc(sizeof(float) * (positions > 0 ? positions : 1));
    float denom = sqrtf((float)head_dim);
    for (int h = 0; h < heads; h++) {
        int kvh = h / (heads / kv_heads);
        const float* q = query + h * head_dim;
        for (int p = 0; p < positions; p++) {
            const float* k = keys + (size_t)p * stride + kvh * head_dim;
            float dot = 0.0f;
            for (int i = 0; i < head_dim; i++) dot = dot + q[i] * k[i];
            scores[p] = dot / denom;
        }
        float mx = -INFINITY;
        for (int p = 0; p < positions; p++) mx = fmaxf(mx, scores[p]);
        float sum = 0.0f;
        for (int p = 0; p < positions; p++) {
            scores[p] = expf(scores[p] - mx);
            sum = sum + scores[p];
        }
        for (int p = 0; p < positions; p++) scores[p] = scores[p] / sum;
        for (int lane = 0; lane < head_dim; lane++) {
            float acc = 0.0f;
            for (int p = 0; p < positions; p++)
                acc = acc + values[(size_t)p * stride + kvh * head_dim + lane] * scores[p];
            out[h * head_dim + lane] = acc;
        }
    }
    free(scores);
}

/* spm-granite-moe/src/math.rs:23-29. */
void or_softmax_route(const float* values, int n, float* out) {
    float mx = -INFINITY;
    for (int i = 0; i < n; i++) mx = fmaxf(mx, values[i]);
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        out[i] = expf(values[i] - mx);
        sum = sum + out[i];
    }
    for (int i = 0; i < n; i++) out[i] = out[i] / sum;
}

/* f32::total_cmp key. */
static int32_t total_key(float f) {
    int32_t b;
    memcpy(&b, &f, 4);
    b ^= (int32_t)(((uint32_t)(b >> 31)) >> 1);
    return b;
}

/* spm-granite-moe/src/math.rs:35-39: descending by total_cmp, ties -> lower id. */
void or_top_k(const float* values, int n, int k, int* ids, float* vals) {
    int* used = (int*)calloc((size_t)n, sizeof(int));
    for (int j = 0; j < k && j < n; j++) {
        int best = -1;
        for (int i = 0; i < n; i++) {
            if (used[i]) continue;
            if (best < 0 || total_key(values[i]) > total_key(values[best])) best = i;
        }
        used[best] = 1;
        ids[j] = best;
        vals[j] = values[best];
    }
    free(used);
}

/* spm-batch/examples/serve-demo.rs:74-79: max_by(partial_cmp) keeps the LAST
 * of equal maxima. */
uint32_t or_argmax_last(const float* row, uint64_t n) {
    uint64_t best = 0;
    for (uint64_t i = 1; i < n; i++)
        if (!(row[best] > row[i])) best = i;
    return (uint32_t)best;
}

/* ------------------------------------------------------------------ */
/* Model and token loop.                                               */
/* ------------------------------------------------------------------ */
typedef struct {
    uint32_t dtype;
    uint64_t rows, cols, experts;
    const uint8_t* data;
    uint64_t nbytes;
} or_w;

typedef struct {
    float *attn_norm, *ffn_norm, *q_norm, *k_norm, *router_bias;
    or_w q, k, v, o, gate, up, down, router, gate_exps, up_exps, down_exps;
} or_layer;

struct or_model {
    or_cfg cfg;
    or_gguf* g;
    const uint8_t* base;
    or_layer* layers;
    or_w embed, head;
    float* output_norm;
    int moe;
};

struct or_session {
    or_model* m;
    int clients, context;
    int* len;
    float *keys, *values;   /* [client][layer][context][kv_width] */
    float *states, *normed, *q, *k, *v, *attn, *gate, *up, *proj, *act, *combined;
    float *router, *probs;
    float* margins;         /* [layer][client] routing margin of the last step */
};

static int load_w(or_model* m, const char* name, or_w* w, int required, char* err, int errlen) {
    uint32_t dt, nd;
    uint64_t dims[4], off, nb;
    memset(w, 0, sizeof(*w));
    if (or_gguf_find(m->g, name, &dt, dims, &nd, &off, &nb) != 0) {
        if (required && err) snprintf(err, (size_t)errlen, "missing tensor %s", name);
        return required ? -1 : 0;
    }
    w->dtype = dt;
    w->cols = dims[0];
    w->rows = dims[1];
    w->experts = dims[2];
    w->data = m->base + off;
    w->nbytes = nb;
    return 0;
}

static float* load_f32(or_model* m, const char* name, uint64_t expect, int required, char* err, int errlen) {
    or_w w;
    if (load_w(m, name, &w, required, err, errlen)) return NULL;
    if (!w.data) return NULL;
    uint64_t bv, bb;
    or_type_layout(w.dtype, &bv, &bb);
    uint64_t n = w.nbytes / bb * bv;
    if (n != expect) {
        if (err) snprintf(err, (size_t)errlen, "tensor %s has %llu values, want %llu", name,
                          (unsigned long long)n, (unsigned long long)expect);
        return NULL;
    }
    float* out = (float*)malloc(n * sizeof(float));
    or_decode(w.dtype, w.data, w.nbytes, out);
    return out;
}

void or_model_free(or_model* m) {
    if (!m) return;
    if (m->layers) {
        for (uint32_t l = 0; l < m->cfg.layers; l++) {
            or_layer* L = &m->layers[l];
            free(L->attn_norm); free(L->ffn_norm); free(L->q_norm); free(L->k_norm); free(L->router_bias);
        }
        free(m->layers);
    }
    free(m->output_norm);
    or_gguf_free(m->g);
    free(m);
}

or_model* or_model_new(const uint8_t* gguf, uint64_t len, const or_cfg* cfg, char* err, int errlen) {
    or_model* m = (or_model*)calloc(1, sizeof(or_model));
    m->cfg = *cfg;
    m->base = gguf;
    if (or_gguf_parse(gguf, len, &m->g, err, errlen)) { free(m); return NULL; }
    const or_cfg* c = &m->cfg;
    m->moe = c->family == OR_FAMILY_OLMOE || c->family == OR_FAMILY_QWEN3MOE;
    uint64_t qw = (uint64_t)c->heads * c->head_dim;
    m->layers = (or_layer*)calloc(c->layers, sizeof(or_layer));
    char name[256];
#define NEED(expr) do { if (expr) goto fail; } while (0)
    for (uint32_t l = 0; l < c->layers; l++) {
        or_layer* L = &m->layers[l];
        snprintf(name, sizeof name, "blk.%u.attn_norm.weight", l);
        NEED(!(L->attn_norm = load_f32(m, name, c->hidden, 1, err, errlen)));
        snprintf(name, sizeof name, "blk.%u.ffn_norm.weight", l);
        NEED(!(L->ffn_norm = load_f32(m, name, c->hidden, 1, err, errlen)));
        if (c->family != OR_FAMILY_LLAMA) {
            uint64_t qn = c->family == OR_FAMILY_OLMOE ? qw : c->head_dim;
            uint64_t kn = c->family == OR_FAMILY_OLMOE ? (uint64_t)c->kv_heads * c->head_dim : c->head_dim;
            snprintf(name, sizeof name, "blk.%u.attn_q_norm.weight", l);
            NEED(!(L->q_norm = load_f32(m, name, qn, 1, err, errlen)));
            snprintf(name, sizeof name, "blk.%u.attn_k_norm.weight", l);
            NEED(!(L->k_norm = load_f32(m, name, kn, 1, err, errlen)));
        }
        snprintf(name, sizeof name, "blk.%u.attn_q.weight", l); NEED(load_w(m, name, &L->q, 1, err, errlen));
        snprintf(name, sizeof name, "blk.%u.attn_k.weight", l); NEED(load_w(m, name, &L->k, 1, err, errlen));
        snprintf(name, sizeof name, "blk.%u.attn_v.weight", l); NEED(load_w(m, name, &L->v, 1, err, errlen));
        snprintf(name, sizeof name, "blk.%u.attn_output.weight", l); NEED(load_w(m, name, &L->o, 1, err, errlen));
        if (m->moe) {
            snprintf(name, sizeof name, "blk.%u.ffn_gate_inp.weight", l); NEED(load_w(m, name, &L->router, 1, err, errlen));
            snprintf(name, sizeof name, "blk.%u.ffn_gate_exps.weight", l); NEED(load_w(m, name, &L->gate_exps, 1, err, errlen));
            snprintf(name, sizeof name, "blk.%u.ffn_up_exps.weight", l); NEED(load_w(m, name, &L->up_exps, 1, err, errlen));
            snprintf(name, sizeof name, "blk.%u.ffn_down_exps.weight", l); NEED(load_w(m, name, &L->down_exps, 1, err, errlen));
            snprintf(name, sizeof name, "blk.%u.exp_probs_b.bias", l);
            L->router_bias = load_f32(m, name, c->experts, 0, err, errlen);
        } else {
            snprintf(name, sizeof name, "blk.%u.ffn_gate.weight", l); NEED(load_w(m, name, &L->gate, 1, err, errlen));
            snprintf(name, sizeof name, "blk.%u.ffn_up.weight", l); NEED(load_w(m, name, &L->up, 1, err, errlen));
            snprintf(name, sizeof name, "blk.%u.ffn_down.weight", l); NEED(load_w(m, name, &L->down, 1, err, errlen));
        }
    }
    NEED(load_w(m, "token_embd.weight", &m->embed, 1, err, errlen));
    if (c->tied) m->head = m->embed;
    else NEED(load_w(m, "output.weight", &m->head, 1, err, errlen));
    NEED(!(m->output_norm = load_f32(m, "output_norm.weight", c->hidden, 1, err, errlen)));
#undef NEED
    return m;
fail:
    or_model_free(m);
    return NULL;
}

or_session* or_session_new(or_model* m, int clients, int context) {
    const or_cfg* c = &m->cfg;
    or_session* s = (or_session*)calloc(1, sizeof(or_session));
    s->m = m;
    s->clients = clients;
    s->context = context;
    size_t kvw = (size_t)c->kv_heads * c->head_dim;
    size_t qw = (size_t)c->heads * c->head_dim;
    size_t ff = c->intermediate > c->expert_ff ? c->intermediate : c->expert_ff;
    s->len = (int*)calloc((size_t)clients, sizeof(int));
    s->keys = (float*)calloc((size_t)clients * c->layers * context * kvw, sizeof(float));
    s->values = (float*)calloc((size_t)clients * c->layers * context * kvw, sizeof(float));
    s->states = (float*)calloc((size_t)clients * c->hidden, sizeof(float));
    s->normed = (float*)calloc((size_t)clients * c->hidden, sizeof(float));
    s->q = (float*)calloc((size_t)clients * qw, sizeof(float));
    s->k = (float*)calloc((size_t)clients * kvw, sizeof(float));
    s->v = (float*)calloc((size_t)clients * kvw, sizeof(float));
    s->attn = (float*)calloc((size_t)clients * qw, sizeof(float));
    s->gate = (float*)calloc((size_t)clients * ff, sizeof(float));
    s->up = (float*)calloc((size_t)clients * ff, sizeof(float));
    s->act = (float*)calloc((size_t)clients * ff, sizeof(float));
    s->proj = (float*)calloc((size_t)clients * c->hidden, sizeof(float));
    s->combined = (float*)calloc((size_t)clients * c->hidden, sizeof(float));
    s->router = (float*)calloc((size_t)clients * (c->experts ? c->experts : 1), sizeof(float));
    s->probs = (float*)calloc((size_t)clients * (c->experts ? c->experts : 1), sizeof(float));
    s->margins = (float*)calloc((size_t)clients * c->layers, sizeof(float));
    for (size_t i = 0; i < (size_t)clients * c->layers; i++) s->margins[i] = 1.0f;
    return s;
}

void or_session_free(or_session* s) {
    if (!s) return;
    free(s->len); free(s->keys); free(s->values); free(s->states); free(s->normed); free(s->q);
    free(s->k); free(s->v); free(s->attn); free(s->gate); free(s->up); free(s->act); free(s->proj);
    free(s->combined); free(s->router); free(s->probs); free(s->margins);
    free(s);
}

int or_session_len(const or_session* s, int client) { return s->len[client]; }

int or_session_route_margins(const or_session* s, float* out) {
    const size_t count = (size_t)s->clients * s->m->cfg.layers;
    for (size_t i = 0; i < count; i++) out[i] = s->margins[i];
    return 0;
}

static int gemv_w(const or_w* w, uint64_t expert, const float* x, int n, float* y, int threads) {
    uint64_t bv, bb;
    or_type_layout(w->dtype, &bv, &bb);
    uint64_t mat = w->rows * (w->cols / bv) * bb;
    return or_gemv_fma(w->dtype, w->data + expert * mat, w->rows, w->cols, x, n, y, threads);
}

static void norm_rows(const or_model* m, const float* src, float* dst, const float* gain, int n) {
    const or_cfg* c = &m->cfg;
    if (c->family == OR_FAMILY_LLAMA) {
        /* spm-smol-ops/src/norm.rs:29-32 (pre_norm) */
        memcpy(dst, src, sizeof(float) * (size_t)n * c->hidden);
        or_scaled_rms_norm(dst, gain, c->eps, (int)c->hidden, n);
    } else {
        for (int i = 0; i < n; i++)
            or_rms_norm_slice(src + (size_t)i * c->hidden, gain, (int)c->hidden, c->eps,
                              dst + (size_t)i * c->hidden);
    }
}

/* Router, top-k, renormalised expert mixture: spm-granite-moe/src/moe.rs:17-35,
 * layout.rs:244-333 (experts in ascending id, up/gate/down FMA chains,
 * combined += down * p_e / sum(p_sel)).  The router bias is this build's
 * Zipf skew, added to each logit before the softmax. */
static void moe_half(or_session* s, const or_layer* L, int threads, int32_t* routes, float* margins) {
    or_model* m = s->m;
    const or_cfg* c = &m->cfg;
    int n = s->clients, E = (int)c->experts, K = (int)c->experts_used;
    size_t d = c->hidden, ff = c->expert_ff;
    gemv_w(&L->router, 0, s->normed, n, s->router, threads);
    int* sel = (int*)malloc(sizeof(int) * (size_t)n * K);
    float* selv = (float*)malloc(sizeof(float) * (size_t)n * K);
    float* normv = (float*)malloc(sizeof(float) * (size_t)n);
    for (int i = 0; i < n; i++) {
        float* logit = s->router + (size_t)i * E;
        if (L->router_bias)
            for (int e = 0; e < E; e++) logit[e] = logit[e] + L->router_bias[e];
        or_softmax_route(logit, E, s->probs + (size_t)i * E);
        or_top_k(s->probs + (size_t)i * E, E, K, sel + (size_t)i * K, selv + (size_t)i * K);
        {
            /* how close the selection came to another expert set: the K-th
             * probability against the largest one left out (a record only) */
            const float* pr = s->probs + (size_t)i * E;
            float best = -1.0f;
            for (int e = 0; e < E; e++) {
                int taken = 0;
                for (int j = 0; j < K; j++) taken |= sel[(size_t)i * K + j] == e;
                if (!taken && pr[e] > best) best = pr[e];
            }
            const float pk = selv[(size_t)i * K + K - 1];
            margins[i] = best < 0.0f ? 1.0f : (pk - best) / pk;
        }
        float sum = 0.0f;
        for (int j = 0; j < K; j++) sum = sum + s->probs[(size_t)i * E + sel[(size_t)i * K + j]];
        normv[i] = sum;
        if (routes)
            for (int j = 0; j < K; j++) routes[(size_t)i * K + j] = sel[(size_t)i * K + j];
    }
    memset(s->combined, 0, sizeof(float) * (size_t)n * d);
    /* The active experts run in parallel (one thread each, every GEMV chain
     * unchanged); the combine below then adds their outputs in ascending
     * expert id, as the reference's serial loop does. */
    int* active = (int*)malloc(sizeof(int) * (size_t)E);
    int* ntok = (int*)malloc(sizeof(int) * (size_t)E);
    int* toks = (int*)malloc(sizeof(int) * (size_t)E * n);
    int na = 0;
    for (int e = 0; e < E; e++) {
        int nt = 0;
        for (int i = 0; i < n; i++)
            for (int j = 0; j < K; j++)
                if (sel[(size_t)i * K + j] == e) { toks[(size_t)na * n + nt++] = i; break; }
        if (nt == 0) continue;
        ntok[na] = nt;
        active[na++] = e;
    }
    float* proj = (float*)malloc(sizeof(float) * (size_t)na * n * d + 1);
    int nth = nthreads(threads);
#pragma omp parallel num_threads(nth)
    {
        float* xs = (float*)malloc(sizeof(float) * (size_t)n * d);
        float* up = (float*)malloc(sizeof(float) * (size_t)n * ff);
        float* gate = (float*)malloc(sizeof(float) * (size_t)n * ff);
        float* act = (float*)malloc(sizeof(float) * (size_t)n * ff);
#pragma omp for schedule(dynamic, 1)
        for (int a = 0; a < na; a++) {
            const int e = active[a], nt = ntok[a];
            for (int t = 0; t < nt; t++)
                memcpy(xs + (size_t)t * d, s->normed + (size_t)toks[(size_t)a * n + t] * d, sizeof(float) * d);
            gemv_w(&L->up_exps, (uint64_t)e, xs, nt, up, 1);
            gemv_w(&L->gate_exps, (uint64_t)e, xs, nt, gate, 1);
            for (size_t i = 0; i < (size_t)nt * ff; i++) {
                float g = gate[i];
                act[i] = g / (1.0f + expf(-g)) * up[i];
            }
            gemv_w(&L->down_exps, (uint64_t)e, act, nt, proj + (size_t)a * n * d, 1);
        }
        free(xs); free(up); free(gate); free(act);
    }
    for (int a = 0; a < na; a++) {
        const int e = active[a];
        for (int t = 0; t < ntok[a]; t++) {
            int i = toks[(size_t)a * n + t];
            float pe = s->probs[(size_t)i * E + e];
            float* total = s->combined + (size_t)i * d;
            const float* lane = proj + ((size_t)a * n + t) * d;
            for (size_t col = 0; col < d; col++) total[col] = total[col] + lane[col] * pe / normv[i];
        }
    }
    free(active); free(ntok); free(proj);
    for (size_t i = 0; i < (size_t)n * d; i++) s->states[i] = s->states[i] + s->combined[i];
    free(sel); free(selv); free(normv); free(toks);
}

int or_decode_step(or_session* s, const uint32_t* tokens, float* logits, int threads, int32_t* routes) {
    or_model* m = s->m;
    const or_cfg* c = &m->cfg;
    int n = s->clients;
    size_t d = c->hidden, hd = c->head_dim;
    size_t qw = (size_t)c->heads * hd, kvw = (size_t)c->kv_heads * hd;
    uint64_t ebv, ebb;
    or_type_layout(m->embed.dtype, &ebv, &ebb);
    uint64_t erow = d / ebv * ebb;
    for (int i = 0; i < n; i++) {
        if (tokens[i] >= c->vocab) return -2;
        if (s->len[i] >= s->context) return -1;
    }
    /* spm-batch/src/step.rs:27-30: gather each client's embedding row. */
    for (int i = 0; i < n; i++)
        or_decode(m->embed.dtype, m->embed.data + (uint64_t)tokens[i] * erow, erow, s->states + (size_t)i * d);
    for (uint32_t l = 0; l < c->layers; l++) {
        const or_layer* L = &m->layers[l];
        /* attention half: spm-batch/src/inner.rs:16-34, 66-86 */
        norm_rows(m, s->states, s->normed, L->attn_norm, n);
        gemv_w(&L->q, 0, s->normed, n, s->q, threads);
        gemv_w(&L->k, 0, s->normed, n, s->k, threads);
        gemv_w(&L->v, 0, s->normed, n, s->v, threads);
        for (int i = 0; i < n; i++) {
            int at = s->len[i];
            float* q = s->q + (size_t)i * qw;
            float* k = s->k + (size_t)i * kvw;
            if (c->family == OR_FAMILY_LLAMA) {
                /* spm-kv/src/attend.rs:13-19 */
                for (uint32_t h = 0; h < c->heads; h++) or_rope_smol(q + h * hd, (int)hd, at, c->rope_base);
                for (uint32_t h = 0; h < c->kv_heads; h++) or_rope_smol(k + h * hd, (int)hd, at, c->rope_base);
            } else {
                if (c->family == OR_FAMILY_OLMOE) {
                    float* tmp = (float*)malloc(sizeof(float) * qw);
                    or_rms_norm_slice(q, L->q_norm, (int)qw, c->eps, tmp);
                    memcpy(q, tmp, sizeof(float) * qw);
                    or_rms_norm_slice(k, L->k_norm, (int)kvw, c->eps, tmp);
                    memcpy(k, tmp, sizeof(float) * kvw);
                    free(tmp);
                } else {
                    /* spm-qwen3-slice/src/attention.rs:27-34 (normalize_rope) */
                    float tmp[1024];
                    for (uint32_t h = 0; h < c->heads; h++) {
                        or_rms_norm_slice(q + h * hd, L->q_norm, (int)hd, c->eps, tmp);
                        memcpy(q + h * hd, tmp, sizeof(float) * hd);
                    }
                    for (uint32_t h = 0; h < c->kv_heads; h++) {
                        or_rms_norm_slice(k + h * hd, L->k_norm, (int)hd, c->eps, tmp);
                        memcpy(k + h * hd, tmp, sizeof(float) * hd);
                    }
                }
                for (uint32_t h = 0; h < c->heads; h++) or_rope_slice(q + h * hd, (int)hd, at, c->rope_base);
                for (uint32_t h = 0; h < c->kv_heads; h++) or_rope_slice(k + h * hd, (int)hd, at, c->rope_base);
            }
            /* spm-kv/src/cache.rs:49-58 (append at len) */
            size_t layer_base = (((size_t)i * c->layers + l) * s->context) * kvw;
            memcpy(s->keys + layer_base + (size_t)at * kvw, k, sizeof(float) * kvw);
            memcpy(s->values + layer_base + (size_t)at * kvw, s->v + (size_t)i * kvw, sizeof(float) * kvw);
            if (c->family == OR_FAMILY_LLAMA)
                or_attend_cached(q, s->keys + layer_base, s->values + layer_base, at + 1, (int)c->heads,
                                 (int)c->kv_heads, (int)hd, s->attn + (size_t)i * qw);
            else
                or_attend_slice(q, s->keys + layer_base, s->values + layer_base, at + 1, (int)c->heads,
                                (int)c->kv_heads, (int)hd, s->attn + (size_t)i * qw);
        }
        gemv_w(&L->o, 0, s->attn, n, s->proj, threads);
        for (size_t i = 0; i < (size_t)n * d; i++) s->states[i] = s->states[i] + s->proj[i];
        /* feed-forward half: spm-batch/src/inner.rs:40-58 */
        norm_rows(m, s->states, s->normed, L->ffn_norm, n);
        if (m->moe) {
            moe_half(s, L, threads, routes ? routes + (size_t)l * n * c->experts_used : NULL,
                     s->margins + (size_t)l * n);
        } else {
            size_t ff = c->intermediate;
            gemv_w(&L->gate, 0, s->normed, n, s->gate, threads);
            gemv_w(&L->up, 0, s->normed, n, s->up, threads);
            for (size_t i = 0; i < (size_t)n * ff; i++) s->act[i] = or_silu(s->gate[i]) * s->up[i];
            gemv_w(&L->down, 0, s->act, n, s->proj, threads);
            for (size_t i = 0; i < (size_t)n * d; i++) s->states[i] = s->states[i] + s->proj[i];
        }
    }
    /* spm-batch/src/step.rs:34-36 */
    for (int i = 0; i < n; i++) s->len[i] += 1;
    /* spm-batch/src/inner.rs:89-105 (finish): final norm, then plain dots. */
    if (c->family == OR_FAMILY_LLAMA) {
        or_scaled_rms_norm(s->states, m->output_norm, c->eps, (int)d, n);
        memcpy(s->normed, s->states, sizeof(float) * (size_t)n * d);
    } else {
        norm_rows(m, s->states, s->normed, m->output_norm, n);
    }
    if (logits)
        or_gemv_dot(m->head.dtype, m->head.data, c->vocab, d, s->normed, n, logits, threads);
    return 0;
}

/* spm-batch/examples/serve-demo.rs:45-91: lockstep ticks, prompt tokens fed
 * one per tick, generation starts when a client's prompt is exhausted. */
int or_serve(or_model* m, const uint32_t* prompts_flat, const int* prompt_lens, int clients,
             int steps, uint32_t* produced, int* produced_lens, float* last_logits, int threads,
             int max_ticks) {
    int longest = 0;
    for (int i = 0; i < clients; i++) longest = prompt_lens[i] > longest ? prompt_lens[i] : longest;
    int context = longest + steps + 1;
    int total = longest + steps - 1;
    if (max_ticks > 0 && max_ticks < total) total = max_ticks;
    or_session* s = or_session_new(m, clients, context);
    int* starts = (int*)calloc((size_t)clients, sizeof(int));
    for (int i = 1; i < clients; i++) starts[i] = starts[i - 1] + prompt_lens[i - 1];
    uint32_t* tokens = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)clients);
    float* logits = (float*)malloc(sizeof(float) * (size_t)clients * m->cfg.vocab);
    int cap = longest + steps - 1;
    for (int i = 0; i < clients; i++) {
        tokens[i] = prompts_flat[starts[i]];
        produced_lens[i] = 0;
    }
    int rc = 0;
    for (int tick = 0; tick < total; tick++) {
        rc = or_decode_step(s, tokens, logits, threads, NULL);
        if (rc) break;
        for (int i = 0; i < clients; i++) {
            uint32_t next = or_argmax_last(logits + (size_t)i * m->cfg.vocab, m->cfg.vocab);
            if (tick + 1 < prompt_lens[i]) {
                tokens[i] = prompts_flat[starts[i] + tick + 1];
            } else {
                produced[(size_t)i * cap + produced_lens[i]++] = next;
                tokens[i] = next;
            }
        }
    }
    if (last_logits) memcpy(last_logits, logits, sizeof(float) * (size_t)clients * m->cfg.vocab);
    free(starts); free(tokens); free(logits);
    or_session_free(s);
    return rc;
}

/* ------------------------------------------------------------------ */
/* .spm files and the ternary GEMV of spm-gemv-ref.                    */
/* ------------------------------------------------------------------ */

typedef struct {
    uint32_t rows, cols, group_size;
    uint8_t encoding;
} or_spm_desc;

static int spm_err(char* err, int errlen, int code, const char* msg) {
    if (err && errlen > 0) snprintf(err, (size_t)errlen, "%s", msg);
    return code;
}

static uint32_t rd_le32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* Encoding::bytes_for (spm-layout/src/model.rs): bytes a group of `count`
 * weights occupies on the wire. */
static uint64_t spm_bytes_for(uint8_t enc, uint64_t count) {
    switch (enc) {
        case 1: return (count + 3) / 4;              /* Ternary2F32I32 */
        case 2: return count * 4;                    /* F32            */
        case 3: return count * 2;                    /* Bf16           */
        case 4: return (count + 255) / 256 * 210;    /* Q6K            */
        case 5: return (count + 255) / 256 * 176;    /* Q5K            */
        default: return (count + 31) / 32 * 34;      /* Q8_0           */
    }
}

/* spm-header/src/parse.rs:12-59 then the directory loop of
 * spm-file/src/read.rs:51-60 with spm-layout/src/wire.rs:12-30. */
static int spm_parse(const uint8_t* src, uint64_t len, uint32_t* count, or_spm_desc** out, uint64_t* payload,
                     char* err, int errlen) {
    static const uint8_t magic[8] = {0x89, 'S', 'P', 'M', 0x0D, 0x0A, 0x1A, 0x0A};
    char msg[128];
    *out = NULL;
    if (len < 32) {
        snprintf(msg, sizeof msg, "header truncated: %llu bytes available, need 32", (unsigned long long)len);
        return spm_err(err, errlen, OR_SPM_TRUNCATED, msg);
    }
    if (memcmp(src, magic, 8) != 0)
        return spm_err(err, errlen, OR_SPM_MALFORMED, "bad magic: not a .spm file, or corrupted in transit");
    const uint16_t major = le16(src + 8);
    if (major > 1) {
        snprintf(msg, sizeof msg, "unsupported .spm major version %u: this build reads up to 1", major);
        return spm_err(err, errlen, OR_SPM_MALFORMED, msg);
    }
    if (src[12] != 0) {
        snprintf(msg, sizeof msg, "unknown endianness discriminant %u", src[12]);
        return spm_err(err, errlen, OR_SPM_MALFORMED, msg);
    }
    const uint32_t n = rd_le32(src + 16);
    /* only as many entries as the file can hold: a hostile count fails as a
     * truncated directory, not as a huge allocation */
    const uint64_t fit = (len - 32) / 32;
    const uint64_t room = n < fit ? n : fit;
    or_spm_desc* d = (or_spm_desc*)calloc(room ? room : 1, sizeof(or_spm_desc));
    if (!d) return spm_err(err, errlen, OR_SPM_TRUNCATED, "out of memory");
    uint64_t at = 32;
    for (uint32_t i = 0; i < n; ++i) {
        const uint64_t avail = at <= len ? len - at : 0;
        if (avail < 32) {
            free(d);
            snprintf(msg, sizeof msg, "descriptor truncated: %llu bytes, need 32", (unsigned long long)avail);
            return spm_err(err, errlen, OR_SPM_TRUNCATED, msg);
        }
        const uint8_t* p = src + at;
        d[i].group_size = rd_le32(p + 8);
        if (d[i].group_size == 0) {
            free(d);
            return spm_err(err, errlen, OR_SPM_MALFORMED, "group_size must be at least 1");
        }
        if (p[12] < 1 || p[12] > 6) {
            free(d);
            snprintf(msg, sizeof msg, "unknown .spm encoding profile %u", p[12]);
            return spm_err(err, errlen, OR_SPM_ENCODING, msg);
        }
        d[i].rows = rd_le32(p);
        d[i].cols = rd_le32(p + 4);
        d[i].encoding = p[12];
        at += 32;
    }
    *count = n;
    *out = d;
    *payload = at;
    return 0;
}

int or_spm_describe(const uint8_t* spm, uint64_t len, int32_t index, uint32_t* streams, uint32_t* rows,
                    uint32_t* cols, uint32_t* group_size, uint32_t* encoding, char* err, int errlen) {
    uint32_t n = 0;
    or_spm_desc* d = NULL;
    uint64_t payload = 0;
    int rc = spm_parse(spm, len, &n, &d, &payload, err, errlen);
    if (rc) return rc;
    if (streams) *streams = n;
    if (index >= 0 && (uint32_t)index < n) {
        if (rows) *rows = d[index].rows;
        if (cols) *cols = d[index].cols;
        if (group_size) *group_size = d[index].group_size;
        if (encoding) *encoding = d[index].encoding;
    }
    free(d);
    return 0;
}

/* Cursor (spm-walk/src/cursor.rs:20-58): a (stream, group) position that
 * skips streams with no groups left. */
typedef struct {
    uint32_t stream;
    uint64_t group;
} or_cursor;

static uint64_t spm_total(const or_spm_desc* d) { return (uint64_t)d->rows * d->cols; }

static void cursor_settle(or_cursor* c, const or_spm_desc* d, uint32_t n) {
    while (c->stream < n) {
        const uint64_t total = spm_total(&d[c->stream]);
        const uint64_t groups = (total + d[c->stream].group_size - 1) / d[c->stream].group_size;
        if (c->group < groups) return;
        c->stream++;
        c->group = 0;
    }
}

/* spm-layout/src/tiling.rs:37-51 group_len. */
static uint64_t cursor_group_len(const or_cursor* c, const or_spm_desc* d) {
    const uint64_t total = spm_total(&d[c->stream]);
    const uint64_t start = (uint64_t)d[c->stream].group_size * c->group;
    const uint64_t left = total - start;
    return left < d[c->stream].group_size ? left : d[c->stream].group_size;
}

int or_spm_run_gemv(const uint8_t* spm, uint64_t len, const float* x, int lanes, uint64_t x_cols,
                    float* bank, uint64_t bank_cap, char* err, int errlen) {
    uint32_t n = 0;
    or_spm_desc* d = NULL;
    uint64_t at = 0;
    char msg[128];
    int rc = spm_parse(spm, len, &n, &d, &at, err, errlen);
    if (rc) return rc;
    /* prepare (gemv.rs:66-85) */
    if (n == 0) {
        free(d);
        return spm_err(err, errlen, OR_SPM_NO_STREAMS, "parameter stream declares no operations");
    }
    const uint64_t rows = d[0].rows, cols = d[0].cols;
    if (x_cols < cols) {
        free(d);
        snprintf(msg, sizeof msg, "need %llu activations per lane, got %llu", (unsigned long long)cols,
                 (unsigned long long)x_cols);
        return spm_err(err, errlen, OR_SPM_ACTIVATIONS, msg);
    }
    if (lanes < 0 || rows * (uint64_t)lanes > bank_cap) {
        free(d);
        return spm_err(err, errlen, OR_SPM_ACTIVATIONS, "bank capacity too small");
    }
    memset(bank, 0, sizeof(float) * rows * (uint64_t)lanes);
    float* scaled = (float*)calloc(lanes > 0 ? (size_t)lanes : 1, sizeof(float));
    or_cursor cur = {0, 0};
    cursor_settle(&cur, d, n);
    uint64_t position = 0;
    /* drive (gemv.rs:88-104): pull groups until the first one of another stream */
    while (cur.stream < n) {
        const uint32_t stream = cur.stream;
        const uint64_t count = cursor_group_len(&cur, d);
        const uint64_t bytes = spm_bytes_for(d[stream].encoding, count);
        const uint64_t needed = 4 + bytes, available = len - at;
        if (available < needed) { /* spm-file/src/read.rs:91-101 */
            free(scaled);
            free(d);
            snprintf(msg, sizeof msg, "payload truncated: group needs %llu bytes, %llu remain",
                     (unsigned long long)needed, (unsigned long long)available);
            return spm_err(err, errlen, OR_SPM_TRUNCATED, msg);
        }
        float scale;
        memcpy(&scale, spm + at, 4); /* f32::from_le_bytes on a little-endian host */
        const uint8_t* packed = spm + at + 4;
        at += needed;
        cur.group++;
        cursor_settle(&cur, d, n);
        if (stream != 0) break;
        /* apply_group (datapath.rs:19-40): the scaled activations are
         * refreshed whenever the column changes, starting afresh in every
         * group; each weight then adds or subtracts them, never multiplies. */
        uint64_t current_col = UINT64_MAX;
        for (uint64_t local = 0; local < count; ++local) {
            const uint8_t code = (uint8_t)((packed[local / 4] >> ((local % 4) * 2)) & 3);
            const uint64_t index = position + local;
            const uint64_t col = index / rows;
            if (col != current_col) {
                for (int l = 0; l < lanes; ++l) scaled[l] = scale * x[(uint64_t)l * x_cols + col];
                current_col = col;
            }
            if (code & 1) { /* NONZERO_BIT: accumulator enable (datapath.rs:50-55) */
                float* slot = bank + (index % rows) * (uint64_t)lanes;
                if (code & 2) /* NEGATIVE_BIT: subtract (bank.rs:56-66) */
                    for (int l = 0; l < lanes; ++l) slot[l] -= scaled[l];
                else
                    for (int l = 0; l < lanes; ++l) slot[l] += scaled[l];
            }
        }
        position += count;
    }
    free(scaled);
    free(d);
    return 0;
}

/* spm_linear::resident / apply_weight (resident.rs:79-137): for every weight
 * in stream order, every position: out = fma(w, x, out). */
void or_resident(const float* w, uint32_t rows, uint32_t cols, const float* x, int positions, float* out) {
    memset(out, 0, sizeof(float) * (size_t)positions * rows);
    const uint64_t total = (uint64_t)rows * cols;
    for (uint64_t k = 0; k < total; ++k) {
        const uint64_t row = k % rows, col = k / rows;
        for (int p = 0; p < positions; ++p) {
            float* slot = out + (uint64_t)p * rows + row;
            *slot = fmaf(w[k], x[(uint64_t)p * cols + col], *slot);
        }
    }
}

static const char* spm_encoding_name(uint8_t enc) {
    switch (enc) { /* Debug names of spm_layout::Encoding */
        case 1: return "Ternary2F32I32";
        case 2: return "F32";
        case 3: return "Bf16";
        case 4: return "Q6K";
        case 5: return "Q5K";
        default: return "Q8_0";
    }
}

int or_spm_streamed(const uint8_t* spm, uint64_t len, int32_t index, uint32_t rows, uint32_t cols,
                    const float* x, uint64_t x_len, int positions, float* out, char* err, int errlen) {
    uint32_t n = 0;
    or_spm_desc* d = NULL;
    uint64_t at = 0;
    char msg[160];
    int rc = spm_parse(spm, len, &n, &d, &at, err, errlen);
    if (rc) return rc;
    /* check (stream.rs:63-76): before any group is pulled */
    const uint64_t need = (uint64_t)positions * cols;
    if (x_len < need) {
        free(d);
        snprintf(msg, sizeof msg, "need %llu activations, got %llu", (unsigned long long)need,
                 (unsigned long long)x_len);
        return spm_err(err, errlen, OR_SPM_ACTIVATIONS, msg);
    }
    const uint64_t total = (uint64_t)rows * cols;
    memset(out, 0, sizeof(float) * (size_t)positions * rows);
    or_cursor cur = {0, 0};
    cursor_settle(&cur, d, n);
    /* the streams before `index` are read past group by group */
    while (cur.stream < n && cur.stream < (uint32_t)index) {
        const uint64_t count = cursor_group_len(&cur, d);
        const uint64_t needed = 4 + spm_bytes_for(d[cur.stream].encoding, count), available = len - at;
        if (available < needed) {
            free(d);
            snprintf(msg, sizeof msg, "payload truncated: group needs %llu bytes, %llu remain",
                     (unsigned long long)needed, (unsigned long long)available);
            return spm_err(err, errlen, OR_SPM_TRUNCATED, msg);
        }
        at += needed;
        cur.group++;
        cursor_settle(&cur, d, n);
    }
    float* buf = NULL;
    uint64_t done = 0;
    while (done < total) { /* streamed (stream.rs:31-55) */
        if (cur.stream >= n) {
            free(buf);
            free(d);
            snprintf(msg, sizeof msg, "stream ended after %llu of %llu weights", (unsigned long long)done,
                     (unsigned long long)total);
            return spm_err(err, errlen, OR_SPM_STREAMED_TRUNCATED, msg);
        }
        const uint8_t enc = d[cur.stream].encoding;
        const uint64_t count = cursor_group_len(&cur, d);
        const uint64_t needed = 4 + spm_bytes_for(enc, count), available = len - at;
        if (available < needed) {
            free(buf);
            free(d);
            snprintf(msg, sizeof msg, "payload truncated: group needs %llu bytes, %llu remain",
                     (unsigned long long)needed, (unsigned long long)available);
            return spm_err(err, errlen, OR_SPM_TRUNCATED, msg);
        }
        const uint8_t* p = spm + at + 4;
        at += needed;
        cur.group++;
        cursor_settle(&cur, d, n);
        if (enc != 2 && enc != 3) { /* spm-codec-any/src/decode.rs:36-45 */
            free(buf);
            free(d);
            snprintf(msg, sizeof msg, "parameter stream: %s needs a scale-aware engine", spm_encoding_name(enc));
            return spm_err(err, errlen, OR_SPM_UNSUPPORTED, msg);
        }
        float* nb = (float*)realloc(buf, sizeof(float) * (count ? count : 1));
        if (!nb) {
            free(buf);
            free(d);
            return spm_err(err, errlen, OR_SPM_TRUNCATED, "out of memory");
        }
        buf = nb;
        for (uint64_t i = 0; i < count; ++i) {
            if (enc == 2) {
                memcpy(&buf[i], p + 4 * i, 4);
            } else { /* widen: the bf16 bits become the high half of an f32 */
                const uint32_t bits = ((uint32_t)p[2 * i] | ((uint32_t)p[2 * i + 1] << 8)) << 16;
                memcpy(&buf[i], &bits, 4);
            }
        }
        /* apply (stream.rs:107-125): every weight, every position */
        for (uint64_t i = 0; i < count; ++i) {
            const uint64_t k = done + i;
            if (k >= total) break; /* a group that runs past the matrix: its tail is not applied */
            const uint64_t row = k % rows, col = k / rows;
            for (int q = 0; q < positions; ++q) {
                float* slot = out + (uint64_t)q * rows + row;
                *slot = fmaf(buf[i], x[(uint64_t)q * cols + col], *slot);
            }
        }
        done += count;
    }
    free(buf);
    free(d);
    return 0;
}

int or_spm_qblocks(const uint8_t* spm, uint64_t len, int32_t index, const float* x, uint64_t x_len,
                   int positions, float* out, char* err, int errlen) {
    uint32_t n = 0;
    or_spm_desc* d = NULL;
    uint64_t at = 0;
    char msg[160];
    int rc = spm_parse(spm, len, &n, &d, &at, err, errlen);
    if (rc) return rc;
    if (index < 0 || (uint32_t)index >= n) {
        free(d);
        return spm_err(err, errlen, OR_SPM_NO_STREAMS, "stream index out of range");
    }
    const uint8_t enc = d[index].encoding;
    uint32_t type, bv;
    if (enc == 6) type = OR_Q8_0, bv = 32;
    else if (enc == 4) type = OR_Q6_K, bv = 256;
    else if (enc == 5) type = OR_Q5_K, bv = 256;
    else {
        free(d);
        snprintf(msg, sizeof msg, "stream is %s, not a block profile (Q8_0, Q6K or Q5K)", spm_encoding_name(enc));
        return spm_err(err, errlen, OR_SPM_UNSUPPORTED, msg);
    }
    const uint64_t rows = d[index].rows, cols = d[index].cols, total = rows * cols;
    if (x_len < (uint64_t)positions * cols) {
        free(d);
        snprintf(msg, sizeof msg, "need %llu activations, got %llu", (unsigned long long)((uint64_t)positions * cols),
                 (unsigned long long)x_len);
        return spm_err(err, errlen, OR_SPM_ACTIVATIONS, msg);
    }
    memset(out, 0, sizeof(float) * (size_t)positions * rows);
    or_cursor cur = {0, 0};
    cursor_settle(&cur, d, n);
    float block[256];
    uint64_t k = 0;
    while (cur.stream < n && cur.stream <= (uint32_t)index) {
        const uint32_t stream = cur.stream;
        const uint64_t count = cursor_group_len(&cur, d);
        const uint64_t needed = 4 + spm_bytes_for(d[stream].encoding, count), available = len - at;
        if (available < needed) {
            free(d);
            snprintf(msg, sizeof msg, "payload truncated: group needs %llu bytes, %llu remain",
                     (unsigned long long)needed, (unsigned long long)available);
            return spm_err(err, errlen, OR_SPM_TRUNCATED, msg);
        }
        const uint8_t* p = spm + at + 4;
        at += needed;
        cur.group++;
        cursor_settle(&cur, d, n);
        if (stream != (uint32_t)index) continue;
        if (count != bv) { /* layout.rs:225-227, gemma_smoke.rs:219-221 */
            free(d);
            snprintf(msg, sizeof msg, "unexpected packed group: %s streams hold one %u-value block per group",
                     spm_encoding_name(enc), bv);
            return spm_err(err, errlen, OR_SPM_UNSUPPORTED, msg);
        }
        or_decode(type, p, needed - 4, block);
        for (uint32_t i = 0; i < bv; ++i, ++k) {
            const uint64_t row = k / cols, col = k % cols;
            for (int q = 0; q < positions; ++q) {
                float* slot = out + (uint64_t)q * rows + row;
                *slot = fmaf(block[i], x[(uint64_t)q * cols + col], *slot);
            }
        }
    }
    free(d);
    (void)total;
    return 0;
}
