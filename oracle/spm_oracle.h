/*
 * spm_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of emufpga's CPU token loop (the reference is Rust
 * and cannot be built in this image: no cargo/rustc).  It is the checker the
 * parity tests compare the CUDA path against, and the timed CPU baseline in
 * bench.py.  Nothing in the product library links, loads or calls it.
 *
 * Every function names the reference file:line it follows (paths relative to
 * the emufpga tree).  Compiled with -ffp-contract=off so that every `a*b+c`
 * written here rounds twice, exactly like Rust, which never contracts; the
 * Rust `mul_add` calls are spelled fmaf() here.
 *
 * Pinning: the block decoders are checked against the reference's own
 * known-answer tests (spm-gguf/tests/decode.rs) and bit-for-bit against the
 * gguf-py 0.19.0 dequantizers on committed fixtures (tests/golden/).  Q2_K has
 * no decoder in the reference; it follows ggml's published block format and is
 * pinned only against gguf-py.  The .spm restatements (run_gemv, streamed,
 * resident, q6_operation / stream_matrix) are pinned against the reference's
 * own tests read from their sources: the tiny.spm layout and the header,
 * descriptor and payload refusals (spm-file, spm-header, spm-layout tests),
 * the gemv-ref correctness and batch cases, and spm-linear's agreement cases.
 */
#ifndef SPM_ORACLE_H
#define SPM_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML dtype codes (spm-gguf/src/parse.rs:26-45). */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q8_0 = 8, OR_Q2_K = 10, OR_Q5_K = 13, OR_Q6_K = 14 };

/* Model families: which equations a layer uses. */
enum {
    OR_FAMILY_LLAMA = 1,    /* spm-smol / spm-batch / spm-kv equations (SmolLM2) */
    OR_FAMILY_QWEN3 = 2,    /* spm-qwen3-slice equations, per-head QK-norm       */
    OR_FAMILY_OLMOE = 3,    /* qwen3-slice equations, full-width QK-norm, MoE FFN */
    OR_FAMILY_QWEN3MOE = 4  /* qwen3-slice equations, per-head QK-norm, MoE FFN   */
};

typedef struct or_cfg {
    uint32_t family;
    uint32_t layers, hidden, intermediate, heads, kv_heads, head_dim, vocab;
    uint32_t experts, experts_used, expert_ff;
    uint32_t tied;          /* 1: logits use token_embd (SmolLM2)            */
    float rope_base, eps;   /* eps also serves the QK-norm                   */
} or_cfg;

/* ---- decoders (spm-gguf/src/tensor.rs) ---- */
float or_f16_to_f32(uint16_t bits);
/* 0 ok; -1 nbytes is not whole blocks; -2 unknown type. out gets nbytes/bb*bs values. */
int or_decode(uint32_t ggml_type, const uint8_t* bytes, uint64_t nbytes, float* out);
int or_type_layout(uint32_t ggml_type, uint64_t* block_values, uint64_t* block_bytes);

/* ---- GGUF (spm-gguf/src/parse.rs) over an in-memory image ---- */
typedef struct or_gguf or_gguf;
int or_gguf_parse(const uint8_t* buf, uint64_t len, or_gguf** out, char* err, int errlen);
/* returns 0 and fills the outputs, or -1 when no tensor has that name */
int or_gguf_find(const or_gguf* g, const char* name, uint32_t* dtype, uint64_t* dims4,
                 uint32_t* ndims, uint64_t* offset, uint64_t* nbytes);
uint64_t or_gguf_tensor_count(const or_gguf* g);
void or_gguf_free(or_gguf* g);

/* ---- engine pieces ---- */
/* y[p][r] = fma chain over c ascending (spm-linear/src/resident.rs:124-137,
 * spm-granite-moe/src/layout.rs:208-242). `blocks` are row-major GGML blocks
 * (or row-major f32 for OR_F32). threads<=0 means all cores. */
int or_gemv_fma(uint32_t ggml_type, const uint8_t* blocks, uint64_t rows, uint64_t cols,
                const float* x, int positions, float* y, int threads);
/* logits-style plain multiply + sequential sum (spm-batch/src/inner.rs:89-105, finish). */
int or_gemv_dot(uint32_t ggml_type, const uint8_t* blocks, uint64_t rows, uint64_t cols,
                const float* x, int positions, float* y, int threads);

void or_scaled_rms_norm(float* values, const float* weight, float eps, int width, int rows);
void or_rms_norm_slice(const float* input, const float* weight, int n, float eps, float* out);
void or_rope_smol(float* head, int dim, int position, float base);
void or_rope_slice(float* head, int dim, int position, float base);
float or_silu(float x);
void or_attend_cached(const float* query, const float* keys, const float* values, int positions,
                      int heads, int kv_heads, int head_dim, float* out);
void or_attend_slice(const float* query, const float* keys, const float* values, int positions,
                     int heads, int kv_heads, int head_dim, float* out);
void or_softmax_route(const float* values, int n, float* out);
void or_top_k(const float* values, int n, int k, int* ids, float* vals);
uint32_t or_argmax_last(const float* row, uint64_t n);

/* ---- model / token loop (spm-batch/src/step.rs:19-53) ---- */
typedef struct or_model or_model;
typedef struct or_session or_session;
or_model* or_model_new(const uint8_t* gguf, uint64_t len, const or_cfg* cfg, char* err, int errlen);
void or_model_free(or_model* m);
or_session* or_session_new(or_model* m, int clients, int context);
void or_session_free(or_session* s);
/* One decode step for every client; logits is clients x vocab. Returns 0 ok,
 * -1 context exhausted, -2 bad token.  Routes (if non-NULL) receive, per MoE
 * layer and client, the selected expert ids (layers x clients x used). */
int or_decode_step(or_session* s, const uint32_t* tokens, float* logits, int threads, int32_t* routes);
int or_session_len(const or_session* s, int client);
/* After a step: each routed layer's margin per client, layers x clients,
 * (p_K - p_K+1) / p_K of the routing probabilities (the K-th selected and
 * the largest left out; 1 where every expert is selected and for dense
 * layers).  A record for the parity tests: how close the routing came to
 * another expert set. */
int or_session_route_margins(const or_session* s, float* out);

/* The lockstep serving loop of spm-batch/examples/serve-demo.rs:59-91.
 * prompts_flat holds each prompt back to back. produced must have room for
 * clients x (longest+steps-1) tokens; produced_lens receives each count. */
int or_serve(or_model* m, const uint32_t* prompts_flat, const int* prompt_lens, int clients,
             int steps, uint32_t* produced, int* produced_lens, float* last_logits, int threads,
             int max_ticks);

/* ---- .spm files and the ternary profile ----
 * spm-header/src/parse.rs (32-byte header), spm-layout/src/wire.rs:12-30 and
 * model.rs (32-byte descriptors, Encoding::bytes_for), spm-walk/src/cursor.rs
 * (group order), spm-file/src/read.rs:69-101 (scale, then payload) and
 * spm-gemv-ref/src/{gemv.rs:39-126, datapath.rs:19-55} with
 * spm-accum/src/bank.rs:56-66 (run_gemv).  Status codes: */
enum {
    OR_SPM_NO_STREAMS = -1,   /* GemvError::NoStreams                        */
    OR_SPM_ACTIVATIONS = -2,  /* GemvError::MissingActivations               */
    OR_SPM_TRUNCATED = -3,    /* HeaderError/LayoutError::TooShort, PayloadTruncated */
    OR_SPM_MALFORMED = -4,    /* BadMagic, UnsupportedVersion, UnknownEndianness, ZeroGroupSize */
    OR_SPM_ENCODING = -5      /* LayoutError::UnknownEncoding                */
};
/* Header and directory: stream count, and rows/cols/group/encoding of stream
 * `index` (any of them may be NULL). */
int or_spm_describe(const uint8_t* spm, uint64_t len, int32_t index, uint32_t* streams, uint32_t* rows,
                    uint32_t* cols, uint32_t* group_size, uint32_t* encoding, char* err, int errlen);
/* spm_gemv_ref::run_gemv over the first stream with `lanes` activation vectors
 * (lane-major, x_cols floats each).  bank receives rows x lanes floats in the
 * reference's row-major AccumulatorBank order; bank_cap is its capacity in
 * floats.  Like the reference, the scan reads the first group after the stream
 * before it stops, so a truncated one is an error too. */
int or_spm_run_gemv(const uint8_t* spm, uint64_t len, const float* x, int lanes, uint64_t x_cols,
                    float* bank, uint64_t bank_cap, char* err, int errlen);

/* spm_linear::streamed (spm-linear/src/stream.rs:31-125) for the stream
 * `index` of a .spm file: skip the groups of the streams before it, then pull
 * groups until rows x cols weights, decoding F32 (spm-codec-dense) or Bf16
 * (spm-codec-bf16/src/convert.rs widen) and applying each weight to every
 * position as out = fma(w, x, out) (resident.rs:124-137).  x holds x_len
 * floats (positions x cols); out positions x rows.  Extra status codes: */
enum {
    OR_SPM_STREAMED_TRUNCATED = -6,  /* LinearError::Truncated: stream ended early     */
    OR_SPM_UNSUPPORTED = -7          /* DecodeError::Unsupported -> LinearError::Stream */
};
int or_spm_streamed(const uint8_t* spm, uint64_t len, int32_t index, uint32_t rows, uint32_t cols,
                    const float* x, uint64_t x_len, int positions, float* out, char* err, int errlen);
/* q6_operation (spm-granite-moe/src/layout.rs:208-242) and stream_matrix
 * (gemma_smoke.rs:201-236) for the block stream `index` (Q8_0, Q6K or Q5K,
 * one block per group): decode each group's block (or_decode), then apply
 * value k = W[k / cols][k % cols] to every input as out = fma(w, x, out).
 * A group that is not one whole block of the stream's profile is
 * OR_SPM_UNSUPPORTED ("unexpected packed group"). */
int or_spm_qblocks(const uint8_t* spm, uint64_t len, int32_t index, const float* x, uint64_t x_len,
                   int positions, float* out, char* err, int errlen);
/* spm_linear::resident (resident.rs:79-96): the same product with the weights
 * given in stream order (w[k] = W[k % rows][k / rows]). */
void or_resident(const float* w, uint32_t rows, uint32_t cols, const float* x, int positions, float* out);

#ifdef __cplusplus
}
#endif
#endif
