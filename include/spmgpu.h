/*
 * spmgpu.h -- C ABI of libspmgpu.so, the sm_100a backend for emufpga's
 * decode token loop (the streamed low-bit weight pass shared by N clients).
 *
 * Every entry point returns an spm_status (0 = ok, negative = error; the
 * message is available from spm_last_error() on the calling thread).  All
 * pointers are plain host or device pointers; no framework types cross the
 * boundary.  Handles are opaque; there is no global model state.
 *
 * Reference interfaces replaced (paths inside the emufpga tree):
 *   spm_gguf_*            spm-gguf/src/parse.rs:153-182 (read), tensor.rs:21-67
 *   spm_decode_blocks     spm-gguf/src/tensor.rs:69-210 (decode_f32/q8_0/q5_k/q6_k)
 *   spm_order_check       spm-order/src/order.rs:28-111 (parse_order, reorder)
 *   spm_model_open*       spm-stream-groups/src/groups.rs:54-117 (GroupStream::open)
 *                         + spm-smol/src/config.rs (SmolConfig) + the .order layout
 *   spm_model_weight_bytes spm-batch/src/session.rs:83-121 (StepReport::for_sweep)
 *   spm_session_create    spm-batch/src/session.rs:25-34, :64-78 (Client::new, Scratch::new)
 *   spm_decode_step       spm-batch/src/step.rs:19-40 (decode_step) + the greedy pick
 *                         of spm-batch/examples/serve-demo.rs:72-90
 *   spm_prefill           spm-batch/examples/serve-demo.rs:84-89 (prompt tokens fed one
 *                         per tick) run as one pass, as spm-qwen3-slice/src/model.rs:10-171
 *   spm_streamed          spm-linear/src/stream.rs:31-55 (streamed) for one stream
 *   spm_dequant_rows      parity hook for the decoders above, run on the device
 *   spm_file_*            spm-file/src/read.rs:46-101 (SpmReader) over .spm files
 *   spm_dense_*           spm-linear/src/stream.rs:31-125 (streamed) on dense .spm streams
 *   spm_qblocks_*         spm-granite-moe/src/layout.rs:208-242 (q6_operation),
 *                         gemma_smoke.rs:201-236 (stream_matrix) on block-profile streams
 *   spm_ternary_*         spm-gemv-ref/src/gemv.rs:39-126 (run_gemv)
 *   spm_sweep_*           spm-stream-file/src/prefetch.rs + spm-stream-groups rewind:
 *                         .spm files streamed from host memory through a device ring
 */
#ifndef SPMGPU_H
#define SPMGPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t spm_status;
enum {
    SPM_OK = 0,
    SPM_E_ARG = -1,            /* bad argument / shape (LinearError::WeightCount)  */
    SPM_E_ACTIVATION_LEN = -2, /* LinearError::ActivationLen                      */
    SPM_E_TRUNCATED = -3,      /* LinearError::Truncated / StreamError::Truncated */
    SPM_E_STREAM = -4,         /* LinearError::Stream (I/O, parse, layout)        */
    SPM_E_ENCODING = -5,       /* LayoutError::UnknownEncoding / unsupported dtype */
    SPM_E_CUDA = -6,
    SPM_E_NCCL = -7,
    SPM_E_TIMEOUT = -8,        /* a bounded device wait gave up                   */
    SPM_E_CONTEXT = -9,        /* KvCache::append: context exhausted              */
    SPM_E_NO_DEVICE = -10
};

/* GGML dtype codes (spm-gguf/src/parse.rs:26-45). */
enum { SPM_F32 = 0, SPM_F16 = 1, SPM_Q8_0 = 8, SPM_Q2_K = 10, SPM_Q5_K = 13, SPM_Q6_K = 14 };

/* Which layer equations a model uses. */
enum {
    SPM_FAMILY_LLAMA = 1,    /* SmolLM2: spm-smol / spm-batch / spm-kv equations     */
    SPM_FAMILY_QWEN3 = 2,    /* Qwen3 dense: spm-qwen3-slice equations, head QK-norm */
    SPM_FAMILY_OLMOE = 3,    /* OLMoE: full-width QK-norm, softmax top-k experts     */
    SPM_FAMILY_QWEN3MOE = 4  /* Qwen3-MoE: head QK-norm, softmax top-k experts       */
};

/* Model shape.  Field order and meaning match the oracle's or_cfg. */
typedef struct spm_model_cfg {
    uint32_t family;
    uint32_t layers, hidden, intermediate, heads, kv_heads, head_dim, vocab;
    uint32_t experts, experts_used, expert_ff;
    uint32_t tied;            /* logits reuse token_embd (SmolLM2)   */
    float rope_base, eps;
} spm_model_cfg;

/* Synthetic GGUF recipe: seeded N(0, sigma) weights quantised by this
 * library's encoders; norm gains 1; optional Zipf router bias. */
typedef struct spm_synth_spec {
    spm_model_cfg cfg;
    uint32_t layer_type;      /* dtype of attention / dense FFN matrices */
    uint32_t expert_type;     /* dtype of expert matrices (MoE)          */
    uint32_t embed_type;      /* dtype of token_embd                     */
    uint32_t head_type;       /* dtype of output.weight (untied)         */
    uint64_t seed;
    float sigma;              /* 0.02 in every benchmark configuration */
    float zipf_s;             /* 0 = no router bias                      */
    float gain_sigma;         /* 0: norm gains are 1 (the benchmark setting); else 1+N(0,gain_sigma) */
    int32_t threads;          /* <=0: all cores                          */
} spm_synth_spec;

typedef struct spm_model spm_model;
typedef struct spm_session spm_session;
typedef struct spm_weights spm_weights;

const char* spm_last_error(void);
const char* spm_version(void);

/* ---- host-side format pieces ---- */
/* Write a synthetic model as a GGUF v3 image into a malloc'd buffer
 * (release with spm_free).  Deterministic in spec (threads do not matter). */
spm_status spm_synth_gguf(const spm_synth_spec* spec, uint8_t** out, uint64_t* len);
void spm_free(void* p);
/* Bounded GGUF parse (spm-gguf limits); reports tensor count and data offset. */
spm_status spm_gguf_probe(const uint8_t* buf, uint64_t len, uint64_t* tensors, uint64_t* data_offset);
spm_status spm_gguf_probe_file(const char* path, uint64_t* tensors, uint64_t* data_offset);
/* Tensor lookup by name: dtype, up to 4 dims, absolute offset and byte length. */
spm_status spm_gguf_find(const uint8_t* buf, uint64_t len, const char* name, uint32_t* dtype,
                         uint64_t* dims4, uint64_t* offset, uint64_t* nbytes);
/* Host decode of whole GGML blocks (CPU, for loaders and tests). */
spm_status spm_decode_blocks(uint32_t dtype, const uint8_t* bytes, uint64_t nbytes, float* out);
/* Validate an .order text against a model's tensor names (both directions). */
spm_status spm_order_check(const char* order_text, const uint8_t* gguf, uint64_t len);
/* Default consumption order for a model shape as .order text (malloc'd).
 * When gguf is given, optional tensors it holds (router biases) are listed. */
spm_status spm_order_default(const spm_model_cfg* cfg, const uint8_t* gguf, uint64_t len, char** text);

/* ---- device model: the weight stream laid out in HBM in consumption order ---- */
spm_status spm_model_open(const char* gguf_path, const char* order_path,
                          const spm_model_cfg* cfg, int device, spm_model** out);
spm_status spm_model_open_memory(const uint8_t* gguf, uint64_t len, const char* order_text,
                                 const spm_model_cfg* cfg, int device, spm_model** out);
/* Packed device image files (the reference lays a model out once, in
 * consumption order, in .spm/.order files, spm-file/src and
 * spm-order/src/order.rs:28-52; here the file holds the packed HBM image
 * itself): spm_pack_image packs a GGUF model on the host (no GPU) into a .spm
 * container -- the .spm header and one descriptor per stream, with encoding
 * 0x80 + GGML type for this library's tiled layout of that block type (group
 * size = values per block, lane count = rows per tile), then the stream table,
 * the norm gains and every matrix's tiles in consumption order.  A stock .spm
 * reader refuses those encodings; spm_model_open_image uploads the file with
 * one sequential read, without re-packing; spm_image_probe validates a file
 * (every descriptor must match its stream) and reports its image bytes and
 * stream count. */
spm_status spm_pack_image(const uint8_t* gguf, uint64_t len, const char* order_text,
                          const spm_model_cfg* cfg, const char* path);
spm_status spm_image_probe(const char* path, uint64_t* image_bytes, int32_t* streams);
spm_status spm_model_open_image(const char* path, int device, spm_model** out);
spm_status spm_model_close(spm_model* m);
/* Weight bytes one decode sweep reads (descriptor sizes, LM head included). */
spm_status spm_model_weight_bytes(const spm_model* m, uint64_t* bytes);
spm_status spm_model_stream_count(const spm_model* m, int32_t* streams);
/* rows, cols, dtype and quantized byte size of stream `index` (consumption order). */
spm_status spm_model_stream_info(const spm_model* m, int32_t index, uint64_t* rows,
                                 uint64_t* cols, uint32_t* dtype, uint64_t* bytes);
spm_status spm_model_stream_index(const spm_model* m, const char* tensor_name, int32_t* index);
/* Dequantize rows [row0, row0+rows) of stream `index` on the device into host
 * memory (rows x cols floats).  Bit-exact with spm_decode_blocks. */
spm_status spm_dequant_rows(const spm_model* m, int32_t index, uint64_t row0, uint64_t rows,
                            float* out_host);
/* spm_dequant_rows without any device allocation; no counterpart in the
 * reference.  For callers that cannot allocate device memory: a parity or
 * monitoring hook beside a session that holds the rest of HBM, or one that must
 * not add the device-wide synchronisation of cudaMalloc/cudaFree to a device
 * that is decoding.  Decodes into one static 4 MiB buffer per device, part of
 * the library's device image and held until exit: rows x cols must not exceed
 * 1048576 floats (SPM_E_ARG otherwise).  Calls that overlap on the GPU share
 * the buffer and race, so serialise them.  Each call looks the buffer's
 * address up in the current context, so it stays valid across a context
 * reset.  The first call on a device loads the library's device code there;
 * make it before any stream capture on that device. */
spm_status spm_dequant_rows_static(const spm_model* m, int32_t index, uint64_t row0, uint64_t rows,
                                   float* out_host);
/* y[p][r] = sum_c W[r][c] * x[p][c] for one stream; x_dev is positions x cols,
 * y_dev positions x rows (device pointers); cuda_stream may be NULL.  Up to 15
 * positions stream the weights through GEMVs of at most eight positions; 16 or
 * more (a prompt's positions) run as one product on the tensor cores when cols
 * is a multiple of 64 and x_dev 16-byte aligned.  spm_weights_gemv likewise. */
spm_status spm_streamed(const spm_model* m, int32_t index, const float* x_dev, int32_t positions,
                        float* y_dev, void* cuda_stream);

/* ---- standalone operator: one quantized matrix, no model ---- */
spm_status spm_weights_upload(uint32_t dtype, uint64_t rows, uint64_t cols,
                              const uint8_t* gguf_blocks_host, int device, spm_weights** out);
spm_status spm_weights_free(spm_weights* w);
spm_status spm_weights_gemv(const spm_weights* w, const float* x_dev, int32_t positions,
                            float* y_dev, void* cuda_stream);
spm_status spm_weights_dequant(const spm_weights* w, uint64_t row0, uint64_t rows, float* out_host);

/* ---- sessions: N clients, one weight sweep per step ---- */
spm_status spm_session_create(spm_model* m, int32_t max_clients, int32_t max_context,
                              spm_session** out);
spm_status spm_session_destroy(spm_session* s);
/* Empty client `client`'s KV cache (position 0). */
spm_status spm_client_reset(spm_session* s, int32_t client);
spm_status spm_client_len(const spm_session* s, int32_t client, int32_t* len);
/* One decode step for clients 0..n-1: tokens (host) in, greedy argmax (host,
 * last index on ties) out; logits (host, n x vocab) optional. */
spm_status spm_decode_step(spm_session* s, const uint32_t* tokens, int32_t n, float* logits_host,
                           uint32_t* argmax_host);
/* Same step on device buffers (no host copies): tokens_dev n uint32,
 * argmax_dev n uint32, logits_dev n x vocab (may be NULL). Enqueued on the
 * session stream; use spm_session_sync to wait. */
spm_status spm_decode_step_device(spm_session* s, const uint32_t* tokens_dev, int32_t n,
                                  float* logits_dev, uint32_t* argmax_dev);
spm_status spm_session_sync(spm_session* s);
/* Run a prompt through the model for `client`: its next `len` positions take
 * tokens[0..len), their keys and values are appended to the client's cache,
 * and the client's length grows by `len`.  The layers' products over all the
 * prompt's positions run on the tensor cores (tcgen05, weights decoded exactly
 * and split into bf16 parts, fp32 accumulation); each position computes what
 * a decode step computes for it, up to the rounding of sums.  No logits are
 * produced: feed the prompt's last token through spm_decode_step for the
 * first greedy pick.  Single-GPU models; prompts longer than 1024 tokens run
 * in chunks of 1024.  The reference feeds prompts one token per decode tick
 * (spm-batch/examples/serve-demo.rs:84-89); its Qwen3 slice runs a whole
 * prompt in one forward pass (spm-qwen3-slice/src/model.rs:10-171). */
spm_status spm_prefill(spm_session* s, int32_t client, const uint32_t* tokens, int32_t len);
/* The session's CUDA stream (cudaStream_t as void*). */
spm_status spm_session_stream(const spm_session* s, void** cuda_stream);
/* Capture steps as a CUDA graph per client count (1) or launch eagerly (0). */
spm_status spm_session_set_graphs(spm_session* s, int32_t enable);
/* Routes of the last step (MoE): layers x n x experts_used expert ids. */
spm_status spm_session_routes(const spm_session* s, int32_t n, int32_t* routes_host);
/* Margins of the last step's routing (MoE), layers x n floats: for each
 * client and routed layer (p_K - p_K+1) / p_K, p_K the smallest selected
 * routing probability and p_K+1 the largest left out (1 when every expert is
 * selected).  A margin near zero marks a near tie between two experts, which
 * the order of fp32 sums can decide either way (spm-granite-moe/src/moe.rs:
 * 17-35 selects by the same order, ties to the lower id). */
spm_status spm_session_route_gaps(const spm_session* s, int32_t n, float* gaps_host);
/* ---- expert parallel (routed models over 1..8 GPUs of one node) ----
 * Replaces the reference's single-process expert loop
 * (spm-granite-moe/src/layout.rs:244-304) across GPUs, with data-parallel
 * attention.  The client count n of a step must be a multiple of world;
 * rank r owns clients r*n/world .. (r+1)*n/world - 1 and their KV cache.
 * Per layer each rank runs the attention block of its own clients and the O
 * projection stores their rows (and norm partials) over NVLink into every
 * rank's states; the router waits (bounded) until every rank's rows are in,
 * so every rank routes every client; each rank computes only the experts e
 * with e % world == rank, writes their output rows into every rank's
 * exchange buffer, and the combine waits (bounded) for all ranks' rows and
 * adds them, in ascending expert id, into its own clients' states.  Each
 * rank runs the LM head for its own clients (their logits alone are
 * written) and the greedy picks are gathered, so every rank returns all n.
 * Open the model with spm_model_open_ep (only this rank's experts are
 * uploaded; the file is memory-mapped, so ranks share its pages), create
 * the session, exchange the 64-byte handles of spm_session_ep_handle between
 * the ranks (rank order), and pass them all to spm_session_ep_connect before
 * the first step. */
spm_status spm_model_open_ep(const char* gguf_path, const char* order_path, const spm_model_cfg* cfg, int device,
                             int32_t world, int32_t rank, spm_model** out);
spm_status spm_model_open_memory_ep(const uint8_t* gguf, uint64_t len, const char* order_text,
                                    const spm_model_cfg* cfg, int device, int32_t world, int32_t rank,
                                    spm_model** out);
spm_status spm_session_ep_handle(spm_session* s, void* handle64);
/* handles: the world ranks' 64-byte handles in rank order; a handle equal to
 * this session's own maps this session's own buffer. */
spm_status spm_session_ep_connect(spm_session* s, const void* handles);
/* Kernel launches issued by one step at client count n (graph nodes). */
spm_status spm_session_launches_per_step(spm_session* s, int32_t n, int32_t* launches);
/* Launch profile; no counterpart in the reference (its StepReport counts
 * weight bytes, spm-batch/src/session.rs:83-121, but times nothing).  While
 * enabled, steps run without the CUDA graph and every kernel launch of a step
 * is bracketed by a CUDA event pair on the session stream.  Enabling or
 * disabling clears the record.  spm_session_profile returns, for up to `max`
 * recorded launches, the device milliseconds, the algorithmic bytes (for a
 * GEMV the quantized weight bytes it streams, expert launches counting this
 * rank's active experts of that step; 0 for the other kernels) and the kind;
 * *count receives the number recorded. */
enum {
    SPM_GEMV_DENSE = 0,          /* GEMV: attention q/k/v, o; dense feed-forward */
    SPM_GEMV_ROUTER = 1,         /* GEMV: MoE router logits (expert parallel) */
    SPM_GEMV_EXPERT_GATE_UP = 2, /* GEMV: gate/up of the active experts       */
    SPM_GEMV_EXPERT_DOWN = 3,    /* GEMV: down projection of the active experts */
    SPM_GEMV_HEAD = 4,           /* GEMV: LM head                             */
    SPM_KERNEL_ATTENTION = 5,    /* QK-norm, RoPE, KV append, decode attention */
    SPM_KERNEL_ROUTE = 6,        /* router softmax, top-k, expert plan; on one
                                    GPU the router logits too (one launch)    */
    SPM_KERNEL_COMBINE = 7,      /* weighted expert combine + residual         */
    SPM_KERNEL_OTHER = 8         /* embedding gather, greedy pick, positions   */
};
spm_status spm_session_set_profile(spm_session* s, int32_t enable);
/* How long a device wait on other ranks (the expert-parallel combine waiting
 * for every rank's expert rows) may spin before it gives up, sets the
 * session's status word and goes on; the step then returns SPM_E_TIMEOUT and
 * its outputs are not to be used.  Default 1 s.  No counterpart in the
 * reference, which runs its experts in one process and reports typed errors
 * instead of panicking (spm-linear/src/stream.rs:31-55). */
spm_status spm_session_set_wait_limit(spm_session* s, uint64_t nanoseconds);
spm_status spm_session_profile(const spm_session* s, int32_t max, float* ms, uint64_t* bytes,
                               int32_t* kind, int32_t* count);

/* ---- .spm files and the ternary profile (Encoding::Ternary2F32I32) ----
 * A .spm file is a 32-byte header (spm-header/src/parse.rs:12-59), one
 * 32-byte descriptor per stream (spm-layout/src/wire.rs:12-30), then every
 * stream's scale groups in order, each an f32 scale followed by its payload
 * (spm-file/src/read.rs:69-101).  Errors follow the reference's:
 * HeaderError/LayoutError::TooShort and FileError::PayloadTruncated ->
 * SPM_E_TRUNCATED; BadMagic, UnsupportedVersion, UnknownEndianness,
 * ZeroGroupSize -> SPM_E_STREAM; UnknownEncoding -> SPM_E_ENCODING.  These
 * two calls run on the host only. */
typedef struct spm_file_stream_info {
    uint32_t rows, cols, group_size, encoding, lane_count, pad_;
    uint64_t groups;   /* scale groups in the stream                      */
    uint64_t offset;   /* file offset of its first group                  */
    uint64_t bytes;    /* its scales and payloads                         */
} spm_file_stream_info;
/* Header and directory (SpmReader::parse, spm-file/src/read.rs:46-67). */
spm_status spm_file_probe(const uint8_t* spm, uint64_t len, uint32_t* version_major, uint32_t* version_minor,
                          int32_t* streams);
/* Descriptor and placement of stream `index`; every group of streams
 * 0..index must be whole (SpmReader::next_group, read.rs:69-89). */
spm_status spm_file_stream(const uint8_t* spm, uint64_t len, int32_t index, spm_file_stream_info* out);

/* The ternary GEMV of spm_gemv_ref::run_gemv (spm-gemv-ref/src/gemv.rs:39-57,
 * datapath.rs:19-55) on the device.  Stream position k holds W[k % rows]
 * [k / rows]; a weight's group scale multiplies the activation, and each
 * nonzero code (bit 0) adds or, with bit 1, subtracts that product into the
 * row's f32 accumulator, in stream order.  Results are bit-identical to the
 * reference's for every input: each output keeps the reference's sequential
 * order of additions.  The reserved code 0b10 is a no-op, as in the
 * reference's datapath (spm_ternary_upload counts them).
 * spm_ternary_upload packs stream `index` into HBM; like run_gemv's scan, it
 * refuses a file whose next group after the stream is cut short, and it
 * refuses non-ternary streams (SPM_E_ENCODING) and files with no streams
 * (GemvError::NoStreams -> SPM_E_ARG). */
typedef struct spm_ternary spm_ternary;
spm_status spm_ternary_upload(const uint8_t* spm, uint64_t len, int32_t index, int device, spm_ternary** out);
spm_status spm_ternary_free(spm_ternary* t);
typedef struct spm_ternary_info {
    uint32_t rows, cols, group_size, pad_;
    uint64_t groups;
    uint64_t payload_bytes;   /* packed weight bytes of the stream (scales excluded) */
    uint64_t reserved_codes;  /* 0b10 codes in the stream                          */
    uint64_t device_bytes;    /* HBM held by the packed codes and scales           */
} spm_ternary_info;
spm_status spm_ternary_describe(const spm_ternary* t, spm_ternary_info* out);
/* y = W x for `lanes` activation vectors: x_dev is lanes x x_cols floats
 * (lane-major, Activations::per_lane), y_dev lanes x rows (bank.lane(l) for
 * each lane).  x_cols < cols is GemvError::MissingActivations
 * (SPM_E_ACTIVATION_LEN); extra activations are ignored.  Device pointers;
 * enqueued on cuda_stream (NULL = default stream). */
spm_status spm_ternary_gemv(const spm_ternary* t, const float* x_dev, int32_t lanes, uint64_t x_cols,
                            float* y_dev, void* cuda_stream);

/* spm_linear::streamed (spm-linear/src/stream.rs:31-125) for one dense .spm
 * stream (Encoding::F32 or Bf16; the group scale is inert): y[p][r] =
 * sum over c ascending of fma(W[r][c], x[p][c], .) from +0, one fused
 * multiply-add per weight and position as in resident.rs:124-137, so results
 * are bit-identical to the reference's.  spm_dense_upload packs stream
 * `index` into HBM; a profile without a dense decoder is refused as the
 * reference's DecodeError::Unsupported (SPM_E_STREAM, "parameter stream: Q6K
 * needs a scale-aware engine").  spm_dense_streamed: x_dev holds x_len floats
 * (positions x cols, LinearError::ActivationLen -> SPM_E_ACTIVATION_LEN when
 * x_len < positions x cols), y_dev positions x rows; device pointers,
 * enqueued on cuda_stream (NULL = default stream). */
typedef struct spm_dense spm_dense;
typedef struct spm_dense_info {
    uint32_t rows, cols, group_size, encoding;
    uint64_t groups;
    uint64_t payload_bytes;   /* weight bytes of the stream (scales excluded) */
    uint64_t device_bytes;    /* HBM held by the packed stream                */
} spm_dense_info;
spm_status spm_dense_upload(const uint8_t* spm, uint64_t len, int32_t index, int device, spm_dense** out);
spm_status spm_dense_free(spm_dense* t);
spm_status spm_dense_describe(const spm_dense* t, spm_dense_info* out);
spm_status spm_dense_streamed(const spm_dense* t, const float* x_dev, uint64_t x_len, int32_t positions,
                              float* y_dev, void* cuda_stream);

/* The block profiles of .spm files (Encoding::Q8_0, Q6K, Q5K: GGML blocks in
 * source row-major order, one block per group) as the reference's block
 * consumers compute them: q6_operation (spm-granite-moe/src/layout.rs:208-242)
 * and stream_matrix (gemma_smoke.rs:201-236) decode each block with
 * spm-gguf's decoders and apply value k = W[k / cols][k % cols] to every input
 * as out = fma(w, x, out).  Bit-identical results; a group that is not one
 * whole block is refused (SPM_E_STREAM, "unexpected packed group"), as the
 * reference refuses it.  x_dev holds x_len floats (positions x cols), y_dev
 * positions x rows; device pointers, enqueued on cuda_stream.  The fast GEMV
 * over the same blocks is the GGUF model path above. */
typedef struct spm_qblocks spm_qblocks;
spm_status spm_qblocks_upload(const uint8_t* spm, uint64_t len, int32_t index, int device, spm_qblocks** out);
spm_status spm_qblocks_free(spm_qblocks* t);
spm_status spm_qblocks_describe(const spm_qblocks* t, spm_dense_info* out);
spm_status spm_qblocks_gemv(const spm_qblocks* t, const float* x_dev, uint64_t x_len, int32_t positions,
                            float* y_dev, void* cuda_stream);

/* ---- host-to-HBM streaming of a .spm file ----
 * The reference's file-backed weight stream (spm-stream-file/src/prefetch.rs:
 * PrefetchFileWeightStream reads ahead into a bounded buffer) consumed stream
 * by stream in file order by streamed()/run_gemv and rewound between sweeps
 * (spm-stream-groups/src/groups.rs:88-117).  spm_sweep_open packs every stream
 * into pinned host memory (dense F32/Bf16, ternary and block-profile streams,
 * each refused as its own upload call refuses it) and keeps only a ring of
 * device_bytes on the device (0: twice the largest packed stream; less than
 * the largest is SPM_E_ARG).  spm_sweep_next runs the next stream in file
 * order on cuda_stream -- dense streams as spm_dense_streamed, ternary ones
 * as spm_ternary_gemv with x_cols = cols, block-profile ones as
 * spm_qblocks_gemv, bit-identical to the reference --
 * and copies the following streams into the ring meanwhile, as far as it
 * holds them, on a copy stream of its own.  x_dev holds x_len floats
 * (positions x cols), y_dev positions x rows; *stream_index receives the
 * stream run.  Once every stream has run, spm_sweep_next is SPM_E_TRUNCATED
 * until spm_sweep_rewind; a rewind in mid-sweep drops what was read ahead. */
typedef struct spm_sweep spm_sweep;
typedef struct spm_sweep_info {
    int32_t streams, position;   /* stream count; streams run in this sweep */
    uint64_t host_bytes;         /* pinned host memory of the packed streams */
    uint64_t device_bytes;       /* the ring                                 */
    uint64_t copies, bytes_copied;
} spm_sweep_info;
spm_status spm_sweep_open(const uint8_t* spm, uint64_t len, int device, uint64_t device_bytes, spm_sweep** out);
spm_status spm_sweep_open_file(const char* path, int device, uint64_t device_bytes, spm_sweep** out);
spm_status spm_sweep_close(spm_sweep* s);
spm_status spm_sweep_describe(const spm_sweep* s, spm_sweep_info* out);
spm_status spm_sweep_stream(const spm_sweep* s, int32_t index, uint32_t* rows, uint32_t* cols, uint32_t* encoding);
spm_status spm_sweep_next(spm_sweep* s, const float* x_dev, uint64_t x_len, int32_t positions, float* y_dev,
                          void* cuda_stream, int32_t* stream_index);
spm_status spm_sweep_rewind(spm_sweep* s);
/* The ring schedule of a sweep on the host, for checking it without a device:
 * streams regions of region_bytes (256-byte multiples) in a ring of
 * device_bytes, driven by `script` (SPM_PLAN_NEXT / SPM_PLAN_REWIND); *log_len
 * receives the number of log records and, when log is not NULL (log_cap
 * records of 4 int64: kind, stream, ring offset, event pair), the records in
 * issue order.  The CUDA backend issues exactly these actions for the same
 * calls: SPM_PLAN_EVENTS creates an event pair, SPM_PLAN_WAIT makes the copy
 * stream wait for a pair's consumed event, SPM_PLAN_COPY copies a stream then
 * records its copied event, SPM_PLAN_LAUNCH waits for copied, runs the kernel
 * and records consumed. */
enum { SPM_PLAN_NEXT = 1, SPM_PLAN_REWIND = 2 };
enum { SPM_PLAN_EVENTS = 1, SPM_PLAN_WAIT = 2, SPM_PLAN_COPY = 3, SPM_PLAN_LAUNCH = 4, SPM_PLAN_REFUSED = 5,
       SPM_PLAN_REWOUND = 6 };
spm_status spm_sweep_plan(const uint64_t* region_bytes, int32_t streams, uint64_t device_bytes,
                          const int32_t* script, int32_t script_len, int64_t* log, int64_t log_cap,
                          int64_t* log_len);

#ifdef __cplusplus
}
#endif
#endif
