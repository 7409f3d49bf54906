/*
 * llmx -- B200-native drop-in for LLM-ACCEL's resident decoder-layer path.
 *
 * C ABI (plain pointers and sizes, no C++ or torch types).  Each entry point
 * names the reference interface it replaces (paths relative to the
 * LLM-ACCEL tree).  The boundary is the XRT accelerator object
 * (host/host_qwen_8x64.cpp: accelerator_t, lines 1024-3087) plus the
 * controller/compute-CU pair it drives (kernel/control_cache_8x64.cpp:5767,
 * kernel/compute_core_8x64_unified.cpp:281).  The host runtime above it
 * (qwen_executor_t, host:7607-8161; model_data_t, host:779-1022) is also
 * provided here in C++ so that a caller can switch wholesale.
 *
 * Numerics: every result is bit-identical to the fixed-point golden model
 * (Q8.8 activations, Q4.12 weights, Q16.16 accumulators, Q2.14 softmax).
 *
 * Return codes: 0 = OK; 1..5 are the controller status codes of
 * include/control_cache_8x64.hpp:279-286; >= 100 are runtime errors of this
 * library (no exceptions cross the ABI).
 */
#ifndef LLMX_H
#define LLMX_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes: cc8_status_code_t include/control_cache_8x64.hpp:279-286 */
#define LLMX_OK 0
#define LLMX_BAD_OPERATOR 1
#define LLMX_BAD_TOKEN_COUNT 2
#define LLMX_BAD_TILE_LENGTH 3
#define LLMX_BAD_POSITION 4
#define LLMX_BAD_LAYER 5
#define LLMX_ERR_CUDA 100     /* a CUDA runtime call failed */
#define LLMX_ERR_ARG 101      /* null pointer / size mismatch / bad buffer id */
#define LLMX_ERR_STATE 102    /* model not loaded, context not ready */
#define LLMX_ERR_NCCL 103     /* collective failed (an asynchronous NCCL error aborts the communicator) */
#define LLMX_ERR_RANGE 104    /* value outside the weight range the kernels accept */
#define LLMX_ERR_NOMEM 105    /* device or host allocation failed */
#define LLMX_ERR_IO 106       /* checkpoint file missing or wrong size */
#define LLMX_ERR_UNSUPPORTED 107
#define LLMX_ERR_TIMEOUT 108     /* a kernel's bounded wait expired (device error flag), or NCCL
                                    collectives were still pending after LLMX_NCCL_TIMEOUT_MS (the
                                    communicator is aborted; the context then answers
                                    LLMX_ERR_STATE until llmx_destroy) */

/* ---- operators: operator_kind_t host:69-91 / cc8_operator_t
 *      include/control_cache_8x64.hpp:252-277 ---- */
#define LLMX_OP_NOP 0
/* per-operator (feature) modes, llmx_run_feature */
#define LLMX_OP_Q_PROJECTION 1
#define LLMX_OP_K_PROJECTION 2
#define LLMX_OP_V_PROJECTION 3
#define LLMX_OP_O_PROJECTION 4
#define LLMX_OP_FFN_GATE 5
#define LLMX_OP_FFN_UP 6
#define LLMX_OP_FFN_DOWN 7
#define LLMX_OP_RMSNORM 8
#define LLMX_OP_SILU_MUL 9
#define LLMX_OP_RESIDUAL_ADD 10
/* 11-15 (QK, PV, softmax, flash, decode smoke tile diagnostics): not served */
#define LLMX_OP_DECODER_LAYER 16      /* full layer = Task 18 then Task 19, llmx_task */
#define LLMX_OP_ATTN_PREFILL_BLOCK 17 /* llmx_run_prefill_attention_block */
/* coarse resident tasks, llmx_task / llmx_stack */
#define LLMX_OP_ATTENTION_SUBLAYER 18 /* Task 18 */
#define LLMX_OP_FFN_SUBLAYER 19       /* Task 19 */
#define LLMX_OP_FINAL_NORM 20         /* Task 20 */

#define LLMX_MAX_ROWS 8 /* kMaxTokensPerLaunch host:38 */

/* Model shape: model_shape_t host:110-236. */
typedef struct llmx_shape {
    int32_t vocab;
    int32_t hidden;
    int32_t inter;
    int32_t layers;
    int32_t heads;
    int32_t kv_heads;
    int32_t max_seq;
} llmx_shape;

/* 64-byte status record: cc8_status_packet_t include/control_cache_8x64.hpp:298-307,
 * packed by kernel/cc8_status_sink.cpp:4-15, decoded by decode_status host:670-684. */
typedef struct llmx_status {
    uint32_t op;
    uint32_t code;
    uint32_t token_count;
    uint32_t output_waves;
    uint32_t mm_tasks;
    uint32_t vector_tasks;
    uint32_t completed_packets;
    uint32_t last_task;
    uint32_t reserved[8];
} llmx_status;

typedef struct llmx_ctx llmx_ctx;     /* one per GPU / tensor-parallel rank */
typedef struct llmx_model llmx_model; /* host-side model container */

/* ---------------------------------------------------------------------------
 * Shapes, validation, status (pure host functions, no GPU needed)
 * ------------------------------------------------------------------------- */

/* parse_profile host:348-379 ("small", "medium", "qwen-layer",
 * "qwen-layer-long", "qwen2.5-3b"). Returns LLMX_ERR_ARG for an unknown name. */
int llmx_profile(const char *name, llmx_shape *out);

/* model_shape_t::validate host:224-236 plus this library's own limits. */
int llmx_shape_validate(const llmx_shape *shape);

/* Controller argument validation kernel/control_cache_8x64.cpp:5891-5972,
 * 5974-5984, 6041-6054, run on the host before any launch.  Fills *st with the
 * record the controller would emit (counters included) and returns st->code. */
int llmx_validate_task(const llmx_shape *shape, uint32_t op, uint32_t layer,
                       uint32_t position, uint32_t rows, llmx_status *st);
/* The same for the controller image with the per-operator schedulers
 * (kernel/control_cache_8x64.cpp:6496-7497): additionally accepts the feature
 * operators 1-10 (no position check; counters of :7273-7497) and the prefill
 * block attention 17 (:6496-6522, counters of check_prefill_block_attention_status
 * host:5587-5604).  Ops 11-15 get LLMX_BAD_OPERATOR. */
int llmx_validate_operator(const llmx_shape *shape, uint32_t op, uint32_t layer,
                           uint32_t position, uint32_t rows, llmx_status *st);
/* feature_input_dim / feature_output_dim / needs_rhs host:2015-2061 of a feature
 * operator (1-10); LLMX_ERR_ARG for any other operator. */
int llmx_feature_dims(const llmx_shape *shape, uint32_t op, uint32_t *in_dim,
                      uint32_t *out_dim, int *needs_rhs);

/* Human-readable name of a return code. */
const char *llmx_strerror(int code);
/* Detail of the last runtime error on the calling thread ("" if none). */
const char *llmx_last_error(void);

/* Constant tables the device path uses, for inspection and tests:
 * exp tables (index = Q8.8 input + 2048, input in [-8, 0]) standing in for
 * hls::exp(ap_fixed<16,8>) -> Q8.8 (SiLU, kernel/compute_stream.cpp:50-55) and
 * hls::exp(ap_fixed<18,4>) -> Q2.14 (softmax, kernel/control_cache_8x64.cpp:4079-4091);
 * RoPE table [max_seq][cos half | sin half] of host:2162-2190. */
int llmx_exp_tables(int16_t *e16_8, int16_t *p18_4);
int llmx_rope_table(int head_dim, int max_seq, int16_t *table);
/* Seeded N(0, sigma_raw) integer sampler of the synthetic benchmark model
 * (round-half-up quantisation of a Gaussian; see llmx_model_init_gaussian). */
int llmx_gauss_fill(uint64_t seed, uint64_t stream, double sigma_raw, uint64_t index0,
                    int16_t *out, size_t n);

/* ---------------------------------------------------------------------------
 * Host model container: model_data_t host:779-1022
 * ------------------------------------------------------------------------- */
int llmx_model_create(const llmx_shape *shape, llmx_model **out);
void llmx_model_destroy(llmx_model *m);
/* initialize_random_model host:842-869 (mt19937 + libstdc++-9 uniform_int,
 * tied embeddings).  Keeps layers < keep_layers resident in host memory
 * (keep_layers <= 0 keeps all). */
int llmx_model_init_reference_random(llmx_model *m, uint32_t seed, int keep_layers);
/* Seeded synthetic model for the benchmark configurations: linear weights and
 * LM head N(0, w_sigma) quantised to Q4.12, embeddings N(0, 1) quantised to
 * Q8.8, norm weights 1.0.  lm_head != 0 materialises an untied LM head. */
int llmx_model_init_gaussian(llmx_model *m, uint64_t seed, double w_sigma, int lm_head);
/* model_data_t::load host:789-840: token_embedding.fix16.bin,
 * norm_weights.fix16.bin, layer_weights_shardNN.fix16.bin (packed 16x16 tile
 * layout of projection_weight_raw host:899-935), optional lm_head.fix16.bin. */
int llmx_model_load_packed(llmx_model *m, const char *dir, int tie_embeddings);
/* Raw access for callers that build their own weights: the dense per-layer
 * blob (Q,K,V,O,Gate,Up,Down, each [out][in] row-major int16). */
size_t llmx_layer_weight_elems(const llmx_shape *shape);
int16_t *llmx_model_layer(llmx_model *m, uint32_t layer);
int16_t *llmx_model_norms(llmx_model *m);        /* [2L+1][hidden] */
int16_t *llmx_model_embedding(llmx_model *m);    /* [vocab][hidden] or NULL */
/* model_data_t::embedding host:871-884 (rows of token ids -> Q8.8 rows). */
int llmx_model_embed(const llmx_model *m, const uint32_t *tokens, uint32_t n,
                     int16_t *out_rows);
/* model_data_t::lm_head_argmax host:937-977: argmax_t sum int64(h*W), the first
 * maximum wins.  threads <= 0 uses all host cores. */
int llmx_model_lm_head_argmax(const llmx_model *m, const int16_t *hidden_row,
                              int threads, uint32_t *token);

/* ---------------------------------------------------------------------------
 * Device context: accelerator_t host:1024-3087
 * ------------------------------------------------------------------------- */
/* 128-byte opaque id used to form a tensor-parallel group (ncclUniqueId). */
int llmx_tp_unique_id(void *id128);
/* Create a context on `device`.  tp_size > 1 shards Q/O heads and FFN columns
 * over the group (K/V heads replicated) and all-reduces exact int64 partial
 * sums after the O and Down projections; tp_id is the llmx_tp_unique_id of
 * rank 0 broadcast to every rank. */
int llmx_create(const llmx_shape *shape, int device, int tp_rank, int tp_size,
                const void *tp_id, llmx_ctx **out);
int llmx_destroy(llmx_ctx *ctx);
/* migrate_initial_model_state host:2458-2478: upload weights (re-laid-out for
 * the GPU kernels and sliced for this rank), norm table and RoPE table. */
int llmx_upload_model(llmx_ctx *ctx, const llmx_model *m);
/* Same, one layer from a dense blob (Q,K,V,O,Gate,Up,Down [out][in]). */
int llmx_upload_layer(llmx_ctx *ctx, uint32_t layer, const int16_t *dense);
int llmx_upload_norms(llmx_ctx *ctx, const int16_t *norms);
/* Clears the device KV cache (accelerator_t ctor clears kv_cache_*_words_). */
int llmx_reset_kv(llmx_ctx *ctx);
/* initialize_kv_cache_heads host:1729-1843: preload / read back the post-RoPE K
 * and the V rows of positions [position, position+count) of one layer.  Host
 * layout of k and v: [kv_head][count][head_dim] Q8.8. */
int llmx_write_kv(llmx_ctx *ctx, uint32_t layer, uint32_t position, uint32_t count,
                  const int16_t *k, const int16_t *v);
int llmx_read_kv(llmx_ctx *ctx, uint32_t layer, uint32_t position, uint32_t count,
                 int16_t *k, int16_t *v);

/* Hidden-state buffers: the four feature buffers of create_buffers
 * host:2296-2385 used as two pairs; pair 0 = buffers {0,1}, pair 1 = {2,3}.
 * Each pair holds up to 8 rows x hidden Q8.8 values (row-major on device). */
/* pack_feature host:2062-2080 + H2D migration. */
int llmx_write_hidden(llmx_ctx *ctx, uint32_t pair, const int16_t *rows_host,
                      uint32_t rows);
/* D2H migration + unpack_feature host:2082-2100. */
int llmx_read_hidden(llmx_ctx *ctx, uint32_t pair, int16_t *rows_host, uint32_t rows);
/* bind_controller_data_ports host:1846-1888 (output pair, input pair). */
int llmx_bind(llmx_ctx *ctx, uint32_t out_pair, uint32_t in_pair);
/* execute_bound_resident_task host:1890-2053: runs Task 18/19/20, the
 * compatibility full-layer Task 16 (run_decoder_layer host:1136-1176; the
 * input pair is left unchanged) or NOP on the bound pairs, stream-ordered,
 * waits for completion and returns the status record.  Returns st->code (0 = OK). */
int llmx_task(llmx_ctx *ctx, uint32_t op, uint32_t layer, uint32_t position,
              uint32_t rows, llmx_status *st);
/* run_feature host:1088-1130: one feature operator (1-10) on host rows.
 * lhs [rows][lhs_cols] with lhs_cols == in_dim; rhs (RMSNorm: the [1][hidden]
 * weight row; SiLU-Mul: up rows; residual add: the second rows) [rhs_rows][rhs_cols];
 * out [rows][out_cols] with out_cols == out_dim.  Projections use layer's
 * weights (golden_projection host:3105-3142: exact sum, one double rounding);
 * RMSNorm, SiLU-Mul and the residual add are the resident path's own kernels.
 * Shape mismatches (the reference's runtime_error) return LLMX_ERR_ARG before
 * any launch; controller codes come back in st->code.  Single-GPU contexts
 * only (LLMX_ERR_UNSUPPORTED on a tensor-parallel rank). */
int llmx_run_feature(llmx_ctx *ctx, uint32_t op, const int16_t *lhs, uint32_t rows,
                     uint32_t lhs_cols, const int16_t *rhs, uint32_t rhs_rows,
                     uint32_t rhs_cols, uint32_t layer, uint32_t position, int16_t *out,
                     uint32_t out_cols, llmx_status *st);
/* run_prefill_attention_block host:1647-1690 (op 17): attention of `rows`
 * consecutive query tokens at positions position..position+rows-1 against
 * layer's KV cache (which already holds those rows, e.g. via llmx_write_kv),
 * causal per token.  query / out: kv_heads ports, port p = [rows][G][head_dim]
 * of the G query heads of KV head p (token-major, then local head; ports back
 * to back).  Same arithmetic as Task 18's attention.  Single-GPU only. */
int llmx_run_prefill_attention_block(llmx_ctx *ctx, const int16_t *query, uint32_t position,
                                     uint32_t rows, uint32_t layer, int16_t *out,
                                     llmx_status *st);
/* run_composed_decoder_stack host:1258-1493: host rows in -> layers
 * [layer_begin, layer_begin+layer_count) as Task 18/19 pairs -> optional
 * Task 20 -> optional host rows out.  Launched as one CUDA graph (cached per
 * row count); kernels read the position from device memory so one graph
 * serves every position.  `last` receives the final task's status. */
int llmx_stack(llmx_ctx *ctx, const int16_t *hidden_in, uint32_t rows,
               uint32_t layer_begin, uint32_t layer_count, uint32_t position,
               int include_final_norm, int materialize, int16_t *hidden_out,
               llmx_status *last);
/* Stream-ordered variant of llmx_stack on device rows (no host copies, no
 * wait): input rows already in pair 1, result in pair 0 (final norm) or
 * pair 1.  For timing loops and graph capture by the caller. */
int llmx_stack_async(llmx_ctx *ctx, uint32_t rows, uint32_t layer_begin,
                     uint32_t layer_count, uint32_t position, int include_final_norm);
int llmx_synchronize(llmx_ctx *ctx);
/* The CUDA stream the context launches on (cudaStream_t as void*). */
void *llmx_stream(llmx_ctx *ctx);
/* Device pointer of a hidden pair ([8][hidden] int16) for zero-copy callers. */
void *llmx_hidden_device_ptr(llmx_ctx *ctx, uint32_t pair);
/* Number of kernels the last llmx_stack/llmx_stack_async launched. */
uint64_t llmx_kernel_launches(const llmx_ctx *ctx);
/* Bytes of device memory the context holds. */
uint64_t llmx_device_bytes(const llmx_ctx *ctx);
/* How a tensor-parallel context adds the ranks' exact partial sums after the
 * O and Down projections (no reference counterpart: the reference runs on one
 * device; this is the all-reduce of the tensor-parallel split).  Every rank of
 * a group reports the same kind: the ranks agree on it in llmx_create. */
#define LLMX_AR_NONE 0   /* one GPU: no all-reduce */
#define LLMX_AR_NCCL 1   /* ncclAllReduce(int64) + rounding kernel (LLMX_TP_NCCL=1, or some rank
                            could not map a peer's exchange region) */
#define LLMX_AR_PEER 2   /* peer stores over NVLink, finished in the next projection's prologue */
int llmx_allreduce_kind(const llmx_ctx *ctx);
/* 1 when one-row stacks run the O projection inside the attention kernel (single
 * GPU; LLMX_ATTN_FUSE_O=0 disables): each attention cluster adds its head's exact
 * partial of every O row into int64 sums that the Gate/Up prologue rounds (with
 * the residual), so a decode layer is four launches instead of five. */
int llmx_decode_fuses_o(const llmx_ctx *ctx);
/* Failure-detection self-test (no reference counterpart; the reference's
 * controller has no waits that can expire).  Runs the receiving side of the
 * peer all-reduce on an exchange region that no rank writes, with a wait of
 * at most poll_limit polls per word: the kernel gives up, records its error
 * status and returns, and the call returns LLMX_ERR_TIMEOUT with the context
 * still usable.  Works on one GPU; overwrites hidden pair 0. */
int llmx_selftest_ar_timeout(llmx_ctx *ctx, uint32_t poll_limit);

/* Kernels of the path, for per-kernel timing (no reference counterpart: the
 * reference reads its CU running times from the XRT profile_kernels.csv,
 * scripts/report_hwemu_kernel_cycles.sh:25-38). */
#define LLMX_KERNEL_QKV 0        /* RMSNorm + Q/K/V + RoPE + KV append */
#define LLMX_KERNEL_ATTN 1       /* tile-exact online-softmax attention */
#define LLMX_KERNEL_O 2          /* O projection + residual */
#define LLMX_KERNEL_GATE_UP 3    /* RMSNorm + Gate/Up + SiLU x Up */
#define LLMX_KERNEL_DOWN 4       /* Down projection + residual */
#define LLMX_KERNEL_FINAL_NORM 5
/* Launch one kernel of the path `iters` times back to back on the context
 * stream (operating on whatever the buffers hold; launch i uses layer
 * (layer + i) mod layers so consecutive launches stream distinct weights)
 * between two CUDA events and return the mean device time per launch in ms. */
int llmx_time_kernel(llmx_ctx *ctx, int kernel, uint32_t layer, uint32_t position,
                     uint32_t rows, int iters, double *ms_per_launch);

/* ---------------------------------------------------------------------------
 * LM-head argmax on the device, without allocation.  No counterpart in the
 * reference: its argmax runs on the host (model_data_t::lm_head_argmax
 * host:937-977), which llmx_model_lm_head_argmax mirrors; this returns the
 * same tokens (exact int64 scores, the first maximum wins).
 *
 * For callers that cannot allocate device memory at sampling time: a serving
 * loop whose HBM is fully committed to weights and KV cache, or code running
 * several streams where cudaMalloc / cudaFree would synchronise the device.
 * The call allocates nothing; its scratch is one fixed 128 KiB device array
 * per device (8 rows x 1024 blocks of partial results), shared by every call.
 *
 *   hidden   device, [rows][hidden_size] int16 (Q8.8), 16-byte aligned
 *   lm_head  device, [vocab][hidden_size] int16 (Q4.12), 16-byte aligned
 *   tokens   device, [rows] uint32 (written in stream order)
 *   stream   cudaStream_t as void* (NULL = legacy default stream)
 * Limits: 1 <= rows <= 8 (LLMX_ERR_ARG beyond), hidden_size a multiple of 8.
 * The first call on each device does a one-time set-up there (looks up the
 * scratch array's address); make that first call before any stream capture.
 * The address is kept for the life of the process, so do not call this after
 * cudaDeviceReset() on a device it has already been used on.
 * Calls share the scratch, so calls that may overlap on the device (different
 * streams without ordering) race: order them on one stream or with events.
 * Stream-ordered: returns after enqueueing two kernels. */
int llmx_lm_head_argmax_device(const int16_t *hidden, uint32_t rows, uint32_t hidden_size,
                               const int16_t *lm_head, uint32_t vocab, uint32_t *tokens,
                               void *stream);

/* ---------------------------------------------------------------------------
 * Host runtime: qwen_executor_t host:7607-8161
 * ------------------------------------------------------------------------- */
/* run_prompt_block host:7840-7918: embedding rows of 1..8 tokens at
 * `position`, full stack; final norm + output only when materialize != 0. */
int llmx_run_prompt_block(llmx_ctx *ctx, const llmx_model *m, const uint32_t *tokens,
                          uint32_t n, uint32_t position, int materialize,
                          int16_t *hidden_out);
/* run_token host:7665-7700: one decode forward, final-normed hidden out. */
int llmx_run_token(llmx_ctx *ctx, const llmx_model *m, uint32_t token,
                   uint32_t position, int16_t *hidden_out);

/* ---------------------------------------------------------------------------
 * Greedy generation on the device: the coarse-task branch of the reference's
 * generate mode (main, host:9016-9132), with the embedding gather
 * (model_data_t::embedding host:871-884) and the LM-head argmax
 * (model_data_t::lm_head_argmax host:937-977) moved onto the GPU.  Same
 * tokens as the host loop; the host waits once, at the end.
 * ------------------------------------------------------------------------- */
/* Copies the model's token-embedding table and LM head (the embedding itself
 * when tied) into device memory owned by the context: 2 * vocab * hidden bytes,
 * twice that when untied.  A synthetic model's embedding is materialised on the
 * host first.  May be called again to replace the tables. */
int llmx_upload_vocab(llmx_ctx *ctx, llmx_model *m);
/* Prompt tokens in blocks of block_rows (1..8) rows at positions 0, block_rows,
 * ... (run_prompt_block host:7840-7918; only the last block is final-normed),
 * then max_new tokens: each is the argmax of the previous final-normed row and,
 * except the last, runs as one decode row (run_token host:7665-7700) at the
 * next position.  layer_count 0 = every layer (the executor's --layers,
 * host:7621-7640).  out_tokens[max_new]; last_block_out (may be NULL) receives
 * the last prompt block's final-normed rows [rows][hidden], whose per-row
 * FNV-1a checksums the reference prints (host:9042-9057).  Needs
 * n_prompt + max_new - 1 <= max_seq, uploaded layers [0, layer_count), norms
 * and llmx_upload_vocab.  All ranks of a tensor-parallel group call it with
 * the same arguments. */
int llmx_generate(llmx_ctx *ctx, const uint32_t *prompt, uint32_t n_prompt, uint32_t block_rows,
                  uint32_t layer_count, uint32_t max_new, uint32_t *out_tokens, int16_t *last_block_out);

#ifdef __cplusplus
}
#endif
#endif
