/*
 * CPU oracle for the resident decoder-layer path (TEST INFRASTRUCTURE ONLY).
 *
 * This is an integer-only restatement of the reference's ap_fixed "golden"
 * model in host/host_qwen_8x64.cpp.  It exists to check the CUDA product
 * path; nothing in the shipped library links, loads or calls it.  Only the
 * pytest suite, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * use it, and only as the checker / timed CPU baseline.
 *
 * Pinning: the restatement is pinned against the reference's own golden
 * regression values (scripts/test_q214_payload_golden.sh:30-63 and
 * results/q214-resident-fix-20260818/raw/q214_payload_golden_regression.log)
 * and end-to-end logs (results/qwen3b-e2e-20260820/host.evidence.log,
 * results/qwen3b-e2e-l2-20260821/host.raw.log).  See tests/test_oracle_kat.py.
 *
 * Fixed-point notation used below (raw = stored integer):
 *   fm      Q8.8   int16   ap_fixed<16,8,AP_RND,AP_SAT>   (activations)
 *   w       Q4.12  int16   ap_fixed<16,4,AP_RND,AP_SAT>   (linear weights)
 *   accum   Q16.16 int32   ap_fixed<32,16,AP_RND,AP_SAT>
 *   prob    Q2.14  int16   ap_fixed<16,2,AP_RND,AP_SAT>
 * AP_RND = floor(x + half LSB); AP_SAT = clamp to the signed range.
 */
#ifndef LLMX_ORACLE_H
#define LLMX_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int32_t vocab;
    int32_t hidden;
    int32_t inter;
    int32_t layers;
    int32_t heads;
    int32_t kv_heads;
    int32_t max_seq;
} orc_shape_t;

/* ---- exp lookup tables (hls::exp stand-ins; index = raw Q8.8 input + 2048,
 *      input domain [-8, 0]) ------------------------------------------------ */
#define ORC_EXP_ROUND 0 /* round-half-up of the exact exponential */
#define ORC_EXP_TRUNC 1 /* truncation (floor) of the exact exponential */
void orc_exp_tables(int mode, int16_t *e16_8, int16_t *p18_4);
void orc_set_exp_mode(int mode);
int orc_get_exp_mode(void);
void orc_set_tables(const int16_t *e16_8, const int16_t *p18_4);

/* ---- scalar primitives ---------------------------------------------------- */
int16_t orc_recip(int16_t x);      /* golden_recip  host:537-576 */
int16_t orc_rsqrt(int32_t x);      /* golden_rsqrt  host:621-656 */
int16_t orc_silu(int16_t x);       /* golden_silu   host:658-668 */
int16_t orc_exp_fm(int16_t x);     /* golden_exp    host:578-586 */
int16_t orc_prob(int16_t x);       /* golden_attention_probability host:588-596 */
int16_t orc_inv_rms_const(int32_t n); /* inv_rms when recip(fm(n)) == 0 */

/* ---- tensor ops (row-major int16) ---------------------------------------- */
void orc_set_threads(int n); /* host threads for the projections (default 1) */
void orc_projection(const int16_t *x, int rows, int in_dim, const int16_t *w,
                    int out_dim, int16_t *y);
void orc_projection_partial(const int16_t *x, int rows, int in_dim,
                            const int16_t *w, int w_stride, int out_dim,
                            int k_begin, int k_end, int64_t *partial);
void orc_round_partial(const int64_t *partial, size_t n, int16_t *y);
void orc_rmsnorm(const int16_t *x, int rows, int n, const int16_t *w,
                 int16_t *y);
void orc_silu_mul(const int16_t *g, const int16_t *u, size_t n, int16_t *y);
void orc_residual(const int16_t *a, const int16_t *b, size_t n, int16_t *y);
void orc_rope_table(int head_dim, int max_seq, int16_t *table);
void orc_attention_group(const int16_t *q, int group, const int16_t *k,
                         const int16_t *v, int ctx, int head_dim, int payload,
                         int16_t *out);

/* ---- coarse tasks (dense per-layer weight blob: Q,K,V,O,Gate,Up,Down,
 *      each [out][in] row-major, concatenated) ----------------------------- */
size_t orc_layer_weight_elems(const orc_shape_t *s);
void orc_task18(const orc_shape_t *s, const int16_t *layer_w,
                const int16_t *attn_norm, const int16_t *rope,
                int16_t *k_cache, int16_t *v_cache, const int16_t *hidden_in,
                int rows, int position, int payload, int16_t *hidden_out);
void orc_task19(const orc_shape_t *s, const int16_t *layer_w,
                const int16_t *ffn_norm, const int16_t *hidden_in, int rows,
                int16_t *hidden_out);
void orc_prefill_sequence_layer(const orc_shape_t *s, const int16_t *layer_w,
                                const int16_t *attn_norm,
                                const int16_t *ffn_norm, const int16_t *rope,
                                const int16_t *hidden, int rows, int payload,
                                int16_t *post_attention, int16_t *out);
int32_t orc_lm_head_argmax(const int16_t *h, const int16_t *w, int vocab,
                           int hidden, int threads);
uint64_t orc_checksum(const int16_t *x, size_t n);

/* ---- reference random model (mt19937 + libstdc++-9 uniform_int) -------- */
void orc_mt_uniform_fill(uint32_t seed, int lo, int hi, int16_t *out,
                         size_t n);
int orc_ref_random_model(const orc_shape_t *s, uint32_t seed, int keep_layers,
                         int16_t *embedding, int16_t *norms, int16_t *dense);

/* ---- synthetic N(0, sigma) fixed-point generator ------------------------ */
int orc_gauss_table(double sigma_raw, uint64_t *thresholds, int max_entries,
                    int *kmin);
void orc_gauss_fill(uint64_t seed, uint64_t stream, double sigma_raw,
                    uint64_t index0, int16_t *out, size_t n);

#ifdef __cplusplus
}
#endif
#endif
