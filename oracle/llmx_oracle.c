/*
 * CPU oracle for the resident decoder-layer path -- TEST INFRASTRUCTURE ONLY.
 *
 * Integer-only restatement of the reference's ap_fixed golden model
 * (host/host_qwen_8x64.cpp).  Every function names the reference lines it
 * follows.  The shipped library never links this file; the pytest suite,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load it as the
 * checker and as the timed CPU baseline.
 *
 * ap_fixed semantics restated here (Vitis HLS 2022.2, non SC_COMPATIBLE):
 *  - an expression of ap_fixed operands is evaluated at full precision
 *    (a*b keeps all bits, a+b keeps all bits);
 *  - assignment/conversion quantises once: AP_RND = floor(x + half LSB),
 *    then AP_SAT clamps to the destination range;
 *  - a / b on ap_fixed yields (a_raw << F_b) / b_raw with C integer
 *    division (truncation toward zero) and F_a fraction bits.
 */
#include "llmx_oracle.h"

#include <limits.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* rounding / saturation helpers                                             */
/* ------------------------------------------------------------------------ */
static inline int64_t rnd64(int64_t v, int k) {
    /* AP_RND dropping k fraction bits: floor(v / 2^k + 1/2). */
    return (v + ((int64_t)1 << (k - 1))) >> k;
}
static inline __int128 rnd128(__int128 v, int k) {
    return (v + ((__int128)1 << (k - 1))) >> k;
}
static inline int32_t sat32(int64_t v) {
    return v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
}
static inline int32_t sat32_128(__int128 v) {
    return v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : (int32_t)v);
}
static inline int16_t sat16(int64_t v) {
    return v > INT16_MAX ? INT16_MAX : (v < INT16_MIN ? INT16_MIN : (int16_t)v);
}
/* Q8.8 -> Q4.12 with saturation (golden_weight_t(fm) in host:3249,3719). */
static inline int32_t to_w412(int16_t fm) { return sat16((int32_t)fm * 16); }
/* ap_fixed<W,I,AP_RND> constructed from a double: floor(x*2^F + 1/2). */
static inline int64_t fixed_from_double(double x, int frac) {
    return (int64_t)floor(ldexp(x, frac) + 0.5);
}

/* ------------------------------------------------------------------------ */
/* exp tables                                                                */
/* ------------------------------------------------------------------------ */
/* Stand-ins for hls::exp(ap_fixed<16,8>) (host:578-586, kernel/compute_stream.cpp:50-55)
 * and hls::exp(ap_fixed<18,4>) (host:588-596, kernel/control_cache_8x64.cpp:4079-4091).
 * On this path both only see Q8.8 inputs clamped to [-8, 0] (2049 values). The Xilinx
 * source is not available; candidates are built from the exact exponential and the
 * one that reproduces the reference's golden regression values is selected. */
static int16_t g_e16[2049];
static int16_t g_p18[2049];
static int g_exp_mode = -1;

void orc_exp_tables(int mode, int16_t *e16_8, int16_t *p18_4) {
    for (int i = 0; i <= 2048; i++) {
        const long double x = (long double)(i - 2048) / 256.0L;
        const long double e = expl(x);
        const long double a = e * 256.0L;
        const long double b = e * 16384.0L;
        if (mode == ORC_EXP_TRUNC) {
            e16_8[i] = (int16_t)floorl(a);
            p18_4[i] = (int16_t)floorl(b);
        } else {
            e16_8[i] = (int16_t)floorl(a + 0.5L);
            p18_4[i] = (int16_t)floorl(b + 0.5L);
        }
    }
}

void orc_set_exp_mode(int mode) {
    orc_exp_tables(mode, g_e16, g_p18);
    g_exp_mode = mode;
}

int orc_get_exp_mode(void) { return g_exp_mode; }

/* Install explicit tables (used to evaluate candidate hls::exp tables). */
void orc_set_tables(const int16_t *e16_8, const int16_t *p18_4) {
    memcpy(g_e16, e16_8, sizeof(g_e16));
    memcpy(g_p18, p18_4, sizeof(g_p18));
    g_exp_mode = 99;
}

static void ensure_tables(void) {
    if (g_exp_mode < 0) orc_set_exp_mode(ORC_EXP_TRUNC);
}

/* golden_exp host:578-586: clamp to [-8, 8]; only [-8, 0] occurs on the path. */
int16_t orc_exp_fm(int16_t x) {
    ensure_tables();
    int32_t c = x < -2048 ? -2048 : x;
    if (c > 0) c = 0; /* never reached on the path: SiLU passes -|x| */
    return g_e16[c + 2048];
}

/* golden_attention_probability host:588-596: clamp to [-8, 0], exp at Q4.14 -> Q2.14 */
int16_t orc_prob(int16_t x) {
    ensure_tables();
    int32_t c = x < -2048 ? -2048 : (x > 0 ? 0 : x);
    return g_p18[c + 2048];
}

/* ------------------------------------------------------------------------ */
/* recip / rsqrt / silu                                                      */
/* ------------------------------------------------------------------------ */
/* golden_recip host:537-576 (kernel twin: kernel/compute_stream.cpp:15-48). */
int16_t orc_recip(int16_t x) {
    /* fm(0.000244140625) rounds to raw 0, so safe = value < 0 ? 0 : value. */
    const int64_t safe = x < 0 ? 0 : x;
    int64_t e;
    if (safe >= 64 * 256) e = 4;
    else if (safe >= 32 * 256) e = 8;
    else if (safe >= 16 * 256) e = 16;
    else if (safe >= 8 * 256) e = 32;
    else if (safe >= 4 * 256) e = 64;
    else if (safe >= 2 * 256) e = 128;
    else if (safe >= 256) e = 256;
    else if (safe >= 128) e = 512;
    else if (safe >= 64) e = 1024;
    else if (safe >= 32) e = 2048;
    else e = 4096;
    for (int i = 0; i < 3; i++) {
        /* e * (2 - safe*e): exact at 24 fraction bits, one rounding to Q8.8 */
        const int64_t diff = 2 * 65536 - safe * e;
        e = sat16(rnd64(e * diff, 16));
    }
    if (e < 0) e = 0;
    if (e > 64 * 256) e = 64 * 256;
    return (int16_t)e;
}

/* golden_rsqrt host:621-656 (kernel twin: kernel/compute_stream.cpp:57-86). */
int16_t orc_rsqrt(int32_t x) {
    const int64_t safe = x < 16 ? 16 : x; /* accum(2^-12) = raw 16 */
    int64_t e;
    if (safe >= ((int64_t)64 << 16)) e = 32;
    else if (safe >= ((int64_t)16 << 16)) e = 64;
    else if (safe >= ((int64_t)4 << 16)) e = 128;
    else if (safe >= ((int64_t)1 << 16)) e = 256;
    else if (safe >= 16384) e = 512;
    else if (safe >= 4096) e = 1024;
    else e = 2048;
    for (int i = 0; i < 3; i++) {
        const int64_t ea = e * 256; /* accum(e) */
        const int32_t square = sat32(rnd64(ea * ea, 16));
        /* 1.5 - 0.5*safe*square at 48 fraction bits, rounded once to Q16.16 */
        const __int128 t = ((__int128)3 << 47) - (__int128)32768 * safe * square;
        const int32_t refine = sat32_128(rnd128(t, 32));
        e = sat16(rnd64(ea * (int64_t)refine, 24));
    }
    if (e < 0) e = 0;
    if (e > 32 * 256) e = 32 * 256;
    return (int16_t)e;
}

/* golden_silu host:658-668 (kernel twin: kernel/compute_stream.cpp:88-96). */
int16_t orc_silu(int16_t v) {
    if (v >= 0) {
        const int16_t e = orc_exp_fm(sat16(-(int32_t)v));
        const int16_t r = orc_recip(sat16(256 + (int32_t)e));
        return sat16(rnd64((int64_t)v * r, 8));
    }
    const int16_t e = orc_exp_fm(v);
    const int16_t r = orc_recip(sat16(256 + (int32_t)e));
    return sat16(rnd64((int64_t)v * e * r, 16));
}

/* ------------------------------------------------------------------------ */
/* tensor ops                                                                */
/* ------------------------------------------------------------------------ */
/* Exact 48-bit (ap_int<48>, AP_WRAP) MAC total, then Q28.20 -> Q16.16 -> Q8.8:
 * golden_projection host:3105-3142; kernel/mm_stream_8x64_fused_mac.cpp:11-22,89-96;
 * kernel/compute_core_8x64_unified.cpp:31-35. */
static inline int16_t round_mac_total(int64_t s) {
    s = (int64_t)((uint64_t)s << 16) >> 16; /* ap_int<48> wrap (never reached) */
    const int32_t accum = sat32(rnd64(s, 4));
    return sat16(rnd64(accum, 8));
}

static int g_threads = 1;
void orc_set_threads(int n) { g_threads = n < 1 ? 1 : (n > 256 ? 256 : n); }

typedef struct {
    const int16_t *x, *w;
    int16_t *y;
    int rows, in_dim, out_dim, o_begin, o_end;
} proj_job_t;

static void *proj_worker(void *arg) {
    const proj_job_t *j = (const proj_job_t *)arg;
    for (int o = j->o_begin; o < j->o_end; o++) {
        const int16_t *wr = j->w + (size_t)o * j->in_dim;
        for (int r = 0; r < j->rows; r++) {
            const int16_t *xr = j->x + (size_t)r * j->in_dim;
            int64_t s = 0;
            for (int i = 0; i < j->in_dim; i++) s += (int32_t)xr[i] * (int32_t)wr[i];
            j->y[(size_t)r * j->out_dim + o] = round_mac_total(s);
        }
    }
    return NULL;
}

/* Rows x out_dim exact dot products; output features split over g_threads. */
void orc_projection(const int16_t *x, int rows, int in_dim, const int16_t *w,
                    int out_dim, int16_t *y) {
    int t = g_threads;
    if ((int64_t)out_dim * in_dim * rows < (1 << 22) || t > out_dim) t = 1;
    proj_job_t jobs[256];
    pthread_t tid[256];
    for (int i = 0; i < t; i++) {
        jobs[i] = (proj_job_t){x, w, y, rows, in_dim, out_dim, (int)((int64_t)out_dim * i / t),
                               (int)((int64_t)out_dim * (i + 1) / t)};
        if (t == 1) proj_worker(&jobs[0]);
        else pthread_create(&tid[i], NULL, proj_worker, &jobs[i]);
    }
    if (t > 1)
        for (int i = 0; i < t; i++) pthread_join(tid[i], NULL);
}

/* Exact integer partial dot products over input columns [k_begin, k_end):
 * the quantity a tensor-parallel rank exports before the all-reduce. */
void orc_projection_partial(const int16_t *x, int rows, int in_dim,
                            const int16_t *w, int w_stride, int out_dim,
                            int k_begin, int k_end, int64_t *partial) {
    for (int r = 0; r < rows; r++) {
        const int16_t *xr = x + (size_t)r * in_dim;
        for (int o = 0; o < out_dim; o++) {
            const int16_t *wr = w + (size_t)o * w_stride;
            int64_t s = 0;
            for (int i = k_begin; i < k_end; i++) s += (int32_t)xr[i] * (int32_t)wr[i];
            partial[(size_t)r * out_dim + o] = s;
        }
    }
}

void orc_round_partial(const int64_t *partial, size_t n, int16_t *y) {
    for (size_t i = 0; i < n; i++) y[i] = round_mac_total(partial[i]);
}

/* golden_rmsnorm host:3162-3197 (kernel: compute_stream.cpp:227-288). */
void orc_rmsnorm(const int16_t *x, int rows, int n, const int16_t *w,
                 int16_t *y) {
    /* golden_fm_t(input.cols): an unsigned count saturates at 127.996. */
    const int16_t n_fm = (int16_t)(n >= 128 ? 32767 : n * 256);
    const int16_t inv_elems = orc_recip(n_fm);
    const int64_t eps = fixed_from_double(0.000001, 16); /* rounds to 0 */
    for (int r = 0; r < rows; r++) {
        const int16_t *xr = x + (size_t)r * n;
        int32_t sum = 0;
        for (int e = 0; e < n; e++) sum = sat32((int64_t)sum + (int64_t)xr[e] * xr[e]);
        const int32_t mean = sat32(rnd64((int64_t)sum * ((int64_t)inv_elems * 256), 16));
        const int16_t inv_rms = orc_rsqrt(sat32((int64_t)mean + eps));
        for (int e = 0; e < n; e++) {
            const int64_t p = (int64_t)xr[e] * inv_rms * w[e];
            y[(size_t)r * n + e] = sat16(rnd64(p, 16));
        }
    }
}

int16_t orc_inv_rms_const(int32_t n) {
    const int16_t n_fm = (int16_t)(n >= 128 ? 32767 : n * 256);
    (void)orc_recip(n_fm);
    return orc_rsqrt(sat32(fixed_from_double(0.000001, 16)));
}

/* golden_silu_mul host:3199-3217 */
void orc_silu_mul(const int16_t *g, const int16_t *u, size_t n, int16_t *y) {
    for (size_t i = 0; i < n; i++) y[i] = sat16(rnd64((int64_t)orc_silu(g[i]) * u[i], 8));
}

/* golden_residual host:3144-3160 */
void orc_residual(const int16_t *a, const int16_t *b, size_t n, int16_t *y) {
    for (size_t i = 0; i < n; i++) y[i] = sat16((int32_t)a[i] + b[i]);
}

/* quantize_fix16 host:496-505: std::round (half away from zero) then clamp. */
static int16_t quantize_fix16(double v) {
    const double s = round(v * 256.0);
    if (s > 32767.0) return 32767;
    if (s < -32768.0) return -32768;
    return (int16_t)s;
}

/* RoPE table [pos][cos half | sin half] as built at host:2162-2190 and used
 * directly by profile_apply_rope host:4790-4852 (theta = 1e6). */
void orc_rope_table(int head_dim, int max_seq, int16_t *table) {
    const int half = head_dim / 2;
    for (int p = 0; p < max_seq; p++) {
        for (int i = 0; i < half; i++) {
            const double exponent = (double)(2 * i) / head_dim;
            const double inv_freq = 1.0 / pow(1000000.0, exponent);
            const double angle = (double)(unsigned)p * inv_freq;
            table[(size_t)p * head_dim + i] = quantize_fix16(cos(angle));
            table[(size_t)p * head_dim + half + i] = quantize_fix16(sin(angle));
        }
    }
}

/* rotate_fix16_pair_with_quantized_rope host:4765-4788 */
static void rope_rotate(int16_t *vec, int heads, int head_dim, const int16_t *row) {
    const int half = head_dim / 2;
    for (int h = 0; h < heads; h++) {
        int16_t *b = vec + (size_t)h * head_dim;
        for (int i = 0; i < half; i++) {
            const int64_t x0 = b[i], x1 = b[half + i];
            const int64_t c = row[i], s = row[half + i];
            b[i] = sat16(rnd64(x0 * c - x1 * s, 8));
            b[half + i] = sat16(rnd64(x1 * c + x0 * s, 8));
        }
    }
}

/* golden_tiled_flash_attention_q2_14_impl host:3610-3739, with the QK scores of
 * golden_attention_mm host:3219-3278 (per-product rounding to Q16.16, four
 * saturating banks over k mod 4, sum, x fm(1/sqrt(d))).  payload=1 is the
 * production raw-payload semantics; payload=0 the "direct" Q2.14 variant. */
void orc_attention_group(const int16_t *q, int group, const int16_t *k,
                         const int16_t *v, int ctx, int hd, int payload,
                         int16_t *out) {
    enum { TILE = 64 };
    const int64_t scale = fixed_from_double(1.0 / sqrt((double)hd), 8) * 256;
    int16_t *omax = (int16_t *)malloc(sizeof(int16_t) * group);
    int32_t *osum = (int32_t *)calloc((size_t)group, sizeof(int32_t));
    int32_t *acc = (int32_t *)calloc((size_t)group * hd, sizeof(int32_t));
    int16_t *score = (int16_t *)malloc(sizeof(int16_t) * group * TILE);
    int16_t *prob = (int16_t *)malloc(sizeof(int16_t) * group * TILE);
    for (int g = 0; g < group; g++) omax[g] = -32768; /* fm(-128) */
    for (int t0 = 0; t0 < ctx; t0 += TILE) {
        const int tl = ctx - t0 < TILE ? ctx - t0 : TILE;
        for (int g = 0; g < group; g++) {
            for (int p = 0; p < tl; p++) {
                int32_t bank[4] = {0, 0, 0, 0};
                const int16_t *kr = k + (size_t)(t0 + p) * hd;
                for (int e = 0; e < hd; e++) {
                    const int64_t prod = rnd64((int64_t)q[(size_t)g * hd + e] * to_w412(kr[e]), 4);
                    if (e < 4) bank[e & 3] = (int32_t)prod;
                    else bank[e & 3] = sat32((int64_t)bank[e & 3] + prod);
                }
                int32_t tot = sat32((int64_t)bank[0] + bank[1] + bank[2] + bank[3]);
                tot = sat32(rnd64((int64_t)tot * scale, 16));
                score[g * TILE + p] = sat16(rnd64(tot, 8));
            }
        }
        for (int g = 0; g < group; g++) {
            int16_t rm = omax[g];
            for (int p = 0; p < tl; p++)
                if (score[g * TILE + p] > rm) rm = score[g * TILE + p];
            const int64_t old = (int64_t)orc_prob(sat16((int32_t)omax[g] - rm)) * 4;
            int32_t tsum = 0;
            for (int p = 0; p < tl; p++) {
                const int16_t pr = orc_prob(sat16((int32_t)score[g * TILE + p] - rm));
                prob[g * TILE + p] = pr;
                tsum = sat32((int64_t)tsum + (int64_t)pr * 4);
            }
            osum[g] = sat32(rnd64((int64_t)osum[g] * old, 16) + tsum);
            omax[g] = rm;
            for (int e = 0; e < hd; e++)
                acc[(size_t)g * hd + e] = sat32(rnd64((int64_t)acc[(size_t)g * hd + e] * old, 16));
        }
        for (int g = 0; g < group; g++) {
            for (int e = 0; e < hd; e++) {
                int32_t bank[4] = {0, 0, 0, 0};
                for (int p = 0; p < tl; p++) {
                    const int64_t pw = (int64_t)prob[g * TILE + p] * to_w412(v[(size_t)(t0 + p) * hd + e]);
                    const int64_t prod = payload ? rnd64(pw, 4) : rnd64(pw, 10);
                    if (p < 4) bank[p & 3] = (int32_t)prod;
                    else bank[p & 3] = sat32((int64_t)bank[p & 3] + prod);
                }
                int32_t ts = sat32((int64_t)bank[0] + bank[1] + bank[2] + bank[3]);
                if (payload) ts = sat32(rnd64((int64_t)ts * 1024, 16)); /* x accum(fm(1/64)) */
                const int16_t tv = sat16(rnd64(ts, 8));
                acc[(size_t)g * hd + e] = sat32((int64_t)acc[(size_t)g * hd + e] + (int64_t)tv * 256);
            }
        }
    }
    for (int g = 0; g < group; g++) {
        const int64_t s = osum[g] < 16 ? 16 : osum[g];
        const int64_t quot = ((int64_t)1 << 32) / s; /* accum(1)/safe: 16 fraction bits */
        const int64_t inv = sat16(rnd64(quot, 8));
        for (int e = 0; e < hd; e++)
            out[(size_t)g * hd + e] = sat16(rnd64((int64_t)acc[(size_t)g * hd + e] * inv * 256, 24));
    }
    free(omax);
    free(osum);
    free(acc);
    free(score);
    free(prob);
}

/* ------------------------------------------------------------------------ */
/* coarse tasks                                                              */
/* ------------------------------------------------------------------------ */
typedef struct {
    const int16_t *q, *k, *v, *o, *g, *u, *d;
} layer_ptrs_t;

static layer_ptrs_t layer_ptrs(const orc_shape_t *s, const int16_t *w) {
    const size_t H = (size_t)s->hidden, I = (size_t)s->inter;
    const size_t KV = (size_t)s->kv_heads * (H / s->heads);
    layer_ptrs_t p;
    p.q = w;
    p.k = p.q + H * H;
    p.v = p.k + KV * H;
    p.o = p.v + KV * H;
    p.g = p.o + H * H;
    p.u = p.g + I * H;
    p.d = p.u + I * H;
    return p;
}

size_t orc_layer_weight_elems(const orc_shape_t *s) {
    const size_t H = (size_t)s->hidden, I = (size_t)s->inter;
    const size_t KV = (size_t)s->kv_heads * (H / s->heads);
    return 2 * H * H + 2 * KV * H + 3 * I * H;
}

/* Task 18 (attention sublayer) with an incremental KV cache for one layer
 * ([kv_head][max_seq][head_dim]).  Row t of the block sits at position+t and
 * attends to positions <= position+t.  Equivalent to the golden full-prefix
 * recompute golden_prefill_decoder_layer_sequence host:4854-4978 (attention
 * half) -- proven equal in tests/test_oracle_incremental.py. */
void orc_task18(const orc_shape_t *s, const int16_t *layer_w,
                const int16_t *attn_norm, const int16_t *rope,
                int16_t *k_cache, int16_t *v_cache, const int16_t *hidden_in,
                int rows, int position, int payload, int16_t *hidden_out) {
    const int H = s->hidden, hd = H / s->heads, KV = s->kv_heads * hd;
    const int G = s->heads / s->kv_heads;
    const layer_ptrs_t W = layer_ptrs(s, layer_w);
    int16_t *xn = (int16_t *)malloc(sizeof(int16_t) * rows * H);
    int16_t *q = (int16_t *)malloc(sizeof(int16_t) * rows * H);
    int16_t *kk = (int16_t *)malloc(sizeof(int16_t) * rows * KV);
    int16_t *vv = (int16_t *)malloc(sizeof(int16_t) * rows * KV);
    int16_t *att = (int16_t *)malloc(sizeof(int16_t) * rows * H);
    int16_t *proj = (int16_t *)malloc(sizeof(int16_t) * rows * H);
    orc_rmsnorm(hidden_in, rows, H, attn_norm, xn);
    orc_projection(xn, rows, H, W.q, H, q);
    orc_projection(xn, rows, H, W.k, KV, kk);
    orc_projection(xn, rows, H, W.v, KV, vv);
    for (int t = 0; t < rows; t++) {
        const int pos = position + t;
        const int16_t *row = rope + (size_t)pos * hd;
        rope_rotate(q + (size_t)t * H, s->heads, hd, row);
        rope_rotate(kk + (size_t)t * KV, s->kv_heads, hd, row);
        for (int h = 0; h < s->kv_heads; h++) {
            memcpy(k_cache + ((size_t)h * s->max_seq + pos) * hd, kk + (size_t)t * KV + (size_t)h * hd,
                   sizeof(int16_t) * hd);
            memcpy(v_cache + ((size_t)h * s->max_seq + pos) * hd, vv + (size_t)t * KV + (size_t)h * hd,
                   sizeof(int16_t) * hd);
        }
        for (int h = 0; h < s->kv_heads; h++) {
            orc_attention_group(q + (size_t)t * H + (size_t)h * G * hd, G,
                                k_cache + (size_t)h * s->max_seq * hd,
                                v_cache + (size_t)h * s->max_seq * hd, pos + 1, hd, payload,
                                att + (size_t)t * H + (size_t)h * G * hd);
        }
    }
    orc_projection(att, rows, H, W.o, H, proj);
    orc_residual(hidden_in, proj, (size_t)rows * H, hidden_out);
    free(xn);
    free(q);
    free(kk);
    free(vv);
    free(att);
    free(proj);
}

/* Task 19 (FFN sublayer): golden_prefill_decoder_layer_sequence host:4962-4977 */
void orc_task19(const orc_shape_t *s, const int16_t *layer_w,
                const int16_t *ffn_norm, const int16_t *hidden_in, int rows,
                int16_t *hidden_out) {
    const int H = s->hidden, I = s->inter;
    const layer_ptrs_t W = layer_ptrs(s, layer_w);
    int16_t *xn = (int16_t *)malloc(sizeof(int16_t) * rows * H);
    int16_t *g = (int16_t *)malloc(sizeof(int16_t) * (size_t)rows * I);
    int16_t *u = (int16_t *)malloc(sizeof(int16_t) * (size_t)rows * I);
    int16_t *d = (int16_t *)malloc(sizeof(int16_t) * rows * H);
    orc_rmsnorm(hidden_in, rows, H, ffn_norm, xn);
    orc_projection(xn, rows, H, W.g, I, g);
    orc_projection(xn, rows, H, W.u, I, u);
    orc_silu_mul(g, u, (size_t)rows * I, g);
    orc_projection(g, rows, I, W.d, H, d);
    orc_residual(hidden_in, d, (size_t)rows * H, hidden_out);
    free(xn);
    free(g);
    free(u);
    free(d);
}

/* golden_prefill_decoder_layer_sequence host:4854-4978: the whole sequence at
 * position 0 with a private cache (full-prefix recompute form). */
void orc_prefill_sequence_layer(const orc_shape_t *s, const int16_t *layer_w,
                                const int16_t *attn_norm,
                                const int16_t *ffn_norm, const int16_t *rope,
                                const int16_t *hidden, int rows, int payload,
                                int16_t *post_attention, int16_t *out) {
    const int hd = s->hidden / s->heads;
    orc_shape_t t = *s;
    if (t.max_seq < rows) t.max_seq = rows;
    int16_t *kc = (int16_t *)calloc((size_t)t.kv_heads * t.max_seq * hd, sizeof(int16_t));
    int16_t *vc = (int16_t *)calloc((size_t)t.kv_heads * t.max_seq * hd, sizeof(int16_t));
    int16_t *pa = (int16_t *)malloc(sizeof(int16_t) * rows * s->hidden);
    orc_task18(&t, layer_w, attn_norm, rope, kc, vc, hidden, rows, 0, payload, pa);
    if (post_attention) memcpy(post_attention, pa, sizeof(int16_t) * rows * s->hidden);
    orc_task19(&t, layer_w, ffn_norm, pa, rows, out);
    free(kc);
    free(vc);
    free(pa);
}

/* lm_head_argmax host:937-977: int64 dot products, strict '>' keeps the first max. */
typedef struct {
    const int16_t *h, *w;
    int begin, end, hidden;
    int64_t best;
    int32_t token;
} argmax_job_t;

static void *argmax_worker(void *arg) {
    argmax_job_t *j = (argmax_job_t *)arg;
    j->best = INT64_MIN;
    j->token = j->begin;
    for (int t = j->begin; t < j->end; t++) {
        const int16_t *wr = j->w + (size_t)t * j->hidden;
        int64_t s = 0;
        for (int e = 0; e < j->hidden; e++) s += (int64_t)j->h[e] * wr[e];
        if (s > j->best) {
            j->best = s;
            j->token = t;
        }
    }
    return NULL;
}

int32_t orc_lm_head_argmax(const int16_t *h, const int16_t *w, int vocab,
                           int hidden, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    argmax_job_t jobs[256];
    pthread_t tid[256];
    for (int i = 0; i < threads; i++) {
        jobs[i].h = h;
        jobs[i].w = w;
        jobs[i].hidden = hidden;
        jobs[i].begin = (int)((int64_t)vocab * i / threads);
        jobs[i].end = (int)((int64_t)vocab * (i + 1) / threads);
        pthread_create(&tid[i], NULL, argmax_worker, &jobs[i]);
    }
    int64_t best = INT64_MIN;
    int32_t token = 0;
    for (int i = 0; i < threads; i++) {
        pthread_join(tid[i], NULL);
        if (jobs[i].end > jobs[i].begin && jobs[i].best > best) {
            best = jobs[i].best;
            token = jobs[i].token;
        }
    }
    return token;
}

/* tensor_checksum host:8542-8549: FNV-1a-64 over the uint16 values. */
uint64_t orc_checksum(const int16_t *x, size_t n) {
    uint64_t c = 1469598103934665603ull;
    for (size_t i = 0; i < n; i++) {
        c ^= (uint16_t)x[i];
        c *= 1099511628211ull;
    }
    return c;
}

/* ------------------------------------------------------------------------ */
/* reference random model                                                    */
/* ------------------------------------------------------------------------ */
/* std::mt19937 (the published MT19937 algorithm, 32-bit). */
typedef struct {
    uint32_t mt[624];
    int idx;
} mt19937_t;

static void mt_seed(mt19937_t *m, uint32_t seed) {
    m->mt[0] = seed;
    for (int i = 1; i < 624; i++)
        m->mt[i] = 1812433253u * (m->mt[i - 1] ^ (m->mt[i - 1] >> 30)) + (uint32_t)i;
    m->idx = 624;
}

static void mt_twist(mt19937_t *m) {
    for (int i = 0; i < 624; i++) {
        const uint32_t y = (m->mt[i] & 0x80000000u) | (m->mt[(i + 1) % 624] & 0x7fffffffu);
        uint32_t v = m->mt[(i + 397) % 624] ^ (y >> 1);
        if (y & 1u) v ^= 0x9908b0dfu;
        m->mt[i] = v;
    }
    m->idx = 0;
}

static inline uint32_t mt_next(mt19937_t *m) {
    if (m->idx >= 624) mt_twist(m);
    uint32_t y = m->mt[m->idx++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* std::uniform_int_distribution<int>(lo, hi) as shipped in libstdc++ of GCC 9
 * (Ubuntu 20.04, the reference's host): the "division downscaling" rejection
 * sampler (urng range 2^32-1 > requested range). */
typedef struct {
    uint64_t scaling, past;
    int lo;
} uniform_t;

static uniform_t uniform_make(int lo, int hi) {
    uniform_t u;
    const uint64_t urngrange = 0xffffffffull;
    const uint64_t uerange = (uint64_t)((int64_t)hi - lo) + 1;
    u.scaling = urngrange / uerange;
    u.past = uerange * u.scaling;
    u.lo = lo;
    return u;
}

static inline int uniform_draw(const uniform_t *u, mt19937_t *m) {
    uint64_t r;
    do {
        r = mt_next(m);
    } while (r >= u->past);
    return (int)(r / u->scaling) + u->lo;
}

/* make_random_tensor host:3089-3103 */
void orc_mt_uniform_fill(uint32_t seed, int lo, int hi, int16_t *out, size_t n) {
    mt19937_t m;
    mt_seed(&m, seed);
    const uniform_t u = uniform_make(lo, hi);
    for (size_t i = 0; i < n; i++) out[i] = (int16_t)uniform_draw(&u, &m);
}

/* projection_spec host:270-331 base tiles, in 16x16 tile units. */
static void op_tiles(const orc_shape_t *s, size_t base[8], size_t in_tiles[7],
                     int out_dim[7], int in_dim[7]) {
    const int H = s->hidden, I = s->inter, KV = s->kv_heads * (H / s->heads);
    const int od[7] = {H, KV, KV, H, I, I, H};
    const int id[7] = {H, H, H, H, H, H, I};
    base[0] = 0;
    for (int op = 0; op < 7; op++) {
        out_dim[op] = od[op];
        in_dim[op] = id[op];
        in_tiles[op] = (size_t)(id[op] + 15) / 16;
        base[op + 1] = base[op] + ((size_t)(od[op] + 15) / 16) * in_tiles[op];
    }
}

/* model_data_t::initialize_random_model host:842-869 (draw order: embedding,
 * norms, then 16 shards word by word), decoded into the dense per-layer blob
 * through the tile/shard mapping of projection_weight_raw host:899-935.
 * Only layers < keep_layers are stored; the rest of the stream is drawn and
 * discarded so that later shards line up.  embedding may be NULL. */
int orc_ref_random_model(const orc_shape_t *s, uint32_t seed, int keep_layers,
                         int16_t *embedding, int16_t *norms, int16_t *dense) {
    size_t base[8], in_tiles[7];
    int od[7], id[7];
    op_tiles(s, base, in_tiles, od, id);
    const size_t layer_tiles = base[7];
    const size_t shard_words = (layer_tiles * (size_t)s->layers + 1) / 2;
    const size_t layer_elems = orc_layer_weight_elems(s);
    size_t dense_off[7];
    dense_off[0] = 0;
    for (int op = 0; op < 6; op++) dense_off[op + 1] = dense_off[op] + (size_t)od[op] * id[op];

    mt19937_t m;
    mt_seed(&m, seed);
    const uniform_t feat = uniform_make(-128, 128);
    const uniform_t nrm = uniform_make(224, 288);
    const uniform_t wt = uniform_make(-64, 64);
    const size_t emb_n = (size_t)s->vocab * s->hidden;
    for (size_t i = 0; i < emb_n; i++) {
        const int v = uniform_draw(&feat, &m);
        if (embedding) embedding[i] = (int16_t)v;
    }
    const size_t norm_n = ((size_t)s->layers * 2 + 1) * s->hidden;
    for (size_t i = 0; i < norm_n; i++) norms[i] = (int16_t)uniform_draw(&nrm, &m);
    const size_t keep_words = (layer_tiles * (size_t)keep_layers + 1) / 2;
    for (int shard = 0; shard < 16; shard++) {
        const int group = shard / 8, tile_word = shard % 8;
        for (size_t word = 0; word < shard_words; word++) {
            if (word >= keep_words || !dense) {
                for (int lane = 0; lane < 32; lane++) (void)uniform_draw(&wt, &m);
                continue;
            }
            const size_t gtile = 2 * word + (size_t)group;
            const size_t layer = gtile / layer_tiles;
            const size_t t = gtile % layer_tiles;
            int op = 0;
            while (op < 6 && t >= base[op + 1]) op++;
            const size_t local = t - base[op];
            const size_t trow = local / in_tiles[op], tcol = local % in_tiles[op];
            for (int lane = 0; lane < 32; lane++) {
                const int v = uniform_draw(&wt, &m);
                const int lane_in_tile = tile_word * 32 + lane;
                const size_t out = trow * 16 + (size_t)(lane_in_tile / 16);
                const size_t in = tcol * 16 + (size_t)(lane_in_tile % 16);
                if ((int)layer < keep_layers && out < (size_t)od[op] && in < (size_t)id[op])
                    dense[layer * layer_elems + dense_off[op] + out * (size_t)id[op] + in] = (int16_t)v;
            }
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* synthetic N(0, sigma) generator (the workload definition for the BASELINE */
/* configs; the product library carries its own implementation of the same  */
/* definition and a CPU test proves the two identical)                        */
/* ------------------------------------------------------------------------ */
/* Definition: element i of stream (seed, stream) is the smallest integer k
 * with U < T(k), where U = top 32 bits of splitmix64(key + i),
 * key = splitmix64(seed ^ (stream * 0xD1B54A32D192ED03)), and
 * T(k) = round(2^32 * Phi((k + 1/2) / sigma_raw)) for k in [-K, K), T(K) = 2^32,
 * K = min(ceil(8 sigma_raw), 32767).  This samples round-half-up(N(0, sigma_raw))
 * exactly up to the 2^-32 resolution of U (the AP_RND quantisation of a Gaussian). */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int orc_gauss_table(double sigma_raw, uint64_t *thresholds, int max_entries, int *kmin) {
    int K = (int)ceil(8.0 * sigma_raw);
    if (K > 32767) K = 32767;
    const int n = 2 * K + 1;
    if (n > max_entries) return -1;
    for (int j = 0; j < n - 1; j++) {
        const int k = j - K;
        const double x = ((double)k + 0.5) / sigma_raw;
        const double phi = 0.5 * erfc(-x * 0.70710678118654752440);
        thresholds[j] = (uint64_t)llround(ldexp(phi, 32));
    }
    thresholds[n - 1] = (uint64_t)1 << 32;
    *kmin = -K;
    return n;
}

typedef struct {
    const uint64_t *tab;
    int cnt, kmin;
    uint64_t key, index0;
    int16_t *out;
    size_t begin, end;
} gauss_job_t;

static void *gauss_worker(void *arg) {
    const gauss_job_t *j = (const gauss_job_t *)arg;
    for (size_t i = j->begin; i < j->end; i++) {
        const uint64_t u = mix64(j->key + j->index0 + i) >> 32;
        int lo = 0, hi = j->cnt - 1; /* smallest index with u < tab[index] */
        while (lo < hi) {
            const int mid = (lo + hi) / 2;
            if (u < j->tab[mid]) hi = mid;
            else lo = mid + 1;
        }
        j->out[i] = (int16_t)(lo + j->kmin);
    }
    return NULL;
}

void orc_gauss_fill(uint64_t seed, uint64_t stream, double sigma_raw,
                    uint64_t index0, int16_t *out, size_t n) {
    uint64_t *tab = (uint64_t *)malloc(sizeof(uint64_t) * 65536);
    int kmin = 0;
    const int cnt = orc_gauss_table(sigma_raw, tab, 65536, &kmin);
    const uint64_t key = mix64(seed ^ (stream * 0xD1B54A32D192ED03ull));
    int t = n < (1u << 20) ? 1 : g_threads;
    gauss_job_t jobs[256];
    pthread_t tid[256];
    for (int i = 0; i < t; i++) {
        jobs[i] = (gauss_job_t){tab, cnt, kmin, key, index0, out, n * i / t, n * (i + 1) / t};
        if (t == 1) gauss_worker(&jobs[0]);
        else pthread_create(&tid[i], NULL, gauss_worker, &jobs[i]);
    }
    if (t > 1)
        for (int i = 0; i < t; i++) pthread_join(tid[i], NULL);
    free(tab);
}
