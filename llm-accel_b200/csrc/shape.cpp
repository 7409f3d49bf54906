// Shapes, controller argument validation, status records and constant tables.
#include <cmath>
#include <cstring>

#include "host_model.h"

namespace llmx {

static inline uint32_t cdiv(uint64_t a, uint64_t b) { return (uint32_t)((a + b - 1) / b); }

// hls::exp stand-ins for the two instantiations on the path (inputs are Q8.8
// clamped to [-8, 0], index = raw + 2048):
//  - ap_fixed<18,4> -> Q2.14 softmax probability (kernel/control_cache_8x64.cpp:4079-4091)
//  - ap_fixed<16,8> -> Q8.8 SiLU exponential (kernel/compute_stream.cpp:50-55)
// Both are the truncated exact exponential; the Q2.14 table reproduces the
// reference's golden regression values exactly.
void build_exp_tables(int16_t *e16_8, int16_t *p18_4) {
    for (int i = 0; i <= 2048; i++) {
        const long double x = (long double)(i - 2048) / 256.0L;
        const long double e = expl(x);
        e16_8[i] = (int16_t)floorl(e * 256.0L);
        p18_4[i] = (int16_t)floorl(e * 16384.0L);
    }
}

// quantize_fix16 host:496-505 (std::round, clamp) of the persistent RoPE
// table host:2162-2190: row = position, [cos(hd/2) | sin(hd/2)], theta 1e6.
static int16_t quantize_fix16(double v) {
    const double s = std::round(v * 256.0);
    if (s > 32767.0) return 32767;
    if (s < -32768.0) return -32768;
    return (int16_t)s;
}

void build_rope_table(int head_dim, int max_seq, int16_t *table) {
    const int half = head_dim / 2;
    for (int p = 0; p < max_seq; p++) {
        for (int i = 0; i < half; i++) {
            const double exponent = (double)(2 * i) / head_dim;
            const double inv_freq = 1.0 / std::pow(1000000.0, exponent);
            const double angle = (double)(unsigned)p * inv_freq;
            table[(size_t)p * head_dim + i] = quantize_fix16(std::cos(angle));
            table[(size_t)p * head_dim + half + i] = quantize_fix16(std::sin(angle));
        }
    }
}

// golden_attention_mm host:3226-3228: fm(1/sqrt(d)) (AP_RND from double), as Q16.16.
int32_t qk_scale_q1616(int head_dim) {
    const int32_t fm = (int32_t)std::floor(std::ldexp(1.0 / std::sqrt((double)head_dim), 8) + 0.5);
    return fm * 256;
}

}  // namespace llmx

using namespace llmx;

namespace {

// Controller argument validation and the status record of a completed task
// (kernel/control_cache_8x64.cpp:5869-5972, then the per-operator checks of
// Task 20 :5974-5984, the resident layer tasks :6031-6054, the prefill block
// :6496-6522 and the legacy feature scheduler :7273-7497).  full == false is
// the production resident-layer image: every operator other than NOP and Tasks
// 16, 18, 19, 20 is rejected (:6484-6494).  full == true is the image with the
// per-operator schedulers; of those this library serves ops 1-10 and 17, and
// answers the tile-diagnostic ops 11-15 as the resident image does.
int validate_op(const llmx_shape *s, uint32_t op, uint32_t layer, uint32_t position, uint32_t rows,
                llmx_status *st, bool full) {
    if (!s || !st) return LLMX_ERR_ARG;
    std::memset(st, 0, sizeof(*st));
    st->op = LLMX_OP_NOP;
    st->token_count = rows;
    st->last_task = 1;
    // :5891-5897: row count first, before the operator
    if (rows > LLMX_MAX_ROWS) return st->code = LLMX_BAD_TOKEN_COUNT;
    st->op = op;
    const bool resident = op == LLMX_OP_NOP || op == LLMX_OP_DECODER_LAYER || op == LLMX_OP_ATTENTION_SUBLAYER ||
                          op == LLMX_OP_FFN_SUBLAYER || op == LLMX_OP_FINAL_NORM;
    const bool feature = op >= LLMX_OP_Q_PROJECTION && op <= LLMX_OP_RESIDUAL_ADD;
    if (!resident && !(full && (feature || op == LLMX_OP_ATTN_PREFILL_BLOCK))) return st->code = LLMX_BAD_OPERATOR;
    if (op == LLMX_OP_NOP) return st->code = LLMX_OK;
    if (layer >= (uint32_t)s->layers) return st->code = LLMX_BAD_LAYER;
    const uint32_t H = s->hidden, I = s->inter, hd = s->hidden / s->heads;
    const uint32_t KV = s->kv_heads * hd, G = s->heads / s->kv_heads;
    const uint32_t pv_waves = cdiv(hd, 64);  // CC8_ATTN_PV_WAVES: 64 outputs per MM wave
    if (feature) {
        uint32_t in_dim = 0, out_dim = 0;
        int rhs = 0;
        llmx_feature_dims(s, op, &in_dim, &out_dim, &rhs);
        if (op <= LLMX_OP_FFN_DOWN) {  // one projection: 128 outputs per wave on both cores
            const uint32_t waves = cdiv(out_dim, 128);
            st->output_waves = waves;
            st->mm_tasks = 2 * waves;
            st->completed_packets = waves * 2 * 32;
        } else {  // vector operator: tokens 0-3 on core 0, 4-7 on core 1
            st->vector_tasks = (rows > 0 ? 1u : 0u) + (rows > 4 ? 1u : 0u);
            st->completed_packets = rows * cdiv(out_dim, 16);
        }
        return st->code = LLMX_OK;
    }
    if (rows == 0) return st->code = LLMX_BAD_TOKEN_COUNT;
    if (op != LLMX_OP_FINAL_NORM &&
        (position >= (uint32_t)s->max_seq || (uint64_t)position + rows > (uint64_t)s->max_seq))
        return st->code = LLMX_BAD_POSITION;
    // status counters of a completed task (tests/closed_loop_8x64_cosim_tb.cpp:523-626)
    const uint32_t fanout = cdiv(rows, 4);
    uint32_t waves = 0, vec = 0, packets = 0;
    if (op == LLMX_OP_ATTENTION_SUBLAYER || op == LLMX_OP_DECODER_LAYER) {
        uint32_t w = cdiv(H, 128) + 2 * cdiv(KV, 128) + cdiv(H, 128);
        for (uint32_t t = 0; t < rows; t++) w += cdiv((uint64_t)position + t + 1, 64) * (1 + pv_waves);
        waves += w;
        vec += 2 * fanout;
        packets += w * 2 * 32 + 2 * rows * cdiv(H, 16);
    }
    if (op == LLMX_OP_FFN_SUBLAYER || op == LLMX_OP_DECODER_LAYER) {
        const uint32_t w = 2 * cdiv(I, 128) + cdiv(H, 128);
        waves += w;
        vec += 3 * fanout;
        packets += w * 2 * 32 + rows * (2 * cdiv(H, 16) + cdiv(I, 16));
    }
    if (op == LLMX_OP_FINAL_NORM) {
        vec = fanout;
        packets = rows * cdiv(H, 16);
    }
    if (op == LLMX_OP_ATTN_PREFILL_BLOCK) {
        // :6511-6522 and check_prefill_block_attention_status host:5587-5604: every
        // context tile runs QK plus the PV waves for each GQA head on both cores
        // (the per-launch task limit is never reached for position + rows <= max_seq)
        const uint32_t tasks_per_core = cdiv((uint64_t)position + rows, 64) * G * (1 + pv_waves);
        st->output_waves = pv_waves;
        st->mm_tasks = 2 * tasks_per_core;
        st->completed_packets = st->mm_tasks * 32;
        return st->code = LLMX_OK;
    }
    st->output_waves = waves;
    st->mm_tasks = 2 * waves;
    st->vector_tasks = vec;
    st->completed_packets = packets;
    return st->code = LLMX_OK;
}

}  // namespace

extern "C" {

int llmx_profile(const char *name, llmx_shape *out) {
    if (!name || !out) return LLMX_ERR_ARG;
    struct P {
        const char *n;
        llmx_shape s;
    };
    static const P table[] = {
        {"small", {64, 64, 128, 2, 4, 2, 32}},
        {"medium", {128, 128, 256, 2, 4, 2, 64}},
        {"qwen-layer", {128, 2048, 11008, 1, 16, 2, 96}},
        {"qwen-layer-long", {128, 2048, 11008, 1, 16, 2, 2048}},
        {"qwen2.5-3b", {151936, 2048, 11008, 36, 16, 2, 2048}},
    };
    for (const auto &p : table)
        if (std::strcmp(p.n, name) == 0) {
            *out = p.s;
            return LLMX_OK;
        }
    return LLMX_ERR_ARG;
}

int llmx_shape_validate(const llmx_shape *s) {
    if (!s) return LLMX_ERR_ARG;
    if (s->hidden <= 0 || s->inter <= 0 || s->layers <= 0 || s->heads <= 0 || s->kv_heads <= 0 ||
        s->max_seq <= 0 || s->vocab <= 0)
        return LLMX_ERR_ARG;
    if (s->hidden % s->heads || s->heads % s->kv_heads) return LLMX_ERR_ARG;
    const int hd = s->hidden / s->heads;
    // model_shape_t::validate host:224-236 (even head_dim, GQA group <= 8), plus the
    // kernels' limits: 128-bit rows (multiples of 8 features), head_dim a multiple
    // of 8 and <= 128.
    if (hd % 8 || hd > 128 || s->heads / s->kv_heads > 8) return LLMX_ERR_UNSUPPORTED;
    if (s->hidden % 8 || s->inter % 8) return LLMX_ERR_UNSUPPORTED;
    // one attention cluster (8 CTAs x 5 tiles of 64) covers the context
    if (s->max_seq > 8 * 5 * 64) return LLMX_ERR_UNSUPPORTED;
    return LLMX_OK;
}

int llmx_validate_task(const llmx_shape *s, uint32_t op, uint32_t layer, uint32_t position, uint32_t rows,
                       llmx_status *st) {
    return validate_op(s, op, layer, position, rows, st, false);
}

int llmx_validate_operator(const llmx_shape *s, uint32_t op, uint32_t layer, uint32_t position, uint32_t rows,
                           llmx_status *st) {
    return validate_op(s, op, layer, position, rows, st, true);
}

int llmx_feature_dims(const llmx_shape *s, uint32_t op, uint32_t *in_dim, uint32_t *out_dim, int *needs_rhs) {
    if (!s || !in_dim || !out_dim || !needs_rhs) return LLMX_ERR_ARG;
    const uint32_t H = s->hidden, I = s->inter, KV = (uint32_t)s->kv_heads * (s->hidden / s->heads);
    // feature_input_dim / feature_output_dim / needs_rhs host:2015-2061
    switch (op) {
    case LLMX_OP_Q_PROJECTION: *in_dim = H, *out_dim = H; break;
    case LLMX_OP_K_PROJECTION:
    case LLMX_OP_V_PROJECTION: *in_dim = H, *out_dim = KV; break;
    case LLMX_OP_O_PROJECTION: *in_dim = H, *out_dim = H; break;
    case LLMX_OP_FFN_GATE:
    case LLMX_OP_FFN_UP: *in_dim = H, *out_dim = I; break;
    case LLMX_OP_FFN_DOWN: *in_dim = I, *out_dim = H; break;
    case LLMX_OP_RMSNORM:
    case LLMX_OP_RESIDUAL_ADD: *in_dim = H, *out_dim = H; break;
    case LLMX_OP_SILU_MUL: *in_dim = I, *out_dim = I; break;
    default: return LLMX_ERR_ARG;  // "operator is not a feature operator"
    }
    *needs_rhs = op == LLMX_OP_RMSNORM || op == LLMX_OP_SILU_MUL || op == LLMX_OP_RESIDUAL_ADD;
    return LLMX_OK;
}

const char *llmx_strerror(int code) {
    switch (code) {
    case LLMX_OK: return "ok";
    case LLMX_BAD_OPERATOR: return "bad operator";
    case LLMX_BAD_TOKEN_COUNT: return "bad token count";
    case LLMX_BAD_TILE_LENGTH: return "bad tile length";
    case LLMX_BAD_POSITION: return "bad position";
    case LLMX_BAD_LAYER: return "bad layer";
    case LLMX_ERR_CUDA: return "CUDA runtime error";
    case LLMX_ERR_ARG: return "invalid argument";
    case LLMX_ERR_STATE: return "invalid state";
    case LLMX_ERR_NCCL: return "NCCL error";
    case LLMX_ERR_RANGE: return "value out of supported range";
    case LLMX_ERR_NOMEM: return "out of memory";
    case LLMX_ERR_IO: return "checkpoint file missing or wrong size";
    case LLMX_ERR_UNSUPPORTED: return "unsupported shape";
    case LLMX_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown error";
    }
}

// Constant tables, exported for the CPU tests that compare them with the oracle.
int llmx_exp_tables(int16_t *e16_8, int16_t *p18_4) {
    if (!e16_8 || !p18_4) return LLMX_ERR_ARG;
    build_exp_tables(e16_8, p18_4);
    return LLMX_OK;
}
int llmx_rope_table(int head_dim, int max_seq, int16_t *table) {
    if (!table || head_dim <= 0 || head_dim % 2 || max_seq <= 0) return LLMX_ERR_ARG;
    build_rope_table(head_dim, max_seq, table);
    return LLMX_OK;
}

}  // extern "C"
