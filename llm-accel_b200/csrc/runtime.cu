// Device context of the resident decoder-layer path: accelerator_t
// (host/host_qwen_8x64.cpp:1024-3087) rebuilt around one CUDA stream, HBM-
// resident weights / KV cache / hidden ping-pong buffers, and one CUDA graph per
// decoder stack (2L+1 coarse tasks) instead of per-task XRT enqueues.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "fixed.cuh"
#include "host_model.h"
#include "kernels.cuh"
#include "stream_watch.h"

using namespace llmx;

namespace {

thread_local std::string g_last_error;

int fail_cuda(cudaError_t e, const char *what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return LLMX_ERR_CUDA;
}

#define CK(call)                                          \
    do {                                                  \
        cudaError_t e_ = (call);                          \
        if (e_ != cudaSuccess) return fail_cuda(e_, #call); \
    } while (0)

#define CKN(call)                                                             \
    do {                                                                      \
        ncclResult_t r_ = (call);                                             \
        if (r_ != ncclSuccess) {                                              \
            g_last_error = std::string(#call) + ": " + ncclGetErrorString(r_); \
            return LLMX_ERR_NCCL;                                             \
        }                                                                     \
    } while (0)

__global__ void k_set_step(Step *dst, int32_t position, int32_t rows, uint32_t ar_base LLMX_TL_PARAM) {
    LLMX_TL_GUARD(tl_slot);
    asm volatile("griddepcontrol.launch_dependents;");
    dst->position = position;
    dst->rows = rows;
    dst->ar_base = ar_base;
}

int rows_template(uint32_t rows) { return rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8; }

}  // namespace

void llmx::set_last_error(const std::string &msg) { g_last_error = msg; }

// Geometry of one projection in the tensor-core item layout.
struct MmaGeom {
    int T = 0, C = 0, K = 0, n_out = 0;
    size_t offset = 0;  // bytes from the start of the layer's item blob
    size_t wsum_offset = 0;  // int32 entries from the start of the layer's weight-sum tables (T*(C+1)*128)
    size_t items() const { return (size_t)T * C; }
};

struct llmx_ctx {
    llmx_shape s{};
    int dev = 0, rank = 0, size = 1, nsm = 148;
    ncclComm_t comm = nullptr;
    // NCCL waits of this rank: deadline (LLMX_NCCL_TIMEOUT_MS) and whether the
    // communicator was aborted (the context then refuses further work)
    int nccl_timeout_ms = 60000;
    bool comm_failed = false;
    cudaStream_t stream = nullptr;
    // geometry of this rank
    int hd = 0, G = 0, KV = 0, hq = 0, h0 = 0, Hq = 0, Il = 0, c0 = 0, tpc_max = 0;
    // 16-CTA attention clusters when rows x local heads x 16 CTAs fit in one wave
    // and the context can exceed 16 tiles (tensor-parallel ranks of 8, 4 or 2
    // heads; measured at context 2049 with 4 heads: 14.5 -> 11.0 us; 16 heads,
    // 256 CTAs, oversubscribe the SMs and stay on 8-CTA clusters)
    int tpc_max_wide = 0;
    bool attn_wide = false;
    int attn_rows_min = 2;  // blocks of at least this many rows use the all-rows attention kernel (LLMX_ATTN_ROWS_MIN)
    bool attn_rows_wide = false;  // all-rows kernel on 16-CTA clusters (LLMX_ATTN_ROWS_WIDE)
    int attn_wide_div = 1;  // wide clusters while rows x heads x 16 CTAs <= SMs / div (LLMX_ATTN_WIDE_DIV)
    // weights: per layer [QKV | O | GU | D] words
    size_t w_qkv = 0, w_o = 0, w_gu = 0, w_d = 0, layer_words = 0;
    uint32_t *wbuf = nullptr;
    int16_t *staging = nullptr;
    int32_t *slot_qkv = nullptr, *slot_o = nullptr, *slot_gu = nullptr, *slot_d = nullptr;
    int16_t *norms = nullptr, *rope = nullptr, *etab = nullptr, *ptab = nullptr;
    int16_t *kc = nullptr, *vc = nullptr;
    // hidden pairs 0 and 1 (bound by the caller) and 2, the sublayer boundary of
    // the full-layer Task 16 (the input pair stays unchanged)
    int16_t *hid[3] = {nullptr, nullptr, nullptr};
    int16_t *q = nullptr, *att = nullptr, *act = nullptr;
    int64_t *partial = nullptr;
    // one-row attention with the O projection fused (single GPU, LLMX_ATTN_FUSE_O):
    // the exact O sums [kMaxRows][hidden], finished by the next kernel's prologue
    bool fuse_o = true;
    // the fused kernel's split variant (LLMX_ATTN_SPLIT_O=1; off by default):
    // O slice copied from the start, no head-output exchange
    bool attn_split_o = false;
    // tensor-parallel ranks: O fused into one-row attention with the peer push
    // (LLMX_ATTN_FUSE_O_TP=1; off by default); o_cnt counts the heads done per
    // [row][cluster CTA] slice of O rows
    bool fuse_o_tp = false;
    int *o_cnt = nullptr;
    // blocks of several rows: the row-inner loop order of the rows kernel
    // (LLMX_ATTN_ROWS_INNER=1; off by default)
    bool attn_rows_inner = false;
    int64_t *o_acc = nullptr;
    // the O weights once more, head-major ([head][hidden rows][hd/2] words per
    // layer), so that a fused-attention CTA's slice is one contiguous copy
    uint32_t *o_heads = nullptr;
    Step *step = nullptr;
    int *err = nullptr;
    // pinned host copy of *err, read on the stream together with a call's results
    // (null when pinned memory was not available: then read with a blocking copy)
    int *err_host = nullptr;
    int ring_kb = 96, ring_wide_kb = 176, ring_gu_kb = 160, gemv_ctas_per_sm = 1;
    int gemv_warps = 16;  // consumer warps of a projection CTA at most (LLMX_GEMV_WARPS)
    // preferred shared-memory carveout of the projection kernels in percent
    // (LLMX_PROJ_CARVEOUT, -1: the driver's choice). Maximum shared memory measured
    // on B200: prefill 2582 -> 2598 tok/s, decode 690 -> 692
    int proj_carveout = 100;
    // L2 warm-up during attention of stacks of at most attn_pf_rows rows: attn_pf_tile_kb
    // KiB per 64-position context tile from the layer's O weights on, at most
    // attn_pf_kb KiB and the end of Gate/Up (LLMX_ATTN_PREFETCH_TILE_KB, _KB, _ROWS).
    // Measured on B200: ~33 MiB best at context ~600, ~70 MiB at ~2200 (98 MiB
    // slower); no gain at 8 rows.
    int attn_pf_tile_kb = 3584, attn_pf_kb = 72 * 1024, attn_pf_rows = 2;
    int attn_pf_late = 1;  // after attention's K/V loads (LLMX_ATTN_PREFETCH_LATE=0: at kernel start)
    // one-row attention triggers the next kernel's launch at its start above this
    // context (64-position tiles), else once PV is done (LLMX_ATTN_TRIGGER_TILES;
    // measured: late +2.2 % at 9 tiles, early +2.2 % at 33)
    int attn_trigger_tiles = 16;
    // peer all-reduce (tensor parallel): exchange regions of every rank (IPC-mapped)
    ArPeers ar{};
    char *ar_region = nullptr;
    std::vector<char *> ar_opened;
    // all-reduces enqueued so far (the same count on every rank); a call's first
    // all-reduce number reaches the kernels in the step record
    uint32_t ar_count = 0;
    char *probe_region = nullptr;  // llmx_selftest_ar_timeout: an exchange region nobody writes
    // blocks of at most this many rows finish a peer all-reduce in the next
    // projection's prologue (every CTA reads all rows' words); larger blocks
    // use the finishing kernel once (LLMX_AR_FUSE_ROWS)
    int ar_fuse_rows = 2;
    // tensor-core projections (mma_proj.cu) for blocks of at least mma_min_rows
    // rows: a second copy of every layer's weights in item layout, stream-K
    // scratch and tile counters (LLMX_MMA=0 disables, LLMX_MMA_MIN_ROWS)
    bool mma = false;
    int mma_min_rows = 3;
    // projections on the tensor cores: bits MP_QKV, MP_O, MP_GU, MP_D (LLMX_MMA_PROJ).
    // Default Gate/Up + Down: measured on B200 at 8 rows, Gate/Up 26.5 vs 39.0 us and
    // Down 18.3 vs 31.0 us on the tensor cores, while QKV (11.2 vs 10.0) and O (12.0
    // vs 5.9) are latency bound and stay on the dp2a kernel
    int mma_proj = 0xC;
    MmaGeom mg[4]{};             // QKV, O, Gate/Up, Down of this rank
    size_t mma_layer_bytes = 0;
    uint8_t *mbuf = nullptr;
    int32_t *mma_wsum = nullptr;  // per layer: the projections' weight-sum prefix tables
    size_t mma_wsum_layer = 0;    // int32 entries per layer
    int64_t *mma_scratch = nullptr;
    int *mma_cnt = nullptr;
    int32_t *mma_rows[4] = {nullptr, nullptr, nullptr, nullptr};
    int32_t inv_elems = 0, inv_rms_const = 0, qk_scale = 0;
    uint32_t out_pair = 0, in_pair = 1;
    // per-operator (feature) calls: operand rows and exact sums, allocated on first use
    int16_t *feat_lhs = nullptr, *feat_rhs = nullptr, *feat_out = nullptr;
    int64_t *feat_sums = nullptr;
    std::vector<bool> layer_loaded;
    bool norms_loaded = false;
    uint64_t launches = 0, last_launches = 0, device_bytes = 0;
    std::map<std::tuple<uint32_t, uint32_t, uint32_t, int>, std::pair<cudaGraphExec_t, uint64_t>> graphs;
    std::vector<void *> allocations;
    // device generate loop: vocabulary tables, argmax scratch, token ids by position
    int16_t *emb_dev = nullptr, *head_dev = nullptr, *gen_rows = nullptr;
    void *lm_scratch = nullptr;
    uint32_t *tok_dev = nullptr;
    bool vocab_loaded = false;
};

namespace {

template <typename T>
int dalloc(llmx_ctx *c, T **p, size_t count) {
    void *v = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess) {
        g_last_error = std::string("cudaMalloc: ") + cudaGetErrorString(e);
        return LLMX_ERR_NOMEM;
    }
    CK(cudaMemset(v, 0, bytes));
    c->allocations.push_back(v);
    c->device_bytes += bytes;
    *p = static_cast<T *>(v);
    return LLMX_OK;
}

// Wait for everything enqueued on the context stream. While the stream can hold
// NCCL collectives (the set-up exchange, the NCCL all-reduce path) the rank waits
// with a deadline and watches its communicator: on expiry or an asynchronous
// error the communicator is aborted, which ends its kernels, and the context
// refuses further work. The peer all-reduce kernels bound their own waits.
int stream_wait(llmx_ctx *c) {
    if (!c->comm || c->ar.n > 1) {
        CK(cudaStreamSynchronize(c->stream));
        return LLMX_OK;
    }
    cudaError_t qerr = cudaSuccess;
    ncclResult_t aerr = ncclSuccess;
    const WatchOutcome w = watch_stream(
        [&] {
            qerr = cudaStreamQuery(c->stream);
            return qerr == cudaSuccess ? 0 : qerr == cudaErrorNotReady ? 1 : -1;
        },
        [&] { return ncclCommGetAsyncError(c->comm, &aerr) != ncclSuccess || aerr != ncclSuccess; },
        [&] {
            ncclCommAbort(c->comm);
            c->comm = nullptr;
            c->comm_failed = true;
        },
        [] {
            return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch())
                .count();
        },
        (double)c->nccl_timeout_ms);
    switch (w) {
    case kWatchDone: return LLMX_OK;
    case kWatchStreamError: return fail_cuda(qerr, "cudaStreamQuery");
    case kWatchCommError:
        g_last_error = std::string("NCCL asynchronous error: ") + ncclGetErrorString(aerr) + "; communicator aborted";
        return LLMX_ERR_NCCL;
    default:
        g_last_error = "collective still pending after " + std::to_string(c->nccl_timeout_ms) +
                       " ms (LLMX_NCCL_TIMEOUT_MS); communicator aborted";
        return LLMX_ERR_TIMEOUT;
    }
}

#define SYNC(c)                          \
    do {                                 \
        int rc_ = stream_wait(c);        \
        if (rc_ != LLMX_OK) return rc_;  \
    } while (0)

int16_t *kc_layer(const llmx_ctx *c, uint32_t layer) {
    return c->kc + (size_t)layer * c->s.kv_heads * c->s.max_seq * c->hd;
}
int16_t *vc_layer(const llmx_ctx *c, uint32_t layer) {
    return c->vc + (size_t)layer * c->s.kv_heads * c->s.max_seq * c->hd;
}
const uint32_t *wl(const llmx_ctx *c, uint32_t layer) { return c->wbuf + (size_t)layer * c->layer_words; }

constexpr int kProjSmem = 225 * 1024;  // 227 KiB per CTA minus the kernels' static shared memory

// Persistent projection CTAs: gemv_ctas_per_sm per SM (LLMX_GEMV_CTAS_PER_SM),
// each streaming through a ring of about ring_kb KiB (LLMX_RING_KB; LLMX_RING_WIDE_KB
// for the FFN-wide Down projection, LLMX_RING_GU_KB for Gate/Up).
int grid_for(llmx_ctx *c, int npairs, int rt, int K) {
    (void)rt;
    (void)K;
    return std::max(1, std::min(c->nsm * c->gemv_ctas_per_sm, npairs));
}

void set_stages(llmx_ctx *c, ProjArgs &a, int epi, int rt) {
    const int smem = kProjSmem / c->gemv_ctas_per_sm - 1024;
    // FFN-wide inputs (the Down projection) may take their own ring size
    const int ring = a.K > 4 * c->s.hidden ? c->ring_wide_kb : (epi == EPI_SILU ? c->ring_gu_kb : c->ring_kb);
    a.stages = gemv_stages(rt, epi, a.K, smem, ring * 1024, &a.units_per_chunk, &a.parts, c->gemv_warps);
    a.error = c->err;
}

int env_int(const char *name, int def, int lo, int hi) {
    const char *v = std::getenv(name);
    if (!v || !*v) return def;
    const int x = std::atoi(v);
    return x < lo ? lo : (x > hi ? hi : x);
}

// All-reduce `ar_off` of the call as a kernel of its own: wait for every rank's
// sums, add, round, + residual (peer path); or NCCL + the rounding kernel.
int allreduce_resid(llmx_ctx *c, uint32_t rows, uint32_t ar_off, int16_t *out, const int16_t *resid) {
    if (c->ar.n > 1) {  // the projection pushed its sums to every rank: wait, add, round
        ArFinishArgs f{c->ar, ar_off, resid, out, c->step, c->err};
        CK(launch_ar_finish(f, c->stream));
        c->launches += 1;
        return LLMX_OK;
    }
    CKN(ncclAllReduce(c->partial, c->partial, (size_t)rows * c->s.hidden, ncclInt64, ncclSum, c->comm,
                      c->stream));
    ResidArgs r{c->partial, resid, out, c->s.hidden, c->step, nullptr};
    CK(launch_round_resid(r, (int)rows, c->stream));
    c->launches += 1;
    return LLMX_OK;
}

// Kernel-level pieces of the coarse tasks (ids of LLMX_KERNEL_*).
ProjArgs qkv_args(llmx_ctx *c, uint32_t layer, const int16_t *in) {
    const llmx_shape &s = c->s;
    ProjArgs a{};
    a.w = wl(c, layer);
    a.K = s.hidden;
    a.npairs = (c->Hq + 2 * c->KV) / 2;
    a.x = in;
    a.norm = c->norms + (size_t)2 * layer * s.hidden;
    a.inv_elems = c->inv_elems;
    a.inv_rms_const = c->inv_rms_const;
    a.step = c->step;
    a.out = c->q;
    a.out_stride = c->Hq;
    a.kc = kc_layer(c, layer);
    a.vc = vc_layer(c, layer);
    a.rope = c->rope;
    a.hd = c->hd;
    a.q_pairs = c->Hq / 2;
    a.kv_pairs = c->KV / 2;
    a.max_seq = s.max_seq;
    return a;
}

AttnArgs attn_args(llmx_ctx *c, uint32_t layer) {
    AttnArgs t{};
    t.q = c->q;
    t.kc = kc_layer(c, layer);
    t.vc = vc_layer(c, layer);
    t.out = c->att;
    t.ptab = c->ptab;
    t.step = c->step;
    t.q_heads = c->hq;
    t.first_head = c->h0;
    t.gqa = c->G;
    t.hd = c->hd;
    t.max_seq = c->s.max_seq;
    t.tpc_max = c->tpc_max;
    t.cluster = kCluster;
    t.qk_scale = c->qk_scale;
    t.error = c->err;
    t.trigger_tiles = c->attn_trigger_tiles;
    // O then Gate/Up follow the QKV words of the layer blob
    t.pf = reinterpret_cast<const char *>(wl(c, layer) + c->w_qkv);
    t.pf_bytes = (c->w_o + c->w_gu) * 4ull;
    if (c->attn_pf_kb) t.pf_bytes = std::min<unsigned long long>(t.pf_bytes, (unsigned long long)c->attn_pf_kb << 10);
    t.pf_per_tile = (unsigned long long)c->attn_pf_tile_kb << 10;
    t.pf_late = c->attn_pf_late;
    return t;
}

// Attention of a block: the per-(row, head) kernel, or for blocks of at least
// attn_rows_min rows one cluster per head covering every row.
cudaError_t launch_attention(llmx_ctx *c, AttnArgs t, uint32_t rows);

// One-row attention with the O projection fused: single GPU, the per-(row, head)
// kernel, and Gate/Up + Down on the dp2a kernel (whose prologue / clearing
// finish the sums).
bool use_fuse_o(const llmx_ctx *c, uint32_t rows);
void set_fuse_o(llmx_ctx *c, AttnArgs &t, uint32_t layer);

// Cluster size of an attention launch of `rows` rows.
void pick_attn_cluster(const llmx_ctx *c, AttnArgs &t, uint32_t rows) {
    if (c->attn_wide && c->attn_wide_div * (int)rows * c->hq * kClusterWide <= c->nsm) {
        t.cluster = kClusterWide;
        t.tpc_max = c->tpc_max_wide;
    }
}

cudaError_t launch_attention(llmx_ctx *c, AttnArgs t, uint32_t rows) {
    if ((int)rows >= c->attn_rows_min) {
        t.pf_per_tile = 0;
        t.rows_inner = c->attn_rows_inner ? 1 : 0;
        if (c->attn_rows_wide) {  // 16 CTAs per head: the block's rows multiply each CTA's work
            t.cluster = kClusterWide;
            t.tpc_max = c->tpc_max_wide;
        }
        return launch_attn_rows(t, c->stream);
    }
    pick_attn_cluster(c, t, rows);
    if (t.o_w != nullptr) t.o_rows = t.hidden / t.cluster;  // O rows per CTA of the chosen cluster
    if (rows > (uint32_t)c->attn_pf_rows) t.pf_per_tile = 0;
    return launch_attn(t, (int)rows, c->stream);
}

ProjArgs o_args(llmx_ctx *c, uint32_t layer, int16_t *out, const int16_t *in) {
    ProjArgs o{};
    o.w = wl(c, layer) + c->w_qkv;
    o.K = c->Hq;
    o.npairs = c->s.hidden / 2;
    o.x = c->att;
    o.step = c->step;
    o.out = out;
    o.out_stride = c->s.hidden;
    o.resid = in;
    o.partial = c->partial;
    o.ar = c->ar;
    return o;
}

ProjArgs gu_args(llmx_ctx *c, uint32_t layer, const int16_t *in) {
    const llmx_shape &s = c->s;
    ProjArgs g{};
    g.w = wl(c, layer) + c->w_qkv + c->w_o;
    g.K = s.hidden;
    g.npairs = c->Il;
    g.x = in;
    g.norm = c->norms + (size_t)(2 * layer + 1) * s.hidden;
    g.inv_elems = c->inv_elems;
    g.inv_rms_const = c->inv_rms_const;
    g.step = c->step;
    g.out = c->act;
    g.out_stride = c->Il;
    g.etab = c->etab;
    return g;
}

ProjArgs down_args(llmx_ctx *c, uint32_t layer, int16_t *out, const int16_t *in) {
    ProjArgs d{};
    d.w = wl(c, layer) + c->w_qkv + c->w_o + c->w_gu;
    d.K = c->Il;
    d.npairs = c->s.hidden / 2;
    d.x = c->act;
    d.step = c->step;
    d.out = out;
    d.out_stride = c->s.hidden;
    d.resid = in;
    d.partial = c->partial;
    d.ar = c->ar;
    return d;
}

enum { MP_QKV = 0, MP_O = 1, MP_GU = 2, MP_D = 3 };

bool use_mma(const llmx_ctx *c, uint32_t rows, int proj) {
    return c->mma && (int)rows >= c->mma_min_rows && ((c->mma_proj >> proj) & 1);
}

bool use_fuse_o(const llmx_ctx *c, uint32_t rows) {
    // tensor parallel: only with the peer all-reduce (the NCCL path reduces the O projection's partials)
    return c->fuse_o && (c->size == 1 || c->ar.n > 1) && rows == 1 && (int)rows < c->attn_rows_min && c->s.hidden % kClusterWide == 0 &&
           !use_mma(c, rows, MP_GU) &&
           !use_mma(c, rows, MP_D);
}

void set_fuse_o(llmx_ctx *c, AttnArgs &t, uint32_t layer) {
    t.o_w = c->o_heads + (size_t)layer * c->w_o;
    t.split_o = c->attn_split_o ? 1 : 0;
    t.o_rows = c->s.hidden / t.cluster;
    t.hidden = c->s.hidden;
    t.o_acc = c->o_acc;
    // the L2 warm-up starts after the O weights, which this kernel reads itself
    const unsigned long long o_bytes = c->w_o * 4ull;
    t.pf += o_bytes;
    t.pf_bytes = t.pf_bytes > o_bytes ? t.pf_bytes - o_bytes : 0;
}


// Exact sums whose rounding (+ residual) is still to come: a peer all-reduce
// (its number within the call), or the fused attention's O sums (local); the
// residual to add and where the finished rows belong.
struct PendingAr {
    bool active = false;
    bool local = false;
    uint32_t off = 0;
    const int16_t *resid = nullptr;
    int16_t *out = nullptr;
};

// Route a projection's activation input through pending sums (the projection's
// prologue finishes them).
void take_input(llmx_ctx *c, ProjArgs &a, PendingAr &pend) {
    if (!pend.active) return;
    if (pend.local) {
        a.in.sums = c->o_acc;
    } else {
        a.in.ar = c->ar;
        a.in.ar_off = pend.off;
    }
    a.in.resid = pend.resid;
    a.in.hid_out = pend.out;
    pend.active = pend.local = false;
}

// The fused attention's O sums as a kernel of their own: round, + residual,
// clear the sums.
int finish_o_sums(llmx_ctx *c, uint32_t rows, int16_t *out, const int16_t *resid) {
    ResidArgs r{c->o_acc, resid, out, c->s.hidden, c->step, c->o_acc};
    CK(launch_round_resid(r, (int)rows, c->stream));
    c->launches += 1;
    return LLMX_OK;
}

// After a tensor-parallel O / Down projection: leave the all-reduce pending for
// the next projection (peer path inside a stack) or finish it now.
int after_partial(llmx_ctx *c, uint32_t rows, uint32_t &ar_next, int16_t *out, const int16_t *resid, bool fuse,
                  PendingAr &pend) {
    const uint32_t off = ar_next++;
    if (fuse && c->ar.n > 1 && (int)rows <= c->ar_fuse_rows && !use_mma(c, rows, MP_QKV) && !use_mma(c, rows, MP_GU)) {
        pend.active = true;
        pend.off = off;
        pend.resid = resid;
        pend.out = out;
        return LLMX_OK;
    }
    return allreduce_resid(c, rows, off, out, resid);
}

// A projection on the tensor cores (mma_proj.cu); the dp2a arguments p carry
// the epilogue's operands (inputs, outputs, residual, caches, tables).
int launch_mma(llmx_ctx *c, const ProjArgs &p, int proj, uint32_t layer, int epi) {
    const MmaGeom &g = c->mg[proj];
    MmaArgs m{};
    m.w = c->mbuf + (size_t)layer * c->mma_layer_bytes + g.offset;
    m.K = g.K;
    m.C = g.C;
    m.T = g.T;
    m.n_out = g.n_out;
    m.x = p.x;
    m.norm = p.norm;
    m.inv_elems = p.inv_elems;
    m.inv_rms_const = p.inv_rms_const;
    m.step = c->step;
    m.out = p.out;
    m.out_stride = p.out_stride;
    m.resid = p.resid;
    m.partial = p.partial;
    m.etab = p.etab;
    m.kc = p.kc;
    m.vc = p.vc;
    m.rope = p.rope;
    m.q_tiles = c->hq;
    m.kv_tiles = c->s.kv_heads;
    m.max_seq = c->s.max_seq;
    m.ar = p.ar;
    m.ar_off = p.ar_off;
    m.scratch = c->mma_scratch;
    m.tile_cnt = c->mma_cnt;
    m.error = c->err;
    m.wsum = c->mma_wsum + (size_t)layer * c->mma_wsum_layer + g.wsum_offset;
    const int items = (int)g.items();
    const int grid = std::min(c->nsm, items);
    m.max_items = (items + grid - 1) / grid;
    m.stages = mma_stages(m.max_items, kProjSmem);
    if (m.stages < 2) {
        g_last_error = "tensor-core projection: the item ring does not fit shared memory";
        return LLMX_ERR_UNSUPPORTED;
    }
    CK(launch_mma_proj(m, epi, grid, c->stream));
    return LLMX_OK;
}

// Enqueue the kernels of one coarse task on the context stream.  ar_next counts
// the call's all-reduces; with `fuse` (stacks) the finishing step of a peer
// all-reduce moves into the next projection's prologue (pend).
int enqueue_task(llmx_ctx *c, uint32_t op, uint32_t layer, uint32_t rows, uint32_t in_pair,
                 uint32_t out_pair, uint32_t &ar_next, bool fuse, PendingAr &pend) {
    const llmx_shape &s = c->s;
    const int rt = rows_template(rows);
    const int16_t *in = c->hid[in_pair];
    int16_t *out = c->hid[out_pair];
    const int ge = c->size > 1 ? EPI_PARTIAL : EPI_RESID;
    if (op == LLMX_OP_DECODER_LAYER) {  // Task 18 into pair 2, then Task 19 from it
        int rc = enqueue_task(c, LLMX_OP_ATTENTION_SUBLAYER, layer, rows, in_pair, 2, ar_next, fuse, pend);
        if (!rc) rc = enqueue_task(c, LLMX_OP_FFN_SUBLAYER, layer, rows, 2, out_pair, ar_next, fuse, pend);
        return rc;
    }
    if (op == LLMX_OP_ATTENTION_SUBLAYER) {
        ProjArgs a = qkv_args(c, layer, in);
        take_input(c, a, pend);
        if (use_mma(c, rows, MP_QKV)) {
            const int rc = launch_mma(c, a, MP_QKV, layer, EPI_QKV);
            if (rc) return rc;
        } else {
            set_stages(c, a, EPI_QKV, rt);
            CK(launch_proj(a, EPI_QKV, rt, grid_for(c, a.npairs, rt, a.K), c->stream));
        }
        AttnArgs t = attn_args(c, layer);
        if (use_fuse_o(c, rows)) {  // O inside attention; the next prologue (or a finisher) rounds
            set_fuse_o(c, t, layer);
            if (c->size > 1) {  // the last head of each O-row slice pushes the rank's sums to every rank
                t.ar = c->ar;
                t.ar_off = ar_next;
                t.o_cnt = c->o_cnt;
                CK(launch_attention(c, t, rows));
                c->launches += 2;
                return after_partial(c, rows, ar_next, out, in, fuse, pend);
            }
            CK(launch_attention(c, t, rows));
            c->launches += 2;
            if (fuse) {
                pend.active = pend.local = true;
                pend.resid = in;
                pend.out = out;
                return LLMX_OK;
            }
            return finish_o_sums(c, rows, out, in);
        }
        CK(launch_attention(c, t, rows));
        ProjArgs o = o_args(c, layer, out, in);
        o.ar_off = ar_next;
        if (use_mma(c, rows, MP_O)) {
            const int rc = launch_mma(c, o, MP_O, layer, ge);
            if (rc) return rc;
        } else {
            set_stages(c, o, ge, rt);
            CK(launch_proj(o, ge, rt, grid_for(c, o.npairs, rt, o.K), c->stream));
        }
        c->launches += 3;
        if (c->size > 1) return after_partial(c, rows, ar_next, out, in, fuse, pend);
        return LLMX_OK;
    }
    if (op == LLMX_OP_FFN_SUBLAYER) {
        ProjArgs g = gu_args(c, layer, in);
        take_input(c, g, pend);
        ProjArgs d = down_args(c, layer, out, in);
        d.ar_off = ar_next;
        if (g.in.sums != nullptr) {  // Gate/Up finished the fused O sums: Down clears them
            d.zero = c->o_acc;
            d.zero_n = (int)rows * s.hidden;
        }
        if (use_mma(c, rows, MP_GU)) {
            const int rc = launch_mma(c, g, MP_GU, layer, EPI_SILU);
            if (rc) return rc;
        } else {
            set_stages(c, g, EPI_SILU, rt);
            CK(launch_proj(g, EPI_SILU, rt, grid_for(c, g.npairs, rt, g.K), c->stream));
        }
        if (use_mma(c, rows, MP_D)) {
            const int rc = launch_mma(c, d, MP_D, layer, ge);
            if (rc) return rc;
            c->launches += 2;
        } else if (rt == 8 && c->size == 1) {
            // an 8-row block as two 4-row launches: 8 FFN-wide activation rows would
            // fill shared memory and starve the weight ring; 4 rows leave it room
            for (int half = 0; half < 2; half++) {
                ProjArgs h = d;
                h.row0 = 4 * half;
                h.x += (size_t)h.row0 * c->Il;
                h.out += (size_t)h.row0 * c->s.hidden;
                h.resid += (size_t)h.row0 * c->s.hidden;
                set_stages(c, h, ge, 4);
                CK(launch_proj(h, ge, 4, grid_for(c, h.npairs, 4, h.K), c->stream));
            }
            c->launches += 3;
        } else {
            set_stages(c, d, ge, rt);
            CK(launch_proj(d, ge, rt, grid_for(c, d.npairs, rt, d.K), c->stream));
            c->launches += 2;
        }
        if (c->size > 1) return after_partial(c, rows, ar_next, out, in, fuse, pend);
        return LLMX_OK;
    }
    if (op == LLMX_OP_FINAL_NORM) {
        NormArgs n{in, c->norms + (size_t)2 * s.layers * s.hidden, out, s.hidden, c->inv_elems,
                   c->inv_rms_const, c->step};
        CK(launch_rmsnorm(n, (int)rows, c->stream));
        c->launches += 1;
        return LLMX_OK;
    }
    return LLMX_OK;  // NOP
}

// All-reduces of one coarse task / one stack (tensor parallel).
uint32_t task_allreduces(const llmx_ctx *c, uint32_t op) {
    if (c->size == 1) return 0u;
    if (op == LLMX_OP_DECODER_LAYER) return 2u;
    return op == LLMX_OP_ATTENTION_SUBLAYER || op == LLMX_OP_FFN_SUBLAYER ? 1u : 0u;
}
uint32_t stack_allreduces(const llmx_ctx *c, uint32_t layer_count) { return c->size > 1 ? 2u * layer_count : 0u; }

int set_step(llmx_ctx *c, uint32_t position, uint32_t rows) {
    k_set_step<<<1, 1, 0, c->stream>>>(c->step, (int32_t)position, (int32_t)rows, c->ar_count LLMX_TL_ARG("set_step"));
    CK(cudaGetLastError());
    c->launches += 1;
    return LLMX_OK;
}

// Kernels record an expired bounded wait in c->err; report (v = the value read)
// and clear it.
int report_device_error(llmx_ctx *c, int v) {
    if (v != 0) {
        CK(cudaMemset(c->err, 0, sizeof(int)));
        // a call that stopped part-way may leave fused-O sums (and head counts) behind
        CK(cudaMemset(c->o_acc, 0, sizeof(int64_t) * kMaxRows * c->s.hidden));
        if (c->o_cnt) CK(cudaMemset(c->o_cnt, 0, sizeof(int) * kMaxRows * kClusterWide));
        if (v == kErrTokenRange) {
            g_last_error = "a token id reached the embedding gather outside the vocabulary";
            return LLMX_ERR_RANGE;
        }
        g_last_error = "a kernel's bounded wait expired (code " + std::to_string(v) + ")";
        return LLMX_ERR_TIMEOUT;
    }
    return LLMX_OK;
}

// End of a synchronous call: the device error word is copied on the stream
// behind the call's work, so one stream wait covers both (no second round trip
// to the device after the wait), then reported.
int finish(llmx_ctx *c) {
    if (c->err_host) CK(cudaMemcpyAsync(c->err_host, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    SYNC(c);
    int v = 0;
    if (c->err_host) v = *c->err_host;
    else CK(cudaMemcpy(&v, c->err, sizeof(int), cudaMemcpyDeviceToHost));
    return report_device_error(c, v);
}

bool model_ready(const llmx_ctx *c, uint32_t layer_begin, uint32_t layer_count) {
    if (c->comm_failed) {
        g_last_error = "the tensor-parallel communicator was aborted; destroy the context";
        return false;
    }
    if (!c->norms_loaded) return false;
    for (uint32_t l = layer_begin; l < layer_begin + layer_count; l++)
        if (!c->layer_loaded[l]) return false;
    return true;
}

// Kernels of a stack, enqueued (graph capture body).
// On the peer all-reduce path each all-reduce is finished by the next
// projection's prologue (Gate/Up after O, the next layer's QKV after Down); only
// the stack's last one runs as a kernel of its own.
int enqueue_stack(llmx_ctx *c, uint32_t rows, uint32_t layer_begin, uint32_t layer_count, int final_norm) {
    uint32_t ar_next = 0;
    PendingAr pend;
    for (uint32_t l = layer_begin; l < layer_begin + layer_count; l++) {
        int rc = enqueue_task(c, LLMX_OP_ATTENTION_SUBLAYER, l, rows, 1, 0, ar_next, true, pend);
        if (rc) return rc;
        rc = enqueue_task(c, LLMX_OP_FFN_SUBLAYER, l, rows, 0, 1, ar_next, true, pend);
        if (rc) return rc;
    }
    if (pend.active) {
        const int rc = pend.local ? finish_o_sums(c, rows, pend.out, pend.resid)
                                  : allreduce_resid(c, rows, pend.off, pend.out, pend.resid);
        if (rc) return rc;
    }
    if (final_norm) return enqueue_task(c, LLMX_OP_FINAL_NORM, 0, rows, 1, 0, ar_next, false, pend);
    return LLMX_OK;
}

int launch_stack_graph(llmx_ctx *c, uint32_t rows, uint32_t layer_begin, uint32_t layer_count, int final_norm) {
    const auto key = std::make_tuple(rows, layer_begin, layer_count, final_norm);
    auto it = c->graphs.find(key);
    if (it == c->graphs.end()) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        const uint64_t before = c->launches;
        const int rc = enqueue_stack(c, rows, layer_begin, layer_count, final_norm);
        cudaError_t e = cudaStreamEndCapture(c->stream, &g);
        if (rc) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return fail_cuda(e, "cudaStreamEndCapture");
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) return fail_cuda(e, "cudaGraphInstantiate");
        it = c->graphs.emplace(key, std::make_pair(exec, c->launches - before)).first;
        c->launches = before;
    }
    CK(cudaGraphLaunch(it->second.first, c->stream));
    c->launches += it->second.second;
    c->ar_count += stack_allreduces(c, layer_count);
    return LLMX_OK;
}

// Step record + the stack (its captured graph).  Arguments already validated.
int launch_stack_at(llmx_ctx *c, uint32_t rows, uint32_t layer_begin, uint32_t layer_count, uint32_t position,
                    int final_norm) {
    int rc = set_step(c, position, rows);
    if (rc) return rc;
    return launch_stack_graph(c, rows, layer_begin, layer_count, final_norm);
}

// Peer all-reduce set-up: one zeroed exchange region per rank, its IPC handle
// all-gathered over NCCL, the other ranks' regions mapped.  Every rank must take
// the same path (a rank on NCCL and one on peer stores would wait on each other
// for good), so the ranks agree over NCCL: the peer path is used only if every
// rank wants it (LLMX_TP_NCCL unset) and mapped every peer region; otherwise
// every rank unmaps what it opened and keeps the NCCL all-reduce.
int setup_peer_allreduce(llmx_ctx *c, bool want_peer) {
    const size_t bytes = kArHeader + (size_t)2 * kMaxTp * kMaxRows * c->s.hidden * sizeof(uint64_t);
    int rc;
    char *hbuf = nullptr;
    int *okbuf = nullptr;
    if ((rc = dalloc(c, &hbuf, (size_t)c->size * sizeof(cudaIpcMemHandle_t))) || (rc = dalloc(c, &okbuf, 1)))
        return rc;
    cudaIpcMemHandle_t mine{};
    int ok = want_peer && c->size <= kMaxTp ? 1 : 0;
    if (ok) {
        if ((rc = dalloc(c, &c->ar_region, bytes))) return rc;
        CK(cudaIpcGetMemHandle(&mine, c->ar_region));
    }
    CK(cudaMemcpy(hbuf + (size_t)c->rank * sizeof(mine), &mine, sizeof(mine), cudaMemcpyHostToDevice));
    CKN(ncclAllGather(hbuf + (size_t)c->rank * sizeof(mine), hbuf, sizeof(mine), ncclChar, c->comm, c->stream));
    SYNC(c);
    std::vector<cudaIpcMemHandle_t> all(c->size);
    CK(cudaMemcpy(all.data(), hbuf, all.size() * sizeof(mine), cudaMemcpyDeviceToHost));
    ArPeers a{};
    for (int p = 0; p < c->size && ok; p++) {
        if (p == c->rank) {
            a.base[p] = c->ar_region;
            continue;
        }
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            (void)cudaGetLastError();
            ok = 0;
            break;
        }
        a.base[p] = static_cast<char *>(ptr);
        c->ar_opened.push_back(a.base[p]);
    }
    CK(cudaMemcpy(okbuf, &ok, sizeof(int), cudaMemcpyHostToDevice));
    CKN(ncclAllReduce(okbuf, okbuf, 1, ncclInt32, ncclMin, c->comm, c->stream));
    SYNC(c);
    CK(cudaMemcpy(&ok, okbuf, sizeof(int), cudaMemcpyDeviceToHost));
    if (!ok) {
        for (char *q : c->ar_opened) cudaIpcCloseMemHandle(q);
        c->ar_opened.clear();
        return LLMX_OK;  // every rank keeps the NCCL all-reduce
    }
    a.n = c->size;
    a.me = c->rank;
    a.hidden = c->s.hidden;
    a.poll_limit = (uint32_t)env_int("LLMX_AR_POLL_LIMIT", 1 << 24, 1, 1 << 30);
    c->ar = a;
    return LLMX_OK;
}

void release(llmx_ctx *c) {
    if (!c) return;
    cudaSetDevice(c->dev);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto &g : c->graphs) cudaGraphExecDestroy(g.second.first);
    c->graphs.clear();
    for (char *p : c->ar_opened) cudaIpcCloseMemHandle(p);
    c->ar_opened.clear();
    if (c->comm) ncclCommDestroy(c->comm);
    for (void *p : c->allocations) cudaFree(p);
    if (c->err_host) cudaFreeHost(c->err_host);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

}  // namespace

extern "C" {

const char *llmx_last_error(void) { return g_last_error.c_str(); }

int llmx_tp_unique_id(void *id128) {
    if (!id128) return LLMX_ERR_ARG;
    ncclUniqueId id;
    CKN(ncclGetUniqueId(&id));
    std::memcpy(id128, &id, sizeof(id));
    return LLMX_OK;
}

int llmx_create(const llmx_shape *shape, int device, int tp_rank, int tp_size, const void *tp_id,
                llmx_ctx **out) {
    if (!shape || !out) return LLMX_ERR_ARG;
    *out = nullptr;
    int rc = llmx_shape_validate(shape);
    if (rc) return rc;
    if (tp_size < 1 || tp_rank < 0 || tp_rank >= tp_size || (tp_size > 1 && !tp_id)) return LLMX_ERR_ARG;
    const llmx_shape &s = *shape;
    // tensor parallel split: Q/O heads and FFN columns; 8-feature granularity
    if (s.heads % tp_size || s.inter % (8 * tp_size)) return LLMX_ERR_UNSUPPORTED;
    const int hd = s.hidden / s.heads, G = s.heads / s.kv_heads, hq = s.heads / tp_size;
    if (!(hq % G == 0 || G % hq == 0) || (hq * hd) % 8) return LLMX_ERR_UNSUPPORTED;
    llmx_ctx *c = new llmx_ctx();
    c->s = s;
    c->dev = device;
    c->rank = tp_rank;
    c->size = tp_size;
    c->hd = hd;
    c->G = G;
    c->KV = s.kv_heads * hd;
    c->hq = hq;
    c->h0 = tp_rank * hq;
    c->Hq = hq * hd;
    c->Il = s.inter / tp_size;
    c->c0 = tp_rank * c->Il;
    const int max_tiles = (s.max_seq + kTile - 1) / kTile;
    c->tpc_max = (max_tiles + kCluster - 1) / kCluster;
    c->tpc_max_wide = (max_tiles + kClusterWide - 1) / kClusterWide;
    c->layer_loaded.assign(s.layers, false);
    c->ring_kb = env_int("LLMX_RING_KB", 96, 8, 220);
    c->ring_wide_kb = env_int("LLMX_RING_WIDE_KB", 176, 8, 200);  // measured best for Down on B200
    c->ring_gu_kb = env_int("LLMX_RING_GU_KB", 160, 8, 200);  // 160: 685.9/672.7 -> 696.8/696.1 tok/s
    c->attn_pf_tile_kb = env_int("LLMX_ATTN_PREFETCH_TILE_KB", 3584, 0, 1 << 20);
    c->attn_pf_kb = env_int("LLMX_ATTN_PREFETCH_KB", 72 * 1024, 0, 1 << 22);
    c->attn_pf_rows = env_int("LLMX_ATTN_PREFETCH_ROWS", 2, 1, 8);
    c->attn_pf_late = env_int("LLMX_ATTN_PREFETCH_LATE", 1, 0, 1);
    c->attn_trigger_tiles = env_int("LLMX_ATTN_TRIGGER_TILES", 16, 0, 1 << 20);
    c->gemv_ctas_per_sm = env_int("LLMX_GEMV_CTAS_PER_SM", 1, 1, 2);
    c->gemv_warps = env_int("LLMX_GEMV_WARPS", 16, 2, 16);
    c->proj_carveout = env_int("LLMX_PROJ_CARVEOUT", 100, -1, 100);
    c->ar_fuse_rows = env_int("LLMX_AR_FUSE_ROWS", 2, 0, 8);
    c->fuse_o_tp = c->size > 1 && env_int("LLMX_ATTN_FUSE_O_TP", 0, 0, 1) == 1;
    c->fuse_o = env_int("LLMX_ATTN_FUSE_O", 1, 0, 1) == 1 && (c->size == 1 || c->fuse_o_tp);
    auto bail = [&](int code) {
        release(c);
        return code;
    };
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return bail(fail_cuda(e, "cudaSetDevice"));
    cudaDeviceProp prop{};
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return bail(fail_cuda(e, "cudaGetDeviceProperties"));
    c->nsm = prop.multiProcessorCount;
    e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return bail(fail_cuda(e, "cudaStreamCreate"));
    e = proj_configure(kProjSmem, c->proj_carveout);
    if (e != cudaSuccess) return bail(fail_cuda(e, "proj_configure"));
    e = attn_configure((int)attn_smem_bytes(c->tpc_max, hd, kCluster, s.hidden / kCluster), kCluster, c->fuse_o_tp);
    if (e == cudaSuccess) e = attn_rows_configure((int)attn_rows_smem_bytes(c->tpc_max, kCluster), kCluster);
    if (e != cudaSuccess) return bail(fail_cuda(e, "attn_configure"));
    c->attn_rows_min = env_int("LLMX_ATTN_ROWS_MIN", 2, 2, 9);
    c->attn_rows_inner = env_int("LLMX_ATTN_ROWS_INNER", 0, 0, 1) == 1;
    if (hd % kClusterWide == 0 && env_int("LLMX_ATTN_ROWS_WIDE", 0, 0, 1) == 1) {
        e = attn_rows_configure((int)attn_rows_smem_bytes(c->tpc_max_wide, kClusterWide), kClusterWide);
        if (e == cudaSuccess) c->attn_rows_wide = true;
        else (void)cudaGetLastError();
    }
    // LLMX_ATTN_WIDE=0 keeps 8-CTA clusters everywhere
    c->attn_wide_div = env_int("LLMX_ATTN_WIDE_DIV", 1, 1, 8);
    // LLMX_ATTN_WIDE=2: 16-CTA clusters whatever the head count (every one-row
    // attention launch; several CTAs then share an SM)
    const int wide_env = env_int("LLMX_ATTN_WIDE", 1, 0, 2);
    if (wide_env == 2) c->attn_wide_div = 0;
    if (max_tiles > 2 * kCluster && hd % kClusterWide == 0 && c->attn_wide_div * c->hq * kClusterWide <= c->nsm &&
        wide_env >= 1) {
        e = attn_configure((int)attn_smem_bytes(c->tpc_max_wide, hd, kClusterWide, s.hidden / kClusterWide),
                           kClusterWide, c->fuse_o_tp);
        if (e == cudaSuccess)
            e = attn_rows_configure((int)attn_rows_smem_bytes(c->tpc_max_wide, kClusterWide), kClusterWide);
        if (e == cudaSuccess) c->attn_wide = true;
        else (void)cudaGetLastError();  // keep 8-CTA clusters
    }

    const size_t H = s.hidden;
    c->w_qkv = (size_t)(c->Hq + 2 * c->KV) * H / 2;
    c->w_o = H * (size_t)c->Hq / 2;
    c->w_gu = (size_t)2 * c->Il * H / 2;
    c->w_d = H * (size_t)c->Il / 2;
    c->layer_words = c->w_qkv + c->w_o + c->w_gu + c->w_d;
    const size_t kv_elems = (size_t)s.layers * s.kv_heads * s.max_seq * hd;
    // the softmax table (2049 entries) is padded to 2056: attention copies it in 16-byte chunks
    if ((rc = dalloc(c, &c->wbuf, c->layer_words * s.layers)) ||
        (rc = dalloc(c, &c->staging, layer_elems(s))) ||
        (rc = dalloc(c, &c->slot_qkv, c->Hq + 2 * c->KV)) || (rc = dalloc(c, &c->slot_o, H)) ||
        (rc = dalloc(c, &c->slot_gu, 2 * c->Il)) || (rc = dalloc(c, &c->slot_d, H)) ||
        (rc = dalloc(c, &c->norms, (2 * (size_t)s.layers + 1) * H)) ||
        (rc = dalloc(c, &c->rope, (size_t)s.max_seq * hd)) || (rc = dalloc(c, &c->etab, 2049)) ||
        (rc = dalloc(c, &c->ptab, 2056)) || (rc = dalloc(c, &c->kc, kv_elems)) ||
        (rc = dalloc(c, &c->vc, kv_elems)) || (rc = dalloc(c, &c->hid[0], kMaxRows * H)) ||
        (rc = dalloc(c, &c->hid[1], kMaxRows * H)) || (rc = dalloc(c, &c->hid[2], kMaxRows * H)) ||
        (rc = dalloc(c, &c->q, kMaxRows * (size_t)c->Hq)) ||
        (rc = dalloc(c, &c->att, kMaxRows * (size_t)c->Hq)) ||
        (rc = dalloc(c, &c->act, kMaxRows * (size_t)c->Il)) || (rc = dalloc(c, &c->partial, kMaxRows * H)) ||
        (rc = dalloc(c, &c->o_acc, kMaxRows * H)) ||
        (rc = dalloc(c, &c->step, 1)) || (rc = dalloc(c, &c->err, 1)))
        return bail(rc);
    if (cudaHostAlloc(&c->err_host, sizeof(int), cudaHostAllocDefault) != cudaSuccess) {
        c->err_host = nullptr;  // finish() falls back to a blocking read
        (void)cudaGetLastError();
    }
    // head-major O weights for the fused decode attention (w_o words per layer);
    // without the memory the O projection stays a kernel of its own
    if (c->fuse_o && dalloc(c, &c->o_heads, c->w_o * s.layers) != LLMX_OK) {
        c->fuse_o = false;
        (void)cudaGetLastError();
    }
    if (c->fuse_o && c->size > 1 && (rc = dalloc(c, &c->o_cnt, (size_t)kMaxRows * kClusterWide)))
        return bail(rc);
    if (c->fuse_o && c->size == 1 && env_int("LLMX_ATTN_SPLIT_O", 0, 0, 1) == 1) {
        int ok = 0;
        const size_t b = attn_smem_bytes(c->tpc_max, hd, kCluster, (int)(H / kCluster), true);
        if (attn_split_configure((int)b, c->hq, &ok) != cudaSuccess) {
            ok = 0;
            (void)cudaGetLastError();
        }
        c->attn_split_o = ok != 0;  // else the default kernel (every cluster must be resident at once)
    }

    // tensor-core projections for blocks of mma_min_rows..8 rows: QKV tiles are
    // heads, so head_dim must be 128 (every Qwen profile); LLMX_MMA=0 disables
    c->mma_min_rows = env_int("LLMX_MMA_MIN_ROWS", 3, 1, 9);
    c->mma_proj = env_int("LLMX_MMA_PROJ", 0xC, 0, 0xF);
    if (hd == 128 && env_int("LLMX_MMA", 1, 0, 1) == 1) {
        auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
        MmaGeom *g = c->mg;
        const int Hi = (int)H;
        g[MP_QKV].T = hq + 2 * s.kv_heads, g[MP_QKV].C = cdiv(Hi, 128), g[MP_QKV].K = Hi;
        g[MP_QKV].n_out = g[MP_QKV].T * 128;
        g[MP_O].T = cdiv(Hi, 128), g[MP_O].C = cdiv(c->Hq, 128), g[MP_O].K = c->Hq, g[MP_O].n_out = Hi;
        g[MP_GU].T = cdiv(c->Il, 64), g[MP_GU].C = cdiv(Hi, 128), g[MP_GU].K = Hi, g[MP_GU].n_out = c->Il;
        g[MP_D].T = cdiv(Hi, 128), g[MP_D].C = cdiv(c->Il, 128), g[MP_D].K = c->Il, g[MP_D].n_out = Hi;
        size_t off = 0, woff = 0;
        int tmax = 0;
        for (int p = 0; p < 4; p++) {
            g[p].offset = off;
            off += g[p].items() * kMmaItemBytes;
            g[p].wsum_offset = woff;
            woff += (size_t)g[p].T * (g[p].C + 1) * 128;
            tmax = std::max(tmax, g[p].T);
        }
        c->mma_layer_bytes = off;
        c->mma_wsum_layer = woff;
        if ((rc = dalloc(c, &c->mbuf, off * s.layers)) || (rc = dalloc(c, &c->mma_wsum, woff * s.layers)) ||
            (rc = dalloc(c, &c->mma_scratch, (size_t)c->nsm * 2 * kMaxRows * 128)) ||
            (rc = dalloc(c, &c->mma_cnt, (size_t)tmax)))
            return bail(rc);
        // tile row -> dense row of each projection's source matrix (-1: zero padding)
        for (int p = 0; p < 4; p++) {
            std::vector<int32_t> rows((size_t)g[p].T * 128, -1);
            for (int t = 0; t < g[p].T; t++)
                for (int m = 0; m < 128; m++) {
                    int32_t r = -1;
                    if (p == MP_QKV) {
                        const int kvh = t - hq;
                        r = t < hq ? (c->h0 + t) * 128 + m
                                   : (kvh < s.kv_heads ? Hi + kvh * 128 + m : Hi + c->KV + (kvh - s.kv_heads) * 128 + m);
                    } else if (p == MP_GU) {
                        const int u = t * 64 + (m & 63);
                        if (u < c->Il) r = m < 64 ? c->c0 + u : s.inter + c->c0 + u;
                    } else if (t * 128 + m < Hi) {
                        r = t * 128 + m;
                    }
                    rows[(size_t)t * 128 + m] = r;
                }
            if ((rc = dalloc(c, &c->mma_rows[p], rows.size()))) return bail(rc);
            e = cudaMemcpy(c->mma_rows[p], rows.data(), rows.size() * 4, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) return bail(fail_cuda(e, "tile row upload"));
        }
        e = mma_configure(kProjSmem);
        if (e != cudaSuccess) return bail(fail_cuda(e, "mma_configure"));
        c->mma = true;
    }

    // slot -> dense row tables of the pair-interleaved layout
    {
        std::vector<int32_t> t;
        const int half = hd / 2;
        for (int lh = 0; lh < hq; lh++)  // Q rows of this rank's heads: pairs (i, i+hd/2)
            for (int i = 0; i < half; i++) {
                t.push_back((c->h0 + lh) * hd + i);
                t.push_back((c->h0 + lh) * hd + half + i);
            }
        for (int seg = 1; seg <= 2; seg++)  // K then V rows (dense rows after Q)
            for (int kh = 0; kh < s.kv_heads; kh++)
                for (int i = 0; i < half; i++) {
                    t.push_back((int)H + (seg - 1) * c->KV + kh * hd + i);
                    t.push_back((int)H + (seg - 1) * c->KV + kh * hd + half + i);
                }
        e = cudaMemcpy(c->slot_qkv, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(fail_cuda(e, "slot upload"));
        t.clear();
        for (int r = 0; r < (int)H; r++) t.push_back(r);
        e = cudaMemcpy(c->slot_o, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(c->slot_d, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(fail_cuda(e, "slot upload"));
        t.clear();
        for (int p = 0; p < c->Il; p++) {  // gate row, up row (up rows follow the gate rows)
            t.push_back(c->c0 + p);
            t.push_back(s.inter + c->c0 + p);
        }
        e = cudaMemcpy(c->slot_gu, t.data(), t.size() * 4, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(fail_cuda(e, "slot upload"));
    }
    // constant tables
    {
        std::vector<int16_t> e16(2049), p18(2049), rope((size_t)s.max_seq * hd);
        build_exp_tables(e16.data(), p18.data());
        build_rope_table(hd, s.max_seq, rope.data());
        e = cudaMemcpy(c->etab, e16.data(), 2049 * 2, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(c->ptab, p18.data(), 2049 * 2, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = cudaMemcpy(c->rope, rope.data(), rope.size() * 2, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return bail(fail_cuda(e, "table upload"));
        c->inv_elems = recip_q88(fm_from_count(s.hidden));
        c->inv_rms_const = inv_rms_q88(0, 0);
        c->qk_scale = qk_scale_q1616(hd);
    }
    if (tp_size > 1) {
        c->nccl_timeout_ms = env_int("LLMX_NCCL_TIMEOUT_MS", 60000, 1, 3600 * 1000);
        ncclUniqueId id;
        std::memcpy(&id, tp_id, sizeof(id));
        ncclResult_t r = ncclCommInitRank(&c->comm, tp_size, id, tp_rank);
        if (r != ncclSuccess) {
            g_last_error = std::string("ncclCommInitRank: ") + ncclGetErrorString(r);
            return bail(LLMX_ERR_NCCL);
        }
        if ((rc = setup_peer_allreduce(c, env_int("LLMX_TP_NCCL", 0, 0, 1) == 0))) return bail(rc);
    }
    *out = c;
    return LLMX_OK;
}

int llmx_destroy(llmx_ctx *c) {
    release(c);
    return LLMX_OK;
}

int llmx_upload_layer(llmx_ctx *c, uint32_t layer, const int16_t *dense) {
    if (!c || !dense || layer >= (uint32_t)c->s.layers) return LLMX_ERR_ARG;
    const llmx_shape &s = c->s;
    CK(cudaSetDevice(c->dev));
    size_t off[8];
    layer_offsets(s, off);
    CK(cudaMemcpyAsync(c->staging, dense, layer_elems(s) * 2, cudaMemcpyHostToDevice, c->stream));
    uint32_t *w = c->wbuf + (size_t)layer * c->layer_words;
    const int H = s.hidden;
    // Q,K,V are consecutive dense matrices with row length H
    CK(launch_pack_pairs(c->staging + off[0], H, 0, H, c->slot_qkv, c->Hq + 2 * c->KV, w, c->stream));
    CK(launch_pack_pairs(c->staging + off[3], H, c->h0 * c->hd, c->Hq, c->slot_o, H, w + c->w_qkv, c->stream));
    if (c->o_heads)  // head h: its hd columns of every O row, rows contiguous
        for (int h = 0; h < c->hq; h++)
            CK(launch_pack_pairs(c->staging + off[3], H, (c->h0 + h) * c->hd, c->hd, c->slot_o, H,
                                 c->o_heads + (size_t)layer * c->w_o + (size_t)h * H * (c->hd / 2), c->stream));
    CK(launch_pack_pairs(c->staging + off[4], H, 0, H, c->slot_gu, 2 * c->Il, w + c->w_qkv + c->w_o, c->stream));
    CK(launch_pack_pairs(c->staging + off[6], s.inter, c->c0, c->Il, c->slot_d, H,
                         w + c->w_qkv + c->w_o + c->w_gu, c->stream));
    if (c->mma) {  // the tensor-core item layout of the same weights
        uint8_t *mb = c->mbuf + (size_t)layer * c->mma_layer_bytes;
        const MmaGeom *g = c->mg;
        CK(launch_pack_mma(c->staging + off[0], H, 0, H, g[MP_QKV].C, c->mma_rows[MP_QKV], g[MP_QKV].T,
                           mb + g[MP_QKV].offset, c->stream));
        CK(launch_pack_mma(c->staging + off[3], H, c->h0 * c->hd, c->Hq, g[MP_O].C, c->mma_rows[MP_O], g[MP_O].T,
                           mb + g[MP_O].offset, c->stream));
        CK(launch_pack_mma(c->staging + off[4], H, 0, H, g[MP_GU].C, c->mma_rows[MP_GU], g[MP_GU].T,
                           mb + g[MP_GU].offset, c->stream));
        CK(launch_pack_mma(c->staging + off[6], s.inter, c->c0, c->Il, g[MP_D].C, c->mma_rows[MP_D], g[MP_D].T,
                           mb + g[MP_D].offset, c->stream));
        // weight-sum prefix tables (the signed low activation bytes' correction)
        int32_t *ws = c->mma_wsum + (size_t)layer * c->mma_wsum_layer;
        CK(launch_mma_wsum(c->staging + off[0], H, 0, H, g[MP_QKV].C, c->mma_rows[MP_QKV], g[MP_QKV].T,
                           ws + g[MP_QKV].wsum_offset, c->stream));
        CK(launch_mma_wsum(c->staging + off[3], H, c->h0 * c->hd, c->Hq, g[MP_O].C, c->mma_rows[MP_O], g[MP_O].T,
                           ws + g[MP_O].wsum_offset, c->stream));
        CK(launch_mma_wsum(c->staging + off[4], H, 0, H, g[MP_GU].C, c->mma_rows[MP_GU], g[MP_GU].T,
                           ws + g[MP_GU].wsum_offset, c->stream));
        CK(launch_mma_wsum(c->staging + off[6], s.inter, c->c0, c->Il, g[MP_D].C, c->mma_rows[MP_D], g[MP_D].T,
                           ws + g[MP_D].wsum_offset, c->stream));
    }
    SYNC(c);
    c->layer_loaded[layer] = true;
    for (auto &g : c->graphs) cudaGraphExecDestroy(g.second.first);
    c->graphs.clear();
    return LLMX_OK;
}

int llmx_upload_norms(llmx_ctx *c, const int16_t *norms) {
    if (!c || !norms) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    CK(cudaMemcpy(c->norms, norms, (2 * (size_t)c->s.layers + 1) * c->s.hidden * 2, cudaMemcpyHostToDevice));
    c->norms_loaded = true;
    return LLMX_OK;
}

int llmx_upload_model(llmx_ctx *c, const llmx_model *m) {
    if (!c || !m) return LLMX_ERR_ARG;
    if (std::memcmp(&c->s, &m->shape, sizeof(llmx_shape)) != 0) return LLMX_ERR_ARG;
    if (m->norms.empty()) return LLMX_ERR_STATE;
    int rc = llmx_upload_norms(c, m->norms.data());
    if (rc) return rc;
    for (size_t l = 0; l < m->layers.size(); l++)
        if (!m->layers[l].empty() && (rc = llmx_upload_layer(c, (uint32_t)l, m->layers[l].data()))) return rc;
    return LLMX_OK;
}

int llmx_reset_kv(llmx_ctx *c) {
    if (!c) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    const size_t n = (size_t)c->s.layers * c->s.kv_heads * c->s.max_seq * c->hd * 2;
    CK(cudaMemsetAsync(c->kc, 0, n, c->stream));
    CK(cudaMemsetAsync(c->vc, 0, n, c->stream));
    SYNC(c);
    return LLMX_OK;
}

static int kv_copy(llmx_ctx *c, uint32_t layer, uint32_t position, uint32_t count, int16_t *k, int16_t *v,
                   bool to_device) {
    if (!c || !k || !v || layer >= (uint32_t)c->s.layers || (uint64_t)position + count > (uint64_t)c->s.max_seq)
        return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    const size_t row = (size_t)c->hd * 2, n = (size_t)count * row;
    for (int h = 0; h < c->s.kv_heads; h++) {
        int16_t *dk = kc_layer(c, layer) + ((size_t)h * c->s.max_seq + position) * c->hd;
        int16_t *dv = vc_layer(c, layer) + ((size_t)h * c->s.max_seq + position) * c->hd;
        int16_t *hk = k + (size_t)h * count * c->hd, *hv = v + (size_t)h * count * c->hd;
        if (to_device) {
            CK(cudaMemcpyAsync(dk, hk, n, cudaMemcpyHostToDevice, c->stream));
            CK(cudaMemcpyAsync(dv, hv, n, cudaMemcpyHostToDevice, c->stream));
        } else {
            CK(cudaMemcpyAsync(hk, dk, n, cudaMemcpyDeviceToHost, c->stream));
            CK(cudaMemcpyAsync(hv, dv, n, cudaMemcpyDeviceToHost, c->stream));
        }
    }
    SYNC(c);
    return LLMX_OK;
}

int llmx_write_kv(llmx_ctx *c, uint32_t layer, uint32_t position, uint32_t count, const int16_t *k,
                  const int16_t *v) {
    return kv_copy(c, layer, position, count, const_cast<int16_t *>(k), const_cast<int16_t *>(v), true);
}

int llmx_read_kv(llmx_ctx *c, uint32_t layer, uint32_t position, uint32_t count, int16_t *k, int16_t *v) {
    return kv_copy(c, layer, position, count, k, v, false);
}

int llmx_write_hidden(llmx_ctx *c, uint32_t pair, const int16_t *rows_host, uint32_t rows) {
    if (!c || pair > 1 || !rows_host || rows > LLMX_MAX_ROWS) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    CK(cudaMemcpyAsync(c->hid[pair], rows_host, (size_t)rows * c->s.hidden * 2, cudaMemcpyHostToDevice,
                       c->stream));
    SYNC(c);
    return LLMX_OK;
}

int llmx_read_hidden(llmx_ctx *c, uint32_t pair, int16_t *rows_host, uint32_t rows) {
    if (!c || pair > 1 || !rows_host || rows > LLMX_MAX_ROWS) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    CK(cudaMemcpyAsync(rows_host, c->hid[pair], (size_t)rows * c->s.hidden * 2, cudaMemcpyDeviceToHost,
                       c->stream));
    SYNC(c);
    return LLMX_OK;
}

int llmx_bind(llmx_ctx *c, uint32_t out_pair, uint32_t in_pair) {
    if (!c || out_pair > 1 || in_pair > 1 || out_pair == in_pair) return LLMX_ERR_ARG;
    c->out_pair = out_pair;
    c->in_pair = in_pair;
    return LLMX_OK;
}

int llmx_task(llmx_ctx *c, uint32_t op, uint32_t layer, uint32_t position, uint32_t rows, llmx_status *st) {
    llmx_status local;
    if (!st) st = &local;
    if (!c) return LLMX_ERR_ARG;
    const int code = llmx_validate_task(&c->s, op, layer, position, rows, st);
    if (code != LLMX_OK || op == LLMX_OP_NOP) return code;
    if (op != LLMX_OP_FINAL_NORM && !model_ready(c, layer, 1)) return LLMX_ERR_STATE;
    if (op == LLMX_OP_FINAL_NORM && !c->norms_loaded) return LLMX_ERR_STATE;
    CK(cudaSetDevice(c->dev));
    const uint64_t before = c->launches;
    int rc = set_step(c, position, rows);
    uint32_t ar_next = 0;
    PendingAr pend;
    if (!rc) rc = enqueue_task(c, op, layer, rows, c->in_pair, c->out_pair, ar_next, false, pend);
    if (rc) return rc;
    c->ar_count += task_allreduces(c, op);
    c->last_launches = c->launches - before;
    return finish(c);
}

// Per-operator (feature) modes, ops 1-10 (run_feature host:1088-1130).
int llmx_run_feature(llmx_ctx *c, uint32_t op, const int16_t *lhs, uint32_t rows, uint32_t lhs_cols,
                     const int16_t *rhs, uint32_t rhs_rows, uint32_t rhs_cols, uint32_t layer, uint32_t position,
                     int16_t *out, uint32_t out_cols, llmx_status *st) {
    llmx_status local;
    if (!st) st = &local;
    if (!c || !lhs || !out) return LLMX_ERR_ARG;
    const llmx_shape &s = c->s;
    uint32_t in_dim = 0, out_dim = 0;
    int needs_rhs = 0;
    if (llmx_feature_dims(&s, op, &in_dim, &out_dim, &needs_rhs) != LLMX_OK) {
        g_last_error = "operator is not a feature operator";
        return LLMX_ERR_ARG;
    }
    // the host's shape checks (runtime_error in the reference) come before any launch
    if (rows == 0 || rows > LLMX_MAX_ROWS || lhs_cols != in_dim || out_cols != out_dim) {
        g_last_error = "feature operator input shape mismatch";
        return LLMX_ERR_ARG;
    }
    if (needs_rhs && (!rhs || rhs_cols != in_dim || rhs_rows != (op == LLMX_OP_RMSNORM ? 1u : rows))) {
        g_last_error = "feature operator RHS shape mismatch";
        return LLMX_ERR_ARG;
    }
    if (c->size > 1) {
        g_last_error = "feature operators run on single-GPU contexts";
        return LLMX_ERR_UNSUPPORTED;
    }
    const int code = llmx_validate_operator(&s, op, layer, position, rows, st);
    if (code != LLMX_OK) return code;
    const bool projection = op <= LLMX_OP_FFN_DOWN;
    if (projection && !c->layer_loaded[layer]) return LLMX_ERR_STATE;
    CK(cudaSetDevice(c->dev));
    const size_t width = (size_t)std::max(s.hidden, s.inter);
    const size_t slots = std::max<size_t>({(size_t)c->Hq + 2 * c->KV, (size_t)2 * c->Il, (size_t)s.hidden});
    int rc = LLMX_OK;
    // feat_sums is allocated last: a failed allocation is retried as a whole on the next call
    if (!c->feat_sums && ((rc = dalloc(c, &c->feat_lhs, kMaxRows * width)) ||
                         (rc = dalloc(c, &c->feat_rhs, kMaxRows * width)) ||
                         (rc = dalloc(c, &c->feat_out, kMaxRows * width)) ||
                         (rc = dalloc(c, &c->feat_sums, kMaxRows * slots))))
        return rc;
    const uint64_t before = c->launches;
    CK(cudaMemcpyAsync(c->feat_lhs, lhs, (size_t)rows * in_dim * 2, cudaMemcpyHostToDevice, c->stream));
    if (needs_rhs)
        CK(cudaMemcpyAsync(c->feat_rhs, rhs, (size_t)rhs_rows * in_dim * 2, cudaMemcpyHostToDevice, c->stream));
    if ((rc = set_step(c, position, rows))) return rc;
    if (projection) {
        // the operator's slots of the packed layer blob: [slot0, slot0 + nslots) of
        // a region whose rows are K inputs long
        const uint32_t *w = wl(c, layer);
        uint32_t K = s.hidden, slot0 = 0, nslots = 0;
        int order = kSlotIdentity;
        switch (op) {
        case LLMX_OP_Q_PROJECTION: nslots = c->Hq, order = kSlotRopePairs; break;
        case LLMX_OP_K_PROJECTION: slot0 = c->Hq, nslots = c->KV, order = kSlotRopePairs; break;
        case LLMX_OP_V_PROJECTION: slot0 = c->Hq + c->KV, nslots = c->KV, order = kSlotRopePairs; break;
        case LLMX_OP_O_PROJECTION: w += c->w_qkv, K = c->Hq, nslots = s.hidden; break;
        case LLMX_OP_FFN_GATE:
        case LLMX_OP_FFN_UP:
            w += c->w_qkv + c->w_o, nslots = 2 * c->Il;
            order = op == LLMX_OP_FFN_GATE ? kSlotEven : kSlotOdd;
            break;
        default: w += c->w_qkv + c->w_o + c->w_gu, K = c->Il, nslots = s.hidden; break;  // Down
        }
        const int rt = rows_template(rows);
        ProjArgs a{};
        a.w = w + (size_t)slot0 * (K / 2);
        a.K = (int)K;
        a.npairs = (int)nslots / 2;
        a.x = c->feat_lhs;
        a.step = c->step;
        a.partial = c->feat_sums;
        a.out_stride = (int)nslots;
        set_stages(c, a, EPI_PARTIAL, rt);
        CK(launch_proj(a, EPI_PARTIAL, rt, grid_for(c, a.npairs, rt, a.K), c->stream));
        FeatureRoundArgs f{c->feat_sums, (int)nslots, c->feat_out, (int)rows, (int)out_dim, order, c->hd};
        CK(launch_feature_round(f, c->stream));
        c->launches += 2;
    } else if (op == LLMX_OP_RMSNORM) {
        NormArgs n{c->feat_lhs, c->feat_rhs, c->feat_out, s.hidden, c->inv_elems, c->inv_rms_const, c->step};
        CK(launch_rmsnorm(n, (int)rows, c->stream));
        c->launches += 1;
    } else {
        FeatureVecArgs v{c->feat_lhs, c->feat_rhs, c->feat_out, c->etab, (int)(rows * in_dim),
                         op == LLMX_OP_SILU_MUL ? 1 : 0};
        CK(launch_feature_vec(v, c->stream));
        c->launches += 1;
    }
    CK(cudaMemcpyAsync(out, c->feat_out, (size_t)rows * out_dim * 2, cudaMemcpyDeviceToHost, c->stream));
    c->last_launches = c->launches - before;
    return finish(c);
}

// Prefill block attention, op 17 (run_prefill_attention_block host:1647-1690).
int llmx_run_prefill_attention_block(llmx_ctx *c, const int16_t *query, uint32_t position, uint32_t rows,
                                     uint32_t layer, int16_t *out, llmx_status *st) {
    llmx_status local;
    if (!st) st = &local;
    if (!c || !query || !out) return LLMX_ERR_ARG;
    const llmx_shape &s = c->s;
    if (c->size > 1) {
        g_last_error = "the prefill block operator runs on single-GPU contexts";
        return LLMX_ERR_UNSUPPORTED;
    }
    // host:1655-1666: shape checks before the launch
    if (rows == 0 || rows > LLMX_MAX_ROWS || (uint64_t)position + rows > (uint64_t)s.max_seq) {
        g_last_error = "prefill attention block shape mismatch";
        return LLMX_ERR_ARG;
    }
    const int code = llmx_validate_operator(&s, LLMX_OP_ATTN_PREFILL_BLOCK, layer, position, rows, st);
    if (code != LLMX_OK) return code;
    CK(cudaSetDevice(c->dev));
    // ports (KV head p: [rows][G][hd], token-major then local head) <-> rows of all
    // query heads [rows][heads][hd] (head = p * G + g): the host's pack_tight step
    const int hd = c->hd, G = c->G, KVh = s.kv_heads, Hq = c->Hq;
    std::vector<int16_t> rowbuf((size_t)rows * Hq);
    for (int p = 0; p < KVh; p++)
        for (uint32_t r = 0; r < rows; r++)
            for (int g = 0; g < G; g++)
                std::memcpy(&rowbuf[(size_t)r * Hq + (size_t)(p * G + g) * hd],
                            query + (((size_t)p * rows + r) * G + g) * hd, (size_t)hd * 2);
    const uint64_t before = c->launches;
    CK(cudaMemcpyAsync(c->q, rowbuf.data(), rowbuf.size() * 2, cudaMemcpyHostToDevice, c->stream));
    int rc = set_step(c, position, rows);
    if (rc) return rc;
    AttnArgs t = attn_args(c, layer);
    t.pf_bytes = 0;  // no projection follows
    t.pf_per_tile = 0;
    CK(launch_attention(c, t, rows));
    c->launches += 1;
    CK(cudaMemcpyAsync(rowbuf.data(), c->att, rowbuf.size() * 2, cudaMemcpyDeviceToHost, c->stream));
    c->last_launches = c->launches - before;
    if ((rc = finish(c))) return rc;
    for (int p = 0; p < KVh; p++)
        for (uint32_t r = 0; r < rows; r++)
            for (int g = 0; g < G; g++)
                std::memcpy(out + (((size_t)p * rows + r) * G + g) * hd,
                            &rowbuf[(size_t)r * Hq + (size_t)(p * G + g) * hd], (size_t)hd * 2);
    return LLMX_OK;
}

int llmx_stack_async(llmx_ctx *c, uint32_t rows, uint32_t layer_begin, uint32_t layer_count, uint32_t position,
                     int include_final_norm) {
    if (!c) return LLMX_ERR_ARG;
    const llmx_shape &s = c->s;
    if (rows == 0 || rows > LLMX_MAX_ROWS || layer_count == 0 || layer_begin >= (uint32_t)s.layers ||
        layer_begin + layer_count > (uint32_t)s.layers || position >= (uint32_t)s.max_seq ||
        position + rows > (uint32_t)s.max_seq)
        return LLMX_ERR_ARG;  // run_composed_decoder_stack host:1266-1281
    if (!model_ready(c, layer_begin, layer_count)) return LLMX_ERR_STATE;
    CK(cudaSetDevice(c->dev));
    const uint64_t before = c->launches;
    const int rc = launch_stack_at(c, rows, layer_begin, layer_count, position, include_final_norm ? 1 : 0);
    c->last_launches = c->launches - before;
    return rc;
}

int llmx_stack(llmx_ctx *c, const int16_t *hidden_in, uint32_t rows, uint32_t layer_begin, uint32_t layer_count,
               uint32_t position, int include_final_norm, int materialize, int16_t *hidden_out,
               llmx_status *last) {
    if (!c || !hidden_in || (materialize && !hidden_out)) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    if (rows == 0 || rows > LLMX_MAX_ROWS) return LLMX_ERR_ARG;
    CK(cudaMemcpyAsync(c->hid[1], hidden_in, (size_t)rows * c->s.hidden * 2, cudaMemcpyHostToDevice, c->stream));
    int rc = llmx_stack_async(c, rows, layer_begin, layer_count, position, include_final_norm);
    if (rc) return rc;
    if (materialize)
        CK(cudaMemcpyAsync(hidden_out, c->hid[include_final_norm ? 0 : 1], (size_t)rows * c->s.hidden * 2,
                           cudaMemcpyDeviceToHost, c->stream));
    if ((rc = finish(c))) return rc;
    if (last) {
        const uint32_t op = include_final_norm ? LLMX_OP_FINAL_NORM : LLMX_OP_FFN_SUBLAYER;
        llmx_validate_task(&c->s, op, include_final_norm ? 0 : layer_begin + layer_count - 1, position, rows,
                           last);
    }
    return LLMX_OK;
}

int llmx_synchronize(llmx_ctx *c) {
    if (!c) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    return finish(c);
}

int llmx_time_kernel(llmx_ctx *c, int kernel, uint32_t layer, uint32_t position, uint32_t rows, int iters,
                     double *ms_per_launch) {
    if (!c || !ms_per_launch || iters < 1 || rows == 0 || rows > LLMX_MAX_ROWS ||
        layer >= (uint32_t)c->s.layers || position + rows > (uint32_t)c->s.max_seq)
        return LLMX_ERR_ARG;
    if (!model_ready(c, 0, (uint32_t)c->s.layers)) return LLMX_ERR_STATE;
    CK(cudaSetDevice(c->dev));
    const int rt = rows_template(rows);
    const int ge = c->size > 1 ? EPI_PARTIAL : EPI_RESID;
    int16_t *out = c->hid[0];
    const int16_t *in = c->hid[1];
    int rc = set_step(c, position, rows);
    if (rc) return rc;
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    uint32_t cur = layer;  // rotate layers so that repeated launches stream distinct weights
    auto one = [&]() -> cudaError_t {
        const uint32_t layer = cur;
        cur = (cur + 1) % (uint32_t)c->s.layers;
        switch (kernel) {
        case LLMX_KERNEL_QKV: {
            ProjArgs a = qkv_args(c, layer, in);
            if (use_mma(c, rows, MP_QKV)) return launch_mma(c, a, MP_QKV, layer, EPI_QKV) ? cudaErrorUnknown : cudaSuccess;
            set_stages(c, a, EPI_QKV, rt);
            return launch_proj(a, EPI_QKV, rt, grid_for(c, a.npairs, rt, a.K), c->stream);
        }
        case LLMX_KERNEL_ATTN: {  // as a stack launches it (with the O projection when fused)
            AttnArgs t = attn_args(c, layer);
            if (use_fuse_o(c, rows)) set_fuse_o(c, t, layer);
            return launch_attention(c, t, rows);
        }
        case LLMX_KERNEL_O: {
            ProjArgs o = o_args(c, layer, out, in);
            o.ar.n = 0;  // timing only: keep the partial sums local, signal no rank
            if (use_mma(c, rows, MP_O)) return launch_mma(c, o, MP_O, layer, ge) ? cudaErrorUnknown : cudaSuccess;
            set_stages(c, o, ge, rt);
            return launch_proj(o, ge, rt, grid_for(c, o.npairs, rt, o.K), c->stream);
        }
        case LLMX_KERNEL_GATE_UP: {
            ProjArgs g = gu_args(c, layer, in);
            if (use_mma(c, rows, MP_GU)) return launch_mma(c, g, MP_GU, layer, EPI_SILU) ? cudaErrorUnknown : cudaSuccess;
            set_stages(c, g, EPI_SILU, rt);
            return launch_proj(g, EPI_SILU, rt, grid_for(c, g.npairs, rt, g.K), c->stream);
        }
        case LLMX_KERNEL_DOWN: {
            ProjArgs d = down_args(c, layer, out, in);
            d.ar.n = 0;  // timing only: keep the partial sums local, signal no rank
            if (use_mma(c, rows, MP_D)) return launch_mma(c, d, MP_D, layer, ge) ? cudaErrorUnknown : cudaSuccess;
            set_stages(c, d, ge, rt);
            return launch_proj(d, ge, rt, grid_for(c, d.npairs, rt, d.K), c->stream);
        }
        case LLMX_KERNEL_FINAL_NORM: {
            NormArgs n{in, c->norms + (size_t)2 * c->s.layers * c->s.hidden, out, c->s.hidden, c->inv_elems,
                       c->inv_rms_const, c->step};
            return launch_rmsnorm(n, (int)rows, c->stream);
        }
        default: return cudaErrorInvalidValue;
        }
    };
    cudaError_t e = one();  // warm-up launch
    if (e == cudaSuccess) e = cudaEventRecord(e0, c->stream);
    for (int i = 0; i < iters && e == cudaSuccess; i++) e = one();
    if (e == cudaSuccess) e = cudaEventRecord(e1, c->stream);
    if (e == cudaSuccess) e = cudaEventSynchronize(e1);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    // repeated fused-attention launches accumulate into the O sums: clear them
    if (e == cudaSuccess) e = cudaMemsetAsync(c->o_acc, 0, sizeof(int64_t) * kMaxRows * c->s.hidden, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return fail_cuda(e, "llmx_time_kernel");
    *ms_per_launch = (double)ms / iters;
    return LLMX_OK;
}

void *llmx_stream(llmx_ctx *c) { return c ? (void *)c->stream : nullptr; }
void *llmx_hidden_device_ptr(llmx_ctx *c, uint32_t pair) { return c && pair < 2 ? c->hid[pair] : nullptr; }
uint64_t llmx_kernel_launches(const llmx_ctx *c) { return c ? c->last_launches : 0; }
uint64_t llmx_device_bytes(const llmx_ctx *c) { return c ? c->device_bytes : 0; }

int llmx_selftest_ar_timeout(llmx_ctx *c, uint32_t poll_limit) {
    if (!c || poll_limit == 0) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    const size_t bytes = kArHeader + (size_t)2 * kMaxTp * kMaxRows * c->s.hidden * sizeof(uint64_t);
    int rc;
    if (!c->probe_region && (rc = dalloc(c, &c->probe_region, bytes))) return rc;
    ArPeers a{};
    a.base[0] = c->probe_region;  // zeroed words: no tag ever matches
    a.n = 1;
    a.me = 0;
    a.hidden = c->s.hidden;
    a.poll_limit = poll_limit;
    if ((rc = set_step(c, 0, 1))) return rc;
    ArFinishArgs f{a, 0, c->hid[1], c->hid[0], c->step, c->err};
    CK(launch_ar_finish(f, c->stream));
    return finish(c);
}

int llmx_decode_fuses_o(const llmx_ctx *c) { return c && use_fuse_o(c, 1) ? 1 : 0; }

int llmx_allreduce_kind(const llmx_ctx *c) {
    if (!c) return -1;
    if (c->size == 1) return LLMX_AR_NONE;
    return c->ar.n > 1 ? LLMX_AR_PEER : LLMX_AR_NCCL;
}

int llmx_run_prompt_block(llmx_ctx *c, const llmx_model *m, const uint32_t *tokens, uint32_t n, uint32_t position,
                          int materialize, int16_t *hidden_out) {
    if (!c || !m || !tokens || n == 0 || n > LLMX_MAX_ROWS) return LLMX_ERR_ARG;
    std::vector<int16_t> rows((size_t)n * c->s.hidden);
    int rc = llmx_model_embed(m, tokens, n, rows.data());
    if (rc) return rc;
    return llmx_stack(c, rows.data(), n, 0, (uint32_t)c->s.layers, position, materialize, materialize,
                      hidden_out, nullptr);
}

int llmx_run_token(llmx_ctx *c, const llmx_model *m, uint32_t token, uint32_t position, int16_t *hidden_out) {
    if (!c || !m || !hidden_out) return LLMX_ERR_ARG;
    std::vector<int16_t> row(c->s.hidden);
    int rc = llmx_model_embed(m, &token, 1, row.data());
    if (rc) return rc;
    return llmx_stack(c, row.data(), 1, 0, (uint32_t)c->s.layers, position, 1, 1, hidden_out, nullptr);
}

int llmx_upload_vocab(llmx_ctx *c, llmx_model *m) {
    if (!c || !m) return LLMX_ERR_ARG;
    const llmx_shape &s = c->s, &ms = m->shape;
    if (ms.hidden != s.hidden || ms.vocab != s.vocab) {
        g_last_error = "upload_vocab: model hidden size / vocabulary differ from the context's shape";
        return LLMX_ERR_ARG;
    }
    const int16_t *emb = model_embedding_table(m);
    const int16_t *head = model_lm_head_table(m);
    if (!emb || !head) {
        g_last_error = "upload_vocab: the model holds no embedding table or LM head";
        return LLMX_ERR_STATE;
    }
    CK(cudaSetDevice(c->dev));
    const size_t n = (size_t)s.vocab * s.hidden;
    int rc = LLMX_OK;
    if (!c->emb_dev) {
        if ((rc = dalloc(c, &c->emb_dev, n)) || (rc = dalloc(c, &c->gen_rows, (size_t)LLMX_MAX_ROWS * s.hidden)) ||
            (rc = dalloc(c, &c->tok_dev, (size_t)s.max_seq + LLMX_MAX_ROWS)))
            return rc;
        char *scratch = nullptr;
        if ((rc = dalloc(c, &scratch, lm_argmax_scratch_bytes()))) return rc;
        c->lm_scratch = scratch;
    }
    if (head != emb && (!c->head_dev || c->head_dev == c->emb_dev)) {
        if ((rc = dalloc(c, &c->head_dev, n))) return rc;
    }
    CK(cudaMemcpy(c->emb_dev, emb, n * 2, cudaMemcpyHostToDevice));
    if (head == emb) {
        c->head_dev = c->emb_dev;
    } else {
        CK(cudaMemcpy(c->head_dev, head, n * 2, cudaMemcpyHostToDevice));
    }
    c->vocab_loaded = true;
    return LLMX_OK;
}

int llmx_generate(llmx_ctx *c, const uint32_t *prompt, uint32_t n_prompt, uint32_t block_rows, uint32_t layer_count,
                  uint32_t max_new, uint32_t *out_tokens, int16_t *last_block_out) {
    if (!c || !prompt || n_prompt == 0 || block_rows == 0 || block_rows > LLMX_MAX_ROWS ||
        (max_new && !out_tokens))
        return LLMX_ERR_ARG;
    const llmx_shape &s = c->s;
    const uint32_t L = layer_count ? layer_count : (uint32_t)s.layers;
    if (L > (uint32_t)s.layers) return LLMX_ERR_ARG;  // "--layers exceeds the selected profile" host:7638-7640
    // decode forwards run at positions n_prompt .. n_prompt + max_new - 2
    if ((uint64_t)n_prompt + (max_new ? max_new - 1 : 0) > (uint64_t)s.max_seq) return LLMX_ERR_ARG;
    for (uint32_t i = 0; i < n_prompt; i++)
        if (prompt[i] >= (uint32_t)s.vocab) return LLMX_ERR_ARG;
    if (!c->vocab_loaded || !model_ready(c, 0, L)) return LLMX_ERR_STATE;
    CK(cudaSetDevice(c->dev));
    const uint64_t before = c->launches;
    const int H = s.hidden;
    CK(cudaMemcpyAsync(c->tok_dev, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, c->stream));
    int rc = LLMX_OK;
    // prompt in blocks of block_rows rows; only the last block is final-normed (host:9018-9063)
    uint32_t last_rows = 0;
    for (uint32_t b0 = 0; b0 < n_prompt && !rc; b0 += block_rows) {
        const uint32_t n = std::min(block_rows, n_prompt - b0);
        const int last = b0 + n == n_prompt;
        CK(launch_embed_rows(c->emb_dev, c->tok_dev + b0, (int)n, H, (unsigned)s.vocab, c->hid[1], c->err,
                             c->stream));
        c->launches += 1;
        rc = launch_stack_at(c, n, 0, L, b0, last);
        last_rows = n;
    }
    if (!rc && last_block_out)
        CK(cudaMemcpyAsync(c->gen_rows, c->hid[0], (size_t)last_rows * H * 2, cudaMemcpyDeviceToDevice, c->stream));
    // greedy decode (host:9087-9132): argmax of the last final-normed row, fed back
    // as one decode row unless it is the last token asked for
    const int16_t *h = c->hid[0] + (size_t)(last_rows - 1) * H;
    for (uint32_t step = 0; step < max_new && !rc; step++) {
        uint32_t *tok = c->tok_dev + n_prompt + step;
        CK(launch_lm_argmax(h, 1, H, c->head_dev, (unsigned)s.vocab, tok, c->lm_scratch, c->nsm, c->stream));
        c->launches += 2;
        if (step + 1 == max_new) break;
        CK(launch_embed_rows(c->emb_dev, tok, 1, H, (unsigned)s.vocab, c->hid[1], c->err, c->stream));
        c->launches += 1;
        rc = launch_stack_at(c, 1, 0, L, n_prompt + step, 1);
        h = c->hid[0];
    }
    c->last_launches = c->launches - before;
    if (rc) return rc;
    if (max_new)
        CK(cudaMemcpyAsync(out_tokens, c->tok_dev + n_prompt, (size_t)max_new * 4, cudaMemcpyDeviceToHost,
                           c->stream));
    if (last_block_out)
        CK(cudaMemcpyAsync(last_block_out, c->gen_rows, (size_t)last_rows * H * 2, cudaMemcpyDeviceToHost,
                           c->stream));
    return finish(c);
}

}  // extern "C"

#ifdef LLMX_TIMELINE
// ---------------------------------------------------------------------------
// Launch timeline (measurement builds only; see timeline.cuh).  Slots are taken
// for the life of the process, so a graph captured earlier keeps reporting
// under the names its launches took at capture.
// ---------------------------------------------------------------------------
namespace llmx {
static std::mutex g_tl_mu;
static std::vector<std::string> g_tl_names;

int tl_take(const char *name) {
    std::lock_guard<std::mutex> lock(g_tl_mu);
    if ((int)g_tl_names.size() >= kTlSlots) return -1;
    g_tl_names.emplace_back(name);
    return (int)g_tl_names.size() - 1;
}
}  // namespace llmx

LLMX_TL_READER(runtime)
extern "C" int llmx_tl_table_kernels(void *, int, int);
extern "C" int llmx_tl_table_gemv(void *, int, int);
extern "C" int llmx_tl_table_attention(void *, int, int);
extern "C" int llmx_tl_table_mma_proj(void *, int, int);
extern "C" int llmx_tl_table_feature(void *, int, int);

namespace {
using TlReader = int (*)(void *, int, int);
const TlReader kTlReaders[] = {llmx_tl_table_runtime, llmx_tl_table_kernels, llmx_tl_table_gemv,
                               llmx_tl_table_attention, llmx_tl_table_mma_proj, llmx_tl_table_feature};
}  // namespace

extern "C" {

// Clear every stamp on the context's device (after the work enqueued so far).
int llmx_timeline_reset(llmx_ctx *c) {
    if (!c) return LLMX_ERR_ARG;
    CK(cudaSetDevice(c->dev));
    SYNC(c);
    for (TlReader rd : kTlReaders) CK((cudaError_t)rd(nullptr, 0, 1));
    return LLMX_OK;
}

// Number of slots taken so far in this process.
int llmx_timeline_slots(void) {
    std::lock_guard<std::mutex> lock(g_tl_mu);
    return (int)g_tl_names.size();
}

// Name under which slot `slot` was taken ("" for an unknown slot).
const char *llmx_timeline_name(int slot) {
    std::lock_guard<std::mutex> lock(g_tl_mu);
    return slot >= 0 && slot < (int)g_tl_names.size() ? g_tl_names[slot].c_str() : "";
}

// Stamps of slots [0, n) on the context's device after the stream's work:
// out[2*s] = first CTA start, out[2*s+1] = last warp exit (%globaltimer ns);
// a slot that did not run since the last reset reads start = ~0, end = 0.
int llmx_timeline_read(llmx_ctx *c, unsigned long long *out, int n) {
    if (!c || !out || n < 0) return LLMX_ERR_ARG;
    if (n > kTlSlots) n = kTlSlots;
    CK(cudaSetDevice(c->dev));
    SYNC(c);
    std::vector<TlEntry> merged((size_t)n, TlEntry{~0ull, 0ull}), part((size_t)n);
    for (TlReader rd : kTlReaders) {
        CK((cudaError_t)rd(part.data(), n, 0));
        for (int s = 0; s < n; s++)
            if (part[s].start != ~0ull) merged[s] = part[s];
    }
    for (int s = 0; s < n; s++) {
        out[2 * s] = merged[s].start;
        out[2 * s + 1] = merged[s].end;
    }
    return LLMX_OK;
}

}  // extern "C"
#endif  // LLMX_TIMELINE
