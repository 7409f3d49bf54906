// Kernel argument blocks and launch entry points of the resident layer path.
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <cstdint>

#include "timeline.cuh"

namespace llmx {

constexpr int kTile = 64;     // online-softmax tile: include/control_cache_8x64.hpp:72
constexpr int kMaxRows = 8;   // kMaxTokensPerLaunch host:38

// Position/row count of the running task, read by every kernel from device
// memory so that one captured graph serves every position.
struct Step {
    int32_t position;
    int32_t rows;
    uint32_t ar_base;  // tensor parallel: number of the call's first all-reduce
    int32_t pad;
};

// The step record of the running call, read before griddepcontrol.wait: only
// k_set_step writes it, with an ordinary (non-dependent) launch, so every
// kernel of the call starts after that write has completed.  Read through L2
// (ld.global.cg) so that no L1 line of an earlier call is seen.
static __device__ __forceinline__ Step load_step(const Step *p) {
    const int4 v = __ldcg(reinterpret_cast<const int4 *>(p));
    Step s;
    s.position = v.x;
    s.rows = v.y;
    s.ar_base = (uint32_t)v.z;
    s.pad = v.w;
    return s;
}

enum Epi : int {
    EPI_QKV = 0,   // RoPE on Q/K, Q -> q buffer, K/V -> KV cache
    EPI_RESID = 1, // + residual -> hidden out (O and Down projections)
    EPI_SILU = 2,  // gate/up pair -> SiLU(g)*u -> FFN activation
    EPI_PARTIAL = 3 // exact int64 partial sums (tensor-parallel ranks)
};

// Peer all-reduce over NVLink (tensor parallel): each rank owns one exchange
// region and every rank stores its exact int64 partial sums straight into every
// rank's region.  A sum travels as one 64-bit word {sum in the upper 48 bits,
// 16-bit tag in the lower 16}; any partial sum of the path fits 48 bits
// (|sum| < 2^15 * 2^15 * 11008 < 2^44).  A 64-bit store is single-copy atomic,
// so the receiver polls the words themselves and needs no fence or flag.
// All-reduce number n (counted per context, the same on every rank) uses slot
// n & 1 and tag (n mod 65535) + 1.  Two slots suffice: a rank produces
// all-reduce n + 2 only after every rank contributed to n + 1, which each rank
// does only after its readers of n have finished.  Layout:
//   256 B header | uint64 word[2 slots][kMaxTp sources][kMaxRows][hidden]
constexpr int kMaxTp = 8;
constexpr int kArHeader = 256;
constexpr int kErrArTimeout = 5;  // device error code: a peer's sums did not arrive in time
struct ArPeers {
    char *base[kMaxTp];  // exchange region of every rank (this rank's own included)
    int n;               // ranks (0: the partial sums stay local, NCCL reduces them)
    int me;
    int hidden;
    uint32_t poll_limit; // bounded wait for a peer's word (polls about 64 ns apart)
};
static __host__ __device__ __forceinline__ uint32_t ar_tag(uint32_t n) { return n % 65535u + 1u; }
static __host__ __device__ __forceinline__ size_t ar_word_index(int slot, int src, int row, int hidden, int e) {
    return (((size_t)slot * kMaxTp + src) * kMaxRows + row) * hidden + e;
}
// Consumer side of a peer all-reduce, fused into the next projection's
// activation prologue: x = sat16(resid + round(sum over ranks)), also written
// to hid_out by block 0 (the residual of the following sublayer).
struct ArInput {
    ArPeers ar;          // n <= 1: plain activation input
    uint32_t ar_off;     // all-reduce number = step->ar_base + ar_off
    const int16_t *resid;
    int16_t *hid_out;
    // single GPU: the exact O sums [kMaxRows][K] the attention kernel added up
    // (attention with the O projection fused); x = sat16(resid + round(sum))
    const int64_t *sums;
};

struct ProjArgs {
    const uint32_t *w;   // unit-ordered, byte-split weights (see launch_pack_pairs)
    int K;               // input features
    int npairs;          // output row pairs
    const int16_t *x;    // input rows [kMaxRows][K]
    const int16_t *norm; // RMSNorm weights [K] (nullptr: no norm prologue)
    int32_t inv_elems;   // recip(fm(K)) in Q8.8
    int32_t inv_rms_const; // inv_rms when inv_elems == 0 (input-independent)
    const Step *step;
    int16_t *out;        // EPI_QKV: q [8][Hq]; EPI_RESID: hidden [8][Ho]; EPI_SILU: act [8][I]
    int out_stride;
    const int16_t *resid; // EPI_RESID residual rows [8][out_stride]
    int64_t *partial;    // EPI_PARTIAL [8][2*npairs]
    const int16_t *etab; // SiLU exp table (2049 entries, index raw+2048)
    // EPI_QKV
    int16_t *kc;         // K cache of this layer [kv_heads][max_seq][hd]
    int16_t *vc;
    const int16_t *rope; // [max_seq][hd]: cos half | sin half, Q8.8
    int hd;
    int q_pairs;         // pairs belonging to Q (local heads * hd/2)
    int kv_pairs;        // pairs of K (= of V) (kv_heads * hd/2)
    int max_seq;
    int stages;          // shared-memory ring stages G (gemv_stages)
    int units_per_chunk; // units B per stage / bulk copy
    int parts;           // warps sharing one unit along K (1, 2 or 4); G*B*parts consumer warps
    int *error;          // device word: nonzero after a bounded wait expired
    ArPeers ar;          // EPI_PARTIAL with ar.n > 1: push the sums to every rank
    uint32_t ar_off;     // EPI_PARTIAL: all-reduce number = step->ar_base + ar_off
    ArInput in;          // activation rows from a peer all-reduce (in.ar.n > 1) instead of x
    int row0;            // first row of this launch (x / out / resid already offset)
    // words [0, zero_n) of zero are cleared once the previous kernel has finished
    // (the fused attention's O sums, read by that kernel's prologue)
    int64_t *zero;
    int zero_n;
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};

// Tensor-core projection of blocks of 3..8 rows (mma_proj.cu): weights in
// "items" of 128 output rows x 128 inputs, high and low byte planes in the
// tensor cores' K-major core-matrix order (k_pack_mma).
constexpr int kMmaItemBytes = 2 * 128 * 128;
struct MmaArgs {
    const uint8_t *w;    // items of this projection, tile-major then K-chunk
    int K;               // input features (<= C * 128)
    int C;               // K-chunks of 128 inputs
    int T;               // tiles of 128 output rows
    int n_out;           // valid output units (EPI_RESID / PARTIAL: rows; EPI_SILU: FFN columns)
    const int16_t *x;    // input rows [kMaxRows][K]
    const int16_t *norm; // RMSNorm weights [K] (nullptr: none)
    int32_t inv_elems, inv_rms_const;
    const Step *step;
    int16_t *out;
    int out_stride;
    const int16_t *resid;
    int64_t *partial;
    const int16_t *etab;
    int16_t *kc, *vc;    // EPI_QKV: this layer's caches [kv_heads][max_seq][128]
    const int16_t *rope; // [max_seq][128]
    int q_tiles;         // EPI_QKV: tiles (heads) of Q; then kv_tiles of K, kv_tiles of V
    int kv_tiles;
    int max_seq;
    ArPeers ar;          // EPI_PARTIAL with ar.n > 1: push the sums to every rank
    uint32_t ar_off;
    int64_t *scratch;    // [grid][2][kMaxRows][128] partial sums of shared tiles
    int *tile_cnt;       // [T] arrivals at shared tiles (zero between launches)
    int stages;          // ring stages of kMmaItemBytes
    int max_items;       // items of the largest CTA range (activation slots)
    int *error;
    const int32_t *wsum; // [T][C+1][128] prefix over chunks of each tile row's weight sums (k_mma_wsum)
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};
cudaError_t launch_mma_proj(const MmaArgs &a, int epi, int grid, cudaStream_t s);
cudaError_t mma_configure(int max_smem_bytes);
size_t mma_smem_bytes(int stages, int max_items);
int mma_stages(int max_items, int max_smem);
cudaError_t launch_pack_mma(const int16_t *dense, int ld, int col0, int K, int C, const int32_t *rows_of, int T,
                            uint8_t *dst, cudaStream_t s);
cudaError_t launch_mma_wsum(const int16_t *dense, int ld, int col0, int K, int C, const int32_t *rows_of, int T,
                            int32_t *wsum, cudaStream_t s);

// CTAs per (row, query head) attention cluster: 8, or 16 (a non-portable size
// B200 supports) when few heads leave most SMs idle, so that the contexts
// longer than 16 tiles are spread 3 tiles per CTA instead of 5.
constexpr int kCluster = 8;
constexpr int kClusterWide = 16;
constexpr int kMaxTilesPerCta = 5;  // bounds the cluster's shared memory: max_seq <= 2560

struct AttnArgs {
    const int16_t *q;    // [8][q_heads*hd] post-RoPE queries of this rank
    const int16_t *kc;   // layer K cache [kv_heads][max_seq][hd]
    const int16_t *vc;
    int16_t *out;        // [8][q_heads*hd]
    const int16_t *ptab; // softmax exp table (2049 entries)
    const Step *step;
    int q_heads;         // query heads on this rank
    int first_head;      // global index of local head 0
    int gqa;             // query heads per KV head (model)
    int hd;
    int max_seq;
    int cluster;         // CTAs per cluster (kCluster or kClusterWide)
    int tpc_max;         // ceil(ceil(max_seq/64) / cluster): tiles per CTA at most
    int32_t qk_scale;    // accum(fm(1/sqrt(hd))) raw, Q16.16
    // Weights the next kernels stream (this layer's O, then Gate/Up), warmed into
    // L2 while attention leaves HBM idle: pf_per_tile bytes per 64-position tile
    // of the longest row's context (attention time grows with it), at most
    // pf_bytes, from pf; all multiples of 16.
    const char *pf;
    unsigned long long pf_bytes;
    unsigned long long pf_per_tile;
    int pf_late;         // issue it after the first cluster barrier (K and V in shared memory)
    int *error;          // device word: nonzero after a bounded wait expired
    // O projection fused (k_attn, one row): o_w = the layer's O weights, head-major
    // in the pair layout (head lh, O row j: hd/2 words at o_w + (lh*hidden + j)*hd/2),
    // o_rows = O rows per CTA (hidden / cluster); each cluster adds its head's
    // exact int64 partial of every O row into o_acc[row][hidden].
    // o_w == nullptr: the head output goes to out.
    const uint32_t *o_w;
    int o_rows;
    int hidden;
    int64_t *o_acc;
    int trigger_tiles;   // k_attn: let the next kernel launch at the start when the row's context exceeds
                         // this many 64-position tiles, else once PV is done
    // fused O on a tensor-parallel rank (k_attn<C, *, true>, LLMX_ATTN_FUSE_O_TP): the rank's exact O sums
    // go to every rank's exchange region as all-reduce number step->ar_base + ar_off, pushed by the last
    // of the rank's heads to finish each slice of O rows (arrivals counted in o_cnt[row][cluster CTA])
    ArPeers ar;
    uint32_t ar_off;
    int *o_cnt;
    int split_o;         // with o_w on 8-CTA clusters: the k_attn<C, true> variant (O slice in a buffer of
                         // its own from the start, no head-output exchange; LLMX_ATTN_SPLIT_O)
    int rows_inner;      // k_attn_rows: the row-inner loop order (LLMX_ATTN_ROWS_INNER)
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};

struct NormArgs {
    const int16_t *x;
    const int16_t *w;
    int16_t *y;
    int n;
    int32_t inv_elems;
    int32_t inv_rms_const;
    const Step *step;
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};

struct ResidArgs {  // round exact int64 sums + residual (after the TP all-reduce)
    const int64_t *partial;
    const int16_t *resid;
    int16_t *out;
    int n;
    const Step *step;
    int64_t *clear;      // non-null (== partial): each sum is cleared once read (the fused O sums)
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};

// Per-operator (feature) kernels, feature.cu.  Slot orders of the packed
// layout: output column o of the operator is sum column feature_slot(o).
enum SlotOrder : int {
    kSlotIdentity = 0,   // O, Down
    kSlotRopePairs = 1,  // Q, K, V: head h, pair i -> slots h*hd + 2i (i < hd/2), + 1 (i + hd/2)
    kSlotEven = 2,       // Gate of the interleaved Gate/Up slots
    kSlotOdd = 3         // Up
};
struct FeatureRoundArgs {  // out[r][o] = round_mac(sums[r][slot(o)])
    const int64_t *sums;
    int sum_stride;
    int16_t *out;
    int rows;
    int n_out;
    int order;
    int hd;
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};
struct FeatureVecArgs {  // out = silu ? SiLU(lhs) x rhs : sat16(lhs + rhs), n elements
    const int16_t *lhs;
    const int16_t *rhs;
    int16_t *out;
    const int16_t *etab;
    int n;
    int silu;
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};
cudaError_t launch_feature_round(const FeatureRoundArgs &a, cudaStream_t s);
cudaError_t launch_feature_vec(const FeatureVecArgs &a, cudaStream_t s);

struct ArFinishArgs {  // wait for every rank's sums, add them, round, + residual
    ArPeers ar;
    uint32_t ar_off;
    const int16_t *resid;
    int16_t *out;
    const Step *step;
    int *error;
    LLMX_TL_FIELD        // timeline builds only: this launch's slot
};
cudaError_t launch_ar_finish(const ArFinishArgs &a, cudaStream_t s);

// Launchers (stream-ordered, programmatic-dependent launch enabled).
cudaError_t launch_proj(const ProjArgs &a, int epi, int rows_tmpl, int grid, cudaStream_t s);
cudaError_t launch_attn(const AttnArgs &a, int rows, cudaStream_t s);
// tp: also the tensor-parallel fused-O instantiations (LLMX_ATTN_FUSE_O_TP)
cudaError_t attn_configure(int max_smem_bytes, int cluster, bool tp = false);
// The split variant of the fused one-row kernel (8-CTA clusters): sets its shared
// memory limit; *ok = 1 when every cluster of a grid of q_heads clusters fits at once.
cudaError_t attn_split_configure(int smem_bytes, int q_heads, int *ok);
// Blocks of several rows: one cluster per query head for all rows (K/V read once).
cudaError_t launch_attn_rows(const AttnArgs &a, cudaStream_t s);
cudaError_t attn_rows_configure(int max_smem_bytes, int cluster);
size_t attn_rows_smem_bytes(int tpc, int cluster);
size_t attn_smem_bytes(int tpc, int hd, int cluster, int o_rows, bool split = false);
cudaError_t launch_rmsnorm(const NormArgs &a, int rows, cudaStream_t s);
cudaError_t launch_round_resid(const ResidArgs &a, int rows, cudaStream_t s);
// carveout: preferred shared-memory carveout in percent for every projection
// kernel, or -1 to leave the driver's choice
cudaError_t proj_configure(int max_smem_bytes, int carveout);
size_t gemv_smem_bytes(int rows_tmpl, int epi, int K, int stages, int units_per_chunk, int parts);
int gemv_stages(int rows_tmpl, int epi, int K, int max_smem, int ring_bytes, int *units_per_chunk, int *parts,
                int max_warps);

// Weight layout kernel (model upload): slot s of the destination receives
// dense row row_of_slot[s], columns [col0, col0+K), as K/2 32-bit words; word j
// holds bytes {lo(w[2j]), lo(w[2j+1]), hi(w[2j]), hi(w[2j+1])} so that one dp2a.lo
// (unsigned low bytes) plus one dp2a.hi (signed high bytes) form two exact
// int16 x int16 products against a packed pair of activations.
cudaError_t launch_pack_pairs(const int16_t *dense, int ld, int col0, int K,
                              const int32_t *row_of_slot, int nslots, uint32_t *dst,
                              cudaStream_t s);

// Greedy generation on the device (lm_head.cu, kernels.cu).  LM-head argmax
// over caller-owned scratch of lm_argmax_scratch_bytes(); token-embedding
// gather of rows tokens[0..rows) (a token id >= vocab sets *err to
// kErrTokenRange and writes a zero row).
constexpr int kErrTokenRange = 7;
size_t lm_argmax_scratch_bytes();
cudaError_t launch_lm_argmax(const int16_t *h, int rows, int hidden, const int16_t *w, unsigned vocab,
                             uint32_t *tokens, void *scratch, int nsm, cudaStream_t s);
cudaError_t launch_embed_rows(const int16_t *table, const uint32_t *tokens, int rows, int hidden, unsigned vocab,
                              int16_t *out, int *err, cudaStream_t s);

// Message returned by llmx_last_error() on this thread.
void set_last_error(const std::string &msg);

}  // namespace llmx
