// Internal declarations shared by the host-side translation units.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include "llmx.h"

struct llmx_model {
    llmx_shape shape{};
    std::vector<std::vector<int16_t>> layers;  // dense blobs Q,K,V,O,Gate,Up,Down [out][in]
    std::vector<int16_t> norms;                // [2L+1][hidden]
    std::vector<int16_t> embedding;            // [vocab][hidden] (may be empty: generated rows)
    std::vector<int16_t> lm_head;              // untied LM head (empty when tied)
    bool tied = true;
    int kind = 0;  // 0 empty, 1 reference random, 2 synthetic Gaussian, 3 packed checkpoint
    uint64_t gseed = 0;
    double w_sigma = 0.0;
};

namespace llmx {

size_t layer_elems(const llmx_shape &s);
void layer_offsets(const llmx_shape &s, size_t off[8]);
int host_threads();

// Streams of the synthetic Gaussian model (seeded benchmark workload).
constexpr uint64_t kGaussStreamEmbedding = 0x10;
constexpr uint64_t kGaussStreamLmHead = 0x20;
inline uint64_t gauss_stream_layer(int layer, int op) { return 0x1000 + (uint64_t)layer * 16 + (uint64_t)op; }

struct GaussSampler {
    std::vector<uint64_t> thr;
    std::vector<int32_t> guide;
    int kmin = 0;
    explicit GaussSampler(double sigma_raw);
    void fill(uint64_t seed, uint64_t stream, uint64_t index0, int16_t *out, size_t n, int threads) const;
};

// The model's [vocab][hidden] token-embedding table, materialised first for a
// synthetic model whose rows are otherwise generated on demand; nullptr when the
// model has none.  The LM head is that table when tied, else the separate head.
const int16_t *model_embedding_table(llmx_model *m);
const int16_t *model_lm_head_table(llmx_model *m);

// Tables shared by every context (host-built, uploaded once).
void build_exp_tables(int16_t *e16_8, int16_t *p18_4);
void build_rope_table(int head_dim, int max_seq, int16_t *table);
int32_t qk_scale_q1616(int head_dim);

}  // namespace llmx

extern "C" int llmx_gauss_fill(uint64_t seed, uint64_t stream, double sigma_raw, uint64_t index0,
                               int16_t *out, size_t n);
