// Host-side model container, generators, checkpoint loader and LM head of the
// resident decoder-layer path (model_data_t, host/host_qwen_8x64.cpp:779-1022).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <limits>
#include <new>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "host_model.h"

namespace llmx {

// --------------------------------------------------------------------------
// shapes
// --------------------------------------------------------------------------
size_t layer_elems(const llmx_shape &s) {
    const size_t H = s.hidden, I = s.inter, KV = (size_t)s.kv_heads * (s.hidden / s.heads);
    return 2 * H * H + 2 * KV * H + 3 * I * H;
}

void layer_offsets(const llmx_shape &s, size_t off[8]) {
    const size_t H = s.hidden, I = s.inter, KV = (size_t)s.kv_heads * (s.hidden / s.heads);
    const size_t sz[7] = {H * H, KV * H, KV * H, H * H, I * H, I * H, H * I};
    off[0] = 0;
    for (int i = 0; i < 7; i++) off[i + 1] = off[i] + sz[i];
}

int host_threads() {
    const unsigned n = std::thread::hardware_concurrency();
    return n == 0 ? 1 : (int)std::min(n, 64u);
}

template <typename F>
static void parallel_for(size_t n, int threads, F fn) {
    if (threads <= 1 || n < 4096) {
        fn(0, n);
        return;
    }
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; t++) {
        const size_t b = n * t / threads, e = n * (t + 1) / threads;
        pool.emplace_back([=, &fn] { fn(b, e); });
    }
    for (auto &th : pool) th.join();
}

// --------------------------------------------------------------------------
// N(0, sigma) fixed-point sampler.  Definition (shared with the test oracle):
// element i of stream (seed, stream) is the smallest integer k with U < T(k),
// U = top 32 bits of splitmix64(key + i), key = splitmix64(seed ^ stream*C),
// T(k) = round(2^32 Phi((k + 1/2)/sigma_raw)), i.e. round-half-up quantisation
// (AP_RND) of a Gaussian at the resolution of U.  A 4096-bucket guide table
// makes each draw O(1).
// --------------------------------------------------------------------------
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

GaussSampler::GaussSampler(double sigma_raw) {
    int K = (int)std::ceil(8.0 * sigma_raw);
    if (K > 32767) K = 32767;
    const int n = 2 * K + 1;
    thr.resize(n);
    for (int j = 0; j < n - 1; j++) {
        const int k = j - K;
        const double x = ((double)k + 0.5) / sigma_raw;
        const double phi = 0.5 * std::erfc(-x * 0.70710678118654752440);
        thr[j] = (uint64_t)std::llround(std::ldexp(phi, 32));
    }
    thr[n - 1] = (uint64_t)1 << 32;
    kmin = -K;
    guide.resize(4096);
    int j = 0;
    for (int b = 0; b < 4096; b++) {
        const uint64_t lo = (uint64_t)b << 20;
        while (thr[j] <= lo) j++;
        guide[b] = j;
    }
}

void GaussSampler::fill(uint64_t seed, uint64_t stream, uint64_t index0, int16_t *out, size_t n,
                        int threads) const {
    const uint64_t key = mix64(seed ^ (stream * 0xD1B54A32D192ED03ull));
    parallel_for(n, threads, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; i++) {
            const uint64_t u = mix64(key + index0 + i) >> 32;
            int j = guide[u >> 20];
            while (u >= thr[j]) j++;
            out[i] = (int16_t)(j + kmin);
        }
    });
}

// --------------------------------------------------------------------------
// reference random model: std::mt19937 with the libstdc++-9 (Ubuntu 20.04)
// uniform_int_distribution<int> algorithm ("division downscaling": draw
// r < past = range' * floor((2^32-1)/range'), return r / scaling + lo).
// initialize_random_model host:842-869 draws embedding, norms, then the 16
// weight shards word by word (32 lanes per 512-bit word).
// --------------------------------------------------------------------------
struct Uniform9 {
    uint64_t scaling, past;
    int lo;
    Uniform9(int a, int b) {
        const uint64_t urng = 0xffffffffull, range = (uint64_t)((int64_t)b - a) + 1;
        scaling = urng / range;
        past = range * scaling;
        lo = a;
    }
    int operator()(std::mt19937 &g) const {
        uint64_t r;
        do r = g();
        while (r >= past);
        return (int)(r / scaling) + lo;
    }
};

// Tile/shard geometry of projection_weight_raw host:899-935.
struct ShardGeom {
    size_t base[8], in_tiles[7], dense_off[8];
    int od[7], id[7];
    size_t layer_tiles, shard_words;
    explicit ShardGeom(const llmx_shape &s) {
        const int H = s.hidden, I = s.inter, KV = s.kv_heads * (s.hidden / s.heads);
        const int o[7] = {H, KV, KV, H, I, I, H}, i[7] = {H, H, H, H, H, H, I};
        base[0] = 0;
        dense_off[0] = 0;
        for (int k = 0; k < 7; k++) {
            od[k] = o[k];
            id[k] = i[k];
            in_tiles[k] = (size_t)(i[k] + 15) / 16;
            base[k + 1] = base[k] + ((size_t)(o[k] + 15) / 16) * in_tiles[k];
            dense_off[k + 1] = dense_off[k] + (size_t)o[k] * i[k];
        }
        layer_tiles = base[7];
        shard_words = (layer_tiles * (size_t)s.layers + 1) / 2;
    }
    // Decode word `word` of shard `shard` (32 lanes) into dense layer blobs.
    template <typename Store>
    void decode(int shard, size_t word, const int16_t *lanes, Store store) const {
        const int group = shard / 8, tile_word = shard % 8;
        const size_t gtile = 2 * word + (size_t)group;
        const size_t layer = gtile / layer_tiles, t = gtile % layer_tiles;
        int op = 0;
        while (op < 6 && t >= base[op + 1]) op++;
        const size_t local = t - base[op];
        const size_t trow = local / in_tiles[op], tcol = local % in_tiles[op];
        for (int lane = 0; lane < 32; lane++) {
            const int lt = tile_word * 32 + lane;
            const size_t out = trow * 16 + (size_t)(lt / 16), in = tcol * 16 + (size_t)(lt % 16);
            if (out < (size_t)od[op] && in < (size_t)id[op])
                store(layer, dense_off[op] + out * (size_t)id[op] + in, lanes[lane]);
        }
    }
};

}  // namespace llmx

using namespace llmx;

// --------------------------------------------------------------------------
// C ABI: model container
// --------------------------------------------------------------------------
const int16_t *llmx::model_embedding_table(llmx_model *m) {
    const llmx_shape &s = m->shape;
    if (m->embedding.empty() && m->kind == 2) {
        // synthetic model: materialise the N(0, 1) Q8.8 rows once
        m->embedding.resize((size_t)s.vocab * s.hidden);
        const GaussSampler emb(256.0);
        emb.fill(m->gseed, kGaussStreamEmbedding, 0, m->embedding.data(), m->embedding.size(), host_threads());
    }
    return m->embedding.empty() ? nullptr : m->embedding.data();
}

const int16_t *llmx::model_lm_head_table(llmx_model *m) {
    if (!m->tied) return m->lm_head.empty() ? nullptr : m->lm_head.data();
    return model_embedding_table(m);
}

extern "C" {

size_t llmx_layer_weight_elems(const llmx_shape *shape) { return shape ? layer_elems(*shape) : 0; }

int llmx_model_create(const llmx_shape *shape, llmx_model **out) {
    if (!shape || !out) return LLMX_ERR_ARG;
    const int v = llmx_shape_validate(shape);
    if (v) return v;
    llmx_model *m = new (std::nothrow) llmx_model();
    if (!m) return LLMX_ERR_NOMEM;
    m->shape = *shape;
    *out = m;
    return LLMX_OK;
}

void llmx_model_destroy(llmx_model *m) { delete m; }

static int alloc_layers(llmx_model *m, int keep) {
    try {
        m->layers.assign(keep, {});
        for (auto &l : m->layers) l.assign(layer_elems(m->shape), 0);
        m->norms.assign(((size_t)m->shape.layers * 2 + 1) * m->shape.hidden, 0);
    } catch (const std::bad_alloc &) {
        return LLMX_ERR_NOMEM;
    }
    return LLMX_OK;
}

int llmx_model_init_reference_random(llmx_model *m, uint32_t seed, int keep_layers) {
    if (!m) return LLMX_ERR_ARG;
    const llmx_shape &s = m->shape;
    const int keep = keep_layers <= 0 ? s.layers : std::min(keep_layers, s.layers);
    int rc = alloc_layers(m, keep);
    if (rc) return rc;
    try {
        m->embedding.assign((size_t)s.vocab * s.hidden, 0);
    } catch (const std::bad_alloc &) {
        return LLMX_ERR_NOMEM;
    }
    m->lm_head.clear();
    m->tied = true;
    m->kind = 1;
    std::mt19937 g(seed);
    const Uniform9 feat(-128, 128), nrm(224, 288), wt(-64, 64);
    for (auto &v : m->embedding) v = (int16_t)feat(g);
    for (auto &v : m->norms) v = (int16_t)nrm(g);
    const ShardGeom geo(s);
    const size_t keep_words = (geo.layer_tiles * (size_t)keep + 1) / 2;
    int16_t lanes[32];
    for (int shard = 0; shard < 16; shard++) {
        for (size_t w = 0; w < geo.shard_words; w++) {
            for (int l = 0; l < 32; l++) lanes[l] = (int16_t)wt(g);
            if (w < keep_words)
                geo.decode(shard, w, lanes, [&](size_t layer, size_t idx, int16_t v) {
                    if (layer < (size_t)keep) m->layers[layer][idx] = v;
                });
        }
    }
    return LLMX_OK;
}

int llmx_model_init_gaussian(llmx_model *m, uint64_t seed, double w_sigma, int lm_head) {
    if (!m || !(w_sigma > 0)) return LLMX_ERR_ARG;
    const llmx_shape &s = m->shape;
    int rc = alloc_layers(m, s.layers);
    if (rc) return rc;
    m->kind = 2;
    m->gseed = seed;
    m->w_sigma = w_sigma;
    m->embedding.clear();
    const GaussSampler ws(w_sigma * 4096.0);
    const int threads = host_threads();
    size_t off[8];
    layer_offsets(s, off);
    for (int l = 0; l < s.layers; l++)
        for (int op = 0; op < 7; op++)
            ws.fill(seed, gauss_stream_layer(l, op), 0, m->layers[l].data() + off[op], off[op + 1] - off[op],
                    threads);
    std::fill(m->norms.begin(), m->norms.end(), (int16_t)256);
    if (lm_head) {
        try {
            m->lm_head.assign((size_t)s.vocab * s.hidden, 0);
        } catch (const std::bad_alloc &) {
            return LLMX_ERR_NOMEM;
        }
        ws.fill(seed, kGaussStreamLmHead, 0, m->lm_head.data(), m->lm_head.size(), threads);
        m->tied = false;
    } else {
        m->lm_head.clear();
        m->tied = true;
    }
    return LLMX_OK;
}

static bool read_exact(const std::string &path, void *dst, size_t bytes) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f.good() || (size_t)f.tellg() != bytes) return false;
    f.seekg(0);
    f.read(reinterpret_cast<char *>(dst), (std::streamsize)bytes);
    return (bool)f;
}

int llmx_model_load_packed(llmx_model *m, const char *dir, int tie_embeddings) {
    if (!m || !dir) return LLMX_ERR_ARG;
    const llmx_shape &s = m->shape;
    int rc = alloc_layers(m, s.layers);
    if (rc) return rc;
    const std::string d(dir);
    try {
        m->embedding.assign((size_t)s.vocab * s.hidden, 0);
    } catch (const std::bad_alloc &) {
        return LLMX_ERR_NOMEM;
    }
    // load_exact_file host:736-777: every file must have exactly the expected size.
    if (!read_exact(d + "/token_embedding.fix16.bin", m->embedding.data(), m->embedding.size() * 2))
        return LLMX_ERR_IO;
    if (!read_exact(d + "/norm_weights.fix16.bin", m->norms.data(), m->norms.size() * 2)) return LLMX_ERR_IO;
    const ShardGeom geo(s);
    std::vector<int16_t> shard(geo.shard_words * 32);
    for (int k = 0; k < 16; k++) {
        char name[64];
        std::snprintf(name, sizeof(name), "/layer_weights_shard%02d.fix16.bin", k);
        if (!read_exact(d + name, shard.data(), shard.size() * 2)) return LLMX_ERR_IO;
        for (size_t w = 0; w < geo.shard_words; w++)
            geo.decode(k, w, shard.data() + w * 32, [&](size_t layer, size_t idx, int16_t v) {
                if (layer < (size_t)s.layers) m->layers[layer][idx] = v;
            });
    }
    m->kind = 3;
    m->tied = tie_embeddings != 0;
    m->lm_head.clear();
    if (!m->tied) {
        m->lm_head.assign((size_t)s.vocab * s.hidden, 0);
        if (!read_exact(d + "/lm_head.fix16.bin", m->lm_head.data(), m->lm_head.size() * 2)) return LLMX_ERR_IO;
    }
    return LLMX_OK;
}

int16_t *llmx_model_layer(llmx_model *m, uint32_t layer) {
    if (!m || layer >= m->layers.size() || m->layers[layer].empty()) return nullptr;
    return m->layers[layer].data();
}
int16_t *llmx_model_norms(llmx_model *m) { return m && !m->norms.empty() ? m->norms.data() : nullptr; }
int16_t *llmx_model_embedding(llmx_model *m) {
    return m && !m->embedding.empty() ? m->embedding.data() : nullptr;
}

int llmx_model_embed(const llmx_model *m, const uint32_t *tokens, uint32_t n, int16_t *out) {
    if (!m || (!tokens && n) || (!out && n)) return LLMX_ERR_ARG;
    const llmx_shape &s = m->shape;
    for (uint32_t r = 0; r < n; r++) {
        if (tokens[r] >= (uint32_t)s.vocab) return LLMX_ERR_ARG;
        int16_t *dst = out + (size_t)r * s.hidden;
        if (!m->embedding.empty()) {
            std::memcpy(dst, m->embedding.data() + (size_t)tokens[r] * s.hidden, (size_t)s.hidden * 2);
        } else if (m->kind == 2) {
            // synthetic model: embedding rows N(0, 1) in Q8.8, generated on demand
            static const GaussSampler emb(256.0);
            emb.fill(m->gseed, kGaussStreamEmbedding, (uint64_t)tokens[r] * s.hidden, dst, s.hidden, 1);
        } else {
            return LLMX_ERR_STATE;
        }
    }
    return LLMX_OK;
}

int llmx_model_lm_head_argmax(const llmx_model *m, const int16_t *h, int threads, uint32_t *token) {
    if (!m || !h || !token) return LLMX_ERR_ARG;
    const llmx_shape &s = m->shape;
    const int16_t *w = model_lm_head_table(const_cast<llmx_model *>(m));
    if (!w) return LLMX_ERR_STATE;
    const int T = threads > 0 ? threads : host_threads();
    std::vector<int64_t> best(T, std::numeric_limits<int64_t>::min());
    std::vector<uint32_t> arg(T, 0);
    std::vector<std::thread> pool;
    for (int t = 0; t < T; t++) {
        pool.emplace_back([&, t] {
            const size_t b = (size_t)s.vocab * t / T, e = (size_t)s.vocab * (t + 1) / T;
            int64_t bs = std::numeric_limits<int64_t>::min();
            uint32_t bt = (uint32_t)b;
            for (size_t v = b; v < e; v++) {
                const int16_t *row = w + v * s.hidden;
                int64_t acc = 0;
                for (int i = 0; i < s.hidden; i++) acc += (int64_t)h[i] * row[i];
                if (acc > bs) {  // strict '>' keeps the first maximum (host:961-967)
                    bs = acc;
                    bt = (uint32_t)v;
                }
            }
            best[t] = bs;
            arg[t] = bt;
        });
    }
    for (auto &th : pool) th.join();
    int64_t bs = std::numeric_limits<int64_t>::min();
    uint32_t bt = 0;
    for (int t = 0; t < T; t++)
        if (best[t] > bs) {
            bs = best[t];
            bt = arg[t];
        }
    *token = bt;
    return LLMX_OK;
}

// Expose the synthetic sampler for tests that compare it with the oracle.
int llmx_gauss_fill(uint64_t seed, uint64_t stream, double sigma_raw, uint64_t index0, int16_t *out,
                    size_t n) {
    if (!out || !(sigma_raw > 0)) return LLMX_ERR_ARG;
    const GaussSampler g(sigma_raw);
    g.fill(seed, stream, index0, out, n, host_threads());
    return LLMX_OK;
}

}  // extern "C"
