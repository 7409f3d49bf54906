// LM-head argmax on the GPU for callers that must not allocate device memory.
//
// The host path (model_data_t::lm_head_argmax, host/host_qwen_8x64.cpp:937-977)
// scores every vocabulary row with an exact int64 dot product against one
// final-normed hidden row and keeps the first maximum.  This file computes the
// same tokens on the device.  It is meant for callers that cannot allocate at
// the point where they sample: a serving loop whose HBM is already committed
// in full to weights and KV cache (an allocation there fails or evicts), and
// code that runs between tokens on several streams, where cudaMalloc/cudaFree
// would serialise the whole device.  So the entry point allocates nothing.
// Its per-block partial results live in one file-scope device array; every
// call on a device shares that array.
//
// Kernels: k_lm_scan (one pass over the LM head; each block keeps the best
// (score, token) per row of its contiguous vocabulary range) and k_lm_pick
// (one block reduces the block results in vocabulary order).
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <mutex>
#include <string>

#include "llmx.h"
#include "device_util.cuh"
#include "kernels.cuh"

namespace {

constexpr int kPickRows = 8;           // rows per call (the controller's block size)
constexpr int kScanBlocks = 1024;      // upper bound of the scan grid
constexpr int kScanThreads = 256;
constexpr int kScanBlocksPerSm = 2;    // resident scan blocks per SM (about 100 registers a thread)
constexpr int kMaxDevices = 64;

struct Best {
    long long score;
    unsigned int token;
    unsigned int pad;
};

// Scratch: Best[row][block], 8 x 1024 x 16 B = 128 KiB per device.  Every slot
// that k_lm_pick reads is written by k_lm_scan earlier in the same call, so
// nothing in it has to start at zero and nothing is cleared between calls.
static __device__ __align__(256) Best g_pick_scratch[kPickRows * kScanBlocks];

// Better = higher score; among equal scores the lower token (the first
// maximum of a scan in vocabulary order).
static __device__ __forceinline__ bool better(long long s, unsigned t, long long bs, unsigned bt) {
    return s > bs || (s == bs && t < bt);
}

static __device__ __forceinline__ long long dot8(uint4 h, uint4 w) {
    const uint32_t hv[4] = {h.x, h.y, h.z, h.w}, wv[4] = {w.x, w.y, w.z, w.w};
    long long s = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        s += (long long)(int32_t)llmx::lo16(hv[k]) * (int32_t)llmx::lo16(wv[k]);
        s += (long long)(int32_t)llmx::hi16(hv[k]) * (int32_t)llmx::hi16(wv[k]);
    }
    return s;
}

// Each warp scores V consecutive vocabulary rows per iteration, with every
// 16-byte load of those rows (8 per lane per 4 KiB row) issued before the dot
// products, so that enough of the table is in flight to stream it at HBM rate.
template <int R>
__global__ void __launch_bounds__(kScanThreads, kScanBlocksPerSm)
    k_lm_scan(const int16_t *__restrict__ h, int hidden, const int16_t *__restrict__ w, unsigned vocab, int rows,
              Best *__restrict__ part) {
    constexpr int V = R <= 2 ? 2 : 1;  // vocabulary rows per warp iteration
    constexpr int J = 8;               // 16-byte loads per lane per row and chunk
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const unsigned v0 = (unsigned)((unsigned long long)vocab * blockIdx.x / gridDim.x);
    const unsigned v1 = (unsigned)((unsigned long long)vocab * (blockIdx.x + 1) / gridDim.x);
    const int nvec = hidden >> 3;
    const uint4 *h4 = reinterpret_cast<const uint4 *>(h);
    long long best[R];
    unsigned arg[R];
#pragma unroll
    for (int r = 0; r < R; r++) {
        best[r] = LLONG_MIN;
        arg[r] = 0xffffffffu;
    }
    for (unsigned v = v0 + (unsigned)warp * V; v < v1; v += (unsigned)nw * V) {
        long long acc[V][R];
#pragma unroll
        for (int u = 0; u < V; u++)
#pragma unroll
            for (int r = 0; r < R; r++) acc[u][r] = 0;
        for (int kb = 0; kb < nvec; kb += 32 * J) {
            uint4 wv[V][J];
#pragma unroll
            for (int u = 0; u < V; u++) {
                const uint4 *wr = reinterpret_cast<const uint4 *>(w + (size_t)(v + u) * hidden);
#pragma unroll
                for (int j = 0; j < J; j++) {
                    const int k = kb + j * 32 + lane;
                    wv[u][j] = (k < nvec && v + u < v1) ? llmx::ld_stream(wr + k) : make_uint4(0, 0, 0, 0);
                }
            }
#pragma unroll
            for (int j = 0; j < J; j++) {
                const int k = kb + j * 32 + lane;
                if (k < nvec) {
#pragma unroll
                    for (int r = 0; r < R; r++)
                        if (r < rows) {
                            const uint4 hv = __ldg(h4 + (size_t)r * nvec + k);
#pragma unroll
                            for (int u = 0; u < V; u++) acc[u][r] += dot8(hv, wv[u][j]);
                        }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < V; u++) {
#pragma unroll
            for (int r = 0; r < R; r++) {
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) acc[u][r] += llmx::shfl_xor64(acc[u][r], o);
                // this warp visits its tokens in increasing order: '>' keeps the first maximum
                if (v + u < v1 && acc[u][r] > best[r]) {
                    best[r] = acc[u][r];
                    arg[r] = v + u;
                }
            }
        }
    }
    __shared__ long long sb[kScanThreads / 32][R];
    __shared__ unsigned st[kScanThreads / 32][R];
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < R; r++) {
            sb[warp][r] = best[r];
            st[warp][r] = arg[r];
        }
    }
    __syncthreads();
    if (threadIdx.x < rows) {
        const int r = threadIdx.x;
        long long bs = LLONG_MIN;
        unsigned bt = 0xffffffffu;
        for (int q = 0; q < nw; q++)
            if (st[q][r] != 0xffffffffu && better(sb[q][r], st[q][r], bs, bt)) {
                bs = sb[q][r];
                bt = st[q][r];
            }
        part[(size_t)r * kScanBlocks + blockIdx.x] = Best{bs, bt, 0u};
    }
}

__global__ void __launch_bounds__(kPickRows * 32) k_lm_pick(const Best *__restrict__ part, int nblocks, int rows,
                                                           uint32_t *__restrict__ tokens) {
    const int r = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (r >= rows) return;
    long long bs = LLONG_MIN;
    unsigned bt = 0xffffffffu;
    for (int b = lane; b < nblocks; b += 32) {
        const Best p = part[(size_t)r * kScanBlocks + b];
        if (p.token != 0xffffffffu && better(p.score, p.token, bs, bt)) {
            bs = p.score;
            bt = p.token;
        }
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const long long os = llmx::shfl_xor64(bs, o);
        const unsigned ot = __shfl_xor_sync(0xffffffffu, bt, o);
        if (ot != 0xffffffffu && (bt == 0xffffffffu || better(os, ot, bs, bt))) {
            bs = os;
            bt = ot;
        }
    }
    if (lane == 0) tokens[r] = bt;
}

// Per-device set-up: the scratch array's device address and the SM count,
// looked up once with that device current.
struct DeviceSetup {
    bool ready = false;
    Best *scratch = nullptr;
    int nsm = 0;
};
std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];

int fail(int code, const std::string &msg) {
    llmx::set_last_error(msg);
    return code;
}

template <int R>
cudaError_t launch_scan(const int16_t *h, int hidden, const int16_t *w, unsigned vocab, int rows, Best *part,
                        int grid, cudaStream_t s) {
    k_lm_scan<R><<<grid, kScanThreads, 0, s>>>(h, hidden, w, vocab, rows, part);
    return cudaGetLastError();
}

}  // namespace

// The same two kernels on scratch owned by the caller (a context's generate
// loop), so that contexts on different streams never share partial results.
size_t llmx::lm_argmax_scratch_bytes() { return sizeof(Best) * kPickRows * kScanBlocks; }

cudaError_t llmx::launch_lm_argmax(const int16_t *h, int rows, int hidden, const int16_t *w, unsigned vocab,
                                   uint32_t *tokens, void *scratch, int nsm, cudaStream_t s) {
    if (rows < 1 || rows > kPickRows) return cudaErrorInvalidValue;
    long long grid = (long long)nsm * kScanBlocksPerSm;
    if (grid > kScanBlocks) grid = kScanBlocks;
    if (grid > (long long)vocab) grid = vocab;
    Best *part = static_cast<Best *>(scratch);
    cudaError_t e;
    switch (rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8) {
    case 1: e = launch_scan<1>(h, hidden, w, vocab, rows, part, (int)grid, s); break;
    case 2: e = launch_scan<2>(h, hidden, w, vocab, rows, part, (int)grid, s); break;
    case 4: e = launch_scan<4>(h, hidden, w, vocab, rows, part, (int)grid, s); break;
    default: e = launch_scan<8>(h, hidden, w, vocab, rows, part, (int)grid, s); break;
    }
    if (e != cudaSuccess) return e;
    k_lm_pick<<<1, kPickRows * 32, 0, s>>>(part, (int)grid, rows, tokens);
    return cudaGetLastError();
}

extern "C" int llmx_lm_head_argmax_device(const int16_t *hidden, uint32_t rows, uint32_t hidden_size,
                                          const int16_t *lm_head, uint32_t vocab, uint32_t *tokens,
                                          void *stream) {
    if (!hidden || !lm_head || !tokens) return fail(LLMX_ERR_ARG, "lm_head_argmax_device: null pointer");
    if (rows == 0 || rows > (uint32_t)kPickRows)
        return fail(LLMX_ERR_ARG, "lm_head_argmax_device: rows must be 1..8 (the scratch array holds 8 rows), got " +
                                      std::to_string(rows));
    if (hidden_size == 0 || hidden_size % 8 != 0 || hidden_size > (1u << 20))
        return fail(LLMX_ERR_ARG, "lm_head_argmax_device: hidden_size must be a positive multiple of 8 up to 2^20");
    if (vocab == 0 || vocab > (uint32_t)INT_MAX)
        return fail(LLMX_ERR_ARG, "lm_head_argmax_device: vocab must be 1..2^31-1");
    if (((uintptr_t)hidden | (uintptr_t)lm_head) & 15u)
        return fail(LLMX_ERR_ARG, "lm_head_argmax_device: hidden and lm_head must be 16-byte aligned");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return fail(LLMX_ERR_UNSUPPORTED, "lm_head_argmax_device: device ordinal >= 64");
    DeviceSetup su;
    {
        std::lock_guard<std::mutex> lock(g_setup_mu);
        if (!g_setup[dev].ready) {
            void *p = nullptr;
            e = cudaGetSymbolAddress(&p, g_pick_scratch);
            if (e != cudaSuccess)
                return fail(LLMX_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            int nsm = 0;
            e = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess)
                return fail(LLMX_ERR_CUDA, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
            g_setup[dev].scratch = static_cast<Best *>(p);
            g_setup[dev].nsm = nsm;
            g_setup[dev].ready = true;
        }
        su = g_setup[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // one wave of resident blocks (each warp keeps two 4 KiB rows in flight);
    // never more blocks than the scratch holds or than vocabulary rows
    long long grid = (long long)su.nsm * kScanBlocksPerSm;
    if (grid > kScanBlocks) grid = kScanBlocks;
    if (grid > (long long)vocab) grid = vocab;
    const int R = rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8;
    switch (R) {
    case 1: e = launch_scan<1>(hidden, (int)hidden_size, lm_head, vocab, (int)rows, su.scratch, (int)grid, s); break;
    case 2: e = launch_scan<2>(hidden, (int)hidden_size, lm_head, vocab, (int)rows, su.scratch, (int)grid, s); break;
    case 4: e = launch_scan<4>(hidden, (int)hidden_size, lm_head, vocab, (int)rows, su.scratch, (int)grid, s); break;
    default: e = launch_scan<8>(hidden, (int)hidden_size, lm_head, vocab, (int)rows, su.scratch, (int)grid, s); break;
    }
    if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("k_lm_scan: ") + cudaGetErrorString(e));
    k_lm_pick<<<1, kPickRows * 32, 0, s>>>(su.scratch, (int)grid, (int)rows, tokens);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(LLMX_ERR_CUDA, std::string("k_lm_pick: ") + cudaGetErrorString(e));
    return LLMX_OK;
}
