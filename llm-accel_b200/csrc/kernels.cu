// Small kernels of the resident decoder-layer path: the final RMSNorm
// (Task 20), the tensor-parallel round-and-residual step and the weight layout
// kernel used at upload.  The projections live in gemv.cu, attention in
// attention.cu.
#include <cuda_runtime.h>

#include "device_util.cuh"
#include "fixed.cuh"
#include "kernels.cuh"
#include "gemv_common.cuh"

namespace llmx {

cudaError_t launch_pdl(const void *fn, dim3 grid, dim3 block, void **args, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// --------------------------------------------------------------------------
// Task 20: final RMSNorm of 1..8 rows (stream_rmsnorm compute_stream.cpp:227-288)
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(const NormArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    __shared__ int64_t red[8];
    __shared__ int32_t inv_s;
    const int rows = load_step(a.step).rows;
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int16_t *x = a.x + (size_t)r * a.n;
    if (a.inv_elems == 0) {
        if (threadIdx.x == 0) inv_s = a.inv_rms_const;
    } else {
        int64_t part = 0;
        for (int i = threadIdx.x; i < a.n; i += blockDim.x) part += (int64_t)x[i] * x[i];
        for (int o = 16; o >= 1; o >>= 1) part += shfl_xor64(part, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
        __syncthreads();
        if (threadIdx.x == 0) {
            int64_t s = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
            inv_s = inv_rms_q88(s > INT32_MAX ? INT32_MAX : (int32_t)s, a.inv_elems);
        }
    }
    __syncthreads();
    const int64_t inv = inv_s;
    for (int i = threadIdx.x; i < a.n; i += blockDim.x)
        a.y[(size_t)r * a.n + i] = (int16_t)sat16(rnd((int64_t)x[i] * inv * a.w[i], 16));
}

cudaError_t launch_rmsnorm(const NormArgs &a, int rows, cudaStream_t s) {
    NormArgs c = a;
    LLMX_TL_TAKE(c, "rmsnorm");
    void *args[] = {&c};
    return launch_pdl((const void *)k_rmsnorm, dim3(rows), dim3(256), args, s);
}

// --------------------------------------------------------------------------
// tensor parallel: round the all-reduced exact sums and add the residual
// --------------------------------------------------------------------------
__global__ void k_round_resid(const ResidArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    const int rows = load_step(a.step).rows;
    pdl_wait();
    pdl_trigger();
    const int total = rows * a.n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        a.out[i] = (int16_t)sat16((int32_t)a.resid[i] + round_mac(a.partial[i]));
        if (a.clear != nullptr) a.clear[i] = 0;
    }
}

// Peer all-reduce, receiving side, as a kernel of its own (single coarse
// tasks and the end of a stack; inside a stack the next projection's prologue
// does this): every thread waits (bounded) for the words of one element from
// every rank, adds the ranks' exact sums (order-free), rounds as round_mac and
// adds the residual -- the same result on every rank.
__global__ void __launch_bounds__(256) k_ar_finish(const ArFinishArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    const Step st = load_step(a.step);
    pdl_wait();
    pdl_trigger();
    __shared__ int fail_s;
    if (threadIdx.x == 0) fail_s = 0;
    __syncthreads();
    const uint32_t n = st.ar_base + a.ar_off;
    const int H = a.ar.hidden;
    const int i = 4 * (blockIdx.x * blockDim.x + threadIdx.x);  // 4 consecutive elements (H % 8 == 0)
    if (i >= st.rows * H) return;
    int64_t sum[4];
    if (!ar_gather4(a.ar, (int)(n & 1u), ar_tag(n), i / H, i % H, &fail_s, sum)) {
        if (!fail_s) atomicCAS(a.error, 0, kErrArTimeout);
        fail_s = 1;
        sum[0] = sum[1] = sum[2] = sum[3] = 0;
    }
#pragma unroll
    for (int j = 0; j < 4; j++) a.out[i + j] = (int16_t)sat16((int32_t)a.resid[i + j] + round_mac(sum[j]));
}

cudaError_t launch_ar_finish(const ArFinishArgs &a, cudaStream_t s) {
    ArFinishArgs c = a;
    LLMX_TL_TAKE(c, "ar_finish");
    void *args[] = {&c};
    return launch_pdl((const void *)k_ar_finish, dim3((kMaxRows * a.ar.hidden / 4 + 255) / 256), dim3(256), args, s);
}

cudaError_t launch_round_resid(const ResidArgs &a, int rows, cudaStream_t s) {
    ResidArgs c = a;
    LLMX_TL_TAKE(c, "round_resid");
    void *args[] = {&c};
    const int blocks = (rows * a.n + 255) / 256;
    return launch_pdl((const void *)k_round_resid, dim3(blocks), dim3(256), args, s);
}

// --------------------------------------------------------------------------
// token embedding gather (model_data_t::embedding host:871-884): one block per
// row, 16-byte copies of the table row of that row's token id
// --------------------------------------------------------------------------
__global__ void k_embed_rows(const int16_t *__restrict__ table, const uint32_t *__restrict__ tokens, int hidden,
                             unsigned vocab, int16_t *__restrict__ out, int *err) {
    const uint32_t t = tokens[blockIdx.x];
    uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)blockIdx.x * hidden);
    const int nvec = hidden >> 3;
    if (t >= vocab) {
        for (int i = threadIdx.x; i < nvec; i += blockDim.x) dst[i] = make_uint4(0, 0, 0, 0);
        if (threadIdx.x == 0) atomicExch(err, kErrTokenRange);
        return;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(table + (size_t)t * hidden);
    for (int i = threadIdx.x; i < nvec; i += blockDim.x) dst[i] = src[i];
}

cudaError_t launch_embed_rows(const int16_t *table, const uint32_t *tokens, int rows, int hidden, unsigned vocab,
                              int16_t *out, int *err, cudaStream_t s) {
    k_embed_rows<<<rows, 256, 0, s>>>(table, tokens, hidden, vocab, out, err);
    return cudaGetLastError();
}

// --------------------------------------------------------------------------
// weight layout
// --------------------------------------------------------------------------
__global__ void k_pack_pairs(const int16_t *__restrict__ dense, int ld, int col0, int K,
                             const int32_t *__restrict__ row_of_slot, int nslots,
                             uint32_t *__restrict__ dst) {
    const int KW = K >> 1;
    const size_t total = (size_t)nslots * KW;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int slot = (int)(i / KW);
        const int j = (int)(i - (size_t)slot * KW);
        const int16_t *row = dense + (size_t)row_of_slot[slot] * ld + col0;
        const uint32_t w0 = (uint16_t)row[2 * j], w1 = (uint16_t)row[2 * j + 1];
        dst[i] = (w0 & 0xffu) | ((w1 & 0xffu) << 8) | ((w0 >> 8) << 16) | ((w1 >> 8) << 24);
    }
}

cudaError_t launch_pack_pairs(const int16_t *dense, int ld, int col0, int K,
                              const int32_t *row_of_slot, int nslots, uint32_t *dst,
                              cudaStream_t s) {
    const size_t total = (size_t)nslots * (K >> 1);
    int blocks = (int)((total + 255) / 256);
    if (blocks > 65535 * 8) blocks = 65535 * 8;
    k_pack_pairs<<<blocks, 256, 0, s>>>(dense, ld, col0, K, row_of_slot, nslots, dst);
    return cudaGetLastError();
}

}  // namespace llmx

LLMX_TL_READER(kernels)
