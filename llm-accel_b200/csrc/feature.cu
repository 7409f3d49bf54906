// Per-operator (feature) kernels: the reference controller's legacy operator
// modes 1-10 (kernel/control_cache_8x64.cpp:20-132, scheduler :7273-7497),
// driven on the host by run_feature (host/host_qwen_8x64.cpp:1088-1130).
//
// A single projection (ops 1-7) runs the resident weight-streaming kernel
// (gemv.cu) on the matrix's slots of the packed layer blob with the
// exact-sum epilogue, then k_feature_round rounds each sum once to Q8.8
// (golden_projection host:3105-3142, the same double rounding as the fused
// epilogues) and undoes the slot order of the packed layout: Q/K/V rows are
// stored as RoPE pairs (i, i + hd/2) of each head, Gate/Up rows interleaved.
// RMSNorm (op 8) is the Task 20 kernel with the caller's weight row; SiLU-Mul
// (op 9) and the residual add (op 10) are k_feature_vec.
#include <cuda_runtime.h>

#include "device_util.cuh"
#include "fixed.cuh"
#include "kernels.cuh"
#include "gemv_common.cuh"

namespace llmx {

// output column o of the operator -> slot of the computed range
static __device__ __forceinline__ int feature_slot(int o, int order, int hd) {
    switch (order) {
    case kSlotRopePairs: {
        const int half = hd >> 1, head = o / hd, d = o - head * hd;
        const int i = d < half ? d : d - half;
        return head * hd + 2 * i + (d < half ? 0 : 1);
    }
    case kSlotEven: return 2 * o;
    case kSlotOdd: return 2 * o + 1;
    default: return o;
    }
}

__global__ void __launch_bounds__(256) k_feature_round(const FeatureRoundArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    pdl_wait();
    pdl_trigger();
    const int total = a.rows * a.n_out;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int r = i / a.n_out, o = i - r * a.n_out;
        a.out[i] = (int16_t)round_mac(a.sums[(size_t)r * a.sum_stride + feature_slot(o, a.order, a.hd)]);
    }
}

cudaError_t launch_feature_round(const FeatureRoundArgs &a, cudaStream_t s) {
    FeatureRoundArgs c = a;
    LLMX_TL_TAKE(c, "feature_round");
    void *args[] = {&c};
    int blocks = (a.rows * a.n_out + 255) / 256;
    if (blocks < 1) blocks = 1;
    return launch_pdl((const void *)k_feature_round, dim3(blocks), dim3(256), args, s);
}

// SiLU(lhs) x rhs (stream_silu_mul kernel/compute_stream.cpp:123-164) or the
// saturating residual add (stream_add :205-225), element by element.
__global__ void __launch_bounds__(256) k_feature_vec(const FeatureVecArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
        const int32_t x = a.lhs[i], y = a.rhs[i];
        a.out[i] = (int16_t)(a.silu ? silu_mul(x, y, a.etab) : sat16(x + y));
    }
}

cudaError_t launch_feature_vec(const FeatureVecArgs &a, cudaStream_t s) {
    FeatureVecArgs c = a;
    LLMX_TL_TAKE(c, "feature_vec");
    void *args[] = {&c};
    int blocks = (a.n + 255) / 256;
    if (blocks < 1) blocks = 1;
    return launch_pdl((const void *)k_feature_vec, dim3(blocks), dim3(256), args, s);
}

}  // namespace llmx

LLMX_TL_READER(feature)
