// In-graph launch timeline for measurement builds (compiled with -DLLMX_TIMELINE,
// `python llm-accel_b200/build.py --timeline` -> libllmx_timeline.so).
//
// ncu runs every launch on its own with cold caches, so it cannot show how the
// kernels of a CUDA graph overlap under programmatic dependent launch, where the
// device idles between them, or how long a tensor-parallel rank waits for its
// peers.  In a timeline build every instrumented launch takes a slot number on
// the host when it is enqueued or captured into a graph (the slot is a member of
// the kernel's argument struct, so a graph replays the same slots), and its CTAs
// stamp %globaltimer into the slot: the earliest CTA start (thread 0 of every
// CTA, atomicMin) and the latest warp exit (lane 0 of every warp, atomicMax,
// from a guard object whose destructor runs on every return path).  The host
// clears the stamps, runs one step and reads them back (llmx_timeline_* in
// runtime.cu).  The default build compiles none of this: the macros below are
// empty and the argument structs are unchanged.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#ifdef LLMX_TIMELINE
#include <vector>

namespace llmx {

constexpr int kTlSlots = 8192;
struct TlEntry {
    unsigned long long start, end;  // %globaltimer ns; start = ~0 when the slot never ran
};

// One table per translation unit (no relocatable device code): only the unit
// that launched slot s writes entry s; the host merges the tables.
static __device__ TlEntry g_tl[kTlSlots];

static __device__ __forceinline__ unsigned long long tl_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

struct TlGuard {
    int slot;
    __device__ explicit TlGuard(int s) : slot(s) {
        if (slot >= 0 && slot < kTlSlots && threadIdx.x == 0) atomicMin(&g_tl[slot].start, tl_now());
    }
    __device__ ~TlGuard() {
        if (slot >= 0 && slot < kTlSlots && (threadIdx.x & 31) == 0) atomicMax(&g_tl[slot].end, tl_now());
    }
};

// Host: the next slot, recorded under `name` (runtime.cu); -1 once the slots run out.
int tl_take(const char *name);

// Host: clear (reset != 0: start = ~0, end = 0) or read this unit's table.
static inline cudaError_t tl_table(TlEntry *out, int n, int reset) {
    if (reset) {
        std::vector<TlEntry> init(kTlSlots, TlEntry{~0ull, 0ull});
        return cudaMemcpyToSymbol(g_tl, init.data(), sizeof(TlEntry) * kTlSlots);
    }
    return cudaMemcpyFromSymbol(out, g_tl, sizeof(TlEntry) * (size_t)(n < kTlSlots ? n : kTlSlots));
}

}  // namespace llmx

#define LLMX_TL_FIELD int tl_slot = -1;
#define LLMX_TL_PARAM , int tl_slot
#define LLMX_TL_ARG(name) , ::llmx::tl_take(name)
#define LLMX_TL_GUARD(slot) ::llmx::TlGuard tl_guard_(slot)
#define LLMX_TL_TAKE(args, name) ((args).tl_slot = ::llmx::tl_take(name))
// Defines the exported reader of one translation unit's table.
#define LLMX_TL_READER(unit)                                                                  \
    extern "C" int llmx_tl_table_##unit(void *out, int n, int reset) {                        \
        return (int)::llmx::tl_table(static_cast<::llmx::TlEntry *>(out), n, reset);          \
    }
#else
#define LLMX_TL_FIELD
#define LLMX_TL_PARAM
#define LLMX_TL_ARG(name)
#define LLMX_TL_GUARD(slot)
#define LLMX_TL_TAKE(args, name)
#define LLMX_TL_READER(unit)
#endif
