// tp.cuh -- tensor parallelism across the GPUs of one node over NVLink peer
// memory (CUDA IPC mappings), no collective library on the data path.
//
// Every rank (one process per GPU) owns one device block that every other
// rank maps: a flag array, then the full-size activation buffers the ranks
// keep replicated (decode x / att / ff / logits, prefill X / ATT / FF).  A
// kernel that produces a rank's slice of such a buffer stores it into every
// rank's copy (plain peer stores, no multicast) and then *publishes* an epoch:
// its last CTA to finish raises flags[rank] = epoch on every rank after a
// system-scope fence.  A kernel that needs the whole buffer *waits* until
// flags[src] >= epoch for every src before reading.  Epochs are
//     step * points_per_step + point + 1,
// step a device counter every rank advances identically once per decode step
// (or prefill chunk), point the sync point's index within the step, so the
// same CUDA graph serves every step and no flag is ever reset.
//
// Waits are bounded: after *limit_ns without the epoch the waiting thread
// records a site code in the status word and carries on (outputs invalid),
// so no kernel hangs on a rank that died; once the status word is set, later
// waits return at once.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace mvb {

constexpr int kTpMaxWorld = 8;

struct TpCtx {
    int world = 1, rank = 0;
    char* base[kTpMaxWorld] = {};  // every rank's shared block (own included)
    const int* step = nullptr;     // this rank's step counter (device)
    int pps = 0;                   // sync points per step
    unsigned* counters = nullptr;  // this rank's arrival counters, one per signalling kernel slot
    int* status = nullptr;         // this rank's status word (device)
    const long long* limit_ns = nullptr;  // bound of every wait (device word, settable between calls)
};

// byte offsets inside every rank's shared block
constexpr uint64_t kTpFlagsBytes = 256;  // int flags[kTpMaxWorld], padded

constexpr long long kTpDefaultLimitNs = 5000000000ll;

#if defined(__CUDACC__)

// base[r] for a run-time r without indexing the (parameter-space) array
// dynamically, which would copy the whole context to local memory.
__device__ __forceinline__ char* tp_base(const TpCtx& t, int r) {
    char* p = t.base[0];
#pragma unroll
    for (int d = 1; d < kTpMaxWorld; ++d)
        if (r == d) p = t.base[d];
    return p;
}
__device__ __forceinline__ int* tp_flags(const TpCtx& t, int rank) { return reinterpret_cast<int*>(tp_base(t, rank)); }

// f(d, base[d]) for every rank d, with constant indices.
template <class F>
__device__ __forceinline__ void tp_for_each(const TpCtx& t, F&& f) {
#pragma unroll
    for (int d = 0; d < kTpMaxWorld; ++d)
        if (d < t.world) f(d, t.base[d]);
}

__device__ __forceinline__ int tp_epoch(const TpCtx& t, int point) { return *t.step * t.pps + point + 1; }

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long tp_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One thread: wait until every rank has published `epoch` (bounded).
__device__ __forceinline__ void tp_wait_thread(const TpCtx& t, int epoch, int site) {
    const int* f = tp_flags(t, t.rank);
    if (*reinterpret_cast<volatile int*>(t.status)) return;  // an earlier wait already gave up
    const unsigned long long limit = (unsigned long long)*t.limit_ns;
    const unsigned long long t0 = tp_now();
    for (int src = 0; src < t.world; ++src) {
        while (ld_acquire_sys(f + src) < epoch) {
            if (tp_now() - t0 > limit) {
                atomicCAS(t.status, 0, site);
                return;
            }
            __nanosleep(32);
        }
    }
}

// Whole CTA: thread 0 waits, everyone continues after it.
__device__ __forceinline__ void tp_wait_cta(const TpCtx& t, int point, int site) {
    if (threadIdx.x == 0 && threadIdx.y == 0) tp_wait_thread(t, tp_epoch(t, point), site);
    __syncthreads();
}

// Whole CTA, after its last peer store: the grid's last CTA publishes the
// point's epoch to every rank.  `slot` picks the arrival counter.
__device__ __forceinline__ void tp_signal_cta(const TpCtx& t, int point, int slot) {
    __syncthreads();
    if (threadIdx.x == 0 && threadIdx.y == 0) {
        __threadfence_system();
        const unsigned n = gridDim.x * gridDim.y * gridDim.z;
        if (atomicAdd(t.counters + slot, 1u) == n - 1) {
            t.counters[slot] = 0;
            __threadfence_system();
            const int e = tp_epoch(t, point);
            tp_for_each(t, [&](int, char* base) { st_release_sys(reinterpret_cast<int*>(base) + t.rank, e); });
        }
    }
}
#endif

}  // namespace mvb
