// tp.cuh -- tensor parallelism across the GPUs of one node over NVLink peer
// memory (CUDA IPC mappings), no collective library on the data path.
//
// Every rank (one process per GPU) owns one device block that every other
// rank maps: a flag array, then the full-size activation buffers the ranks
// keep replicated (decode x / att / ff / logits in the LL form below,
// prefill X / ATT / FF as floats).  A prefill kernel that produces a rank's
// slice of such a buffer stores it into every rank's copy (plain peer
// stores, no multicast) and then *publishes* an epoch:
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
__device__ __forceinline__ unsigned tp_uepoch(const TpCtx& t, int point) { return (unsigned)tp_epoch(t, point); }

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

// ---- LL (low-latency) replicated buffers, used by the decode step.  Every
// element is 8 bytes, {float bits, epoch}, written with ONE 8-byte store to
// every rank's copy; a reader polls the elements it needs until they carry
// the expected epoch.  No fence, flag or counter sits between producer and
// consumer, so a kernel's end costs nothing extra and the consumer starts on
// each element as soon as it lands.  Epochs follow tp_epoch (never 0, so a
// cleared buffer never matches).
__device__ __forceinline__ void ll_store(void* p, float v, unsigned ep) {
    asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(ep) : "memory");
}
__device__ __forceinline__ uint4 ll_ld16(const void* p) {
    uint4 r;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
__device__ __forceinline__ uint2 ll_ld8(const void* p) {
    uint2 r;
    asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
    return r;
}

// Bound of one polling thread: gives up after the wait limit (recording
// `site`), or at once when an earlier wait of this rank gave up.
struct LLWait {
    unsigned long long t0 = 0;
    __device__ __forceinline__ bool expired(const TpCtx& t, int site) {
        if (*reinterpret_cast<volatile int*>(t.status)) return true;
        const unsigned long long now = tp_now();
        if (t0 == 0) {
            t0 = now;
            return false;
        }
        if (now - t0 > (unsigned long long)*t.limit_ns) {
            atomicCAS(t.status, 0, site);
            return true;
        }
        return false;
    }
};

// 8 consecutive elements (64 bytes at p, 16-byte aligned) once all carry ep.
__device__ __forceinline__ void ll_load8(const TpCtx& t, const uint2* p, unsigned ep, int site, float4& lo,
                                         float4& hi) {
    uint4 q0, q1, q2, q3;
    LLWait w;
    unsigned ns = 32;
    for (;;) {
        q0 = ll_ld16(p);
        q1 = ll_ld16(p + 2);
        q2 = ll_ld16(p + 4);
        q3 = ll_ld16(p + 6);
        if (((q0.y ^ ep) | (q0.w ^ ep) | (q1.y ^ ep) | (q1.w ^ ep) | (q2.y ^ ep) | (q2.w ^ ep) | (q3.y ^ ep) |
             (q3.w ^ ep)) == 0)
            break;
        if (w.expired(t, site)) break;
        __nanosleep(ns);  // back off: many threads poll while the weight stream runs
        ns = ns < 256 ? 2 * ns : 256;
    }
    lo = make_float4(__uint_as_float(q0.x), __uint_as_float(q0.z), __uint_as_float(q1.x), __uint_as_float(q1.z));
    hi = make_float4(__uint_as_float(q2.x), __uint_as_float(q2.z), __uint_as_float(q3.x), __uint_as_float(q3.z));
}

// One element once it carries ep.
__device__ __forceinline__ float ll_load1(const TpCtx& t, const uint2* p, unsigned ep, int site) {
    uint2 q;
    LLWait w;
    unsigned ns = 32;
    for (;;) {
        q = ll_ld8(p);
        if (q.y == ep || w.expired(t, site)) break;
        __nanosleep(ns);
        ns = ns < 256 ? 2 * ns : 256;
    }
    return __uint_as_float(q.x);
}

// v into element i of the LL buffer at byte offset `off` of every rank's block.
__device__ __forceinline__ void ll_put_all(const TpCtx& t, uint64_t off, uint64_t i, float v, unsigned ep) {
    tp_for_each(t, [&](int, char* base) { ll_store(reinterpret_cast<uint2*>(base + off) + i, v, ep); });
}
#endif

}  // namespace mvb
