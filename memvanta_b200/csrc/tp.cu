// tp.cu -- the stand-alone tensor-parallel kernels (tp.cuh has the protocols).
// Prefill (flags): wait for a sync point; scatter a rank's slice into every
// rank's replicated buffer (optionally adding it to what is there -- the
// residual stream).  Decode (LL buffers): pack the embedding into this rank's
// copy, unpack a copy into a float vector once complete, scatter the logits
// slice.  Both: advance the step counter.  The decode GEMV and attention
// store their LL slices from their own epilogues.
#include "common.cuh"
#include "kernels.cuh"
#include "tp.cuh"

namespace mvb {

namespace {

__global__ void tp_wait_kernel(TpCtx tp, int point) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) tp_wait_thread(tp, tp_epoch(tp, point), 200 + point);
}

// dst[t * dst_ld + col_off + j] (= or +=) src[t * src_ld + j] on every rank.
// add reads this rank's copy of dst; every copy holds the same values.
__global__ void tp_scatter_kernel(TpCtx tp, const float* __restrict__ src, int rows, int w, int src_ld,
                                  uint64_t dst_shared, int dst_ld, int col_off, int add, int point, int slot) {
    pdl_trigger();
    pdl_wait();
    const float* mine = reinterpret_cast<const float*>(tp_base(tp, tp.rank) + dst_shared);
    const uint64_t n = (uint64_t)rows * w;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / w), j = (int)(i % w);
        const uint64_t at = (uint64_t)t * dst_ld + col_off + j;
        float v = src[(uint64_t)t * src_ld + j];
        if (add) v = __ldcg(mine + at) + v;  // the reference's x + y
        tp_for_each(tp, [&](int, char* base) { reinterpret_cast<float*>(base + dst_shared)[at] = v; });
    }
    tp_signal_cta(tp, point, slot);
}

__global__ void tp_pack_kernel(TpCtx tp, const float* __restrict__ src, int n, uint64_t dst_shared, int point) {
    pdl_trigger();
    pdl_wait();
    const unsigned ep = tp_uepoch(tp, point);
    uint2* dst = reinterpret_cast<uint2*>(tp_base(tp, tp.rank) + dst_shared);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        ll_store(dst + i, src[i], ep);
}

__global__ void tp_unpack_kernel(TpCtx tp, uint64_t src_shared, int n, float* __restrict__ dst, int point) {
    pdl_trigger();
    pdl_wait();
    const unsigned ep = tp_uepoch(tp, point);
    const uint2* src = reinterpret_cast<const uint2*>(tp_base(tp, tp.rank) + src_shared);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        dst[i] = ll_load1(tp, src + i, ep, 300 + point);
}

__global__ void tp_scatter_ll_kernel(TpCtx tp, const float* __restrict__ src, int n, uint64_t dst_shared,
                                     uint64_t col_off, int point) {
    pdl_trigger();
    pdl_wait();
    const unsigned ep = tp_uepoch(tp, point);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        ll_put_all(tp, dst_shared, col_off + i, src[i], ep);
}

__global__ void tp_step_kernel(int* step) {
    pdl_wait();
    if (threadIdx.x == 0) *step += 1;
}

}  // namespace

cudaError_t tp_wait(const TpCtx& tp, int point, cudaStream_t s) {
    return launch_pdl(tp_wait_kernel, dim3(1), dim3(32), 0, s, tp, point);
}

cudaError_t tp_scatter(const TpCtx& tp, const float* src, uint64_t rows, uint64_t w, uint64_t src_ld,
                       uint64_t dst_shared, uint64_t dst_ld, uint64_t col_off, bool add, int point, int slot,
                       cudaStream_t s) {
    const uint64_t n = rows * w;
    uint64_t ctas = (n + 255) / 256;
    const uint64_t cap = (uint64_t)num_sms() * 4;
    if (ctas > cap) ctas = cap;
    if (ctas == 0) ctas = 1;
    return launch_pdl(tp_scatter_kernel, dim3((unsigned)ctas), dim3(256), 0, s, tp, src, (int)rows, (int)w,
                      (int)src_ld, dst_shared, (int)dst_ld, (int)col_off, add ? 1 : 0, point, slot);
}

cudaError_t tp_step(int* step, cudaStream_t s) { return launch_pdl(tp_step_kernel, dim3(1), dim3(32), 0, s, step); }

namespace {
dim3 ll_grid(uint64_t n) {
    uint64_t ctas = (n + 255) / 256;
    const uint64_t cap = (uint64_t)num_sms() * 4;
    return dim3((unsigned)(ctas > cap ? cap : ctas ? ctas : 1));
}
}  // namespace

cudaError_t tp_pack(const TpCtx& tp, const float* src, uint64_t n, uint64_t dst_shared, int point, cudaStream_t s) {
    return launch_pdl(tp_pack_kernel, ll_grid(n), dim3(256), 0, s, tp, src, (int)n, dst_shared, point);
}

cudaError_t tp_unpack(const TpCtx& tp, uint64_t src_shared, uint64_t n, float* dst, int point, cudaStream_t s) {
    return launch_pdl(tp_unpack_kernel, ll_grid(n), dim3(256), 0, s, tp, src_shared, (int)n, dst, point);
}

cudaError_t tp_scatter_ll(const TpCtx& tp, const float* src, uint64_t n, uint64_t dst_shared, uint64_t col_off,
                          int point, cudaStream_t s) {
    return launch_pdl(tp_scatter_ll_kernel, ll_grid(n), dim3(256), 0, s, tp, src, (int)n, dst_shared, col_off, point);
}

}  // namespace mvb
