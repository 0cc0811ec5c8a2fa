// noalloc.cu -- mv_gemm_q8_noalloc: the Q4_0 x Q8-activation batched matmul
// (mv_gemm with MV_ACT_Q8) without allocating any device memory.
//
// Who needs it: callers that are not allowed to allocate device memory while
// they run -- for example a host framework that hands all of the GPU's
// memory to its own pool allocator and forbids allocations from outside it,
// a service holding a fixed device-memory budget where an allocation in the
// middle of a request could fail, or a latency-critical loop that must not
// take the allocator's locks or wait on its synchronisation.  mv_gemm
// quantises the activations into stream-ordered scratch (cudaMallocAsync);
// this entry point writes them into a fixed array compiled into the library.
//
// The array (kScratchBytes, 8 MiB) is a file-scope __device__ variable: every
// GPU that loads the library holds it until the process exits.  In host code
// its name is only a host-side stand-in, so its device address is looked up
// with cudaGetSymbolAddress once per device, with that device current, on the
// first call made on that device; make that first call before any stream
// capture.  The address is kept for the life of the process, so the device
// must not be reset (cudaDeviceReset) after that first call.  All calls share the one array: calls whose work overlaps on the
// GPU (other streams, other threads) race on it and must be serialised by the
// caller.  Nothing needs clearing between calls -- each call writes every
// scratch byte it later reads.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/memvanta_b200.h"
#include "kernels.cuh"
#include "weights.cuh"

namespace {

constexpr size_t kScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return e;
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return cudaSuccess;
}

int fail(int code, const std::string& msg) {
    mvb::set_last_error(msg);
    return code;
}

}  // namespace

extern "C" MV_API int mv_gemm_q8_noalloc(mv_weight_t w, const float* x, uint64_t batch, float* y, void* stream) {
    if (!w) return fail(MV_ERR_INVALID, "null weight handle");
    if (batch == 0) return MV_OK;
    if (!x || !y) return fail(MV_ERR_INVALID, "null x or y");
    if (w->type != MV_TYPE_Q4_0)
        return fail(MV_ERR_UNSUPPORTED, "mv_gemm_q8_noalloc needs a Q4_0 weight (the Q8-activation path)");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (batch < 2) {
        // as mv_gemm: one token takes the fp32-activation path, which needs no scratch
        e = mvb::matmul_f32act(*w, x, batch, y, s);
    } else {
        const uint64_t ldb = mvb::gemm_tc_ldb(batch);
        const uint64_t q_bytes = (batch * w->cols + 255) / 256 * 256;
        const uint64_t d_bytes = 2 * ldb * (w->cols / 32) * sizeof(float);
        if (q_bytes + d_bytes > kScratchBytes)
            return fail(MV_ERR_INVALID, "batch x cols needs " + std::to_string(q_bytes + d_bytes) +
                                            " bytes of scratch; mv_gemm_q8_noalloc has " +
                                            std::to_string(kScratchBytes) + " (use mv_gemm)");
        void* base = nullptr;
        e = scratch_address(&base);
        if (e == cudaSuccess) {
            int8_t* q = static_cast<int8_t*>(base);
            float* d = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + q_bytes);
            e = mvb::quantize_q8_rows_t(x, batch, w->cols, q, d, ldb, s);
            if (e == cudaSuccess) e = mvb::gemm_q4_q8_tc(*w, q, d, ldb, batch, y, s);
        }
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(MV_ERR_CUDA, std::string("mv_gemm_q8_noalloc: ") + cudaGetErrorString(e));
    }
    return MV_OK;
}
