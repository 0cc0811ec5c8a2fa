// model.cu -- device-resident LlamaModel backend (placeholder until the
// model lands; every entry point reports MV_ERR_NOT_BUILT).
#include "../../include/memvanta_b200.h"

extern "C" {
MV_API int mv_model_open(const char*, uint64_t, uint64_t, int, mv_model_t* out) {
    if (out) *out = nullptr;
    return MV_ERR_NOT_BUILT;
}
MV_API int mv_model_close(mv_model_t) { return MV_OK; }
MV_API int mv_model_config(mv_model_t, uint64_t*) { return MV_ERR_NOT_BUILT; }
MV_API int mv_model_reset(mv_model_t) { return MV_ERR_NOT_BUILT; }
MV_API uint64_t mv_model_position(mv_model_t) { return 0; }
MV_API uint64_t mv_model_kv_bytes(mv_model_t) { return 0; }
MV_API int mv_model_forward(mv_model_t, int32_t, int, float*) { return MV_ERR_NOT_BUILT; }
MV_API int mv_model_prefill(mv_model_t, const int32_t*, uint64_t, uint64_t, int, float*) { return MV_ERR_NOT_BUILT; }
MV_API int mv_model_generate_greedy(mv_model_t, int32_t, uint64_t, int32_t*) { return MV_ERR_NOT_BUILT; }
MV_API void* mv_model_stream(mv_model_t) { return nullptr; }
}
