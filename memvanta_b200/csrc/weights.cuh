// weights.cuh -- device layout of an uploaded GGUF weight.
//
// GGUF blocks are 18 B (Q4_0), 34 B (Q8_0) and 210 B (Q6_K): none of them
// keeps the nibble/int8 payload 16-byte aligned, so every upload is repacked
// once into planes ("structure of arrays"), row-major [rows][blocks]:
//
//   Q4_0  qs  u8  [rows][nb][16]   the 16 nibble bytes of each block, as in GGUF
//         d   f16 [rows][dstride]  dstride = nb rounded up to 8, so every row's
//                                  scales start 16-byte aligned (zero padding)
//   Q8_0  qs  i8  [rows][nb][32]
//         d   f16 [rows][nb]
//   Q6_K  qs  u8  [rows][nsb][128] ql
//         qh  u8  [rows][nsb][64]
//         sc  i8  [rows][nsb][16]
//         d   f16 [rows][nsb]
//   F16 / F32     unchanged, row-major
//
// The repack keeps every byte (mv_weight_download inverts it exactly); it only
// moves the scale out of line so a lane can fetch a block payload with one
// 128-bit load.
#pragma once
#include <cstdint>

struct mv_weight_s {
    int type = 0;
    uint64_t rows = 0, cols = 0;
    uint64_t nb = 0;          // blocks per row (32-element; 256 for Q6_K)
    uint64_t dstride = 0;     // fp16 scales per row in the d plane (>= nb)
    void* base = nullptr;     // single device allocation holding all planes
    uint64_t bytes = 0;
    uint8_t* qs = nullptr;    // payload plane (Q4_0/Q8_0 qs, Q6_K ql, F16/F32 data)
    uint8_t* qh = nullptr;    // Q6_K high bits
    int8_t* sc = nullptr;     // Q6_K sub-block scales
    uint16_t* d = nullptr;    // fp16 block scales
    int device = 0;
};

namespace mvb {

inline uint64_t ggml_block_elems(int type) { return type == 14 ? 256 : (type == 2 || type == 8) ? 32 : 1; }
inline uint64_t ggml_block_bytes(int type) {
    switch (type) {
        case 0: return 4;
        case 1: return 2;
        case 2: return 18;
        case 8: return 34;
        case 14: return 210;
    }
    return 0;
}

}  // namespace mvb
