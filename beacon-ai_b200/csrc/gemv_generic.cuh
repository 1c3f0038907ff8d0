// gemv_generic.cuh -- the GGUF block formats without a dedicated tile
// layout: Q4_1, Q5_0, Q5_1 (32-element blocks, eight per 256-column tile) and
// Q2_K, Q3_K, Q5_K, Q6_K, Q8_K (one 256-element super-block per tile).
//
// Tile layout (same interleave as the dedicated formats): each row's raw GGUF
// bytes for the tile's 256 columns, zero-padded to whole 16-byte chunks;
// chunk c of row l sits at tile + c * 512 + l * 16, so a warp-wide 128-bit
// load reads 512 contiguous bytes and lane l holds row l. A lane decodes its
// row slice from registers with the arithmetic of
// crates/beacon-format/src/dequant.rs (the same f32 operations in the same
// order), so the dequantised values are the reference's.
#pragma once

#include "common.cuh"

namespace bc {

// Format ids of the device code (the dedicated formats are 0..2).
enum { FMT_Q4_1 = 3, FMT_Q5_0, FMT_Q5_1, FMT_Q2_K, FMT_Q3_K, FMT_Q5_K, FMT_Q6_K, FMT_Q8_K };

template <int FMT>
struct GenericFmt {
    // raw bytes of one row over a 256-column tile
    static constexpr int BYTES = FMT == FMT_Q4_1   ? 8 * 20
                                 : FMT == FMT_Q5_0 ? 8 * 22
                                 : FMT == FMT_Q5_1 ? 8 * 24
                                 : FMT == FMT_Q2_K ? 84
                                 : FMT == FMT_Q3_K ? 110
                                 : FMT == FMT_Q5_K ? 176
                                 : FMT == FMT_Q6_K ? 210
                                                   : 292;
    static constexpr int CHUNKS = (BYTES + 15) / 16;
    static constexpr int WORDS = 4 * CHUNKS;
};

__device__ __forceinline__ float x86_add(float a, float b) { return x86_nan(__fadd_rn(a, b), a, b); }

// Byte i of a row slice held as 32-bit words (i known at compile time after unrolling).
__device__ __forceinline__ uint32_t sbyte(const uint32_t* w, int i) { return (w[i >> 2] >> (8 * (i & 3))) & 0xFFu; }
__device__ __forceinline__ float sf16(const uint32_t* w, int i) {
    return f16_to_f32((uint16_t)(sbyte(w, i) | (sbyte(w, i + 1) << 8)));
}

// f32 operations of the reference: X86 selects x86 NaN propagation (the
// bit-exact dequantisation); without it the plain IEEE operations.
template <bool X86>
struct RefOps {
    __device__ __forceinline__ static float mul(float a, float b) { return X86 ? x86_mul(a, b) : __fmul_rn(a, b); }
    __device__ __forceinline__ static float add(float a, float b) { return X86 ? x86_add(a, b) : __fadd_rn(a, b); }
    __device__ __forceinline__ static float sub(float a, float b) { return X86 ? x86_sub(a, b) : __fsub_rn(a, b); }
};

// Calls emit(e, v) for the 256 values (e = column within the tile) of one
// row slice, each computed as dequant.rs computes it.
template <int FMT, bool X86, typename Emit>
__device__ __forceinline__ void decode_slice(const uint32_t* w, Emit&& emit) {
    using O = RefOps<X86>;
    if (FMT == FMT_Q4_1 || FMT == FMT_Q5_0 || FMT == FMT_Q5_1) {
        constexpr int BB = FMT == FMT_Q4_1 ? 20 : FMT == FMT_Q5_0 ? 22 : 24;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int o = b * BB;
            if (FMT == FMT_Q4_1) {  // dequant.rs:182-201
                const float scale = sf16(w, o), min_val = sf16(w, o + 2);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t byte = sbyte(w, o + 4 + i);
                    emit(32 * b + 2 * i, O::add(O::mul((float)(byte & 0x0Fu), scale), min_val));
                    emit(32 * b + 2 * i + 1, O::add(O::mul((float)(byte >> 4), scale), min_val));
                }
            } else {  // Q5_0 dequant.rs:205-228, Q5_1 dequant.rs:232-254
                const bool q51 = FMT == FMT_Q5_1;
                const float scale = sf16(w, o), min_val = q51 ? sf16(w, o + 2) : 0.0f;
                const int ho = q51 ? o + 4 : o + 2, qo = q51 ? o + 8 : o + 6;
                const uint32_t hb = sbyte(w, ho) | (sbyte(w, ho + 1) << 8) | (sbyte(w, ho + 2) << 16) |
                                    (sbyte(w, ho + 3) << 24);
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const uint32_t byte = sbyte(w, qo + i);
                    const uint32_t lo = (byte & 0x0Fu) | (((hb >> i) & 1u) << 4);
                    const uint32_t hi = (byte >> 4) | (((hb >> (i + 16)) & 1u) << 4);
                    if (q51) {
                        emit(32 * b + 2 * i, O::add(O::mul((float)lo, scale), min_val));
                        emit(32 * b + 2 * i + 1, O::add(O::mul((float)hi, scale), min_val));
                    } else {
                        emit(32 * b + 2 * i, O::mul((float)lo - 16.0f, scale));
                        emit(32 * b + 2 * i + 1, O::mul((float)hi - 16.0f, scale));
                    }
                }
            }
        }
    } else if (FMT == FMT_Q5_K) {  // dequant.rs:377-429
        const float d = sf16(w, 0), dmin = sf16(w, 2);
        float sc[8], mn[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // decode_k_scales_mins (dequant.rs:289-307)
            const uint32_t s = j < 4 ? (sbyte(w, 4 + j) & 0x3Fu)
                                     : ((sbyte(w, 4 + j + 4) & 0x0Fu) | ((sbyte(w, 4 + j - 4) >> 6) << 4));
            const uint32_t m = j < 4 ? (sbyte(w, 4 + j + 4) & 0x3Fu)
                                     : ((sbyte(w, 4 + j + 4) >> 4) | ((sbyte(w, 4 + j) >> 6) << 4));
            sc[j] = O::mul((float)s, d);
            mn[j] = O::mul((float)m, dmin);
        }
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int e = 64 * p + 32 * h + j;
                    const uint32_t q4 = h ? (sbyte(w, 48 + 32 * p + j) >> 4) : (sbyte(w, 48 + 32 * p + j) & 0x0Fu);
                    const uint32_t hb = ((sbyte(w, 16 + e / 8) >> (e % 8)) & 1u) << 4;
                    emit(e, O::sub(O::mul((float)(q4 | hb), sc[2 * p + h]), mn[2 * p + h]));
                }
    } else if (FMT == FMT_Q6_K) {  // dequant.rs:440-477
        const float super_scale = sf16(w, 208);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int j = 0; j < 128; ++j) {
                const float scale = O::mul((float)(int8_t)sbyte(w, 192 + 8 * c + j / 16), super_scale);
                const uint32_t low4 = (sbyte(w, 64 * c + j % 64) >> ((j / 64) * 4)) & 0x0Fu;
                const uint32_t high2 = (sbyte(w, 128 + 32 * c + j % 32) >> ((j / 32) * 2)) & 0x03u;
                const int q6 = (int)(low4 | (high2 << 4)) - 32;
                emit(128 * c + j, O::mul((float)q6, scale));
            }
    } else if (FMT == FMT_Q2_K) {  // dequant.rs:488-514
        const float d = sf16(w, 80), dmin = sf16(w, 82);
#pragma unroll
        for (int sb = 0; sb < 16; ++sb) {
            const float sc = O::mul((float)(sbyte(w, sb) & 0x0Fu), d);
            const float mn = O::mul((float)(sbyte(w, sb) >> 4), dmin);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const uint32_t q = (sbyte(w, 16 + sb * 4 + i / 4) >> ((i % 4) * 2)) & 0x03u;
                emit(sb * 16 + i, O::sub(O::mul((float)q, sc), mn));
            }
        }
    } else if (FMT == FMT_Q3_K) {  // dequant.rs:525-572
        const float d = sf16(w, 108);
        int sc[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            sc[i] = (int)(sbyte(w, 96 + i) & 0x0Fu);
            sc[i + 8] = (int)(sbyte(w, 96 + i) >> 4);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t up = sbyte(w, 104 + i);
            sc[2 * i] |= (int)(up & 0x03u) << 4;
            sc[2 * i + 1] |= (int)((up >> 2) & 0x03u) << 4;
            sc[2 * i + 8] |= (int)((up >> 4) & 0x03u) << 4;
            sc[2 * i + 9] |= (int)((up >> 6) & 0x03u) << 4;
        }
#pragma unroll
        for (int sb = 0; sb < 16; ++sb) {
            const float sub_scale = O::mul((float)(sc[sb] - 32), d);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int e = sb * 16 + i;
                const uint32_t lo = (sbyte(w, 32 + e / 4) >> ((e % 4) * 2)) & 0x03u;
                const uint32_t hb = (sbyte(w, e / 8) >> (e % 8)) & 1u;
                emit(e, O::mul((float)(lo | (hb << 2)) - 4.0f, sub_scale));
            }
        }
    } else {  // Q8_K dequant.rs:582-597
        const float d = __uint_as_float(w[0]);
#pragma unroll
        for (int i = 0; i < 256; ++i) emit(i, O::mul((float)(int8_t)sbyte(w, 4 + i), d));
    }
}

}  // namespace bc
