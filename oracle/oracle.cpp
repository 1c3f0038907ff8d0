// oracle.cpp -- CPU restatement of the reference's quantized decode path.
//
// TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA backend. Only the
// tests, the smoke check and the bench's CPU-baseline leg load this library.
//
// Build: g++ -O2 -ffp-contract=off -fopenmp (see oracle/Makefile). Every sum is
// kept in the reference's sequential order; no a*b+c is fused, as in Rust.
// Parallelism (OpenMP) is only ever across independent output rows, so results
// do not depend on the thread count.

#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

thread_local std::string g_err;

int fail(const std::string& msg) {
    g_err = msg;
    return -1;
}

inline float bits_f32(uint32_t b) {
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}
inline uint32_t f32_bits(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    return b;
}
inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

}  // namespace

// ---------------------------------------------------------------------------
// f16 <-> f32  (crates/beacon-format/src/dequant.rs:78-152; q4.rs:210-250)
// ---------------------------------------------------------------------------

extern "C" float orc_f16_to_f32(uint16_t bits) {
    // dequant.rs:80-109
    uint32_t sign = (uint32_t)(bits >> 15) << 31;
    uint32_t exponent = (bits >> 10) & 0x1F;
    uint32_t mantissa = bits & 0x3FF;
    if (exponent == 0) {
        if (mantissa == 0) return bits_f32(sign);
        uint32_t m = mantissa;
        int32_t e = -14;
        while ((m & 0x400) == 0) {
            m <<= 1;
            e -= 1;
        }
        m &= 0x3FF;
        return bits_f32(sign | ((uint32_t)(e + 127) << 23) | (m << 13));
    }
    if (exponent == 31) return bits_f32(sign | 0x7F800000u | (mantissa << 13));
    return bits_f32(sign | ((exponent + 112) << 23) | (mantissa << 13));
}

extern "C" uint16_t orc_f32_to_f16_rtz(float val) {
    // dequant.rs:116-152: truncation, flush below 2^-24, overflow to Inf.
    uint32_t bits = f32_bits(val);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
    int32_t exponent = (int32_t)((bits >> 23) & 0xFF);
    uint32_t mantissa = bits & 0x007FFFFF;
    if (exponent == 255) {
        if (mantissa == 0) return sign | 0x7C00;
        uint16_t m = (uint16_t)(mantissa >> 13);
        if (m < 1) m = 1;
        return sign | 0x7C00 | m;
    }
    int32_t new_exp = exponent - 127 + 15;
    if (new_exp >= 31) return sign | 0x7C00;
    if (new_exp <= 0) {
        if (new_exp < -10) return sign;
        uint32_t m = (mantissa | 0x00800000u) >> (1 - new_exp + 13);
        return sign | (uint16_t)m;
    }
    return sign | (uint16_t)((uint32_t)new_exp << 10) | (uint16_t)(mantissa >> 13);
}

// Round-to-nearest-even single -> half. Not a reference function: it stores
// the block scales written by the fixture quantizer below.
extern "C" uint16_t orc_f32_to_f16_rne(float f) {
    uint32_t x = f32_bits(f);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return sign | (ax > 0x7F800000u ? 0x7E00 : 0x7C00);
    if (ax >= 0x477FF000u) return sign | 0x7C00;
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return sign;
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126 - e;
        uint32_t r = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1))) r++;
        return sign | (uint16_t)r;
    }
    uint32_t r = (ax >> 13) - (112u << 10);
    uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) r++;
    return sign | (uint16_t)r;
}

extern "C" void orc_f32_to_f16_rtz_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16_rtz(in[i]);
}

extern "C" void orc_f32_to_f16_rne_array(const float* in, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f32_to_f16_rne(in[i]);
}

// ---------------------------------------------------------------------------
// Block formats (crates/beacon-format/src/dtype.rs:56-82)
// ---------------------------------------------------------------------------

extern "C" int64_t orc_block_size(int dtype) {
    switch (dtype) {
        case ORC_F32: case ORC_F16: case ORC_BF16: case ORC_I32: case ORC_I8: return 1;
        case ORC_Q4_0: case ORC_Q4_1: case ORC_Q5_0: case ORC_Q5_1: case ORC_Q8_0: return 32;
        case ORC_Q2_K: case ORC_Q3_K: case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K:
        case ORC_Q8_K: return 256;
        default: return 0;
    }
}

extern "C" int64_t orc_block_bytes(int dtype) {
    switch (dtype) {
        case ORC_F32: case ORC_I32: return 4;
        case ORC_F16: case ORC_BF16: return 2;
        case ORC_I8: return 1;
        case ORC_Q4_0: return 18;
        case ORC_Q4_1: return 20;
        case ORC_Q5_0: return 22;
        case ORC_Q5_1: return 24;
        case ORC_Q8_0: return 34;
        case ORC_Q2_K: return 84;
        case ORC_Q3_K: return 110;
        case ORC_Q4_K: return 144;
        case ORC_Q5_K: return 176;
        case ORC_Q6_K: return 210;
        case ORC_Q8_K: return 292;
        default: return 0;
    }
}

namespace {

// decode_k_scales_mins (dequant.rs:289-307)
void decode_k_scales_mins(const uint8_t* q, uint8_t* scales, uint8_t* mins) {
    for (int j = 0; j < 4; ++j) {
        scales[j] = q[j] & 0x3F;
        mins[j] = q[j + 4] & 0x3F;
    }
    for (int j = 4; j < 8; ++j) {
        scales[j] = (uint8_t)((q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4));
        mins[j] = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

// Every block dequantizer produces the f32 value that dequant.rs hands to
// f32_to_f16; `emit` receives (element index, f32 value).
template <typename Emit>
int dequant_values(const uint8_t* data, int dtype, uint64_t n, int nibble_order, Emit emit) {
    const int64_t bs = orc_block_size(dtype);
    const int64_t bb = orc_block_bytes(dtype);
    if (bs <= 1) return fail("dequant: dtype is not quantized");
    if (n % (uint64_t)bs != 0) return fail("dequant: element count is not a whole number of blocks");
    const uint64_t nb = n / (uint64_t)bs;
    for (uint64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = data + b * (uint64_t)bb;
        const uint64_t base = b * (uint64_t)bs;
        switch (dtype) {
            case ORC_Q4_0: {  // dequant.rs:160-178 / q4.rs:26-42
                float scale = orc_f16_to_f32(rd16(blk));
                for (int i = 0; i < 16; ++i) {
                    uint8_t byte = blk[2 + i];
                    int8_t lo = (int8_t)((byte & 0x0F)) - 8;
                    int8_t hi = (int8_t)((byte >> 4) & 0x0F) - 8;
                    float vlo = (float)lo * scale;
                    float vhi = (float)hi * scale;
                    if (nibble_order == ORC_NIBBLE_GGUF_SPLIT) {
                        emit(base + i, vlo);
                        emit(base + i + 16, vhi);
                    } else {
                        emit(base + 2 * i, vlo);
                        emit(base + 2 * i + 1, vhi);
                    }
                }
                break;
            }
            case ORC_Q4_1: {  // dequant.rs:182-201
                float scale = orc_f16_to_f32(rd16(blk));
                float min_val = orc_f16_to_f32(rd16(blk + 2));
                for (int i = 0; i < 16; ++i) {
                    uint8_t byte = blk[4 + i];
                    float lo = (float)(byte & 0x0F);
                    float hi = (float)(byte >> 4);
                    float a = lo * scale;
                    float c = hi * scale;
                    emit(base + 2 * i, a + min_val);
                    emit(base + 2 * i + 1, c + min_val);
                }
                break;
            }
            case ORC_Q5_0: {  // dequant.rs:205-228
                float scale = orc_f16_to_f32(rd16(blk));
                uint32_t hb = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) |
                              ((uint32_t)blk[4] << 16) | ((uint32_t)blk[5] << 24);
                for (int i = 0; i < 16; ++i) {
                    uint8_t byte = blk[6 + i];
                    uint32_t lo = byte & 0x0F;
                    uint32_t hi = byte >> 4;
                    lo |= ((hb >> i) & 1) << 4;
                    hi |= ((hb >> (i + 16)) & 1) << 4;
                    float a = (float)lo - 16.0f;
                    float c = (float)hi - 16.0f;
                    emit(base + 2 * i, a * scale);
                    emit(base + 2 * i + 1, c * scale);
                }
                break;
            }
            case ORC_Q5_1: {  // dequant.rs:232-254
                float scale = orc_f16_to_f32(rd16(blk));
                float min_val = orc_f16_to_f32(rd16(blk + 2));
                uint32_t hb = (uint32_t)blk[4] | ((uint32_t)blk[5] << 8) |
                              ((uint32_t)blk[6] << 16) | ((uint32_t)blk[7] << 24);
                for (int i = 0; i < 16; ++i) {
                    uint8_t byte = blk[8 + i];
                    uint32_t lo = byte & 0x0F;
                    uint32_t hi = byte >> 4;
                    lo |= ((hb >> i) & 1) << 4;
                    hi |= ((hb >> (i + 16)) & 1) << 4;
                    float a = (float)lo * scale;
                    float c = (float)hi * scale;
                    emit(base + 2 * i, a + min_val);
                    emit(base + 2 * i + 1, c + min_val);
                }
                break;
            }
            case ORC_Q8_0: {  // dequant.rs:258-273
                float scale = orc_f16_to_f32(rd16(blk));
                for (int i = 0; i < 32; ++i) {
                    int8_t w = (int8_t)blk[2 + i];
                    emit(base + i, (float)w * scale);
                }
                break;
            }
            case ORC_Q4_K: {  // dequant.rs:318-365
                float d = orc_f16_to_f32(rd16(blk));
                float dmin = orc_f16_to_f32(rd16(blk + 2));
                uint8_t rs[8], rm[8];
                decode_k_scales_mins(blk + 4, rs, rm);
                float sc[8], mn[8];
                for (int j = 0; j < 8; ++j) {
                    sc[j] = (float)rs[j] * d;
                    mn[j] = (float)rm[j] * dmin;
                }
                const uint8_t* qs = blk + 16;
                uint64_t di = base;
                int qp = 0;
                for (int sb = 0; sb < 8; sb += 2) {
                    for (int j = 0; j < 32; ++j) {
                        float w = (float)(qs[qp + j] & 0x0F);
                        float t = w * sc[sb];
                        emit(di++, t - mn[sb]);
                    }
                    for (int j = 0; j < 32; ++j) {
                        float w = (float)(qs[qp + j] >> 4);
                        float t = w * sc[sb + 1];
                        emit(di++, t - mn[sb + 1]);
                    }
                    qp += 32;
                }
                break;
            }
            case ORC_Q5_K: {  // dequant.rs:377-429
                float d = orc_f16_to_f32(rd16(blk));
                float dmin = orc_f16_to_f32(rd16(blk + 2));
                uint8_t rs[8], rm[8];
                decode_k_scales_mins(blk + 4, rs, rm);
                const uint8_t* qh = blk + 16;
                const uint8_t* ql = blk + 48;
                float sc[8], mn[8];
                for (int j = 0; j < 8; ++j) {
                    sc[j] = (float)rs[j] * d;
                    mn[j] = (float)rm[j] * dmin;
                }
                uint64_t di = base;
                int qp = 0;
                for (int sb = 0; sb < 8; sb += 2) {
                    for (int j = 0; j < 32; ++j) {
                        uint32_t lo4 = ql[qp + j] & 0x0F;
                        uint64_t elem = di - base;
                        uint32_t h = (uint32_t)((qh[elem / 8] >> (elem % 8)) & 1) << 4;
                        float t = (float)(lo4 | h) * sc[sb];
                        emit(di++, t - mn[sb]);
                    }
                    for (int j = 0; j < 32; ++j) {
                        uint32_t hi4 = ql[qp + j] >> 4;
                        uint64_t elem = di - base;
                        uint32_t h = (uint32_t)((qh[elem / 8] >> (elem % 8)) & 1) << 4;
                        float t = (float)(hi4 | h) * sc[sb + 1];
                        emit(di++, t - mn[sb + 1]);
                    }
                    qp += 32;
                }
                break;
            }
            case ORC_Q6_K: {  // dequant.rs:440-477
                float super_scale = orc_f16_to_f32(rd16(blk + 208));
                uint64_t di = base;
                int l_ptr = 0, h_ptr = 128, sc_ptr = 192;
                for (int cluster = 0; cluster < 2; ++cluster) {
                    for (uint32_t j = 0; j < 128; ++j) {
                        float scale = (float)(int8_t)blk[sc_ptr + j / 16] * super_scale;
                        uint8_t low4 = (blk[l_ptr + (j % 64)] >> ((j / 64) * 4)) & 0x0F;
                        uint8_t high2 = (blk[h_ptr + (j % 32)] >> ((j / 32) * 2)) & 0x03;
                        int8_t q6 = (int8_t)(low4 | (high2 << 4)) - 32;
                        emit(di++, (float)q6 * scale);
                    }
                    l_ptr += 64;
                    h_ptr += 32;
                    sc_ptr += 8;
                }
                break;
            }
            case ORC_Q2_K: {  // dequant.rs:488-514
                const uint8_t* scd = blk;
                const uint8_t* qs = blk + 16;
                float d = orc_f16_to_f32(rd16(blk + 80));
                float dmin = orc_f16_to_f32(rd16(blk + 82));
                for (int sub = 0; sub < 16; ++sub) {
                    float sc = (float)(scd[sub] & 0x0F) * d;
                    float mn = (float)(scd[sub] >> 4) * dmin;
                    for (int i = 0; i < 16; ++i) {
                        int byte_idx = sub * 4 + i / 4;
                        int shift = (i % 4) * 2;
                        float q = (float)((qs[byte_idx] >> shift) & 0x03);
                        float t = q * sc;
                        emit(base + sub * 16 + i, t - mn);
                    }
                }
                break;
            }
            case ORC_Q3_K: {  // dequant.rs:525-572
                const uint8_t* hmask = blk;
                const uint8_t* qs = blk + 32;
                const uint8_t* scd = blk + 96;
                float d = orc_f16_to_f32(rd16(blk + 108));
                int32_t sc[16];
                for (int i = 0; i < 8; ++i) {
                    sc[i] = scd[i] & 0x0F;
                    sc[i + 8] = scd[i] >> 4;
                }
                for (int i = 0; i < 4; ++i) {
                    uint8_t up = scd[8 + i];
                    sc[2 * i] |= (int32_t)(up & 0x03) << 4;
                    sc[2 * i + 1] |= (int32_t)((up >> 2) & 0x03) << 4;
                    sc[2 * i + 8] |= (int32_t)((up >> 4) & 0x03) << 4;
                    sc[2 * i + 9] |= (int32_t)((up >> 6) & 0x03) << 4;
                }
                for (int sub = 0; sub < 16; ++sub) {
                    float sub_scale = (float)(sc[sub] - 32) * d;
                    for (int i = 0; i < 16; ++i) {
                        int elem = sub * 16 + i;
                        uint32_t lo = (qs[elem / 4] >> ((elem % 4) * 2)) & 0x03;
                        uint32_t hb = (hmask[elem / 8] >> (elem % 8)) & 1;
                        uint32_t q = lo | (hb << 2);
                        float t = (float)q - 4.0f;
                        emit(base + elem, t * sub_scale);
                    }
                }
                break;
            }
            case ORC_Q8_K: {  // dequant.rs:582-597
                float d;
                std::memcpy(&d, blk, 4);
                for (int i = 0; i < 256; ++i) emit(base + i, (float)(int8_t)blk[4 + i] * d);
                break;
            }
            default:
                return fail("dequant: unsupported dtype");
        }
    }
    return 0;
}

}  // namespace

extern "C" int orc_dequantize_to_f16(const uint8_t* data, int dtype, uint64_t n,
                                     int nibble_order, uint16_t* out) {
    // dequantize_to_f16 (dequant.rs:33-60)
    return dequant_values(data, dtype, n, nibble_order,
                          [&](uint64_t i, float v) { out[i] = orc_f32_to_f16_rtz(v); });
}

extern "C" int orc_dequantize_to_f32(const uint8_t* data, int dtype, uint64_t n,
                                     int nibble_order, int rtz, float* out) {
    if (dtype == ORC_F32) {
        std::memcpy(out, data, n * 4);
        return 0;
    }
    if (dtype == ORC_F16) {
        for (uint64_t i = 0; i < n; ++i) out[i] = orc_f16_to_f32(rd16(data + 2 * i));
        return 0;
    }
    // Large tensors: independent block ranges on all threads (results do not
    // depend on the split).
    const int64_t bs = orc_block_size(dtype), bb = orc_block_bytes(dtype);
    const uint64_t chunk_blocks = 1 << 14;
    if (bs > 1 && n % (uint64_t)bs == 0 && n / (uint64_t)bs > chunk_blocks) {
        const int64_t nchunks = (int64_t)((n / (uint64_t)bs + chunk_blocks - 1) / chunk_blocks);
        int err = 0;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) reduction(| : err)
#endif
        for (int64_t c = 0; c < nchunks; ++c) {
            const uint64_t b0 = (uint64_t)c * chunk_blocks;
            const uint64_t nb = std::min<uint64_t>(chunk_blocks, n / (uint64_t)bs - b0);
            float* o = out + b0 * (uint64_t)bs;
            err |= orc_dequantize_to_f32(data + b0 * (uint64_t)bb, dtype, nb * (uint64_t)bs, nibble_order, rtz, o);
        }
        return err ? fail("dequant: failed") : 0;
    }
    if (rtz)
        return dequant_values(data, dtype, n, nibble_order, [&](uint64_t i, float v) {
            out[i] = orc_f16_to_f32(orc_f32_to_f16_rtz(v));
        });
    return dequant_values(data, dtype, n, nibble_order,
                          [&](uint64_t i, float v) { out[i] = v; });
}

// ---------------------------------------------------------------------------
// Fixture quantizer. The reference has no GGUF quantizer (its only "quantize"
// is MLX affine, shim/src/ops.cpp:433-461), so this is a deterministic one of
// our own that writes blocks in the layouts dequant.rs reads. The CUDA
// library's quantizer must produce the same bytes.
// ---------------------------------------------------------------------------

namespace {

inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
inline int rint_i(float v) { return (int)std::nearbyint(v); }

}  // namespace

extern "C" int orc_quantize(const float* x, int dtype, uint64_t n, int nibble_order,
                            uint8_t* out) {
    const int64_t bs = orc_block_size(dtype);
    const int64_t bb = orc_block_bytes(dtype);
    if (dtype != ORC_Q4_0 && dtype != ORC_Q8_0 && dtype != ORC_Q4_K)
        return fail("quantize: only Q4_0, Q8_0 and Q4_K are written");
    if (n % (uint64_t)bs) return fail("quantize: element count is not a whole number of blocks");
    const uint64_t nb = n / (uint64_t)bs;
    for (uint64_t b = 0; b < nb; ++b) {
        const float* v = x + b * (uint64_t)bs;
        uint8_t* blk = out + b * (uint64_t)bb;
        if (dtype == ORC_Q4_0 || dtype == ORC_Q8_0) {
            const float qmax = dtype == ORC_Q4_0 ? 7.0f : 127.0f;
            float amax = 0.0f;
            for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(v[i]));
            uint16_t dh = orc_f32_to_f16_rne(amax / qmax);
            float df = orc_f16_to_f32(dh);
            float id = df != 0.0f ? 1.0f / df : 0.0f;
            blk[0] = (uint8_t)(dh & 0xFF);
            blk[1] = (uint8_t)(dh >> 8);
            if (dtype == ORC_Q8_0) {
                for (int i = 0; i < 32; ++i)
                    blk[2 + i] = (uint8_t)(int8_t)clampi(rint_i(v[i] * id), -127, 127);
            } else {
                int q[32];
                for (int i = 0; i < 32; ++i) q[i] = clampi(rint_i(v[i] * id), -8, 7) + 8;
                for (int i = 0; i < 16; ++i) {
                    int lo, hi;
                    if (nibble_order == ORC_NIBBLE_GGUF_SPLIT) {
                        lo = q[i];
                        hi = q[i + 16];
                    } else {
                        lo = q[2 * i];
                        hi = q[2 * i + 1];
                    }
                    blk[2 + i] = (uint8_t)(lo | (hi << 4));
                }
            }
        } else {  // Q4_K
            float scale[8], minv[8];
            float max_scale = 0.0f, max_min = 0.0f;
            for (int j = 0; j < 8; ++j) {
                float lo = 0.0f, hi = -INFINITY;
                for (int i = 0; i < 32; ++i) {
                    lo = std::fmin(lo, v[32 * j + i]);
                    hi = std::fmax(hi, v[32 * j + i]);
                }
                scale[j] = (hi - lo) / 15.0f;
                minv[j] = -lo;
                max_scale = std::fmax(max_scale, scale[j]);
                max_min = std::fmax(max_min, minv[j]);
            }
            uint16_t dh = orc_f32_to_f16_rne(max_scale / 63.0f);
            uint16_t mh = orc_f32_to_f16_rne(max_min / 63.0f);
            float df = orc_f16_to_f32(dh), mf = orc_f16_to_f32(mh);
            int sc[8], mn[8];
            for (int j = 0; j < 8; ++j) {
                sc[j] = df > 0.0f ? clampi(rint_i(scale[j] / df), 0, 63) : 0;
                mn[j] = mf > 0.0f ? clampi(rint_i(minv[j] / mf), 0, 63) : 0;
            }
            blk[0] = (uint8_t)(dh & 0xFF);
            blk[1] = (uint8_t)(dh >> 8);
            blk[2] = (uint8_t)(mh & 0xFF);
            blk[3] = (uint8_t)(mh >> 8);
            uint8_t* s = blk + 4;
            for (int j = 0; j < 4; ++j) {
                s[j] = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
                s[j + 4] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
                s[j + 8] = (uint8_t)((sc[j + 4] & 0x0F) | ((mn[j + 4] & 0x0F) << 4));
            }
            uint8_t* qs = blk + 16;
            int q[256];
            for (int j = 0; j < 8; ++j) {
                float es = df * (float)sc[j];
                float em = mf * (float)mn[j];
                for (int i = 0; i < 32; ++i) {
                    float t = v[32 * j + i] + em;
                    q[32 * j + i] = es > 0.0f ? clampi(rint_i(t / es), 0, 15) : 0;
                }
            }
            for (int p = 0; p < 4; ++p)
                for (int j = 0; j < 32; ++j)
                    qs[32 * p + j] = (uint8_t)(q[64 * p + j] | (q[64 * p + 32 + j] << 4));
        }
    }
    return 0;
}

// ---------------------------------------------------------------------------
// beacon-kernels ops (crates/beacon-kernels/src/ops.rs, q4.rs)
// ---------------------------------------------------------------------------

extern "C" void orc_q4_dequantize_block(const uint8_t* block, float* out) {
    // q4.rs:26-42 (f32 values, no f16 rounding)
    float scale = orc_f16_to_f32(rd16(block));
    for (int i = 0; i < 16; ++i) {
        uint8_t byte = block[2 + i];
        int8_t lo = (int8_t)(byte & 0x0F) - 8;
        int8_t hi = (int8_t)((byte >> 4) & 0x0F) - 8;
        out[i * 2] = (float)lo * scale;
        out[i * 2 + 1] = (float)hi * scale;
    }
}

extern "C" float orc_q4_dot_f32(const float* x, const uint8_t* w_q4, size_t k) {
    // ops.rs:38-56: one sequential f32 accumulator over blocks and elements.
    size_t nb = k / 32;
    float sum = 0.0f;
    float deq[32];
    for (size_t b = 0; b < nb; ++b) {
        orc_q4_dequantize_block(w_q4 + b * 18, deq);
        for (int i = 0; i < 32; ++i) sum += deq[i] * x[b * 32 + i];
    }
    return sum;
}

extern "C" void orc_q4_matmul_f32(const uint8_t* w_q4, const float* x, float* out,
                                  size_t m, size_t k) {
    // ops.rs:62-70
    size_t row_bytes = k / 32 * 18;
    for (size_t i = 0; i < m; ++i) out[i] = orc_q4_dot_f32(x, w_q4 + i * row_bytes, k);
}

// Quantized GEMV for every format: y[b][n] = sum_k deq[n][k] * x[b][k], one
// sequential accumulator per output in ascending k -- the order of
// q4_dot_f32 (ops.rs:38-56) and of matmul_f32 (ops.rs:16-30) after the
// engine's transpose (engine.rs:150-152). `rtz` selects the weight values the
// CPU engine uses (f16-rounded by dequantize_to_f16) or the unrounded ones.
extern "C" int orc_qgemv_f32(const uint8_t* w, int dtype, int nibble_order, int rtz,
                             int64_t n, int64_t k, const float* x, int64_t batch,
                             float* y, int threads) {
    const int64_t bs = orc_block_size(dtype);
    if (bs <= 1 && dtype != ORC_F32 && dtype != ORC_F16) return fail("qgemv: bad dtype");
    if (bs > 1 && k % bs) return fail("qgemv: k is not a whole number of blocks");
    const int64_t row_bytes = bs > 1 ? k / bs * orc_block_bytes(dtype) : k * orc_block_bytes(dtype);
    int err = 0;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for num_threads(threads) schedule(static) reduction(| : err)
#endif
    for (int64_t r = 0; r < n; ++r) {
        std::vector<float> row((size_t)k);
        if (orc_dequantize_to_f32(w + r * row_bytes, dtype, (uint64_t)k, nibble_order, rtz,
                                  row.data()) != 0) {
            err |= 1;
            continue;
        }
        for (int64_t b = 0; b < batch; ++b) {
            const float* xb = x + b * k;
            float sum = 0.0f;
            for (int64_t i = 0; i < k; ++i) sum += row[(size_t)i] * xb[i];
            y[b * n + r] = sum;
        }
    }
    return err ? fail("qgemv: dequant failed") : 0;
}

extern "C" void orc_matmul_f32(const float* a, const float* b, float* c, size_t m,
                               size_t k, size_t n) {
    // ops.rs:16-30
    for (size_t i = 0; i < m; ++i)
        for (size_t j = 0; j < n; ++j) {
            float sum = 0.0f;
            for (size_t p = 0; p < k; ++p) sum += a[i * k + p] * b[p * n + j];
            c[i * n + j] = sum;
        }
}

extern "C" void orc_transpose_f32(const float* x, float* out, size_t batch, size_t m,
                                  size_t n) {
    // cpu_backend.rs:330-366
    for (size_t b = 0; b < batch; ++b) {
        size_t off = b * m * n;
        for (size_t i = 0; i < m; ++i)
            for (size_t j = 0; j < n; ++j) out[off + j * m + i] = x[off + i * n + j];
    }
}

extern "C" void orc_rms_norm(const float* x, const float* w, float* out, size_t n, float eps) {
    // ops.rs:77-93
    float sum_sq = 0.0f;
    for (size_t i = 0; i < n; ++i) sum_sq += x[i] * x[i];
    float rms = std::sqrt(sum_sq / (float)n + eps);
    float inv_rms = 1.0f / rms;
    for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv_rms * w[i];
}

extern "C" void orc_silu_inplace(float* x, size_t n) {
    // ops.rs:96-100
    for (size_t i = 0; i < n; ++i) x[i] *= 1.0f / (1.0f + std::exp(-x[i]));
}

extern "C" void orc_softmax_inplace(float* x, size_t n) {
    // ops.rs:105-116
    float mx = -INFINITY;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, x[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        x[i] = std::exp(x[i] - mx);
        sum += x[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

extern "C" void orc_rope_inplace(float* x, size_t seq_len, size_t dim, size_t position_offset,
                                 float theta) {
    // ops.rs:124-142: interleaved pairs (i, i+1)
    for (size_t s = 0; s < seq_len; ++s) {
        float pos = (float)(position_offset + s);
        float* row = x + s * dim;
        for (size_t i = 0; i < dim; i += 2) {
            float freq = 1.0f / std::pow(theta, (float)i / (float)dim);
            float angle = pos * freq;
            float c = std::cos(angle), sn = std::sin(angle);
            float x0 = row[i], x1 = row[i + 1];
            float a = x0 * c, b = x1 * sn, d = x0 * sn, e = x1 * c;
            row[i] = a - b;
            row[i + 1] = d + e;
        }
    }
}

extern "C" void orc_add(const float* a, const float* b, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] + b[i];  // ops.rs:145-151
}

extern "C" void orc_mul(const float* a, const float* b, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = a[i] * b[i];  // ops.rs:154-160
}

extern "C" int orc_attention(const float* q, const float* k, const float* v, const float* mask,
                             size_t mask_numel, float scale, size_t batch, size_t n_heads,
                             size_t seq_q, size_t head_dim, size_t n_kv_heads, size_t seq_kv,
                             int causal, float* out) {
    // cpu_backend.rs:511-598. `causal` adds the -inf upper triangle that the
    // MLX path enables for seq_q > 1 (shim/src/ops.cpp:216-223), aligned to
    // the end of the key range.
    if (n_kv_heads == 0 || n_heads % n_kv_heads) return fail("attention: n_heads % n_kv_heads != 0");
    size_t per = n_heads / n_kv_heads;
    std::vector<float> scores(seq_kv);
    for (size_t b = 0; b < batch; ++b)
        for (size_t h = 0; h < n_heads; ++h) {
            size_t kv_h = h / per;
            for (size_t sq = 0; sq < seq_q; ++sq) {
                size_t qo = ((b * n_heads + h) * seq_q + sq) * head_dim;
                for (size_t sk = 0; sk < seq_kv; ++sk) {
                    size_t ko = ((b * n_kv_heads + kv_h) * seq_kv + sk) * head_dim;
                    float dot = 0.0f;
                    for (size_t d = 0; d < head_dim; ++d) dot += q[qo + d] * k[ko + d];
                    scores[sk] = dot * scale;
                }
                if (mask) {
                    size_t row_len = mask_numel >= seq_q * seq_kv ? seq_kv : mask_numel;
                    if (row_len == seq_kv) {
                        size_t mo = sq * seq_kv;
                        for (size_t sk = 0; sk < seq_kv; ++sk)
                            if (mo + sk < mask_numel) scores[sk] += mask[mo + sk];
                    }
                }
                if (causal) {
                    size_t limit = sq + (seq_kv - seq_q);
                    for (size_t sk = limit + 1; sk < seq_kv; ++sk) scores[sk] += -INFINITY;
                }
                orc_softmax_inplace(scores.data(), seq_kv);
                size_t oo = ((b * n_heads + h) * seq_q + sq) * head_dim;
                for (size_t d = 0; d < head_dim; ++d) {
                    float val = 0.0f;
                    for (size_t sk = 0; sk < seq_kv; ++sk) {
                        size_t vo = ((b * n_kv_heads + kv_h) * seq_kv + sk) * head_dim;
                        val += scores[sk] * v[vo + d];
                    }
                    out[oo + d] = val;
                }
            }
        }
    return 0;
}

extern "C" uint32_t orc_argmax(const float* logits, size_t n) {
    // sampling.rs:60-66 / engine.rs:256-261: Iterator::max_by keeps the
    // current best only when it compares Greater, so ties (and NaN, which
    // compares Equal) move to the later index; empty -> 0.
    if (n == 0) return 0;
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (!(logits[best] > logits[i])) best = i;
    return (uint32_t)best;
}

// ---------------------------------------------------------------------------
// Engine (crates/beacon-core/src/engine.rs:86-456 with CpuBackend)
// ---------------------------------------------------------------------------

namespace {

struct Layer {
    std::vector<float> attn_norm, ffn_norm, q, k, v, o, gate, up, down;
};

struct Model {
    OrcModelConfig cfg;
    std::vector<float> embed, final_norm, lm_head;
    std::vector<Layer> layers;
    std::vector<std::vector<float>> cache_k, cache_v;  // [max_ctx, n_kv, hd]
};

// proj_matmul(Plain) = transpose + matmul (engine.rs:150-152): for every row
// of x and output column j, sum_p x[i][p] * W[j][p] in ascending p. The
// transpose only relabels W, so reading W row-major gives the same sums.
void linear(const Model& m, const float* x, size_t rows, const std::vector<float>& w,
            size_t n, size_t k, float* y) {
    if (m.cfg.ref_faithful) {
        // the reference's own loop order, single-threaded: transpose W [n, k]
        // into a new [k, n] buffer on every call, then matmul_f32 with its
        // column-strided inner loop
        std::vector<float> wt(n * k);
        orc_transpose_f32(w.data(), wt.data(), 1, n, k);
        orc_matmul_f32(x, wt.data(), y, rows, k, n);
        return;
    }
    int threads = m.cfg.threads;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for num_threads(threads) schedule(static)
#endif
    for (int64_t j = 0; j < (int64_t)n; ++j) {
        const float* wr = w.data() + (size_t)j * k;
        for (size_t i = 0; i < rows; ++i) {
            const float* xr = x + i * k;
            float sum = 0.0f;
            for (size_t p = 0; p < k; ++p) sum += xr[p] * wr[p];
            y[i * n + (size_t)j] = sum;
        }
    }
}

}  // namespace

extern "C" void* orc_model_create(const OrcModelConfig* cfg) {
    if (!cfg) return nullptr;
    Model* m = new Model();
    m->cfg = *cfg;
    m->layers.resize((size_t)cfg->num_layers);
    size_t kv = (size_t)cfg->max_context * cfg->num_kv_heads * cfg->head_dim;
    m->cache_k.assign((size_t)cfg->num_layers, std::vector<float>(kv, 0.0f));
    m->cache_v.assign((size_t)cfg->num_layers, std::vector<float>(kv, 0.0f));
    return m;
}

extern "C" void orc_model_destroy(void* model) { delete static_cast<Model*>(model); }

extern "C" void orc_model_reset(void* model) {
    Model* m = static_cast<Model*>(model);
    for (auto& c : m->cache_k) std::fill(c.begin(), c.end(), 0.0f);
    for (auto& c : m->cache_v) std::fill(c.begin(), c.end(), 0.0f);
}

extern "C" int orc_model_set_weight(void* model, int layer, int which, const void* data,
                                    int dtype, int nibble_order) {
    Model* m = static_cast<Model*>(model);
    const OrcModelConfig& c = m->cfg;
    size_t H = (size_t)c.hidden_size, F = (size_t)c.intermediate_size, V = (size_t)c.vocab_size;
    size_t QD = (size_t)c.num_heads * c.head_dim, KD = (size_t)c.num_kv_heads * c.head_dim;
    std::vector<float>* dst = nullptr;
    size_t n = 0;
    if (which < 10) {
        switch (which) {
            case ORC_W_EMBED: dst = &m->embed; n = V * H; break;
            case ORC_W_FINAL_NORM: dst = &m->final_norm; n = H; break;
            case ORC_W_LM_HEAD: dst = &m->lm_head; n = V * H; break;
            default: return fail("set_weight: unknown slot");
        }
    } else {
        if (layer < 0 || layer >= c.num_layers) return fail("set_weight: bad layer");
        Layer& L = m->layers[(size_t)layer];
        switch (which) {
            case ORC_W_ATTN_NORM: dst = &L.attn_norm; n = H; break;
            case ORC_W_FFN_NORM: dst = &L.ffn_norm; n = H; break;
            case ORC_W_Q: dst = &L.q; n = QD * H; break;
            case ORC_W_K: dst = &L.k; n = KD * H; break;
            case ORC_W_V: dst = &L.v; n = KD * H; break;
            case ORC_W_O: dst = &L.o; n = H * QD; break;
            case ORC_W_GATE: dst = &L.gate; n = F * H; break;
            case ORC_W_UP: dst = &L.up; n = F * H; break;
            case ORC_W_DOWN: dst = &L.down; n = H * F; break;
            default: return fail("set_weight: unknown slot");
        }
    }
    dst->assign(n, 0.0f);
    return orc_dequantize_to_f32(static_cast<const uint8_t*>(data), dtype, n, nibble_order,
                                 c.weights_rtz, dst->data());
}

extern "C" int orc_model_forward(void* model, const uint32_t* tokens, size_t S, size_t position,
                                 float* logits_out) {
    Model* m = static_cast<Model*>(model);
    const OrcModelConfig& c = m->cfg;
    const size_t H = (size_t)c.hidden_size, F = (size_t)c.intermediate_size;
    const size_t V = (size_t)c.vocab_size, NH = (size_t)c.num_heads, NKV = (size_t)c.num_kv_heads;
    const size_t D = (size_t)c.head_dim, QD = NH * D, KD = NKV * D;
    if (S == 0) return fail("forward: empty token list");
    // 1. embedding (cpu_backend.rs:387-418)
    std::vector<float> h(S * H);
    for (size_t s = 0; s < S; ++s) {
        size_t idx = (size_t)(float)tokens[s];  // create_token_tensor stores ids as f32
        if (idx >= V) return fail("forward: embedding index out of bounds");
        std::memcpy(&h[s * H], &m->embed[idx * H], H * 4);
    }
    std::vector<float> normed(S * H), q(S * QD), k(S * KD), v(S * KD);
    std::vector<float> qt(S * QD), kt(S * KD), vt(S * KD), attn(S * QD), attn_sd(S * QD);
    std::vector<float> o(S * H), gate(S * F), up(S * F), inter(S * F), down(S * H);
    const float scale = 1.0f / std::sqrt((float)D);  // engine.rs:415
    for (size_t li = 0; li < (size_t)c.num_layers; ++li) {
        const Layer& L = m->layers[li];
        for (size_t s = 0; s < S; ++s)
            orc_rms_norm(&h[s * H], L.attn_norm.data(), &normed[s * H], H, c.rms_norm_eps);
        // attention_block (engine.rs:277-429)
        linear(*m, normed.data(), S, L.q, QD, H, q.data());
        linear(*m, normed.data(), S, L.k, KD, H, k.data());
        linear(*m, normed.data(), S, L.v, KD, H, v.data());
        // reshape [1,S,heads,D] + swapaxes(1,2) -> [1,heads,S,D]
        for (size_t s = 0; s < S; ++s) {
            for (size_t hh = 0; hh < NH; ++hh)
                std::memcpy(&qt[(hh * S + s) * D], &q[s * QD + hh * D], D * 4);
            for (size_t hh = 0; hh < NKV; ++hh) {
                std::memcpy(&kt[(hh * S + s) * D], &k[s * KD + hh * D], D * 4);
                std::memcpy(&vt[(hh * S + s) * D], &v[s * KD + hh * D], D * 4);
            }
        }
        // rope per (batch*head) group (cpu_backend.rs:141-180)
        for (size_t hh = 0; hh < NH; ++hh)
            orc_rope_inplace(&qt[hh * S * D], S, D, position, c.rope_theta);
        for (size_t hh = 0; hh < NKV; ++hh)
            orc_rope_inplace(&kt[hh * S * D], S, D, position, c.rope_theta);
        if (position + S > (size_t)c.max_context) return fail("forward: context overflow");
        // kv_cache_update (cpu_backend.rs:435-483): rows [position, position+S)
        const size_t L_len = position + S;
        std::vector<float> ck, cv;
        std::vector<float>* kc;
        std::vector<float>* vc;
        if (c.kv_persist) {
            kc = &m->cache_k[li];
            vc = &m->cache_v[li];
        } else {  // the literal CPU path writes into a clone that is dropped
            ck = m->cache_k[li];
            cv = m->cache_v[li];
            kc = &ck;
            vc = &cv;
        }
        for (size_t s = 0; s < S; ++s)
            for (size_t hh = 0; hh < NKV; ++hh) {
                std::memcpy(&(*kc)[((position + s) * NKV + hh) * D], &kt[(hh * S + s) * D], D * 4);
                std::memcpy(&(*vc)[((position + s) * NKV + hh) * D], &vt[(hh * S + s) * D], D * 4);
            }
        // views [L, NKV, D] -> [1, NKV, L, D]
        std::vector<float> kf(NKV * L_len * D), vf(NKV * L_len * D);
        for (size_t t = 0; t < L_len; ++t)
            for (size_t hh = 0; hh < NKV; ++hh) {
                std::memcpy(&kf[(hh * L_len + t) * D], &(*kc)[(t * NKV + hh) * D], D * 4);
                std::memcpy(&vf[(hh * L_len + t) * D], &(*vc)[(t * NKV + hh) * D], D * 4);
            }
        if (orc_attention(qt.data(), kf.data(), vf.data(), nullptr, 0, scale, 1, NH, S, D, NKV,
                          L_len, c.causal_prefill && S > 1, attn.data()) != 0)
            return -1;
        // swapaxes back -> [S, NH*D]
        for (size_t s = 0; s < S; ++s)
            for (size_t hh = 0; hh < NH; ++hh)
                std::memcpy(&attn_sd[s * QD + hh * D], &attn[(hh * S + s) * D], D * 4);
        linear(*m, attn_sd.data(), S, L.o, H, QD, o.data());
        orc_add(h.data(), o.data(), h.data(), S * H);
        // ffn_block (engine.rs:436-456)
        for (size_t s = 0; s < S; ++s)
            orc_rms_norm(&h[s * H], L.ffn_norm.data(), &normed[s * H], H, c.rms_norm_eps);
        linear(*m, normed.data(), S, L.gate, F, H, gate.data());
        orc_silu_inplace(gate.data(), S * F);
        linear(*m, normed.data(), S, L.up, F, H, up.data());
        orc_mul(gate.data(), up.data(), inter.data(), S * F);
        linear(*m, inter.data(), S, L.down, H, F, down.data());
        orc_add(h.data(), down.data(), h.data(), S * H);
    }
    for (size_t s = 0; s < S; ++s)
        orc_rms_norm(&h[s * H], m->final_norm.data(), &normed[s * H], H, c.rms_norm_eps);
    linear(*m, normed.data(), S, m->lm_head, V, H, logits_out);
    return 0;
}

extern "C" const char* orc_last_error(void) { return g_err.c_str(); }

// ---------------------------------------------------------------------------
// Sampling pipeline (crates/beacon-scheduler/src/sampling.rs:15-186):
// repeat penalty -> temperature (greedy at <= f32::EPSILON) -> top-k -> top-p
// -> min-p -> softmax -> multinomial draw. The reference draws
// r = rng.random::<f32>() from an unseeded thread RNG; here r is an input so
// that the draw can be replayed. The stages run in the reference's order and
// its f32 arithmetic (sequential sums in index order, sort by descending
// value). probs_out (optional, n floats): the distribution the draw used.
// ---------------------------------------------------------------------------

namespace {

const float kF32Eps = 1.1920929e-07f;  // f32::EPSILON

// sampling.rs:173-186 (softmax_inplace)
void sample_softmax(std::vector<float>& x) {
    float mx = -INFINITY;
    for (float v : x) mx = std::fmax(mx, v);  // fold(NEG_INFINITY, f32::max)
    float sum = 0.0f;
    for (float& v : x) {
        v = std::exp(v - mx);
        sum += v;
    }
    if (sum > 0.0f) {
        const float inv = 1.0f / sum;
        for (float& v : x) v *= inv;
    }
}

// partial_cmp(a, b).unwrap_or(Equal) == Greater, i.e. a > b without NaN
bool desc_before(float a, float b) { return a > b; }

}  // namespace

extern "C" uint32_t orc_sample(const float* logits_in, size_t n, const uint32_t* prev, size_t n_prev,
                               const OrcSampleParams* p, float r, float* probs_out) {
    std::vector<float> logits(logits_in, logits_in + n);
    // 1. repeat penalty (sampling.rs:77-88), once per occurrence
    if (std::fabs(p->repeat_penalty - 1.0f) > kF32Eps) {
        for (size_t i = 0; i < n_prev; ++i) {
            const size_t idx = prev[i];
            if (idx < n) logits[idx] = logits[idx] > 0.0f ? logits[idx] / p->repeat_penalty
                                                          : logits[idx] * p->repeat_penalty;
        }
    }
    // 2. temperature (sampling.rs:27-34, 91-96)
    if (p->temperature <= kF32Eps) return orc_argmax(logits.data(), n);
    if (std::fabs(p->temperature - 1.0f) > kF32Eps) {
        const float inv_t = 1.0f / p->temperature;
        for (float& v : logits) v *= inv_t;
    }
    // 3. top-k (sampling.rs:99-114): threshold = sorted_desc[k], drop v < threshold
    if (p->has_top_k && (size_t)p->top_k < n) {
        std::vector<float> sorted(logits);
        std::sort(sorted.begin(), sorted.end(), desc_before);
        const float threshold = sorted[(size_t)p->top_k];
        for (float& v : logits)
            if (v < threshold) v = -INFINITY;
    }
    // 4. top-p (sampling.rs:117-145)
    if (p->has_top_p && p->top_p < 1.0f) {
        std::vector<float> probs(logits);
        sample_softmax(probs);
        std::vector<size_t> idx(n);
        for (size_t i = 0; i < n; ++i) idx[i] = i;
        std::sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return probs[a] > probs[b]; });
        float cumulative = 0.0f;
        size_t cutoff = n;
        for (size_t i = 0; i < n; ++i) {
            cumulative += probs[idx[i]];
            if (cumulative > p->top_p) {
                cutoff = i + 1;
                break;
            }
        }
        for (size_t i = cutoff; i < n; ++i) logits[idx[i]] = -INFINITY;
    }
    // 5. min-p (sampling.rs:148-160)
    if (p->has_min_p && p->min_p > 0.0f) {
        std::vector<float> probs(logits);
        sample_softmax(probs);
        float max_prob = 0.0f;
        for (float v : probs) max_prob = std::fmax(max_prob, v);
        const float threshold = p->min_p * max_prob;
        for (size_t i = 0; i < n; ++i)
            if (probs[i] < threshold) logits[i] = -INFINITY;
    }
    // 6. softmax + multinomial (sampling.rs:53-56, 163-186)
    sample_softmax(logits);
    if (probs_out) std::memcpy(probs_out, logits.data(), n * sizeof(float));
    float cumulative = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        cumulative += logits[i];
        if (cumulative >= r) return (uint32_t)i;
    }
    return n ? (uint32_t)(n - 1) : 0u;
}
