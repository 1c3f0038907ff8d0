// quant.cu -- GGUF block layout kernels:
//  * repack: raw GGUF rows (blocks along K) -> row-group tiles (QLayout);
//  * dequant_f16: tiles -> f16 bits, bit-exact with dequantize_to_f16
//    (crates/beacon-format/src/dequant.rs:33-60, 160-178, 258-273, 289-365);
//  * quantize: f32 -> GGUF blocks with the deterministic fixture quantizer
//    (the reference has none; the CPU oracle writes identical bytes).
// The other block types (Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q5_K, Q6_K, Q8_K,
// dequant.rs:182-254, 377-597) keep their raw bytes per tile
// (gemv_generic.cuh).
#include <algorithm>

#include "common.cuh"
#include "gemv_generic.cuh"
#include "internal.h"
#include "kernels.h"

namespace bc {

namespace {

__device__ __forceinline__ void store16(uint8_t* dst, const uint8_t (&b)[16]) {
    uint4 v;
    uint32_t* w = &v.x;
#pragma unroll
    for (int i = 0; i < 4; ++i)
        w[i] = (uint32_t)b[4 * i] | ((uint32_t)b[4 * i + 1] << 8) | ((uint32_t)b[4 * i + 2] << 16) |
               ((uint32_t)b[4 * i + 3] << 24);
    *reinterpret_cast<uint4*>(dst) = v;
}

// One thread per (tiled row r, k-tile t): writes the row's 16-byte meta and
// its 16-byte qs chunks. row_map (optional) names the raw row that fills
// tiled row r (-1: zero row).
__global__ void repack_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ tiled,
                              int32_t dtype, int64_t n, int64_t k, int64_t n_pad, int64_t ktiles,
                              int64_t tile_bytes, int chunks, int nibble_split,
                              const int64_t* __restrict__ row_map) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_pad * ktiles) return;
    const int64_t r = idx / ktiles, t = idx - r * ktiles;
    int64_t src_row = r < n ? r : -1;
    if (row_map) {
        src_row = row_map[r];
        if (src_row == -2) return;
    }
    const int64_t g = r / 32, lane = r % 32;
    uint8_t* base = tiled + (g * ktiles + t) * tile_bytes;
    uint8_t meta[16] = {0};
    if (dtype == BEACON_CUDA_DTYPE_Q4_K) {
        const int64_t nsb = k / 256, row_bytes = nsb * 144;
        const uint8_t* src = (src_row >= 0 && t < nsb) ? raw + src_row * row_bytes + t * 144 : nullptr;
        if (src) {
#pragma unroll
            for (int i = 0; i < 16; ++i) meta[i] = src[i];
        }
        store16(base + lane * 16, meta);
        for (int c = 0; c < 8; ++c) {
            uint8_t q[16] = {0};
            if (src) {
#pragma unroll
                for (int i = 0; i < 16; ++i) q[i] = src[16 + 16 * c + i];
            }
            store16(base + 512 + c * 512 + lane * 16, q);
        }
        return;
    }
    // 32-element formats: 8 blocks per 256-column tile
    const int64_t nb = k / 32;
    const int64_t bbytes = dtype == BEACON_CUDA_DTYPE_Q8_0 ? 34 : 18;
    const int64_t row_bytes = nb * bbytes;
    for (int c = 0; c < 8; ++c) {
        const int64_t blk = t * 8 + c;
        const uint8_t* src = (src_row >= 0 && blk < nb) ? raw + src_row * row_bytes + blk * bbytes : nullptr;
        if (src) {
            meta[2 * c] = src[0];
            meta[2 * c + 1] = src[1];
        }
        if (dtype == BEACON_CUDA_DTYPE_Q8_0) {
            for (int h = 0; h < 2; ++h) {
                uint8_t q[16] = {0};
                if (src) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) q[i] = src[2 + 16 * h + i];
                }
                store16(base + 512 + (2 * c + h) * 512 + lane * 16, q);
            }
        } else {
            uint8_t q[16] = {0};
            if (src) {
                if (nibble_split) {
                    // GGUF order (byte i -> elements i, i+16) to the canonical
                    // interleaved order (byte i -> elements 2i, 2i+1).
                    uint8_t nib[32];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        nib[i] = src[2 + i] & 0x0F;
                        nib[i + 16] = src[2 + i] >> 4;
                    }
#pragma unroll
                    for (int i = 0; i < 16; ++i) q[i] = (uint8_t)(nib[2 * i] | (nib[2 * i + 1] << 4));
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) q[i] = src[2 + i];
                }
            }
            store16(base + 512 + c * 512 + lane * 16, q);
        }
    }
    store16(base + lane * 16, meta);
}

// One thread per (row, 32-element group): 32 f16 outputs.
__global__ void dequant_f16_kernel(const uint8_t* __restrict__ tiled, uint16_t* __restrict__ out,
                                   int32_t dtype, int64_t n, int64_t k, int64_t ktiles,
                                   int64_t tile_bytes) {
    const int64_t ngrp = k / 32;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n * ngrp) return;
    const int64_t r = idx / ngrp, j = idx - r * ngrp;
    const int64_t t = j / 8, sub = j % 8;
    const int64_t g = r / 32, lane = r % 32;
    const uint8_t* base = tiled + (g * ktiles + t) * tile_bytes;
    const uint4 meta = *reinterpret_cast<const uint4*>(base + lane * 16);
    uint16_t o[32];
    if (dtype == BEACON_CUDA_DTYPE_Q4_0) {
        const uint32_t mw = (&meta.x)[sub >> 1];
        const float d = f16_to_f32((uint16_t)((sub & 1) ? (mw >> 16) : (mw & 0xFFFF)));
        const uint4 q = *reinterpret_cast<const uint4*>(base + 512 + sub * 512 + lane * 16);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            uint32_t byte = ((&q.x)[i >> 2] >> (8 * (i & 3))) & 0xFF;
            float lo = (float)((int)(byte & 0x0F) - 8), hi = (float)((int)(byte >> 4) - 8);
            o[2 * i] = f32_to_f16_rtz(x86_mul(lo, d));
            o[2 * i + 1] = f32_to_f16_rtz(x86_mul(hi, d));
        }
    } else if (dtype == BEACON_CUDA_DTYPE_Q8_0) {
        const uint32_t mw = (&meta.x)[sub >> 1];
        const float d = f16_to_f32((uint16_t)((sub & 1) ? (mw >> 16) : (mw & 0xFFFF)));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 q = *reinterpret_cast<const uint4*>(base + 512 + (2 * sub + h) * 512 + lane * 16);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                int8_t v = (int8_t)(((&q.x)[i >> 2] >> (8 * (i & 3))) & 0xFF);
                o[16 * h + i] = f32_to_f16_rtz(x86_mul((float)v, d));
            }
        }
    } else {  // Q4_K: group sub = sub-block; pair p = sub/2, high nibbles when sub is odd
        const float d = f16_to_f32((uint16_t)(meta.x & 0xFFFF));
        const float dmin = f16_to_f32((uint16_t)(meta.x >> 16));
        uint8_t sq[12];
#pragma unroll
        for (int i = 0; i < 12; ++i) sq[i] = (uint8_t)((&meta.y)[i >> 2] >> (8 * (i & 3)));
        int rs, rm;
        if (sub < 4) {
            rs = sq[sub] & 0x3F;
            rm = sq[sub + 4] & 0x3F;
        } else {
            rs = (sq[sub + 4] & 0x0F) | ((sq[sub - 4] >> 6) << 4);
            rm = (sq[sub + 4] >> 4) | ((sq[sub] >> 6) << 4);
        }
        const float sc = x86_mul((float)rs, d), mn = x86_mul((float)rm, dmin);
        const int p = (int)(sub / 2), hi = (int)(sub & 1);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint4 q = *reinterpret_cast<const uint4*>(base + 512 + (2 * p + h) * 512 + lane * 16);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                uint32_t byte = ((&q.x)[i >> 2] >> (8 * (i & 3))) & 0xFF;
                float w = (float)(hi ? (byte >> 4) : (byte & 0x0F));
                o[16 * h + i] = f32_to_f16_rtz(x86_sub(x86_mul(w, sc), mn));
            }
        }
    }
    uint4* dst = reinterpret_cast<uint4*>(out + r * k + j * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint4 v;
        uint32_t* w = &v.x;
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = (uint32_t)o[8 * c + 2 * i] | ((uint32_t)o[8 * c + 2 * i + 1] << 16);
        dst[c] = v;
    }
}

__device__ __forceinline__ uint16_t f16_rne_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Deterministic quantizer; operation for operation the same as
// orc_quantize in the oracle (explicit _rn intrinsics, nothing contracted).
__global__ void quantize_kernel(const float* __restrict__ x, uint8_t* __restrict__ out, int32_t dtype,
                                int64_t nblocks, int nibble_split) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblocks) return;
    if (dtype == BEACON_CUDA_DTYPE_Q4_0 || dtype == BEACON_CUDA_DTYPE_Q8_0) {
        const float* v = x + b * 32;
        uint8_t* blk = out + b * (dtype == BEACON_CUDA_DTYPE_Q4_0 ? 18 : 34);
        const float qmax = dtype == BEACON_CUDA_DTYPE_Q4_0 ? 7.0f : 127.0f;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        uint16_t dh = f16_rne_bits(__fdiv_rn(amax, qmax));
        float df = f16_to_f32(dh);
        float id = df != 0.0f ? __fdiv_rn(1.0f, df) : 0.0f;
        blk[0] = (uint8_t)(dh & 0xFF);
        blk[1] = (uint8_t)(dh >> 8);
        if (dtype == BEACON_CUDA_DTYPE_Q8_0) {
            for (int i = 0; i < 32; ++i)
                blk[2 + i] = (uint8_t)(int8_t)clampi(__float2int_rn(__fmul_rn(v[i], id)), -127, 127);
        } else {
            int q[32];
            for (int i = 0; i < 32; ++i) q[i] = clampi(__float2int_rn(__fmul_rn(v[i], id)), -8, 7) + 8;
            for (int i = 0; i < 16; ++i) {
                int lo = nibble_split ? q[i] : q[2 * i];
                int hi = nibble_split ? q[i + 16] : q[2 * i + 1];
                blk[2 + i] = (uint8_t)(lo | (hi << 4));
            }
        }
        return;
    }
    // Q4_K
    const float* v = x + b * 256;
    uint8_t* blk = out + b * 144;
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = -INFINITY;
        for (int i = 0; i < 32; ++i) {
            lo = fminf(lo, v[32 * j + i]);
            hi = fmaxf(hi, v[32 * j + i]);
        }
        scale[j] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        minv[j] = -lo;
        max_scale = fmaxf(max_scale, scale[j]);
        max_min = fmaxf(max_min, minv[j]);
    }
    uint16_t dh = f16_rne_bits(__fdiv_rn(max_scale, 63.0f));
    uint16_t mh = f16_rne_bits(__fdiv_rn(max_min, 63.0f));
    float df = f16_to_f32(dh), mf = f16_to_f32(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = df > 0.0f ? clampi(__float2int_rn(__fdiv_rn(scale[j], df)), 0, 63) : 0;
        mn[j] = mf > 0.0f ? clampi(__float2int_rn(__fdiv_rn(minv[j], mf)), 0, 63) : 0;
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
    for (int p = 0; p < 4; ++p) {
        for (int h = 0; h < 2; ++h) {
            const int j = 2 * p + h;
            const float es = __fmul_rn(df, (float)sc[j]);
            const float em = __fmul_rn(mf, (float)mn[j]);
            for (int i = 0; i < 32; ++i) {
                float t = __fadd_rn(v[32 * j + i], em);
                int q = es > 0.0f ? clampi(__float2int_rn(__fdiv_rn(t, es)), 0, 15) : 0;
                if (h == 0)
                    qs[32 * p + i] = (uint8_t)q;
                else
                    qs[32 * p + i] |= (uint8_t)(q << 4);
            }
        }
    }
}

inline unsigned blocks_for(int64_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

// Generic formats (gemv_generic.cuh): tile t of row r holds the raw bytes of
// the row's 256 columns [256 t, 256 t + 256), zero-padded to whole chunks.
// One thread per (tiled row, k-tile); row_map as for repack_kernel.
__global__ void repack_generic_kernel(const uint8_t* __restrict__ raw, uint8_t* __restrict__ tiled, int64_t n,
                                      int64_t row_bytes, int64_t slice, int64_t n_pad, int64_t ktiles,
                                      int64_t tile_bytes, int chunks_total, const int64_t* __restrict__ row_map) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_pad * ktiles) return;
    const int64_t r = idx / ktiles, t = idx - r * ktiles;
    int64_t src_row = r < n ? r : -1;
    if (row_map) {
        src_row = row_map[r];
        if (src_row == -2) return;
    }
    const int64_t g = r / 32, lane = r % 32;
    uint8_t* base = tiled + (g * ktiles + t) * tile_bytes + lane * 16;
    const int64_t off = t * slice;
    const int64_t avail = src_row >= 0 ? std::max<int64_t>(0, std::min<int64_t>(slice, row_bytes - off)) : 0;
    const uint8_t* src = src_row >= 0 ? raw + src_row * row_bytes + off : nullptr;
    for (int c = 0; c < chunks_total; ++c) {
        uint8_t b[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int64_t j = (int64_t)c * 16 + i;
            b[i] = j < avail ? src[j] : 0;
        }
        store16(base + (int64_t)c * 512, b);
    }
}

// Generic formats: one thread per (row, k-tile), 256 f16 values (fewer in a
// ragged last tile), bit-exact with dequantize_to_f16.
template <int FMT>
__global__ void dequant_generic_kernel(const uint8_t* __restrict__ tiled, uint16_t* __restrict__ out, int64_t n,
                                       int64_t k, int64_t ktiles, int64_t tile_bytes) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n * ktiles) return;
    const int64_t r = idx / ktiles, t = idx - r * ktiles;
    const uint8_t* base = tiled + ((r / 32) * ktiles + t) * tile_bytes + (r % 32) * 16;
    uint32_t w[GenericFmt<FMT>::WORDS];
#pragma unroll
    for (int c = 0; c < GenericFmt<FMT>::CHUNKS; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(base + c * 512);
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
    }
    const int64_t c0 = t * 256, ncol = std::min<int64_t>(256, k - c0);
    uint16_t* o = out + r * k + c0;
    decode_slice<FMT, true>(w, [&](int e, float v) {
        if (e < ncol) o[e] = f32_to_f16_rtz(v);
    });
}

template <int FMT>
void launch_dequant_generic(const QLayout& L, const uint8_t* tiled, uint16_t* out, cudaStream_t s) {
    const int64_t total = L.n * L.ktiles();
    dequant_generic_kernel<FMT><<<blocks_for(total, 64), 64, 0, s>>>(tiled, out, L.n, L.k, L.ktiles(), L.tile_bytes);
    BC_LAUNCHED("dequant_generic_kernel");
}

}  // namespace

void launch_repack(const QLayout& L, const uint8_t* raw, int nibble_order, uint8_t* tiled,
                   const int64_t* row_map, cudaStream_t s) {
    const int64_t total = L.n_pad * L.ktiles();
    if (total == 0) return;
    if (!is_core_format(L.dtype)) {
        const int64_t row_bytes = L.k / block_size(L.dtype) * block_bytes(L.dtype);
        const int64_t slice = 256 / block_size(L.dtype) * block_bytes(L.dtype);
        repack_generic_kernel<<<blocks_for(total, 128), 128, 0, s>>>(raw, tiled, L.n, row_bytes, slice, L.n_pad,
                                                                     L.ktiles(), L.tile_bytes, L.chunks + 1, row_map);
        BC_LAUNCHED("repack_generic_kernel");
        return;
    }
    repack_kernel<<<blocks_for(total, 128), 128, 0, s>>>(
        raw, tiled, L.dtype, L.n, L.k, L.n_pad, L.ktiles(), L.tile_bytes, L.chunks,
        nibble_order == BEACON_CUDA_NIBBLE_GGUF_SPLIT ? 1 : 0, row_map);
    BC_LAUNCHED("repack_kernel");
}

void launch_dequant_f16(const QLayout& L, const uint8_t* tiled, uint16_t* out, cudaStream_t s) {
    if (L.n == 0) return;
    switch (L.dtype) {
        case BEACON_CUDA_DTYPE_Q4_1: return launch_dequant_generic<FMT_Q4_1>(L, tiled, out, s);
        case BEACON_CUDA_DTYPE_Q5_0: return launch_dequant_generic<FMT_Q5_0>(L, tiled, out, s);
        case BEACON_CUDA_DTYPE_Q5_1: return launch_dequant_generic<FMT_Q5_1>(L, tiled, out, s);
        case BEACON_CUDA_DTYPE_Q2_K: return launch_dequant_generic<FMT_Q2_K>(L, tiled, out, s);
        case BEACON_CUDA_DTYPE_Q3_K: return launch_dequant_generic<FMT_Q3_K>(L, tiled, out, s);
        case BEACON_CUDA_DTYPE_Q5_K: return launch_dequant_generic<FMT_Q5_K>(L, tiled, out, s);
        case BEACON_CUDA_DTYPE_Q6_K: return launch_dequant_generic<FMT_Q6_K>(L, tiled, out, s);
        case BEACON_CUDA_DTYPE_Q8_K: return launch_dequant_generic<FMT_Q8_K>(L, tiled, out, s);
        default: break;
    }
    const int64_t total = L.n * (L.k / 32);
    if (total == 0) return;
    dequant_f16_kernel<<<blocks_for(total, 128), 128, 0, s>>>(tiled, out, L.dtype, L.n, L.k,
                                                              L.ktiles(), L.tile_bytes);
    BC_LAUNCHED("dequant_f16_kernel");
}

void launch_quantize(int32_t dtype, const float* x, int64_t n_rows, int64_t k, int nibble_order,
                     uint8_t* raw, cudaStream_t s) {
    const int64_t bs = dtype == BEACON_CUDA_DTYPE_Q4_K ? 256 : 32;
    const int64_t nb = n_rows * k / bs;
    if (nb == 0) return;
    quantize_kernel<<<blocks_for(nb, 128), 128, 0, s>>>(
        x, raw, dtype, nb, nibble_order == BEACON_CUDA_NIBBLE_GGUF_SPLIT ? 1 : 0);
    BC_LAUNCHED("quantize_kernel");
}

}  // namespace bc
