// gemv.cuh -- fused GGUF dequant + GEMV (decode, batch 1-16) for sm_100a.
//
// Replaces the reference's quantized GEMV (q4_matmul_f32, ops.rs:62-70, and
// the row loop of q4_dot_f32, ops.rs:38-56) and serves
// ComputeBackend::quantized_matmul (backend.rs:32-41) for small batches.
//
// Design (HBM-bound, ~0.56 B of weight per multiply-add):
//  * weights in row-group tiles (QLayout): 32 rows x 256 columns; lane l of a
//    warp owns row l, so every warp-wide 128-bit load reads 512 contiguous
//    bytes and no cross-lane reduction is needed;
//  * the activation slice of the CTA is staged once in shared memory and read
//    as broadcasts (every lane of a warp reads the same address);
//  * FAST mode: activations quantized per 32 elements to int16, products
//    summed exactly with dp2a against the unsigned 4-bit / signed 8-bit codes,
//    block scales applied once per block in f32;
//    F32 mode: f32 activations times the reference's f32 weight value
//    (optionally truncated to f16 as the CPU engine's weights are);
//  * 4 warps split the CTA's tiles; optional split-K over CTAs with a
//    deterministic last-arriver reduction (fixed summation order).
#pragma once

#include "common.cuh"
#include "kernels.h"
#include "qx.cuh"

namespace bc {

enum { FMT_Q4_0 = 0, FMT_Q8_0 = 1, FMT_Q4_K = 2 };

}  // namespace bc
#include "gemv_generic.cuh"
namespace bc {

// 16-byte chunks per row per tile after the first (the meta chunk)
template <int FMT>
struct Fmt {
    static constexpr int CH = FMT == FMT_Q8_0 ? 16 : FMT <= FMT_Q4_K ? 8 : GenericFmt<FMT>::CHUNKS - 1;
};

struct GemvParams {
    const uint8_t* w;
    int64_t ktiles;
    int64_t tile_bytes;
    int64_t n;      // rows of W that hold data
    int64_t n_pad;  // rows of the tiled layout
    int tps;
    int ksplit;
    const void* x;
    int x_f16;
    int64_t x_ld;
    int64_t k;  // logical columns; staged elements beyond k are zero
    int batch;
    float* y;
    int64_t y_ld;
    const float* res;
    int64_t res_ld;
    float* partial;
    int* counters;
    int rtz;
    const float* norm_w;  // persistent kernel only: RMSNorm of each x row fused into the staging
    float norm_eps;
    QkvEpi qkv;           // EPI_QKV destinations
    QxImage qx;           // pre-quantised activations (persistent kernel, FAST)
    QxImage qy;           // EPI_ADD: y also written quantised for the next GEMV
};

__device__ __forceinline__ float load_x(const GemvParams& p, int b, int64_t kk) {
    if (b >= p.batch || kk >= p.k) return 0.0f;
    if (p.x_f16) return __half2float(reinterpret_cast<const __half*>(p.x)[b * p.x_ld + kk]);
    return reinterpret_cast<const float*>(p.x)[b * p.x_ld + kk];
}

// Small integer q (0 <= q < 2^22) to float with one OR and one FADD:
// 2^23 + q is exact in f32, subtract 2^23 + bias.
__device__ __forceinline__ float small_int_f32(uint32_t q, float magic_plus_bias) {
    return __fsub_rn(__uint_as_float(0x4B000000u | q), magic_plus_bias);
}

__device__ __forceinline__ float f16_round_trip_rtz(float v) {
    return __uint_as_float(f16_to_f32_bits(f32_to_f16_rtz(v)));
}

// Shared-memory staging -------------------------------------------------------
// F32 mode:  float xs[B][span]
// FAST mode: int16 xq[B][span] (Q4_0: each 8-element group stored as
//            e0 e2 e4 e6 e1 e3 e5 e7 to match the interleaved nibbles),
//            float2 [B][span/32] = (scale, sum of the block's int16 codes).
template <int FMT, int MODE, int B>
__device__ __forceinline__ void stage_x(const GemvParams& p, uint8_t* smem, int64_t k_base,
                                        int span) {
    if (MODE == MODE_F32) {
        float* xs = reinterpret_cast<float*>(smem);
        for (int i = threadIdx.x; i < B * span; i += blockDim.x) {
            int b = i / span, e = i - b * span;
            xs[i] = load_x(p, b, k_base + e);
        }
    } else {
        int16_t* xq = reinterpret_cast<int16_t*>(smem);
        const int nblk = span / 32;
        float2* sxq = reinterpret_cast<float2*>(smem + (size_t)B * span * 2);
        for (int i = threadIdx.x; i < B * nblk; i += blockDim.x) {
            int b = i / nblk, j = i - b * nblk;
            float v[32];
            float amax = 0.0f;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                v[e] = load_x(p, b, k_base + j * 32 + e);
                amax = fmaxf(amax, fabsf(v[e]));
            }
            float inv = amax > 0.0f ? __fdiv_rn(32767.0f, amax) : 0.0f;
            int qv[32];
            int sum = 0;
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                int q = __float2int_rn(__fmul_rn(v[e], inv));
                q = max(-32767, min(32767, q));
                qv[e] = q;
                sum += q;
            }
            uint32_t packed[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                int a0, a1;
                if (FMT == FMT_Q4_0) {
                    // slot s of an 8-group holds element (s<4 ? 2s : 2(s-4)+1)
                    int grp = e & ~7, s0 = e & 7, s1 = s0 + 1;
                    int e0 = grp + (s0 < 4 ? 2 * s0 : 2 * (s0 - 4) + 1);
                    int e1 = grp + (s1 < 4 ? 2 * s1 : 2 * (s1 - 4) + 1);
                    a0 = qv[e0];
                    a1 = qv[e1];
                } else {
                    a0 = qv[e];
                    a1 = qv[e + 1];
                }
                packed[e / 2] = (uint32_t)(a0 & 0xFFFF) | ((uint32_t)a1 << 16);
            }
            uint4* dst = reinterpret_cast<uint4*>(xq + (size_t)b * span + j * 32);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                dst[c] = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2],
                                    packed[4 * c + 3]);
            sxq[b * nblk + j] = make_float2(amax > 0.0f ? __fdiv_rn(amax, 32767.0f) : 0.0f, (float)sum);
        }
    }
}

// Tile consumers --------------------------------------------------------------

__device__ __forceinline__ float half_at(const uint4& m, int i) {
    uint32_t w = (&m.x)[i >> 1];
    uint16_t h = (uint16_t)((i & 1) ? (w >> 16) : (w & 0xFFFF));
    return f16_to_f32(h);
}

template <int B>
__device__ __forceinline__ void fma8(float (&acc)[B], const float (&w)[8], const float* xs, int span,
                                     int e0) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
        const float4* xp = reinterpret_cast<const float4*>(xs + (size_t)b * span + e0);
        float4 xa = xp[0], xb = xp[1];
        acc[b] = fmaf(w[0], xa.x, acc[b]);
        acc[b] = fmaf(w[1], xa.y, acc[b]);
        acc[b] = fmaf(w[2], xa.z, acc[b]);
        acc[b] = fmaf(w[3], xa.w, acc[b]);
        acc[b] = fmaf(w[4], xb.x, acc[b]);
        acc[b] = fmaf(w[5], xb.y, acc[b]);
        acc[b] = fmaf(w[6], xb.z, acc[b]);
        acc[b] = fmaf(w[7], xb.w, acc[b]);
    }
}

template <int B>
__device__ __forceinline__ void fma4(float (&acc)[B], const float (&w)[4], const float* xs, int span,
                                     int e0) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float4 xa = *reinterpret_cast<const float4*>(xs + (size_t)b * span + e0);
        acc[b] = fmaf(w[0], xa.x, acc[b]);
        acc[b] = fmaf(w[1], xa.y, acc[b]);
        acc[b] = fmaf(w[2], xa.z, acc[b]);
        acc[b] = fmaf(w[3], xa.w, acc[b]);
    }
}

// Q4_0: meta = 8 f16 block scales; chunk c = block c, byte i -> elements 2i, 2i+1.
template <int MODE, int B>
__device__ __forceinline__ void consume_q4_0(const uint4& meta, const uint4 (&q)[8], const uint8_t* smem,
                                             int span, int tile, float (&acc)[B], bool rtz) {
    if (MODE == MODE_F32) {
        const float* xs = reinterpret_cast<const float*>(smem);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float d = half_at(meta, c);
            const uint32_t* wq = &q[c].x;
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                float w[8];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t byte = (wq[wd] >> (8 * j)) & 0xFFu;
                    float lo = small_int_f32(byte & 0xFu, 8388616.0f);  // q - 8
                    float hi = small_int_f32(byte >> 4, 8388616.0f);
                    w[2 * j] = __fmul_rn(lo, d);
                    w[2 * j + 1] = __fmul_rn(hi, d);
                    if (rtz) {
                        w[2 * j] = f16_round_trip_rtz(w[2 * j]);
                        w[2 * j + 1] = f16_round_trip_rtz(w[2 * j + 1]);
                    }
                }
                fma8<B>(acc, w, xs, span, tile * 256 + c * 32 + wd * 8);
            }
        }
    } else {
        const int16_t* xq = reinterpret_cast<const int16_t*>(smem);
        const int nblk = span / 32;
        const float2* sxq = reinterpret_cast<const float2*>(smem + (size_t)B * span * 2);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float d = half_at(meta, c);
            const uint32_t* wq = &q[c].x;
            uint32_t lo[4], hi[4];  // high nibbles in place (16 x value), see consume_q4_k
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                lo[wd] = wq[wd] & 0x0F0F0F0Fu;
                hi[wd] = wq[wd] & 0xF0F0F0F0u;
            }
            const int blk = tile * 8 + c;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)b * span + blk * 32);
                int al = 0, ah = 0;
#pragma unroll
                for (int wd = 0; wd < 4; ++wd) {
                    int4 X = xp[wd];
                    al = dp2a_lo_u8(X.x, lo[wd], al);
                    ah = dp2a_lo_u8(X.z, hi[wd], ah);
                    al = dp2a_hi_u8(X.y, lo[wd], al);
                    ah = dp2a_hi_u8(X.w, hi[wd], ah);
                }
                const int ai = al + (ah >> 4);
                const int bi = b * nblk + blk;
                const float2 xb = sxq[bi];
                acc[b] = fmaf(d * xb.x, fmaf(-8.0f, xb.y, (float)ai), acc[b]);
            }
        }
    }
}

// Q8_0: meta = 8 f16 block scales; chunks 2c, 2c+1 = the 32 int8 codes of block c.
template <int MODE, int B>
__device__ __forceinline__ void consume_q8_0(const uint4& meta, const uint4 (&q)[16], const uint8_t* smem,
                                             int span, int tile, float (&acc)[B], bool rtz) {
    if (MODE == MODE_F32) {
        const float* xs = reinterpret_cast<const float*>(smem);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            const float d = half_at(meta, c >> 1);
            const uint32_t* wq = &q[c].x;
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                float w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t u = ((wq[wd] >> (8 * j)) & 0xFFu) ^ 0x80u;  // int8 + 128
                    w[j] = __fmul_rn(small_int_f32(u, 8388736.0f), d);
                    if (rtz) w[j] = f16_round_trip_rtz(w[j]);
                }
                fma4<B>(acc, w, xs, span, tile * 256 + c * 16 + wd * 4);
            }
        }
    } else {
        const int16_t* xq = reinterpret_cast<const int16_t*>(smem);
        const int nblk = span / 32;
        const float2* sxq = reinterpret_cast<const float2*>(smem + (size_t)B * span * 2);
#pragma unroll
        for (int bl = 0; bl < 8; ++bl) {
            const float d = half_at(meta, bl);
            const int blk = tile * 8 + bl;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const int4* xp = reinterpret_cast<const int4*>(xq + (size_t)b * span + blk * 32);
                int a2[2] = {0, 0};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint32_t* wq = &q[2 * bl + h].x;
                    int4 X = xp[2 * h], Y = xp[2 * h + 1];
                    a2[h] = dp2a_lo_s8(X.x, wq[0], a2[h]);
                    a2[h] = dp2a_hi_s8(X.y, wq[0], a2[h]);
                    a2[h] = dp2a_lo_s8(X.z, wq[1], a2[h]);
                    a2[h] = dp2a_hi_s8(X.w, wq[1], a2[h]);
                    a2[h] = dp2a_lo_s8(Y.x, wq[2], a2[h]);
                    a2[h] = dp2a_hi_s8(Y.y, wq[2], a2[h]);
                    a2[h] = dp2a_lo_s8(Y.z, wq[3], a2[h]);
                    a2[h] = dp2a_hi_s8(Y.w, wq[3], a2[h]);
                }
                const int ai = a2[0] + a2[1];
                acc[b] = fmaf(d * sxq[b * nblk + blk].x, (float)ai, acc[b]);
            }
        }
    }
}

// decode_k_scales_mins (dequant.rs:289-307) from the 12 packed bytes in
// meta words 1..3.
__device__ __forceinline__ void k_scales(const uint4& meta, int (&sc)[8], int (&mn)[8]) {
    uint8_t q[12];
#pragma unroll
    for (int i = 0; i < 12; ++i) q[i] = (uint8_t)((&meta.y)[i >> 2] >> (8 * (i & 3)));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        sc[j] = q[j] & 0x3F;
        mn[j] = q[j + 4] & 0x3F;
    }
#pragma unroll
    for (int j = 4; j < 8; ++j) {
        sc[j] = (q[j + 4] & 0x0F) | ((q[j - 4] >> 6) << 4);
        mn[j] = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Q4_K: meta = [d, dmin, 12 scale bytes]; chunk c: pair p = c/2, half h = c%2,
// byte i -> element 64p+16h+i (low nibble, sub-block 2p) and
// 64p+32+16h+i (high nibble, sub-block 2p+1).
template <int MODE, int B>
__device__ __forceinline__ void consume_q4_k(const uint4& meta, const uint4 (&q)[8], const uint8_t* smem,
                                             int span, int tile, float (&acc)[B], bool rtz) {
    const float d = f16_to_f32((uint16_t)(meta.x & 0xFFFF));
    const float dmin = f16_to_f32((uint16_t)(meta.x >> 16));
    int sc[8], mn[8];
    k_scales(meta, sc, mn);
    if (MODE == MODE_F32) {
        const float* xs = reinterpret_cast<const float*>(smem);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const int pr = c >> 1, h = c & 1;
            const float sl = __fmul_rn((float)sc[2 * pr], d), ml = __fmul_rn((float)mn[2 * pr], dmin);
            const float sh = __fmul_rn((float)sc[2 * pr + 1], d),
                        mh = __fmul_rn((float)mn[2 * pr + 1], dmin);
            const uint32_t* wq = &q[c].x;
#pragma unroll
            for (int wd = 0; wd < 4; ++wd) {
                float wl[4], wh[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t byte = (wq[wd] >> (8 * j)) & 0xFFu;
                    wl[j] = __fsub_rn(__fmul_rn(small_int_f32(byte & 0xFu, 8388608.0f), sl), ml);
                    wh[j] = __fsub_rn(__fmul_rn(small_int_f32(byte >> 4, 8388608.0f), sh), mh);
                    if (rtz) {
                        wl[j] = f16_round_trip_rtz(wl[j]);
                        wh[j] = f16_round_trip_rtz(wh[j]);
                    }
                }
                fma4<B>(acc, wl, xs, span, tile * 256 + 64 * pr + 16 * h + 4 * wd);
                fma4<B>(acc, wh, xs, span, tile * 256 + 64 * pr + 32 + 16 * h + 4 * wd);
            }
        }
    } else {
        const int16_t* xq = reinterpret_cast<const int16_t*>(smem);
        const int nblk = span / 32;
        const float2* sxq = reinterpret_cast<const float2*>(smem + (size_t)B * span * 2);
        // the eight 6-bit scales and mins as bytes of four words; byte k of a
        // word becomes a float through 2^23 + byte (one byte permute) - 2^23
        const uint32_t w0 = meta.y, w1 = meta.z, w2 = meta.w;
        const uint32_t s03 = w0 & 0x3F3F3F3Fu, m03 = w1 & 0x3F3F3F3Fu;
        const uint32_t s47 = (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u);
        const uint32_t m47 = ((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u);
        auto byte_f32 = [](uint32_t w, int k) {
            return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)k)) - 8388608.0f;
        };
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            // low nibbles as bytes; high nibbles kept in place (16 x value): the
            // integer sums below are exact, so >> 4 recovers the true sum
            uint32_t lo[2][4], hi[2][4];
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int wd = 0; wd < 4; ++wd) {
                    uint32_t w = (&q[2 * pr + h].x)[wd];
                    lo[h][wd] = w & 0x0F0F0F0Fu;
                    hi[h][wd] = w & 0xF0F0F0F0u;
                }
            const uint32_t sw = pr < 2 ? s03 : s47, mw = pr < 2 ? m03 : m47;
            const int k0 = (2 * pr) & 3;
            const float dl = d * byte_f32(sw, k0), dh = d * byte_f32(sw, k0 + 1);
            const float ml = dmin * byte_f32(mw, k0), mh = dmin * byte_f32(mw, k0 + 1);
            const int jl = tile * 8 + 2 * pr, jh = jl + 1;
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const int4* xl = reinterpret_cast<const int4*>(xq + (size_t)b * span + jl * 32);
                const int4* xh = reinterpret_cast<const int4*>(xq + (size_t)b * span + jh * 32);
                int al[2] = {0, 0}, ah[2] = {0, 0};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    int4 L0 = xl[2 * h], L1 = xl[2 * h + 1];
                    int4 H0 = xh[2 * h], H1 = xh[2 * h + 1];
                    al[h] = dp2a_lo_u8(L0.x, lo[h][0], al[h]);
                    ah[h] = dp2a_lo_u8(H0.x, hi[h][0], ah[h]);
                    al[h] = dp2a_hi_u8(L0.y, lo[h][0], al[h]);
                    ah[h] = dp2a_hi_u8(H0.y, hi[h][0], ah[h]);
                    al[h] = dp2a_lo_u8(L0.z, lo[h][1], al[h]);
                    ah[h] = dp2a_lo_u8(H0.z, hi[h][1], ah[h]);
                    al[h] = dp2a_hi_u8(L0.w, lo[h][1], al[h]);
                    ah[h] = dp2a_hi_u8(H0.w, hi[h][1], ah[h]);
                    al[h] = dp2a_lo_u8(L1.x, lo[h][2], al[h]);
                    ah[h] = dp2a_lo_u8(H1.x, hi[h][2], ah[h]);
                    al[h] = dp2a_hi_u8(L1.y, lo[h][2], al[h]);
                    ah[h] = dp2a_hi_u8(H1.y, hi[h][2], ah[h]);
                    al[h] = dp2a_lo_u8(L1.z, lo[h][3], al[h]);
                    ah[h] = dp2a_lo_u8(H1.z, hi[h][3], ah[h]);
                    al[h] = dp2a_hi_u8(L1.w, lo[h][3], al[h]);
                    ah[h] = dp2a_hi_u8(H1.w, hi[h][3], ah[h]);
                }
                const float sl = (float)(al[0] + al[1]), sh = (float)((ah[0] + ah[1]) >> 4);
                const float2 pl = sxq[b * nblk + jl], ph = sxq[b * nblk + jh];
                acc[b] = fmaf(pl.x, fmaf(dl, sl, -ml * pl.y), acc[b]);
                acc[b] = fmaf(ph.x, fmaf(dh, sh, -mh * ph.y), acc[b]);
            }
        }
    }
}

// Generic formats (gemv_generic.cuh): the row slice (meta chunk + CH chunks)
// decoded from registers to the reference's f32 weights (f16-truncated for
// the CPU-reproducing numerics) against f32 activations staged in shared
// memory.
template <int FMT, int B>
__device__ __forceinline__ void consume_generic(const uint4& meta, const uint4* q, const uint8_t* smem, int span,
                                                int tile, float (&acc)[B], bool rtz) {
    uint32_t w[GenericFmt<FMT>::WORDS];
    w[0] = meta.x;
    w[1] = meta.y;
    w[2] = meta.z;
    w[3] = meta.w;
#pragma unroll
    for (int c = 0; c < GenericFmt<FMT>::CHUNKS - 1; ++c) {
        w[4 + 4 * c] = q[c].x;
        w[5 + 4 * c] = q[c].y;
        w[6 + 4 * c] = q[c].z;
        w[7 + 4 * c] = q[c].w;
    }
    const float* xs = reinterpret_cast<const float*>(smem) + tile * 256;
    decode_slice<FMT, false>(w, [&](int e, float v) {
        if (rtz) v = f16_round_trip_rtz(v);
#pragma unroll
        for (int b = 0; b < B; ++b) acc[b] = fmaf(v, xs[(size_t)b * span + e], acc[b]);
    });
}

// Epilogue --------------------------------------------------------------------
// The SwiGLU outputs of row groups 2j and 2j+1 form the 32-element block j of
// the next GEMV's input: the second of the two groups to finish (an
// acquire/release arrival counter per pair) reads both halves back and writes
// the block into the consumer's staging image. Whole warp.
template <int B>
__device__ __forceinline__ void swiglu_handoff(const GemvParams& p, int64_t g, int lane) {
    const int64_t j = g >> 1;
    int second = 1;  // a last group without a partner writes its block alone
    if ((g | 1) < p.n_pad / 32) {
        __syncwarp();
        if (lane == 0) second = atomic_add_acq_rel_gpu(&p.qy.pairs[j], 1) == 1;
        second = __shfl_sync(0xffffffffu, second, 0);
        if (!second) return;
        if (lane == 0) p.qy.pairs[j] = 0;
    }
    const int64_t fe = j * 32 + lane;
    const bool valid = 2 * fe < p.n;
#pragma unroll
    for (int b = 0; b < B; ++b) {
        if (b >= p.batch) break;
        const float x = valid ? __ldcg(&p.y[b * p.y_ld + fe]) : 0.0f;
        qx_write_group(p.qy, b, j, lane, x, valid);
    }
}

// Epilogue operands of one row group loaded ahead of its finish (lane = row):
// the residual rows and the next GEMV's norm weight.
template <int B>
struct EpiPre {
    int g = -1;      // the group they belong to; -1: none
    float res[B];
    float nw;
};

template <int B>
__device__ __forceinline__ void gemv_store(const GemvParams& p, int epi, int64_t g, int lane,
                                           const float (&v)[B], const EpiPre<B>* pre = nullptr) {
    const int64_t row = g * 32 + lane;
    const bool have = pre && (int64_t)pre->g == g;
    if (epi == EPI_QKV) {
        // the whole warp takes part: pairs (2i, 2i+1) are lanes (l, l ^ 1)
        const QkvEpi& e = p.qkv;
        const int r = (int)row, half = e.d / 2;
        const int pos0 = e.pos_ptr ? *e.pos_ptr : e.pos_imm;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float x = v[b];
            const float partner = __shfl_xor_sync(0xffffffffu, x, 1);
            if (b >= p.batch || row >= p.n) continue;
            const int rr = e.row0 + b;
            const int pos = pos0 + rr * e.pos_step;
            if (pos < 0 || pos >= e.max_ctx) {  // a device-advanced position ran past the cache
                atomicExch(e.err, kErrContext);
                continue;
            }
            const int64_t cache_at = (int64_t)rr * e.seq_step * e.cache_sb + (int64_t)pos * e.kd;
            if (r < e.qd + e.kd) {
                const int ee = r < e.qd ? r : r - e.qd;
                const int i = (ee % e.d) / 2;
                const float c = e.cs[(int64_t)pos * half + i], s = e.sn[(int64_t)pos * half + i];
                const bool odd = (r & 1) != 0;
                const float x0 = odd ? partner : x, x1 = odd ? x : partner;
                const float o = odd ? x0 * s + x1 * c : x0 * c - x1 * s;
                if (r < e.qd)
                    e.q[(int64_t)rr * e.qd + ee] = o;
                else if (e.kv_f16)
                    static_cast<__half*>(e.kc)[cache_at + ee] = __float2half(o);
                else
                    static_cast<float*>(e.kc)[cache_at + ee] = o;
            } else {
                const int ee = r - e.qd - e.kd;
                if (e.kv_f16)
                    static_cast<__half*>(e.vc)[cache_at + ee] = __float2half(x);
                else
                    static_cast<float*>(e.vc)[cache_at + ee] = x;
            }
        }
        return;
    }
    if (epi == EPI_SWIGLU) {
        // lanes 0..15: gate rows, lanes 16..31: the matching up rows
        const int64_t f = g * 16 + lane;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            float up = __shfl_down_sync(0xffffffffu, v[b], 16);
            if (lane < 16 && b < p.batch && 2 * f < p.n) {
                float gte = v[b];
                float sig = 1.0f / (1.0f + expf(-gte));
                p.y[b * p.y_ld + f] = (gte * sig) * up;
            }
        }
        if (p.qy.data) swiglu_handoff<B>(p, g, lane);
        return;
    }
    if (epi == EPI_ADD && p.qy.data) {
        // also hand the next GEMV its quantised input (whole warp: shuffles)
#pragma unroll
        for (int b = 0; b < B; ++b) {
            if (b >= p.batch) break;
            const bool ok = row < p.n;
            float r = 0.0f;
            if (ok) {
                r = (have ? pre->res[b] : p.res[b * p.res_ld + row]) + v[b];
                p.y[b * p.y_ld + row] = r;
            }
            qx_write_group(p.qy, b, g, lane, r, ok, have, have ? pre->nw : 0.0f);
        }
        return;
    }
    if (row >= p.n) return;
#pragma unroll
    for (int b = 0; b < B; ++b) {
        if (b >= p.batch) break;
        float r = v[b];
        if (epi == EPI_ADD) r = (have ? pre->res[b] : p.res[b * p.res_ld + row]) + r;
        p.y[b * p.y_ld + row] = r;
    }
}

template <int FMT, int MODE, int B>
__global__ void __launch_bounds__(128) qgemv_kernel(const GemvParams p, const int epi) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float red[4][B][32];
    constexpr int CH = Fmt<FMT>::CH;
    const int64_t g = blockIdx.x / p.ksplit;
    const int s = blockIdx.x - (int)(g * p.ksplit);
    const int t0 = s * p.tps;
    const int t1 = (int)min((int64_t)p.ktiles, (int64_t)t0 + p.tps);
    const int nt = t1 - t0;
    const int span = nt * 256;
    pdl_trigger();
    pdl_wait();
    stage_x<FMT, MODE, B>(p, smem, (int64_t)t0 * 256, span);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.0f;
    const uint8_t* gbase = p.w + (g * p.ktiles + t0) * p.tile_bytes;
    const bool rtz = p.rtz != 0;
    for (int t = warp; t < nt; t += 4) {
        const uint8_t* tp = gbase + (int64_t)t * p.tile_bytes;
        const uint4 meta = ldg_stream(reinterpret_cast<const uint4*>(tp) + lane);
        uint4 q[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) q[c] = ldg_stream(reinterpret_cast<const uint4*>(tp + 512 + c * 512) + lane);
        if constexpr (FMT == FMT_Q4_0)
            consume_q4_0<MODE, B>(meta, *reinterpret_cast<uint4(*)[8]>(q), smem, span, t, acc, rtz);
        else if constexpr (FMT == FMT_Q8_0)
            consume_q8_0<MODE, B>(meta, *reinterpret_cast<uint4(*)[16]>(q), smem, span, t, acc, rtz);
        else if constexpr (FMT == FMT_Q4_K)
            consume_q4_k<MODE, B>(meta, *reinterpret_cast<uint4(*)[8]>(q), smem, span, t, acc, rtz);
        else
            consume_generic<FMT, B>(meta, q, smem, span, t, acc, rtz);
    }
#pragma unroll
    for (int b = 0; b < B; ++b) red[warp][b][lane] = acc[b];
    __syncthreads();
    if (warp != 0) return;
    float v[B];
#pragma unroll
    for (int b = 0; b < B; ++b) v[b] = ((red[0][b][lane] + red[1][b][lane]) + red[2][b][lane]) + red[3][b][lane];
    if (p.ksplit == 1) {
        gemv_store<B>(p, epi, g, lane, v);
        return;
    }
    // split-K: publish the partial, the last CTA of the row group reduces the
    // partials in split order and runs the epilogue.
    const int64_t row = g * 32 + lane;
#pragma unroll
    for (int b = 0; b < B; ++b)
        if (b < p.batch) p.partial[((int64_t)s * p.batch + b) * p.n_pad + row] = v[b];
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&p.counters[g], 1) == p.ksplit - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
#pragma unroll
    for (int b = 0; b < B; ++b) {
        float sum = 0.0f;
        if (b < p.batch)
            for (int s2 = 0; s2 < p.ksplit; ++s2)
                sum += __ldcg(&p.partial[((int64_t)s2 * p.batch + b) * p.n_pad + row]);
        v[b] = sum;
    }
    gemv_store<B>(p, epi, g, lane, v);
    if (lane == 0) p.counters[g] = 0;
}

inline size_t gemv_smem_bytes(int mode, int bpad, int span) {
    if (mode == MODE_F32) return (size_t)bpad * span * 4;
    return (size_t)bpad * span * 2 + (size_t)bpad * (span / 32) * 8;
}

template <int FMT, int MODE, int B>
void launch_qgemv_t(const GemvLaunch& a) {
    const GemvPlan& pl = *a.plan;
    GemvParams p;
    p.w = static_cast<const uint8_t*>(a.w);
    p.ktiles = a.L->ktiles();
    p.tile_bytes = a.L->tile_bytes;
    p.n = a.L->n;
    p.n_pad = a.L->n_pad;
    p.tps = pl.tps;
    p.ksplit = pl.ksplit;
    p.x = a.x;
    p.x_f16 = a.x_f16 ? 1 : 0;
    p.x_ld = a.x_ld;
    p.k = a.L->k;
    p.batch = a.batch;
    p.y = a.y;
    p.y_ld = a.y_ld;
    p.res = a.res;
    p.res_ld = a.res_ld;
    p.partial = a.scratch.partial;
    p.counters = a.scratch.counters;
    p.rtz = a.rtz ? 1 : 0;
    p.norm_w = nullptr;
    p.norm_eps = 0.0f;
    p.qkv = a.qkv ? *a.qkv : QkvEpi{};
    p.qx = QxImage{};  // the tiled kernel stages its own activations
    p.qy = a.qy;
    auto kern = qgemv_kernel<FMT, MODE, B>;
    if (pl.smem > 48 * 1024) allow_max_dynamic_smem(kern);
    const int64_t grid = a.L->groups() * pl.ksplit;
    launch_kernel(kern, dim3((unsigned)grid), dim3(128), pl.smem, a.s, a.pdl, p, a.epi);
}

template <int FMT>
void launch_qgemv_fmt(const GemvLaunch& a) {
    const int bp = a.plan->bpad;
    // the generic formats always compute in f32 (their slices decode to the
    // reference's f32 values; there is no integer fast path for them)
    if constexpr (FMT <= FMT_Q4_K) {
        if (a.mode == MODE_FAST) {
            switch (bp) {
                case 1: return launch_qgemv_t<FMT, MODE_FAST, 1>(a);
                case 2: return launch_qgemv_t<FMT, MODE_FAST, 2>(a);
                case 4: return launch_qgemv_t<FMT, MODE_FAST, 4>(a);
                case 8: return launch_qgemv_t<FMT, MODE_FAST, 8>(a);
                default: return launch_qgemv_t<FMT, MODE_FAST, 16>(a);
            }
        }
    }
    switch (bp) {
        case 1: return launch_qgemv_t<FMT, MODE_F32, 1>(a);
        case 2: return launch_qgemv_t<FMT, MODE_F32, 2>(a);
        case 4: return launch_qgemv_t<FMT, MODE_F32, 4>(a);
        case 8: return launch_qgemv_t<FMT, MODE_F32, 8>(a);
        default: return launch_qgemv_t<FMT, MODE_F32, 16>(a);
    }
}

}  // namespace bc
