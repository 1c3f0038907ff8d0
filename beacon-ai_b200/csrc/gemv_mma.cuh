// gemv_mma.cuh -- tensor-core consumer of the persistent dequant-GEMV's weight
// tiles in the fast numerics: integer mma.sync m16n8k32 (8-bit operands, s32
// accumulation) instead of per-lane dp2a dot products.
//
// The integer sums are the same exact sums the dp2a consumer forms
// (sum over a 32-element block of code(weight) * code(activation), with the
// int16 activation code split into a signed high byte and an unsigned low
// byte: code = 256 * hi + lo, one MMA each); the f32 block scaling that
// follows uses the same expressions. Only the order in which the per-block
// f32 terms of a row are added differs.
//
// Operands, per warp and 32-row x 256-column tile (lane = (g, t), g = lane/4,
// t = lane%4; M halves mh = rows 16mh..16mh+15):
//  * A (16 rows x 32 k, 8-bit): one ldmatrix.x4 of the tile's chunk pair
//    (2q, 2q+1) gives each thread word t (bytes 4t..4t+3) of rows g and g+8
//    of both chunks -- exactly an A fragment's k = 4t..4t+3 and 16+4t..+3.
//      Q4_K: chunk pair q holds qs bytes 32q..32q+31 of each row; the low
//            nibbles are sub-block 2q, the high nibbles (kept in place, x16)
//            sub-block 2q+1, both in natural element order.
//      Q4_0: chunks are blocks; byte i holds elements 2i (low nibble) and
//            2i+1 (high). The MMA's k order is: k = 4t+i <-> element 8t+2i,
//            k = 16+4t+i <-> element 8t+2i+1, which is the order in which
//            the activation image already stores each 8-group for Q4_0
//            (e0 e2 e4 e6 e1 e3 e5 e7).
//      Q8_0: chunks 2j and 2j+1 are block j's 32 signed codes.
//  * B (32 k x 8 columns, 8-bit): column n = g of thread (g, t). The eight
//    columns are NB batch rows times SB = 8 / NB blocks: column n is batch
//    n % NB of block-in-set n / NB. Block j belongs to set j / SB; a column is
//    nonzero only for the block it stands for, so one set's SB MMAs fill the
//    8 columns of one accumulator with SB blocks x NB rows of sums, and the
//    f32 scaling runs once per set instead of once per block (batch 1: once
//    per tile).
#pragma once

#include "gemv.cuh"

namespace bc {

// D = A * B + C with 8-bit A (16x32, row) and B (32x8, col), s32 C/D.
template <bool A_S8, bool B_S8>
__device__ __forceinline__ void mma_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                        const int (&c)[4]) {
#define BC_MMA_K32(AT, BT)                                                                                       \
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." AT "." BT ".s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, " \
                 "{%10,%11,%12,%13};"                                                                            \
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])                                                \
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c[0]), "r"(c[1]), "r"(c[2]), \
                   "r"(c[3]))
    if (A_S8 && B_S8)
        BC_MMA_K32("s8", "s8");
    else if (A_S8)
        BC_MMA_K32("s8", "u8");
    else if (B_S8)
        BC_MMA_K32("u8", "s8");
    else
        BC_MMA_K32("u8", "u8");
#undef BC_MMA_K32
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

// Words t of rows (16mh+g, 16mh+g+8) of chunks 2q and 2q+1 of the tile at tp:
// r[0] = (2q, g), r[1] = (2q, g+8), r[2] = (2q+1, g), r[3] = (2q+1, g+8).
__device__ __forceinline__ void ldsm_chunk_pair(uint32_t (&r)[4], const uint8_t* tp, int q, int mh, int lane) {
    const int m = lane >> 3, rr = lane & 7;
    ldsm_x4(r, smem_u32(tp + 512 + (2 * q + (m >> 1)) * 512 + (16 * mh + 8 * (m & 1) + rr) * 16));
}

// Per-warp scratch (floats): the tile's block scales, row-major by row.
//   Q4_K: [32 rows][8 sub-blocks] float2 (d*sc, dmin*m), d*sc already
//         divided by 16 for the odd (high-nibble) sub-blocks;
//   Q4_0 / Q8_0: [32 rows][8 blocks] float d.
// At the end of a row group it holds the accumulators for the transpose to
// one row per lane ([32 rows][B] floats).
template <int FMT, int B>
__host__ __device__ constexpr int mma_scratch_floats() {
    return (FMT == FMT_Q4_K ? 512 : 256) > 32 * B ? (FMT == FMT_Q4_K ? 512 : 256) : 32 * B;
}

// Lane r writes row r's scales of the tile at tp into the scratch.
template <int FMT>
__device__ __forceinline__ void mma_scales(const uint8_t* tp, int lane, float* scr) {
    const uint4 meta = *reinterpret_cast<const uint4*>(tp + lane * 16);
    if (FMT == FMT_Q4_K) {
        const float d = f16_to_f32((uint16_t)(meta.x & 0xFFFF));
        const float dmin = f16_to_f32((uint16_t)(meta.x >> 16));
        const uint32_t w0 = meta.y, w1 = meta.z, w2 = meta.w;
        const uint32_t s03 = w0 & 0x3F3F3F3Fu, m03 = w1 & 0x3F3F3F3Fu;
        const uint32_t s47 = (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u);
        const uint32_t m47 = ((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u);
        auto byte_f32 = [](uint32_t w, int k) {
            return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)k)) - 8388608.0f;
        };
        float4* out = reinterpret_cast<float4*>(scr + lane * 16);
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            const uint32_t sw = pr < 2 ? s03 : s47, mw = pr < 2 ? m03 : m47;
            const int k0 = (2 * pr) & 3;
            out[pr] = make_float4(d * byte_f32(sw, k0), dmin * byte_f32(mw, k0),
                                  (d * byte_f32(sw, k0 + 1)) * 0.0625f, dmin * byte_f32(mw, k0 + 1));
        }
    } else {
        float4* out = reinterpret_cast<float4*>(scr + lane * 8);
        out[0] = make_float4(half_at(meta, 0), half_at(meta, 1), half_at(meta, 2), half_at(meta, 3));
        out[1] = make_float4(half_at(meta, 4), half_at(meta, 5), half_at(meta, 6), half_at(meta, 7));
    }
}

// The A fragments of a tile: Q4 formats keep the raw words of all four
// chunk pairs and both halves (32 registers) so the ring slot can be refilled
// before the MMAs run; Q8_0 reads its fragments from the slot while it runs.
template <int FMT>
struct MmaTileRegs {
    uint32_t w[FMT == FMT_Q8_0 ? 1 : 4][2][4];  // [chunk pair][mh][ldmatrix word]
};

template <int FMT>
__device__ __forceinline__ void mma_load_tile(const uint8_t* tp, int lane, MmaTileRegs<FMT>& r) {
    if constexpr (FMT != FMT_Q8_0) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int mh = 0; mh < 2; ++mh) ldsm_chunk_pair(r.w[q][mh], tp, q, mh, lane);
    }
}

// A fragment of block j (0..7), half mh.
template <int FMT>
__device__ __forceinline__ void mma_a_frag(uint32_t (&a)[4], const MmaTileRegs<FMT>& r, const uint8_t* tp, int j,
                                           int mh, int lane) {
    constexpr uint32_t LO = 0x0F0F0F0Fu, HI = 0xF0F0F0F0u;
    if (FMT == FMT_Q4_K) {
        const uint32_t(&w)[4] = r.w[j >> 1][mh];
        const uint32_t m = (j & 1) ? HI : LO;
        a[0] = w[0] & m;
        a[1] = w[1] & m;
        a[2] = w[2] & m;
        a[3] = w[3] & m;
    } else if (FMT == FMT_Q4_0) {
        const uint32_t(&w)[4] = r.w[j >> 1][mh];
        const uint32_t w0 = (j & 1) ? w[2] : w[0], w1 = (j & 1) ? w[3] : w[1];
        a[0] = w0 & LO;
        a[1] = w1 & LO;
        a[2] = (w0 >> 4) & LO;
        a[3] = (w1 >> 4) & LO;
    } else {
        ldsm_chunk_pair(a, tp, j, mh, lane);
    }
}

// Accumulators of one thread: rows {g, g+8, 16+g, 24+g} x the two columns
// 2t, 2t+1 it holds in every set.
struct MmaAcc {
    float v[4][2];
};

// Consume one tile. xs: the staged activation image (int16 codes of B rows
// xstride apart, then (scale, code sum) float2 [B][kspan/32]); tile: the
// k-tile index.
template <int FMT, int B>
__device__ __forceinline__ void mma_consume_tile(const MmaTileRegs<FMT>& r, const uint8_t* tp, const uint8_t* xs,
                                                 int kspan, int xstride, int tile, const float* scr, MmaAcc& acc,
                                                 int lane) {
    static_assert(B == 1 || B == 2 || B == 4 || B == 8, "batch rows per MMA column set");
    constexpr int NB = B, SB = 8 / B;
    constexpr bool AS = FMT == FMT_Q8_0;
    const int g = lane >> 2, t = lane & 3;
    const int jj_g = g / NB, b_g = g % NB;  // the block-in-set and batch row this thread's column stands for
    const int16_t* xq = reinterpret_cast<const int16_t*>(xs);
    const int nblk = kspan / 32;
    const float2* sx = reinterpret_cast<const float2*>(xs + (size_t)B * xstride * 2);
    const int zero[4] = {0, 0, 0, 0};
#pragma unroll
    for (int s = 0; s < NB; ++s) {
        // activation codes of this thread's block of the set, split into bytes
        const int blk_g = tile * 8 + s * SB + jj_g;
        const int16_t* src = xq + (size_t)b_g * xstride + blk_g * 32;
        uint32_t h0, h1, l0, l1;
        if (FMT == FMT_Q4_0) {
            const uint4 v = *reinterpret_cast<const uint4*>(src + 8 * t);
            h0 = __byte_perm(v.x, v.y, 0x7531u);
            l0 = __byte_perm(v.x, v.y, 0x6420u);
            h1 = __byte_perm(v.z, v.w, 0x7531u);
            l1 = __byte_perm(v.z, v.w, 0x6420u);
        } else {
            const uint2 u = *reinterpret_cast<const uint2*>(src + 4 * t);
            const uint2 w = *reinterpret_cast<const uint2*>(src + 16 + 4 * t);
            h0 = __byte_perm(u.x, u.y, 0x7531u);
            l0 = __byte_perm(u.x, u.y, 0x6420u);
            h1 = __byte_perm(w.x, w.y, 0x7531u);
            l1 = __byte_perm(w.x, w.y, 0x6420u);
        }
        int dh[2][4], dl[2][4];
#pragma unroll
        for (int jj = 0; jj < SB; ++jj) {
            const int j = s * SB + jj;
            const bool on = SB == 1 || jj == jj_g;
            const uint32_t bh0 = on ? h0 : 0u, bh1 = on ? h1 : 0u, bl0 = on ? l0 : 0u, bl1 = on ? l1 : 0u;
#pragma unroll
            for (int mh = 0; mh < 2; ++mh) {
                uint32_t a[4];
                mma_a_frag<FMT>(a, r, tp, j, mh, lane);
                if (jj == 0) {  // the set's first block starts its accumulators
                    mma_k32<AS, true>(dh[mh], a, bh0, bh1, zero);
                    mma_k32<AS, false>(dl[mh], a, bl0, bl1, zero);
                } else {
                    mma_k32<AS, true>(dh[mh], a, bh0, bh1, dh[mh]);
                    mma_k32<AS, false>(dl[mh], a, bl0, bl1, dl[mh]);
                }
            }
        }
        // f32 scaling of the set: column n = 2t + c is batch n % NB of block s*SB + n / NB
#pragma unroll
        for (int mh = 0; mh < 2; ++mh)
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int row = 16 * mh + g + 8 * (c >> 1);
                const int n = 2 * t + (c & 1);
                const int j = s * SB + n / NB, b = n % NB;
                const float f = (float)(dh[mh][c] * 256 + dl[mh][c]);
                const float2 xp = sx[b * nblk + tile * 8 + j];
                float& o = acc.v[2 * mh + (c >> 1)][c & 1];
                if (FMT == FMT_Q4_K) {
                    const float2 sc = reinterpret_cast<const float2*>(scr)[row * 8 + j];
                    o = fmaf(xp.x, fmaf(sc.x, f, -sc.y * xp.y), o);
                } else if (FMT == FMT_Q4_0) {
                    o = fmaf(scr[row * 8 + j] * xp.x, fmaf(-8.0f, xp.y, f), o);
                } else {
                    o = fmaf(scr[row * 8 + j] * xp.x, f, o);
                }
            }
    }
}

// End of a row group: the thread accumulators -> one row per lane (lane =
// row), through the scratch; the accumulators are reset. Whole warp.
template <int B>
__device__ __forceinline__ void mma_rows_to_lanes(MmaAcc& acc, float* scr, float (&out)[B], int lane) {
    const int g = lane >> 2, t = lane & 3;
    __syncwarp();  // the tile's scales have been read
#pragma unroll
    for (int rs = 0; rs < 4; ++rs) {
        const int row = g + 8 * rs;  // rs = 2 mh + h: rows g, g+8, 16+g, 24+g
        float v0 = acc.v[rs][0], v1 = acc.v[rs][1];
        if (B == 1) {
            v0 += v1;
            v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
            v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
            if (t == 0) scr[row] = v0;
        } else if (B == 2) {  // column c = batch c; the four t hold four blocks each
            v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
            v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
            if (t == 0) {
                scr[row * 2] = v0;
                scr[row * 2 + 1] = v1;
            }
        } else if (B == 4) {  // batch 2 (t & 1) + c; t and t ^ 2 hold different blocks
            v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
            if (t < 2) {
                scr[row * 4 + 2 * t] = v0;
                scr[row * 4 + 2 * t + 1] = v1;
            }
        } else {  // batch 2t + c
            scr[row * 8 + 2 * t] = v0;
            scr[row * 8 + 2 * t + 1] = v1;
        }
        acc.v[rs][0] = acc.v[rs][1] = 0.0f;
    }
    __syncwarp();
#pragma unroll
    for (int b = 0; b < B; ++b) out[b] = scr[lane * B + b];
    __syncwarp();  // before the next tile's scales overwrite the scratch
}

}  // namespace bc
