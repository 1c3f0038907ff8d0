// gemv3.cuh -- persistent, TMA-fed dequant-GEMV (decode) for sm_100a.
//
// Same math as gemv.cuh (the tile consumers are shared); different schedule:
//  * persistent CTAs (one per SM) of 8 warps; the activations are staged once
//    per CTA, for all K, with an optional fused RMSNorm of each row
//    (ops.rs:77-93) so the norm needs no kernel of its own;
//  * stream-K over tiles: the row-group tiles form one contiguous array; CTA
//    c of C takes tiles [c*T/C, (c+1)*T/C) and its warp w the w-th eighth of
//    that range, so every warp reads the same number of bytes (+-1 tile)
//    whatever N and K are. When there are no more row groups than CTA slots
//    (and a group has at least 8 tiles) each CTA takes exactly one group;
//  * each warp owns a ring of S tile buffers in shared memory filled by 1-D
//    bulk asynchronous copies (cp.async.bulk, completion on an mbarrier) that
//    lane 0 issues S tiles ahead, across row-group boundaries too;
//  * a row group wholly inside one warp's range is finished by that warp; a
//    group cut by warp ranges is summed in two levels: the warps of a CTA
//    through shared memory (the last of them to arrive sums in warp order),
//    then, for a group cut by a CTA range boundary, the CTAs through global
//    slots (the last CTA to arrive sums in CTA order); fixed orders, so
//    results are deterministic;
//  * programmatic dependent launch: the first S tiles of every warp are
//    requested before waiting on the previous kernel (weights are never
//    written), so the weight stream overlaps the previous kernel's tail.
// Every mbarrier wait is bounded: after the runtime limit the warp records
// an error (kErrGemvWait), drains its own copies still in flight, and
// returns.
#pragma once

#include "gemv.cuh"
#include "gemv_mma.cuh"

namespace bc {

constexpr int kG3Warps = 8;
constexpr int kG3MaxCtaGroups = 64;  // row groups one CTA range may touch (shared arrival counters)

struct Gemv3Params {
    GemvParams p;         // w, n, n_pad, x, x_f16, x_ld, k, batch, y, y_ld, res, res_ld, rtz, norm_w
    int64_t ktiles;
    int64_t total_tiles;  // groups * ktiles
    int64_t total_warps;
    int stages;
    int kspan;            // staged activation columns (k_pad)
    int xstride;          // int16 codes between staged rows (kspan, +8 for the tensor-core consumer)
    float* slots;         // [CTAs][2][B][32] partial sums of the CTAs' first and last groups
    int* counters;        // [groups], zero at rest
    int* err;             // set to kErrGemvWait when a wait gives up
};

// Staging of the activations. Thread t of pass i covers columns
// c = (256 i + t) * 4 .. c + 3, so the 8 lanes t = 8m .. 8m+7 of a warp hold
// one 32-column block and reduce its absmax and code sum with shuffles. Up to
// kStageRegPasses passes (8192 columns) stay in registers, so the fused
// RMSNorm reads each activation once; the norm weights are fetched before the
// kernel waits on its predecessor (weights are never written).
constexpr int kStageRegPasses = 8;

__device__ __forceinline__ float4 load_x4(const GemvParams& p, bool vec, int b, int64_t c) {
    if (b >= p.batch || c >= p.k) return make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (vec && c + 3 < p.k) {
        if (p.x_f16) {
            const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(p.x) + b * p.x_ld + c);
            const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            return make_float4(lo.x, lo.y, hi.x, hi.y);
        }
        return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + b * p.x_ld + c);
    }
    return make_float4(load_x(p, b, c), load_x(p, b, c + 1), load_x(p, b, c + 2), load_x(p, b, c + 3));
}

// norm weights of columns c .. c+3 (zero past k)
__device__ __forceinline__ float4 load_norm4(const GemvParams& p, bool vec, int64_t c) {
    if (vec && c + 3 < p.k) return __ldg(reinterpret_cast<const float4*>(p.norm_w + c));
    float4 w;
    w.x = c < p.k ? p.norm_w[c] : 0.0f;
    w.y = c + 1 < p.k ? p.norm_w[c + 1] : 0.0f;
    w.z = c + 2 < p.k ? p.norm_w[c + 2] : 0.0f;
    w.w = c + 3 < p.k ? p.norm_w[c + 3] : 0.0f;
    return w;
}

__device__ __forceinline__ int stage_passes(int kspan) { return (kspan + 1023) / 1024; }

__device__ __forceinline__ bool norm_vec_ok(const GemvParams& p) {
    return (reinterpret_cast<uintptr_t>(p.norm_w) & 15) == 0;
}

// Norm weights of the register-resident passes; called before the wait on
// the previous kernel.
__device__ __forceinline__ void prefetch_norm(const GemvParams& p, int kspan, float4 (&nw)[kStageRegPasses]) {
#pragma unroll
    for (int i = 0; i < kStageRegPasses; ++i) nw[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const int passes = stage_passes(kspan);
    if (!p.norm_w || passes > kStageRegPasses) return;
    const bool vec = norm_vec_ok(p);
#pragma unroll
    for (int i = 0; i < kStageRegPasses; ++i)
        if (i < passes) nw[i] = load_norm4(p, vec, (int64_t)(i * 256 + threadIdx.x) * 4);
}

__device__ __forceinline__ uint32_t pack_i16x2(int lo, int hi) { return (uint32_t)(lo & 0xFFFF) | ((uint32_t)hi << 16); }

// Quantise NP passes of 4 activations per lane to int16 codes with one scale
// per 32-column block (scale ~ absmax / 32767, codes = round(v * 32767 /
// absmax) with a correctly rounded reciprocal, clamped to +-32767); Q4_0 takes
// each 8-group in the order e0 e2 e4 e6 e1 e3 e5 e7 to match its nibble pairs.
// The passes are processed stage by stage (all absmax shuffles, then all
// codes, ...) so they overlap. Every lane of the warp calls this; only
// columns c < kspan are stored. v: activations (already normalised), pass i
// covers columns (p0 + i) * 1024 + 4 * threadIdx.x.
template <int FMT, int MODE, int NP>
__device__ __forceinline__ void store_passes(const float4 (&v)[NP], int p0, int kspan, uint8_t* xs, int b, int B,
                                             int nblk, int xstride) {
    const int tid = threadIdx.x;
    if (MODE == MODE_F32) {
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            const int c = (p0 + i) * 1024 + 4 * tid;
            if (c < kspan) *reinterpret_cast<float4*>(reinterpret_cast<float*>(xs) + (size_t)b * kspan + c) = v[i];
        }
        return;
    }
    // code rows xstride int16 apart (the tensor-core consumer pads them so
    // that the batch rows of one column fall in different banks)
    int16_t* xq = reinterpret_cast<int16_t*>(xs) + (size_t)b * xstride;
    float2* sxq = reinterpret_cast<float2*>(xs + (size_t)B * xstride * 2) + b * nblk;  // (scale, code sum)
    float am[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) am[i] = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int i = 0; i < NP; ++i) am[i] = fmaxf(am[i], __shfl_xor_sync(0xffffffffu, am[i], o));
    int q[NP][4], sum[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        const float qi = am[i] > 0.0f ? 32767.0f * __frcp_rn(am[i]) : 0.0f;
        q[i][0] = max(-32767, min(32767, __float2int_rn(__fmul_rn(v[i].x, qi))));
        q[i][1] = max(-32767, min(32767, __float2int_rn(__fmul_rn(v[i].y, qi))));
        q[i][2] = max(-32767, min(32767, __float2int_rn(__fmul_rn(v[i].z, qi))));
        q[i][3] = max(-32767, min(32767, __float2int_rn(__fmul_rn(v[i].w, qi))));
        sum[i] = (q[i][0] + q[i][1]) + (q[i][2] + q[i][3]);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1)
#pragma unroll
        for (int i = 0; i < NP; ++i) sum[i] += __shfl_xor_sync(0xffffffffu, sum[i], o);
    const bool even = (tid & 1) == 0;  // Q4_0: even lanes hold e0..e3 of an 8-group, odd lanes e4..e7
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        uint32_t lo, hi;
        if (FMT == FMT_Q4_0) {
            const uint32_t send = even ? pack_i16x2(q[i][1], q[i][3]) : pack_i16x2(q[i][0], q[i][2]);
            const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, 1);
            lo = even ? pack_i16x2(q[i][0], q[i][2]) : recv;
            hi = even ? recv : pack_i16x2(q[i][1], q[i][3]);
        } else {
            lo = pack_i16x2(q[i][0], q[i][1]);
            hi = pack_i16x2(q[i][2], q[i][3]);
        }
        const int c = (p0 + i) * 1024 + 4 * tid;
        if (c < kspan) {
            *reinterpret_cast<uint2*>(xq + c) = make_uint2(lo, hi);
            if ((tid & 7) == 0) {
                sxq[c >> 5] = make_float2(am[i] * (1.0f / 32767.0f), (float)sum[i]);
            }
        }
    }
}

// One chunk of NP passes loaded from global (rows beyond the register-held
// size), normalised with inv and the norm weights when given, then stored.
template <int FMT, int MODE, int NP>
__device__ __forceinline__ void stage_chunk(const GemvParams& p, bool vec, bool wvec, int b, int p0, float inv,
                                            int kspan, uint8_t* xs, int B, int nblk, int xstride) {
    float4 v[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) v[i] = load_x4(p, vec, b, (int64_t)((p0 + i) * 256 + threadIdx.x) * 4);
    if (p.norm_w) {
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            const float4 w = load_norm4(p, wvec, (int64_t)((p0 + i) * 256 + threadIdx.x) * 4);
            v[i].x = v[i].x * inv * w.x;  // (x * inv_rms) * w, ops.rs:91
            v[i].y = v[i].y * inv * w.y;
            v[i].z = v[i].z * inv * w.z;
            v[i].w = v[i].w * inv * w.w;
        }
    }
    store_passes<FMT, MODE, NP>(v, p0, kspan, xs, b, B, nblk, xstride);
}

// Register-held rows (passes <= 8): NP = passes rounded up to a power of two.
template <int FMT, int MODE, int NP>
__device__ __forceinline__ void stage_held(const GemvParams& p, const float4 (&xr)[kStageRegPasses],
                                           const float4 (&nwr)[kStageRegPasses], float inv, int kspan, uint8_t* xs,
                                           int b, int B, int nblk, int xstride) {
    float4 v[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i) {
        v[i] = xr[i];
        if (p.norm_w) {
            v[i].x = v[i].x * inv * nwr[i].x;  // (x * inv_rms) * w, ops.rs:91
            v[i].y = v[i].y * inv * nwr[i].y;
            v[i].z = v[i].z * inv * nwr[i].z;
            v[i].w = v[i].w * inv * nwr[i].w;
        }
    }
    store_passes<FMT, MODE, NP>(v, 0, kspan, xs, b, B, nblk, xstride);
}

// Staging of all K columns (FAST: int16 codes + scale + code sum per 32;
// F32: floats), rows b >= batch and columns >= k as zeros, with the optional
// RMSNorm (x * inv_rms) * w of ops.rs:77-93. All threads of the CTA take part.
template <int FMT, int MODE, int B>
__device__ __forceinline__ void stage_x_full(const GemvParams& p, uint8_t* xs, int kspan, int xstride,
                                             const float4 (&nwr)[kStageRegPasses]) {
    __shared__ float part[B][kG3Warps];
    constexpr int R = kStageRegPasses;
    const bool vec = (p.x_ld % 4 == 0) &&
                     ((reinterpret_cast<uintptr_t>(p.x) & (p.x_f16 ? 7 : 15)) == 0);
    const bool wvec = p.norm_w && norm_vec_ok(p);
    const int passes = stage_passes(kspan);
    const bool held = passes <= R;
    const int nblk = kspan / 32;
    const int warp = threadIdx.x >> 5;
#pragma unroll 1
    for (int b = 0; b < B; ++b) {
        float4 xr[R];
#pragma unroll
        for (int i = 0; i < R; ++i) xr[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (held) {
#pragma unroll
            for (int i = 0; i < R; ++i)
                if (i < passes) xr[i] = load_x4(p, vec, b, (int64_t)(i * 256 + threadIdx.x) * 4);
        }
        float inv = 1.0f;
        if (p.norm_w) {
            // sum of squares in a fixed order: passes per lane, lanes, warps
            float ss = 0.0f;
            if (held) {
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    ss = fmaf(xr[i].x, xr[i].x, ss);
                    ss = fmaf(xr[i].y, xr[i].y, ss);
                    ss = fmaf(xr[i].z, xr[i].z, ss);
                    ss = fmaf(xr[i].w, xr[i].w, ss);
                }
            } else {
                for (int p0 = 0; p0 < passes; p0 += R) {
                    float4 t[R];
#pragma unroll
                    for (int i = 0; i < R; ++i)
                        t[i] = p0 + i < passes ? load_x4(p, vec, b, (int64_t)((p0 + i) * 256 + threadIdx.x) * 4)
                                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        ss = fmaf(t[i].x, t[i].x, ss);
                        ss = fmaf(t[i].y, t[i].y, ss);
                        ss = fmaf(t[i].z, t[i].z, ss);
                        ss = fmaf(t[i].w, t[i].w, ss);
                    }
                }
            }
            ss = warp_sum(ss);
            if ((threadIdx.x & 31) == 0) part[b][warp] = ss;
            __syncthreads();
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kG3Warps; ++w) tot += part[b][w];
            inv = 1.0f / sqrtf(tot / (float)p.k + p.norm_eps);
        }
        if (held) {
            if (passes <= 1)
                stage_held<FMT, MODE, 1>(p, xr, nwr, inv, kspan, xs, b, B, nblk, xstride);
            else if (passes <= 2)
                stage_held<FMT, MODE, 2>(p, xr, nwr, inv, kspan, xs, b, B, nblk, xstride);
            else if (passes <= 4)
                stage_held<FMT, MODE, 4>(p, xr, nwr, inv, kspan, xs, b, B, nblk, xstride);
            else
                stage_held<FMT, MODE, 8>(p, xr, nwr, inv, kspan, xs, b, B, nblk, xstride);
        } else {
            int p0 = 0;
            for (; p0 + 8 <= passes; p0 += 8) stage_chunk<FMT, MODE, 8>(p, vec, wvec, b, p0, inv, kspan, xs, B, nblk, xstride);
            if (p0 + 4 <= passes) {
                stage_chunk<FMT, MODE, 4>(p, vec, wvec, b, p0, inv, kspan, xs, B, nblk, xstride);
                p0 += 4;
            }
            if (p0 + 2 <= passes) {
                stage_chunk<FMT, MODE, 2>(p, vec, wvec, b, p0, inv, kspan, xs, B, nblk, xstride);
                p0 += 2;
            }
            if (p0 < passes) stage_chunk<FMT, MODE, 1>(p, vec, wvec, b, p0, inv, kspan, xs, B, nblk, xstride);
        }
    }
}

// One tile of a warp's stream, read from its ring slot (lane = row).
template <int FMT>
struct G3Tile {
    uint4 meta;
    uint4 q[Fmt<FMT>::CH];
};

template <int FMT>
__device__ __forceinline__ void g3_load_tile(const uint8_t* tp, int lane, G3Tile<FMT>& r) {
    r.meta = reinterpret_cast<const uint4*>(tp)[lane];
#pragma unroll
    for (int c = 0; c < Fmt<FMT>::CH; ++c) r.q[c] = reinterpret_cast<const uint4*>(tp + 512 + c * 512)[lane];
}

template <int FMT, int MODE, int B>
__device__ __forceinline__ void g3_consume_tile(const G3Tile<FMT>& r, const uint8_t* xs, int kspan, int t,
                                                float (&acc)[B], bool rtz) {
    if (FMT == FMT_Q4_0)
        consume_q4_0<MODE, B>(r.meta, *reinterpret_cast<const uint4(*)[8]>(r.q), xs, kspan, t, acc, rtz);
    else if (FMT == FMT_Q8_0)
        consume_q8_0<MODE, B>(r.meta, *reinterpret_cast<const uint4(*)[16]>(r.q), xs, kspan, t, acc, rtz);
    else
        consume_q4_k<MODE, B>(r.meta, *reinterpret_cast<const uint4(*)[8]>(r.q), xs, kspan, t, acc, rtz);
}

// Bytes of the staged activations (FAST: int16 codes, then per 32-column
// block a float scale and an int code sum; F32: floats), 16-byte multiple.
template <int MODE, int B>
__host__ __device__ __forceinline__ size_t g3_x_bytes(int kspan, int xstride) {
    return MODE == MODE_F32 ? (size_t)B * kspan * 4 : (size_t)B * xstride * 2 + (size_t)B * (kspan / 32) * 8;
}
inline size_t gemv3_red_bytes(int bpad) { return (size_t)kG3Warps * 2 * bpad * 32 * 4; }

// Tile ranges of one warp: the grid's T tiles over C CTAs, the CTA's n
// tiles [cb, ce) over its 8 warps; this warp (w) holds [wb, we).
struct G3Range {
    uint32_t T, C, c, cb, ce, n, w, wb, we;
};

// This warp's ranges (32-bit tile arithmetic: the host keeps total_tiles *
// CTAs < 2^32). Recomputed where needed rather than held in registers
// through the tile loop.
__device__ __forceinline__ G3Range g3_range(uint32_t T) {
    G3Range r;
    r.T = T;
    r.C = gridDim.x;
    r.c = blockIdx.x;
    r.cb = r.c * r.T / r.C;
    r.ce = (r.c + 1) * r.T / r.C;
    r.n = r.ce - r.cb;
    r.w = threadIdx.x >> 5;
    r.wb = r.cb + r.w * r.n / kG3Warps;
    r.we = r.cb + (r.w + 1) * r.n / kG3Warps;
    return r;
}

// End of row group g in this warp's range: store it if the warp holds all of
// it; else leave the warp's partial in shared memory, and the last warp of
// the CTA to arrive sums the CTA's share of g in warp order; if other CTAs
// hold part of g that sum goes to the CTA's global slot and the last CTA to
// arrive (acquire/release arrival counter) sums the slots in CTA order and
// stores. Whole warp. The sum is scaled by inv (1/rms rows) before the
// epilogue. red: [8 warps][2][B][32] floats; cnt: the CTA's arrival counters.
template <int B>
__device__ __forceinline__ void g3_finish_group(const Gemv3Params& a, int epi, uint32_t g, uint32_t KT, int lane,
                                                float (&acc)[B], const float (&inv)[B], float* red, int* cnt,
                                                const EpiPre<B>& pre) {
    const GemvParams& p = a.p;
    const G3Range r = g3_range((uint32_t)a.total_tiles);
    const uint32_t g0 = g * KT, g1 = g0 + KT;
    float v[B];
    if (g0 >= r.wb && g1 <= r.we) {
#pragma unroll
        for (int b = 0; b < B; ++b) v[b] = acc[b] * inv[b];
        gemv_store<B>(p, epi, g, lane, v, &pre);
        return;
    }
    // level 1: the CTA's warps holding part of g, [wf, wl]
    const uint32_t lo = max(g0, r.cb) - r.cb, hi = min(g1, r.ce) - r.cb;
    const uint32_t wf = ((lo + 1) * kG3Warps - 1) / r.n, wl = (hi * kG3Warps - 1) / r.n;
#pragma unroll
    for (int b = 0; b < B; ++b) v[b] = acc[b];
    if (wf < wl) {
        float* mine = red + ((r.w * 2 + (r.wb >= g0 ? 0 : 1)) * B) * 32;
#pragma unroll
        for (int b = 0; b < B; ++b) mine[b * 32 + lane] = acc[b];
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&cnt[g - r.cb / KT], 1) == (int)(wl - wf);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) return;
        __threadfence_block();
#pragma unroll
        for (int b = 0; b < B; ++b) v[b] = 0.0f;
        for (uint32_t w2 = wf; w2 <= wl; ++w2) {
            const uint32_t s2 = r.cb + w2 * r.n / kG3Warps;  // g is w2's first group iff its range starts in g
            const float* src = red + ((w2 * 2 + (s2 >= g0 ? 0 : 1)) * B) * 32;
#pragma unroll
            for (int b = 0; b < B; ++b) v[b] += src[b * 32 + lane];
        }
    }
    if (g0 >= r.cb && g1 <= r.ce) {
#pragma unroll
        for (int b = 0; b < B; ++b) v[b] *= inv[b];
        gemv_store<B>(p, epi, g, lane, v, &pre);
        return;
    }
    // level 2: the CTAs holding part of g, [cf, cl]
    const uint32_t cf = ((g0 + 1) * r.C - 1) / r.T, cl = (g1 * r.C - 1) / r.T;
    float* mine = a.slots + (((int64_t)r.c * 2 + (r.cb >= g0 ? 0 : 1)) * B) * 32;
#pragma unroll
    for (int b = 0; b < B; ++b) __stcg(&mine[b * 32 + lane], v[b]);
    // __syncwarp orders the lanes' stores before lane 0's release;
    // the last arriver's acquire makes every contributor's visible
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomic_add_acq_rel_gpu(&a.counters[g], 1) == (int)(cl - cf);
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    if (!last) return;
    constexpr int U = B >= 8 ? 1 : 8 / B;  // contributor slots loaded together
#pragma unroll
    for (int b = 0; b < B; ++b) v[b] = 0.0f;
    for (uint32_t c0 = cf; c0 <= cl; c0 += U) {
        float part[U][B];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint32_t c2 = c0 + u;
            if (c2 <= cl) {
                const uint32_t s2 = (uint32_t)((uint64_t)c2 * r.T / r.C);
                const int sl = (s2 >= g0) ? 0 : 1;  // g is c2's first group iff its range starts in g
                const float* src = a.slots + (((int64_t)c2 * 2 + sl) * B) * 32;
#pragma unroll
                for (int b = 0; b < B; ++b) part[u][b] = __ldcg(&src[b * 32 + lane]);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (c0 + u <= cl) {
#pragma unroll
                for (int b = 0; b < B; ++b) v[b] += part[u][b];
            }
    }
#pragma unroll
    for (int b = 0; b < B; ++b) v[b] *= inv[b];
    gemv_store<B>(p, epi, g, lane, v, &pre);
    if (lane == 0) a.counters[g] = 0;
}

template <int FMT, int MODE, int B, bool MMA>
__global__ void __launch_bounds__(kG3Warps * 32, (B <= 2 ? 2 : 1)) qgemv3_kernel(const Gemv3Params a, const int epi) {
    static_assert(!MMA || MODE == MODE_FAST, "the tensor-core consumer serves the fast numerics");
    extern __shared__ __align__(128) uint8_t g3_smem[];
    uint8_t* smem = g3_smem;
    const GemvParams& p = a.p;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;
    const int64_t tb = p.tile_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                       // [warps][S]
    uint8_t* ring = smem + 128 * ((kG3Warps * S * 8 + 127) / 128);           // [warps][S][tile]
    uint8_t* xs = ring + (size_t)kG3Warps * S * tb;                          // staged activations
    float* red = reinterpret_cast<float*>(xs + g3_x_bytes<MODE, B>(a.kspan, a.xstride));  // [warps][2][B][32] partials
    uint64_t* mybar = bars + warp * S;
    uint8_t* myring = ring + (size_t)warp * S * tb;

    // 32-bit tile arithmetic (the host keeps total_tiles * CTAs < 2^32)
    const G3Range rg = g3_range((uint32_t)a.total_tiles);
    const int64_t t_begin = rg.wb;
    const int n = (int)(rg.we - rg.wb);
    __shared__ int cta_cnt[kG3MaxCtaGroups];  // arrivals per row group of this CTA's range
    for (int i = threadIdx.x; i < kG3MaxCtaGroups; i += blockDim.x) cta_cnt[i] = 0;

    if (lane == 0)
        for (int s = 0; s < S; ++s) mbar_init(&mybar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncwarp();
    // start the weight stream before anything that depends on earlier kernels
    if (lane == 0)
        for (int i = 0; i < min(S, n); ++i) {
            mbar_expect_tx(&mybar[i], (uint32_t)tb);
            bulk_g2s(myring + (size_t)i * tb, p.w + (t_begin + i) * tb, (uint32_t)tb, &mybar[i]);
        }
    __shared__ __align__(8) uint64_t qx_bar;
    __shared__ float inv_s[B];
    float inv[B];  // 1/rms per row when the producer quantised x * norm_w
#pragma unroll
    for (int b = 0; b < B; ++b) inv[b] = 1.0f;
    const bool from_image = MODE == MODE_FAST && p.qx.data != nullptr;
    float4 nwr[kStageRegPasses];
    if (from_image) {
        if (threadIdx.x == 0) {
            mbar_init(&qx_bar, 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
    } else {
        prefetch_norm(p, a.kspan, nwr);
    }
    // the epilogue operands of the group this warp finishes last: the next
    // GEMV's norm weight now (a weight), the residual once the wait is over
    EpiPre<B> pre;
    const uint32_t g_last = (rg.we - 1) / (uint32_t)a.ktiles;
    const int64_t pre_row = (int64_t)g_last * 32 + lane;
    pre.nw = 0.0f;
#pragma unroll
    for (int b = 0; b < B; ++b) pre.res[b] = 0.0f;
    if (epi == EPI_ADD && p.qy.data && p.qy.norm_w && pre_row < p.n) pre.nw = __ldg(&p.qy.norm_w[pre_row]);
    pdl_trigger();
    pdl_wait();
    if (epi == EPI_ADD && p.res) {
        pre.g = (int)g_last;
#pragma unroll
        for (int b = 0; b < B; ++b)
            pre.res[b] = (b < p.batch && pre_row < p.n) ? __ldcg(&p.res[b * p.res_ld + pre_row]) : 0.0f;
    }
    if (from_image) {
        // the producer's staging image: bulk copies, and 1/rms from its block sums
        __syncthreads();
        // the FAST image: B rows of kspan codes, then the block scales; rows
        // land xstride codes apart
        const uint32_t row_bytes = (uint32_t)a.kspan * 2, sc_bytes = (uint32_t)B * (a.kspan / 32) * 8;
        if (threadIdx.x == 0) {
            mbar_expect_tx(&qx_bar, (uint32_t)B * row_bytes + sc_bytes);
            for (int b = 0; b < B; ++b)
                for (uint32_t off = 0; off < row_bytes; off += 16384u)
                    bulk_g2s(xs + (size_t)b * a.xstride * 2 + off, p.qx.data + (size_t)b * row_bytes + off,
                             min(16384u, row_bytes - off), &qx_bar);
            for (uint32_t off = 0; off < sc_bytes; off += 16384u)
                bulk_g2s(xs + (size_t)B * a.xstride * 2 + off, p.qx.data + (size_t)B * row_bytes + off,
                         min(16384u, sc_bytes - off), &qx_bar);
        }
        // warp b sums row b's block sums of squares (B <= 8 warps)
        if (p.qx.ss && warp < B) {
            const int nblk = a.kspan / 32;
            float t = 0.0f;
            for (int j = lane; j < nblk; j += 32) t += __ldcg(&p.qx.ss[warp * nblk + j]);
            t = warp_sum(t);
            if (lane == 0) inv_s[warp] = 1.0f / sqrtf(t / (float)p.k + p.norm_eps);
        }
        if (!mbar_wait_bounded(&qx_bar, 0)) {
            if (threadIdx.x == 0) {
                atomicExch(a.err, kErrGemvWait);
                mbar_drain(&qx_bar, 0);  // the image copy must land before the CTA exits
            }
        }
    } else {
        stage_x_full<FMT, MODE, B>(p, xs, a.kspan, a.xstride, nwr);
    }
    __syncthreads();
    if (from_image && p.qx.ss) {
#pragma unroll
        for (int b = 0; b < B; ++b) inv[b] = inv_s[b];
    }

    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.0f;
    const bool rtz = p.rtz != 0;
    bool ok = true;
    const uint32_t KT = (uint32_t)a.ktiles;
    uint32_t g = rg.wb / KT;      // row group of the current tile
    uint32_t t = rg.wb - g * KT;  // its k-tile
    int i = 0;
    // tensor-core consumer: per-warp scratch after the split-K partials
    float* scr = red + kG3Warps * 2 * B * 32 + warp * mma_scratch_floats<FMT, B>();
    MmaAcc macc;
#pragma unroll
    for (int r = 0; r < 4; ++r) macc.v[r][0] = macc.v[r][1] = 0.0f;
    for (; i < n; ++i) {
        const int st = i % S;
        if (!mbar_wait_bounded(&mybar[st], (uint32_t)((i / S) & 1))) {
            ok = false;
            break;
        }
        const uint8_t* tp = myring + (size_t)st * tb;
        auto refill = [&]() {
            if (lane == 0 && i + S < n) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect_tx(&mybar[st], (uint32_t)tb);
                bulk_g2s(myring + (size_t)st * tb, p.w + (t_begin + i + S) * tb, (uint32_t)tb, &mybar[st]);
            }
        };
        if constexpr (MMA) {
            MmaTileRegs<FMT> regs;
            mma_load_tile<FMT>(tp, lane, regs);
            mma_scales<FMT>(tp, lane, scr);
            __syncwarp();
            if (FMT != FMT_Q8_0) refill();  // Q4 tiles are in registers now
            mma_consume_tile<FMT, B>(regs, tp, xs, a.kspan, a.xstride, (int)t, scr, macc, lane);
            if (FMT == FMT_Q8_0) {
                __syncwarp();
                refill();
            }
        } else {
            G3Tile<FMT> tile;
            g3_load_tile<FMT>(tp, lane, tile);
            __syncwarp();
            refill();
            g3_consume_tile<FMT, MODE, B>(tile, xs, a.kspan, (int)t, acc, rtz);
        }
        // end of a row group (or of this warp's range): finish it
        if (t == KT - 1 || i == n - 1) {
            if constexpr (MMA) mma_rows_to_lanes<B>(macc, scr, acc, lane);
            g3_finish_group<B>(a, epi, g, KT, lane, acc, inv, red, cta_cnt, pre);
#pragma unroll
            for (int b = 0; b < B; ++b) acc[b] = 0.0f;
        } else if constexpr (MMA) {
            __syncwarp();  // the tile's scales have been read before the next tile's overwrite them
        }
        if (++t == KT) {
            t = 0;
            ++g;
        }
    }
    if (!ok) {
        if (lane == 0) atomicExch(a.err, kErrGemvWait);
        // let this warp's copies still in flight land before the CTA exits
        for (int j = i; j < n && j < i + S; ++j) mbar_drain(&mybar[j % S], (uint32_t)((j / S) & 1));
    }
}

// Staged row stride in int16 codes: the tensor-core consumer reads one column
// block of all B rows together, so its rows are padded by 16 bytes to fall in
// different shared-memory banks.
inline int64_t gemv3_xstride(bool mma, int64_t kspan) { return mma ? kspan + 8 : kspan; }
inline size_t gemv3_x_bytes(int mode, int bpad, int64_t kspan, bool mma = false) {
    return mode == MODE_F32 ? (size_t)bpad * kspan * 4
                            : (size_t)bpad * gemv3_xstride(mma, kspan) * 2 + (size_t)bpad * (kspan / 32) * 8;
}
inline size_t gemv3_bar_bytes(int stages) { return 128 * (((size_t)kG3Warps * stages * 8 + 127) / 128); }
// Per-CTA scratch of the tensor-core consumer (block scales / row transpose).
inline size_t gemv3_mma_bytes(int32_t dtype, int bpad) {
    const size_t scales = dtype == BEACON_CUDA_DTYPE_Q4_K ? 512 : 256;
    return (size_t)kG3Warps * 4 * std::max<size_t>(scales, (size_t)32 * bpad);
}

template <int FMT, int MODE, int B, bool MMA>
void launch_qgemv3_t(const LinearPlan& pl, const GemvLaunch& a) {
    Gemv3Params q;
    GemvParams& p = q.p;
    p.w = static_cast<const uint8_t*>(a.w);
    p.ktiles = a.L->ktiles();
    p.tile_bytes = a.L->tile_bytes;
    p.n = a.L->n;
    p.n_pad = a.L->n_pad;
    p.tps = 0;
    p.ksplit = 1;
    p.x = a.x;
    p.x_f16 = a.x_f16 ? 1 : 0;
    p.x_ld = a.x_ld;
    p.k = a.L->k;
    p.batch = a.batch;
    p.y = a.y;
    p.y_ld = a.y_ld;
    p.res = a.res;
    p.res_ld = a.res_ld;
    p.partial = nullptr;
    p.counters = nullptr;
    p.rtz = a.rtz ? 1 : 0;
    p.norm_w = a.norm_w;
    p.norm_eps = a.norm_eps;
    p.qkv = a.qkv ? *a.qkv : QkvEpi{};
    p.qx = a.qx;
    p.qy = a.qy;
    q.ktiles = a.L->ktiles();
    q.total_tiles = a.L->groups() * q.ktiles;
    q.total_warps = pl.total_warps;
    q.stages = pl.stages;
    q.kspan = (int)a.L->k_pad;
    q.xstride = (int)gemv3_xstride(MMA, a.L->k_pad);
    q.slots = a.scratch.partial;
    q.counters = a.scratch.counters;
    q.err = a.scratch.err;
    auto kern = qgemv3_kernel<FMT, MODE, B, MMA>;
    allow_max_dynamic_smem(kern);
    launch_kernel(kern, dim3((unsigned)pl.nctas), dim3(kG3Warps * 32), pl.smem, a.s, a.pdl, q, a.epi);
}

template <int FMT>
void launch_qgemv3_fmt(const LinearPlan& pl, const GemvLaunch& a) {
    if (a.mode == MODE_FAST && pl.mma) {
        switch (pl.bpad) {
            case 1: return launch_qgemv3_t<FMT, MODE_FAST, 1, true>(pl, a);
            case 2: return launch_qgemv3_t<FMT, MODE_FAST, 2, true>(pl, a);
            case 4: return launch_qgemv3_t<FMT, MODE_FAST, 4, true>(pl, a);
            default: return launch_qgemv3_t<FMT, MODE_FAST, 8, true>(pl, a);
        }
    }
    if (a.mode == MODE_FAST) {
        switch (pl.bpad) {
            case 1: return launch_qgemv3_t<FMT, MODE_FAST, 1, false>(pl, a);
            case 2: return launch_qgemv3_t<FMT, MODE_FAST, 2, false>(pl, a);
            case 4: return launch_qgemv3_t<FMT, MODE_FAST, 4, false>(pl, a);
            default: return launch_qgemv3_t<FMT, MODE_FAST, 8, false>(pl, a);
        }
    }
    switch (pl.bpad) {
        case 1: return launch_qgemv3_t<FMT, MODE_F32, 1, false>(pl, a);
        case 2: return launch_qgemv3_t<FMT, MODE_F32, 2, false>(pl, a);
        case 4: return launch_qgemv3_t<FMT, MODE_F32, 4, false>(pl, a);
        default: return launch_qgemv3_t<FMT, MODE_F32, 8, false>(pl, a);
    }
}

}  // namespace bc
