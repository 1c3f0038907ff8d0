// gemv3.cuh -- persistent, TMA-fed dequant-GEMV (decode) for sm_100a.
//
// Same math as gemv.cuh (the tile consumers are shared); different schedule:
//  * persistent CTAs (one per SM) of 8 warps; the activations are staged once
//    per CTA, for all K, with an optional fused RMSNorm of each row
//    (ops.rs:77-93) so the norm needs no kernel of its own;
//  * stream-K over tiles: the row-group tiles form one contiguous array, and
//    warp w of W streams tiles [w*T/W, (w+1)*T/W), so every warp reads the
//    same number of bytes (+-1 tile) whatever N and K are;
//  * each warp owns a ring of S tile buffers in shared memory filled by 1-D
//    bulk asynchronous copies (cp.async.bulk, completion on an mbarrier) that
//    lane 0 issues S tiles ahead, across row-group boundaries too;
//  * a row group wholly inside one warp's range is finished by that warp; a
//    group cut by a range boundary is summed by its last contributor in warp
//    order (fixed order, so results are deterministic);
//  * programmatic dependent launch: the first S tiles of every warp are
//    requested before waiting on the previous kernel (weights are never
//    written), so the weight stream overlaps the previous kernel's tail.
// Every mbarrier wait is bounded: after ~2^31 clock cycles the warp records
// an error, waits (again bounded) for its own copies still in flight, and
// returns.
#pragma once

#include "gemv.cuh"

namespace bc {

constexpr int kG3Warps = 8;
constexpr long long kG3WaitLimit = 1LL << 31;

struct Gemv3Params {
    GemvParams p;         // w, n, n_pad, x, x_f16, x_ld, k, batch, y, y_ld, res, res_ld, rtz, norm_w
    int64_t ktiles;
    int64_t total_tiles;  // groups * ktiles
    int64_t total_warps;
    int stages;
    int kspan;            // staged activation columns (k_pad)
    float* slots;         // [total_warps][2][B][32] partial sums
    int* counters;        // [groups], zero at rest
    int* err;             // set to 1 when a wait gives up
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait; false if the limit was reached.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kG3WaitLimit) return false;
    return true;
}

// 32 consecutive activations of row b starting at column c (zero past k),
// RMSNorm-scaled when a norm weight is given.
template <int B>
__device__ __forceinline__ void load_x32(const GemvParams& p, bool vec, int b, int64_t c, const float* inv,
                                         float (&v)[32]) {
    if (vec && b < p.batch && c + 31 < p.k) {
        const float4* src = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + b * p.x_ld + c);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 f = src[q];
            v[4 * q] = f.x;
            v[4 * q + 1] = f.y;
            v[4 * q + 2] = f.z;
            v[4 * q + 3] = f.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = load_x(p, b, c + e);
    }
    if (p.norm_w && b < p.batch) {
        const float r = inv[b];
#pragma unroll
        for (int e = 0; e < 32; ++e)
            if (c + e < p.k) v[e] = v[e] * r * p.norm_w[c + e];  // (x * inv_rms) * w, ops.rs:91
    }
}

// Staging of all K columns (FAST: int16 codes + scale + sum per 32 with the
// format's element order; F32: floats). Same layout as gemv.cuh's stage_x
// with span = kspan. All threads of the CTA take part.
template <int FMT, int MODE, int B>
__device__ __forceinline__ void stage_x_full(const GemvParams& p, uint8_t* xs, int kspan) {
    __shared__ float part[kG3Warps][B];
    __shared__ float inv[B];
    const bool vec = !p.x_f16 && (p.x_ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0);
    if (p.norm_w) {
        // sum of squares per row in a fixed order: lanes, then warps
        float ss[B];
#pragma unroll
        for (int b = 0; b < B; ++b) ss[b] = 0.0f;
        for (int64_t c = (int64_t)threadIdx.x * 4; c < p.k; c += (int64_t)blockDim.x * 4) {
#pragma unroll
            for (int b = 0; b < B; ++b) {
                if (b >= p.batch) break;
                float4 f;
                if (vec && c + 3 < p.k) {
                    f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + b * p.x_ld + c);
                } else {
                    f.x = load_x(p, b, c);
                    f.y = load_x(p, b, c + 1);
                    f.z = load_x(p, b, c + 2);
                    f.w = load_x(p, b, c + 3);
                }
                ss[b] = fmaf(f.x, f.x, ss[b]);
                ss[b] = fmaf(f.y, f.y, ss[b]);
                ss[b] = fmaf(f.z, f.z, ss[b]);
                ss[b] = fmaf(f.w, f.w, ss[b]);
            }
        }
        const int warp = threadIdx.x >> 5;
#pragma unroll
        for (int b = 0; b < B; ++b) {
            const float w = warp_sum(ss[b]);
            if ((threadIdx.x & 31) == 0) part[warp][b] = w;
        }
        __syncthreads();
        if (threadIdx.x < B) {
            float t = 0.0f;
            for (int w = 0; w < kG3Warps; ++w) t += part[w][threadIdx.x];
            inv[threadIdx.x] = 1.0f / sqrtf(t / (float)p.k + p.norm_eps);
        }
        __syncthreads();
    }
    if (MODE == MODE_F32) {
        float* o = reinterpret_cast<float*>(xs);
        const int nblk = kspan / 32;
        for (int i = threadIdx.x; i < B * nblk; i += blockDim.x) {
            const int b = i / nblk, j = i - b * nblk;
            float v[32];
            load_x32<B>(p, vec, b, (int64_t)j * 32, inv, v);
            float4* dst = reinterpret_cast<float4*>(o + (size_t)b * kspan + j * 32);
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        }
        return;
    }
    int16_t* xq = reinterpret_cast<int16_t*>(xs);
    const int nblk = kspan / 32;
    float* sx = reinterpret_cast<float*>(xs + (size_t)B * kspan * 2);
    int* sq = reinterpret_cast<int*>(sx + B * nblk);
    for (int i = threadIdx.x; i < B * nblk; i += blockDim.x) {
        const int b = i / nblk, j = i - b * nblk;
        float v[32];
        load_x32<B>(p, vec, b, (int64_t)j * 32, inv, v);
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
        const float qi = amax > 0.0f ? __fdiv_rn(32767.0f, amax) : 0.0f;
        int sum = 0;
        int qv[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            qv[e] = max(-32767, min(32767, __float2int_rn(__fmul_rn(v[e], qi))));
            sum += qv[e];
        }
        uint32_t packed[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
            int a0, a1;
            if (FMT == FMT_Q4_0) {  // 8-groups as e0 e2 e4 e6 e1 e3 e5 e7, matching the nibble pairs
                const int grp = e & ~7, s0 = e & 7, s1 = s0 + 1;
                a0 = qv[grp + (s0 < 4 ? 2 * s0 : 2 * (s0 - 4) + 1)];
                a1 = qv[grp + (s1 < 4 ? 2 * s1 : 2 * (s1 - 4) + 1)];
            } else {
                a0 = qv[e];
                a1 = qv[e + 1];
            }
            packed[e / 2] = (uint32_t)(a0 & 0xFFFF) | ((uint32_t)a1 << 16);
        }
        uint4* dst = reinterpret_cast<uint4*>(xq + (size_t)b * kspan + j * 32);
#pragma unroll
        for (int c = 0; c < 4; ++c)
            dst[c] = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
        sx[b * nblk + j] = amax > 0.0f ? __fdiv_rn(amax, 32767.0f) : 0.0f;
        sq[b * nblk + j] = sum;
    }
}

template <int FMT, int MODE, int B>
__global__ void __launch_bounds__(kG3Warps * 32, 1) qgemv3_kernel(const Gemv3Params a, const int epi) {
    extern __shared__ __align__(128) uint8_t g3_smem[];
    uint8_t* smem = g3_smem;
    constexpr int CH = Fmt<FMT>::CH;
    const GemvParams& p = a.p;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;
    const int64_t tb = p.tile_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                       // [warps][S]
    uint8_t* ring = smem + 128 * ((kG3Warps * S * 8 + 127) / 128);           // [warps][S][tile]
    uint8_t* xs = ring + (size_t)kG3Warps * S * tb;                          // staged activations
    uint64_t* mybar = bars + warp * S;
    uint8_t* myring = ring + (size_t)warp * S * tb;

    const int64_t gw = (int64_t)blockIdx.x * kG3Warps + warp;
    const int64_t t_begin = gw * a.total_tiles / a.total_warps;
    const int64_t t_end = (gw + 1) * a.total_tiles / a.total_warps;
    const int n = (int)(t_end - t_begin);

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
    pdl_trigger();
    pdl_wait();
    stage_x_full<FMT, MODE, B>(p, xs, a.kspan);
    __syncthreads();

    float acc[B];
#pragma unroll
    for (int b = 0; b < B; ++b) acc[b] = 0.0f;
    const bool rtz = p.rtz != 0;
    bool ok = true;
    int i = 0;
    for (; i < n; ++i) {
        const int st = i % S;
        if (!mbar_wait_bounded(&mybar[st], (uint32_t)((i / S) & 1))) {
            ok = false;
            break;
        }
        const uint8_t* tp = myring + (size_t)st * tb;
        const uint4 meta = reinterpret_cast<const uint4*>(tp)[lane];
        uint4 q[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) q[c] = reinterpret_cast<const uint4*>(tp + 512 + c * 512)[lane];
        __syncwarp();
        if (lane == 0 && i + S < n) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(&mybar[st], (uint32_t)tb);
            bulk_g2s(myring + (size_t)st * tb, p.w + (t_begin + i + S) * tb, (uint32_t)tb, &mybar[st]);
        }
        const int64_t tl = t_begin + i;
        const int64_t g = tl / a.ktiles;
        const int t = (int)(tl - g * a.ktiles);
        if (FMT == FMT_Q4_0)
            consume_q4_0<MODE, B>(meta, *reinterpret_cast<uint4(*)[8]>(q), xs, a.kspan, t, acc, rtz);
        else if (FMT == FMT_Q8_0)
            consume_q8_0<MODE, B>(meta, *reinterpret_cast<uint4(*)[16]>(q), xs, a.kspan, t, acc, rtz);
        else
            consume_q4_k<MODE, B>(meta, *reinterpret_cast<uint4(*)[8]>(q), xs, a.kspan, t, acc, rtz);
        // end of a row group (or of this warp's range): finish it
        if (t == a.ktiles - 1 || i == n - 1) {
            const int64_t g0 = g * a.ktiles, g1 = g0 + a.ktiles;
            if (g0 >= t_begin && g1 <= t_end) {
                gemv_store<B>(p, epi, g, lane, acc);
            } else {
                // contributors to group g: warps whose ranges meet [g0, g1)
                const int64_t wf = ((g0 + 1) * a.total_warps - 1) / a.total_tiles;
                const int64_t wl = (g1 * a.total_warps - 1) / a.total_tiles;
                const int slot = (t_begin >= g0) ? 0 : 1;  // 0: g is the first group of my range
                float* mine = a.slots + ((gw * 2 + slot) * B) * 32;
#pragma unroll
                for (int b = 0; b < B; ++b) mine[b * 32 + lane] = acc[b];
                __threadfence();
                __syncwarp();
                int last = 0;
                if (lane == 0) last = atomicAdd(&a.counters[g], 1) == (int)(wl - wf);
                last = __shfl_sync(0xffffffffu, last, 0);
                if (last) {
                    __threadfence();
                    float v[B];
#pragma unroll
                    for (int b = 0; b < B; ++b) v[b] = 0.0f;
                    for (int64_t w2 = wf; w2 <= wl; ++w2) {
                        const int64_t s2 = w2 * a.total_tiles / a.total_warps;
                        const int sl = (s2 >= g0) ? 0 : 1;  // g is w2's first group iff its range starts in g
                        const float* src = a.slots + ((w2 * 2 + sl) * B) * 32;
#pragma unroll
                        for (int b = 0; b < B; ++b) v[b] += __ldcg(&src[b * 32 + lane]);
                    }
                    gemv_store<B>(p, epi, g, lane, v);
                    if (lane == 0) a.counters[g] = 0;
                }
            }
#pragma unroll
            for (int b = 0; b < B; ++b) acc[b] = 0.0f;
        }
    }
    if (!ok) {
        if (lane == 0) atomicExch(a.err, 1);
        // let this warp's copies still in flight land before the CTA exits
        for (int j = i; j < n && j < i + S; ++j) mbar_wait_bounded(&mybar[j % S], (uint32_t)((j / S) & 1));
    }
}

inline size_t gemv3_x_bytes(int mode, int bpad, int64_t kspan) {
    return mode == MODE_F32 ? (size_t)bpad * kspan * 4 : (size_t)bpad * kspan * 2 + (size_t)bpad * (kspan / 32) * 8;
}
inline size_t gemv3_bar_bytes(int stages) { return 128 * (((size_t)kG3Warps * stages * 8 + 127) / 128); }

template <int FMT, int MODE, int B>
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
    q.ktiles = a.L->ktiles();
    q.total_tiles = a.L->groups() * q.ktiles;
    q.total_warps = pl.total_warps;
    q.stages = pl.stages;
    q.kspan = (int)a.L->k_pad;
    q.slots = a.scratch.partial;
    q.counters = a.scratch.counters;
    q.err = a.scratch.err;
    auto kern = qgemv3_kernel<FMT, MODE, B>;
    BC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
    launch_kernel(kern, dim3((unsigned)pl.nctas), dim3(kG3Warps * 32), pl.smem, a.s, a.pdl, q, a.epi);
}

template <int FMT>
void launch_qgemv3_fmt(const LinearPlan& pl, const GemvLaunch& a) {
    if (a.mode == MODE_FAST) {
        switch (pl.bpad) {
            case 1: return launch_qgemv3_t<FMT, MODE_FAST, 1>(pl, a);
            case 2: return launch_qgemv3_t<FMT, MODE_FAST, 2>(pl, a);
            case 4: return launch_qgemv3_t<FMT, MODE_FAST, 4>(pl, a);
            default: return launch_qgemv3_t<FMT, MODE_FAST, 8>(pl, a);
        }
    }
    switch (pl.bpad) {
        case 1: return launch_qgemv3_t<FMT, MODE_F32, 1>(pl, a);
        case 2: return launch_qgemv3_t<FMT, MODE_F32, 2>(pl, a);
        case 4: return launch_qgemv3_t<FMT, MODE_F32, 4>(pl, a);
        default: return launch_qgemv3_t<FMT, MODE_F32, 8>(pl, a);
    }
}

}  // namespace bc
