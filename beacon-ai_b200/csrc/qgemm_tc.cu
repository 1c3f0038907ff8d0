// qgemm_tc.cu -- prefill dequant-GEMM on the 5th-generation tensor cores.
//
// Y[M, N] = X[M, K] W[N, K]^T for a tiled quantized W (QLayout: 32-row x
// 256-column tiles of Q4_0 / Q8_0 / Q4_K blocks), the prefill counterpart of
// quantized_matmul (backend.rs:32-41 via proj_matmul, engine.rs:159-169).
//
// One CTA computes a 256 x 256 output tile as two 128-row halves, each a
// tcgen05.mma chain (cta_group::1, kind::f16, M = 128, N = 256, K = 16 per
// instruction) accumulating in f32 in its own 256 tensor-memory columns, so
// every dequantised weight slice feeds both halves. The K loop runs over
// 64-column slices through a 3-stage shared-memory ring:
//  * one thread loads the activation slice (256 rows x 64 f16) with a tensor
//    TMA copy in the 128-byte swizzle (rows past M and columns past K arrive
//    as zeros); f32 activations are first converted to an f16 copy;
//  * 16 producer warps dequantise the weight slice (256 rows x 64), two
//    threads per row (32 columns each), from its blocks (q * d, q * sc*d -
//    m*dmin as in dequant.rs:160-365, in f32, then rounded to f16) into the
//    K-major 128-byte-swizzled layout the MMA reads (16-byte chunk j of row r
//    at j ^ (r % 8) within each 8-row atom); each thread fetches the next
//    slice's block bytes before it converts the current one, then
//    fence.proxy.async and an mbarrier arrival;
//  * one thread of the MMA warp waits for the stage, issues 8 MMAs and
//    commits them to the stage's "empty" mbarrier, which the producers wait
//    on before refilling; a final commit signals the epilogue;
//  * the 16 producer warps then read the accumulators with tcgen05.ld (warp
//    w: lanes 32 (w % 4) .., row half (w / 4) % 2, columns 128 (w / 8) ..)
//    and run the epilogue (store, residual add, SwiGLU, or the fused q/k/v
//    write).
// Operands are f16 x f16 (one MMA type for A and B). Every mbarrier wait is
// bounded; a wait that gives up sets *err = 4, the kernel stops issuing work,
// waits (bounded) for the MMAs already issued and frees its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "gemv.cuh"
#include "internal.h"
#include "kernels.h"
#include "qgemm_tc.h"

namespace bc {
namespace {

constexpr int kTcBM = 256, kTcBN = 256, kTcBK = 64, kTcStages = 3;
constexpr int kTcHalf = 128;                 // rows per MMA (M)
constexpr int kTcProducerWarps = 16;  // two threads per weight row
constexpr int kTcMmaWarp = kTcProducerWarps;
constexpr int kTcTmaWarp = kTcProducerWarps + 1;
constexpr int kTcThreads = (kTcProducerWarps + 2) * 32;
constexpr int kTcATile = kTcBM * kTcBK * 2;  // 32 KB
constexpr int kTcBTile = kTcBN * kTcBK * 2;  // 32 KB
constexpr int kTcStage = kTcATile + kTcBTile;
constexpr size_t kTcSmem = (size_t)kTcStages * kTcStage + 1024;  // + alignment slack
constexpr uint32_t kTcTmemCols = 512;

// K-major, 128-byte swizzle: 8-row atoms of 1024 bytes, rows of 128 bytes.
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// UMMA shared-memory descriptor: start >> 4, leading offset 1 (unused for
// swizzled K-major), stride 1024 bytes between 8-row atoms, version 1,
// layout SWIZZLE_128B (2).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D f32, A = B = f16, both K-major,
// N = 256, M = 128.
constexpr uint32_t kTcIdesc = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(kTcBN >> 3) << 17) |
                              ((uint32_t)(kTcHalf >> 4) << 24);

// 2-D tensor copy of one box into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(adesc), "l"(bdesc), "r"(kTcIdesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b, bool rtz) {
    if (rtz) return (uint32_t)f32_to_f16_rtz(a) | ((uint32_t)f32_to_f16_rtz(b) << 16);
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

struct TcParams {
    const uint8_t* w;
    int64_t ktiles, tile_bytes, n, n_pad, k;
    int m;
    float* y;
    int64_t y_ld;
    const float* res;
    int64_t res_ld;
    int epi;
    int rtz;
    QkvEpi qkv;
    int* err;
};

// Block bytes of one half (h) of a 64-column slice of a W row: its meta
// lane and the 1 (Q4_0, Q4_K) or 2 (Q8_0) 16-byte chunks that half covers.
struct RawSlice {
    uint4 meta;
    uint4 c[2];
};

template <int FMT>
__device__ __forceinline__ void load_slice(const TcParams& p, int64_t row, int kb, int h, RawSlice& r) {
    const int64_t g = row >> 5;
    const int li = (int)(row & 31);
    const int t = kb >> 2, qk = kb & 3;
    const uint8_t* tile = p.w + (g * p.ktiles + t) * p.tile_bytes;
    r.meta = __ldg(reinterpret_cast<const uint4*>(tile) + li);
    constexpr int NC = FMT == FMT_Q8_0 ? 2 : 1;  // chunks per half slice
#pragma unroll
    for (int i = 0; i < NC; ++i)
        r.c[i] = __ldg(reinterpret_cast<const uint4*>(tile + 512 + (2 * NC * qk + NC * h + i) * 512) + li);
}

// 32 dequantised weights (half h of slice kb of a W row) as 4 f16 chunks
// with their chunk indices (0..7) within the 64-column slice.
template <int FMT>
__device__ __forceinline__ void dequant_half(const RawSlice& raw, int kb, int h, bool rtz, uint4 (&out)[4],
                                             int (&pos)[4]) {
    const int qk = kb & 3;
    const uint4 meta = raw.meta;
    if (FMT == FMT_Q4_0) {
        // block 2qk + h = chunk 2qk + h; byte i -> elements 2i (lo), 2i + 1 (hi): chunks 4h .. 4h + 3
        const uint4 c = raw.c[0];
        const float d = half_at(meta, 2 * qk + h);
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float v[8];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t byte = (wd[u] >> (8 * j)) & 0xFFu;
                v[2 * j] = __fmul_rn(small_int_f32(byte & 0xFu, 8388616.0f), d);
                v[2 * j + 1] = __fmul_rn(small_int_f32(byte >> 4, 8388616.0f), d);
            }
            out[u] = make_uint4(pack_h2(v[0], v[1], rtz), pack_h2(v[2], v[3], rtz), pack_h2(v[4], v[5], rtz),
                                pack_h2(v[6], v[7], rtz));
            pos[u] = 4 * h + u;
        }
    } else if (FMT == FMT_Q8_0) {
        // block 2qk + h = chunks 4qk + 2h, 4qk + 2h + 1 of 16 int8 codes: chunks 4h .. 4h + 3
        const float d = half_at(meta, 2 * qk + h);
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
            const uint4 c = raw.c[ch];
            const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const uint32_t u = ((wd[2 * hh + (j >> 2)] >> (8 * (j & 3))) & 0xFFu) ^ 0x80u;  // int8 + 128
                    v[j] = __fmul_rn(small_int_f32(u, 8388736.0f), d);
                }
                out[ch * 2 + hh] = make_uint4(pack_h2(v[0], v[1], rtz), pack_h2(v[2], v[3], rtz),
                                              pack_h2(v[4], v[5], rtz), pack_h2(v[6], v[7], rtz));
                pos[ch * 2 + hh] = 4 * h + ch * 2 + hh;
            }
        }
    } else {
        // pair qk, chunk 2qk + h; byte i -> element 16h + i (low nibble, sub-block
        // 2qk: chunks 2h, 2h + 1) and 32 + 16h + i (high, 2qk + 1: chunks 4 + 2h, 5 + 2h)
        const float d = f16_to_f32((uint16_t)(meta.x & 0xFFFF));
        const float dmin = f16_to_f32((uint16_t)(meta.x >> 16));
        int sc[8], mn[8];
        k_scales(meta, sc, mn);
        int scl = sc[0], mnl = mn[0], sch = sc[1], mnh = mn[1];
#pragma unroll
        for (int j = 1; j < 4; ++j)
            if (qk == j) {
                scl = sc[2 * j];
                mnl = mn[2 * j];
                sch = sc[2 * j + 1];
                mnh = mn[2 * j + 1];
            }
        const float sl = __fmul_rn((float)scl, d), ml = __fmul_rn((float)mnl, dmin);
        const float sh = __fmul_rn((float)sch, d), mh = __fmul_rn((float)mnh, dmin);
        const uint4 c = raw.c[0];
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {  // bytes 8hb .. 8hb + 7 of the chunk
            float lo[8], hi[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t byte = (wd[2 * hb + (j >> 2)] >> (8 * (j & 3))) & 0xFFu;
                lo[j] = __fsub_rn(__fmul_rn(small_int_f32(byte & 0xFu, 8388608.0f), sl), ml);
                hi[j] = __fsub_rn(__fmul_rn(small_int_f32(byte >> 4, 8388608.0f), sh), mh);
            }
            out[hb] = make_uint4(pack_h2(lo[0], lo[1], rtz), pack_h2(lo[2], lo[3], rtz), pack_h2(lo[4], lo[5], rtz),
                                 pack_h2(lo[6], lo[7], rtz));
            pos[hb] = 2 * h + hb;
            out[2 + hb] = make_uint4(pack_h2(hi[0], hi[1], rtz), pack_h2(hi[2], hi[3], rtz), pack_h2(hi[4], hi[5], rtz),
                                     pack_h2(hi[6], hi[7], rtz));
            pos[2 + hb] = 4 + 2 * h + hb;
        }
    }
}

// Epilogue of 32 accumulator columns n0 .. n0 + 31 of row m (n0 % 32 == 0).
__device__ __forceinline__ void tc_epilogue32(const TcParams& p, int64_t m, int64_t n0, const float (&v)[32]) {
    if (m >= p.m) return;
    if (p.epi == EPI_SWIGLU) {
        // W rows interleave gate/up per 16: columns n0 .. n0+15 gate, n0+16 .. n0+31 up
        const int64_t f0 = (n0 >> 5) * 16;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (2 * (f0 + j) >= p.n) break;
            const float gte = v[j], up = v[16 + j];
            const float sig = 1.0f / (1.0f + expf(-gte));
            p.y[m * p.y_ld + f0 + j] = (gte * sig) * up;
        }
        return;
    }
    if (p.epi == EPI_QKV) {
        const QkvEpi& e = p.qkv;
        const int rr = e.row0 + (int)m;
        const int pos = (e.pos_ptr ? *e.pos_ptr : e.pos_imm) + rr * e.pos_step;
        if (pos < 0 || pos >= e.max_ctx) {
            atomicExch(e.err, kErrContext);
            return;
        }
        const int64_t cache_at = (int64_t)rr * e.seq_step * e.cache_sb + (int64_t)pos * e.kd;
        const int half = e.d / 2;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            const int r = (int)(n0 + j);
            if (r >= p.n) break;
            if (r < e.qd + e.kd) {
                const int ee = r < e.qd ? r : r - e.qd;
                const int i = (ee % e.d) / 2;
                const float c = e.cs[(int64_t)pos * half + i], s = e.sn[(int64_t)pos * half + i];
                const float x0 = v[j], x1 = v[j + 1];
                const float o0 = x0 * c - x1 * s, o1 = x0 * s + x1 * c;
                if (r < e.qd) {
                    e.q[(int64_t)rr * e.qd + ee] = o0;
                    e.q[(int64_t)rr * e.qd + ee + 1] = o1;
                } else if (e.kv_f16) {
                    static_cast<__half*>(e.kc)[cache_at + ee] = __float2half(o0);
                    static_cast<__half*>(e.kc)[cache_at + ee + 1] = __float2half(o1);
                } else {
                    static_cast<float*>(e.kc)[cache_at + ee] = o0;
                    static_cast<float*>(e.kc)[cache_at + ee + 1] = o1;
                }
            } else {
                const int ee = r - e.qd - e.kd;
                if (e.kv_f16) {
                    static_cast<__half*>(e.vc)[cache_at + ee] = __float2half(v[j]);
                    static_cast<__half*>(e.vc)[cache_at + ee + 1] = __float2half(v[j + 1]);
                } else {
                    static_cast<float*>(e.vc)[cache_at + ee] = v[j];
                    static_cast<float*>(e.vc)[cache_at + ee + 1] = v[j + 1];
                }
            }
        }
        return;
    }
    float* dst = p.y + m * p.y_ld + n0;
    const bool vec = n0 + 31 < p.n && (p.y_ld % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0) &&
                     (p.epi != EPI_ADD || ((p.res_ld % 4 == 0) && (reinterpret_cast<uintptr_t>(p.res) & 15) == 0));
    if (vec) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            if (p.epi == EPI_ADD) {
                const float4 r = *reinterpret_cast<const float4*>(p.res + m * p.res_ld + n0 + j);
                o.x = r.x + o.x;
                o.y = r.y + o.y;
                o.z = r.z + o.z;
                o.w = r.w + o.w;
            }
            *reinterpret_cast<float4*>(dst + j) = o;
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (n0 + j >= p.n) break;
        float o = v[j];
        if (p.epi == EPI_ADD) o = p.res[m * p.res_ld + n0 + j] + o;
        dst[j] = o;
    }
}

// PRE: the weights were dequantised to f16 rows beforehand (wmap); the TMA
// thread brings both operands' slices in and the producer warps only run the
// epilogue.
template <int FMT, bool PRE>
__global__ void __launch_bounds__(kTcThreads, 1) qgemm_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap xmap,
                                                                  const __grid_constant__ CUtensorMap wmap) {
    extern __shared__ uint8_t tc_smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[kTcStages], aload_bar[kTcStages], empty_bar[kTcStages], done_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int failed_s;
    // 1024-byte aligned ring (the swizzle pattern follows address bits 4-9)
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // consecutive CTAs share a weight tile (x runs over the row tiles), so each
    // weight slice comes from HBM once and from L2 for the other row tiles
    const int64_t m0 = (int64_t)blockIdx.x * kTcBM, n0 = (int64_t)blockIdx.y * kTcBN;
    const int nkb = (int)((p.k + kTcBK - 1) / kTcBK);
    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mbar_init(&full_bar[s], kTcProducerWarps * 32);  // weight producers (one arrival each)
            mbar_init(&aload_bar[s], 1);                     // the activation copy (bytes)
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&done_bar, 1);
        failed_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kTcMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    if (warp < kTcProducerWarps) {
        // weight producers (PRE: idle until the epilogue): half tid % 2 of W
        // row n0 + tid / 2 of every slice
        if constexpr (!PRE) {
            const int brow = tid >> 1, bh = tid & 1;
            const int64_t wrow = n0 + brow;
            const bool live = wrow < p.n_pad;
            const bool rtz = p.rtz != 0;
            RawSlice cur{}, nxt{};
            if (live && nkb > 0) load_slice<FMT>(p, wrow, 0, bh, cur);
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kTcStages;
                if (live && kb + 1 < nkb) load_slice<FMT>(p, wrow, kb + 1, bh, nxt);  // in flight while this slice converts
                if (kb >= kTcStages && !mbar_wait_bounded(&empty_bar[s], (uint32_t)((kb / kTcStages - 1) & 1))) {
                    atomicExch(p.err, kErrGemmWait);
                    failed_s = 1;
                    break;
                }
                uint8_t* b_s = ring + (size_t)s * kTcStage + kTcATile;
                uint4 bv[4];
                int bp[4] = {4 * bh, 4 * bh + 1, 4 * bh + 2, 4 * bh + 3};
                if (live) {
                    dequant_half<FMT>(cur, kb, bh, rtz, bv, bp);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) bv[i] = make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) *reinterpret_cast<uint4*>(b_s + sw128(brow, bp[i])) = bv[i];
                // generic-proxy stores -> visible to the tensor core (async proxy)
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(&full_bar[s]);
                cur = nxt;
            }
        }
    } else if (warp == kTcTmaWarp) {
        if (lane == 0) {
            // activation slices by tensor copy
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % kTcStages;
                if (kb >= kTcStages && !mbar_wait_bounded(&empty_bar[s], (uint32_t)((kb / kTcStages - 1) & 1))) {
                    atomicExch(p.err, kErrGemmWait);
                    failed_s = 1;
                    break;
                }
                mbar_expect_tx(&aload_bar[s], (uint32_t)(PRE ? kTcATile + kTcBTile : kTcATile));
                tma_load_2d(ring + (size_t)s * kTcStage, &xmap, kb * kTcBK, (int)m0, &aload_bar[s]);
                if (PRE) tma_load_2d(ring + (size_t)s * kTcStage + kTcATile, &wmap, kb * kTcBK, (int)n0, &aload_bar[s]);
                issued = kb + 1;
            }
            // no copy may still be landing when the CTA exits
            for (int kb = issued - 1; kb >= 0 && kb >= issued - kTcStages; --kb)
                mbar_drain(&aload_bar[kb % kTcStages], (uint32_t)((kb / kTcStages) & 1));
        }
    } else if (lane == 0) {
        // MMA issuer: both 128-row halves against the same weight slice
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % kTcStages;
            if (!mbar_wait_bounded(&aload_bar[s], (uint32_t)((kb / kTcStages) & 1)) ||
                (!PRE && !mbar_wait_bounded(&full_bar[s], (uint32_t)((kb / kTcStages) & 1))) || failed_s) {
                atomicExch(p.err, kErrGemmWait);
                failed_s = 1;
                break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(ring + (size_t)s * kTcStage);
            const uint32_t b_addr = a_addr + kTcATile;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int k16 = 0; k16 < kTcBK / 16; ++k16)
                    tc_mma(tmem + (uint32_t)(h * kTcBN), umma_desc(a_addr + h * (kTcHalf * 128) + k16 * 32),
                           umma_desc(b_addr + k16 * 32), (kb | k16) != 0 ? 1u : 0u);
            tc_commit(&empty_bar[s]);
        }
        tc_commit(&done_bar);  // completes once every MMA issued above has
    }

    // epilogue: warp w owns accumulator lanes 32 (w % 4) .. + 31 of row half
    // (w / 4) % 2, columns 128 (w / 8) .. + 127
    if (warp < kTcProducerWarps) {
        // every issued MMA completes: wait for them before TMEM is read or freed
        const bool ok = mbar_drain(&done_bar, 0);
        if (!ok) atomicExch(p.err, kErrGemmWait);
        tc_fence_after();
        if (ok && !failed_s && nkb > 0) {
            const int q = warp & 3, h = (warp >> 2) & 1, cb = (warp >> 3) * (kTcBN / 2);
            const int64_t m = m0 + h * kTcHalf + q * 32 + lane;
            const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * kTcBN);
            for (int c0 = cb; c0 < cb + kTcBN / 2; c0 += 32) {
                if (n0 + c0 >= p.n) break;
                float v[32];
                float(&v0)[16] = *reinterpret_cast<float(*)[16]>(v);
                float(&v1)[16] = *reinterpret_cast<float(*)[16]>(v + 16);
                tmem_ld16(lane_addr + (uint32_t)c0, v0);
                tmem_ld16(lane_addr + (uint32_t)c0 + 16, v1);
                tc_epilogue32(p, m, n0 + c0, v);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
    }
}

// W dequantised once to f16 rows [n_pad][ld] (ld = k_pad) with the same
// arithmetic and rounding as the producer warps (load_slice, dequant_half):
// thread i takes half i % 2 of 64-column slice (i / 2) % nkb of row i / (2 nkb).
template <int FMT>
__global__ void tc_dequant_kernel(const TcParams p, __half* __restrict__ out, int64_t ld) {
    const int nkb = (int)(ld / kTcBK);
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= p.n_pad * nkb * 2) return;
    const int h = (int)(i & 1);
    const int kb = (int)((i >> 1) % nkb);
    const int64_t row = (i >> 1) / nkb;
    RawSlice raw;
    load_slice<FMT>(p, row, kb, h, raw);
    uint4 v[4];
    int pos[4];
    dequant_half<FMT>(raw, kb, h, p.rtz != 0, v, pos);
    uint4* dst = reinterpret_cast<uint4*>(out + row * ld + (int64_t)kb * kTcBK);
#pragma unroll
    for (int u = 0; u < 4; ++u) dst[pos[u]] = v[u];
}

// f32 rows -> contiguous f16 rows (the GEMM's activation operand).
__global__ void to_f16_kernel(const float* __restrict__ x, int64_t ld, int64_t rows, int64_t k, __half* __restrict__ out) {
    const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
    if (i >= rows * k) return;
    const int64_t r = i / k, c = i - r * k;
    const float* src = x + r * ld + c;
    uint32_t h[4];
    if (c + 7 < k) {
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = pack_h2(src[2 * j], src[2 * j + 1], false);
        *reinterpret_cast<uint4*>(out + i) = make_uint4(h[0], h[1], h[2], h[3]);
    } else {
        for (int j = 0; j < 8 && c + j < k; ++j) out[i + j] = __float2half_rn(src[j]);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        BC_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !ptr) fail(BEACON_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

// [rows, k] f16 with row stride ld, boxes of 64 columns x 256 rows, 128-byte swizzle.
CUtensorMap activation_map(const __half* x, int64_t rows, int64_t k, int64_t ld) {
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ld * 2) % 16) invalid("tensor-core GEMM: activations must be 16-byte aligned");
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)kTcBM};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), dims,
                                            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(BEACON_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the GEMM activations");
    return map;
}

// [n_pad, k_pad] f16 weight rows, boxes of 64 columns x 256 rows, 128-byte swizzle.
CUtensorMap weight_map(const __half* w, int64_t n_pad, int64_t k_pad) {
    if (reinterpret_cast<uintptr_t>(w) & 15) invalid("tensor-core GEMM: the f16 weight scratch must be 16-byte aligned");
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)k_pad, (cuuint64_t)n_pad};
    const cuuint64_t strides[1] = {(cuuint64_t)k_pad * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)kTcBN};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(w), dims,
                                            strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) fail(BEACON_CUDA_ERR_CUDA, "cuTensorMapEncodeTiled failed for the GEMM weights");
    return map;
}

template <int FMT>
void launch_tc_t(const TcParams& p, const CUtensorMap& map, void* w16, bool w16_ready, int64_t k_pad, cudaStream_t s) {
    dim3 grid((unsigned)((p.m + kTcBM - 1) / kTcBM), (unsigned)((p.n + kTcBN - 1) / kTcBN));
    if (w16) {
        __half* wh = static_cast<__half*>(w16);
        if (!w16_ready) {
            const int64_t threads = p.n_pad * (k_pad / kTcBK) * 2;
            tc_dequant_kernel<FMT><<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(p, wh, k_pad);
            BC_LAUNCHED("tc_dequant_kernel");
        }
        const CUtensorMap wmap = weight_map(wh, p.n_pad, k_pad);
        auto kern = qgemm_tc_kernel<FMT, true>;
        allow_max_dynamic_smem(kern);
        kern<<<grid, kTcThreads, kTcSmem, s>>>(p, map, wmap);
        BC_LAUNCHED("qgemm_tc_kernel");
        return;
    }
    auto kern = qgemm_tc_kernel<FMT, false>;
    allow_max_dynamic_smem(kern);
    kern<<<grid, kTcThreads, kTcSmem, s>>>(p, map, map);
    BC_LAUNCHED("qgemm_tc_kernel");
}

}  // namespace

bool qgemm_tc_supported(const QLayout& L) {
    return L.dtype == BEACON_CUDA_DTYPE_Q4_0 || L.dtype == BEACON_CUDA_DTYPE_Q8_0 || L.dtype == BEACON_CUDA_DTYPE_Q4_K;
}

size_t qgemm_tc_scratch_bytes(int64_t rows, int64_t k) { return (size_t)(rows * k * 2 + 256); }

size_t qgemm_tc_weight_scratch_bytes(const QLayout& L) { return (size_t)(L.n_pad * L.k_pad * 2); }

void launch_qgemm_tc(const QLayout& L, const void* w, const void* x, bool x_f16, int64_t x_ld, int64_t rows, float* y,
                     int64_t y_ld, int epi, const float* res, int64_t res_ld, bool rtz, int* err, cudaStream_t s,
                     void* x16_scratch, const QkvEpi* qkv, void* w16_scratch, bool w16_ready) {
    if (rows <= 0) return;
    if (!qgemm_tc_supported(L)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "tensor-core GEMM: unsupported block type");
    if (epi == EPI_QKV && !qkv) invalid("fused q/k/v epilogue launched without its destinations");
    if ((L.n + kTcBN - 1) / kTcBN > 65535) invalid("tensor-core GEMM: too many output columns");
    const __half* xh = static_cast<const __half*>(x);
    int64_t ld = x_ld;
    if (!x_f16 || (reinterpret_cast<uintptr_t>(x) & 15) || (x_ld * 2) % 16) {
        if (!x16_scratch) invalid("tensor-core GEMM: f32 activations need an f16 scratch");
        __half* dst = static_cast<__half*>(x16_scratch);
        if (x_f16) {
            BC_CUDA(cudaMemcpy2DAsync(dst, (size_t)L.k * 2, x, (size_t)x_ld * 2, (size_t)L.k * 2, (size_t)rows,
                                      cudaMemcpyDeviceToDevice, s));
        } else {
            const int64_t n8 = (rows * L.k + 7) / 8;
            to_f16_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(static_cast<const float*>(x), x_ld, rows, L.k, dst);
            BC_LAUNCHED("to_f16_kernel");
        }
        xh = dst;
        ld = L.k;
    }
    const CUtensorMap map = activation_map(xh, rows, L.k, ld);
    TcParams p{};
    p.w = static_cast<const uint8_t*>(w);
    p.ktiles = L.ktiles();
    p.tile_bytes = L.tile_bytes;
    p.n = L.n;
    p.n_pad = L.n_pad;
    p.k = L.k;
    p.m = (int)rows;
    p.y = y;
    p.y_ld = y_ld;
    p.res = res;
    p.res_ld = res_ld;
    p.epi = epi;
    p.rtz = rtz ? 1 : 0;
    if (qkv) p.qkv = *qkv;
    p.err = err;
    switch (L.dtype) {
        case BEACON_CUDA_DTYPE_Q4_0: return launch_tc_t<FMT_Q4_0>(p, map, w16_scratch, w16_ready, L.k_pad, s);
        case BEACON_CUDA_DTYPE_Q8_0: return launch_tc_t<FMT_Q8_0>(p, map, w16_scratch, w16_ready, L.k_pad, s);
        default: return launch_tc_t<FMT_Q4_K>(p, map, w16_scratch, w16_ready, L.k_pad, s);
    }
}

}  // namespace bc
