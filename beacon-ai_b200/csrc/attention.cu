// attention.cu -- GQA attention kernels.
//  * attention_rows: one CTA per query row, exact softmax in the reference's
//    order of operations (cpu_backend.rs:511-598, ops.rs:105-116): scores,
//    optional additive mask, optional causal -inf triangle, max-subtracted
//    exp, normalise, then sum_k p[k] * v[k] per output dim. Strided, so it
//    serves both the trait op ([B, H, S, D] tensors) and the fused runtime
//    (KV cache rows [ctx, Hkv, D]).
//  * decode_attention: split-K flash decoding over the KV cache for one new
//    token per sequence; each CTA owns one (sequence, KV head, key chunk) and
//    all query heads of that KV head, so K/V are read once per group.
#include <algorithm>

#include "attention.h"
#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "qx.cuh"
#include "attn_unit.cuh"

namespace bc {

namespace {

__device__ __forceinline__ float ldf(const void* p, int f16, int64_t i) {
    return f16 ? __half2float(static_cast<const __half*>(p)[i]) : static_cast<const float*>(p)[i];
}

__global__ void attention_rows_kernel(const AttnRowsArgs a) {
    extern __shared__ float sm[];
    float* qs = sm;              // [D]
    float* sc = sm + a.d;        // [skv]
    __shared__ float red[32];
    const int64_t row = blockIdx.x;  // over batch * heads * sq
    const int64_t sq = row % a.sq, h = (row / a.sq) % a.heads, b = row / (a.sq * a.heads);
    const int64_t kvh = h / (a.heads / a.kv_heads);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int64_t qoff = b * a.q_sb + h * a.q_sh + sq * a.q_ss;
    for (int i = tid; i < a.d; i += blockDim.x) qs[i] = ldf(a.q, a.q_f16, qoff + i);
    __syncthreads();
    const int64_t kbase = b * a.kv_sb + kvh * a.kv_sh;
    const int64_t limit = a.causal ? sq + (a.skv - a.sq) : a.skv - 1;  // last visible key
    for (int64_t k = warp; k < a.skv; k += nw) {
        float dot = 0.0f;
        const int64_t ko = kbase + k * a.kv_ss;
        for (int i = lane; i < a.d; i += 32) dot = fmaf(qs[i], ldf(a.k, a.kv_f16, ko + i), dot);
        dot = warp_sum(dot);
        if (lane == 0) {
            float s = dot * a.scale;
            if (a.mask) {
                // cpu_backend.rs:560-575: a mask shorter than sq*skv applies only
                // when its length equals skv
                int64_t row_len = a.mask_numel >= a.sq * a.skv ? a.skv : a.mask_numel;
                if (row_len == a.skv) {
                    int64_t mo = sq * a.skv + k;
                    if (mo < a.mask_numel) s += a.mask[mo];
                }
            }
            if (k > limit) s += -INFINITY;
            sc[k] = s;
        }
    }
    __syncthreads();
    float m = -INFINITY;
    for (int64_t k = tid; k < a.skv; k += blockDim.x) m = fmaxf(m, sc[k]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = -INFINITY;
    for (int i = 0; i < nw; ++i) m = fmaxf(m, red[i]);
    __syncthreads();
    float s = 0.0f;
    for (int64_t k = tid; k < a.skv; k += blockDim.x) {
        float e = expf(sc[k] - m);
        sc[k] = e;
        s += e;
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    s = 0.0f;
    for (int i = 0; i < nw; ++i) s += red[i];
    const float inv = 1.0f / s;
    for (int64_t k = tid; k < a.skv; k += blockDim.x) sc[k] *= inv;
    __syncthreads();
    const int64_t ooff = b * a.o_sb + h * a.o_sh + sq * a.o_ss;
    for (int i = tid; i < a.d; i += blockDim.x) {
        float acc = 0.0f;
        for (int64_t k = 0; k < a.skv; ++k) acc = fmaf(sc[k], ldf(a.v, a.kv_f16, kbase + k * a.kv_ss + i), acc);
        a.out[ooff + i] = acc;
    }
}

// Split-K decode attention -------------------------------------------------------
// grid: (batch * kv_heads, nsplit). 4 warps; each warp takes 32-key blocks of
// the CTA's chunk. Phase 1: lane = key, scores for the G query heads of this
// KV head. Phase 2: lanes over head dims, acc += p * v. Online softmax per
// warp, then merged across warps and written as one partial per split.
template <int D, int G, typename KV>
__global__ void __launch_bounds__(128) decode_attn_kernel(const DecodeAttnArgs a) {
    constexpr int DPL = D / 32;  // head dims per lane in phase 2
    __shared__ float qs[G][D];
    __shared__ float ps[4][G][32];
    __shared__ float wm[4][G], wl[4][G];
    __shared__ float wacc[4][G][D];
    pdl_trigger();
    pdl_wait();
    const int bk = blockIdx.x, split = blockIdx.y;
    const int b = bk / a.kv_heads, kvh = bk % a.kv_heads;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // q rows of the G heads, pre-multiplied by the softmax scale
    for (int i = tid; i < G * D; i += 128) {
        int g = i / D, dd = i % D;
        qs[g][dd] = a.q[((int64_t)b * a.heads + kvh * G + g) * D + dd] * a.scale;
    }
    __syncthreads();
    const int kv_len = max(1, min(a.max_kv, a.pos_ptr ? *a.pos_ptr + 1 : a.kv_len));
    const int chunk = ((kv_len + a.nsplit - 1) / a.nsplit + 31) / 32 * 32;
    const int64_t k0 = (int64_t)split * chunk;
    const int64_t k1 = min((int64_t)kv_len, k0 + chunk);
    const KV* kc = reinterpret_cast<const KV*>(a.k_cache) + (int64_t)b * a.cache_sb + (int64_t)kvh * D;
    const KV* vc = reinterpret_cast<const KV*>(a.v_cache) + (int64_t)b * a.cache_sb + (int64_t)kvh * D;
    const int64_t ks = (int64_t)a.kv_heads * D;  // key stride in elements
    float m[G], l[G], acc[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[g][j] = 0.0f;
    }
    for (int64_t kb = k0 + warp * 32; kb < k1; kb += 128) {
        const int64_t key = kb + lane;
        const bool valid = key < k1;
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.0f;
        if (valid) {
            const KV* kr = kc + key * ks;
#pragma unroll 4
            for (int dd = 0; dd < D; dd += 8) {
                float kf[8];
                if (sizeof(KV) == 2) {
                    uint4 raw = *reinterpret_cast<const uint4*>(kr + dd);
                    const __half2* h2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float2 f = __half22float2(h2[j]);
                        kf[2 * j] = f.x;
                        kf[2 * j + 1] = f.y;
                    }
                } else {
                    float4 x0 = *reinterpret_cast<const float4*>(kr + dd);
                    float4 x1 = *reinterpret_cast<const float4*>(kr + dd + 4);
                    kf[0] = x0.x; kf[1] = x0.y; kf[2] = x0.z; kf[3] = x0.w;
                    kf[4] = x1.x; kf[5] = x1.y; kf[6] = x1.z; kf[7] = x1.w;
                }
#pragma unroll
                for (int g = 0; g < G; ++g)
#pragma unroll
                    for (int j = 0; j < 8; ++j) s[g] = fmaf(qs[g][dd + j], kf[j], s[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float sv = valid ? s[g] : -INFINITY;
            float bm = warp_max(sv);
            float mn = fmaxf(m[g], bm);
            float corr = m[g] == -INFINITY ? 0.0f : expf(m[g] - mn);
            float p = valid ? expf(sv - mn) : 0.0f;
            l[g] = l[g] * corr + warp_sum(p);
            m[g] = mn;
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[g][j] *= corr;
            ps[warp][g][lane] = p;
        }
        __syncwarp();
        // phase 2: 8 V rows per round, all loads issued before any use
        const int nk = (int)min((int64_t)32, k1 - kb);
        for (int j0 = 0; j0 < nk; j0 += 8) {
            float vf[8][DPL];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const bool ok = j0 + u < nk;
                const KV* vr = vc + (kb + j0 + u) * ks + lane * DPL;
                if (sizeof(KV) == 2) {
#pragma unroll
                    for (int t = 0; t < DPL; t += 2) {
                        float2 f = ok ? __half22float2(*reinterpret_cast<const __half2*>(vr + t)) : make_float2(0.f, 0.f);
                        vf[u][t] = f.x;
                        vf[u][t + 1] = f.y;
                    }
                } else {
#pragma unroll
                    for (int t = 0; t < DPL; ++t) vf[u][t] = ok ? reinterpret_cast<const float*>(vr)[t] : 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float p = (j0 + u < nk) ? ps[warp][g][j0 + u] : 0.0f;
#pragma unroll
                    for (int t = 0; t < DPL; ++t) acc[g][t] = fmaf(p, vf[u][t], acc[g][t]);
                }
            }
        }
        __syncwarp();
    }
    // merge the 4 warps
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
#pragma unroll
        for (int t = 0; t < DPL; ++t) wacc[warp][g][lane * DPL + t] = acc[g][t];
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += 128) {
        const int g = i / D, dd = i % D;
        float M = -INFINITY;
        for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.0f, o = 0.0f;
        for (int w = 0; w < 4; ++w) {
            float c = wm[w][g] == -INFINITY ? 0.0f : expf(wm[w][g] - M);
            L += wl[w][g] * c;
            o += wacc[w][g][dd] * c;
        }
        const int64_t hb = ((int64_t)b * a.heads + kvh * G + g);
        a.part_acc[(hb * a.nsplit + split) * D + dd] = o;
        if (dd == 0) {
            a.part_m[hb * a.nsplit + split] = M;
            a.part_l[hb * a.nsplit + split] = L;
        }
    }
}

// One CTA (d threads) per (sequence, head): the split weights exp(m_s - M)
// are computed once in shared memory, then every thread sums its head dim
// over the splits with all loads independent.
__global__ void decode_attn_combine_kernel(const DecodeAttnArgs a, int d) {
    __shared__ float wsh[kMaxDecodeSplits];
    __shared__ float inv_l;
    pdl_trigger();
    pdl_wait();
    const int64_t hb = blockIdx.x;
    const int tid = threadIdx.x, ns = a.nsplit;
    const float* pm = a.part_m + hb * ns;
    const float* pl = a.part_l + hb * ns;
    if (tid < 32) {
        float M = -INFINITY;
        for (int s = tid; s < ns; s += 32) M = fmaxf(M, pm[s]);
        M = warp_max(M);
        float L = 0.0f;
        for (int s = tid; s < ns; s += 32) {
            const float mm = pm[s];
            const float wgt = mm == -INFINITY ? 0.0f : expf(mm - M);
            wsh[s] = wgt;
            L += pl[s] * wgt;
        }
        L = warp_sum(L);
        if (tid == 0) inv_l = 1.0f / L;
    }
    __syncthreads();
    const float* acc = a.part_acc + hb * ns * d;
    for (int dd = tid; dd < d; dd += blockDim.x) {
        float o = 0.0f;
#pragma unroll 8
        for (int s = 0; s < ns; ++s) o = fmaf(acc[(int64_t)s * d + dd], wsh[s], o);
        a.out[hb * d + dd] = o * inv_l;
    }
}

// Prefill attention, tiled -----------------------------------------------------------
// One CTA (8 warps) per (tile of 128/G query rows, KV head): the G query heads
// of the KV head make 128 (row, head) pairs that share every key/value tile
// staged in shared memory (64 keys at a time), so each K/V row is read once
// per CTA instead of once per query. Scores: thread t owns pairs 4(t/8) ..
// +3 and keys 8(t%8) .. +7 of a tile; the online softmax (engine.rs:415-440
// semantics: max-subtracted exp, normalised at the end) reduces over the 8
// threads of a pair group with shuffles; the same thread then owns those
// pairs' outputs for dims (t%8) D/8 .. +D/8, so the rescale stays local.
// f32 arithmetic; used for prefill in the fast numerics over f32 caches (f16
// caches take the tensor-core kernel below; the row kernel above keeps the
// reference's summation order for the exact numerics).
constexpr int kPfKeys = 64;
constexpr int kPfPairs = 128;
constexpr int kPfThreads = 256;

template <int D>
struct PfLayout {
    static constexpr int kT = kPfKeys + 4;   // transposed key tile row (padded): [D][kT]
    static constexpr int q = D * kPfPairs;   // qsT [D][pairs]
    static constexpr int k = D * kT;         // ksT [D][kT]
    static constexpr int v = kPfKeys * D;    // vs  [keys][D]
    static constexpr int p = kPfKeys * kPfPairs;  // psT [keys][pairs]
    static constexpr size_t bytes = (size_t)(q + k + v + p) * 4;
};

template <int D, int G, typename KV>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_attn_kernel(const AttnRowsArgs a) {
    using Lay = PfLayout<D>;
    constexpr int RT = kPfPairs / G;  // query rows per CTA
    constexpr int DPT = D / 8;        // output dims per thread
    extern __shared__ __align__(16) float pf_smem[];
    float* qsT = pf_smem;
    float* ksT = qsT + Lay::q;
    float* vs = ksT + Lay::k;
    float* psT = vs + Lay::v;
    const int tid = threadIdx.x;
    const int kvh = blockIdx.y;
    const int64_t r0 = (int64_t)blockIdx.x * RT;
    const int pg = tid >> 3, kg = tid & 7;  // pair group (4 pairs), key / dim group
    // q tile, pre-scaled, transposed: qsT[d][pair], pair = row * G + g
    for (int i = tid; i < kPfPairs * D; i += kPfThreads) {
        const int pr = i / D, d = i - pr * D;
        const int64_t row = r0 + pr / G;
        const int h = kvh * G + pr % G;
        float v = 0.0f;
        if (row < a.sq) v = reinterpret_cast<const float*>(a.q)[h * a.q_sh + row * a.q_ss + d] * a.scale;
        qsT[d * kPfPairs + pr] = v;
    }
    float m[4], l[4], acc[4][DPT];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        m[j] = -INFINITY;
        l[j] = 0.0f;
#pragma unroll
        for (int e = 0; e < DPT; ++e) acc[j][e] = 0.0f;
    }
    // keys [0, skv); causal: row s sees keys <= skv - sq + s
    const int64_t last_row = min((int64_t)a.sq - 1, r0 + RT - 1);
    const int64_t kend = a.causal ? min((int64_t)a.skv, a.skv - a.sq + last_row + 1) : (int64_t)a.skv;
    const KV* kbase = reinterpret_cast<const KV*>(a.k) + (int64_t)kvh * a.kv_sh;
    const KV* vbase = reinterpret_cast<const KV*>(a.v) + (int64_t)kvh * a.kv_sh;
    for (int64_t k0 = 0; k0 < kend; k0 += kPfKeys) {
        __syncthreads();  // previous tile fully consumed
        for (int i = tid; i < kPfKeys * D; i += kPfThreads) {
            const int kk = i / D, d = i - kk * D;
            const int64_t key = k0 + kk;
            float kv = 0.0f, vv = 0.0f;
            if (key < kend) {
                if (sizeof(KV) == 2) {
                    kv = __half2float(reinterpret_cast<const __half*>(kbase)[key * a.kv_ss + d]);
                    vv = __half2float(reinterpret_cast<const __half*>(vbase)[key * a.kv_ss + d]);
                } else {
                    kv = reinterpret_cast<const float*>(kbase)[key * a.kv_ss + d];
                    vv = reinterpret_cast<const float*>(vbase)[key * a.kv_ss + d];
                }
            }
            ksT[d * Lay::kT + kk] = kv;
            vs[kk * D + d] = vv;
        }
        __syncthreads();
        // scores s[4 pairs][8 keys]
        float s[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 8; ++e) s[j][e] = 0.0f;
#pragma unroll 4
        for (int d = 0; d < D; ++d) {
            const float4 q4 = *reinterpret_cast<const float4*>(qsT + d * kPfPairs + pg * 4);
            const float4 ka = *reinterpret_cast<const float4*>(ksT + d * Lay::kT + kg * 8);
            const float4 kb = *reinterpret_cast<const float4*>(ksT + d * Lay::kT + kg * 8 + 4);
            const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
            const float kv8[8] = {ka.x, ka.y, ka.z, ka.w, kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int e = 0; e < 8; ++e) s[j][e] = fmaf(qv[j], kv8[e], s[j][e]);
        }
        // mask, online softmax over the 8 threads of the pair group
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int pr = pg * 4 + j;
            const int64_t row = r0 + pr / G;
            const int64_t lim = a.causal ? (int64_t)a.skv - a.sq + row : (int64_t)a.skv - 1;  // last visible key
            float mx = -INFINITY;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int64_t key = k0 + kg * 8 + e;
                if (key > lim || key >= kend) s[j][e] = -INFINITY;
                mx = fmaxf(mx, s[j][e]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            const float mn = fmaxf(m[j], mx);
            const float c = (m[j] == -INFINITY) ? 0.0f : expf(m[j] - mn);
            float sum = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float pv = mn == -INFINITY ? 0.0f : expf(s[j][e] - mn);
                s[j][e] = pv;
                sum += pv;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            l[j] = l[j] * c + sum;
            m[j] = mn;
#pragma unroll
            for (int e = 0; e < DPT; ++e) acc[j][e] *= c;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e)
            *reinterpret_cast<float4*>(psT + (kg * 8 + e) * kPfPairs + pg * 4) =
                make_float4(s[0][e], s[1][e], s[2][e], s[3][e]);
        __syncthreads();
        // acc[4 pairs][DPT dims] += P V
        const int kn = (int)min((int64_t)kPfKeys, kend - k0);
        for (int kk = 0; kk < kn; ++kk) {
            const float4 p4 = *reinterpret_cast<const float4*>(psT + kk * kPfPairs + pg * 4);
            const float pv[4] = {p4.x, p4.y, p4.z, p4.w};
            float vv[DPT];
#pragma unroll
            for (int e = 0; e < DPT; e += 4) {
                const float4 t4 = *reinterpret_cast<const float4*>(vs + kk * D + kg * DPT + e);
                vv[e] = t4.x;
                vv[e + 1] = t4.y;
                vv[e + 2] = t4.z;
                vv[e + 3] = t4.w;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int e = 0; e < DPT; ++e) acc[j][e] = fmaf(pv[j], vv[e], acc[j][e]);
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int pr = pg * 4 + j;
        const int64_t row = r0 + pr / G;
        if (row >= a.sq) continue;
        const int h = kvh * G + pr % G;
        const float inv = l[j] > 0.0f ? 1.0f / l[j] : 0.0f;
        float* o = a.out + h * a.o_sh + row * a.o_ss + kg * DPT;
#pragma unroll
        for (int e = 0; e < DPT; e += 4)
            *reinterpret_cast<float4*>(o + e) =
                make_float4(acc[j][e] * inv, acc[j][e + 1] * inv, acc[j][e + 2] * inv, acc[j][e + 3] * inv);
    }
}

// Prefill attention on the tensor cores (fast numerics, f16 caches) ----------------
// Same work split as prefill_attn_kernel: one CTA (8 warps) per (128/G query
// rows, KV head); warp w owns the 16 (row, head) pairs 16w .. 16w+15 (pair =
// row * G + head) as the M dimension of m16n8k16 f16 MMAs with f32
// accumulation. Key/value tiles of 64 keys are double-buffered in shared
// memory by 16-byte asynchronous copies at swizzled positions (chunk ^ (row &
// 7), conflict-free ldmatrix). Scores S = Q K^T with the pre-scaled query in
// registers as f16 high and low parts (two MMAs, ~22-bit query precision),
// pre-scaled by log2(e) so the softmax exponentials are exp2; online softmax
// on the accumulator fragments (row max and sum over the 4 lanes of a row;
// the causal / end-of-keys mask only on the tiles that cross a row's last
// visible key); P rounded to f16 is re-packed in registers as the A
// operand of O += P V, V^T fragments from transposing ldmatrix. The causal CTAs
// are launched heaviest (latest query rows) first.
constexpr int kPtKeys = 64;

template <int D>
struct PtLayout {
    static constexpr int row = 2 * D;                 // bytes of one key or value row
    static constexpr int stage = 2 * kPtKeys * row;   // keys, then values
    static constexpr size_t smem = 2 * (size_t)stage;  // two stages
};

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int D, int G>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_attn_tc_kernel(const AttnRowsArgs a) {
    using Lay = PtLayout<D>;
    constexpr int RT = kPfPairs / G;  // query rows per CTA
    constexpr int KS = D / 16;        // 16-dim k-steps of the scores
    constexpr int NT = kPtKeys / 8;   // 8-key n-tiles of the scores
    constexpr int ND = D / 8;         // 8-dim n-tiles of the output
    constexpr int CPR = D / 8;        // 16-byte chunks per row
    extern __shared__ __align__(128) uint8_t pt_smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int kvh = blockIdx.y;
    const int64_t r0 = (int64_t)(gridDim.x - 1 - blockIdx.x) * RT;  // heaviest tiles first
    // the two pairs of this thread's fragment rows
    const int pa = warp * 16 + g, pb = pa + 8;
    const int64_t row_a = r0 + pa / G, row_b = r0 + pb / G;
    const int ha = kvh * G + pa % G, hb = kvh * G + pb % G;
    // query fragments (A operand, 16 pairs x 16 dims per k-step), pre-scaled,
    // as f16 high and low parts: regs (pair a, dims 2t..), (pair b, 2t..),
    // (pair a, 8 + 2t..), (pair b, 8 + 2t..)
    uint32_t qh[KS][4], ql[KS][4];
    const float qscale = a.scale * 1.4426950408889634f;  // scores in log2 units: softmax by exp2
    {
        const float* q = reinterpret_cast<const float*>(a.q);
#pragma unroll
        for (int j = 0; j < KS; ++j)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const bool second = r & 1;
                const int64_t row = second ? row_b : row_a;
                const int h = second ? hb : ha;
                const int d = 16 * j + 2 * t + (r >> 1) * 8;
                float x0 = 0.0f, x1 = 0.0f;
                if (row < a.sq) {
                    const float* qp = q + h * a.q_sh + row * a.q_ss + d;
                    x0 = qp[0] * qscale;
                    x1 = qp[1] * qscale;
                }
                const __half2 hh = __floats2half2_rn(x0, x1);
                const float2 hf = __half22float2(hh);
                qh[j][r] = *reinterpret_cast<const uint32_t*>(&hh);
                ql[j][r] = pack_f16x2(x0 - hf.x, x1 - hf.y);
            }
    }
    // keys [0, skv); causal: row s sees keys <= skv - sq + s
    const int64_t last_row = min((int64_t)a.sq - 1, r0 + RT - 1);
    const int64_t kend = a.causal ? min((int64_t)a.skv, a.skv - a.sq + last_row + 1) : (int64_t)a.skv;
    // last visible key of each fragment row, also bounded by the keys there are
    // (keys and rows fit 32 bits: the cache is at most 2^31 rows)
    const int lim_a = (int)min(kend - 1, a.causal ? (int64_t)a.skv - a.sq + row_a : (int64_t)a.skv - 1);
    const int lim_b = (int)min(kend - 1, a.causal ? (int64_t)a.skv - a.sq + row_b : (int64_t)a.skv - 1);
    const __half* kc = reinterpret_cast<const __half*>(a.k) + (int64_t)kvh * a.kv_sh;
    const __half* vc = reinterpret_cast<const __half*>(a.v) + (int64_t)kvh * a.kv_sh;
    const int ntiles = (int)((kend + kPtKeys - 1) / kPtKeys);
    auto issue = [&](int it) {
        uint8_t* base = pt_smem + (size_t)(it & 1) * Lay::stage;
        const int64_t k0 = (int64_t)it * kPtKeys;
        for (int c = tid; c < 2 * kPtKeys * CPR; c += kPfThreads) {
            const int rw = c / CPR, part = c - rw * CPR;
            const int r = rw & (kPtKeys - 1);
            const int64_t key = k0 + r;
            uint8_t* dst = base + (rw < kPtKeys ? 0 : kPtKeys * Lay::row) + tc_swz(r, part, Lay::row);
            if (key < kend)
                cp_async16(dst, (rw < kPtKeys ? kc : vc) + key * a.kv_ss + part * 8);
            else
                *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);  // past the keys: finite zeros
        }
        cp_async_commit();
    };
    float o[ND][4];
#pragma unroll
    for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
    const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: the matrix this lane addresses, its row
    if (ntiles > 0) issue(0);
    for (int it = 0; it < ntiles; ++it) {
        if (it + 1 < ntiles) {
            issue(it + 1);
            cp_async_wait_group<1>();
        } else {
            cp_async_wait_group<0>();
        }
        __syncthreads();  // every thread's copies of tile it have landed
        const uint32_t kb = smem_u32(pt_smem + (size_t)(it & 1) * Lay::stage);
        const uint32_t vb = kb + kPtKeys * Lay::row;
        const int64_t k0 = (int64_t)it * kPtKeys;
        // scores: s[n] = pairs (a, b) x keys k0 + 8n + 2t, +1
        float sc[NT][4];
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
            for (int j = 0; j < KS; j += 2) {
                uint32_t b0, b1, b2, b3;  // k-step j: (b0, b1); k-step j + 1: (b2, b3)
                ldsm_x4(kb + tc_swz(8 * n + rr, 2 * j + mi, Lay::row), b0, b1, b2, b3);
                mma_f16(sc[n], qh[j][0], qh[j][1], qh[j][2], qh[j][3], b0, b1);
                mma_f16(sc[n], ql[j][0], ql[j][1], ql[j][2], ql[j][3], b0, b1);
                mma_f16(sc[n], qh[j + 1][0], qh[j + 1][1], qh[j + 1][2], qh[j + 1][3], b2, b3);
                mma_f16(sc[n], ql[j + 1][0], ql[j + 1][1], ql[j + 1][2], ql[j + 1][3], b2, b3);
            }
        }
        // mask (tiles crossing a row's last visible key) and online softmax
        // (rows a: sc[.][0..1], b: sc[.][2..3])
        const int kt0 = (int)k0;
        if (kt0 + kPtKeys - 1 > min(lim_a, lim_b)) {
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int key = kt0 + 8 * n + 2 * t + e;
                    if (key > lim_a) sc[n][e] = -INFINITY;
                    if (key > lim_b) sc[n][2 + e] = -INFINITY;
                }
        }
        float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            mx_a = fmaxf(mx_a, fmaxf(sc[n][0], sc[n][1]));
            mx_b = fmaxf(mx_b, fmaxf(sc[n][2], sc[n][3]));
        }
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        const float c_a = m_a == -INFINITY ? 0.0f : exp2f(m_a - mn_a);
        const float c_b = m_b == -INFINITY ? 0.0f : exp2f(m_b - mn_b);
        // a row with no visible key yet keeps max -inf: its exponentials are 0
        const float sa = mn_a == -INFINITY ? 0.0f : mn_a, sb = mn_b == -INFINITY ? 0.0f : mn_b;
        float su_a = 0.0f, su_b = 0.0f;
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                sc[n][e] = exp2f(sc[n][e] - sa);  // exp2(-inf) = 0 for masked keys
                sc[n][2 + e] = exp2f(sc[n][2 + e] - sb);
                su_a += sc[n][e];
                su_b += sc[n][2 + e];
            }
        su_a += __shfl_xor_sync(0xffffffffu, su_a, 1);
        su_a += __shfl_xor_sync(0xffffffffu, su_a, 2);
        su_b += __shfl_xor_sync(0xffffffffu, su_b, 1);
        su_b += __shfl_xor_sync(0xffffffffu, su_b, 2);
        l_a = l_a * c_a + su_a;
        l_b = l_b * c_b + su_b;
        m_a = mn_a;
        m_b = mn_b;
#pragma unroll
        for (int n = 0; n < ND; ++n) {
            o[n][0] *= c_a;
            o[n][1] *= c_a;
            o[n][2] *= c_b;
            o[n][3] *= c_b;
        }
        // O += P V: P (16 pairs x 16 keys per k-step) from the score fragments
#pragma unroll
        for (int kk = 0; kk < kPtKeys / 16; ++kk) {
            const uint32_t p0 = pack_f16x2(sc[2 * kk][0], sc[2 * kk][1]);
            const uint32_t p1 = pack_f16x2(sc[2 * kk][2], sc[2 * kk][3]);
            const uint32_t p2 = pack_f16x2(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
            const uint32_t p3 = pack_f16x2(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
            for (int n = 0; n < ND; n += 2) {
                uint32_t b0, b1, b2, b3;  // dims 8n..: (b0, b1); dims 8(n+1)..: (b2, b3)
                ldsm_x4_t(vb + tc_swz(16 * kk + (mi & 1) * 8 + rr, n + (mi >> 1), Lay::row), b0, b1, b2, b3);
                mma_f16(o[n], p0, p1, p2, p3, b0, b1);
                mma_f16(o[n + 1], p0, p1, p2, p3, b2, b3);
            }
        }
        __syncthreads();  // every warp is done with this stage before it is refilled
    }
    const float inv_a = l_a > 0.0f ? 1.0f / l_a : 0.0f, inv_b = l_b > 0.0f ? 1.0f / l_b : 0.0f;
#pragma unroll
    for (int n = 0; n < ND; ++n) {
        const int d = 8 * n + 2 * t;
        __half* o16 = static_cast<__half*>(a.out16);
        if (row_a < a.sq) {
            const float2 r = make_float2(o[n][0] * inv_a, o[n][1] * inv_a);
            *reinterpret_cast<float2*>(a.out + ha * a.o_sh + row_a * a.o_ss + d) = r;
            if (o16) *reinterpret_cast<__half2*>(o16 + ha * a.o_sh + row_a * a.o_ss + d) = __floats2half2_rn(r.x, r.y);
        }
        if (row_b < a.sq) {
            const float2 r = make_float2(o[n][2] * inv_b, o[n][3] * inv_b);
            *reinterpret_cast<float2*>(a.out + hb * a.o_sh + row_b * a.o_ss + d) = r;
            if (o16) *reinterpret_cast<__half2*>(o16 + hb * a.o_sh + row_b * a.o_ss + d) = __floats2half2_rn(r.x, r.y);
        }
    }
}

template <int D, int G>
bool launch_prefill_t(const AttnRowsArgs& a, cudaStream_t s) {
    constexpr int RT = kPfPairs / G;
    dim3 grid((unsigned)((a.sq + RT - 1) / RT), (unsigned)a.kv_heads);
    if (a.kv_f16 && a.kv_ss % 8 == 0 && a.kv_sh % 8 == 0 && a.q_ss % 2 == 0 && a.q_sh % 2 == 0 &&
        a.o_ss % 2 == 0 && a.o_sh % 2 == 0) {  // 16-byte cache rows, paired q / out elements
        BC_CUDA(cudaFuncSetAttribute(prefill_attn_tc_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)PtLayout<D>::smem));
        prefill_attn_tc_kernel<D, G><<<grid, kPfThreads, PtLayout<D>::smem, s>>>(a);
        BC_LAUNCHED("prefill_attn_tc_kernel");
        return a.out16 != nullptr;
    }
    if (a.kv_f16) {
        allow_max_dynamic_smem(prefill_attn_kernel<D, G, __half>);
        prefill_attn_kernel<D, G, __half><<<grid, kPfThreads, PfLayout<D>::bytes, s>>>(a);
    } else {
        allow_max_dynamic_smem(prefill_attn_kernel<D, G, float>);
        prefill_attn_kernel<D, G, float><<<grid, kPfThreads, PfLayout<D>::bytes, s>>>(a);
    }
    BC_LAUNCHED("prefill_attn_kernel");
    return false;
}

template <int D, int G>
__global__ void __launch_bounds__(kAttThreads, 2) decode_attn_bulk_kernel(const DecodeAttnArgs a) {
    extern __shared__ __align__(128) uint8_t att_smem[];
    __shared__ __align__(8) uint64_t bars[kAttStages];
    attn_unit<D, G, kAttStages>(a, blockIdx.x, blockIdx.y, att_smem, bars, [] {
        pdl_trigger();
        pdl_wait();
    });
}

template <int D, int G>
__global__ void __launch_bounds__(kAttThreads, 2) decode_attn_tc_kernel(const DecodeAttnArgs a) {
    extern __shared__ __align__(128) uint8_t att_smem[];
    __shared__ __align__(8) uint64_t bars[kTcStages];
    attn_unit_tc<D, G>(a, blockIdx.x, blockIdx.y, att_smem, bars, [] {
        pdl_trigger();
        pdl_wait();
    });
}

template <int D, int G>
void launch_decode_tc_t(const DecodeAttnArgs& a, cudaStream_t s, bool pdl) {
    auto kern = decode_attn_tc_kernel<D, G>;
    BC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TcLayout<D>::smem));
    dim3 grid((unsigned)(a.batch * a.kv_heads), (unsigned)a.nsplit);
    launch_kernel(kern, grid, dim3(kAttThreads), TcLayout<D>::smem, s, pdl, a);
}

template <int D, int G>
void launch_decode_bulk_t(const DecodeAttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.tc) return launch_decode_tc_t<D, G>(a, s, pdl);
    auto kern = decode_attn_bulk_kernel<D, G>;
    BC_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AttLayout<D>::smem));
    dim3 grid((unsigned)(a.batch * a.kv_heads), (unsigned)a.nsplit);
    launch_kernel(kern, grid, dim3(kAttThreads), AttLayout<D>::smem, s, pdl, a);
    BC_LAUNCHED("decode_attn_bulk_kernel");
}

template <int D, int G>
void launch_decode_t(const DecodeAttnArgs& a, cudaStream_t s, bool pdl) {
    dim3 grid((unsigned)(a.batch * a.kv_heads), (unsigned)a.nsplit);
    if (a.kv_f16)
        launch_kernel(decode_attn_kernel<D, G, __half>, grid, dim3(128), 0, s, pdl, a);
    else
        launch_kernel(decode_attn_kernel<D, G, float>, grid, dim3(128), 0, s, pdl, a);
    BC_LAUNCHED("decode_attn_kernel");
}

}  // namespace

void launch_attention_rows(const AttnRowsArgs& a, cudaStream_t s) {
    const int64_t rows = a.batch * a.heads * a.sq;
    if (rows == 0 || a.skv == 0) return;
    const size_t smem = (size_t)(a.d + a.skv) * sizeof(float);
    if (smem > 200 * 1024) shape_err("attention: key length too long for the single-row kernel");
    if (smem > 48 * 1024)
        allow_max_dynamic_smem(attention_rows_kernel);
    attention_rows_kernel<<<(unsigned)rows, 128, smem, s>>>(a);
    BC_LAUNCHED("attention_rows_kernel");
}

int plan_decode_splits(int batch, int kv_heads, int kv_len, int sm_count, int max_splits) {
    const int64_t want = 2LL * sm_count;
    int64_t per = std::max<int64_t>(1, (int64_t)batch * kv_heads);
    int64_t ns = (want + per - 1) / per;
    ns = std::min<int64_t>(ns, (kv_len + 127) / 128);  // at least 128 keys (one per lane-warp pass) each
    ns = std::max<int64_t>(1, std::min<int64_t>(ns, max_splits));
    return (int)ns;
}

bool decode_attention_supported(int head_dim, int group) {
    return (head_dim == 64 || head_dim == 128) && (group == 1 || group == 2 || group == 4 || group == 8);
}

bool prefill_attention_supported(const AttnRowsArgs& a) {
    const int64_t G = a.kv_heads > 0 ? a.heads / a.kv_heads : 0;
    return a.batch == 1 && !a.mask && a.q_f16 == 0 && (a.d == 64 || a.d == 128) &&
           (G == 1 || G == 2 || G == 4 || G == 8) && a.heads == G * a.kv_heads && a.q_ss % 4 == 0 &&
           a.o_ss % 4 == 0 && a.o_sh % 4 == 0;
}

bool launch_prefill_attention(const AttnRowsArgs& a, cudaStream_t s) {
    if (a.sq == 0 || a.skv == 0) return false;
    if (!prefill_attention_supported(a)) invalid("prefill attention: unsupported layout");
    const int G = (int)(a.heads / a.kv_heads);
    if (a.d == 128) {
        if (G == 8) return launch_prefill_t<128, 8>(a, s);
        if (G == 4) return launch_prefill_t<128, 4>(a, s);
        if (G == 2) return launch_prefill_t<128, 2>(a, s);
        return launch_prefill_t<128, 1>(a, s);
    }
    if (G == 8) return launch_prefill_t<64, 8>(a, s);
    if (G == 4) return launch_prefill_t<64, 4>(a, s);
    if (G == 2) return launch_prefill_t<64, 2>(a, s);
    return launch_prefill_t<64, 1>(a, s);
}

int decode_bulk_splits(int batch, int kv_heads, int sm_count) {
    const int64_t per = std::max<int64_t>(1, (int64_t)batch * kv_heads);
    return (int)std::max<int64_t>(1, std::min<int64_t>(kMaxBulkSplits, sm_count / per));
}

size_t decode_bulk_scratch_floats(int max_batch, int heads, int kv_heads, int d, int sm_count) {
    const int64_t g = heads / std::max(1, kv_heads);
    const int64_t units = std::max<int64_t>((int64_t)sm_count, (int64_t)max_batch * kv_heads) +
                          (int64_t)max_batch * kv_heads;  // + one split of slack per (sequence, KV head)
    return (size_t)(g * units * (d + 2));
}

void launch_decode_attention(DecodeAttnArgs a, cudaStream_t s, bool pdl) {
    const int G = a.heads / a.kv_heads;
    if (!decode_attention_supported(a.d, G)) fail(BEACON_CUDA_ERR_SHAPE_MISMATCH, "decode attention: unsupported head shape");
    if (a.kv_f16 && a.counters && a.err) {
        if (a.nsplit < 1 || a.nsplit > kMaxBulkSplits) invalid("decode attention: bad split count");
        if (a.d == 128) {
            if (G == 8) return launch_decode_bulk_t<128, 8>(a, s, pdl);
            if (G == 4) return launch_decode_bulk_t<128, 4>(a, s, pdl);
            if (G == 2) return launch_decode_bulk_t<128, 2>(a, s, pdl);
            return launch_decode_bulk_t<128, 1>(a, s, pdl);
        }
        if (G == 8) return launch_decode_bulk_t<64, 8>(a, s, pdl);
        if (G == 4) return launch_decode_bulk_t<64, 4>(a, s, pdl);
        if (G == 2) return launch_decode_bulk_t<64, 2>(a, s, pdl);
        return launch_decode_bulk_t<64, 1>(a, s, pdl);
    }
    if (a.nsplit < 1 || a.nsplit > kMaxDecodeSplits) invalid("decode attention: bad split count");
    if (a.d == 128) {
        if (G == 8) launch_decode_t<128, 8>(a, s, pdl);
        else if (G == 4) launch_decode_t<128, 4>(a, s, pdl);
        else if (G == 2) launch_decode_t<128, 2>(a, s, pdl);
        else launch_decode_t<128, 1>(a, s, pdl);
    } else {
        if (G == 8) launch_decode_t<64, 8>(a, s, pdl);
        else if (G == 4) launch_decode_t<64, 4>(a, s, pdl);
        else if (G == 2) launch_decode_t<64, 2>(a, s, pdl);
        else launch_decode_t<64, 1>(a, s, pdl);
    }
    launch_kernel(decode_attn_combine_kernel, dim3((unsigned)((int64_t)a.batch * a.heads)), dim3(a.d), 0, s, pdl, a,
                  (int)a.d);
    BC_LAUNCHED("decode_attn_combine_kernel");
}

}  // namespace bc

using namespace bc;

extern "C" int32_t beacon_cuda_op_attention(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                            const BeaconCudaTensor* q, const BeaconCudaTensor* k,
                                            const BeaconCudaTensor* v, const BeaconCudaTensor* mask, float scale,
                                            int32_t causal, BeaconCudaTensor** out) {
    return guard([&]() -> int32_t {
        require(ctx && stream && q && k && v && out, "attention: null argument");
        set_device(ctx);
        if (q->shape.size() != 4 || k->shape.size() != 4 || v->shape.size() != 4)
            shape_err("attention: q/k/v must be 4-D");  // cpu_backend.rs:518-522
        auto isf = [](const BeaconCudaTensor* t) {
            return t->dtype == BEACON_CUDA_DTYPE_F32 || t->dtype == BEACON_CUDA_DTYPE_F16;
        };
        if (!isf(q) || !isf(k) || !isf(v) || k->dtype != v->dtype)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "attention: q/k/v must be F32 or F16 (k and v alike)");
        const int64_t B = q->shape[0], H = q->shape[1], Sq = q->shape[2], D = q->shape[3];
        const int64_t Hkv = k->shape[1], Skv = k->shape[2];
        if (k->shape != v->shape || k->shape[0] != B || k->shape[3] != D) shape_err("attention: k/v shape mismatch");
        if (Hkv == 0 || H % Hkv) shape_err("attention: n_heads must be divisible by n_kv_heads");
        if (mask && mask->dtype != BEACON_CUDA_DTYPE_F32) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "attention: mask must be F32");
        if (causal < -1 || causal > 1) invalid("attention: causal must be -1, 0 or 1");
        const bool use_causal = causal == 1 || (causal == -1 && !mask && Sq > 1);
        if (use_causal && Skv < Sq) shape_err("attention: causal needs at least as many keys as queries");
        BeaconCudaTensor* o = new_tensor(ctx, q->shape, BEACON_CUDA_DTYPE_F32);
        try {
            AttnRowsArgs a{};
            a.q = q->data();
            a.q_f16 = q->dtype == BEACON_CUDA_DTYPE_F16;
            a.k = k->data();
            a.v = v->data();
            a.kv_f16 = k->dtype == BEACON_CUDA_DTYPE_F16;
            a.out = static_cast<float*>(o->data());
            a.mask = mask ? static_cast<const float*>(mask->data()) : nullptr;
            a.mask_numel = mask ? mask->numel() : 0;
            a.batch = B;
            a.heads = H;
            a.kv_heads = Hkv;
            a.sq = Sq;
            a.skv = Skv;
            a.d = (int)D;
            a.scale = scale;
            a.causal = use_causal ? 1 : 0;
            a.q_sb = H * Sq * D;
            a.q_sh = Sq * D;
            a.q_ss = D;
            a.kv_sb = Hkv * Skv * D;
            a.kv_sh = Skv * D;
            a.kv_ss = D;
            a.o_sb = H * Sq * D;
            a.o_sh = Sq * D;
            a.o_ss = D;
            launch_attention_rows(a, stream->s);
        } catch (...) {
            delete o;
            throw;
        }
        *out = o;
        return BEACON_CUDA_OK;
    });
}
