// attn_unit.cuh -- one unit of split-K decode attention over an f16 KV cache
// on a whole CTA, shared by the decode attention kernel (attention.cu) and the
// fused decode step (decode_mega.cu).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "attention.h"
#include "common.cuh"
#include "qx.cuh"

namespace bc {

// Decode attention over an f16 KV cache ------------------------------------------
// One CTA (8 warps) per (sequence, KV head, split of the keys). The split's
// key and value rows are staged in shared memory with 16-byte asynchronous
// copies, 64 keys per stage in a ring of up to 4 stages whose completion is
// tracked by one mbarrier per stage. Every row except the decoded token's
// (written by the previous kernel) is requested before the kernel waits on its
// predecessor, so the cache stream overlaps the preceding GEMV.
// Scores: lane l holds head dims [l*DPL, l*DPL+DPL) of all G query heads in
// registers; a warp takes 32/G keys at a time and a transposing butterfly
// (31 shuffles) leaves lane l with the full dot product of (key l/G, head
// l%G). Values: lanes over head dims, warps over keys, with an online softmax
// across stages (engine.rs:415-440). The splits of a (sequence, KV head) are
// merged in split order by the last of its CTAs to finish (arrival counter),
// so no separate combine kernel runs.
constexpr int kAttKeys = 64;
constexpr int kAttStages = 4;
constexpr int kAttThreads = 256;
constexpr int kAttWarps = kAttThreads / 32;

template <int D>
struct AttLayout {
    static constexpr int row = 2 * D;                      // bytes of one key or value row
    static constexpr int stage = 2 * kAttKeys * row;       // keys, then values
    static constexpr int chunks = 2 * kAttKeys * row / 16;  // 16-byte copies per stage
    static constexpr size_t smem = (size_t)kAttStages * stage;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// The barrier receives one arrival from this thread once all of its earlier
// asynchronous copies have landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Split partials that fit the ring (both decode kernels' rings hold at
// least 1024 * D bytes) are merged from shared memory, fetched with one bulk
// copy per head: the copy engine keeps them all in flight, where a thread's
// share of hundreds of loads would queue behind its SM's outstanding-request
// limit.
template <int D>
constexpr size_t merge_bulk_cap() { return (size_t)1024 * D - 1024; }

// The merge of attn_split_merge from shared memory: the last CTA of (b, kvh)
// copies the G heads' [nsplit][D] partial sums into att_smem, reads every
// split's m and l, and sums in split order. Whole CTA; G * nsplit * (D + 1)
// floats fit in merge_bulk_cap<D>().
template <int D, int G>
__device__ __forceinline__ void attn_split_merge_bulk(const DecodeAttnArgs& a, int b, int kvh, int bk,
                                                      uint8_t* att_smem, float* m_s, float* l_s) {
    __shared__ __align__(8) uint64_t mbar;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ns = a.nsplit;
    float* pbuf = reinterpret_cast<float*>(att_smem);  // [G][ns][D]
    float* wts = pbuf + (size_t)G * ns * D;            // [G][ns]
    const int64_t hb0 = (int64_t)b * a.heads + kvh * G;
    if (tid == 0) {
        mbar_init(&mbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        // the ring was last used, and the other units' partials were written
        // (acquired above), through the generic proxy; the copies use the async one
        asm volatile("fence.proxy.async;" ::: "memory");
        const uint32_t per = (uint32_t)ns * D * 4;
        mbar_expect_tx(&mbar, per * G);
        for (int g = 0; g < G; ++g)
            bulk_g2s(pbuf + (size_t)g * ns * D, a.part_acc + (hb0 + g) * ns * D, per, &mbar);
    }
    // warp g < G: head g's weights e^(m_s - M) and l = sum_s l_s e^(m_s - M)
    if (warp < G) {
        const int64_t hb = hb0 + warp;
        float M = -INFINITY;
        for (int s2 = lane; s2 < ns; s2 += 32) M = fmaxf(M, __ldcg(&a.part_m[hb * ns + s2]));
        M = warp_max(M);
        float lw = 0.0f;
        for (int s2 = lane; s2 < ns; s2 += 32) {
            const float mm = __ldcg(&a.part_m[hb * ns + s2]);
            const float w = mm == -INFINITY ? 0.0f : expf(mm - M);
            wts[warp * ns + s2] = w;
            lw += __ldcg(&a.part_l[hb * ns + s2]) * w;
        }
        lw = warp_sum(lw);
        if (lane == 0) l_s[warp] = lw;
    }
    __syncthreads();  // thread 0's barrier initialisation, the weights
    const bool ok = mbar_wait_bounded(&mbar, 0);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) {
            mbar_drain(&mbar, 0);  // the partial sums' copy must land before the CTA exits
            atomicExch(a.err, kErrAttnWait);
            a.counters[bk] = 0;
        }
        return;
    }
    for (int i = tid; i < G * D; i += kAttThreads) {
        const int g = i / D, dd = i - g * D;
        const float* src = pbuf + (size_t)g * ns * D + dd;
        const float* w = wts + g * ns;
        float o = 0.0f;
        for (int s2 = 0; s2 < ns; ++s2) o = fmaf(src[(size_t)s2 * D], w[s2], o);
        const float r = o * (1.0f / l_s[g]);
        a.out[(hb0 + g) * D + dd] = r;
        // a warp holds 32 consecutive dims of one head: one block of the o input
        if (a.qy.data) qx_write_group(a.qy, b, ((int64_t)(kvh * G + g) * D + dd) >> 5, lane, r, true);
    }
    if (tid == 0) a.counters[bk] = 0;
}

// The split partials of one (sequence, KV head) were stored by its units;
// this unit's arrival is counted and the last unit to arrive merges them in
// split order into out (and the o projection's quantised image). Whole CTA of
// kAttThreads threads; m_s, l_s: G floats of shared memory; flag_s one int.
template <int D, int G>
__device__ __forceinline__ void attn_split_merge(const DecodeAttnArgs& a, int b, int kvh, int bk, uint8_t* att_smem,
                                                 float* m_s, float* l_s, int& flag_s) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __syncthreads();  // every partial store precedes thread 0's release
    if (tid == 0) flag_s = atomic_add_acq_rel_gpu(&a.counters[bk], 1) == a.nsplit - 1;
    __syncthreads();
    if (!flag_s) return;
    if ((size_t)G * a.nsplit * (D + 1) * 4 <= merge_bulk_cap<D>()) {
        attn_split_merge_bulk<D, G>(a, b, kvh, bk, att_smem, m_s, l_s);
        return;
    }
    // the last CTA of (b, kvh): out = sum_s acc_s e^(m_s - M) / sum_s l_s e^(m_s - M)
    // in split order, MR splits per round (32 while a thread's share of the
    // round fits in 64 registers, else 16). The first round's partial sums and
    // every split's m and l are requested together, so the common case (up to
    // MR splits) costs one round trip to L2.
    static_assert(G <= kAttWarps, "one head per warp in the merge");
    const int ns = a.nsplit;
    constexpr int OPT = (G * D + kAttThreads - 1) / kAttThreads;        // outputs per thread
    constexpr int MR = OPT <= 2 ? 32 : 16;                              // splits per round
    float* wts = reinterpret_cast<float*>(att_smem) + kAttWarps * G * D;  // [G][MR]
    float o[OPT], pa[OPT][MR];
#pragma unroll
    for (int t = 0; t < OPT; ++t) o[t] = 0.0f;
    auto load_round = [&](int s0) {
        const int nr = min(MR, ns - s0);
#pragma unroll
        for (int t = 0; t < OPT; ++t) {
            const int i = tid + t * kAttThreads;
            const int g = i / D, dd = i - g * D;
            const int64_t hb = (int64_t)b * a.heads + kvh * G + (g < G ? g : 0);
#pragma unroll
            for (int u = 0; u < MR; ++u)
                pa[t][u] = (i < G * D && u < nr) ? __ldcg(&a.part_acc[(hb * ns + s0 + u) * D + dd]) : 0.0f;
        }
    };
    load_round(0);
    // warp g < G: head g. Lane j holds split j's m and l when there are at
    // most 32 splits (else they are re-read per round).
    const int64_t hbw = (int64_t)b * a.heads + kvh * G + (warp < G ? warp : 0);
    float mreg = -INFINITY, lreg = 0.0f;
    if (warp < G) {
        if (lane < ns) {
            mreg = __ldcg(&a.part_m[hbw * ns + lane]);
            lreg = __ldcg(&a.part_l[hbw * ns + lane]);
        }
        float M = mreg;
        for (int s2 = lane + 32; s2 < ns; s2 += 32) M = fmaxf(M, __ldcg(&a.part_m[hbw * ns + s2]));
        M = warp_max(M);
        if (lane == 0) {
            m_s[warp] = M;
            l_s[warp] = 0.0f;
        }
    }
    __syncthreads();
    for (int s0 = 0; s0 < ns; s0 += MR) {
        const int nr = min(MR, ns - s0);
        if (s0 > 0) load_round(s0);
        if (warp < G) {
            float mm, ll;
            if (ns <= 32) {
                mm = __shfl_sync(0xffffffffu, mreg, (s0 + lane) & 31);
                ll = __shfl_sync(0xffffffffu, lreg, (s0 + lane) & 31);
            } else {
                mm = lane < nr ? __ldcg(&a.part_m[hbw * ns + s0 + lane]) : -INFINITY;
                ll = lane < nr ? __ldcg(&a.part_l[hbw * ns + s0 + lane]) : 0.0f;
            }
            float w = 0.0f, lw = 0.0f;
            if (lane < nr) {
                w = mm == -INFINITY ? 0.0f : expf(mm - m_s[warp]);
                lw = ll * w;
            }
            if (lane < MR) wts[warp * MR + lane] = w;
            lw = warp_sum(lw);
            if (lane == 0) l_s[warp] += lw;
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < OPT; ++t) {
            const int i = tid + t * kAttThreads;
            const int g = i / D;
            if (i < G * D)
#pragma unroll
                for (int u = 0; u < MR; ++u)
                    if (u < nr) o[t] = fmaf(pa[t][u], wts[g * MR + u], o[t]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int t = 0; t < OPT; ++t) {
        const int i = tid + t * kAttThreads;
        if (i >= G * D) continue;
        const int g = i / D, dd = i - g * D;
        const int64_t hb = (int64_t)b * a.heads + kvh * G + g;
        const float r = o[t] * (1.0f / l_s[g]);
        a.out[hb * D + dd] = r;
        if (a.qy.data) qx_write_group(a.qy, b, ((int64_t)(kvh * G + g) * D + dd) >> 5, lane, r, true);
    }
    if (tid == 0) a.counters[bk] = 0;
}

// One (sequence, KV head, split) unit on the whole CTA (kAttThreads threads):
// ring = ST stages of staged K/V rows, bars = ST mbarriers (initialised here).
// wait() separates the requests that depend on nothing in flight from the
// rest (the kernel's wait on its predecessor, or a grid barrier).
template <int D, int G, int ST, typename Wait>
__device__ __forceinline__ void attn_unit(const DecodeAttnArgs& a, int bk, int split, uint8_t* att_smem,
                                          uint64_t* bars, Wait wait) {
    using Lay = AttLayout<D>;
    constexpr int kAttStages = ST;
    constexpr int DPL = D / 32;   // head dims per lane
    constexpr int KB = 32 / G;    // keys per score batch
    constexpr int NB = kAttKeys / KB;  // score batches per stage
    __shared__ __align__(16) float ps[kAttKeys][G];
    __shared__ float corr_s[G], m_s[G], l_s[G];
    __shared__ int flag_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = bk / a.kv_heads, kvh = bk - b * a.kv_heads;
    // the key range: the position counter is not written during a step
    const int kv_len = max(1, min(a.max_kv, a.pos_ptr ? *a.pos_ptr + 1 : a.kv_len));
    const int chunk = (kv_len + a.nsplit - 1) / a.nsplit;
    const int k0 = min(kv_len, split * chunk), k1 = min(kv_len, k0 + chunk);
    const int nkeys = k1 - k0;
    const int nsteps = (nkeys + kAttKeys - 1) / kAttKeys;
    const int cur = kv_len - 1;  // the decoded token's row
    const int cur_step = (cur >= k0 && cur < k1) ? (cur - k0) / kAttKeys : -1;
    const int64_t ks = (int64_t)a.kv_heads * D;
    const __half* kc = reinterpret_cast<const __half*>(a.k_cache) + (int64_t)b * a.cache_sb + (int64_t)kvh * D;
    const __half* vc = reinterpret_cast<const __half*>(a.v_cache) + (int64_t)b * a.cache_sb + (int64_t)kvh * D;
    // 16-byte chunk c of a stage: row c / (D/8) (keys, then values), part c % (D/8)
    constexpr int CPR = D / 8;
    auto issue = [&](int s, bool skip_cur) {
        uint8_t* base = att_smem + (size_t)(s % kAttStages) * Lay::stage;
        for (int c = tid; c < Lay::chunks; c += kAttThreads) {
            const int row = c / CPR, part = c - row * CPR;
            const int r = row & (kAttKeys - 1);
            const int key = k0 + s * kAttKeys + r;
            if (key >= k1 || (skip_cur && key == cur)) continue;
            const __half* src = (row < kAttKeys ? kc : vc) + key * ks + part * 8;
            cp_async16(base + row * Lay::row + part * 16, src);
        }
    };
    const int npre = min(kAttStages, nsteps);
    if (tid == 0) {
        for (int s = 0; s < kAttStages; ++s) mbar_init(&bars[s], kAttThreads);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    for (int s = 0; s < npre; ++s) {
        issue(s, true);
        // the decoded token's rows come after the wait: their copiers arrive then
        if (s != cur_step || tid >= 2 * CPR) cp_async_arrive(&bars[s]);
    }
    wait();
    if (cur_step >= 0 && cur_step < npre && tid < 2 * CPR) {
        uint8_t* base = att_smem + (size_t)cur_step * Lay::stage;
        const int r = cur - k0 - cur_step * kAttKeys;
        const int row = tid < CPR ? r : kAttKeys + r, part = tid < CPR ? tid : tid - CPR;
        cp_async16(base + row * Lay::row + part * 16, (tid < CPR ? kc : vc) + cur * ks + part * 8);
        cp_async_arrive(&bars[cur_step]);
    }
    // this lane's head dims of the G queries, pre-scaled
    float qr[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < DPL; ++j)
            qr[g][j] = a.q[((int64_t)b * a.heads + kvh * G + g) * D + lane * DPL + j] * a.scale;
    if (tid < G) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.0f;
    }
    float acc[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[g][j] = 0.0f;
    __syncthreads();
    int s = 0;
    bool failed = false;
    for (; s < nsteps; ++s) {
        const int st = s % kAttStages;
        const bool ok = mbar_wait_bounded(&bars[st], (uint32_t)((s / kAttStages) & 1));
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
        const int n = min(kAttKeys, k1 - (k0 + s * kAttKeys));
        const uint8_t* kbase = att_smem + (size_t)st * Lay::stage;
        const uint8_t* vbase = kbase + kAttKeys * Lay::row;
        // scores: batches of KB keys, transposed across the warp
        for (int bt = warp; bt < NB; bt += kAttWarps) {
            float v[32];
#pragma unroll
            for (int kk = 0; kk < KB; ++kk) {
                const __half* kr = reinterpret_cast<const __half*>(kbase + (bt * KB + kk) * Lay::row) + lane * DPL;
                float kf[DPL];
#pragma unroll
                for (int j = 0; j < DPL; j += 2) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(kr + j));
                    kf[j] = f.x;
                    kf[j + 1] = f.y;
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float t = 0.0f;
#pragma unroll
                    for (int j = 0; j < DPL; ++j) t = fmaf(qr[g][j], kf[j], t);
                    v[kk * G + g] = t;
                }
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) {
                const bool upper = (lane & o) != 0;
#pragma unroll
                for (int i = 0; i < o; ++i) {
                    const float send = upper ? v[i] : v[i + o];
                    const float keep = upper ? v[i + o] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            const int key = bt * KB + lane / G;
            ps[key][lane % G] = key < n ? v[0] : -INFINITY;
        }
        __syncthreads();
        // online softmax bookkeeping: warp w keeps heads w, w + 8, ...
        for (int g = warp; g < G; g += kAttWarps) {
            const float s0 = ps[lane][g], s1 = ps[lane + 32][g];
            const float mo = m_s[g];
            const float mn = fmaxf(mo, warp_max(fmaxf(s0, s1)));
            const float c = mo == -INFINITY ? 0.0f : expf(mo - mn);
            const float p0 = lane < n ? expf(s0 - mn) : 0.0f;
            const float p1 = lane + 32 < n ? expf(s1 - mn) : 0.0f;
            ps[lane][g] = p0;
            ps[lane + 32][g] = p1;
            const float sum = warp_sum(p0 + p1);
            if (lane == 0) {
                l_s[g] = l_s[g] * c + sum;
                m_s[g] = mn;
                corr_s[g] = c;
            }
        }
        __syncthreads();
        // values: warp w takes keys w, w + 8, ... of the stage
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float c = corr_s[g];
#pragma unroll
            for (int j = 0; j < DPL; ++j) acc[g][j] *= c;
        }
#pragma unroll 2
        for (int r = warp; r < n; r += kAttWarps) {
            const __half* vr = reinterpret_cast<const __half*>(vbase + r * Lay::row) + lane * DPL;
            float vf[DPL];
#pragma unroll
            for (int j = 0; j < DPL; j += 2) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vr + j));
                vf[j] = f.x;
                vf[j + 1] = f.y;
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float p = ps[r][g];
#pragma unroll
                for (int j = 0; j < DPL; ++j) acc[g][j] = fmaf(p, vf[j], acc[g][j]);
            }
        }
        __syncthreads();  // stage st is free again
        if (s + kAttStages < nsteps) {
            issue(s + kAttStages, false);
            cp_async_arrive(&bars[st]);
        }
    }
    if (failed) {
        // let the copies still in flight land before the CTA exits
        for (int s2 = s; s2 < nsteps && s2 < s + kAttStages; ++s2)
            mbar_drain(&bars[s2 % kAttStages], (uint32_t)((s2 / kAttStages) & 1));
        if (tid == 0) atomicExch(a.err, kErrAttnWait);
        return;
    }
    // merge the warps (the ring is idle now)
    float* wacc = reinterpret_cast<float*>(att_smem);  // [warps][G][D]
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < DPL; ++j) wacc[(warp * G + g) * D + lane * DPL + j] = acc[g][j];
    __syncthreads();
    for (int i = tid; i < G * D; i += kAttThreads) {
        const int g = i / D, dd = i - g * D;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttWarps; ++w) o += wacc[(w * G + g) * D + dd];
        const int64_t hb = (int64_t)b * a.heads + kvh * G + g;
        if (a.nsplit == 1) {
            const float r = o * (1.0f / l_s[g]);
            a.out[hb * D + dd] = r;
            // a warp holds 32 consecutive dims of one head: one block of the o input
            if (a.qy.data) qx_write_group(a.qy, b, ((int64_t)(kvh * G + g) * D + dd) >> 5, lane, r, true);
        } else {
            a.part_acc[(hb * a.nsplit + split) * D + dd] = o;
            if (dd == 0) {
                a.part_m[hb * a.nsplit + split] = m_s[g];
                a.part_l[hb * a.nsplit + split] = l_s[g];
            }
        }
    }
    if (a.nsplit == 1) return;
    attn_split_merge<D, G>(a, b, kvh, bk, att_smem, m_s, l_s, flag_s);
}

// Decode attention on the tensor cores (fast numerics) ------------------------
// Same unit and split merge as above; the dot products run as warp-level
// m16n8k16 f16 MMAs with f32 accumulation. Stages hold 128 keys (16 per warp)
// whose K and V rows are staged with 16-byte chunks at swizzled positions
// (chunk ^ (row & 7)) so the 8x8 ldmatrix loads are free of bank conflicts.
// Each warp keeps its own online softmax over its keys, with the G <= 8
// query heads as the MMA N dimension: scores S = K Q^T (16 keys x 8 heads,
// the query split into f16 high and low parts, ~22-bit precision), then
// O^T += V^T P^T with P rounded to f16 and transposed in registers
// (movmatrix). The warps' (m, l, O) are combined at the end in warp order.
constexpr int kTcKeys = 128;   // keys per stage: 16 per warp
constexpr int kTcStages = 2;

template <int D>
struct TcLayout {
    static constexpr int row = 2 * D;                   // bytes of one key or value row
    static constexpr int stage = 2 * kTcKeys * row;     // keys, then values
    static constexpr int chunks = stage / 16;           // 16-byte copies per stage
    static constexpr size_t smem = (size_t)kTcStages * stage;
};

__device__ __forceinline__ uint32_t tc_swz(int row, int chunk, int row_bytes) {
    return (uint32_t)(row * row_bytes + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
// d += A B for one m16n8k16 tile
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <int D, int G, typename Wait>
__device__ __forceinline__ void attn_unit_tc(const DecodeAttnArgs& a, int bk, int split, uint8_t* att_smem,
                                             uint64_t* bars, Wait wait) {
    static_assert(G <= 8 && (D == 64 || D == 128), "tensor-core decode attention shape");
    using Lay = TcLayout<D>;
    constexpr int KS = D / 16;  // 16-dim steps (score k-steps, output m-tiles)
    constexpr int CPR = D / 8;  // 16-byte chunks per row
    __shared__ float m_s[G], l_s[G];
    __shared__ int flag_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int b = bk / a.kv_heads, kvh = bk - b * a.kv_heads;
    const int kv_len = max(1, min(a.max_kv, a.pos_ptr ? *a.pos_ptr + 1 : a.kv_len));
    const int chunk = (kv_len + a.nsplit - 1) / a.nsplit;
    const int k0 = min(kv_len, split * chunk), k1 = min(kv_len, k0 + chunk);
    const int nkeys = k1 - k0;
    const int nsteps = (nkeys + kTcKeys - 1) / kTcKeys;
    const int cur = kv_len - 1;
    const int cur_step = (cur >= k0 && cur < k1) ? (cur - k0) / kTcKeys : -1;
    const int64_t ks = (int64_t)a.kv_heads * D;
    const __half* kc = reinterpret_cast<const __half*>(a.k_cache) + (int64_t)b * a.cache_sb + (int64_t)kvh * D;
    const __half* vc = reinterpret_cast<const __half*>(a.v_cache) + (int64_t)b * a.cache_sb + (int64_t)kvh * D;
    // chunk c of a stage: row c / CPR of the keys (rows 0..127), then of the values
    auto issue = [&](int s, bool skip_cur) {
        uint8_t* base = att_smem + (size_t)(s % kTcStages) * Lay::stage;
        for (int c = tid; c < Lay::chunks; c += kAttThreads) {
            const int row = c / CPR, part = c - row * CPR;
            const int r = row & (kTcKeys - 1);
            const int key = k0 + s * kTcKeys + r;
            uint8_t* dst = base + (row < kTcKeys ? 0 : kTcKeys * Lay::row) + tc_swz(r, part, Lay::row);
            if (key >= k1) {
                // rows past the split feed the MMAs with probability 0: keep them finite
                *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
                continue;
            }
            if (skip_cur && key == cur) continue;
            cp_async16(dst, (row < kTcKeys ? kc : vc) + key * ks + part * 8);
        }
    };
    const int npre = min(kTcStages, nsteps);
    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) mbar_init(&bars[s], kAttThreads);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    for (int s = 0; s < npre; ++s) {
        issue(s, true);
        if (s != cur_step || tid >= 2 * CPR) cp_async_arrive(&bars[s]);
    }
    wait();
    if (cur_step >= 0 && cur_step < npre && tid < 2 * CPR) {
        uint8_t* base = att_smem + (size_t)cur_step * Lay::stage;
        const int r = cur - k0 - cur_step * kTcKeys;
        const bool is_k = tid < CPR;
        const int part = is_k ? tid : tid - CPR;
        cp_async16(base + (is_k ? 0 : kTcKeys * Lay::row) + tc_swz(r, part, Lay::row),
                   (is_k ? kc : vc) + cur * ks + part * 8);
        cp_async_arrive(&bars[cur_step]);
    }
    // query fragments (MMA B operand, N = heads): head hq = lane / 4, dims
    // 16 j + 2 (lane % 4) + {0, 1} and + 8, pre-scaled, as f16 high + low parts
    const int hq = lane >> 2, q4 = lane & 3, r8 = lane >> 2;
    uint32_t qh0[KS], qh1[KS], ql0[KS], ql1[KS];
    {
        const float* qrow = a.q + ((int64_t)b * a.heads + kvh * G + (hq < G ? hq : 0)) * D;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            float x[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int d = 16 * j + 2 * q4 + (e & 1) + (e >> 1) * 8;
                x[e] = hq < G ? qrow[d] * a.scale : 0.0f;
            }
            const __half2 h01 = __floats2half2_rn(x[0], x[1]), h23 = __floats2half2_rn(x[2], x[3]);
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            qh0[j] = *reinterpret_cast<const uint32_t*>(&h01);
            qh1[j] = *reinterpret_cast<const uint32_t*>(&h23);
            ql0[j] = pack_f16x2(x[0] - f01.x, x[1] - f01.y);
            ql1[j] = pack_f16x2(x[2] - f23.x, x[3] - f23.y);
        }
    }
    // O^T accumulators: m-tile t = dims 16 t + r8 (+8) x heads 2 q4 + {0, 1}
    float o[KS][4];
#pragma unroll
    for (int t = 0; t < KS; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};  // heads 2 q4 + {0, 1}
    const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: the matrix this lane addresses, its row
    int s = 0;
    bool failed = false;
    for (; s < nsteps; ++s) {
        const int st = s % kTcStages;
        if (!mbar_wait_bounded(&bars[st], (uint32_t)((s / kTcStages) & 1))) failed = true;
        if (__syncthreads_or(failed)) {
            failed = true;
            break;
        }
        const int kt = warp * 16;                               // this warp's 16 keys of the stage
        const int nv = min(kTcKeys, nkeys - s * kTcKeys) - kt;  // of which valid
        if (nv > 0) {
            const uint32_t kbase = smem_u32(att_smem + (size_t)st * Lay::stage);
            const uint32_t vbase = kbase + kTcKeys * Lay::row;
            // scores (16 keys x 8 heads): A = K rows via ldmatrix (keys kt.., dims 16 j..)
            float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const int krow = kt + (mi & 1) * 8 + rr;
#pragma unroll
            for (int j = 0; j < KS; ++j) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(kbase + tc_swz(krow, 2 * j + (mi >> 1), Lay::row), a0, a1, a2, a3);
                mma_f16(sc, a0, a1, a2, a3, qh0[j], qh1[j]);
                mma_f16(sc, a0, a1, a2, a3, ql0[j], ql1[j]);
            }
            // sc: keys r8 (sc[0..1]) and r8 + 8 (sc[2..3]) x heads 2 q4 + {0, 1};
            // online softmax per head over the 8 lanes that share q4
            if (r8 >= nv) sc[0] = sc[1] = -INFINITY;
            if (r8 + 8 >= nv) sc[2] = sc[3] = -INFINITY;
            float p[4];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float mx = fmaxf(sc[c], sc[2 + c]);
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float mn = fmaxf(m_run[c], mx);  // finite: every tile has a valid key
                const float corr = m_run[c] == -INFINITY ? 0.0f : expf(m_run[c] - mn);
                p[c] = sc[c] == -INFINITY ? 0.0f : expf(sc[c] - mn);
                p[2 + c] = sc[2 + c] == -INFINITY ? 0.0f : expf(sc[2 + c] - mn);
                float rs = p[c] + p[2 + c];
                rs += __shfl_xor_sync(0xffffffffu, rs, 4);
                rs += __shfl_xor_sync(0xffffffffu, rs, 8);
                rs += __shfl_xor_sync(0xffffffffu, rs, 16);
                l_run[c] = l_run[c] * corr + rs;
                m_run[c] = mn;
#pragma unroll
                for (int t = 0; t < KS; ++t) {
                    o[t][c] *= corr;
                    o[t][2 + c] *= corr;
                }
            }
            // P^T (16 keys x 8 heads) as the B operand: transpose the two 8x8 blocks
            const uint32_t pb0 = movm_t(pack_f16x2(p[0], p[1])), pb1 = movm_t(pack_f16x2(p[2], p[3]));
            // O^T += V^T P^T: A = V^T via transposing ldmatrix (dims 16 t.., keys kt..)
            const int vrow = kt + (mi >> 1) * 8 + rr;
#pragma unroll
            for (int t = 0; t < KS; ++t) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4_t(vbase + tc_swz(vrow, 2 * t + (mi & 1), Lay::row), a0, a1, a2, a3);
                mma_f16(o[t], a0, a1, a2, a3, pb0, pb1);
            }
        }
        if (s + kTcStages < nsteps) {
            __syncthreads();  // every warp is done with stage st
            issue(s + kTcStages, false);
            cp_async_arrive(&bars[st]);
        }
    }
    if (failed) {
        for (int s2 = s; s2 < nsteps && s2 < s + kTcStages; ++s2)
            mbar_drain(&bars[s2 % kTcStages], (uint32_t)((s2 / kTcStages) & 1));
        if (tid == 0) atomicExch(a.err, kErrAttnWait);
        return;
    }
    // combine the warps in warp order (the ring is idle now)
    __syncthreads();
    float* wo = reinterpret_cast<float*>(att_smem);       // [warps][G][D]
    float* wm = wo + kAttWarps * G * D;                    // [warps][G]
    float* wl = wm + kAttWarps * G;                        // [warps][G]
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const int hh = 2 * q4 + c;
        if (hh < G) {
#pragma unroll
            for (int t = 0; t < KS; ++t) {
                wo[(warp * G + hh) * D + 16 * t + r8] = o[t][c];
                wo[(warp * G + hh) * D + 16 * t + r8 + 8] = o[t][2 + c];
            }
            if (r8 == 0) {
                wm[warp * G + hh] = m_run[c];
                wl[warp * G + hh] = l_run[c];
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += kAttThreads) {
        const int g = i / D, dd = i - g * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttWarps; ++w) M = fmaxf(M, wm[w * G + g]);
        float acc = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < kAttWarps; ++w) {
            const float mw = wm[w * G + g];
            const float f = mw == -INFINITY ? 0.0f : expf(mw - M);
            acc = fmaf(wo[(w * G + g) * D + dd], f, acc);
            L = fmaf(wl[w * G + g], f, L);
        }
        const int64_t hb = (int64_t)b * a.heads + kvh * G + g;
        if (a.nsplit == 1) {
            const float r = acc * (1.0f / L);
            a.out[hb * D + dd] = r;
            if (a.qy.data) qx_write_group(a.qy, b, ((int64_t)(kvh * G + g) * D + dd) >> 5, lane, r, true);
        } else {
            a.part_acc[(hb * a.nsplit + split) * D + dd] = acc;
            if (dd == 0) {
                a.part_m[hb * a.nsplit + split] = M;
                a.part_l[hb * a.nsplit + split] = L;
            }
        }
    }
    if (a.nsplit == 1) return;
    attn_split_merge<D, G>(a, b, kvh, bk, att_smem, m_s, l_s, flag_s);
}

}  // namespace bc
