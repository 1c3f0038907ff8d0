// gemv_dispatch.cu -- planning and format dispatch for the dequant-GEMV
// kernels: the tiled split-K kernel (gemv.cuh) and the persistent TMA-fed
// stream-K kernel (gemv3.cuh).
#include <algorithm>
#include <cstdlib>

#include "gemv3.cuh"
#include "qgemm_tc.h"

namespace bc {

GemvPlan plan_qgemv(const BeaconCudaContext* ctx, const QLayout& L, int batch, int mode) {
    if (batch < 1 || batch > 16) invalid("quantized GEMV supports batch 1..16");
    if (!is_core_format(L.dtype)) mode = MODE_F32;  // generic formats stage f32 activations
    GemvPlan pl;
    pl.bpad = batch <= 1 ? 1 : batch <= 2 ? 2 : batch <= 4 ? 4 : batch <= 8 ? 8 : 16;
    const int64_t groups = L.groups(), ktiles = L.ktiles();
    const size_t per_tile = gemv_smem_bytes(mode, pl.bpad, 256);
    const int64_t tps_max = std::max<int64_t>(1, (int64_t)((96 * 1024) / per_tile));
    // Enough CTAs for two per SM, but keep at least 4 tiles (one per warp)
    // per CTA unless shared memory forces a finer split.
    const int64_t target = 2 * (int64_t)(ctx ? ctx->sm_count : 148);
    int64_t ks = (target + groups - 1) / groups;
    ks = std::min<int64_t>(ks, std::max<int64_t>(1, ktiles / 4));
    ks = std::max<int64_t>(ks, (ktiles + tps_max - 1) / tps_max);
    ks = std::max<int64_t>(1, std::min<int64_t>(ks, ktiles));
    int64_t tps = (ktiles + ks - 1) / ks;
    ks = (ktiles + tps - 1) / tps;
    pl.ksplit = (int)ks;
    pl.tps = (int)tps;
    pl.smem = gemv_smem_bytes(mode, pl.bpad, (int)tps * 256);
    return pl;
}

void launch_qgemv(const GemvPlan& plan, const QLayout& L, const void* w, const void* x, bool x_f16,
                  int64_t x_ld, int batch, float* y, int64_t y_ld, int epi, const float* res,
                  int64_t res_ld, int mode, bool rtz, const GemvScratch& scratch, cudaStream_t s) {
    if (plan.ksplit > 1) {
        if (!scratch.partial || !scratch.counters ||
            scratch.partial_floats < (size_t)plan.ksplit * batch * L.n_pad ||
            scratch.counter_count < L.groups())
            invalid("split-K GEMV launched without enough scratch");
    }
    GemvLaunch a{&plan, &L, w, x, x_f16, x_ld, batch, y, y_ld, epi, res, res_ld, mode, rtz, scratch, s};
    launch_qgemv_any(a);
}

void launch_qgemv_any(const GemvLaunch& a) {
    switch (a.L->dtype) {
        case BEACON_CUDA_DTYPE_Q4_0: return launch_qgemv_q4_0(a);
        case BEACON_CUDA_DTYPE_Q8_0: return launch_qgemv_q8_0(a);
        case BEACON_CUDA_DTYPE_Q4_K: return launch_qgemv_q4_k(a);
        case BEACON_CUDA_DTYPE_Q4_1: return launch_qgemv_q4_1(a);
        case BEACON_CUDA_DTYPE_Q5_0: return launch_qgemv_q5_0(a);
        case BEACON_CUDA_DTYPE_Q5_1: return launch_qgemv_q5_1(a);
        case BEACON_CUDA_DTYPE_Q2_K: return launch_qgemv_q2_k(a);
        case BEACON_CUDA_DTYPE_Q3_K: return launch_qgemv_q3_k(a);
        case BEACON_CUDA_DTYPE_Q5_K: return launch_qgemv_q5_k(a);
        case BEACON_CUDA_DTYPE_Q6_K: return launch_qgemv_q6_k(a);
        case BEACON_CUDA_DTYPE_Q8_K: return launch_qgemv_q8_k(a);
        default: fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "quantized GEMV: unsupported block type");
    }
}

// The persistent kernel is used for batch <= 8 when at least 2 ring stages
// per warp and the staged activations fit under the opt-in shared memory, and
// there are at least as many tiles as warps (every warp range non-empty).
// Batch <= 2 builds hold at most 128 registers per thread, so two CTAs fit on
// an SM: the ring is then sized to keep a CTA under half the SM's shared
// memory, which lets the next kernel's CTA start (and fetch its weights)
// while this one finishes, and GEMVs with many tiles per warp run two CTAs
// per SM for more warps in flight. A GEMV with no more row groups than CTA
// slots, whose groups have 8 to 8 * stages k-tiles, runs one CTA per row
// group, whose warps split the group's K and sum in shared memory: no
// cross-CTA exchange.
int device_smem_optin() {
    int dev = 0, v = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    cuda_check(cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev), "cudaDeviceGetAttribute");
    return v;
}

// Dynamic shared memory that keeps a CTA alone on its SM (two need more than
// the SM's 228 KB) but leaves room for a half-SM CTA of another kernel.
constexpr size_t kSpreadSmem = 117 * 1024;

LinearPlan plan_linear(const BeaconCudaContext* ctx, const QLayout& L, int batch, int mode) {
    LinearPlan pl;
    pl.v2 = plan_qgemv(ctx, L, batch, mode);
    if (batch > 8 || !is_core_format(L.dtype)) return pl;  // the persistent kernel serves the dedicated layouts
    pl.bpad = batch <= 1 ? 1 : batch <= 2 ? 2 : batch <= 4 ? 4 : 8;
    const size_t budget = 220 * 1024, half_sm = 110 * 1024;
    // The fast numerics consume tiles with the tensor-core (mma.sync) consumer
    // from 4 rows on, and for Q8_0 (no nibble unpacking); 4-bit weights at 1-2
    // rows keep the dp2a consumer, measured faster there (its per-row
    // accumulation needs no transpose and no scale table).
    // BEACON_CUDA_GEMV_MMA=0: dp2a everywhere; =2: tensor cores everywhere.
    static const int mma_env = [] {
        const char* e = std::getenv("BEACON_CUDA_GEMV_MMA");
        return e ? std::atoi(e) : 1;
    }();
    bool mma = mode == MODE_FAST && mma_env != 0 &&
               (mma_env == 2 || pl.bpad >= 4 || L.dtype == BEACON_CUDA_DTYPE_Q8_0);
    const size_t tb = (size_t)L.tile_bytes;
    auto x_bytes = [&](bool use_mma) {
        return gemv3_x_bytes(mode, pl.bpad, L.k_pad, use_mma) + gemv3_red_bytes(pl.bpad) +
               (use_mma ? gemv3_mma_bytes(L.dtype, pl.bpad) : 0);
    };
    auto ring_stages = [&](bool use_mma) {
        const size_t x = x_bytes(use_mma);
        return x + 256 + 2 * kG3Warps * tb > budget ? 0 : (int)std::min<size_t>(6, (budget - x - 256) / (kG3Warps * tb));
    };
    // The tensor-core consumer's scratch must leave room for two ring stages
    // (three for Q8_0, whose slot is refilled only after its MMAs read it);
    // where it does not, the dp2a consumer (no scratch) keeps the plan.
    if (mma && ring_stages(true) < (L.dtype == BEACON_CUDA_DTYPE_Q8_0 ? 3 : 2)) mma = false;
    const size_t xb = x_bytes(mma);
    if (xb + 256 + 2 * kG3Warps * tb > budget) return pl;
    int stages = (int)std::min<size_t>(6, (budget - xb - 256) / (kG3Warps * tb));
    const bool pairable = pl.bpad <= 2 && xb + 256 + 2 * kG3Warps * tb <= half_sm;
    if (pairable) stages = (int)std::min<size_t>(stages, (half_sm - xb - 256) / (kG3Warps * tb));
    const int64_t total_tiles = L.groups() * L.ktiles();
    const int sms = ctx ? ctx->sm_count : 148;
    // BEACON_CUDA_GEMV_PAIR_TILES: tiles per warp from which two CTAs share an
    // SM (default 1: 16 warps per SM measured fastest in the decode step; a
    // large value keeps one CTA per SM everywhere)
    static const int64_t pair_tiles = [] {
        const char* e = std::getenv("BEACON_CUDA_GEMV_PAIR_TILES");
        return e ? std::max<int64_t>(1, std::atoll(e)) : (int64_t)1;
    }();
    const int cps = pairable && total_tiles >= (int64_t)sms * kG3Warps * pair_tiles ? 2 : 1;
    // BEACON_CUDA_GEMV_WHOLE_GROUPS=0: stream-K even where one CTA per row
    // group fits (default: one CTA per group, reduced in shared memory only)
    static const bool whole_ok = [] {
        const char* e = std::getenv("BEACON_CUDA_GEMV_WHOLE_GROUPS");
        return !(e && std::atoi(e) == 0);
    }();
    // one CTA per row group when the groups fit the SM slots and a group's
    // tiles fit its CTA's ring (all of its weights are requested at launch)
    const bool whole = whole_ok && L.ktiles() >= kG3Warps && L.ktiles() <= (int64_t)kG3Warps * stages &&
                       L.groups() <= (int64_t)sms * (pairable ? 2 : 1);
    const int64_t nctas = whole ? L.groups() : std::min<int64_t>((int64_t)sms * cps, total_tiles / kG3Warps);
    if (nctas < 1) return pl;
    if ((uint64_t)total_tiles * (uint64_t)nctas >= (1ull << 32)) return pl;  // 32-bit tile arithmetic
    const int64_t per_cta = (total_tiles + nctas - 1) / nctas;
    if (per_cta / L.ktiles() + 2 > kG3MaxCtaGroups) return pl;  // the CTA's arrival counters
    pl.v3 = true;
    pl.mma = mma;
    pl.stages = stages;
    pl.nctas = (int)nctas;
    pl.total_warps = nctas * kG3Warps;
    pl.smem = gemv3_bar_bytes(stages) + (size_t)kG3Warps * stages * tb + xb;
    // no more CTAs than SMs: ask for more than half an SM's shared memory so
    // the block scheduler cannot put two on one SM (it packs CTAs that fit,
    // leaving SMs idle), while one CTA of the next kernel still fits beside
    if (nctas <= sms && pairable) pl.smem = std::max<size_t>(pl.smem, kSpreadSmem);
    return pl;
}

// Rows of the next launch out of `rem` (1..16): the persistent kernel takes
// up to 8 rows at a time, in the largest of 8-, 4-, 2- or 1-row launches
// whose plan fits shared memory (staged activations of a long K); each reads
// the weights again, still faster than one launch of the tiled kernel (which
// is issue-bound at many rows: 1.3 ms against 0.23 ms for a 16-row 128256 x
// 4096 Q4_0 GEMV, measured). Only when no persistent plan fits at all does
// the tiled kernel take them all.
int linear_chunk_rows(const BeaconCudaContext* ctx, const QLayout& L, int rem, int mode) {
    const int b = std::min(16, rem);
    if (b <= 8 && plan_linear(ctx, L, b, mode).v3) return b;
    for (int c : {8, 4, 2, 1})
        if (c < b && plan_linear(ctx, L, c, mode).v3) return c;
    return b;
}

size_t LinearPlan::scratch_floats(int batch, const QLayout& L) const {
    if (v3) return (size_t)nctas * 2 * bpad * 32;
    return v2.ksplit > 1 ? (size_t)v2.ksplit * batch * L.n_pad : 0;
}

void launch_linear(const LinearPlan& plan, const QLayout& L, const void* w, const void* x, bool x_f16, int64_t x_ld,
                   int batch, float* y, int64_t y_ld, int epi, const float* res, int64_t res_ld, int mode, bool rtz,
                   const GemvScratch& scratch, cudaStream_t s, const float* norm_w, float norm_eps, bool pdl,
                   const QkvEpi* qkv, const QxImage* qx, const QxImage* qy) {
    GemvLaunch a{&plan.v2, &L, w, x, x_f16, x_ld, batch, y, y_ld, epi, res, res_ld, mode, rtz, scratch, s};
    a.pdl = pdl;
    if (epi == EPI_QKV && !qkv) invalid("fused q/k/v epilogue launched without its destinations");
    a.qkv = qkv;
    if (qx && qx->data) {
        if (!plan.v3 || mode != MODE_FAST || qx->bpad != plan.bpad || qx->kspan != (int)L.k_pad)
            invalid("pre-quantised activations need the persistent fast GEMV with the image's shape");
        a.qx = *qx;
    }
    if (qy && qy->data) {
        if (!plan.v3 || mode != MODE_FAST || batch > qy->bpad)
            invalid("quantised output needs the persistent fast GEMV and an image covering the batch");
        if (epi == EPI_ADD) {
            if (qy->kspan < (int)L.n_pad) invalid("quantised output: the image is narrower than the rows");
        } else if (epi == EPI_SWIGLU) {
            if (qy->kspan < (int)(L.n_pad / 2) || qy->norm_w || qy->ss)
                invalid("quantised SwiGLU output: the image must cover n/2 columns, without a norm");
            if (!scratch.counters || scratch.counter_count < L.groups() + (L.groups() + 1) / 2)
                invalid("quantised SwiGLU output launched without its pair counters");
        } else {
            invalid("quantised output needs the residual or SwiGLU epilogue");
        }
        a.qy = *qy;
        if (epi == EPI_SWIGLU) a.qy.pairs = scratch.counters + L.groups();
    }
    if (!plan.v3) {
        if (norm_w) invalid("the tiled GEMV has no fused RMSNorm; normalise first");
        if (plan.v2.ksplit > 1 &&
            (!scratch.partial || !scratch.counters || scratch.partial_floats < (size_t)plan.v2.ksplit * batch * L.n_pad ||
             scratch.counter_count < L.groups()))
            invalid("split-K GEMV launched without enough scratch");
        return launch_qgemv_any(a);
    }
    if (!scratch.partial || !scratch.counters || !scratch.err ||
        scratch.partial_floats < plan.scratch_floats(batch, L) || scratch.counter_count < L.groups())
        invalid("stream-K GEMV launched without enough scratch");
    a.norm_w = norm_w;
    a.norm_eps = norm_eps;
    switch (L.dtype) {
        case BEACON_CUDA_DTYPE_Q4_0: return launch_qgemv3_q4_0(plan, a);
        case BEACON_CUDA_DTYPE_Q8_0: return launch_qgemv3_q8_0(plan, a);
        case BEACON_CUDA_DTYPE_Q4_K: return launch_qgemv3_q4_k(plan, a);
        default: fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "quantized GEMV: unsupported block type");
    }
}

GemvScratch stream_gemv_scratch(BeaconCudaStream* stream, const LinearPlan& pl, int batch, const QLayout& L) {
    GemvScratch sc;
    Workspace& ws = stream->ws;
    const size_t pf = pl.scratch_floats(batch, L);
    void* data = ws.get(pf * sizeof(float), stream->s);  // grows (and zeroes) the arena when needed
    sc.err = ws.flags() + Workspace::kTimeoutFlag;
    if (pf == 0) return sc;
    if ((size_t)L.groups() > Workspace::kCounterInts) shape_err("too many rows for the split-K counters");
    sc.partial = static_cast<float*>(data);
    sc.partial_floats = pf;
    sc.counters = ws.counters();
    sc.counter_count = (int64_t)Workspace::kCounterInts;
    return sc;
}

// Prefill-sized matmul: the tensor-core GEMM in the fast numerics, otherwise
// the GEMV in 16-row chunks (each chunk streams the weight once), which
// follows the exact and CPU-reproducing numerics to the bit.
void dense_qmatmul(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* w, const void* x,
                   bool x_f16, int64_t rows, float* out, int numerics) {
    const int mode = numerics == BEACON_CUDA_NUMERICS_FAST ? MODE_FAST : MODE_F32;
    const bool rtz = numerics == BEACON_CUDA_NUMERICS_REF_RTZ;
    const QLayout& L = w->q;
    const size_t eb = x_f16 ? 2 : 4;
    cudaStream_t s = stream->s;
    if (mode == MODE_FAST && qgemm_tc_supported(L)) {
        void* x16 = stream->ws.get(qgemm_tc_scratch_bytes(rows, L.k), s);
        launch_qgemm_tc(L, w->data(), x, x_f16, L.k, rows, out, L.n, EPI_STORE, nullptr, 0, false,
                        stream->ws.flags() + Workspace::kTimeoutFlag, s, x16);
        return;
    }
    for (int64_t r0 = 0, b = 0; r0 < rows; r0 += b) {
        b = linear_chunk_rows(ctx, L, (int)std::min<int64_t>(rows - r0, 16), mode);
        LinearPlan pl = plan_linear(ctx, L, b, mode);
        GemvScratch sc = stream_gemv_scratch(stream, pl, b, L);
        launch_linear(pl, L, w->data(), static_cast<const uint8_t*>(x) + (size_t)r0 * L.k * eb, x_f16, L.k, b,
                      out + r0 * L.n, L.n, EPI_STORE, nullptr, 0, mode, rtz, sc, s);
    }
}

}  // namespace bc
