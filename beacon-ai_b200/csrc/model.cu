// model.cu -- fused Llama-style decoder runtime on one GPU (or one tensor-
// parallel rank): the op sequence of Engine<B>::forward (engine.rs:190-456)
// with the seven projections per layer and lm_head served by the dequant-GEMV
// kernels, the decode step captured once per batch size in a CUDA graph.
//
// Per layer (decode, B sequences, one token each):
//   rms_norm(h)                       -> xn
//   [Wq;Wk;Wv] xn          (one GEMV) -> qkv
//   rope(q,k) + K/V cache write       -> q, cache[b][pos]
//   split-K decode attention          -> attn
//   h += Wo attn           (GEMV, residual add fused; TP: + all-reduce)
//   rms_norm(h)                       -> xn
//   silu(Wg xn) * (Wu xn)  (one GEMV over interleaved gate/up rows)
//   h += Wd act            (GEMV, residual add fused; TP: + all-reduce)
// then rms_norm, lm_head GEMV (vocab-split under TP, all-gathered) and
// greedy argmax with the reference's tie rule (sampling.rs:60-66).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "argmax.h"
#include "attention.h"
#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "qx.cuh"
#include "qgemm_tc.h"

namespace bc {

namespace {

constexpr int kPrefillChunk = 2048;
constexpr int kDecodeGemvRows = 64;  // decode steps up to this many sequences keep the GEMV

// --- small kernels ------------------------------------------------------------

// h[row] = E[tok[row]] (f32). Out-of-range ids write zeros and raise *err.
// qy (hid % 32 == 0): also the first layer's quantised q/k/v input. Grid
// (rows, ceil(hid / 256)) of 256 threads, one element each: a row's loads
// are all in flight at once (one CTA looping over the row waited for each
// 256-element step in turn).
constexpr int kEmbedThreads = 256;
__global__ void __launch_bounds__(kEmbedThreads) embed_kernel(const void* E, int e_f16, int64_t vocab, int64_t hid,
                                                              const int32_t* tok, float* h, int* err, QxImage qy) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x;
    const int32_t t = tok[row];
    const bool ok = t >= 0 && t < vocab;
    if (!ok && threadIdx.x == 0 && blockIdx.y == 0) atomicExch(err, kErrTokenRange);
    const int64_t i = (int64_t)blockIdx.y * kEmbedThreads + threadIdx.x;
    if (i >= hid) return;  // whole warps when hid % 32 == 0
    float v = 0.0f;
    if (ok) v = e_f16 ? __half2float(static_cast<const __half*>(E)[(int64_t)t * hid + i])
                      : static_cast<const float*>(E)[(int64_t)t * hid + i];
    h[(int64_t)row * hid + i] = v;
    if (qy.data) qx_write_group(qy, row, i >> 5, (int)(i & 31), v, true);
}
inline dim3 embed_grid(int rows, int64_t hid) {
    return dim3((unsigned)rows, (unsigned)((hid + kEmbedThreads - 1) / kEmbedThreads));
}

// ops.rs:77-93 per row; w is f32. d % 4 == 0 and d <= 4 * 256 * kRmsVec: each
// thread keeps its float4s in registers, so the row is read once.
constexpr int kRmsVec = 8;
// out16 (or NULL): also the f16 copy a tensor-core GEMM reads as its operand.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           float* __restrict__ out, int64_t d, float eps,
                                                           __half* __restrict__ out16) {
    __shared__ float sh[8];
    pdl_trigger();
    pdl_wait();
    const int64_t row = blockIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + row * d);
    const float4* wr = reinterpret_cast<const float4*>(w);
    const int n4 = (int)(d / 4);
    float4 v[kRmsVec];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kRmsVec; ++i) {
        const int j = threadIdx.x + i * 256;
        v[i] = j < n4 ? xr[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        ss = fmaf(v[i].x, v[i].x, ss);
        ss = fmaf(v[i].y, v[i].y, ss);
        ss = fmaf(v[i].z, v[i].z, ss);
        ss = fmaf(v[i].w, v[i].w, ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = ss;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += sh[i];
    const float inv = 1.0f / sqrtf(t / (float)d + eps);
    float4* o = reinterpret_cast<float4*>(out + row * d);
#pragma unroll
    for (int i = 0; i < kRmsVec; ++i) {
        const int j = threadIdx.x + i * 256;
        if (j < n4) {
            const float4 g = wr[j];
            const float4 r = make_float4(v[i].x * inv * g.x, v[i].y * inv * g.y, v[i].z * inv * g.z, v[i].w * inv * g.w);
            o[j] = r;
            if (out16) {
                const __half2 lo = __floats2half2_rn(r.x, r.y), hi = __floats2half2_rn(r.z, r.w);
                reinterpret_cast<uint2*>(out16 + row * d)[j] =
                    make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
            }
        }
    }
}

// cos/sin table [max_ctx][D/2] with the CPU formula (ops.rs:131-135)
__global__ void rope_table_kernel(float* cs, float* sn, int max_ctx, int d, float theta) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int half = d / 2;
    if (idx >= (int64_t)max_ctx * half) return;
    const int p = (int)(idx / half), i = (int)(idx % half);
    const float freq = 1.0f / powf(theta, (float)(2 * i) / (float)d);
    const float angle = (float)p * freq;
    float s, c;
    sincosf(angle, &s, &c);
    cs[idx] = c;
    sn[idx] = s;
}

// [parts][rows][per] -> [rows][parts*per]
__global__ void unshard_kernel(const float* in, float* out, int parts, int rows, int64_t per) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t n = (int64_t)parts * rows * per;
    if (i >= n) return;
    const int64_t p = i / (rows * per), r = (i / per) % rows, j = i % per;
    out[r * (parts * per) + p * per + j] = in[i];
}

__global__ void advance_kernel(int* pos) {
    pdl_trigger();
    pdl_wait();
    *pos += 1;
}

// Seeded pseudo-random cache rows (splitmix64 of the element index), |v| < 1.
__global__ void fill_random_kernel(void* dst, int f16, int64_t n, int64_t per_seq, int64_t seq_stride,
                                   uint64_t seed) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint64_t z = seed + (uint64_t)i * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    const float v = (float)(int32_t)(z & 0xFFFFFF) / 8388608.0f - 1.0f;
    const int64_t off = (i / per_seq) * seq_stride + i % per_seq;
    if (f16)
        static_cast<__half*>(dst)[off] = __float2half_rn(v);
    else
        static_cast<float*>(dst)[off] = v;
}

inline unsigned cdiv(int64_t a, int64_t b) { return (unsigned)std::max<int64_t>(1, (a + b - 1) / b); }

}  // namespace

struct LayerW {
    std::unique_ptr<DeviceBuffer> attn_norm, ffn_norm;
    std::unique_ptr<DeviceBuffer> wqkv, wo, wgu, wd;
    std::unique_ptr<DeviceBuffer> kc, vc;
    unsigned set = 0;
};

}  // namespace bc

struct BeaconCudaModel {
    BeaconCudaContext* ctx = nullptr;
    BeaconCudaModelConfig cfg{};
    int tp = 1, rank = 0;
    int h_loc = 0, kv_loc = 0, f_loc = 0;
    int64_t v_loc = 0, v0 = 0, qd = 0, kd = 0, qkv_n = 0;
    int32_t wdtype = -1;
    int32_t kind_dtype[5] = {-1, -1, -1, -1, -1};  // block type of lm_head, q/k/v, o, gate/up, down
    bc::QLayout Lqkv, Lo, Lgu, Ld, Llm;
    std::vector<bc::LayerW> layers;
    std::unique_ptr<bc::DeviceBuffer> embed, final_norm, wlm, rope_cs, rope_sn;
    int32_t embed_dtype = BEACON_CUDA_DTYPE_F16;
    unsigned global_set = 0;
    int max_rows = 1;
    // activations
    std::unique_ptr<bc::DeviceBuffer> act;
    float *h = nullptr, *xn = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *ffn = nullptr;
    float *logits_loc = nullptr, *logits_all = nullptr, *logits = nullptr;
    int32_t *tok = nullptr, *next = nullptr;
    int* pos_dev = nullptr;
    int* err_dev = nullptr;
    // scratch
    bc::GemvScratch gsc;
    std::unique_ptr<bc::DeviceBuffer> gemv_buf, attn_buf;
    std::unique_ptr<bc::DeviceBuffer> x16;  // f16 activations of the prefill GEMM
    std::unique_ptr<bc::DeviceBuffer> w16;  // f16 weights of one layer linear (dequantise-first GEMM)
    // f16 copies of every layer linear, kept between prefills when they fit
    // the budget (w16_keep: 0 undecided, 1 kept, -1 over budget); filled by
    // the first prefill that uses each, dropped by any weight upload
    std::map<const void*, std::unique_ptr<bc::DeviceBuffer>> w16_kept;
    std::map<const void*, bool> w16_filled;
    int w16_keep = 0;
    // decode hand-off of quantised activations between kernels (one GPU, fast
    // numerics, batch <= 8): the hidden-state image (q/k/v, gate/up, lm_head
    // inputs, with per-block sums of squares for their RMSNorm) and the
    // attention-output image (o input)
    std::unique_ptr<bc::DeviceBuffer> qx_buf;
    uint8_t *qx_h = nullptr, *qx_a = nullptr, *qx_f = nullptr;
    float* qx_h_ss = nullptr;
    int attn_nsplit = 1;
    float *pacc = nullptr, *pm = nullptr, *pl = nullptr;
    int* attn_cnt = nullptr;
    size_t attn_cnt_count = 0;
    std::unique_ptr<bc::DeviceBuffer> argmax_buf;
    bool pdl = true;  // programmatic dependent launch between the step's kernels
    // rows above which a fast-numerics linear runs as the tensor-core GEMM
    // (prefill: 16; a decode step of up to kDecodeGemvRows sequences keeps the
    // persistent GEMV in 8-row launches, which stream the weights at a far
    // higher rate than the GEMM's 256-row tiles filled by a few rows)
    int gemm_rows = 16;
    bc::ArgmaxSummary* argmax_scratch = nullptr;
    // device sampling: [work rows | argmax summaries | uniforms | previous tokens | next tokens]
    std::unique_ptr<bc::DeviceBuffer> samp_buf;
    // host staging (pinned)
    int32_t* h_stage = nullptr;  // [0] = position, [1..] tokens
    int32_t* h_next = nullptr;
    // graphs: key = batch * 2 + autoregressive
    std::map<int, cudaGraphExec_t> graphs;
    std::map<int, int> graph_kernels;  // kernel nodes per captured step
    ~BeaconCudaModel();
};

namespace bc {
namespace {

int gemv_mode(const BeaconCudaModel* m) { return m->cfg.numerics == BEACON_CUDA_NUMERICS_FAST ? MODE_FAST : MODE_F32; }
bool gemv_rtz(const BeaconCudaModel* m) { return m->cfg.numerics == BEACON_CUDA_NUMERICS_REF_RTZ; }

// y = W x over `rows` rows of x, in launches of up to 16 rows (see gemv_rows).
// The quantised-activation hand-off applies to a decode step of the fast
// numerics on one GPU whose consumers all run the persistent GEMV and whose
// attention is the f16-cache kernel (the o input's producer).
bool qx_active(const BeaconCudaModel* m, int rows, bool decode) {
    if (!decode || !m->qx_buf || m->tp != 1 || gemv_mode(m) != MODE_FAST || rows > 8) return false;
    if (m->cfg.kv_dtype != BEACON_CUDA_DTYPE_F16) return false;
    for (const QLayout* L : {&m->Lqkv, &m->Lo, &m->Lgu, &m->Ld, &m->Llm})
        if (!plan_linear(m->ctx, *L, rows, MODE_FAST).v3) return false;
    return true;
}

// which: 0 the hidden-state image (norm_w: the consumer's RMSNorm weight), 1 the attention-output image,
// 2 the SwiGLU-output image (the down projection's input)
QxImage qx_image(BeaconCudaModel* m, int which, const QLayout& consumer, int rows, const float* norm_w) {
    QxImage q;
    q.data = which == 0 ? m->qx_h : which == 1 ? m->qx_a : m->qx_f;
    q.ss = which == 0 ? m->qx_h_ss : nullptr;
    q.kspan = (int)consumer.k_pad;
    q.bpad = plan_linear(m->ctx, consumer, rows, MODE_FAST).bpad;
    q.perm = consumer.dtype == BEACON_CUDA_DTYPE_Q4_0 ? 1 : 0;
    q.norm_w = norm_w;
    return q;
}

// Rows per GEMV launch: up to 16. Up to 8 rows whose persistent plan does
// not fit (staged activations of a long K) go in 4-, 2- or 1-row launches
// that take the persistent kernel -- each reads the weights again, still far
// faster than the tiled kernel -- else the tiled kernel takes them all.
int gemv_rows(const BeaconCudaModel* m, const QLayout& L, int rem) {
    return linear_chunk_rows(m->ctx, L, rem, gemv_mode(m));
}

// From this many rows a layer linear's tensor-core GEMM dequantises the
// weights once into f16 rows and loads them by TMA (the fused dequantisation
// would be repeated by every 256-row tile: 8 times at 2048 rows).
constexpr int kDequantFirstRows = 1024;

// The f16 weights of the dequantise-first GEMM for weight w. When the f16
// copies of every layer linear fit 40% of the free device memory (decided at
// the first use) each linear keeps its own copy, dequantised by its first
// prefill only (*ready: already filled); otherwise one scratch sized for the
// largest layer linear is refilled by every launch. Allocated outside stream
// capture only: NULL while capturing (the fused form runs then).
void* dequant_first_scratch(BeaconCudaModel* m, const QLayout& L, const void* w, cudaStream_t s, bool* ready) {
    *ready = false;
    if (&L == &m->Llm) return nullptr;  // vocab-sized: not worth the memory
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    BC_CUDA(cudaStreamIsCapturing(s, &cs));
    if (m->w16_keep == 0 && cs == cudaStreamCaptureStatusNone) {
        size_t total = 0;
        for (const QLayout* l : {&m->Lqkv, &m->Lo, &m->Lgu, &m->Ld})
            if (qgemm_tc_supported(*l)) total += qgemm_tc_weight_scratch_bytes(*l);
        total *= m->layers.size();
        size_t free_b = 0, total_b = 0;
        BC_CUDA(cudaMemGetInfo(&free_b, &total_b));
        m->w16_keep = total > 0 && total <= free_b / 10 * 4 ? 1 : -1;
    }
    if (m->w16_keep == 1) {
        auto it = m->w16_kept.find(w);
        if (it != m->w16_kept.end()) {
            *ready = m->w16_filled[w];
            m->w16_filled[w] = true;  // the launch this returns for fills it, in stream order
            return it->second->ptr;
        }
        if (cs != cudaStreamCaptureStatusNone) return nullptr;
        auto buf = std::make_unique<DeviceBuffer>(qgemm_tc_weight_scratch_bytes(L));
        void* p = buf->ptr;
        m->w16_kept[w] = std::move(buf);
        m->w16_filled[w] = true;
        return p;
    }
    if (!m->w16) {
        if (cs != cudaStreamCaptureStatusNone) return nullptr;
        size_t bytes = 0;
        for (const QLayout* l : {&m->Lqkv, &m->Lo, &m->Lgu, &m->Ld})
            if (qgemm_tc_supported(*l)) bytes = std::max(bytes, qgemm_tc_weight_scratch_bytes(*l));
        if (bytes == 0) return nullptr;
        m->w16 = std::make_unique<DeviceBuffer>(bytes);
    }
    return m->w16->bytes >= qgemm_tc_weight_scratch_bytes(L) ? m->w16->ptr : nullptr;
}

// qkv (EPI_QKV only): destinations; chunk r0 is model row r0 onwards.
// More than 16 rows in the fast numerics run as one tensor-core GEMM.
bool takes_gemm(const BeaconCudaModel* m, const QLayout& L, int rows) {
    return rows > m->gemm_rows && gemv_mode(m) == MODE_FAST && qgemm_tc_supported(L);
}

// The tensor-core GEMM of a linear; x is f32, or f16 when x_f16.
void gemm_linear(BeaconCudaModel* m, const QLayout& L, const void* w, const void* x, bool x_f16, int64_t x_ld,
                 int rows, float* y, int64_t y_ld, int epi, const float* res, int64_t res_ld, cudaStream_t s,
                 const QkvEpi* qkv) {
    QkvEpi qe;
    if (qkv) {
        qe = *qkv;
        qe.row0 = 0;
    }
    bool ready = false;
    void* w16 = rows >= kDequantFirstRows ? dequant_first_scratch(m, L, w, s, &ready) : nullptr;
    launch_qgemm_tc(L, w, x, x_f16, x_ld, rows, y, y_ld, epi, res, res_ld, false, m->err_dev, s, m->x16->ptr,
                    qkv ? &qe : nullptr, w16, ready);
}

void linear(BeaconCudaModel* m, const QLayout& L, const void* w, const float* x, int64_t x_ld, int rows, float* y,
            int64_t y_ld, int epi, const float* res, int64_t res_ld, cudaStream_t s, const QkvEpi* qkv = nullptr,
            const QxImage* qx = nullptr, const QxImage* qy = nullptr) {
    if (takes_gemm(m, L, rows)) return gemm_linear(m, L, w, x, false, x_ld, rows, y, y_ld, epi, res, res_ld, s, qkv);
    for (int r0 = 0, b = 0; r0 < rows; r0 += b) {
        b = gemv_rows(m, L, rows - r0);
        LinearPlan pl = plan_linear(m->ctx, L, b, gemv_mode(m));
        QkvEpi qe;
        if (qkv) {
            qe = *qkv;
            qe.row0 = r0;
        }
        launch_linear(pl, L, w, x + (int64_t)r0 * x_ld, false, x_ld, b, y + (int64_t)r0 * y_ld, y_ld, epi,
                      res ? res + (int64_t)r0 * res_ld : nullptr, res_ld, gemv_mode(m), gemv_rtz(m), m->gsc, s,
                      nullptr, 0.0f, m->pdl, qkv ? &qe : nullptr, r0 == 0 ? qx : nullptr, r0 == 0 ? qy : nullptr);
    }
}

void rmsnorm(BeaconCudaModel* m, const float* x, const float* w, float* out, int rows, cudaStream_t s,
             __half* out16 = nullptr) {
    launch_kernel(rmsnorm_rows_kernel, dim3(rows), dim3(256), 0, s, m->pdl, x, w, out, (int64_t)m->cfg.hidden_size,
                  m->cfg.rms_norm_eps, out16);
}

// y = W rmsnorm(x, norm_w): the norm rides in the persistent GEMV's staging
// when every row chunk takes that kernel, otherwise it runs on its own first.
void normed_linear(BeaconCudaModel* m, const QLayout& L, const void* w, const float* x, const float* norm_w, int rows,
                   float* y, int64_t y_ld, int epi, cudaStream_t s, const QkvEpi* qkv = nullptr,
                   const QxImage* qx = nullptr, const QxImage* qy = nullptr) {
    const int64_t hid = m->cfg.hidden_size;
    // the tensor-core GEMM takes the rows: normalise first, the norm writing
    // the GEMM's f16 operand as well (no separate conversion)
    if (takes_gemm(m, L, rows) && hid % 8 == 0) {
        __half* x16 = static_cast<__half*>(m->x16->ptr);
        rmsnorm(m, x, norm_w, m->xn, rows, s, x16);
        gemm_linear(m, L, w, x16, true, hid, rows, y, y_ld, epi, nullptr, 0, s, qkv);
        return;
    }
    bool fused = !takes_gemm(m, L, rows);
    for (int r0 = 0, b = 0; r0 < rows && fused; r0 += b) {
        b = gemv_rows(m, L, rows - r0);
        fused = plan_linear(m->ctx, L, b, gemv_mode(m)).v3;
    }
    if (!fused) {
        rmsnorm(m, x, norm_w, m->xn, rows, s);
        linear(m, L, w, m->xn, hid, rows, y, y_ld, epi, nullptr, 0, s, qkv);
        return;
    }
    for (int r0 = 0, b = 0; r0 < rows; r0 += b) {
        b = gemv_rows(m, L, rows - r0);
        LinearPlan pl = plan_linear(m->ctx, L, b, gemv_mode(m));
        QkvEpi qe;
        if (qkv) {
            qe = *qkv;
            qe.row0 = r0;
        }
        launch_linear(pl, L, w, x + (int64_t)r0 * hid, false, hid, b, y + (int64_t)r0 * y_ld, y_ld, epi, nullptr, 0,
                      gemv_mode(m), gemv_rtz(m), m->gsc, s, norm_w, m->cfg.rms_norm_eps, m->pdl, qkv ? &qe : nullptr,
                      r0 == 0 ? qx : nullptr, r0 == 0 ? qy : nullptr);
    }
}

// One pass of the decoder over `rows` rows that are either B sequences at
// one position (decode) or consecutive tokens of sequence 0 (prefill chunk).
// pos_ptr != nullptr: positions come from device memory (graph capture).
// lm_rows: rows the final norm + lm_head run on -- all `rows` (-1), only the
// last (1: a prefill chunk whose logits nobody reads, where time to first
// token needs only the last row's argmax) or none (0: an earlier chunk).
void run_layers(BeaconCudaModel* m, int rows, bool decode, const int* pos_ptr, int pos_imm, cudaStream_t s,
                int lm_rows = -1) {
    m->gemm_rows = decode ? kDecodeGemvRows : 16;
    const auto& c = m->cfg;
    const int64_t hid = c.hidden_size;
    const int D = c.head_dim;
    const bool f16kv = c.kv_dtype == BEACON_CUDA_DTYPE_F16;
    const int64_t cache_sb = (int64_t)c.max_context * m->kd;
    const bool qxa = qx_active(m, rows, decode);
    for (int li = 0; li < c.num_layers; ++li) {
        LayerW& L = m->layers[li];
        const float* attn_nw = static_cast<const float*>(L.attn_norm->ptr);
        const float* ffn_nw = static_cast<const float*>(L.ffn_norm->ptr);
        {
            // q/k/v projection with RoPE and the KV cache write in its epilogue
            QkvEpi qe;
            qe.q = m->q;
            qe.kc = L.kc->ptr;
            qe.vc = L.vc->ptr;
            qe.kv_f16 = f16kv ? 1 : 0;
            qe.cs = static_cast<const float*>(m->rope_cs->ptr);
            qe.sn = static_cast<const float*>(m->rope_sn->ptr);
            qe.qd = (int)m->qd;
            qe.kd = (int)m->kd;
            qe.d = D;
            qe.cache_sb = cache_sb;
            qe.pos_ptr = pos_ptr;
            qe.pos_imm = pos_imm;
            qe.pos_step = decode ? 0 : 1;
            qe.seq_step = decode ? 1 : 0;
            qe.max_ctx = (int)c.max_context;
            qe.err = m->err_dev;
            const QxImage in = qxa ? qx_image(m, 0, m->Lqkv, rows, attn_nw) : QxImage{};
            normed_linear(m, m->Lqkv, L.wqkv->ptr, m->h, attn_nw, rows, m->qkv, m->qkv_n, EPI_QKV, s, &qe,
                          qxa ? &in : nullptr);
        }
        const float scale = 1.0f / sqrtf((float)D);  // engine.rs:415
        bool o16 = false;  // the attention also wrote the o GEMM's f16 operand
        if (decode) {
            DecodeAttnArgs a{};
            a.q = m->q;
            a.k_cache = L.kc->ptr;
            a.v_cache = L.vc->ptr;
            a.kv_f16 = f16kv;
            a.cache_sb = cache_sb;
            a.batch = rows;
            a.heads = m->h_loc;
            a.kv_heads = m->kv_loc;
            a.d = D;
            a.pos_ptr = pos_ptr;
            a.kv_len = pos_imm + 1;
            a.max_kv = c.max_context;
            a.scale = scale;
            a.nsplit = f16kv ? decode_bulk_splits(rows, m->kv_loc, m->ctx->sm_count) : m->attn_nsplit;
            a.counters = m->attn_cnt;
            a.err = m->err_dev;
            a.part_acc = m->pacc;
            a.part_m = m->pm;
            a.part_l = m->pl;
            a.out = m->attn;
            if (qxa) a.qy = qx_image(m, 1, m->Lo, rows, nullptr);
            a.tc = gemv_mode(m) == MODE_FAST ? 1 : 0;
            launch_decode_attention(a, s, m->pdl);
        } else {
            AttnRowsArgs a{};
            a.q = m->q;
            a.q_f16 = 0;
            a.k = L.kc->ptr;
            a.v = L.vc->ptr;
            a.kv_f16 = f16kv;
            a.out = m->attn;
            a.batch = 1;
            a.heads = m->h_loc;
            a.kv_heads = m->kv_loc;
            a.sq = rows;
            a.skv = pos_imm + rows;
            a.d = D;
            a.scale = scale;
            a.causal = c.causal_prefill && rows > 1 ? 1 : 0;
            a.q_sb = 0;
            a.q_sh = D;
            a.q_ss = m->qd;
            a.kv_sb = 0;
            a.kv_sh = D;
            a.kv_ss = m->kd;
            a.o_sb = 0;
            a.o_sh = D;
            a.o_ss = m->qd;
            // the o projection's tensor-core GEMM reads an f16 copy the
            // attention writes beside its f32 output
            if (takes_gemm(m, m->Lo, rows) && m->qd % 8 == 0) a.out16 = m->x16->ptr;
            // the tiled kernel in the fast numerics; the row kernel keeps the
            // reference's summation order for the exact ones
            if (gemv_mode(m) == MODE_FAST && prefill_attention_supported(a))
                o16 = launch_prefill_attention(a, s);
            else
                launch_attention_rows(a, s);
        }
        // h = h + Wo attn ; under TP only rank 0 adds the residual, then sum
        const bool r0 = m->rank == 0;
        {
            const QxImage in = qxa ? qx_image(m, 1, m->Lo, rows, nullptr) : QxImage{};
            const QxImage out = qxa ? qx_image(m, 0, m->Lgu, rows, ffn_nw) : QxImage{};
            if (o16)
                gemm_linear(m, m->Lo, L.wo->ptr, m->x16->ptr, true, m->qd, rows, m->h, hid, r0 ? EPI_ADD : EPI_STORE,
                            r0 ? m->h : nullptr, hid, s, nullptr);
            else
                linear(m, m->Lo, L.wo->ptr, m->attn, m->qd, rows, m->h, hid, r0 ? EPI_ADD : EPI_STORE,
                       r0 ? m->h : nullptr, hid, s, nullptr, qxa ? &in : nullptr, qxa ? &out : nullptr);
        }
        comm_all_reduce_sum(m->ctx, m->h, (size_t)rows * hid, s);
        {
            const QxImage in = qxa ? qx_image(m, 0, m->Lgu, rows, ffn_nw) : QxImage{};
            const QxImage out = qxa ? qx_image(m, 2, m->Ld, rows, nullptr) : QxImage{};
            normed_linear(m, m->Lgu, L.wgu->ptr, m->h, ffn_nw, rows, m->ffn, m->f_loc, EPI_SWIGLU, s, nullptr,
                          qxa ? &in : nullptr, qxa ? &out : nullptr);
        }
        {
            // the next consumer of h: the next layer's q/k/v, or the lm_head after the last layer
            const bool last = li + 1 == c.num_layers;
            const float* next_nw = last ? static_cast<const float*>(m->final_norm->ptr)
                                        : static_cast<const float*>(m->layers[li + 1].attn_norm->ptr);
            const QxImage in = qxa ? qx_image(m, 2, m->Ld, rows, nullptr) : QxImage{};
            const QxImage out = qxa ? qx_image(m, 0, last ? m->Llm : m->Lqkv, rows, next_nw) : QxImage{};
            linear(m, m->Ld, L.wd->ptr, m->ffn, m->f_loc, rows, m->h, hid, r0 ? EPI_ADD : EPI_STORE,
                   r0 ? m->h : nullptr, hid, s, nullptr, qxa ? &in : nullptr, qxa ? &out : nullptr);
        }
        comm_all_reduce_sum(m->ctx, m->h, (size_t)rows * hid, s);
    }
    // final norm + lm_head (engine.rs:230-234)
    if (lm_rows == 0) return;
    const int lr = lm_rows < 0 ? rows : 1;
    {
        const float* fnw = static_cast<const float*>(m->final_norm->ptr);
        const QxImage in = qxa && lm_rows < 0 ? qx_image(m, 0, m->Llm, rows, fnw) : QxImage{};
        normed_linear(m, m->Llm, m->wlm->ptr, m->h + (int64_t)(rows - lr) * hid, fnw, lr, m->logits_loc, m->v_loc,
                      EPI_STORE, s, nullptr, qxa && lm_rows < 0 ? &in : nullptr);
    }
    if (m->tp > 1) {
        comm_all_gather(m->ctx, m->logits_loc, m->logits_all, (size_t)lr * m->v_loc, s);
    }
}

// logits [rows][V] (unsharded) and argmax -> next (and tok, for the next step)
void finish_logits(BeaconCudaModel* m, int rows, bool need_full_logits, bool feed_back, cudaStream_t s) {
    const float* src = m->tp > 1 ? m->logits_all : m->logits_loc;
    launch_argmax(src, m->v_loc, m->tp, rows, m->next, feed_back ? m->tok : nullptr, m->argmax_scratch, s, m->pdl);
    if (need_full_logits && m->tp > 1)
        launch_kernel(unshard_kernel, dim3(cdiv((int64_t)rows * m->v_loc * m->tp, 256)), dim3(256), 0, s, m->pdl,
                      (const float*)m->logits_all, m->logits, (int)m->tp, rows, (int64_t)m->v_loc);
}

float* full_logits(BeaconCudaModel* m) { return m->tp > 1 ? m->logits : m->logits_loc; }

void decode_body(BeaconCudaModel* m, int batch, bool autoregressive, cudaStream_t s) {
    const QxImage qy = qx_active(m, batch, true)
                           ? qx_image(m, 0, m->Lqkv, batch, static_cast<const float*>(m->layers[0].attn_norm->ptr))
                           : QxImage{};
    launch_kernel(embed_kernel, embed_grid(batch, m->cfg.hidden_size), dim3(kEmbedThreads), 0, s, m->pdl,
                  (const void*)m->embed->ptr,
                  (int)(m->embed_dtype == BEACON_CUDA_DTYPE_F16), (int64_t)m->cfg.vocab_size,
                  (int64_t)m->cfg.hidden_size, (const int32_t*)m->tok, m->h, m->err_dev, qy);
    run_layers(m, batch, true, m->pos_dev, 0, s);
    finish_logits(m, batch, m->tp > 1, autoregressive, s);
    if (autoregressive) launch_kernel(advance_kernel, dim3(1), dim3(1), 0, s, m->pdl, m->pos_dev);
}

void check_ready(const BeaconCudaModel* m) {
    const unsigned layer_all = (1u << 9) - 1;
    if ((m->global_set & 7u) != 7u) invalid("model: embed / final_norm / lm_head not set");
    for (size_t i = 0; i < m->layers.size(); ++i)
        if (m->layers[i].set != layer_all) invalid("model: layer " + std::to_string(i) + " has unset weights");
}

// Reads the model's error word after the stream's work (synchronises). A
// bounded wait that gave up leaves arrival counters of the warps that never
// arrived: they are re-zeroed, so the next step starts clean.
void check_err(BeaconCudaModel* m, cudaStream_t s) {
    int herr = 0;
    BC_CUDA(cudaMemcpyAsync(&herr, m->err_dev, sizeof(int), cudaMemcpyDeviceToHost, s));
    BC_CUDA(cudaStreamSynchronize(s));
    if (!herr) return;
    BC_CUDA(cudaMemsetAsync(m->err_dev, 0, sizeof(int), s));
    if (herr == kErrAttnWait || herr == kErrGemmWait || herr == kErrGemvWait) {
        if (m->gsc.counters)
            BC_CUDA(cudaMemsetAsync(m->gsc.counters, 0, (size_t)m->gsc.counter_count * sizeof(int), s));
        if (m->attn_cnt)
            BC_CUDA(cudaMemsetAsync(m->attn_cnt, 0, (size_t)m->attn_cnt_count * sizeof(int), s));
        BC_CUDA(cudaStreamSynchronize(s));
        const char* what = herr == kErrAttnWait   ? "decode attention: a bounded wait for its copies gave up"
                           : herr == kErrGemmWait ? "tensor-core GEMM: a bounded pipeline wait gave up"
                                                  : "dequant-GEMV: a bounded wait for its weight tiles gave up";
        fail(BEACON_CUDA_ERR_DEVICE_TIMEOUT, std::string(what) + "; the step's outputs are invalid");
    }
    BC_CUDA(cudaStreamSynchronize(s));
    if (herr == kErrContext) fail(BEACON_CUDA_ERR_CONTEXT_OVERFLOW, "context overflow: KV cache exhausted");
    shape_err("token id out of range for the vocabulary");
}

// Copy the raw GGUF bytes of rows [r0, r0+nr) and columns [c0, c0+nc) of a
// [N, K] tensor into a packed device buffer.
std::unique_ptr<DeviceBuffer> slice_raw(const void* data, bool on_device, int32_t dtype, int64_t K, int64_t r0,
                                        int64_t nr, int64_t c0, int64_t nc, cudaStream_t s) {
    const int64_t bs = block_size(dtype), bb = block_bytes(dtype);
    if (c0 % bs || nc % bs) shape_err("tensor-parallel shard is not a whole number of blocks");
    const int64_t row_bytes = K / bs * bb, off = c0 / bs * bb, w = nc / bs * bb;
    auto buf = std::make_unique<DeviceBuffer>((size_t)(nr * w));
    const uint8_t* src = static_cast<const uint8_t*>(data) + r0 * row_bytes + off;
    BC_CUDA(cudaMemcpy2DAsync(buf->ptr, (size_t)w, src, (size_t)row_bytes, (size_t)w, (size_t)nr,
                              on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
    return buf;
}

void repack_into(BeaconCudaModel* m, const QLayout& L, void* dst, const void* raw, int nibble,
                 const std::vector<int64_t>& row_map, cudaStream_t s) {
    DeviceBuffer map((size_t)L.n_pad * sizeof(int64_t));
    BC_CUDA(cudaMemcpyAsync(map.ptr, row_map.data(), row_map.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s));
    launch_repack(L, static_cast<const uint8_t*>(raw), nibble, static_cast<uint8_t*>(dst),
                  static_cast<const int64_t*>(map.ptr), s);
    BC_CUDA(cudaStreamSynchronize(s));
    (void)m;
}

std::unique_ptr<DeviceBuffer> upload_plain_f32(const void* data, bool on_device, int32_t dtype, int64_t n,
                                               cudaStream_t s) {
    // norm weights -> f32 on the device
    auto out = std::make_unique<DeviceBuffer>((size_t)n * 4);
    std::vector<float> host((size_t)n);
    if (dtype != BEACON_CUDA_DTYPE_F32 && dtype != BEACON_CUDA_DTYPE_F16)
        fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "norm weights must be F32 or F16");
    const size_t eb = dtype == BEACON_CUDA_DTYPE_F32 ? 4 : 2;
    std::vector<uint8_t> raw((size_t)n * eb);
    if (on_device)
        BC_CUDA(cudaMemcpy(raw.data(), data, raw.size(), cudaMemcpyDeviceToHost));
    else
        std::memcpy(raw.data(), data, raw.size());
    for (int64_t i = 0; i < n; ++i) {
        if (eb == 4) {
            std::memcpy(&host[i], &raw[4 * i], 4);
        } else {
            uint16_t hbits;
            std::memcpy(&hbits, &raw[2 * i], 2);
            uint32_t b = f16_to_f32_bits(hbits);
            std::memcpy(&host[i], &b, 4);
        }
    }
    BC_CUDA(cudaMemcpyAsync(out->ptr, host.data(), (size_t)n * 4, cudaMemcpyHostToDevice, s));
    BC_CUDA(cudaStreamSynchronize(s));
    return out;
}

void release_graphs(BeaconCudaModel* m) {
    for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
    m->graphs.clear();
}

}  // namespace
}  // namespace bc

const BeaconCudaModelConfig& bc::model_config_of(const BeaconCudaModel* m) { return m->cfg; }
BeaconCudaContext* bc::model_context_of(const BeaconCudaModel* m) { return m->ctx; }

BeaconCudaModel::~BeaconCudaModel() {
    bc::release_graphs(this);
    if (h_stage) cudaFreeHost(h_stage);
    if (h_next) cudaFreeHost(h_next);
}

using namespace bc;

extern "C" {

int32_t beacon_cuda_model_create(BeaconCudaContext* ctx, const BeaconCudaModelConfig* cfg, BeaconCudaModel** out) {
    return guard([&]() -> int32_t {
        require(ctx && cfg && out, "model_create: null argument");
        set_device(ctx);
        const BeaconCudaModelConfig& c = *cfg;
        if (c.vocab_size <= 0 || c.hidden_size <= 0 || c.num_layers <= 0 || c.num_heads <= 0 ||
            c.num_kv_heads <= 0 || c.head_dim <= 0 || c.intermediate_size <= 0 || c.max_context <= 0 ||
            c.max_batch <= 0)
            invalid("model_create: every dimension must be positive");
        if (c.num_heads % c.num_kv_heads) shape_err("model_create: num_heads % num_kv_heads != 0");
        if (c.num_heads * c.head_dim != c.hidden_size) shape_err("model_create: num_heads * head_dim != hidden_size");
        if (c.head_dim % 32) shape_err("model_create: head_dim must be a multiple of 32");
        if (c.hidden_size % 4 || c.hidden_size > 4 * 256 * kRmsVec)
            shape_err("model_create: hidden_size must be a multiple of 4 and at most 8192");
        if (c.kv_dtype != BEACON_CUDA_DTYPE_F16 && c.kv_dtype != BEACON_CUDA_DTYPE_F32)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "model_create: kv_dtype must be F16 or F32");
        if (c.numerics < 0 || c.numerics > 2) invalid("model_create: unknown numerics");
        const int tp = std::max(1, c.tp_size);
        if (c.tp_rank < 0 || c.tp_rank >= tp) invalid("model_create: bad tp_rank");
        if (tp != ctx->nranks || (tp > 1 && c.tp_rank != ctx->rank))
            invalid("model_create: tp_size/tp_rank must match the context's communicator");
        if (c.num_kv_heads % tp || c.intermediate_size % tp || c.vocab_size % tp)
            shape_err("model_create: kv heads, intermediate size and vocab must divide by tp_size");
        auto m = std::make_unique<BeaconCudaModel>();
        m->ctx = ctx;
        if (std::getenv("BEACON_CUDA_NO_PDL")) m->pdl = false;
        m->cfg = c;
        m->tp = tp;
        m->rank = c.tp_rank;
        m->h_loc = c.num_heads / tp;
        m->kv_loc = c.num_kv_heads / tp;
        m->f_loc = c.intermediate_size / tp;
        m->v_loc = c.vocab_size / tp;
        m->v0 = m->v_loc * m->rank;
        m->qd = (int64_t)m->h_loc * c.head_dim;
        m->kd = (int64_t)m->kv_loc * c.head_dim;
        m->qkv_n = m->qd + 2 * m->kd;
        if (!decode_attention_supported(c.head_dim, c.num_heads / c.num_kv_heads))
            shape_err("model_create: head_dim must be 64 or 128 and heads/kv_heads in {1, 2, 4, 8}");
        m->layers.resize(c.num_layers);
        // KV caches [max_batch][max_ctx][kv_loc][D]
        const size_t kvb = (size_t)c.max_batch * c.max_context * m->kd * (c.kv_dtype == BEACON_CUDA_DTYPE_F16 ? 2 : 4);
        for (auto& L : m->layers) {
            L.kc = std::make_unique<DeviceBuffer>(kvb);
            L.vc = std::make_unique<DeviceBuffer>(kvb);
            BC_CUDA(cudaMemset(L.kc->ptr, 0, kvb));
            BC_CUDA(cudaMemset(L.vc->ptr, 0, kvb));
        }
        // rope table
        const int half = c.head_dim / 2;
        m->rope_cs = std::make_unique<DeviceBuffer>((size_t)c.max_context * half * 4);
        m->rope_sn = std::make_unique<DeviceBuffer>((size_t)c.max_context * half * 4);
        rope_table_kernel<<<cdiv((int64_t)c.max_context * half, 256), 256>>>(
            static_cast<float*>(m->rope_cs->ptr), static_cast<float*>(m->rope_sn->ptr), c.max_context, c.head_dim,
            c.rope_theta);
        BC_LAUNCHED("rope_table_kernel");
        // activations
        m->max_rows = std::max(c.max_batch, std::min(c.max_context, kPrefillChunk));
        const int64_t R = m->max_rows;
        const int64_t Vt = (int64_t)m->v_loc * tp;
        size_t floats = 0;
        auto carve = [&](int64_t n) {
            size_t off = floats;
            floats += (size_t)((n + 63) / 64 * 64);
            return off;
        };
        size_t o_h = carve(R * c.hidden_size), o_xn = carve(R * c.hidden_size), o_qkv = carve(R * m->qkv_n),
               o_q = carve(R * m->qd), o_attn = carve(R * m->qd), o_ffn = carve(R * m->f_loc),
               o_ll = carve(R * m->v_loc), o_la = carve(tp > 1 ? R * Vt : 64), o_lg = carve(tp > 1 ? R * Vt : 64),
               o_tok = carve(R), o_next = carve(R), o_pos = carve(64);
        m->act = std::make_unique<DeviceBuffer>(floats * 4);
        // f16 activations of the prefill GEMM (largest K: hidden, q width or FFN shard)
        m->x16 = std::make_unique<DeviceBuffer>(
            qgemm_tc_scratch_bytes(R, std::max<int64_t>(c.hidden_size, std::max<int64_t>(m->qd, m->f_loc))));
        BC_CUDA(cudaMemset(m->act->ptr, 0, floats * 4));
        float* base = static_cast<float*>(m->act->ptr);
        m->h = base + o_h;
        m->xn = base + o_xn;
        m->qkv = base + o_qkv;
        m->q = base + o_q;
        m->attn = base + o_attn;
        m->ffn = base + o_ffn;
        m->logits_loc = base + o_ll;
        m->logits_all = base + o_la;
        m->logits = base + o_lg;
        m->tok = reinterpret_cast<int32_t*>(base + o_tok);
        m->next = reinterpret_cast<int32_t*>(base + o_next);
        m->pos_dev = reinterpret_cast<int*>(base + o_pos);
        m->err_dev = m->pos_dev + 16;
        // attention split scratch (decode)
        m->attn_nsplit = plan_decode_splits(c.max_batch, m->kv_loc, c.max_context, ctx->sm_count, 64);
        // partial rows (head, split) of either decode kernel, then the f16
        // kernel's arrival counters (zero at rest)
        const size_t pa = std::max((size_t)c.max_batch * m->h_loc * m->attn_nsplit,
                                   decode_bulk_scratch_floats((int)c.max_batch, (int)m->h_loc, (int)m->kv_loc,
                                                              (int)c.head_dim, ctx->sm_count) /
                                       (size_t)(c.head_dim + 2));
        const size_t ncnt = (size_t)c.max_batch * m->kv_loc;
        m->attn_buf = std::make_unique<DeviceBuffer>((pa * c.head_dim + 2 * pa) * 4 + ncnt * 4);
        m->pacc = static_cast<float*>(m->attn_buf->ptr);
        m->pm = m->pacc + pa * c.head_dim;
        m->pl = m->pm + pa;
        m->attn_cnt = reinterpret_cast<int*>(m->pl + pa);
        m->attn_cnt_count = ncnt;
        BC_CUDA(cudaMemset(m->attn_cnt, 0, ncnt * 4));
        if (tp == 1 && c.hidden_size % 32 == 0) {
            const int64_t kh = (c.hidden_size + 255) / 256 * 256, ka = (m->qd + 255) / 256 * 256,
                          kf = (m->f_loc + 255) / 256 * 256;  // the down projection's k_pad
            auto image_bytes = [](int64_t kspan) { return (size_t)8 * kspan * 2 + (size_t)8 * (kspan / 32) * 8; };
            const size_t img_h = image_bytes(kh), img_a = image_bytes(ka), img_f = image_bytes(kf);
            const size_t ss_bytes = (size_t)8 * (kh / 32) * 4;
            const size_t total = img_h + img_a + img_f + ss_bytes;
            m->qx_buf = std::make_unique<DeviceBuffer>(total);
            BC_CUDA(cudaMemset(m->qx_buf->ptr, 0, total));
            m->qx_h = static_cast<uint8_t*>(m->qx_buf->ptr);
            m->qx_a = m->qx_h + img_h;
            m->qx_f = m->qx_a + img_a;
            m->qx_h_ss = reinterpret_cast<float*>(m->qx_f + img_f);
        }
        const size_t na = argmax_scratch_count(m->v_loc, tp, (int)R);
        m->argmax_buf = std::make_unique<DeviceBuffer>(na * sizeof(ArgmaxSummary));
        m->argmax_scratch = static_cast<ArgmaxSummary*>(m->argmax_buf->ptr);
        BC_CUDA(cudaMallocHost(&m->h_stage, (size_t)(R + 1) * 4));
        BC_CUDA(cudaMallocHost(&m->h_next, (size_t)R * 4));
        BC_CUDA(cudaDeviceSynchronize());
        *out = m.release();
        return BEACON_CUDA_OK;
    });
}

void beacon_cuda_model_destroy(BeaconCudaModel* model) {
    if (!model) return;
    cudaSetDevice(model->ctx->device);
    cudaDeviceSynchronize();
    delete model;
}

int32_t beacon_cuda_model_set_weight(BeaconCudaModel* m, int32_t layer, int32_t slot, const void* data, int32_t dtype,
                                     int32_t nibble_order, int32_t on_device) {
    return guard([&]() -> int32_t {
        require(m && data, "model_set_weight: null argument");
        set_device(m->ctx);
        release_graphs(m);
        if (!m->w16_kept.empty()) BC_CUDA(cudaDeviceSynchronize());  // no queued prefill still reads them
        m->w16_kept.clear();
        m->w16_filled.clear();
        m->w16_keep = 0;
        const auto& c = m->cfg;
        cudaStream_t s = m->ctx->internal;
        const bool dev = on_device != 0;
        const int64_t H = c.hidden_size, D = c.head_dim;
        // One tile layout per projection kind serves every layer, and q/k/v
        // (and gate/up) share one fused tile: each kind needs one block type
        // across the model. Anything else is refused rather than misread.
        auto quant_check = [&]() {
            if (!is_quantized(dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "linear weights must be GGUF blocks");
            if (m->wdtype < 0) {
                m->wdtype = dtype;
            }
            const int kind = slot == BEACON_CUDA_W_LM_HEAD ? 0
                             : (slot == BEACON_CUDA_W_Q || slot == BEACON_CUDA_W_K || slot == BEACON_CUDA_W_V) ? 1
                             : slot == BEACON_CUDA_W_O ? 2
                             : (slot == BEACON_CUDA_W_GATE || slot == BEACON_CUDA_W_UP) ? 3 : 4;
            if (m->kind_dtype[kind] >= 0 && m->kind_dtype[kind] != dtype)
                fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE,
                     "model_set_weight: block type " + std::to_string(dtype) + " after " +
                         std::to_string(m->kind_dtype[kind]) +
                         ": q/k/v, o, gate/up and down each need one block type across all layers");
            m->kind_dtype[kind] = dtype;
        };
        auto identity_map = [](const QLayout& L, int64_t r0, int64_t nr, int64_t src0) {
            std::vector<int64_t> map((size_t)L.n_pad, -2);
            for (int64_t r = 0; r < nr; ++r) map[(size_t)(r0 + r)] = src0 + r;
            return map;
        };
        if (slot == BEACON_CUDA_W_EMBED) {
            if (dtype != BEACON_CUDA_DTYPE_F16 && dtype != BEACON_CUDA_DTYPE_F32)
                fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "embedding must be F16 or F32");
            const size_t n = (size_t)c.vocab_size * H * (dtype == BEACON_CUDA_DTYPE_F16 ? 2 : 4);
            m->embed = std::make_unique<DeviceBuffer>(n);
            BC_CUDA(cudaMemcpy(m->embed->ptr, data, n, dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
            m->embed_dtype = dtype;
            m->global_set |= 1u;
            return BEACON_CUDA_OK;
        }
        if (slot == BEACON_CUDA_W_FINAL_NORM) {
            m->final_norm = upload_plain_f32(data, dev, dtype, H, s);
            m->global_set |= 2u;
            return BEACON_CUDA_OK;
        }
        if (slot == BEACON_CUDA_W_LM_HEAD) {
            quant_check();
            m->Llm = make_qlayout(dtype, m->v_loc, H);
            auto raw = slice_raw(data, dev, dtype, H, m->v0, m->v_loc, 0, H, s);
            m->wlm = std::make_unique<DeviceBuffer>((size_t)m->Llm.total_bytes());
            repack_into(m, m->Llm, m->wlm->ptr, raw->ptr, nibble_order, identity_map(m->Llm, 0, m->v_loc, 0), s);
            m->global_set |= 4u;
            return BEACON_CUDA_OK;
        }
        if (layer < 0 || layer >= c.num_layers) invalid("model_set_weight: bad layer");
        LayerW& L = m->layers[layer];
        switch (slot) {
            case BEACON_CUDA_W_ATTN_NORM:
                L.attn_norm = upload_plain_f32(data, dev, dtype, H, s);
                L.set |= 1u << 0;
                break;
            case BEACON_CUDA_W_FFN_NORM:
                L.ffn_norm = upload_plain_f32(data, dev, dtype, H, s);
                L.set |= 1u << 1;
                break;
            case BEACON_CUDA_W_Q:
            case BEACON_CUDA_W_K:
            case BEACON_CUDA_W_V: {
                quant_check();
                m->Lqkv = make_qlayout(dtype, m->qkv_n, H);
                if (!L.wqkv) {
                    L.wqkv = std::make_unique<DeviceBuffer>((size_t)m->Lqkv.total_bytes());
                    BC_CUDA(cudaMemset(L.wqkv->ptr, 0, (size_t)m->Lqkv.total_bytes()));
                }
                int64_t src0, nr, dst0;
                if (slot == BEACON_CUDA_W_Q) {
                    src0 = (int64_t)m->rank * m->h_loc * D; nr = m->qd; dst0 = 0;
                } else {
                    src0 = (int64_t)m->rank * m->kv_loc * D; nr = m->kd;
                    dst0 = slot == BEACON_CUDA_W_K ? m->qd : m->qd + m->kd;
                }
                auto raw = slice_raw(data, dev, dtype, H, src0, nr, 0, H, s);
                repack_into(m, m->Lqkv, L.wqkv->ptr, raw->ptr, nibble_order, identity_map(m->Lqkv, dst0, nr, 0), s);
                L.set |= 1u << (2 + slot - BEACON_CUDA_W_Q);
                break;
            }
            case BEACON_CUDA_W_O: {  // row-split: columns of this rank's heads
                quant_check();
                m->Lo = make_qlayout(dtype, H, m->qd);
                auto raw = slice_raw(data, dev, dtype, (int64_t)c.num_heads * D, 0, H, (int64_t)m->rank * m->qd, m->qd, s);
                L.wo = std::make_unique<DeviceBuffer>((size_t)m->Lo.total_bytes());
                repack_into(m, m->Lo, L.wo->ptr, raw->ptr, nibble_order, identity_map(m->Lo, 0, H, 0), s);
                L.set |= 1u << 5;
                break;
            }
            case BEACON_CUDA_W_GATE:
            case BEACON_CUDA_W_UP: {  // column-split, interleaved per 16 rows
                quant_check();
                const int64_t fl = m->f_loc;
                if (fl % 16) shape_err("intermediate size per rank must be a multiple of 16");
                m->Lgu = make_qlayout(dtype, 2 * fl, H);
                if (!L.wgu) {
                    L.wgu = std::make_unique<DeviceBuffer>((size_t)m->Lgu.total_bytes());
                    BC_CUDA(cudaMemset(L.wgu->ptr, 0, (size_t)m->Lgu.total_bytes()));
                }
                auto raw = slice_raw(data, dev, dtype, H, (int64_t)m->rank * fl, fl, 0, H, s);
                std::vector<int64_t> map((size_t)m->Lgu.n_pad, -2);
                const bool up = slot == BEACON_CUDA_W_UP;
                for (int64_t r = 0; r < m->Lgu.n_pad; ++r) {
                    const int64_t lane = r % 32, f = (r / 32) * 16 + (lane % 16);
                    if ((lane >= 16) == up) map[(size_t)r] = f < fl ? f : -1;
                }
                repack_into(m, m->Lgu, L.wgu->ptr, raw->ptr, nibble_order, map, s);
                L.set |= 1u << (up ? 7 : 6);
                break;
            }
            case BEACON_CUDA_W_DOWN: {  // row-split: columns of this rank's FFN slice
                quant_check();
                m->Ld = make_qlayout(dtype, H, m->f_loc);
                auto raw = slice_raw(data, dev, dtype, c.intermediate_size, 0, H, (int64_t)m->rank * m->f_loc, m->f_loc, s);
                L.wd = std::make_unique<DeviceBuffer>((size_t)m->Ld.total_bytes());
                repack_into(m, m->Ld, L.wd->ptr, raw->ptr, nibble_order, identity_map(m->Ld, 0, H, 0), s);
                L.set |= 1u << 8;
                break;
            }
            default:
                invalid("model_set_weight: unknown slot");
        }
        // (re)size the GEMV split-K scratch for every layout and batch in use
        size_t need_p = 0;
        int64_t need_c = 0;
        for (const QLayout* Lp : {&m->Lqkv, &m->Lo, &m->Lgu, &m->Ld, &m->Llm}) {
            if (Lp->n == 0) continue;
            for (int b = 1; b <= 16; ++b) {
                LinearPlan pl = plan_linear(m->ctx, *Lp, b, gemv_mode(m));
                need_p = std::max(need_p, pl.scratch_floats(b, *Lp));
            }
            // gate/up adds one SwiGLU hand-off counter per two row groups
            need_c = std::max(need_c, Lp->groups() + (Lp == &m->Lgu ? (Lp->groups() + 1) / 2 : 0));
        }
        if (need_p > m->gsc.partial_floats || need_c > m->gsc.counter_count || !m->gsc.err) {
            const size_t pf = std::max(need_p, m->gsc.partial_floats), cc = (size_t)std::max(need_c, m->gsc.counter_count);
            const size_t coff = (pf * 4 + 255) / 256 * 256;
            auto buf = std::make_unique<DeviceBuffer>(coff + cc * 4 + 256);
            BC_CUDA(cudaMemset(buf->ptr, 0, coff + cc * 4 + 256));
            m->gemv_buf = std::move(buf);
            m->gsc.partial = static_cast<float*>(m->gemv_buf->ptr);
            m->gsc.partial_floats = pf;
            m->gsc.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(m->gemv_buf->ptr) + coff);
            m->gsc.counter_count = (int64_t)cc;
            m->gsc.err = m->err_dev;  // GEMV timeouts surface through check_err like every other device error
        }
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_reset(BeaconCudaModel* m) {
    return guard([&]() -> int32_t {
        require(m != nullptr, "model_reset: null argument");
        set_device(m->ctx);
        // Engine::reset_cache only rewinds current_length (engine.rs:176-180);
        // the rows are overwritten before they are read again, but zeroing
        // keeps the literal (non-persisting) mode exact.
        const auto& c = m->cfg;
        const size_t kvb = (size_t)c.max_batch * c.max_context * m->kd * (c.kv_dtype == BEACON_CUDA_DTYPE_F16 ? 2 : 4);
        for (auto& L : m->layers) {
            BC_CUDA(cudaMemset(L.kc->ptr, 0, kvb));
            BC_CUDA(cudaMemset(L.vc->ptr, 0, kvb));
        }
        BC_CUDA(cudaDeviceSynchronize());
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_forward(BeaconCudaModel* m, BeaconCudaStream* stream, const uint32_t* tokens,
                                  int32_t n_tokens, int32_t position, float* logits_out) {
    return guard([&]() -> int32_t {
        require(m && stream && tokens, "model_forward: null argument");
        set_device(m->ctx);
        check_ready(m);
        const auto& c = m->cfg;
        if (n_tokens <= 0) invalid("model_forward: empty token list");
        if (position < 0) invalid("model_forward: negative position");
        if ((int64_t)position + n_tokens > c.max_context) fail(BEACON_CUDA_ERR_CONTEXT_OVERFLOW, "context overflow: KV cache exhausted");
        for (int i = 0; i < n_tokens; ++i)
            if (tokens[i] >= (uint32_t)c.vocab_size) shape_err("embedding index out of bounds for the vocabulary");
        if (!c.kv_persist && n_tokens > m->max_rows)
            invalid("model_forward: the non-persisting cache mode needs the whole prompt in one chunk");
        cudaStream_t s = stream->s;
        if (!c.kv_persist) {
            // cpu_backend.rs:459-460: the cache the engine holds is never
            // written, so every call starts from zeros
            const size_t kvb = (size_t)c.max_batch * c.max_context * m->kd * (c.kv_dtype == BEACON_CUDA_DTYPE_F16 ? 2 : 4);
            for (auto& L : m->layers) {
                BC_CUDA(cudaMemsetAsync(L.kc->ptr, 0, kvb, s));
                BC_CUDA(cudaMemsetAsync(L.vc->ptr, 0, kvb, s));
            }
        }
        const int64_t V = c.vocab_size;
        for (int t0 = 0; t0 < n_tokens; t0 += m->max_rows) {
            const int rows = std::min(m->max_rows, n_tokens - t0);
            for (int i = 0; i < rows; ++i) m->h_stage[i] = (int32_t)tokens[t0 + i];
            BC_CUDA(cudaMemcpyAsync(m->tok, m->h_stage, (size_t)rows * 4, cudaMemcpyHostToDevice, s));
            embed_kernel<<<embed_grid(rows, c.hidden_size), kEmbedThreads, 0, s>>>(
                m->embed->ptr, m->embed_dtype == BEACON_CUDA_DTYPE_F16, V, c.hidden_size, m->tok, m->h, m->err_dev,
                QxImage{});
            BC_LAUNCHED("embed_kernel");
            // without logits_out only the last row of the last chunk reaches the lm_head
            const bool last_chunk = t0 + rows >= n_tokens;
            run_layers(m, rows, false, nullptr, position + t0, s, logits_out ? -1 : (last_chunk ? 1 : 0));
            if (logits_out || last_chunk) finish_logits(m, logits_out ? rows : 1, logits_out != nullptr, false, s);
            if (logits_out)
                BC_CUDA(cudaMemcpyAsync(logits_out + (int64_t)t0 * V, full_logits(m), (size_t)rows * V * 4,
                                        cudaMemcpyDeviceToHost, s));
            BC_CUDA(cudaStreamSynchronize(s));
        }
        check_err(m, s);
        return BEACON_CUDA_OK;
    });
}

static void launch_decode_graph(BeaconCudaModel* m, int batch, bool autoregressive, cudaStream_t s) {
    const int key = batch * 2 + (autoregressive ? 1 : 0);
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        // One eager run first, so kernel modules load outside the capture. The
        // host-fed body only rewrites the same cache rows from the same inputs.
        decode_body(m, batch, false, s);
        BC_CUDA(cudaStreamSynchronize(s));
        cudaGraph_t g = nullptr;
        BC_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        try {
            decode_body(m, batch, autoregressive, s);
        } catch (...) {
            cudaStreamEndCapture(s, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        BC_CUDA(cudaStreamEndCapture(s, &g));
        size_t nn = 0;
        int kernels = 0;
        if (cudaGraphGetNodes(g, nullptr, &nn) == cudaSuccess && nn) {
            std::vector<cudaGraphNode_t> nodes(nn);
            if (cudaGraphGetNodes(g, nodes.data(), &nn) == cudaSuccess)
                for (auto nd : nodes) {
                    cudaGraphNodeType ty;
                    if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++kernels;
                }
        }
        m->graph_kernels[key] = kernels;
        cudaGraphExec_t ge = nullptr;
        cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        cuda_check(e, "cudaGraphInstantiate");
        it = m->graphs.emplace(key, ge).first;
    }
    BC_CUDA(cudaGraphLaunch(it->second, s));
}

int32_t beacon_cuda_model_decode_step(BeaconCudaModel* m, BeaconCudaStream* stream, const uint32_t* tokens,
                                      int32_t batch, int32_t position, uint32_t* next_tokens, float* logits_out) {
    return guard([&]() -> int32_t {
        require(m && stream && tokens, "model_decode_step: null argument");
        set_device(m->ctx);
        check_ready(m);
        const auto& c = m->cfg;
        if (batch <= 0 || batch > c.max_batch) invalid("model_decode_step: batch out of range");
        if (position < 0 || position + 1 > c.max_context) fail(BEACON_CUDA_ERR_CONTEXT_OVERFLOW, "context overflow: KV cache exhausted");
        for (int i = 0; i < batch; ++i)
            if (tokens[i] >= (uint32_t)c.vocab_size) shape_err("embedding index out of bounds for the vocabulary");
        cudaStream_t s = stream->s;
        m->h_stage[0] = position;
        for (int i = 0; i < batch; ++i) m->h_stage[1 + i] = (int32_t)tokens[i];
        BC_CUDA(cudaMemcpyAsync(m->pos_dev, m->h_stage, 4, cudaMemcpyHostToDevice, s));
        BC_CUDA(cudaMemcpyAsync(m->tok, m->h_stage + 1, (size_t)batch * 4, cudaMemcpyHostToDevice, s));
        if (!c.kv_persist) {
            const size_t kvb = (size_t)c.max_batch * c.max_context * m->kd * (c.kv_dtype == BEACON_CUDA_DTYPE_F16 ? 2 : 4);
            for (auto& L : m->layers) {
                BC_CUDA(cudaMemsetAsync(L.kc->ptr, 0, kvb, s));
                BC_CUDA(cudaMemsetAsync(L.vc->ptr, 0, kvb, s));
            }
        }
        launch_decode_graph(m, batch, false, s);
        if (next_tokens) BC_CUDA(cudaMemcpyAsync(m->h_next, m->next, (size_t)batch * 4, cudaMemcpyDeviceToHost, s));
        if (logits_out)
            BC_CUDA(cudaMemcpyAsync(logits_out, full_logits(m), (size_t)batch * c.vocab_size * 4, cudaMemcpyDeviceToHost, s));
        check_err(m, s);  // synchronises the stream
        if (next_tokens)
            for (int i = 0; i < batch; ++i) next_tokens[i] = (uint32_t)m->h_next[i];
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_decode_step_sampled(BeaconCudaModel* m, BeaconCudaStream* stream, const uint32_t* tokens,
                                              int32_t batch, int32_t position, const BeaconCudaSamplingParams* params,
                                              const float* uniforms, const uint32_t* previous, int32_t n_prev,
                                              uint32_t* next_tokens) {
    return guard([&]() -> int32_t {
        require(m && stream && tokens && params && uniforms && next_tokens, "model_decode_step_sampled: null argument");
        require(n_prev >= 0 && (n_prev == 0 || previous), "model_decode_step_sampled: previous tokens missing");
        set_device(m->ctx);
        check_ready(m);
        const auto& c = m->cfg;
        if (batch <= 0 || batch > c.max_batch) invalid("model_decode_step_sampled: batch out of range");
        if (position < 0 || position + 1 > c.max_context)
            fail(BEACON_CUDA_ERR_CONTEXT_OVERFLOW, "context overflow: KV cache exhausted");
        for (int i = 0; i < batch; ++i)
            if (tokens[i] >= (uint32_t)c.vocab_size) shape_err("embedding index out of bounds for the vocabulary");
        if (params->has_top_k && params->top_k < 0) invalid("model_decode_step_sampled: top_k must be >= 0");
        if (!(params->repeat_penalty > 0.0f)) invalid("model_decode_step_sampled: repeat_penalty must be positive");
        const int64_t V = c.vocab_size;
        const size_t work = (sample_scratch_bytes(V, batch) + 255) / 256 * 256;
        const size_t need = work + (size_t)batch * 4 * (2 + (size_t)n_prev) + 256;
        if (!m->samp_buf || m->samp_buf->bytes < need) {
            BC_CUDA(cudaStreamSynchronize(stream->s));
            m->samp_buf = std::make_unique<DeviceBuffer>(need);
        }
        uint8_t* base = static_cast<uint8_t*>(m->samp_buf->ptr);
        float* d_work = reinterpret_cast<float*>(base);
        auto* d_am = reinterpret_cast<ArgmaxSummary*>(base + ((size_t)batch * V * 4 + 255) / 256 * 256);
        float* d_unif = reinterpret_cast<float*>(base + work);
        int32_t* d_prev = reinterpret_cast<int32_t*>(d_unif + batch);
        int32_t* d_next = d_prev + (size_t)batch * n_prev;
        cudaStream_t s = stream->s;
        m->h_stage[0] = position;
        for (int i = 0; i < batch; ++i) m->h_stage[1 + i] = (int32_t)tokens[i];
        BC_CUDA(cudaMemcpyAsync(m->pos_dev, m->h_stage, 4, cudaMemcpyHostToDevice, s));
        BC_CUDA(cudaMemcpyAsync(m->tok, m->h_stage + 1, (size_t)batch * 4, cudaMemcpyHostToDevice, s));
        BC_CUDA(cudaMemcpyAsync(d_unif, uniforms, (size_t)batch * 4, cudaMemcpyHostToDevice, s));
        if (n_prev)
            BC_CUDA(cudaMemcpyAsync(d_prev, previous, (size_t)batch * n_prev * 4, cudaMemcpyHostToDevice, s));
        if (!c.kv_persist) {
            const size_t kvb = (size_t)c.max_batch * c.max_context * m->kd * (c.kv_dtype == BEACON_CUDA_DTYPE_F16 ? 2 : 4);
            for (auto& L : m->layers) {
                BC_CUDA(cudaMemsetAsync(L.kc->ptr, 0, kvb, s));
                BC_CUDA(cudaMemsetAsync(L.vc->ptr, 0, kvb, s));
            }
        }
        launch_decode_graph(m, batch, false, s);
        launch_sample(full_logits(m), V, V, batch, n_prev ? d_prev : nullptr, n_prev, *params, d_unif, d_work, d_next,
                      d_am, s);
        BC_CUDA(cudaMemcpyAsync(m->h_next, d_next, (size_t)batch * 4, cudaMemcpyDeviceToHost, s));
        check_err(m, s);  // synchronises the stream
        for (int i = 0; i < batch; ++i) next_tokens[i] = (uint32_t)m->h_next[i];
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_decode_step_device(BeaconCudaModel* m, BeaconCudaStream* stream, const int32_t* d_tokens,
                                             int32_t batch, int32_t position, int32_t* d_next_tokens,
                                             float* d_logits) {
    return guard([&]() -> int32_t {
        require(m && stream, "model_decode_step_device: null argument");
        set_device(m->ctx);
        check_ready(m);
        const auto& c = m->cfg;
        if (batch <= 0 || batch > c.max_batch) invalid("model_decode_step_device: batch out of range");
        cudaStream_t s = stream->s;
        // d_tokens == NULL and position < 0: continue from the previous step on
        // the device (tokens = last argmax, position advanced in the graph).
        const bool autoregressive = d_tokens == nullptr && position < 0;
        if (!autoregressive) {
            require(d_tokens != nullptr, "model_decode_step_device: tokens required unless continuing");
            if (position + 1 > c.max_context) fail(BEACON_CUDA_ERR_CONTEXT_OVERFLOW, "context overflow: KV cache exhausted");
            m->h_stage[0] = position;
            BC_CUDA(cudaMemcpyAsync(m->pos_dev, m->h_stage, 4, cudaMemcpyHostToDevice, s));
            if (d_tokens != m->tok)
                BC_CUDA(cudaMemcpyAsync(m->tok, d_tokens, (size_t)batch * 4, cudaMemcpyDeviceToDevice, s));
        }
        launch_decode_graph(m, batch, autoregressive, s);
        if (d_next_tokens) BC_CUDA(cudaMemcpyAsync(d_next_tokens, m->next, (size_t)batch * 4, cudaMemcpyDeviceToDevice, s));
        if (d_logits)
            BC_CUDA(cudaMemcpyAsync(d_logits, full_logits(m), (size_t)batch * c.vocab_size * 4, cudaMemcpyDeviceToDevice, s));
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_synchronize(BeaconCudaModel* m, BeaconCudaStream* stream) {
    return guard([&]() -> int32_t {
        require(m && stream, "model_synchronize: null argument");
        set_device(m->ctx);
        check_err(m, stream->s);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_profile_linear(BeaconCudaModel* m, BeaconCudaStream* stream, int32_t slot, int32_t batch,
                                         int32_t iters, float* out_avg_us, uint64_t* out_bytes) {
    return guard([&]() -> int32_t {
        require(m && stream && out_avg_us && out_bytes, "model_profile_linear: null argument");
        set_device(m->ctx);
        check_ready(m);
        if (batch < 1 || batch > m->max_rows || iters < 1) invalid("model_profile_linear: bad batch/iters");
        cudaStream_t s = stream->s;
        const int64_t hid = m->cfg.hidden_size;
        const QLayout* Lp;
        const float* x;
        int64_t x_ld, y_ld, out_n;
        float* y;
        int epi = EPI_STORE;
        switch (slot) {
            case BEACON_CUDA_W_Q: Lp = &m->Lqkv; x = m->xn; x_ld = hid; y = m->qkv; y_ld = m->qkv_n; out_n = m->qkv_n; break;
            case BEACON_CUDA_W_O: Lp = &m->Lo; x = m->attn; x_ld = m->qd; y = m->xn; y_ld = hid; out_n = hid; break;
            case BEACON_CUDA_W_GATE: Lp = &m->Lgu; x = m->xn; x_ld = hid; y = m->ffn; y_ld = m->f_loc; out_n = m->f_loc;
                epi = EPI_SWIGLU; break;
            case BEACON_CUDA_W_DOWN: Lp = &m->Ld; x = m->ffn; x_ld = m->f_loc; y = m->xn; y_ld = hid; out_n = hid; break;
            case BEACON_CUDA_W_LM_HEAD: Lp = &m->Llm; x = m->xn; x_ld = hid; y = m->logits_loc; y_ld = m->v_loc;
                out_n = m->v_loc; break;
            default: invalid("model_profile_linear: slot must be Q, O, GATE, DOWN or LM_HEAD");
        }
        const int nl = slot == BEACON_CUDA_W_LM_HEAD ? 1 : m->cfg.num_layers;
        auto weight = [&](int li) -> const void* {
            const LayerW& L = m->layers[li];
            switch (slot) {
                case BEACON_CUDA_W_Q: return L.wqkv->ptr;
                case BEACON_CUDA_W_O: return L.wo->ptr;
                case BEACON_CUDA_W_GATE: return L.wgu->ptr;
                case BEACON_CUDA_W_DOWN: return L.wd->ptr;
                default: return m->wlm->ptr;
            }
        };
        // the kernels a decode step of `batch` sequences runs (or a prefill chunk's),
        // with the decode step's quantised-activation hand-offs where it uses
        // them: o, gate/up and down read their input image (left valid by the
        // decode steps run before) and write the next projection's
        m->gemm_rows = batch <= kDecodeGemvRows ? kDecodeGemvRows : 16;
        const bool qxa = qx_active(m, batch, true) && m->layers[0].ffn_norm;
        QxImage in{}, out{};
        bool images = false;
        const float* res = nullptr;  // o and down: the residual add of the decode step (into the scratch row)
        if (qxa && slot == BEACON_CUDA_W_O) {
            in = qx_image(m, 1, m->Lo, batch, nullptr);
            out = qx_image(m, 0, m->Lgu, batch, static_cast<const float*>(m->layers[0].ffn_norm->ptr));
            images = true;
        } else if (qxa && slot == BEACON_CUDA_W_GATE) {
            in = qx_image(m, 0, m->Lgu, batch, static_cast<const float*>(m->layers[0].ffn_norm->ptr));
            out = qx_image(m, 2, m->Ld, batch, nullptr);
            images = true;
        } else if (qxa && slot == BEACON_CUDA_W_DOWN) {
            in = qx_image(m, 2, m->Ld, batch, nullptr);
            out = qx_image(m, 0, m->Lqkv, batch, static_cast<const float*>(m->layers[0].attn_norm->ptr));
            images = true;
        }
        if (images && (slot == BEACON_CUDA_W_O || slot == BEACON_CUDA_W_DOWN)) {
            epi = EPI_ADD;
            res = m->h;
        }
        auto pass = [&]() {
            for (int li = 0; li < nl; ++li)
                linear(m, *Lp, weight(li), x, x_ld, batch, y, y_ld, epi, res, hid, s, nullptr,
                       images ? &in : nullptr, images ? &out : nullptr);
        };
        pass();  // warm-up
        cudaEvent_t e0, e1;
        BC_CUDA(cudaEventCreate(&e0));
        BC_CUDA(cudaEventCreate(&e1));
        BC_CUDA(cudaEventRecord(e0, s));
        for (int it = 0; it < iters; ++it) pass();
        BC_CUDA(cudaEventRecord(e1, s));
        BC_CUDA(cudaEventSynchronize(e1));
        float ms = 0.0f;
        BC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        *out_avg_us = ms * 1000.0f / (float)(iters * nl);
        const int64_t wbytes = Lp->n * (Lp->k / block_size(Lp->dtype)) * block_bytes(Lp->dtype);
        *out_bytes = (uint64_t)(wbytes + (int64_t)batch * Lp->k * 4 + (int64_t)batch * out_n * 4);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_fill_kv_random(BeaconCudaModel* m, int32_t n_rows, uint64_t seed) {
    return guard([&]() -> int32_t {
        require(m != nullptr, "model_fill_kv_random: null argument");
        if (n_rows < 0 || n_rows > m->cfg.max_context) fail(BEACON_CUDA_ERR_CONTEXT_OVERFLOW, "fill_kv_random: too many rows");
        set_device(m->ctx);
        const auto& c = m->cfg;
        const bool f16 = c.kv_dtype == BEACON_CUDA_DTYPE_F16;
        const int64_t per_seq = (int64_t)n_rows * m->kd, seq_stride = (int64_t)c.max_context * m->kd;
        const int64_t n = per_seq * c.max_batch;
        for (size_t li = 0; li < m->layers.size(); ++li)
            for (int which = 0; which < 2; ++which) {
                void* dst = which ? m->layers[li].vc->ptr : m->layers[li].kc->ptr;
                fill_random_kernel<<<cdiv(n, 256), 256>>>(dst, f16, n, per_seq, seq_stride,
                                                          seed * 0x9E3779B97F4A7C15ull + li * 2 + which);
                BC_LAUNCHED("fill_random_kernel");
            }
        BC_CUDA(cudaDeviceSynchronize());
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_launches_per_step(BeaconCudaModel* m, int32_t batch, int32_t continuing, int32_t* out) {
    return guard([&]() -> int32_t {
        require(m && out, "model_launches_per_step: null argument");
        auto it = m->graph_kernels.find(batch * 2 + (continuing ? 1 : 0));
        if (it == m->graph_kernels.end()) invalid("model_launches_per_step: that step has not been captured yet");
        *out = it->second;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_model_memory(const BeaconCudaModel* m, uint64_t* out_bytes) {
    return guard([&]() -> int32_t {
        require(m && out_bytes, "model_memory: null argument");
        uint64_t t = 0;
        auto add = [&](const std::unique_ptr<DeviceBuffer>& b) {
            if (b) t += b->bytes;
        };
        for (const auto& L : m->layers) {
            add(L.attn_norm); add(L.ffn_norm); add(L.wqkv); add(L.wo); add(L.wgu); add(L.wd); add(L.kc); add(L.vc);
        }
        add(m->embed); add(m->final_norm); add(m->wlm); add(m->rope_cs); add(m->rope_sn); add(m->act);
        add(m->gemv_buf); add(m->attn_buf); add(m->argmax_buf);
        *out_bytes = t;
        return BEACON_CUDA_OK;
    });
}

}  // extern "C"
