// sample.cu -- the token sampling pipeline of the reference
// (crates/beacon-scheduler/src/sampling.rs:15-186) on the device:
// repeat penalty -> temperature (greedy argmax at <= f32::EPSILON) -> top-k
// -> top-p -> min-p -> softmax -> multinomial draw, one CTA per row, so a
// decode step hands the host one token id per sequence instead of the whole
// logits row.
//
// Arithmetic follows the reference stage by stage (the same f32 operations on
// each element, the same comparisons and thresholds). Its sequential f32 sums
// over the vocabulary (softmax normalisers, the top-p and multinomial
// cumulative sums) become parallel sums: the normalisers are f32 tree sums in
// a fixed order, and the cumulative sums are exact sums of the probabilities
// in 2^-40 fixed point, so results are deterministic and differ from the
// reference's only where a draw or a top-p cut lies within rounding of a
// cumulative boundary. The reference draws r from an unseeded thread RNG
// (rand::rng, crates/beacon-cli/src/main.rs:267); here r is an input.
#include <cfloat>

#include "argmax.h"
#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace bc {

namespace {

constexpr int kSampleThreads = 1024;
constexpr float kF32Eps = FLT_EPSILON;  // f32::EPSILON
constexpr double kFx = 1099511627776.0;  // 2^40: fixed-point scale of the cumulative sums

struct SampleArgs {
    const float* logits;
    int64_t ld;
    int64_t V;
    const int32_t* prev;  // [rows][n_prev]
    int n_prev;
    BeaconCudaSamplingParams p;
    float inv_t;
    const float* uniforms;  // [rows]
    float* work;            // [rows][V]
    int32_t* out;           // [rows]
};

// Order-preserving map of floats to unsigned keys (larger float, larger key).
__device__ __forceinline__ uint32_t f2key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < kSampleThreads / 32; ++i) r = fmaxf(r, red[i]);
    return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = 0.0f;
    for (int i = 0; i < kSampleThreads / 32; ++i) r += red[i];
    return r;
}

// softmax_inplace (sampling.rs:173-186) split into its parameters:
// p_i = exp(w_i - mx) * inv when the sum is positive, exp(w_i - mx) otherwise.
struct Softmax {
    float mx, inv;
    bool scale;
    __device__ __forceinline__ float prob(float w) const {
        const float e = expf(w - mx);
        return scale ? e * inv : e;
    }
};

__device__ Softmax softmax_of(const float* w, int64_t V, float* red) {
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < V; i += kSampleThreads) m = fmaxf(m, w[i]);
    Softmax s;
    s.mx = block_max(m, red);
    float sum = 0.0f;
    for (int64_t i = threadIdx.x; i < V; i += kSampleThreads) sum += expf(w[i] - s.mx);
    const float total = block_sum(sum, red);
    s.scale = total > 0.0f;
    s.inv = s.scale ? 1.0f / total : 1.0f;
    return s;
}

__device__ __forceinline__ unsigned long long to_fx(float p) {
    return p > 0.0f ? (unsigned long long)((double)p * kFx) : 0ull;
}

__global__ void __launch_bounds__(kSampleThreads) sample_penalty_kernel(SampleArgs a) {
    const int row = blockIdx.x;
    float* w = a.work + (int64_t)row * a.V;
    const float* src = a.logits + (int64_t)row * a.ld;
    for (int64_t i = threadIdx.x; i < a.V; i += kSampleThreads) w[i] = src[i];
    __syncthreads();
    // repeat penalty, once per occurrence in the reference's order (sampling.rs:77-88)
    if (threadIdx.x == 0 && a.prev && fabsf(a.p.repeat_penalty - 1.0f) > kF32Eps)
        for (int j = 0; j < a.n_prev; ++j) {
            const int32_t idx = a.prev[(int64_t)row * a.n_prev + j];
            if (idx >= 0 && idx < a.V) {
                const float v = w[idx];
                w[idx] = v > 0.0f ? v / a.p.repeat_penalty : v * a.p.repeat_penalty;
            }
        }
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleArgs a) {
    __shared__ float red[kSampleThreads / 32];
    __shared__ unsigned int hist[256];
    __shared__ unsigned long long hsum[256];
    __shared__ uint32_t sel_digit;
    __shared__ int sel_found;
    __shared__ long long cand;
    __shared__ unsigned long long chunk_fx[kSampleThreads];
    const int row = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t V = a.V;
    float* w = a.work + (int64_t)row * V;

    // penalty already applied; temperature (sampling.rs:31-34, 91-96)
    if (fabsf(a.p.temperature - 1.0f) > kF32Eps)
        for (int64_t i = tid; i < V; i += kSampleThreads) w[i] *= a.inv_t;
    __syncthreads();

    // top-k (sampling.rs:99-114): threshold = the k-th value in descending
    // order (0-based), found by an 8-bit radix descent over the keys
    if (a.p.has_top_k && (int64_t)a.p.top_k < V) {
        uint32_t prefix = 0, mask = 0;
        long long kr = a.p.top_k;
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            for (int d = tid; d < 256; d += kSampleThreads) hist[d] = 0;
            __syncthreads();
            for (int64_t i = tid; i < V; i += kSampleThreads) {
                const uint32_t key = f2key(w[i]);
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int d = 255;
                for (; d > 0; --d) {
                    if (kr < (long long)hist[d]) break;
                    kr -= hist[d];
                }
                sel_digit = (uint32_t)d;
            }
            __syncthreads();
            prefix |= sel_digit << shift;
            mask |= 255u << shift;
        }
        const float threshold = key2f(prefix);
        for (int64_t i = tid; i < V; i += kSampleThreads)
            if (w[i] < threshold) w[i] = -INFINITY;
        __syncthreads();
    }

    // top-p (sampling.rs:117-145): the cut element is the first, in
    // descending probability order, whose cumulative probability exceeds p;
    // found by a radix descent that carries the mass above the bucket
    if (a.p.has_top_p && a.p.top_p < 1.0f) {
        const Softmax sm = softmax_of(w, V, red);
        const unsigned long long p_fx = a.p.top_p > 0.0f ? (unsigned long long)((double)a.p.top_p * kFx) : 0ull;
        uint32_t prefix = 0, mask = 0;
        unsigned long long above = 0;
        bool found = true;
        for (int pass = 0; pass < 4 && found; ++pass) {
            const int shift = 24 - 8 * pass;
            for (int d = tid; d < 256; d += kSampleThreads) {
                hist[d] = 0;
                hsum[d] = 0;
            }
            __syncthreads();
            for (int64_t i = tid; i < V; i += kSampleThreads) {
                const float pr = sm.prob(w[i]);
                const uint32_t key = f2key(pr);
                if ((key & mask) == prefix) {
                    atomicAdd(&hist[(key >> shift) & 255u], 1u);
                    atomicAdd(&hsum[(key >> shift) & 255u], to_fx(pr));
                }
            }
            __syncthreads();
            if (tid == 0) {
                int d = 255, f = 0;
                for (; d >= 0; --d) {
                    if (!hist[d]) continue;
                    if (above + hsum[d] > p_fx) {
                        f = 1;
                        break;
                    }
                    above += hsum[d];
                }
                sel_digit = (uint32_t)(d < 0 ? 0 : d);
                sel_found = f;
            }
            __syncthreads();
            found = sel_found != 0;
            prefix |= sel_digit << shift;
            mask |= 255u << shift;
        }
        if (found) {  // else the cumulative sum never exceeds p: everything stays
            const float cut = key2f(prefix);
            for (int64_t i = tid; i < V; i += kSampleThreads)
                if (sm.prob(w[i]) < cut) w[i] = -INFINITY;
        }
        __syncthreads();
    }

    // min-p (sampling.rs:148-160)
    if (a.p.has_min_p && a.p.min_p > 0.0f) {
        const Softmax sm = softmax_of(w, V, red);
        float m = 0.0f;  // fold(0.0, f32::max)
        for (int64_t i = tid; i < V; i += kSampleThreads) m = fmaxf(m, sm.prob(w[i]));
        const float threshold = a.p.min_p * block_max(m, red);
        for (int64_t i = tid; i < V; i += kSampleThreads)
            if (sm.prob(w[i]) < threshold) w[i] = -INFINITY;
        __syncthreads();
    }

    // softmax + multinomial draw (sampling.rs:53-56, 163-186): the first index
    // whose cumulative probability reaches r, else the last index. Thread t
    // scans its contiguous chunk after the exclusive prefix of the chunks
    // before it.
    const Softmax sm = softmax_of(w, V, red);
    const float r = a.uniforms[row];
    const unsigned long long r_fx = r > 0.0f ? (unsigned long long)((double)r * kFx) : 0ull;
    const int64_t chunk = (V + kSampleThreads - 1) / kSampleThreads;
    const int64_t c0 = (int64_t)tid * chunk, c1 = c0 + chunk < V ? c0 + chunk : V;
    unsigned long long mine = 0;
    for (int64_t i = c0; i < c1; ++i) mine += to_fx(sm.prob(w[i]));
    chunk_fx[tid] = mine;
    if (tid == 0) cand = V - 1;
    __syncthreads();
    if (tid == 0) {  // exclusive prefix over the chunks, in order
        unsigned long long run = 0;
        for (int t = 0; t < kSampleThreads; ++t) {
            const unsigned long long c = chunk_fx[t];
            chunk_fx[t] = run;
            run += c;
        }
    }
    __syncthreads();
    unsigned long long cum = chunk_fx[tid];
    if (c0 < c1 && cum + mine >= r_fx) {
        for (int64_t i = c0; i < c1; ++i) {
            cum += to_fx(sm.prob(w[i]));
            if (cum >= r_fx) {
                atomicMin(&cand, (long long)i);
                break;
            }
        }
    }
    __syncthreads();
    if (tid == 0) a.out[row] = (int32_t)cand;
}

}  // namespace

void launch_sample(const float* logits, int64_t ld, int64_t V, int rows, const int32_t* prev, int n_prev,
                   const BeaconCudaSamplingParams& p, const float* uniforms, float* work, int32_t* out,
                   ArgmaxSummary* argmax_scratch, cudaStream_t s) {
    if (rows <= 0 || V <= 0) return;
    SampleArgs a;
    a.logits = logits;
    a.ld = ld;
    a.V = V;
    a.prev = prev;
    a.n_prev = n_prev;
    a.p = p;
    a.inv_t = p.temperature > 0.0f ? 1.0f / p.temperature : 0.0f;
    a.uniforms = uniforms;
    a.work = work;
    a.out = out;
    sample_penalty_kernel<<<rows, kSampleThreads, 0, s>>>(a);
    BC_LAUNCHED("sample_penalty_kernel");
    if (p.temperature <= kF32Eps) {  // greedy (sampling.rs:27-30)
        launch_argmax(work, V, 1, rows, out, nullptr, argmax_scratch, s);
        return;
    }
    sample_kernel<<<rows, kSampleThreads, 0, s>>>(a);
    BC_LAUNCHED("sample_kernel");
}

size_t sample_scratch_bytes(int64_t V, int rows) {
    return (size_t)rows * V * sizeof(float) + argmax_scratch_count(V, 1, rows) * sizeof(ArgmaxSummary) + 256;
}

}  // namespace bc

using namespace bc;

extern "C" int32_t beacon_cuda_op_sample(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                         const BeaconCudaTensor* logits, const BeaconCudaTensor* previous_tokens,
                                         const BeaconCudaSamplingParams* params, const BeaconCudaTensor* uniforms,
                                         BeaconCudaTensor** out) {
    return guard([&]() -> int32_t {
        require(ctx && stream && logits && params && uniforms && out, "sample: null argument");
        require(stream->ctx == ctx, "sample: the stream belongs to another context");
        if (logits->dtype != BEACON_CUDA_DTYPE_F32) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "sample: logits must be F32");
        if (uniforms->dtype != BEACON_CUDA_DTYPE_F32) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "sample: uniforms must be F32");
        if (logits->shape.empty()) shape_err("sample: logits have no dimensions");
        const int64_t V = logits->shape.back();
        const int64_t rows = logits->shape.size() == 1 ? 1 : logits->numel() / std::max<int64_t>(V, 1);
        if (V <= 0) shape_err("sample: empty vocabulary");
        if (uniforms->numel() != rows) shape_err("sample: one uniform draw per row is needed");
        if (rows > 65535) shape_err("sample: too many rows");
        int n_prev = 0;
        const int32_t* prev = nullptr;
        if (previous_tokens) {
            if (previous_tokens->dtype != BEACON_CUDA_DTYPE_I32)
                fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "sample: previous tokens must be I32");
            if (previous_tokens->numel() % rows) shape_err("sample: previous tokens must be [rows, n]");
            n_prev = (int)(previous_tokens->numel() / rows);
            prev = static_cast<const int32_t*>(previous_tokens->data());
        }
        const BeaconCudaSamplingParams& p = *params;
        if (p.has_top_k && p.top_k < 0) invalid("sample: top_k must be >= 0");
        if (!(p.repeat_penalty > 0.0f)) invalid("sample: repeat_penalty must be positive");
        set_device(ctx);
        BeaconCudaTensor* o = new_tensor(ctx, {rows}, BEACON_CUDA_DTYPE_I32);
        try {
            uint8_t* scratch = static_cast<uint8_t*>(stream->ws.get(sample_scratch_bytes(V, (int)rows), stream->s));
            float* work = reinterpret_cast<float*>(scratch);
            auto* am = reinterpret_cast<ArgmaxSummary*>(scratch + ((size_t)rows * V * 4 + 255) / 256 * 256);
            launch_sample(static_cast<const float*>(logits->data()), V, V, (int)rows, prev, n_prev, p,
                          static_cast<const float*>(uniforms->data()), work, static_cast<int32_t*>(o->data()), am,
                          stream->s);
        } catch (...) {
            delete o;
            throw;
        }
        *out = o;
        return BEACON_CUDA_OK;
    });
}
