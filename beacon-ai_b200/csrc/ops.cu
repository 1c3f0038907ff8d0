// ops.cu -- the non-GEMV methods of ComputeBackend (backend.rs:21-166) as
// sm_100a kernels behind the C ABI: rms_norm, rope, silu, softmax, add, mul,
// reshape, transpose, swapaxes, embedding, kv_cache_update, argmax, matmul
// (f32), token tensors. Semantics follow the CPU backend
// (crates/beacon-core/src/cpu_backend.rs) unless stated.
#include <algorithm>
#include <string>
#include <vector>

#include "argmax.h"
#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace bc {
namespace {

__device__ __forceinline__ float ld_any(const void* p, int32_t dtype, int64_t i) {
    switch (dtype) {
        case BEACON_CUDA_DTYPE_F16: return __half2float(static_cast<const __half*>(p)[i]);
        case BEACON_CUDA_DTYPE_BF16: return __uint_as_float((uint32_t)static_cast<const uint16_t*>(p)[i] << 16);
        case BEACON_CUDA_DTYPE_I32: return (float)static_cast<const int32_t*>(p)[i];
        default: return static_cast<const float*>(p)[i];
    }
}

__device__ __forceinline__ void st_any(void* p, int32_t dtype, int64_t i, float v) {
    if (dtype == BEACON_CUDA_DTYPE_F16)
        static_cast<__half*>(p)[i] = __float2half_rn(v);
    else
        static_cast<float*>(p)[i] = v;
}

__device__ float block_sum(float v, float* sh) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    float r = 0.0f;
    for (int i = 0; i < nw; ++i) r += sh[i];
    return r;
}

// ops.rs:77-93 per row (cpu_backend.rs:103-139)
__global__ void rms_norm_kernel(const void* x, int32_t xt, const void* w, int32_t wt, float* out, int64_t d,
                                float eps) {
    __shared__ float sh[32];
    const int64_t row = blockIdx.x;
    float ss = 0.0f;
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
        float v = ld_any(x, xt, row * d + i);
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, sh);
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x)
        out[row * d + i] = ld_any(x, xt, row * d + i) * inv * ld_any(w, wt, i);
}

// ops.rs:124-142: interleaved pairs, one thread per pair.
__global__ void rope_kernel(const void* x, int32_t xt, float* out, int64_t groups, int64_t seq, int64_t dim,
                            int64_t pos0, float theta) {
    const int64_t half = dim / 2;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= groups * seq * half) return;
    const int64_t i2 = idx % half, s = (idx / half) % seq;
    const int64_t base = (idx / half) * dim + 2 * i2;
    const float freq = 1.0f / powf(theta, (float)(2 * i2) / (float)dim);
    const float angle = (float)(pos0 + s) * freq;
    float sn, c;
    sincosf(angle, &sn, &c);
    const float x0 = ld_any(x, xt, base), x1 = ld_any(x, xt, base + 1);
    out[base] = x0 * c - x1 * sn;
    out[base + 1] = x0 * sn + x1 * c;
}

__global__ void silu_kernel(const void* x, int32_t xt, float* out, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v = ld_any(x, xt, i);
    out[i] = v * (1.0f / (1.0f + expf(-v)));
}

// ops.rs:105-116 over the last dim, one CTA per row
__global__ void softmax_kernel(const void* x, int32_t xt, float* out, int64_t d) {
    __shared__ float sh[32];
    const int64_t row = blockIdx.x;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) m = fmaxf(m, ld_any(x, xt, row * d + i));
    m = warp_max(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = m;
    __syncthreads();
    m = -INFINITY;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, sh[i]);
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) {
        float e = expf(ld_any(x, xt, row * d + i) - m);
        out[row * d + i] = e;
        s += e;
    }
    s = block_sum(s, sh);
    const float inv = 1.0f / s;
    for (int64_t i = threadIdx.x; i < d; i += blockDim.x) out[row * d + i] *= inv;
}

__global__ void binary_kernel(const void* a, int32_t at, const void* b, int32_t bt, float* out, int64_t n, int op) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float x = ld_any(a, at, i), y = ld_any(b, bt, i);
    out[i] = op == 0 ? x + y : x * y;
}

struct Perm {
    int ndim;
    int64_t out_dims[8];
    int64_t in_strides[8];  // input stride of each output axis
};

__global__ void permute_kernel(const uint8_t* in, uint8_t* out, int64_t n, int eb, Perm p) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int64_t rem = i, src = 0;
    for (int d = p.ndim - 1; d >= 0; --d) {
        int64_t c = rem % p.out_dims[d];
        rem /= p.out_dims[d];
        src += c * p.in_strides[d];
    }
    for (int b = 0; b < eb; ++b) out[i * eb + b] = in[src * eb + b];
}

// cpu_backend.rs:387-418; an out-of-range id sets *err and writes zeros.
__global__ void embedding_kernel(const void* w, int32_t wt, int64_t vocab, int64_t h, const void* idx,
                                 int32_t it, float* out, int64_t seq, int* err) {
    const int64_t s = blockIdx.x;
    if (s >= seq) return;
    const float f = ld_any(idx, it, s);
    const int64_t tok = (int64_t)f;
    const bool ok = f >= 0.0f && tok < vocab;
    if (!ok && threadIdx.x == 0) atomicExch(err, 1);
    for (int64_t i = threadIdx.x; i < h; i += blockDim.x) out[s * h + i] = ok ? ld_any(w, wt, tok * h + i) : 0.0f;
}

// cache rows [pos, pos+S) <- new rows (any float dtype, converted)
__global__ void kv_write_kernel(void* cache, int32_t ct, const void* nw, int32_t nt, int64_t pos, int64_t row,
                                int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    st_any(cache, ct, pos * row + i, ld_any(nw, nt, i));
}

// ops.rs:16-30 (a [m,k] x b [k,n]), 16x16 shared-memory tiles
__global__ void matmul_kernel(const void* a, int32_t at, const void* b, int32_t bt, float* c, int64_t m, int64_t k,
                              int64_t n) {
    __shared__ float sa[16][17], sb[16][17];
    const int64_t row = (int64_t)blockIdx.y * 16 + threadIdx.y, col = (int64_t)blockIdx.x * 16 + threadIdx.x;
    float acc = 0.0f;
    for (int64_t k0 = 0; k0 < k; k0 += 16) {
        sa[threadIdx.y][threadIdx.x] = (row < m && k0 + threadIdx.x < k) ? ld_any(a, at, row * k + k0 + threadIdx.x) : 0.0f;
        sb[threadIdx.y][threadIdx.x] = (k0 + threadIdx.y < k && col < n) ? ld_any(b, bt, (k0 + threadIdx.y) * n + col) : 0.0f;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 16; ++i) acc = fmaf(sa[threadIdx.y][i], sb[i][threadIdx.x], acc);
        __syncthreads();
    }
    if (row < m && col < n) c[row * n + col] = acc;
}

inline unsigned nblk(int64_t n, int t = 256) { return (unsigned)std::max<int64_t>(1, (n + t - 1) / t); }

void check_float(const BeaconCudaTensor* t, const char* what) {
    if (t->dtype != BEACON_CUDA_DTYPE_F32 && t->dtype != BEACON_CUDA_DTYPE_F16 && t->dtype != BEACON_CUDA_DTYPE_BF16)
        fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, std::string(what) + ": expected a float tensor");
}

template <typename F>
int32_t op_guard(BeaconCudaContext* ctx, BeaconCudaStream* stream, BeaconCudaTensor** out, F&& body) {
    return guard([&]() -> int32_t {
        require(ctx && stream && out, "null context, stream or output");
        if (stream->ctx != ctx) invalid("the stream belongs to another context");
        set_device(ctx);
        *out = body();
        return BEACON_CUDA_OK;
    });
}

struct TensorHolder {  // frees an output tensor if the launch throws
    BeaconCudaTensor* t;
    explicit TensorHolder(BeaconCudaTensor* x) : t(x) {}
    ~TensorHolder() { delete t; }
    BeaconCudaTensor* release() {
        auto* r = t;
        t = nullptr;
        return r;
    }
};

}  // namespace
}  // namespace bc

using namespace bc;

extern "C" {

int32_t beacon_cuda_op_rms_norm(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                                const BeaconCudaTensor* weight, float eps, BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(x && weight, "rms_norm: null argument");
        check_float(x, "rms_norm");
        check_float(weight, "rms_norm");
        if (x->shape.empty()) shape_err("rms_norm: empty shape");
        const int64_t d = x->shape.back();
        if (weight->numel() != d) shape_err("rms_norm: weight length != last dim");
        TensorHolder o(new_tensor(ctx, x->shape, BEACON_CUDA_DTYPE_F32));
        const int64_t rows = d ? x->numel() / d : 0;
        if (rows)
            rms_norm_kernel<<<(unsigned)rows, 256, 0, stream->s>>>(x->data(), x->dtype, weight->data(), weight->dtype,
                                                                   static_cast<float*>(o.t->data()), d, eps);
        BC_LAUNCHED("rms_norm_kernel");
        return o.release();
    });
}

int32_t beacon_cuda_op_rope(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                            int32_t position_offset, float theta, int32_t dim, const BeaconCudaTensor* freqs,
                            BeaconCudaTensor** out) {
    (void)freqs;  // the CPU backend ignores custom frequencies too (cpu_backend.rs:150-151)
    return op_guard(ctx, stream, out, [&]() {
        require(x != nullptr, "rope: null argument");
        check_float(x, "rope");
        if (dim <= 0 || dim % 2) invalid("rope: dim must be positive and even");
        if (position_offset < 0) invalid("rope: negative position");
        const int64_t seq = x->shape.size() >= 2 ? x->shape[x->shape.size() - 2] : 1;
        const int64_t total = x->numel();
        if (seq == 0 || total % (seq * dim)) shape_err("rope: tensor is not [.., seq, dim]");
        const int64_t groups = total / (seq * dim);
        TensorHolder o(new_tensor(ctx, x->shape, BEACON_CUDA_DTYPE_F32));
        const int64_t work = groups * seq * (dim / 2);
        if (work)
            rope_kernel<<<nblk(work), 256, 0, stream->s>>>(x->data(), x->dtype, static_cast<float*>(o.t->data()),
                                                           groups, seq, dim, position_offset, theta);
        BC_LAUNCHED("rope_kernel");
        return o.release();
    });
}

int32_t beacon_cuda_op_silu(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                            BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(x != nullptr, "silu: null argument");
        check_float(x, "silu");
        TensorHolder o(new_tensor(ctx, x->shape, BEACON_CUDA_DTYPE_F32));
        if (x->numel())
            silu_kernel<<<nblk(x->numel()), 256, 0, stream->s>>>(x->data(), x->dtype, static_cast<float*>(o.t->data()),
                                                                 x->numel());
        BC_LAUNCHED("silu_kernel");
        return o.release();
    });
}

int32_t beacon_cuda_op_softmax(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                               int32_t axis, BeaconCudaTensor** out) {
    (void)axis;  // the CPU backend normalises over the last dim whatever the axis (cpu_backend.rs:203-224)
    return op_guard(ctx, stream, out, [&]() {
        require(x != nullptr, "softmax: null argument");
        check_float(x, "softmax");
        if (x->shape.empty()) shape_err("softmax: empty shape");
        const int64_t d = x->shape.back();
        TensorHolder o(new_tensor(ctx, x->shape, BEACON_CUDA_DTYPE_F32));
        const int64_t rows = d ? x->numel() / d : 0;
        if (rows)
            softmax_kernel<<<(unsigned)rows, 256, 0, stream->s>>>(x->data(), x->dtype, static_cast<float*>(o.t->data()), d);
        BC_LAUNCHED("softmax_kernel");
        return o.release();
    });
}

static int32_t binary(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* a,
                      const BeaconCudaTensor* b, BeaconCudaTensor** out, int op) {
    return op_guard(ctx, stream, out, [&]() {
        require(a && b, "add/mul: null argument");
        check_float(a, "add/mul");
        check_float(b, "add/mul");
        if (a->numel() != b->numel()) shape_err("add/mul: length mismatch");  // cpu_backend.rs:232-238
        TensorHolder o(new_tensor(ctx, a->shape, BEACON_CUDA_DTYPE_F32));
        if (a->numel())
            binary_kernel<<<nblk(a->numel()), 256, 0, stream->s>>>(a->data(), a->dtype, b->data(), b->dtype,
                                                                   static_cast<float*>(o.t->data()), a->numel(), op);
        BC_LAUNCHED("binary_kernel");
        return o.release();
    });
}

int32_t beacon_cuda_op_add(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* a,
                           const BeaconCudaTensor* b, BeaconCudaTensor** out) {
    return binary(ctx, stream, a, b, out, 0);
}

int32_t beacon_cuda_op_elementwise_mul(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* a,
                                       const BeaconCudaTensor* b, BeaconCudaTensor** out) {
    return binary(ctx, stream, a, b, out, 1);
}

int32_t beacon_cuda_op_reshape(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                               const int64_t* new_shape, size_t new_ndim, BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(x && (new_shape || new_ndim == 0), "reshape: null argument");
        if (is_quantized(x->dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "reshape of a quantized tensor");
        std::vector<int64_t> s(new_shape, new_shape + new_ndim);
        int64_t n = 1;
        for (int64_t d : s) {
            if (d < 0) shape_err("reshape: negative dimension");
            n *= d;
        }
        if (n != x->numel()) shape_err("reshape: element count mismatch");  // cpu_backend.rs:374-380
        return view_tensor(x, s, 0, x->dtype);
    });
}

static BeaconCudaTensor* permute_swap(BeaconCudaContext* ctx, cudaStream_t s, const BeaconCudaTensor* x, int a1,
                                      int a2) {
    const int nd = (int)x->shape.size();
    std::vector<int64_t> os = x->shape;
    std::swap(os[a1], os[a2]);
    std::vector<int64_t> in_str(nd, 1);
    for (int i = nd - 2; i >= 0; --i) in_str[i] = in_str[i + 1] * x->shape[i + 1];
    Perm p;
    p.ndim = nd;
    for (int i = 0; i < nd; ++i) {
        p.out_dims[i] = os[i];
        int src_axis = i == a1 ? a2 : (i == a2 ? a1 : i);
        p.in_strides[i] = in_str[src_axis];
    }
    TensorHolder o(new_tensor(ctx, os, x->dtype));
    const int64_t n = x->numel();
    if (n)
        permute_kernel<<<nblk(n), 256, 0, s>>>(static_cast<const uint8_t*>(x->data()), static_cast<uint8_t*>(o.t->data()),
                                               n, (int)plain_elem_bytes(x->dtype), p);
    BC_LAUNCHED("permute_kernel");
    return o.release();
}

int32_t beacon_cuda_op_swapaxes(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                                int32_t axis1, int32_t axis2, BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(x != nullptr, "swapaxes: null argument");
        if (is_quantized(x->dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "swapaxes of a quantized tensor");
        const int nd = (int)x->shape.size();
        int a1 = axis1 < 0 ? nd + axis1 : axis1, a2 = axis2 < 0 ? nd + axis2 : axis2;
        if (a1 < 0 || a2 < 0 || a1 >= nd || a2 >= nd) shape_err("swapaxes: axis out of range");
        if (a1 == a2) {
            TensorHolder o(new_tensor(ctx, x->shape, x->dtype));
            BC_CUDA(cudaMemcpyAsync(o.t->data(), x->data(), x->nbytes(), cudaMemcpyDeviceToDevice, stream->s));
            return o.release();
        }
        return permute_swap(ctx, stream->s, x, a1, a2);
    });
}

int32_t beacon_cuda_op_transpose(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                                 BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(x != nullptr, "transpose: null argument");
        if (is_quantized(x->dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "transpose of a quantized tensor");
        const int nd = (int)x->shape.size();
        if (nd < 2) shape_err("transpose needs >= 2 dims");  // cpu_backend.rs:336-340
        return permute_swap(ctx, stream->s, x, nd - 2, nd - 1);
    });
}

int32_t beacon_cuda_op_embedding(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* weight,
                                 const BeaconCudaTensor* indices, BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(weight && indices, "embedding: null argument");
        if (weight->shape.size() != 2) shape_err("embedding: weight must be 2-D");
        check_float(weight, "embedding");
        if (indices->dtype != BEACON_CUDA_DTYPE_I32 && indices->dtype != BEACON_CUDA_DTYPE_F32)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "embedding: indices must be I32 or F32");
        const int64_t vocab = weight->shape[0], h = weight->shape[1], seq = indices->numel();
        TensorHolder o(new_tensor(ctx, {seq, h}, BEACON_CUDA_DTYPE_F32));
        stream->ws.get(0, stream->s);
        int* err = stream->ws.flags();
        BC_CUDA(cudaMemsetAsync(err, 0, sizeof(int), stream->s));
        if (seq)
            embedding_kernel<<<(unsigned)seq, 256, 0, stream->s>>>(weight->data(), weight->dtype, vocab, h,
                                                                   indices->data(), indices->dtype,
                                                                   static_cast<float*>(o.t->data()), seq, err);
        BC_LAUNCHED("embedding_kernel");
        int herr = 0;
        BC_CUDA(cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, stream->s));
        BC_CUDA(cudaStreamSynchronize(stream->s));
        if (herr) shape_err("embedding index out of bounds for the vocabulary");  // cpu_backend.rs:406-411
        return o.release();
    });
}

int32_t beacon_cuda_create_token_tensor(BeaconCudaContext* ctx, const uint32_t* tokens, size_t n,
                                        BeaconCudaTensor** out) {
    return guard([&]() -> int32_t {
        require(ctx && out && (tokens || n == 0), "create_token_tensor: null argument");
        set_device(ctx);
        for (size_t i = 0; i < n; ++i)
            if (tokens[i] > 0x7FFFFFFFu) invalid("token id does not fit in int32");
        TensorHolder o(new_tensor(ctx, {(int64_t)n}, BEACON_CUDA_DTYPE_I32));
        if (n) BC_CUDA(cudaMemcpy(o.t->data(), tokens, n * 4, cudaMemcpyHostToDevice));
        *out = o.release();
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_op_kv_cache_update(BeaconCudaContext* ctx, BeaconCudaStream* stream, BeaconCudaTensor* cache_k,
                                       BeaconCudaTensor* cache_v, const BeaconCudaTensor* new_k,
                                       const BeaconCudaTensor* new_v, int64_t position,
                                       BeaconCudaTensor** out_k_view, BeaconCudaTensor** out_v_view) {
    return guard([&]() -> int32_t {
        require(ctx && stream && cache_k && cache_v && new_k && new_v && out_k_view && out_v_view,
                "kv_cache_update: null argument");
        set_device(ctx);
        if (cache_k->shape.size() != 3 || cache_v->shape != cache_k->shape)
            shape_err("kv_cache_update: caches must be [max_context, num_kv_heads, head_dim]");
        check_float(cache_k, "kv_cache_update");
        check_float(new_k, "kv_cache_update");
        check_float(new_v, "kv_cache_update");
        const int64_t max_ctx = cache_k->shape[0], row = cache_k->shape[1] * cache_k->shape[2];
        if (new_k->numel() != new_v->numel() || row == 0 || new_k->numel() % row)
            shape_err("kv_cache_update: new rows do not match the cache row size");
        const int64_t seq = new_k->numel() / row;
        if (position < 0 || position >= max_ctx || position + seq > max_ctx)
            fail(BEACON_CUDA_ERR_CONTEXT_OVERFLOW, "kv_cache_update: position out of range");
        const int64_t n = seq * row;
        if (n) {
            kv_write_kernel<<<nblk(n), 256, 0, stream->s>>>(cache_k->data(), cache_k->dtype, new_k->data(), new_k->dtype,
                                                            position, row, n);
            kv_write_kernel<<<nblk(n), 256, 0, stream->s>>>(cache_v->data(), cache_v->dtype, new_v->data(), new_v->dtype,
                                                            position, row, n);
            BC_LAUNCHED("kv_write_kernel");
        }
        std::vector<int64_t> vs = {position + seq, cache_k->shape[1], cache_k->shape[2]};
        TensorHolder kv(view_tensor(cache_k, vs, 0, cache_k->dtype));
        *out_v_view = view_tensor(cache_v, vs, 0, cache_v->dtype);
        *out_k_view = kv.release();
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_op_argmax(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* logits,
                              BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(logits != nullptr, "argmax: null argument");
        if (logits->dtype != BEACON_CUDA_DTYPE_F32) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "argmax: logits must be F32");
        const int64_t d = logits->shape.empty() ? 1 : logits->shape.back();
        const int64_t rows = logits->shape.size() <= 1 ? 1 : logits->numel() / std::max<int64_t>(d, 1);
        TensorHolder o(new_tensor(ctx, {rows}, BEACON_CUDA_DTYPE_I32));
        if (rows && d == 0) {
            BC_CUDA(cudaMemsetAsync(o.t->data(), 0, (size_t)rows * 4, stream->s));  // empty -> 0 (sampling.rs:65)
        } else if (rows) {
            auto* scratch = static_cast<ArgmaxSummary*>(
                stream->ws.get(argmax_scratch_count(d, 1, (int)rows) * sizeof(ArgmaxSummary), stream->s));
            launch_argmax(static_cast<const float*>(logits->data()), d, 1, (int)rows,
                          static_cast<int32_t*>(o.t->data()), nullptr, scratch, stream->s);
        }
        return o.release();
    });
}

int32_t beacon_cuda_op_matmul(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* a,
                              const BeaconCudaTensor* b, BeaconCudaTensor** out) {
    return op_guard(ctx, stream, out, [&]() {
        require(a && b, "matmul: null argument");
        if (a->shape.size() != 2 || b->shape.size() != 2) shape_err("matmul requires 2-D tensors");
        check_float(a, "matmul");
        check_float(b, "matmul");
        const int64_t m = a->shape[0], k = a->shape[1], k2 = b->shape[0], n = b->shape[1];
        if (k != k2) shape_err("matmul inner dim mismatch");
        TensorHolder o(new_tensor(ctx, {m, n}, BEACON_CUDA_DTYPE_F32));
        if (m && n) {
            dim3 grid((unsigned)((n + 15) / 16), (unsigned)((m + 15) / 16)), blk(16, 16);
            matmul_kernel<<<grid, blk, 0, stream->s>>>(a->data(), a->dtype, b->data(), b->dtype,
                                                       static_cast<float*>(o.t->data()), m, k, n);
            BC_LAUNCHED("matmul_kernel");
        }
        return o.release();
    });
}

}  // extern "C"
