// runtime.cu -- contexts, streams, tensors and the quantized ops of the C ABI
// (include/beacon_cuda.h). Conventions follow the MLX shim
// (shim/include/beacon_shim.h, shim/src/guard.h, shim/src/errors.cpp).
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace bc {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) noexcept {
    try {
        g_last_error = msg;
    } catch (...) {
        g_last_error.clear();
    }
}
void clear_error() noexcept { g_last_error.clear(); }
const char* get_error() noexcept { return g_last_error.c_str(); }

bool is_quantized(int32_t dtype) { return dtype >= 100 && dtype <= 110; }

int64_t block_size(int32_t dtype) {
    switch (dtype) {
        case BEACON_CUDA_DTYPE_Q4_0: case BEACON_CUDA_DTYPE_Q4_1: case BEACON_CUDA_DTYPE_Q5_0:
        case BEACON_CUDA_DTYPE_Q5_1: case BEACON_CUDA_DTYPE_Q8_0: return 32;
        case BEACON_CUDA_DTYPE_Q2_K: case BEACON_CUDA_DTYPE_Q3_K: case BEACON_CUDA_DTYPE_Q4_K:
        case BEACON_CUDA_DTYPE_Q5_K: case BEACON_CUDA_DTYPE_Q6_K: case BEACON_CUDA_DTYPE_Q8_K: return 256;
        default: return 1;
    }
}

int64_t block_bytes(int32_t dtype) {
    switch (dtype) {
        case BEACON_CUDA_DTYPE_Q4_0: return 18;
        case BEACON_CUDA_DTYPE_Q4_1: return 20;
        case BEACON_CUDA_DTYPE_Q5_0: return 22;
        case BEACON_CUDA_DTYPE_Q5_1: return 24;
        case BEACON_CUDA_DTYPE_Q8_0: return 34;
        case BEACON_CUDA_DTYPE_Q2_K: return 84;
        case BEACON_CUDA_DTYPE_Q3_K: return 110;
        case BEACON_CUDA_DTYPE_Q4_K: return 144;
        case BEACON_CUDA_DTYPE_Q5_K: return 176;
        case BEACON_CUDA_DTYPE_Q6_K: return 210;
        case BEACON_CUDA_DTYPE_Q8_K: return 292;
        default: return (int64_t)plain_elem_bytes(dtype);
    }
}

size_t plain_elem_bytes(int32_t dtype) {
    switch (dtype) {
        case BEACON_CUDA_DTYPE_F32: case BEACON_CUDA_DTYPE_I32: return 4;
        case BEACON_CUDA_DTYPE_F16: case BEACON_CUDA_DTYPE_BF16: return 2;
        case BEACON_CUDA_DTYPE_I8: return 1;
        default: return 0;
    }
}

static bool gemv_supported(int32_t dtype) { return is_quantized(dtype); }

// Nominal bits per weight code of each block type (the `bits` argument of
// quantized_matmul, backend.rs:32-41).
static int code_bits(int32_t dtype) {
    switch (dtype) {
        case BEACON_CUDA_DTYPE_Q2_K: return 2;
        case BEACON_CUDA_DTYPE_Q3_K: return 3;
        case BEACON_CUDA_DTYPE_Q5_0: case BEACON_CUDA_DTYPE_Q5_1: case BEACON_CUDA_DTYPE_Q5_K: return 5;
        case BEACON_CUDA_DTYPE_Q6_K: return 6;
        case BEACON_CUDA_DTYPE_Q8_0: case BEACON_CUDA_DTYPE_Q8_K: return 8;
        default: return 4;
    }
}

QLayout make_qlayout(int32_t dtype, int64_t n, int64_t k) {
    if (!gemv_supported(dtype))
        fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE,
             "block type " + std::to_string(dtype) + " has no device kernels yet (Q4_0, Q8_0, Q4_K do)");
    if (n <= 0 || k <= 0) shape_err("quantized tensor needs positive [N, K]");
    if (k % block_size(dtype)) shape_err("K is not a whole number of blocks");
    QLayout L;
    L.dtype = dtype;
    L.n = n;
    L.k = k;
    L.n_pad = (n + 31) / 32 * 32;
    L.k_pad = (k + 255) / 256 * 256;
    if (is_core_format(dtype)) {
        L.chunks = dtype == BEACON_CUDA_DTYPE_Q8_0 ? 16 : 8;
    } else {
        // raw bytes of 256 columns, in 16-byte chunks (the first is the "meta" chunk)
        const int64_t slice = 256 / block_size(dtype) * block_bytes(dtype);
        L.chunks = (int32_t)((slice + 15) / 16 - 1);
    }
    L.tile_bytes = 32 * (16 + 16 * (int64_t)L.chunks);
    return L;
}

DeviceBuffer::DeviceBuffer(size_t n) : bytes(n) {
    if (n) BC_CUDA(cudaMalloc(&ptr, n));
}
DeviceBuffer::~DeviceBuffer() {
    if (owned && ptr) cudaFree(ptr);
}

void* Workspace::get(size_t data_bytes, cudaStream_t s) {
    const size_t bytes = kDataOffset + data_bytes;
    if (!buf || buf->bytes < bytes) {
        if (s) {
            cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
            cudaStreamIsCapturing(s, &st);
            if (st != cudaStreamCaptureStatusNone)
                invalid("workspace must grow outside stream capture; run the op once before capturing");
        }
        size_t want = std::max<size_t>(bytes, 1 << 20);
        if (buf) want = std::max(want, 2 * buf->bytes);
        auto nb = std::make_unique<DeviceBuffer>(want);
        // zeroed in stream order: earlier work on this stream keeps using the
        // old buffer, which stays allocated until the stream is destroyed
        BC_CUDA(cudaMemsetAsync(nb->ptr, 0, want, s));
        if (buf) {
            // carry the error flags over (an op that timed out before the
            // growth must still be reported)
            BC_CUDA(cudaMemcpyAsync(static_cast<int*>(nb->ptr) + kCounterInts,
                                    static_cast<int*>(buf->ptr) + kCounterInts, kFlagInts * sizeof(int),
                                    cudaMemcpyDeviceToDevice, s));
            retired.push_back(std::move(buf));
        }
        buf = std::move(nb);
    }
    return static_cast<uint8_t*>(buf->ptr) + kDataOffset;
}

// Setters of the per-translation-unit copies of the device wait limit.
static std::vector<cudaError_t (*)(long long)>& wait_limit_setters() {
    static std::vector<cudaError_t (*)(long long)> v;
    return v;
}
void register_wait_limit_setter(cudaError_t (*setter)(long long)) { wait_limit_setters().push_back(setter); }

void check_stream_timeout(BeaconCudaStream* stream) {
    if (!stream || !stream->ws.buf) return;
    if (stream->ctx) set_device(stream->ctx);
    int flag = 0;
    BC_CUDA(cudaMemcpy(&flag, stream->ws.flags() + Workspace::kTimeoutFlag, sizeof(int), cudaMemcpyDeviceToHost));
    if (!flag) return;
    BC_CUDA(cudaDeviceSynchronize());
    BC_CUDA(cudaMemset(stream->ws.flags() + Workspace::kTimeoutFlag, 0, sizeof(int)));
    BC_CUDA(cudaMemset(stream->ws.counters(), 0, Workspace::kCounterInts * sizeof(int)));
    BC_CUDA(cudaDeviceSynchronize());
    fail(BEACON_CUDA_ERR_DEVICE_TIMEOUT,
         "a bounded device-side wait gave up (code " + std::to_string(flag) +
             "); the op's output is invalid. The stream's scratch counters were reset");
}

void check_context_timeouts(BeaconCudaContext* ctx) {
    std::vector<BeaconCudaStream*> ss;
    {
        std::lock_guard<std::mutex> lk(ctx->streams_mu);
        ss.assign(ctx->streams.begin(), ctx->streams.end());
    }
    for (BeaconCudaStream* st : ss) check_stream_timeout(st);
}

void set_device(BeaconCudaContext* ctx) { BC_CUDA(cudaSetDevice(ctx->device)); }

BeaconCudaTensor* new_tensor(BeaconCudaContext* ctx, const std::vector<int64_t>& shape, int32_t dtype) {
    auto* t = new BeaconCudaTensor();
    t->ctx = ctx;
    t->shape = shape;
    t->dtype = dtype;
    size_t nb = t->nbytes();
    try {
        t->storage = std::make_shared<DeviceBuffer>(nb);
    } catch (...) {
        delete t;
        throw;
    }
    return t;
}

BeaconCudaTensor* view_tensor(const BeaconCudaTensor* base, const std::vector<int64_t>& shape,
                              size_t byte_offset, int32_t dtype) {
    auto* t = new BeaconCudaTensor();
    t->ctx = base->ctx;
    t->shape = shape;
    t->dtype = dtype;
    t->storage = base->storage;
    t->offset = base->offset + byte_offset;
    t->q = base->q;
    return t;
}

}  // namespace bc

size_t BeaconCudaTensor::nbytes() const {
    if (bc::is_quantized(dtype)) return (size_t)q.total_bytes();
    return (size_t)numel() * bc::plain_elem_bytes(dtype);
}

using namespace bc;

namespace {

std::vector<int64_t> to_shape(const int64_t* shape, size_t ndim) {
    if (ndim > 0 && !shape) invalid("null shape");
    if (ndim > 8) invalid("at most 8 dimensions");
    std::vector<int64_t> s(shape, shape + ndim);
    for (int64_t d : s)
        if (d < 0) shape_err("negative dimension");
    return s;
}

void check_dtype_known(int32_t dtype) {
    if (!is_quantized(dtype) && plain_elem_bytes(dtype) == 0)
        fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "unknown dtype " + std::to_string(dtype));
}

BeaconCudaTensor* make_quantized(BeaconCudaContext* ctx, const void* raw, bool raw_on_device,
                                 const std::vector<int64_t>& shape, int32_t dtype, int32_t nibble_order) {
    if (shape.size() != 2) shape_err("quantized tensors are 2-D [N, K]");
    if (nibble_order != BEACON_CUDA_NIBBLE_REF_INTERLEAVED && nibble_order != BEACON_CUDA_NIBBLE_GGUF_SPLIT)
        invalid("unknown nibble order");
    QLayout L = make_qlayout(dtype, shape[0], shape[1]);
    auto* t = new BeaconCudaTensor();
    t->ctx = ctx;
    t->shape = shape;
    t->dtype = dtype;
    t->q = L;
    try {
        t->storage = std::make_shared<DeviceBuffer>((size_t)L.total_bytes());
        const size_t raw_bytes = (size_t)(L.n * (L.k / block_size(dtype)) * block_bytes(dtype));
        const uint8_t* src = static_cast<const uint8_t*>(raw);
        std::unique_ptr<DeviceBuffer> tmp;
        if (raw_on_device) BC_CUDA(cudaDeviceSynchronize());  // bytes may come from any stream
        if (!raw_on_device) {
            tmp = std::make_unique<DeviceBuffer>(raw_bytes);
            BC_CUDA(cudaMemcpyAsync(tmp->ptr, raw, raw_bytes, cudaMemcpyHostToDevice, ctx->internal));
            src = static_cast<const uint8_t*>(tmp->ptr);
        }
        launch_repack(L, src, nibble_order, static_cast<uint8_t*>(t->storage->ptr), nullptr, ctx->internal);
        BC_CUDA(cudaStreamSynchronize(ctx->internal));
    } catch (...) {
        delete t;
        throw;
    }
    return t;
}

}  // namespace

extern "C" {

const char* beacon_cuda_last_error_message(void) { return get_error(); }

int32_t beacon_cuda_context_create(int32_t device, BeaconCudaContext** out_ctx) {
    return guard([&]() -> int32_t {
        require(out_ctx != nullptr, "beacon_cuda_context_create: null argument");
        int count = 0;
        BC_CUDA(cudaGetDeviceCount(&count));
        if (device < 0 || device >= count) invalid("beacon_cuda_context_create: no such device");
        auto ctx = std::make_unique<BeaconCudaContext>();
        ctx->device = device;
        BC_CUDA(cudaSetDevice(device));
        BC_CUDA(cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device));
        int major = 0, minor = 0;
        BC_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
        BC_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
        if (major != 10 || minor != 0)
            fail(BEACON_CUDA_ERR_CUDA, "this build targets sm_100a (B200); device is sm_" +
                                           std::to_string(major) + std::to_string(minor));
        BC_CUDA(cudaStreamCreateWithFlags(&ctx->internal, cudaStreamNonBlocking));
        *out_ctx = ctx.release();
        return BEACON_CUDA_OK;
    });
}

void beacon_cuda_context_destroy(BeaconCudaContext* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    {
        // streams outliving their context keep their handles but lose the link
        std::lock_guard<std::mutex> lk(ctx->streams_mu);
        for (BeaconCudaStream* st : ctx->streams) st->ctx = nullptr;
        ctx->streams.clear();
    }
    if (ctx->internal) cudaStreamDestroy(ctx->internal);
    comm_destroy(ctx);
    delete ctx;
}

int32_t beacon_cuda_context_set_wait_limit(BeaconCudaContext* ctx, int64_t cycles) {
    return guard([&]() -> int32_t {
        require(ctx != nullptr, "null context");
        if (cycles < 0) invalid("set_wait_limit: the limit must be >= 0 clock cycles (0 restores the default)");
        set_device(ctx);
        BC_CUDA(cudaDeviceSynchronize());
        const long long v = cycles == 0 ? kBoundedWaitLimit : (long long)cycles;
        for (auto setter : wait_limit_setters()) BC_CUDA(setter(v));
        BC_CUDA(cudaDeviceSynchronize());
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_context_set_numerics(BeaconCudaContext* ctx, int32_t numerics) {
    return guard([&]() -> int32_t {
        require(ctx != nullptr, "null context");
        if (numerics < BEACON_CUDA_NUMERICS_FAST || numerics > BEACON_CUDA_NUMERICS_REF_RTZ)
            invalid("unknown numerics mode");
        ctx->numerics = numerics;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_stream_create(BeaconCudaContext* ctx, BeaconCudaStream** out_stream) {
    return guard([&]() -> int32_t {
        require(ctx && out_stream, "beacon_cuda_stream_create: null argument");
        set_device(ctx);
        auto s = std::make_unique<BeaconCudaStream>();
        s->ctx = ctx;
        s->owned = true;
        BC_CUDA(cudaStreamCreateWithFlags(&s->s, cudaStreamNonBlocking));
        {
            std::lock_guard<std::mutex> lk(ctx->streams_mu);
            ctx->streams.insert(s.get());
        }
        *out_stream = s.release();
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_stream_wrap(BeaconCudaContext* ctx, void* cuda_stream, BeaconCudaStream** out_stream) {
    return guard([&]() -> int32_t {
        require(ctx && out_stream, "beacon_cuda_stream_wrap: null argument");
        auto s = std::make_unique<BeaconCudaStream>();
        s->ctx = ctx;
        s->owned = false;
        s->s = static_cast<cudaStream_t>(cuda_stream);
        {
            std::lock_guard<std::mutex> lk(ctx->streams_mu);
            ctx->streams.insert(s.get());
        }
        *out_stream = s.release();
        return BEACON_CUDA_OK;
    });
}

void beacon_cuda_stream_destroy(BeaconCudaStream* stream) {
    if (!stream) return;
    if (stream->ctx) {
        std::lock_guard<std::mutex> lk(stream->ctx->streams_mu);
        stream->ctx->streams.erase(stream);
    }
    if (stream->s) cudaStreamSynchronize(stream->s);  // its workspace may still be in use
    if (stream->owned && stream->s) cudaStreamDestroy(stream->s);
    delete stream;
}

int32_t beacon_cuda_stream_synchronize(BeaconCudaStream* stream) {
    return guard([&]() -> int32_t {
        require(stream != nullptr, "null stream");
        BC_CUDA(cudaStreamSynchronize(stream->s));
        check_stream_timeout(stream);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_stream_handle(BeaconCudaStream* stream, void** out_cuda_stream) {
    return guard([&]() -> int32_t {
        require(stream && out_cuda_stream, "beacon_cuda_stream_handle: null argument");
        *out_cuda_stream = stream->s;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_upload(BeaconCudaContext* ctx, const void* host, const int64_t* shape,
                                  size_t ndim, int32_t dtype, int32_t nibble_order,
                                  BeaconCudaTensor** out_tensor) {
    return guard([&]() -> int32_t {
        require(ctx && out_tensor && (host || ndim == 0), "beacon_cuda_tensor_upload: null argument");
        check_dtype_known(dtype);
        set_device(ctx);
        auto s = to_shape(shape, ndim);
        if (is_quantized(dtype)) {
            *out_tensor = make_quantized(ctx, host, false, s, dtype, nibble_order);
            return BEACON_CUDA_OK;
        }
        BeaconCudaTensor* t = new_tensor(ctx, s, dtype);
        cudaError_t e = cudaMemcpy(t->data(), host, t->nbytes(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            delete t;
            cuda_check(e, "tensor upload");
        }
        *out_tensor = t;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_from_device_blocks(BeaconCudaContext* ctx, const void* device_bytes,
                                              const int64_t* shape, size_t ndim, int32_t dtype,
                                              int32_t nibble_order, BeaconCudaTensor** out_tensor) {
    return guard([&]() -> int32_t {
        require(ctx && out_tensor && device_bytes, "beacon_cuda_tensor_from_device_blocks: null argument");
        if (!is_quantized(dtype)) invalid("from_device_blocks needs a quantized dtype");
        set_device(ctx);
        *out_tensor = make_quantized(ctx, device_bytes, true, to_shape(shape, ndim), dtype, nibble_order);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_zeros(BeaconCudaContext* ctx, const int64_t* shape, size_t ndim, int32_t dtype,
                                 BeaconCudaTensor** out_tensor) {
    return guard([&]() -> int32_t {
        require(ctx && out_tensor, "beacon_cuda_tensor_zeros: null argument");
        check_dtype_known(dtype);
        if (is_quantized(dtype)) invalid("zeros of a quantized dtype is not meaningful");
        set_device(ctx);
        BeaconCudaTensor* t = new_tensor(ctx, to_shape(shape, ndim), dtype);
        cudaError_t e = cudaMemset(t->data(), 0, t->nbytes());
        if (e != cudaSuccess) {
            delete t;
            cuda_check(e, "tensor zeros");
        }
        *out_tensor = t;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_wrap_device(BeaconCudaContext* ctx, void* device_ptr, const int64_t* shape,
                                       size_t ndim, int32_t dtype, BeaconCudaTensor** out_tensor) {
    return guard([&]() -> int32_t {
        require(ctx && out_tensor && device_ptr, "beacon_cuda_tensor_wrap_device: null argument");
        check_dtype_known(dtype);
        if (is_quantized(dtype)) invalid("wrap_device takes plain dtypes only");
        auto* t = new BeaconCudaTensor();
        t->ctx = ctx;
        t->shape = to_shape(shape, ndim);
        t->dtype = dtype;
        t->storage = std::make_shared<DeviceBuffer>(device_ptr, t->nbytes());
        *out_tensor = t;
        return BEACON_CUDA_OK;
    });
}

void beacon_cuda_tensor_destroy(BeaconCudaTensor* tensor) { delete tensor; }

int32_t beacon_cuda_tensor_shape(const BeaconCudaTensor* t, int64_t* out_shape, size_t* inout_ndim) {
    return guard([&]() -> int32_t {
        require(t && inout_ndim, "beacon_cuda_tensor_shape: null argument");
        size_t cap = *inout_ndim;
        *inout_ndim = t->shape.size();
        if (cap < t->shape.size()) invalid("beacon_cuda_tensor_shape: capacity too small");
        if (!t->shape.empty()) {
            require(out_shape != nullptr, "beacon_cuda_tensor_shape: null shape buffer");
            std::copy(t->shape.begin(), t->shape.end(), out_shape);
        }
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_dtype(const BeaconCudaTensor* t, int32_t* out_dtype) {
    return guard([&]() -> int32_t {
        require(t && out_dtype, "beacon_cuda_tensor_dtype: null argument");
        *out_dtype = t->dtype;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_device_ptr(const BeaconCudaTensor* t, void** out_ptr) {
    return guard([&]() -> int32_t {
        require(t && out_ptr, "beacon_cuda_tensor_device_ptr: null argument");
        *out_ptr = t->data();
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_eval(BeaconCudaTensor* t, BeaconCudaStream* stream) {
    return guard([&]() -> int32_t {
        require(t != nullptr, "beacon_cuda_tensor_eval: null tensor");
        if (stream) {
            BC_CUDA(cudaStreamSynchronize(stream->s));
            check_stream_timeout(stream);
        } else {
            set_device(t->ctx);
            BC_CUDA(cudaDeviceSynchronize());
            check_context_timeouts(t->ctx);
        }
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_read_raw(const BeaconCudaTensor* t, void* out, size_t n_bytes) {
    return guard([&]() -> int32_t {
        require(t && out, "beacon_cuda_tensor_read_raw: null argument");
        if (n_bytes > t->nbytes()) shape_err("read_raw: more bytes requested than the tensor holds");
        set_device(t->ctx);
        BC_CUDA(cudaDeviceSynchronize());
        check_context_timeouts(t->ctx);
        BC_CUDA(cudaMemcpy(out, t->data(), n_bytes, cudaMemcpyDeviceToHost));
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_tensor_read_f32(const BeaconCudaTensor* t, float* out, size_t n_elements) {
    return guard([&]() -> int32_t {
        require(t && out, "beacon_cuda_tensor_read_f32: null argument");
        // cpu_backend.rs:425-433: reading more elements than exist is an error
        if (n_elements > (size_t)t->numel()) shape_err("read_f32: requested more elements than the tensor has");
        if (is_quantized(t->dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "read_f32 of a quantized tensor");
        set_device(t->ctx);
        BC_CUDA(cudaDeviceSynchronize());
        check_context_timeouts(t->ctx);
        const size_t eb = plain_elem_bytes(t->dtype);
        if (t->dtype == BEACON_CUDA_DTYPE_F32) {
            BC_CUDA(cudaMemcpy(out, t->data(), n_elements * 4, cudaMemcpyDeviceToHost));
            return BEACON_CUDA_OK;
        }
        std::vector<uint8_t> tmp(n_elements * eb);
        BC_CUDA(cudaMemcpy(tmp.data(), t->data(), tmp.size(), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n_elements; ++i) {
            switch (t->dtype) {
                case BEACON_CUDA_DTYPE_F16: {
                    uint16_t h;
                    std::memcpy(&h, &tmp[2 * i], 2);
                    uint32_t b = f16_to_f32_bits(h);
                    std::memcpy(&out[i], &b, 4);
                    break;
                }
                case BEACON_CUDA_DTYPE_BF16: {
                    uint16_t h;
                    std::memcpy(&h, &tmp[2 * i], 2);
                    uint32_t b = (uint32_t)h << 16;
                    std::memcpy(&out[i], &b, 4);
                    break;
                }
                case BEACON_CUDA_DTYPE_I32: {
                    int32_t v;
                    std::memcpy(&v, &tmp[4 * i], 4);
                    out[i] = (float)v;
                    break;
                }
                default: {
                    int8_t v;
                    std::memcpy(&v, &tmp[i], 1);
                    out[i] = (float)v;
                }
            }
        }
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_op_quantized_matmul(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                        const BeaconCudaTensor* x, const BeaconCudaTensor* w,
                                        const BeaconCudaTensor* scales, const BeaconCudaTensor* biases,
                                        int32_t group_size, int32_t bits, BeaconCudaTensor** out) {
    (void)scales;
    (void)biases;
    return guard([&]() -> int32_t {
        require(ctx && stream && x && w && out, "beacon_cuda_op_quantized_matmul: null argument");
        if (!is_quantized(w->dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "quantized_matmul: w is not quantized");
        const int exp_gs = (int)block_size(w->dtype);
        const int exp_bits = code_bits(w->dtype);
        if ((group_size != 0 && group_size != exp_gs) || (bits != 0 && bits != exp_bits))
            invalid("quantized_matmul: group_size/bits disagree with the weight's block type");
        if (x->dtype != BEACON_CUDA_DTYPE_F32 && x->dtype != BEACON_CUDA_DTYPE_F16)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "quantized_matmul: x must be F32 or F16");
        if (x->shape.empty()) shape_err("quantized_matmul: x has no dimensions");
        const int64_t K = x->shape.back();
        if (K != w->q.k) shape_err("quantized_matmul: inner dimension mismatch");
        const int64_t rows = x->numel() / std::max<int64_t>(K, 1);
        set_device(ctx);
        std::vector<int64_t> oshape = x->shape;
        oshape.back() = w->q.n;
        BeaconCudaTensor* o = new_tensor(ctx, oshape, BEACON_CUDA_DTYPE_F32);
        try {
            const int mode = ctx->numerics == BEACON_CUDA_NUMERICS_FAST ? MODE_FAST : MODE_F32;
            const bool rtz = ctx->numerics == BEACON_CUDA_NUMERICS_REF_RTZ;
            if (stream->ctx != ctx || w->ctx != ctx || x->ctx != ctx)
                invalid("quantized_matmul: the stream and tensors must belong to the context");
            if (rows > 16) {
                dense_qmatmul(ctx, stream, w, x->data(), x->dtype == BEACON_CUDA_DTYPE_F16, rows,
                              static_cast<float*>(o->data()), ctx->numerics);
            } else {
                const bool x16 = x->dtype == BEACON_CUDA_DTYPE_F16;
                for (int r0 = 0, b = 0; r0 < (int)rows; r0 += b) {
                    b = linear_chunk_rows(ctx, w->q, (int)rows - r0, mode);
                    LinearPlan pl = plan_linear(ctx, w->q, b, mode);
                    GemvScratch sc = stream_gemv_scratch(stream, pl, b, w->q);
                    // programmatic dependent launch: the weight stream may start
                    // while the stream's previous kernel finishes (weights are
                    // never written by other work; x is read after the wait)
                    launch_linear(pl, w->q, w->data(), static_cast<const uint8_t*>(x->data()) + (size_t)r0 * K * (x16 ? 2 : 4),
                                  x16, K, b, static_cast<float*>(o->data()) + (size_t)r0 * w->q.n, w->q.n, EPI_STORE,
                                  nullptr, 0, mode, rtz, sc, stream->s, nullptr, 0.0f, /*pdl=*/true);
                }
            }
        } catch (...) {
            delete o;
            throw;
        }
        *out = o;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_profile_quantized_matmul(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                             const BeaconCudaTensor* const* w, int32_t n_w,
                                             const BeaconCudaTensor* x, int32_t iters, float* out_avg_us,
                                             uint64_t* out_bytes) {
    return guard([&]() -> int32_t {
        require(ctx && stream && w && x && out_avg_us && out_bytes, "profile_quantized_matmul: null argument");
        require(n_w >= 1 && iters >= 1, "profile_quantized_matmul: need at least one weight and one iteration");
        require(stream->ctx == ctx, "profile_quantized_matmul: the stream belongs to another context");
        const QLayout& L0 = w[0]->q;
        for (int i = 0; i < n_w; ++i) {
            require(w[i] != nullptr && is_quantized(w[i]->dtype), "profile_quantized_matmul: w must be quantized");
            if (w[i]->dtype != L0.dtype || w[i]->q.n != L0.n || w[i]->q.k != L0.k)
                shape_err("profile_quantized_matmul: every weight must have the same block type and shape");
        }
        if (x->dtype != BEACON_CUDA_DTYPE_F32 && x->dtype != BEACON_CUDA_DTYPE_F16)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "profile_quantized_matmul: x must be F32 or F16");
        if (x->shape.empty() || x->shape.back() != L0.k) shape_err("profile_quantized_matmul: inner dimension");
        const int64_t rows = x->numel() / L0.k;
        if (rows < 1 || rows > 16) invalid("profile_quantized_matmul: 1..16 activation rows");
        set_device(ctx);
        const int mode = ctx->numerics == BEACON_CUDA_NUMERICS_FAST ? MODE_FAST : MODE_F32;
        const bool rtz = ctx->numerics == BEACON_CUDA_NUMERICS_REF_RTZ;
        const bool x16 = x->dtype == BEACON_CUDA_DTYPE_F16;
        DeviceBuffer y((size_t)rows * L0.n * 4);
        // the same row chunks as quantized_matmul
        std::vector<int> chunks;
        for (int r0 = 0, b = 0; r0 < (int)rows; r0 += b) chunks.push_back(b = linear_chunk_rows(ctx, L0, (int)rows - r0, mode));
        std::vector<LinearPlan> plans;
        std::vector<GemvScratch> scs;
        for (int b : chunks) plans.push_back(plan_linear(ctx, L0, b, mode));
        for (size_t c = 0; c < chunks.size(); ++c) scs.push_back(stream_gemv_scratch(stream, plans[c], chunks[c], L0));
        auto round = [&]() {
            for (int i = 0; i < n_w; ++i)
                for (size_t c = 0, r0 = 0; c < chunks.size(); r0 += chunks[c], ++c)
                    launch_linear(plans[c], L0, w[i]->data(),
                                  static_cast<const uint8_t*>(x->data()) + r0 * L0.k * (x16 ? 2 : 4), x16, L0.k,
                                  chunks[c], static_cast<float*>(y.ptr) + r0 * L0.n, L0.n, EPI_STORE, nullptr, 0, mode,
                                  rtz, scs[c], stream->s, nullptr, 0.0f, /*pdl=*/true);
        };
        round();  // warm-up (module load, shared-memory opt-in)
        cudaEvent_t e0, e1;
        BC_CUDA(cudaEventCreate(&e0));
        BC_CUDA(cudaEventCreate(&e1));
        BC_CUDA(cudaEventRecord(e0, stream->s));
        for (int it = 0; it < iters; ++it) round();
        BC_CUDA(cudaEventRecord(e1, stream->s));
        BC_CUDA(cudaEventSynchronize(e1));
        float ms = 0.0f;
        BC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        check_stream_timeout(stream);
        *out_avg_us = ms * 1000.0f / (float)(iters * n_w);
        const int64_t wbytes = L0.n * (L0.k / block_size(L0.dtype)) * block_bytes(L0.dtype);
        *out_bytes = (uint64_t)(wbytes + rows * L0.k * (x16 ? 2 : 4) + rows * L0.n * 4);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_op_dequantize_to_f16(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                         const BeaconCudaTensor* w, BeaconCudaTensor** out) {
    return guard([&]() -> int32_t {
        require(ctx && stream && w && out, "beacon_cuda_op_dequantize_to_f16: null argument");
        if (!is_quantized(w->dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "dequantize: w is not quantized");
        set_device(ctx);
        BeaconCudaTensor* o = new_tensor(ctx, {w->q.n, w->q.k}, BEACON_CUDA_DTYPE_F16);
        try {
            launch_dequant_f16(w->q, static_cast<const uint8_t*>(w->data()), static_cast<uint16_t*>(o->data()),
                               stream->s);
        } catch (...) {
            delete o;
            throw;
        }
        *out = o;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_op_quantize(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* x,
                                int32_t dtype, int32_t nibble_order, BeaconCudaTensor** out) {
    return guard([&]() -> int32_t {
        require(ctx && stream && x && out, "beacon_cuda_op_quantize: null argument");
        if (x->dtype != BEACON_CUDA_DTYPE_F32 || x->shape.size() != 2) shape_err("quantize: x must be F32 [N, K]");
        QLayout L = make_qlayout(dtype, x->shape[0], x->shape[1]);
        set_device(ctx);
        const size_t raw_bytes = (size_t)(L.n * (L.k / block_size(dtype)) * block_bytes(dtype));
        DeviceBuffer raw(raw_bytes);
        launch_quantize(dtype, static_cast<const float*>(x->data()), L.n, L.k, nibble_order,
                        static_cast<uint8_t*>(raw.ptr), stream->s);
        BC_CUDA(cudaStreamSynchronize(stream->s));
        *out = make_quantized(ctx, raw.ptr, true, x->shape, dtype, nibble_order);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_quantize_blocks(BeaconCudaContext* ctx, BeaconCudaStream* stream, const float* d_x,
                                    int64_t n_rows, int64_t k, int32_t dtype, int32_t nibble_order, void* d_out) {
    return guard([&]() -> int32_t {
        require(ctx && stream && d_x && d_out, "beacon_cuda_quantize_blocks: null argument");
        if (dtype != BEACON_CUDA_DTYPE_Q4_0 && dtype != BEACON_CUDA_DTYPE_Q8_0 && dtype != BEACON_CUDA_DTYPE_Q4_K)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "quantize: Q4_0, Q8_0 and Q4_K only");
        if (n_rows < 0 || k <= 0 || k % block_size(dtype)) shape_err("quantize: k must be a whole number of blocks");
        set_device(ctx);
        launch_quantize(dtype, d_x, n_rows, k, nibble_order, static_cast<uint8_t*>(d_out), stream->s);
        return BEACON_CUDA_OK;
    });
}

}  // extern "C"
