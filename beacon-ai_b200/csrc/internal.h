// internal.h -- handle definitions and the ABI exception guard shared by the
// translation units of libbeacon_cuda.so. Nothing here crosses the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/beacon_cuda.h"

namespace bc {

// ---------------------------------------------------------------------------
// Errors. Thread-local message as in shim/src/errors.cpp:13; the guard maps
// exception types to status codes as shim/src/guard.h:12-39 does.
// ---------------------------------------------------------------------------
void set_error(const std::string& msg) noexcept;
void clear_error() noexcept;
const char* get_error() noexcept;

struct Error : std::runtime_error {
    int32_t status;
    Error(int32_t s, const std::string& m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void fail(int32_t status, const std::string& msg) { throw Error(status, msg); }
[[noreturn]] inline void invalid(const std::string& msg) {
    throw Error(BEACON_CUDA_ERR_INVALID_ARGUMENT, msg);
}
[[noreturn]] inline void shape_err(const std::string& msg) {
    throw Error(BEACON_CUDA_ERR_SHAPE_MISMATCH, msg);
}

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        int32_t st = e == cudaErrorMemoryAllocation ? BEACON_CUDA_ERR_OUT_OF_MEMORY
                                                    : BEACON_CUDA_ERR_CUDA;
        throw Error(st, std::string(what) + ": " + cudaGetErrorString(e));
    }
}
#define BC_CUDA(call) ::bc::cuda_check((call), #call)
// After a kernel launch: reports configuration errors without synchronizing.
#define BC_LAUNCHED(name) ::bc::cuda_check(cudaGetLastError(), name)

template <typename F>
int32_t guard(F&& fn) noexcept {
    try {
        clear_error();
        return fn();
    } catch (const Error& e) {
        set_error(e.what());
        return e.status;
    } catch (const std::bad_alloc& e) {
        set_error(e.what());
        return BEACON_CUDA_ERR_OUT_OF_MEMORY;
    } catch (const std::invalid_argument& e) {
        set_error(e.what());
        return BEACON_CUDA_ERR_INVALID_ARGUMENT;
    } catch (const std::out_of_range& e) {
        set_error(e.what());
        return BEACON_CUDA_ERR_SHAPE_MISMATCH;
    } catch (const std::exception& e) {
        set_error(e.what());
        return BEACON_CUDA_ERR_UNKNOWN;
    } catch (...) {
        set_error("unknown C++ exception caught at the ABI boundary");
        return BEACON_CUDA_ERR_UNKNOWN;
    }
}

inline void require(bool ok, const char* msg) {
    if (!ok) invalid(msg);
}

// ---------------------------------------------------------------------------
// Dtypes and the quantized device layout.
// ---------------------------------------------------------------------------
bool is_quantized(int32_t dtype);
int64_t block_size(int32_t dtype);   // elements per GGUF block
int64_t block_bytes(int32_t dtype);  // bytes per GGUF block
size_t plain_elem_bytes(int32_t dtype);

// Quantized weights live on the device in "row-group tiles": 32 rows x 256
// columns, [16-byte meta x 32 lanes][16-byte chunks x 32 lanes] so that each
// warp-wide 128-bit load covers 512 contiguous bytes and lane l owns row l.
struct QLayout {
    int32_t dtype = 0;
    int64_t n = 0, k = 0;        // logical rows / columns
    int64_t n_pad = 0, k_pad = 0;  // rounded to 32 rows / 256 columns
    int32_t chunks = 0;          // 16-byte qs chunks per row per tile
    int64_t tile_bytes = 0;      // 32 * (16 + 16 * chunks)
    int64_t groups() const { return n_pad / 32; }
    int64_t ktiles() const { return k_pad / 256; }
    int64_t total_bytes() const { return groups() * ktiles() * tile_bytes; }
};
QLayout make_qlayout(int32_t dtype, int64_t n, int64_t k);

// ---------------------------------------------------------------------------
// Device memory.
// ---------------------------------------------------------------------------
struct DeviceBuffer {
    void* ptr = nullptr;
    size_t bytes = 0;
    bool owned = true;
    DeviceBuffer(size_t n);
    DeviceBuffer(void* p, size_t n) : ptr(p), bytes(n), owned(false) {}
    ~DeviceBuffer();
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
};

// Grow-only scratch arena of one stream. Layout: [counters | flags | data].
// The split-K arrival counters sit at a fixed offset and are zero whenever no
// kernel is running (each launch resets the ones it used), so data written
// by one op can never be mistaken for counters by the next. Each stream has
// its own, so ops on different streams of a context never share scratch.
// Growing is refused during stream capture, and a replaced buffer is kept
// (not freed) until the stream is destroyed, so work already enqueued -- or a
// graph captured earlier -- never touches freed memory.
struct Workspace {
    static constexpr size_t kCounterInts = 1 << 16;  // one per 32-row group: 2M rows
    static constexpr size_t kFlagInts = 64;
    static constexpr size_t kDataOffset = (kCounterInts + kFlagInts) * sizeof(int);
    std::unique_ptr<DeviceBuffer> buf;
    std::vector<std::unique_ptr<DeviceBuffer>> retired;
    void* get(size_t data_bytes, cudaStream_t s);  // returns the data region
    int* counters() const { return static_cast<int*>(buf->ptr); }
    int* flags() const { return static_cast<int*>(buf->ptr) + kCounterInts; }
    // flags()[kTimeoutFlag]: a bounded device wait of an op on this stream gave up
    static constexpr int kTimeoutFlag = 1;
};

}  // namespace bc

struct BeaconCudaContext {
    int device = 0;
    int sm_count = 148;
    int32_t numerics = BEACON_CUDA_NUMERICS_FAST;
    cudaStream_t internal = nullptr;  // uploads and frees outside any user stream
    // streams made on this context (their workspaces are checked for device
    // timeouts at the context-wide synchronisation points)
    std::mutex streams_mu;
    std::set<BeaconCudaStream*> streams;
    // tensor parallelism
    void* comm = nullptr;  // ncclComm_t
    bool comm_aborted = false;  // a failed or timed-out collective aborted the communicator
    int nranks = 1, rank = 0;
    int comm_timeout_ms = 60000;
};

struct BeaconCudaStream {
    BeaconCudaContext* ctx = nullptr;
    cudaStream_t s = nullptr;
    bool owned = false;
    bc::Workspace ws;  // split-K scratch, arrival counters and error flags of ops on this stream
};

struct BeaconCudaTensor {
    BeaconCudaContext* ctx = nullptr;
    std::vector<int64_t> shape;
    int32_t dtype = BEACON_CUDA_DTYPE_F32;
    std::shared_ptr<bc::DeviceBuffer> storage;
    size_t offset = 0;  // bytes into storage
    bc::QLayout q;      // quantized tensors only
    void* data() const { return static_cast<char*>(storage->ptr) + offset; }
    int64_t numel() const {
        int64_t n = 1;
        for (int64_t d : shape) n *= d;
        return n;
    }
    size_t nbytes() const;
};

namespace bc {

BeaconCudaTensor* new_tensor(BeaconCudaContext* ctx, const std::vector<int64_t>& shape,
                             int32_t dtype);
BeaconCudaTensor* view_tensor(const BeaconCudaTensor* base, const std::vector<int64_t>& shape,
                              size_t byte_offset, int32_t dtype);
void set_device(BeaconCudaContext* ctx);
inline cudaStream_t stream_of(BeaconCudaStream* s) { return s ? s->s : nullptr; }

// After the stream (or the whole device) has been synchronised: if a bounded
// device wait of an op on this stream gave up, clear the flag, re-zero the
// stream's arrival counters (a warp that gave up never arrived) and throw
// BEACON_CUDA_ERR_DEVICE_TIMEOUT.
void check_stream_timeout(BeaconCudaStream* stream);
// The same for every stream of the context (after a device synchronisation).
void check_context_timeouts(BeaconCudaContext* ctx);

}  // namespace bc
