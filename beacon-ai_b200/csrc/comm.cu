// comm.cu -- tensor-parallel communicator (NCCL over NVLink / NVSwitch).
// The reference has no multi-GPU code (README.md:475-476); this is the
// exchange step of Megatron-style tensor parallelism: one f32 sum all-reduce
// after o_proj and one after down_proj, an all-gather of the vocab-split
// logits. Initialisation is non-blocking and bounded by a host timeout, and a
// failed or timed-out communicator is aborted, never waited on forever.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>

#include "internal.h"
#include "kernels.h"

namespace bc {

static void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess && r != ncclInProgress)
        fail(BEACON_CUDA_ERR_COMM, std::string(what) + ": " + ncclGetErrorString(r));
}

// Wait until a non-blocking NCCL call has finished, at most timeout_ms. On an
// error or a timeout the communicator is aborted (which frees it) and
// `aborted` is called first, so no caller keeps a pointer to it.
template <typename OnAbort>
static void nccl_wait(ncclComm_t comm, int timeout_ms, const char* what, OnAbort&& aborted) {
    auto t0 = std::chrono::steady_clock::now();
    auto abort_with = [&](const std::string& msg) {
        aborted();
        ncclCommAbort(comm);
        fail(BEACON_CUDA_ERR_COMM, msg);
    };
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(comm, &st);
        if (r != ncclSuccess) abort_with(std::string(what) + ": " + ncclGetErrorString(r));
        if (st == ncclSuccess) return;
        if (st != ncclInProgress) abort_with(std::string(what) + ": " + ncclGetErrorString(st));
        const auto us =
            std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count();
        if (us > (int64_t)timeout_ms * 1000) abort_with(std::string(what) + ": timed out");
        // an enqueue finishes within microseconds; an initialisation takes longer
        if (us > 1000) std::this_thread::sleep_for(std::chrono::microseconds(200));
        else std::this_thread::yield();
    }
}

// The context's communicator, or an error if a failed collective aborted it.
static ncclComm_t live_comm(BeaconCudaContext* ctx, const char* what) {
    if (ctx->comm_aborted || !ctx->comm)
        fail(BEACON_CUDA_ERR_COMM, std::string(what) + ": the communicator was aborted by an earlier failure");
    return static_cast<ncclComm_t>(ctx->comm);
}

static void mark_aborted(BeaconCudaContext* ctx) {
    ctx->comm = nullptr;
    ctx->comm_aborted = true;
}

void comm_destroy(BeaconCudaContext* ctx) {
    if (ctx && ctx->comm) {
        ncclCommDestroy(static_cast<ncclComm_t>(ctx->comm));
        ctx->comm = nullptr;
    }
}

// The communicator is non-blocking (bounded initialisation), so every call may
// return ncclInProgress and must have finished enqueueing before the next one.
void comm_all_reduce_sum(BeaconCudaContext* ctx, float* buf, size_t count, cudaStream_t s) {
    if (ctx->nranks <= 1) return;
    ncclComm_t comm = live_comm(ctx, "ncclAllReduce");
    const ncclResult_t r = ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, comm, s);
    if (r != ncclSuccess && r != ncclInProgress) {
        mark_aborted(ctx);
        ncclCommAbort(comm);
        nccl_check(r, "ncclAllReduce");
    }
    nccl_wait(comm, ctx->comm_timeout_ms, "ncclAllReduce", [&] { mark_aborted(ctx); });
}

void comm_all_gather(BeaconCudaContext* ctx, const float* send, float* recv, size_t count, cudaStream_t s) {
    if (ctx->nranks <= 1) {
        if (send != recv) BC_CUDA(cudaMemcpyAsync(recv, send, count * 4, cudaMemcpyDeviceToDevice, s));
        return;
    }
    ncclComm_t comm = live_comm(ctx, "ncclAllGather");
    const ncclResult_t r = ncclAllGather(send, recv, count, ncclFloat32, comm, s);
    if (r != ncclSuccess && r != ncclInProgress) {
        mark_aborted(ctx);
        ncclCommAbort(comm);
        nccl_check(r, "ncclAllGather");
    }
    nccl_wait(comm, ctx->comm_timeout_ms, "ncclAllGather", [&] { mark_aborted(ctx); });
}

}  // namespace bc

using namespace bc;

extern "C" {

int32_t beacon_cuda_comm_unique_id(void* out_id_128) {
    return guard([&]() -> int32_t {
        require(out_id_128 != nullptr, "comm_unique_id: null argument");
        static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
        ncclUniqueId id;
        nccl_check(ncclGetUniqueId(&id), "ncclGetUniqueId");
        std::memcpy(out_id_128, &id, 128);
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_comm_init(BeaconCudaContext* ctx, int32_t nranks, int32_t rank, const void* id_128,
                              int32_t timeout_ms) {
    return guard([&]() -> int32_t {
        require(ctx && id_128, "comm_init: null argument");
        if (nranks < 1 || rank < 0 || rank >= nranks) invalid("comm_init: bad rank / nranks");
        if (ctx->comm) invalid("comm_init: context already has a communicator");
        if (ctx->comm_aborted) fail(BEACON_CUDA_ERR_COMM, "comm_init: this context's communicator was aborted");
        set_device(ctx);
        ctx->comm_timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
        if (nranks == 1) {
            ctx->nranks = 1;
            ctx->rank = 0;
            return BEACON_CUDA_OK;
        }
        ncclUniqueId id;
        std::memcpy(&id, id_128, 128);
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        ncclComm_t comm = nullptr;
        nccl_check(ncclCommInitRankConfig(&comm, nranks, id, rank, &cfg), "ncclCommInitRankConfig");
        // on failure the half-made communicator is aborted here and never stored
        nccl_wait(comm, ctx->comm_timeout_ms, "ncclCommInitRankConfig", [] {});
        ctx->comm = comm;
        ctx->nranks = nranks;
        ctx->rank = rank;
        return BEACON_CUDA_OK;
    });
}

int32_t beacon_cuda_op_all_reduce_f32(BeaconCudaContext* ctx, BeaconCudaStream* stream, BeaconCudaTensor* t) {
    return guard([&]() -> int32_t {
        require(ctx && stream && t, "all_reduce: null argument");
        if (t->dtype != BEACON_CUDA_DTYPE_F32) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "all_reduce: F32 only");
        set_device(ctx);
        comm_all_reduce_sum(ctx, static_cast<float*>(t->data()), (size_t)t->numel(), stream->s);
        return BEACON_CUDA_OK;
    });
}

}  // extern "C"
