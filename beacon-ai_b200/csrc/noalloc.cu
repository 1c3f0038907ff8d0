// noalloc.cu -- a quantized matvec that allocates no memory at all.
//
// Some callers cannot let a library call cudaMalloc on their behalf: a
// serving process that reserves all device memory up front in its own arena
// (a stray allocation either fails or steals from the arena's budget), code
// that runs while another thread captures a CUDA graph on the device
// (cudaMalloc/cudaFree are not stream-ordered and may synchronise the device),
// and real-time decode loops that must never wait inside the allocator.
// beacon_cuda_quantized_matvec_noalloc serves them: the caller passes device
// pointers for the activations and the output, and the split-K scratch of the
// GEMV lives in one fixed array inside the library image.
//
// The array is 2 MiB (a file-scope __device__ variable, so every GPU that
// loads the library holds it until the process exits). Calls that overlap on
// the GPU, from any stream or thread, share it and race; the caller must
// order them. Its address is looked up once per device with
// cudaGetSymbolAddress on the first call made with that device current, so
// make the first call on each device outside any stream capture.
#include <algorithm>
#include <mutex>
#include <string>

#include "gemv.cuh"
#include "internal.h"
#include "kernels.h"

namespace bc {
namespace {

constexpr size_t kNoallocScratchBytes = 2u << 20;
constexpr size_t kNoallocCounterInts = 4096;  // split-K arrival counters: up to 4096 row groups
constexpr size_t kNoallocPartialFloats = (kNoallocScratchBytes - kNoallocCounterInts * sizeof(int)) / sizeof(float);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};

// Device address of the scratch array for `device` (which must be current).
void* noalloc_scratch(int device) {
    if (device < 0 || device >= kMaxDevices) invalid("quantized_matvec_noalloc: device index out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        cuda_check(e, "cudaGetSymbolAddress(no-alloc scratch)");
        if (!p) fail(BEACON_CUDA_ERR_CUDA, "cudaGetSymbolAddress returned a null scratch address");
        g_noalloc_addr[device] = p;
    }
    return g_noalloc_addr[device];
}

}  // namespace
}  // namespace bc

using namespace bc;

extern "C" int32_t beacon_cuda_quantized_matvec_noalloc(BeaconCudaStream* stream, const BeaconCudaTensor* w,
                                                        const void* d_x, int32_t x_dtype, int32_t batch,
                                                        float* d_y) {
    return guard([&]() -> int32_t {
        require(stream && w && d_x && d_y, "quantized_matvec_noalloc: null argument");
        if (!is_quantized(w->dtype)) fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "quantized_matvec_noalloc: w is not quantized");
        if (x_dtype != BEACON_CUDA_DTYPE_F32 && x_dtype != BEACON_CUDA_DTYPE_F16)
            fail(BEACON_CUDA_ERR_UNSUPPORTED_DTYPE, "quantized_matvec_noalloc: x must be F32 or F16");
        if (batch < 1 || batch > 16) invalid("quantized_matvec_noalloc: batch must be 1..16");
        BeaconCudaContext* ctx = w->ctx;
        require(stream->ctx == ctx, "quantized_matvec_noalloc: the stream belongs to another context than w");
        set_device(ctx);
        const QLayout& L = w->q;
        const int mode = ctx->numerics == BEACON_CUDA_NUMERICS_FAST ? MODE_FAST : MODE_F32;
        const bool rtz = ctx->numerics == BEACON_CUDA_NUMERICS_REF_RTZ;
        GemvPlan pl = plan_qgemv(ctx, L, batch, mode);
        if (pl.ksplit > 1 && (size_t)pl.ksplit * batch * L.n_pad > kNoallocPartialFloats) {
            // Fewer K-splits so the partial sums fit the fixed array; the
            // shared-memory bound on the tiles per CTA sets the minimum.
            const int64_t ktiles = L.ktiles();
            const size_t per_tile = gemv_smem_bytes(mode, pl.bpad, 256);
            const int64_t tps_max = std::max<int64_t>(1, (int64_t)((96 * 1024) / per_tile));
            const int64_t ks_min = (ktiles + tps_max - 1) / tps_max;
            const int64_t ks_fit = (int64_t)(kNoallocPartialFloats / ((size_t)batch * L.n_pad));
            int64_t ks = std::max<int64_t>(1, ks_fit);
            if (ks_min > 1 && ks < ks_min)
                shape_err("quantized_matvec_noalloc: batch x rows x K-splits exceeds the fixed 2 MiB scratch (" +
                          std::to_string((size_t)ks_min * batch * L.n_pad) + " partial sums > " +
                          std::to_string(kNoallocPartialFloats) + ")");
            ks = std::max(ks, ks_min);
            const int64_t tps = (ktiles + ks - 1) / ks;
            pl.tps = (int)tps;
            pl.ksplit = (int)((ktiles + tps - 1) / tps);
            pl.smem = gemv_smem_bytes(mode, pl.bpad, (int)tps * 256);
        }
        GemvScratch sc;
        if (pl.ksplit > 1) {
            if ((size_t)L.groups() > kNoallocCounterInts)
                shape_err("quantized_matvec_noalloc: more than " + std::to_string(kNoallocCounterInts * 32) +
                          " rows need a K-split larger than the fixed scratch holds");
            uint8_t* base = static_cast<uint8_t*>(noalloc_scratch(ctx->device));
            sc.counters = reinterpret_cast<int*>(base);
            sc.counter_count = (int64_t)kNoallocCounterInts;
            sc.partial = reinterpret_cast<float*>(base + kNoallocCounterInts * sizeof(int));
            sc.partial_floats = kNoallocPartialFloats;
            // the array keeps whatever the previous call left: the arrival
            // counters must start at zero
            BC_CUDA(cudaMemsetAsync(sc.counters, 0, (size_t)L.groups() * sizeof(int), stream->s));
        }
        launch_qgemv(pl, L, w->data(), d_x, x_dtype == BEACON_CUDA_DTYPE_F16, L.k, batch, d_y, L.n, EPI_STORE,
                     nullptr, 0, mode, rtz, sc, stream->s);
        return BEACON_CUDA_OK;
    });
}
