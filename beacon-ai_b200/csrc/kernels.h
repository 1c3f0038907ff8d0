// kernels.h -- host-side launchers shared between translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <utility>

#include "internal.h"

namespace bc {

enum GemvMode { MODE_FAST = 0, MODE_F32 = 1 };
enum GemvEpilogue { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_QKV = 3 };

// EPI_QKV: the fused q/k/v projection of one decoder layer writes its rows
// straight to their consumers. Rows [0, qd) are queries, [qd, qd + kd) keys,
// then kd value rows. Query and key pairs (2i, 2i+1) of each head are rotated
// at the row's position (RoPE with interleaved pairs, rope.rs:10-60): queries
// go to q[row][qd] as f32, keys and values to the caches at [seq][pos].
// Batch row b of the launch is model row row0 + b, at position
// *pos_ptr (or pos_imm) + row * pos_step, in sequence row * seq_step; a
// position outside [0, max_ctx) sets *err = 2 and writes nothing.
// Activations quantised by the kernel that produces them (decode, fast
// numerics): the consumer GEMV's shared-memory staging image, in global
// memory -- int16 codes [bpad][kspan], then per 32-block of each row the
// pair (f32 scale, code sum as f32) [bpad][kspan/32] -- plus, when the consumer fuses an
// RMSNorm, the sums of squares of the unnormalised values per 32-block
// [bpad][kspan/32] (the codes are then of x * norm_w, and the consumer scales
// its outputs by 1/rms). The producer writes rows b < batch only; rows
// b >= batch stay as they were (the consumer never stores them).
struct QxImage {
    uint8_t* data = nullptr;         // staging image; null: none
    float* ss = nullptr;             // per-block sums of squares; null: no norm
    int kspan = 0;                   // consumer's padded K (multiple of 256)
    int bpad = 1;                    // consumer's staged rows
    int perm = 0;                    // 1: Q4_0 element order within 8-groups
    const float* norm_w = nullptr;   // producer side: the consumer's norm weight
    int* pairs = nullptr;            // SwiGLU producer: one arrival counter per two 16-output groups (zero at rest)
};

struct QkvEpi {
    float* q = nullptr;
    void* kc = nullptr;
    void* vc = nullptr;
    int kv_f16 = 1;
    const float* cs = nullptr;  // rope tables [max_ctx][d / 2]
    const float* sn = nullptr;
    int qd = 0, kd = 0, d = 0;
    int64_t cache_sb = 0;
    const int* pos_ptr = nullptr;
    int pos_imm = 0, pos_step = 0, seq_step = 0, row0 = 0, max_ctx = 0;
    int* err = nullptr;
};

// Scratch for split-K GEMV: partial sums and one arrival counter per 32-row
// group. Counters must be zero before the first launch; every launch leaves
// them at zero again.
struct GemvScratch {
    float* partial = nullptr;
    int* counters = nullptr;
    size_t partial_floats = 0;
    int64_t counter_count = 0;
    int* err = nullptr;  // set by a kernel whose bounded wait gave up
};

struct GemvPlan {
    int ksplit = 1;
    int tps = 1;  // 256-column tiles per CTA
    int bpad = 1;
    size_t smem = 0;
};

// y[b, n] (+)= sum_k W[n, k] x[b, k] for a tiled quantized W (QLayout).
//  x: batch rows of x_ld elements, f32 or f16. y: f32, row stride y_ld.
//  EPI_ADD: y = res + W x.  EPI_SWIGLU: rows of W interleave gate/up per
//  16-row half group; y has n/2 columns = silu(gate) * up.
GemvPlan plan_qgemv(const BeaconCudaContext* ctx, const QLayout& L, int batch, int mode);
void launch_qgemv(const GemvPlan& plan, const QLayout& L, const void* w, const void* x,
                  bool x_f16, int64_t x_ld, int batch, float* y, int64_t y_ld, int epi,
                  const float* res, int64_t res_ld, int mode, bool rtz, const GemvScratch& scratch,
                  cudaStream_t s);

// Per-format instantiation entry points (gemv_<fmt>.cu).
struct GemvLaunch {
    const GemvPlan* plan;
    const QLayout* L;
    const void* w;
    const void* x;
    bool x_f16;
    int64_t x_ld;
    int batch;
    float* y;
    int64_t y_ld;
    int epi;
    const float* res;
    int64_t res_ld;
    int mode;
    bool rtz;
    GemvScratch scratch;
    cudaStream_t s;
    const float* norm_w = nullptr;  // fused RMSNorm weight (persistent kernel only)
    float norm_eps = 0.0f;
    bool pdl = false;               // launch with programmatic stream serialisation
    const QkvEpi* qkv = nullptr;    // EPI_QKV destinations
    QxImage qx;                     // consumer: pre-quantised activations (persistent kernel, FAST)
    QxImage qy;                     // producer (EPI_ADD): also write y quantised for the next GEMV
};

// cudaLaunchKernelEx with programmatic stream serialisation when `pdl`.
template <typename... KArgs, typename... Args>
void launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl,
                   Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    cuda_check(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), "cudaLaunchKernelEx");
}
// Opt a kernel in to the device's largest dynamic shared memory. Kernels
// launched with several sizes (and captured into graphs) are covered for all
// of them, whichever launch set the attribute last.
int device_smem_optin();
template <typename... KArgs>
void allow_max_dynamic_smem(void (*kern)(KArgs...)) {
    cudaFuncAttributes fa;
    cuda_check(cudaFuncGetAttributes(&fa, kern), "cudaFuncGetAttributes");
    cuda_check(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    device_smem_optin() - (int)fa.sharedSizeBytes),
               "cudaFuncSetAttribute");
}
void launch_qgemv_q4_0(const GemvLaunch& a);
void launch_qgemv_q8_0(const GemvLaunch& a);
void launch_qgemv_q4_k(const GemvLaunch& a);
// Formats with a dedicated tile layout and integer fast path (the others
// keep raw block bytes per tile and compute in f32, gemv_generic.cuh).
inline bool is_core_format(int32_t dtype) {
    return dtype == BEACON_CUDA_DTYPE_Q4_0 || dtype == BEACON_CUDA_DTYPE_Q8_0 || dtype == BEACON_CUDA_DTYPE_Q4_K;
}
void launch_qgemv_q4_1(const GemvLaunch& a);
void launch_qgemv_q5_0(const GemvLaunch& a);
void launch_qgemv_q5_1(const GemvLaunch& a);
void launch_qgemv_q2_k(const GemvLaunch& a);
void launch_qgemv_q3_k(const GemvLaunch& a);
void launch_qgemv_q5_k(const GemvLaunch& a);
void launch_qgemv_q6_k(const GemvLaunch& a);
void launch_qgemv_q8_k(const GemvLaunch& a);
// The tiled kernel of any block format.
void launch_qgemv_any(const GemvLaunch& a);

// The persistent TMA-fed GEMV (gemv3.cuh) for batch <= 8 when its ring and the
// staged activations fit in shared memory; otherwise the tiled GEMV above.
struct LinearPlan {
    bool v3 = false;
    bool mma = false;  // persistent kernel, fast numerics: tensor-core tile consumer
    GemvPlan v2;
    int nctas = 0, stages = 0, bpad = 1;
    size_t smem = 0;
    int64_t total_warps = 0;
    size_t scratch_floats(int batch, const QLayout& L) const;
};
LinearPlan plan_linear(const BeaconCudaContext* ctx, const QLayout& L, int batch, int mode);
// Rows (of up to 16 remaining) for the next GEMV launch.
int linear_chunk_rows(const BeaconCudaContext* ctx, const QLayout& L, int rem, int mode);
// norm_w (persistent plan only): y = W rmsnorm(x, norm_w, norm_eps).
void launch_linear(const LinearPlan& plan, const QLayout& L, const void* w, const void* x, bool x_f16, int64_t x_ld,
                   int batch, float* y, int64_t y_ld, int epi, const float* res, int64_t res_ld, int mode, bool rtz,
                   const GemvScratch& scratch, cudaStream_t s, const float* norm_w = nullptr, float norm_eps = 0.0f,
                   bool pdl = false, const QkvEpi* qkv = nullptr, const QxImage* qx = nullptr,
                   const QxImage* qy = nullptr);
void launch_qgemv3_q4_0(const LinearPlan& pl, const GemvLaunch& a);
void launch_qgemv3_q8_0(const LinearPlan& pl, const GemvLaunch& a);
void launch_qgemv3_q4_k(const LinearPlan& pl, const GemvLaunch& a);

// Quantized layout kernels (quant.cu). row_map (device, one entry per tiled
// row, optional): raw row to copy, -1 = zero row, -2 = leave the row as is.
void launch_repack(const QLayout& L, const uint8_t* raw, int nibble_order, uint8_t* tiled,
                   const int64_t* row_map, cudaStream_t s);
void launch_dequant_f16(const QLayout& L, const uint8_t* tiled, uint16_t* out, cudaStream_t s);
void launch_quantize(int32_t dtype, const float* x, int64_t n_rows, int64_t k, int nibble_order,
                     uint8_t* raw, cudaStream_t s);

// Split-K scratch carved from the stream's workspace (fixed zeroed counters).
struct LinearPlan;
GemvScratch stream_gemv_scratch(BeaconCudaStream* stream, const LinearPlan& pl, int batch, const QLayout& L);

// Prefill-sized quantized matmul (rows > 16): out[rows, N] = x @ W^T.
void dense_qmatmul(BeaconCudaContext* ctx, BeaconCudaStream* stream, const BeaconCudaTensor* w, const void* x,
                   bool x_f16, int64_t rows, float* out, int numerics);

// The model's configuration and context (model.cu), for the GGUF loader.
const BeaconCudaModelConfig& model_config_of(const BeaconCudaModel* m);
BeaconCudaContext* model_context_of(const BeaconCudaModel* m);

// Token sampling (sample.cu): rows of logits [rows][ld] (V used) -> out[rows].
struct ArgmaxSummary;
void launch_sample(const float* logits, int64_t ld, int64_t V, int rows, const int32_t* prev, int n_prev,
                   const BeaconCudaSamplingParams& p, const float* uniforms, float* work, int32_t* out,
                   ArgmaxSummary* argmax_scratch, cudaStream_t s);
// Scratch of launch_sample: work rows, then (256-byte aligned) the argmax summaries.
size_t sample_scratch_bytes(int64_t V, int rows);

// Tensor parallelism (comm.cu).
void comm_destroy(BeaconCudaContext* ctx);
void comm_all_reduce_sum(BeaconCudaContext* ctx, float* buf, size_t count, cudaStream_t s);
void comm_all_gather(BeaconCudaContext* ctx, const float* send, float* recv, size_t count, cudaStream_t s);

}  // namespace bc
