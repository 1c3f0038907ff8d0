/*
 * beacon_cuda.h -- C ABI of the B200 (sm_100a) backend for Beacon's
 * quantized decode path.
 *
 * This is the surface a `beacon-cuda` crate binds to implement beacon-core's
 * `ComputeBackend` trait (crates/beacon-core/src/backend.rs:14-167). It copies
 * the conventions of the MLX shim (shim/include/beacon_shim.h):
 *   - opaque handles (beacon_shim.h:18-21);
 *   - every call returns an int32_t status, BEACON_CUDA_OK == 0
 *     (beacon_shim.h:24-33), output parameters come last;
 *   - *_destroy returns void;
 *   - beacon_cuda_last_error_message() is thread-local and valid until the
 *     next call on the same thread (beacon_shim.h:222-227,
 *     shim/src/errors.cpp:13);
 *   - C++ exceptions never cross the ABI (shim/src/guard.h:12-39): bad_alloc
 *     maps to OUT_OF_MEMORY, invalid_argument to INVALID_ARGUMENT,
 *     out_of_range to SHAPE_MISMATCH.
 * No torch or CUDA types appear in any signature: streams and device
 * pointers travel as void*.
 *
 * Quantized weights are uploaded as raw GGUF block bytes, row-major [N, K]
 * with blocks along K (crates/beacon-format/src/gguf/tensor_info.rs:40-48).
 * The tensor remembers its block type, so `quantized_matmul` needs no
 * separate scales/biases tensors (they are MLX-affine only and may be NULL).
 */
#ifndef BEACON_CUDA_H
#define BEACON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* === Handles (opaque) === */
typedef struct BeaconCudaContext BeaconCudaContext;
typedef struct BeaconCudaStream BeaconCudaStream;
typedef struct BeaconCudaTensor BeaconCudaTensor;
typedef struct BeaconCudaModel BeaconCudaModel;

/* === Status codes (values 0-4 and 99 as BeaconStatus, beacon_shim.h:24-33) === */
typedef enum {
    BEACON_CUDA_OK = 0,
    BEACON_CUDA_ERR_INVALID_ARGUMENT = 1,
    BEACON_CUDA_ERR_OUT_OF_MEMORY = 2,
    BEACON_CUDA_ERR_SHAPE_MISMATCH = 3,
    BEACON_CUDA_ERR_UNSUPPORTED_DTYPE = 4,
    BEACON_CUDA_ERR_KERNEL_LAUNCH = 5,  /* slot of BEACON_ERR_METAL_COMPILE */
    BEACON_CUDA_ERR_CUDA = 6,           /* slot of BEACON_ERR_MLX_INTERNAL */
    BEACON_CUDA_ERR_CONTEXT_OVERFLOW = 7, /* EngineError::ContextOverflow (error.rs:24-26) */
    BEACON_CUDA_ERR_COMM = 8,           /* NCCL failure or timeout */
    BEACON_CUDA_ERR_DEVICE_TIMEOUT = 9, /* a bounded device-side wait ran out */
    BEACON_CUDA_ERR_UNKNOWN = 99
} BeaconCudaStatus;

/* === Dtypes: the BeaconDtype discriminants (crates/beacon-format/src/dtype.rs:12-29) === */
typedef enum {
    BEACON_CUDA_DTYPE_F32 = 0,
    BEACON_CUDA_DTYPE_F16 = 1,
    BEACON_CUDA_DTYPE_BF16 = 2,
    BEACON_CUDA_DTYPE_I32 = 3,
    BEACON_CUDA_DTYPE_I8 = 4,
    BEACON_CUDA_DTYPE_Q4_0 = 100,
    BEACON_CUDA_DTYPE_Q4_K = 101,
    BEACON_CUDA_DTYPE_Q5_K = 102,
    BEACON_CUDA_DTYPE_Q6_K = 103,
    BEACON_CUDA_DTYPE_Q8_0 = 104,
    BEACON_CUDA_DTYPE_Q4_1 = 105,
    BEACON_CUDA_DTYPE_Q5_0 = 106,
    BEACON_CUDA_DTYPE_Q5_1 = 107,
    BEACON_CUDA_DTYPE_Q2_K = 108,
    BEACON_CUDA_DTYPE_Q3_K = 109,
    BEACON_CUDA_DTYPE_Q8_K = 110
} BeaconCudaDtype;

/* Q4_0 nibble order of uploaded bytes. REF_INTERLEAVED is what the reference's
 * CPU code computes (byte i -> elements 2i, 2i+1; dequant.rs:170-176,
 * q4.rs:33-41). GGUF_SPLIT is the GGUF file order (byte i -> i, i+16). */
typedef enum {
    BEACON_CUDA_NIBBLE_REF_INTERLEAVED = 0,
    BEACON_CUDA_NIBBLE_GGUF_SPLIT = 1
} BeaconCudaNibbleOrder;

/* Arithmetic of quantized_matmul and of the model's linears.
 *  FAST:    activations quantized per 32 elements to int16, integer dot
 *           products (dp2a) against the 4/8-bit codes, f32 block scaling.
 *  EXACT:   f32 activations times the unrounded f32 weight q*d (the values
 *           of q4::dequantize_q4_0_block, q4.rs:26-42), f32 accumulation.
 *  REF_RTZ: f32 activations times the f16-truncated weights that the CPU
 *           engine consumes (f16_to_f32(dequantize_to_f16(.)),
 *           dequant.rs:33-60), f32 accumulation. */
typedef enum {
    BEACON_CUDA_NUMERICS_FAST = 0,
    BEACON_CUDA_NUMERICS_EXACT = 1,
    BEACON_CUDA_NUMERICS_REF_RTZ = 2
} BeaconCudaNumerics;

/* === Lifecycle (beacon_shim.h:49-54) === */
int32_t beacon_cuda_context_create(int32_t device, BeaconCudaContext** out_ctx);
void    beacon_cuda_context_destroy(BeaconCudaContext* ctx);
int32_t beacon_cuda_context_set_numerics(BeaconCudaContext* ctx, int32_t numerics);
/* Limit, in SM clock cycles, of every bounded device-side wait on progress
 * (tile copies, pipeline stages, split merges) of the kernels on this
 * context's device; 0 restores the default 2^31 (about 1.1 s at 1965 MHz).
 * A wait that runs out makes its kernel record the failure, let the work it
 * already issued finish, and return. The failure is reported as
 * BEACON_CUDA_ERR_DEVICE_TIMEOUT by the next synchronising call
 * (stream_synchronize, tensor_eval, tensor_read_*, model_decode_step,
 * model_forward, model_synchronize), which also resets the scratch counters
 * so the context stays usable. No reference counterpart (the reference runs
 * no device code); shim/src/guard.h:12-39 is the status convention. */
int32_t beacon_cuda_context_set_wait_limit(BeaconCudaContext* ctx, int64_t cycles);

int32_t beacon_cuda_stream_create(BeaconCudaContext* ctx, BeaconCudaStream** out_stream);
/* Borrow an existing cudaStream_t (passed as void*); destroy does not free it. */
int32_t beacon_cuda_stream_wrap(BeaconCudaContext* ctx, void* cuda_stream,
                                BeaconCudaStream** out_stream);
void    beacon_cuda_stream_destroy(BeaconCudaStream* stream);
int32_t beacon_cuda_stream_synchronize(BeaconCudaStream* stream);

/* === Tensors (beacon_shim.h:56-88) === */
/* Replaces beacon_tensor_from_mmap (beacon_shim.h:59-64): copies host bytes
 * to the device once. Quantized: shape is the logical [N, K] element shape and
 * `host` holds N * K / block_size GGUF blocks. */
int32_t beacon_cuda_tensor_upload(BeaconCudaContext* ctx, const void* host,
                                  const int64_t* shape, size_t ndim, int32_t dtype,
                                  int32_t nibble_order, BeaconCudaTensor** out_tensor);
/* Same as upload but the GGUF bytes are already in device memory. */
int32_t beacon_cuda_tensor_from_device_blocks(BeaconCudaContext* ctx, const void* device_bytes,
                                              const int64_t* shape, size_t ndim, int32_t dtype,
                                              int32_t nibble_order, BeaconCudaTensor** out_tensor);
/* beacon_tensor_zeros (beacon_shim.h:66-71). */
int32_t beacon_cuda_tensor_zeros(BeaconCudaContext* ctx, const int64_t* shape, size_t ndim,
                                 int32_t dtype, BeaconCudaTensor** out_tensor);
/* Non-owning view of caller device memory (plain dtypes only). */
int32_t beacon_cuda_tensor_wrap_device(BeaconCudaContext* ctx, void* device_ptr,
                                       const int64_t* shape, size_t ndim, int32_t dtype,
                                       BeaconCudaTensor** out_tensor);
void    beacon_cuda_tensor_destroy(BeaconCudaTensor* tensor);
int32_t beacon_cuda_tensor_shape(const BeaconCudaTensor* t, int64_t* out_shape, size_t* inout_ndim);
int32_t beacon_cuda_tensor_dtype(const BeaconCudaTensor* t, int32_t* out_dtype);
int32_t beacon_cuda_tensor_device_ptr(const BeaconCudaTensor* t, void** out_ptr);
/* beacon_tensor_eval (beacon_shim.h:84): waits for the stream. */
int32_t beacon_cuda_tensor_eval(BeaconCudaTensor* t, BeaconCudaStream* stream);
/* beacon_tensor_read_f32 (beacon_shim.h:88); F16/BF16/I32 are converted. */
int32_t beacon_cuda_tensor_read_f32(const BeaconCudaTensor* t, float* out, size_t n_elements);
int32_t beacon_cuda_tensor_read_raw(const BeaconCudaTensor* t, void* out, size_t n_bytes);

/* === Ops: ComputeBackend methods (backend.rs:21-166; beacon_shim.h:90-189) === */
int32_t beacon_cuda_op_matmul(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                              const BeaconCudaTensor* a, const BeaconCudaTensor* b,
                              BeaconCudaTensor** out);
/* backend.rs:32-41: out = x @ dequant(w)^T, x [S, K] (F32 or F16), out [S, N] F32.
 * scales/biases may be NULL; group_size/bits must agree with w's block type
 * (32/4 Q4_0, 32/8 Q8_0, 256/4 Q4_K) or be 0. */
int32_t beacon_cuda_op_quantized_matmul(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                        const BeaconCudaTensor* x, const BeaconCudaTensor* w,
                                        const BeaconCudaTensor* scales,
                                        const BeaconCudaTensor* biases, int32_t group_size,
                                        int32_t bits, BeaconCudaTensor** out);
int32_t beacon_cuda_op_rms_norm(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                const BeaconCudaTensor* x, const BeaconCudaTensor* weight,
                                float eps, BeaconCudaTensor** out);
/* Interleaved-pair RoPE of the CPU backend (ops.rs:124-142, cpu_backend.rs:141-180);
 * freqs (custom frequencies) may be NULL. */
int32_t beacon_cuda_op_rope(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                            const BeaconCudaTensor* x, int32_t position_offset, float theta,
                            int32_t dim, const BeaconCudaTensor* freqs, BeaconCudaTensor** out);
int32_t beacon_cuda_op_silu(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                            const BeaconCudaTensor* x, BeaconCudaTensor** out);
int32_t beacon_cuda_op_softmax(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                               const BeaconCudaTensor* x, int32_t axis, BeaconCudaTensor** out);
/* q [B, H, Sq, D], k/v [B, Hkv, Skv, D]; mask (additive, NULL = none).
 * `causal`: -1 = as the MLX shim (causal when mask is NULL and Sq > 1,
 * shim/src/ops.cpp:216-223), 0 = never (cpu_backend.rs:511-598), 1 = always. */
int32_t beacon_cuda_op_attention(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                 const BeaconCudaTensor* q, const BeaconCudaTensor* k,
                                 const BeaconCudaTensor* v, const BeaconCudaTensor* mask,
                                 float scale, int32_t causal, BeaconCudaTensor** out);
int32_t beacon_cuda_op_add(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                           const BeaconCudaTensor* a, const BeaconCudaTensor* b,
                           BeaconCudaTensor** out);
int32_t beacon_cuda_op_elementwise_mul(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                       const BeaconCudaTensor* a, const BeaconCudaTensor* b,
                                       BeaconCudaTensor** out);
/* backend.rs:152-160 / beacon_shim.h:155-160. Writes new_k/new_v [S, Hkv, D]
 * into the caches [max_ctx, Hkv, D] at `position` IN PLACE (the MLX
 * semantics, shim/src/ops.cpp:318-324) and returns views of rows
 * [0, position + S). */
int32_t beacon_cuda_op_kv_cache_update(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                       BeaconCudaTensor* cache_k, BeaconCudaTensor* cache_v,
                                       const BeaconCudaTensor* new_k,
                                       const BeaconCudaTensor* new_v, int64_t position,
                                       BeaconCudaTensor** out_k_view,
                                       BeaconCudaTensor** out_v_view);
int32_t beacon_cuda_op_reshape(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                               const BeaconCudaTensor* x, const int64_t* new_shape,
                               size_t new_ndim, BeaconCudaTensor** out);
int32_t beacon_cuda_op_transpose(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                 const BeaconCudaTensor* x, BeaconCudaTensor** out);
int32_t beacon_cuda_op_swapaxes(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                const BeaconCudaTensor* x, int32_t axis1, int32_t axis2,
                                BeaconCudaTensor** out);
/* weight [vocab, hidden] (F16/F32), indices I32 or F32 (cpu_backend.rs:387-418). */
int32_t beacon_cuda_op_embedding(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                 const BeaconCudaTensor* weight, const BeaconCudaTensor* indices,
                                 BeaconCudaTensor** out);
/* backend.rs:166: token ids -> I32 tensor [n]. */
int32_t beacon_cuda_create_token_tensor(BeaconCudaContext* ctx, const uint32_t* tokens,
                                        size_t n, BeaconCudaTensor** out);
/* Greedy argmax per row of the last dim with the reference's rule: last index
 * among equal maxima, NaN compares equal (sampling.rs:60-66). out: I32 [rows]. */
int32_t beacon_cuda_op_argmax(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                              const BeaconCudaTensor* logits, BeaconCudaTensor** out);
/* Measurement of quantized_matmul's decode path (rows 1..16): times `iters`
 * rounds of the op's own plan, kernels and scratch over the weights
 * w[0..n_w) in turn (same block type and shape; distinct copies whose total
 * exceeds L2 make every launch read its weights from HBM), with CUDA events
 * on `stream`. out_avg_us: mean duration of one launch; out_bytes:
 * algorithmic bytes of one launch (weight blocks + activations + f32 out).
 * No reference counterpart: the reference's kernel benches
 * (crates/beacon-kernels/benches/kernels.rs:88-108) time q4_matmul_f32. */
int32_t beacon_cuda_profile_quantized_matmul(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                             const BeaconCudaTensor* const* w, int32_t n_w,
                                             const BeaconCudaTensor* x, int32_t iters, float* out_avg_us,
                                             uint64_t* out_bytes);
/* The sampling fields of GenerationParams (crates/beacon-scheduler/src/
 * params.rs:6-31); has_top_k / has_top_p / has_min_p stand for Some(.) of the
 * Option fields (Some(0) top_k and Some(p) with p >= 1 keep their reference
 * meaning). */
typedef struct {
    float temperature;     /* <= f32::EPSILON: greedy argmax after the penalty */
    int32_t has_top_k, top_k;
    int32_t has_top_p;
    float top_p;
    int32_t has_min_p;
    float min_p;
    float repeat_penalty;  /* 1.0: none */
} BeaconCudaSamplingParams;
/* sampling::sample (crates/beacon-scheduler/src/sampling.rs:15-57) per row
 * of logits [rows, V] F32: repeat penalty over previous_tokens (I32
 * [rows, n], NULL = none), temperature, top-k, top-p, min-p, softmax and the
 * multinomial draw with uniforms[row] (F32 [rows], values in [0, 1)) in place
 * of the reference's rng.random::<f32>(). out: I32 [rows]. The logits are
 * not modified. Cumulative sums run in parallel (exact fixed-point sums of
 * the f32 probabilities), so a draw within rounding of a cumulative boundary
 * may land on the neighbouring token; everything else matches the reference. */
int32_t beacon_cuda_op_sample(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                              const BeaconCudaTensor* logits, const BeaconCudaTensor* previous_tokens,
                              const BeaconCudaSamplingParams* params, const BeaconCudaTensor* uniforms,
                              BeaconCudaTensor** out);
/* dequantize_to_f16 (dequant.rs:33-60), bit-exact: out F16 [N, K]. */
int32_t beacon_cuda_op_dequantize_to_f16(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                         const BeaconCudaTensor* w, BeaconCudaTensor** out);
/* f32 [N, K] -> GGUF blocks (Q4_0, Q8_0, Q4_K), returned as a quantized tensor.
 * The same deterministic quantizer as the test fixtures; no reference
 * counterpart (the reference has no GGUF quantizer). */
int32_t beacon_cuda_op_quantize(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                const BeaconCudaTensor* x, int32_t dtype, int32_t nibble_order,
                                BeaconCudaTensor** out);
/* Allocation-free quantized matvec; it has no counterpart in the reference.
 * d_y[b, n] = sum_k dequant(w)[n, k] * d_x[b, k] for b < batch (1..16), with
 * d_x a contiguous [batch, K] device array (x_dtype F32 or F16) and d_y a
 * contiguous f32 [batch, N] device array, same numerics as quantized_matmul.
 * For callers that may not allocate device memory (a fixed arena that owns
 * all HBM, work overlapping another thread's graph capture, latency-critical
 * loops): it calls no cudaMalloc/cudaFree. Its split-K scratch is one 2 MiB
 * array in the library image, held by every GPU that loads the library until
 * exit. Every call shares it and leaves its contents behind (the arrival
 * counters are cleared on each call), so calls that overlap on the GPU race:
 * order them. The first call on a device looks the array up with that device
 * current; make it outside stream capture. Shapes whose split partial sums do
 * not fit (batch x rows x K-splits > 520,192) return SHAPE_MISMATCH. */
int32_t beacon_cuda_quantized_matvec_noalloc(BeaconCudaStream* stream, const BeaconCudaTensor* w,
                                             const void* d_x, int32_t x_dtype, int32_t batch,
                                             float* d_y);

/* Device-to-device form of the quantizer: d_x f32 [n_rows, k] -> GGUF block
 * bytes at d_out (n_rows * k / block_size * block_bytes bytes), enqueued on
 * `stream`. No reference counterpart (fixture/synthetic-weight generation). */
int32_t beacon_cuda_quantize_blocks(BeaconCudaContext* ctx, BeaconCudaStream* stream, const float* d_x,
                                    int64_t n_rows, int64_t k, int32_t dtype, int32_t nibble_order,
                                    void* d_out);

/* === Fused decoder runtime (Engine<B>::forward, engine.rs:190-456) === */
typedef struct {
    int32_t vocab_size, hidden_size, num_layers, num_heads, num_kv_heads, head_dim;
    int32_t intermediate_size, max_context, max_batch;
    float rope_theta, rms_norm_eps;
    int32_t numerics;      /* BeaconCudaNumerics */
    int32_t kv_dtype;      /* BEACON_CUDA_DTYPE_F16 or _F32 */
    int32_t kv_persist;    /* 0 reproduces cpu_backend.rs:459-460 (cache never written back) */
    int32_t causal_prefill;/* 0 reproduces engine.rs:418 (mask None) */
    int32_t tp_size, tp_rank;
} BeaconCudaModelConfig;

/* Weight slots (also used by the oracle). */
typedef enum {
    BEACON_CUDA_W_EMBED = 0, BEACON_CUDA_W_FINAL_NORM = 1, BEACON_CUDA_W_LM_HEAD = 2,
    BEACON_CUDA_W_ATTN_NORM = 10, BEACON_CUDA_W_Q = 11, BEACON_CUDA_W_K = 12,
    BEACON_CUDA_W_V = 13, BEACON_CUDA_W_O = 14, BEACON_CUDA_W_FFN_NORM = 15,
    BEACON_CUDA_W_GATE = 16, BEACON_CUDA_W_UP = 17, BEACON_CUDA_W_DOWN = 18
} BeaconCudaWeightSlot;

int32_t beacon_cuda_model_create(BeaconCudaContext* ctx, const BeaconCudaModelConfig* cfg,
                                 BeaconCudaModel** out_model);
void    beacon_cuda_model_destroy(BeaconCudaModel* model);
/* Full (unsharded) tensor bytes: GGUF blocks for linears, F16/F32 for norms
 * and embeddings. `on_device` != 0: `data` is a device pointer. Under tensor
 * parallelism each rank keeps only its shard. */
int32_t beacon_cuda_model_set_weight(BeaconCudaModel* model, int32_t layer, int32_t slot,
                                     const void* data, int32_t dtype, int32_t nibble_order,
                                     int32_t on_device);
/* Engine::reset_cache (engine.rs:176-180). */
int32_t beacon_cuda_model_reset(BeaconCudaModel* model);
/* Engine::forward (engine.rs:190-241) for one sequence: tokens (host) ->
 * logits [n_tokens, vocab] F32 written to host `logits_out`. NULL: no logits
 * are returned, and only the last prompt row goes through the final norm and
 * lm_head (its greedy token is computed; time to first token). Under tensor
 * parallelism every rank passes logits_out, or NULL, alike: the two forms
 * run different collectives. */
int32_t beacon_cuda_model_forward(BeaconCudaModel* model, BeaconCudaStream* stream,
                                  const uint32_t* tokens, int32_t n_tokens, int32_t position,
                                  float* logits_out);
/* One greedy decode step for `batch` independent sequences at the same
 * position: tokens [batch] (host) -> next tokens [batch] (host), and logits
 * [batch, vocab] to host when logits_out != NULL. Engine::generate_next_token
 * (engine.rs:249-264) for batch == 1. */
int32_t beacon_cuda_model_decode_step(BeaconCudaModel* model, BeaconCudaStream* stream,
                                      const uint32_t* tokens, int32_t batch, int32_t position,
                                      uint32_t* next_tokens, float* logits_out);
/* One decode step whose next tokens are sampled on the device with `params`
 * (beacon_cuda_op_sample): the host sends tokens [batch], uniforms [batch]
 * (the draws, in [0, 1)) and previous [batch][n_prev] generated tokens for
 * the repeat penalty (NULL / 0 = none) and receives next_tokens [batch]; the
 * logits stay on the device. The CLI's generation loop
 * (crates/beacon-cli/src/main.rs:306-333) without its per-step logits copy. */
int32_t beacon_cuda_model_decode_step_sampled(BeaconCudaModel* model, BeaconCudaStream* stream,
                                              const uint32_t* tokens, int32_t batch, int32_t position,
                                              const BeaconCudaSamplingParams* params, const float* uniforms,
                                              const uint32_t* previous, int32_t n_prev,
                                              uint32_t* next_tokens);
/* Same step with device buffers (int32 tokens in, int32 next tokens out,
 * logits F32 [batch, vocab] or NULL); enqueued only, nothing is copied.
 * Device-side errors of enqueued steps (context overflow, bounded waits that
 * ran out) are reported by the next model_synchronize / decode_step / forward. */
int32_t beacon_cuda_model_decode_step_device(BeaconCudaModel* model, BeaconCudaStream* stream,
                                             const int32_t* d_tokens, int32_t batch,
                                             int32_t position, int32_t* d_next_tokens,
                                             float* d_logits);
/* Waits for the model's work on `stream` and reports its device-side errors:
 * CONTEXT_OVERFLOW, SHAPE_MISMATCH (token id out of range) or DEVICE_TIMEOUT.
 * (Engine::generate_next_token's error paths, engine.rs:249-264.) */
int32_t beacon_cuda_model_synchronize(BeaconCudaModel* model, BeaconCudaStream* stream);
/* Times `iters` passes of one projection over every layer, using the model's
 * own kernels and buffers (each layer's weight is distinct, so reads are
 * L2-cold), with CUDA events on `stream`. slot: BEACON_CUDA_W_Q (the fused
 * q/k/v projection), _O, _GATE (the fused gate/up projection with SwiGLU),
 * _DOWN or _LM_HEAD. batch: rows, up to the model's row capacity; more than
 * 16 rows in the fast numerics run the prefill tensor-core GEMM. Where the
 * decode step hands quantised activations from kernel to kernel (fast
 * numerics, f16 cache, one GPU), _O, _GATE and _DOWN run exactly as there:
 * they read their input image (left by the decode steps run before) and
 * write the next projection's, with the residual add for _O and _DOWN.
 * out_avg_us: mean duration of one launch; out_bytes: algorithmic bytes of
 * one launch (weight blocks + f32 activations in + f32 out). */
int32_t beacon_cuda_model_profile_linear(BeaconCudaModel* model, BeaconCudaStream* stream, int32_t slot,
                                         int32_t batch, int32_t iters, float* out_avg_us,
                                         uint64_t* out_bytes);
/* Fills KV-cache rows [0, n_rows) of every layer and sequence with seeded
 * pseudo-random values (|v| < 1), standing in for a long prefilled context
 * when only the decode step is measured: the step's work does not depend on
 * the cached values. */
int32_t beacon_cuda_model_fill_kv_random(BeaconCudaModel* model, int32_t n_rows, uint64_t seed);
/* Kernel launches in one captured decode step (after it has run once). */
int32_t beacon_cuda_model_launches_per_step(BeaconCudaModel* model, int32_t batch, int32_t continuing,
                                            int32_t* out_launches);
/* The cudaStream_t behind a stream handle (as void*). */
int32_t beacon_cuda_stream_handle(BeaconCudaStream* stream, void** out_cuda_stream);
/* Bytes of device memory held by the model (weights + KV cache + workspace). */
int32_t beacon_cuda_model_memory(const BeaconCudaModel* model, uint64_t* out_bytes);

/* === GGUF v3 files (crates/beacon-format/src/gguf) === */
typedef struct BeaconCudaGguf BeaconCudaGguf;
/* GgufFile::open (gguf/mod.rs:39-68): memory-maps the file and parses the
 * header (header.rs:17-47), the metadata key-value pairs (metadata.rs:133-151)
 * and the tensor infos, dims reversed to row-major (tensor_info.rs:13-77);
 * data offsets are resolved against general.alignment (default 32). A bad
 * magic or an unknown value type is INVALID_ARGUMENT, a version other than 3
 * or an unknown tensor type UNSUPPORTED_DTYPE, a truncated file
 * SHAPE_MISMATCH. Needs no GPU. */
int32_t beacon_cuda_gguf_open(const char* path, BeaconCudaGguf** out);
void    beacon_cuda_gguf_close(BeaconCudaGguf* f);
int32_t beacon_cuda_gguf_version(const BeaconCudaGguf* f, uint32_t* out);
int32_t beacon_cuda_gguf_tensor_count(const BeaconCudaGguf* f, int64_t* out);
/* Tensor `index`: name (valid while the file is open), BeaconDtype tag (-1
 * for GGUF types without one), row-major shape, bytes in the mapping
 * (GgufFile::tensor_data, mod.rs:79-84) and their length. */
int32_t beacon_cuda_gguf_tensor_info(const BeaconCudaGguf* f, int64_t index, const char** out_name,
                                     int32_t* out_dtype, int64_t* out_shape, size_t* inout_ndim,
                                     const void** out_data, uint64_t* out_nbytes);
int32_t beacon_cuda_gguf_find_tensor(const BeaconCudaGguf* f, const char* name, int64_t* out_index);
/* Metadata values by key (integers of every width and bools; f32/f64;
 * strings; array lengths). */
int32_t beacon_cuda_gguf_get_int(const BeaconCudaGguf* f, const char* key, int64_t* out);
int32_t beacon_cuda_gguf_get_float(const BeaconCudaGguf* f, const char* key, double* out);
int32_t beacon_cuda_gguf_get_string(const BeaconCudaGguf* f, const char* key, const char** out);
int32_t beacon_cuda_gguf_get_array_len(const BeaconCudaGguf* f, const char* key, uint64_t* out);
/* GgufFile::model_config (config_map.rs:14-100): fills the architecture
 * fields of `cfg` from {arch}.embedding_length, block_count,
 * attention.head_count(_kv), attention.key_length, feed_forward_length,
 * vocab_size (or the tokenizer.ggml.tokens length), rope.freq_base and
 * attention.layer_norm_rms_epsilon; max_context from context_length only
 * when cfg->max_context is 0. Other fields are left as they are. */
int32_t beacon_cuda_gguf_model_config(const BeaconCudaGguf* f, BeaconCudaModelConfig* cfg);
/* Engine weight loading from a GGUF file (crates/beacon-core/src/weights.rs:
 * 116-166 name mapping): token_embd (quantized embeddings are dequantised to
 * f16 on the device), output_norm, output (or the tied token_embd),
 * blk.N.{attn_norm, attn_q, attn_k, attn_v, attn_output, ffn_norm, ffn_gate,
 * ffn_up, ffn_down}. Q4_0 bytes are read in the GGUF split nibble order. A
 * missing tensor is INVALID_ARGUMENT (EngineError::WeightNotFound), a shape
 * that disagrees with the model SHAPE_MISMATCH, bias tensors
 * UNSUPPORTED_DTYPE. */
int32_t beacon_cuda_model_load_gguf(BeaconCudaModel* model, const BeaconCudaGguf* f);

/* === Tensor parallelism (NCCL over NVLink) === */
/* 128-byte ncclUniqueId, made on rank 0 and shared by the caller. */
int32_t beacon_cuda_comm_unique_id(void* out_id_128);
int32_t beacon_cuda_comm_init(BeaconCudaContext* ctx, int32_t nranks, int32_t rank,
                              const void* id_128, int32_t timeout_ms);
int32_t beacon_cuda_op_all_reduce_f32(BeaconCudaContext* ctx, BeaconCudaStream* stream,
                                      BeaconCudaTensor* t);

/* === Error introspection (beacon_shim.h:222-227) === */
const char* beacon_cuda_last_error_message(void);

#ifdef __cplusplus
}
#endif

#endif /* BEACON_CUDA_H */
