/*
 * oracle.h -- CPU restatement of the reference's quantized decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * backend: only tests, the smoke check and the CPU-baseline leg of the bench
 * may load it. The product (libbeacon_cuda.so) never links or calls it.
 *
 * Every function restates one reference function (Rust, crate paths given
 * relative to the reference project root) in plain C++ with the same
 * floating-point operation order. It is compiled with -ffp-contract=off
 * because Rust never contracts a*b+c into an FMA.
 *
 * Parity pins: the reference's own known-answer tests (dequant.rs:633-684,
 * q4.rs:96-125, beacon-kernels/src/tests.rs:52-227,
 * beacon-core/src/tests.rs:67-316, beacon-scheduler/src/tests.rs:10-28) are
 * replayed against this library by tests/test_oracle_kat.py.
 */
#ifndef BEACON_ORACLE_H
#define BEACON_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype tags: identical to BeaconDtype (crates/beacon-format/src/dtype.rs:12-29) */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2, ORC_I32 = 3, ORC_I8 = 4,
    ORC_Q4_0 = 100, ORC_Q4_K = 101, ORC_Q5_K = 102, ORC_Q6_K = 103,
    ORC_Q8_0 = 104, ORC_Q4_1 = 105, ORC_Q5_0 = 106, ORC_Q5_1 = 107,
    ORC_Q2_K = 108, ORC_Q3_K = 109, ORC_Q8_K = 110
};

/* Q4_0 nibble order. REF_INTERLEAVED is what dequant.rs:170-176 and
 * q4.rs:33-41 compute (byte i -> elements 2i, 2i+1); GGUF_SPLIT is the GGUF
 * file convention (byte i -> elements i, i+16). */
enum { ORC_NIBBLE_REF_INTERLEAVED = 0, ORC_NIBBLE_GGUF_SPLIT = 1 };

float    orc_f16_to_f32(uint16_t bits);
uint16_t orc_f32_to_f16_rtz(float v);
uint16_t orc_f32_to_f16_rne(float v);
void     orc_f32_to_f16_rtz_array(const float* in, uint16_t* out, size_t n);
void     orc_f32_to_f16_rne_array(const float* in, uint16_t* out, size_t n);

int64_t orc_block_size(int dtype);
int64_t orc_block_bytes(int dtype);

int orc_dequantize_to_f16(const uint8_t* data, int dtype, uint64_t n,
                          int nibble_order, uint16_t* out);
int orc_dequantize_to_f32(const uint8_t* data, int dtype, uint64_t n,
                          int nibble_order, int rtz, float* out);
int orc_quantize(const float* x, int dtype, uint64_t n, int nibble_order,
                 uint8_t* out);

void  orc_q4_dequantize_block(const uint8_t* block, float* out32);
float orc_q4_dot_f32(const float* x, const uint8_t* w_q4, size_t k);
void  orc_q4_matmul_f32(const uint8_t* w_q4, const float* x, float* out,
                        size_t m, size_t k);
int   orc_qgemv_f32(const uint8_t* w, int dtype, int nibble_order, int rtz,
                    int64_t n, int64_t k, const float* x, int64_t batch,
                    float* y, int threads);

void orc_matmul_f32(const float* a, const float* b, float* c,
                    size_t m, size_t k, size_t n);
void orc_transpose_f32(const float* x, float* out, size_t batch, size_t m,
                       size_t n);
void orc_rms_norm(const float* x, const float* w, float* out, size_t n,
                  float eps);
void orc_silu_inplace(float* x, size_t n);
void orc_softmax_inplace(float* x, size_t n);
void orc_rope_inplace(float* x, size_t seq_len, size_t dim,
                      size_t position_offset, float theta);
void orc_add(const float* a, const float* b, float* out, size_t n);
void orc_mul(const float* a, const float* b, float* out, size_t n);
int  orc_attention(const float* q, const float* k, const float* v,
                   const float* mask, size_t mask_numel, float scale,
                   size_t batch, size_t n_heads, size_t seq_q,
                   size_t head_dim, size_t n_kv_heads, size_t seq_kv,
                   int causal, float* out);
uint32_t orc_argmax(const float* logits, size_t n);

/* GenerationParams' sampling fields (crates/beacon-scheduler/src/params.rs:6-31);
 * the has_* flags stand for Some(.) of the Option fields. */
typedef struct {
    float temperature;
    int32_t has_top_k, top_k;
    int32_t has_top_p;
    float top_p;
    int32_t has_min_p;
    float min_p;
    float repeat_penalty;
} OrcSampleParams;
/* sampling.rs:15-57 with the draw r in [0, 1) given. */
uint32_t orc_sample(const float* logits, size_t n, const uint32_t* prev, size_t n_prev,
                    const OrcSampleParams* p, float r, float* probs_out);

/* Llama-style engine (crates/beacon-core/src/engine.rs:190-456). */
typedef struct {
    int32_t vocab_size, hidden_size, num_layers, num_heads, num_kv_heads;
    int32_t head_dim, intermediate_size, max_context;
    float rope_theta, rms_norm_eps;
    int32_t kv_persist;      /* 0 = cpu_backend.rs literal (cache never written back) */
    int32_t causal_prefill;  /* 0 = engine.rs:418 literal (mask None) */
    int32_t weights_rtz;     /* 1 = weights f16_to_f32(dequantize_to_f16(.)) as the
                                CPU engine consumes them; 0 = unrounded q*d */
    int32_t threads;
    int32_t ref_faithful;    /* 1 = every projection runs as the reference does it:
                                a fresh transposed copy of W per call
                                (cpu_backend.rs:330-366) then the column-strided
                                matmul_f32 loop (ops.rs:16-30), one thread. Same
                                sums in the same order, so the same results. */
} OrcModelConfig;

enum {
    ORC_W_EMBED = 0, ORC_W_FINAL_NORM = 1, ORC_W_LM_HEAD = 2,
    ORC_W_ATTN_NORM = 10, ORC_W_Q = 11, ORC_W_K = 12, ORC_W_V = 13,
    ORC_W_O = 14, ORC_W_FFN_NORM = 15, ORC_W_GATE = 16, ORC_W_UP = 17,
    ORC_W_DOWN = 18
};

void* orc_model_create(const OrcModelConfig* cfg);
int   orc_model_set_weight(void* model, int layer, int which, const void* data,
                           int dtype, int nibble_order);
int   orc_model_forward(void* model, const uint32_t* tokens, size_t seq_len,
                        size_t position, float* logits_out);
void  orc_model_reset(void* model);
void  orc_model_destroy(void* model);
const char* orc_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
