// attention.h -- argument blocks of the attention kernels (attention.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace bc {

// Strided exact attention, one CTA per query row. Element offsets:
// q/out: b*sb + h*sh + s*ss; k/v: b*kv_sb + kvh*kv_sh + key*kv_ss.
struct AttnRowsArgs {
    const void* q;
    int q_f16;
    const void* k;
    const void* v;
    int kv_f16;
    float* out;
    const float* mask;
    int64_t mask_numel;
    int64_t batch, heads, kv_heads, sq, skv;
    int d;
    float scale;
    int causal;
    int64_t q_sb, q_sh, q_ss;
    int64_t kv_sb, kv_sh, kv_ss;
    int64_t o_sb, o_sh, o_ss;
    void* out16 = nullptr;  // tensor-core prefill kernel: also an f16 copy of out (same layout)
};
void launch_attention_rows(const AttnRowsArgs& a, cudaStream_t s);
// Tiled prefill attention (one sequence, no additive mask, f32 q): 128
// (row, head) pairs of one KV head per CTA share each staged key/value tile.
bool prefill_attention_supported(const AttnRowsArgs& a);
// True when the f16 copy (a.out16) was written too (the tensor-core kernel ran).
bool launch_prefill_attention(const AttnRowsArgs& a, cudaStream_t s);

// Split-K decode attention over KV caches laid out [batch][max_ctx][kv_heads][d].
// q: f32 [batch][heads][d]; out: f32 [batch][heads][d]. Scratch: part_acc
// [batch*heads*nsplit*d], part_m / part_l [batch*heads*nsplit].
struct DecodeAttnArgs {
    const float* q;
    const void* k_cache;
    const void* v_cache;
    int kv_f16;
    int64_t cache_sb;  // elements between sequences
    int batch, heads, kv_heads, d;
    int kv_len;        // keys [0, kv_len) are attended ...
    const int* pos_ptr;  // ... or, when set, keys [0, *pos_ptr + 1) (graph replay)
    int max_kv;          // cache rows; kv_len is clamped to it
    float scale;
    int nsplit;
    float* part_acc;
    float* part_m;
    float* part_l;
    float* out;
    int* counters;  // [batch * kv_heads] arrival counters, zero at rest (f16 caches)
    int* err;       // set to 3 when a bounded wait gives up (f16 caches)
    QxImage qy;     // f16 caches: also write the output quantised for the o projection
    int tc = 0;     // f16 caches, fast numerics: the tensor-core kernel
};
constexpr int kMaxDecodeSplits = 64;
constexpr int kMaxBulkSplits = 256;
int plan_decode_splits(int batch, int kv_heads, int kv_len, int sm_count, int max_splits);
// f16 caches: one CTA per (sequence, KV head, split), splits = SMs / (batch *
// kv_heads) (at least 1), so partials need heads/kv_heads * max(SMs, batch *
// kv_heads) * (d + 2) floats and the counters batch * kv_heads ints.
int decode_bulk_splits(int batch, int kv_heads, int sm_count);
size_t decode_bulk_scratch_floats(int max_batch, int heads, int kv_heads, int d, int sm_count);
bool decode_attention_supported(int head_dim, int group);
void launch_decode_attention(DecodeAttnArgs a, cudaStream_t s, bool pdl = false);

}  // namespace bc
