// qgemm_tc.h -- prefill dequant-GEMM on tcgen05 tensor cores (qgemm_tc.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "internal.h"
#include "kernels.h"

namespace bc {

bool qgemm_tc_supported(const QLayout& L);
// Bytes of f16 activation scratch a launch with f32 (or unaligned) x needs.
size_t qgemm_tc_scratch_bytes(int64_t rows, int64_t k);
// Bytes of f16 weight scratch for the dequantise-first form (n_pad x k_pad).
size_t qgemm_tc_weight_scratch_bytes(const QLayout& L);
// y[rows, N] (epilogue epi) = x[rows, K] W^T for a tiled quantized W; x f32 or
// f16 with row stride x_ld (f32 x is first converted to f16 in x16_scratch).
// rtz: weights rounded toward zero to f16 (the CPU engine's weights) instead
// of to nearest. w16_scratch (qgemm_tc_weight_scratch_bytes, or NULL): W is
// first dequantised into it as f16 rows (same values) and the GEMM loads both
// operands by TMA instead of dequantising in its producer warps -- the form
// for many rows, where the dequantisation would otherwise be repeated by
// every row tile. w16_ready: w16_scratch already holds this W's f16 rows (the
// dequantisation is skipped). *err = 4 if a bounded wait gave up.
void launch_qgemm_tc(const QLayout& L, const void* w, const void* x, bool x_f16, int64_t x_ld, int64_t rows, float* y,
                     int64_t y_ld, int epi, const float* res, int64_t res_ld, bool rtz, int* err, cudaStream_t s,
                     void* x16_scratch, const QkvEpi* qkv = nullptr, void* w16_scratch = nullptr,
                     bool w16_ready = false);

}  // namespace bc
