// qx.cuh -- writing a consumer GEMV's quantised-activation image (QxImage)
// from the kernel that produces the activations.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace bc {

// Quantise one 32-element block of a producer's output (one value per lane,
// element g*32 + lane of batch row b) into the consumer's staging image: codes of
// x * norm_w with the scale absmax / 32767 (the consumer's own rule), their
// sum, and the sum of squares of x for the consumer's RMSNorm. All 32 lanes
// take part; `valid` = the row exists (zero otherwise).
// has_nw: the caller loaded this lane's norm weight ahead (nw), else it is read here.
__device__ __forceinline__ void qx_write_group(const QxImage& q, int b, int64_t g, int lane, float x, bool valid,
                                               bool has_nw = false, float nw = 0.0f) {
    const int64_t row = g * 32 + lane;
    const float xv = valid ? x : 0.0f;
    const float yv = (valid && q.norm_w) ? xv * (has_nw ? nw : q.norm_w[row]) : xv;
    float am = fabsf(yv);
#pragma unroll
    for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const float qi = am > 0.0f ? 32767.0f * __frcp_rn(am) : 0.0f;
    const int code = max(-32767, min(32767, __float2int_rn(__fmul_rn(yv, qi))));
    int sum = code;
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    float ss = xv * xv;
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int nblk = q.kspan / 32;
    const int e = lane & 7;
    const int pos = q.perm ? ((lane & ~7) | ((e & 1) ? 4 + (e >> 1) : (e >> 1))) : lane;
    reinterpret_cast<int16_t*>(q.data)[(int64_t)b * q.kspan + g * 32 + pos] = (int16_t)code;
    if (lane == 0) {
        float2* sxq = reinterpret_cast<float2*>(q.data + (size_t)q.bpad * q.kspan * 2);  // (scale, code sum)
        sxq[b * nblk + g] = make_float2(am * (1.0f / 32767.0f), (float)sum);
        if (q.ss) q.ss[b * nblk + g] = ss;
    }
}

}  // namespace bc
