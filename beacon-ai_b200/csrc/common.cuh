// common.cuh -- device helpers shared by the kernels of libbeacon_cuda.so.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bc {

constexpr int kWarp = 32;

__device__ __forceinline__ float bits_f32(uint32_t b) { return __uint_as_float(b); }
__device__ __forceinline__ uint32_t f32_bits(float f) { return __float_as_uint(f); }

// Half -> single exactly as dequant.rs:80-109 does it (payload-preserving for
// NaN, exact for subnormals). Written with integer operations so that NaN
// payloads survive, which the hardware conversion does not promise.
__host__ __device__ __forceinline__ uint32_t f16_to_f32_bits(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exponent = (h >> 10) & 0x1Fu;
    uint32_t mantissa = h & 0x3FFu;
    if (exponent == 0) {
        if (mantissa == 0) return sign;
        // normalise: shift the leading one into bit 10
#ifdef __CUDA_ARCH__
        int lz = __clz((int)mantissa) - 21;  // zeros above bit 10 in an 11-bit field
#else
        int lz = __builtin_clz(mantissa) - 21;
#endif
        uint32_t m = (mantissa << lz) & 0x3FFu;
        int32_t e = -14 - lz;
        return sign | ((uint32_t)(e + 127) << 23) | (m << 13);
    }
    if (exponent == 31) return sign | 0x7F800000u | (mantissa << 13);
    return sign | ((exponent + 112) << 23) | (mantissa << 13);
}

__device__ __forceinline__ float f16_to_f32(uint16_t h) {
    // For finite inputs (every scale in practice) the hardware conversion is
    // exact; keep the integer path so NaN payloads match the reference.
    return bits_f32(f16_to_f32_bits(h));
}

// Single -> half with truncation, dequant.rs:116-152 restated on integers:
// flush below 2^-24 to zero, overflow to Inf, NaN keeps (payload >> 13) >= 1.
__device__ __forceinline__ uint16_t f32_to_f16_rtz(float v) {
    uint32_t bits = f32_bits(v);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    int32_t exponent = (int32_t)((bits >> 23) & 0xFFu);
    uint32_t mantissa = bits & 0x007FFFFFu;
    if (exponent == 255) {
        if (mantissa == 0) return sign | 0x7C00u;
        uint32_t m = mantissa >> 13;
        return sign | 0x7C00u | (uint16_t)(m < 1u ? 1u : m);
    }
    int32_t new_exp = exponent - 112;
    if (new_exp >= 31) return sign | 0x7C00u;
    if (new_exp <= 0) {
        if (new_exp < -10) return sign;
        return sign | (uint16_t)((mantissa | 0x00800000u) >> (14 - new_exp));
    }
    return sign | (uint16_t)((uint32_t)new_exp << 10) | (uint16_t)(mantissa >> 13);
}

// The reference's arithmetic runs on x86 SSE (or AArch64 with the same
// propagation for one NaN operand): a NaN operand comes out quieted, an
// invalid operation (0*Inf, Inf-Inf) yields the default NaN 0xFFC00000. GPU
// arithmetic returns a canonical NaN instead, so the bit-exact dequant kernel
// fixes the result up after each operation.
__device__ __forceinline__ float x86_nan(float r, float a, float b) {
    if (!isnan(r)) return r;
    if (isnan(a)) return bits_f32(f32_bits(a) | 0x00400000u);
    if (isnan(b)) return bits_f32(f32_bits(b) | 0x00400000u);
    return bits_f32(0xFFC00000u);
}
__device__ __forceinline__ float x86_mul(float a, float b) { return x86_nan(__fmul_rn(a, b), a, b); }
__device__ __forceinline__ float x86_sub(float a, float b) { return x86_nan(__fsub_rn(a, b), a, b); }

// dp2a: d = c + a.h0 * b.byte(0|2) + a.h1 * b.byte(1|3); `a` holds two signed
// 16-bit values, `b` four 8-bit values (unsigned or signed).
__device__ __forceinline__ int dp2a_lo_u8(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_u8(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_lo_s8(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp2a_hi_s8(int a, uint32_t b, int c) {
    int d;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Programmatic dependent launch. A kernel launched with programmatic stream
// serialisation may start while the previous kernel in the stream is still
// running; before pdl_wait() it may only touch data no earlier kernel writes
// (weights, its own shared memory). pdl_trigger() lets the next kernel launch.
// Both are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 128-bit read-only load that does not allocate in L1 (weights are streamed once).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Shared-memory barriers and 1-D bulk copies (cp.async.bulk). Every wait is
// bounded. Two kinds:
//  * mbar_wait_bounded: a wait the kernel's progress depends on (a tile copy,
//    another warp's arrival). It gives up after g_wait_limit SM clock cycles
//    (default 2^31, about 1.1 s at 1965 MHz), a per-device runtime value
//    (beacon_cuda_context_set_wait_limit); the caller records an error and
//    winds down.
//  * mbar_drain: a wait for work this CTA itself already issued (copies into
//    its shared memory, MMAs into its tensor memory) before the CTA may exit
//    or release that memory. That work always completes, so the drain keeps
//    the fixed long limit even when the runtime limit is shortened.
constexpr long long kBoundedWaitLimit = 1LL << 31;

// One copy per translation unit (internal linkage); every copy registers a
// setter at load time so the runtime can update all of them for a device.
static __device__ long long g_wait_limit = kBoundedWaitLimit;
void register_wait_limit_setter(cudaError_t (*setter)(long long));
namespace {
cudaError_t set_wait_limit_here(long long cycles) {
    return cudaMemcpyToSymbol(g_wait_limit, &cycles, sizeof(cycles));
}
struct WaitLimitRegistration {
    WaitLimitRegistration() { register_wait_limit_setter(&set_wait_limit_here); }
};
const WaitLimitRegistration g_wait_limit_registration;
}  // namespace

// Error codes written by kernels to an error word (0 = none).
enum DeviceErr : int {
    kErrTokenRange = 1,    // a token id outside the vocabulary
    kErrContext = 2,       // a device-advanced position ran past the KV cache
    kErrAttnWait = 3,      // decode attention: a bounded wait gave up
    kErrGemmWait = 4,      // tensor-core GEMM: a bounded pipeline wait gave up
    kErrGemvWait = 5,      // persistent GEMV: a bounded wait gave up
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Arrival counter with acquire-release semantics at GPU scope.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* ptr, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(ptr), "r"(v) : "memory");
    return old;
}

// Non-blocking test of a phase (no suspension).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on progress; false if the runtime limit was reached. At the
// default limit the wait uses try_wait, which lets the hardware suspend the
// thread; a shortened limit polls with test_wait so that the limit, not the
// hardware's suspend interval, decides when the wait gives up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    const long long limit = g_wait_limit;  // constant during a kernel
    const long long t0 = clock64();
    if (limit >= kBoundedWaitLimit) {
        while (!mbar_try_wait(bar, parity))
            if (clock64() - t0 > limit) return false;
        return true;
    }
    while (!mbar_test_wait(bar, parity))
        if (clock64() - t0 > limit) return false;
    return true;
}

// Bounded wait for this CTA's own issued work; false only after the fixed
// long limit.
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kBoundedWaitLimit) return false;
    return true;
}


}  // namespace bc
