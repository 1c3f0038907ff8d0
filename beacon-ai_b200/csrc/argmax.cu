// argmax.cu -- greedy argmax over logits with the reference's rule, on many CTAs.
//
// Rule (engine.rs:256-261, sampling.rs:60-66): a left-to-right scan keeps the
// current best only while v[best] > v[i], so equal maxima move to the later
// index and a NaN (which compares Equal) takes over, after which the very next
// element takes over again. Summarise a chunk of the row as
//   forced = the chunk holds a NaN: the scan leaves the chunk at
//            lastmax(v[j+1 ..]) for the chunk's last NaN j, or at j itself when
//            j ends the chunk, whatever came in;
//   else     the chunk's last maximum m replaces the incoming best b exactly
//            when !(v[b] > v[m]).
// Chunks then fold left to right in a second tiny kernel, so the result is the
// scan's result for any chunking.
#include "argmax.h"
#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace bc {
namespace {

// logits are [parts][rows][per]; global index = part * per + j
__global__ void argmax_chunks_kernel(const float* __restrict__ x, int64_t per, int parts, int rows, int chunks_per_part,
                                     ArgmaxSummary* __restrict__ out) {
    __shared__ int64_t sh_i[32];
    __shared__ float sh_v[32];
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.y;
    const int c = blockIdx.x;  // chunk over parts * chunks_per_part
    const int part = c / chunks_per_part, cc = c % chunks_per_part;
    const int64_t clen = (per + chunks_per_part - 1) / chunks_per_part;
    const int64_t j0 = (int64_t)cc * clen, j1 = min(per, j0 + clen);
    const float* v = x + ((int64_t)part * rows + row) * per;
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    int64_t last_nan = -1;
    for (int64_t j = j0 + threadIdx.x; j < j1; j += blockDim.x)
        if (isnan(v[j])) last_nan = j;
#pragma unroll
    for (int o = 16; o; o >>= 1) last_nan = max(last_nan, __shfl_xor_sync(0xffffffffu, last_nan, o));
    if (l == 0) sh_i[w] = last_nan;
    __syncthreads();
    last_nan = -1;
    for (int i = 0; i < nw; ++i) last_nan = max(last_nan, sh_i[i]);
    __syncthreads();
    const int64_t start = last_nan >= 0 ? last_nan + 1 : j0;
    float bv = -INFINITY;
    int64_t bi = -1;
    for (int64_t j = start + threadIdx.x; j < j1; j += blockDim.x) {
        const float cv = v[j];
        if (bi < 0 || cv > bv || (cv == bv && j > bi)) {
            bv = cv;
            bi = j;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi > bi))) {
            bv = ov;
            bi = oi;
        }
    }
    if (l == 0) {
        sh_v[w] = bv;
        sh_i[w] = bi;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    bv = -INFINITY;
    bi = -1;
    for (int i = 0; i < nw; ++i)
        if (sh_i[i] >= 0 && (bi < 0 || sh_v[i] > bv || (sh_v[i] == bv && sh_i[i] > bi))) {
            bv = sh_v[i];
            bi = sh_i[i];
        }
    ArgmaxSummary s;
    s.forced = last_nan >= 0 ? 1 : 0;
    if (last_nan >= 0 && bi < 0) {  // the NaN ends the chunk
        bi = last_nan;
        bv = v[last_nan];
    }
    s.valid = bi >= 0 ? 1 : 0;
    s.idx = bi >= 0 ? (int64_t)part * per + bi : -1;
    s.val = bv;
    out[(int64_t)row * parts * chunks_per_part + c] = s;
}

__global__ void argmax_fold_kernel(const ArgmaxSummary* __restrict__ sums, int nchunks, int rows,
                                   int32_t* __restrict__ out, int32_t* __restrict__ out2) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    int64_t bi = -1;
    float bv = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
        const ArgmaxSummary s = sums[(int64_t)row * nchunks + c];
        if (!s.valid) continue;
        if (s.forced || bi < 0 || !(bv > s.val)) {
            bi = s.idx;
            bv = s.val;
        }
    }
    const int32_t r = bi < 0 ? 0 : (int32_t)bi;
    out[row] = r;
    if (out2) out2[row] = r;
}

}  // namespace

int argmax_chunks_per_part(int64_t per) {
    int64_t c = (per + 2047) / 2048;
    return (int)std::max<int64_t>(1, std::min<int64_t>(c, 128));
}

void launch_argmax(const float* x, int64_t per, int parts, int rows, int32_t* out, int32_t* out2,
                   ArgmaxSummary* scratch, cudaStream_t s, bool pdl) {
    if (rows <= 0) return;
    const int cpp = argmax_chunks_per_part(per);
    dim3 grid((unsigned)(parts * cpp), (unsigned)rows);
    launch_kernel(argmax_chunks_kernel, grid, dim3(256), 0, s, pdl, x, per, parts, rows, cpp, scratch);
    launch_kernel(argmax_fold_kernel, dim3((rows + 127) / 128), dim3(128), 0, s, pdl, (const ArgmaxSummary*)scratch,
                  parts * cpp, rows, out, out2);
}

}  // namespace bc
