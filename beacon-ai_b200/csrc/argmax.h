// argmax.h -- greedy argmax with the reference's tie and NaN rule (argmax.cu).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

namespace bc {

struct ArgmaxSummary {
    int64_t idx;  // global index of the chunk's candidate, -1 if none
    float val;
    int forced;   // the chunk holds a NaN: its candidate wins whatever came before
    int valid;
};

int argmax_chunks_per_part(int64_t per);
inline size_t argmax_scratch_count(int64_t per, int parts, int rows) {
    return (size_t)argmax_chunks_per_part(per) * parts * rows;
}
// logits [parts][rows][per] (parts = 1: plain [rows][per]); out[row] = index
// over parts*per; out2 (optional) receives a copy.
void launch_argmax(const float* x, int64_t per, int parts, int rows, int32_t* out, int32_t* out2,
                   ArgmaxSummary* scratch, cudaStream_t s, bool pdl = false);

}  // namespace bc
