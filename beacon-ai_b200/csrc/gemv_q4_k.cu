// gemv_q4_k.cu -- instantiates the dequant-GEMV kernels for one block format
// (split per format so nvcc compiles them in parallel).
#include "gemv3.cuh"

namespace bc {
void launch_qgemv_q4_k(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q4_K>(a); }
void launch_qgemv3_q4_k(const LinearPlan& pl, const GemvLaunch& a) { launch_qgemv3_fmt<FMT_Q4_K>(pl, a); }
}  // namespace bc
