// gemv_q4_0.cu -- instantiates the dequant-GEMV kernels for one block format
// (split per format so nvcc compiles them in parallel).
#include "gemv3.cuh"

namespace bc {
void launch_qgemv_q4_0(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q4_0>(a); }
void launch_qgemv3_q4_0(const LinearPlan& pl, const GemvLaunch& a) { launch_qgemv3_fmt<FMT_Q4_0>(pl, a); }
}  // namespace bc
