// gemv_q8_0.cu -- instantiates the dequant-GEMV kernels for one block format
// (split per format so nvcc compiles them in parallel).
#include "gemv3.cuh"

namespace bc {
void launch_qgemv_q8_0(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q8_0>(a); }
void launch_qgemv3_q8_0(const LinearPlan& pl, const GemvLaunch& a) { launch_qgemv3_fmt<FMT_Q8_0>(pl, a); }
}  // namespace bc
