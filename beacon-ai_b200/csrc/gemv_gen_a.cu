// gemv_gen_a.cu -- instantiates the tiled dequant-GEMV for generic block
// formats (split across units so nvcc compiles them in parallel).
#include "gemv.cuh"

namespace bc {
void launch_qgemv_q4_1(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q4_1>(a); }
void launch_qgemv_q5_0(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q5_0>(a); }
void launch_qgemv_q5_1(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q5_1>(a); }
}  // namespace bc
