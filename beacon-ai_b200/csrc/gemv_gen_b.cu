// gemv_gen_b.cu -- instantiates the tiled dequant-GEMV for generic block
// formats (split across units so nvcc compiles them in parallel).
#include "gemv.cuh"

namespace bc {
void launch_qgemv_q2_k(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q2_K>(a); }
void launch_qgemv_q3_k(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q3_K>(a); }
}  // namespace bc
