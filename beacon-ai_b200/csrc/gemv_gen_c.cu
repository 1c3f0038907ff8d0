// gemv_gen_c.cu -- instantiates the tiled dequant-GEMV for generic block
// formats (split across units so nvcc compiles them in parallel).
#include "gemv.cuh"

namespace bc {
void launch_qgemv_q5_k(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q5_K>(a); }
void launch_qgemv_q6_k(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q6_K>(a); }
void launch_qgemv_q8_k(const GemvLaunch& a) { launch_qgemv_fmt<FMT_Q8_K>(a); }
}  // namespace bc
