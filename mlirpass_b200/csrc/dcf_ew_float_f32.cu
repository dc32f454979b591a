// dcf_ew_float_f32.cu — float fold kernels instantiated for f32.
#include "dcf_float_ops.cuh"

namespace dcf {

int float_binary_f32(const EwLaunch& a) { return float_binary_for<F32L>(a); }
int reciprocal_f32(const EwLaunch& a) { return reciprocal_for<F32L>(a); }

}  // namespace dcf
