// dcf_ew_float_f64.cu — float fold kernels instantiated for f64.
#include "dcf_float_ops.cuh"

namespace dcf {

int float_binary_f64(const EwLaunch& a) { return float_binary_for<F64L>(a); }
int reciprocal_f64(const EwLaunch& a) { return reciprocal_for<F64L>(a); }

}  // namespace dcf
