// dcf_ew_float_f8.cu — float fold kernels instantiated for the three f8 layouts.
#include "dcf_float_ops.cuh"

namespace dcf {

int float_binary_f8e5m2(const EwLaunch& a) { return float_binary_for<F8E5M2L>(a); }
int reciprocal_f8e5m2(const EwLaunch& a) { return reciprocal_for<F8E5M2L>(a); }
int float_binary_f8e4m3(const EwLaunch& a) { return float_binary_for<F8E4M3L>(a); }
int reciprocal_f8e4m3(const EwLaunch& a) { return reciprocal_for<F8E4M3L>(a); }
int float_binary_f8e3m4(const EwLaunch& a) { return float_binary_for<F8E3M4L>(a); }
int reciprocal_f8e3m4(const EwLaunch& a) { return reciprocal_for<F8E3M4L>(a); }

}  // namespace dcf
