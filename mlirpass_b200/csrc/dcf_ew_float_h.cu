// dcf_ew_float_h.cu — float fold kernels instantiated for f16 and bf16.
#include "dcf_float_ops.cuh"

namespace dcf {

int float_binary_f16(const EwLaunch& a) { return float_binary_for<F16L>(a); }
int reciprocal_f16(const EwLaunch& a) { return reciprocal_for<F16L>(a); }
int float_binary_bf16(const EwLaunch& a) { return float_binary_for<BF16L>(a); }
int reciprocal_bf16(const EwLaunch& a) { return reciprocal_for<BF16L>(a); }

}  // namespace dcf
