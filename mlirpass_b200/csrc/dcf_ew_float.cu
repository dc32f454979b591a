// dcf_ew_float.cu — dispatch of the float folds (addf, subf, mulf, divf,
// remf, the four min/max ops, dense cmpf and tosa reciprocal) by layout.
#include "dcf_float_ops.cuh"

namespace dcf {

int launch_float_binary(const EwLaunch& a) {
  switch (a.dtype) {
    case DCF_F16: return float_binary_f16(a);
    case DCF_BF16: return float_binary_bf16(a);
    case DCF_F32: return float_binary_f32(a);
    case DCF_F64: return float_binary_f64(a);
    case DCF_F8E5M2: return float_binary_f8e5m2(a);
    case DCF_F8E4M3: return float_binary_f8e4m3(a);
    case DCF_F8E3M4: return float_binary_f8e3m4(a);
    default: return DCF_EUNSUPPORTED;
  }
}

int launch_reciprocal(const EwLaunch& a) {
  switch (a.dtype) {
    case DCF_F16: return reciprocal_f16(a);
    case DCF_BF16: return reciprocal_bf16(a);
    case DCF_F32: return reciprocal_f32(a);
    case DCF_F64: return reciprocal_f64(a);
    case DCF_F8E5M2: return reciprocal_f8e5m2(a);
    case DCF_F8E4M3: return reciprocal_f8e4m3(a);
    case DCF_F8E3M4: return reciprocal_f8e3m4(a);
    default: return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
