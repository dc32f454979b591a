// dcf_ew_convert_ff.cu — float -> float (extf / truncf / convertf) conversion kernels.
#include "dcf_convert_ops.cuh"

namespace dcf {

int launch_convert_ff(const EwLaunch& a) {
  switch (a.op) {
    case DCF_EXTF:
    case DCF_TRUNCF:
      return with_float(a.dtype, [&](auto s) {
        return with_float(a.out_dtype, [&](auto d) {
          using S = decltype(s);
          using D = decltype(d);
          return launch_one<CvtFF<S, D>>(a);
        });
      });
    default:
      return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
