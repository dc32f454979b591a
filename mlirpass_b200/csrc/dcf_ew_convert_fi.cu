// dcf_ew_convert_fi.cu — float -> int (fptosi / fptoui) conversion kernels.
#include "dcf_convert_ops.cuh"

namespace dcf {

int launch_convert_fi(const EwLaunch& a) {
  switch (a.op) {
    case DCF_FPTOSI:
    case DCF_FPTOUI: {
      const bool sg = a.op == DCF_FPTOSI;
      return with_float(a.dtype, [&](auto s) {
        return with_int(a.out_dtype, [&](auto i) {
          using S = decltype(s);
          constexpr int W = decltype(i)::w;
          return sg ? launch_one<CvtFI<S, W, true>>(a) : launch_one<CvtFI<S, W, false>>(a);
        });
      });
    }
    default:
      return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
