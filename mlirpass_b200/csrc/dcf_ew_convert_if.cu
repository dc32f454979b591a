// dcf_ew_convert_if.cu — int -> float (sitofp / uitofp) conversion kernels.
#include "dcf_convert_ops.cuh"

namespace dcf {

int launch_convert_if(const EwLaunch& a) {
  switch (a.op) {
    case DCF_SITOFP:
    case DCF_UITOFP: {
      const bool sg = a.op == DCF_SITOFP;
      return with_int(a.dtype, [&](auto i) {
        return with_float(a.out_dtype, [&](auto d) {
          using D = decltype(d);
          constexpr int W = decltype(i)::w;
          return sg ? launch_one<CvtIF<W, true, D>>(a) : launch_one<CvtIF<W, false, D>>(a);
        });
      });
    }
    default:
      return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
