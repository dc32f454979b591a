// dcf_ew_convert.cu — dispatch of the conversion folds, and the kernels of
// negf, flush_denormals and extsi / extui / trunci.
#include "dcf_convert_ops.cuh"

namespace dcf {

int launch_convert(const EwLaunch& a) {
  switch (a.op) {
    case DCF_EXTF:
    case DCF_TRUNCF:
      return launch_convert_ff(a);
    case DCF_SITOFP:
    case DCF_UITOFP:
      return launch_convert_if(a);
    case DCF_FPTOSI:
    case DCF_FPTOUI:
      return launch_convert_fi(a);
    case DCF_NEGF:
    case DCF_FLUSH_DENORMALS: {
      if (a.dtype != a.out_dtype) return DCF_EUNSUPPORTED;
      const bool neg = a.op == DCF_NEGF;
      return with_float(a.dtype, [&](auto s) {
        using S = decltype(s);
        return neg ? launch_one<FSign<S, true>>(a) : launch_one<FSign<S, false>>(a);
      });
    }
    case DCF_EXTSI:
    case DCF_EXTUI:
    case DCF_TRUNCI: {
      const bool sg = a.op == DCF_EXTSI;
      return with_int(a.dtype, [&](auto i) {
        return with_int(a.out_dtype, [&](auto o) {
          constexpr int WI = decltype(i)::w, WO = decltype(o)::w;
          return sg ? launch_one<CvtII<WI, WO, true>>(a) : launch_one<CvtII<WI, WO, false>>(a);
        });
      });
    }
    default:
      return launch_math_unary(a);
  }
}

}  // namespace dcf
