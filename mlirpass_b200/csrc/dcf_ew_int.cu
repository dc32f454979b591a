// dcf_ew_int.cu — integer binary folds (wraparound ApInt arithmetic, the
// refusing ops shli/shrui/shrsi, divsi/divui, remsi/remui) and dense cmpi.
#include "dcf_kernels.cuh"

namespace dcf {

template <int OP, int W> struct IOp {
  using In = typename IntW<W>::T;
  using Out = typename IntW<W>::T;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t, Out& o) {
    uint64_t r = 0;
    const bool ok = int_op<OP, W>(a, b, r);
    o = (Out)r;
    return ok;
  }
};

template <int W> struct ICmp {
  using In = typename IntW<W>::T;
  using Out = uint8_t;
  static constexpr bool kBinary = true;
  __device__ static __forceinline__ bool apply(In a, In b, uint32_t flags, Out& o) {
    o = cmpi<W>((int)((flags & DCF_FLAG_PRED_MASK) >> DCF_FLAG_PRED_SHIFT), a, b);
    return true;
  }
};

template <int W> static int int_binary_for(const EwLaunch& a) {
  switch (a.op) {
    case DCF_ADDI: return launch_one<IOp<DCF_ADDI, W>>(a);
    case DCF_SUBI: return launch_one<IOp<DCF_SUBI, W>>(a);
    case DCF_MULI: return launch_one<IOp<DCF_MULI, W>>(a);
    case DCF_ANDI: return launch_one<IOp<DCF_ANDI, W>>(a);
    case DCF_ORI: return launch_one<IOp<DCF_ORI, W>>(a);
    case DCF_XORI: return launch_one<IOp<DCF_XORI, W>>(a);
    case DCF_SHLI: return launch_one<IOp<DCF_SHLI, W>>(a);
    case DCF_SHRUI: return launch_one<IOp<DCF_SHRUI, W>>(a);
    case DCF_SHRSI: return launch_one<IOp<DCF_SHRSI, W>>(a);
    case DCF_DIVSI: return launch_one<IOp<DCF_DIVSI, W>>(a);
    case DCF_DIVUI: return launch_one<IOp<DCF_DIVUI, W>>(a);
    case DCF_REMSI: return launch_one<IOp<DCF_REMSI, W>>(a);
    case DCF_REMUI: return launch_one<IOp<DCF_REMUI, W>>(a);
    case DCF_MAXSI: return launch_one<IOp<DCF_MAXSI, W>>(a);
    case DCF_MAXUI: return launch_one<IOp<DCF_MAXUI, W>>(a);
    case DCF_MINSI: return launch_one<IOp<DCF_MINSI, W>>(a);
    case DCF_MINUI: return launch_one<IOp<DCF_MINUI, W>>(a);
    case DCF_CMPI: return launch_one<ICmp<W>>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

int launch_int_binary(const EwLaunch& a) {
  switch (a.dtype) {
    case DCF_I1: return int_binary_for<1>(a);
    case DCF_I8: return int_binary_for<8>(a);
    case DCF_I16: return int_binary_for<16>(a);
    case DCF_I32: return int_binary_for<32>(a);
    case DCF_I64: return int_binary_for<64>(a);
    default: return DCF_EUNSUPPORTED;
  }
}

}  // namespace dcf
