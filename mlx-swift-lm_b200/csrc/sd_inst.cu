// sd_inst.cu -- instantiates the kernels of one storage format. Compiled once
// per (SD_E, SD_BITS) pair by the build script: SD_E 0 = fp32, 1 = fp16,
// 2 = bf16 (dense element, or scale/bias type of the codes); SD_BITS 0/4/8.
#include "sd_decode.cuh"
#include "sd_kernels.h"

#if !defined(SD_E) || !defined(SD_BITS)
#error "SD_E and SD_BITS must be defined"
#endif

#if SD_E == 0
using ET = float;
#elif SD_E == 1
using ET = __half;
#else
using ET = __nv_bfloat16;
#endif

#define SD_NAME2(e, b) kernels_e##e##_b##b
#define SD_NAME(e, b) SD_NAME2(e, b)

namespace sd {

template <int D, int G>
static KernelSet make_set() {
  KernelSet k;
  k.decode = reinterpret_cast<const void*>(&decode_kernel<ET, SD_BITS, D, G>);
  k.append = reinterpret_cast<const void*>(&append_kernel<ET, SD_BITS, D>);
  k.summary = reinterpret_cast<const void*>(&summary_kernel<ET, SD_BITS, D>);
  k.merge = reinterpret_cast<const void*>(&merge_kernel<ET>);
  return k;
}

KernelSet SD_NAME(SD_E, SD_BITS)(int D, int G) {
  switch (D * 16 + G) {
    case 64 * 16 + 1: return make_set<64, 1>();
    case 64 * 16 + 2: return make_set<64, 2>();
    case 64 * 16 + 4: return make_set<64, 4>();
    case 64 * 16 + 8: return make_set<64, 8>();
    case 128 * 16 + 1: return make_set<128, 1>();
    case 128 * 16 + 2: return make_set<128, 2>();
    case 128 * 16 + 4: return make_set<128, 4>();
    case 128 * 16 + 8: return make_set<128, 8>();
    default: return KernelSet{nullptr, nullptr, nullptr, nullptr};
  }
}

}  // namespace sd
