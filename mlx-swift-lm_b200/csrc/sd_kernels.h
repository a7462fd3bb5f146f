// sd_kernels.h -- table of kernel entry points, one instantiation unit per
// storage format (element type x code bits). Host-side only.
#pragma once

namespace sd {

struct KernelSet {
  const void* decode;   // decode_kernel<E, BITS, D, G>(DecodeParams, CUtensorMap x3)
  const void* append;   // append_kernel<E, BITS, D>(AppendParams)
  const void* summary;  // summary_kernel<E, BITS, D>(SummaryParams)
  const void* merge;    // merge_kernel<E>(int, int, int, const float*, const float*, E*, const float*, int)
};

// e: 0 = fp32, 1 = fp16, 2 = bf16; b: code bits (0 = dense). Null members
// when (D, G) has no instantiation.
KernelSet kernels_e0_b0(int D, int G);
KernelSet kernels_e1_b0(int D, int G);
KernelSet kernels_e2_b0(int D, int G);
KernelSet kernels_e0_b4(int D, int G);
KernelSet kernels_e1_b4(int D, int G);
KernelSet kernels_e2_b4(int D, int G);
KernelSet kernels_e0_b8(int D, int G);
KernelSet kernels_e1_b8(int D, int G);
KernelSet kernels_e2_b8(int D, int G);

}  // namespace sd
