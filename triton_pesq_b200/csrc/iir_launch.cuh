// Launch of one IIR scan instantiation; included by the iir_k*.cu units, each
// of which instantiates a few state counts (they compile in parallel).
#pragma once

#include "iir.cuh"

namespace pesq {
namespace iir {

template <int P, bool kLower, bool kRerun>
cudaError_t launch(const Args& a, const void* tab, cudaStream_t s) {
  static_assert(sizeof(Tab<P>) == sizeof(float) * (kL + 2 * kL * P + (kLevels + 1) * P * P + 2 * P + 1),
                "Tab<P> is a packed array of floats");
  const size_t smem = smem_bytes(P);
  auto kern = a.reverse ? scan_kernel<P, kLower, kRerun, true> : scan_kernel<P, kLower, kRerun, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)a.tiles, kThreads, smem, s>>>(a, *static_cast<const Tab<P>*>(tab));
  return cudaGetLastError();
}

#define PESQ_IIR_INSTANTIATE(P)                                                            \
  template cudaError_t launch<P, false, false>(const Args&, const void*, cudaStream_t);   \
  template cudaError_t launch<P, false, true>(const Args&, const void*, cudaStream_t);    \
  template cudaError_t launch<P, true, false>(const Args&, const void*, cudaStream_t);    \
  template cudaError_t launch<P, true, true>(const Args&, const void*, cudaStream_t);

}  // namespace iir
}  // namespace pesq
