// IIR scan instantiations for state counts: 8 10
#include "iir_launch.cuh"

namespace pesq {
namespace iir {
PESQ_IIR_INSTANTIATE(8)
PESQ_IIR_INSTANTIATE(10)
}  // namespace iir
}  // namespace pesq

#ifdef PESQ_PHASE_PROBE
// probe builds only: the stamps of this unit's kernels (8 and 10 states)
extern "C" int g_iir_probe_read_kb(unsigned long long* host) {
  return (int)cudaMemcpyFromSymbol(host, pesq::iir::g_iir_probe, sizeof(unsigned long long) * 1024 * 8);
}
#endif
