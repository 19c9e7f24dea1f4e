// IIR scan instantiations for state counts: 12 14
#include "iir_launch.cuh"

namespace pesq {
namespace iir {
PESQ_IIR_INSTANTIATE(12)
PESQ_IIR_INSTANTIATE(14)
}  // namespace iir
}  // namespace pesq
