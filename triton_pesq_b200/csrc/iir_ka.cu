// IIR scan instantiations for state counts: 2 4 6
#include "iir_launch.cuh"

namespace pesq {
namespace iir {
PESQ_IIR_INSTANTIATE(2)
PESQ_IIR_INSTANTIATE(4)
PESQ_IIR_INSTANTIATE(6)
}  // namespace iir
}  // namespace pesq
