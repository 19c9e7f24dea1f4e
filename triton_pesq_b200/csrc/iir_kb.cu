// IIR scan instantiations for state counts: 8 10
#include "iir_launch.cuh"

namespace pesq {
namespace iir {
PESQ_IIR_INSTANTIATE(8)
PESQ_IIR_INSTANTIATE(10)
}  // namespace iir
}  // namespace pesq
