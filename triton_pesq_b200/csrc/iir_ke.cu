// IIR scan instantiations for state counts: 20
#include "iir_launch.cuh"

namespace pesq {
namespace iir {
PESQ_IIR_INSTANTIATE(20)
}  // namespace iir
}  // namespace pesq
