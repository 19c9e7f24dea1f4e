// IIR scan instantiations for state counts: 24
#include "iir_launch.cuh"

namespace pesq {
namespace iir {
PESQ_IIR_INSTANTIATE(24)
}  // namespace iir
}  // namespace pesq
