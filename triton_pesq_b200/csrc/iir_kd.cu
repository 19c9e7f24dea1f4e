// IIR scan instantiations for state counts: 16
#include "iir_launch.cuh"

namespace pesq {
namespace iir {
PESQ_IIR_INSTANTIATE(16)
}  // namespace iir
}  // namespace pesq
