// Level-alignment adjoint of the backward pass, one CTA per (gradient row,
// segment):
//
//   z = H_pow^T f            on [a, send) of one 16 kHz row, f = H_pow x
//
// The loss depends on x through the alignment scale s = sqrt(c / sum f^2)
// (torch_pesq/loss.py:132-139), whose gradient is
// ds/dx = -s / sum f^2 * H_pow^T f; the back kernel scales z by the per-row
// factor kappa the chain adjoint produces.  f was saved by the front kernel,
// so z depends on nothing the backward computes and is evaluated while the
// chain adjoint (which occupies one cluster of SMs per utterance) is still
// running:
//
//   * this kernel is launched with programmatic stream serialisation right
//     after the chain adjoint, which releases it as soon as its own CTAs are
//     resident, so its CTAs fill the SMs the chain leaves idle;
//   * it reads nothing the chain adjoint writes, and it waits for the chain
//     adjoint's grid to complete (pdl_wait) only after its own work, so its
//     completion implies the chain adjoint's; the back kernel that follows
//     (launched the same way, released at the end of this kernel's CTAs)
//     waits for this kernel's completion before reading.
//
// The adjoint filter runs backwards in time: the CTA stages f on
// [a, send + kHorizon) (zero past the row end, where f is not part of the
// signal) and scans it from the far end, the first kHorizon outputs being the
// warm-up.
#include "kernels.cuh"

namespace pesq {

PESQ_PHASE_TABLE(g_phase_align)
PESQ_SPAN_TABLE(g_span_align)
PESQ_CTA_TABLE(g_cta_align)

namespace {

constexpr int kAlignSmemBytes = kSpan * 4 + scan_scratch_floats<10>() * 4;

__global__ void __launch_bounds__(kThreads, 2)
    align_adjoint_kernel(const __grid_constant__ AlignArgs p, const __grid_constant__ PowTab pow) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;  // kSpan: f, then z = H^T f in place
  float* scratch = xs + kSpan;

  const int tid = threadIdx.x;
  const int row = p.row_begin + blockIdx.x / p.nseg;
  const int seg = blockIdx.x % p.nseg;
  const int64_t n_row = p.n;
  const int64_t a = (int64_t)seg * p.seg_frames * kHop;
  const int64_t send = min(a + (int64_t)p.seg_frames * kHop, n_row);
  const int64_t base = a - kHorizon;
  PESQ_SPAN_BEGIN(g_span_align, 0);
  PESQ_CTA_BEGIN(g_cta_align);
  PESQ_STAMP(g_phase_align, 0);

  // f on [a, send + kHorizon) at physical indices kHorizon.., zeros elsewhere
  const int64_t f_end = min(send + kHorizon, n_row);
  const float* fr = p.fpow + (int64_t)row * n_row;
  {
    constexpr int kPer = kSpan / kThreads;
    float v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int64_t g = base + tid + k * kThreads;
      v[k] = (g >= a && g < f_end) ? __ldg(fr + g) : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) xs[tid + k * kThreads] = v[k];
  }
  __syncthreads();
  PESQ_STAMP(g_phase_align, 1);

  // z = H^T f on [a, send): logical position q at physical index top - q
  const int top = 2 * kHorizon + (int)(send - a) - 1;
  chunk_scan<10, false, float, true, kThreads, true>(
      pow, scratch,
      [&](int q) {
        const int idx = top - q;
        return idx >= 0 ? xs[idx] : 0.0f;
      },
      [&](int q, float y) {
        const int idx = top - q;
        if (idx >= 0) xs[idx] = y;
      });
  __syncthreads();
  PESQ_STAMP(g_phase_align, 2);

  float* zr = p.z + (int64_t)row * n_row;
  for (int i = tid; i < (int)(send - a); i += kThreads) zr[a + i] = xs[kHorizon + i];
  PESQ_STAMP(g_phase_align, 3);
  PESQ_CTA_END(g_cta_align);
  PESQ_SPAN_END(g_span_align, 0);

  // the back kernel may be scheduled once every CTA is here; this kernel
  // completes only after the kernel it was released early from
  pdl_trigger();
  pdl_wait();
}

}  // namespace

size_t align_smem_bytes() { return (size_t)kAlignSmemBytes; }

cudaError_t configure_align() {
  return cudaFuncSetAttribute(align_adjoint_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)align_smem_bytes());
}

cudaError_t launch_align(const AlignArgs& a, const PowTab& pow, int rows, cudaStream_t s) {
  const int64_t blocks = (int64_t)rows * a.nseg;
  if (blocks <= 0) return cudaSuccess;
  LaunchShape l((unsigned)blocks, kThreads, align_smem_bytes(), s, true);
  return cudaLaunchKernelEx(&l.cfg, align_adjoint_kernel, a, pow);
}

}  // namespace pesq
