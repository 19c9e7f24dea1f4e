// Level-alignment adjoint of the backward pass, one CTA per (gradient row,
// segment):
//
//   z = H_pow^T H_pow x      on [a, send) of one 16 kHz row
//
// The loss depends on x through the alignment scale s = sqrt(c / sum f^2),
// f = H_pow x (torch_pesq/loss.py:132-139), whose gradient is
// ds/dx = -s / sum f^2 * H_pow^T f; the back kernel scales z by the per-row
// factor kappa the chain adjoint produces.  z depends on the input only, so
// it is evaluated here, in the backward, while the chain adjoint (which
// occupies one cluster of SMs per utterance) is still running:
//
//   * this kernel is launched with programmatic stream serialisation right
//     after the chain adjoint, which releases it as soon as its own CTAs are
//     resident, so its CTAs fill the SMs the chain leaves idle;
//   * it reads nothing the chain adjoint writes, and it waits for the chain
//     adjoint's grid to complete (pdl_wait) only after its own work, so the
//     next kernel on the stream (the back kernel, launched normally) starts
//     after both.
//
// The CTA stages kSpan samples from kHorizon before the segment: the forward
// scan H_pow runs in place over them (the first kHorizon outputs are warm-up),
// then the adjoint scan runs backwards in time from kHorizon samples past the
// segment end, again in place; f past the row end is not part of the signal.
#include "kernels.cuh"

namespace pesq {

PESQ_PHASE_TABLE(g_phase_align)

namespace {

constexpr int kAlignSmemBytes = kSpan * 4 + scan_scratch_floats<10>() * 4;

__global__ void __launch_bounds__(kThreads, 1)
    align_adjoint_kernel(const __grid_constant__ AlignArgs p, const __grid_constant__ PowTab pow) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;  // kSpan: x, then f = H x, then z = H^T f, all in place
  float* scratch = xs + kSpan;

  const int tid = threadIdx.x;
  const int row = p.row_begin + blockIdx.x / p.nseg;
  const int seg = blockIdx.x % p.nseg;
  const int64_t n_row = p.n;
  const int64_t a = (int64_t)seg * p.seg_frames * kHop;
  const int64_t send = min(a + (int64_t)p.seg_frames * kHop, n_row);
  const int64_t base = a - kHorizon;
  const float* xr = p.src.row(row);
  PESQ_STAMP(g_phase_align, 0);

  // zeros outside the row reproduce the zero initial state
  stage_span(xs, xr, base, n_row);
  __syncthreads();
  PESQ_STAMP(g_phase_align, 1);

  // pass 0: f = H x over the span, in place; pass 1: z = H^T f on [a, send),
  // logical position q at physical index top - q.  One instance of the scan
  // code serves both passes, which keeps two unrolled order-10 scans from
  // competing for registers.
  const int top = 2 * kHorizon + (int)(send - a) - 1;
  for (int pass = 0; pass < 2; ++pass) {
    chunk_scan<10, false, float>(
        pow, scratch,
        [&](int q) {
          if (pass == 0) return xs[q];
          const int idx = top - q;
          return (idx >= 0 && base + idx < n_row) ? xs[idx] : 0.0f;
        },
        [&](int q, float y) {
          const int idx = pass == 0 ? q : top - q;
          if (idx >= 0) xs[idx] = y;
        });
    __syncthreads();
  }
  PESQ_STAMP(g_phase_align, 2);

  float* zr = p.z + (int64_t)row * n_row;
  for (int i = tid; i < (int)(send - a); i += kThreads) zr[a + i] = xs[kHorizon + i];
  PESQ_STAMP(g_phase_align, 3);

  // complete only after the kernel this one was released early from
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
