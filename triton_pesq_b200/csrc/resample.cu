// Polyphase sinc resampler to 16 kHz and its adjoint.
//
// Output m = l * new_step + j of a row is (accumulated in double)
//   y[m] = sum_k taps[j][k] x[l * orig_step + k - width]     (x = 0 outside)
// which is torchaudio's strided conv1d over the (width, width + orig_step)
// padded input (torch_pesq/loss.py:76, Resample(sample_rate, 16000)).  Only
// the nonzero taps of each phase are stored (their float32 values round to
// exactly zero elsewhere), e.g. 33-34 of 475 at 44.1 kHz.
//
// The adjoint is a gather over input samples: with n + width = l * orig + k,
// every tap that reaches sample n has k = n + width (mod orig_step), so the
// host lists, per residue, the (frame offset, phase, tap) triples that
// contribute.  No atomics; the result is bitwise reproducible.
#include "kernels.cuh"

namespace pesq {

namespace {

constexpr int kResampleThreads = 256;

__global__ void __launch_bounds__(kResampleThreads) resample_fwd_kernel(const __grid_constant__ ResampleArgs p) {
  const int r = p.row_begin + (int)blockIdx.y;
  const int64_t m = (int64_t)blockIdx.x * kResampleThreads + threadIdx.x;
  if (m >= p.n_out) return;
  const int64_t l = m / p.new_step;
  const int j = (int)(m - l * p.new_step);
  const int cnt = p.count[j];
  const float* taps = p.taps + (int64_t)j * p.max_count;
  const float* x = p.src.row(r);
  const int64_t s0 = l * p.orig_step + p.first[j] - p.width;
  // accumulated in double and returned as a float hi/lo pair: the resampled
  // signal feeds the double precision pre-emphasis and spectrum of the front
  // kernel, and near-silent bands make the loss gradient sensitive to its
  // rounding
  double acc = 0.0;
  if (s0 >= 0 && s0 + cnt <= p.n_in) {
    for (int i = 0; i < cnt; ++i) acc = fma((double)taps[i], (double)__ldg(x + s0 + i), acc);
  } else {
    for (int i = 0; i < cnt; ++i) {
      const int64_t s = s0 + i;
      const float v = (s >= 0 && s < p.n_in) ? __ldg(x + s) : 0.0f;
      acc = fma((double)taps[i], (double)v, acc);
    }
  }
  const float hi = (float)acc;
  p.dst.row(r)[m] = hi;
  p.dst_lo.row(r)[m] = (float)(acc - (double)hi);
}

__global__ void __launch_bounds__(kResampleThreads) resample_adj_kernel(const __grid_constant__ ResampleArgs p) {
  const int r = p.row_begin + (int)blockIdx.y;
  const int64_t n = (int64_t)blockIdx.x * kResampleThreads + threadIdx.x;
  if (n >= p.n_in) return;
  const int64_t pos = n + p.width;
  const int64_t l0 = pos / p.orig_step;
  const int rho = (int)(pos - l0 * p.orig_step);
  const float* g = p.src.row(r);
  float acc = 0.0f;
  for (int e = p.adj_offset[rho]; e < p.adj_offset[rho + 1]; ++e) {
    const int4 ent = p.adj_entries[e];
    const int64_t l = l0 - ent.x;
    if (l < 0) continue;
    const int64_t m = l * p.new_step + ent.y;
    if (m < p.n_out) acc = fmaf(__int_as_float(ent.z), __ldg(g + m), acc);
  }
  p.dst.row(r)[n] = acc;
}

}  // namespace

cudaError_t launch_resample_fwd(const ResampleArgs& a, cudaStream_t s) {
  if (a.rows <= 0 || a.n_out <= 0) return cudaSuccess;
  dim3 grid((unsigned)ceil_div(a.n_out, kResampleThreads), (unsigned)a.rows);
  resample_fwd_kernel<<<grid, kResampleThreads, 0, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_resample_adj(const ResampleArgs& a, cudaStream_t s) {
  if (a.rows <= 0 || a.n_in <= 0) return cudaSuccess;
  dim3 grid((unsigned)ceil_div(a.n_in, kResampleThreads), (unsigned)a.rows);
  resample_adj_kernel<<<grid, kResampleThreads, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace pesq
