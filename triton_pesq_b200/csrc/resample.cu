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
#include <string.h>

#include <algorithm>
#include <vector>

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
  if (p.dst_lo.ref) p.dst_lo.row(r)[m] = (float)(acc - (double)hi);
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

// Rows go in grid y, at most kMaxGridRows per launch.
constexpr int kMaxGridRows = 65535;

cudaError_t launch_resample_fwd(const ResampleArgs& a, cudaStream_t s) {
  if (a.rows <= 0 || a.n_out <= 0) return cudaSuccess;
  for (int r0 = 0; r0 < a.rows; r0 += kMaxGridRows) {
    ResampleArgs c = a;
    c.row_begin = a.row_begin + r0;
    c.rows = std::min(kMaxGridRows, a.rows - r0);
    dim3 grid((unsigned)ceil_div(a.n_out, kResampleThreads), (unsigned)c.rows);
    resample_fwd_kernel<<<grid, kResampleThreads, 0, s>>>(c);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_resample_adj(const ResampleArgs& a, cudaStream_t s) {
  if (a.rows <= 0 || a.n_in <= 0) return cudaSuccess;
  for (int r0 = 0; r0 < a.rows; r0 += kMaxGridRows) {
    ResampleArgs c = a;
    c.row_begin = a.row_begin + r0;
    c.rows = std::min(kMaxGridRows, a.rows - r0);
    dim3 grid((unsigned)ceil_div(a.n_in, kResampleThreads), (unsigned)c.rows);
    resample_adj_kernel<<<grid, kResampleThreads, 0, s>>>(c);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int64_t resample_length(int orig_step, int new_step, int64_t n) {
  const float q = (float)((double)new_step * (double)n / (double)orig_step);
  return (int64_t)ceilf(q);
}

const char* build_resample_tables(int os, int ns, int width, int wt, const double* d_taps, ResampleTables& t) {
  if (os <= 0 || ns <= 0 || wt <= 0 || width < 0 || !d_taps) return "invalid resampler description";
  t.orig_step = os;
  t.new_step = ns;
  t.width = width;
  // compact taps: the nonzero range of every phase
  std::vector<int> first(ns), count(ns);
  int maxc = 1;
  for (int j = 0; j < ns; ++j) {
    int lo = -1, hi = -1;
    for (int k = 0; k < wt; ++k)
      if ((float)d_taps[(size_t)j * wt + k] != 0.0f) {
        if (lo < 0) lo = k;
        hi = k;
      }
    first[j] = lo < 0 ? 0 : lo;
    count[j] = lo < 0 ? 0 : hi + 1 - lo;
    maxc = std::max(maxc, count[j]);
  }
  std::vector<float> taps((size_t)ns * maxc, 0.0f);
  for (int j = 0; j < ns; ++j)
    for (int i = 0; i < count[j]; ++i) taps[(size_t)j * maxc + i] = (float)d_taps[(size_t)j * wt + first[j] + i];
  t.max_count = maxc;
  // adjoint: per residue rho = k mod orig_step the (k / orig_step, phase, tap) triples
  std::vector<int> offs(os + 1, 0);
  std::vector<int4> ents;
  for (int rho = 0; rho < os; ++rho) {
    offs[rho] = (int)ents.size();
    for (int k = rho; k < wt; k += os)
      for (int j = 0; j < ns; ++j) {
        const float v = (float)d_taps[(size_t)j * wt + k];
        if (v != 0.0f) {
          int bits;
          memcpy(&bits, &v, 4);
          ents.push_back(make_int4((k - rho) / os, j, bits, 0));
        }
      }
  }
  offs[os] = (int)ents.size();
  if (ents.empty()) ents.push_back(make_int4(0, 0, 0, 0));
  bool ok = cudaMalloc(&t.taps, taps.size() * 4) == cudaSuccess && cudaMalloc(&t.first, ns * 4) == cudaSuccess &&
            cudaMalloc(&t.count, ns * 4) == cudaSuccess && cudaMalloc(&t.adj_offset, (os + 1) * 4) == cudaSuccess &&
            cudaMalloc(&t.adj_entries, ents.size() * sizeof(int4)) == cudaSuccess;
  ok = ok && cudaMemcpy(t.taps, taps.data(), taps.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.first, first.data(), ns * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.count, count.data(), ns * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.adj_offset, offs.data(), (os + 1) * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.adj_entries, ents.data(), ents.size() * sizeof(int4), cudaMemcpyHostToDevice) == cudaSuccess;
  if (!ok) {
    free_resample_tables(t);
    return "upload of the resampler tables failed";
  }
  return nullptr;
}

void free_resample_tables(ResampleTables& t) {
  cudaFree(t.taps);
  cudaFree(t.first);
  cudaFree(t.count);
  cudaFree(t.adj_offset);
  cudaFree(t.adj_entries);
  t = ResampleTables{};
}

ResampleArgs resample_args(const ResampleTables& t, int64_t n_in, int64_t n_out) {
  ResampleArgs ra{};
  ra.n_in = n_in;
  ra.n_out = n_out;
  ra.orig_step = t.orig_step;
  ra.new_step = t.new_step;
  ra.width = t.width;
  ra.taps = t.taps;
  ra.first = t.first;
  ra.count = t.count;
  ra.max_count = t.max_count;
  ra.adj_offset = t.adj_offset;
  ra.adj_entries = t.adj_entries;
  return ra;
}

}  // namespace pesq
