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
//
// For the rate pairs whose tables fit (all the usual ones), both directions
// run staged kernels: a few CTAs per row, each with the filter bank (the
// gather lists) staged once and the input (gradient) window of each block of
// 1024 outputs (inputs) staged before it, in shared memory.
#include <string.h>

#include <algorithm>
#include <vector>

#include "kernels.cuh"

namespace pesq {

namespace {

constexpr int kResampleThreads = 256;
// outputs (forward) / inputs (adjoint) per step of the staged kernels
constexpr int kResampleBlock = 1024;
// shared memory a staged CTA may use
constexpr size_t kResampleSmemLimit = 96 * 1024;
// CTAs the staged kernels aim for (several waves), split over the rows
constexpr int kResampleTargetCtas = 16 * 148;

// q / d for 0 <= q < 2^32 / d from inv = ceil(2^32 / d) (d >= 2), or q for d = 1
__device__ __forceinline__ uint32_t div_small(uint32_t q, uint32_t d, uint32_t inv) {
  return d == 1u ? q : __umulhi(q, inv);
}
inline uint32_t div_inverse(int d) { return d <= 1 ? 0u : (uint32_t)((((uint64_t)1 << 32) + (uint64_t)d - 1) / (uint64_t)d); }

// staged geometry shared by host and device
__host__ __device__ inline int fwd_span(int os, int ns, int wt) { return ((kResampleBlock - 1) / ns + 1) * os + wt; }
__host__ __device__ inline int tap_pitch(int max_count) { return max_count | 1; }
__host__ __device__ inline int adj_span(int os, int ns, int max_dl) {
  return ((kResampleBlock - 1) / os + 2 + max_dl) * ns;
}
size_t fwd_smem(int os, int ns, int wt, int max_count) {
  return ((size_t)ns * tap_pitch(max_count) + fwd_span(os, ns, wt) + 2 * (size_t)ns) * 4;
}
size_t adj_smem(int os, int ns, int max_dl, int max_e) {
  return ((size_t)adj_span(os, ns, max_dl) + 2 * (size_t)max_e * os) * 4;
}
// staged CTAs per row and the (block multiple) share of the row each handles
void staged_split(int rows, int64_t n, int& ctas, int64_t& chunk) {
  const int64_t blocks = ceil_div(n, (int64_t)kResampleBlock);
  const int64_t want = std::max<int64_t>(1, ceil_div((int64_t)kResampleTargetCtas, (int64_t)std::max(rows, 1)));
  const int64_t k = std::min(blocks, want);
  chunk = ceil_div(blocks, k) * kResampleBlock;
  ctas = (int)ceil_div(n, chunk);
}

// one output per thread, taps and input read from global memory (any ratio)
__global__ void __launch_bounds__(kResampleThreads) resample_fwd_kernel(const __grid_constant__ ResampleArgs p) {
  const int r = p.row_begin + (int)blockIdx.y;
  const int64_t m = (int64_t)blockIdx.x * kResampleThreads + threadIdx.x;
  if (m >= p.n_out) return;
  const int64_t l = m / p.new_step;
  const int j = (int)(m - l * p.new_step);
  const int cnt = p.count[j];
  const float* taps = p.taps + (int64_t)j * p.max_count;
  const int64_t s0 = l * p.orig_step + p.first[j] - p.width;
  // accumulated in double and returned as a float hi/lo pair: the resampled
  // signal feeds the double precision pre-emphasis and spectrum of the front
  // kernel, and near-silent bands make the loss gradient sensitive to its
  // rounding
  double acc = 0.0;
  if (p.src.type == kInF32) {
    const float* x = p.src.row(r);
    if (s0 >= 0 && s0 + cnt <= p.n_in) {
      for (int i = 0; i < cnt; ++i) acc = fma((double)taps[i], (double)__ldg(x + s0 + i), acc);
    } else {
      for (int i = 0; i < cnt; ++i) {
        const int64_t s = s0 + i;
        const float v = (s >= 0 && s < p.n_in) ? __ldg(x + s) : 0.0f;
        acc = fma((double)taps[i], (double)v, acc);
      }
    }
  } else {
    const void* x = p.src.row_any(r);
    for (int i = 0; i < cnt; ++i) {
      const int64_t s = s0 + i;
      const float v = (s >= 0 && s < p.n_in) ? load_elem(x, s, p.src.type) : 0.0f;
      acc = fma((double)taps[i], (double)v, acc);
    }
  }
  const float hi = (float)acc;
  p.dst.row(r)[m] = hi;
  if (p.dst_lo.ref) p.dst_lo.row(r)[m] = (float)(acc - (double)hi);
}

// A CTA handles `chunk` consecutive outputs of a row in steps of
// kResampleBlock: the filter bank (odd row pitch: the phases of consecutive
// lanes hit distinct banks) is staged once, the input window of every step
// before it.
__global__ void __launch_bounds__(kResampleThreads)
    resample_fwd_staged_kernel(const __grid_constant__ ResampleArgs p, int64_t chunk) {
  extern __shared__ __align__(16) float rsm[];
  const int os = p.orig_step, ns = p.new_step, tpitch = p.tpitch;
  float* tp = rsm;                                               // [ns][tpitch]
  float* xs = tp + (size_t)ns * tpitch;                          // input window
  int* fi = reinterpret_cast<int*>(xs + fwd_span(os, ns, p.width_total));  // first [ns]
  int* co = fi + ns;                                             // count [ns]
  const int tid = threadIdx.x;
  const int r = p.row_begin + (int)blockIdx.y;

  for (int i = tid; i < ns * tpitch; i += kResampleThreads) {
    const int j = i / tpitch, k = i - j * tpitch;
    tp[i] = k < p.max_count ? __ldg(p.taps + j * p.max_count + k) : 0.0f;
  }
  for (int i = tid; i < ns; i += kResampleThreads) {
    fi[i] = __ldg(p.first + i);
    co[i] = __ldg(p.count + i);
  }
  const void* x = p.src.row_any(r);  // the caller's rows (any element type)
  const int xtype = p.src.type;
  float* y = p.dst.row(r);
  const int64_t c0 = (int64_t)blockIdx.x * chunk;
  const int64_t c1 = min(c0 + chunk, p.n_out);
  for (int64_t m0 = c0; m0 < c1; m0 += kResampleBlock) {
    const int64_t m_end = min(m0 + kResampleBlock, c1);
    const int64_t l_first = m0 / ns;
    const int64_t base = l_first * os - p.width;  // input index of xs[0]
    const int span = (int)(((m_end - 1) / ns - l_first) * os + p.width_total);
    __syncthreads();  // the previous step is done with xs
    if (xtype == kInF32) {
      const float* xf = static_cast<const float*>(x);
      for (int i = tid; i < span; i += kResampleThreads) {
        const int64_t g = base + i;
        xs[i] = (g >= 0 && g < p.n_in) ? __ldg(xf + g) : 0.0f;
      }
    } else {
      for (int i = tid; i < span; i += kResampleThreads) {
        const int64_t g = base + i;
        xs[i] = (g >= 0 && g < p.n_in) ? load_elem(x, g, xtype) : 0.0f;
      }
    }
    __syncthreads();
    const int j0 = (int)(m0 - l_first * ns);  // phase of m0
    for (int64_t m = m0 + tid; m < m_end; m += kResampleThreads) {
      // frame and phase of m relative to the step (32-bit, no 64-bit division)
      const uint32_t tq = (uint32_t)(j0 + (m - m0));
      const int dl = (int)div_small(tq, (uint32_t)ns, p.inv_ns);
      const int j = (int)tq - dl * ns;
      const float* t = tp + j * tpitch;
      const float* xv = xs + dl * os + fi[j];
      const int cnt = co[j];
      // two partial sums halve the dependent chain of the tap loop
      double acc0 = 0.0, acc1 = 0.0;
      int i = 0;
#pragma unroll 4
      for (; i + 1 < cnt; i += 2) {
        acc0 = fma((double)t[i], (double)xv[i], acc0);
        acc1 = fma((double)t[i + 1], (double)xv[i + 1], acc1);
      }
      if (i < cnt) acc0 = fma((double)t[i], (double)xv[i], acc0);
      const double acc = acc0 + acc1;
      const float hi = (float)acc;
      y[m] = hi;
      if (p.dst_lo.ref) p.dst_lo.row(r)[m] = (float)(acc - (double)hi);
    }
  }
}

// one input sample per thread, per-residue gather lists from global memory
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

// A CTA handles `chunk` consecutive input samples of a row in steps of
// kResampleBlock: the residue-major gather lists are staged once (consecutive
// samples have consecutive residues), the gradient window of every step
// before it.
__global__ void __launch_bounds__(kResampleThreads)
    resample_adj_staged_kernel(const __grid_constant__ ResampleArgs p, int64_t chunk) {
  extern __shared__ __align__(16) float rsm[];
  const int os = p.orig_step, ns = p.new_step, ne = p.max_entries;
  // entry e of residue rho: (window offset j - dl * ns, tap); unused entries
  // have tap 0 and offset 0, so every lane runs the same ne iterations
  int2* ent = reinterpret_cast<int2*>(rsm);
  float* gs = reinterpret_cast<float*>(ent + (size_t)ne * os);  // gradient window
  const int tid = threadIdx.x;
  const int r = p.row_begin + (int)blockIdx.y;
  for (int i = tid; i < ne * os; i += kResampleThreads) {
    const int cd = __ldg(p.adj_code + i);
    ent[i] = cd < 0 ? make_int2(0, 0)
                    : make_int2((cd & 0xffffff) - (cd >> 24) * ns, __float_as_int(__ldg(p.adj_tap + i)));
  }
  const float* g = p.src.row(r);
  float* out = p.dst.row(r);
  const int64_t c0 = (int64_t)blockIdx.x * chunk;
  const int64_t c1 = min(c0 + chunk, p.n_in);
  for (int64_t n0 = c0; n0 < c1; n0 += kResampleBlock) {
    const int64_t n_end = min(n0 + kResampleBlock, c1);
    const int64_t l0_first = (n0 + p.width) / os;
    const int64_t mbase = (l0_first - p.max_dl) * ns;  // gradient index of gs[0]
    const int span = (int)(((n_end - 1 + p.width) / os - l0_first + 1 + p.max_dl) * ns);
    __syncthreads();  // the previous step is done with gs
    for (int i = tid; i < span; i += kResampleThreads) {
      const int64_t m = mbase + i;
      gs[i] = (m >= 0 && m < p.n_out) ? __ldg(g + m) : 0.0f;
    }
    __syncthreads();
    const int r0 = (int)(n0 + p.width - l0_first * os);  // residue of n0
    for (int64_t n = n0 + tid; n < n_end; n += kResampleThreads) {
      // frame and residue of n relative to the step (32-bit, no 64-bit division)
      const uint32_t tq = (uint32_t)(r0 + (n - n0));
      const int dl0 = (int)div_small(tq, (uint32_t)os, p.inv_os);
      const int rho = (int)tq - dl0 * os;
      // slot of (l0, phase 0) in the window; entry (dl, j) reads slot + j - dl * ns
      const int slot = (dl0 + p.max_dl) * ns;
      float acc = 0.0f;
      const int2* en = ent + rho;
      const float* gw = gs + slot;
#pragma unroll 4
      for (int e = 0; e < ne; ++e) {
        const int2 v = en[e * os];
        acc = fmaf(__int_as_float(v.y), gw[v.x], acc);
      }
      out[n] = acc;
    }
  }
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
    if (a.fwd_staged) {
      int ctas;
      int64_t chunk;
      staged_split(a.rows, a.n_out, ctas, chunk);
      dim3 grid((unsigned)ctas, (unsigned)c.rows);
      const size_t smem = fwd_smem(a.orig_step, a.new_step, a.width_total, a.max_count);
      resample_fwd_staged_kernel<<<grid, kResampleThreads, smem, s>>>(c, chunk);
    } else {
      dim3 grid((unsigned)ceil_div(a.n_out, kResampleThreads), (unsigned)c.rows);
      resample_fwd_kernel<<<grid, kResampleThreads, 0, s>>>(c);
    }
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
    if (a.adj_staged) {
      int ctas;
      int64_t chunk;
      staged_split(a.rows, a.n_in, ctas, chunk);
      dim3 grid((unsigned)ctas, (unsigned)c.rows);
      const size_t smem = adj_smem(a.orig_step, a.new_step, a.max_dl, a.max_entries);
      resample_adj_staged_kernel<<<grid, kResampleThreads, smem, s>>>(c, chunk);
    } else {
      dim3 grid((unsigned)ceil_div(a.n_in, kResampleThreads), (unsigned)c.rows);
      resample_adj_kernel<<<grid, kResampleThreads, 0, s>>>(c);
    }
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t configure_resample() {
  cudaError_t e = cudaFuncSetAttribute(resample_fwd_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kResampleSmemLimit);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(resample_adj_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kResampleSmemLimit);
}

int64_t resample_length(int orig_step, int new_step, int64_t n) {
  const float q = (float)((double)new_step * (double)n / (double)orig_step);
  return (int64_t)ceilf(q);
}

const char* build_resample_tables(int os, int ns, int width, int wt, const double* d_taps, ResampleTables& t) {
  if (os <= 0 || ns <= 0 || wt <= 0 || width < 0 || !d_taps) return "invalid resampler description";
  if (configure_resample() != cudaSuccess) return "configuring the resampler kernels failed";
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
  // residue-major copy of the lists for the staged adjoint
  int max_e = 0, max_dl = 0;
  for (int rho = 0; rho < os; ++rho) max_e = std::max(max_e, offs[rho + 1] - offs[rho]);
  for (const int4& e : ents) max_dl = std::max(max_dl, e.x);
  t.max_entries = max_e;
  t.max_dl = max_dl;
  t.width_total = wt;
  std::vector<int> code((size_t)std::max(max_e, 1) * os, -1);
  std::vector<float> ctap((size_t)std::max(max_e, 1) * os, 0.0f);
  for (int rho = 0; rho < os; ++rho)
    for (int e = offs[rho]; e < offs[rho + 1]; ++e) {
      const int slot = (e - offs[rho]) * os + rho;
      code[slot] = (ents[e].x << 24) | ents[e].y;
      memcpy(&ctap[slot], &ents[e].z, 4);
    }
  t.fwd_staged = fwd_smem(os, ns, wt, maxc) <= kResampleSmemLimit;
  t.adj_staged = max_dl < 128 && ns < (1 << 24) && adj_smem(os, ns, max_dl, max_e) <= kResampleSmemLimit;
  if (ents.empty()) ents.push_back(make_int4(0, 0, 0, 0));
  bool ok = cudaMalloc(&t.taps, taps.size() * 4) == cudaSuccess && cudaMalloc(&t.first, ns * 4) == cudaSuccess &&
            cudaMalloc(&t.count, ns * 4) == cudaSuccess && cudaMalloc(&t.adj_offset, (os + 1) * 4) == cudaSuccess &&
            cudaMalloc(&t.adj_entries, ents.size() * sizeof(int4)) == cudaSuccess &&
            cudaMalloc(&t.adj_code, code.size() * 4) == cudaSuccess &&
            cudaMalloc(&t.adj_tap, ctap.size() * 4) == cudaSuccess;
  ok = ok && cudaMemcpy(t.taps, taps.data(), taps.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.first, first.data(), ns * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.count, count.data(), ns * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.adj_offset, offs.data(), (os + 1) * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.adj_entries, ents.data(), ents.size() * sizeof(int4), cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.adj_code, code.data(), code.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
       cudaMemcpy(t.adj_tap, ctap.data(), ctap.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
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
  cudaFree(t.adj_code);
  cudaFree(t.adj_tap);
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
  ra.width_total = t.width_total;
  ra.adj_code = t.adj_code;
  ra.adj_tap = t.adj_tap;
  ra.max_entries = t.max_entries;
  ra.max_dl = t.max_dl;
  ra.fwd_staged = t.fwd_staged;
  ra.adj_staged = t.adj_staged;
  ra.tpitch = tap_pitch(t.max_count);
  ra.inv_os = div_inverse(t.orig_step);
  ra.inv_ns = div_inverse(t.new_step);
  return ra;
}

}  // namespace pesq
