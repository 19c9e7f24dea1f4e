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
// For the usual rate pairs (8 to 48 kHz, tap spans of up to 64 samples per
// block of 8 phases) both directions run on the float64 tensor cores
// (mma.sync m8n8k4: tcgen05 has no float64 kind): 8 x 8 output tiles of
// (super-)frames x consecutive phases (forward) or residues (adjoint), the
// staged samples widened to double once per fragment element, each widening
// feeding 8 outputs.  Other pairs whose tables fit run the staged CUDA-core
// kernels: a few CTAs per row, each with the filter bank (the gather lists)
// staged once and the input (gradient) window of each block of 1024 outputs
// (inputs) staged before it, in shared memory.
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

// D (8 x 8, two per lane) += A (8 x 4, one per lane) * B (4 x 8, one per
// lane) in float64 on the tensor cores.  Lane l holds A[l / 4][l % 4],
// B[l % 4][l / 4] and D[l / 4][2 (l % 4) + {0, 1}].
__device__ __forceinline__ void dmma_8x8x4(double& d0, double& d1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};\n"
               : "+d"(d0), "+d"(d1)
               : "d"(a), "d"(b));
}

constexpr int kMmaMaxWarps = 16;
constexpr int kMmaGroups = 4;  // 8-row groups of one tile pass (independent accumulators)

// Forward on the float64 tensor cores.  G frames form a super-frame of
// mma_ns = G * new_step outputs whose window starts at input sample
// L * mma_os - width (mma_os = G * orig_step).  A CTA stages mma_frames
// consecutive super-frame windows, one per row of pitch mma_pitch (4 mod 32:
// the 8 rows of an A fragment hit distinct banks), and its warps run the
// (block of 8 super-phases, 4 groups of 8 super-frames) units of that window:
// B = the block's taps (one k-step of 4 taps per fragment, from a table laid
// out in fragment order), A = the staged samples widened to double, each
// widening feeding 8 phases.  Each output is the same float64 sum of its
// nonzero taps in a fixed order, whatever the batch or the CTA split.
template <int KS>
__global__ void __launch_bounds__(kMmaMaxWarps * 32)
    resample_fwd_mma_kernel(const __grid_constant__ ResampleArgs p) {
  extern __shared__ __align__(16) float win[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int r = p.row_begin + (int)blockIdx.y;
  const int P = p.mma_pitch, S = p.mma_span, F = p.mma_frames;
  const int64_t frames = ceil_div(p.n_out, (int64_t)p.mma_ns);
  const int64_t L0 = (int64_t)blockIdx.x * F;
  const int nf = (int)min((int64_t)F, frames - L0);

  // stage: row f holds samples [0, S) of super-frame L0 + f's window, rows
  // P apart: padded rows (P >= S), or with P = mma_os the window itself,
  // each sample once (rows overlap), where padding would copy samples
  // several times over.  float32 rows go by asynchronous copies (every load
  // of the window in flight at once), others through registers.
  const void* x = p.src.row_any(r);
  const int xtype = p.src.type;
  const int64_t base = L0 * p.mma_os - p.width;
  const bool contiguous = P == p.mma_os;
  const int span = contiguous ? (nf - 1) * P + S : 0;
  if (xtype == kInF32) {
    const float* xf = static_cast<const float*>(x);
    if (contiguous) {
      for (int i = threadIdx.x; i < span; i += blockDim.x) {
        const int64_t g = base + i;
        const bool valid = g >= 0 && g < p.n_in;
        cp_async4_zfill(win + i, valid ? xf + g : xf, valid);
      }
    } else {
      for (int f = warp; f < nf; f += nw) {
        const int64_t g0 = base + (int64_t)f * p.mma_os;
        for (int t = lane; t < S; t += 32) {
          const int64_t g = g0 + t;
          const bool valid = g >= 0 && g < p.n_in;
          cp_async4_zfill(win + f * P + t, valid ? xf + g : xf, valid);
        }
      }
    }
    cp_async_commit();
    cp_async_wait_all();
  } else if (contiguous) {
    for (int i = threadIdx.x; i < span; i += blockDim.x) {
      const int64_t g = base + i;
      win[i] = (g >= 0 && g < p.n_in) ? load_elem(x, g, xtype) : 0.0f;
    }
  } else {
    for (int f = warp; f < nf; f += nw) {
      const int64_t g0 = base + (int64_t)f * p.mma_os;
      for (int t = lane; t < S; t += 32) {
        const int64_t g = g0 + t;
        win[f * P + t] = (g >= 0 && g < p.n_in) ? load_elem(x, g, xtype) : 0.0f;
      }
    }
  }
  __syncthreads();

  const int chunks = F / (8 * kMmaGroups);  // units per block
  const int units = p.mma_blocks * chunks;
  float* y = p.dst.row(r);
  float* ylo = p.dst_lo.ref ? p.dst_lo.row(r) : nullptr;
  for (int u = warp; u < units; u += nw) {
    const int b = u / chunks;
    const int g0 = (u - b * chunks) * kMmaGroups;  // first 8-row group
    if (g0 * 8 >= nf) continue;
    double bf[KS];
    const double* bp = p.mma_b + (size_t)b * KS * 32 + lane;
#pragma unroll
    for (int k = 0; k < KS; ++k) bf[k] = __ldg(bp + k * 32);
    // rows past nf hold stale samples: their outputs are not stored
    const float* a = win + (g0 * 8 + (lane >> 2)) * P + __ldg(p.mma_s + b) + (lane & 3);
    double acc[kMmaGroups][2];
#pragma unroll
    for (int gi = 0; gi < kMmaGroups; ++gi) acc[gi][0] = acc[gi][1] = 0.0;
#pragma unroll
    for (int k = 0; k < KS; ++k) {
#pragma unroll
      for (int gi = 0; gi < kMmaGroups; ++gi)
        dmma_8x8x4(acc[gi][0], acc[gi][1], (double)a[gi * 8 * P + 4 * k], bf[k]);
    }
#pragma unroll
    for (int gi = 0; gi < kMmaGroups; ++gi) {
      const int f = (g0 + gi) * 8 + (lane >> 2);
      if (f >= nf) continue;
      const int64_t m = (L0 + f) * p.mma_ns + 8 * b + 2 * (lane & 3);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if (m + i < p.n_out) {
          const float hi = (float)acc[gi][i];
          y[m + i] = hi;
          if (ylo) ylo[m + i] = (float)(acc[gi][i] - (double)hi);
        }
      }
    }
  }
}

// k-steps of the instantiated tensor-core kernels: even counts up to 16
// (tap spans of up to 64 samples per block of 8 super-phases)
constexpr int kMmaMaxKSteps = 16;

template <int KS>
cudaError_t launch_fwd_mma_ks(dim3 grid, int threads, size_t smem, cudaStream_t s, const ResampleArgs& c) {
  resample_fwd_mma_kernel<KS><<<grid, threads, smem, s>>>(c);
  return cudaSuccess;
}

cudaError_t launch_fwd_mma(int ks, dim3 grid, int threads, size_t smem, cudaStream_t s, const ResampleArgs& c) {
  switch (ks) {
    case 2: return launch_fwd_mma_ks<2>(grid, threads, smem, s, c);
    case 4: return launch_fwd_mma_ks<4>(grid, threads, smem, s, c);
    case 6: return launch_fwd_mma_ks<6>(grid, threads, smem, s, c);
    case 8: return launch_fwd_mma_ks<8>(grid, threads, smem, s, c);
    case 10: return launch_fwd_mma_ks<10>(grid, threads, smem, s, c);
    case 12: return launch_fwd_mma_ks<12>(grid, threads, smem, s, c);
    case 14: return launch_fwd_mma_ks<14>(grid, threads, smem, s, c);
    case 16: return launch_fwd_mma_ks<16>(grid, threads, smem, s, c);
    default: return cudaErrorInvalidValue;
  }
}

template <int KS>
cudaError_t configure_fwd_mma() {
  return cudaFuncSetAttribute(resample_fwd_mma_kernel<KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kResampleSmemLimit);
}

// Adjoint on the float64 tensor cores.  Input sample n = L * amma_os + rho -
// width (residue rho of super-frame L) gathers
//   sum over entries (dL, q) of tap(q, rho + dL * amma_os) * g[(L - dL) * amma_ns + q];
// for a block of 8 consecutive residues the entries that reach any of them
// form the K dimension of an m8n8k4 tile whose rows are 8 super-frames
// (A = the staged gradient rows at offsets -dL * pitch + q, widened to
// double; B = the taps, zero where an entry misses a residue).  A CTA stages
// amma_frames + amma_maxdl rows of the upstream gradient (column amma_ns
// holds zero: the padding entries point there) and owns the input samples of
// amma_frames super-frames: every sample is written once, a fixed float64
// sum, no atomics.
__global__ void __launch_bounds__(kMmaMaxWarps * 32)
    resample_adj_mma_kernel(const __grid_constant__ ResampleArgs p) {
  extern __shared__ __align__(16) float gw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  const int r = p.row_begin + (int)blockIdx.y;
  const int P = p.amma_pitch, F = p.amma_frames, D = p.amma_maxdl, ns2 = p.amma_ns, os2 = p.amma_os;
  const int64_t frames = ceil_div(p.n_in + p.width, (int64_t)os2);
  const int64_t L0 = (int64_t)blockIdx.x * F;
  const int nf = (int)min((int64_t)F, frames - L0);

  // stage gradient rows L0 - D .. L0 + nf - 1 (row f holds super-frame L0 - D
  // + f; column ns2 is the zero the padding entries read), by asynchronous
  // copies: every load of the window in flight at once
  const float* g = p.src.row(r);
  for (int f = warp; f < nf + D; f += nw) {
    const int64_t m0 = (L0 - D + f) * ns2;
    float* row = gw + f * P;
    for (int t = lane; t <= ns2; t += 32) {
      const int64_t m = m0 + t;
      const bool valid = t < ns2 && m >= 0 && m < p.n_out;
      cp_async4_zfill(row + t, valid ? g + m : g, valid);
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();

  const int chunks = F / (8 * kMmaGroups);
  const int units = p.amma_blocks * chunks;
  float* out = p.dst.row(r);
  for (int u = warp; u < units; u += nw) {
    const int c = u / chunks;
    const int g0 = (u - c * chunks) * kMmaGroups;
    if (g0 * 8 >= nf) continue;
    const int k0 = __ldg(p.amma_off + c), k1 = __ldg(p.amma_off + c + 1);
    // rows past nf + D - 1 hold stale values: their outputs are not stored
    const float* a = gw + (D + g0 * 8 + (lane >> 2)) * P;
    double acc[kMmaGroups][2];
#pragma unroll
    for (int gi = 0; gi < kMmaGroups; ++gi) acc[gi][0] = acc[gi][1] = 0.0;
    // (loading a few k-steps' operands ahead of their MMAs cut the load
    // stalls but cost a CTA per SM in registers: no faster)
#pragma unroll 2
    for (int k = k0; k < k1; ++k) {
      const double b = __ldg(p.amma_b + (size_t)k * 32 + lane);
      const int ao = __ldg(p.amma_a + k * 4 + (lane & 3));
#pragma unroll
      for (int gi = 0; gi < kMmaGroups; ++gi) dmma_8x8x4(acc[gi][0], acc[gi][1], (double)a[gi * 8 * P + ao], b);
    }
#pragma unroll
    for (int gi = 0; gi < kMmaGroups; ++gi) {
      const int f = (g0 + gi) * 8 + (lane >> 2);
      if (f >= nf) continue;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int rho = 8 * c + 2 * (lane & 3) + i;
        const int64_t n = (L0 + f) * os2 + rho - p.width;
        if (rho < os2 && n >= 0 && n < p.n_in) out[n] = (float)acc[gi][i];
      }
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
    if (a.fwd_mma) {
      const int64_t frames = ceil_div(a.n_out, (int64_t)a.mma_ns);
      dim3 grid((unsigned)ceil_div(frames, (int64_t)a.mma_frames), (unsigned)c.rows);
      // rows of mma_pitch floats, the last one mma_span long
      const size_t smem = ((size_t)a.mma_frames * a.mma_pitch + (size_t)std::max(0, a.mma_span - a.mma_pitch)) * 4;
      const cudaError_t e = launch_fwd_mma(a.fwd_mma, grid, a.mma_warps * 32, smem, s, c);
      if (e != cudaSuccess) return e;
    } else if (a.fwd_staged) {
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
    if (a.adj_mma) {
      const int64_t frames = ceil_div(a.n_in + a.width, (int64_t)a.amma_os);
      dim3 grid((unsigned)ceil_div(frames, (int64_t)a.amma_frames), (unsigned)c.rows);
      const size_t smem = (size_t)(a.amma_frames + a.amma_maxdl) * a.amma_pitch * 4;
      resample_adj_mma_kernel<<<grid, a.amma_warps * 32, smem, s>>>(c);
    } else if (a.adj_staged) {
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
  const cudaError_t mma[] = {configure_fwd_mma<2>(),  configure_fwd_mma<4>(),  configure_fwd_mma<6>(),
                             configure_fwd_mma<8>(),  configure_fwd_mma<10>(), configure_fwd_mma<12>(),
                             configure_fwd_mma<14>(), configure_fwd_mma<16>()};
  for (cudaError_t m : mma)
    if (m != cudaSuccess) return m;
  e = cudaFuncSetAttribute(resample_adj_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kResampleSmemLimit);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(resample_adj_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kResampleSmemLimit);
}

namespace {

// staged window of the tensor-core forward, bytes (two CTAs per SM)
constexpr size_t kMmaWindowBytes = 72 * 1024;

int gcd_int(int a, int b) {
  while (b) {
    const int r = a % b;
    a = b;
    b = r;
  }
  return a;
}

// Geometry and B table of the tensor-core forward for compact taps
// (first, count, taps [ns][maxc]); leaves t.fwd_mma = 0 where the tap spans
// of a block of 8 super-phases exceed 4 * kMmaMaxKSteps samples.
void plan_fwd_mma(int os, int ns, const std::vector<int>& first, const std::vector<int>& count,
                  const std::vector<float>& taps, int maxc, ResampleTables& t, std::vector<double>& bfrag,
                  std::vector<int>& sblock) {
  t.fwd_mma = 0;
  const int G = 8 / gcd_int(ns, 8);
  if ((int64_t)os * G > (1 << 20) || (int64_t)ns * G > (1 << 20)) return;
  const int os2 = os * G, ns2 = ns * G, nb = ns2 / 8;
  // offset (from the super-frame window's first sample) and length of each super-phase's taps
  std::vector<int> off(ns2), cnt(ns2);
  for (int q = 0; q < ns2; ++q) {
    off[q] = (q / ns) * os + first[q % ns];
    cnt[q] = count[q % ns];
  }
  sblock.assign(nb, 0);
  int K = 1, smax = 0;
  for (int b = 0; b < nb; ++b) {
    int lo = 0, hi = 0;
    bool any = false;
    for (int n = 0; n < 8; ++n) {
      const int q = 8 * b + n;
      if (cnt[q] <= 0) continue;
      lo = any ? std::min(lo, off[q]) : off[q];
      hi = any ? std::max(hi, off[q] + cnt[q]) : off[q] + cnt[q];
      any = true;
    }
    sblock[b] = lo;
    K = std::max(K, hi - lo);
    smax = std::max(smax, lo);
  }
  int ks = (K + 3) / 4;
  ks += ks & 1;
  if (ks > kMmaMaxKSteps) return;
  const int S = smax + 4 * ks;
  // padded rows (pitch >= S, 4 mod 32: the 8 rows of an A fragment hit
  // distinct banks), or the contiguous window (pitch os2, rows overlapping,
  // some A fragments 2-way bank conflicted) where padded rows would stage
  // every sample more than 1.25 times
  const int P = 4 * S > 5 * os2 ? os2 : S + ((36 - S % 32) % 32);
  const size_t row_bytes = (size_t)P * 4;
  int F = std::min(256, (int)((kMmaWindowBytes - (size_t)(S - std::min(S, P)) * 4) / row_bytes) / 32 * 32);
  if (F < 8 * kMmaGroups) return;
  const int units = nb * (F / (8 * kMmaGroups));
  int warps = std::min(units, 8);
  for (int d = kMmaMaxWarps; d >= 4; --d)
    if (units % d == 0) {
      warps = d;
      break;
    }
  bfrag.assign((size_t)nb * ks * 32, 0.0);
  for (int b = 0; b < nb; ++b)
    for (int k = 0; k < ks; ++k)
      for (int lane = 0; lane < 32; ++lane) {
        const int q = 8 * b + lane / 4;
        const int i = sblock[b] + 4 * k + lane % 4 - off[q];
        if (i >= 0 && i < cnt[q]) bfrag[((size_t)b * ks + k) * 32 + lane] = (double)taps[(size_t)(q % ns) * maxc + i];
      }
  t.fwd_mma = ks;
  t.mma_os = os2;
  t.mma_ns = ns2;
  t.mma_blocks = nb;
  t.mma_span = S;
  t.mma_pitch = P;
  t.mma_frames = F;
  t.mma_warps = warps;
}

// Geometry and tables of the tensor-core adjoint for float32-valued taps
// [ns][wt]; leaves t.adj_mma false for rate pairs whose tables or staged
// window would be too large.
void plan_adj_mma(int os, int ns, int wt, const double* d_taps, ResampleTables& t, std::vector<double>& bfrag,
                  std::vector<int>& aoffs, std::vector<int>& koff) {
  t.adj_mma = false;
  const int G = os >= 64 ? 1 : 8 / gcd_int(os, 8);
  if ((int64_t)os * G > 4096 || (int64_t)ns * G > 4096) return;
  const int os2 = os * G, ns2 = ns * G, wt2 = (G - 1) * os + wt;
  const int nc = (os2 + 7) / 8;
  const int maxdl = (wt2 - 1) / os2;
  if ((int64_t)nc * (maxdl + 1) * ns2 * 8 > ((int64_t)1 << 26)) return;
  const int P = (ns2 + 1) + ((36 - (ns2 + 1) % 32) % 32);  // >= ns2 + 1 (zero column), 4 mod 32
  const int chunks = std::max(1, (8 + nc - 1) / nc);
  const int F = 8 * kMmaGroups * chunks;
  if ((size_t)(F + maxdl) * P * 4 > kResampleSmemLimit) return;
  // float32 tap of super-phase q at super-tap k2 (the phase's taps shifted by (q / ns) * os)
  auto tap2 = [&](int q, int k2) -> float {
    const int k = k2 - (q / ns) * os;
    return (k >= 0 && k < wt) ? (float)d_taps[(size_t)(q % ns) * wt + k] : 0.0f;
  };
  koff.assign(nc + 1, 0);
  bfrag.clear();
  aoffs.clear();
  std::vector<int> edl, eq;
  for (int c = 0; c < nc; ++c) {
    edl.clear();
    eq.clear();
    for (int dl = 0; dl <= maxdl; ++dl)
      for (int q = 0; q < ns2; ++q)
        for (int rr = 0; rr < 8; ++rr) {
          const int rho = 8 * c + rr, k2 = rho + dl * os2;
          if (rho < os2 && k2 < wt2 && tap2(q, k2) != 0.0f) {
            edl.push_back(dl);
            eq.push_back(q);
            break;
          }
        }
    const int ne = (int)edl.size();
    const int ks = std::max(1, (ne + 3) / 4);
    koff[c + 1] = koff[c] + ks;
    for (int k = 0; k < ks; ++k) {
      for (int kk = 0; kk < 4; ++kk) {
        const int e = 4 * k + kk;
        aoffs.push_back(e < ne ? -edl[e] * P + eq[e] : ns2);
      }
      for (int lane = 0; lane < 32; ++lane) {
        const int e = 4 * k + lane % 4, rho = 8 * c + lane / 4;
        double v = 0.0;
        if (e < ne && rho < os2) {
          const int k2 = rho + edl[e] * os2;
          if (k2 < wt2) v = (double)tap2(eq[e], k2);
        }
        bfrag.push_back(v);
      }
    }
  }
  const int units = nc * chunks;
  int warps = std::min(units, kMmaMaxWarps);
  for (int d = kMmaMaxWarps; d >= 4; --d)
    if (units % d == 0) {
      warps = d;
      break;
    }
  t.adj_mma = true;
  t.amma_os = os2;
  t.amma_ns = ns2;
  t.amma_blocks = nc;
  t.amma_pitch = P;
  t.amma_frames = F;
  t.amma_warps = warps;
  t.amma_maxdl = maxdl;
}

}  // namespace

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
  std::vector<double> bfrag;
  std::vector<int> sblock;
  plan_fwd_mma(os, ns, first, count, taps, maxc, t, bfrag, sblock);
  std::vector<double> abfrag;
  std::vector<int> aoffs, akoff;
  plan_adj_mma(os, ns, wt, d_taps, t, abfrag, aoffs, akoff);
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
  if (ok && t.fwd_mma) {
    ok = cudaMalloc(&t.mma_b, bfrag.size() * 8) == cudaSuccess &&
         cudaMalloc(&t.mma_s, sblock.size() * 4) == cudaSuccess &&
         cudaMemcpy(t.mma_b, bfrag.data(), bfrag.size() * 8, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(t.mma_s, sblock.data(), sblock.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  }
  if (ok && t.adj_mma) {
    ok = cudaMalloc(&t.amma_b, abfrag.size() * 8) == cudaSuccess &&
         cudaMalloc(&t.amma_a, aoffs.size() * 4) == cudaSuccess &&
         cudaMalloc(&t.amma_off, akoff.size() * 4) == cudaSuccess &&
         cudaMemcpy(t.amma_b, abfrag.data(), abfrag.size() * 8, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(t.amma_a, aoffs.data(), aoffs.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
         cudaMemcpy(t.amma_off, akoff.data(), akoff.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  }
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
  cudaFree(t.mma_b);
  cudaFree(t.mma_s);
  cudaFree(t.amma_b);
  cudaFree(t.amma_a);
  cudaFree(t.amma_off);
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
  ra.mma_b = t.mma_b;
  ra.mma_s = t.mma_s;
  ra.fwd_mma = t.fwd_mma;
  ra.mma_os = t.mma_os;
  ra.mma_ns = t.mma_ns;
  ra.mma_blocks = t.mma_blocks;
  ra.mma_span = t.mma_span;
  ra.mma_pitch = t.mma_pitch;
  ra.mma_frames = t.mma_frames;
  ra.mma_warps = t.mma_warps;
  ra.amma_b = t.amma_b;
  ra.amma_a = t.amma_a;
  ra.amma_off = t.amma_off;
  ra.adj_mma = t.adj_mma;
  ra.amma_os = t.amma_os;
  ra.amma_ns = t.amma_ns;
  ra.amma_blocks = t.amma_blocks;
  ra.amma_pitch = t.amma_pitch;
  ra.amma_frames = t.amma_frames;
  ra.amma_warps = t.amma_warps;
  ra.amma_maxdl = t.amma_maxdl;
  return ra;
}

}  // namespace pesq
