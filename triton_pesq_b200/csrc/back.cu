// Back end of the PESQ backward pass, one CTA per (gradient row, segment).
//
// With F the unscaled Bark spectrum of a row and g = dL/dF (from the chain
// backward, which already folded in the alignment scale s^2), the gradient of
// the loss w.r.t. the 16 kHz row x is
//
//   dL/dx = ramp . H_pre^T [ sum_t w . adj_t(g_t) ]  -  kappa * H_pow^T H_pow x
//
// where adj_t is the adjoint of "power spectrum -> Bark segment sums" of frame
// t, evaluated as an inverse real FFT of (dL/dP_f) X_f, and
// kappa = 2 <g, F> / sum (H_pow x)^2 is the derivative through the level
// alignment scale (torch_pesq/loss.py:132-139).  z = H_pow^T H_pow x was saved
// by the front kernel.
//
// The CTA recomputes y = H_pre ramp(x) over its span (forward warm-up before
// the segment, frames around it), overlap-adds the per-frame gradients in a
// fixed order (even frames, then odd frames: no atomics, bitwise
// reproducible), and runs the pre-emphasis adjoint backwards in time with
// kHorizon samples of look-ahead.
#include "fft.cuh"
#include "kernels.cuh"

namespace pesq {

namespace {

constexpr int kBackSmemFloats = 2 * kSpan + scan_scratch_floats<2>() + kWarps * kFftScratch * 2 +
                                kWarps * kNfft + kWarps * kMaxBands + sizeof(DevTables) / 4 + 64;

__global__ void __launch_bounds__(kThreads, 1)
    back_kernel(const __grid_constant__ BackArgs p, const __grid_constant__ PreTab pre) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                 // kSpan: input, then y in place
  float* gy = xs + kSpan;           // kSpan: dL/dy, then dL/d(ramped x) in place
  float* es = gy + kSpan;
  float2* fft = reinterpret_cast<float2*>(es + scan_scratch_floats<2>());
  float* gu = reinterpret_cast<float*>(fft + kWarps * kFftScratch);  // per warp kNfft
  float* gb = gu + kWarps * kNfft;                                    // per warp kMaxBands
  DevTables* tab = reinterpret_cast<DevTables*>(gb + kWarps * kMaxBands);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = p.row_begin + blockIdx.x / p.nseg;
  const int seg = blockIdx.x % p.nseg;
  const int64_t n_row = p.n;
  const int64_t a = (int64_t)seg * p.seg_frames * kHop;
  const int64_t send = min(a + (int64_t)p.seg_frames * kHop, n_row);
  // one hop before the segment (frame t0-1 overlaps it) plus the warm-up
  const int64_t base = a - kHop - kHorizon;
  const float* xr = p.src.row(row);

  {
    const float4* src4 = reinterpret_cast<const float4*>(p.tab);
    float4* dst4 = reinterpret_cast<float4*>(tab);
    for (int i = tid; i < (int)(sizeof(DevTables) / 16); i += kThreads) dst4[i] = src4[i];
  }
  for (int i = tid; i < kSpan; i += kThreads) {
    const int64_t n = base + i;
    xs[i] = (n >= 0 && n < n_row) ? __ldg(xr + n) : 0.0f;
    gy[i] = 0.0f;
  }
  __syncthreads();

  // y = H_pre ramp(x), zero past the row end
  chunk_scan<2, true>(
      pre, es,
      [&](int q) {
        const int64_t n = base + q;
        return (n >= 0 && n < n_row) ? edge_ramp(xs[q], n, n_row) : 0.0f;
      },
      [&](int q, float y) { xs[q] = (base + q < n_row) ? y : 0.0f; });
  __syncthreads();

  // frames that touch [a, send + kHorizon)
  const int nb = tab->nb;
  const int t0 = seg * p.seg_frames;
  const int t_lo = max(0, t0 - 1);
  const int t_hi = min(p.frames - 1, (int)((send + kHorizon - 1) / kHop));
  const float kappa = p.kappa[row];
  float2* sh = fft + warp * kFftScratch;
  float* gw = gu + warp * kNfft;
  float* gbw = gb + warp * kMaxBands;

  for (int parity = 0; parity < 2; ++parity) {
    const int first = t_lo + ((t_lo & 1) != parity ? 1 : 0);
    for (int t = first + 2 * warp; t <= t_hi; t += 2 * kWarps) {
      const int off = (int)(t * (int64_t)kHop - base);
      const float* gsrc = p.g_bark + ((int64_t)row * p.frames + t) * nb;
      for (int b = lane; b < nb; b += 32) gbw[b] = gsrc[b] * tab->band_corr[b];
      __syncwarp();
      float2 X[8];
      warp_rfft512(xs + off, tab->window, sh, tab->tw256, tab->tw512, lane, X);
      // V_f = dL/dP_f * X_f, with dL/dP_f = corr_b dL/dB_b for the band b of bin f
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int f = lane + 32 * m;
        const int b = tab->bin_band[f];
        X[m] = c_scale(X[m], b >= 0 ? gbw[b] : 0.0f);
      }
      warp_irfft512_adjoint(X, sh, tab->tw256, tab->tw512, lane, gw);
      for (int k = lane; k < kNfft; k += 32) gy[off + k] += tab->window[k] * gw[k];
      __syncwarp();
    }
    __syncthreads();
  }

  // pre-emphasis adjoint on [a, send): backwards in time from send + kHorizon;
  // the gradient of the zero padding after the row end is dropped
  const int top = kHop + 2 * kHorizon + (int)(send - a) - 1;
  chunk_scan<2, true>(
      pre, es,
      [&](int q) {
        const int idx = top - q;
        return (idx >= 0 && base + idx < n_row) ? gy[idx] : 0.0f;
      },
      [&](int q, float y) {
        const int idx = top - q;
        if (idx >= 0) gy[idx] = y;
      });
  __syncthreads();

  const float* zr = p.z + (int64_t)row * n_row;
  float* outr = p.out.row(row);
  for (int i = tid; i < (int)(send - a); i += kThreads) {
    const int64_t n = a + i;
    const float g = edge_ramp(gy[kHop + kHorizon + i], n, n_row);
    outr[n] = fmaf(-kappa, zr[n], g);
  }
}

}  // namespace

size_t back_smem_bytes() { return (size_t)kBackSmemFloats * sizeof(float); }

cudaError_t launch_back(const BackArgs& a, const PreTab& pre, int rows, cudaStream_t s) {
  const int64_t blocks = (int64_t)rows * a.nseg;
  if (blocks <= 0) return cudaSuccess;
  back_kernel<<<(unsigned)blocks, kThreads, back_smem_bytes(), s>>>(a, pre);
  return cudaGetLastError();
}

cudaError_t configure_back() {
  return cudaFuncSetAttribute(back_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)back_smem_bytes());
}

}  // namespace pesq
