// Front end of the PESQ forward pass, one CTA per (row, segment).
//
// For the samples [a, a + S) of one row (a 16 kHz signal) the CTA evaluates,
// in shared memory and without touching HBM in between:
//
//   f  = H_pow x            level-alignment band pass (order 10)    -> sum f^2
//   z  = H_pow^T f          (only for rows that need a gradient)    -> HBM
//   y  = H_pre ramp(x)      edge fade + pre-emphasis biquad
//   B  = corr * segsum |rfft512(w * y_t)|^2   for the frames starting in [a, a+S)
//
// all on the *unscaled* signal: everything up to the power spectrum is linear,
// so the level alignment scale s = sqrt(1e7 / P) enters the Bark spectrum as
// s^2 and is applied later by the chain kernel (torch_pesq/loss.py:127-203
// evaluated in a different but algebraically identical order).  The peak
// normalisation of loss.py:179-183 is a no-op for the same reason: the
// pipeline output is invariant to the scale of each input.
//
// The CTA stages kSpan samples starting kHorizon before `a`: the first
// kHorizon are the warm-up of the forward scans, and the reverse scan that
// produces z looks kHorizon samples past the end of the segment.
#include "fft.cuh"
#include "kernels.cuh"

namespace pesq {

namespace {

constexpr int kFrontSmemFloats = 2 * kSpan + scan_scratch_floats<10>() + kWarps * kFftScratch * 2 +
                                 sizeof(DevTables) / 4 + 2 * kWarps + 64;

__global__ void __launch_bounds__(kThreads, 1)
    front_kernel(const __grid_constant__ FrontArgs p, const __grid_constant__ PowTab pow,
                 const __grid_constant__ PreTab pre) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                       // kSpan: input, then y in place
  float* fb = xs + kSpan;                 // kSpan: f, then z in place
  float* es = fb + kSpan;                 // scan scratch
  float2* fft = reinterpret_cast<float2*>(es + scan_scratch_floats<10>());  // per-warp FFT scratch
  DevTables* tab = reinterpret_cast<DevTables*>(fft + kWarps * kFftScratch);
  double* red = reinterpret_cast<double*>(tab + 1);  // kWarps

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x / p.nseg;
  const int seg = blockIdx.x - row * p.nseg;
  const int64_t n_row = p.n;
  const int64_t a = (int64_t)seg * p.seg_frames * kHop;
  const int64_t send = min(a + (int64_t)p.seg_frames * kHop, n_row);
  const int64_t base = a - kHorizon;
  const float* xr = p.src.row(row);

  // constant tables
  {
    const float4* src4 = reinterpret_cast<const float4*>(p.tab);
    float4* dst4 = reinterpret_cast<float4*>(tab);
    for (int i = tid; i < (int)(sizeof(DevTables) / 16); i += kThreads) dst4[i] = src4[i];
  }
  // stage the span; zeros outside the row reproduce the zero initial state
  for (int i = tid; i < kSpan; i += kThreads) {
    const int64_t n = base + i;
    xs[i] = (n >= 0 && n < n_row) ? __ldg(xr + n) : 0.0f;
  }
  __syncthreads();

  // 1. level alignment filter f = H x, sum of squares over [a, send)
  // 2. z = H^T f on [a, send): the adjoint filter runs backwards in time from
  //    send + kHorizon; f beyond the row end is not part of the signal.
  // Both passes share one instance of the scan code (pass 0 forward from xs
  // into fb, pass 1 backward over fb in place), which keeps the two unrolled
  // scans from competing for registers.
  const int passes = (row >= p.z_begin && row < p.z_end) ? 2 : 1;
  const int top = 2 * kHorizon + (int)(send - a) - 1;
  double ssq = 0.0;
  for (int pass = 0; pass < passes; ++pass) {
    chunk_scan<10, false>(
        pow, es,
        [&](int q) {
          if (pass == 0) return xs[q];
          const int idx = top - q;
          return (idx >= 0 && base + idx < n_row) ? fb[idx] : 0.0f;
        },
        [&](int q, float y) {
          const int idx = pass == 0 ? q : top - q;
          if (idx >= 0) fb[idx] = y;
          const int64_t n = base + q;
          if (pass == 0 && n >= a && n < send) ssq = fma((double)y, (double)y, ssq);
        });
    if (pass == 0) {
      ssq = warp_sum(ssq);
      if (lane == 0) red[warp] = ssq;
    }
    __syncthreads();
  }
  if (tid == 0) {
    double tot = 0.0;
    for (int w = 0; w < kWarps; ++w) tot += red[w];
    p.partial[(int64_t)row * p.nseg + seg] = tot;
  }
  if (passes == 2) {
    float* zr = p.z + (int64_t)row * n_row;
    for (int i = tid; i < (int)(send - a); i += kThreads) zr[a + i] = fb[kHorizon + i];
  }

  // 3. edge fade + pre-emphasis, in place; the padding after the row end is 0
  chunk_scan<2, true>(
      pre, es,
      [&](int q) {
        const int64_t n = base + q;
        return (n >= 0 && n < n_row) ? edge_ramp(xs[q], n, n_row) : 0.0f;
      },
      [&](int q, float y) { xs[q] = (base + q < n_row) ? y : 0.0f; });
  __syncthreads();

  // 4. frames starting in this segment: window, rfft, power, Bark segment sums
  const int nb = tab->nb;
  const int t0 = seg * p.seg_frames;
  const int t1 = min(t0 + p.seg_frames, p.frames);
  float2* sh = fft + warp * kFftScratch;
  float* pw = reinterpret_cast<float*>(fft + warp * kFftScratch);
  for (int t = t0 + warp; t < t1; t += kWarps) {
    const float* frame = xs + kHorizon + (t - t0) * kHop;
    float2 X[8];
    warp_rfft512(frame, tab->window, sh, tab->tw256, tab->tw512, lane, X);
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int f = lane + 32 * m;
      pw[f] = f == 0 ? 0.0f : fmaf(X[m].x, X[m].x, X[m].y * X[m].y);
    }
    __syncwarp();
    float* out = p.bark + ((int64_t)row * p.frames + t) * nb;
    for (int b = lane; b < nb; b += 32) {
      float acc = 0.0f;
      for (int f = tab->band_start[b]; f < tab->band_end[b]; ++f) acc += pw[f];
      out[b] = acc * tab->band_corr[b];
    }
    __syncwarp();
  }
}

}  // namespace

size_t front_smem_bytes() { return (size_t)kFrontSmemFloats * sizeof(float); }

cudaError_t configure_front() {
  return cudaFuncSetAttribute(front_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)front_smem_bytes());
}

cudaError_t launch_front(const FrontArgs& a, const PowTab& pow, const PreTab& pre, int rows, cudaStream_t s) {
  const int64_t blocks = (int64_t)rows * a.nseg;
  if (blocks <= 0) return cudaSuccess;
  front_kernel<<<(unsigned)blocks, kThreads, front_smem_bytes(), s>>>(a, pow, pre);
  return cudaGetLastError();
}

}  // namespace pesq
