// Back end of the PESQ backward pass, one CTA per (gradient row, segment).
//
// With F the unscaled Bark spectrum of a row and g = dL/dF (from the chain
// backward, which already folded in the alignment scale s^2), the gradient of
// the loss w.r.t. the 16 kHz row x is
//
//   dL/dx = ramp . H_pre^T [ sum_t w . adj_t(g_t) ]  -  kappa * H_pow^T H_pow x
//
// where adj_t is the adjoint of "power spectrum -> Bark segment sums" of frame
// t, evaluated as an inverse real FFT of (dL/dP_f) X_f with the spectrum X_t
// the front kernel saved, and kappa = 2 <g, F> / sum (H_pow x)^2 is the
// derivative through the level alignment scale (torch_pesq/loss.py:132-139).
// z = H_pow^T H_pow x was saved by the front kernel as well.
//
// The CTA overlap-adds the per-frame gradients around its segment in a fixed
// order (even frames, then odd frames: no atomics, bitwise reproducible) and
// runs the pre-emphasis adjoint backwards in time with kBackHorizon samples
// of look-ahead.
#include "kernels.cuh"

namespace pesq {

PESQ_PHASE_TABLE(g_phase_back)
PESQ_SPAN_TABLE(g_span_back)
PESQ_CTA_TABLE(g_cta_back)

namespace {

constexpr int kSegMax = kBackSegFrames * kHop;  // samples of the longest segment
// frames a CTA processes: one before its segment, the segment and those
// reaching kBackHorizon past its end
constexpr int kBackFrames = kBackSegFrames + 1 + kBackHorizon / kHop;

// Shared-memory geometry of a back CTA of NT threads.  A full-size CTA (one
// per SM) processes one frame per warp and parity pass; a half-size one (two
// per SM, for batches of many waves) two.  Both stage the same segment: the
// span of a half-size CTA (8448 samples) still covers the hop before it, the
// segment and the look-ahead, so the results are the same bit for bit.
template <int NT>
struct BackGeom {
  static constexpr int kSpanT = NT * kChunk;
  static constexpr int kWarpsT = NT / 32;
  static constexpr int kSmemBytes = kSpanT * 4 + scan_scratch_floats<2, float, NT>() * 4 +
                                    kWarpsT * FftLayout<float>::kSlots * 8 + kWarpsT * kMaxBands * 4 +
                                    (int)sizeof(DevTables) + kSegMax * 4 + kBackFrames * kMaxBands * 4;
  static_assert(kHop + kSegMax + kBackHorizon <= kSpanT, "back kernel span");
};
static_assert(2 * (BackGeom<kThreads / 2>::kSmemBytes + 1024) <= 228 * 1024, "two half-size CTAs per SM");

// kGather: general frame geometry, dL/dy is gathered from the frame gradients
// of the spectrum kernel (spectrum.cu) instead of the fused transforms
template <bool kGather, int NT>
__global__ void __launch_bounds__(NT, kThreads / NT)
    back_kernel(const __grid_constant__ BackArgs p, const __grid_constant__ PreTab pre) {
  constexpr int kSpan = BackGeom<NT>::kSpanT;  // (shadow the 512-thread constants)
  constexpr int kWarps = BackGeom<NT>::kWarpsT;
  extern __shared__ __align__(16) float smem[];
  float* gy = smem;  // kSpan: dL/dy, then dL/d(ramped x) in place
  float* es = gy + kSpan;
  Cx<float>* fft = reinterpret_cast<Cx<float>*>(es + scan_scratch_floats<2, float, NT>());
  float* gb = reinterpret_cast<float*>(fft + kWarps * FftLayout<float>::kSlots);  // per warp kMaxBands
  DevTables* tab = reinterpret_cast<DevTables*>(gb + kWarps * kMaxBands);
  float* zs = reinterpret_cast<float*>(tab + 1);  // z on [a, send), staged asynchronously
  float* gs = zs + kSegMax;                       // dL/dB of frames t_lo..t_hi

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = p.row_begin + blockIdx.x / p.nseg;
  const int seg = blockIdx.x % p.nseg;
  const int64_t n_row = p.n;
  const int64_t a = (int64_t)seg * p.seg_frames * kHop;
  const int64_t send = min(a + (int64_t)p.seg_frames * kHop, n_row);
  // the span starts at frame t0 - 1, which overlaps the segment
  const int64_t base = a - kHop;
  PESQ_SPAN_BEGIN(g_span_back, 0);
  PESQ_CTA_BEGIN(g_cta_back);
  PESQ_STAMP(g_phase_back, 0);

  if constexpr (kGather) {
    pdl_wait();
    // dL/dy on [a, send + kBackHorizon): sum over the frames covering each sample
    // (frame order), z staged in the background
    const float* zr = p.z + (int64_t)row * n_row;
    for (int i = tid; i < (int)(send - a); i += NT) cp_async4(zs + i, zr + a + i);
    cp_async_commit();
    const float* fg = p.frame_grad + (int64_t)(row - p.row_begin) * p.frames * p.nfft;
    const int top_g = kHop + kBackHorizon + (int)(send - a);
    for (int i = tid; i < kSpan; i += NT) {
      const int64_t n = base + i;
      float acc = 0.0f;
      if (i >= kHop && i < top_g && n < n_row) {
        // rows hold at most 2^31 samples: 32-bit divisions
        const unsigned un = (unsigned)n, hop = (unsigned)p.hop, nfft = (unsigned)p.nfft;
        const int t_hi = min(p.frames - 1, (int)(un / hop));
        const int t_lo = un >= nfft ? (int)((un - nfft) / hop) + 1 : 0;
        for (int t = t_lo; t <= t_hi; ++t) acc += __ldg(fg + (int64_t)t * p.nfft + (n - (int64_t)t * p.hop));
      }
      gy[i] = acc;
    }
    __syncthreads();
  } else {
  // frames that touch [a, send + kBackHorizon)
  const int nb = p.nb;
  const int t0 = seg * p.seg_frames;
  const int t_lo = max(0, t0 - 1);
  const int t_hi = min(p.frames - 1, (int)((send + kBackHorizon - 1) / kHop));

  // first copy group: constant tables and dL/dB of the CTA's frames; second
  // group: z = H^T H x of the segment, only needed at the very end, copied in
  // the background of the frame loop
  copy_async<NT>(tab, p.tab, (int)sizeof(DevTables));
  // launched with programmatic serialisation: what follows reads the output
  // of the kernels before this one
  pdl_wait();
  {
    const float* src = p.g_bark + ((int64_t)row * p.frames + t_lo) * nb;
    const int cnt = (t_hi - t_lo + 1) * nb;
    for (int i = tid; i < cnt; i += NT) cp_async4(gs + i, src + i);
  }
  cp_async_commit();
  for (int i = tid; i < kSpan; i += NT) gy[i] = 0.0f;
  const float* zr = p.z + (int64_t)row * n_row;
  for (int i = tid; i < (int)(send - a); i += NT) cp_async4(zs + i, zr + a + i);
  cp_async_commit();
  cp_async_wait_group<1>();
  __syncthreads();
  PESQ_STAMP(g_phase_back, 1);

  Cx<float>* sh = fft + warp * FftLayout<float>::kSlots;
  float* gbw = gb + warp * kMaxBands;
  int band_of[8];  // band of bin lane + 32 m (-1: none)
#pragma unroll
  for (int m = 0; m < 8; ++m) band_of[m] = tab->bin_band[lane + 32 * m];

  for (int parity = 0; parity < 2; ++parity) {
    const int first = t_lo + ((t_lo & 1) != parity ? 1 : 0);
    // the saved spectrum of the warp's next frame is loaded one frame ahead
    Cx<float> X[8];
    auto load_spec = [&](int t, Cx<float> dst[8]) {
      const Cx<float>* spec = p.spec + ((int64_t)row * p.frames + t) * kBins;
#pragma unroll
      for (int m = 0; m < 8; ++m) dst[m] = spec[lane + 32 * m];
    };
    if (first + 2 * warp <= t_hi) load_spec(first + 2 * warp, X);
    for (int t = first + 2 * warp; t <= t_hi; t += 2 * kWarps) {
      Cx<float> Xn[8];
      if (t + 2 * kWarps <= t_hi) load_spec(t + 2 * kWarps, Xn);
      const int off = (int)(t * (int64_t)kHop - base);
      const float* gsrc = gs + (t - t_lo) * nb;
      for (int b = lane; b < nb; b += 32) gbw[b] = gsrc[b] * tab->band_corr[b];
      __syncwarp();
      // V_f = dL/dP_f * X_f, with dL/dP_f = corr_b dL/dB_b for the band b of bin f
      Cx<float> V[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) V[m] = c_scale(X[m], band_of[m] >= 0 ? gbw[band_of[m]] : 0.0f);
      Cx<float> g[8];
      warp_irfft512_adjoint(V, sh, tab->fft, lane, g);
      // overlap-add of the windowed frame gradient: samples 2n, 2n + 1 with
      // n = lane + 32 m (frames of one parity never overlap)
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int k = 2 * (lane + 32 * m);
        const float2 w = *reinterpret_cast<const float2*>(tab->window + k);
        float2* dst = reinterpret_cast<float2*>(gy + off + k);
        float2 acc = *dst;
        acc.x = fmaf(w.x, g[m].x, acc.x);
        acc.y = fmaf(w.y, g[m].y, acc.y);
        *dst = acc;
      }
      __syncwarp();
#pragma unroll
      for (int m = 0; m < 8; ++m) X[m] = Xn[m];
    }
    __syncthreads();
  }
  }
  const float kappa = p.kappa[row];
  PESQ_STAMP(g_phase_back, 2);

  // pre-emphasis adjoint on [a, send): backwards in time from send + kBackHorizon;
  // the gradient of the zero padding after the row end is dropped
  const int top = kHop + kBackHorizon + (int)(send - a) - 1;
  chunk_scan<2, true, float, false, NT>(
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

  cp_async_wait_all();
  __syncthreads();
  PESQ_STAMP(g_phase_back, 3);
  float* outr = p.out.row(row);
  for (int i = tid; i < (int)(send - a); i += NT) {
    const int64_t n = a + i;
    const float g = edge_ramp(gy[kHop + i], n, n_row);
    outr[n] = fmaf(-kappa, zs[i], g);
  }
  PESQ_STAMP(g_phase_back, 4);
  PESQ_CTA_END(g_cta_back);
  PESQ_SPAN_END(g_span_back, 0);
}

}  // namespace

size_t back_smem_bytes(int threads) {
  return (size_t)(threads == kThreads ? BackGeom<kThreads>::kSmemBytes : BackGeom<kThreads / 2>::kSmemBytes);
}

cudaError_t launch_back(const BackArgs& a, const PreTab& pre, int rows, cudaStream_t s) {
  const int64_t blocks = (int64_t)rows * a.nseg;
  if (blocks <= 0) return cudaSuccess;
  // programmatic serialisation: the CTAs may be scheduled while the align
  // kernel finishes and wait (pdl_wait) before reading its output
  if (a.threads == kThreads / 2 && !a.frame_grad) {
    LaunchShape l((unsigned)blocks, kThreads / 2, back_smem_bytes(kThreads / 2), s, true);
    return cudaLaunchKernelEx(&l.cfg, back_kernel<false, kThreads / 2>, a, pre);
  }
  LaunchShape l((unsigned)blocks, kThreads, back_smem_bytes(kThreads), s, true);
  if (a.frame_grad) return cudaLaunchKernelEx(&l.cfg, back_kernel<true, kThreads>, a, pre);
  return cudaLaunchKernelEx(&l.cfg, back_kernel<false, kThreads>, a, pre);
}

cudaError_t configure_back() {
  cudaError_t e = cudaFuncSetAttribute(back_kernel<false, kThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)back_smem_bytes(kThreads));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(back_kernel<true, kThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)back_smem_bytes(kThreads));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(back_kernel<false, kThreads / 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)back_smem_bytes(kThreads / 2));
}

}  // namespace pesq
