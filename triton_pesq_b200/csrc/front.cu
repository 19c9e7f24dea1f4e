// Front end of the PESQ forward pass, one CTA per (row, segment).
//
// For the samples [a, a + S) of one row (a 16 kHz signal) the CTA evaluates,
// in shared memory and without touching HBM in between:
//
//   f  = H_pow x            level-alignment band pass (order 10)    -> sum f^2
//                           (rows that need a gradient: f itself)  -> HBM
//   y  = H_pre ramp(x)      edge fade + pre-emphasis biquad, float64
//   X_t = rfft512(w * y_t)  for the frames starting in [a, a+S), float64
//   B  = corr * segsum |X_t|^2                                      -> HBM
//   X_t                     (rows that need a gradient)             -> HBM
//
// all on the *unscaled* signal: everything up to the power spectrum is linear,
// so the level alignment scale s = sqrt(1e7 / P) enters the Bark spectrum as
// s^2 and is applied later by the chain kernel (torch_pesq/loss.py:127-203
// evaluated in a different but algebraically identical order).  The peak
// normalisation of loss.py:179-183 is a no-op for the same reason: the
// pipeline output is invariant to the scale of each input.
//
// y and the spectrum are evaluated in double precision: the weak high bands
// of speech sit 50-60 dB below the frame peak, where float32 rounding of the
// signal would leave ~1e-4 relative error in their power, and the loss
// gradient is most sensitive exactly there.  y is kept in shared memory in
// double precision.
//
// The CTA stages kSpan samples starting kHorizon before `a`: the first
// kHorizon are the warm-up of the forward scans.
#include "kernels.cuh"

namespace pesq {

PESQ_PHASE_TABLE(g_phase_front)
PESQ_SPAN_TABLE(g_span_front)
PESQ_CTA_TABLE(g_cta_front)

namespace {

constexpr int kFftFloats = kWarps * FftLayout<double>::kSlots * 4;
constexpr int kFrontScratchFloats =
    kFftFloats > scan_scratch_floats<10>() ? kFftFloats : scan_scratch_floats<10>();
constexpr int kFrontSmemBytes = 2 * kSpan * 4 + kFrontScratchFloats * 4 + (int)sizeof(DevTables) +
                                (int)sizeof(DevTwiddle64) + kWarps * 8 + 16;
static_assert(sizeof(DevTables) % 16 == 0 && sizeof(DevTwiddle64) % 16 == 0, "bulk copies of the tables");
static_assert((2 * kSpan * 4 + kFrontScratchFloats * 4) % 16 == 0, "16-byte aligned tables in shared memory");

// kSignal: general frame geometry, y is written to p.y64 and the frames are
// left to the spectrum kernel (spectrum.cu)
template <bool kSignal>
__global__ void __launch_bounds__(kThreads, 1)
    front_kernel(const __grid_constant__ FrontArgs p, const __grid_constant__ PowTab pow,
                 const __grid_constant__ PreTab64 pre) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                 // kSpan: input (hi part)
  float* fb = xs + kSpan;           // kSpan: [f = H x,] low part of a resampled x
                                    // (xs, fb) then hold y as kSpan doubles
  float* scratch = fb + kSpan;      // scan scratch, later the per-warp FFT scratch
  DevTables* tab = reinterpret_cast<DevTables*>(scratch + kFrontScratchFloats);
  DevTwiddle64* tw = reinterpret_cast<DevTwiddle64*>(tab + 1);
  double* red = reinterpret_cast<double*>(tw + 1);  // kWarps
  uint64_t* bar = reinterpret_cast<uint64_t*>(red + kWarps);  // completion of the bulk copies

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = blockIdx.x / p.nseg;
  const int seg = blockIdx.x - row * p.nseg;
  const int64_t n_row = p.n;
  const int64_t a = (int64_t)seg * p.seg_frames * kHop;
  const int64_t send = min(a + (int64_t)p.seg_frames * kHop, n_row);
  const int64_t base = a - kHorizon;
  const void* xr = p.src.row_any(row);  // the caller's rows (any element type)
  const bool grad_row = row >= p.spec_begin && row < p.spec_end;
  PESQ_SPAN_BEGIN(g_span_front, 0);
  PESQ_CTA_BEGIN(g_cta_front);
  PESQ_STAMP(g_phase_front, 0);

  // the chain forward that follows on the stream counts its clusters here
  if (blockIdx.x == 0 && tid == 0) *p.done = 0u;
  // Stage the span (zeros outside the row reproduce the zero initial state)
  // and the constant tables.  The tables, and the part of a float32 row's
  // span that starts on a 16-byte boundary in both memories, arrive by bulk
  // copies (TMA, this GPU's memory, no multicast) signalled on one mbarrier;
  // the ragged tail, the zeros and other rows (16-bit, misaligned) are staged
  // by the threads meanwhile.
  const float* xf = static_cast<const float*>(xr);
  const int64_t lo = base > 0 ? base : 0;
  const int64_t hi = min(base + (int64_t)kSpan, n_row);
  const int64_t cnt4 = hi > lo ? ((hi - lo) & ~(int64_t)3) : 0;
  const bool bulk_span = p.src.type == kInF32 && cnt4 > 0 && ((lo - base) & 3) == 0 &&
                         (reinterpret_cast<uintptr_t>(xf + lo) & 15) == 0;
  if (tid == 0) mbar_init(bar);
  __syncthreads();
  if (tid == 0) {
    const uint32_t span_bytes = bulk_span ? (uint32_t)(cnt4 * 4) : 0u;
    mbar_arrive_expect_tx(bar, (uint32_t)(sizeof(DevTables) + sizeof(DevTwiddle64)) + span_bytes);
    bulk_g2s(tab, p.tab, (uint32_t)sizeof(DevTables), bar);
    bulk_g2s(tw, p.tw64, (uint32_t)sizeof(DevTwiddle64), bar);
    if (bulk_span) bulk_g2s(xs + (lo - base), xf + lo, span_bytes, bar);
  }
  if (bulk_span) {
    for (int i = tid; i < kSpan; i += kThreads) {
      const int64_t q = base + i;
      if (q < lo || q >= lo + cnt4) xs[i] = q >= lo && q < hi ? __ldg(xf + q) : 0.0f;
    }
  } else {
    stage_span_any(xs, xr, base, n_row, p.src.type);
  }
  // The low part of a resampled input (x = hi + lo) joins the pre-emphasis.
  // On gradient rows fb first holds f = H x (below), the low part only after.
  const bool has_lo = p.src_lo.ref != nullptr;
  if (has_lo && !grad_row) stage_span(fb, p.src_lo.row(row), base, n_row);
  if (!mbar_wait(bar, 0)) {
    // the copies did not land in time: flag it, give them one more bounded
    // wait (they write into this CTA's shared memory) and carry on
    if (tid == 0) atomicOr(p.err, kErrBulkTimeout);
    mbar_wait(bar, 0);
  }
  __syncthreads();
  PESQ_STAMP(g_phase_front, 1);

  // 1. level alignment filter f = H x: its sum of squares over [a, send), and
  //    on gradient rows f itself on [a, send), from which the align kernel of
  //    the backward evaluates the adjoint term H^T f
  double ssq = 0.0;
  chunk_scan<10, false, float, true>(
      pow, scratch, [&](int q) { return xs[q]; },
      [&](int q, float y) {
        const int64_t n = base + q;
        if (n >= a && n < send) ssq = fma((double)y, (double)y, ssq);
        if (grad_row) fb[q] = y;
      });
  PESQ_STAMP(g_phase_front, 2);
  ssq = warp_sum(ssq);
  if (lane == 0) red[warp] = ssq;
  __syncthreads();
  if (tid == 0) {
    double tot = 0.0;
    for (int w = 0; w < kWarps; ++w) tot += red[w];
    p.partial[(int64_t)row * p.nseg + seg] = tot;
  }
  if (grad_row) {
    float* fr = p.fpow + (int64_t)row * n_row;
    for (int i = tid; i < (int)(send - a); i += kThreads) fr[a + i] = fb[kHorizon + i];
    __syncthreads();
    if (has_lo) stage_span(fb, p.src_lo.row(row), base, n_row);
  }
  PESQ_STAMP(g_phase_front, 3);
  // x = xs + fb from here on (fb = 0 for a 16 kHz input)
  if (!has_lo)
    for (int i = tid; i < kSpan; i += kThreads) fb[i] = 0.0f;
  __syncthreads();
  // 2. edge fade (15 samples at each end of the row), in place: the product
  //    of x with the ramp value k/16 is exact in double and splits exactly
  //    into a float hi/lo pair
  if (tid < 30) {
    const int64_t n = tid < 15 ? tid : n_row - 30 + tid;
    const int idx = (int)(n - base);
    // (a sample in both ranges, possible only for rows shorter than 30, is
    // handled once, by the head branch)
    if (n >= 0 && n < n_row && (tid < 15 || n >= 15) && idx >= 0 && idx < kSpan) {
      const double head = n < 15 ? (double)(n + 1) * 0.0625 : 1.0;
      const double tail = n >= n_row - 15 ? (double)(n_row - n) * 0.0625 : 1.0;
      const double v = (((double)xs[idx] + (double)fb[idx]) * head) * tail;
      const float hi = (float)v;
      xs[idx] = hi;
      fb[idx] = (float)(v - (double)hi);
    }
  }
  __syncthreads();
  PESQ_STAMP(g_phase_front, 4);

  // 3. pre-emphasis in double precision, y written as doubles over the
  //    (xs, fb) pair (every thread reads all of its inputs before the scan's
  //    first barrier, so the overlapping in-place writes are safe); the
  //    padding after the row end is 0
  double* yd = reinterpret_cast<double*>(xs);
  const int q_end = (int)min((int64_t)kSpan, n_row - base);
  chunk_scan<2, true, double>(
      pre, reinterpret_cast<double*>(scratch), [&](int q) { return (double)xs[q] + (double)fb[q]; },
      [&](int q, double y) { yd[q] = q < q_end ? y : 0.0; });
  __syncthreads();
  PESQ_STAMP(g_phase_front, 5);

  if constexpr (kSignal) {
    double* yo = p.y64 + (int64_t)row * n_row;
    for (int i = tid; i < (int)(send - a); i += kThreads) yo[a + i] = yd[kHorizon + i];
  } else {
  // 4. frames starting in this segment: window, rfft, power, Bark segment sums
  const int nb = tab->nb;
  const int t0 = seg * p.seg_frames;
  const int t1 = min(t0 + p.seg_frames, p.frames);
  Cx<double>* sh = reinterpret_cast<Cx<double>*>(scratch) + warp * FftLayout<double>::kSlots;
  double* pw = reinterpret_cast<double*>(sh);
  for (int t = t0 + warp; t < t1; t += kWarps) {
    const int off = kHorizon + (t - t0) * kHop;
    Cx<double> v[8], X[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int n = 2 * (lane + 32 * m);
      const double2 y = *reinterpret_cast<const double2*>(yd + off + n);
      const float2 w = *reinterpret_cast<const float2*>(tab->window + n);
      v[m] = mk(y.x * (double)w.x, y.y * (double)w.y);
    }
    warp_rfft512<double>(v, sh, *tw, lane, X);
    if (grad_row) {
      Cx<float>* out = p.spec + ((int64_t)row * p.frames + t) * kBins;
#pragma unroll
      for (int m = 0; m < 8; ++m) out[lane + 32 * m] = mk((float)X[m].x, (float)X[m].y);
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int f = lane + 32 * m;
      pw[f] = f == 0 ? 0.0 : fma(X[m].x, X[m].x, X[m].y * X[m].y);
    }
    __syncwarp();
    float* out = p.bark + ((int64_t)row * p.frames + t) * nb;
    for (int b = lane; b < nb; b += 32) {
      // the band's bins in order, eight loads in flight at a time (the
      // padding past the band's end adds exact zeros)
      const int f1 = tab->band_end[b];
      double acc = 0.0;
#pragma unroll 1
      for (int f = tab->band_start[b]; f < f1; f += 8) {
        double v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = f + i < f1 ? pw[f + i] : 0.0;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc += v[i];
      }
      out[b] = (float)(acc * (double)tab->band_corr[b]);
    }
    __syncwarp();
  }
  }
  PESQ_STAMP(g_phase_front, 6);
  PESQ_CTA_END(g_cta_front);
  PESQ_SPAN_END(g_span_front, 0);
  // the chain forward (launched with programmatic serialisation) may be
  // scheduled once every CTA of this grid is here
  pdl_trigger();
}

}  // namespace

size_t front_smem_bytes() { return (size_t)kFrontSmemBytes; }

cudaError_t configure_front() {
  const cudaError_t e =
      cudaFuncSetAttribute(front_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)front_smem_bytes());
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(front_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)front_smem_bytes());
}

cudaError_t launch_front(const FrontArgs& a, const PowTab& pow, const PreTab64& pre, int rows, cudaStream_t s) {
  const int64_t blocks = (int64_t)rows * a.nseg;
  if (blocks <= 0) return cudaSuccess;
  LaunchShape l((unsigned)blocks, kThreads, front_smem_bytes(), s, false);
  if (a.y64) return cudaLaunchKernelEx(&l.cfg, front_kernel<true>, a, pow, pre);
  return cudaLaunchKernelEx(&l.cfg, front_kernel<false>, a, pow, pre);
}

}  // namespace pesq
