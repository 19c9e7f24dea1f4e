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

// Shared-memory geometry of a front CTA of NT threads: NT chunks of kChunk
// samples, NT / 32 warps.  The 512-thread CTA holds the forward twiddles in
// shared memory too (one CTA per SM); the 256-thread one, which runs two
// CTAs per SM, reads them through L1.
template <int NT>
struct FrontGeom {
  static constexpr int kSpanT = NT * kChunk;
  static constexpr int kWarpsT = NT / 32;
  static constexpr bool kTwInSmem = NT == kThreads;
  static constexpr int kFftFloats = kWarpsT * FftLayout<double>::kSlots * 4;
  static constexpr int kScratchFloats =
      kFftFloats > scan_scratch_floats<10, float, NT>() ? kFftFloats : scan_scratch_floats<10, float, NT>();
  static constexpr int kSmemBytes = 2 * kSpanT * 4 + kScratchFloats * 4 + (int)sizeof(DevTables) +
                                    (kTwInSmem ? (int)sizeof(DevTwiddle64) : 0) + kWarpsT * 8 + 16;
  static_assert((2 * kSpanT * 4 + kScratchFloats * 4) % 16 == 0, "16-byte aligned tables in shared memory");
};
static_assert(sizeof(DevTables) % 16 == 0 && sizeof(DevTwiddle64) % 16 == 0, "bulk copies of the tables");
static_assert(2 * (FrontGeom<kThreads / 2>::kSmemBytes + 1024) <= 228 * 1024, "two half-size CTAs per SM");

// kSignal: general frame geometry, y is written to p.y64 and the frames are
// left to the spectrum kernel (spectrum.cu)
template <bool kSignal, int NT>
__global__ void __launch_bounds__(NT, kThreads / NT)
    front_kernel(const __grid_constant__ FrontArgs p, const __grid_constant__ PowTab pow,
                 const __grid_constant__ PreTab64 pre) {
  using G = FrontGeom<NT>;
  constexpr int kSpan = G::kSpanT;    // (shadow the 512-thread constants)
  constexpr int kWarps = G::kWarpsT;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                 // kSpan: input (hi part)
  float* fb = xs + kSpan;           // kSpan: [f = H x,] low part of a resampled x
                                    // (xs, fb) then hold y as kSpan doubles
  float* scratch = fb + kSpan;      // scan scratch, later the per-warp FFT scratch
  DevTables* tab = reinterpret_cast<DevTables*>(scratch + G::kScratchFloats);
  DevTwiddle64* tw_s = reinterpret_cast<DevTwiddle64*>(tab + 1);
  const DevTwiddle64* tw = G::kTwInSmem ? tw_s : p.tw64;
  double* red = reinterpret_cast<double*>(reinterpret_cast<char*>(tab + 1) + (G::kTwInSmem ? sizeof(DevTwiddle64) : 0));
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
    const uint32_t tw_bytes = G::kTwInSmem ? (uint32_t)sizeof(DevTwiddle64) : 0u;
    mbar_arrive_expect_tx(bar, (uint32_t)sizeof(DevTables) + tw_bytes + span_bytes);
    bulk_g2s(tab, p.tab, (uint32_t)sizeof(DevTables), bar);
    if (G::kTwInSmem) bulk_g2s(tw_s, p.tw64, tw_bytes, bar);
    if (bulk_span) bulk_g2s(xs + (lo - base), xf + lo, span_bytes, bar);
  }
  if (bulk_span) {
    for (int i = tid; i < kSpan; i += NT) {
      const int64_t q = base + i;
      if (q < lo || q >= lo + cnt4) xs[i] = q >= lo && q < hi ? __ldg(xf + q) : 0.0f;
    }
  } else {
    stage_span_any<NT>(xs, xr, base, n_row, p.src.type);
  }
  // The low part of a resampled input (x = hi + lo) joins the pre-emphasis.
  // On gradient rows fb first holds f = H x (below), the low part only after.
  const bool has_lo = p.src_lo.ref != nullptr;
  if (has_lo && !grad_row) stage_span<NT>(fb, p.src_lo.row(row), base, n_row);
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
  chunk_scan<10, false, float, true, NT, true>(
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
    for (int i = tid; i < (int)(send - a); i += NT) fr[a + i] = fb[kHorizon + i];
    __syncthreads();
    if (has_lo) stage_span<NT>(fb, p.src_lo.row(row), base, n_row);
  }
  PESQ_STAMP(g_phase_front, 3);
  // x = xs + fb from here on (fb = 0 for a 16 kHz input)
  if (!has_lo)
    for (int i = tid; i < kSpan; i += NT) fb[i] = 0.0f;
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
  chunk_scan<2, true, double, false, NT, true>(
      pre, reinterpret_cast<double*>(scratch), [&](int q) { return (double)xs[q] + (double)fb[q]; },
      [&](int q, double y) { yd[q] = q < q_end ? y : 0.0; });
  __syncthreads();
  PESQ_STAMP(g_phase_front, 5);

  if constexpr (kSignal) {
    double* yo = p.y64 + (int64_t)row * n_row;
    for (int i = tid; i < (int)(send - a); i += NT) yo[a + i] = yd[kHorizon + i];
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

size_t front_smem_bytes(int threads) {
  return (size_t)(threads == kThreads ? FrontGeom<kThreads>::kSmemBytes : FrontGeom<kThreads / 2>::kSmemBytes);
}

cudaError_t configure_front() {
  cudaError_t e = cudaFuncSetAttribute(front_kernel<false, kThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)front_smem_bytes(kThreads));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(front_kernel<true, kThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)front_smem_bytes(kThreads));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(front_kernel<false, kThreads / 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)front_smem_bytes(kThreads / 2));
}

cudaError_t launch_front(const FrontArgs& a, const PowTab& pow, const PreTab64& pre, int rows, cudaStream_t s) {
  const int64_t blocks = (int64_t)rows * a.nseg;
  if (blocks <= 0) return cudaSuccess;
  if (a.threads == kThreads / 2 && !a.y64) {
    LaunchShape l((unsigned)blocks, kThreads / 2, front_smem_bytes(kThreads / 2), s, false);
    return cudaLaunchKernelEx(&l.cfg, front_kernel<false, kThreads / 2>, a, pow, pre);
  }
  LaunchShape l((unsigned)blocks, kThreads, front_smem_bytes(kThreads), s, false);
  if (a.y64) return cudaLaunchKernelEx(&l.cfg, front_kernel<true, kThreads>, a, pow, pre);
  return cudaLaunchKernelEx(&l.cfg, front_kernel<false, kThreads>, a, pow, pre);
}

}  // namespace pesq
