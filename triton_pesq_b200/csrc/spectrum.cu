// Power spectrum -> Bark bands and its adjoint for frame geometries other than
// n_fft 512 / hop 256 (PesqLoss(..., win_length, n_fft, hop_length) with any
// power-of-two n_fft in [32, 4096] and any hop; torch_pesq/loss.py:78-90,
// torch_pesq/bark.py:131-173, torch_pesq/triton_ops/spectral.py:138-202).
//
// The front kernel writes the pre-emphasised rows y (float64); here one warp
// evaluates one frame t of one row:
//
//   forward   u_k = w_k y[t hop + k]  (0 past the row end: the N % 256 padding)
//             X_f = sum_k u_k exp(-2 pi i f k / n_fft),  f < n_fft / 2      float64
//             B_b = corr_b sum_{f in band b, f >= 1} |X_f|^2               -> Bark
//             X_f as float (rows that need a gradient)                      -> spectrum
//   adjoint   V_f = corr_b dL/dB_b X_f
//             dL/du_k = 2 Re sum_f conj(V_f) exp(-2 pi i f k / n_fft)        float32
//             G_t[k] = w_k dL/du_k                                          -> frame gradients
//
// n_fft 512 (the PESQ frame with another hop or window) uses the register /
// shared-memory transposed 512-point real transform of the fused path
// (fft.cuh).  Every other n_fft packs the real frame into n_fft / 2 complex
// points (even samples real, odd imaginary) and runs an in-place radix-2
// transform of those in the warp's slice of shared memory, instantiated per
// log2 n_fft so that its loops unroll (inputs stored at bit-reversed
// positions, butterfly stages separated by __syncwarp, twiddles from a table
// the CTA stages in shared memory); the even / odd split of the result gives
// the real spectrum, and its adjoint the inverse.  The back kernel overlap-adds
// the frame gradients by a gather in frame order (no atomics, bitwise
// reproducible).
#include "kernels.cuh"

namespace pesq {

namespace {

constexpr int kSmemBudget = 226 * 1024;

// warps per CTA of the generic transform: up to 8, as many frames (n_fft / 2
// packed complex points each) as fit next to the CTA's two twiddle tables of
// n_fft / 2 entries (the real split's, and the butterfly stages')
__host__ __device__ constexpr int gen_warps(int nfft, int elem_bytes) {
  const int w = (kSmemBudget - 2 * (nfft / 2) * elem_bytes) / ((nfft / 2) * elem_bytes);
  return w < 1 ? 1 : (w > kGenThreads / 32 ? kGenThreads / 32 : w);
}
__host__ __device__ constexpr size_t gen_smem(int nfft, int elem_bytes) {
  return (size_t)(gen_warps(nfft, elem_bytes) + 2) * (nfft / 2) * elem_bytes;
}

// The 512-point path: per warp the transposes' scratch, per CTA the twiddles.
constexpr int kWarps512 = kGenThreads / 32;
constexpr size_t kStft512Smem = sizeof(FftTwiddles<double>) + (size_t)kWarps512 * FftLayout<double>::kSlots * 16;
constexpr size_t kIstft512Smem = sizeof(FftTwiddles<float>) + (size_t)kWarps512 * FftLayout<float>::kSlots * 8;

__device__ __forceinline__ int bit_reverse(int k, int log2n) { return (int)(__brev((unsigned)k) >> (32 - log2n)); }

// CTA copy of `bytes` (a multiple of 16) global -> shared
__device__ __forceinline__ void stage_table(void* dst, const void* src, int bytes) {
  for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x)
    reinterpret_cast<float4*>(dst)[i] = __ldg(reinterpret_cast<const float4*>(src) + i);
}

// In-place decimation-in-time FFT of M = 2^LOG2M points (input in
// bit-reversed order, output in natural order).  The twiddles of each
// butterfly stage lie contiguously, ts[half - 1 + k] = exp(-2 pi i k / (2 half)),
// k < half, so that the lanes of a stage read consecutive entries (or one).
template <int LOG2M, class R>
__device__ __forceinline__ void warp_fft(Cx<R>* z, const Cx<R>* ts, int lane) {
  constexpr int kHalfM = 1 << (LOG2M - 1);
#pragma unroll
  for (int s = 0; s < LOG2M; ++s) {
    const int half = 1 << s;
#pragma unroll 4
    for (int i = lane; i < kHalfM; i += 32) {
      const int k = i & (half - 1);
      const int j = ((i >> s) << (s + 1)) + k;
      const Cx<R> a = z[j];
      const Cx<R> b = c_mul(z[j + half], ts[half - 1 + k]);
      z[j] = c_add(a, b);
      z[j + half] = c_sub(a, b);
    }
    __syncwarp();
  }
}

// Bin of a real n_fft-point frame from the n_fft/2-point transform Z of its
// packed samples z[n] = u[2n] + i u[2n+1]: with Zc = conj Z[n_fft/2 - f],
// X_f = (Z_f + Zc) / 2 + w^f (-i) (Z_f - Zc) / 2, w = exp(-2 pi i / n_fft).
__device__ __forceinline__ Cx<double> real_bin(Cx<double> zf, Cx<double> zc, Cx<double> w) {
  const Cx<double> e = c_scale(c_add(zf, zc), 0.5);
  const Cx<double> o = c_scale(c_rot90<-1>(c_sub(zf, zc)), 0.5);
  return c_add(e, c_mul(w, o));
}

// Stage twiddles of an M = 2^LOG2M point transform from the n_fft = 2M
// table tw[k] = exp(-2 pi i k / n_fft): ts[half - 1 + k] = tw[k << (LOG2M - s)]
template <int LOG2M, class R, class Src>
__device__ __forceinline__ void stage_twiddles(Cx<R>* ts, const Src* tw) {
  constexpr int kM = 1 << LOG2M;
  for (int idx = threadIdx.x; idx < kM - 1; idx += blockDim.x) {
    const int s = 31 - __clz(idx + 1), half = 1 << s;
    const int k = idx + 1 - half;
    const Src w = tw[k << (LOG2M - s)];
    ts[idx] = mk((R)w.x, (R)w.y);
  }
}

struct Frame {
  int row, t;
  bool valid;
};

__device__ __forceinline__ Frame frame_of(const SpecArgs& p, int warp) {
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
  Frame f;
  f.valid = item < (int64_t)p.rows * p.frames;
  const int local = f.valid ? (int)(item / p.frames) : 0;
  f.row = p.row_begin + local;
  f.t = f.valid ? (int)(item - (int64_t)local * p.frames) : 0;
  return f;
}

// Bark segment sums of the power spectrum pw[f * STRIDE] (bin 0 already dropped)
template <int STRIDE>
__device__ __forceinline__ void bark_sums(const SpecArgs& p, const double* pw, int row, int t, int lane) {
  const DevTables* tab = p.tab;
  const int nb = tab->nb;
  float* bark = p.bark + ((int64_t)row * p.frames + t) * nb;
  for (int b = lane; b < nb; b += 32) {
    const int f0 = tab->band_start[b], f1 = tab->band_end[b];
    double acc = 0.0;
    for (int f = f0; f < f1; ++f) acc += pw[f * STRIDE];
    bark[b] = (float)(acc * (double)tab->band_corr[b]);
  }
}

template <int LOG2N>
__global__ void __launch_bounds__(kGenThreads) stft_kernel(const __grid_constant__ SpecArgs p) {
  constexpr int kLog2M = LOG2N - 1, kM = 1 << kLog2M;  // packed complex points = bins
  extern __shared__ __align__(16) double smem_d[];
  Cx<double>* tw = reinterpret_cast<Cx<double>*>(smem_d);  // exp(-2 pi i k / n_fft), k < kM
  Cx<double>* ts = tw + kM;                                   // the butterfly stages' twiddles
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  stage_table(tw, p.g.tw, kM * 16);
  stage_twiddles<kLog2M, double>(ts, p.g.tw);
  __syncthreads();
  const Frame fr = frame_of(p, warp);
  if (!fr.valid) return;  // whole warps only: no CTA barrier below
  Cx<double>* z = ts + kM + (size_t)warp * kM;

  const double* yr = p.y + (int64_t)fr.row * p.n;
  const int64_t start = (int64_t)fr.t * p.g.hop;
#pragma unroll 4
  for (int k = lane; k < kM; k += 32) {
    const int64_t m = start + 2 * k;
    const double y0 = m < p.n ? __ldg(yr + m) : 0.0;
    const double y1 = m + 1 < p.n ? __ldg(yr + m + 1) : 0.0;
    const float2 w = __ldg(reinterpret_cast<const float2*>(p.g.window + 2 * k));
    z[bit_reverse(k, kLog2M)] = mk(y0 * (double)w.x, y1 * (double)w.y);
  }
  __syncwarp();
  warp_fft<kLog2M, double>(z, ts, lane);

  // bins f and kM - f from the same two values (one lane owns both slots):
  // the spectrum, then the power in place of the real part (bin 0 dropped)
  const bool save = fr.row >= p.spec_begin && fr.row < p.spec_end;
  Cx<float>* out = p.spec + ((int64_t)fr.row * p.frames + fr.t) * kM;
  for (int f = lane; f <= kM / 2; f += 32) {
    const int g = (kM - f) & (kM - 1);
    const Cx<double> zf = z[f], zg = z[g];
    const Cx<double> xf = real_bin(zf, c_conj(zg), tw[f]);
    const Cx<double> xg = real_bin(zg, c_conj(zf), tw[g]);
    if (save) {
      out[f] = mk((float)xf.x, (float)xf.y);
      if (g != f) out[g] = mk((float)xg.x, (float)xg.y);
    }
    z[f].x = f == 0 ? 0.0 : fma(xf.x, xf.x, xf.y * xf.y);
    if (g != f) z[g].x = fma(xg.x, xg.x, xg.y * xg.y);
  }
  __syncwarp();
  bark_sums<2>(p, reinterpret_cast<const double*>(z), fr.row, fr.t, lane);
}

template <int LOG2N>
__global__ void __launch_bounds__(kGenThreads) istft_kernel(const __grid_constant__ SpecArgs p) {
  constexpr int kLog2M = LOG2N - 1, kM = 1 << kLog2M;
  extern __shared__ __align__(16) double smem_d[];
  Cx<float>* tw = reinterpret_cast<Cx<float>*>(smem_d);
  Cx<float>* ts = tw + kM;  // the butterfly stages' twiddles
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int k = threadIdx.x; k < kM; k += blockDim.x) {
    const double2 w = __ldg(reinterpret_cast<const double2*>(p.g.tw) + k);
    tw[k] = mk((float)w.x, (float)w.y);
  }
  stage_twiddles<kLog2M, float>(ts, reinterpret_cast<const double2*>(p.g.tw));
  __syncthreads();
  const Frame fr = frame_of(p, warp);
  if (!fr.valid) return;
  const int local = fr.row - p.row_begin;
  Cx<float>* z = ts + kM + (size_t)warp * kM;

  // V_f = corr_b dL/dB_b X_f (0 for bin 0 and bins outside every band);
  // the frame gradient g_k = sum_f U_f exp(+2 pi i f k / n_fft) over the
  // Hermitian extension U of V is, packed as g_2n + i g_2n+1, the inverse
  // kM-point transform of Z'_f = (V_f + conj V_{kM-f}) + i conj(w^f) (V_f - conj V_{kM-f})
  // (V_kM = 0), evaluated as conj(DFT(conj Z')).
  const DevTables* tab = p.tab;
  const Cx<float>* X = p.spec + ((int64_t)fr.row * p.frames + fr.t) * kM;
  const float* gb = p.g_bark + ((int64_t)fr.row * p.frames + fr.t) * tab->nb;
  auto vbin = [&](int f) {
    const int b = f < kM ? __ldg(p.g.bin_band + f) : -1;
    return b >= 0 ? c_scale(X[f], gb[b] * tab->band_corr[b]) : mk(0.0f, 0.0f);
  };
#pragma unroll 4
  for (int f = lane; f < kM; f += 32) {
    const Cx<float> v = vbin(f);
    const Cx<float> vc = c_conj(vbin(kM - f));
    const Cx<float> d = c_mul(c_conj(tw[f]), c_sub(v, vc));
    z[bit_reverse(f, kLog2M)] = c_conj(c_add(c_add(v, vc), c_rot90<1>(d)));
  }
  __syncwarp();
  warp_fft<kLog2M, float>(z, ts, lane);
  float* out = p.frame_grad + ((int64_t)local * p.frames + fr.t) * (2 * kM);
#pragma unroll 4
  for (int n = lane; n < kM; n += 32) {
    const Cx<float> r = z[n];
    const float2 w = __ldg(reinterpret_cast<const float2*>(p.g.window + 2 * n));
    *reinterpret_cast<float2*>(out + 2 * n) = make_float2(w.x * r.x, -w.y * r.y);
  }
}

// n_fft 512: the transposed warp transforms of fft.cuh
__global__ void __launch_bounds__(kGenThreads) stft512_kernel(const __grid_constant__ SpecArgs p) {
  extern __shared__ __align__(16) double smem_d[];
  FftTwiddles<double>* tw = reinterpret_cast<FftTwiddles<double>*>(smem_d);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  stage_table(tw, p.tw512, (int)sizeof(FftTwiddles<double>));
  __syncthreads();
  const Frame fr = frame_of(p, warp);
  if (!fr.valid) return;
  Cx<double>* sh = reinterpret_cast<Cx<double>*>(tw + 1) + (size_t)warp * FftLayout<double>::kSlots;

  const double* yr = p.y + (int64_t)fr.row * p.n;
  const int64_t start = (int64_t)fr.t * p.g.hop;
  Cx<double> v[8], X[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int k = 2 * (lane + 32 * m);
    const int64_t s0 = start + k;
    const double y0 = s0 < p.n ? __ldg(yr + s0) : 0.0;
    const double y1 = s0 + 1 < p.n ? __ldg(yr + s0 + 1) : 0.0;
    const float2 w = __ldg(reinterpret_cast<const float2*>(p.g.window + k));
    v[m] = mk(y0 * (double)w.x, y1 * (double)w.y);
  }
  warp_rfft512<double>(v, sh, *tw, lane, X);
  if (fr.row >= p.spec_begin && fr.row < p.spec_end) {
    Cx<float>* out = p.spec + ((int64_t)fr.row * p.frames + fr.t) * kBins;
#pragma unroll
    for (int m = 0; m < 8; ++m) out[lane + 32 * m] = mk((float)X[m].x, (float)X[m].y);
  }
  double* pw = reinterpret_cast<double*>(sh);
  __syncwarp();
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int f = lane + 32 * m;
    pw[f] = f == 0 ? 0.0 : fma(X[m].x, X[m].x, X[m].y * X[m].y);
  }
  __syncwarp();
  bark_sums<1>(p, pw, fr.row, fr.t, lane);
}

__global__ void __launch_bounds__(kGenThreads) istft512_kernel(const __grid_constant__ SpecArgs p) {
  extern __shared__ __align__(16) double smem_d[];
  FftTwiddles<float>* tw = reinterpret_cast<FftTwiddles<float>*>(smem_d);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  stage_table(tw, &p.tab->fft, (int)sizeof(FftTwiddles<float>));
  __syncthreads();
  const Frame fr = frame_of(p, warp);
  if (!fr.valid) return;
  const int local = fr.row - p.row_begin;
  Cx<float>* sh = reinterpret_cast<Cx<float>*>(tw + 1) + (size_t)warp * FftLayout<float>::kSlots;

  const DevTables* tab = p.tab;
  const Cx<float>* X = p.spec + ((int64_t)fr.row * p.frames + fr.t) * kBins;
  const float* g = p.g_bark + ((int64_t)fr.row * p.frames + fr.t) * tab->nb;
  Cx<float> V[8], gr[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int f = lane + 32 * m;
    const int b = __ldg(p.g.bin_band + f);
    V[m] = b >= 0 ? c_scale(X[f], g[b] * tab->band_corr[b]) : mk(0.0f, 0.0f);
  }
  warp_irfft512_adjoint(V, sh, *tw, lane, gr);
  float* out = p.frame_grad + ((int64_t)local * p.frames + fr.t) * 512;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int k = 2 * (lane + 32 * m);
    const float2 w = __ldg(reinterpret_cast<const float2*>(p.g.window + k));
    *reinterpret_cast<float2*>(out + k) = make_float2(w.x * gr[m].x, w.y * gr[m].y);
  }
}

template <class Kernel>
cudaError_t launch_frames(Kernel kernel, const SpecArgs& a, int warps, size_t smem, cudaStream_t s) {
  const int64_t items = (int64_t)a.rows * a.frames;
  if (items <= 0) return cudaSuccess;
  const int64_t blocks = (items + warps - 1) / warps;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  LaunchShape l((unsigned)blocks, (unsigned)(warps * 32), smem, s, false);
  return cudaLaunchKernelEx(&l.cfg, kernel, a);
}

template <int LOG2N>
cudaError_t configure_log2() {
  cudaError_t e = cudaFuncSetAttribute(stft_kernel<LOG2N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)gen_smem(1 << LOG2N, 16));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(istft_kernel<LOG2N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)gen_smem(1 << LOG2N, 8));
}

template <int LOG2N>
cudaError_t launch_log2(const SpecArgs& a, bool adjoint, cudaStream_t s) {
  constexpr int kN = 1 << LOG2N;
  if (adjoint) return launch_frames(istft_kernel<LOG2N>, a, gen_warps(kN, 8), gen_smem(kN, 8), s);
  return launch_frames(stft_kernel<LOG2N>, a, gen_warps(kN, 16), gen_smem(kN, 16), s);
}

cudaError_t launch_spectrum(const SpecArgs& a, bool adjoint, cudaStream_t s) {
  switch (a.g.log2n) {
    case 5: return launch_log2<5>(a, adjoint, s);
    case 6: return launch_log2<6>(a, adjoint, s);
    case 7: return launch_log2<7>(a, adjoint, s);
    case 8: return launch_log2<8>(a, adjoint, s);
    case 9:
      if (adjoint) return launch_frames(istft512_kernel, a, kWarps512, kIstft512Smem, s);
      return launch_frames(stft512_kernel, a, kWarps512, kStft512Smem, s);
    case 10: return launch_log2<10>(a, adjoint, s);
    case 11: return launch_log2<11>(a, adjoint, s);
    case 12: return launch_log2<12>(a, adjoint, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t configure_spectrum() {
  cudaError_t e = cudaSuccess;
  if ((e = configure_log2<5>()) != cudaSuccess || (e = configure_log2<6>()) != cudaSuccess ||
      (e = configure_log2<7>()) != cudaSuccess || (e = configure_log2<8>()) != cudaSuccess ||
      (e = configure_log2<10>()) != cudaSuccess || (e = configure_log2<11>()) != cudaSuccess ||
      (e = configure_log2<12>()) != cudaSuccess)
    return e;
  e = cudaFuncSetAttribute(stft512_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStft512Smem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(istft512_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kIstft512Smem);
}

cudaError_t launch_stft(const SpecArgs& a, cudaStream_t s) { return launch_spectrum(a, false, s); }

cudaError_t launch_istft(const SpecArgs& a, cudaStream_t s) { return launch_spectrum(a, true, s); }

}  // namespace pesq
