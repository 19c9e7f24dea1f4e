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
// both with an in-place radix-2 transform of n_fft complex points in the
// warp's slice of shared memory (inputs stored at bit-reversed positions,
// log2 n_fft butterfly stages separated by __syncwarp, twiddles from a float64
// table).  The back kernel overlap-adds the frame gradients by a gather in
// frame order (no atomics, bitwise reproducible).  The default geometry keeps
// the fused warp FFTs of the front and back kernels.
#include "kernels.cuh"

namespace pesq {

namespace {

// warps per CTA: up to 8, as many n_fft-point frames as fit in 192 KB
__host__ __device__ constexpr int gen_warps(int nfft, int elem_bytes) {
  const int w = (192 * 1024) / (nfft * elem_bytes);
  return w < 1 ? 1 : (w > kGenThreads / 32 ? kGenThreads / 32 : w);
}

// In-place decimation-in-time FFT of 2^log2n points (input in bit-reversed
// order, output in natural order), twiddle w^k = exp(-2 pi i k / 2^log2n).
template <class R>
__device__ __forceinline__ void warp_fft(Cx<R>* z, int log2n, const Cx<double>* tw, int lane) {
  const int half_n = 1 << (log2n - 1);
  for (int s = 0; s < log2n; ++s) {
    const int half = 1 << s;
    const int shift = log2n - 1 - s;  // butterfly k of this stage uses w^(k 2^shift)
    for (int i = lane; i < half_n; i += 32) {
      const int k = i & (half - 1);
      const int j = ((i >> s) << (s + 1)) + k;
      const double2 wd = __ldg(reinterpret_cast<const double2*>(tw) + (k << shift));
      const Cx<R> w = mk((R)wd.x, (R)wd.y);
      const Cx<R> a = z[j];
      const Cx<R> b = c_mul(z[j + half], w);
      z[j] = c_add(a, b);
      z[j + half] = c_sub(a, b);
    }
    __syncwarp();
  }
}

__device__ __forceinline__ int bit_reverse(int k, int log2n) { return (int)(__brev((unsigned)k) >> (32 - log2n)); }

__global__ void __launch_bounds__(kGenThreads) stft_kernel(const __grid_constant__ SpecArgs p) {
  extern __shared__ __align__(16) double smem_d[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int64_t item = (int64_t)blockIdx.x * warps + warp;
  if (item >= (int64_t)p.rows * p.frames) return;  // whole warps only: no CTA barrier below
  const int row = p.row_begin + (int)(item / p.frames);
  const int t = (int)(item - (int64_t)(row - p.row_begin) * p.frames);
  const int nfft = p.g.nfft, log2n = p.g.log2n, nfreq = p.g.nfreq;
  Cx<double>* z = reinterpret_cast<Cx<double>*>(smem_d) + (size_t)warp * nfft;

  const double* yr = p.y + (int64_t)row * p.n;
  const int64_t start = (int64_t)t * p.g.hop;
  for (int k = lane; k < nfft; k += 32) {
    const int64_t m = start + k;
    const double v = m < p.n ? __ldg(yr + m) * (double)__ldg(p.g.window + k) : 0.0;
    z[bit_reverse(k, log2n)] = mk(v, 0.0);
  }
  __syncwarp();
  warp_fft<double>(z, log2n, p.g.tw, lane);

  if (row >= p.spec_begin && row < p.spec_end) {
    Cx<float>* out = p.spec + ((int64_t)row * p.frames + t) * nfreq;
    for (int f = lane; f < nfreq; f += 32) out[f] = mk((float)z[f].x, (float)z[f].y);
  }
  // power in place (the DC bin is dropped), then the Bark segment sums
  for (int f = lane; f < nfreq; f += 32) {
    const Cx<double> X = z[f];
    z[f].x = f == 0 ? 0.0 : fma(X.x, X.x, X.y * X.y);
  }
  __syncwarp();
  const DevTables* tab = p.tab;
  const int nb = tab->nb;
  float* bark = p.bark + ((int64_t)row * p.frames + t) * nb;
  for (int b = lane; b < nb; b += 32) {
    double acc = 0.0;
    for (int f = tab->band_start[b]; f < tab->band_end[b]; ++f) acc += z[f].x;
    bark[b] = (float)(acc * (double)tab->band_corr[b]);
  }
}

__global__ void __launch_bounds__(kGenThreads) istft_kernel(const __grid_constant__ SpecArgs p) {
  extern __shared__ __align__(16) double smem_d[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int64_t item = (int64_t)blockIdx.x * warps + warp;
  if (item >= (int64_t)p.rows * p.frames) return;
  const int local = (int)(item / p.frames);
  const int row = p.row_begin + local;
  const int t = (int)(item - (int64_t)local * p.frames);
  const int nfft = p.g.nfft, log2n = p.g.log2n, nfreq = p.g.nfreq;
  Cx<float>* z = reinterpret_cast<Cx<float>*>(smem_d) + (size_t)warp * nfft;

  const DevTables* tab = p.tab;
  const Cx<float>* X = p.spec + ((int64_t)row * p.frames + t) * nfreq;
  const float* g = p.g_bark + ((int64_t)row * p.frames + t) * tab->nb;
  for (int f = lane; f < nfft; f += 32) {
    Cx<float> v = mk(0.0f, 0.0f);
    const int b = f < nfreq ? __ldg(p.g.bin_band + f) : -1;
    if (b >= 0) {
      const float scale = g[b] * tab->band_corr[b];
      const Cx<float> x = X[f];
      v = mk(x.x * scale, -x.y * scale);  // conj(V_f)
    }
    z[bit_reverse(f, log2n)] = v;
  }
  __syncwarp();
  warp_fft<float>(z, log2n, p.g.tw, lane);
  float* out = p.frame_grad + ((int64_t)local * p.frames + t) * nfft;
  for (int k = lane; k < nfft; k += 32) out[k] = 2.0f * z[k].x * __ldg(p.g.window + k);
}

size_t stft_smem(int nfft) { return (size_t)gen_warps(nfft, 16) * nfft * 16; }
size_t istft_smem(int nfft) { return (size_t)gen_warps(nfft, 8) * nfft * 8; }

template <class Kernel>
cudaError_t launch_frames(Kernel kernel, const SpecArgs& a, int elem_bytes, cudaStream_t s) {
  const int64_t items = (int64_t)a.rows * a.frames;
  if (items <= 0) return cudaSuccess;
  const int warps = gen_warps(a.g.nfft, elem_bytes);
  const int64_t blocks = (items + warps - 1) / warps;
  if (blocks > 0x7fffffff) return cudaErrorInvalidConfiguration;
  LaunchShape l((unsigned)blocks, (unsigned)(warps * 32), (size_t)warps * a.g.nfft * elem_bytes, s, false);
  return cudaLaunchKernelEx(&l.cfg, kernel, a);
}

}  // namespace

cudaError_t configure_spectrum() {
  cudaError_t e = cudaFuncSetAttribute(stft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)stft_smem(kGenMaxFft));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(istft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)istft_smem(kGenMaxFft));
}

cudaError_t launch_stft(const SpecArgs& a, cudaStream_t s) {
  return launch_frames(stft_kernel, a, 16, s);
}

cudaError_t launch_istft(const SpecArgs& a, cudaStream_t s) {
  return launch_frames(istft_kernel, a, 8, s);
}

}  // namespace pesq
