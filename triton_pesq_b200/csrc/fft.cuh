// Warp-level 512-point real FFT (and its adjoint) for the PESQ power spectrum.
//
// A 512-point real frame u is packed as z[n] = u[2n] + i u[2n+1] and
// transformed by a 256-point complex DFT, Z = DFT256(z), evaluated by one warp
// as 8 x 8 x 4:
//
//   n = l + 32 m  (lane l holds m = 0..7),  f = q + 8 (j + 8 k)
//   Z[q + 8j + 64k] = sum_r w4^{rk} w32^{rj} sum_i w8^{ij} [w256^{lq} sum_m w8^{mq} z[l+32m]]_{l=r+4i}
//
// with two shared memory exchanges between the radix-8 / radix-8 / radix-4
// passes.  The real spectrum follows from X[f] = E[f] + w512^f O[f] with
// E = (Z[f] + conj Z[256-f]) / 2 and O = -i (Z[f] - conj Z[256-f]) / 2.
//
// The routines are templated on the real type: the forward spectrum of the
// front kernel runs in double precision (weak high bands of a speech signal
// sit 50-60 dB below the frame peak, and the loss gradient is most sensitive
// exactly there), the adjoint of the back kernel in single precision.
// Twiddles come from host float64 tables: w256[k] = exp(-2 pi i k / 256),
// w512[k] = exp(-2 pi i k / 512).
#pragma once

#include "common.cuh"

namespace pesq {

template <class R>
struct __align__(2 * sizeof(R)) Cx {
  R x, y;
};

template <class R>
__device__ __forceinline__ Cx<R> mk(R a, R b) {
  Cx<R> c;
  c.x = a;
  c.y = b;
  return c;
}
template <class R>
__device__ __forceinline__ Cx<R> c_add(Cx<R> a, Cx<R> b) { return mk(a.x + b.x, a.y + b.y); }
template <class R>
__device__ __forceinline__ Cx<R> c_sub(Cx<R> a, Cx<R> b) { return mk(a.x - b.x, a.y - b.y); }
template <class R>
__device__ __forceinline__ Cx<R> c_mul(Cx<R> a, Cx<R> b) {
  return mk<R>(fma(a.x, b.x, -a.y * b.y), fma(a.x, b.y, a.y * b.x));
}
template <class R>
__device__ __forceinline__ Cx<R> c_conj(Cx<R> a) { return mk(a.x, -a.y); }
template <class R>
__device__ __forceinline__ Cx<R> c_scale(Cx<R> a, R s) { return mk(a.x * s, a.y * s); }

// multiply by exp(DIR * i pi / 2), i.e. -i for the forward (DIR = -1) transform
template <int DIR, class R>
__device__ __forceinline__ Cx<R> c_rot90(Cx<R> a) {
  return DIR < 0 ? mk(a.y, -a.x) : mk(-a.y, a.x);
}

// per-warp shared scratch of the FFT, in complex elements
constexpr int kFftRow = 36;  // padded row of the first exchange (8 x 32 used)
constexpr int kFftScratch = 8 * kFftRow;

// twiddle exp(DIR * 2 pi i k / 256) from the forward table
template <int DIR, class R>
__device__ __forceinline__ Cx<R> twiddle256(const Cx<R>* tw, int k) {
  const Cx<R> w = tw[k & 255];
  return DIR < 0 ? w : c_conj(w);
}

template <int DIR, class R>
__device__ __forceinline__ void dft4(Cx<R>& a0, Cx<R>& a1, Cx<R>& a2, Cx<R>& a3) {
  const Cx<R> t0 = c_add(a0, a2), t1 = c_sub(a0, a2);
  const Cx<R> t2 = c_add(a1, a3), t3 = c_rot90<DIR>(c_sub(a1, a3));
  a0 = c_add(t0, t2);
  a2 = c_sub(t0, t2);
  a1 = c_add(t1, t3);
  a3 = c_sub(t1, t3);
}

// in-place 8-point DFT, natural order in and out
template <int DIR, class R>
__device__ __forceinline__ void dft8(Cx<R> v[8]) {
  const R kS = R(0.70710678118654752440);
  Cx<R> e0 = v[0], e1 = v[2], e2 = v[4], e3 = v[6];
  Cx<R> o0 = v[1], o1 = v[3], o2 = v[5], o3 = v[7];
  dft4<DIR>(e0, e1, e2, e3);
  dft4<DIR>(o0, o1, o2, o3);
  o1 = c_scale(c_add(o1, c_rot90<DIR>(o1)), kS);
  o2 = c_rot90<DIR>(o2);
  o3 = c_scale(c_sub(c_rot90<DIR>(o3), o3), kS);
  v[0] = c_add(e0, o0);
  v[4] = c_sub(e0, o0);
  v[1] = c_add(e1, o1);
  v[5] = c_sub(e1, o1);
  v[2] = c_add(e2, o2);
  v[6] = c_sub(e2, o2);
  v[3] = c_add(e3, o3);
  v[7] = c_sub(e3, o3);
}

// 256-point complex DFT of one warp.  On entry lane l holds z[l + 32 m] in
// v[m]; on exit sh[0..255] holds the transform in natural order (the call ends
// with __syncwarp).  sh is the warp's kFftScratch elements of shared memory.
template <int DIR, class R>
__device__ __forceinline__ void warp_fft256(Cx<R> v[8], Cx<R>* sh, const Cx<R>* tw256, int lane) {
  dft8<DIR>(v);
#pragma unroll
  for (int q = 1; q < 8; ++q) v[q] = c_mul(v[q], twiddle256<DIR>(tw256, lane * q));
#pragma unroll
  for (int q = 0; q < 8; ++q) sh[q * kFftRow + lane] = v[q];
  __syncwarp();

  const int q = lane >> 2, r = lane & 3;
  Cx<R> a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = sh[q * kFftRow + r + 4 * i];
  __syncwarp();
  dft8<DIR>(a);
#pragma unroll
  for (int j = 1; j < 8; ++j) a[j] = c_mul(a[j], twiddle256<DIR>(tw256, 8 * r * j));
#pragma unroll
  for (int j = 0; j < 8; ++j) sh[q * kFftRow + r * 8 + j] = a[j];
  __syncwarp();

  const int c = r;
  Cx<R> b0[4], b1[4];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    b0[rr] = sh[q * kFftRow + rr * 8 + c];
    b1[rr] = sh[q * kFftRow + rr * 8 + c + 4];
  }
  __syncwarp();
  dft4<DIR>(b0[0], b0[1], b0[2], b0[3]);
  dft4<DIR>(b1[0], b1[1], b1[2], b1[3]);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    sh[q + 8 * c + 64 * k] = b0[k];
    sh[q + 8 * (c + 4) + 64 * k] = b1[k];
  }
  __syncwarp();
}

// Real spectrum of a 512-sample frame given lane l's packed inputs
// v[m] = (u[2n], u[2n+1]), n = l + 32 m.  On exit X[m] holds bin
// f = lane + 32 m (bins 0..255); `sh` is clobbered.
template <class R>
__device__ __forceinline__ void warp_rfft512(Cx<R> v[8], Cx<R>* sh, const Cx<R>* tw256, const Cx<R>* tw512,
                                             int lane, Cx<R> X[8]) {
  warp_fft256<-1>(v, sh, tw256, lane);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int f = lane + 32 * m;
    const Cx<R> zf = sh[f];
    const Cx<R> zc = c_conj(sh[(256 - f) & 255]);
    const Cx<R> e = c_scale(c_add(zf, zc), R(0.5));
    const Cx<R> o = c_scale(c_rot90<-1>(c_sub(zf, zc)), R(0.5));
    X[m] = c_add(e, c_mul(tw512[f], o));
  }
  __syncwarp();
}

// Adjoint of |rfft|^2 in the sense needed by the backward pass: given
// V[f] = dL/dP_f * X_f for bins f = lane + 32 m (V must be 0 for f = 0), writes
// g[k] = sum_{f=0}^{511} U_f exp(+2 pi i f k / 512) for k = 0..511 into `out`
// (shared, 8-byte aligned), where U is the Hermitian extension of V with
// U_256 = 0.  That is the gradient of sum_f dL/dP_f |X_f|^2 w.r.t. the
// windowed frame.  `out` may alias `sh`.
__device__ __forceinline__ void warp_irfft512_adjoint(const Cx<float> V[8], Cx<float>* sh,
                                                      const Cx<float>* tw256, const Cx<float>* tw512, int lane,
                                                      float* out) {
#pragma unroll
  for (int m = 0; m < 8; ++m) sh[lane + 32 * m] = V[m];
  __syncwarp();
  Cx<float> v[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int f = lane + 32 * m;
    const Cx<float> vf = V[m];
    const Cx<float> vc = c_conj(sh[(256 - f) & 255]);
    // Z'[f] = (V_f + conj V_{256-f}) + i conj(w512^f) (V_f - conj V_{256-f})
    const Cx<float> d = c_mul(c_conj(tw512[f]), c_sub(vf, vc));
    v[m] = c_add(c_add(vf, vc), c_rot90<1>(d));
  }
  __syncwarp();
  warp_fft256<1>(v, sh, tw256, lane);
  Cx<float> o[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) o[m] = sh[lane + 32 * m];
  __syncwarp();
#pragma unroll
  for (int m = 0; m < 8; ++m) reinterpret_cast<Cx<float>*>(out)[lane + 32 * m] = o[m];
  __syncwarp();
}

}  // namespace pesq
