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
// All twiddles come from float64-accurate tables (host float64 rounded to
// float32): w256[k] = exp(-2 pi i k / 256), w512[k] = exp(-2 pi i k / 512).
#pragma once

#include "common.cuh"

namespace pesq {

// per-warp shared scratch of the FFT, in float2
constexpr int kFftRow = 36;  // padded row of the first exchange (8 x 32 used)
constexpr int kFftScratch = 8 * kFftRow;

__device__ __forceinline__ float2 c_add(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 c_sub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 c_mul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
__device__ __forceinline__ float2 c_conj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 c_scale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }

// multiply by exp(DIR * i pi / 2), i.e. -i for the forward (DIR = -1) transform
template <int DIR>
__device__ __forceinline__ float2 c_rot90(float2 a) {
  return DIR < 0 ? make_float2(a.y, -a.x) : make_float2(-a.y, a.x);
}

// twiddle exp(DIR * 2 pi i k / 256) from the forward table
template <int DIR>
__device__ __forceinline__ float2 twiddle256(const float2* tw, int k) {
  const float2 w = tw[k & 255];
  return DIR < 0 ? w : c_conj(w);
}

template <int DIR>
__device__ __forceinline__ void dft4(float2& a0, float2& a1, float2& a2, float2& a3) {
  const float2 t0 = c_add(a0, a2), t1 = c_sub(a0, a2);
  const float2 t2 = c_add(a1, a3), t3 = c_rot90<DIR>(c_sub(a1, a3));
  a0 = c_add(t0, t2);
  a2 = c_sub(t0, t2);
  a1 = c_add(t1, t3);
  a3 = c_sub(t1, t3);
}

// in-place 8-point DFT, natural order in and out
template <int DIR>
__device__ __forceinline__ void dft8(float2 v[8]) {
  constexpr float kS = 0.70710678118654752440f;
  float2 e0 = v[0], e1 = v[2], e2 = v[4], e3 = v[6];
  float2 o0 = v[1], o1 = v[3], o2 = v[5], o3 = v[7];
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
// with __syncwarp).  sh is the warp's kFftScratch float2 of shared memory.
template <int DIR>
__device__ __forceinline__ void warp_fft256(float2 v[8], float2* sh, const float2* tw256, int lane) {
  dft8<DIR>(v);
#pragma unroll
  for (int q = 1; q < 8; ++q) v[q] = c_mul(v[q], twiddle256<DIR>(tw256, lane * q));
#pragma unroll
  for (int q = 0; q < 8; ++q) sh[q * kFftRow + lane] = v[q];
  __syncwarp();

  const int q = lane >> 2, r = lane & 3;
  float2 a[8];
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
  float2 b0[4], b1[4];
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

// Real spectrum of a windowed 512-sample frame.  `frame` and `win` are shared
// memory (frame 8-byte aligned).  On exit X[m] holds bin f = lane + 32 m of
// the DFT of frame * win (bins 0..255); `sh` is clobbered.
__device__ __forceinline__ void warp_rfft512(const float* frame, const float* win, float2* sh,
                                             const float2* tw256, const float2* tw512, int lane,
                                             float2 X[8]) {
  float2 v[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int n = lane + 32 * m;
    const float2 s = reinterpret_cast<const float2*>(frame)[n];
    const float2 w = reinterpret_cast<const float2*>(win)[n];
    v[m] = make_float2(s.x * w.x, s.y * w.y);
  }
  warp_fft256<-1>(v, sh, tw256, lane);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int f = lane + 32 * m;
    const float2 zf = sh[f];
    const float2 zc = c_conj(sh[(256 - f) & 255]);
    const float2 e = c_scale(c_add(zf, zc), 0.5f);
    const float2 o = c_scale(c_rot90<-1>(c_sub(zf, zc)), 0.5f);
    X[m] = c_add(e, c_mul(tw512[f], o));
  }
  __syncwarp();
}

// Adjoint of |rfft|^2 in the sense needed by the backward pass: given
// V[f] = dL/dP_f * X_f for bins f = lane + 32 m (V must be 0 for f = 0), writes
// g[k] = sum_{f=0}^{511} U_f exp(+2 pi i f k / 512) for k = 0..511 into `out`
// (shared, 8-byte aligned), where U is the Hermitian extension of V with
// U_256 = 0.  That is the gradient of sum_f dL/dP_f |X_f|^2 w.r.t. the
// windowed frame.
__device__ __forceinline__ void warp_irfft512_adjoint(const float2 V[8], float2* sh, const float2* tw256,
                                                      const float2* tw512, int lane, float* out) {
#pragma unroll
  for (int m = 0; m < 8; ++m) sh[lane + 32 * m] = V[m];
  __syncwarp();
  float2 v[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int f = lane + 32 * m;
    const float2 vf = V[m];
    const float2 vc = c_conj(sh[(256 - f) & 255]);
    // Z'[f] = (V_f + conj V_{256-f}) + i conj(w512^f) (V_f - conj V_{256-f})
    const float2 d = c_mul(c_conj(tw512[f]), c_sub(vf, vc));
    v[m] = c_add(c_add(vf, vc), c_rot90<1>(d));
  }
  __syncwarp();
  warp_fft256<1>(v, sh, tw256, lane);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int n = lane + 32 * m;
    reinterpret_cast<float2*>(out)[n] = sh[n];
  }
  __syncwarp();
}

}  // namespace pesq
