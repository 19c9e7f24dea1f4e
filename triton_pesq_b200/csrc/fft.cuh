// Warp-level 512-point real FFT (and its adjoint) for the PESQ power spectrum.
//
// A 512-point real frame u is packed as z[n] = u[2n] + i u[2n+1] and
// transformed by a 256-point complex DFT, Z = DFT256(z), evaluated by one warp
// as 8 x 8 x 4.  With n = l + 32 m (lane l holds m = 0..7) and
// f = q + 8 (j + 8 k):
//
//   stage 1 (lane l):      B_q(l)   = w256^{l q} sum_m w8^{m q} z[l + 32 m]
//   stage 2 (lane q, r):   D_qr(j)  = w32^{r j}  sum_i w8^{i j} B_q(r + 4 i)
//   stage 3 (lane q, c):   Z[q + 8 j + 64 k] = sum_r w4^{r k} D_qr(j),  j = c, c + 4
//
// where the lanes of stages 2 and 3 are numbered lane = q + 8 r (= q + 8 c).
// Stage 3 then leaves bin q + 8 (c + 4 s) + 64 k = lane + 32 (s + 2 k) in
// register s + 2 k: every lane ends up holding bins lane + 32 m, the same
// distribution the input had.  The two transposes between the stages go
// through shared memory with row pitches chosen so that no access has a bank
// conflict (per quarter warp for the 16-byte complex double, per half warp for
// the 8-byte complex float), and the pairing of bin f with bin 256 - f that
// the real-signal post-processing needs is a warp shuffle from lane 32 - l.
// Twiddles are read from tables laid out in the order the lanes use them (in
// double precision: one entry per stage and lane, the rest by products).
//
// The real spectrum follows from X[f] = E[f] + w512^f O[f] with
// E = (Z[f] + conj Z[256-f]) / 2 and O = -i (Z[f] - conj Z[256-f]) / 2.
//
// The routines are templated on the real type: the forward spectrum of the
// front kernel runs in double precision (weak high bands of a speech signal
// sit 50-60 dB below the frame peak, and the loss gradient is most sensitive
// exactly there), the adjoint of the back kernel in single precision.
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

// Twiddle tables in the order the lanes read them (forward direction).
template <class R>
struct alignas(16) FftTwiddles {
  Cx<R> lane[7][32];    // [q - 1][l] = exp(-2 pi i l q / 256), q = 1..7
  Cx<R> quarter[4][8];  // [r][j]     = exp(-2 pi i r j / 32)
  Cx<R> bin[256];       // [f]        = exp(-2 pi i f / 512)
};

// Shared memory layout of the two transposes, in complex elements:
//   first  B_q(l)  at q * kP1 + l
//   second D_qr(j) at q * kQ2 + r * kR2 + j
// double (16-byte elements, 8 per bank cycle): odd row pitches make the 8
// lanes of a quarter warp (fixed r or c, q = 0..7) hit 8 distinct slots;
// float (8-byte elements, 16 per bank cycle): the 16 lanes of a half warp
// (two values of r or c, q = 0..7) hit 16 distinct slots when the q pitch is
// 2 mod 16 and the r pitch is odd.
template <class R>
struct FftLayout;
template <>
struct FftLayout<double> {
  static constexpr int kP1 = 33, kQ2 = 33, kR2 = 8;
  static constexpr int kSlots = 264;  // per warp, covers 7 * 33 + 31 + 1
};
template <>
struct FftLayout<float> {
  static constexpr int kP1 = 34, kQ2 = 50, kR2 = 9;
  static constexpr int kSlots = 386;  // per warp, covers 7 * 50 + 3 * 9 + 7 + 1, 16-byte multiple
};

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

// Powers w^1 .. w^7 of a twiddle, pw[k - 1] = w^k, by complex products (a few
// ulp in double precision): the double precision transform derives its
// per-lane twiddles this way from one table entry instead of reading seven.
template <class R>
__device__ __forceinline__ void twiddle_powers(Cx<R> w, Cx<R> pw[7]) {
  pw[0] = w;
  pw[1] = c_mul(w, w);
  pw[2] = c_mul(pw[1], w);
  pw[3] = c_mul(pw[1], pw[1]);
  pw[4] = c_mul(pw[3], w);
  pw[5] = c_mul(pw[2], pw[2]);
  pw[6] = c_mul(pw[5], w);
}

// Per-lane twiddles of stage 1 (w256^{l q}) and stage 2 (w32^{r q}), q = 1..7:
// table reads in single precision, products of one table entry in double.
template <class R>
__device__ __forceinline__ Cx<R> stage1_twiddle(const FftTwiddles<R>& tw, const Cx<R>* pw, int q, int lane) {
  if constexpr (sizeof(R) == 8) return pw[q - 1];
  else return tw.lane[q - 1][lane];
}
template <class R>
__device__ __forceinline__ Cx<R> stage2_twiddle(const FftTwiddles<R>& tw, const Cx<R>* pw, int q, int r) {
  if constexpr (sizeof(R) == 8) return pw[q - 1];
  else return tw.quarter[r][q];
}

// Forward 256-point complex DFT of one warp, Z[f] = sum_n z[n] w256^{n f}.
// On entry v[m] = z[lane + 32 m], on exit v[m] = Z[lane + 32 m].  `sh` is the
// warp's FftLayout<R>::kSlots elements of shared memory; the call starts and
// ends on a __syncwarp boundary of its own accesses.
template <class R>
__device__ __forceinline__ void warp_dft256(Cx<R> v[8], Cx<R>* sh, const FftTwiddles<R>& tw, int lane) {
  using L = FftLayout<R>;
  const int q = lane & 7, r = lane >> 3;
  Cx<R> pw[7];
  if constexpr (sizeof(R) == 8) twiddle_powers(tw.lane[0][lane], pw);
  dft8<-1>(v);
#pragma unroll
  for (int k = 1; k < 8; ++k) v[k] = c_mul(v[k], stage1_twiddle(tw, pw, k, lane));
#pragma unroll
  for (int k = 0; k < 8; ++k) sh[k * L::kP1 + lane] = v[k];
  __syncwarp();
  Cx<R> a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = sh[q * L::kP1 + r + 4 * i];
  __syncwarp();
  if constexpr (sizeof(R) == 8) twiddle_powers(tw.quarter[r][1], pw);
  dft8<-1>(a);
#pragma unroll
  for (int j = 1; j < 8; ++j) a[j] = c_mul(a[j], stage2_twiddle(tw, pw, j, r));
#pragma unroll
  for (int j = 0; j < 8; ++j) sh[q * L::kQ2 + r * L::kR2 + j] = a[j];
  __syncwarp();
  const int c = r;
  Cx<R> b0[4], b1[4];
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    b0[rr] = sh[q * L::kQ2 + rr * L::kR2 + c];
    b1[rr] = sh[q * L::kQ2 + rr * L::kR2 + c + 4];
  }
  __syncwarp();
  dft4<-1>(b0[0], b0[1], b0[2], b0[3]);
  dft4<-1>(b1[0], b1[1], b1[2], b1[3]);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = b0[k];
    v[2 * k + 1] = b1[k];
  }
}

// Inverse (unscaled) 256-point DFT, z[n] = sum_f Z[f] w256^{-n f}: the
// transpose of warp_dft256 with conjugated twiddles.  On entry
// v[m] = Z[lane + 32 m], on exit v[m] = z[lane + 32 m].
template <class R>
__device__ __forceinline__ void warp_idft256(Cx<R> v[8], Cx<R>* sh, const FftTwiddles<R>& tw, int lane) {
  using L = FftLayout<R>;
  const int q = lane & 7, r = lane >> 3, c = r;
  Cx<R> b0[4] = {v[0], v[2], v[4], v[6]};
  Cx<R> b1[4] = {v[1], v[3], v[5], v[7]};
  dft4<1>(b0[0], b0[1], b0[2], b0[3]);
  dft4<1>(b1[0], b1[1], b1[2], b1[3]);
#pragma unroll
  for (int rr = 0; rr < 4; ++rr) {
    sh[q * L::kQ2 + rr * L::kR2 + c] = b0[rr];
    sh[q * L::kQ2 + rr * L::kR2 + c + 4] = b1[rr];
  }
  __syncwarp();
  Cx<R> a[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) a[j] = sh[q * L::kQ2 + r * L::kR2 + j];
  __syncwarp();
#pragma unroll
  for (int j = 1; j < 8; ++j) a[j] = c_mul(a[j], c_conj(tw.quarter[r][j]));
  dft8<1>(a);
#pragma unroll
  for (int i = 0; i < 8; ++i) sh[q * L::kP1 + r + 4 * i] = a[i];
  __syncwarp();
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = sh[k * L::kP1 + lane];
  __syncwarp();
#pragma unroll
  for (int k = 1; k < 8; ++k) v[k] = c_mul(v[k], c_conj(tw.lane[k - 1][lane]));
  dft8<1>(v);
}

// For v[m] = Y[lane + 32 m], returns p[m] = Y[(256 - lane - 32 m) mod 256]:
// the partner bin lives in register 7 - m of lane 32 - lane, except on lane 0
// whose bins 32 m pair among themselves.
template <class R>
__device__ __forceinline__ void warp_mirror_bins(const Cx<R> v[8], Cx<R> p[8], int lane) {
  const int src = (32 - lane) & 31;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const R x = __shfl_sync(0xffffffffu, v[7 - m].x, src);
    const R y = __shfl_sync(0xffffffffu, v[7 - m].y, src);
    p[m] = lane == 0 ? v[(8 - m) & 7] : mk(x, y);
  }
}

// Real spectrum of a 512-sample frame given lane l's packed inputs
// v[m] = (u[2n], u[2n+1]), n = l + 32 m.  On exit X[m] holds bin
// f = lane + 32 m (bins 0..255); `sh` is clobbered.
// exp(-2 pi i m / 16), m = 0..7 (cos and sin of multiples of pi / 8)
template <class R>
__device__ __forceinline__ Cx<R> w16(int m) {
  const R c1 = R(0.92387953251128675613), s1 = R(0.38268343236508977173), h = R(0.70710678118654752440);
  switch (m) {
    case 0: return mk(R(1), R(0));
    case 1: return mk(c1, -s1);
    case 2: return mk(h, -h);
    case 3: return mk(s1, -c1);
    case 4: return mk(R(0), R(-1));
    case 5: return mk(-s1, -c1);
    case 6: return mk(-h, -h);
    default: return mk(-c1, -s1);
  }
}

template <class R>
__device__ __forceinline__ void warp_rfft512(Cx<R> v[8], Cx<R>* sh, const FftTwiddles<R>& tw, int lane,
                                             Cx<R> X[8]) {
  warp_dft256(v, sh, tw, lane);
  Cx<R> p[8];
  warp_mirror_bins(v, p, lane);
  const Cx<R> wl = tw.bin[lane];  // w512^lane; w512^(lane + 32 m) = w512^lane w16^m
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const Cx<R> zc = c_conj(p[m]);
    const Cx<R> e = c_scale(c_add(v[m], zc), R(0.5));
    const Cx<R> o = c_scale(c_rot90<-1>(c_sub(v[m], zc)), R(0.5));
    Cx<R> w;
    if constexpr (sizeof(R) == 8) w = m == 0 ? wl : (m == 4 ? c_rot90<-1>(wl) : c_mul(wl, w16<R>(m)));
    else w = tw.bin[lane + 32 * m];
    X[m] = c_add(e, c_mul(w, o));
  }
}

// Adjoint of |rfft|^2 in the sense needed by the backward pass: given
// V[f] = dL/dP_f * X_f for bins f = lane + 32 m (V must be 0 for f = 0),
// returns in g[m] = (g[2n], g[2n+1]), n = lane + 32 m, the values
// g[k] = sum_{f=0}^{511} U_f exp(+2 pi i f k / 512) for k = 0..511, where U is
// the Hermitian extension of V with U_256 = 0.  That is the gradient of
// sum_f dL/dP_f |X_f|^2 w.r.t. the windowed frame.  `sh` is clobbered.
__device__ __forceinline__ void warp_irfft512_adjoint(const Cx<float> V[8], Cx<float>* sh,
                                                      const FftTwiddles<float>& tw, int lane, Cx<float> g[8]) {
  Cx<float> p[8];
  warp_mirror_bins(V, p, lane);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const Cx<float> vc = c_conj(p[m]);
    // Z'[f] = (V_f + conj V_{256-f}) + i conj(w512^f) (V_f - conj V_{256-f})
    const Cx<float> d = c_mul(c_conj(tw.bin[lane + 32 * m]), c_sub(V[m], vc));
    g[m] = c_add(c_add(V[m], vc), c_rot90<1>(d));
  }
  warp_idft256(g, sh, tw, lane);
}

}  // namespace pesq
