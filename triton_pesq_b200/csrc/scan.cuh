// Chunked parallel scan of a causal LTI filter over one CTA span.
//
// The filter is a state space recursion s[n+1] = A s[n] + B x[n],
// y[n] = C s[n] + D x[n] (a series of balanced second order sections, built on
// the host in float64, see triton_pesq_b200/tables.py).  A CTA covers
// kSpan = kThreads * kChunk consecutive samples; thread c owns chunk c.
//
//   1. every thread forms the zero-state end state of its chunk,
//      a_c = sum_k A^(L-1-k) B x[k]  (table W)
//   2. a Kogge-Stone scan over the chunks with the doubling steps
//      M_i = A^(L 2^i) turns a_c into E_c = sum_{j < 32} A^(L j) a_{c-j}: the
//      end state of chunk c with everything older than kHorizon samples
//      dropped.  The dropped term is bounded by ||A^kHorizon|| (< 1e-11,
//      checked on the host), far below float32 rounding, so E_{c-1} is the
//      state chunk c starts in for every c >= kHorizonChunks.
//   3. each chunk evaluates its outputs from that state: either the impulse
//      response convolution plus the state read-out,
//      y[t] = sum_{k<=t} h[t-k] x[k] + C A^t S   (kRerun == false), or by
//      re-running the recursion from S (kRerun == true, cheaper for P <= 4).
//
// The first kHorizonChunks chunks of the span are the warm-up: their inputs
// must be the true signal (zeros before the start of a row, which reproduces
// the zero initial state exactly) but their outputs are not exact and are
// never used.  The same routine evaluates the adjoint (time reversed) filter
// when the caller's load/store map logical positions backwards in time.
#pragma once

#include "common.cuh"

namespace pesq {

// Tables of the scan in the arithmetic type R (float or double).
template <int P, class R = float>
struct ScanTab {
  R h[kChunk];         // impulse response h[0..L-1]
  R G[kChunk][P];      // C A^t
  R W[kChunk][P];      // A^(L-1-k) B
  R M[kLevels][P][P];  // A^(L * 2^i)
  R A[P][P];           // one step, for the re-run form
  R B[P];
  R C[P];
  R D;
};

// Shared memory floats the scan needs as scratch (CTAs of NT threads).
template <int P, class R = float, int NT = kThreads>
__host__ __device__ constexpr int scan_scratch_floats() {
  return P * NT * (int)(sizeof(R) / sizeof(float));
}

// `load(p)` returns the input at logical position p (0 <= p < NT * kChunk)
// and `store(p, y)` consumes the output there.  `es` is scan scratch of
// scan_scratch_floats<P, R, NT>() floats.  Must be called by all NT threads
// of the CTA (a span of NT chunks; the horizon is kHorizonChunks chunks
// whatever NT).
// kBlockLower: A (hence every doubling matrix M) is block lower triangular in
// 2 x 2 blocks, as for a series of second order sections; the structurally
// zero entries above the block diagonal are skipped (the host checks them).
// kSkipWarmup: the caller uses no output of the warm-up chunks (the first
// kHorizonChunks, warp 0), which then skip step 3.
template <int P, bool kRerun, class R, bool kBlockLower = false, int NT = kThreads, bool kSkipWarmup = false,
          class Load, class Store>
__device__ __forceinline__ void chunk_scan(const ScanTab<P, R>& tab, R* es, Load&& load, Store&& store) {
  const int c = threadIdx.x;
  const int p0 = c * kChunk;

  R x[kChunk];
#pragma unroll
  for (int k = 0; k < kChunk; ++k) x[k] = load(p0 + k);

  // 1. zero-state end state of the chunk
  R e[P];
#pragma unroll
  for (int j = 0; j < P; ++j) {
    R acc = R(0);
#pragma unroll
    for (int k = 0; k < kChunk; ++k) acc = fma(tab.W[k][j], x[k], acc);
    e[j] = acc;
  }

  // 2. Kogge-Stone over the chunks of the span
#pragma unroll
  for (int j = 0; j < P; ++j) es[j * NT + c] = e[j];
  __syncthreads();
#pragma unroll
  for (int lv = 0; lv < kLevels; ++lv) {
    const int d = 1 << lv;
    R prev[P];
#pragma unroll
    for (int j = 0; j < P; ++j) prev[j] = c >= d ? es[j * NT + c - d] : R(0);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < P; ++i) {
      R acc = e[i];
#pragma unroll
      for (int j = 0; j < P; ++j) {
        if (kBlockLower && (j >> 1) > (i >> 1)) continue;
        acc = fma(tab.M[lv][i][j], prev[j], acc);
      }
      e[i] = acc;
    }
#pragma unroll
    for (int j = 0; j < P; ++j) es[j * NT + c] = e[j];
    __syncthreads();
  }

  R s[P];
#pragma unroll
  for (int j = 0; j < P; ++j) s[j] = c >= 1 ? es[j * NT + c - 1] : R(0);
  // the scratch is free again once every thread holds its start state
  __syncthreads();

  // 3. outputs of the chunk
  static_assert(kHorizonChunks == 32, "the warm-up chunks are warp 0");
  if (kSkipWarmup && c < kHorizonChunks) {
    // warm-up chunk: no output needed
  } else if constexpr (kRerun) {
#pragma unroll
    for (int t = 0; t < kChunk; ++t) {
      R y = tab.D * x[t];
#pragma unroll
      for (int j = 0; j < P; ++j) y = fma(tab.C[j], s[j], y);
      R nxt[P];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        R acc = tab.B[i] * x[t];
#pragma unroll
        for (int j = 0; j < P; ++j) acc = fma(tab.A[i][j], s[j], acc);
        nxt[i] = acc;
      }
#pragma unroll
      for (int i = 0; i < P; ++i) s[i] = nxt[i];
      store(p0 + t, y);
    }
  } else {
#pragma unroll
    for (int t = 0; t < kChunk; ++t) {
      R y = R(0);
#pragma unroll
      for (int j = 0; j < P; ++j) y = fma(tab.G[t][j], s[j], y);
#pragma unroll
      for (int k = 0; k <= t; ++k) y = fma(tab.h[t - k], x[k], y);
      store(p0 + t, y);
    }
  }
}

}  // namespace pesq
