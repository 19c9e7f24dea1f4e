// Standalone causal IIR filter: an exact chunked scan over whole rows.
//
// The filter is a state space recursion s[n+1] = A s[n] + B x[n],
// y[n] = C s[n] + D x[n] (realisation chosen on the host in float64,
// triton_pesq_b200/iir_design.py), applied with zero initial state to every
// row of a [rows, n] float32 array -- lfilter(x, a, b, clamp=False), as the
// reference's TritonIIR (torch_pesq/triton_ops/iir.py:1266-1482).  With
// `reverse` the rows are read and written back to front, which evaluates the
// adjoint (the vector-Jacobian product) of the filter (iir.py:1232-1258).
//
// One CTA of kThreads threads filters one tile.  Thread c owns a chunk of kL
// consecutive samples:
//
//   1. e_c = sum_k A^(kL-1-k) B x[k], the chunk's end state from zero (table W),
//      and (impulse form) the chunk's zero-state outputs sum_k h[t-k] x[k];
//   2. a segmented Kogge-Stone scan over the 32 chunks of a warp with the
//      doubling steps M_i = A^(kL 2^i) (warp shuffles), restarted at every
//      row start ("head");
//   3. every warp forms its own start state from the totals of the warps
//      before it and the warp powers A^(32 kL k), back to the last head or
//      to the tile's start state S (no serial chain across the warps);
//   4. each chunk's start state is the warp-exclusive prefix plus
//      A^(kL lane) times its warp's start state (lane table, shared memory);
//   5. outputs: zero-state part + C A^t s (impulse form) or the recursion
//      re-run from s (re-run form); staged through shared memory and stored
//      coalesced.
//
// Tile geometry.  Rows of at most kThreads chunks are packed whole, several to
// a tile (segments of cpr chunks, a head at each segment start): nothing
// crosses a tile.  Longer rows of a filter whose state dies out within one
// warp's span (||A^kOverlap|| < 1e-11, checked on the host, as for the loss
// path's level-alignment scan) run overlapped tiles: tile k stages the kOverlap
// samples before its kTile - kOverlap outputs as well and starts from zero
// state there (warp 0's chunks are the warm-up and store nothing), so no tile
// waits for another.  Otherwise the tiles of kTile samples are
// chained by a decoupled look-back (single pass, 8 bytes of HBM traffic per
// sample): a CTA takes its tile from a ticket counter (so every tile it waits
// for belongs to a CTA that is already running), publishes its zero-start
// aggregate, sums the aggregates of its predecessors with the powers
// A^(k kTile) (float64) back to the first one that has published its
// inclusive end state, and publishes its own inclusive state.  Published
// states are self-validating tagged words (no memory fences, see publish).  Nothing is
// truncated: the result is exact for any stable or unstable filter.  Every
// wait is bounded (Args::spin_limit polls, kSpinLimit unless the caller set
// another with pesq_iir_set_spin_limit); a wait that gives up records an error
// in the filter's error word and treats the predecessor as zero.
//
// Every warp-collective operation (shuffle, ballot) is executed by all 32
// lanes of the warp: a lane that skips one leaves the others waiting forever.
#pragma once

#include "common.cuh"

namespace pesq {
namespace iir {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kL = 33;                  // samples per thread chunk (coprime with the banks)
constexpr int kLevels = 5;              // warp scan levels
constexpr int kTile = kThreads * kL;    // 8448 samples per tile
constexpr int kLook = 32;               // predecessors per look-back window (a warp)
constexpr int kFar = 256;               // predecessors the look-back reaches (8 windows)
constexpr int kMaxStates = 24;
constexpr unsigned kSpinLimit = 1u << 21;
constexpr int kOverlap = 32 * kL;       // warm-up of an overlapped tile: warp 0's chunks (1056 samples)
static_assert(kOverlap % 4 == 0 && (kTile - kOverlap) % 4 == 0, "overlapped tiles store in 16-byte pieces");

// Per-filter constants in float32, passed as a kernel parameter (constant
// bank operands of the FMAs).
template <int P>
struct Tab {
  float h[kL];              // impulse response h[0..kL-1]
  float G[kL][P];           // C A^t
  float W[kL][P];           // A^(kL-1-k) B
  float M[kLevels][P][P];   // A^(kL 2^i)
  float A[P][P];
  float B[P];
  float C[P];
  float D;
};

// Lane table pitch: A^(kL l) for lane l at l * lane_pitch(P) floats; odd, so
// the per-lane reads of a warp never share a bank.
__host__ __device__ constexpr int lane_pitch(int P) { return P * P + 1; }
__host__ __device__ constexpr int lane_floats(int P) { return 32 * lane_pitch(P); }
// Warp powers A^(32 kL k), k = 0..kWarps.
__host__ __device__ constexpr int wpow_floats(int P) { return (kWarps + 1) * P * P; }

struct Args {
  const float* x;
  int64_t ld_x;
  float* y;
  int64_t ld_y;
  int64_t rows;
  int64_t n;
  int reverse;
  int cpr;                 // chunks per row (rows packed whole), else kThreads
  int rows_per_tile;       // whole rows per tile (1 for chained rows)
  int seg;                 // samples per segment: cpr * kL, or kTile
  int64_t tiles_per_row;   // > 1: the tiles of a row are chained
  int64_t tiles;
  const float* lanes;      // [32][lane_pitch]  A^(kL l)
  const float* wpow;       // [kWarps + 1][P][P] A^(32 kL k)
  const double* look;      // [kFar + 1][P][P] A^(k kTile)
  uint32_t* ticket;        // tile counter (zero before the launch)
  unsigned long long* slots;  // [tiles][2][P][2]: aggregate / inclusive state, zero before the launch
  uint32_t* err;
  uint32_t spin_limit;     // polls a look-back wait makes before it gives up (normally kSpinLimit)
  int overlap;             // > 0: overlapped tiles (below) instead of chained ones
};

constexpr int kNearPowers = 4;  // A^(k kTile), k < 4, staged for the look-back
__host__ __device__ constexpr size_t smem_bytes(int P) {
  return (size_t)kTile * 4 + (size_t)kNearPowers * P * P * 8 + (size_t)lane_floats(P) * 4 +
         (size_t)wpow_floats(P) * 4 + (size_t)kWarps * P * 4 + (size_t)P * 4 + 16;
}

#ifdef PESQ_PHASE_PROBE
// [tile][phase] globaltimer of the first 1024 tiles of a launch (probe builds
// only; one copy per translation unit, read by the unit's own reader)
static __device__ unsigned long long g_iir_probe[1024 * 8];
#define PESQ_IIR_STAMP(tile, i)                                                      \
  do {                                                                               \
    if (threadIdx.x == 0 && (tile) < 1024) g_iir_probe[(tile) * 8 + (i)] = pesq_globaltimer(); \
  } while (0)
#else
#define PESQ_IIR_STAMP(tile, i) \
  do {                          \
  } while (0)
#endif

template <int P, bool kLower>
__device__ __forceinline__ bool skip(int i, int j) {
  return kLower && (j >> 1) > (i >> 1);
}

// Published states need no fences: component i of a tile's aggregate (slot
// 0) or inclusive end state (slot 1) is the float pair (hi, lo) with
// hi + lo = the float64 value to ~48 bits, each in its own 64-bit word with
// the tag 1 in its upper half.  A naturally aligned 64-bit access is
// single-copy atomic, so a reader that sees every word of a slot tagged has
// the whole state, whatever order the words became visible in.
__device__ __forceinline__ unsigned long long slot_word(float v) {
  return (1ull << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Warp 0: lanes i < P publish component i (lane i holds it).
template <int P>
__device__ __forceinline__ void publish(const Args& a, int64_t tile, int slot, double mine, int lane) {
  if (lane < P) {
    unsigned long long* dst = a.slots + ((tile * 2 + slot) * P + lane) * 2;
    const float hi = (float)mine;
    st_relaxed64(dst, slot_word(hi));
    st_relaxed64(dst + 1, slot_word((float)(mine - (double)hi)));
  }
}

// Reads slot `slot` of tile `t`: true (and its P components in v) when every
// word is tagged.
template <int P>
__device__ __forceinline__ bool read_slot(const Args& a, int64_t t, int slot, double (&v)[P]) {
  const unsigned long long* src = a.slots + (t * 2 + slot) * P * 2;
  bool ok = true;
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const unsigned long long hi = ld_relaxed64(src + 2 * j), lo = ld_relaxed64(src + 2 * j + 1);
    ok = ok && (hi >> 32) == 1u && (lo >> 32) == 1u;
    v[j] = (double)__uint_as_float((unsigned)hi) + (double)__uint_as_float((unsigned)lo);
  }
  return ok;
}

// Warp 0: start state of tile `tile` (its index in the row is tin >= 1), from
// the published states of its predecessors; lane i returns component i.
// Windows of 32 predecessors, lane k of a window the one k + done back: the
// aggregates before the first inclusive state, and that state, each times
// A^(distance kTile) from the table (k < kNearPowers from shared memory,
// `near`).  The last lane of the last window (256 back) waits for an
// inclusive state, so at most 8 windows are read.
template <int P>
__device__ double lookback(const Args& a, int64_t tile, int64_t tin, const double* near, int lane) {
  double S[P];
#pragma unroll
  for (int j = 0; j < P; ++j) S[j] = 0.0;
  for (int64_t done = 0;; done += kLook) {
    const int64_t k = done + lane;
    const bool valid = k < tin;
    const int64_t pred = tile - 1 - k;
    const uint32_t need = (done + kLook >= kFar && lane == kLook - 1) ? 2u : 1u;
    // st: 0 nothing yet, 1 aggregate, 2 inclusive (v holds it), 3 gave up
    uint32_t st = 0;
    double v[P];
#pragma unroll
    for (int j = 0; j < P; ++j) v[j] = 0.0;
    if (valid) {
      unsigned it = 0;
      for (;;) {
        if (read_slot<P>(a, pred, 1, v)) {
          st = 2u;
          break;
        }
        if (need == 1u && read_slot<P>(a, pred, 0, v)) {
          st = 1u;
          break;
        }
        if (++it > a.spin_limit) {
          atomicOr(a.err, 1u);
          st = 3u;  // give up: the predecessor counts as a zero inclusive state
          break;
        }
        __nanosleep(64);
      }
    }
    const unsigned incl = __ballot_sync(0xffffffffu, valid && st >= 2u);
    const int m = incl ? __ffs(incl) - 1 : kLook;
    const bool take = valid && lane <= m && st != 3u;
    // (a lane before m holds its predecessor's aggregate: that one had no
    // inclusive state when it was read)
    // c = A^(k kTile) v (the identity for k = 0)
    double c[P];
    if (!take) {
#pragma unroll
      for (int i = 0; i < P; ++i) c[i] = 0.0;
    } else if (k == 0) {
#pragma unroll
      for (int i = 0; i < P; ++i) c[i] = v[i];
    } else {
      const bool staged = k < kNearPowers;
      const double* L = staged ? near + (size_t)k * P * P : a.look + (size_t)k * P * P;
#pragma unroll
      for (int i = 0; i < P; ++i) {
        double acc = 0.0;
        if (staged) {
#pragma unroll
          for (int j = 0; j < P; ++j) acc = fma(L[i * P + j], v[j], acc);
        } else {
#pragma unroll
          for (int j = 0; j < P; ++j) acc = fma(__ldg(L + i * P + j), v[j], acc);
        }
        c[i] = acc;
      }
    }
#pragma unroll
    for (int i = 0; i < P; ++i) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) c[i] += __shfl_xor_sync(0xffffffffu, c[i], off);
      S[i] += c[i];
    }
    if (m < kLook || done + kLook >= tin) break;
  }
  double mine = 0.0;
#pragma unroll
  for (int j = 0; j < P; ++j)
    if (j == lane) mine = S[j];
  return mine;
}

// Lane i < P: component i of sum_{v = v0}^{v1 - 1} A^(32 kL (v1 - 1 - v)) T_v
// (warp totals T in shared memory).
template <int P, bool kLower>
__device__ __forceinline__ float warp_sum(const float* wpow, const float* tot, int v0, int v1, int i) {
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // independent chains, one per warp mod 4
  for (int v = v0; v < v1; ++v) {
    const float* Wm = wpow + (v1 - 1 - v) * P * P + i * P;
    const float* T = tot + v * P;
    float part = 0.0f;
#pragma unroll
    for (int j = 0; j < P; ++j)
      if (!skip<P, kLower>(i, j)) part = fmaf(Wm[j], T[j], part);
    acc[v & 3] += part;
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// kRev: the rows are filtered back to front (a.reverse; a compile-time
// direction turns every staged-tile index into a constant offset)
template <int P, bool kLower, bool kRerun, bool kRev>
__global__ void __launch_bounds__(kThreads, P <= 2 ? 4 : (P <= 10 ? 3 : 1)) scan_kernel(const __grid_constant__ Args a,
                                                                        const __grid_constant__ Tab<P> tab) {
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;                              // kTile samples
  double* near = reinterpret_cast<double*>(xs + kTile);  // A^(k kTile), k < kNearPowers
  float* lanes = reinterpret_cast<float*>(near + kNearPowers * P * P);  // lane table
  float* wpow = lanes + lane_floats(P);          // warp powers
  float* tot = wpow + wpow_floats(P);            // [kWarps][P] warp totals
  float* sin_s = tot + kWarps * P;               // [P] start state of the tile
  __shared__ int64_t s_tile;
  __shared__ int s_whead[kWarps];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool chained = a.tiles_per_row > 1;
  const bool ovl = chained && a.overlap > 0;  // overlapped tiles: no look-back
  const bool looks = chained && !ovl;
  if (tid == 0) s_tile = looks ? (int64_t)atomicAdd(a.ticket, 1u) : (int64_t)blockIdx.x;
  copy_async<kThreads>(lanes, a.lanes, lane_floats(P) * 4);
  copy_async<kThreads>(wpow, a.wpow, wpow_floats(P) * 4);
  if (looks) copy_async<kThreads>(near, a.look, kNearPowers * P * P * 8);
  __syncthreads();

  // tile geometry: rows [row0, row0 + nrows), memory span [m0, m0 + seg) of each
  const int64_t tile = s_tile;
  PESQ_IIR_STAMP(tile, 0);
  const int seg = a.seg;
  int64_t row0, tin, m0;
  int nrows;
  if (ovl) {
    // outputs [tin E, (tin + 1) E) after a warm-up of the kOverlap samples
    // before them (E = kTile - kOverlap); reversed, the warm-up lies above
    const int64_t E = kTile - kOverlap;
    row0 = tile / a.tiles_per_row;
    tin = tile - row0 * a.tiles_per_row;
    nrows = 1;
    m0 = kRev ? a.n - (tin + 1) * E : tin * E - kOverlap;
  } else if (chained) {
    row0 = tile / a.tiles_per_row;
    tin = tile - row0 * a.tiles_per_row;
    nrows = 1;
    m0 = kRev ? a.n - (tin + 1) * (int64_t)kTile : tin * (int64_t)kTile;
  } else {
    row0 = tile * a.rows_per_tile;
    tin = 0;
    nrows = (int)min((int64_t)a.rows_per_tile, a.rows - row0);
    m0 = kRev ? a.n - seg : 0;
  }
  // a whole, 16-byte aligned tile of one row moves in 16-byte pieces
  const float* xrow = a.x + row0 * a.ld_x;
  float* yrow = a.y + row0 * a.ld_y;
  const bool full = chained && m0 >= 0 && m0 + kTile <= a.n;
  // staged samples [qa, qb) of the tile are outputs (all but the warm-up)
  const int qa = ovl && !kRev ? kOverlap : 0;
  const int qb = ovl && kRev ? kTile - kOverlap : kTile;
  const bool vec_in = full && ((reinterpret_cast<uintptr_t>(xrow + m0) & 15) == 0);
  const bool vec_out = full && ((reinterpret_cast<uintptr_t>(yrow + m0 + qa) & 15) == 0);

  // stage the tile in memory order (zeros outside the rows)
  if (vec_in) {
    for (int i = tid; i < kTile / 4; i += kThreads) cp_async16(xs + 4 * i, xrow + m0 + 4 * i);
  } else if (chained) {
#pragma unroll 11
    for (int k = 0; k < kL; ++k) {
      const int q = tid + k * kThreads;
      const int64_t m = m0 + q;
      const bool valid = m >= 0 && m < a.n;
      cp_async4_zfill(xs + q, valid ? xrow + m : a.x, valid);
    }
  } else {
    // packed rows: warp w stages rows w, w + kWarps, ... (segments of seg
    // samples, the row's n samples at the front or, reversed, at the back)
    const int n = (int)a.n;
    const int lead = kRev ? seg - n : 0;
    for (int rr = warp; rr < a.rows_per_tile; rr += kWarps) {
      float* dst = xs + rr * seg;
      if (rr < nrows) {
        const float* src = xrow + rr * a.ld_x;
        for (int i = lane; i < seg; i += 32) {
          const int m = i - lead;
          const bool valid = m >= 0 && m < n;
          cp_async4_zfill(dst + i, valid ? src + m : a.x, valid);
        }
      } else {
        for (int i = lane; i < seg; i += 32) dst[i] = 0.0f;
      }
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();
  PESQ_IIR_STAMP(tile, 1);

  // this thread's chunk: segment r, chunk lc of the segment; its sample t
  // sits at xs[base + dir * t]
  const int r = chained ? 0 : tid / a.cpr;
  const int lc = chained ? tid : tid - r * a.cpr;
  const bool used = chained || r < nrows;
  const bool head = ovl ? tid == 0 : chained ? (tin == 0 && tid == 0) : (!used || lc == 0);
  constexpr int dir = kRev ? -1 : 1;
  const int base = kRev ? r * seg + seg - 1 - lc * kL : r * seg + lc * kL;

  // (chunks past the last packed row hold no data and store nothing; their
  // shared memory index could lie past the tile)
  float x[kL];
#pragma unroll
  for (int k = 0; k < kL; ++k) x[k] = used ? xs[base + dir * k] : 0.0f;

  // 1. end state from zero, and the zero-state outputs (in place, last first).
  // Every thread reads and writes only its own chunk's slots of the staged
  // tile, so the zero-state outputs (impulse form) or the inputs (re-run form)
  // wait there, not in registers, until the chunk's start state is known.
  float e[P];
#pragma unroll
  for (int j = 0; j < P; ++j) {
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < kL; ++k) acc = fmaf(tab.W[k][j], x[k], acc);
    e[j] = acc;
  }
  if constexpr (!kRerun) {
#pragma unroll
    for (int t = kL - 1; t >= 0; --t) {
      float acc = 0.0f;
#pragma unroll
      for (int k = 0; k <= t; ++k) acc = fmaf(tab.h[t - k], x[k], acc);
      x[t] = acc;
    }
    if (used) {
#pragma unroll
      for (int t = 0; t < kL; ++t) xs[base + dir * t] = x[t];
    }
  }

  // 2. segmented scan over the warp's chunks
  bool f = head;
#pragma unroll
  for (int lv = 0; lv < kLevels; ++lv) {
    const int d = 1 << lv;
    float pv[P];
#pragma unroll
    for (int j = 0; j < P; ++j) pv[j] = __shfl_up_sync(0xffffffffu, e[j], d);
    const bool pf = __shfl_up_sync(0xffffffffu, (int)f, d) != 0;
    if (lane >= d) {
      if (!f) {
        float ne[P];
#pragma unroll
        for (int i = 0; i < P; ++i) {
          float acc = e[i];
#pragma unroll
          for (int j = 0; j < P; ++j)
            if (!skip<P, kLower>(i, j)) acc = fmaf(tab.M[lv][i][j], pv[j], acc);
          ne[i] = acc;
        }
#pragma unroll
        for (int i = 0; i < P; ++i) e[i] = ne[i];
      }
      f = f || pf;
    }
  }
  // exclusive prefix within the warp, and whether a head precedes this lane
  float ex[P];
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const float v = __shfl_up_sync(0xffffffffu, e[j], 1);
    ex[j] = lane == 0 ? 0.0f : v;
  }
  const int fup = __shfl_up_sync(0xffffffffu, (int)f, 1);
  const bool fex = lane != 0 && fup != 0;
  if (lane == 31) {
#pragma unroll
    for (int j = 0; j < P; ++j) tot[warp * P + j] = e[j];
    s_whead[warp] = f;
  }
  __syncthreads();
  PESQ_IIR_STAMP(tile, 2);

  // 3. start state of this warp: back to the last warp with a head, or to
  //    the tile's start state (lane i < P holds component i)
  int h = -1;
  for (int v = 0; v < warp; ++v)
    if (s_whead[v]) h = v;
  const int ci = lane < P ? lane : 0;
  float xw = warp_sum<P, kLower>(wpow, tot, h < 0 ? 0 : h, warp, ci);
  if (looks) {
    const bool successor = tin + 1 < a.tiles_per_row;
    if (tin == 0) {
      if (warp == 0 && successor)
        publish<P>(a, tile, 1, (double)warp_sum<P, kLower>(wpow, tot, 0, kWarps, ci), lane);
    } else {
      if (warp == 0) {
        const double agg = (double)warp_sum<P, kLower>(wpow, tot, 0, kWarps, ci);
        if (successor) publish<P>(a, tile, 0, agg, lane);
        PESQ_IIR_STAMP(tile, 5);
        const double sv = lookback<P>(a, tile, tin, near, lane);
        PESQ_IIR_STAMP(tile, 6);
        if (successor) {
          // inclusive end state: A^kTile S + aggregate
          const double* T1 = near + P * P;
          double acc = agg;
#pragma unroll
          for (int j = 0; j < P; ++j) {
            const double sj = __shfl_sync(0xffffffffu, sv, j);
            acc = fma(T1[ci * P + j], sj, acc);
          }
          publish<P>(a, tile, 1, acc, lane);
        }
        PESQ_IIR_STAMP(tile, 7);
        if (lane < P) sin_s[lane] = (float)sv;
      }
      __syncthreads();
      PESQ_IIR_STAMP(tile, 3);
      // no head in a tile after the first of its row: add A^(32 kL warp) S
      const float* Wm = wpow + warp * P * P + ci * P;
#pragma unroll
      for (int j = 0; j < P; ++j)
        if (!skip<P, kLower>(ci, j)) xw = fmaf(Wm[j], sin_s[j], xw);
    }
  }

  // 4. start state of the chunk
  float s[P];
  {
    float xv[P];
#pragma unroll
    for (int j = 0; j < P; ++j) xv[j] = __shfl_sync(0xffffffffu, xw, j);
    const float* Lm = lanes + lane * lane_pitch(P);
#pragma unroll
    for (int i = 0; i < P; ++i) {
      float acc = ex[i];
      if (!fex) {
#pragma unroll
        for (int j = 0; j < P; ++j)
          if (!skip<P, kLower>(i, j)) acc = fmaf(Lm[i * P + j], xv[j], acc);
      }
      s[i] = head ? 0.0f : acc;
    }
  }

  // 5. outputs, back into the staged tile
  if (!used) {
    // no data in this chunk
  } else if constexpr (kRerun) {
#pragma unroll
    for (int t = 0; t < kL; ++t) {
      const float xt = xs[base + dir * t];
      float yv = tab.D * xt;
#pragma unroll
      for (int j = 0; j < P; ++j) yv = fmaf(tab.C[j], s[j], yv);
      float ns[P];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        float acc = tab.B[i] * xt;
#pragma unroll
        for (int j = 0; j < P; ++j)
          if (!skip<P, kLower>(i, j)) acc = fmaf(tab.A[i][j], s[j], acc);
        ns[i] = acc;
      }
#pragma unroll
      for (int i = 0; i < P; ++i) s[i] = ns[i];
      xs[base + dir * t] = yv;
    }
  } else {
#pragma unroll
    for (int t = 0; t < kL; ++t) {
      float yv = xs[base + dir * t];
#pragma unroll
      for (int j = 0; j < P; ++j) yv = fmaf(tab.G[t][j], s[j], yv);
      xs[base + dir * t] = yv;
    }
  }
  __syncthreads();

  PESQ_IIR_STAMP(tile, 4);
  if (vec_out) {
    // (qa and qb - qa are multiples of 4)
    float4* dst = reinterpret_cast<float4*>(yrow + m0 + qa);
    const float4* src = reinterpret_cast<const float4*>(xs + qa);
    for (int i = tid; i < (qb - qa) / 4; i += kThreads) dst[i] = src[i];
  } else if (chained) {
#pragma unroll 11
    for (int k = 0; k < kL; ++k) {
      const int q = tid + k * kThreads;
      const int64_t m = m0 + q;
      if (q >= qa && q < qb && m >= 0 && m < a.n) yrow[m] = xs[q];
    }
  } else {
    const int n = (int)a.n;
    const int lead = kRev ? seg - n : 0;
    for (int rr = warp; rr < nrows; rr += kWarps) {
      float* dst = yrow + rr * a.ld_y;
      const float* src = xs + rr * seg + lead;
      for (int i = lane; i < n; i += 32) dst[i] = src[i];
    }
  }
}

// Launch of one instantiation (defined in iir_k*.cu).
template <int P, bool kLower, bool kRerun>
cudaError_t launch(const Args& a, const void* tab, cudaStream_t s);

}  // namespace iir
}  // namespace pesq
