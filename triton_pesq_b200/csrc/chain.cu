// Perceptual chain of the PESQ model, forward and adjoint.
//
// One thread block cluster per utterance; CTA q of the cluster owns a
// contiguous slice of frames and each of its 16 warps a contiguous sub-slice
// (lanes cover the Bark bands k and k + 32).  The slice's Bark spectra (and,
// in the adjoint, their gradient accumulators) are staged in shared memory.
// The genuine whole-signal dependencies of the model -- the band means over
// all non-silent frames (torch_pesq/loss.py:205-216), the two-tap smoothing of
// the frame power ratio across frames (loss.py:224-226), the overlapping
// 20-frame windows and the RMS over them (loss.py:257-266) -- are resolved
// with cluster barriers: band partial sums are exchanged through distributed
// shared memory, per-frame values through the saved-state arrays in global
// memory.  Every reduction has a fixed order, so results are bitwise
// reproducible.
//
// The Bark spectra arrive unscaled; the level alignment (loss.py:132-139)
// enters as s^2 = 1e7 / P with P = sum (H x)^2 / (N + 5120) / 1.04684.
#include <math.h>

#include <stdint.h>

#include "kernels.cuh"

namespace pesq {

constexpr int kChainThreads = 512;
constexpr int kChainWarps = kChainThreads / 32;
// Largest slice (frames of a CTA) whose pass B runs cell by cell.
constexpr int kCellSlice = 128;
// Dynamic shared memory the staged kernels may use.
constexpr size_t kChainSmemLimit = 180 * 1024;

ChainLayout ChainLayout::make(int T, int nb) {
  ChainLayout l;
  l.T = T;
  l.nb = nb;
  l.L = T >= 20 ? (T - 20) / 10 + 1 : 0;
  auto up = [](int64_t v) { return (v + 3) & ~int64_t(3); };
  int64_t o = 0;
  auto take = [&](int64_t n) {
    const int64_t at = o;
    o += up(n);
    return at;
  };
  l.keep = take(T);
  l.taer = take(T);
  l.tad = take(T);
  l.fpr0 = take(T);
  l.fpr1 = take(T);
  l.h = take(T);
  l.sraw = take(T);
  l.araw = take(T);
  l.sp = take(T);
  l.ap = take(T);
  l.gfpr = 0;
  l.psqm_s = take(l.L);
  l.psqm_a = take(l.L);
  l.bpr = take(nb);
  l.ratio = take(nb);
  l.mref = take(nb);
  l.mdeg = take(nb);
  l.scal = take(kNumScalars);
  l.stride = o;
  return l;
}

int chain_slice_frames(int T, int cluster) { return (int)ceil_div(T, cluster); }
// Bark spectra of the slice and the frame before it; with `cells`, also the
// slice's adjoint coefficients, written to shared memory and stored with one
// bulk copy per field
size_t chain_fwd_smem_bytes(int slice, int nb, bool cells) {
  const size_t spectra = ((size_t)2 * (slice + 1) * nb + 3) & ~(size_t)3;
  const size_t cblk = ((size_t)slice * nb + 3) & ~(size_t)3;
  return (spectra + (cells ? (size_t)kCellFields * cblk : 0)) * sizeof(float);
}
// Bark spectra and their gradient accumulators (4 slices), with `cells` the
// forward's adjoint coefficients of the slice (kCellFields slices), the ten
// per-frame saved arrays and two per-frame gradients of frames c_lo..c_hi, and
// the two window arrays over the slice
size_t chain_bwd_smem_bytes(int slice, int nb, bool cells) {
  const size_t cblk = ((size_t)slice * nb + 3) & ~(size_t)3;
  return ((cells ? (size_t)kCellFields * cblk : 0) + (size_t)4 * slice * nb + (size_t)12 * (slice + 1) +
          (size_t)2 * (slice / 10 + 4)) *
         sizeof(float);
}
size_t chain_smem_limit() { return kChainSmemLimit; }

PESQ_PHASE_TABLE(g_phase_chain_fwd)
PESQ_SPAN_TABLE(g_span_chain)
PESQ_PHASE_TABLE(g_phase_chain_bwd)

namespace {

__device__ __forceinline__ float sgnf(float v) { return v > 0.0f ? 1.0f : (v < 0.0f ? -1.0f : 0.0f); }

struct Band {
  int k;
  bool ok;    // k < nb
  bool norm;  // contributes to the weighted norms (k >= 1)
  float th, inv2th, e, ls, dls, w, th100;
  __device__ void load(const DevTables& t, int kk) {
    k = kk;
    ok = kk < t.nb;
    norm = ok && kk >= 1;
    const int i = ok ? kk : 0;
    th = t.thresh[i];
    inv2th = t.inv2th[i];
    e = t.expo[i];
    ls = t.loud_scale[i];
    dls = t.dloud_scale[i];
    w = t.width[i];
    th100 = th * 100.0f;
  }
};

// Zwicker loudness of one band (loudness.py:52-61),
//   L = Sl (2 th)^e ((0.5 + 0.5 x / th)^e - 1) = ls ((1 + bm1)^e - 1),
//   bm1 = (x - th) / (2 th),
// evaluated as ls * expm1(e log1p(bm1)), which keeps full relative precision
// as x approaches the threshold and needs one log1p / expm1 pair at any
// distance from it.  `pw` returns (1 + bm1)^e and `base` 1 + bm1 for the
// derivative dL/dx = dls (1 + bm1)^(e - 1) = dls pw / base.
__device__ __forceinline__ float loudness(float x, const Band& b, float& pw, float& base) {
  if (!(x > b.th)) {
    pw = 0.0f;
    base = 1.0f;
    return 0.0f;
  }
  const float bm1 = (x - b.th) * b.inv2th;
  const float em1 = expm1f(b.e * log1pf(bm1));
  pw = 1.0f + em1;
  base = 1.0f + bm1;
  return b.ls * em1;
}

// loudness, disturbance and the asymmetry factor of one band of one frame
// (loss.py:228-255)
struct Cell {
  float er, ed, lr, ld, u, zz, dist, asc_raw, asc;
  float pr, br, pd, bd;  // (1 + bm1)^e and 1 + bm1 of er and ed
  __device__ void eval(const Band& b, float R, float D, float bpr, float fpr) {
    er = bpr * R;
    ed = fpr * D;
    lr = loudness(er, b, pr, br);
    ld = loudness(ed, b, pd, bd);
    u = ld - lr;
    zz = fabsf(u) - 0.25f * fminf(ld, lr);
    dist = sgnf(u) * fmaxf(zz, 0.0f);
    // ((ed + 50) / (er + 50))^1.2 with the hardware exp2 / log2 (about
    // 1e-6 relative: asc only enters through its clamp to [3, 12] and the
    // asymmetric norm)
    asc_raw = exp2f_fast(1.2f * log2f_fast(__fdividef(ed + 50.0f, er + 50.0f)));
    asc = asc_raw < 3.0f ? 0.0f : fminf(asc_raw, 12.0f);
  }
  // The adjoint of eval for the two norms' gradients g_dist and g_asc, as the
  // coefficients of kCellEdDist .. kCellErAsc (loss.py:236-255 differentiated;
  // gradient only, so the 2-ulp fast division is far inside the tolerance):
  //   dist = sgn(u) max(|u| - min(ld, lr) / 4, 0), u = ld - lr,
  //   asc  = clamp(((ed + 50) / (er + 50))^1.2 -> 0 below 3, 12 above).
  __device__ void adjoint(const Band& b, float co[4]) const {
    const float su = sgnf(u);
    const float live = zz >= 0.0f ? 1.0f : 0.0f;  // the dead zone is not active
    const float e = live * su * su;
    const float wd = ld < lr ? 1.0f : (ld == lr ? 0.5f : 0.0f);  // d min(ld, lr) / d ld
    const float wr = lr < ld ? 1.0f : (ld == lr ? 0.5f : 0.0f);
    const float dld = ed > b.th ? b.dls * __fdividef(pd, bd) : 0.0f;  // dL/dx of the loudnesses
    const float dlr = er > b.th ? b.dls * __fdividef(pr, br) : 0.0f;
    const bool slope = asc_raw >= 3.0f && asc_raw <= 12.0f;
    co[0] = dld * (e - 0.25f * live * su * wd);
    co[1] = slope ? __fdividef(1.2f * asc_raw, ed + 50.0f) : 0.0f;
    co[2] = dlr * (-e - 0.25f * live * su * wr);
    co[3] = slope ? -__fdividef(1.2f * asc_raw, er + 50.0f) : 0.0f;
  }
};

// Frames of this CTA (a contiguous slice of the utterance) and of this warp
// (a contiguous sub-slice of that).
struct Slice {
  int c_lo, c_hi, w_lo, w_hi;
  __device__ Slice(int T) {
    const int C = (int)cluster_nctarank(), q = (int)cluster_ctarank();
    const int per = (int)ceil_div(T, C);
    c_lo = min(T, q * per);
    c_hi = min(T, c_lo + per);
    const int n = c_hi - c_lo;
    const int warp = threadIdx.x >> 5;
    w_lo = c_lo + warp * n / kChainWarps;
    w_hi = c_lo + (warp + 1) * n / kChainWarps;
  }
};

// Sum over the cluster of a per-CTA shared double, identical order in every CTA.
__device__ __forceinline__ double cluster_sum(const double* local, int C) {
  double v[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) v[c] = c < C ? dsmem_ld_f64(dsmem_addr(local, c)) : 0.0;
  double s = 0.0;
#pragma unroll
  for (int c = 0; c < 16; ++c) s += v[c];
  return s;
}

// sum of squares of a row from its per-segment partials, one warp
__device__ __forceinline__ double warp_row_sumsq(const double* partial, int nseg, int lane) {
  double s = 0.0;
  for (int i = lane; i < nseg; i += 32) s += partial[i];
  return warp_sum(s);
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------

// kMinBlocks 2: the many-waves variant (64 registers, two CTAs per SM; its
// shared-memory layout leaves the adjoint coefficients unstaged and its cell
// passes run on their global copy, so both variants give the same results)
template <int kMinBlocks>
__global__ void __launch_bounds__(kChainThreads, kMinBlocks) chain_fwd_kernel(const __grid_constant__ ChainFwdArgs p) {
  extern __shared__ __align__(16) float dsm[];
  __shared__ DevTables tab;
  __shared__ double wpr[kChainWarps][kMaxBands], wpd[kChainWarps][kMaxBands];
  __shared__ double part_r[kMaxBands], part_d[kMaxBands];
  __shared__ double band_tot[2][kMaxBands];
  __shared__ float bpr_s[kMaxBands];
  __shared__ float s2s[2];
  __shared__ float fpr_s[kCellSlice], h_s[kCellSlice];  // per frame of the slice (cell-wise pass B)

  const int C = (int)cluster_nctarank(), q = (int)cluster_ctarank();
  const int u = blockIdx.x / C;
  const int B = p.batch, T = p.lay.T, L = p.lay.L;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const Slice sl(T);
  PESQ_SPAN_BEGIN(g_span_chain, 0);
  PESQ_STAMP(g_phase_chain_fwd, 0);

  // tables and the slice's spectra are copied asynchronously while warps 0-1
  // reduce the level alignment power; the tables do not depend on the front
  // kernel, everything after pdl_wait does
  copy_async<kChainThreads>(&tab, p.tab, (int)sizeof(DevTables));
  pdl_wait();
  const float* Fr = p.bark + (int64_t)u * T * p.lay.nb;
  const float* Fd = p.bark + (int64_t)(B + u) * T * p.lay.nb;
  const int nb = p.lay.nb;
  // staged frames c_lo - 1 .. c_hi - 1 (the one before the slice feeds the
  // frame power ratio smoothing of its first frame)
  const int t_first = sl.c_lo - 1;
  const float* fr = Fr;
  const float* fd = Fd;
  int64_t origin = 0;
  if (p.staged) {
    const int pitch = (sl.c_hi - sl.c_lo + 1) * nb;
    float* sr = dsm;
    float* sd = dsm + pitch;
    // frame -1 (before the signal) reads as zeros
    const int skip = t_first < 0 ? nb : 0;
    for (int i = threadIdx.x; i < skip; i += kChainThreads) sr[i] = sd[i] = 0.0f;
    stage_rows_async<kChainThreads>(sr + skip, pitch, Fr + (int64_t)t_first * nb + skip, Fd - Fr, 2,
                                    (sl.c_hi - t_first) * nb - skip);
    fr = sr;
    fd = sd;
    origin = (int64_t)t_first * nb;
  }
  cp_async_commit();
  // adjoint coefficients of the slice: staged in shared memory after the
  // spectra when they fit (p.stage_cells), else stored directly
  const int64_t cblk = cell_block(T, C, nb);
  float* cst = nullptr;
  if (p.cells && p.staged && p.stage_cells) cst = dsm + ((2 * (sl.c_hi - sl.c_lo + 1) * nb + 3) & ~3);
  if (warp < 2) {
    // level alignment power of both rows, loss.py:132-136
    const int r = warp == 0 ? u : B + u;
    const double tot = warp_row_sumsq(p.partial + (int64_t)r * p.nseg, p.nseg, lane);
    if (lane == 0) {
      const double denom = ((double)p.n + 5120.0) * 1.04684;
      s2s[warp] = (float)(1e7 / (tot / denom));
      if (q == 0) p.sumsq[r] = tot;
    }
  }
  cp_async_wait_all();
  __syncthreads();
  PESQ_STAMP(g_phase_chain_fwd, 1);
  const float s2r = s2s[0], s2d = s2s[1];
  float* sv = p.saved + (int64_t)u * p.lay.stride;
  auto at = [&](int t, int k) { return (int64_t)t * nb + k - origin; };

  Band b0, b1;
  b0.load(tab, lane);
  b1.load(tab, lane + 32);

  // pass A: silent frames (loss.py:206) and band sums of audible power over
  // the non-silent frames (loudness.py:297-320)
  {
    // four frames at a time: their band sums go through the warp's shuffle
    // tree side by side (the same tree per frame as warp_sum), then the
    // frames are accumulated in order
    constexpr int kG = 4;
    double ar0 = 0.0, ar1 = 0.0, ad0 = 0.0, ad1 = 0.0;
    for (int t = sl.w_lo; t < sl.w_hi; t += kG) {
      float a0[kG], a1[kG], e0[kG], e1[kG], tot[kG];
#pragma unroll
      for (int i = 0; i < kG; ++i) {
        const bool v = t + i < sl.w_hi;
        const float R0 = v && b0.ok ? s2r * fr[at(t + i, b0.k)] : 0.0f;
        const float R1 = v && b1.ok ? s2r * fr[at(t + i, b1.k)] : 0.0f;
        const float D0 = v && b0.ok ? s2d * fd[at(t + i, b0.k)] : 0.0f;
        const float D1 = v && b1.ok ? s2d * fd[at(t + i, b1.k)] : 0.0f;
        a0[i] = R0 > b0.th100 ? R0 : 0.0f;
        a1[i] = R1 > b1.th100 ? R1 : 0.0f;
        e0[i] = D0 > b0.th100 ? D0 : 0.0f;
        e1[i] = D1 > b1.th100 ? D1 : 0.0f;
        tot[i] = a0[i] + a1[i];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int i = 0; i < kG; ++i) tot[i] += __shfl_xor_sync(0xffffffffu, tot[i], o);
      }
#pragma unroll
      for (int i = 0; i < kG; ++i) {
        if (t + i >= sl.w_hi) break;
        const bool keep = !(tot[i] < 1e7f);
        if (lane == 0) sv[p.lay.keep + t + i] = keep ? 1.0f : 0.0f;
        if (keep) {
          ar0 += a0[i];
          ar1 += a1[i];
          ad0 += e0[i];
          ad1 += e1[i];
        }
      }
    }
    wpr[warp][lane] = ar0;
    wpd[warp][lane] = ad0;
    wpr[warp][lane + 32] = ar1;
    wpd[warp][lane + 32] = ad1;
  }
  __syncthreads();
  if (threadIdx.x < nb) {
    const int k = threadIdx.x;
    double r = 0.0, d = 0.0;
    for (int w = 0; w < kChainWarps; ++w) {
      r += wpr[w][k];
      d += wpd[w][k];
    }
    part_r[k] = r;
    part_d[k] = d;
  }
  cluster_sync();
  if (threadIdx.x < 2 * nb) {
    const int k = threadIdx.x % nb, side = threadIdx.x / nb;
    band_tot[side][k] = cluster_sum(side == 0 ? &part_r[k] : &part_d[k], C);
  }
  __syncthreads();
  if (threadIdx.x < nb) {
    const int k = threadIdx.x;
    // band power ratio, loss.py:212-216
    const float mr = (float)(band_tot[0][k] / T), md = (float)(band_tot[1][k] / T);
    const float ratio = (md + 1000.0f) / (mr + 1000.0f);
    const float bpr = fminf(fmaxf(ratio, 0.01f), 100.0f);
    bpr_s[k] = bpr;
    if (q == 0) {
      sv[p.lay.bpr + k] = bpr;
      sv[p.lay.ratio + k] = ratio;
      sv[p.lay.mref + k] = mr;
      sv[p.lay.mdeg + k] = md;
    }
  }
  if (q == 0 && threadIdx.x == 0) {
    sv[p.lay.scal + kS2Ref] = s2r;
    sv[p.lay.scal + kS2Deg] = s2d;
  }
  __syncthreads();
  PESQ_STAMP(g_phase_chain_fwd, 2);

  // pass B: frame power ratio, loudness, disturbance and the weighted norms
  // (loss.py:217-255).  A warp takes its frames in chunks of up to 32: the
  // band sums of every frame first, then the per-frame scalars (frame power
  // ratio and its smoothing, h) one frame per lane, then the bands of each
  // frame, and the frame distances again one frame per lane -- the same
  // operations in the same order per frame as one frame at a time, with the
  // divisions and transcendentals of the frames side by side.
  {
    const float bpr0 = b0.ok ? bpr_s[b0.k] : 0.0f, bpr1 = b1.ok ? bpr_s[b1.k] : 0.0f;
    const float sqW = tab.sqrt_total_width;
    auto audible = [&](int t, float& taer, float& tad) {
      const float er0 = b0.ok ? bpr0 * (s2r * fr[at(t, b0.k)]) : 0.0f;
      const float er1 = b1.ok ? bpr1 * (s2r * fr[at(t, b1.k)]) : 0.0f;
      const float D0 = b0.ok ? s2d * fd[at(t, b0.k)] : 0.0f, D1 = b1.ok ? s2d * fd[at(t, b1.k)] : 0.0f;
      taer = warp_sum((er0 > b0.th ? er0 : 0.0f) + (er1 > b1.th ? er1 : 0.0f));
      tad = warp_sum((D0 > b0.th ? D0 : 0.0f) + (D1 > b1.th ? D1 : 0.0f));
    };
    // fpr0 of the frame before the warp's first (its smoothing partner)
    float fpr0_carry = 0.0f;
    if (sl.w_lo < sl.w_hi && sl.w_lo > 0) {
      float ta, td;
      audible(sl.w_lo - 1, ta, td);
      fpr0_carry = (ta + 5e3f) / (td + 5e3f);
    }
    // With the adjoint coefficients staged in shared memory, the bands of the
    // slice are spread over all threads of the CTA, a (frame, band) cell at a
    // time, between a per-frame pass that sets the frame power ratios and one
    // that forms the norms from the staged disturbances; each cell and each
    // norm is evaluated exactly as below, so the results are the same.
    // the cell pass works on the staged coefficients, or (many-waves variant)
    // on their global copy: a compile-time choice of shared or global accesses
    constexpr bool kDual = kMinBlocks == 2;
    float* const cb = kDual ? (p.cells ? p.cells + ((int64_t)u * C + q) * cblk : nullptr) : cst;
    const int64_t cbs = kDual ? p.cell_stride : cblk;  // floats between the fields of cb
    const bool by_cell = cb != nullptr && sl.c_hi - sl.c_lo <= kCellSlice;
    for (int t_base = sl.w_lo; t_base < sl.w_hi; t_base += 32) {
      const int nf = min(32, sl.w_hi - t_base);
      // 1. total audible energies of each frame (lane j keeps frame j's)
      float my_taer = 0.0f, my_tad = 0.0f;
      for (int j = 0; j < nf; ++j) {
        float taer, tad;
        audible(t_base + j, taer, tad);
        if (lane == j) {
          my_taer = taer;
          my_tad = tad;
        }
      }
      // 2. frame power ratio, its two-tap smoothing and clamp, h
      const int tl = t_base + lane;
      const float fpr0 = (my_taer + 5e3f) / (my_tad + 5e3f);
      const float prev = __shfl_up_sync(0xffffffffu, fpr0, 1);
      const float fpr0_prev = lane == 0 ? fpr0_carry : prev;
      const float fpr1 = tl == 0 ? fpr0 : fpr0 * 0.8f + fpr0_prev * 0.2f;
      const float my_fpr = fminf(fmaxf(fpr1, 3e-4f), 5.0f);
      const float my_h = exp2f_fast(0.04f * log2f_fast((my_taer + 1e5f) * 1e-7f));
      fpr0_carry = __shfl_sync(0xffffffffu, fpr0, nf - 1);
      if (by_cell) {
        if (lane < nf) {
          fpr_s[tl - sl.c_lo] = my_fpr;
          h_s[tl - sl.c_lo] = my_h;
          sv[p.lay.taer + tl] = my_taer;
          sv[p.lay.tad + tl] = my_tad;
          sv[p.lay.fpr0 + tl] = fpr0;
          sv[p.lay.fpr1 + tl] = fpr1;
          sv[p.lay.h + tl] = my_h;
        }
        continue;
      }
      // 3. bands of each frame: loudness, disturbance, asymmetry, adjoint
      //    coefficients, and the two norms (lane j keeps frame j's)
      float my_qs = 0.0f, my_qa = 0.0f;
      for (int j = 0; j < nf; ++j) {
        const int t = t_base + j;
        const float fpr = __shfl_sync(0xffffffffu, my_fpr, j);
        const float R0 = b0.ok ? s2r * fr[at(t, b0.k)] : 0.0f, R1 = b1.ok ? s2r * fr[at(t, b1.k)] : 0.0f;
        const float D0 = b0.ok ? s2d * fd[at(t, b0.k)] : 0.0f, D1 = b1.ok ? s2d * fd[at(t, b1.k)] : 0.0f;
        Cell c0, c1;
        c0.eval(b0, R0, D0, bpr0, fpr);
        c1.eval(b1, R1, D1, bpr1, fpr);
        if (p.cells) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const Band& b = half == 0 ? b0 : b1;
            const Cell& c = half == 0 ? c0 : c1;
            if (!b.ok) continue;
            float co[4];
            c.adjoint(b, co);
            const int i = (t - sl.c_lo) * nb + b.k;
            // shared memory block (bulk-stored after the pass) or straight to global
            float* dst = cst ? cst + i : p.cells + ((int64_t)u * C + q) * cblk + i;
            const int64_t fs = cst ? cblk : p.cell_stride;
            dst[kCellDist * fs] = c.dist;
            dst[kCellAsc * fs] = c.asc;
            dst[kCellEdDist * fs] = co[0];
            dst[kCellEdAsc * fs] = co[1];
            dst[kCellErDist * fs] = co[2];
            dst[kCellErAsc * fs] = co[3];
          }
        }
        float qs = 0.0f, qa = 0.0f;
        if (b0.norm) {
          const float v = b0.w * c0.dist;
          qs = v * v;
          qa = fabsf(b0.w * (c0.dist * c0.asc));
        }
        if (b1.norm) {
          const float v = b1.w * c1.dist;
          qs = fmaf(v, v, qs);
          qa += fabsf(b1.w * (c1.dist * c1.asc));
        }
        qs = warp_sum(qs);
        qa = warp_sum(qa);
        if (lane == j) {
          my_qs = qs;
          my_qa = qa;
        }
      }
      // 4. frame distances, and the frame's saved state
      if (lane < nf) {
        const float sraw = sqW * sqrtf(my_qs);
        const float araw = my_qa;
        sv[p.lay.taer + tl] = my_taer;
        sv[p.lay.tad + tl] = my_tad;
        sv[p.lay.fpr0 + tl] = fpr0;
        sv[p.lay.fpr1 + tl] = fpr1;
        sv[p.lay.h + tl] = my_h;
        sv[p.lay.sraw + tl] = sraw;
        sv[p.lay.araw + tl] = araw;
        sv[p.lay.sp + tl] = fminf(fmaxf(sraw, 1e-20f) / my_h, 45.0f);
        sv[p.lay.ap + tl] = fminf(fmaxf(araw, 1e-20f) / my_h, 45.0f);
      }
    }
    if (by_cell) {
      __syncthreads();
      // cells (t, k) of the slice, k fastest, over all threads
      const int ncell = (sl.c_hi - sl.c_lo) * nb;
      int ct = threadIdx.x / nb, ck = threadIdx.x - ct * nb;
      const int dt = kChainThreads / nb, dk = kChainThreads - dt * nb;
      for (int c = threadIdx.x; c < ncell; c += kChainThreads) {
        Band b;
        b.load(tab, ck);
        const int t = sl.c_lo + ct;
        const float R = s2r * fr[at(t, ck)], D = s2d * fd[at(t, ck)];
        Cell cl;
        cl.eval(b, R, D, bpr_s[ck], fpr_s[ct]);
        float co[4];
        cl.adjoint(b, co);
        float* dst = cb + c;
        dst[kCellDist * cbs] = cl.dist;
        dst[kCellAsc * cbs] = cl.asc;
        dst[kCellEdDist * cbs] = co[0];
        dst[kCellEdAsc * cbs] = co[1];
        dst[kCellErDist * cbs] = co[2];
        dst[kCellErAsc * cbs] = co[3];
        ct += dt;
        ck += dk;
        if (ck >= nb) {
          ck -= nb;
          ++ct;
        }
      }
      __syncthreads();
      // the two norms of each frame from the staged disturbances (lane j
      // keeps frame j's), then the frame distances
      for (int t_base = sl.w_lo; t_base < sl.w_hi; t_base += 32) {
        const int nf = min(32, sl.w_hi - t_base);
        float my_qs = 0.0f, my_qa = 0.0f;
        for (int j = 0; j < nf; ++j) {
          const int i = (t_base + j - sl.c_lo) * nb;
          float qs = 0.0f, qa = 0.0f;
          if (b0.norm) {
            const float dist = cb[kCellDist * cbs + i + b0.k], asc = cb[kCellAsc * cbs + i + b0.k];
            const float v = b0.w * dist;
            qs = v * v;
            qa = fabsf(b0.w * (dist * asc));
          }
          if (b1.norm) {
            const float dist = cb[kCellDist * cbs + i + b1.k], asc = cb[kCellAsc * cbs + i + b1.k];
            const float v = b1.w * dist;
            qs = fmaf(v, v, qs);
            qa += fabsf(b1.w * (dist * asc));
          }
          qs = warp_sum(qs);
          qa = warp_sum(qa);
          if (lane == j) {
            my_qs = qs;
            my_qa = qa;
          }
        }
        const int tl = t_base + lane;
        if (lane < nf) {
          const float h = h_s[tl - sl.c_lo];
          const float sraw = sqW * sqrtf(my_qs);
          const float araw = my_qa;
          sv[p.lay.sraw + tl] = sraw;
          sv[p.lay.araw + tl] = araw;
          sv[p.lay.sp + tl] = fminf(fmaxf(sraw, 1e-20f) / h, 45.0f);
          sv[p.lay.ap + tl] = fminf(fmaxf(araw, 1e-20f) / h, 45.0f);
        }
      }
    }
  }
  if (cst) {
    // the slice's coefficients: one bulk copy per field
    fence_proxy_async_shared();
    __syncthreads();
    if (threadIdx.x == 0) {
      float* dst = p.cells + ((int64_t)u * C + q) * cblk;
      for (int f = 0; f < kCellFields; ++f)
        bulk_s2g(dst + f * p.cell_stride, cst + f * cblk, (uint32_t)(cblk * sizeof(float)));
      bulk_commit();
    }
  }
  cluster_sync();
  PESQ_STAMP(g_phase_chain_fwd, 3);

  // pass C: sixth-power means over 20-frame windows (loss.py:257-266),
  // normalised by the window maximum so that the 1e-20 floor of the
  // disturbance does not underflow; every CTA evaluates the windows that start
  // in its slice
  {
    const int l_lo = (sl.c_lo + 9) / 10, l_hi = min(L, (sl.c_hi + 9) / 10);
    const int nw = max(0, l_hi - l_lo);
    for (int job = warp; job < 2 * nw; job += kChainWarps) {
      const int side = job / nw, l = l_lo + job % nw;
      const int64_t src = side == 0 ? p.lay.sp : p.lay.ap;
      const int64_t dst = side == 0 ? p.lay.psqm_s : p.lay.psqm_a;
      const float s = lane < 20 ? __ldcg(sv + src + 10 * l + lane) : 0.0f;
      const float mx = warp_max(s);
      const float sc = mx > 0.0f ? mx : 1.0f;
      const float v = s / sc, v2 = v * v;
      const float m6 = warp_sum(lane < 20 ? v2 * v2 * v2 : 0.0f) / 20.0f;
      if (lane == 0) sv[dst + l] = mx * powf(m6, 1.0f / 6.0f);
    }
  }
  cluster_sync();
  PESQ_STAMP(g_phase_chain_fwd, 4);

  // RMS over the windows (rank 0), then MOS and loss (loss.py:289-297, 320-322)
  if (q == 0 && warp < 2) {
    const int64_t src = warp == 0 ? p.lay.psqm_s : p.lay.psqm_a;
    // the windows of two strides of the warp stay in registers between the
    // maximum and the sum (one memory round trip for up to 64 windows)
    const float w0 = lane < L ? __ldcg(sv + src + lane) : 0.0f;
    const float w1 = lane + 32 < L ? __ldcg(sv + src + lane + 32) : 0.0f;
    float mx = fmaxf(w0, w1);
    for (int l = lane + 64; l < L; l += 32) mx = fmaxf(mx, __ldcg(sv + src + l));
    mx = warp_max(mx);
    const float sc = mx > 0.0f ? mx : 1.0f;
    float acc = 0.0f;
    for (int l = lane; l < L; l += 32) {
      const float v = (l < lane + 64 ? (l < 32 ? w0 : w1) : __ldcg(sv + src + l)) / sc;
      acc = fmaf(v, v, acc);
    }
    acc = warp_sum(acc);
    const float d = mx * sqrtf(acc / (float)L);
    if (lane == 0) {
      sv[p.lay.scal + (warp == 0 ? kDSymm : kDAsymm)] = d;
      if (warp == 0 && p.d_symm) p.d_symm[u] = d;
      if (warp == 1 && p.d_asymm) p.d_asymm[u] = d;
    }
  }
  if (q == 0) {
    __syncthreads();
    if (warp == 0) {
      uint32_t last = 0;
      if (lane == 0) {
        const float ds = sv[p.lay.scal + kDSymm], da = sv[p.lay.scal + kDAsymm];
        const float m = 4.5f - 0.1f * ds - 0.0309f * da;
        const float loss = (float)(p.factor * (0.1 * (double)ds + 0.0309 * (double)da));
        if (p.mos) p.mos[u] = 0.999f + 4.0f / (1.0f + expf(-1.3669f * m + 3.8224f));
        if (p.loss) p.loss[u] = loss;
        sv[p.lay.scal + kLoss] = loss;
        // batch sum of the losses (the global mean of a data-parallel step
        // reduces it over the ranks): the cluster that arrives last adds the
        // batch up, in a fixed order whichever cluster that is
        __threadfence();
        last = atomicAdd(p.done, 1u) == (uint32_t)(B - 1) ? 1u : 0u;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence();
        double acc = 0.0;
        for (int i = lane; i < B; i += 32) acc += (double)__ldcg(p.saved + (int64_t)i * p.lay.stride + p.lay.scal + kLoss);
        acc = warp_sum(acc);
        if (lane == 0) {
          p.loss_sum[0] = acc;
          p.loss_sum[1] = (double)B;
        }
      }
    }
  }
  if (cst && threadIdx.x == 0) bulk_wait_all();
  PESQ_STAMP(g_phase_chain_fwd, 5);
  PESQ_SPAN_END(g_span_chain, 0);
  pdl_trigger();
}

// ---------------------------------------------------------------------------
// adjoint
// ---------------------------------------------------------------------------

template <int kMinBlocks>
__global__ void __launch_bounds__(kChainThreads, kMinBlocks) chain_bwd_kernel(const __grid_constant__ ChainBwdArgs p) {
  extern __shared__ __align__(16) float dsm[];
  __shared__ DevTables tab;
  __shared__ double wpart[kChainWarps][kMaxBands];
  __shared__ double part[kMaxBands];
  __shared__ float gm_r[kMaxBands], gm_d[kMaxBands];
  __shared__ double kap[kChainWarps][2];
  __shared__ double kpart[2];
  __shared__ float coef_s[kCellSlice], garaw_s[kCellSlice];  // per frame of the slice (cell-wise pass 1)

  const int C = (int)cluster_nctarank(), q = (int)cluster_ctarank();
  const int u = blockIdx.x / C;
  const int B = p.batch, T = p.lay.T, L = p.lay.L, nb = p.lay.nb;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const Slice sl(T);
  PESQ_SPAN_BEGIN(g_span_chain, 1);
  PESQ_STAMP(g_phase_chain_bwd, 0);

  // the next kernel on the stream (the align kernel, which reads nothing this
  // kernel writes) may start on the SMs the clusters leave free
  pdl_trigger();
  copy_async<kChainThreads>(&tab, p.tab, (int)sizeof(DevTables));
  // everything below reads what the forward (or the caller's upstream
  // gradient) wrote
  pdl_wait();
  const float* sv = p.saved + (int64_t)u * p.lay.stride;
  float* gf = p.scratch + (int64_t)u * 2 * T;  // [g_fpr | g_h] per frame
  const float* Fr = p.bark + (int64_t)u * T * nb;
  const float* Fd = p.bark + (int64_t)(B + u) * T * nb;
  float* GR = p.g_bark + (int64_t)u * T * nb;
  float* GD = p.g_bark + (int64_t)(B + u) * T * nb;
  // the slice's spectra and gradient accumulators: shared memory if staged,
  // else the gradient outputs themselves serve as accumulators
  const float* fr = Fr;
  const float* fd = Fd;
  float* gr = GR;
  float* gd = GD;
  int64_t origin = 0;
  // per-frame saved state (frames c_lo..c_hi) and the 20-frame windows over
  // the slice: staged next to the spectra, or read from global memory
  enum { kKeep, kTaer, kTad, kFpr0, kFpr1, kH, kSraw, kAraw, kSp, kAp, kFrameArrays };
  const int64_t upT = p.lay.taer - p.lay.keep;  // pitch of the saved per-frame arrays
  const int fpitch = sl.c_hi - sl.c_lo + 1;
  const int l_min = sl.c_lo >= 19 ? (sl.c_lo - 10) / 10 : 0;
  const int l_max = min(L - 1, (sl.c_hi - 1) / 10);
  const int wpitch = (T + C - 1) / C / 10 + 4;
  // the coefficients of this CTA's slice: one 16-byte aligned block per field
  const int64_t cblk = cell_block(T, C, nb);
  const float* cells = p.cells + ((int64_t)u * C + q) * cblk;
  const int cpitch = (int)cblk;  // floats between the staged fields
  float* cs = nullptr;   // [kCellFields][cpitch]
  float* fs = nullptr;   // [kFrameArrays][fpitch]
  float* gfs = nullptr;  // [2][fpitch]: dL/dfpr, dL/dh of the slice's frames
  float* ws = nullptr;   // [2][wpitch]: psqm_s, psqm_a of windows l_min..l_max
  const bool cells_staged = p.staged && p.stage_cells;
  if (p.staged) {
    const int n = (sl.c_hi - sl.c_lo) * nb;
    float* sr = dsm;  // 16-byte aligned
    if (cells_staged) {
      cs = dsm;  // first
      for (int f = 0; f < kCellFields; ++f)
        copy_async<kChainThreads>(cs + f * cpitch, cells + f * p.cell_stride, ((n + 3) & ~3) * 4);
      sr = cs + kCellFields * cpitch;
    }
    float* sd = sr + n;
    stage_rows_async<kChainThreads>(sr, n, Fr + (int64_t)sl.c_lo * nb, Fd - Fr, 2, n);
    fr = sr;
    fd = sd;
    gr = sd + n;
    gd = gr + n;
    origin = (int64_t)sl.c_lo * nb;
    fs = gd + n;
    gfs = fs + kFrameArrays * fpitch;
    ws = gfs + 2 * fpitch;
    stage_rows_async<kChainThreads>(fs, fpitch, sv + p.lay.keep + sl.c_lo, upT, kFrameArrays,
                                    min(sl.c_hi + 1, T) - sl.c_lo);
    stage_rows_async<kChainThreads>(ws, wpitch, sv + p.lay.psqm_s + l_min, p.lay.psqm_a - p.lay.psqm_s, 2,
                                    max(0, l_max - l_min + 1));
  }
  cp_async_commit();
  auto at = [&](int t, int k) { return (int64_t)t * nb + k - origin; };
  auto FS = [&](int k, int t) -> float {
    return p.staged ? fs[k * fpitch + (t - sl.c_lo)] : __ldg(sv + p.lay.keep + k * upT + t);
  };
  auto CELL = [&](int f, int t, int k) -> float {
    const int i = (t - sl.c_lo) * nb + k;
    return cells_staged ? cs[f * cpitch + i] : __ldg(cells + f * p.cell_stride + i);
  };
  auto PQ = [&](int side, int l) -> float {
    return p.staged ? ws[side * wpitch + (l - l_min)] : __ldg(sv + (side ? p.lay.psqm_a : p.lay.psqm_s) + l);
  };
  const float s2r = sv[p.lay.scal + kS2Ref], s2d = sv[p.lay.scal + kS2Deg];
  const float ds = sv[p.lay.scal + kDSymm], da = sv[p.lay.scal + kDAsymm];

  // upstream gradients of both distances (epilogue adjoint)
  const int gu = u * p.g_stride;
  float gds = p.g_dsymm ? p.g_dsymm[gu] : 0.0f;
  float gda = p.g_dasymm ? p.g_dasymm[gu] : 0.0f;
  if (p.g_loss) {
    gds += (float)(p.g_loss[gu] * p.factor * 0.1);
    gda += (float)(p.g_loss[gu] * p.factor * 0.0309);
  }
  if (p.g_mos) {
    const float m = 4.5f - 0.1f * ds - 0.0309f * da;
    const float ex = expf(-1.3669f * m + 3.8224f);
    const float den = 1.0f + ex;
    const float dm = 4.0f * 1.3669f * ex / (den * den);
    gds += p.g_mos[gu] * dm * -0.1f;
    gda += p.g_mos[gu] * dm * -0.0309f;
  }

  cp_async_wait_all();
  __syncthreads();
  PESQ_STAMP(g_phase_chain_bwd, 1);

  Band b0, b1;
  b0.load(tab, lane);
  b1.load(tab, lane + 32);
  const float bpr0 = b0.ok ? sv[p.lay.bpr + b0.k] : 0.0f, bpr1 = b1.ok ? sv[p.lay.bpr + b1.k] : 0.0f;
  const float W = tab.total_width;

  // dL/d(frame distance) through the windows, the RMS, the 45 clamp, /h and
  // the 1e-20 floor
  auto frame_grads = [&](int t, float& g_sraw, float& g_araw, float& g_h) {
    const float h = FS(kH, t);
    g_sraw = g_araw = g_h = 0.0f;
#pragma unroll
    for (int side = 0; side < 2; ++side) {
      const float d = side == 0 ? ds : da;
      const float gdist = side == 0 ? gds : gda;
      const float s = FS(side == 0 ? kSp : kAp, t);
      const float raw = FS(side == 0 ? kSraw : kAraw, t);
      float gs = 0.0f;
      if (d > 0.0f) {
        const int l_lo = t >= 19 ? (t - 19 + 9) / 10 : 0;
        const int l_hi = min(L - 1, t / 10);
        for (int l = l_lo; l <= l_hi; ++l) {
          const float pl = PQ(side, l);
          if (pl > 0.0f) {
            const float r = __fdividef(s, pl), r2 = r * r;
            gs += pl * (r2 * r2 * r);
          }
        }
        gs *= gdist / (20.0f * (float)L * d);
      }
      const float c = fmaxf(raw, 1e-20f);
      const bool inside = c / h <= 45.0f;
      const float gc = inside ? gs / h : 0.0f;
      g_h -= inside ? gs * c / (h * h) : 0.0f;
      const float graw = raw >= 1e-20f ? gc : 0.0f;
      if (side == 0)
        g_sraw = graw;
      else
        g_araw = graw;
    }
  };

  // pass 1: norm / disturbance / loudness adjoint per band from the forward's
  // coefficients; per-frame dL/dfpr.  The per-frame scalars are evaluated one
  // frame per lane for up to 32 frames at a time, then each frame's bands --
  // or, with the slice staged, the cells (frame, band) of the slice over all
  // threads, and the per-frame sums after them (the same operations, so the
  // same results).
  // (the many-waves variant reads its unstaged coefficients in the same cell
  // pass: the same results as the staged variant)
  const bool by_cell = (kMinBlocks == 2 ? p.staged : cells_staged) && sl.c_hi - sl.c_lo <= kCellSlice;
  for (int t_base = sl.w_lo; t_base < sl.w_hi; t_base += 32) {
    const int nf = min(32, sl.w_hi - t_base);
    float l_coef = 0.0f, l_garaw = 0.0f, l_gh = 0.0f, l_gfpr = 0.0f;
    if (lane < nf) {
      const int t = t_base + lane;
      const float sraw = FS(kSraw, t);
      float g_sraw;
      frame_grads(t, g_sraw, l_garaw, l_gh);
      l_coef = sraw > 0.0f ? g_sraw * W / sraw : 0.0f;
    }
    if (by_cell) {
      if (lane < nf) {
        const int t = t_base + lane;
        coef_s[t - sl.c_lo] = l_coef;
        garaw_s[t - sl.c_lo] = l_garaw;
        gf[T + t] = l_gh;
        gfs[fpitch + t - sl.c_lo] = l_gh;
      }
      continue;
    }
    for (int j = 0; j < nf; ++j) {
      const int t = t_base + j;
      const float coef = __shfl_sync(0xffffffffu, l_coef, j);
      const float g_araw = __shfl_sync(0xffffffffu, l_garaw, j);

      float gfpr = 0.0f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const Band& b = half == 0 ? b0 : b1;
        if (!b.ok) continue;
        const int64_t o = at(t, b.k);
        const float D = s2d * fd[o];
        float g_dist = 0.0f, g_asc = 0.0f;
        if (b.norm) {
          const float dist = CELL(kCellDist, t, b.k), asc = CELL(kCellAsc, t, b.k);
          g_dist = coef * (b.w * b.w) * dist;
          const float g_y = g_araw * b.w * sgnf(dist * asc);
          g_dist += g_y * asc;
          g_asc = g_y * dist;
        }
        const float g_ed = g_dist * CELL(kCellEdDist, t, b.k) + g_asc * CELL(kCellEdAsc, t, b.k);
        const float g_er = g_dist * CELL(kCellErDist, t, b.k) + g_asc * CELL(kCellErAsc, t, b.k);
        gfpr = fmaf(g_ed, D, gfpr);
        gd[o] = g_ed;
        gr[o] = g_er;
      }
      gfpr = warp_sum(gfpr);
      if (lane == j) l_gfpr = gfpr;
    }
    if (lane < nf) {
      const int t = t_base + lane;
      gf[t] = l_gfpr;
      gf[T + t] = l_gh;
      if (p.staged) {
        gfs[t - sl.c_lo] = l_gfpr;
        gfs[fpitch + t - sl.c_lo] = l_gh;
      }
    }
  }
  if (by_cell) {
    __syncthreads();
    const int ncell = (sl.c_hi - sl.c_lo) * nb;
    // the adjoint of cell (frame sl.c_lo + ct, band ck) from its coefficients
    // v[kCell...] (v[kCellDist] and v[kCellAsc] are used for bands >= 1 only)
    auto cell_adjoint = [&](int ct, int ck, const float* v) {
      const int64_t o = at(sl.c_lo + ct, ck);
      const float w = tab.width[ck];
      float g_dist = 0.0f, g_asc = 0.0f;
      if (ck >= 1) {
        const float coef = coef_s[ct], g_araw = garaw_s[ct];
        const float dist = v[kCellDist], asc = v[kCellAsc];
        g_dist = coef * (w * w) * dist;
        const float g_y = g_araw * w * sgnf(dist * asc);
        g_dist += g_y * asc;
        g_asc = g_y * dist;
      }
      gd[o] = g_dist * v[kCellEdDist] + g_asc * v[kCellEdAsc];
      gr[o] = g_dist * v[kCellErDist] + g_asc * v[kCellErAsc];
    };
    if constexpr (kMinBlocks == 2) {
      // The coefficients come from global memory (L2, or DRAM once a large
      // batch's no longer fit): each thread issues the loads of kAhead of its
      // cells before it uses the first, instead of waiting on every cell's.
      constexpr int kAhead = 3;
      for (int c0 = threadIdx.x; c0 < ncell; c0 += kAhead * kChainThreads) {
        float v[kAhead][kCellFields];
#pragma unroll
        for (int a = 0; a < kAhead; ++a) {
          const int c = c0 + a * kChainThreads;
#pragma unroll
          for (int f = 0; f < kCellFields; ++f) v[a][f] = c < ncell ? __ldg(cells + f * p.cell_stride + c) : 0.0f;
        }
#pragma unroll
        for (int a = 0; a < kAhead; ++a) {
          const int c = c0 + a * kChainThreads;
          if (c < ncell) {
            const int ct = c / nb;
            cell_adjoint(ct, c - ct * nb, v[a]);
          }
        }
      }
    } else {
      int ct = threadIdx.x / nb, ck = threadIdx.x - ct * nb;
      const int dt = kChainThreads / nb, dk = kChainThreads - dt * nb;
      for (int c = threadIdx.x; c < ncell; c += kChainThreads) {
        const int t = sl.c_lo + ct;
        float v[kCellFields];
#pragma unroll
        for (int f = 0; f < kCellFields; ++f) v[f] = (ck >= 1 || f >= kCellEdDist) ? CELL(f, t, ck) : 0.0f;
        cell_adjoint(ct, ck, v);
        ct += dt;
        ck += dk;
        if (ck >= nb) {
          ck -= nb;
          ++ct;
        }
      }
    }
    __syncthreads();
    // dL/dfpr of each frame: sum over bands of g_ed * D (lane j keeps frame j's)
    for (int t_base = sl.w_lo; t_base < sl.w_hi; t_base += 32) {
      const int nf = min(32, sl.w_hi - t_base);
      float l_gfpr = 0.0f;
      for (int j = 0; j < nf; ++j) {
        const int t = t_base + j;
        float gfpr = 0.0f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const Band& b = half == 0 ? b0 : b1;
          if (!b.ok) continue;
          const int64_t o = at(t, b.k);
          gfpr = fmaf(gd[o], s2d * fd[o], gfpr);
        }
        gfpr = warp_sum(gfpr);
        if (lane == j) l_gfpr = gfpr;
      }
      if (lane < nf) {
        const int t = t_base + lane;
        gf[t] = l_gfpr;
        gfs[t - sl.c_lo] = l_gfpr;
      }
    }
  }
  cluster_sync();
  PESQ_STAMP(g_phase_chain_bwd, 2);

  // pass 2: smoothing / clamp / frame ratio adjoint, then the total audible
  // energies; band sums of dL/dbpr
  {
    double acc0 = 0.0, acc1 = 0.0;
    // dL/dfpr of frame tt; the first frame after the slice belongs to the
    // next CTA of the cluster (visible after the cluster barrier)
    auto clamp_pass = [&](int tt) {
      const float f1 = FS(kFpr1, tt);
      const float g = (p.staged && tt < sl.c_hi) ? gfs[tt - sl.c_lo] : __ldcg(gf + tt);
      return (f1 >= 3e-4f && f1 <= 5.0f) ? g : 0.0f;
    };
    for (int t_base = sl.w_lo; t_base < sl.w_hi; t_base += 32) {
      const int nf = min(32, sl.w_hi - t_base);
      // per-frame scalars, one frame per lane
      float l_gtaer = 0.0f, l_gtad = 0.0f, l_fpr = 0.0f;
      if (lane < nf) {
        const int t = t_base + lane;
        const float g1 = clamp_pass(t);
        const float g1n = t + 1 < T ? clamp_pass(t + 1) : 0.0f;
        const float g_fpr0 = (t == 0 ? g1 : 0.8f * g1) + 0.2f * g1n;
        const float taer = FS(kTaer, t), tad = FS(kTad, t);
        const float fpr0 = FS(kFpr0, t), h = FS(kH, t);
        l_fpr = fminf(fmaxf(FS(kFpr1, t), 3e-4f), 5.0f);
        const float g_h = p.staged ? gfs[fpitch + t - sl.c_lo] : __ldcg(gf + T + t);
        l_gtaer = g_fpr0 / (tad + 5e3f) + g_h * 0.04f * h / (taer + 1e5f);
        l_gtad = -g_fpr0 * fpr0 / (tad + 5e3f);
      }
      for (int j = 0; j < nf; ++j) {
        const int t = t_base + j;
        const float fpr = __shfl_sync(0xffffffffu, l_fpr, j);
        const float g_taer = __shfl_sync(0xffffffffu, l_gtaer, j);
        const float g_tad = __shfl_sync(0xffffffffu, l_gtad, j);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const Band& b = half == 0 ? b0 : b1;
          if (!b.ok) continue;
          const int64_t o = at(t, b.k);
          const float R = s2r * fr[o], D = s2d * fd[o];
          const float bpr = half == 0 ? bpr0 : bpr1;
          const float er = bpr * R;
          const float g_er = gr[o] + (er > b.th ? g_taer : 0.0f);
          gr[o] = g_er * bpr;
          const double contrib = (double)g_er * (double)R;
          if (half == 0)
            acc0 += contrib;
          else
            acc1 += contrib;
          gd[o] = gd[o] * fpr + (D > b.th ? g_tad : 0.0f);
        }
      }
    }
    wpart[warp][lane] = acc0;
    wpart[warp][lane + 32] = acc1;
  }
  __syncthreads();
  if (threadIdx.x < nb) {
    double s = 0.0;
    for (int w = 0; w < kChainWarps; ++w) s += wpart[w][threadIdx.x];
    part[threadIdx.x] = s;
  }
  cluster_sync();
  if (threadIdx.x < nb) {
    const int k = threadIdx.x;
    const double g = cluster_sum(&part[k], C);
    // band ratio clamp and quotient (loss.py:212-216), then the mean over T
    const float ratio = sv[p.lay.ratio + k], mr = sv[p.lay.mref + k];
    const float g_ratio = (ratio >= 0.01f && ratio <= 100.0f) ? (float)g : 0.0f;
    gm_r[k] = -g_ratio * ratio / (mr + 1000.0f) / (float)T;
    gm_d[k] = g_ratio / (mr + 1000.0f) / (float)T;
  }
  __syncthreads();
  PESQ_STAMP(g_phase_chain_bwd, 3);

  // pass 3: band means over the non-silent frames; scale to the unscaled
  // spectrum and accumulate <g, F> for the alignment term
  {
    double kr = 0.0, kd = 0.0;
    const float gmr0 = b0.ok ? gm_r[b0.k] : 0.0f, gmr1 = b1.ok ? gm_r[b1.k] : 0.0f;
    const float gmd0 = b0.ok ? gm_d[b0.k] : 0.0f, gmd1 = b1.ok ? gm_d[b1.k] : 0.0f;
    for (int t = sl.w_lo; t < sl.w_hi; ++t) {
      const bool keep = FS(kKeep, t) != 0.0f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const Band& b = half == 0 ? b0 : b1;
        if (!b.ok) continue;
        const int64_t o = at(t, b.k);
        const int64_t og = (int64_t)t * nb + b.k;
        const float Fv = fr[o], Gv = fd[o];
        const float R = s2r * Fv, D = s2d * Gv;
        float vr = gr[o], vd = gd[o];
        if (keep && R > b.th100) vr += half == 0 ? gmr0 : gmr1;
        if (keep && D > b.th100) vd += half == 0 ? gmd0 : gmd1;
        vr *= s2r;
        vd *= s2d;
        GR[og] = vr;
        GD[og] = vd;
        kr += (double)vr * (double)Fv;
        kd += (double)vd * (double)Gv;
      }
    }
    kr = warp_sum(kr);
    kd = warp_sum(kd);
    if (lane == 0) {
      kap[warp][0] = kr;
      kap[warp][1] = kd;
    }
  }
  __syncthreads();
  PESQ_STAMP(g_phase_chain_bwd, 4);
  if (threadIdx.x < 2) {
    double s = 0.0;
    for (int w = 0; w < kChainWarps; ++w) s += kap[w][threadIdx.x];
    kpart[threadIdx.x] = s;
  }
  cluster_sync();
  if (q == 0 && threadIdx.x < 2) {
    const double s = cluster_sum(&kpart[threadIdx.x], C);
    const int r = threadIdx.x == 0 ? u : B + u;
    p.kappa[r] = (float)(2.0 * s / p.sumsq[r]);
  }
  // keep every CTA's shared memory alive until rank 0 has read it
  cluster_sync();
  PESQ_STAMP(g_phase_chain_bwd, 5);
  PESQ_SPAN_END(g_span_chain, 1);
}

// Both chain kernels are launched with programmatic stream serialisation:
// their CTAs may be scheduled once the preceding kernel's CTAs have all
// signalled (front / chain forward: at their end), copy their constant
// tables, and wait for that kernel's completion (pdl_wait) before reading
// anything it wrote.
template <class Kernel, class Args>
cudaError_t launch_cluster(Kernel k, const Args& a, int batch, int cluster, size_t smem, cudaStream_t s) {
  if (batch <= 0) return cudaSuccess;
  LaunchShape l((unsigned)(batch * cluster), kChainThreads, smem, s, true, cluster);
  return cudaLaunchKernelEx(&l.cfg, k, a);
}

}  // namespace

cudaError_t configure_chain() {
  const void* kernels[] = {reinterpret_cast<const void*>(chain_fwd_kernel<1>),
                           reinterpret_cast<const void*>(chain_bwd_kernel<1>),
                           reinterpret_cast<const void*>(chain_fwd_kernel<2>),
                           reinterpret_cast<const void*>(chain_bwd_kernel<2>)};
  for (const void* k : kernels) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kChainSmemLimit);
    if (e != cudaSuccess) return e;
    // clusters of up to 16 CTAs (beyond the portable 8) for long utterances
    e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

int chain_active_clusters(int cluster) {
  // clusters of `cluster` CTAs of both chain kernels that the current device
  // runs at once with the full shared memory allocation (0: none)
  int fewest = 1 << 30;
  for (const void* k : {reinterpret_cast<const void*>(chain_fwd_kernel<1>),
                        reinterpret_cast<const void*>(chain_bwd_kernel<1>)}) {
    LaunchShape l((unsigned)cluster, kChainThreads, kChainSmemLimit, nullptr, false, cluster);
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, k, &l.cfg) != cudaSuccess) {
      cudaGetLastError();  // a refused query leaves no error behind
      return 0;
    }
    fewest = clusters < fewest ? clusters : fewest;
  }
  return fewest;
}

namespace {
// static shared memory of a many-waves chain kernel (queried once), or
// SIZE_MAX when the query fails
size_t dual_static_smem(const void* k) {
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) {
    cudaGetLastError();
    return SIZE_MAX;
  }
  return fa.sharedSizeBytes;
}
}  // namespace

bool chain_dual_fits(int slice, int nb) {
  // both kernels' static and dynamic shared memory (coefficients unstaged)
  // within half an SM's, with the 1 KB the system reserves per CTA
  static const size_t fwd_static = dual_static_smem(reinterpret_cast<const void*>(chain_fwd_kernel<2>));
  static const size_t bwd_static = dual_static_smem(reinterpret_cast<const void*>(chain_bwd_kernel<2>));
  const size_t half = 228 * 1024 / 2 - 1024;
  return fwd_static <= half && bwd_static <= half &&
         fwd_static + chain_fwd_smem_bytes(slice, nb, false) <= half &&
         bwd_static + chain_bwd_smem_bytes(slice, nb, false) <= half;
}

cudaError_t launch_chain_fwd(const ChainFwdArgs& a, int cluster, cudaStream_t s) {
  const int slice = chain_slice_frames(a.lay.T, cluster);
  const size_t smem = a.staged ? chain_fwd_smem_bytes(slice, a.lay.nb, a.cells && a.stage_cells) : 0;
  if (a.dual) return launch_cluster(chain_fwd_kernel<2>, a, a.batch, cluster, smem, s);
  return launch_cluster(chain_fwd_kernel<1>, a, a.batch, cluster, smem, s);
}

cudaError_t launch_chain_bwd(const ChainBwdArgs& a, int cluster, cudaStream_t s) {
  const int slice = chain_slice_frames(a.lay.T, cluster);
  const size_t smem = a.staged ? chain_bwd_smem_bytes(slice, a.lay.nb, a.stage_cells != 0) : 0;
  if (a.dual) return launch_cluster(chain_bwd_kernel<2>, a, a.batch, cluster, smem, s);
  return launch_cluster(chain_bwd_kernel<1>, a, a.batch, cluster, smem, s);
}

}  // namespace pesq
