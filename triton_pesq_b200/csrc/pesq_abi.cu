// C ABI of the PESQ engine: plans, workspace layout and launch sequencing.
//
// Forward  : [resample] -> front (per row segment) -> chain forward (per utterance cluster)
// Backward : chain adjoint (per utterance cluster)
//              || align (per gradient row segment, overlapping the chain adjoint)
//            -> back (per gradient row segment) -> [resample adjoint]
//
// Two kernels forward and three backward at 16 kHz (the reference issues
// about forty).
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "../../include/pesq_cuda.h"
#include "kernels.cuh"

using namespace pesq;

namespace pesq {
cudaError_t configure_front();
cudaError_t configure_back();
}  // namespace pesq

struct pesq_plan {
  int device;
  int sample_rate;
  int nb;
  double factor;
  PowTab pow;
  PreTab pre;        // float32 tables: pre-emphasis adjoint of the back kernel
  PreTab64 pre64;    // float64 tables: pre-emphasis of the front kernel
  DevTables* dtab;   // device copy
  DevTwiddle64* tw64;
  uint32_t* err;     // device error word (kErr* flags), read and cleared by pesq_plan_check
  // frame geometry; `general` when it is not n_fft 512 / hop 256 (the
  // spectrum kernels with the tables in `gen_buf`)
  int nfft, hop;
  bool general;
  void* gen_buf;
  int active_clusters[17];  // [c]: chain clusters of c CTAs the plan's device runs at once (c = 8..16)
  int sms;                  // streaming multiprocessors of the plan's device
  GenTables gen;
  // resampler to 16 kHz (sample_rate != 16000)
  bool resample;
  ResampleTables rs;
};

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PESQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define PESQ_CUDA_TRY(expr, what)             \
  do {                                        \
    cudaError_t _e = (expr);                  \
    if (_e != cudaSuccess) return cuda_fail(_e, what); \
  } while (0)

// Max-abs-row-sum norm of A^k for the P x P row-major float64 matrix a.
double power_norm(const double* a, int P, int k) {
  std::vector<double> r((size_t)P * P, 0.0), b(a, a + (size_t)P * P), t((size_t)P * P);
  for (int i = 0; i < P; ++i) r[(size_t)i * P + i] = 1.0;
  auto mul = [&](const std::vector<double>& x, const std::vector<double>& y, std::vector<double>& z) {
    for (int i = 0; i < P; ++i)
      for (int j = 0; j < P; ++j) {
        double acc = 0.0;
        for (int l = 0; l < P; ++l) acc += x[(size_t)i * P + l] * y[(size_t)l * P + j];
        z[(size_t)i * P + j] = acc;
      }
  };
  for (; k > 0; k >>= 1) {
    if (k & 1) {
      mul(r, b, t);
      r.swap(t);
    }
    mul(b, b, t);
    b.swap(t);
  }
  double norm = 0.0;
  for (int i = 0; i < P; ++i) {
    double row = 0.0;
    for (int j = 0; j < P; ++j) row += fabs(r[(size_t)i * P + j]);
    norm = std::max(norm, row);
  }
  return norm;
}

template <int P, class R>
int fill_scan(ScanTab<P, R>& t, const pesq_scan_desc& d, const char* name) {
  if (d.states != P) return fail(PESQ_ERR_UNSUPPORTED, "%s: %d states, the kernels need %d", name, d.states, P);
  if (d.chunk != kChunk || d.levels != kLevels)
    return fail(PESQ_ERR_UNSUPPORTED, "%s: chunk %d / levels %d, the kernels need %d / %d", name, d.chunk,
                d.levels, kChunk, kLevels);
  if (!d.impulse || !d.carry || !d.drive || !d.power || !d.trans || !d.input || !d.output)
    return fail(PESQ_ERR_INVALID_ARGUMENT, "%s: missing table", name);
  for (int k = 0; k < kChunk; ++k) {
    t.h[k] = (R)d.impulse[k];
    for (int j = 0; j < P; ++j) {
      t.G[k][j] = (R)d.carry[k * P + j];
      t.W[k][j] = (R)d.drive[k * P + j];
    }
  }
  for (int l = 0; l < kLevels; ++l)
    for (int i = 0; i < P; ++i)
      for (int j = 0; j < P; ++j) t.M[l][i][j] = (R)d.power[(l * P + i) * P + j];
  for (int i = 0; i < P; ++i) {
    for (int j = 0; j < P; ++j) t.A[i][j] = (R)d.trans[i * P + j];
    t.B[i] = (R)d.input[i];
    t.C[i] = (R)d.output[i];
  }
  t.D = (R)d.feed;
  return PESQ_OK;
}

// ---------------------------------------------------------------------------
// per-call geometry and workspace layout
// ---------------------------------------------------------------------------

// Frames per segment: the align kernel stages kHorizon before and after the
// segment, the back kernel one hop before and kHorizon + 3 hops after it.
constexpr int kMaxSegFrames = (kSpan - 2 * kHorizon) / kHop;  // 57
static_assert(kMaxSegFrames * kHop + kHorizon + 3 * kHop <= kSpan, "back kernel span");
// Frames per segment of a half-size front CTA (kThreads / 2 threads, two per
// SM): its span holds the warm-up and the frames that start in the segment.
constexpr int kMaxSegFramesHalf = ((kThreads / 2) * kChunk - kHorizon - kHop) / kHop;  // 27
// Waves of full-size CTAs (one per SM) beyond which the front and back
// kernels launch half-size CTAs and the chain kernels their two-CTAs-per-SM
// variant: from two waves on, two CTAs per SM overlap each other's phases
// (the front's float32 scan and float64 transforms) and fill the second
// wave's idle SMs.  Measured graph-replayed steps, one wave -> two-wave
// threshold: 16 x 4 s @44.1 kHz 0.160 -> 0.150 ms, 8 x 10 s @48 kHz 0.183 ->
// 0.170 ms, 64 x 3 s @16 kHz 0.220 -> 0.205 ms.
constexpr int kManyWaves = 1;
// chain cluster sizing (frames per CTA slice, CTAs of a small batch)
constexpr int kChainSliceMax = 104;
constexpr int kChainSliceMin = 32;
constexpr int kChainFillCtas = 64;

struct Geometry {
  int64_t batch, rows, n_src, n16;
  int T, L, nb;
  int seg, nseg;      // segmentation of a row (align; the front unless half-size)
  int seg_f, nseg_f;  // segmentation of a row for the front kernel and its partial sums
  int front_threads;  // kThreads or kThreads / 2
  int seg_b, nseg_b;  // segmentation of a row for the back kernel
  int cluster;
  bool fwd_staged, fwd_stage_cells, bwd_staged, bwd_stage_cells;
  bool chain_dual;  // chain kernels two CTAs per SM (many waves of clusters)
  bool resample, grad, general;
  int nfreq;  // spectrum bins saved per frame
  int grad_begin, grad_end;
  ChainLayout lay;
  // byte offsets
  size_t x16, x16lo, partial, sumsq, bark, fpow, z, spec, saved, cells, gbark, kappa, cscratch, gx16, y64, fgrad, lsum,
      total;
  int64_t cell_stride;  // floats between the fields of the chain's adjoint coefficients
};

void balance(int64_t n16, int max_frames, int& seg, int& nseg) {
  const int64_t hops = ceil_div(n16, kHop);
  nseg = (int)std::max<int64_t>(1, ceil_div(hops, max_frames));
  seg = (int)ceil_div(hops, nseg);
}

int64_t resampled_length(const pesq_plan* p, int64_t n) {
  if (!p->resample) return n;
  return resample_length(p->rs.orig_step, p->rs.new_step, n);
}

int geometry(const pesq_plan* p, int64_t batch, int64_t n_src, uint32_t flags, Geometry& g) {
  if (flags & ~(PESQ_GRAD_REF | PESQ_GRAD_DEG | PESQ_UPSTREAM_SCALAR | PESQ_INPUT_BF16 | PESQ_INPUT_F16))
    return fail(PESQ_ERR_INVALID_ARGUMENT, "unknown flag bits 0x%x", flags);
  if ((flags & PESQ_INPUT_BF16) && (flags & PESQ_INPUT_F16))
    return fail(PESQ_ERR_INVALID_ARGUMENT, "PESQ_INPUT_BF16 and PESQ_INPUT_F16 together");
  if (batch < 0) return fail(PESQ_ERR_INVALID_ARGUMENT, "negative batch %lld", (long long)batch);
  if (n_src <= 0) return fail(PESQ_ERR_INVALID_ARGUMENT, "signals need at least one sample");
  g.batch = batch;
  g.rows = 2 * batch;
  g.n_src = n_src;
  g.resample = p->resample;
  g.n16 = resampled_length(p, n_src);
  // loss.py:191-192 pads by N % 256 whatever the hop; torch.stft, center=False
  const int64_t padded = g.n16 + g.n16 % 256;
  g.T = padded < p->nfft ? 0 : (int)std::min<int64_t>(INT32_MAX, 1 + (padded - p->nfft) / p->hop);
  if (g.T < 20)
    return fail(PESQ_ERR_INVALID_ARGUMENT,
                "The PESQ chain needs at least 20 frames for the overlapping sums, got %d (%lld samples at 16 kHz).",
                g.T, (long long)g.n16);
  if (g.n16 > (int64_t)1 << 31 || g.rows > INT32_MAX)
    return fail(PESQ_ERR_INVALID_ARGUMENT, "signal or batch too large (%lld samples, %lld rows)",
                (long long)g.n16, (long long)g.rows);
  if ((int64_t)g.T * p->nfft > (int64_t)1 << 33)
    return fail(PESQ_ERR_INVALID_ARGUMENT, "%d frames of %d samples: too many for one call", g.T, p->nfft);
  g.L = (g.T - 20) / 10 + 1;
  g.nb = p->nb;
  g.general = p->general;
  g.nfreq = p->general ? p->gen.nfreq : kBins;
  balance(g.n16, kMaxSegFrames, g.seg, g.nseg);
  balance(g.n16, kBackSegFrames, g.seg_b, g.nseg_b);
  g.seg_f = g.seg;
  g.nseg_f = g.nseg;
  g.front_threads = kThreads;
  if (!p->general) {
    // Half-size front CTAs (two per SM, segments of at most kMaxSegFramesHalf
    // frames) unless the full-size ones fit one wave and the half-size ones
    // do not (the 8 x 8 s batch: 144 full-size CTAs in 32.8 us against 304
    // half-size ones in 42.8 us).  A small batch gains from the shorter
    // segments' extra CTAs (8 x 3 s: 29.4 -> 22.6 us, 1 x 1 s: 26.7 -> 20.6
    // us), a large one from two CTAs per SM overlapping their phases.
    int seg_h = 0, nseg_h = 0;
    balance(g.n16, kMaxSegFramesHalf, seg_h, nseg_h);
    const int64_t sms = std::max(1, p->sms);
    const bool full_one_wave = g.rows * g.nseg <= (int64_t)kManyWaves * sms;
    const bool half_one_wave = g.rows * nseg_h <= 2 * (int64_t)kManyWaves * sms;
    if (!full_one_wave || half_one_wave) {
      g.seg_f = seg_h;
      g.nseg_f = nseg_h;
      g.front_threads = kThreads / 2;
    }
  }
  // Chain cluster size (CTAs per utterance; the results do not depend on it):
  // slices of at most kChainSliceMax frames, and for small batches enough
  // CTAs per utterance to reach kChainFillCtas in all -- the rest of the SMs
  // run the align kernel beside the chain adjoint -- with slices of at least
  // kChainSliceMin frames and at most 8 CTAs (a portable cluster).  Larger
  // slices amortise each CTA's fixed cost (its cluster reductions and the
  // staging of the tables) once the batch fills the GPU.  Measured steps
  // (graph replay, fwd+bwd): 512 x 3 s 1.196 -> 1.133 ms with 2 CTAs
  // instead of 3, 64 x 3 s 0.205 -> 0.199 ms, 4 x 3 s 0.088 -> 0.082 ms
  // with 6, 1 x 1 s 0.086-0.090 -> 0.082-0.084 ms with 2; 128 x 6 s best
  // with 4 (0.596 ms; 0.610 with 2, 0.627 with 3), 64 x 10 s at 48 kHz
  // with 6 or 8 (0.797 ms; odd sizes 5 and 7 measured slower there).
  g.cluster = (int)std::max<int64_t>(ceil_div(g.T, kChainSliceMax), ceil_div(kChainFillCtas, std::max<int64_t>(batch, 1)));
  g.cluster = (int)std::min<int64_t>({(int64_t)g.cluster, 8, std::max<int64_t>(1, ceil_div(g.T, kChainSliceMin))});
  g.cluster = std::max(g.cluster, 1);
  // a long utterance whose 8-CTA slices do not fit the chain backward's
  // shared memory layout takes the smallest larger cluster (up to 16) whose
  // slices fit, unless the device runs fewer of those at once than it
  // needs for the batch in as many waves as with 8
  if (g.cluster == 8 && chain_bwd_smem_bytes(chain_slice_frames(g.T, 8), p->nb) > chain_smem_limit()) {
    const int64_t waves8 = ceil_div(std::max<int64_t>(batch, 1), std::max(1, p->active_clusters[8]));
    for (int c = 9; c <= 16; ++c) {
      if (p->active_clusters[c] < 1 ||
          chain_bwd_smem_bytes(chain_slice_frames(g.T, c), p->nb) > chain_smem_limit() ||
          ceil_div(std::max<int64_t>(batch, 1), p->active_clusters[c]) > waves8)
        continue;
      g.cluster = c;
      break;
    }
  }
  {
    const int slice = chain_slice_frames(g.T, g.cluster);
    g.fwd_staged = chain_fwd_smem_bytes(slice, p->nb, false) <= chain_smem_limit();
    g.fwd_stage_cells = chain_fwd_smem_bytes(slice, p->nb, true) <= chain_smem_limit();
    g.bwd_stage_cells = chain_bwd_smem_bytes(slice, p->nb, true) <= chain_smem_limit();
    g.bwd_staged = chain_bwd_smem_bytes(slice, p->nb, false) <= chain_smem_limit();
    // many waves of clusters: two CTAs per SM, the coefficients through L2
    g.chain_dual = !p->general && g.batch * g.cluster > (int64_t)kManyWaves * std::max(1, p->sms) &&
                   g.fwd_staged && g.bwd_staged && chain_dual_fits(slice, p->nb);
    if (g.chain_dual) g.fwd_stage_cells = g.bwd_stage_cells = false;
  }
  // every kernel folds rows x segments (or utterances x cluster CTAs) onto
  // grid x; the resampler launches at most 65535 rows at a time in grid y
  if (g.rows * g.nseg_b > INT32_MAX || g.rows * g.nseg_f > INT32_MAX || g.batch * g.cluster > INT32_MAX)
    return fail(PESQ_ERR_INVALID_ARGUMENT, "batch too large for one call (%lld rows of %d segments)",
                (long long)g.rows, g.nseg);
  g.grad = (flags & (PESQ_GRAD_REF | PESQ_GRAD_DEG)) != 0;
  g.grad_begin = (flags & PESQ_GRAD_REF) ? 0 : (int)batch;
  g.grad_end = (flags & PESQ_GRAD_DEG) ? (int)g.rows : (int)batch;
  g.lay = ChainLayout::make(g.T, g.nb);

  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o += (bytes + 255) & ~(size_t)255;
    return at;
  };
  const size_t rows = (size_t)g.rows;
  g.x16 = take(g.resample ? rows * g.n16 * 4 : 0);
  g.x16lo = take(g.resample ? rows * g.n16 * 4 : 0);
  g.partial = take(rows * g.nseg_f * 8);
  g.sumsq = take(rows * 8);
  g.bark = take(rows * (size_t)g.T * g.nb * 4);
  g.fpow = take(g.grad ? rows * g.n16 * 4 : 0);
  g.z = take(g.grad ? rows * g.n16 * 4 : 0);
  g.spec = take(g.grad ? rows * (size_t)g.T * g.nfreq * 8 : 0);
  g.saved = take((size_t)batch * g.lay.stride * 4);
  g.cell_stride = (int64_t)batch * g.cluster * cell_block(g.T, g.cluster, g.nb);
  g.cells = take(g.grad ? (size_t)kCellFields * g.cell_stride * 4 : 0);
  g.gbark = take(g.grad ? rows * (size_t)g.T * g.nb * 4 : 0);
  g.kappa = take(g.grad ? rows * 4 : 0);
  g.cscratch = take(g.grad ? (size_t)batch * 2 * g.T * 4 : 0);
  g.gx16 = take(g.grad && g.resample ? rows * g.n16 * 4 : 0);
  g.y64 = take(g.general ? rows * g.n16 * 8 : 0);
  g.fgrad = take(g.grad && g.general ? (size_t)(g.grad_end - g.grad_begin) * g.T * p->nfft * 4 : 0);
  g.lsum = take(32);  // double[2] batch loss sum and count, uint32 arrival counter at +16
  g.total = o;
  return PESQ_OK;
}

template <class T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

int check_call(const pesq_plan* p, const Geometry& g, void* ws, size_t ws_bytes) {
  if (!ws && g.total) return fail(PESQ_ERR_WORKSPACE, "workspace is NULL");
  if (ws_bytes < g.total)
    return fail(PESQ_ERR_WORKSPACE, "workspace of %zu bytes, the call needs %zu", ws_bytes, g.total);
  if (((uintptr_t)ws & 255) != 0) return fail(PESQ_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != p->device)
    return fail(PESQ_ERR_INVALID_ARGUMENT, "plan lives on device %d but device %d is current", p->device, dev);
  return PESQ_OK;
}

}  // namespace

namespace pesq {
// Records `msg` as the calling thread's last error (used by the entry points
// that live in other translation units) and returns `code`.
int set_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace pesq

extern "C" {

int pesq_abi_version(void) { return PESQ_CUDA_ABI_VERSION; }

const char* pesq_last_error(void) { return g_error.c_str(); }

int pesq_plan_create(const pesq_plan_desc* d, pesq_plan** out) {
  g_error.clear();
  if (!d || !out) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  *out = nullptr;
  if (d->abi_version != PESQ_CUDA_ABI_VERSION)
    return fail(PESQ_ERR_UNSUPPORTED, "ABI version %d, library has %d", d->abi_version, PESQ_CUDA_ABI_VERSION);
  if (d->n_fft < kGenMinFft || d->n_fft > kGenMaxFft || (d->n_fft & (d->n_fft - 1)) != 0)
    return fail(PESQ_ERR_UNSUPPORTED, "n_fft %d: the kernels implement powers of two from %d to %d", d->n_fft,
                kGenMinFft, kGenMaxFft);
  if (d->hop_length < 1) return fail(PESQ_ERR_INVALID_ARGUMENT, "hop_length %d must be positive", d->hop_length);
  if (d->nbarks < 1 || d->nbarks > kMaxBands)
    return fail(PESQ_ERR_UNSUPPORTED, "%d Bark bands, the kernels support 1..%d", d->nbarks, kMaxBands);
  if (d->sample_rate <= 0) return fail(PESQ_ERR_INVALID_ARGUMENT, "sample rate must be positive");
  if (!d->window || !d->band_start || !d->band_end || !d->band_corr || !d->threshold || !d->exponent || !d->width)
    return fail(PESQ_ERR_INVALID_ARGUMENT, "missing table");

  pesq_plan* p = new pesq_plan();
  memset(p, 0, sizeof(*p));
  auto bail = [&](int code) {
    pesq_plan_destroy(p);
    return code;
  };
  if (cudaGetDevice(&p->device) != cudaSuccess) return bail(fail(PESQ_ERR_CUDA, "no CUDA device"));
  p->sample_rate = d->sample_rate;
  p->nb = d->nbarks;
  p->nfft = d->n_fft;
  p->hop = d->hop_length;
  p->general = d->n_fft != kNfft || d->hop_length != kHop;
  const int nfreq = d->n_fft / 2;
  p->factor = d->factor;
  int rc = fill_scan(p->pow, d->power_filter, "power filter");
  if (rc) return bail(rc);
  // the kernels skip the structural zeros of the band pass's doubling
  // matrices (a series of second order sections: block lower triangular)
  for (int l = 0; l < kLevels; ++l)
    for (int i = 0; i < 10; ++i)
      for (int j = 0; j < 10; ++j)
        if ((j >> 1) > (i >> 1) && p->pow.M[l][i][j] != 0.0f)
          return bail(fail(PESQ_ERR_UNSUPPORTED,
                           "level-alignment filter: the state matrix must be block lower triangular in 2 x 2 blocks"));
  rc = fill_scan(p->pre, d->pre_filter, "pre-emphasis filter");
  if (rc) return bail(rc);
  rc = fill_scan(p->pre64, d->pre_filter, "pre-emphasis filter");
  if (rc) return bail(rc);
  // the back kernel folds in kBackHorizon samples of look-ahead of the
  // pre-emphasis adjoint and drops the rest, which A^kBackHorizon bounds
  if (!(power_norm(d->pre_filter.trans, 2, kBackHorizon) < 1e-9))
    return bail(fail(PESQ_ERR_UNSUPPORTED, "pre-emphasis filter: its impulse response decays too slowly for the "
                                           "%d-sample look-ahead of the backward", kBackHorizon));

  // constant tables
  DevTables h;
  memset(&h, 0, sizeof(h));
  if (!p->general)
    for (int k = 0; k < kNfft; ++k) h.window[k] = (float)d->window[k];
  DevTwiddle64 h64;
  // exp(-2 pi i k / n); the argument reduction k mod n, k / n is exact in double
  auto root = [](int k, int n, Cx<double>& w64, Cx<float>& w32) {
    const double t = -2.0 * M_PI * ((double)(k % n) / (double)n);
    w64.x = cos(t);
    w64.y = sin(t);
    w32.x = (float)w64.x;
    w32.y = (float)w64.y;
  };
  for (int q = 1; q < 8; ++q)
    for (int l = 0; l < 32; ++l) root(l * q, 256, h64.lane[q - 1][l], h.fft.lane[q - 1][l]);
  for (int r = 0; r < 4; ++r)
    for (int j = 0; j < 8; ++j) root(r * j, 32, h64.quarter[r][j], h.fft.quarter[r][j]);
  for (int k = 0; k < 256; ++k) {
    root(k, 512, h64.bin[k], h.fft.bin[k]);
    h.bin_band[k] = -1;
  }
  int prev_end = 0;
  for (int b = 0; b < d->nbarks; ++b) {
    const int s = d->band_start[b], e = d->band_end[b];
    if (s < 0 || e < s || e > nfreq || s < prev_end)
      return bail(fail(PESQ_ERR_INVALID_ARGUMENT, "band %d covers [%d, %d): bands must be sorted, disjoint and below bin %d",
                       b, s, e, nfreq));
    prev_end = e;
    h.band_start[b] = s;
    h.band_end[b] = e;
    if (!p->general)
      for (int f = std::max(s, 1); f < e; ++f) h.bin_band[f] = b;
    const double th = d->threshold[b], ex = d->exponent[b];
    if (!(th > 0.0)) return bail(fail(PESQ_ERR_INVALID_ARGUMENT, "hearing thresholds must be positive"));
    h.band_corr[b] = (float)d->band_corr[b];
    h.thresh[b] = (float)th;
    h.inv2th[b] = (float)(0.5 / (double)(float)th);
    h.expo[b] = (float)ex;
    const double ls = d->loudness_sl * pow(2.0 * th, ex);
    h.loud_scale[b] = (float)ls;
    h.dloud_scale[b] = (float)(ls * ex * 0.5 / th);
    h.width[b] = (float)d->width[b];
    h.width_sq[b] = (float)(d->width[b] * d->width[b]);
  }
  h.nb = d->nbarks;
  h.total_width = (float)d->total_width;
  h.sqrt_total_width = (float)sqrt(d->total_width);

  if (cudaMalloc(&p->dtab, sizeof(DevTables)) != cudaSuccess)
    return bail(fail(PESQ_ERR_CUDA, "cudaMalloc of the constant tables failed"));
  if (cudaMemcpy(p->dtab, &h, sizeof(h), cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(fail(PESQ_ERR_CUDA, "upload of the constant tables failed"));
  if (cudaMalloc(&p->tw64, sizeof(DevTwiddle64)) != cudaSuccess ||
      cudaMemcpy(p->tw64, &h64, sizeof(h64), cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(fail(PESQ_ERR_CUDA, "upload of the twiddle tables failed"));

  // general frame geometry: window, twiddles exp(-2 pi i k / n_fft) and the
  // band of every bin, in one device buffer
  if (p->general) {
    const int n = d->n_fft;
    const size_t tw_bytes = (size_t)(n / 2) * sizeof(Cx<double>), win_bytes = (size_t)n * 4;
    const size_t band_bytes = (size_t)nfreq * 4;
    std::vector<char> host(tw_bytes + win_bytes + band_bytes);
    Cx<double>* tw = reinterpret_cast<Cx<double>*>(host.data());
    float* win = reinterpret_cast<float*>(host.data() + tw_bytes);
    int* band = reinterpret_cast<int*>(host.data() + tw_bytes + win_bytes);
    for (int k = 0; k < n / 2; ++k) {
      const double t = -2.0 * M_PI * ((double)k / (double)n);
      tw[k].x = cos(t);
      tw[k].y = sin(t);
    }
    for (int k = 0; k < n; ++k) win[k] = (float)d->window[k];
    for (int f = 0; f < nfreq; ++f) band[f] = -1;
    for (int b = 0; b < d->nbarks; ++b)
      for (int f = std::max(d->band_start[b], 1); f < d->band_end[b]; ++f) band[f] = b;
    if (cudaMalloc(&p->gen_buf, host.size()) != cudaSuccess ||
        cudaMemcpy(p->gen_buf, host.data(), host.size(), cudaMemcpyHostToDevice) != cudaSuccess)
      return bail(fail(PESQ_ERR_CUDA, "upload of the spectrum tables failed"));
    char* dev = static_cast<char*>(p->gen_buf);
    p->gen.nfft = n;
    p->gen.log2n = 0;
    while ((1 << p->gen.log2n) < n) ++p->gen.log2n;
    p->gen.hop = d->hop_length;
    p->gen.nfreq = nfreq;
    p->gen.tw = reinterpret_cast<const Cx<double>*>(dev);
    p->gen.window = reinterpret_cast<const float*>(dev + tw_bytes);
    p->gen.bin_band = reinterpret_cast<const int*>(dev + tw_bytes + win_bytes);
  }

  if (cudaMalloc(&p->err, 16) != cudaSuccess || cudaMemset(p->err, 0, 16) != cudaSuccess)
    return bail(fail(PESQ_ERR_CUDA, "allocating the error word"));

  // resampler tables
  p->resample = d->sample_rate != 16000;
  if (p->resample) {
    const char* msg = build_resample_tables(d->rs_orig_step, d->rs_new_step, d->rs_width, d->rs_width_total,
                                            d->rs_taps, p->rs);
    if (msg) return bail(fail(PESQ_ERR_INVALID_ARGUMENT, "%s", msg));
  }

  cudaError_t e = configure_front();
  if (e != cudaSuccess) return bail(cuda_fail(e, "configuring the front kernel"));
  e = configure_back();
  if (e != cudaSuccess) return bail(cuda_fail(e, "configuring the back kernel"));
  e = configure_chain();
  if (e != cudaSuccess) return bail(cuda_fail(e, "configuring the chain kernels"));
  for (int c = 8; c <= 16; ++c) p->active_clusters[c] = chain_active_clusters(c);
  if (cudaDeviceGetAttribute(&p->sms, cudaDevAttrMultiProcessorCount, p->device) != cudaSuccess) p->sms = 1;
  e = configure_align();
  if (e != cudaSuccess) return bail(cuda_fail(e, "configuring the align kernel"));
  e = configure_spectrum();
  if (e != cudaSuccess) return bail(cuda_fail(e, "configuring the spectrum kernels"));
  *out = p;
  return PESQ_OK;
}

int pesq_plan_destroy(pesq_plan* p) {
  if (!p) return PESQ_OK;
  cudaFree(p->dtab);
  cudaFree(p->tw64);
  cudaFree(p->gen_buf);
  cudaFree(p->err);
  free_resample_tables(p->rs);
  delete p;
  return PESQ_OK;
}

int pesq_plan_check(const pesq_plan* p, void* stream, uint32_t* flags) {
  if (!p || !flags) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, p->err, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(p->err, 0, 4, s);
  if (e != cudaSuccess) return cuda_fail(e, "pesq_plan_check");
  *flags = v;
  return PESQ_OK;
}

int pesq_plan_device(const pesq_plan* p, int* device) {
  if (!p || !device) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  *device = p->device;
  return PESQ_OK;
}

int pesq_query_shape(const pesq_plan* p, int64_t n_src, pesq_shape* s) {
  if (!p || !s) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  Geometry g;
  const int rc = geometry(p, 1, n_src, 0, g);
  if (rc) return rc;
  s->n16 = g.n16;
  s->frames = g.T;
  s->windows = g.L;
  return PESQ_OK;
}

int pesq_workspace_size(const pesq_plan* p, int64_t batch, int64_t n_src, uint32_t flags, size_t* bytes) {
  if (!p || !bytes) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  Geometry g;
  const int rc = geometry(p, batch, n_src, flags, g);
  if (rc) return rc;
  *bytes = g.total;
  return PESQ_OK;
}

int pesq_loss_sum_offset(const pesq_plan* p, int64_t batch, int64_t n_src, uint32_t flags, size_t* offset) {
  if (!p || !offset) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  Geometry g;
  const int rc = geometry(p, batch, n_src, flags, g);
  if (rc) return rc;
  *offset = g.lsum;
  return PESQ_OK;
}

int pesq_forward_front(const pesq_plan* p, void* stream, const void* ref_in, int64_t ld_ref, const void* deg_in,
                       int64_t ld_deg, int64_t batch, int64_t n_src, uint32_t flags, void* ws, size_t ws_bytes) {
  // the caller's rows; 16-bit rows are widened to float as the first kernel reads them
  const float* ref = static_cast<const float*>(ref_in);
  const float* deg = static_cast<const float*>(deg_in);
  const int in_type = (flags & PESQ_INPUT_BF16) ? kInBF16 : (flags & PESQ_INPUT_F16) ? kInF16 : kInF32;
  if (!p) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL plan");
  Geometry g;
  int rc = geometry(p, batch, n_src, flags, g);
  if (rc) return rc;
  if (batch == 0) return PESQ_OK;
  if (!ref || !deg) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL input");
  if (ld_ref < n_src || ld_deg < n_src) return fail(PESQ_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
  rc = check_call(p, g, ws, ws_bytes);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  RowSource src16{ref, deg, ld_ref, ld_deg, (int)batch, in_type};
  RowSource lo16{nullptr, nullptr, 0, 0, (int)batch};
  if (g.resample) {
    float* x16 = at<float>(ws, g.x16);
    float* x16lo = at<float>(ws, g.x16lo);
    ResampleArgs ra = resample_args(p->rs, n_src, g.n16);
    ra.src = RowSource{ref, deg, ld_ref, ld_deg, (int)batch, in_type};
    ra.dst = RowSink{x16, x16 + batch * g.n16, g.n16, g.n16, (int)batch};
    ra.dst_lo = RowSink{x16lo, x16lo + batch * g.n16, g.n16, g.n16, (int)batch};
    ra.rows = (int)g.rows;
    ra.row_begin = 0;
    PESQ_CUDA_TRY(launch_resample_fwd(ra, s), "resample kernel");
    src16 = RowSource{x16, x16 + batch * g.n16, g.n16, g.n16, (int)batch};
    lo16 = RowSource{x16lo, x16lo + batch * g.n16, g.n16, g.n16, (int)batch};
  }

  FrontArgs fa{};
  fa.src = src16;
  fa.src_lo = lo16;
  fa.n = g.n16;
  fa.frames = g.T;
  fa.seg_frames = g.seg_f;
  fa.nseg = g.nseg_f;
  fa.threads = g.front_threads;
  fa.spec_begin = g.grad ? g.grad_begin : 0;
  fa.spec_end = g.grad ? g.grad_end : 0;
  fa.tab = p->dtab;
  fa.tw64 = p->tw64;
  fa.bark = at<float>(ws, g.bark);
  fa.partial = at<double>(ws, g.partial);
  fa.spec = at<Cx<float>>(ws, g.spec);
  fa.fpow = at<float>(ws, g.fpow);
  fa.err = p->err;
  fa.done = at<uint32_t>(ws, g.lsum + 16);
  fa.y64 = g.general ? at<double>(ws, g.y64) : nullptr;
  PESQ_CUDA_TRY(launch_front(fa, p->pow, p->pre64, (int)g.rows, s), "front kernel");
  if (g.general) {
    SpecArgs sa{};
    sa.g = p->gen;
    sa.tab = p->dtab;
    sa.tw512 = p->tw64;
    sa.n = g.n16;
    sa.frames = g.T;
    sa.rows = (int)g.rows;
    sa.row_begin = 0;
    sa.y = fa.y64;
    sa.bark = fa.bark;
    sa.spec = fa.spec;
    sa.spec_begin = fa.spec_begin;
    sa.spec_end = fa.spec_end;
    PESQ_CUDA_TRY(launch_stft(sa, s), "spectrum kernel");
  }
  return PESQ_OK;
}

int pesq_forward_chain(const pesq_plan* p, void* stream, int64_t batch, int64_t n_src, uint32_t flags, void* ws,
                       size_t ws_bytes, float* d_symm, float* d_asymm, float* mos, float* loss) {
  if (!p) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL plan");
  Geometry g;
  int rc = geometry(p, batch, n_src, flags, g);
  if (rc) return rc;
  if (batch == 0) return PESQ_OK;
  rc = check_call(p, g, ws, ws_bytes);
  if (rc) return rc;
  ChainFwdArgs ca{};
  ca.batch = (int)batch;
  ca.nseg = g.nseg_f;
  ca.n = g.n16;
  ca.tab = p->dtab;
  ca.bark = at<float>(ws, g.bark);
  ca.partial = at<double>(ws, g.partial);
  ca.sumsq = at<double>(ws, g.sumsq);
  ca.saved = at<float>(ws, g.saved);
  ca.lay = g.lay;
  ca.factor = p->factor;
  ca.d_symm = d_symm;
  ca.d_asymm = d_asymm;
  ca.mos = mos;
  ca.loss = loss;
  ca.loss_sum = at<double>(ws, g.lsum);
  ca.done = at<uint32_t>(ws, g.lsum + 16);
  ca.staged = g.fwd_staged;
  ca.dual = g.chain_dual;
  ca.cells = g.grad ? at<float>(ws, g.cells) : nullptr;
  ca.cell_stride = g.cell_stride;
  ca.stage_cells = g.fwd_stage_cells;
  PESQ_CUDA_TRY(launch_chain_fwd(ca, g.cluster, static_cast<cudaStream_t>(stream)), "chain forward kernel");
  return PESQ_OK;
}

int pesq_forward(const pesq_plan* p, void* stream, const void* ref, int64_t ld_ref, const void* deg,
                 int64_t ld_deg, int64_t batch, int64_t n_src, uint32_t flags, void* ws, size_t ws_bytes,
                 float* d_symm, float* d_asymm, float* mos, float* loss) {
  const int rc = pesq_forward_front(p, stream, ref, ld_ref, deg, ld_deg, batch, n_src, flags, ws, ws_bytes);
  if (rc) return rc;
  return pesq_forward_chain(p, stream, batch, n_src, flags, ws, ws_bytes, d_symm, d_asymm, mos, loss);
}

int pesq_backward_chain(const pesq_plan* p, void* stream, int64_t batch, int64_t n_src, uint32_t flags, void* ws,
                        size_t ws_bytes, const float* g_loss, const float* g_mos, const float* g_dsymm,
                        const float* g_dasymm) {
  if (!p) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL plan");
  Geometry g;
  int rc = geometry(p, batch, n_src, flags, g);
  if (rc) return rc;
  if (!g.grad) return fail(PESQ_ERR_INVALID_ARGUMENT, "backward without PESQ_GRAD_REF or PESQ_GRAD_DEG");
  if (batch == 0) return PESQ_OK;
  rc = check_call(p, g, ws, ws_bytes);
  if (rc) return rc;
  ChainBwdArgs cb{};
  cb.batch = (int)batch;
  cb.tab = p->dtab;
  cb.bark = at<float>(ws, g.bark);
  cb.sumsq = at<double>(ws, g.sumsq);
  cb.saved = at<float>(ws, g.saved);
  cb.scratch = at<float>(ws, g.cscratch);
  cb.lay = g.lay;
  cb.factor = p->factor;
  cb.g_loss = g_loss;
  cb.g_mos = g_mos;
  cb.g_dsymm = g_dsymm;
  cb.g_dasymm = g_dasymm;
  cb.g_stride = (flags & PESQ_UPSTREAM_SCALAR) ? 0 : 1;
  cb.want_ref = (flags & PESQ_GRAD_REF) != 0;
  cb.want_deg = (flags & PESQ_GRAD_DEG) != 0;
  cb.g_bark = at<float>(ws, g.gbark);
  cb.kappa = at<float>(ws, g.kappa);
  cb.staged = g.bwd_staged;
  cb.dual = g.chain_dual;
  cb.stage_cells = g.bwd_stage_cells;
  cb.cells = at<float>(ws, g.cells);
  cb.cell_stride = g.cell_stride;
  PESQ_CUDA_TRY(launch_chain_bwd(cb, g.cluster, static_cast<cudaStream_t>(stream)), "chain backward kernel");
  return PESQ_OK;
}

int pesq_backward_align(const pesq_plan* p, void* stream, int64_t batch, int64_t n_src, uint32_t flags, void* ws,
                        size_t ws_bytes) {
  if (!p) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL plan");
  Geometry g;
  int rc = geometry(p, batch, n_src, flags, g);
  if (rc) return rc;
  if (!g.grad) return fail(PESQ_ERR_INVALID_ARGUMENT, "backward without PESQ_GRAD_REF or PESQ_GRAD_DEG");
  if (batch == 0) return PESQ_OK;
  rc = check_call(p, g, ws, ws_bytes);
  if (rc) return rc;
  AlignArgs aa{};
  aa.fpow = at<float>(ws, g.fpow);
  aa.row_begin = g.grad_begin;
  aa.n = g.n16;
  aa.seg_frames = g.seg;
  aa.nseg = g.nseg;
  aa.z = at<float>(ws, g.z);
  PESQ_CUDA_TRY(launch_align(aa, p->pow, g.grad_end - g.grad_begin, static_cast<cudaStream_t>(stream)),
                "align kernel");
  return PESQ_OK;
}

int pesq_backward_back(const pesq_plan* p, void* stream, int64_t batch, int64_t n_src, uint32_t flags, void* ws,
                       size_t ws_bytes, float* g_ref, int64_t ld_gref, float* g_deg, int64_t ld_gdeg) {
  if (!p) return fail(PESQ_ERR_INVALID_ARGUMENT, "NULL plan");
  Geometry g;
  int rc = geometry(p, batch, n_src, flags, g);
  if (rc) return rc;
  if (!g.grad) return fail(PESQ_ERR_INVALID_ARGUMENT, "backward without PESQ_GRAD_REF or PESQ_GRAD_DEG");
  if (batch == 0) return PESQ_OK;
  if ((flags & PESQ_GRAD_REF) && (!g_ref || ld_gref < n_src))
    return fail(PESQ_ERR_INVALID_ARGUMENT, "missing dL/dref output");
  if ((flags & PESQ_GRAD_DEG) && (!g_deg || ld_gdeg < n_src))
    return fail(PESQ_ERR_INVALID_ARGUMENT, "missing dL/ddeg output");
  rc = check_call(p, g, ws, ws_bytes);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  float* gx16 = at<float>(ws, g.gx16);
  BackArgs ba{};
  ba.row_begin = g.grad_begin;
  ba.nb = g.nb;
  ba.n = g.n16;
  ba.frames = g.T;
  ba.seg_frames = g.seg_b;
  ba.nseg = g.nseg_b;
  // half-size CTAs (two per SM, the same results) from two waves of
  // full-size ones on
  ba.threads = (int64_t)(g.grad_end - g.grad_begin) * g.nseg_b > (int64_t)kManyWaves * std::max(1, p->sms)
                   ? kThreads / 2
                   : kThreads;
  ba.tab = p->dtab;
  ba.g_bark = at<float>(ws, g.gbark);
  ba.kappa = at<float>(ws, g.kappa);
  ba.z = at<float>(ws, g.z);
  ba.spec = at<Cx<float>>(ws, g.spec);
  ba.out = g.resample ? RowSink{gx16, gx16 + batch * g.n16, g.n16, g.n16, (int)batch}
                      : RowSink{g_ref, g_deg, ld_gref, ld_gdeg, (int)batch};
  ba.err = p->err;
  if (g.general) {
    SpecArgs sa{};
    sa.g = p->gen;
    sa.tab = p->dtab;
    sa.tw512 = p->tw64;
    sa.n = g.n16;
    sa.frames = g.T;
    sa.rows = g.grad_end - g.grad_begin;
    sa.row_begin = g.grad_begin;
    sa.spec = ba.spec ? const_cast<Cx<float>*>(ba.spec) : nullptr;
    sa.g_bark = ba.g_bark;
    sa.frame_grad = at<float>(ws, g.fgrad);
    PESQ_CUDA_TRY(launch_istft(sa, s), "spectrum adjoint kernel");
    ba.frame_grad = sa.frame_grad;
    ba.nfft = p->nfft;
    ba.hop = p->hop;
  }
  PESQ_CUDA_TRY(launch_back(ba, p->pre, g.grad_end - g.grad_begin, s), "back kernel");

  if (g.resample) {
    ResampleArgs ra = resample_args(p->rs, n_src, g.n16);
    ra.src = RowSource{gx16, gx16 + batch * g.n16, g.n16, g.n16, (int)batch};
    ra.dst = RowSink{g_ref, g_deg, ld_gref, ld_gdeg, (int)batch};
    ra.rows = g.grad_end - g.grad_begin;
    ra.row_begin = g.grad_begin;
    PESQ_CUDA_TRY(launch_resample_adj(ra, s), "resample adjoint kernel");
  }
  return PESQ_OK;
}

int pesq_backward(const pesq_plan* p, void* stream, const float* ref, int64_t ld_ref, const float* deg,
                  int64_t ld_deg, int64_t batch, int64_t n_src, uint32_t flags, void* ws, size_t ws_bytes,
                  const float* g_loss, const float* g_mos, const float* g_dsymm, const float* g_dasymm,
                  float* g_ref, int64_t ld_gref, float* g_deg, int64_t ld_gdeg) {
  (void)ref;
  (void)ld_ref;
  (void)deg;
  (void)ld_deg;
  int rc = pesq_backward_chain(p, stream, batch, n_src, flags, ws, ws_bytes, g_loss, g_mos, g_dsymm, g_dasymm);
  if (rc) return rc;
  rc = pesq_backward_align(p, stream, batch, n_src, flags, ws, ws_bytes);
  if (rc) return rc;
  return pesq_backward_back(p, stream, batch, n_src, flags, ws, ws_bytes, g_ref, ld_gref, g_deg, ld_gdeg);
}

}  // extern "C"
