// C ABI of the standalone IIR filter (the reference's TritonIIR,
// torch_pesq/triton_ops/iir.py:1266-1482): a filter object holds the tables of
// one state space realisation on one device; pesq_iir_filter is a
// stream-ordered launch over a [rows, n] float32 array, forwards in time or
// (PESQ_IIR_REVERSE) backwards, which is the filter's adjoint.
//
// The tables are derived here in float64 from (A, B, C, D), so any host can
// drive the filter through this file alone; the realisation itself is chosen
// by the caller (triton_pesq_b200/iir_design.py scores the candidates).
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <vector>

#include "../../include/pesq_cuda.h"
#include "iir.cuh"

namespace pesq {
int set_error(int code, const char* msg);
}  // namespace pesq

using namespace pesq::iir;
using pesq::set_error;

namespace pesq {
namespace iir {
#define PESQ_IIR_DECLARE(P)                                                         \
  extern template cudaError_t launch<P, false, false>(const Args&, const void*, cudaStream_t); \
  extern template cudaError_t launch<P, false, true>(const Args&, const void*, cudaStream_t);  \
  extern template cudaError_t launch<P, true, false>(const Args&, const void*, cudaStream_t);  \
  extern template cudaError_t launch<P, true, true>(const Args&, const void*, cudaStream_t);
PESQ_IIR_DECLARE(2)
PESQ_IIR_DECLARE(4)
PESQ_IIR_DECLARE(6)
PESQ_IIR_DECLARE(8)
PESQ_IIR_DECLARE(10)
PESQ_IIR_DECLARE(12)
PESQ_IIR_DECLARE(14)
PESQ_IIR_DECLARE(16)
PESQ_IIR_DECLARE(20)
PESQ_IIR_DECLARE(24)
}  // namespace iir
}  // namespace pesq

struct pesq_iir {
  int device = -1;
  int states = 0;         // realisation
  int kstates = 0;        // kernel instantiation (>= states)
  bool lower = false;     // A block lower triangular in 2 x 2 blocks
  std::vector<float> tab; // Tab<kstates> image
  float* lanes = nullptr;
  float* wpow = nullptr;
  double* look = nullptr;
  uint32_t* err = nullptr;
  uint32_t spin_limit = pesq::iir::kSpinLimit;
  double largest32 = 0.0, largest64 = 0.0;
  // ||A^kOverlap|| (max row sum) < kOverlapTol: long rows may run overlapped tiles
  bool overlap_ok = false;
};

namespace {

constexpr int kKernelStates[] = {2, 4, 6, 8, 10, 12, 14, 16, 20, 24};
// state an overlapped tile may drop after its kOverlap-sample warm-up, relative
// (the same bound as the loss path's level-alignment horizon)
constexpr double kOverlapTol = 1e-11;

using Mat = std::vector<double>;  // row-major P x P

Mat eye(int p) {
  Mat m((size_t)p * p, 0.0);
  for (int i = 0; i < p; ++i) m[(size_t)i * p + i] = 1.0;
  return m;
}
Mat mul(const Mat& a, const Mat& b, int p) {
  Mat c((size_t)p * p, 0.0);
  for (int i = 0; i < p; ++i)
    for (int k = 0; k < p; ++k) {
      const double v = a[(size_t)i * p + k];
      if (v == 0.0) continue;
      for (int j = 0; j < p; ++j) c[(size_t)i * p + j] += v * b[(size_t)k * p + j];
    }
  return c;
}
std::vector<double> matvec(const Mat& a, const std::vector<double>& v, int p) {
  std::vector<double> out(p, 0.0);
  for (int i = 0; i < p; ++i)
    for (int j = 0; j < p; ++j) out[i] += a[(size_t)i * p + j] * v[j];
  return out;
}
std::vector<double> vecmat(const std::vector<double>& v, const Mat& a, int p) {
  std::vector<double> out(p, 0.0);
  for (int i = 0; i < p; ++i)
    for (int j = 0; j < p; ++j) out[j] += v[i] * a[(size_t)i * p + j];
  return out;
}
double absmax(const Mat& m) {
  double r = 0.0;
  for (double v : m) {
    if (!std::isfinite(v)) return INFINITY;
    r = std::fmax(r, std::fabs(v));
  }
  return r;
}

// Host image of Tab<P> (a packed array of floats in declaration order).
struct TabLayout {
  int P;
  size_t h() const { return 0; }
  size_t G() const { return kL; }
  size_t W() const { return G() + (size_t)kL * P; }
  size_t M() const { return W() + (size_t)kL * P; }
  size_t A() const { return M() + (size_t)kLevels * P * P; }
  size_t B() const { return A() + (size_t)P * P; }
  size_t C() const { return B() + P; }
  size_t D() const { return C() + P; }
  size_t size() const { return D() + 1; }
};

void free_tables(pesq_iir* f) {
  cudaFree(f->lanes);
  cudaFree(f->wpow);
  cudaFree(f->look);
  cudaFree(f->err);
  f->lanes = nullptr;
  f->wpow = nullptr;
  f->look = nullptr;
  f->err = nullptr;
}

struct Geometry {
  int cpr, rows_per_tile, seg;
  int64_t tiles_per_row, tiles;
  bool overlap;  // overlapped tiles of long rows (no look-back, no workspace)
  bool chained() const { return tiles_per_row > 1; }
  bool lookback() const { return chained() && !overlap; }
};

// overlap: the filter allows overlapped tiles and the caller did not ask for
// the look-back
Geometry geometry(int64_t rows, int64_t n, bool overlap = false) {
  Geometry g{};
  const int64_t cpr = (n + kL - 1) / kL;
  if (cpr <= kThreads) {
    g.cpr = (int)cpr;
    g.rows_per_tile = kThreads / g.cpr;
    g.seg = g.cpr * kL;
    g.tiles_per_row = 1;
    g.tiles = (rows + g.rows_per_tile - 1) / g.rows_per_tile;
  } else {
    g.cpr = kThreads;
    g.rows_per_tile = 1;
    g.seg = kTile;
    g.overlap = overlap;
    const int64_t out = overlap ? kTile - kOverlap : kTile;  // outputs per tile
    g.tiles_per_row = (n + out - 1) / out;
    g.tiles = rows * g.tiles_per_row;
  }
  return g;
}

// chained rows: the tile ticket (16 bytes) and two published states of P
// components per tile, two tagged 64-bit words each; all zero before a launch
size_t workspace_bytes(const pesq_iir* f, const Geometry& g) {
  if (!g.lookback()) return 0;
  return 16 + (size_t)g.tiles * 2 * f->kstates * 2 * 8;
}

template <int P>
cudaError_t dispatch(const pesq_iir* f, const Args& a, bool rerun, cudaStream_t s) {
  const void* t = f->tab.data();
  if (f->lower) return rerun ? launch<P, true, true>(a, t, s) : launch<P, true, false>(a, t, s);
  return rerun ? launch<P, false, true>(a, t, s) : launch<P, false, false>(a, t, s);
}

}  // namespace

extern "C" {

int pesq_iir_create(const pesq_iir_desc* d, pesq_iir** out) {
  if (!d || !out) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  *out = nullptr;
  if (d->abi_version != PESQ_CUDA_ABI_VERSION) return set_error(PESQ_ERR_UNSUPPORTED, "ABI version mismatch");
  const int n = d->states;
  if (n < 1 || n > kMaxStates) return set_error(PESQ_ERR_UNSUPPORTED, "the IIR kernel handles 1 to 24 states");
  if (!d->trans || !d->input || !d->output) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL realisation");
  int P = 0;
  for (int k : kKernelStates)
    if (k >= n) {
      P = k;
      break;
    }
  // zero padded realisation
  Mat A((size_t)P * P, 0.0);
  std::vector<double> B(P, 0.0), C(P, 0.0);
  for (int i = 0; i < n; ++i) {
    for (int j = 0; j < n; ++j) A[(size_t)i * P + j] = d->trans[(size_t)i * n + j];
    B[i] = d->input[i];
    C[i] = d->output[i];
  }
  const double D = d->feed;
  for (double v : A)
    if (!std::isfinite(v)) return set_error(PESQ_ERR_INVALID_ARGUMENT, "non-finite transition matrix");
  for (int i = 0; i < P; ++i)
    if (!std::isfinite(B[i]) || !std::isfinite(C[i]))
      return set_error(PESQ_ERR_INVALID_ARGUMENT, "non-finite input or read-out vector");
  if (!std::isfinite(D)) return set_error(PESQ_ERR_INVALID_ARGUMENT, "non-finite feed-through");

  pesq_iir* f = new pesq_iir();
  if (cudaGetDevice(&f->device) != cudaSuccess) {
    delete f;
    return set_error(PESQ_ERR_CUDA, "no CUDA device");
  }
  f->states = n;
  f->kstates = P;
  f->lower = true;
  for (int i = 0; i < P; ++i)
    for (int j = 0; j < P; ++j)
      if ((j >> 1) > (i >> 1) && A[(size_t)i * P + j] != 0.0) f->lower = false;

  // chunk tables: G[t] = C A^t, W[k] = A^(L-1-k) B, h
  std::vector<std::vector<double>> G(kL), W(kL);
  Mat pw = eye(P);
  for (int t = 0; t < kL; ++t) {
    G[t] = vecmat(C, pw, P);
    pw = mul(A, pw, P);
  }
  const Mat chunk_step = pw;  // A^L
  Mat acc = eye(P);
  for (int k = kL - 1; k >= 0; --k) {
    W[k] = matvec(acc, B, P);
    acc = mul(A, acc, P);
  }
  std::vector<double> h(kL, 0.0);
  h[0] = D;
  for (int t = 1; t < kL; ++t)
    for (int j = 0; j < P; ++j) h[t] += G[t - 1][j] * B[j];
  std::vector<Mat> M(kLevels);
  Mat step = chunk_step;
  for (int i = 0; i < kLevels; ++i) {
    M[i] = step;
    step = mul(step, step, P);
  }
  std::vector<Mat> lanes(32);
  Mat cur = eye(P);
  for (int l = 0; l < 32; ++l) {
    lanes[l] = cur;
    cur = mul(chunk_step, cur, P);
  }
  const Mat wstep = cur;  // A^(32 L) = A^kOverlap
  double wnorm = 0.0;
  for (int i = 0; i < P; ++i) {
    double row = 0.0;
    for (int j = 0; j < P; ++j) row += std::fabs(wstep[(size_t)i * P + j]);
    wnorm = std::fmax(wnorm, row);
  }
  std::vector<Mat> wp(kWarps + 1);  // A^(32 L k), k = 0..kWarps
  wp[0] = eye(P);
  for (int w = 1; w <= kWarps; ++w) wp[w] = mul(wstep, wp[w - 1], P);
  const Mat tile_step = wp[kWarps];
  std::vector<double> look((size_t)(kFar + 1) * P * P);
  cur = eye(P);
  for (int k = 0; k <= kFar; ++k) {
    std::memcpy(look.data() + (size_t)k * P * P, cur.data(), sizeof(double) * P * P);
    cur = mul(tile_step, cur, P);
  }

  // float32 kernel parameter image
  TabLayout L{P};
  f->tab.assign(L.size(), 0.0f);
  double big32 = 0.0;
  auto put = [&](size_t off, double v) {
    f->tab[off] = (float)v;
  };
  for (int t = 0; t < kL; ++t) {
    put(L.h() + t, h[t]);
    for (int j = 0; j < P; ++j) {
      put(L.G() + (size_t)t * P + j, G[t][j]);
      put(L.W() + (size_t)t * P + j, W[t][j]);
      big32 = std::fmax(big32, std::fmax(std::fabs(G[t][j]), std::fabs(W[t][j])));
    }
  }
  for (int i = 0; i < kLevels; ++i) {
    for (size_t q = 0; q < (size_t)P * P; ++q) put(L.M() + (size_t)i * P * P + q, M[i][q]);
    big32 = std::fmax(big32, absmax(M[i]));
  }
  for (size_t q = 0; q < (size_t)P * P; ++q) put(L.A() + q, A[q]);
  big32 = std::fmax(big32, absmax(A));
  for (int j = 0; j < P; ++j) {
    put(L.B() + j, B[j]);
    put(L.C() + j, C[j]);
    big32 = std::fmax(big32, std::fmax(std::fabs(B[j]), std::fabs(C[j])));
  }
  put(L.D(), D);
  std::vector<float> lane_img((size_t)lane_floats(P), 0.0f);
  for (int l = 0; l < 32; ++l) {
    for (size_t q = 0; q < (size_t)P * P; ++q) lane_img[(size_t)l * lane_pitch(P) + q] = (float)lanes[l][q];
    big32 = std::fmax(big32, absmax(lanes[l]));
  }
  std::vector<float> wpow_img((size_t)wpow_floats(P), 0.0f);
  for (int w = 0; w <= kWarps; ++w) {
    for (size_t q = 0; q < (size_t)P * P; ++q) wpow_img[(size_t)w * P * P + q] = (float)wp[w][q];
    big32 = std::fmax(big32, absmax(wp[w]));
  }
  f->largest32 = big32;
  f->largest64 = absmax(look);
  f->overlap_ok = std::isfinite(wnorm) && wnorm < kOverlapTol;
  if (!std::isfinite(f->largest32) || !std::isfinite(f->largest64)) {
    delete f;
    return set_error(PESQ_ERR_INVALID_ARGUMENT, "the realisation's tables overflow");
  }

  cudaError_t e = cudaMalloc(&f->lanes, lane_img.size() * 4);
  if (e == cudaSuccess) e = cudaMalloc(&f->wpow, wpow_img.size() * 4);
  if (e == cudaSuccess) e = cudaMalloc(&f->look, sizeof(double) * look.size());
  if (e == cudaSuccess) e = cudaMalloc(&f->err, 16);
  if (e == cudaSuccess) e = cudaMemcpy(f->lanes, lane_img.data(), lane_img.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(f->wpow, wpow_img.data(), wpow_img.size() * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(f->look, look.data(), sizeof(double) * look.size(), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(f->err, 0, 16);
  if (e != cudaSuccess) {
    free_tables(f);
    delete f;
    return set_error(PESQ_ERR_CUDA, cudaGetErrorString(e));
  }
  *out = f;
  return PESQ_OK;
}

int pesq_iir_destroy(pesq_iir* f) {
  if (!f) return PESQ_OK;
  free_tables(f);
  delete f;
  return PESQ_OK;
}

int pesq_iir_query(const pesq_iir* f, pesq_iir_info* info) {
  if (!f || !info) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  info->states = f->states;
  info->kernel_states = f->kstates;
  info->block_lower = f->lower ? 1 : 0;
  info->chunk = kL;
  info->tile = kTile;
  info->largest32 = f->largest32;
  info->largest64 = f->largest64;
  info->overlap = f->overlap_ok ? kOverlap : 0;
  return PESQ_OK;
}

size_t pesq_iir_workspace_bytes(const pesq_iir* f, int64_t rows, int64_t n) {
  if (!f || rows <= 0 || n <= 0) return 0;
  // enough for either tiling (the look-back one needs it; PESQ_IIR_CHAINED
  // is a per-call flag)
  return workspace_bytes(f, geometry(rows, n));
}

int pesq_iir_filter(const pesq_iir* f, void* stream, const float* x, int64_t ld_x, int64_t rows, int64_t n,
                    float* y, int64_t ld_y, uint32_t flags, void* workspace, size_t workspace_bytes_) {
  if (!f) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL filter");
  if (rows < 0 || n < 0) return set_error(PESQ_ERR_INVALID_ARGUMENT, "negative rows or samples");
  if (flags & ~(uint32_t)(PESQ_IIR_REVERSE | PESQ_IIR_RERUN | PESQ_IIR_CHAINED))
    return set_error(PESQ_ERR_INVALID_ARGUMENT, "unknown flags");
  if (rows == 0 || n == 0) return PESQ_OK;
  if (!x || !y) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL signal");
  if (ld_x < n || ld_y < n) return set_error(PESQ_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != f->device) return set_error(PESQ_ERR_INVALID_ARGUMENT, "the filter lives on another device");
  const Geometry g = geometry(rows, n, f->overlap_ok && !(flags & PESQ_IIR_CHAINED));
  if (g.tiles > ((int64_t)1 << 31) - 1) return set_error(PESQ_ERR_INVALID_ARGUMENT, "more than 2^31 - 1 tiles");
  const size_t need = workspace_bytes(f, g);
  if (need > 0 && (!workspace || workspace_bytes_ < need))
    return set_error(PESQ_ERR_INVALID_ARGUMENT, "workspace missing or too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  Args a{};
  a.x = x;
  a.ld_x = ld_x;
  a.y = y;
  a.ld_y = ld_y;
  a.rows = rows;
  a.n = n;
  a.reverse = (flags & PESQ_IIR_REVERSE) ? 1 : 0;
  a.cpr = g.cpr;
  a.rows_per_tile = g.rows_per_tile;
  a.seg = g.seg;
  a.tiles_per_row = g.tiles_per_row;
  a.tiles = g.tiles;
  a.lanes = f->lanes;
  a.wpow = f->wpow;
  a.look = f->look;
  a.err = f->err;
  a.spin_limit = f->spin_limit;
  a.overlap = g.overlap ? kOverlap : 0;
  if (g.lookback()) {
    char* w = static_cast<char*>(workspace);
    a.ticket = reinterpret_cast<uint32_t*>(w);
    a.slots = reinterpret_cast<unsigned long long*>(w + 16);
    const cudaError_t e = cudaMemsetAsync(w, 0, need, s);
    if (e != cudaSuccess) return set_error(PESQ_ERR_CUDA, cudaGetErrorString(e));
  }
  const bool rerun = (flags & PESQ_IIR_RERUN) != 0;
  cudaError_t e = cudaErrorInvalidValue;
  switch (f->kstates) {
    case 2: e = dispatch<2>(f, a, rerun, s); break;
    case 4: e = dispatch<4>(f, a, rerun, s); break;
    case 6: e = dispatch<6>(f, a, rerun, s); break;
    case 8: e = dispatch<8>(f, a, rerun, s); break;
    case 10: e = dispatch<10>(f, a, rerun, s); break;
    case 12: e = dispatch<12>(f, a, rerun, s); break;
    case 14: e = dispatch<14>(f, a, rerun, s); break;
    case 16: e = dispatch<16>(f, a, rerun, s); break;
    case 20: e = dispatch<20>(f, a, rerun, s); break;
    case 24: e = dispatch<24>(f, a, rerun, s); break;
    default: break;
  }
  if (e != cudaSuccess) return set_error(PESQ_ERR_CUDA, cudaGetErrorString(e));
  return PESQ_OK;
}

int pesq_iir_set_spin_limit(pesq_iir* f, uint32_t polls) {
  if (!f) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  f->spin_limit = polls;
  return PESQ_OK;
}

int pesq_iir_check(pesq_iir* f, void* stream, uint32_t* failed) {
  if (!f || !failed) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, f->err, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaMemsetAsync(f->err, 0, 4, s);
  if (e != cudaSuccess) return set_error(PESQ_ERR_CUDA, cudaGetErrorString(e));
  *failed = v;
  return PESQ_OK;
}

}  // extern "C"
