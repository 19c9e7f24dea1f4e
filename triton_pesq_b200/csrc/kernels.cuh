// Launch-side declarations shared by the kernels and the C-ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fft.cuh"
#include "scan.cuh"

namespace pesq {

using PowTab = ScanTab<10>;
using PreTab = ScanTab<2>;
using PreTab64 = ScanTab<2, double>;

// Device constant tables of a plan (uploaded once, read-only afterwards).
struct alignas(16) DevTables {
  float window[kNfft];      // analysis window, zero padded/centred to n_fft
  FftTwiddles<float> fft;   // twiddles of the backward (single precision) transform
  int bin_band[kBins];         // band owning bin f, -1 if none (bin 0 never has one)
  int band_start[kMaxBands];
  int band_end[kMaxBands];
  float band_corr[kMaxBands];  // power density correction
  float thresh[kMaxBands];     // hearing threshold
  float inv2th[kMaxBands];     // 0.5 / threshold
  float expo[kMaxBands];       // loudness exponent
  float loud_scale[kMaxBands]; // Sl * (2 th)^e
  float dloud_scale[kMaxBands];// Sl * (2 th)^e * e * 0.5 / th
  float width[kMaxBands];      // band width in Bark
  float width_sq[kMaxBands];   // width^2
  int nb;
  float total_width;           // sum of widths of bands 1..nb-1
  float sqrt_total_width;
};

// Double precision twiddles of the forward spectrum.
using DevTwiddle64 = FftTwiddles<double>;

// Rows of one call: ref rows are 0..B-1, deg rows B..2B-1.
// Element type of a caller's input rows; every buffer of the engine itself is
// float32.
enum InputType : int { kInF32 = 0, kInBF16 = 1, kInF16 = 2 };

struct RowSource {
  const float* ref;
  const float* deg;
  int64_t ld_ref;  // row strides in elements
  int64_t ld_deg;
  int batch;
  int type = kInF32;  // caller rows only: bf16 / fp16 rows are widened to float as they are read
  // float rows
  __device__ __forceinline__ const float* row(int r) const {
    return r < batch ? ref + (int64_t)r * ld_ref : deg + (int64_t)(r - batch) * ld_deg;
  }
  // rows of any element type (read through load_elem)
  __device__ __forceinline__ const void* row_any(int r) const {
    const char* base = reinterpret_cast<const char*>(r < batch ? ref : deg);
    const int64_t off = r < batch ? (int64_t)r * ld_ref : (int64_t)(r - batch) * ld_deg;
    return base + off * (type == kInF32 ? 4 : 2);
  }
};

// Element i of a row of the given type, widened to float (exact for bf16 and
// fp16).
__device__ __forceinline__ float load_elem(const void* p, int64_t i, int type) {
  if (type == kInF32) return __ldg(static_cast<const float*>(p) + i);
  const unsigned short u = __ldg(static_cast<const unsigned short*>(p) + i);
  return type == kInBF16 ? __uint_as_float((unsigned)u << 16) : __half2float(__ushort_as_half(u));
}

struct RowSink {
  float* ref;
  float* deg;
  int64_t ld_ref;
  int64_t ld_deg;
  int batch;
  __device__ __forceinline__ float* row(int r) const {
    return r < batch ? ref + (int64_t)r * ld_ref : deg + (int64_t)(r - batch) * ld_deg;
  }
};

struct FrontArgs {
  RowSource src;     // 16 kHz rows
  RowSource src_lo;  // low parts of the resampled rows (x = hi + lo), ref == nullptr if none
  int64_t n;         // samples per row
  int frames;        // T
  int seg_frames;    // frames per segment
  int nseg;          // segments per row
  int threads;       // CTA size: kThreads, or kThreads / 2 (half spans, two CTAs per SM)
  int spec_begin;    // rows [spec_begin, spec_end) also save the spectrum X
  int spec_end;      // for the backward
  const DevTables* tab;
  const DevTwiddle64* tw64;
  float* bark;       // [rows][T][nb]   unscaled Bark spectrum
  double* partial;   // [rows][nseg]    partial sums of (H x)^2
  Cx<float>* spec;   // [rows][T][256]  rfft bins 0..255 of every frame
  float* fpow;       // [rows][n]       f = H x, written for the rows that save the spectrum
  uint32_t* err;
  uint32_t* done;    // arrival counter of the chain forward's batch sum, zeroed here
  // general frame geometry (n_fft / hop other than 512 / 256): the kernel
  // writes the pre-emphasised rows y here instead of evaluating the frames
  double* y64;       // [rows][n], or nullptr
};

// Frame geometry other than n_fft 512 / hop 256 (spectrum.cu): a warp per
// frame, an n_fft-point complex FFT in shared memory.
constexpr int kGenMinFft = 32;
constexpr int kGenMaxFft = 4096;
constexpr int kGenThreads = 256;

struct GenTables {
  int nfft, log2n, hop, nfreq;   // nfreq = n_fft / 2 bins (the Nyquist bin is never used)
  const float* window;           // [nfft] analysis window, zero padded/centred
  const Cx<double>* tw;          // [nfft / 2] exp(-2 pi i k / nfft)
  const int* bin_band;           // [nfreq] band owning bin f, -1 if none (bin 0 never has one)
};

struct SpecArgs {
  GenTables g;
  const DevTables* tab;
  const FftTwiddles<double>* tw512;  // n_fft 512: twiddles of the forward transform (the plan's)
  int64_t n;           // samples per row
  int frames;          // T
  int rows;            // rows (frames) of this launch: rows [row_begin, row_begin + rows)
  int row_begin;
  // forward: y -> Bark spectrum, and X on rows [spec_begin, spec_end)
  const double* y;     // [all rows][n]
  float* bark;         // [all rows][T][nb]
  Cx<float>* spec;     // [all rows][T][nfreq]
  int spec_begin, spec_end;
  // adjoint: dL/dBark and X -> windowed frame gradients
  const float* g_bark;  // [all rows][T][nb]
  float* frame_grad;    // [rows][T][nfft], row r at r - row_begin
};

struct AlignArgs {
  const float* fpow; // [rows][n]  f = H x saved by the front kernel (gradient rows)
  int row_begin;     // rows [row_begin, row_begin + rows) get z
  int64_t n;
  int seg_frames;
  int nseg;
  float* z;          // [rows][n]  H^T f
};

// Segmentation of the back kernel: at most kBackSegFrames hops of output per
// CTA (with the frame before the segment and the kBackHorizon samples after
// it, whose frames' gradients run back into the segment through the
// pre-emphasis adjoint: 32 frames, one per warp in each of the two parity
// passes of its overlap-add).  The gradient beyond the horizon reaches the
// segment through A_pre^768 (norm below 1e-9 for the pre-emphasis biquad,
// checked at plan creation), far below float32 rounding.
constexpr int kBackSegFrames = 28;
constexpr int kBackHorizon = 3 * kHop;

struct BackArgs {
  int row_begin;     // rows [row_begin, row_end) get a gradient
  int nb;            // Bark bands
  int64_t n;
  int frames;
  int seg_frames;
  int nseg;
  int threads;          // CTA size: kThreads, or kThreads / 2 (two CTAs per SM)
  const DevTables* tab;
  const float* g_bark;  // [rows][T][nb]  dL/d(unscaled Bark)
  const float* kappa;   // [rows]
  const float* z;       // [rows][n]
  const Cx<float>* spec;  // [rows][T][256] saved by the front kernel
  RowSink out;          // gradient rows (16 kHz)
  uint32_t* err;
  // general frame geometry: dL/dy is the overlap-add (a gather, in frame
  // order) of these windowed frame gradients instead of the fused transforms
  const float* frame_grad;  // [rows - row_begin][T][nfft], or nullptr
  int nfft, hop;
};

// Chain state saved by the forward for the backward, per utterance.
struct ChainLayout {
  int T;   // frames
  int L;   // psqm windows
  int nb;  // bands
  int64_t stride;  // floats per utterance
  // offsets (floats) of the per-utterance arrays
  int64_t keep, taer, tad, fpr0, fpr1, h, sraw, araw, sp, ap, gfpr, psqm_s, psqm_a;
  int64_t bpr, ratio, mref, mdeg, scal;
  static ChainLayout make(int T, int nb);
};

enum ChainScalar { kS2Ref = 0, kS2Deg, kDSymm, kDAsymm, kLoss, kNumScalars = 8 };

struct ChainFwdArgs {
  int batch;
  int nseg;                 // partial sums per row
  int64_t n;                // samples per row (for the power denominator)
  const DevTables* tab;
  const float* bark;        // [2B][T][nb]
  const double* partial;    // [2B][nseg]
  double* sumsq;            // [2B]  out
  float* saved;             // [B][layout.stride]
  ChainLayout lay;
  double factor;
  float* d_symm;            // [B] (nullable)
  float* d_asymm;
  float* mos;
  float* loss;
  // [sum of the batch's losses, batch] (float64), written by the cluster that
  // finishes last, which `done` (zeroed by the front kernel) identifies
  double* loss_sum;
  uint32_t* done;
  int staged;               // Bark slice staged in shared memory
  // per (frame, band) adjoint coefficients for the backward (nullable: no
  // gradient requested), see CellField and cell_block
  float* cells;
  int64_t cell_stride;
  int stage_cells;          // write them to shared memory first (when staged and they fit)
  int dual;                 // many-waves variant: two CTAs per SM (64 registers, cells unstaged)
};

// Layout of the adjoint coefficients: field f of frame t, band k of utterance
// u lives at f * cell_stride + (u * C + q) * cell_block(T, C, nb)
// + (t - c_lo) * nb + k, where q is the cluster rank whose frame slice
// [c_lo, c_hi) holds t: every CTA's block starts on a 16-byte boundary.
__host__ __device__ inline int64_t cell_block(int T, int C, int nb) {
  return ((int64_t)((T + C - 1) / C) * nb + 3) & ~(int64_t)3;
}

// Fields of the per (frame, band) record the forward chain saves for its
// adjoint: the disturbance, the clamped asymmetry factor and the derivatives
// of the two scaled spectra's gradients w.r.t. the gradients of those two,
//   g_ed = g_dist * ed_dist + g_asc * ed_asc,  g_er = g_dist * er_dist + g_asc * er_asc.
enum CellField { kCellDist = 0, kCellAsc, kCellEdDist, kCellEdAsc, kCellErDist, kCellErAsc, kCellFields };

struct ChainBwdArgs {
  int batch;
  const DevTables* tab;
  const float* bark;
  const double* sumsq;
  const float* saved;       // forward state (read only)
  float* scratch;           // [B][T] per-frame scratch (g_fpr)
  ChainLayout lay;
  double factor;
  const float* g_loss;      // [B] nullable
  const float* g_mos;       // [B] nullable
  const float* g_dsymm;     // [B] nullable
  const float* g_dasymm;    // [B] nullable
  int g_stride;             // element stride of the four upstream gradients (0: one shared value)
  int want_ref, want_deg;
  float* g_bark;            // [2B][T][nb]  out
  float* kappa;             // [2B]         out
  int staged;               // Bark slice and its gradients live in shared memory
  const float* cells;       // the forward's adjoint coefficients (see CellField)
  int64_t cell_stride;
  int stage_cells;          // (staged) the slice's coefficients are staged too, else read from L2
  int dual;                 // many-waves variant: two CTAs per SM (64 registers, cells unstaged)
};

struct ResampleArgs {
  RowSource src;        // source rows (fwd) / gradient of 16 kHz rows (adjoint)
  RowSink dst;
  RowSink dst_lo;       // forward only: float32 rounding residual of each output
  int rows;             // 2B or the gradient rows
  int row_begin;
  int64_t n_in;
  int64_t n_out;
  int orig_step, new_step, width, width_total;
  const float* taps;    // compact nonzero taps [new_step][max_count]
  const int* first;     // [new_step]
  const int* count;     // [new_step]
  int max_count;
  // adjoint gather lists per residue mod orig_step
  const int* adj_offset;   // [orig_step + 1]
  const int4* adj_entries; // (dl, phase, tap bits, 0)
  // the same lists residue-major for the staged adjoint: entry e of residue
  // rho at e * orig_step + rho, (dl << 24 | phase) or -1 past the end
  const int* adj_code;
  const float* adj_tap;
  int max_entries, max_dl;
  int fwd_staged, adj_staged;  // shared memory kernels (the tables fit)
  int tpitch;                  // odd row pitch of the staged taps
  uint32_t inv_os, inv_ns;     // ceil(2^32 / orig_step), ceil(2^32 / new_step): 32-bit divisions
  // float64 tensor-core forward (ResampleMma): 8 x 8 output tiles of
  // super-frames x consecutive super-phases
  const double* mma_b;  // B fragments [blocks][ksteps][32 lanes]
  const int* mma_s;     // first sample of each block's tap span in a super-frame window [blocks]
  int fwd_mma;          // 0, or the tile k-steps (taps / 4) of the kernel to run
  int mma_os, mma_ns;   // input samples / outputs per super-frame
  int mma_blocks;       // super-phases / 8
  int mma_span, mma_pitch, mma_frames, mma_warps;  // staged window: samples per super-frame, row pitch, rows; warps
  // float64 tensor-core adjoint: 8 x 8 tiles of super-frames x consecutive
  // residues, K = the block's (super-frame offset, super-phase) entries
  const double* amma_b;  // B fragments [k-steps of all blocks][32 lanes]
  const int* amma_a;     // A offsets in the staged window [k-steps][4]: -offset * pitch + super-phase
  const int* amma_off;   // first k-step of each block [blocks + 1]
  int adj_mma;           // tensor-core adjoint available
  int amma_os, amma_ns, amma_blocks, amma_pitch, amma_frames, amma_warps, amma_maxdl;
};

// Device tables of one polyphase resampler: the compact nonzero taps of every
// phase and the adjoint's per-residue gather lists, built on the host from
// float32-valued taps [new_step][width_total].
struct ResampleTables {
  int orig_step = 0, new_step = 0, width = 0, width_total = 0, max_count = 0;
  float* taps = nullptr;        // [new_step][max_count]
  int* first = nullptr;         // [new_step]
  int* count = nullptr;         // [new_step]
  int* adj_offset = nullptr;    // [orig_step + 1]
  int4* adj_entries = nullptr;  // (frame offset, phase, tap bits, 0)
  int* adj_code = nullptr;      // [max_entries][orig_step]
  float* adj_tap = nullptr;     // [max_entries][orig_step]
  int max_entries = 0, max_dl = 0;
  bool fwd_staged = false, adj_staged = false;
  // float64 tensor-core forward: G = 8 / gcd(new_step, 8) frames form a
  // super-frame of G * new_step outputs (a multiple of 8), whose super-phases
  // go in blocks of 8; each block's taps, shifted to a common first sample,
  // are the B operand of an m8n8k4 tile (zero outside each phase's span)
  double* mma_b = nullptr;  // [mma_blocks][fwd_mma][32]
  int* mma_s = nullptr;     // [mma_blocks]
  int fwd_mma = 0, mma_os = 0, mma_ns = 0, mma_blocks = 0;
  int mma_span = 0, mma_pitch = 0, mma_frames = 0, mma_warps = 0;
  // float64 tensor-core adjoint: G' frames (G' = 1 for orig_step >= 64, else
  // 8 / gcd(orig_step, 8)) form a super-frame of G' * orig_step input samples
  // (residues), taken in blocks of 8; a block's K operand lists the
  // (super-frame offset, super-phase) pairs whose taps reach any of its residues
  double* amma_b = nullptr;  // [k-steps][32]
  int* amma_a = nullptr;     // [k-steps][4]
  int* amma_off = nullptr;   // [amma_blocks + 1]
  bool adj_mma = false;
  int amma_os = 0, amma_ns = 0, amma_blocks = 0, amma_pitch = 0, amma_frames = 0, amma_warps = 0, amma_maxdl = 0;
};
// Allows the staged resampler kernels their shared memory (once per process).
cudaError_t configure_resample();
// Builds t on the current device; returns nullptr or a message.
const char* build_resample_tables(int orig_step, int new_step, int width, int width_total, const double* taps,
                                  ResampleTables& t);
void free_resample_tables(ResampleTables& t);
// Arguments of the resampler kernels for tables t, rows [row_begin, row_begin + rows).
ResampleArgs resample_args(const ResampleTables& t, int64_t n_in, int64_t n_out);
// Output length of the resampler: ceil(new_step * n / orig_step) evaluated
// on a float32 scalar, as torchaudio does.
int64_t resample_length(int orig_step, int new_step, int64_t n);

// Launch configuration of one kernel; `pdl` adds programmatic stream
// serialisation (the kernel may start while its predecessor on the stream
// runs, see pdl_wait), `cluster` > 0 a thread block cluster dimension.
struct LaunchShape {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[2];
  LaunchShape(unsigned blocks, unsigned threads, size_t smem, cudaStream_t s, bool pdl, int cluster = 0) {
    cfg = cudaLaunchConfig_t{};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    int n = 0;
    if (pdl) {
      attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[n].val.programmaticStreamSerializationAllowed = 1;
      ++n;
    }
    if (cluster > 0) {
      attr[n].id = cudaLaunchAttributeClusterDimension;
      attr[n].val.clusterDim.x = (unsigned)cluster;
      attr[n].val.clusterDim.y = 1;
      attr[n].val.clusterDim.z = 1;
      ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
  }
};

cudaError_t launch_front(const FrontArgs& a, const PowTab& pow, const PreTab64& pre, int rows, cudaStream_t s);
cudaError_t launch_back(const BackArgs& a, const PreTab& pre, int rows, cudaStream_t s);
// launched with programmatic stream serialisation: it may start while the
// preceding kernel on the stream runs, and completes after it
cudaError_t launch_align(const AlignArgs& a, const PowTab& pow, int rows, cudaStream_t s);
cudaError_t configure_align();
cudaError_t launch_stft(const SpecArgs& a, cudaStream_t s);
cudaError_t launch_istft(const SpecArgs& a, cudaStream_t s);
cudaError_t configure_spectrum();
cudaError_t launch_chain_fwd(const ChainFwdArgs& a, int cluster, cudaStream_t s);
cudaError_t launch_chain_bwd(const ChainBwdArgs& a, int cluster, cudaStream_t s);
cudaError_t configure_chain();
int chain_active_clusters(int cluster);  // chain clusters of that size the current device runs at once
// frames of the largest cluster slice, and the dynamic shared memory of the
// staged forward / backward chain kernels for it
int chain_slice_frames(int T, int cluster);
size_t chain_fwd_smem_bytes(int slice, int nb, bool cells);
size_t chain_bwd_smem_bytes(int slice, int nb, bool cells = true);
size_t chain_smem_limit();
// The many-waves chain variant (two CTAs per SM, coefficients unstaged) fits
// slices of `slice` frames.
bool chain_dual_fits(int slice, int nb);
cudaError_t launch_resample_fwd(const ResampleArgs& a, cudaStream_t s);
cudaError_t launch_resample_adj(const ResampleArgs& a, cudaStream_t s);

size_t front_smem_bytes(int threads);
size_t back_smem_bytes(int threads);
size_t align_smem_bytes();

}  // namespace pesq
