/*
 * pesq_cuda.h -- C ABI of the B200 PESQ loss engine (libpesq_cuda.so).
 *
 * The reference exposes this path only as the Python module
 * `PesqLossTriton` (torch_pesq/triton_ops/loss.py:18-215); there is no native
 * FFI in the reference.  The entry points below are the boundary a binding of
 * that module needs: a plan replaces the module constructor
 * (triton_ops/loss.py:60-92, which builds the stage modules and their host
 * float64 tables), pesq_forward replaces `raw` / `mos` / `forward`
 * (triton_ops/loss.py:104-147 and 203-215) and pesq_backward replaces the
 * autograd backward of the whole chain (the `backward` methods of
 * triton_ops/elementwise.py, resample.py, iir.py, spectral.py and chain.py).
 *
 * Conventions
 *   - every function returns a pesq_status (0 = success); no exception crosses
 *     the ABI; pesq_last_error() returns a message for the calling thread;
 *   - plain pointers and sizes only; all device pointers are CUDA device
 *     memory of the plan's device, all arrays row-major float32;
 *   - `stream` is a cudaStream_t (CUstream); every launch is stream-ordered,
 *     nothing synchronises and nothing allocates inside pesq_forward /
 *     pesq_backward, so both can be captured in a CUDA graph;
 *   - calls on distinct plans are thread safe; a plan is read only after
 *     creation and can be shared by concurrent calls with distinct workspaces.
 */
#ifndef PESQ_CUDA_H_
#define PESQ_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PESQ_CUDA_ABI_VERSION 2

typedef enum pesq_status {
  PESQ_OK = 0,
  PESQ_ERR_INVALID_ARGUMENT = 1, /* bad shape, pointer or flag; ValueError in Python */
  PESQ_ERR_UNSUPPORTED = 2,      /* configuration outside what the kernels implement */
  PESQ_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  PESQ_ERR_CUDA = 4,             /* a CUDA runtime call failed */
  PESQ_ERR_DEVICE = 5            /* a kernel reported an error flag */
} pesq_status;

/* flags of a forward / backward pair */
#define PESQ_GRAD_REF 1u /* the backward will be asked for dL/dref */
#define PESQ_GRAD_DEG 2u /* the backward will be asked for dL/ddeg */
/* backward only: each non-NULL upstream gradient (g_loss, g_mos, g_dsymm,
 * g_dasymm) points to ONE value shared by every utterance of the batch, as
 * the gradient of a sum or mean over the batch is; saves materialising it */
#define PESQ_UPSTREAM_SCALAR 4u
/* forward: element type of ref / deg (float32 without either flag).  Each
 * sample is widened to float as the first kernel reads it; everything after
 * runs in float32 / float64 exactly as for float32 inputs of the same values,
 * and the gradients of the backward are float32.  (The reference accepts
 * float32 only; this serves a caller training in mixed precision.) */
#define PESQ_INPUT_BF16 8u
#define PESQ_INPUT_F16 16u

typedef struct pesq_plan pesq_plan;

/* Constant tables of one causal LTI filter for the chunked scan, float64.
 * Built by triton_pesq_b200/tables.py (ScanTables); the state space is a
 * series of balanced second order sections, s[n+1] = A s[n] + B x[n],
 * y[n] = C s[n] + D x[n]. */
typedef struct pesq_scan_desc {
  int32_t states;        /* P: 10 for the level-alignment band pass, 2 for pre-emphasis */
  int32_t chunk;         /* samples per thread chunk, must be 33 */
  int32_t levels;        /* Kogge-Stone doubling levels, must be 5 */
  const double* impulse; /* [chunk]            h[t] */
  const double* carry;   /* [chunk * states]   C A^t */
  const double* drive;   /* [chunk * states]   A^(chunk-1-k) B */
  const double* power;   /* [levels * states * states]  A^(chunk 2^i) */
  const double* trans;   /* [states * states]  A */
  const double* input;   /* [states]           B */
  const double* output;  /* [states]           C */
  double feed;           /* D */
} pesq_scan_desc;

/* Everything `PesqLoss.__init__` (torch_pesq/loss.py:61-108) derives from its
 * arguments, as float64 host arrays.  Only read during pesq_plan_create. */
typedef struct pesq_plan_desc {
  int32_t abi_version; /* PESQ_CUDA_ABI_VERSION */
  int32_t sample_rate; /* input rate; 16000 skips the resampler */
  int32_t n_fft;       /* power of two in [32, 4096]; 512 runs the fused default path */
  int32_t hop_length;  /* >= 1; other than 256 (or n_fft other than 512) runs the spectrum kernels */
  int32_t nbarks;      /* 1 .. 64 (49 for P.862) */
  int32_t reserved0;
  double factor;       /* loss = factor * (0.1 d_symm + 0.0309 d_asymm) */
  const double* window;      /* [n_fft] analysis window, centred, zero padded */
  const int32_t* band_start; /* [nbarks] first bin of each Bark band (bands sorted, disjoint, below n_fft / 2) */
  const int32_t* band_end;   /* [nbarks] one past the last bin */
  const double* band_corr;   /* [nbarks] power density correction */
  const double* threshold;   /* [nbarks] absolute hearing threshold */
  const double* exponent;    /* [nbarks] Zwicker loudness exponent */
  const double* width;       /* [nbarks] band width in Bark */
  double total_width;        /* sum of width[1:] */
  double loudness_sl;        /* Sl calibration, 0.1866055 */
  pesq_scan_desc power_filter; /* level alignment band pass (states = 10) */
  pesq_scan_desc pre_filter;   /* pre-emphasis (states = 2) */
  int32_t rs_orig_step;  /* resampler: orig_freq / gcd      (sample_rate != 16000) */
  int32_t rs_new_step;   /*            16000 / gcd */
  int32_t rs_width;      /*            left zero padding */
  int32_t rs_width_total;/*            taps per phase */
  const double* rs_taps; /* [new_step * width_total] float32-valued taps */
} pesq_plan_desc;

/* Shape of one call. */
typedef struct pesq_shape {
  int64_t n16;     /* samples per row after resampling to 16 kHz */
  int32_t frames;  /* STFT frames (loss.py:191-196) */
  int32_t windows; /* 20-frame overlapping windows (loss.py:258-266) */
} pesq_shape;

int pesq_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* pesq_last_error(void);

/* Build a plan on the current CUDA device (uploads the constant tables).
 * Replaces PesqLossTriton.__init__ (triton_ops/loss.py:60-92). */
int pesq_plan_create(const pesq_plan_desc* desc, pesq_plan** plan);

int pesq_plan_destroy(pesq_plan* plan);

/* Synchronises `stream`, then reads and clears the plan's device error word:
 * nonzero (PESQ_DEVICE_* flags) when a kernel of an earlier call gave up a
 * bounded wait (a bulk copy into shared memory that did not complete in
 * time) -- the outputs of that call are then not valid.  The reference has
 * no device-side waits; its errors are Python exceptions on bad input. */
int pesq_plan_check(const pesq_plan* plan, void* stream, uint32_t* flags);
#define PESQ_DEVICE_BULK_TIMEOUT 1u

/* CUDA device ordinal the plan lives on. */
int pesq_plan_device(const pesq_plan* plan, int* device);

/* Shape of a call with `n_src` input samples per row.  Fails with
 * PESQ_ERR_INVALID_ARGUMENT below 20 frames (triton_ops/chain.py:775-779). */
int pesq_query_shape(const pesq_plan* plan, int64_t n_src, pesq_shape* shape);

/* Bytes of device workspace a forward/backward pair needs.  The forward
 * stores the state its backward reads in this workspace, so a pair must use
 * the same buffer and it must not be reused in between. */
int pesq_workspace_size(const pesq_plan* plan, int64_t batch, int64_t n_src, uint32_t flags, size_t* bytes);

/* Forward pass of `batch` utterance pairs.  ref / deg: [batch, n_src] rows
 * with row strides ld_ref / ld_deg (elements, >= n_src) of float32, or of
 * bf16 / fp16 with PESQ_INPUT_BF16 / PESQ_INPUT_F16.  Any of the four
 * outputs ([batch] each) may be NULL.  Replaces PesqLossTriton.raw / mos /
 * forward (triton_ops/loss.py:104-147, 203-215). */
int pesq_forward(const pesq_plan* plan, void* stream, const void* ref, int64_t ld_ref, const void* deg,
                 int64_t ld_deg, int64_t batch, int64_t n_src, uint32_t flags, void* workspace,
                 size_t workspace_bytes, float* d_symm, float* d_asymm, float* mos, float* loss);

/* Byte offset in the workspace of two doubles that pesq_forward leaves there:
 * the sum over the batch of the losses (factor * (0.1 d_symm + 0.0309
 * d_asymm), whether or not `loss` was requested) and the batch size, summed in
 * a fixed order by the last utterance's cluster of the chain forward (the
 * numerator and denominator of the global mean a data-parallel caller
 * all-reduces; there is no collective in the reference, whose callers take
 * loss.mean() of the [batch] loss, triton_ops/loss.py:210-215).  Valid after
 * a pesq_forward (or pesq_forward_front followed by one pesq_forward_chain)
 * with batch >= 1, until the workspace is reused. */
int pesq_loss_sum_offset(const pesq_plan* plan, int64_t batch, int64_t n_src, uint32_t flags, size_t* offset);

/* Backward of the preceding pesq_forward with the same inputs, flags and
 * workspace.  Upstream gradients g_loss / g_mos / g_dsymm / g_dasymm ([batch],
 * any may be NULL = zero) are summed.  Writes dL/dref into g_ref (row stride
 * ld_gref) if flags has PESQ_GRAD_REF and dL/ddeg into g_deg if it has
 * PESQ_GRAD_DEG.  ref / deg are those of the forward; everything the
 * backward needs from them was saved in the workspace, so they are not read
 * again.  Replaces the autograd backward of PesqLossTriton. */
int pesq_backward(const pesq_plan* plan, void* stream, const float* ref, int64_t ld_ref, const float* deg,
                  int64_t ld_deg, int64_t batch, int64_t n_src, uint32_t flags, void* workspace,
                  size_t workspace_bytes, const float* g_loss, const float* g_mos, const float* g_dsymm,
                  const float* g_dasymm, float* g_ref, int64_t ld_gref, float* g_deg, int64_t ld_gdeg);

/* The two stages of pesq_forward, callable on their own with the same
 * arguments (used to time the stages separately; pesq_forward is exactly
 * pesq_forward_front followed by pesq_forward_chain):
 *   front: [resampling to 16 kHz] + level alignment, pre-emphasis, STFT -> Bark
 *          (replaces triton_ops/loss.py:133-143: peak_normalize .. spectral)
 *   chain: perceptual model, distances, MOS and loss
 *          (replaces triton_ops/loss.py:145-147 and elementwise.py:683-747) */
int pesq_forward_front(const pesq_plan* plan, void* stream, const void* ref, int64_t ld_ref, const void* deg,
                       int64_t ld_deg, int64_t batch, int64_t n_src, uint32_t flags, void* workspace,
                       size_t workspace_bytes);
int pesq_forward_chain(const pesq_plan* plan, void* stream, int64_t batch, int64_t n_src, uint32_t flags,
                       void* workspace, size_t workspace_bytes, float* d_symm, float* d_asymm, float* mos,
                       float* loss);

/* The three stages of pesq_backward (pesq_backward is exactly
 * pesq_backward_chain, pesq_backward_align and pesq_backward_back in this
 * order on one stream):
 *   chain: adjoint of the perceptual model and of the epilogue
 *          (replaces chain.py:892-1021 and elementwise.py:800-827)
 *   align: z = H^T f of the level-alignment band pass H, from the f = H x
 *          the forward saved for the gradient rows: the input of the
 *          alignment-scale term (replaces the adjoint IIR of
 *          iir.py:1249-1258 on the level-alignment filter); it reads nothing
 *          the chain stage writes and is launched with programmatic stream
 *          serialisation, so it overlaps the chain stage before it
 *   back:  spectral adjoint, pre-emphasis adjoint, level-alignment term
 *          [+ resampler adjoint] (replaces spectral.py:526-581, iir.py:1249-1258,
 *          elementwise.py:234-265, 372-389, 608-652, resample.py:431-439) */
int pesq_backward_chain(const pesq_plan* plan, void* stream, int64_t batch, int64_t n_src, uint32_t flags,
                        void* workspace, size_t workspace_bytes, const float* g_loss, const float* g_mos,
                        const float* g_dsymm, const float* g_dasymm);
int pesq_backward_align(const pesq_plan* plan, void* stream, int64_t batch, int64_t n_src, uint32_t flags,
                        void* workspace, size_t workspace_bytes);
int pesq_backward_back(const pesq_plan* plan, void* stream, int64_t batch, int64_t n_src, uint32_t flags,
                       void* workspace, size_t workspace_bytes, float* g_ref, int64_t ld_gref, float* g_deg,
                       int64_t ld_gdeg);

/* Forward pass (distances, MOS, loss; no gradient) that allocates nothing and
 * takes no workspace: for callers that cannot allocate device memory when they
 * evaluate, such as real-time audio callbacks, plugins whose host owns all
 * device memory, or code running during a global-mode stream capture.  Its
 * scratch is a 16 MiB static device array of the library, held on every
 * device this entry point has been used on; the first call on a device looks
 * up that array and should come before any stream capture; calls sharing a
 * device must not overlap on the GPU (they share the array).  Batches needing
 * more than 16 MiB of scratch get PESQ_ERR_WORKSPACE.  The array's address
 * is cached per device for the runtime's primary context: do not call this
 * after cudaDeviceReset in the same process, nor with a context of your own
 * (driver API) current.  This entry point has no counterpart in the
 * reference. */
int pesq_forward_noalloc(const pesq_plan* plan, void* stream, const float* ref, int64_t ld_ref, const float* deg,
                         int64_t ld_deg, int64_t batch, int64_t n_src, float* d_symm, float* d_asymm, float* mos,
                         float* loss);

/* ---------------------------------------------------------------------------
 * Standalone polyphase resampler: the reference's TritonResample
 * (torch_pesq/triton_ops/resample.py:381-574), numerically torchaudio's
 * Resample(orig_freq, new_freq) with float32 taps, accumulated in float64.
 * Output m = l * new_step + j of a row is
 *   y[m] = sum_k taps[j][k] x[l * orig_step + k - width],  x = 0 outside,
 * for m < ceil(new_step * n_in / orig_step) (evaluated in float32).
 * ------------------------------------------------------------------------- */
typedef struct pesq_resampler pesq_resampler;

typedef struct pesq_resample_desc {
  int32_t abi_version;  /* PESQ_CUDA_ABI_VERSION */
  int32_t orig_step;    /* orig_freq / gcd */
  int32_t new_step;     /* new_freq / gcd */
  int32_t width;        /* left zero padding of the input */
  int32_t width_total;  /* taps per phase */
  int32_t reserved0;
  const double* taps;   /* [new_step * width_total], float32-valued */
} pesq_resample_desc;

/* Uploads the filter bank to the current device (replaces
 * TritonResample.__init__, resample.py:490-528). */
int pesq_resampler_create(const pesq_resample_desc* desc, pesq_resampler** out);
int pesq_resampler_destroy(pesq_resampler* resampler);
/* Output length for n_in input samples (resample.py:_target_length). */
int pesq_resampler_length(const pesq_resampler* resampler, int64_t n_in, int64_t* n_out);
/* y = A x for `rows` rows of n_in samples (row strides in elements; replaces
 * _ResampleFunction.forward, resample.py:422-435). */
int pesq_resample_forward(const pesq_resampler* resampler, void* stream, const float* x, int64_t ld_x,
                          int64_t rows, int64_t n_in, float* y, int64_t ld_y);
/* gx = A^T gy: the adjoint, a gather over input samples, deterministic
 * (replaces _ResampleAdjoint.forward, resample.py:396-401).  n_in is the
 * length of gx; gy has pesq_resampler_length(n_in) samples per row. */
int pesq_resample_adjoint(const pesq_resampler* resampler, void* stream, const float* gy, int64_t ld_gy,
                          int64_t rows, int64_t n_in, float* gx, int64_t ld_gx);

/* ---------------------------------------------------------------------------
 * Standalone causal IIR filter: the reference's TritonIIR
 * (torch_pesq/triton_ops/iir.py:1266-1482), lfilter(x, a, b, clamp=False) with
 * zero initial state along every row, through a state space realisation
 *   s[n+1] = A s[n] + B x[n],  y[n] = C s[n] + D x[n]
 * chosen on the host in float64 (triton_pesq_b200/iir_design.py, which
 * replaces iir.py:187-599).  The rows are split into chunks whose states are
 * combined by an exact parallel scan (no truncation), single pass.
 * ------------------------------------------------------------------------- */
typedef struct pesq_iir pesq_iir;

typedef struct pesq_iir_desc {
  int32_t abi_version;   /* PESQ_CUDA_ABI_VERSION */
  int32_t states;        /* P, 1 .. 24 */
  const double* trans;   /* A, [P][P] row-major */
  const double* input;   /* B, [P] */
  const double* output;  /* C, [P] */
  double feed;           /* D */
} pesq_iir_desc;

typedef struct pesq_iir_info {
  int32_t states;         /* P of the realisation */
  int32_t kernel_states;  /* state count of the kernel instantiation (>= P, zero padded) */
  int32_t block_lower;    /* A is block lower triangular in 2 x 2 blocks (zero blocks skipped) */
  int32_t chunk;          /* samples per thread chunk */
  int32_t tile;           /* samples per tile of a long row */
  int32_t overlap;        /* warm-up samples of the overlapped tiles long rows run when the
                             filter's state dies out within them (||A^overlap|| < 1e-11);
                             0: long rows chain their tiles by the look-back */
  double largest32;       /* largest entry of the float32 tables */
  double largest64;       /* largest entry of the float64 tile chaining tables */
} pesq_iir_info;

/* flags of pesq_iir_filter */
#define PESQ_IIR_REVERSE 1u /* filter each row back to front: the adjoint (iir.py:1232-1258) */
#define PESQ_IIR_RERUN 2u   /* chunk outputs by re-running the recursion ("scan") instead of the
                               impulse response product ("matmul", the default) */
#define PESQ_IIR_CHAINED 4u /* long rows chain their tiles by the decoupled look-back even where
                               the filter allows overlapped tiles (pesq_iir_info.overlap > 0):
                               exact for any filter, at the cost of the waits */

/* Builds the kernel tables (float64, then float32) on the current device
 * (replaces TritonIIR.__init__'s table build, iir.py:602-667 and 1343-1397). */
int pesq_iir_create(const pesq_iir_desc* desc, pesq_iir** out);
int pesq_iir_destroy(pesq_iir* filter);
int pesq_iir_query(const pesq_iir* filter, pesq_iir_info* info);
/* Device workspace of one pesq_iir_filter call (0 when no row spans more than
 * one tile; sized for the look-back, which overlapped tiles do not use); a
 * workspace serves one call in flight at a time. */
size_t pesq_iir_workspace_bytes(const pesq_iir* filter, int64_t rows, int64_t n);
/* y = filter(x) over `rows` rows of n samples, row strides in elements; x and
 * y must not overlap (replaces _launch, iir.py:1016-1161, and
 * _IIRFunction, iir.py:1232-1263). */
int pesq_iir_filter(const pesq_iir* filter, void* stream, const float* x, int64_t ld_x, int64_t rows, int64_t n,
                    float* y, int64_t ld_y, uint32_t flags, void* workspace, size_t workspace_bytes);
/* Polls a tile of a chained row makes while it waits for a predecessor's
 * published state before it gives up (its error word then reads nonzero and
 * the predecessor counts as zero).  Default 2^21 (about 0.1 s with the 64 ns
 * back-off); small values make the waits run out on purpose, e.g. to test
 * that a caller notices.  The reference's IIR has no device-side waits: it
 * chains its tiles with a separate sequential carry kernel
 * (triton_ops/iir.py:766-796). */
int pesq_iir_set_spin_limit(pesq_iir* filter, uint32_t polls);
/* Synchronises `stream`, then reads and clears the filter's error word:
 * nonzero when a tile of an earlier call stopped waiting for its predecessor
 * (a bounded wait that ran out; its rows are then wrong). */
int pesq_iir_check(pesq_iir* filter, void* stream, uint32_t* failed);

#ifdef __cplusplus
}
#endif

#endif /* PESQ_CUDA_H_ */
