// C ABI of the standalone polyphase resampler (the reference's TritonResample,
// torch_pesq/triton_ops/resample.py:381-574): a resampler object holds the
// device tables of one (orig_freq, new_freq) filter bank; forward and adjoint
// are stream-ordered kernel launches over [rows, samples] float32 arrays.
#include <cuda_runtime.h>

#include "../../include/pesq_cuda.h"
#include "kernels.cuh"

using namespace pesq;

namespace pesq {
int set_error(int code, const char* msg);
}  // namespace pesq

struct pesq_resampler {
  int device;
  ResampleTables tables;
};

namespace {

int check_rows(const pesq_resampler* r, int64_t rows, int64_t n_in, const void* in, int64_t ld_in, int64_t n_in_row,
               const void* out, int64_t ld_out, int64_t n_out_row) {
  if (!r) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL resampler");
  if (rows < 0 || n_in < 0) return set_error(PESQ_ERR_INVALID_ARGUMENT, "negative rows or samples");
  if (rows > ((int64_t)1 << 31) - 1 || n_in > ((int64_t)1 << 31) - 1)
    return set_error(PESQ_ERR_INVALID_ARGUMENT, "more than 2^31 - 1 rows or samples");
  if (rows == 0) return PESQ_OK;
  if ((n_in_row > 0 && !in) || (n_out_row > 0 && !out)) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL signal");
  if (ld_in < n_in_row || ld_out < n_out_row)
    return set_error(PESQ_ERR_INVALID_ARGUMENT, "row stride smaller than the row");
  int dev = -1;
  cudaGetDevice(&dev);
  if (dev != r->device) return set_error(PESQ_ERR_INVALID_ARGUMENT, "the resampler lives on another device");
  return PESQ_OK;
}

}  // namespace

extern "C" {

int pesq_resampler_create(const pesq_resample_desc* d, pesq_resampler** out) {
  if (!d || !out) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  *out = nullptr;
  if (d->abi_version != PESQ_CUDA_ABI_VERSION) return set_error(PESQ_ERR_UNSUPPORTED, "ABI version mismatch");
  pesq_resampler* r = new pesq_resampler();
  if (cudaGetDevice(&r->device) != cudaSuccess) {
    delete r;
    return set_error(PESQ_ERR_CUDA, "no CUDA device");
  }
  const char* msg = build_resample_tables(d->orig_step, d->new_step, d->width, d->width_total, d->taps, r->tables);
  if (msg) {
    delete r;
    return set_error(PESQ_ERR_INVALID_ARGUMENT, msg);
  }
  *out = r;
  return PESQ_OK;
}

int pesq_resampler_destroy(pesq_resampler* r) {
  if (!r) return PESQ_OK;
  free_resample_tables(r->tables);
  delete r;
  return PESQ_OK;
}

int pesq_resampler_length(const pesq_resampler* r, int64_t n_in, int64_t* n_out) {
  if (!r || !n_out) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL argument");
  if (n_in < 0) return set_error(PESQ_ERR_INVALID_ARGUMENT, "negative length");
  *n_out = resample_length(r->tables.orig_step, r->tables.new_step, n_in);
  return PESQ_OK;
}

int pesq_resample_forward(const pesq_resampler* r, void* stream, const float* x, int64_t ld_x, int64_t rows,
                          int64_t n_in, float* y, int64_t ld_y) {
  if (!r) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL resampler");
  const int64_t n_out = resample_length(r->tables.orig_step, r->tables.new_step, n_in);
  int rc = check_rows(r, rows, n_in, x, ld_x, n_in, y, ld_y, n_out);
  if (rc || rows == 0 || n_out == 0) return rc;
  ResampleArgs a = resample_args(r->tables, n_in, n_out);
  a.src = RowSource{x, x, ld_x, ld_x, (int)rows};
  a.dst = RowSink{y, y, ld_y, ld_y, (int)rows};
  a.rows = (int)rows;
  a.row_begin = 0;
  const cudaError_t e = launch_resample_fwd(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(PESQ_ERR_CUDA, cudaGetErrorString(e));
  return PESQ_OK;
}

int pesq_resample_adjoint(const pesq_resampler* r, void* stream, const float* gy, int64_t ld_gy, int64_t rows,
                          int64_t n_in, float* gx, int64_t ld_gx) {
  if (!r) return set_error(PESQ_ERR_INVALID_ARGUMENT, "NULL resampler");
  const int64_t n_out = resample_length(r->tables.orig_step, r->tables.new_step, n_in);
  int rc = check_rows(r, rows, n_in, gy, ld_gy, n_out, gx, ld_gx, n_in);
  if (rc || rows == 0 || n_in == 0) return rc;
  ResampleArgs a = resample_args(r->tables, n_in, n_out);
  a.src = RowSource{gy, gy, ld_gy, ld_gy, (int)rows};
  a.dst = RowSink{gx, gx, ld_gx, ld_gx, (int)rows};
  a.rows = (int)rows;
  a.row_begin = 0;
  const cudaError_t e = launch_resample_adj(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return set_error(PESQ_ERR_CUDA, cudaGetErrorString(e));
  return PESQ_OK;
}

}  // extern "C"
