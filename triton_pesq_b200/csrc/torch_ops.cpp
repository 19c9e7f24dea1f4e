// torch custom ops over the C ABI of libpesq_cuda.so.
//
// The ops only allocate tensors with torch's caching allocator (so they are
// safe under CUDA graph capture), pick the current stream and forward to
// pesq_forward / pesq_backward.  Plans are created from Python through the
// same C ABI (ctypes) and passed in as an opaque integer handle.
#include <algorithm>

#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include "../../include/pesq_cuda.h"

namespace {

void check_status(int status, const char* what) {
  if (status == PESQ_OK) return;
  const char* msg = pesq_last_error();
  if (status == PESQ_ERR_INVALID_ARGUMENT) {
    TORCH_CHECK_VALUE(false, what, ": ", msg);
  }
  TORCH_CHECK(false, what, " failed (status ", status, "): ", msg);
}

void check_signal(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "The CUDA PESQ backend needs `", name, "` to live on a GPU.");
  TORCH_CHECK(t.scalar_type() == at::kFloat || t.scalar_type() == at::kBFloat16 || t.scalar_type() == at::kHalf,
              "The CUDA PESQ backend supports float32 (and bfloat16 / float16 inputs), `", name, "` is ",
              t.scalar_type(), ".");
  TORCH_CHECK(t.dim() == 2, "`", name, "` must be [batch, sample], got ", t.sizes());
  TORCH_CHECK(t.stride(1) == 1, "`", name, "` rows must be contiguous");
}

// PESQ_INPUT_* flag of the inputs' element type
uint32_t input_flag(const at::Tensor& ref, const at::Tensor& deg) {
  TORCH_CHECK_VALUE(ref.scalar_type() == deg.scalar_type(), "ref and deg must have the same dtype, got ",
                    ref.scalar_type(), " and ", deg.scalar_type(), ".");
  if (ref.scalar_type() == at::kBFloat16) return PESQ_INPUT_BF16;
  if (ref.scalar_type() == at::kHalf) return PESQ_INPUT_F16;
  return 0u;
}

const pesq_plan* as_plan(int64_t handle) {
  TORCH_CHECK(handle != 0, "invalid PESQ plan handle");
  return reinterpret_cast<const pesq_plan*>(static_cast<uintptr_t>(handle));
}

std::tuple<at::Tensor, at::Tensor, at::Tensor, at::Tensor, at::Tensor> pesq_forward_op(int64_t plan_handle,
                                                                                       const at::Tensor& ref,
                                                                                       const at::Tensor& deg,
                                                                                       int64_t flags) {
  check_signal(ref, "ref");
  check_signal(deg, "deg");
  TORCH_CHECK_VALUE(ref.sizes() == deg.sizes(), "Reference and degraded signal must have the same shape, got ",
                    ref.sizes(), " and ", deg.sizes(), ".");
  TORCH_CHECK(ref.device() == deg.device(), "ref and deg must be on the same device");
  const pesq_plan* plan = as_plan(plan_handle);
  c10::cuda::CUDAGuard guard(ref.device());
  const int64_t batch = ref.size(0), n = ref.size(1);
  flags |= input_flag(ref, deg);
  size_t bytes = 0;
  check_status(pesq_workspace_size(plan, batch, n, (uint32_t)flags, &bytes), "pesq_workspace_size");
  auto opts = ref.options().dtype(at::kFloat);
  at::Tensor ws = at::empty({(int64_t)((bytes + 3) / 4)}, opts);
  at::Tensor d_symm = at::empty({batch}, opts), d_asymm = at::empty({batch}, opts);
  at::Tensor mos = at::empty({batch}, opts), loss = at::empty({batch}, opts);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(ref.device().index());
  check_status(pesq_forward(plan, stream, ref.data_ptr(), ref.stride(0), deg.data_ptr(),
                            deg.stride(0), batch, n, (uint32_t)flags, ws.data_ptr(), bytes,
                            d_symm.data_ptr<float>(), d_asymm.data_ptr<float>(), mos.data_ptr<float>(),
                            loss.data_ptr<float>()),
               "pesq_forward");
  return {d_symm, d_asymm, mos, loss, ws};
}

// The four upstream gradients of one backward call.  When every one that is
// present is a broadcast of one value over the batch (stride 0, as autograd
// hands over the gradient of a sum or mean) they are passed as that single
// value with PESQ_UPSTREAM_SCALAR; otherwise as contiguous [batch] arrays.
struct Upstream {
  at::Tensor t[4];
  const float* ptr[4] = {nullptr, nullptr, nullptr, nullptr};
  uint32_t flag = 0;
  Upstream(const c10::optional<at::Tensor>* g[4], int64_t batch) {
    static const char* names[4] = {"g_loss", "g_mos", "g_dsymm", "g_dasymm"};
    bool any = false, shared = true;
    for (int i = 0; i < 4; ++i) {
      if (!g[i]->has_value() || !(*g[i])->defined()) continue;
      const at::Tensor& v = **g[i];
      TORCH_CHECK(v.is_cuda() && v.scalar_type() == at::kFloat && v.dim() == 1 && v.numel() == batch,
                  "upstream gradient `", names[i], "` must be a float32 CUDA tensor of ", batch, " elements");
      any = true;
      shared = shared && batch > 1 && v.stride(0) == 0;
    }
    if (!any) return;
    if (shared) flag = PESQ_UPSTREAM_SCALAR;
    for (int i = 0; i < 4; ++i) {
      if (!g[i]->has_value() || !(*g[i])->defined()) continue;
      t[i] = shared ? **g[i] : (*g[i])->contiguous();
      ptr[i] = t[i].data_ptr<float>();
    }
  }
};

std::tuple<at::Tensor, at::Tensor> pesq_backward_op(int64_t plan_handle, const at::Tensor& ref,
                                                    const at::Tensor& deg, int64_t flags, const at::Tensor& ws,
                                                    const c10::optional<at::Tensor>& g_loss,
                                                    const c10::optional<at::Tensor>& g_mos,
                                                    const c10::optional<at::Tensor>& g_dsymm,
                                                    const c10::optional<at::Tensor>& g_dasymm) {
  check_signal(ref, "ref");
  check_signal(deg, "deg");
  const pesq_plan* plan = as_plan(plan_handle);
  c10::cuda::CUDAGuard guard(ref.device());
  const int64_t batch = ref.size(0), n = ref.size(1);
  flags |= input_flag(ref, deg);
  // a gradient that was not asked for comes back as an empty tensor; the
  // engine writes float32 gradients, returned in the inputs' dtype
  const auto fopts = ref.options().dtype(at::kFloat);
  at::Tensor g_ref = (flags & PESQ_GRAD_REF) ? at::empty({batch, n}, fopts) : at::empty({0}, ref.options());
  at::Tensor g_deg = (flags & PESQ_GRAD_DEG) ? at::empty({batch, n}, fopts) : at::empty({0}, deg.options());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(ref.device().index());
  const c10::optional<at::Tensor>* g[4] = {&g_loss, &g_mos, &g_dsymm, &g_dasymm};
  const Upstream up(g, batch);
  // (ref / deg are not read by the backward)
  check_status(pesq_backward(plan, stream, static_cast<const float*>(ref.data_ptr()), ref.stride(0),
                             static_cast<const float*>(deg.data_ptr()), deg.stride(0), batch, n,
                             (uint32_t)flags | up.flag, ws.data_ptr(),
                             (size_t)ws.numel() * 4, up.ptr[0], up.ptr[1], up.ptr[2], up.ptr[3],
                             (flags & PESQ_GRAD_REF) ? g_ref.data_ptr<float>() : nullptr, n,
                             (flags & PESQ_GRAD_DEG) ? g_deg.data_ptr<float>() : nullptr, n),
               "pesq_backward");
  if (ref.scalar_type() != at::kFloat) {
    if (flags & PESQ_GRAD_REF) g_ref = g_ref.to(ref.scalar_type());
    if (flags & PESQ_GRAD_DEG) g_deg = g_deg.to(deg.scalar_type());
  }
  return {g_ref, g_deg};
}

const pesq_resampler* as_resampler(int64_t handle) {
  TORCH_CHECK(handle != 0, "invalid resampler handle");
  return reinterpret_cast<const pesq_resampler*>(static_cast<uintptr_t>(handle));
}

void check_rows(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "The CUDA resampler needs `", name, "` to live on a GPU.");
  TORCH_CHECK(t.scalar_type() == at::kFloat, "The CUDA resampler only supports float32, `", name, "` is ",
              t.scalar_type(), ".");
  TORCH_CHECK(t.dim() == 2, "`", name, "` must be [rows, samples], got ", t.sizes());
}

// y = A x over the rows of x [rows, n_in]
at::Tensor resample_op(int64_t handle, const at::Tensor& x_in) {
  check_rows(x_in, "waveform");
  const pesq_resampler* r = as_resampler(handle);
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.stride(1) == 1 ? x_in : x_in.contiguous();
  const int64_t rows = x.size(0), n_in = x.size(1);
  int64_t n_out = 0;
  check_status(pesq_resampler_length(r, n_in, &n_out), "pesq_resampler_length");
  at::Tensor y = at::empty({rows, n_out}, x.options());
  if (rows == 0 || n_out == 0) return y;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(x.device().index());
  check_status(pesq_resample_forward(r, stream, x.data_ptr<float>(), std::max<int64_t>(x.stride(0), n_in), rows,
                                     n_in, y.data_ptr<float>(), n_out),
               "pesq_resample_forward");
  return y;
}

// gx = A^T gy, gx [rows, n_in]
at::Tensor resample_adjoint_op(int64_t handle, const at::Tensor& g_in, int64_t n_in) {
  check_rows(g_in, "grad");
  const pesq_resampler* r = as_resampler(handle);
  c10::cuda::CUDAGuard guard(g_in.device());
  const at::Tensor g = g_in.stride(1) == 1 ? g_in : g_in.contiguous();
  const int64_t rows = g.size(0);
  int64_t n_out = 0;
  check_status(pesq_resampler_length(r, n_in, &n_out), "pesq_resampler_length");
  TORCH_CHECK_VALUE(g.size(1) == n_out, "gradient of ", g.size(1), " samples, the resampler produces ", n_out,
                    " from ", n_in);
  at::Tensor gx = at::empty({rows, n_in}, g.options());
  if (rows == 0 || n_in == 0) return gx;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(g.device().index());
  check_status(pesq_resample_adjoint(r, stream, g.data_ptr<float>(), std::max<int64_t>(g.stride(0), n_out), rows,
                                     n_in, gx.data_ptr<float>(), n_in),
               "pesq_resample_adjoint");
  return gx;
}

const pesq_iir* as_iir(int64_t handle) {
  TORCH_CHECK(handle != 0, "invalid IIR filter handle");
  return reinterpret_cast<const pesq_iir*>(static_cast<uintptr_t>(handle));
}

// y = filter(x) along the rows of x [rows, n]; flags: PESQ_IIR_REVERSE (the
// adjoint), PESQ_IIR_RERUN
at::Tensor iir_op(int64_t handle, const at::Tensor& x_in, int64_t flags) {
  TORCH_CHECK(x_in.is_cuda(), "The CUDA IIR filter needs `signal` to live on a GPU.");
  TORCH_CHECK(x_in.scalar_type() == at::kFloat, "The CUDA IIR filter only supports float32, `signal` is ",
              x_in.scalar_type(), ".");
  TORCH_CHECK(x_in.dim() == 2, "The CUDA IIR filter needs a [batch, sample] tensor, got ", x_in.sizes(), ".");
  const pesq_iir* f = as_iir(handle);
  c10::cuda::CUDAGuard guard(x_in.device());
  const at::Tensor x = x_in.stride(1) == 1 ? x_in : x_in.contiguous();
  const int64_t rows = x.size(0), n = x.size(1);
  at::Tensor y = at::empty({rows, n}, x.options());
  if (rows == 0 || n == 0) return y;
  const size_t ws_bytes = pesq_iir_workspace_bytes(f, rows, n);
  at::Tensor ws;
  if (ws_bytes > 0) ws = at::empty({(int64_t)ws_bytes}, x.options().dtype(at::kByte));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(x.device().index());
  check_status(pesq_iir_filter(f, stream, x.data_ptr<float>(), std::max<int64_t>(x.stride(0), n), rows, n,
                               y.data_ptr<float>(), n, (uint32_t)flags, ws_bytes ? ws.data_ptr() : nullptr,
                               ws_bytes),
               "pesq_iir_filter");
  return y;
}

}  // namespace

TORCH_LIBRARY(pesq_cuda, m) {
  m.def("forward(int plan, Tensor ref, Tensor deg, int flags) -> (Tensor, Tensor, Tensor, Tensor, Tensor)");
  m.def(
      "backward(int plan, Tensor ref, Tensor deg, int flags, Tensor(a!) workspace, Tensor? g_loss, Tensor? g_mos, "
      "Tensor? g_dsymm, Tensor? g_dasymm) -> (Tensor, Tensor)");
  m.def("resample(int resampler, Tensor waveform) -> Tensor");
  m.def("resample_adjoint(int resampler, Tensor grad, int n_in) -> Tensor");
  m.def("iir(int filter, Tensor signal, int flags) -> Tensor");
}

TORCH_LIBRARY_IMPL(pesq_cuda, CUDA, m) {
  m.impl("forward", &pesq_forward_op);
  m.impl("backward", &pesq_backward_op);
  m.impl("resample", &resample_op);
  m.impl("resample_adjoint", &resample_adjoint_op);
  m.impl("iir", &iir_op);
}
