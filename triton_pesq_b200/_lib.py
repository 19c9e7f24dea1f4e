"""Loading of the native libraries and plan creation through the C ABI.

``libpesq_cuda.so`` carries every kernel and the C ABI of
``include/pesq_cuda.h``; ``_pesq_torch_ops.so`` registers the
``torch.ops.pesq_cuda`` custom ops on top of it.  Both are built in-tree by
``triton_pesq_b200.build``.  There is no fallback: if they are missing the
import of the ops fails with an explicit error.
"""

from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpesq_cuda.so")
OPS_PATH = os.path.join(HERE, "_pesq_torch_ops.so")

ABI_VERSION = 2
GRAD_REF = 1
GRAD_DEG = 2
UPSTREAM_SCALAR = 4
INPUT_BF16 = 8
INPUT_F16 = 16

PESQ_OK = 0
PESQ_ERR_INVALID_ARGUMENT = 1
PESQ_ERR_WORKSPACE = 3

_lock = threading.Lock()
_lib = None
_ops_loaded = False


class ScanDesc(ctypes.Structure):
    _fields_ = [
        ("states", ctypes.c_int32),
        ("chunk", ctypes.c_int32),
        ("levels", ctypes.c_int32),
        ("impulse", ctypes.POINTER(ctypes.c_double)),
        ("carry", ctypes.POINTER(ctypes.c_double)),
        ("drive", ctypes.POINTER(ctypes.c_double)),
        ("power", ctypes.POINTER(ctypes.c_double)),
        ("trans", ctypes.POINTER(ctypes.c_double)),
        ("input", ctypes.POINTER(ctypes.c_double)),
        ("output", ctypes.POINTER(ctypes.c_double)),
        ("feed", ctypes.c_double),
    ]


class PlanDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("sample_rate", ctypes.c_int32),
        ("n_fft", ctypes.c_int32),
        ("hop_length", ctypes.c_int32),
        ("nbarks", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("factor", ctypes.c_double),
        ("window", ctypes.POINTER(ctypes.c_double)),
        ("band_start", ctypes.POINTER(ctypes.c_int32)),
        ("band_end", ctypes.POINTER(ctypes.c_int32)),
        ("band_corr", ctypes.POINTER(ctypes.c_double)),
        ("threshold", ctypes.POINTER(ctypes.c_double)),
        ("exponent", ctypes.POINTER(ctypes.c_double)),
        ("width", ctypes.POINTER(ctypes.c_double)),
        ("total_width", ctypes.c_double),
        ("loudness_sl", ctypes.c_double),
        ("power_filter", ScanDesc),
        ("pre_filter", ScanDesc),
        ("rs_orig_step", ctypes.c_int32),
        ("rs_new_step", ctypes.c_int32),
        ("rs_width", ctypes.c_int32),
        ("rs_width_total", ctypes.c_int32),
        ("rs_taps", ctypes.POINTER(ctypes.c_double)),
    ]


class ResampleDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("orig_step", ctypes.c_int32),
        ("new_step", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("width_total", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("taps", ctypes.POINTER(ctypes.c_double)),
    ]


class IirDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32),
        ("states", ctypes.c_int32),
        ("trans", ctypes.POINTER(ctypes.c_double)),
        ("input", ctypes.POINTER(ctypes.c_double)),
        ("output", ctypes.POINTER(ctypes.c_double)),
        ("feed", ctypes.c_double),
    ]


class IirInfo(ctypes.Structure):
    _fields_ = [
        ("states", ctypes.c_int32),
        ("kernel_states", ctypes.c_int32),
        ("block_lower", ctypes.c_int32),
        ("chunk", ctypes.c_int32),
        ("tile", ctypes.c_int32),
        ("overlap", ctypes.c_int32),
        ("largest32", ctypes.c_double),
        ("largest64", ctypes.c_double),
    ]


#: pesq_iir_filter flags
IIR_REVERSE = 1
IIR_RERUN = 2
IIR_CHAINED = 4


class Shape(ctypes.Structure):
    _fields_ = [("n16", ctypes.c_int64), ("frames", ctypes.c_int32), ("windows", ctypes.c_int32)]


#: every function of include/pesq_cuda.h with its ctypes signature
SIGNATURES = {
    "pesq_abi_version": (ctypes.c_int, []),
    "pesq_last_error": (ctypes.c_char_p, []),
    "pesq_plan_create": (ctypes.c_int, [ctypes.POINTER(PlanDesc), ctypes.POINTER(ctypes.c_void_p)]),
    "pesq_plan_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "pesq_plan_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]),
    "pesq_plan_check": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "pesq_query_shape": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(Shape)]),
    "pesq_workspace_size": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.POINTER(ctypes.c_size_t)],
    ),
    "pesq_loss_sum_offset": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.POINTER(ctypes.c_size_t)],
    ),
    "pesq_forward": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
         ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "pesq_backward": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
         ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t,
         ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64],
    ),
    "pesq_forward_front": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
         ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t],
    ),
    "pesq_forward_chain": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p,
         ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "pesq_backward_chain": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p,
         ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
    "pesq_backward_align": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p,
         ctypes.c_size_t],
    ),
    "pesq_backward_back": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p,
         ctypes.c_size_t, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64],
    ),
    "pesq_resampler_create": (ctypes.c_int, [ctypes.POINTER(ResampleDesc), ctypes.POINTER(ctypes.c_void_p)]),
    "pesq_resampler_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "pesq_resampler_length": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)]),
    "pesq_resample_forward": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
         ctypes.c_void_p, ctypes.c_int64],
    ),
    "pesq_resample_adjoint": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
         ctypes.c_void_p, ctypes.c_int64],
    ),
    "pesq_iir_create": (ctypes.c_int, [ctypes.POINTER(IirDesc), ctypes.POINTER(ctypes.c_void_p)]),
    "pesq_iir_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "pesq_iir_query": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(IirInfo)]),
    "pesq_iir_workspace_bytes": (ctypes.c_size_t, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64]),
    "pesq_iir_filter": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
         ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t],
    ),
    "pesq_iir_check": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "pesq_iir_set_spin_limit": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32]),
    "pesq_forward_noalloc": (
        ctypes.c_int,
        [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
         ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p],
    ),
}


def library() -> ctypes.CDLL:
    """The C ABI library, loaded once (RTLD_GLOBAL so the ops library binds to it)."""

    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"The CUDA PESQ engine is not built ({LIB_PATH} is missing); run "
                    "`python -m triton_pesq_b200.build` first."
                )
            lib = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            if lib.pesq_abi_version() != ABI_VERSION:
                raise RuntimeError("libpesq_cuda.so has an incompatible ABI version")
            _lib = lib
        return _lib


def load_ops() -> None:
    """Register ``torch.ops.pesq_cuda`` (idempotent)."""

    global _ops_loaded
    library()
    with _lock:
        if not _ops_loaded:
            if not os.path.exists(OPS_PATH):
                raise RuntimeError(
                    f"The CUDA PESQ torch ops are not built ({OPS_PATH} is missing); run "
                    "`python -m triton_pesq_b200.build` first."
                )
            import torch

            torch.ops.load_library(OPS_PATH)
            _register_fakes()
            _ops_loaded = True


def _register_fakes() -> None:
    """Shape functions of the ``torch.ops.pesq_cuda`` ops for tracing
    (``torch.compile``, ``torch.export``, fake tensors): every output shape
    follows from the input shapes and the plan, through the same host
    functions of the C ABI that size the real outputs."""

    import torch

    def workspace_floats(plan, batch, n, flags):
        nbytes = ctypes.c_size_t()
        check(library().pesq_workspace_size(ctypes.c_void_p(plan), int(batch), int(n), int(flags),
                                            ctypes.byref(nbytes)), "pesq_workspace_size")
        return (nbytes.value + 3) // 4

    def input_flag(ref):
        return INPUT_BF16 if ref.dtype == torch.bfloat16 else INPUT_F16 if ref.dtype == torch.float16 else 0

    @torch.library.register_fake("pesq_cuda::forward")
    def _forward(plan, ref, deg, flags):
        torch._check(ref.dim() == 2 and ref.shape == deg.shape, lambda: "ref and deg must be [batch, sample]")
        batch, n = ref.shape
        outs = [ref.new_empty((batch,), dtype=torch.float32) for _ in range(4)]
        ws = ref.new_empty((workspace_floats(plan, batch, n, flags | input_flag(ref)),), dtype=torch.float32)
        return (*outs, ws)

    @torch.library.register_fake("pesq_cuda::backward")
    def _backward(plan, ref, deg, flags, workspace, g_loss, g_mos, g_dsymm, g_dasymm):
        batch, n = ref.shape
        g_ref = ref.new_empty((batch, n)) if flags & GRAD_REF else ref.new_empty((0,))
        g_deg = deg.new_empty((batch, n)) if flags & GRAD_DEG else deg.new_empty((0,))
        return g_ref, g_deg

    @torch.library.register_fake("pesq_cuda::resample")
    def _resample(resampler, waveform):
        n_out = ctypes.c_int64()
        check(library().pesq_resampler_length(ctypes.c_void_p(resampler), int(waveform.shape[1]),
                                              ctypes.byref(n_out)), "pesq_resampler_length")
        return waveform.new_empty((waveform.shape[0], n_out.value))

    @torch.library.register_fake("pesq_cuda::resample_adjoint")
    def _resample_adjoint(resampler, grad, n_in):
        return grad.new_empty((grad.shape[0], n_in))

    @torch.library.register_fake("pesq_cuda::iir")
    def _iir(filt, signal, flags):
        return signal.new_empty(signal.shape)


def plan_check(handle: int, stream: int = 0) -> int:
    """Synchronise ``stream`` and return (and clear) the plan's device error word."""

    flags = ctypes.c_uint32(0)
    check(library().pesq_plan_check(ctypes.c_void_p(handle), ctypes.c_void_p(stream), ctypes.byref(flags)),
          "pesq_plan_check")
    return int(flags.value)


def loss_sum_offset(handle: int, batch: int, n: int, flags: int) -> int:
    """Byte offset of the [loss sum, batch] float64 pair in a call's workspace."""

    off = ctypes.c_size_t()
    check(library().pesq_loss_sum_offset(ctypes.c_void_p(handle), int(batch), int(n), int(flags),
                                         ctypes.byref(off)), "pesq_loss_sum_offset")
    return int(off.value)


def last_error() -> str:
    msg = library().pesq_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status == PESQ_OK:
        return
    msg = f"{what}: {last_error()}"
    if status == PESQ_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise RuntimeError(f"{msg} (status {status})")


def _dptr(arr: np.ndarray):
    return arr.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def _scan_desc(tab, keep: list) -> ScanDesc:
    arrays = [
        np.ascontiguousarray(tab.impulse, dtype=np.float64),
        np.ascontiguousarray(tab.carry, dtype=np.float64),
        np.ascontiguousarray(tab.drive, dtype=np.float64),
        np.ascontiguousarray(tab.power, dtype=np.float64),
        np.ascontiguousarray(tab.trans, dtype=np.float64),
        np.ascontiguousarray(tab.input, dtype=np.float64),
        np.ascontiguousarray(tab.output, dtype=np.float64),
    ]
    keep.extend(arrays)
    return ScanDesc(
        states=tab.states, chunk=tab.chunk, levels=tab.levels,
        impulse=_dptr(arrays[0]), carry=_dptr(arrays[1]), drive=_dptr(arrays[2]), power=_dptr(arrays[3]),
        trans=_dptr(arrays[4]), input=_dptr(arrays[5]), output=_dptr(arrays[6]), feed=float(tab.feed),
    )


def create_plan(cfg) -> int:
    """Build a plan on the current CUDA device from a :class:`PlanConfig`."""

    lib = library()
    keep: list = []

    def arr(values, dtype=np.float64):
        a = np.ascontiguousarray(values, dtype=dtype)
        keep.append(a)
        return a

    window = arr(cfg.window)
    starts = arr(cfg.layout.starts, np.int32)
    ends = arr(cfg.layout.ends, np.int32)
    corr = arr(cfg.layout.pow_dens_correction)
    thr = arr(cfg.thresholds)
    expo = arr(cfg.exponents)
    width = arr(cfg.layout.width_bark)

    desc = PlanDesc()
    desc.abi_version = ABI_VERSION
    desc.sample_rate = int(cfg.sample_rate)
    desc.n_fft = int(cfg.n_fft)
    desc.hop_length = int(cfg.hop_length)
    desc.nbarks = int(cfg.layout.nbarks)
    desc.factor = float(cfg.factor)
    desc.window = _dptr(window)
    desc.band_start = starts.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
    desc.band_end = ends.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))
    desc.band_corr = _dptr(corr)
    desc.threshold = _dptr(thr)
    desc.exponent = _dptr(expo)
    desc.width = _dptr(width)
    desc.total_width = float(cfg.layout.total_width)
    desc.loudness_sl = float(cfg.loudness_sl)
    desc.power_filter = _scan_desc(cfg.power_scan, keep)
    desc.pre_filter = _scan_desc(cfg.pre_scan, keep)
    if cfg.kernel is not None:
        taps = arr(cfg.kernel.taps)
        desc.rs_orig_step = cfg.kernel.orig_step
        desc.rs_new_step = cfg.kernel.new_step
        desc.rs_width = cfg.kernel.width
        desc.rs_width_total = cfg.kernel.width_total
        desc.rs_taps = _dptr(taps)

    handle = ctypes.c_void_p()
    check(lib.pesq_plan_create(ctypes.byref(desc), ctypes.byref(handle)), "pesq_plan_create")
    return int(handle.value)


def destroy_plan(handle: int) -> None:
    if handle and _lib is not None:
        _lib.pesq_plan_destroy(ctypes.c_void_p(handle))


def destroy_resampler(handle: int) -> None:
    if handle and _lib is not None:
        _lib.pesq_resampler_destroy(ctypes.c_void_p(handle))


class Owned:
    """A native handle (plan, resampler) owned from Python.

    The handle is released when the last reference goes: the module's table of
    per-device handles holds one, and every autograd node that may still run a
    backward with the handle holds another, so a module that is dropped right
    after its forward (``PesqLossCuda(...)(ref, deg).sum().backward()``) keeps
    its plan until the backward is done.  ``release(handle)`` runs once."""

    def __init__(self, handle: int, release):
        self.handle = int(handle)
        self._release = release

    def __del__(self):
        handle, self.handle = self.handle, 0
        if handle:
            try:
                self._release(handle)
            except Exception:  # pragma: no cover - interpreter shutdown
                pass


def query_shape(handle: int, n_src: int):
    shape = Shape()
    check(library().pesq_query_shape(ctypes.c_void_p(handle), int(n_src), ctypes.byref(shape)), "pesq_query_shape")
    return shape.n16, shape.frames, shape.windows


def create_resampler(kernel) -> int:
    """Upload a :class:`~triton_pesq_b200.tables.ResampleKernel` to the current
    CUDA device; returns the resampler handle."""

    lib = library()
    taps = np.ascontiguousarray(kernel.taps, dtype=np.float64)
    desc = ResampleDesc()
    desc.abi_version = ABI_VERSION
    desc.orig_step = int(kernel.orig_step)
    desc.new_step = int(kernel.new_step)
    desc.width = int(kernel.width)
    desc.width_total = int(kernel.width_total)
    desc.taps = _dptr(taps)
    handle = ctypes.c_void_p()
    check(lib.pesq_resampler_create(ctypes.byref(desc), ctypes.byref(handle)), "pesq_resampler_create")
    return int(handle.value)


def create_iir(design) -> int:
    """Build the kernel tables of an :class:`~triton_pesq_b200.iir_design.IIRDesign`
    on the current CUDA device; returns the filter handle."""

    lib = library()
    keep = [np.ascontiguousarray(design.trans, dtype=np.float64),
            np.ascontiguousarray(design.input, dtype=np.float64),
            np.ascontiguousarray(design.output, dtype=np.float64)]
    desc = IirDesc()
    desc.abi_version = ABI_VERSION
    desc.states = int(design.trans.shape[0])
    desc.trans, desc.input, desc.output = (_dptr(k) for k in keep)
    desc.feed = float(design.feed)
    handle = ctypes.c_void_p()
    check(lib.pesq_iir_create(ctypes.byref(desc), ctypes.byref(handle)), "pesq_iir_create")
    return int(handle.value)


def destroy_iir(handle: int) -> None:
    if handle and _lib is not None:
        _lib.pesq_iir_destroy(ctypes.c_void_p(handle))


def iir_info(handle: int) -> IirInfo:
    info = IirInfo()
    check(library().pesq_iir_query(ctypes.c_void_p(handle), ctypes.byref(info)), "pesq_iir_query")
    return info


def iir_check(handle: int, stream: int = 0) -> int:
    """Synchronise ``stream`` and return (and clear) the filter's error word."""

    failed = ctypes.c_uint32(0)
    check(library().pesq_iir_check(ctypes.c_void_p(handle), ctypes.c_void_p(stream), ctypes.byref(failed)),
          "pesq_iir_check")
    return int(failed.value)
