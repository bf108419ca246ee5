"""ctypes binding of liblowbit.so (the C ABI in include/lowbit.h) for PyTorch CUDA tensors.

This replaces the reference's device runtime for the low-bit path: the session LRU and
``_run/_run_many/_run_chain`` of torch_intel_npu.py:322-570 and the pybind boundary of
npunlock-probe/torch-device/backend.cpp:253-347.  There is no session, IR or compile
step: tensors are bound by pointer and launched on the caller's CUDA stream, and
chained submission is a CUDA graph (see ``torch_npu_smollm``).

There is no CPU fallback: without a CUDA device or without the built library every
entry point raises.
"""
import ctypes
import functools
import os
import threading
from pathlib import Path

import torch

LB_FMT = {'int4': 0, 'nf4': 1, 'int8': 2, 'fp16': 3}
OK, INVALID, UNSUPPORTED, CUDA_ERR, NONFINITE, OVERFLOW, WORKSPACE, ALIAS, INJECTED, TIMEOUT = range(10)
PATH = {'auto': 0, 'gemv': 1, 'tc': 2, 'generic': 3}
PATH_NAME = {v: k for k, v in PATH.items()}

_LIB = None
_LIB_LOCK = threading.Lock()
LIB_PATH = Path(__file__).resolve().with_name('liblowbit.so')

_P, _I, _S, _F, _L = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_float, ctypes.c_int64
SIGNATURES = {
    'lb_status_string': ([_I], ctypes.c_char_p),
    'lb_abi_version': ([], _I),
    'lb_last_cuda_error': ([], _I),
    'lb_inject_fault': ([ctypes.c_char_p, _I], _I),
    'lb_workspace_status': ([_P, _P], _I),
    'lb_quantize_workspace_bytes': ([], _S),
    'lb_quantize_pack': ([_I, _I, _P, _I, _I, _I, _P, _P, _P, _S, _P], _I),
    'lb_dequantize': ([_I, _I, _I, _I, _P, _P, _P, _P], _I),
    'lb_linear_workspace_bytes': ([_I, _I, _I, _I, _I, _I], _S),
    'lb_linear': ([_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _S, _P], _I),
    'lb_linear_path': ([_I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _S, _P], _I),
    'lb_linear_select': ([_I, _I, _I, _I, _I, _I], _I),
    'lb_attention_decode_rope': ([_P, _I, _P, _P, _I, _P, _P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _S, _P],
                                 _I),
    'lb_linear_stacked': ([_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P, _S, _P], _I),
    'lb_rmsnorm_project': ([_P, _P, _P, _P, _P, _I, _I, _F, _P, _I, _P, _P], _I),
    'lb_silu_mul_project': ([_P, _P, _I, _P, _I, _I, _P, _I, _P, _P], _I),
    'lb_rmsnorm': ([_P, _P, _P, _P, _P, _I, _I, _F, _P], _I),
    'lb_rope': ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P], _I),
    'lb_kv_append': ([_P, _P, _I, _P, _P, _P, _I, _I, _I, _I, _P], _I),
    'lb_attention_decode': ([_P, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _S, _P], _I),
    'lb_attention_workspace_bytes': ([_I, _I, _I], _S),
    'lb_silu_mul': ([_P, _P, _I, _P, _I, _I, _P], _I),
    'lb_add': ([_P, _P, _P, _L, _P], _I),
    'lb_embed': ([_P, _P, _P, _L, _I, _L, _P], _I),
    'lb_argmax': ([_P, _I, _I, _P, _P, _S, _P], _I),
    'lb_argmax_workspace_bytes': ([_I, _I], _S),
    'lb_linear_gemv_noalloc': ([_I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P], _I),
    'lb_noalloc_status': ([_P], _I),
    'lb_workspace_check': ([_P, _S, _P], _I),
    'lb_test_wait_override': ([ctypes.c_longlong, _I], _I),
}


class LowbitCudaError(RuntimeError):
    """A CUDA launch or runtime failure reported by liblowbit (status LB_ERR_CUDA)."""


class LowbitTimeoutError(RuntimeError):
    """A bounded device-side wait gave up (status LB_ERR_TIMEOUT): the kernel returned
    without faulting, but the output of the call that recorded it is not valid."""


def load_library():
    """Load liblowbit.so and bind every declared symbol; raises if it is missing."""
    global _LIB
    with _LIB_LOCK:
        if _LIB is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f'{LIB_PATH.name} is not built (run torch-intel-npu_b200/build.py)')
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _bind_fast_call(lib)
            _LIB = lib
    return _LIB


# lb_linear_path through the _lowbit_call module (built beside liblowbit.so): the same C
# entry point of the same loaded library, without ctypes' per-argument conversion.  When
# the module is absent the ctypes binding is used.
_FAST_LINEAR = None


def _bind_fast_call(lib):
    global _FAST_LINEAR
    try:
        import _lowbit_call
    except ImportError:
        _FAST_LINEAR = None
        return
    _lowbit_call.bind(ctypes.cast(lib.lb_linear_path, ctypes.c_void_p).value)
    _FAST_LINEAR = _lowbit_call.linear_path


_RAW_STREAM = getattr(torch._C, '_cuda_getCurrentRawStream', None)


def raw_stream(index):
    """Raw handle of torch's current stream on CUDA device ``index``."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(index)
    return torch.cuda.current_stream(torch.device('cuda', index)).cuda_stream


def _current_stream(dev):
    """Raw handle of torch's current stream on CUDA device ``dev``."""
    return raw_stream(dev.index)


def linear_call():
    """The callable that reaches lb_linear_path: the _lowbit_call module when built, else
    the ctypes binding (same arguments: ints for pointers, None for null)."""
    return _FAST_LINEAR if _FAST_LINEAR is not None else lib().lb_linear_path


def lib():
    return _LIB if _LIB is not None else load_library()


_CUDA_OK = False


def require_cuda():
    global _CUDA_OK
    if not _CUDA_OK:
        if not torch.cuda.is_available():
            raise RuntimeError('The B200 low-bit path requires a CUDA device; there is no CPU fallback')
        _CUDA_OK = True
    return lib()


def cuda_device(device=None):
    """Normalise a device spec to an indexed CUDA device (``cuda`` -> ``cuda:<current>``)."""
    dev = torch.device('cuda') if device is None else torch.device(device)
    if dev.type != 'cuda':
        raise ValueError('The B200 low-bit path runs on CUDA devices only')
    return torch.device('cuda', torch.cuda.current_device() if dev.index is None else dev.index)


def check(status, what):
    if status == OK:
        return
    text = lib().lb_status_string(status).decode()
    if status in (INVALID, NONFINITE, OVERFLOW, ALIAS, WORKSPACE, UNSUPPORTED):
        raise ValueError(f'{what}: {text}')
    if status == CUDA_ERR:
        raise LowbitCudaError(f'{what}: {text} (cudaError {lib().lb_last_cuda_error()})')
    if status == TIMEOUT:
        raise LowbitTimeoutError(f'{what}: {text}')
    raise RuntimeError(f'{what}: {text}')


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


class Workspace:
    """Caller-owned scratch for one (device, stream): grown on demand, never shrunk.

    Kernels on the same stream are ordered, so one buffer per stream is race free.
    Inside a CUDA graph capture the buffer must already be large enough
    (``reserve`` before capturing).
    """
    _lock = threading.Lock()
    _buffers = {}

    @classmethod
    def get(cls, nbytes, device=None):
        dev = torch.device('cuda', torch.cuda.current_device() if device is None else torch.device(device).index or 0)
        return cls.for_stream(nbytes, dev.index, torch.cuda.current_stream(dev).cuda_stream)

    @classmethod
    def for_stream(cls, nbytes, index, stream_handle):
        """The buffer of device ``index`` / stream handle, grown to ``nbytes``."""
        key = (index, stream_handle)
        buf = cls._buffers.get(key)
        if buf is not None and buf.numel() >= nbytes:   # common case: no lock needed to read
            return buf
        dev = torch.device('cuda', index)
        with cls._lock:
            buf = cls._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError('workspace must be reserved before CUDA graph capture')
                buf = torch.zeros(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
                cls._buffers[key] = buf
            return buf

    @classmethod
    def reserve(cls, nbytes, device=None):
        return cls.get(nbytes, device)

    @classmethod
    def check(cls, index=None):
        """SYNCHRONOUS: read (and on a set word, reset) the status word of every workspace
        of device ``index`` (all devices when None); raises LowbitTimeoutError if a
        bounded device-side wait of a kernel that used one gave up."""
        L = lib()
        for (dev, stream), buf in list(cls._buffers.items()):
            if index is not None and dev != index:
                continue
            with torch.cuda.device(dev):
                check(L.lb_workspace_check(buf.data_ptr(), buf.numel(), stream), 'workspace status')


def check_device_waits(device=None):
    """Raise LowbitTimeoutError if any linear on ``device`` recorded a timed-out device
    wait since the last check (synchronises the device's workspace streams)."""
    Workspace.check(None if device is None else cuda_device(device).index)


# LOWBIT_CHECK_WAITS=1: every eager ``linear`` call (not under CUDA graph capture) reads
# its workspace status word afterwards and raises on a timed-out wait.  Synchronous, so
# for debugging; graph replays are checked with check_device_waits().
CHECK_WAITS = os.environ.get('LOWBIT_CHECK_WAITS', '0') == '1'


def set_wait_checks(enabled):
    global CHECK_WAITS
    CHECK_WAITS = bool(enabled)


def inject_fault(entry='*', count=1):
    """Make the next ``count`` calls of C entry point ``entry`` fail with LB_ERR_INJECTED."""
    lib().lb_inject_fault(entry.encode(), int(count))


def _contig_cuda(t, name, dtype=None):
    if not isinstance(t, torch.Tensor) or t.device.type != 'cuda':
        raise ValueError(f'{name} must be a CUDA tensor')
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f'{name} must be {dtype}')
    if not t.is_contiguous():
        raise ValueError(f'{name} must be contiguous')
    return t


# ---- thin typed wrappers -------------------------------------------------------------
def quantize_pack(weight, fmt, group):
    """Device quantize+pack: returns (codes uint8, scales fp16) CUDA tensors (synchronous)."""
    L = require_cuda()
    w = _contig_cuda(weight, 'weight')
    if w.dtype not in (torch.float16, torch.float32) or w.ndim != 2:
        raise ValueError('Quantization preparation requires a 2D FP16/FP32 tensor')
    n, k = w.shape
    nbytes = n * k if fmt == 'int8' else (n * k + 1) // 2
    codes = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
    scales = torch.empty(n * (k // group), dtype=torch.float16, device=w.device)
    ws = Workspace.get(L.lb_quantize_workspace_bytes(), w.device)
    with torch.cuda.device(w.device):
        status = L.lb_quantize_pack(LB_FMT[fmt], group, ptr(w), 0 if w.dtype == torch.float32 else 1, n, k,
                                    ptr(codes), ptr(scales), ptr(ws), ws.numel(), stream_ptr(w.device))
    if status == NONFINITE:
        raise ValueError('Nonfinite weights cannot be quantized')
    if status == OVERFLOW:
        raise ValueError('Weight scale overflows FP16')
    check(status, 'lb_quantize_pack')
    return codes, scales


def dequantize(fmt, group, n, k, codes, scales):
    L = require_cuda()
    out = torch.empty(n, k, dtype=torch.float16, device=codes.device)
    check(L.lb_dequantize(LB_FMT[fmt], group, n, k, ptr(codes), ptr(scales), ptr(out), stream_ptr(codes.device)),
          'lb_dequantize')
    return out


def linear_workspace_bytes(fmt, group, m, n, k, rank):
    return lib().lb_linear_workspace_bytes(LB_FMT[fmt], group, m, n, k, rank)


@functools.lru_cache(maxsize=4096)
def _linear_ws_bytes(fmt_id, group, m, n, k, rank):
    return lib().lb_linear_workspace_bytes(fmt_id, group, m, n, k, rank)


linear_ws_bytes_id = _linear_ws_bytes


def _addr(t):
    return None if t is None else t.data_ptr()


def linear(x, fmt, group, n, codes, scales, *, down=None, up=None, bias=None, out=None, path='auto'):
    """y = x . deq(W)^T (+ bias) (+ correction) through lb_linear_path."""
    L = require_cuda()
    x = _contig_cuda(x, 'x', torch.float16)
    m, k = x.shape
    rank = 0 if down is None else down.shape[0]
    fmt_id = LB_FMT[fmt]
    dev = x.device
    y = out if out is not None else torch.empty(m, n, dtype=torch.float16, device=dev)
    stream = _current_stream(dev)
    ws = Workspace.for_stream(_linear_ws_bytes(fmt_id, group, m, n, k, rank), dev.index, stream)
    call = _FAST_LINEAR if _FAST_LINEAR is not None else L.lb_linear_path
    status = call(PATH[path], fmt_id, group, m, n, k, x.data_ptr(), codes.data_ptr(), _addr(scales), _addr(down),
                  _addr(up), rank, _addr(bias), y.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    if status != OK:
        check(status, 'lb_linear')
    if CHECK_WAITS and not torch.cuda.is_current_stream_capturing():
        check(L.lb_workspace_check(ws.data_ptr(), ws.numel(), stream), 'lb_linear')
    return y


def linear_stacked(x, fmt, group, n, codes, scales, *, down=None, up=None, z=None, bias=None, residual=None, out=None):
    """One decode-GEMV launch over several stacked linears (lb_linear_stacked): codes /
    scales / bias are the row-wise concatenation, down / up the block-diagonal stack of
    their corrections (rank <= 128); z, when given, is their projection already computed
    (it replaces down); residual [M, N] is added last."""
    L = require_cuda()
    x = _contig_cuda(x, 'x', torch.float16)
    m, k = x.shape
    rank = 0 if up is None else up.shape[1]
    y = out if out is not None else torch.empty(m, n, dtype=torch.float16, device=x.device)
    if residual is not None:
        residual = _contig_cuda(residual, 'residual', torch.float16)
    ws = Workspace.get(L.lb_linear_workspace_bytes(LB_FMT[fmt], group, m, n, k, rank), x.device)
    status = L.lb_linear_stacked(LB_FMT[fmt], group, m, n, k, ptr(x), ptr(codes), ptr(scales),
                                 ptr(down if z is None else None), ptr(up), ptr(z), rank, ptr(bias), ptr(residual),
                                 ptr(y), ptr(ws), ws.numel(), stream_ptr(x.device))
    check(status, 'lb_linear_stacked')
    return y


def linear_select(fmt, group, m, n, k, rank=0):
    return PATH_NAME[lib().lb_linear_select(LB_FMT[fmt], group, m, n, k, rank)]
