"""Immutable INT4/NF4/INT8 weights with FP16 IO on B200 (drop-in for torch_npu_lowbit).

Same public names, argument meaning and errors as the reference module
(torch_npu_lowbit.py): ``NF4``, ``pack_codes``, ``PackedWeight``, ``quantize_weight``,
``QuantizedLinear``.  The packed bytes are the reference's canonical format, so a
``PackedWeight`` built by either implementation is accepted by the other.

What changes underneath:
* ``quantize_weight`` runs the quantize/pack kernel on the GPU (bit-exact with the
  reference's numpy code) instead of numpy on the CPU;
* ``PackedWeight.dequantize`` runs the GPU dequant kernel (bit-exact) and returns the
  same fp16 numpy array;
* ``QuantizedLinear.forward`` takes CUDA fp16 activations and calls ``lb_linear``
  (dequant-GEMV for decode-sized M, tcgen05 GEMM otherwise) on the current stream,
  instead of compiling an NPU graph and submitting it through ``npu._run``.
The NPU IR builders (``weight_graph``, ``compile_weight``, ``dpu_modes``) and the
offline GPTQ ``calibrate_int8`` have no counterpart here.
"""
from dataclasses import dataclass
from math import prod

import numpy as np
import torch

import lowbit_runtime as rt

# torch_npu_lowbit.py:17-20 -- published NF4 codebook (QLoRA / OpenVINO nf4.cpp)
NF4 = np.array([-1., -.6961928009986877, -.5250730514526367, -.39491748809814453,
                -.28444138169288635, -.18477343022823334, -.09105003625154495, 0.,
                .07958029955625534, .16093020141124725, .24611230194568634, .33791524171829224,
                .44070982933044434, .5626170039176941, .7229568362236023, 1.], dtype=np.float32)
NF4.flags.writeable = False

# The reference bounds N*K by an NPU storage limit (npunlock/npu4000.py:23, 2^20).  HBM on
# a B200 holds far larger weights; the bound kept here only protects 32-bit row indexing.
MAX_TENSOR_ELEMENTS = 1 << 31

_LIMITS = {'int4': 7, 'nf4': 1, 'int8': 127}


def pack_codes(codes):
    """Two 4-bit codes per byte, even element in the low nibble (torch_npu_lowbit.py:24-30)."""
    values = np.asarray(codes)
    if values.dtype != np.uint8 or not values.size or np.any(values > 15):
        raise ValueError('Codes must be a nonempty uint8 array in 0..15')
    flat = values.reshape(-1)
    if flat.size % 2:
        flat = np.concatenate((flat, np.zeros(1, np.uint8)))
    return (flat[0::2] | (flat[1::2] << 4)).astype(np.uint8).tobytes()


@dataclass(frozen=True)
class PackedWeight:
    """Immutable packed weight (torch_npu_lowbit.py:33-75); same fields and validation."""
    shape: tuple
    format: str
    group_size: int
    data: bytes
    scales: bytes

    def __post_init__(self):
        if (type(self.shape) is not tuple or len(self.shape) != 2 or any(type(v) is not int or v <= 0 for v in self.shape)
                or prod(self.shape) > MAX_TENSOR_ELEMENTS or self.format not in ('int4', 'nf4', 'int8')
                or type(self.group_size) is not int or not 1 <= self.group_size <= self.shape[1]
                or self.shape[1] % self.group_size):
            raise ValueError('Weight requires bounded (N,K), int4/nf4/int8, and a group size dividing K')
        if not isinstance(self.data, bytes) or not isinstance(self.scales, bytes):
            raise ValueError('Packed data/scales must be immutable bytes')
        count = prod(self.shape)
        if len(self.data) != (count if self.format == 'int8' else (count + 1) // 2) or (
                self.format != 'int8' and count % 2 and self.data[-1] & 0xf0):
            raise ValueError('Packed weight extent/padding differs')
        if len(self.scales) != 2 * count // self.group_size:
            raise ValueError('Scale extent differs')
        scales = np.frombuffer(self.scales, dtype=np.float16)
        if not np.all(np.isfinite(scales)) or np.any(scales <= 0):
            raise ValueError('Scales must be finite, positive FP16 values')

    @property
    def dtype(self):
        return {'int4': 'i4', 'nf4': 'nf4', 'int8': 'i8'}[self.format]

    @property
    def grouped_shape(self):
        n, k = self.shape
        return n, k // self.group_size, self.group_size

    def to_device(self, device=None):
        """Upload codes and scales once: (codes uint8, scales fp16) CUDA tensors."""
        rt.require_cuda()
        dev = rt.cuda_device(device)
        codes = torch.frombuffer(bytearray(self.data), dtype=torch.uint8).to(dev)
        scales = torch.frombuffer(bytearray(self.scales), dtype=torch.float16).to(dev)
        return codes, scales

    def dequantize(self):
        """fp16 weights rn16(code * scale) computed by the GPU dequant kernel (bit-exact)."""
        codes, scales = self.to_device()
        n, k = self.shape
        out = rt.dequantize(self.format, self.group_size, n, k, codes, scales)
        return out.cpu().numpy()


@dataclass(frozen=True, eq=False)
class DevicePackedWeight:
    """A PackedWeight whose codes and scales already live on a CUDA device (loaded straight
    there from a packed checkpoint).  Same shape / format / group fields and the same
    canonical byte layout; no counterpart in the reference, whose packed weights are host
    bytes compiled into NPU graphs."""
    shape: tuple
    format: str
    group_size: int
    codes: torch.Tensor
    scales: torch.Tensor

    def __post_init__(self):
        if (type(self.shape) is not tuple or len(self.shape) != 2 or any(type(v) is not int or v <= 0 for v in self.shape)
                or prod(self.shape) > MAX_TENSOR_ELEMENTS or self.format not in ('int4', 'nf4', 'int8')
                or type(self.group_size) is not int or not 1 <= self.group_size <= self.shape[1]
                or self.shape[1] % self.group_size):
            raise ValueError('Weight requires bounded (N,K), int4/nf4/int8, and a group size dividing K')
        count = prod(self.shape)
        if (not isinstance(self.codes, torch.Tensor) or self.codes.device.type != 'cuda' or self.codes.dtype != torch.uint8
                or self.codes.numel() != (count if self.format == 'int8' else (count + 1) // 2)):
            raise ValueError('Packed weight extent/padding differs')
        if (not isinstance(self.scales, torch.Tensor) or self.scales.device != self.codes.device
                or self.scales.dtype != torch.float16 or self.scales.numel() != count // self.group_size):
            raise ValueError('Scale extent differs')
        if not bool((torch.isfinite(self.scales) & (self.scales > 0)).all()):
            raise ValueError('Scales must be finite, positive FP16 values')
        if self.format != 'int8' and count % 2 and int(self.codes[-1]) & 0xf0:
            raise ValueError('Packed weight extent/padding differs')

    def to_device(self, device=None):
        dev = rt.cuda_device(device) if device is not None else self.codes.device
        return self.codes.to(dev).contiguous(), self.scales.to(dev).contiguous()

    def to_host(self):
        """The host PackedWeight with the same bytes."""
        return PackedWeight(self.shape, self.format, self.group_size, self.codes.cpu().numpy().tobytes(),
                            self.scales.cpu().numpy().tobytes())

    def dequantize(self):
        n, k = self.shape
        return rt.dequantize(self.format, self.group_size, n, k, self.codes, self.scales).cpu().numpy()


def quantize_weight(weight, *, format='int4', group_size=None):
    """Symmetric per-group quantization with fp16 scales (torch_npu_lowbit.py:78-105), on the GPU.

    Accepts a 2-D fp16/fp32 tensor on the CPU (as the reference) or on a CUDA device.
    """
    if (not isinstance(weight, torch.Tensor) or weight.device.type not in ('cpu', 'cuda') or weight.ndim != 2
            or weight.dtype not in (torch.float16, torch.float32)):
        raise ValueError('Quantization preparation requires a CPU 2D Tensor')
    n, k = weight.shape
    size = k if group_size is None else group_size
    if (format not in _LIMITS or type(size) is not int or not 1 <= size <= k
            or k % size or not 0 < n * k <= MAX_TENSOR_ELEMENTS):
        raise ValueError('Requires int4/nf4/int8 and a group size dividing bounded K')
    rt.require_cuda()
    w = weight.detach()
    if w.device.type != 'cuda':
        w = w.to('cuda', non_blocking=False)
    codes, scales = rt.quantize_pack(w.contiguous(), format, size)
    return PackedWeight((n, k), format, size, codes.cpu().numpy().tobytes(), scales.cpu().numpy().tobytes())


def quantize_weight_device(weight, *, format='int4', group_size=None):
    """Device-resident variant: returns (codes, scales) CUDA tensors without a host round trip."""
    n, k = weight.shape
    size = k if group_size is None else group_size
    if format not in _LIMITS or type(size) is not int or not 1 <= size <= k or k % size:
        raise ValueError('Requires int4/nf4/int8 and a group size dividing bounded K')
    return rt.quantize_pack(weight.detach().contiguous(), format, size)


class QuantizedLinear(torch.nn.Module):
    """Frozen fp16-IO low-bit linear on the GPU (torch_npu_lowbit.py:300-360).

    ``correction`` (keyword-only, not in the reference module) attaches a
    ``LowRankCorrection``; the output then follows the reference's corrected-projection
    staging (torch_npu_smollm.py:160-163).  ``compact_groups`` and ``activation_scale``
    select NPU-specific graph variants and raise ``NotImplementedError`` when set.
    """

    def __init__(self, weight, *, bias=None, compact_groups=False, activation_scale=None, correction=None, device=None):
        super().__init__()
        if not isinstance(weight, PackedWeight):
            raise ValueError('Requires a PackedWeight')
        if type(compact_groups) is not bool:
            raise ValueError('compact_groups requires bool and at most 32 groups')
        if compact_groups:
            raise NotImplementedError('compact_groups is an NPU graph variant with no B200 counterpart')
        if activation_scale is not None:
            raise NotImplementedError('W8A8 activation quantization is outside the B200 low-bit path')
        self._weight = weight
        self._compact_groups = False
        self._activation_scale = None
        rt.require_cuda()
        self._device = rt.cuda_device(device)
        self._codes, self._scales = weight.to_device(self._device)
        if bias is not None:
            if (not isinstance(bias, torch.Tensor) or bias.device.type != 'cpu' or bias.shape != (weight.shape[0],)
                    or bias.dtype not in (torch.float16, torch.float32) or not torch.isfinite(bias).all()):
                raise ValueError('Bias preparation requires N finite CPU FP16/FP32 values')
            converted = bias.detach().half()
            if not torch.isfinite(converted).all():
                raise ValueError('Bias overflows FP16')
            self._bias = converted.contiguous().numpy().tobytes()
            self._bias_dev = converted.to(self._device)
        else:
            self._bias = None
            self._bias_dev = None
        self._down = self._up = None
        if correction is not None:
            from torch_npu_lowbit_correction import LowRankCorrection
            if not isinstance(correction, LowRankCorrection) or correction.shape != weight.shape or correction.rank > 32:
                raise ValueError('Correction requires matching rank<=32 factors')
            down, up = correction.tensors()
            self._down, self._up = down.to(self._device), up.to(self._device)
        self._correction = correction
        # per-call constants of the lb_linear_path call (forward's fast path)
        n, k = weight.shape
        self._n, self._k, self._dev_index = n, k, self._device.index
        self._fmt_id = rt.LB_FMT[weight.format]
        self._rank = 0 if self._down is None else self._down.shape[0]
        self._ptrs = (self._codes.data_ptr(), self._scales.data_ptr(),
                      None if self._down is None else self._down.data_ptr(),
                      None if self._up is None else self._up.data_ptr())
        self._bias_ptr = None if self._bias_dev is None else self._bias_dev.data_ptr()
        self._ws = {}

    @property
    def weight(self):
        return self._weight

    @property
    def bias(self):
        return self._bias

    @property
    def compact_groups(self):
        return self._compact_groups

    @property
    def activation_scale(self):
        return self._activation_scale

    @property
    def correction(self):
        return self._correction

    @classmethod
    def from_float(cls, module, *, format='int4', group_size=None, compact_groups=False, activation_scale=None,
                   correction=None, device=None):
        if not isinstance(module, torch.nn.Linear) or module.weight.device.type != 'cpu':
            raise ValueError('Requires a CPU nn.Linear for preparation')
        return cls(quantize_weight(module.weight, format=format, group_size=group_size), bias=module.bias,
                   compact_groups=compact_groups, activation_scale=activation_scale, correction=correction,
                   device=device)

    def _check_input(self, x):
        if (not isinstance(x, torch.Tensor) or x.dtype != torch.float16 or x.ndim != 2
                or x.shape[1] != self.weight.shape[1]):
            raise ValueError('QuantizedLinear requires 2D FP16 activations with matching K')
        if x.device != self._device:
            raise ValueError(f'QuantizedLinear lives on {self._device}; got activations on {x.device}')

    def forward(self, x, *, out=None, path='auto'):
        # fast checks first (a decode call is a few microseconds of GPU work); any mismatch
        # takes the full validation, which raises the reference's error
        if (type(x) is not torch.Tensor or x.dtype is not torch.float16 or x.dim() != 2 or x.shape[1] != self._k
                or x.get_device() != self._dev_index):
            self._check_input(x)
        if not x.is_contiguous():
            x = x.contiguous()
        m, n = x.shape[0], self._n
        if out is None:
            out = torch.empty(m, n, dtype=torch.float16, device=self._device)
        elif (type(out) is not torch.Tensor or out.dtype is not torch.float16 or out.dim() != 2 or out.shape[0] != m
              or out.shape[1] != n or out.get_device() != self._dev_index or not out.is_contiguous()):
            raise ValueError('out must be a contiguous FP16 [M, N] tensor on the module device')
        stream = rt.raw_stream(self._dev_index)
        ws = self._ws.get((stream, m))
        if ws is None:
            if len(self._ws) > 64:
                self._ws.clear()
            ws = rt.Workspace.for_stream(rt.linear_ws_bytes_id(self._fmt_id, self.weight.group_size, m, n, self._k,
                                                               self._rank), self._dev_index, stream)
            if not torch.cuda.is_current_stream_capturing():
                self._ws[(stream, m)] = ws
        codes, scales, down, up = self._ptrs
        status = rt.linear_call()(rt.PATH[path], self._fmt_id, self.weight.group_size, m, n, self._k, x.data_ptr(),
                                  codes, scales, down, up, self._rank, self._bias_ptr, out.data_ptr(), ws.data_ptr(),
                                  ws.numel(), stream)
        if status != rt.OK:
            rt.check(status, 'lb_linear')
        if rt.CHECK_WAITS and not torch.cuda.is_current_stream_capturing():
            rt.check(rt.lib().lb_workspace_check(ws.data_ptr(), ws.numel(), stream), 'lb_linear')
        return out
