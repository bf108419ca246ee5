"""CPU restatement of the reference low-bit codec and linear staging (TEST INFRASTRUCTURE).

This module is the parity oracle for the B200 path.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it, and only as the checker or the timed CPU baseline; the
product path (``torch-intel-npu_b200/``) never imports it.

Every function restates one piece of the reference (LCS-Official/torch-intel-npu)
and cites the line it follows.  Byte and integer work is numpy; the floating
point linear staging uses torch CPU ops in the same order as the reference so the
restatement can be pinned bitwise against the reference's own outputs
(``tests/golden/make_golden.py`` generated the fixtures it is checked against).
"""
from math import prod

import numpy as np
import torch
import torch.nn.functional as F

# torch_npu_lowbit.py:17-20 -- the 16-entry normal-float codebook (the published
# NF4 table from QLoRA / OpenVINO nf4.cpp), fp32.
NF4 = np.array([-1., -.6961928009986877, -.5250730514526367, -.39491748809814453,
                -.28444138169288635, -.18477343022823334, -.09105003625154495, 0.,
                .07958029955625534, .16093020141124725, .24611230194568634, .33791524171829224,
                .44070982933044434, .5626170039176941, .7229568362236023, 1.], dtype=np.float32)
NF4.flags.writeable = False

# torch_npu_lowbit.py:92 -- symmetric code limits per format.
LIMITS = {'int4': 7, 'nf4': 1, 'int8': 127}


def nf4_midpoints():
    """torch_npu_lowbit.py:102 -- fp32 decision boundaries between adjacent NF4 codes."""
    return (NF4[:-1] + NF4[1:]) / 2


def pack_codes(codes):
    """torch_npu_lowbit.py:24-30 -- two 4-bit codes per byte, even element in the low nibble.

    An odd element count is padded with a zero high nibble.
    """
    values = np.asarray(codes)
    if values.dtype != np.uint8 or not values.size or np.any(values > 15):
        raise ValueError('Codes must be a nonempty uint8 array in 0..15')
    flat = values.reshape(-1)
    if flat.size % 2:
        flat = np.concatenate((flat, np.zeros(1, np.uint8)))
    return (flat[0::2] | (flat[1::2] << 4)).astype(np.uint8).tobytes()


def unpack_codes(data, count):
    """Inverse of pack_codes (torch_npu_lowbit.py:71-72): bytes -> ``count`` uint8 codes."""
    raw = np.frombuffer(data, dtype=np.uint8)
    return np.stack((raw & 15, raw >> 4), axis=1).reshape(-1)[:count]


def validate_packed(shape, fmt, group_size, data, scales, max_elements):
    """torch_npu_lowbit.py:41-56 -- PackedWeight.__post_init__ checks, same order."""
    if (type(shape) is not tuple or len(shape) != 2 or any(type(v) is not int or v <= 0 for v in shape)
            or prod(shape) > max_elements or fmt not in ('int4', 'nf4', 'int8')
            or type(group_size) is not int or not 1 <= group_size <= shape[1] or shape[1] % group_size):
        raise ValueError('Weight requires bounded (N,K), int4/nf4/int8, and a group size dividing K')
    if not isinstance(data, bytes) or not isinstance(scales, bytes):
        raise ValueError('Packed data/scales must be immutable bytes')
    count = prod(shape)
    expected = count if fmt == 'int8' else (count + 1) // 2
    if len(data) != expected or (fmt != 'int8' and count % 2 and data[-1] & 0xf0):
        raise ValueError('Packed weight extent/padding differs')
    if len(scales) != 2 * count // group_size:
        raise ValueError('Scale extent differs')
    s = np.frombuffer(scales, dtype=np.float16)
    if not np.all(np.isfinite(s)) or np.any(s <= 0):
        raise ValueError('Scales must be finite, positive FP16 values')


def decode_values(fmt, data, count):
    """torch_npu_lowbit.py:69-73 -- per-element fp16 code values before scaling."""
    if fmt == 'int8':
        return np.frombuffer(data, dtype=np.int8)[:count].astype(np.float16)
    codes = unpack_codes(data, count)
    if fmt == 'int4':
        return ((codes.astype(np.int8) ^ 8) - 8).astype(np.float16)
    return NF4[codes].astype(np.float16)


def dequantize(shape, fmt, group_size, data, scales):
    """torch_npu_lowbit.py:67-75 -- fp16 weight = rn16(code_value_fp16 * scale_fp16)."""
    n, k = shape
    values = decode_values(fmt, data, n * k).reshape(n, k // group_size, group_size)
    s = np.frombuffer(scales, dtype=np.float16).reshape(n, k // group_size, 1)
    return (values * s).reshape(n, k)


def quantize(weight, fmt, group_size=None):
    """torch_npu_lowbit.py:78-105 -- symmetric per-group absmax round-to-nearest.

    ``weight`` is a 2-D float array (fp16 or fp32).  Returns ``(group, data, scales)``.
    """
    values = np.asarray(weight)
    if values.ndim != 2 or values.dtype not in (np.float16, np.float32):
        raise ValueError('Quantization preparation requires a CPU 2D Tensor')
    n, k = values.shape
    size = k if group_size is None else group_size
    if fmt not in LIMITS or type(size) is not int or not 1 <= size <= k or k % size or not 0 < n * k:
        raise ValueError('Requires int4/nf4/int8 and a group size dividing bounded K')
    v = values.astype(np.float32).reshape(n, k // size, size)
    if not np.all(np.isfinite(v)):
        raise ValueError('Nonfinite weights cannot be quantized')
    maximum = np.max(np.abs(v), axis=-1, keepdims=True)
    limit = LIMITS[fmt]
    scale = maximum / np.float32(limit)
    if np.any(scale > np.finfo(np.float16).max):
        raise ValueError('Weight scale overflows FP16')
    scale = np.maximum(scale, np.float32(2 ** -24)).astype(np.float16)
    normalized = v / scale.astype(np.float32)
    if fmt in ('int4', 'int8'):
        codes = np.clip(np.rint(normalized), -limit, limit).astype(np.int8)
        data = codes.tobytes() if fmt == 'int8' else pack_codes((codes & 15).astype(np.uint8))
    else:
        codes = np.searchsorted(nf4_midpoints(), normalized, side='left').astype(np.uint8)
        data = pack_codes(codes)
    return size, data, scale.tobytes()


def prepare_weight(shape, fmt, group_size, data, scales):
    """The weight operand of the per-format staging below, computed once.

    * int8 with per-row scales: ``codes * scales`` in float64 (torch_npu_smollm.py:153-157).
    * every other format: ``float32(dequantize())`` (torch_npu_smollm.py:158-159).
    Caching it is the reference's own demo path (torch_npu_lowbit_demo.py:65-71: the
    dequantized weight is computed once and reused); the values are the same as
    dequantizing on every call.
    """
    n, k = shape
    if fmt == 'int8' and group_size == k:
        codes = np.frombuffer(data, dtype=np.int8).reshape(shape)
        s = np.frombuffer(scales, dtype=np.float16).astype(np.float64)
        return torch.from_numpy(codes.astype(np.float64) * s[:, None])
    return torch.from_numpy(dequantize(shape, fmt, group_size, data, scales).copy()).float()


def linear_prepared(x, weight, *, down=None, up=None, bias=None):
    """torch_npu_smollm.py:150-164 with the weight operand from ``prepare_weight``."""
    x = x.detach().half()
    if weight.dtype == torch.float64:
        value = (x.double() @ weight.t()).half()
    else:
        value = F.linear(x.float(), weight).half()
    if bias is not None:
        value = (value + bias.half()).half()
    if down is not None:
        delta = F.linear(F.linear(x.float(), down.float()).half().float(), up.float()).half()
        value = (value + delta).half()
    return value


def linear(x, shape, fmt, group_size, data, scales, *, down=None, up=None, bias=None):
    """Per-format CPU linear staging, torch_npu_smollm.py:150-164 (plus a bias add).

    * int8 (per-row scales): ``half(float64(x) @ (codes * scales)^T)`` (:153-157).
    * int8 grouped / int4 / nf4: ``half(F.linear(float32(x), float32(dequantize())))`` (:158-159).
    * bias (torch_npu_lowbit.py:262-266, an fp16 graph Add): ``half(y + bias)``.
    * correction (:160-163): ``delta = half(F.linear(half(F.linear(x, V)), U))``; ``y = half(y + delta)``.

    ``x`` is a CPU fp16 tensor [M, K]; ``down`` = V [r, K] and ``up`` = U [N, r] fp16 tensors.
    The weight is dequantized on every call, as ``reference_cpu`` does (:159).
    """
    return linear_prepared(x, prepare_weight(shape, fmt, group_size, data, scales), down=down, up=up, bias=bias)


def correction_delta(x, down, up):
    """torch_npu_smollm.py:162 -- the rank-r correction term alone, fp16."""
    return F.linear(F.linear(x.float(), down.float()).half().float(), up.float()).half()


def validate_correction(shape, rank, down, up, max_elements):
    """torch_npu_lowbit_correction.py:22-28 -- LowRankCorrection.__post_init__ checks."""
    if (type(shape) is not tuple or len(shape) != 2 or any(type(v) is not int or v <= 0 for v in shape)
            or prod(shape) > max_elements or type(rank) is not int or not 1 <= rank <= min(shape)):
        raise ValueError('Correction requires bounded (N,K) and rank in 1..min(N,K)')
    for blob, count in ((down, rank * shape[1]), (up, shape[0] * rank)):
        if type(blob) is not bytes or len(blob) != count * 2 or not np.isfinite(np.frombuffer(blob, dtype=np.float16)).all():
            raise ValueError('Correction factors require finite immutable FP16 data of the declared shape')


def gemv_bytes(m, n, k, fmt, group_size, rank=32):
    """Algorithmic HBM bytes of one dequant-GEMV call: codes + scales + factors + x + y."""
    bits = 8 if fmt == 'int8' else 4
    return (n * k * bits) // 8 + 2 * n * (k // group_size) + 2 * rank * (n + k) + 2 * m * k + 2 * m * n


def gemm_flops(m, n, k, rank=32):
    """Algorithmic flops of one dequant-GEMM call including the rank-r correction."""
    return 2 * m * n * k + 2 * m * rank * (n + k)
