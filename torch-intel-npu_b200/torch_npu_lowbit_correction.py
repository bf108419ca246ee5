"""Immutable low-rank residual factors (drop-in for torch_npu_lowbit_correction).

``LowRankCorrection`` keeps the reference's fields, validation and ``tensors``/``truncated``
behaviour (torch_npu_lowbit_correction.py:15-39).  At inference the correction is fused
into the B200 linear kernels (z = half(x V^T) projected once, delta = half(z U^T) in the
GEMV epilogue or as a second TMEM accumulator of the tcgen05 GEMM).  The offline
ridge-SVD fitting (``fit_lowrank_correction``, CPU fp64 preparation) has no GPU
counterpart in this package.
"""
from dataclasses import dataclass
from math import prod

import numpy as np
import torch

from torch_npu_lowbit import MAX_TENSOR_ELEMENTS


@dataclass(frozen=True)
class LowRankCorrection:
    shape: tuple
    rank: int
    down: bytes
    up: bytes

    def __post_init__(self):
        if (type(self.shape) is not tuple or len(self.shape) != 2 or any(type(n) is not int or n <= 0 for n in self.shape)
                or prod(self.shape) > MAX_TENSOR_ELEMENTS or type(self.rank) is not int
                or not 1 <= self.rank <= min(self.shape)):
            raise ValueError('Correction requires bounded (N,K) and rank in 1..min(N,K)')
        for data, count in ((self.down, self.rank * self.shape[1]), (self.up, self.shape[0] * self.rank)):
            if type(data) is not bytes or len(data) != count * 2 or not np.isfinite(np.frombuffer(data, dtype=np.float16)).all():
                raise ValueError('Correction factors require finite immutable FP16 data of the declared shape')

    def tensors(self, rank=None):
        """(V [rank, K], U [N, rank]) fp16 CPU tensors, a prefix of the stored rank."""
        rank = self.rank if rank is None else rank
        if type(rank) is not int or not 1 <= rank <= self.rank:
            raise ValueError('Invalid correction rank')
        a = torch.from_numpy(np.frombuffer(self.down, dtype=np.float16).reshape(self.rank, self.shape[1]).copy())
        b = torch.from_numpy(np.frombuffer(self.up, dtype=np.float16).reshape(self.shape[0], self.rank).copy())
        return a[:rank].contiguous(), b[:, :rank].contiguous()

    def truncated(self, rank):
        a, b = self.tensors(rank)
        return LowRankCorrection(self.shape, rank, a.numpy().tobytes(), b.numpy().tobytes())

    @classmethod
    def from_tensors(cls, down, up):
        """Build from fp16 V [r, K] and U [N, r] tensors (any device)."""
        down = down.detach().half().cpu().contiguous()
        up = up.detach().half().cpu().contiguous()
        return cls((up.shape[0], down.shape[1]), down.shape[0], down.numpy().tobytes(), up.numpy().tobytes())
