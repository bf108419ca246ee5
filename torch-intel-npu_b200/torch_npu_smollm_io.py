"""Tied SmolLM embedding and final-norm / LM-head endpoints on the GPU (drop-in for
torch_npu_smollm_io).

Same class, constructor, ``from_checkpoint``, ``embed_tokens`` and ``logits`` as the
reference's ``FrozenSmolIO`` (torch_npu_smollm_io.py:14-61), with the same validation
and fp16 staging: fp32 variance and inverse, fp16 scaling by the norm weight, fp16 tied
head.  What changes: the endpoint buffers live on a CUDA device and both calls run there
(the library's embedding gather, RMSNorm and fp16 GEMV/GEMM kernels), so the decoder's
hidden states never leave the GPU; the hidden size comes from the config instead of
being fixed at 576.
"""
import json
from pathlib import Path

import torch

import lowbit_runtime as rt


class FrozenSmolIO(torch.nn.Module):
    """Inference-only tied embedding and norm/output head on a CUDA device."""

    def __init__(self, config, embedding, norm, *, device=None):
        super().__init__()
        d = config.get('hidden_size')
        if (config.get('model_type') != 'llama' or type(d) is not int or d <= 0
                or config.get('tie_word_embeddings') is not True or config.get('rms_norm_eps') != 1e-5
                or type(config.get('vocab_size')) is not int or config['vocab_size'] <= 0):
            raise ValueError('Requires tied SmolLM endpoints with RMSNorm eps=1e-5')
        rt.require_cuda()
        self.device = rt.cuda_device(device)
        for name, value, shape in (('embedding', embedding, (config['vocab_size'], d)), ('norm', norm, (d,))):
            if (not isinstance(value, torch.Tensor) or tuple(value.shape) != shape
                    or value.dtype not in (torch.float16, torch.bfloat16, torch.float32) or not torch.isfinite(value).all()):
                raise ValueError('Requires finite floating endpoint weights of the expected shape')
            half = value.detach().to(device=self.device, dtype=torch.float16, copy=True,
                                     memory_format=torch.contiguous_format)
            if not torch.isfinite(half).all():
                raise ValueError('Endpoint weight overflows FP16')
            self.register_buffer(name, half)
        self.hidden = d
        self.vocab = config['vocab_size']
        self.eps = float(config['rms_norm_eps'])
        self.eval()

    @classmethod
    def from_checkpoint(cls, directory, *, device=None):
        from safetensors import safe_open
        directory = Path(directory)
        config = json.loads((directory / 'config.json').read_text())
        with safe_open(directory / 'model.safetensors', framework='pt', device='cpu') as file:
            if 'lm_head.weight' in file.keys():
                raise ValueError('Requires the canonical tied checkpoint without a separate lm_head weight')
            return cls(config, file.get_tensor('model.embed_tokens.weight'), file.get_tensor('model.norm.weight'),
                       device=device)

    def _check_eval(self):
        if self.training:
            raise ValueError('FrozenSmolIO requires eval mode')

    def embed_rows(self, ids):
        """Rows of the table for flat int64 ids already on the device: [T, d] fp16."""
        t = ids.numel()
        out = torch.empty(t, self.hidden, dtype=torch.float16, device=self.device)
        rt.check(rt.lib().lb_embed(rt.ptr(ids), rt.ptr(self.embedding), rt.ptr(out), t, self.hidden, self.vocab,
                                   rt.stream_ptr(self.device)), 'lb_embed')
        return out

    def embed_tokens(self, ids):
        """(B, S) int64 token ids -> (B, S, d) fp16 on the device (torch_npu_smollm_io.py:45-50)."""
        self._check_eval()
        if (not isinstance(ids, torch.Tensor) or ids.dtype != torch.int64 or ids.ndim != 2
                or any(size <= 0 for size in ids.shape)):
            raise ValueError('Embedding requires nonempty int64 (B,S) token IDs')
        b, s = ids.shape
        return self.embed_rows(ids.to(self.device).contiguous().reshape(-1)).view(b, s, self.hidden)

    def head_rows(self, h, residual=None):
        """Final RMSNorm (fused with a last residual add when given) + tied head of [T, d]
        rows -> [T, vocab] fp16 logits."""
        normed = torch.empty_like(h)
        res_out = torch.empty_like(h) if residual is not None else None
        rt.check(rt.lib().lb_rmsnorm(rt.ptr(h), rt.ptr(residual), rt.ptr(res_out), rt.ptr(self.norm), rt.ptr(normed),
                                     h.shape[0], h.shape[1], self.eps, rt.stream_ptr(self.device)), 'lb_rmsnorm')
        return rt.linear(normed, 'fp16', self.hidden, self.vocab, self.embedding.view(torch.uint8).reshape(-1), None)

    def logits(self, hidden):
        """(B, S, d) fp16 hidden states -> (B, S, vocab) fp16 logits (torch_npu_smollm_io.py:52-61)."""
        self._check_eval()
        if (not isinstance(hidden, torch.Tensor) or hidden.device != self.device or hidden.dtype != torch.float16
                or hidden.ndim != 3 or hidden.shape[-1] != self.hidden or any(size <= 0 for size in hidden.shape)):
            raise ValueError(f'Output head requires nonempty FP16 (B,S,{self.hidden}) hidden states on {self.device}')
        b, s, _ = hidden.shape
        return self.head_rows(hidden.reshape(b * s, self.hidden).contiguous()).view(b, s, self.vocab)
