"""CPU restatement of the reference SmolLM decoder staging (TEST INFRASTRUCTURE).

Restates ``FrozenSmolLayer.reference_cpu`` (torch_npu_smollm.py:142-193) and
``FrozenSmolIO.embed_tokens/logits`` (torch_npu_smollm_io.py:45-61), generalised to
configurable dimensions and RoPE theta and extended with an explicit KV cache so
that prefill + greedy decode can be run position by position.  The reference layer
is hard-wired to hidden 576, 9/3 heads, theta 100000 and <=64 positions
(torch_npu_smollm.py:79-83, :111-116); at those dimensions this restatement is
pinned bitwise against the reference (tests/golden/make_golden.py).

Only tests, smoke() and the CPU-baseline legs of bench.py may use this module.
"""
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import lowbit_ref

PROJECTIONS = ('self_attn.q_proj.weight', 'self_attn.k_proj.weight', 'self_attn.v_proj.weight',
               'self_attn.o_proj.weight', 'mlp.gate_proj.weight', 'mlp.up_proj.weight',
               'mlp.down_proj.weight')


@dataclass(frozen=True)
class DecoderDims:
    hidden: int = 576
    intermediate: int = 1536
    heads: int = 9
    kv_heads: int = 3
    head_dim: int = 64
    vocab: int = 49152
    eps: float = 1e-5
    theta: float = 100000.0

    def shapes(self):
        q = self.heads * self.head_dim
        kv = self.kv_heads * self.head_dim
        d, f = self.hidden, self.intermediate
        return {'self_attn.q_proj.weight': (q, d), 'self_attn.k_proj.weight': (kv, d),
                'self_attn.v_proj.weight': (kv, d), 'self_attn.o_proj.weight': (d, q),
                'mlp.gate_proj.weight': (f, d), 'mlp.up_proj.weight': (f, d),
                'mlp.down_proj.weight': (d, f),
                'input_layernorm.weight': (d,), 'post_attention_layernorm.weight': (d,)}


def rope_tables(dims, positions):
    """torch_npu_smollm.py:113-116 -- fp16 cos/sin tables [positions, head_dim]."""
    hd = dims.head_dim
    frequency = 1. / (dims.theta ** (torch.arange(0, hd, 2).float() / hd))
    angles = torch.outer(torch.arange(positions).float(), frequency)
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos().half(), angles.sin().half()


class LayerRef:
    """One decoder layer; ``packed[name]`` = (shape, fmt, group, data, scales) or None for fp16."""

    def __init__(self, dims, weights, packed=None, corrections=None, cache_weights=False):
        """``cache_weights`` dequantizes each projection once and reuses it (the same
        values; torch_npu_lowbit_demo.py:65-71), instead of per call as reference_cpu does."""
        self.dims = dims
        self.weights = {k: v.detach().half() for k, v in weights.items()}
        self.packed = packed or {}
        self.corrections = corrections or {}
        self.cache_weights = cache_weights
        self._prepared = {}

    def linear(self, v, name):
        """torch_npu_smollm.py:150-165."""
        q = self.packed.get(name)
        corr = self.corrections.get(name)
        if q is None:
            value = F.linear(v.float(), self.weights[name].float()).half()
            if corr is not None:
                value = (value + lowbit_ref.correction_delta(v, *corr)).half()
            return value
        shape = q[0]
        lead = v.shape[:-1]
        flat = v.reshape(-1, v.shape[-1])
        down, up = corr if corr is not None else (None, None)
        if self.cache_weights:
            w = self._prepared.get(name)
            if w is None:
                w = self._prepared[name] = lowbit_ref.prepare_weight(*q)
            out = lowbit_ref.linear_prepared(flat, w, down=down, up=up)
        else:
            out = lowbit_ref.linear(flat, *q, down=down, up=up)
        return out.reshape(*lead, shape[0])

    def norm(self, v, name):
        """torch_npu_smollm.py:166-168 -- fp32 statistics, fp16 scaling."""
        value = v.float()
        normalized = (value * torch.rsqrt(value.square().mean(-1, keepdim=True) + self.dims.eps)).half()
        return (normalized * self.weights[name]).half()

    def forward(self, x, cos, sin, cache=None):
        """torch_npu_smollm.py:169-193 with a KV cache.

        ``x`` fp16 [B,S,d] holds positions ``start .. start+S-1`` where ``start`` is the
        cache length; ``cos``/``sin`` are full tables.  Returns (output, (keys, values)).
        """
        dm = self.dims
        b, length, d = x.shape
        start = 0 if cache is None else cache[0].shape[2]
        hd, h, kvh = dm.head_dim, dm.heads, dm.kv_heads
        half = hd // 2
        normalized = self.norm(x, 'input_layernorm.weight')
        q = self.linear(normalized, 'self_attn.q_proj.weight').view(b, length, h, hd).transpose(1, 2)
        k = self.linear(normalized, 'self_attn.k_proj.weight').view(b, length, kvh, hd).transpose(1, 2)
        v = self.linear(normalized, 'self_attn.v_proj.weight').view(b, length, kvh, hd).transpose(1, 2)
        c = cos[start:start + length][None, None]
        s = sin[start:start + length][None, None]

        def rotate(value):
            return (value * c + torch.cat((-value[..., half:], value[..., :half]), -1) * s).half()

        q = rotate(q)
        k = rotate(k)
        if cache is not None:
            k = torch.cat((cache[0], k), dim=2)
            v = torch.cat((cache[1], v), dim=2)
        new_cache = (k, v)
        rep = h // kvh
        kk = k.repeat_interleave(rep, dim=1)
        vv = v.repeat_interleave(rep, dim=1)
        total = start + length
        scores = (q.float() @ kk.float().transpose(-1, -2)).half()
        scores = (scores * (1.0 / hd ** 0.5)).half()
        mask = torch.triu(torch.full((total, total), float('-inf')), diagonal=1)[start:total]
        probs = (scores + mask).float().softmax(-1).half()
        attended = (probs.float() @ vv.float()).half().transpose(1, 2).reshape(b, length, h * hd)
        value = (x + self.linear(attended, 'self_attn.o_proj.weight')).half()
        normalized = self.norm(value, 'post_attention_layernorm.weight')
        gate = self.linear(normalized, 'mlp.gate_proj.weight')
        up = self.linear(normalized, 'mlp.up_proj.weight')
        hidden = (F.silu(gate.float()).half() * up).half()
        value = (value + self.linear(hidden, 'mlp.down_proj.weight')).half()
        return value, new_cache


class DecoderRef:
    """Stack of LayerRef plus the tied fp16 embedding / final-norm endpoints."""

    def __init__(self, dims, layers, embedding, norm, max_positions):
        self.dims = dims
        self.layers = layers
        self.embedding = embedding.detach().half()
        self.final_norm = norm.detach().half()
        self.cos, self.sin = rope_tables(dims, max_positions)

    def embed(self, ids):
        """torch_npu_smollm_io.py:45-50."""
        return F.embedding(ids, self.embedding)

    def logits(self, hidden):
        """torch_npu_smollm_io.py:52-61 -- fp32 variance, fp16 scale, fp16 tied head."""
        value = hidden.float()
        inverse = torch.rsqrt(value.square().mean(-1, keepdim=True) + self.dims.eps)
        normalized = (value * inverse).half() * self.final_norm
        return F.linear(normalized.float(), self.embedding.float()).half()

    def step(self, x, caches):
        out = []
        for i, layer in enumerate(self.layers):
            x, cache = layer.forward(x, self.cos, self.sin, None if caches is None else caches[i])
            out.append(cache)
        return x, out

    def generate(self, ids, steps):
        """Prefill ``ids`` [B,S] then ``steps`` greedy tokens; returns (tokens [B,steps], logits list)."""
        hidden, caches = self.step(self.embed(ids), None)
        logits = [self.logits(hidden[:, -1:])[:, 0]]
        tokens = [logits[-1].float().argmax(-1)]
        for _ in range(steps - 1):
            hidden, caches = self.step(self.embed(tokens[-1][:, None]), caches)
            logits.append(self.logits(hidden[:, -1:])[:, 0])
            tokens.append(logits[-1].float().argmax(-1))
        return torch.stack(tokens, 1), logits
