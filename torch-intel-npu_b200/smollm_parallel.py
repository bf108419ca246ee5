"""Multi-GPU partitioning of the SmolLM low-bit decoder (one process per GPU).

Two strategies, both for configs the reference (single NPU, torch_intel_npu.py:102-107)
has no counterpart for:

* batch sharding (SmolLM-360M, batch 64): every rank holds a full weight replica and
  decodes its own slice of the independent sequences -- no collective on the data path;
* tensor parallelism (SmolLM-1.7B): q/k/v/gate/up are column-sharded (output rows, i.e.
  whole heads and FFN columns), o/down are row-sharded (input columns).  The row-sharded
  projections produce fp32 partial sums that one NCCL all-reduce over NVLink combines
  before the reference's fp16 rounding; their rank-32 correction needs z = x V^T over the
  full K, so the [M, 32] partial projections are summed in the same all-reduce.

Packed weights are split on the reference's canonical bytes (torch_npu_lowbit.py:24-30):
column shards are whole rows (byte ranges when K is even), row shards take a byte range
of every row and the matching scale groups, so every shard is itself a valid
PackedWeight whose quantization equals the unsharded one.
"""
from math import prod

import numpy as np
import torch

from torch_npu_lowbit import PackedWeight
from torch_npu_lowbit_correction import LowRankCorrection

COLUMN = ('self_attn.q_proj.weight', 'self_attn.k_proj.weight', 'self_attn.v_proj.weight',
          'mlp.gate_proj.weight', 'mlp.up_proj.weight')
ROW = ('self_attn.o_proj.weight', 'mlp.down_proj.weight')


def batch_shard(batch, rank, world):
    """[start, stop) of the sequences rank ``rank`` decodes (contiguous, sizes differ by <= 1)."""
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _bits(fmt):
    return 8 if fmt == 'int8' else 4


def shard_packed_rows(q, rank, world):
    """Column-parallel shard: output rows [n0, n1) of a PackedWeight."""
    n, k = q.shape
    if n % world or (_bits(q.format) == 4 and k % 2):
        raise ValueError('Column sharding requires N divisible by the world size and even K for 4-bit codes')
    rows = n // world
    n0 = rank * rows
    row_bytes = k * _bits(q.format) // 8
    gpr = k // q.group_size
    data = q.data[n0 * row_bytes:(n0 + rows) * row_bytes]
    scales = q.scales[2 * n0 * gpr:2 * (n0 + rows) * gpr]
    return PackedWeight((rows, k), q.format, q.group_size, data, scales)


def shard_packed_cols(q, rank, world):
    """Row-parallel shard: input columns [k0, k1) of a PackedWeight, on group boundaries."""
    n, k = q.shape
    cols = k // world
    per_row = q.group_size == k     # per-row INT8 scales stay whole
    if k % world or (not per_row and cols % q.group_size) or (_bits(q.format) == 4 and cols % 2):
        raise ValueError('Row sharding requires K/world to be a multiple of the group size (and even for 4-bit)')
    k0 = rank * cols
    bits = _bits(q.format)
    raw = np.frombuffer(q.data, dtype=np.uint8).reshape(n, k * bits // 8)
    data = raw[:, k0 * bits // 8:(k0 + cols) * bits // 8].tobytes()
    if per_row:
        return PackedWeight((n, cols), q.format, cols, data, q.scales), True
    sc = np.frombuffer(q.scales, dtype=np.uint16).reshape(n, k // q.group_size)
    g0, g1 = k0 // q.group_size, (k0 + cols) // q.group_size
    return PackedWeight((n, cols), q.format, q.group_size, data, sc[:, g0:g1].tobytes()), False


def shard_correction_rows(c, rank, world):
    """Column-parallel layer: V [r, K] replicated, U [N, r] split by output rows."""
    down, up = c.tensors()
    rows = up.shape[0] // world
    return LowRankCorrection((rows, down.shape[1]), c.rank, down.numpy().tobytes(),
                             up[rank * rows:(rank + 1) * rows].contiguous().numpy().tobytes())


def shard_correction_cols(c, rank, world):
    """Row-parallel layer: V split by input columns, U replicated.  The partial z of each
    rank is summed before delta = half(half(z) U^T)."""
    down, up = c.tensors()
    cols = down.shape[1] // world
    return down[:, rank * cols:(rank + 1) * cols].contiguous(), up


def shard_layer_weights(weights, packed, corrections, rank, world, config):
    """Per-rank weights for one layer: (fp16 weights dict, packed dict, corrections dict,
    row-parallel extras).  Heads are split whole: heads and kv heads divisible by world."""
    heads, kvh = config['num_attention_heads'], config.get('num_key_value_heads', config['num_attention_heads'])
    if heads % world or kvh % world:
        raise ValueError('Tensor parallelism requires heads and KV heads divisible by the world size')
    out_w, out_p, out_c, row_extra = {}, {}, {}, {}
    for name, w in weights.items():
        if w.ndim == 1:
            out_w[name] = w
        elif name in COLUMN:
            rows = w.shape[0] // world
            out_w[name] = w[rank * rows:(rank + 1) * rows]
        else:
            cols = w.shape[1] // world
            out_w[name] = w[:, rank * cols:(rank + 1) * cols]
    if packed is not None:
        for name, q in packed.items():
            if name in COLUMN:
                out_p[name] = shard_packed_rows(q, rank, world)
            else:
                out_p[name], _ = shard_packed_cols(q, rank, world)
    for name, c in (corrections or {}).items():
        if name in COLUMN:
            out_c[name] = shard_correction_rows(c, rank, world)
        else:
            row_extra[name] = shard_correction_cols(c, rank, world)
    return out_w, (out_p or None), out_c, row_extra


def tp_config(config, world):
    """Per-rank config: heads, kv heads and FFN width divided by the world size."""
    c = dict(config)
    c['head_dim'] = config.get('head_dim', config['hidden_size'] // config['num_attention_heads'])
    c['num_attention_heads'] = config['num_attention_heads'] // world
    c['num_key_value_heads'] = config.get('num_key_value_heads', config['num_attention_heads']) // world
    c['intermediate_size'] = config['intermediate_size'] // world
    c['tp_world'] = world
    return c


def packed_equal(a, b):
    return a.shape == b.shape and a.format == b.format and a.group_size == b.group_size and a.data == b.data and \
        a.scales == b.scales


def unsharded_elements(shards):
    return sum(prod(s.shape) for s in shards)


def build_tp_causal_lm(config, layer_weights, embedding, norm, *, mode='nf4a16', group_size=64, corrections=None,
                       rank=0, world=1, group=None, device=None, max_positions=None):
    """Per-rank tensor-parallel SmolForCausalLM: full weights in, this rank's shard built.

    Weights are quantized whole (GPU quantize_weight) and then sliced, so every rank's
    codes and scales are byte ranges of the single-GPU model's."""
    import torch_npu_smollm as sm
    from torch_npu_lowbit import quantize_weight
    fmt = sm._WEIGHT_FORMATS[mode]
    cfg_r = tp_config(config, world)
    layers = []
    for i, w in enumerate(layer_weights):
        packed = None
        if fmt is not None:
            packed = {name: quantize_weight(w[name].to(device or 'cuda'), format=fmt,
                                            group_size=None if fmt == 'int8' else group_size)
                      for name in sm._PROJECTIONS}
        corr = None if corrections is None else corrections[i]
        w_r, p_r, c_r, row_extra = shard_layer_weights(w, packed, corr, rank, world, config)
        layers.append(sm.FrozenSmolLayer({k: v for k, v in cfg_r.items() if k != 'tp_world'}, w_r, mode=mode,
                                         packed_weights=p_r, corrections=c_r or None, device=device,
                                         max_positions=max_positions, tp_group=group, row_corrections=row_extra))
    return sm.SmolForCausalLM(sm.FrozenSmolStack.from_layers(layers), embedding, norm)
