"""Packed on-disk format and checkpoint-directory validation, without a GPU."""
import json

import numpy as np
import pytest
import torch

from oracle import lowbit_ref as ref

PROJ = ('self_attn.q_proj.weight', 'mlp.down_proj.weight')


def _packed(seed):
    from torch_npu_lowbit import PackedWeight
    from torch_npu_lowbit_correction import LowRankCorrection
    gen = torch.Generator().manual_seed(seed)
    packed, corr = {}, {}
    for layer in (3, 4):
        packed[layer], corr[layer] = {}, {}
        for name, (n, k), fmt, g in ((PROJ[0], (64, 128), 'nf4', 64), (PROJ[1], (128, 96), 'int8', 96)):
            w = (torch.randn(n, k, generator=gen) * 0.02).half()
            group, data, scales = ref.quantize(w.numpy(), fmt, g)
            packed[layer][name] = PackedWeight((n, k), fmt, group, data, scales)
            corr[layer][name] = LowRankCorrection.from_tensors((torch.randn(8, k, generator=gen) * 1e-3).half(),
                                                               (torch.randn(n, 8, generator=gen) * 1e-3).half())
    return packed, corr


def test_packed_checkpoint_round_trip(tmp_path):
    """save_packed / load_packed keep every byte: codes, scales, shapes, formats, groups
    and the correction factors, keyed by checkpoint layer."""
    import torch_npu_lowbit_checkpoint as ck
    packed, corr = _packed(1)
    path = tmp_path / 'packed.safetensors'
    ck.save_packed(path, packed, corr)
    got, got_corr = ck.load_packed(path)
    assert set(got) == {3, 4} and set(got_corr) == {3, 4}
    for layer in packed:
        for name, q in packed[layer].items():
            g = got[layer][name]
            assert (g.shape, g.format, g.group_size, g.data, g.scales) == (q.shape, q.format, q.group_size, q.data,
                                                                          q.scales)
            assert got_corr[layer][name] == corr[layer][name]


def test_packed_checkpoint_rejects_foreign_files(tmp_path):
    from safetensors.torch import save_file
    import torch_npu_lowbit_checkpoint as ck
    path = tmp_path / 'plain.safetensors'
    save_file({'x': torch.zeros(4)}, str(path))
    with pytest.raises(ValueError):
        ck.load_packed(path)
    with pytest.raises(ValueError):
        ck.save_packed(tmp_path / 'bad.safetensors', {})


def test_packed_checkpoint_validates_like_packed_weight(tmp_path):
    """A file whose scales are not positive is rejected by the same PackedWeight checks."""
    from safetensors.torch import save_file
    import torch_npu_lowbit_checkpoint as ck
    meta = {'lowbit_packed': ck.VERSION,
            'model.layers.0.mlp.up_proj.weight': json.dumps({'shape': [2, 64], 'format': 'int4', 'group_size': 64})}
    t = {'model.layers.0.mlp.up_proj.weight.codes': torch.zeros(64, dtype=torch.uint8),
         'model.layers.0.mlp.up_proj.weight.scales': torch.tensor([1.0, -1.0], dtype=torch.float16)}
    save_file(t, str(tmp_path / 'neg.safetensors'), metadata=meta)
    with pytest.raises(ValueError, match='Scales'):
        ck.load_packed(tmp_path / 'neg.safetensors')


def test_stack_checks_the_layer_range_before_loading(tmp_path):
    """FrozenSmolStack(directory, ...) validates its range and maps as the reference does
    (torch_npu_smollm.py:566-585) before any weight is read."""
    import torch_npu_smollm as sm
    (tmp_path / 'config.json').write_text(json.dumps({'num_hidden_layers': 4}))
    for kw in (dict(start_layer=3, num_layers=2), dict(start_layer=-1), dict(num_layers=0), dict(start_layer=1.0)):
        with pytest.raises(ValueError, match='contiguous'):
            sm.FrozenSmolStack(tmp_path, **kw)
    with pytest.raises(ValueError, match='indexed by checkpoint layer'):
        sm.FrozenSmolStack(tmp_path, start_layer=1, num_layers=2, mode='nf4a16', packed_weights={1: {}})
    with pytest.raises(ValueError, match='indexed by checkpoint layer'):
        sm.FrozenSmolStack(tmp_path, start_layer=0, num_layers=1, mode='nf4a16', corrections={1: {}})
    with pytest.raises(ValueError):
        sm.FrozenSmolStack(tmp_path, mode='int3')
