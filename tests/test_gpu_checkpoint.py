"""Loading a SmolLM checkpoint directory and a packed checkpoint on the GPU.

* FrozenSmolStack(directory, ...) / SmolForCausalLM.from_checkpoint with packed weights
  read straight to the device (torch_npu_lowbit_checkpoint.load_packed) generates exactly
  what the model built in memory from the same packed bytes generates;
* FrozenSmolIO on the device: embed_tokens is the table gather, logits within 0.5%
  relative L2 of the reference staging (torch_npu_smollm_io.py:52-61, restated in the
  oracle).
"""
import json

import pytest
import torch

from oracle import decoder_ref as dref
from oracle import lowbit_ref as ref

pytestmark = pytest.mark.gpu
CONFIG = dict(model_type='llama', hidden_size=192, intermediate_size=512, num_attention_heads=3, num_key_value_heads=1,
              hidden_act='silu', rms_norm_eps=1e-5, rope_theta=10000.0, vocab_size=1024, num_hidden_layers=3,
              tie_word_embeddings=True)


def _write_checkpoint(path, seed=0):
    from safetensors.torch import save_file
    import torch_npu_smollm as sm
    layers, emb, norm = sm.random_smollm_weights(CONFIG, seed=seed)
    tensors = {'model.embed_tokens.weight': emb, 'model.norm.weight': norm}
    for i, w in enumerate(layers):
        for name, t in w.items():
            tensors[f'model.layers.{i}.{name}'] = t.contiguous()
    save_file(tensors, str(path / 'model.safetensors'))
    (path / 'config.json').write_text(json.dumps(CONFIG))
    return layers, emb, norm


def _packed_model(layers, fmt, group, seed):
    import torch_npu_lowbit as lb
    import torch_npu_smollm as sm
    from torch_npu_lowbit_correction import LowRankCorrection
    gen = torch.Generator().manual_seed(seed)
    packed, corr = {}, {}
    for i, w in enumerate(layers):
        packed[i], corr[i] = {}, {}
        for name in sm._PROJECTIONS:
            n, k = w[name].shape
            g, data, scales = ref.quantize(w[name].numpy(), fmt, group)
            packed[i][name] = lb.PackedWeight((n, k), fmt, g, data, scales)
            corr[i][name] = LowRankCorrection.from_tensors((torch.randn(32, k, generator=gen) * 1e-3).half(),
                                                           (torch.randn(n, 32, generator=gen) * 1e-3).half())
    return packed, corr


def test_checkpoint_directory_and_packed_file_generate_like_the_in_memory_model(tmp_path):
    import torch_npu_lowbit as lb
    import torch_npu_lowbit_checkpoint as ck
    import torch_npu_smollm as sm
    layers, emb, norm = _write_checkpoint(tmp_path)
    packed, corr = _packed_model(layers, 'nf4', 64, seed=5)
    ck.save_packed(tmp_path / 'packed.safetensors', packed, corr)
    dev_packed, dev_corr = ck.load_packed(tmp_path / 'packed.safetensors', device='cuda')
    q = dev_packed[0]['mlp.gate_proj.weight']
    assert isinstance(q, lb.DevicePackedWeight) and q.codes.is_cuda
    assert q.codes.cpu().numpy().tobytes() == packed[0]['mlp.gate_proj.weight'].data
    loaded = sm.SmolForCausalLM.from_checkpoint(tmp_path, mode='nf4a16', packed_weights=dev_packed,
                                                corrections=dev_corr, max_positions=64)
    assert loaded.stack.num_layers == 3 and loaded.stack.start_layer == 0
    built = sm.SmolForCausalLM.from_weights(CONFIG, layers, emb, norm, mode='nf4a16', max_positions=64)
    built = sm.SmolForCausalLM(sm.FrozenSmolStack.from_layers(
        [sm.FrozenSmolLayer(CONFIG, w, mode='nf4a16', packed_weights=packed[i], corrections=corr[i], max_positions=64)
         for i, w in enumerate(layers)]), emb, norm)
    ids = torch.randint(0, 1024, (2, 8), generator=torch.Generator().manual_seed(1)).cuda()
    a, la = loaded.generate(ids, 12, return_logits=True)
    b, lb_ = built.generate(ids, 12, return_logits=True)
    assert torch.equal(a, b)
    assert all(torch.equal(x, y) for x, y in zip(la, lb_))
    # a sub-range of the checkpoint, as the reference's FrozenSmolStack(start_layer=...)
    part = sm.FrozenSmolStack(tmp_path, start_layer=1, num_layers=2, mode='nf4a16',
                              packed_weights={i: dev_packed[i] for i in (1, 2)},
                              corrections={i: dev_corr[i] for i in (1, 2)}, max_positions=64)
    assert part.start_layer == 1 and part.num_layers == 2
    single = sm.FrozenSmolLayer.from_checkpoint(tmp_path, layer_index=2, mode='nf4a16', packed_weights=dev_packed[2],
                                                corrections=dev_corr[2], max_positions=64)
    x = (torch.randn(1, 4, 192, generator=torch.Generator().manual_seed(2)) * 0.5).half().cuda()
    assert torch.equal(single(x), part.layers[1](x))
    with pytest.raises(NotImplementedError):
        single.reference_cpu(x.cpu())


def test_io_endpoints_follow_the_reference_staging(tmp_path):
    import torch_npu_smollm_io as sio
    _, emb, norm = _write_checkpoint(tmp_path, seed=3)
    io = sio.FrozenSmolIO.from_checkpoint(tmp_path)
    ids = torch.randint(0, 1024, (2, 5), generator=torch.Generator().manual_seed(4))
    x = io.embed_tokens(ids)
    assert torch.equal(x.cpu(), torch.nn.functional.embedding(ids, emb.half()))
    hidden = (torch.randn(2, 5, 192, generator=torch.Generator().manual_seed(5))).half()
    oracle = dref.DecoderRef(dref.DecoderDims(hidden=192, intermediate=512, heads=3, kv_heads=1, vocab=1024), [],
                             emb, norm, 8)
    got, expected = io.logits(hidden.cuda()).float().cpu(), oracle.logits(hidden).float()
    assert float((got - expected).norm() / expected.norm()) < 5e-3
    with pytest.raises(ValueError):
        io.logits(hidden.cuda().float())
    with pytest.raises(ValueError):
        io.embed_tokens(ids.int())
    with pytest.raises(ValueError):
        sio.FrozenSmolIO(dict(CONFIG, tie_word_embeddings=False), emb, norm)
