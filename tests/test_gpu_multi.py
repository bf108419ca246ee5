"""Tensor-parallel SmolLM decode on 2 GPUs (NCCL) against the single-GPU model.

Needs two CUDA devices; skipped otherwise.  NVLS is disabled for the test's NCCL
communicator, and every rank takes the same collective steps in the same order.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CONFIG = dict(model_type='llama', hidden_size=256, intermediate_size=512, num_attention_heads=4,
              num_key_value_heads=2, hidden_act='silu', rms_norm_eps=1e-5, rope_theta=10000.0, vocab_size=1024,
              num_hidden_layers=2, tie_word_embeddings=True)


def _port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _corrections(config, seed):
    import torch_npu_smollm as sm
    from torch_npu_lowbit_correction import LowRankCorrection
    shapes = sm.SmolConfig.from_dict(config).shapes()
    gen = torch.Generator().manual_seed(seed)
    return [{n: LowRankCorrection.from_tensors((torch.randn(32, s[1], generator=gen) * 1e-3).half(),
                                               (torch.randn(s[0], 32, generator=gen) * 1e-3).half())
             for n, s in shapes.items() if len(s) == 2} for _ in range(config['num_hidden_layers'])]


SMOL1700_2L = dict(CONFIG, hidden_size=2048, intermediate_size=8192, num_attention_heads=32, num_key_value_heads=32,
                   vocab_size=49152, num_hidden_layers=2)


def _worker(rank, world, port, results, config=CONFIG, graph=False, steps=16):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / 'torch-intel-npu_b200')]
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
    import torch.distributed as dist
    import smollm_parallel as sp
    import torch_npu_smollm as sm
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device('cuda', rank))
    lw, emb, norm = sm.random_smollm_weights(config, seed=0)
    corr = _corrections(config, 1)
    ids = torch.randint(0, config['vocab_size'], (2, 12), generator=torch.Generator().manual_seed(2)).cuda()
    tp = sp.build_tp_causal_lm(config, lw, emb, norm, mode='nf4a16', group_size=64, corrections=corr, rank=rank,
                               world=world, group=dist.group.WORLD, max_positions=64)
    tokens, logits = tp.generate(ids, steps, graph=graph, return_logits=True)
    if rank == 0:
        single = sp.build_tp_causal_lm(config, lw, emb, norm, mode='nf4a16', group_size=64, corrections=corr,
                                       rank=0, world=1, group=None, max_positions=64)
        t1, l1 = single.generate(ids, steps, graph=graph, return_logits=True)
        errs = [float((a.float() - b.float()).norm() / b.float().norm()) for a, b in zip(logits, l1)]
        results['errs'] = errs
        results['err'] = max(errs)
        results['same_tokens'] = bool(torch.equal(tokens, t1))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs two GPUs')
@pytest.mark.parametrize('dims,graph', [('small', False), ('1.7b', False), ('small', True), ('1.7b', True)])
def test_tensor_parallel_decode_matches_single_gpu(dims, graph):
    """Tensor parallel x2 against the same model on one GPU, at small and configs[4] dims,
    eager and graphed.  A graphed tensor-parallel step is CUDA graphs split at the NCCL
    all-reduces, which run eagerly between them (the path the benchmark times); the
    single-GPU model it is compared with replays one graph per step."""
    manager = mp.Manager()
    results = manager.dict()
    config = CONFIG if dims == 'small' else SMOL1700_2L
    mp.spawn(_worker, args=(2, _port(), results, config, graph, 16 if dims == 'small' else 8), nprocs=2, join=True)
    assert results['err'] < 5e-3, results['errs']
    assert results['same_tokens']
