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


def _worker(rank, world, port, results):
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
    lw, emb, norm = sm.random_smollm_weights(CONFIG, seed=0)
    corr = _corrections(CONFIG, 1)
    ids = torch.randint(0, 1024, (2, 12), generator=torch.Generator().manual_seed(2)).cuda()
    tp = sp.build_tp_causal_lm(CONFIG, lw, emb, norm, mode='nf4a16', group_size=64, corrections=corr, rank=rank,
                               world=world, group=dist.group.WORLD, max_positions=64)
    tokens, logits = tp.generate(ids, 16, graph=False, return_logits=True)
    if rank == 0:
        single = sp.build_tp_causal_lm(CONFIG, lw, emb, norm, mode='nf4a16', group_size=64, corrections=corr,
                                       rank=0, world=1, group=None, max_positions=64)
        t1, l1 = single.generate(ids, 16, graph=False, return_logits=True)
        err = max(float((a.float() - b.float()).norm() / b.float().norm()) for a, b in zip(logits, l1))
        results['err'] = err
        results['same_tokens'] = bool(torch.equal(tokens, t1))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs two GPUs')
def test_tensor_parallel_decode_matches_single_gpu():
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_worker, args=(2, _port(), results), nprocs=2, join=True)
    assert results['err'] < 5e-3
    assert results['same_tokens']
