"""Multi-rank logic on CPU (gloo, world size 2): tensor-parallel shards of packed weights,
scales and correction factors recombine to the unsharded oracle result; batch shards
cover every sequence once; a rank that fails is detected by its peer."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import lowbit_ref as ref


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import datetime
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _tp_worker(rank, world, port, fmt, group, results):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / 'torch-intel-npu_b200')]
    import smollm_parallel as sp
    from torch_npu_lowbit import PackedWeight
    from torch_npu_lowbit_correction import LowRankCorrection
    _init(rank, world, port)
    gen = torch.Generator().manual_seed(3)
    n, k, m = 64, 256, 3
    w = (torch.randn(n, k, generator=gen) * 0.05).half()
    down = (torch.randn(32, k, generator=gen) * 1e-2).half()
    up = (torch.randn(n, 32, generator=gen) * 1e-2).half()
    x = torch.randn(m, k, generator=gen).half()
    g, data, scales = ref.quantize(w.numpy(), fmt, group)
    q = PackedWeight((n, k), fmt, g, data, scales)
    corr = LowRankCorrection((n, k), 32, down.numpy().tobytes(), up.numpy().tobytes())
    full = ref.linear(x, (n, k), fmt, g, data, scales, down=down, up=up).float()
    # column parallel: local rows, replicated V, U shard -> concatenate
    qc = sp.shard_packed_rows(q, rank, world)
    cc = sp.shard_correction_rows(corr, rank, world)
    d, u = cc.tensors()
    part = ref.linear(x, qc.shape, qc.format, qc.group_size, qc.data, qc.scales, down=d, up=u)
    gathered = [torch.empty_like(part) for _ in range(world)]
    dist.all_gather(gathered, part)
    col = torch.cat(gathered, 1).float()
    # row parallel: local K slice, fp32 partials + partial z summed by one all-reduce
    qr, _ = sp.shard_packed_cols(q, rank, world)
    vr, ur = sp.shard_correction_cols(corr, rank, world)
    cols = k // world
    xr = x[:, rank * cols:(rank + 1) * cols]
    if qr.format == 'int8' and qr.group_size == qr.shape[1]:
        wr = np.frombuffer(qr.data, np.int8).reshape(qr.shape).astype(np.float64) * \
            np.frombuffer(qr.scales, np.float16).astype(np.float64)[:, None]
        y = xr.double() @ torch.from_numpy(wr).t()
    else:
        y = xr.double() @ torch.from_numpy(ref.dequantize(qr.shape, qr.format, qr.group_size, qr.data, qr.scales)).double().t()
    z = xr.float() @ vr.float().t()
    buf = torch.cat([y.float().reshape(-1), z.reshape(-1)])
    dist.all_reduce(buf)
    y = buf[:m * n].view(m, n).half()
    z = buf[m * n:].view(m, 32).half()
    delta = (z.float() @ ur.float().t()).half()
    row = (y + delta).half().float()
    results[rank] = (float((col - full).abs().max() / full.abs().max()),
                     float((row - full).abs().max() / full.abs().max()))
    dist.destroy_process_group()


@pytest.mark.parametrize('fmt,group', [('nf4', 64), ('int4', 32), ('int8', None), ('int8', 64)])
def test_tensor_parallel_shards_recombine(fmt, group):
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_tp_worker, args=(world, _free_port(), fmt, group, results), nprocs=world, join=True)
    for rank in range(world):
        col_err, row_err = results[rank]
        assert col_err == 0.0          # column shards are exact slices of the same staging
        assert row_err < 1e-2          # partial-sum order and the z all-reduce only


def test_shards_are_byte_slices_of_the_reference_packing():
    import smollm_parallel as sp
    from torch_npu_lowbit import PackedWeight
    w = (torch.randn(8, 256) * 0.05).float()
    g, data, scales = ref.quantize(w.numpy(), 'nf4', 64)
    q = PackedWeight((8, 256), 'nf4', g, data, scales)
    rows = [sp.shard_packed_rows(q, r, 4) for r in range(4)]
    assert b''.join(s.data for s in rows) == q.data and b''.join(s.scales for s in rows) == q.scales
    cols = [sp.shard_packed_cols(q, r, 2)[0] for r in range(2)]
    for r, c in enumerate(cols):
        gg, dd, ss = ref.quantize(w[:, r * 128:(r + 1) * 128].numpy(), 'nf4', 64)
        assert c.data == dd and c.scales == ss      # a column shard is the quantization of the slice
    with pytest.raises(ValueError):
        sp.shard_packed_cols(q, 0, 8)               # 32 columns would split a group of 64


def test_batch_shards_cover_every_sequence_once():
    import smollm_parallel as sp
    for batch in (1, 7, 64):
        for world in (1, 2, 4, 8):
            spans = [sp.batch_shard(batch, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(e - s for s, e in spans) - min(e - s for s, e in spans) <= 1


@pytest.mark.parametrize('world', [2, 4, 8])
def test_configs4_layer_shards_at_every_scaling_world_size(world):
    """configs[4] (SmolLM-1.7B: hidden 2048, 32 / 32 heads, FFN 8192, NF4 group 64) runs tensor
    parallel at every world size of the benchmark's scaling run.  Its per-rank config keeps
    whole 64-wide heads; every column-parallel projection (real N, a short K) splits into
    row-byte ranges that concatenate to the whole packing; every row-parallel projection (real
    K, a few rows) splits on group boundaries, each shard of the rank's local K."""
    import smollm_parallel as sp
    import torch_npu_smollm as sm
    from torch_npu_lowbit import PackedWeight
    config = dict(model_type='llama', hidden_size=2048, intermediate_size=8192, num_attention_heads=32,
                  num_key_value_heads=32, rms_norm_eps=1e-5, rope_theta=10000.0, vocab_size=49152,
                  num_hidden_layers=24)
    local = sm.SmolConfig.from_dict({k: v for k, v in sp.tp_config(config, world).items() if k != 'tp_world'})
    assert (local.heads * world, local.kv_heads * world, local.intermediate * world, local.head_dim) == (32, 32, 8192, 64)
    full_shapes, local_shapes = sm.SmolConfig.from_dict(config).shapes(), local.shapes()
    gen = torch.Generator().manual_seed(5)
    for name, shape in full_shapes.items():
        if len(shape) != 2:
            continue
        n, k = shape
        if name in sp.COLUMN:
            w = (torch.randn(n, 64, generator=gen) * 0.02).numpy()
            g, data, scales = ref.quantize(w, 'nf4', 64)
            q = PackedWeight((n, 64), 'nf4', g, data, scales)
            shards = [sp.shard_packed_rows(q, r, world) for r in range(world)]
            assert all(s.shape == (local_shapes[name][0], 64) for s in shards), name
            assert b''.join(s.data for s in shards) == q.data and b''.join(s.scales for s in shards) == q.scales
        else:
            w = (torch.randn(4, k, generator=gen) * 0.02).numpy()
            g, data, scales = ref.quantize(w, 'nf4', 64)
            q = PackedWeight((4, k), 'nf4', g, data, scales)
            shards = [sp.shard_packed_cols(q, r, world)[0] for r in range(world)]
            assert all(s.shape == (4, local_shapes[name][1]) for s in shards), name
            rows = [np.frombuffer(s.data, np.uint8).reshape(4, -1) for s in shards]
            assert np.concatenate(rows, 1).tobytes() == q.data


def _fail_worker(rank, world, port, results):
    _init(rank, world, port, timeout_s=5)
    t = torch.ones(4)
    dist.all_reduce(t)                # step 1: both ranks healthy
    if rank == 1:
        os._exit(0)                   # rank 1 leaves between steps, nothing in flight
    try:
        dist.all_reduce(t)            # step 2: the peer is gone
        results[rank] = 'no error'
    except Exception as e:            # noqa: BLE001  (gloo raises RuntimeError / DistBackendError)
        results[rank] = type(e).__name__
    os._exit(0)


def test_peer_failure_is_detected_on_the_host():
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    ctx = mp.get_context('spawn')
    port = _free_port()
    procs = [ctx.Process(target=_fail_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    assert results.get(0) not in (None, 'no error')
