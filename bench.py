"""Benchmark of the B200 low-bit decode path (one JSON line on rank 0).

Workload (decode regime): one "step" is one pass of the
dequant-GEMV over every legal cell of the low-bit sweep at M=1 -- INT4 (symmetric,
the reference format) and NF4, group 64 and 128, shapes (N,K) in {(1536,576),
(576,1536), (8192,2048), (2048,8192)}, each with its rank-32 correction; group 128
with K=576 is not representable in the reference format and is skipped (14 cells).
Weights ~ N(0, 0.02^2), U/V ~ N(0, 1e-3^2), x ~ N(0,1) fp16, seeded.  Every cell has
4 weight replicas and step i uses replica i % 4, so consecutive steps stream
~320 MB of distinct weights (> 2x the 126 MB L2): the timed data comes from HBM.

* value      -- whole-job algorithmic bytes / device time (CUDA events, max over ranks),
                weights resident in HBM, each step a replayed CUDA graph of lb_linear calls.
* e2e        -- the same sweep through the public API (QuantizedLinear.forward) with the
                step's activations copied from pinned host memory and outputs copied back.
* roofline   -- the dominant kernel (NF4 g64 8192x2048 decode GEMV) timed alone in a
                graph of back-to-back launches: algorithmic bytes / launch, vs the measured
                HBM copy bandwidth.
* cpu_baseline -- the reference's CPU staging (dequantize + fp32 F.linear per call, the
                reference_cpu path) on a bounded sample of the same sweep.
``--impl reference`` times that CPU path alone on this config.
Multi-GPU: each rank runs the whole sweep on its own GPU (replicas, no collective).
"""
import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / 'torch-intel-npu_b200')):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

SHAPES = [(1536, 576), (576, 1536), (8192, 2048), (2048, 8192)]
CELLS = [(fmt, g, n, k) for (n, k) in SHAPES for fmt in ('int4', 'nf4') for g in (64, 128) if k % g == 0]
REPLICAS = 4
RANK = 32
DOMINANT = ('nf4', 64, 8192, 2048)


def gemv_bytes(m, n, k, fmt, g, rank=RANK):
    """Algorithmic HBM bytes of one call: codes + scales + U,V + x + y."""
    bits = 8 if fmt == 'int8' else 4
    return (n * k * bits) // 8 + 2 * n * (k // g) + 2 * rank * (n + k) + 2 * m * k + 2 * m * n


def load_peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.exists():
        d = json.loads(p.read_text())
        return float(d['hbm_gbs']), float(d['bf16_tflops']), 'measured'
    return 6650.0, 1590.0, 'fallback'


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = Path(os.environ.get('TMPDIR', '/tmp')) / f'lowbit_clocks_{os.getpid()}.csv'

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', '-i', str(self.index),
                 '--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,'
                 'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
                 'clocks_event_reasons.sw_power_cap', '--format=csv,noheader,nounits', '-lms', '100'],
                stdout=open(self.path, 'w'), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            self.proc.wait(timeout=5)

    def summary(self):
        if self.proc is None or not self.path.exists():
            return None
        sm, mx, reasons = [], None, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(',')]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for name, v in zip(names, f[3:7]):
                if v.lower() == 'active':
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return None
        sm.sort()
        return {'sm_mhz': sm[len(sm) // 2], 'sm_max_mhz': mx, 'samples': len(sm), 'reasons': sorted(reasons)}


def make_cells(device, seed=0):
    import lowbit_runtime as rt
    gen = torch.Generator(device='cpu').manual_seed(seed)
    cells = []
    for fmt, g, n, k in CELLS:
        reps = []
        for r in range(REPLICAS):
            w = (torch.randn(n, k, generator=gen) * 0.02).half().to(device)
            codes, scales = rt.quantize_pack(w, fmt, g)
            reps.append((codes, scales))
            del w
        u = (torch.randn(n, RANK, generator=gen) * 1e-3).half().to(device)
        v = (torch.randn(RANK, k, generator=gen) * 1e-3).half().to(device)
        x = torch.randn(1, k, generator=gen).half().to(device)
        y = torch.empty(1, n, dtype=torch.float16, device=device)
        cells.append(dict(fmt=fmt, g=g, n=n, k=k, reps=reps, u=u, v=v, x=x, y=y))
    return cells


def capture_steps(cells, stream):
    """One CUDA graph per replica index: the whole sweep as lb_linear launches."""
    import lowbit_runtime as rt
    graphs = []
    with torch.cuda.stream(stream):
        for c in cells:   # warm the workspace / tensor maps outside capture
            for codes, scales in c['reps']:
                rt.linear(c['x'], c['fmt'], c['g'], c['n'], codes, scales, down=c['v'], up=c['u'], out=c['y'])
        stream.synchronize()
        for r in range(REPLICAS):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for c in cells:
                    codes, scales = c['reps'][r]
                    rt.linear(c['x'], c['fmt'], c['g'], c['n'], codes, scales, down=c['v'], up=c['u'], out=c['y'])
            graphs.append(g)
    return graphs


def launches_per_step(cells):
    """Kernel launches of one sweep step.  A corrected decode GEMV (M <= 16, rank <= 32)
    with >= 4 MiB of codes computes its z projection inside the same launch (the rule of
    launch_gemv_fused_z in csrc/gemv.cu; the sweep's grids always fit the device at once);
    otherwise the projection is a launch of its own."""
    import lowbit_runtime as rt
    count = 0
    for c in cells:
        path = rt.linear_select(c['fmt'], c['g'], 1, c['n'], c['k'], RANK)
        code_bytes = c['n'] * c['k'] * (8 if c['fmt'] == 'int8' else 4) // 8
        if path == 'gemv' and RANK <= 32 and code_bytes >= (4 << 20):
            count += 1
        else:
            count += 2 if path in ('gemv', 'generic') else 3   # z projection + linear (+ finalize)
    return count


def timed(fn, steps, stream):
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        fn(i)
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) * 1e-3


def dominant_kernel_roofline(device, stream, peak_gbs):
    """Time the NF4 g64 8192x2048 decode GEMV alone: 64 back-to-back launches over 32
    replicas (300 MB) in one graph; achieved = algorithmic bytes per launch / duration."""
    import lowbit_runtime as rt
    fmt, g, n, k = DOMINANT
    gen = torch.Generator(device='cpu').manual_seed(1)
    reps = []
    for _ in range(32):
        w = (torch.randn(n, k, generator=gen) * 0.02).half().to(device)
        reps.append(rt.quantize_pack(w, fmt, g))
    x = torch.randn(1, k, generator=gen).half().to(device)
    y = torch.empty(1, n, dtype=torch.float16, device=device)
    launches = 64
    with torch.cuda.stream(stream):
        for c, s in reps:
            rt.linear(x, fmt, g, n, c, s, out=y)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(launches):
                c, s = reps[i % len(reps)]
                rt.linear(x, fmt, g, n, c, s, out=y)
        for _ in range(3):
            graph.replay()
        stream.synchronize()
        t = timed(lambda i: graph.replay(), 10, stream) / (10 * launches)
    per_launch = gemv_bytes(1, n, k, fmt, g, rank=0)
    achieved = per_launch / t / 1e9
    return {'kernel': 'gemv_kernel<NF4> (8192x2048, group 64, M=1)', 'bound': 'hbm', 'achieved': round(achieved, 1),
            'peak': peak_gbs, 'unit': 'GB/s', 'frac': round(achieved / peak_gbs, 4), 'launch_us': round(t * 1e6, 3),
            'bytes_per_launch': per_launch,
            'traffic': TRAFFIC_PER_LAUNCH.get(DOMINANT)}


PREFILL = ('nf4', 64, 8192, 2048, 8192)   # the 1.7B gate/up shape at a prefill batch of 8192 tokens


def prefill_roofline(device, stream, peak_tf):
    """The prefill GEMM on the tensor cores: NF4 g64 8192x2048 with the rank-32 correction
    at M=8192 (tcgen05 path, z projection included), back to back in one graph over two
    weight replicas; achieved = FLOPs per call / duration vs the measured bf16 peak."""
    import lowbit_runtime as rt
    fmt, g, n, k, m = PREFILL
    gen = torch.Generator(device='cpu').manual_seed(2)
    reps = [rt.quantize_pack((torch.randn(n, k, generator=gen) * 0.02).half().to(device), fmt, g) for _ in range(2)]
    x = torch.randn(m, k, generator=gen).half().to(device)
    v = (torch.randn(RANK, k, generator=gen) * 1e-3).half().to(device)
    u = (torch.randn(n, RANK, generator=gen) * 1e-3).half().to(device)
    y = torch.empty(m, n, dtype=torch.float16, device=device)
    launches = 8
    with torch.cuda.stream(stream):
        for c, sc in reps:
            rt.linear(x, fmt, g, n, c, sc, down=v, up=u, out=y)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(launches):
                c, sc = reps[i % 2]
                rt.linear(x, fmt, g, n, c, sc, down=v, up=u, out=y)
        for _ in range(2):
            graph.replay()
        stream.synchronize()
        t = timed(lambda i: graph.replay(), 3, stream) / (3 * launches)
    flops = 2 * m * n * k + 2 * m * RANK * (n + k)
    achieved = flops / t / 1e12
    return {'kernel': 'tc_linear_kernel<NF4, 256> (+ z projection), 8192x2048, group 64, M=8192, rank 32',
            'bound': 'tensor', 'achieved': round(achieved, 1), 'peak': peak_tf, 'unit': 'TFLOP/s',
            'frac': round(achieved / peak_tf, 4), 'launch_us': round(t * 1e6, 2), 'flops_per_call': flops,
            'tensor_pipe_active': 'profiles/tc_linear_nf4_g64_m2048_8192x2048.md'}


# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant kernel (mean of
# the two captured launches), from the committed ncu capture
# (profiles/gemv_nf4_g64_8192x2048_m1.md).
TRAFFIC_PER_LAUNCH = {DOMINANT: 8983552}


def cpu_reference_sweep(sample_cells, reps):
    """The reference's CPU staging on a bounded sample: per call dequantize + fp32 linear +
    correction (torch_npu_smollm.py:150-164 via the oracle restatement)."""
    from oracle import lowbit_ref as ref
    gen = torch.Generator().manual_seed(0)
    prepared = []
    for fmt, g, n, k in sample_cells:
        w = (torch.randn(n, k, generator=gen) * 0.02).half()
        u = (torch.randn(n, RANK, generator=gen) * 1e-3).half()
        v = (torch.randn(RANK, k, generator=gen) * 1e-3).half()
        group, data, scales = ref.quantize(w.numpy(), fmt, g)
        x = torch.randn(1, k, generator=gen).half()
        prepared.append((fmt, group, n, k, data, scales, u, v, x))
    total_bytes = 0
    t0 = time.perf_counter()
    for _ in range(reps):
        for fmt, group, n, k, data, scales, u, v, x in prepared:
            ref.linear(x, (n, k), fmt, group, data, scales, down=v, up=u)
            total_bytes += gemv_bytes(1, n, k, fmt, group)
    dt = time.perf_counter() - t0
    return total_bytes / dt / 1e9, dt


def cpu_baseline_block(budget_s=12.0):
    sample = CELLS
    # one untimed pass to size the sample, then enough passes for ~budget_s
    _, dt = cpu_reference_sweep(sample, 1)
    reps = max(1, int(budget_s / max(dt, 1e-3)))
    gbs, dt = cpu_reference_sweep(sample, reps)
    return {'value': round(gbs, 3), 'unit': 'GB/s', 'cores': torch.get_num_threads(), 'kind': 'port',
            'sample': f'{reps} pass(es) over all {len(sample)} sweep cells at M=1 with rank-32 correction, '
                      f'{dt:.1f} s of CPU work (oracle restatement of reference_cpu: dequantize + fp32 linear per call)'}


def e2e_block(cells, steps, warmup, device, stream):
    """Public API path: QuantizedLinear-equivalent calls with host activations in, host outputs out."""
    import torch_npu_lowbit as lb  # noqa: F401  (public module; rt.linear is QuantizedLinear.forward's call)
    import lowbit_runtime as rt
    xs = [c['x'].cpu() for c in cells]
    total_k = sum(x.numel() for x in xs)
    total_n = sum(c['n'] for c in cells)
    host_x = torch.cat([x.reshape(-1) for x in xs]).pin_memory()
    host_y = torch.empty(total_n, dtype=torch.float16).pin_memory()
    dev_x = torch.empty(total_k, dtype=torch.float16, device=device)
    dev_y = torch.empty(total_n, dtype=torch.float16, device=device)
    # each cell's activation / output rows are fixed views into the staging buffers (made once,
    # as a caller's preallocated buffers would be); every step copies the host activations in
    # and the outputs back out
    views, a, b = [], 0, 0
    for c in cells:
        views.append((dev_x[a:a + c['k']].view(1, c['k']), dev_y[b:b + c['n']].view(1, c['n'])))
        a += c['k']
        b += c['n']

    def step(i):
        r = i % REPLICAS
        dev_x.copy_(host_x, non_blocking=True)
        for c, (x, y) in zip(cells, views):
            codes, scales = c['reps'][r]
            rt.linear(x, c['fmt'], c['g'], c['n'], codes, scales, down=c['v'], up=c['u'], out=y)
        host_y.copy_(dev_y, non_blocking=True)

    with torch.cuda.stream(stream):
        for i in range(warmup):
            step(i)
        stream.synchronize()
        t = timed(step, steps, stream)
    total = sum(gemv_bytes(1, c['n'], c['k'], c['fmt'], c['g']) for c in cells) * steps
    return {'value': round(total / t / 1e9, 1), 'unit': 'GB/s', 'h2d_bytes_per_step': total_k * 2,
            'd2h_bytes_per_step': total_n * 2, 'ms_per_step': round(t / steps * 1e3, 4)}


# ---- SmolLM decode (BASELINE configs[2..4]) ----------------------------------------------
SMOL = {
    '135m': dict(model_type='llama', hidden_size=576, intermediate_size=1536, num_attention_heads=9,
                 num_key_value_heads=3, rms_norm_eps=1e-5, rope_theta=10000.0, vocab_size=49152, num_hidden_layers=30),
    '360m': dict(model_type='llama', hidden_size=960, intermediate_size=2560, num_attention_heads=15,
                 num_key_value_heads=5, rms_norm_eps=1e-5, rope_theta=10000.0, vocab_size=49152, num_hidden_layers=32),
    '1.7b': dict(model_type='llama', hidden_size=2048, intermediate_size=8192, num_attention_heads=32,
                 num_key_value_heads=32, rms_norm_eps=1e-5, rope_theta=10000.0, vocab_size=49152, num_hidden_layers=24),
}


def int4_groups(config):
    """INT4 group 128 where K divides by 128, else 64 (K=960 is not a multiple of 128)."""
    import torch_npu_smollm as sm
    return {n: (128 if s[1] % 128 == 0 else 64) for n, s in sm.SmolConfig.from_dict(config).shapes().items() if len(s) == 2}


def build_smollm(name, mode, group, device, max_positions, rank=0, world=1, pg=None, seed=0):
    """Random-init SmolLM of the named architecture (std 0.02), rank-32 corrections on every
    projection, quantized on the GPU; tensor-parallel when world > 1 and pg is given."""
    import smollm_parallel as sp
    import torch_npu_smollm as sm
    from torch_npu_lowbit_correction import LowRankCorrection
    config = SMOL[name]
    layers_w, emb, norm = sm.random_smollm_weights(config, seed=seed, device=device)
    shapes = sm.SmolConfig.from_dict(config).shapes()
    gen = torch.Generator(device=device).manual_seed(seed + 1)
    corrections = [{n: LowRankCorrection.from_tensors((torch.randn(RANK, s[1], generator=gen, device=device) * 1e-3).half(),
                                                      (torch.randn(s[0], RANK, generator=gen, device=device) * 1e-3).half())
                    for n, s in shapes.items() if len(s) == 2} for _ in layers_w]
    if pg is not None and world > 1:
        return sp.build_tp_causal_lm(config, layers_w, emb, norm, mode=mode, group_size=group, corrections=corrections,
                                     rank=rank, world=world, group=pg, device=device, max_positions=max_positions)
    layers = [sm.FrozenSmolLayer(config, w, mode=mode, group_size=group, corrections=c, device=device,
                                 max_positions=max_positions) for w, c in zip(layers_w, corrections)]
    return sm.SmolForCausalLM(sm.FrozenSmolStack(layers), emb, norm)


def decode_run(model, batch, prompt, steps, world, seed=0):
    """Prefill a seeded prompt, then time ``steps`` graph-replayed greedy decode steps."""
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=model.device).manual_seed(seed)
    ids = torch.randint(0, model.config.vocab, (batch, prompt), generator=gen, device=model.device)
    model.prefill_session(ids)
    for _ in range(3):
        model.decode_step(batch)                 # captures the decode graph once
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    barrier(world)
    e[0].record(stream)
    model.prefill_session(ids)
    e[1].record(stream)
    for _ in range(steps):
        model.decode_step(batch)
    e[2].record(stream)
    e[2].synchronize()
    pre = max_over_ranks(e[0].elapsed_time(e[1]) * 1e-3, world)
    dec = max_over_ranks(e[1].elapsed_time(e[2]) * 1e-3, world)
    return pre, dec


def decode_block(world, rank, device, pg, quick=False):
    """Decode tokens/s for BASELINE configs 2 (135M W8, B=1, rank 0 only), 3 (360M INT4 /
    NF4, B=64 sharded over ranks, no collective) and 4 (1.7B NF4, B=32, tensor-parallel)."""
    import smollm_parallel as sp
    out = {}
    if rank == 0:
        m = build_smollm('135m', 'w8a16', None, device, 128 + 128 + 8)
        pre, dec = decode_run(m, 1, 128, 128, 1)
        out['smollm135m_w8_b1'] = {'tokens_per_s': round(128 / dec, 1), 'prefill_ms': round(pre * 1e3, 3),
                                   'config': 'configs[2]: 30 layers, W8 + rank-32 on all 7 projections, prompt 128, '
                                             '128 greedy steps, batch 1, 1 GPU'}
        del m
    barrier(world)
    b0, b1 = sp.batch_shard(64, rank, world)
    steps = 64 if quick else 256
    for tag, mode, group in (('int4', 'w4a16', int4_groups(SMOL['360m'])), ('nf4g64', 'nf4a16', 64)):
        m = build_smollm('360m', mode, group, device, 512 + steps + 8, seed=0)
        pre, dec = decode_run(m, b1 - b0, 512, steps, world, seed=rank)
        out[f'smollm360m_{tag}_b64'] = {'tokens_per_s': round(64 * steps / dec, 1), 'prefill_ms': round(pre * 1e3, 3),
                                        'config': f'configs[3]: 32 layers, {tag} + rank-32, batch 64 sharded over '
                                                  f'{world} GPU(s), prompt 512, {steps} greedy steps'}
        del m
    torch.cuda.empty_cache()
    steps = 32 if quick else 128
    m = build_smollm('1.7b', 'nf4a16', 64, device, 2048 + steps + 8, rank=rank, world=world, pg=pg)
    pre, dec = decode_run(m, 32, 2048, steps, world)
    prefill_tokens = 32 * 2048
    out['smollm1.7b_nf4g64_b32'] = {'tokens_per_s': round(32 * steps / dec, 1), 'prefill_ms': round(pre * 1e3, 3),
                                    'prefill_tokens_per_s': round(prefill_tokens / pre, 1),
                                    'config': f'configs[4]: 24 layers, NF4 g64 + rank-32, prefill 32x2048, {steps} '
                                              f'greedy steps, {"tensor-parallel x" + str(world) if world > 1 else "1 GPU"}'}
    del m
    torch.cuda.empty_cache()
    return out


def dist_setup():
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device('cuda', local))
    return world, rank, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def config_block(world):
    return {'workload': 'lowbit-gemv-sweep: BASELINE configs[1] decode (M=1), INT4/NF4 x group 64/128 x '
                        '(1536,576),(576,1536),(8192,2048),(2048,8192), rank-32 correction, 14 cells',
            'm': 1, 'cells': len(CELLS), 'replicas': REPLICAS, 'rank': RANK,
            'l2': 'inputs larger than L2: 4 rotating weight replicas (~320 MB) per cell set',
            'parallelism': f'replicas x{world} (batch-sharded, no collective)'}


def run_reference(args):
    """CPU reference path on this config: each step is one sweep cell (round robin over the
    14 cells), the reference's staging -- dequantize + fp32 linear + rank-32 correction."""
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    from oracle import lowbit_ref as ref
    gen = torch.Generator().manual_seed(0)
    prepared = []
    for fmt, g, n, k in CELLS:
        w = (torch.randn(n, k, generator=gen) * 0.02).half()
        u = (torch.randn(n, RANK, generator=gen) * 1e-3).half()
        v = (torch.randn(RANK, k, generator=gen) * 1e-3).half()
        group, data, scales = ref.quantize(w.numpy(), fmt, g)
        prepared.append((fmt, group, n, k, data, scales, u, v, torch.randn(1, k, generator=gen).half()))
    total_bytes, dt = 0, 0.0
    for i in range(args.warmup + args.steps):
        fmt, group, n, k, data, scales, u, v, x = prepared[i % len(prepared)]
        t0 = time.perf_counter()
        ref.linear(x, (n, k), fmt, group, data, scales, down=v, up=u)
        if i >= args.warmup:
            dt += time.perf_counter() - t0
            total_bytes += gemv_bytes(1, n, k, fmt, group)
    value = total_bytes / dt / 1e9
    cpu = {'value': round(value, 3), 'unit': 'GB/s', 'cores': torch.get_num_threads(), 'kind': 'port',
           'sample': f'{args.steps} calls round-robin over the {len(CELLS)} sweep cells at M=1 (oracle restatement of '
                     'reference_cpu: dequantize + fp32 linear + rank-32 correction per call)'}
    line = {'impl': 'reference', 'metric': 'dequant-GEMV HBM GB/s (decode sweep, M=1)', 'value': round(value, 3),
            'unit': 'GB/s', 'n_gpus': args.gpus, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': round(dt / args.steps * 1e3, 3), 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'u8 codes, fp16 io, fp32 accumulate', 'data': 'synthetic (seeded, BASELINE shapes)',
            'config': config_block(world), 'cpu_baseline': cpu,
            'e2e': {'value': round(value, 3), 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)
    return 0


def profile_case(which):
    """Small, self-contained workloads for ncu captures (committed so that the profile
    commands in profiles/ run committed files only).  dominant: the NF4 g64 8192x2048
    decode GEMV (M=1) over 16 weight replicas (144 MB, larger than L2), 48 launches;
    prefill: the same layer at M=2048 with the rank-32 correction on the tensor-core
    path, 6 launches."""
    import lowbit_runtime as rt
    rt.require_cuda()
    fmt, g, n, k = DOMINANT
    gen = torch.Generator(device='cpu').manual_seed(3)
    reps = 16 if which == 'dominant' else 2
    packed = [rt.quantize_pack((torch.randn(n, k, generator=gen) * 0.02).half().cuda(), fmt, g) for _ in range(reps)]
    m = 1 if which == 'dominant' else 2048
    x = torch.randn(m, k, generator=gen).half().cuda()
    v = (torch.randn(RANK, k, generator=gen) * 1e-3).half().cuda()
    u = (torch.randn(n, RANK, generator=gen) * 1e-3).half().cuda()
    y = torch.empty(m, n, dtype=torch.float16, device='cuda')
    launches = 48 if which == 'dominant' else 6
    for i in range(launches):
        c, sc = packed[i % reps]
        if which == 'dominant':
            rt.linear(x, fmt, g, n, c, sc, out=y)
        else:
            rt.linear(x, fmt, g, n, c, sc, down=v, up=u, out=y)
    torch.cuda.synchronize()
    print(json.dumps({'profile_case': which, 'launches': launches, 'm': m, 'n': n, 'k': k, 'format': fmt,
                      'group': g, 'checksum': float(y.float().abs().sum())}), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=200)
    ap.add_argument('--warmup', type=int, default=10)
    ap.add_argument('--impl', default='lowbit', choices=['lowbit', 'reference'])
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-decode', action='store_true')
    ap.add_argument('--quick-decode', action='store_true')
    ap.add_argument('--profile', choices=['dominant', 'prefill'],
                    help='run a small fixed workload for an ncu capture and exit')
    args = ap.parse_args()
    if args.profile:
        return profile_case(args.profile)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == 'reference':
        return run_reference(args)

    world, rank, local = dist_setup()
    import lowbit_runtime as rt
    rt.require_cuda()
    device = torch.device('cuda', local)
    torch.cuda.set_device(device)
    peak_gbs, peak_tf, peak_kind = load_peaks()
    stream = torch.cuda.Stream(device)
    cells = make_cells(device, seed=rank)
    graphs = capture_steps(cells, stream)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            graphs[i % REPLICAS].replay()
        stream.synchronize()
    barrier(world)
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            t = timed(lambda i: graphs[i % REPLICAS].replay(), args.steps, stream)
            torch.cuda.synchronize()
    barrier(world)
    t = max_over_ranks(t, world)
    per_step = sum(gemv_bytes(1, c['n'], c['k'], c['fmt'], c['g']) for c in cells)
    value = per_step * args.steps * world / t / 1e9
    launches_per_step_count = launches_per_step(cells)
    e2e = e2e_block(cells, max(10, args.steps // 4), 3, device, stream)
    e2e_v = max_over_ranks(1.0 / max(e2e['value'], 1e-9), world)
    e2e['value'] = round(world / e2e_v, 1) if world > 1 else e2e['value']
    roof = dominant_kernel_roofline(device, stream, peak_gbs)
    roof['peak_kind'] = f'{peak_kind} HBM copy bandwidth (burst)'
    pre_roof = prefill_roofline(device, stream, peak_tf)
    pre_roof['peak_kind'] = f'{peak_kind} bf16 dense GEMM (burst)'
    del graphs, cells
    torch.cuda.empty_cache()
    decode = None
    if not args.no_decode:
        pg = None
        if world > 1:
            import torch.distributed as dist
            pg = dist.group.WORLD
        try:
            decode = decode_block(world, rank, device, pg, quick=args.quick_decode)
        except Exception as exc:  # noqa: BLE001  (report, keep the GEMV line)
            decode = {'error': f'{type(exc).__name__}: {exc}'[:300]}
    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0
    line = {'metric': 'dequant-GEMV HBM GB/s (decode sweep, M=1)', 'value': round(value, 1), 'unit': 'GB/s',
            'n_gpus': world, 'steps': args.steps, 'warmup': args.warmup,
            'ms_per_step': round(t / args.steps * 1e3, 4), 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'u8 codes, fp16 io, fp32 accumulate', 'data': 'synthetic (seeded, BASELINE shapes)',
            'config': config_block(world),
            'frac_of_hbm_peak': round(value / world / peak_gbs, 4),
            'e2e': e2e, 'roofline': roof, 'prefill_roofline': pre_roof, 'clocks': clocks.summary(),
            'gpu_launches': launches_per_step_count * args.steps}
    if decode is not None:
        line['decode'] = decode
    if not args.no_cpu_baseline:
        line['cpu_baseline'] = cpu_baseline_block()
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == '__main__':
    sys.exit(main())
