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
    launch_gemv_fused_z in csrc/gemv.cu, for the one-row kernel of csrc/gemv1.cu as for the
    general one; the sweep's grids always fit the device at once); otherwise the projection
    is a launch of its own.  The count follows the default settings: LOWBIT_G1_FUSE_MIN and
    LOWBIT_G1_ZSELF change which cells fuse their projection."""
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
    return {'kernel': 'gemv1_kernel<NF4, group 64> (8192x2048, M=1)', 'bound': 'hbm', 'achieved': round(achieved, 1),
            'peak': peak_gbs, 'unit': 'GB/s', 'frac': round(achieved / peak_gbs, 4), 'launch_us': round(t * 1e6, 3),
            'bytes_per_launch': per_launch,
            'traffic': TRAFFIC_PER_LAUNCH.get(DOMINANT),
            'traffic_source': 'ncu dram__bytes_read.sum + dram__bytes_write.sum per launch of bench.py --profile dominant'}


PREFILL_SHAPE = ('nf4', 64, 8192, 2048)   # the 1.7B gate/up projection
PREFILL_MS = (2048, 8192, 65536)           # configs[1]'s largest M, a mid batch, configs[4]'s 32 x 2048 tokens


def prefill_roofline(device, stream, peak_tf, m):
    """The prefill GEMM on the tensor cores: NF4 g64 8192x2048 with the rank-32 correction
    (tcgen05 path, z projection included), back to back in one graph over two weight
    replicas; achieved = FLOPs per call / duration vs the measured bf16 peak."""
    import lowbit_runtime as rt
    fmt, g, n, k = PREFILL_SHAPE
    gen = torch.Generator(device='cpu').manual_seed(2)
    reps = [rt.quantize_pack((torch.randn(n, k, generator=gen) * 0.02).half().to(device), fmt, g) for _ in range(2)]
    x = torch.randn(m, k, generator=gen).half().to(device)
    v = (torch.randn(RANK, k, generator=gen) * 1e-3).half().to(device)
    u = (torch.randn(n, RANK, generator=gen) * 1e-3).half().to(device)
    y = torch.empty(m, n, dtype=torch.float16, device=device)
    launches = 8 if m <= 8192 else 4
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
    flops = gemm_flops(m, n, k)
    achieved = flops / t / 1e12
    del graph, x, y, reps
    return {'kernel': f'tc_linear_kernel<NF4> (+ z projection), 8192x2048, group 64, M={m}, rank 32',
            'bound': 'tensor', 'achieved': round(achieved, 1), 'peak': peak_tf, 'unit': 'TFLOP/s',
            'frac': round(achieved / peak_tf, 4), 'launch_us': round(t * 1e6, 2), 'flops_per_call': flops}


# dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant kernel (mean of
# the captured launches), from an ncu capture of `bench.py --profile dominant`.
TRAFFIC_PER_LAUNCH = {DOMINANT: 8973824}


def cpu_reference_sweep(sample_cells, reps, cached=False):
    """The reference's CPU staging on a bounded sample: per call dequantize + fp32 linear +
    correction (torch_npu_smollm.py:150-164 via the oracle restatement); with ``cached``
    the dequantized weight is computed once and reused (torch_npu_lowbit_demo.py:65-71)."""
    from oracle import lowbit_ref as ref
    gen = torch.Generator().manual_seed(0)
    prepared = []
    for fmt, g, n, k in sample_cells:
        w = (torch.randn(n, k, generator=gen) * 0.02).half()
        u = (torch.randn(n, RANK, generator=gen) * 1e-3).half()
        v = (torch.randn(RANK, k, generator=gen) * 1e-3).half()
        group, data, scales = ref.quantize(w.numpy(), fmt, g)
        x = torch.randn(1, k, generator=gen).half()
        wp = ref.prepare_weight((n, k), fmt, group, data, scales) if cached else None
        prepared.append((fmt, group, n, k, data, scales, u, v, x, wp))
    total_bytes = 0
    t0 = time.perf_counter()
    for _ in range(reps):
        for fmt, group, n, k, data, scales, u, v, x, wp in prepared:
            if wp is None:
                ref.linear(x, (n, k), fmt, group, data, scales, down=v, up=u)
            else:
                ref.linear_prepared(x, wp, down=v, up=u)
            total_bytes += gemv_bytes(1, n, k, fmt, group)
    dt = time.perf_counter() - t0
    return total_bytes / dt / 1e9, dt


def cpu_decode_baseline(budget_s=8.0):
    """Decode on the host cores through the oracle restatement of reference_cpu
    (torch_npu_smollm.py:142-193, per-call dequantization) and FrozenSmolIO.logits.
    configs[2] runs whole (30 layers, batch 1, prompt 128, then greedy steps until
    ``budget_s``); configs[3] and [4] time one layer's decode step at their batch over a
    random KV cache of their prompt length plus the tied LM head, and extrapolate to all
    layers (configs[4]'s prefill: one layer over a 256-token prompt, scaled linearly to
    32 x 2048 tokens and 24 layers, which leaves out attention's quadratic part)."""
    import torch_npu_smollm as sm
    from oracle import decoder_ref as dref
    from oracle import lowbit_ref as ref
    out = {}

    def dims(name):
        c = SMOL[name]
        return dref.DecoderDims(hidden=c['hidden_size'], intermediate=c['intermediate_size'],
                                heads=c['num_attention_heads'], kv_heads=c['num_key_value_heads'],
                                vocab=c['vocab_size'], theta=c['rope_theta'])

    def layer(name, mode, group, seed):
        d = dims(name)
        gen = torch.Generator().manual_seed(seed)
        w, packed, corr = {}, {}, {}
        for pname, (sh, fmt, g) in projection_formats(name, mode, group).items():
            w[pname] = (torch.randn(sh, generator=gen) * 0.02).half()
            gg, data, scales = ref.quantize(w[pname].numpy(), fmt, None if fmt == 'int8' else g)
            packed[pname] = (sh, fmt, gg, data, scales)
            corr[pname] = ((torch.randn(RANK, sh[1], generator=gen) * 1e-3).half(),
                           (torch.randn(sh[0], RANK, generator=gen) * 1e-3).half())
        for nname in ('input_layernorm.weight', 'post_attention_layernorm.weight'):
            w[nname] = torch.ones(d.hidden, dtype=torch.float16)
        return dref.LayerRef(d, w, packed, corr)

    def head_time(name, batch):
        d = dims(name)
        emb = (torch.randn(d.vocab, d.hidden, generator=torch.Generator().manual_seed(1)) * 0.02).half()
        dec = dref.DecoderRef(d, [], emb, torch.ones(d.hidden, dtype=torch.float16), 8)
        h = torch.randn(batch, 1, d.hidden).half()
        t0 = time.perf_counter()
        dec.logits(h)
        return time.perf_counter() - t0

    # the whole 135M model, batch 1
    d = dims('135m')
    layers = [layer('135m', 'w8a16', None, 10 + i) for i in range(SMOL['135m']['num_hidden_layers'])]
    emb = (torch.randn(d.vocab, d.hidden, generator=torch.Generator().manual_seed(2)) * 0.02).half()
    model = dref.DecoderRef(d, layers, emb, torch.ones(d.hidden, dtype=torch.float16), 128 + 64)
    ids = torch.randint(0, d.vocab, (1, 128), generator=torch.Generator().manual_seed(3))
    t0 = time.perf_counter()
    hidden, caches = model.step(model.embed(ids), None)
    token = model.logits(hidden[:, -1:])[:, 0].float().argmax(-1)
    pre = time.perf_counter() - t0
    steps, t0 = 0, time.perf_counter()
    while steps < 64 and (steps < 2 or time.perf_counter() - t0 < budget_s):
        hidden, caches = model.step(model.embed(token[:, None]), caches)
        token = model.logits(hidden[:, -1:])[:, 0].float().argmax(-1)
        steps += 1
    dec = time.perf_counter() - t0
    out['smollm135m_w8_b1'] = {'tokens_per_s': round(steps / dec, 2), 'prefill_ms': round(pre * 1e3, 1),
                               'sample': f'whole model, prompt 128, {steps} greedy steps timed'}
    del layers, model, caches

    def one_layer_decode(name, mode, group, batch, prompt, tag):
        d = dims(name)
        lay = layer(name, mode, group, 20)
        gen = torch.Generator().manual_seed(4)
        cache = ((torch.randn(batch, d.kv_heads, prompt, d.head_dim, generator=gen) * 0.5).half(),
                 (torch.randn(batch, d.kv_heads, prompt, d.head_dim, generator=gen) * 0.5).half())
        cos, sin = dref.rope_tables(d, prompt + 4)
        x = torch.randn(batch, 1, d.hidden, generator=gen).half()
        lay.forward(x, cos, sin, cache)                    # warm-up
        t0 = time.perf_counter()
        for _ in range(2):
            lay.forward(x, cos, sin, cache)
        t_layer = (time.perf_counter() - t0) / 2
        n_layers = SMOL[name]['num_hidden_layers']
        step = n_layers * t_layer + head_time(name, batch)
        out[tag] = {'tokens_per_s': round(batch / step, 3), 'layer_step_ms': round(t_layer * 1e3, 1),
                    'sample': f'1 layer x 2 decode steps at batch {batch} over a {prompt}-position cache, '
                              f'extrapolated to {n_layers} layers + LM head'}
        return lay

    one_layer_decode('360m', 'w4a16', int4_groups(SMOL['360m']), 64, 512, 'smollm360m_int4_b64')
    one_layer_decode('360m', 'nf4a16', 64, 64, 512, 'smollm360m_nf4g64_b64')
    lay = one_layer_decode('1.7b', 'nf4a16', 64, 32, 2048, 'smollm1.7b_nf4g64_b32')
    d = dims('1.7b')
    cos, sin = dref.rope_tables(d, 260)
    x = torch.randn(1, 256, d.hidden, generator=torch.Generator().manual_seed(5)).half()
    t0 = time.perf_counter()
    lay.forward(x, cos, sin)
    t_pre = time.perf_counter() - t0
    total = t_pre * (32 * 2048 / 256) * SMOL['1.7b']['num_hidden_layers']
    out['smollm1.7b_nf4g64_b32']['prefill_ms_extrapolated'] = round(total * 1e3, 1)
    out['smollm1.7b_nf4g64_b32']['prefill_sample'] = '1 layer over a 256-token prompt, x 256 and x 24 layers'
    return out


def cpu_baseline_block(budget_s=12.0, decode=True):
    sample = CELLS
    # one untimed pass to size the sample, then enough passes for ~budget_s
    _, dt = cpu_reference_sweep(sample, 1)
    reps = max(1, int(budget_s / max(dt, 1e-3)))
    gbs, dt = cpu_reference_sweep(sample, reps)
    _, dtc = cpu_reference_sweep(sample, 1, cached=True)
    reps_c = max(1, int(budget_s / 2 / max(dtc, 1e-3)))
    gbs_c, dtc = cpu_reference_sweep(sample, reps_c, cached=True)
    out = {'value': round(gbs, 3), 'unit': 'GB/s', 'cores': torch.get_num_threads(), 'host_cpus': os.cpu_count(),
           'kind': 'port',
           'sample': f'{reps} pass(es) over all {len(sample)} sweep cells at M=1 with rank-32 correction, '
                     f'{dt:.1f} s of CPU work (oracle restatement of reference_cpu: dequantize + fp32 linear per call)',
           'cached_dequant': {'value': round(gbs_c, 3), 'unit': 'GB/s',
                              'sample': f'{reps_c} pass(es), dequantized weights computed once and reused '
                                        f'(torch_npu_lowbit_demo.py:65-71), {dtc:.1f} s'}}
    if decode:
        out['decode'] = cpu_decode_baseline()
    return out


def e2e_block(cells, steps, warmup, device, stream):
    """The sweep through the public module, QuantizedLinear.forward (torch_npu_lowbit.py:339
    in the reference), one module per cell and replica built from the packed bytes and
    its LowRankCorrection.  Every step copies that step's activations from pinned host
    memory to the device, runs every cell's forward, and copies all outputs back."""
    import torch_npu_lowbit as lb
    from torch_npu_lowbit_correction import LowRankCorrection
    modules = []
    for c in cells:
        corr = LowRankCorrection.from_tensors(c['v'].cpu(), c['u'].cpu())
        reps = []
        for codes, scales in c['reps']:
            pw = lb.PackedWeight((c['n'], c['k']), c['fmt'], c['g'], codes.cpu().numpy().tobytes(),
                                 scales.cpu().numpy().tobytes())
            reps.append(lb.QuantizedLinear(pw, correction=corr, device=device))
        modules.append(reps)
    xs = [c['x'].cpu() for c in cells]
    total_k = sum(x.numel() for x in xs)
    total_n = sum(c['n'] for c in cells)
    host_x = torch.cat([x.reshape(-1) for x in xs]).pin_memory()
    host_y = torch.empty(total_n, dtype=torch.float16).pin_memory()
    dev_x = torch.empty(total_k, dtype=torch.float16, device=device)
    dev_y = torch.empty(total_n, dtype=torch.float16, device=device)
    # each cell's activation / output rows are fixed views into the staging buffers (made once,
    # as a caller's preallocated buffers would be)
    views, a, b = [], 0, 0
    for c in cells:
        views.append((dev_x[a:a + c['k']].view(1, c['k']), dev_y[b:b + c['n']].view(1, c['n'])))
        a += c['k']
        b += c['n']

    def step(i):
        r = i % REPLICAS
        dev_x.copy_(host_x, non_blocking=True)
        for mods, (x, y) in zip(modules, views):
            mods[r](x, out=y)
        host_y.copy_(dev_y, non_blocking=True)

    with torch.cuda.stream(stream):
        for i in range(warmup):
            step(i)
        stream.synchronize()
        t = timed(step, steps, stream)
    total = sum(gemv_bytes(1, c['n'], c['k'], c['fmt'], c['g']) for c in cells) * steps
    del modules
    return {'value': round(total / t / 1e9, 1), 'unit': 'GB/s', 'h2d_bytes_per_step': total_k * 2,
            'd2h_bytes_per_step': total_n * 2, 'ms_per_step': round(t / steps * 1e3, 4),
            'api': 'QuantizedLinear.forward per cell (fp16 activations copied in, outputs copied out every step)'}


def gemm_flops(m, n, k, rank=RANK):
    return 2 * m * n * k + 2 * m * rank * (n + k)


def sweep_m_block(cells, device, stream, peak_gbs, peak_tf, ms=(16, 128, 2048), steps=10):
    """configs[1] at its other batch sizes: every legal cell with rank-32 correction at
    M = 16 (batched decode GEMV), 128 and 2048 (tcgen05 GEMM), each step a replayed graph
    over all 14 cells on one of the 4 weight replicas.  Per M: GB/s and TFLOP/s of the
    algorithmic bytes / FLOPs, and the fraction of the bound that applies (HBM while the
    step's FLOP per byte is below the measured ridge, tensor above it)."""
    import lowbit_runtime as rt
    out = {}
    gen = torch.Generator(device='cpu').manual_seed(5)
    for m in ms:
        xs = [torch.randn(m, c['k'], generator=gen).half().to(device) for c in cells]
        ys = [torch.empty(m, c['n'], dtype=torch.float16, device=device) for c in cells]
        graphs = []
        with torch.cuda.stream(stream):
            for c, x, y in zip(cells, xs, ys):
                for codes, scales in c['reps']:
                    rt.linear(x, c['fmt'], c['g'], c['n'], codes, scales, down=c['v'], up=c['u'], out=y)
            stream.synchronize()
            for r in range(REPLICAS):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for c, x, y in zip(cells, xs, ys):
                        codes, scales = c['reps'][r]
                        rt.linear(x, c['fmt'], c['g'], c['n'], codes, scales, down=c['v'], up=c['u'], out=y)
                graphs.append(g)
            for i in range(3):
                graphs[i % REPLICAS].replay()
            stream.synchronize()
            t = timed(lambda i: graphs[i % REPLICAS].replay(), steps, stream) / steps
        nbytes = sum(gemv_bytes(m, c['n'], c['k'], c['fmt'], c['g']) for c in cells)
        flops = sum(gemm_flops(m, c['n'], c['k']) for c in cells)
        gbs, tfs = nbytes / t / 1e9, flops / t / 1e12
        bound = 'hbm' if flops / nbytes < peak_tf * 1e12 / (peak_gbs * 1e9) else 'tensor'
        paths = sorted({rt.linear_select(c['fmt'], c['g'], m, c['n'], c['k'], RANK) for c in cells})
        out[f'm{m}'] = {'ms_per_step': round(t * 1e3, 4), 'GB_per_s': round(gbs, 1), 'TFLOP_per_s': round(tfs, 1),
                        'bound': bound, 'frac': round(gbs / peak_gbs if bound == 'hbm' else tfs / peak_tf, 4),
                        'bytes_per_step': nbytes, 'flops_per_step': flops, 'paths': paths}
        del graphs, xs, ys
    return out


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


def build_smollm(name, mode, group, device, max_positions, rank=0, world=1, pg=None, seed=0, layers=None):
    """Random-init SmolLM of the named architecture (std 0.02), rank-32 corrections on every
    projection, quantized on the GPU; tensor-parallel when world > 1 and pg is given.
    ``layers`` overrides the layer count (the dimensions stay the architecture's)."""
    import smollm_parallel as sp
    import torch_npu_smollm as sm
    from torch_npu_lowbit_correction import LowRankCorrection
    config = SMOL[name] if layers is None else dict(SMOL[name], num_hidden_layers=layers)
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
    return sm.SmolForCausalLM(sm.FrozenSmolStack.from_layers(layers), emb, norm)


def projection_formats(name, mode, group):
    """(format, group) of each of the 7 projections for a decode entry."""
    import torch_npu_smollm as sm
    fmt = sm._WEIGHT_FORMATS[mode]
    shapes = sm.SmolConfig.from_dict(SMOL[name]).shapes()
    out = {}
    for pname, sh in shapes.items():
        if len(sh) != 2:
            continue
        g = sh[1] if fmt == 'int8' else (group.get(pname) if isinstance(group, dict) else group)
        out[pname] = (sh, fmt, g)
    return out


def decode_step_bytes(name, mode, group, batch, positions, world=1, tp=False):
    """Algorithmic HBM bytes of one decode step of the whole job: per layer the 7
    projections' bytes_gemv (codes, scales, rank-32 factors, activations in and out), the
    KV cache read over ``positions`` attended positions (K and V, fp16), and the tied fp16
    LM head (2 vocab d + 2 B vocab).  Batch sharding: every rank reads the whole weights
    for its own sequences.  Tensor parallel: weights and KV are split, the LM head is read
    by every rank."""
    cfg = SMOL[name]
    layers, d, vocab = cfg['num_hidden_layers'], cfg['hidden_size'], cfg['vocab_size']
    kvh, hd = cfg['num_key_value_heads'], 64

    def one(b):
        proj = sum(gemv_bytes(b, sh[0], sh[1], fmt, g) for sh, fmt, g in projection_formats(name, mode, group).values())
        kv = 2 * 2 * kvh * hd * positions * b
        return layers * (proj + kv)

    head = 2 * vocab * d + 2 * batch * vocab
    if tp:
        return one(batch) + world * head
    import smollm_parallel as sp
    per = [b1 - b0 for b0, b1 in (sp.batch_shard(batch, r, world) for r in range(world))]
    return sum(one(b) + 2 * vocab * d + 2 * b * vocab for b in per)


def graph_kernel_nodes(graph):
    """Kernel nodes of a captured CUDA graph (cuda-python), or None when unavailable."""
    try:
        from cuda.bindings import runtime as cr
        g = cr.cudaGraph_t(init_value=graph.raw_cuda_graph())
        err, _, count = cr.cudaGraphGetNodes(g, 0)
        err, nodes, count = cr.cudaGraphGetNodes(g, count)
        kernels = 0
        for node in nodes:
            err, kind = cr.cudaGraphNodeGetType(node)
            if kind == cr.cudaGraphNodeType.cudaGraphNodeTypeKernel:
                kernels += 1
        return kernels
    except Exception:  # noqa: BLE001
        return None


def decode_entry(model, name, mode, group, batch, local_batch, prompt, steps, world, tp, pre, dec, peak_gbs, extra):
    """One decode line: tokens/s of the whole job (``batch`` sequences), algorithmic bytes
    per step, their rate and fraction of the HBM roofline of all GPUs, and the kernel
    launches of this rank's captured step graph (``local_batch`` sequences)."""
    positions = prompt + (steps + 1) / 2          # mean attended positions over the timed steps
    nbytes = decode_step_bytes(name, mode, group, batch, positions, world, tp)
    st = model.session(local_batch)
    launches = None
    if st.get('graph') is not None:
        launches = graph_kernel_nodes(st['graph'])
    elif st.get('piecewise') is not None:   # tensor parallel: graphs between the all-reduces
        counts = [graph_kernel_nodes(g) for g in st['piecewise'].graphs()]
        launches = None if None in counts else sum(counts)
    out = {'tokens_per_s': round(batch * steps / dec, 1), 'prefill_ms': round(pre * 1e3, 3),
           'ms_per_step': round(dec / steps * 1e3, 4), 'bytes_per_step': int(nbytes),
           'GB_per_s': round(nbytes * steps / dec / 1e9, 1),
           'frac_of_hbm': round(nbytes * steps / dec / 1e9 / (world * peak_gbs), 4),
           'launches_per_step': launches}
    out.update(extra)
    return out


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


def tp_parity_block(world, rank, device, pg, layers=2, batch=2, prompt=16, steps=16):
    """Tensor-parallel correctness on this run's GPUs: configs[4] layer dimensions (2048,
    32/32 heads, FFN 8192, NF4 g64, rank-32 corrections) with ``layers`` layers, greedy
    generation tensor-parallel over all ranks vs the same model on rank 0's GPU alone.

    ``rel_l2`` is the largest per-step logits error with the single-GPU model fed the
    tensor-parallel run's own tokens (teacher forcing), so both see the same inputs at every
    step.  ``same_tokens`` compares the two free-running greedy generations; tensor parallelism
    sums the o and down projections in another order, so at a near-tie (two logits a few fp16
    ulps apart, frequent among 49,152 random-weight logits) the greedy choices may part.  When
    they do, ``first_diff`` gives the step and the single-GPU model's gap between the two tokens."""
    ids = torch.randint(0, SMOL['1.7b']['vocab_size'], (batch, prompt),
                        generator=torch.Generator().manual_seed(3)).to(device)
    tp = build_smollm('1.7b', 'nf4a16', 64, device, prompt + steps + 8, rank=rank, world=world, pg=pg, seed=7,
                      layers=layers)
    tokens, logits = tp.generate(ids, steps, return_logits=True)
    result = None
    if rank == 0:
        single = build_smollm('1.7b', 'nf4a16', 64, device, prompt + steps + 8, seed=7, layers=layers)
        t1, _ = single.generate(ids, steps, return_logits=True)
        st = single.session(batch)
        forced = [single.prefill_session(ids).clone()]
        for t in range(1, steps):
            st['ids'].copy_(tokens[:, t - 1])
            forced.append(single.decode_step(batch, graph=False).clone())
        errs = [float((a.float() - b.float()).norm() / b.float().norm()) for a, b in zip(logits, forced)]
        result = {'rel_l2': round(max(errs), 6), 'same_tokens': bool(torch.equal(tokens, t1)), 'layers': layers,
                  'batch': batch, 'prompt': prompt, 'steps': steps, 'comparison': 'teacher-forced logits',
                  'config': f'configs[4] dims, NF4 g64 + rank-32, tensor-parallel x{world} vs 1 GPU'}
        diff = (tokens != t1).any(0).nonzero()
        if diff.numel():
            s = int(diff[0])
            row = int((tokens[:, s] != t1[:, s]).nonzero()[0])
            f = forced[s][row].float()
            result['first_diff'] = {'step': s, 'row': row,
                                    'single_gap': round(float(f[t1[row, s]] - f[tokens[row, s]]), 6),
                                    'logit_scale': round(float(f.abs().max()), 4)}
        del single
    del tp
    barrier(world)
    torch.cuda.empty_cache()
    return result


def decode_block(world, rank, device, pg, peak_gbs, quick=False):
    """Decode tokens/s for BASELINE configs 2 (135M W8, B=1, rank 0 only), 3 (360M INT4 /
    NF4, B=64 sharded over ranks, no collective) and 4 (1.7B NF4, B=32, tensor-parallel),
    each with its algorithmic bytes per step and the fraction of the HBM roofline."""
    import smollm_parallel as sp
    out = {}
    if rank == 0:
        m = build_smollm('135m', 'w8a16', None, device, 128 + 128 + 8)
        pre, dec = decode_run(m, 1, 128, 128, 1)
        out['smollm135m_w8_b1'] = decode_entry(
            m, '135m', 'w8a16', None, 1, 1, 128, 128, 1, False, pre, dec, peak_gbs,
            {'config': 'configs[2]: 30 layers, W8 + rank-32 on all 7 projections, prompt 128, 128 greedy steps, '
                       'batch 1, 1 GPU'})
        del m
    barrier(world)
    b0, b1 = sp.batch_shard(64, rank, world)
    steps = 64 if quick else 256
    for tag, mode, group in (('int4', 'w4a16', int4_groups(SMOL['360m'])), ('nf4g64', 'nf4a16', 64)):
        m = build_smollm('360m', mode, group, device, 512 + steps + 8, seed=0)
        pre, dec = decode_run(m, b1 - b0, 512, steps, world, seed=rank)
        out[f'smollm360m_{tag}_b64'] = decode_entry(
            m, '360m', mode, group, 64, b1 - b0, 512, steps, world, False, pre, dec, peak_gbs,
            {'config': f'configs[3]: 32 layers, {tag} + rank-32, batch 64 sharded over {world} GPU(s), prompt 512, '
                       f'{steps} greedy steps'})
        del m
    torch.cuda.empty_cache()
    steps = 32 if quick else 128
    m = build_smollm('1.7b', 'nf4a16', 64, device, 2048 + steps + 8, rank=rank, world=world, pg=pg)
    pre, dec = decode_run(m, 32, 2048, steps, world)
    prefill_tokens = 32 * 2048
    out['smollm1.7b_nf4g64_b32'] = decode_entry(
        m, '1.7b', 'nf4a16', 64, 32, 32, 2048, steps, world, True, pre, dec, peak_gbs,
        {'prefill_tokens_per_s': round(prefill_tokens / pre, 1),
         'config': f'configs[4]: 24 layers, NF4 g64 + rank-32, prefill 32x2048, {steps} greedy steps, '
                   f'{"tensor-parallel x" + str(world) if world > 1 else "1 GPU"}'})
    del m
    torch.cuda.empty_cache()
    if world > 1:
        out['tp_parity'] = tp_parity_block(world, rank, device, pg)
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
    """Small, self-contained workloads for ncu captures (committed, so that a capture runs
    committed files only); each holds a few GB on the device at most.
      dominant  -- the NF4 g64 8192x2048 decode GEMV (M=1) over 16 weight replicas (144 MB,
                   larger than L2), 48 launches;
      prefill   -- the same layer at M=2048 with the rank-32 correction on the tcgen05 path,
                   6 launches;
      batched   -- the same layer at M=64 with the correction (batched-decode GEMV), 12
                   launches over 4 replicas;
      attention -- one-token GQA attention of configs[4] at batch 32 (32 heads / 32 KV heads,
                   2176 cached positions, 570 MB of K/V), 4 launches;
      quantize  -- NF4 g64 quantize + pack of a 8192x2048 fp16 weight, 3 launches;
      decode    -- one greedy decode step of two configs[4] layers (+ head) at batch 32,
                   replayed 3 times;
      decode360 -- one greedy decode step of two configs[3] layers (INT4, group 128 / 64,
                   + head) at batch 64 over a 512-token prompt, replayed 3 times."""
    import lowbit_runtime as rt
    rt.require_cuda()
    fmt, g, n, k = DOMINANT
    gen = torch.Generator(device='cpu').manual_seed(3)
    info = {'profile_case': which}
    if which in ('dominant', 'prefill', 'batched'):
        reps = {'dominant': 16, 'prefill': 2, 'batched': 4}[which]
        packed = [rt.quantize_pack((torch.randn(n, k, generator=gen) * 0.02).half().cuda(), fmt, g) for _ in range(reps)]
        m = {'dominant': 1, 'prefill': 2048, 'batched': 64}[which]
        x = torch.randn(m, k, generator=gen).half().cuda()
        v = (torch.randn(RANK, k, generator=gen) * 1e-3).half().cuda()
        u = (torch.randn(n, RANK, generator=gen) * 1e-3).half().cuda()
        y = torch.empty(m, n, dtype=torch.float16, device='cuda')
        launches = {'dominant': 48, 'prefill': 6, 'batched': 12}[which]
        for i in range(launches):
            c, sc = packed[i % reps]
            if which == 'dominant':
                rt.linear(x, fmt, g, n, c, sc, out=y)
            else:
                rt.linear(x, fmt, g, n, c, sc, down=v, up=u, out=y)
        info.update(launches=launches, m=m, n=n, k=k, format=fmt, group=g)
    elif which == 'attention':
        b, heads, kvh, hd, max_pos = 32, 32, 32, 64, 2176
        L = rt.lib()
        q = torch.randn(b, heads * hd, generator=gen).half().cuda()
        kc = (torch.randn(b, kvh, max_pos, hd, generator=gen) * 0.5).half().cuda()
        vc = (torch.randn(b, kvh, max_pos, hd, generator=gen) * 0.5).half().cuda()
        lengths = torch.full((b,), max_pos - 1, dtype=torch.int32, device='cuda')
        out = torch.empty(b, heads * hd, dtype=torch.float16, device='cuda')
        ws = rt.Workspace.get(L.lb_attention_workspace_bytes(b, heads, max_pos))
        for _ in range(4):
            rt.check(L.lb_attention_decode(rt.ptr(q), heads * hd, rt.ptr(kc), rt.ptr(vc), rt.ptr(lengths), rt.ptr(out),
                                           b, heads, kvh, hd, max_pos, 0.125, rt.ptr(ws), ws.numel(), rt.stream_ptr()),
                     'lb_attention_decode')
        info.update(batch=b, heads=heads, kv_heads=kvh, positions=max_pos, kv_bytes=2 * b * kvh * max_pos * hd * 2)
    elif which == 'quantize':
        w = (torch.randn(n, k, generator=gen) * 0.02).half().cuda()
        for _ in range(3):
            rt.quantize_pack(w, fmt, g)
        info.update(n=n, k=k, format=fmt, group=g)
    elif which == 'decode360':
        m = build_smollm('360m', 'w4a16', int4_groups(SMOL['360m']), torch.device('cuda'), 512 + 16, layers=2)
        ids = torch.randint(0, m.config.vocab, (64, 512), generator=gen).cuda()
        m.prefill_session(ids)
        for _ in range(3):
            m.decode_step(64)
        info.update(layers=2, batch=64, prompt=512, launches_per_step=graph_kernel_nodes(m.session(64)['graph']))
    elif which == 'decode':
        m = build_smollm('1.7b', 'nf4a16', 64, torch.device('cuda'), 64 + 16, layers=2)
        ids = torch.randint(0, m.config.vocab, (32, 64), generator=gen).cuda()
        m.prefill_session(ids)
        for _ in range(3):
            m.decode_step(32)
        info.update(layers=2, batch=32, prompt=64, launches_per_step=graph_kernel_nodes(m.session(32)['graph']))
    else:
        raise ValueError(which)
    torch.cuda.synchronize()
    print(json.dumps(info), flush=True)
    return 0


def cells_report(steps=5):
    """Per-cell device time of the sweep (``--cells``): each cell alone, with and without its
    rank-32 correction, over enough weight replicas to stream ~300 MB per pass (> 2x L2),
    one graph of back-to-back lb_linear calls per case; then the sweep graph itself with and
    without the corrections.  CUDA events on the launching stream; one JSON line."""
    import lowbit_runtime as rt
    rt.require_cuda()
    device = torch.device('cuda')
    stream = torch.cuda.Stream()
    cells = make_cells(device)
    gen = torch.Generator(device='cpu').manual_seed(1)

    def graph_us(calls, per_replay):
        with torch.cuda.stream(stream):
            for f in calls:   # workspaces sized outside the capture
                f()
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for f in calls:
                    f()
            for _ in range(3):
                g.replay()
            t = timed(lambda i: g.replay(), steps, stream)
        return t / steps / per_replay * 1e6

    def call(c, codes, scales, corr):
        kw = dict(down=c['v'], up=c['u']) if corr else {}
        return lambda: rt.linear(c['x'], c['fmt'], c['g'], c['n'], codes, scales, out=c['y'], **kw)

    out = {'cells': {}}
    for c in cells:
        plain = gemv_bytes(1, c['n'], c['k'], c['fmt'], c['g'], 0)
        reps = min(512, -(-300_000_000 // plain))
        w = (torch.randn(c['n'], c['k'], generator=gen) * 0.02).half().to(device)
        packed = [rt.quantize_pack(w, c['fmt'], c['g']) for _ in range(reps)]
        row = {'replicas': reps}
        for corr in (True, False):
            us = graph_us([call(c, cs, sc, corr) for cs, sc in packed], reps)
            nbytes = gemv_bytes(1, c['n'], c['k'], c['fmt'], c['g'], RANK if corr else 0)
            row['corrected' if corr else 'plain'] = {'us': round(us, 2), 'GB_per_s': round(nbytes / us / 1e3, 1)}
        out['cells'][f"{c['fmt']} g{c['g']} {c['n']}x{c['k']}"] = row
        del packed, w
    for corr in (True, False):
        calls = [call(c, *c['reps'][r], corr) for r in range(REPLICAS) for c in cells]
        us = graph_us(calls, REPLICAS)
        nbytes = sum(gemv_bytes(1, c['n'], c['k'], c['fmt'], c['g'], RANK if corr else 0) for c in cells)
        out['sweep_corrected' if corr else 'sweep_plain'] = {'us': round(us, 2), 'GB_per_s': round(nbytes / us / 1e3, 1)}
    print(json.dumps(out), flush=True)
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
    ap.add_argument('--profile', choices=['dominant', 'prefill', 'batched', 'attention', 'quantize', 'decode',
                                          'decode360'],
                    help='run a small fixed workload for an ncu capture and exit')
    ap.add_argument('--cells', action='store_true',
                    help='print the per-cell device time of the sweep, with and without corrections, and exit')
    args = ap.parse_args()
    if args.profile:
        return profile_case(args.profile)
    if args.cells:
        return cells_report()
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
    sweep_m = sweep_m_block(cells, device, stream, peak_gbs, peak_tf)
    pre_roofs = {}
    for m in PREFILL_MS:
        pre_roofs[f'm{m}'] = prefill_roofline(device, stream, peak_tf, m)
        pre_roofs[f'm{m}']['peak_kind'] = f'{peak_kind} bf16 dense GEMM (burst)'
        torch.cuda.empty_cache()
    del graphs, cells
    torch.cuda.empty_cache()
    decode = None
    if not args.no_decode:
        pg = None
        if world > 1:
            import torch.distributed as dist
            pg = dist.group.WORLD
        try:
            decode = decode_block(world, rank, device, pg, peak_gbs, quick=args.quick_decode)
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
            'e2e': e2e, 'roofline': roof, 'prefill_roofline': pre_roofs, 'sweep_m': sweep_m, 'clocks': clocks.summary(),
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
