"""GPU parity of the low-bit path against the CPU oracle (which is pinned to the reference).

* quantize/pack and dequantize: bit-exact.
* linear (GEMV / tcgen05 GEMM / generic kernels, with bias and rank-r correction):
  max |y - y_ref| / max |y_ref| <= 1e-2 (the north-star fp16 tolerance), and the mean
  relative error must stay at fp16-rounding level (<= 2e-3).
"""
import hashlib

import numpy as np
import pytest
import torch

from oracle import lowbit_ref as ref

pytestmark = pytest.mark.gpu
TOL_MAX = 1e-2
TOL_MEAN = 2e-3


@pytest.fixture(scope='module')
def rt():
    import lowbit_runtime
    lowbit_runtime.require_cuda()
    return lowbit_runtime


def sha(b):
    return hashlib.sha256(b).hexdigest()


def _quant_cases(z):
    for key in z.files:
        if key.endswith('/data'):
            wname, case, _ = key.split('/')
            fmt, g = case.split('_g')
            yield wname, fmt, int(g)


def test_quantize_bit_exact_on_reference_fixtures(rt, golden):
    z = golden('quantize.npz')
    n_cases = 0
    for wname, fmt, g in _quant_cases(z):
        w = torch.from_numpy(z[f'{wname}/w']).cuda()
        codes, scales = rt.quantize_pack(w, fmt, g)
        key = f'{wname}/{fmt}_g{g}'
        assert codes.cpu().numpy().tobytes() == z[key + '/data'].tobytes(), key
        assert scales.cpu().numpy().tobytes() == z[key + '/scales'].tobytes(), key
        n, k = w.shape
        deq = rt.dequantize(fmt, g, n, k, codes, scales)
        assert sha(deq.cpu().numpy().tobytes()) == str(z[key + '/deq_sha']), key
        n_cases += 1
    assert n_cases == 162


def baseline_weight(n, k, seed=0):
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=gen) * 0.02).half()
    u = (torch.randn(n, 32, generator=gen) * 1e-3).half()
    v = (torch.randn(32, k, generator=gen) * 1e-3).half()
    return w, u, v


@pytest.mark.parametrize('shape', [(1536, 576), (576, 1536), (8192, 2048), (2048, 8192)])
def test_quantize_baseline_shapes_match_reference_digests(rt, golden, shape):
    z = golden('baseline_digests.npz')
    n, k = shape
    w, _, _ = baseline_weight(n, k)
    for fmt, g in (('int8', k), ('int4', 64), ('int4', 128), ('nf4', 64), ('nf4', 128)):
        if k % g:
            continue
        codes, scales = rt.quantize_pack(w.cuda(), fmt, g)
        key = f'{n}x{k}/{fmt}_g{g}'
        assert sha(codes.cpu().numpy().tobytes()) == str(z[key + '/data_sha']), key
        assert sha(scales.cpu().numpy().tobytes()) == str(z[key + '/scales_sha']), key
        deq = rt.dequantize(fmt, g, n, k, codes, scales)
        assert sha(deq.cpu().numpy().tobytes()) == str(z[key + '/deq_sha']), key


def test_quantize_errors_match_reference(rt):
    with pytest.raises(ValueError, match='Nonfinite'):
        rt.quantize_pack(torch.full((2, 16), float('nan'), device='cuda'), 'int4', 16)
    with pytest.raises(ValueError, match='Nonfinite'):
        rt.quantize_pack(torch.tensor([[1.0, float('inf')] * 8], device='cuda'), 'nf4', 16)
    with pytest.raises(ValueError, match='overflows'):
        rt.quantize_pack(torch.full((1, 8), 3e38, device='cuda'), 'int8', 8)


def _compare(y, expected, label):
    y = y.float().cpu()
    e = expected.float()
    assert torch.isfinite(y).all(), label
    denom = e.abs().max().clamp_min(1e-6)
    err = (y - e).abs()
    assert float(err.max() / denom) <= TOL_MAX, (label, float(err.max() / denom))
    assert float(err.mean() / e.abs().mean().clamp_min(1e-6)) <= TOL_MEAN, (label, float(err.mean()))


def _oracle(x, w_shape, fmt, g, data, scales, down=None, up=None, bias=None):
    return ref.linear(x.cpu(), w_shape, fmt, g, data, scales, down=down, up=up, bias=bias)


CASES = [
    # (n, k, fmt, group)
    (1536, 576, 'int8', 576), (1536, 576, 'int4', 64), (1536, 576, 'nf4', 64),
    (576, 1536, 'int4', 128), (576, 1536, 'nf4', 128), (576, 1536, 'int8', 1536),
    (8192, 2048, 'nf4', 64), (8192, 2048, 'int4', 128), (2048, 8192, 'nf4', 128), (2048, 8192, 'int4', 64),
    (192, 576, 'nf4', 32), (320, 960, 'int4', 64), (960, 2560, 'nf4', 64), (2048, 2048, 'int8', 2048),
    (576, 576, 'int8', 64),
]


@pytest.mark.parametrize('n,k,fmt,g', CASES)
@pytest.mark.parametrize('m', [1, 2, 3, 4, 16, 24, 40, 64, 100, 256])
def test_linear_matches_oracle_with_correction(rt, n, k, fmt, g, m):
    w, u, v = baseline_weight(n, k, seed=n + k)
    group, data, scales = ref.quantize(w.numpy(), fmt, g)
    gen = torch.Generator().manual_seed(7 + m)
    x = torch.randn(m, k, generator=gen).half()
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    expected = _oracle(x, (n, k), fmt, group, data, scales, down=v, up=u)
    y = rt.linear(x.cuda(), fmt, group, n, codes, sc, down=v.cuda(), up=u.cuda())
    _compare(y, expected, (n, k, fmt, g, m, rt.linear_select(fmt, group, m, n, k, 32)))


@pytest.mark.parametrize('path', ['gemv', 'tc', 'generic'])
@pytest.mark.parametrize('fmt,g', [('int4', 64), ('nf4', 128), ('int8', 2048), ('int8', 64)])
def test_every_path_agrees(rt, path, fmt, g):
    n, k = 2048, 2048
    m = 4 if path == 'gemv' else 48
    w, u, v = baseline_weight(n, k, seed=3)
    group, data, scales = ref.quantize(w.numpy(), fmt, g)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(1)).half()
    bias = (torch.randn(n, generator=torch.Generator().manual_seed(2)) * 0.1).half()
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    expected = _oracle(x, (n, k), fmt, group, data, scales, down=v, up=u, bias=bias)
    y = rt.linear(x.cuda(), fmt, group, n, codes, sc, down=v.cuda(), up=u.cuda(), bias=bias.cuda(), path=path)
    _compare(y, expected, (path, fmt, g))


@pytest.mark.parametrize('m', [1, 64, 2048])
def test_fp16_weights_path(rt, m):
    n, k = 1024, 576
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(5)) * 0.02).half()
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(6)).half()
    expected = torch.nn.functional.linear(x.float(), w.float()).half()
    y = rt.linear(x.cuda(), 'fp16', k, n, w.cuda().view(torch.uint8).reshape(-1), None)
    _compare(y, expected, ('fp16', m))


@pytest.mark.parametrize('n,k,fmt,g,rank', [(3, 17, 'int4', 17, 2), (5, 9, 'nf4', 3, 4), (7, 64, 'int8', 32, 7),
                                            (33, 96, 'nf4', 32, 16), (130, 640, 'int4', 64, 8)])
def test_ragged_shapes_and_ranks(rt, n, k, fmt, g, rank):
    w = (torch.randn(n, k, generator=torch.Generator().manual_seed(n)) * 0.05).float()
    group, data, scales = ref.quantize(w.numpy(), fmt, g)
    v = (torch.randn(rank, k, generator=torch.Generator().manual_seed(9)) * 1e-2).half()
    u = (torch.randn(n, rank, generator=torch.Generator().manual_seed(10)) * 1e-2).half()
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    for m in (1, 5, 33):
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(m)).half()
        expected = _oracle(x, (n, k), fmt, group, data, scales, down=v, up=u)
        y = rt.linear(x.cuda(), fmt, group, n, codes, sc, down=v.cuda(), up=u.cuda())
        _compare(y, expected, (n, k, fmt, g, rank, m))


@pytest.mark.parametrize('plan', ['1,1,1', '2,4,1', '8,2,1', '8,1,4', '4,2,2', '1,4,8'])
@pytest.mark.parametrize('fmt,g,m', [('nf4', 64, 1), ('int4', 128, 5), ('int8', 2048, 16), ('int8', 64, 3),
                                     ('nf4', 128, 37), ('int4', 64, 64)])
def test_gemv_work_splits_agree(rt, monkeypatch, plan, fmt, g, m):
    """Every GEMV work split (warps over K, rows per warp, cross-CTA K splits with the
    workspace reduction) gives the same parity; cross-CTA splits are deterministic."""
    monkeypatch.setenv('LOWBIT_GEMV_PLAN', plan)
    n, k = 2048, 2048
    w, u, v = baseline_weight(n, k, seed=21)
    group, data, scales = ref.quantize(w.numpy(), fmt, g)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(22)).half()
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    expected = _oracle(x, (n, k), fmt, group, data, scales, down=v, up=u)
    y1 = rt.linear(x.cuda(), fmt, group, n, codes, sc, down=v.cuda(), up=u.cuda(), path='gemv')
    y2 = rt.linear(x.cuda(), fmt, group, n, codes, sc, down=v.cuda(), up=u.cuda(), path='gemv')
    _compare(y1, expected, (plan, fmt, g, m))
    assert torch.equal(y1, y2)


@pytest.mark.parametrize('fmt,g', [('nf4', 128), ('int4', 64)])
@pytest.mark.parametrize('m', [4096, 4133])
def test_prefill_batches_from_4096_rows_match_oracle(rt, fmt, g, m):
    """From 4096 activation rows the correction's projection runs with two m16 tiles per
    CTA (ragged M included); the tcgen05 result with correction matches the oracle."""
    n, k = 576, 1536
    w, u, v = baseline_weight(n, k, seed=41)
    group, data, scales = ref.quantize(w.numpy(), fmt, g)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(42)).half()
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    assert rt.linear_select(fmt, group, m, n, k, 32) == 'tc'
    expected = _oracle(x, (n, k), fmt, group, data, scales, down=v, up=u)
    y = rt.linear(x.cuda(), fmt, group, n, codes, sc, down=v.cuda(), up=u.cuda())
    _compare(y, expected, (fmt, g, m))


def test_large_prefill_shape_properties(rt):
    """Full BASELINE prefill size: deterministic, zero-in gives the correction-free zero,
    and a row sample matches the oracle."""
    n, k, m = 8192, 2048, 2048
    w, u, v = baseline_weight(n, k)
    codes, sc = rt.quantize_pack(w.cuda(), 'nf4', 64)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(11)).half().cuda()
    y1 = rt.linear(x, 'nf4', 64, n, codes, sc, down=v.cuda(), up=u.cuda())
    y2 = rt.linear(x, 'nf4', 64, n, codes, sc, down=v.cuda(), up=u.cuda())
    assert torch.equal(y1, y2)
    zero = rt.linear(torch.zeros_like(x), 'nf4', 64, n, codes, sc, down=v.cuda(), up=u.cuda())
    assert int(zero.abs().max().item()) == 0
    rows = torch.arange(0, m, 97)
    data, scales = codes.cpu().numpy().tobytes(), sc.cpu().numpy().tobytes()
    expected = _oracle(x[rows].cpu(), (n, k), 'nf4', 64, data, scales, down=v, up=u)
    _compare(y1[rows.cuda()], expected, 'prefill-sample')


def test_quantized_linear_module(rt):
    import torch_npu_lowbit as lb
    from torch_npu_lowbit_correction import LowRankCorrection
    lin = torch.nn.Linear(576, 1536, bias=True)
    with torch.no_grad():
        lin.weight.copy_(torch.randn(1536, 576) * 0.02)
        lin.bias.copy_(torch.randn(1536) * 0.1)
    _, u, v = baseline_weight(1536, 576)
    corr = LowRankCorrection((1536, 576), 32, v.numpy().tobytes(), u.numpy().tobytes())
    q = lb.QuantizedLinear.from_float(lin, format='int8', correction=corr)
    assert q.weight.format == 'int8' and q.weight.group_size == 576
    # the packed bytes equal the reference quantizer's
    g, data, scales = ref.quantize(lin.weight.detach().numpy(), 'int8')
    assert q.weight.data == data and q.weight.scales == scales
    np.testing.assert_array_equal(q.weight.dequantize(), ref.dequantize((1536, 576), 'int8', g, data, scales))
    x = torch.randn(3, 576).half()
    expected = ref.linear(x, (1536, 576), 'int8', g, data, scales, down=v, up=u, bias=lin.bias.detach().half())
    _compare(q(x.cuda()), expected, 'module')
    with pytest.raises(ValueError):
        q(x.cuda().float())
    with pytest.raises(ValueError):
        q(x.cuda()[:, :100])
    with pytest.raises(NotImplementedError):
        lb.QuantizedLinear(q.weight, compact_groups=True)


@pytest.mark.parametrize('fmt,g', [('nf4', 64), ('int4', 32), ('int8', 576)])
@pytest.mark.parametrize('m', [1, 5, 64])
def test_stacked_linear_matches_separate_projections(rt, fmt, g, m):
    """lb_linear_stacked over q/k/v-shaped rows with their three rank-32 corrections as one
    block-diagonal rank-96 correction, and the fused residual add: every output row matches
    the oracle of its own projection, staged as the reference stages it."""
    k = 576
    widths = (576, 192, 192)
    gen = torch.Generator().manual_seed(31 + m)
    parts = []
    for n in widths:
        w = (torch.randn(n, k, generator=gen) * 0.02).half()
        v = (torch.randn(32, k, generator=gen) * 1e-3).half()
        u = (torch.randn(n, 32, generator=gen) * 1e-3).half()
        group, data, scales = ref.quantize(w.numpy(), fmt, g)
        parts.append((n, group, data, scales, v, u))
    x = torch.randn(m, k, generator=gen).half()
    ntot = sum(widths)
    codes = torch.frombuffer(bytearray(b''.join(p[2] for p in parts)), dtype=torch.uint8).cuda()
    scales = torch.frombuffer(bytearray(b''.join(p[3] for p in parts)), dtype=torch.float16).cuda()
    down = torch.zeros(96, k, dtype=torch.float16)
    up = torch.zeros(ntot, 96, dtype=torch.float16)
    row = 0
    for i, (n, _, _, _, v, u) in enumerate(parts):
        down[32 * i:32 * i + 32] = v
        up[row:row + n, 32 * i:32 * i + 32] = u
        row += n
    group = parts[0][1]
    expected = torch.cat([_oracle(x, (n, k), fmt, group, data, sc, down=v, up=u) for n, _, data, sc, v, u in parts], 1)
    y = rt.linear_stacked(x.cuda(), fmt, group, ntot, codes, scales, down=down.cuda(), up=up.cuda())
    _compare(y, expected, (fmt, g, m))
    resid = (torch.randn(m, ntot, generator=gen) * 0.5).half()
    y2 = rt.linear_stacked(x.cuda(), fmt, group, ntot, codes, scales, down=down.cuda(), up=up.cuda(), residual=resid.cuda())
    assert torch.equal(y2.cpu(), (y.float().cpu() + resid.float()).half())
    with pytest.raises(ValueError):
        rt.linear_stacked(torch.zeros(65, k, dtype=torch.float16, device='cuda'), fmt, group, ntot, codes, scales)


# ---- BASELINE configs[0] and configs[1] at their own sizes --------------------------------
SWEEP_SHAPES = [(1536, 576), (576, 1536), (8192, 2048), (2048, 8192)]
SWEEP_CELLS = [(fmt, g, n, k) for (n, k) in SWEEP_SHAPES for fmt in ('int4', 'nf4') for g in (64, 128) if k % g == 0]
_SWEEP_CACHE = {}


def _sweep_cell(n, k, fmt, g):
    """Seed-0 weight and factors of the shape, quantized by the oracle once
    per module; group 128 with K=576 is not representable and is not a cell."""
    key = (n, k, fmt, g)
    if key not in _SWEEP_CACHE:
        w, u, v = baseline_weight(n, k, seed=0)
        group, data, scales = ref.quantize(w.numpy(), fmt, g)
        prepared = ref.prepare_weight((n, k), fmt, group, data, scales)
        _SWEEP_CACHE.clear()   # one cell at a time: the big shapes' prepared weights are 64 MB
        _SWEEP_CACHE[key] = (group, data, scales, prepared, u, v)
    return _SWEEP_CACHE[key]


def test_sweep_has_fourteen_legal_cells():
    assert len(SWEEP_CELLS) == 14
    assert ('int4', 128, 1536, 576) not in SWEEP_CELLS and ('nf4', 128, 1536, 576) not in SWEEP_CELLS


@pytest.mark.parametrize('m', [16, 128, 2048])
@pytest.mark.parametrize('fmt,g,n,k', SWEEP_CELLS)
def test_sweep_cell_matches_oracle_at_full_batch(rt, fmt, g, n, k, m):
    """Every legal configs[1] cell at M = 16, 128 and 2048, every output row against the
    oracle (rank-32 correction included): the batched-decode GEMV and the tcgen05 GEMM at
    the sweep's own sizes."""
    group, data, scales, prepared, u, v = _sweep_cell(n, k, fmt, g)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(1000 + m)).half()
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    expected = ref.linear_prepared(x, prepared, down=v, up=u)
    y = rt.linear(x.cuda(), fmt, group, n, codes, sc, down=v.cuda(), up=u.cuda())
    _compare(y, expected, (fmt, g, n, k, m, rt.linear_select(fmt, group, m, n, k, 32)))


@pytest.mark.parametrize('m', [1, 128])
def test_config0_w8_linear_matches_oracle(rt, m):
    """W (1536, 576) ~ N(0, 0.02^2) from seed 0, per-channel symmetric int8,
    U [1536, 32] and V [32, 576] ~ N(0, 1e-3^2) drawn after W from the same generator,
    X ~ N(0, 1) of shape [1, 576] (decode) and [128, 576] (prefill)."""
    n, k = 1536, 576
    w, u, v = baseline_weight(n, k, seed=0)
    group, data, scales = ref.quantize(w.numpy(), 'int8')
    assert group == k
    codes, sc = rt.quantize_pack(w.cuda(), 'int8', k)
    assert codes.cpu().numpy().tobytes() == data and sc.cpu().numpy().tobytes() == scales
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(2000 + m)).half()
    expected = _oracle(x, (n, k), 'int8', group, data, scales, down=v, up=u)
    y = rt.linear(x.cuda(), 'int8', group, n, codes, sc, down=v.cuda(), up=u.cuda())
    _compare(y, expected, ('config0', m, rt.linear_select('int8', group, m, n, k, 32)))


def test_forced_plan_the_shape_cannot_take_falls_back_consistently(rt, monkeypatch):
    """A forced work split the shape cannot take (8 K-splitting warps over 5 K blocks) falls
    back to one row group per warp; its grid covers exactly the rows, with the correction."""
    monkeypatch.setenv('LOWBIT_GEMV_PLAN', '8,2,1')
    n, k = 1536, 576
    w, u, v = baseline_weight(n, k, seed=55)
    group, data, scales = ref.quantize(w.numpy(), 'nf4', 64)
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    for m in (1, 3):
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(56 + m)).half()
        expected = _oracle(x, (n, k), 'nf4', group, data, scales, down=v, up=u)
        y = rt.linear(x.cuda(), 'nf4', group, n, codes, sc, down=v.cuda(), up=u.cuda(), path='gemv')
        _compare(y, expected, ('fallback plan', m))
