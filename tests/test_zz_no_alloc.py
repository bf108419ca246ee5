"""The allocation-free decode GEMV entry point (lb_linear_gemv_noalloc).

It exists for callers that cannot give the library a workspace (their device memory
belongs to an allocator they may not call, or a first cudaMalloc would stall a
latency-critical thread).  This file is collected last on purpose: if the fixed
scratch array misbehaves, every other test has already run.  It also passes when run on
its own, and one test makes the first call of a fresh process in a child process, which
exercises the first-call look-up of the array's device address.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from oracle import lowbit_ref as ref

pytestmark = pytest.mark.gpu
TOL_MAX = 1e-2


def _rel_max(y, e):
    y, e = y.float().cpu(), e.float().cpu()
    return float((y - e).abs().max() / e.abs().max().clamp_min(1e-6))


def _weights(n, k, fmt, g, seed):
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=gen) * 0.02).half()
    u = (torch.randn(n, 32, generator=gen) * 1e-3).half()
    v = (torch.randn(32, k, generator=gen) * 1e-3).half()
    group, data, scales = ref.quantize(w.numpy(), fmt, g)
    codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
    sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
    return group, codes, sc, u.cuda(), v.cuda()


def _noalloc(rt, fmt, group, x, n, codes, sc, v, u, y):
    m, k = x.shape
    return rt.lib().lb_linear_gemv_noalloc(rt.LB_FMT[fmt], group, m, n, k, rt.ptr(x), rt.ptr(codes), rt.ptr(sc),
                                           rt.ptr(v), rt.ptr(u), 0 if v is None else v.shape[0], None, rt.ptr(y),
                                           rt.stream_ptr(x.device))


@pytest.mark.parametrize('fmt,g,n,k,m,plan', [
    ('nf4', 64, 8192, 2048, 1, None),
    ('int4', 128, 2048, 8192, 4, None),
    ('int8', 2048, 2048, 2048, 16, None),
    ('nf4', 64, 2048, 2048, 3, '8,1,4'),     # cross-CTA split: partials + arrival counters in the array
    ('int4', 64, 1536, 576, 1, '2,2,2'),
])
def test_noalloc_matches_lb_linear_on_consecutive_calls(monkeypatch, fmt, g, n, k, m, plan):
    import lowbit_runtime as rt
    rt.require_cuda()
    if plan:
        monkeypatch.setenv('LOWBIT_GEMV_PLAN', plan)
    group, codes, sc, u, v = _weights(n, k, fmt, g, seed=n + k + m)
    for call in range(2):
        x = torch.randn(m, k, generator=torch.Generator().manual_seed(100 + call)).half().cuda()
        expected = rt.linear(x, fmt, group, n, codes, sc, down=v, up=u, path='gemv')
        y = torch.empty(m, n, dtype=torch.float16, device='cuda')
        status = _noalloc(rt, fmt, group, x, n, codes, sc, v, u, y)
        assert status == 0, rt.lib().lb_status_string(status)
        torch.cuda.synchronize()
        assert _rel_max(y, expected) <= TOL_MAX
        assert torch.equal(y, expected)   # same kernel and work split as lb_linear


def test_noalloc_rejects_what_it_cannot_hold(monkeypatch):
    """Every buffer here is sized for the problem, so a wrong acceptance would still be a
    valid computation; the split plan makes the partials exceed the fixed array."""
    import lowbit_runtime as rt
    rt.require_cuda()
    group, codes, sc, u, v = _weights(1024, 2048, 'nf4', 64, seed=1)
    x = torch.randn(65, 2048).half().cuda()
    y = torch.empty(65, 1024, dtype=torch.float16, device='cuda')
    assert _noalloc(rt, 'nf4', group, x, 1024, codes, sc, v, u, y) == rt.UNSUPPORTED   # M > 64 is not the GEMV
    monkeypatch.setenv('LOWBIT_GEMV_PLAN', '8,1,8')
    m, n, k = 16, 32768, 4096                                   # partials: 8 x 16 x 32768 fp32 = 16 MiB
    x = torch.randn(m, k).half().cuda()
    codes = torch.zeros(n * k, dtype=torch.uint8, device='cuda')
    scales = torch.ones(n, dtype=torch.float16, device='cuda')
    y = torch.empty(m, n, dtype=torch.float16, device='cuda')
    status = rt.lib().lb_linear_gemv_noalloc(rt.LB_FMT['int8'], k, m, n, k, rt.ptr(x), rt.ptr(codes), rt.ptr(scales),
                                             None, None, 0, None, rt.ptr(y), rt.stream_ptr(x.device))
    assert status == rt.WORKSPACE, rt.lib().lb_status_string(status)


def test_noalloc_reports_a_timed_out_wait_and_recovers():
    """The fused correction projection's bounded wait, made to run out with the test hook
    (about 1 ms, one arrival more than any CTA makes): the call returns, lb_noalloc_status
    reports LB_ERR_TIMEOUT and clears the word, and the next call is correct again."""
    import lowbit_runtime as rt
    rt.require_cuda()
    L = rt.lib()
    n, k, m = 8192, 2048, 1        # >= 4 MB of codes at M <= 16: the projection runs in the GEMV launch
    group, codes, sc, u, v = _weights(n, k, 'nf4', 64, seed=5)
    x = torch.randn(m, k, generator=torch.Generator().manual_seed(6)).half().cuda()
    expected = rt.linear(x, 'nf4', group, n, codes, sc, down=v, up=u, path='gemv')
    y = torch.empty(m, n, dtype=torch.float16, device='cuda')
    try:
        L.lb_test_wait_override(2_000_000, 1)
        assert _noalloc(rt, 'nf4', group, x, n, codes, sc, v, u, y) == 0
    finally:
        L.lb_test_wait_override(0, 0)
    assert L.lb_noalloc_status(rt.stream_ptr(x.device)) == rt.TIMEOUT
    assert L.lb_noalloc_status(rt.stream_ptr(x.device)) == rt.OK
    assert _noalloc(rt, 'nf4', group, x, n, codes, sc, v, u, y) == 0
    assert L.lb_noalloc_status(rt.stream_ptr(x.device)) == rt.OK
    assert torch.equal(y, expected)


def test_noalloc_rejects_an_output_that_aliases_an_input():
    import lowbit_runtime as rt
    rt.require_cuda()
    group, codes, sc, u, v = _weights(1024, 2048, 'int4', 64, seed=2)
    x = torch.randn(1, 2048).half().cuda()
    assert _noalloc(rt, 'int4', group, x, 1024, codes, sc, v, u, x) == rt.ALIAS


_FRESH = """
import sys, torch
sys.path[:0] = [{root!r}, {pkg!r}]
import lowbit_runtime as rt
rt.require_cuda()
gen = torch.Generator().manual_seed(9)
n, k = 4096, 2048
w = (torch.randn(n, k, generator=gen) * 0.02).half()
u = (torch.randn(n, 32, generator=gen) * 1e-3).half().cuda()
v = (torch.randn(32, k, generator=gen) * 1e-3).half().cuda()
codes, sc = rt.quantize_pack(w.cuda(), 'int4', 128)
L = rt.lib()
for call in range(2):
    x = torch.randn(2, k, generator=gen).half().cuda()
    y = torch.empty(2, n, dtype=torch.float16, device='cuda')
    s = L.lb_linear_gemv_noalloc(rt.LB_FMT['int4'], 128, 2, n, k, rt.ptr(x), rt.ptr(codes), rt.ptr(sc), rt.ptr(v),
                                 rt.ptr(u), 32, None, rt.ptr(y), rt.stream_ptr(x.device))
    assert s == 0, s
    assert L.lb_noalloc_status(rt.stream_ptr(x.device)) == 0
    expected = rt.linear(x, 'int4', 128, n, codes, sc, down=v, up=u, path='gemv')
    torch.cuda.synchronize()
    assert torch.equal(y, expected), call
print('fresh-process ok')
"""


def test_noalloc_first_call_in_a_fresh_process():
    """The very first call of a new process on a device looks up the array's address;
    run it in a child process so that the look-up really is the first one."""
    root = Path(__file__).resolve().parents[1]
    code = _FRESH.format(root=str(root), pkg=str(root / 'torch-intel-npu_b200'))
    r = subprocess.run([sys.executable, '-c', code], capture_output=True, text=True, timeout=600,
                       env=dict(os.environ, CUDA_VISIBLE_DEVICES=os.environ.get('CUDA_VISIBLE_DEVICES', '0')))
    assert r.returncode == 0, r.stdout + r.stderr
    assert 'fresh-process ok' in r.stdout
