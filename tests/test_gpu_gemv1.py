"""The one-activation-row decode GEMV for 4-bit codes (csrc/gemv1.cu) against the CPU oracle.

Covers the shapes its partition meets: a CTA per row group and several row groups per CTA,
row groups owned by one warp and split between warps (pieces summed in warp order), warps
with one unit, with many and with none, the largest staged K, 4092 row groups; INT4 (whose
code offset is removed per group from the activation sums) and NF4; group 64 and 128;
no correction, a partial rank and rank 32, with and without bias.  The tolerance is the
suite's: max |dy| / max |y_ref| <= 1e-2 and mean relative error <= 2e-3.  Settings read
once per process (the launch shape, the kernel itself) run in child processes.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from oracle import lowbit_ref as ref

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
TOL_MAX = 1e-2
TOL_MEAN = 2e-3

SHAPES = [(16, 128), (48, 16384), (576, 1536), (1536, 1536), (8192, 2048), (2048, 8192), (960, 2560),
          (65472, 128)]


def _case(n, k, fmt, g, rank, bias, seed):
    gen = torch.Generator().manual_seed(seed)
    w = (torch.randn(n, k, generator=gen) * 0.02).half()
    u = (torch.randn(n, 32, generator=gen) * 1e-3).half()[:, :rank].contiguous() if rank else None
    v = (torch.randn(32, k, generator=gen) * 1e-3).half()[:rank].contiguous() if rank else None
    b = (torch.randn(n, generator=gen) * 0.1).half() if bias else None
    x = torch.randn(1, k, generator=gen).half()
    return w, u, v, b, x


def run_cases(cases):
    """Max / mean relative error against the oracle and call-to-call equality per case."""
    import lowbit_runtime as rt
    rt.require_cuda()
    out = []
    for n, k, fmt, g, rank, bias in cases:
        w, u, v, b, x = _case(n, k, fmt, g, rank, bias, seed=n + 3 * k + rank)
        group, data, scales = ref.quantize(w.numpy(), fmt, g)
        codes = torch.frombuffer(bytearray(data), dtype=torch.uint8).cuda()
        sc = torch.frombuffer(bytearray(scales), dtype=torch.float16).cuda()
        kw = {}
        if rank:
            kw.update(down=v.cuda(), up=u.cuda())
        if bias:
            kw['bias'] = b.cuda()
        y1 = rt.linear(x.cuda(), fmt, group, n, codes, sc, **kw)
        y2 = rt.linear(x.cuda(), fmt, group, n, codes, sc, **kw)
        torch.cuda.synchronize()
        e = ref.linear(x, (n, k), fmt, group, data, scales, down=v, up=u, bias=b).float()
        d = (y1.float().cpu() - e).abs()
        out.append([float(d.max() / e.abs().max().clamp_min(1e-6)), float(d.mean() / e.abs().mean().clamp_min(1e-6)),
                    bool(torch.equal(y1, y2))])
    return out


@pytest.mark.parametrize('n,k', SHAPES)
@pytest.mark.parametrize('fmt,g', [('int4', 64), ('nf4', 64), ('int4', 128), ('nf4', 128)])
def test_one_row_gemv_matches_oracle(n, k, fmt, g):
    cases = [(n, k, fmt, g, rank, bias) for rank, bias in ((0, False), (min(32, n), True), (5, False))]
    for case, (mx, mean, same) in zip(cases, run_cases(cases)):
        assert mx <= TOL_MAX and mean <= TOL_MEAN, (case, mx, mean)
        assert same, case   # deterministic: a row group's pieces are summed in warp order


CHILD = r'''
import json, sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/torch-intel-npu_b200"]
from tests.test_gpu_gemv1 import run_cases
print(json.dumps(run_cases(json.loads(sys.argv[2]))))
'''


@pytest.mark.parametrize('env', [{'LOWBIT_G1_MODE': '1x8'}, {'LOWBIT_G1_MODE': '1x16'}, {'LOWBIT_GEMV1': '0'}])
def test_one_row_gemv_settings(env):
    cases = [[8192, 2048, 'nf4', 64, 32, True], [2048, 8192, 'int4', 128, 32, False], [576, 1536, 'int4', 64, 5, True],
             [1536, 1536, 'nf4', 128, 0, False]]
    r = subprocess.run([sys.executable, '-c', CHILD, str(ROOT), json.dumps(cases)], capture_output=True, text=True,
                       timeout=600, env={**os.environ, **env})
    assert r.returncode == 0, r.stderr[-2000:]
    for case, (mx, mean, same) in zip(cases, json.loads(r.stdout.strip().splitlines()[-1])):
        assert mx <= TOL_MAX and mean <= TOL_MEAN and same, (env, case, mx, mean)


ZSELF_SHAPES = [(16, 128), (576, 1536), (64, 2048), (32, 4096), (1536, 1536)]


def test_one_row_gemv_cta_local_projection():
    """LOWBIT_G1_ZSELF=1: below 4 MiB of codes every CTA computes the correction projection
    itself from the activation row it staged (no projection launch, no wait between CTAs);
    K = 4096 is the longest it takes, and 1536x1536 reads more V than it allows over all its
    CTAs, so that call keeps the projection launch.  Same oracle tolerance, deterministic."""
    cases = [[n, k, fmt, g, rank, bias] for n, k in ZSELF_SHAPES
             for fmt, g in (('int4', 64), ('nf4', 64), ('int4', 128), ('nf4', 128))
             for rank, bias in ((min(32, n), True), (5, False))]
    r = subprocess.run([sys.executable, '-c', CHILD, str(ROOT), json.dumps(cases)], capture_output=True, text=True,
                       timeout=600, env={**os.environ, 'LOWBIT_G1_ZSELF': '1'})
    assert r.returncode == 0, r.stderr[-2000:]
    for case, (mx, mean, same) in zip(cases, json.loads(r.stdout.strip().splitlines()[-1])):
        assert mx <= TOL_MAX and mean <= TOL_MEAN and same, (case, mx, mean)
