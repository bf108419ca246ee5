"""Device-side bounded waits that run out are reported, and leave the library usable.

The decode GEMV computes its rank-32 correction projection inside the same launch when
the weight is large (>= 4 MB of codes, <= 16 activation rows; one row of 4-bit codes runs
the one-row kernel, 2 rows the general one, each with its own projection CTAs): CTAs wait, with
a bound, for the CTAs that reduce the projection's K slices.  lb_test_wait_override
shortens that bound to ~1 ms and makes the wait expect one arrival that no CTA makes, so
the wait runs out for certain: the kernel records LB_ERR_TIMEOUT in the workspace status
word and returns normally (no fault, no trap, no hang).  The host must surface it as an
error and reset the status word and arrival counters, after which calls are correct again.
"""
import pytest
import torch

from oracle import lowbit_ref as ref

pytestmark = pytest.mark.gpu
SHORT_WAIT = 2_000_000   # SM clock cycles, about 1 ms


@pytest.fixture()
def rt():
    import lowbit_runtime
    lowbit_runtime.require_cuda()
    yield lowbit_runtime
    lowbit_runtime.lib().lb_test_wait_override(0, 0)
    lowbit_runtime.set_wait_checks(False)


def _fused_case(m):
    n, k = 8192, 2048
    gen = torch.Generator().manual_seed(77)
    w = (torch.randn(n, k, generator=gen) * 0.02).half()
    u = (torch.randn(n, 32, generator=gen) * 1e-3).half().cuda()
    v = (torch.randn(32, k, generator=gen) * 1e-3).half().cuda()
    x = torch.randn(m, k, generator=gen).half().cuda()
    return n, k, w, u, v, x


@pytest.mark.parametrize('m', [1, 2])
def test_timed_out_wait_raises_and_the_next_call_is_clean(rt, m):
    n, k, w, u, v, x = _fused_case(m)
    codes, sc = rt.quantize_pack(w.cuda(), 'nf4', 64)
    good = rt.linear(x, 'nf4', 64, n, codes, sc, down=v, up=u)
    torch.cuda.synchronize()
    rt.check_device_waits()                       # nothing recorded so far
    rt.set_wait_checks(True)
    rt.lib().lb_test_wait_override(SHORT_WAIT, 1)
    with pytest.raises(rt.LowbitTimeoutError):
        rt.linear(x, 'nf4', 64, n, codes, sc, down=v, up=u)
    rt.lib().lb_test_wait_override(0, 0)
    for _ in range(2):                            # status word and counters were reset
        again = rt.linear(x, 'nf4', 64, n, codes, sc, down=v, up=u)
        torch.cuda.synchronize()
        assert torch.equal(again, good)


@pytest.mark.parametrize('m', [1, 2])
def test_timeout_is_found_by_a_later_device_check(rt, m):
    """Without per-call checks (the CUDA-graph case), check_device_waits() reports it."""
    n, k, w, u, v, x = _fused_case(m)
    codes, sc = rt.quantize_pack(w.cuda(), 'nf4', 64)
    rt.lib().lb_test_wait_override(SHORT_WAIT, 1)
    rt.linear(x, 'nf4', 64, n, codes, sc, down=v, up=u)
    rt.lib().lb_test_wait_override(0, 0)
    with pytest.raises(rt.LowbitTimeoutError):
        rt.check_device_waits()
    rt.check_device_waits()                       # cleared by the first check
    y = rt.linear(x, 'nf4', 64, n, codes, sc, down=v, up=u)
    group, data, scales = 64, codes.cpu().numpy().tobytes(), sc.cpu().numpy().tobytes()
    expected = ref.linear(x.cpu(), (n, k), 'nf4', group, data, scales, down=v.cpu(), up=u.cpu()).float()
    err = float((y.float().cpu() - expected).abs().max() / expected.abs().max())
    assert err <= 1e-2
