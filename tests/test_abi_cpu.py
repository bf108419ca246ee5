"""C-ABI library checks that need no GPU: it loads, exports every symbol the header
declares, and its host-side validation / path selection / fault injection behave."""
import ctypes
import re
from pathlib import Path

import pytest
import torch  # noqa: F401  (loads libcudart for the library's dynamic dependency)

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / 'include' / 'lowbit.h'
LIB = ROOT / 'torch-intel-npu_b200' / 'liblowbit.so'


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    return sorted(set(re.findall(r'\b(lb_\w+)\s*\(', text)))


@pytest.fixture(scope='module')
def lib():
    import lowbit_runtime as rt
    if not LIB.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location('lowbit_build', ROOT / 'torch-intel-npu_b200' / 'build.py')
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return rt.load_library()


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 20
    raw = ctypes.CDLL(str(LIB))
    missing = [n for n in names if not hasattr(raw, n)]
    assert not missing, missing


def test_runtime_binds_the_whole_header():
    import lowbit_runtime as rt
    assert set(declared_symbols()) == set(rt.SIGNATURES)


def test_status_strings_and_version(lib):
    assert lib.lb_abi_version() == 2
    assert lib.lb_status_string(0) == b'ok'
    assert b'Nonfinite' in lib.lb_status_string(4)
    assert lib.lb_status_string(12345) == b'unknown status'


def test_validation_rejects_before_any_launch(lib):
    P = ctypes.c_void_p
    # bad format / shapes / group: INVALID_ARGUMENT without touching CUDA
    assert lib.lb_linear(9, 64, 1, 8, 64, P(16), P(16), P(16), None, None, 0, None, P(16), P(16), 4096, None) == 1
    assert lib.lb_linear(0, 3, 1, 8, 64, P(16), P(16), P(16), None, None, 0, None, P(16), P(16), 4096, None) == 1
    assert lib.lb_linear(0, 64, 0, 8, 64, P(16), P(16), P(16), None, None, 0, None, P(16), P(16), 4096, None) == 1
    # correction factors must come in pairs with 1 <= rank <= 32
    assert lib.lb_linear(0, 64, 1, 8, 64, P(16), P(16), P(16), P(16), None, 32, None, P(16), P(16), 4096, None) == 1
    assert lib.lb_linear(0, 64, 1, 8, 64, P(16), P(16), P(16), P(16), P(16), 33, None, P(16), P(16), 4096, None) == 1
    # workspace too small
    assert lib.lb_linear(0, 64, 1, 8, 64, P(16), P(4096), P(8192), None, None, 0, None, P(1 << 20), P(1 << 24), 8, None) == 6
    # output aliasing the activations
    assert lib.lb_linear(0, 64, 1, 8, 64, P(1 << 20), P(4096), P(8192), None, None, 0, None, P(1 << 20), P(1 << 24),
                         1 << 16, None) == 7
    assert lib.lb_quantize_pack(0, 3, P(16), 1, 2, 16, P(16), P(16), P(16), 256, None) == 1
    assert lib.lb_quantize_pack(0, 16, P(16), 1, 2, 16, P(16), P(16), None, 0, None) == 6


def test_fast_call_module_matches_the_ctypes_binding(lib):
    """lowbit_runtime.linear calls lb_linear_path through the _lowbit_call module (plain C
    over the same entry point of the same loaded library); on host-validated inputs it
    returns exactly the statuses the ctypes binding returns, and rejects malformed calls."""
    import lowbit_runtime as rt
    fast = rt._FAST_LINEAR
    assert fast is not None, '_lowbit_call was not built beside liblowbit.so'
    cases = [
        (0, 9, 64, 1, 8, 64, 16, 16, 16, None, None, 0, None, 16, 16, 4096, None),           # bad format
        (0, 0, 3, 1, 8, 64, 16, 16, 16, None, None, 0, None, 16, 16, 4096, None),            # bad group
        (0, 0, 64, 0, 8, 64, 16, 16, 16, None, None, 0, None, 16, 16, 4096, None),           # M = 0
        (0, 0, 64, 1, 8, 64, 16, 16, 16, 16, None, 32, None, 16, 16, 4096, None),            # unpaired factors
        (0, 0, 64, 1, 8, 64, 16, 4096, 8192, None, None, 0, None, 1 << 20, 1 << 24, 8, None),  # workspace
        (0, 0, 64, 1, 8, 64, 1 << 20, 4096, 8192, None, None, 0, None, 1 << 20, 1 << 24, 1 << 16, None),  # alias
        (0, 0, 64, 1, 8, 64, 1 << 47, 1 << 46, 1 << 45, None, None, 0, None, 1 << 47, 1 << 44, 4, 0),
    ]
    for args in cases:
        assert fast(*args) == lib.lb_linear_path(*args), args
    with pytest.raises(TypeError):
        fast(0, 0, 64)
    with pytest.raises(OverflowError):
        fast(0, 1 << 40, 64, 1, 8, 64, 16, 16, 16, None, None, 0, None, 16, 16, 4096, None)


def test_path_selection():
    import lowbit_runtime as rt
    assert rt.linear_select('nf4', 64, 1, 8192, 2048) == 'gemv'
    assert rt.linear_select('int4', 128, 4, 2048, 8192) == 'gemv'
    assert rt.linear_select('nf4', 64, 16, 8192, 2048) == 'gemv'
    assert rt.linear_select('nf4', 64, 64, 8192, 2048) == 'gemv'     # batched decode stays on the GEMV
    assert rt.linear_select('nf4', 64, 65, 8192, 2048) == 'tc'
    assert rt.linear_select('fp16', 960, 64, 49152, 960) == 'tc'    # tied LM head at a decode batch
    assert rt.linear_select('fp16', 960, 8, 49152, 960) == 'gemv'
    assert rt.linear_select('fp16', 64, 64, 2048, 64) == 'gemv'      # narrow fp16 projections stay on the GEMV
    assert rt.linear_select('int8', 576, 128, 1536, 576) == 'tc'
    assert rt.linear_select('int4', 3, 1, 5, 9) == 'generic'      # odd shapes / groups
    assert rt.linear_select('nf4', 64, 128, 8192, 2048, 32) == 'tc'
    assert rt.linear_select('nf4', 64, 128, 8192, 2048, 5) == 'generic'  # rank not a multiple of 8


def test_workspace_query_covers_correction_and_split_k():
    import lowbit_runtime as rt
    small = rt.linear_workspace_bytes('nf4', 64, 1, 8192, 2048, 0)
    corr = rt.linear_workspace_bytes('nf4', 64, 1, 8192, 2048, 32)
    assert small >= 256 and corr >= small + 64
    split = rt.linear_workspace_bytes('nf4', 64, 32, 2048, 8192, 32)
    assert split >= 32 * 2048 * 4


def test_host_fault_injection(lib):
    import lowbit_runtime as rt
    P = ctypes.c_void_p
    rt.inject_fault('lb_linear', 2)
    args = (0, 64, 1, 8, 64, P(16), P(16), P(16), None, None, 0, None, P(16), P(16), 4096, None)
    assert lib.lb_linear(*args) == 8
    assert lib.lb_linear(*args) == 8
    assert lib.lb_linear(*args) != 8          # injection consumed
    rt.inject_fault('lb_rmsnorm', 1)
    assert lib.lb_linear(*args) != 8          # other entry points unaffected
    assert lib.lb_rmsnorm(P(16), None, None, P(16), P(4096), 1, 8, 1e-5, None) == 8
    with pytest.raises(RuntimeError, match='injected'):
        rt.check(8, 'lb_linear')


def test_noalloc_entry_validates_and_injects_before_any_launch(lib):
    """The allocation-free GEMV takes the same host-side failure paths as lb_linear: the
    injection hook, argument checks and the alias check, all before touching CUDA."""
    import lowbit_runtime as rt
    P = ctypes.c_void_p
    f = lib.lb_linear_gemv_noalloc
    rt.inject_fault('lb_linear_gemv_noalloc', 1)
    assert f(1, 64, 1, 64, 128, P(16), P(4096), P(8192), None, None, 0, None, P(1 << 20), None) == rt.INJECTED
    assert f(9, 64, 1, 64, 128, P(16), P(4096), P(8192), None, None, 0, None, P(1 << 20), None) == rt.INVALID
    assert f(1, 64, 1, 64, 128, P(16), P(4096), P(8192), P(16), None, 32, None, P(1 << 20), None) == rt.INVALID
    assert f(1, 64, 65, 64, 128, P(16), P(4096), P(8192), None, None, 0, None, P(1 << 20), None) == rt.UNSUPPORTED
    # y overlapping x / the codes / the correction factors
    assert f(1, 64, 1, 64, 128, P(1 << 20), P(4096), P(8192), None, None, 0, None, P(1 << 20), None) == rt.ALIAS
    assert f(1, 64, 1, 64, 128, P(16), P(1 << 20), P(8192), None, None, 0, None, P(1 << 20), None) == rt.ALIAS
    assert f(1, 64, 1, 64, 128, P(16), P(4096), P(8192), P(1 << 20), P(1 << 16), 32, None, P(1 << 20), None) == rt.ALIAS


def test_timeout_status_maps_to_its_own_error():
    import lowbit_runtime as rt
    with pytest.raises(rt.LowbitTimeoutError, match='timed out'):
        rt.check(rt.TIMEOUT, 'lb_linear')
    assert issubclass(rt.LowbitTimeoutError, RuntimeError)
