"""Build liblowbit.so (sm_100a) in-tree with nvcc.

Usage: python torch-intel-npu_b200/build.py [--force]
The shared library lands next to this file so it travels with the source tree.
"""
import hashlib
import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / 'csrc'
OUT = HERE / 'liblowbit.so'
# CPython fast path for the per-call entry point (plain C over the C ABI, see csrc/pycall.c)
PYCALL_OUT = HERE / ('_lowbit_call' + (sysconfig.get_config_var('EXT_SUFFIX') or '.so'))
INCLUDE = HERE.parent / 'include'
SOURCES = ['abi.cu', 'quantize.cu', 'gemv.cu', 'gemv1.cu', 'tc_gemm.cu', 'decoder_ops.cu', 'noalloc.cu']
NVCC = os.environ.get('NVCC', '/usr/local/cuda/bin/nvcc')
FLAGS = ['-gencode', 'arch=compute_100a,code=sm_100a', '-O3', '-lineinfo', '-std=c++17',
         '-Xcompiler', '-fPIC', '-shared', '-cudart', 'shared', '--expt-relaxed-constexpr',
         '-Xlinker', '-rpath,/usr/local/cuda/lib64']


def _digest():
    h = hashlib.sha256()
    for f in sorted(CSRC.glob('*')) + [INCLUDE / 'lowbit.h']:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    h.update(' '.join(FLAGS).encode())
    return h.hexdigest()


def build(force=False, verbose=False):
    stamp = HERE / '.liblowbit.sha256'
    digest = _digest()
    if not force and OUT.exists() and PYCALL_OUT.exists() and stamp.exists() and stamp.read_text() == digest:
        return OUT
    cmd = [NVCC, *FLAGS, '-I', str(INCLUDE), *[str(CSRC / s) for s in SOURCES], '-o', str(OUT) + '.tmp']
    if verbose:
        cmd.insert(1, '-Xptxas=-v')
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError('nvcc failed:\n' + r.stdout + r.stderr)
    if verbose:
        print(r.stdout + r.stderr)
    os.replace(str(OUT) + '.tmp', OUT)
    cc = os.environ.get('CC', 'gcc')
    r = subprocess.run([cc, '-O2', '-shared', '-fPIC', '-I', sysconfig.get_paths()['include'], str(CSRC / 'pycall.c'),
                        '-o', str(PYCALL_OUT) + '.tmp'], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError('building the _lowbit_call module failed:\n' + r.stdout + r.stderr)
    os.replace(str(PYCALL_OUT) + '.tmp', PYCALL_OUT)
    stamp.write_text(digest)
    return OUT


if __name__ == '__main__':
    print(build(force='--force' in sys.argv, verbose='-v' in sys.argv))
