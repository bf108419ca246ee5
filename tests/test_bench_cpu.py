"""The benchmark's reference arm on CPU: `bench.py --impl reference` times the CPU restatement
of the reference's path on the host cores and prints one JSON line with the contract's keys
(the metric, unit and direction of the GPU arm, a cpu_baseline block describing the run, and an
e2e block with no host<->device bytes)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, str(ROOT / 'bench.py'), '--impl', 'reference', '--steps', '1',
                        '--warmup', '3'], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith('{')]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d['impl'] == 'reference'
    assert d['metric'] == 'dequant-GEMV HBM GB/s (decode sweep, M=1)' and d['unit'] == 'GB/s'
    assert d['higher_is_better'] is True and d['n_gpus'] == 1 and d['steps'] == 1 and d['warmup'] == 3
    assert d['value'] > 0 and d['config']['workload'].startswith('lowbit-gemv-sweep')
    cpu = d['cpu_baseline']
    assert cpu['kind'] in ('port', 'reference') and cpu['cores'] >= 1 and cpu['sample'] and cpu['value'] == d['value']
    assert d['e2e'] == {'value': d['value'], 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}
