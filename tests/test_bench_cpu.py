"""bench.py's reference arm on the host cores: one JSON line with the contract's keys, the reference's
own ES update timed (kind 'reference' from baseline/_ref, or 'port', the oracle restatement, when the
install is absent), on the headline's metric, unit and configuration."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, 'bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '1'],
                         cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [line for line in out.stdout.splitlines() if line.startswith('{')]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d['impl'] == 'reference' and d['unit'] == 'member-tokens/s' and d['higher_is_better'] is True
    assert d['metric'].startswith('member-tokens/sec/GPU')
    assert d['value'] > 0 and d['value'] == d['cpu_baseline']['value'] == d['e2e']['value']
    assert d['cpu_baseline']['kind'] in ('reference', 'port') and d['cpu_baseline']['cores'] >= 1
    assert d['e2e']['h2d_bytes_per_step'] == 0 and d['e2e']['d2h_bytes_per_step'] == 0
    assert d['config']['workload'] == 'eggroll-rank1-antithetic'
