"""bench.py's reference arm runs on the host cores alone, so its JSON line can
be checked here: the contract keys the driver reads, the reference arm's
cpu_baseline and its e2e object without any host/device copies."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, str(ROOT / 'bench.py'), '--impl', 'reference', '--steps', '1', '--warmup', '1'],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith('{')]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better',
                'scaling', 'vs_baseline', 'dtype', 'config', 'cpu_baseline', 'e2e'):
        assert key in d, key
    assert d['impl'] == 'reference' and d['metric'] == 'encoder_frames_per_s' and d['value'] > 0
    assert d['cpu_baseline']['value'] == d['value'] and d['cpu_baseline']['cores'] >= 1
    assert d['e2e']['value'] == d['value'] and d['e2e']['unit'] == d['unit']
    assert d['e2e']['h2d_bytes_per_step'] == 0 and d['e2e']['d2h_bytes_per_step'] == 0
    assert d['steps'] == 1 and d['warmup'] == 1


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location('bench_under_test', ROOT / 'bench.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


class _FinishedProc:
    def terminate(self):
        pass

    def wait(self, timeout=None):
        return 0

    def poll(self):
        return 0


def _sampler(bench, path, gpus):
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.gpus, s.start, s.path = gpus, 0, path
    s.proc, s.f = _FinishedProc(), open(path.parent / 'sink', 'w')
    return s


def _row(gpu, mhz, cap):
    return f'{gpu}, {mhz}, 1965, 500.0, 0x0, Not Active, Not Active, Not Active, {"Active" if cap else "Not Active"}'


def test_clock_sampler_keeps_the_timed_region(tmp_path):
    """nvidia-smi rows written before mark() (start-up, warm-up) are left out
    of the clocks summary; a power cap seen during the timed region is kept."""
    bench = _bench_module()
    path = tmp_path / 'clocks.csv'
    path.write_text('\n'.join([_row(0, 1200, False), _row(1, 1200, False)]) + '\n')
    s = _sampler(bench, path, 2)
    s.mark()
    with open(path, 'a') as f:
        f.write('\n'.join([_row(0, 1965, True), _row(1, 1950, False), _row(0, 1965, False)]) + '\n')
    info = s.stop()
    assert info == {'sm_mhz': 1965.0, 'sm_max_mhz': 1965.0, 'reasons': ['sw_power_cap'], 'samples': 3}


def test_clock_sampler_short_region_uses_last_samples(tmp_path):
    """A timed region shorter than one sampling period still reports the last
    sample of every GPU instead of no clocks at all."""
    bench = _bench_module()
    path = tmp_path / 'clocks.csv'
    path.write_text('\n'.join([_row(0, 1000, False), _row(1, 1000, False), _row(0, 1900, False),
                               _row(1, 1910, False)]) + '\n')
    s = _sampler(bench, path, 2)
    s.mark()
    info = s.stop()
    assert info is not None and info['samples'] == 2 and info['sm_mhz'] == 1905.0
