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


def test_sweep_shards_partition_the_rows():
    bench = _bench_module()
    for m in bench.SWEEP_M + (0, 3, 7):
        for world in (1, 2, 3, 4, 8):
            spans = [bench.shard_rows(m, r, world) for r in range(world)]
            assert spans[0][0] == 0 and sum(c for _, c in spans) == m
            assert all(s + c == spans[i + 1][0] for i, (s, c) in enumerate(spans[:-1]))
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def _sweep_worker(rank, world, port, q):
    import os
    os.environ.update({'RANK': str(rank), 'WORLD_SIZE': str(world), 'LOCAL_RANK': str(rank),
                       'MASTER_ADDR': '127.0.0.1', 'MASTER_PORT': str(port)})
    from parakeet_cuda_b200.scheduler import WindowScheduler
    bench = _bench_module()
    sched = WindowScheduler(backend='gloo', timeout_s=60)
    # fake timer: 1 ns per row, rank r runs (r + 1) times slower
    pts = bench.sweep_local(sched.rank, sched.world, lambda n, k, rows: rows * 1e-9 * (sched.rank + 1))
    parts = sched.gather([pts])
    peaks = {'bf16_tflops': 1200.0, 'bf16_tflops_sustained': 1000.0, 'hbm_gbs': 5000.0}
    q.put((sched.rank, bench.merge_sweep(parts, peaks) if sched.rank == 0 else None))
    sched.close()


def test_sweep_m_sharded_over_two_gloo_ranks():
    """Each rank times only its share of M; rank 0 merges the gathered points,
    a point lasting as long as its slowest rank, with the roofline over the
    GPUs that had rows."""
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        port = s.getsockname()[1]
    bench = _bench_module()
    world = 2
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_sweep_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    merged = out[0]
    assert out[1] is None
    assert [(p['n'], p['k'], p['m']) for p in merged] == [(n, k, m) for n, k in bench.SWEEP_SHAPES
                                                         for m in bench.SWEEP_M]
    for p in merged:
        shares = [bench.shard_rows(p['m'], r, world)[1] for r in range(world)]
        assert p['gpus'] == sum(1 for c in shares if c)
        assert abs(p['us'] - max(c * 1e-3 * (r + 1) for r, c in enumerate(shares))) < 1e-9
        assert p['bound'] in ('hbm', 'tensor') and p['frac_of_roofline'] > 0
    one = [p for p in merged if p['m'] == 1]
    assert all(p['gpus'] == 1 for p in one)
