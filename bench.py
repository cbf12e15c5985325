"""Benchmark: Q8_0 encoder GEMM stack on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl pq8|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P bench.py --gpus N ...

One step = every Q8_0 linear of the 24 FastConformer layers (9 per layer, run
as one persistent launch of pq8_sequence_run) over this GPU's windows: 8 windows x 375 frames = 3000
activation rows per GPU, weights replicated, no collective on the data path
(weak scaling: 8/16/32/64 windows on 1/2/4/8 GPUs). Rank 0 prints one JSON
line. The metric is encoder frames per second for the whole job.

Extra keys on the line: ``roofline`` (the GEMM kernel against the TF32 tensor
peak derived from MEASURED_PEAKS.json), ``gemv`` (the M = 1 decoder-regime
kernel streaming all 642 MB of encoder weights, against HBM bandwidth),
``cpu_baseline`` (the reference's NumPy path on this host), ``e2e`` (the same
metric through the public host API with H2D/D2H copies in the timed region),
``clocks`` (nvidia-smi samples during the timed region) and ``gpu_launches``.

``--impl reference`` times the reference's CPU implementation (NumPy: Q8_0
decode + FP32 matmul) on the host cores instead; under torchrun only rank 0
runs it.
"""
from __future__ import annotations

import argparse
import json
import os
from pathlib import Path
import statistics
import subprocess
import sys
import time

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

WINDOW_FRAMES = 375
METRIC = 'encoder_frames_per_s'
UNIT = 'frames/s'


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=30)
    ap.add_argument('--warmup', type=int, default=3)
    ap.add_argument('--impl', choices=('pq8', 'reference'), default='pq8')
    ap.add_argument('--windows-per-gpu', type=int, default=8)
    ap.add_argument('--layers', type=int, default=24)
    ap.add_argument('--no-cpu-baseline', action='store_true')
    ap.add_argument('--no-extras', action='store_true', help='skip the GEMV and cuBLAS-TF32 side measurements')
    ap.add_argument('--tdt-batches', default='1,64', help='decode batch sizes of the tdt extra')
    ap.add_argument('--extras', default=None,
                    help=('comma list of side measurements to run (config0, refkernels, gemv, cublas, tdt, sweep, '
                          'load, block, refgpu, cpu); default all of them on one GPU, and on several GPUs only '
                          'the ones that measure the job (sweep, block): the others repeat the one-GPU figures '
                          'on every rank while all N GPUs are held'))
    args = ap.parse_args()
    if args.extras is None:
        world = int(os.environ.get('WORLD_SIZE', 1))
        args.extras = ('config0,refkernels,gemv,cublas,tdt,sweep,load,block,refgpu,cpu' if world == 1
                       else 'sweep,block')
    return args


def config(args, n_gpus):
    return {
        'workload': (f'config 2: {args.layers}-layer FastConformer Q8_0 linear stack (FFN x2, QKV, pos, out, '
                     f'pointwise GLU, pointwise) over {args.windows_per_gpu} windows x {WINDOW_FRAMES} frames '
                     f'per GPU'),
        'rows_per_gpu': args.windows_per_gpu * WINDOW_FRAMES,
        'windows_total': args.windows_per_gpu * n_gpus,
        'layers': args.layers,
        'parallelism': f'windows sharded over {n_gpus} GPU(s), weights replicated, no data-path collective',
        'l2': 'weights streamed per step (642 MB packed Q8_0 > 126 MB L2); no flush needed',
        'execution': ('one persistent launch per step (pq8_sequence_run): the 216 linears as tiles with '
                      'row-block dependencies that follow the block\'s data flow'),
        'weights': 'random Q8_0, int8 U[-127,127], fp16 scales U[1e-3,2e-2]; activations N(0,1)',
    }


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling every 50 ms. It is started before the warm-up (the
    tool takes a moment to come up, longer with several GPUs); ``wait_ready``
    waits for its first samples and ``mark`` notes where the timed region
    starts, so that ``stop`` summarises the samples taken during it."""

    def __init__(self, gpus: int):
        self.proc = None
        self.gpus = gpus
        self.start = 0
        self.path = Path(os.environ.get('TMPDIR', '/tmp')) / f'pq8_clocks_{os.getpid()}.csv'
        q = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
             'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
             'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')
        try:
            self.f = open(self.path, 'w')
            self.proc = subprocess.Popen(['nvidia-smi', f'--query-gpu={q}', '--format=csv,noheader,nounits',
                                          '-i', ','.join(str(i) for i in range(gpus)), '-lms', '50'],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def _lines(self):
        try:
            return [l for l in self.path.read_text().splitlines() if l.strip()]
        except OSError:
            return []

    def wait_ready(self, timeout_s: float = 10.0):
        t0 = time.time()
        while self.proc is not None and self.proc.poll() is None and time.time() - t0 < timeout_s:
            if len(self._lines()) >= self.gpus:
                return
            time.sleep(0.05)

    def mark(self):
        self.start = len(self._lines())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], 0, set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        lines = self._lines()
        during = lines[self.start:]
        # a timed region shorter than one sampling period: the last sample of each GPU
        for line in (during if len(during) >= self.gpus else lines[-self.gpus:]):
            parts = [p.strip() for p in line.split(',')]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for name, v in zip(names, parts[5:9]):
                if v.lower().startswith('active'):
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return None
        return {'sm_mhz': statistics.median(sm), 'sm_max_mhz': mx, 'reasons': sorted(reasons), 'samples': len(sm)}


def measured_peaks():
    p = ROOT / 'MEASURED_PEAKS.json'
    if p.is_file():
        d = json.loads(p.read_text())
        return d, 'measured'
    return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0, 'bf16_tflops_sustained': 1400.0}, 'fallback'


def ncu_traffic():
    """Per-launch DRAM bytes of the GEMM kernel from the committed ncu summary, if any."""
    p = ROOT / 'profiles' / 'gemm_traffic.json'
    if p.is_file():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


# ------------------------------------------------------------------ CPU legs
def host_cores() -> int:
    """CPUs this process may run on."""
    return len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else (os.cpu_count() or 1)


def all_blas_threads():
    """BLAS thread pool raised to every usable host core for the CPU legs
    (torchrun starts each rank with OMP_NUM_THREADS=1)."""
    from threadpoolctl import threadpool_limits
    return threadpool_limits(limits=host_cores(), user_api='blas')


def one_blas_thread():
    from threadpoolctl import threadpool_limits
    return threadpool_limits(limits=1, user_api='blas')


def cpu_sample(model, rows=WINDOW_FRAMES, repeats=3):
    """Config 2 on the host: the reference's NumPy path with the BLAS pool at every
    usable core (the reported baseline) and at one thread (``single_thread``)."""
    from oracle.cpu_path import blas_threads, time_layer_window
    with all_blas_threads():
        times = [time_layer_window(model, rows, layer=0, seed=i) for i in range(repeats)]
        cores = blas_threads()
    with one_blas_thread():
        t1 = time_layer_window(model, rows, layer=0, seed=9)
    t = min(times)
    return {'value': rows / (t * 24), 'unit': UNIT, 'cores': cores, 'kind': 'port',
            'sample': (f'NumPy restatement of the reference CPU path (gguf.array Q8_0 decode + FP32 x @ W.T, '
                       f'reference.py:37): one layer x one {rows}-frame window, best of {repeats} '
                       f'({t:.3f} s), scaled to 24 layers'),
            'single_thread': {'value': rows / (t1 * 24), 'unit': UNIT, 'cores': 1,
                              'sample': f'the same layer x window once at OPENBLAS threads = 1 ({t1:.3f} s)'},
            'host_cpus': host_cores(), 'cpu_model': cpu_model()}


def cpu_model() -> str:
    try:
        for line in Path('/proc/cpuinfo').read_text().splitlines():
            if line.startswith('model name'):
                return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


def cpu_other_configs():
    """CPU baselines of the other BASELINE configs (reference NumPy path restated in
    oracle/cpu_path.py), each at every usable core and at one BLAS thread, on
    bounded samples: config 0 (one Q8_0 linear, M=128, K=1024, N=4096), config 3
    (the reference's float32 CPUDecoder driven by its greedy loop; the reference
    decodes streams one after another, so batch 64 runs at the batch-1 rate per
    joint call) and config 4 (the sweep shapes at M up to 1024; larger M is a
    proportionally longer matmul)."""
    import numpy as np
    from oracle.cpu_path import blas_threads, time_decode, time_linear
    from parakeet_cuda_b200.synthetic import DECODER_SCALE, SyntheticParakeet, q8_0_blocks
    out = {}
    raw0 = q8_0_blocks(np.random.default_rng(0), 4096, 1024)
    model = SyntheticParakeet(seed=11, encoder_layers=0)
    proj = np.random.default_rng(2026).normal(size=(400, 640)).astype(np.float32)
    for label, ctx in (('all_cores', all_blas_threads), ('one_thread', one_blas_thread)):
        with ctx():
            cores = blas_threads()
            t0 = time_linear(raw0, 4096, 1024, 128, repeats=5)
            td, calls = time_decode(model, [proj], [0, 1, 2, 3, 4])
            sweep = []
            for n, k in SWEEP_SHAPES:
                raw = q8_0_blocks(np.random.default_rng(n + k), n, k)
                for m in (1, 16, 128, 1024):
                    t = time_linear(raw, n, k, m, repeats=3)
                    sweep.append({'m': m, 'n': n, 'k': k, 'us': t * 1e6, 'gflops': 2 * m * n * k / t / 1e9,
                                  'gbs': (1.0625 * n * k + 4 * m * (n + k)) / t / 1e9})
        out[label] = {
            'cores': cores,
            'config0': {'us': t0 * 1e6, 'gflops': 2 * 128 * 4096 * 1024 / t0 / 1e9,
                        'sample': 'x @ W.T, M=128 K=1024 N=4096, weight decoded beforehand, best of 5'},
            'config3': {'joint_calls': calls, 'seconds': td, 'joint_calls_per_s': calls / td,
                        'sample': ('one stream of 400 projected frames through the greedy loop with the float32 '
                                   'CPUDecoder restatement; steps/s at batch 1 = joint calls/s')},
            'config4': sweep,
        }
    return out


def run_reference(args):
    rank = int(os.environ.get('RANK', 0))
    if rank != 0:
        return
    from parakeet_cuda_b200.synthetic import SyntheticParakeet
    model = SyntheticParakeet(seed=0, encoder_layers=1, decoder=False)
    from oracle.cpu_path import blas_threads, time_layer_window
    with all_blas_threads():
        for i in range(args.warmup):
            time_layer_window(model, WINDOW_FRAMES, 0, seed=i)
        times = [time_layer_window(model, WINDOW_FRAMES, 0, seed=100 + i) for i in range(args.steps)]
        cores = blas_threads()
    t = sum(times) / len(times)
    value = WINDOW_FRAMES / (t * 24)
    n = args.gpus
    line = {'impl': 'reference', 'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': n,
            'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': t * 1000, 'higher_is_better': True,
            'scaling': 'weak', 'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'config': config(args, n),
            'cpu_baseline': {'value': value, 'unit': UNIT, 'cores': cores, 'kind': 'port',
                             'sample': (f'each step: one encoder layer (Q8_0 decode + 9 FP32 linears) over one '
                                        f'{WINDOW_FRAMES}-frame window; frames/s = {WINDOW_FRAMES} / '
                                        f'(24 x step time)')},
            'e2e': {'value': value, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
class LaunchTimer:
    """CUDA events around each launch on the launching stream, grouped by name."""

    def __init__(self, torch):
        self.torch = torch
        self.pairs = []
        self.open = None

    def start(self, name):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        self.open = (name, e)

    def stop(self, name):
        e = self.torch.cuda.Event(enable_timing=True)
        e.record()
        self.pairs.append((self.open[0], self.open[1], e))

    def totals(self):
        out = {}
        for name, a, b in self.pairs:
            ms = a.elapsed_time(b)
            c, t = out.get(name, (0, 0.0))
            out[name] = (c + 1, t + ms)
        return out


def run_gpu(args):
    import numpy as np
    import torch
    from parakeet_cuda_b200.encoder import LAYER_PLAN, EncoderStack
    from parakeet_cuda_b200.runtime import Runtime
    from parakeet_cuda_b200.scheduler import WindowScheduler
    from parakeet_cuda_b200.synthetic import SyntheticParakeet

    sched = WindowScheduler(timeout_s=300)
    n = sched.world
    if n != args.gpus:
        print(f'warning: --gpus {args.gpus} but WORLD_SIZE {n}; using {n}', file=sys.stderr)
    dev = sched.local_rank if n > 1 else 0
    torch.cuda.set_device(dev)
    rows = args.windows_per_gpu * WINDOW_FRAMES
    model = SyntheticParakeet(seed=0, encoder_layers=args.layers, decoder=False)
    for name in model.tensors:  # generate the random GGUF bytes before the upload is timed
        model.raw(name)
    rt = Runtime(dev)
    stack = EncoderStack(model, rt, rows, layers=args.layers, seed=1 + sched.rank)
    load = {'device_upload': {'layers': args.layers, 'seconds': stack.load_seconds,
                              'gguf_bytes': rt.uploader().bytes_uploaded,
                              'gbs': rt.uploader().bytes_uploaded / stack.load_seconds / 1e9}}
    if sched.rank == 0 and not args.no_extras and 'load' in args.extras.split(','):
        load.update(load_measure(torch, rt, model))
    ref_raw = None
    if not args.no_extras and 'refgpu' in args.extras.split(','):
        ref_raw = upload_raw_layers(torch, model, args.layers, dev)
    # the same stack on the torch-free host layer (driver API + ctypes): the e2e path
    from parakeet_cuda_b200.host import EncoderStackHost, HostRuntime
    hrt = HostRuntime(dev)
    hstack = EncoderStackHost(model, hrt, rows, layers=args.layers, seed=1 + sched.rank)
    del model
    torch.cuda.synchronize()

    # The timed step: every Q8_0 linear of the 24 layers as ONE persistent launch
    # (pq8_sequence_run of a plan with the block's data-flow dependencies) on the
    # torch-free host stack, replayed from a CUDA graph captured with
    # cuStreamBeginCapture and timed with driver events on its stream.
    from parakeet_cuda_b200.cuda_driver import Event as DrvEvent, PinnedArray
    hstack.make_sequence('model')
    hstack.step_sequence()
    hrt.synchronize()
    hgraph = hstack.capture(sequence=True)
    clocks = ClockSampler(n) if sched.rank == 0 else None
    for _ in range(args.warmup):
        hgraph.launch(hrt.stream)
    hrt.synchronize()
    if clocks:
        clocks.wait_ready()
    sched.barrier()
    d0, d1 = DrvEvent(hrt.drv), DrvEvent(hrt.drv)
    hrt.synchronize()
    sched.barrier()
    if clocks:
        clocks.mark()
    d0.record(hrt.stream)
    for _ in range(args.steps):
        hgraph.launch(hrt.stream)
    d1.record(hrt.stream)
    d1.synchronize()
    sched.barrier()
    clock_info = clocks.stop() if clocks else None
    ms = d0.elapsed_ms(d1) / args.steps
    ms_max = sched.max_over_ranks(ms)

    # The same linears as one launch each (216 launches, programmatic dependent
    # launch between them, graph replay): the launch-per-linear step, beside it.
    stack.step()
    torch.cuda.synchronize()
    graph = stack.capture()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    sched.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    ms_launches = sched.max_over_ranks(start.elapsed_time(end) / args.steps)

    # Per-shape context: the same launches issued eagerly, each bracketed by
    # CUDA events on the launching stream (the events break the overlap of
    # consecutive launches and add launch gaps, so these run slower than the
    # graph).
    timer = LaunchTimer(torch)
    for _ in range(args.steps):
        stack.step(timer)
    torch.cuda.synchronize()
    per_name = timer.totals()
    kernel_ms_step = sum(t for _, t in per_name.values()) / args.steps

    # same stack with every GEMM rounding its activation tile in shared memory
    stack.producer_tf32 = False
    graph_rnd = stack.capture()
    graph_rnd.replay()
    torch.cuda.synchronize()
    sched.barrier()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    for _ in range(args.steps):
        graph_rnd.replay()
    k1.record()
    torch.cuda.synchronize()
    ms_kernel_rounding = sched.max_over_ranks(k0.elapsed_time(k1) / args.steps)
    stack.producer_tf32 = True
    del graph_rnd
    status = rt.device_status()

    # e2e: the public host API without PyTorch (EncoderStackHost: driver-API memory and
    # streams, the sequence graph), page-locked H2D of each step's input and D2H of
    # its result inside the timed region. The headline uses run_host_pipelined (copies of
    # neighbouring steps overlap the compute; two host buffers per direction in rotation);
    # one run_host per step, copies and compute back to back, is reported beside it.
    hx = [PinnedArray(hrt.drv, (rows, 1024)) for _ in range(2)]
    hout = [PinnedArray(hrt.drv, (rows, 1024)) for _ in range(2)]
    for i, a in enumerate(hx):
        a.array[...] = np.random.default_rng(100 + i).standard_normal((rows, 1024), np.float32)
    h_in = [hx[i % 2] for i in range(args.steps)]
    h_out = [hout[i % 2] for i in range(args.steps)]
    for _ in range(2):
        hstack.run_host(hx[0], hout[0], hgraph)
    hstack.run_host_pipelined(h_in[:2], h_out[:2], hgraph)
    hrt.synchronize()
    sched.barrier()
    d0.record(hrt.stream)
    hstack.run_host_pipelined(h_in, h_out, hgraph)
    d1.record(hrt.stream)
    d1.synchronize()
    e2e_host_ms = sched.max_over_ranks(d0.elapsed_ms(d1) / args.steps)
    sched.barrier()
    d0.record(hrt.stream)
    for i in range(args.steps):
        hstack.run_host(h_in[i], h_out[i], hgraph)
    d1.record(hrt.stream)
    d1.synchronize()
    e2e_host_serial_ms = sched.max_over_ranks(d0.elapsed_ms(d1) / args.steps)
    seq_status = hrt.device_status()
    hgraph.close()
    hstack.close()
    for a in hx + hout:
        a.close()
    hrt.close()
    del hstack, hrt

    # the same public calls on the PyTorch-hosted stack, for comparison
    x_hosts = [torch.randn(rows, 1024).pin_memory() for _ in range(2)]
    out_hosts = [torch.empty(rows, 1024).pin_memory() for _ in range(2)]
    step_in = [x_hosts[i % 2] for i in range(args.steps)]
    step_out = [out_hosts[i % 2] for i in range(args.steps)]
    for _ in range(2):
        stack.run_host(x_hosts[0], out_hosts[0], graph)
    stack.run_host_pipelined(step_in[:2], step_out[:2], graph)
    torch.cuda.synchronize()
    sched.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    stack.run_host_pipelined(step_in, step_out, graph)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = sched.max_over_ranks(e0.elapsed_time(e1) / args.steps)
    sched.barrier()
    e0.record()
    for i in range(args.steps):
        stack.run_host(step_in[i], step_out[i], graph)
    e1.record()
    torch.cuda.synchronize()
    e2e_serial_ms = sched.max_over_ranks(e0.elapsed_time(e1) / args.steps)
    del graph

    extras = {}
    sweep_points = None
    if not args.no_extras:
        wanted = set(args.extras.split(','))
        if 'gemv' in wanted:
            extras['gemv'] = gemv_measure(torch, rt, stack)
        if 'cublas' in wanted:
            extras['tf32_cublas_tflops'] = cublas_tf32(torch)
        if 'config0' in wanted:
            extras['config0'] = config0_measure(torch, rt)
        if 'refkernels' in wanted and sched.rank == 0:
            extras['reference_gpu_kernels'] = reference_gpu_kernels()
        if 'tdt' in wanted:
            extras['tdt'] = tdt_measure(torch, rt, [int(b) for b in args.tdt_batches.split(',')])
        if 'sweep' in wanted:
            sweep_points = sweep_measure(torch, rt, sched.rank, n)
        if 'load' in wanted:
            extras['weight_load'] = load
        if 'refgpu' in wanted:
            extras['reference_gpu_method'] = reference_gpu_method(torch, rt, ref_raw, stack)
        ref_raw = None
        if 'block' in wanted:
            extras['full_block'] = block_measure(torch, rt, args, ms)
    sched.barrier()
    if sweep_points is not None:  # every rank ran its share (the arguments are the same on every rank)
        parts = sched.gather([sweep_points])
        if sched.rank == 0:
            extras['sweep'] = merge_sweep(parts, measured_peaks()[0])

    if sched.rank == 0:
        peaks, peak_src = measured_peaks()
        flops_step = stack.flops_per_step()
        # The timed step is one launch of the sequence kernel and nothing else,
        # so the step time is that kernel's average launch duration.
        launch_ms = ms
        achieved = flops_step / (ms / 1e3) / 1e12
        # the timed region is args.steps graph replays (a fraction of a second):
        # the burst peak applies; the sustained one is reported beside it
        peak = peaks['bf16_tflops'] / 2
        shapes = {}
        for entry in LAYER_PLAN:
            name, _, nn, kk = entry[:4]
            cnt, tot = per_name.get(name, (0, 0.0))
            if cnt:
                shapes[name] = {'n': nn, 'k': kk, 'ms': tot / cnt,
                                'tflops': 2 * rows * nn * kk / (tot / cnt / 1e3) / 1e12}
        traffic = ncu_traffic()
        frames = rows * n
        line = {
            'metric': METRIC, 'value': frames / (ms_max / 1e3), 'unit': UNIT, 'n_gpus': n, 'steps': args.steps,
            'warmup': args.warmup, 'ms_per_step': ms_max, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'tf32', 'data': 'synthetic (random Q8_0 weights, N(0,1) activations)',
            'config': config(args, n),
            'roofline': {
                'bound': 'tensor', 'achieved': achieved,
                'peak': peak, 'unit': 'TFLOP/s', 'frac': achieved / peak,
                'traffic': traffic.get('bytes_per_launch') if traffic else None,
                'traffic_unit': 'DRAM bytes per launch (one sequence launch = the whole step; ncu capture)',
                'traffic_bytes_per_step': traffic.get('bytes_per_step_24_layers') if traffic else None,
                'peak_source': (f'{peak_src}: MEASURED_PEAKS.json bf16_tflops / 2 (burst; dense TF32 is half '
                                f'the BF16 rate; timed region {args.steps * ms / 1e3:.2f} s)'),
                'frac_of_sustained': achieved / (peaks['bf16_tflops_sustained'] / 2),
                'cublas_tf32_tflops': extras.get('tf32_cublas_tflops'),
                'frac_of_cublas_tf32': (achieved / extras['tf32_cublas_tflops']
                                        if extras.get('tf32_cublas_tflops') else None),
                'kernel': ('pq8::gemm_tc_kernel, sequence form (every tile of the 216 linears of a step in one '
                           'persistent launch)'),
                'flops_per_step': flops_step, 'launches_per_step': 1,
                'launch_ms_mean': launch_ms,
                'achieved_basis': ('algorithmic FLOPs per step / timed graph step (driver events on the launching '
                                   'stream; the step is the one sequence launch)'),
                'per_linear_launches': {'ms_per_step': ms_launches, 'launches_per_step': stack.launches_per_step,
                                        'tflops': flops_step / (ms_launches / 1e3) / 1e12,
                                        'frac': flops_step / (ms_launches / 1e3) / 1e12 / peak,
                                        'frames_per_s': rows * n / (ms_launches / 1e3),
                                        'what': 'the same linears as one pq8_gemm launch each (PDL, graph replay)'},
                'eager_isolated_launches': {'kernel_ms_per_step': kernel_ms_step,
                                            'tflops': flops_step / (kernel_ms_step / 1e3) / 1e12,
                                            'per_shape': shapes},
                'traffic_source': traffic.get('source') if traffic else None,
            },
            'e2e': {'value': frames / (e2e_host_ms / 1e3), 'unit': UNIT, 'h2d_bytes_per_step': rows * 1024 * 4,
                    'd2h_bytes_per_step': rows * 1024 * 4, 'gpu_launches_per_step': 2,
                    'api': ('parakeet_cuda_b200.host.EncoderStackHost.run_host_pipelined: no PyTorch (CUDA driver '
                            'API through ctypes, page-locked host in/out, cuStreamBeginCapture graph of the '
                            'sequence launch; one pq8_round_tf32 launch per step on the uploaded input); each step '
                            'copies its own input and result, overlapped with the neighbouring steps\' compute'),
                    'serial': {'value': frames / (e2e_host_serial_ms / 1e3),
                               'api': 'EncoderStackHost.run_host once per step (copies not overlapped)'},
                    'torch_hosted': {'value': frames / (e2e_ms / 1e3),
                                     'serial': frames / (e2e_serial_ms / 1e3),
                                     'api': 'parakeet_cuda_b200.encoder.EncoderStack.run_host_pipelined / run_host'}},
            'gpu_launches': args.steps,
            'device_status': status or seq_status,
            'x_rounding': ('GEMM inputs from outside the path (LayerNorm output, attention context, positional '
                           'table stand-ins) are produced TF32-rounded; SiLU/GLU outputs are rounded by the fused '
                           'epilogue; e2e rounds its uploaded input with one pq8_round_tf32 launch per step'),
            'in_kernel_rounding': {'ms_per_step': ms_kernel_rounding,
                                   'value': frames / (ms_kernel_rounding / 1e3),
                                   'note': ('the launch-per-linear step with every GEMM rounding its own X tile '
                                            '(no producer help)')},
        }
        if clock_info:
            line['clocks'] = clock_info
        line.update(extras)
        if 'full_block' in extras:
            fb = extras['full_block']
            line['model_level'] = {
                'value': fb['frames_per_s'] * n, 'unit': UNIT, 'with_stem': fb['encoder_with_stem_frames_per_s'] * n,
                'what': ('whole FastConformer blocks (LayerNorms, rel-pos attention, conv module and the same Q8_0 '
                         'linears), 24 layers over this GPU\'s windows, one graph replay per step; with_stem adds '
                         'the subsampling stem from 8x mel frames'),
                'gpus_measured': 'rank 0 (every rank runs the same shapes)'}
        if n == 1 and not args.no_cpu_baseline:
            from parakeet_cuda_b200.synthetic import SyntheticParakeet as SP
            line['cpu_baseline'] = cpu_sample(SP(seed=0, encoder_layers=1, decoder=False))
            if not args.no_extras and 'cpu' in args.extras.split(','):
                line['cpu_baseline']['other_configs'] = cpu_other_configs()
        print(json.dumps(line), flush=True)
    sched.close()


# the reference's own GEMM benchmark shapes (M, K, N) and its published GTX 750 Ti
# times in microseconds, direct q8_gemm and dequant_q8 + cuBLAS SGEMM
# (analysis/CUDA_RESULTS.md:117-120, analysis/benchmark_dense.py)
REFERENCE_SHAPES = ((1, 32, 3, 5.216, 4.416), (17, 640, 65, 104.926, 21.688), (33, 1024, 129, 194.363, 40.280),
                    (441, 1024, 4096, 14971.336, 4701.824))


def config0_measure(torch, rt):
    """BASELINE config 0 (X [128, 1024] ~ N(0, 1), W [4096, 1024] Q8_0, scales
    U[1e-3, 2e-2]) through pq8_linear, and the reference's own benchmark shapes.

    ``warm``: a CUDA graph of 20 back-to-back launches (the 4.4 MB weight stays in
    L2), ``cold``: one launch at a time after writing a 256 MB buffer (L2
    flushed), each bracketed by CUDA events. Roofline time = the larger of the
    FLOPs over the burst TF32 peak and the algorithmic bytes over HBM bandwidth."""
    import numpy as np
    from parakeet_cuda_b200.synthetic import q8_0_blocks
    peaks, src = measured_peaks()
    p_tf32, bw = peaks['bf16_tflops'] / 2 * 1e12, peaks['hbm_gbs'] * 1e9
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=rt.device)

    def point(m, k, n, seed):
        rng = np.random.default_rng(seed)
        w = rt.pack(q8_0_blocks(rng, n, k), n, k)
        x = torch.from_numpy(rng.normal(size=(m, k)).astype(np.float32)).to(rt.device)
        y = torch.empty(m, n, device=rt.device)
        for _ in range(3):
            rt.linear(x, w, out=y)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(rt.device)
        side.wait_stream(torch.cuda.current_stream(rt.device))
        reps = 20
        with torch.cuda.stream(side):
            g.capture_begin()
            for _ in range(reps):
                rt.linear(x, w, out=y)
            g.capture_end()
        torch.cuda.current_stream(rt.device).wait_stream(side)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        warm_us = a.elapsed_time(b) * 1e3 / (5 * reps)
        cold = []
        for _ in range(10):
            flush.fill_(1)
            a.record()
            rt.linear(x, w, out=y)
            b.record()
            torch.cuda.synchronize()
            cold.append(a.elapsed_time(b) * 1e3)
        del g
        flops = 2 * m * n * k
        nbytes = 1.0625 * n * k + 4 * m * k + 4 * m * n
        t_roof = max(flops / p_tf32, nbytes / bw) * 1e6
        cold_us = statistics.median(cold)
        return {'m': m, 'k': k, 'n': n, 'warm_us': warm_us, 'cold_us': cold_us,
                'warm_tflops': flops / warm_us / 1e6, 'cold_tflops': flops / cold_us / 1e6,
                'roofline_us': t_roof, 'frac_warm': t_roof / warm_us, 'frac_cold': t_roof / cold_us,
                'bound': 'hbm' if nbytes / bw > flops / p_tf32 else 'tensor'}

    out = point(128, 1024, 4096, 0)
    out['peak_source'] = f'{src}: bf16_tflops / 2 (burst TF32), hbm_gbs'
    out['reference_benchmark_shapes'] = []
    for m, k, n, direct_us, sgemm_us in REFERENCE_SHAPES:
        r = point(m, k, n, 903 + m)
        r['gtx750ti_us'] = {'q8_gemm_direct': direct_us, 'dequant_sgemm': sgemm_us}
        out['reference_benchmark_shapes'].append(r)
    del flush
    return out


REF_CUBINS = ROOT / 'baseline' / '_ref'
# (label, m, k, n): the reference's benchmark shapes, config 0, and the decoder's M = 1 shapes
REF_KERNEL_CASES = (('ref 1x32x3', 1, 32, 3), ('ref 17x640x65', 17, 640, 65), ('ref 33x1024x129', 33, 1024, 129),
                    ('ref 441x1024x4096', 441, 1024, 4096), ('config0 128x1024x4096', 128, 1024, 4096),
                    ('lstm gates 1x640x2560', 1, 640, 2560), ('joint.pred 1x640x640', 1, 640, 640),
                    ('joint 1x640x8198', 1, 640, 8198))


def reference_gpu_kernels():
    """The reference's own GPU kernels on this B200, built from its sources for
    sm_100a (baseline/Makefile), against pq8 on the same shapes and inputs.

    Methods (analysis/benchmark_dense.py): (i) ``dequant_q8`` + ``cublasSgemm_v2``
    (the production path, gpu.py:87-90,169-184: FP32 weights expanded, FP32
    SGEMM), (ii) the direct ``q8_gemm`` kernel (kernels/q8_gemm.cu), (iii)
    ``q8_gemv`` (runtime.cu:180-188) for M = 1; pq8 through ``pq8_linear``.
    Each is captured as a CUDA graph of 10 calls; the graphs are replayed
    alternately 10 times and the first 2 replays dropped; microseconds per call
    (median). Outputs are checked against each other (max |diff| / RMS).
    Driver API and cuBLAS through ctypes, no PyTorch."""
    import ctypes as C
    import numpy as np
    from parakeet_cuda_b200 import pq8
    from parakeet_cuda_b200.cuda_driver import Event
    from parakeet_cuda_b200.host import HostRuntime
    from parakeet_cuda_b200.synthetic import q8_0_blocks
    rt_cubin, gemm_cubin = REF_CUBINS / 'runtime_sm100a.cubin', REF_CUBINS / 'q8_gemm_sm100a.cubin'
    if not (rt_cubin.is_file() and gemm_cubin.is_file()):
        return {'unavailable': 'baseline/_ref cubins not built (make -C baseline REFERENCE=<checkout>)'}
    rt = HostRuntime(0, weight_bytes=256 << 20, work_bytes=256 << 20)
    drv = rt.drv
    blas = C.CDLL('libcublas.so.12')
    for name, args in {'cublasCreate_v2': [C.POINTER(C.c_void_p)], 'cublasSetStream_v2': [C.c_void_p, C.c_void_p],
                       'cublasDestroy_v2': [C.c_void_p],
                       'cublasSgemm_v2': [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                          C.POINTER(C.c_float), C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                          C.POINTER(C.c_float), C.c_void_p, C.c_int]}.items():
        fn = getattr(blas, name)
        fn.argtypes, fn.restype = args, C.c_int
    handle = C.c_void_p()
    if blas.cublasCreate_v2(C.byref(handle)):
        return {'unavailable': 'cublasCreate failed'}
    blas.cublasSetStream_v2(handle, rt.stream.handle)
    one, zero = C.c_float(1.0), C.c_float(0.0)
    modules = {}
    funcs = {}
    for path, names in ((rt_cubin, (b'dequant_q8', b'q8_gemv')), (gemm_cubin, (b'q8_gemm',))):
        mod = C.c_void_p()
        drv.call('cuModuleLoad', C.byref(mod), str(path).encode())
        modules[path] = mod
        for nm in names:
            f = C.c_void_p()
            drv.call('cuModuleGetFunction', C.byref(f), mod, nm)
            funcs[nm.decode()] = f

    def launch(f, grid, params):
        holders = [C.c_uint64(v) if isinstance(v, Ptr) else C.c_int(v) for v in params]
        ptrs = (C.c_void_p * len(holders))(*(C.addressof(h) for h in holders))
        launch.keep.append((holders, ptrs))
        drv.call('cuLaunchKernel', f, grid, 1, 1, 256, 1, 1, 0, rt.stream.handle, ptrs, None)
    launch.keep = []

    class Ptr(int):
        pass

    out = {'method': 'graph of 10 calls, 10 alternating replays, first 2 dropped, median us per call',
           'build': 'nvcc --cubin -O3 -std=c++17 -lineinfo -arch=sm_100a (baseline/Makefile)', 'cases': []}
    rng = np.random.default_rng(17)
    up = rt.uploader()
    for label, m, k, n in REF_KERNEL_CASES:
        rt.work.reset()
        raw = q8_0_blocks(rng, n, k)
        x = rng.standard_normal((m, k), np.float32)
        d_raw = rt.upload(raw.reshape(-1))
        d_x = rt.upload(x)
        d_wf = rt.work.alloc((n, k))
        ys = {name: rt.work.alloc((m, n)) for name in ('pq8', 'sgemm', 'direct', 'gemv')}
        w = up.pack_rows([raw], n, k)
        up.finish()
        calls = {
            'pq8': lambda: rt.linear(d_x, w, ys['pq8'], m),
            'dequant_sgemm': lambda: (
                launch(funcs['dequant_q8'], (n * k + 255) // 256, [Ptr(d_raw.pointer), Ptr(d_wf.pointer), n * k]),
                blas.cublasSgemm_v2(handle, 1, 0, n, m, k, C.byref(one), d_wf.pointer, k, d_x.pointer, k,
                                    C.byref(zero), ys['sgemm'].pointer, n)),
            'q8_gemm_direct': lambda: launch(funcs['q8_gemm'], ((m + 31) // 32) * ((n + 63) // 64),
                                             [Ptr(w_raw), Ptr(d_x.pointer), Ptr(ys['direct'].pointer), m, k, n]),
        }
        w_raw = d_raw.pointer
        if m == 1:
            calls['q8_gemv'] = lambda: launch(funcs['q8_gemv'], n, [Ptr(d_raw.pointer), Ptr(d_x.pointer),
                                                                     Ptr(ys['gemv'].pointer), k, n])
        for fn in calls.values():
            fn()
        rt.synchronize()
        res = {n_: rt.download(b) for n_, b in ys.items()}
        scale = float(np.sqrt(np.mean(res['sgemm'].astype(np.float64) ** 2))) or 1.0
        check = {name: float(np.max(np.abs(res[key] - res['sgemm']))) / scale
                 for name, key in (('pq8', 'pq8'), ('q8_gemm_direct', 'direct')) + ((('q8_gemv', 'gemv'),) if m == 1 else ())}
        graphs = {name: rt.stream.capture(lambda fn=fn: [fn() for _ in range(10)]) for name, fn in calls.items()}
        samples = {name: [] for name in calls}
        a, b = Event(drv), Event(drv)
        order = list(calls)
        for rep in range(10):
            for name in (order if rep % 2 == 0 else order[::-1]):
                a.record(rt.stream)
                graphs[name].launch(rt.stream)
                b.record(rt.stream)
                b.synchronize()
                if rep >= 2:
                    samples[name].append(a.elapsed_ms(b) * 1e3 / 10)
        for g in graphs.values():
            g.close()
        us = {name: float(np.median(v)) for name, v in samples.items()}
        flops = 2.0 * m * n * k
        out['cases'].append({'case': label, 'm': m, 'k': k, 'n': n, 'us': us,
                             'gflops': {name: flops / t / 1e3 for name, t in us.items()},
                             'pq8_speedup': {name: t / us['pq8'] for name, t in us.items() if name != 'pq8'},
                             'max_diff_over_rms_vs_sgemm': check})
    launch.keep.clear()
    for mod in modules.values():
        drv.call('cuModuleUnload', mod)
    blas.cublasDestroy_v2(handle)
    rt.close()
    return out


def gemv_measure(torch, rt, stack):
    """M = 1 GEMV (decoder-regime kernel) against HBM bandwidth.

    ``stack``: one CUDA-graph replay of a GEMV over every packed encoder weight
    (216 launches, 642 MB > L2, so every byte comes from HBM).
    ``single``: one launch over a [32768, 8192] Q8_0 matrix (285 MB)."""
    from parakeet_cuda_b200.runtime import pack_host
    from parakeet_cuda_b200.synthetic import q8_0_blocks
    import numpy as np
    x = {k: torch.randn(1, k, device=rt.device) for k in (1024, 4096, 8192)}
    y = torch.empty(1, 32768, device=rt.device)
    for layer in stack.weights:
        for w in layer.values():
            rt.ensure_workspace(1, w.n, w.k)
    big_n, big_k = 32768, 8192
    big = rt.upload_packed(pack_host(q8_0_blocks(np.random.default_rng(5), big_n, big_k), big_n, big_k, 0,
                                     rt.lib), big_n, big_k, 0)
    rt.ensure_workspace(1, big_n, big_k)
    ws = rt.workspace

    def one(w, glu=False):
        rt.lib.call('pq8_gemv', w.pointer, x[w.k].data_ptr(), y.data_ptr(), None, None, 1, w.n, w.k,
                    3 if glu else 0, 1.0, ws.data_ptr(), ws.numel(), rt.stream())

    def sweep():
        for layer in stack.weights:
            for name, w in layer.items():
                one(w, name == 'pw1_glu')

    sweep()
    one(big)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
        sweep()
    torch.cuda.current_stream().wait_stream(side)
    peaks, src = measured_peaks()
    out = {'m': 1, 'peak_gbs': peaks['hbm_gbs'], 'peak_source': f'{src}: MEASURED_PEAKS.json hbm_gbs'}
    reps = 5
    for key, fn, nbytes in (('stack', g.replay, stack.weight_bytes), ('single', lambda: one(big), big.data.numel())):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / reps
        gbs = nbytes / (ms / 1e3) / 1e9
        out[key] = {'bytes': nbytes, 'ms': ms, 'achieved_gbs': gbs, 'frac': gbs / peaks['hbm_gbs']}
    out['stack']['launches'] = stack.launches_per_step
    out['single']['shape'] = [big_n, big_k]
    del g, big
    # the same 216 products as one pq8_gemv_batch launch
    from parakeet_cuda_b200.pq8 import GemvBatchTask
    ys = []
    tasks = []
    for layer in stack.weights:
        for name, w in layer.items():
            glu = name == 'pw1_glu'
            yt = torch.empty(1, w.n // 2 if glu else w.n, device=rt.device)
            ys.append(yt)
            tasks.append(GemvBatchTask(w.pointer, x[w.k].data_ptr(), yt.data_ptr(), None, None, w.n, w.k,
                                       3 if glu else 0, 1.0))
    plan_bytes, ws_bytes = rt.lib.gemv_batch_sizes(tasks)
    plan = torch.empty(plan_bytes, dtype=torch.uint8, device=rt.device)
    bws = torch.empty(ws_bytes, dtype=torch.uint8, device=rt.device)
    ctas = rt.lib.gemv_batch_plan(tasks, plan.data_ptr(), plan_bytes, bws.data_ptr(), ws_bytes, rt.stream())
    run = lambda: rt.lib.call('pq8_gemv_batch_run', plan.data_ptr(), ctas, rt.stream())
    run()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        run()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    gbs = stack.weight_bytes / (ms / 1e3) / 1e9
    out['stack_batch'] = {'bytes': stack.weight_bytes, 'ms': ms, 'achieved_gbs': gbs, 'frac': gbs / peaks['hbm_gbs'],
                          'launches': 1, 'ctas': ctas,
                          'api': 'pq8_gemv_batch_plan / pq8_gemv_batch_run: the 216 products in one launch'}
    return out


def tdt_measure(torch, rt, batches=(1, 64)):
    """greedy TDT loop with random weights, ~1000 decode steps per stream,
    batch 1 and batch 64 (lock-step; one joint launch for all streams per step)."""
    import time
    import numpy as np
    from parakeet_cuda_b200.decoder import PQ8Decoder
    from parakeet_cuda_b200.pq8 import EPI_NONE
    from parakeet_cuda_b200.synthetic import SyntheticParakeet
    from parakeet_cuda_b200.tdt import greedy_decode_batch, greedy_decode_device, greedy_decode_persistent
    model = SyntheticParakeet(seed=11, encoder_layers=0)
    rt.load_weights(model, ['joint.enc.weight', 'joint.enc.bias'])
    w_enc, b_enc = rt.weight('joint.enc.weight'), rt.weight('joint.enc.bias').reshape(-1)
    frames = 1150   # ~1000 joint calls per stream with these weights
    out = {'frames_per_stream': frames, 'durations': [0, 1, 2, 3, 4]}
    for batch in batches:
        enc = torch.randn(batch * frames, 1024, device=rt.device)      # encoder outputs ~ N(0, 1)
        t0 = time.perf_counter()
        projected = rt.gemm(enc, w_enc, bias=b_enc, epilogue=EPI_NONE)  # joint.enc projection (Encoder.project)
        torch.cuda.synchronize()
        t_proj = time.perf_counter() - t0
        streams_dev = list(projected.reshape(batch, frames, -1))
        streams = [p.cpu().numpy() for p in streams_dev]
        dec = PQ8Decoder(model, rt, batch=batch)
        greedy_decode_batch([s[:20] for s in streams], PQ8Decoder(model, rt, batch=batch), model.metadata['asr.tdt.durations'])
        t0 = time.perf_counter()
        res = greedy_decode_batch(streams, dec, model.metadata['asr.tdt.durations'])
        t_dec = time.perf_counter() - t0
        calls = sum(r['joint_calls'] for r in res)
        steps = dec.joint_calls
        out[f'batch{batch}'] = {'lockstep_steps': steps, 'joint_calls': calls,
                                'tokens': sum(len(r['tokens']) for r in res), 'predict_launches': dec.predict_calls,
                                'seconds': t_dec, 'steps_per_s': steps / t_dec, 'joint_calls_per_s': calls / t_dec,
                                'projection_ms': t_proj * 1e3, 'loop': 'host (reads ids every step)'}
        # the same decode with the control on the device (graph of 16 steps, host polls between replays)
        # The projections stay on the device (Encoder.project's output feeds the loop directly).
        ddev = PQ8Decoder(model, rt, batch=batch)
        greedy_decode_device([s[:20] for s in streams_dev], ddev, model.metadata['asr.tdt.durations'])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res_dev = greedy_decode_device(streams_dev, ddev, model.metadata['asr.tdt.durations'])
        t_dev = time.perf_counter() - t0
        calls_dev = sum(r['joint_calls'] for r in res_dev)
        out[f'batch{batch}_device_loop'] = {
            'lockstep_steps': ddev.steps, 'joint_calls': calls_dev,
            'loop_seconds': ddev.loop_seconds, 'steps_per_s': ddev.steps / ddev.loop_seconds,
            'joint_calls_per_s': calls_dev / ddev.loop_seconds,
            'call_seconds': t_dev, 'call_joint_calls_per_s': calls_dev / t_dev,
            'same_result_as_host_loop': res_dev == res,
            'loop': 'device (pq8_tdt_advance; CUDA graph of 16 steps, host polls the remaining count); '
                    'steps_per_s over the replay loop, call_* over the whole call (frame table, graph capture, '
                    'results to host lists)'}
        # the whole loop in one persistent launch (pq8_tdt_decode: weights resident in shared memory)
        dper = PQ8Decoder(model, rt, batch=1)
        greedy_decode_persistent([s[:20] for s in streams_dev], dper, model.metadata['asr.tdt.durations'])
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res_per = greedy_decode_persistent(streams_dev, dper, model.metadata['asr.tdt.durations'])
        t_per = time.perf_counter() - t0
        calls_per = sum(r['joint_calls'] for r in res_per)
        out[f'batch{batch}_persistent'] = {
            'lockstep_steps': dper.steps, 'joint_calls': calls_per, 'kernel_seconds': dper.loop_seconds,
            'us_per_step': dper.loop_seconds / max(dper.steps, 1) * 1e6,
            'steps_per_s': dper.steps / dper.loop_seconds, 'joint_calls_per_s': calls_per / dper.loop_seconds,
            'call_seconds': t_per, 'call_joint_calls_per_s': calls_per / t_per,
            'same_result_as_host_loop': res_per == res,
            'loop': 'device (pq8_tdt_decode: one cooperative launch for the whole decode); steps_per_s over the '
                    'launch (CUDA events), call_* over the whole call'}
    return out


def block_measure(torch, rt, args, linear_ms):
    """Whole FastConformer blocks (the rest of the block on the device): every layer of config 2's shapes with
    LayerNorms, rel-pos attention and the conv module on the device around the same Q8_0
    linears, 8 windows x 375 frames per GPU; one CUDA-graph replay per step. Random
    block-scale weights (SyntheticParakeet(block=True))."""
    from parakeet_cuda_b200.block import EncoderBlocks, EncoderStem
    from parakeet_cuda_b200.synthetic import SyntheticParakeet
    model = SyntheticParakeet(seed=5, encoder_layers=args.layers, decoder=False, block=True)
    blocks = EncoderBlocks(model, rt, args.windows_per_gpu, WINDOW_FRAMES, layers=args.layers)
    mel_frames = 8 * WINDOW_FRAMES  # 10 ms mel hop, 8x subsampling
    stem = EncoderStem(model, rt, args.windows_per_gpu, mel_frames)
    del model
    mel = torch.randn(args.windows_per_gpu, mel_frames, 128, device=rt.device)
    stem.forward(mel)
    torch.cuda.synchronize()
    sg = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(rt.device)
    side.wait_stream(torch.cuda.current_stream(rt.device))
    with torch.cuda.stream(side):
        sg.capture_begin()
        stem.forward(mel)
        sg.capture_end()
    torch.cuda.current_stream(rt.device).wait_stream(side)
    for _ in range(3):
        sg.replay()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(10):
        sg.replay()
    s1.record()
    torch.cuda.synchronize()
    stem_ms = s0.elapsed_time(s1) / 10
    del sg
    blocks.buf['x'].normal_()
    blocks.step()
    torch.cuda.synchronize()
    graph = blocks.capture()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    a.record()
    for _ in range(reps):
        graph.replay()
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / reps
    del graph
    frames = args.windows_per_gpu * WINDOW_FRAMES
    return {'layers': args.layers, 'windows': args.windows_per_gpu, 'frames_per_window': WINDOW_FRAMES,
            'ms_per_step': ms, 'frames_per_s': frames / ms * 1e3,
            'stem_ms_per_step': stem_ms, 'stem_mel_frames_per_window': mel_frames,
            'encoder_with_stem_frames_per_s': frames / (ms + stem_ms) * 1e3,
            'tflops_algorithmic': blocks.flops_per_step() / ms / 1e9,
            'linear_stack_ms_per_step': linear_ms,
            'attention': 'fused pq8 kernel on tcgen05 (FP16 operands, FP32 accumulation in tensor memory, online softmax)',
            'note': 'linear_pos once per layer on the 2T-1 positional rows, shared by all windows'}


def load_measure(torch, rt, model):
    """Weight upload: GGUF bytes -> resident packed weights.
    device_upload (measured by the caller on the full stack): pinned staging,
    async H2D, repack kernel. Here: the same for 2 layers packed on the host
    (pq8_pack_q8_0, then the packed bytes copied), the pinned H2D copy rate
    that bounds the device path, and the repack kernel alone."""
    import numpy as np
    from parakeet_cuda_b200.encoder import EncoderStack
    out = {}
    layers = min(2, len([n for n in model.tensors if n.endswith('feed_forward1.linear1.weight')]))
    host = EncoderStack(model, rt, 375, layers=layers, upload='host')
    nbytes = sum(int(np.asarray(model.raw(n)).size) for n in model.tensors
                 if n.startswith('encoder.') and any(n.startswith(f'encoder.layers.{l}.') for l in range(layers))
                 and model.tensors[n].kind == 8)
    out['host_pack_upload'] = {'layers': layers, 'seconds': host.load_seconds, 'gguf_bytes': nbytes,
                               'gbs': nbytes / host.load_seconds / 1e9}
    del host
    pinned = torch.empty(256 << 20, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(256 << 20, dtype=torch.uint8, device=rt.device)
    dst.copy_(pinned, non_blocking=True)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(4):
        dst.copy_(pinned, non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    out['pinned_h2d_gbs'] = 4 * pinned.numel() / (a.elapsed_time(b) / 1e3) / 1e9
    # the repack kernel alone: FFN up weight (4096 x 1024), device to device
    n, k = 4096, 1024
    raw = torch.from_numpy(np.asarray(model.raw('encoder.layers.0.feed_forward1.linear1.weight')).copy()).to(rt.device)
    packed = torch.empty(rt.lib.packed_size(n, k, 0), dtype=torch.uint8, device=rt.device)
    for _ in range(3):
        rt.lib.call('pq8_pack_q8_0_device', raw.data_ptr(), n, k, 0, packed.data_ptr(), rt.stream())
    torch.cuda.synchronize()
    reps = 50
    a.record()
    for _ in range(reps):
        rt.lib.call('pq8_pack_q8_0_device', raw.data_ptr(), n, k, 0, packed.data_ptr(), rt.stream())
    b.record()
    torch.cuda.synchronize()
    us = a.elapsed_time(b) * 1e3 / reps
    moved = raw.numel() + packed.numel()
    out['repack_kernel'] = {'shape': [n, k], 'us': us, 'bytes_moved': moved, 'gbs': moved / us / 1e3,
                            'note': 'reads the 34-byte blocks, writes the 4352-byte records; L2-resident at this size'}
    return out


SWEEP_SHAPES = ((1024, 1024), (4096, 1024), (1024, 4096), (2560, 640), (8197, 640))
SWEEP_M = (1, 16, 128, 1024, 8192, 65536)


def shard_rows(m, rank, world):
    """This rank's contiguous, balanced share of m rows: (first row, count)."""
    start = m * rank // world
    return start, m * (rank + 1) // world - start


def sweep_local(rank, world, time_point):
    """BASELINE config 4, M-sharded: for every (N, K) and M, this rank times its
    share of the M rows with ``time_point(n, k, rows) -> seconds`` (no work and
    0 s for an empty share). The points come in the same order on every rank."""
    out = []
    for n, k in SWEEP_SHAPES:
        for m in SWEEP_M:
            _, rows = shard_rows(m, rank, world)
            out.append({'m': m, 'n': n, 'k': k, 'rows': rows, 's': time_point(n, k, rows) if rows else 0.0})
    return out


def merge_sweep(parts, peaks):
    """Whole-job sweep from every rank's ``sweep_local`` points: a point takes as
    long as its slowest rank. Roofline of a point = the larger of its FLOPs over
    the active GPUs' TF32 peak and its bytes (each active GPU reads the whole
    Q8_0 matrix, 1.0625 N K, plus its rows of X and Y) over their HBM
    bandwidth; AI = FLOPs / bytes."""
    p_tf32, bw = peaks['bf16_tflops'] / 2 * 1e12, peaks['hbm_gbs'] * 1e9  # 10-launch points: burst peak
    res = []
    for pts in zip(*parts):
        m, n, k = pts[0]['m'], pts[0]['n'], pts[0]['k']
        gpus = sum(1 for p in pts if p['rows'])
        s_ = max(p['s'] for p in pts)
        if gpus == 0 or s_ <= 0:  # no rank had rows (only when some ranks' points are missing)
            res.append({'m': m, 'n': n, 'k': k, 'gpus': gpus, 'us': None})
            continue
        flops = 2 * m * n * k
        nbytes = gpus * 1.0625 * n * k + 4 * m * k + 4 * m * n
        t_tensor, t_hbm = flops / (gpus * p_tf32), nbytes / (gpus * bw)
        res.append({'m': m, 'n': n, 'k': k, 'gpus': gpus, 'us': s_ * 1e6, 'tflops': flops / s_ / 1e12,
                    'gbs': nbytes / s_ / 1e9, 'frac_of_roofline': max(t_tensor, t_hbm) / s_,
                    'bound': 'hbm' if t_hbm > t_tensor else 'tensor'})
    return res


def sweep_measure(torch, rt, rank=0, world=1):
    """This rank's config-4 points through pq8_linear, each timed as a CUDA graph
    of back-to-back launches (the reference's own graph method,
    analysis/benchmark_dense.py:47-63: launch overhead out of the figure), best
    of 3 replays. Where the Q8_0 matrix would stay in the 126 MB L2 between
    launches, the launches rotate over copies of it totalling >= 256 MB, so
    every launch streams its weights from HBM. ``merge_sweep`` combines the
    ranks."""
    import dataclasses
    import numpy as np
    from parakeet_cuda_b200.synthetic import q8_0_blocks
    weights = {}

    def time_point(n, k, rows):
        if (n, k) not in weights:
            weights.clear()
            torch.cuda.empty_cache()
            w0 = rt.pack(q8_0_blocks(np.random.default_rng(n + k), n, k), n, k)
            nbytes = w0.data.numel()
            copies = [w0] + [dataclasses.replace(w0, data=w0.data.clone())
                             for _ in range(min(255, -(-(256 << 20) // nbytes) - 1))]
            weights[(n, k)] = copies
        ws = weights[(n, k)]
        x = torch.randn(rows, k, device=rt.device)
        y = torch.empty(rows, n, device=rt.device)
        rt.linear(x, ws[0], out=y)  # workspace sized outside the capture
        torch.cuda.synchronize()
        reps = max(10, len(ws)) if rows <= 1024 else 4
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(rt.device)
        side.wait_stream(torch.cuda.current_stream(rt.device))
        with torch.cuda.stream(side):
            g.capture_begin()
            for i in range(reps):
                rt.linear(x, ws[i % len(ws)], out=y)
            g.capture_end()
        torch.cuda.current_stream(rt.device).wait_stream(side)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = float('inf')
        for _ in range(3):
            a.record()
            g.replay()
            b.record()
            torch.cuda.synchronize()
            best = min(best, a.elapsed_time(b) / reps / 1e3)
        del g
        return best

    return sweep_local(rank, world, time_point)


def upload_raw_layers(torch, model, layers, dev):
    """Raw GGUF Q8_0 bytes of every encoder linear on the device (Q, K, V stacked along N)."""
    import numpy as np
    from parakeet_cuda_b200.encoder import LAYER_PLAN
    raw = []
    for l in range(layers):
        base = f'encoder.layers.{l}.'
        raw.append({name: torch.from_numpy(np.concatenate(
            [np.asarray(model.raw(base + key + '.weight'), np.uint8).reshape(-1) for key in keys])).to(dev)
            for name, keys, *_ in LAYER_PLAN})
    return raw


def reference_gpu_method(torch, rt, raw, stack, steps=3):
    """Context, not the product: config 2 by the reference's GPU method on this B200,
    restated with library calls on the same shapes and buffers as the timed step.
    For every layer (``encoder.py:204``, ``gpu.py:169-184``) each Q8_0 weight of
    the layer is expanded to FP32 (``pq8_dequant_q8_0``, bit-identical to
    ``dequant_q8``, ``runtime.cu:26-33``), each linear is one cuBLAS GEMM on the
    FP32 weights (``torch.mm``; TF32 off is the reference's ``cublasSgemm_v2``,
    ``gpu.py:87-90``) and each epilogue a separate elementwise pass
    (``runtime.cu:49-62``). Timed again with TF32 allowed: a library TF32 port of
    the same method. Both are captured in CUDA graphs (no host launch cost)."""
    from parakeet_cuda_b200.encoder import LAYER_PLAN
    from parakeet_cuda_b200.pq8 import EPI_GLU, EPI_RESIDUAL, EPI_SILU
    dev = rt.device
    rows = stack.rows
    b = stack.buffers
    wf = {name: torch.empty(n, k, device=dev) for name, _, n, k, *_ in LAYER_PLAN}
    y = {name: torch.empty(rows, n, device=dev) for name, _, n, _, epi, *_ in LAYER_PLAN
         if epi in (EPI_RESIDUAL, EPI_GLU)}
    sig = torch.empty(rows, LAYER_PLAN[5][2] // 2, device=dev)

    def step():
        for layer in raw:
            for name, _, n, k, *_ in LAYER_PLAN:  # the whole layer is expanded first, as gpu.py does
                rt.lib.call('pq8_dequant_q8_0', layer[name].data_ptr(), wf[name].data_ptr(), n * k, rt.stream())
            for name, _, n, k, epi, alpha, src, dst, _ in LAYER_PLAN:
                if epi == EPI_RESIDUAL:  # x += alpha * y
                    torch.mm(b[src], wf[name].t(), out=y[name])
                    b[dst].add_(y[name], alpha=alpha)
                elif epi == EPI_GLU:     # a * sigmoid(b) over the two halves of N
                    torch.mm(b[src], wf[name].t(), out=y[name])
                    half = n // 2
                    torch.sigmoid(y[name][:, half:], out=sig)
                    torch.mul(y[name][:, :half], sig, out=b[dst])
                else:                    # written in place, SiLU applied over it
                    torch.mm(b[src], wf[name].t(), out=b[dst])
                    if epi == EPI_SILU:
                        torch.nn.functional.silu(b[dst], inplace=True)

    res = {'method': 'pq8_dequant_q8_0 per layer + torch.mm (cuBLAS) per linear + elementwise epilogues',
           'layers': len(raw), 'rows': rows, 'steps': steps}
    flops = stack.flops_per_step()
    for key, tf32 in (('fp32_sgemm', False), ('tf32', True)):
        torch.backends.cuda.matmul.allow_tf32 = tf32
        step()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.cuda.graph(g, stream=side):
            step()
        torch.cuda.current_stream(dev).wait_stream(side)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        res[key] = {'ms_per_step': ms, 'frames_per_s': rows / (ms / 1e3), 'tflops': flops / (ms / 1e3) / 1e12}
        del g
    torch.backends.cuda.matmul.allow_tf32 = False
    return res


def cublas_tf32(torch):
    """Context only: cuBLAS FP32 GEMM with TF32 tensor cores, 8192^3, best of 5."""
    torch.backends.cuda.matmul.allow_tf32 = True
    a = torch.randn(8192, 8192, device='cuda')
    b = torch.randn(8192, 8192, device='cuda')
    best = None
    for _ in range(6):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.matmul(a, b)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1)
        best = t if best is None else min(best, t)
    torch.backends.cuda.matmul.allow_tf32 = False
    return 2 * 8192 ** 3 / (best / 1e3) / 1e12


def main():
    args = parse()
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == '__main__':
    main()
