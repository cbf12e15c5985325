"""GEMM sequences (pq8_sequence_plan / pq8_sequence_run): many GEMMs as one
persistent launch, each CTA running its list of the plan's tile schedule and
each tile waiting only for the row blocks it depends on.

Every tile runs the same single-CTA BN = 192 kernel configuration as
pq8_gemm with PQ8_GEMM_CONFIG=1, so a sequence must reproduce those launches
bit for bit; a missing dependency would let a tile read rows before they are
written (or overwrite rows still being read) and show up as a difference.
"""
import numpy as np
import pytest

from parakeet_cuda_b200 import pq8
from parakeet_cuda_b200.cuda_driver import Event
from parakeet_cuda_b200.host import EncoderStackHost, HostRuntime
from parakeet_cuda_b200.layers import LAYER_PLAN
from parakeet_cuda_b200.synthetic import SyntheticParakeet, q8_0_blocks

pytestmark = pytest.mark.gpu

BN192 = '1'  # PQ8_GEMM_CONFIG index of the single-CTA BN = 192 configuration


@pytest.fixture(scope='module')
def hrt():
    rt = HostRuntime(0)
    yield rt
    rt.close()


def snapshot(rt, stack):
    return {k: rt.download(v) for k, v in stack.buffers.items()}


@pytest.mark.parametrize('rows', [750, 3000])
def test_stack_sequence_equals_per_linear_launches(hrt, rows, monkeypatch):
    model = SyntheticParakeet(seed=21, encoder_layers=2, decoder=False)
    stack = EncoderStackHost(model, hrt, rows, layers=2, seed=3)
    resid = stack.buffers['resid']
    monkeypatch.setenv('PQ8_GEMM_CONFIG', BN192)
    hrt.drv.memset(resid.pointer, 0, resid.nbytes, hrt.stream)
    stack.step()
    hrt.synchronize()
    want = snapshot(hrt, stack)
    monkeypatch.delenv('PQ8_GEMM_CONFIG')
    layer_order = tuple(entry[0] for entry in LAYER_PLAN)
    # the plan's list schedule (default), and the strided assignment in the layer's own order
    for deps, schedule, order in (('model', None, None), ('buffers', None, None), ('model', 'strided', layer_order)):
        if schedule:
            monkeypatch.setenv('PQ8_SEQUENCE_SCHEDULE', schedule)
        stack.make_sequence(deps, order=order)
        monkeypatch.delenv('PQ8_SEQUENCE_SCHEDULE', raising=False)
        for _ in range(2):  # the second run finds the counters reset by the first
            hrt.drv.memset(resid.pointer, 0, resid.nbytes, hrt.stream)
            stack.step_sequence()
            hrt.synchronize()
            got = snapshot(hrt, stack)
            for name in want:
                np.testing.assert_array_equal(got[name], want[name], err_msg=f'{deps} {schedule} {name}')
    stack.make_sequence('model')
    graph = stack.capture(sequence=True)
    for _ in range(3):
        hrt.drv.memset(resid.pointer, 0, resid.nbytes, hrt.stream)
        graph.launch(hrt.stream)
        hrt.synchronize()
        np.testing.assert_array_equal(hrt.download(resid), want['resid'])
    graph.close()
    stack.close()
    assert hrt.device_status() == 0


def test_chain_of_dependent_gemms(hrt, monkeypatch):
    """y1 = x W1, y2 = y1 W2 (+ residual into y1's rows later), ...: each task
    reads rows the previous task writes, with shapes whose tile counts differ
    (rows not a multiple of 192, N not a multiple of 128, GLU in between)."""
    rng = np.random.default_rng(5)
    m = 1000
    up = hrt.uploader()
    shapes = [(640, 256, pq8.EPI_SILU), (256, 640, pq8.EPI_NONE), (512, 256, pq8.EPI_GLU), (256, 256, pq8.EPI_RESIDUAL),
              (384, 256, pq8.EPI_RELU)]
    x = hrt.upload(rng.standard_normal((m, 256), np.float32))
    bufs = [x]
    tasks = []
    for i, (n, k, epi) in enumerate(shapes):
        w = up.pack_rows([q8_0_blocks(rng, n, k, 2e-3, 8e-3)], n, k, pq8.LAYOUT_GLU if epi == pq8.EPI_GLU else 0)
        out_cols = n // 2 if epi == pq8.EPI_GLU else n
        if epi == pq8.EPI_RESIDUAL:
            y = bufs[-2]  # accumulate into the rows the task before last wrote, which this task's x came from
        else:
            y = hrt.work.alloc((m, out_cols))
        bias = hrt.upload(rng.standard_normal(n).astype(np.float32))
        tasks.append(pq8.GemmTask(w.pointer, bufs[-1].pointer, y.pointer, bias.pointer,
                                  y.pointer if epi == pq8.EPI_RESIDUAL else None, m, n, k, epi, 0.5,
                                  pq8.FLAG_OUT_TF32, -1, 0))
        bufs.append(y)
    up.finish()
    # x of task 4 is task 3's y (= task 1's output): every rewrite must be ordered
    assert tasks[3].y == tasks[1].y
    outs = sorted({t.y for t in tasks})
    by_ptr = {b.pointer: b for b in bufs}

    def run_launches():
        for t in tasks:
            hrt.lib.call('pq8_gemm', t.w, t.x, t.y, t.bias, t.resid, t.m, t.n, t.k, t.epilogue, t.alpha, t.flags,
                         hrt.stream.handle)
        hrt.synchronize()
        return {p: hrt.download(by_ptr[p]) for p in outs}

    monkeypatch.setenv('PQ8_GEMM_CONFIG', BN192)
    want = run_launches()
    monkeypatch.delenv('PQ8_GEMM_CONFIG')
    plan_bytes = hrt.lib.sequence_plan_size(tasks)
    plan = hrt.work.alloc(plan_bytes, np.uint8)
    hrt.lib.sequence_plan(tasks, plan.pointer, plan.nbytes, hrt.stream.handle)
    for _ in range(3):
        for p in outs:  # poison the outputs
            hrt.drv.memset(p, 0xFF, by_ptr[p].nbytes, hrt.stream)
        hrt.lib.call('pq8_sequence_run', plan.pointer, hrt.stream.handle)
        hrt.synchronize()
        for p in outs:
            np.testing.assert_array_equal(hrt.download(by_ptr[p]), want[p])
    assert hrt.device_status() == 0


def test_sequence_plan_rejections(hrt):
    rng = np.random.default_rng(6)
    up = hrt.uploader()
    w = up.pack_rows([q8_0_blocks(rng, 256, 256)], 256, 256)
    up.finish()
    x = hrt.work.alloc((400, 256))
    y = hrt.work.alloc((400, 256))
    plan = hrt.work.alloc(1 << 20, np.uint8)
    ok = pq8.GemmTask(w.pointer, x.pointer, y.pointer, None, None, 400, 256, 256, 0, 1.0, 0, -1, 0)

    def plan_of(tasks):
        hrt.lib.sequence_plan(tasks, plan.pointer, plan.nbytes, hrt.stream.handle)

    plan_of([ok])
    # a second task reading y shifted by one row: overlapping rows that do not line up
    shifted = pq8.GemmTask(w.pointer, y.pointer + 1024, x.pointer, None, None, 300, 256, 256, 0, 1.0, 0, -1, 0)
    with pytest.raises(pq8.PQ8Error) as e:
        plan_of([ok, shifted])
    assert e.value.code == pq8.ERR_UNSUPPORTED_SHAPE
    # `after` must name an earlier task
    with pytest.raises(pq8.PQ8Error) as e:
        plan_of([pq8.GemmTask(w.pointer, x.pointer, y.pointer, None, None, 400, 256, 256, 0, 1.0, 0, 0, 0)])
    assert e.value.code == pq8.ERR_INVALID_ARGUMENT
    # packed for another shape
    x2 = hrt.work.alloc((400, 512))
    with pytest.raises(pq8.PQ8Error) as e:
        plan_of([pq8.GemmTask(w.pointer, x2.pointer, y.pointer, None, None, 400, 128, 512, 0, 1.0, 0, -1, 0)])
    assert e.value.code == pq8.ERR_LAYOUT
    # in place (x = y)
    with pytest.raises(pq8.PQ8Error) as e:
        plan_of([pq8.GemmTask(w.pointer, x.pointer, x.pointer, None, None, 400, 256, 256, 0, 1.0, 0, -1, 0)])
    assert e.value.code == pq8.ERR_UNSUPPORTED_SHAPE
    with pytest.raises(pq8.PQ8Error) as e:
        hrt.lib.sequence_plan([ok], plan.pointer, 64, hrt.stream.handle)
    assert e.value.code == pq8.ERR_WORKSPACE
    assert hrt.device_status() == 0
