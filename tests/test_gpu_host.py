"""The torch-free host layer on the GPU: EncoderStackHost (driver-API memory,
cuStreamBeginCapture graphs, page-locked copies) runs the same launches as the
PyTorch-hosted EncoderStack, so every buffer must agree bit for bit, and its
pipelined end-to-end call must equal one run_host per step."""
import numpy as np
import pytest
import torch

from parakeet_cuda_b200.cuda_driver import PinnedArray
from parakeet_cuda_b200.encoder import EncoderStack
from parakeet_cuda_b200.host import EncoderStackHost, HostRuntime
from parakeet_cuda_b200.runtime import Runtime
from parakeet_cuda_b200.synthetic import SyntheticParakeet

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def setup():
    model = SyntheticParakeet(seed=5, encoder_layers=2, decoder=False)
    rows = 750
    ref = EncoderStack(model, Runtime(0), rows, layers=2, seed=2)
    standins = {k: ref.buffers[k].cpu().numpy() for k in ('norm', 'ctx', 'pos')}
    hrt = HostRuntime(0)
    host = EncoderStackHost(model, hrt, rows, layers=2, standins=standins)
    yield ref, hrt, host
    host.close()
    hrt.close()


def test_host_stack_equals_torch_stack(setup):
    ref, hrt, host = setup
    ref.buffers['resid'].zero_()
    ref.step()
    torch.cuda.synchronize()
    hrt.drv.memset(host.buffers['resid'].pointer, 0, host.buffers['resid'].nbytes, hrt.stream)
    host.step()
    hrt.synchronize()
    for name, t in ref.buffers.items():
        np.testing.assert_array_equal(hrt.download(host.buffers[name]), t.cpu().numpy(), err_msg=name)
    graph = host.capture()
    hrt.drv.memset(host.buffers['resid'].pointer, 0, host.buffers['resid'].nbytes, hrt.stream)
    graph.launch(hrt.stream)
    hrt.synchronize()
    np.testing.assert_array_equal(hrt.download(host.buffers['resid']), ref.buffers['resid'].cpu().numpy())
    graph.close()
    assert hrt.device_status() == 0


@pytest.mark.parametrize('use_graph', [True, False])
def test_host_pipelined_equals_run_host(setup, use_graph):
    ref, hrt, host = setup
    graph = host.capture() if use_graph else None
    rng = np.random.default_rng(4)
    inputs = []
    for _ in range(5):
        a = PinnedArray(hrt.drv, (host.rows, 1024))
        a.array[...] = rng.standard_normal((host.rows, 1024), np.float32)
        inputs.append(a)
    want = []
    for x in inputs:
        out = PinnedArray(hrt.drv, (host.rows, 1024))
        host.run_host(x, out, graph)
        hrt.synchronize()
        want.append(out.array.copy())
        out.close()
    # the torch-hosted public call on the same input gives the same result
    x0 = torch.from_numpy(inputs[0].array.copy()).pin_memory()
    o0 = torch.empty(host.rows, 1024).pin_memory()
    ref.run_host(x0, o0)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(o0.numpy(), want[0])
    for _ in range(2):  # the second call reuses the staging buffers
        outs = [PinnedArray(hrt.drv, (host.rows, 1024)) for _ in inputs]
        for o in outs:
            o.array[...] = np.nan
        host.run_host_pipelined(inputs, outs, graph)
        hrt.synchronize()
        for i, (o, w) in enumerate(zip(outs, want)):
            np.testing.assert_array_equal(o.array, w, err_msg=str(i))
        for o in outs:
            o.close()
    assert not np.array_equal(want[0], want[1])
    for a in inputs:
        a.close()
    if graph is not None:
        graph.close()
    assert hrt.device_status() == 0
