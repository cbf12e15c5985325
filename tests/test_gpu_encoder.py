"""The encoder GEMM stack as the benchmark runs it: chains of dependent GEMMs.

Consecutive GEMMs are launched with programmatic dependent launch, so a
kernel starts (set-up, weight fetch and conversion) while its predecessor is
still running and waits for it only before reading activations or writing
outputs. Every kernel here is deterministic, so a graph replay, plain stream
launches and launches separated by a device synchronization must produce the
same bits; a GEMM that touched its input or output too early would not.
The numerics of each linear against the oracle are covered in
test_gpu_linear.py.
"""
import pytest
import torch

from parakeet_cuda_b200.encoder import LAYER_PLAN, EncoderStack
from parakeet_cuda_b200.runtime import Runtime
from parakeet_cuda_b200.synthetic import SyntheticParakeet

pytestmark = pytest.mark.gpu


def snapshot(stack):
    return {k: v.clone() for k, v in stack.buffers.items()}


def run(stack, mode, graph=None):
    stack.buffers['resid'].zero_()
    if mode == 'graph':
        graph.replay()
    elif mode == 'stream':
        stack.step()
    else:
        for layer in range(stack.layers):
            for entry in LAYER_PLAN:
                stack.launch(layer, entry)
                torch.cuda.synchronize()
    torch.cuda.synchronize()
    return snapshot(stack)


@pytest.mark.parametrize('rows', [750, 3000])
def test_dependent_gemm_chains_are_exact(rows):
    rt = Runtime(0)
    stack = EncoderStack(SyntheticParakeet(seed=5, encoder_layers=2, decoder=False), rt, rows, layers=2, seed=2)
    want = run(stack, 'serial')
    got_stream = run(stack, 'stream')
    graph = stack.capture()
    for _ in range(3):
        got_graph = run(stack, 'graph', graph)
        for name in want:
            assert torch.equal(got_graph[name], want[name]), name
    for name in want:
        assert torch.equal(got_stream[name], want[name]), name
    assert want['resid'].abs().max().item() > 0
    del graph
    assert rt.device_status() == 0


@pytest.mark.parametrize('use_graph', [True, False])
def test_pipelined_host_steps_match_serial(use_graph):
    """run_host_pipelined overlaps each step's copies with its neighbours'
    compute through two staging buffers per direction; with five distinct
    inputs (more steps than buffers) every result must equal a plain run_host
    of the same input, bit for bit."""
    rt = Runtime(0)
    rows = 750
    stack = EncoderStack(SyntheticParakeet(seed=6, encoder_layers=2, decoder=False), rt, rows, layers=2, seed=3)
    graph = stack.capture() if use_graph else None
    g = torch.Generator().manual_seed(11)
    inputs = [torch.randn(rows, 1024, generator=g).pin_memory() for _ in range(5)]
    want = []
    for x in inputs:
        out = torch.empty(rows, 1024).pin_memory()
        stack.run_host(x, out, graph)
        torch.cuda.synchronize()
        want.append(out.clone())
    for _ in range(2):  # the second call reuses the staging buffers
        outputs = [torch.full((rows, 1024), float('nan')).pin_memory() for _ in inputs]
        stack.run_host_pipelined(inputs, outputs, graph)
        torch.cuda.synchronize()
        for i, (got, exp) in enumerate(zip(outputs, want)):
            assert torch.equal(got, exp), i
    assert not torch.equal(want[0], want[1])
    del graph
    assert rt.device_status() == 0
