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
import numpy as np
import pytest
import torch

from oracle import q8
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


def test_chained_stack_rows_match_float64_chain():
    """Two layers of the config-2 stack (3000 rows, every linear with its fused
    epilogue, the residual stream carried through 8 residual updates): sampled
    rows of every output against the same chain in float64 from the decoded
    Q8_0 weights and the stack's own stand-in inputs. North-star bar on each
    output, max |err| <= 2e-3 x RMS (the GLU output through its first-order
    bound, the SiLU hidden state with SiLU's Lipschitz factor 1.1). The hidden
    state and the GLU output are written TF32-rounded for the next GEMM
    (PQ8_FLAG_OUT_TF32), which adds up to half a TF32 ulp, 2^-11 |y|, per
    element on top of the bar."""
    rt = Runtime(0)
    model = SyntheticParakeet(seed=7, encoder_layers=2, decoder=False)
    rows, layers = 3000, 2
    stack = EncoderStack(model, rt, rows, layers=layers, seed=4)
    stack.buffers['resid'].zero_()
    stack.step()
    torch.cuda.synchronize()
    got = {k: v.cpu().numpy() for k, v in stack.buffers.items()}
    pick = np.random.default_rng(3000).choice(rows, 48, replace=False)
    norm, ctx, pos = (got[k][pick].astype(np.float64) for k in ('norm', 'ctx', 'pos'))
    weights = {}
    for name, keys, n, k, *_ in LAYER_PLAN:
        for l in range(layers):
            parts = [q8.decode(model.raw(f'encoder.layers.{l}.{key}.weight'), n // len(keys), k) for key in keys]
            weights[l, name] = np.concatenate(parts)
    silu = lambda z: z * q8.sigmoid(z)
    x = np.zeros((len(pick), 1024))
    for l in range(layers):
        w = lambda name: weights[l, name]
        h1 = silu(norm @ w('ffn1_up').T)
        x = x + 0.5 * (h1 @ w('ffn1_down').T)
        qkv = norm @ w('qkv').T
        pos_out = pos @ w('pos').T
        x = x + ctx @ w('out').T
        z = norm @ w('pw1_glu').T
        gate = z[:, :1024] * q8.sigmoid(z[:, 1024:])
        x = x + gate @ w('pw2').T
        h2 = silu(norm @ w('ffn2_up').T)
        x = x + 0.5 * (h2 @ w('ffn2_down').T)
    ulp = 2.0 ** -11
    errs = {'resid': q8.max_err_over_rms(got['resid'][pick], x),
            'qkv': q8.max_err_over_rms(got['qkv'][pick], qkv),
            'pos_out': q8.max_err_over_rms(got['pos_out'][pick], pos_out)}
    z_up = norm @ weights[layers - 1, 'ffn2_up'].T
    bound = 1.1 * 2e-3 * q8.rms(z_up) + ulp * np.abs(h2)
    errs['hidden (x bound)'] = float(np.max(np.abs(got['hidden'][pick] - h2) / bound)) * 2e-3
    s = q8.sigmoid(z[:, 1024:])
    bound = 1.05 * 2e-3 * q8.rms(z) * (s + np.abs(z[:, :1024]) * s * (1 - s)) + ulp * np.abs(gate) + 1e-9 * q8.rms(z)
    errs['gate (x bound)'] = float(np.max(np.abs(got['gate'][pick] - gate) / bound)) * 2e-3
    print({k: f'{v:.2e}' for k, v in errs.items()})
    for name, e in errs.items():
        assert e <= 2e-3, (name, e)
    assert rt.device_status() == 0
