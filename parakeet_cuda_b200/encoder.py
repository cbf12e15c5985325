"""FastConformer encoder GEMM stack on resident packed Q8_0 weights (encoder regime).

Each encoder layer of the reference issues these Q8_0 linears
(``parakeet_cuda/encoder.py``; all ``use_bias=False``, ``gguf.py:91``):

====================  ==============  =========================================
linear                shape (N x K)   reference epilogue (call site)
====================  ==============  =========================================
FFN1 linear1          4096 x 1024     + SiLU            (``encoder.py:31-33``)
FFN1 linear2          1024 x 4096     x += 0.5 * y      (``encoder.py:34-35``)
Q/K/V (packed)        3072 x 1024     -                 (``encoder.py:75-84``)
linear_pos            1024 x 1024     -                 (``encoder.py:103``)
linear_out            1024 x 1024     x += y            (``encoder.py:111-112``)
pointwise_conv1       2048 x 1024     GLU -> 1024       (``encoder.py:117-119``)
pointwise_conv2       1024 x 1024     x += y            (``encoder.py:125-126``)
FFN2 linear1/linear2  as FFN1         as FFN1           (``encoder.py:132``)
====================  ==============  =========================================

Here every epilogue is fused into the GEMM launch (the reference runs one
SGEMM plus one elementwise kernel per linear, after a ``dequant_q8`` of the
layer). LayerNorm, attention, the depthwise convolution and the stem are not
part of the contraction path: their outputs are represented by fixed input
buffers (``norm`` for every LayerNorm output, ``ctx`` for the attention
context, ``pos`` for the positional embeddings), so the stack performs
exactly the linears of the encoder on realistic shapes. Intermediate
activations that feed another GEMM (FFN hidden, GLU output) are written
TF32-rounded and consumed without re-rounding (``PQ8_FLAG_OUT_TF32`` /
``PQ8_FLAG_X_TF32``), which is value-identical to rounding them in the
consumer.

Config 1 of the benchmark is one layer at T = 375 frames; config 2 is 24
layers over ``windows x 375`` rows, with windows independent (``recording.py``
segments) so that rows from several windows share one launch.
"""
from __future__ import annotations

import time

import numpy as np
import torch

from .layers import D_FF, D_MODEL, FRAMES_PER_WINDOW, LAYER_PLAN, flops_per_row_per_layer  # noqa: F401
from .pq8 import EPI_GLU, EPI_RESIDUAL, FLAG_X_TF32, LAYOUT_GLU
from .runtime import PackedWeight, Runtime, pack_host

class EncoderStack:
    """All Q8_0 linears of ``layers`` encoder layers over ``rows`` activation rows on one device."""

    def __init__(self, model, runtime: Runtime, rows: int, layers: int = 24, seed: int = 0,
                 producer_tf32: bool = True, upload: str = 'device'):
        """``producer_tf32``: the GEMM inputs that come from outside the contraction path
        (LayerNorm outputs, attention context, positional table) are produced TF32-rounded,
        as a fused producer would write them, and every GEMM skips its rounding pass.
        With False, those GEMMs round their input tile in shared memory themselves.
        ``upload``: 'device' copies the GGUF bytes and repacks them on the GPU
        (``WeightUploader``); 'host' packs on the host and copies the packed bytes
        (the same result, kept to measure the difference)."""
        self.rt, self.rows, self.layers = runtime, rows, layers
        self.producer_tf32 = producer_tf32
        dev = runtime.device
        self.weights: list[dict[str, PackedWeight]] = []
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        up = runtime.uploader()
        for l in range(layers):
            base = f'encoder.layers.{l}.'
            packed = {}
            for name, keys, n, k, epi, _, _, _, _ in LAYER_PLAN:
                raws = [model.raw(base + key + '.weight') for key in keys]
                layout = LAYOUT_GLU if epi == EPI_GLU else 0
                if upload == 'device':
                    packed[name] = up.pack_rows(raws, n, k, layout)
                else:
                    raw = np.concatenate([np.asarray(r, np.uint8).reshape(-1) for r in raws])
                    packed[name] = runtime.upload_packed(pack_host(raw, n, k, layout, runtime.lib), n, k, layout)
            self.weights.append(packed)
        up.finish()
        torch.cuda.synchronize(dev)
        self.load_seconds = time.perf_counter() - t0
        self.weight_bytes = sum(w.data.numel() for layer in self.weights for w in layer.values())
        g = torch.Generator(device='cpu').manual_seed(seed)
        f32 = dict(dtype=torch.float32, device=dev)
        self.buffers = {
            'norm': torch.randn(rows, D_MODEL, generator=g).to(dev),
            'ctx': torch.randn(rows, D_MODEL, generator=g).to(dev),
            'pos': torch.randn(rows, D_MODEL, generator=g).to(dev),
            'resid': torch.zeros(rows, D_MODEL, **f32),
            'hidden': torch.empty(rows, D_FF, **f32),
            'qkv': torch.empty(rows, 3 * D_MODEL, **f32),
            'pos_out': torch.empty(rows, D_MODEL, **f32),
            'gate': torch.empty(rows, D_MODEL, **f32),
        }
        if producer_tf32:
            for name in ('norm', 'ctx', 'pos'):
                self.round_buffer(name)

    @property
    def launches_per_step(self) -> int:
        return self.layers * len(LAYER_PLAN)

    def flops_per_step(self) -> int:
        return self.rows * self.layers * flops_per_row_per_layer()

    def round_buffer(self, name: str) -> None:
        t = self.buffers[name]
        self.rt.lib.call('pq8_round_tf32', t.data_ptr(), t.numel(), self.rt.stream())

    def launch(self, layer: int, entry) -> None:
        name, _, n, k, epi, alpha, src, dst, flags = entry
        w = self.weights[layer][name]
        b = self.buffers
        resid = b['resid'] if epi == EPI_RESIDUAL else None
        if self.producer_tf32:
            flags |= FLAG_X_TF32
        self.rt.gemm(b[src], w, out=b[dst], resid=resid, epilogue=epi, alpha=alpha, flags=flags)

    def step(self, timer=None) -> None:
        """Enqueue every linear of every layer on the current stream."""
        for l in range(self.layers):
            for entry in LAYER_PLAN:
                if timer is not None:
                    timer.start(entry[0])
                self.launch(l, entry)
                if timer is not None:
                    timer.stop(entry[0])

    def capture(self) -> torch.cuda.CUDAGraph:
        """Record one step (every launch of ``step``) as a CUDA graph on a side stream.

        Replaying it removes the host's per-launch cost (argument checks, tensor-map
        encoding, ctypes) from the critical path; the launches and their arguments
        are identical. Call ``step`` once before capturing so that per-device state
        (kernel attributes) is initialised outside the capture."""
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.rt.device)
        side.wait_stream(torch.cuda.current_stream(self.rt.device))
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                self.step()
        torch.cuda.current_stream(self.rt.device).wait_stream(side)
        return graph

    def run_host(self, x_host: torch.Tensor, out_host: torch.Tensor, graph=None) -> torch.Tensor:
        """Public end-to-end call on host buffers (pinned for asynchronous copies):
        ``x_host`` [rows, 1024] is the windows' encoder input, which starts the
        residual stream and stands in for every LayerNorm output; the final
        residual stream is copied back into ``out_host``. All work is on the
        current stream; the caller synchronizes."""
        self.buffers['norm'].copy_(x_host, non_blocking=True)
        self.buffers['resid'].copy_(self.buffers['norm'], non_blocking=True)
        if self.producer_tf32:
            self.round_buffer('norm')
        if graph is not None:
            graph.replay()
        else:
            self.step()
        out_host.copy_(self.buffers['resid'], non_blocking=True)
        return out_host

    def run_host_pipelined(self, inputs, outputs, graph=None):
        """One step per (``inputs[i]``, ``outputs[i]``) pair of pinned host buffers,
        as ``run_host`` does for each, with the copies overlapped: step i+1's
        host-to-device copy and step i-1's device-to-host copy run on two copy
        streams while step i computes. Two device staging buffers per direction
        decouple the copies from the step's own buffers (a device-to-device copy
        at each end of the step). Every step still moves its whole input and
        result across PCIe; only the waiting is gone. Returns ``outputs``; the
        current stream waits for the last copy, so the caller synchronizes as
        for ``run_host``."""
        if len(inputs) != len(outputs):
            raise ValueError('inputs and outputs must pair up')
        dev = self.rt.device
        compute = torch.cuda.current_stream(dev)
        if not hasattr(self, '_pipe'):
            shape = self.buffers['resid'].shape
            self._pipe = {
                'h2d': torch.cuda.Stream(dev), 'd2h': torch.cuda.Stream(dev),
                'in': [torch.empty(shape, dtype=torch.float32, device=dev) for _ in range(2)],
                'out': [torch.empty(shape, dtype=torch.float32, device=dev) for _ in range(2)],
            }
        pipe = self._pipe
        h2d, d2h = pipe['h2d'], pipe['d2h']
        ev = {name: [torch.cuda.Event() for _ in range(2)]
              for name in ('in_ready', 'in_free', 'out_ready', 'out_free')}
        used = [False, False]
        h2d.wait_stream(compute)
        d2h.wait_stream(compute)
        for i, (x_host, out_host) in enumerate(zip(inputs, outputs)):
            s = i & 1
            with torch.cuda.stream(h2d):
                if used[s]:
                    h2d.wait_event(ev['in_free'][s])  # step i-2 has taken its input out of this buffer
                pipe['in'][s].copy_(x_host, non_blocking=True)
                ev['in_ready'][s].record(h2d)
            compute.wait_event(ev['in_ready'][s])
            self.buffers['norm'].copy_(pipe['in'][s], non_blocking=True)
            self.buffers['resid'].copy_(pipe['in'][s], non_blocking=True)
            ev['in_free'][s].record(compute)
            if self.producer_tf32:
                self.round_buffer('norm')
            if graph is not None:
                graph.replay()
            else:
                self.step()
            if used[s]:
                compute.wait_event(ev['out_free'][s])  # step i-2's result has left this buffer
            pipe['out'][s].copy_(self.buffers['resid'], non_blocking=True)
            ev['out_ready'][s].record(compute)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev['out_ready'][s])
                out_host.copy_(pipe['out'][s], non_blocking=True)
                ev['out_free'][s].record(d2h)
            used[s] = True
        compute.wait_stream(h2d)
        compute.wait_stream(d2h)
        return outputs
