"""The reference's CPU path for the encoder linears, as the timed CPU baseline.

Test/benchmark infrastructure only (see ``oracle/__init__.py``): ``bench.py``
times it in its ``cpu_baseline`` leg and in ``--impl reference``; the product
never calls it.

The reference's NumPy path decodes each Q8_0 tensor to FP32 on the host
(``gguf.Model.array``, ``parakeet_cuda/gguf.py:140-149``) and multiplies with
``x @ W.T`` in FP32 (``parakeet_cuda/reference.py:37``), applying SiLU
(``reference.py:41-42``), the 0.5 residual (``reference.py:43``), GLU
(``reference.py:57``) and the residual adds (``reference.py:55,62``) as
separate NumPy operations. NumPy's BLAS uses every host thread it is given.
"""
from __future__ import annotations

import os
import time

import numpy as np


def decode_f32(raw, n: int, k: int) -> np.ndarray:
    blocks = np.asarray(raw, np.uint8).reshape(-1, 34)
    scales = blocks[:, :2].copy().view('<f2').astype(np.float32)
    return (blocks[:, 2:].view(np.int8).astype(np.float32) * scales).reshape(n, k)


def _silu(z):
    return z / (1 + np.exp(-np.clip(z, -80, 80)))


def encoder_layer_linears(model, layer: int, norm, ctx, pos, resid):
    """One layer's nine Q8_0 linears on the CPU, reference-style (decode, then FP32 matmul)."""
    base = f'encoder.layers.{layer}.'

    def w(name):
        t = model.tensors[base + name + '.weight']
        return decode_f32(model.raw(base + name + '.weight'), *t.shape)

    for ffn in ('feed_forward1', 'feed_forward2'):
        h = _silu(norm @ w(ffn + '.linear1').T)
        resid = resid + 0.5 * (h @ w(ffn + '.linear2').T)
    qkv = [norm @ w('self_attn.linear_' + c).T for c in 'qkv']
    pos_out = pos @ w('self_attn.linear_pos').T
    resid = resid + ctx @ w('self_attn.linear_out').T
    a, b = np.split(norm @ w('conv.pointwise_conv1').T, 2, axis=-1)
    resid = resid + (a / (1 + np.exp(-np.clip(b, -80, 80)))) @ w('conv.pointwise_conv2').T
    return resid, qkv, pos_out


def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [p.get('num_threads') for p in threadpool_info() if p.get('user_api') == 'blas']
        if n and n[0]:
            return int(n[0])
    except Exception:
        pass
    return os.cpu_count() or 1


def time_layer_window(model, rows: int, layer: int = 0, seed: int = 0) -> float:
    """Seconds for one layer's linears (including the per-layer Q8_0 decode) over ``rows`` frames."""
    rng = np.random.default_rng(seed)
    norm, ctx, pos = (rng.normal(size=(rows, 1024)).astype(np.float32) for _ in range(3))
    resid = np.zeros((rows, 1024), np.float32)
    t0 = time.perf_counter()
    encoder_layer_linears(model, layer, norm, ctx, pos, resid)
    return time.perf_counter() - t0
