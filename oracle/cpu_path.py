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


class Decoder32:
    """The reference's NumPy predictor/joint (``parakeet_cuda/decoder.py:6-34``,
    ``CPUDecoder``) restated in float32: Q8_0 weights decoded to FP32 once,
    FP32 LSTM state, one matrix-vector product per weight per call. Driven by
    ``oracle.tdt.greedy_decode`` it is the reference's CPU decode loop
    (``decoder.py:78-97``), timed as the config-3 CPU baseline."""

    def __init__(self, model, layers: int = 2, hidden: int = 640):
        def f32(name):
            t = model.tensors[name]
            if t.kind == 8:
                return decode_f32(model.raw(name), *t.shape)
            return np.ascontiguousarray(np.asarray(model.array(name), np.float32))
        self.layers = layers
        self.w = {}
        for l in range(layers):
            for kind in ('ih', 'hh'):
                base = f'decoder.prediction.dec_rnn.lstm.{kind}_l{l}'
                self.w[base + '.weight'] = f32(base + '.weight')
                self.w[base + '.bias'] = f32(base + '.bias').reshape(-1)
        for name in ('joint.pred', 'joint.joint_net.2'):
            self.w[name + '.weight'] = f32(name + '.weight')
            self.w[name + '.bias'] = f32(name + '.bias').reshape(-1)
        self.embed = np.asarray(model.array('decoder.prediction.embed.weight'))
        self.h = [np.zeros(hidden, np.float32) for _ in range(layers)]
        self.c = [np.zeros(hidden, np.float32) for _ in range(layers)]
        self.candidate = self.pred = None

    def predict(self, token: int):
        x = self.embed[token].astype(np.float32)
        hn, cn = [], []
        for l in range(self.layers):
            ih = f'decoder.prediction.dec_rnn.lstm.ih_l{l}'
            hh = f'decoder.prediction.dec_rnn.lstm.hh_l{l}'
            z = (self.w[ih + '.weight'] @ x + self.w[ih + '.bias'] + self.w[hh + '.weight'] @ self.h[l]
                 + self.w[hh + '.bias'])
            gi, gf, gg, go = np.split(z, 4)
            c = _sigmoid(gf) * self.c[l] + _sigmoid(gi) * np.tanh(gg)
            x = _sigmoid(go) * np.tanh(c)
            hn.append(x)
            cn.append(c)
        self.candidate = (hn, cn)
        self.pred = self.w['joint.pred.weight'] @ x + self.w['joint.pred.bias']

    def joint(self, frame):
        z = self.w['joint.joint_net.2.weight'] @ np.maximum(frame + self.pred, 0) + self.w['joint.joint_net.2.bias']
        return int(np.argmax(z[:8193])), int(np.argmax(z[8193:]))

    def commit(self):
        self.h, self.c = self.candidate


def _sigmoid(a):
    return 1 / (1 + np.exp(-np.clip(a, -80, 80)))


def time_decode(model, projected, durations):
    """Seconds and joint calls of the reference-style CPU decode of each stream
    in ``projected`` (streams decoded one after another, as the reference
    decodes windows)."""
    from .tdt import greedy_decode
    decoders = [Decoder32(model) for _ in projected]  # weights decoded at load, outside the timing
    calls = 0
    t0 = time.perf_counter()
    for p, d in zip(projected, decoders):
        calls += greedy_decode(p, d, durations)['joint_calls']
    return time.perf_counter() - t0, calls


def time_linear(raw, n: int, k: int, m: int, repeats: int = 3, seed: int = 0) -> float:
    """Best-of-``repeats`` seconds of the reference CPU linear ``x @ W.T`` (FP32,
    ``reference.py:37``) on ``m`` rows, the Q8_0 weight decoded beforehand as
    ``gguf.Model.array`` does at load time."""
    w = decode_f32(raw, n, k)
    x = np.random.default_rng(seed).normal(size=(m, k)).astype(np.float32)
    best = None
    for _ in range(repeats):
        t0 = time.perf_counter()
        x @ w.T
        t = time.perf_counter() - t0
        best = t if best is None else min(best, t)
    return best
