"""NumPy restatement of one FastConformer encoder block (float64).

Test infrastructure only (see ``oracle/__init__.py``).

Reference citations (mgostIH/parakeet_cuda):

* The block as a whole: ``parakeet_cuda/reference.py:33-66`` (``block``); the
  CUDA launch sequence it mirrors: ``parakeet_cuda/encoder.py:28-127``.
* LayerNorm, eps 1e-5: ``reference.py:6-8``, kernel ``layer_norm``
  ``kernels/runtime.cu:38-48``.
* Macaron feed-forward (LN, linear1, SiLU, linear2, x + 0.5 y):
  ``reference.py:41-44``, ``encoder.py:28-36``.
* Relative-position self-attention, 8 heads of 128: ``reference.py:46-56``;
  the positional rows are ``pe[limit - t : limit + t - 1]`` (``encoder.py:71-73``);
  scores ``((q + u) k + (q + v) p) / sqrt(128)`` where query i and key j use
  positional row ``t - 1 + j - i`` (``rel_scores``, ``kernels/runtime.cu:122-128``).
* Conv module (LN, pointwise 1024 -> 2048, GLU, depthwise k = 9 with 4 rows of
  zero padding per window, BatchNorm with running statistics, SiLU, pointwise
  1024 -> 1024, residual): ``reference.py:58-64``, ``depthwise1``
  ``kernels/runtime.cu:63-71``.
* Second feed-forward and the final LayerNorm: ``reference.py:65-66``.

Everything is computed in float64 from the decoded weights, with the
positional shift written as the index ``t - 1 + j - i`` rather than the
reference's pad/reshape trick, so it is an independent check.
"""
from __future__ import annotations

import numpy as np

HEADS = 8
HEAD_DIM = 128
EPS = 1e-5


def layer_norm(x, w, b):
    x = np.asarray(x, np.float64)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + EPS) * w + b


def silu(z):
    return z / (1.0 + np.exp(-np.clip(z, -80, 80)))


def rel_shift_scores(qu, qv, k, p):
    """Per head h: s[i, j] = (qu[i] . k[j] + qv[i] . p[t - 1 + j - i]) / sqrt(128).
    qu, qv, k: [H, t, D]; p: [H, 2t - 1, D]. Returns [H, t, t]."""
    t = k.shape[1]
    ac = qu @ k.transpose(0, 2, 1)
    bd_full = qv @ p.transpose(0, 2, 1)          # [H, t, 2t-1]
    rows = np.arange(t)[:, None]
    cols = (t - 1) + np.arange(t)[None, :] - rows  # positional row of (i, j)
    bd = bd_full[:, rows, cols]
    return (ac + bd) / np.sqrt(HEAD_DIM)


def softmax(s):
    e = np.exp(s - s.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


class BlockWeights:
    """Decoded float64 parameters of layer ``layer`` of a gguf-style model."""

    def __init__(self, model, layer: int):
        base = f'encoder.layers.{layer}.'
        a = lambda n: np.asarray(model.array(base + n), np.float64)
        self.ln = {n: (a(n + '.weight').reshape(-1), a(n + '.bias').reshape(-1))
                   for n in ('norm_feed_forward1', 'norm_self_att', 'norm_conv', 'norm_feed_forward2', 'norm_out')}
        self.lin = {}
        for n in ('feed_forward1.linear1', 'feed_forward1.linear2', 'feed_forward2.linear1', 'feed_forward2.linear2',
                  'self_attn.linear_q', 'self_attn.linear_k', 'self_attn.linear_v', 'self_attn.linear_out',
                  'self_attn.linear_pos', 'conv.pointwise_conv1', 'conv.pointwise_conv2'):
            w = a(n + '.weight')
            self.lin[n] = w.reshape(w.shape[0], -1)
        self.u = a('self_attn.pos_bias_u').reshape(HEADS, HEAD_DIM)
        self.v = a('self_attn.pos_bias_v').reshape(HEADS, HEAD_DIM)
        self.dw = a('conv.depthwise_conv.weight').reshape(1024, 9)
        self.bn = {n: a('conv.batch_norm.' + n).reshape(-1) for n in ('weight', 'bias', 'running_mean', 'running_var')}
        self.limit = int(model.metadata['asr.encoder.pos_emb_max_len'])
        self.pe = np.asarray(model.array('encoder.pos_enc.pe'), np.float64)


def positions(w: BlockWeights, t: int):
    """linear_pos of the 2t - 1 positional rows shared by every window of t frames."""
    return w.pe[w.limit - t:w.limit + t - 1] @ w.lin['self_attn.linear_pos'].T


def attention(w: BlockWeights, x_norm, t: int):
    lin = w.lin
    heads = lambda y: y.reshape(t, HEADS, HEAD_DIM).transpose(1, 0, 2)
    q, k, v = (heads(x_norm @ lin['self_attn.linear_' + c].T) for c in 'qkv')
    p = positions(w, t).reshape(2 * t - 1, HEADS, HEAD_DIM).transpose(1, 0, 2)
    s = rel_shift_scores(q + w.u[:, None, :], q + w.v[:, None, :], k, p)
    return (softmax(s) @ v).transpose(1, 0, 2).reshape(t, HEADS * HEAD_DIM)


def conv_module_depthwise(w: BlockWeights, gate):
    """Depthwise k = 9 over the frames of one window (zero rows beyond its ends),
    BatchNorm with running statistics, SiLU."""
    t = gate.shape[0]
    padded = np.zeros((t + 8, gate.shape[1]))
    padded[4:4 + t] = gate
    y = sum(padded[k:k + t] * w.dw[:, k] for k in range(9))
    bn = w.bn
    y = (y - bn['running_mean']) / np.sqrt(bn['running_var'] + EPS) * bn['weight'] + bn['bias']
    return silu(y)


def block(x, w: BlockWeights, final_norm: bool = True):
    """One block over one window ``x`` [t, 1024]; float64 throughout. With
    ``final_norm=False`` the residual stream before ``norm_out`` is returned."""
    x = np.asarray(x, np.float64)
    t = x.shape[0]
    lin = w.lin

    def ff(x, n):
        z = silu(layer_norm(x, *w.ln[f'norm_feed_forward{n}']) @ lin[f'feed_forward{n}.linear1'].T)
        return x + 0.5 * (z @ lin[f'feed_forward{n}.linear2'].T)

    x = ff(x, 1)
    x = x + attention(w, layer_norm(x, *w.ln['norm_self_att']), t) @ lin['self_attn.linear_out'].T
    pw = layer_norm(x, *w.ln['norm_conv']) @ lin['conv.pointwise_conv1'].T
    gate = pw[:, :1024] * (1.0 / (1.0 + np.exp(-np.clip(pw[:, 1024:], -80, 80))))
    x = x + conv_module_depthwise(w, gate) @ lin['conv.pointwise_conv2'].T
    x = ff(x, 2)
    return layer_norm(x, *w.ln['norm_out']) if final_norm else x


def blocks(x, model, layers, windows: int = 1, final_norm: bool = True):
    """``layers`` blocks over ``windows`` independent windows stacked in ``x`` [windows * t, 1024]
    (the last block stops before its ``norm_out`` when ``final_norm`` is False)."""
    x = np.asarray(x, np.float64)
    t = x.shape[0] // windows
    layers = list(layers)
    for j, layer in enumerate(layers):
        w = BlockWeights(model, layer)
        last = final_norm or j + 1 < len(layers)
        x = np.concatenate([block(x[i * t:(i + 1) * t], w, last) for i in range(windows)])
    return x
