"""NumPy restatement of the subsampling stem (float64).

Test infrastructure only (see ``oracle/__init__.py``).

Reference citations (mgostIH/parakeet_cuda): ``parakeet_cuda/reference.py:11-30``
(``stem``), the CUDA launch sequence ``parakeet_cuda/encoder.py:38-66`` with
``conv_first`` / ``conv_dw2`` / ``flatten_stem`` (``kernels/runtime.cu:73-101``).

Mel features ``[frames, 128]`` are one input plane. Three stages, each a 3 x 3
window with stride 2 in time and frequency and one zero row / column of
padding on every side: a full convolution to 256 channels + ReLU, then twice a
depthwise convolution followed by a 256 x 256 pointwise convolution + ReLU.
The ``[t, 16 frequencies, 256 channels]`` result is flattened channel-major
(index ``c * 16 + f``) and projected 4096 -> 1024 with a bias.
"""
from __future__ import annotations

import numpy as np


def _a(model, name):
    return np.asarray(model.array('encoder.pre_encode.' + name), np.float64)


def _strided_taps(x):
    """x [T, F, C] -> for each (kt, kf) the [ceil(T/2), ceil(F/2), C] input seen by tap (kt, kf)."""
    t, f = x.shape[0], x.shape[1]
    nt, nf = (t + 1) // 2, (f + 1) // 2
    padded = np.zeros((t + 2, f + 2, x.shape[2]))
    padded[1:t + 1, 1:f + 1] = x
    return {(kt, kf): padded[kt:kt + 2 * nt:2, kf:kf + 2 * nf:2] for kt in range(3) for kf in range(3)}


def stem(mel, model):
    x = np.asarray(mel, np.float64)[:, :, None]
    for index, depthwise in ((0, False), (2, True), (5, True)):
        w = _a(model, f'conv.{index}.weight').reshape(256, 3, 3)
        taps = _strided_taps(x)
        y = _a(model, f'conv.{index}.bias').reshape(256) + sum(
            taps[kt, kf] * w[:, kt, kf] for kt in range(3) for kf in range(3))
        if depthwise:
            pw = f'conv.{index + 1}'
            y = y @ _a(model, pw + '.weight').reshape(256, 256).T + _a(model, pw + '.bias').reshape(256)
        x = np.maximum(y, 0.0)
    t = x.shape[0]
    flat = x.transpose(0, 2, 1).reshape(t, 256 * x.shape[1])
    return flat @ _a(model, 'out.weight').T + _a(model, 'out.bias')
