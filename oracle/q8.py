"""NumPy restatement of the reference's Q8_0 contraction and its epilogues.

Test infrastructure only (see ``oracle/__init__.py``).

Reference citations (paths inside mgostIH/parakeet_cuda):

* Q8_0 block layout ``<f2 scale><32 x i8>``: ``parakeet_cuda/gguf.py:63-65,143-146``.
* Expansion kernel ``dequant_q8``: ``parakeet_cuda/kernels/runtime.cu:26-33``.
* Float64 golden ``x @ W.T``: ``workloads/q8_gemm.py:19-21``.
* GEMV ``q8_gemv``: ``parakeet_cuda/kernels/runtime.cu:180-188``; golden in
  ``tests/test_cuda.py:34-50``.
* Epilogues: ``silu`` ``runtime.cu:49-51``, ``residual`` ``runtime.cu:52-54``,
  ``bias_act`` ``runtime.cu:55-58``, ``glu`` ``runtime.cu:59-62``; their call
  sites ``parakeet_cuda/encoder.py:15-36,115-127``.
"""
from __future__ import annotations

import numpy as np

BLOCK = 32
BLOCK_BYTES = 34

# Epilogue codes shared with include/pq8.h (the oracle keeps its own copy of
# the numbers so that it does not import the product).
EPI_NONE = 0
EPI_RELU = 1
EPI_SILU = 2
EPI_GLU = 3
EPI_RESIDUAL = 4


def decode(raw, n: int, k: int) -> np.ndarray:
    """Q8_0 bytes -> float64 ``[n, k]``; element i of block b is ``f16(b*34) * i8(b*34+2+i)``."""
    if k % BLOCK:
        raise ValueError('K must be a multiple of 32')
    blocks = np.frombuffer(np.ascontiguousarray(raw, dtype=np.uint8).tobytes(), np.uint8)
    blocks = blocks.reshape(n * k // BLOCK, BLOCK_BYTES)
    scale = blocks[:, 0:2].copy().view('<f2')[:, 0].astype(np.float64)
    quant = blocks[:, 2:].copy().view(np.int8).astype(np.float64)
    return (quant * scale[:, None]).reshape(n, k)


def dequant_f32(raw, n: int, k: int) -> np.ndarray:
    """What ``dequant_q8`` writes: ``float(scale) * float(q)`` in FP32 (exact: <=19 significant bits)."""
    return decode(raw, n, k).astype(np.float32)


def gemm(x, raw, n: int, k: int) -> np.ndarray:
    """Float64 ``Y[m, n] = sum_k X[m, k] * W[n, k]`` (``workloads/q8_gemm.py:19-21``)."""
    return np.asarray(x, np.float64) @ decode(raw, n, k).T


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-np.clip(v, -80.0, 80.0)))


def epilogue(acc, epi: int, bias=None, resid=None, alpha: float = 1.0, relu: bool = False):
    """Apply a fused epilogue to a float64 accumulator ``acc[m, n]``.

    * ``EPI_NONE``: ``y = acc + bias``
    * ``EPI_RELU``: ``y = max(acc + bias, 0)`` (``bias_act`` with ``relu=1``)
    * ``EPI_SILU``: ``y = z * sigmoid(z)``, ``z = acc + bias`` (FFN up, ``encoder.py:31-33``)
    * ``EPI_GLU``: ``y[:, j] = a * sigmoid(b)`` over the two halves of ``acc + bias``
      (conv pointwise_conv1, ``encoder.py:117-119``)
    * ``EPI_RESIDUAL``: ``y = resid + alpha * (acc + bias)`` (``residual``; 0.5 for FFN,
      1 for attention/conv, ``encoder.py:35,112,126``)
    """
    z = np.asarray(acc, np.float64)
    if bias is not None:
        z = z + np.asarray(bias, np.float64)[None, :]
    if epi == EPI_NONE:
        return z
    if epi == EPI_RELU:
        return np.maximum(z, 0.0)
    if epi == EPI_SILU:
        return z * sigmoid(z)
    if epi == EPI_GLU:
        h = z.shape[1] // 2
        return z[:, :h] * sigmoid(z[:, h:])
    if epi == EPI_RESIDUAL:
        return np.asarray(resid, np.float64) + alpha * z
    raise ValueError(f'unknown epilogue {epi}')


def tf32_round(a) -> np.ndarray:
    """Round float32 values to TF32 (10 explicit mantissa bits), nearest, ties away from zero.

    This models the operand rounding done before the tensor-core MMA: the
    13 low mantissa bits are rounded off. Used to build a golden that differs
    from the kernel only in summation order.
    """
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    finite = (u & 0x7F800000) != 0x7F800000
    r = np.where(finite, (u + 0x1000) & 0xFFFFE000, u).astype(np.uint32)
    return r.view(np.float32)


def tf32_round_even(a) -> np.ndarray:
    """Round float32 values to TF32, nearest, ties to even.

    This is how the tensor-core GEMM rounds the expanded weights: it forms
    ``q * scale`` as an fp16 product (11 significant bits, IEEE
    round-to-nearest-even), which is exactly TF32 precision whenever the
    product is a normal fp16 number, and rounds the rare rows whose scale
    falls outside that range to nearest-even in fp32 arithmetic.
    """
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    finite = (u & 0x7F800000) != 0x7F800000
    r = np.where(finite, (u + 0xFFF + ((u >> 13) & 1)) & 0xFFFFE000, u).astype(np.uint32)
    return r.view(np.float32)


def gemm_tf32(x, raw, n: int, k: int) -> np.ndarray:
    """Float64 product of TF32-rounded operands: the expanded W rounded to
    nearest-even (``tf32_round_even``), X to nearest with ties away
    (``tf32_round``, the rounding of the activation producers)."""
    w = tf32_round_even(dequant_f32(raw, n, k)).astype(np.float64)
    return tf32_round(np.asarray(x, np.float32)).astype(np.float64) @ w.T


def rms(a) -> float:
    a = np.asarray(a, np.float64)
    return float(np.sqrt(np.mean(a * a))) if a.size else 0.0


def max_err_over_rms(actual, golden) -> float:
    """North-star tolerance metric: ``max|actual - golden| / rms(golden)``."""
    g = np.asarray(golden, np.float64)
    r = rms(g)
    d = float(np.max(np.abs(np.asarray(actual, np.float64) - g))) if g.size else 0.0
    return d / r if r else d
