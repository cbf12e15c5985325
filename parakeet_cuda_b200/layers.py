"""The Q8_0 linears of one FastConformer encoder layer, as data (no PyTorch).

Each encoder layer of the reference issues these linears
(``parakeet_cuda/encoder.py``; all ``use_bias=False``, ``gguf.py:91``); the
entries are (name, weight key(s), N, K, epilogue, alpha, input buffer, output
buffer, flags). Both host layers (``encoder.py`` on PyTorch memory and
``host.py`` on driver-API memory) run this plan.
"""
from __future__ import annotations

from .pq8 import EPI_GLU, EPI_NONE, EPI_RESIDUAL, EPI_SILU, FLAG_OUT_TF32, FLAG_X_TF32

D_MODEL, D_FF, D_CONV = 1024, 4096, 2048
FRAMES_PER_WINDOW = 375   # 30 s at 80 ms per encoder frame


def flops_per_row_per_layer(pos_rows_per_row: float = 1.0) -> int:
    """Algorithmic FLOPs (2 N K per linear) per activation row per layer."""
    nk = (2 * D_FF * D_MODEL * 2 + 3 * D_MODEL * D_MODEL + D_MODEL * D_MODEL + D_CONV * D_MODEL
          + D_MODEL * D_MODEL)
    return int(2 * (nk + pos_rows_per_row * D_MODEL * D_MODEL))


# (name, weight key(s), N, K, epilogue, alpha, input buffer, output buffer, flags)
LAYER_PLAN = (
    ('ffn1_up', ('feed_forward1.linear1',), D_FF, D_MODEL, EPI_SILU, 1.0, 'norm', 'hidden', FLAG_OUT_TF32),
    ('ffn1_down', ('feed_forward1.linear2',), D_MODEL, D_FF, EPI_RESIDUAL, 0.5, 'hidden', 'resid', FLAG_X_TF32),
    ('qkv', ('self_attn.linear_q', 'self_attn.linear_k', 'self_attn.linear_v'), 3 * D_MODEL, D_MODEL, EPI_NONE,
     1.0, 'norm', 'qkv', 0),
    ('pos', ('self_attn.linear_pos',), D_MODEL, D_MODEL, EPI_NONE, 1.0, 'pos', 'pos_out', 0),
    ('out', ('self_attn.linear_out',), D_MODEL, D_MODEL, EPI_RESIDUAL, 1.0, 'ctx', 'resid', 0),
    ('pw1_glu', ('conv.pointwise_conv1',), D_CONV, D_MODEL, EPI_GLU, 1.0, 'norm', 'gate', FLAG_OUT_TF32),
    ('pw2', ('conv.pointwise_conv2',), D_MODEL, D_MODEL, EPI_RESIDUAL, 1.0, 'gate', 'resid', FLAG_X_TF32),
    ('ffn2_up', ('feed_forward2.linear1',), D_FF, D_MODEL, EPI_SILU, 1.0, 'norm', 'hidden', FLAG_OUT_TF32),
    ('ffn2_down', ('feed_forward2.linear2',), D_MODEL, D_FF, EPI_RESIDUAL, 0.5, 'hidden', 'resid', FLAG_X_TF32),
)
