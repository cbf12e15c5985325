"""Seeded synthetic Parakeet weights and activations in the GGUF Q8_0 block format.

No real checkpoint is available offline, so every workload runs on random
weights that follow the reference's tensor schema (``parakeet_cuda/gguf.py:86-133``)
and the value distributions of its kernel contract
(``workloads/q8_gemm.py:12-24``): int8 values uniform in [-127, 127] and one
fp16 scale per 32-value K block.

``SyntheticParakeet`` exposes the same duck-typed surface as the reference's
``gguf.Model`` (``tensors``, ``raw``, ``array``, ``names``, ``metadata``,
``text``), so the reference decoder and our host code can both consume it.
Tensors are generated lazily and deterministically from ``(seed, name)``.
"""
from __future__ import annotations

from dataclasses import dataclass
import hashlib
import math

import numpy as np

Q8_BLOCK = 32          # values per Q8_0 block along K (gguf.py:63-65)
Q8_BLOCK_BYTES = 34    # <f2 scale><32 x i8>
BLANK = 8192           # TDT blank id (decoder.py:80)
VOCAB = 8193           # 8192 pieces + blank
DURATIONS = [0, 1, 2, 3, 4]
JOINT_OUT = VOCAB + len(DURATIONS)   # 8198 rows of joint.joint_net.2 (gguf.py:130)

# Scale range for the encoder linears: config 0 of the benchmark (U[1e-3, 2e-2]).
ENCODER_SCALE = (1e-3, 2e-2)
# Scale range for the prediction/joint network. With the encoder range the random
# 2-layer LSTM is chaotic (gate pre-activations ~N(0, 20^2)): float32 and float64
# trajectories of the same decoder separate after ~15 steps, so no two
# implementations with different summation orders could agree on a long token
# sequence. U[2e-4, 1.2e-3] gives O(1) pre-activations, like a trained LSTM.
DECODER_SCALE = (2e-4, 1.2e-3)
# Scale range for the encoder linears of a model built for whole FastConformer
# blocks (``block=True``): weight std ~ 1/sqrt(1024) as in a trained layer, so
# the residual stream, the attention scores and the softmax stay O(1) through
# the block instead of saturating (with the config-0 range a 1024 -> 4096
# linear alone multiplies the RMS by ~25).
BLOCK_SCALE = (2e-4, 6e-4)
STEM_OUT_SCALE = (1e-4, 3e-4)  # fan-in 4096: weight std ~ 1/64
POS_EMB_MAX_LEN = 5000  # asr.encoder.pos_emb_max_len (gguf.py:95); pe has 2 * 5000 - 1 rows


def q8_0_blocks(rng: np.random.Generator, n: int, k: int, scale_lo: float = 1e-3,
                scale_hi: float = 2e-2, qmin: int = -127, qmax: int = 127) -> np.ndarray:
    """Random ``[n, k]`` weight as GGUF Q8_0 blocks, shape ``(n*k/32, 34)`` uint8.

    The draw order (all scales, then all values) and the byte packing follow
    ``workloads/q8_gemm.py:15-18`` so that seed 903 with ``scale_lo=1e-4``
    reproduces the reference's own contract inputs byte for byte.
    """
    if k % Q8_BLOCK:
        raise ValueError(f'Q8_0 needs K % 32 == 0, got K={k}')
    nb = n * k // Q8_BLOCK
    scales = rng.uniform(scale_lo, scale_hi, (nb, 1)).astype(np.float16)
    values = rng.integers(qmin, qmax + 1, (nb, Q8_BLOCK), dtype=np.int8)
    packed = np.empty((nb, Q8_BLOCK_BYTES), np.uint8)
    packed[:, :2] = scales.view(np.uint8).reshape(-1, 2)
    packed[:, 2:] = values.view(np.uint8)
    return packed


def decode_q8_0(raw: np.ndarray, n: int, k: int) -> np.ndarray:
    """GGUF Q8_0 bytes -> float32 ``[n, k]`` (value = f16(scale) * int8, ``gguf.py:143-146``)."""
    blocks = np.asarray(raw, np.uint8).reshape(-1, Q8_BLOCK_BYTES)
    scales = blocks[:, :2].copy().view('<f2').astype(np.float32)
    return (blocks[:, 2:].view(np.int8).astype(np.float32) * scales).reshape(n, k)


@dataclass(frozen=True)
class Tensor:
    """Mirror of ``gguf.Tensor`` (gguf.py:10-24): GGUF dims are reversed into row-major ``shape``."""
    name: str
    dims: tuple
    kind: int      # 0 = F32, 1 = F16, 8 = Q8_0
    offset: int
    nbytes: int

    @property
    def shape(self):
        return tuple(reversed(self.dims))

    @property
    def elements(self):
        return math.prod(self.dims)


def _decoder_schema():
    s = {'decoder.prediction.embed.weight': ((640, VOCAB), 1)}
    for l in range(2):
        for kind in ('ih', 'hh'):
            base = f'decoder.prediction.dec_rnn.lstm.{kind}_l{l}'
            s[base + '.weight'] = ((640, 2560), 8)
            s[base + '.bias'] = ((2560,), 0)
    for name, dims in (('joint.enc', (1024, 640)), ('joint.pred', (640, 640)),
                       ('joint.joint_net.2', (640, JOINT_OUT))):
        s[name + '.weight'] = (dims, 8)
        s[name + '.bias'] = ((dims[1],), 0)
    return s


def _encoder_layer_schema(layer: int):
    base = f'encoder.layers.{layer}.'
    s = {}
    for n in ('feed_forward1', 'feed_forward2'):
        s[base + n + '.linear1.weight'] = ((1024, 4096), 8)
        s[base + n + '.linear2.weight'] = ((4096, 1024), 8)
    for n in ('q', 'k', 'v', 'out', 'pos'):
        s[base + 'self_attn.linear_' + n + '.weight'] = ((1024, 1024), 8)
    s[base + 'conv.pointwise_conv1.weight'] = ((1024, 2048), 8)
    s[base + 'conv.pointwise_conv2.weight'] = ((1024, 1024), 8)
    return s


def _encoder_block_schema(layer: int):
    """The non-linear parameters of one block (gguf.py:113-124): LayerNorms,
    rel-pos attention biases, the conv module's depthwise kernel and BatchNorm."""
    base = f'encoder.layers.{layer}.'
    s = {}
    for n in ('norm_feed_forward1', 'norm_self_att', 'norm_conv', 'norm_feed_forward2', 'norm_out'):
        for suffix in ('weight', 'bias'):
            s[base + n + '.' + suffix] = ((1024,), 0)
    for n in ('u', 'v'):
        s[base + 'self_attn.pos_bias_' + n] = ((128, 8), 0)
    s[base + 'conv.depthwise_conv.weight'] = ((9, 1, 1024), 1)
    for n in ('weight', 'bias', 'running_mean', 'running_var'):
        s[base + 'conv.batch_norm.' + n] = ((1024,), 0)
    return s


def _stem_schema():
    """Subsampling stem (gguf.py:104-111): a 3x3 convolution from the single mel
    plane to 256 channels, two depthwise 3x3 + pointwise 256 x 256 stages (all
    stride 2 in time and frequency), and the Q8_0 4096 -> 1024 output linear."""
    s = {}
    for i in (0, 2, 5):
        s[f'encoder.pre_encode.conv.{i}.weight'] = ((3, 3, 1, 256), 1)
        s[f'encoder.pre_encode.conv.{i}.bias'] = ((256,), 0)
    for i in (3, 6):
        s[f'encoder.pre_encode.conv.{i}.weight'] = ((1, 1, 256, 256), 1)
        s[f'encoder.pre_encode.conv.{i}.bias'] = ((256,), 0)
    s['encoder.pre_encode.out.weight'] = ((4096, 1024), 8)
    s['encoder.pre_encode.out.bias'] = ((1024,), 0)
    return s


def relative_sinusoids(max_len: int, d: int) -> np.ndarray:
    """Relative positional table ``[2 max_len - 1, d]``: row i encodes the
    relative position ``max_len - 1 - i`` with interleaved sin / cos of
    geometrically spaced frequencies (the FastConformer rel-pos encoding)."""
    pos = (max_len - 1 - np.arange(2 * max_len - 1, dtype=np.float64))[:, None]
    freq = np.exp(-np.log(10000.0) * np.arange(0, d, 2, dtype=np.float64) / d)[None, :]
    pe = np.empty((2 * max_len - 1, d), np.float64)
    pe[:, 0::2] = np.sin(pos * freq)
    pe[:, 1::2] = np.cos(pos * freq)
    return pe.astype(np.float32)


class SyntheticParakeet:
    """Random-weight stand-in for ``gguf.Model`` with the Parakeet TDT schema.

    Only the tensors the Q8_0 contraction path touches are present: the 24
    encoder layers' linears and the TDT prediction/joint network. Q8_0
    tensors draw int8 values from U[-127, 127]; encoder scales follow config 0
    (``ENCODER_SCALE``) and decoder/joint scales ``DECODER_SCALE``. F32 biases
    are N(0, 0.1); the F16 embedding is N(0, 1).
    """

    def __init__(self, seed: int = 0, encoder_layers: int = 24, decoder: bool = True,
                 blank_bias: float = 0.0, duration0_bias: float = 0.0, block: bool = False):
        """``block``: also the non-linear block parameters and the positional
        table, with ``BLOCK_SCALE`` encoder weights, for whole-block runs."""
        self.seed = seed
        self.block = block
        # Optional offsets on the joint bias so that random weights also exercise
        # blank emissions and zero-duration steps of the greedy loop.
        self.blank_bias, self.duration0_bias = blank_bias, duration0_bias
        self.metadata = {'asr.tdt.durations': list(DURATIONS),
                         'asr.tokenizer.vocab': [f'<{i}>' for i in range(BLANK)],
                         'asr.encoder.pos_emb_max_len': POS_EMB_MAX_LEN}
        schema = {}
        if block:
            schema['encoder.pos_enc.pe'] = ((1024, 2 * POS_EMB_MAX_LEN - 1), 0)
            schema.update(_stem_schema())
        for layer in range(encoder_layers):
            schema.update(_encoder_layer_schema(layer))
            if block:
                schema.update(_encoder_block_schema(layer))
        if decoder:
            schema.update(_decoder_schema())
        self.tensors, offset = {}, 0
        for name, (dims, kind) in schema.items():
            n = math.prod(dims)
            size = n * {0: 4, 1: 2, 8: 34}[kind] // (32 if kind == 8 else 1)
            self.tensors[name] = Tensor(name, dims, kind, offset, size)
            offset += (size + 31) // 32 * 32
        self._cache = {}

    def _rng(self, name: str) -> np.random.Generator:
        digest = hashlib.sha256(f'{self.seed}:{name}'.encode()).digest()
        return np.random.default_rng(int.from_bytes(digest[:8], 'little'))

    def raw(self, name: str) -> np.ndarray:
        """Raw GGUF bytes of a tensor (``gguf.py:135-138``)."""
        if name not in self._cache:
            t = self.tensors[name]
            rng = self._rng(name)
            if t.kind == 8:
                n, k = t.shape
                lo, hi = ((BLOCK_SCALE if self.block else ENCODER_SCALE) if name.startswith('encoder.')
                          else DECODER_SCALE)
                if name == 'encoder.pre_encode.out.weight':
                    lo, hi = STEM_OUT_SCALE
                data = q8_0_blocks(rng, n, k, lo, hi).reshape(-1)
            elif t.kind == 1:
                # fan-in 9 (3 x 3 and depthwise kernels), 256 (stem pointwise), 1 (embedding)
                scale = (1.0 / 16.0 if name.endswith(('conv.3.weight', 'conv.6.weight'))
                         else 1.0 / 3.0 if name.endswith('.weight') and 'conv' in name else 1.0)
                data = (scale * rng.normal(size=t.elements)).astype('<f2').view(np.uint8)
            elif name == 'encoder.pos_enc.pe':
                data = relative_sinusoids(POS_EMB_MAX_LEN, 1024).astype('<f4').view(np.uint8).reshape(-1)
            else:
                values = 0.1 * rng.normal(size=t.elements)
                if name.endswith(('norm_feed_forward1.weight', 'norm_self_att.weight', 'norm_conv.weight',
                                  'norm_feed_forward2.weight', 'norm_out.weight', 'batch_norm.weight')):
                    values += 1.0
                elif name.endswith('batch_norm.running_var'):
                    values = rng.uniform(0.5, 1.5, size=t.elements)
                if name == 'joint.joint_net.2.bias':
                    values[BLANK] += self.blank_bias
                    values[VOCAB] += self.duration0_bias
                data = values.astype('<f4').view(np.uint8)
            self._cache[name] = data
        return self._cache[name]

    def array(self, name: str) -> np.ndarray:
        """Decoded tensor in row-major ``shape`` (``gguf.py:140-149``)."""
        t = self.tensors[name]
        raw = self.raw(name)
        if t.kind == 8:
            return decode_q8_0(raw, *t.shape)
        return raw.view('<f4' if t.kind == 0 else '<f2').reshape(t.shape)

    def names(self, prefix: str):
        return [n for n in self.tensors if n.startswith(prefix)]

    def text(self, ids):
        return ' '.join(str(i) for i in ids)


def activations(seed: int, rows: int, width: int) -> np.ndarray:
    """Seeded fp32 activations ~ N(0, 1) of shape ``[rows, width]``."""
    return np.random.default_rng(seed).normal(size=(rows, width)).astype(np.float32)
