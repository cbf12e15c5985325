"""Whole FastConformer encoder blocks on the device (``parakeet_cuda/reference.py:33-66``).

``EncoderBlocks`` runs the reference's block for ``windows`` independent
windows of ``t`` frames stacked as rows of one ``[windows * t, 1024]``
residual stream, entirely on the GPU:

=====================  ===========================================================
step                   kernel
=====================  ===========================================================
LayerNorm (x5)         ``pq8_layer_norm`` (output TF32-rounded when a GEMM reads it)
FFN1 / FFN2            ``pq8_gemm`` + SiLU, ``pq8_gemm`` with ``x += 0.5 y``: the pair
                       as one ``pq8_sequence_run`` (down-projection tiles start as
                       soon as their rows of the hidden state are written)
Q, K, V                one ``pq8_gemm`` on the packed ``[3072, 1024]`` weight
linear_pos             one ``pq8_gemm`` on the ``2t - 1`` positional rows, once per
                       layer for all windows (their positions are identical);
                       QKV and linear_pos run as one sequence launch
attention              ``pq8_rel_attention`` (one fused kernel: products, shift, softmax)
linear_out             ``pq8_gemm`` with ``x += y``
conv module            ``pq8_gemm`` + GLU, ``pq8_conv_depthwise_bn_silu``,
                       ``pq8_gemm`` with ``x += y``
=====================  ===========================================================

The reference launches the same block per window as one SGEMM plus an
elementwise kernel per linear after a ``dequant_q8`` of the layer's weights
(``parakeet_cuda/encoder.py:28-127``); here the Q8_0 weights stay resident and
packed, the epilogues are fused, and all windows share every launch.
"""
from __future__ import annotations

import numpy as np
import torch

from .encoder import D_FF, D_MODEL, EncoderStack, LAYER_PLAN
from .pq8 import ATTN_FP32, EPI_RESIDUAL, FLAG_OUT_TF32, FLAG_X_TF32, GemmTask
from .runtime import Runtime

LN_NAMES = ('norm_feed_forward1', 'norm_self_att', 'norm_conv', 'norm_feed_forward2', 'norm_out')


class EncoderBlocks:
    """``layers`` encoder blocks over ``windows`` windows of ``t`` frames on one device."""

    def __init__(self, model, runtime: Runtime, windows: int, t: int, layers: int = 24,
                 attention_fp32: bool = False, sequences: bool = True):
        self.rt, self.windows, self.t, self.layers = runtime, windows, t, layers
        self.rows = windows * t
        self.attn_flags = FLAG_OUT_TF32 | (ATTN_FP32 if attention_fp32 else 0)
        dev = runtime.device
        # packed Q8_0 linears (device repack), the same set as the linear stack
        self.linears = EncoderStack(model, runtime, 1, layers=layers).weights
        f32 = dict(dtype=torch.float32, device=dev)
        to_dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
        self.params = []
        for l in range(layers):
            base = f'encoder.layers.{l}.'
            p = {n: (to_dev(model.array(base + n + '.weight').reshape(-1)),
                     to_dev(model.array(base + n + '.bias').reshape(-1))) for n in LN_NAMES}
            p['u'] = to_dev(model.array(base + 'self_attn.pos_bias_u').reshape(-1))
            p['v'] = to_dev(model.array(base + 'self_attn.pos_bias_v').reshape(-1))
            # the GGUF's fp16 [1024][1][9] depthwise kernel, bit for bit
            raw = np.ascontiguousarray(model.raw(base + 'conv.depthwise_conv.weight')).view(np.int16)
            p['dw'] = torch.from_numpy(raw.copy()).to(dev)
            p['bn'] = tuple(to_dev(model.array(base + 'conv.batch_norm.' + n).reshape(-1))
                            for n in ('weight', 'bias', 'running_mean', 'running_var'))
            self.params.append(p)
        limit = int(model.metadata['asr.encoder.pos_emb_max_len'])
        if t > limit:
            raise ValueError(f'{t} frames exceed pos_emb_max_len {limit}')
        # positional rows pe[limit - t : limit + t - 1] (encoder.py:71-73), TF32-rounded for linear_pos
        self.pe = to_dev(np.asarray(model.array('encoder.pos_enc.pe'))[limit - t:limit + t - 1])
        runtime.lib.call('pq8_round_tf32', self.pe.data_ptr(), self.pe.numel(), runtime.stream())
        rows = self.rows
        self.buf = {
            'x': torch.zeros(rows, D_MODEL, **f32),
            'norm': torch.empty(rows, D_MODEL, **f32),
            'hidden': torch.empty(rows, D_FF, **f32),
            'qkv': torch.empty(rows, 3 * D_MODEL, **f32),
            'pos': torch.empty(2 * t - 1, D_MODEL, **f32),
            'ctx': torch.empty(rows, D_MODEL, **f32),
            'gate': torch.empty(rows, D_MODEL, **f32),
            'dw': torch.empty(rows, D_MODEL, **f32),
        }
        need = runtime.lib.attention_workspace_size(windows, t)
        self.attn_ws = torch.empty(need, dtype=torch.uint8, device=dev)
        self._plan = {e[0]: e for e in LAYER_PLAN}
        # linears that follow one another with nothing in between, as sequence
        # launches (plans bound to the buffers above)
        self.seq_plans = None
        if sequences:
            self.seq_plans = []
            for l in range(layers):
                groups = {
                    'ffn1': [self._task(l, 'ffn1_up', 'norm', 'hidden'), self._task(l, 'ffn1_down', 'hidden', 'x')],
                    'att_in': [self._task(l, 'qkv', 'norm', 'qkv'), self._task(l, 'pos', self.pe, 'pos')],
                    'ffn2': [self._task(l, 'ffn2_up', 'norm', 'hidden'), self._task(l, 'ffn2_down', 'hidden', 'x')],
                }
                plans = {}
                for key, tasks in groups.items():
                    nbytes = runtime.lib.sequence_plan_size(tasks)
                    plan = torch.empty(nbytes, dtype=torch.uint8, device=dev)
                    runtime.lib.sequence_plan(tasks, plan.data_ptr(), nbytes, runtime.stream())
                    plans[key] = plan
                self.seq_plans.append(plans)

    # -- pieces ----------------------------------------------------------------
    def _ln(self, l: int, name: str, src: str, dst: str, tf32: bool = True) -> None:
        w, b = self.params[l][name]
        x, y = self.buf[src], self.buf[dst]
        self.rt.lib.call('pq8_layer_norm', x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(), x.shape[0],
                         x.shape[1], FLAG_OUT_TF32 if tf32 else 0, self.rt.stream())

    def _task(self, l: int, name: str, src, dst: str) -> GemmTask:
        """The linear as a ``pq8_gemm_task`` on the block's buffers (as ``_gemm`` launches it)."""
        _, _, n, k, epi, alpha, _, _, flags = self._plan[name]
        x = self.buf[src] if isinstance(src, str) else src
        out = self.buf[dst]
        w = self.linears[l][name]
        resid = out.data_ptr() if epi == EPI_RESIDUAL else None
        return GemmTask(w.pointer, x.data_ptr(), out.data_ptr(), None, resid, x.shape[0], w.n, w.k, epi, alpha,
                        flags | FLAG_X_TF32, -1, 0)

    def _sequence(self, l: int, key: str) -> None:
        self.rt.lib.call('pq8_sequence_run', self.seq_plans[l][key].data_ptr(), self.rt.stream())

    def _gemm(self, l: int, name: str, src, dst: str, out_tf32: bool | None = None) -> None:
        _, _, n, k, epi, alpha, _, _, flags = self._plan[name]
        if out_tf32 is not None:
            flags = (flags & ~FLAG_OUT_TF32) | (FLAG_OUT_TF32 if out_tf32 else 0)
        x = self.buf[src] if isinstance(src, str) else src
        out = self.buf[dst]
        resid = out if epi == EPI_RESIDUAL else None
        self.rt.gemm(x, self.linears[l][name], out=out, resid=resid, epilogue=epi, alpha=alpha,
                     flags=flags | FLAG_X_TF32)

    def layer(self, l: int, final_norm: bool = True) -> None:
        """One block on the residual stream ``buf['x']`` (reference.py:33-66).
        ``final_norm=False`` leaves out the block's last LayerNorm (``norm_out``)
        and keeps the residual stream as it stands before it."""
        b, p, lib, st = self.buf, self.params[l], self.rt.lib, self.rt.stream()
        seq = self.seq_plans is not None
        self._ln(l, 'norm_feed_forward1', 'x', 'norm')
        if seq:
            self._sequence(l, 'ffn1')
        else:
            self._gemm(l, 'ffn1_up', 'norm', 'hidden')
            self._gemm(l, 'ffn1_down', 'hidden', 'x')
        self._ln(l, 'norm_self_att', 'x', 'norm')
        if seq:
            self._sequence(l, 'att_in')
        else:
            self._gemm(l, 'qkv', 'norm', 'qkv')
            self._gemm(l, 'pos', self.pe, 'pos')
        lib.call('pq8_rel_attention', b['qkv'].data_ptr(), b['pos'].data_ptr(), p['u'].data_ptr(), p['v'].data_ptr(),
                 b['ctx'].data_ptr(), self.windows, self.t, self.attn_flags, self.attn_ws.data_ptr(),
                 self.attn_ws.numel(), st)
        self._gemm(l, 'out', 'ctx', 'x')
        self._ln(l, 'norm_conv', 'x', 'norm')
        self._gemm(l, 'pw1_glu', 'norm', 'gate', out_tf32=False)  # the depthwise conv reads it, not a GEMM
        bw, bb, bm, bv = p['bn']
        lib.call('pq8_conv_depthwise_bn_silu', b['gate'].data_ptr(), p['dw'].data_ptr(), bw.data_ptr(),
                 bb.data_ptr(), bm.data_ptr(), bv.data_ptr(), b['dw'].data_ptr(), self.windows, self.t, D_MODEL,
                 FLAG_OUT_TF32, st)
        self._gemm(l, 'pw2', 'dw', 'x')
        self._ln(l, 'norm_feed_forward2', 'x', 'norm')
        if seq:
            self._sequence(l, 'ffn2')
        else:
            self._gemm(l, 'ffn2_up', 'norm', 'hidden')
            self._gemm(l, 'ffn2_down', 'hidden', 'x')
        if final_norm:
            self._ln(l, 'norm_out', 'x', 'x', tf32=False)  # the block's output, next block's input

    def step(self, final_norm: bool = True) -> None:
        """Every layer; ``final_norm=False`` stops the last one before its ``norm_out``."""
        for l in range(self.layers):
            self.layer(l, final_norm or l + 1 < self.layers)

    def forward(self, x: torch.Tensor, final_norm: bool = True) -> torch.Tensor:
        """``x`` [windows * t, 1024] (device) through every layer; returns the output stream
        (before the last layer's ``norm_out`` when ``final_norm`` is False)."""
        self.buf['x'].copy_(x)
        self.step(final_norm)
        return self.buf['x']

    def capture(self) -> torch.cuda.CUDAGraph:
        """One ``step`` as a CUDA graph (call ``step`` once first so that per-device state
        and cuBLAS are initialised outside the capture)."""
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream(self.rt.device)
        side.wait_stream(torch.cuda.current_stream(self.rt.device))
        with torch.cuda.stream(side):
            graph.capture_begin()
            try:
                self.step()
            finally:
                graph.capture_end()
        torch.cuda.current_stream(self.rt.device).wait_stream(side)
        return graph

    def flops_per_step(self) -> int:
        """Algorithmic FLOPs of one step: the linears (linear_pos on 2t - 1 rows per layer) and
        the attention products (content t x t, positional t x (2t - 1), context t x t, 8 x 128)."""
        lin = self.rows * (2 * D_FF * D_MODEL * 2 + 3 * D_MODEL * D_MODEL + D_MODEL * D_MODEL
                           + 2 * D_MODEL * D_MODEL + D_MODEL * D_MODEL) * 2
        pos = (2 * self.t - 1) * D_MODEL * D_MODEL * 2
        att = self.windows * 8 * 128 * 2 * (self.t * self.t * 2 + self.t * (2 * self.t - 1))
        return self.layers * (lin + pos + att)


class EncoderStem:
    """The subsampling stem (``parakeet_cuda/reference.py:11-30``) for ``windows`` windows of
    ``frames`` mel frames: ``forward(mel [windows, frames, 128])`` returns the encoder input
    ``[windows * t, 1024]`` (t = frames / 8, rounded up per stage) for ``EncoderBlocks``."""

    def __init__(self, model, runtime: Runtime, windows: int, frames: int, fp32_products: bool = False):
        from .pq8 import FLAG_FP32_PRODUCTS
        self.rt, self.windows, self.frames = runtime, windows, frames
        self.flags = FLAG_FP32_PRODUCTS if fp32_products else 0
        dev = runtime.device
        to_dev = lambda a: torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).to(dev)
        name = 'encoder.pre_encode.'
        self.w = {i: to_dev(np.asarray(model.array(f'{name}conv.{i}.weight')).reshape(256, -1)) for i in (0, 2, 3, 5, 6)}
        self.b = {i: to_dev(np.asarray(model.array(f'{name}conv.{i}.bias')).reshape(-1)) for i in (0, 2, 3, 5, 6)}
        up = runtime.uploader()
        self.w_out = up.pack([(model.raw(name + 'out.weight'), 4096)], 1024)
        up.finish()
        self.b_out = to_dev(np.asarray(model.array(name + 'out.bias')).reshape(-1))
        t = frames
        for _ in range(3):
            t = (t + 1) // 2
        self.t = t
        self.ws = torch.empty(runtime.lib.stem_workspace_size(windows, frames), dtype=torch.uint8, device=dev)
        self.out = torch.empty(windows * t, D_MODEL, dtype=torch.float32, device=dev)

    def forward(self, mel: torch.Tensor) -> torch.Tensor:
        if tuple(mel.shape) != (self.windows, self.frames, 128) or mel.dtype != torch.float32:
            raise ValueError(f'mel must be float32 [{self.windows}, {self.frames}, 128]')
        mel = mel.contiguous()
        w, b = self.w, self.b
        self.rt.lib.call('pq8_stem', mel.data_ptr(), self.windows, self.frames, w[0].data_ptr(), b[0].data_ptr(),
                         w[2].data_ptr(), b[2].data_ptr(), w[3].data_ptr(), b[3].data_ptr(), w[5].data_ptr(),
                         b[5].data_ptr(), w[6].data_ptr(), b[6].data_ptr(), self.w_out.pointer, self.b_out.data_ptr(),
                         self.out.data_ptr(), self.flags, self.ws.data_ptr(), self.ws.numel(), self.rt.stream())
        return self.out
