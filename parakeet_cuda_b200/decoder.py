"""TDT prediction/joint network on resident packed Q8_0 weights (decoder regime).

``PQ8Decoder`` is the counterpart of the reference's ``CUDADecoder``
(``parakeet_cuda/decoder.py:37-75``) and speaks the same duck-typed protocol
(``predict(token)``, ``joint(frame) -> (token, duration)``, ``commit()``), so
it also plugs into the reference's own ``decode()`` loop. It runs ``batch``
independent streams at once (rows of every buffer), which is what the batched
greedy loop in ``parakeet_cuda_b200.tdt`` uses.

Per predict: two fused LSTM-layer kernels (both gate GEMVs + cell update in
one launch each; layer 0 reads the fp16 embedding row on the device) and the
joint.pred GEMV. Per joint: one fused kernel (ReLU(enc + pred), 640 -> 8198
GEMV, bias, arg-max over tokens and durations). The reference needs 5 SGEMMs
plus 6 elementwise launches per predict and 4 launches per joint.
"""
from __future__ import annotations

import numpy as np
import torch

from .pq8 import EPI_NONE, GEMV_MAX_M, LAYOUT_GATES4
from .runtime import PackedWeight, Runtime

HIDDEN = 640
LAYERS = 2
VOCAB = 8193


class PQ8Decoder:
    """Prediction/joint network for ``batch`` streams. Every launch covers all
    streams (up to ``PQ8_GEMV_MAX_M``; beyond 8 rows the kernels run their row
    groups side by side in one grid)."""

    MAX_BATCH = GEMV_MAX_M

    def __init__(self, model, runtime: Runtime, batch: int = 1, keep_logits: bool = False):
        if not 1 <= batch <= self.MAX_BATCH:
            raise ValueError(f'batch must be in [1, {self.MAX_BATCH}]')
        self.model, self.rt, self.batch = model, runtime, batch
        dev = runtime.device
        self.lstm = []
        for l in range(LAYERS):
            ih, hh = f'decoder.prediction.dec_rnn.lstm.ih_l{l}', f'decoder.prediction.dec_rnn.lstm.hh_l{l}'
            n, k_in = model.tensors[ih + '.weight'].shape
            k_h = model.tensors[hh + '.weight'].shape[1]
            # [W_ih | W_hh] side by side along K, repacked on the device
            w = runtime.uploader().pack([(model.raw(ih + '.weight'), k_in), (model.raw(hh + '.weight'), k_h)], n,
                                        LAYOUT_GATES4)
            bias = (np.asarray(model.array(ih + '.bias'), np.float32).reshape(-1)
                    + np.asarray(model.array(hh + '.bias'), np.float32).reshape(-1))
            self.lstm.append((w, torch.from_numpy(bias).to(dev), k_in))
        runtime.load_weights(model, ['decoder.prediction.embed.weight', 'joint.pred.weight', 'joint.pred.bias',
                                     'joint.joint_net.2.weight', 'joint.joint_net.2.bias'])
        self.embed = runtime.weight('decoder.prediction.embed.weight')  # fp16 [vocab, 640]
        self.w_pred: PackedWeight = runtime.weight('joint.pred.weight')
        self.b_pred = runtime.weight('joint.pred.bias').reshape(-1)
        self.w_joint: PackedWeight = runtime.weight('joint.joint_net.2.weight')
        self.b_joint = runtime.weight('joint.joint_net.2.bias').reshape(-1)
        self.n_out = self.w_joint.n
        f32 = dict(dtype=torch.float32, device=dev)
        self.h = torch.zeros(LAYERS, batch, HIDDEN, **f32)
        self.c = torch.zeros(LAYERS, batch, HIDDEN, **f32)
        self.hn = torch.zeros(LAYERS, batch, HIDDEN, **f32)
        self.cn = torch.zeros(LAYERS, batch, HIDDEN, **f32)
        self.pred = torch.zeros(batch, HIDDEN, **f32)
        self.enc = torch.zeros(batch, HIDDEN, **f32)
        # joint logits are written only on request (the greedy loop needs the ids alone)
        self.logits = torch.zeros(batch, self.n_out, **f32) if keep_logits else None
        self.tokens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.enc_rows = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.commit_mask = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.ids = torch.zeros(batch, 2, dtype=torch.int32, device=dev)
        self.ids_host = torch.zeros(batch, 2, dtype=torch.int32).pin_memory()
        for l in range(LAYERS):
            runtime.ensure_workspace(batch, 4 * HIDDEN, self.lstm[l][2] + HIDDEN)
        runtime.ensure_workspace(batch, self.n_out, HIDDEN)
        runtime.ensure_workspace(batch, HIDDEN, HIDDEN)
        self.predict_calls = self.joint_calls = 0

    # -- batched device-side steps ------------------------------------------
    def predict_device(self, tokens: torch.Tensor | None = None):
        """Candidate LSTM state and joint.pred output for all rows from ``self.tokens``."""
        if tokens is not None:
            self.tokens.copy_(tokens, non_blocking=True)
        rt, lib, ws = self.rt, self.rt.lib, self.rt.workspace
        st = rt.stream()
        m = self.batch
        for l, (w, bias, k_in) in enumerate(self.lstm):
            x = None if l == 0 else self.hn[l - 1].data_ptr()
            embed = self.embed.data_ptr() if l == 0 else None
            toks = self.tokens.data_ptr() if l == 0 else None
            lib.call('pq8_lstm_layer', w.pointer, x, embed, toks, self.h[l].data_ptr(), self.c[l].data_ptr(),
                     bias.data_ptr(), self.hn[l].data_ptr(), self.cn[l].data_ptr(), m, HIDDEN, k_in, ws.data_ptr(),
                     ws.numel(), st)
        lib.call('pq8_gemv', self.w_pred.pointer, self.hn[LAYERS - 1].data_ptr(), self.pred.data_ptr(),
                 self.b_pred.data_ptr(), None, m, self.w_pred.n, self.w_pred.k, EPI_NONE, 1.0, ws.data_ptr(),
                 ws.numel(), st)
        self.predict_calls += 1

    def joint_device(self, enc: torch.Tensor, enc_rows: torch.Tensor | None = None):
        """Token/duration ids of all rows into ``self.ids`` (device); ``enc`` rows selected by ``enc_rows``."""
        rows = None
        if enc_rows is not None:
            if enc_rows.data_ptr() != self.enc_rows.data_ptr():  # a device loop writes self.enc_rows itself
                self.enc_rows.copy_(enc_rows, non_blocking=True)
            rows = self.enc_rows.data_ptr()
        ws = self.rt.workspace
        self.rt.lib.call('pq8_joint_argmax', self.w_joint.pointer, enc.data_ptr(), rows, self.pred.data_ptr(),
                         self.b_joint.data_ptr(), None if self.logits is None else self.logits.data_ptr(),
                         self.ids.data_ptr(), self.batch,
                         self.n_out, self.w_joint.k, VOCAB, ws.data_ptr(), ws.numel(), self.rt.stream())
        self.joint_calls += 1

    def commit_rows(self, mask: torch.Tensor):
        """Rows with ``mask != 0`` adopt their candidate state."""
        if mask.data_ptr() != self.commit_mask.data_ptr():  # a device loop writes self.commit_mask itself
            self.commit_mask.copy_(mask, non_blocking=True)
        self.rt.lib.call('pq8_tdt_commit', self.h.data_ptr(), self.c.data_ptr(), self.hn.data_ptr(),
                         self.cn.data_ptr(), self.commit_mask.data_ptr(), self.batch, LAYERS, HIDDEN,
                         self.rt.stream())

    def reset_state(self):
        """Zero the LSTM state of every row (a fresh decode)."""
        for t in (self.h, self.c, self.hn, self.cn, self.pred):
            t.zero_()

    def read_ids(self) -> np.ndarray:
        self.ids_host.copy_(self.ids, non_blocking=True)
        torch.cuda.current_stream(self.rt.device).synchronize()
        return self.ids_host.numpy()

    # -- reference protocol (single stream) ----------------------------------
    def predict(self, token: int):
        self.predict_device(torch.full((self.batch,), int(token), dtype=torch.int32))

    def joint(self, frame):
        row = torch.from_numpy(np.array(frame, np.float32).reshape(1, HIDDEN))
        self.enc.copy_(row.expand(self.batch, HIDDEN))
        self.joint_device(self.enc)
        ids = self.read_ids()
        return int(ids[0, 0]), int(ids[0, 1])

    def commit(self):
        if self.batch == 1:
            self.h, self.hn = self.hn, self.h
            self.c, self.cn = self.cn, self.c
        else:
            self.commit_rows(torch.ones(self.batch, dtype=torch.int32))
