"""NumPy restatement of the reference's TDT prediction/joint network and greedy loop.

Test infrastructure only (see ``oracle/__init__.py``).

Reference citations (mgostIH/parakeet_cuda):

* Predictor (2-layer LSTM, gate order i, f, g, o) and joint: ``parakeet_cuda/decoder.py:6-34``
  (``CPUDecoder``), CUDA tails ``lstm`` ``runtime.cu:155-163``, ``joint_relu``
  ``runtime.cu:164-166``, ``argmax_tdt`` ``runtime.cu:167-179`` (ties -> lowest index).
* Greedy TDT loop: ``parakeet_cuda/decoder.py:78-97`` (blank 8192, at most 10
  symbols per frame, blank with duration 0 advances one frame, the predictor
  runs only after an emitted token).

The arithmetic here is float64 from the decoded Q8_0 weights, so it is an
independent check of the float32 reference rather than a copy of it.
"""
from __future__ import annotations

import numpy as np

from .q8 import decode, sigmoid

BLANK = 8192
TOKENS = 8193
MAX_SYMBOLS = 10
FRAME_SECONDS = 0.08


def _q8(model, name):
    t = model.tensors[name]
    if t.kind == 8:
        return decode(model.raw(name), *t.shape)
    return np.asarray(model.array(name), np.float64)


class Decoder64:
    """Float64 predictor/joint with the ``predict`` / ``joint`` / ``commit`` protocol."""

    def __init__(self, model, layers: int = 2, hidden: int = 640):
        self.model, self.layers, self.hidden = model, layers, hidden
        self.w = {}
        for l in range(layers):
            for kind in ('ih', 'hh'):
                base = f'decoder.prediction.dec_rnn.lstm.{kind}_l{l}'
                self.w[base + '.weight'] = _q8(model, base + '.weight')
                self.w[base + '.bias'] = _q8(model, base + '.bias').reshape(-1)
        for name in ('joint.pred', 'joint.joint_net.2'):
            self.w[name + '.weight'] = _q8(model, name + '.weight')
            self.w[name + '.bias'] = _q8(model, name + '.bias').reshape(-1)
        self.embed = np.asarray(model.array('decoder.prediction.embed.weight'), np.float64)
        self.h = np.zeros((layers, hidden))
        self.c = np.zeros((layers, hidden))
        self.pending = None
        self.pred = None
        self.last_logits = None

    def predict(self, token: int):
        x = self.embed[token]
        h_new, c_new = np.empty_like(self.h), np.empty_like(self.c)
        for l in range(self.layers):
            ih = f'decoder.prediction.dec_rnn.lstm.ih_l{l}'
            hh = f'decoder.prediction.dec_rnn.lstm.hh_l{l}'
            gates = (self.w[ih + '.weight'] @ x + self.w[ih + '.bias']
                     + self.w[hh + '.weight'] @ self.h[l] + self.w[hh + '.bias'])
            gi, gf, gg, go = gates.reshape(4, self.hidden)
            c_new[l] = sigmoid(gf) * self.c[l] + sigmoid(gi) * np.tanh(gg)
            h_new[l] = sigmoid(go) * np.tanh(c_new[l])
            x = h_new[l]
        self.pending = (h_new, c_new)
        self.pred = self.w['joint.pred.weight'] @ x + self.w['joint.pred.bias']

    def joint(self, frame):
        act = np.maximum(np.asarray(frame, np.float64) + self.pred, 0.0)
        logits = self.w['joint.joint_net.2.weight'] @ act + self.w['joint.joint_net.2.bias']
        self.last_logits = logits
        return argmax_tdt(logits)

    def commit(self):
        self.h, self.c = self.pending


def argmax_tdt(logits):
    """(token, duration index); ties resolve to the lowest index."""
    logits = np.asarray(logits)
    return int(np.argmax(logits[:TOKENS])), int(np.argmax(logits[TOKENS:]))


def top2_margin(logits) -> float:
    """Gap between the two largest token logits (how close a call was to a tie)."""
    s = np.sort(np.asarray(logits[:TOKENS], np.float64))
    return float(s[-1] - s[-2])


def greedy_decode(projected, decoder, durations):
    """Greedy TDT loop over encoder frames ``projected[t]`` (already joint.enc-projected).

    Returns the emitted token ids, the per-call trace ``[frame, token, skip]``
    and the number of joint calls, as ``decoder.py:78-97`` defines them.
    """
    tokens, trace = [], []
    previous, needs_predict, frame, calls = BLANK, True, 0, 0
    while frame < len(projected):
        emitted, skip = 0, 0
        while emitted < MAX_SYMBOLS:
            if needs_predict:
                decoder.predict(previous)
                needs_predict = False
            token, dur = decoder.joint(projected[frame])
            calls += 1
            skip = durations[dur]
            if token == BLANK and skip == 0:
                skip = 1
            trace.append([frame, token, skip])
            if token != BLANK:
                tokens.append(token)
                previous = token
                decoder.commit()
                needs_predict = True
            emitted += 1
            frame += skip
            if skip:
                break
        if emitted == MAX_SYMBOLS and skip == 0:
            frame += 1
    return {'tokens': tokens, 'decode_trace': trace, 'joint_calls': calls}


def lstm_cell(gates, c_prev):
    """One LSTM cell from pre-activation gates ``[4, H]`` (order i, f, g, o)."""
    gi, gf, gg, go = np.asarray(gates, np.float64).reshape(4, -1)
    c = sigmoid(gf) * c_prev + sigmoid(gi) * np.tanh(gg)
    return sigmoid(go) * np.tanh(c), c
