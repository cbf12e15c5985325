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


class BatchDecoder64:
    """``Decoder64`` for many independent streams at once (float64).

    Row ``i`` is stream ``i``'s predictor/joint state; ``predict(rows, tokens)``
    and ``joint(rows, frames)`` run the same arithmetic as ``Decoder64`` on the
    selected rows with one matrix product per weight, so a 64-stream decode of
    1000+ steps finishes in seconds. Per row it is ``Decoder64`` exactly
    (``decoder.py:6-34``); only the summation order of the float64 products
    differs, which no arg-max decision of a float32 implementation can see.
    """

    def __init__(self, model, streams: int, layers: int = 2, hidden: int = 640):
        one = Decoder64(model, layers, hidden)
        self.w, self.embed, self.layers, self.hidden = one.w, one.embed, layers, hidden
        self.h = np.zeros((layers, streams, hidden))
        self.c = np.zeros((layers, streams, hidden))
        self.h_new = np.zeros_like(self.h)
        self.c_new = np.zeros_like(self.c)
        self.pred = np.zeros((streams, self.w['joint.pred.weight'].shape[0]))

    def predict(self, rows, tokens):
        rows = np.asarray(rows, np.int64)
        x = self.embed[np.asarray(tokens, np.int64)]
        for l in range(self.layers):
            ih = f'decoder.prediction.dec_rnn.lstm.ih_l{l}'
            hh = f'decoder.prediction.dec_rnn.lstm.hh_l{l}'
            gates = (x @ self.w[ih + '.weight'].T + self.w[ih + '.bias']
                     + self.h[l, rows] @ self.w[hh + '.weight'].T + self.w[hh + '.bias'])
            gi, gf, gg, go = (gates[:, j * self.hidden:(j + 1) * self.hidden] for j in range(4))
            c = sigmoid(gf) * self.c[l, rows] + sigmoid(gi) * np.tanh(gg)
            h = sigmoid(go) * np.tanh(c)
            self.h_new[l, rows], self.c_new[l, rows] = h, c
            x = h
        self.pred[rows] = x @ self.w['joint.pred.weight'].T + self.w['joint.pred.bias']

    def joint(self, rows, frames):
        """Joint logits ``[len(rows), 8198]`` of the selected rows."""
        act = np.maximum(np.asarray(frames, np.float64) + self.pred[np.asarray(rows, np.int64)], 0.0)
        return act @ self.w['joint.joint_net.2.weight'].T + self.w['joint.joint_net.2.bias']

    def commit(self, rows):
        rows = np.asarray(rows, np.int64)
        self.h[:, rows], self.c[:, rows] = self.h_new[:, rows], self.c_new[:, rows]


def greedy_decode_streams(projected, model, durations, follow=None, tie_eps: float = 0.0):
    """``greedy_decode`` of every stream in ``projected`` (a list of ``[T_i, 640]``
    arrays), run in lock step on ``BatchDecoder64``.

    Each stream follows ``decoder.py:78-97`` on its own: the loop below is the
    single-stream loop of ``greedy_decode`` with its local variables turned
    into per-stream arrays, and one joint call per live stream per step.
    Returns one result dict per stream (as ``greedy_decode``) with two extras:
    ``min_margin``, the smallest top-2 token-logit gap over the stream's calls,
    and ``ties``, the calls decided by ``follow`` (below).

    ``follow``: per stream, the ``decode_trace`` of an implementation under
    test. Where its decision (token, frames skipped) differs from this
    oracle's, it is adopted if it is a near-tie: its token's logit is within
    ``tie_eps`` of the largest token logit, and one duration that gives its
    skip is within ``tie_eps`` of the largest duration logit. A float32
    implementation may break such a tie either way. Any other difference ends
    the stream and is reported in ``mismatch`` (call index, both decisions and
    the logit gaps).
    """
    b = len(projected)
    dec = BatchDecoder64(model, b)
    out = [{'tokens': [], 'decode_trace': [], 'joint_calls': 0, 'min_margin': np.inf, 'ties': 0, 'mismatch': None}
           for _ in range(b)]
    frame = np.zeros(b, np.int64)
    emitted = np.zeros(b, np.int64)
    previous = np.full(b, BLANK, np.int64)
    needs_predict = np.ones(b, bool)
    lengths = np.array([len(p) for p in projected], np.int64)
    while True:
        live = np.flatnonzero(frame < lengths)
        if live.size == 0:
            return out
        todo = live[needs_predict[live]]
        if todo.size:
            dec.predict(todo, previous[todo])
            needs_predict[todo] = False
        logits = dec.joint(live, np.stack([projected[i][frame[i]] for i in live]))
        tok_logits, dur_logits = logits[:, :TOKENS], logits[:, TOKENS:]
        tok = np.argmax(tok_logits, axis=1)
        dur = np.argmax(dur_logits, axis=1)
        top2 = np.partition(tok_logits, TOKENS - 2, axis=1)[:, -2:]
        margin = top2[:, 1] - top2[:, 0]
        commit = []
        for j, i in enumerate(live):
            r = out[i]
            call = r['joint_calls']
            r['joint_calls'] += 1
            r['min_margin'] = min(r['min_margin'], float(margin[j]))
            token, skip = int(tok[j]), durations[int(dur[j])]
            if token == BLANK and skip == 0:
                skip = 1
            if follow is not None:
                theirs = follow[i][call] if call < len(follow[i]) else None
                if theirs is None or int(theirs[0]) != frame[i]:
                    r['mismatch'] = {'call': call, 'oracle': [int(frame[i]), token, skip], 'theirs': theirs}
                    lengths[i] = frame[i]
                    continue
                if (int(theirs[1]), int(theirs[2])) != (token, skip):
                    t_tok, t_skip = int(theirs[1]), int(theirs[2])
                    tok_gap = float(tok_logits[j].max() - tok_logits[j, t_tok]) if 0 <= t_tok < TOKENS else np.inf
                    cands = [d for d, s in enumerate(durations) if s == t_skip]
                    if t_tok == BLANK and t_skip == 1:
                        cands += [d for d, s in enumerate(durations) if s == 0]
                    dur_gap = min((float(dur_logits[j].max() - dur_logits[j, d]) for d in cands), default=np.inf)
                    if tok_gap > tie_eps or dur_gap > tie_eps:
                        r['mismatch'] = {'call': call, 'oracle': [int(frame[i]), token, skip],
                                         'theirs': [int(v) for v in theirs], 'token_gap': tok_gap,
                                         'duration_gap': dur_gap}
                        lengths[i] = frame[i]
                        continue
                    token, skip = t_tok, t_skip
                    r['ties'] += 1
            r['decode_trace'].append([int(frame[i]), token, skip])
            if token != BLANK:
                r['tokens'].append(token)
                previous[i] = token
                commit.append(i)
                needs_predict[i] = True
            emitted[i] += 1
            frame[i] += skip
            if skip:
                emitted[i] = 0
            elif emitted[i] == MAX_SYMBOLS:
                frame[i] += 1
                emitted[i] = 0
        if commit:
            dec.commit(commit)
