"""Greedy TDT token loop (host state machine) for one or many streams.

The rules follow the reference's ``decode`` (``parakeet_cuda/decoder.py:78-97``):
blank id 8192; durations from the model metadata; at most 10 symbols per
frame; a blank with duration 0 advances one frame; the predictor runs only
after an emitted token; an emitted token commits the candidate LSTM state.

``greedy_decode`` drives any decoder with the reference protocol
(``predict``/``joint``/``commit``). ``greedy_decode_batch`` drives a
``PQ8Decoder`` over B independent streams in lock-step: one fused joint launch
per step for all streams, one predict for all streams whenever any stream
needs it (a stream whose inputs did not change gets bit-identical candidates
again, so this is equivalent to predicting it alone), and a masked commit.
``greedy_decode_device`` runs the same loop without the host: the control
rules and the commit run in one kernel (``pq8_tdt_advance``), so a step is a
fixed launch sequence (predict, joint, advance) replayed from a CUDA graph of
several steps, and the host only polls how many streams remain between
replays. It predicts every step: a stream that emitted nothing recomputes
bit-identical candidates, so the results equal ``greedy_decode_batch``'s.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
import time

import numpy as np
import torch

from .decoder import HIDDEN, LAYERS

BLANK = 8192
MAX_SYMBOLS = 10
FRAME_SECONDS = 0.08


@dataclass
class Stream:
    """State of one stream's greedy loop between joint calls."""
    frames: int
    t: int = 0
    symbols: int = 0
    previous: int = BLANK
    needs_predict: bool = True
    tokens: list = field(default_factory=list)
    token_times: list = field(default_factory=list)
    trace: list = field(default_factory=list)
    calls: int = 0

    @property
    def done(self) -> bool:
        return self.t >= self.frames

    def advance(self, token: int, dur_index: int, durations) -> bool:
        """Apply one joint result; returns True when the candidate state must be committed."""
        self.calls += 1
        skip = durations[dur_index]
        if token == BLANK and skip == 0:
            skip = 1
        self.trace.append([self.t, token, skip])
        commit = token != BLANK
        if commit:
            self.tokens.append(token)
            self.token_times.append([self.t * FRAME_SECONDS, (self.t + max(1, skip)) * FRAME_SECONDS])
            self.previous = token
            self.needs_predict = True
        self.symbols += 1
        self.t += skip
        if skip:
            self.symbols = 0
        elif self.symbols == MAX_SYMBOLS:
            self.t += 1
            self.symbols = 0
        return commit

    def result(self) -> dict:
        return {'tokens': self.tokens, 'token_times': self.token_times, 'decode_trace': self.trace,
                'joint_calls': self.calls}


def greedy_decode(projected, decoder, durations) -> dict:
    """One stream through any decoder with the reference's predict/joint/commit protocol."""
    s = Stream(len(projected))
    while not s.done:
        if s.needs_predict:
            decoder.predict(s.previous)
            s.needs_predict = False
        token, dur = decoder.joint(projected[s.t])
        if s.advance(token, dur, durations):
            decoder.commit()
    return s.result()


def greedy_decode_batch(projected, decoder, durations, max_steps: int | None = None) -> list:
    """B streams (``projected[b]`` = frames of stream b, [T_b, 640]) on a batched PQ8Decoder."""
    b = decoder.batch
    if len(projected) != b:
        raise ValueError(f'decoder has {b} rows, got {len(projected)} streams')
    t_max = max(len(p) for p in projected)
    table = np.zeros((b * max(t_max, 1), projected[0].shape[1]), np.float32)
    for i, p in enumerate(projected):
        table[i * t_max:i * t_max + len(p)] = p
    dev = decoder.rt.device
    enc = torch.from_numpy(table).to(dev)
    streams = [Stream(len(p)) for p in projected]
    tokens_h = torch.zeros(b, dtype=torch.int32).pin_memory()
    rows_h = torch.zeros(b, dtype=torch.int32).pin_memory()
    mask_h = torch.zeros(b, dtype=torch.int32).pin_memory()
    steps = 0
    while any(not s.done for s in streams):
        if max_steps is not None and steps >= max_steps:
            break
        if any(s.needs_predict and not s.done for s in streams):
            tokens_h.copy_(torch.tensor([s.previous for s in streams], dtype=torch.int32))
            decoder.predict_device(tokens_h)
            for s in streams:
                s.needs_predict = False
        rows_h.copy_(torch.tensor([i * t_max + min(s.t, s.frames - 1) for i, s in enumerate(streams)],
                                  dtype=torch.int32))
        decoder.joint_device(enc, rows_h)
        ids = decoder.read_ids()
        commit = [0] * b
        for i, s in enumerate(streams):
            if not s.done:
                commit[i] = int(s.advance(int(ids[i, 0]), int(ids[i, 1]), durations))
        if any(commit):
            mask_h.copy_(torch.tensor(commit, dtype=torch.int32))
            decoder.commit_rows(mask_h)
        steps += 1
    return [s.result() for s in streams]


def greedy_decode_device(projected, decoder, durations, steps_per_graph: int = 16,
                         max_steps: int | None = None) -> list:
    """B streams (``projected[b]`` = frames of stream b, [T_b, 640], a host array or a
    device tensor) on a batched PQ8Decoder, with the greedy control on the device;
    same results as ``greedy_decode_batch``. ``decoder.loop_seconds`` records the
    wall time of the replay loop alone (first replay to the last poll)."""
    b = decoder.batch
    if len(projected) != b:
        raise ValueError(f'decoder has {b} rows, got {len(projected)} streams')
    rt, dev = decoder.rt, decoder.rt.device
    frames = [int(p.shape[0]) for p in projected]
    t_max = max(max(frames), 1)
    # frame table [b * t_max, 640] on the device: stream i's frames at rows i * t_max ...
    enc = torch.zeros(b * t_max, int(projected[0].shape[1]), dtype=torch.float32, device=dev)
    for i, p in enumerate(projected):
        if frames[i]:
            src = p if isinstance(p, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(p, np.float32))
            enc[i * t_max:i * t_max + frames[i]].copy_(src)
    cap = t_max * MAX_SYMBOLS  # a frame takes at most MAX_SYMBOLS joint calls
    i32 = dict(dtype=torch.int32, device=dev)
    state = torch.zeros(b, 8, dtype=torch.int32)
    state[:, 0] = torch.tensor(frames, dtype=torch.int32)
    state[:, 3] = BLANK
    state[:, 6] = (state[:, 0] == 0).to(torch.int32)
    state = state.to(dev)
    dur = torch.tensor(list(durations), **i32)
    emitted = torch.zeros(b, cap, 3, **i32)
    trace = torch.zeros(b, cap, 3, **i32)
    remaining = torch.zeros(1, **i32)
    decoder.reset_state()
    decoder.tokens.fill_(BLANK)
    decoder.enc_rows.copy_(torch.arange(b, dtype=torch.int32) * t_max)
    lib = rt.lib

    def step():
        decoder.predict_device()
        decoder.joint_device(enc, decoder.enc_rows)
        # control and commit in one launch
        lib.call('pq8_tdt_advance', decoder.ids.data_ptr(), dur.data_ptr(), dur.numel(), state.data_ptr(), b,
                 t_max, decoder.tokens.data_ptr(), decoder.enc_rows.data_ptr(), decoder.commit_mask.data_ptr(),
                 emitted.data_ptr(), cap, trace.data_ptr(), cap, remaining.data_ptr(), decoder.h.data_ptr(),
                 decoder.c.data_ptr(), decoder.hn.data_ptr(), decoder.cn.data_ptr(), LAYERS, HIDDEN, rt.stream())

    # Kernel attributes and workspaces are set up outside the capture: this
    # predict/joint pair computes exactly what the first step will compute.
    decoder.predict_device()
    decoder.joint_device(enc, decoder.enc_rows)
    torch.cuda.synchronize(dev)
    # capture_begin/end rather than the torch.cuda.graph context, which also
    # runs a garbage collection and empties the allocator cache on entry.
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        graph.capture_begin()
        try:
            for _ in range(steps_per_graph):
                step()
        finally:
            graph.capture_end()
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize(dev)
    t_loop = time.perf_counter()
    steps = 0
    limit = max_steps if max_steps is not None else None
    while limit is None or steps < limit:
        if limit is not None and limit - steps < steps_per_graph:
            for _ in range(limit - steps):
                step()
            steps = limit
        else:
            graph.replay()
            steps += steps_per_graph
        if int(remaining.item()) == 0 and steps > 0:
            break
    torch.cuda.synchronize(dev)
    decoder.loop_seconds = time.perf_counter() - t_loop
    del graph
    decoder.steps = steps
    status = rt.device_status()
    if status:
        raise RuntimeError(f'device status {status} after the device TDT loop')
    return _device_results(state, emitted, trace, b)


def _device_results(state, emitted, trace, b: int) -> list:
    """Per-stream results from the device records of pq8_tdt_control's layout."""
    st = state.cpu().numpy()
    # only the filled prefix of the per-stream records crosses to the host
    em = emitted[:, :max(1, int(st[:, 4].max()))].cpu().numpy()
    tr = trace[:, :max(1, int(st[:, 5].max()))].cpu().numpy()
    out = []
    for i in range(b):
        ne, nc = int(st[i, 4]), int(st[i, 5])
        t = em[i, :ne, 1].astype(np.float64)
        span = np.maximum(1, em[i, :ne, 2]).astype(np.float64)
        out.append({
            'tokens': em[i, :ne, 0].tolist(),
            'token_times': np.stack([t * FRAME_SECONDS, (t + span) * FRAME_SECONDS], axis=1).tolist(),
            'decode_trace': tr[i, :nc].tolist(),
            'joint_calls': nc,
        })
    return out


def greedy_decode_persistent(projected, decoder, durations, max_steps: int | None = None,
                             steps_per_launch: int | None = None) -> list:
    """B <= 64 streams (``projected[b]`` = frames of stream b, [T_b, 640], a host
    array or a device tensor) through ``pq8_tdt_decode``: the whole greedy loop
    in one persistent launch on ``decoder``'s resident weights (or one launch
    per ``steps_per_launch`` lock-step steps, each resuming the last). Same
    results as ``greedy_decode_batch`` up to the order of FP32 additions in the
    products. ``decoder.loop_seconds`` = device time of the launches (CUDA
    events), ``decoder.steps`` = lock-step steps."""
    from .decoder import VOCAB
    from .pq8 import TdtWeights
    b = len(projected)
    if not 1 <= b <= 64:
        raise ValueError(f'pq8_tdt_decode takes 1..64 streams, got {b}')
    rt, dev = decoder.rt, decoder.rt.device
    frames = [int(p.shape[0]) for p in projected]
    t_max = max(max(frames), 1)
    enc = torch.zeros(b * t_max, int(projected[0].shape[1]), dtype=torch.float32, device=dev)
    for i, p in enumerate(projected):
        if frames[i]:
            src = p if isinstance(p, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(p, np.float32))
            enc[i * t_max:i * t_max + frames[i]].copy_(src)
    cap = t_max * MAX_SYMBOLS
    i32 = dict(dtype=torch.int32, device=dev)
    state = torch.zeros(b, 8, dtype=torch.int32)
    state[:, 0] = torch.tensor(frames, dtype=torch.int32)
    state[:, 3] = BLANK
    state[:, 6] = (state[:, 0] == 0).to(torch.int32)
    state = state.to(dev)
    dur = torch.tensor(list(durations), **i32)
    emitted = torch.zeros(b, cap, 3, **i32)
    trace = torch.zeros(b, cap, 3, **i32)
    counters = torch.zeros(2, **i32)  # steps run, streams remaining
    w = TdtWeights()
    for l in range(LAYERS):
        w.lstm[l] = decoder.lstm[l][0].pointer
        w.lstm_bias[l] = decoder.lstm[l][1].data_ptr()
    w.pred, w.pred_bias = decoder.w_pred.pointer, decoder.b_pred.data_ptr()
    w.joint, w.joint_bias = decoder.w_joint.pointer, decoder.b_joint.data_ptr()
    w.embed = decoder.embed.data_ptr()
    w.hidden, w.embed_k, w.joint_k = HIDDEN, decoder.lstm[0][2], decoder.w_joint.k
    w.n_joint, w.vocab = decoder.n_out, VOCAB
    lib = rt.lib
    ws = torch.empty(lib.tdt_decode_workspace_size(b, HIDDEN, w.joint_k), dtype=torch.uint8, device=dev)
    # a stream of T frames takes at most T * MAX_SYMBOLS joint calls
    limit = cap if max_steps is None else max_steps
    per = steps_per_launch or max(limit, 1)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st = rt.stream()
    steps, resume, seconds = 0, 0, 0.0
    while steps < limit or (steps == 0 and limit == 0):
        n = min(per, limit - steps)
        e0.record()
        lib.call('pq8_tdt_decode', C.byref(w), enc.data_ptr(), t_max, dur.data_ptr(), dur.numel(), state.data_ptr(),
                 b, emitted.data_ptr(), cap, trace.data_ptr(), cap, n, resume, counters[0:1].data_ptr(),
                 counters[1:2].data_ptr(), ws.data_ptr(), ws.numel(), st)
        e1.record()
        e1.synchronize()
        seconds += e0.elapsed_time(e1) / 1e3
        ran, remaining = (int(v) for v in counters.cpu().tolist())
        steps += ran
        resume = 1
        if remaining == 0 or ran < n or n == 0:
            break
    decoder.loop_seconds, decoder.steps = seconds, steps
    status = rt.device_status()
    if status:
        raise RuntimeError(f'device status {status} after pq8_tdt_decode')
    return _device_results(state, emitted, trace, b)


# Streams up to which the persistent launch beats the graph-replayed loop
# (measured per lock-step step on the config-3 decode: 16.8-17.4 vs 20.4 us
# at one stream, 45.1 vs 52.0 at 16, 64.9 vs 58.6 at 24, 150 vs 96 at 64).
PERSISTENT_MAX_STREAMS = 16


def greedy_decode_gpu(projected, decoder, durations) -> list:
    """The faster device decode for this many streams: ``greedy_decode_persistent``
    up to ``PERSISTENT_MAX_STREAMS`` streams, else ``greedy_decode_device`` (which
    needs ``decoder.batch == len(projected)``). Same results either way, up to the
    order of FP32 additions in the products."""
    if len(projected) <= PERSISTENT_MAX_STREAMS:
        return greedy_decode_persistent(projected, decoder, durations)
    return greedy_decode_device(projected, decoder, durations)
