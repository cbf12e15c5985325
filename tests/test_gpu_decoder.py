"""GPU parity of the decoder regime: fused LSTM layer, fused joint + arg-max,
and the greedy TDT loop against the reference's golden token ids."""
import ctypes as C
import json

import numpy as np
import pytest
import torch

from oracle import q8, tdt as otdt
from parakeet_cuda_b200 import pq8
from parakeet_cuda_b200.decoder import PQ8Decoder
from parakeet_cuda_b200.runtime import Runtime, pack_concat_host
from parakeet_cuda_b200.synthetic import SyntheticParakeet, q8_0_blocks
from parakeet_cuda_b200.tdt import (greedy_decode, greedy_decode_batch, greedy_decode_device, greedy_decode_gpu,
                                     greedy_decode_persistent)

pytestmark = pytest.mark.gpu

DURATIONS = [0, 1, 2, 3, 4]


@pytest.fixture(scope='module')
def rt():
    return Runtime(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize('m', [1, 3, 8, 19, 64])
def test_lstm_layer_matches_oracle(rt, m):
    rng = np.random.default_rng(20 + m)
    hid, k_in = 640, 640
    w_ih, w_hh = q8_0_blocks(rng, 4 * hid, k_in, 2e-4, 1.2e-3), q8_0_blocks(rng, 4 * hid, hid, 2e-4, 1.2e-3)
    packed = pack_concat_host([(w_ih, k_in), (w_hh, hid)], 4 * hid, pq8.LAYOUT_GATES4)
    w = rt.upload_packed(packed, 4 * hid, k_in + hid, pq8.LAYOUT_GATES4)
    x = rng.normal(size=(m, k_in)).astype(np.float32)
    h = np.tanh(rng.normal(size=(m, hid))).astype(np.float32)
    c = rng.normal(size=(m, hid)).astype(np.float32)
    bias = (0.1 * rng.normal(size=4 * hid)).astype(np.float32)
    h_out, c_out = torch.empty(m, hid, device='cuda'), torch.empty(m, hid, device='cuda')
    rt.ensure_workspace(m, 4 * hid, k_in + hid)
    ws = rt.workspace
    xd, hd, cd, bd = dev(x), dev(h), dev(c), dev(bias)  # keep the device copies alive across the launch
    rt.lib.call('pq8_lstm_layer', w.pointer, xd.data_ptr(), None, None, hd.data_ptr(), cd.data_ptr(),
                bd.data_ptr(), h_out.data_ptr(), c_out.data_ptr(), m, hid, k_in, ws.data_ptr(), ws.numel(),
                rt.stream())
    gates = q8.gemm(x, w_ih, 4 * hid, k_in) + q8.gemm(h, w_hh, 4 * hid, hid) + bias
    for i in range(m):
        hr, cr = otdt.lstm_cell(gates[i], c[i])
        np.testing.assert_allclose(h_out[i].cpu().numpy(), hr, atol=2e-5, rtol=1e-4)
        np.testing.assert_allclose(c_out[i].cpu().numpy(), cr, atol=2e-5, rtol=1e-4)


def test_lstm_layer_embedding_input(rt):
    model = SyntheticParakeet(seed=3, encoder_layers=0)
    d = PQ8Decoder(model, rt, batch=2)
    o = otdt.Decoder64(model)
    for tok in (8192, 17):
        d.predict_device(torch.tensor([tok, tok], dtype=torch.int32))
        o.predict(tok)
        np.testing.assert_allclose(d.pred[0].cpu().numpy(), o.pred, atol=1e-4, rtol=1e-4)
        np.testing.assert_allclose(d.pred[1].cpu().numpy(), o.pred, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize('m', [1, 5, 12, 64])
def test_joint_argmax_matches_oracle(rt, m):
    rng = np.random.default_rng(30 + m)
    n, k = 8198, 640
    raw = q8_0_blocks(rng, n, k, 2e-4, 1.2e-3)
    w = rt.pack(raw, n, k)
    enc = rng.normal(size=(3 * m, k)).astype(np.float32)
    rows = np.array([(2 * i + 1) % (3 * m) for i in range(m)], np.int32)
    pred = rng.normal(size=(m, k)).astype(np.float32)
    bias = (0.1 * rng.normal(size=n)).astype(np.float32)
    logits = torch.empty(m, n, device='cuda')
    ids = torch.empty(m, 2, dtype=torch.int32, device='cuda')
    rt.ensure_workspace(m, n, k)
    ws = rt.workspace
    ed, rd, pd, bd = dev(enc), dev(rows), dev(pred), dev(bias)
    for _ in range(2):  # second call checks the self-resetting tickets
        rt.lib.call('pq8_joint_argmax', w.pointer, ed.data_ptr(), rd.data_ptr(), pd.data_ptr(),
                    bd.data_ptr(), logits.data_ptr(), ids.data_ptr(), m, n, k, 8193, ws.data_ptr(),
                    ws.numel(), rt.stream())
        act = np.maximum(enc[rows] + pred, 0)
        gold = q8.gemm(act, raw, n, k) + bias
        np.testing.assert_allclose(logits.cpu().numpy(), gold, atol=2e-4, rtol=2e-4)
        got = ids.cpu().numpy()
        for i in range(m):
            assert tuple(got[i]) == otdt.argmax_tdt(gold[i]), (i, otdt.top2_margin(gold[i]))
    # without a logits buffer: the same ids
    ids2 = torch.full((m, 2), -1, dtype=torch.int32, device='cuda')
    rt.lib.call('pq8_joint_argmax', w.pointer, ed.data_ptr(), rd.data_ptr(), pd.data_ptr(), bd.data_ptr(), None,
                ids2.data_ptr(), m, n, k, 8193, ws.data_ptr(), ws.numel(), rt.stream())
    np.testing.assert_array_equal(ids2.cpu().numpy(), got)


def test_joint_argmax_ties_lowest_index(rt):
    """runtime.cu:167-179 / tests/test_cuda.py:78-82: ties resolve to the lowest index."""
    n, k = 8198, 32
    raw = np.zeros((n * k // 32, 34), np.uint8)  # all-zero weights: logits == bias
    w = rt.pack(raw, n, k)
    bias = np.zeros(n, np.float32)
    bias[19] = bias[37] = 2
    bias[8195] = bias[8197] = 3
    ids = torch.empty(1, 2, dtype=torch.int32, device='cuda')
    logits = torch.empty(1, n, device='cuda')
    z = dev(np.zeros((1, k), np.float32))
    bd = dev(bias)
    rt.ensure_workspace(1, n, k)
    rt.lib.call('pq8_joint_argmax', w.pointer, z.data_ptr(), None, z.data_ptr(), bd.data_ptr(),
                logits.data_ptr(), ids.data_ptr(), 1, n, k, 8193, rt.workspace.data_ptr(), rt.workspace.numel(),
                rt.stream())
    assert ids.cpu().numpy().tolist() == [[19, 2]]


def test_tdt_decode_matches_reference_golden(rt, golden_dir):
    meta = json.loads((golden_dir / 'golden_meta.json').read_text())
    data = np.load(golden_dir / 'tdt_decode.npz')
    for case in meta['tdt_random']:
        seed = case['seed']
        model = SyntheticParakeet(seed=seed, encoder_layers=0, blank_bias=case['blank_bias'],
                                  duration0_bias=case['duration0_bias'])
        d = PQ8Decoder(model, rt, batch=1)
        r = greedy_decode(data[f'seed{seed}_projected'], d, DURATIONS)
        np.testing.assert_array_equal(np.asarray(r['tokens'], np.int32), data[f'seed{seed}_tokens'])
        np.testing.assert_array_equal(np.asarray(r['decode_trace'], np.int32).reshape(-1, 3),
                                      data[f'seed{seed}_trace'])
        assert r['joint_calls'] == case['joint_calls']


@pytest.mark.parametrize('batch', [1, 4, 8, 13, 40])
def test_tdt_batched_decode_matches_oracle(rt, batch):
    model = SyntheticParakeet(seed=12, encoder_layers=0, blank_bias=3.0)
    rng = np.random.default_rng(40 + batch)
    projected = [rng.normal(size=(int(rng.integers(20, 40)), 640)).astype(np.float32) for _ in range(batch)]
    d = PQ8Decoder(model, rt, batch=batch)
    got = greedy_decode_batch(projected, d, DURATIONS)
    for p, g in zip(projected, got):
        ref = otdt.greedy_decode(p, otdt.Decoder64(model), DURATIONS)
        assert g['tokens'] == ref['tokens']
        assert g['decode_trace'] == ref['decode_trace']


def test_tdt_1000_steps_matches_oracle(rt):
    """BASELINE config 3 at batch 1: ~1000 joint calls, ids identical to the float64 oracle."""
    model = SyntheticParakeet(seed=11, encoder_layers=0)
    projected = np.random.default_rng(2026).normal(size=(1150, 640)).astype(np.float32)
    got = greedy_decode(projected, PQ8Decoder(model, rt, batch=1), DURATIONS)
    ref = otdt.greedy_decode(projected, otdt.Decoder64(model), DURATIONS)
    assert got["joint_calls"] >= 1000
    assert got['tokens'] == ref['tokens']
    assert got['decode_trace'] == ref['decode_trace']


def test_tdt_device_loop_matches_reference_golden(rt, golden_dir):
    """The device-resident loop (control kernel + graph replay) on the
    reference's own decodes: blanks, zero durations and the 10-symbol cap."""
    meta = json.loads((golden_dir / 'golden_meta.json').read_text())
    data = np.load(golden_dir / 'tdt_decode.npz')
    for case in meta['tdt_random']:
        seed = case['seed']
        model = SyntheticParakeet(seed=seed, encoder_layers=0, blank_bias=case['blank_bias'],
                                  duration0_bias=case['duration0_bias'])
        [r] = greedy_decode_device([data[f'seed{seed}_projected']], PQ8Decoder(model, rt, batch=1), DURATIONS,
                                   steps_per_graph=4)
        np.testing.assert_array_equal(np.asarray(r['tokens'], np.int32), data[f'seed{seed}_tokens'])
        np.testing.assert_array_equal(np.asarray(r['decode_trace'], np.int32).reshape(-1, 3),
                                      data[f'seed{seed}_trace'])
        assert r['joint_calls'] == case['joint_calls']


@pytest.mark.parametrize('batch', [1, 4, 13, 64])
def test_tdt_device_loop_matches_host_loop(rt, batch):
    """Streams of different lengths (and one empty) through the device loop and
    the host loop: identical tokens, times and per-call traces."""
    model = SyntheticParakeet(seed=12, encoder_layers=0, blank_bias=1.0)
    rng = np.random.default_rng(70 + batch)
    lengths = [int(rng.integers(5, 60)) for _ in range(batch)]
    if batch > 1:
        lengths[1] = 0
    projected = [rng.normal(size=(n, 640)).astype(np.float32) for n in lengths]
    want = greedy_decode_batch([p if len(p) else np.zeros((0, 640), np.float32) for p in projected],
                               PQ8Decoder(model, rt, batch=batch), DURATIONS)
    got = greedy_decode_device(projected, PQ8Decoder(model, rt, batch=batch), DURATIONS, steps_per_graph=8)
    for g, w in zip(got, want):
        assert g == w


# A float32 decode may break a tie the float64 oracle decides by less than
# this (logits are O(1); their FP32 error is ~1e-6).
TIE_EPS = 1e-4


def test_tdt_device_loop_batch64_1000_steps_matches_oracle(rt):
    """BASELINE config 3 at batch 64: 64 streams of 1400 frames, at least 1000
    joint calls each, through the device-resident loop, against the float64
    oracle (oracle.tdt.greedy_decode_streams, Decoder64 arithmetic per stream).
    Every call's (frame, token, skip) must agree; a different call is accepted
    only as a near-tie (the device's token and duration within TIE_EPS of the
    oracle's best logits), counted, and adopted by the oracle."""
    model = SyntheticParakeet(seed=11, encoder_layers=0)
    rng = np.random.default_rng(2027)
    projected = [rng.normal(size=(1400, 640)).astype(np.float32) for _ in range(64)]
    got = greedy_decode_device(projected, PQ8Decoder(model, rt, batch=64), DURATIONS, steps_per_graph=16)
    ref = otdt.greedy_decode_streams(projected, model, DURATIONS, follow=[g['decode_trace'] for g in got],
                                     tie_eps=TIE_EPS)
    ties = 0
    for i, (g, r) in enumerate(zip(got, ref)):
        assert r['mismatch'] is None, (i, r['mismatch'])
        assert g['decode_trace'] == r['decode_trace'], i
        assert g['tokens'] == r['tokens'], i
        assert g['joint_calls'] == r['joint_calls'] >= 1000, (i, g['joint_calls'])
        ties += r['ties']
    calls = sum(g['joint_calls'] for g in got)
    print(f'batch 64: {calls} joint calls, {ties} near-ties decided by float32 rounding')
    assert ties <= 8
    assert rt.device_status() == 0


def test_tdt_device_loop_step_limit(rt):
    """max_steps stops the loop after exactly that many lock-step steps."""
    model = SyntheticParakeet(seed=11, encoder_layers=0)
    projected = [np.random.default_rng(5).normal(size=(200, 640)).astype(np.float32)]
    d = PQ8Decoder(model, rt, batch=1)
    [r] = greedy_decode_device(projected, d, DURATIONS, steps_per_graph=16, max_steps=37)
    assert d.steps == 37 and r['joint_calls'] == 37
    ref = otdt.greedy_decode(projected[0], otdt.Decoder64(model), DURATIONS)
    assert r['decode_trace'] == ref['decode_trace'][:37]


def check_streams_vs_oracle(projected, got, model, max_ties):
    """Every call's (frame, token, skip) equals the float64 oracle's, or is a
    near-tie (within TIE_EPS) that the oracle adopts; returns the tie count."""
    ref = otdt.greedy_decode_streams(projected, model, DURATIONS, follow=[g['decode_trace'] for g in got],
                                     tie_eps=TIE_EPS)
    ties = 0
    for i, (g, r) in enumerate(zip(got, ref)):
        assert r['mismatch'] is None, (i, r['mismatch'])
        assert g['decode_trace'] == r['decode_trace'], i
        assert g['tokens'] == r['tokens'], i
        assert g['joint_calls'] == r['joint_calls'], i
        ties += r['ties']
    assert ties <= max_ties
    return ties


def test_tdt_persistent_matches_reference_golden(rt, golden_dir):
    """pq8_tdt_decode (the whole loop in one launch) on the reference's own
    decodes: blanks, zero durations and the 10-symbol cap."""
    meta = json.loads((golden_dir / 'golden_meta.json').read_text())
    data = np.load(golden_dir / 'tdt_decode.npz')
    for case in meta['tdt_random']:
        seed = case['seed']
        model = SyntheticParakeet(seed=seed, encoder_layers=0, blank_bias=case['blank_bias'],
                                  duration0_bias=case['duration0_bias'])
        [r] = greedy_decode_persistent([data[f'seed{seed}_projected']], PQ8Decoder(model, rt, batch=1), DURATIONS)
        np.testing.assert_array_equal(np.asarray(r['tokens'], np.int32), data[f'seed{seed}_tokens'])
        np.testing.assert_array_equal(np.asarray(r['decode_trace'], np.int32).reshape(-1, 3),
                                      data[f'seed{seed}_trace'])
        assert r['joint_calls'] == case['joint_calls']
    assert rt.device_status() == 0


@pytest.mark.parametrize('batch', [1, 4, 13, 64])
def test_tdt_persistent_matches_oracle(rt, batch):
    """Streams of different lengths (one empty) with blanks in the mix: the
    persistent decode against the float64 oracle, call by call."""
    model = SyntheticParakeet(seed=12, encoder_layers=0, blank_bias=1.0)
    rng = np.random.default_rng(90 + batch)
    lengths = [int(rng.integers(5, 60)) for _ in range(batch)]
    if batch > 1:
        lengths[1] = 0
    projected = [rng.normal(size=(n, 640)).astype(np.float32) for n in lengths]
    got = greedy_decode_persistent(projected, PQ8Decoder(model, rt, batch=1), DURATIONS)
    check_streams_vs_oracle(projected, got, model, max_ties=2)
    assert rt.device_status() == 0


def test_tdt_persistent_batch64_1000_steps_matches_oracle(rt):
    """BASELINE config 3 at batch 64 through pq8_tdt_decode: 64 streams of
    1400 frames, at least 1000 joint calls each, against the float64 oracle."""
    model = SyntheticParakeet(seed=11, encoder_layers=0)
    rng = np.random.default_rng(2027)
    projected = [rng.normal(size=(1400, 640)).astype(np.float32) for _ in range(64)]
    d = PQ8Decoder(model, rt, batch=1)
    got = greedy_decode_persistent(projected, d, DURATIONS)
    assert min(g['joint_calls'] for g in got) >= 1000
    ties = check_streams_vs_oracle(projected, got, model, max_ties=8)
    print(f'batch 64: {d.steps} steps in {d.loop_seconds * 1e3:.2f} ms, {ties} near-ties')
    assert rt.device_status() == 0


def test_tdt_persistent_resume_and_step_limit(rt):
    """A decode split over launches of 37 steps (each resuming the last from
    the workspace) equals the one-launch decode bit for bit; max_steps stops
    after exactly that many steps."""
    model = SyntheticParakeet(seed=12, encoder_layers=0, blank_bias=1.0)
    rng = np.random.default_rng(123)
    projected = [rng.normal(size=(int(n), 640)).astype(np.float32) for n in (80, 3, 51, 120)]
    d = PQ8Decoder(model, rt, batch=1)
    whole = greedy_decode_persistent(projected, d, DURATIONS)
    steps = d.steps
    pieces = greedy_decode_persistent(projected, d, DURATIONS, steps_per_launch=37)
    assert d.steps == steps
    assert pieces == whole
    cut = greedy_decode_persistent(projected, d, DURATIONS, max_steps=37)
    assert d.steps == 37
    for c, w in zip(cut, whole):
        assert c['decode_trace'] == w['decode_trace'][:37]
    assert rt.device_status() == 0


@pytest.mark.parametrize('batch', [5, 20])
def test_tdt_gpu_dispatch_matches_oracle(rt, batch):
    """greedy_decode_gpu takes the persistent launch for few streams and the
    graph loop for many; both match the oracle call by call."""
    model = SyntheticParakeet(seed=12, encoder_layers=0, blank_bias=1.0)
    rng = np.random.default_rng(500 + batch)
    projected = [rng.normal(size=(int(rng.integers(10, 50)), 640)).astype(np.float32) for _ in range(batch)]
    got = greedy_decode_gpu(projected, PQ8Decoder(model, rt, batch=batch), DURATIONS)
    check_streams_vs_oracle(projected, got, model, max_ties=2)
    assert rt.device_status() == 0


def test_tdt_persistent_rejects_bad_arguments(rt):
    """pq8_tdt_decode validates before launching: more than 64 streams, a
    misaligned frame table, a short workspace."""
    from parakeet_cuda_b200.pq8 import PQ8Error, TdtWeights
    model = SyntheticParakeet(seed=12, encoder_layers=0)
    d = PQ8Decoder(model, rt, batch=1)
    w = TdtWeights()
    for l in range(2):
        w.lstm[l] = d.lstm[l][0].pointer
        w.lstm_bias[l] = d.lstm[l][1].data_ptr()
    w.pred, w.pred_bias = d.w_pred.pointer, d.b_pred.data_ptr()
    w.joint, w.joint_bias = d.w_joint.pointer, d.b_joint.data_ptr()
    w.embed = d.embed.data_ptr()
    w.hidden, w.embed_k, w.joint_k, w.n_joint, w.vocab = 640, 640, 640, d.n_out, 8193
    enc = torch.zeros(65 * 4 + 1, 640, device='cuda')
    i32 = dict(dtype=torch.int32, device='cuda')
    state, rec, cnt = torch.zeros(65, 8, **i32), torch.zeros(65, 40, 3, **i32), torch.zeros(2, **i32)
    dur = torch.tensor(DURATIONS, **i32)
    ws = torch.empty(rt.lib.tdt_decode_workspace_size(64, 640, 640), dtype=torch.uint8, device='cuda')

    def call(m, enc_ptr, ws_bytes):
        rt.lib.call('pq8_tdt_decode', C.byref(w), enc_ptr, 4, dur.data_ptr(), 5, state.data_ptr(), m,
                    rec.data_ptr(), 40, rec.data_ptr(), 40, 10, 0, cnt[0:1].data_ptr(), cnt[1:2].data_ptr(),
                    ws.data_ptr(), ws_bytes, rt.stream())

    with pytest.raises(PQ8Error, match='UNSUPPORTED_SHAPE'):
        call(65, enc.data_ptr(), ws.numel())
    with pytest.raises(PQ8Error, match='MISALIGNED'):
        call(1, enc.data_ptr() + 4, ws.numel())
    with pytest.raises(PQ8Error, match='PQ8_ERR_WORKSPACE'):
        call(64, enc.data_ptr(), ws.numel() - 256)
    torch.cuda.synchronize()
    assert rt.device_status() == 0


@pytest.mark.parametrize('m', [1, 7, 300])
def test_tdt_advance_equals_control_then_commit(rt, m):
    """pq8_tdt_advance (one launch) against pq8_tdt_control + pq8_tdt_commit on
    the same random step: streams done and live, blanks and tokens, every
    duration, a stream at the 10-symbol cap, a trace buffer that is full for
    some streams (m = 300 also runs block 0's stream loop past 256 threads).
    All control outputs must be identical; the LSTM state too, except that
    advance also commits done streams that drew a token."""
    rng = np.random.default_rng(400 + m)
    layers, hidden, stride, cap = 2, 640, 50, 6
    frames = rng.integers(0, 12, size=m)
    state = np.zeros((m, 8), np.int32)
    state[:, 0] = frames
    state[:, 1] = rng.integers(0, 13, size=m)             # t; some already past the end
    state[:, 2] = rng.integers(0, 10, size=m)             # symbols (9 = one call from the cap)
    state[:, 3] = rng.integers(0, 8193, size=m)
    state[:, 4] = rng.integers(0, cap + 1, size=m)        # emitted so far; cap = full
    state[:, 5] = rng.integers(0, cap + 1, size=m)        # joint calls so far; cap = full trace
    state[:, 6] = (state[:, 1] >= frames).astype(np.int32)
    ids = np.stack([np.where(rng.random(m) < 0.5, 8192, rng.integers(0, 8192, size=m)),
                    rng.integers(0, 5, size=m)], axis=1).astype(np.int32)
    h0 = rng.normal(size=(layers, m, hidden)).astype(np.float32)
    c0 = rng.normal(size=(layers, m, hidden)).astype(np.float32)
    hn = rng.normal(size=(layers, m, hidden)).astype(np.float32)
    cn = rng.normal(size=(layers, m, hidden)).astype(np.float32)
    dur = dev(np.asarray(DURATIONS, np.int32))

    def run(fused):
        out = {'state': dev(state), 'tokens': torch.zeros(m, dtype=torch.int32, device='cuda'),
               'enc_rows': torch.zeros(m, dtype=torch.int32, device='cuda'),
               'mask': torch.zeros(m, dtype=torch.int32, device='cuda'),
               'emitted': torch.full((m, cap, 3), -1, dtype=torch.int32, device='cuda'),
               'trace': torch.full((m, cap, 3), -1, dtype=torch.int32, device='cuda'),
               'remaining': torch.zeros(1, dtype=torch.int32, device='cuda'),
               'h': dev(h0), 'c': dev(c0)}
        g_ids, g_hn, g_cn = dev(ids), dev(hn), dev(cn)
        ctl = (g_ids.data_ptr(), dur.data_ptr(), len(DURATIONS), out['state'].data_ptr(), m, stride,
               out['tokens'].data_ptr(), out['enc_rows'].data_ptr(), out['mask'].data_ptr(),
               out['emitted'].data_ptr(), cap, out['trace'].data_ptr(), cap, out['remaining'].data_ptr())
        if fused:
            rt.lib.call('pq8_tdt_advance', *ctl, out['h'].data_ptr(), out['c'].data_ptr(), g_hn.data_ptr(),
                        g_cn.data_ptr(), layers, hidden, rt.stream())
        else:
            rt.lib.call('pq8_tdt_control', *ctl, rt.stream())
            rt.lib.call('pq8_tdt_commit', out['h'].data_ptr(), out['c'].data_ptr(), g_hn.data_ptr(),
                        g_cn.data_ptr(), out['mask'].data_ptr(), m, layers, hidden, rt.stream())
        torch.cuda.synchronize()
        return {k: v.cpu().numpy() for k, v in out.items()}

    want, got = run(False), run(True)
    for key in ('state', 'tokens', 'enc_rows', 'mask', 'emitted', 'trace', 'remaining'):
        np.testing.assert_array_equal(got[key], want[key], err_msg=key)
    done_token = (state[:, 6] == 1) & (ids[:, 0] != 8192)
    for key, new in (('h', hn), ('c', cn)):
        np.testing.assert_array_equal(got[key][:, ~done_token], want[key][:, ~done_token], err_msg=key)
        np.testing.assert_array_equal(got[key][:, done_token], new[:, done_token], err_msg=key)
    if m > 1:
        assert want['mask'].any() and not want['mask'].all()
    # full trace or token buffers make both runs record PQ8_ERR_WORKSPACE; reading the status clears it
    assert rt.device_status() in (0, pq8.ERR_WORKSPACE)


def test_status_clean(rt):
    torch.cuda.synchronize()
    assert rt.device_status() == 0
