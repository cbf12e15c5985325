"""The lock-step float64 TDT oracle (``oracle.tdt.greedy_decode_streams``)
against the single-stream oracle it batches (``Decoder64`` + ``greedy_decode``,
itself pinned to the reference's decodes in test_oracle_golden.py), and its
near-tie follow mode: a planted wrong decision is reported, not adopted."""
import numpy as np

from oracle import tdt as otdt
from parakeet_cuda_b200.synthetic import SyntheticParakeet

DURATIONS = [0, 1, 2, 3, 4]


def streams(seed, count):
    rng = np.random.default_rng(seed)
    out = [rng.normal(size=(int(rng.integers(1, 30)), 640)).astype(np.float32) for _ in range(count)]
    out[1] = np.zeros((0, 640), np.float32)  # an empty stream makes no call
    return out


def test_lock_step_oracle_equals_single_stream_oracle():
    for seed, blank_bias, d0 in ((12, 3.0, 0.0), (11, 0.0, 0.0), (13, 0.0, 4.0)):
        model = SyntheticParakeet(seed=seed, encoder_layers=0, blank_bias=blank_bias, duration0_bias=d0)
        proj = streams(seed, 7)
        got = otdt.greedy_decode_streams(proj, model, DURATIONS)
        for p, g in zip(proj, got):
            ref = otdt.greedy_decode(p, otdt.Decoder64(model), DURATIONS)
            assert g['tokens'] == ref['tokens']
            assert g['decode_trace'] == ref['decode_trace']
            assert g['joint_calls'] == ref['joint_calls']
            assert g['ties'] == 0 and g['mismatch'] is None


def test_follow_mode_reports_a_planted_decision():
    model = SyntheticParakeet(seed=12, encoder_layers=0, blank_bias=1.0)
    proj = streams(5, 4)
    base = otdt.greedy_decode_streams(proj, model, DURATIONS)
    same = otdt.greedy_decode_streams(proj, model, DURATIONS, follow=[b['decode_trace'] for b in base],
                                      tie_eps=1e-4)
    assert all(s['mismatch'] is None and s['ties'] == 0 and s['decode_trace'] == b['decode_trace']
               for s, b in zip(same, base))
    planted = [[list(c) for c in b['decode_trace']] for b in base]
    planted[0][2][1] = (planted[0][2][1] + 1) % 8192  # a token that is not a near-tie
    bad = otdt.greedy_decode_streams(proj, model, DURATIONS, follow=planted, tie_eps=1e-4)
    assert bad[0]['mismatch']['call'] == 2 and bad[0]['mismatch']['token_gap'] > 1e-4
    short = [b['decode_trace'][:-1] for b in base]  # an implementation that stopped one call early
    cut = otdt.greedy_decode_streams(proj, model, DURATIONS, follow=short, tie_eps=1e-4)
    assert cut[0]['mismatch']['theirs'] is None
