"""Pin the CPU oracle to golden vectors produced by the reference's own code.

Fixtures come from ``tests/golden/make_golden.py`` (run against the reference
checkout). These tests need no GPU.
"""
import hashlib
import json

import numpy as np
import pytest

from oracle import q8, tdt
from parakeet_cuda_b200.synthetic import SyntheticParakeet, q8_0_blocks


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope='module')
def meta(golden_dir):
    return json.loads((golden_dir / 'golden_meta.json').read_text())


def contract_inputs(m, k, n):
    """Regenerate workloads/q8_gemm.py:cases() inputs (seed 903) in their draw order."""
    rng = np.random.default_rng(903)
    for mm, kk, nn in ((1, 32, 3), (17, 640, 65), (33, 1024, 129), (441, 1024, 4096)):
        packed = q8_0_blocks(rng, nn, kk, scale_lo=1e-4, scale_hi=2e-2)
        x = rng.normal(size=(mm, kk)).astype(np.float32)
        if (mm, kk, nn) == (m, k, n):
            return packed, x
    raise KeyError((m, k, n))


def test_contract_generator_reproduces_reference_inputs(meta):
    for case in meta['q8_gemm']:
        packed, x = contract_inputs(case['m'], case['k'], case['n'])
        assert sha(packed) == case['sha_packed'], case['name']
        assert sha(x) == case['sha_x'], case['name']


def test_oracle_gemm_matches_reference_golden(meta, golden_dir):
    data = np.load(golden_dir / 'q8_gemm_contract.npz')
    for case in meta['q8_gemm']:
        m, k, n = case['m'], case['k'], case['n']
        tag = f'm{m}_k{k}_n{n}'
        packed, x = contract_inputs(m, k, n)
        y = q8.gemm(x, packed, n, k).astype(np.float32)
        if tag + '_golden' in data:
            np.testing.assert_array_equal(data[tag + '_packed'], packed)
            golden = data[tag + '_golden']
            assert sha(golden) == case['sha_golden']
            np.testing.assert_allclose(y, golden, atol=case['atol'], rtol=case['rtol'])
            # float64 oracle rounded to float32 reproduces the float64 reference golden
            assert np.max(np.abs(y - golden)) <= 1e-5 * q8.rms(golden)
        else:
            idx, val = data[tag + '_sample_idx'], data[tag + '_sample_val']
            np.testing.assert_allclose(y.reshape(-1)[idx], val, atol=case['atol'], rtol=case['rtol'])
            assert np.max(np.abs(y.reshape(-1)[idx] - val)) <= 1e-5 * q8.rms(val)


def test_oracle_decode_and_gemv_match_reference(golden_dir):
    data = np.load(golden_dir / 'q8_decode_gemv.npz')
    for n, k in ((3, 32), (7, 640), (5, 1024)):
        tag = f'n{n}_k{k}'
        raw = data[tag + '_raw']
        # exact expansion (runtime.cu:26-33 semantics), including int8 value -128
        np.testing.assert_array_equal(q8.dequant_f32(raw, n, k).reshape(-1), data[tag + '_decoded'])
        gemv = q8.gemm(data[tag + '_x'][None, :], raw, n, k)[0]
        np.testing.assert_allclose(gemv, data[tag + '_gemv'], atol=2e-4, rtol=2e-4)


def test_oracle_tdt_state_machine(meta):
    fake = meta['tdt_fake']

    class FakeDecoder:
        def __init__(self):
            self.predicted, self.committed, self.calls = [], 0, 0

        def predict(self, token):
            self.predicted.append(token)

        def joint(self, frame):
            self.calls += 1
            return (8192, 0) if self.calls in (1, 2) else (7, 0)

        def commit(self):
            self.committed += 1

    d = FakeDecoder()
    r = tdt.greedy_decode(np.zeros((3, 640), np.float32), d, [0, 1, 2, 3, 4])
    assert d.predicted == fake['predicted']
    assert r['tokens'] == fake['tokens']
    assert d.committed == fake['committed']
    assert r['joint_calls'] == fake['joint_calls']
    assert r['decode_trace'] == fake['trace']


def test_oracle_tdt_random_weights_match_reference(meta, golden_dir):
    data = np.load(golden_dir / 'tdt_decode.npz')
    for case in meta['tdt_random']:
        seed = case['seed']
        model = SyntheticParakeet(seed=seed, encoder_layers=0, blank_bias=case['blank_bias'],
                                  duration0_bias=case['duration0_bias'])
        assert sha(model.raw('joint.joint_net.2.weight')) == case['sha_raw_joint']
        dec = tdt.Decoder64(model)
        r = tdt.greedy_decode(data[f'seed{seed}_projected'], dec, [0, 1, 2, 3, 4])
        np.testing.assert_array_equal(np.asarray(r['tokens'], np.int32), data[f'seed{seed}_tokens'])
        np.testing.assert_array_equal(np.asarray(r['decode_trace'], np.int32).reshape(-1, 3),
                                      data[f'seed{seed}_trace'])
        assert r['joint_calls'] == case['joint_calls']


def test_tf32_rounding_model():
    x = np.array([1.0, 1.0 + 2**-11, 1.0 + 2**-12, -(1.0 + 3 * 2**-11), np.inf, -np.inf], np.float32)
    r = q8.tf32_round(x)
    assert r[0] == 1.0
    assert r[1] == np.float32(1.0 + 2**-10)        # tie rounds away from zero
    assert r[2] == 1.0
    assert r[3] == np.float32(-(1.0 + 2 * 2**-10))
    assert np.isinf(r[4]) and np.isinf(r[5])
    assert np.all((r[:4].view(np.uint32) & 0x1FFF) == 0)
    e = q8.tf32_round_even(np.array([1.0 + 2**-11, 1.0 + 3 * 2**-11, -(1.0 + 3 * 2**-11), 1.0 + 2**-11 + 2**-20,
                                     np.inf], np.float32))
    assert e[0] == 1.0                               # tie rounds to the even neighbour (down)
    assert e[1] == np.float32(1.0 + 2 * 2**-10)      # tie rounds to the even neighbour (up)
    assert e[2] == np.float32(-(1.0 + 2 * 2**-10))
    assert e[3] == np.float32(1.0 + 2**-10)          # above the tie rounds up
    assert np.isinf(e[4])
    # TF32-RN on both operands meets the north-star tolerance on config 0 shapes
    rng = np.random.default_rng(0)
    raw = q8_0_blocks(rng, 512, 1024)
    x = rng.normal(size=(64, 1024)).astype(np.float32)
    gold = q8.gemm(x, raw, 512, 1024)
    assert q8.max_err_over_rms(q8.gemm_tf32(x, raw, 512, 1024), gold) < 2e-3


def test_epilogues():
    acc = np.array([[-2.0, -0.5, 0.5, 3.0]])
    bias = np.array([0.5, 0.0, -1.0, 1.0])
    np.testing.assert_allclose(q8.epilogue(acc, q8.EPI_NONE, bias), acc + bias)
    np.testing.assert_allclose(q8.epilogue(acc, q8.EPI_RELU, bias), np.maximum(acc + bias, 0))
    z = acc + bias
    np.testing.assert_allclose(q8.epilogue(acc, q8.EPI_SILU, bias), z / (1 + np.exp(-z)))
    np.testing.assert_allclose(q8.epilogue(acc, q8.EPI_GLU), acc[:, :2] / (1 + np.exp(-acc[:, 2:])))
    resid = np.ones_like(acc)
    np.testing.assert_allclose(q8.epilogue(acc, q8.EPI_RESIDUAL, None, resid, 0.5), 1 + 0.5 * acc)
