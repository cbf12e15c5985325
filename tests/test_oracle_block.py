"""The block oracle (float64 restatement) against golden outputs of the
reference's own NumPy block (tests/golden/make_block_golden.py)."""
import numpy as np
import pytest

from oracle import block as ob
from parakeet_cuda_b200.synthetic import SyntheticParakeet


@pytest.fixture(scope='module')
def model():
    return SyntheticParakeet(seed=31, encoder_layers=2, decoder=False, block=True)


def test_block_oracle_matches_reference(model, golden_dir):
    d = np.load(golden_dir / 'block.npz')
    for t in (40, 7):
        y = ob.blocks(d[f't{t}_x'], model, [0])
        np.testing.assert_allclose(y, d[f't{t}_layer0'], atol=2e-5, rtol=0)
    y = ob.blocks(d['t40_x'], model, [0, 1])
    np.testing.assert_allclose(y, d['t40_layer1'], atol=2e-5, rtol=0)


def test_rel_shift_index():
    """s[i, j] takes positional row t - 1 + j - i: the diagonal of the positional
    scores that the reference's pad / reshape / drop / reshape shift selects."""
    rng = np.random.default_rng(3)
    h, t, d = 2, 5, 4
    qu, qv, k = (rng.normal(size=(h, t, d)) for _ in range(3))
    p = rng.normal(size=(h, 2 * t - 1, d))
    s = ob.rel_shift_scores(qu, qv, k, p)
    bd = qv @ p.transpose(0, 2, 1)
    trick = np.pad(bd, ((0, 0), (0, 0), (1, 0))).reshape(h, 2 * t, t)[:, 1:, :].reshape(h, t, 2 * t - 1)[:, :, :t]
    np.testing.assert_allclose(s, (qu @ k.transpose(0, 2, 1) + trick) / np.sqrt(128), atol=1e-12)


def test_stem_oracle_matches_reference(model, golden_dir):
    from oracle import stem as ostem
    d = np.load(golden_dir / 'block.npz')
    for frames in (50, 17, 1):
        np.testing.assert_allclose(ostem.stem(d[f'stem{frames}_mel'], model), d[f'stem{frames}_out'], atol=5e-6, rtol=0)
