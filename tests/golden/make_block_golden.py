"""Golden vectors for whole FastConformer blocks, made by running the
reference's own NumPy block (``parakeet_cuda/reference.py:33-66``, ``block``)
on a seeded ``SyntheticParakeet(block=True)`` model.

Run where the reference checkout is present (it is never read at test time):

    python tests/golden/make_block_golden.py /path/to/parakeet_cuda

Cases (seed 31, two layers): T = 40 frames through layer 0, then layer 1 on
layer 0's output; and T = 7 (fewer frames than the depthwise kernel's 9 taps)
through layer 0. The subsampling stem (``reference.py:11-30``, ``stem``) on
N(0, 1) mel features of 50, 17 and 1 frames. Inputs are N(0, 1) float32.
Output: ``block.npz``.
"""
from __future__ import annotations

import importlib.util
import os
from pathlib import Path
import sys

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
SEED = 31


def main(ref_root: str) -> None:
    sys.path.insert(0, str(REPO))
    from parakeet_cuda_b200.synthetic import SyntheticParakeet
    spec = importlib.util.spec_from_file_location('ref_reference', Path(ref_root) / 'parakeet_cuda' / 'reference.py')
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    model = SyntheticParakeet(seed=SEED, encoder_layers=2, decoder=False, block=True)
    out = {}
    for t in (40, 7):
        x = np.random.default_rng(100 + t).normal(size=(t, 1024)).astype(np.float32)
        y0 = ref.block(x, model, 0)
        out[f't{t}_x'] = x
        out[f't{t}_layer0'] = y0.astype(np.float32)
        if t == 40:
            out[f't{t}_layer1'] = ref.block(y0, model, 1).astype(np.float32)
    for frames in (50, 17, 1):
        mel = np.random.default_rng(200 + frames).normal(size=(frames, 128)).astype(np.float32)
        out[f'stem{frames}_mel'] = mel
        out[f'stem{frames}_out'] = np.asarray(ref.stem(mel, model), np.float32)
    np.savez_compressed(HERE / 'block.npz', **out)
    print({k: (v.shape, float(np.sqrt((v.astype(np.float64) ** 2).mean()))) for k, v in out.items()})


if __name__ == '__main__':
    if len(sys.argv) < 2 and 'PARAKEET_CUDA_REFERENCE' not in os.environ:
        raise SystemExit('usage: make_block_golden.py <parakeet_cuda checkout> (or set PARAKEET_CUDA_REFERENCE)')
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ['PARAKEET_CUDA_REFERENCE'])
