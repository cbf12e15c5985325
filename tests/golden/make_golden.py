"""Generate the golden fixtures in this folder by running the reference's own code.

Run in a container where the reference checkout is present (it is never read
at test time):

    python tests/golden/make_golden.py /path/to/parakeet_cuda

It imports, from the reference checkout:

* ``workloads/q8_gemm.py:cases()`` - the fixed Q8 x FP32 kernel contract
  (seed 903, shapes (1,32,3), (17,640,65), (33,1024,129), (441,1024,4096),
  float64 goldens, atol 8e-4 / rtol 3e-4). ``txir_tools`` is not available,
  so two tiny stand-ins for its ``Case`` and ``CUDAKernel`` types are
  installed first; they only record their arguments.
* ``parakeet_cuda/decoder.py`` - ``CPUDecoder`` and ``decode`` run on a
  seeded ``SyntheticParakeet`` model to give golden TDT token ids, and the
  fake-decoder state-machine case of ``tests/test_host.py:34-49``.

The seed-17 decode/GEMV case of ``tests/test_cuda.py:34-50`` builds its inputs
inside a GPU-only test method, so its input construction and its scalar
``struct``-based golden are restated here step by step.

Outputs: ``q8_gemm_contract.npz``, ``q8_decode_gemv.npz``, ``tdt_decode.npz``
and ``golden_meta.json`` (hashes and summary numbers).
"""
from __future__ import annotations

import hashlib
import json
import os
from pathlib import Path
import struct
import sys
import types

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def install_txir_stub():
    pkg = types.ModuleType('txir_tools')
    compiler = types.ModuleType('txir_tools.compiler')
    workload = types.ModuleType('txir_tools.workload')

    class CUDAKernel:
        def __init__(self, path, arch=None):
            self.path, self.arch = path, arch

    class Case:
        def __init__(self, name, args, expected, grid=None, block=None, atol=None, rtol=None):
            self.name, self.args, self.expected = name, args, expected
            self.grid, self.block, self.atol, self.rtol = grid, block, atol, rtol

    compiler.CUDAKernel = CUDAKernel
    workload.Case = Case
    pkg.compiler, pkg.workload = compiler, workload
    sys.modules.update({'txir_tools': pkg, 'txir_tools.compiler': compiler,
                        'txir_tools.workload': workload})


def q8_contract(ref: Path, meta: dict) -> dict:
    sys.path.insert(0, str(ref))
    from workloads.q8_gemm import cases
    out = {}
    sample_rng = np.random.default_rng(1234)
    meta['q8_gemm'] = []
    for case in cases():
        packed, x, _, m, k, n = case.args
        m, k, n = int(m), int(k), int(n)
        golden = case.expected[2]
        tag = f'm{m}_k{k}_n{n}'
        entry = {'name': case.name, 'm': m, 'k': k, 'n': n, 'atol': case.atol, 'rtol': case.rtol,
                 'grid': case.grid, 'block': case.block,
                 'sha_packed': sha(packed), 'sha_x': sha(x), 'sha_golden': sha(golden)}
        meta['q8_gemm'].append(entry)
        if packed.nbytes + x.nbytes + golden.nbytes < 1 << 20:
            out[tag + '_packed'] = packed
            out[tag + '_x'] = x
            out[tag + '_golden'] = golden
        else:
            # Too large to commit: keep hashes plus a seeded sample of golden entries.
            idx = sample_rng.choice(golden.size, 8192, replace=False)
            out[tag + '_sample_idx'] = idx.astype(np.int64)
            out[tag + '_sample_val'] = golden.reshape(-1)[idx]
    return out


def decode_gemv_case() -> dict:
    # Restated from tests/test_cuda.py:34-50 (seed 17).
    rng = np.random.default_rng(17)
    out = {}
    for n, k in ((3, 32), (7, 640), (5, 1024)):
        scales = rng.uniform(.001, .1, (n * k // 32)).astype(np.float16)
        values = rng.integers(-128, 128, (n * k // 32, 32), dtype=np.int8)
        raw = np.empty((len(scales), 34), dtype=np.uint8)
        raw[:, :2] = scales.view(np.uint8).reshape(-1, 2)
        raw[:, 2:] = values.view(np.uint8)
        golden = np.empty(n * k, np.float32)
        data = raw.tobytes()
        for i in range(n * k):
            golden[i] = (struct.unpack_from('<e', data, (i // 32) * 34)[0]
                         * struct.unpack_from('b', data, (i // 32) * 34 + 2 + i % 32)[0])
        x = rng.normal(size=k).astype(np.float32)
        gemv = (golden.reshape(n, k).astype(np.float64) @ x).astype(np.float32)
        out[f'n{n}_k{k}_raw'] = raw
        out[f'n{n}_k{k}_decoded'] = golden
        out[f'n{n}_k{k}_x'] = x
        out[f'n{n}_k{k}_gemv'] = gemv
    return out


def tdt_cases(ref: Path, meta: dict) -> dict:
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(REPO))
    from parakeet_cuda.decoder import CPUDecoder, decode
    from parakeet_cuda_b200.synthetic import SyntheticParakeet

    # tests/test_host.py:34-49: fake model + fake decoder state machine.
    class FakeModel:
        metadata = {'asr.tdt.durations': [0, 1, 2, 3, 4]}

        def text(self, ids):
            return str(ids)

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
    r = decode(np.zeros((3, 640), np.float32), d, FakeModel())
    meta['tdt_fake'] = {'predicted': d.predicted, 'tokens': r['tokens'],
                        'committed': d.committed, 'joint_calls': r['joint_calls'],
                        'trace': r['decode_trace']}

    out = {}
    meta['tdt_random'] = []
    for seed, frames, blank_bias, dur0_bias in ((11, 64, 0.0, 0.0), (12, 64, 3.0, 0.0),
                                                (13, 32, 2.5, 1.0)):
        model = SyntheticParakeet(seed=seed, encoder_layers=0, blank_bias=blank_bias,
                                  duration0_bias=dur0_bias)
        projected = np.random.default_rng(seed + 1000).normal(size=(frames, 640)).astype(np.float32)
        dec = CPUDecoder(model)
        res = decode(projected, dec, model)
        out[f'seed{seed}_projected'] = projected
        out[f'seed{seed}_tokens'] = np.asarray(res['tokens'], np.int32)
        out[f'seed{seed}_trace'] = np.asarray(res['decode_trace'], np.int32).reshape(-1, 3)
        meta['tdt_random'].append({'seed': seed, 'frames': frames, 'blank_bias': blank_bias,
                                   'duration0_bias': dur0_bias, 'joint_calls': res['joint_calls'],
                                   'tokens': len(res['tokens']),
                                   'sha_raw_joint': hashlib.sha256(model.raw('joint.joint_net.2.weight').tobytes()).hexdigest()})
    return out


def main():
    if len(sys.argv) < 2 and 'PARAKEET_CUDA_REFERENCE' not in os.environ:
        raise SystemExit('usage: make_golden.py <parakeet_cuda checkout> (or set PARAKEET_CUDA_REFERENCE)')
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else os.environ['PARAKEET_CUDA_REFERENCE']).resolve()
    if not (ref / 'parakeet_cuda' / 'decoder.py').is_file():
        raise SystemExit(f'reference checkout not found at {ref}')
    install_txir_stub()
    meta = {'numpy': np.__version__}
    np.savez_compressed(HERE / 'q8_gemm_contract.npz', **q8_contract(ref, meta))
    np.savez_compressed(HERE / 'q8_decode_gemv.npz', **decode_gemv_case())
    np.savez_compressed(HERE / 'tdt_decode.npz', **tdt_cases(ref, meta))
    (HERE / 'golden_meta.json').write_text(json.dumps(meta, indent=1) + '\n')
    print(json.dumps({k: (v if not isinstance(v, list) else len(v)) for k, v in meta.items()}))


if __name__ == '__main__':
    main()
