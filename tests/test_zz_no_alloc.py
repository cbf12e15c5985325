"""pq8_gemv_static: the GEMV entry point that needs no caller-provided workspace.

It exists for callers that cannot allocate device memory for the library (a
host that keeps every device byte in its own pre-reserved pool, or a decode
loop that must not call cudaMalloc because cudaMalloc synchronizes the
device); its scratch is a fixed array built into libpq8.so. This file is
collected last so that a failure here does not stop the rest of the GPU suite.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from parakeet_cuda_b200 import pq8
from parakeet_cuda_b200.runtime import Runtime
from parakeet_cuda_b200.synthetic import q8_0_blocks

pytestmark = pytest.mark.gpu


def test_static_scratch_gemv_matches_workspace_gemv():
    rt = Runtime(0)
    lib = rt.lib
    rng = np.random.default_rng(77)
    for m, n, k, epi, layout in ((1, 8198, 640, pq8.EPI_NONE, pq8.LAYOUT_ROWS),
                                 (3, 2560, 1280, pq8.EPI_RELU, pq8.LAYOUT_ROWS),
                                 (8, 2048, 1024, pq8.EPI_GLU, pq8.LAYOUT_GLU)):
        w = rt.pack(q8_0_blocks(rng, n, k), n, k, layout)
        out_n = n // 2 if epi == pq8.EPI_GLU else n
        x = torch.from_numpy(rng.normal(size=(m, k)).astype(np.float32)).cuda()
        bias = torch.from_numpy(rng.normal(size=n).astype(np.float32)).cuda()
        ref = torch.empty(m, out_n, device='cuda')
        rt.ensure_workspace(m, n, k)
        lib.call('pq8_gemv', w.pointer, x.data_ptr(), ref.data_ptr(), bias.data_ptr(), None, m, n, k, epi, 1.0,
                 rt.workspace.data_ptr(), rt.workspace.numel(), rt.stream())
        want = ref.cpu().numpy()
        for _ in range(2):  # the second call reuses whatever the first left in the static array
            got = torch.full((m, out_n), float('nan'), device='cuda')
            lib.call('pq8_gemv_static', w.pointer, x.data_ptr(), got.data_ptr(), bias.data_ptr(), None, m, n, k, epi,
                     1.0, rt.stream())
            np.testing.assert_allclose(got.cpu().numpy(), want, atol=2e-4, rtol=2e-4)
    assert rt.device_status() == 0


def test_static_scratch_rejects_oversized_shape():
    rt = Runtime(0)
    w = torch.zeros(4096, dtype=torch.uint8, device='cuda')
    x = torch.zeros(8, 32, device='cuda')
    # K longer than 16 splits of the activation staging area: the splits
    # reduce through workspace partials, 25 MB of them for 313 tiles
    n, k = 40_000, 25_600
    assert rt.lib.gemv_workspace_size(8, n, k) > 4 << 20
    with pytest.raises(pq8.PQ8Error) as e:
        rt.lib.call('pq8_gemv_static', w.data_ptr(), x.data_ptr(), x.data_ptr(), None, None, 8, n, k, pq8.EPI_NONE,
                    1.0, rt.stream())
    assert e.value.code == pq8.ERR_WORKSPACE
