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


# (m, n, k, epilogue, layout). The first three reduce their K splits inside a
# thread-block cluster and use only the counter area of the static array; the
# M = 1 streaming shape and the 8-row shape with more than 16 K splits reduce
# through split-K partial sums stored in the array (more than the 64 KiB of
# counters), and m = 40 runs five row groups side by side.
SHAPES = ((1, 8198, 640, pq8.EPI_NONE, pq8.LAYOUT_ROWS),
          (3, 2560, 1280, pq8.EPI_RELU, pq8.LAYOUT_ROWS),
          (8, 2048, 1024, pq8.EPI_GLU, pq8.LAYOUT_GLU),
          (1, 1024, 32768, pq8.EPI_NONE, pq8.LAYOUT_ROWS),
          (8, 256, 24576, pq8.EPI_NONE, pq8.LAYOUT_ROWS),
          (40, 1280, 640, pq8.EPI_RESIDUAL, pq8.LAYOUT_ROWS))


def test_static_scratch_gemv_matches_workspace_gemv():
    """Both entry points run the same plan and kernel, so the outputs must be
    identical bit for bit, on the first call and on a second call that finds
    the array as the first one left it."""
    rt = Runtime(0)
    lib = rt.lib
    rng = np.random.default_rng(77)
    partial_shapes = 0
    for m, n, k, epi, layout in SHAPES:
        need = lib.gemv_workspace_size(m, n, k)
        assert need <= 4 << 20, (m, n, k, need)
        partial_shapes += need > 64 << 10
        w = rt.pack(q8_0_blocks(rng, n, k), n, k, layout)
        out_n = n // 2 if epi == pq8.EPI_GLU else n
        x = torch.from_numpy(rng.normal(size=(m, k)).astype(np.float32)).cuda()
        bias = torch.from_numpy(rng.normal(size=n).astype(np.float32)).cuda()
        resid = torch.from_numpy(rng.normal(size=(m, out_n)).astype(np.float32)).cuda()
        r_ptr = resid.data_ptr() if epi == pq8.EPI_RESIDUAL else None
        ref = torch.empty(m, out_n, device='cuda')
        rt.ensure_workspace(m, n, k)
        lib.call('pq8_gemv', w.pointer, x.data_ptr(), ref.data_ptr(), bias.data_ptr(), r_ptr, m, n, k, epi, 0.5,
                 rt.workspace.data_ptr(), rt.workspace.numel(), rt.stream())
        want = ref.cpu().numpy()
        for call in range(2):  # the second call reuses whatever the first left in the static array
            got = torch.full((m, out_n), float('nan'), device='cuda')
            lib.call('pq8_gemv_static', w.pointer, x.data_ptr(), got.data_ptr(), bias.data_ptr(), r_ptr, m, n, k,
                     epi, 0.5, rt.stream())
            np.testing.assert_array_equal(got.cpu().numpy(), want, err_msg=f'{(m, n, k)} call {call}')
    assert partial_shapes == 2
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
