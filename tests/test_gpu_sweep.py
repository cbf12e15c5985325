"""BASELINE config 4 shapes through the public dispatcher (pq8_linear): every
M in {1, 16, 128, 1024, 8192, 65536} x (N, K) in {(1024,1024), (4096,1024),
(1024,4096), (2560,640), (8197,640), (8198,640)}. Rows are sampled for the
float64 check at large M (size-independent property: every sampled row must
meet the bar); M = 1 goes through the GEMV (FP32, 2e-4), the rest through the
tensor-core GEMM (2e-3 x RMS)."""
import numpy as np
import pytest
import torch

from oracle import q8
from parakeet_cuda_b200.runtime import Runtime
from parakeet_cuda_b200.synthetic import q8_0_blocks

pytestmark = pytest.mark.gpu

SHAPES = [(1024, 1024), (4096, 1024), (1024, 4096), (2560, 640), (8197, 640), (8198, 640)]
MS = [1, 16, 128, 1024, 8192, 65536]


@pytest.fixture(scope='module')
def rt():
    return Runtime(0)


@pytest.mark.parametrize('n,k', SHAPES)
def test_config4_sweep(rt, n, k):
    rng = np.random.default_rng(n + k)
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k)
    g = torch.Generator(device='cuda').manual_seed(n * 7 + k)
    for m in MS:
        x = torch.randn(m, k, device='cuda', generator=g)
        y = rt.linear(x, w)
        rows = np.unique(np.concatenate([[0, m - 1], rng.integers(0, m, size=min(m, 48))]))
        xs = x[torch.from_numpy(rows).cuda()].cpu().numpy()
        got = y[torch.from_numpy(rows).cuda()].cpu().numpy()
        gold = q8.gemm(xs, raw, n, k)
        if m == 1:
            np.testing.assert_allclose(got, gold, atol=2e-4, rtol=2e-4)
        else:
            assert q8.max_err_over_rms(got, gold) <= 2e-3, (m, n, k)
        assert np.isfinite(y[-1].cpu().numpy()).all()
        del x, y
    torch.cuda.synchronize()
    assert rt.device_status() == 0
