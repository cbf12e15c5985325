"""GPU parity of the Q8_0 contraction kernels against the CPU oracle.

Tolerances:
* GEMM (tensor cores, TF32 operands rounded to nearest: weights ties-to-even,
  activations ties-away)
  ``max|y - golden| <= 2e-3 * rms(golden)`` against the float64 golden, and
  ``<= 1e-4 * rms`` against ``oracle.q8.gemm_tf32`` (the same TF32-rounded
  operands summed in float64): what remains is FP32 accumulation order, while
  truncating instead of rounding an operand would show up at the 1e-3 level.
* GEMV (FP32 FMA): ``atol = rtol = 2e-4`` as ``tests/test_cuda.py:34-50`` of
  the reference.
* Q8_0 expansion: bit-exact.
"""
import os

import numpy as np
import pytest
import torch

from oracle import q8
from parakeet_cuda_b200 import pq8
from parakeet_cuda_b200.pq8 import EPI_GLU, EPI_NONE, EPI_RELU, EPI_RESIDUAL, EPI_SILU, LAYOUT_GLU, LAYOUT_ROWS
from parakeet_cuda_b200.runtime import Runtime
from parakeet_cuda_b200.synthetic import q8_0_blocks

pytestmark = pytest.mark.gpu

NORTH_STAR = 2e-3
TF32_EXACT = 1e-4


@pytest.fixture(scope='module')
def rt():
    return Runtime(0)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def contract_cases():
    """workloads/q8_gemm.py:cases() inputs (seed 903), regenerated in draw order."""
    rng = np.random.default_rng(903)
    for m, k, n in ((1, 32, 3), (17, 640, 65), (33, 1024, 129), (441, 1024, 4096)):
        raw = q8_0_blocks(rng, n, k, scale_lo=1e-4, scale_hi=2e-2)
        x = rng.normal(size=(m, k)).astype(np.float32)
        yield m, k, n, raw, x


# Lipschitz factor of each epilogue with respect to the GEMM output z: the
# north-star bar applies to z, so an epilogue may scale the error by this much.
# GLU has no constant factor (its gradient grows with |a|); glu_bar below
# bounds it element by element.
LIPSCHITZ = {EPI_NONE: 1.0, EPI_RELU: 1.0, EPI_SILU: 1.1, EPI_RESIDUAL: 1.0, EPI_GLU: None}


def glu_bar(z):
    """North-star bar carried through GLU, per output element: with
    y = a * sigmoid(b) and |da|, |db| <= 2e-3 * rms(z) (the bar on the GEMM
    output z = [a | b]), |dy| <= 2e-3 * rms(z) * (sigmoid(b) + |a| sigmoid'(b))
    to first order; 5 % covers the second-order term at this error size. The
    floor of 1e-6 of the bar admits FP32's sigmoid underflowing to 0 where
    b < -88 and the exact output is below 1e-36."""
    h = z.shape[1] // 2
    a, b = z[:, :h], z[:, h:]
    s = q8.sigmoid(b)
    bar = NORTH_STAR * q8.rms(z)
    return 1.05 * bar * (s + np.abs(a) * s * (1.0 - s)) + 1e-6 * bar


def check_gemm(y, x, raw, n, k, epi=EPI_NONE, bias=None, resid=None, alpha=1.0):
    """North-star bar on the GEMM output (scaled through the epilogue) and an
    exact-numerics bar against the TF32-rounded-operand model."""
    y = y.cpu().numpy().astype(np.float64)
    z_gold, z_tf = q8.gemm(x, raw, n, k), q8.gemm_tf32(x, raw, n, k)
    if bias is not None:
        z_gold, z_tf = z_gold + bias, z_tf + bias
    gold = q8.epilogue(z_gold, epi, None, resid, alpha)
    tf = q8.epilogue(z_tf, epi, None, resid, alpha)
    assert np.isfinite(y).all()
    e_gold = float(np.max(np.abs(y - gold))) / q8.rms(z_gold)
    e_tf = float(np.max(np.abs(y - tf))) / q8.rms(z_tf)
    assert e_tf <= TF32_EXACT, (e_gold, e_tf)
    if LIPSCHITZ[epi] is not None:
        assert e_gold <= NORTH_STAR * LIPSCHITZ[epi] * (alpha if epi == EPI_RESIDUAL else 1.0), (e_gold, e_tf)
    else:
        ratio = float(np.max(np.abs(y - gold) / glu_bar(z_gold)))
        assert ratio <= 1.0, (ratio, e_gold, e_tf)
    return e_gold, e_tf


def test_dequant_bit_exact(rt, golden_dir):
    data = np.load(golden_dir / 'q8_decode_gemv.npz')
    for n, k in ((3, 32), (7, 640), (5, 1024)):
        raw = dev(data[f'n{n}_k{k}_raw'].reshape(-1))
        out = torch.empty(n * k, dtype=torch.float32, device='cuda')
        rt.lib.call('pq8_dequant_q8_0', raw.data_ptr(), out.data_ptr(), n * k, rt.stream())
        np.testing.assert_array_equal(out.cpu().numpy(), data[f'n{n}_k{k}_decoded'])


def test_gemv_reference_cases(rt, golden_dir):
    data = np.load(golden_dir / 'q8_decode_gemv.npz')
    for n, k in ((3, 32), (7, 640), (5, 1024)):
        w = rt.pack(data[f'n{n}_k{k}_raw'], n, k)
        x = dev(data[f'n{n}_k{k}_x'][None, :])
        y = rt.linear(x, w)
        np.testing.assert_allclose(y.cpu().numpy()[0], data[f'n{n}_k{k}_gemv'], atol=2e-4, rtol=2e-4)


# Tile configurations of pq8_gemm (PQ8_GEMM_CONFIG): single CTA with 256/192/128/64
# activation rows per tile, then CTA pairs (tcgen05 cta_group::2) with 256/192/128.
CONFIGS = [str(i) for i in range(7)]


@pytest.mark.parametrize('cfg', CONFIGS)
def test_gemm_reference_contract(rt, golden_dir, cfg, monkeypatch):
    monkeypatch.setenv('PQ8_GEMM_CONFIG', cfg)
    data = np.load(golden_dir / 'q8_gemm_contract.npz')
    for m, k, n, raw, x in contract_cases():
        w = rt.pack(raw, n, k)
        y = rt.gemm(dev(x), w)
        check_gemm(y, x, raw, n, k)
        tag = f'm{m}_k{k}_n{n}'
        gold = data[tag + '_golden'] if tag + '_golden' in data else None
        if gold is not None:
            assert q8.max_err_over_rms(y.cpu().numpy(), gold) <= NORTH_STAR
        else:
            idx, val = data[tag + '_sample_idx'], data[tag + '_sample_val']
            got = y.cpu().numpy().reshape(-1)[idx]
            assert np.max(np.abs(got - val)) <= NORTH_STAR * q8.rms(val)


def test_gemm_config0(rt):
    """X [128, 1024] ~ N(0, 1), W [4096, 1024] Q8_0, scales U[1e-3, 2e-2]."""
    rng = np.random.default_rng(0)
    raw = q8_0_blocks(rng, 4096, 1024)
    x = rng.normal(size=(128, 1024)).astype(np.float32)
    y = rt.gemm(dev(x), rt.pack(raw, 4096, 1024))
    e_gold, _ = check_gemm(y, x, raw, 4096, 1024)
    assert e_gold < 1.8e-3


@pytest.mark.parametrize('cfg', CONFIGS)
@pytest.mark.parametrize('m,n,k', [(1, 3, 32), (31, 200, 64), (65, 128, 96), (200, 385, 160), (257, 64, 32),
                                   (300, 1000, 640), (521, 300, 128)])
def test_gemm_tails(rt, cfg, m, n, k, monkeypatch):
    monkeypatch.setenv('PQ8_GEMM_CONFIG', cfg)
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    raw = q8_0_blocks(rng, n, k, qmin=-128)
    x = rng.normal(size=(m, k)).astype(np.float32)
    check_gemm(rt.gemm(dev(x), rt.pack(raw, n, k)), x, raw, n, k)


@pytest.mark.parametrize('cfg', ['0', '3', '4', '6'])
@pytest.mark.parametrize('epi', [EPI_NONE, EPI_RELU, EPI_SILU, EPI_RESIDUAL, EPI_GLU])
def test_gemm_epilogues(rt, epi, cfg, monkeypatch):
    monkeypatch.setenv('PQ8_GEMM_CONFIG', cfg)
    rng = np.random.default_rng(epi + 10)
    m, n, k = 150, 384, 256
    raw = q8_0_blocks(rng, n, k)
    x = rng.normal(size=(m, k)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    out_n = n // 2 if epi == EPI_GLU else n
    resid = rng.normal(size=(m, out_n)).astype(np.float32)
    w = rt.pack(raw, n, k, LAYOUT_GLU if epi == EPI_GLU else LAYOUT_ROWS)
    y = dev(resid) if epi == EPI_RESIDUAL else None
    y = rt.gemm(dev(x), w, out=y, bias=dev(bias), resid=y, epilogue=epi, alpha=0.5)
    check_gemm(y, x, raw, n, k, epi, bias, resid, 0.5)


def test_gemm_glu_pointwise_conv1_shape(rt):
    """pointwise_conv1 of a config-1 layer (M = 375, N = 2048, K = 1024) with the
    GLU epilogue, held element by element to the north-star bar carried through
    GLU, in the tile configuration the library picks."""
    rng = np.random.default_rng(2048)
    m, n, k = 375, 2048, 1024
    raw = q8_0_blocks(rng, n, k)
    x = rng.normal(size=(m, k)).astype(np.float32)
    y = rt.gemm(dev(x), rt.pack(raw, n, k, LAYOUT_GLU), epilogue=EPI_GLU)
    check_gemm(y, x, raw, n, k, EPI_GLU)


@pytest.mark.parametrize('cfg', CONFIGS)
def test_gemm_config0_every_tile_config(rt, cfg, monkeypatch):
    monkeypatch.setenv('PQ8_GEMM_CONFIG', cfg)
    rng = np.random.default_rng(0)
    raw = q8_0_blocks(rng, 4096, 1024)
    x = rng.normal(size=(128, 1024)).astype(np.float32)
    check_gemm(rt.gemm(dev(x), rt.pack(raw, 4096, 1024)), x, raw, 4096, 1024)


def test_gemm_tf32_flags(rt):
    rng = np.random.default_rng(3)
    m, n, k = 256, 512, 512
    raw1, raw2 = q8_0_blocks(rng, n, k), q8_0_blocks(rng, k, n)
    x = rng.normal(size=(m, k)).astype(np.float32)
    w1, w2 = rt.pack(raw1, n, k), rt.pack(raw2, k, n)
    h = rt.gemm(dev(x), w1, epilogue=EPI_SILU, flags=pq8.FLAG_OUT_TF32)
    hn = h.cpu().numpy()
    assert np.all((hn.view(np.uint32) & 0x1FFF) == 0)
    y_pre = rt.gemm(h, w2, flags=pq8.FLAG_X_TF32).cpu().numpy()
    y_in = rt.gemm(h, w2).cpu().numpy()
    np.testing.assert_array_equal(y_pre, y_in)  # rounding an already-rounded X is the identity


def test_linear_dispatch_gemv_matches_gemm(rt):
    rng = np.random.default_rng(4)
    n, k = 2560, 640
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k)
    for m in (1, 2, 3, 5, 8):
        x = rng.normal(size=(m, k)).astype(np.float32)
        bias = rng.normal(size=n).astype(np.float32)
        y = rt.linear(dev(x), w, bias=dev(bias)).cpu().numpy()
        gold = q8.epilogue(q8.gemm(x, raw, n, k), EPI_NONE, bias)
        np.testing.assert_allclose(y, gold, atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize('m,n,k,kernel', [(16, 1024, 4096, 'gemm'), (24, 640, 640, 'gemv'), (48, 8198, 640, 'gemm'),
                                          (64, 4096, 1024, 'gemm'), (9, 129, 1024, 'gemv'), (16, 4096, 1024, 'gemv'),
                                          (24, 4096, 1024, 'gemm')])
def test_linear_dispatch_9_to_64_rows(rt, m, n, k, kernel, monkeypatch):
    """pq8_linear sends 9..64 rows to whichever kernel its measured cost model
    finds faster: the result is bit for bit that kernel's (for the tensor-core
    GEMM, its unsplit form: PQ8_LINEAR_SPLITS=1 turns split K off)."""
    rng = np.random.default_rng(m + n)
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k)
    xd = dev(rng.normal(size=(m, k)).astype(np.float32))
    got = rt.linear(xd, w).cpu().numpy()
    if kernel == 'gemm':
        want = rt.gemm(xd, w).cpu().numpy()
        y = torch.empty(m, n, device='cuda')
        monkeypatch.setenv('PQ8_LINEAR_SPLITS', '1')
        rt.lib.call('pq8_linear', w.pointer, xd.data_ptr(), y.data_ptr(), None, None, m, n, k, EPI_NONE, 1.0, 0,
                    None, 0, rt.stream())
        np.testing.assert_array_equal(y.cpu().numpy(), want)
        check_gemm(torch.from_numpy(got), xd.cpu().numpy(), raw, n, k)
        return
    else:
        rt.ensure_workspace(m, n, k)
        y = torch.empty(m, n, device='cuda')
        rt.lib.call('pq8_gemv', w.pointer, xd.data_ptr(), y.data_ptr(), None, None, m, n, k, EPI_NONE, 1.0,
                    rt.workspace.data_ptr(), rt.workspace.numel(), rt.stream())
        want = y.cpu().numpy()
    np.testing.assert_array_equal(got, want)
    gold = q8.gemm(np.asarray(xd.cpu().numpy()), raw, n, k)
    assert q8.max_err_over_rms(got, gold) <= NORTH_STAR


SPLIT_CASES = [  # m, n, k, epilogue, bias, forced splits: units = M tiles x N tiles of 128
    (128, 1024, 4096, EPI_NONE, False, None),     # 8 units, 8 splits of 16 K blocks
    (441, 1024, 4096, EPI_NONE, True, None),      # reference contract shape: 32 units, 4 splits
    (1024, 1024, 4096, EPI_NONE, False, None),    # 64 units, 2 splits
    (130, 1000, 2080, EPI_SILU, True, None),      # ragged M and N, 65 K blocks: 8 splits, 7 x 9 and one of 2
    (100, 640, 2048, EPI_RESIDUAL, False, None),  # 5 units, 8 splits
    (128, 2048, 2048, EPI_GLU, True, None),       # GLU pairs split like any row
    (64, 4096, 2048, EPI_NONE, False, None),      # 64 rows on the GEMM side of the dispatch: 4 splits
    (128, 4096, 1024, EPI_NONE, False, None),     # config 0: 4 splits of 8
    (128, 4096, 1024, EPI_RESIDUAL, True, 2),     # config 0, forced: 2 splits of 16
    (128, 1024, 1056, EPI_RESIDUAL, True, 8),     # forced 8 -> 4 (8 would leave the last empty): 9, 9, 9, 6
]


@pytest.mark.parametrize('m,n,k,epi,with_bias,forced', SPLIT_CASES)
def test_linear_split_k_matches_oracle(rt, m, n, k, epi, with_bias, forced, monkeypatch):
    """pq8_linear splits K when the GEMM's tiles would fill at most half of the
    SMs (PQ8_LINEAR_SPLITS forces a count): the splits of a tile run as one
    cluster and, after a cluster barrier, push each other the rows each
    finishes (bulk copies between their shared memories); each adds its rows'
    partials in split order. The result meets the north-star bar and the
    TF32-operand model bar, a repeat call is bit for bit the same, and so is a
    call without any workspace (split K needs none)."""
    if forced:
        monkeypatch.setenv('PQ8_LINEAR_SPLITS', str(forced))
    # the GEMV's scratch, or (256 rows and more) the once-rounded activations after the 64 KiB counter area
    copy = (64 << 10) + ((4 * m * k + 255) // 256) * 256 if m >= 256 else 0
    assert rt.lib.linear_workspace_size(m, n, k) == max(rt.lib.gemv_workspace_size(m, n, k) if m <= 64 else 0, copy)
    rng = np.random.default_rng(1000 + m + n + k)
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k, LAYOUT_GLU if epi == EPI_GLU else LAYOUT_ROWS)
    x = rng.normal(size=(m, k)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32) if with_bias else None
    n_out = n // 2 if epi == EPI_GLU else n
    resid = rng.normal(size=(m, n_out)).astype(np.float32) if epi == EPI_RESIDUAL else None
    alpha = 0.5 if epi == EPI_RESIDUAL else 1.0
    xd = dev(x)
    args = dict(bias=dev(bias) if with_bias else None, resid=dev(resid) if resid is not None else None,
                epilogue=epi, alpha=alpha)
    y1 = rt.linear(xd, w, **args)
    y2 = rt.linear(xd, w, **args)
    y3 = torch.empty_like(y1)
    rt.lib.call('pq8_linear', w.pointer, xd.data_ptr(), y3.data_ptr(),
                args['bias'].data_ptr() if with_bias else None, args['resid'].data_ptr() if resid is not None else None,
                m, n, k, epi, alpha, 0, None, 0, rt.stream())
    torch.cuda.synchronize()
    assert rt.device_status() == 0
    np.testing.assert_array_equal(y1.cpu().numpy(), y2.cpu().numpy())
    check_gemm(y1, x, raw, n, k, epi=epi, bias=bias, resid=resid, alpha=alpha)
    if m > 64:  # (up to 64 rows the dispatch may pick the GEMV, which needs its workspace)
        np.testing.assert_array_equal(y1.cpu().numpy(), y3.cpu().numpy())


@pytest.mark.parametrize('m,n,k,epi', [(300, 1024, 2048, EPI_RESIDUAL), (3000, 1024, 4096, EPI_NONE),
                                      (256, 2048, 1024, EPI_GLU)])
def test_linear_rounds_raw_activations_once(rt, m, n, k, epi):
    """Raw activations of 256 or more rows: pq8_linear rounds them into its
    workspace with one streaming pass and runs the GEMM on the rounded copy.
    The result is bit for bit what rounding inside the GEMM gives (pq8_linear
    without the workspace room, the same split decision; and pq8_gemm when
    the shape is not split), and the caller's activations are left as they
    were."""
    rng = np.random.default_rng(m + k)
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k, LAYOUT_GLU if epi == EPI_GLU else LAYOUT_ROWS)
    x = rng.normal(size=(m, k)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    n_out = n // 2 if epi == EPI_GLU else n
    resid = rng.normal(size=(m, n_out)).astype(np.float32) if epi == EPI_RESIDUAL else None
    xd = dev(x)
    args = dict(bias=dev(bias), resid=dev(resid) if resid is not None else None, epilogue=epi,
                alpha=0.5 if epi == EPI_RESIDUAL else 1.0)
    assert rt.lib.linear_workspace_size(m, n, k) >= (64 << 10) + 4 * m * k
    got = rt.linear(xd, w, **args)
    want = rt.gemm(xd, w, **args)
    small = torch.empty_like(got)
    rt.lib.call('pq8_linear', w.pointer, xd.data_ptr(), small.data_ptr(), args['bias'].data_ptr(),
                args['resid'].data_ptr() if resid is not None else None, m, n, k, epi, args['alpha'], 0,
                rt.workspace.data_ptr(), 64 << 10, rt.stream())
    torch.cuda.synchronize()
    assert rt.device_status() == 0
    np.testing.assert_array_equal(xd.cpu().numpy(), x)
    np.testing.assert_array_equal(got.cpu().numpy(), small.cpu().numpy())
    units = ((m + 127) // 128) * ((n + 127) // 128)
    if 2 * units > 148:  # not split: the launch pq8_gemm makes
        np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())
    check_gemm(got, x, raw, n, k, epi=epi, bias=bias, resid=resid, alpha=args['alpha'])


def test_linear_split_k_in_graph_repeats(rt):
    """Twenty split launches captured in one CUDA graph and replayed three
    times give the bits of the eager calls every time."""
    m, n, k = 128, 1024, 4096
    rng = np.random.default_rng(5)
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k)
    xs = [dev(rng.normal(size=(m, k)).astype(np.float32)) for _ in range(2)]
    ys = [torch.empty(m, n, device='cuda') for _ in range(20)]
    want = [rt.linear(xs[i % 2], w).clone() for i in range(2)]
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        g.capture_begin()
        for i, y in enumerate(ys):
            rt.lib.call('pq8_linear', w.pointer, xs[i % 2].data_ptr(), y.data_ptr(), None, None, m, n, k, EPI_NONE,
                        1.0, 0, rt.workspace.data_ptr(), rt.workspace.numel(), side.cuda_stream)
        g.capture_end()
    torch.cuda.current_stream().wait_stream(side)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert rt.device_status() == 0
    for i, y in enumerate(ys):
        assert torch.equal(y, want[i % 2])
    del g


def test_gemv_epilogues(rt):
    rng = np.random.default_rng(6)
    m, n, k = 4, 1280, 640
    raw = q8_0_blocks(rng, n, k)
    x = rng.normal(size=(m, k)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    for epi in (EPI_RELU, EPI_SILU, EPI_GLU, EPI_RESIDUAL):
        out_n = n // 2 if epi == EPI_GLU else n
        resid = rng.normal(size=(m, out_n)).astype(np.float32)
        w = rt.pack(raw, n, k, LAYOUT_GLU if epi == EPI_GLU else LAYOUT_ROWS)
        y = dev(resid) if epi == EPI_RESIDUAL else None
        y = rt.linear(dev(x), w, out=y, bias=dev(bias), resid=y, epilogue=epi, alpha=0.5).cpu().numpy()
        gold = q8.epilogue(q8.gemm(x, raw, n, k), epi, bias, resid, 0.5)
        np.testing.assert_allclose(y, gold, atol=2e-4 * max(1.0, q8.rms(gold)), rtol=2e-4)


def test_gemv_deterministic(rt):
    rng = np.random.default_rng(8)
    n, k = 8198, 640
    w = rt.pack(q8_0_blocks(rng, n, k), n, k)
    x = dev(rng.normal(size=(1, k)).astype(np.float32))
    ys = [rt.linear(x, w).cpu().numpy() for _ in range(5)]
    for y in ys[1:]:
        np.testing.assert_array_equal(y, ys[0])


def test_layout_mismatch_reports_status(rt):
    rng = np.random.default_rng(9)
    raw = q8_0_blocks(rng, 256, 64)
    glu = rt.pack(raw, 256, 64, LAYOUT_GLU)
    x = dev(rng.normal(size=(40, 64)).astype(np.float32))
    assert rt.device_status() == 0
    rt.gemm(x, glu)  # GLU-packed weights used without the GLU epilogue
    assert rt.device_status() == pq8.ERR_LAYOUT
    rt.linear(x[:2], glu)
    assert rt.device_status() == pq8.ERR_LAYOUT
    assert rt.device_status() == 0


def test_large_shape_rows_sampled(rt):
    """Full-size FFN down projection (M=3000, K=4096, N=1024), sampled rows vs float64."""
    rng = np.random.default_rng(12)
    m, n, k = 3000, 1024, 4096
    raw = q8_0_blocks(rng, n, k)
    x = rng.normal(size=(m, k)).astype(np.float32)
    y = rt.gemm(dev(x), rt.pack(raw, n, k)).cpu().numpy()
    rows = rng.choice(m, 96, replace=False)
    gold = q8.gemm(x[rows], raw, n, k)
    assert q8.max_err_over_rms(y[rows], gold) <= NORTH_STAR
    assert q8.max_err_over_rms(y[rows], q8.gemm_tf32(x[rows], raw, n, k)) <= TF32_EXACT


@pytest.mark.parametrize('cfg', CONFIGS)
def test_gemm_scales_outside_fp16_exact_range(rt, cfg, monkeypatch):
    """Rows whose fp16 scale is subnormal (< 2^-14) or above 511 take the
    fp32 expansion path instead of the fp16 product; both must match the
    TF32 model (weights rounded to nearest-even)."""
    monkeypatch.setenv('PQ8_GEMM_CONFIG', cfg)
    rng = np.random.default_rng(41)
    m, n, k = 96, 256, 256
    raw = q8_0_blocks(rng, n, k, qmin=-128)
    scales = raw[:, :2].copy().view('<f2')
    nb = raw.shape[0]
    pick = rng.integers(0, 4, nb)
    scales[pick == 0, 0] = rng.uniform(1e-7, 6e-5, (pick == 0).sum()).astype(np.float16)  # fp16 subnormals
    scales[pick == 1, 0] = rng.uniform(512.0, 3000.0, (pick == 1).sum()).astype(np.float16)
    scales[pick == 2, 0] = 0
    raw[:, :2] = scales.view(np.uint8)
    x = rng.normal(size=(m, k)).astype(np.float32)
    y = rt.gemm(dev(x), rt.pack(raw, n, k)).cpu().numpy().astype(np.float64)
    tf = q8.gemm_tf32(x, raw, n, k)
    assert np.isfinite(y).all()
    assert float(np.max(np.abs(y - tf))) / q8.rms(tf) <= TF32_EXACT


@pytest.mark.parametrize('cfg', ['0', '1', '4'])
def test_gemm_inplace_rounding_repeatable(rt, cfg, monkeypatch):
    """Several output tiles per CTA with the activations rounded to TF32 inside
    the kernel: every launch must equal the launch on pre-rounded activations
    bit for bit (the same operands in the same order). This catches a weight
    record or activation stage being refilled while still being read."""
    monkeypatch.setenv('PQ8_GEMM_CONFIG', cfg)
    rng = np.random.default_rng(8)
    m, n, k = 8192, 4096, 1024
    w = rt.pack(q8_0_blocks(rng, n, k), n, k)
    x = torch.randn(m, k, device='cuda', generator=torch.Generator(device='cuda').manual_seed(3))
    xr = x.clone()
    rt.lib.call('pq8_round_tf32', xr.data_ptr(), xr.numel(), rt.stream())
    want = rt.gemm(xr, w, flags=pq8.FLAG_X_TF32)
    for _ in range(12):
        got = rt.gemm(x, w)
        assert torch.equal(got, want)
    assert rt.device_status() == 0


@pytest.mark.parametrize('m', [1, 2])
@pytest.mark.parametrize('n,k', [(8192, 2080), (16384, 4096)])
def test_gemv_streamed_weights_match_oracle(rt, m, n, k):
    """Shapes where each CTA streams a long run of K blocks (the HBM regime):
    the weights come in by bulk copies into a shared-memory ring. (8192, 2080)
    ends on a partial chunk and splits K unevenly."""
    rng = np.random.default_rng(n + k + m)
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k)
    x = rng.normal(size=(m, k)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    resid = rng.normal(size=(m, n)).astype(np.float32)
    y, xd, bd = dev(resid), dev(x), dev(bias)  # keep the device copies alive across the launch
    rt.linear(xd, w, out=y, bias=bd, resid=y, epilogue=EPI_RESIDUAL, alpha=0.5)
    gold = resid + 0.5 * (q8.gemm(x, raw, n, k) + bias)
    np.testing.assert_allclose(y.cpu().numpy(), gold, atol=2e-4, rtol=2e-4)
    assert rt.device_status() == 0


@pytest.mark.parametrize('m', [9, 23, 64])
@pytest.mark.parametrize('epi', [EPI_NONE, EPI_GLU, EPI_RESIDUAL])
def test_gemv_row_groups_match_oracle(rt, m, epi):
    """m > 8: one launch runs ceil(m / 8) row groups side by side (grid y),
    each with its own split-K partials and tickets; called twice to check that
    every group's tickets reset themselves."""
    rng = np.random.default_rng(100 + m + epi)
    n, k = 1280, 640
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k, LAYOUT_GLU if epi == EPI_GLU else LAYOUT_ROWS)
    out_n = n // 2 if epi == EPI_GLU else n
    x = rng.normal(size=(m, k)).astype(np.float32)
    bias = rng.normal(size=n).astype(np.float32)
    resid = rng.normal(size=(m, out_n)).astype(np.float32)
    gold = q8.epilogue(q8.gemm(x, raw, n, k), epi, bias, resid, 0.5)
    rt.ensure_workspace(m, n, k)
    xd, bd = dev(x), dev(bias)
    for _ in range(2):
        y = dev(resid)
        rt.lib.call('pq8_gemv', w.pointer, xd.data_ptr(), y.data_ptr(), bd.data_ptr(),
                    y.data_ptr() if epi == EPI_RESIDUAL else None, m, n, k, epi, 0.5, rt.workspace.data_ptr(),
                    rt.workspace.numel(), rt.stream())
        np.testing.assert_allclose(y.cpu().numpy(), gold, atol=2e-4 * max(1.0, q8.rms(gold)), rtol=2e-4)
    assert rt.device_status() == 0


def test_workspace_shared_across_shapes(rt):
    """One workspace for a sequence of shapes: a plan with many split tiles
    after a plan that left split-K partial sums in the same buffer. The
    counters live in an area no plan stores data in, so each call starts from
    zeroed tickets."""
    rng = np.random.default_rng(77)
    # the last shape needs more than 16 K splits, which reduce through workspace partials
    for m, n, k in ((8, 640, 4096), (9, 20000, 2048), (3, 640, 4096), (17, 9000, 1536), (8, 256, 24576)):
        raw = q8_0_blocks(rng, n, k)
        w = rt.pack(raw, n, k)
        x = rng.normal(size=(m, k)).astype(np.float32)
        rt.ensure_workspace(m, n, k)
        xd = dev(x)
        y = torch.empty(m, n, device='cuda')
        rt.lib.call('pq8_gemv', w.pointer, xd.data_ptr(), y.data_ptr(), None, None, m, n, k, EPI_NONE, 1.0,
                    rt.workspace.data_ptr(), rt.workspace.numel(), rt.stream())
        gold = q8.gemm(x, raw, n, k)
        np.testing.assert_allclose(y.cpu().numpy(), gold, atol=2e-4 * max(1.0, q8.rms(gold)), rtol=2e-4)
    assert rt.device_status() == 0


def test_status_clean_at_end(rt):
    torch.cuda.synchronize()
    assert rt.device_status() == 0


def test_gemv_batch_matches_oracle(rt):
    """pq8_gemv_batch: a mix of M = 1 products (short and long K, GLU, residual,
    bias, ragged N) in one launch, each against the float64 product; replays
    of the planned launch give the same bits (the split tickets reset
    themselves)."""
    rng = np.random.default_rng(321)
    shapes = [(1024, 1024, EPI_NONE), (4096, 1024, EPI_SILU), (1024, 4096, EPI_RESIDUAL), (2048, 1024, EPI_GLU),
              (8198, 640, EPI_NONE), (200, 2080, EPI_RELU), (129, 32, EPI_NONE), (640, 8192, EPI_NONE)]
    tasks, keep, golds = [], [], []
    for n, k, epi in shapes:
        raw = q8_0_blocks(rng, n, k)
        w = rt.pack(raw, n, k, LAYOUT_GLU if epi == EPI_GLU else LAYOUT_ROWS)
        x = rng.normal(size=(1, k)).astype(np.float32)
        bias = rng.normal(size=n).astype(np.float32)
        n_out = n // 2 if epi == EPI_GLU else n
        resid = rng.normal(size=(1, n_out)).astype(np.float32) if epi == EPI_RESIDUAL else None
        xd, bd = dev(x), dev(bias)
        rd = dev(resid) if resid is not None else None
        y = torch.full((1, n_out), float('nan'), device='cuda')
        tasks.append(pq8.GemvBatchTask(w.pointer, xd.data_ptr(), y.data_ptr(), bd.data_ptr(),
                                       rd.data_ptr() if rd is not None else None, n, k, epi, 0.5))
        keep += [w, xd, bd, rd, y]
        z = q8.gemm(x, raw, n, k) + bias
        golds.append((y, q8.epilogue(z, epi, None, resid, 0.5), z, epi))
    plan_bytes, ws_bytes = rt.lib.gemv_batch_sizes(tasks)
    plan = torch.empty(plan_bytes, dtype=torch.uint8, device='cuda')
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device='cuda')
    ctas = rt.lib.gemv_batch_plan(tasks, plan.data_ptr(), plan_bytes, ws.data_ptr(), ws_bytes, rt.stream())
    rt.lib.call('pq8_gemv_batch_run', plan.data_ptr(), ctas, rt.stream())
    torch.cuda.synchronize()
    assert rt.device_status() == 0
    first = [g[0].clone() for g in golds]
    for y, gold, z, epi in golds:
        got = y.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all()
        scale = max(1.0, float(np.sqrt((z ** 2).mean())))
        np.testing.assert_allclose(got, gold, atol=2e-4 * scale, rtol=2e-4)
    for _ in range(3):
        rt.lib.call('pq8_gemv_batch_run', plan.data_ptr(), ctas, rt.stream())
    torch.cuda.synchronize()
    for (y, *_), f in zip(golds, first):
        assert torch.equal(y, f)
    assert rt.device_status() == 0


def test_gemv_first_call_in_graph_matches_eager(rt):
    """A GEMV shape whose K splits would form clusters of more than 8 CTAs
    asks, on its first call, how many such clusters the GPU holds (an
    occupancy query, which may fall on a stream being captured into a graph):
    the captured launch must run the same plan as an eager call, bit for bit.
    (N = 4096, K = 1024 at 3 rows: 32 clusters of 16, which do not all fit.)"""
    rng = np.random.default_rng(31)
    m, n, k = 3, 4096, 1024
    raw = q8_0_blocks(rng, n, k)
    w = rt.pack(raw, n, k)
    xh = rng.normal(size=(m, k)).astype(np.float32)
    x = dev(xh)
    rt.ensure_workspace(m, n, k)
    ws = rt.workspace
    y_graph = torch.empty(m, n, device='cuda')
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            rt.lib.call('pq8_gemv', w.pointer, x.data_ptr(), y_graph.data_ptr(), None, None, m, n, k, EPI_NONE,
                        1.0, ws.data_ptr(), ws.numel(), s.cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    y = torch.empty(m, n, device='cuda')
    rt.lib.call('pq8_gemv', w.pointer, x.data_ptr(), y.data_ptr(), None, None, m, n, k, EPI_NONE, 1.0,
                ws.data_ptr(), ws.numel(), rt.stream())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y_graph.cpu().numpy(), y.cpu().numpy())
    np.testing.assert_allclose(y.cpu().numpy(), q8.gemm(xh, raw, n, k), atol=2e-4, rtol=2e-4)
    del g
    assert rt.device_status() == 0
