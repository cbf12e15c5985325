"""GPU parity of the block around the linears: LayerNorm, the conv module's
depthwise/BatchNorm/SiLU, the relative-position attention, and whole blocks
against the reference's own block outputs (tests/golden/block.npz) and the
float64 oracle (oracle/block.py).

Tolerances: the LayerNorm and the depthwise kernel are FP32 arithmetic
(1e-5 absolute on O(1) values, 1 TF32 ulp when the output is TF32-rounded).
The attention with FP32 products (cuBLAS) is checked at 2e-5; the fused
kernel (FP16 operands: TF32's significand, FP32 accumulation) at the
north-star GEMM bar (max |err| <= 2e-3 x RMS). A whole block chains 11
TF32 GEMMs and the attention, then LayerNorms the result: its bar is
max |err| <= 1e-2 and RMS error <= 2e-3 on the unit-RMS output.
"""
import numpy as np
import pytest
import torch

from oracle import block as ob
from parakeet_cuda_b200 import pq8
from parakeet_cuda_b200.block import EncoderBlocks
from parakeet_cuda_b200.runtime import Runtime
from parakeet_cuda_b200.synthetic import SyntheticParakeet

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def rt():
    return Runtime(0)


@pytest.fixture(scope='module')
def model():
    return SyntheticParakeet(seed=31, encoder_layers=2, decoder=False, block=True)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def tf32_rna(a):
    """Round float32 to TF32, ties away from zero (the kernels' output rounding)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)


@pytest.mark.parametrize('rows,width', [(37, 1024), (5, 256), (300, 640)])
@pytest.mark.parametrize('flags', [0, pq8.FLAG_OUT_TF32])
def test_layer_norm(rt, rows, width, flags):
    rng = np.random.default_rng(rows + width)
    x = (3.0 * rng.normal(size=(rows, width)) + 0.5).astype(np.float32)
    w = (1 + 0.1 * rng.normal(size=width)).astype(np.float32)
    b = (0.1 * rng.normal(size=width)).astype(np.float32)
    xd, wd, bd = dev(x), dev(w), dev(b)
    y = torch.empty_like(xd)
    rt.lib.call('pq8_layer_norm', xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), y.data_ptr(), rows, width, flags,
                rt.stream())
    gold = ob.layer_norm(x, w, b)
    got = y.cpu().numpy()
    if flags:
        assert np.array_equal(got, tf32_rna(got))
        np.testing.assert_allclose(got, gold, atol=2e-5, rtol=2 ** -10)
    else:
        np.testing.assert_allclose(got, gold, atol=2e-5, rtol=0)


def test_layer_norm_in_place(rt):
    x = np.random.default_rng(1).normal(size=(64, 1024)).astype(np.float32)
    w, b = np.ones(1024, np.float32), np.zeros(1024, np.float32)
    xd, wd, bd = dev(x), dev(w), dev(b)
    rt.lib.call('pq8_layer_norm', xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), xd.data_ptr(), 64, 1024, 0, rt.stream())
    np.testing.assert_allclose(xd.cpu().numpy(), ob.layer_norm(x, w, b), atol=2e-5)


@pytest.mark.parametrize('windows,t', [(3, 50), (1, 7), (2, 33)])
def test_conv_depthwise_bn_silu(rt, model, windows, t):
    wts = ob.BlockWeights(model, 0)
    x = np.random.default_rng(windows * t).normal(size=(windows * t, 1024)).astype(np.float32)
    raw = np.ascontiguousarray(model.raw('encoder.layers.0.conv.depthwise_conv.weight')).view(np.int16)
    wd = torch.from_numpy(raw.copy()).cuda()
    bn = [dev(wts.bn[n]) for n in ('weight', 'bias', 'running_mean', 'running_var')]
    xd = dev(x)
    y = torch.empty_like(xd)
    rt.lib.call('pq8_conv_depthwise_bn_silu', xd.data_ptr(), wd.data_ptr(), *[p.data_ptr() for p in bn], y.data_ptr(),
                windows, t, 1024, 0, rt.stream())
    gold = np.concatenate([ob.conv_module_depthwise(wts, x[i * t:(i + 1) * t]) for i in range(windows)])
    np.testing.assert_allclose(y.cpu().numpy(), gold, atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize('fp32', [True, False])
# t = 200 / 300 / 500 take the register softmax with 8 / 12 / 16 scores per
# lane, t = 600 the three-pass form
@pytest.mark.parametrize('windows,t', [(2, 40), (1, 9), (3, 64), (1, 200), (2, 300), (1, 500), (1, 600)])
def test_rel_attention(rt, windows, t, fp32):
    rng = np.random.default_rng(7 * windows + t)
    qkv = (0.5 * rng.normal(size=(windows * t, 3072))).astype(np.float32)
    pos = (0.5 * rng.normal(size=(2 * t - 1, 1024))).astype(np.float32)
    u, v = (0.1 * rng.normal(size=1024)).astype(np.float32), (0.1 * rng.normal(size=1024)).astype(np.float32)
    ws = torch.empty(rt.lib.attention_workspace_size(windows, t), dtype=torch.uint8, device='cuda')
    qd, pd, ud, vd = dev(qkv), dev(pos), dev(u), dev(v)
    ctx = torch.empty(windows * t, 1024, device='cuda')
    rt.lib.call('pq8_rel_attention', qd.data_ptr(), pd.data_ptr(), ud.data_ptr(), vd.data_ptr(), ctx.data_ptr(),
                windows, t, pq8.ATTN_FP32 if fp32 else 0, ws.data_ptr(), ws.numel(), rt.stream())
    heads = lambda y: y.reshape(-1, 8, 128).transpose(1, 0, 2).astype(np.float64)
    p = heads(pos)
    gold = []
    for w in range(windows):
        blk = qkv[w * t:(w + 1) * t]
        q, k, vv = heads(blk[:, :1024]), heads(blk[:, 1024:2048]), heads(blk[:, 2048:])
        s = ob.rel_shift_scores(q + u.reshape(8, 1, 128), q + v.reshape(8, 1, 128), k, p)
        gold.append((ob.softmax(s) @ vv).transpose(1, 0, 2).reshape(t, 1024))
    gold = np.concatenate(gold)
    got = ctx.cpu().numpy()
    err = np.abs(got - gold).max() / np.sqrt((gold ** 2).mean())
    assert err <= (2e-5 if fp32 else 2e-3), err
    assert rt.device_status() == 0


def _block_errors(got, gold):
    d = got.astype(np.float64) - gold
    return float(np.abs(d).max()), float(np.sqrt((d ** 2).mean()))


@pytest.mark.parametrize('t,layers', [(40, 1), (40, 2), (7, 1)])
def test_blocks_match_reference_golden(rt, model, golden_dir, t, layers):
    d = np.load(golden_dir / 'block.npz')
    gold = d[f't{t}_layer{layers - 1}'].astype(np.float64)
    blocks = EncoderBlocks(model, rt, 1, t, layers=layers)
    got = blocks.forward(dev(d[f't{t}_x'])).cpu().numpy()
    mx, rms = _block_errors(got, gold)
    print(f't={t} layers={layers}: max {mx:.2e} rms {rms:.2e}')
    assert mx <= 1e-2 and rms <= 2e-3, (mx, rms)
    assert rt.device_status() == 0


def test_blocks_config1_length_match_oracle(rt, model):
    """One and two blocks over 8 windows of T = 375 frames (the config-1 window
    length, as the benchmark's whole-block leg runs them) against the float64
    oracle. The residual stream before a block's norm_out is its unit-RMS
    input plus four branch outputs, each ending in a GEMM (FFN down,
    linear_out, pointwise_conv2): after one block it is held to the north-star
    bar, max |err| <= 2e-3 x RMS; after two blocks to twice that, since the
    second block starts from the first block's output with that error. The
    LayerNormed outputs are held to the whole-block bar above."""
    windows, t = 8, 375
    x = np.random.default_rng(375).normal(size=(windows * t, 1024)).astype(np.float32)
    gold_in = np.asarray(x, np.float64)
    for layers, bar in ((1, 2e-3), (2, 4e-3)):
        blocks = EncoderBlocks(model, rt, windows, t, layers=layers)
        pre = blocks.forward(dev(x), final_norm=False).cpu().numpy()
        post = blocks.forward(dev(x)).cpu().numpy()
        gold_pre = ob.blocks(gold_in, model, [layers - 1], windows=windows, final_norm=False)
        gold_post = ob.layer_norm(gold_pre, *ob.BlockWeights(model, layers - 1).ln['norm_out'])
        e_pre = _rel_max(pre, gold_pre)
        mx, rms = _block_errors(post, gold_post)
        print(f'8 x 375, {layers} layer(s): before norm_out max err / rms {e_pre:.2e}; '
              f'output max {mx:.2e} rms {rms:.2e}')
        assert e_pre <= bar, (layers, e_pre)
        assert mx <= 1e-2 and rms <= 2e-3, (layers, mx, rms)
        gold_in = gold_post
    assert rt.device_status() == 0


def test_blocks_windows_are_independent(rt, model):
    """Three windows in one stream give each window's own result: the depthwise
    convolution and the attention stop at window boundaries."""
    t = 50
    x = np.random.default_rng(9).normal(size=(3 * t, 1024)).astype(np.float32)
    many = EncoderBlocks(model, rt, 3, t, layers=1).forward(dev(x)).cpu().numpy()
    one = EncoderBlocks(model, rt, 1, t, layers=1)
    for w in range(3):
        single = one.forward(dev(x[w * t:(w + 1) * t])).cpu().numpy()
        np.testing.assert_allclose(many[w * t:(w + 1) * t], single, atol=1e-5, rtol=0)
    gold = ob.blocks(x, model, [0], windows=3)
    mx, rms = _block_errors(many, gold)
    assert mx <= 1e-2 and rms <= 2e-3, (mx, rms)


def test_blocks_graph_replay_matches_eager(rt, model):
    t = 40
    x = dev(np.random.default_rng(10).normal(size=(2 * t, 1024)))
    blocks = EncoderBlocks(model, rt, 2, t, layers=2)
    eager = blocks.forward(x).clone()
    blocks.buf['x'].copy_(x)
    graph = blocks.capture()
    blocks.buf['x'].copy_(x)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(blocks.buf['x'], eager)


def _rel_max(got, gold):
    return float(np.abs(got.astype(np.float64) - gold).max() / np.sqrt((gold.astype(np.float64) ** 2).mean()))


@pytest.mark.parametrize('fp32', [False, True])
def test_stem_matches_reference_golden(rt, model, golden_dir, fp32):
    """The reference's own stem on 50, 17 and 1 mel frames. Bar: the GEMM
    north-star bar on the output (TF32 pointwise products and output linear),
    max |err| <= 2e-3 x RMS; the output linear alone is TF32 with FP32 products."""
    from parakeet_cuda_b200.block import EncoderStem
    d = np.load(golden_dir / 'block.npz')
    for frames in (50, 17, 1):
        stem = EncoderStem(model, rt, 1, frames, fp32_products=fp32)
        got = stem.forward(dev(d[f'stem{frames}_mel'])[None]).cpu().numpy()
        err = _rel_max(got, d[f'stem{frames}_out'])
        print(f'stem frames={frames} fp32={fp32}: max err / rms {err:.2e}')
        assert err <= 2e-3, err
    assert rt.device_status() == 0


def test_stem_windows_are_independent(rt, model):
    from oracle import stem as ostem
    from parakeet_cuda_b200.block import EncoderStem
    frames = 45
    mel = np.random.default_rng(11).normal(size=(3, frames, 128)).astype(np.float32)
    many = EncoderStem(model, rt, 3, frames).forward(dev(mel)).cpu().numpy()
    t = many.shape[0] // 3
    for w in range(3):
        one = EncoderStem(model, rt, 1, frames).forward(dev(mel[w:w + 1])).cpu().numpy()
        np.testing.assert_allclose(many[w * t:(w + 1) * t], one, atol=1e-6, rtol=0)
        assert _rel_max(one, ostem.stem(mel[w], model)) <= 2e-3


@pytest.mark.parametrize('windows,t', [(1, 1), (2, 1), (1, 2), (3, 65)])
def test_blocks_edge_lengths(rt, model, windows, t):
    """One-frame windows (one key, one positional row), two frames, and a window
    one frame past a 64-query tile, against the float64 oracle."""
    x = np.random.default_rng(40 + t).normal(size=(windows * t, 1024)).astype(np.float32)
    got = EncoderBlocks(model, rt, windows, t, layers=1).forward(dev(x)).cpu().numpy()
    mx, rms = _block_errors(got, ob.blocks(x, model, [0], windows=windows))
    assert mx <= 1e-2 and rms <= 2e-3, (mx, rms)
    assert rt.device_status() == 0


@pytest.mark.parametrize('frames', [2, 3, 8, 9])
def test_stem_edge_lengths(rt, model, frames):
    from oracle import stem as ostem
    from parakeet_cuda_b200.block import EncoderStem
    mel = np.random.default_rng(60 + frames).normal(size=(2, frames, 128)).astype(np.float32)
    got = EncoderStem(model, rt, 2, frames).forward(dev(mel)).cpu().numpy()
    t = got.shape[0] // 2
    for w in range(2):
        assert _rel_max(got[w * t:(w + 1) * t], ostem.stem(mel[w], model)) <= 2e-3
