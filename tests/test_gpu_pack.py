"""GPU parity of the device repack (GGUF Q8_0 bytes copied raw, packed in HBM):
bit-identical to the host packer (pq8_pack.cpp, itself checked against a
restatement of the layout in test_abi.py) for every layout, ragged tiles,
K parts and row-stacked sources."""
import numpy as np
import pytest
import torch

from parakeet_cuda_b200 import pq8
from parakeet_cuda_b200.pq8 import LAYOUT_GATES4, LAYOUT_GLU, LAYOUT_ROWS
from parakeet_cuda_b200.runtime import Runtime, pack_concat_host, pack_host
from parakeet_cuda_b200.synthetic import q8_0_blocks

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def rt():
    return Runtime(0)


@pytest.mark.parametrize('n,k,layout', [(3, 32, LAYOUT_ROWS), (200, 96, LAYOUT_ROWS), (1000, 1024, LAYOUT_ROWS),
                                        (2048, 1024, LAYOUT_GLU), (302, 64, LAYOUT_GLU), (2560, 640, LAYOUT_GATES4),
                                        (400, 288, LAYOUT_GATES4)])
def test_device_pack_matches_host(rt, n, k, layout):
    raw = q8_0_blocks(np.random.default_rng(n + k + layout), n, k)
    want = pack_host(raw, n, k, layout, rt.lib)
    got = rt.pack(raw, n, k, layout).data.cpu().numpy()
    np.testing.assert_array_equal(got, want)
    assert rt.device_status() == 0


def test_device_pack_k_parts_match_host(rt):
    """GATES4 [W_ih | W_hh] along K, as the LSTM layers are packed; a K part
    that is not a multiple of the 8-block chunk of the kernel."""
    rng = np.random.default_rng(5)
    n, k1, k2 = 2560, 640, 96
    a, b = q8_0_blocks(rng, n, k1), q8_0_blocks(rng, n, k2)
    want = pack_concat_host([(a, k1), (b, k2)], n, LAYOUT_GATES4, rt.lib)
    up = rt.uploader()
    w = up.pack([(a, k1), (b, k2)], n, LAYOUT_GATES4)
    up.finish()
    np.testing.assert_array_equal(w.data.cpu().numpy(), want)


def test_device_pack_rows_from_memmap(rt, tmp_path):
    """Q, K and V stacked along N from read-only memory maps of a file (the
    way gguf.py hands out tensor bytes): one packed [3n, k] matrix."""
    rng = np.random.default_rng(6)
    n, k = 256, 1024
    parts = [q8_0_blocks(rng, n, k) for _ in range(3)]
    path = tmp_path / 'blocks.bin'
    np.concatenate([p.reshape(-1) for p in parts]).tofile(path)
    size = parts[0].size
    maps = [np.memmap(path, np.uint8, 'r', offset=i * size, shape=(size,)) for i in range(3)]
    want = pack_host(np.concatenate([p.reshape(-1) for p in parts]), 3 * n, k, LAYOUT_ROWS, rt.lib)
    up = rt.uploader()
    w = up.pack_rows(maps, 3 * n, k, LAYOUT_ROWS)
    up.finish()
    np.testing.assert_array_equal(w.data.cpu().numpy(), want)


def test_device_pack_many_tensors_in_flight(rt):
    """More tensors than staging buffers, of growing size (the buffers are
    reallocated): every result still equals the host packer's."""
    rng = np.random.default_rng(7)
    shapes = [(128, 64), (4096, 1024), (640, 640), (8198, 640), (1024, 4096), (64, 32)]
    raws = [q8_0_blocks(rng, n, k) for n, k in shapes]
    up = rt.uploader()
    ws = [up.pack([(r, k)], n, LAYOUT_ROWS) for r, (n, k) in zip(raws, shapes)]
    up.finish()
    for w, r, (n, k) in zip(ws, raws, shapes):
        np.testing.assert_array_equal(w.data.cpu().numpy(), pack_host(r, n, k, LAYOUT_ROWS, rt.lib))


def test_device_pack_part_header_mismatch(rt):
    """A later K part whose packed buffer carries another shape's header
    records PQ8_ERR_LAYOUT (the host packer returns it)."""
    rng = np.random.default_rng(8)
    n, k = 256, 64
    raw = q8_0_blocks(rng, n, 32)
    buf = torch.zeros(rt.lib.packed_size(n, k, LAYOUT_ROWS), dtype=torch.uint8, device='cuda')
    dev_raw = torch.from_numpy(raw.reshape(-1).copy()).cuda()
    assert rt.device_status() == 0
    rt.lib.call('pq8_pack_q8_0_part_device', dev_raw.data_ptr(), n, 32, k, 32, LAYOUT_ROWS, buf.data_ptr(),
                rt.stream())
    assert rt.device_status() == pq8.ERR_LAYOUT
    rt.lib.call('pq8_pack_q8_0_part_device', dev_raw.data_ptr(), n, 32, k, 0, LAYOUT_ROWS, buf.data_ptr(),
                rt.stream())
    rt.lib.call('pq8_pack_q8_0_part_device', dev_raw.data_ptr(), n, 32, k, 32, LAYOUT_ROWS, buf.data_ptr(),
                rt.stream())
    assert rt.device_status() == 0
