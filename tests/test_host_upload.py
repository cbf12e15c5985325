"""Host side of the weight upload (no GPU): the bytes handed to the staging
copy are the source's bytes, also from a read-only memory map as gguf.py
hands them out."""
import numpy as np

from parakeet_cuda_b200.runtime import _host_bytes


def test_host_bytes_of_memmap(tmp_path):
    blocks = np.random.default_rng(1).integers(0, 256, (3000, 34), dtype=np.uint8)
    path = tmp_path / 't.bin'
    blocks.tofile(path)
    m = np.memmap(path, np.uint8, 'r', shape=blocks.shape)
    flat = _host_bytes(m)
    assert flat.dtype.itemsize == 1 and flat.numel() == blocks.size
    np.testing.assert_array_equal(flat.numpy(), blocks.reshape(-1))


def test_host_bytes_of_strided_view():
    a = np.arange(68, dtype=np.uint8).reshape(2, 34)
    flat = _host_bytes(a[:, :])
    np.testing.assert_array_equal(flat.numpy(), a.reshape(-1))
