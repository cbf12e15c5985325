"""The torch-free host layer (parakeet_cuda_b200.host over cuda_driver.py and
the ctypes binding) imports and loads libpq8.so in a process where importing
PyTorch fails, as the reference's host code runs without it."""
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

BLOCK_TORCH = '''
import sys
class _NoTorch:
    def find_spec(self, name, path=None, target=None):
        if name == 'torch' or name.startswith('torch.'):
            raise ImportError('torch is not available in this process')
        return None
sys.meta_path.insert(0, _NoTorch())
'''


def test_host_layer_imports_without_torch():
    code = BLOCK_TORCH + '''
try:
    import torch
    raise SystemExit('torch import was not blocked')
except ImportError:
    pass
from parakeet_cuda_b200 import cuda_driver, host, layers, pq8, synthetic
lib = pq8.Library()
assert lib.packed_size(4096, 1024, 0) > 4096 * 1024
assert len(layers.LAYER_PLAN) == 9
assert 'torch' not in sys.modules
print('ok')
'''
    r = subprocess.run([sys.executable, '-c', code], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().endswith('ok')


def test_arena_and_buffer_views_without_a_device():
    from parakeet_cuda_b200.host import Arena, Buffer

    class FakeDriver:
        def alloc(self, n):
            return 1 << 20

        def free(self, p):
            pass

    a = Arena(FakeDriver(), 4096, 'test')
    x = a.alloc((3, 5))
    y = a.alloc(10)
    assert x.pointer == 1 << 20 and x.nbytes == 60
    assert y.pointer == (1 << 20) + 256  # 256-byte aligned pieces
    v = x.view(4, 8, (2,))
    assert v.pointer == x.pointer + 4 and v.nbytes == 8
    try:
        x.view(56, 8)
        raise AssertionError('view past the end was accepted')
    except ValueError:
        pass
    try:
        a.alloc(4096)
        raise AssertionError('arena overflow was accepted')
    except MemoryError:
        pass
    a.reset()
    assert a.alloc(16).pointer == 1 << 20
    assert isinstance(Buffer(0, 0), Buffer)
