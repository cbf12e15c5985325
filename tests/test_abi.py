"""C-ABI checks that need no GPU: the library loads, exports every symbol the
header declares, rejects bad arguments before touching a device, and its
host-side packer produces the documented layout."""
import ctypes as C
import subprocess

import numpy as np
import pytest

from parakeet_cuda_b200 import pq8
from parakeet_cuda_b200.runtime import pack_concat_host, pack_host
from parakeet_cuda_b200.synthetic import q8_0_blocks


@pytest.fixture(scope='module')
def lib():
    return pq8.library()


def test_library_exports_every_header_symbol(lib):
    declared = pq8.header_symbols()
    assert len(declared) >= 14
    for name in declared:
        assert hasattr(lib.lib, name), name
    out = subprocess.run(['nm', '-D', '--defined-only', str(lib.path)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if ' T ' in line}
    assert set(declared) <= exported
    # nothing but the C ABI is exported
    assert {s for s in exported if s.startswith('pq8_')} == set(declared)
    assert set(pq8.SIGNATURES) == set(declared)


def test_error_strings(lib):
    assert lib.error_string(0) == 'PQ8_OK'
    for code in range(1001, 1010):
        assert lib.error_string(code).startswith('PQ8_ERR_')
    assert 'unknown' in lib.error_string(4242)


def test_argument_validation_without_device(lib):
    with pytest.raises(pq8.PQ8Error) as e:
        lib.call('pq8_gemm', None, None, None, None, None, 4, 128, 33, 0, 1.0, 0, None)
    assert e.value.code == pq8.ERR_UNSUPPORTED_SHAPE
    with pytest.raises(pq8.PQ8Error) as e:
        lib.call('pq8_gemm', None, None, None, None, None, 4, 128, 64, 9, 1.0, 0, None)
    assert e.value.code == pq8.ERR_INVALID_ARGUMENT
    with pytest.raises(pq8.PQ8Error) as e:
        lib.call('pq8_gemm', None, None, None, None, None, 4, 128, 64, 0, 1.0, 0, None)
    assert e.value.code == pq8.ERR_INVALID_ARGUMENT
    # m == 0 is a no-op that needs no device
    lib.call('pq8_gemm', None, None, None, None, None, 0, 128, 64, 0, 1.0, 0, None)
    with pytest.raises(pq8.PQ8Error) as e:
        lib.call('pq8_packed_size', 10, 48, 0, C.byref(C.c_size_t()))
    assert e.value.code == pq8.ERR_UNSUPPORTED_SHAPE
    with pytest.raises(pq8.PQ8Error):
        lib.packed_size(3, 64, pq8.LAYOUT_GLU)


def test_batch_and_decode_sizing_without_device(lib):
    """The GEMV batch and persistent-decode sizing entry points validate and
    size on the host: per task its tile tickets (and split partials when K is
    longer than 32 blocks per CTA); the decode workspace scales with streams."""
    t = lambda n, k, epi=0, resid=None: pq8.GemvBatchTask(16, 16, 16, None, resid, n, k, epi, 1.0)
    plan, ws = lib.gemv_batch_sizes([t(1024, 1024)])
    assert ws == 256  # 8 tiles x 4-byte tickets, rounded to 256; one split: no partials
    _, ws2 = lib.gemv_batch_sizes([t(1024, 4096)])  # 4 splits of 32 K blocks
    assert ws2 == 256 + 8 * 4 * 128 * 4  # tickets + [8 tiles][4 splits][128 rows] partial sums
    plan3, ws3 = lib.gemv_batch_sizes([t(1024, 1024), t(1024, 4096)])
    assert ws3 == ws + ws2
    assert plan3 - plan == plan - 16  # a 16-byte header and one fixed-size entry per task
    for bad, code in ((t(1024, 1000), pq8.ERR_UNSUPPORTED_SHAPE), (t(1023, 64, 3), pq8.ERR_UNSUPPORTED_SHAPE),
                      (t(64, 64, 4), pq8.ERR_INVALID_ARGUMENT), (t(64, 64, 9), pq8.ERR_INVALID_ARGUMENT)):
        with pytest.raises(pq8.PQ8Error) as e:
            lib.gemv_batch_sizes([bad])
        assert e.value.code == code
    bad_align = pq8.GemvBatchTask(16, 20, 16, None, None, 64, 64, 0, 1.0)
    with pytest.raises(pq8.PQ8Error) as e:
        lib.gemv_batch_sizes([bad_align])
    assert e.value.code == pq8.ERR_MISALIGNED
    one, many = lib.tdt_decode_workspace_size(1, 640, 640), lib.tdt_decode_workspace_size(64, 640, 640)
    assert 0 < one < many
    with pytest.raises(pq8.PQ8Error) as e:
        lib.tdt_decode_workspace_size(65, 640, 640)
    assert e.value.code == pq8.ERR_UNSUPPORTED_SHAPE


def reference_pack(raw, n, k, layout):
    """Restatement of the packed layout documented in include/pq8.h / pq8_pack.cpp."""
    blocks = np.asarray(raw, np.uint8).reshape(n, k // 32, 34)
    tiles = (n + 127) // 128
    kb = k // 32
    data = np.zeros((tiles, kb, 4352), np.uint8)
    for t in range(tiles):
        for r in range(128):
            p = t * 128 + r
            if layout == pq8.LAYOUT_ROWS:
                src = p if p < n else -1
            elif layout == pq8.LAYOUT_GLU:
                h, w, l = n // 2, r // 32, r % 32
                j = t * 64 + w * 16 + l % 16
                src = -1 if j >= h else (j if l < 16 else h + j)
            else:
                h, g, u = n // 4, r // 32, t * 32 + r % 32
                src = g * h + u if u < h else -1
            if src < 0:
                continue
            data[t, :, r * 16:r * 16 + 16] = blocks[src, :, 2:18]
            data[t, :, 2048 + r * 16:2048 + r * 16 + 16] = blocks[src, :, 18:34]
            data[t, :, 4096 + 2 * r:4096 + 2 * r + 2] = blocks[src, :, 0:2]
    return data.reshape(-1)


@pytest.mark.parametrize('n,k,layout', [(3, 32, 0), (129, 64, 0), (256, 96, 1), (130, 32, 1), (2560, 64, 2),
                                        (640, 32, 2)])
def test_host_packer_layout(lib, n, k, layout):
    raw = q8_0_blocks(np.random.default_rng(n + k), n, k, qmin=-128)
    packed = pack_host(raw, n, k, layout)
    assert packed.size == lib.packed_size(n, k, layout)
    hdr = packed[:32].view(np.int32)
    assert packed[:4].tobytes() == b'PQ8P'
    assert list(hdr[2:8]) == [n, k, layout, (n + 127) // 128, k // 32,
                              n // 2 if layout == 1 else n // 4 if layout == 2 else n]
    np.testing.assert_array_equal(packed[256:], reference_pack(raw, n, k, layout))


def test_host_packer_k_concat(lib):
    rng = np.random.default_rng(5)
    a, b = q8_0_blocks(rng, 256, 64), q8_0_blocks(rng, 256, 96)
    both = np.concatenate([a.reshape(256, 2, 34), b.reshape(256, 3, 34)], axis=1).reshape(-1, 34)
    np.testing.assert_array_equal(pack_concat_host([(a, 64), (b, 96)], 256, pq8.LAYOUT_GATES4),
                                  pack_host(both, 256, 160, pq8.LAYOUT_GATES4))


C_PROGRAM = r'''
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "pq8.h"

int main(void) {
  const int n = 130, k = 64; /* two 128-row tiles, two 32-wide K blocks */
  size_t bytes = 0;
  unsigned char *gguf, *packed;
  int r, b, i;
  if (pq8_version() <= 0) return 1;
  if (strncmp(pq8_error_string(PQ8_ERR_WORKSPACE), "PQ8_ERR_WORKSPACE", 17) != 0) return 2;
  if (pq8_packed_size(n, k, PQ8_LAYOUT_ROWS, &bytes) != PQ8_OK) return 3;
  if (bytes != 256 + 2 * 2 * 4352) return 4; /* header + tiles x K blocks x record */
  gguf = calloc((size_t)n * (k / 32), 34);
  packed = malloc(bytes);
  if (!gguf || !packed) return 5;
  for (r = 0; r < n; ++r)
    for (b = 0; b < k / 32; ++b) {
      unsigned char* blk = gguf + ((size_t)r * (k / 32) + b) * 34;
      blk[0] = 0x00; blk[1] = 0x3c; /* fp16 1.0 */
      for (i = 0; i < 32; ++i) blk[2 + i] = (unsigned char)(r + i);
    }
  if (pq8_pack_q8_0(gguf, n, k, PQ8_LAYOUT_ROWS, packed) != PQ8_OK) return 6;
  if (memcmp(packed, "PQ8P", 4) != 0) return 7;
  /* a bad shape is rejected before any device is touched */
  if (pq8_gemm(NULL, NULL, NULL, NULL, NULL, 4, 128, 33, 0, 1.0f, 0, NULL) != PQ8_ERR_UNSUPPORTED_SHAPE) return 8;
  printf("ok %d\n", pq8_version());
  free(gguf);
  free(packed);
  return 0;
}
'''


def test_header_is_plain_c_and_links(lib, tmp_path):
    """include/pq8.h compiles as strict C99 and a C program linked against
    libpq8.so calls the host-side entry points (no GPU involved): the boundary
    is a C ABI, not a C++ or Python one."""
    src = tmp_path / 'abi.c'
    src.write_text(C_PROGRAM)
    exe = tmp_path / 'abi'
    libdir = str(lib.path.parent)
    include = str(lib.path.parents[1] / 'include')
    r = subprocess.run(['gcc', '-std=c99', '-Wall', '-Wextra', '-Werror', '-pedantic', '-I', include, str(src), '-o',
                        str(exe), '-L', libdir, '-lpq8', f'-Wl,-rpath,{libdir}'], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.startswith('ok '), (run.returncode, run.stdout, run.stderr)
