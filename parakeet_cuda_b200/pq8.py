"""ctypes binding of libpq8.so, in the style of the reference's Driver adapter.

The reference drives CUDA through ctypes (``parakeet_cuda/cuda_driver.py:29-118``)
and turns every nonzero status into ``RuntimeError`` (``cuda_driver.py:90-96``,
``gpu.py:83-85``). This module does the same for the pq8 C ABI declared in
``include/pq8.h``: ``Library.call(name, *args)`` raises ``PQ8Error`` (a
``RuntimeError``) carrying the library's error string and code.

Device pointers are passed as Python ints (``c_void_p``), exactly as the
reference marshals its ``Buffer`` objects (``gpu.py:147-153``). There is no
CPU fallback: loading fails loudly when the shared library is missing.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path
import re

LIB_PATH = Path(__file__).resolve().parent / 'libpq8.so'
HEADER = Path(__file__).resolve().parents[1] / 'include' / 'pq8.h'

OK = 0
ERR_INVALID_ARGUMENT = 1001
ERR_UNSUPPORTED_SHAPE = 1002
ERR_MISALIGNED = 1003
ERR_ARCH = 1004
ERR_WORKSPACE = 1005
ERR_LAYOUT = 1006
ERR_TIMEOUT = 1007
ERR_DRIVER = 1008
ERR_LIBRARY = 1009

LAYOUT_ROWS, LAYOUT_GLU, LAYOUT_GATES4 = 0, 1, 2
EPI_NONE, EPI_RELU, EPI_SILU, EPI_GLU, EPI_RESIDUAL = 0, 1, 2, 3, 4
FLAG_X_TF32, FLAG_OUT_TF32, FLAG_FP32_PRODUCTS = 1, 2, 4
ATTN_FP32 = FLAG_FP32_PRODUCTS
HEADER_BYTES, TILE_ROWS, RECORD_BYTES = 256, 128, 4352
GEMV_MAX_M = 64          # rows the GEMV entry points take (row groups of 8 run in one launch)
LINEAR_GEMV_MAX_M = 8    # pq8_linear's GEMV/GEMM dispatch threshold

_P, _I, _F, _SZ, _LL = C.c_void_p, C.c_int, C.c_float, C.c_size_t, C.c_longlong


class GemmTask(C.Structure):
    """``pq8_gemm_task``: one GEMM of a sequence (``pq8_sequence_plan``)."""
    _fields_ = [('w', _P), ('x', _P), ('y', _P), ('bias', _P), ('resid', _P), ('m', _I), ('n', _I), ('k', _I),
                ('epilogue', _I), ('alpha', _F), ('flags', _I), ('after', _I), ('after_window', _I)]


class GemvBatchTask(C.Structure):
    """``pq8_gemv_task``: one M = 1 product of a GEMV batch (``pq8_gemv_batch_plan``)."""
    _fields_ = [('w', _P), ('x', _P), ('y', _P), ('bias', _P), ('resid', _P), ('n', _I), ('k', _I),
                ('epilogue', _I), ('alpha', _F)]


class TdtWeights(C.Structure):
    """``pq8_tdt_weights``: the prediction and joint networks for ``pq8_tdt_decode``."""
    _fields_ = [('lstm', _P * 2), ('lstm_bias', _P * 2), ('pred', _P), ('pred_bias', _P), ('joint', _P),
                ('joint_bias', _P), ('embed', _P), ('hidden', _I), ('embed_k', _I), ('joint_k', _I),
                ('n_joint', _I), ('vocab', _I)]


SIGNATURES = {
    'pq8_error_string': ([_I], C.c_char_p),
    'pq8_version': ([], _I),
    'pq8_packed_size': ([_I, _I, _I, C.POINTER(_SZ)], _I),
    'pq8_pack_q8_0': ([_P, _I, _I, _I, _P], _I),
    'pq8_pack_q8_0_part': ([_P, _I, _I, _I, _I, _I, _P], _I),
    'pq8_pack_q8_0_device': ([_P, _I, _I, _I, _P, _P], _I),
    'pq8_layer_norm': ([_P, _P, _P, _P, _I, _I, _I, _P], _I),
    'pq8_conv_depthwise_bn_silu': ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P], _I),
    'pq8_attention_workspace_size': ([_I, _I, C.POINTER(_SZ)], _I),
    'pq8_rel_attention': ([_P, _P, _P, _P, _P, _I, _I, _I, _P, _SZ, _P], _I),
    'pq8_stem_workspace_size': ([_I, _I, C.POINTER(_SZ)], _I),
    'pq8_stem': ([_P, _I, _I] + [_P] * 13 + [_I, _P, _SZ, _P], _I),
    'pq8_pack_q8_0_part_device': ([_P, _I, _I, _I, _I, _I, _P, _P], _I),
    'pq8_dequant_q8_0': ([_P, _P, _LL, _P], _I),
    'pq8_round_tf32': ([_P, _LL, _P], _I),
    'pq8_gemm': ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P], _I),
    'pq8_gemv_workspace_size': ([_I, _I, _I, C.POINTER(_SZ)], _I),
    'pq8_linear_workspace_size': ([_I, _I, _I, C.POINTER(_SZ)], _I),
    'pq8_workspace_init': ([_P, _SZ, _P], _I),
    'pq8_gemv': ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P, _SZ, _P], _I),
    'pq8_gemv_static': ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _P], _I),
    'pq8_linear': ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P, _SZ, _P], _I),
    'pq8_lstm_layer': ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _P, _SZ, _P], _I),
    'pq8_joint_argmax': ([_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _SZ, _P], _I),
    'pq8_tdt_commit': ([_P, _P, _P, _P, _P, _I, _I, _I, _P], _I),
    'pq8_tdt_control': ([_P, _P, _I, _P, _I, _I, _P, _P, _P, _P, _I, _P, _I, _P, _P], _I),
    'pq8_tdt_advance': ([_P, _P, _I, _P, _I, _I, _P, _P, _P, _P, _I, _P, _I, _P, _P, _P, _P, _P, _I, _I, _P], _I),
    'pq8_device_status': ([C.POINTER(_I), _P], _I),
    'pq8_sequence_plan_size': ([C.POINTER(GemmTask), _I, C.POINTER(_SZ)], _I),
    'pq8_sequence_plan': ([C.POINTER(GemmTask), _I, _P, _SZ, _P], _I),
    'pq8_sequence_run': ([_P, _P], _I),
    'pq8_gemv_batch_sizes': ([C.POINTER(GemvBatchTask), _I, C.POINTER(_SZ), C.POINTER(_SZ)], _I),
    'pq8_gemv_batch_plan': ([C.POINTER(GemvBatchTask), _I, _P, _SZ, _P, _SZ, C.POINTER(_I), _P], _I),
    'pq8_gemv_batch_run': ([_P, _I, _P], _I),
    'pq8_tdt_decode_workspace_size': ([_I, _I, _I, C.POINTER(_SZ)], _I),
    'pq8_tdt_decode': ([C.POINTER(TdtWeights), _P, _I, _P, _I, _P, _I, _P, _I, _P, _I, _I, _I, _P, _P, _P, _SZ,
                        _P], _I),
}


def header_symbols(path: Path = HEADER):
    """Every function the C header declares (``pq8_*(``)."""
    text = re.sub(r'/\*.*?\*/', '', path.read_text(), flags=re.S)
    return sorted(set(re.findall(r'\b(pq8_\w+)\s*\(', text)))


class PQ8Error(RuntimeError):
    def __init__(self, name: str, code: int, message: str):
        super().__init__(f'{name}: {message} (pq8 {code})')
        self.name, self.code = name, code


class Library:
    """Loaded ``libpq8.so`` with typed entry points."""

    def __init__(self, path: Path | str = LIB_PATH):
        path = Path(path)
        if not path.is_file():
            raise FileNotFoundError(f'{path} is missing: build it with `python -m parakeet_cuda_b200.build`')
        self.path = path
        self.lib = C.CDLL(str(path))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.argtypes, fn.restype = args, res

    def error_string(self, code: int) -> str:
        return self.lib.pq8_error_string(int(code)).decode()

    def call(self, name: str, *args) -> None:
        code = getattr(self.lib, name)(*args)
        if code:
            raise PQ8Error(name, code, self.error_string(code))

    def packed_size(self, n: int, k: int, layout: int = LAYOUT_ROWS) -> int:
        out = _SZ()
        self.call('pq8_packed_size', n, k, layout, C.byref(out))
        return out.value

    def gemv_workspace_size(self, m: int, n: int, k: int) -> int:
        out = _SZ()
        self.call('pq8_gemv_workspace_size', m, n, k, C.byref(out))
        return out.value

    def gemv_batch_sizes(self, tasks) -> tuple[int, int]:
        """(plan bytes, workspace bytes) for a list of ``GemvBatchTask``."""
        arr = (GemvBatchTask * len(tasks))(*tasks)
        plan, ws = _SZ(), _SZ()
        self.call('pq8_gemv_batch_sizes', arr, len(tasks), C.byref(plan), C.byref(ws))
        return plan.value, ws.value

    def gemv_batch_plan(self, tasks, plan, plan_bytes, workspace, workspace_bytes, stream) -> int:
        """Writes the plan; returns the grid size for ``pq8_gemv_batch_run``."""
        arr = (GemvBatchTask * len(tasks))(*tasks)
        ctas = _I()
        self.call('pq8_gemv_batch_plan', arr, len(tasks), plan, plan_bytes, workspace, workspace_bytes,
                  C.byref(ctas), stream)
        return ctas.value

    def tdt_decode_workspace_size(self, m: int, hidden: int, joint_k: int) -> int:
        out = _SZ()
        self.call('pq8_tdt_decode_workspace_size', m, hidden, joint_k, C.byref(out))
        return out.value

    def linear_workspace_size(self, m: int, n: int, k: int) -> int:
        out = _SZ()
        self.call('pq8_linear_workspace_size', m, n, k, C.byref(out))
        return out.value

    def stem_workspace_size(self, windows: int, frames: int) -> int:
        out = _SZ()
        self.call('pq8_stem_workspace_size', windows, frames, C.byref(out))
        return out.value

    def attention_workspace_size(self, windows: int, t: int) -> int:
        out = _SZ()
        self.call('pq8_attention_workspace_size', windows, t, C.byref(out))
        return out.value

    def sequence_plan_size(self, tasks) -> int:
        arr = (GemmTask * len(tasks))(*tasks)
        out = _SZ()
        self.call('pq8_sequence_plan_size', arr, len(tasks), C.byref(out))
        return out.value

    def sequence_plan(self, tasks, plan: int, plan_bytes: int, stream=None) -> None:
        arr = (GemmTask * len(tasks))(*tasks)
        self.call('pq8_sequence_plan', arr, len(tasks), plan, plan_bytes, stream)

    def device_status(self, stream=None) -> int:
        out = _I()
        self.call('pq8_device_status', C.byref(out), stream)
        return out.value


_default = None


def library() -> Library:
    """Process-wide library instance (loaded on first use)."""
    global _default
    if _default is None:
        _default = Library()
    return _default
