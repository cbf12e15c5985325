"""Host-side mirror of the reference's device runtime for the Q8_0 contraction path.

The reference keeps weights as GGUF Q8_0 bytes on the host, uploads a layer
at a time and expands it to FP32 with ``dequant_q8`` before every
``cublasSgemm_v2`` (``GPU.load_weights`` ``parakeet_cuda/gpu.py:169-184``,
``Blas.linear`` ``gpu.py:87-90``). Here the Q8_0 bytes are repacked once
(``pq8_pack_q8_0``), uploaded once and stay resident (all 24 encoder layers
are 642 MB), and every linear runs the fused library kernel on them.

``Runtime.load_weights(model, names)`` and ``Runtime.linear(...)`` keep the
reference's call shapes (``model`` is any object with ``gguf.Model``'s
``tensors``/``raw``/``array``). PyTorch is used only to own device memory and
streams; all arithmetic is in ``libpq8.so``.
"""
from __future__ import annotations

from dataclasses import dataclass
import ctypes as C
import warnings

import numpy as np
import torch

from . import pq8
from .pq8 import EPI_GLU, EPI_NONE, GEMV_MAX_M, LAYOUT_GATES4, LAYOUT_GLU, LAYOUT_ROWS

MIB = 1 << 20


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


@dataclass
class PackedWeight:
    """A resident packed Q8_0 tensor: ``n`` rows x ``k`` columns in ``layout``."""
    data: torch.Tensor  # uint8, device
    n: int
    k: int
    layout: int

    @property
    def pointer(self) -> int:
        return self.data.data_ptr()

    @property
    def out_features(self) -> int:
        return self.n // 2 if self.layout == LAYOUT_GLU else self.n // 4 if self.layout == LAYOUT_GATES4 else self.n


def pack_host(raw, n: int, k: int, layout: int = LAYOUT_ROWS, lib=None) -> np.ndarray:
    """Repack GGUF Q8_0 bytes (``n*k/32`` x 34) into the packed format on the host."""
    lib = lib or pq8.library()
    raw = np.ascontiguousarray(raw, np.uint8)
    if raw.size != n * k // 32 * 34:
        raise ValueError(f'expected {n * k // 32 * 34} Q8_0 bytes for [{n}, {k}], got {raw.size}')
    out = np.empty(lib.packed_size(n, k, layout), np.uint8)
    lib.call('pq8_pack_q8_0', raw.ctypes.data, n, k, layout, out.ctypes.data)
    return out


def pack_concat_host(parts, n: int, layout: int, lib=None) -> np.ndarray:
    """Pack several ``[n, k_i]`` Q8_0 sources side by side along K (``parts = [(raw, k_i), ...]``)."""
    lib = lib or pq8.library()
    k_total = sum(k for _, k in parts)
    out = np.empty(lib.packed_size(n, k_total, layout), np.uint8)
    off = 0
    for raw, k in parts:
        raw = np.ascontiguousarray(raw, np.uint8)
        lib.call('pq8_pack_q8_0_part', raw.ctypes.data, n, k, k_total, off, layout, out.ctypes.data)
        off += k
    return out


def _host_bytes(raw) -> torch.Tensor:
    """A uint8 CPU tensor over ``raw``'s bytes (a GGUF memmap slice or any array), without a copy
    when ``raw`` is contiguous."""
    arr = np.ascontiguousarray(raw).reshape(-1).view(np.uint8)
    with warnings.catch_warnings():
        warnings.simplefilter('ignore')  # read-only memmaps: the tensor is only ever read
        return torch.from_numpy(arr)


class _Slot:
    def __init__(self, nbytes: int, device, side: torch.cuda.Stream):
        self.host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
        self.dev = torch.empty(nbytes, dtype=torch.uint8, device=device)
        self.dev.record_stream(side)
        self.done = torch.cuda.Event()
        self.done.record(torch.cuda.current_stream(device))


class WeightUploader:
    """GGUF Q8_0 bytes -> resident packed weights, repacked on the device.

    Each tensor's raw bytes are copied (by torch's multi-threaded CPU copy)
    into one of two pinned staging buffers, sent to the device by an
    asynchronous copy on a side stream and repacked there by
    ``pq8_pack_q8_0_part_device``; meanwhile the host fills the other staging
    buffer. Nothing is packed or expanded on the host. This replaces the
    per-layer upload and ``dequant_q8`` of ``GPU.load_weights``
    (``parakeet_cuda/gpu.py:169-184``), which the reference repeats for every
    window. ``finish()`` makes the caller's stream wait for the uploads."""

    def __init__(self, runtime: 'Runtime', slot_bytes: int = 8 * MIB):
        self.rt = runtime
        self.side = torch.cuda.Stream(runtime.device)
        self.side.wait_stream(torch.cuda.current_stream(runtime.device))
        self.slots = [_Slot(slot_bytes, runtime.device, self.side) for _ in range(2)]
        self.turn = 0
        self.bytes_uploaded = 0

    def _slot(self, nbytes: int) -> _Slot:
        slot = self.slots[self.turn]
        self.turn ^= 1
        slot.done.synchronize()  # its previous copy and repack have finished reading it
        if slot.host.numel() < nbytes:
            self.slots[self.turn ^ 1] = slot = _Slot(max(nbytes, 2 * slot.host.numel()), self.rt.device, self.side)
            self.side.wait_stream(torch.cuda.current_stream(self.rt.device))
        return slot

    def _stage(self, raws) -> tuple[_Slot, int]:
        """Copy ``raws`` back to back into a staging buffer and start its upload."""
        srcs = [_host_bytes(r) for r in raws]
        nbytes = sum(t.numel() for t in srcs)
        slot = self._slot(nbytes)
        off = 0
        for t in srcs:  # torch's CPU copy (threaded for large tensors) into pinned memory
            slot.host[off:off + t.numel()].copy_(t)
            off += t.numel()
        with torch.cuda.stream(self.side):
            slot.dev[:nbytes].copy_(slot.host[:nbytes], non_blocking=True)
        self.bytes_uploaded += nbytes
        return slot, nbytes

    def _output(self, nbytes: int) -> torch.Tensor:
        # allocated for the caller's stream, written on the side stream
        out = torch.empty(nbytes, dtype=torch.uint8, device=self.rt.device)
        self.side.wait_stream(torch.cuda.current_stream(self.rt.device))
        out.record_stream(self.side)
        return out

    def pack(self, parts, n: int, layout: int = LAYOUT_ROWS) -> PackedWeight:
        """``parts = [(raw, k_i), ...]``: GGUF Q8_0 ``[n, k_i]`` sources packed side by side along K."""
        lib = self.rt.lib
        k_total = sum(k for _, k in parts)
        packed = self._output(lib.packed_size(n, k_total, layout))
        off = 0
        for raw, k in parts:
            slot, nbytes = self._stage([raw])
            if nbytes != n * k // 32 * 34:
                raise ValueError(f'expected {n * k // 32 * 34} Q8_0 bytes for [{n}, {k}], got {nbytes}')
            with torch.cuda.stream(self.side):
                lib.call('pq8_pack_q8_0_part_device', slot.dev.data_ptr(), n, k, k_total, off, layout,
                         packed.data_ptr(), C.c_void_p(self.side.cuda_stream))
                slot.done.record(self.side)
            off += k
        return PackedWeight(packed, n, k_total, layout)

    def pack_rows(self, raws, n: int, k: int, layout: int = LAYOUT_ROWS) -> PackedWeight:
        """GGUF Q8_0 sources stacked along N (e.g. Q, K, V into one [3n', k] matrix)."""
        lib = self.rt.lib
        packed = self._output(lib.packed_size(n, k, layout))
        slot, nbytes = self._stage(raws)
        if nbytes != n * k // 32 * 34:
            raise ValueError(f'expected {n * k // 32 * 34} Q8_0 bytes for [{n}, {k}], got {nbytes}')
        with torch.cuda.stream(self.side):
            lib.call('pq8_pack_q8_0_device', slot.dev.data_ptr(), n, k, layout, packed.data_ptr(),
                     C.c_void_p(self.side.cuda_stream))
            slot.done.record(self.side)
        return PackedWeight(packed, n, k, layout)

    def finish(self) -> None:
        torch.cuda.current_stream(self.rt.device).wait_stream(self.side)


class Runtime:
    """One device's resident weights, workspace and launch helpers."""

    def __init__(self, device: int | torch.device = 0, workspace_bytes: int = 8 * MIB):
        if not torch.cuda.is_available():
            raise RuntimeError('pq8 needs a CUDA device (B200, sm_100a); no CPU fallback exists')
        self.device = torch.device('cuda', device) if isinstance(device, int) else torch.device(device)
        self.lib = pq8.library()
        with torch.cuda.device(self.device):
            self.workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device=self.device)
            self.lib.call('pq8_workspace_init', self.workspace.data_ptr(), workspace_bytes, self.stream())
        self.weights: dict[str, object] = {}
        self._uploader: WeightUploader | None = None

    # -- plumbing ---------------------------------------------------------
    def stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def upload_packed(self, packed: np.ndarray, n: int, k: int, layout: int) -> PackedWeight:
        host = torch.from_numpy(np.ascontiguousarray(packed))
        return PackedWeight(host.to(self.device, non_blocking=False), n, k, layout)

    def uploader(self) -> WeightUploader:
        if self._uploader is None:
            self._uploader = WeightUploader(self)
        return self._uploader

    def pack(self, raw, n: int, k: int, layout: int = LAYOUT_ROWS) -> PackedWeight:
        """Resident packed copy of GGUF Q8_0 bytes ``raw`` ([n, k]), repacked on the device."""
        up = self.uploader()
        w = up.pack([(raw, k)], n, layout)
        up.finish()
        return w

    # -- GPU.load_weights counterpart ---------------------------------------
    def load_weights(self, model, names, layouts: dict | None = None) -> dict:
        """Upload tensors once and keep them resident.

        Q8_0 tensors are repacked (``layouts[name]`` selects GLU pairing);
        F32 tensors become float32 device tensors; F16 tensors stay fp16.
        """
        layouts = layouts or {}
        up = self.uploader()
        for name in names:
            t = model.tensors[name]
            if t.kind == 8:
                n, k = t.shape[0], int(np.prod(t.shape[1:]))
                self.weights[name] = up.pack([(model.raw(name), k)], n, layouts.get(name, LAYOUT_ROWS))
            elif t.kind == 1:
                self.weights[name] = torch.from_numpy(np.ascontiguousarray(model.raw(name)).view(np.float16).copy()
                                                      ).reshape(t.shape).to(self.device)
            else:
                self.weights[name] = torch.from_numpy(np.ascontiguousarray(model.raw(name)).view(np.float32).copy()
                                                      ).reshape(t.shape).to(self.device)
        up.finish()
        return self.weights

    def weight(self, name):
        return self.weights[name]

    # -- workspace ----------------------------------------------------------
    def ensure_workspace(self, m: int, n: int, k: int) -> None:
        need = self.lib.linear_workspace_size(m, n, k)
        if need > self.workspace.numel():
            with torch.cuda.device(self.device):
                self.workspace = torch.empty(max(need, 2 * self.workspace.numel()), dtype=torch.uint8,
                                             device=self.device)
                self.lib.call('pq8_workspace_init', self.workspace.data_ptr(), self.workspace.numel(), self.stream())

    # -- Blas.linear counterpart ---------------------------------------------
    def linear(self, x: torch.Tensor, w: PackedWeight, out: torch.Tensor | None = None, bias=None, resid=None,
               epilogue: int = EPI_NONE, alpha: float = 1.0, flags: int = 0) -> torch.Tensor:
        """``out = epilogue(x @ W^T + bias)`` for a resident packed ``w`` (any number of rows)."""
        rows, k = x.shape
        if k != w.k:
            raise ValueError(f'x has {k} columns, weight has {w.k}')
        if out is None:
            out = torch.empty(rows, w.out_features if epilogue == EPI_GLU else w.n, dtype=torch.float32,
                              device=self.device)
        if rows >= 1:
            self.ensure_workspace(rows, w.n, k)
        self.lib.call('pq8_linear', w.pointer, x.data_ptr(), out.data_ptr(), _ptr(bias), _ptr(resid), rows, w.n, k,
                      epilogue, float(alpha), flags, self.workspace.data_ptr(), self.workspace.numel(),
                      self.stream())
        return out

    def gemm(self, x, w: PackedWeight, out=None, bias=None, resid=None, epilogue=EPI_NONE, alpha=1.0, flags=0):
        """Always the tensor-core kernel (any m), regardless of the GEMV dispatch threshold."""
        rows, k = x.shape
        if out is None:
            out = torch.empty(rows, w.out_features if epilogue == EPI_GLU else w.n, dtype=torch.float32,
                              device=self.device)
        self.lib.call('pq8_gemm', w.pointer, x.data_ptr(), out.data_ptr(), _ptr(bias), _ptr(resid), rows, w.n, k,
                      epilogue, float(alpha), flags, self.stream())
        return out

    def device_status(self) -> int:
        return self.lib.device_status(self.stream())
