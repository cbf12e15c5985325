"""The host side of the Q8_0 contraction path without PyTorch: CUDA driver API
through ctypes (``cuda_driver.py``) and libpq8.so through ctypes (``pq8.py``).

This is the reference's own host model (``parakeet_cuda/gpu.py:17-49,147-153``):
device memory as non-owning ``Buffer`` views ``(pointer, nbytes, shape)`` into
``Arena`` bump allocators, launches on one stream, errors as ``RuntimeError``.
What changes is the work behind the calls:

* ``HostRuntime.load_weights`` replaces ``GPU.load_weights`` (``gpu.py:169-184``):
  each tensor's GGUF Q8_0 bytes go through one of two page-locked staging
  buffers, an asynchronous copy on a side stream, and ``pq8_pack_q8_0_device``,
  which repacks them in HBM into the resident record layout (no FP32 expansion,
  no per-window re-upload).
* ``HostRuntime.linear`` replaces ``Blas.linear`` (``gpu.py:87-90``) plus the
  epilogue kernels: one ``pq8_linear`` / ``pq8_gemm`` launch per linear.
* ``EncoderStackHost`` runs the encoder's Q8_0 linears over windows stacked
  as rows, captures a step as a CUDA graph with
  ``cuStreamBeginCapture``, and moves each step's input and result between
  page-locked host memory and the device.

Importing this module needs neither PyTorch nor a GPU; ``HostRuntime`` opens
the driver and fails loudly without an sm_100 device or a built libpq8.so.
"""
from __future__ import annotations

from dataclasses import dataclass
import time

import numpy as np

from . import pq8
from .cuda_driver import Driver, Event, PinnedArray
from .layers import D_FF, D_MODEL, FRAMES_PER_WINDOW, LAYER_PLAN, flops_per_row_per_layer
from .pq8 import EPI_GLU, EPI_RESIDUAL, FLAG_X_TF32, LAYOUT_GATES4, LAYOUT_GLU, LAYOUT_ROWS, GEMV_MAX_M

MIB = 1 << 20
ALIGN = 256


class Buffer:
    """Non-owning view of device memory, as the reference's ``Buffer`` (``gpu.py:17-24``)."""

    def __init__(self, pointer: int, nbytes: int, shape=None, dtype=np.float32):
        self.pointer, self.nbytes, self.shape, self.dtype = int(pointer), int(nbytes), shape, np.dtype(dtype)

    def view(self, offset: int, nbytes: int, shape=None, dtype=None) -> 'Buffer':
        if offset < 0 or nbytes < 0 or offset + nbytes > self.nbytes:
            raise ValueError('device view exceeds buffer')
        return Buffer(self.pointer + offset, nbytes, shape, self.dtype if dtype is None else dtype)


class Arena:
    """One device allocation handed out in 256-byte aligned pieces (``gpu.py:27-49``)."""

    def __init__(self, drv: Driver, size: int, name: str = 'arena'):
        self.drv, self.size, self.name = drv, int(size), name
        self.base = drv.alloc(self.size)
        self.offset = self.peak = 0

    def alloc(self, shape, dtype=np.float32) -> Buffer:
        shape = (shape,) if isinstance(shape, int) else tuple(shape)
        nbytes = int(np.prod(shape)) * np.dtype(dtype).itemsize
        offset = (self.offset + ALIGN - 1) // ALIGN * ALIGN
        if offset + nbytes > self.size:
            raise MemoryError(f'{self.name}: {offset + nbytes} bytes exceed the fixed {self.size}-byte arena')
        self.offset = offset + nbytes
        self.peak = max(self.peak, self.offset)
        return Buffer(self.base + offset, nbytes, shape, dtype)

    def reset(self, mark: int = 0) -> None:
        self.offset = mark  # one ordered stream: earlier readers finish before reuse

    def close(self) -> None:
        if self.base:
            self.drv.free(self.base)
            self.base = 0


@dataclass
class PackedQ8:
    """A resident packed Q8_0 tensor (``n`` rows x ``k`` columns in ``layout``)."""
    buf: Buffer
    n: int
    k: int
    layout: int

    @property
    def pointer(self) -> int:
        return self.buf.pointer

    @property
    def out_features(self) -> int:
        return self.n // 2 if self.layout == LAYOUT_GLU else self.n // 4 if self.layout == LAYOUT_GATES4 else self.n


def _ptr(b) -> int | None:
    return None if b is None else b.pointer


class HostRuntime:
    """One device: driver context, compute stream, weight arena, GEMV workspace."""

    def __init__(self, index: int = 0, weight_bytes: int = 1024 * MIB, work_bytes: int = 256 * MIB,
                 workspace_bytes: int = 16 * MIB, lib: pq8.Library | None = None):
        self.drv = Driver(index)
        info = self.drv.info()
        if info['sm'] != 100:
            raise RuntimeError(f'pq8 needs an sm_100 device (B200); device {index} is {info["name"]} sm_{info["sm"]}')
        self.info = info
        self.lib = lib or pq8.library()
        self.stream = self.drv.stream()
        self.weights_arena = Arena(self.drv, weight_bytes, 'weights')
        self.work = Arena(self.drv, work_bytes, 'activations')
        self.workspace = Buffer(self.drv.alloc(workspace_bytes), workspace_bytes, (workspace_bytes,), np.uint8)
        self.lib.call('pq8_workspace_init', self.workspace.pointer, workspace_bytes, self.stream.handle)
        self.weights: dict[str, object] = {}
        self._uploader = None

    # -- memory ---------------------------------------------------------------
    def upload(self, array, arena: Arena | None = None) -> Buffer:
        """A device copy of a host array (synchronous; for parameters and test inputs)."""
        a = np.ascontiguousarray(array)
        buf = (arena or self.work).alloc(a.shape, a.dtype)
        staging = PinnedArray(self.drv, a.shape, a.dtype)
        try:
            staging.array[...] = a
            self.drv.h2d(buf.pointer, staging.pointer, a.nbytes, self.stream)
            self.stream.synchronize()
        finally:
            staging.close()
        return buf

    def download(self, buf: Buffer) -> np.ndarray:
        staging = PinnedArray(self.drv, buf.shape, buf.dtype)
        try:
            self.drv.d2h(staging.pointer, buf.pointer, buf.nbytes, self.stream)
            self.stream.synchronize()
            return staging.array.copy()
        finally:
            staging.close()

    # -- weights (GPU.load_weights counterpart) ----------------------------------
    def uploader(self) -> 'HostWeightUploader':
        if self._uploader is None:
            self._uploader = HostWeightUploader(self)
        return self._uploader

    def load_weights(self, model, names, layouts: dict | None = None) -> dict:
        """Q8_0 tensors become resident packed weights (``layouts[name]`` picks GLU pairing),
        others device copies of their values; all stay resident."""
        layouts = layouts or {}
        up = self.uploader()
        for name in names:
            t = model.tensors[name]
            if t.kind == 8:
                n, k = t.shape[0], int(np.prod(t.shape[1:]))
                self.weights[name] = up.pack_rows([model.raw(name)], n, k, layouts.get(name, LAYOUT_ROWS))
            else:
                self.weights[name] = self.upload(np.asarray(model.array(name), np.float32).reshape(t.shape),
                                                 self.weights_arena)
        up.finish()
        return self.weights

    # -- linears (Blas.linear counterpart) ---------------------------------------
    def gemm(self, x: Buffer, w: PackedQ8, out: Buffer, m: int, bias: Buffer | None = None,
             resid: Buffer | None = None, epilogue: int = pq8.EPI_NONE, alpha: float = 1.0, flags: int = 0) -> None:
        """``out[m, :] = epilogue(x @ W^T + bias)`` on the tensor-core kernel (any m)."""
        self.lib.call('pq8_gemm', w.pointer, x.pointer, out.pointer, _ptr(bias), _ptr(resid), m, w.n, w.k, epilogue,
                      float(alpha), flags, self.stream.handle)

    def linear(self, x: Buffer, w: PackedQ8, out: Buffer, m: int, bias: Buffer | None = None,
               resid: Buffer | None = None, epilogue: int = pq8.EPI_NONE, alpha: float = 1.0, flags: int = 0) -> None:
        """As ``gemm``, with the library choosing the GEMV for a few rows."""
        if 1 <= m <= GEMV_MAX_M and self.lib.gemv_workspace_size(m, w.n, w.k) > self.workspace.nbytes:
            raise MemoryError(f'GEMV workspace of {self.workspace.nbytes} bytes is too small for [{m}, {w.n}, {w.k}]')
        # (a workspace too small for split K only runs the GEMM unsplit)
        self.lib.call('pq8_linear', w.pointer, x.pointer, out.pointer, _ptr(bias), _ptr(resid), m, w.n, w.k, epilogue,
                      float(alpha), flags, self.workspace.pointer, self.workspace.nbytes, self.stream.handle)

    def round_tf32(self, buf: Buffer) -> None:
        self.lib.call('pq8_round_tf32', buf.pointer, buf.nbytes // 4, self.stream.handle)

    def device_status(self) -> int:
        return self.lib.device_status(self.stream.handle)

    def synchronize(self) -> None:
        self.stream.synchronize()

    def close(self) -> None:
        """Free this runtime's device memory (after its work has finished)."""
        self.stream.synchronize()
        if self._uploader is not None:
            self._uploader.close()
            self._uploader = None
        self.weights_arena.close()
        self.work.close()
        if self.workspace.pointer:
            self.drv.free(self.workspace.pointer)
            self.workspace = Buffer(0, 0)
        self.stream.close()


class HostWeightUploader:
    """GGUF Q8_0 bytes -> resident packed weights, repacked on the device.

    The host copies each tensor's bytes into one of two page-locked staging
    buffers while the other one's asynchronous copy and repack run on a side
    stream; ``finish()`` makes the compute stream wait for the side stream."""

    def __init__(self, rt: HostRuntime, slot_bytes: int = 16 * MIB):
        self.rt, self.drv = rt, rt.drv
        self.side = self.drv.stream()
        self.slots = []
        self.turn = 0
        self.bytes_uploaded = 0
        self._grow(slot_bytes)

    def _grow(self, nbytes: int) -> None:
        for s in self.slots:
            s['done'].synchronize()
            s['host'].close()
            self.drv.free(s['dev'])
        self.slots = [{'host': PinnedArray(self.drv, nbytes, np.uint8), 'dev': self.drv.alloc(nbytes),
                       'done': Event(self.drv, timing=False).record(self.side), 'bytes': nbytes} for _ in range(2)]

    def _stage(self, raws) -> tuple[dict, int]:
        arrays = [np.ascontiguousarray(r).reshape(-1).view(np.uint8) for r in raws]
        nbytes = sum(a.size for a in arrays)
        if nbytes > self.slots[0]['bytes']:
            self._grow(max(nbytes, 2 * self.slots[0]['bytes']))
        slot = self.slots[self.turn]
        self.turn ^= 1
        slot['done'].synchronize()  # its previous copy and repack have finished reading it
        off = 0
        for a in arrays:
            slot['host'].array[off:off + a.size] = a
            off += a.size
        self.drv.h2d(slot['dev'], slot['host'].pointer, nbytes, self.side)
        self.bytes_uploaded += nbytes
        return slot, nbytes

    def pack_rows(self, raws, n: int, k: int, layout: int = LAYOUT_ROWS) -> PackedQ8:
        """GGUF Q8_0 sources stacked along N (Q, K and V into one [3n', k] matrix)."""
        lib = self.rt.lib
        out = self.rt.weights_arena.alloc(lib.packed_size(n, k, layout), np.uint8)
        slot, nbytes = self._stage(raws)
        if nbytes != n * k // 32 * 34:
            raise ValueError(f'expected {n * k // 32 * 34} Q8_0 bytes for [{n}, {k}], got {nbytes}')
        lib.call('pq8_pack_q8_0_device', slot['dev'], n, k, layout, out.pointer, self.side.handle)
        slot['done'].record(self.side)
        return PackedQ8(out, n, k, layout)

    def pack(self, parts, n: int, layout: int = LAYOUT_ROWS) -> PackedQ8:
        """``parts = [(raw, k_i), ...]``: Q8_0 ``[n, k_i]`` sources side by side along K
        (an LSTM layer's ``[W_ih | W_hh]``)."""
        lib = self.rt.lib
        k_total = sum(k for _, k in parts)
        out = self.rt.weights_arena.alloc(lib.packed_size(n, k_total, layout), np.uint8)
        off = 0
        for raw, k in parts:
            slot, nbytes = self._stage([raw])
            if nbytes != n * k // 32 * 34:
                raise ValueError(f'expected {n * k // 32 * 34} Q8_0 bytes for [{n}, {k}], got {nbytes}')
            lib.call('pq8_pack_q8_0_part_device', slot['dev'], n, k, k_total, off, layout, out.pointer,
                     self.side.handle)
            slot['done'].record(self.side)
            off += k
        return PackedQ8(out, n, k_total, layout)

    def finish(self) -> None:
        ev = Event(self.drv, timing=False).record(self.side)
        self.rt.stream.wait(ev)
        ev.close()

    def close(self) -> None:
        self.side.synchronize()
        for s in self.slots:
            s['host'].close()
            self.drv.free(s['dev'])
            s['done'].close()
        self.slots = []
        self.side.close()


class EncoderStackHost:
    """All Q8_0 linears of ``layers`` encoder layers over ``rows`` activation rows
    (windows stacked as rows), on driver-API memory.

    The same launches as ``encoder.EncoderStack``: LayerNorm, attention and
    positional outputs, which are not on the contraction path, are fixed
    stand-in buffers (``norm``, ``ctx``, ``pos``), produced TF32-rounded as a
    fused producer would write them; ``standins`` supplies their values (else
    seeded N(0, 1))."""

    def __init__(self, model, rt: HostRuntime, rows: int, layers: int = 24, seed: int = 0, standins=None):
        self.rt, self.rows, self.layers = rt, rows, layers
        drv = rt.drv
        t0 = time.perf_counter()
        up = rt.uploader()
        self.weights = []
        for l in range(layers):
            base = f'encoder.layers.{l}.'
            self.weights.append({name: up.pack_rows([model.raw(base + key + '.weight') for key in keys], n, k,
                                                    LAYOUT_GLU if epi == EPI_GLU else LAYOUT_ROWS)
                                 for name, keys, n, k, epi, *_ in LAYER_PLAN})
        up.finish()
        rt.synchronize()
        self.load_seconds = time.perf_counter() - t0
        self.weight_bytes = sum(w.buf.nbytes for layer in self.weights for w in layer.values())
        widths = {'norm': D_MODEL, 'ctx': D_MODEL, 'pos': D_MODEL, 'resid': D_MODEL, 'hidden': D_FF,
                  'qkv': 3 * D_MODEL, 'pos_out': D_MODEL, 'gate': D_MODEL}
        self.buffers = {name: rt.work.alloc((rows, w)) for name, w in widths.items()}
        rng = np.random.default_rng(seed)
        for name in ('norm', 'ctx', 'pos'):
            v = standins[name] if standins is not None else rng.standard_normal((rows, D_MODEL), np.float32)
            self._fill(self.buffers[name], np.asarray(v, np.float32))
            rt.round_tf32(self.buffers[name])
        drv.memset(self.buffers['resid'].pointer, 0, self.buffers['resid'].nbytes, rt.stream)
        rt.synchronize()
        self._pipe = None

    def _fill(self, buf: Buffer, values: np.ndarray) -> None:
        staging = PinnedArray(self.rt.drv, values.shape, np.float32)
        staging.array[...] = values
        self.rt.drv.h2d(buf.pointer, staging.pointer, buf.nbytes, self.rt.stream)
        self.rt.synchronize()
        staging.close()

    @property
    def launches_per_step(self) -> int:
        return self.layers * len(LAYER_PLAN)

    def flops_per_step(self) -> int:
        return self.rows * self.layers * flops_per_row_per_layer()

    def launch(self, layer: int, entry) -> None:
        name, _, n, k, epi, alpha, src, dst, flags = entry
        b = self.buffers
        self.rt.gemm(b[src], self.weights[layer][name], b[dst], self.rows,
                     resid=b['resid'] if epi == EPI_RESIDUAL else None, epilogue=epi, alpha=alpha,
                     flags=flags | FLAG_X_TF32)

    def step(self) -> None:
        """Enqueue every linear of every layer on the runtime's stream."""
        for l in range(self.layers):
            for entry in LAYER_PLAN:
                self.launch(l, entry)

    # Order of a layer's linears in a sequence plan: the layer's order with
    # linear_pos, which depends on nothing in the layer, ahead of QKV, so that
    # its tiles are there to take while QKV waits for the rows of the FFN1
    # residual (the plan's schedule hands tiles out in plan order).
    SEQUENCE_ORDER = ('ffn1_up', 'ffn1_down', 'pos', 'qkv', 'out', 'pw1_glu', 'pw2', 'ffn2_up', 'ffn2_down')

    def sequence_tasks(self, dependencies: str = 'model', window: int = FRAMES_PER_WINDOW, order=None) -> list:
        """Every linear of every layer as ``pq8_gemm_task``s, in plan order
        (``order``: names of a layer's linears, default ``SEQUENCE_ORDER``).

        Dependencies the buffers show (the FFN hidden state, the GLU output, the
        residual stream, and every rewrite of a buffer) are found by the library.
        ``dependencies='model'`` adds the ones the stand-in buffers hide, as a
        whole block would have them: each LayerNorm reads the residual stream as
        the previous residual linear left it (FFN1 up, QKV, pointwise 1, FFN2 up
        wait for those rows), and linear_out reads the attention of each window
        of ``window`` frames (it waits for QKV on all rows of the windows its
        rows belong to); the positional projection waits for nothing.
        ``'buffers'`` keeps only the buffer dependencies."""
        if dependencies not in ('model', 'buffers'):
            raise ValueError(dependencies)
        b = self.buffers
        plan = {entry[0]: entry for entry in LAYER_PLAN}
        names = self.SEQUENCE_ORDER if order is None else tuple(order)
        if sorted(names) != sorted(plan):
            raise ValueError(f'order must name each of {sorted(plan)} once')
        tasks, index = [], {}
        last_residual = -1
        for l in range(self.layers):
            for name, _, n, k, epi, alpha, src, dst, flags in (plan[nm] for nm in names):
                after, after_window = -1, 0
                if dependencies == 'model':
                    if name in ('ffn1_up', 'qkv', 'pw1_glu', 'ffn2_up'):
                        after = last_residual
                    elif name == 'out':
                        after, after_window = index[l, 'qkv'], window
                w = self.weights[l][name]
                resid = b['resid'].pointer if epi == EPI_RESIDUAL else None
                tasks.append(pq8.GemmTask(w.pointer, b[src].pointer, b[dst].pointer, None, resid, self.rows, n, k,
                                          epi, alpha, flags | FLAG_X_TF32, after, after_window))
                index[l, name] = len(tasks) - 1
                if epi == EPI_RESIDUAL:
                    last_residual = len(tasks) - 1
        return tasks

    def make_sequence(self, dependencies: str = 'model', order=None) -> Buffer:
        """Plan every linear of a step as one persistent launch (``pq8_sequence_plan``);
        ``step_sequence`` runs it."""
        tasks = self.sequence_tasks(dependencies, order=order)
        nbytes = self.rt.lib.sequence_plan_size(tasks)
        if getattr(self, '_plan', None) is None or self._plan.nbytes < nbytes:
            self._plan = Buffer(self.rt.drv.alloc(nbytes), nbytes, (nbytes,), np.uint8)
        self.rt.lib.sequence_plan(tasks, self._plan.pointer, self._plan.nbytes, self.rt.stream.handle)
        return self._plan

    def step_sequence(self) -> None:
        """One step as a single persistent launch of the plan made by ``make_sequence``."""
        self.rt.lib.call('pq8_sequence_run', self._plan.pointer, self.rt.stream.handle)

    def capture(self, sequence: bool = False):
        """One step as a CUDA graph (``cuStreamBeginCapture``): the per-linear launches of
        ``step``, or the single launch of ``step_sequence``. Run the step once first so
        that per-device library state is set up outside the capture."""
        return self.rt.stream.capture(self.step_sequence if sequence else self.step)

    def _enqueue(self, graph) -> None:
        if graph is not None:
            graph.launch(self.rt.stream)
        else:
            self.step()

    def run_host(self, x_host: PinnedArray, out_host: PinnedArray, graph=None) -> None:
        """Public end-to-end call on page-locked host arrays ``[rows, 1024]``: the input
        starts the residual stream and stands in for every LayerNorm output; the final
        residual stream is copied back. Enqueued on the runtime's stream; the caller
        synchronizes."""
        drv, st, b = self.rt.drv, self.rt.stream, self.buffers
        nbytes = b['resid'].nbytes
        drv.h2d(b['norm'].pointer, x_host.pointer, nbytes, st)
        drv.d2d(b['resid'].pointer, b['norm'].pointer, nbytes, st)
        self.rt.round_tf32(b['norm'])
        self._enqueue(graph)
        drv.d2h(out_host.pointer, b['resid'].pointer, nbytes, st)

    def run_host_pipelined(self, inputs, outputs, graph=None) -> None:
        """One step per (``inputs[i]``, ``outputs[i]``) pair as ``run_host`` does, with
        step i+1's host-to-device copy and step i-1's device-to-host copy on two copy
        streams while step i computes (two device staging buffers per direction). The
        runtime's stream waits for the last copy; the caller synchronizes."""
        if len(inputs) != len(outputs):
            raise ValueError('inputs and outputs must pair up')
        drv, compute, b = self.rt.drv, self.rt.stream, self.buffers
        nbytes = b['resid'].nbytes
        if self._pipe is None:
            self._pipe = {'h2d': drv.stream(), 'd2h': drv.stream(),
                          'in': [drv.alloc(nbytes) for _ in range(2)], 'out': [drv.alloc(nbytes) for _ in range(2)],
                          'ev': {k: [Event(drv, timing=False) for _ in range(2)]
                                 for k in ('in_ready', 'in_free', 'out_ready', 'out_free')}}
        p = self._pipe
        h2d, d2h, ev = p['h2d'], p['d2h'], p['ev']
        start = Event(drv, timing=False).record(compute)
        h2d.wait(start)
        d2h.wait(start)
        used = [False, False]
        for i, (x_host, out_host) in enumerate(zip(inputs, outputs)):
            s = i & 1
            if used[s]:
                h2d.wait(ev['in_free'][s])      # step i-2 has taken its input out of this buffer
            drv.h2d(p['in'][s], x_host.pointer, nbytes, h2d)
            ev['in_ready'][s].record(h2d)
            compute.wait(ev['in_ready'][s])
            drv.d2d(b['norm'].pointer, p['in'][s], nbytes, compute)
            drv.d2d(b['resid'].pointer, p['in'][s], nbytes, compute)
            ev['in_free'][s].record(compute)
            self.rt.round_tf32(b['norm'])
            self._enqueue(graph)
            if used[s]:
                compute.wait(ev['out_free'][s])  # step i-2's result has left this buffer
            drv.d2d(p['out'][s], b['resid'].pointer, nbytes, compute)
            ev['out_ready'][s].record(compute)
            d2h.wait(ev['out_ready'][s])
            drv.d2h(out_host.pointer, p['out'][s], nbytes, d2h)
            ev['out_free'][s].record(d2h)
            used[s] = True
        done_h2d = Event(drv, timing=False).record(h2d)
        done_d2h = Event(drv, timing=False).record(d2h)
        compute.wait(done_h2d)
        compute.wait(done_d2h)
        for e in (start, done_h2d, done_d2h):
            e.close()

    def close(self) -> None:
        if getattr(self, '_plan', None) is not None:
            self.rt.drv.free(self._plan.pointer)
            self._plan = None
        if self._pipe is not None:
            for ptr in self._pipe['in'] + self._pipe['out']:
                self.rt.drv.free(ptr)
            self._pipe = None
