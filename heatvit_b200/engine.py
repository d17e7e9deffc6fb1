"""Device-resident model (the hv_model of the C ABI) with torch-managed buffers.

``Engine`` packs a parameter set onto one GPU once and runs batched integer
inference through ``hv_infer_batch`` (the fused CUDA pipeline).  Buffers are
torch CUDA tensors; the launches go on the caller's current torch stream.
"""

import ctypes as C
import weakref

import numpy as np

from . import abi
from ._lib import check, lib
from .params import (
    HeatViTParams, PackedParams, _Keep, block_from, from_reference, pack_block, pack_selector, selector_from,
)


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("heatvit_b200 needs a CUDA device (there is no CPU fallback)")
    return torch


def _ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _stream(torch):
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


class _Handle:
    """Owns an hv_model handle; destroyed with the Python object."""

    def __init__(self, struct, device, keep):
        self.device = device
        h = C.c_void_p()
        check(lib().hv_model_create(C.addressof(struct), device, C.byref(h)))
        self.h = h
        self._keep = keep
        self._fin = weakref.finalize(self, lib().hv_model_destroy, h)

    def close(self):
        self._fin()


class Engine:
    """A parameter set packed on one GPU.

    ``infer(images)`` takes a CUDA int8 tensor [B, 150528] (or [B, 224, 224, 3],
    NHWC) and returns CUDA tensors: logits [B, 1000] int32 at 2^-14, token
    counts [B, S+1], selector summaries [B, S, 6], warnings [B] uint8; with
    ``checkpoints=True`` also the golden checkpoints [B, 26, 197, 192] and their
    row counts [B, 26] (slot layout of include/heatvit_b200.h)."""

    def __init__(self, params, device=None):
        torch = _torch()
        self.params = from_reference(params)
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                           torch.device(device).index or 0)
        self.device = dev
        self.packed = PackedParams(self.params)
        with torch.cuda.device(dev):
            self._h = _Handle(self.packed.struct, dev.index, self.packed)
        self.num_selectors = self.packed.used_selectors
        self._inflight = []  # arrays of submitted host calls, oldest first

    @property
    def handle(self):
        return self._h.h

    def close(self):
        self._h.close()

    def _images(self, images):
        torch = _torch()
        if images.dtype != torch.int8:
            raise TypeError("images must be int8")
        if images.device != self.device:
            raise ValueError(f"images must live on {self.device}")
        images = images.reshape(images.shape[0], -1)
        if images.shape[1] != abi.IMAGE_BYTES:
            raise ValueError("each image must hold 224*224*3 int8 values")
        return images.contiguous()

    def alloc_outputs(self, batch):
        """Output buffers for ``infer(..., out=...)``: logits, token counts and
        warnings are views of ONE contiguous int32 buffer (``packed``), so a
        single collective can move all three; the summaries sit beside it."""
        torch = _torch()
        b, ns = batch, self.num_selectors
        n_lg, n_tc, n_w = b * abi.CLASSES, b * (ns + 1), (b + 3) // 4
        packed = torch.zeros(n_lg + n_tc + n_w, dtype=torch.int32, device=self.device)
        return dict(packed=packed,
                    logits=packed[:n_lg].view(b, abi.CLASSES),
                    token_counts=packed[n_lg:n_lg + n_tc].view(b, ns + 1),
                    warnings=packed[n_lg + n_tc:].view(torch.uint8)[:b],
                    summary=torch.zeros((b, max(ns, 1), 6), dtype=torch.int32, device=self.device))

    @staticmethod
    def unpack_outputs(packed, batch, num_selectors):
        """Split one rank's ``packed`` buffer of ``alloc_outputs``, as a host
        numpy int32 array, into logits [batch, 1000], token counts [batch, S+1]
        and warnings [batch] uint8."""
        b, ns = batch, num_selectors
        n_lg, n_tc = b * abi.CLASSES, b * (ns + 1)
        packed = np.ascontiguousarray(packed, dtype=np.int32)
        warn = packed[n_lg + n_tc:n_lg + n_tc + (b + 3) // 4].view(np.uint8)[:b]
        return packed[:n_lg].reshape(b, abi.CLASSES), packed[n_lg:n_lg + n_tc].reshape(b, ns + 1), warn

    def infer(self, images, checkpoints=False, out=None):
        torch = _torch()
        images = self._images(images)
        b = images.shape[0]
        ns = self.num_selectors
        dev = self.device
        if out is not None:
            if out["logits"].shape[0] != b or out["token_counts"].shape[1] != ns + 1:
                raise ValueError("output buffers were allocated for another batch or model")
            logits, counts, summary, warnings = out["logits"], out["token_counts"], out["summary"], out["warnings"]
        else:
            logits = torch.empty((b, abi.CLASSES), dtype=torch.int32, device=dev)
            counts = torch.empty((b, ns + 1), dtype=torch.int32, device=dev)
            summary = torch.zeros((b, max(ns, 1), 6), dtype=torch.int32, device=dev)
            warnings = torch.empty(b, dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            st = _stream(torch)
            if checkpoints:
                ck = torch.zeros((b, abi.CKPT_SLOTS, abi.TOKENS, abi.EMBED), dtype=torch.int8, device=dev)
                rows = torch.zeros((b, abi.CKPT_SLOTS), dtype=torch.int32, device=dev)
                check(lib().hv_infer_batch_checkpoints(self.handle, _ptr(images), b, _ptr(logits), _ptr(counts),
                                                       _ptr(summary), _ptr(warnings), _ptr(ck), _ptr(rows), st))
            else:
                ck = rows = None
                check(lib().hv_infer_batch(self.handle, _ptr(images), b, _ptr(logits), _ptr(counts),
                                           _ptr(summary), _ptr(warnings), st))
        out = dict(logits=logits, token_counts=counts, summary=summary[:, :ns], warnings=warnings)
        if checkpoints:
            out.update(checkpoints=ck, checkpoint_rows=rows)
        return out

    def device_error(self):
        """Read and clear the device error word (0 = every bounded wait completed)."""
        torch = _torch()
        code = C.c_int()
        with torch.cuda.device(self.device):
            check(lib().hv_device_error(self.handle, C.byref(code)))
        return code.value

    def infer_host(self, images, logits=None, token_counts=None, summary=None, warnings=None):
        """Host-buffer entry: numpy int8 [B, 150528] in, numpy logits out.
        Copies overlap compute chunk by chunk inside the library (pinned input
        memory makes the copies asynchronous)."""
        images = np.ascontiguousarray(images).reshape(-1, abi.IMAGE_BYTES)
        if images.dtype != np.int8:
            raise TypeError("images must be int8")
        b = images.shape[0]
        ns = self.num_selectors
        if logits is None:
            logits = np.empty((b, abi.CLASSES), np.int32)
        pl = lambda a: None if a is None else a.ctypes.data_as(C.c_void_p)
        torch = _torch()
        with torch.cuda.device(self.device):
            check(lib().hv_infer_host(self.handle, pl(images), b, pl(logits), pl(token_counts), pl(summary),
                                      pl(warnings)))
        return logits

    def infer_host_submit(self, images, logits, token_counts=None, summary=None, warnings=None):
        """Asynchronous host entry (serving loops): enqueue one call and return;
        ``infer_host_wait()`` finishes the oldest call and returns its logits.
        The arrays stay referenced (and must stay untouched) until then."""
        images = np.ascontiguousarray(images).reshape(-1, abi.IMAGE_BYTES)
        if images.dtype != np.int8:
            raise TypeError("images must be int8")
        if logits.dtype != np.int32 or logits.shape != (images.shape[0], abi.CLASSES) or \
                not logits.flags.c_contiguous:
            raise ValueError("logits must be a contiguous int32 [B, 1000] array")
        if len(self._inflight) == 2:
            self.infer_host_wait()  # the library would wait for the oldest call itself
        pl = lambda a: None if a is None else a.ctypes.data_as(C.c_void_p)
        torch = _torch()
        with torch.cuda.device(self.device):
            check(lib().hv_infer_host_submit(self.handle, pl(images), images.shape[0], pl(logits),
                                             pl(token_counts), pl(summary), pl(warnings)))
        self._inflight.append((images, logits, token_counts, summary, warnings))

    def infer_host_wait(self):
        torch = _torch()
        done = self._inflight.pop(0) if self._inflight else None
        with torch.cuda.device(self.device):
            check(lib().hv_infer_host_wait(self.handle))
        return None if done is None else done[1]

    def transformer_block(self, block_index, x, offsets):
        """Fused block over a ragged batch: x [T, 192] int8, offsets [B+1] int32 (CUDA)."""
        torch = _torch()
        images = offsets.numel() - 1
        z = torch.empty_like(x)
        with torch.cuda.device(self.device):
            check(lib().hv_transformer_block(self.handle, block_index, _ptr(x), _ptr(offsets), images, x.shape[0],
                                             _ptr(z), _stream(torch)))
        return z


class _PartialModel:
    """An hv_model holding only some parts (one block, or selectors), used by
    the per-component golden entry points."""

    def __init__(self, device, blocks=None, selectors=None):
        keep = _Keep()
        s = abi.HvParams()
        for i in range(abi.BLOCKS):
            s.selector_before[i] = -1
        if blocks:
            for i, b in blocks.items():
                pack_block(b, keep, s.blocks[i])
        if selectors:
            for i, sp in enumerate(selectors):
                pack_selector(sp, keep, s.selectors[i])
            s.num_selectors = len(selectors)
        self._h = _Handle(s, device, keep)

    @property
    def handle(self):
        return self._h.h


_CACHE = {}


def _cached(kind, obj, device, factory):
    key = (kind, id(obj), device)
    hit = _CACHE.get(key)
    if hit is not None and hit[0]() is obj:
        return hit[1]
    val = factory()
    try:
        ref = weakref.ref(obj)
    except TypeError:
        ref = (lambda o: (lambda: o))(obj)
    if len(_CACHE) > 64:
        _CACHE.clear()
    _CACHE[key] = (ref, val)
    return val


def engine_for(params):
    torch = _torch()
    dev = torch.cuda.current_device()
    return _cached("engine", params, dev, lambda: Engine(params, dev))


def block_model_for(block_params):
    torch = _torch()
    dev = torch.cuda.current_device()
    return _cached("block", block_params, dev, lambda: _PartialModel(dev, blocks={0: block_from(block_params)}))


def selector_model_for(selector_params):
    torch = _torch()
    dev = torch.cuda.current_device()
    return _cached("selector", selector_params, dev,
                   lambda: _PartialModel(dev, selectors=[selector_from(selector_params)]))
