"""Model-level Python front end over libiq's C ABI.

Mirrors the reference's ``QuantizedModel`` / ``QuantizedModelState`` surface
(src/qwen/quantized_model.rs): ``forward`` (forward_detailed), ``verify``
(verify_rows + accepted_draft_prefix + rollback, done on the device) and
``rollback``.  Tensors are GGUF blocks handed over as host or device buffers.
"""
from __future__ import annotations

import ctypes
from typing import Iterable

import numpy as np
import torch

from . import _lib
from .synth import Config, IqConfigFields, Tensor
import dataclasses


class IqConfig(ctypes.Structure):
    _fields_ = [(f.name, ctypes.c_float if f.name == "rms_norm_eps" else
                 ctypes.c_double if f.name == "rope_theta" else ctypes.c_int32)
                for f in dataclasses.fields(IqConfigFields)]


class IqTensorView(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("ndim", ctypes.c_int32),
                ("shape", ctypes.c_int64 * 4), ("data", ctypes.c_void_p), ("location", ctypes.c_int32)]


class IqVerifyResult(ctypes.Structure):
    _fields_ = [("accepted", ctypes.c_int32), ("authoritative", ctypes.c_int32), ("committed", ctypes.c_int32)]


P = ctypes.c_void_p


def _declare(L):
    sig = {
        "iq_model_create": (ctypes.c_int, [P, ctypes.c_int, P, ctypes.POINTER(P)]),
        "iq_model_create_ep": (ctypes.c_int, [P, ctypes.c_int, P, ctypes.c_int, ctypes.c_int, P, ctypes.POINTER(P)]),
        "iq_model_destroy": (None, [P]),
        "iq_model_weight_bytes": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64)]),
        "iq_state_create": (ctypes.c_int, [P, ctypes.c_int64, ctypes.POINTER(P)]),
        "iq_state_destroy": (None, [P]),
        "iq_state_reset": (ctypes.c_int, [P]),
        "iq_state_position": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64)]),
        "iq_state_stream": (ctypes.c_int, [P, ctypes.POINTER(P)]),
        "iq_forward": (ctypes.c_int, [P, P, ctypes.c_int, P, P, P]),
        "iq_verify": (ctypes.c_int, [P, P, ctypes.c_int, ctypes.POINTER(IqVerifyResult), P, P]),
        "iq_rollback": (ctypes.c_int, [P, ctypes.c_int]),
        "iq_state_union_sizes": (ctypes.c_int, [P, P]),
        "iq_state_launch_count": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64)]),
        "iq_state_routes": (ctypes.c_int, [P, ctypes.c_int, P]),
        "iq_state_set_profiling": (ctypes.c_int, [P, ctypes.c_int]),
        "iq_state_profile": (ctypes.c_int, [P, ctypes.c_char_p, ctypes.c_int]),
        "iq_mtp_sync": (ctypes.c_int, [P, ctypes.c_int64, P, P, ctypes.c_int, P]),
        "iq_mtp_draft": (ctypes.c_int, [P, ctypes.c_uint32, P, ctypes.c_int, ctypes.c_int, ctypes.c_float, P, P, P,
                                        ctypes.POINTER(ctypes.c_int)]),
        "iq_mtp_position": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64)]),
        "iq_state_image_size": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_int64)]),
        "iq_state_export": (ctypes.c_int, [P, P, ctypes.c_int64]),
        "iq_state_import": (ctypes.c_int, [P, P, ctypes.c_int64]),
    }
    for n, (r, a) in sig.items():
        f = getattr(L, n)
        f.restype = r
        f.argtypes = a


def lib():
    L = _lib.lib()
    if not getattr(L, "_model_declared", False):
        _declare(L)
        L._model_declared = True
    return L


def iq_config(cfg: Config) -> IqConfig:
    return IqConfig(**cfg.abi_fields())


class Model:
    """A checkpoint resident on the current CUDA device."""

    def __init__(self, cfg: Config, tensors: Iterable[Tensor], *, ep_rank: int = 0, ep_world: int = 1,
                 nccl_id: bytes | None = None):
        """`ep_world` > 1: expert-parallel rank `ep_rank`; every rank passes the
        same 128-byte `nccl_id` (inferq_b200.ep.shared_unique_id)."""
        self.cfg = cfg
        keep, views = [], []
        names = []
        for t in tensors:
            data = t.data.contiguous()
            keep.append(data)
            nm = t.name.encode()
            names.append(nm)
            v = IqTensorView()
            v.name = nm
            v.dtype = t.dtype
            v.ndim = len(t.shape)
            for i, s in enumerate(t.shape):
                v.shape[i] = s
            v.data = data.data_ptr()
            v.location = 1 if data.is_cuda else 0
            views.append(v)
        arr = (IqTensorView * len(views))(*views)
        c = iq_config(cfg)
        h = P()
        L = lib()
        if ep_world == 1:
            _lib.check(L.iq_model_create(arr, len(views), ctypes.byref(c), ctypes.byref(h)))
        else:
            if nccl_id is None or len(nccl_id) != 128:
                raise ValueError("expert parallelism needs the ranks' shared 128-byte NCCL unique id")
            idbuf = ctypes.create_string_buffer(nccl_id, 128)
            _lib.check(L.iq_model_create_ep(arr, len(views), ctypes.byref(c), ep_rank, ep_world, idbuf,
                                            ctypes.byref(h)))
        self._h = h
        del keep, arr

    def weight_bytes(self) -> int:
        b = ctypes.c_int64()
        _lib.check(lib().iq_model_weight_bytes(self._h, ctypes.byref(b)))
        return b.value

    def __del__(self):
        if getattr(self, "_h", None) is not None and _lib._lib is not None:
            torch.cuda.synchronize()
            _lib._lib.iq_model_destroy(self._h)
            self._h = None


class State:
    """Decode state (KV cache + DeltaNet state) of one sequence."""

    def __init__(self, model: Model, max_positions: int):
        self.model = model
        h = P()
        _lib.check(lib().iq_state_create(model._h, max_positions, ctypes.byref(h)))
        self._h = h

    @property
    def position(self) -> int:
        v = ctypes.c_int64()
        _lib.check(lib().iq_state_position(self._h, ctypes.byref(v)))
        return v.value

    def reset(self):
        _lib.check(lib().iq_state_reset(self._h))

    def forward(self, tokens, *, logits=False, hidden=False):
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        n = len(tok)
        V, H = self.model.cfg.vocab_size, self.model.cfg.hidden_size
        lg = np.empty((n, V), np.float32) if logits else None
        hd = np.empty((n, H), np.float32) if hidden else None
        am = np.empty(n, np.int32)
        _lib.check(lib().iq_forward(self._h, tok.ctypes.data, n, _lib.ptr(lg), _lib.ptr(hd), am.ctypes.data))
        return am, lg, hd

    def verify(self, tokens, *, logits=False, hidden=False):
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        n = len(tok)
        V, H = self.model.cfg.vocab_size, self.model.cfg.hidden_size
        lg = np.empty((n, V), np.float32) if logits else None
        hd = np.empty((n, H), np.float32) if hidden else None
        r = IqVerifyResult()
        _lib.check(lib().iq_verify(self._h, tok.ctypes.data, n, ctypes.byref(r), _lib.ptr(lg), _lib.ptr(hd)))
        return (r.accepted, r.authoritative, r.committed), lg, hd

    def rollback(self, committed_rows: int):
        _lib.check(lib().iq_rollback(self._h, committed_rows))

    # ---------------------------------------------------------- images
    def export_image(self) -> np.ndarray:
        """The state as a host image (iq_state_export); see inferq_b200.image."""
        n = ctypes.c_int64()
        _lib.check(lib().iq_state_image_size(self._h, ctypes.byref(n)))
        buf = np.empty(n.value, np.uint8)
        _lib.check(lib().iq_state_export(self._h, buf.ctypes.data, n.value))
        return buf

    def import_image(self, buf) -> None:
        b = np.ascontiguousarray(np.frombuffer(bytes(buf), np.uint8) if not isinstance(buf, np.ndarray) else buf,
                                 dtype=np.uint8)
        _lib.check(lib().iq_state_import(self._h, b.ctypes.data, b.size))

    # ------------------------------------------------------------ MTP
    @property
    def mtp_position(self) -> int:
        v = ctypes.c_int64()
        _lib.check(lib().iq_mtp_position(self._h, ctypes.byref(v)))
        return v.value

    def mtp_sync(self, position: int, prev_hidden, tokens, target_hidden):
        """Catch the MTP cache up over committed `tokens` (synchronize_mtp)."""
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        th = np.ascontiguousarray(target_hidden, dtype=np.float32)
        ph = None if prev_hidden is None else np.ascontiguousarray(prev_hidden, dtype=np.float32)
        _lib.check(lib().iq_mtp_sync(self._h, position, _lib.ptr(ph), tok.ctypes.data, len(tok), th.ctypes.data))

    def mtp_draft(self, seed: int, hidden, depth: int, draft_vocab: int, min_conf: float = 0.0):
        """`depth` MTP draft steps; returns (tokens, probs, margins, n_confident)."""
        h = np.ascontiguousarray(hidden, dtype=np.float32)
        tok = np.empty(depth, np.uint32)
        pr = np.empty(depth, np.float32)
        mg = np.empty(depth, np.float32)
        n = ctypes.c_int()
        _lib.check(lib().iq_mtp_draft(self._h, seed, h.ctypes.data, depth, draft_vocab, min_conf, tok.ctypes.data,
                                      pr.ctypes.data, mg.ctypes.data, ctypes.byref(n)))
        return tok, pr, mg, n.value

    def union_sizes(self) -> np.ndarray:
        out = np.zeros(self.model.cfg.num_hidden_layers, np.int32)
        _lib.check(lib().iq_state_union_sizes(self._h, out.ctypes.data))
        return out

    def launch_count(self) -> int:
        v = ctypes.c_int64()
        _lib.check(lib().iq_state_launch_count(self._h, ctypes.byref(v)))
        return v.value

    def stream(self) -> int:
        v = P()
        _lib.check(lib().iq_state_stream(self._h, ctypes.byref(v)))
        return v.value or 0

    def routes(self, rows: int) -> np.ndarray:
        c = self.model.cfg
        out = np.zeros((c.num_hidden_layers, rows, c.num_experts_per_tok), np.int32)
        _lib.check(lib().iq_state_routes(self._h, rows, out.ctypes.data))
        return out

    def set_profiling(self, on: bool):
        _lib.check(lib().iq_state_set_profiling(self._h, int(on)))

    def profile(self) -> dict:
        buf = ctypes.create_string_buffer(1 << 16)
        _lib.check(lib().iq_state_profile(self._h, buf, len(buf)))
        out = {}
        for line in buf.value.decode().splitlines():
            name, cnt, us = line.split()
            out[name] = (int(cnt), float(us))
        return out

    def __del__(self):
        if getattr(self, "_h", None) is not None and _lib._lib is not None:
            _lib._lib.iq_state_destroy(self._h)
            self._h = None
