"""ctypes front end of the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker.  The product never imports it.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
_lib = None

P, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        _lib.or_row_bytes.restype = I64
        _lib.or_row_bytes.argtypes = [I32, I64]
        _lib.or_dequant_rows.argtypes = [I32, P, I64, I64, P]
        _lib.or_quant_q8k.argtypes = [P, I64, P]
        _lib.or_quant_q80.argtypes = [P, I64, P]
        _lib.or_qmatvec.argtypes = [I32, P, I64, I64, P, I32, P, I32, I32]
        _lib.or_argmax.restype = I64
        _lib.or_argmax.argtypes = [P, I64]
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def dequant(dtype: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    out = np.empty((rows, cols), np.float32)
    w = np.ascontiguousarray(w)
    assert lib().or_dequant_rows(dtype, _p(w), rows, cols, _p(out)) == 0
    return out


def quant_q8k(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(len(x) // 256 * 292, np.uint8)
    lib().or_quant_q8k(_p(x), len(x), _p(out))
    return out


def quant_q80(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32).ravel()
    out = np.zeros(len(x) // 32 * 34, np.uint8)
    lib().or_quant_q80(_p(x), len(x), _p(out))
    return out


def qmatvec(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, *, order: int = 0,
            ksplit: int = 1) -> np.ndarray:
    """y[i, r]; order 0 = reference AVX2 lane order, 1 = device chunk order."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
    y = np.empty((x.shape[0], rows), np.float32)
    w = np.ascontiguousarray(w)
    rc = lib().or_qmatvec(dtype, _p(w), rows, cols, _p(x), x.shape[0], _p(y), order, ksplit)
    assert rc == 0, rc
    return y


def set_gemv_order(order: int) -> None:
    """0: reference lane order (default); 1: device chunk order (diagnostic)."""
    lib().or_set_gemv_order(order)


def force_scalar(on: bool) -> None:
    """Use the scalar restatement of the reference order even where the
    AVX2 form (bitwise the same) is available."""
    lib().or_force_scalar(int(on))


def have_avx2() -> bool:
    return bool(lib().or_have_avx2())


def set_perturb(mode: int) -> None:
    """Diagnostic: 1 or 2 moves every RMSNorm output by one ulp (two
    opposite patterns), 0 turns it off: the conditioning of the reference
    arithmetic itself under rounding-level changes."""
    lib().or_set_perturb(int(mode))


def argmax(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(lib().or_argmax(_p(v), len(v)))


# ------------------------------------------------------- layer primitives
def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def conv_step(inp, weights, kernel: int, state):
    """causal_depthwise_conv_step + SiLU; returns (output, new state)."""
    inp, w, st = _f32(inp), _f32(weights), _f32(state).copy()
    out = np.empty_like(inp)
    lib().or_conv_step.argtypes = [P, P, I32, I32, P, P]
    lib().or_conv_step(_p(inp), _p(w), len(inp), kernel, _p(st), _p(out))
    return out, st


def l2_normalize(a):
    a = _f32(a).copy()
    lib().or_l2_normalize.argtypes = [P, I32]
    lib().or_l2_normalize(_p(a), len(a))
    return a


def softplus(v: float) -> float:
    L = lib()
    L.or_softplus.restype = ctypes.c_float
    L.or_softplus.argtypes = [ctypes.c_float]
    return float(L.or_softplus(v))


def delta_step(q, k, v, g, beta, heads: int, key_dim: int, value_dim: int, state):
    """recurrent_delta_step; returns (out, new state)."""
    q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
    st = _f32(state).copy()
    out = np.empty(heads * value_dim, np.float32)
    lib().or_delta_step.argtypes = [P, P, P, P, P, I32, I32, I32, P, P]
    lib().or_delta_step(_p(q), _p(k), _p(v), _p(g), _p(beta), heads, key_dim, value_dim, _p(st), _p(out))
    return out, st


def delta_chunk(q, k, v, beta, log_decay, state):
    """The wide pass's chunked recurrence over C <= 32 rows of one value head
    (the device's order): q, k [C][dk], v [C][dv], beta and log-decay [C],
    state [dk][dv]; returns (outputs [C][dv], new state)."""
    q, k, v, beta, lg = map(_f32, (q, k, v, beta, log_decay))
    C, dk = q.shape
    dv = v.shape[1]
    st = _f32(state).copy()
    out = np.empty((C, dv), np.float32)
    lib().or_delta_chunk.argtypes = [P, P, P, P, P, I32, I32, I32, P, P]
    rc = lib().or_delta_chunk(_p(q), _p(k), _p(v), _p(beta), _p(lg), C, dk, dv, _p(st), _p(out))
    if rc:
        raise ValueError(f"or_delta_chunk: unsupported shape ({C}, {dk}, {dv})")
    return out, st


def route(logits, topk: int, norm_topk: bool = True):
    """top_k_routes for one row: (experts, weights)."""
    lg = _f32(logits)
    rank = np.empty(len(lg), np.int32)
    w = np.empty(topk, np.float32)
    lib().or_route.argtypes = [P, I32, I32, I32, P, P]
    lib().or_route(_p(lg), len(lg), topk, int(norm_topk), _p(rank), _p(w))
    return rank[:topk].copy(), w


def rms_norm(x, w, eps: float):
    """gguf_rms_norm of one row (w already 1 + gamma)."""
    L = lib()
    L.or_rms_norm.argtypes = [P, P, I32, ctypes.c_float, P]
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    L.or_rms_norm(_p(x), _p(w), len(x), eps, _p(out))
    return out


def converted_norm(v, w, eps: float):
    L = lib()
    L.or_converted_norm.argtypes = [P, P, I32, ctypes.c_float]
    v, w = _f32(v).copy(), _f32(w)
    L.or_converted_norm(_p(v), _p(w), len(v), eps)
    return v


def dot8(a, b) -> float:
    L = lib()
    L.or_dot8.restype = ctypes.c_float
    L.or_dot8.argtypes = [P, P, I32]
    a, b = _f32(a), _f32(b)
    return float(L.or_dot8(_p(a) if a.size else None, _p(b) if b.size else None, len(a)))


def attend(q, gate, keys, values, nh: int, nkv: int, hd: int):
    """The per-head scan of one query row over keys/values [positions][nkv][hd]."""
    L = lib()
    L.or_attend.argtypes = [P, P, P, P, I32, I32, I32, I64, P]
    q, gate, keys, values = map(_f32, (q, gate, keys, values))
    out = np.empty(nh * hd, np.float32)
    L.or_attend(_p(q), _p(gate), _p(keys), _p(values), nh, nkv, hd, keys.size // (nkv * hd), _p(out))
    return out


def value_head(key: int, repeat: int, key_heads: int, ratio: int, tiled: bool) -> int:
    L = lib()
    L.or_value_head.argtypes = [I32, I32, I32, I32, I32]
    return int(L.or_value_head(key, repeat, key_heads, ratio, int(tiled)))


def accepted_prefix(drafts, logits) -> int:
    L = lib()
    L.or_accepted_prefix.argtypes = [P, I32, P, I64]
    d = np.ascontiguousarray(drafts, np.uint32)
    lg = _f32(logits)
    return int(L.or_accepted_prefix(_p(d) if d.size else None, len(d), _p(lg), lg.shape[-1]))


# ------------------------------------------------------------------ model
class OracleModel:
    """The CPU restatement of the reference model over host tensors.

    ``tensors`` are inferq_b200.synth.Tensor objects (CPU); the config is a
    synth.Config.  Rows are evaluated one at a time in the reference's own
    arithmetic order (see iq_oracle_model.c).
    """

    def __init__(self, cfg, tensors):
        from inferq_b200.model import IqConfig, IqTensorView, iq_config
        L = lib()
        P = ctypes.c_void_p
        L.or_model_create.restype = P
        L.or_model_create.argtypes = [P, P, ctypes.c_int]
        L.or_model_destroy.argtypes = [P]
        L.or_state_create.restype = P
        L.or_state_create.argtypes = [P, ctypes.c_int64]
        L.or_state_destroy.argtypes = [P]
        L.or_state_copy.argtypes = [P, P, P]
        L.or_forward.argtypes = [P, P, P, ctypes.c_int, P, P, P]
        L.or_mtp_forward.argtypes = [P, P, ctypes.c_uint32, P, ctypes.c_int64, P, P]
        L.or_state_set_mtp_position.argtypes = [P, ctypes.c_int64]
        L.or_state_image_size.restype = ctypes.c_int64
        L.or_state_image_size.argtypes = [P, P]
        L.or_state_export.argtypes = [P, P, P, ctypes.c_int64]
        L.or_state_import.argtypes = [P, P, P, ctypes.c_int64]
        self.cfg = cfg
        self._keep = []
        views = []
        for t in tensors:
            d = t.data.detach().cpu().contiguous()
            self._keep.append(d)
            v = IqTensorView()
            nm = t.name.encode()
            self._keep.append(nm)
            v.name = nm
            v.dtype = t.dtype
            v.ndim = len(t.shape)
            for i, s in enumerate(t.shape):
                v.shape[i] = s
            v.data = d.data_ptr()
            v.location = 0
            views.append(v)
        self._views = (IqTensorView * len(views))(*views)
        self._cfg = iq_config(cfg)
        self._h = L.or_model_create(ctypes.byref(self._cfg), self._views, len(views))
        assert self._h, "oracle model creation failed (missing tensor)"

    def state(self, max_pos: int) -> "OracleState":
        return OracleState(self, max_pos)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_model_destroy(self._h)
            self._h = None


class OracleState:
    def __init__(self, model: OracleModel, max_pos: int):
        self.model = model
        self.max_pos = max_pos
        self._h = lib().or_state_create(model._h, max_pos)

    def forward(self, tokens, *, logits=True, hidden=False, experts=False):
        c = self.model.cfg
        tok = np.ascontiguousarray(tokens, dtype=np.uint32)
        n = len(tok)
        lg = np.empty((n, c.vocab_size), np.float32) if logits else None
        hd = np.empty((n, c.hidden_size), np.float32) if hidden else None
        ex = np.empty((n, c.num_hidden_layers, c.num_experts_per_tok), np.int32) if experts else None
        rc = lib().or_forward(self.model._h, self._h, _p(tok), n, None if lg is None else _p(lg),
                              None if hd is None else _p(hd), None if ex is None else _p(ex))
        assert rc == 0, rc
        return lg, hd, ex

    def mtp(self, token: int, hidden_in: np.ndarray, head_rows: int):
        c = self.model.cfg
        h = np.ascontiguousarray(hidden_in, np.float32)
        lg = np.empty(head_rows, np.float32) if head_rows else None
        out = np.empty(c.hidden_size, np.float32)
        rc = lib().or_mtp_forward(self.model._h, self._h, token, _p(h), head_rows,
                                  None if lg is None else _p(lg), _p(out))
        assert rc == 0, rc
        return lg, out

    @property
    def position(self) -> int:
        L = lib()
        L.or_state_position.restype = ctypes.c_int64
        L.or_state_position.argtypes = [ctypes.c_void_p]
        return int(L.or_state_position(self._h))

    def export_image(self) -> np.ndarray:
        """The state in the library's image layout (inferq_b200.image)."""
        n = lib().or_state_image_size(self.model._h, self._h)
        buf = np.empty(n, np.uint8)
        assert lib().or_state_export(self.model._h, self._h, _p(buf), n) == 0
        return buf

    def import_image(self, buf) -> None:
        b = np.ascontiguousarray(buf, np.uint8)
        rc = lib().or_state_import(self.model._h, self._h, _p(b), b.size)
        assert rc == 0, rc

    def enable_snapshots(self, rows: int) -> None:
        """Keep the DeltaNet state after each row of a pass of up to `rows`
        rows, so rollback() is a copy (QuantizedStateSnapshots)."""
        L = lib()
        L.or_state_enable_snapshots.argtypes = [P, P, I32]
        assert L.or_state_enable_snapshots(self.model._h, self._h, rows) == 0

    def rollback(self, committed: int) -> None:
        """Keep the first `committed` rows of the last pass."""
        L = lib()
        L.or_state_rollback.argtypes = [P, P, I32]
        assert L.or_state_rollback(self.model._h, self._h, committed) == 0

    def set_mtp_position(self, position: int) -> None:
        lib().or_state_set_mtp_position(self._h, position)

    def copy_from(self, other: "OracleState"):
        lib().or_state_copy(self.model._h, self._h, other._h)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_state_destroy(self._h)
            self._h = None
