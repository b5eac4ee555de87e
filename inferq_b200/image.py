"""Layout of the state image exported by iq_state_export (see include/iq.h):
a 56-byte header, then per decoder layer the KV rows (full attention) or the
DeltaNet conv + recurrent state, then the MTP block's KV rows; all f32."""
from __future__ import annotations

import numpy as np

from .synth import Config

HEADER = np.dtype([("magic", "S8"), ("version", "<i4"), ("layers", "<i4"), ("position", "<i8"),
                   ("mtp_position", "<i8"), ("has_mtp", "<i4"), ("kv_dim", "<i4"), ("conv_dim", "<i4"),
                   ("conv_taps", "<i4"), ("rec_size", "<i4"), ("pad", "<i4")])
assert HEADER.itemsize == 56
MAGIC = b"IQSTATE1"


def shapes(cfg: Config) -> dict:
    vdim = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    return {"kv_dim": cfg.num_key_value_heads * cfg.head_dim,
            "conv_dim": 2 * cfg.linear_num_key_heads * cfg.linear_key_head_dim + vdim,
            "conv_taps": cfg.linear_conv_kernel_dim - 1,
            "rec_size": cfg.linear_num_value_heads * cfg.linear_key_head_dim * cfg.linear_value_head_dim}


def image_bytes(cfg: Config, position: int, mtp_position: int = 0) -> int:
    sh = shapes(cfg)
    b = HEADER.itemsize
    for l in range(cfg.num_hidden_layers):
        if cfg.layer_is_full(l):
            b += 2 * position * sh["kv_dim"] * 4
        else:
            b += (sh["conv_dim"] * sh["conv_taps"] + sh["rec_size"]) * 4
    if cfg.mtp_num_hidden_layers:
        b += 2 * mtp_position * sh["kv_dim"] * 4
    return b


def parse(buf: bytes | np.ndarray, cfg: Config) -> dict:
    """Split an image into its header and per-layer f32 arrays (validating)."""
    raw = np.frombuffer(bytes(buf), np.uint8)
    h = raw[:HEADER.itemsize].view(HEADER)[0]
    if h["magic"] != MAGIC or h["version"] != 1:
        raise ValueError("not a version-1 state image")
    sh = shapes(cfg)
    for k, v in sh.items():
        if int(h[k]) != v:
            raise ValueError(f"image {k} {int(h[k])} does not match the model's {v}")
    pos, mpos = int(h["position"]), int(h["mtp_position"])
    if len(raw) != image_bytes(cfg, pos, mpos):
        raise ValueError("image length does not match its header")
    f = raw[HEADER.itemsize:].view(np.float32)
    out, o = {"position": pos, "mtp_position": mpos, "layers": []}, 0
    for l in range(cfg.num_hidden_layers):
        if cfg.layer_is_full(l):
            n = pos * sh["kv_dim"]
            out["layers"].append({"keys": f[o:o + n].reshape(pos, cfg.num_key_value_heads, cfg.head_dim),
                                  "values": f[o + n:o + 2 * n].reshape(pos, cfg.num_key_value_heads, cfg.head_dim)})
            o += 2 * n
        else:
            nc = sh["conv_dim"] * sh["conv_taps"]
            out["layers"].append({"conv": f[o:o + nc].reshape(sh["conv_dim"], sh["conv_taps"]),
                                  "recurrent": f[o + nc:o + nc + sh["rec_size"]].reshape(
                                      cfg.linear_num_value_heads, cfg.linear_key_head_dim,
                                      cfg.linear_value_head_dim)})
            o += nc + sh["rec_size"]
    if cfg.mtp_num_hidden_layers:
        n = mpos * sh["kv_dim"]
        out["mtp"] = {"keys": f[o:o + n], "values": f[o + n:o + 2 * n]}
    return out


def build(cfg: Config, parts: dict) -> np.ndarray:
    """The inverse of ``parse``: an image from a dict of the same form
    (``position``, ``mtp_position``, ``layers`` and, with an MTP block, ``mtp``)."""
    sh = shapes(cfg)
    pos, mpos = int(parts["position"]), int(parts.get("mtp_position", 0))
    h = np.zeros(1, HEADER)
    h["magic"], h["version"], h["layers"] = MAGIC, 1, cfg.num_hidden_layers
    h["position"], h["mtp_position"] = pos, mpos
    h["has_mtp"] = 1 if cfg.mtp_num_hidden_layers else 0
    for k, v in sh.items():
        h[k] = v
    chunks = [h.view(np.uint8)]
    for l, layer in enumerate(parts["layers"]):
        if cfg.layer_is_full(l):
            for k in ("keys", "values"):
                a = np.ascontiguousarray(layer[k], np.float32).reshape(-1)
                assert a.size == pos * sh["kv_dim"], (l, k)
                chunks.append(a.view(np.uint8))
        else:
            c = np.ascontiguousarray(layer["conv"], np.float32).reshape(-1)
            r = np.ascontiguousarray(layer["recurrent"], np.float32).reshape(-1)
            assert c.size == sh["conv_dim"] * sh["conv_taps"] and r.size == sh["rec_size"], l
            chunks += [c.view(np.uint8), r.view(np.uint8)]
    if cfg.mtp_num_hidden_layers:
        for k in ("keys", "values"):
            a = np.ascontiguousarray(parts["mtp"][k], np.float32).reshape(-1)
            assert a.size == mpos * sh["kv_dim"], k
            chunks.append(a.view(np.uint8))
    out = np.concatenate(chunks)
    assert out.size == image_bytes(cfg, pos, mpos)
    return out


def synthetic(cfg: Config, position: int, seed: int = 0) -> np.ndarray:
    """A seeded state image at `position` (KV rows and conv history N(0, 1),
    recurrent state N(0, 0.05^2); all zeros at position 0, the true fresh
    state): a long-context starting point that costs no prefill."""
    rng = np.random.default_rng(seed)
    sh = shapes(cfg)
    layers = []
    for l in range(cfg.num_hidden_layers):
        if cfg.layer_is_full(l):
            layers.append({"keys": rng.standard_normal((position, sh["kv_dim"]), np.float32),
                           "values": rng.standard_normal((position, sh["kv_dim"]), np.float32)})
        else:
            conv = np.zeros((sh["conv_dim"], sh["conv_taps"]), np.float32)
            rec = np.zeros(sh["rec_size"], np.float32)
            if position:
                conv = rng.standard_normal(conv.shape, np.float32)
                rec = (0.05 * rng.standard_normal(rec.shape)).astype(np.float32)
            layers.append({"conv": conv, "recurrent": rec})
    parts = {"position": position, "mtp_position": position if cfg.mtp_num_hidden_layers else 0, "layers": layers}
    if cfg.mtp_num_hidden_layers:
        parts["mtp"] = {"keys": rng.standard_normal((position, sh["kv_dim"]), np.float32),
                        "values": rng.standard_normal((position, sh["kv_dim"]), np.float32)}
    return build(cfg, parts)
