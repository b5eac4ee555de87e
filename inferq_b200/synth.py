"""Seeded random-init checkpoints with the tensor names, shapes and dtypes of
the GGUF files inferq loads (tiny Qwen3-Next, Qwen3.6-35B-A3B Q4_K_M,
Qwen3-Coder-Next-80B), generated directly on the host or on a CUDA device.

No public weights are available here, so every benchmark and parity test runs
on these.  Weights are N(0, 0.02) unless a tensor kind says otherwise; norm
vectors are stored with GGUF's ``1 + w`` already applied
(src/qwen/quantized_layer.rs:227-236); ``ssm_a`` holds ``-exp(A_log)``
(src/qwen/quantized_deltanet.rs:898-906).

Router popularity: embedding dimension 0 carries a constant 1.0 and each
expert's router row gets weight ``zipf_bias[e] / 30`` on that dimension, where
``zipf_bias[e] = -1.1 * ln(1 + rank(e))`` over a seeded permutation.  After the
RMSNorm that dimension is a near-constant ~30, so expert popularity follows a
Zipf(1.1)-shaped prior while the token-dependent part still varies the routes.
"""
from __future__ import annotations

import dataclasses
import hashlib
import math

import torch

from . import quants as Q


@dataclasses.dataclass
class Config:
    name: str
    hidden_size: int
    num_hidden_layers: int
    vocab_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rotary_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    shared_expert_intermediate_size: int
    full_attention_interval: int = 4
    mtp_num_hidden_layers: int = 0
    norm_topk_prob: int = 1
    value_heads_tiled: int = 0  # 1: model_type qwen3_5_moe_text
    max_position_embeddings: int = 262144
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10_000_000.0
    ba_fused: bool = True        # Qwen3-Next ssm_ba vs Qwen3.6 ssm_beta + ssm_alpha
    dtypes: dict = dataclasses.field(default_factory=dict)
    zipf_router: bool = False
    conv_scale: float = 0.02

    def dtype(self, kind: str) -> int:
        return self.dtypes.get(kind, self.dtypes.get("default", Q.Q8_0))

    def layer_is_full(self, layer: int) -> bool:
        return (layer + 1) % self.full_attention_interval == 0

    def abi_fields(self) -> dict:
        names = [f.name for f in dataclasses.fields(IqConfigFields)]
        return {n: getattr(self, n) for n in names}


@dataclasses.dataclass
class IqConfigFields:  # the iq_config members, in order
    hidden_size: int
    num_hidden_layers: int
    vocab_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rotary_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    shared_expert_intermediate_size: int
    full_attention_interval: int
    mtp_num_hidden_layers: int
    norm_topk_prob: int
    value_heads_tiled: int
    max_position_embeddings: int
    rms_norm_eps: float
    rope_theta: float


# Real Q4_K_M mix (multirow report / speculative-decoding notes):
# Q4_K experts gate/up, attn_q, attn_gate; Q6_K expert down, attn_qkv, LM head;
# Q8_0 ssm_out, attn_k; Q5_K attn_output.  Choices for tensors the notes do not
# list: attn_v Q6_K, shared experts like the routed ones, ssm_beta/alpha Q8_0,
# eh_proj Q8_0, token_embd Q4_K, router F32.
Q4_K_M = {
    "exp_gate": Q.Q4_K, "exp_up": Q.Q4_K, "exp_down": Q.Q6_K,
    "sh_gate": Q.Q4_K, "sh_up": Q.Q4_K, "sh_down": Q.Q6_K,
    "attn_q": Q.Q4_K, "attn_gate": Q.Q4_K, "attn_qkv": Q.Q6_K, "output": Q.Q6_K,
    "ssm_out": Q.Q8_0, "attn_k": Q.Q8_0, "attn_v": Q.Q6_K, "attn_output": Q.Q5_K,
    "ssm_ba": Q.Q8_0, "eh_proj": Q.Q8_0, "token_embd": Q.Q4_K, "router": Q.F32,
}


def tiny() -> Config:
    """The tiny Qwen3-Next-style model (hidden 512, 4 layers), every matrix Q8_0."""
    return Config(
        name="tiny-qwen3next-q8_0", hidden_size=512, num_hidden_layers=4, vocab_size=8192,
        num_attention_heads=8, num_key_value_heads=2, head_dim=64, rotary_dim=16,
        linear_num_key_heads=4, linear_num_value_heads=8, linear_key_head_dim=64,
        linear_value_head_dim=64, linear_conv_kernel_dim=4, num_experts=32, num_experts_per_tok=4,
        moe_intermediate_size=256, shared_expert_intermediate_size=256, ba_fused=True,
        value_heads_tiled=0, dtypes={"default": Q.Q8_0}, max_position_embeddings=4096,
        conv_scale=0.3)


def qwen36_35b() -> Config:
    """Qwen3.6-35B-A3B shapes (40 layers, 256 experts), Q4_K_M mix, one MTP layer."""
    return Config(
        name="qwen3.6-35b-a3b-q4_k_m", hidden_size=2048, num_hidden_layers=40, vocab_size=248320,
        num_attention_heads=16, num_key_value_heads=2, head_dim=256, rotary_dim=64,
        linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128,
        linear_value_head_dim=128, linear_conv_kernel_dim=4, num_experts=256, num_experts_per_tok=8,
        moe_intermediate_size=512, shared_expert_intermediate_size=512, mtp_num_hidden_layers=1,
        value_heads_tiled=1, ba_fused=False, dtypes=dict(Q4_K_M), zipf_router=True,
        max_position_embeddings=262144, conv_scale=0.3)


def coder_next_80b() -> Config:
    """Qwen3-Next-80B / Coder-Next shapes (48 layers, 512 experts), Q4_K_M mix."""
    c = qwen36_35b()
    c.name = "qwen3-coder-next-80b-q4_k_m"
    c.num_hidden_layers = 48
    c.num_experts = 512
    c.num_experts_per_tok = 10
    c.vocab_size = 151936
    c.mtp_num_hidden_layers = 0
    c.value_heads_tiled = 0
    c.ba_fused = True
    return c


def mini_35b() -> Config:
    """The 35B layout (Q4_K_M mix, tiled heads, split beta/alpha, MTP) at a
    size the CPU oracle runs in seconds: the parity-test model."""
    return Config(
        name="mini-35b-layout", hidden_size=512, num_hidden_layers=4, vocab_size=4096,
        num_attention_heads=4, num_key_value_heads=2, head_dim=128, rotary_dim=32,
        linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=128,
        linear_value_head_dim=128, linear_conv_kernel_dim=4, num_experts=16, num_experts_per_tok=4,
        moe_intermediate_size=256, shared_expert_intermediate_size=256, mtp_num_hidden_layers=1,
        value_heads_tiled=1, ba_fused=False, dtypes=dict(Q4_K_M), zipf_router=True,
        max_position_embeddings=4096, conv_scale=0.3)


CONFIGS = {"tiny": tiny, "qwen36_35b": qwen36_35b, "coder_next_80b": coder_next_80b, "mini_35b": mini_35b}


@dataclasses.dataclass
class Tensor:
    name: str
    dtype: int
    shape: tuple
    data: torch.Tensor  # uint8 bytes (quantized) or float32 values


def _gen(name: str, seed: int, device) -> torch.Generator:
    h = int.from_bytes(hashlib.sha256(f"{seed}:{name}".encode()).digest()[:8], "little") & ((1 << 63) - 1)
    g = torch.Generator(device=device)
    g.manual_seed(h)
    return g


def _randn(shape, name, seed, device, std=0.02) -> torch.Tensor:
    return torch.randn(shape, generator=_gen(name, seed, device), device=device, dtype=torch.float32) * std


def generate(cfg: Config, seed: int = 0, device="cpu", *, only_layers=None):
    """Yield the checkpoint's tensors one at a time (memory stays one tensor)."""
    H = cfg.hidden_size
    E, F, Fs = cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    nk, nv, dk, dv = (cfg.linear_num_key_heads, cfg.linear_num_value_heads,
                      cfg.linear_key_head_dim, cfg.linear_value_head_dim)
    conv_dim = 2 * nk * dk + nv * dv
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim

    def mat(name, kind, rows, cols, extra=None):
        x = _randn((rows, cols), name, seed, device)
        if extra is not None:
            x = extra(x)
        dt = cfg.dtype(kind)
        return Tensor(name, dt, (rows, cols), Q.encode(x, dt))

    def experts(name, kind, rows, cols):
        dt = cfg.dtype(kind)
        parts = [Q.encode(_randn((rows, cols), f"{name}#{e}", seed, device), dt) for e in range(E)]
        return Tensor(name, dt, (E, rows, cols), torch.stack(parts).reshape(E, rows, -1))

    def norm(name, n):
        return Tensor(name, Q.F32, (n,), 1.0 + _randn((n,), name, seed, device))

    def vec(name, n, std=0.02, mean=0.0):
        return Tensor(name, Q.F32, (n,), mean + _randn((n,), name, seed, device, std))

    def embed_fix(x):
        x[:, 0] = 1.0
        return x

    yield mat("token_embd.weight", "token_embd", cfg.vocab_size, H, embed_fix if cfg.zipf_router else None)
    yield norm("output_norm.weight", H)
    yield mat("output.weight", "output", cfg.vocab_size, H)
    perm = torch.randperm(E, generator=_gen("zipf", seed, "cpu"))
    zipf = torch.tensor([-1.1 * math.log(1 + int(perm[e])) for e in range(E)], dtype=torch.float32)

    def router_fix(x):
        if cfg.zipf_router:
            x[:, 0] = (zipf / 30.0).to(x.device)
        return x

    def layer(l, mtp=False):
        p = f"blk.{l}"
        yield norm(f"{p}.attn_norm.weight", H)
        yield norm(f"{p}.post_attention_norm.weight", H)
        if mtp or cfg.layer_is_full(l):
            yield mat(f"{p}.attn_q.weight", "attn_q", nh * hd * 2, H)
            yield mat(f"{p}.attn_k.weight", "attn_k", nkv * hd, H)
            yield mat(f"{p}.attn_v.weight", "attn_v", nkv * hd, H)
            yield mat(f"{p}.attn_output.weight", "attn_output", H, nh * hd)
            yield norm(f"{p}.attn_q_norm.weight", hd)
            yield norm(f"{p}.attn_k_norm.weight", hd)
        else:
            yield mat(f"{p}.attn_qkv.weight", "attn_qkv", conv_dim, H)
            yield mat(f"{p}.attn_gate.weight", "attn_gate", nv * dv, H)
            if cfg.ba_fused:
                yield mat(f"{p}.ssm_ba.weight", "ssm_ba", 2 * nv, H)
            else:
                yield mat(f"{p}.ssm_beta.weight", "ssm_ba", nv, H)
                yield mat(f"{p}.ssm_alpha.weight", "ssm_ba", nv, H)
            yield mat(f"{p}.ssm_out.weight", "ssm_out", H, nv * dv)
            cw = _randn((conv_dim, cfg.linear_conv_kernel_dim), f"{p}.ssm_conv1d.weight", seed, device,
                        cfg.conv_scale)
            yield Tensor(f"{p}.ssm_conv1d.weight", Q.F32, (conv_dim, cfg.linear_conv_kernel_dim), cw)
            a_log = _randn((nv,), f"{p}.ssm_a", seed, device, 0.5)
            yield Tensor(f"{p}.ssm_a", Q.F32, (nv,), -torch.exp(a_log))
            yield vec(f"{p}.ssm_dt.bias", nv, 0.5)
            yield norm(f"{p}.ssm_norm.weight", dv)
        rdt = cfg.dtype("router")
        rx = router_fix(_randn((E, H), f"{p}.ffn_gate_inp.weight", seed, device))
        yield Tensor(f"{p}.ffn_gate_inp.weight", rdt, (E, H), rx if rdt == Q.F32 else Q.encode(rx, rdt))
        yield vec(f"{p}.ffn_gate_inp_shexp.weight", H)
        yield experts(f"{p}.ffn_gate_exps.weight", "exp_gate", F, H)
        yield experts(f"{p}.ffn_up_exps.weight", "exp_up", F, H)
        yield experts(f"{p}.ffn_down_exps.weight", "exp_down", H, F)
        yield mat(f"{p}.ffn_gate_shexp.weight", "sh_gate", Fs, H)
        yield mat(f"{p}.ffn_up_shexp.weight", "sh_up", Fs, H)
        yield mat(f"{p}.ffn_down_shexp.weight", "sh_down", H, Fs)
        if mtp:
            yield norm(f"{p}.nextn.enorm.weight", H)
            yield norm(f"{p}.nextn.hnorm.weight", H)
            yield norm(f"{p}.nextn.shared_head_norm.weight", H)
            yield mat(f"{p}.nextn.eh_proj.weight", "eh_proj", H, 2 * H)

    for l in range(cfg.num_hidden_layers):
        if only_layers is None or l in only_layers:
            yield from layer(l)
    if cfg.mtp_num_hidden_layers == 1:
        yield from layer(cfg.num_hidden_layers, mtp=True)
