"""Luciole-1B-shaped training step over the SSA kernels (benchmark config 5).

The caller of the SSA path in the reference is a NeMo / Megatron GPT decoder built from
``get_ssa_triton_gpt_layer_spec`` (training/train/train_ssa_triton/train_ssa_triton.py:401-413,
SSA/ssa_triton_layer_specs.py:63-127). Megatron and NeMo are not part of this image, so this
module restates that decoder in plain PyTorch with the same shapes and the same attention call:

    Llama-style decoder, 16 layers, hidden 2048, 32 query heads / 8 KV heads (D = 64), SwiGLU
    FFN 5632, RMSNorm, RoPE theta 10000, vocab 65,536, untied LM head; SSA attention through
    ``SSA.ssa_flash_attention`` (the tcgen05 kernels) with a learnable per-head n and fixed b.

Weights are bf16 for compute with fp32 master copies updated by AdamW (``MasterWeightAdamW``);
data parallelism is torch DDP over NCCL, one process per GPU. Everything here except the
attention is ordinary PyTorch (cuBLAS GEMMs, eager elementwise ops): this module is the
workload that measures the attention path inside a training step, not a training framework.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class LucioleConfig:
    layers: int = 16
    hidden: int = 2048
    heads: int = 32
    kv_heads: int = 8
    ffn: int = 5632
    vocab: int = 65536
    rope_theta: float = 10000.0
    norm_eps: float = 1e-5
    ssa_n: float = 0.43   # initial per-head n (learnable)
    ssa_b: float = 0.8    # fixed b
    init_std: float = 0.02

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def rope_tables(seq: int, head_dim: int, theta: float, device) -> tuple:
    """cos / sin tables [seq, head_dim] (fp32) for the rotate-half RoPE convention."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32)
                           / head_dim))
    ang = torch.outer(torch.arange(seq, device=device, dtype=torch.float32), inv)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos(), ang.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, S, H, D]; rotate-half RoPE, computed in fp32 and returned in x's dtype."""
    xf = x.float()
    h = xf.shape[-1] // 2
    rot = torch.cat([-xf[..., h:], xf[..., :h]], dim=-1)
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return (xf * c + rot * s).to(x.dtype)


def _default_attention(q, k, v, softmax_scale, ssa_n, ssa_b):
    from SSA.ssa_flash_attention import ssa_flash_attention
    return ssa_flash_attention(q, k, v, softmax_scale, ssa_n, ssa_b, causal=True)


class DecoderLayer(nn.Module):
    def __init__(self, cfg: LucioleConfig, attn_fn: Callable):
        super().__init__()
        self.cfg = cfg
        D = cfg.head_dim
        self.attn_norm = nn.RMSNorm(cfg.hidden, eps=cfg.norm_eps)
        self.qkv = nn.Linear(cfg.hidden, (cfg.heads + 2 * cfg.kv_heads) * D, bias=False)
        self.o_proj = nn.Linear(cfg.heads * D, cfg.hidden, bias=False)
        self.mlp_norm = nn.RMSNorm(cfg.hidden, eps=cfg.norm_eps)
        self.gate_up = nn.Linear(cfg.hidden, 2 * cfg.ffn, bias=False)
        self.down = nn.Linear(cfg.ffn, cfg.hidden, bias=False)
        self.ssa_n = nn.Parameter(torch.full((cfg.heads,), cfg.ssa_n))
        self.register_buffer("ssa_b", torch.tensor(cfg.ssa_b), persistent=True)
        self.attn_fn = attn_fn

    def forward(self, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        Bsz, S, _ = x.shape
        D, H, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        qkv = self.qkv(self.attn_norm(x)).view(Bsz, S, H + 2 * Hkv, D)
        q = apply_rope(qkv[:, :, :H], cos, sin)
        k = apply_rope(qkv[:, :, H:H + Hkv], cos, sin)
        v = qkv[:, :, H + Hkv:]
        # [B, S, H, D] -> [B, H, S, D] views: the kernels read the strides, and the output
        # keeps q's layout, so the permute back below is free.
        o = self.attn_fn(q.permute(0, 2, 1, 3), k.permute(0, 2, 1, 3), v.permute(0, 2, 1, 3),
                         D ** -0.5, self.ssa_n, self.ssa_b)
        x = x + self.o_proj(o.permute(0, 2, 1, 3).reshape(Bsz, S, H * D))
        g, u = self.gate_up(self.mlp_norm(x)).chunk(2, dim=-1)
        return x + self.down(F.silu(g) * u)


class LucioleDecoder(nn.Module):
    def __init__(self, cfg: LucioleConfig, attn_fn: Optional[Callable] = None):
        super().__init__()
        self.cfg = cfg
        fn = attn_fn or _default_attention
        self.embed = nn.Embedding(cfg.vocab, cfg.hidden)
        self.layers = nn.ModuleList(DecoderLayer(cfg, fn) for _ in range(cfg.layers))
        self.norm = nn.RMSNorm(cfg.hidden, eps=cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.hidden, cfg.vocab, bias=False)
        self._rope = {}
        self.reset_parameters()

    def reset_parameters(self) -> None:
        std = self.cfg.init_std
        for name, p in self.named_parameters():
            if p.dim() >= 2:
                # scaled init of the residual-branch outputs (GPT-2 / Megatron convention)
                s = std / math.sqrt(2 * self.cfg.layers) if name.endswith(("o_proj.weight",
                                                                           "down.weight")) else std
                nn.init.normal_(p, 0.0, s)

    def rope(self, seq: int, device) -> tuple:
        key = (seq, str(device))
        if key not in self._rope:
            self._rope[key] = rope_tables(seq, self.cfg.head_dim, self.cfg.rope_theta, device)
        return self._rope[key]

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        """tokens [B, S] int64 -> logits [B, S, vocab] (in the weights' dtype)."""
        cos, sin = self.rope(tokens.shape[1], tokens.device)
        x = self.embed(tokens)
        for layer in self.layers:
            x = layer(x, cos, sin)
        return self.lm_head(self.norm(x))

    def loss(self, tokens: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
        logits = self(tokens)
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1))


class MasterWeightAdamW:
    """AdamW on fp32 master copies of a bf16 model: grads are read in fp32, the step runs on
    the masters, and the bf16 weights are refreshed from them (round to nearest)."""

    def __init__(self, params: List[nn.Parameter], lr: float = 3e-4, betas=(0.9, 0.95),
                 weight_decay: float = 0.1, eps: float = 1e-8):
        self.params = [p for p in params if p.requires_grad]
        self.master = [p.detach().float().clone().requires_grad_(True) for p in self.params]
        fused = all(m.is_cuda for m in self.master)
        self.opt = torch.optim.AdamW(self.master, lr=lr, betas=betas, eps=eps,
                                     weight_decay=weight_decay, fused=fused)

    @torch.no_grad()
    def step(self) -> None:
        for p, m in zip(self.params, self.master):
            if p.grad is None:
                m.grad = None
                continue
            if m.grad is None:
                m.grad = torch.empty_like(m)
            m.grad.copy_(p.grad)
        self.opt.step()
        for p, m in zip(self.params, self.master):
            p.copy_(m)

    def zero_grad(self) -> None:
        for p in self.params:
            p.grad = None


def build(cfg: LucioleConfig, device, dtype=torch.bfloat16, seed: int = 0,
          attn_fn: Optional[Callable] = None) -> LucioleDecoder:
    """Random-init model (same weights on every rank for a given seed) in `dtype`."""
    dev = torch.device(device)
    with torch.random.fork_rng(devices=[dev] if dev.type == "cuda" else []):
        torch.manual_seed(seed)
        with dev:  # initialise in place on the target device
            model = LucioleDecoder(cfg, attn_fn)
    return model.to(dtype=dtype)


def train_step(model: nn.Module, opt: MasterWeightAdamW, tokens: torch.Tensor,
               targets: torch.Tensor) -> torch.Tensor:
    """One optimizer step on one micro-batch: forward, loss, backward (DDP all-reduces the
    gradients when `model` is wrapped), AdamW on the fp32 masters. Returns the loss (device)."""
    logits = model(tokens)
    loss = F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1))
    loss.backward()
    opt.step()
    opt.zero_grad()
    return loss.detach()


def param_count(cfg: LucioleConfig) -> int:
    D = cfg.head_dim
    per_layer = (cfg.hidden * (cfg.heads + 2 * cfg.kv_heads) * D + cfg.heads * D * cfg.hidden
                 + 3 * cfg.hidden * cfg.ffn + 2 * cfg.hidden + cfg.heads)
    return cfg.vocab * cfg.hidden * 2 + cfg.layers * per_layer + cfg.hidden


def train_flops_per_token(cfg: LucioleConfig, seq: int) -> float:
    """6 x (matmul parameters) + attention (14 * D * S / 2 per token per layer per q-head, the
    FlashAttention causal convention used for the attention metric)."""
    D = cfg.head_dim
    mm = (cfg.hidden * (cfg.heads + 2 * cfg.kv_heads) * D + cfg.heads * D * cfg.hidden
          + 3 * cfg.hidden * cfg.ffn) * cfg.layers + cfg.vocab * cfg.hidden
    attn = 14 * D * (seq / 2) * cfg.heads * cfg.layers
    return 6.0 * mm + attn
