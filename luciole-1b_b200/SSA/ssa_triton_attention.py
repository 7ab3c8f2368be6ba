"""Megatron-compatible SSA core attention over libssa_b200.so.

Drop-in for the reference ``SSA.ssa_triton_attention.SSATritonAttention``
(training/train/train_ssa_triton/SSA/ssa_triton_attention.py:32-202): same constructor
arguments, the same checkpoint keys (``ssa_n_raw`` parameter, ``ssa_b`` buffer or
``ssa_b_raw`` parameter, ``ssa_n`` buffer when not learnable; reference :99-108), the same
``forward(query, key, value, attention_mask, attn_mask_type, attention_bias,
packed_seq_params)`` on Megatron ``[S, B, H, D]`` tensors returning ``[S, B, H*D]``.

When megatron-core is importable its classes are used; otherwise small stand-ins with the
same behaviour (tensor-parallel world size 1, a plain ``nn.Module`` base) keep the module
usable and testable without Megatron.

Additions: ``ssa_n`` may be a per-head list/tensor (``[Hq]``, as the legacy FlexAttention
variant had); ``packed_seq_params`` (THD + ``cu_seqlens_q``) runs the varlen kernels instead of
asserting (reference :154-156).

Output dropout (training with ``attention_dropout > 0``). The reference runs ``nn.Dropout`` on the
kernel's output, inside Megatron's CUDA RNG tracker fork unless sequence parallelism is on
(reference :186-193). Here the kernels apply it (forward epilogue; the backward's delta pass masks
the incoming gradient), keyed by a seed drawn from torch's CUDA generator in the same tracker
context; the distribution is the same, the random stream is the kernels' own. Setting
``SSA_FUSED_DROPOUT=0`` in the environment restores the reference's ``nn.Dropout`` after the
kernel.
"""

from __future__ import annotations

import contextlib
import enum
import math
import os
import warnings
from typing import Optional

import torch
import torch.nn as nn
from torch import Tensor

from .ssa_flash_attention import ssa_flash_attention, ssa_flash_attn_varlen_func
from .ssa_triton_kernel import make_dropout_seed

try:  # pragma: no cover - exercised only where megatron-core is installed
    from megatron.core import parallel_state, tensor_parallel
    from megatron.core.transformer.enums import AttnMaskType
    from megatron.core.transformer.module import MegatronModule
    from megatron.core.utils import divide
    HAVE_MEGATRON = True
except Exception:  # megatron-core absent: minimal stand-ins with the same semantics
    HAVE_MEGATRON = False

    class AttnMaskType(enum.Enum):
        padding = 1
        causal = 2
        no_mask = 3
        padding_causal = 4
        arbitrary = 5

    class MegatronModule(nn.Module):
        def __init__(self, config=None):
            super().__init__()
            self.config = config

    class _PS:
        @staticmethod
        def get_tensor_model_parallel_world_size():
            return 1

    parallel_state = _PS()

    class _TP:
        @staticmethod
        def get_cuda_rng_tracker():
            class _T:
                def fork(self):
                    return contextlib.nullcontext()
            return _T()

    tensor_parallel = _TP()

    def divide(a, b):
        if a % b != 0:
            raise ValueError(f"{a} is not divisible by {b}")
        return a // b


class SSAAttentionConfig:
    """The TransformerConfig fields SSATritonAttention reads, for use without Megatron."""

    def __init__(self, num_attention_heads: int, kv_channels: int,
                 num_query_groups: Optional[int] = None, attention_dropout: float = 0.0,
                 apply_query_key_layer_scaling: bool = False, context_parallel_size: int = 1,
                 window_size=None, sequence_parallel: bool = False):
        self.num_attention_heads = num_attention_heads
        self.kv_channels = kv_channels
        self.num_query_groups = num_query_groups or num_attention_heads
        self.attention_dropout = attention_dropout
        self.apply_query_key_layer_scaling = apply_query_key_layer_scaling
        self.context_parallel_size = context_parallel_size
        self.window_size = window_size
        self.sequence_parallel = sequence_parallel


def _same(a: Optional[Tensor], b: Tensor) -> bool:
    """a is absent, the same storage as b, or equal to b."""
    if a is None or a is b or (a.data_ptr() == b.data_ptr() and a.shape == b.shape):
        return True
    return torch.equal(a.to(b.dtype), b)


def _megatron_to_kernel_view(t: Tensor) -> Tensor:
    """[S, B, H, D] -> [B, H, S, D] (zero-copy permute; the kernels take arbitrary strides)."""
    return t.permute(1, 2, 0, 3)


def _kernel_to_megatron_view(t: Tensor) -> Tensor:
    """[B, H, S, D] -> [S, B, H, D] (zero-copy permute)."""
    return t.permute(2, 0, 1, 3)


class SSATritonAttention(MegatronModule):
    """SSA core attention: w(s) = (1 + b|s|)^(n sign(s)), P = w / sum(w), out = P V."""

    def __init__(self, config, layer_number: int, attn_mask_type=AttnMaskType.causal,
                 attention_type: str = "self", attention_dropout: Optional[float] = None,
                 softmax_scale: Optional[float] = None, cp_comm_type: str = None,
                 ssa_n=1.5, ssa_b: float = 0.8, learnable_ssa: bool = True,
                 learnable_b: bool = False, force_contiguous_qkv: bool = False):
        super().__init__(config=config)
        self.config = config
        self.layer_number = max(1, layer_number)
        self.attn_mask_type = attn_mask_type
        self.attention_type = attention_type
        self.learnable_ssa = learnable_ssa
        self.learnable_b = learnable_b
        self.force_contiguous_qkv = force_contiguous_qkv

        assert self.config.context_parallel_size == 1, (
            "Context parallelism is only supported by TEDotProductAttention!")
        assert self.config.window_size is None, (
            "Sliding Window Attention is only supported by TEDotProductAttention!")

        projection_size = self.config.kv_channels * self.config.num_attention_heads
        world_size = parallel_state.get_tensor_model_parallel_world_size()
        self.hidden_size_per_partition = divide(projection_size, world_size)
        self.hidden_size_per_attention_head = divide(projection_size, config.num_attention_heads)
        self.num_attention_heads_per_partition = divide(self.config.num_attention_heads, world_size)
        self.num_query_groups_per_partition = divide(self.config.num_query_groups, world_size)
        self.gqa_ratio = self.num_attention_heads_per_partition // self.num_query_groups_per_partition

        self.softmax_scale = (1.0 / math.sqrt(self.hidden_size_per_attention_head)
                              if softmax_scale is None else softmax_scale)
        if self.config.apply_query_key_layer_scaling:
            self.softmax_scale /= self.layer_number

        n_init = torch.as_tensor(ssa_n, dtype=torch.float32).clone()
        if learnable_ssa:
            self.ssa_n_raw = nn.Parameter(n_init)
            if learnable_b:
                self.ssa_b_raw = nn.Parameter(torch.tensor(float(ssa_b)))
            else:
                self.register_buffer("ssa_b", torch.tensor(float(ssa_b)))
        else:
            self.register_buffer("ssa_n", n_init)
            self.register_buffer("ssa_b", torch.tensor(float(ssa_b)))

        dropout_rate = self.config.attention_dropout if attention_dropout is None else attention_dropout
        self.attention_dropout = nn.Dropout(dropout_rate)
        self.dropout_p = dropout_rate
        if self.dropout_p > 0.0:
            warnings.warn(
                "SSATritonAttention applies dropout to output (post-V-matmul), "
                "not to attention probs. Set attention_dropout=0.0 for exact parity.",
                stacklevel=2)

    def _dropout_seed(self, device) -> Optional[Tensor]:
        """Seed of the fused output dropout for this call, or None when no dropout runs in the
        kernels (eval mode, p = 0, or SSA_FUSED_DROPOUT=0). Drawn in the RNG context the
        reference's nn.Dropout runs in (:186-193)."""
        if not (self.training and self.dropout_p > 0):
            return None
        if os.environ.get("SSA_FUSED_DROPOUT", "1") in ("0", "false", "False"):
            return None
        if not getattr(self.config, "sequence_parallel", False):
            with tensor_parallel.get_cuda_rng_tracker().fork():
                return make_dropout_seed(device)
        return make_dropout_seed(device)

    def _eager_dropout(self, context: Tensor) -> Tensor:
        """The reference's dropout after the kernel (:186-193)."""
        if not getattr(self.config, "sequence_parallel", False):
            with tensor_parallel.get_cuda_rng_tracker().fork():
                return self.attention_dropout(context)
        return self.attention_dropout(context)

    def get_ssa_params(self):
        """Current (n, b) (reference :123-130)."""
        if self.learnable_ssa:
            n = self.ssa_n_raw
            b = self.ssa_b_raw if self.learnable_b else self.ssa_b
        else:
            n, b = self.ssa_n, self.ssa_b
        return n, b

    def forward(self, query: Tensor, key: Tensor, value: Tensor, attention_mask: Tensor,
                attn_mask_type=None, attention_bias: Tensor = None, packed_seq_params=None) -> Tensor:
        """query [sq, b, np, hn], key/value [sk, b, ng, hn] -> context [sq, b, np*hn].

        The causal mask is applied inside the kernel; ``attention_mask`` is ignored, as in the
        reference (:149).
        """
        assert attention_bias is None, "Attention bias not supported."
        is_causal = self.attn_mask_type == AttnMaskType.causal
        if attn_mask_type is not None:
            is_causal = attn_mask_type == AttnMaskType.causal
        ssa_n, ssa_b = self.get_ssa_params()

        if packed_seq_params is not None:
            return self._forward_packed(query, key, value, ssa_n, ssa_b, is_causal,
                                        packed_seq_params)

        query_t = _megatron_to_kernel_view(query)
        key_t = _megatron_to_kernel_view(key)
        value_t = _megatron_to_kernel_view(value)
        if self.force_contiguous_qkv:
            query_t, key_t, value_t = query_t.contiguous(), key_t.contiguous(), value_t.contiguous()

        seed = self._dropout_seed(query.device)
        context = ssa_flash_attention(query_t, key_t, value_t, softmax_scale=self.softmax_scale,
                                      ssa_n=ssa_n, ssa_b=ssa_b, causal=is_causal,
                                      dropout_p=self.dropout_p, training=self.training,
                                      dropout_seed=seed)
        if self.training and self.dropout_p > 0 and seed is None:
            context = self._eager_dropout(context)
        context = _kernel_to_megatron_view(context)
        return context.reshape(*context.size()[:-2], self.hidden_size_per_partition)

    def _forward_packed(self, query, key, value, ssa_n, ssa_b, is_causal, psp):
        """THD packed sequences: query [T, 1, np, hn] or [T, np, hn] with Megatron's
        PackedSeqParams: cu_seqlens_q (document lengths), optionally cu_seqlens_q_padded
        (document start rows when the packer pads each document, as NeMo's packed datasets do
        for context parallelism: training/finetune/nemo_patch/data/core.py:874-999) and
        max_seqlen_q. Padding rows get zero output and zero gradient."""
        cu = getattr(psp, "cu_seqlens_q", None)
        if cu is None:
            raise ValueError("packed_seq_params needs cu_seqlens_q")
        # Same-tensor checks first: comparing contents synchronises with the device.
        cu_kv = getattr(psp, "cu_seqlens_kv", None)
        if not _same(cu_kv, cu):
            raise ValueError("self-attention packing needs cu_seqlens_kv == cu_seqlens_q")
        cu = cu.to(torch.int32)
        cu_pad = getattr(psp, "cu_seqlens_q_padded", None)
        if cu_pad is not None:
            if not _same(getattr(psp, "cu_seqlens_kv_padded", None), cu_pad):
                raise ValueError("self-attention packing needs cu_seqlens_kv_padded == "
                                 "cu_seqlens_q_padded")
            cu_pad = cu_pad.to(torch.int32)
        max_s = getattr(psp, "max_seqlen_q", None)
        if max_s is None:
            max_s = int((cu[1:] - cu[:-1]).max().item())
        squeeze = query.dim() == 4
        q3 = query.squeeze(1) if squeeze else query
        k3 = key.squeeze(1) if squeeze else key
        v3 = value.squeeze(1) if squeeze else value
        seed = self._dropout_seed(q3.device)
        out = ssa_flash_attn_varlen_func(q3, k3, v3, cu, int(max_s), self.softmax_scale, ssa_n,
                                         ssa_b, is_causal, cu_pad, self.dropout_p if seed is not
                                         None else 0.0, seed)
        if self.training and self.dropout_p > 0 and seed is None:
            out = self._eager_dropout(out)
        out = out.reshape(out.shape[0], self.hidden_size_per_partition)
        return out.unsqueeze(1) if squeeze else out
