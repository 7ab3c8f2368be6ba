"""Megatron GPT layer spec with SSA core attention (drop-in for the reference's
``SSA.ssa_triton_layer_specs``, training/train/train_ssa_triton/SSA/ssa_triton_layer_specs.py).

Same layer-spec function and signature, and the same bias-dropout-add factories
(``get_bias_dropout_add``, ``get_compiled_bias_dropout_add``, reference :27-60). Megatron-core
is imported lazily, so importing this module works without it; building a spec needs it. The
residual bias-dropout-add is Megatron's own
(``megatron.core.fusions.fused_bias_dropout.get_bias_dropout_add``) when megatron-core is
importable, optionally compiled with ``torch.compile`` as the reference does
(``SSA_TRITON_COMPILE_BDA``, default on).
"""

from __future__ import annotations

import functools
import os
from typing import Optional

from .ssa_triton_attention import SSATritonAttention


def _residual_dropout(training: bool, x_with_bias, residual, prob: float):
    """residual + dropout(x + bias): the TransformerLayer's bias-dropout-add contract, eager."""
    import torch.nn.functional as F
    x, bias = x_with_bias
    if bias is not None:
        x = x + bias
    return residual + (F.dropout(x, p=prob, training=True) if training and prob > 0.0 else x)


def get_bias_dropout_add(training, fused_bias_dropout_add):
    """Bias-dropout-add factory with the reference's signature (ssa_triton_layer_specs.py:27-42):
    a function (x_with_bias, residual, prob) -> residual + dropout(x + bias). Megatron's own
    factory when megatron-core is importable, else the eager equivalent."""
    try:
        from megatron.core.fusions.fused_bias_dropout import get_bias_dropout_add as mcore_bda
    except ImportError:
        return functools.partial(_residual_dropout, bool(training))
    return mcore_bda(training, fused_bias_dropout_add)


def get_compiled_bias_dropout_add(training, fused_bias_dropout_add):
    """The unfused bias-dropout-add of :func:`get_bias_dropout_add` compiled with
    ``torch.compile`` once per ``training`` flag (reference :45-60); the eager function when no
    compiler backend is available."""
    return _compiled_bda(bool(training))


@functools.lru_cache(maxsize=None)
def _compiled_bda(training: bool):
    import torch
    eager = get_bias_dropout_add(training, False)
    try:
        return torch.compile(eager, mode="reduce-overhead")
    except Exception:  # no compiler backend here: the eager function computes the same thing
        return eager


def get_ssa_triton_gpt_layer_spec(num_experts: Optional[int] = None,
                                  moe_grouped_gemm: bool = False, qk_layernorm: bool = False,
                                  ssa_n: float = 1.5, ssa_b: float = 0.8,
                                  learnable_ssa: bool = True, learnable_b: bool = False,
                                  use_compiled_bda: Optional[bool] = None,
                                  force_contiguous_qkv: bool = False):
    """GPT layer ModuleSpec whose core attention is :class:`SSATritonAttention` (reference :63-127)."""
    from megatron.core.fusions.fused_layer_norm import FusedLayerNorm
    from megatron.core.tensor_parallel.layers import ColumnParallelLinear, RowParallelLinear
    from megatron.core.transformer.attention import SelfAttention, SelfAttentionSubmodules
    from megatron.core.transformer.enums import AttnMaskType
    from megatron.core.transformer.identity_op import IdentityOp
    from megatron.core.transformer.spec_utils import ModuleSpec
    from megatron.core.transformer.transformer_layer import (TransformerLayer,
                                                             TransformerLayerSubmodules)

    if use_compiled_bda is None:
        use_compiled_bda = os.environ.get("SSA_TRITON_COMPILE_BDA", "1") != "0"
    bda_factory = get_compiled_bias_dropout_add if use_compiled_bda else get_bias_dropout_add
    mlp = _get_mlp_module_spec(num_experts=num_experts, moe_grouped_gemm=moe_grouped_gemm)
    core = ModuleSpec(module=SSATritonAttention,
                      params={"ssa_n": ssa_n, "ssa_b": ssa_b, "learnable_ssa": learnable_ssa,
                              "learnable_b": learnable_b,
                              "force_contiguous_qkv": force_contiguous_qkv})
    return ModuleSpec(
        module=TransformerLayer,
        submodules=TransformerLayerSubmodules(
            input_layernorm=FusedLayerNorm,
            self_attention=ModuleSpec(
                module=SelfAttention, params={"attn_mask_type": AttnMaskType.causal},
                submodules=SelfAttentionSubmodules(
                    linear_qkv=ColumnParallelLinear, core_attention=core,
                    linear_proj=RowParallelLinear,
                    q_layernorm=FusedLayerNorm if qk_layernorm else IdentityOp,
                    k_layernorm=FusedLayerNorm if qk_layernorm else IdentityOp)),
            self_attn_bda=bda_factory, pre_mlp_layernorm=FusedLayerNorm, mlp=mlp,
            mlp_bda=bda_factory))


def _get_mlp_module_spec(num_experts: Optional[int] = None, moe_grouped_gemm: bool = False):
    """MLP spec (reference :130-150)."""
    from megatron.core.tensor_parallel.layers import ColumnParallelLinear, RowParallelLinear
    from megatron.core.transformer.mlp import MLP, MLPSubmodules
    from megatron.core.transformer.spec_utils import ModuleSpec

    if num_experts is None:
        return ModuleSpec(module=MLP, submodules=MLPSubmodules(linear_fc1=ColumnParallelLinear,
                                                               linear_fc2=RowParallelLinear))
    from megatron.core.transformer.moe.moe_layer import MoELayer
    if moe_grouped_gemm:
        from megatron.core.transformer.moe.experts import GroupedMLP
        return ModuleSpec(module=MoELayer, submodules=GroupedMLP)
    from megatron.core.transformer.moe.experts import SequentialMLP
    return ModuleSpec(module=MoELayer, submodules=SequentialMLP)
