"""Megatron GPT layer spec with SSA core attention (drop-in for the reference's
``SSA.ssa_triton_layer_specs``, training/train/train_ssa_triton/SSA/ssa_triton_layer_specs.py).

Same function names and signatures. Megatron-core is imported lazily, so importing this
module works without it; building a spec needs it.
"""

from __future__ import annotations

import os
from typing import Optional

from .ssa_triton_attention import SSATritonAttention


def get_bias_dropout_add(training, fused_bias_dropout_add):
    """Bias-dropout-add function factory expected by TransformerLayer (reference :27-39)."""
    import torch

    def bias_dropout_add(x_with_bias, residual, prob):
        x, bias = x_with_bias
        if bias is not None:
            x = x + bias
        if training and prob > 0.0:
            x = torch.nn.functional.dropout(x, p=prob, training=True)
        return x + residual

    return bias_dropout_add


_compiled_bda_cache = {}


def get_compiled_bias_dropout_add(training, fused_bias_dropout_add):
    """torch.compile'd bias-dropout-add (reference :45-60); falls back to eager on failure."""
    import torch

    key = (training,)
    if key in _compiled_bda_cache:
        return _compiled_bda_cache[key]
    fn = get_bias_dropout_add(training, fused_bias_dropout_add)
    try:
        compiled = torch.compile(fn, mode="reduce-overhead")
        _compiled_bda_cache[key] = compiled
        return compiled
    except Exception:
        _compiled_bda_cache[key] = fn
        return fn


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
