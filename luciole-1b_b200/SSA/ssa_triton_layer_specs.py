"""Megatron GPT layer spec with SSA core attention (drop-in for the reference's
``SSA.ssa_triton_layer_specs``, training/train/train_ssa_triton/SSA/ssa_triton_layer_specs.py).

Same layer-spec function and signature. Megatron-core is imported lazily, so importing this
module works without it; building a spec needs it. The residual bias-dropout-add is Megatron's
own (``megatron.core.fusions.fused_bias_dropout.get_bias_dropout_add``), optionally compiled with
``torch.compile`` as the reference does (``SSA_TRITON_COMPILE_BDA``, default on).
"""

from __future__ import annotations

import functools
import os
from typing import Optional

from .ssa_triton_attention import SSATritonAttention


def _compiled_bda_factory(training, fused):
    """Bias-dropout-add factory for ``use_compiled_bda`` (the reference compiles its unfused
    bias-dropout-add with ``torch.compile``, ssa_triton_layer_specs.py:45-60): Megatron's own
    unfused function for ``training``, compiled once per flag."""
    return _compiled_bda(bool(training))


@functools.lru_cache(maxsize=None)
def _compiled_bda(training: bool):
    import torch
    from megatron.core.fusions.fused_bias_dropout import get_bias_dropout_add
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

    from megatron.core.fusions.fused_bias_dropout import get_bias_dropout_add

    if use_compiled_bda is None:
        use_compiled_bda = os.environ.get("SSA_TRITON_COMPILE_BDA", "1") != "0"
    bda_factory = _compiled_bda_factory if use_compiled_bda else get_bias_dropout_add
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
