# SSA: Softmax-Substituted Attention on B200 (sm_100a).
# Drop-in for the reference package of the same name (training/train/train_ssa_triton/SSA):
#   ssa_triton_kernel.py        - forward / backward wrappers over libssa_b200.so (C ABI)
#   ssa_flash_attention.py      - autograd.Function + high-level API (+ varlen)
#   ssa_triton_attention.py     - Megatron-compatible core-attention module
#   ssa_triton_layer_specs.py   - Megatron GPT layer spec using the module
# The module names are the reference's; the kernels are hand-written CUDA, not Triton.

from .ssa_triton_kernel import check_device_status  # noqa: E402,F401
