"""B200-native (sm_100a) MoE-layer hot path with the call signatures of the
reference's components: ``PermutedSparseMoE`` (C5), ``fused_moe_forward``
(C9), the expert-parallel ``EPSparseMoE`` schedules (C6 lean all_reduce, C7
all_to_all) and ``HybridMoE`` (C8).  The kernels live in ``libmoe_b200.so``
behind the C ABI of ``include/moe_b200.h``."""

from .experts import SwiGLU_MLP, load_qwen3_moe_layer
from .fused_moe import fused_moe_forward
from .permuted_moe import PermutedSparseMoE

__all__ = ["PermutedSparseMoE", "SwiGLU_MLP", "fused_moe_forward", "load_qwen3_moe_layer"]
