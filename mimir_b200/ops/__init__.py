"""Hot ops with hand-written sm_100a CUDA kernels and PyTorch oracles.

Every public function here dispatches to the compiled extension ``mimir_b200._C`` for
CUDA tensors and to a plain PyTorch formulation otherwise (CPU, or
``MIMIR_DISABLE_KERNELS=1``).
"""
from mimir_b200.ops._ext import ext, available, kernels_enabled  # noqa: F401
from mimir_b200.ops.norm import add_rms_norm, rms_norm  # noqa: F401
from mimir_b200.ops.swiglu import swiglu, swiglu_reference  # noqa: F401
from mimir_b200.ops.attention import (  # noqa: F401
    dense_prefixlm_attention, prefixlm_attention, gated_prefixlm_attention, gated_attention_composite)
from mimir_b200.ops.loss import linear_cross_entropy, linear_cross_entropy_reference  # noqa: F401
from mimir_b200.ops.moe import moe_plan  # noqa: F401
from mimir_b200.ops.ngram import ngram_lookup  # noqa: F401
from mimir_b200.ops.embedding import scaled_embedding  # noqa: F401
from mimir_b200.ops.gemm import linear, swiglu_mlp, swiglu_mlp_supported  # noqa: F401
