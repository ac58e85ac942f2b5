"""tideway_b200: B200-native (sm_100a) MoE expert-execution path for Tideway.

Router top-k, the fixed-address expert-slot table, the slot-indirect SwiGLU expert FFN
over BF16/NVFP4 banks and the weighted combine with RMSNorm, as hand-written CUDA behind a
C ABI (include/tideway_b200.h), with Python shims that keep the reference's operator
signatures (fused.py, OffloadMoeCache, OffloadMoELayer).  ``runtime`` is the offload
manager with the reference runtime's ``ensure`` / ``prefill`` interface and its installer;
``geometry`` derives the expert banks of a safetensors checkpoint and reads them into host
banks; ``ds_fp4`` re-encodes DeepSeek-V4 FP4 experts for the NVFP4 kernels; ``library``
registers the entry points as ``torch.ops.tideway_b200`` custom ops.
"""

from . import ds_fp4, geometry, library, ops, runtime  # noqa: F401
from ._lib import LIB_PATH, load  # noqa: F401
from .fused import (FusedMoe, fused_experts_decode_impl, fused_experts_impl,  # noqa: F401
                    fused_topk, moe_align_block_size)
from .moe_layer import (OffloadMoELayer, attach_offload_moe_cache, batch_context,  # noqa: F401
                        iter_offload_moe_layers)
from .offload_cache import BANK_SCHEMAS, OffloadMoeCache  # noqa: F401

__all__ = [
    "ops", "geometry", "library", "runtime", "ds_fp4", "load", "LIB_PATH", "FusedMoe",
    "fused_topk", "moe_align_block_size", "fused_experts_impl", "fused_experts_decode_impl",
    "OffloadMoELayer", "attach_offload_moe_cache", "iter_offload_moe_layers", "batch_context",
    "OffloadMoeCache",
    "BANK_SCHEMAS",
]
