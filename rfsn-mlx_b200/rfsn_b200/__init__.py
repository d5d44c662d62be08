"""B200-native exact segmented attention for rfsn-MLX's cache/attention API.

Module layout mirrors the reference package ``rfsn_v10_5`` for the path it
replaces: ``config``, ``block_manager``, ``storage``, ``residency``,
``cache``, ``attention_exact``, the attention step of ``layer`` and the
``model`` driver (dense parts in torch). Tensors
are torch CUDA tensors; the compute runs in ``librfsn_b200.so`` (sm_100a),
bound through ``_native``. Multi-GPU sharded decode lives in ``sharded``.
"""

from .config import RFSNConfig, RuntimeMode, resolve_dtype, validate_session_id  # noqa: F401
from .block_manager import BlockId, BlockLocation, BlockManager, BlockManifest, BlockSpan, PageTable  # noqa: F401
from .storage import BlockStorage  # noqa: F401
from .residency import ResidencyManager, ResidencyMetrics  # noqa: F401
from .cache import LayerKVCache, PagedSegments, RFSNCache, derive_model_id  # noqa: F401
from .attention_exact import (  # noqa: F401
    build_causal_mask,
    exact_attention,
    exact_decode_attention,
    exact_prefill_attention,
    run_exact_attention,
    run_segmented_attention,
)
from .layer import GraphedDecodeStep, attention_step, build_rope_tables  # noqa: F401
from .model import RFSNMLX, RFSNLayer, RFSNLayerMLX, RFSNLayerNorm, RFSNModel  # noqa: F401

__all__ = [
    "RFSNConfig",
    "RuntimeMode",
    "RFSNCache",
    "LayerKVCache",
    "PagedSegments",
    "BlockId",
    "BlockLocation",
    "BlockManager",
    "BlockManifest",
    "BlockSpan",
    "PageTable",
    "ResidencyManager",
    "BlockStorage",
    "build_rope_tables",
    "attention_step",
    "GraphedDecodeStep",
    "run_segmented_attention",
    "run_exact_attention",
    "exact_attention",
    "exact_prefill_attention",
    "exact_decode_attention",
    "build_causal_mask",
    "RFSNModel",
    "RFSNMLX",
    "RFSNLayer",
    "RFSNLayerMLX",
]
