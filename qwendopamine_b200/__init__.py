"""B200-native GatedDeltaNet2 (GDN-2) token mixer.

Drop-in for ``qwendopamine.models.gdn2``: :class:`GatedDeltaNet2` keeps the
reference module's API; :func:`chunk_gdn2` and :func:`fused_recurrent_gdn2`
keep the reference kernel entry points.  All compute runs in
``libgdn2_b200.so`` (hand-written CUDA for sm_100a) through a C ABI.
"""

from .gdn2 import GDN2_BACKENDS, GatedDeltaNet2, RMSNormGated, ShortConvolution, resolve_gdn2_backend
from .gdn2_ops import ChunkGDN2Function, chunk_gdn2, fused_recurrent_gdn2, fused_recurrent_gdn2_fwd
from .registry import BLOCKS, build_block

__all__ = [
    "BLOCKS",
    "ChunkGDN2Function",
    "GDN2_BACKENDS",
    "GatedDeltaNet2",
    "RMSNormGated",
    "ShortConvolution",
    "build_block",
    "chunk_gdn2",
    "fused_recurrent_gdn2",
    "fused_recurrent_gdn2_fwd",
    "resolve_gdn2_backend",
]
