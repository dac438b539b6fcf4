"""B200 kernels behind the GDN-2 token mixer (chunkwise and recurrent)."""

from .chunk_gdn2 import ChunkGDN2Function, chunk_gdn2
from .fused_recurrent_gdn2 import fused_recurrent_gdn2, fused_recurrent_gdn2_fwd

__all__ = ["ChunkGDN2Function", "chunk_gdn2", "fused_recurrent_gdn2", "fused_recurrent_gdn2_fwd"]
