"""B200 kernels behind the GDN-2 token mixer (chunkwise and recurrent)."""

from .chunk_gdn2 import ChunkGDN2Function, chunk_gdn2
from .cp import CPChunkGDN2Function, chunk_gdn2_cp, gather_span_maps
from .fused_recurrent_gdn2 import fused_recurrent_gdn2, fused_recurrent_gdn2_fwd

__all__ = ["CPChunkGDN2Function", "ChunkGDN2Function", "chunk_gdn2", "chunk_gdn2_cp",
           "fused_recurrent_gdn2", "fused_recurrent_gdn2_fwd", "gather_span_maps"]
