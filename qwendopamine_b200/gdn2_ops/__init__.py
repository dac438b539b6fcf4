"""B200 kernels behind the GDN-2 token mixer (chunkwise and recurrent)."""

from .chunk_gdn2 import ChunkGDN2Function, chunk_gdn2
from .block_ops import gated_rms_norm, short_conv
from .cp import CPChunkGDN2Function, chunk_gdn2_cp, gather_span_maps, short_conv_cp
from .fused_recurrent_gdn2 import fused_recurrent_gdn2, fused_recurrent_gdn2_fwd

__all__ = ["CPChunkGDN2Function", "ChunkGDN2Function", "chunk_gdn2", "chunk_gdn2_cp",
           "fused_recurrent_gdn2", "fused_recurrent_gdn2_fwd", "gated_rms_norm",
           "gather_span_maps", "short_conv", "short_conv_cp"]
