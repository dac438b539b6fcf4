"""Block registry entries for the GDN-2 mixer (reference
``models/blocks/registry.py:16-45``): ``"gdn2"`` and ``"qwen35_gdn2"`` build
:class:`~qwendopamine_b200.gdn2.GatedDeltaNet2`; a host that keeps its own
registry can point those two keys at this class instead."""

from __future__ import annotations

from typing import Any

from torch import nn

from .gdn2 import GatedDeltaNet2

BLOCKS: dict[str, type] = {
    "gdn2": GatedDeltaNet2,
    "qwen35_gdn2": GatedDeltaNet2,
}


def build_block(block_type: str, config: Any, layer_idx: int) -> nn.Module:
    """Instantiate a registered block by name (``KeyError`` if unknown)."""
    if block_type not in BLOCKS:
        raise KeyError(f"Unknown block type: {block_type}. Available: {list(BLOCKS)}")
    return BLOCKS[block_type](config, layer_idx)
