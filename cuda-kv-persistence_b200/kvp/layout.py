"""Tile layout (src/tile_layout.h:13-31) through the C ABI."""

from __future__ import annotations

from ._lib import lib


class TileLayout:
    def __init__(self, tokens_per_frame: int, tile_tokens: int):
        self.tokens_per_frame = tokens_per_frame
        self.tile_tokens = tile_tokens
        self.tiles_per_frame = int(lib().kvtm_layout_tiles_per_frame(tokens_per_frame, tile_tokens))

    def tile_start(self, tile_id: int) -> int:
        return int(lib().kvtm_layout_tile_start(self.tokens_per_frame, self.tile_tokens, tile_id))

    def tile_count(self, tile_id: int) -> int:
        return int(lib().kvtm_layout_tile_count(self.tokens_per_frame, self.tile_tokens, tile_id))
