// Spatial tiles of one frame: fixed-size row-major runs of tile_tokens
// tokens, the last one short when tile_tokens does not divide the frame.
// Same arithmetic as the reference's TileLayout (src/tile_layout.h:13-31):
// 1560 tokens in tiles of 16 gives 97 full tiles and one of 8 tokens.
#pragma once

namespace kvp {

struct TileLayout {
    int tokens_per_frame;
    int tile_tokens;
    int tiles_per_frame;

    TileLayout(int tpf, int tt)
        : tokens_per_frame(tpf), tile_tokens(tt), tiles_per_frame((tpf + tt - 1) / tt) {}

    long tile_start(long tile_id) const { return tile_id * tile_tokens; }

    // May be <= 0 for ids past the last tile (no tokens to stage).
    int tile_count(long tile_id) const {
        const long left = (long)tokens_per_frame - tile_start(tile_id);
        return (int)(left < tile_tokens ? left : tile_tokens);
    }

    long tile_of_token(long token) const { return token / tile_tokens; }
};

}  // namespace kvp
