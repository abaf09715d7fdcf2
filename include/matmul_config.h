#pragma once
// Tile parameters of the TileMix drop-in surface (reference include/matmul_config.h:3-7).
//
// The names and values are part of the interface: they fix the routing
// granularity of the mask format (one bit per kBlockM query rows x
// kBlockN * key_tiles_per_group keys). The B200 kernels do not run the
// reference's 16x16x16 WMMA fragments; they compute 128-row x 128-key tcgen05
// tiles and apply routing per 16-row / 32-key sub-tile, which the asserts
// below guarantee fits exactly.

inline constexpr int kBlockM = 16;    // query rows per routing tile
inline constexpr int kBlockN = 32;    // keys per routing key tile
inline constexpr int kTileK = 16;     // fp16 MMA K step (head-dim padding unit)
inline constexpr int kThreads = 64;   // reference launch width; sizes kFusedRowThreads
inline constexpr int kWarpSize = 32;

// The tcgen05 tile is 128 query rows x 128 keys; routing tiles must tile it.
static_assert(128 % kBlockM == 0 && 128 % kBlockN == 0,
              "routing tiles must evenly divide the 128x128 tcgen05 tile");
static_assert(kBlockM == 16 && kTileK == 16 && kWarpSize == 32,
              "the mask format and padding rules assume 16-row tiles and 16-wide K steps");
static_assert(kBlockN > 0 && kBlockN % 16 == 0 && kThreads % kWarpSize == 0,
              "key tiles must be whole MMA N steps");
