// Single-launch tensor-core forward for the d_model = ffn_dim = 128, 4-head
// model on batches of short sequences (see tile_forward.cu).
#pragma once

#include "image.cuh"
#include "tt_common.cuh"

namespace tt {

struct TileArgs {
  const char *image;
  size_t layer_stride;  // bytes between consecutive layers' arrays in the image
  LayerOffsets off;     // layer 0's offsets
  const float *final_w, *final_b;
  const float *x;       // [rows, 128]
  const uint8_t *mask;  // [rows] (batch x seq, row-major) or null
  float *y;             // [rows, 128]
  DeviceStatus *status;
  int64_t rows;  // batch * seq
  int seq, num_layers, causal;
  float scale, eps;
};

// Whether the tile forward takes this shape: d_model = ffn_dim = 128,
// 4 heads, and sequences that tile 128 rows exactly (seq a divisor of 128).
bool tile_forward_supported(const tt_config &cfg, int64_t batch, int64_t seq);

int launch_tile_forward(const TileArgs &a, cudaStream_t stream);

}  // namespace tt
