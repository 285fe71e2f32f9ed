// Single-launch cluster forward for d_model = 128, ffn_dim = 128 and short
// sequences (see cluster_forward.cu for the schedule).
#pragma once

#include "image.cuh"
#include "tt_common.cuh"

namespace tt {

struct ClusterArgs {
  const char *image;        // packed model image
  size_t layer_stride;      // bytes between consecutive layers in the image
  LayerOffsets off;         // offsets of layer 0's arrays
  const float *final_w, *final_b;
  const float *x;           // [nseq * seq, 128]
  const uint8_t *mask;      // [nseq * seq] or null
  float *y;                 // [nseq * seq, 128]
  DeviceStatus *status;
  int seq, nseq, seq_per_cluster, num_layers, causal;
  float scale, eps;
};

struct ClusterChoice {
  int cluster = 0;          // 0: the cluster forward does not apply
  int rmax = 0;             // token rows a cluster can hold
  int seq_per_cluster = 0;
  int nclusters = 0;
};

// Whether (and how) the single-launch cluster forward runs this call on the
// current device.
ClusterChoice choose_cluster(const tt_config &cfg, int64_t batch, int64_t seq);

int launch_cluster_forward(const ClusterChoice &c, const ClusterArgs &a, int heads,
                           cudaStream_t stream);

}  // namespace tt
