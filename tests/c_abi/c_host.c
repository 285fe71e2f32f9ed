/*
 * A plain C host of the C ABI (include/ttjam_b200.h): no Python, no torch.
 * Reads a model's parameters and one input from binary files written by the
 * test that drives it, packs the image, runs tt_forward with a caller
 * workspace and tt_forward_noalloc, and writes both outputs. Device memory and
 * streams come from the CUDA runtime, as a C or C++ serving host would use it.
 *
 *   c_host <dir>   reads  <dir>/cfg.txt      "d_model num_heads ffn_dim num_layers causal batch seq has_mask"
 *                         <dir>/params.bin   the parameters, fp32, in the reference's state-dict order
 *                         <dir>/x.bin        [batch, seq, d_model] fp32
 *                         <dir>/mask.bin     [batch, seq] bytes (when has_mask)
 *                  writes <dir>/y.bin, <dir>/y_noalloc.bin, and prints the status lines
 */
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ttjam_b200.h"

#define CHECK_CUDA(e)                                                             \
  do {                                                                            \
    cudaError_t err_ = (e);                                                       \
    if (err_ != cudaSuccess) {                                                    \
      fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(err_), __FILE__, __LINE__); \
      return 2;                                                                   \
    }                                                                             \
  } while (0)

#define CHECK_TT(e)                                                               \
  do {                                                                            \
    int rc_ = (e);                                                                \
    if (rc_ != TT_OK) {                                                           \
      char msg_[512];                                                             \
      tt_last_error(msg_, sizeof msg_);                                           \
      fprintf(stderr, "%s failed: %d (%s)\n", #e, rc_, msg_);                     \
      return 3;                                                                   \
    }                                                                             \
  } while (0)

static void *read_file(const char *dir, const char *name, size_t *len) {
  char path[1024];
  snprintf(path, sizeof path, "%s/%s", dir, name);
  FILE *f = fopen(path, "rb");
  if (!f) return NULL;
  fseek(f, 0, SEEK_END);
  *len = (size_t)ftell(f);
  fseek(f, 0, SEEK_SET);
  void *buf = malloc(*len ? *len : 1);
  if (buf && fread(buf, 1, *len, f) != *len) {
    free(buf);
    buf = NULL;
  }
  fclose(f);
  return buf;
}

static int write_file(const char *dir, const char *name, const void *data, size_t len) {
  char path[1024];
  snprintf(path, sizeof path, "%s/%s", dir, name);
  FILE *f = fopen(path, "wb");
  if (!f) return 1;
  const size_t n = fwrite(data, 1, len, f);
  fclose(f);
  return n == len ? 0 : 1;
}

int main(int argc, char **argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: c_host <dir>\n");
    return 1;
  }
  const char *dir = argv[1];
  tt_config cfg;
  memset(&cfg, 0, sizeof cfg);
  long long batch = 0, seq = 0;
  int has_mask = 0;
  {
    char path[1024];
    snprintf(path, sizeof path, "%s/cfg.txt", dir);
    FILE *f = fopen(path, "r");
    if (!f || fscanf(f, "%d %d %d %d %d %lld %lld %d", &cfg.d_model, &cfg.num_heads, &cfg.ffn_dim,
                     &cfg.num_layers, &cfg.causal, &batch, &seq, &has_mask) != 8) {
      fprintf(stderr, "bad cfg.txt\n");
      return 1;
    }
    fclose(f);
  }
  if (tt_abi_version() != TT_ABI_VERSION) {
    fprintf(stderr, "ABI version mismatch\n");
    return 1;
  }
  CHECK_TT(tt_validate_config(&cfg));
  const size_t D = (size_t)cfg.d_model, F = (size_t)cfg.ffn_dim, L = (size_t)cfg.num_layers;
  /* per layer, in state-dict order: norm1 w b, q w b, k w b, v w b, out w b,
     norm2 w b, ffn_in w b, ffn_out w b; then final_norm w b */
  const size_t sizes[16] = {D, D, D * D, D, D * D, D, D * D, D, D * D, D, D, D, F * D, F, D * F, D};
  size_t per_layer = 0;
  for (int i = 0; i < 16; ++i) per_layer += sizes[i];
  const size_t n_params = L * per_layer + 2 * D;
  size_t len = 0;
  float *params = (float *)read_file(dir, "params.bin", &len);
  if (!params || len != n_params * sizeof(float)) {
    fprintf(stderr, "params.bin: expected %zu floats\n", n_params);
    return 1;
  }
  const size_t n_x = (size_t)batch * (size_t)seq * D;
  float *x = (float *)read_file(dir, "x.bin", &len);
  if (!x || len != n_x * sizeof(float)) {
    fprintf(stderr, "x.bin: expected %zu floats\n", n_x);
    return 1;
  }
  unsigned char *mask = NULL;
  if (has_mask) {
    mask = (unsigned char *)read_file(dir, "mask.bin", &len);
    if (!mask || len != (size_t)(batch * seq)) {
      fprintf(stderr, "mask.bin: expected %lld bytes\n", batch * seq);
      return 1;
    }
  }

  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreate(&stream));
  float *d_params = NULL, *d_x = NULL, *d_y = NULL, *d_y2 = NULL;
  unsigned char *d_mask = NULL;
  CHECK_CUDA(cudaMalloc((void **)&d_params, n_params * sizeof(float)));
  CHECK_CUDA(cudaMemcpy(d_params, params, n_params * sizeof(float), cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMalloc((void **)&d_x, n_x * sizeof(float)));
  CHECK_CUDA(cudaMemcpy(d_x, x, n_x * sizeof(float), cudaMemcpyHostToDevice));
  CHECK_CUDA(cudaMalloc((void **)&d_y, n_x * sizeof(float)));
  CHECK_CUDA(cudaMalloc((void **)&d_y2, n_x * sizeof(float)));
  if (mask) {
    CHECK_CUDA(cudaMalloc((void **)&d_mask, (size_t)(batch * seq)));
    CHECK_CUDA(cudaMemcpy(d_mask, mask, (size_t)(batch * seq), cudaMemcpyHostToDevice));
  }

  tt_layer_params *layers = (tt_layer_params *)calloc(L, sizeof(tt_layer_params));
  const float *p = d_params;
  for (size_t l = 0; l < L; ++l) {
    const float **fields[16] = {
        &layers[l].norm1_weight,  &layers[l].norm1_bias,   &layers[l].q_weight,
        &layers[l].q_bias,        &layers[l].k_weight,     &layers[l].k_bias,
        &layers[l].v_weight,      &layers[l].v_bias,       &layers[l].out_weight,
        &layers[l].out_bias,      &layers[l].norm2_weight, &layers[l].norm2_bias,
        &layers[l].ffn_in_weight, &layers[l].ffn_in_bias,  &layers[l].ffn_out_weight,
        &layers[l].ffn_out_bias};
    for (int i = 0; i < 16; ++i) {
      *fields[i] = p;
      p += sizes[i];
    }
  }
  const float *final_w = p, *final_b = p + D;

  const size_t image_bytes = tt_image_bytes(&cfg);
  void *d_image = NULL;
  CHECK_CUDA(cudaMalloc(&d_image, image_bytes));
  CHECK_TT(tt_pack_image(&cfg, layers, final_w, final_b, d_image, image_bytes, stream));
  float bound = 0.f;
  CHECK_TT(tt_fp16_operand_bound(&cfg, d_image, &bound, stream));
  if (!(bound < TT_FP16_MAX)) cfg.flags |= TT_FLAG_FP32_ONLY;

  const size_t ws_bytes = tt_workspace_bytes(&cfg, batch, seq);
  void *d_ws = NULL;
  if (ws_bytes) CHECK_CUDA(cudaMalloc(&d_ws, ws_bytes));
  const int plan = tt_forward_plan(&cfg, batch, seq);
  CHECK_TT(tt_forward(&cfg, d_image, d_x, d_mask, batch, seq, d_y, d_ws, ws_bytes, stream));
  /* a second call with the same pointers replays the cached graph */
  CHECK_TT(tt_forward(&cfg, d_image, d_x, d_mask, batch, seq, d_y, d_ws, ws_bytes, stream));
  int noalloc_rc = tt_forward_noalloc(&cfg, d_image, d_x, d_mask, batch, seq, d_y2, stream);
  CHECK_CUDA(cudaStreamSynchronize(stream));
  int32_t code = 0, detail = 0;
  CHECK_TT(tt_read_status(&cfg, d_image, &code, &detail, stream));

  float *y = (float *)malloc(n_x * sizeof(float));
  CHECK_CUDA(cudaMemcpy(y, d_y, n_x * sizeof(float), cudaMemcpyDeviceToHost));
  if (write_file(dir, "y.bin", y, n_x * sizeof(float))) return 1;
  if (noalloc_rc == TT_OK) {
    CHECK_CUDA(cudaMemcpy(y, d_y2, n_x * sizeof(float), cudaMemcpyDeviceToHost));
    if (write_file(dir, "y_noalloc.bin", y, n_x * sizeof(float))) return 1;
  }
  printf("plan %d launches %d image_bytes %zu workspace_bytes %zu bound %g status %d detail %d "
         "noalloc %d\n",
         plan, tt_forward_launch_count(&cfg, batch, seq), image_bytes, ws_bytes, (double)bound,
         code, detail, noalloc_rc);

  free(y);
  free(layers);
  free(params);
  free(x);
  free(mask);
  cudaFree(d_ws);
  cudaFree(d_image);
  cudaFree(d_mask);
  cudaFree(d_y2);
  cudaFree(d_y);
  cudaFree(d_x);
  cudaFree(d_params);
  cudaStreamDestroy(stream);
  return 0;
}
