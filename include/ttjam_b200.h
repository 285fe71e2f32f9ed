/*
 * ttjam_b200.h -- C ABI of the B200 (sm_100a) pre-norm Transformer forward.
 *
 * The reference exposes this path as a PyTorch module contract
 * (torch_transformer_benchmark.py): a `TransformerConfig` shape record
 * (:29-56), `UserOptimizedTransformer.forward(x, valid_token_mask)` (:175-200)
 * whose weights arrive through `load_state_dict` (`copy_model_weights`,
 * :203-213), and an optimised implementation of it (final_submission.py) with
 * module-level `build_model` / `load_from_baseline` (final_submission.py:528-539).
 * This header is the native boundary under that contract: plain pointers and
 * sizes, no torch types. Every pointer argument that names tensor data is a
 * device pointer unless stated otherwise; every entry point that launches work
 * takes a `cudaStream_t` passed as `void*` and never synchronises it (except
 * `tt_read_status` and `tt_fp16_operand_bound`, which say so).
 *
 * Ownership: the caller owns the packed model image (`tt_image_bytes`), the
 * per-call workspace (`tt_workspace_bytes`), the input, the mask and the
 * output; the library never allocates device memory for tensors. Two things
 * it does create on its own: the 16 MiB static scratch array behind
 * `tt_forward_noalloc` (reserved per device when the module loads), and, from
 * the second `tt_forward` call with the same pointers and sizes on, one
 * private capture stream per device and an instantiated CUDA graph per cached
 * call (at most 16), which the driver backs with memory of its own. Setting
 * TT_GRAPHS=0 in the environment turns the graphs off.
 *
 * Return codes: 0 on success, a negative `tt_status` value on failure; the last
 * failure's message is available from `tt_last_error` (per host thread).
 */
#ifndef TTJAM_B200_H
#define TTJAM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TT_ABI_VERSION 2

typedef enum tt_status {
  TT_OK = 0,
  TT_ERR_INVALID_CONFIG = -1,  /* mirrors the ValueErrors of TransformerConfig.validate */
  TT_ERR_INVALID_ARGUMENT = -2,/* null pointer, bad size, misaligned pointer */
  TT_ERR_UNSUPPORTED = -3,     /* a shape this build has no kernel for */
  TT_ERR_WORKSPACE = -4,       /* workspace or image smaller than required */
  TT_ERR_CUDA = -5,            /* a CUDA runtime call or launch failed */
  TT_ERR_DEVICE_TIMEOUT = -6,  /* a bounded device-side wait gave up (status word) */
  TT_ERR_DEVICE_FAULT = -7,    /* a device-side self-check failed (status word) */
  TT_ERR_DEVICE_RANGE = -8     /* an attention operand beyond the fp16 range (status word) */
} tt_status;

/* Shape record: the fields of TransformerConfig that fix the weights
 * (torch_transformer_benchmark.py:29-37). batch_size/seq_len are per call. */
typedef struct tt_config {
  int32_t d_model;
  int32_t num_heads;
  int32_t ffn_dim;
  int32_t num_layers;
  int32_t causal;      /* 0 or 1 */
  int32_t plan;        /* 0 = pick automatically; else force one TT_PLAN_* schedule
                          (tests and benchmarks); an inapplicable plan is
                          TT_ERR_UNSUPPORTED */
  int32_t flags;       /* TT_FLAG_* bits, 0 by default */
  int32_t reserved;    /* must be 0 */
} tt_config;

/* tt_config.flags: TT_PLAN_AUTO never picks TT_PLAN_OPS_TC or TT_PLAN_TILE. Set it for a model
 * whose tt_fp16_operand_bound is not below TT_FP16_MAX: the split-precision
 * schedule stores activations as fp16 pieces, which cannot hold such values,
 * while the FFMA and cluster schedules compute in fp32 throughout. */
#define TT_FLAG_FP32_ONLY 1
#define TT_FP16_MAX 65504.0f

/* Kernel schedules of tt_forward. */
#define TT_PLAN_AUTO 0
#define TT_PLAN_CLUSTER 1   /* one launch: thread-block clusters run all layers */
#define TT_PLAN_OPS_FFMA 2  /* per-op kernels, fp32 FFMA GEMMs */
#define TT_PLAN_OPS_TC 3    /* per-op kernels, split-precision tcgen05 GEMMs and attention */
#define TT_PLAN_TILE 4      /* one launch: one CTA per 128 token rows of whole sequences runs
                               all layers on split-precision tcgen05 MMAs (d_model = ffn_dim =
                               128, 4 heads, seq a divisor of 128) */

/* One BaselineTransformerBlock's parameters, nn.Linear layout W[out,in]
 * (torch_transformer_benchmark.py:125-132, :72-75). Device pointers, fp32,
 * contiguous. */
typedef struct tt_layer_params {
  const float *norm1_weight, *norm1_bias;     /* [D] */
  const float *q_weight, *q_bias;             /* [D,D], [D] */
  const float *k_weight, *k_bias;
  const float *v_weight, *v_bias;
  const float *out_weight, *out_bias;         /* [D,D], [D] */
  const float *norm2_weight, *norm2_bias;     /* [D] */
  const float *ffn_in_weight, *ffn_in_bias;   /* [F,D], [F] */
  const float *ffn_out_weight, *ffn_out_bias; /* [D,F], [D] */
} tt_layer_params;

/* ABI version of the loaded library (TT_ABI_VERSION at build time). */
int tt_abi_version(void);

/* TransformerConfig.validate (torch_transformer_benchmark.py:39-56) plus the
 * limits of this build. Returns TT_OK, TT_ERR_INVALID_CONFIG or
 * TT_ERR_UNSUPPORTED; the message names the failing field. */
int tt_validate_config(const tt_config *cfg);

/* Bytes of the packed model image for `cfg` (0 if cfg is invalid). */
size_t tt_image_bytes(const tt_config *cfg);

/* Pack one model's parameters into `image` on `stream`: q/k/v concatenated
 * into one [3D,D] projection, precision splits for the tensor-core path, a
 * zeroed device status word. Replaces the weight delivery of
 * `copy_model_weights` / `load_state_dict` (torch_transformer_benchmark.py:
 * 203-213) and the repack of final_submission.py:426-466. `layers` is a host
 * array of `cfg->num_layers` entries. The source parameters may be freed or
 * changed once the stream has passed this call. */
int tt_pack_image(const tt_config *cfg, const tt_layer_params *layers,
                  const float *final_norm_weight, const float *final_norm_bias,
                  void *image, size_t image_bytes, void *stream);

/* An upper bound, valid for every input, on the magnitude of each activation
 * that the split-precision schedule (TT_PLAN_OPS_TC) stores as fp16 pieces:
 * the LayerNorm outputs (|gamma_i| * sqrt(D - 1) + |beta_i|, since a
 * normalised row has at most sqrt(D - 1) in any element), the q|k|v
 * projections and the attention contexts they average (row sums of
 * |W_qkv| times the LayerNorm bound, plus |b|), and the GELU outputs of ffn_in
 * (likewise). The residual stream, the scores and every accumulator stay fp32
 * and need no bound. Reads the packed fp32 weights of `image` on `stream`,
 * synchronises it and writes the bound to *bound (+inf when a weight is not
 * finite). When the bound is not below TT_FP16_MAX, the caller sets
 * TT_FLAG_FP32_ONLY (the Python module does so when it packs the weights); a
 * forced TT_PLAN_OPS_TC then produces non-finite outputs and latches
 * TT_ERR_DEVICE_RANGE. The reference computes every such model in fp32
 * (torch_transformer_benchmark.py:93-95, :141); this keeps that true here. */
int tt_fp16_operand_bound(const tt_config *cfg, const void *image, float *bound, void *stream);

/* Bytes of scratch `tt_forward` needs for one [batch, seq] call. */
size_t tt_workspace_bytes(const tt_config *cfg, int64_t batch, int64_t seq);

/* The forward pass, BaselineTransformer.forward / UserOptimizedTransformer.forward
 * (torch_transformer_benchmark.py:162-172, :185-199):
 *   x    [batch, seq, d_model] fp32, contiguous;
 *   mask [batch, seq] bytes (torch.bool layout: 0 = padding, 1 = valid), or NULL
 *        for "no mask";
 *   y    [batch, seq, d_model] fp32, written in full (padding rows are 0);
 *        may not alias x.
 * Enqueues all work on `stream`; returns after launching, without a sync.
 * Errors found on the device (a bounded wait that gave up) are latched in the
 * image's status word; read them with tt_read_status. */
int tt_forward(const tt_config *cfg, const void *image, const float *x,
               const uint8_t *mask, int64_t batch, int64_t seq, float *y,
               void *workspace, size_t workspace_bytes, void *stream);

/* Which kernel schedule (TT_PLAN_*) tt_forward runs for this call on the
 * current device. Negative on error (TT_ERR_UNSUPPORTED when cfg->plan forces
 * a schedule that cannot run this shape). */
int tt_forward_plan(const tt_config *cfg, int64_t batch, int64_t seq);

/* Number of kernel launches tt_forward makes for this call (what a profiler
 * sees per forward). Negative on error. */
int tt_forward_launch_count(const tt_config *cfg, int64_t batch, int64_t seq);

/* Element types of the typed entry points below. */
#define TT_DTYPE_F32 0   /* float32: the typed calls are then tt_pack_image / tt_forward */
#define TT_DTYPE_F16 1   /* IEEE binary16 (torch.float16) */
#define TT_DTYPE_BF16 2  /* bfloat16 (torch.bfloat16) */

/* tt_pack_image for a model whose parameters are stored in `dtype`. The
 * reference benchmarks float16 and bfloat16 by moving the whole model and its
 * input to that type (torch_transformer_benchmark.py:225-231, :698-699).
 * Every pointer in `layers` and the two final-norm pointers address elements
 * of `dtype` (cast to the struct's pointer type), at any alignment. Each value
 * widens exactly to fp32, and the image is the one tt_pack_image makes from
 * those fp32 values: a 16-bit model runs the same fp32-accurate schedules. */
int tt_pack_image_typed(const tt_config *cfg, int dtype, const tt_layer_params *layers,
                        const void *final_norm_weight, const void *final_norm_bias,
                        void *image, size_t image_bytes, void *stream);

/* Bytes of scratch tt_forward_typed needs for one [batch, seq] call:
 * tt_workspace_bytes plus, for a 16-bit dtype, fp32 copies of x and y. */
size_t tt_typed_workspace_bytes(const tt_config *cfg, int dtype, int64_t batch, int64_t seq);

/* tt_forward with x and y of element type `dtype` (the reference's forward of
 * a float16 or bfloat16 model, torch_transformer_benchmark.py:698-699, :185-199).
 * For TT_DTYPE_F16 and TT_DTYPE_BF16 it widens x exactly to fp32 (one
 * kernel), runs tt_forward's schedule on it, and rounds the fp32 output to
 * nearest even in `dtype` (one kernel): two launches more than tt_forward
 * (TT_KERNEL_CONVERT). So y is the fp32-accurate forward of the 16-bit model
 * rounded once; the reference's own 16-bit forward rounds after every
 * operation and lands farther from that value. x and y are 16-byte aligned. */
int tt_forward_typed(const tt_config *cfg, const void *image, int dtype, const void *x,
                     const uint8_t *mask, int64_t batch, int64_t seq, void *y,
                     void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of scratch tt_forward_host needs for one [batch, seq] call: device
 * room for x, y and the mask plus tt_workspace_bytes. */
size_t tt_host_workspace_bytes(const tt_config *cfg, int64_t batch, int64_t seq);

/* One forward step from and to host memory, in one call: the whole step of a
 * caller whose input arrives in, and whose output leaves through, host
 * buffers (the reference's benchmark moves x to the device and the output
 * back around each forward, torch_transformer_benchmark.py:381-392,
 * :486-506). Enqueues on `stream` the copy of x (and of the mask, unless it is
 * NULL) into the workspace, tt_forward on it, and the copy of y back; returns
 * after enqueuing, and y is complete once `stream` has passed the call.
 * Page-locked host buffers keep the copies asynchronous (pageable ones work,
 * with the driver's staging). For small calls, where the caller's own per-call
 * work is what limits the step, this is one entry instead of four. When x is
 * at most 1 MiB and every host buffer is page-locked and mapped for the device
 * (cudaHostAlloc'd memory on this platform; checked with
 * cudaPointerGetAttributes), the copies are small kernels that put every
 * 16-byte piece in flight at once (TT_KERNEL_CONVERT in the launch probe)
 * instead of DMA copies, whose fixed set-up cost dominates a short step. */
int tt_forward_host(const tt_config *cfg, const void *image, const float *x_host,
                    const uint8_t *mask_host, int64_t batch, int64_t seq, float *y_host,
                    void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of the device scratch array behind tt_forward_noalloc. */
#define TT_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)

/* tt_forward for callers that cannot allocate device memory when they run the
 * forward pass: a plugin whose host owns the whole device-memory budget, a
 * serving loop that may not call cudaMalloc (it can synchronise the device),
 * or a process whose device memory already belongs to its own pool. It takes
 * no workspace: its per-call scratch is a TT_NOALLOC_SCRATCH_BYTES (16 MiB)
 * array of static device memory inside the library, which every GPU that
 * loads the library holds until the process exits. It launches its kernels
 * directly on `stream` (never through the cached CUDA graphs of tt_forward)
 * and calls no allocator.
 *
 * The array is committed on a device when the library's module is loaded
 * there, which tt_pack_image forces: it looks up the array's device address
 * with the image's device current and caches it. So a caller that packs its
 * model before it hands its memory to a pool has the array in place, and the
 * no-alloc calls themselves only read the cached address. Should a no-alloc
 * call find no cached address for its device (no image was packed there), it
 * looks the address up then, which may load the module and reserve the array
 * at that moment; make such a first call before any stream capture.
 *
 * It runs the per-op schedule (TT_PLAN_OPS_*; TT_PLAN_AUTO picks the one
 * tt_forward uses when it does not take a single-launch path, and
 * TT_PLAN_CLUSTER and TT_PLAN_TILE, which need no scratch, are
 * TT_ERR_UNSUPPORTED). A call
 * whose scratch (tt_workspace_bytes of that schedule) exceeds the array is
 * rejected with TT_ERR_WORKSPACE and a message giving both sizes.
 *
 * All calls share the one array and it keeps the previous call's contents:
 * calls whose GPU work overlaps (unordered streams, concurrent host threads)
 * race on it. Each call writes every scratch element before reading it, so
 * nothing in it needs to start at zero. Arguments as for tt_forward. This
 * entry point has no counterpart in the reference. */
int tt_forward_noalloc(const tt_config *cfg, const void *image, const float *x,
                       const uint8_t *mask, int64_t batch, int64_t seq, float *y,
                       void *stream);

/* Synchronises `stream`, reads and clears the image's device status word.
 * *code receives TT_OK or the latched device error (TT_ERR_DEVICE_*),
 * *detail a kernel-specific location code. Returns TT_OK unless the read
 * itself failed. */
int tt_read_status(const tt_config *cfg, const void *image, int32_t *code,
                   int32_t *detail, void *stream);

/* Copies the calling thread's last error message into buf (NUL-terminated,
 * truncated to len). Returns the message length. */
int tt_last_error(char *buf, size_t len);

/* Kinds of kernel launch that tt_launch_probe_read reports. */
#define TT_KERNEL_LAYERNORM 1     /* LayerNorm (+ fp16 split) ahead of a GEMM */
#define TT_KERNEL_QKV 2           /* LN1 (when fused) + q|k|v projection */
#define TT_KERNEL_ATTENTION 3     /* masked softmax(q k^T) v */
#define TT_KERNEL_OUT_PROJ 4      /* out_proj + padded-row zeroing + residual */
#define TT_KERNEL_FFN_IN 5        /* LN2 (when fused) + ffn_in + GELU */
#define TT_KERNEL_FFN_OUT 6       /* ffn_out + residual + padded-row zeroing */
#define TT_KERNEL_FINAL_NORM 7    /* final LayerNorm + padded-row zeroing */
#define TT_KERNEL_WHOLE_FORWARD 8 /* a single-launch forward (TT_PLAN_CLUSTER, TT_PLAN_TILE) */
#define TT_KERNEL_ROW_SCAN 9      /* valid lengths and live row tiles of a padded batch */
#define TT_KERNEL_CONVERT 10      /* 16-bit x widened to fp32, fp32 y rounded to 16 bits, or a
                                     copy kernel of tt_forward_host (x, mask in; y out) */

/* Launch timing probe, a measurement aid with no counterpart in the
 * reference. tt_launch_probe_start(capacity) creates 2 * capacity timing
 * events for the calling host thread; from then on every kernel launch that
 * tt_forward, tt_forward_typed, tt_forward_host and tt_forward_noalloc make on
 * this thread is bracketed by two
 * events recorded on the launch's stream, until `capacity` launches have been
 * recorded (later launches are not bracketed). capacity 0 stops the probe and
 * destroys its events. Returns TT_OK or TT_ERR_CUDA. */
int tt_launch_probe_start(int capacity);

/* Waits for the probe's recorded events and writes, for each bracketed launch
 * i < min(count, capacity), its device time in milliseconds to ms[i] and its
 * TT_KERNEL_* kind to kinds[i]; then restarts the count at 0 (the events are
 * kept). Returns the number of launches recorded since the last read, or a
 * negative status. */
int tt_launch_probe_read(float *ms, int32_t *kinds, int capacity);

/* Test support, with no counterpart in the reference: shows that a bounded
 * device wait that runs out ends its kernel cleanly. Arms a one-shot switch:
 * the next launch, in this process, of the single-CTA split-precision GEMM
 * kernel (the tensor-core schedule's projections when the 256-row CTA-pair
 * tiles would not fill the GPU) runs with CTA 0's TMA producer skipping the
 * loads of its first k-block, so nothing ever completes that stage, and with
 * bounded waits of 2^budget_log2 cycles (16..28; 2^28 is the normal budget).
 * The waits held up by that stage then run out: the kernel latches
 * TT_ERR_DEVICE_TIMEOUT in the image's status word (detail 0x1000, 0x2000 or
 * 0x3000: the producer's, the MMA thread's or the epilogue's wait, whichever
 * gives up first), stops issuing work, waits (bounded) for the copies and tensor-core operations it
 * already started, frees its tensor memory and returns; that call's output is
 * not meaningful, later calls are unaffected. While armed, tt_forward launches
 * directly (no cached graph takes the switch). Returns TT_OK or
 * TT_ERR_INVALID_ARGUMENT. */
int tt_test_arm_wait_timeout(int budget_log2);

/* Test support, with no counterpart in the reference: y[i] = GELU(x[i]) for
 * n device floats on `stream`, computed by the device function every schedule
 * applies after ffn_in (F.gelu(approximate="none"), torch_transformer_benchmark.py:141),
 * so that its accuracy can be checked against a float64 GELU over any set of
 * arguments. Returns TT_OK, TT_ERR_INVALID_ARGUMENT or TT_ERR_CUDA. */
int tt_test_gelu(const float *x, float *y, int64_t n, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TTJAM_B200_H */
