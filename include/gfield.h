/*
 * gfield.h -- C ABI of libgfield.so, the B200 (sm_100a) Gaussian-field
 * weight-delta renderer.
 *
 * A field is one patched linear layer: K anisotropic 2-D Gaussians
 * (mu [K,2], chol_raw [K,3], amp [K,1], all fp32) over the axes
 * row_coords [out] and col_coords [in].  The forward renders
 * delta [out*in] (row-major [out,in]) and the stable tile binning
 * (tile_ptr [T+1], gaussian_ids_sorted [P]); the backward turns
 * dL/d(delta) into d_mu [K,2], d_chol_raw [K,3], d_amp [K,1].
 *
 * Drop-in boundary: these entry points replace the pybind module
 * `gaussian_peft_cuda_field_reference` of GUASS
 * (gaussian_peft/cuda_field/csrc/ext.cpp:9-110, loaded by
 * gaussian_peft/cuda_field/loader.py:96-109).  A Python shim
 * (guass_b200/cuda_field) presents the same three methods on top of them.
 *
 * Conventions
 *  - Every pointer inside gf_field / gf_batch is a DEVICE pointer unless
 *    stated otherwise; the gf_field array itself lives in host memory and is
 *    read during the call only.
 *  - The caller owns all memory, including the scratch workspace, whose size
 *    gf_workspace_bytes() returns.  The library never allocates or frees.
 *  - All work is enqueued on `stream`; no call synchronises the stream except
 *    gf_workspace_status().  Calls on different streams must use different
 *    workspaces.
 *  - A workspace must be zero-filled once after allocation; the kernels keep
 *    their own counters consistent afterwards.
 *  - Errors: every call returns a gf_status; gf_last_error() gives the
 *    message of the last failure on the calling thread.  Conditions found on
 *    the device (pair capacity, inconsistent saved binning) are recorded in
 *    the workspace and read with gf_workspace_status().
 */
#ifndef GFIELD_H
#define GFIELD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GF_ABI_VERSION 2
/* Upper bound on fields per call (one kernel-parameter descriptor each). */
#define GF_MAX_FIELDS 192

typedef struct CUstream_st* gf_stream; /* == cudaStream_t */

typedef enum gf_status {
  GF_OK = 0,
  GF_ERR_INVALID_ARG = 1, /* bad pointer, shape or config (TORCH_CHECK in the reference) */
  GF_ERR_CAPACITY = 2,    /* gaussian_ids buffer smaller than the pair count */
  GF_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed */
  GF_ERR_STATE = 4,       /* saved binning inconsistent with the parameters */
  GF_ERR_UNSUPPORTED = 5  /* request outside the implemented envelope */
} gf_status;

typedef enum gf_dtype { GF_F32 = 0, GF_BF16 = 1 } gf_dtype;

/* Device-side condition bits returned by gf_workspace_status(). */
#define GF_FLAG_CAPACITY 0x1u /* pairs exceeded ids capacity; ids truncated */
#define GF_FLAG_STATE 0x2u    /* backward: tile_ptr/ids do not match mu/chol_raw */
#define GF_FLAG_INTERNAL 0x4u /* forward: per-tile list disagreed with tile_ptr */
#define GF_FLAG_BOUNDS 0x8u   /* debug build (libgfield_check.so) only: an index fell outside its
                                 buffer; the access was skipped */

/* Render options; mirrors ForwardConfig (gaussian_peft/cuda_field/csrc/field.h:11-18)
 * plus the output/gradient storage types. */
typedef struct gf_config {
  int64_t tile_out;        /* > 0 */
  int64_t tile_in;         /* > 0 */
  double sigma_multiplier; /* > 0 */
  int32_t normalize;       /* multiply the basis by 1/(2*pi*sqrt(det)) */
  int32_t has_clamp_quad;  /* clamp the quadratic form at clamp_quad */
  double clamp_quad;
  float out_scale;    /* delta is stored as out_scale * value (1.0 = reference);
                         the backward takes dL/d(value), i.e. the caller scales */
  int32_t out_dtype;  /* gf_dtype of delta */
  int32_t grad_dtype; /* gf_dtype of grad_delta */
  uint32_t flags;     /* GF_CFG_* options, 0 = the reference's arithmetic */
} gf_config;

/* gf_config.flags: the 32x32-tile backward evaluates its basis as
 * exp(q) = 2^(q*log2 e) with the hardware base-2 approximation instead of
 * expf (a few 1e-7 relative per term; the backward is tolerance-bound, the
 * forward's delta stays bit-exact either way). */
#define GF_CFG_BWD_EXP2 0x1u
/* gf_config.flags: with out_dtype == GF_BF16 and 32x32 tiles, the forward
 * evaluates its basis in base 2 with the hardware approximation (relative
 * error per term well below bf16's rounding; results within the bf16
 * tolerance of the reference, not bit-identical to RNE of its fp32 sum).
 * fp32 outputs and other tile shapes keep the reference's expf. */
#define GF_CFG_FWD_EXP2 0x2u

/* One field (layer).  Forward reads the inputs and writes delta, tile_ptr and
 * (in per-field id mode) gaussian_ids; backward reads grad_delta, tile_ptr and
 * the ids and writes d_mu, d_chol_raw, d_amp. */
typedef struct gf_field {
  int64_t out_features; /* rows of delta, > 0 */
  int64_t in_features;  /* cols of delta, > 0 */
  int64_t num_gaussians;/* K >= 0 */
  const float* row_coords; /* [out] */
  const float* col_coords; /* [in] */
  const float* mu;         /* [K,2] */
  const float* chol_raw;   /* [K,3] */
  const float* amp;        /* [K] */
  void* delta;             /* [out*in] out_dtype (forward output) */
  int64_t* tile_ptr;       /* [T+1], T = ceil(out/tile_out)*ceil(in/tile_in) */
  int64_t* gaussian_ids;   /* per-field id mode: [ids_capacity] */
  int64_t ids_capacity;    /* forward: capacity; backward: number of pairs */
  const void* grad_delta;  /* [out*in] grad_dtype (backward input) */
  float* d_mu;             /* [K,2] (backward output) */
  float* d_chol_raw;       /* [K,3] (backward output) */
  float* d_amp;            /* [K]   (backward output) */
  /* Optional fused weight (NULL = plain delta).  [out*in] of out_dtype; the
   * forward then stores delta[i] = out_dtype(float(base_weight[i]) +
   * out_scale * value[i]) with one rounding, i.e. W0 + delta for a layer
   * that applies one weight instead of the reference's base + delta GEMMs
   * (gaussian_peft/layers/gaussian_linear.py:222-242).  May equal `delta`
   * (in place).  The backward is unchanged: grad_delta is dL/d(value),
   * which for W_eff = W0 + out_scale * value is out_scale * dL/dW_eff. */
  const void* base_weight;
  /* Optional NVLink multicast (NVLS) address of `delta` (NULL = plain
   * stores).  The forward then writes every output row through multimem
   * stores to this address, so the switch updates the copy of `delta` on
   * every GPU bound to the multicast object while the tile is produced --
   * the render and the all-gather of the result are one kernel.  It needs
   * 16-byte aligned rows (delta and this address 16-byte aligned, in_features
   * and tile_in multiples of 16/sizeof(out_dtype)); other fields are
   * rejected with GF_ERR_UNSUPPORTED.  The kernel ends with a system-scope
   * fence; the caller synchronises the group (a barrier) before any GPU
   * reads the result. */
  void* delta_multicast;
} gf_field;

/* A batch of fields rendered by one set of launches.
 * Id mode: when `ids` is NULL, each field uses its own gaussian_ids /
 * ids_capacity.  When `ids` is non-NULL, all fields share it: the forward
 * writes field f's pairs at ids[pair_base[f] ...] and pair_base [n+1]
 * (device, exclusive prefix of the per-field pair counts), and the backward
 * reads both back. */
typedef struct gf_batch {
  int32_t num_fields;      /* 1 .. GF_MAX_FIELDS */
  const gf_field* fields;  /* HOST array of num_fields descriptors */
  int64_t* ids;            /* shared id buffer or NULL */
  int64_t ids_capacity;    /* its length */
  int64_t* pair_base;      /* [num_fields+1] device, used with `ids` */
} gf_batch;

typedef enum gf_pass { GF_PASS_FORWARD = 0, GF_PASS_BACKWARD = 1 } gf_pass;

/* ABI version compiled into the library (GF_ABI_VERSION). */
int gf_abi_version(void);

/* Stages of gf_forward, for gf_forward_stages. */
#define GF_STAGE_BIN 1u    /* per-field preprocess + binning: tile_ptr, ids, pair_base */
#define GF_STAGE_RENDER 2u /* the delta render, from the binning and workspace of the BIN stage */

/* Message for the last non-OK status returned on this thread. */
const char* gf_last_error(void);

/* Number of tiles of a field: ceil(out/tile_out) * ceil(in/tile_in). */
int64_t gf_num_tiles(int64_t out_features, int64_t in_features, int64_t tile_out, int64_t tile_in);

/* Bytes of scratch workspace a pass needs for this batch. */
size_t gf_workspace_bytes(const gf_config* cfg, const gf_batch* batch, gf_pass pass);

/* Forward render.  Replaces gaussian_field_forward
 * (gaussian_peft/cuda_field/csrc/ext.cpp:9-37, field_impl.cu:135-163,
 * forward.cu:372-569): per-Gaussian preprocess, stable tile binning and the
 * tile render, for every field of the batch.  delta is fully written (no
 * pre-zeroing needed).  tile_ptr values are relative to the field's own ids. */
gf_status gf_forward(const gf_config* cfg, const gf_batch* batch, void* workspace,
                     size_t workspace_bytes, gf_stream stream);

/* Training backward.  Replaces gaussian_field_backward
 * (gaussian_peft/cuda_field/csrc/ext.cpp:38-72, field_impl.cu:165-179,
 * backward.cu:541-716).  Reads the binning saved by gf_forward; the
 * gradients are reduced in a fixed order (bitwise reproducible). */
gf_status gf_backward(const gf_config* cfg, const gf_batch* batch, void* workspace,
                      size_t workspace_bytes, gf_stream stream);

/* Synchronises `stream`, returns the device condition bits (GF_FLAG_*)
 * accumulated in `workspace` since the last reset, optionally clearing them. */
gf_status gf_workspace_status(void* workspace, gf_stream stream, int reset, uint32_t* flags_out);

/* Profiling hook (no reference counterpart; the reference has no timing
 * facility).  After this call, gf_forward / gf_backward on any thread of the
 * process (an autograd backward runs on its own thread) record the caller's
 * CUDA events (cudaEvent_t, passed as void*) on their
 * stream: one before their first kernel and one after each kernel
 * (forward: 3 = start, bin, render; backward: 4 = start, prep, render,
 * finalize), consuming events[0..n) in order until all n are used.  n = 0
 * turns tracing off.  gf_trace_count() returns how many have been recorded. */
gf_status gf_trace_events(void* const* events, int n);
int gf_trace_count(void);

/* gf_forward in stages: `stages` is GF_STAGE_BIN, GF_STAGE_RENDER or both
 * (== gf_forward).  A RENDER stage must follow a BIN stage of the same batch,
 * parameters and workspace, in stream order.  Work that needs only the
 * binning -- gf_backward on another stream with its own workspace -- may
 * start once the BIN stage is complete, so that it overlaps the render.  (A
 * BIN stage run alone also writes the per-tile id lists, which gf_forward
 * leaves to its render kernel: one extra small launch.)
 * Trace events: BIN records 2 (start, bin), RENDER 1 (render). */
gf_status gf_forward_stages(const gf_config* cfg, const gf_batch* batch, void* workspace, size_t workspace_bytes,
                            unsigned stages, gf_stream stream);

/* The RENDER stage of gf_forward_stages for the fields [first_field,
 * first_field + num_fields) of the batch only (no reference counterpart: the
 * reference renders one layer per call).  It must follow a BIN stage of the
 * same batch, parameters and workspace in stream order; disjoint ranges may
 * be rendered by separate calls, so that work on one range's delta (an
 * exchange to other GPUs) starts while the next range renders.  The batch
 * descriptors are those of the BIN stage; only the range's delta is written.
 * Trace events: 1 (render). */
gf_status gf_forward_render_fields(const gf_config* cfg, const gf_batch* batch, void* workspace,
                                   size_t workspace_bytes, int32_t first_field, int32_t num_fields,
                                   gf_stream stream);

/* Multi-GPU publish (no reference counterpart; GUASS has no layer
 * partitioning).  Copies `bytes` from the local device buffer `src` to
 * `mc_dst`, an NVLink multicast (NVLS) address of a buffer that every GPU of
 * the group has mapped, with multimem stores: the NVSwitch delivers the data
 * to every GPU's copy, so each GPU sends its share once.  Uses at most
 * `max_blocks` CTAs (so it can run beside a render kernel), ends with a
 * system-scope fence; the caller synchronises the group afterwards (for
 * example with a symmetric-memory barrier) before reading peers' data.
 * src, mc_dst and bytes must be multiples of 16. */
gf_status gf_multicast_store(const void* src, void* mc_dst, size_t bytes, int max_blocks, gf_stream stream);

/* Densify statistics of one layer, for gf_grad_stats_accumulate. */
typedef struct gf_stats_layer {
  int64_t num_gaussians;   /* K >= 0 */
  const float* d_mu_raw;   /* [K,2] gradient of mu_raw, or NULL (adds nothing) */
  const float* d_chol_raw; /* [K,3] gradient of chol_raw, or NULL */
  const float* d_amp;      /* [K]   gradient of amp, or NULL */
  const float* amp;        /* [K]   amplitudes, or NULL (contrib not updated) */
  float* stats;            /* [5,K] planes: grad_mu, grad_cov, grad_amp, contrib, active_steps */
} gf_stats_layer;

/* One training step of GUASS's densify statistics for up to GF_MAX_FIELDS
 * layers in one launch (GaussianStatsTracker.update_from_layer_grads,
 * gaussian_peft/controllers/stats.py:47-66, which the reference runs as ~10
 * tensor ops per layer): per Gaussian k
 *   grad_mu += ||d_mu_raw[k]||_2, grad_cov += ||d_chol_raw[k]||_2,
 *   grad_amp += |d_amp[k]|, contrib += |amp[k]|, active_steps += 1
 * (stats.py:116-131).  `layers` is a HOST array read during the call. */
gf_status gf_grad_stats_accumulate(int32_t num_layers, const gf_stats_layer* layers, gf_stream stream);

/* Bytes of the library's static forward scratch (see gf_forward_noalloc). */
#define GF_NOALLOC_SCRATCH_BYTES (4u << 20)

/* Forward render that allocates nothing.  No counterpart in the reference:
 * it exists for callers that cannot allocate device memory or supply a
 * workspace -- code running inside a host that owns all device memory and
 * only hands it input and output buffers (inference-engine plugins,
 * framework custom calls, fixed-budget runtimes).  Same inputs, outputs and
 * results as gf_forward; the scratch gf_forward takes as `workspace` is a
 * 4 MiB array inside the library instead, held by every GPU that loads the
 * library until the process exits.  Batches whose forward scratch
 * (gf_workspace_bytes(cfg, batch, GF_PASS_FORWARD)) exceeds
 * GF_NOALLOC_SCRATCH_BYTES are rejected with GF_ERR_UNSUPPORTED.  The
 * device status bits of gf_workspace_status() stay inside the array, so a
 * caller detects an id buffer that was too small from the pair counts: in
 * per-field id mode tile_ptr[T] > ids_capacity, in shared-id mode
 * pair_base[num_fields] > ids_capacity (then the ids, not delta, are
 * truncated).  The first call on a device looks up the array's device
 * address on that device and keeps it for the life of the process, so make
 * it before any stream capture, and do not use this entry point on a device
 * after cudaDeviceReset() (the kept address would be stale).  All calls
 * share the one array: calls whose work overlaps on the GPU race on it and
 * must be ordered by the caller. */
gf_status gf_forward_noalloc(const gf_config* cfg, const gf_batch* batch, gf_stream stream);

#ifdef __cplusplus
}
#endif
#endif
