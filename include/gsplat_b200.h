/*
 * gsplat_b200.h — C ABI of the B200 (sm_100a) differentiable Gaussian-splat rasterizer.
 *
 * Every entry point takes raw device pointers, element counts and a CUDA stream
 * (passed as `void*`, a `cudaStream_t`; NULL means the legacy default stream),
 * enqueues its kernels on that stream and returns an `int` status (GSB_OK == 0).
 * Nothing here allocates memory: outputs, the per-call workspace (sized by the
 * matching `*_workspace_size` query) and the status block are caller-owned.
 * No call synchronises the device; the caller reads the status block when it
 * needs a device-side result (the pair total, error flags, the max tile count).
 *
 * Layouts (all row-major, fp32 unless stated):
 *   2D splats   means2d [B*G,2], conics [B*G,3] (a,b,c of the inverse 2D covariance),
 *               colors [B*G,3], opacities [B*G], depths [B*G]  (view-major: index b*G+g)
 *   records     rec [B*G,12]: splat params in depth-rank order (see GSB_REC_* below)
 *   pair keys   keys [P] uint64 = (global_tile << 32) | depth_key, sorted ascending
 *   binned ids  binned_ids [P] int32 = depth-rank index b*G+rank, tile-major
 *   tile ranges tile_offsets [B*tiles+1] int32 (exclusive prefix of per-tile counts)
 *   image       out_rgb [B,H,W,3]; per-pixel state final_T [B,H,W], last_idx [B,H,W] int32
 *
 * Each entry point names the reference interface it replaces (paths inside
 * nbardy/fast-mac-gsplat).
 */
#ifndef GSPLAT_B200_H
#define GSPLAT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define GSB_OK 0
#define GSB_ERR_INVALID_ARGUMENT 1 /* bad pointer / shape / config */
#define GSB_ERR_UNSUPPORTED 2      /* e.g. tile_size != 16 */
#define GSB_ERR_WORKSPACE 3        /* workspace smaller than *_workspace_size */
#define GSB_ERR_CAPACITY 4         /* pair count beyond the int32 index range, or a size beyond
                                      an allocation-free entry point's fixed maximum */
#define GSB_ERR_DEVICE_TIMEOUT 5   /* a bounded device-side wait ran out */
#define GSB_ERR_CUDA 6             /* a CUDA runtime call failed */
#define GSB_ERR_DEVICE_BOUNDS 7    /* a device-side bounds check fired */

/* ---- device status block (caller-owned, GSB_STATUS_WORDS x uint32) ------ *
 * gsb_bin_count clears it; the render and backward calls of that binning use
 * it too (error flags, the backward's tile claim counter), so calls sharing a
 * status block must be ordered on one stream.                              */
#define GSB_STATUS_TOTAL_PAIRS 0    /* written by gsb_bin_prepare */
#define GSB_STATUS_ERROR 1          /* OR of GSB_DEVERR_* flags */
#define GSB_STATUS_MAX_TILE_COUNT 2 /* written by gsb_tile_stats */
#define GSB_STATUS_ERROR_SITE 3     /* first kernel site that raised an error */
#define GSB_STATUS_PAIR_TOTAL64 4   /* words 4-5: 64-bit pair total, written by gsb_bin_count */
#define GSB_STATUS_MASK_WORDS 6     /* hit-bit words of tile_masks handed out (gsb_bin_count) */
#define GSB_STATUS_TILE_CLAIM 8     /* tile claim counter of the backward warp kernel (0 between calls) */
#define GSB_STATUS_WORDS 16

#define GSB_DEVERR_LOOKBACK_TIMEOUT 1u /* decoupled look-back spin limit hit */
#define GSB_DEVERR_PAIR_OVERFLOW 2u    /* emit wrote past its scan slot / P >= 2^31 */
#define GSB_DEVERR_BOUNDS 4u           /* index outside its buffer */
#define GSB_DEVERR_PEER_TIMEOUT 8u     /* a peer did not reach a gsb_peer_allreduce_sum barrier in time */

/* ---- packed splat record (12 floats, 48 B, 16-B aligned) --------------- */
#define GSB_REC_FLOATS 12
/* rec[r*12 + ...]: 0 mean_x, 1 mean_y, 2 conic_a, 3 conic_b,
 *                  4 conic_c, 5 opacity, 6 color_r, 7 color_g,
 *                  8 color_b, 9 depth_key (uint32 bits),
 *                  10 ln(alpha_threshold/opacity)  (visible iff power in [this, 0]),
 *                  11 ln(max_alpha/opacity)        (alpha saturates iff power >= this) */
/* grad record (same 12-float stride, depth-rank order):
 *   0 g_mean_x, 1 g_mean_y, 2 g_a, 3 g_b, 4 g_c, 5 g_opacity, 6 g_r, 7 g_g, 8 g_b_color */

/* ---- raster meta (replaces the meta_i32 / meta_f32 tensors) ------------ */
typedef struct gsb_raster_meta {
  int32_t height;
  int32_t width;
  int32_t tile_size;           /* must be 16 */
  int32_t batch_size;          /* B (views) */
  int32_t gaussians_per_batch; /* G */
  float alpha_threshold;       /* 1/255 */
  float transmittance_threshold; /* 1e-4 */
  float background[3];
  float eps;       /* 1e-8 */
  float max_alpha; /* 0.99 */
} gsb_raster_meta;

/* Library version (major*10000 + minor*100 + patch). */
int gsb_version(void);
/* Human-readable text for a status code. */
const char* gsb_status_string(int code);
/* Number of kernels this library has launched in this process (all devices);
 * a diagnostic for launch accounting, no reference counterpart. */
uint64_t gsb_kernel_launches(void);
/* FP32 throughput probe, a measurement diagnostic with no reference counterpart:
 * blocks_per_sm x SMs blocks of 256 threads, each thread running 8 independent
 * chains of `iters` fused multiply-adds (packed != 0: fma.rn.f32x2, two per
 * instruction). FLOPs per launch = gsb_fma_probe_out_floats(blocks_per_sm) x
 * iters x 8 x 2 (x 2 packed). out receives one float per thread. */
int64_t gsb_fma_probe_out_floats(int32_t blocks_per_sm);
int gsb_fma_probe(int32_t packed, int32_t blocks_per_sm, int32_t iters, float* out, void* stream);

/* ---- binning, phase 1 ---------------------------------------------------
 * Replaces: the depth sort + gathers of
 *   torch_gsplat_bridge_fast/rasterize.py:43-47 and
 *   variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:708-717,
 * `count_tiles` (variants/v8_project3d/csrc/metal/gsplat_v8_project3d_kernels.metal:697-741)
 * and the cumsum + `.item()` of metal_bin
 *   (variants/v8_project3d/csrc/metal/gsplat_metal.mm:341-364).
 * Stable per-view depth sort, gather into packed records, exact per-splat tile
 * counts, exclusive scan of those counts in depth-rank order.
 * Outputs: perm [B*G] int32 (perm[b*G+rank] = original index g within view b),
 *          rec [B*G*12], pair_offsets [B*G+1] int32,
 *          status[GSB_STATUS_TOTAL_PAIRS] = total pair count P. */
size_t gsb_bin_prepare_workspace_size(const gsb_raster_meta* meta);
int gsb_bin_prepare(const gsb_raster_meta* meta, const float* means2d, const float* conics,
                    const float* colors, const float* opacities, const float* depths,
                    int32_t* perm, float* rec, int32_t* pair_offsets, uint32_t* status,
                    void* workspace, size_t workspace_bytes, void* stream);

/* gsb_bin_prepare in two calls on the same workspace, so the caller can read the
 * pair total early: gsb_bin_count zeroes the status block and counts each splat's
 * tiles (status words GSB_STATUS_PAIR_TOTAL64.. = 64-bit total P); a device-to-host
 * copy of that word enqueued right after it completes while gsb_bin_sort_scan
 * (depth sort, gather, scan) still runs. */
int gsb_bin_count(const gsb_raster_meta* meta, const float* means2d, const float* conics,
                  const float* opacities, const float* depths, uint64_t* tile_masks, uint32_t* status,
                  void* workspace, size_t workspace_bytes, void* stream);
/* tile_masks (optional; NULL in all three calls, or the same buffer of
 * gsb_bin_tile_masks_size bytes in gsb_bin_count, gsb_bin_sort_scan and
 * gsb_bin_emit) records which candidate tiles of each splat were hit, so
 * gsb_bin_emit writes the pairs without testing the tiles again. It starts with
 * B*G 64-bit slots in rank order: for a splat whose snugbox holds at most 64
 * candidate tiles, bit k marks candidate k (row-major in its box) as hit; for a
 * larger splat, the slot is the word offset of its hit bits in the uint32 region
 * after the slots (bit k of word offset + k/32), or all ones when the region
 * (8 words per splat) was full and the splat is tested again. */
size_t gsb_bin_tile_masks_size(const gsb_raster_meta* meta);
int gsb_bin_sort_scan(const gsb_raster_meta* meta, const float* means2d, const float* conics,
                      const float* colors, const float* opacities, const float* depths, int32_t* perm,
                      float* rec, int32_t* pair_offsets, uint64_t* tile_masks, uint32_t* status,
                      void* workspace, size_t workspace_bytes, void* stream);

/* ---- binning, phase 2 ---------------------------------------------------
 * Replaces: `emit_binned_ids` (…/gsplat_v8_project3d_kernels.metal:743-780), the per-tile
 * `bitonic_sort_ids` (…:594-617) and the tile offsets of metal_bin (…/gsplat_metal.mm:358-361).
 * Emits (tile, rank) pairs at the scan offsets, stable radix-sorts them by tile (32-bit
 * keys), and writes tile ranges. `total_pairs` is status[GSB_STATUS_TOTAL_PAIRS].
 * `keys` is optional (NULL skips it): it receives (tile<<32 | depth_key) of each sorted
 * pair, the full 64-bit order key. `tile_masks` is optional: the masks written by
 * gsb_bin_sort_scan for these records. */
size_t gsb_bin_emit_workspace_size(const gsb_raster_meta* meta, int64_t total_pairs);
int gsb_bin_emit(const gsb_raster_meta* meta, const float* rec, const int32_t* pair_offsets,
                 const uint64_t* tile_masks, int64_t total_pairs, uint64_t* keys, int32_t* binned_ids,
                 int32_t* tile_offsets, uint32_t* status, void* workspace, size_t workspace_bytes,
                 void* stream);
/* gsb_bin_emit without `keys`, with the tile ranges taken from the last sort
 * pass (same workspace size; same binned_ids and tile_offsets): that pass
 * records each tile's first pair position instead of writing the sorted tile
 * keys, and a short kernel turns them into offsets. It saves 8 bytes of
 * traffic per pair against a fixed cost per tile, so it pays for many pairs
 * per tile (this library's host runtime uses it from 64 on average). No
 * reference counterpart of its own. */
int gsb_bin_emit_ranges(const gsb_raster_meta* meta, const float* rec, const int32_t* pair_offsets,
                        const uint64_t* tile_masks, int64_t total_pairs, int32_t* binned_ids,
                        int32_t* tile_offsets, uint32_t* status, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Max pairs over tiles -> status[GSB_STATUS_MAX_TILE_COUNT] (overflow check of
 * variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:756-760). */
int gsb_tile_stats(const gsb_raster_meta* meta, const int32_t* tile_offsets, uint32_t* status,
                   void* stream);

/* ---- compositing ---------------------------------------------------------
 * Workspace of gsb_render_forward / gsb_render_backward: now 0 bytes (short
 * tiles get a warp each; the kernel for long tiles finds them itself). The
 * workspace arguments are kept for ABI stability and may be NULL. */
size_t gsb_render_workspace_size(const gsb_raster_meta* meta);

/* Replaces `tile_fast_forward_eval` / `tile_fast_forward_state`
 * (…/gsplat_v8_project3d_kernels.metal:783-929; root csrc/metal/gsplat_fast_kernels.metal:221-294).
 * Training state: final_T, last_idx and pair_rec [P*12] (the records of each
 * short tile in list order, read back by the backward) are all given, or all
 * NULL (eval). */
int gsb_render_forward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                       const int32_t* binned_ids, float* out_rgb, float* final_T,
                       int32_t* last_idx, float* pair_rec, uint32_t* status, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Replaces `tile_fast_backward_saved` (…/gsplat_v8_project3d_kernels.metal:931-1063; root
 * csrc/metal/gsplat_fast_kernels.metal:296-395). Zeroes and accumulates grad_rec [B*G*12].
 * pair_rec must be 16-byte aligned (its tiles are staged with 16-byte asynchronous copies). */
int gsb_render_backward(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                        const int32_t* binned_ids, const float* final_T, const int32_t* last_idx,
                        const float* pair_rec, const float* grad_rgb, float* grad_rec, uint32_t* status,
                        void* workspace, size_t workspace_bytes, void* stream);

/* gsb_render_backward with the un-sort folded into its atomics (no reference
 * counterpart of its own): each splat's gradients are added straight at its
 * input position (view b, index perm[r] of rank r), so no grad_rec and no
 * gsb_unsort_grads launch are needed. The outputs must be zeroed by the
 * caller; any output pointer may be NULL (that gradient is skipped). The
 * permuted targets cost the atomics more L2 traffic, so it pays for large
 * splat counts (this library's host runtime uses it from 2^18 splats). */
int gsb_render_backward_inputs(const gsb_raster_meta* meta, const float* rec, const int32_t* tile_offsets,
                               const int32_t* binned_ids, const float* final_T, const int32_t* last_idx,
                               const float* pair_rec, const float* grad_rgb, const int32_t* perm,
                               float* g_means2d, float* g_conics, float* g_colors, float* g_opacities,
                               uint32_t* status, void* stream);

/* Replaces the un-sort scatter of the autograd backward
 * (torch_gsplat_bridge_fast/rasterize.py:96-105; …/v8_project3d/…/rasterize.py:583-591, 847-851).
 * Any output pointer may be NULL (that gradient is skipped). */
int gsb_unsort_grads(const gsb_raster_meta* meta, const int32_t* perm, const float* grad_rec,
                     float* g_means2d, float* g_conics, float* g_colors, float* g_opacities,
                     void* stream);

/* ---- pinhole projection --------------------------------------------------
 * Replaces `project_pinhole_forward` (…/gsplat_v8_project3d_kernels.metal:66-174).
 * camera_to_world [B,4,4] row-major, camera_params [B,4] = (fx, fy, cx, cy). */
int gsb_project_forward(int32_t batch_size, int32_t gaussians_per_batch, const float* means3d,
                        const float* scales, const float* quats, const float* opacities,
                        const float* camera_to_world, const float* camera_params, float near_plane,
                        float* out_means2d, float* out_conics, float* out_opacities,
                        float* out_depths, void* stream);

/* Replaces `project_pinhole_backward` (…/gsplat_v8_project3d_kernels.metal:217-501).
 * Any incoming gradient pointer may be NULL (treated as zeros). g_camera_to_world [B,16]
 * and g_camera_params [B,4] are zeroed and accumulated. */
int gsb_project_backward(int32_t batch_size, int32_t gaussians_per_batch,
                         const float* grad_means2d, const float* grad_conics,
                         const float* grad_opacities, const float* grad_depths,
                         const float* means3d, const float* scales, const float* quats,
                         const float* opacities, const float* camera_to_world,
                         const float* camera_params, float near_plane, float* g_means3d,
                         float* g_scales, float* g_quats, float* g_opacities,
                         float* g_camera_to_world, float* g_camera_params, void* stream);

/* ---- spherical-harmonic colours -------------------------------------------
 * No reference counterpart: the reference takes raw RGB colours
 * (variants/v8_project3d/torch_gsplat_bridge_v8_project3d/rasterize.py:958-1003). These
 * turn per-Gaussian real-SH coefficients sh_coeffs [G, (degree+1)^2, 3] (degree 0-3,
 * shared by all views) into colours [B, G, 3] for each camera:
 *   colour = max(0, 0.5 + sum_k coeff_k Y_k(normalize(mean - camera centre))),
 * the camera centre being column 3 of the row-major camera_to_world [B,4,4].
 * The backward takes the forward's colours (for the clamp) and writes
 * g_sh_coeffs [G,K,3], g_means3d [G,3] (optional, the SH term only) and
 * g_camera_to_world [B,16] (optional; only the centre column is nonzero). */
int gsb_sh_forward(int32_t batch_size, int32_t gaussians, int32_t degree, const float* sh_coeffs,
                   const float* means3d, const float* camera_to_world, float* colors, void* stream);
int gsb_sh_backward(int32_t batch_size, int32_t gaussians, int32_t degree, const float* sh_coeffs,
                    const float* means3d, const float* camera_to_world, const float* colors,
                    const float* grad_colors, float* g_sh_coeffs, float* g_means3d,
                    float* g_camera_to_world, void* stream);

/* ---- multi-GPU: gradient sum over NVLink peer memory -----------------------
 * No counterpart in the reference, which is single-device. Sums a float buffer
 * across the ranks of one node in place, replacing the NCCL all-reduce of the
 * shared-Gaussian gradients. Each rank owns one peer buffer: GSB_PEER_FLAG_BYTES
 * of barrier flags followed by the data. The buffer is exported with a
 * GSB_PEER_HANDLE_BYTES CUDA IPC handle and mapped by every other rank, which
 * passes all ranks' base pointers in rank order. */
#define GSB_PEER_MAX_RANKS 8
#define GSB_PEER_FLAG_BYTES 256
#define GSB_PEER_HANDLE_BYTES 64
/* cudaMalloc of GSB_PEER_FLAG_BYTES + data_bytes on the current device, flags zeroed. */
int gsb_peer_buffer_alloc(size_t data_bytes, void** base);
int gsb_peer_buffer_free(void* base);
/* IPC handle of a buffer from gsb_peer_buffer_alloc; a peer process maps it with gsb_peer_open. */
int gsb_peer_handle(const void* base, void* handle);
int gsb_peer_open(const void* handle, void** base);
int gsb_peer_close(void* base);
/* bases[r] = rank r's buffer as mapped in this process (bases[rank] = own).
 * Sums data[0 .. n_floats) over all ranks and leaves the sum in every rank's
 * buffer. One kernel: a start barrier (every rank's data is final), rank r
 * adds shard r of all buffers over NVLink and stores the sum into all of them,
 * then an end barrier. Every rank calls it with the same n_floats and epoch;
 * epoch counts the calls from 1 and grows by one per call. Each barrier wait is
 * bounded by wait_ns nanoseconds (0: 10 s). A rank whose wait runs out, that
 * finds a peer already at a later epoch, or that finds a peer's abort mark for
 * this epoch, gives up the call: it marks its abort in every peer's buffer,
 * raises GSB_DEVERR_PEER_TIMEOUT in status[GSB_STATUS_ERROR] and returns. After
 * a call that raised it, the buffer's contents are undefined on every rank that
 * reports it, and the group must not call again. */
int gsb_peer_allreduce_sum(int32_t rank, int32_t world, void* const* bases, int64_t n_floats, uint32_t epoch,
                           uint64_t wait_ns, uint32_t* status, void* stream);

/* ---- building blocks, exported for parity tests -------------------------
 * Stable LSD radix sort of (uint64 key, uint32 value) pairs on key bits
 * [begin_bit, end_bit) (onesweep: one histogram pass + one pass per 8-bit digit).
 * keys_in/vals_in are read only; the result lands in keys_out/vals_out. */
size_t gsb_radix_sort_pairs_workspace_size(int64_t n, int begin_bit, int end_bit);
int gsb_radix_sort_pairs(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                         uint32_t* vals_out, int64_t n, int begin_bit, int end_bit,
                         uint32_t* status, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free variant of gsb_radix_sort_pairs. It has no counterpart in the
 * reference. Some callers cannot allocate device memory: a host application that
 * budgets all GPU memory itself and gives a plugin only the buffers of each call,
 * or a loop that must not reach cudaFree, which synchronizes the device. This
 * entry point takes no workspace and allocates nothing: its scratch is a fixed
 * array of GSB_SORT_NOALLOC_SCRATCH_BYTES inside the library, which every GPU
 * that loads the library holds until the process exits. Sorts of more than
 * GSB_SORT_NOALLOC_MAX_PAIRS pairs are refused with GSB_ERR_CAPACITY.
 *
 * The first call on a device looks up that device's address of the array (a
 * cudaGetSymbolAddress call, made with that device current); make that first
 * call before any stream capture. All calls on a device share the one array,
 * and each call clears the parts that must start at zero, so calls that can
 * overlap on the GPU (on different streams, or from different host threads
 * without ordering) race and corrupt each other: order them on one stream.
 * Same arguments and results as gsb_radix_sort_pairs otherwise. */
#define GSB_SORT_NOALLOC_MAX_PAIRS 262144
#define GSB_SORT_NOALLOC_SCRATCH_BYTES (6u << 20)
int gsb_radix_sort_pairs_noalloc(const uint64_t* keys_in, const uint32_t* vals_in, uint64_t* keys_out,
                                 uint32_t* vals_out, int64_t n, int begin_bit, int end_bit, uint32_t* status,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GSPLAT_B200_H */
