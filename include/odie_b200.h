/*
 * odie_b200 C-ABI: the drop-in boundary of the ODIE hot path on B200 (sm_100a).
 *
 * Plain C types only.  Every pointer argument is a device pointer unless its
 * name ends in _host; `stream` is a cudaStream_t passed as uint64.  Integer
 * returns are 0 on success; on failure they are -1 (runtime calls, with the
 * message in odie_error()) or a nonzero cudaError_t (selection/residual calls,
 * as in the reference).  Each entry point cites the reference interface it
 * replaces (paths relative to the ODIE project root).
 */
#ifndef ODIE_B200_H
#define ODIE_B200_H
#include <stdbool.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ODIE_API __attribute__((visibility("default")))
#else
#define ODIE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------
 * Native training runtime.  Replaces odie/native/runtime.cu:318-331 (the
 * odie_* symbols bound by odie/native_backend.py:32-44) with the same JSON
 * contract (odie/native_backend.py:50-59), plus the keys that the reference
 * bakes in at compile time (odie/build.py:26-30): "levels", "raw_width",
 * "router", "gate_k", "softplus", "rgb8", and "batch" (maximum coordinates per
 * step; the reference fixes 65536).
 * "mode" takes the reference's bits (1 fused target, 4 half-precision grid
 * gradients, 8 dirty-tile clearing, 16 parallel gate) and rejects others:
 * targets are always read in the input kernel and the gate always runs fused in
 * the heads kernel; grid gradients are always fp32 and Adam clears the entries
 * it consumed, so bits 4 and 8 select nothing further ("half_grad" and
 * "output" in odie_pointers are 0; "grid_gradient_precision" is "fp32").
 * Routed experts (no reference counterpart): "experts" (1..64 tables held)
 * with "hash_encoding" (one expert's grid; "grid" holds experts x its
 * parameters, expert-major), "router_encoding" (the coarse shared grid; fp32
 * master in "router_grid") and "gate" (router MLP W1 | W2 | W3 with
 * router_out = 16 (up to 16 model experts) or 64 logit rows, fp32 master,
 * "gate_lr").  Spatial expert ownership: "bands" (rows of the full image cut
 * into this many equal bands, default 1), "experts_per_band" (8 or 16 when
 * bands > 1; default: experts), "first_band" (the first band held here,
 * default 0): band b owns the model's experts [b * per, (b + 1) * per) and a
 * coordinate chooses among its band's experts only.  "full_height" and
 * "row_offset" (defaults: height, 0) place this image's rows in the full
 * image, whose rows the coordinates use.  "router_grad" (optional, device
 * f32[router grid params], zeroed here): a caller-owned router-grid gradient
 * (a router grid shared across ranks); its update then runs in
 * odie_step_heads, after the caller has summed it.
 * ------------------------------------------------------------------------ */
/* Thread-local message of the last failure. runtime.cu:320 */
ODIE_API const char* odie_error(void);
/* Kernels this library has launched since it was loaded, all threads and
 * devices (no reference counterpart; read before and after a region to count
 * its launches). */
ODIE_API long long odie_launch_count(void);
/* Create a runtime for one stream; NULL on failure. runtime.cu:321 */
ODIE_API void* odie_create(const char* json);
/* One fwd/bwd(/Adam when update) step over n int64 pixel ids. runtime.cu:322 */
ODIE_API int odie_step(void* handle, uint64_t ids, int n, int update);
/* JSON of internal device buffers ("squares", "grid_grad", "head_grad", ...). runtime.cu:323
 * "scatter_strategy": two device ints, the strategy the last step's router-grid
 * and main grid scatters chose from the batch (0: per-block shared-memory
 * tables, 1: global reductions for spatially coherent batches). */
ODIE_API const char* odie_pointers(void* handle);
/* {"pristine": bool} for a grid range, or {"hash_fnv1a64", "bytes"} of all
 * optimizer state when begin < 0. runtime.cu:324 */
ODIE_API const char* odie_state(void* handle, int begin, int end);
/* Change active prefix, layout pointers and learning rates. runtime.cu:325 */
ODIE_API int odie_configure(void* handle, const char* json);
/* No TCNN contexts exist here; kept for the binding. runtime.cu:326,328 */
ODIE_API void odie_release_contexts(void* handle);
ODIE_API void odie_pin_contexts(void* handle);
/* Refresh every fp16 copy from the caller's fp32 masters. runtime.cu:327 */
ODIE_API int odie_sync_weights(void* handle);
/* cudaMemcpyAsync device-to-device. runtime.cu:329 */
ODIE_API int odie_copy(uint64_t dst, uint64_t src, uint64_t bytes, uint64_t stream);
/* Destroy the runtime. runtime.cu:330 */
ODIE_API void odie_destroy(void* handle);

/* Split step for data-parallel training (no reference counterpart; the
 * reference is single-GPU): odie_step_grads runs the forward/backward, the
 * grid update (when update) and leaves the summed fp32 head gradient in the
 * "head_grad" buffer; the caller all-reduces it; odie_step_heads applies the
 * head update.  odie_step == odie_step_grads + odie_step_heads.  update: 0
 * discards the gradients, 1 applies the grid update, 2 keeps the fp32 grid
 * gradient ("grid_grad", loss scale 128) for inspection; odie_grid_update then
 * applies the grid update to it. */
ODIE_API int odie_step_grads(void* handle, uint64_t ids, int n, int update);
ODIE_API int odie_step_heads(void* handle);
ODIE_API int odie_grid_update(void* handle);

/* Pipeline mode (no reference counterpart): with "pipeline": 1 in the create
 * JSON (routed experts, library-owned head and router-grid gradients: one
 * GPU), odie_step / odie_step_stratified with update return while the step's
 * backward branches (router-grid scatter and the router grid's and heads'
 * Adam; expert-table scatter and the expert tables' Adam) still run on the
 * runtime's own streams; the next step's forward overlaps them as far as its
 * data allow.  The step's loss ("squares") is ready in stream order as usual;
 * the parameters are final once the runtime's stream has passed odie_join (or
 * any other call on the handle, each of which joins first).  "xy", "target"
 * and "expert_ids" of odie_pointers then alternate between two buffers.
 * odie_join: the runtime's stream waits for those branches (a no-op outside
 * pipeline mode). */
ODIE_API int odie_join(void* handle);

/* Stratified batches on the device (replaces the reference's per-step sampler,
 * odie/data.py:63-80, stratified_batches, which draws torch.rand and then
 * gathers targets in separate kernels): slot j of step `step` takes stratum
 * (j mod side, j / side), side = sqrt(n), and offsets r = (word >> 8) 2^-24
 * from a Philox4x32-10 stream (key = seed, counter = (j, step));
 * uv = r / side + stratum / side in fp32; pixel = trunc(uv (W, H)) clamped;
 * id = y W + x.  n must be a square power of two, as in the reference.
 * odie_stratified_ids writes the n int64 ids; odie_step_stratified is
 * odie_step on the batch of (seed, step), with the sampler fused into the
 * step's input kernel (ids -> coordinates and targets). */
ODIE_API int odie_stratified_ids(uint64_t seed, uint64_t step, int width, int height, int64_t n, int64_t* ids,
                   uint64_t stream);
ODIE_API int odie_step_stratified(void* handle, uint64_t seed, uint64_t step, int n, int update);

/* Stage timers (no reference counterpart): enable (1) / disable (0) CUDA-event
 * timing of every stage launch on the stream it runs on (resets the record), or
 * enable with the step's concurrent branches run one after the other on the
 * runtime's stream (2), so that each stage's time is its kernels' own; and a
 * JSON report {stage: {"launches": k, "ms": total}} of what was recorded. */
ODIE_API int odie_profile(void* handle, int enable);
ODIE_API const char* odie_profile_report(void* handle);

/* Full-image decode of pixel ids [begin, begin+n) through the model: fp32 RGB
 * [n][3] and/or uint8 RGB rint(clip(x,0,1)*255) (scripts/reconstruct.py:39-44,
 * odie/evaluation.py:12-36; either output may be NULL). */
ODIE_API int odie_decode(void* handle, int64_t begin, int64_t n, float* rgb, uint8_t* rgb8);

/* ------------------------------------------------------------------------
 * Packed-plane query.  Replaces the pybind extension odie/packed_bindings.cpp:4-12
 * (packed_forward_cuda / packed_backward_cuda, odie/packed_kernels.cu:107-145).
 * coords f32[n][2]; grid f32[P]; descriptors i32[levels][8]; node_bitmap
 * u64[words]; node_prefix i32[words]; bitmap u8[bytes].
 * ------------------------------------------------------------------------ */
/* features f16 bits [n][width], visible u8 [n][levels]. packed_kernels.cu:107-125 */
ODIE_API int odie_query_forward(const float* coords, int64_t n, const float* grid, const int32_t* descriptors, int levels,
                       const uint64_t* node_bitmap, const int32_t* node_prefix, const uint8_t* bitmap, int width,
                       uint16_t* features, uint8_t* visible, uint64_t stream);
/* gradient f32[parameter_count], zeroed then scatter-added. packed_kernels.cu:127-145 */
ODIE_API int odie_query_backward(const float* coords, int64_t n, const uint16_t* upstream, int width,
                        const int32_t* descriptors, int levels, const uint64_t* node_bitmap,
                        const int32_t* node_prefix, const uint8_t* bitmap, float* gradient,
                        int64_t parameter_count, uint64_t stream);

/* ------------------------------------------------------------------------
 * Hashed multiresolution grid (the TCNN HashGrid encoding used by
 * odie/hash_grid.py:27-34 and odie/native/runtime.cu:184-193,260,287; TCNN is
 * not vendored in the reference).  Level table on the host.
 * ------------------------------------------------------------------------ */
typedef struct {
    float scale;          /* fp32 grid scale of odie/config.py:92 */
    int32_t resolution;   /* ceil(scale) + 1 */
    int32_t capacity;     /* table entries: min(align8(resolution^2), 2^log2_hashmap_size) */
    int32_t offset;       /* first parameter of the level */
    int32_t features;     /* features per entry */
    int32_t column;       /* first output column */
    int32_t hashed;       /* 1: spatial hash, 0: dense x + y*resolution (both modulo capacity) */
    int32_t cells;        /* byte offset of the level's cell-visibility bitmap (routed-expert calls that take
                             a bitmap), -1: every cell visible; odie_hash_forward/backward need -1 */
} odie_hash_level;
ODIE_API int odie_hash_forward(const float* coords, int64_t n, const float* table, const odie_hash_level* levels_host,
                      int levels, int width, uint16_t* features, uint64_t stream);
ODIE_API int odie_hash_backward(const float* coords, int64_t n, const uint16_t* upstream, int width,
                       const odie_hash_level* levels_host, int levels, float* gradient, int64_t parameter_count,
                       uint64_t stream);

/* ------------------------------------------------------------------------
 * Live residual scoring.  Replaces odie/residual_cuda.cu:45-52 (same arguments).
 * ------------------------------------------------------------------------ */
ODIE_API int score_chunk(const float* prediction, const void* target, int64_t begin, int64_t end, int width, int resolution,
                int first_y, int active_cells, const int* xb, const int* yb, double* totals, bool rgb8,
                uint64_t stream);

/* ------------------------------------------------------------------------
 * Exact greedy selection.  Replaces odie/native/selection_cuda.cu:208-230
 * (same arguments and buffer sizes, bound at odie/selection_cuda.py:43-46).
 * ------------------------------------------------------------------------ */
ODIE_API int selection_init(const double* scores, int n, int points, int* missing, uint8_t* chosen, uint8_t* nodes, int* tree,
                   int64_t* stats, const int* host_offsets, const int* host_sizes, int levels, uint64_t stream);
ODIE_API int selection_chunk(const double* scores, int n, int points, int resolution, int cap, bool normalized, int* missing,
                    uint8_t* chosen, uint8_t* nodes, int* tree, const int* offsets, const int* sizes, int levels,
                    int chunk, int64_t* stats, int* trace, uint64_t stream);

/* ------------------------------------------------------------------------
 * Routed multi-expert encoding (no reference counterpart).
 * odie_router_forward_banded: features f16[n][width] (width 16 or 32,
 * row-major), xy f32[n][2] (read when bands > 1: the band of a coordinate is
 * floor(row * bands / rows) with row = rint(y * (rows - 1))), weights
 * f16 [32*width | 32*32 | OUT*32] (router W1, W2, W3, row-major [out][in];
 * OUT = 16 for up to 16 model experts (bands x experts_per_band), else 64).
 * Writes expert i32[n] (local number: (band - first_band) * experts_per_band
 * + the first maximum of the fp16 logits of the band's experts), prob f32[n]
 * (softmax probability of that expert over its band's) and, when logits is
 * non-NULL, f16[n][live] (the band's logits; live 8 or 16, >= experts_per_band,
 * zero padded).  Bit-exact: fp32 fma chains in input order.
 * odie_router_forward: the unbanded form (experts 1..16, logits f16[n][16]).
 * odie_expert_hash_forward/backward: odie_hash_forward/backward with one table
 * per expert; coordinate i uses the table starting expert[i] * expert_stride
 * parameters into `tables` / `gradient` (same level records for every expert).
 * bitmap (may be NULL): cell-visibility bytes of the on-demand allocation,
 * addressed by each level's `cells` offset; a hidden cell gives zero features
 * and receives no gradient.
 * ------------------------------------------------------------------------ */
ODIE_API int odie_router_forward(const uint16_t* features, int64_t n, int width, const uint16_t* weights, int experts,
                   int32_t* expert, float* prob, uint16_t* logits, uint64_t stream);
ODIE_API int odie_router_forward_banded(const uint16_t* features, const float* xy, int64_t n, int width,
                   const uint16_t* weights, int experts, int bands, int first_band, int experts_per_band, int rows,
                   int32_t* expert, float* prob, uint16_t* logits, int live, uint64_t stream);
ODIE_API int odie_expert_hash_forward(const float* coords, int64_t n, const float* tables, int64_t expert_stride,
                   const int32_t* expert, const odie_hash_level* levels, int level_count, int width,
                   const uint8_t* bitmap, uint16_t* features, uint64_t stream);
ODIE_API int odie_expert_hash_backward(const float* coords, int64_t n, const uint16_t* upstream, int width,
                   int64_t expert_stride, const int32_t* expert, const odie_hash_level* levels, int level_count,
                   const uint8_t* bitmap, float* gradient, int64_t parameter_count, uint64_t stream);

/* ------------------------------------------------------------------------
 * On-device packed-plane index of one level (replaces the host-side
 * plane_closure / make_node_index / cell bitmap of odie/model.py:36-61,108-110,
 * rebuilt at every stage boundary).  support: R*R bytes (0/1, a torch bool
 * tensor), points = align8(R^2).  Writes node_bitmap u64[ceil(points/64)]
 * (closure presence, bit b of word w = node 64w+b), node_prefix
 * i32[ceil(points/64)] (exclusive popcount prefix), cell_bitmap u8[points/8]
 * (LSB-first cell bits), *node_count (closure size, device int64) and, when
 * nodes is non-NULL, the sorted closure i64[node count] (capacity points).
 * scratch: i32[odie_plane_index_scratch(R)], caller-owned.  Returns -1 with
 * odie_error() on invalid sizes.
 * ------------------------------------------------------------------------ */
ODIE_API int64_t odie_plane_index_scratch(int resolution);
ODIE_API int odie_plane_index(const uint8_t* support, int resolution, uint64_t* node_bitmap, int32_t* node_prefix,
                   uint8_t* cell_bitmap, int64_t* node_count, int64_t* nodes, int32_t* scratch, uint64_t stream);

/* ------------------------------------------------------------------------
 * On-demand allocation of routed experts (the allocation benchmark; no reference
 * counterpart): the cell-visibility bitmap of one hash level (resolution R,
 * ceil(R^2 / 8) bytes, LSB-first) from an allocated-tile mask tiles
 * u8[tiles_y][tiles_x] of tile_px x tile_px tiles over a height x width image:
 * cell (ix, iy) is visible iff the pixel nearest its centre, column
 * floor(ix (width - 1) / (R - 1) + 1/2) and row likewise, lies in an allocated
 * tile.
 * ------------------------------------------------------------------------ */
ODIE_API int odie_allocation_bitmap(const uint8_t* tiles, int tiles_x, int tiles_y, int tile_px, int height, int width,
                   int resolution, uint8_t* bitmap, uint64_t stream);

/* ------------------------------------------------------------------------
 * L2 probe (measurement; no reference counterpart): `operations` random
 * accesses over `table` (table_bytes in 4 KiB..64 MiB, so it stays in L2):
 * mode 0 = 4-byte loads, 1 = 16-byte loads, 2 = 4-byte fp32 reductions,
 * 3 = 8-byte fp32x2 reductions (each adds 1e-30).  sink: one float, written
 * only to keep the loads alive.  Time it with CUDA events on `stream`.
 * ------------------------------------------------------------------------ */
ODIE_API int odie_l2_probe(float* table, int64_t table_bytes, int mode, int64_t operations, float* sink,
                   uint64_t stream);

/* Failure-detection check (no reference counterpart): one block waits on an
 * mbarrier that nothing completes, with the bounded wait the fused heads
 * kernel uses, giving up after `limit` polls (1..2^20).  *status (device
 * int32) = 2 when the wait ran out -- the code the heads kernel leaves in
 * its error flag -- and 0 if it completed.  The context stays usable. */
ODIE_API int odie_wait_probe(uint32_t limit, int32_t* status, uint64_t stream);
/* fp32 FMA throughput probe (no reference counterpart): one launch of 8 x SMs blocks of 256 threads, each
 * running 8 independent fma chains of `iterations` steps; returns the launch's FLOP (-1 on bad input).
 * The caller times it: the roofline denominator of the fp32 CUDA-core MLP. */
ODIE_API int64_t odie_fma_probe(int iterations, float* sink, uint64_t stream);

/* ------------------------------------------------------------------------
 * Tile top-k allocation (the allocation benchmark; no reference counterpart).
 * prediction f32[H*W][3], target u8[H*W][3]; row_sums f64[tiles*tile] scratch;
 * scores f64[tiles]; chosen i64[k] (tile ids by rank); selected u8[tiles].
 * ------------------------------------------------------------------------ */
ODIE_API int odie_tile_topk(const float* prediction, const uint8_t* target, int height, int width, int tile, int k,
                   double* row_sums, double* scores, int64_t* chosen, uint8_t* selected, uint64_t stream);
/* The exact top-k alone: chosen i64[k] = the k highest of scores f64[count] by
 * (score descending, index ascending), selected u8[count] (1 for those).  For
 * tile scores gathered from several ranks before one global choice.  Requires
 * 0 <= k <= count (else cudaErrorInvalidValue with a message). */
ODIE_API int odie_topk(const double* scores, int count, int k, int64_t* chosen, uint8_t* selected, uint64_t stream);

/* ------------------------------------------------------------------------
 * Procedural gigapixel test image (benchmark input; no reference counterpart).
 * Writes rows [row0, row0 + rows) of a height x width u8 RGB image into
 * rgb u8[rows][width][3]: seeded fractal value noise with a 1/f^2 spectrum,
 * Voronoi regions with sharp borders and a 64 x 64-cell atlas of patterns.
 * Each pixel depends only on (seed, column, row, width, height), so ranks that
 * draw their own bands draw one image.  -1 with odie_error() on bad rows.
 * ------------------------------------------------------------------------ */
ODIE_API int odie_procedural_image(uint64_t seed, int width, int height, int row0, int rows, uint8_t* rgb,
                   uint64_t stream);

/* ------------------------------------------------------------------------
 * Single fp32 hash grid with an fp32 MLP (the hash-grid encoding of
 * odie/hash_grid.py:8-80 with the layout of odie/config.py:83-94, in fp32:
 * 16 levels x 2 features, MLP 32 -> 64 -> 64 -> 3, no biases, ReLU hidden
 * layers, sigmoid output).
 * odie_hashgrid32_create: JSON {"image": ptr f32[height][width][3],
 * "width", "height", "grid": ptr f32[total], "heads": ptr f32[6336]
 * (W1 [64][32] | W2 [64][64] | W3 [3][64], row-major [out][in]),
 * "hash_encoding": {n_levels 16, n_features_per_level 2, log2_hashmap_size,
 * base_resolution, per_level_scale}, optional "total" (checked), "capacity"
 * (largest batch, default 2^18), "grid_lr", "head_lr" (1e-2), "beta1" (0.9),
 * "beta2" (0.99), "eps" (1e-15)}.  Image, grid and heads stay caller-owned;
 * Adam updates grid and heads in place.  NULL with odie_error() on bad input.
 * odie_hashgrid32_step: one step on n coordinates: xy f32[n][2] on the device,
 * or NULL for uniform coordinates in [0, 1)^2 drawn from Philox4x32-10 (key
 * seed, counter (slot, step); x = (word0 >> 8) 2^-24, y = (word1 >> 8) 2^-24).
 * Targets are the image bilinearly sampled at the coordinates; loss = mean
 * of the 3 n squared errors.  update = 0 computes the gradients only
 * (grid_grad accumulates until an update consumes it).  Every call runs on the
 * stream it is given (0: the legacy default stream).
 * odie_hashgrid32_update: the Adam update alone on the accumulated gradients.
 * odie_hashgrid32_decode: fp32 RGB rgb[n][3] at xy f32[n][2], or at the pixel
 * centres (col / (W - 1), row / (H - 1)) of pixels [begin, begin + n) when
 * xy is NULL.
 * odie_hashgrid32_pointers: JSON with the library-owned device buffers
 * (grid_grad, head_grad, moments, steps, xy, dx, squares, error_flag), the
 * handle's stream and the sizes.
 * ------------------------------------------------------------------------ */
ODIE_API void* odie_hashgrid32_create(const char* json);
ODIE_API int odie_hashgrid32_step(void* handle, uint64_t seed, uint64_t step, int64_t n, const float* xy, int update,
                   uint64_t stream);
ODIE_API int odie_hashgrid32_update(void* handle, uint64_t stream);
ODIE_API int odie_hashgrid32_decode(void* handle, int64_t begin, int64_t n, const float* xy, float* rgb,
                   uint64_t stream);
ODIE_API const char* odie_hashgrid32_pointers(void* handle);
/* Stage timers of the steps (CUDA events on the step's stream): enable 1 / disable 0 (resets the record);
 * report {stage: {"launches": k, "ms": total}} for fused_step, encode_backward, reduce_partials, adam_grid,
 * adam_heads. */
ODIE_API int odie_hashgrid32_profile(void* handle, int enable);
ODIE_API const char* odie_hashgrid32_profile_report(void* handle);
ODIE_API void odie_hashgrid32_destroy(void* handle);

/* ------------------------------------------------------------------------
 * Allocation-free tile top-k (no counterpart in the reference).
 * Same arguments and results as odie_tile_topk minus row_sums: the row sums
 * live in a fixed 2 MiB array inside this library (262144 f64 entries), so the
 * call allocates no device memory.  It is for callers that may not allocate at
 * all: a host whose device memory is owned by another allocator or held to a
 * hard budget, and code running where an allocation would synchronise the
 * device or is forbidden.  tiles * tile above 262144 returns
 * cudaErrorInvalidValue with a message in odie_error().  The first call on each
 * device looks up the array's device address (cudaGetSymbolAddress); make that
 * first call before any stream capture.  The address is kept for the
 * process: after a cudaDeviceReset of that device, do not call this entry
 * point there.  tile must not exceed max(height, width).  All calls on one
 * device share the
 * array: calls that can overlap on the GPU (different streams, or several host
 * threads) race and must be serialised by the caller.
 * ------------------------------------------------------------------------ */
ODIE_API int odie_tile_topk_noalloc(const float* prediction, const uint8_t* target, int height, int width, int tile,
                   int k, double* scores, int64_t* chosen, uint8_t* selected, uint64_t stream);

#ifdef __cplusplus
}
#endif
#endif
