// Training/decoding step kernels (step.cu).
#pragma once
#include "common.cuh"

namespace odie {

// Head network shapes (the reference's TCNN FullyFusedMLP heads,
// odie/native/runtime.cu:155-157, odie/model.py:186-188): no biases, ReLU hidden
// layers, linear output, fp16 weights with fp32 masters, parameters row-major
// [out][in] per layer in the order gate W1, gate W2 | decoder W1, W2, W3.
constexpr int GATE_HIDDEN = 32, GATE_OUT = 16, DEC_HIDDEN = 64, DEC_OUT = 16;
__host__ __device__ constexpr int gate_params(int w) { return GATE_HIDDEN * w + GATE_OUT * GATE_HIDDEN; }
__host__ __device__ constexpr int decoder_params(int w) { return DEC_HIDDEN * w + DEC_HIDDEN * DEC_HIDDEN + DEC_OUT * DEC_HIDDEN; }

struct FeatureMap {
    int8_t level_of_col[64];  // level of each decoder-input column, -1 for pad columns (constant 1)
    int8_t col_of_level[32];  // first column of each level
    int8_t dim_of_level[32];  // features of each level
};

// Gating of the decoder input: none, the reference's per-level gate
// (odie/native/runtime.cu:66-75), or a routed expert scaled by its router
// probability.
enum GateMode : int { GATE_NONE = 0, GATE_LEVELS = 1, GATE_EXPERTS = 2 };

struct MlpArgs {
    long long n;          // coordinates of this launch
    long long stride;     // pair-major stride of raw/gvals and level stride of vis
    const __half* raw;    // [W/2][stride] half2 features, or [stride][W] rows when raw_rows
    bool raw_rows;
    const uint32_t* vis;  // bit-packed visibility [levels][stride / 32]
    const float* target;  // [n][3] fp32 (training) or nullptr
    const __half* gate_w;     // fp16 gate weights (may be null without router)
    const __half* decoder_w;  // fp16 decoder weights
    int levels, raw_width, k_fixed, softplus;
    float three_real;     // fp32(3 * real) of the loss gradient
    FeatureMap fmap;
    __half* gvals;        // [stride][W] grid-gradient values, row-major (training)
    float* squares;       // [n] per-sample mean-RGB squared error (training)
    float* partials;      // [gridDim.x][head params] weight-gradient partials (training)
    float* rgb;           // [n][3] fp32 decode output (decode)
    uint8_t* rgb8;        // [n][3] u8 decode output (decode)
    // GATE_EXPERTS: raw holds the routed expert's features; gate_w the router weights
    const __half* router_in;  // [stride][W] row-major router-grid features
    const float* prob;        // [n] router probability of the chosen expert
    const int* expert;        // [n] chosen expert
    __half* router_gvals;     // [stride][W] router-grid gradient values, row-major (training)
    int experts;              // expert tables held here
    const __half* logits;     // [stride][live] fp16 logits of each coordinate's live experts (training)
    int live;                 // logits row width: 8 or 16
    // spatial expert ownership (router.cuh Banding): a coordinate's live logit columns are
    // [band * per_band, (band + 1) * per_band) with band = first_band + expert / per_band
    int per_band, first_band;
    int model_experts;        // experts of the whole model (the router's logit rows before padding)
};

// tcgen05/TMEM fused heads (mlp_tc.cu), decoder input width 16 or 32.  uniform:
// every level has 2 features at columns (2l, 2l+1).  vis is bit-packed
// [levels][stride / 32]; stride is a multiple of 128.  A wait that runs out
// sets *error_flag = 2 and the kernel returns.
int mlp_tc_blocks(long long n);
// CTAs of a training launch (the weight-gradient partials it writes): at most mlp_tc_blocks(n).
int mlp_tc_train_blocks(long long n, GateMode gate);
void launch_mlp_tc_train(const MlpArgs& args, int width, GateMode gate, bool uniform, int blocks, int* error_flag,
                         cudaStream_t stream);
void launch_mlp_tc_decode(const MlpArgs& args, int width, GateMode gate, bool uniform, int* error_flag,
                          cudaStream_t stream);

// Image rows seen by the coordinates: the local image (height rows) is rows [row0, row0 + height) of a full
// image of `rows` rows, and y = (row0 + local row) / (rows - 1) (row0 = 0, rows = height: the whole image).
struct RowFrame {
    int row0 = 0, rows = 0;
};
void launch_input_batch(const int64_t* ids, long long n, const uint8_t* rgb, bool rgb8, int width, int height,
                        RowFrame frame, float* xy, float* target, cudaStream_t stream);
void launch_coords_range(long long begin, long long n, int width, int height, RowFrame frame, float* xy,
                         cudaStream_t stream);
// Stratified pixel ids (the reference's sampler, odie/data.py:63-80, on a Philox4x32-10 stream keyed by
// seed, counter (slot, step)); n a square power of two.  The batch variant fuses the step's input stage.
void launch_stratified_ids(uint64_t seed, uint64_t step, int width, int height, long long n, int64_t* ids,
                           cudaStream_t stream);
void launch_stratified_batch(uint64_t seed, uint64_t step, long long n, const uint8_t* rgb, bool rgb8, int width,
                             int height, RowFrame frame, float* xy, float* target, cudaStream_t stream);

// Sum of the per-block weight-gradient partials in block order (deterministic).
void launch_reduce_partials(const float* partials, int blocks, int count, float* out, cudaStream_t stream);

struct AdamTables {
    const float* step_size;  // fp32(lr / (1 - beta1^s)) for s = 1..size (index s-1), evaluated in double
    const float* bc2_sqrt;   // fp32(sqrt(1 - beta2^s)), evaluated in double
    long long size;
};
// Adam over one parameter group with device-side per-parameter step counters
// (so a captured CUDA graph replays correct bias corrections).  skip_zero:
// entries whose gradient is exactly zero keep their state and step (the native
// grid optimizer, odie/native/runtime.cu:212-213); without it every entry steps
// (torch.optim.Adam on a dense tensor).  The gradient is consumed (zeroed) and
// the fp16 copy refreshed for every updated entry.
void launch_adam(float* master, __half* copy, float* m, float* v, uint32_t* steps, float* grad, long long count,
                 float inv_scale, AdamTables tables, float beta1w, float beta2, float beta2w, float eps, bool skip_zero,
                 int* error_flag, cudaStream_t stream);
// Two parameter groups with their own masters and learning-rate tables, one launch: group 1's copy,
// moments, steps and gradient follow group 0's in the same arrays (the heads: gate, then decoder).
void launch_adam2(float* master0, float* master1, __half* copy, float* m, float* v, uint32_t* steps, float* grad,
                  long long count0, long long count1, float inv_scale, AdamTables tables0, AdamTables tables1,
                  float beta1w, float beta2, float beta2w, float eps, bool skip_zero, int* error_flag,
                  cudaStream_t stream);
void launch_zero(float* p, long long count, cudaStream_t stream);
void launch_cast_half(const float* in, __half* out, long long count, cudaStream_t stream);

}  // namespace odie
