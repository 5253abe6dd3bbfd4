// Top-1 expert router (router.cu).
#pragma once
#include "common.cuh"

namespace odie {

// Router MLP shape: W -> 32 -> 32 -> OUT, ReLU hidden layers, linear logits, no biases;
// fp16 weights row-major [out][in] in the order W1, W2, W3.  OUT is 16 for up to 16
// experts and 64 for up to 64 (rows past the expert count are padding that no choice reads).
constexpr int ROUTER_HIDDEN = 32, ROUTER_MAX_OUT = 64, ROUTER_MAX_LIVE = 16;
__host__ __device__ constexpr int router_out(int experts) { return experts <= 16 ? 16 : ROUTER_MAX_OUT; }
__host__ __device__ constexpr int router_params(int w, int out) {
    return ROUTER_HIDDEN * w + ROUTER_HIDDEN * ROUTER_HIDDEN + out * ROUTER_HIDDEN;
}

// Spatial expert ownership.  The full image's rows are cut into `bands` equal bands (band of global row y:
// floor(y * bands / rows)); band b owns experts [b * per_band, (b + 1) * per_band) of the model (the router's
// logit rows), and a coordinate chooses only among its band's experts.  A rank that holds bands
// [first_band, first_band + experts / per_band) numbers its expert tables locally: local expert =
// (band - first_band) * per_band + choice.  bands = 1: every coordinate chooses among all experts.
struct Banding {
    int bands = 1, first_band = 0, per_band = 0;
    int rows = 0;  // full-image height: y = row / (rows - 1)
    __host__ __device__ int model_experts() const { return bands * per_band; }
};

struct RouterArgs {
    const __half* features = nullptr;  // router-grid features: pair-major [W/2][stride] half2, or row-major [n][W]
    long long stride = 0;
    bool row_major = false;
    long long n = 0;
    const __half* weights = nullptr;   // fp16 [router_params(W, router_out(banding.model_experts()))]
    int experts = 0;                   // expert tables held here (local numbering)
    Banding banding;
    const float* xy = nullptr;         // [n][2] coordinates (banded routing only: the band comes from y)
    int* expert = nullptr;             // [n] chosen expert (local numbering)
    float* prob = nullptr;             // [n] softmax probability of the chosen expert over its band's experts
    __half* logits = nullptr;          // optional [n][live] fp16 logits of the coordinate's live experts
    int live = 0;                      // logits row width: 8 or 16 (>= per_band)
};

// Band of a coordinate, clamped to the bands held here.  The global row is recovered exactly from
// y = fl(row * fl(1 / (rows - 1))): fl(y (rows - 1)) is within row x 2^-22 + 2^-24 of the row, below 1/2 for
// rows < 2^20, so rounding it to the nearest integer gives the row.
__host__ __device__ inline int band_of(const Banding& b, float y, int experts) {
    if (b.bands <= 1) return 0;
    const float scaled = y * float(b.rows - 1);  // one fp32 product, as fl() above
    int row = scaled > 0.0f ? int(scaled + 0.5f) : 0;  // scaled < 2^20: the sum is exact to well below 1/2
    row = row >= b.rows ? b.rows - 1 : row;
    int band = int((unsigned)row * (unsigned)b.bands / (unsigned)b.rows);  // row * bands < 2^26
    const int first = b.first_band, last = b.first_band + experts / b.per_band - 1;
    band = band < first ? first : band > last ? last : band;
    return band;
}

// Rejects a banding that the router and the heads cannot serve (throws std::invalid_argument).
void check_banding(const Banding& b, int experts);
void launch_router_forward(const RouterArgs& a, int width, cudaStream_t stream);

}  // namespace odie
