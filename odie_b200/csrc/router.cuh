// Top-1 expert router (router.cu).
#pragma once
#include "common.cuh"

namespace odie {

// Router MLP shape: W -> 32 -> 32 -> 16, ReLU hidden layers, linear logits,
// no biases; fp16 weights row-major [out][in] in the order W1, W2, W3.
constexpr int ROUTER_HIDDEN = 32, ROUTER_OUT = 16;
__host__ __device__ constexpr int router_params(int w) {
    return ROUTER_HIDDEN * w + ROUTER_HIDDEN * ROUTER_HIDDEN + ROUTER_OUT * ROUTER_HIDDEN;
}

struct RouterArgs {
    const __half* features = nullptr;  // router-grid features: pair-major [W/2][stride] half2, or row-major [n][W]
    long long stride = 0;
    bool row_major = false;
    long long n = 0;
    const __half* weights = nullptr;   // fp16 [router_params(W)]
    int experts = 0;                   // live experts (logit columns 0..experts-1)
    int* expert = nullptr;             // [n] chosen expert
    float* prob = nullptr;             // [n] softmax probability of the chosen expert
    __half* logits = nullptr;          // optional [n][16] fp16 logits
};

void launch_router_forward(const RouterArgs& a, int width, cudaStream_t stream);

}  // namespace odie
