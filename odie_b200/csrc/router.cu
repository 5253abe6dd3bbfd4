// Top-1 expert routing (routed multi-expert encoding; no reference counterpart).
//
// The router is a small MLP over the coarse shared grid's features: W -> 32
// (ReLU) -> 32 (ReLU) -> 16 logits, fp16 weights [out][in], no biases.  The
// routing decision must be reproducible bit for bit, so this forward pass does
// not use the tensor cores (whose fp32 accumulation order is unspecified): one
// thread per coordinate evaluates every output as an fp32 fused-multiply-add
// chain in ascending input order from +0, rounds every layer's output to fp16,
// and picks the first maximum of the fp16 logits over the live experts.  The
// gate probability of the chosen expert is 1 / sum_j exp(z_j - z_max), the sum
// taken in ascending expert order.  2 560 FMAs per coordinate; the weights are
// held as fp32 in shared memory and read as warp-wide broadcasts.
#include "router.cuh"

namespace odie {

namespace {

constexpr int ROUTER_THREADS = 128;

__device__ __forceinline__ float half_round(float x) { return __half2float(__float2half_rn(x)); }

template <int W>
__global__ void __launch_bounds__(ROUTER_THREADS) router_forward_kernel(const RouterArgs a) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN, P3 = ROUTER_OUT * ROUTER_HIDDEN;
    __shared__ __align__(16) float w[P1 + P2 + P3];
    for (int j = threadIdx.x; j < P1 + P2 + P3; j += blockDim.x) w[j] = __half2float(a.weights[j]);
    __syncthreads();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n) return;
    float x[W];
#pragma unroll
    for (int p = 0; p < W / 2; ++p) {
        const __half2 v = __ldg(reinterpret_cast<const __half2*>(a.features) +
                                (a.row_major ? i * (W / 2) + p : (long long)p * a.stride + i));
        x[2 * p] = __low2float(v);
        x[2 * p + 1] = __high2float(v);
    }
    float h1[ROUTER_HIDDEN], h2[ROUTER_HIDDEN], z[ROUTER_OUT];
#pragma unroll
    for (int o = 0; o < ROUTER_HIDDEN; ++o) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < W; ++k) acc = __fmaf_rn(w[o * W + k], x[k], acc);
        h1[o] = half_round(acc > 0.0f ? acc : 0.0f);
    }
#pragma unroll
    for (int o = 0; o < ROUTER_HIDDEN; ++o) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < ROUTER_HIDDEN; ++k) acc = __fmaf_rn(w[P1 + o * ROUTER_HIDDEN + k], h1[k], acc);
        h2[o] = half_round(acc > 0.0f ? acc : 0.0f);
    }
#pragma unroll
    for (int o = 0; o < ROUTER_OUT; ++o) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < ROUTER_HIDDEN; ++k) acc = __fmaf_rn(w[P1 + P2 + o * ROUTER_HIDDEN + k], h2[k], acc);
        z[o] = half_round(acc);
    }
    int best = 0;
    float zbest = z[0];
#pragma unroll
    for (int e = 1; e < ROUTER_OUT; ++e)
        if (e < a.experts && z[e] > zbest) {
            best = e;
            zbest = z[e];
        }
    float sum = 0.0f;
#pragma unroll
    for (int e = 0; e < ROUTER_OUT; ++e)
        if (e < a.experts) sum = __fadd_rn(sum, expf(__fsub_rn(z[e], zbest)));
    a.expert[i] = best;
    a.prob[i] = __fdiv_rn(1.0f, sum);
    if (a.logits) {
#pragma unroll
        for (int o = 0; o < ROUTER_OUT; o += 2)
            reinterpret_cast<__half2*>(a.logits)[(i * ROUTER_OUT + o) / 2] = __floats2half2_rn(z[o], z[o + 1]);
    }
}

}  // namespace

void launch_router_forward(const RouterArgs& a, int width, cudaStream_t stream) {
    if (a.n <= 0) return;
    ODIE_REQUIRE(a.experts >= 1 && a.experts <= ROUTER_OUT, "the router chooses among 1..16 experts");
    const unsigned blocks = blocks_for(a.n, ROUTER_THREADS);
    if (width == 32) router_forward_kernel<32><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    else if (width == 16) router_forward_kernel<16><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    else throw std::invalid_argument("the router takes 16 or 32 input features");
}

}  // namespace odie
