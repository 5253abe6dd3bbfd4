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
// held as fp32 in shared memory and read as warp-wide broadcasts, each one
// feeding the chains of two coordinates.
#include "router.cuh"

namespace odie {

namespace {

constexpr int ROUTER_THREADS = 128;

__device__ __forceinline__ float half_round(float x) { return __half2float(__float2half_rn(x)); }

// Each thread routes ROUTER_PER_THREAD coordinates (i, i + blockDim.x, ...) so that every
// shared-memory weight it loads feeds that many fused multiply-adds.
constexpr int ROUTER_PER_THREAD = 2;

template <int W>
__global__ void __launch_bounds__(ROUTER_THREADS) router_forward_kernel(const RouterArgs a) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN, P3 = ROUTER_OUT * ROUTER_HIDDEN;
    constexpr int C = ROUTER_PER_THREAD;
    __shared__ __align__(16) float w[P1 + P2 + P3];
    for (int j = threadIdx.x; j < P1 + P2 + P3; j += blockDim.x) w[j] = __half2float(a.weights[j]);
    __syncthreads();
    const long long first = (long long)blockIdx.x * blockDim.x * C + threadIdx.x;
    if (first >= a.n) return;
    long long row[C];
    float x[C][W];
#pragma unroll
    for (int c = 0; c < C; ++c) {
        row[c] = first + (long long)c * blockDim.x;
        const long long i = row[c] < a.n ? row[c] : first;  // a missing second row repeats the first, unstored
        if (a.row_major) {  // the coordinate's row as 16-byte loads
#pragma unroll
            for (int j = 0; j < W / 8; ++j) {
                const uint4 q = __ldg(reinterpret_cast<const uint4*>(a.features) + i * (W / 8) + j);
                const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int h = 0; h < 4; ++h) {
                    x[c][8 * j + 2 * h] = __half2float(__ushort_as_half(uint16_t(w4[h] & 0xffffu)));
                    x[c][8 * j + 2 * h + 1] = __half2float(__ushort_as_half(uint16_t(w4[h] >> 16)));
                }
            }
        } else {
#pragma unroll
            for (int p = 0; p < W / 2; ++p) {
                const __half2 v = __ldg(reinterpret_cast<const __half2*>(a.features) + (long long)p * a.stride + i);
                x[c][2 * p] = __low2float(v);
                x[c][2 * p + 1] = __high2float(v);
            }
        }
    }
    float h1[C][ROUTER_HIDDEN], h2[C][ROUTER_HIDDEN], z[C][ROUTER_OUT];
#pragma unroll
    for (int o = 0; o < ROUTER_HIDDEN; ++o) {
        float acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = 0.0f;
#pragma unroll
        for (int k = 0; k < W; ++k) {
            const float wk = w[o * W + k];
#pragma unroll
            for (int c = 0; c < C; ++c) acc[c] = __fmaf_rn(wk, x[c][k], acc[c]);
        }
#pragma unroll
        for (int c = 0; c < C; ++c) h1[c][o] = half_round(acc[c] > 0.0f ? acc[c] : 0.0f);
    }
#pragma unroll
    for (int o = 0; o < ROUTER_HIDDEN; ++o) {
        float acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = 0.0f;
#pragma unroll
        for (int k = 0; k < ROUTER_HIDDEN; ++k) {
            const float wk = w[P1 + o * ROUTER_HIDDEN + k];
#pragma unroll
            for (int c = 0; c < C; ++c) acc[c] = __fmaf_rn(wk, h1[c][k], acc[c]);
        }
#pragma unroll
        for (int c = 0; c < C; ++c) h2[c][o] = half_round(acc[c] > 0.0f ? acc[c] : 0.0f);
    }
#pragma unroll
    for (int o = 0; o < ROUTER_OUT; ++o) {
        float acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = 0.0f;
#pragma unroll
        for (int k = 0; k < ROUTER_HIDDEN; ++k) {
            const float wk = w[P1 + P2 + o * ROUTER_HIDDEN + k];
#pragma unroll
            for (int c = 0; c < C; ++c) acc[c] = __fmaf_rn(wk, h2[c][k], acc[c]);
        }
#pragma unroll
        for (int c = 0; c < C; ++c) z[c][o] = half_round(acc[c]);
    }
#pragma unroll
    for (int c = 0; c < C; ++c) {
        if (row[c] >= a.n) continue;
        const long long i = row[c];
        int best = 0;
        float zbest = z[c][0];
#pragma unroll
        for (int e = 1; e < ROUTER_OUT; ++e)
            if (e < a.experts && z[c][e] > zbest) {
                best = e;
                zbest = z[c][e];
            }
        float sum = 0.0f;
#pragma unroll
        for (int e = 0; e < ROUTER_OUT; ++e)
            if (e < a.experts) sum = __fadd_rn(sum, expf(__fsub_rn(z[c][e], zbest)));
        a.expert[i] = best;
        a.prob[i] = __fdiv_rn(1.0f, sum);
        if (a.logits) {
#pragma unroll
            for (int o = 0; o < ROUTER_OUT; o += 2)
                reinterpret_cast<__half2*>(a.logits)[(i * ROUTER_OUT + o) / 2] = __floats2half2_rn(z[c][o], z[c][o + 1]);
        }
    }
}

}  // namespace

void launch_router_forward(const RouterArgs& a, int width, cudaStream_t stream) {
    if (a.n <= 0) return;
    ODIE_REQUIRE(a.experts >= 1 && a.experts <= ROUTER_OUT, "the router chooses among 1..16 experts");
    const unsigned blocks = blocks_for(a.n, ROUTER_THREADS * ROUTER_PER_THREAD);
    if (width == 32) router_forward_kernel<32><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    else if (width == 16) router_forward_kernel<16><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    else throw std::invalid_argument("the router takes 16 or 32 input features");
    note_launch();
}

}  // namespace odie
