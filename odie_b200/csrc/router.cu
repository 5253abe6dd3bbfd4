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
// taken in ascending expert order.  2 560 FMAs per coordinate.
#include "router.cuh"

namespace odie {

namespace {

constexpr int ROUTER_THREADS = 128;

__device__ __forceinline__ float half_round(float x) { return __half2float(__float2half_rn(x)); }

// One thread per coordinate.  Every layer runs its outputs in pairs (o, o + 1)
// as packed fma chains (fma.rn.f32x2: two IEEE fp32 fused multiply-adds, each
// rounded exactly as __fmaf_rn) over the input broadcast as {x_k, x_k}; the
// weights sit in shared memory pair-interleaved, {W[o][k], W[o + 1][k]}, so one
// 8-byte load feeds one packed instruction.
constexpr int ROUTER_PER_THREAD = 1;

using f32x2 = unsigned long long;
__device__ __forceinline__ f32x2 pack2(float a, float b) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unpack2(f32x2 v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// out[o] = act(sum_k W[o][k] in[k]) for OUT outputs over IN inputs; w: pair-interleaved weights.
// The input stays in registers (broadcast pairs); the output pairs are produced in a
// loop that is not unrolled (the kernel's code stays small enough for the
// instruction cache) and written to this thread's column of act[][blockDim].
template <int IN, int OUT, bool RELU>
__device__ __forceinline__ void layer(const f32x2* __restrict__ w, const float* in, float* act) {
    f32x2 bcast[IN];
#pragma unroll
    for (int k = 0; k < IN; ++k) bcast[k] = pack2(in[k], in[k]);
#pragma unroll 1
    for (int o = 0; o < OUT; o += 2) {
        const f32x2* wo = w + (o / 2) * IN;
        f32x2 acc = 0;  // {+0, +0}
#pragma unroll
        for (int k = 0; k < IN; ++k) acc = fma2(wo[k], bcast[k], acc);
        float a, b;
        unpack2(acc, a, b);
        if (RELU) {
            a = a > 0.0f ? a : 0.0f;
            b = b > 0.0f ? b : 0.0f;
        }
        act[o * ROUTER_THREADS + threadIdx.x] = half_round(a);
        act[(o + 1) * ROUTER_THREADS + threadIdx.x] = half_round(b);
    }
}

template <int N>
__device__ __forceinline__ void read_column(const float* act, float* out) {
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = act[k * ROUTER_THREADS + threadIdx.x];
}

template <int W>
__device__ __forceinline__ void route_one(const RouterArgs& a, const f32x2* __restrict__ w, float* act, long long i) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN;
    float x[W];
    if (a.row_major) {  // the coordinate's row as 16-byte loads
#pragma unroll
        for (int j = 0; j < W / 8; ++j) {
            const uint4 q = __ldg(reinterpret_cast<const uint4*>(a.features) + i * (W / 8) + j);
            const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                x[8 * j + 2 * h] = __half2float(__ushort_as_half(uint16_t(w4[h] & 0xffffu)));
                x[8 * j + 2 * h + 1] = __half2float(__ushort_as_half(uint16_t(w4[h] >> 16)));
            }
        }
    } else {
#pragma unroll
        for (int p = 0; p < W / 2; ++p) {
            const __half2 v = __ldg(reinterpret_cast<const __half2*>(a.features) + (long long)p * a.stride + i);
            x[2 * p] = __low2float(v);
            x[2 * p + 1] = __high2float(v);
        }
    }
    float h[ROUTER_HIDDEN], z[ROUTER_OUT];
    layer<W, ROUTER_HIDDEN, true>(w, x, act);
    read_column<ROUTER_HIDDEN>(act, h);
    layer<ROUTER_HIDDEN, ROUTER_HIDDEN, true>(w + P1 / 2, h, act);
    read_column<ROUTER_HIDDEN>(act, h);
    layer<ROUTER_HIDDEN, ROUTER_OUT, false>(w + (P1 + P2) / 2, h, act);
    read_column<ROUTER_OUT>(act, z);
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

template <int W>
__global__ void __launch_bounds__(ROUTER_THREADS) router_forward_kernel(const RouterArgs a) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN, P3 = ROUTER_OUT * ROUTER_HIDDEN;
    __shared__ __align__(16) f32x2 w[(P1 + P2 + P3) / 2];
    __shared__ float act[ROUTER_HIDDEN * ROUTER_THREADS];  // each thread's layer outputs, one column per thread
    // pair-interleave each layer's rows: entry (o / 2) * IN + k = {W[o][k], W[o + 1][k]}
    for (int j = threadIdx.x; j < (P1 + P2 + P3) / 2; j += blockDim.x) {
        int base = 0, in = W, e = j;
        if (e >= P1 / 2) { base = P1; in = ROUTER_HIDDEN; e -= P1 / 2; }
        if (base == P1 && e >= P2 / 2) { base = P1 + P2; e -= P2 / 2; }
        const int o = 2 * (e / in), k = e % in;
        w[j] = pack2(__half2float(a.weights[base + o * in + k]), __half2float(a.weights[base + (o + 1) * in + k]));
    }
    __syncthreads();
    // persistent blocks: the weights are staged once per block, then the block walks the coordinates
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += (long long)gridDim.x * blockDim.x) {
        route_one<W>(a, w, act, i);
    }
}

}  // namespace

void launch_router_forward(const RouterArgs& a, int width, cudaStream_t stream) {
    if (a.n <= 0) return;
    ODIE_REQUIRE(a.experts >= 1 && a.experts <= ROUTER_OUT, "the router chooses among 1..16 experts");
    const long long needed = blocks_for(a.n, ROUTER_THREADS * ROUTER_PER_THREAD);
    const unsigned blocks = unsigned(needed < 8LL * sm_count() ? needed : 8LL * sm_count());
    if (width == 32) router_forward_kernel<32><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    else if (width == 16) router_forward_kernel<16><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    else throw std::invalid_argument("the router takes 16 or 32 input features");
    note_launch();
}

}  // namespace odie
