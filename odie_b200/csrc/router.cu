// Top-1 expert routing (routed multi-expert encoding; no reference counterpart).
//
// The router is a small MLP over the coarse shared grid's features: W -> 32
// (ReLU) -> 32 (ReLU) -> 16 logits, fp16 weights [out][in], no biases.  The
// routing decision must be reproducible bit for bit, so this forward pass does
// not use the tensor cores (whose fp32 accumulation order is unspecified): every
// output of a coordinate is an fp32 fused-multiply-add chain in ascending input
// order from +0 on the CUDA cores; every layer's output is rounded to fp16, and
// the choice is the first maximum of the fp16 logits over the live experts.  The
// gate probability of the chosen expert is 1 / sum_j exp(z_j - z_max), the sum
// taken in ascending expert order.  2 560 FMAs per coordinate.
#include "router.cuh"

namespace odie {

namespace {

constexpr int ROUTER_THREADS = 128;

__device__ __forceinline__ float half_round(float x) { return __half2float(__float2half_rn(x)); }

// Two coordinates per thread.  Every layer runs its outputs in pairs (o, o + 1)
// as packed fma chains (fma.rn.f32x2: two IEEE fp32 fused multiply-adds, each
// rounded exactly as __fmaf_rn) over the input broadcast as {x_k, x_k}; the
// weights sit in shared memory pair-interleaved, {W[o][k], W[o + 1][k]}, and each
// weight load serves both coordinates (the kernel is bound by shared-memory loads).
constexpr int ROUTER_PER_THREAD = 2;

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

// Two coordinates a and b per thread: out[o] = act(sum_k W[o][k] in[k]) for OUT outputs over
// IN inputs (IN even), for both.  w: pair-interleaved weights {W[o][k], W[o + 1][k]}, 16-byte
// aligned rows, so one 16-byte shared load (a broadcast) brings pairs k and k + 1 and feeds
// four packed FMAs.  Each coordinate's outputs are its own fma chains in ascending k from +0,
// exactly as one coordinate per thread computes them.  The inputs stay in registers
// (broadcast pairs); the output pairs come from a loop that is not unrolled (the code stays
// small enough for the instruction cache) and go to the coordinates' columns of act.
template <int IN, int OUT, bool RELU>
__device__ __forceinline__ void layer(const f32x2* __restrict__ w, const float* in_a, const float* in_b, float* act_a,
                                      float* act_b) {
    f32x2 ba[IN], bb[IN];
#pragma unroll
    for (int k = 0; k < IN; ++k) {
        ba[k] = pack2(in_a[k], in_a[k]);
        bb[k] = pack2(in_b[k], in_b[k]);
    }
#pragma unroll 1
    for (int o = 0; o < OUT; o += 2) {
        const ulonglong2* wo = reinterpret_cast<const ulonglong2*>(w + (o / 2) * IN);
        f32x2 acc_a = 0, acc_b = 0;  // {+0, +0}
#pragma unroll
        for (int k = 0; k < IN; k += 2) {
            const ulonglong2 q = wo[k / 2];
            acc_a = fma2(q.x, ba[k], acc_a);
            acc_b = fma2(q.x, bb[k], acc_b);
            acc_a = fma2(q.y, ba[k + 1], acc_a);
            acc_b = fma2(q.y, bb[k + 1], acc_b);
        }
        float a0, a1, b0, b1;
        unpack2(acc_a, a0, a1);
        unpack2(acc_b, b0, b1);
        if (RELU) {
            a0 = a0 > 0.0f ? a0 : 0.0f;
            a1 = a1 > 0.0f ? a1 : 0.0f;
            b0 = b0 > 0.0f ? b0 : 0.0f;
            b1 = b1 > 0.0f ? b1 : 0.0f;
        }
        act_a[o * ROUTER_THREADS + threadIdx.x] = half_round(a0);
        act_a[(o + 1) * ROUTER_THREADS + threadIdx.x] = half_round(a1);
        act_b[o * ROUTER_THREADS + threadIdx.x] = half_round(b0);
        act_b[(o + 1) * ROUTER_THREADS + threadIdx.x] = half_round(b1);
    }
}

template <int N>
__device__ __forceinline__ void read_column(const float* act, float* out) {
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = act[k * ROUTER_THREADS + threadIdx.x];
}

// Router-grid features of coordinate i (zeros past the end).
template <int W>
__device__ __forceinline__ void load_features(const RouterArgs& a, long long i, float* x) {
    if (i >= a.n) {
#pragma unroll
        for (int k = 0; k < W; ++k) x[k] = 0.0f;
        return;
    }
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
}

// Top-1 over the live experts (first maximum of the fp16 logits) and its softmax probability.
__device__ __forceinline__ void choose(const RouterArgs& a, const float* z, long long i) {
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

// Coordinates i and j (j may lie past the end: computed on zeros, not stored).
template <int W>
__device__ __forceinline__ void route_two(const RouterArgs& a, const f32x2* __restrict__ w, float* act_a, float* act_b,
                                          long long i, long long j) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN;
    float xa[W], xb[W];
    load_features<W>(a, i, xa);
    load_features<W>(a, j, xb);
    float ha[ROUTER_HIDDEN], hb[ROUTER_HIDDEN];
    layer<W, ROUTER_HIDDEN, true>(w, xa, xb, act_a, act_b);
    read_column<ROUTER_HIDDEN>(act_a, ha);
    read_column<ROUTER_HIDDEN>(act_b, hb);
    layer<ROUTER_HIDDEN, ROUTER_HIDDEN, true>(w + P1 / 2, ha, hb, act_a, act_b);
    read_column<ROUTER_HIDDEN>(act_a, ha);
    read_column<ROUTER_HIDDEN>(act_b, hb);
    layer<ROUTER_HIDDEN, ROUTER_OUT, false>(w + (P1 + P2) / 2, ha, hb, act_a, act_b);
    float z[ROUTER_OUT];
    read_column<ROUTER_OUT>(act_a, z);
    choose(a, z, i);
    if (j < a.n) {
        read_column<ROUTER_OUT>(act_b, z);
        choose(a, z, j);
    }
}

template <int W>
__global__ void __launch_bounds__(ROUTER_THREADS) router_forward_kernel(const RouterArgs a) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN, P3 = ROUTER_OUT * ROUTER_HIDDEN;
    __shared__ __align__(16) f32x2 w[(P1 + P2 + P3) / 2];
    __shared__ float act[2][ROUTER_HIDDEN * ROUTER_THREADS];  // each thread's layer outputs, one column per coordinate
    // pair-interleave each layer's rows: entry (o / 2) * IN + k = {W[o][k], W[o + 1][k]}
    for (int j = threadIdx.x; j < (P1 + P2 + P3) / 2; j += blockDim.x) {
        int base = 0, in = W, e = j;
        if (e >= P1 / 2) { base = P1; in = ROUTER_HIDDEN; e -= P1 / 2; }
        if (base == P1 && e >= P2 / 2) { base = P1 + P2; e -= P2 / 2; }
        const int o = 2 * (e / in), k = e % in;
        w[j] = pack2(__half2float(a.weights[base + o * in + k]), __half2float(a.weights[base + (o + 1) * in + k]));
    }
    __syncthreads();
    // persistent blocks: the weights are staged once per block, then the block walks the coordinates,
    // 2 x blockDim at a time (thread t: base + t and base + blockDim + t)
    for (long long base = (long long)blockIdx.x * 2 * blockDim.x; base < a.n; base += (long long)gridDim.x * 2 * blockDim.x)
        route_two<W>(a, w, act[0], act[1], base + threadIdx.x, base + blockDim.x + threadIdx.x);
}

}  // namespace

void launch_router_forward(const RouterArgs& a, int width, cudaStream_t stream) {
    if (a.n <= 0) return;
    ODIE_REQUIRE(a.experts >= 1 && a.experts <= ROUTER_OUT, "the router chooses among 1..16 experts");
    if (width != 32 && width != 16) throw std::invalid_argument("the router takes 16 or 32 input features");
    // persistent blocks: as many as fit on the GPU at once
    int per_sm = 0;
    if (width == 32) ODIE_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, router_forward_kernel<32>, ROUTER_THREADS, 0));
    else ODIE_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, router_forward_kernel<16>, ROUTER_THREADS, 0));
    const long long resident = (long long)(per_sm > 0 ? per_sm : 1) * sm_count();
    const long long needed = blocks_for(a.n, ROUTER_THREADS * ROUTER_PER_THREAD);
    const unsigned blocks = unsigned(needed < resident ? needed : resident);
    if (width == 32) router_forward_kernel<32><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    else router_forward_kernel<16><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    note_launch();
}

}  // namespace odie
