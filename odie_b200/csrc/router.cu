// Top-1 expert routing (routed multi-expert encoding; no reference counterpart).
//
// The router is a small MLP over the coarse shared grid's features: W -> 32
// (ReLU) -> 32 (ReLU) -> OUT logits (OUT = 16 or 64), fp16 weights [out][in], no
// biases.  The routing decision must be reproducible bit for bit, so this forward
// pass does not use the tensor cores (whose fp32 accumulation order is
// unspecified): every output of a coordinate is an fp32 fused-multiply-add chain in
// ascending input order from +0 on the CUDA cores; every layer's output is rounded to
// fp16, and the choice is the first maximum of the fp16 logits over the
// coordinate's live experts (its band's, under spatial expert ownership).  Only the
// live logits are computed.  The gate probability of the chosen expert is
// 1 / sum_j exp(z_j - z_max) over the live experts, the sum taken in ascending
// expert order.  2 048 + 32 x live FMAs per coordinate.
#include "router.cuh"

namespace odie {

namespace {

constexpr int ROUTER_THREADS = 128;

// ROUTER_PER_THREAD coordinates per thread.  Every layer runs its outputs in pairs (o, o + 1)
// as packed fma chains (fma.rn.f32x2: two IEEE fp32 fused multiply-adds, each
// rounded exactly as __fmaf_rn) over the input broadcast as {x_k, x_k}; the
// weights sit in shared memory pair-interleaved, {W[o][k], W[o + 1][k]}, and each
// weight load serves all of the thread's coordinates.  Two coordinates per thread keep 96 registers, so 20
// warps share an SM; four halved the weight loads but held 168 registers (12 warps) and ran 3.5 % slower.
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

// C coordinates per thread: out[o] = act(sum_k W[o][k] in[k]) for `out` outputs (even) over IN
// inputs (IN even), for each.  w: pair-interleaved weights {W[o][k], W[o + 1][k]}, 16-byte
// aligned rows; rows[c] is coordinate c's first weight row (even; all equal for the hidden
// layers).  When the C coordinates share their rows, one 16-byte shared load (a broadcast)
// brings pairs k and k + 1 and feeds 2 C packed FMAs; otherwise each coordinate loads its own.
// Each coordinate's outputs are its own fma chains in ascending k from +0, exactly as one
// coordinate per thread computes them.  The output pairs come from a loop that is not unrolled
// (the code stays small enough for the instruction cache) and land as fp16 pairs in the
// coordinates' columns of act.
template <int C, int IN, bool RELU>
__device__ __forceinline__ void layer(const f32x2* __restrict__ w, const int (&rows)[C], int out,
                                      const float (&in)[C][IN], __half2* act) {
    f32x2 bc[C][IN];
#pragma unroll
    for (int c = 0; c < C; ++c)
#pragma unroll
        for (int k = 0; k < IN; ++k) bc[c][k] = pack2(in[c][k], in[c][k]);
    bool shared = true;
#pragma unroll
    for (int c = 1; c < C; ++c) shared = shared && rows[c] == rows[0];
#pragma unroll 1
    for (int o = 0; o < out; o += 2) {
        f32x2 acc[C];
#pragma unroll
        for (int c = 0; c < C; ++c) acc[c] = 0;  // {+0, +0}
        if (shared) {
            const ulonglong2* wo = reinterpret_cast<const ulonglong2*>(w + ((rows[0] + o) / 2) * IN);
#pragma unroll
            for (int k = 0; k < IN; k += 2) {
                const ulonglong2 q = wo[k / 2];
#pragma unroll
                for (int c = 0; c < C; ++c) acc[c] = fma2(q.x, bc[c][k], acc[c]);
#pragma unroll
                for (int c = 0; c < C; ++c) acc[c] = fma2(q.y, bc[c][k + 1], acc[c]);
            }
        } else {
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const ulonglong2* wo = reinterpret_cast<const ulonglong2*>(w + ((rows[c] + o) / 2) * IN);
#pragma unroll
                for (int k = 0; k < IN; k += 2) {
                    const ulonglong2 q = wo[k / 2];
                    acc[c] = fma2(q.x, bc[c][k], acc[c]);
                    acc[c] = fma2(q.y, bc[c][k + 1], acc[c]);
                }
            }
        }
#pragma unroll
        for (int c = 0; c < C; ++c) {
            float v0, v1;
            unpack2(acc[c], v0, v1);
            if (RELU) {
                v0 = v0 > 0.0f ? v0 : 0.0f;
                v1 = v1 > 0.0f ? v1 : 0.0f;
            }
            // the pair rounded to fp16, as one 4-byte store
            act[(c * ROUTER_HIDDEN / 2 + o / 2) * ROUTER_THREADS + threadIdx.x] = __floats2half2_rn(v0, v1);
        }
    }
}

// The N fp16 outputs of coordinate c of this thread (pairs stored as half2).
template <int N>
__device__ __forceinline__ void read_column(const __half2* act, int c, float* out) {
#pragma unroll
    for (int p = 0; p < N / 2; ++p) {
        const __half2 v = act[(c * ROUTER_HIDDEN / 2 + p) * ROUTER_THREADS + threadIdx.x];
        out[2 * p] = __low2float(v);
        out[2 * p + 1] = __high2float(v);
    }
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

// Top-1 over the coordinate's live experts (first maximum of their fp16 logits z[0..per)) and its softmax
// probability; first: the local number of its band's first expert.  The live logits are optionally stored as
// a row of a.live halves.
__device__ __forceinline__ void choose(const RouterArgs& a, const float* z, int first, long long i) {
    const int per = a.banding.per_band;
    int best = 0;
    float zbest = z[0];
#pragma unroll
    for (int e = 1; e < ROUTER_MAX_LIVE; ++e)
        if (e < per && z[e] > zbest) {
            best = e;
            zbest = z[e];
        }
    float sum = 0.0f;
#pragma unroll
    for (int e = 0; e < ROUTER_MAX_LIVE; ++e)
        if (e < per) sum = __fadd_rn(sum, expf(__fsub_rn(z[e], zbest)));
    a.expert[i] = first + best;
    a.prob[i] = __fdiv_rn(1.0f, sum);
    if (a.logits) {
        __half2* row = reinterpret_cast<__half2*>(a.logits + i * a.live);
#pragma unroll
        for (int o = 0; o < ROUTER_MAX_LIVE; o += 2)
            if (o < a.live) row[o / 2] = __floats2half2_rn(o < per ? z[o] : 0.0f, o + 1 < per ? z[o + 1] : 0.0f);
    }
}

// Coordinates first + c * blockDim for c < C (those past the end: computed on zeros, not stored).
// BANDED: coordinates choose among their band's experts (bands > 1); otherwise among all, logit rows from 0.
template <int C, int W, bool BANDED>
__device__ __forceinline__ void route_group(const RouterArgs& a, const f32x2* __restrict__ w, __half2* act,
                                            long long first) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN;
    float x[C][W];
    int zero[C], band[C], rows3[C];  // rows3: the first logit row of the coordinate's band
    const Banding& b = a.banding;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const long long i = first + (long long)c * blockDim.x;
        load_features<W>(a, i, x[c]);
        zero[c] = 0;
        band[c] = (BANDED && i < a.n) ? band_of(b, __ldg(a.xy + 2 * i + 1), a.experts) : b.first_band;
        rows3[c] = BANDED ? band[c] * b.per_band : 0;
    }
    float h[C][ROUTER_HIDDEN];
    layer<C, W, true>(w, zero, ROUTER_HIDDEN, x, act);
#pragma unroll
    for (int c = 0; c < C; ++c) read_column<ROUTER_HIDDEN>(act, c, h[c]);
    layer<C, ROUTER_HIDDEN, true>(w + P1 / 2, zero, ROUTER_HIDDEN, h, act);
#pragma unroll
    for (int c = 0; c < C; ++c) read_column<ROUTER_HIDDEN>(act, c, h[c]);
    // only the live rows of the logit layer, rounded up to whole pairs (the padding rows exist)
    layer<C, ROUTER_HIDDEN, false>(w + (P1 + P2) / 2, rows3, (b.per_band + 1) & ~1, h, act);
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const long long i = first + (long long)c * blockDim.x;
        if (i < a.n) {
            float z[ROUTER_MAX_LIVE];
            read_column<ROUTER_MAX_LIVE>(act, c, z);
            choose(a, z, (band[c] - b.first_band) * b.per_band, i);
        }
    }
}

template <int W, int OUT, bool BANDED>
__global__ void __launch_bounds__(ROUTER_THREADS) router_forward_kernel(const RouterArgs a) {
    constexpr int P1 = ROUTER_HIDDEN * W, P2 = ROUTER_HIDDEN * ROUTER_HIDDEN, P3 = OUT * ROUTER_HIDDEN;
    constexpr int C = ROUTER_PER_THREAD;
    __shared__ __align__(16) f32x2 w[(P1 + P2 + P3) / 2];
    __shared__ __half2 act[C * ROUTER_HIDDEN / 2 * ROUTER_THREADS];  // each coordinate's layer outputs (fp16 pairs)
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
    // C x blockDim at a time (thread t: base + t, base + blockDim + t, ...); the next group's rows are
    // prefetched into L2 while this group computes
    const long long step = (long long)gridDim.x * C * blockDim.x;
    for (long long base = (long long)blockIdx.x * C * blockDim.x; base < a.n; base += step) {
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const long long next = base + step + (long long)c * blockDim.x + threadIdx.x;
            if (a.row_major && next < a.n) {
                asm volatile("prefetch.global.L2 [%0];" ::"l"(a.features + next * W));
                if (BANDED) asm volatile("prefetch.global.L2 [%0];" ::"l"(a.xy + 2 * next));
            }
        }
        route_group<C, W, BANDED>(a, w, act, base + threadIdx.x);
    }
}

template <int W, int OUT, bool BANDED>
void launch_router(const RouterArgs& a, cudaStream_t stream) {
    // persistent blocks: as many as fit on the GPU at once
    int per_sm = 0;
    ODIE_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, router_forward_kernel<W, OUT, BANDED>,
                                                            ROUTER_THREADS, 0));
    const long long resident = (long long)(per_sm > 0 ? per_sm : 1) * sm_count();
    const long long needed = blocks_for(a.n, ROUTER_THREADS * ROUTER_PER_THREAD);
    const unsigned blocks = unsigned(needed < resident ? needed : resident);
    router_forward_kernel<W, OUT, BANDED><<<blocks, ROUTER_THREADS, 0, stream>>>(a);
    note_launch();
}

}  // namespace

void check_banding(const Banding& b, int experts) {
    ODIE_REQUIRE(b.bands >= 1 && b.bands <= ROUTER_MAX_OUT, "bands must be within 1..64");
    ODIE_REQUIRE(b.per_band >= 1 && b.per_band <= ROUTER_MAX_LIVE && b.model_experts() <= ROUTER_MAX_OUT,
                 "experts per band must be within 1..16 and the model's experts within 1..64");
    ODIE_REQUIRE(experts >= b.per_band && experts % b.per_band == 0, "the experts held must be whole bands");
    ODIE_REQUIRE(b.first_band >= 0 && b.first_band + experts / b.per_band <= b.bands,
                 "the bands held must lie within the image's bands");
    ODIE_REQUIRE(b.bands == 1 || ((b.per_band == 8 || b.per_band == 16) && b.rows >= 2 && b.rows < (1 << 20)),
                 "banded routing needs 8 or 16 experts per band and 2 <= rows < 2^20");
}

void launch_router_forward(const RouterArgs& a, int width, cudaStream_t stream) {
    if (a.n <= 0) return;
    check_banding(a.banding, a.experts);
    ODIE_REQUIRE(a.banding.bands == 1 || a.xy, "banded routing needs the coordinates");
    ODIE_REQUIRE(!a.logits || (a.live >= a.banding.per_band && (a.live == 8 || a.live == 16)),
                 "the logits row holds 8 or 16 halves, at least the experts per band");
    if (width != 32 && width != 16) throw std::invalid_argument("the router takes 16 or 32 input features");
    const bool wide = router_out(a.banding.model_experts()) == ROUTER_MAX_OUT, banded = a.banding.bands > 1;
    if (width == 32 && wide) banded ? launch_router<32, 64, true>(a, stream) : launch_router<32, 64, false>(a, stream);
    else if (width == 32) banded ? launch_router<32, 16, true>(a, stream) : launch_router<32, 16, false>(a, stream);
    else if (wide) banded ? launch_router<16, 64, true>(a, stream) : launch_router<16, 64, false>(a, stream);
    else banded ? launch_router<16, 16, true>(a, stream) : launch_router<16, 16, false>(a, stream);
}

}  // namespace odie
