// L2 bandwidth probe: the roofline denominator of the gather and scatter kernels.
//
// The grid tables of every benchmark configuration fit in the 126 MB L2, so
// their random 4-corner gathers and reductions are bounded by L2 throughput,
// not HBM.  This probe measures that bound on the running GPU: random 4-byte
// and 16-byte loads, and random 4-byte and 8-byte fp32 reductions, over a table
// of `table_bytes` (kept <= 64 MiB so it stays L2-resident), every thread
// drawing its indices from a hash of its id (no index traffic).  One launch per
// mode; the caller times it with CUDA events.
#include "common.cuh"
#include "tc.cuh"

namespace odie {

namespace {

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// mode 0: 4-byte loads, 1: 16-byte loads, 2: red.add.f32, 3: red.add.v2.f32
__global__ void __launch_bounds__(256) l2_probe_kernel(float* table, uint32_t words, int mode, int per_thread,
                                                       float* sink) {
    const uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    float acc = 0.0f;
    uint32_t state = mix32(t * 0x9e3779b9u + 0x1234567u);
    for (int j = 0; j < per_thread; ++j) {
        state = mix32(state + uint32_t(j));
        if (mode == 0) {
            acc += __ldcg(table + (state % words));
        } else if (mode == 1) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(table) + (state % (words / 4)));
            acc += v.x + v.y + v.z + v.w;
        } else if (mode == 2) {
            red_add_f32(table + (state % words), 1e-30f);
        } else {
            red_add_v2(table + 2 * (state % (words / 2)), 1e-30f, 1e-30f);
        }
    }
    if (acc == 1234.5f) sink[0] = acc;  // keeps the loads alive
}

// fp32 FMA throughput: 8 independent fma chains per thread (enough to hide the pipe's latency at full
// occupancy); the roofline denominator of the fp32 CUDA-core MLP.  2 x 8 x iterations FLOP per thread.
__global__ void __launch_bounds__(256) fma_probe_kernel(int iterations, float* sink) {
    float a[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = float(threadIdx.x + k) * 1e-3f;
    const float b = 0.999f, c = 1e-4f;
    for (int j = 0; j < iterations; ++j)
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = __fmaf_rn(a[k], b, c);
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s += a[k];
    if (s == 1234.5f) sink[0] = s;  // keeps the chains alive
}

// The bounded mbarrier wait of the heads kernel, made to run out: one block waits on a barrier
// that expects one arrival which nothing makes.  tc::bar_wait gives up after `limit` polls and
// the block reports 2 (the heads kernel's "a wait ran out" code) instead of hanging.
__global__ void wait_probe_kernel(uint32_t limit, int* __restrict__ status) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        tc::bar_init(&bar, 1);
        tc::fence_bar_init();
    }
    __syncthreads();
    const bool done = tc::bar_wait(&bar, 0, limit);
    const int ok = __syncthreads_and(done);
    if (threadIdx.x == 0) *status = ok ? 0 : 2;
}

}  // namespace

void launch_wait_probe(uint32_t limit, int* status, cudaStream_t stream) {
    ODIE_REQUIRE(limit >= 1 && limit <= (1u << 20), "wait probe limit must be 1..2^20 polls");
    wait_probe_kernel<<<1, 128, 0, stream>>>(limit, status);
    note_launch();
}

long long launch_fma_probe(int iterations, float* sink, cudaStream_t stream) {
    ODIE_REQUIRE(iterations >= 1 && iterations <= (1 << 24), "fma probe iterations must be 1..2^24");
    const int blocks = 8 * sm_count();
    fma_probe_kernel<<<blocks, 256, 0, stream>>>(iterations, sink);
    note_launch();
    return 2LL * 8 * iterations * blocks * 256;  // FLOP
}

void launch_l2_probe(float* table, long long table_bytes, int mode, long long operations, float* sink,
                     cudaStream_t stream) {
    ODIE_REQUIRE(mode >= 0 && mode <= 3, "probe mode must be 0..3");
    ODIE_REQUIRE(table_bytes >= 4096 && table_bytes <= (64LL << 20), "probe table must be 4 KiB..64 MiB");
    const int per_thread = 64;
    const long long threads = (operations + per_thread - 1) / per_thread;
    ODIE_REQUIRE(threads >= 1 && threads <= (1LL << 31) - 1, "probe operation count out of range");
    l2_probe_kernel<<<blocks_for(threads, 256), 256, 0, stream>>>(table, uint32_t(table_bytes / 4), mode, per_thread,
                                                                  sink);
    note_launch();
}

}  // namespace odie
