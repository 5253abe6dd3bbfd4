// Input stage, weight-gradient reduction and Adam of the training step.
#include "step.cuh"

namespace odie {

namespace {

// Coordinates of local pixel id: fp32(column) * fp32(1 / (W - 1)), the reciprocal in double rounded to
// fp32 (odie/native/runtime.cu:34-36); the row is the full image's, row0 + id / W, over its rows.
__device__ __forceinline__ float2 coords_of(uint32_t id, int width, RowFrame frame) {
    const float rx = float(1.0 / double(width - 1)), ry = float(1.0 / double(frame.rows - 1));
    return make_float2(__fmul_rn(float(id % uint32_t(width)), rx),
                       __fmul_rn(float(uint32_t(frame.row0) + id / uint32_t(width)), ry));
}

// Coordinates and target of pixel id for batch slot i.
__device__ __forceinline__ void input_of(long long i, uint32_t id, const uint8_t* __restrict__ rgb, bool rgb8, int width,
                                         int height, RowFrame frame, float* __restrict__ xy, float* __restrict__ target) {
    // an id outside the image (never produced by the samplers) reads pixel 0
    // instead of memory outside the target
    if ((unsigned long long)id >= (unsigned long long)width * (unsigned long long)height) id = 0;
    reinterpret_cast<float2*>(xy)[i] = coords_of(id, width, frame);
    if (target) {
        for (int c = 0; c < 3; ++c)
            target[3 * i + c] = rgb8 ? __fmul_rn(float(rgb[3ull * id + c]), 1.0f / 255.0f)
                                     : reinterpret_cast<const float*>(rgb)[3ull * id + c];
    }
}

__global__ void input_batch_kernel(const int64_t* __restrict__ ids, long long n, const uint8_t* __restrict__ rgb,
                                   bool rgb8, int width, int height, RowFrame frame, float* __restrict__ xy,
                                   float* __restrict__ target) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t id = ids[i];
    // ids outside [0, 2^32) become an out-of-image id (pixel 0) instead of wrapping
    input_of(i, (id < 0 || id > 0xffffffffLL) ? 0xffffffffu : uint32_t(id), rgb, rgb8, width, height, frame, xy, target);
}

// Stratified pixel id of slot j (the reference's sampler, odie/data.py:63-80, with this generator):
// stratum (j mod side, j / side); uv = r / side + stratum / side in fp32 (side a power of two, so the
// quotients are exact), r = (philox word >> 8) 2^-24 in [0, 1); pixel = trunc(uv (W, H)) clamped.
__device__ __forceinline__ uint32_t stratified_id(uint64_t seed, uint64_t step, long long j, int side_log2, int width,
                                                  int height) {
    const Philox4 r = philox4x32_10(Philox4{{uint32_t(j), uint32_t(uint64_t(j) >> 32), uint32_t(step),
                                             uint32_t(step >> 32)}},
                                    uint32_t(seed), uint32_t(seed >> 32));
    const float inv = __uint_as_float(uint32_t(127 - side_log2) << 23);  // 2^-side_log2, exact
    const long long sx = j & ((1LL << side_log2) - 1), sy = j >> side_log2;
    const float ux = __fadd_rn(__fmul_rn(float(r.v[0] >> 8) * 0x1p-24f, inv), __fmul_rn(float(sx), inv));
    const float uy = __fadd_rn(__fmul_rn(float(r.v[1] >> 8) * 0x1p-24f, inv), __fmul_rn(float(sy), inv));
    int x = int(__fmul_rn(ux, float(width))), y = int(__fmul_rn(uy, float(height)));
    x = x < width - 1 ? x : width - 1;
    y = y < height - 1 ? y : height - 1;
    return uint32_t(y) * uint32_t(width) + uint32_t(x);
}

__global__ void stratified_ids_kernel(uint64_t seed, uint64_t step, int side_log2, int width, int height, long long n,
                                      int64_t* __restrict__ ids) {
    const long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) ids[j] = stratified_id(seed, step, j, side_log2, width, height);
}

// The step's input stage with the sampler fused in: stratified id -> coordinates and target.
__global__ void stratified_batch_kernel(uint64_t seed, uint64_t step, int side_log2, long long n,
                                        const uint8_t* __restrict__ rgb, bool rgb8, int width, int height,
                                        RowFrame frame, float* __restrict__ xy, float* __restrict__ target) {
    const long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n)
        input_of(j, stratified_id(seed, step, j, side_log2, width, height), rgb, rgb8, width, height, frame, xy, target);
}

__global__ void coords_range_kernel(long long begin, long long n, int width, RowFrame frame, float* __restrict__ xy) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    reinterpret_cast<float2*>(xy)[i] = coords_of(uint32_t(begin + i), width, frame);
}

// Sum of the per-CTA partials of every head parameter, in a fixed order (deterministic): a block
// takes 32 parameters; slice k of its 8 threads per parameter sums partials k, k + 8, k + 16, ...
// in ascending order, then the 8 slice sums are added in slice order.
constexpr int RP_PARAMS = 32, RP_SLICES = 8;
__global__ void __launch_bounds__(RP_PARAMS * RP_SLICES) reduce_partials_kernel(const float* __restrict__ partials,
                                                                              int blocks, int count,
                                                                              float* __restrict__ out) {
    __shared__ float part[RP_SLICES][RP_PARAMS + 1];
    const int lane = threadIdx.x % RP_PARAMS, slice = threadIdx.x / RP_PARAMS;
    const int j = blockIdx.x * RP_PARAMS + lane;
    float s = 0.0f;
    if (j < count) {
#pragma unroll 4
        for (int b = slice; b < blocks; b += RP_SLICES) s = __fadd_rn(s, partials[(long long)b * count + j]);
    }
    part[slice][lane] = s;
    __syncthreads();
    if (slice == 0 && j < count) {
        float t = part[0][lane];
#pragma unroll
        for (int k = 1; k < RP_SLICES; ++k) t = __fadd_rn(t, part[k][lane]);
        out[j] = t;
    }
}

// One Adam update (fp32): m = fma(w1, g - m, m); v = fma(w2 * g, g, v * b2);
// p += (-step_size * m) / (sqrt(v) / bc2_sqrt + eps).
__device__ __forceinline__ void adam_update(float& p, float& m, float& v, float g, float step_size, float bc2_sqrt,
                                            float beta1w, float beta2, float beta2w, float eps) {
    m = __fmaf_rn(beta1w, __fsub_rn(g, m), m);
    v = __fmaf_rn(__fmul_rn(beta2w, g), g, __fmul_rn(v, beta2));
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), bc2_sqrt), eps);
    p = __fadd_rn(p, __fdiv_rn(__fmul_rn(-step_size, m), denom));
}

// One Adam segment: parameters, fp16 copy (null: none), moments, per-parameter steps, gradient, learning-rate table.
struct AdamSegment {
    float* master;
    __half* copy;
    float* m;
    float* v;
    uint32_t* steps;
    float* grad;
    long long count;
    const float* step_size;
};

// Quad q (VEC: parameters 4q..4q+3) or parameter q of a segment.
template <bool VEC>
__device__ __forceinline__ void adam_at(const AdamSegment& a, long long q, float inv_scale, const float* __restrict__ bc2_sqrt,
                                        long long table, float beta1w, float beta2, float beta2w, float eps,
                                        bool skip_zero, int* error_flag) {
    const long long count = a.count;
    if (VEC && (q + 1) * 4 <= count) {
        float4 g4 = reinterpret_cast<float4*>(a.grad)[q];
        if (skip_zero && g4.x == 0.0f && g4.y == 0.0f && g4.z == 0.0f && g4.w == 0.0f) return;
        float4 p4 = reinterpret_cast<float4*>(a.master)[q];
        float4 m4 = reinterpret_cast<float4*>(a.m)[q];
        float4 v4 = reinterpret_cast<float4*>(a.v)[q];
        uint4 s4 = reinterpret_cast<uint4*>(a.steps)[q];
        float* gp = &g4.x; float* pp = &p4.x; float* mp = &m4.x; float* vp = &v4.x; uint32_t* sp = &s4.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float gj = __fmul_rn(gp[j], inv_scale);
            if (skip_zero && gj == 0.0f) continue;
            const uint32_t s = ++sp[j];
            if ((long long)s > table) { atomicExch(error_flag, 1); continue; }
            adam_update(pp[j], mp[j], vp[j], gj, a.step_size[s - 1], bc2_sqrt[s - 1], beta1w, beta2, beta2w, eps);
        }
        reinterpret_cast<float4*>(a.master)[q] = p4;
        reinterpret_cast<float4*>(a.m)[q] = m4;
        reinterpret_cast<float4*>(a.v)[q] = v4;
        reinterpret_cast<uint4*>(a.steps)[q] = s4;
        reinterpret_cast<float4*>(a.grad)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (a.copy) {
            __half2* ch = reinterpret_cast<__half2*>(a.copy + 4 * q);
            ch[0] = __floats2half2_rn(p4.x, p4.y);
            ch[1] = __floats2half2_rn(p4.z, p4.w);
        }
        return;
    }
    const long long first = VEC ? 4 * q : q, last = VEC ? (4 * q + 4 < count ? 4 * q + 4 : count) : (q < count ? q + 1 : q);
    for (long long i = first; i < last; ++i) {
        const float gj = __fmul_rn(a.grad[i], inv_scale);
        if (skip_zero && gj == 0.0f) continue;
        const uint32_t s = ++a.steps[i];
        if ((long long)s > table) { atomicExch(error_flag, 1); continue; }
        float p = a.master[i], mi = a.m[i], vi = a.v[i];
        adam_update(p, mi, vi, gj, a.step_size[s - 1], bc2_sqrt[s - 1], beta1w, beta2, beta2w, eps);
        a.master[i] = p; a.m[i] = mi; a.v[i] = vi; a.grad[i] = 0.0f;
        if (a.copy) a.copy[i] = __float2half_rn(p);
    }
}

// Four parameters per thread (16-byte vectors) when every array is 16-byte
// aligned; one per thread otherwise.  Blocks [0, blocks0) update segment s0, the rest s1
// (s1.count == 0: one segment).
template <bool VEC>
__global__ void adam_kernel(const AdamSegment s0, const AdamSegment s1, long long blocks0, float inv_scale,
                            const float* __restrict__ bc2_sqrt, long long table, float beta1w, float beta2,
                            float beta2w, float eps, bool skip_zero, int* error_flag) {
    const bool second = blockIdx.x >= blocks0;
    const long long q = (long long)(blockIdx.x - (second ? blocks0 : 0)) * blockDim.x + threadIdx.x;
    adam_at<VEC>(second ? s1 : s0, q, inv_scale, bc2_sqrt, table, beta1w, beta2, beta2w, eps, skip_zero, error_flag);
}

__global__ void zero_kernel(float* p, long long count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) p[i] = 0.0f;
}
__global__ void cast_half_kernel(const float* __restrict__ in, __half* __restrict__ out, long long count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) out[i] = __float2half_rn(in[i]);
}

}  // namespace

static RowFrame frame_of(RowFrame frame, int height) {
    if (frame.rows <= 0) frame = RowFrame{0, height};
    ODIE_REQUIRE(frame.row0 >= 0 && frame.rows >= 2 && (long long)frame.row0 + height <= frame.rows,
                 "the local rows must lie within the full image");
    return frame;
}

void launch_input_batch(const int64_t* ids, long long n, const uint8_t* rgb, bool rgb8, int width, int height,
                        RowFrame frame, float* xy, float* target, cudaStream_t stream) {
    if (n <= 0) return;
    frame = frame_of(frame, height);
    input_batch_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(ids, n, rgb, rgb8, width, height, frame, xy, target);
    note_launch();
}

// side_log2 of a stratified batch: n must be a square power of two (as the reference's sampler requires).
static int stratified_side_log2(long long n) {
    ODIE_REQUIRE(n >= 1 && n <= (1LL << 30) && (n & (n - 1)) == 0,
                 "stratified sampling requires a square power-of-two batch size");
    int log2n = 0;
    while ((1LL << log2n) < n) ++log2n;
    ODIE_REQUIRE(log2n % 2 == 0, "stratified sampling requires a square power-of-two batch size");
    return log2n / 2;
}

void launch_stratified_ids(uint64_t seed, uint64_t step, int width, int height, long long n, int64_t* ids,
                           cudaStream_t stream) {
    const int side_log2 = stratified_side_log2(n);
    ODIE_REQUIRE(width >= 2 && height >= 2, "the image needs at least 2 x 2 pixels");
    stratified_ids_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(seed, step, side_log2, width, height, n, ids);
    note_launch();
}

void launch_stratified_batch(uint64_t seed, uint64_t step, long long n, const uint8_t* rgb, bool rgb8, int width,
                             int height, RowFrame frame, float* xy, float* target, cudaStream_t stream) {
    const int side_log2 = stratified_side_log2(n);
    frame = frame_of(frame, height);
    stratified_batch_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(seed, step, side_log2, n, rgb, rgb8, width, height,
                                                                    frame, xy, target);
    note_launch();
}

void launch_coords_range(long long begin, long long n, int width, int height, RowFrame frame, float* xy,
                         cudaStream_t stream) {
    if (n <= 0) return;
    frame = frame_of(frame, height);
    coords_range_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(begin, n, width, frame, xy);
    note_launch();
}

void launch_reduce_partials(const float* partials, int blocks, int count, float* out, cudaStream_t stream) {
    if (count <= 0) return;
    reduce_partials_kernel<<<blocks_for(count, RP_PARAMS), RP_PARAMS * RP_SLICES, 0, stream>>>(partials, blocks, count,
                                                                                                out);
    note_launch();
}

static bool adam_vec(const AdamSegment& a) {
    auto aligned = [](const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; };
    return aligned(a.master, 16) && aligned(a.m, 16) && aligned(a.v, 16) && aligned(a.steps, 16) && aligned(a.grad, 16) &&
           (!a.copy || aligned(a.copy, 8));
}

static void launch_adam_segments(const AdamSegment& s0, const AdamSegment& s1, float inv_scale, const float* bc2_sqrt,
                                 long long table, float beta1w, float beta2, float beta2w, float eps, bool skip_zero,
                                 int* error_flag, cudaStream_t stream) {
    const bool vec = adam_vec(s0) && (s1.count == 0 || adam_vec(s1));
    const long long per = vec ? 4 : 1;
    const long long b0 = blocks_for((s0.count + per - 1) / per, 256), b1 = blocks_for((s1.count + per - 1) / per, 256);
    if (b0 + b1 == 0) return;
    if (vec)
        adam_kernel<true><<<unsigned(b0 + b1), 256, 0, stream>>>(s0, s1, b0, inv_scale, bc2_sqrt, table, beta1w, beta2,
                                                                 beta2w, eps, skip_zero, error_flag);
    else
        adam_kernel<false><<<unsigned(b0 + b1), 256, 0, stream>>>(s0, s1, b0, inv_scale, bc2_sqrt, table, beta1w, beta2,
                                                                  beta2w, eps, skip_zero, error_flag);
    note_launch();
}

void launch_adam(float* master, __half* copy, float* m, float* v, uint32_t* steps, float* grad, long long count,
                 float inv_scale, AdamTables tables, float beta1w, float beta2, float beta2w, float eps, bool skip_zero,
                 int* error_flag, cudaStream_t stream) {
    if (count <= 0) return;
    const AdamSegment s0{master, copy, m, v, steps, grad, count, tables.step_size};
    const AdamSegment none{master, copy, m, v, steps, grad, 0, tables.step_size};
    launch_adam_segments(s0, none, inv_scale, tables.bc2_sqrt, tables.size, beta1w, beta2, beta2w, eps, skip_zero,
                         error_flag, stream);
}

void launch_adam2(float* master0, float* master1, __half* copy, float* m, float* v, uint32_t* steps, float* grad,
                  long long count0, long long count1, float inv_scale, AdamTables tables0, AdamTables tables1,
                  float beta1w, float beta2, float beta2w, float eps, bool skip_zero, int* error_flag,
                  cudaStream_t stream) {
    ODIE_REQUIRE(tables0.bc2_sqrt == tables1.bc2_sqrt && tables0.size == tables1.size,
                 "the two segments share their bias-correction table");
    const AdamSegment s0{master0, copy, m, v, steps, grad, count0, tables0.step_size};
    const AdamSegment s1{master1, copy + count0, m + count0, v + count0, steps + count0, grad + count0, count1,
                         tables1.step_size};
    if (count0 <= 0) {
        launch_adam_segments(s1, AdamSegment{master1, copy, m, v, steps, grad, 0, tables1.step_size}, inv_scale,
                             tables1.bc2_sqrt, tables1.size, beta1w, beta2, beta2w, eps, skip_zero, error_flag, stream);
        return;
    }
    launch_adam_segments(s0, s1, inv_scale, tables0.bc2_sqrt, tables0.size, beta1w, beta2, beta2w, eps, skip_zero,
                         error_flag, stream);
}

void launch_zero(float* p, long long count, cudaStream_t stream) {
    if (count <= 0) return;
    zero_kernel<<<blocks_for(count, 256), 256, 0, stream>>>(p, count);
    note_launch();
}
void launch_cast_half(const float* in, __half* out, long long count, cudaStream_t stream) {
    if (count <= 0) return;
    cast_half_kernel<<<blocks_for(count, 256), 256, 0, stream>>>(in, out, count);
    note_launch();
}

}  // namespace odie
