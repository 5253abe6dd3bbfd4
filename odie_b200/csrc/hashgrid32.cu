// Single fp32 hash grid with a fused fp32 MLP on the CUDA cores.
//
// The single-expert fp32 configuration of the hash-grid encoding (the hashed
// multiresolution grid of odie/hash_grid.py:8-80 and odie/config.py:83-94 in
// fp32): L levels of F = 2 features (32 inputs), an MLP 32 -> 64 -> 64 -> 3
// without biases (row-major [out][in] weights, the TCNN FullyFusedMLP
// topology), ReLU hidden layers and a sigmoid output; coordinates uniform in
// [0, 1)^2 from Philox4x32-10, targets bilinearly sampled from an fp32 RGB
// image, mean squared error over the batch's 3 n values, dense Adam.
//
// One training step:
//   hg32_train_kernel (persistent, 128 coordinates per tile, thread = coordinate):
//     coordinates + bilinear target + fp32 gather of the 16 levels
//     -> MLP forward / loss / backward in registers (weights in shared memory)
//     -> weight gradients as tile products over the 128 coordinates from shared
//        memory, accumulated in registers across the CTA's tiles, written once
//        as per-CTA partials
//     -> feature gradients [n][32] and the coordinates for the scatter
//   encode scatter (encode.cu, fp32 values) -> reduce_partials -> Adam (grid, heads).
// Every dot product is one fma chain in ascending input order starting from
// zero, so a CPU restatement with fmaf reproduces the features, activations
// and logits bit for bit.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <sstream>
#include <vector>

#include "encode.cuh"
#include "json_lite.hpp"
#include "odie_b200.h"
#include "step.cuh"

namespace odie {

long long hash_grid_table(const Json& enc, LevelTable& table, int& levels, int& F);

namespace {

constexpr int HG_IN = 32, HG_HID = 64, HG_OUT = 3;
constexpr int HG_W1 = HG_HID * HG_IN, HG_W2 = HG_HID * HG_HID, HG_W3 = HG_OUT * HG_HID;
constexpr int HG_PARAMS = HG_W1 + HG_W2 + HG_W3;  // 6336
constexpr int HG_TILE = 128;                      // coordinates per tile = threads per CTA

// Shared memory (floats).  Weights [in][out] (one float4 holds four outputs of one input); activations of
// the tile's 128 coordinates row-major with the 16-byte chunks of row r XOR-swizzled by r mod 8, so a
// thread's own row and one row read by every thread are both free of bank conflicts.
struct HgSmem {
    static constexpr int w1t = 0;              // [32][64]
    static constexpr int w2t = w1t + HG_W1;    // [64][64]
    static constexpr int w3t = w2t + HG_W2;    // [64][4]: three outputs and a zero
    static constexpr int x = w3t + 4 * HG_HID;  // [128][32] features
    static constexpr int h1 = x + HG_TILE * HG_IN;   // [128][64] hidden 1, then its gradient
    static constexpr int h2 = h1 + HG_TILE * HG_HID;  // [128][64] hidden 2, then its gradient
    static constexpr int dout = h2 + HG_TILE * HG_HID;  // [128][4] output gradients
    static constexpr int total = dout + 4 * HG_TILE;
    static constexpr int bytes = total * 4;
};

// Float index of (row, col) in a swizzled [128][width] buffer (width 32 or 64).
__device__ __forceinline__ int sw(int row, int col, int width) {
    return row * width + ((((col >> 2) ^ (row & 7))) << 2) + (col & 3);
}

struct HgArgs {
    long long n;
    uint64_t seed, step;
    const float* xy_in;   // [n][2] coordinates, or null: Philox uniform coordinates of (seed, step)
    const float* image;   // fp32 [height][width][3] target (training)
    int width, height;
    const float* table;   // fp32 grid
    const float* weights; // fp32 [W1 64x32 | W2 64x64 | W3 3x64], row-major [out][in]
    float loss_scale;     // dL/dy = loss_scale (y - target)
    float* xy;            // [n][2] coordinates of the step (training)
    float* dx;            // [n][32] feature gradients (training)
    float* squares;       // [n] mean of the 3 squared errors (training)
    float* partials;      // [gridDim.x][6336] weight-gradient partials (training)
    float* rgb;           // [n][3] prediction (decode)
    long long begin;      // decode without coordinates: pixels [begin, begin + n) of the image
};

// Uniform coordinate of slot i: (philox word >> 8) 2^-24 for x and y, key seed, counter (i, step).
__device__ __forceinline__ float2 uniform_xy(uint64_t seed, uint64_t step, long long i) {
    const Philox4 r = philox4x32_10(Philox4{{uint32_t(i), uint32_t(uint64_t(i) >> 32), uint32_t(step),
                                             uint32_t(step >> 32)}},
                                    uint32_t(seed), uint32_t(seed >> 32));
    return make_float2(float(r.v[0] >> 8) * 0x1p-24f, float(r.v[1] >> 8) * 0x1p-24f);
}

// Bilinear sample of the fp32 image at (x, y) in [0, 1]^2, pixel centres at (col / (W - 1), row / (H - 1)):
// p = fp32(x (W - 1)), corner = min(trunc(p), W - 2), f = p - corner; weights as geometry()'s; the four
// corners summed as one fma chain from the (0, 0) product.
__device__ __forceinline__ void bilinear(const float* __restrict__ image, int width, int height, float x, float y,
                                         float (&t)[3]) {
    const float px = __fmul_rn(x, float(width - 1)), py = __fmul_rn(y, float(height - 1));
    int x0 = int(px), y0 = int(py);
    x0 = x0 < 0 ? 0 : (x0 > width - 2 ? width - 2 : x0);
    y0 = y0 < 0 ? 0 : (y0 > height - 2 ? height - 2 : y0);
    const float fx = __fsub_rn(px, float(x0)), fy = __fsub_rn(py, float(y0));
    const float gx = __fsub_rn(1.0f, fx), gy = __fsub_rn(1.0f, fy);
    const float w00 = __fmul_rn(gx, gy), w10 = __fmul_rn(fx, gy), w01 = __fmul_rn(gx, fy), w11 = __fmul_rn(fx, fy);
    const float* p00 = image + 3 * ((long long)y0 * width + x0);
    const float* p01 = p00 + 3LL * width;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
        float s = __fmul_rn(w00, __ldg(p00 + c));
        s = __fmaf_rn(w10, __ldg(p00 + 3 + c), s);
        s = __fmaf_rn(w01, __ldg(p01 + c), s);
        t[c] = __fmaf_rn(w11, __ldg(p01 + 3 + c), s);
    }
}

// The 32 fp32 features of (x, y): per level the 4 corner pairs, fma chain over the corners from zero.
// Levels [0, split) are dense, [split, 16) hashed (the hash grid's order).
__device__ __forceinline__ void gather(const LevelTable& table, int split, const float* __restrict__ grid, float x,
                                       float y, float (&f)[HG_IN]) {
#pragma unroll
    for (int l = 0; l < HG_IN / 2; ++l) {
        const Level d = table.level[l];
        const Corner4 g = geometry(x, y, d.scale);
        float2 t[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int row = l < split ? corner_row<HASH_DENSE>(d, g, k, nullptr, nullptr)
                                      : corner_row<HASH_HASHED>(d, g, k, nullptr, nullptr);
            t[k] = __ldg(reinterpret_cast<const float2*>(grid + d.offset) + row);
        }
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a0 = __fmaf_rn(g.w[k], t[k].x, a0);
            a1 = __fmaf_rn(g.w[k], t[k].y, a1);
        }
        f[2 * l] = a0;
        f[2 * l + 1] = a1;
    }
}

// The same features written straight into row r of the swizzled [128][32] feature buffer, one level at a
// time (the training kernel: no register array for the row).
__device__ __forceinline__ void gather_row(const LevelTable& table, int split, const float* __restrict__ grid, float x,
                                           float y, bool valid, float* X, int r) {
#pragma unroll 4
    for (int l = 0; l < HG_IN / 2; ++l) {
        const Level d = table.level[l];
        const Corner4 g = geometry(x, y, d.scale);
        float2 t[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int row = l < split ? corner_row<HASH_DENSE>(d, g, k, nullptr, nullptr)
                                      : corner_row<HASH_HASHED>(d, g, k, nullptr, nullptr);
            t[k] = __ldg(reinterpret_cast<const float2*>(grid + d.offset) + row);
        }
        float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            a0 = __fmaf_rn(g.w[k], t[k].x, a0);
            a1 = __fmaf_rn(g.w[k], t[k].y, a1);
        }
        *reinterpret_cast<float2*>(X + sw(r, 2 * l, HG_IN)) = valid ? make_float2(a0, a1) : make_float2(0.0f, 0.0f);
    }
}

// Weights [out][in] from global memory into the [in][out] shared layout.
__device__ void stage_weights(const float* __restrict__ w, float* s) {
    for (int i = threadIdx.x; i < HG_W1; i += blockDim.x) {
        const int o = i / HG_IN, in = i % HG_IN;
        s[HgSmem::w1t + in * HG_HID + o] = w[i];
    }
    for (int i = threadIdx.x; i < HG_W2; i += blockDim.x) {
        const int o = i / HG_HID, in = i % HG_HID;
        s[HgSmem::w2t + in * HG_HID + o] = w[HG_W1 + i];
    }
    for (int i = threadIdx.x; i < 4 * HG_HID; i += blockDim.x) {
        const int in = i / 4, o = i % 4;
        s[HgSmem::w3t + i] = o < HG_OUT ? w[HG_W1 + HG_W2 + o * HG_HID + in] : 0.0f;
    }
}

// h = relu(W x) for the 64 outputs of one layer: outer loop over the inputs (one register each), the
// weights of four outputs per 16-byte shared-memory load (the same address for every thread).
template <int IN>
__device__ __forceinline__ void dense_relu(const float* __restrict__ wt, const float (&in)[IN], float (&h)[HG_HID]) {
#pragma unroll
    for (int o = 0; o < HG_HID; ++o) h[o] = 0.0f;
#pragma unroll
    for (int i = 0; i < IN; ++i) {
        const float v = in[i];
        const float4* w = reinterpret_cast<const float4*>(wt + i * HG_HID);
#pragma unroll
        for (int q = 0; q < HG_HID / 4; ++q) {
            const float4 c = w[q];
            h[4 * q] = __fmaf_rn(c.x, v, h[4 * q]);
            h[4 * q + 1] = __fmaf_rn(c.y, v, h[4 * q + 1]);
            h[4 * q + 2] = __fmaf_rn(c.z, v, h[4 * q + 2]);
            h[4 * q + 3] = __fmaf_rn(c.w, v, h[4 * q + 3]);
        }
    }
#pragma unroll
    for (int o = 0; o < HG_HID; ++o) h[o] = h[o] > 0.0f ? h[o] : 0.0f;
}

// The three logits of h2 (fma chain over the inputs in ascending order).
__device__ __forceinline__ void logits(const float* __restrict__ w3t, const float (&h)[HG_HID], float (&o)[HG_OUT]) {
    o[0] = o[1] = o[2] = 0.0f;
#pragma unroll
    for (int i = 0; i < HG_HID; ++i) {
        const float4 c = reinterpret_cast<const float4*>(w3t)[i];
        o[0] = __fmaf_rn(c.x, h[i], o[0]);
        o[1] = __fmaf_rn(c.y, h[i], o[1]);
        o[2] = __fmaf_rn(c.z, h[i], o[2]);
    }
}

__device__ __forceinline__ float sigmoid(float z) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z))); }

// Row r of a swizzled [128][W] buffer from W registers.
template <int W>
__device__ __forceinline__ void store_row(float* buf, int r, const float (&v)[W]) {
#pragma unroll
    for (int q = 0; q < W / 4; ++q)
        *reinterpret_cast<float4*>(buf + sw(r, 4 * q, W)) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
}

// h = relu(W in) for the 64 outputs of a layer whose inputs are row r of a swizzled [128][IN] buffer: one
// input at a time (one shared-memory load), the weights of four outputs per 16-byte load.
template <int IN>
__device__ __forceinline__ void dense_row(const float* __restrict__ wt, const float* buf, int r, float (&h)[HG_HID]) {
#pragma unroll
    for (int o = 0; o < HG_HID; ++o) h[o] = 0.0f;
#pragma unroll 1
    for (int i = 0; i < IN; ++i) {
        const float v = buf[sw(r, i, IN)];
        const float4* w = reinterpret_cast<const float4*>(wt + i * HG_HID);
#pragma unroll
        for (int q = 0; q < HG_HID / 4; ++q) {
            const float4 c = w[q];
            h[4 * q] = __fmaf_rn(c.x, v, h[4 * q]);
            h[4 * q + 1] = __fmaf_rn(c.y, v, h[4 * q + 1]);
            h[4 * q + 2] = __fmaf_rn(c.z, v, h[4 * q + 2]);
            h[4 * q + 3] = __fmaf_rn(c.w, v, h[4 * q + 3]);
        }
    }
#pragma unroll
    for (int o = 0; o < HG_HID; ++o) h[o] = h[o] > 0.0f ? h[o] : 0.0f;
}

// DOT_OUTPUTS dot products at once (independent fma chains): out[u] = (row u of the [.][64] weights at w) . v,
// each one chain over ascending k from zero.
constexpr int DOT_OUTPUTS = 8;
__device__ __forceinline__ void dots(const float* w, const float (&v)[HG_HID], float (&out)[DOT_OUTPUTS]) {
#pragma unroll
    for (int u = 0; u < DOT_OUTPUTS; ++u) out[u] = 0.0f;
#pragma unroll
    for (int q = 0; q < HG_HID / 4; ++q) {
#pragma unroll
        for (int u = 0; u < DOT_OUTPUTS; ++u) {
            const float4 c = *reinterpret_cast<const float4*>(w + u * HG_HID + 4 * q);
            out[u] = __fmaf_rn(c.x, v[4 * q], out[u]);
            out[u] = __fmaf_rn(c.y, v[4 * q + 1], out[u]);
            out[u] = __fmaf_rn(c.z, v[4 * q + 2], out[u]);
            out[u] = __fmaf_rn(c.w, v[4 * q + 3], out[u]);
        }
    }
}

// Row r of a swizzled [128][64] buffer into 64 registers.
__device__ __forceinline__ void load_row(const float* buf, int r, float (&v)[HG_HID]) {
#pragma unroll
    for (int q = 0; q < HG_HID / 4; ++q) {
        const float4 u = *reinterpret_cast<const float4*>(buf + sw(r, 4 * q, HG_HID));
        v[4 * q] = u.x;
        v[4 * q + 1] = u.y;
        v[4 * q + 2] = u.z;
        v[4 * q + 3] = u.w;
    }
}

// The tile's data path keeps one 64-wide vector and the weight-gradient accumulators in registers; each
// layer's input is read back from the thread's own shared-memory row.
__global__ void __launch_bounds__(HG_TILE, 2) hg32_train_kernel(const HgArgs a, const __grid_constant__ LevelTable table,
                                                                int split) {
    extern __shared__ __align__(16) float smem[];
    const int t = threadIdx.x;
    stage_weights(a.weights, smem);
    const float* w1t = smem + HgSmem::w1t;
    const float* w2t = smem + HgSmem::w2t;
    const float* w3t = smem + HgSmem::w3t;
    float* X = smem + HgSmem::x;
    float* H1 = smem + HgSmem::h1;
    float* H2 = smem + HgSmem::h2;
    float* DO = smem + HgSmem::dout;
    // Weight-gradient accumulators of this thread, kept across the CTA's tiles:
    //   dW2 rows 4 jb .. 4 jb + 3, columns {4 kb .. 4 kb + 3} and {32 + 4 kb .. 32 + 4 kb + 3}
    //   dW1 rows 4 jb .. 4 jb + 3, columns 4 kb .. 4 kb + 3
    //   dW3 column t (t < 64), its three rows
    const int jb = t >> 3, kb = t & 7;
    float g2[4][8], g1[4][4], g3[3];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
#pragma unroll
        for (int c = 0; c < 8; ++c) g2[r][c] = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; ++c) g1[r][c] = 0.0f;
    }
    g3[0] = g3[1] = g3[2] = 0.0f;
    __syncthreads();

    const long long tiles = (a.n + HG_TILE - 1) / HG_TILE;
    for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const long long i = tile * HG_TILE + t;
        const bool valid = i < a.n;
        // ---- inputs, features, hidden layer 1
        float2 p = make_float2(0.0f, 0.0f);
        float target[3] = {0.0f, 0.0f, 0.0f};
        if (valid) {
            p = a.xy_in ? __ldg(reinterpret_cast<const float2*>(a.xy_in) + i) : uniform_xy(a.seed, a.step, i);
            reinterpret_cast<float2*>(a.xy)[i] = p;
            bilinear(a.image, a.width, a.height, p.x, p.y, target);
        }
        uint64_t m1 = 0, m2 = 0;  // ReLU masks: bit o set where hidden output o is positive
        float h[HG_HID];          // hidden 1, then hidden 2, then the hidden-2 gradient, then the hidden-1 gradient
        gather_row(table, split, a.table, p.x, p.y, valid, X, t);
        dense_row<HG_IN>(w1t, X, t, h);  // the features read back from this thread's X row
        store_row(H1, t, h);
#pragma unroll
        for (int o = 0; o < HG_HID; ++o) m1 |= uint64_t(h[o] > 0.0f) << o;
        // ---- hidden layer 2: the inputs read back from this thread's H1 row
        dense_row<HG_HID>(w2t, H1, t, h);
#pragma unroll
        for (int o = 0; o < HG_HID; ++o) m2 |= uint64_t(h[o] > 0.0f) << o;
        store_row(H2, t, h);
        // ---- sigmoid output, loss, output gradient (h2 read back from this thread's H2 row)
        float z[HG_OUT] = {0.0f, 0.0f, 0.0f};
#pragma unroll 8
        for (int j = 0; j < HG_HID; ++j) {
            const float4 c = reinterpret_cast<const float4*>(w3t)[j];
            const float v = H2[sw(t, j, HG_HID)];
            z[0] = __fmaf_rn(c.x, v, z[0]);
            z[1] = __fmaf_rn(c.y, v, z[1]);
            z[2] = __fmaf_rn(c.z, v, z[2]);
        }
        float dz[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (valid) {
            float s = 0.0f;
#pragma unroll
            for (int c = 0; c < HG_OUT; ++c) {
                const float y = sigmoid(z[c]);
                const float d = __fsub_rn(y, target[c]);
                s = __fmaf_rn(d, d, s);
                dz[c] = __fmul_rn(__fmul_rn(__fmul_rn(a.loss_scale, d), y), __fsub_rn(1.0f, y));
            }
            a.squares[i] = __fdiv_rn(s, 3.0f);
        }
        *reinterpret_cast<float4*>(DO + 4 * t) = make_float4(dz[0], dz[1], dz[2], 0.0f);
        __syncthreads();  // X, H1, H2 and DO of every coordinate are in place
        // ---- dW3 += DO^T H2 (thread t < 64: column t)
        if (t < HG_HID) {
#pragma unroll 4
            for (int r = 0; r < HG_TILE; ++r) {
                const float hv = H2[sw(r, t, HG_HID)];
                const float4 d = *reinterpret_cast<const float4*>(DO + 4 * r);
                g3[0] = __fmaf_rn(d.x, hv, g3[0]);
                g3[1] = __fmaf_rn(d.y, hv, g3[1]);
                g3[2] = __fmaf_rn(d.z, hv, g3[2]);
            }
        }
        __syncthreads();  // H2 is free
        // ---- hidden-2 gradient (W3^T dz) masked, into this thread's H2 row
#pragma unroll 8
        for (int j = 0; j < HG_HID; ++j) {
            const float4 c = reinterpret_cast<const float4*>(w3t)[j];
            float sum = __fmul_rn(c.x, dz[0]);
            sum = __fmaf_rn(c.y, dz[1], sum);
            sum = __fmaf_rn(c.z, dz[2], sum);
            H2[sw(t, j, HG_HID)] = (m2 >> j & 1) ? sum : 0.0f;
        }
        __syncthreads();  // DH2 of every coordinate is in place
        // ---- dW2 += DH2^T H1
#pragma unroll 2
        for (int r = 0; r < HG_TILE; ++r) {
            const float4 d = *reinterpret_cast<const float4*>(H2 + sw(r, 4 * jb, HG_HID));
            const float4 u = *reinterpret_cast<const float4*>(H1 + sw(r, 4 * kb, HG_HID));
            const float4 v = *reinterpret_cast<const float4*>(H1 + sw(r, 32 + 4 * kb, HG_HID));
            const float dd[4] = {d.x, d.y, d.z, d.w}, hh[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
            for (int a2 = 0; a2 < 4; ++a2)
#pragma unroll
                for (int c = 0; c < 8; ++c) g2[a2][c] = __fmaf_rn(dd[a2], hh[c], g2[a2][c]);
        }
        __syncthreads();  // H1 is free
        // ---- hidden-1 gradient: output j = (w2t row j) . dh2 over ascending k, masked; into this thread's H1 row
        load_row(H2, t, h);
#pragma unroll 1
        for (int j0 = 0; j0 < HG_HID; j0 += DOT_OUTPUTS) {
            float sum[DOT_OUTPUTS];
            dots(w2t + j0 * HG_HID, h, sum);
#pragma unroll
            for (int u = 0; u < DOT_OUTPUTS; ++u) H1[sw(t, j0 + u, HG_HID)] = (m1 >> (j0 + u) & 1) ? sum[u] : 0.0f;
        }
        // ---- feature gradients dx = W1^T dh1 (ascending j), written for the scatter
        load_row(H1, t, h);
        if (valid) {
            float4* dst = reinterpret_cast<float4*>(a.dx + i * HG_IN);
#pragma unroll 1
            for (int m0 = 0; m0 < HG_IN; m0 += DOT_OUTPUTS) {
                float sum[DOT_OUTPUTS];
                dots(w1t + m0 * HG_HID, h, sum);
#pragma unroll
                for (int u = 0; u < DOT_OUTPUTS; u += 4)
                    dst[(m0 + u) / 4] = make_float4(sum[u], sum[u + 1], sum[u + 2], sum[u + 3]);
            }
        }
        __syncthreads();  // DH1 of every coordinate is in place
        // ---- dW1 += DH1^T X
#pragma unroll 2
        for (int r = 0; r < HG_TILE; ++r) {
            const float4 d = *reinterpret_cast<const float4*>(H1 + sw(r, 4 * jb, HG_HID));
            const float4 u = *reinterpret_cast<const float4*>(X + sw(r, 4 * kb, HG_IN));
            const float dd[4] = {d.x, d.y, d.z, d.w}, xx[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int a1 = 0; a1 < 4; ++a1)
#pragma unroll
                for (int c = 0; c < 4; ++c) g1[a1][c] = __fmaf_rn(dd[a1], xx[c], g1[a1][c]);
        }
        __syncthreads();  // the next tile may overwrite every buffer
    }
    // ---- this CTA's weight-gradient partials: [W1 | W2 | W3], row-major [out][in]
    float* part = a.partials + (long long)blockIdx.x * HG_PARAMS;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int j = 4 * jb + r;
        *reinterpret_cast<float4*>(part + j * HG_IN + 4 * kb) = make_float4(g1[r][0], g1[r][1], g1[r][2], g1[r][3]);
        float* row2 = part + HG_W1 + j * HG_HID;
        *reinterpret_cast<float4*>(row2 + 4 * kb) = make_float4(g2[r][0], g2[r][1], g2[r][2], g2[r][3]);
        *reinterpret_cast<float4*>(row2 + 32 + 4 * kb) = make_float4(g2[r][4], g2[r][5], g2[r][6], g2[r][7]);
    }
    if (t < HG_HID)
#pragma unroll
        for (int c = 0; c < HG_OUT; ++c) part[HG_W1 + HG_W2 + c * HG_HID + t] = g3[c];
}

// Prediction of coordinates (caller's, or the pixel centres of pixels [begin, begin + n)), fp32 RGB.
__global__ void __launch_bounds__(128) hg32_decode_kernel(const HgArgs a, const __grid_constant__ LevelTable table,
                                                          int split) {
    extern __shared__ __align__(16) float smem[];
    stage_weights(a.weights, smem);
    __syncthreads();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n) return;
    float2 p;
    if (a.xy_in) {
        p = __ldg(reinterpret_cast<const float2*>(a.xy_in) + i);
    } else {  // the pixel's endpoint coordinates, fp32(col) x fp32(1 / (W - 1)) as the training inputs
        const long long id = a.begin + i;
        const float rx = float(1.0 / double(a.width - 1)), ry = float(1.0 / double(a.height - 1));
        p = make_float2(__fmul_rn(float(id % a.width), rx), __fmul_rn(float(id / a.width), ry));
    }
    float f[HG_IN], h1[HG_HID], h2[HG_HID], z[HG_OUT];
    gather(table, split, a.table, p.x, p.y, f);
    dense_relu(smem + HgSmem::w1t, f, h1);
    dense_relu(smem + HgSmem::w2t, h1, h2);
    logits(smem + HgSmem::w3t, h2, z);
#pragma unroll
    for (int c = 0; c < HG_OUT; ++c) a.rgb[3 * i + c] = sigmoid(z[c]);
}

constexpr double TABLE_STEPS32 = double(1 << 20);  // Adam steps the bias-correction tables cover

}  // namespace

// The single fp32 hash grid's trainer: caller-owned image, grid and head masters (updated in place);
// library-owned gradients, Adam state and per-batch buffers.
struct HashGrid32 {
    cudaStream_t stream = nullptr;
    int device = 0;
    long long capacity = 0, total = 0;
    int width = 0, height = 0, split = 16;
    const float* image = nullptr;
    float* grid = nullptr;
    float* heads = nullptr;
    LevelTable table{};
    double lr[2] = {1e-2, 1e-2}, beta1 = 0.9, beta2 = 0.99, eps = 1e-15;
    int blocks = 0;
    DeviceArray<float> grid_grad, grid_m, grid_v, head_grad, head_m, head_v, partials, xy, dx, squares;
    // optional stage timers: CUDA events around each stage's launches on the step's stream
    enum Stage { S_FUSED, S_SCATTER, S_REDUCE, S_ADAM_GRID, S_ADAM_HEADS, S_COUNT };
    static constexpr const char* STAGE_NAMES[S_COUNT] = {"fused_step", "encode_backward", "reduce_partials",
                                                         "adam_grid", "adam_heads"};
    static constexpr int EVENT_PAIRS = 2048;
    bool profiling = false;
    std::vector<cudaEvent_t> events;
    std::vector<int> event_stage;
    int recorded = 0;
    DeviceArray<uint32_t> grid_steps, head_steps;
    DeviceArray<float> bc2, step_size[2];
    DeviceArray<int> error_flag;

    explicit HashGrid32(const Json& j) {
        ODIE_CUDA(cudaGetDevice(&device));
        ODIE_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        image = reinterpret_cast<const float*>(j.at("image").as_u64());
        grid = reinterpret_cast<float*>(j.at("grid").as_u64());
        heads = reinterpret_cast<float*>(j.at("heads").as_u64());
        width = int(j.at("width").as_int());
        height = int(j.at("height").as_int());
        capacity = j.value("capacity", 1LL << 18);
        ODIE_REQUIRE(image && grid && heads, "image, grid and heads must be device pointers");
        ODIE_REQUIRE(width >= 2 && height >= 2, "the image needs at least 2 x 2 pixels");
        ODIE_REQUIRE(capacity >= 1 && capacity <= (1LL << 26), "capacity in [1, 2^26]");
        int levels = 0, F = 0;
        total = hash_grid_table(j.at("hash_encoding"), table, levels, F);
        ODIE_REQUIRE(levels == 16 && F == 2, "the fp32 hash grid has 16 levels of 2 features");
        if (j.contains("total")) ODIE_REQUIRE(j.at("total").as_int() == total, "grid size differs from the layout");
        split = 0;
        while (split < levels && table.level[split].kind == HASH_DENSE) ++split;
        for (int l = split; l < levels; ++l)
            ODIE_REQUIRE(table.level[l].kind == HASH_HASHED, "dense levels precede the hashed ones");
        lr[0] = j.value_double("grid_lr", 1e-2);
        lr[1] = j.value_double("head_lr", 1e-2);
        beta1 = j.value_double("beta1", 0.9);
        beta2 = j.value_double("beta2", 0.99);
        eps = j.value_double("eps", 1e-15);
        ODIE_REQUIRE(beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0 && eps >= 0.0, "invalid Adam settings");
        blocks = 2 * sm_count();
        grid_grad.allocate(total);
        grid_m.allocate(total);
        grid_v.allocate(total);
        grid_steps.allocate(total);
        head_grad.allocate(HG_PARAMS);
        head_m.allocate(HG_PARAMS);
        head_v.allocate(HG_PARAMS);
        head_steps.allocate(HG_PARAMS);
        partials.allocate((long long)blocks * HG_PARAMS);
        xy.allocate(2 * capacity);
        dx.allocate(HG_IN * capacity);
        squares.allocate(capacity);
        error_flag.allocate(1);
        for (auto* a : {&grid_grad, &grid_m, &grid_v, &head_grad, &head_m, &head_v}) a->zero(stream);
        grid_steps.zero(stream);
        head_steps.zero(stream);
        error_flag.zero(stream);
        // torch.optim.Adam's bias corrections, evaluated in double and rounded once
        const long long steps = (long long)TABLE_STEPS32;
        std::vector<float> host_bc2(steps), host_step(steps);
        bc2.allocate(steps);
        for (long long s = 0; s < steps; ++s) host_bc2[s] = float(std::sqrt(1.0 - std::pow(beta2, double(s + 1))));
        ODIE_CUDA(cudaMemcpy(bc2.ptr, host_bc2.data(), steps * 4, cudaMemcpyHostToDevice));
        for (int g = 0; g < 2; ++g) {
            step_size[g].allocate(steps);
            for (long long s = 0; s < steps; ++s) host_step[s] = float(lr[g] / (1.0 - std::pow(beta1, double(s + 1))));
            ODIE_CUDA(cudaMemcpy(step_size[g].ptr, host_step.data(), steps * 4, cudaMemcpyHostToDevice));
        }
        static std::atomic<unsigned long long> configured{0};
        ODIE_REQUIRE(device >= 0 && device < 64, "devices 0..63");  // one bit per device below
        if (!(configured.load() >> device & 1ull)) {
            ODIE_CUDA(cudaFuncSetAttribute(hg32_train_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, HgSmem::bytes));
            ODIE_CUDA(cudaFuncSetAttribute(hg32_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           HgSmem::x * 4));
            configured.fetch_or(1ull << device);
        }
        ODIE_CUDA(cudaStreamSynchronize(stream));
    }
    ~HashGrid32() {
        if (stream) {
            cudaStreamSynchronize(stream);
            cudaStreamDestroy(stream);
        }
        for (auto e : events) cudaEventDestroy(e);
    }

    void profile(bool enable) {
        ODIE_CUDA(cudaDeviceSynchronize());
        if (enable && events.empty()) {
            events.resize(2 * EVENT_PAIRS);
            for (auto& e : events) ODIE_CUDA(cudaEventCreate(&e));
            event_stage.assign(EVENT_PAIRS, -1);
        }
        profiling = enable;
        recorded = 0;
    }
    int stage_begin(Stage stage, cudaStream_t s) {
        if (!profiling || recorded >= EVENT_PAIRS) return -1;
        const int slot = recorded++;
        event_stage[slot] = stage;
        ODIE_CUDA(cudaEventRecord(events[2 * slot], s));
        return slot;
    }
    void stage_end(int slot, cudaStream_t s) {
        if (slot >= 0) ODIE_CUDA(cudaEventRecord(events[2 * slot + 1], s));
    }
    std::string profile_report() {
        ODIE_CUDA(cudaDeviceSynchronize());
        double ms[S_COUNT] = {0};
        int launches[S_COUNT] = {0};
        for (int i = 0; i < recorded; ++i) {
            float t = 0.0f;
            ODIE_CUDA(cudaEventElapsedTime(&t, events[2 * i], events[2 * i + 1]));
            ms[event_stage[i]] += t;
            launches[event_stage[i]] += 1;
        }
        std::ostringstream o;
        o << "{";
        for (int k = 0; k < S_COUNT; ++k)
            o << (k ? "," : "") << "\"" << STAGE_NAMES[k] << "\":{\"launches\":" << launches[k] << ",\"ms\":" << ms[k] << "}";
        o << "}";
        return o.str();
    }

    HgArgs args(long long n) const {
        HgArgs a{};
        a.n = n;
        a.image = image;
        a.width = width;
        a.height = height;
        a.table = grid;
        a.weights = heads;
        return a;
    }

    // One step on `n` coordinates: the caller's (device [n][2]) or Philox uniform ones of (seed, step).
    void step(uint64_t seed, uint64_t step_index, long long n, const float* xy_in, bool update, cudaStream_t s) {
        ODIE_REQUIRE(n >= 1 && n <= capacity, "batch size must be in [1, capacity]");
        HgArgs a = args(n);
        a.seed = seed;
        a.step = step_index;
        a.xy_in = xy_in;
        a.loss_scale = float(2.0 / (3.0 * double(n)));
        a.xy = xy.ptr;
        a.dx = dx.ptr;
        a.squares = squares.ptr;
        a.partials = partials.ptr;
        const long long tiles = (n + HG_TILE - 1) / HG_TILE;
        const int grid_blocks = int(std::min<long long>(tiles, blocks));
        int slot = stage_begin(S_FUSED, s);
        hg32_train_kernel<<<grid_blocks, HG_TILE, HgSmem::bytes, s>>>(a, table, split);
        note_launch();
        stage_end(slot, s);
        EncodeArgs e;
        e.coords = xy.ptr;
        e.n = n;
        e.levels = 16;
        e.active = 16;
        e.row_major = true;
        e.width = HG_IN;
        e.stride = n;
        LevelSource src;
        src.table = table;
        slot = stage_begin(S_SCATTER, s);
        launch_encode_backward(e, src, static_cast<const float*>(dx.ptr), grid_grad.ptr, s);
        stage_end(slot, s);
        slot = stage_begin(S_REDUCE, s);
        launch_reduce_partials(partials.ptr, grid_blocks, HG_PARAMS, head_grad.ptr, s);
        stage_end(slot, s);
        if (update) apply_update(s);
        ODIE_CUDA(cudaGetLastError());
    }

    // Adam on every parameter (dense: torch.optim.Adam's update), consuming both gradients.
    void apply_update(cudaStream_t s) {
        const float b1w = float(1.0 - beta1), b2 = float(beta2), b2w = float(1.0 - beta2), e32 = float(eps);
        const long long steps = (long long)TABLE_STEPS32;
        int slot = stage_begin(S_ADAM_GRID, s);
        launch_adam(grid, nullptr, grid_m.ptr, grid_v.ptr, grid_steps.ptr, grid_grad.ptr, total, 1.0f,
                    AdamTables{step_size[0].ptr, bc2.ptr, steps}, b1w, b2, b2w, e32, false, error_flag.ptr, s);
        stage_end(slot, s);
        slot = stage_begin(S_ADAM_HEADS, s);
        launch_adam(heads, nullptr, head_m.ptr, head_v.ptr, head_steps.ptr, head_grad.ptr, HG_PARAMS, 1.0f,
                    AdamTables{step_size[1].ptr, bc2.ptr, steps}, b1w, b2, b2w, e32, false, error_flag.ptr, s);
        stage_end(slot, s);
        ODIE_CUDA(cudaGetLastError());
    }

    void decode(long long begin, long long n, const float* xy_in, float* rgb, cudaStream_t s) {
        if (n <= 0) return;
        ODIE_REQUIRE(rgb, "decode needs an output buffer");
        ODIE_REQUIRE(xy_in || (begin >= 0 && begin + n <= (long long)width * height),
                     "decode pixels must lie within the image");
        HgArgs a = args(n);
        a.xy_in = xy_in;
        a.begin = begin;
        a.rgb = rgb;
        hg32_decode_kernel<<<blocks_for(n, 128), 128, HgSmem::x * 4, s>>>(a, table, split);
        note_launch();
        ODIE_CUDA(cudaGetLastError());
    }

    std::string pointers() const {
        std::ostringstream o;
        auto u = [](const void* p) { return (unsigned long long)reinterpret_cast<uintptr_t>(p); };
        o << "{\"stream\":" << u(stream) << ",\"grid_grad\":" << u(grid_grad.ptr) << ",\"grid_m\":" << u(grid_m.ptr)
          << ",\"grid_v\":" << u(grid_v.ptr) << ",\"grid_steps\":" << u(grid_steps.ptr)
          << ",\"head_grad\":" << u(head_grad.ptr) << ",\"head_m\":" << u(head_m.ptr) << ",\"head_v\":" << u(head_v.ptr)
          << ",\"head_steps\":" << u(head_steps.ptr) << ",\"xy\":" << u(xy.ptr) << ",\"dx\":" << u(dx.ptr)
          << ",\"squares\":" << u(squares.ptr) << ",\"error_flag\":" << u(error_flag.ptr) << ",\"total\":" << total
          << ",\"head_params\":" << HG_PARAMS << ",\"capacity\":" << capacity << ",\"blocks\":" << blocks
          << ",\"dense_levels\":" << split << "}";
        return o.str();
    }
};

}  // namespace odie

namespace {
thread_local std::string g_hg32_reply;
}

extern "C" {

void* odie_hashgrid32_create(const char* json) {
    try {
        return new odie::HashGrid32(odie::parse_json(json ? json : ""));
    } catch (const std::exception& e) {
        odie::set_error(e.what());
        return nullptr;
    }
}

int odie_hashgrid32_step(void* handle, uint64_t seed, uint64_t step, int64_t n, const float* xy, int update,
                         uint64_t stream) {
    return odie::guarded([&] {
        ODIE_REQUIRE(handle, "null handle");
        auto* h = static_cast<odie::HashGrid32*>(handle);
        h->step(seed, step, n, xy, update != 0, reinterpret_cast<cudaStream_t>(stream));
    });
}

int odie_hashgrid32_update(void* handle, uint64_t stream) {
    return odie::guarded([&] {
        ODIE_REQUIRE(handle, "null handle");
        auto* h = static_cast<odie::HashGrid32*>(handle);
        h->apply_update(reinterpret_cast<cudaStream_t>(stream));
    });
}

int odie_hashgrid32_decode(void* handle, int64_t begin, int64_t n, const float* xy, float* rgb, uint64_t stream) {
    return odie::guarded([&] {
        ODIE_REQUIRE(handle, "null handle");
        auto* h = static_cast<odie::HashGrid32*>(handle);
        h->decode(begin, n, xy, rgb, reinterpret_cast<cudaStream_t>(stream));
    });
}

const char* odie_hashgrid32_pointers(void* handle) {
    if (!handle) {
        odie::set_error("null handle");
        return nullptr;
    }
    g_hg32_reply = static_cast<odie::HashGrid32*>(handle)->pointers();
    return g_hg32_reply.c_str();
}

int odie_hashgrid32_profile(void* handle, int enable) {
    return odie::guarded([&] {
        ODIE_REQUIRE(handle, "null handle");
        static_cast<odie::HashGrid32*>(handle)->profile(enable != 0);
    });
}

const char* odie_hashgrid32_profile_report(void* handle) {
    try {
        ODIE_REQUIRE(handle, "null handle");
        g_hg32_reply = static_cast<odie::HashGrid32*>(handle)->profile_report();
        return g_hg32_reply.c_str();
    } catch (const std::exception& e) {
        odie::set_error(e.what());
        return nullptr;
    }
}

void odie_hashgrid32_destroy(void* handle) { delete static_cast<odie::HashGrid32*>(handle); }

}  // extern "C"
