// Warp-level tensor-core fragments for the small fused MLPs.
//
// Layout facts used throughout (PTX ISA, mma.m16n8k16 with .f16 inputs):
//  lane = 4*g + t (g = lane/4 in 0..7, t = lane%4)
//  A (16x16, row-major): a0 = A[g][2t..2t+1], a1 = A[g+8][2t..], a2 = A[g][8+2t..], a3 = A[g+8][8+2t..]
//  B (16x8, k x n):      b0 = B[2t..2t+1][g],  b1 = B[8+2t..8+2t+1][g]
//  C (16x8, fp32):       c0,c1 = C[g][2t..2t+1], c2,c3 = C[g+8][2t..2t+1]
// so the fp16 packing of two adjacent C tiles is exactly one A k-step, which
// keeps whole layer chains in registers.  movmatrix.trans transposes one 8x8
// block held in the C/A layout, which turns activation fragments into the
// transposed operands of the weight-gradient products.
#pragma once
#include "common.cuh"

namespace odie {
namespace mma {

__device__ __forceinline__ void m16n8k16(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(y) : "r"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float relu(float x) { return x > 0.0f ? x : 0.0f; }

// A fragment of k-step kk from a row-major fp16 matrix in shared memory.
__device__ __forceinline__ void load_a(uint32_t a[4], const __half* s, int ld, int kk, int g, int t) {
    const __half* base = s + 16 * kk + 2 * t;
    a[0] = *reinterpret_cast<const uint32_t*>(base + g * ld);
    a[1] = *reinterpret_cast<const uint32_t*>(base + (g + 8) * ld);
    a[2] = *reinterpret_cast<const uint32_t*>(base + g * ld + 8);
    a[3] = *reinterpret_cast<const uint32_t*>(base + (g + 8) * ld + 8);
}
// B fragment (k-step kk, n-tile nt) of B = M^T where M is a row-major [N][K] matrix in smem.
__device__ __forceinline__ void load_b(uint32_t& b0, uint32_t& b1, const __half* m, int ld, int nt, int kk, int g, int t) {
    const __half* base = m + (8 * nt + g) * ld + 16 * kk + 2 * t;
    b0 = *reinterpret_cast<const uint32_t*>(base);
    b1 = *reinterpret_cast<const uint32_t*>(base + 8);
}

// Two C tiles (2kk, 2kk+1) -> one A k-step (optionally ReLU'd first).
template <bool RELU>
__device__ __forceinline__ void c_to_a(uint32_t a[4], const float c0[4], const float c1[4]) {
    if (RELU) {
        a[0] = pack(relu(c0[0]), relu(c0[1]));
        a[1] = pack(relu(c0[2]), relu(c0[3]));
        a[2] = pack(relu(c1[0]), relu(c1[1]));
        a[3] = pack(relu(c1[2]), relu(c1[3]));
    } else {
        a[0] = pack(c0[0], c0[1]);
        a[1] = pack(c0[2], c0[3]);
        a[2] = pack(c1[0], c1[1]);
        a[3] = pack(c1[2], c1[3]);
    }
}

// Element e (0..3) of C tile nt, read from the A fragments of the same matrix
// (the fp16 activation a ReLU derivative is taken from).
__device__ __forceinline__ float a_elem(const uint32_t (*a)[4], int nt, int e) {
    const uint32_t r = a[nt >> 1][((nt & 1) << 1) + (e >> 1)];
    return __half2float((e & 1) ? hi_half(r) : lo_half(r));
}

// Transposed operands for dW += dO^T * In over the 16 rows of a tile:
// A = (dO^T) m-tile mo, B = In n-tile ni.
__device__ __forceinline__ void a_transposed(uint32_t out[4], const uint32_t in[4]) {
    out[0] = trans(in[0]);
    out[1] = trans(in[2]);
    out[2] = trans(in[1]);
    out[3] = trans(in[3]);
}
__device__ __forceinline__ void b_transposed(uint32_t& b0, uint32_t& b1, const uint32_t (*in)[4], int ni) {
    b0 = trans(in[ni >> 1][(ni & 1) << 1]);
    b1 = trans(in[ni >> 1][((ni & 1) << 1) + 1]);
}

}  // namespace mma
}  // namespace odie
