// Fused MLP heads of the training/decoding step, the input stage and Adam.
//
// mlp_train_kernel: one warp per tile of 16 coordinates, 4 warps per block,
// persistent over tiles.  Per tile, entirely in registers/shared memory:
//   gate MLP forward -> per-level sigmoid gate (odie/native/runtime.cu:66-75)
//   -> decoder MLP forward -> L2 loss gradient (runtime.cu:53-63)
//   -> decoder backward -> gate backward (runtime.cu:76-92) -> gate MLP
//   backward -> grid-gradient values (runtime.cu:117-125)
// and the weight gradients of both heads, accumulated per block in shared
// memory and written once per block as partials (no global atomics).
// Matrix products run on the tensor cores (mma.m16n8k16, fp16 in, fp32
// accumulate); every activation is rounded to fp16 where the reference's fp16
// network stores it.
#include "step.cuh"
#include "mlp.cuh"

namespace odie {

namespace {

constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int LD_G2 = GATE_HIDDEN + 8;   // 40
constexpr int LD_G2T = GATE_OUT + 8;     // 24
constexpr int LD_D = DEC_HIDDEN + 8;     // 72
constexpr int LD_D3T = DEC_OUT + 8;      // 24
constexpr int LD_TM = 72;
constexpr int LD_TQ = 24;

template <int W>
struct Smem {
    static constexpr int LDX = W + 8;
    // weights (halves)
    static constexpr int g1 = 0;                              // [32][LDX]
    static constexpr int g1t = g1 + GATE_HIDDEN * LDX;        // [W][40]
    static constexpr int g2 = g1t + W * LD_G2;                // [16][40]
    static constexpr int g2t = g2 + GATE_OUT * LD_G2;         // [32][24]
    static constexpr int d1 = g2t + GATE_HIDDEN * LD_G2T;     // [64][LDX]
    static constexpr int d1t = d1 + DEC_HIDDEN * LDX;         // [W][72]
    static constexpr int d2 = d1t + W * LD_D;                 // [64][72]
    static constexpr int d2t = d2 + DEC_HIDDEN * LD_D;        // [64][72]
    static constexpr int d3 = d2t + DEC_HIDDEN * LD_D;        // [16][72]
    static constexpr int d3t = d3 + DEC_OUT * LD_D;           // [64][24]
    static constexpr int weight_halves = d3t + DEC_HIDDEN * LD_D3T;
    static constexpr int weight_bytes = (weight_halves * 2 + 15) / 16 * 16;
    static constexpr int fmap_bytes = 128;
    static constexpr int head_params = gate_params(W) + decoder_params(W);
    static constexpr int acc_bytes = WARPS * head_params * 4;  // one private accumulator per warp
    // per-warp staging
    static constexpr int xs_bytes = 16 * LDX * 2;
    static constexpr int tm_bytes = 16 * LD_TM * 2;
    static constexpr int tq_bytes = 16 * LD_TQ * 2;
    static constexpr int sg_bytes = 16 * 16 * 4;
    static constexpr int vb_bytes = 16 * 4;
    static constexpr int warp_bytes = (xs_bytes + tm_bytes + tq_bytes + sg_bytes + vb_bytes + 15) / 16 * 16;
    static constexpr int train_bytes = weight_bytes + fmap_bytes + acc_bytes + WARPS * warp_bytes;
    static constexpr int decode_bytes = weight_bytes + fmap_bytes + WARPS * warp_bytes;
};

template <int W>
struct WarpBufs {
    __half* xs;
    __half* tm;
    __half* tq;
    float* sg;
    uint32_t* vb;
    __device__ WarpBufs(unsigned char* base) {
        xs = reinterpret_cast<__half*>(base);
        tm = reinterpret_cast<__half*>(base + Smem<W>::xs_bytes);
        tq = reinterpret_cast<__half*>(base + Smem<W>::xs_bytes + Smem<W>::tm_bytes);
        sg = reinterpret_cast<float*>(base + Smem<W>::xs_bytes + Smem<W>::tm_bytes + Smem<W>::tq_bytes);
        vb = reinterpret_cast<uint32_t*>(base + Smem<W>::xs_bytes + Smem<W>::tm_bytes + Smem<W>::tq_bytes +
                                         Smem<W>::sg_bytes);
    }
};

// Matrix src [rows][cols] (global fp16, row-major) -> smem copy [rows][ld] and
// transpose [cols][ldt].
__device__ void stage_matrix(const __half* __restrict__ src, int rows, int cols, __half* s, int ld, __half* st, int ldt) {
    for (int idx = threadIdx.x; idx < rows * cols; idx += blockDim.x) {
        const int r = idx / cols, c = idx - r * cols;
        const __half h = src[idx];
        s[r * ld + c] = h;
        st[c * ldt + r] = h;
    }
}

template <int W, bool ROUTER>
__device__ void stage_weights(const MlpArgs& a, __half* ws, int8_t* fmap) {
    using S = Smem<W>;
    if (ROUTER) {
        stage_matrix(a.gate_w, GATE_HIDDEN, W, ws + S::g1, S::LDX, ws + S::g1t, LD_G2);
        stage_matrix(a.gate_w + GATE_HIDDEN * W, GATE_OUT, GATE_HIDDEN, ws + S::g2, LD_G2, ws + S::g2t, LD_G2T);
    }
    stage_matrix(a.decoder_w, DEC_HIDDEN, W, ws + S::d1, S::LDX, ws + S::d1t, LD_D);
    stage_matrix(a.decoder_w + DEC_HIDDEN * W, DEC_HIDDEN, DEC_HIDDEN, ws + S::d2, LD_D, ws + S::d2t, LD_D);
    stage_matrix(a.decoder_w + DEC_HIDDEN * W + DEC_HIDDEN * DEC_HIDDEN, DEC_OUT, DEC_HIDDEN, ws + S::d3, LD_D,
                 ws + S::d3t, LD_D3T);
    const int8_t* src = reinterpret_cast<const int8_t*>(&a.fmap);
    for (int i = threadIdx.x; i < (int)sizeof(FeatureMap); i += blockDim.x) fmap[i] = src[i];
}

// Forward state of one tile that the backward reuses.
template <int W>
struct Fwd {
    uint32_t xa[W / 16][4];  // decoder/gate input (raw features, pad columns 1)
    uint32_t wa[W / 16][4];  // gated decoder input
    uint32_t gha[2][4];      // gate hidden activation
    uint32_t h1a[4][4];      // decoder hidden 1
    uint32_t h2a[4][4];      // decoder hidden 2
    float out[4];            // decoder output, n-tile 0 (columns 0..7)
};

__device__ __forceinline__ float sigmoid_gate(float z, int level, int k_fixed, int softplus) {
    if (level < k_fixed) return 1.0f;
    if (softplus) return z > 20.0f ? z : log1pf(expf(z));
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
}

template <int W, bool ROUTER>
__device__ __forceinline__ void forward_tile(const MlpArgs& a, long long r0, const __half* ws, const int8_t* fmap,
                                             WarpBufs<W>& wb, Fwd<W>& f, int lane) {
    using S = Smem<W>;
    constexpr int KW = W / 16;
    const int g = lane >> 2, t = lane & 3;
    // stage the tile's features (pair-major in global) and visibility bits
    const __half one = __float2half_rn(1.0f);
    for (int idx = lane; idx < 16 * (W / 2); idx += 32) {
        const int row = idx & 15, pair = idx >> 4;
        const long long i = r0 + row;
        uint32_t v = 0;
        if (i < a.n) v = __ldg(reinterpret_cast<const uint32_t*>(a.raw) + (long long)pair * a.stride + i);
        const int c0 = 2 * pair;
        if (c0 >= a.raw_width) v = pack_half2(one, one);
        else if (c0 + 1 >= a.raw_width) v = (v & 0xffffu) | (uint32_t(__half_as_ushort(one)) << 16);
        *reinterpret_cast<uint32_t*>(wb.xs + row * S::LDX + c0) = v;
    }
    if (lane < 16) {
        const long long i = r0 + lane;
        uint32_t mask = 0;
        if (i < a.n)
            for (int l = 0; l < a.levels; ++l) mask |= uint32_t(__ldg(a.vis + (long long)l * a.stride + i) != 0) << l;
        wb.vb[lane] = mask;
    }
    __syncwarp();
#pragma unroll
    for (int kk = 0; kk < KW; ++kk) mma::load_a(f.xa[kk], wb.xs, S::LDX, kk, g, t);

    if (ROUTER) {
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
            float c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < KW; ++kk) {
                uint32_t b0, b1;
                mma::load_b(b0, b1, ws + S::g1, S::LDX, 2 * k2, kk, g, t);
                mma::m16n8k16(c0, f.xa[kk], b0, b1);
                mma::load_b(b0, b1, ws + S::g1, S::LDX, 2 * k2 + 1, kk, g, t);
                mma::m16n8k16(c1, f.xa[kk], b0, b1);
            }
            mma::c_to_a<true>(f.gha[k2], c0, c1);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            float c[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                uint32_t b0, b1;
                mma::load_b(b0, b1, ws + S::g2, LD_G2, nt, kk, g, t);
                mma::m16n8k16(c, f.gha[kk], b0, b1);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = g + 8 * (e >> 1), col = 8 * nt + 2 * t + (e & 1);
                if (col < a.levels) {
                    const float z = __half2float(__float2half_rn(c[e]));
                    wb.sg[row * 16 + col] = sigmoid_gate(z, col, a.k_fixed, a.softplus);
                }
            }
        }
        __syncwarp();
        const FeatureMap* fm = reinterpret_cast<const FeatureMap*>(fmap);
#pragma unroll
        for (int kk = 0; kk < KW; ++kk)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int row = g + 8 * (j & 1), colbase = 16 * kk + 8 * (j >> 1) + 2 * t;
                __half h[2] = {lo_half(f.xa[kk][j]), hi_half(f.xa[kk][j])};
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int lev = fm->level_of_col[colbase + q];
                    if (lev >= 0) {
                        const float vis = float((wb.vb[row] >> lev) & 1u);
                        const __half weight = __float2half_rn(__fmul_rn(wb.sg[row * 16 + lev], vis));
                        h[q] = __hmul_rn(h[q], weight);
                    }
                }
                f.wa[kk][j] = pack_half2(h[0], h[1]);
            }
    } else {
#pragma unroll
        for (int kk = 0; kk < KW; ++kk)
#pragma unroll
            for (int j = 0; j < 4; ++j) f.wa[kk][j] = f.xa[kk][j];
    }
    // decoder
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
        float c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int kk = 0; kk < KW; ++kk) {
            uint32_t b0, b1;
            mma::load_b(b0, b1, ws + S::d1, S::LDX, 2 * k2, kk, g, t);
            mma::m16n8k16(c0, f.wa[kk], b0, b1);
            mma::load_b(b0, b1, ws + S::d1, S::LDX, 2 * k2 + 1, kk, g, t);
            mma::m16n8k16(c1, f.wa[kk], b0, b1);
        }
        mma::c_to_a<true>(f.h1a[k2], c0, c1);
    }
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
        float c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t b0, b1;
            mma::load_b(b0, b1, ws + S::d2, LD_D, 2 * k2, kk, g, t);
            mma::m16n8k16(c0, f.h1a[kk], b0, b1);
            mma::load_b(b0, b1, ws + S::d2, LD_D, 2 * k2 + 1, kk, g, t);
            mma::m16n8k16(c1, f.h1a[kk], b0, b1);
        }
        mma::c_to_a<true>(f.h2a[k2], c0, c1);
    }
    // output layer: only columns 0..2 are used, so only n-tile 0 is formed
#pragma unroll
    for (int e = 0; e < 4; ++e) f.out[e] = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        uint32_t b0, b1;
        mma::load_b(b0, b1, ws + S::d3, LD_D, 0, kk, g, t);
        mma::m16n8k16(f.out, f.h2a[kk], b0, b1);
    }
}

// dW[o][i] += sum_r dO[r][o] * In[r][i] for this tile: dO given as A fragments
// (MO m-tiles of 16 output rows), In as A fragments (NI n-tiles of 8 columns).
template <int MO, int NI>
__device__ __forceinline__ void accumulate_dw(float* acc, int ld, const uint32_t (*dO)[4], const uint32_t (*in)[4],
                                              int g, int t, int row_limit) {
#pragma unroll
    for (int mo = 0; mo < MO; ++mo) {
        uint32_t at[4];
        mma::a_transposed(at, dO[mo]);
#pragma unroll
        for (int ni = 0; ni < NI; ++ni) {
            uint32_t b0, b1;
            mma::b_transposed(b0, b1, in, ni);
            float c[4] = {0, 0, 0, 0};
            mma::m16n8k16(c, at, b0, b1);
            // the warp's private accumulator: plain read-modify-write, no atomics
            const int o0 = 16 * mo + g, col = 8 * ni + 2 * t;
            if (o0 < row_limit) {
                float2* p = reinterpret_cast<float2*>(acc + o0 * ld + col);
                float2 v = *p;
                v.x += c[0];
                v.y += c[1];
                *p = v;
            }
            if (o0 + 8 < row_limit) {
                float2* p = reinterpret_cast<float2*>(acc + (o0 + 8) * ld + col);
                float2 v = *p;
                v.x += c[2];
                v.y += c[3];
                *p = v;
            }
        }
    }
}

template <int W, bool ROUTER>
__global__ void __launch_bounds__(THREADS, 1) mlp_train_kernel(const MlpArgs a) {
    using S = Smem<W>;
    constexpr int NW = W / 8;
    extern __shared__ __align__(16) unsigned char smem[];
    __half* ws = reinterpret_cast<__half*>(smem);
    int8_t* fmap = reinterpret_cast<int8_t*>(smem + S::weight_bytes);
    float* acc_all = reinterpret_cast<float*>(smem + S::weight_bytes + S::fmap_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    WarpBufs<W> wb(smem + S::weight_bytes + S::fmap_bytes + S::acc_bytes + warp * S::warp_bytes);
    stage_weights<W, ROUTER>(a, ws, fmap);
    for (int i = threadIdx.x; i < WARPS * S::head_params; i += blockDim.x) acc_all[i] = 0.0f;
    __syncthreads();
    float* acc = acc_all + warp * S::head_params;  // this warp's weight-gradient accumulator
    float* dg1 = acc;                                   // [32][W]
    float* dg2 = dg1 + GATE_HIDDEN * W;                 // [16][32]
    // head parameters of this launch: gate | decoder, or decoder only without the router
    constexpr int GATE = ROUTER ? gate_params(W) : 0;
    constexpr int P = GATE + decoder_params(W);
    float* dd1 = acc + GATE;                            // [64][W]
    float* dd2 = dd1 + DEC_HIDDEN * W;                  // [64][64]
    float* dd3 = dd2 + DEC_HIDDEN * DEC_HIDDEN;         // [16][64]
    const FeatureMap* fm = reinterpret_cast<const FeatureMap*>(fmap);
    const long long tiles = (a.n + 15) / 16;
    for (long long tile = (long long)blockIdx.x * WARPS + warp; tile < tiles; tile += (long long)gridDim.x * WARPS) {
        const long long r0 = tile * 16;
        Fwd<W> f;
        forward_tile<W, ROUTER>(a, r0, ws, fmap, wb, f, lane);
        // ---- loss gradient (odie/native/runtime.cu:53-63)
        if (t < 2) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 2 * t + (e & 1), row = g + 8 * (e >> 1);
                if (col < 3) wb.tm[row * LD_TM + col] = __float2half_rn(f.out[e]);
            }
        }
        __syncwarp();
        if (lane < 16) {
            const long long i = r0 + lane;
            __half* dy = wb.tq + lane * LD_TQ;
            if (i < a.n) {
                float s = 0.0f;
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const float d = __fsub_rn(__half2float(wb.tm[lane * LD_TM + c]), __ldg(a.target + 3 * i + c));
                    s = __fadd_rn(s, __fmul_rn(d, d));
                    const float scaled = __fmul_rn(__fdiv_rn(__fmul_rn(2.0f, d), a.three_real), 128.0f);
                    dy[c] = __hmul_rn(__float2half_rn(scaled), __float2half_rn(128.0f));
                }
                a.squares[i] = __fdiv_rn(s, 3.0f);
            } else {
#pragma unroll
                for (int c = 0; c < 3; ++c) dy[c] = __float2half_rn(0.0f);
            }
#pragma unroll
            for (int c = 3; c < 16; ++c) dy[c] = __float2half_rn(0.0f);
        }
        __syncwarp();
        uint32_t dya[1][4];
        mma::load_a(dya[0], wb.tq, LD_TQ, 0, g, t);
        // ---- decoder backward
        uint32_t dh2a[4][4];
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
            float c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
            uint32_t b0, b1;
            mma::load_b(b0, b1, ws + S::d3t, LD_D3T, 2 * k2, 0, g, t);
            mma::m16n8k16(c0, dya[0], b0, b1);
            mma::load_b(b0, b1, ws + S::d3t, LD_D3T, 2 * k2 + 1, 0, g, t);
            mma::m16n8k16(c1, dya[0], b0, b1);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (!(mma::a_elem(f.h2a, 2 * k2, e) > 0.0f)) c0[e] = 0.0f;
                if (!(mma::a_elem(f.h2a, 2 * k2 + 1, e) > 0.0f)) c1[e] = 0.0f;
            }
            mma::c_to_a<false>(dh2a[k2], c0, c1);
        }
        accumulate_dw<1, 8>(dd3, DEC_HIDDEN, dya, f.h2a, g, t, 3);
        uint32_t dh1a[4][4];
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2) {
            float c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                uint32_t b0, b1;
                mma::load_b(b0, b1, ws + S::d2t, LD_D, 2 * k2, kk, g, t);
                mma::m16n8k16(c0, dh2a[kk], b0, b1);
                mma::load_b(b0, b1, ws + S::d2t, LD_D, 2 * k2 + 1, kk, g, t);
                mma::m16n8k16(c1, dh2a[kk], b0, b1);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (!(mma::a_elem(f.h1a, 2 * k2, e) > 0.0f)) c0[e] = 0.0f;
                if (!(mma::a_elem(f.h1a, 2 * k2 + 1, e) > 0.0f)) c1[e] = 0.0f;
            }
            mma::c_to_a<false>(dh1a[k2], c0, c1);
        }
        accumulate_dw<4, 8>(dd2, DEC_HIDDEN, dh2a, f.h1a, g, t, DEC_HIDDEN);
        // dz = dh1 * W1 (fp16), staged row-major in tm
#pragma unroll
        for (int nt = 0; nt < NW; ++nt) {
            float c[4] = {0, 0, 0, 0};
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                uint32_t b0, b1;
                mma::load_b(b0, b1, ws + S::d1t, LD_D, nt, kk, g, t);
                mma::m16n8k16(c, dh1a[kk], b0, b1);
            }
            if (ROUTER) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    wb.tm[(g + 8 * (e >> 1)) * LD_TM + 8 * nt + 2 * t + (e & 1)] = __float2half_rn(c[e]);
            } else {
                // grid values without router: half(dz / 128) (runtime.cu:123)
                uint32_t lo = pack_half2(__float2half_rn(__fdiv_rn(__half2float(__float2half_rn(c[0])), 128.0f)),
                                         __float2half_rn(__fdiv_rn(__half2float(__float2half_rn(c[1])), 128.0f)));
                uint32_t hi = pack_half2(__float2half_rn(__fdiv_rn(__half2float(__float2half_rn(c[2])), 128.0f)),
                                         __float2half_rn(__fdiv_rn(__half2float(__float2half_rn(c[3])), 128.0f)));
                const int pair = 4 * nt + t;
                uint32_t* gv = reinterpret_cast<uint32_t*>(a.gvals) + (long long)pair * a.stride;
                if (r0 + g < a.n) gv[r0 + g] = lo;
                if (r0 + g + 8 < a.n) gv[r0 + g + 8] = hi;
            }
        }
        accumulate_dw<4, NW>(dd1, W, dh1a, f.wa, g, t, DEC_HIDDEN);
        if (ROUTER) {
            __syncwarp();
            // ---- gate backward, one (row, level) item per lane iteration
            const int L = a.levels;
            for (int item = lane; item < 16 * L; item += 32) {
                const int row = item / L, l = item - row * L;
                const float s = wb.sg[row * 16 + l];
                const float vis = float((wb.vb[row] >> l) & 1u);
                const __half weight = __float2half_rn(__fmul_rn(s, vis));
                __half reduced = __float2half_rn(0.0f);
                const int c0 = fm->col_of_level[l], dim = fm->dim_of_level[l];
                for (int c = c0; c < c0 + dim; ++c) {
                    const __half value = __float2half_rn(__fdiv_rn(__half2float(wb.tm[row * LD_TM + c]), 128.0f));
                    wb.tm[row * LD_TM + c] = __hmul_rn(value, weight);  // direct gradient
                    reduced = __hadd_rn(reduced, __hmul_rn(value, wb.xs[row * Smem<W>::LDX + c]));
                }
                const float incoming = __fmul_rn(__half2float(reduced), vis);
                float derivative;
                if (l < a.k_fixed) derivative = 0.0f;
                else if (a.softplus) derivative = incoming * (-expm1f(-s));
                else derivative = __fmul_rn(__fmul_rn(incoming, __fsub_rn(1.0f, s)), s);
                wb.tq[row * LD_TQ + l] = __hmul_rn(__float2half_rn(derivative), __float2half_rn(128.0f));
            }
            for (int item = lane; item < 16 * (16 - L); item += 32) {
                const int row = item / (16 - L), c = L + item - row * (16 - L);
                wb.tq[row * LD_TQ + c] = __float2half_rn(0.0f);
            }
            __syncwarp();
            uint32_t daa[1][4];
            mma::load_a(daa[0], wb.tq, LD_TQ, 0, g, t);
            uint32_t dgha[2][4];
#pragma unroll
            for (int k2 = 0; k2 < 2; ++k2) {
                float c0[4] = {0, 0, 0, 0}, c1[4] = {0, 0, 0, 0};
                uint32_t b0, b1;
                mma::load_b(b0, b1, ws + S::g2t, LD_G2T, 2 * k2, 0, g, t);
                mma::m16n8k16(c0, daa[0], b0, b1);
                mma::load_b(b0, b1, ws + S::g2t, LD_G2T, 2 * k2 + 1, 0, g, t);
                mma::m16n8k16(c1, daa[0], b0, b1);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    if (!(mma::a_elem(f.gha, 2 * k2, e) > 0.0f)) c0[e] = 0.0f;
                    if (!(mma::a_elem(f.gha, 2 * k2 + 1, e) > 0.0f)) c1[e] = 0.0f;
                }
                mma::c_to_a<false>(dgha[k2], c0, c1);
            }
            accumulate_dw<1, 4>(dg2, GATE_HIDDEN, daa, f.gha, g, t, L);
            // dr = dgh * Wg1; grid values v = hadd(direct, half(dr / 128)) (runtime.cu:121)
#pragma unroll
            for (int nt = 0; nt < NW; ++nt) {
                float c[4] = {0, 0, 0, 0};
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    uint32_t b0, b1;
                    mma::load_b(b0, b1, ws + S::g1t, LD_G2, nt, kk, g, t);
                    mma::m16n8k16(c, dgha[kk], b0, b1);
                }
                __half v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int row = g + 8 * (e >> 1), col = 8 * nt + 2 * t + (e & 1);
                    const __half dr = __float2half_rn(__fdiv_rn(__half2float(__float2half_rn(c[e])), 128.0f));
                    v[e] = __hadd_rn(wb.tm[row * LD_TM + col], dr);
                }
                const int pair = 4 * nt + t;
                uint32_t* gv = reinterpret_cast<uint32_t*>(a.gvals) + (long long)pair * a.stride;
                if (r0 + g < a.n) gv[r0 + g] = pack_half2(v[0], v[1]);
                if (r0 + g + 8 < a.n) gv[r0 + g + 8] = pack_half2(v[2], v[3]);
            }
            accumulate_dw<2, NW>(dg1, W, dgha, f.xa, g, t, GATE_HIDDEN);
        }
        __syncwarp();
    }
    __syncthreads();
    float* out = a.partials + (long long)blockIdx.x * P;
    for (int i = threadIdx.x; i < P; i += blockDim.x) {
        float s = acc_all[i];
#pragma unroll
        for (int w = 1; w < WARPS; ++w) s = __fadd_rn(s, acc_all[w * S::head_params + i]);
        out[i] = s;
    }
}

template <int W, bool ROUTER>
__global__ void __launch_bounds__(THREADS, 2) mlp_decode_kernel(const MlpArgs a) {
    using S = Smem<W>;
    extern __shared__ __align__(16) unsigned char smem[];
    __half* ws = reinterpret_cast<__half*>(smem);
    int8_t* fmap = reinterpret_cast<int8_t*>(smem + S::weight_bytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    WarpBufs<W> wb(smem + S::weight_bytes + S::fmap_bytes + warp * S::warp_bytes);
    stage_weights<W, ROUTER>(a, ws, fmap);
    __syncthreads();
    const long long tiles = (a.n + 15) / 16;
    for (long long tile = (long long)blockIdx.x * WARPS + warp; tile < tiles; tile += (long long)gridDim.x * WARPS) {
        const long long r0 = tile * 16;
        Fwd<W> f;
        forward_tile<W, ROUTER>(a, r0, ws, fmap, wb, f, lane);
        if (t < 2) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int col = 2 * t + (e & 1);
                const long long i = r0 + g + 8 * (e >> 1);
                if (col < 3 && i < a.n) {
                    const float x = __half2float(__float2half_rn(f.out[e]));
                    if (a.rgb) a.rgb[3 * i + col] = x;
                    if (a.rgb8) {
                        const float clipped = fminf(fmaxf(x, 0.0f), 1.0f);
                        a.rgb8[3 * i + col] = (uint8_t)__float2int_rn(__fmul_rn(clipped, 255.0f));
                    }
                }
            }
        }
        __syncwarp();
    }
}

__global__ void input_batch_kernel(const int64_t* __restrict__ ids, long long n, const uint8_t* __restrict__ rgb,
                                   bool rgb8, int width, int height, float* __restrict__ xy, float* __restrict__ target) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t id = uint32_t(ids[i]);
    // an id outside the image (never produced by the samplers) reads pixel 0
    // instead of memory outside the target
    if ((unsigned long long)id >= (unsigned long long)width * (unsigned long long)height) id = 0;
    // fp32(id % W) * fp32(1 / (W - 1)): the reciprocal in double rounded to fp32
    // (odie/native/runtime.cu:34-36).
    const float rx = float(1.0 / double(width - 1)), ry = float(1.0 / double(height - 1));
    reinterpret_cast<float2*>(xy)[i] = make_float2(__fmul_rn(float(id % uint32_t(width)), rx),
                                                   __fmul_rn(float(id / uint32_t(width)), ry));
    if (target) {
        for (int c = 0; c < 3; ++c)
            target[3 * i + c] = rgb8 ? __fmul_rn(float(rgb[3ull * id + c]), 1.0f / 255.0f)
                                     : reinterpret_cast<const float*>(rgb)[3ull * id + c];
    }
}

__global__ void coords_range_kernel(long long begin, long long n, int width, int height, float* __restrict__ xy) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t id = uint32_t(begin + i);
    const float rx = float(1.0 / double(width - 1)), ry = float(1.0 / double(height - 1));
    reinterpret_cast<float2*>(xy)[i] = make_float2(__fmul_rn(float(id % uint32_t(width)), rx),
                                                   __fmul_rn(float(id / uint32_t(width)), ry));
}

__global__ void reduce_partials_kernel(const float* __restrict__ partials, int blocks, int count, float* __restrict__ out) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= count) return;
    float s = 0.0f;
    for (int b = 0; b < blocks; ++b) s = __fadd_rn(s, partials[(long long)b * count + j]);
    out[j] = s;
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

// Four parameters per thread (16-byte vectors) when every array is 16-byte
// aligned; one per thread otherwise.
template <bool VEC>
__global__ void adam_kernel(float* __restrict__ master, __half* __restrict__ copy, float* __restrict__ m,
                            float* __restrict__ v, uint32_t* __restrict__ steps, float* __restrict__ grad,
                            long long count, float inv_scale, const float* __restrict__ step_size,
                            const float* __restrict__ bc2_sqrt, long long table, float beta1w, float beta2,
                            float beta2w, float eps, bool skip_zero, int* error_flag) {
    const long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (VEC && (q + 1) * 4 <= count) {
        float4 g4 = reinterpret_cast<float4*>(grad)[q];
        if (skip_zero && g4.x == 0.0f && g4.y == 0.0f && g4.z == 0.0f && g4.w == 0.0f) return;
        float4 p4 = reinterpret_cast<float4*>(master)[q];
        float4 m4 = reinterpret_cast<float4*>(m)[q];
        float4 v4 = reinterpret_cast<float4*>(v)[q];
        uint4 s4 = reinterpret_cast<uint4*>(steps)[q];
        float* gp = &g4.x; float* pp = &p4.x; float* mp = &m4.x; float* vp = &v4.x; uint32_t* sp = &s4.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float gj = __fmul_rn(gp[j], inv_scale);
            if (skip_zero && gj == 0.0f) continue;
            const uint32_t s = ++sp[j];
            if ((long long)s > table) { atomicExch(error_flag, 1); continue; }
            adam_update(pp[j], mp[j], vp[j], gj, step_size[s - 1], bc2_sqrt[s - 1], beta1w, beta2, beta2w, eps);
        }
        reinterpret_cast<float4*>(master)[q] = p4;
        reinterpret_cast<float4*>(m)[q] = m4;
        reinterpret_cast<float4*>(v)[q] = v4;
        reinterpret_cast<uint4*>(steps)[q] = s4;
        reinterpret_cast<float4*>(grad)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        __half2* ch = reinterpret_cast<__half2*>(copy + 4 * q);
        ch[0] = __floats2half2_rn(p4.x, p4.y);
        ch[1] = __floats2half2_rn(p4.z, p4.w);
        return;
    }
    const long long first = VEC ? 4 * q : q, last = VEC ? (4 * q + 4 < count ? 4 * q + 4 : count) : (q < count ? q + 1 : q);
    for (long long i = first; i < last; ++i) {
        const float gj = __fmul_rn(grad[i], inv_scale);
        if (skip_zero && gj == 0.0f) continue;
        const uint32_t s = ++steps[i];
        if ((long long)s > table) { atomicExch(error_flag, 1); continue; }
        float p = master[i], mi = m[i], vi = v[i];
        adam_update(p, mi, vi, gj, step_size[s - 1], bc2_sqrt[s - 1], beta1w, beta2, beta2w, eps);
        master[i] = p; m[i] = mi; v[i] = vi; grad[i] = 0.0f;
        copy[i] = __float2half_rn(p);
    }
}

__global__ void zero_kernel(float* p, long long count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) p[i] = 0.0f;
}
__global__ void cast_half_kernel(const float* __restrict__ in, __half* __restrict__ out, long long count) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < count) out[i] = __float2half_rn(in[i]);
}

template <int W, bool ROUTER>
void launch_train_t(const MlpArgs& a, int blocks, cudaStream_t stream) {
    const int bytes = Smem<W>::train_bytes;
    static unsigned long long configured = 0;  // one bit per device
    int device = 0;
    ODIE_CUDA(cudaGetDevice(&device));
    if (!(configured >> device & 1ull)) {
        ODIE_CUDA(cudaFuncSetAttribute(mlp_train_kernel<W, ROUTER>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        configured |= 1ull << device;
    }
    mlp_train_kernel<W, ROUTER><<<blocks, THREADS, bytes, stream>>>(a);
}

template <int W, bool ROUTER>
void launch_decode_t(const MlpArgs& a, cudaStream_t stream) {
    const int bytes = Smem<W>::decode_bytes;
    static unsigned long long configured = 0;  // one bit per device
    int device = 0;
    ODIE_CUDA(cudaGetDevice(&device));
    if (!(configured >> device & 1ull)) {
        ODIE_CUDA(cudaFuncSetAttribute(mlp_decode_kernel<W, ROUTER>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        configured |= 1ull << device;
    }
    const long long tiles = (a.n + 15) / 16;
    long long blocks = (tiles + WARPS - 1) / WARPS;
    const long long cap = 4LL * sm_count();
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    mlp_decode_kernel<W, ROUTER><<<(unsigned)blocks, THREADS, bytes, stream>>>(a);
}

}  // namespace

// The training kernel keeps one fp32 weight-gradient accumulator per warp in
// shared memory, which bounds the decoder input width to 32 (16 levels x F2).
size_t mlp_train_smem(int width) {
    switch (width) {
        case 16: return Smem<16>::train_bytes;
        case 32: return Smem<32>::train_bytes;
    }
    throw std::invalid_argument("decoder input width must be 16 or 32");
}

int mlp_train_blocks(long long n) {
    const long long tiles = (n + 15) / 16;
    long long blocks = (tiles + WARPS - 1) / WARPS;
    const long long cap = 1LL * sm_count();
    if (blocks > cap) blocks = cap;
    return blocks < 1 ? 1 : int(blocks);
}

void launch_mlp_train(const MlpArgs& a, int width, bool router, int blocks, cudaStream_t stream) {
    if (a.n <= 0) return;
#define ODIE_W(WV)                                                    \
    case WV:                                                          \
        if (router) launch_train_t<WV, true>(a, blocks, stream);     \
        else launch_train_t<WV, false>(a, blocks, stream);           \
        return;
    switch (width) { ODIE_W(16) ODIE_W(32) }
#undef ODIE_W
    throw std::invalid_argument("decoder input width must be 16 or 32");
}

void launch_mlp_decode(const MlpArgs& a, int width, bool router, cudaStream_t stream) {
    if (a.n <= 0) return;
#define ODIE_W(WV)                                                 \
    case WV:                                                       \
        if (router) launch_decode_t<WV, true>(a, stream);         \
        else launch_decode_t<WV, false>(a, stream);               \
        return;
    switch (width) { ODIE_W(16) ODIE_W(32) }
#undef ODIE_W
    throw std::invalid_argument("decoder input width must be 16 or 32");
}

void launch_input_batch(const int64_t* ids, long long n, const uint8_t* rgb, bool rgb8, int width, int height,
                        float* xy, float* target, cudaStream_t stream) {
    if (n <= 0) return;
    input_batch_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(ids, n, rgb, rgb8, width, height, xy, target);
}

void launch_coords_range(long long begin, long long n, int width, int height, float* xy, cudaStream_t stream) {
    if (n <= 0) return;
    coords_range_kernel<<<blocks_for(n, 256), 256, 0, stream>>>(begin, n, width, height, xy);
}

void launch_reduce_partials(const float* partials, int blocks, int count, float* out, cudaStream_t stream) {
    reduce_partials_kernel<<<blocks_for(count, 256), 256, 0, stream>>>(partials, blocks, count, out);
}

void launch_adam(float* master, __half* copy, float* m, float* v, uint32_t* steps, float* grad, long long count,
                 float inv_scale, AdamTables tables, float beta1w, float beta2, float beta2w, float eps, bool skip_zero,
                 int* error_flag, cudaStream_t stream) {
    if (count <= 0) return;
    auto aligned = [](const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; };
    const bool vec = aligned(master, 16) && aligned(m, 16) && aligned(v, 16) && aligned(steps, 16) &&
                     aligned(grad, 16) && aligned(copy, 8);
    if (vec) {
        const long long quads = (count + 3) / 4;
        adam_kernel<true><<<blocks_for(quads, 256), 256, 0, stream>>>(
            master, copy, m, v, steps, grad, count, inv_scale, tables.step_size, tables.bc2_sqrt, tables.size, beta1w,
            beta2, beta2w, eps, skip_zero, error_flag);
    } else {
        adam_kernel<false><<<blocks_for(count, 256), 256, 0, stream>>>(
            master, copy, m, v, steps, grad, count, inv_scale, tables.step_size, tables.bc2_sqrt, tables.size, beta1w,
            beta2, beta2w, eps, skip_zero, error_flag);
    }
}

void launch_zero(float* p, long long count, cudaStream_t stream) {
    if (count > 0) zero_kernel<<<blocks_for(count, 256), 256, 0, stream>>>(p, count);
}
void launch_cast_half(const float* in, __half* out, long long count, cudaStream_t stream) {
    if (count > 0) cast_half_kernel<<<blocks_for(count, 256), 256, 0, stream>>>(in, out, count);
}

}  // namespace odie
