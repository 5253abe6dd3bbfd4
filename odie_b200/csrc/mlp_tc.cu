// Fused MLP heads on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA (128 threads) processes tiles of 128 coordinates, one thread per
// coordinate row, persistent over tiles; two CTAs share an SM so one CTA's
// elementwise epilogue overlaps the other's matrix products.  Per tile:
//   gate MLP forward -> per-level sigmoid gate (odie/native/runtime.cu:66-75)
//   -> decoder forward -> L2 loss gradient (runtime.cu:53-63) -> decoder
//   backward -> gate backward (runtime.cu:76-92) -> gate MLP backward
//   -> grid-gradient values (runtime.cu:117-125)
// Every product runs as tcgen05.mma (fp16 operands in shared memory, fp32
// accumulators in TMEM) issued by one thread and tracked by one mbarrier; the
// epilogues read TMEM rows with tcgen05.ld (thread = row) and write the next
// operand to shared memory.  Weight gradients are products over the
// coordinate dimension (K = the 128 rows of a tile) whose accumulators stay in
// TMEM across all tiles of the CTA and are written once as per-CTA partials.
// Activations are rounded to fp16 where the reference's fp16 network stores
// them; every wait is bounded and reports through an error flag.
//
// UNIFORM: every level has 2 features at columns (2l, 2l+1) (the reference's
// default layout); the per-level epilogues are then fully unrolled with
// compile-time indices.  Other layouts take the generic per-column path.
//
// GATE_EXPERTS (routed multi-expert encoding, no reference counterpart): the
// decoder input is the routed expert's features times half(p), p the router
// probability of that expert (chosen bit-exactly by router.cu).  Training
// (experts_train3_kernel) recomputes the router MLP on the tensor cores
// (R -> 32 -> 32 -> 16 or 64 logits) for its backward: dp = sum_c v_c f_c,
// dz_j = dp p (delta_je - p_j), then the router backward down to the
// router-grid gradient values; one CTA per SM keeps three tiles in flight.
// Decode (experts_decode_kernel) keeps only the decoder resident, four CTAs
// per SM.  mlp_tc_kernel serves the per-level gate and the gate-free heads.
#include <atomic>

#include "router.cuh"
#include "step.cuh"
#include "tc.cuh"

namespace odie {

namespace {

constexpr int TC_THREADS = 128;
constexpr int TC_TILE = 128;
constexpr uint32_t WAIT_LIMIT = 1u << 22;
constexpr uint32_t TMEM_COLUMNS = 256;

// TMEM columns: a per-tile accumulator (M=128) and the persistent weight-
// gradient accumulators (M=64: lanes 0-15 of each 32-lane subpartition).
constexpr uint32_t T_ACC = 0, T_DWD2 = 64, T_DWD1 = 128, T_DW3T = 160, T_DWG2T = 176, T_DWG1 = 192, T_DWR2 = 224;

// Shared memory (bytes) for decoder input width W: weights blocked [out x in],
// activations blocked [128 x cols].  GH and DGH are read 64 columns wide as
// M=64 operands; their upper half aliases the following buffers and only
// feeds accumulator rows that are never read.
template <int W>
struct TcSmem {
    static constexpr int XB = 128 * W * 2;              // one [128 x W] buffer
    static constexpr int g1 = 0;                        // [32 x W] gate W1
    static constexpr int g2 = g1 + 32 * W * 2;          // [16 x 32] gate W2
    static constexpr int d1 = g2 + 16 * 32 * 2;         // [64 x W]
    static constexpr int d2 = d1 + 64 * W * 2;          // [64 x 64]
    static constexpr int d3 = d2 + 64 * 64 * 2;         // [16 x 64]
    static constexpr int x = d3 + 16 * 64 * 2;          // [128 x W] raw features
    static constexpr int wx = x + XB;                   // [128 x W] gated decoder input
    static constexpr int gh = wx + XB;                  // [128 x 32] gate hidden
    static constexpr int h1 = gh + 8192;                // [128 x 64] decoder hidden 1, then dh1
    static constexpr int h2 = h1 + 16384;               // [128 x 64] decoder hidden 2, then dh2
    static constexpr int dgh = h2 + 16384;              // [128 x 32] gate hidden gradient
    static constexpr int dy = dgh + 8192;               // [128 x 16] output gradient
    static constexpr int da = dy + 4096;                // [128 x 16] gate logit gradient
    static constexpr int bar = da + 4096;               // mbarrier: data products of a phase
    static constexpr int bar_dw = bar + 8;              // mbarrier: weight-gradient products of a phase
    static constexpr int drain = bar_dw + 8;            // mbarrier: every issuing warp's products (error exit)
    static constexpr int tmem = drain + 8;              // TMEM base address
    static constexpr int total = tmem + 8;
    static_assert(gh + 16384 <= dgh, "GH read 64 wide stays inside the activation buffers");
    static_assert(dgh + 16384 <= bar, "DGH read 64 wide stays inside the activation buffers");
};

// Two floats rounded to fp16 (round to nearest even) in one packed conversion; lo in bits 0..15.
__device__ __forceinline__ uint32_t cvt_pair(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ __half2 as_half2(uint32_t v) { return *reinterpret_cast<const __half2*>(&v); }
__device__ __forceinline__ uint32_t as_u32(__half2 h) { return *reinterpret_cast<const uint32_t*>(&h); }
// half(half(x) / 128) for a pair: an fp16 product with 2^-7 rounds the same real value as the fp32
// quotient does (both exact before the one rounding to fp16), so the pair stays in fp16.
__device__ __forceinline__ __half2 grid_pair(float x0, float x1) {
    return __hmul2_rn(as_half2(cvt_pair(x0, x1)), __float2half2_rn(0.0078125f));
}

__device__ __forceinline__ uint4 pack8(const float* v) {
    return make_uint4(cvt_pair(v[0], v[1]), cvt_pair(v[2], v[3]), cvt_pair(v[4], v[5]), cvt_pair(v[6], v[7]));
}

// Row r, columns [8j, 8j+8) of a blocked [128 x cols] matrix.
__device__ __forceinline__ void store_chunk(unsigned char* smem, int base, int r, int j, uint4 q) {
    *reinterpret_cast<uint4*>(smem + base + tc::blocked(TC_TILE, r, 8 * j)) = q;
}

// 16-byte asynchronous global -> shared copy (L2 only); src_bytes = 0 writes zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

__device__ void stage_blocked(const __half* __restrict__ src, int rows, int cols, unsigned char* smem, int base) {
    for (int idx = threadIdx.x; idx < rows * cols; idx += blockDim.x) {
        const int r = idx / cols, c = idx - r * cols;
        *reinterpret_cast<__half*>(smem + base + tc::blocked(rows, r, c)) = src[idx];
    }
}

struct Issuer {
    uint64_t* bar;
    uint64_t* bar_dw;
    uint32_t phase = 0, phase_dw = 0;
    // ok: CTA-uniform, updated once per tile; fine: this thread's waits all completed.  Each thread
    // waits on the mbarriers itself, so no CTA barrier is needed after a wait; a wait that gives up
    // lets the tile run on and ends the loop at the tile's end, for every thread at once.
    bool ok = true, fine = true;
    // Make every thread's shared-memory writes visible to the tensor cores and
    // every TMEM read complete, then let thread 0 issue.
    __device__ void before_issue() {
        tc::fence_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        if (threadIdx.x == 0) tc::fence_after_sync();
    }
    // Thread 0 commits; everybody waits (bounded) for the products to land.
    __device__ void complete() {
        if (threadIdx.x == 0) tc::commit(bar);
        fine = tc::bar_wait(bar, phase, WAIT_LIMIT) && fine;
        phase ^= 1u;
        tc::fence_after_sync();
    }
    // Backward phases commit the data product (bar) and the weight-gradient
    // products (bar_dw) separately: the epilogue reads the data product while
    // the weight-gradient products still run, and waits for them only before
    // overwriting an operand they read.
    __device__ void wait_data() {
        fine = tc::bar_wait(bar, phase, WAIT_LIMIT) && fine;
        phase ^= 1u;
        tc::fence_after_sync();
    }
    __device__ void wait_dw() {
        fine = tc::bar_wait(bar_dw, phase_dw, WAIT_LIMIT) && fine;
        phase_dw ^= 1u;
        tc::fence_after_sync();
    }
    // End of a tile (CTA-wide): whether every thread's waits completed.
    __device__ bool settle() {
        ok = __syncthreads_and(fine) != 0;
        return ok;
    }
};

// Load 32 TMEM columns, keep those whose forward activation was positive (bit c of mask: column c),
// pack to 16 fp16 pairs.
__device__ __forceinline__ void masked_pack32(uint32_t taddr, uint32_t mask, uint32_t* out) {
    float v[32];
    tc::tmem_ld32(taddr, v);
#pragma unroll
    for (int c = 0; c < 32; c += 2)
        out[c / 2] = cvt_pair((mask >> c & 1u) ? v[c] : 0.0f, (mask >> (c + 1) & 1u) ? v[c + 1] : 0.0f);
}
// Load 32 TMEM columns, apply ReLU, round to fp16, store four chunks from j0; returns the 32-bit
// mask of the values still positive in fp16.
__device__ __forceinline__ uint32_t relu_store32(uint32_t taddr, unsigned char* smem, int base, int r, int j0) {
    float v[32];
    tc::tmem_ld32(taddr, v);
    uint32_t mask = 0, h[16];
#pragma unroll
    for (int c = 0; c < 32; c += 2) {
        h[c / 2] = cvt_pair(v[c] > 0.0f ? v[c] : 0.0f, v[c + 1] > 0.0f ? v[c + 1] : 0.0f);
        mask |= uint32_t((h[c / 2] & 0x7fffu) != 0u) << c;
        mask |= uint32_t((h[c / 2] & 0x7fff0000u) != 0u) << (c + 1);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
        store_chunk(smem, base, r, j0 + q, make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]));
    return mask;
}
// x / 128 as an exact multiply: both round the same real value x * 2^-7, underflow included.
__device__ __forceinline__ float div128(float x) { return __fmul_rn(x, 0.0078125f); }

__device__ __forceinline__ float gate_value(float z, int level, int k_fixed, int softplus) {
    if (level < k_fixed) return 1.0f;
    if (softplus) return z > 20.0f ? z : log1pf(expf(z));
    return __frcp_rn(__fadd_rn(1.0f, expf(-z)));  // the correctly rounded 1 / (1 + e^-z)
}
__device__ __forceinline__ float gate_derivative(float incoming, float s, int level, int k_fixed, int softplus) {
    if (level < k_fixed) return 0.0f;
    if (softplus) return incoming * (-expm1f(-s));
    return __fmul_rn(__fmul_rn(incoming, __fsub_rn(1.0f, s)), s);
}

template <int W, int GATE, bool TRAIN, bool UNIFORM>
__global__ void __launch_bounds__(TC_THREADS, 2) mlp_tc_kernel(const MlpArgs a, int* error_flag) {
    using S = TcSmem<W>;
    constexpr int PAIRS = W / 2, KW = W / 16;
    extern __shared__ __align__(128) unsigned char smem[];
    const int t = threadIdx.x, warp = t >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::bar);
    uint64_t* bar_dw = reinterpret_cast<uint64_t*>(smem + S::bar_dw);
    uint64_t* drain = reinterpret_cast<uint64_t*>(smem + S::drain);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::tmem);
    const uint32_t sbase = tc::smem_u32(smem);

    constexpr bool ROUTER = GATE == GATE_LEVELS;   // the reference's per-level gate
    static_assert(GATE != GATE_EXPERTS, "routed experts train in experts_train3_kernel and decode in experts_decode_kernel");
    if (ROUTER) {
        stage_blocked(a.gate_w, GATE_HIDDEN, W, smem, S::g1);
        stage_blocked(a.gate_w + GATE_HIDDEN * W, GATE_OUT, GATE_HIDDEN, smem, S::g2);
    }
    stage_blocked(a.decoder_w, DEC_HIDDEN, W, smem, S::d1);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W, DEC_HIDDEN, DEC_HIDDEN, smem, S::d2);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W + DEC_HIDDEN * DEC_HIDDEN, DEC_OUT, DEC_HIDDEN, smem, S::d3);
    if (t == 0) {
        tc::bar_init(bar, 1);
        tc::bar_init(bar_dw, TC_THREADS / 32);  // one commit per warp: each warp issues part of every weight-gradient product
        tc::bar_init(drain, TC_THREADS / 32);
        tc::fence_bar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, TMEM_COLUMNS);
        tc::tmem_relinquish();
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);  // this warp's TMEM lanes
    if (TRAIN) {
        // The weight-gradient accumulators start at zero and every product accumulates: the warps issue
        // parts of one product, so no single MMA can be relied on to come first and overwrite.
        float zero[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) zero[c] = 0.0f;
        for (uint32_t col = T_DWD2; col < TMEM_COLUMNS; col += 16) tc::tmem_st16(lane_addr + col, zero);
        tc::tmem_wait_st();
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
    }

    const FeatureMap& fm = a.fmap;
    const int L = a.levels;
    const long long vis_words = a.stride >> 5;
    Issuer is{bar, bar_dw};
    uint32_t dw_accumulate = 0;  // 1 once a tile has added to the weight gradients
    const long long tiles = (a.n + TC_TILE - 1) / TC_TILE;
    constexpr uint32_t ID_G1 = tc::idesc(128, 32, 0, 0), ID_G2 = tc::idesc(128, 16, 0, 0);
    constexpr uint32_t ID_D1 = tc::idesc(128, 64, 0, 0), ID_D3 = tc::idesc(128, 16, 0, 0);
    const int in_buf = GATE != GATE_NONE ? S::wx : S::x;

    // Inputs of a tile: raw feature pairs, this warp's visibility words, target.
    // The next tile's inputs are loaded while the current tile runs its
    // backward products, so their global-memory latency is off the chain.
    uint32_t next_raw[PAIRS], next_vis = 0;
    float next_target[3] = {0.0f, 0.0f, 0.0f};
    auto load_inputs = [&](long long tile) {
        const long long i = tile * TC_TILE + t;
        const bool valid = tile < tiles && i < a.n;
        if (a.raw_rows) {  // the coordinate's row as 16-byte loads
#pragma unroll
            for (int j = 0; j < PAIRS / 4; ++j) {
                const uint4 q = valid ? __ldg(reinterpret_cast<const uint4*>(a.raw) + i * (PAIRS / 4) + j) : make_uint4(0, 0, 0, 0);
                next_raw[4 * j] = q.x;
                next_raw[4 * j + 1] = q.y;
                next_raw[4 * j + 2] = q.z;
                next_raw[4 * j + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int p = 0; p < PAIRS; ++p)
                next_raw[p] = valid ? __ldg(reinterpret_cast<const uint32_t*>(a.raw) + (long long)p * a.stride + i) : 0u;
        }
        if (TRAIN) {
#pragma unroll
            for (int c = 0; c < 3; ++c) next_target[c] = valid ? __ldg(a.target + 3 * i + c) : 0.0f;
        }
    };
    // Visibility: lane l (< levels) loads this warp's word of level l; the
    // words are broadcast with shuffles when the bits are folded per row.
    uint32_t vis_word = 0;
    auto issue_vis = [&](long long tile) {
        const int lane = t & 31;
        vis_word = (ROUTER && tile < tiles && lane < L)
                       ? __ldg(reinterpret_cast<const uint32_t*>(a.vis) + lane * vis_words + tile * (TC_TILE / 32) + warp)
                       : 0u;
    };
    auto fold_vis = [&](long long tile) {
        next_vis = 0;
#pragma unroll
        for (int l = 0; l < 16; ++l) next_vis |= ((__shfl_sync(0xffffffffu, vis_word, l) >> (t & 31)) & 1u) << l;
        if (tile * TC_TILE + t >= a.n) next_vis = 0;
    };
    load_inputs(blockIdx.x);
    issue_vis(blockIdx.x);
    fold_vis(blockIdx.x);

    for (long long tile = blockIdx.x; tile < tiles && is.ok; tile += gridDim.x) {
        const long long i = tile * TC_TILE + t;
        const bool valid = i < a.n;
        // ---- inputs: raw features (pad columns 1.0), visibility bits, target
        uint32_t raw[PAIRS];
        const __half one = __float2half_rn(1.0f);
#pragma unroll
        for (int p = 0; p < PAIRS; ++p) {
            uint32_t v = next_raw[p];
            if (2 * p >= a.raw_width) v = pack_half2(one, one);
            else if (2 * p + 1 >= a.raw_width) v = (v & 0xffffu) | (uint32_t(__half_as_ushort(one)) << 16);
            raw[p] = v;
        }
        const uint32_t visbits = next_vis;
        const float target[3] = {next_target[0], next_target[1], next_target[2]};
        const long long next_tile = tile + gridDim.x;
        {
#pragma unroll
            for (int j = 0; j < W / 8; ++j)
                store_chunk(smem, S::x, t, j, make_uint4(raw[4 * j], raw[4 * j + 1], raw[4 * j + 2], raw[4 * j + 3]));
        }

        float sig[16];
        uint32_t gh_mask = 0;
        if (ROUTER) {
            // ---- gate hidden = relu(X Wg1^T)
            is.before_issue();
            if (t == 0)
                for (int s = 0; s < KW; ++s)
                    tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::x, 128, s), tc::kmajor(sbase + S::g1, 32, s), ID_G1, s > 0);
            is.complete();
            gh_mask = relu_store32(lane_addr + T_ACC, smem, S::gh, t, 0);
            // ---- logits = GH Wg2^T; gated decoder input raw * half(s_l * vis_l) (runtime.cu:66-75)
            is.before_issue();
            if (t == 0)
                for (int s = 0; s < 2; ++s)
                    tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::gh, 128, s), tc::kmajor(sbase + S::g2, 16, s), ID_G2, s > 0);
            is.complete();
            float z[16];
            tc::tmem_ld16(lane_addr + T_ACC, z);
            uint32_t wx[PAIRS];
            if (UNIFORM) {
                float zh[16];  // the fp16-rounded logits, converted in pairs
#pragma unroll
                for (int l = 0; l < 16; l += 2) {
                    const __half2 h = as_half2(cvt_pair(z[l], z[l + 1]));
                    zh[l] = __low2float(h);
                    zh[l + 1] = __high2float(h);
                }
#pragma unroll
                for (int l = 0; l < PAIRS; ++l) {
                    sig[l] = gate_value(zh[l], l, a.k_fixed, a.softplus);
                    if (l < L) {
                        // both features times half(s_l vis_l), each product rounded once as by __hmul_rn
                        const __half2 w = half2_dup(__fmul_rn(sig[l], float((visbits >> l) & 1u)));
                        wx[l] = as_u32(__hmul2_rn(as_half2(raw[l]), w));
                    } else {
                        wx[l] = raw[l];
                    }
                }
            } else {
#pragma unroll
                for (int l = 0; l < 16; ++l) sig[l] = gate_value(__half2float(__float2half_rn(z[l])), l, a.k_fixed, a.softplus);
                for (int p = 0; p < PAIRS; ++p) {
                    __half h[2] = {lo_half(raw[p]), hi_half(raw[p])};
                    for (int q = 0; q < 2; ++q) {
                        const int lev = fm.level_of_col[2 * p + q];
                        if (lev < 0) continue;
                        float sl = 0.0f;
#pragma unroll
                        for (int k = 0; k < 16; ++k) sl = (k == lev) ? sig[k] : sl;
                        h[q] = __hmul_rn(h[q], __float2half_rn(__fmul_rn(sl, float((visbits >> lev) & 1u))));
                    }
                    wx[p] = pack_half2(h[0], h[1]);
                }
            }
#pragma unroll
            for (int j = 0; j < W / 8; ++j)
                store_chunk(smem, S::wx, t, j, make_uint4(wx[4 * j], wx[4 * j + 1], wx[4 * j + 2], wx[4 * j + 3]));
        }
        // ---- decoder hidden 1, hidden 2, output
        uint32_t h1_mask[4], h2_mask[4];
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < KW; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + in_buf, 128, s), tc::kmajor(sbase + S::d1, 64, s), ID_D1, s > 0);
        is.complete();
#pragma unroll
        for (int q = 0; q < 4; q += 2) {
            const uint32_t m = relu_store32(lane_addr + T_ACC + 16 * q, smem, S::h1, t, 2 * q);
            h1_mask[q] = m & 0xffffu;
            h1_mask[q + 1] = m >> 16;
        }
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::h1, 128, s), tc::kmajor(sbase + S::d2, 64, s), ID_D1, s > 0);
        is.complete();
#pragma unroll
        for (int q = 0; q < 4; q += 2) {
            const uint32_t m = relu_store32(lane_addr + T_ACC + 16 * q, smem, S::h2, t, 2 * q);
            h2_mask[q] = m & 0xffffu;
            h2_mask[q + 1] = m >> 16;
        }
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::h2, 128, s), tc::kmajor(sbase + S::d3, 16, s), ID_D3, s > 0);
        is.complete();
        float out[16];
        tc::tmem_ld16(lane_addr + T_ACC, out);
        load_inputs(next_tile);  // prefetch: consumed at the start of the next tile
        issue_vis(next_tile);
        if (!TRAIN) {
            if (valid) {
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const float xo = __half2float(__float2half_rn(out[c]));
                    if (a.rgb) a.rgb[3 * i + c] = xo;
                    if (a.rgb8)
                        a.rgb8[3 * i + c] = (uint8_t)__float2int_rn(__fmul_rn(fminf(fmaxf(xo, 0.0f), 1.0f), 255.0f));
                }
            }
            fold_vis(next_tile);
            continue;
        }
        // ---- loss gradient (odie/native/runtime.cu:53-63)
        {
            float dy[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) dy[c] = 0.0f;
            if (valid) {
                float s = 0.0f;
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const float d = __fsub_rn(__half2float(__float2half_rn(out[c])), target[c]);
                    s = __fadd_rn(s, __fmul_rn(d, d));
                    const float scaled = __fmul_rn(__fdiv_rn(__fmul_rn(2.0f, d), a.three_real), 128.0f);
                    dy[c] = __half2float(__hmul_rn(__float2half_rn(scaled), __float2half_rn(128.0f)));
                }
                a.squares[i] = __fdiv_rn(s, 3.0f);
            }
            store_chunk(smem, S::dy, t, 0, pack8(dy));
            store_chunk(smem, S::dy, t, 1, pack8(dy + 8));
        }
        // ---- dh2 = DY Wd3 (B: Wd3 as MN-major); dW3^T += H2^T DY
        is.before_issue();
        if (t == 0) {
            tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::dy, 128, 0), tc::mnmajor(sbase + S::d3, 16, 0),
                    tc::idesc(128, 64, 0, 1), 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {  // every warp issues two of the eight K-steps of the weight-gradient product
            for (int s = 2 * warp; s < 2 * warp + 2; ++s)
                tc::mma(tmem + T_DW3T, tc::mnmajor(sbase + S::h2, 128, s), tc::mnmajor(sbase + S::dy, 128, s),
                        tc::idesc(64, 16, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        uint32_t packed[32];
        is.wait_data();
#pragma unroll
        for (int q = 0; q < 4; q += 2)
            masked_pack32(lane_addr + T_ACC + 16 * q, h2_mask[q] | (h2_mask[q + 1] << 16), packed + 8 * q);
        is.wait_dw();  // dW3 has read H2: dh2 may overwrite it
#pragma unroll
        for (int j = 0; j < 8; ++j)
            store_chunk(smem, S::h2, t, j, make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]));
        // ---- dh1 = DH2 Wd2; dWd2 += DH2^T H1
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::h2, 128, s), tc::mnmajor(sbase + S::d2, 64, s),
                        tc::idesc(128, 64, 0, 1), s > 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {  // every warp issues two of the eight K-steps of the weight-gradient product
            for (int s = 2 * warp; s < 2 * warp + 2; ++s)
                tc::mma(tmem + T_DWD2, tc::mnmajor(sbase + S::h2, 128, s), tc::mnmajor(sbase + S::h1, 128, s),
                        tc::idesc(64, 64, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
#pragma unroll
        for (int q = 0; q < 4; q += 2)
            masked_pack32(lane_addr + T_ACC + 16 * q, h1_mask[q] | (h1_mask[q + 1] << 16), packed + 8 * q);
        is.wait_dw();  // dWd2 has read H1: dh1 may overwrite it
#pragma unroll
        for (int j = 0; j < 8; ++j)
            store_chunk(smem, S::h1, t, j, make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]));
        // ---- dz = DH1 Wd1; dWd1 += DH1^T WX
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::h1, 128, s), tc::mnmajor(sbase + S::d1, 64, s),
                        tc::idesc(128, W, 0, 1), s > 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {  // every warp issues two of the eight K-steps of the weight-gradient product
            for (int s = 2 * warp; s < 2 * warp + 2; ++s)
                tc::mma(tmem + T_DWD1, tc::mnmajor(sbase + S::h1, 128, s), tc::mnmajor(sbase + in_buf, 128, s),
                        tc::idesc(64, W, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
        float dzf[W];
        if (W == 32) {
            tc::tmem_ld32(lane_addr + T_ACC, dzf);
        } else {
#pragma unroll
            for (int q = 0; q < KW; ++q) tc::tmem_ld16(lane_addr + T_ACC + 16 * q, dzf + 16 * q);
        }
        uint32_t gv[PAIRS];
        if (!ROUTER) {
            is.wait_dw();  // dWd1 has read X: the next tile may overwrite it
            // grid values without router: half(dz / 128) (runtime.cu:123)
#pragma unroll
            for (int p = 0; p < PAIRS; ++p) gv[p] = as_u32(grid_pair(dzf[2 * p], dzf[2 * p + 1]));
        } else {
            // ---- gate backward per level (runtime.cu:76-92): direct and logit gradients
            uint32_t direct[PAIRS];
            float da[16];
#pragma unroll
            for (int l = 0; l < 16; ++l) da[l] = 0.0f;
            if (UNIFORM) {
                float derivative[16];
#pragma unroll
                for (int l = 0; l < 16; ++l) derivative[l] = 0.0f;
#pragma unroll
                for (int l = 0; l < PAIRS; ++l) {
                    direct[l] = 0u;
                    if (l < L) {
                        const float vis = float((visbits >> l) & 1u);
                        const __half2 vv = grid_pair(dzf[2 * l], dzf[2 * l + 1]);
                        // elementwise fp16 products, each rounded once as by __hmul_rn
                        direct[l] = as_u32(__hmul2_rn(vv, half2_dup(__fmul_rn(sig[l], vis))));
                        const __half2 pr = __hmul2_rn(vv, as_half2(raw[l]));
                        __half reduced = __hadd_rn(__float2half_rn(0.0f), __low2half(pr));
                        reduced = __hadd_rn(reduced, __high2half(pr));
                        derivative[l] =
                            gate_derivative(__fmul_rn(__half2float(reduced), vis), sig[l], l, a.k_fixed, a.softplus);
                    }
                }
                // da = fp16(fp16(derivative) x 128), two levels per packed conversion
#pragma unroll
                for (int l = 0; l < 16; l += 2) {
                    if (l >= L) break;
                    const __half2 h = __hmul2_rn(as_half2(cvt_pair(derivative[l], derivative[l + 1])),
                                                 __float2half2_rn(128.0f));
                    da[l] = __low2float(h);
                    if (l + 1 < L) da[l + 1] = __high2float(h);
                }
            } else {
                __half directh[W];
#pragma unroll
                for (int c = 0; c < W; ++c) directh[c] = __float2half_rn(0.0f);
                for (int l = 0; l < L; ++l) {
                    float sl = 0.0f;
#pragma unroll
                    for (int k = 0; k < 16; ++k) sl = (k == l) ? sig[k] : sl;
                    const float vis = float((visbits >> l) & 1u);
                    const __half weight = __float2half_rn(__fmul_rn(sl, vis));
                    __half reduced = __float2half_rn(0.0f);
                    const int c0 = fm.col_of_level[l], dim = fm.dim_of_level[l];
#pragma unroll
                    for (int c = 0; c < W; ++c) {
                        if (c < c0 || c >= c0 + dim) continue;
                        const __half value = __float2half_rn(div128(__half2float(__float2half_rn(dzf[c]))));
                        directh[c] = __hmul_rn(value, weight);
                        const __half rawc = (c & 1) ? hi_half(raw[c >> 1]) : lo_half(raw[c >> 1]);
                        reduced = __hadd_rn(reduced, __hmul_rn(value, rawc));
                    }
                    const float derivative =
                        gate_derivative(__fmul_rn(__half2float(reduced), vis), sl, l, a.k_fixed, a.softplus);
                    const float dal = __half2float(__hmul_rn(__float2half_rn(derivative), __float2half_rn(128.0f)));
#pragma unroll
                    for (int k = 0; k < 16; ++k) da[k] = (k == l) ? dal : da[k];
                }
#pragma unroll
                for (int p = 0; p < PAIRS; ++p) direct[p] = pack_half2(directh[2 * p], directh[2 * p + 1]);
            }
            is.wait_dw();  // dWd1 done before the next products are queued
            store_chunk(smem, S::da, t, 0, pack8(da));
            store_chunk(smem, S::da, t, 1, pack8(da + 8));
            // ---- dgh = DA Wg2; dWg2^T += GH^T DA
            is.before_issue();
            if (t == 0) {
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::da, 128, 0), tc::mnmajor(sbase + S::g2, 16, 0),
                        tc::idesc(128, 32, 0, 1), 0);
                tc::commit(bar);
            }
            if ((t & 31) == 0) {  // every warp issues two of the eight K-steps of the weight-gradient product
                for (int s = 2 * warp; s < 2 * warp + 2; ++s)
                    tc::mma(tmem + T_DWG2T, tc::mnmajor(sbase + S::gh, 128, s), tc::mnmajor(sbase + S::da, 128, s),
                            tc::idesc(64, 16, 1, 1), 1u);
                tc::commit(bar_dw);
            }
            is.wait_data();
            masked_pack32(lane_addr + T_ACC, gh_mask, packed);
            is.wait_dw();
#pragma unroll
            for (int j = 0; j < 4; ++j)
                store_chunk(smem, S::dgh, t, j, make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]));
            // ---- dr = DGH Wg1; dWg1 += DGH^T X; grid values v = hadd(direct, half(dr / 128)) (runtime.cu:121)
            is.before_issue();
            if (t == 0) {
                for (int s = 0; s < 2; ++s)
                    tc::mma(tmem + T_ACC, tc::kmajor(sbase + S::dgh, 128, s), tc::mnmajor(sbase + S::g1, 32, s),
                            tc::idesc(128, W, 0, 1), s > 0);
                tc::commit(bar);
            }
            if ((t & 31) == 0) {  // every warp issues two of the eight K-steps of the weight-gradient product
                for (int s = 2 * warp; s < 2 * warp + 2; ++s)
                    tc::mma(tmem + T_DWG1, tc::mnmajor(sbase + S::dgh, 128, s), tc::mnmajor(sbase + S::x, 128, s),
                            tc::idesc(64, W, 1, 1), 1u);
                tc::commit(bar_dw);
            }
            is.wait_data();
#pragma unroll
            for (int q = 0; q < KW; ++q) {
                float v[16];
                tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
                for (int c = 0; c < 16; c += 2) {
                    const int p = 8 * q + c / 2;
                    gv[p] = as_u32(__hadd2_rn(as_half2(direct[p]), grid_pair(v[c], v[c + 1])));
                }
            }
            is.wait_dw();  // dWg1 has read X and DGH: the next tile may overwrite them
        }
        if (valid) {
#pragma unroll
            for (int j = 0; j < PAIRS / 4; ++j)  // row-major [stride][W]: the coordinate's values in 16-byte runs
                reinterpret_cast<uint4*>(a.gvals + i * W)[j] = make_uint4(gv[4 * j], gv[4 * j + 1], gv[4 * j + 2], gv[4 * j + 3]);
        }
        if (!is.settle()) break;
        dw_accumulate = 1;
        fold_vis(next_tile);
    }
    if (!is.ok) {
        if (t == 0) atomicExch(error_flag, 2);
        // give the products every warp may still have in flight a bounded chance to land before TMEM is released
        if ((t & 31) == 0) tc::commit(drain);
        tc::bar_wait(drain, 0, WAIT_LIMIT);
    }
    if (TRAIN) {
        // ---- weight gradients: TMEM (M=64 layout: rows 16w..16w+15 in lanes 32w..32w+15) -> partials
        constexpr int GP = ROUTER ? gate_params(W) : 0;
        constexpr int P = GP + decoder_params(W);
        float* part = a.partials + (long long)blockIdx.x * P;
        float* dec = part + GP;
        const int row = 16 * warp + (t & 31);
        const bool holds = (t & 31) < 16;
        const bool any = dw_accumulate && is.ok;
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // dWd2 [64][64]
            float v[16];
            tc::tmem_ld16(lane_addr + T_DWD2 + 16 * q, v);
            if (holds)
                for (int c = 0; c < 16; ++c) dec[DEC_HIDDEN * W + row * DEC_HIDDEN + 16 * q + c] = any ? v[c] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < KW; ++q) {  // dWd1 [64][W]
            float v[16];
            tc::tmem_ld16(lane_addr + T_DWD1 + 16 * q, v);
            if (holds)
                for (int c = 0; c < 16; ++c) dec[row * W + 16 * q + c] = any ? v[c] : 0.0f;
        }
        {  // dW3 [16][64] from its transpose [64 in][16 out]
            float v[16];
            tc::tmem_ld16(lane_addr + T_DW3T, v);
            if (holds)
                for (int c = 0; c < 16; ++c)
                    dec[DEC_HIDDEN * W + DEC_HIDDEN * DEC_HIDDEN + c * DEC_HIDDEN + row] = any ? v[c] : 0.0f;
        }
        if (ROUTER) {
            {  // dWg2 [16][32] from its transpose [64 (32 valid) in][16 out]
                float v[16];
                tc::tmem_ld16(lane_addr + T_DWG2T, v);
                if (holds && row < GATE_HIDDEN)
                    for (int c = 0; c < 16; ++c) part[GATE_HIDDEN * W + c * GATE_HIDDEN + row] = any ? v[c] : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < KW; ++q) {  // dWg1 [32][W] from [64 (32 valid)][W]
                float v[16];
                tc::tmem_ld16(lane_addr + T_DWG1 + 16 * q, v);
                if (holds && row < GATE_HIDDEN)
                    for (int c = 0; c < 16; ++c) part[row * W + 16 * q + c] = any ? v[c] : 0.0f;
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLUMNS);
}

// ---------------------------------------------------------------- routed-expert training, three tiles per SM
// Routed-expert training step of the heads (no reference counterpart).  Per 128-coordinate tile: router
// recompute on the tensor cores (GH1 = relu(R Wr1^T), GH2 = relu(GH1 Wr2^T); the logits come from router.cu,
// which chose the expert on the CUDA cores), decoder forward on the gated input fp16(f x fp16(p)), loss
// gradient, decoder backward, expert values v x fp16(p) with v = fp16(dz / 128) and dp = sum_c v_c f_c, logit
// gradients dz_j = dp p (delta_je - p_j) over the coordinate's live experts, da = fp16(fp16(dz_j) x 128),
// router backward down to the router-grid values fp16(dR / 128).  ROUT: router logit rows (16 or 64); LIVE:
// logits per coordinate as router.cu stores them.
// One CTA per SM runs three warpgroups, each its own stream of tiles through that phase chain, so while one
// warpgroup converts an accumulator the tensor cores run the others' products.  The warpgroups share the staged weights and the weight-gradient accumulators in TMEM
// (every product adds into them); each has its own per-tile accumulator, activation buffers, mbarriers and
// named barrier.
constexpr int E3_GROUPS = 3;
constexpr int E3_THREADS = E3_GROUPS * TC_THREADS;
constexpr uint32_t E3_TMEM_COLUMNS = 512;
// TMEM columns: warpgroup g's per-tile accumulator at 64 g, then the shared weight-gradient accumulators
// (M = 64 layout: rows 16 w .. 16 w + 15 in lanes 32 w .. 32 w + 15): dWd2, dWd1, dW3^T, dWr3, dWr1 | dWr2,
// then a second 32-column accumulator per warpgroup.
constexpr uint32_t E3_DWD2 = 64 * E3_GROUPS, E3_DWD1 = E3_DWD2 + 64, E3_DW3T = E3_DWD1 + 32, E3_DWR3 = E3_DW3T + 16,
                   E3_DWR12 = E3_DWR3 + 32, E3_DW_END = E3_DWR12 + 32;
// then each warpgroup's second accumulator (32 columns): the router's hidden layers, computed beside the decoder's
constexpr uint32_t E3_ACC2 = E3_DW_END;
static_assert(E3_ACC2 + 32 * E3_GROUPS <= E3_TMEM_COLUMNS, "the three tiles' accumulators and the weight gradients fit TMEM");

// Shared memory (bytes): the weights once, then one region per warpgroup with the tile's activations.  The
// router backward reuses the decoder's buffers once the decoder's weight-gradient products have read them:
// dgh1 | zero | dgh2 is one contiguous 96-column stretch, so the 64-column MN-major views [dgh1 | zero] and
// [zero | dgh2] feed dWr1 and dWr2 into the two halves of one M = 64 accumulator (the zero columns add exact
// zeros to the other half).  The router features are single-buffered: the next tile's copy starts once the
// last product that reads them has completed.
struct E3Smem {
    static constexpr int W = 32, XB = 128 * W * 2;
    static constexpr int g1 = 0;                     // [32 x 32] router W1
    static constexpr int r2 = g1 + 32 * W * 2;       // [32 x 32] router W2
    static constexpr int g2 = r2 + 32 * 32 * 2;      // [64 x 32] router W3 (ROUT rows)
    static constexpr int d1 = g2 + 64 * 32 * 2;      // [64 x 32]
    static constexpr int d2 = d1 + 64 * W * 2;       // [64 x 64]
    static constexpr int d3 = d2 + 64 * 64 * 2;      // [16 x 64]
    static constexpr int groups = d3 + 16 * 64 * 2;  // the first warpgroup's region
    // offsets within a warpgroup's region
    static constexpr int x = 0;                      // [128 x 32] router features
    static constexpr int gh = x + XB;                // [128 x 32] router hidden 1
    static constexpr int gh2 = gh + XB;              // [128 x 32] router hidden 2
    static constexpr int h1 = gh2 + XB;              // [128 x 64] decoder hidden 1, then dh1
    static constexpr int wx = h1 + 16384;            // [128 x 32] decoder input
    static constexpr int dy = wx + XB;               // [128 x 16] output gradient
    static constexpr int h2 = dy + 4096;             // [128 x 64] decoder hidden 2, then dh2
    static constexpr int dgh1 = h1;                  // [128 x 32] router hidden-1 gradient
    static constexpr int zero = h1 + 8192;           // [128 x 32] zeros
    static constexpr int dgh2 = h1 + 16384;          // [128 x 32] router hidden-2 gradient
    static constexpr int da = h2;                    // [128 x 64] logit gradients
    static constexpr int bars = h2 + 16384;          // bar, bar_dw, drain
    static constexpr int region = bars + 128;
    static constexpr int tmem = groups + E3_GROUPS * region;  // TMEM base address
    static constexpr int total = tmem + 16;
    static_assert(dgh2 == wx && dgh2 + 8192 == dy, "dgh1 | zero | dgh2 is one contiguous stretch ending at dy");
    static_assert(total <= 232448, "fits the 227 KB a CTA may hold");
};

// A warpgroup's named barrier (id 1 + group; id 0 is __syncthreads) over its 128 threads.
__device__ __forceinline__ void group_sync(int group) {
    asm volatile("bar.sync %0, 128;\n" ::"r"(1 + group) : "memory");
}
__device__ __forceinline__ bool group_and(int group, bool value) {
    uint32_t out;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(out)
        : "r"(uint32_t(value)), "r"(1 + group)
        : "memory");
    return out != 0;
}

// Issuer of one warpgroup: as Issuer, with the warpgroup's named barrier in place of __syncthreads.  A wait that
// gives up ends the group's loop at the tile's end, for all its threads at once.
struct GroupIssuer {
    uint64_t* bar;
    uint64_t* bar_dw;
    int group, t;
    uint32_t phase = 0, phase_dw = 0;
    bool ok = true, fine = true;
    __device__ void before_issue() {
        tc::fence_async_smem();
        tc::fence_before_sync();
        group_sync(group);
        if (t == 0) tc::fence_after_sync();
    }
    __device__ void complete() {
        if (t == 0) tc::commit(bar);
        wait_data();
    }
    __device__ void wait_data() {
        fine = tc::bar_wait(bar, phase, WAIT_LIMIT) && fine;
        phase ^= 1u;
        tc::fence_after_sync();
    }
    __device__ void wait_dw() {
        fine = tc::bar_wait(bar_dw, phase_dw, WAIT_LIMIT) && fine;
        phase_dw ^= 1u;
        tc::fence_after_sync();
    }
    __device__ bool settle() {
        ok = group_and(group, fine);
        return ok;
    }
};

// 32 TMEM columns through ReLU, rounded to fp16, stored as chunks j0 .. j0 + 3 of row r.
__device__ __forceinline__ void relu_store32_plain(uint32_t taddr, unsigned char* smem, int base, int r, int j0) {
    float v[32];
    tc::tmem_ld32(taddr, v);
    uint32_t h[16];
#pragma unroll
    for (int c = 0; c < 32; c += 2) h[c / 2] = cvt_pair(v[c] > 0.0f ? v[c] : 0.0f, v[c + 1] > 0.0f ? v[c + 1] : 0.0f);
#pragma unroll
    for (int q = 0; q < 4; ++q)
        store_chunk(smem, base, r, j0 + q, make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]));
}

// 32 TMEM columns of a backward product kept where the layer's forward output -- the fp16 activations in
// chunks j0 .. j0 + 3 of row r of buffer fwd -- is positive (the ReLU's derivative), rounded to fp16 and
// stored as the same chunks of buffer dst (which may be fwd: each chunk is read before it is written).
__device__ __forceinline__ void relu_grad_store32(uint32_t taddr, unsigned char* smem, int fwd, int dst, int r, int j0) {
    const __half2 zero = __float2half2_rn(0.0f);
#pragma unroll
    for (int hlf = 0; hlf < 2; ++hlf) {
        float v[16];
        tc::tmem_ld16(taddr + 16 * hlf, v);
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const int j = j0 + 2 * hlf + q;
            const uint4 a = *reinterpret_cast<const uint4*>(smem + fwd + tc::blocked(TC_TILE, r, 8 * j));
            const uint32_t on[4] = {a.x, a.y, a.z, a.w};
            uint32_t g[4];
#pragma unroll
            for (int p = 0; p < 4; ++p)
                g[p] = cvt_pair(v[8 * q + 2 * p], v[8 * q + 2 * p + 1]) & __hgt2_mask(as_half2(on[p]), zero);
            store_chunk(smem, dst, r, j, make_uint4(g[0], g[1], g[2], g[3]));
        }
    }
}

template <int ROUT, int LIVE>
__global__ void __launch_bounds__(E3_THREADS, 1) experts_train3_kernel(const MlpArgs a, int* error_flag) {
    using S = E3Smem;
    constexpr int W = 32, PAIRS = W / 2, KW = W / 16;
    static_assert(ROUT == 16 || ROUT == 64, "the router has 16 or 64 logit rows");
    static_assert(LIVE == 8 || LIVE == 16, "8 or 16 live logits per coordinate");
    extern __shared__ __align__(128) unsigned char smem[];
    const int group = threadIdx.x >> 7, t = threadIdx.x & 127, warp = threadIdx.x >> 5, quad = warp & 3;
    unsigned char* const mine = smem + S::groups + group * S::region;
    uint64_t* bar = reinterpret_cast<uint64_t*>(mine + S::bars);
    uint64_t* bar_dw = bar + 1;
    uint64_t* drain = bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::tmem);
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t gbase = sbase + S::groups + uint32_t(group) * S::region;

    stage_blocked(a.gate_w, ROUTER_HIDDEN, W, smem, S::g1);
    stage_blocked(a.gate_w + ROUTER_HIDDEN * W, ROUTER_HIDDEN, ROUTER_HIDDEN, smem, S::r2);
    stage_blocked(a.gate_w + ROUTER_HIDDEN * W + ROUTER_HIDDEN * ROUTER_HIDDEN, ROUT, ROUTER_HIDDEN, smem, S::g2);
    stage_blocked(a.decoder_w, DEC_HIDDEN, W, smem, S::d1);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W, DEC_HIDDEN, DEC_HIDDEN, smem, S::d2);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W + DEC_HIDDEN * DEC_HIDDEN, DEC_OUT, DEC_HIDDEN, smem, S::d3);
    if (t == 0) {
        tc::bar_init(bar, 1);
        tc::bar_init(bar_dw, TC_THREADS / 32);  // one commit per warp of the group
        tc::bar_init(drain, TC_THREADS / 32);
        tc::fence_bar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, E3_TMEM_COLUMNS);
        tc::tmem_relinquish();
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_addr = tmem + (uint32_t(quad * 32) << 16);  // this warp's TMEM lanes
    const uint32_t acc = 64u * uint32_t(group);                      // this warpgroup's per-tile accumulator
    const uint32_t acc2 = E3_ACC2 + 32u * uint32_t(group);           // and its router-forward accumulator
    if (group == 0) {  // the weight-gradient accumulators start at zero; every product accumulates
        float zero[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) zero[c] = 0.0f;
        for (uint32_t col = E3_DWD2; col < E3_DW_END; col += 16) tc::tmem_st16(lane_addr + col, zero);
        tc::tmem_wait_st();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    GroupIssuer is{bar, bar_dw, group, t};
    bool added = false;  // this warpgroup has added a tile to the weight gradients
    const long long tiles = (a.n + TC_TILE - 1) / TC_TILE;
    const long long stride = (long long)gridDim.x * E3_GROUPS;
    constexpr uint32_t ID_G1 = tc::idesc(128, 32, 0, 0), ID_D1 = tc::idesc(128, 64, 0, 0), ID_D3 = tc::idesc(128, 16, 0, 0);
    const int per = a.per_band;

    // The routed expert's feature row, logits, target, probability and expert of a tile: read for the first tile
    // here, then for the next tile once the current one has used them (during its router backward).
    uint32_t raw[PAIRS], lg[LIVE / 2];
    float target[3], prob;
    int expert;
    auto load_inputs = [&](long long tile) {
        const long long i = tile * TC_TILE + t;
        const bool valid = tile < tiles && i < a.n;
#pragma unroll
        for (int j = 0; j < PAIRS / 4; ++j) {
            const uint4 q = valid ? __ldg(reinterpret_cast<const uint4*>(a.raw) + i * (PAIRS / 4) + j) : make_uint4(0, 0, 0, 0);
            raw[4 * j] = q.x;
            raw[4 * j + 1] = q.y;
            raw[4 * j + 2] = q.z;
            raw[4 * j + 3] = q.w;
        }
#pragma unroll
        for (int j = 0; j < LIVE / 8; ++j) {
            const uint4 q = valid ? __ldg(reinterpret_cast<const uint4*>(a.logits) + i * (LIVE / 8) + j) : make_uint4(0, 0, 0, 0);
            lg[4 * j] = q.x;
            lg[4 * j + 1] = q.y;
            lg[4 * j + 2] = q.z;
            lg[4 * j + 3] = q.w;
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) target[c] = valid ? __ldg(a.target + 3 * i + c) : 0.0f;
        prob = valid ? __ldg(a.prob + i) : 0.0f;
        expert = valid ? __ldg(a.expert + i) : 0;
    };
    load_inputs((long long)blockIdx.x * E3_GROUPS + group);

    for (long long tile = (long long)blockIdx.x * E3_GROUPS + group; tile < tiles && is.ok; tile += stride) {
        const long long i = tile * TC_TILE + t;
        const bool valid = i < a.n;
        // ---- this tile's router features into x (the previous tile's last product, which read x, has completed)
        {
            const uint4* src = reinterpret_cast<const uint4*>(a.router_in) + (valid ? i * (W / 8) : 0);
#pragma unroll
            for (int j = 0; j < W / 8; ++j) cp_async16(gbase + S::x + tc::blocked(TC_TILE, t, 8 * j), src + j, valid ? 16u : 0u);
            cp_async_commit();
        }
        // decoder input: the routed expert's features x half(p), one rounding per feature
        {
            const __half2 ph = __float2half2_rn(prob);
            uint32_t wx[PAIRS];
#pragma unroll
            for (int p = 0; p < PAIRS; ++p) wx[p] = as_u32(__hmul2(as_half2(raw[p]), ph));
#pragma unroll
            for (int j = 0; j < W / 8; ++j)
                store_chunk(mine, S::wx, t, j, make_uint4(wx[4 * j], wx[4 * j + 1], wx[4 * j + 2], wx[4 * j + 3]));
        }
        asm volatile("cp.async.wait_all;\n" ::: "memory");
        // ---- the router recompute and the decoder forward side by side (independent chains): GH1 = relu(R
        //      Wr1^T) in acc2 with H1 = relu(WX Wd1^T) in acc, then GH2 = relu(GH1 Wr2^T) with H2 = relu(H1 Wd2^T)
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < KW; ++s)
                tc::mma(tmem + acc2, tc::kmajor(gbase + S::x, 128, s), tc::kmajor(sbase + S::g1, 32, s), ID_G1, s > 0);
            for (int s = 0; s < KW; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::wx, 128, s), tc::kmajor(sbase + S::d1, 64, s), ID_D1, s > 0);
        }
        is.complete();
        relu_store32_plain(lane_addr + acc2, mine, S::gh, t, 0);
#pragma unroll
        for (int q = 0; q < 2; ++q) relu_store32_plain(lane_addr + acc + 32 * q, mine, S::h1, t, 4 * q);
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 2; ++s)
                tc::mma(tmem + acc2, tc::kmajor(gbase + S::gh, 128, s), tc::kmajor(sbase + S::r2, 32, s), ID_G1, s > 0);
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::h1, 128, s), tc::kmajor(sbase + S::d2, 64, s), ID_D1, s > 0);
        }
        is.complete();
        relu_store32_plain(lane_addr + acc2, mine, S::gh2, t, 0);
#pragma unroll
        for (int q = 0; q < 2; ++q) relu_store32_plain(lane_addr + acc + 32 * q, mine, S::h2, t, 4 * q);
        // ---- decoder output
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::h2, 128, s), tc::kmajor(sbase + S::d3, 16, s), ID_D3, s > 0);
        is.complete();
        // ---- loss gradient (odie/native/runtime.cu:53-63)
        {
            float out[16];
            tc::tmem_ld16(lane_addr + acc, out);
            float dy[16];
#pragma unroll
            for (int c = 0; c < 16; ++c) dy[c] = 0.0f;
            if (valid) {
                float s = 0.0f;
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    const float d = __fsub_rn(__half2float(__float2half_rn(out[c])), target[c]);
                    s = __fadd_rn(s, __fmul_rn(d, d));
                    const float scaled = __fmul_rn(__fdiv_rn(__fmul_rn(2.0f, d), a.three_real), 128.0f);
                    dy[c] = __half2float(__hmul_rn(__float2half_rn(scaled), __float2half_rn(128.0f)));
                }
                a.squares[i] = __fdiv_rn(s, 3.0f);
            }
            store_chunk(mine, S::dy, t, 0, pack8(dy));
            store_chunk(mine, S::dy, t, 1, pack8(dy + 8));
        }
        const int wq = t >> 5;  // warp within the group: it issues K-steps 2 wq, 2 wq + 1 of each weight-gradient product
        // ---- dh2 = DY Wd3 (B: Wd3 as MN-major); dW3^T += H2^T DY
        is.before_issue();
        if (t == 0) {
            tc::mma(tmem + acc, tc::kmajor(gbase + S::dy, 128, 0), tc::mnmajor(sbase + S::d3, 16, 0), tc::idesc(128, 64, 0, 1), 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {
            for (int s = 2 * wq; s < 2 * wq + 2; ++s)
                tc::mma(tmem + E3_DW3T, tc::mnmajor(gbase + S::h2, 128, s), tc::mnmajor(gbase + S::dy, 128, s),
                        tc::idesc(64, 16, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
        is.wait_dw();  // dW3 has read H2: dh2 may overwrite it
#pragma unroll
        for (int q = 0; q < 2; ++q) relu_grad_store32(lane_addr + acc + 32 * q, mine, S::h2, S::h2, t, 4 * q);
        // ---- dh1 = DH2 Wd2; dWd2 += DH2^T H1
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::h2, 128, s), tc::mnmajor(sbase + S::d2, 64, s), tc::idesc(128, 64, 0, 1), s > 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {
            for (int s = 2 * wq; s < 2 * wq + 2; ++s)
                tc::mma(tmem + E3_DWD2, tc::mnmajor(gbase + S::h2, 128, s), tc::mnmajor(gbase + S::h1, 128, s),
                        tc::idesc(64, 64, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
        is.wait_dw();  // dWd2 has read H1: dh1 may overwrite it
#pragma unroll
        for (int q = 0; q < 2; ++q) relu_grad_store32(lane_addr + acc + 32 * q, mine, S::h1, S::h1, t, 4 * q);
        // ---- dz = DH1 Wd1; dWd1 += DH1^T WX
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::h1, 128, s), tc::mnmajor(sbase + S::d1, 64, s), tc::idesc(128, W, 0, 1), s > 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {
            for (int s = 2 * wq; s < 2 * wq + 2; ++s)
                tc::mma(tmem + E3_DWD1, tc::mnmajor(gbase + S::h1, 128, s), tc::mnmajor(gbase + S::wx, 128, s),
                        tc::idesc(64, W, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
        // ---- expert grid values v_c * half(p) and the probability gradient dp = sum_c v_c f_c
        uint32_t gv[PAIRS];
        float dp = 0.0f;
        {
            const __half2 ph = __float2half2_rn(prob);
#pragma unroll
            for (int hlf = 0; hlf < 2; ++hlf) {
                float dzf[16];
                tc::tmem_ld16(lane_addr + acc + 16 * hlf, dzf);
#pragma unroll
                for (int p = 0; p < 8; ++p) {
                    const int pp = 8 * hlf + p;
                    const __half2 v = grid_pair(dzf[2 * p], dzf[2 * p + 1]);
                    gv[pp] = as_u32(__hmul2_rn(v, ph));
                    dp = __fmaf_rn(__low2float(v), __half2float(lo_half(raw[pp])), dp);
                    dp = __fmaf_rn(__high2float(v), __half2float(hi_half(raw[pp])), dp);
                }
            }
        }
        // ---- logit gradients: softmax of the router's fp16 logits over the coordinate's live experts
        const int choice = expert % per;
        const int lo = (a.first_band + expert / per) * per;
        float da[LIVE];
        {
            float z[LIVE], zmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < LIVE; ++j) {
                z[j] = __half2float((j & 1) ? hi_half(lg[j >> 1]) : lo_half(lg[j >> 1]));
                if (j < per) zmax = fmaxf(zmax, z[j]);
            }
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < LIVE; ++j) {
                z[j] = j < per ? expf(__fsub_rn(z[j], zmax)) : 0.0f;
                sum = __fadd_rn(sum, z[j]);
            }
            const float dpp = __fmul_rn(dp, prob);
            const float inv = __frcp_rn(sum);
#pragma unroll
            for (int j = 0; j < LIVE; j += 2) {
                const float d0 = __fmul_rn(dpp, __fsub_rn(j == choice ? 1.0f : 0.0f, __fmul_rn(z[j], inv)));
                const float d1 = __fmul_rn(dpp, __fsub_rn(j + 1 == choice ? 1.0f : 0.0f, __fmul_rn(z[j + 1], inv)));
                const __half2 h = __hmul2_rn(as_half2(cvt_pair(d0, d1)), __float2half2_rn(128.0f));
                da[j] = j < per ? __low2float(h) : 0.0f;
                da[j + 1] = j + 1 < per ? __high2float(h) : 0.0f;
            }
        }
        load_inputs(tile + stride);  // this tile's inputs are used up; the next tile's arrive during the router backward
        is.wait_dw();  // dWd1 has read WX and DH1: h1, wx, dy and h2 are free for the router backward
        {
            const uint4 zero4 = make_uint4(0, 0, 0, 0);
            const uint4 first = pack8(da), second = LIVE == 16 ? pack8(da + 8) : zero4;
#pragma unroll
            for (int c = 0; c < ROUT / 8; ++c)
                store_chunk(mine, S::da, t, c, 8 * c == lo ? first : (LIVE == 16 && 8 * c == lo + 8) ? second : zero4);
#pragma unroll
            for (int c = 0; c < 4; ++c) store_chunk(mine, S::zero, t, c, zero4);
        }
        // ---- dgh2 = DA Wr3; dWr3 += DA^T GH2
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < ROUT / 16; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::da, 128, s), tc::mnmajor(sbase + S::g2, ROUT, s), tc::idesc(128, 32, 0, 1), s > 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {
            for (int s = 2 * wq; s < 2 * wq + 2; ++s)
                tc::mma(tmem + E3_DWR3, tc::mnmajor(gbase + S::da, 128, s), tc::mnmajor(gbase + S::gh2, 128, s),
                        tc::idesc(64, 32, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
        is.wait_dw();
        relu_grad_store32(lane_addr + acc, mine, S::gh2, S::dgh2, t, 0);
        // ---- dgh1 = DGH2 Wr2; dWr2 (accumulator rows 32-63) += DGH2^T GH1 through the [zero | dgh2] view
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 2; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::dgh2, 128, s), tc::mnmajor(sbase + S::r2, 32, s), tc::idesc(128, 32, 0, 1), s > 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {
            for (int s = 2 * wq; s < 2 * wq + 2; ++s)
                tc::mma(tmem + E3_DWR12, tc::mnmajor(gbase + S::zero, 128, s), tc::mnmajor(gbase + S::gh, 128, s),
                        tc::idesc(64, 32, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
        is.wait_dw();
        relu_grad_store32(lane_addr + acc, mine, S::gh, S::dgh1, t, 0);
        // ---- dR = DGH1 Wr1; dWr1 (accumulator rows 0-31) += DGH1^T R through the [dgh1 | zero] view;
        //      router grid values half(dR / 128)
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 2; ++s)
                tc::mma(tmem + acc, tc::kmajor(gbase + S::dgh1, 128, s), tc::mnmajor(sbase + S::g1, 32, s), tc::idesc(128, W, 0, 1), s > 0);
            tc::commit(bar);
        }
        if ((t & 31) == 0) {
            for (int s = 2 * wq; s < 2 * wq + 2; ++s)
                tc::mma(tmem + E3_DWR12, tc::mnmajor(gbase + S::dgh1, 128, s), tc::mnmajor(gbase + S::x, 128, s),
                        tc::idesc(64, W, 1, 1), 1u);
            tc::commit(bar_dw);
        }
        is.wait_data();
#pragma unroll
        for (int q = 0; q < KW; ++q) {
            float v[16];
            tc::tmem_ld16(lane_addr + acc + 16 * q, v);
            uint32_t rv[8];
#pragma unroll
            for (int c = 0; c < 16; c += 2) rv[c / 2] = as_u32(grid_pair(v[c], v[c + 1]));
            if (valid) {
                uint4* dst = reinterpret_cast<uint4*>(a.router_gvals + i * W + 16 * q);
                dst[0] = make_uint4(rv[0], rv[1], rv[2], rv[3]);
                dst[1] = make_uint4(rv[4], rv[5], rv[6], rv[7]);
            }
        }
        if (valid) {
#pragma unroll
            for (int j = 0; j < PAIRS / 4; ++j)
                reinterpret_cast<uint4*>(a.gvals + i * W)[j] = make_uint4(gv[4 * j], gv[4 * j + 1], gv[4 * j + 2], gv[4 * j + 3]);
        }
        is.wait_dw();  // dWr1 has read R and DGH1: the next tile may overwrite them
        if (!is.settle()) break;
        added = true;
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");  // no copy outlives the block

    if (!is.ok) {
        if (t == 0) atomicExch(error_flag, 2);
        // give the products this group's warps may still have in flight a bounded chance to land
        if ((t & 31) == 0) tc::commit(drain);
        tc::bar_wait(drain, 0, WAIT_LIMIT);
    }
    // ---- weight gradients: TMEM (M = 64 layout) -> this CTA's partials, by the first warpgroup
    tc::fence_before_sync();
    const bool all_ok = __syncthreads_and(is.ok) != 0;
    const bool any = __syncthreads_or(added) != 0;
    tc::fence_after_sync();
    if (group == 0) {
        constexpr int GP = router_params(W, ROUT), R2 = ROUTER_HIDDEN * W, R3 = R2 + ROUTER_HIDDEN * ROUTER_HIDDEN;
        constexpr int P = GP + decoder_params(W);
        float* part = a.partials + (long long)blockIdx.x * P;
        float* dec = part + GP;
        const int row = 16 * quad + (t & 31);
        const bool holds = (t & 31) < 16;
        const bool keep = any && all_ok;
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // dWd2 [64][64]
            float v[16];
            tc::tmem_ld16(lane_addr + E3_DWD2 + 16 * q, v);
            if (holds)
                for (int c = 0; c < 16; ++c) dec[DEC_HIDDEN * W + row * DEC_HIDDEN + 16 * q + c] = keep ? v[c] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < KW; ++q) {  // dWd1 [64][W]
            float v[16];
            tc::tmem_ld16(lane_addr + E3_DWD1 + 16 * q, v);
            if (holds)
                for (int c = 0; c < 16; ++c) dec[row * W + 16 * q + c] = keep ? v[c] : 0.0f;
        }
        {  // dW3 [16][64] from its transpose [64 in][16 out]
            float v[16];
            tc::tmem_ld16(lane_addr + E3_DW3T, v);
            if (holds)
                for (int c = 0; c < 16; ++c) dec[DEC_HIDDEN * W + DEC_HIDDEN * DEC_HIDDEN + c * DEC_HIDDEN + row] = keep ? v[c] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // dWr1 [32][W] (rows 0-31) and dWr2 [32][32] (rows 32-63)
            float v[16];
            tc::tmem_ld16(lane_addr + E3_DWR12 + 16 * q, v);
            if (holds) {
                float* dst = row < ROUTER_HIDDEN ? part + row * W : part + R2 + (row - ROUTER_HIDDEN) * ROUTER_HIDDEN;
                for (int c = 0; c < 16; ++c) dst[16 * q + c] = keep ? v[c] : 0.0f;
            }
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {  // dWr3 [ROUT][32]
            float v[16];
            tc::tmem_ld16(lane_addr + E3_DWR3 + 16 * q, v);
            if (holds && row < ROUT)
                for (int c = 0; c < 16; ++c) part[R3 + row * ROUTER_HIDDEN + 16 * q + c] = keep ? v[c] : 0.0f;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, E3_TMEM_COLUMNS);
}

// ---------------------------------------------------------------- routed-expert decode
// Decode of the routed-expert model (no reference counterpart): decoder input fp16(features x fp16(p)), the
// decoder's two ReLU layers and its output, fp16-rounded RGB out -- the decode variant of mlp_tc_kernel, with
// only what decode needs resident: the decoder weights, the tile's input and one hidden buffer that holds the
// first hidden layer and then the second (its product has read the first when the second is written).  38 KB of
// shared memory and 64 TMEM columns per CTA, so four CTAs (four tiles in flight) share an SM.
struct DecodeSmem {
    static constexpr int W = 32;
    static constexpr int d1 = 0;                   // [64 x 32]
    static constexpr int d2 = d1 + 64 * W * 2;     // [64 x 64]
    static constexpr int d3 = d2 + 64 * 64 * 2;    // [16 x 64]
    static constexpr int wx = d3 + 16 * 64 * 2;    // [128 x 32] decoder input
    static constexpr int h = wx + 128 * W * 2;     // [128 x 64] hidden 1, then hidden 2
    static constexpr int bar = h + 16384;          // mbarrier: the products of a phase
    static constexpr int drain = bar + 8;          // mbarrier: every warp's products (error exit)
    static constexpr int tmem = drain + 8;
    static constexpr int total = tmem + 8;
};
constexpr int DECODE_CTAS_PER_SM = 4;
constexpr uint32_t DECODE_TMEM_COLUMNS = 64;

__global__ void __launch_bounds__(TC_THREADS, DECODE_CTAS_PER_SM) experts_decode_kernel(const MlpArgs a, int* error_flag) {
    using S = DecodeSmem;
    constexpr int W = 32, PAIRS = W / 2, KW = W / 16;
    extern __shared__ __align__(128) unsigned char smem[];
    const int t = threadIdx.x, warp = t >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + S::bar);
    uint64_t* drain = reinterpret_cast<uint64_t*>(smem + S::drain);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::tmem);
    const uint32_t sbase = tc::smem_u32(smem);
    stage_blocked(a.decoder_w, DEC_HIDDEN, W, smem, S::d1);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W, DEC_HIDDEN, DEC_HIDDEN, smem, S::d2);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W + DEC_HIDDEN * DEC_HIDDEN, DEC_OUT, DEC_HIDDEN, smem, S::d3);
    if (t == 0) {
        tc::bar_init(bar, 1);
        tc::bar_init(drain, TC_THREADS / 32);
        tc::fence_bar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(tmem_slot, DECODE_TMEM_COLUMNS);
        tc::tmem_relinquish();
    }
    tc::fence_async_smem();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_addr = tmem + (uint32_t(warp * 32) << 16);
    Issuer is{bar, bar};
    const long long tiles = (a.n + TC_TILE - 1) / TC_TILE;
    constexpr uint32_t ID_D1 = tc::idesc(128, 64, 0, 0), ID_D3 = tc::idesc(128, 16, 0, 0);
    // the routed expert's feature row and probability of a tile, read one tile ahead
    uint32_t raw[PAIRS];
    float prob;
    auto load_inputs = [&](long long tile) {
        const long long i = tile * TC_TILE + t;
        const bool valid = tile < tiles && i < a.n;
#pragma unroll
        for (int j = 0; j < PAIRS / 4; ++j) {
            const uint4 q = valid ? __ldg(reinterpret_cast<const uint4*>(a.raw) + i * (PAIRS / 4) + j) : make_uint4(0, 0, 0, 0);
            raw[4 * j] = q.x;
            raw[4 * j + 1] = q.y;
            raw[4 * j + 2] = q.z;
            raw[4 * j + 3] = q.w;
        }
        prob = valid ? __ldg(a.prob + i) : 0.0f;
    };
    load_inputs(blockIdx.x);
    for (long long tile = blockIdx.x; tile < tiles && is.ok; tile += gridDim.x) {
        const long long i = tile * TC_TILE + t;
        const bool valid = i < a.n;
        {  // decoder input: the routed expert's features x half(p), one rounding per feature
            const __half2 ph = __float2half2_rn(prob);
            uint32_t wx[PAIRS];
#pragma unroll
            for (int p = 0; p < PAIRS; ++p) wx[p] = as_u32(__hmul2(as_half2(raw[p]), ph));
#pragma unroll
            for (int j = 0; j < W / 8; ++j)
                store_chunk(smem, S::wx, t, j, make_uint4(wx[4 * j], wx[4 * j + 1], wx[4 * j + 2], wx[4 * j + 3]));
        }
        load_inputs(tile + gridDim.x);  // the next tile's rows arrive while this one runs
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < KW; ++s)
                tc::mma(tmem, tc::kmajor(sbase + S::wx, 128, s), tc::kmajor(sbase + S::d1, 64, s), ID_D1, s > 0);
        is.complete();
#pragma unroll
        for (int q = 0; q < 2; ++q) relu_store32_plain(lane_addr + 32 * q, smem, S::h, t, 4 * q);
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem, tc::kmajor(sbase + S::h, 128, s), tc::kmajor(sbase + S::d2, 64, s), ID_D1, s > 0);
        is.complete();  // the product has read hidden 1: hidden 2 may take its place
#pragma unroll
        for (int q = 0; q < 2; ++q) relu_store32_plain(lane_addr + 32 * q, smem, S::h, t, 4 * q);
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem, tc::kmajor(sbase + S::h, 128, s), tc::kmajor(sbase + S::d3, 16, s), ID_D3, s > 0);
        is.complete();
        float out[16];
        tc::tmem_ld16(lane_addr, out);
        if (valid) {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                const float xo = __half2float(__float2half_rn(out[c]));
                if (a.rgb) a.rgb[3 * i + c] = xo;
                if (a.rgb8) a.rgb8[3 * i + c] = (uint8_t)__float2int_rn(__fmul_rn(fminf(fmaxf(xo, 0.0f), 1.0f), 255.0f));
            }
        }
        if (!is.settle()) break;
    }
    if (!is.ok) {
        if (t == 0) atomicExch(error_flag, 2);
        if ((t & 31) == 0) tc::commit(drain);
        tc::bar_wait(drain, 0, WAIT_LIMIT);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, DECODE_TMEM_COLUMNS);
}

// cudaFuncSetAttribute once per kernel and device (devices 0..63).
template <typename Kernel>
void set_smem(Kernel kernel, int bytes, std::atomic<unsigned long long>& configured) {
    int device = 0;
    ODIE_CUDA(cudaGetDevice(&device));
    ODIE_REQUIRE(device >= 0 && device < 64, "the fused heads support devices 0..63");
    if (!(configured.load(std::memory_order_acquire) >> device & 1ull)) {
        ODIE_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
        configured.fetch_or(1ull << device, std::memory_order_acq_rel);
    }
}

template <int ROUT, int LIVE>
void launch_experts(const MlpArgs& a, int blocks, int* error_flag, cudaStream_t stream) {
    static std::atomic<unsigned long long> configured{0};
    set_smem(experts_train3_kernel<ROUT, LIVE>, E3Smem::total, configured);
    experts_train3_kernel<ROUT, LIVE><<<blocks, E3_THREADS, E3Smem::total, stream>>>(a, error_flag);
    note_launch();
}

void launch_experts_decode(const MlpArgs& a, int* error_flag, cudaStream_t stream) {
    static std::atomic<unsigned long long> configured{0};
    set_smem(experts_decode_kernel, DecodeSmem::total, configured);
    const long long tiles = (a.n + TC_TILE - 1) / TC_TILE;
    const long long resident = (long long)DECODE_CTAS_PER_SM * sm_count();
    experts_decode_kernel<<<unsigned(tiles < resident ? tiles : resident), TC_THREADS, DecodeSmem::total, stream>>>(
        a, error_flag);
    note_launch();
}

template <int W, int GATE, bool TRAIN, bool UNIFORM>
void launch_tc(const MlpArgs& a, int blocks, int* error_flag, cudaStream_t stream) {
    static std::atomic<unsigned long long> configured{0};
    constexpr int bytes = TcSmem<W>::total;
    set_smem(mlp_tc_kernel<W, GATE, TRAIN, UNIFORM>, bytes, configured);
    mlp_tc_kernel<W, GATE, TRAIN, UNIFORM><<<blocks, TC_THREADS, bytes, stream>>>(a, error_flag);
    note_launch();
}

template <bool TRAIN>
void dispatch(const MlpArgs& a, int width, GateMode gate, bool uniform, int blocks, int* error_flag, cudaStream_t stream) {
#define ODIE_TC(WV, G, U) \
    if (width == WV && gate == G && uniform == U) return launch_tc<WV, G, TRAIN, U>(a, blocks, error_flag, stream);
    ODIE_TC(32, GATE_LEVELS, true) ODIE_TC(32, GATE_LEVELS, false) ODIE_TC(32, GATE_NONE, true) ODIE_TC(32, GATE_NONE, false)
    ODIE_TC(16, GATE_LEVELS, true) ODIE_TC(16, GATE_LEVELS, false) ODIE_TC(16, GATE_NONE, true) ODIE_TC(16, GATE_NONE, false)
#undef ODIE_TC
    if (gate == GATE_EXPERTS) {
        ODIE_REQUIRE(width == 32, "routed experts take 32 input features");
        if (!TRAIN) {
            ODIE_REQUIRE(a.raw_rows, "routed-expert decode reads row-major feature rows");
            return launch_experts_decode(a, error_flag, stream);
        }
        const Banding b{a.model_experts / a.per_band, a.first_band, a.per_band, 2};
        check_banding(b, a.experts);
        ODIE_REQUIRE(a.logits && (a.live == 8 || a.live == 16) && a.live >= a.per_band,
                     "routed-expert training needs the router's logits rows (8 or 16 halves, at least per band)");
        const bool wide = router_out(a.model_experts) == ROUTER_MAX_OUT;
        if (wide && a.live == 8) return launch_experts<64, 8>(a, blocks, error_flag, stream);
        if (wide) return launch_experts<64, 16>(a, blocks, error_flag, stream);
        if (a.live == 8) return launch_experts<16, 8>(a, blocks, error_flag, stream);
        return launch_experts<16, 16>(a, blocks, error_flag, stream);
    }
    throw std::invalid_argument("the fused heads take 16 or 32 input features");
}

}  // namespace

int mlp_tc_blocks(long long n) {
    const long long tiles = (n + TC_TILE - 1) / TC_TILE;
    long long blocks = 2LL * sm_count();
    if (blocks > tiles) blocks = tiles;
    return blocks < 1 ? 1 : int(blocks);
}

int mlp_tc_train_blocks(long long n, GateMode gate) {
    if (gate != GATE_EXPERTS) return mlp_tc_blocks(n);
    const long long tiles = (n + TC_TILE - 1) / TC_TILE;
    long long blocks = (tiles + E3_GROUPS - 1) / E3_GROUPS;  // one CTA per SM, three tiles in flight each
    if (blocks > sm_count()) blocks = sm_count();
    return blocks < 1 ? 1 : int(blocks);
}

void launch_mlp_tc_train(const MlpArgs& a, int width, GateMode gate, bool uniform, int blocks, int* error_flag,
                         cudaStream_t stream) {
    if (a.n <= 0) return;
    ODIE_REQUIRE(a.stride % TC_TILE == 0, "the feature stride must be a multiple of 128");
    dispatch<true>(a, width, gate, uniform, blocks, error_flag, stream);
}

void launch_mlp_tc_decode(const MlpArgs& a, int width, GateMode gate, bool uniform, int* error_flag, cudaStream_t stream) {
    if (a.n <= 0) return;
    ODIE_REQUIRE(a.stride % TC_TILE == 0, "the feature stride must be a multiple of 128");
    dispatch<false>(a, width, gate, uniform, mlp_tc_blocks(a.n), error_flag, stream);
}

}  // namespace odie
