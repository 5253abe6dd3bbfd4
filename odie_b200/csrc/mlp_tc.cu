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
// coordinate dimension (K = 128 rows of a tile) whose accumulators stay in TMEM
// across all tiles of the CTA and are written once as per-CTA partials.
// Activations are rounded to fp16 where the reference's fp16 network stores
// them; every wait is bounded and reports through an error flag.
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
constexpr uint32_t T_ACC = 0, T_DWD2 = 64, T_DWD1 = 128, T_DW3T = 160, T_DWG2T = 176, T_DWG1 = 192;

// Shared memory (bytes), decoder input width 32: weights blocked [out x in],
// activations blocked [128 x cols].  GH and DGH are read 64 columns wide as
// M=64 operands; their upper half aliases the following buffers and only
// feeds accumulator rows that are never read.
struct TcSmem {
    static constexpr int g1 = 0;                  // [32 x 32]
    static constexpr int g2 = g1 + 32 * 32 * 2;   // [16 x 32]
    static constexpr int d1 = g2 + 16 * 32 * 2;   // [64 x 32]
    static constexpr int d2 = d1 + 64 * 32 * 2;   // [64 x 64]
    static constexpr int d3 = d2 + 64 * 64 * 2;   // [16 x 64]
    static constexpr int x = d3 + 16 * 64 * 2;    // [128 x 32] raw features
    static constexpr int wx = x + 8192;           // [128 x 32] gated decoder input
    static constexpr int gh = wx + 8192;          // [128 x 32] gate hidden
    static constexpr int h1 = gh + 8192;          // [128 x 64] decoder hidden 1, then dh1
    static constexpr int h2 = h1 + 16384;         // [128 x 64] decoder hidden 2, then dh2
    static constexpr int dgh = h2 + 16384;        // [128 x 32] gate hidden gradient
    static constexpr int dy = dgh + 8192;         // [128 x 16] output gradient
    static constexpr int da = dy + 4096;          // [128 x 16] gate logit gradient
    static constexpr int bar = da + 4096;         // mbarrier
    static constexpr int tmem = bar + 8;          // TMEM base address
    static constexpr int total = tmem + 8;
};
static_assert(TcSmem::gh + 16384 <= TcSmem::dgh, "GH read 64 wide stays inside shared memory");
static_assert(TcSmem::dgh + 16384 <= TcSmem::bar, "DGH read 64 wide stays inside the activation buffers");

__device__ __forceinline__ uint4 pack8(const float* v) {
    uint4 q;
    q.x = pack_half2(__float2half_rn(v[0]), __float2half_rn(v[1]));
    q.y = pack_half2(__float2half_rn(v[2]), __float2half_rn(v[3]));
    q.z = pack_half2(__float2half_rn(v[4]), __float2half_rn(v[5]));
    q.w = pack_half2(__float2half_rn(v[6]), __float2half_rn(v[7]));
    return q;
}

// Store 8 fp16 values (one 16-byte chunk) of row r, columns [8j, 8j+8) of a blocked [128 x cols] matrix.
__device__ __forceinline__ void store_chunk(unsigned char* smem, int base, int r, int j, uint4 q) {
    *reinterpret_cast<uint4*>(smem + base + tc::blocked(TC_TILE, r, 8 * j)) = q;
}

// Copy a global fp16 matrix [rows x cols] (row-major) into a blocked shared-memory matrix.
__device__ void stage_blocked(const __half* __restrict__ src, int rows, int cols, unsigned char* smem, int base) {
    for (int idx = threadIdx.x; idx < rows * cols; idx += blockDim.x) {
        const int r = idx / cols, c = idx - r * cols;
        *reinterpret_cast<__half*>(smem + base + tc::blocked(rows, r, c)) = src[idx];
    }
}

struct Issuer {
    uint64_t* bar;
    uint32_t phase = 0;
    bool ok = true;
    // Make this thread's shared-memory writes visible to the tensor cores and
    // every thread's TMEM reads complete, then let thread 0 issue.
    __device__ void before_issue() {
        tc::fence_async_smem();
        tc::fence_before_sync();
        __syncthreads();
        if (threadIdx.x == 0) tc::fence_after_sync();
    }
    // Thread 0 commits; everybody waits (bounded) for the products to land.
    __device__ bool complete() {
        if (threadIdx.x == 0) tc::commit(bar);
        const bool done = tc::bar_wait(bar, phase, WAIT_LIMIT);
        phase ^= 1u;
        ok = __syncthreads_and(done) != 0;
        tc::fence_after_sync();
        return ok;
    }
};

template <bool ROUTER, bool TRAIN>
__global__ void __launch_bounds__(TC_THREADS, 2) mlp_tc_kernel(const MlpArgs a, int* error_flag) {
    constexpr int W = 32;
    extern __shared__ __align__(128) unsigned char smem[];
    const int t = threadIdx.x, warp = t >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + TcSmem::bar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::tmem);
    const uint32_t sbase = tc::smem_u32(smem);

    if (ROUTER) {
        stage_blocked(a.gate_w, GATE_HIDDEN, W, smem, TcSmem::g1);
        stage_blocked(a.gate_w + GATE_HIDDEN * W, GATE_OUT, GATE_HIDDEN, smem, TcSmem::g2);
    }
    stage_blocked(a.decoder_w, DEC_HIDDEN, W, smem, TcSmem::d1);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W, DEC_HIDDEN, DEC_HIDDEN, smem, TcSmem::d2);
    stage_blocked(a.decoder_w + DEC_HIDDEN * W + DEC_HIDDEN * DEC_HIDDEN, DEC_OUT, DEC_HIDDEN, smem, TcSmem::d3);
    if (t == 0) {
        tc::bar_init(bar, 1);
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

    const FeatureMap& fm = a.fmap;
    const int L = a.levels;
    Issuer is{bar};
    uint32_t dw_accumulate = 0;  // 0 until the first tile's weight-gradient products
    const long long tiles = (a.n + TC_TILE - 1) / TC_TILE;
    constexpr uint32_t ID_G1 = tc::idesc(128, 32, 0, 0), ID_G2 = tc::idesc(128, 16, 0, 0);
    constexpr uint32_t ID_D1 = tc::idesc(128, 64, 0, 0), ID_D2 = tc::idesc(128, 64, 0, 0), ID_D3 = tc::idesc(128, 16, 0, 0);

    for (long long tile = blockIdx.x; tile < tiles && is.ok; tile += gridDim.x) {
        const long long i = tile * TC_TILE + t;
        const bool valid = i < a.n;
        // ---- inputs: raw features (pad columns 1.0), visibility bits, target
        uint32_t raw[W / 2];
        const __half one = __float2half_rn(1.0f);
#pragma unroll
        for (int p = 0; p < W / 2; ++p) {
            uint32_t v = valid ? __ldg(reinterpret_cast<const uint32_t*>(a.raw) + (long long)p * a.stride + i) : 0u;
            if (2 * p >= a.raw_width) v = pack_half2(one, one);
            else if (2 * p + 1 >= a.raw_width) v = (v & 0xffffu) | (uint32_t(__half_as_ushort(one)) << 16);
            raw[p] = v;
        }
        uint32_t visbits = 0;
        if (valid)
            for (int l = 0; l < L; ++l) visbits |= uint32_t(__ldg(a.vis + (long long)l * a.stride + i) != 0) << l;
#pragma unroll
        for (int j = 0; j < W / 8; ++j)
            store_chunk(smem, TcSmem::x, t, j, make_uint4(raw[4 * j], raw[4 * j + 1], raw[4 * j + 2], raw[4 * j + 3]));

        float sig[16];
        uint32_t gh_mask = 0;
        uint32_t wx[W / 2];
        if (ROUTER) {
            // ---- gate hidden = relu(X Wg1^T)
            is.before_issue();
            if (t == 0)
                for (int s = 0; s < W / 16; ++s)
                    tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::x, 128, s), tc::kmajor(sbase + TcSmem::g1, 32, s), ID_G1, s > 0);
            if (!is.complete()) break;
            for (int q = 0; q < 2; ++q) {
                float v[16];
                tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    v[c] = __half2float(__float2half_rn(v[c] > 0.0f ? v[c] : 0.0f));
                    gh_mask |= uint32_t(v[c] > 0.0f) << (16 * q + c);
                }
                store_chunk(smem, TcSmem::gh, t, 2 * q, pack8(v));
                store_chunk(smem, TcSmem::gh, t, 2 * q + 1, pack8(v + 8));
            }
            // ---- logits = GH Wg2^T; per-level gate s (1 below K, sigmoid or softplus)
            is.before_issue();
            if (t == 0)
                for (int s = 0; s < 2; ++s)
                    tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::gh, 128, s), tc::kmajor(sbase + TcSmem::g2, 16, s), ID_G2, s > 0);
            if (!is.complete()) break;
            {
                float z[16];
                tc::tmem_ld16(lane_addr + T_ACC, z);
#pragma unroll
                for (int l = 0; l < 16; ++l) {
                    const float zl = __half2float(__float2half_rn(z[l]));
                    float s;
                    if (l < a.k_fixed) s = 1.0f;
                    else if (a.softplus) s = zl > 20.0f ? zl : log1pf(expf(zl));
                    else s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-zl)));
                    sig[l] = s;
                }
            }
            // gated input: raw * half(s_l * vis_l) (runtime.cu:72-73); pad columns 1.0
#pragma unroll
            for (int p = 0; p < W / 2; ++p) {
                __half h[2] = {lo_half(raw[p]), hi_half(raw[p])};
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const int lev = fm.level_of_col[2 * p + q];
                    if (lev >= 0) {
                        float sl = 0.0f;
#pragma unroll
                        for (int l = 0; l < 16; ++l) sl = (l == lev) ? sig[l] : sl;
                        const __half weight = __float2half_rn(__fmul_rn(sl, float((visbits >> lev) & 1u)));
                        h[q] = __hmul_rn(h[q], weight);
                    }
                }
                wx[p] = pack_half2(h[0], h[1]);
            }
#pragma unroll
            for (int j = 0; j < W / 8; ++j)
                store_chunk(smem, TcSmem::wx, t, j, make_uint4(wx[4 * j], wx[4 * j + 1], wx[4 * j + 2], wx[4 * j + 3]));
        }
        const int in_buf = ROUTER ? TcSmem::wx : TcSmem::x;
        // ---- decoder hidden 1
        uint64_t h1_mask = 0, h2_mask = 0;
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < W / 16; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + in_buf, 128, s), tc::kmajor(sbase + TcSmem::d1, 64, s), ID_D1, s > 0);
        if (!is.complete()) break;
        for (int q = 0; q < 4; ++q) {
            float v[16];
            tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                v[c] = __half2float(__float2half_rn(v[c] > 0.0f ? v[c] : 0.0f));
                h1_mask |= uint64_t(v[c] > 0.0f) << (16 * q + c);
            }
            store_chunk(smem, TcSmem::h1, t, 2 * q, pack8(v));
            store_chunk(smem, TcSmem::h1, t, 2 * q + 1, pack8(v + 8));
        }
        // ---- decoder hidden 2
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::h1, 128, s), tc::kmajor(sbase + TcSmem::d2, 64, s), ID_D2, s > 0);
        if (!is.complete()) break;
        for (int q = 0; q < 4; ++q) {
            float v[16];
            tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                v[c] = __half2float(__float2half_rn(v[c] > 0.0f ? v[c] : 0.0f));
                h2_mask |= uint64_t(v[c] > 0.0f) << (16 * q + c);
            }
            store_chunk(smem, TcSmem::h2, t, 2 * q, pack8(v));
            store_chunk(smem, TcSmem::h2, t, 2 * q + 1, pack8(v + 8));
        }
        // ---- output
        is.before_issue();
        if (t == 0)
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::h2, 128, s), tc::kmajor(sbase + TcSmem::d3, 16, s), ID_D3, s > 0);
        if (!is.complete()) break;
        float out[16];
        tc::tmem_ld16(lane_addr + T_ACC, out);
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
                    const float d = __fsub_rn(__half2float(__float2half_rn(out[c])), __ldg(a.target + 3 * i + c));
                    s = __fadd_rn(s, __fmul_rn(d, d));
                    const float scaled = __fmul_rn(__fdiv_rn(__fmul_rn(2.0f, d), a.three_real), 128.0f);
                    dy[c] = __half2float(__hmul_rn(__float2half_rn(scaled), __float2half_rn(128.0f)));
                }
                a.squares[i] = __fdiv_rn(s, 3.0f);
            }
            store_chunk(smem, TcSmem::dy, t, 0, pack8(dy));
            store_chunk(smem, TcSmem::dy, t, 1, pack8(dy + 8));
        }
        // ---- dh2 = DY Wd3 (B: Wd3 as MN-major); dW3^T += H2^T DY
        is.before_issue();
        if (t == 0) {
            tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::dy, 128, 0), tc::mnmajor(sbase + TcSmem::d3, 16, 0),
                    tc::idesc(128, 64, 0, 1), 0);
            for (int s = 0; s < 8; ++s)
                tc::mma(tmem + T_DW3T, tc::mnmajor(sbase + TcSmem::h2, 128, s), tc::mnmajor(sbase + TcSmem::dy, 128, s),
                        tc::idesc(64, 16, 1, 1), dw_accumulate | uint32_t(s > 0));
        }
        if (!is.complete()) break;
        for (int q = 0; q < 4; ++q) {  // dh2 = relu'(h2) * (.), stored over H2 (dead after dW3)
            float v[16];
            tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
            for (int c = 0; c < 16; ++c) v[c] = (h2_mask >> (16 * q + c) & 1ull) ? v[c] : 0.0f;
            store_chunk(smem, TcSmem::h2, t, 2 * q, pack8(v));
            store_chunk(smem, TcSmem::h2, t, 2 * q + 1, pack8(v + 8));
        }
        // ---- dh1 = DH2 Wd2; dWd2 += DH2^T H1
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::h2, 128, s), tc::mnmajor(sbase + TcSmem::d2, 64, s),
                        tc::idesc(128, 64, 0, 1), s > 0);
            for (int s = 0; s < 8; ++s)
                tc::mma(tmem + T_DWD2, tc::mnmajor(sbase + TcSmem::h2, 128, s), tc::mnmajor(sbase + TcSmem::h1, 128, s),
                        tc::idesc(64, 64, 1, 1), dw_accumulate | uint32_t(s > 0));
        }
        if (!is.complete()) break;
        for (int q = 0; q < 4; ++q) {  // dh1 = relu'(h1) * (.), stored over H1 (dead after dWd2)
            float v[16];
            tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
            for (int c = 0; c < 16; ++c) v[c] = (h1_mask >> (16 * q + c) & 1ull) ? v[c] : 0.0f;
            store_chunk(smem, TcSmem::h1, t, 2 * q, pack8(v));
            store_chunk(smem, TcSmem::h1, t, 2 * q + 1, pack8(v + 8));
        }
        // ---- dz = DH1 Wd1; dWd1 += DH1^T WX
        is.before_issue();
        if (t == 0) {
            for (int s = 0; s < 4; ++s)
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::h1, 128, s), tc::mnmajor(sbase + TcSmem::d1, 64, s),
                        tc::idesc(128, W, 0, 1), s > 0);
            for (int s = 0; s < 8; ++s)
                tc::mma(tmem + T_DWD1, tc::mnmajor(sbase + TcSmem::h1, 128, s), tc::mnmajor(sbase + in_buf, 128, s),
                        tc::idesc(64, W, 1, 1), dw_accumulate | uint32_t(s > 0));
        }
        if (!is.complete()) break;
        __half dz[W];
        for (int q = 0; q < W / 16; ++q) {
            float v[16];
            tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
            for (int c = 0; c < 16; ++c) dz[16 * q + c] = __float2half_rn(v[c]);
        }
        uint32_t gv[W / 2];
        if (!ROUTER) {
            // grid values without router: half(dz / 128) (runtime.cu:123)
#pragma unroll
            for (int p = 0; p < W / 2; ++p)
                gv[p] = pack_half2(__float2half_rn(__fdiv_rn(__half2float(dz[2 * p]), 128.0f)),
                                   __float2half_rn(__fdiv_rn(__half2float(dz[2 * p + 1]), 128.0f)));
        } else {
            // ---- gate backward per level (runtime.cu:76-92): direct and logit gradients
            __half direct[W];
            float da[16];
#pragma unroll
            for (int c = 0; c < W; ++c) direct[c] = __float2half_rn(0.0f);
#pragma unroll
            for (int l = 0; l < 16; ++l) da[l] = 0.0f;
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
                    const __half value = __float2half_rn(__fdiv_rn(__half2float(dz[c]), 128.0f));
                    direct[c] = __hmul_rn(value, weight);
                    const __half rawc = (c & 1) ? hi_half(raw[c >> 1]) : lo_half(raw[c >> 1]);
                    reduced = __hadd_rn(reduced, __hmul_rn(value, rawc));
                }
                const float incoming = __fmul_rn(__half2float(reduced), vis);
                float derivative;
                if (l < a.k_fixed) derivative = 0.0f;
                else if (a.softplus) derivative = incoming * (-expm1f(-sl));
                else derivative = __fmul_rn(__fmul_rn(incoming, __fsub_rn(1.0f, sl)), sl);
                const float dal = __half2float(__hmul_rn(__float2half_rn(derivative), __float2half_rn(128.0f)));
#pragma unroll
                for (int k = 0; k < 16; ++k) da[k] = (k == l) ? dal : da[k];
            }
            store_chunk(smem, TcSmem::da, t, 0, pack8(da));
            store_chunk(smem, TcSmem::da, t, 1, pack8(da + 8));
            // ---- dgh = DA Wg2; dWg2^T += GH^T DA
            is.before_issue();
            if (t == 0) {
                tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::da, 128, 0), tc::mnmajor(sbase + TcSmem::g2, 16, 0),
                        tc::idesc(128, 32, 0, 1), 0);
                for (int s = 0; s < 8; ++s)
                    tc::mma(tmem + T_DWG2T, tc::mnmajor(sbase + TcSmem::gh, 128, s), tc::mnmajor(sbase + TcSmem::da, 128, s),
                            tc::idesc(64, 16, 1, 1), dw_accumulate | uint32_t(s > 0));
            }
            if (!is.complete()) break;
            for (int q = 0; q < 2; ++q) {
                float v[16];
                tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
                for (int c = 0; c < 16; ++c) v[c] = (gh_mask >> (16 * q + c) & 1u) ? v[c] : 0.0f;
                store_chunk(smem, TcSmem::dgh, t, 2 * q, pack8(v));
                store_chunk(smem, TcSmem::dgh, t, 2 * q + 1, pack8(v + 8));
            }
            // ---- dr = DGH Wg1; dWg1 += DGH^T X
            is.before_issue();
            if (t == 0) {
                for (int s = 0; s < 2; ++s)
                    tc::mma(tmem + T_ACC, tc::kmajor(sbase + TcSmem::dgh, 128, s), tc::mnmajor(sbase + TcSmem::g1, 32, s),
                            tc::idesc(128, W, 0, 1), s > 0);
                for (int s = 0; s < 8; ++s)
                    tc::mma(tmem + T_DWG1, tc::mnmajor(sbase + TcSmem::dgh, 128, s), tc::mnmajor(sbase + TcSmem::x, 128, s),
                            tc::idesc(64, W, 1, 1), dw_accumulate | uint32_t(s > 0));
            }
            if (!is.complete()) break;
            for (int q = 0; q < W / 16; ++q) {
                float v[16];
                tc::tmem_ld16(lane_addr + T_ACC + 16 * q, v);
#pragma unroll
                for (int c = 0; c < 16; c += 2) {
                    const int col = 16 * q + c;
                    const __half r0 = __float2half_rn(__fdiv_rn(__half2float(__float2half_rn(v[c])), 128.0f));
                    const __half r1 = __float2half_rn(__fdiv_rn(__half2float(__float2half_rn(v[c + 1])), 128.0f));
                    gv[col >> 1] = pack_half2(__hadd_rn(direct[col], r0), __hadd_rn(direct[col + 1], r1));
                }
            }
        }
        if (valid) {
#pragma unroll
            for (int p = 0; p < W / 2; ++p) reinterpret_cast<uint32_t*>(a.gvals)[(long long)p * a.stride + i] = gv[p];
        }
        dw_accumulate = 1;
    }

    if (!is.ok) {
        if (t == 0) atomicExch(error_flag, 2);
        // give products still in flight a bounded chance to land before TMEM is released
        if (t == 0) tc::commit(bar);
        tc::bar_wait(bar, is.phase, WAIT_LIMIT);
    }
    if (TRAIN) {
        // ---- weight gradients: TMEM (M=64 layout: rows 16w..16w+15 in lanes 32w..32w+15) -> partials
        constexpr int GATE = ROUTER ? gate_params(W) : 0;
        constexpr int P = GATE + decoder_params(W);
        float* part = a.partials + (long long)blockIdx.x * P;
        const int row = 16 * warp + (t & 31);
        const bool holds = (t & 31) < 16;
        const bool any = dw_accumulate && is.ok;
        tc::fence_before_sync();
        __syncthreads();
        tc::fence_after_sync();
        float* dec = part + GATE;
        for (int q = 0; q < 4; ++q) {  // dWd2 [64][64]
            float v[16];
            tc::tmem_ld16(lane_addr + T_DWD2 + 16 * q, v);
            if (holds)
                for (int c = 0; c < 16; ++c) dec[DEC_HIDDEN * W + row * DEC_HIDDEN + 16 * q + c] = any ? v[c] : 0.0f;
        }
        for (int q = 0; q < W / 16; ++q) {  // dWd1 [64][W]
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
            for (int q = 0; q < W / 16; ++q) {  // dWg1 [32][W] from [64 (32 valid)][W]
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

template <bool ROUTER, bool TRAIN>
void launch_tc(const MlpArgs& a, int blocks, int* error_flag, cudaStream_t stream) {
    static unsigned long long configured = 0;
    int device = 0;
    ODIE_CUDA(cudaGetDevice(&device));
    if (!(configured >> device & 1ull)) {
        ODIE_CUDA(cudaFuncSetAttribute(mlp_tc_kernel<ROUTER, TRAIN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       TcSmem::total));
        configured |= 1ull << device;
    }
    mlp_tc_kernel<ROUTER, TRAIN><<<blocks, TC_THREADS, TcSmem::total, stream>>>(a, error_flag);
}

}  // namespace

int mlp_tc_blocks(long long n) {
    const long long tiles = (n + TC_TILE - 1) / TC_TILE;
    long long blocks = 2LL * sm_count();
    if (blocks > tiles) blocks = tiles;
    return blocks < 1 ? 1 : int(blocks);
}

void launch_mlp_tc_train(const MlpArgs& a, int width, bool router, int blocks, int* error_flag, cudaStream_t stream) {
    ODIE_REQUIRE(width == 32, "the tcgen05 heads take 32 input features");
    if (a.n <= 0) return;
    if (router) launch_tc<true, true>(a, blocks, error_flag, stream);
    else launch_tc<false, true>(a, blocks, error_flag, stream);
}

void launch_mlp_tc_decode(const MlpArgs& a, int width, bool router, int* error_flag, cudaStream_t stream) {
    ODIE_REQUIRE(width == 32, "the tcgen05 heads take 32 input features");
    if (a.n <= 0) return;
    const int blocks = mlp_tc_blocks(a.n);
    if (router) launch_tc<true, false>(a, blocks, error_flag, stream);
    else launch_tc<false, false>(a, blocks, error_flag, stream);
}

}  // namespace odie
