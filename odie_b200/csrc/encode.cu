// Multiresolution 2-D grid encoding: forward gather and backward scatter.
//
// One thread per (coordinate, level); grid = (ceil(n/256), levels).  The
// forward interpolates the 4 corners with the fp16 fused-multiply-add chain of
// the reference (odie/packed_kernels.cu:38-64), reading either the fp32 master
// table (module path) or the library's fp16 mirror (training step; the values
// are bit-identical because the reference rounds every fp32 corner value to
// fp16 before the chain).  The backward scatter-adds w_k * g into an fp32
// gradient (odie/packed_kernels.cu:66-88, odie/native/runtime.cu:111-143) with
// 8-byte vector reductions for F=2, one thread per coordinate in a scrambled
// visiting order, and shared-memory pre-aggregation of coarse levels.
#include <atomic>

#include "encode.cuh"

namespace odie {

namespace {

__device__ __forceinline__ Level level_from_descriptor(const int* __restrict__ d) {
    // Reference descriptor row [R, points, plane offset, node word offset,
    // cell bitmap offset, F, feature offset, direct] (odie/model.py:100-101).
    Level L;
    L.scale = float(__ldg(d + 0) - 1);
    L.res = __ldg(d + 0);
    L.points = __ldg(d + 1);
    L.offset = __ldg(d + 2);
    L.words = __ldg(d + 7) ? -1 : __ldg(d + 3);
    L.cells = __ldg(d + 4);
    L.F = __ldg(d + 5);
    L.col = __ldg(d + 6);
    L.kind = PLANE;
    return L;
}

template <bool FROM_DESC>
__device__ __forceinline__ Level fetch_level(const int* desc, const LevelTable& table, int l) {
    if (FROM_DESC) return level_from_descriptor(desc + 8 * l);
    return table.level[l];
}

// Visibility of a coordinate's cell: plane cells, and hash-level cells when the
// level has an allocation bitmap (cells >= 0; on-demand allocation of routed
// experts), are looked up in the cell bitmap.  A cell outside the R x R grid
// (coordinates outside [0, 1], which the reference never produces) is treated
// as hidden instead of reading outside the bitmap.
__device__ __forceinline__ bool level_on(const Level& d, const Corner4& g, const uint8_t* __restrict__ bitmap) {
    if (d.kind != PLANE && (d.cells < 0 || !bitmap)) return true;
    if (g.ix < 0 || g.iy < 0 || g.ix >= d.res || g.iy >= d.res) return false;
    return cell_visible(d, bitmap, level_cell(d, g));
}

__device__ __forceinline__ __half2 load_pair(const float* __restrict__ t, long long index) {
    const float2 v = __ldg(reinterpret_cast<const float2*>(t + index));
    return __floats2half2_rn(v.x, v.y);
}
__device__ __forceinline__ __half2 load_pair(const __half* __restrict__ t, long long index) {
    return __ldg(reinterpret_cast<const __half2*>(t + index));
}
__device__ __forceinline__ __half load_one(const float* __restrict__ t, long long index) {
    return __float2half_rn(__ldg(t + index));
}
__device__ __forceinline__ __half load_one(const __half* __restrict__ t, long long index) { return __ldg(t + index); }

__device__ __forceinline__ void store_feature(__half* out, bool row_major, long long i, int col, int width,
                                              long long stride, __half v) {
    if (row_major) out[i * width + col] = v;
    else out[((long long)(col >> 1) * stride + i) * 2 + (col & 1)] = v;
}

template <typename T, bool FROM_DESC>
__global__ void __launch_bounds__(256) encode_forward_kernel(const EncodeArgs a, const int* desc,
                                                             const __grid_constant__ LevelTable table,
                                                             const T* __restrict__ params, __half* __restrict__ out,
                                                             uint8_t* __restrict__ vis) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const int l = blockIdx.y;
    const bool inside = i < a.n;
    const Level d = fetch_level<FROM_DESC>(desc, table, l);
    Corner4 g{};
    bool on = false;
    if (inside) {
        const float2 p = __ldg(reinterpret_cast<const float2*>(a.coords) + i);
        g = geometry(p.x, p.y, d.scale);
        on = l < a.active && level_on(d, g, a.bitmap);
    }
    if (vis) {
        if (a.row_major) {
            if (inside) vis[i * a.levels + l] = on;
        } else {
            // bit-packed [levels][stride / 32] words: one ballot per warp of 32 consecutive coordinates
            const unsigned bits = __ballot_sync(0xffffffffu, on);
            if ((threadIdx.x & 31) == 0 && inside)
                reinterpret_cast<uint32_t*>(vis)[(long long)l * (a.stride >> 5) + (i >> 5)] = bits;
        }
    }
    if (!inside) return;
    const long long base = d.offset + (a.expert ? (long long)__ldg(a.expert + i) * a.expert_stride : 0LL);
    if (d.F == 2) {
        __half2 acc = __float2half2_rn(0.0f);
        if (on) {
            int rows[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) rows[k] = corner_row(d, g, k, a.node_bitmap, a.node_prefix);
            __half2 t[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) t[k] = load_pair(params, base + 2LL * rows[k]);
            // __hfma2 rounds each lane once, exactly as the reference's per-channel __hfma chain.
#pragma unroll
            for (int k = 0; k < 4; ++k) acc = __hfma2(half2_dup(g.w[k]), t[k], acc);
        }
        if (!a.row_major && (d.col & 1) == 0) {
            reinterpret_cast<__half2*>(out)[(long long)(d.col >> 1) * a.stride + i] = acc;
        } else if (a.row_major && (d.col & 1) == 0 && (a.width & 1) == 0) {
            reinterpret_cast<__half2*>(out)[(i * a.width + d.col) >> 1] = acc;
        } else {
            store_feature(out, a.row_major, i, d.col, a.width, a.stride, __low2half(acc));
            store_feature(out, a.row_major, i, d.col + 1, a.width, a.stride, __high2half(acc));
        }
        return;
    }
    int rows[4] = {0, 0, 0, 0};
    if (on) {
#pragma unroll
        for (int k = 0; k < 4; ++k) rows[k] = corner_row(d, g, k, a.node_bitmap, a.node_prefix);
    }
    for (int c = 0; c < d.F; ++c) {
        __half acc = __float2half_rn(0.0f);
        if (on) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                acc = __hfma(__float2half_rn(g.w[k]), load_one(params, base + (long long)rows[k] * d.F + c), acc);
        }
        store_feature(out, a.row_major, i, d.col + c, a.width, a.stride, acc);
    }
}

// Row-major forward for tables whose levels all have F=2 at columns (2l, 2l+1)
// (a hash-grid layout) and no visibility output: one thread per coordinate over
// all its levels, its W-half row written as 16-byte stores.  Used for the router
// grid, whose small tables stay in L1.
// The 4 corner pairs of one level of the row gather, corner addressing compiled for KIND.
template <int KIND>
__device__ __forceinline__ void corner_pairs(const EncodeArgs& a, const Level& d, const Corner4& g, long long base,
                                             const __half* __restrict__ params, __half2 (&t)[4]) {
#pragma unroll
    for (int k = 0; k < 4; ++k)
        t[k] = load_pair(params, base + d.offset + 2LL * corner_row<KIND>(d, g, k, a.node_bitmap, a.node_prefix));
}

// KIND: every level's kind when they all share one (compiled out of the corner addressing).
// KIND = -1 with split >= 0: levels [0, split) are dense and [split, levels) hashed (a hash
// grid's usual order), each range addressed with its own compiled kind; split < 0: any kinds,
// read per level.
template <int W, int KIND>
__global__ void __launch_bounds__(256) encode_forward_rows_kernel(const EncodeArgs a,
                                                                  const __grid_constant__ LevelTable table,
                                                                  const __half* __restrict__ params,
                                                                  __half* __restrict__ out, int split) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.n) return;
    const float2 p = __ldg(reinterpret_cast<const float2*>(a.coords) + i);
    const long long base = a.expert ? (long long)__ldg(a.expert + i) * a.expert_stride : 0LL;
    uint4* dst = reinterpret_cast<uint4*>(out + i * W);
    // four levels at a time, each group's 16 bytes stored as soon as they are complete (the row never needs a
    // dynamically indexed array)
#pragma unroll 1
    for (int l0 = 0; l0 < W / 2; l0 += 4) {
        uint32_t row[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int l = l0 + q;
            __half2 acc = __float2half2_rn(0.0f);
            if (l < a.levels && l < a.active) {
                const Level d = table.level[l];
                const Corner4 g = geometry(p.x, p.y, d.scale);
                if (level_on(d, g, a.bitmap)) {
                    __half2 t[4];
                    if (KIND >= 0 || split < 0) corner_pairs<KIND>(a, d, g, base, params, t);
                    else if (l < split) corner_pairs<HASH_DENSE>(a, d, g, base, params, t);
                    else corner_pairs<HASH_HASHED>(a, d, g, base, params, t);
#pragma unroll
                    for (int k = 0; k < 4; ++k) acc = __hfma2(half2_dup(g.w[k]), t[k], acc);
                }
            }
            row[q] = pack_half2(__low2half(acc), __high2half(acc));
        }
        dst[l0 / 4] = make_uint4(row[0], row[1], row[2], row[3]);
    }
}

// Gradient value of column col of coordinate i: fp16 rows (the fp16 network) or fp32 rows (the fp32 hash grid).
__device__ __forceinline__ float as_float(__half v) { return __half2float(v); }
__device__ __forceinline__ float as_float(float v) { return v; }
template <typename U>
__device__ __forceinline__ float upstream_value(const U* __restrict__ up, const EncodeArgs& a, long long i, int col) {
    if (a.row_major) return as_float(up[i * a.width + col]);
    return as_float(up[((long long)(col >> 1) * a.stride + i) * 2 + (col & 1)]);
}
// The value pairs of columns (2c0, 2c0 + 1) .. (2c0 + 6, 2c0 + 7) of row-major row i, 16-byte aligned:
// one 16-byte load of fp16 values, two of fp32 ones.
__device__ __forceinline__ void load_pairs4(const __half* __restrict__ up, long long i, int width, int c0, float (&u)[8]) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(up + i * width + 2 * c0));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        u[2 * g] = __half2float(lo_half(w[g]));
        u[2 * g + 1] = __half2float(hi_half(w[g]));
    }
}
__device__ __forceinline__ void load_pairs4(const float* __restrict__ up, long long i, int width, int c0, float (&u)[8]) {
    const float4* src = reinterpret_cast<const float4*>(up + i * width + 2 * c0);
    const float4 a = __ldg(src), b = __ldg(src + 1);
    u[0] = a.x; u[1] = a.y; u[2] = a.z; u[3] = a.w;
    u[4] = b.x; u[5] = b.y; u[6] = b.z; u[7] = b.w;
}

// Visiting order of the direct scatter kernel.  Training batches are often
// spatially coherent (the reference's default stratified sampler emits
// neighbouring pixels consecutively), and then warps that run together would
// reduce into the same table entries and serialise on them.  The kernel keeps
// each warp on 32 consecutive coordinates (so lanes that share a cell can be
// combined, below) but scrambles the order of these 32-coordinate groups: warp w
// takes group (w * PERM_MULT) mod 2^k, 2^k >= the number of groups (groups past
// the end are skipped) -- a bijection that spreads neighbouring groups across
// the launch.  mask = 2^k - 1.
constexpr uint32_t PERM_MULT = 0x9E3779B1u;
__device__ __forceinline__ long long visit(long long t, uint32_t mask) {
    return mask ? (long long)((uint32_t(t) * PERM_MULT) & mask) : t;
}

// Sum runs of consecutive lanes with equal keys (segmented inclusive scan):
// afterwards the last lane of each run holds the run's totals.
__device__ __forceinline__ void run_sums(float (&v)[8], bool head) {
    const int lane = threadIdx.x & 31;
    bool f = head;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        float up[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) up[j] = __shfl_up_sync(0xffffffffu, v[j], d);
        const bool fu = __shfl_up_sync(0xffffffffu, f, d);
        if (lane >= d && !f) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(up[j], v[j]);
        }
        if (lane >= d) f = f || fu;
    }
}

// Combine the 8 corner updates (4 corners x 2 features) of lanes that share a
// cell (key): all lanes in one cell -> butterfly sum, lane 0 writes; no two
// neighbouring lanes in one cell -> every lane writes; otherwise runs of equal
// keys are summed and the last lane of each run writes.  Returns whether this
// lane writes.  Warp-collective.
__device__ __forceinline__ bool combine_lanes(float (&v)[8], long long key, bool on) {
    const int lane = threadIdx.x & 31;
    const long long prev = __shfl_up_sync(0xffffffffu, key, 1);
    const long long next = __shfl_down_sync(0xffffffffu, key, 1);
    const unsigned joined = __ballot_sync(0xffffffffu, lane > 0 && prev == key);
    if (joined == 0xfffffffeu) {  // one cell for the whole warp
#pragma unroll
        for (int m = 16; m > 0; m >>= 1)
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], __shfl_xor_sync(0xffffffffu, v[j], m));
        return on && lane == 0;
    }
    if (joined) {
        run_sums(v, lane == 0 || prev != key);
        return on && (lane == 31 || next != key);
    }
    return on;
}

// combine_lanes with a two-part key (key, tag): lanes combine when both parts are equal.
__device__ __forceinline__ bool combine_lanes(float (&v)[8], long long key, int tag, bool on) {
    const int lane = threadIdx.x & 31;
    const long long prev = __shfl_up_sync(0xffffffffu, key, 1);
    const long long next = __shfl_down_sync(0xffffffffu, key, 1);
    const int prev_tag = __shfl_up_sync(0xffffffffu, tag, 1);
    const int next_tag = __shfl_down_sync(0xffffffffu, tag, 1);
    const bool same_prev = lane > 0 && prev == key && prev_tag == tag;
    const bool same_next = lane < 31 && next == key && next_tag == tag;
    const unsigned joined = __ballot_sync(0xffffffffu, same_prev);
    if (joined == 0xfffffffeu) {  // one cell for the whole warp
#pragma unroll
        for (int m = 16; m > 0; m >>= 1)
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], __shfl_xor_sync(0xffffffffu, v[j], m));
        return on && lane == 0;
    }
    if (joined) {
        run_sums(v, !same_prev);
        return on && !same_next;
    }
    return on;
}

// Direct scatter: one warp per 32 consecutive coordinates (group order
// scrambled), each lane one coordinate over all its levels not in skip_levels
// (those go through the shared-memory kernel below).  F=2 levels combine lanes
// that share a cell before the 8-byte vector reductions.
// ROWS: the values are row-major rows of 32 (level l in columns 2l, 2l + 1, 16-byte aligned): each thread reads
// its coordinate's row once with 16-byte loads into its own shared-memory row (odd word stride: no bank
// conflicts) instead of two scattered loads per level.
template <typename U>
struct RowWords {
    static constexpr int words = 32 * int(sizeof(U)) / 4;  // 16 for fp16 values, 32 for fp32
    static constexpr int stride = words + 1;
};

template <bool FROM_DESC, typename U, bool ROWS>
__global__ void __launch_bounds__(256) encode_backward_kernel(const EncodeArgs a, const int* desc,
                                                              const __grid_constant__ LevelTable table,
                                                              const U* __restrict__ upstream,
                                                              float* __restrict__ grad, unsigned skip_levels,
                                                              uint32_t mask, int split) {
    using RW = RowWords<U>;
    __shared__ uint32_t s_rows[ROWS ? 256 * RW::stride : 1];
    const long long warp_id = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const long long i = visit(warp_id, mask) * 32 + lane;
    const bool valid = i < a.n;
    if (__all_sync(0xffffffffu, !valid)) return;  // a whole group past the end (uniform per warp)
    float2 p = make_float2(0.0f, 0.0f);
    long long base = 0;
    int e = 0;
    if (valid) {
        p = __ldg(reinterpret_cast<const float2*>(a.coords) + i);
        if (a.expert) {
            e = __ldg(a.expert + i);
            base = (long long)e * a.expert_stride;
        }
    }
    uint32_t* const my_row = s_rows + (ROWS ? threadIdx.x * RW::stride : 0);
    if (ROWS) {
        const uint4* src = reinterpret_cast<const uint4*>(upstream + (valid ? i : 0) * 32);
#pragma unroll
        for (int j = 0; j < RW::words / 4; ++j) {
            const uint4 q = valid ? __ldg(src + j) : make_uint4(0, 0, 0, 0);
            my_row[4 * j] = q.x;
            my_row[4 * j + 1] = q.y;
            my_row[4 * j + 2] = q.z;
            my_row[4 * j + 3] = q.w;
        }
    }
    const int levels = a.active < a.levels ? a.active : a.levels;
#pragma unroll 2
    for (int l = 0; l < levels; ++l) {
        if (skip_levels >> l & 1u) continue;  // uniform
        const Level d = fetch_level<FROM_DESC>(desc, table, l);
        const Corner4 g = geometry(p.x, p.y, d.scale);
        const bool on = valid && level_on(d, g, a.bitmap);
        float* const level_grad = grad + d.offset + base;
        if (d.F == 2) {  // uniform
            float u0 = 0.0f, u1 = 0.0f;
            if (ROWS) {
                if (sizeof(U) == 2) {
                    const uint32_t w = my_row[l];
                    u0 = __half2float(lo_half(w));
                    u1 = __half2float(hi_half(w));
                } else {
                    u0 = __uint_as_float(my_row[2 * l]);
                    u1 = __uint_as_float(my_row[2 * l + 1]);
                }
                if (!on) u0 = u1 = 0.0f;
            } else if (on) {
                u0 = upstream_value(upstream, a, i, d.col);
                u1 = upstream_value(upstream, a, i, d.col + 1);
            }
            float v[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v[2 * k] = __fmul_rn(g.w[k], u0);
                v[2 * k + 1] = __fmul_rn(g.w[k], u1);
            }
            // cell key (expert, cell): equal keys share the 4 corner entries; lanes without a contribution
            // get distinct negative keys
            const long long key = on ? ((long long)e << 32) + level_cell(d, g) : -1LL - lane;
            if (!combine_lanes(v, key, on)) continue;
            if (v[0] == 0.0f && v[1] == 0.0f && v[2] == 0.0f && v[3] == 0.0f && v[4] == 0.0f && v[5] == 0.0f &&
                v[6] == 0.0f && v[7] == 0.0f)
                continue;
            // corner addressing compiled per kind where the level's kind is known: planes (descriptors), or a
            // hash grid's dense levels [0, split) and hashed levels [split, levels)
            int rows[4];
            if (FROM_DESC || split < 0) {
#pragma unroll
                for (int k = 0; k < 4; ++k) rows[k] = corner_row(d, g, k, a.node_bitmap, a.node_prefix);
            } else if (l < split) {
#pragma unroll
                for (int k = 0; k < 4; ++k) rows[k] = corner_row<HASH_DENSE>(d, g, k, a.node_bitmap, a.node_prefix);
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) rows[k] = corner_row<HASH_HASHED>(d, g, k, a.node_bitmap, a.node_prefix);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) red_add_v2(level_grad + 2LL * rows[k], v[2 * k], v[2 * k + 1]);
            continue;
        }
        if (!on) continue;
        int rows[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) rows[k] = corner_row(d, g, k, a.node_bitmap, a.node_prefix);
        for (int c = 0; c < d.F; ++c) {
            const float v = upstream_value(upstream, a, i, d.col + c);
            if (v == 0.0f) continue;
#pragma unroll
            for (int k = 0; k < 4; ++k) red_add_f32(level_grad + (long long)rows[k] * d.F + c, __fmul_rn(g.w[k], v));
        }
    }
}

// Coarse levels: every block accumulates the gradients of all small levels
// (the listed ones) for its share of the coordinates in shared memory, then
// adds each non-zero entry to global memory once.  This turns the heavy
// same-address contention of coarse tables (2^20 coordinates into a few hundred
// nodes) into shared-memory updates plus blocks x table-size global reductions,
// and reads each coordinate and its gradient row once for all those levels.
// With routed experts the block holds each level's table of every expert,
// expert-major.
struct CoarseList {
    int count;                // levels held in shared memory
    int total;                // floats of shared memory they take
    int level[MAX_LEVELS];
    int offset[MAX_LEVELS];   // first float of each listed level's tables in shared memory
};

// Shared-memory atomics serialise on equal addresses too: on levels with at most
// RUN_RES cells per axis the lanes of a warp that share a cell are combined first
// (combine_lanes); any visiting order is correct, the saving grows with the
// coherence of the batch.
constexpr int RUN_RES = 64;

template <typename U>
__global__ void __launch_bounds__(512) encode_backward_shared_kernel(const EncodeArgs a,
                                                                     const __grid_constant__ LevelTable table,
                                                                     const __grid_constant__ CoarseList list,
                                                                     const U* __restrict__ upstream,
                                                                     float* __restrict__ grad) {
    extern __shared__ float acc[];
    const int experts = a.expert ? a.experts : 1;
    const int lane = threadIdx.x & 31;
    for (int j = threadIdx.x; j < list.total; j += blockDim.x) acc[j] = 0.0f;
    __syncthreads();
    const long long chunk = (a.n + gridDim.x - 1) / gridDim.x;
    const long long begin = (long long)blockIdx.x * chunk;
    const long long end = begin + chunk < a.n ? begin + chunk : a.n;
    // whole warps iterate together (the run sums shuffle across the warp)
    for (long long base = begin + (threadIdx.x & ~31); base < end; base += blockDim.x) {
        const long long i = base + lane;
        int e = 0;
        bool valid = i < end;
        float2 p = make_float2(0.0f, 0.0f);
        if (valid) {
            e = a.expert ? __ldg(a.expert + i) : 0;
            valid = e >= 0 && e < experts;  // an id outside the tables would land outside shared memory
            p = __ldg(reinterpret_cast<const float2*>(a.coords) + i);
        }
        for (int c = 0; c < list.count; ++c) {
            const Level d = table.level[list.level[c]];
            const Corner4 g = geometry(p.x, p.y, d.scale);
            const bool on = valid && level_on(d, g, a.bitmap);
            float* const tab = acc + list.offset[c] + e * d.points * d.F;
            if (d.F == 2 && d.res <= RUN_RES) {  // warp-uniform branch
                // cell key within this expert's table; lanes without a contribution get distinct negative keys
                const long long key = on ? ((long long)e << 32) + level_cell(d, g) : -1LL - lane;
                float v[8];
                const float u0 = on ? upstream_value(upstream, a, i, d.col) : 0.0f;
                const float u1 = on ? upstream_value(upstream, a, i, d.col + 1) : 0.0f;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    v[2 * k] = __fmul_rn(g.w[k], u0);
                    v[2 * k + 1] = __fmul_rn(g.w[k], u1);
                }
                if (combine_lanes(v, key, on)) {
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int row = corner_row(d, g, k, a.node_bitmap, a.node_prefix);
                        if (v[2 * k] != 0.0f) atomicAdd(tab + 2 * row, v[2 * k]);
                        if (v[2 * k + 1] != 0.0f) atomicAdd(tab + 2 * row + 1, v[2 * k + 1]);
                    }
                }
                continue;
            }
            if (!on) continue;
            int rows[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) rows[k] = corner_row(d, g, k, a.node_bitmap, a.node_prefix);
            for (int f = 0; f < d.F; ++f) {
                const float v = upstream_value(upstream, a, i, d.col + f);
                if (v == 0.0f) continue;
#pragma unroll
                for (int k = 0; k < 4; ++k) atomicAdd(tab + rows[k] * d.F + f, __fmul_rn(g.w[k], v));
            }
        }
    }
    __syncthreads();
    for (int c = 0; c < list.count; ++c) {
        const Level d = table.level[list.level[c]];
        const int per_table = d.points * d.F;
        const float* tab = acc + list.offset[c];
        for (int j = threadIdx.x; j < per_table * experts; j += blockDim.x) {
            const float v = tab[j];
            if (v == 0.0f) continue;
            const int x = j / per_table;
            red_add_f32(grad + d.offset + (long long)x * a.expert_stride + (j - x * per_table), v);
        }
    }
}


// Lane-contiguous runs over the shared-memory levels (all with F = 2): each
// thread walks its own run of consecutive coordinates and keeps, for each level
// of a group of RUNS_GROUP levels, the running sums of the 8 corner updates
// (4 corners x 2 features) of the cell it is in; it adds them to the block's
// shared tables only when the cell changes and at the end of its run.  On a
// spatially coherent batch (the reference's stratified sampler) a coarse cell
// spans many consecutive coordinates, so most updates are register FMAs and the
// shared-memory atomics -- which serialise on equal addresses -- become rare.
// VEC: the gradient values are row-major and listed level c has columns
// (2c, 2c + 1), so one 16-byte load brings a group's 4 value pairs.
constexpr int RUNS_THREADS = 384;
static_assert(RUNS_THREADS % (32 * 12) == 0, "1 to 4 warp groups of whole warps");
constexpr int RUNS_GROUP = 4;

// Adds one cell's 8 corner sums to the block's shared table of expert e and clears them.
template <int KIND>
__device__ __forceinline__ void runs_flush(const Level& d, float* tab, int e, int ix, int iy, float (&v)[8],
                                           const uint64_t* __restrict__ node_bitmap, const int* __restrict__ prefix) {
    Corner4 g;
    g.ix = ix;
    g.iy = iy;
    float* const t = tab + (long long)e * d.points * 2;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int row = corner_row<KIND>(d, g, k, node_bitmap, prefix);
        // straight-line adds: adding an exact zero leaves an entry as it is
        atomicAdd(t + 2 * row, v[2 * k]);
        atomicAdd(t + 2 * row + 1, v[2 * k + 1]);
        v[2 * k] = 0.0f;
        v[2 * k + 1] = 0.0f;
    }
}

template <bool VEC, int KIND, typename U>
__global__ void __launch_bounds__(RUNS_THREADS, 2) encode_backward_runs_kernel(const EncodeArgs a,
                                                                              const __grid_constant__ LevelTable table,
                                                                              const __grid_constant__ CoarseList list,
                                                                              const U* __restrict__ upstream,
                                                                              float* __restrict__ grad) {
    extern __shared__ float acc[];
    const int experts = a.expert ? a.experts : 1;
    for (int j = threadIdx.x; j < list.total; j += blockDim.x) acc[j] = 0.0f;
    __syncthreads();
    const long long chunk = (a.n + gridDim.x - 1) / gridDim.x;
    const long long begin = (long long)blockIdx.x * chunk;
    const long long end = begin + chunk < a.n ? begin + chunk : a.n;
    const long long run = (chunk + blockDim.x - 1) / blockDim.x;
    const long long first = begin + threadIdx.x * run;
    const long long last = first + run < end ? first + run : end;
    const float2* const coords = reinterpret_cast<const float2*>(a.coords);
    for (int c0 = 0; c0 < list.count; c0 += RUNS_GROUP) {
        int ce[RUNS_GROUP], cx[RUNS_GROUP], cy[RUNS_GROUP];
        float v[RUNS_GROUP][8];
#pragma unroll
        for (int g = 0; g < RUNS_GROUP; ++g) {
            ce[g] = -1;
            cx[g] = cy[g] = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) v[g][j] = 0.0f;
        }
        for (long long i = first; i < last; ++i) {
            int e = 0;
            bool valid = true;
            if (a.expert) {
                e = __ldg(a.expert + i);
                valid = e >= 0 && e < experts;  // an id outside the tables would land outside shared memory
            }
            const float2 p = __ldg(coords + i);
            float pairs[2 * RUNS_GROUP];
            if (VEC) load_pairs4(upstream, i, a.width, c0, pairs);
#pragma unroll
            for (int g = 0; g < RUNS_GROUP; ++g) {
                const int c = c0 + g;
                if (c >= list.count) break;
                const Level d = table.level[list.level[c]];
                const Corner4 geo = geometry(p.x, p.y, d.scale);
                if (!valid || !level_on(d, geo, a.bitmap)) continue;
                if (geo.ix != cx[g] || geo.iy != cy[g] || e != ce[g]) {
                    if (ce[g] >= 0)
                        runs_flush<KIND>(d, acc + list.offset[c], ce[g], cx[g], cy[g], v[g], a.node_bitmap, a.node_prefix);
                    ce[g] = e;
                    cx[g] = geo.ix;
                    cy[g] = geo.iy;
                }
                float u0, u1;
                if (VEC) {
                    u0 = pairs[2 * g];
                    u1 = pairs[2 * g + 1];
                } else {
                    u0 = upstream_value(upstream, a, i, d.col);
                    u1 = upstream_value(upstream, a, i, d.col + 1);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    v[g][2 * k] = __fmaf_rn(geo.w[k], u0, v[g][2 * k]);
                    v[g][2 * k + 1] = __fmaf_rn(geo.w[k], u1, v[g][2 * k + 1]);
                }
            }
        }
        // the runs end together: neighbouring lanes often end in one cell, so they are combined first
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int g = 0; g < RUNS_GROUP; ++g) {
            const int c = c0 + g;
            if (c >= list.count) break;
            const bool on = ce[g] >= 0;
            const long long key = ((long long)cx[g] << 32) | uint32_t(cy[g]);
            if (combine_lanes(v[g], key, on ? ce[g] : -1 - lane, on))
                runs_flush<KIND>(table.level[list.level[c]], acc + list.offset[c], ce[g], cx[g], cy[g], v[g],
                                 a.node_bitmap, a.node_prefix);
        }
    }
    __syncthreads();
    for (int c = 0; c < list.count; ++c) {
        const Level d = table.level[list.level[c]];
        const int per_table = d.points * d.F;
        const float* tab = acc + list.offset[c];
        for (int j = threadIdx.x; j < per_table * experts; j += blockDim.x) {
            const float v = tab[j];
            if (v == 0.0f) continue;
            const int x = j / per_table;
            red_add_f32(grad + d.offset + (long long)x * a.expert_stride + (j - x * per_table), v);
        }
    }
}

// Adds one cell's 8 corner sums straight to the gradient (two-float vector reductions: F = 2 entries are
// adjacent and 8-byte aligned) and clears them.
template <int KIND>
__device__ __forceinline__ void runs_flush_global(const Level& d, float* grad, int ix, int iy, float (&v)[8]) {
    Corner4 g;
    g.ix = ix;
    g.iy = iy;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int row = corner_row<KIND>(d, g, k, nullptr, nullptr);
        red_add_v2(grad + d.offset + 2 * row, v[2 * k], v[2 * k + 1]);
        v[2 * k] = 0.0f;
        v[2 * k + 1] = 0.0f;
    }
}

// The scatter strategy of the plain runs kernel, chosen per launch on the device by runs_probe_kernel.
//
// RUNS_SHARED: each block accumulates the listed levels in its shared-memory tables (shared-memory atomics)
// and adds them to global memory at the end.  Needed when consecutive coordinates rarely share a cell
// (uniform batches): every coordinate then flushes at every level, and global reductions into a coarse
// level's few entries would serialise in L2.
// RUNS_GLOBAL: no shared-memory tables; each flush goes straight to global memory.  On a spatially coherent
// batch (the reference's stratified sampler) flushes are rare, and without the tables' shared-memory
// allocation the L1 keeps the room that the runs' per-lane loads (each lane walks its own run, so one warp
// load touches 32 lines) need to stay in flight: 2.7x faster on the routed-expert benchmark's router grid.
constexpr int RUNS_SHARED = 0, RUNS_GLOBAL = 1;

// The runs scatter for the common case of the single-table grids (the router grid, the fp32 hash grid): no
// expert ids, no cell that visibility can hide, value rows read 16 bytes per group.  The same runs and flushes
// as encode_backward_runs_kernel, with each group's scales read once per run and no per-coordinate checks.
// strategy: the device int runs_probe_kernel wrote (the kernel returns at once unless it names STRATEGY), or
// null (RUNS_SHARED runs unconditionally).
template <int KIND, typename U, int STRATEGY>
__global__ void __launch_bounds__(RUNS_THREADS, 2) encode_backward_runs_plain_kernel(const EncodeArgs a,
                                                                                    const __grid_constant__ LevelTable table,
                                                                                    const __grid_constant__ CoarseList list,
                                                                                    const U* __restrict__ upstream,
                                                                                    float* __restrict__ grad,
                                                                                    const int* __restrict__ strategy) {
    if (strategy && *strategy != STRATEGY) return;
    extern __shared__ float acc[];
    if (STRATEGY == RUNS_SHARED) {
        for (int j = threadIdx.x; j < list.total; j += blockDim.x) acc[j] = 0.0f;
        __syncthreads();
    }
    // RUNS_GLOBAL: the block's threads form one warp group per group of RUNS_GROUP levels (up to four), side
    // by side over the same runs, so that the groups' reads of a value row land close together in time and
    // hit L1 (one pass after another re-read every row from DRAM: four passes over the router grid's rows
    // moved 4x their bytes).  RUNS_SHARED: one group, the passes one after another.
    const int passes = (list.count + RUNS_GROUP - 1) / RUNS_GROUP;
    const int groups = STRATEGY == RUNS_GLOBAL ? (passes < 4 ? passes : 4) : 1;
    const int per = blockDim.x / groups;  // RUNS_THREADS / groups: a multiple of 32, so warps stay whole
    const int group = threadIdx.x / per;
    const long long chunk = (a.n + gridDim.x - 1) / gridDim.x;
    const long long begin = (long long)blockIdx.x * chunk;
    const long long end = begin + chunk < a.n ? begin + chunk : a.n;
    const long long run = (chunk + per - 1) / per;
    const long long first = begin + (threadIdx.x - group * per) * run;
    const long long last = first + run < end ? first + run : end;
    const float2* const coords = reinterpret_cast<const float2*>(a.coords);
    auto flush = [&](int c, int ix, int iy, float (&v)[8]) {
        const Level& d = table.level[list.level[c]];
        if (STRATEGY == RUNS_SHARED) runs_flush<KIND>(d, acc + list.offset[c], 0, ix, iy, v, a.node_bitmap, a.node_prefix);
        else runs_flush_global<KIND>(d, grad, ix, iy, v);
    };
    for (int c0 = group * RUNS_GROUP; c0 < list.count; c0 += groups * RUNS_GROUP) {
        const int here = list.count - c0 < RUNS_GROUP ? list.count - c0 : RUNS_GROUP;
        int cx[RUNS_GROUP], cy[RUNS_GROUP];
        float v[RUNS_GROUP][8], scale[RUNS_GROUP];
        bool open = false;  // a run is open (the first coordinate has been seen)
#pragma unroll
        for (int g = 0; g < RUNS_GROUP; ++g) {
            cx[g] = cy[g] = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) v[g][j] = 0.0f;
            scale[g] = table.level[list.level[g < here ? c0 + g : c0]].scale;
        }
        for (long long i = first; i < last; ++i) {
            const float2 p = __ldg(coords + i);
            float pairs[2 * RUNS_GROUP];
            load_pairs4(upstream, i, a.width, c0, pairs);
#pragma unroll
            for (int g = 0; g < RUNS_GROUP; ++g) {
                if (g >= here) break;
                const Corner4 geo = geometry(p.x, p.y, scale[g]);
                if (open && (geo.ix != cx[g] || geo.iy != cy[g])) flush(c0 + g, cx[g], cy[g], v[g]);
                cx[g] = geo.ix;
                cy[g] = geo.iy;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    v[g][2 * k] = __fmaf_rn(geo.w[k], pairs[2 * g], v[g][2 * k]);
                    v[g][2 * k + 1] = __fmaf_rn(geo.w[k], pairs[2 * g + 1], v[g][2 * k + 1]);
                }
            }
            open = true;
        }
        const int lane = threadIdx.x & 31;
#pragma unroll
        for (int g = 0; g < RUNS_GROUP; ++g) {
            if (g >= here) break;
            const long long key = ((long long)cx[g] << 32) | uint32_t(cy[g]);
            if (combine_lanes(v[g], key, open ? 0 : -1 - lane, open)) flush(c0 + g, cx[g], cy[g], v[g]);
        }
    }
    if (STRATEGY == RUNS_SHARED) {
        __syncthreads();
        for (int c = 0; c < list.count; ++c) {
            const Level d = table.level[list.level[c]];
            const int per_table = d.points * d.F;
            const float* tab = acc + list.offset[c];
            for (int j = threadIdx.x; j < per_table; j += blockDim.x) {
                const float v = tab[j];
                if (v != 0.0f) red_add_f32(grad + d.offset + j, v);
            }
        }
    }
}

// Chooses the plain runs kernel's strategy from the batch: PROBE_PAIRS pairs of consecutive coordinates
// (i, i + 1), one at a hashed position inside each of PROBE_PAIRS equal stretches of the batch (evenly spaced
// positions would alias with a raster-ordered sampler's rows), give each listed level's rate of cell changes
// r, the rate at which a run ends.  RUNS_GLOBAL when the runs are long -- on average over the levels at most one change in
// PROBE_MEAN_RUN consecutive pairs -- and no level's expected flushes per table entry (n r / entries) exceed
// PROBE_ENTRY_FLUSHES, so that global reductions neither serialise on a coarse level's few entries nor
// outnumber what the shared-memory tables absorb; RUNS_SHARED otherwise.  Either strategy gives the same sums
// up to the order of the fp32 additions.  One block; writes *strategy.
constexpr int PROBE_THREADS = 512, PROBE_PAIRS = 4096, PROBE_MEAN_RUN = 8, PROBE_ENTRY_FLUSHES = 4096;
__global__ void __launch_bounds__(PROBE_THREADS) runs_probe_kernel(const EncodeArgs a,
                                                                   const __grid_constant__ LevelTable table,
                                                                   const __grid_constant__ CoarseList list,
                                                                   int* __restrict__ strategy) {
    __shared__ int changes[MAX_LEVELS];
    for (int c = threadIdx.x; c < MAX_LEVELS; c += blockDim.x) changes[c] = 0;
    __syncthreads();
    const long long pairs = a.n - 1 < PROBE_PAIRS ? a.n - 1 : PROBE_PAIRS;
    const long long stretch = pairs > 0 ? (a.n - 1) / pairs : 1;  // >= 1
    const float2* const coords = reinterpret_cast<const float2*>(a.coords);
    for (long long j = threadIdx.x; j < pairs; j += blockDim.x) {
        const uint32_t h = (uint32_t(j) * 0x9E3779B1u) >> 7;
        const long long i = j * stretch + (long long)(h % uint64_t(stretch));  // <= pairs * stretch - 1 < n - 1
        const float2 p = __ldg(coords + i), q = __ldg(coords + i + 1);
        for (int c = 0; c < list.count; ++c) {
            const float s = table.level[list.level[c]].scale;
            const Corner4 g0 = geometry(p.x, p.y, s), g1 = geometry(q.x, q.y, s);
            if (g0.ix != g1.ix || g0.iy != g1.iy) atomicAdd(&changes[c], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        bool global = pairs > 0;
        long long sum = 0;
        for (int c = 0; c < list.count; ++c) {
            sum += changes[c];
            const double flushes_per_entry = double(a.n) * changes[c] / double(pairs > 0 ? pairs : 1) /
                                             double(table.level[list.level[c]].points);
            if (flushes_per_entry > PROBE_ENTRY_FLUSHES) global = false;
        }
        if ((long long)PROBE_MEAN_RUN * sum > (long long)list.count * pairs) global = false;
        *strategy = global ? RUNS_GLOBAL : RUNS_SHARED;
    }
}

}  // namespace

constexpr int COARSE_SMEM_FLOATS = 27648;  // 108 KB of shared memory per block: two blocks per SM

void launch_encode_forward(const EncodeArgs& a, const LevelSource& src, const float* table32, const __half* table16,
                           __half* out, uint8_t* vis, cudaStream_t stream) {
    if (a.n <= 0 || a.levels <= 0) return;
    ODIE_REQUIRE(a.levels <= MAX_LEVELS, "at most 32 levels");
    const dim3 grid(blocks_for(a.n, 256), a.levels);
    bool rows = !src.descriptors && table16 && !vis && a.row_major && (a.width == 16 || a.width == 32) &&
                2 * a.levels <= a.width;
    for (int l = 0; rows && l < a.levels; ++l) rows = src.table.level[l].F == 2 && src.table.level[l].col == 2 * l;
    if (rows) {
        int kind = src.table.level[0].kind;
        for (int l = 1; l < a.levels; ++l)
            if (src.table.level[l].kind != kind) kind = -1;
        // mixed kinds: dense levels first, then hashed ones (split = the first hashed level), else -1
        int split = 0;
        while (split < a.levels && src.table.level[split].kind == HASH_DENSE) ++split;
        for (int l = split; l < a.levels; ++l)
            if (src.table.level[l].kind != HASH_HASHED) split = -1;
        const unsigned blocks = blocks_for(a.n, 256);
        if (a.width == 32) {
            if (kind == HASH_DENSE) encode_forward_rows_kernel<32, HASH_DENSE><<<blocks, 256, 0, stream>>>(a, src.table, table16, out, 0);
            else if (kind == HASH_HASHED) encode_forward_rows_kernel<32, HASH_HASHED><<<blocks, 256, 0, stream>>>(a, src.table, table16, out, 0);
            else encode_forward_rows_kernel<32, -1><<<blocks, 256, 0, stream>>>(a, src.table, table16, out, split);
        } else {
            if (kind == HASH_DENSE) encode_forward_rows_kernel<16, HASH_DENSE><<<blocks, 256, 0, stream>>>(a, src.table, table16, out, 0);
            else if (kind == HASH_HASHED) encode_forward_rows_kernel<16, HASH_HASHED><<<blocks, 256, 0, stream>>>(a, src.table, table16, out, 0);
            else encode_forward_rows_kernel<16, -1><<<blocks, 256, 0, stream>>>(a, src.table, table16, out, split);
        }
        note_launch();
        return;
    }
    if (src.descriptors) {
        if (table32) encode_forward_kernel<float, true><<<grid, 256, 0, stream>>>(a, src.descriptors, src.table, table32, out, vis);
        else encode_forward_kernel<__half, true><<<grid, 256, 0, stream>>>(a, src.descriptors, src.table, table16, out, vis);
    } else {
        if (table32) encode_forward_kernel<float, false><<<grid, 256, 0, stream>>>(a, nullptr, src.table, table32, out, vis);
        else encode_forward_kernel<__half, false><<<grid, 256, 0, stream>>>(a, nullptr, src.table, table16, out, vis);
    }
    note_launch();
}

// Mask of the visiting permutation for n coordinates (0: identity, for n above 2^30).
static uint32_t visit_mask(long long n) {
    if (n > (1LL << 30)) return 0u;
    uint32_t size = 1;
    while ((long long)size < n) size <<= 1;
    return size - 1;
}

template <int KIND, typename U>
static void set_runs_smem() {
    ODIE_CUDA(cudaFuncSetAttribute(encode_backward_runs_kernel<true, KIND, U>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   COARSE_SMEM_FLOATS * 4));
    ODIE_CUDA(cudaFuncSetAttribute(encode_backward_runs_kernel<false, KIND, U>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   COARSE_SMEM_FLOATS * 4));
    if constexpr (KIND != PLANE)
        ODIE_CUDA(cudaFuncSetAttribute(encode_backward_runs_plain_kernel<KIND, U, RUNS_SHARED>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, COARSE_SMEM_FLOATS * 4));
}

template <typename U>
struct RunsLaunch {
    const EncodeArgs& a;
    const LevelTable& table;
    const CoarseList& list;
    const U* upstream;
    float* grad;
    int blocks, smem;
    cudaStream_t stream;
};

// The plain runs scatter, with the probe of its strategy when the call has a strategy int and the gradient
// takes 8-byte vector reductions.  Returns the number of kernels launched.
template <int KIND, typename U>
static int launch_runs_plain(const RunsLaunch<U>& l) {
    const bool probe = l.a.strategy && l.a.n >= 2 && (reinterpret_cast<uintptr_t>(l.grad) & 7) == 0;
    if (probe) {
        runs_probe_kernel<<<1, PROBE_THREADS, 0, l.stream>>>(l.a, l.table, l.list, l.a.strategy);
        // no shared tables: four blocks per SM's worth of shorter chunks (two resident at 80 registers)
        const long long spread = l.a.n / 1024 > 1 ? l.a.n / 1024 : 1;
        const int blocks = int(spread < 4 * sm_count() ? spread : 4 * sm_count());
        encode_backward_runs_plain_kernel<KIND, U, RUNS_GLOBAL><<<blocks, RUNS_THREADS, 0, l.stream>>>(
            l.a, l.table, l.list, l.upstream, l.grad, l.a.strategy);
    }
    encode_backward_runs_plain_kernel<KIND, U, RUNS_SHARED><<<l.blocks, RUNS_THREADS, l.smem, l.stream>>>(
        l.a, l.table, l.list, l.upstream, l.grad, probe ? l.a.strategy : nullptr);
    return probe ? 3 : 1;
}

// Launches the runs scatter; returns the number of kernels launched.
template <int KIND, typename U>
static int launch_runs(const RunsLaunch<U>& l, bool vec, bool plain = false) {
    if constexpr (KIND != PLANE) {
        if (vec && plain) return launch_runs_plain<KIND>(l);
    }
    if (vec)
        encode_backward_runs_kernel<true, KIND, U><<<l.blocks, RUNS_THREADS, l.smem, l.stream>>>(l.a, l.table, l.list,
                                                                                               l.upstream, l.grad);
    else
        encode_backward_runs_kernel<false, KIND, U><<<l.blocks, RUNS_THREADS, l.smem, l.stream>>>(l.a, l.table, l.list,
                                                                                                l.upstream, l.grad);
    return 1;
}

template <typename U>
static void encode_backward(const EncodeArgs& a, const LevelSource& src, const U* upstream, float* grad,
                            cudaStream_t stream) {
    if (a.n <= 0 || a.levels <= 0) return;
    ODIE_REQUIRE(a.levels <= MAX_LEVELS, "at most 32 levels");
    const long long groups = (a.n + 31) / 32;  // the direct scatter scrambles 32-coordinate groups
    const uint32_t mask = visit_mask(groups);
    const long long threads = 32 * (mask ? (long long)mask + 1 : groups);
    if (src.descriptors) {
        encode_backward_kernel<true, U, false><<<blocks_for(threads, 256), 256, 0, stream>>>(
            a, src.descriptors, src.table, upstream, grad, 0u, mask, -1);
        note_launch();
        return;
    }
    // The smallest levels, coarsest first, while all their tables (of every
    // expert) fit in shared memory together and each is small against the
    // coordinates: the blocks' flushes of a level stay below half of the
    // 4 x F per-coordinate updates they absorb.
    CoarseList list{};
    unsigned skip = 0;
    const long long spread = a.n / 1024 > 1 ? a.n / 1024 : 1;
    const int blocks = int(spread < 2 * sm_count() ? spread : 2 * sm_count());
    for (int l = 0; l < a.levels && l < a.active; ++l) {
        const Level& d = src.table.level[l];
        const long long floats = (long long)d.points * d.F * (a.expert ? a.experts : 1);
        if (list.total + floats > COARSE_SMEM_FLOATS || (long long)blocks * floats > 2 * a.n * d.F) continue;
        list.level[list.count] = l;
        list.offset[list.count] = list.total;
        list.total += int(floats);
        ++list.count;
        skip |= 1u << l;
    }
    if (list.count) {
        static std::atomic<unsigned long long> configured{0};  // per value type and device
        int device = 0;
        ODIE_CUDA(cudaGetDevice(&device));
        ODIE_REQUIRE(device >= 0 && device < 64, "devices 0..63");  // one bit per device below
        if (!(configured.load() >> device & 1ull)) {
            ODIE_CUDA(cudaFuncSetAttribute(encode_backward_shared_kernel<U>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           COARSE_SMEM_FLOATS * 4));
            set_runs_smem<PLANE, U>();
            set_runs_smem<HASH_DENSE, U>();
            set_runs_smem<HASH_HASHED, U>();
            set_runs_smem<-1, U>();
            configured.fetch_or(1ull << device);
        }
        // runs kernel: every listed level has F = 2; the 16-byte value loads also need row-major values with
        // listed level c in columns (2c, 2c + 1) and 16-byte aligned rows
        bool pairs = true, vec = a.row_major && (a.width % 8) == 0 && (reinterpret_cast<uintptr_t>(upstream) & 15) == 0 &&
                                 2 * ((list.count + RUNS_GROUP - 1) / RUNS_GROUP * RUNS_GROUP) <= a.width;
        int kind = src.table.level[list.level[0]].kind;
        for (int c = 0; c < list.count; ++c) {
            const Level& d = src.table.level[list.level[c]];
            pairs = pairs && d.F == 2;
            vec = vec && d.col == 2 * c;
            if (d.kind != kind) kind = -1;
        }
        if (pairs) {
            // one table, no cell that visibility can hide: the runs kernel without per-coordinate checks
            bool plain = !a.expert;
            for (int c = 0; c < list.count; ++c) {
                const Level& d = src.table.level[list.level[c]];
                plain = plain && d.kind != PLANE && (d.cells < 0 || !a.bitmap);
            }
            const RunsLaunch<U> l{a, src.table, list, upstream, grad, blocks, list.total * 4, stream};
            int launched;
            if (kind == PLANE) launched = launch_runs<PLANE>(l, vec);
            else if (kind == HASH_DENSE) launched = launch_runs<HASH_DENSE>(l, vec, plain);
            else if (kind == HASH_HASHED) launched = launch_runs<HASH_HASHED>(l, vec, plain);
            else launched = launch_runs<-1>(l, vec, plain);
            note_launch(launched);
        } else {
            encode_backward_shared_kernel<U><<<blocks, 512, list.total * 4, stream>>>(a, src.table, list, upstream, grad);
            note_launch();
        }
    }
    const int active = a.active < a.levels ? a.active : a.levels;
    if (list.count == active) return;  // every level took the shared-memory path
    // a hash grid's dense levels come first, then its hashed ones: split = the first hashed level, else -1
    int split = 0;
    while (split < a.levels && src.table.level[split].kind == HASH_DENSE) ++split;
    for (int l = split; l < a.levels; ++l)
        if (src.table.level[l].kind != HASH_HASHED) split = -1;
    // the values as whole rows when every level is F = 2 at columns (2l, 2l + 1) of 16-byte aligned rows of 32
    bool rows = a.row_major && a.width == 32 && (reinterpret_cast<uintptr_t>(upstream) & 15) == 0;
    for (int l = 0; rows && l < a.levels; ++l) rows = src.table.level[l].F == 2 && src.table.level[l].col == 2 * l;
    if (rows)
        encode_backward_kernel<false, U, true><<<blocks_for(threads, 256), 256, 0, stream>>>(a, nullptr, src.table, upstream,
                                                                                           grad, skip, mask, split);
    else
        encode_backward_kernel<false, U, false><<<blocks_for(threads, 256), 256, 0, stream>>>(a, nullptr, src.table,
                                                                                            upstream, grad, skip, mask,
                                                                                            split);
    note_launch();
}

void launch_encode_backward(const EncodeArgs& a, const LevelSource& src, const __half* upstream, float* grad,
                            cudaStream_t stream) {
    encode_backward(a, src, upstream, grad, stream);
}
void launch_encode_backward(const EncodeArgs& a, const LevelSource& src, const float* upstream, float* grad,
                            cudaStream_t stream) {
    encode_backward(a, src, upstream, grad, stream);
}

}  // namespace odie
