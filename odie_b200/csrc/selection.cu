// Exact greedy support selection (B2 residual/cost and E residual), bit-identical
// to the reference's CPU rule odie/selection.py:129-207:
//   - free cells (no missing closure node) first, in ascending cell id;
//   - otherwise the cell maximising score/cost over the costs 1..min(4, cap-used),
//     compared by cross-multiplication (fp64, round-to-nearest), ties to the
//     lower id; stop when nothing fits.
// The caller-allocated buffers follow the reference's C-ABI
// (odie/native/selection_cuda.cu:208-230): missing int32[n], chosen u8[n],
// nodes u8[points], a 32-ary tournament tree int32 with 5 cost categories per
// parent, level sizes/offsets, stats int64[4] = {used, iterations, done,
// invariant error}.
//
// Each launch runs at most `chunk` iterations in one block of 1024 threads and
// returns; every loop is bounded.  A launch after completion returns at once, so
// the host may queue several launches between status reads.
#include "common.cuh"

namespace odie {

namespace {

constexpr int FAN = 32;
constexpr int SEL_THREADS = 1024;
constexpr int MAX_AFFECTED = 17;  // the chosen cell + up to 16 incident cells
constexpr int MAX_TASKS = 2 * MAX_AFFECTED;

// Ordering key of a leaf inside category c: category 0 orders by ascending id
// only; the others by score (sign bit cleared, so -0 == +0 as in Python, and
// non-negative doubles order as their bit patterns), then ascending id.
__device__ __forceinline__ unsigned long long score_bits(const double* scores, int id) {
    return (unsigned long long)__double_as_longlong(scores[id]) & 0x7fffffffffffffffull;
}
__device__ __forceinline__ bool beats(int a, unsigned long long ka, int b, unsigned long long kb, int category) {
    if (a < 0) return false;
    if (b < 0) return true;
    if (category == 0) return a < b;
    return ka > kb || (ka == kb && a < b);
}

// Warp-wide winner of 32 candidates (id -1 = empty).
__device__ __forceinline__ int warp_winner(int id, const double* scores, int category) {
    unsigned long long key = (id >= 0 && category > 0) ? score_bits(scores, id) : 0ull;
#pragma unroll
    for (int step = 16; step; step >>= 1) {
        const int other = __shfl_xor_sync(0xffffffffu, id, step);
        const unsigned long long okey = __shfl_xor_sync(0xffffffffu, key, step);
        if (beats(other, okey, id, key, category)) { id = other; key = okey; }
    }
    return id;
}

__device__ __forceinline__ int leaf_candidate(int child, int n, const uint8_t* chosen, const int* missing, int category) {
    return (child < n && !chosen[child] && missing[child] == category) ? child : -1;
}

__global__ void init_state_kernel(int n, int points, int* missing, uint8_t* chosen, uint8_t* nodes, long long* stats) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) { missing[i] = 4; chosen[i] = 0; }
    if (i < points) nodes[i] = 0;
    if (i < 4) stats[i] = 0;
}

// One warp per (parent, category) task of one tree level.
__global__ void build_level_kernel(const double* scores, int n, const int* missing, const uint8_t* chosen, int* tree,
                                   int offset, int previous_offset, int children, int parents, bool leaves) {
    const int task = (blockIdx.x * blockDim.x + threadIdx.x) / FAN;
    const int lane = threadIdx.x % FAN;
    if (task >= parents * 5) return;  // whole warp takes the same branch
    const int parent = task / 5, category = task % 5;
    const int child = parent * FAN + lane;
    int id = -1;
    if (child < children) id = leaves ? leaf_candidate(child, n, chosen, missing, category)
                                      : tree[previous_offset + child * 5 + category];
    id = warp_winner(id, scores, category);
    if (lane == 0) tree[offset + parent * 5 + category] = id;
}

__global__ void __launch_bounds__(SEL_THREADS) greedy_kernel(const double* __restrict__ scores, int n, int points,
                                                             int resolution, int cap, bool normalized, int* missing,
                                                             uint8_t* chosen, uint8_t* nodes, int* tree,
                                                             const int* offsets, const int* sizes, int levels,
                                                             int chunk, long long* stats, int* trace) {
    __shared__ int s_cell, s_cost, s_stop, s_nadded, s_naffected, s_ntasks;
    __shared__ int s_added[4], s_affected[MAX_AFFECTED], s_old[MAX_AFFECTED];
    __shared__ int s_tasks[MAX_TASKS];
    __shared__ int s_offsets[32], s_sizes[32];
    const int tid = threadIdx.x, lane = tid % FAN, warp = tid / FAN, warps = SEL_THREADS / FAN;
    if (tid < levels && tid < 32) { s_offsets[tid] = offsets[tid]; s_sizes[tid] = sizes[tid]; }
    if (tid == 0) s_stop = (stats[2] != 0 || stats[3] != 0 || levels > 32);
    __syncthreads();
    if (s_stop) return;
    const int deltas[4] = {0, 1, resolution, resolution + 1};
    for (int iteration = 0; iteration < chunk; ++iteration) {
        if (tid == 0) {
            const int root = s_offsets[levels - 1];
            int cell = tree[root], cost = 0;
            if (cell < 0) {
                const long long remaining = (long long)cap - stats[0];
                for (int k = 1; k <= 4 && k <= remaining; ++k) {
                    const int candidate = tree[root + k];
                    if (candidate < 0) continue;
                    bool take = cell < 0;
                    if (!take) {
                        const double left = normalized ? __dmul_rn(scores[candidate], double(cost)) : scores[candidate];
                        const double right = normalized ? __dmul_rn(scores[cell], double(k)) : scores[cell];
                        take = left > right || (left == right && candidate < cell);
                    }
                    if (take) { cell = candidate; cost = k; }
                }
            }
            s_stop = cell < 0;
            if (s_stop) {
                stats[2] = 1;
            } else {
                chosen[cell] = 1;
                int nadded = 0;
                for (int d = 0; d < 4; ++d) {
                    const int node = (cell + deltas[d]) % points;
                    if (!nodes[node]) { nodes[node] = 1; s_added[nadded++] = node; }
                }
                if (nadded != cost) { stats[3] = 1; s_stop = 1; }
                if (trace) trace[stats[1]] = cell;
                stats[0] += nadded;
                stats[1] += 1;
                s_nadded = nadded;
                s_cell = cell;
                s_cost = cost;
                int naffected = 1;
                s_affected[0] = cell;
                for (int a = 0; a < nadded; ++a)
                    for (int d = 0; d < 4; ++d) {
                        const int id = (s_added[a] - deltas[d] + points) % points;
                        if (id >= n || chosen[id]) continue;
                        bool seen = false;
                        for (int j = 0; j < naffected; ++j) seen |= s_affected[j] == id;
                        if (!seen && naffected < MAX_AFFECTED) s_affected[naffected++] = id;
                    }
                s_naffected = naffected;
            }
        }
        __syncthreads();
        if (s_stop) return;
        // every affected incident cell has exactly one writer
        if (tid < s_naffected) {
            const int id = s_affected[tid];
            const int before = missing[id];
            s_old[tid] = tid == 0 ? s_cost : before;
            if (tid > 0) {
                int decrement = 0;
                for (int a = 0; a < s_nadded; ++a)
                    for (int d = 0; d < 4; ++d) decrement += ((id + deltas[d]) % points) == s_added[a];
                missing[id] = before - decrement;
            }
        }
        __syncthreads();
        // level-0 tasks: (parent, category) pairs whose winner may change
        if (tid == 0) {
            int ntasks = 0;
            for (int j = 0; j < s_naffected; ++j) {
                const int id = s_affected[j];
                const int cats[2] = {s_old[j], j == 0 ? -1 : missing[id]};
                for (int q = 0; q < 2; ++q) {
                    if (cats[q] < 0) continue;
                    const int task = (id / FAN) * 5 + cats[q];
                    bool seen = false;
                    for (int k = 0; k < ntasks; ++k) seen |= s_tasks[k] == task;
                    if (!seen && ntasks < MAX_TASKS) s_tasks[ntasks++] = task;
                }
            }
            s_ntasks = ntasks;
        }
        __syncthreads();
        for (int level = 0; level < levels; ++level) {
            for (int task = warp; task < s_ntasks; task += warps) {
                const int parent = s_tasks[task] / 5, category = s_tasks[task] % 5;
                const int child = parent * FAN + lane;
                int id;
                if (level == 0) id = leaf_candidate(child, n, chosen, missing, category);
                else id = child < s_sizes[level - 1] ? tree[s_offsets[level - 1] + child * 5 + category] : -1;
                id = warp_winner(id, scores, category);
                if (lane == 0) tree[s_offsets[level] + parent * 5 + category] = id;
            }
            __syncthreads();
            if (level + 1 < levels) {
                if (tid == 0) {
                    int count = 0;
                    for (int j = 0; j < s_ntasks; ++j) {
                        const int next = (s_tasks[j] / 5 / FAN) * 5 + s_tasks[j] % 5;
                        bool seen = false;
                        for (int k = 0; k < count; ++k) seen |= s_tasks[k] == next;
                        if (!seen) s_tasks[count++] = next;
                    }
                    s_ntasks = count;
                }
                __syncthreads();
            }
        }
    }
}

}  // namespace

int launch_selection_init(const double* scores, int n, int points, int* missing, uint8_t* chosen, uint8_t* nodes,
                          int* tree, long long* stats, const int* host_offsets, const int* host_sizes, int levels,
                          cudaStream_t stream) {
    const int count = n > points ? n : points;
    init_state_kernel<<<blocks_for(count > 4 ? count : 4, 256), 256, 0, stream>>>(n, points, missing, chosen, nodes, stats);
    for (int l = 0; l < levels; ++l) {
        const int children = l == 0 ? n : host_sizes[l - 1];
        const int tasks = host_sizes[l] * 5;
        build_level_kernel<<<blocks_for((long long)tasks * FAN, 256), 256, 0, stream>>>(
            scores, n, missing, chosen, tree, host_offsets[l], l ? host_offsets[l - 1] : 0, children, host_sizes[l], l == 0);
    }
    note_launch(1 + levels);
    return int(cudaGetLastError());
}

int launch_selection_chunk(const double* scores, int n, int points, int resolution, int cap, bool normalized, int* missing,
                           uint8_t* chosen, uint8_t* nodes, int* tree, const int* offsets, const int* sizes, int levels,
                           int chunk, long long* stats, int* trace, cudaStream_t stream) {
    greedy_kernel<<<1, SEL_THREADS, 0, stream>>>(scores, n, points, resolution, cap, normalized, missing, chosen, nodes, tree,
                                                 offsets, sizes, levels, chunk, stats, trace);
    note_launch();
    return int(cudaGetLastError());
}

}  // namespace odie
