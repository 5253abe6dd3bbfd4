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
// Each launch runs at most `chunk` iterations in one block and returns; every
// loop is bounded.  A launch after completion returns at once, so the host may
// queue several launches between status reads.  The tree's top levels stay in
// shared memory for a launch (with the score bits of their winners), the
// chosen cell's neighbourhood is read in one round, and each level is repaired
// by one warp per changed (parent, category) pair.
#include <atomic>

#include "common.cuh"

namespace odie {

namespace {

constexpr int FAN = 32;

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

// Tree levels as the greedy sees them: levels [0, split) live in the caller's global tree, levels
// [split, levels) in shared memory for the whole launch (ids, and the raw score bits of each category-1..4
// winner so that comparing them needs no score lookup); they are loaded at the launch's start and written
// back to the global tree when it ends.  offset: a level's first global entry; id_at / key_at: its first
// shared-memory id / key.
struct GreedyLevels {
    int levels, split;
    int offset[32], size[32], id_at[32], key_at[32];
};

constexpr int GREEDY_WARPS = 32;
constexpr int GREEDY_THREADS = GREEDY_WARPS * FAN;

__device__ __forceinline__ unsigned long long raw_bits(const double* scores, int id) {
    return id >= 0 ? (unsigned long long)__double_as_longlong(scores[id]) : 0ull;
}

// Warp-wide winner of 32 candidates (id -1 = empty) carrying each candidate's raw score bits.
__device__ __forceinline__ void warp_winner_raw(int& id, unsigned long long& raw, int category) {
    unsigned long long key = raw & 0x7fffffffffffffffull;
#pragma unroll
    for (int step = 16; step; step >>= 1) {
        const int other = __shfl_xor_sync(0xffffffffu, id, step);
        const unsigned long long oraw = __shfl_xor_sync(0xffffffffu, raw, step);
        const unsigned long long okey = oraw & 0x7fffffffffffffffull;
        if (beats(other, okey, id, key, category)) { id = other; key = okey; raw = oraw; }
    }
}

// Unique tasks (lane j: a task or -1) written to out[0 .. count) in lane order of first occurrence; returns
// the count.  Warp-collective.
__device__ __forceinline__ int compact_tasks(int task, int* out) {
    const int lane = threadIdx.x % FAN;
    const unsigned same = __match_any_sync(0xffffffffu, task);
    const unsigned kept = __ballot_sync(0xffffffffu, task >= 0 && (__ffs(same) - 1) == lane);
    if ((kept >> lane) & 1u) out[__popc(kept & ((1u << lane) - 1))] = task;
    __syncwarp();
    return __popc(kept);
}

// One (parent, category) winner of tree level `level` recomputed by a warp from its 32 children (and, when
// out_id is given, handed back through it by lane 0).
__device__ __forceinline__ void repair(const GreedyLevels& L, int level, int task, const double* __restrict__ scores,
                                       int n, const int* missing, const uint8_t* chosen, int* tree, int* s_id,
                                       unsigned long long* s_key, int* out_id = nullptr,
                                       unsigned long long* out_raw = nullptr) {
    const int lane = threadIdx.x % FAN;
    const int parent = task / 5, category = task % 5;
    const int child = parent * FAN + lane;
    int id = -1;
    unsigned long long raw = 0;
    if (level == 0) {  // the three reads of a leaf issued together
        if (child < n) {
            const bool free_leaf = chosen[child] == 0;
            const int m = missing[child];
            const unsigned long long bits = category ? raw_bits(scores, child) : 0ull;
            if (free_leaf && m == category) {
                id = child;
                raw = bits;
            }
        }
    } else if (child < L.size[level - 1]) {
        if (level - 1 >= L.split) {
            id = s_id[L.id_at[level - 1] + child * 5 + category];
            if (category && id >= 0) raw = s_key[L.key_at[level - 1] + child * 4 + category - 1];
        } else {
            id = tree[L.offset[level - 1] + child * 5 + category];
            if (category && id >= 0) raw = raw_bits(scores, id);
        }
    }
    warp_winner_raw(id, raw, category);
    if (out_id && lane == 0) {
        *out_id = id;
        *out_raw = raw;
    }
    if (lane == 0) {
        if (level >= L.split) {
            s_id[L.id_at[level] + parent * 5 + category] = id;
            if (category) s_key[L.key_at[level] + parent * 4 + category - 1] = raw;
        } else {
            tree[L.offset[level] + parent * 5 + category] = id;
        }
    }
}

// Exact greedy, one block: per iteration warp 0 takes the root's winner and updates the chosen cell's
// neighbourhood (one round of parallel global reads), then every level of the tree is repaired for the
// (parent, category) pairs whose winner may change, one warp per pair, one barrier per level.
__global__ void __launch_bounds__(GREEDY_THREADS) greedy_kernel(const double* __restrict__ scores, int n, int points,
                                                                int resolution, int cap, bool normalized, int* missing,
                                                                uint8_t* chosen, uint8_t* nodes, int* tree,
                                                                const __grid_constant__ GreedyLevels L, int chunk,
                                                                long long* stats, int* trace) {
    extern __shared__ __align__(16) unsigned char dyn[];
    unsigned long long* s_key = reinterpret_cast<unsigned long long*>(dyn);
    int* s_id = reinterpret_cast<int*>(dyn + 8 * size_t(L.key_at[L.levels]));
    __shared__ int s_stop, s_count[32], s_tasks[32][32];  // per level: the (parent, category) pairs to repair
    __shared__ int s_new_id[32];                             // level 0's new winners, by task
    __shared__ unsigned long long s_new_raw[32];
    const int tid = threadIdx.x, lane = tid % FAN, warp = tid / FAN;
    if (tid == 0) s_stop = stats[2] != 0 || stats[3] != 0;
    // the shared-memory levels from the global tree
    for (int l = L.split; l < L.levels; ++l)
        for (int e = tid; e < L.size[l] * 5; e += GREEDY_THREADS) {
            const int id = tree[L.offset[l] + e];
            s_id[L.id_at[l] + e] = id;
            const int c = e % 5;
            if (c) s_key[L.key_at[l] + (e / 5) * 4 + c - 1] = raw_bits(scores, id);
        }
    __syncthreads();
    if (s_stop) return;
    long long used = 0, iterations = 0;  // thread 0's copies of stats[0], stats[1]
    if (tid == 0) { used = stats[0]; iterations = stats[1]; }
    const int R = resolution;
    // corner d of a cell is cell + (d & 1) + (d >> 1) R; lane j < 9 of warp 0 looks at the neighbour
    // (j mod 3 - 1, j / 3 - 1), lane 4 being the cell itself
    const int my_diff = (lane / 3 - 1) * R + (lane % 3 - 1);
    bool stop = false;
    for (int iteration = 0; iteration < chunk && !stop; ++iteration) {
        if (warp == 0) {
            // ---- the root's candidates: one per category, with their scores
            const int top = L.levels - 1;
            int rid = -1;
            double rscore = 0.0;
            if (lane < 5) {
                if (top >= L.split) {
                    rid = s_id[L.id_at[top] + lane];
                    if (lane > 0 && rid >= 0) rscore = __longlong_as_double((long long)s_key[L.key_at[top] + lane - 1]);
                } else {
                    rid = tree[L.offset[top] + lane];
                    if (lane > 0 && rid >= 0) rscore = scores[rid];
                }
            }
            int cell = __shfl_sync(0xffffffffu, rid, 0), cost = 0;
            if (cell < 0) {
                const long long remaining = (long long)cap - __shfl_sync(0xffffffffu, used, 0);
                double best = 0.0;
                for (int k = 1; k <= 4 && k <= remaining; ++k) {
                    const int candidate = __shfl_sync(0xffffffffu, rid, k);
                    const double cs = __shfl_sync(0xffffffffu, rscore, k);
                    if (candidate < 0) continue;
                    bool take = cell < 0;
                    if (!take) {
                        const double left = normalized ? __dmul_rn(cs, double(cost)) : cs;
                        const double right = normalized ? __dmul_rn(best, double(k)) : best;
                        take = left > right || (left == right && candidate < cell);
                    }
                    if (take) { cell = candidate; cost = k; best = cs; }
                }
            }
            int ntasks = 0;
            bool halt = cell < 0;
            if (!halt) {
                // ---- the cell's 9-cell neighbourhood and its 4 corner nodes, read together
                int nb = -1, was = 0, node = -1;
                bool present = true, taken = true;
                if (lane < 9) {  // cell + diff lies in [-(R + 1), points + R + 1): one correction wraps it
                    nb = cell + my_diff;
                    nb = nb < 0 ? nb + points : (nb >= points ? nb - points : nb);
                    if (nb < n) {
                        taken = chosen[nb] != 0;
                        was = missing[nb];
                    }
                } else if (lane < 13) {
                    node = cell + ((lane - 9) & 1) + ((lane - 9) >> 1) * R;
                    node = node >= points ? node - points : node;
                    present = nodes[node] != 0;
                }
                const unsigned added = (__ballot_sync(0xffffffffu, lane >= 9 && lane < 13 && !present) >> 9) & 0xfu;
                const int nadded = __popc(added);
                int corner[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) corner[k] = __shfl_sync(0xffffffffu, node, 9 + k);
                if (lane >= 9 && lane < 13 && !present) nodes[node] = 1;
                if (lane == 0) {
                    chosen[cell] = 1;
                    if (trace) trace[iterations] = cell;
                    used += nadded;
                    iterations += 1;
                    if (nadded != cost) { stats[3] = 1; }
                }
                halt = nadded != cost;
                // neighbours that lose missing corners (each distinct cell once, the chosen cell excluded)
                const unsigned same = __match_any_sync(0xffffffffu, lane < 9 ? nb : -1 - lane);
                const bool first = (__ffs(same) - 1) == lane;
                int old_task = -1, new_task = -1;
                if (lane < 9 && first && nb != cell && nb < n && !taken) {
                    int decrement = 0;
#pragma unroll
                    for (int d = 0; d < 4; ++d) {
                        int corner_of_nb = nb + (d & 1) + (d >> 1) * R;
                        corner_of_nb = corner_of_nb >= points ? corner_of_nb - points : corner_of_nb;
#pragma unroll
                        for (int k = 0; k < 4; ++k) decrement += ((added >> k) & 1u) && corner[k] == corner_of_nb;
                    }
                    if (decrement) {
                        missing[nb] = was - decrement;
                        old_task = (nb / FAN) * 5 + was;
                        new_task = (nb / FAN) * 5 + (was - decrement);
                    }
                }
                // the level-0 tasks: lanes 0-8 a neighbour's old category (lane 4: the chosen cell's (parent,
                // cost)), lanes 9-17 the same neighbours' new categories; then each level's from the one below
                int task = lane < 9 ? (lane == 4 ? (cell / FAN) * 5 + cost : old_task) : -1;
                const int w = __shfl_sync(0xffffffffu, new_task, (lane >= 9 && lane < 18) ? lane - 9 : 0);
                if (lane >= 9 && lane < 18) task = w;
                for (int level = 0; level < L.levels; ++level) {
                    ntasks = compact_tasks(task, s_tasks[level]);
                    if (lane == 0) s_count[level] = ntasks;
                    task = lane < ntasks ? s_tasks[level][lane] : -1;
                    task = task >= 0 ? (task / 5 / FAN) * 5 + task % 5 : -1;  // the parent's pair one level up
                }
            }
            if (lane == 0) {
                s_stop = halt;
                if (cell < 0) stats[2] = 1;
            }
        }
        __syncthreads();
        if (s_stop) {
            stop = true;
            break;
        }
        // ---- level 0 on warps 0-15; meanwhile warps 16-31 read the level-1 tasks' 32 children (level-0 entries
        //      and their scores) from global memory, so that after one barrier they only patch in level 0's new
        //      winners and pick; then every further level with one warp per task and one barrier per level
        const int c0 = s_count[0], c1 = L.levels > 1 ? s_count[1] : 0;
        int pre_id[2] = {-1, -1};
        unsigned long long pre_raw[2] = {0ull, 0ull};
        if (warp < GREEDY_WARPS / 2) {
            for (int t = warp; t < c0; t += GREEDY_WARPS / 2)
                repair(L, 0, s_tasks[0][t], scores, n, missing, chosen, tree, s_id, s_key, s_new_id + t, s_new_raw + t);
        } else {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int t = warp - GREEDY_WARPS / 2 + j * (GREEDY_WARPS / 2);
                if (t >= c1) break;
                const int task = s_tasks[1][t], category = task % 5, child = (task / 5) * FAN + lane;
                if (child < L.size[0]) {
                    pre_id[j] = tree[L.offset[0] + child * 5 + category];
                    if (category && pre_id[j] >= 0) pre_raw[j] = raw_bits(scores, pre_id[j]);
                }
            }
        }
        __syncthreads();
        if (warp >= GREEDY_WARPS / 2) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int t = warp - GREEDY_WARPS / 2 + j * (GREEDY_WARPS / 2);
                if (t >= c1) break;
                const int task = s_tasks[1][t], parent = task / 5, category = task % 5, key = (parent * FAN + lane) * 5 + category;
                int id = pre_id[j];
                unsigned long long raw = pre_raw[j];
                for (int k = 0; k < c0; ++k)
                    if (s_tasks[0][k] == key) {
                        id = s_new_id[k];
                        raw = s_new_raw[k];
                    }
                warp_winner_raw(id, raw, category);
                if (lane == 0) {
                    if (1 >= L.split) {
                        s_id[L.id_at[1] + parent * 5 + category] = id;
                        if (category) s_key[L.key_at[1] + parent * 4 + category - 1] = raw;
                    } else {
                        tree[L.offset[1] + parent * 5 + category] = id;
                    }
                }
            }
        }
        __syncthreads();
        for (int level = 2; level < L.levels; ++level) {
            for (int t = warp; t < s_count[level]; t += GREEDY_WARPS)
                repair(L, level, s_tasks[level][t], scores, n, missing, chosen, tree, s_id, s_key);
            __syncthreads();
        }
    }
    // ---- write the shared-memory levels and the counters back
    __syncthreads();
    for (int l = L.split; l < L.levels; ++l)
        for (int e = tid; e < L.size[l] * 5; e += GREEDY_THREADS) tree[L.offset[l] + e] = s_id[L.id_at[l] + e];
    if (tid == 0) {
        stats[0] = used;
        stats[1] = iterations;
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
    (void)offsets;
    (void)sizes;
    // the tree's shape follows from n (32-ary levels up to one parent); the caller's level count must agree
    GreedyLevels L{};
    int count = 0, children = n, total = 0;
    while (count < 32) {
        const int parents = (children + FAN - 1) / FAN;
        L.size[count] = parents;
        L.offset[count] = total;
        total += parents * 5;
        ++count;
        if (parents == 1) break;
        children = parents;
    }
    if (n < 1 || count != levels || levels > 31 || chunk < 0) return int(cudaErrorInvalidValue);
    L.levels = levels;
    // the top levels that fit in shared memory stay there for the launch (level 0 always stays global)
    constexpr long long BUDGET = 220 * 1024;
    int split = levels;
    long long bytes = 0;
    while (split > 1) {
        const long long more = (long long)L.size[split - 1] * (5 * 4 + 4 * 8);
        if (bytes + more > BUDGET) break;
        bytes += more;
        --split;
    }
    L.split = split;
    int ids = 0, keys = 0;
    for (int l = 0; l <= levels; ++l) {
        L.id_at[l] = ids;
        L.key_at[l] = keys;
        if (l < levels && l >= split) {
            ids += L.size[l] * 5;
            keys += L.size[l] * 4;
        }
    }
    const size_t smem = size_t(keys) * 8 + size_t(ids) * 4;
    static std::atomic<unsigned long long> configured{0};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) return int(status);
    if (!(configured.load() >> device & 1ull)) {
        status = cudaFuncSetAttribute(greedy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(BUDGET));
        if (status != cudaSuccess) return int(status);
        configured.fetch_or(1ull << device);
    }
    greedy_kernel<<<1, GREEDY_THREADS, smem, stream>>>(scores, n, points, resolution, cap, normalized, missing, chosen,
                                                      nodes, tree, L, chunk, stats, trace);
    note_launch();
    return int(cudaGetLastError());
}

}  // namespace odie
