// On-device packed-plane index (the reference's plane_closure / make_node_index
// / cell bitmap, odie/model.py:36-61,108-110, built on the CPU at every stage
// boundary).  For one level of resolution R, points = align8(R^2):
//   closure: node n is present iff some selected cell c and corner offset
//     k in {0, 1, R, R + 1} give (c + k) mod points = n;
//   node index: one uint64 presence word per 64 nodes (bit b of word w = node
//     64w + b) and the exclusive prefix of the words' popcounts (int32);
//   cell bitmap: bit (c mod 8) of byte c / 8 = cell c selected, cells padded to
//     points with zeros;
//   node count = number of present nodes; optionally the sorted node list.
// All integer work, bit-identical to the host construction.
#include "common.cuh"

namespace odie {

namespace {

constexpr int SCAN_BLOCK = 1024;  // words per block of the prefix scan

__device__ __forceinline__ bool selected(const uint8_t* __restrict__ support, long long cells, long long c) {
    return c >= 0 && c < cells && __ldg(support + c) != 0;
}

// One thread per node: closure presence (two 32-node ballots per word) and the
// node's own cell bit (cell bitmap bytes, four per 32-node ballot).
__global__ void closure_kernel(const uint8_t* __restrict__ support, int resolution, long long points, long long words,
                               uint32_t* __restrict__ node_words, uint8_t* __restrict__ cell_bitmap) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // blockDim is a multiple of 32
    const long long cells = (long long)resolution * resolution;
    bool present = false, own = false;
    if (n < points) {
        const long long offsets[4] = {0, 1, resolution, (long long)resolution + 1};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            long long c = n - offsets[k];
            if (c < 0) c += points;  // (c + k) mod points == n with c + k < 2 points
            present = present || selected(support, cells, c);
        }
        own = selected(support, cells, n);
    }
    const unsigned p = __ballot_sync(0xffffffffu, present);
    const unsigned o = __ballot_sync(0xffffffffu, own);
    const int lane = threadIdx.x & 31;
    const long long first = n - lane;  // first node of this warp's 32
    if (lane == 0 && first < words * 64) node_words[first / 32] = p;
    if ((lane & 7) == 0 && first + lane < points) cell_bitmap[(first + lane) / 8] = uint8_t(o >> lane);
}

// Exclusive prefix of the words' popcounts within blocks of SCAN_BLOCK words; block totals to sums.
__global__ void __launch_bounds__(SCAN_BLOCK) word_scan_kernel(const unsigned long long* __restrict__ words_in,
                                                               long long words, int* __restrict__ prefix,
                                                               int* __restrict__ sums) {
    __shared__ int warp_totals[SCAN_BLOCK / 32];
    const long long w = (long long)blockIdx.x * SCAN_BLOCK + threadIdx.x;
    const int count = w < words ? __popcll(words_in[w]) : 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inclusive = count;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int up = __shfl_up_sync(0xffffffffu, inclusive, d);
        if (lane >= d) inclusive += up;
    }
    if (lane == 31) warp_totals[warp] = inclusive;
    __syncthreads();
    if (warp == 0) {
        int t = warp_totals[lane];
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int up = __shfl_up_sync(0xffffffffu, t, d);
            if (lane >= d) t += up;
        }
        warp_totals[lane] = t;  // inclusive over warps
    }
    __syncthreads();
    const int before = warp ? warp_totals[warp - 1] : 0;
    if (w < words) prefix[w] = before + inclusive - count;
    if (threadIdx.x == 0) sums[blockIdx.x] = warp_totals[SCAN_BLOCK / 32 - 1];
}

// Exclusive scan of the block totals (one block, any count) and the node count.
__global__ void __launch_bounds__(SCAN_BLOCK) block_scan_kernel(int* __restrict__ sums, int blocks,
                                                                long long* __restrict__ node_count) {
    __shared__ int warp_totals[SCAN_BLOCK / 32];
    __shared__ long long carry;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < blocks; base += SCAN_BLOCK) {
        const int b = base + threadIdx.x;
        const int value = b < blocks ? sums[b] : 0;
        int inclusive = value;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int up = __shfl_up_sync(0xffffffffu, inclusive, d);
            if (lane >= d) inclusive += up;
        }
        if (lane == 31) warp_totals[warp] = inclusive;
        __syncthreads();
        if (warp == 0) {
            int t = warp_totals[lane];
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const int up = __shfl_up_sync(0xffffffffu, t, d);
                if (lane >= d) t += up;
            }
            warp_totals[lane] = t;
        }
        __syncthreads();
        const int before = warp ? warp_totals[warp - 1] : 0;
        if (b < blocks) sums[b] = int(carry) + before + inclusive - value;
        __syncthreads();
        if (threadIdx.x == 0) carry += warp_totals[SCAN_BLOCK / 32 - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0) *node_count = carry;
}

__global__ void add_offsets_kernel(int* __restrict__ prefix, long long words, const int* __restrict__ sums) {
    const long long w = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (w < words) prefix[w] += sums[w / SCAN_BLOCK];
}

// Sorted closure: node n's position is its packed row (prefix + rank in the word).
__global__ void closure_nodes_kernel(const unsigned long long* __restrict__ words_in, const int* __restrict__ prefix,
                                     long long points, long long* __restrict__ nodes) {
    const long long n = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= points) return;
    const unsigned long long word = words_in[n >> 6];
    const int bit = int(n & 63);
    if (!((word >> bit) & 1ull)) return;
    nodes[prefix[n >> 6] + __popcll(word & ((1ull << bit) - 1))] = n;
}

// On-demand allocation of routed experts (the allocation benchmark; no reference
// counterpart): cell (ix, iy) of a level of resolution res is visible iff the
// pixel nearest its centre -- column floor(ix (width - 1) / (res - 1) + 1/2),
// computed exactly in integers, row likewise -- lies in an allocated
// tile_px x tile_px tile.  One thread per bitmap byte (8 cells, LSB first).
__global__ void allocation_kernel(const uint8_t* __restrict__ tiles, int tiles_x, int tiles_y, int tile_px, int height,
                                  int width, int res, uint8_t* __restrict__ bitmap) {
    const long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long cells = (long long)res * res;
    if (b * 8 >= cells) return;
    const long long den = res > 1 ? res - 1 : 1;
    uint32_t bits = 0;
    for (int j = 0; j < 8; ++j) {
        const long long c = b * 8 + j;
        if (c >= cells) break;
        const long long ix = c % res, iy = c / res;
        const long long col = (2 * ix * (width - 1) + den) / (2 * den), row = (2 * iy * (height - 1) + den) / (2 * den);
        const long long tx = col / tile_px < tiles_x ? col / tile_px : tiles_x - 1;
        const long long ty = row / tile_px < tiles_y ? row / tile_px : tiles_y - 1;
        bits |= uint32_t(__ldg(tiles + ty * tiles_x + tx) != 0) << j;
    }
    bitmap[b] = uint8_t(bits);
}

}  // namespace

void launch_allocation_bitmap(const uint8_t* tiles, int tiles_x, int tiles_y, int tile_px, int height, int width,
                              int res, uint8_t* bitmap, cudaStream_t stream) {
    ODIE_REQUIRE(tiles_x >= 1 && tiles_y >= 1 && tile_px >= 1 && height >= 1 && width >= 1 && res >= 1,
                 "allocation sizes must be positive");
    ODIE_REQUIRE((long long)res * res <= (1LL << 34), "resolution too large");
    const long long bytes = ((long long)res * res + 7) / 8;
    allocation_kernel<<<blocks_for(bytes, 256), 256, 0, stream>>>(tiles, tiles_x, tiles_y, tile_px, height, width, res,
                                                                   bitmap);
    note_launch();
}

long long plane_index_scratch(long long points) {
    const long long words = (points + 63) / 64;
    return (words + SCAN_BLOCK - 1) / SCAN_BLOCK;
}

void launch_plane_index(const uint8_t* support, int resolution, unsigned long long* node_words, int* node_prefix,
                        uint8_t* cell_bitmap, long long* node_count, long long* nodes, int* scratch,
                        cudaStream_t stream) {
    ODIE_REQUIRE(resolution >= 1 && (long long)resolution * resolution <= 0x7fffffffLL - 7,
                 "resolution must keep align8(R^2) within int32");
    const long long cells = (long long)resolution * resolution;
    const long long points = (cells + 7) / 8 * 8;
    const long long words = (points + 63) / 64;
    const long long threads = words * 64;
    closure_kernel<<<blocks_for(threads, 256), 256, 0, stream>>>(support, resolution, points, words,
                                                                 reinterpret_cast<uint32_t*>(node_words), cell_bitmap);
    const long long blocks = plane_index_scratch(points);
    word_scan_kernel<<<unsigned(blocks), SCAN_BLOCK, 0, stream>>>(node_words, words, node_prefix, scratch);
    block_scan_kernel<<<1, SCAN_BLOCK, 0, stream>>>(scratch, int(blocks), node_count);
    add_offsets_kernel<<<blocks_for(words, 256), 256, 0, stream>>>(node_prefix, words, scratch);
    note_launch(4);
    if (nodes) {
        closure_nodes_kernel<<<blocks_for(points, 256), 256, 0, stream>>>(node_words, node_prefix, points, nodes);
        note_launch();
    }
}

}  // namespace odie
