// Live residual scoring for on-demand allocation.
//
// score_chunk: per-cell residual of the reference's accumulate
// (odie/residual_cuda.cu:11-43): one thread owns one cell of the new level's
// R x R grid and adds, in raster order, the per-pixel mean-RGB squared error of
// the pixels of the chunk [begin, end) that fall in the cell: fp32 difference
// and square, fp64 sum of the three squares, / 3 in fp64.  One writer per cell
// and a fixed order make the totals bit-identical to the CPU reference
// (odie/selection.py:58-73).
//
// Tile scores (the allocation benchmark, no reference counterpart): per tile of
// tile x tile pixels, fp64 row sums in raster order, then the fp64 sum of the
// row sums in row order; then an exact top-k by (score desc, tile id asc).
#include <mutex>

#include "common.cuh"

namespace odie {

namespace {

__device__ __forceinline__ double pixel_residual(const float* __restrict__ pred, const void* target, long long p, bool rgb8) {
    float t[3];
#pragma unroll
    for (int c = 0; c < 3; ++c)
        t[c] = rgb8 ? __fdiv_rn(float(static_cast<const uint8_t*>(target)[p + c]), 255.0f)
                    : static_cast<const float*>(target)[p + c];
    const float d0 = __fsub_rn(pred[p], t[0]), d1 = __fsub_rn(pred[p + 1], t[1]), d2 = __fsub_rn(pred[p + 2], t[2]);
    double rgb = __dadd_rn(double(__fmul_rn(d0, d0)), double(__fmul_rn(d1, d1)));
    rgb = __dadd_rn(rgb, double(__fmul_rn(d2, d2)));
    return __ddiv_rn(rgb, 3.0);
}

__global__ void score_cells_kernel(const float* __restrict__ prediction, const void* __restrict__ target, long long begin,
                                   long long end, int width, int resolution, int first_y, int active_cells,
                                   const int* __restrict__ xb, const int* __restrict__ yb, double* __restrict__ totals,
                                   bool rgb8) {
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= active_cells) return;
    const int cx = t % resolution, cy = first_y + t / resolution;
    const long long cell = (long long)cy * resolution + cx;
    const int y0 = max(yb[cy], int(begin / width));
    const int y1 = min(yb[cy + 1], int((end - 1) / width) + 1);
    double sum = totals[cell];
    for (int y = y0; y < y1; ++y) {
        const long long row = (long long)y * width;
        const long long x0 = max((long long)xb[cx], begin - row);
        const long long x1 = min((long long)xb[cx + 1], end - row);
        for (long long x = x0; x < x1; ++x) sum = __dadd_rn(sum, pixel_residual(prediction, target, (row + x - begin) * 3, rgb8));
    }
    totals[cell] = sum;
}

// One block per tile, one thread per tile row (looping when tile > blockDim).
__global__ void tile_rows_kernel(const float* __restrict__ prediction, const uint8_t* __restrict__ target, int height,
                                 int width, int tile, double* __restrict__ row_sums) {
    const int tiles_x = int(((long long)width + tile - 1) / tile);  // widened: width + tile may pass INT_MAX
    const int tx = blockIdx.x % tiles_x, ty = blockIdx.x / tiles_x;
    const int x0 = tx * tile, x1 = min(x0 + tile, width);
    for (int r = threadIdx.x; r < tile; r += blockDim.x) {
        const int y = ty * tile + r;
        double sum = 0.0;
        if (y < height)
            for (int x = x0; x < x1; ++x) sum = __dadd_rn(sum, pixel_residual(prediction, target, ((long long)y * width + x) * 3, true));
        row_sums[(long long)blockIdx.x * tile + r] = sum;
    }
}

__global__ void tile_sum_kernel(const double* __restrict__ row_sums, int tiles, int tile, double* __restrict__ scores) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= tiles) return;
    double sum = 0.0;
    for (int r = 0; r < tile; ++r) sum = __dadd_rn(sum, row_sums[(long long)i * tile + r]);
    scores[i] = sum;
}

// rank_i = #{j : s_j > s_i or (s_j == s_i and j < i)}; chosen[rank] = i for rank < k.
__global__ void topk_rank_kernel(const double* __restrict__ scores, int count, int k, long long* __restrict__ chosen,
                                 uint8_t* __restrict__ selected) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const double si = scores[i];
    int rank = 0;
    for (int j = 0; j < count; ++j) {
        const double sj = scores[j];
        rank += (sj > si) || (sj == si && j < i);
    }
    if (selected) selected[i] = rank < k;
    if (rank < k && chosen) chosen[rank] = i;
}

}  // namespace

void launch_score_chunk(const float* prediction, const void* target, long long begin, long long end, int width,
                        int resolution, int first_y, int active_cells, const int* xb, const int* yb, double* totals,
                        bool rgb8, cudaStream_t stream) {
    if (active_cells <= 0) return;
    score_cells_kernel<<<blocks_for(active_cells, 256), 256, 0, stream>>>(prediction, target, begin, end, width, resolution,
                                                                          first_y, active_cells, xb, yb, totals, rgb8);
    note_launch();
}

void launch_tile_scores(const float* prediction, const uint8_t* target, int height, int width, int tile, double* row_sums,
                        double* scores, cudaStream_t stream) {
    const long long tiles = (((long long)width + tile - 1) / tile) * (((long long)height + tile - 1) / tile);
    tile_rows_kernel<<<unsigned(tiles), 256, 0, stream>>>(prediction, target, height, width, tile, row_sums);
    tile_sum_kernel<<<blocks_for(tiles, 256), 256, 0, stream>>>(row_sums, tiles, tile, scores);
    note_launch(2);
}

void launch_topk(const double* scores, int count, int k, long long* chosen, uint8_t* selected, cudaStream_t stream) {
    if (count <= 0) return;
    topk_rank_kernel<<<blocks_for(count, 256), 256, 0, stream>>>(scores, count, k, chosen, selected);
    note_launch();
}

// ---------------------------------------------------------------- allocation-free tile top-k
// Row-sum scratch of odie_tile_topk_noalloc: a fixed device array that every GPU
// loading this library holds until the process exits.  Every call on a device
// shares it, so calls that overlap on the GPU race; each call writes every entry
// it later reads (tiles x tile row sums), so nothing needs clearing.
constexpr long long NOALLOC_TILE_ROWS = 1LL << 18;  // 262 144 fp64 row sums = 2 MiB
static __device__ __align__(256) double g_noalloc_row_sums[NOALLOC_TILE_ROWS];

long long noalloc_tile_rows_max() { return NOALLOC_TILE_ROWS; }

// Device address of the scratch for the current device, resolved once per device
// (host code must not pass the symbol itself: it is a host-side stand-in).  The
// cached address belongs to the device's current context: it does not survive a
// cudaDeviceReset of that device, after which this library must not be called on it.
double* noalloc_row_sums(std::string& error) {
    static std::mutex lock;
    static double* address[64] = {nullptr};
    int device = 0;
    cudaError_t status = cudaGetDevice(&device);
    if (status != cudaSuccess) {
        error = std::string("cudaGetDevice: ") + cudaGetErrorString(status);
        return nullptr;
    }
    if (device < 0 || device >= 64) {
        error = "device " + std::to_string(device) + " is beyond the 64 devices this entry point serves";
        return nullptr;
    }
    std::lock_guard<std::mutex> guard(lock);
    if (!address[device]) {
        void* p = nullptr;
        status = cudaGetSymbolAddress(&p, g_noalloc_row_sums);
        if (status != cudaSuccess) {
            error = std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(status);
            return nullptr;
        }
        address[device] = static_cast<double*>(p);
    }
    return address[device];
}

}  // namespace odie
