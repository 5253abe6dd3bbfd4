// Shared device helpers for the ODIE B200 library (sm_100a only).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string>
#include <stdexcept>

#if !defined(__CUDA_ARCH__) || __CUDA_ARCH__ >= 1000
#else
#error "odie_b200 is built for sm_100a only"
#endif

namespace odie {

// ---------------------------------------------------------------- errors
struct CudaError : std::runtime_error {
    explicit CudaError(const std::string& what) : std::runtime_error(what) {}
};
#define ODIE_CUDA(expr)                                                                  \
    do {                                                                                 \
        cudaError_t odie_status_ = (expr);                                               \
        if (odie_status_ != cudaSuccess)                                                 \
            throw ::odie::CudaError(std::string(#expr) + ": " + cudaGetErrorString(odie_status_)); \
    } while (0)
#define ODIE_REQUIRE(cond, msg)                          \
    do {                                                 \
        if (!(cond)) throw std::invalid_argument(msg);   \
    } while (0)

void set_error(const std::string& message);  // thread-local, read by odie_error()
// Runs f, turning an exception into status -1 and the thread's error message (every C-ABI entry point).
template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        set_error(e.what());
        return -1;
    }
}
void note_launch(int kernels = 1);          // counts this library's kernel launches (odie_launch_count)
int sm_count();                              // cached multiprocessor count of the current device

inline unsigned blocks_for(long long n, int threads) { return unsigned((n + threads - 1) / threads); }

// Device buffer owned by the library (released with its owner).
template <typename T>
struct DeviceArray {
    T* ptr = nullptr;
    long long count = 0;
    DeviceArray() = default;
    DeviceArray(const DeviceArray&) = delete;
    DeviceArray& operator=(const DeviceArray&) = delete;
    ~DeviceArray() { release(); }
    void release() {
        if (ptr) cudaFree(ptr);
        ptr = nullptr;
        count = 0;
    }
    void allocate(long long n) {
        release();
        if (n <= 0) return;
        ODIE_CUDA(cudaMalloc(&ptr, size_t(n) * sizeof(T)));
        count = n;
    }
    void zero(cudaStream_t stream) {
        if (count) ODIE_CUDA(cudaMemsetAsync(ptr, 0, size_t(count) * sizeof(T), stream));
    }
};

// Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC 2011):
// a counter-based generator, so slot j of step s has its own stream with no state to carry.
struct Philox4 {
    uint32_t v[4];
};
__device__ __forceinline__ Philox4 philox4x32_10(Philox4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r > 0) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint32_t lo0 = 0xD2511F53u * c.v[0], hi0 = __umulhi(0xD2511F53u, c.v[0]);
        const uint32_t lo1 = 0xCD9E8D57u * c.v[2], hi1 = __umulhi(0xCD9E8D57u, c.v[2]);
        c = Philox4{{hi1 ^ c.v[1] ^ k0, lo1, hi0 ^ c.v[3] ^ k1, lo0}};
    }
    return c;
}

// ---------------------------------------------------------------- levels
// One encoding level as the kernels see it (built on the host from the
// reference's int32 descriptor rows [R, points, plane offset, node word offset,
// cell bitmap offset, F, feature offset, direct] or from a hash-grid layout).
enum LevelKind : int { PLANE = 0, HASH_DENSE = 1, HASH_HASHED = 2 };
struct __align__(16) Level {
    float scale;     // coordinate scale: R-1 for planes, the fp32 grid scale for hash levels
    int res;         // row stride of cells / integer corners
    int points;      // node universe: modulo for node indices
    int offset;      // first parameter of the level (elements)
    int words;       // first node-index word of a packed plane, -1 for direct addressing
    int cells;       // first byte of the level's cell bitmap, -1 for no bitmap (always visible)
    int F;           // features per node: 1, 2 or 4
    int col;         // first output feature column
    int kind;        // LevelKind
    int pad[3];
};
constexpr int MAX_LEVELS = 32;

// geometry, the reference's packed_kernels.cu:12-22: p = fmaf(scale, x, 0.5),
// integer cell = floor(p), bilinear weights of the 4 corners (x-fastest).
struct Corner4 {
    int ix, iy;
    float w[4];
};
// floor(p) without the conversion unit (whose float/int conversions bound the gathers and scatters):
// p + 1.5 x 2^23 rounded toward minus infinity is floor(p) + 1.5 x 2^23 exactly for |p| < 2^22 (the sum lies
// in [2^23, 2^24), where fp32 spacing is 1), so its bits minus the constant's are floor(p) and the sum minus
// the constant is floor(p) as a float.  Outside that range (coordinates far outside [0, 1], or NaN) the
// integer lands outside [0, 2^22): off every grid, so level_on() hides the level.
constexpr float FLOOR_MAGIC = 12582912.0f;  // 1.5 x 2^23
constexpr int FLOOR_MAGIC_BITS = 0x4B400000;
__device__ __forceinline__ float floor_split(float p, int& i) {
    const float t = __fadd_rd(p, FLOOR_MAGIC);
    i = __float_as_int(t) - FLOOR_MAGIC_BITS;
    return __fsub_rn(t, FLOOR_MAGIC);  // exact: t and the constant share a binade
}
__device__ __forceinline__ Corner4 geometry(float x, float y, float scale) {
    Corner4 c;
    const float px = __fmaf_rn(scale, x, 0.5f), py = __fmaf_rn(scale, y, 0.5f);
    const float bx = floor_split(px, c.ix), by = floor_split(py, c.iy);
    const float fx = __fsub_rn(px, bx), fy = __fsub_rn(py, by);
    const float gx = __fsub_rn(1.0f, fx), gy = __fsub_rn(1.0f, fy);
    c.w[0] = __fmul_rn(gx, gy);
    c.w[1] = __fmul_rn(fx, gy);
    c.w[2] = __fmul_rn(gx, fy);
    c.w[3] = __fmul_rn(fx, fy);
    return c;
}

__device__ __forceinline__ bool cell_visible(const Level& d, const uint8_t* __restrict__ bitmap, int cell) {
    if (d.cells < 0) return true;
    return (__ldg(bitmap + d.cells + (cell >> 3)) >> (cell & 7)) & 1;
}

// Row of a node in a packed plane: exclusive popcount rank over a 64-bit
// presence word plus the word's prefix (node-bitmap64-exclusive-prefix32).
__device__ __forceinline__ int packed_row(const Level& d, const uint64_t* __restrict__ node_bitmap,
                                          const int* __restrict__ prefix, int node) {
    if (d.words < 0) return node;
    const int word = d.words + (node >> 6);
    const uint64_t mask = (uint64_t(1) << (node & 63)) - 1;
    return __ldg(prefix + word) + __popcll(__ldg(reinterpret_cast<const unsigned long long*>(node_bitmap) + word) & mask);
}

// idx mod points without a division in the common cases: a power-of-two table
// (every hashed level) masks; an index below 2 x points (every in-range dense or
// plane corner: at most (R+1)^2 - 1 < 2 align8(R^2)) subtracts once; anything
// else (coordinates outside [0, 1]) takes the full remainder, so no index leaves
// the table.
__device__ __forceinline__ uint32_t wrap_index(uint32_t idx, uint32_t points) {
    if ((points & (points - 1)) == 0) return idx & (points - 1);
    if (idx < points) return idx;
    return idx - points < points ? idx - points : idx % points;
}

// Parameter row of corner k (0: x0y0, 1: x1y0, 2: x0y1, 3: x1y1) of a level.
// KIND: the level's kind when the caller knows it at compile time (smaller code), -1 to read d.kind.
template <int KIND = -1>
__device__ __forceinline__ int corner_row(const Level& d, const Corner4& g, int k,
                                          const uint64_t* __restrict__ node_bitmap, const int* __restrict__ prefix) {
    const int dx = k & 1, dy = k >> 1;
    const int kind = KIND >= 0 ? KIND : d.kind;
    if (kind == PLANE) {
        const int cell = g.ix + g.iy * d.res;
        const int raw = cell + dx + dy * d.res;
        // the reference's (cell + dx + dy R) % points on a non-negative int; level_on() hides cells outside
        // the grid, so raw >= 0 here for every visible corner
        const int node = raw >= 0 ? int(wrap_index(uint32_t(raw), uint32_t(d.points))) : raw % d.points;
        return packed_row(d, node_bitmap, prefix, node);
    }
    const uint32_t cx = uint32_t(g.ix + dx), cy = uint32_t(g.iy + dy);
    uint32_t idx;
    if (kind == HASH_HASHED) idx = cx ^ (cy * 2654435761u);
    else idx = cx + cy * uint32_t(d.res);
    return int(wrap_index(idx, uint32_t(d.points)));
}

__device__ __forceinline__ int level_cell(const Level& d, const Corner4& g) { return g.ix + g.iy * d.res; }

// ---------------------------------------------------------------- fp16 bits
// {half(x), half(x)}: one packed conversion (round to nearest even, as __float2half_rn).
__device__ __forceinline__ __half2 half2_dup(float x) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(r) : "f"(x));
    return *reinterpret_cast<const __half2*>(&r);
}
__device__ __forceinline__ uint32_t pack_half2(__half lo, __half hi) {
    return uint32_t(__half_as_ushort(lo)) | (uint32_t(__half_as_ushort(hi)) << 16);
}
__device__ __forceinline__ __half lo_half(uint32_t v) { return __ushort_as_half(uint16_t(v & 0xffff)); }
__device__ __forceinline__ __half hi_half(uint32_t v) { return __ushort_as_half(uint16_t(v >> 16)); }

// 8-byte vector reduction into global memory (sm_90+).
__device__ __forceinline__ void red_add_v2(float* address, float a, float b) {
    asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(address), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void red_add_f32(float* address, float a) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(address), "f"(a) : "memory");
}

}  // namespace odie
