// Procedural gigapixel test image (benchmark input; no reference counterpart).
//
// The reference measures on gigapixel photographs that are not available here; this
// kernel draws a seeded stand-in of any size, row band by row band, so that every
// data-parallel rank can draw exactly its own rows of the same image.  Every pixel is a
// pure function of (seed, column, row, width, height):
//   * fractal value noise with a 1/f^2 power spectrum: octaves o = 0..11 of lattice
//     spacing S_o = 2^(13 - o) pixels and amplitude proportional to S_o, each a
//     smoothstep-bilinear interpolation of hashed lattice values in [-1, 1], one shared
//     luminance field plus one field per channel;
//   * sharp edges: two Voronoi partitions (jittered lattices of 1024 and 192 pixels), each
//     region a flat colour offset, so region borders are one-pixel steps;
//   * a texture atlas of 64 x 64 cells: each cell takes one of eight seeded patterns
//     (hard stripes, checkers, dots, rings, triangle-wave stripes, grid lines, hatching,
//     none) with its own period, orientation and two colours.
// The sum is clamped to [0, 1] and rounded to u8.  The hash is the 32-bit finaliser of
// MurmurHash3 (Appleby, public domain) applied to mixed integer coordinates.
#include "common.cuh"
#include "odie_b200.h"

namespace odie {

namespace {

__device__ __forceinline__ uint32_t fmix32(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85ebca6bu;
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    h ^= h >> 16;
    return h;
}
__device__ __forceinline__ uint32_t hash4(uint32_t seed, uint32_t a, uint32_t b, uint32_t c) {
    return fmix32(seed ^ fmix32(a * 0x9E3779B1u ^ fmix32(b * 0x85EBCA77u ^ fmix32(c * 0xC2B2AE3Du + 0x27D4EB2Fu))));
}
// uniform in [-1, 1)
__device__ __forceinline__ float signed_unit(uint32_t h) { return float(h >> 8) * (2.0f / 16777216.0f) - 1.0f; }
// uniform in [0, 1)
__device__ __forceinline__ float unit(uint32_t h) { return float(h >> 8) * (1.0f / 16777216.0f); }
__device__ __forceinline__ float smooth(float t) { return t * t * (3.0f - 2.0f * t); }

// Value noise of one octave and field at pixel (x, y): lattice spacing 2^shift.
__device__ __forceinline__ float value_noise(uint32_t seed, uint32_t field, int shift, int x, int y) {
    const int ix = x >> shift, iy = y >> shift;
    const float scale = 1.0f / float(1 << shift);
    const float fx = smooth(float(x - (ix << shift)) * scale), fy = smooth(float(y - (iy << shift)) * scale);
    const uint32_t salt = field * 64u + uint32_t(shift);
    const float v00 = signed_unit(hash4(seed, salt, uint32_t(ix), uint32_t(iy)));
    const float v10 = signed_unit(hash4(seed, salt, uint32_t(ix + 1), uint32_t(iy)));
    const float v01 = signed_unit(hash4(seed, salt, uint32_t(ix), uint32_t(iy + 1)));
    const float v11 = signed_unit(hash4(seed, salt, uint32_t(ix + 1), uint32_t(iy + 1)));
    const float top = v00 + (v10 - v00) * fx, bottom = v01 + (v11 - v01) * fx;
    return top + (bottom - top) * fy;
}

// 1/f^2 fractal: amplitude halves as the frequency doubles; normalised to unit total amplitude.
__device__ __forceinline__ float fractal(uint32_t seed, uint32_t field, int x, int y) {
    float sum = 0.0f, amplitude = 1.0f, total = 0.0f;
#pragma unroll 1
    for (int shift = 13; shift >= 2; --shift) {
        sum += amplitude * value_noise(seed, field, shift, x, y);
        total += amplitude;
        amplitude *= 0.5f;
    }
    return sum / total;
}

// Flat colour offset of the Voronoi region of (x, y) on a jittered lattice of `spacing` pixels.
__device__ __forceinline__ void voronoi(uint32_t seed, uint32_t salt, int spacing, int x, int y, float* rgb) {
    const int cx = x / spacing, cy = y / spacing;
    float best = 3.4e38f;
    uint32_t owner = 0;
#pragma unroll
    for (int dy = -1; dy <= 1; ++dy)
#pragma unroll
        for (int dx = -1; dx <= 1; ++dx) {
            const uint32_t h = hash4(seed, salt, uint32_t(cx + dx), uint32_t(cy + dy));
            const float px = (float(cx + dx) + unit(h)) * float(spacing);
            const float py = (float(cy + dy) + unit(fmix32(h))) * float(spacing);
            const float d = (px - float(x)) * (px - float(x)) + (py - float(y)) * (py - float(y));
            if (d < best) {
                best = d;
                owner = h;
            }
        }
    for (int c = 0; c < 3; ++c) rgb[c] = signed_unit(fmix32(owner + 0x632BE5ABu * uint32_t(c + 1)));
}

// Pattern of the atlas cell holding (x, y): value in [0, 1] and the cell's two colours.
__device__ __forceinline__ float atlas(uint32_t seed, int cell_px, int x, int y, float* c0, float* c1) {
    const int cx = x / cell_px, cy = y / cell_px;
    const uint32_t h = hash4(seed, 0xA71A5u, uint32_t(cx), uint32_t(cy));
    const uint32_t kind = h & 7u;
    const float period = 6.0f + 58.0f * unit(fmix32(h ^ 0x1u));
    const float angle = 6.2831853f * unit(fmix32(h ^ 0x2u));
    const float ca = __cosf(angle), sa = __sinf(angle);
    const float lx = float(x - cx * cell_px), ly = float(y - cy * cell_px);
    const float u = (lx * ca + ly * sa) / period, v = (ly * ca - lx * sa) / period;
    const float fu = u - floorf(u), fv = v - floorf(v);
    for (int c = 0; c < 3; ++c) {
        c0[c] = unit(fmix32(h + 0x3u + 7u * uint32_t(c)));
        c1[c] = unit(fmix32(h + 0x5u + 11u * uint32_t(c)));
    }
    switch (kind) {
        case 0: return fu < 0.5f ? 1.0f : 0.0f;                                        // hard stripes
        case 1: return ((fu < 0.5f) != (fv < 0.5f)) ? 1.0f : 0.0f;                      // checkers
        case 2: return ((fu - 0.5f) * (fu - 0.5f) + (fv - 0.5f) * (fv - 0.5f) < 0.09f) ? 1.0f : 0.0f;  // dots
        case 3: {                                                                        // rings
            const float r = sqrtf((lx - 0.5f * cell_px) * (lx - 0.5f * cell_px) + (ly - 0.5f * cell_px) * (ly - 0.5f * cell_px)) / period;
            return (r - floorf(r)) < 0.5f ? 1.0f : 0.0f;
        }
        case 4: return fabsf(2.0f * fu - 1.0f);                                          // triangle-wave stripes
        case 5: return (fu < 0.12f || fv < 0.12f) ? 1.0f : 0.0f;                         // grid lines
        case 6: return (fu < 0.25f) ? 1.0f : (fabsf(2.0f * fv - 1.0f) > 0.8f ? 1.0f : 0.0f);  // hatching
        default: return 0.5f;                                                            // plain
    }
}

__global__ void procedural_image_kernel(uint32_t seed, int width, int height, int row0, int rows,
                                        uint8_t* __restrict__ rgb) {
    const long long count = (long long)width * rows;
    const int cell_px = (width > height ? width : height) / 64 > 0 ? (width > height ? width : height) / 64 : 1;
    for (long long p = (long long)blockIdx.x * blockDim.x + threadIdx.x; p < count; p += (long long)gridDim.x * blockDim.x) {
        const int x = int(p % width), y = row0 + int(p / width);
        const float luma = fractal(seed, 0u, x, y);
        float edge_big[3], edge_small[3], c0[3], c1[3];
        voronoi(seed, 0xB16u, 1024, x, y, edge_big);
        voronoi(seed, 0x5A11u, 192, x, y, edge_small);
        const float pattern = atlas(seed, cell_px, x, y, c0, c1);
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            const float chroma = fractal(seed, uint32_t(c + 1), x, y);
            const float texture = c0[c] + (c1[c] - c0[c]) * pattern - 0.5f;
            float value = 0.5f + 0.30f * luma + 0.12f * chroma + 0.14f * edge_big[c] + 0.06f * edge_small[c] + 0.22f * texture;
            value = fminf(fmaxf(value, 0.0f), 1.0f);
            rgb[3 * p + c] = uint8_t(__float2int_rn(value * 255.0f));
        }
    }
}

}  // namespace

void launch_procedural_image(uint64_t seed, int width, int height, int row0, int rows, uint8_t* rgb, cudaStream_t stream) {
    ODIE_REQUIRE(width >= 1 && height >= 1 && row0 >= 0 && rows >= 0 && (long long)row0 + rows <= height,
                 "the rows must lie within the image");
    const long long count = (long long)width * rows;
    if (count == 0) return;
    const uint32_t mixed = uint32_t(seed) ^ uint32_t(seed >> 32) * 0x9E3779B1u;
    const long long blocks = (count + 255) / 256;
    const unsigned grid = unsigned(blocks < 16LL * sm_count() ? blocks : 16LL * sm_count());
    procedural_image_kernel<<<grid, 256, 0, stream>>>(mixed, width, height, row0, rows, rgb);
    note_launch();
}

}  // namespace odie

extern "C" int odie_procedural_image(uint64_t seed, int width, int height, int row0, int rows, uint8_t* rgb,
                                     uint64_t stream) {
    try {
        odie::launch_procedural_image(seed, width, height, row0, rows, rgb, reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
        return 0;
    } catch (const std::exception& e) {
        odie::set_error(e.what());
        return -1;
    }
}
