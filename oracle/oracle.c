/*
 * CPU oracle for the ODIE hot path.  TEST INFRASTRUCTURE ONLY: this file is
 * the checker that the CUDA library is compared against.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm may load
 * it; the product path (odie_b200) never does.
 *
 * Every function restates one reference function (file:line cited, paths
 * relative to the ODIE project root).  Floating-point rounding points follow
 * the reference exactly where the reference fixes them:
 *   - fp32 operations are plain IEEE single operations (built with
 *     -ffp-contract=off so no FMA contraction happens behind our back);
 *   - an fp16 operation is computed exactly in double and rounded once to
 *     _Float16 (a product of two fp16 values is exact in double and the sums
 *     used here stay within 53 bits, so this equals a single IEEE fp16
 *     rounding, i.e. __hfma/__hmul_rn/__hadd_rn);
 *   - fp64 sums run in the reference's raster order.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef _Float16 half;

static inline half h_of(double x) { return (half)x; }
static inline float f_of_h(half x) { return (float)x; }
static inline half hfma(half a, half b, half c) { return (half)((double)a * (double)b + (double)c); }
static inline half hmul(half a, half b) { return (half)((double)a * (double)b); }
static inline half hadd(half a, half b) { return (half)((double)a + (double)b); }

static inline uint16_t bits_of_h(half x) { uint16_t u; memcpy(&u, &x, 2); return u; }
static inline half h_of_bits(uint16_t u) { half x; memcpy(&x, &u, 2); return x; }

/* ------------------------------------------------------------------ a1 */
/* input_batch, odie/native/runtime.cu:30-38: x = fp32(id % W) * fp32(1/(W-1)),
 * the reciprocal computed in double and rounded to fp32. ids are truncated to
 * uint32 as in the reference. */
void oracle_coords(const int64_t* ids, int64_t n, int width, int height, float* xy) {
    const float ix = (float)(1.0 / (double)(width - 1));
    const float iy = (float)(1.0 / (double)(height - 1));
    for (int64_t i = 0; i < n; ++i) {
        uint32_t id = (uint32_t)ids[i];
        xy[2 * i] = (float)(id % (uint32_t)width) * ix;
        xy[2 * i + 1] = (float)(id / (uint32_t)width) * iy;
    }
}

/* The same coordinates for the rows of a band of a taller image (no reference counterpart): local
 * pixel id of an image whose rows are rows [row0, row0 + height) of a full image of `rows` rows;
 * y = (row0 + id / width) * fl(1 / (rows - 1)).  row0 = 0, rows = height is oracle_coords. */
void oracle_coords_frame(const int64_t* ids, int64_t n, int width, int row0, int rows, float* xy) {
    const float ix = (float)(1.0 / (double)(width - 1));
    const float iy = (float)(1.0 / (double)(rows - 1));
    for (int64_t i = 0; i < n; ++i) {
        uint32_t id = (uint32_t)ids[i];
        xy[2 * i] = (float)(id % (uint32_t)width) * ix;
        xy[2 * i + 1] = (float)((uint32_t)row0 + id / (uint32_t)width) * iy;
    }
}

/* ------------------------------------------------------------------ a2 */
/* geometry, odie/packed_kernels.cu:12-22 */
static inline void geometry(float x, float y, float scale, int r, int* cell, float* w) {
    const float px = fmaf(scale, x, 0.5f), py = fmaf(scale, y, 0.5f);
    const int ix = (int)floorf(px), iy = (int)floorf(py);
    const float fx = px - (float)ix, fy = py - (float)iy;
    *cell = ix + iy * r;
    w[0] = (1.0f - fx) * (1.0f - fy);
    w[1] = fx * (1.0f - fy);
    w[2] = (1.0f - fx) * fy;
    w[3] = fx * fy;
}

/* Exposed for tests: cell and weights of one level for n coordinates. */
void oracle_geometry(const float* xy, int64_t n, int r, int* cells, float* weights) {
    for (int64_t i = 0; i < n; ++i)
        geometry(xy[2 * i], xy[2 * i + 1], (float)(r - 1), r, cells + i, weights + 4 * i);
}

/* ------------------------------------------------------------------ a3/a4/a5 */
/* visible, odie/packed_kernels.cu:24-26 */
static inline int visible(const uint8_t* bitmap, const int* d, int cell) {
    return (bitmap[d[4] + (cell >> 3)] >> (cell & 7)) & 1;
}
/* packed_row, odie/packed_kernels.cu:28-36 */
static inline int packed_row(const uint64_t* node_bitmap, const int* prefix, const int* d, int node) {
    if (d[7]) return node;
    const int word = d[3] + (node >> 6);
    const uint64_t mask = (((uint64_t)1) << (node & 63)) - 1;
    return prefix[word] + __builtin_popcountll(node_bitmap[word] & mask);
}
/* node addressing, odie/packed_kernels.cu:56 */
static inline int corner_node(const int* d, int cell, int k) {
    return (cell + (k & 1) + (k >> 1) * d[0]) % d[1];
}

/* Per (coordinate, level): visibility and the 4 packed rows (-1 when hidden). */
void oracle_rows(const float* xy, int64_t n, const int* desc, int levels, const uint64_t* node_bitmap,
                 const int* prefix, const uint8_t* bitmap, uint8_t* vis, int* rows) {
    for (int64_t i = 0; i < n; ++i)
        for (int l = 0; l < levels; ++l) {
            const int* d = desc + 8 * l;
            int cell; float w[4];
            geometry(xy[2 * i], xy[2 * i + 1], (float)(d[0] - 1), d[0], &cell, w);
            const int on = visible(bitmap, d, cell);
            vis[i * levels + l] = (uint8_t)on;
            for (int k = 0; k < 4; ++k)
                rows[(i * levels + l) * 4 + k] = on ? packed_row(node_bitmap, prefix, d, corner_node(d, cell, k)) : -1;
        }
}

/* ------------------------------------------------------------------ a6 */
/* query_kernel, odie/packed_kernels.cu:38-64 and query, odie/native/runtime.cu:39-52.
 * out: fp16 bits [n x width]; levels >= active produce +0 and are hidden;
 * when pad_ones is set, columns raw_width..width are 1.0 (runtime.cu:51). */
void oracle_query(const float* xy, int64_t n, const float* grid, const int* desc, int levels,
                  const uint64_t* node_bitmap, const int* prefix, const uint8_t* bitmap, int width,
                  int active, int raw_width, int pad_ones, uint16_t* out, uint8_t* vis) {
    for (int64_t i = 0; i < n; ++i) {
        for (int l = 0; l < levels; ++l) {
            const int* d = desc + 8 * l;
            int cell; float w[4];
            geometry(xy[2 * i], xy[2 * i + 1], (float)(d[0] - 1), d[0], &cell, w);
            const int on = l < active && visible(bitmap, d, cell);
            vis[i * levels + l] = (uint8_t)on;
            for (int c = 0; c < d[5]; ++c) {
                half v = h_of(0.0);
                if (on)
                    for (int k = 0; k < 4; ++k) {
                        const int row = packed_row(node_bitmap, prefix, d, corner_node(d, cell, k));
                        v = hfma(h_of(w[k]), h_of(grid[d[2] + row * d[5] + c]), v);
                    }
                out[i * width + d[6] + c] = bits_of_h(v);
            }
        }
        if (pad_ones)
            for (int c = raw_width; c < width; ++c) out[i * width + c] = bits_of_h(h_of(1.0));
    }
}

/* ------------------------------------------------------------------ a7 */
/* gradient_kernel, odie/packed_kernels.cu:66-88: grad[row*F+c] += w_k * g for
 * visible cells, channels with g == 0 skipped.  Accumulated in double (the
 * reference's fp32 atomics are order-nondeterministic; parity is by tolerance). */
void oracle_query_backward(const float* xy, int64_t n, const uint16_t* upstream, int width,
                           const int* desc, int levels, const uint64_t* node_bitmap, const int* prefix,
                           const uint8_t* bitmap, double* grad) {
    for (int64_t i = 0; i < n; ++i)
        for (int l = 0; l < levels; ++l) {
            const int* d = desc + 8 * l;
            int cell; float w[4];
            geometry(xy[2 * i], xy[2 * i + 1], (float)(d[0] - 1), d[0], &cell, w);
            if (!visible(bitmap, d, cell)) continue;
            for (int c = 0; c < d[5]; ++c) {
                const float g = f_of_h(h_of_bits(upstream[i * width + d[6] + c]));
                if (g == 0.0f) continue;
                for (int k = 0; k < 4; ++k) {
                    const int row = packed_row(node_bitmap, prefix, d, corner_node(d, cell, k));
                    grad[d[2] + row * d[5] + c] += (double)(w[k] * g);
                }
            }
        }
}

/* ------------------------------------------------------------------ a16 */
/* Hashed multiresolution addressing (no code in the ODIE tree: TCNN's HashGrid,
 * called at odie/hash_grid.py:27 and odie/native/runtime.cu:186, is not vendored).
 * Restated from the published Instant-NGP encoding (Mueller et al. 2022):
 *   pos = fmaf(scale_l, x, 0.5), integer corner (ix+dx, iy+dy);
 *   dense levels (res^2 <= capacity): index = (cx + cy*res) mod capacity;
 *   hashed levels: index = (cx * 1 XOR cy * 2654435761) mod capacity (uint32).
 * scale_l and res_l follow odie/config.py:83-94 (hash_grid_layout).
 * lv: per level {float scale, int res, int capacity, int offset, int F, int feature_offset, int hashed}. */
typedef struct { float scale; int res, capacity, offset, F, feature_offset, hashed, cells; } HashLevel;
/* cells: byte offset of the level's cell-visibility bitmap (bit c mod 8 of byte c / 8 for cell
 * c = ix + iy * res), or -1 for a level whose cells are all visible.  A hidden cell (or one outside the
 * res x res grid) contributes zero features and receives no gradient, as the packed planes' cells do. */
static inline int hash_visible(const HashLevel* h, const uint8_t* bitmap, int ix, int iy) {
    if (h->cells < 0 || !bitmap) return 1;
    if (ix < 0 || iy < 0 || ix >= h->res || iy >= h->res) return 0;
    const int64_t c = (int64_t)ix + (int64_t)iy * h->res;
    return (bitmap[h->cells + (c >> 3)] >> (c & 7)) & 1;
}

static inline uint32_t hash_index(const HashLevel* h, int cx, int cy) {
    uint32_t idx;
    if (h->hashed) idx = ((uint32_t)cx * 1u) ^ ((uint32_t)cy * 2654435761u);
    else idx = (uint32_t)cx + (uint32_t)cy * (uint32_t)h->res;
    return idx % (uint32_t)h->capacity;
}

void oracle_hash_indices(const float* xy, int64_t n, const HashLevel* lv, int levels, int* idx, float* weights) {
    for (int64_t i = 0; i < n; ++i)
        for (int l = 0; l < levels; ++l) {
            const HashLevel* h = lv + l;
            const float px = fmaf(h->scale, xy[2 * i], 0.5f), py = fmaf(h->scale, xy[2 * i + 1], 0.5f);
            const int ix = (int)floorf(px), iy = (int)floorf(py);
            const float fx = px - (float)ix, fy = py - (float)iy;
            float* w = weights + (i * levels + l) * 4;
            w[0] = (1.0f - fx) * (1.0f - fy); w[1] = fx * (1.0f - fy);
            w[2] = (1.0f - fx) * fy; w[3] = fx * fy;
            for (int k = 0; k < 4; ++k)
                idx[(i * levels + l) * 4 + k] = (int)hash_index(h, ix + (k & 1), iy + (k >> 1));
        }
}

/* Hash-grid forward with fp16 tables (table bits) and the same fp16 hfma chain as a6; bitmap may be NULL. */
void oracle_hash_query(const float* xy, int64_t n, const uint16_t* table, const HashLevel* lv, int levels,
                       int width, const uint8_t* bitmap, uint16_t* out) {
    for (int64_t i = 0; i < n; ++i)
        for (int l = 0; l < levels; ++l) {
            const HashLevel* h = lv + l;
            const float px = fmaf(h->scale, xy[2 * i], 0.5f), py = fmaf(h->scale, xy[2 * i + 1], 0.5f);
            const int ix = (int)floorf(px), iy = (int)floorf(py);
            const float fx = px - (float)ix, fy = py - (float)iy;
            float w[4] = {(1.0f - fx) * (1.0f - fy), fx * (1.0f - fy), (1.0f - fx) * fy, fx * fy};
            const int on = hash_visible(h, bitmap, ix, iy);
            for (int c = 0; c < h->F; ++c) {
                half v = h_of(0.0);
                for (int k = 0; k < 4 && on; ++k) {
                    uint32_t idx = hash_index(h, ix + (k & 1), iy + (k >> 1));
                    v = hfma(h_of(w[k]), h_of_bits(table[h->offset + idx * h->F + c]), v);
                }
                out[i * width + h->feature_offset + c] = bits_of_h(v);
            }
        }
}

void oracle_hash_backward(const float* xy, int64_t n, const uint16_t* upstream, int width,
                          const HashLevel* lv, int levels, const uint8_t* bitmap, double* grad) {
    for (int64_t i = 0; i < n; ++i)
        for (int l = 0; l < levels; ++l) {
            const HashLevel* h = lv + l;
            const float px = fmaf(h->scale, xy[2 * i], 0.5f), py = fmaf(h->scale, xy[2 * i + 1], 0.5f);
            const int ix = (int)floorf(px), iy = (int)floorf(py);
            if (!hash_visible(h, bitmap, ix, iy)) continue;
            const float fx = px - (float)ix, fy = py - (float)iy;
            float w[4] = {(1.0f - fx) * (1.0f - fy), fx * (1.0f - fy), (1.0f - fx) * fy, fx * fy};
            for (int c = 0; c < h->F; ++c) {
                const float g = f_of_h(h_of_bits(upstream[i * width + h->feature_offset + c]));
                if (g == 0.0f) continue;
                for (int k = 0; k < 4; ++k) {
                    uint32_t idx = hash_index(h, ix + (k & 1), iy + (k >> 1));
                    grad[h->offset + idx * h->F + c] += (double)(w[k] * g);
                }
            }
        }
}

/* ------------------------------------------------------------------ a9 */
/* parallel_gate, odie/native/runtime.cu:66-75.  feature_level[c] maps each raw
 * column to its level (-1 for pad columns, which become 1.0).  logits are fp16
 * bits [n x gate_width]; sigmoid gets fp32 [n x levels]. */
void oracle_gate_forward(const uint16_t* raw, const uint16_t* logits, const uint8_t* vis, int64_t n,
                         int levels, int width, int gate_width, const int* feature_level, int k_fixed,
                         int softplus, uint16_t* weighted, float* sigmoid) {
    for (int64_t i = 0; i < n; ++i) {
        for (int l = 0; l < levels; ++l) {
            const float z = f_of_h(h_of_bits(logits[i * gate_width + l]));
            float s;
            if (l < k_fixed) s = 1.0f;
            else if (softplus) s = z > 20.0f ? z : log1pf(expf(z));
            else s = 1.0f / (1.0f + expf(-z));
            sigmoid[i * levels + l] = s;
        }
        for (int c = 0; c < width; ++c) {
            const int l = feature_level[c];
            if (l < 0) { weighted[i * width + c] = bits_of_h(h_of(1.0)); continue; }
            const half weight = h_of(sigmoid[i * levels + l] * (float)vis[i * levels + l]);
            weighted[i * width + c] = bits_of_h(hmul(h_of_bits(raw[i * width + c]), weight));
        }
    }
}

/* parallel_gate_back, odie/native/runtime.cu:76-92 (fuse_direct = false). */
void oracle_gate_backward(const uint16_t* raw, const float* sigmoid, const uint8_t* vis, const uint16_t* dz,
                          int64_t n, int levels, int width, int gate_width, const int* level_offset,
                          const int* level_dim, int k_fixed, int softplus, uint16_t* direct, uint16_t* da) {
    for (int64_t i = 0; i < n; ++i) {
        for (int c = 0; c < width; ++c) direct[i * width + c] = bits_of_h(h_of(0.0));
        for (int l = 0; l < levels; ++l) {
            const float s = sigmoid[i * levels + l];
            const half weight = h_of(s * (float)vis[i * levels + l]);
            half reduced = h_of(0.0);
            for (int c = 0; c < level_dim[l]; ++c) {
                const int j = i * width + level_offset[l] + c;
                const half value = h_of(f_of_h(h_of_bits(dz[j])) / 128.0f);
                direct[j] = bits_of_h(hmul(value, weight));
                reduced = hadd(reduced, hmul(value, h_of_bits(raw[j])));
            }
            const float incoming = f_of_h(reduced) * (float)vis[i * levels + l];
            float derivative;
            if (l < k_fixed) derivative = 0.0f;
            else if (softplus) derivative = incoming * (-expm1f(-s));
            else derivative = (incoming * (1.0f - s)) * s;
            da[i * gate_width + l] = bits_of_h(hmul(h_of(derivative), h_of(128.0)));
        }
        for (int c = levels; c < gate_width; ++c) da[i * gate_width + c] = bits_of_h(h_of(0.0));
    }
}

/* Grid-gradient values of grid_back, odie/native/runtime.cu:117-125 (router
 * enabled): v = fp32(hadd(direct, half(dr/128))); without router: half(dz/128). */
void oracle_grid_values(const uint16_t* direct, const uint16_t* dr, int64_t count, int router, float* values) {
    for (int64_t j = 0; j < count; ++j) {
        if (router)
            values[j] = f_of_h(hadd(h_of_bits(direct[j]), h_of(f_of_h(h_of_bits(dr[j])) / 128.0f)));
        else
            values[j] = f_of_h(h_of(f_of_h(h_of_bits(direct[j])) / 128.0f));
    }
}

/* ------------------------------------------------------------------ a12 */
/* loss_grad, odie/native/runtime.cu:53-63 (target already in fp32). output/dy
 * are fp16 bits with 16 columns. */
void oracle_loss_grad(const uint16_t* output, const float* target, int64_t n, int64_t real,
                      uint16_t* dy, float* squares) {
    for (int64_t i = 0; i < n; ++i) {
        if (i >= real) {
            for (int c = 0; c < 16; ++c) dy[i * 16 + c] = bits_of_h(h_of(0.0));
            squares[i] = 0.0f;
            continue;
        }
        float s = 0.0f;
        for (int c = 0; c < 3; ++c) {
            const float d = f_of_h(h_of_bits(output[i * 16 + c])) - target[3 * i + c];
            s += d * d;
            const float scaled = ((2.0f * d) / (float)(3 * real)) * 128.0f;
            dy[i * 16 + c] = bits_of_h(hmul(h_of(scaled), h_of(128.0)));
        }
        for (int c = 3; c < 16; ++c) dy[i * 16 + c] = bits_of_h(h_of(0.0));
        squares[i] = s / 3.0f;
    }
}

/* u8 target / 255 with the native __fmul_rn(u8, 1/255) of runtime.cu:37/57. */
void oracle_target_u8(const uint8_t* rgb, const int64_t* ids, int64_t n, float* target) {
    const float inv = 1.0f / 255.0f;
    for (int64_t i = 0; i < n; ++i)
        for (int c = 0; c < 3; ++c) target[3 * i + c] = (float)rgb[3 * (uint64_t)(uint32_t)ids[i] + c] * inv;
}

/* ------------------------------------------------------------------ a13 */
/* Adam with torch.optim.Adam semantics (odie/optimizer.py:33-44, the in-repo
 * reference optimizer, foreach=False):
 *   step += 1; m = lerp(m, g, 1-b1); v = b2 v + (1-b2) g g;
 *   p += (-lr / (1 - b1^step)) m / (sqrt(v) / sqrt(1 - b2^step) + eps)
 * with the per-parameter step counters and zero-gradient skip of the native
 * grid optimizer (odie/native/runtime.cu:212-213, odie/train.py:121-124).
 * g = grad / loss_scale.  Scalars (1-b1, 1-b2, step size, sqrt of the second
 * bias correction) are evaluated in double and rounded to fp32, as torch does
 * with python-float scalars; the element math is fp32 with the lerp and the
 * second-moment update as single-rounding fused multiply-adds (the forms
 * torch's vectorised CPU kernels use). */
void oracle_adam(float* p, float* m, float* v, uint32_t* steps, const float* grad, int64_t count,
                 float loss_scale, double lr, double beta1, double beta2, double eps, int skip_zero,
                 uint16_t* half_copy) {
    const float w1 = (float)(1.0 - beta1), b2 = (float)beta2, w2 = (float)(1.0 - beta2), e = (float)eps;
    for (int64_t i = 0; i < count; ++i) {
        const float g = grad[i] / loss_scale;
        if (skip_zero && g == 0.0f) continue;
        const uint32_t step = ++steps[i];
        m[i] = fmaf(w1, g - m[i], m[i]);
        v[i] = fmaf(w2 * g, g, v[i] * b2);
        const float step_size = (float)(lr / (1.0 - pow(beta1, (double)step)));
        const float bc2_sqrt = (float)sqrt(1.0 - pow(beta2, (double)step));
        const float denom = sqrtf(v[i]) / bc2_sqrt + e;
        p[i] = p[i] + (-step_size * m[i]) / denom;
        if (half_copy) half_copy[i] = bits_of_h(h_of(p[i]));
    }
}

/* ------------------------------------------------------------------ a17 */
/* accumulate, odie/residual_cuda.cu:11-43: one cell at a time, pixels in
 * raster order, fp32 diff/square, fp64 sum.  target is u8 (rgb8) or fp32. */
void oracle_score_chunk(const float* prediction, const void* target, int64_t begin, int64_t end, int width,
                        int resolution, int first_y, int active_cells, const int* xb, const int* yb,
                        double* totals, int rgb8) {
    for (int t = 0; t < active_cells; ++t) {
        const int cx = t % resolution, cy = first_y + t / resolution;
        const int64_t cell = (int64_t)cy * resolution + cx;
        int y0 = yb[cy], y1 = yb[cy + 1];
        if ((int)(begin / width) > y0) y0 = (int)(begin / width);
        if ((int)((end - 1) / width) + 1 < y1) y1 = (int)((end - 1) / width) + 1;
        double sum = totals[cell];
        for (int y = y0; y < y1; ++y) {
            const int64_t row = (int64_t)y * width;
            int64_t x0 = xb[cx] > begin - row ? xb[cx] : begin - row;
            int64_t x1 = xb[cx + 1] < end - row ? xb[cx + 1] : end - row;
            for (int64_t x = x0; x < x1; ++x) {
                const int64_t p = (row + x - begin) * 3;
                float t3[3];
                for (int c = 0; c < 3; ++c)
                    t3[c] = rgb8 ? (float)((const uint8_t*)target)[p + c] / 255.0f : ((const float*)target)[p + c];
                const float d0 = prediction[p] - t3[0], d1 = prediction[p + 1] - t3[1], d2 = prediction[p + 2] - t3[2];
                double rgb = (double)(d0 * d0) + (double)(d1 * d1);
                rgb = rgb + (double)(d2 * d2);
                sum = sum + rgb / 3.0;
            }
        }
        totals[cell] = sum;
    }
}

/* ------------------------------------------------------------------ a18 */
/* select_benefit_cost (B2 / E), odie/selection.py:129-207: exact greedy with
 * five lazy heaps keyed by current missing-corner count.  Free cells first in
 * ascending id; otherwise the best score/cost by cross multiplication, ties to
 * the lower id.  Returns iterations, or -1 on the stale-cost invariant. */
typedef struct { double key; int64_t id; } Entry;
typedef struct { Entry* a; int64_t n, cap; } Heap;

static inline int less(const Entry* x, const Entry* y) {
    return x->key < y->key || (x->key == y->key && x->id < y->id);
}
static void heap_push(Heap* h, Entry e) {
    if (h->n == h->cap) { h->cap = h->cap ? 2 * h->cap : 1024; h->a = (Entry*)realloc(h->a, h->cap * sizeof(Entry)); }
    int64_t i = h->n++;
    while (i > 0) {
        int64_t p = (i - 1) / 2;
        if (!less(&e, &h->a[p])) break;
        h->a[i] = h->a[p]; i = p;
    }
    h->a[i] = e;
}
static void heap_pop(Heap* h) {
    Entry last = h->a[--h->n];
    int64_t i = 0;
    for (;;) {
        int64_t c = 2 * i + 1;
        if (c >= h->n) break;
        if (c + 1 < h->n && less(&h->a[c + 1], &h->a[c])) ++c;
        if (!less(&h->a[c], &last)) break;
        h->a[i] = h->a[c]; i = c;
    }
    if (h->n) h->a[i] = last;
}

int64_t oracle_select_benefit_cost(const double* scores, int resolution, int64_t cap, int normalize,
                                   uint8_t* selected, uint8_t* nodes, int64_t* used_out) {
    const int64_t cells = (int64_t)resolution * resolution, points = (cells + 7) / 8 * 8;
    memset(selected, 0, cells);
    memset(nodes, 0, points);
    uint8_t* missing = (uint8_t*)malloc(cells);
    memset(missing, 4, cells);
    Heap heaps[5] = {{0}};
    heaps[4].cap = cells; heaps[4].a = (Entry*)malloc(cells * sizeof(Entry));
    for (int64_t c = 0; c < cells; ++c) heap_push(&heaps[4], (Entry){-scores[c], c});
    int64_t used = 0, iterations = 0;
    const int64_t deltas[4] = {0, 1, resolution, (int64_t)resolution + 1};
    int64_t changed[16];
    for (;;) {
        int64_t cell = -1; int cost = -1;
        /* clean(0) */
        Heap* h0 = &heaps[0];
        while (h0->n && (selected[h0->a[0].id] || missing[h0->a[0].id] != 0)) heap_pop(h0);
        if (h0->n) { cell = h0->a[0].id; cost = 0; }
        else {
            double best_score = 0; int best_cost = 0; int64_t best_cell = -1;
            int64_t limit = cap - used < 4 ? cap - used : 4;
            for (int k = 1; k <= limit; ++k) {
                Heap* hk = &heaps[k];
                while (hk->n && (selected[hk->a[0].id] || missing[hk->a[0].id] != k)) heap_pop(hk);
                if (!hk->n) continue;
                const double cs = -hk->a[0].key; const int64_t cc = hk->a[0].id;
                if (best_cell < 0) { best_score = cs; best_cost = k; best_cell = cc; }
                else {
                    const double left = normalize ? cs * (double)best_cost : cs;
                    const double right = normalize ? best_score * (double)k : best_score;
                    if (left > right || (left == right && cc < best_cell)) { best_score = cs; best_cost = k; best_cell = cc; }
                }
            }
            if (best_cell < 0) break;
            cell = best_cell; cost = best_cost;
        }
        heap_pop(&heaps[cost]);
        selected[cell] = 1;
        int64_t added[4]; int nadded = 0;
        for (int d = 0; d < 4; ++d) {
            const int64_t node = (cell + deltas[d]) % points;
            int dup = 0;
            for (int a = 0; a < nadded; ++a) dup |= added[a] == node;
            if (!nodes[node] && !dup) added[nadded++] = node;
        }
        if (nadded != cost) { iterations = -1; break; }
        for (int a = 0; a < nadded; ++a) nodes[added[a]] = 1;
        used += cost;
        ++iterations;
        int nchanged = 0;
        for (int a = 0; a < nadded; ++a)
            for (int d = 0; d < 4; ++d) {
                const int64_t inc = ((added[a] - deltas[d]) % points + points) % points;
                if (inc < cells && !selected[inc]) {
                    missing[inc] -= 1;
                    int seen = 0;
                    for (int j = 0; j < nchanged; ++j) seen |= changed[j] == inc;
                    if (!seen) changed[nchanged++] = inc;
                }
            }
        for (int j = 0; j < nchanged; ++j) {
            const int64_t inc = changed[j];
            const int cn = missing[inc];
            heap_push(&heaps[cn], (Entry){cn == 0 ? (double)inc : -scores[inc], inc});
        }
    }
    for (int k = 0; k < 5; ++k) free(heaps[k].a);
    free(missing);
    if (used_out) *used_out = used;
    return iterations;
}

/* select_mean_rank (B1), odie/selection.py:108-126: stable descending ranking,
 * admit a cell when its new closure nodes still fit the cap. */
static const double* g_rank_scores;
static int rank_cmp(const void* a, const void* b) {
    const int64_t x = *(const int64_t*)a, y = *(const int64_t*)b;
    const double sx = g_rank_scores[x], sy = g_rank_scores[y];
    if (sx > sy) return -1;
    if (sx < sy) return 1;
    return x < y ? -1 : (x > y);
}
int64_t oracle_select_mean_rank(const double* scores, int resolution, int64_t cap, uint8_t* selected, uint8_t* nodes) {
    const int64_t cells = (int64_t)resolution * resolution, points = (cells + 7) / 8 * 8;
    memset(selected, 0, cells);
    memset(nodes, 0, points);
    int64_t* order = (int64_t*)malloc(cells * sizeof(int64_t));
    for (int64_t c = 0; c < cells; ++c) order[c] = c;
    g_rank_scores = scores;
    qsort(order, cells, sizeof(int64_t), rank_cmp);
    int64_t used = 0;
    const int64_t deltas[4] = {0, 1, resolution, (int64_t)resolution + 1};
    for (int64_t r = 0; r < cells; ++r) {
        const int64_t cell = order[r];
        int64_t added[4]; int nadded = 0;
        for (int d = 0; d < 4; ++d) {
            const int64_t node = (cell + deltas[d]) % points;
            int dup = 0;
            for (int a = 0; a < nadded; ++a) dup |= added[a] == node;
            if (!nodes[node] && !dup) added[nadded++] = node;
        }
        if (used + nadded <= cap) {
            selected[cell] = 1;
            for (int a = 0; a < nadded; ++a) nodes[added[a]] = 1;
            used += nadded;
        }
    }
    free(order);
    return cells;
}

/* ------------------------------------------------------------------ tiles */
/* Tile top-k selection (the allocation benchmark; no reference counterpart).
 * Per-tile residual: per tile row, the fp64 sum in raster order of the
 * per-pixel (fp64(d0^2)+fp64(d1^2))+fp64(d2^2))/3 with fp32 d = pred - u8/255
 * (the a17 pixel rule); then the fp64 sum of the row sums in row order (rows
 * below the image count as 0).  Ranking: descending score, ascending tile id. */
void oracle_tile_scores(const float* prediction, const uint8_t* target, int height, int width, int tile,
                        double* scores) {
    const int tx = (width + tile - 1) / tile, ty = (height + tile - 1) / tile;
    for (int t = 0; t < tx * ty; ++t) {
        const int x0 = (t % tx) * tile, y0 = (t / tx) * tile;
        const int x1 = x0 + tile < width ? x0 + tile : width;
        double total = 0.0;
        for (int r = 0; r < tile; ++r) {
            const int y = y0 + r;
            double sum = 0.0;
            if (y < height)
                for (int x = x0; x < x1; ++x) {
                    const int64_t p = ((int64_t)y * width + x) * 3;
                    const float d0 = prediction[p] - (float)target[p] / 255.0f;
                    const float d1 = prediction[p + 1] - (float)target[p + 1] / 255.0f;
                    const float d2 = prediction[p + 2] - (float)target[p + 2] / 255.0f;
                    double rgb = (double)(d0 * d0) + (double)(d1 * d1);
                    rgb = rgb + (double)(d2 * d2);
                    sum = sum + rgb / 3.0;
                }
            total = total + sum;
        }
        scores[t] = total;
    }
}
void oracle_topk(const double* scores, int64_t count, int64_t k, int64_t* chosen) {
    int64_t* order = (int64_t*)malloc(count * sizeof(int64_t));
    for (int64_t c = 0; c < count; ++c) order[c] = c;
    g_rank_scores = scores;
    qsort(order, count, sizeof(int64_t), rank_cmp);
    for (int64_t i = 0; i < k && i < count; ++i) chosen[i] = order[i];
    free(order);
}

/* ------------------------------------------------------------------ router */
/* Top-1 expert router (routed experts; no reference counterpart).
 * Input fp16 features [n x in_width]; weights fp16 row-major [out][in];
 * each layer: fp32 accumulation in ascending input order with fmaf, ReLU on
 * hidden layers, fp16 rounding of every layer's output.  Coordinate i chooses
 * among the `live` logits starting at row first[i] (first NULL: row 0): choice =
 * argmax of those fp16 logits relative to first[i] (lowest index on ties);
 * prob = softmax of the fp32 values of those fp16 logits, in the order: max,
 * then sum of expf(z - max) in ascending order, then 1 / sum.  logits_out:
 * every row's fp16 logit, [n][out_width]. */
void oracle_router(const uint16_t* x, int64_t n, int in_width, const uint16_t* w1, int hidden,
                   const uint16_t* w2, const uint16_t* w3, int out_width, const int32_t* first, int live,
                   int32_t* expert, float* prob, uint16_t* logits_out) {
    float h1[256], h2[256], z[256];
    for (int64_t i = 0; i < n; ++i) {
        for (int o = 0; o < hidden; ++o) {
            float acc = 0.0f;
            for (int k = 0; k < in_width; ++k)
                acc = fmaf(f_of_h(h_of_bits(w1[o * in_width + k])), f_of_h(h_of_bits(x[i * in_width + k])), acc);
            h1[o] = f_of_h(h_of(acc > 0.0f ? acc : 0.0f));
        }
        for (int o = 0; o < hidden; ++o) {
            float acc = 0.0f;
            for (int k = 0; k < hidden; ++k) acc = fmaf(f_of_h(h_of_bits(w2[o * hidden + k])), h1[k], acc);
            h2[o] = f_of_h(h_of(acc > 0.0f ? acc : 0.0f));
        }
        for (int o = 0; o < out_width; ++o) {
            float acc = 0.0f;
            for (int k = 0; k < hidden; ++k) acc = fmaf(f_of_h(h_of_bits(w3[o * hidden + k])), h2[k], acc);
            z[o] = f_of_h(h_of(acc));
            if (logits_out) logits_out[i * out_width + o] = bits_of_h(h_of(acc));
        }
        const float* zl = z + (first ? first[i] : 0);
        int best = 0;
        for (int e = 1; e < live; ++e) if (zl[e] > zl[best]) best = e;
        float sum = 0.0f;
        for (int e = 0; e < live; ++e) sum += expf(zl[e] - zl[best]);
        expert[i] = best;
        prob[i] = 1.0f / sum;
    }
}

/* ------------------------------------------------------------------ on-demand allocation (the allocation benchmark) */
/* Per-level cell visibility from a tile mask (no reference counterpart): cell (ix, iy) of a level
 * of resolution res is visible iff the pixel nearest its centre, column
 * floor(ix * (width - 1) / (res - 1) + 0.5) (exact in int64), row likewise, lies in an allocated
 * tile_px x tile_px tile.  Bits LSB-first, res^2 cells padded to whole bytes. */
void oracle_allocation_bitmap(const uint8_t* tiles, int tiles_x, int tiles_y, int tile_px, int height, int width,
                              int res, uint8_t* bitmap) {
    const int64_t cells = (int64_t)res * res;
    memset(bitmap, 0, (size_t)((cells + 7) / 8));
    for (int64_t c = 0; c < cells; ++c) {
        const int64_t ix = c % res, iy = c / res;
        const int64_t den = res > 1 ? res - 1 : 1;
        const int64_t col = (2 * ix * (width - 1) + den) / (2 * den), row = (2 * iy * (height - 1) + den) / (2 * den);
        int64_t tx = col / tile_px, ty = row / tile_px;
        if (tx >= tiles_x) tx = tiles_x - 1;
        if (ty >= tiles_y) ty = tiles_y - 1;
        if (tiles[ty * tiles_x + tx]) bitmap[c >> 3] |= (uint8_t)(1u << (c & 7));
    }
}

/* ------------------------------------------------------------------ fp32 hash grid */
/* The single fp32 hash grid with an fp32 MLP (the hash-grid encoding of odie/hash_grid.py:8-80 and the
 * layout of odie/config.py:83-94, in fp32; the library's hashgrid32 kernels): 16 levels x 2 features,
 * MLP 32 -> 64 -> 64 -> 3 without biases ([out][in] weights W1 | W2 | W3), ReLU hidden layers, sigmoid
 * output.  Every dot product is one fmaf chain in ascending input order starting from zero. */

/* Bilinear sample of an fp32 [height][width][3] image at (x, y): p = fl(x (W - 1)), corner
 * min(trunc(p), W - 2), f = p - corner, weights (1-fx)(1-fy), fx(1-fy), (1-fx)fy, fx fy, sum
 * w00 c00 then fmaf with the (1,0), (0,1), (1,1) corners. */
void oracle_hg32_bilinear(const float* image, int width, int height, const float* xy, int64_t n, float* target) {
    for (int64_t i = 0; i < n; ++i) {
        const float px = xy[2 * i] * (float)(width - 1), py = xy[2 * i + 1] * (float)(height - 1);
        int x0 = (int)px, y0 = (int)py;
        x0 = x0 < 0 ? 0 : (x0 > width - 2 ? width - 2 : x0);
        y0 = y0 < 0 ? 0 : (y0 > height - 2 ? height - 2 : y0);
        const float fx = px - (float)x0, fy = py - (float)y0, gx = 1.0f - fx, gy = 1.0f - fy;
        const float w00 = gx * gy, w10 = fx * gy, w01 = gx * fy, w11 = fx * fy;
        const float* p00 = image + 3 * ((int64_t)y0 * width + x0);
        const float* p01 = p00 + 3 * (int64_t)width;
        for (int c = 0; c < 3; ++c) {
            float s = w00 * p00[c];
            s = fmaf(w10, p00[3 + c], s);
            s = fmaf(w01, p01[c], s);
            target[3 * i + c] = fmaf(w11, p01[3 + c], s);
        }
    }
}

/* fp32 features [n][2 levels]: per level the 4 corners' pairs, fmaf chain over the corners from zero. */
void oracle_hg32_features(const float* xy, int64_t n, const float* grid, const HashLevel* lv, int levels, float* f) {
    for (int64_t i = 0; i < n; ++i)
        for (int l = 0; l < levels; ++l) {
            const HashLevel* h = lv + l;
            const float px = fmaf(h->scale, xy[2 * i], 0.5f), py = fmaf(h->scale, xy[2 * i + 1], 0.5f);
            const int ix = (int)floorf(px), iy = (int)floorf(py);
            const float fx = px - (float)ix, fy = py - (float)iy;
            const float w[4] = {(1.0f - fx) * (1.0f - fy), fx * (1.0f - fy), (1.0f - fx) * fy, fx * fy};
            float a0 = 0.0f, a1 = 0.0f;
            for (int k = 0; k < 4; ++k) {
                const uint32_t idx = hash_index(h, ix + (k & 1), iy + (k >> 1));
                a0 = fmaf(w[k], grid[h->offset + 2 * (int64_t)idx], a0);
                a1 = fmaf(w[k], grid[h->offset + 2 * (int64_t)idx + 1], a1);
            }
            f[i * 2 * levels + 2 * l] = a0;
            f[i * 2 * levels + 2 * l + 1] = a1;
        }
}

/* Forward and backward of one batch: h1 = relu(W1 f), h2 = relu(W2 h1), z = W3 h2, y = 1 / (1 + e^-z),
 * d = y - t, squares = fmaf chain of d^2 / 3, dz = ((s d) y)(1 - y) with s the loss scale (2 / 3n),
 * dh2 = (fl(W3[0] dz0) then fmaf over the outputs) masked by h2 > 0, dh1 = (W2^T dh2) masked by h1 > 0,
 * dx = W1^T dh1.  Arrays are row-major per coordinate. */
void oracle_hg32_step(const float* f, const float* target, int64_t n, const float* w, float loss_scale, float* h1,
                      float* h2, float* z, float* y, float* dz, float* squares, float* dh2, float* dh1, float* dx) {
    const float* w1 = w;
    const float* w2 = w + 64 * 32;
    const float* w3 = w2 + 64 * 64;
    for (int64_t i = 0; i < n; ++i) {
        const float* fi = f + i * 32;
        float* a = h1 + i * 64;
        float* b = h2 + i * 64;
        for (int o = 0; o < 64; ++o) {
            float s = 0.0f;
            for (int m = 0; m < 32; ++m) s = fmaf(w1[o * 32 + m], fi[m], s);
            a[o] = s > 0.0f ? s : 0.0f;
        }
        for (int o = 0; o < 64; ++o) {
            float s = 0.0f;
            for (int j = 0; j < 64; ++j) s = fmaf(w2[o * 64 + j], a[j], s);
            b[o] = s > 0.0f ? s : 0.0f;
        }
        float sq = 0.0f;
        for (int c = 0; c < 3; ++c) {
            float s = 0.0f;
            for (int j = 0; j < 64; ++j) s = fmaf(w3[c * 64 + j], b[j], s);
            z[3 * i + c] = s;
            const float yc = 1.0f / (1.0f + expf(-s));
            const float d = yc - target[3 * i + c];
            sq = fmaf(d, d, sq);
            y[3 * i + c] = yc;
            dz[3 * i + c] = ((loss_scale * d) * yc) * (1.0f - yc);
        }
        squares[i] = sq / 3.0f;
        float* g2 = dh2 + i * 64;
        float* g1 = dh1 + i * 64;
        const float* d = dz + 3 * i;
        for (int j = 0; j < 64; ++j) {
            float s = w3[j] * d[0];
            s = fmaf(w3[64 + j], d[1], s);
            s = fmaf(w3[128 + j], d[2], s);
            g2[j] = b[j] > 0.0f ? s : 0.0f;
        }
        for (int j = 0; j < 64; ++j) {
            float s = 0.0f;
            for (int k = 0; k < 64; ++k) s = fmaf(w2[k * 64 + j], g2[k], s);
            g1[j] = a[j] > 0.0f ? s : 0.0f;
        }
        for (int m = 0; m < 32; ++m) {
            float s = 0.0f;
            for (int j = 0; j < 64; ++j) s = fmaf(w1[j * 32 + m], g1[j], s);
            dx[i * 32 + m] = s;
        }
    }
}
