// Launchers of the grid-encoding kernels (encode.cu).
#pragma once
#include "common.cuh"

namespace odie {

// Level table passed to the kernels by value (__grid_constant__): no device
// allocation is needed to describe a layout.
struct LevelTable {
    Level level[MAX_LEVELS];
};

// Where the levels come from: the reference's int32 descriptor rows in device
// memory (packed planes, odie/model.py:100-101) or a LevelTable.
struct LevelSource {
    const int* descriptors = nullptr;  // device [levels][8] when non-null
    LevelTable table;                  // used when descriptors is null
};

struct EncodeArgs {
    const float* coords = nullptr;          // [n][2] fp32
    long long n = 0;
    int levels = 0, active = 0;
    const uint64_t* node_bitmap = nullptr;  // packed planes
    const int* node_prefix = nullptr;
    const uint8_t* bitmap = nullptr;        // cell visibility bitmaps
    // row-major [n][width] halves (module path) or pair-major [width/2][stride] half2
    bool row_major = true;
    int width = 0;
    long long stride = 0;
    // Routed experts: coordinate i reads and updates the table of expert
    // expert[i], which starts expert[i] * expert_stride parameters after the
    // level offsets (every expert has the same level layout).  Null: one table.
    const int* expert = nullptr;
    long long expert_stride = 0;
    int experts = 1;  // number of expert tables (expert ids are < experts)
    // One device int the backward may use to choose its scatter strategy on the device from the batch itself
    // (spatially coherent batches: global reductions; incoherent ones: per-block shared-memory tables).  Null:
    // the shared-memory tables always.  Calls that may run concurrently need distinct ints.
    int* strategy = nullptr;
};

// Forward: table is fp32 (master) or fp16 (mirror); vis may be null.
void launch_encode_forward(const EncodeArgs& a, const LevelSource& src, const float* table32, const __half* table16,
                           __half* out, uint8_t* vis, cudaStream_t stream);
// Backward: scatter-add w_k * upstream into grad (fp32).  Coordinates are
// visited in a fixed scrambled order; small levels accumulate per block in
// shared memory first.
void launch_encode_backward(const EncodeArgs& a, const LevelSource& src, const __half* upstream, float* grad,
                            cudaStream_t stream);
// The same with fp32 values (the fp32 hash grid's feature gradients, row-major).
void launch_encode_backward(const EncodeArgs& a, const LevelSource& src, const float* upstream, float* grad,
                            cudaStream_t stream);

}  // namespace odie
