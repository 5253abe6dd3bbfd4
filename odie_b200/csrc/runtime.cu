// Training runtime behind the odie_* C-ABI (the reference's Probe,
// odie/native/runtime.cu:163-317, re-designed for B200).
//
// Ownership follows the reference: the caller owns the target image, the fp32
// grid master and the fp32 head masters (updated in place); the library owns
// gradients, fp16 copies, Adam state, per-batch activations and scratch.
// One step on one stream, every launch capturable in a CUDA graph (no host
// synchronisation, no allocation after creation):
//   input_batch -> encode forward (fp16 mirror gather) -> fused MLP heads
//   (gate, decoder, loss, backward, weight-gradient partials) -> encode
//   backward (scatter) -> partial reduction -> Adam (grid, gate, decoder).
// Routed experts ("experts" in the settings; no reference counterpart): the
// router grid is encoded first, router.cu picks one expert per coordinate, the
// expert tables are encoded at that expert's offset, and the fused heads train
// router and decoder together; both grids take the scatter and the Adam step.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <memory>
#include <sstream>
#include <vector>

#include "encode.cuh"
#include "odie_b200.h"
#include "json_lite.hpp"
#include "router.cuh"
#include "step.cuh"

namespace odie {

namespace {
thread_local std::string g_error, g_reply;
}

void set_error(const std::string& message) { g_error = message; }

namespace {
std::atomic<long long> g_launches{0};
}
void note_launch(int kernels) { g_launches.fetch_add(kernels, std::memory_order_relaxed); }

int sm_count() {
    static int cached[64] = {0};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
    if (!cached[device]) {
        int count = 0;
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || count <= 0) count = 148;
        cached[device] = count;
    }
    return cached[device];
}

// TCNN-style HashGrid layout restated from odie/config.py:83-94; returns the parameter count.
long long hash_grid_table(const Json& enc, LevelTable& table, int& levels, int& F) {
    levels = int(enc.at("n_levels").as_int());
    F = int(enc.at("n_features_per_level").as_int());
    const int log2t = int(enc.at("log2_hashmap_size").as_int());
    const int base = int(enc.at("base_resolution").as_int());
    const double growth = double(float(enc.at("per_level_scale").as_double()));
    ODIE_REQUIRE(levels >= 2 && levels <= 16, "hash grid levels in [2, 16]");
    ODIE_REQUIRE(F == 1 || F == 2 || F == 4, "hash grid features per level must be 1, 2 or 4");
    ODIE_REQUIRE(levels * F <= 32, "the fused heads take at most 32 input features");
    const float log_growth = float(std::log2(growth));
    long long offset = 0;
    for (int l = 0; l < levels; ++l) {
        const float e = float(double(l) * double(log_growth));
        const float p = float(std::pow(2.0, double(e)));
        const float scale = float(double(float(double(p) * double(base))) - 1.0);
        const int res = int(std::ceil(double(scale))) + 1;
        const long long dense = ((long long)res * res + 7) / 8 * 8;
        const long long cap = std::min(dense, 1LL << log2t);
        Level& L = table.level[l];
        L.scale = scale;
        L.res = res;
        L.points = int(cap);
        L.offset = int(offset);
        L.words = -1;
        L.cells = -1;
        L.F = F;
        L.col = l * F;
        L.kind = (long long)res * res > cap ? HASH_HASHED : HASH_DENSE;
        offset += cap * F;
    }
    return offset;
}

template <typename T>
T* pointer_of(const Json& j, const char* key) {
    return reinterpret_cast<T*>(j.at(key).as_u64());
}

constexpr double BETA1 = 0.9, BETA2 = 0.999, EPS = 1e-15;
constexpr long long TABLE_STEPS = 1LL << 22;  // Adam bias-correction tables (steps per parameter)

struct Runtime {
    cudaStream_t stream = nullptr;
    // Routed experts: the router-grid scatter runs on a second stream, concurrently with the
    // expert-table scatter (fork/join by events, so a captured graph keeps both branches).
    cudaStream_t side = nullptr;
    cudaEvent_t fork_event = nullptr, join_event = nullptr;
    // Pipeline mode ("pipeline": 1; routed experts with library-owned gradients, i.e. one GPU): a training step
    // (odie_step / odie_step_stratified with update) leaves the two branches of its backward running on the
    // runtime's own streams -- the router-grid scatter, the head-gradient reduction and the router grid's and
    // heads' Adam on `side`; the expert-table scatter and the expert tables' Adam on `tail` -- and returns.  The
    // next step's input kernel starts at once; its router-grid gather and router forward wait only for the side
    // branch (whose updates they read) and run while the tail still scatters; its expert gather waits for the
    // tail.  Coordinates, targets and expert ids alternate between two buffers, so that a step never overwrites
    // what the previous step's branches still read.  The step's forward and heads run on `front`, a stream of the
    // device's highest priority (as is `side`, on the next step's critical path), so that the block scheduler
    // gives them the SMs the tail frees rather than the tail's next blocks; the runtime's stream orders `front`
    // after the caller's work (call_event) and waits for the heads (heads_done), so the step's loss is in the
    // caller's stream order.  Every other call first makes the runtime's stream wait for both branches (join),
    // as odie_join does; until then the parameters may still be changing.
    bool pipeline = false, pending = false;
    cudaStream_t tail = nullptr, front = nullptr;
    cudaEvent_t heads_done = nullptr, side_done = nullptr, tail_done = nullptr, call_event = nullptr;
    int device = 0;
    long long total = 0, capacity = 65536;
    int image_width = 0, image_height = 0, mode = 0, warp_limit = 128;
    int levels = 16, raw_width = 32, input_width = 32, gate_k = 0, active = 16;
    bool router = true, softplus = false, rgb8 = true, hash_mode = false;
    bool uniform = true;   // every level F=2 at columns (2l, 2l+1)
    // routed experts: `experts` tables of expert_total parameters each, plus the router grid
    int experts = 0;
    long long expert_total = 0, router_total = 0;
    int router_levels = 0, router_width = 0;
    LevelTable router_table{};
    float* router_grid = nullptr;  // caller-owned fp32 master of the router grid
    Banding banding;               // spatial expert ownership (router.cuh)
    int live = 16;                 // router logits kept per coordinate for the heads' backward
    RowFrame frame;                // this image's rows within the full image (coordinates are the full image's)
    // Caller-owned router-grid gradient (data-parallel training: the router grid is shared, its gradient is
    // summed across ranks before its update, which then runs in step_heads); null: library-owned.
    float* external_router_grad = nullptr;
    double lr[3] = {1e-2, 1e-3, 1e-3};  // grid, gate, decoder
    double uploaded_lr[3] = {-1.0, -1.0, -1.0};  // the rates the device step tables hold (-1: none yet)
    // caller-owned
    float* grid = nullptr;
    const uint8_t* rgb = nullptr;
    float* gate_master = nullptr;
    float* decoder_master = nullptr;
    const int* descriptors = nullptr;
    const uint64_t* node_bitmap = nullptr;
    const int* node_prefix = nullptr;
    const uint8_t* cell_bitmap = nullptr;
    float* external_head_grad = nullptr;
    // layout
    LevelTable table{};
    FeatureMap fmap{};
    int gate_count = 0, decoder_count = 0, head_count = 0;
    // library-owned
    DeviceArray<__half> grid_half, head_half;
    DeviceArray<float> grid_grad, grid_m, grid_v, head_grad_own, head_m, head_v, partials;
    DeviceArray<uint32_t> grid_steps, head_steps;
    DeviceArray<float> table_bc2, table_step[3];
    DeviceArray<float> xy, target, squares;
    DeviceArray<__half> raw, gvals;
    DeviceArray<uint32_t> vis;
    DeviceArray<int> error_flag;
    // the backward scatters' strategy ints (EncodeArgs::strategy): [0] the router grid's (side stream), [1] the
    // main stream's
    DeviceArray<int> scatter_strategy;
    DeviceArray<__half> router_half, router_in, router_gvals;
    DeviceArray<float> router_grad, router_m, router_v, prob;
    DeviceArray<uint32_t> router_steps;
    DeviceArray<int> expert_ids;
    DeviceArray<float> xy_alt, target_alt;  // pipeline mode: the second buffers
    DeviceArray<int> expert_ids_alt;
    DeviceArray<__half> logits;
    std::vector<double> host_bc1, host_bc2;
    int partial_blocks = 0;

    float* head_grad() { return external_head_grad ? external_head_grad : head_grad_own.ptr; }
    float* router_gradient() { return external_router_grad ? external_router_grad : router_grad.ptr; }
    GateMode gate_mode() const { return experts ? GATE_EXPERTS : router ? GATE_LEVELS : GATE_NONE; }

    explicit Runtime(const Json& j) {
        ODIE_CUDA(cudaGetDevice(&device));
        stream = reinterpret_cast<cudaStream_t>(j.at("stream").as_u64());
        total = j.at("total").as_int();
        image_width = int(j.at("width").as_int());
        image_height = int(j.at("height").as_int());
        // The reference's mode bits (odie/native/runtime.cu:93-143,256): 1 fused target, 4 half-precision grid
        // gradients, 8 dirty-tile gradient clearing, 16 parallel gate.  Each names a path this runtime always
        // takes or supersedes: the target is read inside the input kernel (1); the gate runs fused into the heads
        // kernel (16); grid gradients accumulate in fp32 (4 asks for fp16 to halve the reference's atomic traffic;
        // fp32 keeps the reference's fp32-path precision) and Adam clears exactly the entries it consumed, so no
        // per-step clearing pass exists to restrict to dirty tiles (8).  Any other bit is rejected.
        mode = int(j.value("mode", 20));
        ODIE_REQUIRE((mode & ~(1 | 4 | 8 | 16)) == 0, "mode: only the reference's bits 1, 4, 8 and 16 are defined");
        // The reference's warp-aggregation threshold; accepted for its JSON contract.  The scatter here
        // needs no threshold: it spreads equal addresses apart by its visiting order instead.
        warp_limit = int(j.value("warp_limit", 128));
        // coordinate capacity per step, padded to whole 128-row tiles (the feature stride)
        capacity = (j.value("batch", 65536) + 127) / 128 * 128;
        router = j.value("router", 1) != 0;
        gate_k = int(j.value("gate_k", 0));
        softplus = j.value("softplus", 0) != 0;
        rgb8 = j.value("rgb8", 1) != 0;
        // the full image's rows (coordinates y = (row_offset + row) / (full_height - 1)); default: this image
        frame.row0 = int(j.value("row_offset", 0));
        frame.rows = int(j.value("full_height", image_height));
        ODIE_REQUIRE(frame.row0 >= 0 && frame.rows >= 2 && (long long)frame.row0 + image_height <= frame.rows,
                     "row_offset + height must not exceed full_height");
        ODIE_REQUIRE(total > 0 && total <= 0x7fffffffLL, "total must fit int32 addressing");
        ODIE_REQUIRE(image_width >= 2 && image_height >= 2, "image axes must be >= 2");
        ODIE_REQUIRE(capacity >= 1 && capacity <= (1LL << 26), "batch capacity must be in [1, 2^26]");
        grid = pointer_of<float>(j, "grid");
        rgb = pointer_of<uint8_t>(j, "rgb");
        decoder_master = pointer_of<float>(j, "decoder");
        if (router) gate_master = pointer_of<float>(j, "gate");
        if (j.contains("head_grad")) external_head_grad = pointer_of<float>(j, "head_grad");
        hash_mode = j.contains("hash_encoding");
        experts = int(j.value("experts", 0));
        if (experts) {
            ODIE_REQUIRE(experts >= 1 && experts <= ROUTER_MAX_OUT, "experts must be within 1..64");
            ODIE_REQUIRE(hash_mode && j.contains("router_encoding"), "routed experts need hash_encoding and router_encoding");
            banding.bands = int(j.value("bands", 1));
            banding.first_band = int(j.value("first_band", 0));
            banding.per_band = int(j.value("experts_per_band", experts));
            banding.rows = frame.rows;
            check_banding(banding, experts);
            live = banding.per_band <= 8 ? 8 : 16;
            if (j.contains("router_grad")) external_router_grad = pointer_of<float>(j, "router_grad");
            router = false;
            gate_master = pointer_of<float>(j, "gate");
            router_grid = pointer_of<float>(j, "router_grid");
            int rf = 0;
            router_total = hash_layout(j.at("router_encoding"), router_table, router_levels, rf);
            router_width = (router_levels * rf + 15) / 16 * 16;
        }
        pipeline = j.value("pipeline", 0) != 0;
        ODIE_REQUIRE(!pipeline || (experts && !external_head_grad && !external_router_grad),
                     "pipeline mode needs routed experts with library-owned head and router-grid gradients");
        if (hash_mode) build_hash_table(j.at("hash_encoding"));
        else levels = int(j.value("levels", 16));
        if (experts) ODIE_REQUIRE(router_width == input_width && input_width == 32,
                                  "router and expert encodings must both give 32 features");
        ODIE_REQUIRE(levels >= 2 && levels <= 16, "the fused heads support 2..16 levels");
        ODIE_REQUIRE(gate_k >= 0 && gate_k <= levels, "gate_k outside [0, levels]");
        active = levels;
        for (int g = 0; g < 3; ++g) lr[g] = 0.0;
        host_bc1.resize(TABLE_STEPS);
        host_bc2.resize(TABLE_STEPS);
        for (long long s = 0; s < TABLE_STEPS; ++s) {
            host_bc1[s] = 1.0 - std::pow(BETA1, double(s + 1));
            host_bc2[s] = 1.0 - std::pow(BETA2, double(s + 1));
        }
        table_bc2.allocate(TABLE_STEPS);
        for (int g = 0; g < 3; ++g) table_step[g].allocate(TABLE_STEPS);
        {
            std::vector<float> bc2(TABLE_STEPS);
            for (long long s = 0; s < TABLE_STEPS; ++s) bc2[s] = float(std::sqrt(host_bc2[s]));
            ODIE_CUDA(cudaMemcpy(table_bc2.ptr, bc2.data(), TABLE_STEPS * sizeof(float), cudaMemcpyHostToDevice));
        }
        configure(j);
        gate_count = router ? gate_params(input_width)
                            : experts ? router_params(input_width, router_out(banding.model_experts())) : 0;
        decoder_count = decoder_params(input_width);
        head_count = gate_count + decoder_count;
        // library-owned buffers
        grid_half.allocate(total);
        grid_grad.allocate(total);
        grid_m.allocate(total);
        grid_v.allocate(total);
        grid_steps.allocate(total);
        head_half.allocate(head_count);
        head_grad_own.allocate(head_count);
        head_m.allocate(head_count);
        head_v.allocate(head_count);
        head_steps.allocate(head_count);
        partial_blocks = mlp_tc_blocks(capacity);
        partials.allocate((long long)partial_blocks * head_count);
        xy.allocate(2 * capacity);
        target.allocate(3 * capacity);
        squares.allocate(capacity);
        raw.allocate((long long)input_width * capacity);
        gvals.allocate((long long)input_width * capacity);
        vis.allocate((long long)levels * capacity / 32);  // bit-packed [levels][capacity / 32]
        error_flag.allocate(1);
        scatter_strategy.allocate(2);
        scatter_strategy.zero(stream);
        if (experts) {
            int least = 0, greatest = 0;
            ODIE_CUDA(cudaDeviceGetStreamPriorityRange(&least, &greatest));
            ODIE_CUDA(cudaStreamCreateWithPriority(&side, cudaStreamNonBlocking, pipeline ? greatest : least));
            ODIE_CUDA(cudaEventCreateWithFlags(&fork_event, cudaEventDisableTiming));
            ODIE_CUDA(cudaEventCreateWithFlags(&join_event, cudaEventDisableTiming));
            if (pipeline) {
                ODIE_CUDA(cudaStreamCreateWithPriority(&front, cudaStreamNonBlocking, greatest));
                ODIE_CUDA(cudaStreamCreateWithPriority(&tail, cudaStreamNonBlocking, least));
                for (cudaEvent_t* e : {&heads_done, &side_done, &tail_done, &call_event})
                    ODIE_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
                xy_alt.allocate(2 * capacity);
                target_alt.allocate(3 * capacity);
                expert_ids_alt.allocate(capacity);
                expert_ids_alt.zero(stream);
            }
            router_half.allocate(router_total);
            router_grad.allocate(router_total);
            router_m.allocate(router_total);
            router_v.allocate(router_total);
            router_steps.allocate(router_total);
            router_in.allocate((long long)router_width * capacity);
            router_gvals.allocate((long long)router_width * capacity);
            prob.allocate(capacity);
            expert_ids.allocate(capacity);
            logits.allocate((long long)live * capacity);
            logits.zero(stream);
            if (external_router_grad)
                ODIE_CUDA(cudaMemsetAsync(external_router_grad, 0, size_t(router_total) * sizeof(float), stream));
            for (auto* a : {&router_grad, &router_m, &router_v, &prob}) a->zero(stream);
            router_steps.zero(stream);
            router_in.zero(stream);
            router_gvals.zero(stream);
            expert_ids.zero(stream);
        }
        for (auto* a : {&grid_grad, &grid_m, &grid_v, &head_grad_own, &head_m, &head_v})
            a->zero(stream);
        grid_steps.zero(stream);
        head_steps.zero(stream);
        raw.zero(stream);
        gvals.zero(stream);
        squares.zero(stream);
        error_flag.zero(stream);
        sync_weights();
        ODIE_CUDA(cudaStreamSynchronize(stream));
    }

    static long long hash_layout(const Json& enc, LevelTable& table, int& levels, int& F) {
        return hash_grid_table(enc, table, levels, F);
    }

    void build_hash_table(const Json& enc) {
        int F = 0;
        expert_total = hash_layout(enc, table, levels, F);
        if (experts) {
            ODIE_REQUIRE(expert_total * experts == total, "total must equal experts x the expert grid's parameters");
            check_router_total();
        } else {
            ODIE_REQUIRE(expert_total == total, "hash grid allocation differs from the resolved layout total");
        }
        raw_width = levels * F;
        input_width = (raw_width + 15) / 16 * 16;
        build_feature_map();
    }

    void check_router_total() const {
        ODIE_REQUIRE(router_total > 0 && router_total <= 0x7fffffffLL, "router grid must fit int32 addressing");
    }

    void build_feature_map() {
        uniform = raw_width == 2 * levels;
        for (int l = 0; l < levels; ++l) uniform = uniform && table.level[l].F == 2 && table.level[l].col == 2 * l;
        std::memset(&fmap, 0, sizeof(fmap));
        for (int c = 0; c < 64; ++c) fmap.level_of_col[c] = -1;
        for (int l = 0; l < levels; ++l) {
            const Level& L = table.level[l];
            fmap.col_of_level[l] = int8_t(L.col);
            fmap.dim_of_level[l] = int8_t(L.F);
            for (int c = L.col; c < L.col + L.F; ++c) fmap.level_of_col[c] = int8_t(l);
        }
    }

    void configure(const Json& j) {
        join();
        active = int(j.at("active").as_int());
        ODIE_REQUIRE(active >= 2 && active <= levels, "invalid active prefix");
        if (!hash_mode) {
            descriptors = pointer_of<const int>(j, "descriptors");
            node_bitmap = pointer_of<const uint64_t>(j, "node_bitmap");
            node_prefix = pointer_of<const int>(j, "node_prefix");
            cell_bitmap = pointer_of<const uint8_t>(j, "bitmap");
            std::vector<int> host(levels * 8);
            ODIE_CUDA(cudaMemcpy(host.data(), descriptors, host.size() * sizeof(int), cudaMemcpyDeviceToHost));
            int width = 0;
            for (int l = 0; l < levels; ++l) {
                const int* d = host.data() + 8 * l;
                Level& L = table.level[l];
                L.scale = float(d[0] - 1);
                L.res = d[0];
                L.points = d[1];
                L.offset = d[2];
                L.words = d[7] ? -1 : d[3];
                L.cells = d[4];
                L.F = d[5];
                L.col = d[6];
                L.kind = PLANE;
                ODIE_REQUIRE(L.F == 1 || L.F == 2 || L.F == 4, "plane features must be 1, 2 or 4");
                width = std::max(width, L.col + L.F);
            }
            raw_width = width;
            input_width = (raw_width + 15) / 16 * 16;
            ODIE_REQUIRE(input_width <= 32, "the fused heads take at most 32 input features (16 levels x F2)");
            build_feature_map();
        }
        if (experts && j.contains("allocation")) {
            // on-demand allocation of the expert tables: {"bitmap": device pointer, "cells": per-level byte offsets,
            // -1 for a level whose cells are all visible}; every expert shares the levels' visibility
            const Json& alloc = j.at("allocation");
            cell_bitmap = pointer_of<const uint8_t>(alloc, "bitmap");
            const Json& list = alloc.at("cells");
            ODIE_REQUIRE(list.type == Json::ARRAY, "allocation cells must be a list");
            const auto& cells = list.items;
            ODIE_REQUIRE(int(cells.size()) == levels, "allocation needs one cell offset per expert level");
            for (int l = 0; l < levels; ++l) {
                table.level[l].cells = int(cells[l].as_int());
                ODIE_REQUIRE(table.level[l].cells < 0 || cell_bitmap, "allocation offsets need a bitmap");
            }
        }
        lr[0] = j.at("grid_lr").as_double();
        if (router || experts) lr[1] = j.at("gate_lr").as_double();
        lr[2] = j.at("decoder_lr").as_double();
        upload_step_tables();
        if (grid_half.count) sync_weights();
    }

    // The per-step learning-rate tables (16 MB each); rebuilt only for a group whose rate changed, so a
    // reconfiguration that changes the layout or the allocation costs no table upload.
    void upload_step_tables() {
        std::vector<float> host;
        for (int g = 0; g < 3; ++g) {
            if (!table_step[g].ptr || uploaded_lr[g] == lr[g]) continue;
            host.resize(TABLE_STEPS);
            for (long long s = 0; s < TABLE_STEPS; ++s) host[s] = float(lr[g] / host_bc1[s]);
            ODIE_CUDA(cudaMemcpy(table_step[g].ptr, host.data(), TABLE_STEPS * sizeof(float), cudaMemcpyHostToDevice));
            uploaded_lr[g] = lr[g];
        }
    }

    void sync_weights() {
        join();
        launch_cast_half(grid, grid_half.ptr, total, stream);
        if (experts) launch_cast_half(router_grid, router_half.ptr, router_total, stream);
        if (gate_count) launch_cast_half(gate_master, head_half.ptr, gate_count, stream);
        launch_cast_half(decoder_master, head_half.ptr + gate_count, decoder_count, stream);
        ODIE_CUDA(cudaGetLastError());
    }

    EncodeArgs encode_args(long long n) const {
        EncodeArgs a;
        a.coords = xy.ptr;
        a.n = n;
        a.levels = levels;
        a.active = active;
        a.node_bitmap = node_bitmap;
        a.node_prefix = node_prefix;
        a.bitmap = cell_bitmap;
        a.row_major = false;
        a.width = input_width;
        a.stride = capacity;
        a.strategy = scatter_strategy.ptr + 1;
        return a;
    }

    MlpArgs mlp_args(long long n) {
        MlpArgs m{};
        m.n = n;
        m.stride = capacity;
        m.raw = raw.ptr;
        m.vis = vis.ptr;
        m.target = target.ptr;
        m.gate_w = gate_count ? head_half.ptr : nullptr;
        m.decoder_w = head_half.ptr + gate_count;
        m.levels = levels;
        m.raw_width = raw_width;
        m.k_fixed = gate_k;
        m.softplus = softplus;
        m.three_real = float(3 * n);
        m.fmap = fmap;
        m.gvals = gvals.ptr;
        m.squares = squares.ptr;
        m.partials = partials.ptr;
        m.router_in = router_in.ptr;
        m.prob = prob.ptr;
        m.expert = expert_ids.ptr;
        m.router_gvals = router_gvals.ptr;
        m.experts = experts;
        m.raw_rows = experts != 0;
        m.logits = logits.ptr;
        m.live = live;
        m.per_band = banding.per_band;
        m.first_band = banding.first_band;
        m.model_experts = banding.model_experts();
        return m;
    }

    // Router-grid features are row-major [capacity][router_width]: the heads kernel copies a
    // coordinate's row into shared memory with 16-byte asynchronous copies.
    EncodeArgs router_encode_args(long long n) const {
        EncodeArgs a = encode_args(n);
        a.levels = router_levels;
        a.active = router_levels;
        a.width = router_width;
        a.row_major = true;
        a.strategy = scatter_strategy.ptr;
        return a;
    }

    // Routed experts, forward part shared by training and decode: router grid
    // features -> expert choice -> the chosen experts' features (raw).
    // before_gather: an event the expert gather waits for (pipeline mode: the previous step's tail), or null;
    // on: the stream of the gathers and the router (default: the runtime's)
    void route_and_encode(long long n, cudaEvent_t before_gather = nullptr, cudaStream_t on = nullptr) {
        const cudaStream_t s = on ? on : stream;
        LevelSource rsrc;
        rsrc.table = router_table;
        int slot = stage_begin(S_ENCODE_FWD);
        launch_encode_forward(router_encode_args(n), rsrc, nullptr, router_half.ptr, router_in.ptr, nullptr, s);
        stage_end(slot);
        RouterArgs ra;
        ra.features = router_in.ptr;
        ra.row_major = true;
        ra.stride = capacity;
        ra.n = n;
        ra.weights = head_half.ptr;
        ra.experts = experts;
        ra.banding = banding;
        ra.xy = xy.ptr;
        ra.expert = expert_ids.ptr;
        ra.prob = prob.ptr;
        ra.logits = logits.ptr;
        ra.live = live;
        slot = stage_begin(S_ROUTER);
        launch_router_forward(ra, router_width, s);
        stage_end(slot);
        LevelSource src;
        src.table = table;
        EncodeArgs ea = encode_args(n);
        ea.expert = expert_ids.ptr;
        ea.expert_stride = expert_total;
        ea.experts = experts;
        ea.row_major = true;  // one row per coordinate: the per-coordinate gather over all levels
        if (before_gather) ODIE_CUDA(cudaStreamWaitEvent(s, before_gather, 0));
        slot = stage_begin(S_ENCODE_FWD);
        launch_encode_forward(ea, src, nullptr, grid_half.ptr, raw.ptr, nullptr, s);
        stage_end(slot);
    }

    // ---- optional stage timers (CUDA events on the runtime's stream; off by default)
    enum Stage { S_INPUT, S_ENCODE_FWD, S_ROUTER, S_MLP, S_ENCODE_BWD, S_REDUCE, S_ADAM_GRID, S_ADAM_HEADS, S_COUNT };
    static constexpr const char* STAGE_NAMES[S_COUNT] = {"input_batch", "encode_forward", "router", "mlp_train",
                                                         "encode_backward", "reduce_partials", "adam_grid", "adam_heads"};
    static constexpr int EVENT_PAIRS = 4096;
    bool profiling = false;
    bool serial = false;  // profiling with both branches of the step on one stream: stage times are kernel times
    std::vector<cudaEvent_t> events;            // 2 per recorded stage launch
    std::vector<int> event_stage;
    int recorded = 0;

    void profile(int mode) {
        join();
        const bool enable = mode != 0;
        serial = mode == 2;
        ODIE_CUDA(cudaStreamSynchronize(stream));
        if (enable && events.empty()) {
            events.resize(2 * EVENT_PAIRS);
            for (auto& e : events) ODIE_CUDA(cudaEventCreate(&e));
            event_stage.assign(EVENT_PAIRS, -1);
        }
        profiling = enable;
        recorded = 0;
    }
    // A stage's events go on the stream its kernels run on (the side stream for the router-grid branch);
    // stage_end must name the same stream as stage_begin.
    int stage_begin(Stage s, cudaStream_t on = nullptr) {
        if (!profiling || recorded >= EVENT_PAIRS) return -1;
        const int slot = recorded++;
        event_stage[slot] = s;
        ODIE_CUDA(cudaEventRecord(events[2 * slot], on ? on : stream));
        return slot;
    }
    void stage_end(int slot, cudaStream_t on = nullptr) {
        if (slot >= 0) ODIE_CUDA(cudaEventRecord(events[2 * slot + 1], on ? on : stream));
    }
    std::string profile_report() {
        join();
        ODIE_CUDA(cudaStreamSynchronize(stream));
        double ms[S_COUNT] = {0};
        int launches[S_COUNT] = {0};
        for (int i = 0; i < recorded; ++i) {
            float t = 0.0f;
            ODIE_CUDA(cudaEventElapsedTime(&t, events[2 * i], events[2 * i + 1]));
            ms[event_stage[i]] += t;
            launches[event_stage[i]] += 1;
        }
        std::ostringstream o;
        o << "{";
        for (int s = 0; s < S_COUNT; ++s)
            o << (s ? "," : "") << "\"" << STAGE_NAMES[s] << "\":{\"launches\":" << launches[s] << ",\"ms\":" << ms[s] << "}";
        o << "}";
        return o.str();
    }

    // sampled: the batch is the stratified sampler's (seed, step) instead of the caller's ids
    struct Sampled {
        uint64_t seed, step;
    };
    // pipeline mode: the runtime's stream waits for the branches the last step left running
    void join() {
        if (!pending) return;
        ODIE_CUDA(cudaStreamWaitEvent(stream, side_done, 0));
        ODIE_CUDA(cudaStreamWaitEvent(stream, tail_done, 0));
        pending = false;
    }

    // One training step with update in pipeline mode (see `pipeline`).
    void step_pipelined(const int64_t* ids, int n, const Sampled* sampled) {
        ODIE_REQUIRE(n > 0 && n <= capacity, "invalid batch size for this runtime");
        // the forward comes after the caller's work (its ids); from the router-grid gather on, also after the
        // previous step's side branch, whose router-grid and head updates it reads
        ODIE_CUDA(cudaEventRecord(call_event, stream));
        ODIE_CUDA(cudaStreamWaitEvent(front, call_event, 0));
        std::swap(xy.ptr, xy_alt.ptr);
        std::swap(target.ptr, target_alt.ptr);
        std::swap(expert_ids.ptr, expert_ids_alt.ptr);
        if (sampled)
            launch_stratified_batch(sampled->seed, sampled->step, n, rgb, rgb8, image_width, image_height, frame, xy.ptr,
                                    target.ptr, front);
        else
            launch_input_batch(ids, n, rgb, rgb8, image_width, image_height, frame, xy.ptr, target.ptr, front);
        if (pending) ODIE_CUDA(cudaStreamWaitEvent(front, side_done, 0));
        // the expert gather reads the expert tables that the previous step's tail updates
        route_and_encode(n, pending ? tail_done : nullptr, front);
        const MlpArgs ma = mlp_args(n);
        const int blocks = mlp_tc_train_blocks(n, gate_mode());
        launch_mlp_tc_train(ma, input_width, gate_mode(), uniform, blocks, error_flag.ptr, front);
        ODIE_CUDA(cudaEventRecord(heads_done, front));
        ODIE_CUDA(cudaStreamWaitEvent(stream, heads_done, 0));  // the step's loss, in the caller's stream order
        ODIE_CUDA(cudaStreamWaitEvent(side, heads_done, 0));
        ODIE_CUDA(cudaStreamWaitEvent(tail, heads_done, 0));
        LevelSource rsrc;
        rsrc.table = router_table;
        const EncodeArgs ra = router_encode_args(n);
        launch_encode_backward(ra, rsrc, router_gvals.ptr, router_gradient(), side);
        launch_reduce_partials(partials.ptr, blocks, head_count, head_grad(), side);
        adam_router_grid(side);
        adam_heads(side);
        ODIE_CUDA(cudaEventRecord(side_done, side));
        LevelSource src;
        src.table = table;
        EncodeArgs ea = encode_args(n);
        ea.expert = expert_ids.ptr;
        ea.expert_stride = expert_total;
        ea.experts = experts;
        ea.row_major = true;
        launch_encode_backward(ea, src, gvals.ptr, grid_grad.ptr, tail);
        adam_expert_tables(tail);
        ODIE_CUDA(cudaEventRecord(tail_done, tail));
        pending = true;
        ODIE_CUDA(cudaGetLastError());
    }

    void step_grads(const int64_t* ids, int n, int update, const Sampled* sampled = nullptr) {
        join();
        ODIE_REQUIRE(n > 0 && n <= capacity, "invalid batch size for this runtime");
        int slot = stage_begin(S_INPUT);
        if (sampled)
            launch_stratified_batch(sampled->seed, sampled->step, n, rgb, rgb8, image_width, image_height, frame, xy.ptr,
                                    target.ptr, stream);
        else
            launch_input_batch(ids, n, rgb, rgb8, image_width, image_height, frame, xy.ptr, target.ptr, stream);
        stage_end(slot);
        LevelSource src;
        src.table = table;
        EncodeArgs ea = encode_args(n);
        if (experts) {
            route_and_encode(n);
            ea.expert = expert_ids.ptr;
            ea.expert_stride = expert_total;
            ea.experts = experts;
        } else {
            slot = stage_begin(S_ENCODE_FWD);
            launch_encode_forward(ea, src, nullptr, grid_half.ptr, raw.ptr, reinterpret_cast<uint8_t*>(vis.ptr), stream);
            stage_end(slot);
        }
        const MlpArgs ma = mlp_args(n);
        const int blocks = mlp_tc_train_blocks(n, gate_mode());
        slot = stage_begin(S_MLP);
        launch_mlp_tc_train(ma, input_width, gate_mode(), uniform, blocks, error_flag.ptr, stream);
        stage_end(slot);
        ea.row_major = true;  // the heads write each coordinate's gradient values as one row
        if (experts) {
            // Two branches that meet before the heads' update: the router-grid scatter, the head-gradient
            // reduction and the router grid's Adam on the side stream; the expert-table scatter and the
            // expert tables' Adam on the runtime's stream.  Stage timers run on each branch's own stream.
            // the side branch runs on the main stream when profiling serially
            cudaStream_t side = (profiling && serial) ? stream : this->side;
            ODIE_CUDA(cudaEventRecord(fork_event, stream));
            ODIE_CUDA(cudaStreamWaitEvent(side, fork_event, 0));
            LevelSource rsrc;
            rsrc.table = router_table;
            EncodeArgs ra = router_encode_args(n);  // row-major gradient values too
            slot = stage_begin(S_ENCODE_BWD, side);
            launch_encode_backward(ra, rsrc, router_gvals.ptr, router_gradient(), side);
            stage_end(slot, side);
            slot = stage_begin(S_REDUCE, side);
            launch_reduce_partials(partials.ptr, blocks, head_count, head_grad(), side);  // needs only the heads kernel
            stage_end(slot, side);
            // a shared router grid (caller-owned gradient) is updated in step_heads, after its gradient is summed
            if (update == 1 && !external_router_grad) {
                slot = stage_begin(S_ADAM_GRID, side);
                adam_router_grid(side);
                stage_end(slot, side);
            }
            ODIE_CUDA(cudaEventRecord(join_event, side));
            slot = stage_begin(S_ENCODE_BWD);
            launch_encode_backward(ea, src, gvals.ptr, grid_grad.ptr, stream);
            stage_end(slot);
            if (update == 1) {
                slot = stage_begin(S_ADAM_GRID);
                adam_expert_tables();
                stage_end(slot);
            }
            ODIE_CUDA(cudaStreamWaitEvent(stream, join_event, 0));
        } else {
            slot = stage_begin(S_ENCODE_BWD);
            launch_encode_backward(ea, src, gvals.ptr, grid_grad.ptr, stream);
            stage_end(slot);
            slot = stage_begin(S_REDUCE);
            launch_reduce_partials(partials.ptr, blocks, head_count, head_grad(), stream);
            stage_end(slot);
            if (update == 1) grid_update();
        }
        if (update == 0) {
            launch_zero(grid_grad.ptr, total, stream);
            if (experts) launch_zero(router_gradient(), router_total, stream);
        }
        // update == 2 keeps the grid gradient for inspection; grid_update() consumes it
        ODIE_CUDA(cudaGetLastError());
    }

    // Adam of the grid tables (sparse: zero gradients are skipped), gradients at loss scale 128.
    void adam_expert_tables(cudaStream_t on = nullptr) {
        AdamTables t{table_step[0].ptr, table_bc2.ptr, TABLE_STEPS};
        launch_adam(grid, grid_half.ptr, grid_m.ptr, grid_v.ptr, grid_steps.ptr, grid_grad.ptr, total, 1.0f / 128.0f, t,
                    float(1.0 - BETA1), float(BETA2), float(1.0 - BETA2), float(EPS), true, error_flag.ptr,
                    on ? on : stream);
    }
    void adam_router_grid(cudaStream_t on) {
        AdamTables t{table_step[0].ptr, table_bc2.ptr, TABLE_STEPS};
        launch_adam(router_grid, router_half.ptr, router_m.ptr, router_v.ptr, router_steps.ptr, router_gradient(),
                    router_total, 1.0f / 128.0f, t, float(1.0 - BETA1), float(BETA2), float(1.0 - BETA2), float(EPS),
                    true, error_flag.ptr, on);
    }

    void grid_update() {
        join();
        const int slot = stage_begin(S_ADAM_GRID);
        adam_expert_tables();
        if (experts && !external_router_grad) adam_router_grid(stream);  // a shared router grid: in step_heads
        stage_end(slot);
        ODIE_CUDA(cudaGetLastError());
    }

    void step_heads(bool update) {
        join();
        if (!update) return;
        if (experts && external_router_grad) {
            // the shared router grid: its summed gradient is ready once the caller's reduction has run
            const int grid_slot = stage_begin(S_ADAM_GRID);
            adam_router_grid(stream);
            stage_end(grid_slot);
        }
        const int slot = stage_begin(S_ADAM_HEADS);
        adam_heads(stream);
        stage_end(slot);
        ODIE_CUDA(cudaGetLastError());
    }

    void adam_heads(cudaStream_t on) {
        // head gradients carry the 128 x 128 loss scale (odie/native/runtime.cu:59,300-309)
        const float inv = 1.0f / 16384.0f;
        // gate (or router) and decoder in one launch, each with its own master array and learning rate
        const AdamTables gate_t{table_step[1].ptr, table_bc2.ptr, TABLE_STEPS};
        const AdamTables decoder_t{table_step[2].ptr, table_bc2.ptr, TABLE_STEPS};
        launch_adam2(gate_master, decoder_master, head_half.ptr, head_m.ptr, head_v.ptr, head_steps.ptr, head_grad(),
                     gate_count, decoder_count, inv, gate_t, decoder_t, float(1.0 - BETA1), float(BETA2),
                     float(1.0 - BETA2), float(EPS), false, error_flag.ptr, on);
    }

    ~Runtime() {
        for (cudaStream_t s : {side, tail, front})
            if (s) cudaStreamSynchronize(s);
        for (cudaEvent_t e : {heads_done, side_done, tail_done, call_event})
            if (e) cudaEventDestroy(e);
        if (tail) cudaStreamDestroy(tail);
        if (front) cudaStreamDestroy(front);
        for (auto& e : events) cudaEventDestroy(e);
        if (fork_event) cudaEventDestroy(fork_event);
        if (join_event) cudaEventDestroy(join_event);
        if (side) cudaStreamDestroy(side);
    }

    void decode(long long begin, long long n, float* out_rgb, uint8_t* out_rgb8) {
        join();
        LevelSource src;
        src.table = table;
        for (long long done = 0; done < n; done += capacity) {
            const long long count = std::min(capacity, n - done);
            launch_coords_range(begin + done, count, image_width, image_height, frame, xy.ptr, stream);
            if (experts) {
                route_and_encode(count);
            } else {
                const EncodeArgs ea = encode_args(count);
                launch_encode_forward(ea, src, nullptr, grid_half.ptr, raw.ptr, reinterpret_cast<uint8_t*>(vis.ptr), stream);
            }
            MlpArgs ma = mlp_args(count);
            ma.rgb = out_rgb ? out_rgb + 3 * done : nullptr;
            ma.rgb8 = out_rgb8 ? out_rgb8 + 3 * done : nullptr;
            launch_mlp_tc_decode(ma, input_width, gate_mode(), uniform, error_flag.ptr, stream);
        }
        ODIE_CUDA(cudaGetLastError());
    }

    std::string pointers() {
        std::ostringstream o;
        o << "{\"squares\":" << (unsigned long long)squares.ptr << ",\"grid_grad\":" << (unsigned long long)grid_grad.ptr
          << ",\"half_grad\":0,\"gate_grad\":" << (unsigned long long)(router ? head_grad() : nullptr)
          << ",\"decoder_grad\":" << (unsigned long long)(head_grad() + gate_count)
          << ",\"head_grad\":" << (unsigned long long)head_grad() << ",\"head_count\":" << head_count
          << ",\"gate_count\":" << gate_count << ",\"output\":0,\"raw\":" << (unsigned long long)raw.ptr
          << ",\"mode\":" << mode << ",\"grid_gradient_precision\":\"fp32\""
          << ",\"dirty_count\":0,\"grid_half\":" << (unsigned long long)grid_half.ptr
          << ",\"head_half\":" << (unsigned long long)head_half.ptr << ",\"error_flag\":" << (unsigned long long)error_flag.ptr
          << ",\"capacity\":" << capacity << ",\"input_width\":" << input_width
          << ",\"gvals\":" << (unsigned long long)gvals.ptr << ",\"vis\":" << (unsigned long long)vis.ptr
          << ",\"xy\":" << (unsigned long long)xy.ptr << ",\"target\":" << (unsigned long long)target.ptr
          << ",\"grid_m\":" << (unsigned long long)grid_m.ptr << ",\"grid_v\":" << (unsigned long long)grid_v.ptr
          << ",\"grid_steps\":" << (unsigned long long)grid_steps.ptr << ",\"head_m\":" << (unsigned long long)head_m.ptr
          << ",\"head_v\":" << (unsigned long long)head_v.ptr << ",\"head_steps\":" << (unsigned long long)head_steps.ptr
          << ",\"experts\":" << experts << ",\"expert_total\":" << expert_total << ",\"router_total\":" << router_total
          << ",\"router_width\":" << router_width << ",\"router_half\":" << (unsigned long long)router_half.ptr
          << ",\"router_grad\":" << (unsigned long long)router_gradient() << ",\"logits\":" << (unsigned long long)logits.ptr
          << ",\"live\":" << live << ",\"side_stream\":" << (unsigned long long)side << ",\"router_in\":" << (unsigned long long)router_in.ptr
          << ",\"router_gvals\":" << (unsigned long long)router_gvals.ptr << ",\"prob\":" << (unsigned long long)prob.ptr
          << ",\"expert_ids\":" << (unsigned long long)expert_ids.ptr << ",\"router_m\":" << (unsigned long long)router_m.ptr
          << ",\"router_v\":" << (unsigned long long)router_v.ptr << ",\"router_steps\":" << (unsigned long long)router_steps.ptr
          << ",\"scatter_strategy\":" << (unsigned long long)scatter_strategy.ptr << "}";
        return o.str();
    }

    std::string state(int begin, int end) {
        join();
        ODIE_CUDA(cudaStreamSynchronize(stream));
        int flag = 0;
        ODIE_CUDA(cudaMemcpy(&flag, error_flag.ptr, sizeof(int), cudaMemcpyDeviceToHost));
        ODIE_REQUIRE(flag == 0, "optimizer step table exhausted");
        if (begin >= 0) {
            ODIE_REQUIRE(begin <= end && end <= total, "state range outside the grid");
            const long long count = end - begin;
            bool pristine = true;
            if (count > 0) {
                std::vector<uint32_t> host(count);
                const void* arrays[3] = {grid_m.ptr + begin, grid_v.ptr + begin, grid_steps.ptr + begin};
                for (const void* src : arrays) {
                    ODIE_CUDA(cudaMemcpy(host.data(), src, count * 4, cudaMemcpyDeviceToHost));
                    for (uint32_t x : host) if (x) { pristine = false; break; }
                    if (!pristine) break;
                }
            }
            return std::string("{\"pristine\":") + (pristine ? "true" : "false") + "}";
        }
        // FNV-1a-64 over the raw bytes of every optimizer state array
        unsigned long long hash = 14695981039346656037ull, bytes = 0;
        auto mix = [&](const void* src, long long count) {
            std::vector<unsigned char> host(size_t(count) * 4);
            if (count) ODIE_CUDA(cudaMemcpy(host.data(), src, host.size(), cudaMemcpyDeviceToHost));
            for (unsigned char b : host) { hash ^= b; hash *= 1099511628211ull; }
            bytes += host.size();
        };
        mix(grid_m.ptr, total); mix(grid_v.ptr, total); mix(grid_steps.ptr, total);
        mix(head_m.ptr, head_count); mix(head_v.ptr, head_count); mix(head_steps.ptr, head_count);
        if (experts) { mix(router_m.ptr, router_total); mix(router_v.ptr, router_total); mix(router_steps.ptr, router_total); }
        std::ostringstream o;
        o << "{\"hash_fnv1a64\":\"" << hash << "\",\"bytes\":" << bytes << "}";
        return o.str();
    }
};

LevelTable hash_levels_table(const odie_hash_level* host, int levels) {
    ODIE_REQUIRE(host && levels >= 1 && levels <= MAX_LEVELS, "1..32 hash levels required");
    LevelTable t{};
    for (int l = 0; l < levels; ++l) {
        Level& L = t.level[l];
        L.scale = host[l].scale;
        L.res = host[l].resolution;
        L.points = host[l].capacity;
        L.offset = host[l].offset;
        L.words = -1;
        L.cells = host[l].cells;
        L.F = host[l].features;
        L.col = host[l].column;
        L.kind = host[l].hashed ? HASH_HASHED : HASH_DENSE;
        ODIE_REQUIRE(L.points > 0 && (L.F == 1 || L.F == 2 || L.F == 4), "invalid hash level");
    }
    return t;
}

}  // namespace odie

// ---------------------------------------------------------------- residual / selection (residual.cu, selection.cu)
namespace odie {
void launch_score_chunk(const float* prediction, const void* target, long long begin, long long end, int width,
                        int resolution, int first_y, int active_cells, const int* xb, const int* yb, double* totals,
                        bool rgb8, cudaStream_t stream);
void launch_tile_scores(const float* prediction, const uint8_t* target, int height, int width, int tile, double* row_sums,
                        double* scores, cudaStream_t stream);
void launch_topk(const double* scores, int count, int k, long long* chosen, uint8_t* selected, cudaStream_t stream);
long long noalloc_tile_rows_max();
double* noalloc_row_sums(std::string& error);
int launch_selection_init(const double* scores, int n, int points, int* missing, uint8_t* chosen, uint8_t* nodes,
                          int* tree, long long* stats, const int* host_offsets, const int* host_sizes, int levels,
                          cudaStream_t stream);
int launch_selection_chunk(const double* scores, int n, int points, int resolution, int cap, bool normalized, int* missing,
                           uint8_t* chosen, uint8_t* nodes, int* tree, const int* offsets, const int* sizes, int levels,
                           int chunk, long long* stats, int* trace, cudaStream_t stream);
}  // namespace odie

namespace odie {
long long plane_index_scratch(long long points);
void launch_allocation_bitmap(const uint8_t* tiles, int tiles_x, int tiles_y, int tile_px, int height, int width,
                              int res, uint8_t* bitmap, cudaStream_t stream);
void launch_plane_index(const uint8_t* support, int resolution, unsigned long long* node_words, int* node_prefix,
                        uint8_t* cell_bitmap, long long* node_count, long long* nodes, int* scratch,
                        cudaStream_t stream);
void launch_l2_probe(float* table, long long table_bytes, int mode, long long operations, float* sink,
                     cudaStream_t stream);
void launch_wait_probe(uint32_t limit, int* status, cudaStream_t stream);
long long launch_fma_probe(int iterations, float* sink, cudaStream_t stream);
}  // namespace odie

using odie::guarded;
using odie::Runtime;

extern "C" {

const char* odie_error(void) { return odie::g_error.c_str(); }

long long odie_launch_count(void) { return odie::g_launches.load(std::memory_order_relaxed); }

void* odie_create(const char* json) {
    try {
        return new Runtime(odie::parse_json(json));
    } catch (const std::exception& e) {
        odie::set_error(e.what());
        return nullptr;
    }
}

int odie_step(void* handle, uint64_t ids, int n, int update) {
    return guarded([&] {
        auto* r = static_cast<Runtime*>(handle);
        if (r->pipeline && update && !r->profiling) {
            r->step_pipelined(reinterpret_cast<const int64_t*>(ids), n, nullptr);
            return;
        }
        r->step_grads(reinterpret_cast<const int64_t*>(ids), n, update != 0 ? 1 : 0);
        r->step_heads(update != 0);
    });
}

int odie_step_stratified(void* handle, uint64_t seed, uint64_t step, int n, int update) {
    return guarded([&] {
        auto* r = static_cast<Runtime*>(handle);
        const odie::Runtime::Sampled sampled{seed, step};
        if (r->pipeline && update && !r->profiling) {
            r->step_pipelined(nullptr, n, &sampled);
            return;
        }
        r->step_grads(nullptr, n, update != 0 ? 1 : 0, &sampled);
        r->step_heads(update != 0);
    });
}

int odie_join(void* handle) {
    return guarded([&] { static_cast<Runtime*>(handle)->join(); });
}

int odie_stratified_ids(uint64_t seed, uint64_t step, int width, int height, int64_t n, int64_t* ids, uint64_t stream) {
    return guarded([&] {
        odie::launch_stratified_ids(seed, step, width, height, n, ids, reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_step_grads(void* handle, uint64_t ids, int n, int update) {
    return guarded([&] { static_cast<Runtime*>(handle)->step_grads(reinterpret_cast<const int64_t*>(ids), n, update); });
}

int odie_step_heads(void* handle) {
    return guarded([&] { static_cast<Runtime*>(handle)->step_heads(true); });
}

int odie_grid_update(void* handle) {
    return guarded([&] { static_cast<Runtime*>(handle)->grid_update(); });
}

int odie_profile(void* handle, int enable) {
    return guarded([&] {
        ODIE_REQUIRE(enable >= 0 && enable <= 2, "odie_profile: 0 off, 1 on, 2 on with the step's branches serialised");
        static_cast<Runtime*>(handle)->profile(enable);
    });
}

const char* odie_profile_report(void* handle) {
    try {
        odie::g_reply = static_cast<Runtime*>(handle)->profile_report();
        return odie::g_reply.c_str();
    } catch (const std::exception& e) {
        odie::set_error(e.what());
        return nullptr;
    }
}

const char* odie_pointers(void* handle) {
    odie::g_reply = static_cast<Runtime*>(handle)->pointers();
    return odie::g_reply.c_str();
}

const char* odie_state(void* handle, int begin, int end) {
    try {
        odie::g_reply = static_cast<Runtime*>(handle)->state(begin, end);
        return odie::g_reply.c_str();
    } catch (const std::exception& e) {
        odie::set_error(e.what());
        return nullptr;
    }
}

int odie_configure(void* handle, const char* json) {
    return guarded([&] { static_cast<Runtime*>(handle)->configure(odie::parse_json(json)); });
}

void odie_release_contexts(void*) {}
void odie_pin_contexts(void*) {}

int odie_sync_weights(void* handle) {
    return guarded([&] { static_cast<Runtime*>(handle)->sync_weights(); });
}

int odie_copy(uint64_t dst, uint64_t src, uint64_t bytes, uint64_t stream) {
    return int(cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes,
                               cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)));
}

void odie_destroy(void* handle) { delete static_cast<Runtime*>(handle); }

int odie_decode(void* handle, int64_t begin, int64_t n, float* rgb, uint8_t* rgb8) {
    return guarded([&] {
        ODIE_REQUIRE(n >= 0 && begin >= 0, "invalid decode range");
        static_cast<Runtime*>(handle)->decode(begin, n, rgb, rgb8);
    });
}

int odie_query_forward(const float* coords, int64_t n, const float* grid, const int32_t* descriptors, int levels,
                       const uint64_t* node_bitmap, const int32_t* node_prefix, const uint8_t* bitmap, int width,
                       uint16_t* features, uint8_t* visible, uint64_t stream) {
    return guarded([&] {
        ODIE_REQUIRE(levels >= 2 && levels <= 32, "descriptor must hold 2..32 levels");
        ODIE_REQUIRE(width >= 2 && width <= 128, "feature width must be within 2..128");
        ODIE_REQUIRE(n >= 0, "negative coordinate count");
        odie::EncodeArgs a;
        a.coords = coords;
        a.n = n;
        a.levels = levels;
        a.active = levels;
        a.node_bitmap = node_bitmap;
        a.node_prefix = node_prefix;
        a.bitmap = bitmap;
        a.row_major = true;
        a.width = width;
        a.stride = n;
        odie::LevelSource src;
        src.descriptors = descriptors;
        odie::launch_encode_forward(a, src, grid, nullptr, reinterpret_cast<__half*>(features), visible,
                                    reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_query_backward(const float* coords, int64_t n, const uint16_t* upstream, int width, const int32_t* descriptors,
                        int levels, const uint64_t* node_bitmap, const int32_t* node_prefix, const uint8_t* bitmap,
                        float* gradient, int64_t parameter_count, uint64_t stream) {
    return guarded([&] {
        ODIE_REQUIRE(levels >= 2 && levels <= 32, "descriptor must hold 2..32 levels");
        ODIE_REQUIRE(width >= 2 && width <= 128, "upstream width must be within 2..128");
        ODIE_REQUIRE(parameter_count >= 0 && n >= 0, "negative sizes");
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        if (parameter_count) ODIE_CUDA(cudaMemsetAsync(gradient, 0, size_t(parameter_count) * 4, s));
        odie::EncodeArgs a;
        a.coords = coords;
        a.n = n;
        a.levels = levels;
        a.active = levels;
        a.node_bitmap = node_bitmap;
        a.node_prefix = node_prefix;
        a.bitmap = bitmap;
        a.row_major = true;
        a.width = width;
        a.stride = n;
        odie::LevelSource src;
        src.descriptors = descriptors;
        odie::launch_encode_backward(a, src, reinterpret_cast<const __half*>(upstream), gradient, s);
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_hash_forward(const float* coords, int64_t n, const float* table, const odie_hash_level* levels_host, int levels,
                      int width, uint16_t* features, uint64_t stream) {
    return guarded([&] {
        odie::EncodeArgs a;
        a.coords = coords;
        a.n = n;
        a.levels = levels;
        a.active = levels;
        a.row_major = true;
        a.width = width;
        a.stride = n;
        odie::LevelSource src;
        src.table = odie::hash_levels_table(levels_host, levels);
        odie::launch_encode_forward(a, src, table, nullptr, reinterpret_cast<__half*>(features), nullptr,
                                    reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_hash_backward(const float* coords, int64_t n, const uint16_t* upstream, int width,
                       const odie_hash_level* levels_host, int levels, float* gradient, int64_t parameter_count,
                       uint64_t stream) {
    return guarded([&] {
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        if (parameter_count) ODIE_CUDA(cudaMemsetAsync(gradient, 0, size_t(parameter_count) * 4, s));
        odie::EncodeArgs a;
        a.coords = coords;
        a.n = n;
        a.levels = levels;
        a.active = levels;
        a.row_major = true;
        a.width = width;
        a.stride = n;
        odie::LevelSource src;
        src.table = odie::hash_levels_table(levels_host, levels);
        odie::launch_encode_backward(a, src, reinterpret_cast<const __half*>(upstream), gradient, s);
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_router_forward_banded(const uint16_t* features, const float* xy, int64_t n, int width, const uint16_t* weights,
                               int experts, int bands, int first_band, int experts_per_band, int rows, int32_t* expert,
                               float* prob, uint16_t* logits, int live, uint64_t stream) {
    return guarded([&] {
        ODIE_REQUIRE(n >= 0, "negative coordinate count");
        odie::RouterArgs a;
        a.features = reinterpret_cast<const __half*>(features);
        a.row_major = true;
        a.stride = n;
        a.n = n;
        a.weights = reinterpret_cast<const __half*>(weights);
        a.experts = experts;
        a.banding = odie::Banding{bands, first_band, experts_per_band, rows};
        a.xy = xy;
        a.expert = expert;
        a.prob = prob;
        a.logits = reinterpret_cast<__half*>(logits);
        a.live = live;
        odie::launch_router_forward(a, width, reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_router_forward(const uint16_t* features, int64_t n, int width, const uint16_t* weights, int experts,
                        int32_t* expert, float* prob, uint16_t* logits, uint64_t stream) {
    if (experts < 1 || experts > 16) {
        odie::set_error("odie_router_forward: experts must be within 1..16 (odie_router_forward_banded takes up to 64)");
        return -1;
    }
    return odie_router_forward_banded(features, nullptr, n, width, weights, experts, 1, 0, experts, 2, expert, prob,
                                      logits, 16, stream);
}

int odie_expert_hash_forward(const float* coords, int64_t n, const float* tables, int64_t expert_stride,
                             const int32_t* expert, const odie_hash_level* levels_host, int levels, int width,
                             const uint8_t* bitmap, uint16_t* features, uint64_t stream) {
    return guarded([&] {
        ODIE_REQUIRE(n >= 0 && expert_stride > 0, "invalid sizes");
        odie::EncodeArgs a;
        a.coords = coords;
        a.n = n;
        a.levels = levels;
        a.active = levels;
        a.row_major = true;
        a.width = width;
        a.stride = n;
        a.expert = expert;
        a.expert_stride = expert_stride;
        a.bitmap = bitmap;
        odie::LevelSource src;
        src.table = odie::hash_levels_table(levels_host, levels);
        odie::launch_encode_forward(a, src, tables, nullptr, reinterpret_cast<__half*>(features), nullptr,
                                    reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_expert_hash_backward(const float* coords, int64_t n, const uint16_t* upstream, int width, int64_t expert_stride,
                              const int32_t* expert, const odie_hash_level* levels_host, int levels,
                              const uint8_t* bitmap, float* gradient, int64_t parameter_count, uint64_t stream) {
    return guarded([&] {
        ODIE_REQUIRE(n >= 0 && expert_stride > 0 && parameter_count >= 0, "invalid sizes");
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        if (parameter_count) ODIE_CUDA(cudaMemsetAsync(gradient, 0, size_t(parameter_count) * 4, s));
        odie::EncodeArgs a;
        a.coords = coords;
        a.n = n;
        a.levels = levels;
        a.active = levels;
        a.row_major = true;
        a.width = width;
        a.stride = n;
        a.expert = expert;
        a.expert_stride = expert_stride;
        a.experts = int(std::max<int64_t>(1, parameter_count / expert_stride));
        a.bitmap = bitmap;
        odie::LevelSource src;
        src.table = odie::hash_levels_table(levels_host, levels);
        odie::launch_encode_backward(a, src, reinterpret_cast<const __half*>(upstream), gradient, s);
        ODIE_CUDA(cudaGetLastError());
    });
}

int64_t odie_plane_index_scratch(int resolution) {
    if (resolution < 1) return -1;
    const long long cells = (long long)resolution * resolution;
    return odie::plane_index_scratch((cells + 7) / 8 * 8);
}

int odie_plane_index(const uint8_t* support, int resolution, uint64_t* node_bitmap, int32_t* node_prefix,
                     uint8_t* cell_bitmap, int64_t* node_count, int64_t* nodes, int32_t* scratch, uint64_t stream) {
    return guarded([&] {
        odie::launch_plane_index(support, resolution, reinterpret_cast<unsigned long long*>(node_bitmap), node_prefix,
                                 cell_bitmap, reinterpret_cast<long long*>(node_count), reinterpret_cast<long long*>(nodes),
                                 scratch, reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_allocation_bitmap(const uint8_t* tiles, int tiles_x, int tiles_y, int tile_px, int height, int width,
                           int resolution, uint8_t* bitmap, uint64_t stream) {
    return guarded([&] {
        odie::launch_allocation_bitmap(tiles, tiles_x, tiles_y, tile_px, height, width, resolution, bitmap,
                                       reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int64_t odie_fma_probe(int iterations, float* sink, uint64_t stream) {
    long long flop = -1;
    guarded([&] { flop = odie::launch_fma_probe(iterations, sink, reinterpret_cast<cudaStream_t>(stream)); });
    return flop;
}

int odie_wait_probe(uint32_t limit, int32_t* status, uint64_t stream) {
    return guarded([&] {
        odie::launch_wait_probe(limit, status, reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int odie_l2_probe(float* table, int64_t table_bytes, int mode, int64_t operations, float* sink, uint64_t stream) {
    return guarded([&] {
        odie::launch_l2_probe(table, table_bytes, mode, operations, sink, reinterpret_cast<cudaStream_t>(stream));
        ODIE_CUDA(cudaGetLastError());
    });
}

int score_chunk(const float* prediction, const void* target, int64_t begin, int64_t end, int width, int resolution,
                int first_y, int active_cells, const int* xb, const int* yb, double* totals, bool rgb8, uint64_t stream) {
    odie::launch_score_chunk(prediction, target, begin, end, width, resolution, first_y, active_cells, xb, yb, totals, rgb8,
                             reinterpret_cast<cudaStream_t>(stream));
    return int(cudaGetLastError());
}

int selection_init(const double* scores, int n, int points, int* missing, uint8_t* chosen, uint8_t* nodes, int* tree,
                   int64_t* stats, const int* host_offsets, const int* host_sizes, int levels, uint64_t stream) {
    return odie::launch_selection_init(scores, n, points, missing, chosen, nodes, tree, reinterpret_cast<long long*>(stats),
                                       host_offsets, host_sizes, levels, reinterpret_cast<cudaStream_t>(stream));
}

int selection_chunk(const double* scores, int n, int points, int resolution, int cap, bool normalized, int* missing,
                    uint8_t* chosen, uint8_t* nodes, int* tree, const int* offsets, const int* sizes, int levels, int chunk,
                    int64_t* stats, int* trace, uint64_t stream) {
    return odie::launch_selection_chunk(scores, n, points, resolution, cap, normalized, missing, chosen, nodes, tree,
                                        offsets, sizes, levels, chunk, reinterpret_cast<long long*>(stats), trace,
                                        reinterpret_cast<cudaStream_t>(stream));
}

namespace {
// Tiles of a height x width image cut into tile x tile squares (edge tiles partial), or -1 with a message
// when the arguments are invalid.  Widened to 64 bits before any sum, so no tile size overflows.
long long tile_count(const char* who, int height, int width, int tile, int k) {
    if (height < 1 || width < 1 || tile < 1 || k < 0) {
        odie::set_error(std::string(who) + ": height, width and tile must be >= 1 and k >= 0");
        return -1;
    }
    if (tile > std::max(height, width)) {
        odie::set_error(std::string(who) + ": tile must not exceed the image's larger side");
        return -1;
    }
    const long long tiles = (((long long)width + tile - 1) / tile) * (((long long)height + tile - 1) / tile);
    if (tiles > 0x7fffffffLL || (long long)tile * tiles > (1LL << 40)) {
        odie::set_error(std::string(who) + ": too many tiles");
        return -1;
    }
    if (k > tiles) {
        odie::set_error(std::string(who) + ": k = " + std::to_string(k) + " exceeds the " + std::to_string(tiles) +
                        " tiles");
        return -1;
    }
    return tiles;
}
}  // namespace

int odie_tile_topk(const float* prediction, const uint8_t* target, int height, int width, int tile, int k,
                   double* row_sums, double* scores, int64_t* chosen, uint8_t* selected, uint64_t stream) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const long long tiles = tile_count("odie_tile_topk", height, width, tile, k);
    if (tiles < 0) return int(cudaErrorInvalidValue);
    odie::launch_tile_scores(prediction, target, height, width, tile, row_sums, scores, s);
    odie::launch_topk(scores, int(tiles), k, reinterpret_cast<long long*>(chosen), selected, s);
    return int(cudaGetLastError());
}

int odie_topk(const double* scores, int count, int k, int64_t* chosen, uint8_t* selected, uint64_t stream) {
    if (count < 0 || k < 0 || k > count) {
        odie::set_error("odie_topk: need 0 <= k <= count");
        return int(cudaErrorInvalidValue);
    }
    odie::launch_topk(scores, count, k, reinterpret_cast<long long*>(chosen), selected,
                      reinterpret_cast<cudaStream_t>(stream));
    return int(cudaGetLastError());
}

// odie_tile_topk without the caller-provided row-sum buffer.  Some callers cannot
// hand over device memory: an embedding host whose GPU memory is all owned by its
// own allocator or capped by a budget, or code that runs where a cudaMalloc would
// synchronise the device or is not allowed.  The row sums go to the library's fixed
// array instead (size limit checked here, before anything is launched).
int odie_tile_topk_noalloc(const float* prediction, const uint8_t* target, int height, int width, int tile, int k,
                           double* scores, int64_t* chosen, uint8_t* selected, uint64_t stream) {
    const long long tiles = tile_count("odie_tile_topk_noalloc", height, width, tile, k);
    if (tiles < 0) return int(cudaErrorInvalidValue);
    if (tiles * tile > odie::noalloc_tile_rows_max()) {
        odie::set_error("odie_tile_topk_noalloc: tiles x tile = " + std::to_string(tiles * tile) +
                        " row sums exceed the fixed scratch of " + std::to_string(odie::noalloc_tile_rows_max()));
        return int(cudaErrorInvalidValue);
    }
    std::string error;
    double* row_sums = odie::noalloc_row_sums(error);
    if (!row_sums) {
        odie::set_error("odie_tile_topk_noalloc: " + error);
        return int(cudaErrorInvalidValue);
    }
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    odie::launch_tile_scores(prediction, target, height, width, tile, row_sums, scores, s);
    odie::launch_topk(scores, int(tiles), k, reinterpret_cast<long long*>(chosen), selected, s);
    return int(cudaGetLastError());
}

}  // extern "C"
