// Launch geometry and dispatch of the streaming GEMV (kernel in gemv_impl.cuh,
// instantiated per block type in gemv_<type>.cu).
#include "gemv_impl.cuh"

namespace spm {
namespace gemv {
extern template cudaError_t launch_enc<SPM_Q8_0>(const GemvLaunch&, bool, int, size_t, cudaStream_t, bool);
extern template cudaError_t launch_enc<SPM_Q6_K>(const GemvLaunch&, bool, int, size_t, cudaStream_t, bool);
extern template cudaError_t launch_enc<SPM_Q5_K>(const GemvLaunch&, bool, int, size_t, cudaStream_t, bool);
extern template cudaError_t launch_enc<SPM_Q2_K>(const GemvLaunch&, bool, int, size_t, cudaStream_t, bool);
extern template cudaError_t launch_enc<SPM_F32>(const GemvLaunch&, bool, int, size_t, cudaStream_t, bool);
extern template int occupancy_enc<SPM_Q8_0>(const GemvLaunch&, bool, size_t);
extern template int occupancy_enc<SPM_Q6_K>(const GemvLaunch&, bool, size_t);
extern template int occupancy_enc<SPM_Q5_K>(const GemvLaunch&, bool, size_t);
extern template int occupancy_enc<SPM_Q2_K>(const GemvLaunch&, bool, size_t);
extern template int occupancy_enc<SPM_F32>(const GemvLaunch&, bool, size_t);
}  // namespace gemv

using namespace gemv;

// Bytes of the clients' activations staged in shared memory, with their
// 16-value sums.
static size_t x_stage_bytes(const GemvLaunch& L) { return size_t(L.n) * (L.cols * 4 + (L.cols / 16) * 4); }

static int occupancy(uint32_t dtype, const GemvLaunch& L, bool dual, size_t smem) {
    switch (dtype) {
        case SPM_Q8_0: return occupancy_enc<SPM_Q8_0>(L, dual, smem);
        case SPM_Q6_K: return occupancy_enc<SPM_Q6_K>(L, dual, smem);
        case SPM_Q5_K: return occupancy_enc<SPM_Q5_K>(L, dual, smem);
        case SPM_Q2_K: return occupancy_enc<SPM_Q2_K>(L, dual, smem);
        case SPM_F32: return occupancy_enc<SPM_F32>(L, dual, smem);
        default: return 1;
    }
}

// Geometry with the grid capped at the CTAs that can be resident at once
// (one wave), so that every CTA starts streaming immediately.
static GemvGeometry geometry_resident(uint32_t dtype, const GemvLaunch& L, bool dual, int sms) {
    GemvGeometry g = gemv_geometry(L, dual, sms);
    const int occ = occupancy(dtype, L, dual, g.smem);
    const int cap = occ * sms;
    if (g.grid > cap) g.grid = cap;
    return g;
}

// Ring slots and shared memory for CTAs that each own about `per` tiles.
static GemvGeometry ring_geometry(const GemvLaunch& L, bool dual, int per) {
    GemvGeometry g{};
    const size_t slot = size_t(L.tile_bytes) * (dual ? 2 : 1);
    const size_t xb = x_stage_bytes(L);
    // Two CTAs per SM when ring + activations fit in half the SM's shared
    // memory (the next kernel's CTAs can then start prefetching beside them).
    size_t ring = kRingBytes;
    if (xb + ring > kHalfSm) ring = xb + kRingMin <= kHalfSm ? kHalfSm - xb : kSmemMax - xb;
    if (ring > kRingBytes) ring = kRingBytes;
    int slots = int(ring / slot);
    if (slots > kMaxSlots) slots = kMaxSlots;
    if (slots > per) slots = per;
    if (slots < 1) slots = 1;
    g.slots = slots;
    g.consumers = kConsumers;
    g.smem = slot * size_t(slots) + xb;
    return g;
}

GemvGeometry gemv_geometry(const GemvLaunch& L, bool dual, int sms) {
    const size_t xb = x_stage_bytes(L);
    const int per_sm = xb + kRingMin <= kHalfSm ? 2 : 1;
    const uint32_t gcap = uint32_t(sms) * per_sm;
    const int grid = int(L.total_tiles < gcap ? L.total_tiles : gcap);
    const int per = grid ? int((L.total_tiles + grid - 1) / grid) : 1;
    GemvGeometry g = ring_geometry(L, dual, per);
    g.grid = grid;
    return g;
}

static cudaError_t launch_one(uint32_t dtype, GemvLaunch L, int sms, cudaStream_t s, bool pdl, int grid) {
    const bool dual = L.job[0].b != nullptr;
    GemvGeometry g;
    if (L.plan) {
        // expert mode: a CTA owns 1/expert_chunks of one active expert's tiles
        g = ring_geometry(L, dual, int((L.expert_tiles + L.expert_chunks - 1) / L.expert_chunks));
        g.grid = L.expert_max * L.expert_chunks;
    } else {
        g = geometry_resident(dtype, L, dual, sms);
    }
    if (grid > 0 && grid < g.grid) g.grid = grid;  // more tiles per CTA; the ring stays valid
    L.slots = g.slots;
    L.consumers = g.consumers;
    switch (dtype) {
        case SPM_Q8_0: return launch_enc<SPM_Q8_0>(L, dual, g.grid, g.smem, s, pdl);
        case SPM_Q6_K: return launch_enc<SPM_Q6_K>(L, dual, g.grid, g.smem, s, pdl);
        case SPM_Q5_K: return launch_enc<SPM_Q5_K>(L, dual, g.grid, g.smem, s, pdl);
        case SPM_Q2_K: return launch_enc<SPM_Q2_K>(L, dual, g.grid, g.smem, s, pdl);
        case SPM_F32: return launch_enc<SPM_F32>(L, dual, g.grid, g.smem, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(uint32_t dtype, GemvLaunch L, int sms, cudaStream_t s, bool pdl, int* grid_out) {
    const bool dual = L.job[0].b != nullptr;
    if (grid_out) *grid_out = 0;
    if (L.total_tiles == 0) return cudaSuccess;
    if (L.n < 1 || L.n > 8 || (L.cols & 31)) return cudaErrorInvalidValue;
    const size_t slot = size_t(L.tile_bytes) * (dual ? 2 : 1);
    if (slot + size_t(L.cols) * 4 + (L.cols / 16) * 4 > kSmemMax) return cudaErrorInvalidValue;
    if (L.plan && slot + x_stage_bytes(L) > kSmemMax) return cudaErrorInvalidValue;
    if (slot + x_stage_bytes(L) > kSmemMax) {
        // The clients' activations do not fit beside one tile: one launch per
        // half of the clients (the weights are read twice), on a common grid
        // so that both halves write the same sum-of-squares parts.
        GemvLaunch a = L, b = L;
        a.n = L.n / 2;
        b.n = L.n - a.n;
        b.c0 = L.c0 + a.n;
        b.x = L.x + size_t(a.n) * L.x_stride;
        for (int j = 0; j < L.njobs; j++) {
            b.job[j].y = L.job[j].y + size_t(a.n) * L.job[j].y_stride;
            if (L.job[j].aux) b.job[j].aux = L.job[j].aux + size_t(a.n) * L.job[j].aux_stride;
        }
        const int ga = geometry_resident(dtype, a, dual, sms).grid, gb = geometry_resident(dtype, b, dual, sms).grid;
        const int grid = ga < gb ? ga : gb;
        cudaError_t e = launch_one(dtype, a, sms, s, pdl, grid);
        if (e == cudaSuccess) e = launch_one(dtype, b, sms, s, pdl, grid);
        if (grid_out) *grid_out = grid;
        return e;
    }
    if (grid_out) *grid_out = geometry_resident(dtype, L, dual, sms).grid;
    return launch_one(dtype, L, sms, s, pdl, 0);
}

}  // namespace spm
