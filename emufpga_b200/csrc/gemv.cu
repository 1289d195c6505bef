// Launch geometry and dispatch of the streaming GEMV (kernel in gemv_impl.cuh,
// instantiated per block type in gemv_<type>.cu).
#include <algorithm>

#include "gemv_impl.cuh"

namespace spm {
namespace gemv {
#define SPM_EXTERN(T)                                                                                    \
    extern template cudaError_t launch_enc<T>(const GemvLaunch&, bool, int, int, size_t, cudaStream_t, bool); \
    extern template int occupancy_enc<T>(const GemvLaunch&, bool, int, size_t);
SPM_EXTERN(SPM_Q8_0)
SPM_EXTERN(SPM_Q6_K)
SPM_EXTERN(SPM_Q5_K)
SPM_EXTERN(SPM_Q2_K)
SPM_EXTERN(SPM_F32)
#undef SPM_EXTERN
}  // namespace gemv

using namespace gemv;

static int occupancy(uint32_t dtype, const GemvLaunch& L, bool dual, int threads, size_t smem) {
    switch (dtype) {
        case SPM_Q8_0: return occupancy_enc<SPM_Q8_0>(L, dual, threads, smem);
        case SPM_Q6_K: return occupancy_enc<SPM_Q6_K>(L, dual, threads, smem);
        case SPM_Q5_K: return occupancy_enc<SPM_Q5_K>(L, dual, threads, smem);
        case SPM_Q2_K: return occupancy_enc<SPM_Q2_K>(L, dual, threads, smem);
        case SPM_F32: return occupancy_enc<SPM_F32>(L, dual, threads, smem);
        default: return 1;
    }
}

// CTA size, warp groups and ring slots.  Two CTAs of up to 8 warps share an
// SM when their ring and activations fit in half of its shared memory (the
// next kernel's CTAs can then start prefetching beside them); otherwise one
// CTA of up to 16 warps has the SM to itself.  A group of gw warps works on
// one tile at a time with its lanes over the tile's units; each group owns
// its ring slots (slot s belongs to group s % G), at least two unless it has
// a single tile, so that one slot is read while the next is in flight.
// Among the shapes that fit, the one with the most busy warps per SM wins
// (a warp counts in proportion to the lanes that have a unit, and only in a
// group that has a tile), then two CTAs per SM, then smaller groups.
GemvGeometry gemv_geometry(const GemvLaunch& L, bool dual, int sms, int per_fixed) {
    const uint32_t U = L.cols / 32;
    // work items: tiles, or pairs of tiles for the tensor-core loop (whose
    // warps take whole units of a slot instead of lanes taking units)
    const bool pair = L.tc && !dual;
    // tiles of rows per work item (slot): tc2 four (two gate/up pairs), pair two
    const uint32_t tps = L.tc2 ? (dual ? 2u : 4u) : pair ? 2u : 1u;
    const uint32_t work = (L.total_tiles + tps - 1) / tps;
    if (per_fixed > 0 && tps > 1) per_fixed = int((uint32_t(per_fixed) + tps - 1) / tps);
    GemvGeometry best{};
    double best_score = -1.0;
    for (int per_sm = 2; per_sm >= 1; per_sm--) {
        const int Wmax = per_sm == 2 ? kPairWarps : kMaxWarps;
        const size_t cap = per_sm == 2 ? kHalfSm : kSmemMax;
        int grid = 0, per = per_fixed;
        if (per_fixed <= 0) {
            const uint32_t gcap = uint32_t(sms) * uint32_t(per_sm);
            grid = int(std::min(work, gcap));
            per = int((work + grid - 1) / grid);
        }
        for (int gw = 1; gw <= Wmax; gw *= 2) {
            // at most four units per lane (tensor cores: 32 units per warp)
            const bool warps_take_units = L.tc || L.tc2;
            const uint32_t lanes = warps_take_units ? uint32_t(gw) : 32u * gw, most = warps_take_units ? 32u : 4u;
            if ((U + lanes - 1) / lanes > most && gw < Wmax) continue;
            const double busy = std::min(1.0, double(U) / double(lanes));
            for (int G = Wmax / gw; G >= 1; G--) {
                const int W = G * gw;
                if (W < 4) break;
                const int pg = (per + G - 1) / G;  // tiles per group
                int nsg = std::min(pg, kMaxSlots / G);
                while (nsg >= 1 && smem_bytes(L, dual, G * nsg, gw) > cap) nsg--;
                if (nsg < 1 || nsg < std::min(pg, 2)) continue;
                const double score = per_sm * std::min(G, per) * gw * busy;  // groups without tiles idle
                if (score > best_score + 1e-9) {
                    best_score = score;
                    best = GemvGeometry{grid, G * nsg, W, gw, smem_bytes(L, dual, G * nsg, gw)};
                }
                break;  // fewer groups of this size only score lower
            }
        }
    }
    if (best_score >= 0) return best;
    // one CTA per SM, all its warps on each tile, as many slots as fit
    int ns = kMaxSlots;
    while (ns > 1 && smem_bytes(L, dual, ns, kMaxWarps) > kSmemMax) ns--;
    const int grid = per_fixed > 0 ? 0 : int(std::min(work, uint32_t(sms)));
    return GemvGeometry{grid, ns, kMaxWarps, kMaxWarps, smem_bytes(L, dual, ns, kMaxWarps)};
}

// The launch fields that follow from the block type and client count.
static void prepare(GemvLaunch& L, uint32_t dtype) {
    L.xrec = unit_bytes(int(dtype));
    L.tc = use_tc(int(dtype), L.n) && !L.plan ? 1 : 0;
    L.tc2 = use_tc2(int(dtype), L.n) ? 1 : 0;
}

// Geometry with the grid capped at the CTAs that can be resident at once
// (one wave), so that every CTA starts streaming immediately.
static GemvGeometry geometry_resident(uint32_t dtype, GemvLaunch L, bool dual, int sms) {
    prepare(L, dtype);
    GemvGeometry g = gemv_geometry(L, dual, sms);
    const int occ = occupancy(dtype, L, dual, g.warps * 32, g.smem);
    const int cap = occ * sms;
    if (g.grid > cap) g.grid = cap;
    return g;
}

static cudaError_t launch_one(uint32_t dtype, GemvLaunch L, int sms, cudaStream_t s, bool pdl, int grid) {
    const bool dual = L.job[0].b != nullptr;
    prepare(L, dtype);
    GemvGeometry g;
    if (L.plan) {
        // expert mode: a CTA owns 1/expert_chunks of one active expert's
        // tiles at most; the grid fills the SMs once (the kernel splits the
        // active experts over it), every possible active expert has a CTA
        g = gemv_geometry(L, dual, sms, int((L.expert_tiles + L.expert_chunks - 1) / L.expert_chunks));
        const int occ = occupancy(dtype, L, dual, g.warps * 32, g.smem);
        g.grid = std::max(L.expert_max, std::max(1, occ) * sms);
    } else {
        g = geometry_resident(dtype, L, dual, sms);
    }
    if (grid > 0 && grid < g.grid) g.grid = grid;  // more tiles per CTA; the ring stays valid
    L.slots = g.slots;
    L.group_warps = g.group_warps;
    const int threads = g.warps * 32;
    switch (dtype) {
        case SPM_Q8_0: return launch_enc<SPM_Q8_0>(L, dual, g.grid, threads, g.smem, s, pdl);
        case SPM_Q6_K: return launch_enc<SPM_Q6_K>(L, dual, g.grid, threads, g.smem, s, pdl);
        case SPM_Q5_K: return launch_enc<SPM_Q5_K>(L, dual, g.grid, threads, g.smem, s, pdl);
        case SPM_Q2_K: return launch_enc<SPM_Q2_K>(L, dual, g.grid, threads, g.smem, s, pdl);
        case SPM_F32: return launch_enc<SPM_F32>(L, dual, g.grid, threads, g.smem, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(uint32_t dtype, GemvLaunch L, int sms, cudaStream_t s, bool pdl, int* grid_out) {
    const bool dual = L.job[0].b != nullptr;
    if (grid_out) *grid_out = 0;
    if (L.total_tiles == 0) return cudaSuccess;
    if (L.n < 1 || L.n > 8 || (L.cols & 31)) return cudaErrorInvalidValue;
    prepare(L, dtype);
    GemvLaunch one = L;
    one.n = 1;
    prepare(one, dtype);
    if (smem_bytes(one, dual, 1, kMaxWarps) > kSmemMax) return cudaErrorInvalidValue;
    const bool fits = smem_bytes(L, dual, 1, kMaxWarps) <= kSmemMax;
    if ((L.plan || L.ep_done) && !fits) return cudaErrorInvalidValue;  // one launch raises the flag
    if (!fits) {
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
