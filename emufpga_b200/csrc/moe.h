// Routed (mixture-of-experts) feed-forward: the device-side plan shared by
// the route kernel, the expert-mode GEMVs and the combine kernel.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace spm {

constexpr int kMoeMaxExperts = 256;
constexpr int kMoeMaxClients = 8;
constexpr int kMoeMaxUsed = 8;

// Written by route_kernel once per routed layer and step.
struct MoePlan {
    int32_t count;                                       // active experts U
    int32_t expert[kMoeMaxExperts];                      // ascending expert ids
    int32_t ntok[kMoeMaxExperts];                        // clients routed to it
    int32_t tok[kMoeMaxExperts][kMoeMaxClients];         // those clients, ascending
    int32_t route[kMoeMaxClients][kMoeMaxUsed];          // selected ids, route order
    // a client's routes in ascending expert order (the order outputs are added):
    int32_t slot_a[kMoeMaxClients][kMoeMaxUsed];         // active index
    int32_t slot_pos[kMoeMaxClients][kMoeMaxUsed];       // position among that expert's clients
    float slot_p[kMoeMaxClients][kMoeMaxUsed];           // routing probability
    float norm[kMoeMaxClients];                          // sum of the selected probabilities
    // how close the routing came to a different expert set: (p_K - p_K+1) / p_K
    // for the K-th largest probability and the largest one left out (1 when
    // every expert is selected)
    float gap[kMoeMaxClients];
    // the active experts this rank computes (expert parallel: e % world ==
    // rank; one GPU: all), as active indices ascending
    int32_t nlocal;
    int32_t local[kMoeMaxExperts];
};

// Softmax over (logits + bias), top-`used` (descending, ties to the lower id),
// renormaliser, and the plan (spm-granite-moe/src/moe.rs:17-35, math.rs:23-39).
cudaError_t launch_route(const float* logits, const float* bias, int n, int experts, int used, int world, int rank,
                         MoePlan* plan, cudaStream_t s, bool pdl);
// Router logits and routing in one launch (one GPU): logits[c][e] =
// s_c * sum_k W[e][k] * (x[c][k] * gain[k]) with s_c the RMSNorm scale of
// client c from the producer's per-CTA sums of squares (sumsq[p * 8 + c],
// p < sumsq_parts), then launch_route's softmax, top-k and plan.  W is the
// F32 router, row-major [E][cols]; counter is zero between launches.
struct RouterArgs {
    const float* x;
    int32_t x_stride;
    const float *gain, *sumsq;
    int32_t sumsq_parts;
    float eps;
    const float* w;
    int32_t cols, E, K, n;
    const float* bias;
    float* logits;
    MoePlan* plan;
    uint32_t* counter;
};
cudaError_t launch_router_route(const RouterArgs& A, cudaStream_t s, bool pdl);
// Expert parallel combine: before reading the expert outputs, wait until
// every rank has raised its flag for this layer (flag value E = *step *
// layers + layer + 1, in flags[(E & 1) * 64 + rank]); the outputs are in the
// buffer of parity E & 1, xstride floats after the parity-0 one.  A wait that
// gives up after wait_ns sets *status and goes on.
struct MoeExchange {
    const uint32_t* flags;
    const uint32_t* step;
    int32_t world, layers, layer;
    size_t xstride;
    int32_t* status;
    uint64_t wait_ns;  // give up after this long (the session's wait limit)
};

// states[i] += sum over client i's experts in ascending id of
// (out[a][pos] * p) / norm  (spm-granite-moe/src/layout.rs:283-302); also the
// sums of squares of the new state rows, in combine_parts(width, n) parts:
// part (i * chunks + chunk) holds [c == i ? ss : 0 for c < 8].
int combine_parts(int width, int n);
// Clients c0..c0+n-1 (their plan rows and state rows); the sums of squares go
// to parts blockIdx.y * chunks + chunk with the value at client c0 + blockIdx.y.
cudaError_t launch_combine(const MoePlan* plan, const float* out, int out_stride, float* states, int width, int n,
                           int used, float* sumsq, const MoeExchange* ex, cudaStream_t s, bool pdl, int c0 = 0);
// Data-parallel attention: gather every rank's greedy picks (ep_gather_kernel).
cudaError_t launch_ep_gather(const uint32_t* argmax, uint32_t* const* peer_argmax, uint32_t* const* peer_flags,
                             const uint32_t* own_flags, const uint32_t* step, int c0, int n, int world, int rank,
                             int32_t* status, uint64_t wait_ns, cudaStream_t s, bool pdl);

}  // namespace spm
