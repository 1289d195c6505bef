// Route and combine kernels of the routed feed-forward (moe.h).
#include "device.cuh"
#include "moe.h"

namespace spm {
namespace {
using namespace dev;

// f32::total_cmp order key (spm-granite-moe/src/math.rs:35-39 sorts by it).
__device__ __forceinline__ int32_t total_key(float f) {
    int32_t b = __float_as_int(f);
    return b ^ int32_t(uint32_t(b >> 31) >> 1);
}

// One CTA.  Warp i routes client i with its probabilities in registers
// (lane l holds experts l, l + 32, ..., NV of them); then the plan is built
// from a bitmap of each expert's clients.
//
// Selection: each round every lane offers its largest untaken probability
// (by f32::total_cmp order key, the lower id among equals), the warp agrees
// on the largest key and then on the lowest id holding it with two
// redux.sync reductions, and the owner marks it taken -- the same routes as a
// scan of all experts per round, in far fewer dependent steps.
struct RouteSmem {
    int32_t sel[kMoeMaxClients][kMoeMaxUsed];
    float psel[kMoeMaxClients][kMoeMaxUsed];
    uint32_t cmask[kMoeMaxExperts];  // bit i: client i routes to the expert
    int32_t base[kMoeMaxExperts];
};

// The routing of all n clients by one CTA of 256 threads.  CG: the logits
// were written by other CTAs of this launch (read past L1).
template <int NV, bool CG>
__device__ void route_block(const float* logits, const float* bias, int n, int E, int K, int world, int rank,
                            MoePlan* plan, RouteSmem& S) {
    auto& sel = S.sel;
    auto& psel = S.psel;
    auto& cmask = S.cmask;
    auto& base = S.base;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = threadIdx.x; e < E; e += blockDim.x) cmask[e] = 0;
    __syncthreads();
    if (warp < n) {
        const int i = warp;
        float p[NV];
        // softmax: max by fold, exp(v - max), sum, divide (math.rs:23-29)
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const int e = lane + 32 * j;
            p[j] = -INFINITY;
            if (e < E) {
                const float lg = CG ? __ldcg(logits + i * E + e) : logits[i * E + e];
                p[j] = bias ? lg + bias[e] : lg;
                mx = fmaxf(mx, p[j]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < NV; j++)
            if (lane + 32 * j < E) {
                p[j] = expf(p[j] - mx);
                sum += p[j];
            }
        sum = warp_sum(sum);
        int32_t key[NV];
#pragma unroll
        for (int j = 0; j < NV; j++) {
            p[j] = __fdiv_rn(p[j], sum);
            key[j] = lane + 32 * j < E ? total_key(p[j]) : INT32_MIN;
        }
        // top-K: largest probability first, the lower id among equals
        uint32_t taken = 0;
        float mine = 0.f;  // lane r < K: probability and expert of route r
        int myid = 0;
        for (int r = 0; r < K; r++) {
            int32_t bk = INT32_MIN;
            int bj = -1;
#pragma unroll
            for (int j = 0; j < NV; j++)
                if (lane + 32 * j < E && !((taken >> j) & 1u) && (bj < 0 || key[j] > bk)) {
                    bk = key[j];
                    bj = j;
                }
            const int32_t m = __reduce_max_sync(0xffffffffu, bk);
            const int win = __reduce_min_sync(0xffffffffu, bj >= 0 && bk == m ? lane + 32 * bj : INT32_MAX);
            float pw = 0.f;
            if ((win & 31) == lane) {
                taken |= 1u << (win >> 5);
#pragma unroll
                for (int j = 0; j < NV; j++)
                    if (j == (win >> 5)) pw = p[j];
            }
            pw = __shfl_sync(0xffffffffu, pw, win & 31);
            if (lane == r) {
                mine = pw;
                myid = win;
            }
        }
        // the largest probability left out, for the routing's margin
        float best = -INFINITY;
#pragma unroll
        for (int j = 0; j < NV; j++)
            if (lane + 32 * j < E && !((taken >> j) & 1u)) best = fmaxf(best, p[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
        const float pk = __shfl_sync(0xffffffffu, mine, K - 1);
        if (lane < K) {
            sel[i][lane] = myid;
            psel[i][lane] = mine;
            atomicOr(&cmask[myid], 1u << i);
            plan->route[i][lane] = myid;
        }
        // the renormaliser, in route order (layout.rs:289-293)
        float s = 0.f;
        for (int r = 0; r < K; r++) s += __shfl_sync(0xffffffffu, mine, r);
        if (lane == 0) {
            plan->norm[i] = s;
            plan->gap[i] = best == -INFINITY ? 1.0f : (pk - best) / pk;
        }
    }
    __syncthreads();
    // ---- plan: active experts ascending, their clients ascending ----
    // active index of every expert: exclusive prefix count of the experts
    // with a client, 32 experts per step by ballot
    if (warp == 0) {
        int run = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const bool act = e < E && cmask[e] != 0;
            const uint32_t m = __ballot_sync(0xffffffffu, act);
            if (e < E) base[e] = run + __popc(m & ((1u << lane) - 1u));
            run += __popc(m);
        }
        if (lane == 0) plan->count = run;
    } else if (warp == 1) {
        // this rank's active experts, by the same ballot scan
        int run = 0, local = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const bool act = e < E && cmask[e] != 0;
            const bool own = act && e % world == rank;
            const uint32_t ma = __ballot_sync(0xffffffffu, act), mo = __ballot_sync(0xffffffffu, own);
            if (own) plan->local[local + __popc(mo & ((1u << lane) - 1u))] = run + __popc(ma & ((1u << lane) - 1u));
            run += __popc(ma);
            local += __popc(mo);
        }
        if (lane == 0) plan->nlocal = local;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
        uint32_t m = cmask[e];
        if (!m) continue;
        const int a = base[e];
        plan->expert[a] = e;
        plan->ntok[a] = __popc(m);
        int q = 0;
        for (; m; m &= m - 1u) plan->tok[a][q++] = __ffs(m) - 1;
        for (; q < kMoeMaxClients; q++) plan->tok[a][q] = 0;
    }
    if (threadIdx.x < n) {
        // this client's routes in ascending expert id: route j goes to place
        // rank_j = the number of its routes with a lower expert id
        const int i = threadIdx.x;
        int32_t ids[kMoeMaxUsed];
#pragma unroll
        for (int j = 0; j < kMoeMaxUsed; j++) ids[j] = sel[i][j < K ? j : 0];
#pragma unroll
        for (int j = 0; j < kMoeMaxUsed; j++) {
            if (j >= K) break;
            int rk = 0;
#pragma unroll
            for (int x = 0; x < kMoeMaxUsed; x++) rk += (x < K && ids[x] < ids[j]) ? 1 : 0;
            plan->slot_a[i][rk] = base[ids[j]];
            // its place among the expert's clients (clients ascending)
            plan->slot_pos[i][rk] = __popc(cmask[ids[j]] & ((1u << i) - 1u));
            plan->slot_p[i][rk] = psel[i][j];
        }
    }
}

template <int NV>
__global__ void __launch_bounds__(256) route_kernel(const float* logits, const float* bias, int n, int E, int K,
                                                    int world, int rank, MoePlan* plan) {
    __shared__ RouteSmem S;
    pdl_wait();
    route_block<NV, false>(logits, bias, n, E, K, world, rank, plan, S);
    pdl_trigger();
}

// Router logits and routing in one launch (one GPU).  CTA e computes expert
// e's logit of every client: warp c walks client c's state, normalised on
// load (x * gain, the RMSNorm scale applied to the sum), against row e of the
// F32 router, lane l taking columns 4l + 128j; the warp's sum in butterfly
// order times the scale is the logit.  The last CTA to finish (a launch
// counter that returns to zero) routes: route_block over the logits the
// other CTAs wrote.
template <int NV>
__global__ void __launch_bounds__(256) router_route_kernel(const RouterArgs A) {
    __shared__ RouteSmem S;
    __shared__ int last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, e = int(blockIdx.x);
    const float* wr = A.w + size_t(e) * A.cols;
    pdl_wait();
    if (warp < A.n) {
        const int c = warp;
        // the client's RMSNorm scale from the producer's per-CTA sums of
        // squares, added in the streaming GEMV's order
        const float* sp = A.sumsq + c;
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int p = lane;
        for (; p + 96 < A.sumsq_parts; p += 128) {
            a0 += sp[p * 8];
            a1 += sp[(p + 32) * 8];
            a2 += sp[(p + 64) * 8];
            a3 += sp[(p + 96) * 8];
        }
        for (; p < A.sumsq_parts; p += 32) a0 += sp[p * 8];
        const float ssum = warp_sum((a0 + a1) + (a2 + a3));
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssum, float(A.cols)), A.eps)));
        const float* xr = A.x + size_t(c) * A.x_stride;
        float acc = 0.f;
#pragma unroll 4
        for (int col = lane * 4; col < A.cols; col += 128) {
            const float4 w = ldx4(wr + col), x = ldx4(xr + col), g = ldx4(A.gain + col);
            acc = fmaf(w.x, __fmul_rn(x.x, g.x), acc);
            acc = fmaf(w.y, __fmul_rn(x.y, g.y), acc);
            acc = fmaf(w.z, __fmul_rn(x.z, g.z), acc);
            acc = fmaf(w.w, __fmul_rn(x.w, g.w), acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) A.logits[c * A.E + e] = acc * scale;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(A.counter, 1u);
        last = prev + 1 == gridDim.x;
        if (last) *A.counter = 0;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    route_block<NV, true>(A.logits, A.bias, A.n, A.E, A.K, 1, 0, A.plan, S);
    pdl_trigger();
}

// Grid (column chunk, client): a CTA of kCombineCols threads adds one column
// per thread, and writes its chunk's sum of squares as its own part.
constexpr int kCombineCols = 128;

__global__ void __launch_bounds__(kCombineCols) combine_kernel(const MoePlan* plan, const float* out, int out_stride,
                                                               float* states, int width, int K, float* sumsq,
                                                               MoeExchange ex, int c0) {
    __shared__ float red[kCombineCols / 32];
    pdl_wait();
    if (ex.world > 1) {
        // every rank's expert rows for this layer are in place once all flags are up
        const uint32_t E = *ex.step * uint32_t(ex.layers) + uint32_t(ex.layer) + 1;
        if (threadIdx.x < uint32_t(ex.world)) {
            const uint32_t* f = ex.flags + (E & 1u) * 64 + threadIdx.x;
            if (ld_acquire_sys(f) != E) {
                const uint64_t t0 = now_ns();
                while (ld_acquire_sys(f) != E)
                    if (now_ns() - t0 > ex.wait_ns) {
                        flag(ex.status, 5);
                        break;
                    }
            }
        }
        __syncthreads();
        out += (E & 1u) * ex.xstride;
    }
    const int i = c0 + int(blockIdx.y), col = blockIdx.x * kCombineCols + threadIdx.x;
    float ss = 0.f;
    if (col < width) {
        const float norm = plan->norm[i];
        // the K expert rows' values first (their loads in flight together),
        // then the sum in ascending expert id
        float vals[kMoeMaxUsed], ps[kMoeMaxUsed];
#pragma unroll
        for (int j = 0; j < kMoeMaxUsed; j++) {
            vals[j] = ps[j] = 0.f;
            if (j < K) {
                const float* lane =
                    out + size_t(plan->slot_a[i][j] * kMoeMaxClients + plan->slot_pos[i][j]) * out_stride;
                vals[j] = __ldcg(lane + col);
                ps[j] = plan->slot_p[i][j];
            }
        }
        float total = 0.f;
#pragma unroll
        for (int j = 0; j < kMoeMaxUsed; j++)
            if (j < K) total = total + __fdiv_rn(__fmul_rn(vals[j], ps[j]), norm);
        const float v = states[size_t(i) * width + col] + total;
        states[size_t(i) * width + col] = v;
        ss = v * v;
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    pdl_trigger();
    if (threadIdx.x < 8) {
        float t = 0.f;
        for (int w = 0; w < kCombineCols / 32; w++) t += red[w];
        sumsq[(size_t(blockIdx.y) * gridDim.x + blockIdx.x) * 8 + threadIdx.x] = int(threadIdx.x) == i ? t : 0.f;
    }
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, cudaStream_t s, bool pdl, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// Data-parallel attention: each rank picked the greedy tokens of its own
// clients c0..c0+n-1.  Thread p copies them into rank p's array and raises
// this rank's flag there (value *step + 1), then thread p waits until rank
// p's flag is up here (bounded; status 9), so every rank ends the step with
// every client's pick.
__global__ void ep_gather_kernel(const uint32_t* argmax, uint32_t* const* peer_argmax, uint32_t* const* peer_flags,
                                 const uint32_t* own_flags, const uint32_t* step, int c0, int n, int world, int rank,
                                 int32_t* status, uint64_t wait_ns) {
    pdl_wait();
    const uint32_t E = *step + 1;
    const int p = int(threadIdx.x);
    if (p < world) {
        for (int c = 0; c < n; c++) peer_argmax[p][c0 + c] = argmax[c0 + c];
        __threadfence_system();
        st_release_sys(peer_flags[p] + rank, E);
        if (ld_acquire_sys(own_flags + p) != E) {
            const uint64_t t0 = now_ns();
            while (ld_acquire_sys(own_flags + p) != E)
                if (now_ns() - t0 > wait_ns) {
                    flag(status, 9);
                    break;
                }
        }
    }
    __syncthreads();
    pdl_trigger();
}

}  // namespace

cudaError_t launch_ep_gather(const uint32_t* argmax, uint32_t* const* peer_argmax, uint32_t* const* peer_flags,
                             const uint32_t* own_flags, const uint32_t* step, int c0, int n, int world, int rank,
                             int32_t* status, uint64_t wait_ns, cudaStream_t s, bool pdl) {
    void* args[] = {&argmax, &peer_argmax, &peer_flags, &own_flags, &step, &c0, &n, &world, &rank, &status, &wait_ns};
    return launch_pdl(reinterpret_cast<const void*>(ep_gather_kernel), dim3(1), dim3(32), s, pdl, args);
}

cudaError_t launch_route(const float* logits, const float* bias, int n, int experts, int used, int world, int rank,
                         MoePlan* plan, cudaStream_t s, bool pdl) {
    if (n < 1 || n > kMoeMaxClients || experts < 1 || experts > kMoeMaxExperts || used < 1 || used > kMoeMaxUsed ||
        used > experts)
        return cudaErrorInvalidValue;
    if (world < 1 || rank < 0 || rank >= world) return cudaErrorInvalidValue;
    void* args[] = {&logits, &bias, &n, &experts, &used, &world, &rank, &plan};
    const void* fn = experts <= 64    ? reinterpret_cast<const void*>(route_kernel<2>)
                     : experts <= 128 ? reinterpret_cast<const void*>(route_kernel<4>)
                                      : reinterpret_cast<const void*>(route_kernel<8>);
    return launch_pdl(fn, dim3(1), dim3(256), s, pdl, args);
}

cudaError_t launch_router_route(const RouterArgs& A, cudaStream_t s, bool pdl) {
    if (A.n < 1 || A.n > kMoeMaxClients || A.E < 1 || A.E > kMoeMaxExperts || A.K < 1 || A.K > kMoeMaxUsed ||
        A.K > A.E || A.cols < 4 || A.cols % 4)
        return cudaErrorInvalidValue;
    RouterArgs a = A;
    void* args[] = {&a};
    const void* fn = A.E <= 64    ? reinterpret_cast<const void*>(router_route_kernel<2>)
                     : A.E <= 128 ? reinterpret_cast<const void*>(router_route_kernel<4>)
                                  : reinterpret_cast<const void*>(router_route_kernel<8>);
    return launch_pdl(fn, dim3(A.E), dim3(256), s, pdl, args);
}

int combine_parts(int width, int n) { return ((width + kCombineCols - 1) / kCombineCols) * n; }

cudaError_t launch_combine(const MoePlan* plan, const float* out, int out_stride, float* states, int width, int n,
                           int used, float* sumsq, const MoeExchange* ex, cudaStream_t s, bool pdl, int c0) {
    MoeExchange e = ex ? *ex : MoeExchange{};
    if (!ex) e.world = 1;
    void* args[] = {&plan, &out, &out_stride, &states, &width, &used, &sumsq, &e, &c0};
    return launch_pdl(reinterpret_cast<const void*>(combine_kernel), dim3((width + kCombineCols - 1) / kCombineCols, n),
                      dim3(kCombineCols), s, pdl, args);
}

}  // namespace spm
