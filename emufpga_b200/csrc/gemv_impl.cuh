// The streamed dequant-GEMV: y[p][r] = sum_c W[r][c] * x[p][c] for up to 8
// clients p off ONE pass over the packed weights (host_pack.cpp layout).
//
// Each CTA owns a contiguous run of 4-row tiles and streams them through a
// shared-memory ring with cp.async.bulk (one copy per tile, or per gate/up
// pair, completing on an mbarrier).  The CTA's warps form groups of
// `group_warps` warps; group g works on the CTA's tiles g, g+G, g+2G, ...
// with its lanes split over the 32-weight units of the tile's rows.  There is
// no producer warp: the group that finishes a slot refills it with the tile
// NS further on, so all warps compute and none idles waiting on the ring.
// Short rows (SmolLM2: 18 units) take one warp per tile; long rows spread a
// tile over several warps so that every lane has one to four units.
//
// Per unit a lane unpacks the rows' codes into bytes (four per word) and
// applies them to every client's staged activations.  The activations are
// staged once per CTA in shared memory as 22-bit fixed point per 32-value
// unit (a power-of-two scale and three planes of 8-bit digits), so that four
// codes times four activations are three dp4a, exact in int32 -- the
// reference's "one weight, every position" schedule
// (spm-linear/src/resident.rs:120-137) with the multiply-adds in integer
// units.  Block scales are applied once per sub-block in fp32:
//     sum_c w_c x_c = (d*sc) * s * sum_c q_c m_c  [- (dmin*m or 32 d*sc) * sum_c x_c]
// which is the reference dot product regrouped, with x_c = s * m_c rounded
// to 22 bits below the unit's largest |x| (2^-23 of it at most).  The
// weights are the reference's bit for bit (the dequant kernel checks that);
// the sums are in a different order than the reference's fp32 FMA chain.
// F32 matrices (the MoE router) keep fp32 activations and FMAs.
//
// A lane's partial sums for the pass's rows and clients are reduced across
// the warp by a transposing butterfly (each exchange halves the values a lane
// holds), so that afterwards lane l owns one (row, client) total; groups of
// several warps add their warps' totals through shared memory, in warp order.
// All sums are in a fixed order: results do not depend on timing.
//
// A fused RMSNorm multiplies the staged activations by the gain and applies
// the client's scale 1/sqrt(mean + eps) to the dot product:
// s * sum_c w_c (x_c g_c), the reference's sum_c w_c ((x_c s) g_c) with the
// scale factored out.
//
// Launched with programmatic dependent launch: the ring is filled while the
// previous kernel still runs (weights never depend on it), and the
// activations are read only after griddepcontrol.wait.
#pragma once
#include <type_traits>

#include "device.cuh"
#include "moe.h"

namespace spm {
namespace gemv {
using namespace dev;

constexpr int kMaxWarps = 16;             // warps of a CTA that has an SM to itself
constexpr int kPairWarps = 8;             // warps of each of two CTAs sharing an SM
constexpr int kMaxSlots = 16;
constexpr size_t kSmemMax = 200 * 1024;   // dynamic shared memory of a CTA alone on its SM
// Dynamic shared memory of each of two CTAs per SM: half of the SM's 228 KB,
// less each CTA's static arrays (5.25 KB) and the 1 KB the system reserves.
constexpr size_t kHalfSm = 107 * 1024;
constexpr int kAuxPrefetch = 1024;        // residual values prefetched per CTA, at most
// Staged activations of the integer block types: per client one 112-byte
// record per 32-value unit -- three planes of 32 signed 8-bit digits (8 words
// each), then the unit's scale s and the two 16-value sums of the staged
// values.  The unit's values x are held as m * s, m = rint(x / s) with
// s = 2^(e-22) and max|x| < 2^e, so |m| <= 2^22 and m = d0 + 256 d1 + 65536 d2
// with every digit in [-128, 127]: 22 significant bits against the unit's
// largest value.  A code word (four codes as bytes) times a digit word is one
// dp4a, exact in int32, so sum_c q_c m_c needs three dp4a per four codes and
// one conversion to float per (sub-)block.  F32 weights keep 144-byte records
// of the values themselves (128 bytes, two sums, padding).  Both strides put
// the records of consecutive units 4 banks apart, so the lanes of a
// quarter-warp reading the same part of consecutive units share no bank.
constexpr uint32_t kDigitUnit = 112;
constexpr uint32_t kFloatUnit = 144;
inline __host__ __device__ constexpr uint32_t unit_bytes(int enc) { return enc == SPM_F32 ? kFloatUnit : kDigitUnit; }
// Q8_0 with four or more clients takes the tensor-core inner loop
// (gemv_tc.cuh); its records hold each plane's words in the order
// 0,4,1,5,2,6,3,7, so that lane t reads words t and 4+t with one 8-byte load.
// (Measured on B200: for the K-quants, whose scales change every 16 or 32
// values, the per-sub-block fp32 work that the tensor-core loop keeps on the
// CUDA cores makes it no faster than the dp4a loop even with eight clients.)
inline __host__ __device__ constexpr bool use_tc(int enc, int n) { return enc == SPM_Q8_0 && n >= 4; }
// The K-quants with four or more clients (dense and expert launches) take the
// other tensor-core loop (gemv_tc.cuh: codes as the A operand, sixteen rows
// per product, the clients as the eight columns); a slot then holds four
// tiles, or two gate and two up tiles.
// Tiles of a TC2 slot start kTc2Skew bytes after the previous one ends, so
// that rows of different tiles read by one instruction fall on different banks.
constexpr uint32_t kTc2Skew = 64;
inline __host__ __device__ constexpr bool use_tc2(int enc, int n) {
    return (enc == SPM_Q5_K || enc == SPM_Q6_K || enc == SPM_Q2_K) && n >= 4;
}
// Bytes between two clients' records.  The tensor-core loop reads 8 bytes of
// eight clients at once; a stride of 32 mod 128 bytes keeps them on
// different banks.
inline __host__ __device__ uint32_t client_stride(uint32_t unit, bool tc, uint32_t units) {
    const uint32_t c = units * unit;
    return tc ? c + (160u - c % 128u) % 128u : c;
}

struct XUnit {
    uint32_t d[3][8];  // digit planes, word k = values 4k..4k+3
    float s, sum0, sum1;
};

template <int NC>
struct XDig {
    uint32_t base[NC];  // shared address of client c's records
    int nact;           // clients with data (expert mode: the expert's clients); later ones are skipped
    __device__ __forceinline__ void unit(uint32_t u, int c, XUnit& o) const {
        const uint32_t a = base[c] + u * kDigitUnit;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            const uint4 v0 = lds128(a + j * 32), v1 = lds128(a + j * 32 + 16);
            o.d[j][0] = v0.x, o.d[j][1] = v0.y, o.d[j][2] = v0.z, o.d[j][3] = v0.w;
            o.d[j][4] = v1.x, o.d[j][5] = v1.y, o.d[j][6] = v1.z, o.d[j][7] = v1.w;
        }
        const uint4 t = lds128(a + 96);
        o.s = __uint_as_float(t.x);
        o.sum0 = __uint_as_float(t.y);
        o.sum1 = __uint_as_float(t.z);
    }
};

template <int NC>
struct XIn {
    uint32_t base[NC];  // shared address of client c's float records
    __device__ __forceinline__ void load(uint32_t u, int off, float4 (&o)[NC]) const {
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const uint4 v = lds128(base[c] + u * kFloatUnit + off * 4);
            o[c] = make_float4(__uint_as_float(v.x), __uint_as_float(v.y), __uint_as_float(v.z), __uint_as_float(v.w));
        }
    }
};

template <int NC>
__device__ __forceinline__ void dot4(float (&s)[NC], float f0, float f1, float f2, float f3, const float4 (&x)[NC]) {
#pragma unroll
    for (int c = 0; c < NC; c++) {
        s[c] = fmaf(f0, x[c].x, s[c]);
        s[c] = fmaf(f1, x[c].y, s[c]);
        s[c] = fmaf(f2, x[c].z, s[c]);
        s[c] = fmaf(f3, x[c].w, s[c]);
    }
}

__device__ __forceinline__ uint32_t word(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

// int8 -> float exactly: 2^23 + (b ^ 128) - (2^23 + 128).
__device__ __forceinline__ float i8f(uint32_t b) { return bytef<0>(b ^ 0x80u) - 8388736.0f; }

template <int R, int NC>
__device__ __forceinline__ void zero(float (&s)[R][NC]) {
#pragma unroll
    for (int v = 0; v < R; v++)
#pragma unroll
        for (int c = 0; c < NC; c++) s[v][c] = 0.f;
}

// Digit sums of four codes (the bytes of q; signed for Q8_0, unsigned for
// the K-quants) times staged word k.
template <bool SIGNED>
__device__ __forceinline__ void dot_digits(uint32_t q, const XUnit& x, int k, int (&S)[3]) {
#pragma unroll
    for (int j = 0; j < 3; j++) S[j] = SIGNED ? dp4a_ss(q, x.d[j][k], S[j]) : dp4a_us(q, x.d[j][k], S[j]);
}
// sum_c q_c m_c from the digit sums (float; the low two planes combined
// exactly in int32 first).
__device__ __forceinline__ float digits_total(const int (&S)[3]) {
    return fmaf(__int2float_rn(S[2]), 65536.0f, __int2float_rn(S[1] * 256 + S[0]));
}

// One row of a pass: shared address of its tile, and its row index r inside
// the tile as r * units and r * super-blocks.
struct RowRef {
    uint32_t t, ru, rb;
};

// Every unit function adds unit u of the rows R times the activations into
// acc[row][client]: the rows' codes are unpacked once, then each client's
// record is read and applied to every row.

// ------------------------------------------------------------------ Q8_0 --
template <int NC, int R>
__device__ __forceinline__ void unit_q8_0(const RowRef (&rr)[R], uint32_t u, const GemvLaunch& L, const XDig<NC>& X,
                                          float (&acc)[R][NC]) {
    uint4 q0[R], q1[R];
    float d[R];
#pragma unroll
    for (int v = 0; v < R; v++) {
        const uint32_t unit = rr[v].ru + u;
        q0[v] = lds128(rr[v].t + unit * 32);
        q1[v] = lds128(rr[v].t + unit * 32 + 16);
        d[v] = h2f(lds16(rr[v].t + L.plane1 + unit * 2));
    }
#pragma unroll
    for (int c = 0; c < NC; c++) {
        if (c >= X.nact) break;
        XUnit xu;
        X.unit(u, c, xu);
#pragma unroll
        for (int v = 0; v < R; v++) {
            int S[3] = {0, 0, 0};
#pragma unroll
            for (int k = 0; k < 8; k++) dot_digits<true>(k < 4 ? word(q0[v], k) : word(q1[v], k - 4), xu, k, S);
            // sum w x = d * s * sum q m
            acc[v][c] = fmaf(d[v] * xu.s, digits_total(S), acc[v][c]);
        }
    }
}

// ------------------------------------------------------------------ Q6_K --
template <int NC, int R>
__device__ __forceinline__ void unit_q6_k(const RowRef (&rr)[R], uint32_t u, const GemvLaunch& L, const XDig<NC>& X,
                                          float (&acc)[R][NC]) {
    uint32_t q[R][8];  // 6-bit codes as bytes; word 4*run + k = values 16*run + 4k ..
    float ds[R][2];
#pragma unroll
    for (int v = 0; v < R; v++) {
        const uint32_t unit = rr[v].ru + u;
        const uint4 ql = lds128(rr[v].t + unit * 16);
        const uint2 qh = lds64(rr[v].t + L.plane1 + unit * 8);
        const uint32_t sc = lds16(rr[v].t + L.plane2 + unit * 2);
        const float d = h2f(lds16(rr[v].t + L.plane3 + (rr[v].rb + (u >> 3)) * 2));
        ds[v][0] = d * i8f(sc & 0xffu);
        ds[v][1] = d * i8f(sc >> 8);
#pragma unroll
        for (int run = 0; run < 2; run++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t w = word(ql, k);
                const uint32_t h = run ? qh.y : qh.x;
                const uint32_t hs = (k < 2 ? h << (4 - 2 * k) : h >> (2 * k - 4)) & 0x30303030u;
                q[v][4 * run + k] = ((run ? (w >> 4) : w) & 0x0F0F0F0Fu) | hs;
            }
    }
#pragma unroll
    for (int c = 0; c < NC; c++) {
        if (c >= X.nact) break;
        XUnit xu;
        X.unit(u, c, xu);
        const float o0 = -32.0f * xu.sum0, o1 = -32.0f * xu.sum1;
#pragma unroll
        for (int v = 0; v < R; v++)
#pragma unroll
            for (int run = 0; run < 2; run++) {
                int S[3] = {0, 0, 0};
#pragma unroll
                for (int k = 0; k < 4; k++) dot_digits<false>(q[v][4 * run + k], xu, 4 * run + k, S);
                // sum (q - 32) x = s * sum q m - 32 * sum x
                acc[v][c] = fmaf(ds[v][run], fmaf(digits_total(S), xu.s, run ? o1 : o0), acc[v][c]);
            }
    }
}

// ------------------------------------------------------------------ Q5_K --

template <int NC, int R>
__device__ __forceinline__ void unit_q5_k(const RowRef (&rr)[R], uint32_t u, const GemvLaunch& L, const XDig<NC>& X,
                                          float (&acc)[R][NC]) {
    uint32_t q[R][8];  // 5-bit codes as bytes
    float ds[R], dm[R];
#pragma unroll
    for (int v = 0; v < R; v++) {
        const uint32_t unit = rr[v].ru + u;
        const uint4 qs = lds128(rr[v].t + unit * 16);
        const uint32_t qh = lds32(rr[v].t + L.plane1 + unit * 4);
        const uint32_t sm = lds16(rr[v].t + L.plane2 + unit * 2);
        const uint32_t dd = lds32(rr[v].t + L.plane3 + (rr[v].rb + (u >> 3)) * 4);
        ds[v] = h2f(dd) * (bytef<0>(sm) - 8388608.0f);
        dm[v] = h2f(dd >> 16) * (bytef<1>(sm) - 8388608.0f);
#pragma unroll
        for (int run = 0; run < 2; run++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t w = word(qs, k);
                const uint32_t sp = (((qh >> (16 * run + 4 * k)) & 0xfu) * 0x02040810u) & 0x10101010u;
                q[v][4 * run + k] = ((run ? (w >> 4) : w) & 0x0F0F0F0Fu) | sp;
            }
    }
#pragma unroll
    for (int c = 0; c < NC; c++) {
        if (c >= X.nact) break;
        XUnit xu;
        X.unit(u, c, xu);
        const float xsum = xu.sum0 + xu.sum1;
#pragma unroll
        for (int v = 0; v < R; v++) {
            int S[3] = {0, 0, 0};
#pragma unroll
            for (int k = 0; k < 8; k++) dot_digits<false>(q[v][k], xu, k, S);
            // sum w x = ds * s * sum q m - dm * sum x
            acc[v][c] = fmaf(-dm[v], xsum, fmaf(ds[v], digits_total(S) * xu.s, acc[v][c]));
        }
    }
}

// ------------------------------------------------------------------ Q2_K --
template <int NC, int R>
__device__ __forceinline__ void unit_q2_k(const RowRef (&rr)[R], uint32_t u, const GemvLaunch& L, const XDig<NC>& X,
                                          float (&acc)[R][NC]) {
    uint2 qs[R];
    float dl[R][2], ml[R][2];
#pragma unroll
    for (int v = 0; v < R; v++) {
        const uint32_t unit = rr[v].ru + u;
        qs[v] = lds64(rr[v].t + unit * 8);
        const uint32_t sc = lds16(rr[v].t + L.plane1 + unit * 2);
        const uint32_t dd = lds32(rr[v].t + L.plane2 + (rr[v].rb + (u >> 3)) * 4);
        const float d = h2f(dd), dmin = h2f(dd >> 16);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t b = (sc >> (8 * h)) & 0xffu;
            dl[v][h] = d * (bytef<0>(b & 15u) - 8388608.0f);
            ml[v][h] = dmin * (bytef<0>(b >> 4) - 8388608.0f);
        }
    }
#pragma unroll
    for (int c = 0; c < NC; c++) {
        if (c >= X.nact) break;
        XUnit xu;
        X.unit(u, c, xu);
#pragma unroll
        for (int v = 0; v < R; v++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                int S[3] = {0, 0, 0};
#pragma unroll
                for (int k = 0; k < 4; k++)
                    dot_digits<false>(((h ? qs[v].y : qs[v].x) >> (2 * k)) & 0x03030303u, xu, 4 * h + k, S);
                // sum w x = dl * s * sum q m - ml * sum x
                acc[v][c] = fmaf(-ml[v][h], h ? xu.sum1 : xu.sum0, fmaf(dl[v][h], digits_total(S) * xu.s, acc[v][c]));
            }
    }
}

// ------------------------------------------------------------------- F32 --
template <int NC, int R>
__device__ __forceinline__ void unit_f32(const RowRef (&rr)[R], uint32_t u, const GemvLaunch& L, const XIn<NC>& X,
                                         float (&acc)[R][NC]) {
#pragma unroll
    for (int k = 0; k < 8; k++) {
        float4 x[NC];
        X.load(u, 4 * k, x);
#pragma unroll
        for (int v = 0; v < R; v++) {
            const uint4 w = lds128(rr[v].t + (rr[v].ru + u) * 128 + 16 * k);
            dot4<NC>(acc[v], __uint_as_float(w.x), __uint_as_float(w.y), __uint_as_float(w.z), __uint_as_float(w.w),
                     x);
        }
    }
}

#include "gemv_tc.cuh"

template <int ENC, int NC, int R, class XT>
__device__ __forceinline__ void unit_dot(const RowRef (&rr)[R], uint32_t u, const GemvLaunch& L, const XT& X,
                                         float (&acc)[R][NC]) {
    if constexpr (ENC == SPM_Q8_0) unit_q8_0<NC, R>(rr, u, L, X, acc);
    else if constexpr (ENC == SPM_Q6_K) unit_q6_k<NC, R>(rr, u, L, X, acc);
    else if constexpr (ENC == SPM_Q5_K) unit_q5_k<NC, R>(rr, u, L, X, acc);
    else if constexpr (ENC == SPM_Q2_K) unit_q2_k<NC, R>(rr, u, L, X, acc);
    else unit_f32<NC, R>(rr, u, L, X, acc);
}

__device__ __forceinline__ float silu_mul(float g, float u) { return __fdiv_rn(g, 1.0f + expf(-g)) * u; }

// Expert parallel: the launch's CTA counter.  The last CTA to arrive raises
// this rank's flag in every rank's flag array.  One thread per CTA calls it,
// after the CTA's stores to the ranks' buffers are fenced at system scope.
__device__ __forceinline__ void ep_arrive(const GemvLaunch& L) {
    const uint32_t prev = atomicAdd(L.ep_done, 1u);
    if (prev + 1 == gridDim.x) {
        *L.ep_done = 0;
        __threadfence_system();
        const uint32_t E = *L.ep_step * uint32_t(L.ep_layers) + uint32_t(L.ep_layer) + 1;
        const uint32_t par = E & 1u;
        for (int p = 0; p < L.world; p++) st_release_sys(L.ep_peer_flag[par * L.world + p], E);
    }
}

// The job of global tile g, from the CTA's shared copy of the job table.
__device__ __forceinline__ const GemvJob& pick(const GemvJob* jobs, int njobs, uint32_t g) {
    if (njobs > 3 && g >= jobs[3].tile_begin) return jobs[3];
    if (njobs > 2 && g >= jobs[2].tile_begin) return jobs[2];
    if (njobs > 1 && g >= jobs[1].tile_begin) return jobs[1];
    return jobs[0];
}

// Transposing butterfly over the warp: lane values a[0..N) (N a power of two
// <= 32).  Each exchange at distance O keeps half of the values (the upper
// half on lanes with bit O set) and adds the partner's matching half; once a
// lane holds one value the remaining exchanges are plain.  Afterwards a[0] of
// lane l is the warp total of value (l >> (5 - log2 N)).
template <int N, int O>
struct XRed {
    template <int V>
    static __device__ __forceinline__ void run(float (&a)[V], int lane) {
        if constexpr (O > 0) {
            if constexpr (N > 1) {
                constexpr int H = N / 2;
                const bool up = (lane & O) != 0;
#pragma unroll
                for (int j = 0; j < H; j++) {
                    const float send = up ? a[j] : a[j + H];
                    const float keep = up ? a[j + H] : a[j];
                    a[j] = keep + __shfl_xor_sync(0xffffffffu, send, O);
                }
                XRed<H, O / 2>::run(a, lane);
            } else {
                a[0] += __shfl_xor_sync(0xffffffffu, a[0], O);
                XRed<1, O / 2>::run(a, lane);
            }
        }
    }
};

constexpr int log2i(int v) { return v <= 1 ? 0 : 1 + log2i(v / 2); }

// Rows of each matrix per pass: all four rows of a tile in one pass when the
// lane's partial sums and codes fit in registers (one matrix and up to five
// clients, or a gate/up pair for one client), else passes of two rows (or of
// one row of a gate/up pair for more than five clients).
template <int NC, bool DUAL>
struct Shape {
    static constexpr int VR = DUAL ? (NC == 1 ? 4 : NC <= 5 ? 2 : 1) : (NC <= 5 ? 4 : 2);
    static constexpr int PASSES = kTileRows / VR;
    static constexpr int M = DUAL ? 2 : 1;
    static constexpr int NCP = NC <= 1 ? 1 : NC <= 2 ? 2 : NC <= 4 ? 4 : 8;  // clients, padded to 2^k
    static constexpr int V = VR * NCP;                                        // sums per matrix per pass
    static constexpr int SH = 5 - log2i(V);                                   // lane >> SH = sum index
};

// Bytes of dynamic shared memory the kernel uses: `slots` ring slots, the
// staged activations and, for groups of several warps, one 32-float record
// of partial sums per slot, warp of the group and matrix.
inline size_t smem_bytes(const GemvLaunch& L, bool dual, int slots, int group_warps) {
    // a tensor-core slot holds eight rows: two tiles, or one gate/up pair
    const size_t slot = L.tc2 ? 4 * (size_t(L.tile_bytes) + kTc2Skew) : size_t(L.tile_bytes) * (dual || L.tc ? 2 : 1);
    const size_t xb = size_t(L.n) * client_stride(L.xrec, L.tc != 0 || L.tc2 != 0, L.cols / 32);
    const size_t rec = L.tc2 ? 512 : L.tc ? 256 : (dual ? 256 : 128);  // partials per slot and warp
    const size_t pb = group_warps > 1 ? size_t(slots) * group_warps * rec : 0;
    return slot * size_t(slots) + xb + pb;
}

// TCX: the tensor-core loop is allowed (dense Q8_0 launches of four or more
// clients; expert launches skip client slots without data, which only the
// CUDA-core loop can).
template <int ENC, int NC, bool DUAL, bool TCX>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) gemv_stream(const __grid_constant__ GemvLaunch L) {
    using S = Shape<NC, DUAL>;
    constexpr int VR = S::VR, PASSES = S::PASSES, M = S::M, NCP = S::NCP, V = S::V, SH = S::SH;
    constexpr bool TC = TCX && use_tc(ENC, NC);
    constexpr bool PAIR = TC && !DUAL;  // slot = two consecutive tiles
    constexpr bool TC2 = TCX && use_tc2(ENC, NC);
    // tiles of rows per slot: TC2 four (two gate/up pairs), PAIR two, else one
    constexpr uint32_t TPS = TC2 ? (DUAL ? 2u : 4u) : PAIR ? 2u : 1u;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kMaxSlots], ready[kMaxSlots];
    __shared__ float nscale[8];
    __shared__ float auxs[kAuxPrefetch];
    __shared__ float sqw[kMaxWarps][8];
    __shared__ int32_t xrows[8], yrows[8], srows[8];
    __shared__ GemvJob jobs[4];
    __shared__ float* ep_y[8];  // expert parallel: every rank's output buffer for this layer
    const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
    const int W = int(blockDim.x >> 5), gw = L.group_warps, G = W / gw;
    const int grp = warp / gw, wig = warp % gw;
    uint32_t t0, t1;
    uint32_t rbase = 0, rlim = 0xffffffffu;  // expert mode: rows of the expert's matrix
    int n_act = NC;  // clients of this CTA with data (expert mode: the expert's clients)
    if (L.plan) {
        // expert mode: the plan comes from the previous kernel
        pdl_wait();
        // The grid is one wave of CTAs; with nl active experts on this rank
        // each expert's tiles split into C = grid / nl chunks (at least
        // expert_chunks, at most one tile each), and CTA b works on chunk
        // b % C of active expert b / C.
        const int nl = L.plan->nlocal;
        const int C = max(L.expert_chunks, min(int(L.expert_tiles), int(gridDim.x) / max(nl, 1)));
        const int la = int(blockIdx.x) / C, chunk = int(blockIdx.x) % C;
        if (la >= L.plan->nlocal) {
            pdl_trigger();
            if (L.ep_done && threadIdx.x == 0) ep_arrive(L);
            return;
        }
        const int a = L.plan->local[la];
        if (L.ep_peer_y && threadIdx.x < uint32_t(L.world)) {
            const uint32_t E = *L.ep_step * uint32_t(L.ep_layers) + uint32_t(L.ep_layer) + 1;
            ep_y[threadIdx.x] = L.ep_peer_y[(E & 1u) * L.world + threadIdx.x];
        }
        const uint32_t e = uint32_t(L.plan->expert[a]), Te = L.expert_tiles;
        rbase = e * Te * kTileRows;
        rlim = Te * kTileRows;
        t0 = e * Te + uint32_t(uint64_t(Te) * chunk / uint32_t(C));
        t1 = e * Te + uint32_t(uint64_t(Te) * (chunk + 1) / uint32_t(C));
        n_act = L.plan->ntok[a];
        if (threadIdx.x < 8) {
            const int c = int(threadIdx.x);
            const int client = L.plan->tok[a][c < n_act ? c : 0];
            xrows[c] = L.xmode == 0 ? client : a * kMoeMaxClients + c;
            yrows[c] = a * kMoeMaxClients + c;
            srows[c] = client;
        }
    } else {
        const uint32_t T = L.total_tiles, Gd = gridDim.x;
        if (TPS > 1) {  // whole slots per CTA
            const uint32_t P = (T + TPS - 1) / TPS;
            t0 = TPS * uint32_t(uint64_t(P) * blockIdx.x / Gd);
            t1 = min(T, TPS * uint32_t(uint64_t(P) * (blockIdx.x + 1) / Gd));
        } else {
            t0 = uint32_t(uint64_t(T) * blockIdx.x / Gd);
            t1 = uint32_t(uint64_t(T) * (blockIdx.x + 1) / Gd);
        }
        if (threadIdx.x < 8) {
            xrows[threadIdx.x] = int(threadIdx.x);
            yrows[threadIdx.x] = int(threadIdx.x);
            srows[threadIdx.x] = L.c0 + int(threadIdx.x);
        }
        // data-parallel attention: every rank's copy of the output rows
        // (one job; ep_peer_y[p] is rank p's output base, rows from client c0)
        if (L.ep_dense && threadIdx.x < uint32_t(L.world))
            ep_y[threadIdx.x] = L.ep_peer_y[threadIdx.x] + size_t(L.c0) * L.job[0].y_stride;
    }
    const uint32_t nt = (t1 - t0 + TPS - 1) / TPS, NS = uint32_t(L.slots);  // work items (slots to fill)
    // Slot s belongs to group s % G alone (NS is a multiple of G), so each
    // group waits for its slots' phases in order and refills them itself.
    if (NS % uint32_t(G) != 0 || NS > uint32_t(kMaxSlots) || W * 32 != int(blockDim.x) || G * gw != W) {
        if (threadIdx.x == 0) flag(L.status, 3);
        return;
    }
    const uint32_t tile_bytes = L.tile_bytes;
    const uint32_t tile_step = TC2 ? tile_bytes + kTc2Skew : tile_bytes;  // distance between a slot's tiles
    const uint32_t slot_bytes = TC2 ? 4u * tile_step : tile_bytes * (DUAL || PAIR ? 2u : 1u);
    constexpr uint32_t XREC = unit_bytes(ENC);
    const uint32_t U = L.cols >> 5, cstride = client_stride(XREC, TC || TC2, U);
    const uint32_t xoff = NS * slot_bytes, poff = xoff + NC * cstride;  // activations, group partials
    auto issue = [&](uint32_t i) {
        const uint32_t s = i % NS;
        if (TC2) {
            // tiles g.. of the slot (gate/up: the gate tiles, then the up tiles two further on)
            const uint32_t g = t0 + TPS * i, h = min(TPS, t1 - g);
            mbar_expect_tx(&full[s], tile_bytes * h * (DUAL ? 2u : 1u));
            for (uint32_t k = 0; k < h; k++) {
                const GemvJob& J = pick(jobs, L.njobs, g + k);
                const size_t off = size_t(g + k - J.tile_begin) * tile_bytes;
                bulk_g2s(smem + size_t(s) * slot_bytes + k * tile_step, J.a + off, tile_bytes, &full[s]);
                if (DUAL) bulk_g2s(smem + size_t(s) * slot_bytes + (2 + k) * tile_step, J.b + off, tile_bytes, &full[s]);
            }
            return;
        }
        if (PAIR) {
            const uint32_t g = t0 + 2 * i, h = g + 1 < t1 ? 2u : 1u;
            mbar_expect_tx(&full[s], tile_bytes * h);
            for (uint32_t k = 0; k < h; k++) {
                const GemvJob& J = pick(jobs, L.njobs, g + k);
                bulk_g2s(smem + size_t(s) * slot_bytes + k * tile_bytes, J.a + size_t(g + k - J.tile_begin) * tile_bytes,
                         tile_bytes, &full[s]);
            }
            return;
        }
        const uint32_t g = t0 + i;
        const GemvJob& J = pick(jobs, L.njobs, g);
        const size_t off = size_t(g - J.tile_begin) * tile_bytes;
        mbar_expect_tx(&full[s], slot_bytes);
        bulk_g2s(smem + size_t(s) * slot_bytes, J.a + off, tile_bytes, &full[s]);
        if (DUAL) bulk_g2s(smem + size_t(s) * slot_bytes + tile_bytes, J.b + off, tile_bytes, &full[s]);
    };
    if (threadIdx.x < 4) jobs[threadIdx.x] = L.job[threadIdx.x];
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&ready[s], uint32_t(gw));
        }
        mbar_fence_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < NS && i < nt; i++) issue(i);
        pdl_trigger();
    }
    pdl_wait();  // activations and norm partials come from the previous kernel
    if (L.ep_wait_flags) {
        // the other ranks' rows and sums of squares of this layer must be in place
        const uint32_t E = *L.ep_step * uint32_t(L.ep_layers) + uint32_t(L.ep_layer) + 1;
        if (threadIdx.x < uint32_t(L.world)) {
            const uint32_t* f = L.ep_wait_flags + (E & 1u) * 64 + threadIdx.x;
            if (ld_acquire_sys(f) != E) {
                const uint64_t w0 = now_ns();
                while (ld_acquire_sys(f) != E)
                    if (now_ns() - w0 > L.wait_ns) {
                        flag(L.status, 8);
                        break;
                    }
            }
        }
        __syncthreads();
    }

    // ---- prologue: norm scales, staged activations, residual prefetch ----
    for (int cw = warp; L.gain && cw < NC; cw += W) {
        // warp cw adds client cw's per-CTA sums of squares, 32 lanes in parallel
        const float* sp = L.sumsq + srows[cw];
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int p = lane;
        for (; p + 96 < L.sumsq_parts; p += 128) {
            a0 += sp[p * 8];
            a1 += sp[(p + 32) * 8];
            a2 += sp[(p + 64) * 8];
            a3 += sp[(p + 96) * 8];
        }
        for (; p < L.sumsq_parts; p += 32) a0 += sp[p * 8];
        const float ssum = warp_sum((a0 + a1) + (a2 + a3));
        if (lane == 0) nscale[cw] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ssum, float(L.cols)), L.eps)));
    }
    if constexpr (ENC == SPM_F32) {
        // float records: 16 values per thread
        const uint32_t h16 = L.cols >> 4;
        for (uint32_t idx = threadIdx.x; idx < NC * h16; idx += blockDim.x) {
            const uint32_t c = idx / h16, h = idx % h16, col = h * 16;
            float4 v[4];
            if (int(c) < n_act) {
                const float* xp = L.x + size_t(xrows[c]) * L.x_stride + col;
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = ldx4(xp + 4 * k);
            } else {
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (L.gain) {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const float4 g = ldx4(L.gain + col + 4 * k);
                    v[k] = make_float4(__fmul_rn(v[k].x, g.x), __fmul_rn(v[k].y, g.y), __fmul_rn(v[k].z, g.z),
                                       __fmul_rn(v[k].w, g.w));
                }
            }
            uint8_t* rec = smem + xoff + c * cstride + (h >> 1) * XREC;
#pragma unroll
            for (int k = 0; k < 4; k++) reinterpret_cast<float4*>(rec + (h & 1) * 64)[k] = v[k];
        }
    } else {
        // digit records: each pair of lanes holds one unit, 16 values each,
        // and agrees on the unit's exponent through a shuffle (whole warps
        // step through the loop together so that every lane shuffles)
        const uint32_t total = uint32_t(n_act) * U * 2;  // records of slots without data are never read
        for (uint32_t w0 = uint32_t(warp) * 32; w0 < total; w0 += blockDim.x) {
            const uint32_t idx = w0 + uint32_t(lane);
            const bool live = idx < total;
            const uint32_t c = live ? idx / (2 * U) : 0, u = (idx % (2 * U)) >> 1, half = idx & 1;
            const uint32_t col = u * 32 + half * 16;
            float v[16];
#pragma unroll
            for (int k = 0; k < 16; k++) v[k] = 0.f;
            if (live && int(c) < n_act) {
                const float* xp = L.x + size_t(xrows[c]) * L.x_stride + col;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const float4 t = ldx4(xp + 4 * k);
                    v[4 * k] = t.x, v[4 * k + 1] = t.y, v[4 * k + 2] = t.z, v[4 * k + 3] = t.w;
                }
                if (L.gain)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const float4 g = ldx4(L.gain + col + 4 * k);
                        v[4 * k] = __fmul_rn(v[4 * k], g.x), v[4 * k + 1] = __fmul_rn(v[4 * k + 1], g.y);
                        v[4 * k + 2] = __fmul_rn(v[4 * k + 2], g.z), v[4 * k + 3] = __fmul_rn(v[4 * k + 3], g.w);
                    }
            }
            float mx = 0.f;
#pragma unroll
            for (int k = 0; k < 16; k++) mx = fmaxf(mx, fabsf(v[k]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            // e with mx < 2^e (at least -100, so that 2^(22-e) and 2^(e-22) are normal floats)
            const int e = max(int((__float_as_uint(mx) >> 23) & 0xffu) - 126, -100);
            const float up = __uint_as_float(uint32_t(149 - e) << 23), sc = __uint_as_float(uint32_t(105 + e) << 23);
            uint32_t dw[3][4] = {};
            int msum = 0;
#pragma unroll
            for (int k = 0; k < 16; k++) {
                const int m = __float2int_rn(v[k] * up);
                const int d0 = ((m + 128) & 255) - 128, r = (m - d0) >> 8;
                const int d1 = ((r + 128) & 255) - 128, d2 = (r - d1) >> 8;
                dw[0][k >> 2] |= uint32_t(d0 & 255) << (8 * (k & 3));
                dw[1][k >> 2] |= uint32_t(d1 & 255) << (8 * (k & 3));
                dw[2][k >> 2] |= uint32_t(d2 & 255) << (8 * (k & 3));
                msum += m;
            }
            const float hsum = __int2float_rn(msum) * sc;
            const float other = __shfl_xor_sync(0xffffffffu, hsum, 1);
            if (live) {
                uint8_t* rec = smem + xoff + c * cstride + u * XREC;
#pragma unroll
                for (int j = 0; j < 3; j++) {
                    if (TC || TC2) {  // word w = 4*half + k at (w % 4) * 8 + (w / 4) * 4
#pragma unroll
                        for (int k = 0; k < 4; k++) *reinterpret_cast<uint32_t*>(rec + j * 32 + k * 8 + half * 4) = dw[j][k];
                    } else {
                        *reinterpret_cast<uint4*>(rec + j * 32 + half * 16) = make_uint4(dw[j][0], dw[j][1], dw[j][2], dw[j][3]);
                    }
                }
                if (half == 0)
                    *reinterpret_cast<uint4*>(rec + 96) =
                        make_uint4(__float_as_uint(sc), __float_as_uint(hsum), __float_as_uint(other), 0u);
            }
        }
    }
    // the residual rows this CTA will add to (EPI_ADD)
    const uint32_t ntiles = t1 - t0;
    const bool aux_pre = ntiles * kTileRows * NC <= uint32_t(kAuxPrefetch);
    if (aux_pre)
        for (uint32_t idx = threadIdx.x; idx < ntiles * kTileRows * NC; idx += blockDim.x) {
            const uint32_t i = idx / (kTileRows * NC), e = (idx / NC) % kTileRows, c = idx % NC;
            const GemvJob& J = pick(jobs, L.njobs, t0 + i);
            const uint32_t row = (t0 + i - J.tile_begin) * kTileRows + e;
            if (J.epi == EPI_ADD && row < J.rows) auxs[idx] = J.aux[size_t(yrows[c]) * J.aux_stride + row];
        }
    __syncthreads();

    // ---- main loop ----
    const uint32_t smem_s = saddr(smem);
    using XT = std::conditional_t<ENC == SPM_F32, XIn<NC>, XDig<NC>>;
    XT X;
#pragma unroll
    for (int c = 0; c < NC; c++) X.base[c] = smem_s + xoff + c * cstride;
    if constexpr (ENC != SPM_F32) X.nact = n_act;
    // Totals this thread finishes: with one warp per group, lane l holds
    // (row-in-pass, client) index l >> SH of each pass; with several, lane l
    // of the group's first warp holds index l = row * NCP + client of the
    // tile, all passes together (4 * NCP <= 32).
    const bool finisher = gw == 1 ? (lane & ((1 << SH) - 1)) == 0 : (wig == 0 && lane < kTileRows * NCP);
    const int fc = TC ? (lane >> 2) : (gw == 1 ? (lane >> SH) : lane) % NCP;
    const float fscale = (L.gain && fc < NC) ? nscale[fc] : 1.0f;
    float* part = reinterpret_cast<float*>(smem + poff);  // [NS][gw][M][32]
    float sq = 0.f;
    const uint32_t B = L.cols >> 8;
    float sq2[2] = {0.f, 0.f};  // TC2: sums of squares of the lane's two clients
    if constexpr (TC2) {
        // lane (g, t): A rows g (slot row g, or gate row g) and g + 8 (slot
        // row g + 8, or up row g); outputs for clients 2t and 2t + 1
        const int g = lane >> 2, t = lane & 3;
        const uint32_t xg = smem_s + xoff + uint32_t(g < NC ? g : 0) * cstride;
        const uint32_t xc[2] = {smem_s + xoff + uint32_t(min(2 * t, NC - 1)) * cstride,
                                smem_s + xoff + uint32_t(min(2 * t + 1, NC - 1)) * cstride};
        for (uint32_t i = uint32_t(grp); i < nt; i += uint32_t(G)) {
            const uint32_t s = i % NS, par = (i / NS) & 1;
            if (!mbar_wait(&full[s], par)) {
                flag(L.status, 2);
                break;
            }
            const uint32_t tb = smem_s + s * slot_bytes;
            const uint32_t gt = t0 + TPS * i;  // the slot's first tile
            const Tc2Row ra{tb + uint32_t(g >> 2) * tile_step, uint32_t(g & 3)};
            const Tc2Row rb{tb + (2u + uint32_t(g >> 2)) * tile_step, uint32_t(g & 3)};
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
            for (uint32_t u = uint32_t(wig); u < U; u += uint32_t(gw)) tc2_unit<ENC>(ra, rb, u, t, xg, xc, L, acc);
            bool fin = true;
            if (gw == 1) {
                // this warp alone read the slot: refill it
                __syncwarp();
                if (lane == 0 && i + NS < nt) {
                    fence_proxy_async();
                    issue(i + NS);
                }
            } else {
                // the group's first warp adds the warps' totals in warp order
                float* pr = part + (s * gw + wig) * 128 + lane * 4;
#pragma unroll
                for (int k = 0; k < 4; k++) pr[k] = acc[k];
                __syncwarp();
                if (lane == 0) mbar_arrive(&ready[s]);
                fin = wig == 0;
                if (fin) {
                    if (!mbar_wait(&ready[s], par)) {
                        flag(L.status, 4);
                        break;
                    }
#pragma unroll
                    for (int k = 0; k < 4; k++) acc[k] = 0.f;
                    for (int w = 0; w < gw; w++) {
                        const float* q = part + (s * gw + w) * 128 + lane * 4;
#pragma unroll
                        for (int k = 0; k < 4; k++) acc[k] += q[k];
                    }
                    __syncwarp();
                    if (lane == 0 && i + NS < nt) {
                        fence_proxy_async();
                        issue(i + NS);
                    }
                }
            }
            if (fin) {
                // (row g, row g + 8) x (clients 2t, 2t + 1); gate/up: row g's SwiGLU for both clients
#pragma unroll
                for (int k = 0; k < (DUAL ? 2 : 4); k++) {
                    const int c = 2 * t + (k & 1);
                    const uint32_t sr = DUAL ? uint32_t(g) : uint32_t(g + 8 * (k >> 1));  // slot row
                    const uint32_t tile = gt + (sr >> 2), e = sr & 3;
                    if (tile >= t1 || c >= n_act) continue;
                    const GemvJob& J = pick(jobs, L.njobs, tile);
                    const uint32_t grow = (tile - J.tile_begin) * kTileRows + e;
                    const uint32_t row = grow - rbase;
                    if (grow >= J.rows || row >= rlim) continue;
                    const float fs = L.gain ? nscale[c] : 1.0f;
                    float r = acc[k] * fs;
                    if constexpr (DUAL) r = silu_mul(r, acc[k + 2] * fs);
                    if (J.epi == EPI_ADD)
                        r = (aux_pre ? auxs[((tile - t0) * kTileRows + e) * NC + c]
                                     : J.aux[size_t(yrows[c]) * J.aux_stride + row]) + r;
                    if (L.ep_peer_y) {
                        for (int p = 0; p < L.world; p++) ep_y[p][size_t(yrows[c]) * J.y_stride + row] = r;
                    } else {
                        J.y[size_t(yrows[c]) * J.y_stride + row] = r;
                    }
                    sq2[k & 1] = fmaf(r, r, sq2[k & 1]);
                }
            }
        }
    } else if constexpr (TC) {
        // lane (g, t): client g; codes of slot row g; totals of slot rows 2t, 2t+1
        const int g = lane >> 2, t = lane & 3;
        TcLane z;
        z.t = t;
        z.cl = g < n_act;
        z.xa = smem_s + xoff + uint32_t(g < NC ? g : 0) * cstride;
        for (uint32_t i = uint32_t(grp); i < nt; i += uint32_t(G)) {
            const uint32_t s = i % NS, par = (i / NS) & 1;
            if (!mbar_wait(&full[s], par)) {
                flag(L.status, 2);
                break;
            }
            const uint32_t tb = smem_s + s * slot_bytes;
            const uint32_t tA = PAIR ? t0 + 2 * i : t0 + i;
            z.cb = tb + uint32_t(g >> 2) * tile_bytes;
            z.cr = uint32_t(g & 3);
            z.ob = tb + uint32_t(t >> 1) * tile_bytes;
            z.or0 = uint32_t(2 * t) & 3u;
            float acc[2] = {0.f, 0.f};
            tc_slot<ENC>(z, uint32_t(wig), uint32_t(gw), L, acc);
            bool fin = true;
            if (gw == 1) {
                // this warp alone read the slot: refill it
                __syncwarp();
                if (lane == 0 && i + NS < nt) {
                    fence_proxy_async();
                    issue(i + NS);
                }
            } else {
                // the group's first warp adds the warps' totals in warp order
                float* pr = part + (s * gw + wig) * 64 + g * 8 + 2 * t;
                pr[0] = acc[0];
                pr[1] = acc[1];
                __syncwarp();
                if (lane == 0) mbar_arrive(&ready[s]);
                fin = wig == 0;
                if (fin) {
                    if (!mbar_wait(&ready[s], par)) {
                        flag(L.status, 4);
                        break;
                    }
                    acc[0] = acc[1] = 0.f;
                    for (int w = 0; w < gw; w++) {
                        const float* q = part + (s * gw + w) * 64 + g * 8 + 2 * t;
                        acc[0] += q[0];
                        acc[1] += q[1];
                    }
                    __syncwarp();
                    if (lane == 0 && i + NS < nt) {
                        fence_proxy_async();
                        issue(i + NS);
                    }
                }
            }
            if (fin) {
                // a gate/up pair: lanes t < 2 hold gate rows 2t, 2t+1, lanes t + 2 the up rows
                float b0 = 0.f, b1 = 0.f;
                if (DUAL) {
                    b0 = __shfl_down_sync(0xffffffffu, acc[0], 2);
                    b1 = __shfl_down_sync(0xffffffffu, acc[1], 2);
                }
                const uint32_t tile = PAIR ? tA + uint32_t(t >> 1) : tA;
                if ((!DUAL || t < 2) && tile < t1) {
                    const GemvJob& J = pick(jobs, L.njobs, tile);
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const uint32_t e = uint32_t(2 * t + j) & 3u;
                        const uint32_t grow = (tile - J.tile_begin) * kTileRows + e;
                        const uint32_t row = grow - rbase;
                        if (g < n_act && grow < J.rows && row < rlim) {
                            float r = acc[j] * fscale;
                            if constexpr (DUAL) r = silu_mul(r, (j ? b1 : b0) * fscale);
                            if (J.epi == EPI_ADD)
                                r = (aux_pre ? auxs[((tile - t0) * kTileRows + e) * NC + g]
                                             : J.aux[size_t(yrows[g]) * J.aux_stride + row]) + r;
                            if (L.ep_peer_y) {
                                for (int p = 0; p < L.world; p++) ep_y[p][size_t(yrows[g]) * J.y_stride + row] = r;
                            } else {
                                J.y[size_t(yrows[g]) * J.y_stride + row] = r;
                            }
                            sq = fmaf(r, r, sq);
                        }
                    }
                }
            }
        }
    } else {
    for (uint32_t i = uint32_t(grp); i < nt; i += uint32_t(G)) {
            const uint32_t s = i % NS, par = (i / NS) & 1;
            if (!mbar_wait(&full[s], par)) {
                flag(L.status, 2);
                break;
            }
            const uint32_t g = t0 + i;
            const GemvJob& J = pick(jobs, L.njobs, g);
            const uint32_t tile = g - J.tile_begin;
            const uint32_t tb = smem_s + s * slot_bytes;
            // row e of the tile, client fc: scale, activation, residual, store
            auto finish = [&](uint32_t e, float a, float b) {
                const uint32_t grow = tile * kTileRows + e;
                const uint32_t row = grow - rbase;
                if (fc < n_act && grow < J.rows && row < rlim) {
                    float r = a * fscale;
                    if constexpr (DUAL) r = silu_mul(r, b * fscale);
                    if (J.epi == EPI_ADD)
                        r = (aux_pre ? auxs[(i * kTileRows + e) * NC + fc] : J.aux[size_t(yrows[fc]) * J.aux_stride + row]) + r;
                    if (L.ep_peer_y) {
                        for (int p = 0; p < L.world; p++) ep_y[p][size_t(yrows[fc]) * J.y_stride + row] = r;
                    } else {
                        J.y[size_t(yrows[fc]) * J.y_stride + row] = r;
                    }
                    sq = fmaf(r, r, sq);
                }
            };
    #pragma unroll 1
            for (int pass = 0; pass < PASSES; pass++) {
                RowRef rr[M * VR];
    #pragma unroll
                for (int m = 0; m < M; m++)
    #pragma unroll
                    for (int v = 0; v < VR; v++) {
                        const uint32_t r = uint32_t(pass * VR + v);
                        rr[m * VR + v] = RowRef{tb + uint32_t(m) * tile_bytes, r * U, r * B};
                    }
                float acc[M * VR][NC];
                zero(acc);
    #pragma unroll 1
                for (uint32_t u = uint32_t(wig * 32 + lane); u < U; u += uint32_t(gw * 32))
                    unit_dot<ENC, NC, M * VR, XT>(rr, u, L, X, acc);
                if (gw == 1 && pass + 1 == PASSES) {
                    // this warp alone read the slot: refill it
                    __syncwarp();
                    if (lane == 0 && i + NS < nt) {
                        fence_proxy_async();
                        issue(i + NS);
                    }
                }
                float red[M][V];
    #pragma unroll
                for (int m = 0; m < M; m++)
    #pragma unroll
                    for (int v = 0; v < VR; v++)
    #pragma unroll
                        for (int c = 0; c < NCP; c++) red[m][v * NCP + c] = c < NC ? acc[m * VR + v][c] : 0.f;
    #pragma unroll
                for (int m = 0; m < M; m++) XRed<V, 16>::run(red[m], lane);
                if (gw == 1) {
                    if (finisher) finish(uint32_t(pass * VR + (lane >> SH) / NCP), red[0][0], red[M - 1][0]);
                } else if ((lane & ((1 << SH) - 1)) == 0) {
    #pragma unroll
                    for (int m = 0; m < M; m++) part[((s * gw + wig) * M + m) * 32 + pass * V + (lane >> SH)] = red[m][0];
                }
            }
            if (gw > 1) {
                // partials are in; the group's first warp adds them in warp order
                // once every warp has arrived, then refills the slot
                __syncwarp();
                if (lane == 0) mbar_arrive(&ready[s]);
                if (wig == 0) {
                    if (!mbar_wait(&ready[s], par)) {
                        flag(L.status, 4);
                        break;
                    }
                    if (finisher) {
                        float a = 0.f, b = 0.f;
                        for (int w = 0; w < gw; w++) {
                            a += part[((s * gw + w) * M + 0) * 32 + lane];
                            if (M > 1) b += part[((s * gw + w) * M + M - 1) * 32 + lane];
                        }
                        finish(uint32_t(lane / NCP), a, b);
                    }
                    __syncwarp();
                    if (lane == 0 && i + NS < nt) {
                        fence_proxy_async();
                        issue(i + NS);
                    }
                }
            }
        }
    }
    if (L.sumsq_out) {
        // per-CTA sum of squares of the rows written, reduced in a fixed order
#pragma unroll
        for (int c = 0; c < NC; c++) {
            const int t2 = 2 * (lane & 3);
            const float mine = TC2 ? (c == t2 ? sq2[0] : 0.f) + (c == t2 + 1 ? sq2[1] : 0.f) : (fc == c ? sq : 0.f);
            const float t = warp_sum(mine);
            if (lane == 0) sqw[warp][c] = t;
        }
        __syncthreads();
        if (threadIdx.x < NC) {
            float t = 0.f;
            for (int w = 0; w < W; w++) t += sqw[w][threadIdx.x];
            L.sumsq_out[blockIdx.x * 8 + L.c0 + threadIdx.x] = t;
            if (L.ep_peer_sumsq)
                for (int p = 0; p < L.world; p++) L.ep_peer_sumsq[p][blockIdx.x * 8 + L.c0 + threadIdx.x] = t;
        }
    }
    if (L.ep_done) {
        __threadfence_system();
        __syncthreads();
        if (threadIdx.x == 0) ep_arrive(L);
    }
}

template <int ENC, int NC, bool DUAL, bool TCX>
cudaError_t configure(int* occ, int threads, size_t smem) {
    auto kern = gemv_stream<ENC, NC, DUAL, TCX>;
    static unsigned configured = 0;  // bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kSmemMax));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     int(cudaSharedmemCarveoutMaxShared));
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    if (occ) return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, kern, threads, smem);
    return cudaSuccess;
}

template <int ENC, int NC, bool DUAL, bool TCX>
cudaError_t launch_t(const GemvLaunch& L, int grid, int threads, size_t smem, cudaStream_t s, bool pdl) {
    cudaError_t e = configure<ENC, NC, DUAL, TCX>(nullptr, threads, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_stream<ENC, NC, DUAL, TCX>, L);
}

// All instantiations for one block type (compiled in gemv_<type>.cu).  Dense
// launches with L.tc set by the host take the tensor-core loop; expert
// launches never do.
template <int ENC, int NC, bool DUAL>
cudaError_t launch_n(const GemvLaunch& L, int grid, int threads, size_t smem, cudaStream_t s, bool pdl) {
    if constexpr (use_tc(ENC, NC) || use_tc2(ENC, NC))
        if (L.tc || L.tc2) return launch_t<ENC, NC, DUAL, true>(L, grid, threads, smem, s, pdl);
    return launch_t<ENC, NC, DUAL, false>(L, grid, threads, smem, s, pdl);
}

template <int ENC, int NC, bool DUAL>
cudaError_t configure_n(const GemvLaunch& L, int* occ, int threads, size_t smem) {
    if constexpr (use_tc(ENC, NC) || use_tc2(ENC, NC))
        if (L.tc || L.tc2) return configure<ENC, NC, DUAL, true>(occ, threads, smem);
    return configure<ENC, NC, DUAL, false>(occ, threads, smem);
}

template <int ENC>
cudaError_t launch_enc(const GemvLaunch& L, bool dual, int grid, int threads, size_t smem, cudaStream_t s, bool pdl) {
#define SPM_NC(n)                                                                   \
    case n:                                                                         \
        return dual ? launch_n<ENC, n, true>(L, grid, threads, smem, s, pdl)        \
                    : launch_n<ENC, n, false>(L, grid, threads, smem, s, pdl);
    switch (L.n) {
        SPM_NC(1) SPM_NC(2) SPM_NC(3) SPM_NC(4) SPM_NC(5) SPM_NC(6) SPM_NC(7) SPM_NC(8)
        default: return cudaErrorInvalidValue;
    }
#undef SPM_NC
}

// Resident CTAs per SM of the kernel a launch would use.
template <int ENC>
int occupancy_enc(const GemvLaunch& L, bool dual, int threads, size_t smem) {
    int occ = 0;
    cudaError_t e = cudaErrorInvalidValue;
#define SPM_NC(n)                                                                                        \
    case n:                                                                                              \
        e = dual ? configure_n<ENC, n, true>(L, &occ, threads, smem)                                     \
                 : configure_n<ENC, n, false>(L, &occ, threads, smem);                                  \
        break;
    switch (L.n) {
        SPM_NC(1) SPM_NC(2) SPM_NC(3) SPM_NC(4) SPM_NC(5) SPM_NC(6) SPM_NC(7) SPM_NC(8)
        default: break;
    }
#undef SPM_NC
    return e == cudaSuccess && occ > 0 ? occ : 1;
}

}  // namespace gemv
}  // namespace spm
