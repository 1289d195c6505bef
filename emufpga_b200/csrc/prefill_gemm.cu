// Many-position GEMM on the tensor cores (tcgen05.mma, accumulators in TMEM):
// y[t][f] = sum_k W[f][k] * x[t][k] for every row f of one packed quantized
// matrix and t < tokens -- spm_linear::streamed (spm-linear/src/stream.rs:
// 31-55) with many positions, the shape a prompt's positions take through a
// layer.
//
// Exactness.  The weights are decoded exactly (the reference's arithmetic,
// dequant.cuh) into fp32; every fp32 value v splits exactly into three bf16
// parts, v = hi + mid + lo (hi keeps the top 8 significant bits, mid the next
// 8, lo the rest, each by truncation).  The products hi*hi, hi*mid, mid*hi,
// hi*lo, mid*mid and lo*hi accumulate in fp32 in TMEM; the three dropped
// products are below 2^-23 of |w x|, so a dot product matches an fp32 one to
// rounding (not bit for bit: the sums run in a different order).
//
// Tiles.  A CTA owns 128 matrix rows (the MMA's M, operand A) and 128
// positions (N, operand B) and walks k in steps of 64 through a two-stage
// shared-memory ring.  Eight producer warps decode and split the stage's
// weights (row r, 32 values per thread) and positions into six K-major bf16
// tiles of 128 rows x 128 bytes in the 128-byte swizzled layout the MMA
// descriptors name; one thread of a ninth warp issues 6 x 4 MMAs of
// 128 x 128 x 16 per stage and commits them to the stage's "empty" mbarrier,
// which the producers wait on before refilling it.  The epilogue reads the
// 128 x 128 fp32 accumulator from TMEM (each warp its quarter of the lanes and
// half of the columns) and stores y (plus a residual for EPI_ADD).  All
// operands come from this GPU's own memory, each CTA loading its own tiles; no clusters.
#include <cuda_runtime.h>

#include "dequant.cuh"

namespace spm {
namespace {
using namespace dev;

constexpr int kGM = 128;                       // matrix rows per CTA (MMA M)
constexpr int kGN = 128;                       // positions per CTA (MMA N)
constexpr int kGK = 64;                        // k per stage: one 128-byte row of bf16
constexpr int kParts = 3;                      // hi, mid, lo
constexpr int kProducers = 256;                // eight warps
constexpr int kGemmThreads = kProducers + 32;  // + the MMA warp
constexpr uint32_t kTileBytes = 128u * 128u;   // one part of one operand: 128 rows x 128 bytes
constexpr uint32_t kStageBytes = 2u * kParts * kTileBytes;
constexpr int kStages = 2;
constexpr size_t kGemmSmem = size_t(kStages) * kStageBytes + 1024;  // + alignment of the ring to 1024 bytes
constexpr uint32_t kTmemCols = 128;
// the six part products (A part, B part) that are kept
__constant__ int8_t kPairA[6] = {0, 0, 1, 0, 1, 2};
__constant__ int8_t kPairB[6] = {0, 1, 0, 2, 1, 0};

// Instruction descriptor of tcgen05.mma kind::f16: D f32 (bits 4-5 = 1), A and
// B bf16 (bits 7-9 and 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at
// bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kGN >> 3) << 17) |
                            (uint32_t(kGM >> 4) << 24);

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzled
// layout: start address >> 4 (bits 0-13), leading byte offset 16 (unused by
// this layout; bits 16-29), stride byte offset 1024 between 8-row groups
// (>> 4 at bit 32), descriptor version 1 (bit 46), swizzle mode 2 = 128-byte
// (bits 61-63).  The start must sit in a 1024-byte aligned swizzle atom; the
// k-th 16-element step inside the 128-byte row adds 32 * k bytes to it.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Byte offset of 16-byte chunk c (8 bf16 of k = 8c..8c+7) of row r in a
// 128-row tile of the 128-byte swizzled K-major layout: 8-row atoms of 1024
// bytes, chunk index XOR (row mod 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t r, uint32_t c) {
    return (r >> 3) * 1024u + (r & 7u) * 128u + ((c ^ (r & 7u)) << 4);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem),
        "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Sixteen consecutive accumulator columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]);
}

// v = hi + mid + lo exactly, each part a bf16 (returned as its 16 bits).
__device__ __forceinline__ void split3(float v, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
    const uint32_t b = __float_as_uint(v);
    hi = b >> 16;
    const float r = __fsub_rn(v, __uint_as_float(b & 0xFFFF0000u));
    const uint32_t rb = __float_as_uint(r);
    mid = rb >> 16;
    lo = __float_as_uint(__fsub_rn(r, __uint_as_float(rb & 0xFFFF0000u))) >> 16;
}

// Split 32 values and store their parts as chunks c0..c0+3 of row r of the
// three part tiles at `base` (kTileBytes apart).
__device__ __forceinline__ void store_parts(uint32_t base, uint32_t r, uint32_t c0, const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint32_t w[kParts][4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t h0, m0, l0, h1, m1, l1;
            split3(v[8 * c + 2 * j], h0, m0, l0);
            split3(v[8 * c + 2 * j + 1], h1, m1, l1);
            w[0][j] = h0 | (h1 << 16);
            w[1][j] = m0 | (m1 << 16);
            w[2][j] = l0 | (l1 << 16);
        }
        const uint32_t off = sw128_offset(r, c0 + uint32_t(c));
#pragma unroll
        for (int p = 0; p < kParts; p++)
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(base + uint32_t(p) * kTileBytes + off),
                         "r"(w[p][0]), "r"(w[p][1]), "r"(w[p][2]), "r"(w[p][3])
                         : "memory");
    }
}

__global__ void __launch_bounds__(kGemmThreads, 1) prefill_gemm_kernel(const GemmArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t full[kStages], empty[kStages], done;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    const uint32_t ring = (saddr(smem_raw) + 1023u) & ~1023u;  // 1024-aligned swizzle atoms
    const int warp = int(threadIdx.x >> 5), lane = int(threadIdx.x & 31);
    const uint32_t f0 = blockIdx.x * kGM;
    uint32_t n0 = blockIdx.y * kGN;
    const uint8_t* W = a.w;
    int tokens = a.tokens, first = 0;
    if (a.groups) {
        const int4 g = a.groups[blockIdx.y];
        W = a.w + size_t(g.x) * a.w_stride;
        first = g.y;
        tokens = g.z;
        n0 = 0;
    }
    const int KB = int(a.pk.cols / kGK);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            mbar_init(&full[s], kProducers);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == kProducers / 32) {
        // TMEM for the 128 x 128 fp32 accumulator
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&tmem_base)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;
    pdl_wait();

    if (warp == kProducers / 32) {
        // ---- MMA issue: one thread ----
        if (lane == 0) {
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % kStages;
                if (!mbar_wait(&full[s], uint32_t(kb / kStages) & 1u)) {
                    flag(a.status, 7);
                    abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t A = ring + uint32_t(s) * kStageBytes, B = A + kParts * kTileBytes;
#pragma unroll 1
                for (int kk = 0; kk < kGK / 16; kk++)
#pragma unroll
                    for (int pr = 0; pr < 6; pr++)
                        umma_bf16(tmem, sw128_desc(A + uint32_t(kPairA[pr]) * kTileBytes + 32u * kk),
                                  sw128_desc(B + uint32_t(kPairB[pr]) * kTileBytes + 32u * kk),
                                  (kb | kk | pr) != 0 ? 1u : 0u);
                umma_commit(&empty[s]);
            }
            umma_commit(&done);  // completes when every MMA issued above has
        }
        __syncwarp();
    } else {
        // ---- producers: weights and positions of stage kb ----
        const uint32_t t = threadIdx.x, r = t >> 1, half = t & 1;
        const uint32_t f = f0 + r, n = n0 + r;
        const uint32_t rows = uint32_t(a.pk.rows);
        const uint8_t* tile = W + size_t(f / kTileRows) * a.pk.tile_bytes;
        const float* xr = nullptr;
        const float* x2r = nullptr;
        if (n < uint32_t(tokens)) {
            const size_t place = size_t(first) + n;
            const size_t row = a.x_index ? size_t(a.x_index[place]) : place;
            xr = a.x + row * a.x_stride;
            if (a.x2) x2r = a.x2 + row * a.x_stride;
        }
        for (int kb = 0; kb < KB; kb++) {
            const int s = kb % kStages;
            if (kb >= kStages && !mbar_wait(&empty[s], uint32_t(kb / kStages - 1) & 1u)) {
                flag(a.status, 7);
                abort_flag = 1;
            }
            if (abort_flag) break;
            const uint32_t A = ring + uint32_t(s) * kStageBytes, B = A + kParts * kTileBytes;
            const uint32_t k0 = uint32_t(kb) * kGK + half * 32;
            float v[32];
            if (f < rows) {
                dequant_unit(a.pk.dtype, tile, a.pk, f % kTileRows, k0 >> 5, v);
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = 0.f;
            }
            store_parts(A, r, half * 4, v);
            if (xr) {
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float4 q = *reinterpret_cast<const float4*>(xr + k0 + 4 * j);
                    v[4 * j] = q.x, v[4 * j + 1] = q.y, v[4 * j + 2] = q.z, v[4 * j + 3] = q.w;
                }
                if (x2r) {
                    // SwiGLU input: silu(gate) * up, as the decode path forms it
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float4 u = *reinterpret_cast<const float4*>(x2r + k0 + 4 * j);
                        const float uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const float g = v[4 * j + e];
                            v[4 * j + e] = __fdiv_rn(g, 1.0f + expf(-g)) * uu[e];
                        }
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 32; j++) v[j] = 0.f;
            }
            store_parts(B, r, half * 4, v);
            fence_proxy_async();  // generic-proxy writes before the MMAs (async proxy) read them
            mbar_arrive(&full[s]);
        }
        // ---- epilogue: the accumulator, once every MMA has completed ----
        const bool got = mbar_wait(&done, 0);
        if (!got) flag(a.status, 7);
        tc_fence_after();
        if (__all_sync(0xffffffffu, got && !abort_flag)) {  // tcgen05.ld is warp-wide
            const uint32_t q = uint32_t(warp & 3), ch = uint32_t(warp >> 2);
            const uint32_t frow = f0 + q * 32 + uint32_t(lane);
#pragma unroll 1
            for (uint32_t c0 = ch * 64; c0 < ch * 64 + 64; c0 += 16) {
                float acc[16];
                tmem_ld16(tmem + ((q * 32) << 16) + c0, acc);
                if (frow < rows) {
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const uint32_t tok = n0 + c0 + uint32_t(j);
                        if (tok < uint32_t(tokens)) {
                            const size_t yr = size_t(first) + tok;
                            float y = acc[j];
                            if (a.epi == EPI_ADD) y = a.aux[yr * a.aux_stride + frow] + y;
                            a.y[yr * a.y_stride + frow] = y;
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    pdl_trigger();
    if (warp == kProducers / 32) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

}  // namespace

cudaError_t launch_prefill_gemm(const GemmArgs& a, cudaStream_t s) {
    if (a.groups ? a.ngroups <= 0 : a.tokens <= 0) return cudaSuccess;
    if (a.pk.cols % kGK || a.x_stride % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15)) return cudaErrorInvalidValue;
    static unsigned configured = 0;  // bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && !(configured & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(prefill_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(kGemmSmem));
        if (e != cudaSuccess) return e;
        configured |= 1u << dev;
    }
    const dim3 grid(unsigned((a.pk.rows + kGM - 1) / kGM),
                    unsigned(a.groups ? a.ngroups : (a.tokens + kGN - 1) / kGN));
    prefill_gemm_kernel<<<grid, kGemmThreads, kGemmSmem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace spm
