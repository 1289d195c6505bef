// Device helpers shared by the kernels: loads, exact conversions, bulk copies
// into shared memory, mbarriers with bounded waits, programmatic dependent
// launch.
#pragma once
#include <cuda_fp16.h>

#include "kernels.h"

namespace spm {
namespace dev {

// ---- global loads ----
__device__ __forceinline__ float4 ldx4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// ---- shared loads by 32-bit shared address ----
__device__ __forceinline__ uint32_t saddr(const void* p) { return uint32_t(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(a));
    return r;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 r;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "r"(a));
    return r;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t r;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(r) : "r"(a));
    return r;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short r;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(r) : "r"(a));
    return r;
}

// Exact half -> float.
__device__ __forceinline__ float h2f(uint32_t bits) {
    return __half2float(__ushort_as_half((unsigned short)(bits & 0xffff)));
}
// 2^23 + (byte B of w), exactly; subtracting a constant recovers the code.
template <int B>
__device__ __forceinline__ float bytef(uint32_t w) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | B));
}

// Four-way byte dot products accumulated in int32: a's bytes signed (ss) or
// unsigned (us) times b's signed bytes, plus c.
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// x = hi + mid + lo exactly, each part a bf16 (its bits returned): hi the
// top 16 bits of x, mid those of x - hi, lo those of x - hi - mid (x's 24
// significant bits are 8 + 8 + 8; every subtraction is exact).
__device__ __forceinline__ void split3_bits(float x, uint16_t (&p)[3]) {
    const uint32_t b = __float_as_uint(x);
    const float r = __fsub_rn(x, __uint_as_float(b & 0xffff0000u));
    const uint32_t c = __float_as_uint(r);
    const float l = __fsub_rn(r, __uint_as_float(c & 0xffff0000u));
    p[0] = uint16_t(b >> 16);
    p[1] = uint16_t(c >> 16);
    p[2] = uint16_t(__float_as_uint(l) >> 16);
}
// Row c of a plane row [3][hd] of bf16 bits.
__device__ __forceinline__ void store_planes(uint16_t* row, int hd, int c, float x) {
    uint16_t p[3];
    split3_bits(x, p);
    row[c] = p[0];
    row[hd + c] = p[1];
    row[2 * hd + c] = p[2];
}

// ---- time, errors ----
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s: then give up and flag
__device__ __forceinline__ void flag(int32_t* status, int32_t code) {
    if (status) atomicCAS(status, 0, code);
}

// ---- mbarriers (CTA scope) ----
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(saddr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for phase `parity` to complete; false after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
    if (mbar_try(b, parity)) return true;
    const uint64_t t0 = now_ns();
    while (!mbar_try(b, parity))
        if (now_ns() - t0 > kWaitLimitNs) return false;
    return true;
}
// One bulk copy global -> shared into this CTA alone, completing on `bar`.
// Source, destination and size must be multiples of 16 bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     saddr(dst)),
                 "l"(src), "r"(bytes), "r"(saddr(bar))
                 : "memory");
}

// Asks for `bytes` of global memory to be brought into L2 (no completion
// to wait for).  Address and size must be multiples of 16 bytes.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---- 16-byte asynchronous copies global -> shared (no mbarrier) ----
// Both addresses 16-byte aligned; cp_async_commit closes the thread's current
// group and cp_async_wait<N> waits until at most N of its groups are pending.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- system-scope flags (peer GPUs over NVLink) ----
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---- programmatic dependent launch ----
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier among the first `threads` threads (id 1; 0 is __syncthreads).
__device__ __forceinline__ void bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
// Named barrier `id` over `threads` threads that also ORs a predicate across
// them: every participant learns whether any of them passed true.
__device__ __forceinline__ bool bar_or(int id, int threads, bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(uint32_t(p)), "r"(id), "r"(threads)
        : "memory");
    return r != 0;
}
// Orders this thread's (and, after a barrier, its peers') generic-proxy
// accesses to shared memory before its later async-proxy operations (a bulk
// copy that overwrites a ring slot the warps have just read).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace dev
}  // namespace spm
