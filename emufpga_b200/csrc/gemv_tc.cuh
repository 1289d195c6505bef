// Tensor-core inner loops of the streaming GEMV for four or more clients
// (included by gemv_impl.cuh): the Q8_0 loop first, the K-quant loop below.
//
// With several clients the integer dot products outgrow the CUDA cores, so
// one 32-value unit of eight matrix rows is one small integer matrix product
// on the tensor cores (mma.sync, s8/u8 operands, s32 accumulators):
//     A (16 x k): rows are (client, digit plane) pairs of the staged
//                 activations -- clients 0..7 with plane 0 in rows 0..7 and
//                 plane 1 in rows 8..15, plane 2 in a second product;
//     B (k x 8):  the codes of the slot's eight rows (four rows of two tiles,
//                 or the four gate and four up rows of one tile);
// k = 32 (one scale per 32 values).  The integer
// sums are exact; lane (g, t) of the warp then holds client g's totals for
// slot rows 2t and 2t+1 and applies the block scales in fp32, as the CUDA-core
// loop does per lane.  Fragment layouts are those of the PTX mma.sync m16n8k16
// and m16n8k32 integer shapes.
// Included inside namespace spm::gemv, after the CUDA-core unit functions.
#pragma once

// D = A x B + 0 for the m16n8k32 integer shape (A signed digits, B codes).
template <bool BSIGNED>
__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    if constexpr (BSIGNED)
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// sum_c q_c m_c for the lane's client and slot row 2t + j from the products
// (plane 0 in d01[j], plane 1 in d01[2 + j], plane 2 in d2[j]).
__device__ __forceinline__ float tc_total(const int (&d01)[4], const int (&d2)[4], int j) {
    return fmaf(__int2float_rn(d2[j]), 65536.0f, __int2float_rn(d01[2 + j] * 256 + d01[j]));
}

// The lane's view of one slot: codes of slot row g (tile at cb, row cr) and
// outputs for slot rows 2t, 2t+1 (tile at ob, rows or0, or0 + 1).
struct TcLane {
    uint32_t cb, cr, ob, or0;
    uint32_t xa;  // shared address of client g's records (any value when the client has no data)
    bool cl;      // client g has data
    int t;        // lane & 3
};

// Client g's digits for unit u: (word t, word 4+t) of each plane, and s, sums.
struct TcX {
    uint2 p[3];
    float s, sum0, sum1;
};
__device__ __forceinline__ void tc_load_x(const TcLane& z, uint32_t u, TcX& x) {
    if (z.cl) {
        const uint32_t a = z.xa + u * kDigitUnit;
#pragma unroll
        for (int j = 0; j < 3; j++) x.p[j] = lds64(a + j * 32 + 8 * z.t);
        const uint4 r = lds128(a + 96);
        x.s = __uint_as_float(r.x);
        x.sum0 = __uint_as_float(r.y);
        x.sum1 = __uint_as_float(r.z);
    } else {
#pragma unroll
        for (int j = 0; j < 3; j++) x.p[j] = make_uint2(0u, 0u);
        x.s = x.sum0 = x.sum1 = 0.f;
    }
}

// Codes (the slot row's two code words) and the two output rows' scales of
// one unit, loaded before any product is formed.
struct TcW {
    uint32_t q[2];  // B operand: words t, 4+t
    float sa[2];    // per output row j: the block scale
};

template <int ENC>
__device__ __forceinline__ void tc_load_w(const TcLane& z, uint32_t u, const GemvLaunch& L, TcW& w) {
    static_assert(ENC == SPM_Q8_0, "the Q8_0 tensor-core loop");
    const uint32_t U = L.cols >> 5;
    const int t = z.t;
    const uint32_t unit = z.cr * U + u;
    w.q[0] = lds32(z.cb + unit * 32 + 4 * t);
    w.q[1] = lds32(z.cb + unit * 32 + 16 + 4 * t);
#pragma unroll
    for (int j = 0; j < 2; j++) w.sa[j] = h2f(lds16(z.ob + L.plane1 + ((z.or0 + j) * U + u) * 2));
}

// Products and fp32 scaling of one unit whose operands are loaded.
template <int ENC>
__device__ __forceinline__ void tc_apply(const TcX& x, const TcW& w, float (&acc)[2]) {
    int d01[4], d2[4];
    mma_k32<true>(d01, x.p[0].x, x.p[1].x, x.p[0].y, x.p[1].y, w.q[0], w.q[1]);
    mma_k32<true>(d2, x.p[2].x, 0u, x.p[2].y, 0u, w.q[0], w.q[1]);
#pragma unroll
    for (int j = 0; j < 2; j++) acc[j] = fmaf(w.sa[j] * x.s, tc_total(d01, d2, j), acc[j]);
}

// The group's share of a slot: warp wig takes units wig, wig + gw, ...; two
// units at a time have all their operands loaded before either's products,
// so the loads of the second overlap the first's.
template <int ENC>
__device__ __forceinline__ void tc_slot(const TcLane& z, uint32_t u0, uint32_t step, const GemvLaunch& L,
                                        float (&acc)[2]) {
    const uint32_t U = L.cols >> 5;
    uint32_t u = u0;
#pragma unroll 1
    for (; u + step < U; u += 2 * step) {
        TcX xa, xb;
        TcW wa, wb;
        tc_load_x(z, u, xa);
        tc_load_w<ENC>(z, u, L, wa);
        tc_load_x(z, u + step, xb);
        tc_load_w<ENC>(z, u + step, L, wb);
        tc_apply<ENC>(xa, wa, acc);
        tc_apply<ENC>(xb, wb, acc);
    }
    if (u < U) {
        TcX x;
        TcW w;
        tc_load_x(z, u, x);
        tc_load_w<ENC>(z, u, L, w);
        tc_apply<ENC>(x, w, acc);
    }
}

// ---------------------------------------------------------------------------
// Tensor-core loop of the K-quants (Q5_K, Q6_K, Q2_K) for four or more
// clients, the other way round: A (16 x k) holds the codes of sixteen matrix
// rows (unsigned), B (k x 8) one digit plane of the eight clients' staged
// activations, so one unit of sixteen rows is three products (Q5_K: one per
// plane, k = 32) or six (Q6_K, Q2_K: k = 16 per half, their scales change
// every 16 values).  Lane (g, t) holds rows g and g + 8 of the slot for
// clients 2t and 2t + 1 and applies the block scales in fp32 per (sub-)block,
// as the CUDA-core loop does.  A gate/up slot puts gate row g in A row g and
// up row g in A row g + 8, so each lane holds both halves of its SwiGLU.

// D = A x B for m16n8k32 / m16n8k16 with unsigned A (codes), signed B (digits).
__device__ __forceinline__ void mma_us_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_us_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
                 : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// sum_c q_c m_c of output k from the three planes' products.
__device__ __forceinline__ float tc2_total(const int (&d0)[4], const int (&d1)[4], const int (&d2)[4], int k) {
    return fmaf(__int2float_rn(d2[k]), 65536.0f, __int2float_rn(d1[k] * 256 + d0[k]));
}

// One row of the slot: shared address of its tile and its row in the tile.
struct Tc2Row {
    uint32_t t, e;
};

// Unit u of rows ra (A rows g) and rb (A rows g + 8): products with every
// client's digits and scaling into acc[k] (k: (ra, 2t), (ra, 2t+1), (rb, 2t),
// (rb, 2t+1)).  xg: client g's records; xc[2]: clients 2t, 2t+1's records.
template <int ENC>
__device__ __forceinline__ void tc2_unit(const Tc2Row& ra, const Tc2Row& rb, uint32_t u, int t, uint32_t xg,
                                         const uint32_t (&xc)[2], const GemvLaunch& L, float (&acc)[4]) {
    const uint32_t U = L.cols >> 5, B = L.cols >> 8;
    uint2 p[3];
#pragma unroll
    for (int j = 0; j < 3; j++) p[j] = lds64(xg + u * kDigitUnit + j * 32 + 8 * t);
    float s[2], xs0[2], xs1[2];
#pragma unroll
    for (int c = 0; c < 2; c++) {
        const uint4 r = lds128(xc[c] + u * kDigitUnit + 96);
        s[c] = __uint_as_float(r.x);
        xs0[c] = __uint_as_float(r.y);
        xs1[c] = __uint_as_float(r.z);
    }
    const Tc2Row rows[2] = {ra, rb};
    if constexpr (ENC == SPM_Q5_K) {
        uint32_t lo[2], hi[2];
        float ds[2], dm[2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint32_t unit = rows[r].e * U + u;
            const uint32_t qs = lds32(rows[r].t + unit * 16 + 4 * t);
            const uint32_t qh = lds32(rows[r].t + L.plane1 + unit * 4);
            lo[r] = (qs & 0x0F0F0F0Fu) | ((((qh >> (4 * t)) & 0xfu) * 0x02040810u) & 0x10101010u);
            hi[r] = ((qs >> 4) & 0x0F0F0F0Fu) | ((((qh >> (16 + 4 * t)) & 0xfu) * 0x02040810u) & 0x10101010u);
            const uint32_t sm = lds16(rows[r].t + L.plane2 + unit * 2);
            const uint32_t dd = lds32(rows[r].t + L.plane3 + (rows[r].e * B + (u >> 3)) * 4);
            ds[r] = h2f(dd) * (bytef<0>(sm) - 8388608.0f);
            dm[r] = h2f(dd >> 16) * (bytef<1>(sm) - 8388608.0f);
        }
        int d0[4], d1[4], d2[4];
        mma_us_k32(d0, lo[0], lo[1], hi[0], hi[1], p[0].x, p[0].y);
        mma_us_k32(d1, lo[0], lo[1], hi[0], hi[1], p[1].x, p[1].y);
        mma_us_k32(d2, lo[0], lo[1], hi[0], hi[1], p[2].x, p[2].y);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int r = k >> 1, c = k & 1;
            acc[k] = fmaf(-dm[r], xs0[c] + xs1[c], fmaf(ds[r], tc2_total(d0, d1, d2, k) * s[c], acc[k]));
        }
    } else {
        // k = 16 per half: Q6_K (d * sc) * (q - 32), Q2_K (d * sc) * q - dmin * m
        uint32_t q[2][2];  // [row][half]
        float sa[2][2], sm[2][2];
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const uint32_t unit = rows[r].e * U + u;
            if constexpr (ENC == SPM_Q6_K) {
                const uint32_t ql = lds32(rows[r].t + unit * 16 + 4 * t);
                const uint2 qh = lds64(rows[r].t + L.plane1 + unit * 8);
#pragma unroll
                for (int h = 0; h < 2; h++)
                    q[r][h] = ((h ? (ql >> 4) : ql) & 0x0F0F0F0Fu) |
                              ((((h ? qh.y : qh.x) >> (2 * t)) << 4) & 0x30303030u);
                const uint32_t sc = lds16(rows[r].t + L.plane2 + unit * 2);
                const float d = h2f(lds16(rows[r].t + L.plane3 + (rows[r].e * B + (u >> 3)) * 2));
                sa[r][0] = d * i8f(sc & 0xffu);
                sa[r][1] = d * i8f(sc >> 8);
            } else {
                const uint2 qs = lds64(rows[r].t + unit * 8);
#pragma unroll
                for (int h = 0; h < 2; h++) q[r][h] = ((h ? qs.y : qs.x) >> (2 * t)) & 0x03030303u;
                const uint32_t sc = lds16(rows[r].t + L.plane1 + unit * 2);
                const uint32_t dd = lds32(rows[r].t + L.plane2 + (rows[r].e * B + (u >> 3)) * 4);
                const float d = h2f(dd), dmin = h2f(dd >> 16);
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const uint32_t b = (sc >> (8 * h)) & 0xffu;
                    sa[r][h] = d * (bytef<0>(b & 15u) - 8388608.0f);
                    sm[r][h] = dmin * (bytef<0>(b >> 4) - 8388608.0f);
                }
            }
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            int d0[4], d1[4], d2[4];
            mma_us_k16(d0, q[0][h], q[1][h], h ? p[0].y : p[0].x);
            mma_us_k16(d1, q[0][h], q[1][h], h ? p[1].y : p[1].x);
            mma_us_k16(d2, q[0][h], q[1][h], h ? p[2].y : p[2].x);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int r = k >> 1, c = k & 1;
                const float xs = h ? xs1[c] : xs0[c];
                if constexpr (ENC == SPM_Q6_K)
                    acc[k] = fmaf(sa[r][h], fmaf(tc2_total(d0, d1, d2, k), s[c], -32.0f * xs), acc[k]);
                else
                    acc[k] = fmaf(-sm[r][h], xs, fmaf(sa[r][h], tc2_total(d0, d1, d2, k) * s[c], acc[k]));
            }
        }
    }
}
