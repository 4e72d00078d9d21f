// q8_dev.cuh -- device building blocks of the Q8_0 GEMV (gemv_q8_0.cu), shared
// with the persistent decode kernel (decode_mega.cu): the 32-row-group record
// layout and the exact per-tile integer dot products (numerics at the top of
// gemv_q8_0.cu).
#pragma once

#include "common.cuh"

namespace tmac {

struct Q8Layout {
    int T;               // 64-column tiles per row
    int stages;          // shared-memory pipeline depth (2..4)
    int64_t groups;      // 32-row groups
    int64_t group_bytes; // T*2048 + T*128 + 128
    __host__ __device__ int64_t cs_off() const { return (int64_t)T * 2048; }
    __host__ __device__ int64_t rs_off() const { return (int64_t)T * 2176; }
};

// Exact sum over one 32-column block: 8 words of biased quants, the split
// activations, the block's combined scale and activation sum.
TMAC_DEV long long q8_block_dot(const uint32_t (&q)[8], const uint4& xh0, const uint4& xh1, const uint4& xl0,
                                const uint4& xl1, uint32_t cs, int sx)
{
    const uint32_t cl = cs & 255u, ch = cs >> 8;
    const uint32_t K2 = (128u * (256u - cl)) * 0x00010001u;
    const uint32_t xh[8] = {xh0.x, xh0.y, xh0.z, xh0.w, xh1.x, xh1.y, xh1.z, xh1.w};
    const uint32_t xl[8] = {xl0.x, xl0.y, xl0.z, xl0.w, xl1.x, xl1.y, xl1.z, xl1.w};
    int qh = 0, ql = 0, eh = 0, el = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        const uint32_t a = __byte_perm(q[w], 0u, 0x4240);  // q'0 | q'2 << 16
        const uint32_t b = __byte_perm(q[w], 0u, 0x4341);  // q'1 | q'3 << 16
        const uint32_t ea = a * cl + K2;
        const uint32_t eb = b * cl + K2;
        const uint32_t e = __byte_perm(ea, eb, 0x7351);    // eb0 eb1 eb2 eb3
        qh = dp4a_us(q[w], xh[w], qh);
        ql = dp4a_uu(q[w], xl[w], ql);
        eh = dp4a_us(e, xh[w], eh);
        el = dp4a_uu(e, xl[w], el);
    }
    const int qx = qh * 256 + ql - 128 * sx;
    const int ex = eh * 256 + el - 128 * sx;
    return (long long)ch * (long long)qx + (long long)ex;
}

// Tile sums of tile t for the 32 rows of a staged group (lane = row).
TMAC_DEV long long q8_tile_dot(const uint8_t* st, const Q8Layout& L, int t, int lane, const uint4 (&xh)[4],
                               const uint4 (&xl)[4], int2 sx)
{
    const uint4* qv = reinterpret_cast<const uint4*>(st);
    uint4 c[4];
#pragma unroll
    for (int j = 0; j < 4; j++) c[j] = qv[(t * 4 + j) * 32 + lane];
    const uint32_t csw = reinterpret_cast<const uint32_t*>(st + L.cs_off())[t * 32 + lane];
    const uint32_t q0[8] = {c[0].x, c[0].y, c[0].z, c[0].w, c[1].x, c[1].y, c[1].z, c[1].w};
    const uint32_t q1[8] = {c[2].x, c[2].y, c[2].z, c[2].w, c[3].x, c[3].y, c[3].z, c[3].w};
    return q8_block_dot(q0, xh[0], xh[1], xl[0], xl[1], csw & 0xFFFFu, sx.x) +
           q8_block_dot(q1, xh[2], xh[3], xl[2], xl[3], csw >> 16, sx.y);
}

}  // namespace tmac
