// blockq_dev.cuh -- device building blocks of the Q5_0 / Q4_K / Q6_K GEMV
// (gemv_blockq.cu), shared with the persistent decode kernel (decode_mega.cu):
// the 8-row-group layout, chunk loads, the exact and the fast (fp32x2) decode
// of the reference's int16 weights, the split-activation chunk dot product and
// the shared-memory int64 accumulator.  The numerics are described at the top
// of gemv_blockq.cu.
#pragma once

#include "common.cuh"
#include "dequant.cuh"

namespace tmac {

// ------------------------------------------------------------------ layout --
template <int TYPE>
struct Geo;
template <>
struct Geo<TMAC_TYPE_Q5_0> {
    static constexpr int kBlockBytes = 22, kBlockVals = 32;
    __host__ __device__ static int64_t group_bytes(int64_t nblk) { return 176 * nblk; }
};
template <>
struct Geo<TMAC_TYPE_Q4_K> {
    static constexpr int kBlockBytes = 144, kBlockVals = 256;
    __host__ __device__ static int64_t group_bytes(int64_t nblk) { return 1152 * nblk; }
};
template <>
struct Geo<TMAC_TYPE_Q6_K> {
    static constexpr int kBlockBytes = 210, kBlockVals = 256;
    __host__ __device__ static int64_t group_bytes(int64_t nblk) { return 1680 * nblk; }
};


// ------------------------------------------------------- chunk field loads --
// A chunk is 32 consecutive values of a row.  Its raw codes go into R[8]:
// byte k of R[i] is the unsigned code of value 4i+k (Q5_0: q+16, Q4_K: q,
// Q6_K: q+32), together with the chunk's fp32 scale factors.
struct Chunk {
    uint32_t R[8];
    float s0, s1;  // Q5_0: d, d   Q4_K: A = d*sc, B = dmin*m   Q6_K: A0, A1 (values 0-15, 16-31)
};

// Byte loads of a row group, through generic pointers (registration kernels,
// global memory) or 32-bit shared-memory addresses (the GEMV).
struct GlobalBytes {
    const uint8_t* p;
    TMAC_DEV uint4 ld128(uint32_t off) const { return *reinterpret_cast<const uint4*>(p + off); }
    TMAC_DEV uint32_t ld32(uint32_t off) const { return *reinterpret_cast<const uint32_t*>(p + off); }
    TMAC_DEV uint32_t ld16(uint32_t off) const { return *reinterpret_cast<const uint16_t*>(p + off); }
};
struct SharedBytes {
    uint32_t a;
    TMAC_DEV uint4 ld128(uint32_t off) const
    {
        uint4 v;
        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(a + off));
        return v;
    }
    TMAC_DEV uint32_t ld32(uint32_t off) const
    {
        uint32_t v;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a + off));
        return v;
    }
    TMAC_DEV uint32_t ld16(uint32_t off) const
    {
        uint16_t v;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a + off));
        return v;
    }
};

// Q5_0 block k of group G (cpr blocks per row).
template <class M>
TMAC_DEV void load_q5_0(const M& G, uint32_t cpr, uint32_t k, Chunk& c)
{
    const uint4 qs = G.ld128(16 * k);
    const uint32_t qh = G.ld32(128 * cpr + 4 * k);
    c.s0 = c.s1 = f16_bits_to_f32((uint16_t)G.ld16(160 * cpr + 2 * k));
    const uint32_t w[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        // bit e of qh is the fifth bit of value e: spread 4 bits to bit 4 of 4 bytes
        const uint32_t lo = ((qh >> (4 * i)) & 0xFu) * 0x02040810u;
        const uint32_t hi = ((qh >> (16 + 4 * i)) & 0xFu) * 0x02040810u;
        c.R[i] = (lo & 0x10101010u) | (w[i] & 0x0F0F0F0Fu);
        c.R[4 + i] = (hi & 0x10101010u) | ((w[i] >> 4) & 0x0F0F0F0Fu);
    }
}

// Q4_K sub-block `sub` (0..7) of the 144-byte block at offset b.
template <class M>
TMAC_DEV void load_q4_k(const M& G, uint32_t b, int sub, Chunk& c)
{
    const uint4 hdr = G.ld128(b);
    const uint8_t* hb = reinterpret_cast<const uint8_t*>(&hdr);
    const float d = f16_bits_to_f32((uint16_t)(hdr.x & 0xFFFF));
    const float dmin = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
    int sc, m;
    q4_k_scale_min(hb + 4, sub, sc, m);
    c.s0 = __fmul_rn(d, (float)sc);
    c.s1 = __fmul_rn(dmin, (float)m);
    const uint32_t qo = b + 16 + (sub >> 1) * 32;
    const uint4 q0 = G.ld128(qo), q1 = G.ld128(qo + 16);
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    const int shift = (sub & 1) * 4;
#pragma unroll
    for (int i = 0; i < 8; i++) c.R[i] = (qw[i] >> shift) & 0x0F0F0F0Fu;
}

// Q6_K sub-block `sub` (0..7) of block k of group G (nsb blocks per row).
template <class M>
TMAC_DEV void load_q6_k(const M& G, uint32_t nsb, uint32_t k, int sub, Chunk& c)
{
    const int half = sub >> 2, s4 = sub & 3;
    const uint32_t lo = 128 * k + half * 64 + (s4 & 1) * 32, ho = 1024 * nsb + 64 * k + half * 32;
    const uint32_t scw = G.ld16(1536 * nsb + 16 * k + half * 8 + s4 * 2);
    const float d = f16_bits_to_f32((uint16_t)G.ld16(1664 * nsb + 2 * k));
    c.s0 = __fmul_rn(d, (float)(int8_t)(scw & 0xFF));
    c.s1 = __fmul_rn(d, (float)(int8_t)(scw >> 8));
    const uint4 l0 = G.ld128(lo), l1 = G.ld128(lo + 16), h0 = G.ld128(ho), h1 = G.ld128(ho + 16);
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const int lshift = (s4 < 2) ? 0 : 4, hshift = 2 * s4;
#pragma unroll
    for (int i = 0; i < 8; i++)
        c.R[i] = ((lw[i] >> lshift) & 0x0F0F0F0Fu) | (((hw[i] >> hshift) << 4) & 0x30303030u);
}

template <int TYPE>
__host__ __device__ constexpr int code_bias()
{
    return TYPE == TMAC_TYPE_Q5_0 ? 16 : (TYPE == TMAC_TYPE_Q6_K ? 32 : 0);
}

// ------------------------------------------------------------ exact decode --
// roundf(t) of the reference (round half away from zero), exact for every
// finite |t| < 2^22 without a float->int conversion:
//   floor(RD(|t| + 0.5)) == floor(|t| + 0.5)   (integers are representable)
//   RD(w + 2^23) = 2^23 + floor(w)             (the ulp there is 1)
// then the sign of t.  |t| never exceeds 32767.5: max|w| * (32767/max|w|) rounds
// to within an ulp of 32767.
TMAC_DEV int round_ref(float t)
{
    const float w = __fadd_rd(fabsf(t), 0.5f);
    const int va = __float_as_int(__fadd_rd(w, 8388608.0f)) - 0x4B000000;
    return (t < 0.0f) ? -va : va;
}

// Value e (0..31) of the chunk with the reference's fp32 expression.
template <int TYPE>
TMAC_DEV int exact_value(const Chunk& c, int e, float ri)
{
    const int code = (int)((c.R[e >> 2] >> (8 * (e & 3))) & 0xFFu);
    const float q = (float)(code - code_bias<TYPE>());
    float w;
    if (TYPE == TMAC_TYPE_Q5_0) w = __fmul_rn(c.s0, q);                           // fpga_sim.hpp:1030-1037
    else if (TYPE == TMAC_TYPE_Q4_K) w = __fsub_rn(__fmul_rn(c.s0, q), c.s1);     // :773-778
    else w = __fmul_rn(e < 16 ? c.s0 : c.s1, q);                                  // :1099-1104
    return round_ref(__fmul_rn(w, ri));
}

// ------------------------------------------------------------- fast decode --
TMAC_DEV uint64_t pk2(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
TMAC_DEV uint64_t pk2u(uint32_t lo, uint32_t hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
    return r;
}
TMAC_DEV uint64_t add2(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
TMAC_DEV uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
// The low 16 bits of both halves of a pair of floats in [2^23, 2^24), as one
// word of two int16 (the integers RNE(.) - 1.5*2^23 in two's complement).
TMAC_DEV uint32_t lo16x2(uint64_t v)
{
    uint32_t lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
    return __byte_perm(lo, hi, 0x5410);
}

constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: x + kMagic = kMagic + RNE(x) for |x| < 2^22

// Fast values v' of the chunk as 16 words of int16 pairs (values 2i, 2i+1).
template <int TYPE>
TMAC_DEV void fast_values(const Chunk& c, float ri, uint32_t (&vw)[16])
{
    const uint64_t off = pk2(-(8388608.0f + code_bias<TYPE>()), -(8388608.0f + code_bias<TYPE>()));
    const uint64_t mag = pk2(kMagic, kMagic);
    uint64_t m0, m1, a1;
    if (TYPE == TMAC_TYPE_Q4_K) {
        m0 = pk2(c.s0, c.s0);
        a1 = pk2(-c.s1, -c.s1);
        m1 = pk2(ri, ri);
    } else {
        const float c0 = __fmul_rn(c.s0, ri), c1 = __fmul_rn(c.s1, ri);
        m0 = pk2(c0, c0);
        m1 = pk2(c1, c1);
        a1 = 0;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t R = c.R[i];
        // float(2^23 + code) for the four codes, then q = code - bias exactly
        const uint64_t q01 = add2(pk2u(__byte_perm(R, 0x4B000000u, 0x7540), __byte_perm(R, 0x4B000000u, 0x7541)), off);
        const uint64_t q23 = add2(pk2u(__byte_perm(R, 0x4B000000u, 0x7542), __byte_perm(R, 0x4B000000u, 0x7543)), off);
        uint64_t u01, u23;
        if (TYPE == TMAC_TYPE_Q4_K) {
            u01 = fma2(fma2(q01, m0, a1), m1, mag);
            u23 = fma2(fma2(q23, m0, a1), m1, mag);
        } else {
            const uint64_t cc = (i < 4) ? m0 : m1;
            u01 = fma2(q01, cc, mag);
            u23 = fma2(q23, cc, mag);
        }
        vw[2 * i] = lo16x2(u01);
        vw[2 * i + 1] = lo16x2(u23);
    }
}

// Exact sum of 32 int16 weights (16 packed words) times the chunk's activations
// given as signed high bytes xh and unsigned low bytes xl (x_q = 256*xh + xl):
// dp2a products fit int32 for a chunk (|sum| < 2^28).
TMAC_DEV long long chunk_dot(const uint32_t (&vw)[16], const uint8_t* xh, const uint8_t* xl)
{
    int sh = 0, sl = 0;
#pragma unroll
    for (int q = 0; q < 2; q++) {
        const uint4 H = reinterpret_cast<const uint4*>(xh)[q];
        const uint4 L = reinterpret_cast<const uint4*>(xl)[q];
        const uint32_t h[4] = {H.x, H.y, H.z, H.w}, l[4] = {L.x, L.y, L.z, L.w};
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int i = 4 * q + t;
            asm("dp2a.lo.s32.s32 %0, %1, %2, %0;" : "+r"(sh) : "r"(vw[2 * i]), "r"(h[t]));
            asm("dp2a.hi.s32.s32 %0, %1, %2, %0;" : "+r"(sh) : "r"(vw[2 * i + 1]), "r"(h[t]));
            asm("dp2a.lo.s32.u32 %0, %1, %2, %0;" : "+r"(sl) : "r"(vw[2 * i]), "r"(l[t]));
            asm("dp2a.hi.s32.u32 %0, %1, %2, %0;" : "+r"(sl) : "r"(vw[2 * i + 1]), "r"(l[t]));
        }
    }
    return (long long)sh * 256 + (long long)sl;
}

// Loads chunk `ch` (0..cpr-1) of row r (0..7) of a group.
template <int TYPE, class M>
TMAC_DEV void load_chunk(const M& G, int r, uint32_t nblk, uint32_t ch, Chunk& c)
{
    if (TYPE == TMAC_TYPE_Q5_0) load_q5_0(G, nblk, ch * 8 + r, c);
    else if (TYPE == TMAC_TYPE_Q4_K) load_q4_k(G, 144 * (r * nblk + (ch >> 3)), (int)(ch & 7), c);
    else load_q6_k(G, nblk, r * nblk + (ch >> 3), (int)(ch & 7), c);
}

// int64 accumulation in shared memory as two 32-bit words with native 32-bit
// atomics: the carry out of the low word is added to the high word.
TMAC_DEV void acc_add(uint32_t* lo, uint32_t* hi, long long v)
{
    const uint32_t l = (uint32_t)(unsigned long long)v;
    const uint32_t old = atomicAdd(lo, l);
    const uint32_t carry = (old + l < old) ? 1u : 0u;
    atomicAdd(hi, (uint32_t)((unsigned long long)v >> 32) + carry);
}

TMAC_DEV long long xq_at(const uint8_t* xpl, int64_t cols, int b, int64_t col)
{
    const uint8_t* p = xpl + (int64_t)b * 2 * cols;
    return (long long)(int8_t)p[col] * 256 + (long long)p[cols + col];
}


}  // namespace tmac
