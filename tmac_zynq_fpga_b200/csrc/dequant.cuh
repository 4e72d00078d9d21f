// dequant.cuh -- element dequantisation of raw GGUF blocks (device).
//
// Restates read_tensor and the dequant_* helpers of the reference
// (sim/tmac_gguf.cpp:225-411) with the same fp32 operation order:
//   Q8_0: q * d                  Q5_0: d * q
//   Q6_K: (d * sc) * q           Q4_K: (d * sc) * q4 - dmin * m
// W[row][col] sits at flat index col + row * cols (GGUF ne[0] = cols).
#pragma once

#include "common.cuh"

namespace tmac {

TMAC_DEV void q4_k_scale_min(const uint8_t* scales, int sub, int& sc, int& m)
{
    if (sub < 4) {
        sc = scales[sub] & 63;
        m = scales[sub + 4] & 63;
    } else {
        sc = (scales[sub + 4] & 0xF) | ((scales[sub - 4] >> 6) << 4);
        m = (scales[sub + 4] >> 4) | ((scales[sub] >> 6) << 4);
    }
}

TMAC_DEV float dequant_element(int type, const uint8_t* w, int64_t cols, int64_t row, int64_t col)
{
    const int64_t idx = (cols == 1) ? row : (col + row * cols);
    switch (type) {
    case TMAC_TYPE_F32: return __ldg(reinterpret_cast<const float*>(w) + idx);
    case TMAC_TYPE_F16: return f16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(w) + idx));
    case TMAC_TYPE_Q8_0: {
        const uint8_t* b = w + (idx / 32) * 34;
        float d = f16_bits_to_f32(ld_u16_unaligned(b));
        return __fmul_rn((float)(int8_t)b[2 + idx % 32], d);
    }
    case TMAC_TYPE_Q5_0: {
        const uint8_t* b = w + (idx / 32) * 22;
        float d = f16_bits_to_f32(ld_u16_unaligned(b));
        uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
        int wi = (int)(idx % 32), j = wi < 16 ? wi : wi - 16;
        int ql = wi < 16 ? (b[6 + j] & 0xF) : (b[6 + j] >> 4);
        int q = ((((qh >> wi) & 1) << 4) | ql) - 16;
        return __fmul_rn(d, (float)q);
    }
    case TMAC_TYPE_Q6_K: {
        const uint8_t* b = w + (idx / 256) * 210;
        float d = f16_bits_to_f32(ld_u16_unaligned(b + 208));
        int wi = (int)(idx % 256), half = wi / 128, pos = wi % 128, l = pos % 32, sub = pos / 32;
        uint8_t lb = b[half * 64 + l + (sub % 2) * 32];
        int ql = (sub < 2) ? (lb & 0xF) : (lb >> 4);
        int qh = (b[128 + half * 32 + l] >> (sub * 2)) & 0x3;
        int q = ((qh << 4) | ql) - 32;
        int sc = (int8_t)b[192 + half * 8 + (l / 16) + sub * 2];
        return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
    case TMAC_TYPE_Q4_K: {
        const uint8_t* b = w + (idx / 256) * 144;
        float d = f16_bits_to_f32(ld_u16_unaligned(b));
        float dmin = f16_bits_to_f32(ld_u16_unaligned(b + 2));
        int wi = (int)(idx % 256), sub = wi / 32, j = wi % 32, sc, m;
        q4_k_scale_min(b + 4, sub, sc, m);
        uint8_t qb = b[16 + (sub / 2) * 32 + j];
        int q4 = (sub % 2 == 0) ? (qb & 0xF) : (qb >> 4);
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q4), __fmul_rn(dmin, (float)m));
    }
    default: return 0.0f;
    }
}

}  // namespace tmac
