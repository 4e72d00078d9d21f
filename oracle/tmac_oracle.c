/*
 * tmac_oracle.c -- CPU restatement of the reference's quantized-GEMV hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; never part of the product).
 * Restates, in plain C, the algorithms of liuwantao3/tmac-zynq-fpga
 * sim/tmac_gguf.cpp (matmul_fpga_* drivers, FP32 path) and the bit-accurate
 * core models of sim/fpga_sim.hpp.  Each function cites the reference lines it
 * follows.  Compile with -O2 -ffp-contract=off (no FMA contraction).
 */
#include "tmac_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fp16 decode.  fpga_sim.hpp:113-123 builds the value as
 * sign * (1 + mant/1024) * 2^(exp-15) (subnormals: mant/1024 * 2^-14); every
 * step is exact, so an exact bit decode gives identical floats.              */
float orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    float v;
    if (e == 0) {
        v = ldexpf((float)m, -24);
    } else if (e == 31) {
        v = m ? NAN : INFINITY;
    } else {
        v = ldexpf((float)(m | 0x400u), (int)e - 25);
    }
    return sign ? -v : v;
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline uint32_t rd32(const uint8_t* p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* float -> int16 with the clamp used by every core model
 * (fpga_sim.hpp:775-778, :1034-1037, :1101-1104). */
static inline int16_t clamp_round_i16(float v)
{
    if (v > 32767.0f) return 32767;
    if (v < -32768.0f) return -32768;
    return (int16_t)roundf(v);
}

/* tmac_gguf.cpp:889-896 (identical in every matmul_fpga_* driver). */
float orc_quantize_x(const float* x, int64_t n, int16_t* x_q)
{
    float xs = 0.0f;
    for (int64_t j = 0; j < n; j++) xs = fmaxf(xs, fabsf(x[j]));
    xs = (xs < 1e-10f) ? 1.0f : xs / 32767.0f;
    for (int64_t j = 0; j < n; j++) x_q[j] = (int16_t)roundf(x[j] / xs);
    return xs;
}

/* ------------------------------------------------------------------------ */
/* Block field decoders.                                                      */

/* Q5_0 element wi of a 22-byte block: fp16 d, u32 qh, 16 B qs
 * (tmac_gguf.cpp:1250-1257, fpga_sim.hpp:1023-1029). */
static inline int q5_0_quant(const uint8_t* blk, uint32_t qh, int wi)
{
    int j = wi < 16 ? wi : wi - 16;
    uint8_t b = blk[6 + j];
    int ql = wi < 16 ? (b & 0xF) : (b >> 4);
    int hb = (qh >> wi) & 1;
    return ((hb << 4) | ql) - 16;
}

/* Q4_K sub-block scale/min (ggml get_scale_min_k4 order, fpga_sim.hpp:756-765). */
static inline void q4_k_scale_min(const uint8_t* scales, int sub, int* sc, int* m)
{
    if (sub < 4) {
        *sc = scales[sub] & 63;
        *m = scales[sub + 4] & 63;
    } else {
        *sc = (scales[sub + 4] & 0xF) | ((scales[sub - 4] >> 6) << 4);
        *m = (scales[sub + 4] >> 4) | ((scales[sub] >> 6) << 4);
    }
    if (*sc > 63) *sc = 63;
    if (*m > 63) *m = 63;
}

/* Q4_K 4-bit quant of element wi (fpga_sim.hpp:767-768). */
static inline int q4_k_quant(const uint8_t* blk, int wi)
{
    int sub = wi / 32, j = wi % 32;
    uint8_t b = blk[16 + (sub / 2) * 32 + j];
    return (sub % 2 == 0) ? (b & 0xF) : (b >> 4);
}

/* Q6_K element wi of a 210-byte block: quant and int8 sub-scale
 * (fpga_sim.hpp:1074-1097). */
static inline void q6_k_quant(const uint8_t* blk, int wi, int* q6, int* sc)
{
    int half = wi / 128, pos = wi % 128, l = pos % 32, sub = pos / 32;
    uint8_t lb = blk[half * 64 + l + (sub % 2) * 32];
    int ql = (sub < 2) ? (lb & 0xF) : (lb >> 4);
    int qh = (blk[128 + half * 32 + l] >> (sub * 2)) & 0x3;
    *q6 = ((qh << 4) | ql) - 32;
    *sc = (int8_t)blk[192 + half * 8 + (l / 16) + sub * 2];
}

/* ------------------------------------------------------------------------ */
/* read_tensor (tmac_gguf.cpp:398-411) with the per-type dequant functions
 * dequant_q8_0 :225-234, dequant_q5_0 :305-322, dequant_q6_k :324-365,
 * dequant_q4_k :367-393.  W[row][col] lives at flat index col + row*cols.    */
float orc_dequant(int type, const uint8_t* w, int64_t cols, int64_t row, int64_t col)
{
    int64_t idx = (cols == 1) ? row : (col + row * cols);
    switch (type) {
    case ORC_F32: { float f; memcpy(&f, w + idx * 4, 4); return f; }
    case ORC_F16: return orc_f16_to_f32(rd16(w + idx * 2));
    case ORC_Q8_0: {
        const uint8_t* b = w + (idx / 32) * 34;
        float s = orc_f16_to_f32(rd16(b));
        int8_t v = (int8_t)b[2 + idx % 32];
        return v * s;
    }
    case ORC_Q5_0: {
        const uint8_t* b = w + (idx / 32) * 22;
        float d = orc_f16_to_f32(rd16(b));
        int q = q5_0_quant(b, rd32(b + 2), (int)(idx % 32));
        return d * (float)q;
    }
    case ORC_Q6_K: {
        const uint8_t* b = w + (idx / 256) * 210;
        float d = orc_f16_to_f32(rd16(b + 208));
        int q, sc;
        q6_k_quant(b, (int)(idx % 256), &q, &sc);
        return d * (int8_t)sc * (int8_t)q;
    }
    case ORC_Q4_K: {
        const uint8_t* b = w + (idx / 256) * 144;
        float d = orc_f16_to_f32(rd16(b));
        float dmin = orc_f16_to_f32(rd16(b + 2));
        int wi = (int)(idx % 256), sc, m;
        /* dequant_q4_k does not apply the min(.,63) clamp; the fields are 6-bit
         * so the clamp in q4_k_scale_min is a no-op. */
        q4_k_scale_min(b + 4, wi / 32, &sc, &m);
        return d * (float)sc * (float)q4_k_quant(b, wi) - dmin * (float)m;
    }
    default: return 0.0f;
    }
}

/* ------------------------------------------------------------------------ */
/* Row normalisers.                                                           */

void orc_row_inv_q5_0(const uint8_t* w, int64_t rows, int64_t cols, float* row_inv)
{
    int64_t bpr = cols / 32;
    for (int64_t r = 0; r < rows; r++) {
        float mx = 0.0f;
        for (int64_t b = 0; b < bpr; b++) {
            const uint8_t* blk = w + (r * bpr + b) * 22;
            float d = orc_f16_to_f32(rd16(blk));
            uint32_t qh = rd32(blk + 2);
            for (int wi = 0; wi < 32; wi++) {
                float ab = fabsf(d * (float)q5_0_quant(blk, qh, wi));
                if (ab > mx) mx = ab;
            }
        }
        mx = (mx < 1e-10f) ? 1.0f : mx;
        row_inv[r] = 32767.0f / mx;
    }
}

void orc_row_inv_q4_k(const uint8_t* w, int64_t rows, int64_t cols, float* row_inv)
{
    int64_t bpr = cols / 256;
    for (int64_t r = 0; r < rows; r++) {
        float mx = 0.0f;
        for (int64_t b = 0; b < bpr; b++) {
            const uint8_t* blk = w + (r * bpr + b) * 144;
            float d = orc_f16_to_f32(rd16(blk));
            float dmin = orc_f16_to_f32(rd16(blk + 2));
            for (int wi = 0; wi < 256; wi++) {
                int sc, m;
                q4_k_scale_min(blk + 4, wi / 32, &sc, &m);
                /* dequant_q4k_block_to_float, fpga_sim.hpp:1118-1142 */
                float v = d * (float)sc * (float)q4_k_quant(blk, wi) - dmin * (float)m;
                float ab = fabsf(v);
                if (ab > mx) mx = ab;
            }
        }
        mx = (mx < 1e-10f) ? 1.0f : mx;
        row_inv[r] = 32767.0f / mx;
    }
}

void orc_row_inv_q6_k(const uint8_t* w, int64_t rows, int64_t cols, float* row_inv)
{
    int64_t bpr = cols / 256;
    for (int64_t r = 0; r < rows; r++) {
        float mx = 0.0f;
        for (int64_t b = 0; b < bpr; b++) {
            const uint8_t* blk = w + (r * bpr + b) * 210;
            float d = orc_f16_to_f32(rd16(blk + 208));
            for (int wi = 0; wi < 256; wi++) {
                int q, sc;
                q6_k_quant(blk, wi, &q, &sc);
                float ab = fabsf(d * (float)sc * (float)q);
                if (ab > mx) mx = ab;
            }
        }
        mx = (mx < 1e-10f) ? 1.0f : mx;
        row_inv[r] = 32767.0f / mx;
    }
}

void orc_row_scale_q8_0(const uint8_t* w, int64_t rows, int64_t cols,
                        const float* row_max_abs, float* row_scale)
{
    for (int64_t r = 0; r < rows; r++) {
        float mx;
        if (row_max_abs) {
            mx = row_max_abs[r];
        } else {
            mx = 0.0f;
            for (int64_t j = 0; j < cols; j++) {
                int64_t idx = r * cols + j;
                const uint8_t* b = w + (idx / 32) * 34;
                float dq = (int8_t)b[2 + idx % 32] * orc_f16_to_f32(rd16(b));
                float a = fabsf(dq);
                if (a > mx) mx = a;
            }
        }
        row_scale[r] = (mx < 1e-10f) ? 1.0f : mx / 32767.0f;
    }
}

uint16_t orc_q8_combined_scale(float block_scale, float row_scale)
{
    float row_inv = (row_scale < 1e-10f) ? 1.0f : (1.0f / row_scale);
    float c = block_scale * row_inv;
    if (c >= 256.0f) c = 255.996f;
    if (c < 0.0f) c = 0.0f;
    return (uint16_t)(c * 256.0f + 0.5f);
}

static int64_t units_native(int type, int64_t cols)
{
    switch (type) {
    case ORC_Q8_0: return (cols + 63) / 64;
    case ORC_Q5_0: return cols / 32;
    case ORC_Q4_K:
    case ORC_Q6_K: return cols / 256;
    default: return -1;
    }
}

/* ------------------------------------------------------------------------ */
/* Native drivers.                                                            */

/* matmul_fpga_q8 (tmac_gguf.cpp:948-1085) + axi_vecmul_tile_q8 and the
 * MatmulAccel Q8 dequant (fpga_sim.hpp:322-349, :466-491). */
static void gemv_q8_0(const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                      const float* row_max_abs, float* y, int64_t* row_acc, int64_t* unit_acc)
{
    int16_t* xq = (int16_t*)malloc((size_t)cols * sizeof(int16_t));
    float xs = orc_quantize_x(x, cols, xq);
    int64_t ntiles = (cols + 63) / 64;
    for (int64_t r = 0; r < rows; r++) {
        float rs;
        /* rows are contiguous runs of cols/32 blocks */
        if (row_max_abs) orc_row_scale_q8_0(w, 1, cols, row_max_abs + r, &rs);
        else orc_row_scale_q8_0(w + r * (cols / 32) * 34, 1, cols, NULL, &rs);
        float yr = 0.0f;
        int64_t rsum = 0;
        for (int64_t t = 0; t < ntiles; t++) {
            int64_t c = t * 64;
            int64_t csize = cols - c < 64 ? cols - c : 64;
            uint16_t cs[2];
            for (int blk = 0; blk < 2; blk++) {
                int64_t first = c + blk * 32;
                if (first >= cols) { cs[blk] = 0; continue; }
                const uint8_t* b = w + ((r * cols + first) / 32) * 34;
                cs[blk] = orc_q8_combined_scale(orc_f16_to_f32(rd16(b)), rs);
            }
            int64_t acc = 0;
            for (int64_t k = 0; k < csize; k++) {
                int64_t idx = r * cols + c + k;
                int8_t q = (int8_t)w[(idx / 32) * 34 + 2 + idx % 32];
                int32_t prod = (int32_t)q * (int32_t)cs[k / 32];
                int16_t deq = (int16_t)(prod >> 8);
                acc += (int64_t)xq[c + k] * (int64_t)deq;
            }
            if (unit_acc) unit_acc[r * ntiles + t] = acc;
            rsum += acc;
            yr = (float)((double)yr + (double)acc * xs * rs);
        }
        y[r] = yr;
        if (row_acc) row_acc[r] = rsum;
    }
    free(xq);
}

/* matmul_fpga_q5_0 (tmac_gguf.cpp:1221-1362) + axi_vecmul_tile_q5_0_8x896_axilite
 * (fpga_sim.hpp:1004-1052).  The reference hard-codes cols = 896; for other
 * multiples of 32 this follows the same per-row block stream. */
static void gemv_q5_0(const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                      float* y, int64_t* row_acc, int64_t* unit_acc)
{
    int16_t* xq = (int16_t*)malloc((size_t)cols * sizeof(int16_t));
    float* ri = (float*)malloc((size_t)rows * sizeof(float));
    float xs = orc_quantize_x(x, cols, xq);
    orc_row_inv_q5_0(w, rows, cols, ri);
    int64_t bpr = cols / 32;
    for (int64_t r = 0; r < rows; r++) {
        int64_t acc = 0;
        for (int64_t b = 0; b < bpr; b++) {
            const uint8_t* blk = w + (r * bpr + b) * 22;
            float d = orc_f16_to_f32(rd16(blk));
            uint32_t qh = rd32(blk + 2);
            int64_t bacc = 0;
            for (int wi = 0; wi < 32; wi++) {
                float val = d * (float)q5_0_quant(blk, qh, wi);
                float norm = val * ri[r];
                bacc += (int64_t)clamp_round_i16(norm) * (int64_t)xq[b * 32 + wi];
            }
            if (unit_acc) unit_acc[r * bpr + b] = bacc;
            acc += bacc;
        }
        if (row_acc) row_acc[r] = acc;
        y[r] = (float)((double)acc * xs / (double)ri[r]);
    }
    free(xq);
    free(ri);
}

/* matmul_fpga_q4_k (tmac_gguf.cpp:1097-1215) + axilite_q4k_run
 * (fpga_sim.hpp:730-788). */
static void gemv_q4_k(const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                      float* y, int64_t* row_acc, int64_t* unit_acc)
{
    int16_t* xq = (int16_t*)malloc((size_t)cols * sizeof(int16_t));
    float* ri = (float*)malloc((size_t)rows * sizeof(float));
    float xs = orc_quantize_x(x, cols, xq);
    orc_row_inv_q4_k(w, rows, cols, ri);
    int64_t bpr = cols / 256;
    for (int64_t r = 0; r < rows; r++) {
        int64_t acc = 0;
        for (int64_t b = 0; b < bpr; b++) {
            const uint8_t* blk = w + (r * bpr + b) * 144;
            float d = orc_f16_to_f32(rd16(blk));
            float dmin = orc_f16_to_f32(rd16(blk + 2));
            int64_t bacc = 0;
            for (int wi = 0; wi < 256; wi++) {
                int sc, m;
                q4_k_scale_min(blk + 4, wi / 32, &sc, &m);
                float val = (d * (float)sc * (float)q4_k_quant(blk, wi) - dmin * (float)m) * ri[r];
                bacc += (int64_t)xq[b * 256 + wi] * (int64_t)clamp_round_i16(val);
            }
            if (unit_acc) unit_acc[r * bpr + b] = bacc;
            acc += bacc;
        }
        if (row_acc) row_acc[r] = acc;
        y[r] = (float)((double)acc * xs / (double)ri[r]);
    }
    free(xq);
    free(ri);
}

/* matmul_fpga_q6_k (tmac_gguf.cpp:1367-1523) + axi_vecmul_tile_q6_k_axilite
 * (fpga_sim.hpp:1058-1115). */
static void gemv_q6_k(const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                      float* y, int64_t* row_acc, int64_t* unit_acc)
{
    int16_t* xq = (int16_t*)malloc((size_t)cols * sizeof(int16_t));
    float* ri = (float*)malloc((size_t)rows * sizeof(float));
    float xs = orc_quantize_x(x, cols, xq);
    orc_row_inv_q6_k(w, rows, cols, ri);
    int64_t bpr = cols / 256;
    for (int64_t r = 0; r < rows; r++) {
        int64_t acc = 0;
        for (int64_t b = 0; b < bpr; b++) {
            const uint8_t* blk = w + (r * bpr + b) * 210;
            float d = orc_f16_to_f32(rd16(blk + 208));
            int64_t bacc = 0;
            for (int wi = 0; wi < 256; wi++) {
                int q, sc;
                q6_k_quant(blk, wi, &q, &sc);
                float val = d * (float)sc * (float)q * ri[r];
                bacc += (int64_t)xq[b * 256 + wi] * (int64_t)clamp_round_i16(val);
            }
            if (unit_acc) unit_acc[r * bpr + b] = bacc;
            acc += bacc;
        }
        if (row_acc) row_acc[r] = acc;
        y[r] = (float)((double)acc * xs / (double)ri[r]);
    }
    free(xq);
    free(ri);
}

/* matmul_fpga_int16 (tmac_gguf.cpp:887-941) + axi_vecmul_tile_int16
 * (fpga_sim.hpp:437-446): FP32 dequant, per-row int16 requantisation, int64
 * 64-column tiles, float accumulation of y in tile order. */
static void gemv_int16(int type, const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                       float* y, int64_t* row_acc, int64_t* unit_acc)
{
    int16_t* xq = (int16_t*)malloc((size_t)cols * sizeof(int16_t));
    float* wr = (float*)malloc((size_t)cols * sizeof(float));
    float xs = orc_quantize_x(x, cols, xq);
    int64_t ntiles = (cols + 63) / 64;
    for (int64_t r = 0; r < rows; r++) {
        float m = 0.0f;
        for (int64_t j = 0; j < cols; j++) {
            wr[j] = orc_dequant(type, w, cols, r, j);
            m = fmaxf(m, fabsf(wr[j]));
        }
        float rs = (m < 1e-10f) ? 1.0f : m / 32767.0f;
        float yr = 0.0f;
        int64_t rsum = 0;
        for (int64_t t = 0; t < ntiles; t++) {
            int64_t c = t * 64, csize = cols - c < 64 ? cols - c : 64;
            int64_t acc = 0;
            for (int64_t k = 0; k < csize; k++) {
                int16_t wq = (int16_t)roundf(wr[c + k] / rs);
                acc += (int64_t)xq[c + k] * (int64_t)wq;
            }
            if (unit_acc) unit_acc[r * ntiles + t] = acc;
            rsum += acc;
            yr = (float)((double)yr + (double)acc * xs * rs);
        }
        y[r] = yr;
        if (row_acc) row_acc[r] = rsum;
    }
    free(xq);
    free(wr);
}

/* FP32 path: matmul() with g_use_fpga == false (tmac_gguf.cpp:488-492). */
static void gemv_f32(int type, const uint8_t* w, int64_t rows, int64_t cols, const float* x, float* y)
{
    for (int64_t i = 0; i < rows; i++) {
        float sum = 0.0f;
        for (int64_t j = 0; j < cols; j++) sum += orc_dequant(type, w, cols, i, j) * x[j];
        y[i] = sum;
    }
}

int64_t orc_units_per_row(int type, int path, int64_t cols)
{
    if (path == ORC_PATH_NATIVE) return units_native(type, cols);
    if (path == ORC_PATH_INT16) return (cols + 63) / 64;
    return 0;
}

int orc_gemv(int type, int path, const uint8_t* w, int64_t rows, int64_t cols,
             const float* x, const float* row_max_abs,
             float* y, int64_t* row_acc, int64_t* unit_acc)
{
    if (rows <= 0 || cols <= 0) return -1;
    if (path == ORC_PATH_F32) {
        gemv_f32(type, w, rows, cols, x, y);
        return 0;
    }
    if (path == ORC_PATH_INT16) {
        if (type != ORC_Q8_0 && type != ORC_Q5_0 && type != ORC_Q4_K && type != ORC_Q6_K &&
            type != ORC_F32 && type != ORC_F16)
            return -1;
        gemv_int16(type, w, rows, cols, x, y, row_acc, unit_acc);
        return 0;
    }
    if (units_native(type, cols) < 0) return -1;
    switch (type) {
    case ORC_Q8_0:
        if (cols % 32) return -1;
        gemv_q8_0(w, rows, cols, x, row_max_abs, y, row_acc, unit_acc);
        return 0;
    case ORC_Q5_0:
        if (cols % 32) return -1;
        gemv_q5_0(w, rows, cols, x, y, row_acc, unit_acc);
        return 0;
    case ORC_Q4_K:
        if (cols % 256) return -1;
        gemv_q4_k(w, rows, cols, x, y, row_acc, unit_acc);
        return 0;
    case ORC_Q6_K:
        if (cols % 256) return -1;
        gemv_q6_k(w, rows, cols, x, y, row_acc, unit_acc);
        return 0;
    }
    return -1;
}

/* ------------------------------------------------------------------------ */
/* Phase-B chain replay: phaseb_run_descriptor (tmac_gguf.cpp:761-831) on an
 * arena holding DDR bytes [base, base + bytes).  Writes the zero-initialised
 * accumulator acc[] and returns the rows, 0 for CPU_OP / unsupported types,
 * -1 for an offset outside the arena. */
static int in_arena(uint64_t off, uint64_t n, uint64_t base, uint64_t bytes)
{
    return off >= base && off - base <= bytes && n <= bytes - (off - base);
}

int64_t orc_phaseb_run(const uint8_t* arena, uint32_t base, uint64_t bytes, uint32_t desc_off, int64_t* acc)
{
    if (!in_arena(desc_off, 32, base, bytes)) return -1;
    const uint8_t* dsc = arena + (desc_off - base);
    uint32_t wt = rd32(dsc + 4), act = rd32(dsc + 8);
    int ntiles = rd16(dsc + 0x10), tb = rd16(dsc + 0x12), type = dsc[0x14], tr = dsc[0x15], cg = dsc[0x19];
    if (type == ORC_Q5_0) {
        int64_t rows = (int64_t)ntiles * tr;
        if (!in_arena(wt, (uint64_t)ntiles * tb, base, bytes) || !in_arena(act, 896 * 2, base, bytes)) return -1;
        const uint8_t* xa = arena + (act - base);
        for (int64_t r = 0; r < rows; r++) acc[r] = 0;
        for (int t = 0; t < ntiles; t++) {
            const uint8_t* tile = arena + (wt - base) + (int64_t)t * tb;
            float ri[8];
            orc_row_inv_q5_0(tile, 8, 896, ri); /* phaseb_q5_0_row_inv, :740-759 */
            for (int i = 0; i < 8; i++)
                for (int b = 0; b < 28; b++) {
                    const uint8_t* blk = tile + (i * 28 + b) * 22;
                    float d = orc_f16_to_f32(rd16(blk));
                    uint32_t qh = rd32(blk + 2);
                    for (int wi = 0; wi < 32; wi++) {
                        float norm = (d * (float)q5_0_quant(blk, qh, wi)) * ri[i];
                        acc[(int64_t)t * tr + i] +=
                            (int64_t)clamp_round_i16(norm) * (int16_t)rd16(xa + 2 * (b * 32 + wi));
                    }
                }
        }
        return rows;
    }
    if (type == ORC_Q4_K || type == ORC_Q6_K) {
        int q4 = type == ORC_Q4_K, bb = q4 ? 144 : 210, blkb = q4 ? 56 * 144 : 32 * 210;
        if (cg == 0) return -1;
        int64_t rows = (int64_t)(ntiles / cg) * tr;
        if (!in_arena(wt, (uint64_t)ntiles * tb, base, bytes) || !in_arena(act, (uint64_t)cg * 512, base, bytes))
            return -1;
        for (int64_t r = 0; r < rows; r++) acc[r] = 0;
        for (int ti = 0; ti < ntiles; ti++) {
            int c = ti % cg, rg = ti / cg;
            const uint8_t* tile = arena + (wt - base) + (int64_t)ti * tb;
            const uint8_t* xa = arena + (act - base) + c * 512;
            for (int bi = 0; bi < tr; bi++) {
                int out_row = rg * tr + bi;
                float inv = (float)rd32(tile + blkb + bi * 4) / 256.0f; /* :790-795 */
                const uint8_t* blk = tile + bi * bb;
                int64_t s = 0;
                for (int wi = 0; wi < 256; wi++) {
                    float val;
                    if (q4) {
                        int sc, m;
                        q4_k_scale_min(blk + 4, wi / 32, &sc, &m);
                        float d = orc_f16_to_f32(rd16(blk)), dmin = orc_f16_to_f32(rd16(blk + 2));
                        val = (d * (float)sc * (float)q4_k_quant(blk, wi) - dmin * (float)m) * inv;
                    } else {
                        int q, sc;
                        q6_k_quant(blk, wi, &q, &sc);
                        val = orc_f16_to_f32(rd16(blk + 208)) * (float)sc * (float)q * inv;
                    }
                    s += (int64_t)(int16_t)rd16(xa + 2 * wi) * (int64_t)clamp_round_i16(val);
                }
                if (out_row < 896) acc[out_row] += s;
            }
        }
        return rows;
    }
    return 0;
}
