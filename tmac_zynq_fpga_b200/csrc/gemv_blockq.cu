// gemv_blockq.cu -- Q5_0 / Q4_K / Q6_K GEMV, bit-exact with the reference's
// FPGA core models driven by their matmul_fpga_* drivers:
//   Q5_0: matmul_fpga_q5_0 (sim/tmac_gguf.cpp:1221-1362) +
//         axi_vecmul_tile_q5_0_8x896_axilite (sim/fpga_sim.hpp:1004-1052)
//   Q4_K: matmul_fpga_q4_k (tmac_gguf.cpp:1097-1215) + axilite_q4k_run (fpga_sim.hpp:730-788)
//   Q6_K: matmul_fpga_q6_k (tmac_gguf.cpp:1367-1523) +
//         axi_vecmul_tile_q6_k_axilite (fpga_sim.hpp:1058-1115)
//
// Per row r: row_inv[r] = 32767 / max|w| (weight-only, computed once at
// registration), every weight becomes
//   v = clamp_round_i16(w_f32 * row_inv)      with w_f32 in the reference's order:
//       Q5_0: d*q     Q4_K: (d*sc)*q4 - dmin*m     Q6_K: (d*sc)*q6
// the int64 row sum is  acc = sum v * x_q  and  y = (float)((double)acc * x_scale / (double)row_inv).
// The integer sum is order-free, so the work is split freely: one warp per row,
// each lane decoding one 32-value chunk (a Q5_0 block, a Q4_K sub-block, a Q6_K
// 32-value run) per iteration, row sums by warp shuffle.
#include "common.cuh"
#include "dequant.cuh"

#include <algorithm>

namespace tmac {
namespace {

constexpr int kThreads = 256;

TMAC_DEV uint16_t ldg16(const uint8_t* p) { return __ldg(reinterpret_cast<const uint16_t*>(p)); }

// ------------------------------------------------------------ row_inv pass --
template <int TYPE>
__global__ void row_inv_kernel(const uint8_t* __restrict__ raw, int64_t rows, int64_t cols, float* __restrict__ ri)
{
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float mx = 0.0f;
    for (int64_t c = lane; c < cols; c += 32) {
        // |w| with the reference's fp32 expression (tmac_gguf.cpp:1258, :1131, :1415)
        float v = dequant_element(TYPE, raw, cols, r, c);
        mx = fmaxf(mx, fabsf(v));
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) ri[r] = __fdiv_rn(32767.0f, (mx < 1e-10f) ? 1.0f : mx);
}

// --------------------------------------------------- chunk decode (32 values)
// roundf(t) of the reference (round half away from zero) as an int16 in the
// low 16 bits, exact for every finite |t| < 2^22 without a float->int
// conversion instruction:
//   floor(RD(|t| + 0.5)) == floor(|t| + 0.5)   (integers are representable, so
//                                               rounding down never crosses one)
//   RD(w + 2^23) = 2^23 + floor(w)             (the ulp there is 1)
// then the sign of t is applied.  No clamp is needed: every |t| is at most
// max|w| * (32767 / max|w|) rounded, i.e. below 32767.5.
TMAC_DEV uint32_t round_i16(float t)
{
    const float w = __fadd_rd(fabsf(t), 0.5f);
    const int va = __float_as_int(__fadd_rd(w, 8388608.0f)) - 0x4B000000;
    const int m = __float_as_int(t) >> 31;
    return (uint32_t)((va ^ m) - m);
}

// float(n) for 0 <= n < 2^23 minus a constant: exact, via the 2^23 exponent.
TMAC_DEV float small_int_f(uint32_t n, float minus) { return __fsub_rn(__uint_as_float(0x4B000000u | n), minus); }

TMAC_DEV uint32_t pack2(uint32_t lo, uint32_t hi) { return __byte_perm(lo, hi, 0x5410); }

// Decodes chunk `ch` of row `r` into 16 words of int16 pairs (values 2i, 2i+1),
// each value = roundf(w_f32 * row_inv) with w_f32 in the reference's fp32 order
// (fpga_sim.hpp:1030-1037, :773-778, :1099-1104).
template <int TYPE>
TMAC_DEV void decode_chunk(const uint8_t* __restrict__ raw, int64_t r, int64_t cpr, int64_t ch, float ri,
                           uint32_t (&vw)[16])
{
    if (TYPE == TMAC_TYPE_Q5_0) {
        const uint8_t* b = raw + (r * cpr + ch) * 22;  // 2-byte aligned
        const float d = f16_bits_to_f32(ldg16(b));
        const uint32_t qh = (uint32_t)ldg16(b + 2) | ((uint32_t)ldg16(b + 4) << 16);
        uint32_t qw[4];
#pragma unroll
        for (int i = 0; i < 4; i++) qw[i] = (uint32_t)ldg16(b + 6 + 4 * i) | ((uint32_t)ldg16(b + 8 + 4 * i) << 16);
#pragma unroll
        for (int wi = 0; wi < 32; wi += 2) {
            uint32_t v2[2];
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const int e = wi + k, j = e & 15;
                const uint32_t nib = (qw[j >> 2] >> (8 * (j & 3) + (e >= 16 ? 4 : 0))) & 0xFu;
                const uint32_t raw5 = nib | (((qh >> e) & 1u) << 4);
                const float q = small_int_f(raw5, 8388624.0f);  // raw5 - 16
                v2[k] = round_i16(__fmul_rn(__fmul_rn(d, q), ri));
            }
            vw[wi / 2] = pack2(v2[0], v2[1]);
        }
    } else if (TYPE == TMAC_TYPE_Q4_K) {
        const int64_t sb = ch >> 3;
        const int sub = (int)(ch & 7);
        const uint8_t* b = raw + (r * (cpr >> 3) + sb) * 144;  // 16-byte aligned
        const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(b));
        const uint8_t* hb = reinterpret_cast<const uint8_t*>(&hdr);
        const float d = f16_bits_to_f32((uint16_t)(hb[0] | (hb[1] << 8)));
        const float dmin = f16_bits_to_f32((uint16_t)(hb[2] | (hb[3] << 8)));
        int sc, m;
        q4_k_scale_min(hb + 4, sub, sc, m);
        const float A = __fmul_rn(d, (float)sc), B = __fmul_rn(dmin, (float)m);
        const uint4* qp = reinterpret_cast<const uint4*>(b + 16 + (sub >> 1) * 32);
        const uint4 q0 = __ldg(qp), q1 = __ldg(qp + 1);
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const int shift = (sub & 1) * 4;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            uint32_t v2[2];
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const int e = j + k;
                const uint32_t q4 = (qw[e >> 2] >> (8 * (e & 3) + shift)) & 0xFu;
                const float q = small_int_f(q4, 8388608.0f);
                v2[k] = round_i16(__fmul_rn(__fsub_rn(__fmul_rn(A, q), B), ri));
            }
            vw[j / 2] = pack2(v2[0], v2[1]);
        }
    } else {  // Q6_K
        const int64_t sb = ch >> 3;
        const int within = (int)(ch & 7), half = within >> 2, sub = within & 3;
        const uint8_t* b = raw + (r * (cpr >> 3) + sb) * 210;  // 2-byte aligned
        const float d = f16_bits_to_f32(ldg16(b + 208));
        const uint16_t scw = ldg16(b + 192 + half * 8 + sub * 2);
        const float A0 = __fmul_rn(d, (float)(int8_t)(scw & 0xFF));
        const float A1 = __fmul_rn(d, (float)(int8_t)(scw >> 8));
        const uint8_t* ql = b + half * 64 + (sub & 1) * 32;
        const uint8_t* qhp = b + 128 + half * 32;
        const int lshift = (sub < 2) ? 0 : 4, hshift = sub * 2;
        uint32_t lw[8], hw[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            lw[i] = (uint32_t)ldg16(ql + 4 * i) | ((uint32_t)ldg16(ql + 4 * i + 2) << 16);
            hw[i] = (uint32_t)ldg16(qhp + 4 * i) | ((uint32_t)ldg16(qhp + 4 * i + 2) << 16);
        }
#pragma unroll
        for (int l = 0; l < 32; l += 2) {
            uint32_t v2[2];
#pragma unroll
            for (int k = 0; k < 2; k++) {
                const int e = l + k, bs = 8 * (e & 3);
                const uint32_t lo = (lw[e >> 2] >> (bs + lshift)) & 0xFu;
                const uint32_t hi = (hw[e >> 2] >> (bs + hshift)) & 0x3u;
                const float q = small_int_f((hi << 4) | lo, 8388640.0f);  // q6 = raw6 - 32
                v2[k] = round_i16(__fmul_rn(__fmul_rn(e < 16 ? A0 : A1, q), ri));
            }
            vw[l / 2] = pack2(v2[0], v2[1]);
        }
    }
}

// Exact sum of 32 int16 weights (16 packed words) times the chunk's activations
// given as signed high bytes xh and unsigned low bytes xl (x_q = 256*xh + xl):
// dp2a products fit int32 for a chunk (|sum| < 2^28).
TMAC_DEV long long chunk_dot(const uint32_t (&vw)[16], const uint32_t* xh, const uint32_t* xl)
{
    int sh = 0, sl = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t h = xh[i], l = xl[i];
        asm("dp2a.lo.s32.s32 %0, %1, %2, %0;" : "+r"(sh) : "r"(vw[2 * i]), "r"(h));
        asm("dp2a.hi.s32.s32 %0, %1, %2, %0;" : "+r"(sh) : "r"(vw[2 * i + 1]), "r"(h));
        asm("dp2a.lo.s32.u32 %0, %1, %2, %0;" : "+r"(sl) : "r"(vw[2 * i]), "r"(l));
        asm("dp2a.hi.s32.u32 %0, %1, %2, %0;" : "+r"(sl) : "r"(vw[2 * i + 1]), "r"(l));
    }
    return (long long)sh * 256 + (long long)sl;
}

struct BlockqArgs {
    const uint8_t* raw;
    const float* row_inv;
    int64_t rows, cols;
    const float* x;        // [nb][cols] fp32 activations, or
    const int16_t* xq_in;  // [nb][cols] already-quantised activations with
    const float* xs_in;    // [nb] their x_scale (tmac_quantize_x)
    float* y;              // [nb][rows]
    int64_t* row_acc;
    int64_t* unit_acc;
    int nb;                // activation vectors handled by this launch (<= NB)
};

TMAC_DEV long long warp_sum_ll(long long v)
{
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// A CTA works on rows in groups of `rpc` rows, `wpr` warps per row; thread t of
// a row decodes chunk t (then t + 32*wpr, ...) and reuses the decoded values for
// every activation vector of the launch.  Row sums: warp shuffle, then the
// row's warps combine through shared memory.
template <int TYPE, int NB>
__global__ void __launch_bounds__(kThreads) blockq_gemv_kernel(BlockqArgs a, int wpr, int rpc)
{
    extern __shared__ __align__(16) uint8_t smem[];
    const int64_t cols = a.cols, cpr = cols / 32;
    const int nb = a.nb;
    // activations as byte planes: x_q = 256 * xh (signed) + xl (unsigned)
    uint8_t* xh = smem;                                                                // [nb][cols]
    uint8_t* xl = smem + (size_t)nb * cols;                                            // [nb][cols]
    float* xs = reinterpret_cast<float*>(smem + ((size_t)nb * cols * 2 + 15) / 16 * 16);  // [16]
    float* red = xs + 16;                                                              // [8]
    long long* part_s = reinterpret_cast<long long*>(red + 8);                        // [8 warps][NB]
    pdl_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rw = warp % wpr, rr = warp / wpr;  // warp within the row, row within the group
    const int tpr = wpr * 32;
    // The weights do not depend on the preceding kernel: fetch and decode this
    // thread's first chunk before waiting for the activations.
    uint32_t v0[16];
    bool have_v0 = false;
    {
        const int64_t r = (int64_t)blockIdx.x * rpc + rr, ch = rw * 32 + lane;
        if (r < a.rows && ch < cpr) {
            decode_chunk<TYPE>(a.raw, r, cpr, ch, __ldg(a.row_inv + r), v0);
            have_v0 = true;
        }
    }
    pdl_wait();  // activations come from the preceding kernel

    if (a.xq_in) {
        const uint2* src = reinterpret_cast<const uint2*>(a.xq_in);
        uint32_t* h4 = reinterpret_cast<uint32_t*>(xh);
        uint32_t* l4 = reinterpret_cast<uint32_t*>(xl);
        for (int64_t j = threadIdx.x; j < (int64_t)nb * cols / 4; j += blockDim.x) {
            const uint2 w = src[j];  // four int16
            h4[j] = __byte_perm(w.x, w.y, 0x7531);
            l4[j] = __byte_perm(w.x, w.y, 0x6420);
        }
        if (threadIdx.x < nb) xs[threadIdx.x] = a.xs_in[threadIdx.x];
    } else {
        // activation quantisation, one vector at a time (tmac_gguf.cpp:889-896)
        for (int b = 0; b < nb; b++) {
            const float* xb = a.x + (int64_t)b * cols;
            float mx = 0.0f;
            for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) mx = fmaxf(mx, fabsf(xb[j]));
            mx = block_max(mx, red, blockDim.x);
            const float s = x_scale_from_max(mx);
            if (threadIdx.x == 0) xs[b] = s;
            for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
                const int16_t q = quantize_one(xb[j], s);
                xh[b * cols + j] = (uint8_t)((uint16_t)q >> 8);
                xl[b * cols + j] = (uint8_t)(q & 0xFF);
            }
        }
    }
    __syncthreads();

    const int64_t upr = (TYPE == TMAC_TYPE_Q5_0) ? cpr : cpr / 8;
    for (int64_t r0 = (int64_t)blockIdx.x * rpc; r0 < a.rows; r0 += (int64_t)gridDim.x * rpc) {
        const int64_t r = r0 + rr;
        const bool row_live = r < a.rows;
        const float ri = row_live ? __ldg(a.row_inv + r) : 1.0f;
        long long acc[NB];
#pragma unroll
        for (int b = 0; b < NB; b++) acc[b] = 0;
        for (int64_t base = 0; base < cpr; base += tpr) {
            const int64_t ch = base + rw * 32 + lane;
            const bool live = row_live && ch < cpr;
            uint32_t v[16];
            if (r0 == (int64_t)blockIdx.x * rpc && base == 0 && have_v0) {
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] = v0[i];
            } else if (live) {
                decode_chunk<TYPE>(a.raw, r, cpr, ch, ri, v);
            }
#pragma unroll
            for (int b = 0; b < NB; b++) {
                if (b >= nb) break;
                long long part = 0;
                if (live) {
                    const uint32_t* h4 = reinterpret_cast<const uint32_t*>(xh + b * cols + ch * 32);
                    const uint32_t* l4 = reinterpret_cast<const uint32_t*>(xl + b * cols + ch * 32);
                    part = chunk_dot(v, h4, l4);
                }
                acc[b] += part;
                if (a.unit_acc) {
                    long long* u = (long long*)a.unit_acc + ((int64_t)b * a.rows + r) * upr;
                    if (TYPE == TMAC_TYPE_Q5_0) {
                        if (live) u[ch] = part;
                    } else {  // a 256-value block = 8 consecutive chunks = 8 consecutive lanes
                        long long sb = part;
                        for (int o = 1; o < 8; o <<= 1) sb += __shfl_xor_sync(0xffffffffu, sb, o);
                        if (live && (lane & 7) == 0) u[ch / 8] = sb;
                    }
                }
            }
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            if (b >= nb) break;
            const long long t = warp_sum_ll(acc[b]);
            if (lane == 0) part_s[warp * NB + b] = t;
        }
        __syncthreads();
        if (rw == 0 && lane < nb && row_live) {
            long long tot = 0;
            for (int w = 0; w < wpr; w++) tot += part_s[(rr * wpr + w) * NB + lane];
            const double v = __ddiv_rn(__dmul_rn((double)tot, (double)xs[lane]), (double)ri);
            a.y[(int64_t)lane * a.rows + r] = (float)v;
            if (a.row_acc) a.row_acc[(int64_t)lane * a.rows + r] = tot;
        }
        __syncthreads();
    }
}

template <int TYPE, int NB>
int launch_nb(const tmac_weight_s* w, const BlockqArgs& a, cudaStream_t s)
{
    const int64_t max_smem = 200 * 1024;
    static bool attr[64] = {};
    if (!attr[w->device & 63]) {
        TMAC_CUDA_TRY(cudaFuncSetAttribute(blockq_gemv_kernel<TYPE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)max_smem));
        attr[w->device & 63] = true;
    }
    // warps per row: enough lanes for every 32-value chunk of a row (at most 8)
    const int64_t cpr = a.cols / 32;
    const int wpr = (int)std::min<int64_t>(8, (cpr + 31) / 32);
    const int rpc = 8 / wpr;
    const size_t smem = ((size_t)a.nb * a.cols * 2 + 15) / 16 * 16 + 24 * 4 + 8 * NB * 8;
    // few enough CTAs that the per-CTA activation quantisation (when x is fp32)
    // stays small next to the rows each CTA works through
    const int64_t cap = (int64_t)num_sms(w->device) * (a.xq_in ? 16 : 2);
    const int grid = (int)std::min<int64_t>((a.rows + rpc - 1) / rpc, cap);
    TMAC_CUDA_TRY(launch_k(blockq_gemv_kernel<TYPE, NB>, dim3(grid), dim3(wpr * rpc * 32), smem, s, a, wpr, rpc));
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

template <int TYPE>
int launch_type(const tmac_weight_s* w, const float* x, const int16_t* xq, const float* xs, float* y,
                int64_t* row_acc, int64_t* unit_acc, int batch, cudaStream_t s)
{
    const int64_t cols = w->cols, cpr = cols / 32;
    const int64_t max_smem = 200 * 1024;
    const int bmax = (int)std::max<int64_t>(1, std::min<int64_t>(16, (max_smem - 4096) / (cols * 2)));
    const int64_t upr = (TYPE == TMAC_TYPE_Q5_0) ? cpr : cpr / 8;
    for (int b0 = 0; b0 < batch; b0 += bmax) {
        BlockqArgs a;
        a.raw = w->data;
        a.row_inv = w->row_norm;
        a.rows = w->rows;
        a.cols = cols;
        a.nb = std::min(bmax, batch - b0);
        a.x = x ? x + (int64_t)b0 * cols : nullptr;
        a.xq_in = xq ? xq + (int64_t)b0 * cols : nullptr;
        a.xs_in = xs ? xs + b0 : nullptr;
        a.y = y + (int64_t)b0 * w->rows;
        a.row_acc = row_acc ? row_acc + (int64_t)b0 * w->rows : nullptr;
        a.unit_acc = unit_acc ? unit_acc + (int64_t)b0 * w->rows * upr : nullptr;
        int rc;
        if (a.nb == 1) rc = launch_nb<TYPE, 1>(w, a, s);
        else if (a.nb <= 2) rc = launch_nb<TYPE, 2>(w, a, s);
        else if (a.nb <= 4) rc = launch_nb<TYPE, 4>(w, a, s);
        else if (a.nb <= 8) rc = launch_nb<TYPE, 8>(w, a, s);
        else rc = launch_nb<TYPE, 16>(w, a, s);
        if (rc) return rc;
    }
    return TMAC_OK;
}

}  // namespace

int register_blockq(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s)
{
    TMAC_CUDA_TRY(cudaMalloc(&w->row_norm, (size_t)w->rows * sizeof(float)));
    const int wpb = 8;
    const unsigned grid = (unsigned)((w->rows + wpb - 1) / wpb);
    switch (w->type) {
    case TMAC_TYPE_Q5_0: row_inv_kernel<TMAC_TYPE_Q5_0><<<grid, wpb * 32, 0, s>>>(d_raw, w->rows, w->cols, w->row_norm); break;
    case TMAC_TYPE_Q4_K: row_inv_kernel<TMAC_TYPE_Q4_K><<<grid, wpb * 32, 0, s>>>(d_raw, w->rows, w->cols, w->row_norm); break;
    case TMAC_TYPE_Q6_K: row_inv_kernel<TMAC_TYPE_Q6_K><<<grid, wpb * 32, 0, s>>>(d_raw, w->rows, w->cols, w->row_norm); break;
    default: return fail(TMAC_ERR_TYPE, "register_blockq: unsupported type");
    }
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int launch_blockq(const tmac_weight_s* w, const float* x, const int16_t* xq, const float* xs, float* y,
                  int64_t* row_acc, int64_t* unit_acc, int batch, cudaStream_t s)
{
    switch (w->type) {
    case TMAC_TYPE_Q5_0: return launch_type<TMAC_TYPE_Q5_0>(w, x, xq, xs, y, row_acc, unit_acc, batch, s);
    case TMAC_TYPE_Q4_K: return launch_type<TMAC_TYPE_Q4_K>(w, x, xq, xs, y, row_acc, unit_acc, batch, s);
    case TMAC_TYPE_Q6_K: return launch_type<TMAC_TYPE_Q6_K>(w, x, xq, xs, y, row_acc, unit_acc, batch, s);
    default: return fail(TMAC_ERR_TYPE, "launch_blockq: unsupported type");
    }
}

}  // namespace tmac
