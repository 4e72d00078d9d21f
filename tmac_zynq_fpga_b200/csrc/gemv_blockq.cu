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
//   v = roundf(w_f32 * row_inv)      with w_f32 in the reference's fp32 order:
//       Q5_0: d*q     Q4_K: (d*sc)*q4 - dmin*m     Q6_K: (d*sc)*q6
// the int64 row sum is  acc = sum v * x_q  and  y = (float)((double)acc * x_scale / (double)row_inv).
//
// Fast decode + exception list.  The GEMV computes every weight with packed
// fp32x2 arithmetic as v' (two values per instruction):
//   Q5_0, Q6_K: v' = RNE(q * c), c = RN(scale * row_inv) per 16/32 values
//   Q4_K:       v' = RNE((RN(q*A - B)) * row_inv)       (the first product is exact)
// v' equals v except where the value sits within an ulp of a half-integer (the
// reference rounds half away from zero; its product is rounded once more).  At
// registration every (row, col) with v != v' is found by running both decodes
// on the device layout, and stored per row as (col, v - v'); the GEMV adds
// sum (v - v') * x_q[col] for the row, so the int64 row sum is the reference's
// exactly.  Measured: well under one exception per 1000 weights.
//
// Device layout (row groups of 8 rows, every section 16-byte aligned, so that a
// CTA's share of groups is one contiguous bulk copy into shared memory):
//   Q5_0 group:  qs[8*cpr][16] | qh[8*cpr] u32 | d[8*cpr] f16   block k = j*8 + r
//   Q4_K group:  the 144-byte GGUF blocks, k = r*nsb + sb
//   Q6_K group:  ql[8*nsb][128] | qh[8*nsb][64] | sc[8*nsb][16] | d[8*nsb] f16, k = r*nsb + sb
// Same bytes per weight as GGUF (22 / 144 / 210 per block); rows padded to 8.
//
// Kernel: each CTA bulk-copies its groups into shared memory BEFORE waiting on
// the preceding kernel (programmatic dependent launch), so in a chain of GEMVs
// the weight stream of one overlaps the tail of the one before.  Then it
// stages x_q as two byte planes (x_q = 256*xh + xl) and decodes from shared
// memory: Q5_0 with 4 lanes per row (8 rows = one group per warp), K-quants
// one warp per row (lane = 4 super-block phases x 8 sub-blocks).
#include "blockq_dev.cuh"

#include <algorithm>
#include <vector>

namespace tmac {
namespace {


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

// One thread per GGUF block: copies it into the grouped layout.
template <int TYPE>
__global__ void relayout_kernel(const uint8_t* __restrict__ raw, int64_t rows, int64_t nblk, uint8_t* __restrict__ out)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * nblk) return;
    const int64_t row = i / nblk, j = i % nblk, g = row >> 3;
    const int r = (int)(row & 7);
    const uint8_t* b = raw + i * Geo<TYPE>::kBlockBytes;
    uint8_t* G = out + g * Geo<TYPE>::group_bytes(nblk);
    if (TYPE == TMAC_TYPE_Q5_0) {
        const int64_t k = j * 8 + r;
        for (int t = 0; t < 16; t++) G[16 * k + t] = b[6 + t];
        for (int t = 0; t < 4; t++) G[128 * nblk + 4 * k + t] = b[2 + t];
        for (int t = 0; t < 2; t++) G[160 * nblk + 2 * k + t] = b[t];
    } else if (TYPE == TMAC_TYPE_Q4_K) {
        const int64_t k = r * nblk + j;
        for (int t = 0; t < 144; t++) G[144 * k + t] = b[t];
    } else {
        const int64_t k = r * nblk + j;
        for (int t = 0; t < 128; t++) G[128 * k + t] = b[t];
        for (int t = 0; t < 64; t++) G[1024 * nblk + 64 * k + t] = b[128 + t];
        for (int t = 0; t < 16; t++) G[1536 * nblk + 16 * k + t] = b[192 + t];
        for (int t = 0; t < 2; t++) G[1664 * nblk + 2 * k + t] = b[208 + t];
    }
}

// ------------------------------------------------------ exception finding --
// Warp per row.  mode 0: count the values with v != v' into cnt[row];
// mode 1: write (row, col, v - v', 0) at cursor[row]++.
template <int TYPE>
__global__ void exceptions_kernel(const uint8_t* __restrict__ data, const float* __restrict__ row_inv, int64_t rows,
                                  int64_t cols, int* __restrict__ cnt, int* __restrict__ cursor, int4* __restrict__ exc)
{
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int64_t nblk = cols / Geo<TYPE>::kBlockVals, cpr = cols / 32;
    const GlobalBytes G{data + (row >> 3) * Geo<TYPE>::group_bytes(nblk)};
    const float ri = row_inv[row];
    int n = 0;
    for (int64_t ch = lane; ch < cpr; ch += 32) {
        Chunk c;
        load_chunk<TYPE>(G, (int)(row & 7), (uint32_t)nblk, (uint32_t)ch, c);
        uint32_t vw[16];
        fast_values<TYPE>(c, ri, vw);
        for (int e = 0; e < 32; e++) {
            const int vf = (int)(int16_t)((vw[e >> 1] >> (16 * (e & 1))) & 0xFFFFu);
            const int ve = exact_value<TYPE>(c, e, ri);
            if (ve != vf) {
                if (cursor) {
                    const int at = atomicAdd(cursor + row, 1);
                    exc[at] = make_int4((int)row, (int)(ch * 32 + e), ve - vf, 0);
                }
                n++;
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
    if (lane == 0 && cnt) cnt[row] = n;
}

// ------------------------------------------------------ exact int16 planes --
// The reference's int16 weights v (exact decode) as byte planes for the tensor-
// core GEMM: wh[row][col] = v >> 8 (signed), wl[row][col] = v & 0xFF.  One warp
// per row, lane per chunk; rows at or beyond `rows` are left as they are.
template <int TYPE>
__global__ void planes_kernel(const uint8_t* __restrict__ data, const float* __restrict__ row_inv, int64_t rows,
                              int64_t cols, int8_t* __restrict__ wh, uint8_t* __restrict__ wl)
{
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int64_t nblk = cols / Geo<TYPE>::kBlockVals, cpr = cols / 32;
    const GlobalBytes G{data + (row >> 3) * Geo<TYPE>::group_bytes(nblk)};
    const float ri = row_inv[row];
    for (int64_t ch = lane; ch < cpr; ch += 32) {
        Chunk c;
        load_chunk<TYPE>(G, (int)(row & 7), (uint32_t)nblk, (uint32_t)ch, c);
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            uint32_t h = 0, l = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int v = exact_value<TYPE>(c, 4 * i + k, ri);
                h |= (uint32_t)((v >> 8) & 0xFF) << (8 * k);
                l |= (uint32_t)(v & 0xFF) << (8 * k);
            }
            hw[i] = h;
            lw[i] = l;
        }
        uint4* ph = reinterpret_cast<uint4*>(wh + row * cols + ch * 32);
        uint4* pl = reinterpret_cast<uint4*>(wl + row * cols + ch * 32);
        ph[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        ph[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        pl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        pl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    }
}

// ------------------------------------------------------------------ GEMV --
struct BqArgs {
    const uint8_t* data;     // grouped layout
    const float* row_inv;
    const double* rinv;      // RN(1 / row_inv)
    int64_t rows, cols, groups, group_bytes;
    int gpc;                 // groups per CTA
    const float* x;          // [nb][cols] fp32 activations, or
    const int16_t* xq_in;    // [nb][cols] quantised activations, or
    const uint8_t* xp_in;    // [nb][2][cols] the same as byte planes (high, low)
    const float* xs_in;      // [nb] x_scale of xq_in / xp_in
    const float* xmax_parts; // optional (nb 1, fp32 x): max |x| is the maximum of these
    int n_parts;
    float* y;                // [nb][rows]
    int64_t* row_acc;
    int64_t* unit_acc;
    const int* exc_ptr;      // [rows + 1]
    const int4* exc;         // (row, col, v - v', 0), grouped by row
    int* err;
    int nb;
};

#ifdef TMAC_TRACE
// Diagnostic build only (-DTMAC_TRACE): per-CTA clock64 stamps of the kernel's
// phases and per-warp main-loop start/end, read back with tmac_trace_read_blockq*.
__device__ unsigned long long g_bq_trace[1024][12];
__device__ unsigned long long g_bq_wtrace[1024][16][2];  // per warp: main-loop start, end
#define BQ_STAMP(i)                                                                   \
    do {                                                                              \
        if (threadIdx.x == 0 && blockIdx.x < 1024) g_bq_trace[blockIdx.x][i] = clock64(); \
    } while (0)
#else
#define BQ_STAMP(i) \
    do {            \
    } while (0)
#endif

constexpr int kExcCap = 512;  // exception entries staged in shared memory per pass

// Shared memory of one CTA (offsets from the dynamic base; all 16-byte aligned).
struct BqSmem {
    int64_t w, x, acc, ri, ep, exc, xs, red, bar, total;
    __host__ __device__ BqSmem(int64_t gpc, int64_t group_bytes, int64_t nb, int64_t cols)
    {
        const int64_t rows = gpc * 8;
        w = 0;
        x = w + gpc * group_bytes;                   // [nb][2][cols] planes
        acc = x + 2 * nb * cols;                     // uint32 [2][rows][nb]: low, high words
        ri = acc + rows * nb * 8;                    // float [rows]
        ep = ri + (rows * 4 + 15) / 16 * 16;         // int [rows + 4]: exception offsets
        exc = ep + (rows + 4) * 4;                   // int4 [kExcCap]
        xs = exc + kExcCap * 16;                     // float [16]
        red = xs + 64;                               // float [32]
        bar = red + 128;                             // 3 mbarriers
        total = bar + 24;
    }
};

template <int TYPE, int NB>
__global__ void __launch_bounds__(NB == 1 ? 1024 : 512) blockq_gemv_kernel(BqArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int64_t cols = a.cols, cpr = cols / 32, nblk = cols / Geo<TYPE>::kBlockVals;
    const int nb = a.nb;
    const BqSmem L(a.gpc, a.group_bytes, nb, cols);
    const int64_t g0 = (int64_t)blockIdx.x * a.gpc;
    const int ng = (int)min((int64_t)a.gpc, a.groups - g0);
    const int rows_cta = ng * 8;
    const int64_t row0 = g0 * 8;
    uint8_t* wsm = smem + L.w;
    uint8_t* xpl = smem + L.x;
    uint32_t* acc_lo = reinterpret_cast<uint32_t*>(smem + L.acc);   // [rows_cta * nb]
    uint32_t* acc_hi = acc_lo + (int64_t)a.gpc * 8 * nb;
    int* ep_s = reinterpret_cast<int*>(smem + L.ep);
    float* ri_s = reinterpret_cast<float*>(smem + L.ri);
    int4* exc_s = reinterpret_cast<int4*>(smem + L.exc);
    float* xs_s = reinterpret_cast<float*>(smem + L.xs);
    float* red = reinterpret_cast<float*>(smem + L.red);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);  // [0] weights, [1] activations, [2] exceptions
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    // the epilogue's reciprocal of this thread's first (row, vector), loaded now
    // so that its latency hides behind the main loop
    const double rinv0 = NB == 1 && (int)threadIdx.x < rows_cta && row0 + (int)threadIdx.x < a.rows
                             ? __ldg(a.rinv + row0 + (int)threadIdx.x)
                             : 0.0;

    BQ_STAMP(0);
    // ---- prologue: everything here depends on the weights only.  Thread 0
    // stages the CTA's weights, row_inv and exception offsets with bulk copies
    // completing on bar[0]; thread 32 (thread 0 in a one-warp CTA) looks up
    // the CTA's exception range and stages those entries on bar[2], so its
    // global loads do not hold up the weight copies.
    const unsigned exc_thread = blockDim.x > 32 ? 32u : 0u;
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
        const uint32_t wbytes = (uint32_t)(ng * a.group_bytes), rbytes = (uint32_t)(rows_cta * 4);
        const uint32_t ebytes = (uint32_t)((rows_cta + 4) * 4);
        mbar_arrive_expect_tx(&bar[0], wbytes + rbytes + ebytes);
        const uint8_t* src = a.data + g0 * a.group_bytes;
        for (uint32_t off = 0; off < wbytes; off += 32768u)
            bulk_g2s(wsm + off, src + off, min(32768u, wbytes - off), &bar[0]);
        bulk_g2s(ri_s, a.row_inv + row0, rbytes, &bar[0]);  // row_inv and exc_ptr are padded
        bulk_g2s(ep_s, a.exc_ptr + row0, ebytes, &bar[0]);  // to whole groups (+4)
    }
    if (threadIdx.x == exc_thread) {
        mbar_init(&bar[2], 1);
        fence_mbar_init();
        const int e0 = __ldg(a.exc_ptr + row0), e1 = __ldg(a.exc_ptr + min(row0 + rows_cta, a.rows));
        const uint32_t n = (uint32_t)min(e1 - e0, kExcCap);
        mbar_arrive_expect_tx(&bar[2], n * 16);
        if (n) bulk_g2s(exc_s, a.exc + e0, n * 16, &bar[2]);
    }
    pdl_launch();
    for (int t = threadIdx.x; t < rows_cta * nb; t += blockDim.x) acc_lo[t] = acc_hi[t] = 0;

    BQ_STAMP(1);
    // ---- activations come from the preceding kernel
    pdl_wait();
    if (a.xp_in) {
        if (threadIdx.x == 0) {
            const uint32_t bytes = (uint32_t)(2 * nb * cols);
            mbar_arrive_expect_tx(&bar[1], bytes);
            for (uint32_t off = 0; off < bytes; off += 32768u)
                bulk_g2s(xpl + off, a.xp_in + off, min(32768u, bytes - off), &bar[1]);
        }
        if (threadIdx.x < nb) xs_s[threadIdx.x] = a.xs_in[threadIdx.x];
    } else if (a.xq_in) {
        // int16 input: split into the byte planes while staging (4 loads in flight)
        const uint4* src = reinterpret_cast<const uint4*>(a.xq_in);
        const int64_t n8 = (int64_t)nb * cols / 8;
        for (int64_t j0 = threadIdx.x; j0 < n8; j0 += 4 * (int64_t)blockDim.x) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int64_t j = j0 + u * (int64_t)blockDim.x;
                if (j < n8) v[u] = src[j];
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int64_t j = j0 + u * (int64_t)blockDim.x;
                if (j >= n8) break;
                const int64_t e = j * 8, b = e / cols, c = e % cols;
                uint8_t* p = xpl + b * 2 * cols + c;
                *reinterpret_cast<uint2*>(p) =
                    make_uint2(__byte_perm(v[u].x, v[u].y, 0x7531), __byte_perm(v[u].z, v[u].w, 0x7531));
                *reinterpret_cast<uint2*>(p + cols) =
                    make_uint2(__byte_perm(v[u].x, v[u].y, 0x6420), __byte_perm(v[u].z, v[u].w, 0x6420));
            }
        }
        if (threadIdx.x < nb) xs_s[threadIdx.x] = a.xs_in[threadIdx.x];
    } else {
        // activation quantisation, one vector at a time (tmac_gguf.cpp:889-896);
        // x stays in registers between the max and the quantisation
        constexpr int kXr = 12;
        for (int b = 0; b < nb; b++) {
            const float* xb = a.x + (int64_t)b * cols;
            float xv[kXr];
            float mx = 0.0f;
#pragma unroll
            for (int k = 0; k < kXr; k++) {
                const int64_t j = threadIdx.x + (int64_t)k * blockDim.x;
                xv[k] = (j < cols) ? xb[j] : 0.0f;
                mx = fmaxf(mx, fabsf(xv[k]));
            }
            if (a.xmax_parts) {  // the producer left per-CTA maxima: no reduction here
                mx = 0.0f;
                for (int i = 0; i < a.n_parts; i++) mx = fmaxf(mx, __ldg(a.xmax_parts + i));
            } else {
                for (int64_t j = threadIdx.x + (int64_t)kXr * blockDim.x; j < cols; j += blockDim.x)
                    mx = fmaxf(mx, fabsf(xb[j]));
                mx = block_max(mx, red, blockDim.x);
            }
            const float s = x_scale_from_max(mx);
            if (threadIdx.x == 0) xs_s[b] = s;
            uint8_t* p = xpl + (int64_t)b * 2 * cols;
#pragma unroll
            for (int k = 0; k < kXr; k++) {
                const int64_t j = threadIdx.x + (int64_t)k * blockDim.x;
                if (j < cols) {
                    const int16_t q = quantize_one(xv[k], s);
                    p[j] = (uint8_t)((uint16_t)q >> 8);
                    p[cols + j] = (uint8_t)(q & 0xFF);
                }
            }
            for (int64_t j = threadIdx.x + (int64_t)kXr * blockDim.x; j < cols; j += blockDim.x) {
                const int16_t q = quantize_one(xb[j], s);
                p[j] = (uint8_t)((uint16_t)q >> 8);
                p[cols + j] = (uint8_t)(q & 0xFF);
            }
        }
    }
    __syncthreads();
    BQ_STAMP(2);
    // A wait that gives up records TMAC_ERR_TIMEOUT; before the CTA exits, the
    // threads that issued bulk copies wait (bounded again) for those copies, so
    // no copy lands in shared memory after the CTA is gone.
    auto drain_and_exit = [&]() {
        if (threadIdx.x == 0) {
            mbar_wait_bounded(&bar[0], 0, nullptr);
            if (a.xp_in) mbar_wait_bounded(&bar[1], 0, nullptr);
        }
        if (threadIdx.x == exc_thread) mbar_wait_bounded(&bar[2], 0, nullptr);
    };
    if (!mbar_wait_bounded(&bar[0], 0, a.err)) return drain_and_exit();
    BQ_STAMP(3);
    if (a.xp_in && !mbar_wait_bounded(&bar[1], 0, a.err)) return drain_and_exit();
    BQ_STAMP(4);

    // ---- main loop.  Work items are (slot, step): Q5_0 slot = a group of 8
    // rows (lane = row r + 8 * l, chunk j = 4*step + l: 4 lanes per row), K-quant
    // slot = one row (lane = 8 * phase + sub-block, super-block = 4*step +
    // phase).  Each warp takes a contiguous run of items and adds its row sums
    // into acc_s when the slot changes.
    const bool q5 = (TYPE == TMAC_TYPE_Q5_0);
    const int64_t upr = q5 ? cpr : nblk;
    const int slots = q5 ? ng : rows_cta;
    const int steps = (int)(q5 ? (cpr + 3) / 4 : (nblk + 3) / 4);
    const int items = slots * steps;
    const int it0 = (int)((int64_t)items * warp / nwarps), it1 = (int)((int64_t)items * (warp + 1) / nwarps);
    const int r_lane = q5 ? (lane & 7) : 0;
    const int l_lane = q5 ? (lane >> 3) : lane;
    long long acc[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) acc[b] = 0;
#ifdef TMAC_TRACE
    if (lane == 0 && blockIdx.x < 1024) g_bq_wtrace[blockIdx.x][warp][0] = clock64();
#endif
    const uint32_t wsm_a = smem_addr(wsm);
    int slot = it0 / steps, s = it0 % steps;
    for (int it = it0; it < it1; it++) {
        const int rr = q5 ? slot * 8 + r_lane : slot;  // row within the CTA
        const SharedBytes G{wsm_a + (uint32_t)(rr >> 3) * (uint32_t)a.group_bytes};
        const int r = rr & 7;
        const float ri = ri_s[rr];
        const uint32_t ch = q5 ? (uint32_t)(4 * s + l_lane) : (uint32_t)(4 * s + (lane >> 3)) * 8 + (lane & 7);
        const bool cl = ch < cpr;
        uint32_t vw[16];
        if (cl) {
            Chunk c;
            load_chunk<TYPE>(G, r, (uint32_t)nblk, ch, c);
            fast_values<TYPE>(c, ri, vw);
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            if (b >= nb) break;
            long long part = 0;
            if (cl) {
                const uint8_t* p = xpl + (int64_t)b * 2 * cols + ch * 32;
                part = chunk_dot(vw, p, p + cols);
            }
            acc[b] += part;
            if (a.unit_acc) {
                const int64_t row = row0 + rr;
                long long* u = (long long*)a.unit_acc + ((int64_t)b * a.rows + row) * upr;
                if (q5) {
                    if (cl && row < a.rows) u[ch] = part;
                } else {  // a 256-value block = 8 chunks held by 8 consecutive lanes
                    long long sb = part;
                    for (int o = 1; o < 8; o <<= 1) sb += __shfl_xor_sync(0xffffffffu, sb, o);
                    if (cl && (lane & 7) == 0 && row < a.rows) u[ch / 8] = sb;
                }
            }
        }
        // flush the row sums when this warp's next item is in another slot
        if (++s == steps || it + 1 == it1) {
#pragma unroll
            for (int b = 0; b < NB; b++) {
                if (b >= nb) break;
                long long v = acc[b];
                for (int o = q5 ? 8 : 1; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (l_lane == 0) acc_add(&acc_lo[rr * nb + b], &acc_hi[rr * nb + b], v);
                acc[b] = 0;
            }
            if (s == steps) {
                s = 0;
                slot++;
            }
        }
    }
#ifdef TMAC_TRACE
    if (lane == 0 && blockIdx.x < 1024) g_bq_wtrace[blockIdx.x][warp][1] = clock64();
#endif
    BQ_STAMP(5);

    // ---- exceptions: acc += (v - v') * x_q[col], one thread per (entry,
    // vector).  The adds are atomic like the main loop's, so a warp starts on
    // them as soon as its own main-loop items are done -- unless per-unit sums
    // are wanted: the main loop stores those, so it must finish first.
    if (a.unit_acc) __syncthreads();
    if (!mbar_wait_bounded(&bar[2], 0, a.err)) return drain_and_exit();
    const int e0 = ep_s[0], e1 = ep_s[rows_cta];
    for (int base = e0; base < e1; base += kExcCap) {
        const int n = min(e1 - base, kExcCap);
        if (base != e0) {  // more entries than the prologue staged
            __syncthreads();
            for (int t = threadIdx.x; t < n; t += blockDim.x) exc_s[t] = __ldg(a.exc + base + t);
            __syncthreads();
        }
        for (int t = threadIdx.x; t < n * nb; t += blockDim.x) {
            const int4 ex = exc_s[t / nb];
            const int b = t % nb, rr = ex.x - (int)row0;
            const long long d = (long long)ex.z * xq_at(xpl, cols, b, ex.y);
            acc_add(&acc_lo[rr * nb + b], &acc_hi[rr * nb + b], d);
            if (a.unit_acc) {
                long long* u = (long long*)a.unit_acc + ((int64_t)b * a.rows + ex.x) * upr;
                atomicAdd(reinterpret_cast<unsigned long long*>(&u[q5 ? ex.y / 32 : ex.y / 256]), (unsigned long long)d);
            }
        }
    }
    __syncthreads();
    BQ_STAMP(6);
    // ---- rows: y = (float)((double)acc * x_scale / (double)row_inv)
    for (int t = threadIdx.x; t < rows_cta * nb; t += blockDim.x) {
        const int rr = t / nb, b = t % nb;
        const int64_t row = row0 + rr;
        if (row >= a.rows) continue;
        const long long tot = (long long)(((unsigned long long)acc_hi[rr * nb + b] << 32) | acc_lo[rr * nb + b]);
        const double rv = (NB == 1 && t == (int)threadIdx.x) ? rinv0 : __ldg(a.rinv + row);
        a.y[(int64_t)b * a.rows + row] = quotient_f32(__dmul_rn((double)tot, (double)xs_s[b]), rv, ri_s[rr]);
        if (a.row_acc) a.row_acc[(int64_t)b * a.rows + row] = tot;
    }
#ifdef TMAC_TRACE
    __syncthreads();
    if (threadIdx.x == 0 && blockIdx.x < 1024) {
        uint32_t smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        g_bq_trace[blockIdx.x][7] = clock64();
        g_bq_trace[blockIdx.x][8] = smid;
    }
#endif
}

constexpr int64_t kMaxSmem = 220 * 1024;

template <int TYPE, int NB>
int launch_nb(const tmac_weight_s* w, BqArgs a, cudaStream_t s)
{
    static bool attr[64] = {};
    if (!attr[w->device & 63]) {
        TMAC_CUDA_TRY(cudaFuncSetAttribute(blockq_gemv_kernel<TYPE, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kMaxSmem));
        attr[w->device & 63] = true;
    }
    // one wave: every SM gets ceil(groups / SMs) groups, fewer if shared memory
    // cannot hold them next to the activations
    const int64_t sms = num_sms(w->device);
    int64_t gpc = std::max<int64_t>(1, (a.groups + sms - 1) / sms);
    while (gpc > 1 && BqSmem(gpc, a.group_bytes, a.nb, a.cols).total > kMaxSmem) gpc--;
    a.gpc = (int)gpc;
    const int grid = (int)((a.groups + gpc - 1) / gpc);
    const int64_t slots = (TYPE == TMAC_TYPE_Q5_0) ? gpc : gpc * 8;
    const int64_t steps = (TYPE == TMAC_TYPE_Q5_0) ? (a.cols / 32 + 3) / 4 : (a.cols / 256 + 3) / 4;
    // batch 1 fits 64 registers a thread: up to 32 warps hide the decode's latency
    const int warps = (int)std::max<int64_t>(1, std::min<int64_t>(NB == 1 ? 32 : 16, slots * steps));
    TMAC_CUDA_TRY(launch_k(blockq_gemv_kernel<TYPE, NB>, dim3(grid), dim3(warps * 32),
                           (size_t)BqSmem(gpc, a.group_bytes, a.nb, a.cols).total, s, a));
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

template <int TYPE>
int launch_type(const tmac_weight_s* w, const float* x, const int16_t* xq, const uint8_t* xp, const float* xs,
                float* y, int64_t* row_acc, int64_t* unit_acc, int batch, cudaStream_t s, const float* xmax_parts,
                int n_parts)
{
    if (xmax_parts && (batch != 1 || !x)) return fail(TMAC_ERR_SHAPE, "per-CTA maxima need batch 1 and fp32 x");
    const int64_t cols = w->cols, cpr = cols / 32;
    // activation planes take 2*cols bytes per vector next to one group of weights
    const int64_t fixed = BqSmem(1, w->group_bytes, 0, cols).total + 16 * 8 * 8;
    const int bmax = (int)std::max<int64_t>(1, std::min<int64_t>(16, (kMaxSmem - fixed) / (cols * 2)));
    const int64_t upr = (TYPE == TMAC_TYPE_Q5_0) ? cpr : cols / 256;
    int* err = device_error_word(w->device);
    for (int b0 = 0; b0 < batch; b0 += bmax) {
        BqArgs a;
        a.data = w->data;
        a.row_inv = w->row_norm;
        a.rinv = reinterpret_cast<const double*>(w->grinv);
        a.rows = w->rows;
        a.cols = cols;
        a.groups = w->groups;
        a.group_bytes = w->group_bytes;
        a.gpc = 1;
        a.nb = std::min(bmax, batch - b0);
        a.x = x ? x + (int64_t)b0 * cols : nullptr;
        a.xq_in = xq ? xq + (int64_t)b0 * cols : nullptr;
        a.xp_in = xp ? xp + (int64_t)b0 * 2 * cols : nullptr;
        a.xs_in = xs ? xs + b0 : nullptr;
        a.xmax_parts = xmax_parts;
        a.n_parts = n_parts;
        a.y = y + (int64_t)b0 * w->rows;
        a.row_acc = row_acc ? row_acc + (int64_t)b0 * w->rows : nullptr;
        a.unit_acc = unit_acc ? unit_acc + (int64_t)b0 * w->rows * upr : nullptr;
        a.exc_ptr = w->exc_ptr;
        a.exc = reinterpret_cast<const int4*>(w->exc);
        a.err = err;
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

// RN(1 / row_inv) in double for the epilogue (quotient_f32); rows padded to groups.
__global__ void rinv_kernel(const float* __restrict__ ri, int64_t n, double* __restrict__ out)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __ddiv_rn(1.0, (double)ri[i]);
}

template <int TYPE>
int register_type(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s)
{
    const int64_t rows = w->rows, nblk = w->cols / Geo<TYPE>::kBlockVals;
    // row_inv padded to whole row groups (zeros), so a CTA copies its slice in one piece
    TMAC_CUDA_TRY(cudaMalloc(&w->row_norm, (size_t)(rows + 7) / 8 * 8 * sizeof(float)));
    TMAC_CUDA_TRY(cudaMemsetAsync(w->row_norm, 0, (size_t)(rows + 7) / 8 * 8 * sizeof(float), s));
    const int wpb = 8;
    const unsigned rgrid = (unsigned)((rows + wpb - 1) / wpb);
    row_inv_kernel<TYPE><<<rgrid, wpb * 32, 0, s>>>(d_raw, rows, w->cols, w->row_norm);
    TMAC_CUDA_TRY(cudaGetLastError());
    const int64_t prow = (rows + 7) / 8 * 8;
    TMAC_CUDA_TRY(cudaMalloc(&w->grinv, (size_t)prow * sizeof(double)));
    rinv_kernel<<<(unsigned)((prow + 255) / 256), 256, 0, s>>>(w->row_norm, prow, reinterpret_cast<double*>(w->grinv));
    TMAC_CUDA_TRY(cudaGetLastError());

    w->groups = (rows + 7) / 8;
    w->group_bytes = Geo<TYPE>::group_bytes(nblk);
    w->data_bytes = (size_t)(w->groups * w->group_bytes);
    TMAC_CUDA_TRY(cudaMalloc(&w->data, w->data_bytes));
    TMAC_CUDA_TRY(cudaMemsetAsync(w->data, 0, w->data_bytes, s));
    const int64_t nblocks = rows * nblk;
    relayout_kernel<TYPE><<<(unsigned)((nblocks + 255) / 256), 256, 0, s>>>(d_raw, rows, nblk, w->data);
    TMAC_CUDA_TRY(cudaGetLastError());

    // exception lists: count, prefix-sum on the host, fill
    int* d_cnt = nullptr;
    // exc_ptr padded to whole row groups + 4 (a CTA copies rows_cta + 4 offsets)
    const int64_t nptr = w->groups * 8 + 4;
    TMAC_CUDA_TRY(cudaMalloc(&w->exc_ptr, (size_t)nptr * sizeof(int)));
    TMAC_CUDA_TRY(cudaMalloc(&d_cnt, (size_t)rows * sizeof(int)));
    exceptions_kernel<TYPE><<<rgrid, wpb * 32, 0, s>>>(w->data, w->row_norm, rows, w->cols, d_cnt, nullptr, nullptr);
    cudaError_t e = cudaGetLastError();
    std::vector<int> cnt(rows), ptr(nptr, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(cnt.data(), d_cnt, rows * sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        cudaFree(d_cnt);
        return cuda_fail(e, "exception count");
    }
    for (int64_t r = 0; r < rows; r++) ptr[r + 1] = ptr[r] + cnt[r];
    for (int64_t r = rows + 1; r < nptr; r++) ptr[r] = ptr[rows];
    w->n_exc = ptr[rows];
    e = cudaMemcpy(w->exc_ptr, ptr.data(), nptr * sizeof(int), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMalloc(&w->exc, std::max<int64_t>(1, w->n_exc) * sizeof(int4));
    if (e == cudaSuccess) e = cudaMemcpy(d_cnt, ptr.data(), rows * sizeof(int), cudaMemcpyHostToDevice);  // cursors
    if (e == cudaSuccess && w->n_exc > 0) {
        exceptions_kernel<TYPE><<<rgrid, wpb * 32, 0, s>>>(w->data, w->row_norm, rows, w->cols, nullptr, d_cnt,
                                                           reinterpret_cast<int4*>(w->exc));
        e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    }
    cudaFree(d_cnt);
    if (e != cudaSuccess) return cuda_fail(e, "exception fill");
    return TMAC_OK;
}

}  // namespace

#ifdef TMAC_TRACE
extern "C" int tmac_trace_read_blockq(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, g_bq_trace, sizeof(g_bq_trace));
}
extern "C" int tmac_trace_read_blockq_warps(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, g_bq_wtrace, sizeof(g_bq_wtrace));
}
#endif

int register_blockq(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s)
{
    switch (w->type) {
    case TMAC_TYPE_Q5_0: return register_type<TMAC_TYPE_Q5_0>(w, d_raw, s);
    case TMAC_TYPE_Q4_K: return register_type<TMAC_TYPE_Q4_K>(w, d_raw, s);
    case TMAC_TYPE_Q6_K: return register_type<TMAC_TYPE_Q6_K>(w, d_raw, s);
    default: return fail(TMAC_ERR_TYPE, "register_blockq: unsupported type");
    }
}

int blockq_planes(const tmac_weight_s* w, int8_t* wh, uint8_t* wl, cudaStream_t s)
{
    const unsigned grid = (unsigned)((w->rows + 7) / 8);
    switch (w->type) {
    case TMAC_TYPE_Q5_0: planes_kernel<TMAC_TYPE_Q5_0><<<grid, 256, 0, s>>>(w->data, w->row_norm, w->rows, w->cols, wh, wl); break;
    case TMAC_TYPE_Q4_K: planes_kernel<TMAC_TYPE_Q4_K><<<grid, 256, 0, s>>>(w->data, w->row_norm, w->rows, w->cols, wh, wl); break;
    case TMAC_TYPE_Q6_K: planes_kernel<TMAC_TYPE_Q6_K><<<grid, 256, 0, s>>>(w->data, w->row_norm, w->rows, w->cols, wh, wl); break;
    default: return fail(TMAC_ERR_TYPE, "blockq_planes: unsupported type");
    }
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int launch_blockq(const tmac_weight_s* w, const float* x, const int16_t* xq, const uint8_t* xp, const float* xs,
                  float* y, int64_t* row_acc, int64_t* unit_acc, int batch, cudaStream_t s, const float* xmax_parts,
                  int n_parts)
{
    switch (w->type) {
    case TMAC_TYPE_Q5_0:
        return launch_type<TMAC_TYPE_Q5_0>(w, x, xq, xp, xs, y, row_acc, unit_acc, batch, s, xmax_parts, n_parts);
    case TMAC_TYPE_Q4_K:
        return launch_type<TMAC_TYPE_Q4_K>(w, x, xq, xp, xs, y, row_acc, unit_acc, batch, s, xmax_parts, n_parts);
    case TMAC_TYPE_Q6_K:
        return launch_type<TMAC_TYPE_Q6_K>(w, x, xq, xp, xs, y, row_acc, unit_acc, batch, s, xmax_parts, n_parts);
    default: return fail(TMAC_ERR_TYPE, "launch_blockq: unsupported type");
    }
}

}  // namespace tmac
