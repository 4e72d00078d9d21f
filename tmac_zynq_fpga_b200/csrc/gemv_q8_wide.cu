// gemv_q8_wide.cu -- the Q8_0 GEMV of tall matrices (the logits: 151936 x 896)
// on the tensor cores, bit-exact with the reference's Q8_0 FPGA path
// (matmul_fpga_q8, sim/tmac_gguf.cpp:948-1085; MatmulAccel::compute_int16's
// Q8 branch, sim/fpga_sim.hpp:322-349, :466-491) and with gemv_q8_0.cu.
//
// The same exact integer identity as gemv_q8_0.cu: with cs = 256*ch + cl and
// biased quants q' = q + 128,
//   floor(q*cs/256) = q*ch + e,  e + 128 = (q'*cl + 128*(256 - cl)) >> 8,
// so the 32-column block sum of deq*x_q is
//   ch * (S(q',x_q) - 128*Sx) + (S(e',x_q) - 128*Sx)
// with e' = e + 128, S(a,b) the block's dot product and Sx the block's sum of
// x_q.  The CUDA-core GEMV spends ~9 instructions per 4 columns on this; here
// the dot products run as tcgen05.mma kind::i8 and the CUDA cores only form e'
// (5 instructions per 4 columns).
//
// x_q (|x_q| <= 32767) is split into three signed bytes,
//   x_q = 16384*x2 + 128*x1 + x0,  x0, x1 in [0, 127], x2 in [-2, 1],
// so one signed B operand of 96 rows serves the unsigned q' and e' tiles: rows
// n, 32 + n and 64 + n hold x0, x1 and x2 of the 32-column block n and zeros
// outside it, and TMEM column n (+32, +64) of an accumulator collects block
// n's partial sums (cols <= 896: 28 blocks).  Per 32 columns of K that is two
// MMAs (M = 128 weight rows, N = 96), one for q' and one for e'.  Accumulators
// of 96 columns for q' and e' per 128-row group, two groups in flight: 512
// TMEM columns.
//
// Device layout (register_q8_wide): q' as a row-major plane [rows_pad][cols]
// (TMA, 128-byte swizzle, boxes of 128 rows x 128 columns), the combined
// scales as u16 [rows_pad][nbp] (nbp = blocks rounded up to 8) and row_scale
// [rows_pad]: 956 bytes per row for cols = 896 against 952 for the GGUF blocks.
//
// Warp roles (one persistent CTA per SM over 128-row groups):
//   warp 0      TMA loads of q' k-blocks (4-stage ring) and each group's scales
//   warp 1      TMEM owner; one lane issues the q' MMAs
//   warp 2      one lane issues the e' MMAs (two issuing warps: the issue of
//               a small-N MMA, not the tensor pipe, bounds one warp's rate)
//   warps 3-18  e' of each k-block into a 3-slot ring (same swizzled layout)
//   warps 19-22 epilogue: TMEM -> block sums -> tile sums -> y, in tile order
//               with fp64 as tmac_gguf.cpp:1075-1076
// Every wait is bounded (~2 s): on expiry the kernel records TMAC_ERR_TIMEOUT,
// stops issuing, waits (bounded) for the copies and MMAs it has in flight,
// frees its TMEM and returns.
#include "tcgen05.cuh"
#include "xchg.cuh"

#include <algorithm>
#include <cstdlib>

namespace tmac {
namespace {

constexpr int WM = 128;                 // weight rows per group (MMA M)
constexpr int WK = 128;                 // columns per k-block (one swizzle row)
constexpr int kMaxKB = 7;               // cols <= 896
constexpr int kMaxBlk = 32;             // 32-column block slots per row
constexpr int kBN = 96;                 // MMA N: x0 | x1 | x2 rows of every block
constexpr int kAStages = 4, kEStages = 3;
constexpr uint32_t kATile = WM * WK;    // 16 KB
constexpr uint32_t kBTile = kBN * WK;   // 12 KB
constexpr int kEWarps = 16, kEpiWarps = 4;
constexpr int kWarpE0 = 3, kWarpEpi0 = kWarpE0 + kEWarps;
constexpr int kThreads = (kWarpEpi0 + kEpiWarps) * 32;  // 736
constexpr int kPrologueThreads = (kEWarps + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;     // group buffer b at b*256: q' at +0, e' at +128 (96 each)
constexpr int64_t kWideMinRows = 16384;
static_assert(kAStages > kEStages, "an e' slot is reused after its k-block's a_empty phase");

// Shared memory, from a 1024-byte aligned base.
constexpr uint32_t kOffA = 0;
constexpr uint32_t kOffE = kOffA + kAStages * kATile;
constexpr uint32_t kOffB = kOffE + kEStages * kATile;
constexpr uint32_t kOffCs = kOffB + kMaxKB * kBTile;            // [2][128][kMaxBlk] u16
constexpr uint32_t kOffRs = kOffCs + 2 * WM * kMaxBlk * 2;      // [2][128] f32
constexpr uint32_t kOffXq = kOffRs + 2 * WM * 4;                // [kMaxKB * 128] i16
constexpr uint32_t kOffSx = kOffXq + kMaxKB * WK * 2;           // [32] i32
constexpr uint32_t kOffRed = kOffSx + kMaxBlk * 4;              // [32] f32, xs at [24], abort at [25]
constexpr uint32_t kOffBar = kOffRed + 32 * 4;
constexpr int kNumBars = 2 * kAStages + kEStages + 2 + 2 + 2 + 2 + 1 + 2;
constexpr uint32_t kOffSlot = kOffBar + kNumBars * 8;
constexpr size_t kSmem = kOffSlot + 16 + 1024;                  // + alignment slack
static_assert(kSmem <= 227 * 1024, "shared memory budget");
static_assert(kEWarps + kEpiWarps <= 24, "max-reduction slots");

struct WideArgs {
    const float* x;          // fp32 activations, or
    const int16_t* xq_in;    // already-quantised activations and
    const float* xs_in;      // their x_scale
    const uint16_t* cs;      // [rows_pad][nbp]
    const float* rs;         // [rows_pad]
    float* y;
    int64_t* row_acc;
    int64_t* unit_acc;       // [rows][T] tile sums
    unsigned long long* top1;
    int64_t index_base;
    XchgDev xg;
    int64_t rows;
    int cols, nbp, groups;
    int* err;
};

// ---------------------------------------------------------- registration --
// q' plane and combined scales (tmac_gguf.cpp:1022-1039); one thread per
// (row, 16 columns), then one per (row, scale slot).  Padding rows hold q = 0,
// padding scale slots cs = 0.
__global__ void q8_wide_pack_kernel(const uint8_t* __restrict__ raw, int64_t rows, int64_t cols, int64_t rows_pad,
                                    int nbp, const float* __restrict__ row_scale, uint8_t* __restrict__ qp,
                                    uint16_t* __restrict__ cs)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t chunks = cols / 16;
    if (i < rows_pad * chunks) {
        const int64_t r = i / chunks, c0 = (i % chunks) * 16;
        uint8_t b[16];
        for (int k = 0; k < 16; k++) {
            uint8_t v = 0x80;
            if (r < rows) {
                const int64_t idx = r * cols + c0 + k;
                v = raw[(idx / 32) * 34 + 2 + idx % 32] ^ 0x80;
            }
            b[k] = v;
        }
        uint4 u;
        memcpy(&u, b, 16);
        reinterpret_cast<uint4*>(qp + r * cols)[c0 / 16] = u;
    }
    const int64_t j = i - rows_pad * chunks;
    if (j >= 0 && j < rows_pad * nbp) {
        const int64_t r = j / nbp;
        const int blk = (int)(j % nbp);
        uint16_t v = 0;
        if (r < rows && (int64_t)blk * 32 < cols) {
            const uint8_t* b = raw + (r * cols + (int64_t)blk * 32) / 32 * 34;
            v = (uint16_t)q8_combined(f16_bits_to_f32(ld_u16_unaligned(b)), row_scale[r]);
        }
        cs[j] = v;
    }
}

__global__ void fill_f32_kernel(float* p, int64_t n, float v)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

// deq = (q * cs) >> 8 as byte planes for the tensor-core GEMM (prefill).
__global__ void q8_wide_planes_kernel(const uint8_t* __restrict__ qp, const uint16_t* __restrict__ cs, int nbp,
                                      int64_t rows, int64_t cols, int8_t* __restrict__ wh, uint8_t* __restrict__ wl)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * cols) return;
    const int64_t r = i / cols, c = i % cols;
    const int q = (int)(int8_t)(qp[i] ^ 0x80);
    const int deq = (q * (int)cs[r * nbp + c / 32]) >> 8;
    wh[i] = (int8_t)(deq >> 8);
    wl[i] = (uint8_t)(deq & 0xFF);
}

#ifdef TMAC_TRACE
// Diagnostic build only (-DTMAC_TRACE): clock64 stamps per CTA and k-block
// (0 producer issue, 1 e' start, 2 e' done, 3 MMA waits done, 4 MMAs issued)
// and per group (epilogue start, end).
__device__ long long g_wide_trace[160][64][5];
__device__ long long g_wide_gtrace[160][16][2];
#define WIDE_STAMP(k, i)                                                                  \
    do {                                                                                  \
        if (blockIdx.x < 160 && (k) < 64) g_wide_trace[blockIdx.x][(k)][(i)] = clock64(); \
    } while (0)
#define WIDE_GSTAMP(g, i)                                                                 \
    do {                                                                                  \
        if (blockIdx.x < 160 && (g) < 16) g_wide_gtrace[blockIdx.x][(g)][(i)] = clock64(); \
    } while (0)
#else
#define WIDE_STAMP(k, i) \
    do {                 \
    } while (0)
#define WIDE_GSTAMP(g, i) \
    do {                  \
    } while (0)
#endif

// -------------------------------------------------------------- the GEMV --
// e' of 16 biased quants of one block (combined-scale low byte cl): for each
// word, two 16-bit lanes of q'*cl + 128*(256 - cl) per IMAD, high bytes kept.
TMAC_DEV uint4 e_chunk(uint4 q, uint32_t cl)
{
    const uint32_t k2 = (128u * (256u - cl)) * 0x00010001u;
    uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t a = __byte_perm(v[i], 0u, 0x4240);  // q'0 | q'2 << 16
        const uint32_t b = __byte_perm(v[i], 0u, 0x4341);  // q'1 | q'3 << 16
        v[i] = __byte_perm(a * cl + k2, b * cl + k2, 0x7351);
    }
    return make_uint4(v[0], v[1], v[2], v[3]);
}

TMAC_DEV uint4 lds128(uint32_t addr)
{
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}
TMAC_DEV void sts128(uint32_t addr, uint4 v)
{
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Byte offset of logical 16-byte chunk c of row r in a 128-byte-swizzled tile.
TMAC_DEV uint32_t sw128(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// x_q = 16384*x2 + 128*x1 + x0 with x0, x1 in [0, 127] and x2 in [-2, 1].
TMAC_DEV int x_part(int v, int p) { return p == 0 ? (v & 127) : p == 1 ? ((v >> 7) & 127) : (v >> 14); }

__global__ void __launch_bounds__(kThreads, 1) q8_wide_kernel(const __grid_constant__ CUtensorMap tm_q, WideArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ unsigned long long top1_slots[kEpiWarps];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t sbase = smem_addr(smem);
    uint16_t* cs_s = reinterpret_cast<uint16_t*>(smem + kOffCs);
    float* rs_s = reinterpret_cast<float*>(smem + kOffRs);
    int16_t* xq_s = reinterpret_cast<int16_t*>(smem + kOffXq);
    int* sx_s = reinterpret_cast<int*>(smem + kOffSx);
    float* red = reinterpret_cast<float*>(smem + kOffRed);
    volatile int* abort_s = reinterpret_cast<volatile int*>(red + 25);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
    uint64_t* a_full = bars;                 // [kAStages] q' k-block landed
    // [kAStages] the MMAs of k-block gi (stage gi % kAStages, e' slot
    // gi % kEStages) are done (one commit from each issuing warp): the e'
    // warps wait on it kEStages k-blocks later
    uint64_t* a_empty = a_full + kAStages;
    uint64_t* e_full = a_empty + kAStages;   // [kEStages] e' written
    uint64_t* cs_full = e_full + kEStages;   // [2] a group's scales landed
    uint64_t* cs_empty = cs_full + 2;        // [2] e' warps and epilogue are done with them
    uint64_t* t_full = cs_empty + 2;         // [2] accumulator set complete
    uint64_t* t_empty = t_full + 2;          // [2] accumulator set drained
    uint64_t* b_ready = t_empty + 2;         // activation operand built
    uint64_t* drain = b_ready + 1;           // [2] per issuing warp
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffSlot);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = (a.cols + WK - 1) / WK;
    const int nblk = a.cols / 32;
    const int T = (a.cols + 63) / 64;

    pdl_launch();
    if (threadIdx.x == 0) {
        for (int i = 0; i < kAStages; i++) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 2);
        }
        for (int i = 0; i < kEStages; i++) mbar_init(&e_full[i], kEWarps);
        for (int i = 0; i < 2; i++) {
            mbar_init(&cs_full[i], 1);
            mbar_init(&cs_empty[i], kEWarps + kEpiWarps);
            mbar_init(&t_full[i], 2);
            mbar_init(&t_empty[i], kEpiWarps);
            mbar_init(&drain[i], 1);
        }
        mbar_init(b_ready, kEWarps + kEpiWarps);
        *abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------ producer (weights only:
        // they do not depend on the preceding kernel, so no pdl_wait)
        if (lane == 0) {
            const uint32_t cs_bytes = (uint32_t)(WM * a.nbp * 2);
            int64_t gi = 0;  // k-blocks issued
            int i = 0;       // groups issued
            for (int g = blockIdx.x; g < a.groups && !*abort_s; g += gridDim.x, i++) {
                const int gb = i & 1;
                if (i >= 2 && !mbar_wait_sleep(&cs_empty[gb], ((i >> 1) - 1) & 1, a.err)) {
                    *abort_s = 1;
                    break;
                }
                mbar_arrive_expect_tx(&cs_full[gb], cs_bytes + WM * 4);
                bulk_g2s(cs_s + gb * WM * kMaxBlk, a.cs + (int64_t)g * WM * a.nbp, cs_bytes, &cs_full[gb]);
                bulk_g2s(rs_s + gb * WM, a.rs + (int64_t)g * WM, WM * 4, &cs_full[gb]);
                for (int kb = 0; kb < KB; kb++, gi++) {
                    const int s = (int)(gi % kAStages);
                    if (gi >= kAStages && !mbar_wait_sleep(&a_empty[s], (int)((gi / kAStages - 1) & 1), a.err)) {
                        *abort_s = 1;
                        break;
                    }
                    WIDE_STAMP(gi, 0);
                    mbar_arrive_expect_tx(&a_full[s], kATile);
                    tma_load_2d(smem + kOffA + s * kATile, &tm_q, kb * WK, g * WM, &a_full[s]);
                }
                if (*abort_s) {
                    i++;
                    break;
                }
            }
            // Keep the CTA alive until every copy issued has landed (at once on
            // the normal path, where every stage was consumed).
            for (int64_t k = (gi > kAStages ? gi - kAStages : 0); k < gi; k++)
                mbar_wait_bounded(&a_full[k % kAStages], (int)((k / kAStages) & 1), a.err);
            for (int k = (i > 2 ? i - 2 : 0); k < i; k++) mbar_wait_bounded(&cs_full[k & 1], (k >> 1) & 1, a.err);
        }
    } else if (warp == 1 || warp == 2) {
        // ------------------------------------------ MMA issue: q' (warp 1), e' (warp 2)
        if (lane == 0) {
            const bool is_e = warp == 2;
            constexpr uint32_t kID = idesc_i8_mn(0, 1, WM, kBN);  // unsigned q' / e', signed x parts
            if (!mbar_wait_bounded(b_ready, 0, a.err)) *abort_s = 1;
            tc_fence_after();
            const uint64_t dA = desc_sw128(sbase + (is_e ? kOffE : kOffA));
            const uint64_t dB = desc_sw128(sbase + kOffB);
            const int nst = is_e ? kEStages : kAStages;
            uint64_t* ready = is_e ? e_full : a_full;
            int64_t gi = 0;
            int i = 0;
            for (int g = blockIdx.x; g < a.groups && !*abort_s; g += gridDim.x, i++) {
                const int b = i & 1;
                if (i >= 2 && !mbar_wait_bounded(&t_empty[b], ((i >> 1) - 1) & 1, a.err)) {
                    *abort_s = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)b * 256 + (is_e ? 128u : 0u);
                for (int kb = 0; kb < KB; kb++, gi++) {
                    const int s = (int)(gi % nst);
                    if (!mbar_wait_bounded(&ready[s], (int)((gi / nst) & 1), a.err)) {
                        *abort_s = 1;
                        break;
                    }
                    tc_fence_after();
                    if (is_e) WIDE_STAMP(gi, 3);
                    // descriptors advance in 16-byte units: 32 bytes of K = 2
                    const uint64_t ad = dA + (uint64_t)((s * kATile) >> 4);
                    const uint64_t bd = dB + (uint64_t)((kb * kBTile) >> 4);
                    mma_i8(d, ad, bd, kID, kb != 0);
                    mma_i8(d, ad + 2, bd + 2, kID, 1u);
                    mma_i8(d, ad + 4, bd + 4, kID, 1u);
                    mma_i8(d, ad + 6, bd + 6, kID, 1u);
                    if (is_e) WIDE_STAMP(gi, 4);
                    // the q' stage / e' slot is free once both warps' MMAs have read it
                    mma_commit(&a_empty[gi % kAStages]);
                }
                if (*abort_s) break;
                mma_commit(&t_full[b]);
            }
            mma_commit(&drain[warp - 1]);  // completes when every MMA issued above has
            mbar_wait_bounded(&drain[warp - 1], 0, a.err);
        }
    } else {
        // ------------------------- activations: x_q, block sums Sx, B operand
        const int pt = threadIdx.x - kWarpE0 * 32;  // 0 .. kPrologueThreads-1
        // zero the B tiles first: that does not depend on the preceding kernel
        for (int j = pt; j < (int)(kMaxKB * kBTile / 16); j += kPrologueThreads)
            sts128(sbase + kOffB + (uint32_t)j * 16, make_uint4(0, 0, 0, 0));
        pdl_wait();  // x comes from the preceding kernel
        const int ncols = KB * WK;
        if (a.xq_in) {
            for (int j = pt; j < ncols; j += kPrologueThreads) xq_s[j] = (j < a.cols) ? a.xq_in[j] : (int16_t)0;
            if (pt == 0) red[24] = *a.xs_in;
        } else {
            float mx = 0.0f;
            for (int j = pt; j < a.cols; j += kPrologueThreads) mx = fmaxf(mx, fabsf(a.x[j]));
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0) red[pt >> 5] = mx;
            named_bar_sync(1, kPrologueThreads);
            mx = 0.0f;
            for (int w = 0; w < kEWarps + kEpiWarps; w++) mx = fmaxf(mx, red[w]);
            const float xs = x_scale_from_max(mx);
            for (int j = pt; j < ncols; j += kPrologueThreads) xq_s[j] = (j < a.cols) ? quantize_one(a.x[j], xs) : 0;
            if (pt == 0) red[24] = xs;
        }
        named_bar_sync(1, kPrologueThreads);
        if (pt < kMaxBlk) {
            int sum = 0;
            if (pt < nblk)
                for (int k = 0; k < 32; k++) sum += xq_s[pt * 32 + k];
            sx_s[pt] = sum;
        }
        // B: rows n, 32 + n, 64 + n of k-block n / 4 hold x0, x1, x2 of block
        // n in its two 16-byte chunks; one thread per (block, part, chunk).
        if (pt >= kMaxBlk && pt < kMaxBlk + nblk * 6) {
            const int t = pt - kMaxBlk;
            const int n = t / 6, p = (t % 6) >> 1, c = t & 1;
            const int col0 = n * 32 + c * 16;
            uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
            for (int k = 0; k < 16; k++) w[k >> 2] |= (uint32_t)(x_part(xq_s[col0 + k], p) & 0xFF) << (8 * (k & 3));
            const uint32_t off = (uint32_t)(n >> 2) * kBTile + sw128(32 * p + n, 2 * (n & 3) + c);
            sts128(sbase + kOffB + off, make_uint4(w[0], w[1], w[2], w[3]));
        }
        fence_proxy_async_smem();
        named_bar_sync(1, kPrologueThreads);  // sx_s, red[24] visible to every worker
        __syncwarp();
        if (lane == 0) mbar_arrive(b_ready);

        if (warp < kWarpEpi0) {
            // --------------------------------------------------- e' of each k-block
            // thread -> row r of the group and block 4kb + h (logical chunks
            // 2h, 2h + 1) of every k-block
            const int et = threadIdx.x - kWarpE0 * 32;
            const int r = et & (WM - 1), h = et >> 7;
            int64_t gi = 0;
            int i = 0;
            for (int g = blockIdx.x; g < a.groups; g += gridDim.x, i++) {
                const int gb = i & 1;
                if (*abort_s || !mbar_wait_sleep(&cs_full[gb], (i >> 1) & 1, a.err)) {
                    *abort_s = 1;
                    break;
                }
                const uint16_t* csr = cs_s + gb * WM * kMaxBlk + r * a.nbp;
                for (int kb = 0; kb < KB; kb++, gi++) {
                    const int s = (int)(gi % kAStages), es = (int)(gi % kEStages);
                    if (*abort_s || !mbar_wait_sleep(&a_full[s], (int)((gi / kAStages) & 1), a.err) ||
                        (gi >= kEStages &&
                         !mbar_wait_sleep(&a_empty[(gi - kEStages) % kAStages],
                                          (int)(((gi - kEStages) / kAStages) & 1), a.err))) {
                        *abort_s = 1;
                        break;
                    }
                    if (et == 0) WIDE_STAMP(gi, 1);
                    const uint32_t cl = csr[kb * 4 + h] & 0xFFu;
                    const uint32_t at = sbase + kOffA + s * kATile, eo = sbase + kOffE + es * kATile;
                    const uint32_t o0 = sw128(r, 2 * h), o1 = sw128(r, 2 * h + 1);
                    const uint4 q0 = lds128(at + o0), q1 = lds128(at + o1);
                    sts128(eo + o0, e_chunk(q0, cl));
                    sts128(eo + o1, e_chunk(q1, cl));
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&e_full[es]);
                    if (et == 0) WIDE_STAMP(gi, 2);
                }
                if (*abort_s) break;
                __syncwarp();
                if (lane == 0) mbar_arrive(&cs_empty[gb]);
            }
        } else {
            // --------------------------------------------------------- epilogue
            // TMEM lanes 32*(warp%4) .. +31: one weight row per thread
            const int q = warp & 3;
            const int rr = q * 32 + lane;
            const double xsd = (double)red[24];
            unsigned long long best = 0;
            int i = 0;
            for (int g = blockIdx.x; g < a.groups; g += gridDim.x, i++) {
                const int b = i & 1, gb = i & 1;
                if (*abort_s || !mbar_wait_sleep(&t_full[b], (i >> 1) & 1, a.err) ||
                    !mbar_wait_bounded(&cs_full[gb], (i >> 1) & 1, a.err)) {
                    *abort_s = 1;
                    break;
                }
                tc_fence_after();
                if (rr == 0) WIDE_GSTAMP(i, 0);
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)b * 256;
                const uint16_t* csr = cs_s + gb * WM * kMaxBlk + rr * a.nbp;
                const int64_t row = (int64_t)g * WM + rr;
                const bool row_ok = row < a.rows;
                const double rs = (double)rs_s[gb * WM + rr];
                float yr = 0.0f;
                long long rsum = 0;
#pragma unroll 1
                for (int c8 = 0; c8 * 8 < nblk; c8++) {
                    uint32_t v[6][8];  // q' x0 | x1 | x2, e' x0 | x1 | x2 of blocks 8*c8 ..
#pragma unroll
                    for (int p = 0; p < 3; p++) {
                        tmem_ld8(taddr + 32 * p + c8 * 8, v[p]);
                        tmem_ld8(taddr + 128 + 32 * p + c8 * 8, v[3 + p]);
                    }
                    tmem_wait_ld();
                    long long acc_t = 0;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const int blk = c8 * 8 + j;
                        if (blk < nblk) {
                            const uint32_t cs = csr[blk];
                            const int sxb = 128 * sx_s[blk];
                            const int qx = (int)v[2][j] * 16384 + (int)v[1][j] * 128 + (int)v[0][j] - sxb;
                            const int ex = (int)v[5][j] * 16384 + (int)v[4][j] * 128 + (int)v[3][j] - sxb;
                            acc_t += (long long)(cs >> 8) * (long long)qx + (long long)ex;
                        }
                        // tile (blk >> 1) ends here: fold it in order
                        if ((j & 1) && blk - 1 < nblk) {
                            rsum += acc_t;
                            const double y1 = __dmul_rn(__dmul_rn((double)acc_t, xsd), rs);
                            yr = (float)__dadd_rn((double)yr, y1);
                            if (a.unit_acc && row_ok) a.unit_acc[row * T + (blk >> 1)] = acc_t;
                            acc_t = 0;
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&t_empty[b]);
                    mbar_arrive(&cs_empty[gb]);
                }
                if (rr == 0) WIDE_GSTAMP(i, 1);
                if (row_ok) {
                    a.y[row] = yr;
                    if (a.row_acc) a.row_acc[row] = rsum;
                    const unsigned long long k = top1_key(yr, a.index_base + row);
                    best = k > best ? k : best;
                }
            }
            if (a.top1) {
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
                    best = k > best ? k : best;
                }
                top1_cta_finish(a.xg, a.top1, best, top1_slots, warp - kWarpEpi0, warp == kWarpEpi0, 2, kEpiWarps * 32,
                                a.err);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

size_t wide_smem_bytes() { return kSmem; }

}  // namespace

bool q8_wide_eligible(int64_t rows, int64_t cols)
{
    // Opt-in (TMAC_Q8_WIDE=1 at registration): on B200 this kernel is bound by
    // shared-memory bandwidth and MMA issue (every weight byte crosses shared
    // memory five times: TMA write, e' read and write, q' and e' MMA reads) and
    // runs the 151936 x 896 logits in ~57 us against ~35 us for the CUDA-core
    // kernel of gemv_q8_0.cu, which therefore stays the default.
    const char* env = getenv("TMAC_Q8_WIDE");
    if (!env || env[0] != '1') return false;
    return rows >= kWideMinRows && cols >= WK && cols <= kMaxKB * WK && cols % 32 == 0;
}

int register_q8_wide(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s)
{
    const int64_t rows_pad = (w->rows + WM - 1) / WM * WM;
    const int nblk = (int)(w->cols / 32);
    w->q8_wide = 1;
    w->rows_pad = rows_pad;
    w->nbp = (nblk + 7) / 8 * 8;
    w->tiles = (int)((w->cols + 63) / 64);
    w->groups = rows_pad / WM;
    w->group_bytes = 0;
    const int64_t q_bytes = rows_pad * w->cols;
    w->cs_off = (q_bytes + 1023) / 1024 * 1024;
    w->data_bytes = (size_t)(w->cs_off + rows_pad * w->nbp * 2);
    TMAC_CUDA_TRY(cudaMalloc(&w->data, w->data_bytes));
    if (rows_pad > w->rows) {
        const int64_t n = rows_pad - w->rows;
        fill_f32_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(w->row_norm + w->rows, n, 1.0f);
        TMAC_CUDA_TRY(cudaGetLastError());
    }
    const int64_t work = rows_pad * (w->cols / 16) + rows_pad * w->nbp;
    q8_wide_pack_kernel<<<(unsigned)((work + 255) / 256), 256, 0, s>>>(
        d_raw, w->rows, w->cols, rows_pad, w->nbp, w->row_norm, w->data,
        reinterpret_cast<uint16_t*>(w->data + w->cs_off));
    TMAC_CUDA_TRY(cudaGetLastError());

    const auto encode = encode_fn();
    if (!encode) return fail(TMAC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    static_assert(sizeof(CUtensorMap) == sizeof(w->tmap), "tensor map storage");
    const cuuint64_t dims[2] = {(cuuint64_t)w->cols, (cuuint64_t)rows_pad};
    const cuuint64_t strides[1] = {(cuuint64_t)w->cols};
    const cuuint32_t box[2] = {WK, WM};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = encode(reinterpret_cast<CUtensorMap*>(w->tmap), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->data, dims,
                              strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TMAC_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return TMAC_OK;
}

int launch_q8_wide(const tmac_weight_s* w, const float* x, float* y, int64_t* row_acc, int64_t* unit_acc, int batch,
                   cudaStream_t s, unsigned long long* top1, int64_t index_base, const int16_t* xq, const float* xs,
                   const XchgDev* xg)
{
    if (xg && (batch != 1 || !top1)) return fail(TMAC_ERR_SHAPE, "the fused exchange takes batch 1 and a key");
    static bool attr_set[64] = {};
    if (!attr_set[w->device & 63]) {
        TMAC_CUDA_TRY(cudaFuncSetAttribute(q8_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)wide_smem_bytes()));
        attr_set[w->device & 63] = true;
    }
    const int grid = (int)std::min<int64_t>(w->groups, num_sms(w->device));
    const CUtensorMap* tm = reinterpret_cast<const CUtensorMap*>(w->tmap);
    for (int b = 0; b < batch; b++) {
        WideArgs a;
        a.x = x ? x + (int64_t)b * w->cols : nullptr;
        a.xq_in = xq ? xq + (int64_t)b * w->cols : nullptr;
        a.xs_in = xs ? xs + b : nullptr;
        a.cs = reinterpret_cast<const uint16_t*>(w->data + w->cs_off);
        a.rs = w->row_norm;
        a.y = y + (int64_t)b * w->rows;
        a.row_acc = row_acc ? row_acc + (int64_t)b * w->rows : nullptr;
        a.unit_acc = unit_acc ? unit_acc + (int64_t)b * w->rows * w->tiles : nullptr;
        a.top1 = top1 ? top1 + b : nullptr;
        a.index_base = index_base;
        if (xg) {
            a.xg = *xg;
        } else if (top1) {
            a.xg.partial = static_cast<unsigned long long*>(w->top1_scratch);
            a.xg.counter = reinterpret_cast<unsigned*>(a.xg.partial + 1);
        }
        a.rows = w->rows;
        a.cols = (int)w->cols;
        a.nbp = w->nbp;
        a.groups = (int)w->groups;
        a.err = device_error_word(w->device);
        TMAC_CUDA_TRY(launch_k(q8_wide_kernel, dim3(grid), dim3(kThreads), wide_smem_bytes(), s, *tm, a));
        TMAC_CUDA_TRY(cudaGetLastError());
    }
    return TMAC_OK;
}

#ifdef TMAC_TRACE
extern "C" int tmac_trace_read_wide(long long* out, long long* gout)
{
    cudaError_t e = cudaMemcpyFromSymbol(out, g_wide_trace, sizeof(g_wide_trace));
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(gout, g_wide_gtrace, sizeof(g_wide_gtrace));
    return (int)e;
}
#endif

int q8_wide_planes(const tmac_weight_s* w, int8_t* wh, uint8_t* wl, cudaStream_t s)
{
    const int64_t n = w->rows * w->cols;
    q8_wide_planes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        w->data, reinterpret_cast<const uint16_t*>(w->data + w->cs_off), w->nbp, w->rows, w->cols, wh, wl);
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

}  // namespace tmac
