// gemm_tc.cu -- the batched form of the NATIVE Q5_0 / Q4_K / Q6_K matmul on
// the 5th-generation tensor cores: Y[M][N] = the GEMV of every one of M
// activation rows, bit for bit (prefill; the reference has no batched path and
// runs matmul_fpga_* once per token, sim/tmac_gguf.cpp:1992-2023).
//
// Exact int16 x int16 with 8-bit MMAs.  Each weight is the reference's int16
// v (decoded once, gemv_blockq.cu planes_kernel) and each activation the int16
// x_q of its row (tmac_gguf.cpp:889-896); both are split into a signed high
// byte and an unsigned low byte, v = 256*vh + vl, x = 256*xh + xl, and
//   sum v*x = 65536 * sum vh*xh + 256 * (sum vh*xl + sum vl*xh) + sum vl*xl
// with four tcgen05.mma kind::i8 products accumulating in three int32 TMEM
// accumulators (each stays below 2^31 for K <= 32768).  The epilogue forms the
// int64 row sum and y = (float)((double)acc * x_scale / (double)row_inv)
// exactly as the GEMV does.
//
// Persistent kernel, one CTA per SM, tiles of 128 (rows of X) x 80 (weight
// rows) x 128 (K bytes); operands staged by TMA (128-byte swizzle, out-of-range
// rows and columns read as zero) through a 4-stage mbarrier ring.  Warp 0
// issues the copies, warp 1 owns TMEM and issues the MMAs into one of two
// accumulator sets, eight epilogue warps drain the other set.
#include "tcgen05.cuh"

#include <algorithm>
#include <mutex>
#include <vector>

namespace tmac {
namespace {

// Tile 128 (activation rows) x 80 (weight rows) x 128 (K bytes).  Three int32
// accumulators of 80 columns per tile, two tiles in flight: 480 TMEM columns.
constexpr int BM = 128, BN = 80, BK = 128, STAGES = 4;
constexpr uint32_t kTileX = BM * BK, kTileW = BN * BK;     // bytes of one plane tile
constexpr uint32_t kStageBytes = 2 * kTileX + 2 * kTileW;  // xh, xl, wh, wl
constexpr int kEpiWarps = 8;                               // 2 per TMEM lane quarter, 40 columns each
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr uint32_t kTmemCols = 512;                        // buffer b: hh | mid | ll at b*256 + {0, 80, 160}
constexpr int kEpiCols = BN / 2;
constexpr size_t kSmem = STAGES * kStageBytes + 1024 + 256;

struct GemmArgs {
    const float* xs;         // [M] x_scale of each activation row
    const float* row_param;  // [N] row_inv (mode 0) or row_scale (mode 1)
    const double* row_rinv;  // [N] RN(1 / row_inv) in double (mode 0)
    float* y;                // [M][y_stride]
    int64_t* acc_out;        // optional [M][N] int64 sums
    int64_t y_stride;
    int M, N, K;
    int tiles_m, tiles_n;
    int mode;                // 0: y = acc*xs/row_inv   1: y = (float)(y + acc*xs*row_scale)
    int* err;
};

// Instruction descriptor for kind::i8: s32 accumulate, A/B signed (1) or
// unsigned (0), both K-major, M = BM, N = BN.
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t a_signed, uint32_t b_signed)
{
    return (2u << 4) | (a_signed << 7) | (b_signed << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

// ----------------------------------------------------------------- kernel --
// Persistent: CTA c takes tiles c, c + grid, ...; tile i -> (m tile i / tiles_n,
// n tile i % tiles_n), so the tiles in flight share few activation tiles, which
// stay in L2 while every weight tile passes them.  Warp 0
// streams operands through the STAGES ring, warp 1 issues the MMAs into the
// accumulator buffer of the tile's parity, warps 2.. drain a finished buffer
// into registers, release it, then form y while the next tile accumulates.
__global__ void __launch_bounds__(kThreads, 1)
    gemm_i8x4_kernel(const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl,
                     const __grid_constant__ CUtensorMap tm_wh, const __grid_constant__ CUtensorMap tm_wl, GemmArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;   // [2] accumulator buffer ready
    uint64_t* tempty = tfull + 2;       // [2] accumulator buffer drained
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_s = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = (a.K + BK - 1) / BK;
    const int ntiles = a.tiles_m * a.tiles_n;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&tfull[i], 1);
            mbar_init(&tempty[i], kEpiWarps);
        }
        mbar_init(drain, 1);
        *abort_s = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // under programmatic launch only the set-up above overlaps the preceding kernel

    if (warp == 0) {
        if (lane == 0) {
            int64_t g = 0;  // k-blocks issued so far
            for (int tile = blockIdx.x; tile < ntiles && !*abort_s; tile += gridDim.x) {
                const int m0 = (tile / a.tiles_n) * BM, n0 = (tile % a.tiles_n) * BN;
                for (int kb = 0; kb < KB; kb++, g++) {
                    const int s = (int)(g % STAGES);
                    if (g >= STAGES && !mbar_wait_bounded(&empty[s], (int)((g / STAGES - 1) & 1), a.err)) {
                        *abort_s = 1;
                        break;
                    }
                    uint8_t* st = smem + s * kStageBytes;
                    mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tma_load_2d(st, &tm_xh, kb * BK, m0, &full[s]);
                    tma_load_2d(st + kTileX, &tm_xl, kb * BK, m0, &full[s]);
                    tma_load_2d(st + 2 * kTileX, &tm_wh, kb * BK, n0, &full[s]);
                    tma_load_2d(st + 2 * kTileX + kTileW, &tm_wl, kb * BK, n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t kHH = idesc_i8(1, 1), kHL = idesc_i8(1, 0), kLH = idesc_i8(0, 1), kLL = idesc_i8(0, 0);
            int64_t g = 0;
            int li = 0;
            for (int tile = blockIdx.x; tile < ntiles && !*abort_s; tile += gridDim.x, li++) {
                const int b = li & 1, use = li >> 1;
                if (use >= 1 && !mbar_wait_bounded(&tempty[b], (use - 1) & 1, a.err)) {
                    *abort_s = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t acc0 = tmem + (uint32_t)b * 256;
                for (int kb = 0; kb < KB; kb++, g++) {
                    const int s = (int)(g % STAGES);
                    if (*abort_s || !mbar_wait_bounded(&full[s], (int)((g / STAGES) & 1), a.err)) {
                        *abort_s = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_addr(smem + s * kStageBytes);
#pragma unroll
                    for (int kk = 0; kk < BK / 32; kk++) {  // 32 bytes of K per MMA
                        const uint64_t xh = desc_sw128(st + kk * 32), xl = desc_sw128(st + kTileX + kk * 32);
                        const uint64_t wh = desc_sw128(st + 2 * kTileX + kk * 32);
                        const uint64_t wl = desc_sw128(st + 2 * kTileX + kTileW + kk * 32);
                        const uint32_t acc = (kb | kk) != 0;
                        mma_i8(acc0, xh, wh, kHH, acc);
                        mma_i8(acc0 + BN, xh, wl, kHL, acc);
                        mma_i8(acc0 + BN, xl, wh, kLH, 1u);
                        mma_i8(acc0 + 2 * BN, xl, wl, kLL, acc);
                    }
                    mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
                }
                if (*abort_s) break;
                mma_commit(&tfull[b]);
            }
            mma_commit(drain);  // completes when every MMA issued above has
            mbar_wait_bounded(drain, 0, a.err);
        }
    } else {
        // epilogue warp: TMEM lanes 32*(warp%4) .. +31 (one activation row per
        // thread), columns [half*40, half*40 + 40) of the tile
        const int q = warp & 3, half = (warp - 2) >> 2;
        const int c0 = half * kEpiCols;
        int li = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, li++) {
            const int m0 = (tile / a.tiles_n) * BM, n0 = (tile % a.tiles_n) * BN;
            const int m = m0 + q * 32 + lane;
            const int b = li & 1, use = li >> 1;
            const double xsd = (m < a.M) ? (double)a.xs[m] : 0.0;
            const bool ok = !*abort_s && mbar_wait_bounded(&tfull[b], use & 1, a.err);
            if (!ok) {
                *abort_s = 1;
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)b * 256 + c0;
            float* yrow = a.y + (int64_t)m * a.y_stride + n0 + c0;
            const bool row_ok = m < a.M;
            // 8 columns at a time: three TMEM loads, then the 8 outputs
#pragma unroll 1
            for (int c = 0; c < kEpiCols; c += 8) {
                uint32_t hh[8], md[8], ll[8];
                tmem_ld8(taddr + c, hh);
                tmem_ld8(taddr + BN + c, md);
                tmem_ld8(taddr + 2 * BN + c, ll);
                double rinv[8];
                float rp[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int n = min(n0 + c0 + c + j, a.N - 1);
                    rp[j] = __ldg(a.row_param + n);
                    rinv[j] = (a.mode == 0) ? __ldg(a.row_rinv + n) : 0.0;
                }
                tmem_wait_ld();
                if (!row_ok) continue;
                const bool full8 = n0 + c0 + c + 8 <= a.N && ((reinterpret_cast<uintptr_t>(yrow + c) & 15) == 0);
                float out[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const long long acc = (long long)(int32_t)hh[j] * 65536 + (long long)(int32_t)md[j] * 256 +
                                          (long long)(int32_t)ll[j];
                    const double p = __dmul_rn((double)acc, xsd);
                    if (a.mode == 0) {
                        out[j] = quotient_f32(p, rinv[j], rp[j]);
                    } else {  // one 64-column tile of the Q8_0 fold (gemv_q8_0.cu)
                        const double v = __dmul_rn(p, (double)rp[j]);
                        const bool in = n0 + c0 + c + j < a.N;
                        out[j] = (float)__dadd_rn((double)(in ? yrow[c + j] : 0.0f), v);
                    }
                    if (a.acc_out && n0 + c0 + c + j < a.N) a.acc_out[(int64_t)m * a.N + n0 + c0 + c + j] = acc;
                }
                if (full8) {
                    *reinterpret_cast<float4*>(yrow + c) = make_float4(out[0], out[1], out[2], out[3]);
                    *reinterpret_cast<float4*>(yrow + c + 4) = make_float4(out[4], out[5], out[6], out[7]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (n0 + c0 + c + j < a.N) yrow[c + j] = out[j];
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);  // the buffer can take tile li + 2
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ------------------------------------------------- skinny batches, split K --
// M <= 64 activation rows (a batched GEMV): the weights are the 128-row MMA
// operand and the batch the N operand (16..64 columns), and K is split across
// CTAs so that ~one CTA per SM streams its share of the weight planes once.
// CTA (mt, ks) accumulates k-blocks [ks * kchunk, ...) of weight rows
// [128 mt, 128 mt + 128) in TMEM, adds its int64 partial sums into a zeroed
// workspace with atomics (integer sums: the order does not matter), and the
// last CTA of the row tile (counter) takes the totals -- atomicExch leaves the
// workspace zeroed for the next call -- and forms y as the GEMM epilogue does.
constexpr int SK_BM = 128, SK_STAGES = 4, SK_MAXNB = 64;
constexpr int kSkThreads = 6 * 32;  // warp 0 TMA, warp 1 MMA + TMEM, warps 2..5 epilogue (TMEM lane quarters 2,3,0,1)

struct SkArgs {
    const float* xs;           // [batch] x_scale
    const float* ri;           // [rows] row_inv
    const double* rinv;        // [rows] RN(1 / row_inv)
    float* y;                  // [batch][rows]
    int64_t* acc_out;          // optional [batch][rows]
    unsigned long long* ws;    // [batch][rows] zeroed int64 sums
    unsigned* cnt;             // [tiles_m] zeroed arrival counters
    int rows, batch, NB, KB, kchunk, ksplit;
    int* err;
};

#ifdef TMAC_TRACE
__device__ unsigned long long g_sk_trace[160][8];
__device__ unsigned long long g_q_trace[64][4];
#define SK_STAMP(i) do { if (blockIdx.x < 160) g_sk_trace[blockIdx.x][i] = global_timer_ns(); } while (0)
#else
#define SK_STAMP(i) do { } while (0)
#endif

__host__ __device__ constexpr uint32_t sk_stage_bytes(int NB) { return 2u * SK_BM * BK + 2u * (uint32_t)NB * BK; }
__host__ __device__ constexpr uint32_t sk_tmem_cols(int NB) { return 3 * NB <= 64 ? 64u : (3 * NB <= 128 ? 128u : 256u); }

__global__ void __launch_bounds__(kSkThreads, 1)
    gemv_tc_splitk_kernel(const __grid_constant__ CUtensorMap tm_wh, const __grid_constant__ CUtensorMap tm_wl,
                          const __grid_constant__ CUtensorMap tm_xh, const __grid_constant__ CUtensorMap tm_xl, SkArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t stage_bytes = sk_stage_bytes(a.NB), tile_w = SK_BM * BK, tile_x = (uint32_t)a.NB * BK;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + SK_STAGES * stage_bytes);
    uint64_t* empty = full + SK_STAGES;
    uint64_t* tfull = empty + SK_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
    volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 1);  // [0] abort, [1] last CTA of the tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mt = blockIdx.x / a.ksplit, ks = blockIdx.x % a.ksplit;
    const int kb0 = ks * a.kchunk, nkb = min(a.KB, kb0 + a.kchunk) - kb0;
    const uint32_t tcols = sk_tmem_cols(a.NB);

    if (threadIdx.x == 0) {
        SK_STAMP(0);
        for (int i = 0; i < SK_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        mbar_init(tfull, 1);
        flags[0] = 0;
        flags[1] = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch();  // the next kernel's writes of the x planes wait for this grid (its pdl_wait)

    if (warp == 0) {
        if (lane == 0) {
            // the weight planes of the first stages do not depend on the preceding
            // kernel: their copies start before the wait for the x planes
            const int pre = min(nkb, SK_STAGES);
            for (int i = 0; i < pre; i++) {
                uint8_t* st = smem + i * stage_bytes;
                const int kx = (kb0 + i) * BK;
                mbar_arrive_expect_tx(&full[i], stage_bytes);
                tma_load_2d(st, &tm_wh, kx, mt * SK_BM, &full[i]);
                tma_load_2d(st + tile_w, &tm_wl, kx, mt * SK_BM, &full[i]);
            }
            SK_STAMP(1);
            pdl_wait();  // x planes come from the preceding quantisation kernel
            SK_STAMP(2);
            for (int i = 0; i < nkb; i++) {
                const int s = i % SK_STAGES;
                uint8_t* st = smem + s * stage_bytes;
                const int kx = (kb0 + i) * BK;
                if (i >= pre) {
                    if (!mbar_wait_bounded(&empty[s], ((i / SK_STAGES) - 1) & 1, a.err)) {
                        flags[0] = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], stage_bytes);
                    tma_load_2d(st, &tm_wh, kx, mt * SK_BM, &full[s]);
                    tma_load_2d(st + tile_w, &tm_wl, kx, mt * SK_BM, &full[s]);
                }
                tma_load_2d(st + 2 * tile_w, &tm_xh, kx, 0, &full[s]);
                tma_load_2d(st + 2 * tile_w + tile_x, &tm_xl, kx, 0, &full[s]);
            }
        } else {
            pdl_wait();
        }
    } else if (warp == 1) {
        pdl_wait();
        if (lane == 0) {
            const uint32_t NB = (uint32_t)a.NB;
            const uint32_t kHH = idesc_i8_mn(1, 1, SK_BM, NB), kHL = idesc_i8_mn(1, 0, SK_BM, NB);
            const uint32_t kLH = idesc_i8_mn(0, 1, SK_BM, NB), kLL = idesc_i8_mn(0, 0, SK_BM, NB);
            for (int i = 0; i < nkb; i++) {
                const int s = i % SK_STAGES;
                if (flags[0] || !mbar_wait_bounded(&full[s], (i / SK_STAGES) & 1, a.err)) {
                    flags[0] = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_addr(smem + s * stage_bytes);
#pragma unroll
                for (int kk = 0; kk < BK / 32; kk++) {
                    const uint64_t wh = desc_sw128(st + kk * 32), wl = desc_sw128(st + tile_w + kk * 32);
                    const uint64_t xh = desc_sw128(st + 2 * tile_w + kk * 32);
                    const uint64_t xl = desc_sw128(st + 2 * tile_w + tile_x + kk * 32);
                    const uint32_t acc = (i | kk) != 0;
                    mma_i8(tmem, wh, xh, kHH, acc);
                    mma_i8(tmem + NB, wh, xl, kHL, acc);
                    mma_i8(tmem + NB, wl, xh, kLH, 1u);
                    mma_i8(tmem + 2 * NB, wl, xl, kLL, acc);
                }
                mma_commit(&empty[s]);
            }
            mma_commit(tfull);  // completes when every MMA issued above has
        }
    } else {
        pdl_wait();  // x_scale is read by the last CTA's epilogue
        // epilogue: TMEM lane = weight row of the tile, columns = batch entries
        const int q = warp & 3;
        const int row = mt * SK_BM + q * 32 + lane;
        bool ok = !flags[0] && mbar_wait_bounded(tfull, 0, a.err);
        ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below is warp-collective
        if (ok) {
            tc_fence_after();
            if (q == 0 && lane == 0) SK_STAMP(3);
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
            for (int c = 0; c < a.NB; c += 8) {
                uint32_t hh[8], md[8], ll[8];
                tmem_ld8(taddr + c, hh);
                tmem_ld8(taddr + a.NB + c, md);
                tmem_ld8(taddr + 2 * a.NB + c, ll);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int b = c + j;
                    if (b < a.batch && row < a.rows) {
                        const long long part = (long long)(int32_t)hh[j] * 65536 + (long long)(int32_t)md[j] * 256 +
                                               (long long)(int32_t)ll[j];
                        atomicAdd(a.ws + (int64_t)b * a.rows + row, (unsigned long long)part);
                    }
                }
            }
        } else {
            flags[0] = 1;
        }
        __threadfence();
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x == 0) {
        SK_STAMP(4);
        flags[1] = (atomicAdd(a.cnt + mt, 1u) == (unsigned)(a.ksplit - 1)) ? 1 : 0;
        SK_STAMP(5);
    }
    __syncthreads();
    if (flags[1]) {
        __threadfence();
        if (warp >= 2) {
            const int q = warp & 3;
            const int row = mt * SK_BM + q * 32 + lane;
            if (row < a.rows) {
                const double rinv = a.rinv[row];
                const float ri = a.ri[row];
                // every other CTA's atomics on these sums were performed before its
                // counter increment: plain L2 loads, issued 16 at a time, see the
                // totals; the stores of 0 leave the workspace clean for the next call
                for (int b0 = 0; b0 < a.batch; b0 += 16) {
                    long long acc[16];
#pragma unroll
                    for (int j = 0; j < 16; j++)
                        acc[j] = b0 + j < a.batch ? (long long)__ldcg(a.ws + (int64_t)(b0 + j) * a.rows + row) : 0;
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const int b = b0 + j;
                        if (b < a.batch) {
                            a.ws[(int64_t)b * a.rows + row] = 0ull;
                            const double p = __dmul_rn((double)acc[j], (double)a.xs[b]);
                            a.y[(int64_t)b * a.rows + row] = quotient_f32(p, rinv, ri);
                            if (a.acc_out) a.acc_out[(int64_t)b * a.rows + row] = acc[j];
                        }
                    }
                }
            }
        }
        if (threadIdx.x == 0) a.cnt[mt] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        SK_STAMP(6);
    }
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, tcols);
    }
}


// Activation rows -> x_scale and byte planes (one CTA per row, tmac_gguf.cpp:889-896).
#ifndef TMAC_QUANT_THREADS
#define TMAC_QUANT_THREADS 1024
#endif
constexpr int kQuantThreads = TMAC_QUANT_THREADS;
__global__ void __launch_bounds__(kQuantThreads) quantize_rows_kernel(const float* __restrict__ x, int64_t K,
                                                            int8_t* __restrict__ xh, uint8_t* __restrict__ xl,
                                                            float* __restrict__ xs)

{
    __shared__ float red[kQuantThreads / 32];
#ifdef TMAC_TRACE
    if (threadIdx.x == 0 && blockIdx.x < 64) g_q_trace[blockIdx.x][0] = global_timer_ns();
#endif
    pdl_launch();
    pdl_wait();
#ifdef TMAC_TRACE
    if (threadIdx.x == 0 && blockIdx.x < 64) g_q_trace[blockIdx.x][1] = global_timer_ns();
#endif
    const float* xr = x + (int64_t)blockIdx.x * K;
    float mx = 0.0f;
    for (int64_t j = threadIdx.x; j < K; j += blockDim.x) mx = fmaxf(mx, fabsf(xr[j]));
    mx = block_max(mx, red, blockDim.x);
    const float s = x_scale_from_max(mx);
    if (threadIdx.x == 0) xs[blockIdx.x] = s;
    for (int64_t j = threadIdx.x; j < K; j += blockDim.x) {
        const int16_t q = quantize_one(xr[j], s);
        xh[(int64_t)blockIdx.x * K + j] = (int8_t)(q >> 8);
        xl[(int64_t)blockIdx.x * K + j] = (uint8_t)(q & 0xFF);
    }
#ifdef TMAC_TRACE
    __syncthreads();
    if (threadIdx.x == 0 && blockIdx.x < 64) g_q_trace[blockIdx.x][2] = global_timer_ns();
#endif
}

// ------------------------------------------------------------------ host --
int encode_plane_map(CUtensorMap* tm, const void* base, int64_t rows, int64_t K, int64_t stride, uint32_t box_rows)
{
    const auto encode = encode_fn();
    if (!encode) return fail(TMAC_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {BK, box_rows};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                                              strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TMAC_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return TMAC_OK;
}

struct SkWorkspace {
    unsigned long long* acc = nullptr;  // zeroed between calls
    unsigned* cnt = nullptr;
    size_t acc_cap = 0, cnt_cap = 0;
};
std::vector<SkWorkspace> g_sk_ws;

struct GemmWorkspace {
    int8_t* xh = nullptr;
    uint8_t* xl = nullptr;
    float* xs = nullptr;
    size_t cap = 0, rows_cap = 0;
};
std::mutex g_gemm_mutex;
std::vector<GemmWorkspace> g_gemm_ws;

int gemm_workspace(int device, int64_t M, int64_t K, GemmWorkspace** out)
{
    std::lock_guard<std::mutex> lk(g_gemm_mutex);
    if ((int)g_gemm_ws.size() <= device) g_gemm_ws.resize(device + 1);
    GemmWorkspace& w = g_gemm_ws[device];
    const size_t need = (size_t)(M * K);
    if (w.cap < need) {
        if (w.xh) cudaFree(w.xh);
        if (w.xl) cudaFree(w.xl);
        w.xh = nullptr;
        w.xl = nullptr;
        w.cap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&w.xh, need));
        TMAC_CUDA_TRY(cudaMalloc(&w.xl, need));
        w.cap = need;
    }
    if (w.rows_cap < (size_t)M) {
        if (w.xs) cudaFree(w.xs);
        w.xs = nullptr;
        w.rows_cap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&w.xs, (size_t)M * sizeof(float)));
        w.rows_cap = (size_t)M;
    }
    *out = &w;
    return TMAC_OK;
}

int sk_workspace(int device, size_t nacc, size_t ncnt, SkWorkspace** out)
{
    // the caller holds g_gemm_mutex
    if ((int)g_sk_ws.size() <= device) g_sk_ws.resize(device + 1);
    SkWorkspace& w = g_sk_ws[device];
    if (w.acc_cap < nacc) {
        if (w.acc) cudaFree(w.acc);
        w.acc = nullptr;
        w.acc_cap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&w.acc, nacc * sizeof(unsigned long long)));
        TMAC_CUDA_TRY(cudaMemset(w.acc, 0, nacc * sizeof(unsigned long long)));
        w.acc_cap = nacc;
    }
    if (w.cnt_cap < ncnt) {
        if (w.cnt) cudaFree(w.cnt);
        w.cnt = nullptr;
        w.cnt_cap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&w.cnt, ncnt * sizeof(unsigned)));
        TMAC_CUDA_TRY(cudaMemset(w.cnt, 0, ncnt * sizeof(unsigned)));
        w.cnt_cap = ncnt;
    }
    *out = &w;
    return TMAC_OK;
}

}  // namespace

// Exact int16 planes of the weight, decoded on first use.
int gemm_prepare(tmac_weight_s* w, cudaStream_t s)
{
    if (w->gwh) return TMAC_OK;
    const size_t n = (size_t)(w->rows * w->cols);
    TMAC_CUDA_TRY(cudaMalloc(&w->gwh, n));
    TMAC_CUDA_TRY(cudaMalloc(&w->gwl, n));
    int rc = blockq_planes(w, reinterpret_cast<int8_t*>(w->gwh), reinterpret_cast<uint8_t*>(w->gwl), s);
    if (rc) return rc;
    if (!w->grinv) return fail(TMAC_ERR_INVALID, "gemm_prepare: weight has no row reciprocals");
    return TMAC_OK;
}

int quantize_rows(const float* x, int64_t K, int M, int8_t* xh, uint8_t* xl, float* xs, cudaStream_t s)
{
    TMAC_CUDA_TRY(launch_k(quantize_rows_kernel, dim3(M), dim3(kQuantThreads), 0, s, x, K, xh, xl, xs));
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int gemm_planes(const GemmOperands& op, cudaStream_t s)
{
    alignas(64) CUtensorMap tm[4];
    int rc;
    if ((rc = encode_plane_map(&tm[0], op.xh + op.k_off, op.M, op.K, op.x_stride, BM)) ||
        (rc = encode_plane_map(&tm[1], op.xl + op.k_off, op.M, op.K, op.x_stride, BM)) ||
        (rc = encode_plane_map(&tm[2], op.wh + op.k_off, op.N, op.K, op.w_stride, BN)) ||
        (rc = encode_plane_map(&tm[3], op.wl + op.k_off, op.N, op.K, op.w_stride, BN)))
        return rc;
    static bool attr[64] = {};
    if (!attr[op.device & 63]) {
        TMAC_CUDA_TRY(cudaFuncSetAttribute(gemm_i8x4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem));
        attr[op.device & 63] = true;
    }
    GemmArgs a;
    a.xs = op.xs;
    a.row_param = op.row_param;
    a.row_rinv = op.row_rinv;
    a.y = op.y;
    a.acc_out = op.acc_out;
    a.y_stride = op.y_stride;
    a.M = op.M;
    a.N = op.N;
    a.K = (int)op.K;
    a.mode = op.mode;
    a.tiles_m = (op.M + BM - 1) / BM;
    a.tiles_n = (op.N + BN - 1) / BN;
    a.err = device_error_word(op.device);
    const dim3 grid((unsigned)std::min<int64_t>((int64_t)a.tiles_m * a.tiles_n, num_sms(op.device)));
    TMAC_CUDA_TRY(launch_k(gemm_i8x4_kernel, grid, dim3(kThreads), kSmem, s, tm[0], tm[1], tm[2], tm[3], a));
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

// NATIVE Q8_0 (matmul_fpga_q8 per row, tmac_gguf.cpp:948-1085): the int16
// products deq = (q * cs) >> 8 as byte planes (decoded on first use, kept with
// the weight), one GEMM per 64-column tile folding y = (float)(y + acc * x_scale
// * row_scale) in tile order from y = 0, as the Q8_0 GEMV does.
int launch_gemm_q8(tmac_weight_s* w, const float* x, float* y, int M, cudaStream_t s)
{
    if (!w->gwh) {
        const size_t n = (size_t)(w->rows * w->cols);
        TMAC_CUDA_TRY(cudaMalloc(&w->gwh, n));
        TMAC_CUDA_TRY(cudaMalloc(&w->gwl, n));
        int rc = q8_planes(w, reinterpret_cast<int8_t*>(w->gwh), reinterpret_cast<uint8_t*>(w->gwl), s);
        if (rc) return rc;
    }
    GemmWorkspace* ws = nullptr;
    int rc;
    if ((rc = gemm_workspace(w->device, M, w->cols, &ws))) return rc;
    if ((rc = quantize_rows(x, w->cols, M, ws->xh, ws->xl, ws->xs, s))) return rc;
    TMAC_CUDA_TRY(cudaMemsetAsync(y, 0, (size_t)M * w->rows * sizeof(float), s));
    for (int64_t k0 = 0; k0 < w->cols; k0 += 64) {
        GemmOperands op;
        op.xh = reinterpret_cast<const uint8_t*>(ws->xh);
        op.xl = ws->xl;
        op.x_stride = w->cols;
        op.xs = ws->xs;
        op.M = M;
        op.wh = reinterpret_cast<const uint8_t*>(w->gwh);
        op.wl = reinterpret_cast<const uint8_t*>(w->gwl);
        op.w_stride = w->cols;
        op.N = (int)w->rows;
        op.K = std::min<int64_t>(64, w->cols - k0);
        op.k_off = k0;
        op.row_param = w->row_norm;
        op.mode = 1;
        op.y = y;
        op.y_stride = w->rows;
        op.device = w->device;
        if ((rc = gemm_planes(op, s))) return rc;
    }
    return TMAC_OK;
}

// M <= SK_MAXNB rows: gemv_tc_splitk_kernel over the quantised rows in ws.
int launch_gemm_skinny(tmac_weight_s* w, GemmWorkspace* ws, float* y, int64_t* acc_out, int M, cudaStream_t s)
{
    const int NB = (M + 15) / 16 * 16;
    const int tiles_m = (int)((w->rows + SK_BM - 1) / SK_BM);
    const int KB = (int)((w->cols + BK - 1) / BK);
#ifndef TMAC_SK_DIV
#define TMAC_SK_DIV 1
#endif
    const int target = std::max(1, num_sms(w->device) / tiles_m / TMAC_SK_DIV);
    const int kchunk = (KB + target - 1) / target;
    const int ksplit = (KB + kchunk - 1) / kchunk;
    SkWorkspace* sk = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_gemm_mutex);
        int rc = sk_workspace(w->device, (size_t)M * (size_t)w->rows, (size_t)tiles_m, &sk);
        if (rc) return rc;
    }
    alignas(64) CUtensorMap tm[4];
    int rc;
    const uint8_t* wh = reinterpret_cast<const uint8_t*>(w->gwh);
    const uint8_t* wl = reinterpret_cast<const uint8_t*>(w->gwl);
    if ((rc = encode_plane_map(&tm[0], wh, w->rows, w->cols, w->cols, SK_BM)) ||
        (rc = encode_plane_map(&tm[1], wl, w->rows, w->cols, w->cols, SK_BM)) ||
        (rc = encode_plane_map(&tm[2], reinterpret_cast<const uint8_t*>(ws->xh), M, w->cols, w->cols, (uint32_t)NB)) ||
        (rc = encode_plane_map(&tm[3], ws->xl, M, w->cols, w->cols, (uint32_t)NB)))
        return rc;
    const size_t smem = SK_STAGES * (size_t)sk_stage_bytes(NB) + 1024 + 256;
    static bool attr[64] = {};
    if (!attr[w->device & 63]) {
        TMAC_CUDA_TRY(cudaFuncSetAttribute(gemv_tc_splitk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(SK_STAGES * (size_t)sk_stage_bytes(SK_MAXNB) + 1024 + 256)));
        attr[w->device & 63] = true;
    }
    SkArgs a;
    a.xs = ws->xs;
    a.ri = w->row_norm;
    a.rinv = reinterpret_cast<const double*>(w->grinv);
    a.y = y;
    a.acc_out = acc_out;
    a.ws = sk->acc;
    a.cnt = sk->cnt;
    a.rows = (int)w->rows;
    a.batch = M;
    a.NB = NB;
    a.KB = KB;
    a.kchunk = kchunk;
    a.ksplit = ksplit;
    a.err = device_error_word(w->device);
    TMAC_CUDA_TRY(launch_k(gemv_tc_splitk_kernel, dim3((unsigned)(tiles_m * ksplit)), dim3(kSkThreads), smem, s,
                           tm[0], tm[1], tm[2], tm[3], a));
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int launch_gemm(tmac_weight_s* w, const float* x, float* y, int64_t* acc_out, int M, cudaStream_t s)
{
    if (w->type == TMAC_TYPE_Q8_0) return launch_gemm_q8(w, x, y, M, s);
    int rc = gemm_prepare(w, s);
    if (rc) return rc;
    GemmWorkspace* ws = nullptr;
    if ((rc = gemm_workspace(w->device, M, w->cols, &ws))) return rc;
    if ((rc = quantize_rows(x, w->cols, M, ws->xh, ws->xl, ws->xs, s))) return rc;
    if (M <= SK_MAXNB) return launch_gemm_skinny(w, ws, y, acc_out, M, s);
    GemmOperands op;
    op.xh = reinterpret_cast<const uint8_t*>(ws->xh);
    op.xl = ws->xl;
    op.x_stride = w->cols;
    op.xs = ws->xs;
    op.M = M;
    op.wh = reinterpret_cast<const uint8_t*>(w->gwh);
    op.wl = reinterpret_cast<const uint8_t*>(w->gwl);
    op.w_stride = w->cols;
    op.N = (int)w->rows;
    op.K = w->cols;
    op.k_off = 0;
    op.row_param = w->row_norm;
    op.row_rinv = reinterpret_cast<const double*>(w->grinv);
    op.mode = 0;
    op.y = y;
    op.y_stride = w->rows;
    op.acc_out = acc_out;
    op.device = w->device;
    return gemm_planes(op, s);
}

}  // namespace tmac

using namespace tmac;

#ifdef TMAC_TRACE
extern "C" int tmac_trace_read_sk(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, tmac::g_sk_trace, sizeof(tmac::g_sk_trace));
}
extern "C" int tmac_trace_read_q(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, tmac::g_q_trace, sizeof(tmac::g_q_trace));
}
#endif

extern "C" int tmac_gemm(tmac_weight_t w, const float* x, float* y, int64_t* row_acc, int m, void* stream)
{
    if (!w) return fail(TMAC_ERR_INVALID, "NULL weight handle");
    if (!x || !y) return fail(TMAC_ERR_INVALID, "NULL x or y");
    if (m <= 0) return fail(TMAC_ERR_SHAPE, "m must be positive");
    if (w->mode != TMAC_MODE_NATIVE)
        return fail(TMAC_ERR_TYPE, "tmac_gemm: NATIVE Q5_0 / Q8_0 / Q4_K / Q6_K weights only");
    if (w->type == TMAC_TYPE_Q8_0 && row_acc)
        return fail(TMAC_ERR_TYPE, "tmac_gemm: no integer row sums for Q8_0 (its rows fold 64-column tiles in fp64)");
    if (w->cols % 16 || w->cols > 32768) return fail(TMAC_ERR_SHAPE, "tmac_gemm: cols must be a multiple of 16, <= 32768");
    DeviceGuard dg(w->device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    return launch_gemm(w, x, y, row_acc, m, (cudaStream_t)stream);
}
