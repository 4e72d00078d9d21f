// gemv_q8_0.cu -- Q8_0 GEMV, bit-exact with the reference's Q8_0 FPGA path:
// matmul_fpga_q8 (sim/tmac_gguf.cpp:948-1085) driving axi_vecmul_tile_q8 and
// MatmulAccel::compute_int16's Q8 branch (sim/fpga_sim.hpp:322-349, :466-491).
//
// Reference numerics, per row r and 64-column tile t:
//   row_scale  = max_j |q*d| / 32767            (or row_max_abs[r] / 32767)
//   cs(blk)    = (u16)(min(max(d_blk * (1/row_scale), 0), 255.996) * 256 + 0.5)
//   deq        = (int16)((q * cs) >> 8)          (arithmetic shift = floor)
//   acc_t      = sum_k deq * x_q[k]              (int64, 64 columns)
//   y          = (float)((double)y + (double)acc_t * x_scale * row_scale), t = 0..T-1 in order
//
// Device layout (built once by register_q8_0): rows in groups of 32, each group
// one contiguous record so a single 1-D bulk copy stages it in shared memory:
//   [T][4][32 lanes][16 B]  biased quants q ^ 0x80 (16 columns per chunk)
//   [T][32 lanes] u32       cs of the tile's two 32-column blocks (lo | hi << 16)
//   [32] f32                row_scale
// = 952 B per row for cols = 896, the same as the GGUF blocks (34 B / 32 values)
// plus the 4-byte row scale.  Padding rows/columns hold q = 0, cs = 0.
//
// Exact integer identity used by the kernel (no per-element float work):
//   cs = 256*ch + cl  =>  floor(q*cs/256) = q*ch + floor(q*cl/256)
//   with q' = q + 128 in [0,255]:  e + 128 = (q'*cl + 128*(256-cl)) >> 8 in [0,254]
// Two 16-bit lanes of (q'*cl + K) fit one 32-bit IMAD without carries
// (max 65153), so e is produced for 4 columns with 2 IMADs + 3 byte permutes,
// and every dot product is a dp4a against the split activation
// x_q = 256*xh + xl (xh signed byte, xl unsigned byte):
//   sum deq*x = ch*(sum q'*x - 128*Sx) + (sum eb*x - 128*Sx),  Sx = sum of x_q over the block.
#include "q8_dev.cuh"
#include "xchg.cuh"

#include <algorithm>

namespace tmac {
namespace {

// Warp roles: kConsumerWarps compute tile sums (warp w owns tiles t = w mod 14,
// so for cols <= 896 each warp owns one tile and keeps its activations in
// registers), one warp streams row groups into shared memory with bulk copies,
// and kFoldWarps warps fold the tile sums of each group into y in tile order.
constexpr int kConsumerWarps = 14;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kFoldWarp0 = kConsumerWarps + 1;
constexpr int kFoldWarps = 3;  // fold warp f takes groups i = f mod 3
constexpr int kThreads = (kConsumerWarps + 1 + kFoldWarps) * 32;
// Five stages with two groups per consumer iteration measured fastest on the
// 151936 x 896 logits matrix (31.3 us; 4 stages 32.3 us, 6 stages 32.1 us,
// one group per iteration 31.7 us, three 31.6 us, four 37.5 us).
constexpr int kMaxStages = 5;
constexpr int kGroupsPerIter = 2;  // row groups a consumer warp takes per iteration
static_assert(kGroupsPerIter <= 2, "a consumer iteration must never wait on more stages than the minimum ring (2)");
// Tile-sum buffers: group i uses buffer i mod kAccBufs; kAccBufs is a multiple of
// kFoldWarps so each buffer is folded by one warp only, in its own program order.
constexpr int kAccBufs = 2 * kFoldWarps;
constexpr size_t kSmemLimit = 220 * 1024;
// The small scratch at the end of shared memory holds one float per consumer
// warp (max reduction) in [0,16), x_scale at [16] and the abort flag at [20].
static_assert(kConsumerWarps <= 16, "max-reduction slots overlap x_scale / abort flag");

Q8Layout q8_layout(int64_t rows, int64_t cols)
{
    Q8Layout L;
    L.T = (int)((cols + 63) / 64);
    L.groups = (rows + 31) / 32;
    L.group_bytes = (int64_t)L.T * 2176 + 128;
    // Everything but the stages: barriers, tile sums, split activations, scratch.
    const int64_t extra = (2 * kMaxStages + 2 * kAccBufs) * 8 + kAccBufs * ((int64_t)L.T * 32 * 8 + 128) +
                          (int64_t)L.T * 16 * 4 * 2 + (int64_t)L.T * 2 * 4 + (int64_t)L.T * 64 * 2 + 32 * 4;
    const int64_t fit = ((int64_t)kSmemLimit - extra) / L.group_bytes;
    L.stages = (int)std::min<int64_t>(kMaxStages, std::max<int64_t>(fit, 0));
    return L;
}

// ---------------------------------------------------------- registration --
// row_scale per row (tmac_gguf.cpp:980-1004): one warp per row.
__global__ void q8_row_scale_kernel(const uint8_t* __restrict__ raw, int64_t rows, int64_t cols,
                                    const float* __restrict__ row_max_abs, float* __restrict__ row_scale)
{
    int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float mx;
    if (row_max_abs) {
        mx = row_max_abs[r];
    } else {
        mx = 0.0f;
        const int64_t bpr = cols / 32;
        for (int64_t b = lane; b < bpr; b += 32) {
            const uint8_t* blk = raw + (r * bpr + b) * 34;
            float d = f16_bits_to_f32(ld_u16_unaligned(blk));
            for (int k = 0; k < 32; k++) mx = fmaxf(mx, fabsf(__fmul_rn((float)(int8_t)blk[2 + k], d)));
        }
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if (lane == 0) row_scale[r] = (mx < 1e-10f) ? 1.0f : __fdiv_rn(mx, 32767.0f);
}

// One CTA per (group, tile): 128 threads write the 16-byte quant chunks,
// 32 threads the combined scales; tile 0 also writes the row scales.
__global__ void q8_pack_kernel(const uint8_t* __restrict__ raw, int64_t rows, int64_t cols,
                               const float* __restrict__ row_scale, Q8Layout L, uint8_t* __restrict__ out)
{
    const int64_t g = blockIdx.y;
    const int t = blockIdx.x;
    uint8_t* rec = out + g * L.group_bytes;
    const int tid = threadIdx.x;
    if (tid < 128) {
        int j = tid / 32, l = tid % 32;
        int64_t r = g * 32 + l;
        uint8_t buf[16];
        for (int b = 0; b < 16; b++) {
            int64_t c = (int64_t)t * 64 + j * 16 + b;
            uint8_t v = 0x80;
            if (r < rows && c < cols) {
                int64_t idx = r * cols + c;
                v = raw[(idx / 32) * 34 + 2 + idx % 32] ^ 0x80;
            }
            buf[b] = v;
        }
        uint4 u;
        memcpy(&u, buf, 16);
        reinterpret_cast<uint4*>(rec)[((int64_t)t * 4 + j) * 32 + l] = u;
    } else if (tid < 160) {
        int l = tid - 128;
        int64_t r = g * 32 + l;
        uint32_t cs2 = 0;
        if (r < rows) {
            float rs = row_scale[r];
            for (int blk = 0; blk < 2; blk++) {
                int64_t c0 = (int64_t)t * 64 + blk * 32;
                if (c0 >= cols) continue;
                const uint8_t* b = raw + ((r * cols + c0) / 32) * 34;
                cs2 |= q8_combined(f16_bits_to_f32(ld_u16_unaligned(b)), rs) << (16 * blk);
            }
        }
        reinterpret_cast<uint32_t*>(rec + L.cs_off())[t * 32 + l] = cs2;
    } else if (tid < 192 && t == 0) {
        int l = tid - 160;
        int64_t r = g * 32 + l;
        reinterpret_cast<float*>(rec + L.rs_off())[l] = (r < rows) ? row_scale[r] : 1.0f;
    }
}

// deq = (q * cs) >> 8 of every weight (the int16 the reference multiplies,
// fpga_sim.hpp:322-349) as byte planes for the tensor-core GEMM; one thread
// per (row, 16-column chunk) of the packed layout.
__global__ void q8_planes_kernel(const uint8_t* __restrict__ packed, Q8Layout L, int64_t rows, int64_t cols,
                                 int8_t* __restrict__ wh, uint8_t* __restrict__ wl)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // (row, chunk of 16 columns)
    const int64_t chunks = cols / 16;
    if (i >= rows * chunks) return;
    const int64_t r = i / chunks, c0 = (i % chunks) * 16;
    const int64_t g = r / 32;
    const int l = (int)(r % 32), t = (int)(c0 / 64), j = (int)((c0 % 64) / 16);
    const uint8_t* rec = packed + g * L.group_bytes;
    const uint4 qv = reinterpret_cast<const uint4*>(rec)[((int64_t)t * 4 + j) * 32 + l];
    const uint32_t cs2 = reinterpret_cast<const uint32_t*>(rec + L.cs_off())[t * 32 + l];
    const int cs = (int)((cs2 >> (16 * (j >> 1))) & 0xFFFFu);
    const uint8_t* qb = reinterpret_cast<const uint8_t*>(&qv);
    for (int b = 0; b < 16; b++) {
        const int q = (int)(int8_t)(qb[b] ^ 0x80);
        const int deq = (q * cs) >> 8;
        wh[r * cols + c0 + b] = (int8_t)(deq >> 8);
        wl[r * cols + c0 + b] = (uint8_t)(deq & 0xFF);
    }
}

// -------------------------------------------------------------- the GEMV --
struct Q8Args {
    const uint8_t* packed;
    Q8Layout L;
    int64_t rows;
    int cols;
    const float* x;          // fp32 activations, or
    const int16_t* xq_in;    // already-quantised activations and
    const float* xs_in;      // their x_scale (tmac_quantize_x)
    float* y;
    int64_t* row_acc;
    int64_t* unit_acc;
    unsigned long long* top1;  // optional: max packed (value, index) key, see top1_key
    int64_t index_base;        // global row index of row 0 (vocab shard offset)
    XchgDev xg;                // peers != nullptr: merge top1 across ranks (fused exchange)
    int* err;
};

template <bool kPeers>
__global__ void __launch_bounds__(kThreads, 1) q8_gemv_kernel(Q8Args a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long top1_slots[kFoldWarps];
    const Q8Layout L = a.L;
    const int T = L.T;
    uint8_t* stage_base = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.stages * L.group_bytes);  // stage landed
    uint64_t* empty = full + L.stages;                                             // stage consumed
    uint64_t* acc_full = empty + L.stages;                                         // tile sums ready
    uint64_t* acc_empty = acc_full + kAccBufs;                                     // tile sums folded
    long long* accs = reinterpret_cast<long long*>(acc_empty + kAccBufs);           // [kAccBufs][T][32]
    float* rs_buf = reinterpret_cast<float*>(accs + kAccBufs * T * 32);            // [kAccBufs][32]
    uint32_t* xh_s = reinterpret_cast<uint32_t*>(rs_buf + kAccBufs * 32);          // [T*16]
    uint32_t* xl_s = xh_s + T * 16;                                                // [T*16]
    int* sx_s = reinterpret_cast<int*>(xl_s + T * 16);                             // [T*2]
    int16_t* xq_s = reinterpret_cast<int16_t*>(sx_s + T * 2);                      // [T*64]
    float* red = reinterpret_cast<float*>(xq_s + T * 64);                          // [16] + xs + abort
    volatile int* abort_flag = reinterpret_cast<volatile int*>(red + 20);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_launch();
    // CTA c takes groups c, c + grid, c + 2 grid, ...: at any time the SMs
    // stream one contiguous window of the weights.
    const int ng = (int)((L.groups - blockIdx.x + gridDim.x - 1) / gridDim.x);
    auto group_of = [&](int i) -> int64_t { return (int64_t)blockIdx.x + (int64_t)i * gridDim.x; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < L.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        for (int b = 0; b < kAccBufs; b++) {
            mbar_init(&acc_full[b], kConsumerWarps);
            mbar_init(&acc_empty[b], 1);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        // ---------------- producer: one lane streams this CTA's groups ----
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < ng; i++) {
                const int s = i % L.stages;
                if (i >= L.stages && !mbar_wait_sleep(&empty[s], ((i / L.stages) & 1) ^ 1, a.err)) {
                    *abort_flag = 1;
                    break;
                }
                mbar_arrive_expect_tx(&full[s], (uint32_t)L.group_bytes);
                bulk_g2s(stage_base + (int64_t)s * L.group_bytes, a.packed + group_of(i) * L.group_bytes,
                         (uint32_t)L.group_bytes, &full[s]);
                issued = i + 1;
            }
            // Keep the CTA (and its shared memory) alive until every bulk copy
            // issued has landed; on the normal path these waits return at once.
            for (int i = (issued > L.stages ? issued - L.stages : 0); i < issued; i++)
                mbar_wait_bounded(&full[i % L.stages], (i / L.stages) & 1, a.err);
        }
        return;
    }

    if (warp >= kFoldWarp0) {
        const int f = warp - kFoldWarp0;
        // ---------------- fold: y = sum over tiles in order (tmac_gguf.cpp:1075-1076)
        unsigned long long best = 0;  // running top-1 key of this warp's rows
        for (int i = f; i < ng; i += kFoldWarps) {
            const int b = i % kAccBufs;
            if (*abort_flag || !mbar_wait_sleep(&acc_full[b], (i / kAccBufs) & 1, a.err)) {
                *abort_flag = 1;
                break;
            }
            const float xs = red[16];
            const long long* acc_buf = accs + b * T * 32;
            const double rs = (double)rs_buf[b * 32 + lane];
            const int64_t r = group_of(i) * 32 + lane;
            float yr = 0.0f;
            long long rsum = 0;
            for (int t = 0; t < T; t++) {
                const long long acc = acc_buf[t * 32 + lane];
                rsum += acc;
                const double v = __dmul_rn(__dmul_rn((double)acc, (double)xs), rs);
                yr = (float)__dadd_rn((double)yr, v);
                if (a.unit_acc && r < a.rows) a.unit_acc[r * T + t] = acc;
            }
            if (r < a.rows) {
                a.y[r] = yr;
                if (a.xg.vocab) {  // this row of the full logits in every rank (NVLink peer stores)
                    const uint64_t step = *a.xg.step + 1;
                    for (int q = 0; q < a.xg.world; q++) xchg_logits(a.xg, q, step)[a.index_base + r] = yr;
                }
                if (a.row_acc) a.row_acc[r] = rsum;
                const unsigned long long k = top1_key(yr, a.index_base + r);
                best = k > best ? k : best;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
        if (a.top1) {
            for (int o = 16; o > 0; o >>= 1) {
                const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
                best = k > best ? k : best;
            }
            if constexpr (kPeers)
                top1_cta_finish_peers(a.xg, a.top1, best, top1_slots, f, f == 0, 2, kFoldWarps * 32, a.err);
            else
                top1_cta_finish(a.xg, a.top1, best, top1_slots, f, f == 0, 2, kFoldWarps * 32, a.err);
        }
        return;
    }

    // ---------------- consumers: activation quantisation (overlaps the copies)
    const int nct = kConsumerWarps * 32;
    pdl_wait();  // x comes from the preceding kernel; the weights stream already
    float xs;
    if (a.xq_in) {
        for (int j = threadIdx.x; j < T * 64; j += nct) xq_s[j] = (j < a.cols) ? a.xq_in[j] : (int16_t)0;
        xs = *a.xs_in;
        if (threadIdx.x == 0) red[16] = xs;
    } else {
        // x is read from global memory once; xq_s first holds nothing, the values
        // stay in registers between the max reduction and the quantisation.
        constexpr int kXRegs = 4;  // covers T*64 <= kXRegs * 448 (cols <= 1792)
        float xv[kXRegs];
        float mx = 0.0f;
    #pragma unroll
        for (int k = 0; k < kXRegs; k++) {
            const int j = threadIdx.x + k * nct;
            xv[k] = (j < a.cols) ? a.x[j] : 0.0f;
            mx = fmaxf(mx, fabsf(xv[k]));
        }
        for (int j = threadIdx.x + kXRegs * nct; j < a.cols; j += nct) mx = fmaxf(mx, fabsf(a.x[j]));
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) red[warp] = mx;
        named_bar_sync(1, nct);
        mx = 0.0f;
        for (int i = 0; i < kConsumerWarps; i++) mx = fmaxf(mx, red[i]);
        xs = x_scale_from_max(mx);
        if (threadIdx.x == 0) red[16] = xs;
    #pragma unroll
        for (int k = 0; k < kXRegs; k++) {
            const int j = threadIdx.x + k * nct;
            if (j < T * 64) xq_s[j] = (j < a.cols) ? quantize_one(xv[k], xs) : 0;
        }
        for (int j = threadIdx.x + kXRegs * nct; j < T * 64; j += nct)
            xq_s[j] = (j < a.cols) ? quantize_one(a.x[j], xs) : 0;
    }
    named_bar_sync(1, nct);
    for (int j = threadIdx.x; j < T * 16; j += nct) {
        uint32_t h = 0, l = 0;
        for (int b = 0; b < 4; b++) {
            int v = xq_s[j * 4 + b];
            h |= (uint32_t)((v >> 8) & 0xFF) << (8 * b);
            l |= (uint32_t)(v & 0xFF) << (8 * b);
        }
        xh_s[j] = h;
        xl_s[j] = l;
    }
    // block sums of x_q: one warp per 32-column block, a shuffle reduction
    for (int j = warp; j < T * 2; j += kConsumerWarps) {
        int sum = xq_s[j * 32 + lane];
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) sx_s[j] = sum;
    }
    named_bar_sync(1, nct);

    // A warp that owns a single tile keeps its activations in registers.
    const bool one_tile = (T <= kConsumerWarps);
    uint4 xh[4], xl[4];
    int2 sx = make_int2(0, 0);
    if (one_tile && warp < T) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            xh[j] = reinterpret_cast<const uint4*>(xh_s + warp * 16)[j];
            xl[j] = reinterpret_cast<const uint4*>(xl_s + warp * 16)[j];
        }
        sx = reinterpret_cast<const int2*>(sx_s)[warp];
    }

    // ---------------- main loop over this CTA's 32-row groups -------------
    // kGroupsPerIter groups per iteration: their tile sums are independent,
    // which multiplies the work in flight per warp and divides the per-group
    // loop and barrier cost.
    // Ring positions advance by one per group: stage index and phase bit of the
    // weight ring and of the tile-sum buffers (no division by the runtime stage
    // count in the loop).
    int ring_s = 0, ring_b = 0;
    uint32_t ph_s = 0, ph_b = 0;
    for (int i = 0; i < ng; i += kGroupsPerIter) {
        const int cnt = min(kGroupsPerIter, ng - i);
        int sg[kGroupsPerIter], bg[kGroupsPerIter];
        bool ok = !*abort_flag;
#pragma unroll
        for (int g = 0; g < kGroupsPerIter; g++) {
            sg[g] = ring_s;
            bg[g] = ring_b;
            if (g < cnt && ok)
                ok = mbar_wait_sleep(&full[ring_s], ph_s, a.err) &&
                     (i + g < kAccBufs || mbar_wait_sleep(&acc_empty[ring_b], ph_b ^ 1, a.err));
            if (++ring_s == L.stages) { ring_s = 0; ph_s ^= 1; }
            if (++ring_b == kAccBufs) { ring_b = 0; ph_b ^= 1; }
        }
        if (!ok) {
            *abort_flag = 1;
            break;
        }
        const uint8_t* st[kGroupsPerIter];
        long long* acc[kGroupsPerIter];
#pragma unroll
        for (int g = 0; g < kGroupsPerIter; g++) {
            st[g] = stage_base + (int64_t)sg[g] * L.group_bytes;
            acc[g] = accs + bg[g] * T * 32;
        }
        if (warp == 0) {
#pragma unroll
            for (int g = 0; g < kGroupsPerIter; g++)
                if (g < cnt) rs_buf[bg[g] * 32 + lane] = reinterpret_cast<const float*>(st[g] + L.rs_off())[lane];
        }
        if (one_tile) {
            if (warp < T) {
                if (cnt == kGroupsPerIter) {
                    long long v[kGroupsPerIter];
#pragma unroll
                    for (int g = 0; g < kGroupsPerIter; g++) v[g] = q8_tile_dot(st[g], L, warp, lane, xh, xl, sx);
#pragma unroll
                    for (int g = 0; g < kGroupsPerIter; g++) acc[g][warp * 32 + lane] = v[g];
                } else {
#pragma unroll
                    for (int g = 0; g < kGroupsPerIter; g++)
                        if (g < cnt) acc[g][warp * 32 + lane] = q8_tile_dot(st[g], L, warp, lane, xh, xl, sx);
                }
            }
        } else {
            for (int t = warp; t < T; t += kConsumerWarps) {
                uint4 th[4], tl[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    th[j] = reinterpret_cast<const uint4*>(xh_s + t * 16)[j];
                    tl[j] = reinterpret_cast<const uint4*>(xl_s + t * 16)[j];
                }
                const int2 sxt = reinterpret_cast<const int2*>(sx_s)[t];
                for (int g = 0; g < cnt; g++) acc[g][t * 32 + lane] = q8_tile_dot(st[g], L, t, lane, th, tl, sxt);
            }
        }
        __syncwarp();
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < kGroupsPerIter; g++)
                if (g < cnt) {
                    mbar_arrive(&empty[sg[g]]);
                    mbar_arrive(&acc_full[bg[g]]);
                }
        }
    }
}

size_t q8_smem_bytes(const Q8Layout& L)
{
    return (size_t)L.stages * L.group_bytes + (2 * L.stages + 2 * kAccBufs) * sizeof(uint64_t) +
           kAccBufs * ((size_t)L.T * 32 * 8 + 128) + (size_t)L.T * 16 * 4 * 2 + (size_t)L.T * 2 * 4 +
           (size_t)L.T * 64 * 2 + 32 * 4;  // red[16], xs, abort flag
}

}  // namespace

int register_q8_0(tmac_weight_s* w, const uint8_t* d_raw, const float* d_row_max_abs, cudaStream_t s)
{
    if (w->cols % 32) return fail(TMAC_ERR_SHAPE, "Q8_0 needs cols % 32 == 0");
    const int wpb = 8;
    Q8Layout L = q8_layout(w->rows, w->cols);
    w->tiles = L.T;
    w->groups = L.groups;
    w->group_bytes = L.group_bytes;
    w->data_bytes = (size_t)(L.groups * L.group_bytes);
    if (L.stages < 2) return fail(TMAC_ERR_SHAPE, "Q8_0: cols too large for a two-stage row-group pipeline");
    TMAC_CUDA_TRY(cudaMalloc(&w->row_norm, (size_t)w->rows * sizeof(float)));
    TMAC_CUDA_TRY(cudaMalloc(&w->data, w->data_bytes));
    TMAC_CUDA_TRY(cudaMalloc(&w->top1_scratch, 16));
    TMAC_CUDA_TRY(cudaMemsetAsync(w->top1_scratch, 0, 16, s));
    q8_row_scale_kernel<<<(unsigned)((w->rows + wpb - 1) / wpb), wpb * 32, 0, s>>>(d_raw, w->rows, w->cols,
                                                                                   d_row_max_abs, w->row_norm);
    TMAC_CUDA_TRY(cudaGetLastError());
    dim3 grid(L.T, (unsigned)L.groups);
    q8_pack_kernel<<<grid, 192, 0, s>>>(d_raw, w->rows, w->cols, w->row_norm, L, w->data);
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int q8_planes(const tmac_weight_s* w, int8_t* wh, uint8_t* wl, cudaStream_t s)
{
    if (w->cols % 16) return fail(TMAC_ERR_SHAPE, "q8_planes: cols must be a multiple of 16");
    const Q8Layout L = q8_layout(w->rows, w->cols);
    const int64_t n = w->rows * (w->cols / 16);
    q8_planes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(w->data, L, w->rows, w->cols, wh, wl);
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int launch_q8_0(const tmac_weight_s* w, const float* x, float* y, int64_t* row_acc, int64_t* unit_acc, int batch,
                cudaStream_t s, unsigned long long* top1, int64_t index_base, const int16_t* xq, const float* xs,
                const XchgDev* xg)
{
    if (xg && (batch != 1 || !top1)) return fail(TMAC_ERR_SHAPE, "the fused exchange takes batch 1 and a key");
    Q8Layout L = q8_layout(w->rows, w->cols);
    const size_t smem = q8_smem_bytes(L);
    static bool attr_set[64] = {};
    if (!attr_set[w->device & 63]) {
        TMAC_CUDA_TRY(cudaFuncSetAttribute(q8_gemv_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSmemLimit));
        TMAC_CUDA_TRY(cudaFuncSetAttribute(q8_gemv_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSmemLimit));
        attr_set[w->device & 63] = true;
    }
    const int grid = (int)std::min<int64_t>(L.groups, num_sms(w->device));
    for (int b = 0; b < batch; b++) {
        Q8Args a;
        a.packed = w->data;
        a.L = L;
        a.rows = w->rows;
        a.cols = (int)w->cols;
        a.x = x ? x + (int64_t)b * w->cols : nullptr;
        a.xq_in = xq ? xq + (int64_t)b * w->cols : nullptr;
        a.xs_in = xs ? xs + b : nullptr;
        a.y = y + (int64_t)b * w->rows;
        a.row_acc = row_acc ? row_acc + (int64_t)b * w->rows : nullptr;
        a.unit_acc = unit_acc ? unit_acc + (int64_t)b * w->rows * L.T : nullptr;
        a.top1 = top1 ? top1 + b : nullptr;
        a.index_base = index_base;
        if (xg) {
            a.xg = *xg;
        } else if (top1) {
            a.xg.partial = static_cast<unsigned long long*>(w->top1_scratch);
            a.xg.counter = reinterpret_cast<unsigned*>(a.xg.partial + 1);
        }
        a.err = device_error_word(w->device);
        // the exchange across ranks is a separate instantiation (see top1_cta_finish)
        if (a.xg.peers)
            TMAC_CUDA_TRY(launch_k(q8_gemv_kernel<true>, dim3(grid), dim3(kThreads), smem, s, a));
        else
            TMAC_CUDA_TRY(launch_k(q8_gemv_kernel<false>, dim3(grid), dim3(kThreads), smem, s, a));
        TMAC_CUDA_TRY(cudaGetLastError());
    }
    return TMAC_OK;
}

}  // namespace tmac
