// chain.cu -- Phase-B descriptor-chain runner (tmac_chain_run).
//
// Replaces phaseb_run_descriptor as driven by phaseb_verify
// (sim/tmac_gguf.cpp:761-831, :834-880): walk the PhaseBDescriptor list
// (sim/fpga_sim.hpp:1254-1279) held in a DDR-image arena and, per descriptor,
// compute the int64 row accumulators of the packed tiles the way the
// reference's core models do, then store them at result_addr.
//   Q5_0 (type 6): 8x896 tiles of 224 GGUF blocks; row_inv is recomputed from
//                  the tile's own blocks (phaseb_q5_0_row_inv, :740-759) and the
//                  UQ16.8 scale section is ignored, as the reference does.
//   Q4_K (12) / Q6_K (14): 56/32-row x 256-col tiles, tile index
//                  ti = row_group * num_col_groups + col_group; row_inv =
//                  (float)UQ24.8 / 256 from the tile's scale section.
//   CPU_OP (15): no arithmetic, 0 rows.  Any other type: skipped, 0 rows.
// The chain is walked on the host (descriptors are 32 bytes; the arena's host
// mirror is used when the caller has one), every offset is bounds-checked, and
// one kernel per arithmetic descriptor is enqueued in chain order.
//
// tmac_chain_run_hw walks the FPGA's own HP-FSM descriptor format instead
// (tmac_hw_desc, vivado_integration/sw/tmac_baremetal.h:100-113): Q5_0 type 1
// as 4-row tiles of 48-byte two-core blocks (axi_vecmul_tile_q5_0_4x896_axilite,
// fpga_sim.hpp:1194-1249), CPU_OP 15 as the FSM's act -> result passthrough.
#include "common.cuh"
#include "dequant.cuh"

#include <algorithm>
#include <cstring>
#include <vector>

namespace tmac {
namespace {

constexpr int kQ5Cols = 896, kQ5BlocksPerRow = 28, kQ5Rows = 8;
constexpr int kQ4kBlkBytes = 56 * 144, kQ6kBlkBytes = 32 * 210;

TMAC_DEV uint32_t ld_u32_bytes(const uint8_t* p)
{
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
TMAC_DEV int16_t ld_i16_bytes(const uint8_t* p) { return (int16_t)(uint16_t)(p[0] | (p[1] << 8)); }

TMAC_DEV void st_i64_bytes(uint8_t* p, long long v)
{
    if (((uintptr_t)p & 7) == 0) {
        *reinterpret_cast<long long*>(p) = v;
    } else {
        for (int i = 0; i < 8; i++) p[i] = (uint8_t)((unsigned long long)v >> (8 * i));
    }
}

TMAC_DEV long long warp_sum_i64(long long v)
{
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One CTA per tile, one warp per row, one lane per 32-value block.
__global__ void __launch_bounds__(256) chain_q5_0_kernel(const uint8_t* __restrict__ weight, const uint8_t* __restrict__ act,
                                                         uint8_t* result, int tile_bytes)
{
    const int t = blockIdx.x, i = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint8_t* row = weight + (int64_t)t * tile_bytes + i * kQ5BlocksPerRow * 22;
    const bool has = lane < kQ5BlocksPerRow;
    float d = 0.0f;
    uint32_t qh = 0;
    const uint8_t* blk = row + (has ? lane : 0) * 22;
    if (has) {
        d = f16_bits_to_f32(ld_u16_unaligned(blk));
        qh = ld_u32_bytes(blk + 2);
    }
    // row_inv from this tile's blocks (tmac_gguf.cpp:740-759)
    float mx = 0.0f;
    if (has)
        for (int wi = 0; wi < 32; wi++) {
            const int j = wi < 16 ? wi : wi - 16;
            const int ql = wi < 16 ? (blk[6 + j] & 0xF) : (blk[6 + j] >> 4);
            const int q = ((((qh >> wi) & 1) << 4) | ql) - 16;
            mx = fmaxf(mx, fabsf(__fmul_rn(d, (float)q)));
        }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float ri = __fdiv_rn(32767.0f, (mx < 1e-10f) ? 1.0f : mx);
    // axi_vecmul_tile_q5_0_8x896_axilite (fpga_sim.hpp:1004-1052)
    long long acc = 0;
    if (has)
        for (int wi = 0; wi < 32; wi++) {
            const int j = wi < 16 ? wi : wi - 16;
            const int ql = wi < 16 ? (blk[6 + j] & 0xF) : (blk[6 + j] >> 4);
            const int q = ((((qh >> wi) & 1) << 4) | ql) - 16;
            const int v = clamp_round_i16(__fmul_rn(__fmul_rn(d, (float)q), ri));
            acc += (long long)v * (long long)ld_i16_bytes(act + 2 * (lane * 32 + wi));
        }
    acc = warp_sum_i64(acc);
    if (lane == 0) st_i64_bytes(result + ((int64_t)t * kQ5Rows + i) * 8, acc);
}

// Hardware-format Q5_0 tile (tmac_hw_desc type 1): one CTA per 4-row tile,
// warp i = row i, lane j = the row's 32-column block j.  Row i's block j is the
// core (i >> 1) half of 48-byte block (i & 1) * 28 + j (vivado_integration/API.md,
// "Q5_0 (tensor_type=1)"); the arithmetic is axi_vecmul_tile_q5_0_4x896_axilite
// (fpga_sim.hpp:1194-1249) with the row norm recomputed from the row's blocks.
__global__ void __launch_bounds__(128) chain_q5_0_hw_kernel(const uint8_t* __restrict__ weight,
                                                            const uint8_t* __restrict__ act, uint8_t* result)
{
    const int t = blockIdx.x, i = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool has = lane < kQ5BlocksPerRow;
    const uint8_t* blk = weight + (int64_t)t * TMAC_HW_Q5_0_TILE_BYTES +
                         ((i & 1) * kQ5BlocksPerRow + (has ? lane : 0)) * 48 + (i >> 1) * 22;
    float d = 0.0f;
    uint32_t qh = 0;
    uint8_t qs[16];
    if (has) {
        d = f16_bits_to_f32(ld_u16_unaligned(blk));
        qh = ld_u32_bytes(blk + 2);
#pragma unroll
        for (int k = 0; k < 16; k++) qs[k] = blk[6 + k];
    }
    // the row norm of q5_preprocess_tile (tmac_baremetal.cpp:497-516): 32767 / max|d*q|
    float mx = 0.0f;
    if (has) {
#pragma unroll
        for (int wi = 0; wi < 32; wi++) {
            const int ql = wi < 16 ? (qs[wi] & 0xF) : (qs[wi - 16] >> 4);
            const int q = ((((qh >> wi) & 1) << 4) | ql) - 16;
            mx = fmaxf(mx, fabsf(__fmul_rn(d, (float)q)));
        }
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float rn = (mx < 1e-10f) ? 1.0f : __fdiv_rn(32767.0f, mx);
    long long acc = 0;
    if (has) {
        const uint8_t* a = act + 2 * (lane * 32);
#pragma unroll
        for (int wi = 0; wi < 32; wi++) {
            const int ql = wi < 16 ? (qs[wi] & 0xF) : (qs[wi - 16] >> 4);
            const int q = ((((qh >> wi) & 1) << 4) | ql) - 16;
            // d * (float)q5 * row_norm, left to right, then clamp and roundf
            const int v = clamp_round_i16(__fmul_rn(__fmul_rn(d, (float)q), rn));
            acc += (long long)v * (long long)ld_i16_bytes(a + 2 * wi);
        }
    }
    acc = warp_sum_i64(acc);
    if (lane == 0) st_i64_bytes(result + ((int64_t)t * 4 + i) * 8, acc);
}

// Passthrough of a hardware CPU_OP descriptor: act bytes copied to result.
__global__ void chain_copy_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, uint32_t n)
{
    for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < n; k += gridDim.x * blockDim.x) dst[k] = src[k];
}

// One CTA per row group, one warp per row, 8 values per lane per column group.
template <int TYPE>
__global__ void __launch_bounds__(256) chain_kquant_kernel(const uint8_t* __restrict__ weight,
                                                           const uint8_t* __restrict__ act, uint8_t* result,
                                                           int tile_bytes, int tr, int cg)
{
    constexpr int BB = (TYPE == TMAC_TYPE_Q4_K) ? 144 : 210;
    constexpr int BLK = (TYPE == TMAC_TYPE_Q4_K) ? kQ4kBlkBytes : kQ6kBlkBytes;
    const int rg = blockIdx.x, lane = threadIdx.x & 31;
    for (int bi = threadIdx.x >> 5; bi < tr; bi += blockDim.x >> 5) {
        const int out_row = rg * tr + bi;
        long long acc = 0;
        for (int c = 0; c < cg; c++) {
            const uint8_t* tile = weight + ((int64_t)rg * cg + c) * tile_bytes;
            const uint8_t* blk = tile + bi * BB;
            // row_inv from the tile's UQ24.8 scale section (tmac_gguf.cpp:790-795)
            const float ri = __fdiv_rn(__uint2float_rn(ld_u32_bytes(tile + BLK + bi * 4)), 256.0f);
            const uint8_t* a = act + c * 256 * 2;
            long long s = 0;
            for (int k = 0; k < 8; k++) {
                const int wi = lane * 8 + k;
                float val;
                if (TYPE == TMAC_TYPE_Q4_K) {
                    // axilite_q4k_run (fpga_sim.hpp:730-788)
                    const float d = f16_bits_to_f32(ld_u16_unaligned(blk));
                    const float dmin = f16_bits_to_f32(ld_u16_unaligned(blk + 2));
                    int sc, m;
                    q4_k_scale_min(blk + 4, wi / 32, sc, m);
                    if (sc > 63) sc = 63;
                    if (m > 63) m = 63;
                    const int sub = wi / 32, j = wi % 32;
                    const uint8_t qb = blk[16 + (sub / 2) * 32 + j];
                    const int q4 = (sub % 2 == 0) ? (qb & 0xF) : (qb >> 4);
                    val = __fmul_rn(__fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q4), __fmul_rn(dmin, (float)m)),
                                    ri);
                } else {
                    // axi_vecmul_tile_q6_k_axilite (fpga_sim.hpp:1058-1115)
                    const float d = f16_bits_to_f32(ld_u16_unaligned(blk + 208));
                    const int half = wi / 128, pos = wi % 128, l = pos % 32, sub = pos / 32;
                    const uint8_t lb = blk[half * 64 + l + (sub % 2) * 32];
                    const int ql = (sub < 2) ? (lb & 0xF) : (lb >> 4);
                    const int qh = (blk[128 + half * 32 + l] >> (sub * 2)) & 0x3;
                    const int q6 = ((qh << 4) | ql) - 32;
                    const float scf = (float)(int8_t)blk[192 + half * 8 + (l / 16) + sub * 2];
                    val = __fmul_rn(__fmul_rn(__fmul_rn(d, scf), (float)q6), ri);
                }
                s += (long long)ld_i16_bytes(a + 2 * wi) * (long long)clamp_round_i16(val);
            }
            acc += warp_sum_i64(s);
        }
        // the reference's accumulator only takes rows < 896 (fpga_sim.hpp:784, :1110)
        if (lane == 0) st_i64_bytes(result + (int64_t)out_row * 8, out_row < 896 ? acc : 0);
    }
}

struct Walked {
    tmac_phaseb_desc d;
    int64_t rows;
};

bool in_arena(uint64_t off, uint64_t n, uint64_t base, uint64_t bytes)
{
    return off >= base && off - base <= bytes && n <= bytes - (off - base);
}

}  // namespace
}  // namespace tmac

using namespace tmac;

extern "C" int tmac_chain_run(void* arena_dev, size_t arena_bytes, uint32_t arena_base, const void* arena_host,
                              uint32_t head, int max_desc, tmac_chain_stats* stats, void* stream)
{
    if (!arena_dev) return fail(TMAC_ERR_INVALID, "NULL arena");
    if (max_desc <= 0) return fail(TMAC_ERR_INVALID, "max_desc must be positive");
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* dev = static_cast<uint8_t*>(arena_dev);
    const uint8_t* host = static_cast<const uint8_t*>(arena_host);
    std::vector<Walked> chain;
    tmac_chain_stats st{};
    // 1. walk and validate the whole chain before launching anything
    for (uint32_t off = head; off != 0;) {
        if ((int)chain.size() >= max_desc)
            return fail(TMAC_ERR_BOUNDS, "descriptor chain longer than max_desc (cycle?)");
        if (!in_arena(off, sizeof(tmac_phaseb_desc), arena_base, arena_bytes))
            return fail(TMAC_ERR_BOUNDS, "descriptor offset outside the arena");
        Walked w;
        if (host) {
            memcpy(&w.d, host + (off - arena_base), sizeof(w.d));
        } else {
            TMAC_CUDA_TRY(cudaMemcpy(&w.d, dev + (off - arena_base), sizeof(w.d), cudaMemcpyDeviceToHost));
        }
        const tmac_phaseb_desc& d = w.d;
        const uint64_t tiles_end = (uint64_t)d.num_tiles * d.tile_bytes;
        w.rows = 0;
        switch (d.tensor_type) {
        case TMAC_DESC_TYPE_Q5_0:
            if (d.tile_res_rows != 8 || d.tile_bytes < 224 * 22)
                return fail(TMAC_ERR_BOUNDS, "Q5_0 descriptor: tiles must be 8 rows x 896 columns");
            w.rows = (int64_t)d.num_tiles * 8;
            if (!in_arena(d.weight_addr, tiles_end, arena_base, arena_bytes) ||
                !in_arena(d.act_addr, kQ5Cols * 2, arena_base, arena_bytes) ||
                !in_arena(d.result_addr, (uint64_t)w.rows * 8, arena_base, arena_bytes))
                return fail(TMAC_ERR_BOUNDS, "Q5_0 descriptor: weight/act/result outside the arena");
            break;
        case TMAC_DESC_TYPE_Q4_K:
        case TMAC_DESC_TYPE_Q6_K: {
            const bool q4 = d.tensor_type == TMAC_DESC_TYPE_Q4_K;
            const int bb = q4 ? 144 : 210, blk = q4 ? kQ4kBlkBytes : kQ6kBlkBytes;
            if (d.num_col_groups == 0 || d.num_tiles % d.num_col_groups)
                return fail(TMAC_ERR_BOUNDS, "K-quant descriptor: num_tiles must be a multiple of num_col_groups");
            if (d.tile_res_rows == 0 || d.tile_res_rows * bb > blk || d.tile_bytes < blk + d.tile_res_rows * 4)
                return fail(TMAC_ERR_BOUNDS, "K-quant descriptor: tile_res_rows / tile_bytes inconsistent");
            w.rows = (int64_t)(d.num_tiles / d.num_col_groups) * d.tile_res_rows;
            if (!in_arena(d.weight_addr, tiles_end, arena_base, arena_bytes) ||
                !in_arena(d.act_addr, (uint64_t)d.num_col_groups * 512, arena_base, arena_bytes) ||
                !in_arena(d.result_addr, (uint64_t)w.rows * 8, arena_base, arena_bytes))
                return fail(TMAC_ERR_BOUNDS, "K-quant descriptor: weight/act/result outside the arena");
            break;
        }
        case TMAC_DESC_TYPE_CPU_OP: break;
        default: st.unsupported++; break;
        }
        chain.push_back(w);
        off = d.next_desc_addr;
    }
    // 2. enqueue one kernel per arithmetic descriptor, in chain order
    for (const Walked& w : chain) {
        const tmac_phaseb_desc& d = w.d;
        st.descriptors++;
        st.result_rows += w.rows;
        if (w.rows == 0) continue;
        const uint8_t* wt = dev + (d.weight_addr - arena_base);
        const uint8_t* act = dev + (d.act_addr - arena_base);
        uint8_t* res = dev + (d.result_addr - arena_base);
        if (d.tensor_type == TMAC_DESC_TYPE_Q5_0) {
            chain_q5_0_kernel<<<d.num_tiles, 256, 0, s>>>(wt, act, res, d.tile_bytes);
        } else if (d.tensor_type == TMAC_DESC_TYPE_Q4_K) {
            chain_kquant_kernel<TMAC_TYPE_Q4_K><<<d.num_tiles / d.num_col_groups, 256, 0, s>>>(
                wt, act, res, d.tile_bytes, d.tile_res_rows, d.num_col_groups);
        } else {
            chain_kquant_kernel<TMAC_TYPE_Q6_K><<<d.num_tiles / d.num_col_groups, 256, 0, s>>>(
                wt, act, res, d.tile_bytes, d.tile_res_rows, d.num_col_groups);
        }
        TMAC_CUDA_TRY(cudaGetLastError());
    }
    if (stats) *stats = st;
    return TMAC_OK;
}

// Phase-B dump for the Verilog testbench (phaseb_dump_files, tmac_gguf.cpp:597-708):
// the expected rows of every descriptor come from the GPU runner above, one
// descriptor at a time (its next_desc_addr cleared in a scratch copy of the arena),
// exactly as the reference runs phaseb_run_descriptor per descriptor.
extern "C" int tmac_phaseb_dump(const void* arena_host, size_t arena_bytes, uint32_t arena_base, uint32_t head,
                                uint32_t desc_base, uint32_t bin_base, const char* bin_path, const char* hdr_path,
                                int device)
{
    if (!arena_host || !bin_path || !hdr_path) return fail(TMAC_ERR_INVALID, "NULL arena or path");
    const uint8_t* src = static_cast<const uint8_t*>(arena_host);
    // 1. the chain, walked and bounds-checked on the host
    std::vector<uint32_t> offs;
    for (uint32_t off = head; off != 0;) {
        if (offs.size() >= (1u << 20)) return fail(TMAC_ERR_BOUNDS, "descriptor chain too long (cycle?)");
        if (!in_arena(off, sizeof(tmac_phaseb_desc), arena_base, arena_bytes))
            return fail(TMAC_ERR_BOUNDS, "descriptor offset outside the arena");
        offs.push_back(off);
        tmac_phaseb_desc d;
        memcpy(&d, src + (off - arena_base), sizeof(d));
        off = d.next_desc_addr;
    }
    const uint64_t ndesc = offs.size();
    const uint64_t desc_end = (uint64_t)desc_base + ndesc * sizeof(tmac_phaseb_desc);
    if ((desc_base & 31u) || !in_arena(desc_base, ndesc * sizeof(tmac_phaseb_desc), arena_base, arena_bytes))
        return fail(TMAC_ERR_BOUNDS, "desc_base must be 32-byte aligned with room for the descriptors in the arena");
    if (bin_base < arena_base || bin_base > desc_base) return fail(TMAC_ERR_BOUNDS, "bin_base outside [arena, desc_base]");
    // 2. expected rows on the GPU
    DeviceGuard dg(device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    std::vector<uint8_t> mirror(src, src + arena_bytes);
    uint8_t* dev = nullptr;
    TMAC_CUDA_TRY(cudaMalloc(&dev, arena_bytes));
    struct Freer {
        uint8_t* p;
        ~Freer() { cudaFree(p); }
    } freer{dev};
    TMAC_CUDA_TRY(cudaMemcpy(dev, src, arena_bytes, cudaMemcpyHostToDevice));
    struct Info {
        uint32_t result_addr, rows, act_bytes;
        std::vector<int64_t> acc;
    };
    std::vector<Info> info(ndesc);
    for (uint64_t i = 0; i < ndesc; i++) {
        const uint32_t off = offs[i];
        tmac_phaseb_desc d;
        memcpy(&d, src + (off - arena_base), sizeof(d));
        tmac_phaseb_desc alone = d;
        alone.next_desc_addr = 0;
        memcpy(mirror.data() + (off - arena_base), &alone, sizeof(alone));
        TMAC_CUDA_TRY(cudaMemcpy(dev + (off - arena_base), &alone, sizeof(alone), cudaMemcpyHostToDevice));
        tmac_chain_stats st{};
        const int rc = tmac_chain_run(dev, arena_bytes, arena_base, mirror.data(), off, 1, &st, nullptr);
        if (rc) return rc;
        Info& in = info[i];
        in.result_addr = d.result_addr;
        in.rows = (uint32_t)st.result_rows;
        in.act_bytes = d.act_total_bytes;
        in.acc.resize(in.rows);
        if (in.rows)
            TMAC_CUDA_TRY(cudaMemcpy(in.acc.data(), dev + (d.result_addr - arena_base), (size_t)in.rows * 8,
                                     cudaMemcpyDeviceToHost));
        memcpy(mirror.data() + (off - arena_base), &d, sizeof(d));
        TMAC_CUDA_TRY(cudaMemcpy(dev + (off - arena_base), &d, sizeof(d), cudaMemcpyHostToDevice));
    }
    // 3. the DDR image with the descriptors placed contiguously at desc_base
    std::vector<uint8_t> img(src, src + arena_bytes);
    for (uint64_t i = 0; i < ndesc; i++) {
        tmac_phaseb_desc d;
        memcpy(&d, src + (offs[i] - arena_base), sizeof(d));
        d.next_desc_addr = (i + 1 < ndesc) ? 0xFFFFFFFFu : 0u;
        memcpy(img.data() + (desc_base - arena_base) + i * sizeof(d), &d, sizeof(d));
    }
    FILE* fb = fopen(bin_path, "wb");
    if (!fb) return fail(TMAC_ERR_INVALID, std::string("cannot write ") + bin_path);
    const size_t nb = (size_t)(desc_end - bin_base);
    const bool okb = fwrite(img.data() + (bin_base - arena_base), 1, nb, fb) == nb;
    fclose(fb);
    if (!okb) return fail(TMAC_ERR_INVALID, std::string("short write to ") + bin_path);
    // 4. the header
    std::vector<uint32_t> h = {0x50484244u, (uint32_t)ndesc, desc_base, 0u};
    uint32_t pos = 0, prev = 0;
    for (const Info& in : info) {
        h.insert(h.end(), {in.result_addr, in.rows, in.act_bytes, prev, pos});
        pos += in.rows;
        prev = in.result_addr;
    }
    h[3] = pos;
    FILE* fh = fopen(hdr_path, "wb");
    if (!fh) return fail(TMAC_ERR_INVALID, std::string("cannot write ") + hdr_path);
    bool okh = fwrite(h.data(), 4, h.size(), fh) == h.size();
    for (const Info& in : info)
        if (in.rows) okh = okh && fwrite(in.acc.data(), 8, in.rows, fh) == in.rows;
    fclose(fh);
    if (!okh) return fail(TMAC_ERR_INVALID, std::string("short write to ") + hdr_path);
    return TMAC_OK;
}

// Hardware-format chain (tmac_hw_desc, vivado_integration/sw/tmac_baremetal.h:100-113).
extern "C" int tmac_chain_run_hw(void* arena_dev, size_t arena_bytes, uint32_t arena_base, const void* arena_host,
                                 uint32_t head, int max_desc, tmac_chain_stats* stats, void* stream)
{
    if (!arena_dev) return fail(TMAC_ERR_INVALID, "NULL arena");
    if (max_desc <= 0) return fail(TMAC_ERR_INVALID, "max_desc must be positive");
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* dev = static_cast<uint8_t*>(arena_dev);
    const uint8_t* host = static_cast<const uint8_t*>(arena_host);
    struct HwWalked {
        tmac_hw_desc d;
        int tiles;
        uint32_t act_bytes;
        int64_t rows;
    };
    std::vector<HwWalked> chain;
    tmac_chain_stats st{};
    for (uint32_t off = head; off != 0;) {
        if ((int)chain.size() >= max_desc)
            return fail(TMAC_ERR_BOUNDS, "descriptor chain longer than max_desc (cycle?)");
        if (!in_arena(off, sizeof(tmac_hw_desc), arena_base, arena_bytes))
            return fail(TMAC_ERR_BOUNDS, "descriptor offset outside the arena");
        HwWalked w;
        if (host) {
            memcpy(&w.d, host + (off - arena_base), sizeof(w.d));
        } else {
            TMAC_CUDA_TRY(cudaMemcpy(&w.d, dev + (off - arena_base), sizeof(w.d), cudaMemcpyDeviceToHost));
        }
        const tmac_hw_desc& d = w.d;
        w.tiles = d.num_tiles ? d.num_tiles : 1;  // 0 -> 1 (API.md: backward compatible)
        w.act_bytes = (uint32_t)d.act_total_bytes[0] | ((uint32_t)d.act_total_bytes[1] << 8) |
                      ((uint32_t)d.act_total_bytes[2] << 16);
        w.rows = 0;
        if (d.tensor_type == TMAC_HW_DESC_Q5_0) {
            if (w.act_bytes < kQ5Cols * 2)
                return fail(TMAC_ERR_BOUNDS, "HW Q5_0 descriptor: act_total_bytes below 896 int16 values");
            w.rows = (int64_t)w.tiles * 4;
            if (!in_arena(d.weight_addr, (uint64_t)w.tiles * TMAC_HW_Q5_0_TILE_BYTES, arena_base, arena_bytes) ||
                !in_arena(d.act_addr, kQ5Cols * 2, arena_base, arena_bytes) ||
                !in_arena(d.result_addr, (uint64_t)w.rows * 8, arena_base, arena_bytes))
                return fail(TMAC_ERR_BOUNDS, "HW Q5_0 descriptor: weight/act/result outside the arena");
        } else if (d.tensor_type == TMAC_HW_DESC_CPU_OP) {
            if (!in_arena(d.act_addr, w.act_bytes, arena_base, arena_bytes) ||
                !in_arena(d.result_addr, w.act_bytes, arena_base, arena_bytes))
                return fail(TMAC_ERR_BOUNDS, "HW CPU_OP descriptor: act/result outside the arena");
            const uint64_t a0 = d.act_addr, r0 = d.result_addr;
            if (w.act_bytes && a0 < r0 + w.act_bytes && r0 < a0 + w.act_bytes && a0 != r0)
                return fail(TMAC_ERR_BOUNDS, "HW CPU_OP descriptor: act and result ranges overlap");
        } else {
            st.unsupported++;
        }
        chain.push_back(w);
        off = d.next_addr;
    }
    for (const HwWalked& w : chain) {
        const tmac_hw_desc& d = w.d;
        st.descriptors++;
        st.result_rows += w.rows;
        if (d.tensor_type == TMAC_HW_DESC_Q5_0) {
            chain_q5_0_hw_kernel<<<w.tiles, 128, 0, s>>>(dev + (d.weight_addr - arena_base),
                                                         dev + (d.act_addr - arena_base),
                                                         dev + (d.result_addr - arena_base));
            TMAC_CUDA_TRY(cudaGetLastError());
        } else if (d.tensor_type == TMAC_HW_DESC_CPU_OP && w.act_bytes && d.act_addr != d.result_addr) {
            const unsigned grid = std::min(148u, (w.act_bytes + 255u) / 256u);
            chain_copy_kernel<<<grid, 256, 0, s>>>(dev + (d.act_addr - arena_base), dev + (d.result_addr - arena_base),
                                                   w.act_bytes);
            TMAC_CUDA_TRY(cudaGetLastError());
        }
    }
    if (stats) *stats = st;
    return TMAC_OK;
}
