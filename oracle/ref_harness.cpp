// ref_harness.cpp -- exposes the UNMODIFIED reference CPU implementation
// (liuwantao3/tmac-zynq-fpga sim/tmac_gguf.cpp + sim/fpga_sim.hpp +
// sim/matmul_q8.cpp) through a small C ABI, so tests can pin the oracle
// restatement against the reference itself and bench.py can time the
// reference's own CPU path.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile from the reference
// sources where they lie (never copied), with -Dmain=tmac_ref_main so the
// reference's main() does not clash and its file-static state (g_use_fpga,
// g_fpga_*, g_phaseb, g_ddr, dump files) is reachable from here.
#include "tmac_gguf.cpp"

#include <cstdio>
#include <vector>

namespace {

Tensor make_tensor(int type, int64_t rows, int64_t cols, const uint8_t* data, size_t nbytes,
                   const char* name = "w")
{
    Tensor t;
    memset(&t, 0, sizeof(t));
    snprintf(t.name, sizeof(t.name), "%s", name);
    t.rows = (uint64_t)rows;
    t.cols = (uint64_t)cols;
    t.type = (uint32_t)type;
    t.n_bytes = nbytes;
    t.data = const_cast<uint8_t*>(data);
    return t;
}

void set_switches(bool fpga, bool q8, bool q5, bool q4k, bool q6k)
{
    g_use_fpga = fpga;
    g_fpga_q8 = q8;
    g_fpga_q5_0 = q5;
    g_fpga_q4k = q4k;
    g_fpga_q6_k = q6k;
    g_fpga_phaseb = false;
}

}  // namespace

extern "C" {

// path: 0 = the type's FPGA-model driver (matmul_fpga_{q8,q5_0,q4_k,q6_k}),
//       1 = matmul_fpga_int16 (switch off for this type),
//       2 = FP32 path (no --fpga switch).
// Goes through the reference's own matmul() dispatch (tmac_gguf.cpp:473-493),
// except that Q8_0 with a row_max_abs table calls matmul_fpga_q8 directly
// (the reference does this through q8_logits_matmul_with_tensor).
int ref_gemv(int type, int path, const uint8_t* w, int64_t rows, int64_t cols, size_t nbytes,
             const float* x, const float* row_max_abs, float* y)
{
    Tensor t = make_tensor(type, rows, cols, w, nbytes);
    if (path == 0) set_switches(true, true, true, true, true);
    else if (path == 1) set_switches(true, false, false, false, false);
    else set_switches(false, false, false, false, false);
    if (path == 0 && type == TENSOR_Q8_0 && row_max_abs) {
        matmul_fpga_q8(&t, x, y, (int)rows, (int)cols, row_max_abs);
    } else {
        matmul(&t, x, y, (int)rows, (int)cols);
    }
    set_switches(false, false, false, false, false);
    return 0;
}

// Element dequantisation of the FP32 path (read_tensor, tmac_gguf.cpp:398).
float ref_dequant(int type, const uint8_t* w, int64_t rows, int64_t cols, int64_t row, int64_t col)
{
    Tensor t = make_tensor(type, rows, cols, w, 0);
    return read_tensor(&t, (uint64_t)row, (uint64_t)col);
}

// Per-(row, 64-column tile) int64 results of the Q8_0 core model, captured
// through the reference's cosimulation dump (tmac_gguf.cpp:1044-1065): every
// tile matmul_fpga_q8 sends to fpga_sim::axi_vecmul_tile_q8 is written with
// its fpga_sim result.  out[rows * ceil(cols/64)].  Also returns y.
int ref_q8_tile_sums(const uint8_t* w, int64_t rows, int64_t cols, size_t nbytes,
                     const float* x, const float* row_max_abs, float* y, int64_t* out)
{
    Tensor t = make_tensor(TENSOR_Q8_0, rows, cols, w, nbytes);
    int64_t ntiles = (cols + 63) / 64;
    int64_t nbands = (rows + 63) / 64;
    FILE* f = tmpfile();
    if (!f) return -1;
    g_dump_file = f;
    g_dump_tiles_remaining = (int)(nbands * ntiles + 1);  // never reaches 0: we close it
    set_switches(true, true, false, false, false);
    matmul_fpga_q8(&t, x, y, (int)rows, (int)cols, row_max_abs);
    set_switches(false, false, false, false, false);
    g_dump_file = nullptr;
    g_dump_tiles_remaining = 0;
    fflush(f);
    rewind(f);
    std::vector<uint8_t> rec(COSIM_TILE_SIZE);
    for (int64_t band = 0; band < nbands; band++) {
        for (int64_t c = 0; c < ntiles; c++) {
            if (fread(rec.data(), 1, rec.size(), f) != rec.size()) { fclose(f); return -2; }
            const int64_t* res = (const int64_t*)(rec.data() + 4096 + 256 + 128);
            for (int64_t i = 0; i < 64 && band * 64 + i < rows; i++)
                out[(band * 64 + i) * ntiles + c] = res[i];
        }
    }
    fclose(f);
    return 0;
}

// Per-(row, 32-column block) int64 sums of the Q5_0 8x896 core model
// (fpga_sim::axi_vecmul_tile_q5_0_8x896_axilite), obtained by driving the
// model once per block with every other block's activations zeroed.
// rows % 8 == 0, cols == 896 (the model's hard-coded tile).
int ref_q5_0_block_sums(const uint8_t* w, int64_t rows, const int16_t* x_q,
                        const float* row_inv, int64_t* out)
{
    if (rows % 8) return -1;
    std::vector<int16_t> act(896);
    std::vector<int64_t> res(rows);
    for (int b = 0; b < 28; b++) {
        for (int c = 0; c < 896; c++) act[c] = (c / 32 == b) ? x_q[c] : 0;
        std::fill(res.begin(), res.end(), 0);
        for (int64_t row0 = 0; row0 < rows; row0 += 8) {
            fpga_sim::axi_vecmul_tile_q5_0_8x896_axilite(w + row0 * 28 * 22, act.data(),
                                                         row_inv + row0, res.data(), (int)row0);
        }
        for (int64_t r = 0; r < rows; r++) out[r * 28 + b] = res[r];
    }
    return 0;
}

// Same through the hardware-layout 4x896 model
// (fpga_sim::axi_vecmul_tile_q5_0_4x896_axilite) over a pre-packed HW tile
// stream (56 blocks x 48 B per 4-row tile, vivado_integration/API.md); returns
// the int64 row sums for `ntiles` tiles.  row_norm holds 4 floats per tile.
int ref_q5_0_hw_tiles(const uint8_t* tiles, int64_t ntiles, int64_t tile_stride,
                      const int16_t* x_q, const float* row_norm, int64_t* out)
{
    std::vector<int64_t> res(ntiles * 4, 0);
    for (int64_t t = 0; t < ntiles; t++)
        fpga_sim::axi_vecmul_tile_q5_0_4x896_axilite(tiles + t * tile_stride, x_q, row_norm + t * 4,
                                                     res.data(), (int)(t * 4));
    memcpy(out, res.data(), res.size() * sizeof(int64_t));
    return 0;
}

// Per-(row, 256-column block) sums of the Q4_K core model (axilite_q4k_run via
// axi_vecmul_tile_q4k_axilite) and the Q6_K core model
// (axi_vecmul_tile_q6_k_axilite), tiled exactly like matmul_fpga_q4_k /
// matmul_fpga_q6_k (56 / 32 rows x 256 cols).  rows <= 896 (reference arrays).
int ref_kquant_block_sums(int type, const uint8_t* w, int64_t rows, int64_t cols,
                          const int16_t* x_q, const float* row_inv, int64_t* out)
{
    if (rows > 896 || cols % 256) return -1;
    const int bb = (type == TENSOR_Q4_K) ? 144 : 210;
    const int tr = (type == TENSOR_Q4_K) ? 56 : 32;
    const int64_t bpr = cols / 256;
    std::vector<uint8_t> blocks((size_t)tr * bb);
    std::vector<int64_t> res(896);
    std::vector<float> ri(896, 0.0f);
    for (int64_t r = 0; r < rows; r++) ri[r] = row_inv[r];
    for (int64_t cb = 0; cb < bpr; cb++) {
        std::fill(res.begin(), res.end(), 0);
        for (int64_t row0 = 0; row0 < rows; row0 += tr) {
            int nb = (int)std::min<int64_t>(tr, rows - row0);
            for (int bi = 0; bi < nb; bi++)
                memcpy(blocks.data() + bi * bb, w + ((row0 + bi) * bpr + cb) * bb, bb);
            if (type == TENSOR_Q4_K)
                fpga_sim::axi_vecmul_tile_q4k_axilite(blocks.data(), nb, x_q + cb * 256, 256,
                                                      ri.data(), res.data(), (int)row0);
            else
                fpga_sim::axi_vecmul_tile_q6_k_axilite(blocks.data(), nb, x_q + cb * 256, 256,
                                                       ri.data(), res.data(), (int)row0);
        }
        for (int64_t r = 0; r < rows; r++) out[r * bpr + cb] = res[r];
    }
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Phase-B descriptor chain, built and replayed by the reference itself
// (tmac_gguf.cpp:513-880).  The chain lives in the reference's simulated DDR
// (g_ddr) from 0x18000000 up; these entry points expose it byte for byte.
extern "C" {

int ref_phaseb_begin(void)
{
    if (!g_ddr) {
        g_ddr = (uint8_t*)calloc(DDR_SIZE, 1);
        if (!g_ddr) return -1;
    }
    phaseb_init();
    return 0;
}

// One matmul through the reference's FPGA-model driver with --fpga-phaseb on:
// the driver packs the tiles into g_ddr and appends a descriptor.
int ref_phaseb_matmul(int type, const uint8_t* w, int64_t rows, int64_t cols, size_t nbytes,
                      const float* x, float* y)
{
    Tensor t = make_tensor(type, rows, cols, w, nbytes);
    set_switches(true, true, true, true, true);
    g_fpga_phaseb = true;
    matmul(&t, x, y, (int)rows, (int)cols);
    set_switches(false, false, false, false, false);
    return 0;
}

// head: first descriptor; base/end: the allocated arena [0x18000000, next_off).
int ref_phaseb_info(uint32_t* head, uint32_t* base, uint32_t* end, int* nslots)
{
    *head = g_phaseb.head;
    *base = 0x18000000u;
    *end = g_phaseb.next_off;
    *nslots = (int)g_phaseb.slots.size();
    return 0;
}

int ref_phaseb_copy(uint8_t* out, uint32_t off, uint32_t n)
{
    if (!g_ddr || (uint64_t)off + n > DDR_SIZE) return -1;
    memcpy(out, g_ddr + off, n);
    return 0;
}

int ref_phaseb_write(const uint8_t* in, uint32_t off, uint32_t n)
{
    if (!g_ddr || (uint64_t)off + n > DDR_SIZE) return -1;
    memcpy(g_ddr + off, in, n);
    return 0;
}

// phaseb_run_descriptor on a zeroed accumulator; returns the rows it wrote.
int ref_phaseb_run(uint32_t desc_off, int64_t* acc, int64_t cap)
{
    auto* d = (fpga_sim::PhaseBDescriptor*)(g_ddr + desc_off);
    int64_t need = (d->tensor_type == fpga_sim::DESC_TYPE_Q5_0)
                       ? (int64_t)d->num_tiles * d->tile_res_rows
                       : (d->num_col_groups ? (int64_t)(d->num_tiles / d->num_col_groups) * d->tile_res_rows : 0);
    if (need > cap) return -1;
    memset(acc, 0, (size_t)cap * sizeof(int64_t));
    return phaseb_run_descriptor(desc_off, acc);
}

// phaseb_verify: replays the chain, writes int64 results at each result_addr,
// compares against the drivers' y (|err| <= 2); returns the error count.
int ref_phaseb_verify(void) { return phaseb_verify(); }

// phaseb_dump_files (tmac_gguf.cpp:597-708) on the chain built so far: writes
// the reference's testbench files /tmp/tb_phaseb.bin and /tmp/tb_phaseb.hdr.
int ref_phaseb_dump(void)
{
    phaseb_dump_files();
    return 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Whole-model greedy decode with the reference engine itself: load_tmac,
// process_prompt, then per step get_logits_q8 / argmax / process_embedding /
// forward_all_layers -- generate() (tmac_gguf.cpp:2025-2047) with the top-k
// sampler replaced by a lowest-index argmax.
// fpga = 1: --fpga-q8 --fpga-q5-0 --fpga-q4k --fpga-q6-k; 0: FP32 path.
extern "C" int ref_decode(const char* path, const int* tokens, int n_prompt, int n_gen, int fpga,
                          int* out_tokens, float* out_logit, float* out_hidden)
{
    if (!g_ddr) {
        g_ddr = (uint8_t*)calloc(DDR_SIZE, 1);
        if (!g_ddr) return -1;
    }
    if (g_tensors) {
        free(g_tensors);
        g_tensors = nullptr;
    }
    if (load_tmac(path) != 0) return -2;
    set_switches(fpga != 0, fpga != 0, fpga != 0, fpga != 0, fpga != 0);
    std::vector<float> hidden(HIDDEN_DIM), logits(VOCAB_SIZE);
    std::vector<int> prompt(tokens, tokens + n_prompt);
    if (process_prompt(hidden.data(), prompt, false) != 0) return -3;
    if (out_hidden) memcpy(out_hidden, hidden.data(), HIDDEN_DIM * sizeof(float));
    int produced = 0;
    for (int gen = 0; gen < n_gen; gen++) {
        int pos = n_prompt + gen;
        if (pos >= MAX_SEQ_LEN) break;
        if (g_fpga_q8) get_logits_q8(logits.data(), hidden.data());
        else get_logits(logits.data(), hidden.data());
        int best = 0;
        for (int i = 1; i < VOCAB_SIZE; i++)
            if (logits[i] > logits[best]) best = i;
        out_tokens[gen] = best;
        if (out_logit) out_logit[gen] = logits[best];
        process_embedding(hidden.data(), best);
        forward_all_layers(hidden.data(), pos);
        if (out_hidden) memcpy(out_hidden + (size_t)(gen + 1) * HIDDEN_DIM, hidden.data(), HIDDEN_DIM * sizeof(float));
        produced++;
    }
    set_switches(false, false, false, false, false);
    return produced;
}
