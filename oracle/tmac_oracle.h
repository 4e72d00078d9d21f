/*
 * tmac_oracle.h -- CPU restatement of the reference's quantized-GEMV hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * product path; it is never linked into, loaded by, or called from the
 * product (tmac_zynq_fpga_b200/).  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference legs may use it.
 *
 * Every function restates one piece of liuwantao3/tmac-zynq-fpga's CPU code
 * (sim/tmac_gguf.cpp and the bit-accurate core models in sim/fpga_sim.hpp),
 * keeping the exact fp32 / fp64 operation order so results are bit-identical.
 * It is pinned against the reference itself, compiled from its own sources
 * into oracle/_ref/ (see oracle/Makefile, oracle/ref_harness.cpp), and against
 * the known-answer tests of sim/test_integration.cpp.
 *
 * Build with -ffp-contract=off: an FMA contraction changes the fp32 results.
 */
#ifndef TMAC_ORACLE_H
#define TMAC_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type codes as used by sim/tmac_gguf.cpp:151-156. */
enum {
    ORC_F32 = 0, ORC_F16 = 1, ORC_Q5_0 = 6, ORC_Q8_0 = 8, ORC_Q4_K = 12, ORC_Q6_K = 14
};

/* fp16 bits -> fp32 (exact); fpga_sim.hpp:113-123, tmac_gguf.cpp:209-220. */
float orc_f16_to_f32(uint16_t h);

/* Per-call activation quantisation, shared by every matmul_fpga_* driver
 * (tmac_gguf.cpp:889-896, :953-960, :1100-1106, :1225-1231, :1372-1378).
 * Writes x_q[n] and returns x_scale. */
float orc_quantize_x(const float* x, int64_t n, int16_t* x_q);

/* Element dequantisation of the FP32 path, read_tensor (tmac_gguf.cpp:398-411). */
float orc_dequant(int type, const uint8_t* w, int64_t cols, int64_t row, int64_t col);

/* Weight-only row normalisers.
 *   Q5_0: row_inv = 32767/max|d*q|          (tmac_gguf.cpp:1242-1263)
 *   Q4_K: row_inv via block float dequant   (tmac_gguf.cpp:1116-1136)
 *   Q6_K: row_inv                           (tmac_gguf.cpp:1385-1424)
 *   Q8_0: row_scale = max|q*d|/32767, or from row_max_abs (tmac_gguf.cpp:980-1004) */
void orc_row_inv_q5_0(const uint8_t* w, int64_t rows, int64_t cols, float* row_inv);
void orc_row_inv_q4_k(const uint8_t* w, int64_t rows, int64_t cols, float* row_inv);
void orc_row_inv_q6_k(const uint8_t* w, int64_t rows, int64_t cols, float* row_inv);
void orc_row_scale_q8_0(const uint8_t* w, int64_t rows, int64_t cols,
                        const float* row_max_abs, float* row_scale);

/* Q8_0 combined UQ8.8 scale for one (row, 32-col block): tmac_gguf.cpp:1022-1039. */
uint16_t orc_q8_combined_scale(float block_scale, float row_scale);

/* Number of partial-sum units per row for each path:
 *   Q8_0 / INT16: 64-column tiles      (one axi_vecmul_tile_{q8,int16} result)
 *   Q5_0:         32-column blocks     (one Q5_0 block inside the 8x896 tile)
 *   Q4_K / Q6_K:  256-column blocks    (one super-block inside a 56/32-row tile) */
int64_t orc_units_per_row(int type, int path, int64_t cols);

/* Path selectors for orc_units_per_row / orc_gemv. */
enum { ORC_PATH_NATIVE = 0, ORC_PATH_INT16 = 1, ORC_PATH_F32 = 2 };

/*
 * One GEMV y[rows] = W[rows x cols] . x[cols] exactly as the reference driver
 * for `type` computes it.
 *   path = ORC_PATH_NATIVE : matmul_fpga_{q8,q5_0,q4_k,q6_k}
 *   path = ORC_PATH_INT16  : matmul_fpga_int16 (the fallback for a type whose
 *                            switch is off, tmac_gguf.cpp:483-485)
 *   path = ORC_PATH_F32    : the FP32 dequant path (tmac_gguf.cpp:488-492)
 * row_max_abs: optional Q8_0 per-row max table (sim/matmul_q8.cpp:22-35).
 * row_acc[rows]: optional int64 row accumulators (NATIVE and INT16 Q5_0/K-quants:
 *                the single int64 sum; Q8_0/INT16: sum of the tile sums).
 * unit_acc[rows * units]: optional int64 per-unit partial sums.
 * Returns 0, or -1 for an unsupported type/shape.
 */
int orc_gemv(int type, int path, const uint8_t* w, int64_t rows, int64_t cols,
             const float* x, const float* row_max_abs,
             float* y, int64_t* row_acc, int64_t* unit_acc);

/* Phase-B chain replay of one descriptor (phaseb_run_descriptor,
 * tmac_gguf.cpp:761-831) over an arena holding DDR bytes [base, base+bytes).
 * Returns the rows written to acc (0 for CPU_OP / unsupported types), or -1. */
int64_t orc_phaseb_run(const uint8_t* arena, uint32_t base, uint64_t bytes, uint32_t desc_off, int64_t* acc);

#ifdef __cplusplus
}
#endif
#endif /* TMAC_ORACLE_H */
