/*
 * tmac_cuda.h -- C ABI of libtmac_cuda.so, the B200 (sm_100a) replacement for
 * the FPGA compute cores that liuwantao3/tmac-zynq-fpga drives from its host
 * engine (sim/tmac_gguf.cpp) and models in sim/fpga_sim.hpp.
 *
 * Plain C: opaque handles, plain pointers, sizes and int status codes.  No
 * CUDA runtime types appear here; streams are passed as `void*`
 * (a cudaStream_t, NULL = the legacy default stream).
 *
 * Numerics: every GEMV reproduces the reference's CPU result bit for bit
 * (int64 row / per-unit sums exact, fp32 outputs identical), including the
 * per-call activation quantisation x_q = (int16)roundf(x / x_scale),
 * x_scale = max|x| / 32767, of tmac_gguf.cpp:889-896.
 *
 * Threading: a weight handle belongs to the device it was registered on; calls
 * on it must use a stream of that device.  The library keeps one workspace per
 * device; calls from several host threads on one device must be serialised by
 * the caller (as the reference's single-threaded engine does).  The exception
 * is tmac_gemv_host, which holds a per-device lock for its whole call.
 *
 * Device state: addresses of the library's module variables (the device error
 * word, the tmac_gemv_static scratch) are looked up once per device and kept,
 * as are weights and workspaces.  None of it survives cudaDeviceReset or the
 * destruction of a device's primary context: free every handle first and do
 * not call the library on that device afterwards in the same process.
 */
#ifndef TMAC_CUDA_H
#define TMAC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TMAC_ABI_VERSION 1

/* GGUF tensor type codes (sim/tmac_gguf.cpp:151-156). */
enum tmac_type {
    TMAC_TYPE_F32 = 0,
    TMAC_TYPE_F16 = 1,
    TMAC_TYPE_Q5_0 = 6,
    TMAC_TYPE_Q8_0 = 8,
    TMAC_TYPE_Q4_K = 12,
    TMAC_TYPE_Q6_K = 14
};

/* Which reference driver a registered weight reproduces.
 *   NATIVE: the type's FPGA core path  -- matmul_fpga_q8 / _q5_0 / _q4_k /
 *           _q6_k (tmac_gguf.cpp:948, :1221, :1097, :1367)
 *   INT16:  matmul_fpga_int16 (tmac_gguf.cpp:887), the path a type takes
 *           when its --fpga-* switch is off while another switch is on
 *   F32:    the FP32 dequant path taken with no --fpga switch
 *           (tmac_gguf.cpp:488-492)                                       */
enum tmac_mode { TMAC_MODE_NATIVE = 0, TMAC_MODE_INT16 = 1, TMAC_MODE_F32 = 2 };

/* Status codes: 0 = success, negative = failure (message in tmac_last_error). */
enum tmac_status {
    TMAC_OK = 0,
    TMAC_ERR_INVALID = -1,   /* NULL handle/pointer, bad argument */
    TMAC_ERR_TYPE = -2,      /* type/mode combination not supported */
    TMAC_ERR_SHAPE = -3,     /* rows/cols/batch not supported */
    TMAC_ERR_BOUNDS = -4,    /* descriptor/arena offset or size out of range */
    TMAC_ERR_CUDA = -5,      /* CUDA runtime error */
    TMAC_ERR_NCCL = -6,      /* NCCL error */
    TMAC_ERR_TIMEOUT = -7,   /* a bounded device wait gave up */
    TMAC_ERR_NOMEM = -8,     /* device allocation failed */
    TMAC_ERR_NODEV = -9      /* no CUDA device / wrong architecture */
};

typedef struct tmac_weight_s* tmac_weight_t;

/* Library identity and diagnostics. */
int tmac_abi_version(void);
/* Message of the last failing call on this host thread ("" if none). */
const char* tmac_last_error(void);
/* Reads and clears the device-side error word of `device` (synchronises that
 * device).  *code receives 0 or the TMAC_ERR_* a kernel recorded. */
int tmac_device_error(int device, int* code);
/* Programmatic dependent launch for the kernels this host thread launches
 * from now on (default off; returns the previous setting).  When on, a
 * kernel may start while the preceding kernel on the stream finishes: it
 * sets up and streams its weights, and waits for the predecessor before it
 * reads activations or writes outputs, so results are unchanged.  Consecutive
 * GEMVs then overlap one launch's ramp-up with the other's tail. */
int tmac_set_pdl(int on);
/* Limit of every bounded device wait (bulk-copy barriers, the peer exchange) on
 * `device`, in ns; default 2 s.  After the limit a kernel records
 * TMAC_ERR_TIMEOUT (tmac_device_error), waits -- within the limit again -- for
 * the copies it has in flight, and returns without its results.  The
 * counterpart of MatmulAccel::wait_done's timeout (sim/fpga_sim.hpp:232-241) and
 * the hardware chain watchdog.  Synchronous; not during stream capture. */
int tmac_set_wait_limit_ns(int device, uint64_t ns);

/*
 * Register one weight tensor: W[rows][cols] as raw GGUF blocks (the bytes a
 * `.tmac` file / Tensor::data hold, row r = blocks r*(cols/QK) ...).
 * Replaces: Tensor registration by load_tmac (tmac_gguf.cpp:1894-1947) plus
 * the per-call weight-only work of the matmul_fpga_* drivers (row_inv /
 * row_scale passes, Q8_0 combined scales), which is done once here.
 *   blocks:        host pointer (copied) or, if blocks_on_device != 0, a
 *                  device pointer on `device` (read during the call only).
 *   row_max_abs:   optional host float[rows] for Q8_0 NATIVE
 *                  (the `*_row_max_abs` tensor, sim/matmul_q8.cpp:22-35).
 * The handle owns its device memory until tmac_weight_free.
 */
int tmac_weight_register(int type, int mode, int64_t rows, int64_t cols,
                         const void* blocks, size_t n_bytes, int blocks_on_device,
                         const float* row_max_abs, int device, tmac_weight_t* out);
int tmac_weight_free(tmac_weight_t w);
int tmac_weight_info(tmac_weight_t w, int* type, int* mode, int64_t* rows, int64_t* cols,
                     int* device);
/* Device bytes the kernels stream per GEMV (the resident layout). */
int tmac_weight_device_bytes(tmac_weight_t w, size_t* bytes);
/* Host copy of the per-row normaliser: row_inv (Q5_0/Q4_K/Q6_K NATIVE) or
 * row_scale (Q8_0 NATIVE, INT16).  out: float[rows]. */
int tmac_weight_row_norm(tmac_weight_t w, float* out);

/* Partial-sum units per row: Q8_0 NATIVE and INT16 -> 64-column tiles,
 * Q5_0 -> 32-column blocks, Q4_K/Q6_K -> 256-column blocks; F32 -> 0. */
int64_t tmac_units_per_row(int type, int mode, int64_t cols);

/*
 * GEMV on device buffers: y[b][rows] = W . x[b][cols] for b < batch, each
 * activation vector quantised with its own x_scale (as `batch` sequential
 * calls of the reference driver would).  Replaces matmul_fpga_q8/_q5_0/_q4_k/
 * _q6_k/_int16 and the FP32 matmul() branch (tmac_gguf.cpp:466-493).
 *   x, y:      device pointers on the weight's device.
 *   row_acc:   optional int64[batch][rows] device buffer: the exact integer
 *              row accumulator (NATIVE/INT16 modes).
 *   unit_acc:  optional int64[batch][rows][units] device buffer: per-unit
 *              partial sums (see tmac_units_per_row).
 *   stream:    cudaStream_t of the weight's device (NULL = default stream).
 * Asynchronous: returns after enqueueing.
 * NATIVE Q5_0 / Q4_K / Q6_K with 8 <= batch <= 64, no unit_acc and cols a
 * multiple of 16 run on the tensor cores (the split-K path of tmac_gemm), with
 * the same results bit for bit.  The first such call on a weight decodes its
 * int16 planes (2 bytes per weight, kept with the weight) and may grow the
 * per-device workspaces, so before CUDA-graph capture make one call per weight
 * at the largest batch the graph uses.  Calls on one device share the
 * workspaces: order them on one stream.
 */
int tmac_gemv(tmac_weight_t w, const float* x, float* y, int batch, void* stream);
int tmac_gemv_acc(tmac_weight_t w, const float* x, float* y, int64_t* row_acc, int64_t* unit_acc,
                  int batch, void* stream);

/* Type-checked entry points with the per-type names of the reference drivers
 * (tmac_gguf.cpp:466-470): they fail with TMAC_ERR_TYPE if `w` has another
 * type or mode. */
int tmac_gemv_q8_0(tmac_weight_t w, const float* x, float* y, int batch, void* stream);
int tmac_gemv_q5_0(tmac_weight_t w, const float* x, float* y, int batch, void* stream);
int tmac_gemv_q4_k(tmac_weight_t w, const float* x, float* y, int batch, void* stream);
int tmac_gemv_q6_k(tmac_weight_t w, const float* x, float* y, int batch, void* stream);
int tmac_gemv_int16(tmac_weight_t w, const float* x, float* y, int batch, void* stream);

/*
 * Host-buffer GEMV: copies x[batch][cols] host->device, runs tmac_gemv on the
 * weight's device and copies y[batch][rows] back; synchronous.  This is the
 * drop-in for the reference's `void matmul_fpga_X(const Tensor*, const float*
 * x, float* y, int rows, int cols)` calls on host arrays.  For a NATIVE Q8_0
 * weight and a page-locked y (cudaHostAlloc / cudaHostRegister) the kernel
 * stores y straight into host memory, overlapping the transfer with the GEMV.
 */
int tmac_gemv_host(tmac_weight_t w, const float* x_host, float* y_host, int batch);

/*
 * Greedy top-1 over logits: the largest y and, among equal values, the lowest
 * index, packed as a 63-bit key (order-preserving float bits << 31 |
 * 0x7FFFFFFF - index) so that vocab shards on several GPUs merge with one
 * int64 MAX all-reduce.  Stands in for sample_token / the top-10 print of the
 * reference (tmac_gguf.cpp:1974-1990, :2164-2172) in greedy decoding.
 *   tmac_top1:      max-merges the key of y[0..n) (indices + index_base) into
 *                   *key (device); zero *key first for a fresh result.
 *   tmac_gemv_top1: y = W.x and key[b] = top-1 of y[b] (the key's old value
 *                   does not matter).  For Q8_0 the top-1 is fused into the
 *                   GEMV kernel: its CTAs merge into a running key kept with
 *                   the weight and the last CTA writes key[b], so the call is
 *                   one launch per batch row; top-1 calls on one weight must
 *                   not run concurrently.
 *   tmac_top1_decode: host-side unpacking of a key.
 */
int tmac_top1(const float* y, int64_t n, int64_t index_base, uint64_t* key, void* stream);
int tmac_gemv_top1(tmac_weight_t w, const float* x, float* y, uint64_t* key, int64_t index_base, int batch,
                   void* stream);
int tmac_top1_decode(uint64_t key, float* value, int64_t* index);

/*
 * Activation quantisation done once (tmac_gguf.cpp:889-896): x_scale[b] =
 * max|x[b]|/32767 (1 if below 1e-10), xq[b][j] = (int16)roundf(x[b][j]/x_scale[b]).
 * tmac_gemv_xq then runs a NATIVE-mode GEMV on it; the result equals tmac_gemv
 * on x bit for bit (every reference driver quantises its x the same way), so
 * GEMVs sharing one activation vector (q/k/v, gate/up) quantise it once.
 * cols must be a multiple of 8; device pointers; asynchronous.
 */
int tmac_quantize_x(const float* x, int64_t cols, int batch, int16_t* xq, float* xs, void* stream);
int tmac_gemv_xq(tmac_weight_t w, const int16_t* xq, const float* xs, float* y, int batch, void* stream);

/* Allocate the per-device workspace for GEMVs up to batch x cols now, so that
 * later calls allocate nothing (required before CUDA-graph capture).
 * tmac_gemv on a NATIVE Q5_0 / Q4_K / Q6_K weight with batch > 2 quantises x
 * once into this workspace (x_q as byte planes, x_scale [batch]) and grows it
 * with cudaMalloc when a call needs more; calls on one device share it, so they
 * must be ordered on one stream.  Batch 1-2 quantises inside the GEMV. */
int tmac_reserve(int device, int64_t max_batch, int64_t max_cols);

/* Batched matmul on the tensor cores (prefill: m activation rows at once; the
 * reference runs matmul_fpga_q5_0 / _q4_k / _q6_k once per token,
 * sim/tmac_gguf.cpp:1992-2023).  y[m][rows] equals tmac_gemv with batch m bit
 * for bit: every row is quantised like one GEMV call, the products are the
 * reference's exact int16 weights times x_q (tcgen05 int8 MMAs on byte planes),
 * row_acc (optional, int64 [m][rows]) the integer row sums.  NATIVE Q5_0 /
 * Q4_K / Q6_K weights, and NATIVE Q8_0 (matmul_fpga_q8 per row: one GEMM per
 * 64-column tile, folded into y in tile order; row_acc must be NULL); cols a
 * multiple of 16, at most 32768.  The first call on a weight decodes its int16
 * planes (2 bytes per weight, kept with the weight).  For m <= 64 (Q5_0 / Q4_K /
 * Q6_K) the weights are the 128-row MMA operand and K is split across the SMs,
 * with int64 partial sums in a per-device workspace that the call leaves zeroed;
 * calls on one device must then be ordered on one stream.  Device pointers;
 * asynchronous on `stream`. */
int tmac_gemm(tmac_weight_t w, const float* x, float* y, int64_t* row_acc, int m, void* stream);

/* Measurement aid (no reference counterpart): dense int8 tensor-core rate of
 * `device` in TOPS (2 ops per multiply-accumulate), from `iters` x 4
 * back-to-back tcgen05.mma kind::i8 (M 128, N 256, K 32) per SM with operands
 * resident in shared memory; one launch timed with CUDA events.  The roofline
 * denominator of tmac_gemm / tmac_model_prefill.  Synchronous. */
int tmac_probe_mma_i8(int device, int iters, double* tops);

/* NATIVE Q5_0 / Q4_K / Q6_K GEMV that allocates nothing.  No counterpart in
 * the reference (its drivers are host code with no device memory to manage);
 * it is for callers that may not allocate device memory, e.g. code running
 * inside a caller-owned memory pool or a real-time loop that forbids
 * cudaMalloc.  x is quantised into a fixed module-scope scratch of
 * TMAC_STATIC_MAX_VALUES int16 values and TMAC_STATIC_MAX_BATCH scales per
 * device; batch x cols above that fails with TMAC_ERR_SHAPE (use tmac_gemv).
 * Results equal tmac_gemv bit for bit.  The scratch address is resolved on a
 * device's first call, so make that first call before any stream capture.
 * All calls on one device share the scratch: calls that overlap (different
 * streams or threads without ordering) race and give wrong results. */
#define TMAC_STATIC_MAX_VALUES 131072 /* 256 KiB of int16 x_q */
#define TMAC_STATIC_MAX_BATCH 64
int tmac_gemv_static(tmac_weight_t w, const float* x, float* y, int batch, void* stream);

/* ------------------------------------------------------------------------ */
/* Top-1 merge of vocab-sharded logits over NVLink peer memory (multi-GPU
 * greedy step; the reference samples from the whole logits vector on one
 * host, sim/tmac_gguf.cpp:1974-1990).  One exchange object per rank (one
 * process per GPU): create it, pass every rank's IPC handle to every rank
 * (e.g. an all-gather on the host), open, then per step tmac_xchg_top1 turns
 * this rank's shard key (device uint64, from tmac_gemv_top1) into the global
 * maximum key on every rank.  The kernel stores the key into every rank's
 * buffer and waits for all ranks' keys of the same step (bounded by
 * tmac_set_wait_limit_ns: after the limit it records TMAC_ERR_TIMEOUT, read
 * with tmac_device_error, and leaves the key; the ranks' step counts then
 * differ, so free and re-create the exchange on every rank before going on).
 * Ranks in one process (threads) open each other's handles too: the buffer is
 * then reached by its device address instead of an IPC mapping.
 * All ranks must call tmac_xchg_top1 the same number of times. */
typedef struct tmac_xchg_s* tmac_xchg_t;
#define TMAC_XCHG_HANDLE_BYTES 64
int tmac_xchg_create(int device, int world, int rank, tmac_xchg_t* out);
int tmac_xchg_ipc_handle(tmac_xchg_t x, void* handle);           /* TMAC_XCHG_HANDLE_BYTES bytes */
int tmac_xchg_open(tmac_xchg_t x, const void* handles);          /* world x TMAC_XCHG_HANDLE_BYTES */
int tmac_xchg_top1(tmac_xchg_t x, uint64_t* key, void* stream);
/* The logits step of one rank in one launch: y = W.in (batch 1) over this
 * rank's vocab shard (rows index_base ..), and *key = the maximum top-1 key
 * over every rank's shard.  For a Q8_0 weight the exchange runs inside the
 * GEMV (its last CTA publishes the shard key to every rank and waits for
 * theirs), so no key reset or second launch is needed; other weights take
 * tmac_gemv_top1 followed by tmac_xchg_top1.  Shares the step count with
 * tmac_xchg_top1, so the two may be mixed as long as every rank makes the
 * same sequence of calls. */
int tmac_xchg_gemv_top1(tmac_xchg_t x, tmac_weight_t w, const float* in, float* y, uint64_t* key,
                        int64_t index_base, void* stream);
/* The same exchange with the full logits on every rank (get_logits_q8 returns
 * the whole vector, sim/tmac_gguf.cpp:1820-1845): created with the vocabulary
 * size, each rank's buffer also holds two full-logits vectors (by step
 * parity), and tmac_xchg_gemv_top1 on a NATIVE Q8_0 shard stores every row it
 * computes into all ranks' vectors over NVLink peer memory, inside the same
 * launch, before the step's key is published.  tmac_xchg_logits gives the
 * device address of this rank's full vector for the last step enqueued; read
 * it (stream-ordered) before the next exchange call on that stream, which lets
 * the other ranks write the next step. */
int tmac_xchg_create_logits(int device, int world, int rank, int64_t vocab, tmac_xchg_t* out);
int tmac_xchg_logits(tmac_xchg_t x, float** logits);
int tmac_xchg_free(tmac_xchg_t x);

/* ------------------------------------------------------------------------ */
/* Phase-B descriptor chain (sim/fpga_sim.hpp:1254-1310, sim/tmac_gguf.cpp:513-880).
 *
 * A chain is a linked list of 32-byte descriptors inside a byte arena that
 * stands for the FPGA's DDR: every address field is an absolute DDR offset,
 * and the arena holds DDR bytes [arena_base, arena_base + arena_bytes).
 * The descriptor layout is the reference's PhaseBDescriptor, byte for byte. */
#define TMAC_DESC_TYPE_INT16 0
#define TMAC_DESC_TYPE_Q5_0 6
#define TMAC_DESC_TYPE_Q8_0 8
#define TMAC_DESC_TYPE_Q4_K 12
#define TMAC_DESC_TYPE_Q6_K 14
#define TMAC_DESC_TYPE_CPU_OP 15
#define TMAC_DESC_FLAG_INTERRUPT 0x01
/* Tile sizes (blocks + scale section) of the reference's Phase-B packing. */
#define TMAC_PHASEB_Q5_0_TILE_BYTES 4944 /* 8 rows x 896: 224 x 22 B + 8 x UQ16.8 */
#define TMAC_PHASEB_Q6_K_TILE_BYTES 6848 /* 32 rows x 256: 32 x 210 B + 32 x UQ24.8 */
#define TMAC_PHASEB_Q4_K_TILE_BYTES 8288 /* 56 rows x 256: 56 x 144 B + 56 x UQ24.8 */

#pragma pack(push, 1)
typedef struct tmac_phaseb_desc {
    uint32_t next_desc_addr;  /* 0x00, 0 = end of chain */
    uint32_t weight_addr;     /* 0x04 */
    uint32_t act_addr;        /* 0x08, int16 activations */
    uint32_t result_addr;     /* 0x0C, int64 per result row */
    uint16_t num_tiles;       /* 0x10 */
    uint16_t tile_bytes;      /* 0x12 */
    uint8_t tensor_type;      /* 0x14, TMAC_DESC_TYPE_* */
    uint8_t tile_res_rows;    /* 0x15 */
    uint8_t flags;            /* 0x16 */
    uint16_t act_total_bytes; /* 0x17 */
    uint8_t num_col_groups;   /* 0x19 */
    uint8_t reserved[6];      /* 0x1A */
} tmac_phaseb_desc;
#pragma pack(pop)

typedef struct tmac_chain_stats {
    int descriptors;      /* descriptors walked */
    int unsupported;      /* descriptors of a type the reference runner skips (0 rows) */
    int64_t result_rows;  /* int64 results written */
} tmac_chain_stats;

/*
 * Replays a descriptor chain on the GPU: the replacement for phaseb_run_descriptor
 * over the chain walked by phaseb_verify (tmac_gguf.cpp:761-831, :834-880).  For
 * each descriptor the int64 accumulators are computed exactly as the reference
 * runner does (Q5_0: row_inv recomputed from the tile's blocks; Q4_K / Q6_K:
 * row_inv = UQ24.8 scale section / 256; CPU_OP: no rows; other types: skipped,
 * 0 rows, as in the reference) and written at result_addr inside the arena.
 *   arena_dev:   device copy of the DDR bytes [arena_base, arena_base + arena_bytes).
 *   arena_host:  optional host mirror of the same bytes, used to walk the chain
 *                without reading descriptors back from the device; NULL = read them.
 *   head:        DDR offset of the first descriptor.
 *   max_desc:    walk limit (a cycle in next_desc_addr is reported, not followed).
 * Every offset and size is checked against the arena before any launch
 * (TMAC_ERR_BOUNDS).  Asynchronous on `stream` once the walk is done.
 */
int tmac_chain_run(void* arena_dev, size_t arena_bytes, uint32_t arena_base, const void* arena_host,
                   uint32_t head, int max_desc, tmac_chain_stats* stats, void* stream);

/*
 * Hardware-format descriptor chain: the 32-byte descriptor the FPGA's HP FSM
 * walks (vivado_integration/sw/tmac_baremetal.h:100-113, API.md "Descriptor
 * Format"), a different layout from tmac_phaseb_desc above.
 *   type 1 (Q5_0):  num_tiles (0 counts as 1) tiles of TMAC_HW_Q5_0_TILE_BYTES
 *                   at weight_addr + i * 2696, each 4 rows x 896 columns as 56
 *                   48-byte two-core blocks (bytes 0-21 core 0's GGUF block,
 *                   22-43 core 1's, 44-47 zero; blocks 0-27 hold rows 0 / 2 of
 *                   the tile, 28-55 rows 1 / 3) and four UQ8.8 norms at 2688.
 *                   Activations: 896 int16 at act_addr (act_total_bytes >= 1792),
 *                   read once for every tile.  Results: int64 per row,
 *                   consecutive from result_addr (32 bytes per tile).
 *   type 15 (CPU_OP): the FSM's passthrough mode -- act_total_bytes bytes copied
 *                   from act_addr to result_addr (the interrupt mode, where the
 *                   host runs an operation, is the caller's own code).
 *   type 0 (Q8_0):  skipped and counted as unsupported: no CPU model of its
 *                   fixed-point tile exists in the reference.
 * Numerics of a Q5_0 tile: the reference's HP-FSM core model
 * axi_vecmul_tile_q5_0_4x896_axilite (sim/fpga_sim.hpp:1194-1249) with float
 * row norms recomputed from the tile's blocks (32767 / max|d*q|, as
 * q5_preprocess_tile computes them, tmac_baremetal.cpp:497-516); the UQ8.8 norm
 * section overflows for typical rows and is not read.  The int64 row sums are
 * those of matmul_fpga_q5_0 on the same rows.
 * Arena, walk limit, bounds checks, stats and stream as tmac_chain_run. */
#define TMAC_HW_DESC_Q8_0 0
#define TMAC_HW_DESC_Q5_0 1
#define TMAC_HW_DESC_CPU_OP 15
#define TMAC_HW_Q5_0_TILE_BYTES 2696 /* 56 x 48 B blocks + 4 x UQ8.8 norms */

#pragma pack(push, 1)
typedef struct tmac_hw_desc {
    uint32_t next_addr;          /* 0x00, 0 = end of chain */
    uint32_t weight_addr;        /* 0x04 */
    uint32_t act_addr;           /* 0x08 */
    uint32_t result_addr;        /* 0x0C */
    uint16_t tensor_type;        /* 0x10, TMAC_HW_DESC_* */
    uint16_t reserved0;          /* 0x12 */
    uint8_t num_groups;          /* 0x14, Q8_0 column groups in bits 3..0 */
    uint8_t reserved1;           /* 0x15 */
    uint16_t num_tiles;          /* 0x16 */
    uint8_t act_total_bytes[3];  /* 0x18, 24-bit little-endian */
    uint8_t reserved3[5];        /* 0x1B */
} tmac_hw_desc;
#pragma pack(pop)

int tmac_chain_run_hw(void* arena_dev, size_t arena_bytes, uint32_t arena_base, const void* arena_host,
                      uint32_t head, int max_desc, tmac_chain_stats* stats, void* stream);

/*
 * Phase-B dump for the Verilog testbench: the files the reference's
 * --dump-phaseb writes (phaseb_dump_files, tmac_gguf.cpp:597-708), with the
 * expected rows computed on the GPU (tmac_chain_run, one descriptor at a time).
 *   bin_path: DDR bytes [bin_base, desc_base + 32 * ndesc) of the arena with the
 *             chain's descriptors copied in chain order to desc_base and every
 *             next_desc_addr but the last set to 0xFFFFFFFF (the reference uses
 *             bin_base = 0x18000000 and desc_base = its allocator's next free
 *             offset rounded up to 32).
 *   hdr_path: uint32 magic 0x50484244 ("PHBD"), ndesc, desc_base, total rows;
 *             per descriptor uint32 {result_addr, rows, act_total_bytes,
 *             previous descriptor's result_addr, offset of its rows}; then the
 *             int64 rows of every descriptor in chain order.
 * arena_host holds DDR [arena_base, arena_base + arena_bytes) and must reach past
 * the copied descriptors; it is not modified.  Synchronous; uses `device`.
 */
int tmac_phaseb_dump(const void* arena_host, size_t arena_bytes, uint32_t arena_base, uint32_t head,
                     uint32_t desc_base, uint32_t bin_base, const char* bin_path, const char* hdr_path, int device);

/* ------------------------------------------------------------------------ */
/* Whole-model greedy decode (Qwen2-0.5B shape: 24 layers, hidden 896, 14/2
 * heads of 64, SwiGLU 4864, vocab 151936, tied Q8_0 embedding), replacing the
 * reference engine's process_prompt / generate loop (sim/tmac_gguf.cpp:1992-2047,
 * forward_layer_with_cache :1559-1711, get_logits_q8 :1820-1845) with the top-k
 * sampler replaced by greedy top-1 (lowest index on ties).
 * switches: the reference's --fpga-* flags (tmac_gguf.cpp:2084-2091) as bits;
 * a matrix whose type switch is off runs the INT16 path when TMAC_SW_FPGA is
 * set, and everything runs the FP32 path when it is not (matmul(), :473-493). */
#define TMAC_SW_FPGA 1  /* --fpga / --fpga-int16 (implied by every type switch) */
#define TMAC_SW_Q8 2    /* --fpga-q8   */
#define TMAC_SW_Q5_0 4  /* --fpga-q5-0 */
#define TMAC_SW_Q4_K 8  /* --fpga-q4k  */
#define TMAC_SW_Q6_K 16 /* --fpga-q6-k */
#define TMAC_SW_ALL 31  /* all four type switches */

typedef struct tmac_model_s* tmac_model_t;

/* Empty model on `device` with a KV cache of max_seq positions. */
int tmac_model_create(int device, int switches, int max_seq, tmac_model_t* out);
/* Adds one tensor by its GGUF name (copied): the records load_tmac reads. */
int tmac_model_add_tensor(tmac_model_t m, const char* name, int64_t rows, int64_t cols, int type, const void* data,
                          size_t n_bytes);
/* Reads every tensor of a `.tmac` file (load_tmac, tmac_gguf.cpp:1894-1947). */
int tmac_model_load_tmac(tmac_model_t m, const char* path);
/* Registers all matrices on the device and allocates the decode state. */
int tmac_model_finalize(tmac_model_t m);
/* Clears the KV cache (reset_cache, :1950-1956). */
int tmac_model_reset(tmac_model_t m, void* stream);
/* One token through all layers at `pos` (process_embedding + forward_all_layers).
 * token < 0 takes the token from the model's device top-1 key (the last
 * tmac_model_logits), so greedy steps chain without a host round trip. */
int tmac_model_forward(tmac_model_t m, int token, int pos, void* stream);
/* output_norm + logits GEMV of the current hidden state + greedy top-1 key. */
int tmac_model_logits(tmac_model_t m, void* stream);
/* Device addresses of the hidden state [896], logits [151936] and the key. */
int tmac_model_buffers(tmac_model_t m, float** hidden, float** logits, uint64_t** key);
/* Prompt + n_gen greedy steps on the model's own stream, each step replayed
 * from a CUDA graph captured on first use (`stream` is not used; the call
 * returns when done).  out_tokens[n_gen] (host); out_hidden optional
 * host float[(n_gen + 1) * 896]: after the prompt and after each step. */
int tmac_model_generate(tmac_model_t m, const int* prompt, int n_prompt, int n_gen, int* out_tokens,
                        float* out_hidden, void* stream);
/* Which engine tmac_model_generate ran: 1 = the persistent kernel (one
 * cooperative launch per token, every matrix on its FPGA-core path), 0 = the
 * per-kernel engine (CUDA graphs; other switch settings, or TMAC_DECODE=graph in
 * the environment), -1 = not decided yet (no generate call so far).  Both give
 * identical results. */
int tmac_model_decode_engine(tmac_model_t m);
/* Batched prefill (no reference counterpart: the reference feeds a prompt one
 * token at a time, process_prompt, sim/tmac_gguf.cpp:1992-2023).  n_seq
 * independent sequences of len tokens (host ids, [n_seq][len]) run through all
 * layers at once with every projection on the tensor cores (tmac_gemm).  Each
 * position's final hidden state equals what the decode engine computes after
 * feeding that sequence's tokens up to it, bit for bit.  next_tokens (host
 * [n_seq], optional) gets each sequence's greedy next token; hidden_out (host
 * [n_seq][len][896], optional) every position's hidden state before
 * output_norm.  Needs every matrix on its FPGA-core path (TMAC_SW_ALL) and
 * len <= max_seq.  Synchronous. */
int tmac_model_prefill(tmac_model_t m, const int* tokens, int n_seq, int len, int* next_tokens, float* hidden_out,
                       void* stream);
int tmac_model_free(tmac_model_t m);

#ifdef __cplusplus
}
#endif
#endif /* TMAC_CUDA_H */
