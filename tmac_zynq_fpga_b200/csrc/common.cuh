// common.cuh -- shared host/device helpers of libtmac_cuda.so (sm_100a only).
//
// Exactness rules for every kernel in this library (the reference's CPU code is
// the numerics spec):
//  * fp32/fp64 expressions are written with explicit round-to-nearest
//    intrinsics (__fmul_rn, __fadd_rn, __dmul_rn, ...) in the reference's
//    evaluation order, and the library is compiled with -fmad=false, so no FMA
//    contraction changes a rounding.
//  * roundf() is C99 round-half-away-from-zero, as in the reference.
//  * fp16 -> fp32 is exact (__half2float), matching fpga_sim::read_f16.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>

#include "../../include/tmac_cuda.h"

#define TMAC_DEV __device__ __forceinline__

namespace tmac {

// ---------------------------------------------------------------- errors --
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define TMAC_CUDA_TRY(expr)                                  \
    do {                                                     \
        cudaError_t _e = (expr);                             \
        if (_e != cudaSuccess) return tmac::cuda_fail(_e, #expr); \
    } while (0)

// Device-side error word (one per device, in this library's module).
int* device_error_word(int device);

// Switch to `device` for the lifetime of the guard.
struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev)
    {
        if (cudaGetDevice(&prev) != cudaSuccess) { ok = false; return; }
        if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
    }
    ~DeviceGuard()
    {
        int cur;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int num_sms(int device);

// ---------------------------------------------------------- device bits --
TMAC_DEV float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

TMAC_DEV uint16_t ld_u16_unaligned(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

TMAC_DEV int16_t clamp_round_i16(float v)
{
    if (v > 32767.0f) return 32767;
    if (v < -32768.0f) return -32768;
    return (int16_t)(int)roundf(v);
}

// dp4a with unsigned a-bytes and signed / unsigned b-bytes.
TMAC_DEV int dp4a_us(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
TMAC_DEV int dp4a_uu(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Block-wide max of non-negative floats (fmaxf is exact and order-free).
// `red` must hold one float per warp.  All threads get the result.
TMAC_DEV float block_max(float v, float* red, int nthreads)
{
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    float m = 0.0f;
    for (int i = 0; i < (nthreads + 31) / 32; i++) m = fmaxf(m, red[i]);
    __syncthreads();
    return m;
}

// Top-1 key of logit v at global index idx: the float's bits mapped to an
// unsigned order (negatives inverted, positives with the sign bit set) in bits
// 62..31, then 0x7FFFFFFF - idx, so the largest key is the largest logit and,
// among equal logits, the lowest index.  The key is non-negative as an int64,
// so an NCCL / torch int64 MAX all-reduce merges vocab shards.  0 = no key.
TMAC_DEV unsigned long long top1_key(float v, int64_t idx)
{
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 31) | (0x7FFFFFFFull - (unsigned long long)(idx & 0x7FFFFFFF));
}

// x_scale of tmac_gguf.cpp:889-892 from max|x|.
// Combined UQ8.8 scale, tmac_gguf.cpp:1022-1039.
TMAC_DEV uint32_t q8_combined(float d, float rs)
{
    float rinv = (rs < 1e-10f) ? 1.0f : __fdiv_rn(1.0f, rs);
    float c = __fmul_rn(d, rinv);
    if (c >= 256.0f) c = 255.996f;
    if (c < 0.0f) c = 0.0f;
    return (uint32_t)(uint16_t)__fadd_rn(__fmul_rn(c, 256.0f), 0.5f);
}

TMAC_DEV float x_scale_from_max(float mx) { return (mx < 1e-10f) ? 1.0f : __fdiv_rn(mx, 32767.0f); }
// x_q of tmac_gguf.cpp:894-896.
TMAC_DEV int16_t quantize_one(float x, float xs) { return (int16_t)(int)roundf(__fdiv_rn(x, xs)); }

// (float)(p / ri) with p / ri rounded to double first, as the GEMV computes it
// (__ddiv_rn then the float conversion).  p * RN(1/ri) is within 2 double ulps
// of the double quotient; unless its 29 bits below float precision lie within
// 16 units of the float rounding midpoint (or the value is outside the normal
// float range) both round to the same float, else the exact division decides.
TMAC_DEV float quotient_f32(double p, double rinv, float ri)
{
    const double q = __dmul_rn(p, rinv);
    const long long bits = __double_as_longlong(q);
    const int exp = (int)((bits >> 52) & 0x7FF);
    const int low = (int)(bits & 0x1FFFFFFF);
    const bool near_mid = abs(low - 0x10000000) <= 16;
    if (near_mid || exp < 1023 - 120 || exp > 1023 + 120) return (float)__ddiv_rn(p, (double)ri);
    return (float)q;
}

// ----------------------------------------------------- mbarrier / bulk copy
TMAC_DEV uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

TMAC_DEV void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
TMAC_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

TMAC_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// Adds to the transaction count of the current phase without arriving.
TMAC_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
TMAC_DEV void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
TMAC_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
TMAC_DEV uint64_t global_timer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
}  // namespace tmac

// Limit of every bounded device wait, in ns (tmac_set_wait_limit_ns).  Without
// relocatable device code each translation unit has its own copy, so every
// unit that includes this header registers a setter for its copy.
static __device__ unsigned long long g_tmac_wait_limit_ns = 2000000000ull;
static cudaError_t tmac_set_wait_limit_this_unit(unsigned long long ns)
{
    return cudaMemcpyToSymbol(g_tmac_wait_limit_ns, &ns, sizeof(ns));
}
namespace tmac {
int register_wait_limit_setter(cudaError_t (*set)(unsigned long long));  // registry.cu
}
static const int g_tmac_wait_limit_reg = tmac::register_wait_limit_setter(&tmac_set_wait_limit_this_unit);

namespace tmac {
TMAC_DEV unsigned long long wait_limit_ns() { return *(volatile const unsigned long long*)&g_tmac_wait_limit_ns; }
// Bounded wait: gives up after the wait limit (2 s unless set), records
// TMAC_ERR_TIMEOUT and returns false.
TMAC_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err)
{
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; it++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0 && global_timer_ns() - t0 > wait_limit_ns()) {
            if (err) atomicExch(err, (int)TMAC_ERR_TIMEOUT);
            return false;
        }
    }
}
// As mbar_wait_bounded, but every poll may suspend the thread until the
// phase completes or ~hint_ns pass, so a warp that waits long issues few
// instructions (the issue slots stay with the warps doing the work).
TMAC_DEV bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
TMAC_DEV bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* err)
{
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; it++) {
        if (mbar_try_wait_hint(bar, parity, 20000u)) return true;
        if ((it & 15u) == 0 && global_timer_ns() - t0 > wait_limit_ns()) {
            if (err) atomicExch(err, (int)TMAC_ERR_TIMEOUT);
            return false;
        }
    }
}
// 1-D bulk copy global -> shared (no multicast), completion on `bar`.
// dst, src 16-byte aligned, bytes a multiple of 16.
TMAC_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// Programmatic dependent launch.  pdl_wait: wait until the preceding grid in
// the stream has completed and its writes are visible -- a no-op for a kernel
// launched without the programmatic-serialisation attribute, so every kernel
// calls it before its first read of data another kernel produced, and writes
// nothing to global memory before it.  pdl_launch: let the next grid start
// its own prologue now.
TMAC_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
TMAC_DEV void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

TMAC_DEV void named_bar_sync(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Arrive without waiting (producer side of a named barrier some other warps sync on).
TMAC_DEV void named_bar_arrive(int id, int nthreads)
{
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Launches with programmatic stream serialisation while the calling thread has
// PDL enabled (the decode engine enables it around its graph capture).
extern thread_local bool g_pdl;
struct PdlScope {
    bool prev;
    PdlScope() : prev(g_pdl) { g_pdl = true; }
    ~PdlScope() { g_pdl = prev; }
};
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = g_pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace tmac

// ------------------------------------------------------- weight objects --
// Device-resident layouts (all chosen at registration; see each .cu file).
struct tmac_weight_s {
    int type = 0, mode = 0, device = 0;
    int64_t rows = 0, cols = 0;
    uint8_t* data = nullptr;     // layout-specific packed weights
    size_t data_bytes = 0;
    float* row_norm = nullptr;   // row_inv (NATIVE Q5_0/K-quants) or row_scale (Q8_0, INT16)
    int64_t groups = 0;          // row groups (interleaved layouts)
    int64_t group_bytes = 0;     // bytes per row group
    int tiles = 0;               // 64-column tiles per row (Q8_0 / INT16)
    int* exc_ptr = nullptr;      // NATIVE Q5_0/K-quants: per-row exception offsets [rows + 1]
    void* exc = nullptr;         // int4 (row, col, v - v', 0) entries
    int64_t n_exc = 0;
    void* gwh = nullptr;         // tensor-core GEMM: exact int16 weights as byte planes
    void* gwl = nullptr;         // (high, low), decoded on first tmac_gemm
    void* grinv = nullptr;       // double [rows]: RN(1 / row_inv) for the GEMM epilogue
    // Q8_0: running top-1 key (u64) and CTA count (u32) of the call in flight,
    // so a top-1 call needs no key reset (calls on one weight are serial).
    void* top1_scratch = nullptr;
};

namespace tmac {
// Per-path launchers (one per .cu file).  All return TMAC_OK or an error.
int register_q8_0(tmac_weight_s* w, const uint8_t* d_raw, const float* d_row_max_abs, cudaStream_t s);
struct XchgDev;  // xchg.cuh
// With xg, top1 is the global key: the last CTA merges this rank's shard key
// with every rank's over peer memory (batch 1 only, top1 not zeroed first).
int launch_q8_0(const tmac_weight_s* w, const float* x, float* y, int64_t* row_acc, int64_t* unit_acc,
                int batch, cudaStream_t s, unsigned long long* top1 = nullptr, int64_t index_base = 0,
                const int16_t* xq = nullptr, const float* xs = nullptr, const XchgDev* xg = nullptr);
int launch_quantize(const float* x, int64_t cols, int batch, int16_t* xq, float* xs, cudaStream_t s,
                    uint8_t* xp = nullptr);
int launch_top1(const float* y, int64_t n, int64_t index_base, unsigned long long* key, cudaStream_t s);
int register_blockq(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s);
// Activations: fp32 x, or int16 xq, or byte planes xp ([batch][2][cols]: high
// bytes, low bytes) with their x_scale xs.
// xmax_parts: with fp32 x at batch 1, max |x| is the maximum of these n_parts
// values (left by the producer kernel), so the CTAs skip that reduction.
int launch_blockq(const tmac_weight_s* w, const float* x, const int16_t* xq, const uint8_t* xp, const float* xs,
                  float* y, int64_t* row_acc, int64_t* unit_acc, int batch, cudaStream_t s,
                  const float* xmax_parts = nullptr, int n_parts = 0);
// The reference's exact int16 weights of a NATIVE Q5_0 / Q4_K / Q6_K weight as
// byte planes wh (signed high) / wl (low), [rows][cols] row-major.
int blockq_planes(const tmac_weight_s* w, int8_t* wh, uint8_t* wl, cudaStream_t s);
// Tensor-core GEMM (gemm_tc.cu): Y[m][rows] = the GEMV of each of m fp32 rows.
int gemm_prepare(tmac_weight_s* w, cudaStream_t s);
int launch_gemm(tmac_weight_s* w, const float* x, float* y, int64_t* acc_out, int M, cudaStream_t s);
// Batches tmac_gemv sends to the tensor cores (NATIVE Q5_0 / Q4_K / Q6_K).
constexpr int kTcMinBatch = 8, kTcMaxBatch = 64;
// Activation rows -> x_scale and byte planes (x_q = 256*xh + xl).
int quantize_rows(const float* x, int64_t K, int M, int8_t* xh, uint8_t* xl, float* xs, cudaStream_t s);
// One GEMM over byte planes: columns [k_off, k_off + K) of X [M][x_stride] and
// W [N][w_stride]; mode 0: y[m][n] = acc * xs[m] / row_param[n] (block-quant
// row_inv); mode 1: y[m][n] = (float)(y[m][n] + acc * xs[m] * row_param[n]) (one
// 64-column tile of the Q8_0 fold, row_param = row_scale).
struct GemmOperands {
    const uint8_t *xh = nullptr, *xl = nullptr;
    int64_t x_stride = 0;
    const float* xs = nullptr;
    int M = 0;
    const uint8_t *wh = nullptr, *wl = nullptr;
    int64_t w_stride = 0;
    int N = 0;
    int64_t K = 0, k_off = 0;
    const float* row_param = nullptr;
    const double* row_rinv = nullptr;  // mode 0: RN(1 / row_param) in double
    int mode = 0;
    float* y = nullptr;
    int64_t y_stride = 0;
    int64_t* acc_out = nullptr;
    int device = 0;
};
int gemm_planes(const GemmOperands& op, cudaStream_t s);
// Q8_0 weight (NATIVE layout) -> its int16 deq = (q * cs) >> 8 as byte planes
// [rows][cols] (gemv_q8_0.cu).
int q8_planes(const tmac_weight_s* w, int8_t* wh, uint8_t* wl, cudaStream_t s);
int register_int16(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s);
int launch_int16(const tmac_weight_s* w, const float* x, float* y, int64_t* row_acc, int64_t* unit_acc,
                 int batch, cudaStream_t s);
int register_f32(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s);
int launch_f32(const tmac_weight_s* w, const float* x, float* y, int batch, cudaStream_t s);
}  // namespace tmac
