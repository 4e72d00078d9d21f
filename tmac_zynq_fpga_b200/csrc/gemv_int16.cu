// gemv_int16.cu -- the INT16 fallback path and the FP32 path.
//
// INT16 reproduces matmul_fpga_int16 (sim/tmac_gguf.cpp:887-941) with the
// axi_vecmul_tile_int16 core (sim/fpga_sim.hpp:437-446): the reference runs it
// for any tensor whose type switch is off while --fpga* is on (:483-485).
//   W_f32     = read_tensor(A, r, j)                    (FP32 dequant)
//   row_scale = max_j |W_f32| / 32767   (1 if max < 1e-10)
//   W_q       = (int16)roundf(W_f32 / row_scale)         -- weight-only: done once here
//   acc_t     = sum over a 64-column tile of W_q * x_q   (int64)
//   y         = (float)((double)y + (double)acc_t * x_scale * row_scale), tiles in order
// Device layout: rows in groups of 32, [group][tile][8 chunks][32 lanes][8 x int16],
// so a warp (lane = row) reads 512 contiguous bytes per chunk.
//
// FP32 reproduces matmul() with no --fpga switch (tmac_gguf.cpp:488-492):
//   y[i] = sum_j read_tensor(A,i,j) * x[j], a sequential fp32 sum per row.
// One thread per row walks its row in order over the raw GGUF blocks.
#include "common.cuh"
#include "dequant.cuh"

#include <algorithm>

namespace tmac {
namespace {

constexpr int kThreads = 256;

__global__ void int16_row_scale_kernel(int type, const uint8_t* __restrict__ raw, int64_t rows, int64_t cols,
                                       float* __restrict__ rs)
{
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float m = 0.0f;
    for (int64_t j = lane; j < cols; j += 32) m = fmaxf(m, fabsf(dequant_element(type, raw, cols, r, j)));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) rs[r] = (m < 1e-10f) ? 1.0f : __fdiv_rn(m, 32767.0f);
}

// grid (T*8, groups), 32 threads: one 16-byte chunk (8 columns) per lane/row.
__global__ void int16_pack_kernel(int type, const uint8_t* __restrict__ raw, int64_t rows, int64_t cols,
                                  const float* __restrict__ rs, int T, uint8_t* __restrict__ out)
{
    const int64_t g = blockIdx.y;
    const int c8 = blockIdx.x, l = threadIdx.x;
    const int64_t r = g * 32 + l;
    int16_t v[8];
    const float s = (r < rows) ? rs[r] : 1.0f;
    for (int k = 0; k < 8; k++) {
        const int64_t c = (int64_t)c8 * 8 + k;
        v[k] = (r < rows && c < cols) ? (int16_t)(int)roundf(__fdiv_rn(dequant_element(type, raw, cols, r, c), s))
                                      : (int16_t)0;
    }
    uint4 u;
    memcpy(&u, v, 16);
    reinterpret_cast<uint4*>(out)[(g * T * 8 + c8) * 32 + l] = u;
}

struct Int16Args {
    const uint8_t* packed;
    const float* rs;
    int64_t rows, cols, groups;
    int T;
    const float* x;
    float* y;
    int64_t* row_acc;
    int64_t* unit_acc;
    int batch;
};

__global__ void __launch_bounds__(kThreads) int16_gemv_kernel(Int16Args a)
{
    extern __shared__ __align__(16) uint8_t smem[];
    int16_t* xq = reinterpret_cast<int16_t*>(smem);  // [T*64]
    float* red = reinterpret_cast<float*>(smem + (size_t)a.T * 128);
    const int T = a.T;
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    for (int b = 0; b < a.batch; b++) {
        const float* xb = a.x + (int64_t)b * a.cols;
        float mx = 0.0f;
        for (int64_t j = threadIdx.x; j < a.cols; j += kThreads) mx = fmaxf(mx, fabsf(xb[j]));
        mx = block_max(mx, red, kThreads);
        const float xs = x_scale_from_max(mx);
        for (int64_t j = threadIdx.x; j < (int64_t)T * 64; j += kThreads)
            xq[j] = (j < a.cols) ? quantize_one(xb[j], xs) : (int16_t)0;
        __syncthreads();
        for (int64_t g = (int64_t)blockIdx.x * 8 + wib; g < a.groups; g += (int64_t)gridDim.x * 8) {
            const int64_t r = g * 32 + lane;
            const uint4* wp = reinterpret_cast<const uint4*>(a.packed) + g * T * 8 * 32 + lane;
            const float rsv = (r < a.rows) ? __ldg(a.rs + r) : 1.0f;
            float yr = 0.0f;
            long long rsum = 0;
            for (int t = 0; t < T; t++) {
                long long acc = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const uint4 wv = __ldg(wp + (t * 8 + j) * 32);
                    const uint4 xv = reinterpret_cast<const uint4*>(xq)[t * 8 + j];
                    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xx[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int p0 = (int)(int16_t)(ww[k] & 0xFFFF) * (int)(int16_t)(xx[k] & 0xFFFF);
                        const int p1 = (int)(int16_t)(ww[k] >> 16) * (int)(int16_t)(xx[k] >> 16);
                        acc += (long long)p0 + (long long)p1;
                    }
                }
                rsum += acc;
                yr = (float)__dadd_rn((double)yr, __dmul_rn(__dmul_rn((double)acc, (double)xs), (double)rsv));
                if (a.unit_acc && r < a.rows) a.unit_acc[((int64_t)b * a.rows + r) * T + t] = acc;
            }
            if (r < a.rows) {
                a.y[(int64_t)b * a.rows + r] = yr;
                if (a.row_acc) a.row_acc[(int64_t)b * a.rows + r] = rsum;
            }
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kThreads) f32_gemv_kernel(int type, const uint8_t* __restrict__ raw, int64_t rows,
                                                            int64_t cols, const float* __restrict__ x,
                                                            float* __restrict__ y)
{
    const int64_t r = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (r >= rows) return;
    float sum = 0.0f;
    for (int64_t j = 0; j < cols; j++)
        sum = __fadd_rn(sum, __fmul_rn(dequant_element(type, raw, cols, r, j), __ldg(x + j)));
    y[r] = sum;
}

}  // namespace

int register_int16(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s)
{
    const int T = (int)((w->cols + 63) / 64);
    w->tiles = T;
    w->groups = (w->rows + 31) / 32;
    w->group_bytes = (int64_t)T * 4096;
    w->data_bytes = (size_t)(w->groups * w->group_bytes);
    TMAC_CUDA_TRY(cudaMalloc(&w->row_norm, (size_t)w->rows * sizeof(float)));
    TMAC_CUDA_TRY(cudaMalloc(&w->data, w->data_bytes));
    int16_row_scale_kernel<<<(unsigned)((w->rows + 7) / 8), 256, 0, s>>>(w->type, d_raw, w->rows, w->cols,
                                                                         w->row_norm);
    TMAC_CUDA_TRY(cudaGetLastError());
    dim3 grid(T * 8, (unsigned)w->groups);
    int16_pack_kernel<<<grid, 32, 0, s>>>(w->type, d_raw, w->rows, w->cols, w->row_norm, T, w->data);
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int launch_int16(const tmac_weight_s* w, const float* x, float* y, int64_t* row_acc, int64_t* unit_acc, int batch,
                 cudaStream_t s)
{
    Int16Args a;
    a.packed = w->data;
    a.rs = w->row_norm;
    a.rows = w->rows;
    a.cols = w->cols;
    a.groups = w->groups;
    a.T = w->tiles;
    a.x = x;
    a.y = y;
    a.row_acc = row_acc;
    a.unit_acc = unit_acc;
    a.batch = batch;
    const size_t smem = (size_t)w->tiles * 128 + 64;
    if (smem > 48 * 1024) {
        static bool attr[64] = {};
        if (!attr[w->device & 63]) {
            TMAC_CUDA_TRY(cudaFuncSetAttribute(int16_gemv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               200 * 1024));
            attr[w->device & 63] = true;
        }
        if (smem > 200 * 1024) return fail(TMAC_ERR_SHAPE, "INT16 path: cols too large");
    }
    const int grid = (int)std::min<int64_t>((w->groups + 7) / 8, (int64_t)num_sms(w->device) * 4);
    int16_gemv_kernel<<<grid, kThreads, smem, s>>>(a);
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int register_f32(tmac_weight_s* w, const uint8_t* d_raw, cudaStream_t s)
{
    (void)d_raw;
    (void)s;
    (void)w;
    return TMAC_OK;
}

int launch_f32(const tmac_weight_s* w, const float* x, float* y, int batch, cudaStream_t s)
{
    const unsigned grid = (unsigned)((w->rows + kThreads - 1) / kThreads);
    for (int b = 0; b < batch; b++) {
        f32_gemv_kernel<<<grid, kThreads, 0, s>>>(w->type, w->data, w->rows, w->cols, x + (int64_t)b * w->cols,
                                                  y + (int64_t)b * w->rows);
        TMAC_CUDA_TRY(cudaGetLastError());
    }
    return TMAC_OK;
}

}  // namespace tmac
