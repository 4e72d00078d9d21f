// quantize.cu -- the per-call activation quantisation every matmul_fpga_*
// driver starts with (sim/tmac_gguf.cpp:889-896):
//   x_scale = max|x| / 32767 (1 if max < 1e-10),  x_q = (int16)roundf(x / x_scale)
// done once for an activation vector that several GEMVs consume (q/k/v share
// one x, gate/up share one x), which gives the same x_q each driver computes.
#include "common.cuh"

namespace tmac {
namespace {

// xq: int16 [batch][cols]; xp: the same values as byte planes [batch][2][cols]
// (high bytes, then low bytes), the form the block-quant GEMVs stage with one
// bulk copy.  Either may be null.
__global__ void __launch_bounds__(1024) quantize_kernel(const float* __restrict__ x, int64_t cols,
                                                        int16_t* __restrict__ xq, uint8_t* __restrict__ xp,
                                                        float* __restrict__ xs)
{
    __shared__ float red[32];
    pdl_launch();
    pdl_wait();
    const float* xb = x + (int64_t)blockIdx.x * cols;
    float mx = 0.0f;
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) mx = fmaxf(mx, fabsf(xb[j]));
    mx = block_max(mx, red, blockDim.x);
    const float s = x_scale_from_max(mx);
    if (threadIdx.x == 0) xs[blockIdx.x] = s;
    uint8_t* p = xp ? xp + (int64_t)blockIdx.x * 2 * cols : nullptr;
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
        const int16_t q = quantize_one(xb[j], s);
        if (xq) xq[(int64_t)blockIdx.x * cols + j] = q;
        if (p) {
            p[j] = (uint8_t)((uint16_t)q >> 8);
            p[cols + j] = (uint8_t)(q & 0xFF);
        }
    }
}

}  // namespace

int launch_quantize(const float* x, int64_t cols, int batch, int16_t* xq, float* xs, cudaStream_t s, uint8_t* xp)
{
    TMAC_CUDA_TRY(launch_k(quantize_kernel, dim3(batch), dim3(1024), 0, s, x, cols, xq, xp, xs));
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

}  // namespace tmac

using namespace tmac;

extern "C" int tmac_quantize_x(const float* x, int64_t cols, int batch, int16_t* xq, float* xs, void* stream)
{
    if (!x || !xq || !xs) return fail(TMAC_ERR_INVALID, "NULL argument");
    if (cols <= 0 || batch <= 0) return fail(TMAC_ERR_SHAPE, "cols and batch must be positive");
    if (cols % 8) return fail(TMAC_ERR_SHAPE, "cols must be a multiple of 8");
    return launch_quantize(x, cols, batch, xq, xs, (cudaStream_t)stream);
}

extern "C" int tmac_gemv_xq(tmac_weight_t w, const int16_t* xq, const float* xs, float* y, int batch, void* stream)
{
    if (!w || !xq || !xs || !y) return fail(TMAC_ERR_INVALID, "NULL argument");
    if (batch <= 0) return fail(TMAC_ERR_SHAPE, "batch must be positive");
    if (w->mode != TMAC_MODE_NATIVE) return fail(TMAC_ERR_TYPE, "tmac_gemv_xq needs a NATIVE-mode weight");
    DeviceGuard dg(w->device);
    cudaStream_t s = (cudaStream_t)stream;
    if (w->type == TMAC_TYPE_Q8_0) return launch_q8_0(w, nullptr, y, nullptr, nullptr, batch, s, nullptr, 0, xq, xs);
    return launch_blockq(w, nullptr, xq, nullptr, xs, y, nullptr, nullptr, batch, s);
}
