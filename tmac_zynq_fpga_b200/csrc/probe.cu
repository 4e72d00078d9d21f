// probe.cu -- measurement aid: the dense int8 tensor-core rate of this GPU,
// the roofline denominator of the prefill GEMM (gemm_tc.cu).  One CTA per SM;
// one thread issues back-to-back tcgen05.mma kind::i8 (M = 128, N = 256,
// K = 32, s32 accumulate into TMEM) from operands resident in shared memory,
// so nothing but the tensor pipe bounds it.  No reference counterpart.
#include "tcgen05.cuh"

namespace tmac {
namespace {

constexpr int kProbeN = 256;
constexpr uint32_t kProbeA = 128 * 128, kProbeB = kProbeN * 128;  // one 128-byte K slab each
// more shared memory than the operands need, so that one CTA fits an SM and
// every SM runs exactly one
constexpr size_t kProbeSmem = 160 * 1024;

__global__ void __launch_bounds__(128, 1) mma_i8_probe_kernel(int iters, int* err)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* done = reinterpret_cast<uint64_t*>(smem + kProbeA + kProbeB);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    const int warp = threadIdx.x >> 5;
    for (uint32_t i = threadIdx.x; i < (kProbeA + kProbeB) / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(smem)[i] = i * 2654435761u;
    if (threadIdx.x == 0) {
        mbar_init(done, 1);
        fence_mbar_init();
    }
    fence_proxy_async_smem();
    if (warp == 0) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 0) {
        constexpr uint32_t idesc = idesc_i8_mn(1, 1, 128, kProbeN);
        const uint32_t sa = smem_addr(smem), sb = sa + kProbeA;
        for (int it = 0; it < iters; it++) {
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
                mma_i8(tmem + (uint32_t)(it & 1) * kProbeN, desc_sw128(sa + kk * 32), desc_sw128(sb + kk * 32), idesc,
                       (it > 1 || kk) ? 1u : 0u);
        }
        mma_commit(done);
        mbar_wait_bounded(done, 0, err);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace
}  // namespace tmac

using namespace tmac;

// Dense int8 ops per second (2 per multiply-accumulate) of `iters` x 4 MMAs on
// every SM, timed with CUDA events around one launch; *tops in TOPS.
extern "C" int tmac_probe_mma_i8(int device, int iters, double* tops)
{
    if (!tops || iters <= 0) return fail(TMAC_ERR_INVALID, "bad arguments");
    DeviceGuard dg(device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    TMAC_CUDA_TRY(cudaFuncSetAttribute(mma_i8_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kProbeSmem));
    const int sms = num_sms(device);
    int* err = device_error_word(device);
    cudaEvent_t e0, e1;
    TMAC_CUDA_TRY(cudaEventCreate(&e0));
    TMAC_CUDA_TRY(cudaEventCreate(&e1));
    mma_i8_probe_kernel<<<sms, 128, kProbeSmem>>>(iters / 10 + 1, err);  // warm-up
    TMAC_CUDA_TRY(cudaEventRecord(e0));
    mma_i8_probe_kernel<<<sms, 128, kProbeSmem>>>(iters, err);
    TMAC_CUDA_TRY(cudaEventRecord(e1));
    TMAC_CUDA_TRY(cudaEventSynchronize(e1));
    TMAC_CUDA_TRY(cudaGetLastError());
    float ms = 0.0f;
    TMAC_CUDA_TRY(cudaEventElapsedTime(&ms, e0, e1));
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    const double ops = 2.0 * 128.0 * kProbeN * 128.0 * (double)iters * sms;
    *tops = ops / (ms * 1e-3) / 1e12;
    return TMAC_OK;
}
