// top1.cu -- greedy next-token selection over fp32 logits (the argmax the
// decode harness uses in place of the reference's rand()-based top-k sampling,
// sim/tmac_gguf.cpp:1974-1990), as a packed key (top1_key in common.cuh) so
// that vocab shards merge with one int64 MAX all-reduce.
#include "common.cuh"

#include <algorithm>

namespace tmac {
namespace {

__global__ void __launch_bounds__(256) top1_kernel(const float* __restrict__ y, int64_t n, int64_t base,
                                                   unsigned long long* key)
{
    unsigned long long best = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const unsigned long long k = top1_key(y[i], base + i);
        best = k > best ? k : best;
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    __shared__ unsigned long long red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < 8; i++) best = red[i] > best ? red[i] : best;
        if (best) atomicMax(key, best);
    }
}

}  // namespace

int launch_top1(const float* y, int64_t n, int64_t index_base, unsigned long long* key, cudaStream_t s)
{
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 4));
    top1_kernel<<<grid, 256, 0, s>>>(y, n, index_base, key);
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

}  // namespace tmac
