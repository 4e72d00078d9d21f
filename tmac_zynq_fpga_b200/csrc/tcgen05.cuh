// tcgen05.cuh -- the 5th-generation tensor-core and TMA building blocks shared
// by the batched GEMM (gemm_tc.cu) and the int8 tensor peak probe:
// tensor-map loads, shared-memory matrix descriptors (K-major, 128-byte
// swizzle), kind::i8 MMAs with TMEM accumulators, commits and TMEM loads.
#pragma once

#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace tmac {

TMAC_DEV void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 128 bytes (stride 1024 bytes), sm_100 descriptor version 1.
TMAC_DEV uint64_t desc_sw128(uint32_t saddr)
{
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;              // leading byte offset (16 B; unused when swizzled)
    d |= (uint64_t)(1024 >> 4) << 32;    // stride byte offset
    d |= (uint64_t)1 << 46;              // version
    d |= (uint64_t)2 << 61;              // SWIZZLE_128B
    return d;
}

TMAC_DEV void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

TMAC_DEV void mma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
TMAC_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TMAC_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

TMAC_DEV void tmem_ld8(uint32_t taddr, uint32_t* r)
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
TMAC_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// Instruction descriptor for kind::i8 with an s32 accumulator, A/B signed (1)
// or unsigned (0), both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_i8_mn(uint32_t a_signed, uint32_t b_signed, uint32_t M, uint32_t N)
{
    return (2u << 4) | (a_signed << 7) | (b_signed << 10) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

TMAC_DEV void tmem_alloc(uint32_t* slot, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
TMAC_DEV void tmem_dealloc(uint32_t tmem, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(cols));
}
// Orders this thread's generic-proxy shared-memory writes before later reads
// by the async proxy (tensor cores, TMA).
TMAC_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library has no link-time dependency on libcuda.
inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}


}  // namespace tmac
