// decode_ops.cuh -- the decode step's context operations as device functions,
// shared by the per-kernel decode engine (decode.cu) and the persistent decode
// kernel (decode_mega.cu) so that both compute every value identically.
// Reference: forward_layer_with_cache (sim/tmac_gguf.cpp:1559-1711), rms_norm
// (:447-454), apply_rope (:1528-1554), attention (:1625-1660), silu (:459-461).
#pragma once

#include "model.cuh"

namespace tmac {

// rms_norm's scale (:447-454) from the in-order sum of the squares.
TMAC_DEV float rms_scale_from_sum(float sum, int n)
{
    const float mean = __fdiv_rn(sum, (float)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
}

// s + p[0] + p[1] + ... + p[m-1], each add rounded in turn (p 16-byte aligned,
// m a multiple of 16).
TMAC_DEV float seq_sum_from(float s, const float* p, int m)
{
    const float4* p4 = reinterpret_cast<const float4*>(p);
    int i = 0;
    for (; i + 32 <= m; i += 32) {
        float4 f[8];
#pragma unroll
        for (int u = 0; u < 8; u++) f[u] = p4[i / 4 + u];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            s = __fadd_rn(s, f[u].x);
            s = __fadd_rn(s, f[u].y);
            s = __fadd_rn(s, f[u].z);
            s = __fadd_rn(s, f[u].w);
        }
    }
    for (; i < m; i += 16) {
        float4 f[4];
#pragma unroll
        for (int u = 0; u < 4; u++) f[u] = p4[i / 4 + u];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            s = __fadd_rn(s, f[u].x);
            s = __fadd_rn(s, f[u].y);
            s = __fadd_rn(s, f[u].z);
            s = __fadd_rn(s, f[u].w);
        }
    }
    return s;
}

// rms_norm's scale (:447-454): 1 / sqrtf(sum / n + 1e-6) with the sum of the
// squares sq[0..n) taken in order (sq 16-byte aligned; one thread).
TMAC_DEV float rms_scale(const float* sq, int n)
{
    float sum = 0.0f;
    const float4* x4 = reinterpret_cast<const float4*>(sq);
    int i = 0;
    for (; i + 32 <= n; i += 32) {  // 32 values loaded ahead of the sequential adds
        float4 f[8];
#pragma unroll
        for (int u = 0; u < 8; u++) f[u] = x4[i / 4 + u];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            sum = __fadd_rn(sum, f[u].x);
            sum = __fadd_rn(sum, f[u].y);
            sum = __fadd_rn(sum, f[u].z);
            sum = __fadd_rn(sum, f[u].w);
        }
    }
    for (; i < n; i++) sum = __fadd_rn(sum, sq[i]);
    return rms_scale_from_sum(sum, n);
}

// silu(g) * u (:459-461, :1697-1700).
TMAC_DEV float silu_mul(float g, float u) { return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf_ref(-g))), u); }

constexpr int kAttnChunk = 64;    // K/V rows in shared memory at a time
constexpr int kAttnStride = 68;   // floats per staged row (16-byte aligned rows)
constexpr int kAttnThreads = 256; // threads of one head's attention

struct AttnShared {
    // the head's q bias, its KV head's k and v biases, and the RoPE cos / sin of
    // the position (64 + 64 + 64 + 32 + 32), staged by attention_prefetch
    alignas(16) float pre[3 * kHeadDim + kHeadDim];
    float red[kAttnThreads / 32];
    float q[kHeadDim], k[kHeadDim], v[kHeadDim];
    float log_sum;
};

// Floats of the score and exp-term slots for nscore positions, rounded so that
// the K / V row buffers after them start 16-byte aligned (cp.async targets).
__host__ __device__ constexpr int attn_score_floats(int nscore) { return (2 * nscore + 3) / 4 * 4; }

// Bytes of the dynamic scratch `sc` that the attention needs for nscore score
// slots: scores | exp terms | K rows | V rows.
__host__ __device__ constexpr size_t attn_scratch_bytes(int nscore)
{
    return ((size_t)attn_score_floats(nscore) + 2 * kAttnChunk * kAttnStride) * sizeof(float);
}

TMAC_DEV void cp_async16(void* dst, const void* src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
TMAC_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
TMAC_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// First half of a query head's attention, threads 0..255: start copying the
// K and V rows of KV head kvh(h) for positions [0, min(pos, 64)) -- written by
// earlier steps, so they do not depend on this step's q / k / v -- into the
// K / V row buffers of `sc` (asynchronous; attention_head waits for them).
TMAC_DEV void attention_prefetch(int h, const float* __restrict__ kc, const float* __restrict__ vc, int pos,
                                 int nscore, float* sc, const float* __restrict__ bq, const float* __restrict__ bk,
                                 const float* __restrict__ bv, const float* __restrict__ cs,
                                 const float* __restrict__ sn, AttnShared& sh)
{
    const int kvh = h / (kHeads / kKvHeads);
    // biases and RoPE terms: they do not depend on this step's q / k / v
    if (threadIdx.x < 64) {
        const int i = threadIdx.x, part = i >> 4, c4 = (i & 15) * 4;
        const float* src = part == 0   ? (bq ? bq + h * kHeadDim : nullptr)
                           : part == 1 ? (bk ? bk + kvh * kHeadDim : nullptr)
                           : part == 2 ? (bv ? bv + kvh * kHeadDim : nullptr)
                                       : nullptr;
        float* dst = sh.pre + part * kHeadDim + c4;
        if (part < 3) {
            if (src) cp_async16(dst, src + c4);
            else dst[0] = dst[1] = dst[2] = dst[3] = 0.0f;
        } else {  // 8 chunks of cos, 8 of sin
            const float* tab = c4 < 32 ? cs : sn;
            cp_async16(dst, tab + (int64_t)pos * (kHeadDim / 2) + (c4 & 31));
        }
    }
    const int n = min(pos, kAttnChunk);
    float* kb = sc + attn_score_floats(nscore);
    float* vb = kb + kAttnChunk * kAttnStride;
    for (int i = threadIdx.x; i < n * (kHeadDim / 4); i += kAttnThreads) {
        const int r = i / (kHeadDim / 4), d4 = i % (kHeadDim / 4);
        const int64_t g = (int64_t)r * kKvDim + kvh * kHeadDim + 4 * d4;
        cp_async16(kb + r * kAttnStride + 4 * d4, kc + g);
        cp_async16(vb + r * kAttnStride + 4 * d4, vc + g);
    }
    cp_async_commit();
}

// Query head h, run by threads 0..255 of a CTA (they synchronise on named
// barrier `bar`) after attention_prefetch (which staged the biases and RoPE
// terms in sh.pre): q/k/v bias add (:1591-1614), RoPE on
// the head's q and its KV head's k (:1528-1554), KV-cache append by the first
// query head of each KV group (:1622-1623), then attention over positions
// 0..pos (:1625-1660): scores q.k in d order / sqrtf(64), max, exp terms, their
// sum in position order, log-sum-exp weights, context accumulated in position
// order.  The current position's k/v come from shared memory, so the append
// needs no ordering against the other heads.  `sc` holds
// attn_scratch_bytes(nscore).  q_head / k_head / v_head: the head's 64 q values
// and its KV head's k and v (global or shared memory); ctx_head: its 64 context
// outputs.  KV rows past the prefetched chunk are read at L2 (ld.global.cg):
// other CTAs of a persistent kernel write them while this CTA may hold older
// copies in L1.  stamps (diagnostics only): 8 %globaltimer values, or nullptr.
TMAC_DEV void attention_head(int h, const float* q_head, const float* k_head, const float* v_head,
                             int pos, float* __restrict__ kc, float* __restrict__ vc, float* ctx_head,
                             int nscore, float* sc, AttnShared& sh, int bar, unsigned long long* stamps = nullptr)
{
#define ATT_STAMP(i)                                                  \
    do {                                                              \
        if (stamps && threadIdx.x == 0) stamps[i] = global_timer_ns(); \
    } while (0)
    ATT_STAMP(0);
    const int tid = threadIdx.x;
    const int nsc = nscore;
    const int kvh = h / (kHeads / kKvHeads);
    float* kb = sc + attn_score_floats(nsc);  // [kAttnChunk][kAttnStride]
    float* vb = kb + kAttnChunk * kAttnStride;
    cp_async_wait_all();  // biases, RoPE terms and K / V rows of positions [0, min(pos, 64))
    named_bar_sync(bar, kAttnThreads);
    if (tid < kHeadDim) {  // thread j: pair j/2 of q (j even) or of k (j odd)
        const int j = tid, pr = j >> 1, d = 2 * pr;
        const bool isk = j & 1;
        const float* vec = isk ? k_head : q_head;
        const float* b = sh.pre + (isk ? kHeadDim : 0);
        const float c = sh.pre[3 * kHeadDim + pr], sv = sh.pre[3 * kHeadDim + kHeadDim / 2 + pr];
        const float x0 = __fadd_rn(vec[d], b[d]), x1 = __fadd_rn(vec[d + 1], b[d + 1]);
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sv));
        const float y1 = __fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, c));
        float* dst = isk ? sh.k : sh.q;
        dst[d] = y0;
        dst[d + 1] = y1;
        sh.v[j] = __fadd_rn(v_head[j], sh.pre[2 * kHeadDim + j]);
    }
    named_bar_sync(bar, kAttnThreads);
    ATT_STAMP(1);
    if (h % (kHeads / kKvHeads) == 0 && tid < kHeadDim) {
        kc[(int64_t)pos * kKvDim + kvh * kHeadDim + tid] = sh.k[tid];
        vc[(int64_t)pos * kKvDim + kvh * kHeadDim + tid] = sh.v[tid];
    }
    // scores, 64 positions at a time, one position per thread, d in order; the
    // first chunk's earlier rows were prefetched, later chunks are staged here
    for (int c0 = 0; c0 <= pos; c0 += kAttnChunk) {
        const int rows = min(kAttnChunk, pos + 1 - c0);
        if (c0 > 0) named_bar_sync(bar, kAttnThreads);
        for (int i = tid; i < rows * kHeadDim; i += kAttnThreads) {
            const int r = i / kHeadDim, d = i % kHeadDim, p = c0 + r;
            if (p == pos) kb[r * kAttnStride + d] = sh.k[d];
            else if (c0 > 0) kb[r * kAttnStride + d] = __ldcg(kc + (int64_t)p * kKvDim + kvh * kHeadDim + d);
        }
        named_bar_sync(bar, kAttnThreads);
        ATT_STAMP(2);
        for (int r = tid; r < rows; r += kAttnThreads) {
            const float* kp = kb + r * kAttnStride;
            float sum = 0.0f;
            for (int d = 0; d < kHeadDim; d++) sum = __fadd_rn(sum, __fmul_rn(sh.q[d], kp[d]));
            sc[c0 + r] = __fdiv_rn(sum, 8.0f);  // / sqrtf(64)
        }
    }
    named_bar_sync(bar, kAttnThreads);
    ATT_STAMP(3);
    // max (order-free), the exp terms in parallel, their sum in position order
    float mx = -INFINITY;
    for (int p = tid; p <= pos; p += kAttnThreads) mx = fmaxf(mx, sc[p]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) sh.red[tid >> 5] = mx;
    named_bar_sync(bar, kAttnThreads);
    mx = sh.red[0];
    for (int i = 1; i < kAttnThreads / 32; i++) mx = fmaxf(mx, sh.red[i]);
    float* ex = sc + pos + 1;
    for (int p = tid; p <= pos; p += kAttnThreads) ex[p] = expf_ref(__fsub_rn(sc[p], mx));
    named_bar_sync(bar, kAttnThreads);
    if (tid == 0) {
        float es = 0.0f;
        for (int p = 0; p <= pos; p++) es = __fadd_rn(es, ex[p]);
        sh.log_sum = __fadd_rn(logf_ref(es), mx);
    }
    named_bar_sync(bar, kAttnThreads);
    ATT_STAMP(4);
    for (int p = tid; p <= pos; p += kAttnThreads) sc[p] = expf_ref(__fsub_rn(sc[p], sh.log_sum));
    named_bar_sync(bar, kAttnThreads);
    ATT_STAMP(5);
    // context: V rows (first chunk prefetched), positions in order
    float a = 0.0f;
    for (int c0 = 0; c0 <= pos; c0 += kAttnChunk) {
        const int rows = min(kAttnChunk, pos + 1 - c0);
        if (c0 > 0) named_bar_sync(bar, kAttnThreads);
        for (int i = tid; i < rows * kHeadDim; i += kAttnThreads) {
            const int r = i / kHeadDim, d = i % kHeadDim, p = c0 + r;
            if (p == pos) vb[r * kAttnStride + d] = sh.v[d];
            else if (c0 > 0) vb[r * kAttnStride + d] = __ldcg(vc + (int64_t)p * kKvDim + kvh * kHeadDim + d);
        }
        named_bar_sync(bar, kAttnThreads);
        ATT_STAMP(6);
        if (tid < kHeadDim)
            for (int r = 0; r < rows; r++) a = __fadd_rn(a, __fmul_rn(sc[c0 + r], vb[r * kAttnStride + tid]));
    }
    if (tid < kHeadDim) ctx_head[tid] = a;
    ATT_STAMP(7);
#undef ATT_STAMP
}

}  // namespace tmac
