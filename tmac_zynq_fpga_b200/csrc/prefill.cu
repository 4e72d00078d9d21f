// prefill.cu -- batched prefill of the Qwen2-0.5B-shaped model: n_seq
// independent sequences of len tokens go through all 24 layers at once, every
// projection as one tensor-core GEMM over all n_seq*len rows (gemm_tc.cu).
//
// The reference has no batched path: process_prompt (sim/tmac_gguf.cpp:1992-2023)
// feeds the prompt one token at a time through forward_layer_with_cache
// (:1559-1711).  Every per-token operation here is the decode engine's
// (decode.cu), in the same fp32 operation order:
//   embedding  dequant_q8_0 row                      (:225-234, :413-427)
//   rms_norm   sequential sum of squares             (:447-454)
//   matmuls    x_q per row, exact int16 weights      (a3-a5 / a2, as the GEMVs)
//   rope       adjacent pairs, host cos/sin tables   (:1528-1554)
//   attention  causal over the sequence's positions  (:1625-1660)
//   silu       x / (1 + expf(-x)) * up               (:459-461)
// so position t of a sequence gets the hidden state the decode engine computes
// after feeding tokens 0..t, bit for bit.  After the last layer the last
// position of each sequence goes through output_norm and the tied Q8_0 logits;
// its top-1 is the first generated token.
#include "model.cuh"

#include <cstring>

namespace tmac {

struct PrefillState {
    int64_t cap = 0;  // tokens the buffers hold
    float *hidden = nullptr, *qkv = nullptr, *qr = nullptr, *kr = nullptr, *vr = nullptr, *ctx = nullptr,
          *attn = nullptr, *gu = nullptr, *ffn = nullptr, *xlast = nullptr, *logits = nullptr;
    int8_t* xh = nullptr;  // byte planes of the current matmul input [cap][kInter]
    uint8_t* xl = nullptr;
    float* xs = nullptr;
    int* tokens = nullptr;
    unsigned long long* keys = nullptr;
    int64_t cap_seq = 0;
    std::map<std::string, std::pair<int8_t*, uint8_t*>> q8planes;  // Q8_0 matrices (attn_v)
    std::vector<void*> allocs;        // activation buffers (re-made when a larger batch comes)
    std::vector<void*> plane_allocs;  // weight planes (kept for the model's lifetime)
};

namespace {

constexpr int kQkv = kHidden + 2 * kKvDim;  // 1152

// ------------------------------------------------------------------ kernels
__global__ void pf_embed_kernel(const uint8_t* __restrict__ emb, const int* __restrict__ tokens,
                                float* __restrict__ hidden)
{
    const int64_t t = blockIdx.x;
    int tok = tokens[t];
    if (tok < 0 || tok >= kVocab) tok = 0;
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) {
        const int64_t idx = (int64_t)tok * kHidden + i;
        const uint8_t* b = emb + (idx / 32) * 34;
        hidden[t * kHidden + i] = __fmul_rn((float)(int8_t)b[2 + idx % 32], f16_bits_to_f32(ld_u16_unaligned(b)));
    }
}

// One warp per token: x += delta (written back), rms_norm with weights w, then
// x_q of the normalised row as byte planes.  Rows whose position is the last
// of a sequence also store the normalised fp32 row in xlast[seq] (logits).
__global__ void __launch_bounds__(256) pf_rmsnorm_kernel(float* __restrict__ hidden, const float* __restrict__ delta,
                                                         const float* __restrict__ w, int64_t M,
                                                         int8_t* __restrict__ xh, uint8_t* __restrict__ xl,
                                                         float* __restrict__ xs, float* __restrict__ xlast, int len)
{
    __shared__ __align__(16) float buf[8][kHidden];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t t = (int64_t)blockIdx.x * 8 + warp;
    if (t >= M) return;
    float* x = hidden + t * kHidden;
    float* v = buf[warp];
    for (int i = lane; i < kHidden; i += 32) {
        float a = x[i];
        if (delta) {
            a = __fadd_rn(a, delta[t * kHidden + i]);
            x[i] = a;
        }
        v[i] = a;
    }
    __syncwarp();
    float scale = 1.0f;
    if (w) {
        if (lane == 0) {
            float sum = 0.0f;
            const float4* v4 = reinterpret_cast<const float4*>(v);
            for (int i = 0; i < kHidden / 4; i += 8) {  // loads ahead of the sequential adds
                float4 f[8];
#pragma unroll
                for (int u = 0; u < 8; u++) f[u] = v4[i + u];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    sum = __fadd_rn(sum, __fmul_rn(f[u].x, f[u].x));
                    sum = __fadd_rn(sum, __fmul_rn(f[u].y, f[u].y));
                    sum = __fadd_rn(sum, __fmul_rn(f[u].z, f[u].z));
                    sum = __fadd_rn(sum, __fmul_rn(f[u].w, f[u].w));
                }
            }
            const float mean = __fdiv_rn(sum, (float)kHidden);
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
        }
        scale = __shfl_sync(0xffffffffu, scale, 0);
    }
    const bool last = xlast && (t % len) == len - 1;
    float mx = 0.0f;
    for (int i = lane; i < kHidden; i += 32) {
        const float o = w ? __fmul_rn(__fmul_rn(v[i], w[i]), scale) : v[i];
        v[i] = o;
        mx = fmaxf(mx, fabsf(o));
        if (last) xlast[(t / len) * kHidden + i] = o;
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (!xh) return;
    const float s = x_scale_from_max(mx);
    if (lane == 0) xs[t] = s;
    for (int i = lane; i < kHidden; i += 32) {
        const int16_t q = quantize_one(v[i], s);
        xh[t * kHidden + i] = (int8_t)(q >> 8);
        xl[t * kHidden + i] = (uint8_t)(q & 0xFF);
    }
}

// q/k bias + RoPE, v bias (the decode kernel's prologue), one CTA per token.
__global__ void __launch_bounds__(kHidden / 2 + kKvDim / 2) pf_rope_kernel(
    const float* __restrict__ qkv, const float* __restrict__ bq, const float* __restrict__ bk,
    const float* __restrict__ bv, const float* __restrict__ cs, const float* __restrict__ sn, int len,
    float* __restrict__ qr, float* __restrict__ kr, float* __restrict__ vr)
{
    const int64_t t = blockIdx.x;
    const int pos = (int)(t % len);
    const float* c = cs + (int64_t)pos * (kHeadDim / 2);
    const float* sv = sn + (int64_t)pos * (kHeadDim / 2);
    const float* row = qkv + t * kQkv;
    const int j = threadIdx.x;  // pair j: q pairs 0..447, then k pairs 448..511
    const bool isk = j >= kHidden / 2;
    const int jj = isk ? j - kHidden / 2 : j;
    const int d = 2 * jj, pr = (d % kHeadDim) / 2;
    const float* vec = isk ? row + kHidden : row;
    const float* b = isk ? bk : bq;
    const float x0 = __fadd_rn(vec[d], b ? b[d] : 0.0f), x1 = __fadd_rn(vec[d + 1], b ? b[d + 1] : 0.0f);
    const float y0 = __fsub_rn(__fmul_rn(x0, c[pr]), __fmul_rn(x1, sv[pr]));
    const float y1 = __fadd_rn(__fmul_rn(x0, sv[pr]), __fmul_rn(x1, c[pr]));
    float* dst = isk ? kr + t * kKvDim : qr + t * kHidden;
    dst[d] = y0;
    dst[d + 1] = y1;
    if (j < kKvDim) vr[t * kKvDim + j] = __fadd_rn(row[kHidden + kKvDim + j], bv ? bv[j] : 0.0f);
}

constexpr int kGroup = kHeads / kKvHeads;  // 7 query heads per KV head

// Causal attention in one pass over shared memory: one CTA per (sequence, KV
// head, QB queries), the 7 query heads of the KV head together.  The scores
// of its 7*QB (head, query) pairs stay in shared memory (S), so they never go
// through HBM; every value is the decode engine's (rope_attention_kernel) for
// that token: scores in d order /8, max, exp terms summed in position order
// (one thread per pair over the terms computed by all threads), log-sum-exp
// weights, context accumulated in position order.
constexpr int kAThreads = 512;
constexpr int kAPTile = 128;                    // K/V positions staged at a time
constexpr int kARow = kHeadDim + 4;             // staged K/V and q rows: 16-byte aligned, banks spread
// S and E rows are len rounded up to 4 floats, so every region stays 16-byte aligned.
template <int QB>
constexpr size_t attn_smem(int len)
{
    return (size_t)(2 * kGroup * QB * ((len + 3) & ~3) + kAPTile * kARow + kGroup * QB * kARow + 2 * kGroup * QB) *
           sizeof(float);
}

template <int QB>
__global__ void __launch_bounds__(kAThreads) pf_attention_kernel(const float* __restrict__ qr,
                                                                 const float* __restrict__ kr,
                                                                 const float* __restrict__ vr, int len,
                                                                 float* __restrict__ ctx)
{
    constexpr int NP = kGroup * QB;  // pair pr = head * QB + query
    extern __shared__ __align__(16) float asm_[];
    const int ls4 = (len + 3) & ~3;        // row stride of S and E
    float* S = asm_;                       // [NP][ls4] scores
    float* E = S + NP * ls4;               // [NP][ls4] exp terms, then weights
    float* kv = E + NP * ls4;              // [kAPTile][kARow] K, later V
    float* qs = kv + kAPTile * kARow;      // [NP][kARow]
    float* mxs = qs + NP * kARow;          // [NP]
    float* lss = mxs + NP;                 // [NP]
    const int seq = blockIdx.x, kvh = blockIdx.y;
    const int nqb = (len + QB - 1) / QB;
    const int t0 = (nqb - 1 - (int)blockIdx.z) * QB;  // longest rows first
    const int nq = min(QB, len - t0);
    const int tlast = t0 + nq - 1;
    const int64_t base = (int64_t)seq * len;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    for (int i = tid; i < NP * (kHeadDim / 4); i += kAThreads) {
        const int pr = i / (kHeadDim / 4), d4 = i % (kHeadDim / 4), hh = pr / QB, tq = pr % QB;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (tq < nq)
            v = *reinterpret_cast<const float4*>(qr + (base + t0 + tq) * kHidden + (kvh * kGroup + hh) * kHeadDim + 4 * d4);
        *reinterpret_cast<float4*>(qs + pr * kARow + 4 * d4) = v;
    }
    // ---- scores: thread (query, position) of the tile, the 7 heads at once
    for (int p0 = 0; p0 <= tlast; p0 += kAPTile) {
        __syncthreads();
        for (int i = tid; i < kAPTile * (kHeadDim / 4); i += kAThreads) {
            const int pp = i / (kHeadDim / 4), d4 = i % (kHeadDim / 4);
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (p0 + pp <= tlast)
                v = *reinterpret_cast<const float4*>(kr + (base + p0 + pp) * kKvDim + kvh * kHeadDim + 4 * d4);
            *reinterpret_cast<float4*>(kv + pp * kARow + 4 * d4) = v;
        }
        __syncthreads();
        for (int i = tid; i < QB * kAPTile; i += kAThreads) {
            const int tq = i / kAPTile, pp = i % kAPTile, p = p0 + pp;
            if (tq >= nq || p > t0 + tq) continue;
            float acc[kGroup];
#pragma unroll
            for (int hh = 0; hh < kGroup; hh++) acc[hh] = 0.0f;
#pragma unroll 4
            for (int d4 = 0; d4 < kHeadDim / 4; d4++) {
                const float4 k4 = *reinterpret_cast<const float4*>(kv + pp * kARow + 4 * d4);
#pragma unroll
                for (int hh = 0; hh < kGroup; hh++) {
                    const float4 q4 = *reinterpret_cast<const float4*>(qs + (hh * QB + tq) * kARow + 4 * d4);
                    acc[hh] = __fadd_rn(acc[hh], __fmul_rn(q4.x, k4.x));
                    acc[hh] = __fadd_rn(acc[hh], __fmul_rn(q4.y, k4.y));
                    acc[hh] = __fadd_rn(acc[hh], __fmul_rn(q4.z, k4.z));
                    acc[hh] = __fadd_rn(acc[hh], __fmul_rn(q4.w, k4.w));
                }
            }
#pragma unroll
            for (int hh = 0; hh < kGroup; hh++) S[(hh * QB + tq) * ls4 + p] = __fdiv_rn(acc[hh], 8.0f);
        }
    }
    __syncthreads();
    // ---- per pair: max (any order), then the exp terms (one warp per pair)
    for (int pr = warp; pr < NP; pr += kAThreads / 32) {
        const int tq = pr % QB, t = t0 + tq;
        if (tq >= nq) continue;
        const float* row = S + pr * ls4;
        float mx = -INFINITY;
        for (int p = lane; p <= t; p += 32) mx = fmaxf(mx, row[p]);
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        for (int p = lane; p <= t; p += 32) E[pr * ls4 + p] = expf_ref(__fsub_rn(row[p], mx));
        if (lane == 0) mxs[pr] = mx;
    }
    __syncthreads();
    // ---- the sums in position order, one thread per pair
    if (tid < NP && tid % QB < nq) {
        const int pr = tid, t = t0 + pr % QB;
        const float* e = E + pr * ls4;
        float es = 0.0f;
        int p = 0;
        for (; p + 3 <= t; p += 4) {  // rows are 16-byte aligned
            const float4 v = *reinterpret_cast<const float4*>(e + p);
            es = __fadd_rn(es, v.x);
            es = __fadd_rn(es, v.y);
            es = __fadd_rn(es, v.z);
            es = __fadd_rn(es, v.w);
        }
        for (; p <= t; p++) es = __fadd_rn(es, e[p]);
        lss[pr] = __fadd_rn(logf_ref(es), mxs[pr]);
    }
    __syncthreads();
    // ---- weights exp(s - log_sum) over the terms
    for (int pr = warp; pr < NP; pr += kAThreads / 32) {
        const int tq = pr % QB, t = t0 + tq;
        if (tq >= nq) continue;
        const float ls = lss[pr];
        for (int p = lane; p <= t; p += 32) E[pr * ls4 + p] = expf_ref(__fsub_rn(S[pr * ls4 + p], ls));
    }
    // ---- context: thread (query, dim, head half), positions in order
    const int hq = tid / (QB * kHeadDim);               // 0: heads 0..3, 1: heads 4..6
    const int tq = (tid / kHeadDim) % QB, d = tid % kHeadDim;
    const bool active = tid < 2 * QB * kHeadDim && tq < nq;
    const int h0 = hq ? 4 : 0, nh = hq ? kGroup - 4 : 4;
    const int t = t0 + tq;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int p0 = 0; p0 <= tlast; p0 += kAPTile) {
        __syncthreads();
        for (int i = tid; i < kAPTile * (kHeadDim / 4); i += kAThreads) {
            const int pp = i / (kHeadDim / 4), d4 = i % (kHeadDim / 4);
            float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (p0 + pp <= tlast)
                v = *reinterpret_cast<const float4*>(vr + (base + p0 + pp) * kKvDim + kvh * kHeadDim + 4 * d4);
            *reinterpret_cast<float4*>(kv + pp * kARow + 4 * d4) = v;
        }
        __syncthreads();
        if (!active) continue;
        const int np = min(kAPTile, t - p0 + 1);
        for (int pp = 0; pp < np; pp++) {
            const float v = kv[pp * kARow + d];
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (j < nh) acc[j] = __fadd_rn(acc[j], __fmul_rn(E[((h0 + j) * QB + tq) * ls4 + p0 + pp], v));
        }
    }
    if (active) {
#pragma unroll
        for (int j = 0; j < 4; j++)
            if (j < nh) ctx[(base + t) * kHidden + (kvh * kGroup + h0 + j) * kHeadDim + d] = acc[j];
    }
}

// silu(gate) * up for one token per CTA, kept in registers: its absolute
// maximum, x_scale and the byte planes of its x_q are all the down
// projection needs, so h itself is not written back.  kSiluThreads threads x
// kSiluVec float4 = kInter values.
constexpr int kSiluThreads = 304, kSiluVec = 4;
static_assert(kSiluThreads * kSiluVec * 4 == kInter, "silu tiling");
__global__ void __launch_bounds__(kSiluThreads) pf_silu_kernel(const float* __restrict__ gu, int8_t* __restrict__ xh,
                                                              uint8_t* __restrict__ xl, float* __restrict__ xs)
{
    __shared__ float red[(kSiluThreads + 31) / 32];
    const int64_t t = blockIdx.x;
    const float4* g4 = reinterpret_cast<const float4*>(gu + t * 2 * kInter);
    const float4* u4 = reinterpret_cast<const float4*>(gu + t * 2 * kInter + kInter);
    float v[kSiluVec][4];
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < kSiluVec; k++) {
        const int i = threadIdx.x + k * kSiluThreads;
        const float4 g = g4[i], u = u4[i];
        const float gv[4] = {g.x, g.y, g.z, g.w}, uv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            v[k][e] = __fmul_rn(__fdiv_rn(gv[e], __fadd_rn(1.0f, expf_ref(-gv[e]))), uv[e]);
            mx = fmaxf(mx, fabsf(v[k][e]));
        }
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = 0.0f;
#pragma unroll
    for (int w = 0; w < (kSiluThreads + 31) / 32; w++) mx = fmaxf(mx, red[w]);
    const float s = x_scale_from_max(mx);
    if (threadIdx.x == 0) xs[t] = s;
    uint32_t* h4 = reinterpret_cast<uint32_t*>(xh + t * kInter);
    uint32_t* l4 = reinterpret_cast<uint32_t*>(xl + t * kInter);
#pragma unroll
    for (int k = 0; k < kSiluVec; k++) {
        uint32_t hw = 0, lw = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int16_t q = quantize_one(v[k][e], s);
            hw |= (uint32_t)((uint16_t)q >> 8) << (8 * e);
            lw |= (uint32_t)(q & 0xFF) << (8 * e);
        }
        const int i = threadIdx.x + k * kSiluThreads;
        h4[i] = hw;
        l4[i] = lw;
    }
}

// --------------------------------------------------------------------- host
template <typename T>
int ps_alloc(PrefillState* p, T** ptr, size_t n)
{
    TMAC_CUDA_TRY(cudaMalloc((void**)ptr, n * sizeof(T)));
    p->allocs.push_back(*ptr);
    return TMAC_OK;
}

int ensure_state(tmac_model_s* m, int64_t M, int n_seq)
{
    if (!m->prefill) m->prefill = new PrefillState();
    PrefillState* p = m->prefill;
    if (p->cap >= M && p->cap_seq >= n_seq) return TMAC_OK;
    for (void* a : p->allocs) cudaFree(a);
    p->allocs.clear();
    p->cap = 0;
    p->cap_seq = 0;
    int rc;
    if ((rc = ps_alloc(p, &p->hidden, (size_t)M * kHidden)) || (rc = ps_alloc(p, &p->qkv, (size_t)M * kQkv)) ||
        (rc = ps_alloc(p, &p->qr, (size_t)M * kHidden)) || (rc = ps_alloc(p, &p->kr, (size_t)M * kKvDim)) ||
        (rc = ps_alloc(p, &p->vr, (size_t)M * kKvDim)) || (rc = ps_alloc(p, &p->ctx, (size_t)M * kHidden)) ||
        (rc = ps_alloc(p, &p->attn, (size_t)M * kHidden)) || (rc = ps_alloc(p, &p->gu, (size_t)M * 2 * kInter)) ||
        (rc = ps_alloc(p, &p->ffn, (size_t)M * kHidden)) || (rc = ps_alloc(p, &p->xh, (size_t)M * kInter)) ||
        (rc = ps_alloc(p, &p->xl, (size_t)M * kInter)) || (rc = ps_alloc(p, &p->xs, (size_t)M)) ||
        (rc = ps_alloc(p, &p->tokens, (size_t)M)) || (rc = ps_alloc(p, &p->xlast, (size_t)n_seq * kHidden)) ||
        (rc = ps_alloc(p, &p->logits, (size_t)n_seq * kVocab)) || (rc = ps_alloc(p, &p->keys, (size_t)n_seq)))
        return rc;
    p->cap = M;
    p->cap_seq = n_seq;
    return TMAC_OK;
}

// GEMM of the current planes (K columns) with a NATIVE block-quant weight into
// y[M][y_stride] (columns [0, rows)).
int pf_gemm(tmac_model_s* m, tmac_weight_s* w, int64_t M, int64_t K, float* y, int64_t y_stride, cudaStream_t s)
{
    if (w->cols != K) return fail(TMAC_ERR_SHAPE, "prefill: matrix width does not match its input");
    int rc = gemm_prepare(w, s);
    if (rc) return rc;
    PrefillState* p = m->prefill;
    GemmOperands op;
    op.xh = reinterpret_cast<const uint8_t*>(p->xh);
    op.xl = p->xl;
    op.x_stride = K;
    op.xs = p->xs;
    op.M = (int)M;
    op.wh = reinterpret_cast<const uint8_t*>(w->gwh);
    op.wl = reinterpret_cast<const uint8_t*>(w->gwl);
    op.w_stride = K;
    op.N = (int)w->rows;
    op.K = K;
    op.row_param = w->row_norm;
    op.row_rinv = reinterpret_cast<const double*>(w->grinv);
    op.mode = 0;
    op.y = y;
    op.y_stride = y_stride;
    op.device = m->device;
    return gemm_planes(op, s);
}

// Q8_0 matrix (attn_v of the Q8 layers): 64-column tiles folded in order into
// y as the Q8 GEMV does, one GEMM launch per tile.
int pf_gemm_q8(tmac_model_s* m, const std::string& name, tmac_weight_s* w, int64_t M, float* y, int64_t y_stride,
               cudaStream_t s)
{
    PrefillState* p = m->prefill;
    auto it = p->q8planes.find(name);
    if (it == p->q8planes.end()) {
        int8_t* wh = nullptr;
        uint8_t* wl = nullptr;
        int rc;
        TMAC_CUDA_TRY(cudaMalloc(&wh, (size_t)(w->rows * w->cols)));
        p->plane_allocs.push_back(wh);
        TMAC_CUDA_TRY(cudaMalloc(&wl, (size_t)(w->rows * w->cols)));
        p->plane_allocs.push_back(wl);
        if ((rc = q8_planes(w, wh, wl, s))) return rc;
        it = p->q8planes.emplace(name, std::make_pair(wh, wl)).first;
    }
    // the fold starts from 0.0f: y = (float)(0.0 + tile 0), then the other tiles
    for (int64_t r = 0; r < M; r += 65535) {
        const int64_t rows = std::min<int64_t>(65535, M - r);
        TMAC_CUDA_TRY(cudaMemset2DAsync(y + r * y_stride, y_stride * sizeof(float), 0, w->rows * sizeof(float), rows, s));
    }
    for (int64_t k0 = 0; k0 < w->cols; k0 += 64) {
        GemmOperands op;
        op.xh = reinterpret_cast<const uint8_t*>(p->xh);
        op.xl = p->xl;
        op.x_stride = w->cols;
        op.xs = p->xs;
        op.M = (int)M;
        op.wh = reinterpret_cast<const uint8_t*>(it->second.first);
        op.wl = it->second.second;
        op.w_stride = w->cols;
        op.N = (int)w->rows;
        op.K = std::min<int64_t>(64, w->cols - k0);
        op.k_off = k0;
        op.row_param = w->row_norm;
        op.mode = 1;
        op.y = y;
        op.y_stride = y_stride;
        op.device = m->device;
        int rc = gemm_planes(op, s);
        if (rc) return rc;
    }
    return TMAC_OK;
}

tmac_weight_s* mat(tmac_model_s* m, const std::string& name)
{
    auto it = m->mats.find(name);
    return it == m->mats.end() ? nullptr : it->second;
}

int prefill_run(tmac_model_s* m, int64_t M, int n_seq, int len, cudaStream_t s)
{
    PrefillState* p = m->prefill;
    int rc;
    pf_embed_kernel<<<(unsigned)M, 128, 0, s>>>(m->emb_raw, p->tokens, p->hidden);
    TMAC_CUDA_TRY(cudaGetLastError());
    const unsigned nblk8 = (unsigned)((M + 7) / 8);
    // attention: 4 queries per CTA while their scores fit in shared memory
    constexpr size_t kMaxAttnSmem = 227 * 1024;
    const int qb = attn_smem<4>(len) <= kMaxAttnSmem ? 4 : attn_smem<2>(len) <= kMaxAttnSmem ? 2 : 1;
    const size_t asmem = qb == 4 ? attn_smem<4>(len) : qb == 2 ? attn_smem<2>(len) : attn_smem<1>(len);
    if (asmem > kMaxAttnSmem) return fail(TMAC_ERR_SHAPE, "prefill: sequence too long for the attention kernel");
    {
        static bool attr_done[3] = {};
        const int k = qb == 4 ? 0 : qb == 2 ? 1 : 2;
        if (!attr_done[k]) {
            auto fn = qb == 4 ? pf_attention_kernel<4> : qb == 2 ? pf_attention_kernel<2> : pf_attention_kernel<1>;
            TMAC_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxAttnSmem));
            attr_done[k] = true;
        }
    }
    const dim3 agrid((unsigned)n_seq, kKvHeads, (unsigned)((len + qb - 1) / qb));
    for (int l = 0; l < kLayers; l++) {
        const float* an = vec_or_null(m, lname(l, "attn_norm.weight"));
        const float* fn = vec_or_null(m, lname(l, "ffn_norm.weight"));
        if (!an || !fn) return fail(TMAC_ERR_INVALID, "missing norm weights");
        pf_rmsnorm_kernel<<<nblk8, 256, 0, s>>>(p->hidden, l == 0 ? nullptr : p->ffn, an, M, p->xh, p->xl, p->xs,
                                               nullptr, len);
        TMAC_CUDA_TRY(cudaGetLastError());
        if (tmac_weight_s* w = mat(m, lname(l, "attn_qkv"))) {
            if ((rc = pf_gemm(m, w, M, kHidden, p->qkv, kQkv, s))) return rc;
        } else {
            tmac_weight_s* qk = mat(m, lname(l, "attn_qk"));
            tmac_weight_s* v = mat(m, lname(l, "attn_v.weight"));
            if (!qk || !v) return fail(TMAC_ERR_INVALID, "missing attention matrices");
            if ((rc = pf_gemm(m, qk, M, kHidden, p->qkv, kQkv, s))) return rc;
            if (v->type == TMAC_TYPE_Q8_0) {
                if ((rc = pf_gemm_q8(m, lname(l, "attn_v.weight"), v, M, p->qkv + kHidden + kKvDim, kQkv, s)))
                    return rc;
            } else if ((rc = pf_gemm(m, v, M, kHidden, p->qkv + kHidden + kKvDim, kQkv, s))) {
                return rc;
            }
        }
        pf_rope_kernel<<<(unsigned)M, kHidden / 2 + kKvDim / 2, 0, s>>>(
            p->qkv, vec_or_null(m, lname(l, "attn_q.bias")), vec_or_null(m, lname(l, "attn_k.bias")),
            vec_or_null(m, lname(l, "attn_v.bias")), m->rope_c, m->rope_s, len, p->qr, p->kr, p->vr);
        TMAC_CUDA_TRY(cudaGetLastError());
        if (qb == 4)
            pf_attention_kernel<4><<<agrid, kAThreads, asmem, s>>>(p->qr, p->kr, p->vr, len, p->ctx);
        else if (qb == 2)
            pf_attention_kernel<2><<<agrid, kAThreads, asmem, s>>>(p->qr, p->kr, p->vr, len, p->ctx);
        else
            pf_attention_kernel<1><<<agrid, kAThreads, asmem, s>>>(p->qr, p->kr, p->vr, len, p->ctx);
        TMAC_CUDA_TRY(cudaGetLastError());
        if ((rc = quantize_rows(p->ctx, kHidden, (int)M, p->xh, p->xl, p->xs, s))) return rc;
        tmac_weight_s* wo = mat(m, lname(l, "attn_output.weight"));
        if (!wo || (rc = pf_gemm(m, wo, M, kHidden, p->attn, kHidden, s))) return wo ? rc : fail(TMAC_ERR_INVALID, "missing attn_output");
        pf_rmsnorm_kernel<<<nblk8, 256, 0, s>>>(p->hidden, p->attn, fn, M, p->xh, p->xl, p->xs, nullptr, len);
        TMAC_CUDA_TRY(cudaGetLastError());
        tmac_weight_s* gu = mat(m, lname(l, "ffn_gate_up"));
        if (!gu || (rc = pf_gemm(m, gu, M, kHidden, p->gu, 2 * kInter, s))) return gu ? rc : fail(TMAC_ERR_INVALID, "missing ffn_gate_up");
        pf_silu_kernel<<<(unsigned)M, kSiluThreads, 0, s>>>(p->gu, p->xh, p->xl, p->xs);
        TMAC_CUDA_TRY(cudaGetLastError());
        tmac_weight_s* wd = mat(m, lname(l, "ffn_down.weight"));
        if (!wd || (rc = pf_gemm(m, wd, M, kInter, p->ffn, kHidden, s))) return wd ? rc : fail(TMAC_ERR_INVALID, "missing ffn_down");
    }
    // last residual, output_norm of every sequence's last position, logits + top-1
    pf_rmsnorm_kernel<<<nblk8, 256, 0, s>>>(p->hidden, p->ffn, vec_or_null(m, "output_norm.weight"), M, nullptr,
                                           nullptr, nullptr, p->xlast, len);
    TMAC_CUDA_TRY(cudaGetLastError());
    TMAC_CUDA_TRY(cudaMemsetAsync(p->keys, 0, n_seq * sizeof(unsigned long long), s));
    return launch_q8_0(m->mats["token_embd.weight"], p->xlast, p->logits, nullptr, nullptr, n_seq, s, p->keys, 0);
}

}  // namespace

void prefill_free(tmac_model_s* m)
{
    if (!m->prefill) return;
    for (void* a : m->prefill->allocs) cudaFree(a);
    for (void* a : m->prefill->plane_allocs) cudaFree(a);
    delete m->prefill;
    m->prefill = nullptr;
}

}  // namespace tmac

using namespace tmac;

extern "C" int tmac_model_prefill(tmac_model_t m, const int* tokens, int n_seq, int len, int* next_tokens,
                                  float* hidden_out, void* stream)
{
    if (!m || !tokens) return fail(TMAC_ERR_INVALID, "NULL model or tokens");
    if (!m->final) return fail(TMAC_ERR_INVALID, "model not finalized");
    if (n_seq <= 0 || len <= 0 || len > m->max_seq) return fail(TMAC_ERR_SHAPE, "need 0 < len <= max_seq, n_seq > 0");
    for (const auto& kv : m->mats)
        if (kv.second->mode != TMAC_MODE_NATIVE)
            return fail(TMAC_ERR_TYPE, "prefill needs every matrix on its FPGA-core path (all --fpga-* switches)");
    DeviceGuard dg(m->device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    const int64_t M = (int64_t)n_seq * len;
    int rc = ensure_state(m, M, n_seq);
    if (rc) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    PrefillState* p = m->prefill;
    TMAC_CUDA_TRY(cudaMemcpyAsync(p->tokens, tokens, M * sizeof(int), cudaMemcpyHostToDevice, s));
    if ((rc = prefill_run(m, M, n_seq, len, s))) return rc;
    if (next_tokens) {
        std::vector<unsigned long long> keys(n_seq);
        TMAC_CUDA_TRY(cudaMemcpyAsync(keys.data(), p->keys, n_seq * sizeof(unsigned long long), cudaMemcpyDeviceToHost, s));
        TMAC_CUDA_TRY(cudaStreamSynchronize(s));
        for (int i = 0; i < n_seq; i++) next_tokens[i] = (int)(0x7FFFFFFFu - (uint32_t)(keys[i] & 0x7FFFFFFFu));
    }
    if (hidden_out) {
        TMAC_CUDA_TRY(cudaMemcpyAsync(hidden_out, p->hidden, M * kHidden * sizeof(float), cudaMemcpyDeviceToHost, s));
    }
    TMAC_CUDA_TRY(cudaStreamSynchronize(s));
    return TMAC_OK;
}
