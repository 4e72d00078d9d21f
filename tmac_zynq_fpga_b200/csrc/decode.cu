// decode.cu -- device-resident greedy decode of the Qwen2-0.5B-shaped model:
// the reference's forward_layer_with_cache / get_logits_q8 / generate loop
// (sim/tmac_gguf.cpp:1559-1711, :1820-1845, :2025-2047) with every matmul on
// the library's GEMV kernels (dispatch by the --fpga-* switches as matmul(),
// :473-493) and the context ops as small CUDA kernels below.
//
// Numerics of the context ops follow the reference's operation order (fp32,
// no FMA contraction, sequential sums where the reference sums sequentially):
//   rms_norm  :447-454   sum x^2 in order, scale = 1/sqrtf(sum/n + 1e-6), o = x*w*scale
//   rope      :1528-1554 adjacent pairs (d, d+1); cos/sin tables computed on the
//             host with the reference's own float expression (glibc), uploaded
//   attention :1625-1660 scores in d order, /sqrtf(64), log-sum-exp softmax,
//             context accumulated in position order
//   silu      :459-461   x / (1 + expf(-x)), then * up
// expf/logf are evaluated as (float)exp((double)x) like glibc; any remaining
// last-ulp difference is why decode parity is stated as identical greedy tokens
// plus a hidden-state tolerance.
#include "common.cuh"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace tmac {
namespace {

constexpr int kHidden = 896, kInter = 4864, kVocab = 151936, kLayers = 24;
constexpr int kHeads = 14, kKvHeads = 2, kHeadDim = 64, kKvDim = kKvHeads * kHeadDim;

// glibc's expf / logf evaluate in double precision and round once, which makes
// them correctly rounded in nearly all cases; doing the same here reproduces
// the reference's values far more often than the single-precision intrinsics.
TMAC_DEV float expf_ref(float x) { return (float)exp((double)x); }
TMAC_DEV float logf_ref(float x) { return (float)log((double)x); }

// ------------------------------------------------------------------ kernels
// Embedding row of a Q8_0 token_embd (read_embedding / dequant_q8_0, :225-234,
// :413-427).  The token comes from a host int (token >= 0) or a device top-1 key.
__global__ void embed_q8_kernel(const uint8_t* __restrict__ emb, int token, const unsigned long long* key,
                                int* token_log, float* __restrict__ hidden)
{
    int tok = token;
    if (key) {
        const unsigned long long k = *key;
        tok = (int)(0x7FFFFFFFu - (uint32_t)(k & 0x7FFFFFFFu));
    }
    if (tok < 0 || tok >= kVocab) tok = 0;
    if (token_log && threadIdx.x == 0 && blockIdx.x == 0) *token_log = tok;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kHidden; i += gridDim.x * blockDim.x) {
        const int64_t idx = (int64_t)tok * kHidden + i;
        const uint8_t* b = emb + (idx / 32) * 34;
        hidden[i] = __fmul_rn((float)(int8_t)b[2 + idx % 32], f16_bits_to_f32(ld_u16_unaligned(b)));
    }
}

// rms_norm (:447-454): one CTA; the sum of squares is sequential, as in the
// reference (x staged in shared memory first).  With xq != nullptr the kernel
// also quantises its output for the matmuls that read it (:889-896).
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                      float* __restrict__ o, int16_t* __restrict__ xq,
                                                      float* __restrict__ xs, int n)
{
    __shared__ float xsh[kInter];
    __shared__ float red[8];
    __shared__ float scale;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xsh[i] = x[i];
    __syncthreads();
    if (threadIdx.x == 0) {
        float sum = 0.0f;
#pragma unroll 8
        for (int i = 0; i < n; i++) sum = __fadd_rn(sum, __fmul_rn(xsh[i], xsh[i]));
        const float mean = __fdiv_rn(sum, (float)n);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f)));
    }
    __syncthreads();
    float mx = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = __fmul_rn(__fmul_rn(xsh[i], w[i]), scale);
        o[i] = v;
        xsh[i] = v;
        mx = fmaxf(mx, fabsf(v));
    }
    if (!xq) return;
    mx = block_max(mx, red, blockDim.x);
    const float s = x_scale_from_max(mx);
    if (threadIdx.x == 0) *xs = s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xq[i] = quantize_one(xsh[i], s);
}

// q/k/v bias add (:1591-1614), RoPE on q and k (:1528-1554), KV-cache append (:1622-1623).
__global__ void qkv_rope_kernel(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v,
                                const float* __restrict__ bq, const float* __restrict__ bk,
                                const float* __restrict__ bv, const float* __restrict__ cs,
                                const float* __restrict__ sn, int pos, float* __restrict__ kc,
                                float* __restrict__ vc)
{
    const float* c = cs + (int64_t)pos * (kHeadDim / 2);
    const float* s = sn + (int64_t)pos * (kHeadDim / 2);
    for (int p = threadIdx.x; p < (kHidden + kKvDim) / 2; p += blockDim.x) {
        const bool isq = p < kHidden / 2;
        float* vec = isq ? q : k;
        const float* b = isq ? bq : bk;
        const int idx = 2 * (isq ? p : p - kHidden / 2);
        const int d = idx % kHeadDim;
        const float x0 = __fadd_rn(vec[idx], b ? b[idx] : 0.0f), x1 = __fadd_rn(vec[idx + 1], b ? b[idx + 1] : 0.0f);
        const float cv = c[d / 2], sv = s[d / 2];
        const float y0 = __fsub_rn(__fmul_rn(x0, cv), __fmul_rn(x1, sv));
        const float y1 = __fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, cv));
        vec[idx] = y0;
        vec[idx + 1] = y1;
        if (!isq) {
            kc[(int64_t)pos * kKvDim + idx] = y0;
            kc[(int64_t)pos * kKvDim + idx + 1] = y1;
        }
    }
    for (int i = threadIdx.x; i < kKvDim; i += blockDim.x)
        vc[(int64_t)pos * kKvDim + i] = __fadd_rn(v[i], bv ? bv[i] : 0.0f);
}

// Attention of one query head over positions 0..pos (:1625-1660): one CTA per head.
__global__ void __launch_bounds__(256) attention_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                        const float* __restrict__ vc, int pos,
                                                        float* __restrict__ ctx)
{
    extern __shared__ float sc[];  // [pos + 1] scores, then weights
    __shared__ float qs[kHeadDim];
    __shared__ float log_sum;
    const int h = blockIdx.x, kv = h / (kHeads / kKvHeads);
    for (int d = threadIdx.x; d < kHeadDim; d += blockDim.x) qs[d] = q[h * kHeadDim + d];
    __syncthreads();
    for (int p = threadIdx.x; p <= pos; p += blockDim.x) {
        const float* kp = kc + (int64_t)p * kKvDim + kv * kHeadDim;
        float s = 0.0f;
        for (int d = 0; d < kHeadDim; d++) s = __fadd_rn(s, __fmul_rn(qs[d], kp[d]));
        sc[p] = __fdiv_rn(s, 8.0f);  // / sqrtf(64)
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float mx = sc[0];
        for (int p = 1; p <= pos; p++) mx = sc[p] > mx ? sc[p] : mx;
        float es = 0.0f;
        for (int p = 0; p <= pos; p++) es = __fadd_rn(es, expf_ref(__fsub_rn(sc[p], mx)));
        log_sum = __fadd_rn(logf_ref(es), mx);
    }
    __syncthreads();
    for (int p = threadIdx.x; p <= pos; p += blockDim.x) sc[p] = expf_ref(__fsub_rn(sc[p], log_sum));
    __syncthreads();
    for (int d = threadIdx.x; d < kHeadDim; d += blockDim.x) {
        float a = 0.0f;
        for (int p = 0; p <= pos; p++) a = __fadd_rn(a, __fmul_rn(sc[p], vc[(int64_t)p * kKvDim + kv * kHeadDim + d]));
        ctx[h * kHeadDim + d] = a;
    }
}

__global__ void add_kernel(float* __restrict__ h, const float* __restrict__ a, int n)
{
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) h[i] = __fadd_rn(h[i], a[i]);
}

// silu(gate) * up (:459-461, :1697-1700), then the quantisation ffn_down's
// matmul starts with: one CTA.
__global__ void __launch_bounds__(1024) silu_mul_kernel(float* __restrict__ g, const float* __restrict__ u, int n,
                                                        int16_t* __restrict__ xq, float* __restrict__ xs)
{
    __shared__ float red[32];
    float mx = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = g[i];
        const float v = __fmul_rn(__fdiv_rn(x, __fadd_rn(1.0f, expf_ref(-x))), u[i]);
        g[i] = v;
        mx = fmaxf(mx, fabsf(v));
    }
    if (!xq) return;
    mx = block_max(mx, red, blockDim.x);
    const float s = x_scale_from_max(mx);
    if (threadIdx.x == 0) *xs = s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xq[i] = quantize_one(g[i], s);
}

// ----------------------------------------------------------------- the model
struct HostTensor {
    int64_t rows = 0, cols = 0;
    int type = 0;
    std::vector<uint8_t> data;
};

}  // namespace
}  // namespace tmac

struct tmac_model_s {
    int device = 0, switches = 0, max_seq = 0;
    std::map<std::string, tmac::HostTensor> host;  // until finalize
    bool final = false;
    // device state
    std::map<std::string, tmac_weight_t> mats;
    std::map<std::string, float*> vecs;
    uint8_t* emb_raw = nullptr;
    float *hidden = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *ctx = nullptr,
          *attn = nullptr, *gate = nullptr, *up = nullptr, *ffn = nullptr, *logits = nullptr;
    float *kcache = nullptr, *vcache = nullptr, *rope_c = nullptr, *rope_s = nullptr;
    unsigned long long* key = nullptr;
    int* token_log = nullptr;
    int16_t* xq = nullptr;  // quantised activations shared by several matmuls
    float* xs = nullptr;
    std::vector<void*> allocs;
};

namespace tmac {
namespace {

int mode_for(int switches, int type)
{
    if (!(switches & TMAC_SW_FPGA)) return TMAC_MODE_F32;
    if (type == TMAC_TYPE_Q5_0 && (switches & TMAC_SW_Q5_0)) return TMAC_MODE_NATIVE;
    if (type == TMAC_TYPE_Q6_K && (switches & TMAC_SW_Q6_K)) return TMAC_MODE_NATIVE;
    if (type == TMAC_TYPE_Q4_K && (switches & TMAC_SW_Q4_K)) return TMAC_MODE_NATIVE;
    if (type == TMAC_TYPE_Q8_0 && (switches & TMAC_SW_Q8)) return TMAC_MODE_NATIVE;
    return TMAC_MODE_INT16;
}

template <typename T>
int dev_alloc(tmac_model_s* m, T** p, size_t n)
{
    TMAC_CUDA_TRY(cudaMalloc((void**)p, n * sizeof(T)));
    m->allocs.push_back(*p);
    return TMAC_OK;
}

std::string lname(int l, const char* suffix)
{
    char b[128];
    snprintf(b, sizeof(b), "blk.%d.%s", l, suffix);
    return b;
}

// y = W.x; when the activation was already quantised (xq) and W runs a
// NATIVE kernel, the kernel reads x_q instead of quantising x again.
int gemv(tmac_model_s* m, const std::string& name, const float* x, float* y, cudaStream_t s, bool have_xq = false)
{
    auto it = m->mats.find(name);
    if (it == m->mats.end()) return fail(TMAC_ERR_INVALID, "missing matrix " + name);
    if (have_xq && it->second->mode == TMAC_MODE_NATIVE) return tmac_gemv_xq(it->second, m->xq, m->xs, y, 1, s);
    return tmac_gemv(it->second, x, y, 1, s);
}

const float* vec_or_null(tmac_model_s* m, const std::string& name)
{
    auto it = m->vecs.find(name);
    return it == m->vecs.end() ? nullptr : it->second;
}

int layer(tmac_model_s* m, int l, int pos, cudaStream_t s)
{
    int rc;
    const float* an = vec_or_null(m, lname(l, "attn_norm.weight"));
    const float* fn = vec_or_null(m, lname(l, "ffn_norm.weight"));
    if (!an || !fn) return fail(TMAC_ERR_INVALID, "missing norm weights");
    float* kc = m->kcache + (int64_t)l * m->max_seq * kKvDim;
    float* vc = m->vcache + (int64_t)l * m->max_seq * kKvDim;
    rmsnorm_kernel<<<1, 256, 0, s>>>(m->hidden, an, m->xn, m->xq, m->xs, kHidden);
    if ((rc = gemv(m, lname(l, "attn_q.weight"), m->xn, m->q, s, true))) return rc;
    if ((rc = gemv(m, lname(l, "attn_k.weight"), m->xn, m->k, s, true))) return rc;
    if ((rc = gemv(m, lname(l, "attn_v.weight"), m->xn, m->v, s, true))) return rc;
    qkv_rope_kernel<<<1, 512, 0, s>>>(m->q, m->k, m->v, vec_or_null(m, lname(l, "attn_q.bias")),
                                      vec_or_null(m, lname(l, "attn_k.bias")), vec_or_null(m, lname(l, "attn_v.bias")),
                                      m->rope_c, m->rope_s, pos, kc, vc);
    attention_kernel<<<kHeads, 256, (pos + 1) * sizeof(float), s>>>(m->q, kc, vc, pos, m->ctx);
    if ((rc = gemv(m, lname(l, "attn_output.weight"), m->ctx, m->attn, s))) return rc;
    add_kernel<<<4, 256, 0, s>>>(m->hidden, m->attn, kHidden);
    rmsnorm_kernel<<<1, 256, 0, s>>>(m->hidden, fn, m->xn, m->xq, m->xs, kHidden);
    if ((rc = gemv(m, lname(l, "ffn_gate.weight"), m->xn, m->gate, s, true))) return rc;
    if ((rc = gemv(m, lname(l, "ffn_up.weight"), m->xn, m->up, s, true))) return rc;
    silu_mul_kernel<<<1, 1024, 0, s>>>(m->gate, m->up, kInter, m->xq, m->xs);
    if ((rc = gemv(m, lname(l, "ffn_down.weight"), m->gate, m->ffn, s, true))) return rc;
    add_kernel<<<4, 256, 0, s>>>(m->hidden, m->ffn, kHidden);
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

int model_ok(tmac_model_t m, bool need_final = true)
{
    if (!m) return fail(TMAC_ERR_INVALID, "NULL model");
    if (need_final && !m->final) return fail(TMAC_ERR_INVALID, "model not finalized");
    return TMAC_OK;
}

}  // namespace
}  // namespace tmac

using namespace tmac;

extern "C" {

int tmac_model_create(int device, int switches, int max_seq, tmac_model_t* out)
{
    if (!out) return fail(TMAC_ERR_INVALID, "NULL out");
    if (max_seq <= 0 || max_seq > 4096) return fail(TMAC_ERR_SHAPE, "max_seq must be in 1..4096");
    tmac_model_s* m = new tmac_model_s();
    m->device = device;
    m->switches = switches;
    m->max_seq = max_seq;
    *out = m;
    return TMAC_OK;
}

int tmac_model_add_tensor(tmac_model_t m, const char* name, int64_t rows, int64_t cols, int type, const void* data,
                          size_t n_bytes)
{
    int rc = model_ok(m, false);
    if (rc) return rc;
    if (m->final) return fail(TMAC_ERR_INVALID, "model already finalized");
    if (!name || !data) return fail(TMAC_ERR_INVALID, "NULL name or data");
    HostTensor t;
    t.rows = rows;
    t.cols = cols;
    t.type = type;
    t.data.assign((const uint8_t*)data, (const uint8_t*)data + n_bytes);
    m->host[name] = std::move(t);
    return TMAC_OK;
}

int tmac_model_load_tmac(tmac_model_t m, const char* path)
{
    int rc = model_ok(m, false);
    if (rc) return rc;
    FILE* f = fopen(path, "rb");
    if (!f) return fail(TMAC_ERR_INVALID, std::string("cannot open ") + path);
    char magic[4];
    uint64_t n = 0;
    bool ok = fread(magic, 1, 4, f) == 4 && memcmp(magic, "TMAC", 4) == 0 && fread(&n, 8, 1, f) == 1;
    for (uint64_t i = 0; ok && i < n; i++) {
        uint64_t ln, rows, cols, nb;
        uint32_t type;
        ok = fread(&ln, 8, 1, f) == 1 && ln < 4096;
        std::string name(ok ? ln : 0, '\0');
        ok = ok && fread(&name[0], 1, ln, f) == ln && fread(&rows, 8, 1, f) == 1 && fread(&cols, 8, 1, f) == 1 &&
             fread(&type, 4, 1, f) == 1 && fread(&nb, 8, 1, f) == 1;
        if (!ok) break;
        HostTensor t;
        t.rows = (int64_t)rows;
        t.cols = (int64_t)cols;
        t.type = (int)type;
        t.data.resize(nb);
        ok = fread(t.data.data(), 1, nb, f) == nb;
        m->host[name] = std::move(t);
    }
    fclose(f);
    return ok ? TMAC_OK : fail(TMAC_ERR_INVALID, std::string("malformed .tmac file ") + path);
}

int tmac_model_finalize(tmac_model_t m)
{
    int rc = model_ok(m, false);
    if (rc) return rc;
    if (m->final) return TMAC_OK;
    DeviceGuard dg(m->device);
    auto emb = m->host.find("token_embd.weight");
    if (emb == m->host.end() || emb->second.type != TMAC_TYPE_Q8_0 || emb->second.rows != kVocab ||
        emb->second.cols != kHidden)
        return fail(TMAC_ERR_SHAPE, "token_embd.weight must be Q8_0 151936 x 896");
    for (auto& kv : m->host) {
        const std::string& name = kv.first;
        HostTensor& t = kv.second;
        if (name.size() > 12 && name.compare(name.size() - 12, 12, "_row_max_abs") == 0) continue;
        if (t.cols == 1) {
            if (t.type != TMAC_TYPE_F32) return fail(TMAC_ERR_TYPE, "vector tensor " + name + " must be F32");
            float* d = nullptr;
            if ((rc = dev_alloc(m, &d, (size_t)t.rows))) return rc;
            TMAC_CUDA_TRY(cudaMemcpy(d, t.data.data(), t.rows * sizeof(float), cudaMemcpyHostToDevice));
            m->vecs[name] = d;
            continue;
        }
        const float* rma = nullptr;
        auto rt = m->host.find(name + "_row_max_abs");
        if (rt != m->host.end() && rt->second.type == TMAC_TYPE_F32 && rt->second.cols == 1)
            rma = reinterpret_cast<const float*>(rt->second.data.data());
        // token_embd is the tied output: get_logits_q8 (:1820) uses the Q8_0 path with
        // the row_max_abs table when --fpga-q8 is on, else matmul() (:1848-1866).
        tmac_weight_t w = nullptr;
        rc = tmac_weight_register(t.type, mode_for(m->switches, t.type), t.rows, t.cols, t.data.data(),
                                  t.data.size(), 0, rma, m->device, &w);
        if (rc) return rc;
        m->mats[name] = w;
    }
    if ((rc = dev_alloc(m, &m->emb_raw, emb->second.data.size()))) return rc;
    TMAC_CUDA_TRY(cudaMemcpy(m->emb_raw, emb->second.data.data(), emb->second.data.size(), cudaMemcpyHostToDevice));
    const size_t kv = (size_t)kLayers * m->max_seq * kKvDim;
    if ((rc = dev_alloc(m, &m->hidden, kHidden)) || (rc = dev_alloc(m, &m->xn, kHidden)) ||
        (rc = dev_alloc(m, &m->q, kHidden)) || (rc = dev_alloc(m, &m->k, kKvDim)) ||
        (rc = dev_alloc(m, &m->v, kKvDim)) || (rc = dev_alloc(m, &m->ctx, kHidden)) ||
        (rc = dev_alloc(m, &m->attn, kHidden)) || (rc = dev_alloc(m, &m->gate, kInter)) ||
        (rc = dev_alloc(m, &m->up, kInter)) || (rc = dev_alloc(m, &m->ffn, kHidden)) ||
        (rc = dev_alloc(m, &m->logits, kVocab)) || (rc = dev_alloc(m, &m->kcache, kv)) ||
        (rc = dev_alloc(m, &m->vcache, kv)) || (rc = dev_alloc(m, &m->key, 1)) ||
        (rc = dev_alloc(m, &m->token_log, 1)) || (rc = dev_alloc(m, &m->xq, kInter)) ||
        (rc = dev_alloc(m, &m->xs, 1)))
        return rc;
    // RoPE tables with the reference's own float expression (apply_rope, :1528-1554)
    std::vector<float> c((size_t)m->max_seq * 32), sn((size_t)m->max_seq * 32);
    for (int pos = 0; pos < m->max_seq; pos++)
        for (int d = 0; d < kHeadDim; d += 2) {
            const float theta = 1.0f / powf(1000000.0f, (float)d / kHeadDim);
            const float freq = pos * theta;
            c[(size_t)pos * 32 + d / 2] = cosf(freq);
            sn[(size_t)pos * 32 + d / 2] = sinf(freq);
        }
    if ((rc = dev_alloc(m, &m->rope_c, c.size())) || (rc = dev_alloc(m, &m->rope_s, sn.size()))) return rc;
    TMAC_CUDA_TRY(cudaMemcpy(m->rope_c, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice));
    TMAC_CUDA_TRY(cudaMemcpy(m->rope_s, sn.data(), sn.size() * sizeof(float), cudaMemcpyHostToDevice));
    TMAC_CUDA_TRY(cudaMemset(m->kcache, 0, kv * sizeof(float)));
    TMAC_CUDA_TRY(cudaMemset(m->vcache, 0, kv * sizeof(float)));
    m->host.clear();
    m->final = true;
    return TMAC_OK;
}

int tmac_model_reset(tmac_model_t m, void* stream)
{
    int rc = model_ok(m);
    if (rc) return rc;
    DeviceGuard dg(m->device);
    const size_t kv = (size_t)kLayers * m->max_seq * kKvDim * sizeof(float);
    TMAC_CUDA_TRY(cudaMemsetAsync(m->kcache, 0, kv, (cudaStream_t)stream));
    TMAC_CUDA_TRY(cudaMemsetAsync(m->vcache, 0, kv, (cudaStream_t)stream));
    return TMAC_OK;
}

int tmac_model_forward(tmac_model_t m, int token, int pos, void* stream)
{
    int rc = model_ok(m);
    if (rc) return rc;
    if (pos < 0 || pos >= m->max_seq) return fail(TMAC_ERR_SHAPE, "pos outside the KV cache");
    if (token >= kVocab) return fail(TMAC_ERR_SHAPE, "token id out of range");
    DeviceGuard dg(m->device);
    cudaStream_t s = (cudaStream_t)stream;
    embed_q8_kernel<<<4, 256, 0, s>>>(m->emb_raw, token, token < 0 ? m->key : nullptr, m->token_log, m->hidden);
    for (int l = 0; l < kLayers; l++)
        if ((rc = layer(m, l, pos, s))) return rc;
    return TMAC_OK;
}

int tmac_model_logits(tmac_model_t m, void* stream)
{
    int rc = model_ok(m);
    if (rc) return rc;
    DeviceGuard dg(m->device);
    cudaStream_t s = (cudaStream_t)stream;
    const float* on = vec_or_null(m, "output_norm.weight");
    const float* x = m->hidden;
    if (on) {
        rmsnorm_kernel<<<1, 256, 0, s>>>(m->hidden, on, m->xn, nullptr, nullptr, kHidden);
        x = m->xn;
    }
    return tmac_gemv_top1(m->mats["token_embd.weight"], x, m->logits, (uint64_t*)m->key, 0, 1, stream);
}

int tmac_model_buffers(tmac_model_t m, float** hidden, float** logits, uint64_t** key)
{
    int rc = model_ok(m);
    if (rc) return rc;
    if (hidden) *hidden = m->hidden;
    if (logits) *logits = m->logits;
    if (key) *key = (uint64_t*)m->key;
    return TMAC_OK;
}

int tmac_model_generate(tmac_model_t m, const int* prompt, int n_prompt, int n_gen, int* out_tokens,
                        float* out_hidden, void* stream)
{
    int rc = model_ok(m);
    if (rc) return rc;
    if (!prompt || n_prompt <= 0 || n_gen < 0 || !out_tokens) return fail(TMAC_ERR_INVALID, "bad arguments");
    if (n_prompt + n_gen > m->max_seq) return fail(TMAC_ERR_SHAPE, "prompt + generation exceed the KV cache");
    DeviceGuard dg(m->device);
    cudaStream_t s = (cudaStream_t)stream;
    if ((rc = tmac_model_reset(m, stream))) return rc;
    for (int t = 0; t < n_prompt; t++)
        if ((rc = tmac_model_forward(m, prompt[t], t, stream))) return rc;
    if (out_hidden) {
        TMAC_CUDA_TRY(cudaMemcpyAsync(out_hidden, m->hidden, kHidden * sizeof(float), cudaMemcpyDeviceToHost, s));
    }
    for (int g = 0; g < n_gen; g++) {
        // logits of the current hidden state, greedy token (device key), its
        // embedding and the next forward pass: no host round trip per step.
        if ((rc = tmac_model_logits(m, stream))) return rc;
        if ((rc = tmac_model_forward(m, -1, n_prompt + g, stream))) return rc;
        TMAC_CUDA_TRY(cudaMemcpyAsync(out_tokens + g, m->token_log, sizeof(int), cudaMemcpyDeviceToHost, s));
        if (out_hidden)
            TMAC_CUDA_TRY(cudaMemcpyAsync(out_hidden + (size_t)(g + 1) * kHidden, m->hidden, kHidden * sizeof(float),
                                          cudaMemcpyDeviceToHost, s));
    }
    TMAC_CUDA_TRY(cudaStreamSynchronize(s));
    return TMAC_OK;
}

int tmac_model_free(tmac_model_t m)
{
    if (!m) return TMAC_OK;
    DeviceGuard dg(m->device);
    for (auto& kv : m->mats) tmac_weight_free(kv.second);
    for (void* p : m->allocs) cudaFree(p);
    delete m;
    return TMAC_OK;
}

}  // extern "C"
