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
#include "decode_ops.cuh"

#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace tmac {
namespace {


// ------------------------------------------------------------------ kernels
// Embedding row of a Q8_0 token_embd (read_embedding / dequant_q8_0, :225-234,
// :413-427).  The token comes from a host int (token >= 0) or a device top-1 key.
__global__ void embed_q8_kernel(const uint8_t* __restrict__ emb, int token, const unsigned long long* key,
                                int* token_log, float* __restrict__ hidden, const int* pos_dev, int* tokens,
                                int n_prompt)
{
    pdl_launch();
    pdl_wait();
    // token: a host id; or (pos_dev) the prompt token tokens[pos] while
    // pos < n_prompt, else the greedy token of the device top-1 key.
    int tok = token;
    int p = 0;
    if (pos_dev) {
        p = *pos_dev;
        if (p < n_prompt) tok = tokens[p];
        else tok = -1;
    }
    if (tok < 0 && key) {
        const unsigned long long k = *key;
        tok = (int)(0x7FFFFFFFu - (uint32_t)(k & 0x7FFFFFFFu));
    }
    if (tok < 0 || tok >= kVocab) tok = 0;
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        if (token_log) *token_log = tok;
        if (pos_dev) tokens[p] = tok;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < kHidden; i += gridDim.x * blockDim.x) {
        const int64_t idx = (int64_t)tok * kHidden + i;
        const uint8_t* b = emb + (idx / 32) * 34;
        hidden[i] = __fmul_rn((float)(int8_t)b[2 + idx % 32], f16_bits_to_f32(ld_u16_unaligned(b)));
    }
}

// End of one token: log the hidden state at its position, advance the position.
__global__ void step_done_kernel(const float* __restrict__ hidden, float* __restrict__ hidden_log, int* pos_dev,
                                 unsigned long long* key)
{
    pdl_launch();
    pdl_wait();
    const int p = *pos_dev;
    for (int i = threadIdx.x; i < kHidden; i += blockDim.x) hidden_log[(int64_t)p * kHidden + i] = hidden[i];
    __syncthreads();
    if (threadIdx.x == 0) {
        *pos_dev = p + 1;
        *key = 0;  // ready for the next step's top-1 (atomic max)
    }
}

// x_q value i of an n-vector as int16 (Q8_0 kernels) and as byte planes
// (block-quant kernels).
TMAC_DEV void store_xq(int16_t* xq, uint8_t* xp, int n, int i, int16_t q)
{
    xq[i] = q;
    if (xp) {
        xp[i] = (uint8_t)((uint16_t)q >> 8);
        xp[n + i] = (uint8_t)(q & 0xFF);
    }
}

// rms_norm (:447-454): one CTA; the sum of squares is sequential, as in the
// reference (x staged in shared memory first).  With xq != nullptr the kernel
// also quantises its output for the matmuls that read it (:889-896).
// With delta != nullptr the residual add comes first (x += delta, written back:
// :1669 / :1710).  w == nullptr copies x unnormalised (get_logits_q8 without an
// output_norm tensor, :1831-1838).
__global__ void __launch_bounds__(256) rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ delta,
                                                      const float* __restrict__ w, float* __restrict__ o,
                                                      int16_t* __restrict__ xq, uint8_t* __restrict__ xp,
                                                      float* __restrict__ xs, int n)
{
    pdl_launch();
    __shared__ __align__(16) float xsh[kInter];
    __shared__ float red[8];
    __shared__ float scale;
    // the norm weights do not depend on the preceding kernel
    float wv[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        wv[k] = (w && i < n) ? w[i] : 1.0f;
    }
    pdl_wait();
    // the squares in parallel (into xsh[n..2n), n <= kInter / 2), their sum in order
    float* sq = xsh + ((n + 3) & ~3);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float v = x[i];
        if (delta) {
            v = __fadd_rn(v, delta[i]);
            x[i] = v;
        }
        xsh[i] = v;
        sq[i] = __fmul_rn(v, v);
    }
    __syncthreads();
    if (threadIdx.x == 0) scale = w ? rms_scale(sq, n) : 1.0f;
    __syncthreads();
    float mx = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i >= n) break;
        const float v = w ? __fmul_rn(__fmul_rn(xsh[i], wv[k]), scale) : xsh[i];
        o[i] = v;
        xsh[i] = v;
        mx = fmaxf(mx, fabsf(v));
    }
    for (int i = threadIdx.x + 4 * blockDim.x; i < n; i += blockDim.x) {
        const float v = w ? __fmul_rn(__fmul_rn(xsh[i], w[i]), scale) : xsh[i];
        o[i] = v;
        xsh[i] = v;
        mx = fmaxf(mx, fabsf(v));
    }
    if (!xq) return;
    mx = block_max(mx, red, blockDim.x);
    const float s = x_scale_from_max(mx);
    if (threadIdx.x == 0) *xs = s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) store_xq(xq, xp, n, i, quantize_one(xsh[i], s));
}

// One CTA of 256 threads per query head (attention_prefetch + attention_head, decode_ops.cuh).
__global__ void __launch_bounds__(256) rope_attention_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ bq, const float* __restrict__ bk, const float* __restrict__ bv,
    const float* __restrict__ cs, const float* __restrict__ sn, int pos, const int* pos_dev, float* __restrict__ kc,
    float* __restrict__ vc, float* __restrict__ ctx, int nscore)
{
    pdl_launch();
    pdl_wait();
    extern __shared__ __align__(16) float sc[];  // [nsc] scores, then weights; [nsc] exp terms; K/V staging
    __shared__ AttnShared sh;
    if (pos_dev) pos = *pos_dev;
    attention_prefetch(blockIdx.x, kc, vc, pos, nscore, sc, bq, bk, bv, cs, sn, sh);
    const int h = blockIdx.x, kvh = h / (kHeads / kKvHeads);
    attention_head(h, q + h * kHeadDim, k + kvh * kHeadDim, v + kvh * kHeadDim, pos, kc, vc, ctx + h * kHeadDim,
                   nscore, sc, sh, 1);
}

// silu(gate) * up (:459-461, :1697-1700), then the quantisation ffn_down's
// matmul starts with: one CTA.
__global__ void __launch_bounds__(1024) silu_mul_kernel(float* __restrict__ g, const float* __restrict__ u, int n,
                                                        int16_t* __restrict__ xq, uint8_t* __restrict__ xp,
                                                        float* __restrict__ xs)
{
    pdl_launch();
    pdl_wait();
    __shared__ float red[32];
    float mx = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float x = g[i];
        const float v = silu_mul(x, u[i]);
        g[i] = v;
        mx = fmaxf(mx, fabsf(v));
    }
    if (!xq) return;
    mx = block_max(mx, red, blockDim.x);
    const float s = x_scale_from_max(mx);
    if (threadIdx.x == 0) *xs = s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) store_xq(xq, xp, n, i, quantize_one(g[i], s));
}

// silu(gate) * up over kSiluCtas CTAs, one value per thread, written back in
// place; each CTA leaves the maximum |h| of its slice, and ffn_down's GEMV
// quantises h itself from the maximum of those (no single-CTA reduction).
static_assert(kSiluCtas * 256 == kInter, "one value per thread");
__global__ void __launch_bounds__(256) silu_part_kernel(float* __restrict__ g, const float* __restrict__ u,
                                                        float* __restrict__ part_max)
{
    pdl_launch();
    pdl_wait();
    __shared__ float red[8];
    const int i = blockIdx.x * 256 + threadIdx.x;
    const float x = g[i];
    const float v = silu_mul(x, u[i]);
    g[i] = v;
    float mx = fabsf(v);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; w++) mx = fmaxf(mx, red[w]);
        part_max[blockIdx.x] = fmaxf(mx, red[0]);
    }
}

}  // namespace
}  // namespace tmac

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



// y = W.x; when the activation was already quantised (xq) and W runs a
// NATIVE kernel, the kernel reads x_q instead of quantising x again.
int gemv(tmac_model_s* m, const std::string& name, const float* x, float* y, cudaStream_t s, bool have_xq = false)
{
    auto it = m->mats.find(name);
    if (it == m->mats.end()) return fail(TMAC_ERR_INVALID, "missing matrix " + name);
    const tmac_weight_s* w = it->second;
    if (have_xq && w->mode == TMAC_MODE_NATIVE) {
        if (w->type == TMAC_TYPE_Q8_0)
            return launch_q8_0(w, nullptr, y, nullptr, nullptr, 1, s, nullptr, 0, m->xq, m->xs);
        return launch_blockq(w, nullptr, nullptr, m->xp, m->xs, y, nullptr, nullptr, 1, s);
    }
    return tmac_gemv(it->second, x, y, 1, s);
}


const float* next_norm(tmac_model_s* m, int l)
{
    return l + 1 < kLayers ? vec_or_null(m, lname(l + 1, "attn_norm.weight")) : vec_or_null(m, "output_norm.weight");
}

// One layer.  On entry xn / xq / xs hold attn_norm(hidden) of this layer; on
// exit hidden has both residuals and xn / xq / xs hold the next layer's
// attn_norm(hidden) (or output_norm(hidden) after the last layer).
int layer(tmac_model_s* m, int l, int pos, cudaStream_t s, const int* pos_dev = nullptr)
{
    int rc;
    const float* fn = vec_or_null(m, lname(l, "ffn_norm.weight"));
    if (!fn) return fail(TMAC_ERR_INVALID, "missing ffn_norm weights");
    float* kc = m->kcache + (int64_t)l * m->max_seq * kKvDim;
    float* vc = m->vcache + (int64_t)l * m->max_seq * kKvDim;
    // q, k (and v when it has the same type) as one GEMV over concatenated rows
    if (m->mats.count(lname(l, "attn_qkv"))) {
        if ((rc = gemv(m, lname(l, "attn_qkv"), m->xn, m->q, s, true))) return rc;
    } else {
        if ((rc = gemv(m, lname(l, "attn_qk"), m->xn, m->q, s, true))) return rc;
        if ((rc = gemv(m, lname(l, "attn_v.weight"), m->xn, m->v, s, true))) return rc;
    }
    const int nscore = pos_dev ? m->max_seq : pos + 1;
    TMAC_CUDA_TRY(launch_k(rope_attention_kernel, dim3(kHeads), dim3(256),
                           attn_scratch_bytes(nscore), s, (const float*)m->q,
                           (const float*)m->k, (const float*)m->v, vec_or_null(m, lname(l, "attn_q.bias")),
                           vec_or_null(m, lname(l, "attn_k.bias")), vec_or_null(m, lname(l, "attn_v.bias")),
                           (const float*)m->rope_c, (const float*)m->rope_s, pos, pos_dev, kc, vc, m->ctx, nscore));
    if ((rc = gemv(m, lname(l, "attn_output.weight"), m->ctx, m->attn, s))) return rc;
    TMAC_CUDA_TRY(launch_k(rmsnorm_kernel, dim3(1), dim3(256), 0, s, m->hidden, (const float*)m->attn, fn, m->xn,
                           m->xq, m->xp, m->xs, kHidden));
    if ((rc = gemv(m, lname(l, "ffn_gate_up"), m->xn, m->gate, s, true))) return rc;
    const auto wdi = m->mats.find(lname(l, "ffn_down.weight"));
    const tmac_weight_s* wd = wdi == m->mats.end() ? nullptr : wdi->second;
    if (wd && wd->mode == TMAC_MODE_NATIVE && wd->type != TMAC_TYPE_Q8_0) {
        // h over several CTAs; the block-quant GEMV quantises it from their maxima
        TMAC_CUDA_TRY(launch_k(silu_part_kernel, dim3(kSiluCtas), dim3(256), 0, s, m->gate, (const float*)m->up,
                               m->silu_max));
        if ((rc = launch_blockq(wd, m->gate, nullptr, nullptr, nullptr, m->ffn, nullptr, nullptr, 1, s, m->silu_max,
                                kSiluCtas)))
            return rc;
    } else {
        TMAC_CUDA_TRY(launch_k(silu_mul_kernel, dim3(1), dim3(1024), 0, s, m->gate, (const float*)m->up, kInter,
                               m->xq, m->xp, m->xs));
        if ((rc = gemv(m, lname(l, "ffn_down.weight"), m->gate, m->ffn, s, true))) return rc;
    }
    TMAC_CUDA_TRY(launch_k(rmsnorm_kernel, dim3(1), dim3(256), 0, s, m->hidden, (const float*)m->ffn, next_norm(m, l),
                           m->xn, m->xq, m->xp, m->xs, kHidden));
    TMAC_CUDA_TRY(cudaGetLastError());
    return TMAC_OK;
}

// Embedding, then attn_norm of layer 0, then all layers.
int forward_all(tmac_model_s* m, int token, const unsigned long long* key, int pos, cudaStream_t s,
                const int* pos_dev, int n_prompt)
{
    int rc;
    TMAC_CUDA_TRY(launch_k(embed_q8_kernel, dim3(4), dim3(256), 0, s, (const uint8_t*)m->emb_raw, token, key,
                           m->token_log, m->hidden, pos_dev, m->tokens, n_prompt));
    const float* an = vec_or_null(m, lname(0, "attn_norm.weight"));
    if (!an) return fail(TMAC_ERR_INVALID, "missing attn_norm weights");
    TMAC_CUDA_TRY(launch_k(rmsnorm_kernel, dim3(1), dim3(256), 0, s, m->hidden, (const float*)nullptr, an, m->xn, m->xq,
                           m->xp, m->xs, kHidden));
    for (int l = 0; l < kLayers; l++)
        if ((rc = layer(m, l, pos, s, pos_dev))) return rc;
    return TMAC_OK;
}

// Logits of the current hidden state with the top-1 merged into m->key, which
// the caller has zeroed (step_done_kernel does it inside generation graphs).
int logits_into_key(tmac_model_s* m, cudaStream_t s)
{
    return launch_q8_0(m->mats["token_embd.weight"], m->xn, m->logits, nullptr, nullptr, 1, s, m->key, 0);
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
    // Matrices that read the same activation are registered as one weight over
    // their concatenated rows (q|k|v, gate|up): every output row is computed
    // independently, so the results are those of the separate matmuls.
    auto concat = [&](const std::vector<std::string>& parts, const std::string& name) {
        HostTensor t;
        t.type = m->host[parts[0]].type;
        t.cols = m->host[parts[0]].cols;
        for (const auto& p : parts) {
            HostTensor& h = m->host[p];
            t.rows += h.rows;
            t.data.insert(t.data.end(), h.data.begin(), h.data.end());
            m->host.erase(p);
        }
        m->host[name] = std::move(t);
    };
    for (int l = 0; l < kLayers; l++) {
        const std::string q = lname(l, "attn_q.weight"), k = lname(l, "attn_k.weight"), v = lname(l, "attn_v.weight");
        const std::string g = lname(l, "ffn_gate.weight"), u = lname(l, "ffn_up.weight");
        for (const auto& n : {q, k, v, g, u})
            if (!m->host.count(n)) return fail(TMAC_ERR_INVALID, "missing tensor " + n);
        if (m->host[q].type != m->host[k].type || m->host[g].type != m->host[u].type)
            return fail(TMAC_ERR_TYPE, "attn_q/attn_k and ffn_gate/ffn_up must share a type");
        if (m->host[v].type == m->host[q].type) concat({q, k, v}, lname(l, "attn_qkv"));
        else concat({q, k}, lname(l, "attn_qk"));
        concat({g, u}, lname(l, "ffn_gate_up"));
    }
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
        (rc = dev_alloc(m, &m->q, kHidden + 2 * kKvDim)) || (rc = dev_alloc(m, &m->ctx, kHidden)) ||
        (rc = dev_alloc(m, &m->attn, kHidden)) || (rc = dev_alloc(m, &m->gate, 2 * kInter)) ||
        (rc = dev_alloc(m, &m->ffn, kHidden)) ||
        (rc = dev_alloc(m, &m->logits, kVocab)) || (rc = dev_alloc(m, &m->kcache, kv)) ||
        (rc = dev_alloc(m, &m->vcache, kv)) || (rc = dev_alloc(m, &m->key, 1)) ||
        (rc = dev_alloc(m, &m->token_log, 1)) || (rc = dev_alloc(m, &m->xq, kInter)) ||
        (rc = dev_alloc(m, &m->xp, 2 * kInter)) ||
        (rc = dev_alloc(m, &m->xs, 1)) || (rc = dev_alloc(m, &m->pos_dev, 1)) ||
        (rc = dev_alloc(m, &m->silu_max, kSiluCtas)) ||
        (rc = dev_alloc(m, &m->tokens, (size_t)m->max_seq)) ||
        (rc = dev_alloc(m, &m->hidden_log, (size_t)m->max_seq * kHidden)))
        return rc;
    m->k = m->q + kHidden;  // q | k | v and gate | up are contiguous: the concatenated GEMV outputs
    m->v = m->k + kKvDim;
    m->up = m->gate + kInter;
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
    // the attention's score slots grow with the KV cache (above 48 KB past ~1400 positions)
    TMAC_CUDA_TRY(cudaFuncSetAttribute(rope_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)attn_scratch_bytes(m->max_seq)));
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
    if ((rc = forward_all(m, token, token < 0 ? m->key : nullptr, pos, s, nullptr, 0))) return rc;
    return TMAC_OK;
}

int tmac_model_logits(tmac_model_t m, void* stream)
{
    int rc = model_ok(m);
    if (rc) return rc;
    DeviceGuard dg(m->device);
    // xn already holds output_norm(hidden): the last layer's closing norm
    return tmac_gemv_top1(m->mats["token_embd.weight"], m->xn, m->logits, (uint64_t*)m->key, 0, 1, stream);
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
    (void)stream;  // generation runs on the model's own stream (graphs need a non-default stream)
    int rc = model_ok(m);
    if (rc) return rc;
    if (!prompt || n_prompt <= 0 || n_gen < 0 || !out_tokens) return fail(TMAC_ERR_INVALID, "bad arguments");
    if (n_prompt + n_gen > m->max_seq) return fail(TMAC_ERR_SHAPE, "prompt + generation exceed the KV cache");
    for (int t = 0; t < n_prompt; t++)
        if (prompt[t] < 0 || prompt[t] >= kVocab) return fail(TMAC_ERR_SHAPE, "prompt token id out of range");
    DeviceGuard dg(m->device);
    if (!m->stream) TMAC_CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
    cudaStream_t s = m->stream;
    // The persistent kernel (decode_mega.cu) runs a whole token in one launch
    // when every matrix is on its FPGA-core path; TMAC_DECODE=graph selects the
    // per-kernel engine below (identical results).
    const char* engine = getenv("TMAC_DECODE");
    const bool want_mega = !(engine && strcmp(engine, "graph") == 0);
    if (want_mega && m->mega_state == 0) {
        if ((rc = mega_prepare(m, &m->mega))) return rc;
        m->mega_state = m->mega ? 1 : -1;
    }
    if (want_mega && m->mega) {
        if ((rc = tmac_model_reset(m, s))) return rc;
        TMAC_CUDA_TRY(cudaMemsetAsync(m->key, 0, sizeof(unsigned long long), s));
        TMAC_CUDA_TRY(cudaMemcpyAsync(m->tokens, prompt, n_prompt * sizeof(int), cudaMemcpyHostToDevice, s));
        TMAC_CUDA_TRY(cudaMemsetAsync(m->pos_dev, 0, sizeof(int), s));
        for (int t = 0; t < n_prompt; t++)
            if ((rc = mega_launch(m->mega, n_prompt, s))) return rc;
        for (int g = 0; g < n_gen; g++) {
            if ((rc = logits_into_key(m, s))) return rc;  // xn = output_norm(hidden), left by the kernel
            if ((rc = mega_launch(m->mega, n_prompt, s))) return rc;
        }
        TMAC_CUDA_TRY(cudaStreamSynchronize(s));
        TMAC_CUDA_TRY(cudaMemcpy(out_tokens, m->tokens + n_prompt, n_gen * sizeof(int), cudaMemcpyDeviceToHost));
        if (out_hidden)
            TMAC_CUDA_TRY(cudaMemcpy(out_hidden, m->hidden_log + (size_t)(n_prompt - 1) * kHidden,
                                     (size_t)(n_gen + 1) * kHidden * sizeof(float), cudaMemcpyDeviceToHost));
        m->last_engine = 1;
        return TMAC_OK;
    }
    m->last_engine = 0;
    // One graph per step kind: a prompt step (embed + 24 layers) and a greedy
    // step (output norm + logits + top-1, then embed + 24 layers).  Position
    // and tokens live in device memory, so one capture serves every position.
    if (m->graph_n_prompt != n_prompt) {
        if (m->g_prompt) cudaGraphExecDestroy(m->g_prompt);
        if (m->g_gen) cudaGraphExecDestroy(m->g_gen);
        m->g_prompt = m->g_gen = nullptr;
        for (int kind = 0; kind < 2; kind++) {
            cudaGraph_t g = nullptr;
            PdlScope pdl;  // kernels of the step overlap their launch with the previous kernel
            TMAC_CUDA_TRY(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed));
            int crc = TMAC_OK;
            if (kind == 1) {
                tmac_weight_s* lw = m->mats["token_embd.weight"];
                if (lw->mode == TMAC_MODE_NATIVE) crc = logits_into_key(m, s);
                else crc = tmac_model_logits(m, s);
            }
            if (!crc) crc = forward_all(m, -1, m->key, 0, s, m->pos_dev, n_prompt);
            if (!crc) {
                cudaError_t le = launch_k(step_done_kernel, dim3(1), dim3(256), 0, s, (const float*)m->hidden,
                                          m->hidden_log, m->pos_dev, m->key);
                if (le != cudaSuccess) crc = cuda_fail(le, "step_done_kernel");
            }
            cudaError_t e = cudaStreamEndCapture(s, &g);
            if (crc) {
                if (g) cudaGraphDestroy(g);
                return crc;
            }
            if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture");
            e = cudaGraphInstantiate(kind ? &m->g_gen : &m->g_prompt, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate");
        }
        m->graph_n_prompt = n_prompt;
    }
    if ((rc = tmac_model_reset(m, s))) return rc;
    TMAC_CUDA_TRY(cudaMemsetAsync(m->key, 0, sizeof(unsigned long long), s));
    TMAC_CUDA_TRY(cudaMemcpyAsync(m->tokens, prompt, n_prompt * sizeof(int), cudaMemcpyHostToDevice, s));
    TMAC_CUDA_TRY(cudaMemsetAsync(m->pos_dev, 0, sizeof(int), s));
    for (int t = 0; t < n_prompt; t++) TMAC_CUDA_TRY(cudaGraphLaunch(m->g_prompt, s));
    for (int g = 0; g < n_gen; g++) TMAC_CUDA_TRY(cudaGraphLaunch(m->g_gen, s));
    TMAC_CUDA_TRY(cudaStreamSynchronize(s));
    TMAC_CUDA_TRY(cudaMemcpy(out_tokens, m->tokens + n_prompt, n_gen * sizeof(int), cudaMemcpyDeviceToHost));
    if (out_hidden)
        TMAC_CUDA_TRY(cudaMemcpy(out_hidden, m->hidden_log + (size_t)(n_prompt - 1) * kHidden,
                                 (size_t)(n_gen + 1) * kHidden * sizeof(float), cudaMemcpyDeviceToHost));
    return TMAC_OK;
}

int tmac_model_decode_engine(tmac_model_t m)
{
    if (!m) return -1;
    return m->last_engine;
}

int tmac_model_free(tmac_model_t m)
{
    if (!m) return TMAC_OK;
    DeviceGuard dg(m->device);
    if (m->g_prompt) cudaGraphExecDestroy(m->g_prompt);
    if (m->g_gen) cudaGraphExecDestroy(m->g_gen);
    if (m->stream) cudaStreamDestroy(m->stream);
    prefill_free(m);
    mega_free(m->mega);
    for (auto& kv : m->mats) tmac_weight_free(kv.second);
    for (void* p : m->allocs) cudaFree(p);
    delete m;
    return TMAC_OK;
}

}  // extern "C"
