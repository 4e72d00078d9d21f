// model.cuh -- the Qwen2-0.5B-shaped model object shared by the decode
// engine (decode.cu) and the batched prefill (prefill.cu).
#pragma once

#include "common.cuh"

#include <cmath>
#include <cstdio>
#include <map>
#include <string>
#include <vector>

namespace tmac {

constexpr int kHidden = 896, kInter = 4864, kVocab = 151936, kLayers = 24;
constexpr int kSiluCtas = 19;  // x 256 threads = kInter
constexpr int kHeads = 14, kKvHeads = 2, kHeadDim = 64, kKvDim = kKvHeads * kHeadDim;

// glibc's expf / logf evaluate in double precision and round once, which makes
// them correctly rounded in nearly all cases; doing the same here reproduces
// the reference's values far more often than the single-precision intrinsics.
TMAC_DEV float expf_ref(float x) { return (float)exp((double)x); }
TMAC_DEV float logf_ref(float x) { return (float)log((double)x); }

struct HostTensor {
    int64_t rows = 0, cols = 0;
    int type = 0;
    std::vector<uint8_t> data;
};

struct PrefillState;  // prefill.cu
struct MegaState;     // decode_mega.cu

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
    uint8_t* xp = nullptr;  // the same x_q as byte planes (block-quant GEMVs)
    float* xs = nullptr;
    float* silu_max = nullptr;  // [kSiluCtas] per-CTA max |h| of silu(gate) * up
    // graph-driven generation: position, token and hidden-state logs on the device
    int* pos_dev = nullptr;
    int* tokens = nullptr;        // [max_seq]
    float* hidden_log = nullptr;  // [max_seq][896]
    cudaStream_t stream = nullptr;
    cudaGraphExec_t g_prompt = nullptr, g_gen = nullptr;
    int graph_n_prompt = -1;
    std::vector<void*> allocs;
    tmac::PrefillState* prefill = nullptr;  // batched prefill buffers (prefill.cu)
    tmac::MegaState* mega = nullptr;        // persistent decode kernel (decode_mega.cu)
    int mega_state = 0;                     // 0 not tried, 1 ready, -1 not applicable
    int last_engine = -1;                   // tmac_model_decode_engine
};

namespace tmac {

template <typename T>
inline int dev_alloc(tmac_model_s* m, T** p, size_t n)
{
    TMAC_CUDA_TRY(cudaMalloc((void**)p, n * sizeof(T)));
    m->allocs.push_back(*p);
    return TMAC_OK;
}

inline std::string lname(int l, const char* suffix)
{
    char b[128];
    snprintf(b, sizeof(b), "blk.%d.%s", l, suffix);
    return b;
}

inline const float* vec_or_null(tmac_model_s* m, const std::string& name)
{
    auto it = m->vecs.find(name);
    return it == m->vecs.end() ? nullptr : it->second;
}

void prefill_free(tmac_model_s* m);
// Persistent decode kernel: *out stays nullptr when the model does not qualify.
int mega_prepare(tmac_model_s* m, MegaState** out);
int mega_launch(MegaState* st, int n_prompt, cudaStream_t s);
void mega_free(MegaState* st);

}  // namespace tmac
