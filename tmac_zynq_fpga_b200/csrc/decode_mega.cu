// decode_mega.cu -- one token of the greedy decode (embedding + the 24 layers of
// forward_layer_with_cache, sim/tmac_gguf.cpp:1559-1711) as ONE persistent
// kernel: one CTA per SM, launched cooperatively, every CTA resident for the
// whole token.
//
// Why: the per-kernel engine (decode.cu) runs ~200 small kernels per token, and
// each small GEMV pays a fixed ramp (first weight bytes, activation staging,
// finalise) that dwarfs its 0.1-3 MB of HBM traffic.  Here the weight stream
// does not wait for the activations: each CTA owns a fixed share of every
// projection's 8-row groups and bulk-copies its share of layer l + 1 into
// shared memory while layer l computes, so a projection phase only decodes
// from shared memory.  Phases hand activations over through global memory:
// every value is stored together with the tag of the phase that produced it
// (one 8-byte store, so value and tag are seen together), and a reader polls
// the values it needs until their tags are current -- no separate flag, so a
// hand-over costs one L2 round trip once the data is there.
//
// Phases of layer l (weights of phases A, C, D, E are the four shared-memory
// slots of this CTA):
//   A  attn_norm (every CTA with work recomputes it: in-order sum of squares,
//      as rms_norm :447-454) -> x_q; q|k|v rows of this CTA (Q5_0 groups, or
//      one 32-row Q8_0 attn_v group in the Q8_0 layers)
//   B  CTA head_cta0 + h, h < 14: bias + RoPE + KV append + attention of query
//      head h (attention_prefetch before the wait, then attention_head)
//   C  ctx -> x_q; attn_output rows; hidden[r] += y[r]
//   D  ffn_norm -> x_q; gate rows and the matching up rows; h = silu(g) * u,
//      per-CTA max |h|
//   E  x_q of h from the maximum of those maxima; ffn_down rows; hidden[r] += y[r]
// then, after layer 23, CTA 0 logs the hidden state, writes output_norm(hidden)
// for the logits GEMV, advances the position and clears the top-1 key.
//
// Every value is computed with the same device functions and the same
// operation order as the per-kernel engine, so both engines give identical
// hidden states, bit for bit (tests/test_decode_gpu.py checks it).
//
// Buffer reuse: a phase overwrites a tagged buffer only after every reader of
// its previous contents has finished, which the data dependencies guarantee
// (e.g. q|k|v of layer l + 1 needs hidden after layer l's ffn_down, which needs
// h from every CTA, each of which computed it after its layer-l attention).
//
// Waits: every poll of tagged values and every bulk-copy barrier wait is
// bounded (tmac_set_wait_limit_ns); on expiry the kernel records
// TMAC_ERR_TIMEOUT, raises an abort flag that the other CTAs' waits see, waits
// (bounded) for its own copies in flight and returns.
#include "blockq_dev.cuh"
#include "decode_ops.cuh"
#include "q8_dev.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

namespace tmac {
namespace {

constexpr int kMegaThreads = 768;
constexpr int kMegaWarps = kMegaThreads / 32;
constexpr int kSlots = 4;  // weight slots: q|k|v, attn_output, gate|up, ffn_down
constexpr int kMaxSeg = 6;
// Per-row constants of a block-quant matrix as the slots carry them: row_inv
// and RN(1 / row_inv) in double for the epilogue (quotient_f32).
struct RowConst {
    float ri, pad;
    double rinv;
};
enum : uint32_t { SK_NONE = 0, SK_Q5 = 1, SK_Q8 = 2, SK_Q4K = 3, SK_Q6K = 4 };
constexpr size_t kMaxSmemBytes = 227 * 1024;

struct MegaSeg {
    const void* src;
    uint32_t dst, bytes;
};
// What one CTA does with one weight slot in one layer: the bulk copies that fill
// the slot (weights, then row_inv, then exception entries) and the rows they
// hold -- up to two ranges of whole 8-row groups (gate and up), or one 32-row
// Q8_0 group.
struct MegaSlot {
    MegaSeg seg[kMaxSeg];
    uint32_t total, nseg, kind, rows;  // expect-tx bytes, copies, SK_*, local rows
    uint32_t ri_off, exc_off, exc_n, ngate;  // ngate: local rows of range 0; ri_off: RowConst[rows]
    int32_t row0[2];   // first weight row of each range
    int32_t out0[2];   // output index of each range's first row
};
static_assert(sizeof(MegaSlot) % 16 == 0, "slots are bulk-copied");

struct MegaLayer {
    const float *attn_norm, *ffn_norm, *bq, *bk, *bv;
    float *kc, *vc;
};

struct MegaArgs {
    const MegaLayer* layers;
    const MegaSlot* slots;  // [grid][kLayers][kSlots]
    uint32_t slot_off[kSlots];
    uint32_t plan_off, x_off, norm_off, att_off, acc_off, misc_off, max_rows;
    const uint8_t* emb;  // token_embd GGUF Q8_0 blocks
    unsigned long long* key;
    int* token_log;
    int* tokens;
    int* pos_dev;
    int n_prompt;
    float *hidden, *xn, *hidden_log;
    const float *rope_c, *rope_s, *out_norm;
    // Activations handed between CTAs, each value stored with the tag of the
    // phase that wrote it (tag << 32 | float bits, one 8-byte store): a reader
    // polls the values it needs until their tags are the expected ones.
    unsigned long long *hid_t, *qkv_t, *ctx_t, *h_t;
    uint32_t epoch;  // this launch's tag base (128 tags per launch)
    int* abort_flag;  // zeroed per launch
    int* err;
    int max_seq;
    int head_cta0;
    int emb_cta;  // a CTA with layer-0 q|k|v work: it writes the embedding to hidden
};

struct MegaMisc {
    uint64_t bar[kSlots];
    uint64_t plan_bar;
    uint32_t armed[kSlots], waited[kSlots];
    float red[32];
    float xs, scale;
    int abort, token, pos;
    int sx[32];
    AttnShared attn;
};

// --------------------------------------------------------- tagged values --
// Tags of one launch: EMB for the embedding in hidden, then five per layer.
enum : uint32_t { TG_QKV = 0, TG_CTX = 1, TG_HID_C = 2, TG_H = 3, TG_HID_E = 4 };
TMAC_DEV uint32_t tag_of(uint32_t epoch, int l, uint32_t ph) { return epoch * 128u + 1u + (uint32_t)l * 5u + ph; }
TMAC_DEV uint32_t tag_emb(uint32_t epoch) { return epoch * 128u; }

// One value with its tag, as one single-copy-atomic 8-byte store at L2.
TMAC_DEV void st_tagged(unsigned long long* p, float v, uint32_t tag)
{
    const unsigned long long u = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(u) : "memory");
}
TMAC_DEV unsigned long long ld_tagged(const unsigned long long* p)
{
    unsigned long long u;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(u) : "l"(p) : "memory");
    return u;
}

// One more value a thread waits for beside its share of the main array:
// thread tid < n takes src[tid] once its tag equals `tag`.
struct PollExtra {
    const unsigned long long* src = nullptr;
    int n = 0;
    uint32_t tag = 0;
    float* out = nullptr;
};

struct NoHook {
    TMAC_DEV void operator()() const {}
};

// All threads: r[k] = value src[tid + k * kMegaThreads] (k < K, index < n) once
// its tag equals `tag`, and the extras likewise, all in the same polling loop
// (one L2 round trip when everything is already there).  hook() runs once in
// every thread while the first round of loads is in flight.  Bounded: false
// (and ms.abort) on timeout or another CTA's abort.
template <int K, class Hook = NoHook>
TMAC_DEV bool poll_regs(const unsigned long long* src, int n, uint32_t tag, float (&r)[K], MegaMisc& ms,
                        int* abort_g, int* err, PollExtra e0 = PollExtra(), PollExtra e1 = PollExtra(),
                        const Hook& hook = Hook())
{
    const int tid = threadIdx.x;
    uint32_t todo = 0;
#pragma unroll
    for (int k = 0; k < K; k++)
        if (tid + k * kMegaThreads < n) todo |= 1u << k;
    if (tid < e0.n) todo |= 1u << 30;
    if (tid < e1.n) todo |= 1u << 31;
    uint64_t t0 = 0;
    for (uint32_t it = 0;; it++) {
        // loads first, then the hook, then the tag checks: the hook's work
        // overlaps this thread's loads in flight
        unsigned long long u[K], u0 = 0, u1 = 0;
#pragma unroll
        for (int k = 0; k < K; k++) u[k] = (todo & (1u << k)) ? ld_tagged(src + tid + k * kMegaThreads) : 0ull;
        if (todo & (1u << 30)) u0 = ld_tagged(e0.src + tid);
        if (todo & (1u << 31)) u1 = ld_tagged(e1.src + tid);
        if (it == 0) hook();
#pragma unroll
        for (int k = 0; k < K; k++) {
            if ((todo & (1u << k)) && (uint32_t)(u[k] >> 32) == tag) {
                r[k] = __uint_as_float((uint32_t)u[k]);
                todo &= ~(1u << k);
            }
        }
        if ((todo & (1u << 30)) && (uint32_t)(u0 >> 32) == e0.tag) {
            *e0.out = __uint_as_float((uint32_t)u0);
            todo &= ~(1u << 30);
        }
        if ((todo & (1u << 31)) && (uint32_t)(u1 >> 32) == e1.tag) {
            *e1.out = __uint_as_float((uint32_t)u1);
            todo &= ~(1u << 31);
        }
        if (__syncthreads_and(todo == 0)) return true;
        if ((it & 15u) == 15u) {
            if (tid == 0) {
                if (t0 == 0) t0 = global_timer_ns();
                if (*(volatile int*)abort_g) {
                    ms.abort = 1;
                } else if (global_timer_ns() - t0 > wait_limit_ns()) {
                    if (err) atomicExch(err, (int)TMAC_ERR_TIMEOUT);
                    atomicExch(abort_g, 1);
                    ms.abort = 1;
                }
            }
            __syncthreads();
            if (ms.abort) return false;
        }
    }
}

// All threads: dst[i] = value of src[i] for i < n (n <= kMegaThreads * 2),
// waiting for `tag` as poll_regs.
template <class Hook = NoHook>
TMAC_DEV bool poll_smem(const unsigned long long* src, int n, uint32_t tag, float* dst, MegaMisc& ms, int* abort_g,
                        int* err, const Hook& hook = Hook())
{
    float r[2];
    if (!poll_regs<2>(src, n, tag, r, ms, abort_g, err, PollExtra(), PollExtra(), hook)) return false;
    for (int k = 0; k < 2; k++)
        if (threadIdx.x + k * kMegaThreads < n) dst[threadIdx.x + k * kMegaThreads] = r[k];
    __syncthreads();
    return true;
}

// Thread 0: the copies of one slot for one layer.
TMAC_DEV void issue_slot(const MegaSlot& sp, uint8_t* base, MegaMisc& ms, int slot)
{
    if (sp.kind == SK_NONE || sp.total == 0) return;
    mbar_arrive_expect_tx(&ms.bar[slot], sp.total);
    for (uint32_t s = 0; s < sp.nseg; s++) {
        const uint8_t* src = static_cast<const uint8_t*>(sp.seg[s].src);
        for (uint32_t off = 0; off < sp.seg[s].bytes; off += 32768u)
            bulk_g2s(base + sp.seg[s].dst + off, src + off, min(32768u, sp.seg[s].bytes - off), &ms.bar[slot]);
    }
    ms.armed[slot]++;
}

// Warp 0: the same copies, one segment per lane -- a bulk copy takes its
// issuing thread ~0.15 us, so the segments are issued side by side.
TMAC_DEV void issue_slot_warp(const MegaSlot& sp, uint8_t* base, MegaMisc& ms, int slot, int lane)
{
    if (sp.kind == SK_NONE || sp.total == 0) return;
    if (lane == 0) mbar_arrive_expect_tx(&ms.bar[slot], sp.total);
    __syncwarp();
    for (uint32_t sg = lane; sg < sp.nseg; sg += 32) {
        const uint8_t* src = static_cast<const uint8_t*>(sp.seg[sg].src);
        for (uint32_t off = 0; off < sp.seg[sg].bytes; off += 32768u)
            bulk_g2s(base + sp.seg[sg].dst + off, src + off, min(32768u, sp.seg[sg].bytes - off), &ms.bar[slot]);
    }
    __syncwarp();
    if (lane == 0) ms.armed[slot]++;
    __syncwarp();
}

// ---------------------------------------------------------------- compute --
// Block-quant rows of a slot: the main loop, exceptions and finalise of
// blockq_gemv_kernel (gemv_blockq.cu) at batch 1 over the slot's groups.
// yv[rr] = (float)((double)acc * x_scale / (double)row_inv).
template <int TYPE>
TMAC_DEV void mega_blockq(const uint8_t* wsm, const MegaSlot& sp, int cols, const uint8_t* xpl, float xs,
                          uint32_t* acc_lo, uint32_t* acc_hi, float* yv, unsigned long long* stamps = nullptr)
{
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t cpr = cols / 32, nblk = cols / Geo<TYPE>::kBlockVals;
    const int64_t group_bytes = Geo<TYPE>::group_bytes(nblk);
    const int rows_cta = (int)sp.rows, ng = rows_cta / 8;
    const RowConst* rc_s = reinterpret_cast<const RowConst*>(wsm + sp.ri_off);
    const int4* exc_s = reinterpret_cast<const int4*>(wsm + sp.exc_off);
    for (int t = tid; t < rows_cta; t += kMegaThreads) acc_lo[t] = acc_hi[t] = 0;
    __syncthreads();
    const bool q5 = (TYPE == TMAC_TYPE_Q5_0);
    const int slots = q5 ? ng : rows_cta;
    const int steps = (int)(q5 ? (cpr + 3) / 4 : (nblk + 3) / 4);
    const int items = slots * steps;
    const int it0 = (int)((int64_t)items * warp / kMegaWarps), it1 = (int)((int64_t)items * (warp + 1) / kMegaWarps);
    const int r_lane = q5 ? (lane & 7) : 0;
    const int l_lane = q5 ? (lane >> 3) : lane;
    const uint32_t wsm_a = smem_addr(wsm);
    long long acc = 0;
    int slot = items ? it0 / steps : 0, s = items ? it0 % steps : 0;
    if (stamps && lane == 0 && warp == 0) stamps[4] = global_timer_ns();
    for (int it = it0; it < it1; it++) {
        if (stamps && lane == 0 && warp == 0 && it - it0 < 6) stamps[5 + 2 * (it - it0)] = global_timer_ns();
        const int rr = q5 ? slot * 8 + r_lane : slot;
        const SharedBytes G{wsm_a + (uint32_t)(rr >> 3) * (uint32_t)group_bytes};
        const int r = rr & 7;
        const float ri = rc_s[rr].ri;
        const uint32_t ch = q5 ? (uint32_t)(4 * s + l_lane) : (uint32_t)(4 * s + (lane >> 3)) * 8 + (lane & 7);
        if (ch < cpr) {
            Chunk c;
            uint32_t vw[16];
            load_chunk<TYPE>(G, r, (uint32_t)nblk, ch, c);
            fast_values<TYPE>(c, ri, vw);
            acc += chunk_dot(vw, xpl + ch * 32, xpl + cols + ch * 32);
        }
        if (stamps && lane == 0 && warp == 0 && it - it0 < 6) stamps[6 + 2 * (it - it0)] = (unsigned long long)(acc & 1) + global_timer_ns();
        if (++s == steps || it + 1 == it1) {
            long long v = acc;
            for (int o = q5 ? 8 : 1; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (l_lane == 0) acc_add(&acc_lo[rr], &acc_hi[rr], v);
            acc = 0;
            if (s == steps) {
                s = 0;
                slot++;
            }
        }
    }
    if (stamps && threadIdx.x == 0) stamps[0] = global_timer_ns();
    // exceptions: (v - v') * x_q[col] for the entries of this slot's rows
    const int n1 = (int)sp.ngate;
    for (int t = tid; t < (int)sp.exc_n; t += kMegaThreads) {
        const int4 ex = exc_s[t];
        const int rr = (ex.x >= sp.row0[0] && ex.x < sp.row0[0] + n1) ? ex.x - sp.row0[0] : ex.x - sp.row0[1] + n1;
        acc_add(&acc_lo[rr], &acc_hi[rr], (long long)ex.z * xq_at(xpl, cols, 0, ex.y));
    }
    __syncthreads();
    if (stamps && threadIdx.x == 0) stamps[1] = global_timer_ns();
    for (int t = tid; t < rows_cta; t += kMegaThreads) {
        const long long tot = (long long)(((unsigned long long)acc_hi[t] << 32) | acc_lo[t]);
        yv[t] = quotient_f32(__dmul_rn((double)tot, (double)xs), rc_s[t].rinv, rc_s[t].ri);
    }
    __syncthreads();
    if (stamps && threadIdx.x == 0) stamps[2] = global_timer_ns();
}

// One 32-row Q8_0 record (gemv_q8_0.cu layout): tile t on warp t (lane = row),
// then the fold over tiles in order, y = (float)(y + acc * x_scale * row_scale)
// (tmac_gguf.cpp:1075-1076).  sx: the x_q sums of every 32-column block.
TMAC_DEV void mega_q8(const uint8_t* rec, int cols, const uint8_t* xpl, const int* sx, float xs, long long* tsum,
                      float* yv)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Q8Layout L;
    L.T = cols / 64;
    L.stages = 0;
    L.groups = 1;
    L.group_bytes = (int64_t)L.T * 2176 + 128;
    for (int t = warp; t < L.T; t += kMegaWarps) {
        uint4 xh[4], xl[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            xh[j] = reinterpret_cast<const uint4*>(xpl + t * 64)[j];
            xl[j] = reinterpret_cast<const uint4*>(xpl + cols + t * 64)[j];
        }
        tsum[t * 32 + lane] = q8_tile_dot(rec, L, t, lane, xh, xl, make_int2(sx[2 * t], sx[2 * t + 1]));
    }
    __syncthreads();
    if (warp == 0) {
        const double rs = (double)reinterpret_cast<const float*>(rec + L.rs_off())[lane];
        float yr = 0.0f;
        for (int t = 0; t < L.T; t++) {
            const double v = __dmul_rn(__dmul_rn((double)tsum[t * 32 + lane], (double)xs), rs);
            yr = (float)__dadd_rn((double)yr, v);
        }
        yv[lane] = yr;
    }
    __syncthreads();
}

// In-order sum of the kHidden squares, speculated by segment.  The sum
// s_{i+1} = fl(s_i + p_i) is split into kSumSegs segments.  The running sum at
// the start of segment k is estimated as fl(exact prefix sum) (double sums of
// the segments), and 64 threads run segment k from the 64 floats nearest that
// estimate (one each).  One thread runs segment 0 from 0 and then links: the
// true start of segment k is the end of segment k - 1; the candidate that
// started from exactly that float holds the true end of segment k.  A start
// outside the candidates' range is summed again in order (never wrong, only
// slower), so the result is the sequential sum bit for bit.
constexpr int kSumSegs = 8;
constexpr int kSegLen = kHidden / kSumSegs;
constexpr int kSumWarps = 2 * (kSumSegs - 1) + 1;  // two candidate warps per later segment + the linking warp
constexpr int kSumBar = 3;                          // named barrier of the kSumWarps warps
constexpr int kNormBar = 2;                         // linking warp + the warps forming x * w
constexpr int kNormBarThreads = 32 + (kMegaWarps - kSumWarps) * 32;
static_assert(kHidden % (kSumSegs * 16) == 0, "segments of whole 16-value batches");
static_assert(kSumWarps < kMegaWarps, "warps left for x * w");

// Float estimate of the running sum at the start of segment k (same arithmetic
// in every thread that asks).
TMAC_DEV float seg_start_estimate(const double* seg_sum, int k)
{
    double e = 0.0;
    for (int i = 0; i < k; i++) e += seg_sum[i];
    return (float)e;
}

// rms_norm of xv[0..kHidden) with weights w (the order of rmsnorm_kernel,
// decode.cu), then x_q of the result as byte planes xpl[0..n) (high) /
// xpl[n..2n) (low) and x_scale in ms.xs.  All threads; scratch: 2 KB of shared
// memory.  While warps 0..kSumWarps-1 run the sum of squares, the other warps
// form xw = fl(x * w) and max |xw|: the normed value is fl(xw * scale), and
// because rounding is monotonic, max |fl(xw * scale)| = fl(max |xw| * scale).
TMAC_DEV void mega_norm_quantize(float* xv, float* sq, const float* __restrict__ w, int n, uint8_t* xpl,
                                 MegaMisc& ms, float* scratch, unsigned long long* stamps = nullptr)
{
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < n; i += kMegaThreads) sq[i] = __fmul_rn(xv[i], xv[i]);
    __syncthreads();
    float* seg_end = scratch;                                                  // [kSumSegs - 1][64]
    double* seg_sum = reinterpret_cast<double*>(scratch + (kSumSegs - 1) * 64);  // [kSumSegs]
    int* est_bits = reinterpret_cast<int*>(seg_sum + kSumSegs);                   // [kSumSegs] estimates' bits
    if (warp < kSumWarps) {
        if (warp < kSumSegs) {
            double v = 0.0;
            for (int i = lane; i < kSegLen; i += 32) v += (double)sq[warp * kSegLen + i];
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) seg_sum[warp] = v;
        }
        named_bar_sync(kSumBar, kSumWarps * 32);
        if (warp < kSumWarps - 1) {
            const int k = 1 + (warp >> 1);
            const int j = (warp & 1) * 32 + lane - 32;  // candidate: estimate + j ulps
            const int est = __float_as_int(seg_start_estimate(seg_sum, k));
            if ((warp & 1) == 0 && lane == 0) est_bits[k] = est;
            const int bits = est + j;
            seg_end[(k - 1) * 64 + j + 32] =
                bits >= 0 ? seq_sum_from(__int_as_float(bits), sq + k * kSegLen, kSegLen) : __int_as_float(0x7FC00000);
            named_bar_arrive(kSumBar, kSumWarps * 32);
        } else {
            float s = 0.0f;
            if (lane == 0) {
                if (stamps) stamps[0] = global_timer_ns();
                s = seq_sum_from(0.0f, sq, kSegLen);
                if (stamps) stamps[2] = global_timer_ns();
            }
            named_bar_sync(kSumBar, kSumWarps * 32);
            if (lane == 0) {
                if (stamps) stamps[3] = global_timer_ns();
                for (int k = 1; k < kSumSegs; k++) {
                    const int j = __float_as_int(s) - est_bits[k];
                    s = (j >= -32 && j < 32) ? seg_end[(k - 1) * 64 + j + 32] : seq_sum_from(s, sq + k * kSegLen, kSegLen);
                }
                ms.scale = rms_scale_from_sum(s, n);
                if (stamps) stamps[1] = global_timer_ns();
            }
            named_bar_sync(kNormBar, kNormBarThreads);
            if (lane == 0) {
                float mx = 0.0f;
                for (int i = kSumWarps; i < kMegaWarps; i++) mx = fmaxf(mx, ms.red[i]);
                ms.xs = x_scale_from_max(__fmul_rn(mx, ms.scale));
            }
        }
    } else {
        float mx = 0.0f;
        for (int i = tid - kSumWarps * 32; i < n; i += kMegaThreads - kSumWarps * 32) {
            const float v = __fmul_rn(xv[i], __ldg(w + i));
            xv[i] = v;
            mx = fmaxf(mx, fabsf(v));
        }
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) ms.red[warp] = mx;
        named_bar_arrive(kNormBar, kNormBarThreads);
    }
    __syncthreads();
    const float scale = ms.scale, s = ms.xs;
    for (int i = tid; i < n; i += kMegaThreads) {
        const float v = __fmul_rn(xv[i], scale);
        xv[i] = v;
        const int16_t q = quantize_one(v, s);
        xpl[i] = (uint8_t)((uint16_t)q >> 8);
        xpl[n + i] = (uint8_t)(q & 0xFF);
    }
    __syncthreads();
}

// x_q of the values r[k] (index tid + k * kMegaThreads < n) with x_scale from
// max_abs (tmac_gguf.cpp:889-896); planes xpl[0..n) high, [n..2n) low.
constexpr int kMaxQuant = 7;
template <int K>
TMAC_DEV void mega_quantize(const float (&r)[K], int n, float max_abs, uint8_t* xpl, MegaMisc& ms)
{
    const int tid = threadIdx.x;
    const float s = x_scale_from_max(max_abs);
    if (tid == 0) ms.xs = s;
#pragma unroll
    for (int k = 0; k < K; k++) {
        const int i = tid + k * kMegaThreads;
        if (i < n) {
            const int16_t q = quantize_one(r[k], s);
            xpl[i] = (uint8_t)((uint16_t)q >> 8);
            xpl[n + i] = (uint8_t)(q & 0xFF);
        }
    }
    __syncthreads();
}
static_assert(kInter <= kMaxQuant * kMegaThreads, "h fits the registers of mega_quantize");

// x_q sums of every 32-column block (the Q8_0 dot products' correction term).
TMAC_DEV void mega_block_sums(const uint8_t* xpl, int n, int* sx)
{
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < n / 32; j += kMegaWarps) {
        int v = (int)(int8_t)xpl[j * 32 + lane] * 256 + (int)xpl[n + j * 32 + lane];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) sx[j] = v;
    }
    __syncthreads();
}

#ifdef TMAC_TRACE
// Diagnostic build only (-DTMAC_TRACE): %globaltimer stamps of each CTA's phase
// boundaries and of each head's attention steps, read back with
// tmac_trace_read_mega / tmac_trace_read_att.
__device__ unsigned long long g_mega_trace[160][kLayers][24];
__device__ unsigned long long g_att_trace[kHeads][kLayers][8];
__device__ unsigned long long g_bq_trace[160][kLayers][4][20];
__device__ unsigned long long g_norm_trace[160][kLayers][2][8];
#define MEGA_STAMP(l, i)                                                                 \
    do {                                                                                 \
        if (threadIdx.x == 0 && blockIdx.x < 160) g_mega_trace[blockIdx.x][l][i] = global_timer_ns(); \
    } while (0)
#define MEGA_ATT_STAMPS(h, l) (&g_att_trace[h][l][0])
#define MEGA_NORM_STAMPS(l, i) (blockIdx.x < 160 ? &g_norm_trace[blockIdx.x][l][i][0] : nullptr)
#define MEGA_BQ_STAMPS(l, ph) (blockIdx.x < 160 ? &g_bq_trace[blockIdx.x][l][ph][0] : nullptr)
#define MEGA_ISSUE_T0() const unsigned long long it0_ = global_timer_ns()
#define MEGA_ISSUE_T1(l, s) do { if (blockIdx.x < 160) { g_bq_trace[blockIdx.x][l][s][18] = global_timer_ns() - it0_; g_bq_trace[blockIdx.x][l][s][19] = plans[(l + 1) * kSlots + s].nseg; } } while (0)
#define MEGA_BQ_MARK(l, ph, i) do { if (threadIdx.x == 0 && blockIdx.x < 160) g_bq_trace[blockIdx.x][l][ph][i] = global_timer_ns(); } while (0)
#else
#define MEGA_STAMP(l, i) \
    do {                 \
    } while (0)
#define MEGA_ATT_STAMPS(h, l) nullptr
#define MEGA_NORM_STAMPS(l, i) nullptr
#define MEGA_BQ_STAMPS(l, ph) nullptr
#define MEGA_BQ_MARK(l, ph, i) do { } while (0)
#define MEGA_ISSUE_T0() do { } while (0)
#define MEGA_ISSUE_T1(l, s) do { } while (0)
#endif

__global__ void __launch_bounds__(kMegaThreads, 1) decode_mega_kernel(MegaArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, cta = blockIdx.x;
    MegaSlot* plans = reinterpret_cast<MegaSlot*>(smem + a.plan_off);  // [kLayers][kSlots]
    uint8_t* xpl = smem + a.x_off;
    float* xv = reinterpret_cast<float*>(smem + a.norm_off);
    float* sq = xv + kHidden;
    float* att = reinterpret_cast<float*>(smem + a.att_off);
    uint32_t* acc_lo = reinterpret_cast<uint32_t*>(smem + a.acc_off);
    uint32_t* acc_hi = acc_lo + a.max_rows;
    float* yv = reinterpret_cast<float*>(acc_hi + a.max_rows);
    long long* tsum = reinterpret_cast<long long*>(smem + a.acc_off + (((size_t)a.max_rows * 12 + 15) & ~(size_t)15));
    MegaMisc& ms = *reinterpret_cast<MegaMisc*>(smem + a.misc_off);
    uint8_t* slot_base[kSlots];
    for (int s = 0; s < kSlots; s++) slot_base[s] = smem + a.slot_off[s];

    // ---- set-up: this CTA's copy plans, then layer 0's weights for every slot
    if (tid == 0) {
        for (int s = 0; s < kSlots; s++) {
            mbar_init(&ms.bar[s], 1);
            ms.armed[s] = ms.waited[s] = 0;
        }
        mbar_init(&ms.plan_bar, 1);
        ms.abort = 0;
        fence_mbar_init();
        const uint32_t pb = (uint32_t)(kLayers * kSlots * sizeof(MegaSlot));
        mbar_arrive_expect_tx(&ms.plan_bar, pb);
        const uint8_t* src = reinterpret_cast<const uint8_t*>(a.slots + (size_t)cta * kLayers * kSlots);
        for (uint32_t off = 0; off < pb; off += 32768u)
            bulk_g2s(reinterpret_cast<uint8_t*>(plans) + off, src + off, min(32768u, pb - off), &ms.plan_bar);
        if (!mbar_wait_bounded(&ms.plan_bar, 0, a.err)) {
            ms.abort = 1;
            atomicExch(a.abort_flag, 1);
        } else {
            for (int s = 0; s < kSlots; s++) issue_slot(plans[s], slot_base[s], ms, s);
        }
        // token of this position: the prompt, else the greedy key of the last logits
        const int p = *a.pos_dev;
        int tok = p < a.n_prompt ? a.tokens[p] : -1;
        if (tok < 0 && a.key) {
            const unsigned long long k = *a.key;
            tok = (int)(0x7FFFFFFFu - (uint32_t)(k & 0x7FFFFFFFu));
        }
        if (tok < 0 || tok >= kVocab) tok = 0;
        ms.pos = p;
        ms.token = tok;
        if (cta == 0) {
            *a.token_log = tok;
            a.tokens[p] = tok;
        }
    }
    __syncthreads();
    const int pos = ms.pos;
    const uint32_t ep = a.epoch;

    // A wait that failed anywhere ends the token: drain this CTA's copies, return.
    auto drain = [&]() {
        cp_async_wait_all();  // attention prefetches of this thread
        if (tid == 0)
            for (int s = 0; s < kSlots; s++)
                for (; ms.waited[s] < ms.armed[s]; ms.waited[s]++) mbar_wait_bounded(&ms.bar[s], ms.waited[s] & 1, nullptr);
    };
    // Fill `slot` with layer l + 1's weights once its layer-l use is over --
    // whether or not this CTA had layer-l work in it (the splits differ between
    // layers, e.g. q|k|v of the Q5_0 and the Q8_0 layers).  Issuing the bulk
    // copies takes thread 0 a while, so refill() only notes the slot, and
    // flush() issues the noted copies while the next poll's first loads are in
    // flight (every phase polls before it waits for a slot; wait_slot flushes
    // too).
    uint32_t pend_mask = 0;
    int pend_l[kSlots];
    auto refill = [&](int l, int slot) {
        if (tid < 32) {
            pend_mask |= 1u << slot;
            pend_l[slot] = l;
        }
    };
    auto flush = [&]() {
        if (tid < 32 && pend_mask) {
            for (int s = 0; s < kSlots; s++)
                if ((pend_mask >> s) & 1u) {
                    const int l = pend_l[s];
                    if (l + 1 < kLayers && ms.armed[s] == ms.waited[s]) {
                        MEGA_ISSUE_T0();
                        issue_slot_warp(plans[(l + 1) * kSlots + s], slot_base[s], ms, s, tid);
                        if (tid == 0) MEGA_ISSUE_T1(l, s);
                    }
                }
            pend_mask = 0;
        }
    };
    const auto hook = [&]() { flush(); };
    // All threads: wait for this layer's copies of `slot`.
    auto wait_slot = [&](int slot) -> bool {
        flush();
        const uint32_t par = ms.waited[slot] & 1;
        const bool ok = mbar_wait_sleep(&ms.bar[slot], par, a.err);
        if (!ok) ms.abort = 1;
        __syncthreads();
        if (tid == 0 && !ms.abort) ms.waited[slot]++;
        const bool go = !ms.abort;
        __syncthreads();
        if (!go && tid == 0) atomicExch(a.abort_flag, 1);
        return go;
    };
    // End of a phase: every value is stored; refill the phase's slot.
    auto finish = [&](int l, int slot) {
        __syncthreads();
        if (slot >= 0) refill(l, slot);
    };

    if (ms.abort) {
        drain();
        return;
    }

    for (int l = 0; l < kLayers; l++) {
        const MegaLayer& L = a.layers[l];
        MEGA_STAMP(l, 0);
        // ------------------------------------------------ A: q|k|v rows
        const MegaSlot& pa = plans[l * kSlots + 0];
        if (pa.kind != SK_NONE) {
            if (l == 0) {  // embedding row of the token (read_embedding / dequant_q8_0, :225-234)
                const int tok = ms.token;
                for (int i = tid; i < kHidden; i += kMegaThreads) {
                    const int64_t idx = (int64_t)tok * kHidden + i;
                    const uint8_t* b = a.emb + (idx / 32) * 34;
                    const float v = __fmul_rn((float)(int8_t)b[2 + idx % 32], f16_bits_to_f32(ld_u16_unaligned(b)));
                    xv[i] = v;
                    if (cta == a.emb_cta) st_tagged(a.hid_t + i, v, tag_emb(ep));
                }
                __syncthreads();
            } else {
                if (!poll_smem(a.hid_t, kHidden, tag_of(ep, l - 1, TG_HID_E), xv, ms, a.abort_flag, a.err, hook)) break;
                MEGA_STAMP(l, 1);
            }
            mega_norm_quantize(xv, sq, L.attn_norm, kHidden, xpl, ms, att, MEGA_NORM_STAMPS(l, 0));
            if (pa.kind == SK_Q8) mega_block_sums(xpl, kHidden, ms.sx);
            MEGA_STAMP(l, 2);
            if (!wait_slot(0)) break;
            MEGA_STAMP(l, 3);
            if (pa.kind == SK_Q8) mega_q8(slot_base[0], kHidden, xpl, ms.sx, ms.xs, tsum, yv);
            else mega_blockq<TMAC_TYPE_Q5_0>(slot_base[0], pa, kHidden, xpl, ms.xs, acc_lo, acc_hi, yv, MEGA_BQ_STAMPS(l, 0));
            for (int t = tid; t < (int)pa.rows; t += kMegaThreads)
                st_tagged(a.qkv_t + pa.out0[0] + t, yv[t], tag_of(ep, l, TG_QKV));
            MEGA_BQ_MARK(l, 0, 3);
            __syncthreads();
            MEGA_BQ_MARK(l, 0, 17);
            finish(l, 0);
            MEGA_STAMP(l, 4);
        } else {
            refill(l, 0);
        }
        // ------------------------------------------------ B: attention of one head
        const int h = cta - a.head_cta0;
        if (h >= 0 && h < kHeads) {
            // earlier positions' K / V rows do not depend on this step: their
            // copies overlap the wait for q|k|v
            if (tid < kAttnThreads)
                attention_prefetch(h, L.kc, L.vc, pos, a.max_seq, att, L.bq, L.bk, L.bv, a.rope_c, a.rope_s, ms.attn);
            // the head's q, its KV head's k and v (192 values) into sq
            const int kvh = h / (kHeads / kKvHeads);
            float r[1];
            const int src = tid < kHeadDim ? h * kHeadDim + tid
                                           : (tid < 2 * kHeadDim ? kHidden + kvh * kHeadDim + tid - kHeadDim
                                                                 : kHidden + kKvDim + kvh * kHeadDim + tid - 2 * kHeadDim);
            r[0] = 0.0f;
            {
                const int n = tid < 3 * kHeadDim ? 1 : 0;  // threads 0..191 each wait for one value
                uint32_t todo = n;
                uint64_t t0 = 0;
                bool ok = true;
                for (uint32_t it = 0;; it++) {
                    const unsigned long long u = todo ? ld_tagged(a.qkv_t + src) : 0ull;
                    if (it == 0) flush();  // while the load is in flight
                    if (todo && (uint32_t)(u >> 32) == tag_of(ep, l, TG_QKV)) {
                        r[0] = __uint_as_float((uint32_t)u);
                        todo = 0;
                    }
                    if (__syncthreads_and(todo == 0)) break;
                    if ((it & 15u) == 15u) {
                        if (tid == 0) {
                            if (t0 == 0) t0 = global_timer_ns();
                            if (*(volatile int*)a.abort_flag) {
                                ms.abort = 1;
                            } else if (global_timer_ns() - t0 > wait_limit_ns()) {
                                atomicExch(a.err, (int)TMAC_ERR_TIMEOUT);
                                atomicExch(a.abort_flag, 1);
                                ms.abort = 1;
                            }
                        }
                        __syncthreads();
                        if (ms.abort) {
                            ok = false;
                            break;
                        }
                    }
                }
                if (!ok) break;
            }
            if (tid < 3 * kHeadDim) sq[tid] = r[0];
            __syncthreads();
            MEGA_STAMP(l, 5);
            if (tid < kAttnThreads)
                attention_head(h, sq, sq + kHeadDim, sq + 2 * kHeadDim, pos, L.kc, L.vc, sq + 3 * kHeadDim, a.max_seq,
                               att, ms.attn, 1, MEGA_ATT_STAMPS(h, l));
            __syncthreads();
            if (tid < kHeadDim) st_tagged(a.ctx_t + h * kHeadDim + tid, sq[3 * kHeadDim + tid], tag_of(ep, l, TG_CTX));
            MEGA_STAMP(l, 23);
            finish(l, -1);
            MEGA_STAMP(l, 6);
        }
        // ------------------------------------------------ C: attn_output + residual
        const MegaSlot& pc = plans[l * kSlots + 1];
        if (pc.kind != SK_NONE) {
            // ctx, and this CTA's rows of hidden for the residual, in one polling loop
            float r[2], hres = 0.0f;
            PollExtra ex;
            ex.src = a.hid_t + pc.out0[0];
            ex.n = (int)pc.rows;
            ex.tag = l == 0 ? tag_emb(ep) : tag_of(ep, l - 1, TG_HID_E);
            ex.out = &hres;
            if (!poll_regs<2>(a.ctx_t, kHidden, tag_of(ep, l, TG_CTX), r, ms, a.abort_flag, a.err, ex, PollExtra(), hook))
                break;
            MEGA_STAMP(l, 7);
            float mx = fmaxf(fabsf(r[0]), tid + kMegaThreads < kHidden ? fabsf(r[1]) : 0.0f);
            mx = block_max(mx, ms.red, kMegaThreads);
            mega_quantize<2>(r, kHidden, mx, xpl, ms);
            MEGA_STAMP(l, 8);
            if (!wait_slot(1)) break;
            MEGA_STAMP(l, 21);
            mega_blockq<TMAC_TYPE_Q5_0>(slot_base[1], pc, kHidden, xpl, ms.xs, acc_lo, acc_hi, yv, MEGA_BQ_STAMPS(l, 1));
            MEGA_STAMP(l, 22);
            if (tid < (int)pc.rows)
                st_tagged(a.hid_t + pc.out0[0] + tid, __fadd_rn(hres, yv[tid]), tag_of(ep, l, TG_HID_C));
            MEGA_BQ_MARK(l, 1, 3);
            __syncthreads();
            MEGA_BQ_MARK(l, 1, 17);
            finish(l, 1);
            MEGA_STAMP(l, 9);
        } else {
            refill(l, 1);
        }
        // ------------------------------------------------ D: gate|up + silu
        const MegaSlot& pd = plans[l * kSlots + 2];
        if (pd.kind != SK_NONE) {
            if (!poll_smem(a.hid_t, kHidden, tag_of(ep, l, TG_HID_C), xv, ms, a.abort_flag, a.err, hook)) break;
            MEGA_STAMP(l, 10);
            mega_norm_quantize(xv, sq, L.ffn_norm, kHidden, xpl, ms, att, MEGA_NORM_STAMPS(l, 1));
            MEGA_STAMP(l, 11);
            if (!wait_slot(2)) break;
            mega_blockq<TMAC_TYPE_Q5_0>(slot_base[2], pd, kHidden, xpl, ms.xs, acc_lo, acc_hi, yv, MEGA_BQ_STAMPS(l, 2));
            MEGA_STAMP(l, 12);
            const int n = (int)pd.ngate;
            for (int t = tid; t < n; t += kMegaThreads)
                st_tagged(a.h_t + pd.out0[0] + t, silu_mul(yv[t], yv[n + t]), tag_of(ep, l, TG_H));
            MEGA_BQ_MARK(l, 2, 3);
            __syncthreads();
            MEGA_BQ_MARK(l, 2, 17);
            finish(l, 2);
            MEGA_STAMP(l, 13);
        } else {
            refill(l, 2);
        }
        // ------------------------------------------------ E: ffn_down + residual
        const MegaSlot& pe = plans[l * kSlots + 3];
        if (pe.kind != SK_NONE) {
            // h and this CTA's rows of hidden, in one polling loop
            float r[kMaxQuant], hres = 0.0f;
            PollExtra ex1;
            ex1.src = a.hid_t + pe.out0[0];
            ex1.n = (int)pe.rows;
            ex1.tag = tag_of(ep, l, TG_HID_C);
            ex1.out = &hres;
            if (!poll_regs<kMaxQuant>(a.h_t, kInter, tag_of(ep, l, TG_H), r, ms, a.abort_flag, a.err, PollExtra(), ex1, hook))
                break;
            MEGA_STAMP(l, 14);
            // x_scale from max |h| over the values just polled
            float mx = 0.0f;
#pragma unroll
            for (int k = 0; k < kMaxQuant; k++)
                if (tid + k * kMegaThreads < kInter) mx = fmaxf(mx, fabsf(r[k]));
            mx = block_max(mx, ms.red, kMegaThreads);
            mega_quantize<kMaxQuant>(r, kInter, mx, xpl, ms);
            MEGA_STAMP(l, 15);
            if (!wait_slot(3)) break;
            MEGA_STAMP(l, 19);
            if (pe.kind == SK_Q6K)
                mega_blockq<TMAC_TYPE_Q6_K>(slot_base[3], pe, kInter, xpl, ms.xs, acc_lo, acc_hi, yv, MEGA_BQ_STAMPS(l, 3));
            else
                mega_blockq<TMAC_TYPE_Q4_K>(slot_base[3], pe, kInter, xpl, ms.xs, acc_lo, acc_hi, yv, MEGA_BQ_STAMPS(l, 3));
            MEGA_STAMP(l, 20);
            if (tid < (int)pe.rows)
                st_tagged(a.hid_t + pe.out0[0] + tid, __fadd_rn(hres, yv[tid]), tag_of(ep, l, TG_HID_E));
            MEGA_BQ_MARK(l, 3, 3);
            __syncthreads();
            MEGA_BQ_MARK(l, 3, 17);
            finish(l, 3);
            MEGA_STAMP(l, 16);
        } else {
            refill(l, 3);
        }
    }
    if (ms.abort) {
        drain();
        return;
    }
    // ---- end of the token (CTA 0): hidden state and its log, output_norm for
    // the logits GEMV, next position, key cleared for the next step's top-1
    if (cta == 0) {
        if (!poll_smem(a.hid_t, kHidden, tag_of(ep, kLayers - 1, TG_HID_E), xv, ms, a.abort_flag, a.err)) {
            drain();
            return;
        }
        for (int i = tid; i < kHidden; i += kMegaThreads) {
            a.hidden[i] = xv[i];
            a.hidden_log[(int64_t)pos * kHidden + i] = xv[i];
        }
        if (a.out_norm) {
            for (int i = tid; i < kHidden; i += kMegaThreads) sq[i] = __fmul_rn(xv[i], xv[i]);
            __syncthreads();
            if (tid == 0) ms.scale = rms_scale(sq, kHidden);
            __syncthreads();
        } else if (tid == 0) {
            ms.scale = 1.0f;
        }
        __syncthreads();
        for (int i = tid; i < kHidden; i += kMegaThreads)
            a.xn[i] = a.out_norm ? __fmul_rn(__fmul_rn(xv[i], __ldg(a.out_norm + i)), ms.scale) : xv[i];
        if (tid == 0) {
            *a.pos_dev = pos + 1;
            *a.key = 0;
        }
    }
    drain();
}

// Contiguous share [lo, hi) of n items for part i of parts.
inline void split(int64_t n, int parts, int i, int64_t* lo, int64_t* hi)
{
    *lo = n * i / parts;
    *hi = n * (i + 1) / parts;
}

}  // namespace

// ------------------------------------------------------------------ host --
struct MegaState {
    MegaArgs args{};
    size_t smem = 0;
    int grid = 0;
    void* dev_layers = nullptr;
    void* dev_slots = nullptr;
    int* dev_abort = nullptr;                // cleared before every launch
    unsigned long long* dev_tagged = nullptr;  // hidden | q|k|v | ctx | h
    uint32_t epoch = 0;                        // tag base of the last launch
    std::vector<void*> rowc;                   // RowConst arrays of the block-quant matrices
};

namespace {

// Adds a copy of `bytes` from src to offset *off of the slot (skipped when empty).
void add_seg(MegaSlot& sp, const void* src, uint32_t bytes, uint32_t* off)
{
    if (!bytes) return;
    sp.seg[sp.nseg].src = src;
    sp.seg[sp.nseg].dst = *off;
    sp.seg[sp.nseg].bytes = bytes;
    sp.nseg++;
    *off += bytes;
    sp.total += bytes;
}

// A block-quant slot over up to two ranges of 8-row groups [g0, g1) of w.
int blockq_slot(const tmac_weight_s* w, const RowConst* rowc, const std::vector<int>& exc_ptr,
                const int64_t (&g0)[2], const int64_t (&g1)[2], const int32_t (&out0)[2], int nrange, MegaSlot& sp)
{
    sp = MegaSlot{};
    int64_t rows = 0;
    for (int r = 0; r < nrange; r++) rows += 8 * (g1[r] - g0[r]);
    if (rows == 0) return TMAC_OK;
    sp.kind = w->type == TMAC_TYPE_Q5_0 ? SK_Q5 : (w->type == TMAC_TYPE_Q6_K ? SK_Q6K : SK_Q4K);
    sp.rows = (uint32_t)rows;
    uint32_t off = 0;
    for (int r = 0; r < nrange; r++)
        add_seg(sp, w->data + g0[r] * w->group_bytes, (uint32_t)((g1[r] - g0[r]) * w->group_bytes), &off);
    sp.ri_off = off;
    for (int r = 0; r < nrange; r++)
        add_seg(sp, rowc + 8 * g0[r], (uint32_t)(8 * sizeof(RowConst) * (g1[r] - g0[r])), &off);
    sp.exc_off = off;
    for (int r = 0; r < nrange; r++) {
        const int64_t e0 = exc_ptr[std::min<int64_t>(8 * g0[r], w->rows)];
        const int64_t e1 = exc_ptr[std::min<int64_t>(8 * g1[r], w->rows)];
        add_seg(sp, static_cast<const int4*>(w->exc) + e0, (uint32_t)(16 * (e1 - e0)), &off);
        sp.exc_n += (uint32_t)(e1 - e0);
    }
    for (int r = 0; r < 2; r++) {
        sp.row0[r] = r < nrange ? (int32_t)(8 * g0[r]) : 0;
        sp.out0[r] = r < nrange ? out0[r] : 0;
    }
    sp.ngate = (uint32_t)(8 * (g1[0] - g0[0]));
    return TMAC_OK;
}

__global__ void rowconst_kernel(const float* __restrict__ ri, const double* __restrict__ rinv, int64_t n,
                                RowConst* __restrict__ out)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = RowConst{ri[i], 0.0f, rinv[i]};
}

// The RowConst array of w (rows padded to whole groups), made once per weight.
int row_consts(const tmac_weight_s* w, std::map<const tmac_weight_s*, RowConst*>& made, const RowConst** out)
{
    auto it = made.find(w);
    if (it != made.end()) {
        *out = it->second;
        return TMAC_OK;
    }
    const int64_t n = w->groups * 8;
    RowConst* p = nullptr;
    TMAC_CUDA_TRY(cudaMalloc(&p, (size_t)n * sizeof(RowConst)));
    made[w] = p;
    rowconst_kernel<<<(unsigned)((n + 255) / 256), 256>>>(w->row_norm, static_cast<const double*>(w->grinv), n, p);
    TMAC_CUDA_TRY(cudaGetLastError());
    *out = p;
    return TMAC_OK;
}

int host_exc_ptr(const tmac_weight_s* w, std::vector<int>& out)
{
    out.assign((size_t)w->rows + 1, 0);
    TMAC_CUDA_TRY(cudaMemcpy(out.data(), w->exc_ptr, (w->rows + 1) * sizeof(int), cudaMemcpyDeviceToHost));
    return TMAC_OK;
}

const tmac_weight_s* find_mat(tmac_model_s* m, const std::string& name)
{
    auto it = m->mats.find(name);
    return it == m->mats.end() ? nullptr : it->second;
}

bool native_blockq(const tmac_weight_s* w, int type, int64_t rows, int64_t cols)
{
    if (!w || w->mode != TMAC_MODE_NATIVE || w->type != type || w->rows != rows || w->cols != cols || !w->exc ||
        !w->exc_ptr || !w->grinv)
        return false;
    int64_t gb = 0;
    if (type == TMAC_TYPE_Q5_0) gb = Geo<TMAC_TYPE_Q5_0>::group_bytes(cols / 32);
    else if (type == TMAC_TYPE_Q4_K) gb = Geo<TMAC_TYPE_Q4_K>::group_bytes(cols / 256);
    else gb = Geo<TMAC_TYPE_Q6_K>::group_bytes(cols / 256);
    return w->group_bytes == gb && w->groups == (rows + 7) / 8;
}

}  // namespace

void mega_free(MegaState* st)
{
    if (!st) return;
    if (st->dev_layers) cudaFree(st->dev_layers);
    if (st->dev_slots) cudaFree(st->dev_slots);
    if (st->dev_abort) cudaFree(st->dev_abort);
    if (st->dev_tagged) cudaFree(st->dev_tagged);
    for (void* p : st->rowc) cudaFree(p);
    delete st;
}

// Builds the copy plans of every CTA; returns TMAC_OK with *out = nullptr when
// the model cannot run on the persistent kernel (a matrix off its FPGA-core
// path, another shape, or shared memory too small), so the caller keeps the
// per-kernel engine.
int mega_prepare(tmac_model_s* m, MegaState** out)
{
    *out = nullptr;
    if (m->max_seq > 1024) return TMAC_OK;
    const int G = num_sms(m->device);
    if (G < 2 * kHeads) return TMAC_OK;
    std::vector<MegaLayer> layers(kLayers);
    std::vector<MegaSlot> slots((size_t)G * kLayers * kSlots);
    uint32_t slot_bytes[kSlots] = {0, 0, 0, 0};
    uint32_t max_rows = 32;
    std::vector<int> ep_a, ep_o, ep_g, ep_d;
    std::map<const tmac_weight_s*, RowConst*> rowc;  // handed to the state on success, else freed
    struct FreeRowc {
        std::map<const tmac_weight_s*, RowConst*>* m;
        ~FreeRowc()
        {
            for (auto& kv : *m) cudaFree(kv.second);
        }
    } free_rowc{&rowc};
    for (int l = 0; l < kLayers; l++) {
        MegaLayer& L = layers[l];
        L.attn_norm = vec_or_null(m, lname(l, "attn_norm.weight"));
        L.ffn_norm = vec_or_null(m, lname(l, "ffn_norm.weight"));
        L.bq = vec_or_null(m, lname(l, "attn_q.bias"));
        L.bk = vec_or_null(m, lname(l, "attn_k.bias"));
        L.bv = vec_or_null(m, lname(l, "attn_v.bias"));
        L.kc = m->kcache + (int64_t)l * m->max_seq * kKvDim;
        L.vc = m->vcache + (int64_t)l * m->max_seq * kKvDim;
        if (!L.attn_norm || !L.ffn_norm) return TMAC_OK;
        const tmac_weight_s* qkv = find_mat(m, lname(l, "attn_qkv"));
        const tmac_weight_s* qk = find_mat(m, lname(l, "attn_qk"));
        const tmac_weight_s* v8 = find_mat(m, lname(l, "attn_v.weight"));
        const tmac_weight_s* wo = find_mat(m, lname(l, "attn_output.weight"));
        const tmac_weight_s* gu = find_mat(m, lname(l, "ffn_gate_up"));
        const tmac_weight_s* wd = find_mat(m, lname(l, "ffn_down.weight"));
        const bool q5_layer = qkv != nullptr;
        if (q5_layer) {
            if (!native_blockq(qkv, TMAC_TYPE_Q5_0, kHidden + 2 * kKvDim, kHidden)) return TMAC_OK;
        } else {
            if (!native_blockq(qk, TMAC_TYPE_Q5_0, kHidden + kKvDim, kHidden)) return TMAC_OK;
            if (!v8 || v8->mode != TMAC_MODE_NATIVE || v8->type != TMAC_TYPE_Q8_0 || v8->rows != kKvDim ||
                v8->cols != kHidden || v8->groups != kKvDim / 32 || v8->group_bytes != (kHidden / 64) * 2176 + 128)
                return TMAC_OK;
        }
        if (!native_blockq(wo, TMAC_TYPE_Q5_0, kHidden, kHidden) ||
            !native_blockq(gu, TMAC_TYPE_Q5_0, 2 * kInter, kHidden) ||
            !(native_blockq(wd, TMAC_TYPE_Q4_K, kHidden, kInter) || native_blockq(wd, TMAC_TYPE_Q6_K, kHidden, kInter)))
            return TMAC_OK;
        int rc;
        if ((rc = host_exc_ptr(q5_layer ? qkv : qk, ep_a)) || (rc = host_exc_ptr(wo, ep_o)) ||
            (rc = host_exc_ptr(gu, ep_g)) || (rc = host_exc_ptr(wd, ep_d)))
            return rc;
        const RowConst *rc_a = nullptr, *rc_o = nullptr, *rc_g = nullptr, *rc_d = nullptr;
        if ((rc = row_consts(q5_layer ? qkv : qk, rowc, &rc_a)) || (rc = row_consts(wo, rowc, &rc_o)) ||
            (rc = row_consts(gu, rowc, &rc_g)) || (rc = row_consts(wd, rowc, &rc_d)))
            return rc;
        for (int c = 0; c < G; c++) {
            MegaSlot* sp = &slots[((size_t)c * kLayers + l) * kSlots];
            int64_t a0[2] = {0, 0}, a1[2] = {0, 0};
            int32_t o0[2] = {0, 0};
            // A: q|k|v rows (Q8_0 layers: q|k over the first G - 4 CTAs, the four
            // 32-row attn_v groups on the last four)
            if (q5_layer) {
                split(qkv->groups, G, c, &a0[0], &a1[0]);
                o0[0] = (int32_t)(8 * a0[0]);
                if ((rc = blockq_slot(qkv, rc_a, ep_a, a0, a1, o0, 1, sp[0]))) return rc;
            } else if (c < G - 4) {
                split(qk->groups, G - 4, c, &a0[0], &a1[0]);
                o0[0] = (int32_t)(8 * a0[0]);
                if ((rc = blockq_slot(qk, rc_a, ep_a, a0, a1, o0, 1, sp[0]))) return rc;
            } else {
                const int gi = c - (G - 4);
                MegaSlot& s0 = sp[0];
                s0 = MegaSlot{};
                s0.kind = SK_Q8;
                s0.rows = 32;
                uint32_t off = 0;
                add_seg(s0, v8->data + gi * v8->group_bytes, (uint32_t)v8->group_bytes, &off);
                s0.out0[0] = kHidden + kKvDim + 32 * gi;
            }
            // C: attn_output rows
            split(wo->groups, G, c, &a0[0], &a1[0]);
            o0[0] = (int32_t)(8 * a0[0]);
            if ((rc = blockq_slot(wo, rc_o, ep_o, a0, a1, o0, 1, sp[1]))) return rc;
            // D: gate groups [p0, p1) with the up groups holding the same rows
            int64_t p0, p1;
            split(gu->groups / 2, G, c, &p0, &p1);
            a0[0] = p0;
            a1[0] = p1;
            a0[1] = gu->groups / 2 + p0;
            a1[1] = gu->groups / 2 + p1;
            o0[0] = (int32_t)(8 * p0);
            o0[1] = 0;
            if ((rc = blockq_slot(gu, rc_g, ep_g, a0, a1, o0, 2, sp[2]))) return rc;
            // E: ffn_down rows
            split(wd->groups, G, c, &a0[0], &a1[0]);
            o0[0] = (int32_t)(8 * a0[0]);
            if ((rc = blockq_slot(wd, rc_d, ep_d, a0, a1, o0, 1, sp[3]))) return rc;
            if (sp[2].kind == SK_NONE) return TMAC_OK;  // phase E relies on every CTA taking part in D
            for (int s = 0; s < kSlots; s++) {
                slot_bytes[s] = std::max(slot_bytes[s], (sp[s].total + 127) / 128 * 128);
                max_rows = std::max(max_rows, sp[s].rows);
            }
        }
    }
    // shared-memory layout
    MegaArgs a{};
    size_t off = 0;
    for (int s = 0; s < kSlots; s++) {
        a.slot_off[s] = (uint32_t)off;
        off += slot_bytes[s];
    }
    a.plan_off = (uint32_t)off;
    off += (size_t)kLayers * kSlots * sizeof(MegaSlot);
    a.x_off = (uint32_t)off;
    off += 2 * kInter;
    a.norm_off = (uint32_t)off;
    off += 2 * kHidden * sizeof(float);
    a.att_off = (uint32_t)off;
    off += (attn_scratch_bytes(m->max_seq) + 127) / 128 * 128;
    a.acc_off = (uint32_t)off;
    a.max_rows = max_rows;
    off += ((size_t)max_rows * 12 + 15) / 16 * 16 + (size_t)(kHidden / 64) * 32 * 8;
    off = (off + 127) / 128 * 128;
    a.misc_off = (uint32_t)off;
    off += (sizeof(MegaMisc) + 127) / 128 * 128;
    if (off > kMaxSmemBytes) return TMAC_OK;
    int coop = 0;
    TMAC_CUDA_TRY(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->device));
    if (!coop) return TMAC_OK;
    TMAC_CUDA_TRY(cudaFuncSetAttribute(decode_mega_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)off));
    int per_sm = 0;
    TMAC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mega_kernel, kMegaThreads, off));
    if (per_sm < 1) return TMAC_OK;

    MegaState* st = new MegaState();
    st->smem = off;
    st->grid = G;
    const size_t n_tagged = (size_t)kHidden + kHidden + 2 * kKvDim + kHidden + kInter;
    cudaError_t e = cudaMalloc(&st->dev_layers, layers.size() * sizeof(MegaLayer));
    if (e == cudaSuccess) e = cudaMalloc(&st->dev_slots, slots.size() * sizeof(MegaSlot));
    if (e == cudaSuccess) e = cudaMalloc(&st->dev_abort, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(&st->dev_tagged, n_tagged * sizeof(unsigned long long));
    if (e == cudaSuccess)
        e = cudaMemcpy(st->dev_layers, layers.data(), layers.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(st->dev_slots, slots.data(), slots.size() * sizeof(MegaSlot), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(st->dev_tagged, 0, n_tagged * sizeof(unsigned long long));  // tag 0: never current
    if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);  // the RowConst arrays are filled
    if (e != cudaSuccess) {
        mega_free(st);
        return cuda_fail(e, "decode kernel set-up");
    }
    for (auto& kv : rowc) st->rowc.push_back(kv.second);
    rowc.clear();
    a.layers = static_cast<const MegaLayer*>(st->dev_layers);
    a.slots = static_cast<const MegaSlot*>(st->dev_slots);
    a.emb = m->emb_raw;
    a.key = m->key;
    a.token_log = m->token_log;
    a.tokens = m->tokens;
    a.pos_dev = m->pos_dev;
    a.hidden = m->hidden;
    a.xn = m->xn;
    a.hidden_log = m->hidden_log;
    a.rope_c = m->rope_c;
    a.rope_s = m->rope_s;
    a.out_norm = vec_or_null(m, "output_norm.weight");
    a.abort_flag = st->dev_abort;
    a.hid_t = st->dev_tagged;
    a.qkv_t = a.hid_t + kHidden;
    a.ctx_t = a.qkv_t + kHidden + 2 * kKvDim;
    a.h_t = a.ctx_t + kHidden;
    a.err = device_error_word(m->device);
    a.max_seq = m->max_seq;
    a.head_cta0 = G - kHeads;
    // the embedding reaches hidden through a CTA that signals layer 0's q|k|v
    // phase, which every later reader of hidden waits for (directly or not)
    a.emb_cta = -1;
    for (int c = 0; c < G && a.emb_cta < 0; c++)
        if (slots[(size_t)c * kLayers * kSlots].kind != SK_NONE) a.emb_cta = c;
    st->args = a;
    *out = st;
    return TMAC_OK;
}

// One token: abort flag cleared, then the persistent kernel (cooperative launch,
// so every CTA is resident before any waits on another).
int mega_launch(MegaState* st, int n_prompt, cudaStream_t s)
{
    TMAC_CUDA_TRY(cudaMemsetAsync(st->dev_abort, 0, sizeof(int), s));
    MegaArgs a = st->args;
    a.n_prompt = n_prompt;
    // tags of this launch: values of earlier launches never match them (the
    // 25-bit epoch wraps after 2^25 tokens, long after any value is rewritten)
    st->epoch = (st->epoch + 1) & 0x1FFFFFFu;
    if (st->epoch == 0) st->epoch = 1;
    a.epoch = st->epoch;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(st->grid);
    cfg.blockDim = dim3(kMegaThreads);
    cfg.dynamicSmemBytes = st->smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    TMAC_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_mega_kernel, a));
    return TMAC_OK;
}

}  // namespace tmac

#ifdef TMAC_TRACE
extern "C" int tmac_trace_read_mega(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, tmac::g_mega_trace, sizeof(tmac::g_mega_trace));
}
extern "C" int tmac_trace_read_bq(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, tmac::g_bq_trace, sizeof(tmac::g_bq_trace));
}
extern "C" int tmac_trace_read_norm(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, tmac::g_norm_trace, sizeof(tmac::g_norm_trace));
}
extern "C" int tmac_trace_read_att(unsigned long long* out)
{
    return (int)cudaMemcpyFromSymbol(out, tmac::g_att_trace, sizeof(tmac::g_att_trace));
}
#endif
