// xchg.cuh -- the peer-memory top-1 exchange shared by xchg.cu (a kernel of its
// own) and the Q8_0 logits GEMV (fused into its last CTA, gemv_q8_0.cu).
//
// Buffer of each rank: keys[2][world] then tags[2][world] (uint64).  Step s uses
// half s & 1: the key is stored into every rank's buffer, then the tag s with
// release semantics at system scope; the reader acquires each rank's tag in its
// own buffer before reading the key.  A rank can be at most one step ahead of
// another (it cannot finish step s + 1 before every rank has published s + 1,
// which each does only after reading step s), so the other half is never
// overwritten while it is still being read.  Waits are bounded (~2 s).
#pragma once

#include "common.cuh"

#include <vector>

struct tmac_xchg_s {
    int device = 0, world = 0, rank = 0;
    uint64_t* buf = nullptr;           // this rank's keys[2][world] | tags[2][world]
    uint64_t* step = nullptr;          // device step counter of this rank
    unsigned long long* partial = nullptr;  // fused GEMV: running key of this rank's shard
    unsigned* counter = nullptr;            // fused GEMV: CTAs finished
    std::vector<uint64_t*> peer;       // every rank's buffer as mapped here (own = buf)
    std::vector<char> ipc_mapped;      // peer[r] came from cudaIpcOpenMemHandle
    int64_t vocab = 0;                 // > 0: full logits [2][vocab] floats after the keys
    size_t logits_off = 0;             // byte offset of the logits in every rank's buffer
    uint64_t host_steps = 0;           // exchange steps enqueued so far
    uint64_t** peer_dev = nullptr;     // the same table on the device
};

namespace tmac {

struct XchgDev {
    uint64_t** peers = nullptr;  // nullptr: no exchange
    uint64_t* own = nullptr;
    uint64_t* step = nullptr;
    unsigned long long* partial = nullptr;
    unsigned* counter = nullptr;
    int world = 0, rank = 0;
    int64_t vocab = 0;       // > 0: every rank's full-logits buffers are written too
    size_t logits_off = 0;   // their byte offset in each rank's exchange buffer
};

// Full-logits buffer of rank q for the step about to run (its parity half):
// the logits GEMV stores its shard there in every rank, so each rank ends
// the step holding the whole vector.
TMAC_DEV float* xchg_logits(const XchgDev& x, int q, uint64_t step)
{
    return reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(x.peers[q]) + x.logits_off) + (step & 1) * x.vocab;
}

TMAC_DEV void st_release_sys(uint64_t* p, uint64_t v)
{
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
TMAC_DEV uint64_t ld_acquire_sys(const uint64_t* p)
{
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Publishes `k` for this step to rank t (thread t < world).
TMAC_DEV void xchg_publish(const XchgDev& x, int t, uint64_t step, unsigned long long k)
{
    const int half = (int)(step & 1);
    uint64_t* dst = x.peers[t];
    dst[half * x.world + x.rank] = k;
    st_release_sys(dst + 2 * x.world + half * x.world + x.rank, step);
}

// Rank t's key of this step from the own buffer; false after the wait limit.
TMAC_DEV bool xchg_read(const XchgDev& x, int t, uint64_t step, unsigned long long* k)
{
    const int half = (int)(step & 1);
    const uint64_t* tag = x.own + 2 * x.world + half * x.world + t;
    if (ld_acquire_sys(tag) != step) {
        const uint64_t t0 = global_timer_ns();
        for (uint32_t it = 1;; it++) {
            if (ld_acquire_sys(tag) == step) break;
            if ((it & 255u) == 0 && global_timer_ns() - t0 > wait_limit_ns()) return false;
        }
    }
    *k = x.own[half * x.world + t];
    return true;
}

TMAC_DEV void st_relaxed_sys(uint64_t* p, uint64_t v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// One warp (all 32 lanes): publish `k` to every rank, then the maximum of every
// rank's key (*out unchanged and TMAC_ERR_TIMEOUT recorded if a rank does not
// arrive).  Lane t serves ranks t, t + 32, ...: the key stores, ONE
// system-scope fence, then relaxed tag stores (a release pattern for every
// tag), and the tags of all ranks are polled at once.  A release store per rank
// from one thread would pay one system-scope fence per rank, in sequence.
TMAC_DEV void xchg_top1_warp(const XchgDev& x, unsigned long long k, unsigned long long* out, int* err)
{
    const int lane = threadIdx.x & 31;
    uint64_t step = 0;
    if (lane == 0) step = *x.step + 1;
    step = __shfl_sync(0xffffffffu, step, 0);
    k = __shfl_sync(0xffffffffu, k, 0);
    const int half = (int)(step & 1);
    for (int t = lane; t < x.world; t += 32) x.peers[t][half * x.world + x.rank] = k;
    __threadfence_system();
    for (int t = lane; t < x.world; t += 32) st_relaxed_sys(x.peers[t] + 2 * x.world + half * x.world + x.rank, step);
    unsigned long long m = 0;
    bool ok = true;
    for (int t = lane; t < x.world && ok; t += 32) {
        unsigned long long v = 0;
        ok = xchg_read(x, t, step, &v);
        m = v > m ? v : m;
    }
    ok = __all_sync(0xffffffffu, ok);
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, m, o);
        m = v > m ? v : m;
    }
    if (lane == 0) {
        if (ok) *out = m;
        else if (err) atomicExch(err, (int)TMAC_ERR_TIMEOUT);
        *x.step = step;
    }
}

// One thread: publish to every rank, then the maximum of every rank's key
// (*out unchanged and TMAC_ERR_TIMEOUT recorded if a rank does not arrive).
TMAC_DEV void xchg_top1_thread(const XchgDev& x, unsigned long long k, unsigned long long* out, int* err)
{
    const uint64_t step = *x.step + 1;
    for (int t = 0; t < x.world; t++) xchg_publish(x, t, step, k);
    unsigned long long m = 0;
    bool ok = true;
    for (int t = 0; t < x.world && ok; t++) {
        unsigned long long v = 0;
        ok = xchg_read(x, t, step, &v);
        m = v > m ? v : m;
    }
    if (ok) *out = m;
    else if (err) atomicExch(err, (int)TMAC_ERR_TIMEOUT);
    *x.step = step;
}

// End of a GEMV CTA that tracks the top-1 key of its rows: every warp of the
// `bar_threads` (named barrier `bar_id`) calls it with its warp-reduced key;
// `slots` is shared memory for one key per calling warp, `slot` this warp's.
// The CTA's maximum is merged with one atomic.  Without a running key
// (xg.partial == nullptr) it max-merges into *top1, which the caller zeroed.
// With one, it max-merges into the running key and the last CTA to finish
// (atomic count) takes that, resetting it and the count for the next call,
// and writes it to *top1 -- after merging it with every rank's key over peer
// memory when xg.peers is set.
TMAC_DEV void top1_cta_finish(const XchgDev& xg, unsigned long long* top1, unsigned long long best,
                              unsigned long long* slots, int slot, bool leader_warp, int bar_id, int bar_threads,
                              int* err)
{
    const int lane = threadIdx.x & 31;
    if (lane == 0) slots[slot] = best;
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(bar_threads) : "memory");
    if (!(leader_warp && lane == 0)) return;
    // full logits: the peer stores of the CTA's warps (ordered before this
    // thread by the barrier) reach the other GPUs before the key that the last
    // CTA publishes with a system-scope release
    if (xg.vocab) __threadfence_system();
    unsigned long long m = 0;
    for (int w = 0; w < bar_threads / 32; w++) m = slots[w] > m ? slots[w] : m;
    if (!xg.partial) {
        if (m) atomicMax(top1, m);
        return;
    }
    if (m) atomicMax(xg.partial, m);
    // acquire-release count: each CTA's max is ordered before its increment,
    // and the CTA that sees the last increment sees every max
    unsigned done;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(done) : "l"(xg.counter) : "memory");
    if (done == gridDim.x - 1) {
        const unsigned long long k = atomicExch(xg.partial, 0ull);
        atomicExch(xg.counter, 0u);
        if (xg.peers)
            xchg_top1_thread(xg, k, top1, err);
        else
            *top1 = k;
    }
}

// The same end of a GEMV CTA for the fused exchange across ranks (xg.peers
// and xg.partial set): the last CTA's whole leader warp publishes this rank's
// key and merges every rank's (xchg_top1_warp).  A separate function, so the
// kernel without peers carries none of the warp exchange code.
TMAC_DEV void top1_cta_finish_peers(const XchgDev& xg, unsigned long long* top1, unsigned long long best,
                                    unsigned long long* slots, int slot, bool leader_warp, int bar_id,
                                    int bar_threads, int* err)
{
    const int lane = threadIdx.x & 31;
    if (lane == 0) slots[slot] = best;
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(bar_threads) : "memory");
    if (!leader_warp) return;
    unsigned done = 0;
    unsigned long long k = 0;
    if (lane == 0) {
        // full logits: the peer stores of the CTA's warps (ordered before this
        // thread by the barrier) reach the other GPUs before the key that the
        // last CTA publishes with a system-scope release pattern
        if (xg.vocab) __threadfence_system();
        unsigned long long m = 0;
        for (int w = 0; w < bar_threads / 32; w++) m = slots[w] > m ? slots[w] : m;
        if (m) atomicMax(xg.partial, m);
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(done) : "l"(xg.counter) : "memory");
        if (done == gridDim.x - 1) {
            k = atomicExch(xg.partial, 0ull);
            atomicExch(xg.counter, 0u);
        }
    }
    done = __shfl_sync(0xffffffffu, done, 0);
    if (done != gridDim.x - 1) return;
    // what lane 0 acquired is ordered before the other lanes' exchange stores
    __syncwarp();
    xchg_top1_warp(xg, k, top1, err);
}

XchgDev xchg_dev(const tmac_xchg_s* x);  // xchg.cu

}  // namespace tmac
