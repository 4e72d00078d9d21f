// xchg.cu -- the logits top-1 merge across GPUs over NVLink peer memory.
//
// Each rank's logits GEMV leaves the packed top-1 key of its vocab shard on its
// device (tmac_gemv_top1).  The global greedy token is the maximum key over the
// ranks (the reference's sample_token with top-1, sim/tmac_gguf.cpp:1974-1990,
// over the whole vocabulary).  Instead of a library all-reduce, one small kernel
// per step stores the key into a slot of every rank's exchange buffer (plain
// stores to peer memory through CUDA IPC mappings), then waits for every
// rank's slot of this step in its own buffer and takes the maximum.
//
// Buffer of each rank: keys[2][world] then tags[2][world] (uint64).  Step s uses
// half s & 1: the key is stored, then the tag s with release semantics at system
// scope; the reader acquires the tag before reading the key.  A rank can be at
// most one step ahead of another (it cannot finish step s + 1 before every rank
// has published s + 1, which each does only after reading step s), so the other
// half is never overwritten while it is still being read.  Every wait is
// bounded (tmac_set_wait_limit_ns, 2 s by default): on expiry the kernel records
// TMAC_ERR_TIMEOUT, leaves the key as it was and returns.  The step counters of
// the ranks then no longer agree, so an exchange that timed out is freed and
// created again on every rank before the next step.
#include "xchg.cuh"

#include <cstring>
#include <map>
#include <mutex>
#include <string>

namespace tmac {

XchgDev xchg_dev(const tmac_xchg_s* x)
{
    XchgDev d;
    d.peers = x->peer_dev;
    d.own = x->buf;
    d.step = x->step;
    d.partial = x->partial;
    d.counter = x->counter;
    d.world = x->world;
    d.rank = x->rank;
    d.vocab = x->vocab;
    d.logits_off = x->logits_off;
    return d;
}

namespace {

constexpr int kMaxRanks = 64;

// Exchange buffers created in this process, by their IPC handle: a rank whose
// peer lives in the same process (ranks driven by threads of one process)
// reaches that buffer through its device address -- CUDA cannot open an IPC
// handle in the process that exported it.
struct LocalBuf {
    int device;
    uint64_t* buf;
};
std::mutex g_local_mu;
std::map<std::string, LocalBuf>& local_bufs()
{
    static std::map<std::string, LocalBuf> m;
    return m;
}

// One warp per 32 ranks; thread r publishes to rank r and reads rank r's slot.
__global__ void xchg_top1_kernel(unsigned long long* key, XchgDev x, int* err)
{
    __shared__ unsigned long long best[kMaxRanks / 32];
    __shared__ int failed;
    pdl_launch();
    pdl_wait();  // the key comes from the preceding kernel
    const int t = threadIdx.x;
    const uint64_t step = *x.step + 1;
    if (t == 0) failed = 0;
    __syncthreads();
    if (t < x.world) xchg_publish(x, t, step, *key);
    unsigned long long mine = 0;
    if (t < x.world && !xchg_read(x, t, step, &mine)) {
        failed = 1;
        if (err) atomicExch(err, (int)TMAC_ERR_TIMEOUT);
    }
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, mine, o);
        mine = v > mine ? v : mine;
    }
    if ((t & 31) == 0) best[t >> 5] = mine;
    __syncthreads();
    if (t == 0) {
        unsigned long long m = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); w++) m = best[w] > m ? best[w] : m;
        if (!failed) *key = m;
        *x.step = step;
    }
}

}  // namespace
}  // namespace tmac

using namespace tmac;

extern "C" {

int tmac_xchg_create(int device, int world, int rank, tmac_xchg_t* out)
{
    return tmac_xchg_create_logits(device, world, rank, 0, out);
}

int tmac_xchg_create_logits(int device, int world, int rank, int64_t vocab, tmac_xchg_t* out)
{
    if (!out) return fail(TMAC_ERR_INVALID, "NULL output");
    *out = nullptr;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) return fail(TMAC_ERR_SHAPE, "bad world / rank");
    if (vocab < 0 || vocab > 0x7FFFFFFF) return fail(TMAC_ERR_SHAPE, "bad vocabulary size");
    DeviceGuard dg(device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    tmac_xchg_s* x = new tmac_xchg_s();
    x->device = device;
    x->world = world;
    x->rank = rank;
    x->vocab = vocab;
    x->logits_off = ((size_t)4 * world * sizeof(uint64_t) + 255) / 256 * 256;
    // keys | tags, then (vocab > 0) the full logits of the two step parities:
    // one allocation, so one IPC handle maps everything a peer writes
    const size_t bytes = vocab ? x->logits_off + (size_t)2 * vocab * sizeof(float) : (size_t)4 * world * sizeof(uint64_t);
    cudaError_t e = cudaMalloc(&x->buf, bytes);
    if (e == cudaSuccess) e = cudaMemset(x->buf, 0, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&x->step, sizeof(uint64_t));
    if (e == cudaSuccess) e = cudaMemset(x->step, 0, sizeof(uint64_t));
    if (e == cudaSuccess) e = cudaMalloc(&x->peer_dev, world * sizeof(uint64_t*));
    if (e == cudaSuccess) e = cudaMalloc(&x->partial, sizeof(unsigned long long) + sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(x->partial, 0, sizeof(unsigned long long) + sizeof(unsigned));
    if (e == cudaSuccess) x->counter = reinterpret_cast<unsigned*>(x->partial + 1);
    if (e != cudaSuccess) {
        if (x->buf) cudaFree(x->buf);
        if (x->step) cudaFree(x->step);
        if (x->peer_dev) cudaFree(x->peer_dev);
        if (x->partial) cudaFree(x->partial);
        delete x;
        return cuda_fail(e, "tmac_xchg_create");
    }
    x->peer.assign(world, nullptr);
    x->ipc_mapped.assign(world, 0);
    x->peer[rank] = x->buf;
    *out = x;
    return TMAC_OK;
}

int tmac_xchg_ipc_handle(tmac_xchg_t x, void* handle)
{
    if (!x || !handle) return fail(TMAC_ERR_INVALID, "NULL argument");
    DeviceGuard dg(x->device);
    cudaIpcMemHandle_t h;
    TMAC_CUDA_TRY(cudaIpcGetMemHandle(&h, x->buf));
    memcpy(handle, &h, sizeof(h));
    std::lock_guard<std::mutex> lk(g_local_mu);
    local_bufs()[std::string((const char*)&h, sizeof(h))] = LocalBuf{x->device, x->buf};
    return TMAC_OK;
}

int tmac_xchg_open(tmac_xchg_t x, const void* handles)
{
    if (!x || !handles) return fail(TMAC_ERR_INVALID, "NULL argument");
    DeviceGuard dg(x->device);
    for (int r = 0; r < x->world; r++) {
        if (r == x->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t*)handles + (size_t)r * TMAC_XCHG_HANDLE_BYTES, sizeof(h));
        LocalBuf local{-1, nullptr};
        {
            std::lock_guard<std::mutex> lk(g_local_mu);
            auto it = local_bufs().find(std::string((const char*)&h, sizeof(h)));
            if (it != local_bufs().end()) local = it->second;
        }
        if (local.buf) {  // same process: the device address, with peer access across devices
            if (local.device != x->device) {
                const cudaError_t e = cudaDeviceEnablePeerAccess(local.device, 0);
                if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) return cuda_fail(e, "peer access");
                cudaGetLastError();
            }
            x->peer[r] = local.buf;
            x->ipc_mapped[r] = 0;
            continue;
        }
        void* p = nullptr;
        TMAC_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        x->peer[r] = static_cast<uint64_t*>(p);
        x->ipc_mapped[r] = 1;
    }
    TMAC_CUDA_TRY(cudaMemcpy(x->peer_dev, x->peer.data(), x->world * sizeof(uint64_t*), cudaMemcpyHostToDevice));
    return TMAC_OK;
}

int tmac_xchg_top1(tmac_xchg_t x, uint64_t* key, void* stream)
{
    if (!x || !key) return fail(TMAC_ERR_INVALID, "NULL argument");
    for (int r = 0; r < x->world; r++)
        if (!x->peer[r]) return fail(TMAC_ERR_INVALID, "tmac_xchg_open has not mapped every rank");
    DeviceGuard dg(x->device);
    const int threads = (x->world + 31) / 32 * 32;
    TMAC_CUDA_TRY(launch_k(xchg_top1_kernel, dim3(1), dim3(threads), 0, (cudaStream_t)stream,
                           reinterpret_cast<unsigned long long*>(key), xchg_dev(x), device_error_word(x->device)));
    TMAC_CUDA_TRY(cudaGetLastError());
    x->host_steps++;
    return TMAC_OK;
}

int tmac_xchg_gemv_top1(tmac_xchg_t x, tmac_weight_t w, const float* in, float* y, uint64_t* key,
                        int64_t index_base, void* stream)
{
    if (!x || !w || !in || !y || !key) return fail(TMAC_ERR_INVALID, "NULL argument");
    for (int r = 0; r < x->world; r++)
        if (!x->peer[r]) return fail(TMAC_ERR_INVALID, "tmac_xchg_open has not mapped every rank");
    if (w->device != x->device) return fail(TMAC_ERR_INVALID, "weight and exchange on different devices");
    if (!(w->mode == TMAC_MODE_NATIVE && w->type == TMAC_TYPE_Q8_0)) {
        if (x->vocab) return fail(TMAC_ERR_TYPE, "the full-logits exchange needs a NATIVE Q8_0 logits weight");
        const int rc = tmac_gemv_top1(w, in, y, key, index_base, 1, stream);
        return rc ? rc : tmac_xchg_top1(x, key, stream);
    }
    if (index_base < 0 || index_base + w->rows > 0x7FFFFFFF) return fail(TMAC_ERR_SHAPE, "bad index range");
    if (x->vocab && index_base + w->rows > x->vocab) return fail(TMAC_ERR_SHAPE, "shard rows beyond the vocabulary");
    DeviceGuard dg(x->device);
    const XchgDev d = xchg_dev(x);
    const int rc = launch_q8_0(w, in, y, nullptr, nullptr, 1, (cudaStream_t)stream,
                               reinterpret_cast<unsigned long long*>(key), index_base, nullptr, nullptr, &d);
    if (!rc) x->host_steps++;
    return rc;
}

int tmac_xchg_logits(tmac_xchg_t x, float** logits)
{
    if (!x || !logits) return fail(TMAC_ERR_INVALID, "NULL argument");
    if (!x->vocab) return fail(TMAC_ERR_INVALID, "exchange created without a logits buffer");
    if (!x->host_steps) return fail(TMAC_ERR_INVALID, "no exchange step has run yet");
    *logits = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(x->buf) + x->logits_off) +
              (x->host_steps & 1) * x->vocab;
    return TMAC_OK;
}

int tmac_xchg_free(tmac_xchg_t x)
{
    if (!x) return TMAC_OK;
    DeviceGuard dg(x->device);
    for (int r = 0; r < x->world; r++)
        if (r != x->rank && x->peer[r] && x->ipc_mapped[r]) cudaIpcCloseMemHandle(x->peer[r]);
    {
        std::lock_guard<std::mutex> lk(g_local_mu);
        for (auto it = local_bufs().begin(); it != local_bufs().end();)
            it = (it->second.buf == x->buf) ? local_bufs().erase(it) : std::next(it);
    }
    cudaFree(x->peer_dev);
    cudaFree(x->partial);
    cudaFree(x->step);
    cudaFree(x->buf);
    delete x;
    return TMAC_OK;
}

}  // extern "C"
