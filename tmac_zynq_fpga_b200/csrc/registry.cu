// registry.cu -- the C ABI of libtmac_cuda.so (include/tmac_cuda.h): weight
// registration, dispatch to the per-type kernels, host-buffer convenience
// entry, error reporting.
//
// Dispatch mirrors the reference's matmul() switch (sim/tmac_gguf.cpp:473-493)
// at registration time: a weight is registered for one reproduction mode
// (NATIVE = the type's FPGA core path, INT16 = matmul_fpga_int16, F32 = the
// FP32 dequant path), and tmac_gemv runs that mode's kernel.  There is no CPU
// fallback: every path is a CUDA kernel, and a missing device is an error.
#include "common.cuh"

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace tmac {

namespace {
thread_local std::string g_last_error;

__device__ int g_device_error;  // one word per device (module global)

std::mutex g_dev_mutex;
std::vector<cudaError_t (*)(unsigned long long)>& wait_limit_setters();
std::vector<int*> g_err_ptr;    // per device: address of g_device_error
std::vector<int> g_sms;
}  // namespace

thread_local bool g_pdl = false;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg)
{
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char* what)
{
    char buf[512];
    snprintf(buf, sizeof(buf), "CUDA error %d (%s) in %s", (int)e, cudaGetErrorString(e), what);
    g_last_error = buf;
    return (e == cudaErrorMemoryAllocation) ? TMAC_ERR_NOMEM : TMAC_ERR_CUDA;
}

int* device_error_word(int device)
{
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if (device < 0) return nullptr;
    if ((int)g_err_ptr.size() <= device) g_err_ptr.resize(device + 1, nullptr);
    if (!g_err_ptr[device]) {
        DeviceGuard dg(device);
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        g_err_ptr[device] = static_cast<int*>(p);
    }
    return g_err_ptr[device];
}

int num_sms(int device)
{
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if ((int)g_sms.size() <= device) g_sms.resize(device + 1, 0);
    if (!g_sms[device]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
        g_sms[device] = n > 0 ? n : 148;
    }
    return g_sms[device];
}

namespace {

int64_t block_values(int type)
{
    switch (type) {
    case TMAC_TYPE_Q8_0:
    case TMAC_TYPE_Q5_0: return 32;
    case TMAC_TYPE_Q4_K:
    case TMAC_TYPE_Q6_K: return 256;
    case TMAC_TYPE_F32:
    case TMAC_TYPE_F16: return 1;
    default: return 0;
    }
}

int64_t block_bytes(int type)
{
    switch (type) {
    case TMAC_TYPE_Q8_0: return 34;
    case TMAC_TYPE_Q5_0: return 22;
    case TMAC_TYPE_Q4_K: return 144;
    case TMAC_TYPE_Q6_K: return 210;
    case TMAC_TYPE_F32: return 4;
    case TMAC_TYPE_F16: return 2;
    default: return 0;
    }
}

int check_device(int device)
{
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return fail(TMAC_ERR_NODEV, "no CUDA device available");
    if (device < 0 || device >= n) return fail(TMAC_ERR_INVALID, "device index out of range");
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0)
        return fail(TMAC_ERR_NODEV, "libtmac_cuda.so is built for sm_100a (B200) only");
    return TMAC_OK;
}

int weight_ok(tmac_weight_t w)
{
    if (!w) return fail(TMAC_ERR_INVALID, "NULL weight handle");
    return TMAC_OK;
}

// Per-device x/y staging buffers of tmac_gemv_host, grown on demand.
struct Staging {
    float* x = nullptr;
    float* y = nullptr;
    size_t xcap = 0, ycap = 0;
};
std::vector<Staging> g_staging;

int staging(int device, size_t xb, size_t yb, float** dx, float** dy)
{
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if ((int)g_staging.size() <= device) g_staging.resize(device + 1);
    Staging& st = g_staging[device];
    if (st.xcap < xb) {
        if (st.x) cudaFree(st.x);
        st.x = nullptr;
        st.xcap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&st.x, xb));
        st.xcap = xb;
    }
    if (st.ycap < yb) {
        if (st.y) cudaFree(st.y);
        st.y = nullptr;
        st.ycap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&st.y, yb));
        st.ycap = yb;
    }
    *dx = st.x;
    *dy = st.y;
    return TMAC_OK;
}

// Per-device activation workspace of the two-kernel block-quant GEMV path:
// x_q (2 bytes per value, stored as byte planes) and x_scale for up to
// `xq_cap` values / `xs_cap` vectors.
struct Workspace {
    int16_t* xq = nullptr;
    float* xs = nullptr;
    size_t xq_cap = 0, xs_cap = 0;
};
std::vector<Workspace> g_ws;

int workspace(int device, size_t nxq, size_t nxs, int16_t** xq, float** xs)
{
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if ((int)g_ws.size() <= device) g_ws.resize(device + 1);
    Workspace& w = g_ws[device];
    if (w.xq_cap < nxq) {
        if (w.xq) cudaFree(w.xq);
        w.xq = nullptr;
        w.xq_cap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&w.xq, nxq * sizeof(int16_t)));
        w.xq_cap = nxq;
    }
    if (w.xs_cap < nxs) {
        if (w.xs) cudaFree(w.xs);
        w.xs = nullptr;
        w.xs_cap = 0;
        TMAC_CUDA_TRY(cudaMalloc(&w.xs, nxs * sizeof(float)));
        w.xs_cap = nxs;
    }
    *xq = w.xq;
    *xs = w.xs;
    return TMAC_OK;
}

// Fixed scratch of tmac_gemv_static: x_q and x_scale in module memory, so that
// entry point never allocates.  Its address is resolved once per device (with
// that device current) and cached.  Every element the GEMV reads is written by
// the quantise kernel first, so nothing here has to start at zero.
constexpr int64_t kStaticXq = TMAC_STATIC_MAX_VALUES;
constexpr int kStaticXs = TMAC_STATIC_MAX_BATCH;
__device__ __align__(256) int16_t g_static_xq[kStaticXq];
__device__ __align__(256) float g_static_xs[kStaticXs];
std::vector<int16_t*> g_static_xq_ptr;
std::vector<float*> g_static_xs_ptr;

int static_scratch(int device, int16_t** xq, float** xs)
{
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if ((int)g_static_xq_ptr.size() <= device) {
        g_static_xq_ptr.resize(device + 1, nullptr);
        g_static_xs_ptr.resize(device + 1, nullptr);
    }
    if (!g_static_xq_ptr[device]) {
        void* a = nullptr;
        void* b = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&a, g_static_xq);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_static_xq)");
        e = cudaGetSymbolAddress(&b, g_static_xs);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_static_xs)");
        g_static_xq_ptr[device] = static_cast<int16_t*>(a);
        g_static_xs_ptr[device] = static_cast<float*>(b);
    }
    *xq = g_static_xq_ptr[device];
    *xs = g_static_xs_ptr[device];
    return TMAC_OK;
}

std::vector<cudaError_t (*)(unsigned long long)>& wait_limit_setters()
{
    static std::vector<cudaError_t (*)(unsigned long long)> v;
    return v;
}

void free_weight(tmac_weight_s* w)
{
    if (!w) return;
    DeviceGuard dg(w->device);
    if (w->data) cudaFree(w->data);
    if (w->row_norm) cudaFree(w->row_norm);
    if (w->exc_ptr) cudaFree(w->exc_ptr);
    if (w->exc) cudaFree(w->exc);
    if (w->gwh) cudaFree(w->gwh);
    if (w->gwl) cudaFree(w->gwl);
    if (w->grinv) cudaFree(w->grinv);
    if (w->top1_scratch) cudaFree(w->top1_scratch);
    delete w;
}

}  // namespace

int register_wait_limit_setter(cudaError_t (*set)(unsigned long long))
{
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    wait_limit_setters().push_back(set);
    return (int)wait_limit_setters().size();
}

}  // namespace tmac

using namespace tmac;

extern "C" {

int tmac_abi_version(void) { return TMAC_ABI_VERSION; }

const char* tmac_last_error(void) { return g_last_error.c_str(); }

int tmac_set_wait_limit_ns(int device, uint64_t ns)
{
    int rc = check_device(device);
    if (rc) return rc;
    if (ns == 0) return fail(TMAC_ERR_INVALID, "the wait limit must be positive");
    DeviceGuard dg(device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    for (auto set : wait_limit_setters()) TMAC_CUDA_TRY(set((unsigned long long)ns));
    return TMAC_OK;
}

int tmac_set_pdl(int on)
{
    const int prev = g_pdl ? 1 : 0;
    g_pdl = on != 0;
    return prev;
}

int tmac_device_error(int device, int* code)
{
    if (!code) return fail(TMAC_ERR_INVALID, "NULL code pointer");
    int rc = check_device(device);
    if (rc) return rc;
    DeviceGuard dg(device);
    int* p = device_error_word(device);
    if (!p) return fail(TMAC_ERR_CUDA, "cannot resolve device error word");
    TMAC_CUDA_TRY(cudaDeviceSynchronize());
    int v = 0, zero = 0;
    TMAC_CUDA_TRY(cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost));
    TMAC_CUDA_TRY(cudaMemcpy(p, &zero, sizeof(int), cudaMemcpyHostToDevice));
    *code = v;
    return TMAC_OK;
}

int64_t tmac_units_per_row(int type, int mode, int64_t cols)
{
    if (mode == TMAC_MODE_INT16) return (cols + 63) / 64;
    if (mode != TMAC_MODE_NATIVE) return 0;
    switch (type) {
    case TMAC_TYPE_Q8_0: return (cols + 63) / 64;
    case TMAC_TYPE_Q5_0: return cols / 32;
    case TMAC_TYPE_Q4_K:
    case TMAC_TYPE_Q6_K: return cols / 256;
    default: return 0;
    }
}

int tmac_weight_register(int type, int mode, int64_t rows, int64_t cols, const void* blocks, size_t n_bytes,
                         int blocks_on_device, const float* row_max_abs, int device, tmac_weight_t* out)
{
    if (!out || !blocks) return fail(TMAC_ERR_INVALID, "NULL argument");
    *out = nullptr;
    if (rows <= 0 || cols <= 0) return fail(TMAC_ERR_SHAPE, "rows and cols must be positive");
    const int64_t bv = block_values(type);
    if (!bv) return fail(TMAC_ERR_TYPE, "unsupported tensor type " + std::to_string(type));
    if (mode != TMAC_MODE_NATIVE && mode != TMAC_MODE_INT16 && mode != TMAC_MODE_F32)
        return fail(TMAC_ERR_INVALID, "unknown mode");
    if (mode == TMAC_MODE_NATIVE && (type == TMAC_TYPE_F32 || type == TMAC_TYPE_F16))
        return fail(TMAC_ERR_TYPE, "F32/F16 tensors have no FPGA core path; use INT16 or F32 mode");
    if (cols % bv) return fail(TMAC_ERR_SHAPE, "cols is not a multiple of the block size");
    const size_t need = (size_t)(rows * (cols / bv) * block_bytes(type));
    if (n_bytes < need) return fail(TMAC_ERR_BOUNDS, "n_bytes smaller than the tensor's blocks");
    int rc = check_device(device);
    if (rc) return rc;
    DeviceGuard dg(device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");

    tmac_weight_s* w = new tmac_weight_s();
    w->type = type;
    w->mode = mode;
    w->rows = rows;
    w->cols = cols;
    w->device = device;

    uint8_t* d_raw = nullptr;
    float* d_rma = nullptr;
    bool raw_owned = false;
    cudaStream_t s = nullptr;
    auto cleanup = [&](int code) {
        if (raw_owned && d_raw && d_raw != w->data) cudaFree(d_raw);
        if (d_rma) cudaFree(d_rma);
        if (code != TMAC_OK) free_weight(w);
        return code;
    };
    cudaError_t e;
    if (blocks_on_device) {
        d_raw = (uint8_t*)blocks;
    } else {
        if ((e = cudaMalloc(&d_raw, need)) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(raw)"));
        raw_owned = true;
        if ((e = cudaMemcpy(d_raw, blocks, need, cudaMemcpyHostToDevice)) != cudaSuccess)
            return cleanup(cuda_fail(e, "cudaMemcpy(raw)"));
    }
    if (row_max_abs && type == TMAC_TYPE_Q8_0 && mode == TMAC_MODE_NATIVE) {
        if ((e = cudaMalloc(&d_rma, rows * sizeof(float))) != cudaSuccess)
            return cleanup(cuda_fail(e, "cudaMalloc(row_max_abs)"));
        if ((e = cudaMemcpy(d_rma, row_max_abs, rows * sizeof(float), cudaMemcpyHostToDevice)) != cudaSuccess)
            return cleanup(cuda_fail(e, "cudaMemcpy(row_max_abs)"));
    }
    if (mode == TMAC_MODE_NATIVE && type == TMAC_TYPE_Q8_0) {
        rc = register_q8_0(w, d_raw, d_rma, s);
    } else if (mode == TMAC_MODE_NATIVE) {
        // Q5_0 / Q4_K / Q6_K: re-laid out in row groups (gemv_blockq.cu)
        rc = register_blockq(w, d_raw, s);
    } else if (mode == TMAC_MODE_INT16) {
        rc = register_int16(w, d_raw, s);
    } else {
        if (raw_owned) {
            w->data = d_raw;
        } else {
            if ((e = cudaMalloc(&w->data, need)) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(data)"));
            if ((e = cudaMemcpy(w->data, d_raw, need, cudaMemcpyDeviceToDevice)) != cudaSuccess)
                return cleanup(cuda_fail(e, "cudaMemcpy(data)"));
        }
        w->data_bytes = need;
        rc = register_f32(w, w->data, s);
    }
    if (rc != TMAC_OK) return cleanup(rc);
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cleanup(cuda_fail(e, "registration kernels"));
    device_error_word(device);
    *out = w;
    return cleanup(TMAC_OK);
}

int tmac_weight_free(tmac_weight_t w)
{
    if (!w) return TMAC_OK;
    free_weight(w);
    return TMAC_OK;
}

int tmac_weight_info(tmac_weight_t w, int* type, int* mode, int64_t* rows, int64_t* cols, int* device)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (type) *type = w->type;
    if (mode) *mode = w->mode;
    if (rows) *rows = w->rows;
    if (cols) *cols = w->cols;
    if (device) *device = w->device;
    return TMAC_OK;
}

int tmac_weight_device_bytes(tmac_weight_t w, size_t* bytes)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (!bytes) return fail(TMAC_ERR_INVALID, "NULL bytes pointer");
    *bytes = w->data_bytes + (w->row_norm && w->type != TMAC_TYPE_Q8_0 ? w->rows * sizeof(float) : 0) +
             (w->exc_ptr ? (size_t)(w->groups * 8 + 4) * sizeof(int) + w->n_exc * 16 : 0);
    return TMAC_OK;
}

int tmac_weight_row_norm(tmac_weight_t w, float* out)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (!out) return fail(TMAC_ERR_INVALID, "NULL output");
    if (!w->row_norm) return fail(TMAC_ERR_TYPE, "this weight mode has no row normaliser");
    DeviceGuard dg(w->device);
    TMAC_CUDA_TRY(cudaMemcpy(out, w->row_norm, w->rows * sizeof(float), cudaMemcpyDeviceToHost));
    return TMAC_OK;
}

int tmac_gemv_acc(tmac_weight_t w, const float* x, float* y, int64_t* row_acc, int64_t* unit_acc, int batch,
                  void* stream)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (!x || !y) return fail(TMAC_ERR_INVALID, "NULL x or y");
    if (batch <= 0) return fail(TMAC_ERR_SHAPE, "batch must be positive");
    if (w->mode == TMAC_MODE_F32 && (row_acc || unit_acc))
        return fail(TMAC_ERR_TYPE, "the FP32 path has no integer accumulators");
    DeviceGuard dg(w->device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    cudaStream_t s = (cudaStream_t)stream;
    if (w->mode == TMAC_MODE_NATIVE && w->type == TMAC_TYPE_Q8_0)
        return launch_q8_0(w, x, y, row_acc, unit_acc, batch, s);
    if (w->mode == TMAC_MODE_NATIVE) {
        // 8..64 vectors: the tensor-core split-K path (gemm_tc.cu), the same
        // integer sums and epilogue bit for bit, 1.3-3x faster than the CUDA-core
        // GEMV from batch 8 (measured on 896x4864 / 4864x896 / 896x896 at 8, 16, 64)
        if (batch >= kTcMinBatch && batch <= kTcMaxBatch && !unit_acc && w->cols % 16 == 0 && w->cols <= 32768)
            return launch_gemm(w, x, y, row_acc, batch, s);
        // one or two vectors: every CTA quantises x itself (one launch); more:
        // quantise once into the device workspace, then the GEMV
        if (batch <= 2) return launch_blockq(w, x, nullptr, nullptr, nullptr, y, row_acc, unit_acc, batch, s);
        int16_t* xq = nullptr;
        float* xs = nullptr;
        int rc2 = workspace(w->device, (size_t)batch * w->cols, (size_t)batch, &xq, &xs);
        if (rc2) return rc2;
        uint8_t* xp = reinterpret_cast<uint8_t*>(xq);
        if ((rc2 = launch_quantize(x, w->cols, batch, nullptr, xs, s, xp))) return rc2;
        return launch_blockq(w, nullptr, nullptr, xp, xs, y, row_acc, unit_acc, batch, s);
    }
    if (w->mode == TMAC_MODE_INT16) return launch_int16(w, x, y, row_acc, unit_acc, batch, s);
    return launch_f32(w, x, y, batch, s);
}

int tmac_gemv(tmac_weight_t w, const float* x, float* y, int batch, void* stream)
{
    return tmac_gemv_acc(w, x, y, nullptr, nullptr, batch, stream);
}

int tmac_gemv_static(tmac_weight_t w, const float* x, float* y, int batch, void* stream)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (!x || !y) return fail(TMAC_ERR_INVALID, "NULL x or y");
    if (batch <= 0) return fail(TMAC_ERR_SHAPE, "batch must be positive");
    if (w->mode != TMAC_MODE_NATIVE || w->type == TMAC_TYPE_Q8_0)
        return fail(TMAC_ERR_TYPE, "tmac_gemv_static: only NATIVE Q5_0 / Q4_K / Q6_K weights use scratch");
    if (w->cols % 8) return fail(TMAC_ERR_SHAPE, "tmac_gemv_static: cols must be a multiple of 8");
    if (batch > kStaticXs || (int64_t)batch * w->cols > kStaticXq)
        return fail(TMAC_ERR_SHAPE, "tmac_gemv_static: batch x cols = " + std::to_string((int64_t)batch * w->cols) +
                                        " (batch " + std::to_string(batch) + ") exceeds the fixed scratch of " +
                                        std::to_string(kStaticXq) + " values / " + std::to_string(kStaticXs) +
                                        " vectors; use tmac_gemv");
    DeviceGuard dg(w->device);
    if (!dg.ok) return fail(TMAC_ERR_CUDA, "cudaSetDevice failed");
    int16_t* xq = nullptr;
    float* xs = nullptr;
    if ((rc = static_scratch(w->device, &xq, &xs))) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    uint8_t* xp = reinterpret_cast<uint8_t*>(xq);  // the scratch holds x_q as byte planes
    if ((rc = launch_quantize(x, w->cols, batch, nullptr, xs, s, xp))) return rc;
    return launch_blockq(w, nullptr, nullptr, xp, xs, y, nullptr, nullptr, batch, s);
}

static int gemv_typed(tmac_weight_t w, int type, int mode, const float* x, float* y, int batch, void* stream,
                      const char* name)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (w->mode != mode || (type >= 0 && w->type != type))
        return fail(TMAC_ERR_TYPE, std::string(name) + ": weight has another type or mode");
    return tmac_gemv_acc(w, x, y, nullptr, nullptr, batch, stream);
}

int tmac_gemv_q8_0(tmac_weight_t w, const float* x, float* y, int batch, void* stream)
{
    return gemv_typed(w, TMAC_TYPE_Q8_0, TMAC_MODE_NATIVE, x, y, batch, stream, "tmac_gemv_q8_0");
}
int tmac_gemv_q5_0(tmac_weight_t w, const float* x, float* y, int batch, void* stream)
{
    return gemv_typed(w, TMAC_TYPE_Q5_0, TMAC_MODE_NATIVE, x, y, batch, stream, "tmac_gemv_q5_0");
}
int tmac_gemv_q4_k(tmac_weight_t w, const float* x, float* y, int batch, void* stream)
{
    return gemv_typed(w, TMAC_TYPE_Q4_K, TMAC_MODE_NATIVE, x, y, batch, stream, "tmac_gemv_q4_k");
}
int tmac_gemv_q6_k(tmac_weight_t w, const float* x, float* y, int batch, void* stream)
{
    return gemv_typed(w, TMAC_TYPE_Q6_K, TMAC_MODE_NATIVE, x, y, batch, stream, "tmac_gemv_q6_k");
}
int tmac_gemv_int16(tmac_weight_t w, const float* x, float* y, int batch, void* stream)
{
    return gemv_typed(w, -1, TMAC_MODE_INT16, x, y, batch, stream, "tmac_gemv_int16");
}

int tmac_gemv_host(tmac_weight_t w, const float* x_host, float* y_host, int batch)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (!x_host || !y_host) return fail(TMAC_ERR_INVALID, "NULL x or y");
    if (batch <= 0) return fail(TMAC_ERR_SHAPE, "batch must be positive");
    DeviceGuard dg(w->device);
    // The device's staging buffers belong to one call at a time, from the
    // lookup (which may grow them) to the final synchronisation.
    static std::mutex host_mu[64];
    std::lock_guard<std::mutex> hold(host_mu[w->device & 63]);
    const size_t xb = (size_t)batch * w->cols * sizeof(float), yb = (size_t)batch * w->rows * sizeof(float);
    float *dx = nullptr, *dy = nullptr;
    rc = staging(w->device, xb, yb, &dx, &dy);
    if (rc) return rc;
    cudaError_t e;
    if ((e = cudaMemcpyAsync(dx, x_host, xb, cudaMemcpyHostToDevice, nullptr)) != cudaSuccess)
        return cuda_fail(e, "H2D x");
    // A page-locked y that this device can address is written by the Q8_0
    // kernel itself (one plain store per row), so the transfer to the host
    // overlaps the GEMV instead of following it.  Other paths, and pageable y,
    // go through the device staging buffer.
    float* y_dev = nullptr;
    if (w->type == TMAC_TYPE_Q8_0 && w->mode == TMAC_MODE_NATIVE) {
        cudaPointerAttributes pa;
        if (cudaPointerGetAttributes(&pa, y_host) == cudaSuccess && pa.type == cudaMemoryTypeHost &&
            pa.devicePointer)
            y_dev = static_cast<float*>(pa.devicePointer);
        else
            cudaGetLastError();  // clear the lookup's error state
    }
    rc = tmac_gemv(w, dx, y_dev ? y_dev : dy, batch, nullptr);
    if (rc) return rc;
    if (!y_dev && (e = cudaMemcpyAsync(y_host, dy, yb, cudaMemcpyDeviceToHost, nullptr)) != cudaSuccess)
        return cuda_fail(e, "D2H y");
    TMAC_CUDA_TRY(cudaStreamSynchronize(nullptr));
    return TMAC_OK;
}

int tmac_top1(const float* y, int64_t n, int64_t index_base, uint64_t* key, void* stream)
{
    if (!y || !key) return fail(TMAC_ERR_INVALID, "NULL y or key");
    if (n <= 0 || index_base < 0 || index_base + n > 0x7FFFFFFF) return fail(TMAC_ERR_SHAPE, "bad index range");
    return launch_top1(y, n, index_base, reinterpret_cast<unsigned long long*>(key), (cudaStream_t)stream);
}

int tmac_gemv_top1(tmac_weight_t w, const float* x, float* y, uint64_t* key, int64_t index_base, int batch,
                   void* stream)
{
    int rc = weight_ok(w);
    if (rc) return rc;
    if (!x || !y || !key) return fail(TMAC_ERR_INVALID, "NULL x, y or key");
    if (batch <= 0) return fail(TMAC_ERR_SHAPE, "batch must be positive");
    if (index_base < 0 || index_base + w->rows > 0x7FFFFFFF) return fail(TMAC_ERR_SHAPE, "bad index range");
    DeviceGuard dg(w->device);
    cudaStream_t s = (cudaStream_t)stream;
    unsigned long long* k = reinterpret_cast<unsigned long long*>(key);
    if (w->mode == TMAC_MODE_NATIVE && w->type == TMAC_TYPE_Q8_0)  // the kernel writes the key: no reset
        return launch_q8_0(w, x, y, nullptr, nullptr, batch, s, k, index_base);
    TMAC_CUDA_TRY(cudaMemsetAsync(key, 0, (size_t)batch * sizeof(uint64_t), s));
    rc = tmac_gemv(w, x, y, batch, stream);
    for (int b = 0; !rc && b < batch; b++) rc = launch_top1(y + (int64_t)b * w->rows, w->rows, index_base, k + b, s);
    return rc;
}

int tmac_top1_decode(uint64_t key, float* value, int64_t* index)
{
    if (!key) return fail(TMAC_ERR_INVALID, "empty key");
    uint32_t u = (uint32_t)(key >> 31);
    u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    float v;
    memcpy(&v, &u, sizeof(v));
    if (value) *value = v;
    if (index) *index = (int64_t)(0x7FFFFFFFu - (uint32_t)(key & 0x7FFFFFFFu));
    return TMAC_OK;
}

int tmac_reserve(int device, int64_t max_batch, int64_t max_cols)
{
    int rc = check_device(device);
    if (rc) return rc;
    if (max_batch < 0 || max_cols < 0) return fail(TMAC_ERR_SHAPE, "negative size");
    DeviceGuard dg(device);
    int16_t* xq;
    float* xs;
    if (max_batch > 0 && max_cols > 0 && (rc = workspace(device, (size_t)(max_batch * max_cols), (size_t)max_batch, &xq, &xs)))
        return rc;
    if (!device_error_word(device)) return fail(TMAC_ERR_CUDA, "cannot resolve device error word");
    num_sms(device);
    return TMAC_OK;
}

}  // extern "C"
