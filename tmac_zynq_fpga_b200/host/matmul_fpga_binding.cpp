// matmul_fpga_binding.cpp -- the reference engine's matmul_fpga_* drivers
// (sim/tmac_gguf.cpp:466-470, defined at :887, :948, :1097, :1221, :1367)
// re-pointed at libtmac_cuda.so: the code a maintainer puts in place of those
// driver bodies.  Same signatures and the same host-array contract (x in,
// y out, synchronous); the weight-only work (row_inv / row_scale, the Q8_0
// combined scales, the INT16 requantisation) is done once per tensor at its
// first call, since tensors never change after load_tmac.  A failing call
// aborts with the library's message: the reference drivers return void, and
// a stale y must not flow on.
//
// `Tensor` is the reference's struct (sim/tmac_gguf.cpp:163-169), declared
// again here with the same layout, as sim/matmul_q8.cpp does.
#include "tmac_cuda.h"

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>

struct Tensor {
    char name[128];
    uint64_t rows, cols;
    uint32_t type;
    uint64_t n_bytes;
    uint8_t* data;
};

namespace {

std::mutex g_mu;
// Registered weights by (tensor, row_max_abs table), one map per TMAC_MODE_*:
// a Q8_0 tensor called with another row_max_abs table gets its own registration.
std::map<std::pair<const void*, const void*>, tmac_weight_t> g_cache[3];

[[noreturn]] void die(const char* what)
{
    fprintf(stderr, "[TMAC] %s: %s\n", what, tmac_last_error());
    abort();
}

tmac_weight_t weight_for(const Tensor* A, int rows, int cols, int mode, const float* row_max_abs = nullptr)
{
    // y holds A->rows values in every reference call site; a partial call
    // would make tmac_gemv_host write past the caller's y
    if ((uint64_t)rows != A->rows || (uint64_t)cols != A->cols) {
        fprintf(stderr, "[TMAC] %s: rows x cols %d x %d differ from the tensor's %llu x %llu\n", A->name, rows, cols,
                (unsigned long long)A->rows, (unsigned long long)A->cols);
        abort();
    }
    std::lock_guard<std::mutex> lk(g_mu);
    const auto key = std::make_pair((const void*)A, (const void*)row_max_abs);
    auto it = g_cache[mode].find(key);
    if (it != g_cache[mode].end()) return it->second;
    tmac_weight_t w = nullptr;
    if (tmac_weight_register((int)A->type, mode, (int64_t)A->rows, (int64_t)A->cols, A->data, (size_t)A->n_bytes,
                             /*blocks_on_device=*/0, row_max_abs, /*device=*/0, &w) != TMAC_OK)
        die(A->name);
    return g_cache[mode][key] = w;
}

void run(tmac_weight_t w, const float* x, float* y)
{
    if (tmac_gemv_host(w, x, y, /*batch=*/1) != TMAC_OK) die("tmac_gemv_host");
}

}  // namespace

void matmul_fpga_int16(const Tensor* A, const float* x, float* y, int rows, int cols)
{
    run(weight_for(A, rows, cols, TMAC_MODE_INT16), x, y);
}
void matmul_fpga_q8(const Tensor* A, const float* x, float* y, int rows, int cols, const float* row_max_abs)
{
    run(weight_for(A, rows, cols, TMAC_MODE_NATIVE, row_max_abs), x, y);
}
void matmul_fpga_q4_k(const Tensor* A, const float* x, float* y, int rows, int cols)
{
    run(weight_for(A, rows, cols, TMAC_MODE_NATIVE), x, y);
}
void matmul_fpga_q5_0(const Tensor* A, const float* x, float* y, int rows, int cols)
{
    run(weight_for(A, rows, cols, TMAC_MODE_NATIVE), x, y);
}
void matmul_fpga_q6_k(const Tensor* A, const float* x, float* y, int rows, int cols)
{
    run(weight_for(A, rows, cols, TMAC_MODE_NATIVE), x, y);
}
