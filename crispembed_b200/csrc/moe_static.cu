// moe_static.cu -- the MoE feed-forward block without any device allocation.
//
// Some hosts cannot call cudaMalloc once they are running: a serving process
// whose device memory is owned by another allocator (an inference runtime that
// reserved the GPU up front), plugins that are handed a stream but no right to
// allocate, or latency-critical callers that cannot afford the device-wide
// synchronisation cudaMalloc/cudaFree may cause.  ceb_moe_ffn_static serves
// them: its scratch is the file-scope array below, which the CUDA runtime sets
// aside on a GPU when this library's device code is loaded there (at its first use
// on that GPU under lazy module loading, the default; on every GPU the process
// initialises under CUDA_MODULE_LOADING=EAGER) and keeps until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#define CRISPEMBED_BUILD 1
#include "../../include/ceb_ops.h"
#include "ceb_internal.h"
#include "ceb_moe_internal.h"

// The scratch and the device-side error word of ceb_moe_ffn_static.  In host
// code these names are host-side stand-ins, not device addresses: the device
// addresses come from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_moe_static_scratch[CEB_MOE_STATIC_SCRATCH_BYTES];
static __device__ int g_moe_static_err;

namespace {
constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
uint8_t* g_scratch[MAX_DEVICES] = {};
int* g_err[MAX_DEVICES] = {};

// Device addresses of the scratch and error word on the current device, looked
// up once per device (the first call on a device does this set-up).
int static_addresses(uint8_t** scratch, int** err) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return ceb_set_cuda_error(e, "cudaGetDevice", __FILE__, __LINE__);
    if (dev < 0 || dev >= MAX_DEVICES) return ceb_set_error(1, "moe_ffn_static: device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_moe_static_scratch);
        if (e != cudaSuccess) return ceb_set_cuda_error(e, "cudaGetSymbolAddress(scratch)", __FILE__, __LINE__);
        void* q = nullptr;
        e = cudaGetSymbolAddress(&q, g_moe_static_err);
        if (e != cudaSuccess) return ceb_set_cuda_error(e, "cudaGetSymbolAddress(error word)", __FILE__, __LINE__);
        g_scratch[dev] = static_cast<uint8_t*>(p);
        g_err[dev] = static_cast<int*>(q);
    }
    *scratch = g_scratch[dev];
    *err = g_err[dev];
    return 0;
}
}  // namespace

extern "C" int ceb_moe_ffn_static(const ceb_moe_layer* layer, const void* d_x, int x_dtype, int n_tokens, float* d_y,
                                  void* stream) {
    if (!layer || !d_x || !d_y || n_tokens < 0) return ceb_set_error(1, "moe_ffn_static: bad arguments");
    if (x_dtype != CEB_ACT_F32 && x_dtype != CEB_ACT_BF16 && x_dtype != CEB_ACT_F16)
        return ceb_set_error(1, "moe_ffn_static: x_dtype %d unsupported", x_dtype);
    if (n_tokens == 0) return 0;
    const ceb_moe_weights& w = layer->w;
    const size_t need = ceb_moe_ws_layout(n_tokens, w.d, w.n_experts, w.top_k, w.ffn, nullptr, nullptr);
    if (need > (size_t)CEB_MOE_STATIC_SCRATCH_BYTES)
        return ceb_set_error(1,
                             "moe_ffn_static: %d tokens need %zu bytes of scratch, more than the %u-byte static "
                             "buffer; split the batch or use ceb_moe_ffn with a caller workspace",
                             n_tokens, need, (unsigned)CEB_MOE_STATIC_SCRATCH_BYTES);
    uint8_t* scratch = nullptr;
    int* err = nullptr;
    int rc = static_addresses(&scratch, &err);
    if (rc) return rc;
    // Nothing needs clearing.  The routing words this call reads (histograms,
    // offsets, permutation) are all written earlier in the same call.  The grouped
    // GEMMs load whole 128-row tiles, so the tail rows of an expert's last tile in
    // x_perm / h_perm can hold another expert's rows or rows left from an earlier
    // call; the products of those rows are never stored.
    ceb_moe_ws ws;
    ceb_moe_ws_layout(n_tokens, w.d, w.n_experts, w.top_k, w.ffn, &ws, scratch);
    return ceb_moe_run(w, d_x, x_dtype, nullptr, n_tokens, d_y, ws, nullptr, nullptr, err,
                       static_cast<cudaStream_t>(stream));
}

// Reads and clears the static path's device error word on the current device into
// *code (0 when the path was never used there); returns 0, or 3 when the word
// could not be read or cleared.  Called by ceb_sync_check.
int ceb_moe_static_take_error(int* code) {
    *code = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return 3;
    int* err = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        err = g_err[dev];
    }
    if (!err) return 0;
    int h = 0;
    if (cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
    if (h && cudaMemset(err, 0, sizeof(int)) != cudaSuccess) return 3;
    *code = h;
    return 0;
}
