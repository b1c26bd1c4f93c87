// fm_moe_layer_noalloc: the whole MoE layer for callers that cannot allocate device memory.
//
// Who needs it: an inference engine that reserves all of its device memory when it loads a model and
// then hands out fixed buffers -- as the reference's engine does with its per-layer buffer objects --
// has no hook through which a library could ask for an extra, call-sized workspace; and a decode loop
// that must not stall cannot afford cudaMalloc, which may synchronise the device. Such a caller passes
// only its inputs and outputs; the scratch space this call needs lives in a static device array
// compiled into this library instead.
//
// Limits and sharing:
//   * the array is kStaticWorkspaceBytes (24 MiB) on every GPU that loads the library, held until the
//     process exits; a call whose fm_workspace_size() exceeds it is rejected with FM_EWORKSPACE. For the
//     2048-wide layers of top-8 routing that is T <= 456 tokens with 128 experts of F 768, and T <= 497
//     with 256 experts of F 512 plus a shared expert of 512 (every decode batch of up to 128 tokens);
//   * every call on a device uses the same array, which keeps the previous call's contents. Each call
//     clears the status words it reports through and writes every other byte before reading it, so stale
//     contents never leak into a result; but calls that overlap on the GPU (two streams, or two host
//     threads) race on the array and must be serialised by the caller;
//   * the first call on each device does a one-time set-up with that device current: it looks the
//     array's device address up (cudaGetSymbolAddress) and creates the device's side stream and events
//     that the shared expert's kernels use on the tensor-core path, so that no later call creates
//     anything. Make that first call before any stream capture begins.
// No cudaMalloc, cudaFree or allocating library routine is called on this path: every kernel of the
// layer is this library's own (the router included).
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace {

constexpr size_t kStaticWorkspaceBytes = size_t(24) << 20;
constexpr int kMaxDevices = 64;

// In host code this name is a host-side stand-in, not a device address: kernels must be given the
// address cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

void* g_workspace_addr[kMaxDevices];
std::mutex g_workspace_mu;

}  // namespace

extern "C" FM_API int fm_moe_layer_noalloc(const fm_layer* L, const void* xm, int32_t xm_dtype, const float* res,
                                           int32_t T, int32_t t_real, float* out, int32_t* idx, float* w,
                                           void* stream) {
    size_t need = 0;
    if (int rc = fm_workspace_size(L, T, &need)) return rc;
    if (need > kStaticWorkspaceBytes) {
        fm::set_error("fm_moe_layer_noalloc: T=%d needs %zu B of workspace, more than the %zu B static array", T, need,
                      kStaticWorkspaceBytes);
        return FM_EWORKSPACE;
    }
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fm::cuda_status(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) {
        fm::set_error("fm_moe_layer_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
        return FM_EINVAL_SHAPE;
    }
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_workspace_mu);
        if (!g_workspace_addr[dev]) {   // one-time set-up on this device
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_static_workspace);
            if (e != cudaSuccess) return fm::cuda_status(e, "cudaGetSymbolAddress(static workspace)");
            if (int rc = fm::prepare_side_stream()) return rc;
            g_workspace_addr[dev] = p;
        }
        ws = g_workspace_addr[dev];
    }
    return fm_moe_layer(L, xm, xm_dtype, res, T, t_real, out, idx, w, ws, kStaticWorkspaceBytes, stream);
}
