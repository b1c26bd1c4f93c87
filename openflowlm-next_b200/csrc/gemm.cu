// Dense Q4_1 projection GEMM: y[T, N] = bf16(x)[T, K] . dequant(W)[N, K]^T with f32 accumulation, on the
// tcgen05 grouped GEMM of expert_tc.cu run as one group.
//
// The projections of the prefill schedule beside the MoE block (attention q/k/v/o and dense FFN weights)
// are plain Q4_1 matrices; the reference runs them as its gemm_q4_prefill design
// (open_kernels/designs/gemm_q4_prefill/gemm_q4_prefill.py:1-3: Y[N_WEIGHT, T] = W(q4_1)[N_WEIGHT, K] @
// X^T[K, T], the weight dequantised on-core per 64 x 64 tile). Here W is in this library's tile layout
// (fm_q4_1_to_tiles: 128 rows x 64 K per 5120-byte tile, band-major), the work list is one group's rows
// cut into items of at most 256 token rows per 128-row band, and the kernel's unweighted f32 row mode
// writes each item's 128 x n block of y straight to y[t][128 band ..]: the output is token-major, y[t][n],
// the transpose of the reference's device layout.
#include "common.cuh"
#include "kernels.cuh"

namespace fm {
namespace {

size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

struct GemmLayout {
    size_t err, xb, gu_list, dn_list, total;
    int items;
};

GemmLayout gemm_layout(int N, int K, int T, int x_dtype) {
    GemmLayout o{};
    o.items = (T + kTcItemRows - 1) / kTcItemRows * (N / kTileRows);
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t a = off; off = align_up(off + bytes); return a; };
    o.err = take(16);   // first: fm_moe_check reads the status words at the workspace start
    o.xb = take(x_dtype == FM_F32 ? (size_t)T * K * 2 : 0);
    o.gu_list = take(16);   // header only: this GEMM has no gate_up items
    o.dn_list = take((size_t)(4 + 4 * o.items) * 4);
    o.total = off;
    return o;
}

int gemm_check(int N, int K, int T, int x_dtype) {
    if (N <= 0 || N % kTileRows || K <= 0 || K % kTileK || T < 0) {
        set_error("fm_q4_gemm: N=%d must be a positive multiple of %d, K=%d of %d, T=%d >= 0", N, kTileRows, K, kTileK, T);
        return FM_EINVAL_SHAPE;
    }
    if (x_dtype != FM_F32 && x_dtype != FM_BF16) {
        set_error("fm_q4_gemm: x_dtype %d is neither FM_F32 nor FM_BF16", x_dtype);
        return FM_EINVAL_SHAPE;
    }
    return FM_OK;
}

template <typename T>
T* at(void* ws, size_t off) { return reinterpret_cast<T*>(static_cast<char*>(ws) + off); }

}  // namespace
}  // namespace fm

using namespace fm;

extern "C" FM_API int fm_q4_gemm_workspace_size(int32_t N, int32_t K, int32_t T, int32_t x_dtype, size_t* bytes) {
    clear_error();
    if (!bytes) {
        set_error("fm_q4_gemm_workspace_size: bytes is NULL");
        return FM_EINVAL_SHAPE;
    }
    if (int rc = gemm_check(N, K, T, x_dtype)) return rc;
    *bytes = gemm_layout(N, K, T, x_dtype).total;
    return FM_OK;
}

extern "C" FM_API int fm_q4_gemm(const uint8_t* w_tiles, int32_t N, int32_t K, const void* x, int32_t x_dtype, int32_t T,
                                 float* y, void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (int rc = gemm_check(N, K, T, x_dtype)) return rc;
    if (T == 0) return FM_OK;
    if (!w_tiles || !x || !y || !workspace) {
        set_error("fm_q4_gemm: a device pointer is NULL");
        return FM_EINVAL_SHAPE;
    }
    // the activation rows are read by TMA (16-byte aligned base) and y is written 16 bytes at a time
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(workspace)) & 15) {
        set_error("fm_q4_gemm: x, y and the workspace must be 16-byte aligned");
        return FM_EINVAL_SHAPE;
    }
    const GemmLayout lo = gemm_layout(N, K, T, x_dtype);
    if (workspace_bytes < lo.total) {
        set_error("fm_q4_gemm: workspace of %zu bytes, %zu needed (fm_q4_gemm_workspace_size)", workspace_bytes, lo.total);
        return FM_EWORKSPACE;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(workspace, 0, 16, st) != cudaSuccess) return cuda_status(cudaGetLastError(), "memset");
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    if (x_dtype == FM_F32) {
        if (int rc = launch_to_bf16(static_cast<const float*>(x), at<uint16_t>(workspace, lo.xb), (long long)T * K, st))
            return rc;
        xb = at<uint16_t>(workspace, lo.xb);
    }
    // one group (index 0, the kernel's "shared" group) over rows [0, T): items of <= 256 rows per band
    if (int rc = launch_seg_lists(nullptr, 0, 0, 0, T, at<int>(workspace, lo.gu_list), 0, 0, at<int>(workspace, lo.dn_list),
                                  N / kTileRows, kTcItemRows, st))
        return rc;
    TcLaunch d{};
    d.max_items = lo.items;
    d.list = at<int>(workspace, lo.dn_list);
    d.act = xb;
    d.act_rows = T;
    d.act_cols = K;
    d.act_ld = K;
    d.w_routed = w_tiles;
    d.w_routed_stride = 0;
    d.w_shared = w_tiles;
    d.shared_group = 0;
    d.K_routed = K;
    d.K_shared = K;
    d.H = N;      // y row stride
    d.k = 1;
    d.y_f32 = y;  // unweighted f32 rows: y[t][128 band + c]
    d.err = at<int>(workspace, lo.err) + 1;
    return launch_expert_tc(false, d, st);
}
