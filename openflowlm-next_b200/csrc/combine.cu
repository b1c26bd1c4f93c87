// Combine kernels: the ordered weighted sum of each token's expert rows (the scatter of
// src/open_qwen36/core.cpp:5236-5255: a token's expert terms added in ascending expert order), for the
// decode GEMV path (f32 y rows) and the expert-parallel paths (bf16 y rows returned by the expert ranks).
#include "common.cuh"
#include "kernels.cuh"

namespace fm {

// Four consecutive y values of row `row` as floats: f32 rows, or bf16 rows (the tcgen05 path).
__device__ __forceinline__ float4 ld_y4(const float* y, size_t row, int H, int i) {
    return reinterpret_cast<const float4*>(y + row * H)[i];
}
__device__ __forceinline__ float4 ld_y4(const uint16_t* y, size_t row, int H, int i) {
    const uint2 v = reinterpret_cast<const uint2*>(y + row * H)[i];
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u), __uint_as_float(v.y << 16),
                       __uint_as_float(v.y & 0xFFFF0000u));
}

// out[t] = res[t] + sgate[t] * y[P + t] + sum over t's pairs in ascending expert order of w * y[pos].
// Rows t >= t_real: out = res. Grid (T, H / 1024): each thread one float4 column group; every load of a
// thread is issued before the ordered accumulation.
template <class YT>
__global__ void combine_kernel(const float* __restrict__ res, const YT* __restrict__ y, const int* __restrict__ pos,
                               const int32_t* __restrict__ idx, const float* __restrict__ w,
                               const float* __restrict__ sgate, int shared_on, int T, int t_real, int k, int H, int P,
                               float* __restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int t = blockIdx.x;
    __shared__ int srow[kMaxTopK];
    __shared__ float sw[kMaxTopK];
    __shared__ int n_sel;
    const int i = blockIdx.y * blockDim.x + threadIdx.x;   // float4 column group
    const bool col = i < H / 4;
    // the residual and shared-expert loads are issued before the pair lists are read
    float4 o = col ? reinterpret_cast<const float4*>(res + (size_t)t * H)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 vs = make_float4(0.f, 0.f, 0.f, 0.f);
    float g = 0.f;
    if (col && shared_on && t < t_real) {
        vs = ld_y4(y, (size_t)(P + t), H, i);
        g = sgate[t];
    }
    if (threadIdx.x < 32) {
        // lane s < k holds slot s; its place in ascending expert order (ties by slot: the visit order of
        // core.cpp:5163-5165) among the slots routed here (pos >= 0) comes from k shuffles
        const int lane = threadIdx.x;
        const bool on = t < t_real && lane < k;
        const int e = on ? idx[(size_t)t * k + lane] : 0x7fffffff;
        const int p = on ? pos[(size_t)t * k + lane] : -1;
        const float ww = on ? w[(size_t)t * k + lane] : 0.f;
        const bool sel = on && p >= 0;
        int m = 0;
        for (int j = 0; j < k; ++j) {
            const int ej = __shfl_sync(0xffffffffu, e, j);
            const int sj = __shfl_sync(0xffffffffu, sel ? 1 : 0, j);
            if (sj && (ej < e || (ej == e && j < lane))) ++m;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, sel);
        if (sel) {
            srow[m] = p;
            sw[m] = ww;
        }
        if (lane == 0) n_sel = __popc(bal);
    }
    __syncthreads();
    const int n = n_sel;
    if (!col) return;
    if (t < t_real) {
        float4 v[kMaxTopK];
#pragma unroll
        for (int j = 0; j < kMaxTopK; ++j)
            if (j < n) v[j] = ld_y4(y, (size_t)srow[j], H, i);
        if (shared_on) {
            o.x += g * vs.x; o.y += g * vs.y; o.z += g * vs.z; o.w += g * vs.w;
        }
#pragma unroll
        for (int j = 0; j < kMaxTopK; ++j)
            if (j < n) {
                const float ww = sw[j];
                o.x += ww * v[j].x; o.y += ww * v[j].y; o.z += ww * v[j].z; o.w += ww * v[j].w;
            }
    }
    reinterpret_cast<float4*>(out + (size_t)t * H)[i] = o;
}

int launch_combine(const float* res, const float* y, const int* pos, const int32_t* idx, const float* w,
                   const float* sgate, int shared_on, int T, int t_real, int k, int H, int P, float* out, cudaStream_t st) {
    if (T <= 0) return FM_OK;
    dim3 grid(T, (H / 4 + 255) / 256);
    FM_LAUNCH_PDL("combine", combine_kernel<float>, grid, dim3(256), 0, st, res, y, pos, idx, w, sgate, shared_on, T, t_real,
                  k, H, P, out);
    return FM_OK;
}

// Combine of bf16 y rows (the tcgen05 path and the expert-parallel paths), one warp per token. Lanes
// 0..k-1 hold the token's (expert, sorted row, weight); each slot's rank in ascending expert order (ties
// by slot, the visit order of core.cpp:5163-5165) comes from k shuffles, and the rows are then added in
// that order. Lane j owns columns 8j + 256i (16-byte loads of 8 bf16), so a warp keeps up to 4 KB of
// loads in flight per expert row.
//   INIT: out[t] = res[t] + sgate[t] * y[P + t] + sum of w * y[pos]   (rows t >= t_real: out = res)
//   else: out[t] += sum of w * y[pos]                                   (rows t >= t_real untouched)
constexpr int kCombCols = 2048;   // columns per pass (8 chunks of 256 per lane)

__device__ __forceinline__ void add_bf16x8(float* acc, uint4 v, float s) {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(s, __uint_as_float(u[i] << 16), acc[2 * i]);
        acc[2 * i + 1] = fmaf(s, __uint_as_float(u[i] & 0xFFFF0000u), acc[2 * i + 1]);
    }
}

template <bool INIT>
__global__ void __launch_bounds__(256) combine_rows_kernel(const float* __restrict__ res, const uint16_t* __restrict__ y,
                                                           const int* __restrict__ pos, const int32_t* __restrict__ idx,
                                                           const float* __restrict__ w, const float* __restrict__ sgate,
                                                           int shared_on, int T, int t_real, int k, int H, int P,
                                                           float* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + warp;
    if (t >= T) return;
    float* o = out + (size_t)t * H;
    if (t >= t_real) {
        if (INIT)
            for (int c = lane * 4; c < H; c += 128)
                *reinterpret_cast<float4*>(o + c) = *reinterpret_cast<const float4*>(res + (size_t)t * H + c);
        return;
    }
    int e = 0x7fffffff, p = -1;
    float ww = 0.f;
    if (lane < k) {
        e = idx[(size_t)t * k + lane];
        p = pos[(size_t)t * k + lane];
        ww = w[(size_t)t * k + lane];
    }
    int rank = 0;
    for (int s = 0; s < k; ++s) {
        const int es = __shfl_sync(0xffffffffu, e, s);
        rank += (es < e) || (es == e && s < lane);
    }
    const float g = (INIT && shared_on) ? sgate[t] : 0.f;
    for (int c0 = 0; c0 < H; c0 += kCombCols) {
        float acc[8][8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = c0 + 256 * j + 8 * lane;
            const float* src = INIT ? res + (size_t)t * H : o;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (c < H && c < c0 + kCombCols) {
                a = *reinterpret_cast<const float4*>(src + c);
                b = *reinterpret_cast<const float4*>(src + c + 4);
            }
            acc[j][0] = a.x; acc[j][1] = a.y; acc[j][2] = a.z; acc[j][3] = a.w;
            acc[j][4] = b.x; acc[j][5] = b.y; acc[j][6] = b.z; acc[j][7] = b.w;
        }
        if (INIT && shared_on) {
            const uint16_t* yr = y + (size_t)(P + t) * H;
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + 256 * j + 8 * lane;
                v[j] = (c < H && c < c0 + kCombCols) ? *reinterpret_cast<const uint4*>(yr + c) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) add_bf16x8(acc[j], v[j], g);
        }
        for (int r = 0; r < k; ++r) {
            const int src = __ffs(__ballot_sync(0xffffffffu, lane < k && rank == r)) - 1;
            const int row = __shfl_sync(0xffffffffu, p, src);
            const float wr = __shfl_sync(0xffffffffu, ww, src);
            if (row < 0) continue;   // a pair outside the block's experts
            const uint16_t* yr = y + (size_t)row * H;
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int c = c0 + 256 * j + 8 * lane;
                v[j] = (c < H && c < c0 + kCombCols) ? *reinterpret_cast<const uint4*>(yr + c) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) add_bf16x8(acc[j], v[j], wr);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int c = c0 + 256 * j + 8 * lane;
            if (c < H && c < c0 + kCombCols) {
                *reinterpret_cast<float4*>(o + c) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
                *reinterpret_cast<float4*>(o + c + 4) = make_float4(acc[j][4], acc[j][5], acc[j][6], acc[j][7]);
            }
        }
    }
}

int launch_combine_y16(const float* res, const uint16_t* y, const int* pos, const int32_t* idx, const float* w,
                       const float* sgate, int shared_on, int T, int t_real, int k, int H, int P, float* out,
                       cudaStream_t st) {
    if (T <= 0) return FM_OK;
    combine_rows_kernel<true><<<(T + 7) / 8, 256, 0, st>>>(res, y, pos, idx, w, sgate, shared_on, T, t_real, k, H, P, out);
    FM_LAUNCH_CHECK("combine_rows");
    return FM_OK;
}

// Expert-parallel combine: out[t] += sum over t's pairs in ascending expert order of w * y[pos], y the
// bf16 rows returned by the expert ranks in the sender's sorted order; out already holds res plus the
// gated shared expert. Rows t >= t_real are left as they are.
int launch_combine_bf16(float* out, const uint16_t* y, const int* pos, const int32_t* idx, const float* w, int T,
                        int t_real, int k, int H, cudaStream_t st) {
    if (t_real <= 0) return FM_OK;
    combine_rows_kernel<false><<<(t_real + 7) / 8, 256, 0, st>>>(nullptr, y, pos, idx, w, nullptr, 0, t_real, t_real, k,
                                                                 H, 0, out);
    FM_LAUNCH_CHECK("combine_rows_accum");
    (void)T;
    return FM_OK;
}

}  // namespace fm
